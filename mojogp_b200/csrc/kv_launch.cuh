// Host-side launch description for the tiled matvec and the per-evaluator
// dispatch over the compiled (DP, T) instantiations.
#pragma once

#include "kv_tiles.cuh"
#include "kv_tiles_gramh.cuh"

namespace gpb {

// Evaluator ids: the five fast leaves use their GPB_KERNEL_* value,
// kEvalGeneric selects the tree evaluator.
constexpr int kEvalGeneric = 100;

struct KvLaunch {
  int eval;                 // GPB_KERNEL_RBF..RQ or kEvalGeneric
  int DP;                   // padded dims of xrow / packed x (compiled sizes only)
  int T;                    // rhs columns per pass (compiled sizes only)
  const float* xrow;        // [nrow][DP]
  int64_t nrow;
  const float* xv;          // packed [ntiles*kJT][packed_width(DP,T)]
  int ntiles;
  FastParams fp;
  const DevKernel* dk;      // generic evaluator program (host copy, passed by value)
  TileEpilogue ep;          // ep.out = final output (column stride ep.out_ld)
  int tcols;                // valid columns (<= T)
  float* partial;           // scratch for split partial sums (may be null if splits==1)
  int64_t partial_capacity; // floats available in `partial`
  int* err;                 // device error word
  cudaStream_t stream;
  int64_t* launches = nullptr;      // incremented per kernel launched
  cudaEvent_t ev_begin = nullptr;   // if set: recorded around the tile kernel(s)
  cudaEvent_t ev_end = nullptr;
  bool gram_ok = false;             // rows and columns are the provider's training
                                    // inputs and their prescaled norms are bounded
};

// Compiled sizes.
inline bool kv_dp_supported(int eval, int DP) {
  if (eval == kEvalGeneric) return DP == 4 || DP == 8 || DP == 16 || DP == 32 || DP == 64;
  return DP == 1 || DP == 2 || DP == 4 || DP == 8 || DP == 16 || DP == 32;
}
inline int kv_pick_dp(int eval, int d) {
  const int cand_fast[] = {1, 2, 4, 8, 16, 32};
  const int cand_gen[] = {4, 8, 16, 32, 64};
  if (eval == kEvalGeneric) {
    for (int c : cand_gen)
      if (d <= c) return c;
  } else {
    for (int c : cand_fast)
      if (d <= c) return c;
  }
  return -1;
}
inline int kv_pick_t(int64_t remaining) {
  if (remaining >= 16) return 16;
  if (remaining > 8) return 16;
  if (remaining > 4) return 8;
  if (remaining > 1) return 4;
  return 1;
}

// Kernel / packed-layout choice per launch shape:
//   KV_GRAMH  the Gram form on fp16 hi / lo operands (kv_tiles_gramh.cuh):
//             the default for RBF (measured 4-12 % faster than KV_GRAM), while
//             the Matern and RQ leaves keep KV_GRAM (their longer leaf
//             evaluation made the fp16 kernel 0-11 % slower);
//             GPB_KV_GRAMH=0 disables it, =2 takes it for every Gram leaf;
//   KV_GRAM   both contractions on the tensor core (kv_tiles_gram.cuh): RBF,
//             Matérn-3/2, Matérn-5/2 or RQ, T = 16, DP 8 or 16, and only when
//             the caller vouches for bounded input norms (gram_ok);
//             GPB_KV_GRAM=0 in the environment selects KV_TC instead;
//   KV_GRAM1  the Gram kernel's MMA1 with an fp32 CUDA-core contraction
//             (kv_tile_gram1_kernel) for T = 1 under the same conditions
//             (measured at n = 3e5: 3.2e12 entries/s against 2.35e12 for the
//             Gram kernel; at 4 and 8 columns the Gram kernel with padded
//             columns is as fast or faster, so those chunks run at T = 16);
//             GPB_KV_GRAM1=0 pads 1-column chunks to T = 16 as well;
//   KV_TC     tensor-core contraction (kv_tiles_tc.cuh): fast leaves, T = 16,
//             DP a multiple of 4 (default; GPB_KV_TC=0 in the environment
//             selects KV_X2 instead);
//   KV_X2     paired-row FFMA2 kernel (kv_tiles_x2.cuh): fast leaves, even DP,
//             T >= 4; GPB_KV_SCALAR=1 disables it (and the TC kernel);
//   KV_SCALAR everything else (and the composite-tree evaluator).
enum KvLayout { KV_SCALAR = 0, KV_X2 = 1, KV_TC = 2, KV_GRAM = 3, KV_GRAM1 = 4, KV_GRAMH = 5 };
bool kv_x2_disabled();
bool kv_tc_disabled();
bool kv_gram_disabled();
bool kv_gram1_disabled();
// fp16 Gram kernel selection (GPB_KV_GRAMH): 0 never, 1 RBF only (default),
// 2 every Gram leaf.
int kv_gramh_mode();
// Largest max_i |x'_i|^2 (prescaled inputs) for which the Gram expansion keeps
// the matvec within the 1e-5 relative bar (3xTF32 cross term, fp32 norms).
constexpr float kGramMaxSqNorm = 100.f;
constexpr bool gram_leaf(int eval) {
  return eval == GPB_KERNEL_RBF || eval == GPB_KERNEL_MATERN32 || eval == GPB_KERNEL_MATERN52 ||
         eval == GPB_KERNEL_RQ;
}
inline int kv_layout(int eval, int DP, int T, bool gram_ok = false) {
  if (eval == kEvalGeneric || kv_x2_disabled()) return KV_SCALAR;
  if (gram_ok && gram_leaf(eval) && (DP == 8 || DP == 16) && !kv_tc_disabled() &&
      !kv_gram_disabled()) {
    if (T == 16) {
      const int m = kv_gramh_mode();
      return (m == 2 || (m == 1 && eval == GPB_KERNEL_RBF)) ? KV_GRAMH : KV_GRAM;
    }
    if (T == 1 && !kv_gram1_disabled()) return KV_GRAM1;
  }
  if (T == 16 && DP % 4 == 0 && DP <= 32 && !kv_tc_disabled()) return KV_TC;
  if (DP % 2 == 0 && T >= 4) return KV_X2;
  return KV_SCALAR;
}
// Column-chunk width for `remaining` columns. On the Gram path a narrow chunk
// runs on KV_GRAM1, or, when that is disabled, at T = 16 with zero-padded
// columns (the Gram kernel's cost is the per-entry kernel evaluation, nearly
// independent of T).
inline int kv_chunk_t(int eval, int DP, int64_t remaining, bool gram_ok) {
  const int t = kv_pick_t(remaining);
  if (t < 16 && kv_layout(eval, DP, t, gram_ok) != KV_GRAM1 &&
      (kv_layout(eval, DP, 16, gram_ok) == KV_GRAM || kv_layout(eval, DP, 16, gram_ok) == KV_GRAMH))
    return 16;
  return t;
}
inline bool kv_uses_x2(int eval, int DP, int T) { return kv_layout(eval, DP, T) == KV_X2; }
// Floats per packed column row for this launch shape (the TC layout is
// tile-blocked, 128 rows per tile, with the same average width).
inline int kv_packed_width(int eval, int DP, int T, bool gram_ok = false) {
  switch (kv_layout(eval, DP, T, gram_ok)) {
    case KV_GRAM: return 2 * DP + 8 + 32;
    case KV_GRAMH: return gramh_tile_floats(DP) / 128;
    case KV_GRAM1: return 2 * DP + 8 + T;
    case KV_TC: return DP + 32;
    case KV_X2: return 2 * (DP + T);
    default: return ((DP + T) + 3) / 4 * 4;
  }
}

// Rows per thread for a (DP, T, generic) instantiation.
__host__ __device__ constexpr int kv_rows_per_thread(int DP, int T, bool generic) {
  return generic ? 1 : (DP >= 32 ? 2 : 4);
}
constexpr int kKvBlock = 128;

// Per-evaluator launchers (one translation unit each).
int launch_kv_rbf(const KvLaunch& L);
int launch_kv_m12(const KvLaunch& L);
int launch_kv_m32(const KvLaunch& L);
int launch_kv_m52(const KvLaunch& L);
int launch_kv_rq(const KvLaunch& L);
int launch_kv_generic(const KvLaunch& L);

int launch_kv(const KvLaunch& L);

// Choose the number of j-splits for `row_blocks` row tiles so that the grid
// fills the GPU's resident slots with little wave-quantisation loss.
int kv_choose_splits(int64_t row_blocks, int ntiles, int resident_per_sm, int num_sms);

// Deterministic fixed-order reduction of split partials + epilogue.
int launch_kv_reduce(const KvLaunch& L, int splits);

}  // namespace gpb
