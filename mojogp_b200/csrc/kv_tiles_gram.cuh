// Gram-form tensor-core K·V tile kernel (sm_100a tcgen05, kind::tf32).
//
// Both contractions of a K·V tile run on the tensor core:
//   MMA1  u = [x_i | |x_i|^2 parts | 1 1 1] · [-2 y_j | 1 1 1 | |y_j|^2 parts]
//           = |x_i|^2 + |y_j|^2 - 2 x_i·y_j       (3xTF32 on the x·y block)
//   k_ij  = leaf(u_ij), split into tf32 hi / lo   (CUDA cores)   -> TMEM
//   MMA2  D += K_hi V_hi + K_hi V_lo + K_lo V_hi  (A from TMEM)  -> TMEM
// The squared norms ride along as one extra 8-wide k-step: each norm is split
// into three tf32 parts that sum to it exactly, multiplied by exact ones, so
// that k-step needs only the hi x hi product. The CUDA cores are left with the
// leaf function (one MUFU exponential for RBF) and the hi / lo split.
//
// The expansion |x|^2 + |y|^2 - 2 x·y loses absolute accuracy in proportion to
// the squared norms of the prescaled inputs; the host selects this path only
// when max_i |x'_i|^2 is small enough to keep the matvec inside the 1e-5
// relative bar (provider_refresh_xs) and only for the leaves that are smooth in
// u at u = 0 (RBF, Matérn-3/2, Matérn-5/2, RQ); Matérn-1/2 (exp(-sqrt(u)))
// keeps the difference form.
//
// CTA: 3 row tiles of 128 rows (TMEM lanes = rows); chunks of 16 columns.
// Warpgroup r (warps 4r..4r+3) evaluates row tile r. A thread that issues an
// MMA into an accumulator an earlier MMA of its own is still writing stalls
// for that MMA's latency (~150 cycles), and one thread issues one MMA at a
// time, so tensor throughput needs many issuing threads with independent
// accumulators: per row tile one warp issues MMA1 of the even chunks, one of
// the odd chunks, and likewise two warps issue MMA2 into an even and an odd
// accumulator (summed at the end). The last warp streams column tiles through
// a 4-deep TMA ring. Every A operand comes from TMEM (shared-memory A operands
// of 4 KB per MMA would saturate shared memory).
// TMEM columns: [x hi | x lo] per row tile, the norm k-step per row tile,
// three chunk stages per row tile ([16: u, then K hi][16: K lo]) and two
// 16-column accumulators per row tile. Every wait is bounded.
#pragma once

#include "kv_tiles_tc.cuh"

namespace gpb {

#ifdef GPB_GRAM_PROFILE
// Diagnostic build only: cycles spent per role and wait, per translation unit.
static __device__ unsigned long long g_gram_prof[16];
#define GRAM_DECL long long gprof[8] = {0, 0, 0, 0, 0, 0, 0, 0}
#define GRAM_T0(v) const long long v = clock64()
#define GRAM_ACC(slot, t0) gprof[slot] += clock64() - (t0)
#define GRAM_FLUSH                                                        \
  if ((threadIdx.x & 31) == 0)                                            \
    for (int q_ = 0; q_ < 8; ++q_)                                        \
      if (gprof[q_]) atomicAdd(&g_gram_prof[q_], (unsigned long long)gprof[q_])
#else
#define GRAM_DECL
#define GRAM_T0(v)
#define GRAM_ACC(slot, t0)
#define GRAM_FLUSH
#endif

#ifndef GPB_GRAM_R
#define GPB_GRAM_R 3
#endif
#ifndef GPB_GRAM_S
#define GPB_GRAM_S 3
#endif
#ifndef GPB_GRAM_P
#define GPB_GRAM_P 2
#endif
constexpr int kGRowTiles = GPB_GRAM_R;
constexpr int kGChunk = 16;
constexpr int kGStages = 4;    // column-tile ring depth (also keeps one CTA per SM)
constexpr int kGUStages = GPB_GRAM_S;  // chunk stages in TMEM per row tile
constexpr int kGPar = GPB_GRAM_P;      // issuer warps per role and row tile (chunk c -> c % kGPar)
// Accumulation window, in column tiles. The tensor core adds into its fp32
// accumulator with truncation (round toward zero), so a long run of MMAs into
// one accumulator drifts toward zero by up to an ulp of the running sum per
// MMA: over the 6e4 MMAs of a 1e6-column row that is ~1e-3 relative. Each
// window of kGWinTiles tiles starts a fresh accumulator; the epilogue threads
// fold the finished window into an fp32 register sum (round to nearest).
#ifndef GPB_GRAM_WIN
#define GPB_GRAM_WIN 4
#endif
constexpr int kGWinTiles = GPB_GRAM_WIN;
constexpr int kGEpiThreads = 128 * kGRowTiles;
constexpr int kGIssuerWarps = 2 * kGPar * kGRowTiles;  // MMA1 and MMA2 issuers
constexpr int kGThreads = kGEpiThreads + 32 * kGIssuerWarps + 32;
constexpr uint32_t kGTmemCols = 512;
// TMEM column map.
constexpr uint32_t kGColX = 0;                                   // + 32 r : [x hi | x lo]
constexpr uint32_t kGColN = kGColX + 32 * kGRowTiles;            // + 8 r  : norm k-step
constexpr uint32_t kGColS = (40 * kGRowTiles + 31) / 32 * 32;     // + 32 S r + 32 s : stage
constexpr uint32_t kGColAcc = kGColS + 32 * kGUStages * kGRowTiles;  // + 16 P r + 16 class
static_assert(kGColAcc + 16 * kGPar * kGRowTiles <= kGTmemCols, "TMEM budget");

// Packed tile (floats): [B hi : 128 x (DP + 8)][B lo : 128 x DP]
//                      [V : 16 k-steps x 256, N = 32 rows (V hi | V lo)]
// with B = [-2y | 1 1 1 | |y|^2 parts | 0 0]; the row operand A is
// [x | |x|^2 parts | 1 1 1 | 0 0], built in TMEM by the kernel.
__host__ __device__ constexpr int gram_kaug(int DP) { return DP + 8; }
__host__ __device__ constexpr int gram_tile_floats(int DP) { return 128 * (2 * DP + 8) + 4096; }
__host__ __device__ constexpr int gram_v_offset(int DP) { return 128 * (2 * DP + 8); }

// Offset (floats) of element (m, k) in a [128 x DP] K-major operand block:
// 8-column k-steps of 1024 floats, core matrices of 8 rows x 4 k, K-adjacent
// at 2048 B, M/N-adjacent at 128 B.
__host__ __device__ constexpr int gram_xoff(int m, int k) {
  return (k / 8) * 1024 + ((k % 8) / 4) * 512 + (m / 8) * 32 + (m % 8) * 4 + (k % 4);
}

// Squared norm with a fixed summation order; the row side (kernel) and the
// column side (pack) must agree bit for bit so that u_ii cancels.
__host__ __device__ __forceinline__ float gram_sqnorm(const float* x, int DP) {
  float s = 0.f;
  for (int k = 0; k < DP; ++k) s = fmaf(x[k], x[k], s);
  return s;
}

// Three tf32 values (top 19 bits each) whose exact sum is v: a float has 24
// significant bits, two truncations take 11 each, the 2 bits left fit the third.
__host__ __device__ __forceinline__ void gram_split3(float v, float& a, float& b, float& c) {
  auto trunc = [](float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u &= 0xFFFFE000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
  };
  a = trunc(v);
  const float r = v - a;
  b = trunc(r);
  c = r - b;
}

template <int DP, int LEAF>
__global__ void __launch_bounds__(kGThreads, 1) kv_tile_gram_kernel(
    const float* __restrict__ xrow, int64_t nrow, const float* __restrict__ xv, int ntiles_total,
    int tiles_per_split, const __grid_constant__ FastParams fp, TileEpilogue ep, int* err) {
  static_assert(DP % 8 == 0 && DP <= 16, "K = DP in 8-wide tf32 k-steps, x hi / lo in 32 columns");
  constexpr int TILE = gram_tile_floats(DP);
  constexpr int kChunks = 128 / kGChunk;
  constexpr int kIssuer0 = kGEpiThreads / 32;  // warp kIssuer0 + 2 P r + role
  constexpr int kTmaWarp = kIssuer0 + kGIssuerWarps;
  extern __shared__ __align__(1024) float smem[];
  float* ring_buf = smem;
  __shared__ __align__(8) uint64_t full_bar[kGStages];    // TMA landed
  __shared__ __align__(8) uint64_t tile_bar[kGStages];    // MMAs reading the slot are done
  __shared__ __align__(8) uint64_t d1_bar[kGRowTiles][kGUStages];     // MMA1 of a chunk done
  __shared__ __align__(8) uint64_t afull_bar[kGRowTiles][kGUStages];  // K hi / lo in TMEM
  __shared__ __align__(8) uint64_t m2_bar[kGRowTiles][kGUStages];     // MMA2 of a chunk done
  __shared__ __align__(8) uint64_t accfree_bar[kGRowTiles][kGPar];    // window sum folded
  __shared__ __align__(8) uint64_t final_bar;
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  const int G = ntiles * kChunks;
  constexpr int kWin = kGWinTiles * kChunks;  // chunks per accumulation window
  static_assert(kWin % kGPar == 0, "every window starts on chunk class 0");
  const int nwin = (G + kWin - 1) / kWin;
  const uint32_t tile_bytes = TILE * sizeof(float);

  if (tid == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&tile_bar[s], kGRowTiles);
    }
    for (int r = 0; r < kGRowTiles; ++r)
      for (int s = 0; s < kGUStages; ++s) {
        mbar_init(&d1_bar[r][s], 1);
        mbar_init(&afull_bar[r][s], 128);
        mbar_init(&m2_bar[r][s], 1);
      }
    for (int r = 0; r < kGRowTiles; ++r)
      for (int p = 0; p < kGPar; ++p) mbar_init(&accfree_bar[r][p], 128);
    mbar_init(&final_bar, kGPar * kGRowTiles);
    fence_barrier_init();
  }
  if (warp == kTmaWarp) tmem_alloc(&tslot, kGTmemCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  const int rt = tid / 128;
  const int64_t i = (int64_t)blockIdx.x * kGEpiThreads + tid;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  if (tid < kGEpiThreads) {
    // Row operand of row i (TMEM lane i % 128): x hi, x lo, norm k-step.
    float x[DP];
#pragma unroll
    for (int k = 0; k < DP; ++k) x[k] = i < nrow ? xrow[i * DP + k] : 0.f;
    const uint32_t a_row = tmem + lane_off + kGColX + rt * 32;
#pragma unroll
    for (int k8 = 0; k8 < DP; k8 += 8) {
      uint32_t h[8], l[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float hv = tf32_hi(x[k8 + k]);
        h[k] = __float_as_uint(hv);
        l[k] = __float_as_uint(x[k8 + k] - hv);
      }
      tmem_st8(a_row + k8, h);
      tmem_st8(a_row + 16 + k8, l);
    }
    float e[8] = {0.f, 0.f, 0.f, 1.f, 1.f, 1.f, 0.f, 0.f};
    gram_split3(gram_sqnorm(x, DP), e[0], e[1], e[2]);
    uint32_t eb[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) eb[k] = __float_as_uint(e[k]);
    tmem_st8(tmem + lane_off + kGColN + rt * 8, eb);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  GRAM_DECL;
  auto off = [](int floats) -> uint64_t { return (uint64_t)((floats * 4) >> 4); };
  const uint32_t idesc = make_idesc_tf32(128, 16);

  if (warp == kTmaWarp) {
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int kt = 0; kt < ntiles && ok; ++kt) {
        const int slot = kt % kGStages;
        GRAM_T0(tw);
        if (kt >= kGStages) ok = mbar_wait_bounded(&tile_bar[slot], ((kt - kGStages) / kGStages) & 1);
        GRAM_ACC(7, tw);
        if (!ok) break;
        mbar_arrive_expect_tx(&full_bar[slot], tile_bytes);
        bulk_copy_g2s(ring_buf + slot * TILE, xv + (int64_t)(t0 + kt) * TILE, tile_bytes,
                      &full_bar[slot]);
        ++issued;
      }
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
      drain_ring<kGStages>(full_bar, issued);
    }
    __syncwarp();
  } else if (warp >= kIssuer0) {
    const int r = (warp - kIssuer0) / (2 * kGPar), role = (warp - kIssuer0) % (2 * kGPar);
    const int par = role % kGPar;  // chunks c with c % kGPar == par
    if (lane == 0 && role < kGPar) {
      // MMA1 of chunk c into stage c % 3 of row tile r, once MMA2 of chunk
      // c - 3 (the stage's previous reader) has completed.
      const uint64_t dring0 = make_smem_desc(ring_buf, 2048, 128);
      const uint32_t ax = tmem + kGColX + r * 32, an = tmem + kGColN + r * 8;
      bool ok = true;
      GRAM_T0(itot);
      for (int c = par; c < G && ok; c += kGPar) {
        const int st = c % kGUStages;
        const int kt = c / kChunks, q = c % kChunks, slot = kt % kGStages;
        if (c >= kGUStages) {
          GRAM_T0(mw);
          ok = mbar_wait_bounded(&m2_bar[r][st], ((c - kGUStages) / kGUStages) & 1);
          GRAM_ACC(4, mw);
          if (!ok) break;
        }
        if (q < kGPar) {
          GRAM_T0(fw);
          ok = mbar_wait_bounded(&full_bar[slot], (kt / kGStages) & 1);
          GRAM_ACC(5, fw);
          if (!ok) break;
        }
        tc_fence_after();
        const uint64_t db = dring0 + off(slot * TILE + q * 64);
        const uint32_t d = tmem + kGColS + r * 32 * kGUStages + st * 32;
#pragma unroll
        for (int ks = 0; ks < DP / 8; ++ks) {
          mma_tf32_tmem_a(d, ax + ks * 8, db + off(ks * 1024), idesc, ks > 0 ? 1u : 0u);
          mma_tf32_tmem_a(d, ax + ks * 8, db + off(128 * gram_kaug(DP) + ks * 1024), idesc, 1u);
          mma_tf32_tmem_a(d, ax + 16 + ks * 8, db + off(ks * 1024), idesc, 1u);
        }
        // Norm k-step: exact tf32 parts times exact ones, hi x hi only.
        mma_tf32_tmem_a(d, an, db + off(DP / 8 * 1024), idesc, 1u);
        mma_commit(&d1_bar[r][st]);
      }
      GRAM_ACC(3, itot);
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
    } else if (lane == 0) {
      // MMA2 of chunk c (c % 2 == par) into this warp's accumulator.
      const uint64_t dv0 = make_smem_desc(ring_buf + gram_v_offset(DP), 512, 128);
      const uint32_t acc = tmem + kGColAcc + r * 16 * kGPar + par * 16;
      bool ok = true;
      bool first = true;
      GRAM_T0(itot);
      for (int g = par; g < G && ok; g += kGPar) {
        const int st = g % kGUStages;
        const int kt = g / kChunks, q = g % kChunks, slot = kt % kGStages;
        // V is read by this thread's MMAs: observe the TMA completion here too.
        if (q < kGPar) ok = mbar_wait_bounded(&full_bar[slot], (kt / kGStages) & 1);
        if (!ok) break;
        // A new window restarts the accumulator once the epilogue has folded
        // the previous window's value.
        const int w = g / kWin;
        if (w > 0 && g % kWin == par) {
          ok = mbar_wait_bounded(&accfree_bar[r][par], (w - 1) & 1);
          if (!ok) break;
          first = true;
        }
        GRAM_T0(aw);
        ok = mbar_wait_bounded(&afull_bar[r][st], (g / kGUStages) & 1);
        GRAM_ACC(6, aw);
        if (!ok) break;
        tc_fence_after();
        const uint64_t dv = dv0 + off(slot * TILE + 2 * q * 256);
        const uint32_t a = tmem + kGColS + r * 32 * kGUStages + st * 32;
        // K hi V hi + K hi V lo + K lo V hi (N = 16; V lo is the second half).
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          mma_tf32_tmem_a(acc, a + kk * 8, dv + off(kk * 256), idesc, (first && kk == 0) ? 0u : 1u);
          mma_tf32_tmem_a(acc, a + kk * 8, dv + off(kk * 256 + 64), idesc, 1u);
          mma_tf32_tmem_a(acc, a + 16 + kk * 8, dv + off(kk * 256), idesc, 1u);
        }
        first = false;
        mma_commit(&m2_bar[r][st]);
        if (q == kChunks - 1) mma_commit(&tile_bar[slot]);
      }
      GRAM_ACC(2, itot);
      mma_commit(&final_bar);
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
      // No MMA of this thread may still be in flight when TMEM is released.
      mbar_wait_bounded(&final_bar, 0);
    }
    __syncwarp();
  } else {
    const uint32_t s_base = tmem + lane_off + kGColS + rt * 32 * kGUStages;
    const uint32_t acc_col = tmem + lane_off + kGColAcc + rt * 16 * kGPar;
    float wsum[16];  // finished accumulation windows (fp32, round to nearest)
#pragma unroll
    for (int c = 0; c < 16; ++c) wsum[c] = 0.f;
    bool ok = true;
    GRAM_T0(etot);
    for (int g = 0; g < G && ok; ++g) {
      const int st = g % kGUStages;
      GRAM_T0(dw);
      ok = mbar_wait_bounded(&d1_bar[rt][st], (g / kGUStages) & 1);
      GRAM_ACC(0, dw);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = s_base + st * 32;
      float u[16];
      tmem_ld16(taddr, u);  // includes tcgen05.wait::ld
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float kv = FastEval<LEAF>::value(u[h], fp);
        // The tensor core reads the top 19 bits of each 32-bit A element
        // (tf32 truncation), so k itself serves as the hi part and the lo
        // part is k minus its truncation.
        hi[h] = __float_as_uint(kv);
        lo[h] = __float_as_uint(kv - __uint_as_float(__float_as_uint(kv) & 0xFFFFE000u));
      }
      tmem_st16(taddr, hi);
      tmem_st16(taddr + 16, lo);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull_bar[rt][st]);
      if (g % kWin == 0 && g > 0) {
        // First chunk of a window: fold the previous window once its last
        // MMA2 of each chunk class has completed, and free the accumulators.
        // Doing it after this chunk's exponentials (not at the window's last
        // chunk) hides the MMA2 latency behind them.
#pragma unroll
        for (int p = 0; p < kGPar && ok; ++p) {
          const int gp = g - kGPar + p;
          ok = mbar_wait_bounded(&m2_bar[rt][gp % kGUStages], (gp / kGUStages) & 1);
        }
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int p = 0; p < kGPar; ++p) {
          float a[16];
          tmem_ld16(acc_col + 16 * p, a);
#pragma unroll
          for (int c = 0; c < 16; ++c) wsum[c] += a[c];
        }
        tc_fence_before();
#pragma unroll
        for (int p = 0; p < kGPar; ++p) mbar_arrive(&accfree_bar[rt][p]);
      }
    }
    GRAM_ACC(1, etot);
    if (ok) ok = mbar_wait_bounded(&final_bar, 0);
    tc_fence_after();
    if (!ok) {
      atomicExch(err, DEV_WAIT_TIMEOUT);
    } else {
      // The last window's accumulators, for the chunk classes that had a
      // chunk in it (a class without one still holds a folded window).
      float acc[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) acc[c] = 0.f;
      const int last0 = (nwin - 1) * kWin;
      for (int p = 0; p < kGPar && G > 0; ++p) {
        if (last0 + p >= G) break;
        float acc_p[16];
        tmem_ld16(acc_col + 16 * p, acc_p);
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[c] += acc_p[c];
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) acc[c] += wsum[c];
      const bool partial = gridDim.y > 1;
      if (i < nrow) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          if (c >= ep.tcols) continue;
          if (partial) {
            ep.out[((int64_t)split * 16 + c) * ep.out_ld + i] = acc[c];
          } else {
            float o = ep.scale * acc[c];
            if (ep.noise_v) {
              const float nz = ep.noise_vec ? ep.noise_vec[i] : ep.noise;
              o = fmaf(nz, ep.noise_v[c * ep.noise_ld + i], o);
            }
            ep.out[c * ep.out_ld + i] = o;
          }
        }
      }
    }
  }
  GRAM_FLUSH;
  tc_fence_before();
  __syncthreads();
  if (warp == kTmaWarp) tmem_dealloc(tmem, kGTmemCols);
}

// ---------------------------------------------------------------------------
// Narrow Gram kernel: the same MMA1 (u on the tensor core, A from TMEM), but
// the contraction with NV <= 8 columns runs on the CUDA cores in fp32
// (acc_c += k_ij v_jc) instead of the hi / lo split, the TMEM store and the
// three MMA2 products. The host routes only 1-column chunks here (a Lanczos
// step, an alpha solve): those run at 75 % of the MUFU bound, 1.37x the Gram
// kernel's entry rate; at 4 and 8 columns the Gram kernel is as fast or faster.
// CTA: 4 row tiles of 128 rows, 16 epilogue warps; per row tile two MMA1
// issuer warps (even / odd chunks); one TMA warp. TMEM: [x hi | x lo] and the
// norm k-step per row tile, then 5 stages x 16 columns of u per row tile.
// Packed tile (floats): [B hi : 128 x (DP + 8)][B lo : 128 x DP][V : 128 x NV].
constexpr int kG1RowTiles = 4;
constexpr int kG1UStages = 5;
constexpr int kG1Par = 2;
constexpr int kG1Stages = 6;
constexpr int kG1EpiThreads = 128 * kG1RowTiles;
constexpr int kG1IssuerWarps = kG1Par * kG1RowTiles;
constexpr int kG1Threads = kG1EpiThreads + 32 * kG1IssuerWarps + 32;
constexpr uint32_t kG1ColX = 0;
constexpr uint32_t kG1ColN = 32 * kG1RowTiles;
constexpr uint32_t kG1ColS = kG1ColN + 8 * kG1RowTiles;
static_assert(kG1ColS + 16 * kG1UStages * kG1RowTiles <= kGTmemCols, "TMEM budget");
__host__ __device__ constexpr int gram1_tile_floats(int DP, int NV) {
  return 128 * (2 * DP + 8) + 128 * NV;
}

template <int DP, int LEAF, int NV>
__global__ void __launch_bounds__(kG1Threads, 1) kv_tile_gram1_kernel(
    const float* __restrict__ xrow, int64_t nrow, const float* __restrict__ xv, int ntiles_total,
    int tiles_per_split, const __grid_constant__ FastParams fp, TileEpilogue ep, int* err) {
  static_assert(DP % 8 == 0 && DP <= 16, "K = DP in 8-wide tf32 k-steps, x hi / lo in 32 columns");
  static_assert(NV == 1 || NV == 2 || NV == 4 || NV == 8, "narrow column counts");
  constexpr int TILE = gram1_tile_floats(DP, NV);
  constexpr int kChunks = 128 / kGChunk;
  constexpr int kIssuer0 = kG1EpiThreads / 32;
  constexpr int kTmaWarp = kIssuer0 + kG1IssuerWarps;
  constexpr int kVOff = 128 * (2 * DP + 8);
  extern __shared__ __align__(1024) float smem[];
  float* ring_buf = smem;
  __shared__ __align__(8) uint64_t full_bar[kG1Stages];   // TMA landed
  __shared__ __align__(8) uint64_t tile_bar[kG1Stages];   // every epilogue warp is done with the slot
  __shared__ __align__(8) uint64_t d1_bar[kG1RowTiles][kG1UStages];  // MMA1 of a chunk done
  __shared__ __align__(8) uint64_t uf_bar[kG1RowTiles][kG1UStages];  // u of a chunk read
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  const int G = ntiles * kChunks;
  const uint32_t tile_bytes = TILE * sizeof(float);

  if (tid == 0) {
    for (int s = 0; s < kG1Stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&tile_bar[s], kG1EpiThreads / 32);
    }
    for (int r = 0; r < kG1RowTiles; ++r)
      for (int s = 0; s < kG1UStages; ++s) {
        mbar_init(&d1_bar[r][s], 1);
        mbar_init(&uf_bar[r][s], 4);
      }
    fence_barrier_init();
  }
  if (warp == kTmaWarp) tmem_alloc(&tslot, kGTmemCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  const int rt = tid / 128;
  const int64_t i = (int64_t)blockIdx.x * kG1EpiThreads + tid;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  if (tid < kG1EpiThreads) {
    float x[DP];
#pragma unroll
    for (int k = 0; k < DP; ++k) x[k] = i < nrow ? xrow[i * DP + k] : 0.f;
    const uint32_t a_row = tmem + lane_off + kG1ColX + rt * 32;
#pragma unroll
    for (int k8 = 0; k8 < DP; k8 += 8) {
      uint32_t h[8], l[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float hv = tf32_hi(x[k8 + k]);
        h[k] = __float_as_uint(hv);
        l[k] = __float_as_uint(x[k8 + k] - hv);
      }
      tmem_st8(a_row + k8, h);
      tmem_st8(a_row + 16 + k8, l);
    }
    float e[8] = {0.f, 0.f, 0.f, 1.f, 1.f, 1.f, 0.f, 0.f};
    gram_split3(gram_sqnorm(x, DP), e[0], e[1], e[2]);
    uint32_t eb[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) eb[k] = __float_as_uint(e[k]);
    tmem_st8(tmem + lane_off + kG1ColN + rt * 8, eb);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  auto off = [](int floats) -> uint64_t { return (uint64_t)((floats * 4) >> 4); };
  const uint32_t idesc = make_idesc_tf32(128, 16);

  if (warp == kTmaWarp) {
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int kt = 0; kt < ntiles && ok; ++kt) {
        const int slot = kt % kG1Stages;
        if (kt >= kG1Stages) ok = mbar_wait_bounded(&tile_bar[slot], ((kt - kG1Stages) / kG1Stages) & 1);
        if (!ok) break;
        mbar_arrive_expect_tx(&full_bar[slot], tile_bytes);
        bulk_copy_g2s(ring_buf + slot * TILE, xv + (int64_t)(t0 + kt) * TILE, tile_bytes,
                      &full_bar[slot]);
        ++issued;
      }
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
      drain_ring<kG1Stages>(full_bar, issued);
    }
    __syncwarp();
  } else if (warp >= kIssuer0) {
    const int r = (warp - kIssuer0) / kG1Par, par = (warp - kIssuer0) % kG1Par;
    if (lane == 0) {
      // MMA1 of chunk c into stage c % 5 of row tile r, once the epilogue has
      // read the stage's previous chunk.
      const uint64_t dring0 = make_smem_desc(ring_buf, 2048, 128);
      const uint32_t ax = tmem + kG1ColX + r * 32, an = tmem + kG1ColN + r * 8;
      bool ok = true;
      int last = -1;
      for (int c = par; c < G && ok; c += kG1Par) {
        const int st = c % kG1UStages;
        const int kt = c / kChunks, q = c % kChunks, slot = kt % kG1Stages;
        if (c >= kG1UStages) {
          ok = mbar_wait_bounded(&uf_bar[r][st], ((c - kG1UStages) / kG1UStages) & 1);
          if (!ok) break;
        }
        if (q < kG1Par) {
          ok = mbar_wait_bounded(&full_bar[slot], (kt / kG1Stages) & 1);
          if (!ok) break;
        }
        tc_fence_after();
        const uint64_t db = dring0 + off(slot * TILE + q * 64);
        const uint32_t d = tmem + kG1ColS + (r * kG1UStages + st) * 16;
#pragma unroll
        for (int ks = 0; ks < DP / 8; ++ks) {
          mma_tf32_tmem_a(d, ax + ks * 8, db + off(ks * 1024), idesc, ks > 0 ? 1u : 0u);
          mma_tf32_tmem_a(d, ax + ks * 8, db + off(128 * gram_kaug(DP) + ks * 1024), idesc, 1u);
          mma_tf32_tmem_a(d, ax + 16 + ks * 8, db + off(ks * 1024), idesc, 1u);
        }
        mma_tf32_tmem_a(d, an, db + off(DP / 8 * 1024), idesc, 1u);
        mma_commit(&d1_bar[r][st]);
        last = c;
      }
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
      // No MMA of this thread may still be in flight when TMEM is released.
      if (last >= 0) (void)mbar_wait_bounded(&d1_bar[r][last % kG1UStages], (last / kG1UStages) & 1);
    }
    __syncwarp();
  } else {
    const uint32_t s_base = tmem + lane_off + kG1ColS + rt * kG1UStages * 16;
    // Two-level fp32 sum: a running sum per column tile, folded into the
    // total once per tile, so no sum runs over more than 128 columns
    // (a flat fp32 sum over 1e6 columns drifts by ~u * sqrt(n) ~ 6e-5).
    float acc[NV], tot[NV];
#pragma unroll
    for (int c = 0; c < NV; ++c) acc[c] = tot[c] = 0.f;
    bool ok = true;
    for (int g = 0; g < G && ok; ++g) {
      const int st = g % kG1UStages;
      const int kt = g / kChunks, q = g % kChunks, slot = kt % kG1Stages;
      // V is read from shared memory by these threads: observe the TMA completion.
      if (q == 0) ok = mbar_wait_bounded(&full_bar[slot], (kt / kG1Stages) & 1);
      if (ok) ok = mbar_wait_bounded(&d1_bar[rt][st], (g / kG1UStages) & 1);
      if (!ok) break;
      tc_fence_after();
      float u[16];
      tmem_ld16(s_base + st * 16, u);  // includes tcgen05.wait::ld
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&uf_bar[rt][st]);
      const float* vs = ring_buf + slot * TILE + kVOff + q * 16 * NV;
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float kv = FastEval<LEAF>::value(u[h], fp);
#pragma unroll
        for (int c = 0; c < NV; ++c) acc[c] = fmaf(kv, vs[h * NV + c], acc[c]);
      }
      if (q == kChunks - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&tile_bar[slot]);
#pragma unroll
        for (int c = 0; c < NV; ++c) {
          tot[c] += acc[c];
          acc[c] = 0.f;
        }
      }
    }
#pragma unroll
    for (int c = 0; c < NV; ++c) acc[c] += tot[c];
    if (!ok) {
      atomicExch(err, DEV_WAIT_TIMEOUT);
    } else if (i < nrow) {
      const bool partial = gridDim.y > 1;
#pragma unroll
      for (int c = 0; c < NV; ++c) {
        if (c >= ep.tcols) continue;
        if (partial) {
          ep.out[((int64_t)split * NV + c) * ep.out_ld + i] = acc[c];
        } else {
          float o = ep.scale * acc[c];
          if (ep.noise_v) {
            const float nz = ep.noise_vec ? ep.noise_vec[i] : ep.noise;
            o = fmaf(nz, ep.noise_v[c * ep.noise_ld + i], o);
          }
          ep.out[c * ep.out_ld + i] = o;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTmaWarp) tmem_dealloc(tmem, kGTmemCols);
}

}  // namespace gpb
