// Gram-form K·V tile kernel on fp16 tensor-core operands (sm_100a tcgen05,
// kind::f16, fp32 accumulation).
//
// Same product as kv_tile_gram_kernel (kv_tiles_gram.cuh), with both
// contractions on fp16 hi / lo splits instead of tf32 ones. One issuing thread
// completes one tcgen05.mma per ~207 cycles whatever its size (measured on
// this B200), so the kernel is bound by the number of MMAs it issues; a
// kind::f16 MMA has K = 16 where kind::tf32 has K = 8, and fp16 operands take
// half the TMEM. Per 16 columns and 128 rows:
//   MMA1 (u): DP = 16: xh·bh + xl·bh + xh·bl + norms (4 MMAs, was 7);
//             DP = 8:  [xh|xl]·[bh|bh] + [xh|nx]·[bl|ny] (2 MMAs, was 4);
//   MMA2 (K·V): K hi · [V hi | V lo] (N = 32) + K lo · V hi (N = 16)
//             (2 MMAs, was 6); D[:, 0:16] + D[:, 16:32] is the product.
// An fp16 hi / lo pair carries 22 significant bits, as a tf32 pair does. The
// range is handled by exact power-of-two scalings:
//   * inputs: the row side carries x'' = 16 x', the column side -2 y' / 16
//     (so the cross term is -2 x'.y' unscaled); |x'|^2 <= 100 by the Gram
//     gate keeps every operand inside fp16's normal range except components
//     below 2^-7, whose lo parts lose bits far below the 1e-5 bar. The norm
//     k-step also adds -12, so MMA1 yields u - 12 and the RBF value
//     k * 2^12 = 2^-(u - 12) is one MUFU ex2;
//   * kernel values: the lo part of k * 2^12 stays normal down to k ~ 2^-14;
//   * right-hand sides: column c is scaled by 2^e_c so that its largest
//     magnitude lies in [2^12, 2^13) (colmax pass before packing; the raw
//     maxima ride in every packed tile's tail), and the epilogue divides
//     again.
//
// Packed column tile (floats): NB MMA1 B blocks of [128 columns x 16] fp16
// (4 KB each, K-major core matrices: 8 rows x 16 B, K-adjacent 2048 B,
// N-adjacent 128 B), then per 16-column chunk a V block of 32 rows
// [V hi (16 output columns) | V lo (16)] x 16 fp16 (1 KB; K-adjacent 512 B),
// then 16 raw column maxima (float bits) and padding to 128 floats.
//
// CTA: 3 row tiles of 128 rows, 16-column chunks, 12 epilogue warps that take
// the chunks in pairs, per row tile two MMA1 issuer warps (even / odd chunks)
// and two MMA2 issuer warps (even / odd accumulators), one TMA warp; 5 chunk
// stages per row tile. Measured on this B200 at config 3: 202 TF/s with chunk
// pairs against 175 with one chunk per pass (the epilogue is bound by its
// TMEM load / store round trips) and 190 with 2 row tiles and two epilogue
// warpgroups per row tile (fewer issuers and rows per CTA); three MMA1 issuer
// warps per row tile instead of two measured 185 (more threads, fewer
// registers per thread).
// TMEM: accumulators [0, 192) (32 per row tile and class), row operands
// [192, 264) (three 8-column fp16 segments per row tile), stages
// [272, 512) (16 per stage: u in fp32, then K hi | K lo as fp16 pairs).
// Accumulators restart every kGWinTiles column tiles (the tensor core's
// accumulator truncates toward zero); every wait is bounded.
#pragma once

#include <cuda_fp16.h>

#include "kv_tiles_gram.cuh"

namespace gpb {

constexpr int kGHRowTiles = 3;
constexpr int kGHUStages = 5;
constexpr int kGHPar = 2;
constexpr int kGHEpiThreads = 128 * kGHRowTiles;
constexpr int kGHIssuerWarps = 2 * kGHPar * kGHRowTiles;
constexpr int kGHThreads = kGHEpiThreads + 32 * kGHIssuerWarps + 32;
constexpr uint32_t kGHColAcc = 0;    // + 64 r + 32 par
constexpr uint32_t kGHColA = 192;    // + 24 r + 8 seg
constexpr uint32_t kGHColS = 272;    // + 80 r + 16 st
static_assert(kGHColAcc + 32 * kGHPar * kGHRowTiles <= kGHColA, "TMEM map");
static_assert(kGHColA + 24 * kGHRowTiles <= kGHColS, "TMEM map");
static_assert(kGHColS + 16 * kGHUStages * kGHRowTiles <= 512, "TMEM budget");
constexpr float kGHInScale = 16.f;        // row side x'' = 16 x'; column side -2 y' / 16
constexpr float kGHUShift = 12.f;         // MMA1 yields u - 12, so 2^-(u - 12) = k * 2^12
constexpr float kGHKScale = 4096.f;       // K is carried as k * 2^12

__host__ __device__ constexpr int gramh_blocks(int DP) { return DP == 16 ? 3 : 2; }
__host__ __device__ constexpr int gramh_v_offset(int DP) { return gramh_blocks(DP) * 1024; }
__host__ __device__ constexpr int gramh_max_offset(int DP) { return gramh_v_offset(DP) + 2048; }
__host__ __device__ constexpr int gramh_tile_floats(int DP) { return gramh_max_offset(DP) + 128; }

// Byte offset of fp16 element (row n, k) in a K-major block whose 8-row core
// matrices are 128 B apart and whose K-adjacent core matrices are `lbo` apart.
__host__ __device__ constexpr int gramh_boff(int n, int k, int lbo) {
  return (k / 8) * lbo + (n / 8) * 128 + (n % 8) * 16 + (k % 8) * 2;
}

// Power-of-two scale for a column whose largest magnitude is m: m * s lies
// in [2^12, 2^13). Zero, NaN or infinite maxima keep scale 1.
__host__ __device__ inline float gramh_col_scale(float m) {
  if (!(m > 0.f) || !(m < 3.0e38f)) return 1.f;
  int e = 0;
  (void)frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1)
  return ldexpf(1.f, 13 - e);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// fp16 hi / lo parts of a pair (a, b): hi = fp16(v), lo = fp16(v - hi).
// The residual v - hi comes from sm_100's mixed-precision FMA (fp16 a and b,
// fp32 c and d): hi * (-1) + v, one instruction per value where an fp16 ->
// fp32 conversion followed by a subtraction took two; it is exact, since v
// minus its own fp16 rounding is representable in fp32. Measured at config 3:
// 215 TF/s against 204 with the conversion (the epilogue is issue-bound).
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = h2_bits(__floats2half2_rn(a, b));
  float ra, rb;
  asm("{\n\t.reg .f16 h0, h1, m1;\n\t"
      "mov.b16 m1, 0xBC00;\n\t"  // -1.0
      "mov.b32 {h0, h1}, %2;\n\t"
      "fma.rn.f32.f16 %0, h0, m1, %3;\n\t"
      "fma.rn.f32.f16 %1, h1, m1, %4;\n\t}"
      : "=f"(ra), "=f"(rb)
      : "r"(hi), "f"(a), "f"(b));
  lo = h2_bits(__floats2half2_rn(ra, rb));
}

// Three fp16 parts whose sum is v to ~2^-24 |v| (the last part may be
// subnormal; its absolute error stays below 2^-25).
__host__ __device__ inline void gramh_split3(float v, float& a, float& b, float& c) {
  a = __half2float(__float2half_rn(v));
  const float r = v - a;
  b = __half2float(__float2half_rn(r));
  c = __half2float(__float2half_rn(r - b));
}

__device__ __forceinline__ void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for tcgen05.mma kind::f16: D f32, A and B fp16, K-major.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int DP, int LEAF>
__global__ void __launch_bounds__(kGHThreads, 1) kv_tile_gramh_kernel(
    const float* __restrict__ xrow, int64_t nrow, const float* __restrict__ xv, int ntiles_total,
    int tiles_per_split, const __grid_constant__ FastParams fp, TileEpilogue ep, int* err) {
  static_assert(DP == 8 || DP == 16, "DP 8 or 16");
  constexpr int TILE = gramh_tile_floats(DP);
  constexpr int NB = gramh_blocks(DP);
  constexpr int kChunks = 128 / kGChunk;
  constexpr int kIssuer0 = kGHEpiThreads / 32;  // warp kIssuer0 + 2 P r + role
  constexpr int kTmaWarp = kIssuer0 + kGHIssuerWarps;
  constexpr int kWin = kGWinTiles * kChunks;
  static_assert(kWin % kGHPar == 0, "every window starts on chunk class 0");
  extern __shared__ __align__(1024) float smem[];
  float* ring_buf = smem;
  __shared__ __align__(8) uint64_t full_bar[kGStages];
  __shared__ __align__(8) uint64_t tile_bar[kGStages];
  __shared__ __align__(8) uint64_t d1_bar[kGHRowTiles][kGHUStages];
  __shared__ __align__(8) uint64_t afull_bar[kGHRowTiles][kGHUStages];
  __shared__ __align__(8) uint64_t m2_bar[kGHRowTiles][kGHUStages];
  __shared__ __align__(8) uint64_t accfree_bar[kGHRowTiles][kGHPar];
  __shared__ __align__(8) uint64_t final_bar;
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  const int G = ntiles * kChunks;
  const int nwin = (G + kWin - 1) / kWin;
  const uint32_t tile_bytes = TILE * sizeof(float);

  if (tid == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&tile_bar[s], kGHRowTiles * kGHPar);  // both MMA2 classes of each row tile
    }
    for (int r = 0; r < kGHRowTiles; ++r) {
      for (int s = 0; s < kGHUStages; ++s) {
        mbar_init(&d1_bar[r][s], 1);
        mbar_init(&afull_bar[r][s], 128);
        mbar_init(&m2_bar[r][s], 1);
      }
      for (int p = 0; p < kGHPar; ++p) mbar_init(&accfree_bar[r][p], 128);
    }
    mbar_init(&final_bar, kGHPar * kGHRowTiles);
    fence_barrier_init();
  }
  if (warp == kTmaWarp) tmem_alloc(&tslot, kGTmemCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  const int rt = tid / 128;
  const int64_t i = (int64_t)blockIdx.x * kGHEpiThreads + tid;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  if (tid < kGHEpiThreads) {
    // Row operand segments of row i (TMEM lane i % 128), fp16 pairs.
    float x[DP];
#pragma unroll
    for (int k = 0; k < DP; ++k) x[k] = i < nrow ? kGHInScale * xrow[i * DP + k] : 0.f;
    // [|x''|^2 parts | 1 1 1 | 1 (times -12) | 0]; the column side carries
    // 2^-8 on the first three slots, |y'|^2 on the next three, -12 on the 7th.
    float e[8] = {0.f, 0.f, 0.f, 1.f, 1.f, 1.f, 1.f, 0.f};
    gramh_split3(gram_sqnorm(x, DP), e[0], e[1], e[2]);
    const uint32_t a_row = tmem + lane_off + kGHColA + rt * 24;
    uint32_t hi[8], lo[8];
#pragma unroll
    for (int k = 0; k < DP; k += 2) split_h2(x[k], x[k + 1], hi[k / 2], lo[k / 2]);
    if constexpr (DP == 16) {
      uint32_t nv[8];
#pragma unroll
      for (int k = 0; k < 8; k += 2) nv[k / 2] = h2_bits(__floats2half2_rn(e[k], e[k + 1]));
#pragma unroll
      for (int k = 4; k < 8; ++k) nv[k] = 0u;
      tmem_st8(a_row, hi);       // segment 0: x hi
      tmem_st8(a_row + 8, lo);   // segment 1: x lo
      tmem_st8(a_row + 16, nv);  // segment 2: norm parts, ones
    } else {
      uint32_t s0[8], s1[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s0[k] = hi[k];
        s0[4 + k] = lo[k];
        s1[k] = hi[k];
        s1[4 + k] = h2_bits(__floats2half2_rn(e[2 * k], e[2 * k + 1]));
      }
      tmem_st8(a_row, s0);      // [x hi | x lo]
      tmem_st8(a_row + 8, s1);  // [x hi | norm parts, ones]
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  auto off = [](int floats) -> uint64_t { return (uint64_t)((floats * 4) >> 4); };
  const uint32_t idesc16 = make_idesc_f16(128, 16);
  const uint32_t idesc32 = make_idesc_f16(128, 32);

  if (warp == kTmaWarp) {
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int kt = 0; kt < ntiles && ok; ++kt) {
        const int slot = kt % kGStages;
        if (kt >= kGStages) ok = mbar_wait_bounded(&tile_bar[slot], ((kt - kGStages) / kGStages) & 1);
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
    const int r = (warp - kIssuer0) / (2 * kGHPar), role = (warp - kIssuer0) % (2 * kGHPar);
    const int par = role % kGHPar;
    if (lane == 0 && role < kGHPar) {
      // MMA1 of chunk c into stage c % S, once MMA2 of chunk c - S is done.
      const uint64_t dring0 = make_smem_desc(ring_buf, 2048, 128);
      const uint32_t a0 = tmem + kGHColA + r * 24;
      bool ok = true;
      for (int c = par; c < G && ok; c += kGHPar) {
        const int st = c % kGHUStages;
        const int kt = c / kChunks, q = c % kChunks, slot = kt % kGStages;
        if (c >= kGHUStages) {
          ok = mbar_wait_bounded(&m2_bar[r][st], ((c - kGHUStages) / kGHUStages) & 1);
          if (!ok) break;
        }
        if (q < kGHPar) {
          ok = mbar_wait_bounded(&full_bar[slot], (kt / kGStages) & 1);
          if (!ok) break;
        }
        tc_fence_after();
        const uint64_t db = dring0 + off(slot * TILE + q * 64);  // 16 rows = 256 B
        const uint32_t d = tmem + kGHColS + r * 16 * kGHUStages + st * 16;
        if constexpr (DP == 16) {
          mma_f16_tmem_a(d, a0, db, idesc16, 0u);                   // xh . bh
          mma_f16_tmem_a(d, a0 + 8, db, idesc16, 1u);               // xl . bh
          mma_f16_tmem_a(d, a0, db + off(1024), idesc16, 1u);       // xh . bl
          mma_f16_tmem_a(d, a0 + 16, db + off(2048), idesc16, 1u);  // norms
        } else {
          mma_f16_tmem_a(d, a0, db, idesc16, 0u);                // [xh|xl] . [bh|bh]
          mma_f16_tmem_a(d, a0 + 8, db + off(1024), idesc16, 1u);  // [xh|nx] . [bl|ny]
        }
        mma_commit(&d1_bar[r][st]);
      }
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
    } else if (lane == 0) {
      // MMA2 of chunk g (g % 2 == par) into this warp's accumulator.
      const uint64_t dv0 = make_smem_desc(ring_buf + gramh_v_offset(DP), 512, 128);
      const uint32_t acc = tmem + kGHColAcc + r * 32 * kGHPar + par * 32;
      bool ok = true;
      bool first = true;
      for (int g = par; g < G && ok; g += kGHPar) {
        const int st = g % kGHUStages;
        const int kt = g / kChunks, q = g % kChunks, slot = kt % kGStages;
        if (q < kGHPar) ok = mbar_wait_bounded(&full_bar[slot], (kt / kGStages) & 1);
        if (!ok) break;
        const int w = g / kWin;
        if (w > 0 && g % kWin == par) {
          ok = mbar_wait_bounded(&accfree_bar[r][par], (w - 1) & 1);
          if (!ok) break;
          first = true;
        }
        ok = mbar_wait_bounded(&afull_bar[r][st], (g / kGHUStages) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint64_t dv = dv0 + off(slot * TILE + q * 256);
        const uint32_t a = tmem + kGHColS + r * 16 * kGHUStages + st * 16;
        mma_f16_tmem_a(acc, a, dv, idesc32, first ? 0u : 1u);  // K hi . [V hi | V lo]
        mma_f16_tmem_a(acc, a + 8, dv, idesc16, 1u);            // K lo . V hi
        first = false;
        mma_commit(&m2_bar[r][st]);
        if (q >= kChunks - kGHPar) mma_commit(&tile_bar[slot]);
      }
      mma_commit(&final_bar);
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
      mbar_wait_bounded(&final_bar, 0);
    }
    __syncwarp();
  } else {
    const uint32_t s_base = tmem + lane_off + kGHColS + rt * 16 * kGHUStages;
    const uint32_t acc_col = tmem + lane_off + kGHColAcc + rt * 32 * kGHPar;
    float wsum[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) wsum[c] = 0.f;
    auto add_acc = [&](int p, float (&s)[16]) {
      float a[16], b[16];
      tmem_ld16(acc_col + 32 * p, a);
      tmem_ld16(acc_col + 32 * p + 16, b);
#pragma unroll
      for (int c = 0; c < 16; ++c) s[c] += a[c] + b[c];
    };
    // Chunk values of one 16-column stage: k * 2^12 as fp16 hi / lo pairs.
    auto eval16 = [&](const uint32_t (&ub)[16], uint32_t (&hi)[8], uint32_t (&lo)[8]) {
#pragma unroll
      for (int h = 0; h < 16; h += 2) {
        const float u0 = __uint_as_float(ub[h]), u1 = __uint_as_float(ub[h + 1]);
        float k0, k1;
        if constexpr (LEAF == GPB_KERNEL_RBF) {
          k0 = ex2_approx(-u0);
          k1 = ex2_approx(-u1);
        } else {
          k0 = kGHKScale * FastEval<LEAF>::value(u0 + kGHUShift, fp);
          k1 = kGHKScale * FastEval<LEAF>::value(u1 + kGHUShift, fp);
        }
        split_h2(k0, k1, hi[h / 2], lo[h / 2]);
      }
    };
    // Two chunks (one of each MMA1 class) per pass: both TMEM loads are in
    // flight together and one store wait covers both, which halves the
    // per-chunk load / store round trips that bound a one-chunk loop.
    static_assert(kChunks % 2 == 0 && kWin % 2 == 0, "chunk pairs");
    bool ok = true;
    for (int g = 0; g < G && ok; g += 2) {
      const int st0 = g % kGHUStages, st1 = (g + 1) % kGHUStages;
      ok = mbar_wait_bounded(&d1_bar[rt][st0], (g / kGHUStages) & 1) &&
           mbar_wait_bounded(&d1_bar[rt][st1], ((g + 1) / kGHUStages) & 1);
      if (!ok) break;
      tc_fence_after();
      const uint32_t ta0 = s_base + st0 * 16, ta1 = s_base + st1 * 16;
      uint32_t u0[16], u1[16];
      tmem_ld16_async(ta0, u0);
      tmem_ld16_async(ta1, u1);
      tmem_wait_ld();
      {
        uint32_t hi[8], lo[8];
        eval16(u0, hi, lo);
        tmem_st8(ta0, hi);
        tmem_st8(ta0 + 8, lo);
      }
      {
        uint32_t hi[8], lo[8];
        eval16(u1, hi, lo);
        tmem_st8(ta1, hi);
        tmem_st8(ta1 + 8, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull_bar[rt][st0]);
      mbar_arrive(&afull_bar[rt][st1]);
      if (g % kWin == 0 && g > 0) {
        // First chunks of a window: fold the previous window once its last
        // MMA2 of each class has completed (those stages are next used by
        // chunks g + 3 and g + 4, whose MMA2s cannot have run yet), then
        // free the accumulators.
#pragma unroll
        for (int p = 0; p < kGHPar && ok; ++p) {
          const int gp = g - kGHPar + p;
          ok = mbar_wait_bounded(&m2_bar[rt][gp % kGHUStages], (gp / kGHUStages) & 1);
        }
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int p = 0; p < kGHPar; ++p) add_acc(p, wsum);
        tc_fence_before();
#pragma unroll
        for (int p = 0; p < kGHPar; ++p) mbar_arrive(&accfree_bar[rt][p]);
      }
    }
    if (ok) ok = mbar_wait_bounded(&final_bar, 0);
    tc_fence_after();
    if (!ok) {
      atomicExch(err, DEV_WAIT_TIMEOUT);
    } else {
      float acc[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) acc[c] = wsum[c];
      const int last0 = (nwin - 1) * kWin;
      for (int p = 0; p < kGHPar && G > 0; ++p) {
        if (last0 + p >= G) break;
        add_acc(p, acc);
      }
      // Undo the column and kernel-value scalings (raw maxima from the tile tail).
      const float* mx = xv + (int64_t)t0 * TILE + gramh_max_offset(DP);
      const bool partial = gridDim.y > 1;
      if (i < nrow && G > 0) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          if (c >= ep.tcols) continue;
          const float v = acc[c] / (gramh_col_scale(mx[c]) * kGHKScale);
          if (partial) {
            ep.out[((int64_t)split * 16 + c) * ep.out_ld + i] = v;
          } else {
            float o = ep.scale * v;
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
  tc_fence_before();
  __syncthreads();
  if (warp == kTmaWarp) tmem_dealloc(tmem, kGTmemCols);
}

}  // namespace gpb
