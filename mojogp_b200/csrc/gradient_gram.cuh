// Tensor-core (tcgen05, kind::tf32) reduction for the RBF kernel-parameter
// gradients: the bilinear forms sum_ij w_ij dK_ij/dtheta with w_ij = a_i . b_j
// (the data column or the probe columns of one BBMM pass).
//
// For RBF in prescaled coordinates z (k_ij = 2^-u_ij, u_ij = |z_i - z_j|^2):
//   S_k = sum_ij k_ij w_ij (z_ik - z_jk)^2,   S_os = sum_ij k_ij w_ij.
// With e_ij = k_ij w_ij and, per row i, m_i = sum_j e_ij [1 | z_j | z_j^2]
//   S_k = sum_i (z_ik^2 m0_i + m2_ik - 2 z_ik m1_ik),   S_os = sum_i m0_i,
// so the pair loop becomes the Gram K.V kernel with two changes: an extra
// MMA forms w = a_i . b_j (3xTF32, A = a from TMEM) next to u, the epilogue
// writes e = k w (hi / lo) instead of k, and MMA2's B operand is
// B' = [1 | z | z^2] (hi / lo stacked along N, N = 80: [B'hi (40) | B'lo (40)])
// instead of V. The result is the same set of accumulators as the FP32
// bilinear kernel (bilinear_fast_kernel): A[k] = 2 ln2 S_k, A[DP] = S_os.
//
// CTA: 2 row tiles of 128 rows (TMEM lanes = rows). Warps 0-7: epilogue
// (warpgroup r = row tile r); per row tile, warps 8 + 3r and 9 + 3r issue
// MMA1 + MMA_w of the even / odd chunks and warp 10 + 3r issues MMA2 (one
// accumulator, one chain); warp 14 streams the column tiles (2-deep TMA
// ring). TMEM columns per row tile: [x hi | x lo] 32, norm k-step 8,
// [a hi | a lo] 32, three 32-column chunk stages ([16: u -> e hi][16: w -> e lo]),
// an 80-column accumulator. Every wait is bounded; the final per-row sums are
// reduced in a fixed order (deterministic).
#pragma once

#include "kv_tiles_gram.cuh"

namespace gpb {

constexpr int kGBRowTiles = 2;
constexpr int kGBStages = 2;    // column-tile ring
constexpr int kGBUStages = 3;   // chunk stages in TMEM
constexpr int kGBEpi = 128 * kGBRowTiles;
constexpr int kGBThreads = kGBEpi + 32 * 3 * kGBRowTiles + 32;
constexpr int kGBN = 80;        // MMA2 N: [B'hi | B'lo], 40 each (1 + 2 DP <= 40)
// Accumulation window in column tiles: MMA2 restarts its accumulator every
// kGBWinTiles tiles and the epilogue folds each finished window into its
// per-row sums in fp32 registers, because the tensor core's accumulator
// truncates toward zero on every add (see kGWinTiles).
constexpr int kGBWinTiles = 4;
constexpr uint32_t kGBColX = 0;                        // + 32 r
constexpr uint32_t kGBColN = 32 * kGBRowTiles;         // + 8 r
constexpr uint32_t kGBColA = kGBColN + 8 * kGBRowTiles;  // + 32 r : [a hi | a lo]
constexpr uint32_t kGBColS = kGBColA + 32 * kGBRowTiles; // + 96 r + 32 s
constexpr uint32_t kGBColAcc = kGBColS + 32 * kGBUStages * kGBRowTiles;  // + 80 r
static_assert(kGBColAcc + kGBN * kGBRowTiles <= 512, "TMEM budget");

// Gradient tile (floats): [gram B hi | gram B lo] (the K.V Gram layout's first
// part), [b hi : 128 x 16][b lo : 128 x 16] (K-major, gram_xoff), then B' in
// 16 k-steps of 8 columns x 80 rows (core matrices 8 n x 4 k, K-adjacent at
// 1280 B, N-adjacent at 128 B).
__host__ __device__ constexpr int gb_b_offset(int DP) { return 128 * (2 * DP + 8); }
__host__ __device__ constexpr int gb_bp_offset(int DP) { return gb_b_offset(DP) + 4096; }
__host__ __device__ constexpr int gb_tile_floats(int DP) { return gb_bp_offset(DP) + 16 * 8 * kGBN; }
__host__ __device__ constexpr int gb_bp_off(int n, int k) {
  return (k / 8) * (8 * kGBN) + ((k % 8) / 4) * (4 * kGBN) + (n / 8) * 32 + (n % 8) * 4 + (k % 4);
}

__device__ __forceinline__ void named_bar_sync_gb(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Accumulators written per CTA: DP + 2 floats in the bilinear_fast_kernel
// layout of one half (A[k], A[DP]; the last slot is unused for RBF).
template <int DP>
__global__ void __launch_bounds__(kGBThreads, 1) gb_kernel(
    const float* __restrict__ xrow, const float* __restrict__ a, int64_t nrow, int64_t a_ld,
    int col0, int ncol, const float* __restrict__ xv, int ntiles_total, int tiles_per_split,
    float* __restrict__ partial, int* err) {
  static_assert(DP % 8 == 0 && DP <= 16, "DP 8 or 16");
  constexpr int TILE = gb_tile_floats(DP);
  constexpr int kChunks = 128 / kGChunk;
  constexpr int kIss0 = kGBEpi / 32;
  constexpr int kTma = kIss0 + 3 * kGBRowTiles;
  constexpr int NACC = DP + 2;
  extern __shared__ __align__(1024) float smem[];
  float* ring = smem;
  __shared__ __align__(8) uint64_t full_bar[kGBStages], tile_bar[kGBStages];
  __shared__ __align__(8) uint64_t d1_bar[kGBRowTiles][kGBUStages];
  __shared__ __align__(8) uint64_t afull_bar[kGBRowTiles][kGBUStages];
  __shared__ __align__(8) uint64_t m2_bar[kGBRowTiles][kGBUStages];
  __shared__ __align__(8) uint64_t final_bar[kGBRowTiles];
  __shared__ __align__(8) uint64_t accfree_bar[kGBRowTiles];  // window folded
  __shared__ float red[kGBEpi / 32][NACC];
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  const int G = ntiles * kChunks;
  constexpr int kWin = kGBWinTiles * kChunks;  // chunks per accumulation window
  const uint32_t tile_bytes = TILE * sizeof(float);
  if (tid == 0) {
    for (int s = 0; s < kGBStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&tile_bar[s], kGBRowTiles);
    }
    for (int r = 0; r < kGBRowTiles; ++r) {
      for (int s = 0; s < kGBUStages; ++s) {
        mbar_init(&d1_bar[r][s], 1);
        mbar_init(&afull_bar[r][s], 128);
        mbar_init(&m2_bar[r][s], 1);
      }
      mbar_init(&final_bar[r], 1);
      mbar_init(&accfree_bar[r], 128);
    }
    fence_barrier_init();
  }
  if (warp == kTma) tmem_alloc(&tslot, 512);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  const int rt = tid / 128;
  const int64_t i = (int64_t)blockIdx.x * kGBEpi + tid;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  float x[DP];
  if (tid < kGBEpi) {
    // Row operands in TMEM: x hi / lo, the norm k-step, a hi / lo (columns
    // col0 .. col0 + ncol - 1 of this pass; the others zero).
#pragma unroll
    for (int k = 0; k < DP; ++k) x[k] = i < nrow ? xrow[i * DP + k] : 0.f;
    const uint32_t row = tmem + lane_off;
#pragma unroll
    for (int k8 = 0; k8 < DP; k8 += 8) {
      uint32_t h[8], l[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float hv = tf32_hi(x[k8 + k]);
        h[k] = __float_as_uint(hv);
        l[k] = __float_as_uint(x[k8 + k] - hv);
      }
      tmem_st8(row + kGBColX + rt * 32 + k8, h);
      tmem_st8(row + kGBColX + rt * 32 + 16 + k8, l);
    }
    float e[8] = {0.f, 0.f, 0.f, 1.f, 1.f, 1.f, 0.f, 0.f};
    gram_split3(gram_sqnorm(x, DP), e[0], e[1], e[2]);
    uint32_t eb[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) eb[k] = __float_as_uint(e[k]);
    tmem_st8(row + kGBColN + rt * 8, eb);
    uint32_t ah[16], al[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const bool on = i < nrow && c >= col0 && c < col0 + ncol;
      const float av = on ? a[(int64_t)c * a_ld + i] : 0.f;
      const float hv = tf32_hi(av);
      ah[c] = __float_as_uint(hv);
      al[c] = __float_as_uint(av - hv);
    }
    tmem_st16(row + kGBColA + rt * 32, ah);
    tmem_st16(row + kGBColA + rt * 32 + 16, al);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  auto off = [](int floats) -> uint64_t { return (uint64_t)((floats * 4) >> 4); };
  const uint32_t idesc16 = make_idesc_tf32(128, 16);

  if (warp == kTma) {
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int kt = 0; kt < ntiles && ok; ++kt) {
        const int slot = kt % kGBStages;
        if (kt >= kGBStages) ok = mbar_wait_bounded(&tile_bar[slot], ((kt - kGBStages) / kGBStages) & 1);
        if (!ok) break;
        mbar_arrive_expect_tx(&full_bar[slot], tile_bytes);
        bulk_copy_g2s(ring + slot * TILE, xv + (int64_t)(t0 + kt) * TILE, tile_bytes, &full_bar[slot]);
        ++issued;
      }
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
      drain_ring<kGBStages>(full_bar, issued);
    }
    __syncwarp();
  } else if (warp >= kIss0) {
    const int r = (warp - kIss0) / 3, role = (warp - kIss0) % 3;
    if (lane == 0 && role < 2) {
      // MMA1 (u) and MMA_w (w = a . b) of the chunks c with c % 2 == role.
      const uint64_t dring0 = make_smem_desc(ring, 2048, 128);
      const uint32_t ax = tmem + kGBColX + r * 32, an = tmem + kGBColN + r * 8;
      const uint32_t aa = tmem + kGBColA + r * 32;
      bool ok = true;
      for (int c = role; c < G && ok; c += 2) {
        const int st = c % kGBUStages;
        const int kt = c / kChunks, q = c % kChunks, slot = kt % kGBStages;
        if (c >= kGBUStages) ok = mbar_wait_bounded(&m2_bar[r][st], ((c - kGBUStages) / kGBUStages) & 1);
        if (ok && q < 2) ok = mbar_wait_bounded(&full_bar[slot], (kt / kGBStages) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint64_t db = dring0 + off(slot * TILE + q * 64);
        const uint64_t dw = dring0 + off(slot * TILE + gb_b_offset(DP) + q * 64);
        const uint32_t d = tmem + kGBColS + r * 96 + st * 32;
#pragma unroll
        for (int ks = 0; ks < DP / 8; ++ks) {
          mma_tf32_tmem_a(d, ax + ks * 8, db + off(ks * 1024), idesc16, ks > 0 ? 1u : 0u);
          mma_tf32_tmem_a(d, ax + ks * 8, db + off(128 * gram_kaug(DP) + ks * 1024), idesc16, 1u);
          mma_tf32_tmem_a(d, ax + 16 + ks * 8, db + off(ks * 1024), idesc16, 1u);
        }
        mma_tf32_tmem_a(d, an, db + off(DP / 8 * 1024), idesc16, 1u);
        // w = a . b over the 16 right-hand-side columns (two k-steps).
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          mma_tf32_tmem_a(d + 16, aa + ks * 8, dw + off(ks * 1024), idesc16, ks > 0 ? 1u : 0u);
          mma_tf32_tmem_a(d + 16, aa + ks * 8, dw + off(2048 + ks * 1024), idesc16, 1u);
          mma_tf32_tmem_a(d + 16, aa + 16 + ks * 8, dw + off(ks * 1024), idesc16, 1u);
        }
        mma_commit(&d1_bar[r][st]);
      }
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
    } else if (lane == 0) {
      // MMA2: acc += e_hi [B'hi | B'lo] (N = 80) + e_lo B'hi (N = 48).
      const uint32_t idesc80 = make_idesc_tf32(128, kGBN);
      const uint32_t idesc48 = make_idesc_tf32(128, 48);
      // B' k-step: K-adjacent core matrices 4 * 80 floats (1280 B) apart.
      const uint64_t dp0 = make_smem_desc(ring + gb_bp_offset(DP), 4 * kGBN * 4, 128);
      const uint32_t acc = tmem + kGBColAcc + r * kGBN;
      bool ok = true;
      for (int g = 0; g < G && ok; ++g) {
        const int st = g % kGBUStages;
        const int kt = g / kChunks, q = g % kChunks, slot = kt % kGBStages;
        if (q == 0) ok = mbar_wait_bounded(&full_bar[slot], (kt / kGBStages) & 1);
        // A new window restarts the accumulator once the epilogue has folded
        // the previous one.
        if (ok && g > 0 && g % kWin == 0)
          ok = mbar_wait_bounded(&accfree_bar[r], (g / kWin - 1) & 1);
        if (ok) ok = mbar_wait_bounded(&afull_bar[r][st], (g / kGBUStages) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t ae = tmem + kGBColS + r * 96 + st * 32;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t dbp = dp0 + off(slot * TILE + (2 * q + kk) * 8 * kGBN);
          mma_tf32_tmem_a(acc, ae + kk * 8, dbp, idesc80, (g % kWin > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_tmem_a(acc, ae + 16 + kk * 8, dbp, idesc48, 1u);
        }
        mma_commit(&m2_bar[r][st]);
        if (q == kChunks - 1) mma_commit(&tile_bar[slot]);
      }
      mma_commit(&final_bar[r]);
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
      mbar_wait_bounded(&final_bar[r], 0);
    }
    __syncwarp();
  } else {
    const uint32_t s_base = tmem + lane_off + kGBColS + rt * 96;
    const uint32_t ab = tmem + lane_off + kGBColAcc + rt * kGBN;
    // Per-row sums of the folded windows. The accumulators are linear in the
    // pair terms, so each window's m0, m1, m2 are combined into the gradient
    // sums right away.
    float vals[NACC];
#pragma unroll
    for (int q = 0; q < NACC; ++q) vals[q] = 0.f;
    auto fold = [&]() {
      float acc[kGBN];
#pragma unroll
      for (int c = 0; c < kGBN; c += 16) {
        float tmp[16];
        tmem_ld16(ab + c, tmp);
#pragma unroll
        for (int h = 0; h < 16; ++h) acc[c + h] = tmp[h];
      }
      if (i < nrow) {
        const float m0 = acc[0] + acc[40];
#pragma unroll
        for (int k = 0; k < DP; ++k) {
          const float m1 = acc[1 + k] + acc[41 + k];
          const float m2 = acc[1 + DP + k] + acc[41 + DP + k];
          vals[k] += fmaf(x[k] * x[k], m0, fmaf(-2.f * x[k], m1, m2)) * (2.f * kLn2);
        }
        vals[DP] += m0;
      }
    };
    bool ok = true;
    for (int g = 0; g < G && ok; ++g) {
      const int st = g % kGBUStages;
      ok = mbar_wait_bounded(&d1_bar[rt][st], (g / kGBUStages) & 1);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = s_base + st * 32;
      float u[16], w[16];
      tmem_ld16(taddr, u);
      tmem_ld16(taddr + 16, w);
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float ev = ex2_approx(-u[h]) * w[h];
        hi[h] = __float_as_uint(ev);  // the tensor core truncates to tf32
        lo[h] = __float_as_uint(ev - __uint_as_float(__float_as_uint(ev) & 0xFFFFE000u));
      }
      tmem_st16(taddr, hi);
      tmem_st16(taddr + 16, lo);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull_bar[rt][st]);
      if (g % kWin == 0 && g > 0) {
        // First chunk of a window: fold the previous window once its last
        // MMA2 has completed (after this chunk's work, hiding the latency).
        const int gp = g - 1;
        ok = mbar_wait_bounded(&m2_bar[rt][gp % kGBUStages], (gp / kGBUStages) & 1);
        if (!ok) break;
        tc_fence_after();
        fold();
        tc_fence_before();
        mbar_arrive(&accfree_bar[rt]);
      }
    }
    if (ok) ok = mbar_wait_bounded(&final_bar[rt], 0);
    tc_fence_after();
    if (!ok) {
      atomicExch(err, DEV_WAIT_TIMEOUT);
#pragma unroll
      for (int q = 0; q < NACC; ++q) vals[q] = 0.f;
    } else if (G > 0) {
      fold();  // the last window
    }
    // Fixed-order reduction over the CTA's rows.
#pragma unroll
    for (int q = 0; q < NACC; ++q) {
      float v = vals[q];
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp][q] = v;
    }
    named_bar_sync_gb(1, kGBEpi);
    if (tid < NACC) {
      float s = 0.f;
      for (int wv = 0; wv < kGBEpi / 32; ++wv) s += red[wv][tid];
      const int64_t bid = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
      partial[bid * NACC + tid] = s;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTma) tmem_dealloc(tmem, 512);
}

}  // namespace gpb
