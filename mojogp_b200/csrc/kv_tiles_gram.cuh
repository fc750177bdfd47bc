// Gram-form tensor-core K·V tile kernel (sm_100a tcgen05, kind::tf32).
//
// Both contractions of a K·V tile run on the tensor core:
//   MMA1  G = X_rows · (-2 Y_cols)^T      (3xTF32, K = DP)   -> TMEM
//   u_ij  = max(G_ij + |x_i|^2 + |y_j|^2, 0)                  (CUDA cores)
//   k_ij  = leaf(u_ij), split into tf32 hi / lo               -> TMEM
//   MMA2  D += K_hi V_hi + K_hi V_lo + K_lo V_hi  (A from TMEM) -> TMEM
// so the CUDA cores only turn squared distances into kernel values (one MUFU
// exponential per entry). The expansion |x|^2 + |y|^2 - 2 x·y loses absolute
// accuracy in proportion to the squared norms of the prescaled inputs; the
// host selects this path only when max_i |x'_i|^2 is small enough to keep the
// matvec inside the 1e-5 relative bar (provider_refresh_xs) and only for the
// leaves that are smooth in u at u = 0 (RBF, Matérn-3/2, Matérn-5/2, RQ);
// Matérn-1/2 (exp(-sqrt(u))) keeps the difference form.
//
// CTA: 4 row tiles of 128 rows; warpgroup r (warps 4r..4r+3) owns row tile r
// (TMEM lanes = rows), warp 16 + r issues its MMAs, warp 20 streams the
// column tiles. Column tiles of 128 columns stream through a 3-deep TMA ring
// and are consumed in chunks of 16 columns; per row tile the TMEM holds three chunk stages of 32 columns
// ([16 cols: G, then K hi][16 cols: K lo]) and a 16-column accumulator.
// tcgen05.mma instructions from one thread execute in issue order, so MMA1 of
// chunk g+3 may overwrite the stage that MMA2 of chunk g (issued before it)
// reads. Every wait is bounded.
#pragma once

#include "kv_tiles_tc.cuh"

namespace gpb {

constexpr int kGRowTiles = 4;
constexpr int kGChunk = 16;
constexpr int kGStages = 3;
constexpr int kGEpiThreads = 128 * kGRowTiles;
constexpr int kGThreads = kGEpiThreads + 32 * kGRowTiles + 32;
constexpr uint32_t kGTmemCols = 512;
constexpr int kGD1Stages = 3;   // chunk stages in TMEM per row tile
constexpr uint32_t kGAccCol = kGRowTiles * kGD1Stages * 32;

// Packed tile: [-2y hi : 128 x DP][-2y lo : 128 x DP][|y|^2 : 128]
//              [V hi : 16 k-steps x 128][V lo : 16 k-steps x 128] floats.
__host__ __device__ constexpr int gram_tile_floats(int DP) { return 128 * (2 * DP + 1) + 4096; }

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

template <int DP, int LEAF>
__global__ void __launch_bounds__(kGThreads, 1) kv_tile_gram_kernel(
    const float* __restrict__ xrow, int64_t nrow, const float* __restrict__ xv, int ntiles_total,
    int tiles_per_split, const __grid_constant__ FastParams fp, TileEpilogue ep, int* err) {
  // Warps 0-15: four warpgroups, warpgroup r turns G into K hi/lo for row
  // tile r (TMEM lanes = rows). Warps 16-19: issuer of row tile r's MMAs (one
  // per SM sub-partition). Warp 20: streams column tiles into the ring; a slot
  // is refilled once the four issuers' commits show every MMA reading it has
  // completed. Hand-offs are mbarriers only.
  static_assert(DP % 8 == 0, "K = DP in 8-wide tf32 k-steps");
  constexpr int TILE = gram_tile_floats(DP);
  constexpr int kChunks = 128 / kGChunk;
  constexpr int kIssuerWarp0 = kGEpiThreads / 32;
  constexpr int kTmaWarp = kIssuerWarp0 + kGRowTiles;
  extern __shared__ __align__(1024) float smem[];
  float* ring_buf = smem;
  float* a1 = smem + kGStages * TILE;  // per row tile: hi [128 x DP], lo [128 x DP]
  __shared__ __align__(8) uint64_t full_bar[kGStages];                // TMA landed
  __shared__ __align__(8) uint64_t tile_bar[kGStages];                // 4 issuers: slot done
  __shared__ __align__(8) uint64_t d1_bar[kGRowTiles][kGD1Stages];    // G of a stage in TMEM
  __shared__ __align__(8) uint64_t afull_bar[kGRowTiles][kGD1Stages]; // K hi/lo of a stage in TMEM
  __shared__ __align__(8) uint64_t final_bar[kGRowTiles];
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  const int G = ntiles * kChunks;
  const uint32_t tile_bytes = TILE * sizeof(float);

  if (tid == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&tile_bar[s], kGRowTiles);
    }
    for (int r = 0; r < kGRowTiles; ++r) {
      for (int s = 0; s < kGD1Stages; ++s) {
        mbar_init(&d1_bar[r][s], 1);
        mbar_init(&afull_bar[r][s], 128);
      }
      mbar_init(&final_bar[r], 1);
    }
    fence_barrier_init();
  }
  if (warp == kTmaWarp) tmem_alloc(&tslot, kGTmemCols);

  // Row operand: x_i split into tf32 hi / lo in the K-major layout.
  const int rt = tid / 128, m = tid % 128;
  const int64_t i = (int64_t)blockIdx.x * kGEpiThreads + tid;
  float na = 0.f;
  if (tid < kGEpiThreads) {
    float x[DP];
#pragma unroll
    for (int k = 0; k < DP; ++k) x[k] = i < nrow ? xrow[i * DP + k] : 0.f;
    na = gram_sqnorm(x, DP);
    float* ahi = a1 + rt * 2 * 128 * DP;
    float* alo = ahi + 128 * DP;
#pragma unroll
    for (int k = 0; k < DP; k += 4) {
      float4 h, l;
      h.x = tf32_hi(x[k]); l.x = x[k] - h.x;
      h.y = tf32_hi(x[k + 1]); l.y = x[k + 1] - h.y;
      h.z = tf32_hi(x[k + 2]); l.z = x[k + 2] - h.z;
      h.w = tf32_hi(x[k + 3]); l.w = x[k + 3] - h.w;
      *reinterpret_cast<float4*>(ahi + gram_xoff(m, k)) = h;
      *reinterpret_cast<float4*>(alo + gram_xoff(m, k)) = l;
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;

  if (warp == kTmaWarp) {
    if (lane == 0) {
      bool ok = true;
      for (int kt = 0; kt < ntiles && ok; ++kt) {
        const int slot = kt % kGStages;
        if (kt >= kGStages) ok = mbar_wait_bounded(&tile_bar[slot], ((kt - kGStages) / kGStages) & 1);
        if (!ok) break;
        mbar_arrive_expect_tx(&full_bar[slot], tile_bytes);
        bulk_copy_g2s(ring_buf + slot * TILE, xv + (int64_t)(t0 + kt) * TILE, tile_bytes,
                      &full_bar[slot]);
      }
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else if (warp >= kIssuerWarp0) {
    const int r = warp - kIssuerWarp0;
    if (lane == 0) {
      const uint32_t idesc = make_idesc_tf32(128, 16);
      const uint32_t d1_base = tmem + r * (kGD1Stages * 32);
      const uint32_t acc_col = tmem + kGAccCol + r * 16;
      // Descriptor bases; per-MMA offsets are added to the start-address field.
      const float* ahi = a1 + r * 2 * 128 * DP;
      const uint64_t dah0 = make_smem_desc(ahi, 2048, 128);
      const uint64_t dal0 = make_smem_desc(ahi + 128 * DP, 2048, 128);
      const uint64_t dring0 = make_smem_desc(ring_buf, 2048, 128);
      const uint64_t dv0 = make_smem_desc(ring_buf + 256 * DP + 128, 256, 128);
      auto off = [](int floats) -> uint64_t { return (uint64_t)((floats * 4) >> 4); };
      auto issue_mma1 = [&](int c) -> bool {
        const int kt = c / kChunks, q = c % kChunks, slot = kt % kGStages;
        if (q == 0) {
          if (!mbar_wait_bounded(&full_bar[slot], (kt / kGStages) & 1)) return false;
          tc_fence_after();
        }
        const uint64_t db = dring0 + off(slot * TILE + q * 64);
        const uint32_t d = d1_base + (c % kGD1Stages) * 32;
#pragma unroll
        for (int ks = 0; ks < DP / 8; ++ks) {
          mma_tf32(d, dah0 + off(ks * 1024), db + off(ks * 1024), idesc, ks > 0 ? 1u : 0u);
          mma_tf32(d, dah0 + off(ks * 1024), db + off(128 * DP + ks * 1024), idesc, 1u);
          mma_tf32(d, dal0 + off(ks * 1024), db + off(ks * 1024), idesc, 1u);
        }
        mma_commit(&d1_bar[r][c % kGD1Stages]);
        return true;
      };
      bool ok = true;
      for (int c = 0; c < kGD1Stages && c < G && ok; ++c) ok = issue_mma1(c);
      for (int g = 0; g < G && ok; ++g) {
        const int st = g % kGD1Stages;
        const int kt = g / kChunks, q = g % kChunks, slot = kt % kGStages;
        ok = mbar_wait_bounded(&afull_bar[r][st], (g / kGD1Stages) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint64_t dv = dv0 + off(slot * TILE + 2 * q * 128);
        const uint32_t a = d1_base + st * 32;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          mma_tf32_tmem_a(acc_col, a + kk * 8, dv + off(kk * 128), idesc, (g > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_tmem_a(acc_col, a + kk * 8, dv + off(2048 + kk * 128), idesc, 1u);
          mma_tf32_tmem_a(acc_col, a + 16 + kk * 8, dv + off(kk * 128), idesc, 1u);
        }
        if (q == kChunks - 1) mma_commit(&tile_bar[slot]);
        if (g + kGD1Stages < G) ok = issue_mma1(g + kGD1Stages);
      }
      mma_commit(&final_bar[r]);
      if (!ok) atomicExch(err, DEV_WAIT_TIMEOUT);
      // No MMA of this row tile may still be in flight when TMEM is released.
      mbar_wait_bounded(&final_bar[r], 0);
    }
    __syncwarp();
  } else {
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t d1_base = tmem + rt * (kGD1Stages * 32);
    const uint32_t acc_col = tmem + kGAccCol + rt * 16;
    bool ok = true;
    for (int g = 0; g < G && ok; ++g) {
      const int st = g % kGD1Stages;
      const int kt = g / kChunks, q = g % kChunks, slot = kt % kGStages;
      // |y_j|^2 is read from the ring slot with ordinary loads: observe the
      // TMA completion on the slot's barrier.
      if (q == 0) ok = mbar_wait_bounded(&full_bar[slot], (kt / kGStages) & 1);
      if (ok) ok = mbar_wait_bounded(&d1_bar[rt][st], (g / kGD1Stages) & 1);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = d1_base + lane_off + st * 32;
      uint32_t raw[16];
      tmem_ld16_async(taddr, raw);
      const float4* nbp =
          reinterpret_cast<const float4*>(ring_buf + slot * TILE + 256 * DP + q * kGChunk);
      float2 nb2[8];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float4 v = nbp[c];
        nb2[2 * c] = make_float2(v.x, v.y);
        nb2[2 * c + 1] = make_float2(v.z, v.w);
      }
      const float2 na2 = make_float2(na, na);
      tmem_wait_ld();
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float2 g2 = make_float2(__uint_as_float(raw[2 * c]), __uint_as_float(raw[2 * c + 1]));
        const float2 u2 = __fadd2_rn(__fadd2_rn(g2, nb2[c]), na2);
        const float2 k2 = make_float2(FastEval<LEAF>::value(u2.x, fp),
                                      FastEval<LEAF>::value(u2.y, fp));
        // The tensor core reads the top 19 bits of each 32-bit A element
        // (tf32 truncation), so k itself serves as the hi part and the lo
        // part is k minus its truncation.
        const float2 nt2 =
            make_float2(__uint_as_float((__float_as_uint(k2.x) & 0xFFFFE000u) ^ 0x80000000u),
                        __uint_as_float((__float_as_uint(k2.y) & 0xFFFFE000u) ^ 0x80000000u));
        const float2 l2 = __fadd2_rn(k2, nt2);
        hi[2 * c] = __float_as_uint(k2.x);
        hi[2 * c + 1] = __float_as_uint(k2.y);
        lo[2 * c] = __float_as_uint(l2.x);
        lo[2 * c + 1] = __float_as_uint(l2.y);
      }
      tmem_st16(taddr, hi);
      tmem_st16(taddr + 16, lo);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull_bar[rt][st]);
    }
    if (ok) ok = mbar_wait_bounded(&final_bar[rt], 0);
    tc_fence_after();
    if (!ok) {
      atomicExch(err, DEV_WAIT_TIMEOUT);
    } else {
      float acc[16];
      if (G > 0) {
        tmem_ld16(acc_col + lane_off, acc);
      } else {
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[c] = 0.f;
      }
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
  tc_fence_before();
  __syncthreads();
  if (warp == kTmaWarp) tmem_dealloc(tmem, kGTmemCols);
}

}  // namespace gpb
