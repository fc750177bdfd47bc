// Gram-form tensor-core K·V tile kernel (sm_100a tcgen05, kind::tf32).
//
// Both contractions of a K·V tile run on the tensor core:
//   MMA1  u = [x_i | |x_i|^2 parts | 1 1 1] · [-2 y_j | 1 1 1 | |y_j|^2 parts]
//           = |x_i|^2 + |y_j|^2 - 2 x_i·y_j       (3xTF32 on the x·y block)
//   k_ij  = leaf(u_ij), split into tf32 hi / lo   (CUDA cores)   -> TMEM
//   MMA2  D += K_hi [V_hi | V_lo] + K_lo V_hi     (A from TMEM)  -> TMEM
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
// CTA: 4 row tiles of 128 rows; warpgroup r (warps 4r..4r+3) owns row tile r
// (TMEM lanes = rows), warp 16 + r issues its MMAs, warp 20 streams the
// column tiles. Column tiles of 128 columns stream through a 3-deep TMA ring
// and are consumed in chunks of 16 columns; per row tile the TMEM holds three
// chunk stages of 32 columns ([16 cols: u, then K hi][16 cols: K lo]) and a
// 32-column accumulator ([K V hi + K lo V hi | K hi V lo], summed at the end). tcgen05.mma instructions from one thread execute in
// issue order, so MMA1 of chunk g+3 may overwrite the stage that MMA2 of chunk
// g (issued before it) reads. Every wait is bounded.
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

// Packed tile (floats): [B hi : 128 x (DP + 8)][B lo : 128 x DP]
//                      [V : 16 k-steps x 256, N = 32 rows (V hi | V lo)]
// with B = [-2y | 1 1 1 | |y|^2 parts | 0 0]; the row operand A (built by the
// kernel) is [x | |x|^2 parts | 1 1 1 | 0 0].
__host__ __device__ constexpr int gram_kaug(int DP) { return DP + 8; }
__host__ __device__ constexpr int gram_tile_floats(int DP) { return 128 * (2 * DP + 8) + 4096; }
__host__ __device__ constexpr int gram_v_offset(int DP) { return 128 * (2 * DP + 8); }
// Per row tile: A hi [128 x (DP + 8)], A lo [128 x DP].
__host__ __device__ constexpr int gram_a_floats(int DP) { return 128 * (2 * DP + 8); }

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
  float* a1 = smem + kGStages * TILE;  // per row tile: hi [128 x (DP+8)], lo [128 x DP]
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

  // Row operand: x_i split into tf32 hi / lo in the K-major layout, then
  // the norm k-step [|x|^2 parts | 1 1 1 | 0 0] (hi only).
  const int rt = tid / 128, m = tid % 128;
  const int64_t i = (int64_t)blockIdx.x * kGEpiThreads + tid;
  if (tid < kGEpiThreads) {
    float x[DP];
#pragma unroll
    for (int k = 0; k < DP; ++k) x[k] = i < nrow ? xrow[i * DP + k] : 0.f;
    float* ahi = a1 + rt * gram_a_floats(DP);
    float* alo = ahi + 128 * gram_kaug(DP);
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
    float4 e0, e1;
    gram_split3(gram_sqnorm(x, DP), e0.x, e0.y, e0.z);
    e0.w = 1.f;
    e1 = make_float4(1.f, 1.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(ahi + gram_xoff(m, DP)) = e0;
    *reinterpret_cast<float4*>(ahi + gram_xoff(m, DP + 4)) = e1;
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
      const uint32_t acc_col = tmem + kGAccCol + r * 32;
      const uint32_t idesc32 = make_idesc_tf32(128, 32);
      // Descriptor bases; per-MMA offsets are added to the start-address field.
      const float* ahi = a1 + r * gram_a_floats(DP);
      const uint64_t dah0 = make_smem_desc(ahi, 2048, 128);
      const uint64_t dal0 = make_smem_desc(ahi + 128 * gram_kaug(DP), 2048, 128);
      const uint64_t dring0 = make_smem_desc(ring_buf, 2048, 128);
      const uint64_t dv0 = make_smem_desc(ring_buf + gram_v_offset(DP), 512, 128);
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
          mma_tf32(d, dah0 + off(ks * 1024), db + off(128 * gram_kaug(DP) + ks * 1024), idesc, 1u);
          mma_tf32(d, dal0 + off(ks * 1024), db + off(ks * 1024), idesc, 1u);
        }
        // Norm k-step: exact tf32 parts times exact ones, hi x hi only.
        mma_tf32(d, dah0 + off(DP / 8 * 1024), db + off(DP / 8 * 1024), idesc, 1u);
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
        const uint64_t dv = dv0 + off(slot * TILE + 2 * q * 256);
        const uint32_t a = d1_base + st * 32;
        // K hi x [V hi | V lo] (N = 32) and K lo x V hi (N = 16, first half).
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          mma_tf32_tmem_a(acc_col, a + kk * 8, dv + off(kk * 256), idesc32, (g > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_tmem_a(acc_col, a + 16 + kk * 8, dv + off(kk * 256), idesc, 1u);
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
    const uint32_t acc_col = tmem + kGAccCol + rt * 32;
    bool ok = true;
    // Software pipeline: the TMEM load of chunk g+1 is in flight while chunk
    // g is evaluated. Two register buffers alternate (loop unrolled by two).
    auto fetch = [&](int c, uint32_t (&raw)[16]) -> bool {
      if (!mbar_wait_bounded(&d1_bar[rt][c % kGD1Stages], (c / kGD1Stages) & 1)) return false;
      tc_fence_after();
      tmem_ld16_async(d1_base + lane_off + (c % kGD1Stages) * 32, raw);
      return true;
    };
    auto process = [&](int c, const uint32_t (&raw)[16]) {
      const uint32_t taddr = d1_base + lane_off + (c % kGD1Stages) * 32;
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float kv = FastEval<LEAF>::value(__uint_as_float(raw[h]), fp);
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
      mbar_arrive(&afull_bar[rt][c % kGD1Stages]);
    };
    uint32_t rawA[16], rawB[16];
    if (G > 0) ok = fetch(0, rawA);
    for (int g = 0; g < G && ok; g += 2) {
      tmem_wait_ld();
      if (g + 1 < G) ok = fetch(g + 1, rawB);
      if (!ok) break;
      process(g, rawA);
      if (g + 1 >= G) break;
      tmem_wait_ld();
      if (g + 2 < G) ok = fetch(g + 2, rawA);
      if (!ok) break;
      process(g + 1, rawB);
    }
    if (ok) ok = mbar_wait_bounded(&final_bar[rt], 0);
    tc_fence_after();
    if (!ok) {
      atomicExch(err, DEV_WAIT_TIMEOUT);
    } else {
      float acc[16];
      if (G > 0) {
        float acc_lo[16];
        tmem_ld16(acc_col + lane_off, acc);
        tmem_ld16(acc_col + lane_off + 16, acc_lo);
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[c] += acc_lo[c];
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
