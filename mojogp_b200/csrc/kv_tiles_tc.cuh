// Tensor-core K·V tile kernel (sm_100a tcgen05, kind::tf32, 3xTF32 split).
//
// The pair work stays on the CUDA cores: each thread owns two rows x_i (in
// registers) and forms k(x_i, x_j) for 16 columns at a time (FFMA distance +
// one MUFU exponential). The contraction sum_j K_ij V_jc, which is 16 of the
// 48 FP32 lane-operations per kernel entry on the FFMA path, moves to the
// tensor core: the K block is written to shared memory as tf32 hi / lo parts
// (hi = K rounded to tf32 with integer ops, lo = K - hi) in the no-swizzle
// K-major core-matrix layout, V arrives pre-split (hi / lo) in the same layout
// from the packed column tiles, and one elected thread issues
// D += Khi Vhi + Khi Vlo + Klo Vhi (three M=128, N=16, K=8 MMAs per 8 columns
// and row tile) into TMEM accumulators. The dropped lo x lo term and the
// tf32 truncation of the lo parts leave ~2^-21 relative error per product,
// inside the 1e-5 matvec bar.
//
// Pipeline: column tiles (x' block + V hi/lo blocks) stream through a 2-deep
// TMA ring; K blocks double-buffer so threads fill chunk g+1 while the tensor
// core consumes chunk g; tcgen05.commit arrivals on per-stage mbarriers gate
// buffer reuse. Every wait is bounded.
#pragma once

#include "kv_tiles.cuh"
#include "tcgen05.cuh"

namespace gpb {

constexpr int kTcStages = 2;       // column-tile ring depth
constexpr int kTcChunk = 8;        // columns per K block (one MMA k-step)
constexpr int kTcRows = 4;         // row tiles (M = 128 each) per CTA
constexpr int kTcThreads = 128;
constexpr int kTcAStageBytes = kTcRows * 2 * 128 * kTcChunk * 4;  // hi + lo, both row tiles
// Accumulation window in column tiles. The tensor core's fp32 accumulator
// truncates toward zero on every add, so a chain of MMAs over a 1e6-column
// row drifts by ~1e-3 relative. The MMAs of window w accumulate into TMEM
// set w % 2 from zero; while window w runs, the row threads fold window
// w - 1's set into a TMEM sum (fp32, round to nearest). TMEM: [set 0 | set 1 |
// sum], 16 columns per row tile each.
constexpr int kTcWinTiles = 4;
constexpr uint32_t kTcTmemCols = 256;
static_assert(3 * 16 * kTcRows <= kTcTmemCols, "TMEM budget");

// Packed tile: [-x' : 128 x DP][V hi : 16 k-steps x 128][V lo : 16 k-steps x 128] floats.
__host__ __device__ constexpr int tc_tile_floats(int DP) { return 128 * DP + 2 * 16 * 128; }

// Offset (floats) of element (n, k) inside one 8-column k-step of the B block:
// core matrices of 8 rows x 4 k, K-adjacent at 256 B, N-adjacent at 128 B.
__host__ __device__ constexpr int tc_b_offset(int nidx, int k) {
  return (k / 4) * 64 + (nidx / 8) * 32 + (nidx % 8) * 4 + (k % 4);
}

__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

template <int DP, int LEAF>
__global__ void __launch_bounds__(kTcThreads + 32, 2) kv_tile_tc_kernel(
    const float* __restrict__ xrow, int64_t nrow, const float* __restrict__ xv, int ntiles_total,
    int tiles_per_split, const __grid_constant__ FastParams fp, TileEpilogue ep, int* err) {
  // Warps 0-3 form K blocks (one row per thread and row tile); warp 4 is the
  // producer: it streams column tiles (TMA), issues the MMAs once a K block is
  // complete, and refills ring slots when both the x' reads and the MMAs that
  // read the slot's V blocks are done. Hand-offs use mbarriers only.
  constexpr int TILE = tc_tile_floats(DP);
  extern __shared__ __align__(1024) float smem[];
  float* ring_buf = smem;
  float* abuf = smem + kTcStages * TILE;
  __shared__ __align__(8) uint64_t full_bar[kTcStages];   // TMA landed
  __shared__ __align__(8) uint64_t xdone_bar[kTcStages];  // 128 threads done with x'
  __shared__ __align__(8) uint64_t afull_bar[2];          // 128 threads wrote a K block
  __shared__ __align__(8) uint64_t mma_bar[2];            // tensor core consumed a K block
  __shared__ uint32_t tslot;
  __shared__ int abort_flag;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  constexpr int kChunks = 128 / kTcChunk;
  constexpr int kWin = kTcWinTiles * kChunks;  // chunks per accumulation window
  constexpr uint32_t kSumCol = 2 * 16 * kTcRows;

  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&xdone_bar[s], kTcThreads);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&afull_bar[s], kTcThreads);
      mbar_init(&mma_bar[s], 1);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4) tmem_alloc(&tslot, kTcTmemCols);  // two CTAs per SM share the 512 columns
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  const uint32_t tile_bytes = TILE * sizeof(float);

  if (warp == 4) {
    if (lane == 0) {
      int issued = 0;
      for (int s = 0; s < kTcStages && s < ntiles; ++s) {
        mbar_arrive_expect_tx(&full_bar[s], tile_bytes);
        bulk_copy_g2s(ring_buf + s * TILE, xv + (int64_t)(t0 + s) * TILE, tile_bytes, &full_bar[s]);
        ++issued;
      }
      const uint32_t idesc = make_idesc_tf32(128, 16);
      int g = 0;
      bool ok = true;
      for (int kt = 0; kt < ntiles && ok; ++kt) {
        const int slot = kt % kTcStages;
        const float* tile = ring_buf + slot * TILE;
        const float* bhi = tile + 128 * DP;
        const float* blo = bhi + 16 * 128;
        ok = mbar_wait_bounded(&full_bar[slot], (kt / kTcStages) & 1);
        for (int q = 0; q < kChunks && ok; ++q, ++g) {
          const int st = g & 1;
          ok = mbar_wait_bounded(&afull_bar[st], (g >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          const float* ablk = abuf + st * (kTcAStageBytes / 4);
#pragma unroll
          for (int r = 0; r < kTcRows; ++r) {
            const float* ahi = ablk + r * 2 * (128 * kTcChunk);
            const float* alo = ahi + 128 * kTcChunk;
            const uint32_t d = tmem + ((g / kWin) & 1) * (16 * kTcRows) + r * 16;
            static_assert(kTcChunk == 8, "one MMA k-step per K block");
            const uint64_t dah = make_smem_desc(ahi, 2048, 128);
            const uint64_t dal = make_smem_desc(alo, 2048, 128);
            const uint64_t dbh = make_smem_desc(bhi + q * 128, 256, 128);
            const uint64_t dbl = make_smem_desc(blo + q * 128, 256, 128);
            mma_tf32(d, dah, dbh, idesc, g % kWin > 0 ? 1u : 0u);
            mma_tf32(d, dah, dbl, idesc, 1u);
            mma_tf32(d, dal, dbh, idesc, 1u);
          }
          mma_commit(&mma_bar[st]);
        }
        if (ok && kt + kTcStages < ntiles) {
          ok = mbar_wait_bounded(&xdone_bar[slot], (kt / kTcStages) & 1) &&
               mbar_wait_bounded(&mma_bar[(g - 1) & 1], ((g - 1) >> 1) & 1);
          if (ok) {
            mbar_arrive_expect_tx(&full_bar[slot], tile_bytes);
            bulk_copy_g2s(ring_buf + slot * TILE, xv + (int64_t)(t0 + kt + kTcStages) * TILE,
                          tile_bytes, &full_bar[slot]);
            ++issued;
          }
        }
      }
      if (!ok) {
        atomicExch(err, DEV_WAIT_TIMEOUT);
        atomicExch(&abort_flag, 1);
      }
      drain_ring<kTcStages>(full_bar, issued);
    }
  } else {
    const int64_t row0 = (int64_t)blockIdx.x * (128 * kTcRows) + tid;
    // Row pairs (2p, 2p+1) share float2 registers: the distance runs on the
    // packed FADD2 / FFMA2 instructions against duplicated -x'_j.
    static_assert(kTcRows % 2 == 0, "row pairs");
    float2 xi[kTcRows / 2][DP];
#pragma unroll
    for (int rp = 0; rp < kTcRows / 2; ++rp) {
      const int64_t i0 = row0 + (int64_t)(2 * rp) * 128, i1 = i0 + 128;
#pragma unroll
      for (int k = 0; k < DP; ++k)
        xi[rp][k] = make_float2(i0 < nrow ? xrow[i0 * DP + k] : 0.f, i1 < nrow ? xrow[i1 * DP + k] : 0.f);
    }
    const int a_row_off = (tid / 8) * 32 + (tid % 8) * 4;
    const uint32_t lane_sel = (uint32_t)(warp * 32) << 16;
    // sum (+)= accumulator set at `set_col`, for this thread's rows of every row tile.
    auto fold_set = [&](uint32_t set_col, bool add) {
#pragma unroll 1
      for (int r = 0; r < kTcRows; ++r) {
        float a[16];
        tmem_ld16(set_col + lane_sel + r * 16, a);
        if (add) {
          float s[16];
          tmem_ld16(tmem + lane_sel + kSumCol + r * 16, s);
#pragma unroll
          for (int c = 0; c < 16; ++c) a[c] += s[c];
        }
        uint32_t b[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) b[c] = __float_as_uint(a[c]);
        tmem_st16(tmem + lane_sel + kSumCol + r * 16, b);
      }
      tmem_wait_st();
    };
    int g = 0;
    bool ok = true;
    for (int kt = 0; kt < ntiles && ok; ++kt) {
      const int slot = kt % kTcStages;
      ok = mbar_wait_bounded(&full_bar[slot], (kt / kTcStages) & 1);
      if (!ok) break;
      const float* xs = ring_buf + slot * TILE;
      for (int q = 0; q < kChunks; ++q, ++g) {
        const int st = g & 1;
        if (g >= 2) {
          ok = mbar_wait_bounded(&mma_bar[st], ((g - 2) >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
        }
        if (g % kWin == 1 && g > kWin) {
          // The MMAs of chunk g - 2, the last of window w - 1, are complete
          // (and with them all earlier ones): fold that window's set into the
          // sum. Window w + 1 reuses the set only after this chunk's arrival.
          const int w1 = g / kWin - 1;
          fold_set(tmem + (uint32_t)(w1 & 1) * (16 * kTcRows), w1 > 0);
        }
        float* ablk = abuf + st * (kTcAStageBytes / 4);
#pragma unroll
        for (int j4 = 0; j4 < kTcChunk; j4 += 4) {
          float kv[kTcRows][4];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float4* xr = reinterpret_cast<const float4*>(xs + (q * kTcChunk + j4 + jj) * DP);
            float2 xn[DP];
#pragma unroll
            for (int k = 0; k < DP; k += 4) {
              const float4 v = xr[k / 4];
              xn[k] = make_float2(v.x, v.x);
              xn[k + 1] = make_float2(v.y, v.y);
              xn[k + 2] = make_float2(v.z, v.z);
              xn[k + 3] = make_float2(v.w, v.w);
            }
#pragma unroll
            for (int rp = 0; rp < kTcRows / 2; ++rp) {
              float2 u0 = make_float2(0.f, 0.f), u1 = make_float2(0.f, 0.f);
#pragma unroll
              for (int k = 0; k < DP; k += 2) {
                const float2 d0 = __fadd2_rn(xi[rp][k], xn[k]);
                u0 = __ffma2_rn(d0, d0, u0);
                const float2 d1 = __fadd2_rn(xi[rp][k + 1], xn[k + 1]);
                u1 = __ffma2_rn(d1, d1, u1);
              }
              const float2 u = __fadd2_rn(u0, u1);
              kv[2 * rp][jj] = FastEval<LEAF>::value(u.x, fp);
              kv[2 * rp + 1][jj] = FastEval<LEAF>::value(u.y, fp);
            }
          }
#pragma unroll
          for (int r = 0; r < kTcRows; ++r) {
            float4 hi, lo;
            hi.x = tf32_hi(kv[r][0]); lo.x = kv[r][0] - hi.x;
            hi.y = tf32_hi(kv[r][1]); lo.y = kv[r][1] - hi.y;
            hi.z = tf32_hi(kv[r][2]); lo.z = kv[r][2] - hi.z;
            hi.w = tf32_hi(kv[r][3]); lo.w = kv[r][3] - hi.w;
            float* base = ablk + r * 2 * (128 * kTcChunk) + (j4 / 4) * 512 + a_row_off;
            *reinterpret_cast<float4*>(base) = hi;
            *reinterpret_cast<float4*>(base + 128 * kTcChunk) = lo;
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&afull_bar[st]);
      }
      if (!ok) break;
      mbar_arrive(&xdone_bar[slot]);
    }
    // Epilogue: the last commit covers every MMA of this CTA.
    if (ok && g > 0) ok = mbar_wait_bounded(&mma_bar[(g - 1) & 1], ((g - 1) >> 1) & 1);
    tc_fence_after();
    if (!ok) {
      atomicExch(err, DEV_WAIT_TIMEOUT);
    } else {
      const bool partial = gridDim.y > 1;
      // Windows folded during the loop: 0 .. folded - 1 (window w - 1 is
      // folded at chunk w * kWin + 1). The rest (one or two) are added here.
      const int nwin = (g + kWin - 1) / kWin;
      int folded = 0;
      for (int w = 1; w < nwin; ++w)
        if (w * kWin + 1 < g) folded = w;
#pragma unroll 1
      for (int r = 0; r < kTcRows; ++r) {
        float acc[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[c] = 0.f;
        if (folded > 0) tmem_ld16(tmem + lane_sel + kSumCol + r * 16, acc);
        for (int w = folded; w < nwin; ++w) {
          float a[16];
          tmem_ld16(tmem + lane_sel + (uint32_t)(w & 1) * (16 * kTcRows) + r * 16, a);
#pragma unroll
          for (int c = 0; c < 16; ++c) acc[c] += a[c];
        }
        const int64_t i = row0 + (int64_t)r * 128;
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
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) tmem_dealloc(tmem, kTcTmemCols);
}

}  // namespace gpb
