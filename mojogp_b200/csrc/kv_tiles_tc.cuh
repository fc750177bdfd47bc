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
constexpr int kTcChunk = 16;       // columns per K block (2 MMA k-steps)
constexpr int kTcRows = 2;         // row tiles (M = 128 each) per CTA
constexpr int kTcThreads = 128;
constexpr int kTcAStageBytes = kTcRows * 2 * 128 * kTcChunk * 4;  // hi + lo, both row tiles

// Packed tile: [x' : 128 x DP][V hi : 16 k-steps x 128][V lo : 16 k-steps x 128] floats.
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
__global__ void __launch_bounds__(kTcThreads) kv_tile_tc_kernel(
    const float* __restrict__ xrow, int64_t nrow, const float* __restrict__ xv, int ntiles_total,
    int tiles_per_split, const __grid_constant__ FastParams fp, TileEpilogue ep, int* err) {
  constexpr int TILE = tc_tile_floats(DP);
  extern __shared__ __align__(1024) float smem[];
  float* ring_buf = smem;                                         // kTcStages x TILE
  float* abuf = smem + kTcStages * TILE;                           // 2 stages x kTcAStageBytes
  __shared__ __align__(8) uint64_t ring_bars[kTcStages];
  __shared__ __align__(8) uint64_t mma_bars[2];
  __shared__ uint32_t tslot;

  const int tid = threadIdx.x;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);

  if (tid == 0) {
    mbar_init(&mma_bars[0], 1);
    mbar_init(&mma_bars[1], 1);
  }
  if (tid < 32) tmem_alloc(&tslot, 32);  // 2 row tiles x 16 fp32 columns
  TileRingT<kTcStages> ring{ring_buf, ring_bars, xv, t0, ntiles, (uint32_t)TILE};
  ring.start();  // inits ring barriers, fences, __syncthreads, issues first copies
  tc_fence_after();
  const uint32_t tmem = tslot;

  const int64_t row0 = (int64_t)blockIdx.x * (128 * kTcRows) + tid;
  float xi[kTcRows][DP];
#pragma unroll
  for (int r = 0; r < kTcRows; ++r) {
    const int64_t i = row0 + (int64_t)r * 128;
#pragma unroll
    for (int k = 0; k < DP; ++k) xi[r][k] = (i < nrow) ? xrow[i * DP + k] : 0.f;
  }
  const uint32_t idesc = make_idesc_tf32(128, 16);
  // This thread's row inside a K block: core-matrix row (tid/8, tid%8).
  const int a_row_off = (tid / 8) * 32 + (tid % 8) * 4;  // floats
  bool failed = false;
  int g = 0;  // global chunk counter
  for (int kt = 0; kt < ntiles && !failed; ++kt) {
    const float* tile = ring.acquire(kt);
    if (tile == nullptr) {
      failed = true;
      break;
    }
    const float* xs = tile;
    const float* bhi = tile + 128 * DP;
    const float* blo = bhi + 16 * 128;
    for (int q = 0; q < 128 / kTcChunk; ++q, ++g) {
      const int st = g & 1;
      float* ablk = abuf + st * (kTcAStageBytes / 4);
      if (g >= 2) {
        const bool ok = mbar_wait_bounded(&mma_bars[st], ((g - 2) >> 1) & 1);
        if (!__syncthreads_and(ok)) {
          failed = true;
          break;
        }
        tc_fence_after();
      }
#pragma unroll
      for (int j4 = 0; j4 < kTcChunk; j4 += 4) {
        float kv[kTcRows][4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float4* xr = reinterpret_cast<const float4*>(xs + (q * kTcChunk + j4 + jj) * DP);
          float xj[DP];
#pragma unroll
          for (int k = 0; k < DP; k += 4) {
            const float4 v = xr[k / 4];
            xj[k] = v.x; xj[k + 1] = v.y; xj[k + 2] = v.z; xj[k + 3] = v.w;
          }
#pragma unroll
          for (int r = 0; r < kTcRows; ++r) {
            float u0 = 0.f, u1 = 0.f;
#pragma unroll
            for (int k = 0; k < DP; k += 2) {
              const float d0 = xi[r][k] - xj[k];
              u0 = fmaf(d0, d0, u0);
              const float d1 = xi[r][k + 1] - xj[k + 1];
              u1 = fmaf(d1, d1, u1);
            }
            kv[r][jj] = FastEval<LEAF>::value(u0 + u1, fp);
          }
        }
#pragma unroll
        for (int r = 0; r < kTcRows; ++r) {
          float4 hi, lo;
          hi.x = tf32_hi(kv[r][0]); lo.x = kv[r][0] - hi.x;
          hi.y = tf32_hi(kv[r][1]); lo.y = kv[r][1] - hi.y;
          hi.z = tf32_hi(kv[r][2]); lo.z = kv[r][2] - hi.z;
          hi.w = tf32_hi(kv[r][3]); lo.w = kv[r][3] - hi.w;
          // K block (row tile r): hi at r*2*2048 floats, lo right after; k-group j4/4.
          float* base = ablk + r * 2 * (128 * kTcChunk) + (j4 / 4) * 512 + a_row_off;
          *reinterpret_cast<float4*>(base) = hi;
          *reinterpret_cast<float4*>(base + 128 * kTcChunk) = lo;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int r = 0; r < kTcRows; ++r) {
          const float* ahi = ablk + r * 2 * (128 * kTcChunk);
          const float* alo = ahi + 128 * kTcChunk;
          const uint32_t d = tmem + r * 16;
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const int kstep = q * 2 + ks;  // 8-column step inside the 128-column tile
            const uint64_t dah = make_smem_desc(ahi + ks * 1024, 2048, 128);
            const uint64_t dal = make_smem_desc(alo + ks * 1024, 2048, 128);
            const uint64_t dbh = make_smem_desc(bhi + kstep * 128, 256, 128);
            const uint64_t dbl = make_smem_desc(blo + kstep * 128, 256, 128);
            const uint32_t acc0 = (g > 0 || ks > 0) ? 1u : 0u;
            mma_tf32(d, dah, dbh, idesc, acc0);
            mma_tf32(d, dah, dbl, idesc, 1u);
            mma_tf32(d, dal, dbh, idesc, 1u);
          }
        }
        mma_commit(&mma_bars[st]);
      }
    }
    if (failed) break;
    // The ring slot may be refilled once the tensor core has read its V
    // blocks: wait for the commit of this tile's last chunk (thread 0 only,
    // before it issues the next copy inside release()).
    if (tid == 0 && kt + kTcStages < ntiles) {
      const int gl = g - 1;
      if (!mbar_wait_bounded(&mma_bars[gl & 1], (gl >> 1) & 1)) atomicExch(err, DEV_WAIT_TIMEOUT);
    }
    ring.release(kt);
  }

  // Epilogue: wait for the last commit, read the accumulators from TMEM.
  bool have = !failed && g > 0;
  if (have) {
    const int gl = g - 1;
    const bool ok = mbar_wait_bounded(&mma_bars[gl & 1], (gl >> 1) & 1);
    have = __syncthreads_and(ok);
  } else {
    __syncthreads();
  }
  tc_fence_after();
  if (failed || (g > 0 && !have)) {
    if (tid == 0) atomicExch(err, DEV_WAIT_TIMEOUT);
  } else {
    const bool partial = gridDim.y > 1;
#pragma unroll
    for (int r = 0; r < kTcRows; ++r) {
      float acc[16];
      if (g > 0) {
        tmem_ld16(tmem + r * 16 + ((uint32_t)((tid / 32) * 32) << 16), acc);
      } else {
#pragma unroll
        for (int c = 0; c < 16; ++c) acc[c] = 0.f;
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
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tmem, 32);
}

}  // namespace gpb
