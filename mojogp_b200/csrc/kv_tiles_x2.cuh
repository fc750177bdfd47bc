// Paired-row variant of the tiled K·V kernel for the fast single-leaf
// evaluators, written with the sm_100 packed FP32 instructions
// (FADD2 / FFMA2 through __fadd2_rn / __ffma2_rn): two rows of x_i share each
// register pair, the column side is packed pre-duplicated and pre-negated
// ([-x'_0, -x'_0, -x'_1, -x'_1, ..., v_0, v_0, ...]) so one 128-bit shared
// load yields two ready operand pairs. Per kernel entry this issues about half
// the FP32 instructions of the scalar kernel, freeing issue slots for the MUFU
// exponential and the shared-memory loads.
#pragma once

#include "kv_tiles.cuh"

namespace gpb {

__host__ __device__ constexpr int packed_width_x2(int DP, int T) { return 2 * (DP + T); }
constexpr int kStagesX2 = 2;

template <int DP, int T, int R, int BLK, int LEAF>
__global__ void __launch_bounds__(BLK) kv_tile_x2_kernel(const float* __restrict__ xrow,
                                                         int64_t nrow, const float* __restrict__ xv,
                                                         int ntiles_total, int tiles_per_split,
                                                         const __grid_constant__ FastParams fp,
                                                         TileEpilogue ep, int* err) {
  static_assert(R % 2 == 0 && DP % 2 == 0, "paired rows");
  constexpr int W = packed_width_x2(DP, T);
  constexpr int RP = R / 2;
  extern __shared__ __align__(128) float smem[];
  __shared__ __align__(8) uint64_t bars[kStagesX2];
  const int tid = threadIdx.x;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  TileRingT<kStagesX2> ring{smem, bars, xv, t0, ntiles, (uint32_t)(kJT * W)};
  float2* tot = reinterpret_cast<float2*>(smem + kStagesX2 * kJT * W);  // [RP * T][BLK]
  ring.start();

  const int64_t row0 = (int64_t)blockIdx.x * (BLK * R) + tid;
  float2 xi[RP][DP];
#pragma unroll
  for (int q = 0; q < RP; ++q) {
    const int64_t i0 = row0 + (int64_t)(2 * q) * BLK, i1 = i0 + BLK;
#pragma unroll
    for (int k = 0; k < DP; ++k)
      xi[q][k] = make_float2(i0 < nrow ? xrow[i0 * DP + k] : 0.f, i1 < nrow ? xrow[i1 * DP + k] : 0.f);
  }
  float2 acc[RP][T];
#pragma unroll
  for (int q = 0; q < RP; ++q)
#pragma unroll
    for (int c = 0; c < T; ++c) acc[q][c] = make_float2(0.f, 0.f);

  for (int kt = 0; kt < ntiles; ++kt) {
    const float* buf = ring.acquire(kt);
    if (buf == nullptr) {
      ring.fail(err);
      return;
    }
#pragma unroll 2
    for (int j = 0; j < kJT; ++j) {
      const float4* rowp = reinterpret_cast<const float4*>(buf + j * W);
      float2 xn[DP];
#pragma unroll
      for (int k = 0; k < DP; k += 2) {
        const float4 v = rowp[k / 2];
        xn[k] = make_float2(v.x, v.y);
        xn[k + 1] = make_float2(v.z, v.w);
      }
      float2 kv[RP];
#pragma unroll
      for (int q = 0; q < RP; ++q) {
        float2 u0 = make_float2(0.f, 0.f), u1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < DP; k += 2) {
          const float2 d0 = __fadd2_rn(xi[q][k], xn[k]);
          u0 = __ffma2_rn(d0, d0, u0);
          const float2 d1 = __fadd2_rn(xi[q][k + 1], xn[k + 1]);
          u1 = __ffma2_rn(d1, d1, u1);
        }
        const float2 u = __fadd2_rn(u0, u1);
        kv[q] = make_float2(FastEval<LEAF>::value(u.x, fp), FastEval<LEAF>::value(u.y, fp));
      }
      const float4* vp = rowp + DP / 2;
#pragma unroll
      for (int c = 0; c < T; c += 2) {
        const float4 v = vp[c / 2];
        const float2 va = make_float2(v.x, v.y), vb = make_float2(v.z, v.w);
#pragma unroll
        for (int q = 0; q < RP; ++q) {
          acc[q][c] = __ffma2_rn(kv[q], va, acc[q][c]);
          acc[q][c + 1] = __ffma2_rn(kv[q], vb, acc[q][c + 1]);
        }
      }
    }
    ring.release(kt);
    // Fold this tile's sums into the running totals in shared memory (see
    // kv_tile_kernel).
#pragma unroll
    for (int q = 0; q < RP; ++q)
#pragma unroll
      for (int c = 0; c < T; ++c) {
        float2* slot = tot + (q * T + c) * BLK + tid;
        const float2 prev = kt == 0 ? make_float2(0.f, 0.f) : *slot;
        *slot = __fadd2_rn(prev, acc[q][c]);
        acc[q][c] = make_float2(0.f, 0.f);
      }
  }
  if (ntiles > 0) {
#pragma unroll
    for (int q = 0; q < RP; ++q)
#pragma unroll
      for (int c = 0; c < T; ++c) acc[q][c] = tot[(q * T + c) * BLK + tid];
  }

  const bool partial = gridDim.y > 1;
#pragma unroll
  for (int q = 0; q < RP; ++q) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t i = row0 + (int64_t)(2 * q + h) * BLK;
      if (i >= nrow) continue;
#pragma unroll
      for (int c = 0; c < T; ++c) {
        if (c >= ep.tcols) continue;
        const float a = h ? acc[q][c].y : acc[q][c].x;
        if (partial) {
          ep.out[((int64_t)split * T + c) * ep.out_ld + i] = a;
        } else {
          float o = ep.scale * a;
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

}  // namespace gpb
