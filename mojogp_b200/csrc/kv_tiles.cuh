// Tiled matrix-free kernel matvec  out[c][i] = sum_j k(x_i, x_j) v[c][j].
//
// B200 design (replaces the reference's one-thread-per-row shared-memory loop,
// mojogp/codegen_engine/emit/gpu_kernel.py:151-379):
//   * the column side (x_j and the v_j block) is pre-packed into contiguous
//     rows of W floats, so one tile of JT columns is a single contiguous
//     range that the TMA engine moves with a 1-D bulk copy into shared memory
//     (cp.async.bulk + mbarrier, STAGES-deep ring, no multicast);
//   * each thread keeps R rows of x_i and an R x T accumulator tile in
//     registers; every x_j / v_j is a broadcast shared-memory read reused by
//     the R rows;
//   * the pair kernel value is formed in registers (FFMA distance + one MUFU
//     exponential for RBF) and never materialised;
//   * the j range can be split over gridDim.y blocks that write partial
//     sums, reduced in a fixed order by kv_reduce (deterministic), so small n
//     still fills all 148 SMs.
#pragma once

#include "gpb_common.cuh"
#include "kernel_program.cuh"

namespace gpb {

constexpr int kJT = 128;     // columns per TMA tile
constexpr int kStages = 3;   // TMA ring depth

// Packed column row width (floats) for DP padded dims and T rhs columns.
__host__ __device__ constexpr int packed_width(int DP, int T) { return ((DP + T) + 3) / 4 * 4; }


// TMA ring over a contiguous range of packed column tiles [t0, t0+ntiles).
// Thread 0 issues 1-D bulk copies; all threads wait on the stage mbarrier
// with a bounded wait, and a block-wide vote turns a timeout into a clean exit.
template <int S>
struct TileRingT {
  float* smem;
  uint64_t* bars;
  const float* src;
  int t0, ntiles;
  uint32_t tile_floats;

  __device__ __forceinline__ void start() {
    if (threadIdx.x == 0) {
      for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int s = 0; s < S && s < ntiles; ++s) issue(s, s);
    }
  }
  __device__ __forceinline__ void issue(int stage, int kt) {
    const uint32_t bytes = tile_floats * sizeof(float);
    mbar_arrive_expect_tx(&bars[stage], bytes);
    bulk_copy_g2s(smem + (size_t)stage * tile_floats, src + (int64_t)(t0 + kt) * tile_floats, bytes,
                  &bars[stage]);
  }
  // Returns the stage buffer, or nullptr (for every thread) on timeout.
  __device__ __forceinline__ const float* acquire(int kt) {
    const int st = kt % S;
    const bool ok = mbar_wait_bounded(&bars[st], (kt / S) & 1);
    if (!__syncthreads_and(ok)) return nullptr;
    return smem + (size_t)st * tile_floats;
  }
  __device__ __forceinline__ void release(int kt) {
    __syncthreads();
    if (threadIdx.x == 0 && kt + S < ntiles) issue(kt % S, kt + S);
  }
  __device__ __forceinline__ void fail(int* err) {
    if (threadIdx.x == 0) {
      atomicExch(err, DEV_WAIT_TIMEOUT);
      for (int s = 0; s < S; ++s) (void)mbar_wait_bounded(&bars[s], 0, 100000000ull);
    }
  }
};
using TileRing = TileRingT<kStages>;

// ---------------------------------------------------------------- evaluators
// Fast single-leaf evaluators work on prescaled inputs x' so that the inner
// distance is u = |x'_i - x'_j|^2 and the value (without the outputscale) is
// a function of u alone. The host sets the prescale per leaf:
//   RBF:   x' = x * sqrt(log2(e)/2) / l         k = ex2(-u)
//   M12:   x' = x / l                            r = sqrt(max(u+1e-20,1e-20))
//   M32:   x' = x * sqrt(3) / l                  k = (1+r)  e^{-r} (clamped)
//   M52:   x' = x * sqrt(5) / l                  k = (1+r+u/3) e^{-r} (clamped)
//   RQ:    x' = x / l                            k = (1 + u/(2a))^{-a}
struct FastParams {
  float a0;  // RQ: alpha; M12: clamp flag (1 = clamp at -20)
  float a1;  // RQ: 1/(2 alpha); Matern: eps*prescale^2 added under the sqrt
};

template <int LEAF>
struct FastEval {
  using Params = FastParams;
  static constexpr bool kGeneric = false;
  static constexpr int kLeaf = LEAF;
  __device__ __forceinline__ static float value(float u, const FastParams& fp) {
    if constexpr (LEAF == GPB_KERNEL_RBF) {
      return ex2_approx(-u);
    } else if constexpr (LEAF == GPB_KERNEL_MATERN12) {
      const float uu = fmaxf(u + fp.a1, fp.a1);
      const float r = uu * rsqrtf(uu);
      const float a = fp.a0 != 0.f ? fmaxf(-r, -20.f) : -r;
      return exp_fast(a);
    } else if constexpr (LEAF == GPB_KERNEL_MATERN32) {
      const float uu = fmaxf(u + fp.a1, fp.a1);
      const float r = uu * rsqrtf(uu);
      return (1.f + r) * exp_fast(fmaxf(-r, -20.f));
    } else if constexpr (LEAF == GPB_KERNEL_MATERN52) {
      const float uu = fmaxf(u + fp.a1, fp.a1);
      const float r = uu * rsqrtf(uu);
      return (1.f + r + u * (1.f / 3.f)) * exp_fast(fmaxf(-r, -20.f));
    } else {  // RQ
      return ex2_approx(-fp.a0 * lg2_approx(fmaf(u, fp.a1, 1.f)));
    }
  }
};

struct GenericEval {
  using Params = DevKernel;
  static constexpr bool kGeneric = true;
};

struct TileEpilogue {
  float* out;            // [T][out_ld] (or partials [S][T][out_ld])
  int64_t out_ld;
  float scale;           // multiplies the accumulated sum (outputscale)
  const float* noise_v;  // if non-null: out += noise * noise_v[c*noise_ld + i]
  int64_t noise_ld;
  float noise;           // scalar noise (used when noise_vec is null)
  const float* noise_vec;
  int tcols;             // valid rhs columns (<= T); padded columns are not stored
};

// --------------------------------------------------------------- tile kernel
template <int DP, int T, int R, int BLK, class Ev>
__global__ void __launch_bounds__(BLK) kv_tile_kernel(const float* __restrict__ xrow,
                                                      int64_t nrow,
                                                      const float* __restrict__ xv,
                                                      int ntiles_total, int tiles_per_split,
                                                      const __grid_constant__ typename Ev::Params ev,
                                                      TileEpilogue ep, int* err) {
  constexpr int W = packed_width(DP, T);
  extern __shared__ __align__(128) float smem[];
  __shared__ __align__(8) uint64_t bars[kStages];

  const int tid = threadIdx.x;
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  TileRing ring{smem, bars, xv, t0, ntiles, (uint32_t)(kJT * W)};
  float* tot = smem + kStages * kJT * W;  // [R * T][BLK] per-tile fold
  ring.start();

  // Row registers.
  const int64_t row0 = (int64_t)blockIdx.x * (BLK * R) + tid;
  float xi[R][DP];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t i = row0 + (int64_t)r * BLK;
#pragma unroll
    for (int k = 0; k < DP; ++k) xi[r][k] = (i < nrow) ? xrow[i * DP + k] : 0.f;
  }
  float acc[R][T];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int c = 0; c < T; ++c) acc[r][c] = 0.f;

  for (int kt = 0; kt < ntiles; ++kt) {
    const float* buf = ring.acquire(kt);
    if (buf == nullptr) {
      ring.fail(err);
      return;
    }
#pragma unroll 2
    for (int j = 0; j < kJT; ++j) {
      const float* rowp = buf + j * W;
      float xj[DP];
      if constexpr (DP % 4 == 0) {
#pragma unroll
        for (int k = 0; k < DP; k += 4) {
          const float4 q = *reinterpret_cast<const float4*>(rowp + k);
          xj[k] = q.x; xj[k + 1] = q.y; xj[k + 2] = q.z; xj[k + 3] = q.w;
        }
      } else {
#pragma unroll
        for (int k = 0; k < DP; ++k) xj[k] = rowp[k];
      }
      float kv[R];
      if constexpr (!Ev::kGeneric) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float u0 = 0.f, u1 = 0.f;
#pragma unroll
          for (int k = 0; k < DP; k += 2) {
            const float d0 = xi[r][k] - xj[k];
            u0 = fmaf(d0, d0, u0);
            if (k + 1 < DP) {
              const float d1 = xi[r][k + 1] - xj[k + 1];
              u1 = fmaf(d1, d1, u1);
            }
          }
          kv[r] = Ev::value(u0 + u1, ev);
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) kv[r] = tree_eval<false>(ev, xi[r], xj, nullptr);
      }
      float vj[T];
      if constexpr (DP % 4 == 0 && T % 4 == 0) {
#pragma unroll
        for (int c = 0; c < T; c += 4) {
          const float4 q = *reinterpret_cast<const float4*>(rowp + DP + c);
          vj[c] = q.x; vj[c + 1] = q.y; vj[c + 2] = q.z; vj[c + 3] = q.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < T; ++c) vj[c] = rowp[DP + c];
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int c = 0; c < T; ++c) acc[r][c] = fmaf(kv[r], vj[c], acc[r][c]);
    }
    ring.release(kt);
    // Fold this tile's sums into the running totals (shared memory, one slot
    // per thread, row and column): no fp32 sum runs over more than one tile,
    // where a flat sum over 1e6 columns drifts by up to ~u * sqrt(n).
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int c = 0; c < T; ++c) {
        float* slot = tot + (r * T + c) * BLK + tid;
        *slot = (kt == 0 ? 0.f : *slot) + acc[r][c];
        acc[r][c] = 0.f;
      }
  }
  if (ntiles > 0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int c = 0; c < T; ++c) acc[r][c] = tot[(r * T + c) * BLK + tid];
  }

  const bool partial = gridDim.y > 1;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t i = row0 + (int64_t)r * BLK;
    if (i >= nrow) continue;
#pragma unroll
    for (int c = 0; c < T; ++c) {
      if (c >= ep.tcols) continue;
      if (partial) {
        ep.out[((int64_t)split * T + c) * ep.out_ld + i] = acc[r][c];
      } else {
        float o = ep.scale * acc[r][c];
        if (ep.noise_v) {
          const float nz = ep.noise_vec ? ep.noise_vec[i] : ep.noise;
          o = fmaf(nz, ep.noise_v[c * ep.noise_ld + i], o);
        }
        ep.out[c * ep.out_ld + i] = o;
      }
    }
  }
}

}  // namespace gpb
