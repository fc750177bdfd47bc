// Device kernels of the engine: CG vector updates, deterministic column dot
// products, the hash Gaussian generator, column packing, and the Woodbury
// pieces of the pivoted-Cholesky preconditioner. All vectors are column-major
// blocks [t][ld] over the rank's local rows.
#include "engine.cuh"
#include "train.cuh"
#include "matvec.cuh"

namespace gpb {

// ------------------------------------------------------------------ basics
__global__ void fill_kernel(float* p, int64_t count, float v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) p[i] = v;
}
int k_fill(float* p, int64_t count, float v, cudaStream_t st) {
  if (count <= 0) return GPB_OK;
  fill_kernel<<<(unsigned)ceil_div(count, 256), 256, 0, st>>>(p, count, v);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}
int k_copy(float* dst, const float* src, int64_t count, cudaStream_t st) {
  if (count <= 0) return GPB_OK;
  GPB_CHECK_CUDA(cudaMemcpyAsync(dst, src, count * sizeof(float), cudaMemcpyDeviceToDevice, st));
  return GPB_OK;
}
__global__ void sub_kernel(float* r, const float* a, int64_t count) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) r[i] -= a[i];
}
int k_sub(float* r, const float* a, int64_t count, cudaStream_t st) {
  if (count <= 0) return GPB_OK;
  sub_kernel<<<(unsigned)ceil_div(count, 256), 256, 0, st>>>(r, a, count);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

__global__ void sub_scalar_kernel(float* v, int64_t count, float s) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) v[i] -= s;
}
int k_sub_scalar(float* v, int64_t count, float s, cudaStream_t st) {
  if (count <= 0) return GPB_OK;
  sub_scalar_kernel<<<(unsigned)ceil_div(count, 256), 256, 0, st>>>(v, count, s);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// Counter-hash Gaussian of pivoted_cholesky.mojo:51-86 (kernel_gpu_gaussian):
// two 64-bit multiply/xorshift hashes of the global index give u1 in (0,1]
// and u2 in [0,1), then Box-Muller with pi written as 3.14159265.
__device__ __forceinline__ float hash_gaussian(uint64_t idx, uint64_t seed) {
  uint64_t s1 = (idx + 1ull) * 6364136223846793005ull + seed;
  s1 ^= s1 >> 33;
  s1 *= 0xff51afd7ed558ccdull;
  s1 ^= s1 >> 33;
  uint64_t s2 = (idx + 1ull) * 1442695040888963407ull + seed + 0xBEEFull;
  s2 ^= s2 >> 33;
  s2 *= 0xc4ceb9fe1a85ec53ull;
  s2 ^= s2 >> 33;
  const float u1 = ((float)(int64_t)(s1 & 0x7FFFFFull) + 1.0f) / (float)0x800000;
  const float u2 = (float)(int64_t)(s2 & 0xFFFFFFull) / (float)0x1000000;
  return sqrtf(-2.0f * logf(u1)) * cosf(2.0f * 3.14159265f * u2);
}

__global__ void gaussian_kernel(float* out, int t, int64_t nl, int64_t ld, int64_t n_global,
                                int64_t row0, uint64_t seed) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)t * nl) return;
  const int c = (int)(idx / nl);
  const int64_t i = idx - (int64_t)c * nl;
  out[c * ld + i] = hash_gaussian((uint64_t)(c * n_global + row0 + i), seed);
}
int k_gaussian(float* out, int t, int64_t nl, int64_t ld, int64_t n_global, int64_t row0,
               uint64_t seed, cudaStream_t st) {
  const int64_t total = (int64_t)t * nl;
  if (total <= 0) return GPB_OK;
  gaussian_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(out, t, nl, ld, n_global, row0,
                                                                  seed);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// Task-blocked probes over this rank's data rows: element (c, t, i) of a local
// [cols][T][nl] block takes the global index c*T*n + t*n + r0 + i, so every
// sharding draws the same numbers as one GPU.
__global__ void gaussian_tasks_kernel(float* out, int cols, int T, int64_t nl, int64_t n,
                                      int64_t r0, uint64_t seed) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_col = (int64_t)T * nl;
  if (idx >= (int64_t)cols * per_col) return;
  const int64_t c = idx / per_col;
  const int64_t rem = idx - c * per_col;
  const int64_t t = rem / nl;
  const int64_t i = rem - t * nl;
  out[idx] = hash_gaussian((uint64_t)((c * T + t) * n + r0 + i), seed);
}
int k_gaussian_tasks(float* out, int cols, int T, int64_t nl, int64_t n, int64_t r0, uint64_t seed,
                     cudaStream_t st) {
  const int64_t total = (int64_t)cols * T * nl;
  if (total <= 0) return GPB_OK;
  gaussian_tasks_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(out, cols, T, nl, n, r0,
                                                                       seed);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// v[c][i] *= scale[c] (or /= scale[c] when inverse).
__global__ void scale_cols_kernel(float* v, int64_t ld, int64_t nl, int t, const float* scale,
                                  int inverse) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)t * nl) return;
  const int c = (int)(idx / nl);
  const int64_t i = idx - (int64_t)c * nl;
  if (inverse)
    v[c * ld + i] /= scale[c];
  else
    v[c * ld + i] *= scale[c];
}
int k_scale_cols(float* v, int64_t ld, int64_t nl, int t, const float* scale, int inverse,
                 cudaStream_t st) {
  const int64_t total = (int64_t)t * nl;
  if (total <= 0) return GPB_OK;
  scale_cols_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(v, ld, nl, t, scale, inverse);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// ------------------------------------------------------------------ packing
// Local rows -> packed tile rows [x' (DP) | v (T)] with optional in-place
// search-direction update p = z + beta p (cg_solver.mojo:108-135 rules:
// beta == 0 or NaN, or p NaN -> p = z).
__global__ void pack_rows_kernel(const float* __restrict__ xs, int DP, float* __restrict__ v,
                                 int64_t v_ld, int c0, int tcols, int W, int64_t nl,
                                 int64_t nl_pad, float* __restrict__ dst,
                                 const float* __restrict__ upd_z, const float* __restrict__ upd_beta,
                                 bool dup) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nl_pad) return;
  float* row = dst + i * W;
  if (i >= nl) {
    for (int k = 0; k < W; ++k) row[k] = 0.f;
    return;
  }
  if (dup) {
    // paired-row layout: [-x'_k, -x'_k ..., v_c, v_c ...], W = 2 (DP + T)
    for (int k = 0; k < DP; ++k) row[2 * k] = row[2 * k + 1] = -xs[i * DP + k];
    const int T = W / 2 - DP;
    for (int c = 0; c < T; ++c) {
      float val = 0.f;
      if (c < tcols) {
        const int64_t off = (int64_t)(c0 + c) * v_ld + i;
        val = v[off];
        if (upd_beta) {
          const float b = upd_beta[c0 + c];
          const float zz = upd_z[off];
          val = (b == 0.f || b != b || val != val) ? zz : fmaf(b, val, zz);
          v[off] = val;
        }
      }
      row[2 * (DP + c)] = row[2 * (DP + c) + 1] = val;
    }
    return;
  }
  for (int k = 0; k < DP; ++k) row[k] = xs[i * DP + k];
  for (int c = 0; c < W - DP; ++c) {
    float val = 0.f;
    if (c < tcols) {
      const int64_t off = (int64_t)(c0 + c) * v_ld + i;
      val = v[off];
      if (upd_beta) {
        const float b = upd_beta[c0 + c];
        const float zz = upd_z[off];
        val = (b == 0.f || b != b || val != val) ? zz : fmaf(b, val, zz);
        v[off] = val;
      }
    }
    row[DP + c] = val;
  }
}
int k_pack(const float* xs, int DP, float* v, int64_t v_ld, int c0, int tcols, int T, int64_t nl,
           int64_t nl_pad, float* dst, const float* upd_z, const float* upd_beta,
           cudaStream_t st, int layout) {
  if (nl_pad <= 0) return GPB_OK;
  if (layout == KV_TC)
    return launch_pack_tc(xs, DP, v, v_ld, c0, tcols, nl, nl_pad, dst, upd_z, upd_beta, st);
  if (layout == KV_GRAM)
    return launch_pack_gram(xs, DP, v, v_ld, c0, tcols, nl, nl_pad, dst, upd_z, upd_beta, st);
  if (layout == KV_GRAM1)
    return launch_pack_gram1(xs, DP, T, v, v_ld, c0, tcols, nl, nl_pad, dst, upd_z, upd_beta, st);
  const bool dup = layout == KV_X2;
  pack_rows_kernel<<<(unsigned)ceil_div(nl_pad, 256), 256, 0, st>>>(
      xs, DP, v, v_ld, c0, tcols, dup ? 2 * (DP + T) : packed_width(DP, T), nl, nl_pad, dst, upd_z,
      upd_beta, dup);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// ------------------------------------------------------------ reductions
int Reducer::ensure(int max_blocks, int k) {
  // Grow geometrically: callers whose k rises by one per step (Lanczos
  // re-orthogonalisation against a growing basis) must not pay a device
  // free + allocation, and the synchronisation that comes with it, every step.
  const size_t need = (size_t)max_blocks * k * sizeof(double);
  if (partial.bytes < need) GPB_TRY(partial.ensure(std::max(need, 2 * partial.bytes)));
  const size_t need_s = (size_t)k * sizeof(double);
  if (sums.bytes < need_s) GPB_TRY(sums.ensure(std::max(need_s, 2 * sums.bytes)));
  if (counter.bytes < sizeof(unsigned) * 4) {
    GPB_TRY(counter.ensure(sizeof(unsigned) * 4));
    GPB_CHECK_CUDA(cudaMemset(counter.ptr, 0, sizeof(unsigned) * 4));
  }
  return GPB_OK;
}

__device__ __forceinline__ double block_sum_d(double v, double* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  double s = 0.0;
  if (threadIdx.x == 0)
    for (int q = 0; q < (int)(blockDim.x >> 5); ++q) s += sh[q];
  return s;  // valid in thread 0
}

// Last-block-done finalisation: partial[b*K + k] summed over blocks in order.
__device__ __forceinline__ void finalize_partials(const double* partial, int K, unsigned* counter,
                                                  double* sums) {
  __shared__ bool last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    double s = 0.0;
    for (unsigned b = 0; b < gridDim.x; ++b) s += ((volatile const double*)partial)[(size_t)b * K + k];
    sums[k] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = 0u;
}

struct DotArgs {
  const float* a[3];
  const float* b[3];
};

__global__ void __launch_bounds__(256) coldots_kernel(DotArgs args, int npairs, int64_t ld,
                                                      int64_t nl, int t, double* partial,
                                                      unsigned* counter, double* sums) {
  __shared__ double sh[8];
  const int K = npairs * t;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int q = 0; q < npairs; ++q) {
    for (int c = 0; c < t; ++c) {
      const float* a = args.a[q] + (int64_t)c * ld;
      const float* b = args.b[q] + (int64_t)c * ld;
      float acc = 0.f;
      for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nl; i += stride)
        acc = fmaf(a[i], b[i], acc);
      const double s = block_sum_d((double)acc, sh);
      if (threadIdx.x == 0) partial[(size_t)blockIdx.x * K + q * t + c] = s;
    }
  }
  finalize_partials(partial, K, counter, sums);
}

static int dot_blocks(int64_t nl) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(nl, 1024), 296));
}

int k_coldots(int npairs, const float* const* a, const float* const* b, int64_t ld, int64_t nl,
              int t, Reducer& red, cudaStream_t st) {
  GPB_REQUIRE(npairs >= 1 && npairs <= 3, GPB_ERR_INVALID, "coldots: npairs %d", npairs);
  const int G = dot_blocks(nl);
  GPB_TRY(red.ensure(G, npairs * t));
  DotArgs args{};
  for (int q = 0; q < npairs; ++q) {
    args.a[q] = a[q];
    args.b[q] = b[q];
  }
  coldots_kernel<<<G, 256, 0, st>>>(args, npairs, ld, nl, t, red.partial.d(),
                                    (unsigned*)red.counter.ptr, red.sums.d());
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// ------------------------------------------------------------ CG scalars
// alpha = rz / pAp; 0 if either is NaN or pAp < 1e-10 (cg_solver.mojo:181-208).
__global__ void cg_alpha_kernel(const float* rz_old, const double* pap, float* alpha,
                                float* hist, int t) {
  const int c = threadIdx.x;
  if (c >= t) return;
  const float rs = rz_old[c];
  const float pp = (float)pap[c];
  const float a = (rs != rs || pp != pp || pp < 1e-10f) ? 0.f : rs / pp;
  alpha[c] = a;
  if (hist) hist[c] = a;
}
int k_cg_alpha(const float* rz_old, const double* pap, float* alpha, float* hist, int t,
               cudaStream_t st) {
  cg_alpha_kernel<<<1, 32 * (int)ceil_div(t, 32), 0, st>>>(rz_old, pap, alpha, hist, t);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// beta = rz_new / (rz_old + 1e-20), >= 0, NaN -> 0; rz_old <- rz_new
// (cg_solver.mojo:211-250).
__global__ void cg_beta_kernel(float* rz_old, const double* rz_new, float* beta, float* hist,
                               int t) {
  const int c = threadIdx.x;
  if (c >= t) return;
  const float ro = rz_old[c];
  const float rn = (float)rz_new[c];
  float b = 0.f;
  if (ro == ro && rn == rn && ro >= 1e-20f) {
    b = rn / (ro + 1e-20f);
    if (b < 0.f || b != b) b = 0.f;
  }
  beta[c] = b;
  if (hist) hist[c] = b;
  rz_old[c] = (rn == rn) ? rn : 0.f;
}
int k_cg_beta(float* rz_old, const double* rz_new, float* beta, float* hist, int t,
              cudaStream_t st) {
  cg_beta_kernel<<<1, 32 * (int)ceil_div(t, 32), 0, st>>>(rz_old, rz_new, beta, hist, t);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

__global__ void set_rz_kernel(float* rz, const double* sums, int t) {
  const int c = threadIdx.x;
  if (c < t) rz[c] = (float)sums[c];
}
int k_set_rz(float* rz, const double* sums, int t, cudaStream_t st) {
  set_rz_kernel<<<1, 32 * (int)ceil_div(t, 32), 0, st>>>(rz, sums, t);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

__global__ void update_p_kernel(float* p, const float* z, const float* beta, int64_t nl,
                                int64_t ld, int t) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)t * nl) return;
  const int c = (int)(idx / nl);
  const int64_t off = c * ld + (idx - (int64_t)c * nl);
  const float b = beta[c], pv = p[off], zz = z[off];
  p[off] = (b == 0.f || b != b || pv != pv) ? zz : fmaf(b, pv, zz);
}
int k_update_p(float* p, const float* z, const float* beta, int64_t nl, int64_t ld, int t,
               cudaStream_t st) {
  const int64_t total = (int64_t)t * nl;
  if (total <= 0) return GPB_OK;
  update_p_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(p, z, beta, nl, ld, t);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// x += alpha p; r -= alpha Ap, frozen where alpha is 0/NaN or p/Ap is NaN
// (cg_solver.mojo:138-178).
__global__ void cg_update_kernel(const float* __restrict__ alpha, const float* __restrict__ p,
                                 const float* __restrict__ Ap, float* __restrict__ x,
                                 float* __restrict__ r, int64_t nl, int64_t ld, int t) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)t * nl) return;
  const int c = (int)(idx / nl);
  const int64_t i = idx - (int64_t)c * nl;
  const float a = alpha[c];
  if (a == 0.f || a != a) return;
  const int64_t off = c * ld + i;
  const float pv = p[off], av = Ap[off];
  if (pv != pv || av != av) return;
  x[off] = fmaf(a, pv, x[off]);
  r[off] = fmaf(-a, av, r[off]);
}
int k_cg_update(const float* alpha, const float* p, const float* Ap, float* x, float* r,
                int64_t nl, int64_t ld, int t, cudaStream_t st) {
  const int64_t total = (int64_t)t * nl;
  if (total <= 0) return GPB_OK;
  cg_update_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(alpha, p, Ap, x, r, nl, ld, t);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// ------------------------------------------------------------ Woodbury
// sums[c*rank + k] = sum_i L[k][i] v[c][i] over local rows. Each block stages a
// 128-row chunk of v in shared memory; warp w owns rows k = w, w+8, ... of L^T
// and accumulates into a shared [t][rank] block sum (single writer per k).
constexpr int kLtvChunk = 128;

__global__ void __launch_bounds__(256) ltv_kernel(const float* __restrict__ L, int64_t nl,
                                                  int rank, const float* __restrict__ v,
                                                  int64_t ld, int t, double* partial,
                                                  unsigned* counter, double* sums) {
  extern __shared__ float sm[];
  float* vs = sm;                       // [t][kLtvChunk]
  float* acc = sm + t * kLtvChunk;      // [t][rank]
  const int K = t * rank;
  for (int q = threadIdx.x; q < K; q += blockDim.x) acc[q] = 0.f;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int64_t base = (int64_t)blockIdx.x * kLtvChunk; base < nl;
       base += (int64_t)gridDim.x * kLtvChunk) {
    __syncthreads();
    for (int q = threadIdx.x; q < t * kLtvChunk; q += blockDim.x) {
      const int c = q / kLtvChunk, j = q - c * kLtvChunk;
      const int64_t i = base + j;
      vs[q] = (i < nl) ? v[c * ld + i] : 0.f;
    }
    __syncthreads();
    for (int k = warp; k < rank; k += nw) {
      float l[kLtvChunk / 32];
#pragma unroll
      for (int s = 0; s < kLtvChunk / 32; ++s) {
        const int64_t i = base + lane + 32 * s;
        l[s] = (i < nl) ? L[(int64_t)k * nl + i] : 0.f;
      }
      for (int c0 = 0; c0 < t; c0 += 16) {
        float part[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          part[c] = 0.f;
          if (c0 + c < t) {
#pragma unroll
            for (int s = 0; s < kLtvChunk / 32; ++s)
              part[c] = fmaf(l[s], vs[(c0 + c) * kLtvChunk + lane + 32 * s], part[c]);
          }
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float x = part[c];
          for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
          if (lane == 0 && c0 + c < t) acc[(c0 + c) * rank + k] += x;
        }
      }
    }
  }
  __syncthreads();
  for (int q = threadIdx.x; q < K; q += blockDim.x)
    partial[(size_t)blockIdx.x * K + q] = (double)acc[q];
  finalize_partials(partial, K, counter, sums);
}

int k_ltv(const float* L, int64_t nl, int rank, const float* v, int64_t ld, int t, Reducer& red,
          cudaStream_t st) {
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(nl, kLtvChunk), 296));
  GPB_TRY(red.ensure(G, t * rank));
  const size_t smem = ((size_t)t * kLtvChunk + (size_t)t * rank) * sizeof(float);
  GPB_REQUIRE(smem <= 200 * 1024, GPB_ERR_UNSUPPORTED, "L^T v: t*rank too large (%d x %d)", t, rank);
  static bool attr = false;
  if (!attr) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(ltv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        200 * 1024));
    attr = true;
  }
  ltv_kernel<<<G, 256, smem, st>>>(L, nl, rank, v, ld, t, red.partial.d(),
                                   (unsigned*)red.counter.ptr, red.sums.d());
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int k_ltl(const float* L, int64_t nl, int rank, Reducer& red, cudaStream_t st) {
  // L^T L with L viewed as a [rank][nl] block of rhs columns.
  return k_ltv(L, nl, rank, L, nl, rank, red, st);
}

// u[c][k] = sum_m Minv[k][m] w[c][m]
__global__ void minv_apply_kernel(const float* Minv, int rank, const double* w, int t, float* u) {
  const int c = blockIdx.x;
  for (int k = threadIdx.x; k < rank; k += blockDim.x) {
    double s = 0.0;
    for (int m = 0; m < rank; ++m) s += (double)Minv[k * rank + m] * w[c * rank + m];
    u[c * rank + k] = (float)s;
  }
}
int k_minv_apply(const float* Minv, int rank, const double* w, int t, float* u, cudaStream_t st) {
  minv_apply_kernel<<<t, 128, 0, st>>>(Minv, rank, w, t, u);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// out[c][i] = add_coef * src[c][i] + lu_coef * sum_k L[k][i] u[c][k]
__global__ void __launch_bounds__(256) l_times_u_kernel(const float* __restrict__ L, int64_t nl,
                                                        int rank, const float* __restrict__ u,
                                                        int t, const float* __restrict__ src,
                                                        int64_t ld, float add_coef, float lu_coef,
                                                        float* __restrict__ out) {
  extern __shared__ float us[];
  for (int q = threadIdx.x; q < t * rank; q += blockDim.x) us[q] = u[q];
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nl) return;
  for (int c0 = 0; c0 < t; c0 += 16) {
    float acc[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) acc[c] = 0.f;
    for (int k = 0; k < rank; ++k) {
      const float l = L[(int64_t)k * nl + i];
#pragma unroll
      for (int c = 0; c < 16; ++c)
        if (c0 + c < t) acc[c] = fmaf(l, us[(c0 + c) * rank + k], acc[c]);
    }
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      if (c0 + c >= t) break;
      const int64_t off = (int64_t)(c0 + c) * ld + i;
      out[off] = add_coef * src[off] + lu_coef * acc[c];
    }
  }
}

int k_woodbury_out(const float* v, int64_t ld, const float* L, int64_t nl, int rank,
                   const float* u, int t, float inv_noise, float* out, cudaStream_t st) {
  if (nl <= 0) return GPB_OK;
  const size_t smem = (size_t)t * rank * sizeof(float);
  l_times_u_kernel<<<(unsigned)ceil_div(nl, 256), 256, smem, st>>>(L, nl, rank, u, t, v, ld,
                                                                  inv_noise, -inv_noise, out);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int k_l_times_u(const float* L, int64_t nl, int rank, const float* u, int t, const float* src,
                int64_t ld, float add_coef, float lu_coef, float* out, cudaStream_t st) {
  if (nl <= 0) return GPB_OK;
  const size_t smem = (size_t)t * rank * sizeof(float);
  l_times_u_kernel<<<(unsigned)ceil_div(nl, 256), 256, smem, st>>>(L, nl, rank, u, t, src, ld,
                                                                  add_coef, lu_coef, out);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int k_lz_plus_noise(const float* L, int64_t nl, int rank, const float* zr, int t, const float* zn,
                    float sqrt_noise, float* out, cudaStream_t st) {
  if (nl <= 0) return GPB_OK;
  const size_t smem = (size_t)t * rank * sizeof(float);
  l_times_u_kernel<<<(unsigned)ceil_div(nl, 256), 256, smem, st>>>(L, nl, rank, zr, t, zn, nl,
                                                                  sqrt_noise, 1.f, out);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

}  // namespace gpb

extern "C" int gpb_hash_gaussian(int32_t device, float* out_host, int64_t count, uint64_t seed) {
  using namespace gpb;
  GPB_REQUIRE(out_host && count >= 0, GPB_ERR_INVALID, "bad arguments");
  if (count == 0) return GPB_OK;
  GPB_CHECK_CUDA(cudaSetDevice(device));
  float* d = nullptr;
  GPB_CHECK_CUDA(cudaMalloc(&d, count * sizeof(float)));
  int s = k_gaussian(d, 1, count, count, count, 0, seed, 0);
  if (s == GPB_OK) {
    cudaError_t e = cudaMemcpy(out_host, d, count * sizeof(float), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
      set_error("gaussian copy: %s", cudaGetErrorString(e));
      s = GPB_ERR_CUDA;
    }
  }
  cudaFree(d);
  return s;
}
