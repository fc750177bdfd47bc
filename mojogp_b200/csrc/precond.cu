// Greedy pivoted-Cholesky preconditioner P = L L^T + sigma^2 I.
//
// Reference: build_pivoted_cholesky_precond_unified
// (mojogp/kernels/pivoted_cholesky.mojo:2104-2444, precond_method = 0), the
// Woodbury apply (1646-1766), log|P| (1411-1517) and N(0, P) probe sampling
// (1909-2011). B200 changes: the pivot column is one kernel-row evaluation
// K(X, x_piv) (O(n d)) instead of a full K·e_piv matvec (O(n^2 d)); argmax,
// orthogonalisation, scaling and the diagonal update stay on the device with
// no host round trip per pivot; rows may be sharded across GPUs (argmax by an
// all-reduce of packed (value, index) keys).
#include "engine.cuh"
#include "numerics.h"
#include "precond.cuh"

namespace gpb {

__global__ void pc_init_kernel(const float* __restrict__ X, int d, int64_t r0, int64_t nl,
                               const __grid_constant__ DevKernel K, float* __restrict__ diag,
                               float* __restrict__ mask) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nl) return;
  float xi[GPB_MAX_DIM];
  for (int k = 0; k < d; ++k) xi[k] = X[(r0 + i) * d + k];
  diag[i] = tree_eval<false>(K, xi, xi, nullptr);
  mask[i] = 1.f;
}

__device__ __forceinline__ uint32_t ordered_bits(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_ordered_bits(uint32_t o) {
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return __uint_as_float(u);
}

// Masked argmax over local rows; ties go to the lowest global index
// (pivoted_cholesky.mojo:537-539, 573-577). Key = ordered(value) << 32 |
// (0xffffffff - index), so a max-reduction picks the largest value and then
// the smallest index.
__global__ void __launch_bounds__(256) pc_argmax_kernel(const float* __restrict__ diag,
                                                        const float* __restrict__ mask, int64_t nl,
                                                        int64_t r0, const int* __restrict__ done,
                                                        unsigned long long* partial,
                                                        unsigned* counter,
                                                        unsigned long long* result) {
  if (*done) return;
  unsigned long long best = 0ull;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nl;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (mask[i] > 0.5f) {
      const unsigned long long key =
          ((unsigned long long)ordered_bits(diag[i]) << 32) |
          (unsigned long long)(0xffffffffu - (uint32_t)(r0 + i));
      best = key > best ? key : best;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  __shared__ unsigned long long sh[8];
  __shared__ bool last;
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = sh[w] > b ? sh[w] : b;
    partial[blockIdx.x] = b;
    __threadfence();
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    unsigned long long b = 0ull;
    for (unsigned q = 0; q < gridDim.x; ++q) {
      const unsigned long long v = ((volatile unsigned long long*)partial)[q];
      b = v > b ? v : b;
    }
    *result = b;
    *counter = 0u;
  }
}

// Decode the pivot, apply the termination rule (max residual diagonal
// < 1e-10 => stop with rank max(m, 1)), mark the pivot used, and gather the
// pivot's row of L (this rank's contribution; all-reduced when sharded).
__global__ void pc_pivot_kernel(const unsigned long long* result, int m, int64_t r0, int64_t nl,
                                int* done, int* actual_rank, float* mask, const float* L,
                                float* lrow, float* pivinfo, int64_t* piv_out, float* val_out) {
  const unsigned long long key = *result;
  const bool was_done = *done != 0;
  const float maxv = key ? from_ordered_bits((uint32_t)(key >> 32)) : -1e30f;
  const int64_t piv = key ? (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull)) : -1;
  __syncthreads();
  if (was_done) return;
  if (!(maxv >= 1e-10f) || piv < 0) {
    if (threadIdx.x == 0) {
      *done = 1;
      *actual_rank = m > 0 ? m : 1;
    }
    return;
  }
  const bool owner = piv >= r0 && piv < r0 + nl;
  for (int j = threadIdx.x; j < m; j += blockDim.x)
    lrow[j] = owner ? L[(int64_t)j * nl + (piv - r0)] : 0.f;
  if (threadIdx.x == 0) {
    if (owner) mask[piv - r0] = 0.f;
    pivinfo[0] = (float)piv;  // exact for n < 2^24, as in the reference
    pivinfo[1] = maxv;
    piv_out[m] = piv;
    val_out[m] = maxv;
    *actual_rank = m + 1;
  }
}

__global__ void pc_column_kernel(const float* __restrict__ X, int d, int64_t r0, int64_t nl,
                                 const __grid_constant__ DevKernel K, const int* done,
                                 const unsigned long long* result, const float* __restrict__ lrow,
                                 int m, float* __restrict__ L, float* __restrict__ diag,
                                 const float* __restrict__ mask) {
  if (*done) return;
  const unsigned long long key = *result;
  const float maxv = from_ordered_bits((uint32_t)(key >> 32));
  const int64_t piv = (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nl) return;
  float xi[GPB_MAX_DIM], xp[GPB_MAX_DIM];
  for (int k = 0; k < d; ++k) {
    xi[k] = X[(r0 + i) * d + k];
    xp[k] = X[piv * d + k];
  }
  float col = tree_eval<false>(K, xi, xp, nullptr);
  float s = 0.f;
  for (int j = 0; j < m; ++j) s = fmaf(L[(int64_t)j * nl + i], lrow[j], s);
  col -= s;
  col *= 1.f / sqrtf(fmaxf(maxv, 1e-10f));
  L[(int64_t)m * nl + i] = col;
  if (mask[i] > 0.5f) diag[i] -= col * col;
}

int precond_build(Engine& E, int rank_req, Precond& P, bool finalize) {
  P.rank = 0;
  P.logdet = 0.0;
  P.noise = E.p->noise;
  if (rank_req <= 0) return GPB_OK;
  GPB_REQUIRE(E.p->noise_vec_d == nullptr, GPB_ERR_UNSUPPORTED,
              "pivoted-Cholesky preconditioner with a fixed noise vector is not supported");
  const int64_t nl = E.nl;
  const int rmax = (int)std::min<int64_t>(rank_req, E.n);
  GPB_TRY(P.L.ensure((size_t)rmax * std::max<int64_t>(nl, 1) * sizeof(float)));
  GPB_TRY(P.diag.ensure((size_t)std::max<int64_t>(nl, 1) * sizeof(float)));
  GPB_TRY(P.mask.ensure((size_t)std::max<int64_t>(nl, 1) * sizeof(float)));
  GPB_TRY(P.scratch.ensure(4096 + (size_t)rmax * sizeof(float)));
  GPB_TRY(P.keys.ensure(sizeof(unsigned long long) * 512));
  GPB_TRY(P.piv.ensure((size_t)rmax * (sizeof(int64_t) + sizeof(float))));
  int64_t* piv_out = (int64_t*)P.piv.ptr;
  float* val_out = (float*)(piv_out + rmax);
  GPB_CHECK_CUDA(cudaMemsetAsync(P.piv.ptr, 0, P.piv.bytes, E.st));
  cudaStream_t st = E.st;
  char* base = (char*)P.scratch.ptr;
  unsigned long long* result = (unsigned long long*)base;        // 8 B
  int* done = (int*)(base + 8);
  int* actual = (int*)(base + 12);
  unsigned* counter = (unsigned*)(base + 16);
  float* pivinfo = (float*)(base + 32);
  float* lrow = (float*)(base + 64);
  GPB_CHECK_CUDA(cudaMemsetAsync(base, 0, 64, st));
  GPB_CHECK_CUDA(cudaMemsetAsync(P.L.ptr, 0, (size_t)rmax * nl * sizeof(float), st));
  const int bs = 256;
  const unsigned nb = (unsigned)std::max<int64_t>(1, ceil_div(nl, bs));
  gpb_provider* p = E.p;
  pc_init_kernel<<<nb, bs, 0, st>>>(p->X_d, p->d, E.r0, nl, p->dk, P.diag.f(), P.mask.f());
  GPB_CHECK_CUDA(cudaGetLastError());
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(nl, 1024), 296));
  for (int m = 0; m < rmax; ++m) {
    pc_argmax_kernel<<<G, 256, 0, st>>>(P.diag.f(), P.mask.f(), nl, E.r0, done,
                                        (unsigned long long*)P.keys.ptr, counter, result);
    GPB_CHECK_CUDA(cudaGetLastError());
    if (E.dist.world > 1) {
      ncclResult_t r =
          ncclAllReduce(result, result, 1, ncclUint64, ncclMax, E.dist.comm, st);
      GPB_REQUIRE(r == ncclSuccess, GPB_ERR_NCCL, "argmax all-reduce: %s", ncclGetErrorString(r));
    }
    pc_pivot_kernel<<<1, 256, 0, st>>>(result, m, E.r0, nl, done, actual, P.mask.f(), P.L.f(),
                                       lrow, pivinfo, piv_out, val_out);
    GPB_CHECK_CUDA(cudaGetLastError());
    if (E.dist.world > 1 && m > 0) GPB_TRY(E.allreduce_sum_f(lrow, (size_t)m));
    pc_column_kernel<<<nb, bs, 0, st>>>(p->X_d, p->d, E.r0, nl, p->dk, done, result, lrow, m,
                                        P.L.f(), P.diag.f(), P.mask.f());
    GPB_CHECK_CUDA(cudaGetLastError());
    p->launches += 3;
  }
  int act = 0;
  GPB_CHECK_CUDA(cudaMemcpyAsync(&act, actual, sizeof(int), cudaMemcpyDeviceToHost, st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  P.rank = std::max(1, std::min(act, rmax));
  return finalize ? precond_finalize(E, P) : GPB_OK;
}

// M = L^T L; Minv = (M + max(noise, 1e-6) I)^{-1} (pivoted_cholesky.mojo:1083-1207);
// log|P| = n log(noise) + log|I + M / noise| (1411-1517).
int precond_finalize(Engine& E, Precond& P) {
  const int r = P.rank;
  GPB_TRY(k_ltl(P.L.f(), E.nl, r, E.red, E.st));
  GPB_TRY(E.allreduce_sum(E.red.sums.d(), (size_t)r * r));
  std::vector<double> M((size_t)r * r);
  GPB_CHECK_CUDA(cudaMemcpyAsync(M.data(), E.red.sums.ptr, M.size() * sizeof(double),
                                 cudaMemcpyDeviceToHost, E.st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(E.st));
  const double noise = P.noise;
  const double eff = noise > 1e-6 ? noise : 1e-6;
  std::vector<double> A(M), Ainv((size_t)r * r);
  for (int i = 0; i < r; ++i) A[(size_t)i * r + i] += eff;
  GPB_REQUIRE(spd_inverse(A.data(), r, Ainv.data(), nullptr), GPB_ERR_NUMERIC,
              "L^T L + noise I is singular");
  std::vector<float> Af(Ainv.begin(), Ainv.end());
  GPB_TRY(P.Minv.ensure(Af.size() * sizeof(float)));
  GPB_CHECK_CUDA(cudaMemcpyAsync(P.Minv.ptr, Af.data(), Af.size() * sizeof(float),
                                 cudaMemcpyHostToDevice, E.st));
  std::vector<double> B(M), Binv((size_t)r * r);
  for (auto& v : B) v /= noise;
  for (int i = 0; i < r; ++i) B[(size_t)i * r + i] += 1.0;
  double ld = 0.0;
  GPB_REQUIRE(spd_inverse(B.data(), r, Binv.data(), &ld), GPB_ERR_NUMERIC,
              "I + L^T L / noise is singular");
  P.logdet = (double)E.n * std::log(noise) + ld;
  GPB_CHECK_CUDA(cudaStreamSynchronize(E.st));
  return GPB_OK;
}

// out = P^{-1} v = (v - L (L^T L + s I)^{-1} L^T v) / sigma^2 (in place allowed).
int precond_apply(Engine& E, Precond& P, const float* v, float* out, int t) {
  if (P.lmc) return lmc_precond_apply(E, *P.lmc, v, out, t);
  const int r = P.rank;
  GPB_TRY(k_ltv(P.L.f(), E.nl, r, v, E.nl, t, E.red, E.st));
  GPB_TRY(E.allreduce_sum(E.red.sums.d(), (size_t)t * r));
  GPB_TRY(P.u.ensure((size_t)t * r * sizeof(float)));
  GPB_TRY(k_minv_apply(P.Minv.f(), r, E.red.sums.d(), t, P.u.f(), E.st));
  GPB_TRY(k_woodbury_out(v, E.nl, P.L.f(), E.nl, r, P.u.f(), t, 1.f / P.noise, out, E.st));
  E.p->launches += 3;
  return GPB_OK;
}

// N(0, P) probes: L z_rank + sqrt(noise) z_noise with hash Gaussians seeded
// `seed` ([num][rank] layout) and seed + 1e6 ([num][n] layout).
int precond_sample(Engine& E, Precond& P, int num, uint64_t seed, float* out) {
  if (P.lmc) return lmc_precond_sample(E, *P.lmc, num, seed, out);
  const int r = P.rank;
  GPB_TRY(P.u.ensure((size_t)num * r * sizeof(float)));
  GPB_TRY(k_gaussian(P.u.f(), 1, (int64_t)num * r, (int64_t)num * r, (int64_t)num * r, 0, seed, E.st));
  GPB_TRY(k_gaussian(out, num, E.nl, E.nl, E.n, E.r0, seed + 1000000ull, E.st));
  GPB_TRY(k_lz_plus_noise(P.L.f(), E.nl, r, P.u.f(), num, out, std::sqrt(P.noise), out, E.st));
  return GPB_OK;
}

}  // namespace gpb
