// Prediction: alpha solve, LOVE inverse root, predictive mean and variance.
//
// References (MojoGP 0.26.6.0, kernels/jit/jit_prediction.mojo):
//   solve_single_rhs_deterministic_host_jit 681-759 (alpha CG, relative stop)
//   compute_lanczos_inv_root_jit            974-1177 (Lanczos + reorth + T^-1/2)
//   predict_variance_love_from_inv_root_jit 1236-1344, kernel_love_variance 211-232
//   predict_from_alpha_jit noise add        2048-2051
//   predict_variance_exact_jit              1352-1788, kernel_exact_variance 235-256
// B200 changes: every vector update, dot product and the Lanczos
// re-orthogonalisation (two classical Gram-Schmidt passes as GEMVs over the
// device-resident basis) run on the GPU, rows sharded across ranks; only
// scalars cross to the host. The predictive pass is one tiled cross matvec
// with [alpha | S] as right-hand sides.
#include <cmath>
#include <vector>

#include "engine.cuh"
#include "numerics.h"
#include "precond.cuh"
#include "train.cuh"

struct gpb_comm;  // defined in train.cu
namespace gpb {
int engine_from_comm(gpb_provider* p, gpb_comm* c, Engine& E);
}

struct gpb_prediction_cache {
  gpb_provider* p = nullptr;
  gpb_comm* comm = nullptr;
  int rank = 0;
  float mean = 0.f;
  float noise = 0.f;
  gpb::DBuf rhs;  // [1 + rank][n]: alpha then S columns (all rows)
  int love_iters = 0;
};

namespace gpb {

__global__ void axpy2_kernel(float* x, float* r, const float* p, const float* Ap, float alpha,
                             int64_t nl) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nl) return;
  x[i] = fmaf(alpha, p[i], x[i]);
  r[i] = fmaf(-alpha, Ap[i], r[i]);
}
__global__ void xpby_kernel(float* p, const float* r, float beta, int64_t nl) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nl) p[i] = fmaf(beta, p[i], r[i]);
}
__global__ void axpy_kernel(float* y, const float* x, float a, int64_t nl) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nl) y[i] = fmaf(a, x[i], y[i]);
}
__global__ void scale_to_kernel(float* dst, const float* src, float s, int64_t nl) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nl) dst[i] = src[i] * s;
}

// (K + noise) alpha = y_centered by CG with the reference's stopping rule
// |r| / |r0| < tol and pAp < 1e-10 / NaN breakdown (jit_prediction.mojo:681-759).
int alpha_cg(Engine& E, const float* y_local, float* x, int max_iter, float tol, int* iters_out) {
  const int64_t nl = E.nl;
  cudaStream_t st = E.st;
  DBuf r, p, Ap;
  GPB_TRY(r.ensure(E.blk(1) + 16));
  GPB_TRY(p.ensure(E.blk(1) + 16));
  GPB_TRY(Ap.ensure(E.blk(1) + 16));
  GPB_TRY(k_fill(x, nl, 0.f, st));
  GPB_TRY(k_copy(r.f(), y_local, nl, st));
  GPB_TRY(k_copy(p.f(), y_local, nl, st));
  const unsigned nb = (unsigned)std::max<int64_t>(1, ceil_div(nl, 256));
  const float* a1[1] = {r.f()};
  GPB_TRY(E.coldots(1, a1, a1, nl, 1, true));
  float rr_old = (float)E.host_sums[0];
  float r0 = std::sqrt(rr_old);
  if (r0 < 1e-20f) r0 = 1.f;
  int it = 0;
  for (; it < max_iter; ++it) {
    GPB_TRY(E.matvec(p.f(), nl, 1, Ap.f(), nl));
    const float* a[1] = {p.f()};
    const float* b[1] = {Ap.f()};
    GPB_TRY(E.coldots(1, a, b, nl, 1, true));
    const float pAp = (float)E.host_sums[0];
    if (pAp != pAp || pAp < 1e-10f) break;
    const float alpha = rr_old / pAp;
    if (alpha != alpha) break;
    axpy2_kernel<<<nb, 256, 0, st>>>(x, r.f(), p.f(), Ap.f(), alpha, nl);
    GPB_CHECK_CUDA(cudaGetLastError());
    GPB_TRY(E.coldots(1, a1, a1, nl, 1, true));
    const float rr_new = (float)E.host_sums[0];
    if (std::sqrt(rr_new) / r0 < tol) {
      ++it;
      break;
    }
    float beta = 0.f;
    if (rr_old >= 1e-20f) {
      beta = rr_new / (rr_old + 1e-20f);
      if (beta < 0.f || beta != beta) beta = 0.f;
    }
    xpby_kernel<<<nb, 256, 0, st>>>(p.f(), r.f(), beta, nl);
    GPB_CHECK_CUDA(cudaGetLastError());
    rr_old = rr_new;
  }
  if (iters_out) *iters_out = it;
  return GPB_OK;
}

// Deterministic +-1 start vector of compute_lanczos_inv_root_jit (1000-1014).
__global__ void lanczos_start_kernel(float* v, int64_t nl, int64_t row0, int r, float inv_norm) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nl) return;
  const uint64_t gi = (uint64_t)(row0 + i);
  uint64_t s = 0xC0FFEE1234567890ull ^ (gi * 0x9E3779B97F4A7C15ull) ^
               ((uint64_t)r * 0xBF58476D1CE4E5B9ull);
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  s *= 0x2545F4914F6CDD1Dull;
  v[i] = ((s & 0x20000ull) ? 1.f : -1.f) * inv_norm;
}

// S = Q T^{-1/2} with S S^T ~= (K + noise I)^{-1}; S local rows [rank][nl].
int love_root(Engine& E, int r, float* S_local, int* iters_out) {
  const int64_t nl = E.nl;
  cudaStream_t st = E.st;
  const unsigned nb = (unsigned)std::max<int64_t>(1, ceil_div(nl, 256));
  DBuf Q, w, inner;
  GPB_TRY(Q.ensure((size_t)r * std::max<int64_t>(nl, 1) * sizeof(float)));
  GPB_TRY(w.ensure(E.blk(1) + 16));
  GPB_TRY(inner.ensure((size_t)(r + 1) * sizeof(float)));
  GPB_CHECK_CUDA(cudaMemsetAsync(Q.ptr, 0, (size_t)r * nl * sizeof(float), st));
  const float inv_norm = 1.f / std::sqrt((float)E.n);  // |z|^2 = n for a +-1 vector
  lanczos_start_kernel<<<nb, 256, 0, st>>>(Q.f(), nl, E.r0, r, inv_norm);
  GPB_CHECK_CUDA(cudaGetLastError());
  std::vector<double> alpha(r, 0.0), beta(std::max(r - 1, 0), 0.0);
  std::vector<float> hin(r + 1);
  float beta_prev = 0.f;
  int steps = 0;
  for (int j = 0; j < r; ++j) {
    float* vj = Q.f() + (int64_t)j * nl;
    GPB_TRY(E.matvec(vj, nl, 1, w.f(), nl));
    const float* a[1] = {vj};
    const float* b[1] = {w.f()};
    GPB_TRY(E.coldots(1, a, b, nl, 1, true));
    const float aj = (float)E.host_sums[0];
    alpha[j] = aj;
    axpy_kernel<<<nb, 256, 0, st>>>(w.f(), vj, -aj, nl);
    if (j > 0) axpy_kernel<<<nb, 256, 0, st>>>(w.f(), vj - nl, -beta_prev, nl);
    GPB_CHECK_CUDA(cudaGetLastError());
    // Two re-orthogonalisation passes against Q[0..j]; the second is skipped
    // when every inner product of the first is below 1e-5.
    for (int pass = 0; pass < 2; ++pass) {
      GPB_TRY(k_ltv(Q.f(), nl, j + 1, w.f(), nl, 1, E.red, st));
      GPB_TRY(E.allreduce_sum(E.red.sums.d(), (size_t)j + 1));
      std::vector<double> inn(j + 1);
      GPB_CHECK_CUDA(cudaMemcpyAsync(inn.data(), E.red.sums.ptr, (j + 1) * sizeof(double),
                                     cudaMemcpyDeviceToHost, st));
      GPB_CHECK_CUDA(cudaStreamSynchronize(st));
      float max_inner = 0.f;
      for (int k = 0; k <= j; ++k) {
        hin[k] = (float)inn[k];
        max_inner = std::max(max_inner, std::fabs(hin[k]));
      }
      GPB_CHECK_CUDA(cudaMemcpyAsync(inner.ptr, hin.data(), (j + 1) * sizeof(float),
                                     cudaMemcpyHostToDevice, st));
      GPB_TRY(k_l_times_u(Q.f(), nl, j + 1, inner.f(), 1, w.f(), nl, 1.f, -1.f, w.f(), st));
      if (max_inner < 1e-5f) break;
    }
    const float* aw[1] = {w.f()};
    GPB_TRY(E.coldots(1, aw, aw, nl, 1, true));
    const float bj = std::sqrt((float)E.host_sums[0]);
    steps = j + 1;
    if (j < r - 1) beta[j] = bj;
    if (bj < 1e-10f) break;  // breakdown: remaining basis rows stay zero
    if (j + 1 < r) {
      scale_to_kernel<<<nb, 256, 0, st>>>(Q.f() + (int64_t)(j + 1) * nl, w.f(), 1.f / bj, nl);
      GPB_CHECK_CUDA(cudaGetLastError());
    }
    beta_prev = bj;
  }
  // T = tridiag(alpha, beta); T^{-1/2} = V diag(max(lambda, 1e-6 lambda_max)^-1/2) V^T.
  std::vector<double> ev(r), V((size_t)r * r);
  tridiag_eig(alpha.data(), beta.data(), r, ev.data(), V.data());
  double max_eig = 1e-10;
  for (double v : ev) max_eig = std::max(max_eig, v);
  const double clamp = max_eig * 1e-6;
  std::vector<float> Tis((size_t)r * r);
  for (int i = 0; i < r; ++i)
    for (int c = 0; c < r; ++c) {
      double s = 0.0;
      for (int k = 0; k < r; ++k) s += V[(size_t)i * r + k] / std::sqrt(std::max(ev[k], clamp)) * V[(size_t)c * r + k];
      Tis[(size_t)c * r + i] = (float)s;  // stored [c][i] so column c of S uses u[c][k=i]
    }
  DBuf tis;
  GPB_TRY(tis.ensure(Tis.size() * sizeof(float)));
  GPB_CHECK_CUDA(cudaMemcpyAsync(tis.ptr, Tis.data(), Tis.size() * sizeof(float),
                                 cudaMemcpyHostToDevice, st));
  // S[c][i] = sum_k Q[k][i] T^{-1/2}[k][c]
  for (int c0 = 0; c0 < r; c0 += 16) {
    const int tc = std::min(16, r - c0);
    GPB_TRY(k_l_times_u(Q.f(), nl, r, tis.f() + (size_t)c0 * r, tc, Q.f(), nl, 0.f, 1.f,
                        S_local + (int64_t)c0 * nl, st));
  }
  GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  if (iters_out) *iters_out = steps;
  return GPB_OK;
}

__global__ void love_accum_kernel(const float* __restrict__ V, int64_t ld, int c_begin, int c_end,
                                  int64_t nt, float* __restrict__ acc) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nt) return;
  float s = acc[i];
  for (int c = c_begin; c < c_end; ++c) {
    const float v = V[c * ld + i];
    s = fmaf(v, v, s);
  }
  acc[i] = s;
}

__global__ void love_finish_kernel(const float* __restrict__ V0, const float* __restrict__ diag,
                                   const float* __restrict__ acc, float mean, float noise,
                                   int64_t nt, int want_var, float* __restrict__ mean_out,
                                   float* __restrict__ var_out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nt) return;
  mean_out[i] = V0[i] + mean;
  if (want_var) {
    float v = diag[i] - acc[i];
    if (v < 1e-10f) v = 1e-10f;
    var_out[i] = v + noise;
  }
}

}  // namespace gpb

using namespace gpb;

namespace gpb {
// out[c][i] = k(x_{r0 + i}, x*_c) over this rank's training rows (raw inputs,
// tree evaluator), one row of the exact-variance right-hand side per test point.
__global__ void cross_fill_kernel(const float* __restrict__ X, int64_t r0, int64_t nl, int d,
                                  const float* __restrict__ Xt, const __grid_constant__ DevKernel K,
                                  float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int c = blockIdx.y;
  if (i >= nl) return;
  float xi[GPB_MAX_DIM], xc[GPB_MAX_DIM];
  for (int k = 0; k < d; ++k) {
    xi[k] = X[(r0 + i) * d + k];
    xc[k] = Xt[(int64_t)c * d + k];
  }
  out[(int64_t)c * nl + i] = tree_eval<false>(K, xi, xc, nullptr);
}
int cross_fill(gpb_provider* p, int64_t r0, int64_t nl, const float* xt_dev, int m, float* out,
               cudaStream_t st) {
  if (nl <= 0 || m <= 0) return GPB_OK;
  dim3 grid((unsigned)ceil_div(nl, 128), (unsigned)m);
  cross_fill_kernel<<<grid, 128, 0, st>>>(p->X_d, r0, nl, p->d, xt_dev, p->dk, out);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}
}  // namespace gpb

extern "C" {

int gpb_compute_alpha(gpb_provider* p, gpb_comm* comm, const float* y_centered_host, int64_t n,
                      int32_t max_cg_iter, float cg_tol, float* alpha_host_out,
                      int32_t* iters_out) {
  clear_error();
  GPB_REQUIRE(p && y_centered_host && alpha_host_out && n == p->n && max_cg_iter >= 0,
              GPB_ERR_INVALID, "bad arguments");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  Engine E;
  GPB_TRY(engine_from_comm(p, comm, E));
  DBuf y, x, full;
  GPB_TRY(y.ensure(E.blk(1) + 16));
  GPB_TRY(x.ensure(E.blk(1) + 16));
  GPB_CHECK_CUDA(cudaMemcpyAsync(y.ptr, y_centered_host + E.r0, E.nl * sizeof(float),
                                 cudaMemcpyHostToDevice, E.st));
  int it = 0;
  GPB_TRY(alpha_cg(E, y.f(), x.f(), max_cg_iter, cg_tol, &it));
  GPB_TRY(full.ensure((size_t)n * sizeof(float)));
  GPB_TRY(E.allgather_cols(x.f(), E.nl, 1, full.f()));
  GPB_CHECK_CUDA(cudaMemcpyAsync(alpha_host_out, full.ptr, n * sizeof(float),
                                 cudaMemcpyDeviceToHost, E.st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(E.st));
  if (iters_out) *iters_out = it;
  return provider_check_device_error(p);
}

int gpb_prediction_cache_create(gpb_provider* p, gpb_comm* comm, const float* alpha_host,
                                float mean, int32_t love_rank, const float* root_host,
                                gpb_prediction_cache** out) {
  clear_error();
  GPB_REQUIRE(p && alpha_host && out && love_rank >= 0, GPB_ERR_INVALID, "bad arguments");
  *out = nullptr;
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  auto* c = new gpb_prediction_cache();
  c->p = p;
  c->comm = comm;
  c->rank = love_rank;
  c->mean = mean;
  c->noise = p->noise;
  const int64_t n = p->n;
  int s = c->rhs.ensure((size_t)(1 + love_rank) * n * sizeof(float));
  if (s == GPB_OK &&
      cudaMemcpyAsync(c->rhs.ptr, alpha_host, n * sizeof(float), cudaMemcpyHostToDevice,
                      p->stream) != cudaSuccess)
    s = GPB_ERR_CUDA;
  if (s == GPB_OK && love_rank > 0) {
    if (root_host) {
      if (cudaMemcpyAsync(c->rhs.f() + n, root_host, (size_t)love_rank * n * sizeof(float),
                          cudaMemcpyHostToDevice, p->stream) != cudaSuccess)
        s = GPB_ERR_CUDA;
    } else {
      Engine E;
      s = engine_from_comm(p, comm, E);
      DBuf Sl;
      if (s == GPB_OK) s = Sl.ensure((size_t)love_rank * std::max<int64_t>(E.nl, 1) * sizeof(float));
      if (s == GPB_OK) s = love_root(E, love_rank, Sl.f(), &c->love_iters);
      if (s == GPB_OK) s = E.allgather_cols(Sl.f(), E.nl, love_rank, c->rhs.f() + n);
    }
  }
  if (s == GPB_OK && cudaStreamSynchronize(p->stream) != cudaSuccess) s = GPB_ERR_CUDA;
  if (s != GPB_OK) {
    delete c;
    return s;
  }
  *out = c;
  return provider_check_device_error(p);
}

int gpb_prediction_cache_root(gpb_prediction_cache* c, float* root_host_out) {
  GPB_REQUIRE(c && root_host_out, GPB_ERR_INVALID, "bad arguments");
  GPB_CHECK_CUDA(cudaSetDevice(c->p->device));
  GPB_CHECK_CUDA(cudaMemcpy(root_host_out, c->rhs.f() + c->p->n,
                            (size_t)c->rank * c->p->n * sizeof(float), cudaMemcpyDeviceToHost));
  return GPB_OK;
}

int gpb_predict_with_cache(gpb_prediction_cache* c, const float* xtest_host, int64_t n_test,
                           float* mean_out, float* var_out) {
  clear_error();
  GPB_REQUIRE(c && xtest_host && mean_out && n_test >= 0, GPB_ERR_INVALID, "bad arguments");
  GPB_REQUIRE(var_out == nullptr || c->rank > 0, GPB_ERR_INVALID,
              "variance requested but the cache has no LOVE root");
  if (n_test == 0) return GPB_OK;
  gpb_provider* p = c->p;
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  cudaStream_t st = p->stream;
  const int ncols = var_out ? 1 + c->rank : 1;
  DBuf xt, V, acc, diag, mo, vo;
  GPB_TRY(xt.ensure((size_t)n_test * p->d * sizeof(float)));
  GPB_TRY(V.ensure((size_t)std::min(ncols, 16) * n_test * sizeof(float)));
  GPB_TRY(acc.ensure((size_t)n_test * sizeof(float)));
  GPB_TRY(diag.ensure((size_t)n_test * sizeof(float)));
  GPB_TRY(mo.ensure((size_t)n_test * sizeof(float)));
  GPB_TRY(vo.ensure((size_t)n_test * sizeof(float)));
  GPB_CHECK_CUDA(cudaMemcpyAsync(xt.ptr, xtest_host, (size_t)n_test * p->d * sizeof(float),
                                 cudaMemcpyHostToDevice, st));
  GPB_CHECK_CUDA(cudaMemsetAsync(acc.ptr, 0, n_test * sizeof(float), st));
  const float* xs = nullptr;
  GPB_TRY(provider_prescale_rows(p, xt.f(), n_test, WS_XTEST, &xs, st));
  const unsigned nb = (unsigned)ceil_div(n_test, 256);
  DBuf V0;
  GPB_TRY(V0.ensure((size_t)n_test * sizeof(float)));
  for (int c0 = 0; c0 < ncols; c0 += 16) {
    const int tc = std::min(16, ncols - c0);
    GPB_TRY(provider_kv(p, xs, n_test, c->rhs.f() + (int64_t)c0 * p->n, p->n, tc, V.f(), n_test,
                        false, 0, st));
    if (c0 == 0) GPB_TRY(k_copy(V0.f(), V.f(), n_test, st));
    const int cb = (c0 == 0) ? 1 : 0;
    if (tc > cb) {
      love_accum_kernel<<<nb, 256, 0, st>>>(V.f(), n_test, cb, tc, n_test, acc.f());
      GPB_CHECK_CUDA(cudaGetLastError());
    }
  }
  if (var_out) GPB_TRY(gpb_extract_diagonal_test(p, diag.f(), xt.f(), n_test));
  love_finish_kernel<<<nb, 256, 0, st>>>(V0.f(), diag.f(), acc.f(), c->mean, c->noise, n_test,
                                        var_out ? 1 : 0, mo.f(), vo.f());
  GPB_CHECK_CUDA(cudaGetLastError());
  GPB_CHECK_CUDA(cudaMemcpyAsync(mean_out, mo.ptr, n_test * sizeof(float), cudaMemcpyDeviceToHost, st));
  if (var_out)
    GPB_CHECK_CUDA(cudaMemcpyAsync(var_out, vo.ptr, n_test * sizeof(float), cudaMemcpyDeviceToHost, st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  return provider_check_device_error(p);
}

int gpb_prediction_cache_destroy(gpb_prediction_cache* c) {
  if (!c) return GPB_OK;
  cudaSetDevice(c->p->device);
  delete c;
  return GPB_OK;
}

int gpb_predict_exact_variance(gpb_provider* p, gpb_comm* comm, const float* xtest_host,
                               int64_t n_test, int32_t block_cols, int32_t max_cg_iter,
                               float cg_tol, int32_t precond_rank, float* var_out,
                               int32_t* cg_iters_out) {
  clear_error();
  GPB_REQUIRE(p && xtest_host && var_out && n_test >= 0 && max_cg_iter >= 1, GPB_ERR_INVALID,
              "bad arguments");
  if (n_test == 0) return GPB_OK;
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  Engine E;
  GPB_TRY(engine_from_comm(p, comm, E));
  cudaStream_t st = E.st;
  // Block width: all test points up to 512 columns (choose_exact_prediction_block_cols).
  const int b = (int)std::min<int64_t>(n_test, block_cols > 0 ? block_cols : 512);
  Precond P;
  if (precond_rank > 0) GPB_TRY(precond_build(E, precond_rank, P));
  BBMMState S;
  GPB_TRY(S.ensure(E, b, 1));
  DBuf xt, cross, diag;
  GPB_TRY(xt.ensure((size_t)n_test * p->d * sizeof(float)));
  GPB_TRY(cross.ensure((size_t)b * std::max<int64_t>(E.nl, 1) * sizeof(float)));
  GPB_TRY(diag.ensure((size_t)b * sizeof(float)));
  GPB_CHECK_CUDA(cudaMemcpyAsync(xt.ptr, xtest_host, (size_t)n_test * p->d * sizeof(float),
                                 cudaMemcpyHostToDevice, st));
  std::vector<float> norms, dg(b);
  int total_iters = 0;
  for (int64_t c0 = 0; c0 < n_test; c0 += b) {
    const int m = (int)std::min<int64_t>(b, n_test - c0);
    const float* xb = xt.f() + c0 * p->d;
    // 1. K(X_local, X*_block) [m][nl] and k(x*, x*).
    if (E.nl > 0) {
      dim3 grid((unsigned)ceil_div(E.nl, 128), (unsigned)m);
      cross_fill_kernel<<<grid, 128, 0, st>>>(p->X_d, E.r0, E.nl, p->d, xb, p->dk, cross.f());
      GPB_CHECK_CUDA(cudaGetLastError());
    }
    GPB_TRY(gpb_extract_diagonal_test(p, diag.f(), xb, m));
    // 2. (K + noise I) V = K(X, X*) by batched CG on normalised columns.
    float* rhs = S.rhs.f();
    GPB_TRY(k_copy(rhs, cross.f(), (int64_t)m * E.nl, st));
    float* norms_dev = S.scal.f() + 3 * m;
    GPB_TRY(column_norms(E, rhs, m, norms, norms_dev, true));
    CGResult cg;
    GPB_TRY(cg_solve(E, precond_rank > 0 ? &P : nullptr, S, rhs, m, max_cg_iter, 0, cg_tol, false,
                     cg));
    total_iters += cg.iters;
    float* sol = S.x.f();
    GPB_TRY(k_scale_cols(sol, E.nl, E.nl, m, norms_dev, 0, st));
    // 3. var = max(k** - K(X, x*) . v, 1e-10) + noise.
    const float* a[1] = {cross.f()};
    const float* bb[1] = {sol};
    GPB_TRY(E.coldots(1, a, bb, E.nl, m, true));
    GPB_CHECK_CUDA(cudaMemcpyAsync(dg.data(), diag.ptr, m * sizeof(float), cudaMemcpyDeviceToHost, st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(st));
    for (int c = 0; c < m; ++c) {
      float v = dg[c] - (float)E.host_sums[c];
      if (v < 1e-10f) v = 1e-10f;
      var_out[c0 + c] = v + p->noise;
    }
  }
  if (cg_iters_out) *cg_iters_out = total_iters;
  return provider_check_device_error(p);
}

}  // extern "C"
