// Linear model of coregionalisation (LMC), matrix-free:
//   K_full = sum_s (A_s (x) K_s) + diag(noise_t (x) 1_n)
// over task-blocked vectors (element (t, i) at t * n + i), R latent providers
// sharing the inputs X.
//
// References (MojoGP 0.26.6.0): JITLMCGradientAdapter.forward_matvec
// (kernels/jit/jit_lmc.mojo:275-330), kernel_lmc_accumulate_batched and the
// noise kernels (kernels/lmc_provider.mojo:113-192), A_s / noise gradients
// (jit_lmc.mojo:582-691). B200 changes: each latent applies K_s to all
// T * t task-column blocks in one tiled matvec; the A_s mixing and the noise
// term are one fused pass; kernel-parameter gradients use the fused bilinear
// reduction with b = (A_s (x) I) w, and the A_s / noise gradients are batched
// column dot products instead of per-dot host round trips.
#include <cmath>
#include <vector>

#include "engine.cuh"
#include "numerics.h"
#include "train.cuh"

namespace gpb {

// out[c][t][i] (+)= sum_j A[t][j] kv[c][j][i]  (+ noise[t] v[c][t][i] when v != null)
__global__ void lmc_mix_kernel(float* __restrict__ out, const float* __restrict__ kv,
                               const float* __restrict__ A, int T, int64_t n, int cols,
                               int accumulate, const float* __restrict__ noise,
                               const float* __restrict__ v) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nT = (int64_t)T * n;
  if (idx >= (int64_t)cols * nT) return;
  const int64_t c = idx / nT;
  const int64_t rem = idx - c * nT;
  const int t = (int)(rem / n);
  const int64_t i = rem - (int64_t)t * n;
  float s = accumulate ? out[idx] : 0.f;
  const float* kc = kv + c * nT + i;
  for (int j = 0; j < T; ++j) s = fmaf(A[t * T + j], kc[(int64_t)j * n], s);
  if (v) s = fmaf(noise[t], v[idx], s);
  out[idx] = s;
}

struct LmcOp : LinOp {
  std::vector<gpb_provider*> prov;
  int R = 0, T = 0;
  int64_t n = 0;
  std::vector<float> A, noise;  // host copies
  DBuf A_d, noise_d, tmp;
  Engine E;                     // persistent engine over nT rows
  BBMMState S;                  // persistent CG state (warm starts)

  int upload() {
    GPB_TRY(A_d.ensure(A.size() * sizeof(float)));
    GPB_TRY(noise_d.ensure(noise.size() * sizeof(float)));
    GPB_CHECK_CUDA(cudaMemcpyAsync(A_d.ptr, A.data(), A.size() * sizeof(float),
                                   cudaMemcpyHostToDevice, E.st));
    GPB_CHECK_CUDA(cudaMemcpyAsync(noise_d.ptr, noise.data(), noise.size() * sizeof(float),
                                   cudaMemcpyHostToDevice, E.st));
    return GPB_OK;
  }

  // kv_s = K_s v for `cols` task-blocked columns (no noise), v [cols][T][n].
  int latent_kv(int s, const float* v, int cols, float* out, cudaStream_t st) {
    gpb_provider* p = prov[s];
    if (p->xs_dirty) {
      GPB_TRY(provider_refresh_xs(p));
      GPB_CHECK_CUDA(cudaStreamSynchronize(p->stream));
    }
    return provider_kv(p, p->Xs_d, n, v, n, (int64_t)cols * T, out, n, false, 0, st);
  }

  int apply(const float* v, int64_t ld, int t, float* out, cudaStream_t st) override {
    const int64_t total = (int64_t)t * T * n;
    GPB_TRY(tmp.ensure((size_t)total * sizeof(float)));
    for (int s = 0; s < R; ++s) {
      GPB_TRY(latent_kv(s, v, t, tmp.f(), st));
      lmc_mix_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(
          out, tmp.f(), A_d.f() + (size_t)s * T * T, T, n, t, s > 0 ? 1 : 0, noise_d.f(),
          s == R - 1 ? v : nullptr);
      GPB_CHECK_CUDA(cudaGetLastError());
    }
    return GPB_OK;
  }
};

// Gradients of the LMC NLL (per nT, as the reference normalises):
//   kernel params of latent s: (-1/2 a^T (A_s (x) dK_s) a + 1/2 mean_k u_k^T (A_s (x) dK_s) w_k) / nT
//   A_s[i][j]:                 1/2 (-a_i^T K_s a_j + mean_k u_{k,i}^T K_s w_{k,j}) / nT
//   noise_t:                   1/2 (-a_t^T a_t + mean_k u_{k,t}^T w_{k,t}) / nT
// with a = alpha, u_k = probe solutions (scaled), w_k = unnormalised probes.
int lmc_bbmm_gradients(Engine& E, BBMMState& S, float* sol, const float* sampled, int num_probes,
                       BBMMResult& R) {
  LmcOp* op = static_cast<LmcOp*>(E.op);
  const int T = op->T, Rl = op->R;
  const int64_t n = op->n, nT = (int64_t)T * n;
  const int K = 1 + num_probes;  // column blocks: 0 = alpha, k >= 1 = probes
  cudaStream_t st = E.st;
  // Wf = [alpha | w_1 .. w_np] (task-blocked columns of length nT)
  GPB_TRY(S.bfull.ensure((size_t)K * nT * sizeof(float)));
  float* Wf = S.bfull.f();
  GPB_TRY(k_copy(Wf, sol, nT, st));
  GPB_TRY(k_copy(Wf + nT, sampled, (int64_t)num_probes * nT, st));
  DBuf kw, aw;
  GPB_TRY(kw.ensure((size_t)K * nT * sizeof(float)));
  GPB_TRY(aw.ensure((size_t)K * nT * sizeof(float)));
  const double dnT = (double)nT;
  R.grad_A.assign((size_t)Rl * T * T, 0.0);
  std::vector<double> kgrads;
  for (int s = 0; s < Rl; ++s) {
    gpb_provider* p = op->prov[s];
    // A_s gradients from K_s Wf.
    GPB_TRY(op->latent_kv(s, Wf, K, kw.f(), st));
    for (int i = 0; i < T; ++i)
      for (int j = 0; j < T; ++j) {
        const float* a[1] = {sol + (int64_t)i * n};
        const float* b[1] = {kw.f() + (int64_t)j * n};
        // K columns with stride nT: column k = block k of task i / j
        GPB_TRY(k_coldots(1, a, b, nT, n, K, E.red, st));
        std::vector<double> h(K);
        GPB_CHECK_CUDA(cudaMemcpyAsync(h.data(), E.red.sums.ptr, K * sizeof(double),
                                       cudaMemcpyDeviceToHost, st));
        GPB_CHECK_CUDA(cudaStreamSynchronize(st));
        double tr = 0.0;
        for (int k = 1; k < K; ++k) tr += h[k];
        R.grad_A[((size_t)s * T + i) * T + j] = 0.5 * (-h[0] + tr / num_probes) / dnT;
      }
    // Kernel-parameter gradients: b = (A_s (x) I) Wf.
    const int64_t total = (int64_t)K * nT;
    lmc_mix_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(
        aw.f(), Wf, op->A_d.f() + (size_t)s * T * T, T, n, K, 0, nullptr, nullptr);
    GPB_CHECK_CUDA(cudaGetLastError());
    const int P = p->dk.nparams;
    std::vector<double> data(P), trace(P);
    GPB_TRY(provider_bilinear_rows_nd(p, sol, n, aw.f(), (int64_t)K * T, 0, n, T, data.data(),
                                      trace.data(), st));
    for (int q = 0; q < P; ++q) {
      double g = (-0.5 * data[q] + 0.5 * trace[q] / num_probes) / dnT;
      if (!std::isfinite(g)) g = 0.0;
      kgrads.push_back(g);
    }
  }
  // Noise gradients per task and sum(alpha) per task.
  R.grad_noise_task.assign(T, 0.0);
  R.sum_alpha_task.assign(T, 0.0);
  for (int t = 0; t < T; ++t) {
    const float* a[2] = {sol + (int64_t)t * n, sol + (int64_t)t * n};
    const float* b[2] = {Wf + (int64_t)t * n, S.ones.f()};
    GPB_TRY(k_coldots(1, a, b, nT, n, K, E.red, st));
    std::vector<double> h(K);
    GPB_CHECK_CUDA(cudaMemcpyAsync(h.data(), E.red.sums.ptr, K * sizeof(double),
                                   cudaMemcpyDeviceToHost, st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(st));
    double tr = 0.0;
    for (int k = 1; k < K; ++k) tr += h[k];
    R.grad_noise_task[t] = 0.5 * (-h[0] + tr / num_probes) / dnT;
    const float* a1[1] = {sol + (int64_t)t * n};
    const float* b1[1] = {S.ones.f()};
    GPB_TRY(k_coldots(1, a1, b1, n, n, 1, E.red, st));
    double sa = 0.0;
    GPB_CHECK_CUDA(cudaMemcpyAsync(&sa, E.red.sums.ptr, sizeof(double), cudaMemcpyDeviceToHost, st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(st));
    R.sum_alpha_task[t] = sa;
  }
  R.grads = kgrads;
  return GPB_OK;
}

}  // namespace gpb

using namespace gpb;

struct gpb_lmc {
  LmcOp op;
};

extern "C" {

int gpb_lmc_create(gpb_provider* const* providers, int32_t num_latents, int32_t num_tasks,
                   gpb_lmc** out) {
  clear_error();
  GPB_REQUIRE(providers && out && num_latents >= 1 && num_tasks >= 1, GPB_ERR_INVALID,
              "bad LMC arguments");
  const int64_t n = providers[0]->n;
  for (int s = 0; s < num_latents; ++s) {
    GPB_REQUIRE(providers[s] && providers[s]->n == n && providers[s]->device == providers[0]->device,
                GPB_ERR_INVALID, "LMC latent providers must share n and device");
  }
  GPB_CHECK_CUDA(cudaSetDevice(providers[0]->device));
  gpb_lmc* h = new gpb_lmc();
  LmcOp& op = h->op;
  op.prov.assign(providers, providers + num_latents);
  op.R = num_latents;
  op.T = num_tasks;
  op.n = n;
  op.A.assign((size_t)num_latents * num_tasks * num_tasks, 0.f);
  for (int s = 0; s < num_latents; ++s)
    for (int t = 0; t < num_tasks; ++t) op.A[((size_t)s * num_tasks + t) * num_tasks + t] = 1.f;
  op.noise.assign(num_tasks, 0.1f);
  op.E.p = providers[0];
  op.E.op = &op;
  op.E.st = providers[0]->stream;
  op.E.n = op.E.nl = n * num_tasks;
  op.E.r0 = 0;
  op.E.r1 = op.E.n;
  op.E.nl_pad = op.E.n;
  int s = op.upload();
  if (s != GPB_OK) {
    delete h;
    return s;
  }
  *out = h;
  return GPB_OK;
}

int gpb_lmc_destroy(gpb_lmc* h) {
  if (!h) return GPB_OK;
  cudaSetDevice(h->op.prov[0]->device);
  cudaStreamSynchronize(h->op.E.st);
  delete h;
  return GPB_OK;
}

int gpb_lmc_set_coregion(gpb_lmc* h, const float* A, const float* noise) {
  GPB_REQUIRE(h && A && noise, GPB_ERR_INVALID, "null argument");
  LmcOp& op = h->op;
  op.A.assign(A, A + op.A.size());
  op.noise.assign(noise, noise + op.T);
  for (float v : op.noise) GPB_REQUIRE(v >= 0.f && std::isfinite(v), GPB_ERR_INVALID, "bad noise");
  GPB_CHECK_CUDA(cudaSetDevice(op.prov[0]->device));
  return op.upload();
}

int gpb_lmc_matvec(gpb_lmc* h, float* out_dev, const float* v_dev, int64_t ncols) {
  GPB_REQUIRE(h && out_dev && v_dev && ncols >= 0, GPB_ERR_INVALID, "bad arguments");
  GPB_CHECK_CUDA(cudaSetDevice(h->op.prov[0]->device));
  if (ncols == 0) return GPB_OK;
  GPB_TRY(h->op.apply(v_dev, h->op.E.n, (int)ncols, out_dev, h->op.E.st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(h->op.E.st));
  return provider_check_device_error(h->op.prov[0]);
}

int gpb_lmc_bbmm(gpb_lmc* h, const float* y_centered_host, int32_t num_probes, int32_t max_cg_iter,
                 int32_t max_tridiag_iter, float cg_tol, int32_t iteration, int32_t recycle,
                 double* nll_out, double* kernel_grads_out, double* grad_A_out,
                 double* grad_noise_out, double* sum_alpha_out, float* alpha_out,
                 int32_t* cg_iters_out) {
  clear_error();
  GPB_REQUIRE(h && y_centered_host && nll_out && kernel_grads_out && grad_A_out &&
                  grad_noise_out && sum_alpha_out && num_probes >= 1,
              GPB_ERR_INVALID, "null argument");
  LmcOp& op = h->op;
  GPB_CHECK_CUDA(cudaSetDevice(op.prov[0]->device));
  Engine& E = op.E;
  GPB_TRY(op.S.ensure(E, 1 + num_probes, max_tridiag_iter));
  GPB_CHECK_CUDA(cudaMemcpyAsync(op.S.yc.ptr, y_centered_host, E.n * sizeof(float),
                                 cudaMemcpyHostToDevice, E.st));
  BBMMResult R;
  GPB_TRY(bbmm_step(E, nullptr, op.S, num_probes, max_cg_iter, max_tridiag_iter, cg_tol, iteration,
                    recycle != 0, R));
  *nll_out = R.nll;
  for (size_t q = 0; q < R.grads.size(); ++q) kernel_grads_out[q] = R.grads[q];
  for (size_t q = 0; q < R.grad_A.size(); ++q) grad_A_out[q] = R.grad_A[q];
  for (int t = 0; t < op.T; ++t) {
    grad_noise_out[t] = R.grad_noise_task[t];
    sum_alpha_out[t] = R.sum_alpha_task[t];
  }
  if (alpha_out) {
    GPB_CHECK_CUDA(cudaMemcpyAsync(alpha_out, op.S.sol.ptr, E.n * sizeof(float),
                                   cudaMemcpyDeviceToHost, E.st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(E.st));
  }
  if (cg_iters_out) *cg_iters_out = R.cg_iters;
  return provider_check_device_error(op.prov[0]);
}

int gpb_lmc_solve(gpb_lmc* h, const float* rhs_host, int32_t max_cg_iter, float cg_tol,
                  float* x_host_out, int32_t* iters_out) {
  GPB_REQUIRE(h && rhs_host && x_host_out, GPB_ERR_INVALID, "null argument");
  LmcOp& op = h->op;
  GPB_CHECK_CUDA(cudaSetDevice(op.prov[0]->device));
  Engine& E = op.E;
  DBuf y, x;
  GPB_TRY(y.ensure((size_t)E.n * sizeof(float)));
  GPB_TRY(x.ensure((size_t)E.n * sizeof(float)));
  GPB_CHECK_CUDA(cudaMemcpyAsync(y.ptr, rhs_host, E.n * sizeof(float), cudaMemcpyHostToDevice, E.st));
  int it = 0;
  GPB_TRY(alpha_cg(E, y.f(), x.f(), max_cg_iter, cg_tol, &it));
  GPB_CHECK_CUDA(cudaMemcpyAsync(x_host_out, x.ptr, E.n * sizeof(float), cudaMemcpyDeviceToHost, E.st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(E.st));
  if (iters_out) *iters_out = it;
  return provider_check_device_error(op.prov[0]);
}

}  // extern "C"
