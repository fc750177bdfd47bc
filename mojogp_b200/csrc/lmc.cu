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

struct gpb_comm;  // defined in train.cu

namespace gpb {

int engine_from_comm(gpb_provider* p, gpb_comm* c, Engine& E);

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

// ---------------------------------------------------------- preconditioner
// Sum-of-Kronecker Woodbury preconditioner (kernels/lmc_preconditioner.mojo:
// 143-470, built as in jit_lmc.mojo:848-900, 1047-1100):
//   P = sum_s (C_s (x) L_s)(C_s (x) L_s)^T + D = sum_s A_s (x) L_s L_s^T + D,
// with L_s the rank-r_s greedy pivoted-Cholesky factor of K_s (no noise),
// C_s = chol(A_s) and D = diag(noise_t (x) 1_n). With U = [C_s (x) L_s]_s and
// M = I + U^T D^{-1} U (order (s, j, k) -> off_s + j r_s + k):
//   P^{-1} v = D^{-1} v - D^{-1} U M^{-1} U^T D^{-1} v,
//   log|P|   = n sum_t log noise_t + log|M|,
//   z ~ N(0, P): z = D^{1/2} eps + U omega.
// B200 changes: M^{-1} (fp64) lives on the device and every step of an apply
// is a batched kernel over all columns, latents and tasks (no host round trip
// per column / latent / task); probes use the library's counter-hash Gaussian
// (seeds `seed` for omega, `seed + 1e6` for eps) instead of a host generator.
// y_s[j][k] = sum_t C_s[t][j] Z_s[c][t][k]; z = Minv y; u_s[c][t][k] = scale_t *
// sum_j C_s[t][j] z_s[j][k]. One block per column c. With `omega` set, z is
// read from omega[c][Kt] instead (probe sampling: no Z, no Minv).
__global__ void lmc_pc_small_kernel(const double* __restrict__ Z, const float* __restrict__ C,
                                    const double* __restrict__ Minv, const float* __restrict__ omega,
                                    const int* __restrict__ rank, const int* __restrict__ off,
                                    int R, int T, int Kt, const float* __restrict__ scale,
                                    float* __restrict__ u) {
  extern __shared__ double sh[];
  double* y = sh;
  double* z = sh + Kt;
  const int c = blockIdx.x;
  // Z and u: latent s occupies [cols * T][r_s] starting at off_s * cols.
  const int cols = gridDim.x;
  if (omega) {
    for (int q = threadIdx.x; q < Kt; q += blockDim.x) z[q] = omega[(int64_t)c * Kt + q];
  } else {
    for (int q = threadIdx.x; q < Kt; q += blockDim.x) {
      int s = 0;
      while (s + 1 < R && off[s + 1] <= q) ++s;
      const int rs = rank[s], loc = q - off[s];
      const int j = loc / rs, k = loc % rs;
      const double* Zs = Z + (int64_t)off[s] * cols;
      double acc = 0.0;
      for (int t = 0; t < T; ++t)
        acc += (double)C[((size_t)s * T + t) * T + j] * Zs[((int64_t)c * T + t) * rs + k];
      y[q] = acc;
    }
    __syncthreads();
    for (int q = threadIdx.x; q < Kt; q += blockDim.x) {
      double acc = 0.0;
      const double* row = Minv + (int64_t)q * Kt;
      for (int q2 = 0; q2 < Kt; ++q2) acc += row[q2] * y[q2];
      z[q] = acc;
    }
  }
  __syncthreads();
  // u_s laid out like Z_s: u[(off_s * cols) + (c * T + t) * r_s + k].
  for (int q = threadIdx.x; q < Kt; q += blockDim.x) {
    int s = 0;
    while (s + 1 < R && off[s + 1] <= q) ++s;
    const int rs = rank[s], loc = q - off[s];
    const int t = loc / rs, k = loc % rs;  // reuse (j, k) indexing with j -> t
    double acc = 0.0;
    for (int j = 0; j < T; ++j)
      acc += (double)C[((size_t)s * T + t) * T + j] * z[off[s] + j * rs + k];
    u[(int64_t)off[s] * cols + ((int64_t)c * T + t) * rs + k] = (float)(scale[t] * acc);
  }
}

// out[c][t][i] = scale[t] * v[c][t][i]
__global__ void lmc_task_scale_kernel(float* __restrict__ out, const float* __restrict__ v,
                                      const float* __restrict__ scale, int T, int64_t n,
                                      int64_t total) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int t = (int)((idx / n) % T);
  out[idx] = scale[t] * v[idx];
}

struct LmcPrecond {
  int R = 0, T = 0, Kt = 0;
  int64_t n = 0;            // data rows (global)
  int64_t nl = 0, r0 = 0;   // this rank's data rows [r0, r0 + nl)
  std::vector<int> rank, off;       // per latent
  std::vector<Precond> pc;          // per latent: L_s
  std::vector<float> C;             // [R][T][T] row-major lower Cholesky of A_s
  std::vector<float> noise;         // [T]
  double logdet = 0.0;
  DBuf C_d, dinv_d, dsqrt_d, ones_d, Minv_d, rank_d, off_d, Z_d, u_d, w_d, omega_d;
  // Columns per batched pass: L^T v shared memory (t (128 + r) floats) and
  // L u shared memory (t r floats, 48 KB default) bound it.
  int group_cols(int cols) const {
    int rmax = 1;
    for (int r : rank) rmax = std::max(rmax, r);
    int g = std::min(190 * 1024 / (4 * T * (128 + rmax)), 12000 / (T * rmax));
    return std::max(1, std::min(cols, g));
  }
};

int lmc_precond_apply(Engine& E, LmcPrecond& P, const float* v, float* out, int t) {
  const int64_t nT = (int64_t)P.T * P.nl, cnt = (int64_t)t * nT;
  cudaStream_t st = E.st;
  GPB_TRY(P.w_d.ensure((size_t)std::max<int64_t>(cnt, 1) * sizeof(float)));
  float* w = P.w_d.f();
  lmc_task_scale_kernel<<<(unsigned)ceil_div(std::max<int64_t>(cnt, 1), 256), 256, 0, st>>>(
      w, v, P.dinv_d.f(), P.T, std::max<int64_t>(P.nl, 1), cnt);
  GPB_CHECK_CUDA(cudaGetLastError());
  const int gmax = P.group_cols(t);
  GPB_TRY(P.Z_d.ensure((size_t)gmax * P.Kt * sizeof(double)));
  GPB_TRY(P.u_d.ensure((size_t)gmax * P.Kt * sizeof(float)));
  for (int c0 = 0; c0 < t; c0 += gmax) {
    const int g = std::min(gmax, t - c0);
    const float* wg = w + (int64_t)c0 * nT;
    float* og = out + (int64_t)c0 * nT;
    for (int s = 0; s < P.R; ++s) {
      GPB_TRY(k_ltv(P.pc[s].L.f(), P.nl, P.rank[s], wg, P.nl, g * P.T, E.red, st));
      GPB_TRY(E.allreduce_sum(E.red.sums.d(), (size_t)g * P.T * P.rank[s]));
      GPB_CHECK_CUDA(cudaMemcpyAsync(P.Z_d.d() + (int64_t)P.off[s] * g, E.red.sums.ptr,
                                     (size_t)g * P.T * P.rank[s] * sizeof(double),
                                     cudaMemcpyDeviceToDevice, st));
    }
    lmc_pc_small_kernel<<<g, 256, 2 * (size_t)P.Kt * sizeof(double), st>>>(
        P.Z_d.d(), P.C_d.f(), P.Minv_d.d(), nullptr, (const int*)P.rank_d.ptr,
        (const int*)P.off_d.ptr, P.R, P.T, P.Kt, P.dinv_d.f(), P.u_d.f());
    GPB_CHECK_CUDA(cudaGetLastError());
    for (int s = 0; s < P.R; ++s)
      GPB_TRY(k_l_times_u(P.pc[s].L.f(), P.nl, P.rank[s], P.u_d.f() + (int64_t)P.off[s] * g,
                          g * P.T, s == 0 ? wg : og, P.nl, 1.f, -1.f, og, st));
  }
  E.p->launches += 1 + (int64_t)((t + gmax - 1) / gmax) * (2 * P.R + 1);
  return GPB_OK;
}

int lmc_precond_sample(Engine& E, LmcPrecond& P, int num, uint64_t seed, float* out) {
  const int64_t nT = (int64_t)P.T * P.nl, cnt = (int64_t)num * nT;
  cudaStream_t st = E.st;
  GPB_TRY(k_gaussian_tasks(out, num, P.T, P.nl, P.n, P.r0, seed + 1000000ull, st));
  if (cnt > 0) {
    lmc_task_scale_kernel<<<(unsigned)ceil_div(cnt, 256), 256, 0, st>>>(out, out, P.dsqrt_d.f(),
                                                                       P.T, P.nl, cnt);
    GPB_CHECK_CUDA(cudaGetLastError());
  }
  GPB_CHECK_CUDA(cudaGetLastError());
  GPB_TRY(P.omega_d.ensure((size_t)num * P.Kt * sizeof(float)));
  const int64_t no = (int64_t)num * P.Kt;
  GPB_TRY(k_gaussian(P.omega_d.f(), 1, no, no, no, 0, seed, st));
  const int gmax = P.group_cols(num);
  GPB_TRY(P.u_d.ensure((size_t)gmax * P.Kt * sizeof(float)));
  for (int c0 = 0; c0 < num; c0 += gmax) {
    const int g = std::min(gmax, num - c0);
    float* og = out + (int64_t)c0 * nT;
    lmc_pc_small_kernel<<<g, 256, 2 * (size_t)P.Kt * sizeof(double), st>>>(
        nullptr, P.C_d.f(), nullptr, P.omega_d.f() + (int64_t)c0 * P.Kt, (const int*)P.rank_d.ptr,
        (const int*)P.off_d.ptr, P.R, P.T, P.Kt, P.ones_d.f(), P.u_d.f());
    GPB_CHECK_CUDA(cudaGetLastError());
    for (int s = 0; s < P.R; ++s)
      GPB_TRY(k_l_times_u(P.pc[s].L.f(), P.nl, P.rank[s], P.u_d.f() + (int64_t)P.off[s] * g,
                          g * P.T, og, P.nl, 1.f, 1.f, og, st));
  }
  return GPB_OK;
}


struct LmcOp : LinOp {
  std::vector<gpb_provider*> prov;
  int R = 0, T = 0;
  int64_t n = 0;                // data rows (global)
  int64_t nl = 0, r0 = 0;       // this rank's data rows [r0, r0 + nl); all tasks of a row
  std::vector<float> A, noise;  // host copies
  DBuf A_d, noise_d, tmp, vfull;
  Engine Ed;                    // data-row engine (row split, all-gather of columns)
  Engine E;                     // operator engine over the local [T][nl] task blocks
  BBMMState S;                  // persistent CG state (warm starts)
  Precond pc;                   // rank > 0: the LMC preconditioner below is active
  LmcPrecond lp;

  int upload() {
    GPB_TRY(A_d.ensure(A.size() * sizeof(float)));
    GPB_TRY(noise_d.ensure(noise.size() * sizeof(float)));
    GPB_CHECK_CUDA(cudaMemcpyAsync(A_d.ptr, A.data(), A.size() * sizeof(float),
                                   cudaMemcpyHostToDevice, E.st));
    GPB_CHECK_CUDA(cudaMemcpyAsync(noise_d.ptr, noise.data(), noise.size() * sizeof(float),
                                   cudaMemcpyHostToDevice, E.st));
    return GPB_OK;
  }

  // Full task-blocked columns [cols][T][n] from local blocks [cols][T][nl].
  int gather(const float* v_local, int cols, const float** full) {
    if (Ed.dist.world == 1) {
      *full = v_local;
      return GPB_OK;
    }
    GPB_TRY(vfull.ensure((size_t)cols * T * n * sizeof(float)));
    GPB_TRY(Ed.allgather_cols(v_local, nl, cols * T, vfull.f()));
    *full = vfull.f();
    return GPB_OK;
  }

  // out_local [cols][T][nl] = K_s(X_local, X) v_full (no noise), v_full [cols][T][n].
  int latent_kv_full(int s, const float* v_full, int cols, float* out, cudaStream_t st) {
    gpb_provider* p = prov[s];
    if (p->xs_dirty) {
      GPB_TRY(provider_refresh_xs(p));
      GPB_CHECK_CUDA(cudaStreamSynchronize(p->stream));
    }
    return provider_kv(p, p->Xs_d + r0 * p->DP, nl, v_full, n, (int64_t)cols * T, out, nl, false,
                       0, st);
  }

  // Same from local blocks.
  int latent_kv(int s, const float* v_local, int cols, float* out, cudaStream_t st) {
    const float* vf = nullptr;
    GPB_TRY(gather(v_local, cols, &vf));
    return latent_kv_full(s, vf, cols, out, st);
  }

  int apply(const float* v, int64_t ld, int t, float* out, cudaStream_t st) override {
    const int64_t total = (int64_t)t * T * nl;
    if (total == 0) return GPB_OK;
    GPB_TRY(tmp.ensure((size_t)total * sizeof(float)));
    const float* vf = nullptr;
    GPB_TRY(gather(v, t, &vf));
    for (int s = 0; s < R; ++s) {
      GPB_TRY(latent_kv_full(s, vf, t, tmp.f(), st));
      lmc_mix_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(
          out, tmp.f(), A_d.f() + (size_t)s * T * T, T, nl, t, s > 0 ? 1 : 0, noise_d.f(),
          s == R - 1 ? v : nullptr);
      GPB_CHECK_CUDA(cudaGetLastError());
    }
    return GPB_OK;
  }

  // Host [T][n] -> this rank's local block [T][nl].
  int to_local(const float* host, float* local) {
    for (int t = 0; t < T && nl > 0; ++t)
      GPB_CHECK_CUDA(cudaMemcpyAsync(local + (int64_t)t * nl, host + (int64_t)t * n + r0,
                                     nl * sizeof(float), cudaMemcpyHostToDevice, E.st));
    return GPB_OK;
  }
  // Local block [T][nl] -> host [T][n] (gathered over the ranks).
  int to_host(const float* local, float* host) {
    const float* full = nullptr;
    GPB_TRY(gather(local, 1, &full));
    GPB_CHECK_CUDA(cudaMemcpyAsync(host, full, (size_t)T * n * sizeof(float), cudaMemcpyDeviceToHost,
                                   E.st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(E.st));
    return GPB_OK;
  }

  int gaussian(float* out, int t, uint64_t seed, cudaStream_t st) override {
    return k_gaussian_tasks(out, t, T, nl, n, r0, seed, st);
  }
};



// Builds P from the current A_s, noise_t and latent kernels (rank_req <= 0 clears it).
int lmc_build_precond(LmcOp& op, int rank_req) {
  op.pc.rank = 0;
  op.pc.lmc = nullptr;
  op.pc.logdet = 0.0;
  if (rank_req <= 0) return GPB_OK;
  LmcPrecond& P = op.lp;
  const int R = op.R, T = op.T;
  const int64_t n = op.n;
  P.R = R;
  P.T = T;
  P.n = n;
  P.nl = op.nl;
  P.r0 = op.r0;
  P.pc.assign(R, Precond());
  P.rank.assign(R, 0);
  P.off.assign(R, 0);
  cudaStream_t st = op.E.st;
  // 1. Per-latent factors L_s of K_s (no noise).
  for (int s = 0; s < R; ++s) {
    Engine Es;
    GPB_TRY(Es.init(op.prov[s], op.Ed.dist));
    Es.st = st;
    GPB_TRY(precond_build(Es, rank_req, P.pc[s], false));
    P.rank[s] = P.pc[s].rank;
  }
  int Kt = 0;
  for (int s = 0; s < R; ++s) {
    P.off[s] = Kt;
    Kt += T * P.rank[s];
  }
  GPB_REQUIRE(Kt <= 3072, GPB_ERR_UNSUPPORTED,
              "LMC preconditioner: latents x tasks x rank = %d exceeds 3072", Kt);
  P.Kt = Kt;
  // 2. C_s = chol(A_s) (1e-4 diagonal jitter if A_s is not positive definite).
  P.C.assign((size_t)R * T * T, 0.f);
  for (int s = 0; s < R; ++s) {
    std::vector<double> A((size_t)T * T), Lo((size_t)T * T);
    for (int q = 0; q < T * T; ++q) A[q] = op.A[(size_t)s * T * T + q];
    if (!cholesky_lower(A.data(), T, Lo.data())) {
      for (int i = 0; i < T; ++i) A[(size_t)i * T + i] += 1e-4;
      GPB_REQUIRE(cholesky_lower(A.data(), T, Lo.data()), GPB_ERR_NUMERIC,
                  "LMC preconditioner: A_%d is not positive definite", s);
    }
    for (int q = 0; q < T * T; ++q) P.C[(size_t)s * T * T + q] = (float)Lo[q];
  }
  P.noise.assign(op.noise.begin(), op.noise.end());
  for (float v : P.noise)
    GPB_REQUIRE(v > 0.f, GPB_ERR_INVALID, "LMC preconditioner needs positive task noise");
  // 3. M = I + sum_{s1,s2} (C_s1^T D^{-1} C_s2) (x) (L_s1^T L_s2).
  std::vector<double> M((size_t)Kt * Kt, 0.0);
  for (int q = 0; q < Kt; ++q) M[(size_t)q * Kt + q] = 1.0;
  for (int s1 = 0; s1 < R; ++s1)
    for (int s2 = 0; s2 < R; ++s2) {
      const int r1 = P.rank[s1], r2 = P.rank[s2];
      GPB_TRY(k_ltv(P.pc[s1].L.f(), P.nl, r1, P.pc[s2].L.f(), P.nl, r2, op.E.red, st));
      GPB_TRY(op.E.allreduce_sum(op.E.red.sums.d(), (size_t)r1 * r2));
      std::vector<double> ltl((size_t)r1 * r2);  // ltl[c * r1 + k] = (L_s1^T L_s2)[k][c]
      GPB_CHECK_CUDA(cudaMemcpyAsync(ltl.data(), op.E.red.sums.ptr, ltl.size() * sizeof(double),
                                     cudaMemcpyDeviceToHost, st));
      GPB_CHECK_CUDA(cudaStreamSynchronize(st));
      for (int j1 = 0; j1 < T; ++j1)
        for (int j2 = 0; j2 < T; ++j2) {
          double g = 0.0;
          for (int t = 0; t < T; ++t)
            g += (double)P.C[((size_t)s1 * T + t) * T + j1] * P.C[((size_t)s2 * T + t) * T + j2] /
                 (double)P.noise[t];
          if (g == 0.0) continue;
          for (int k1 = 0; k1 < r1; ++k1)
            for (int k2 = 0; k2 < r2; ++k2)
              M[(size_t)(P.off[s1] + j1 * r1 + k1) * Kt + P.off[s2] + j2 * r2 + k2] +=
                  g * ltl[(size_t)k2 * r1 + k1];
        }
    }
  std::vector<double> Minv((size_t)Kt * Kt);
  double ldM = 0.0;
  GPB_REQUIRE(spd_inverse(M.data(), Kt, Minv.data(), &ldM), GPB_ERR_NUMERIC,
              "LMC preconditioner: I + U^T D^-1 U is not positive definite");
  P.logdet = ldM;
  for (int t = 0; t < T; ++t) P.logdet += (double)n * std::log((double)P.noise[t]);
  // 4. Device copies.
  std::vector<float> dinv(T), dsqrt(T), ones(T, 1.f);
  for (int t = 0; t < T; ++t) {
    dinv[t] = 1.f / P.noise[t];
    dsqrt[t] = std::sqrt(P.noise[t]);
  }
  auto up = [&](DBuf& b, const void* src, size_t bytes) -> int {
    GPB_TRY(b.ensure(bytes));
    GPB_CHECK_CUDA(cudaMemcpyAsync(b.ptr, src, bytes, cudaMemcpyHostToDevice, st));
    return GPB_OK;
  };
  GPB_TRY(up(P.C_d, P.C.data(), P.C.size() * sizeof(float)));
  GPB_TRY(up(P.Minv_d, Minv.data(), Minv.size() * sizeof(double)));
  GPB_TRY(up(P.dinv_d, dinv.data(), T * sizeof(float)));
  GPB_TRY(up(P.dsqrt_d, dsqrt.data(), T * sizeof(float)));
  GPB_TRY(up(P.ones_d, ones.data(), T * sizeof(float)));
  GPB_TRY(up(P.rank_d, P.rank.data(), R * sizeof(int)));
  GPB_TRY(up(P.off_d, P.off.data(), R * sizeof(int)));
  GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  op.pc.rank = Kt;
  op.pc.logdet = P.logdet;
  op.pc.lmc = &P;
  return GPB_OK;
}

// Gradients of the LMC NLL (per nT, as the reference normalises):
//   kernel params of latent s: (-1/2 a^T (A_s (x) dK_s) a + 1/2 mean_k u_k^T (A_s (x) dK_s) w_k) / nT
//   A_s[i][j]:                 1/2 (-a_i^T K_s a_j + mean_k u_{k,i}^T K_s w_{k,j}) / nT
//   noise_t:                   1/2 (-a_t^T a_t + mean_k u_{k,t}^T w_{k,t}) / nT
// with a = alpha, u_k = probe solutions (scaled), w_k = P^{-1} z_k (the unnormalised
// probes z_k themselves when there is no preconditioner).
int lmc_bbmm_gradients(Engine& E, BBMMState& S, float* sol, const float* rf, int num_probes,
                       BBMMResult& R) {
  LmcOp* op = static_cast<LmcOp*>(E.op);
  const int T = op->T, Rl = op->R;
  const int64_t nl = op->nl, nTl = (int64_t)T * nl;  // local rows of every task
  const int K = 1 + num_probes;  // column blocks: 0 = alpha, k >= 1 = probes
  cudaStream_t st = E.st;
  // Local dots over this rank's rows, summed over the ranks, to the host.
  auto dots = [&](const float* a, const float* b, int64_t ld, int cols, std::vector<double>& h) {
    const float* pa[1] = {a};
    const float* pb[1] = {b};
    GPB_TRY(k_coldots(1, pa, pb, ld, nl, cols, E.red, st));
    GPB_TRY(E.allreduce_sum(E.red.sums.d(), (size_t)cols));
    h.resize(cols);
    GPB_CHECK_CUDA(cudaMemcpyAsync(h.data(), E.red.sums.ptr, cols * sizeof(double),
                                   cudaMemcpyDeviceToHost, st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(st));
    return GPB_OK;
  };
  // Wf = [alpha | w_1 .. w_np] (local task-blocked columns of length T * nl)
  GPB_TRY(S.bfull.ensure((size_t)std::max<int64_t>(K * nTl, 1) * sizeof(float)));
  float* Wf = S.bfull.f();
  GPB_TRY(k_copy(Wf, sol, nTl, st));
  GPB_TRY(k_copy(Wf + nTl, rf, (int64_t)num_probes * nTl, st));
  DBuf kw, aw, awfull;
  GPB_TRY(kw.ensure((size_t)std::max<int64_t>(K * nTl, 1) * sizeof(float)));
  GPB_TRY(aw.ensure((size_t)std::max<int64_t>(K * nTl, 1) * sizeof(float)));
  const double dnT = (double)T * op->n;
  R.grad_A.assign((size_t)Rl * T * T, 0.0);
  std::vector<double> kgrads, h;
  for (int s = 0; s < Rl; ++s) {
    gpb_provider* p = op->prov[s];
    // A_s gradients from K_s Wf.
    GPB_TRY(op->latent_kv(s, Wf, K, kw.f(), st));
    for (int i = 0; i < T; ++i)
      for (int j = 0; j < T; ++j) {
        // K columns with stride T * nl: column k = block k of task i / j
        GPB_TRY(dots(sol + (int64_t)i * nl, kw.f() + (int64_t)j * nl, nTl, K, h));
        double tr = 0.0;
        for (int k = 1; k < K; ++k) tr += h[k];
        R.grad_A[((size_t)s * T + i) * T + j] = 0.5 * (-h[0] + tr / num_probes) / dnT;
      }
    // Kernel-parameter gradients: b = (A_s (x) I) Wf over all rows.
    const int64_t total = (int64_t)K * nTl;
    if (total > 0) {
      lmc_mix_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(
          aw.f(), Wf, op->A_d.f() + (size_t)s * T * T, T, nl, K, 0, nullptr, nullptr);
      GPB_CHECK_CUDA(cudaGetLastError());
    }
    const float* awf = aw.f();
    if (op->Ed.dist.world > 1) {
      GPB_TRY(awfull.ensure((size_t)K * T * op->n * sizeof(float)));
      GPB_TRY(op->Ed.allgather_cols(aw.f(), nl, K * T, awfull.f()));
      awf = awfull.f();
    }
    const int P = p->dk.nparams;
    std::vector<double> both(2 * P, 0.0);
    if (nl > 0)
      GPB_TRY(provider_bilinear_rows_nd(p, sol, nl, awf, (int64_t)K * T, op->r0, op->r0 + nl, T,
                                        both.data(), both.data() + P, st));
    if (op->Ed.dist.world > 1) {
      DBuf gb;
      GPB_TRY(gb.ensure(both.size() * sizeof(double)));
      GPB_CHECK_CUDA(cudaMemcpyAsync(gb.ptr, both.data(), both.size() * sizeof(double),
                                     cudaMemcpyHostToDevice, st));
      GPB_TRY(E.allreduce_sum(gb.d(), both.size()));
      GPB_CHECK_CUDA(cudaMemcpyAsync(both.data(), gb.ptr, both.size() * sizeof(double),
                                     cudaMemcpyDeviceToHost, st));
      GPB_CHECK_CUDA(cudaStreamSynchronize(st));
    }
    for (int q = 0; q < P; ++q) {
      double g = (-0.5 * both[q] + 0.5 * both[P + q] / num_probes) / dnT;
      if (!std::isfinite(g)) g = 0.0;
      kgrads.push_back(g);
    }
  }
  // Noise gradients per task and sum(alpha) per task.
  R.grad_noise_task.assign(T, 0.0);
  R.sum_alpha_task.assign(T, 0.0);
  for (int t = 0; t < T; ++t) {
    GPB_TRY(dots(sol + (int64_t)t * nl, Wf + (int64_t)t * nl, nTl, K, h));
    double tr = 0.0;
    for (int k = 1; k < K; ++k) tr += h[k];
    R.grad_noise_task[t] = 0.5 * (-h[0] + tr / num_probes) / dnT;
    GPB_TRY(dots(sol + (int64_t)t * nl, S.ones.f(), nl, 1, h));
    R.sum_alpha_task[t] = h[0];
  }
  R.grads = kgrads;
  return GPB_OK;
}

// Exact-variance right-hand sides: column (c, t) of a block of b test points
// is sum_s k_s(X, x*_c) (x) A_s[:, t], i.e. rhs[(c T + t)][t'][i] =
// sum_s A_s[t'][t] cross_s[c][i] (cross [R][b][nl], A [R][T][T]).
__global__ void lmc_exact_rhs_kernel(const float* __restrict__ cross,
                                     const float* __restrict__ A, int R, int T, int b,
                                     int64_t nl, float* __restrict__ rhs) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int col = blockIdx.y;  // c * T + t
  const int tp = blockIdx.z;
  if (i >= nl) return;
  const int c = col / T, t = col % T;
  float acc = 0.f;
  for (int s = 0; s < R; ++s)
    acc += A[((size_t)s * T + tp) * T + t] * cross[((int64_t)s * b + c) * nl + i];
  rhs[((int64_t)col * T + tp) * nl + i] = acc;
}

}  // namespace gpb

using namespace gpb;

struct gpb_lmc {
  LmcOp op;
};

extern "C" {

int gpb_lmc_create_sharded(gpb_provider* const* providers, int32_t num_latents,
                           int32_t num_tasks, gpb_comm* comm, gpb_lmc** out) {
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
  int s = engine_from_comm(providers[0], comm, op.Ed);
  if (s != GPB_OK) {
    delete h;
    return s;
  }
  op.prov.assign(providers, providers + num_latents);
  op.R = num_latents;
  op.T = num_tasks;
  op.n = n;
  op.nl = op.Ed.nl;
  op.r0 = op.Ed.r0;
  op.A.assign((size_t)num_latents * num_tasks * num_tasks, 0.f);
  for (int q = 0; q < num_latents; ++q)
    for (int t = 0; t < num_tasks; ++t) op.A[((size_t)q * num_tasks + t) * num_tasks + t] = 1.f;
  op.noise.assign(num_tasks, 0.1f);
  op.E.p = providers[0];
  op.E.op = &op;
  op.E.st = providers[0]->stream;
  op.E.dist = op.Ed.dist;
  op.E.n = n * num_tasks;
  op.E.nl = op.nl * num_tasks;
  op.E.r0 = op.r0 * num_tasks;
  op.E.r1 = op.E.r0 + op.E.nl;
  op.E.nl_pad = std::max<int64_t>(op.E.nl, 1);
  s = op.upload();
  if (s != GPB_OK) {
    delete h;
    return s;
  }
  *out = h;
  return GPB_OK;
}

int gpb_lmc_create(gpb_provider* const* providers, int32_t num_latents, int32_t num_tasks,
                   gpb_lmc** out) {
  return gpb_lmc_create_sharded(providers, num_latents, num_tasks, nullptr, out);
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
  GPB_TRY(op.to_local(y_centered_host, op.S.yc.f()));
  BBMMResult R;
  GPB_TRY(bbmm_step(E, op.pc.rank > 0 ? &op.pc : nullptr, op.S, num_probes, max_cg_iter,
                    max_tridiag_iter, cg_tol, iteration, recycle != 0, R));
  *nll_out = R.nll;
  for (size_t q = 0; q < R.grads.size(); ++q) kernel_grads_out[q] = R.grads[q];
  for (size_t q = 0; q < R.grad_A.size(); ++q) grad_A_out[q] = R.grad_A[q];
  for (int t = 0; t < op.T; ++t) {
    grad_noise_out[t] = R.grad_noise_task[t];
    sum_alpha_out[t] = R.sum_alpha_task[t];
  }
  if (alpha_out) GPB_TRY(op.to_host(op.S.sol.f(), alpha_out));
  if (cg_iters_out) *cg_iters_out = R.cg_iters;
  return provider_check_device_error(op.prov[0]);
}

int gpb_lmc_build_precond(gpb_lmc* h, int32_t rank, int32_t* ranks_out, double* logdet_out) {
  clear_error();
  GPB_REQUIRE(h, GPB_ERR_INVALID, "null argument");
  LmcOp& op = h->op;
  GPB_CHECK_CUDA(cudaSetDevice(op.prov[0]->device));
  GPB_TRY(lmc_build_precond(op, rank));
  if (ranks_out)
    for (int s = 0; s < op.R; ++s) ranks_out[s] = op.pc.rank > 0 ? op.lp.rank[s] : 0;
  if (logdet_out) *logdet_out = op.pc.logdet;
  return provider_check_device_error(op.prov[0]);
}

int gpb_lmc_precond_apply(gpb_lmc* h, float* out_dev, const float* v_dev, int64_t ncols) {
  GPB_REQUIRE(h && out_dev && v_dev && ncols >= 0, GPB_ERR_INVALID, "bad arguments");
  LmcOp& op = h->op;
  GPB_REQUIRE(op.pc.rank > 0, GPB_ERR_INVALID, "no LMC preconditioner built");
  GPB_CHECK_CUDA(cudaSetDevice(op.prov[0]->device));
  if (ncols == 0) return GPB_OK;
  GPB_TRY(precond_apply(op.E, op.pc, v_dev, out_dev, (int)ncols));
  GPB_CHECK_CUDA(cudaStreamSynchronize(op.E.st));
  return provider_check_device_error(op.prov[0]);
}

int gpb_lmc_precond_sample(gpb_lmc* h, float* out_dev, int32_t num, uint64_t seed) {
  GPB_REQUIRE(h && out_dev && num >= 0, GPB_ERR_INVALID, "bad arguments");
  LmcOp& op = h->op;
  GPB_REQUIRE(op.pc.rank > 0, GPB_ERR_INVALID, "no LMC preconditioner built");
  GPB_CHECK_CUDA(cudaSetDevice(op.prov[0]->device));
  if (num == 0) return GPB_OK;
  GPB_TRY(precond_sample(op.E, op.pc, num, seed, out_dev));
  GPB_CHECK_CUDA(cudaStreamSynchronize(op.E.st));
  return provider_check_device_error(op.prov[0]);
}

int gpb_lmc_solve(gpb_lmc* h, const float* rhs_host, int32_t max_cg_iter, float cg_tol,
                  float* x_host_out, int32_t* iters_out) {
  GPB_REQUIRE(h && rhs_host && x_host_out, GPB_ERR_INVALID, "null argument");
  LmcOp& op = h->op;
  GPB_CHECK_CUDA(cudaSetDevice(op.prov[0]->device));
  Engine& E = op.E;
  DBuf y, x;
  GPB_TRY(y.ensure((size_t)std::max<int64_t>(E.nl, 1) * sizeof(float)));
  GPB_TRY(x.ensure((size_t)std::max<int64_t>(E.nl, 1) * sizeof(float)));
  GPB_TRY(op.to_local(rhs_host, y.f()));
  int it = 0;
  GPB_TRY(alpha_cg(E, y.f(), x.f(), max_cg_iter, cg_tol, &it));
  GPB_TRY(op.to_host(x.f(), x_host_out));
  if (iters_out) *iters_out = it;
  return provider_check_device_error(op.prov[0]);
}

// Exact LMC posterior variance (_predict_lmc_full_exact_variance_backend,
// mojogp/multi_output_gp.py:4360-4519): per test point c and output task t,
// var = max(sum_s A_s[t][t] k_s(x*, x*) - r^T K_full^{-1} r + noise_t, 1e-10)
// with r = sum_s k_s(X, x*_c) (x) A_s[:, t]. The reference solves one
// right-hand side at a time; here a block of test points x all T tasks is one
// batched CG on the LMC operator (with the sum-of-Kronecker preconditioner when
// built), normalised columns, as the single-output exact variance.
int gpb_lmc_predict_exact_variance(gpb_lmc* h, const float* xtest_host, int64_t n_test,
                                   int32_t block_cols, int32_t max_cg_iter, float cg_tol,
                                   float* var_out, int32_t* cg_iters_out) {
  clear_error();
  GPB_REQUIRE(h && xtest_host && var_out && n_test >= 0 && max_cg_iter >= 1, GPB_ERR_INVALID,
              "bad arguments");
  if (n_test == 0) return GPB_OK;
  LmcOp& op = h->op;
  GPB_CHECK_CUDA(cudaSetDevice(op.prov[0]->device));
  Engine& E = op.E;
  cudaStream_t st = E.st;
  const int R = op.R, T = op.T, d = op.prov[0]->d;
  for (int s = 1; s < R; ++s)
    GPB_REQUIRE(op.prov[s]->d == d, GPB_ERR_INVALID, "latent input dims differ");
  // Block of test points: all T task columns of each, at most 512 columns.
  const int cap = block_cols > 0 ? block_cols : 512;
  const int b = (int)std::min<int64_t>(n_test, std::max(1, cap / T));
  const int mc = b * T;
  BBMMState S;
  GPB_TRY(S.ensure(E, mc, 1));
  DBuf xt, cross, rhs0, diag;
  GPB_TRY(xt.ensure((size_t)n_test * d * sizeof(float)));
  GPB_TRY(cross.ensure((size_t)R * b * std::max<int64_t>(op.nl, 1) * sizeof(float)));
  GPB_TRY(rhs0.ensure((size_t)mc * std::max<int64_t>(E.nl, 1) * sizeof(float)));
  GPB_TRY(diag.ensure((size_t)R * b * sizeof(float)));
  GPB_CHECK_CUDA(cudaMemcpyAsync(xt.ptr, xtest_host, (size_t)n_test * d * sizeof(float),
                                 cudaMemcpyHostToDevice, st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  std::vector<float> norms, dg((size_t)R * b);
  int total_iters = 0;
  for (int64_t c0 = 0; c0 < n_test; c0 += b) {
    const int m = (int)std::min<int64_t>(b, n_test - c0);
    const int cols = m * T;
    const float* xb = xt.f() + c0 * d;
    // 1. Per-latent cross blocks K_s(X_local, X*_block) and prior diagonals.
    for (int s = 0; s < R; ++s) {
      GPB_TRY(cross_fill(op.prov[s], op.r0, op.nl, xb, m, cross.f() + (int64_t)s * b * op.nl, st));
      GPB_TRY(gpb_extract_diagonal_test(op.prov[s], diag.f() + (int64_t)s * b, xb, m));
      GPB_CHECK_CUDA(cudaStreamSynchronize(op.prov[s]->stream));
    }
    if (op.nl > 0) {
      dim3 grid((unsigned)ceil_div(op.nl, 128), (unsigned)cols, (unsigned)T);
      lmc_exact_rhs_kernel<<<grid, 128, 0, st>>>(cross.f(), op.A_d.f(), R, T, b, op.nl,
                                                   rhs0.f());
      GPB_CHECK_CUDA(cudaGetLastError());
    }
    // 2. K_full V = rhs by batched CG on normalised columns.
    float* rhs = S.rhs.f();
    GPB_TRY(k_copy(rhs, rhs0.f(), (int64_t)cols * E.nl, st));
    float* norms_dev = S.scal.f() + 3 * cols;
    GPB_TRY(column_norms(E, rhs, cols, norms, norms_dev, true));
    CGResult cg;
    GPB_TRY(cg_solve(E, op.pc.rank > 0 ? &op.pc : nullptr, S, rhs, cols, max_cg_iter, 0, cg_tol,
                     false, cg));
    total_iters += cg.iters;
    float* sol = S.x.f();
    GPB_TRY(k_scale_cols(sol, E.nl, E.nl, cols, norms_dev, 0, st));
    // 3. Correction r^T v per column, then the variance.
    const float* a[1] = {rhs0.f()};
    const float* bb[1] = {sol};
    GPB_TRY(E.coldots(1, a, bb, E.nl, cols, true));
    GPB_CHECK_CUDA(cudaMemcpyAsync(dg.data(), diag.ptr, (size_t)R * b * sizeof(float),
                                   cudaMemcpyDeviceToHost, st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(st));
    for (int c = 0; c < m; ++c)
      for (int t = 0; t < T; ++t) {
        double prior = 0.0;
        for (int s = 0; s < R; ++s)
          prior += (double)op.A[((size_t)s * T + t) * T + t] * dg[(size_t)s * b + c];
        double v = prior - E.host_sums[c * T + t] + op.noise[t];
        var_out[(c0 + c) * T + t] = (float)std::max(v, 1e-10);
      }
  }
  if (cg_iters_out) *cg_iters_out = total_iters;
  return provider_check_device_error(op.prov[0]);
}

}  // extern "C"
