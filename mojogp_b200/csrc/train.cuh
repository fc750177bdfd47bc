// BBMM state and results shared by training and the gpb_bbmm entry point.
#pragma once

#include <vector>

#include "engine.cuh"
#include "precond.cuh"

namespace gpb {

struct BBMMState {
  int t = 0, max_tridiag = 1;
  bool have_x = false;  // x column 0 holds the previous solve (warm start)
  DBuf x, r, z, pv, Ap, rhs, sol, probes, sampled, rf, scal, hist_a, hist_b, yc, ones, bfull, gbuf;
  int ensure(const Engine& E, int t, int max_tridiag);
};

struct CGResult {
  int iters = 0;
  bool converged = false;
  std::vector<std::vector<float>> diag, offdiag;  // per column
};

struct BBMMResult {
  double nll = 0, inv_quad = 0, logdet = 0, sum_alpha = 0;
  std::vector<double> grads;  // P kernel params + noise
  int cg_iters = 0;
  // LMC extras: dNLL/dA_s [R][T][T], per-task noise gradients, per-task sum(alpha)
  std::vector<double> grad_A, grad_noise_task, sum_alpha_task;
};

int cg_solve(Engine& E, Precond* P, BBMMState& S, const float* rhs, int t, int max_iter,
             int max_tridiag, float tol, bool warm, CGResult& out);
int bbmm_step(Engine& E, Precond* P, BBMMState& S, int num_probes, int max_cg, int max_tridiag,
              float tol, int iteration, bool recycle, BBMMResult& R);
int k_sub_scalar(float* v, int64_t count, float s, cudaStream_t st);
// Column 2-norms over all ranks (host and device copies); normalises in place.
int column_norms(Engine& E, float* v, int t, std::vector<float>& norms_h, float* norms_dev,
                 bool normalize);
// (K + noise) x = y by CG with the relative-residual stop (predict.cu).
int alpha_cg(Engine& E, const float* y_local, float* x, int max_iter, float tol, int* iters_out);
// LMC gradients from the BBMM solution (lmc.cu); sol holds [alpha | scaled
// probe solutions], sampled the unnormalised probes.
int lmc_bbmm_gradients(Engine& E, BBMMState& S, float* sol, const float* rf, int num_probes,
                       BBMMResult& R);

}  // namespace gpb
