// mBCG / BBMM and the Adam training loop, plus the NCCL communicator ABI.
//
// References (MojoGP 0.26.6.0):
//   batched_cg_unified      kernels/combined_inv_quad_logdet.mojo:81-445
//   bbmm_with_precond       kernels/combined_inv_quad_logdet.mojo:452-1136
//   train_jit_with_provider kernels/jit/jit_training.mojo:274-1008
//   softplus / Adam / cosine kernels/utils.mojo:14-84, kernels/training_utils.mojo:23-315
#include <chrono>
#include <cmath>
#include <cstdio>
#include <vector>

#include "engine.cuh"
#include "numerics.h"
#include "precond.cuh"
#include "train.cuh"

struct gpb_comm {
  gpb::Dist dist;
  int device = 0;
  cudaStream_t st = nullptr;
  double* buf = nullptr;
};

namespace gpb {

// --------------------------------------------------------------- helpers
static float softplus(float x) {
  if (x > 20.f) return x;
  if (x < -20.f) return std::exp(x);
  return std::log(1.f + std::exp(x));
}
static float inv_softplus(float y) {
  if (y > 20.f) return y;
  if (y < 1e-6f) return std::log(y);
  return std::log(std::exp(y) - 1.f);
}
static float softplus_derivative(float x) {
  if (x > 20.f) return 1.f;
  if (x < -20.f) return std::exp(x);
  return 1.f / (1.f + std::exp(-x));
}
static float clip_gradient(float g, float max_grad = 100.f) {
  if (g != g) return 0.f;
  if (g > 1e30f || g < -1e30f) return 0.f;
  if (g > max_grad) return max_grad;
  if (g < -max_grad) return -max_grad;
  return g;
}
static float powi(float b, int e) {
  float r = 1.f;
  while (e > 0) {
    if (e & 1) r *= b;
    b *= b;
    e >>= 1;
  }
  return r;
}
static float cosine_lr(float lr_max, int it, int total) {
  const float lr_min = lr_max / 20.f;
  const float frac = (float)it / (float)std::max(total, 1);
  return lr_min + 0.5f * (lr_max - lr_min) * (1.f + std::cos(3.14159265358979f * frac));
}

int column_norms(Engine& E, float* v, int t, std::vector<float>& norms_h, float* norms_dev,
                 bool normalize) {
  const float* a[1] = {v};
  GPB_TRY(E.coldots(1, a, a, E.nl, t, true));
  norms_h.resize(t);
  for (int c = 0; c < t; ++c) norms_h[c] = std::sqrt((float)E.host_sums[c]);
  GPB_CHECK_CUDA(cudaMemcpyAsync(norms_dev, norms_h.data(), t * sizeof(float),
                                 cudaMemcpyHostToDevice, E.st));
  if (normalize) GPB_TRY(k_scale_cols(v, E.nl, E.nl, t, norms_dev, 1, E.st));
  return GPB_OK;
}

int BBMMState::ensure(const Engine& E, int t_, int max_tridiag_) {
  t = t_;
  max_tridiag = std::max(max_tridiag_, 1);
  const size_t b = (size_t)t * std::max<int64_t>(E.nl, 1) * sizeof(float);
  GPB_TRY(x.ensure(b));
  GPB_TRY(r.ensure(b));
  GPB_TRY(z.ensure(b));
  GPB_TRY(pv.ensure(b));
  GPB_TRY(Ap.ensure(b));
  GPB_TRY(rhs.ensure(b));
  GPB_TRY(sol.ensure(b));
  GPB_TRY(probes.ensure(b));
  GPB_TRY(sampled.ensure(b));
  GPB_TRY(rf.ensure(b));
  GPB_TRY(scal.ensure(sizeof(float) * 8 * (size_t)t));
  GPB_TRY(hist_a.ensure(sizeof(float) * (size_t)max_tridiag * t));
  GPB_TRY(hist_b.ensure(sizeof(float) * (size_t)max_tridiag * t));
  GPB_TRY(yc.ensure(sizeof(float) * std::max<int64_t>(E.nl, 1)));
  GPB_TRY(ones.ensure(sizeof(float) * std::max<int64_t>(E.nl, 1)));
  return k_fill(ones.f(), E.nl, 1.f, E.st);
}

// ------------------------------------------------------------------ mBCG
int cg_solve(Engine& E, Precond* P, BBMMState& S, const float* rhs, int t, int max_iter,
             int max_tridiag, float tol, bool warm, CGResult& out) {
  const int64_t nl = E.nl;
  cudaStream_t st = E.st;
  float* x = S.x.f();
  float* r = S.r.f();
  float* pv = S.pv.f();
  float* Ap = S.Ap.f();
  const bool use_p = P && P->rank > 0;
  float* z = use_p ? S.z.f() : r;
  float* rz_old = S.scal.f();
  float* alpha = rz_old + t;
  float* beta = alpha + t;
  const int64_t cnt = (int64_t)t * nl;
  if (warm) {
    GPB_TRY(k_copy(r, rhs, cnt, st));
    GPB_TRY(E.matvec(x, nl, t, Ap, nl));
    GPB_TRY(k_sub(r, Ap, cnt, st));
  } else {
    GPB_TRY(k_fill(x, cnt, 0.f, st));
    GPB_TRY(k_copy(r, rhs, cnt, st));
  }
  if (use_p) GPB_TRY(precond_apply(E, *P, r, z, t));
  GPB_TRY(k_copy(pv, z, cnt, st));
  {
    const float* a[1] = {r};
    const float* b[1] = {z};
    GPB_TRY(E.coldots(1, a, b, nl, t, false));
    GPB_TRY(k_set_rz(rz_old, E.red.sums.d(), t, st));
  }
  int iters = 0;
  bool converged = false;
  for (int it = 0; it < max_iter; ++it) {
    iters = it + 1;
    GPB_TRY(E.matvec(pv, nl, t, Ap, nl, it > 0 ? z : nullptr, it > 0 ? beta : nullptr));
    {
      const float* a[1] = {pv};
      const float* b[1] = {Ap};
      GPB_TRY(E.coldots(1, a, b, nl, t, false));
    }
    GPB_TRY(k_cg_alpha(rz_old, E.red.sums.d(), alpha,
                       it < max_tridiag ? S.hist_a.f() + (size_t)it * t : nullptr, t, st));
    GPB_TRY(k_cg_update(alpha, pv, Ap, x, r, nl, nl, t, st));
    if (use_p) GPB_TRY(precond_apply(E, *P, r, z, t));
    const bool check = it >= 10 && (((it + 1) % 10) == 0 || it == max_iter - 1);
    {
      const float* a[2] = {r, r};
      const float* b[2] = {z, r};
      const int np = (check && use_p) ? 2 : 1;
      GPB_TRY(E.coldots(np, a, b, nl, t, check));
    }
    GPB_TRY(k_cg_beta(rz_old, E.red.sums.d(), beta,
                      it < max_tridiag ? S.hist_b.f() + (size_t)it * t : nullptr, t, st));
    E.p->launches += 4;
    if (check) {
      const double* rr = E.host_sums.data() + ((use_p) ? t : 0);
      double mean = 0.0;
      for (int c = 0; c < t; ++c) mean += std::sqrt((float)rr[c]);
      mean /= t;
      if ((float)mean < tol && it >= max_tridiag - 1) {
        converged = true;
        break;
      }
    }
  }
  out.iters = iters;
  out.converged = converged;
  // Tridiagonals (combined_inv_quad_logdet.mojo:356-423).
  const int size = std::min(iters, max_tridiag);
  std::vector<float> ah((size_t)size * t), bh((size_t)size * t);
  if (size > 0) {
    GPB_CHECK_CUDA(cudaMemcpyAsync(ah.data(), S.hist_a.ptr, ah.size() * sizeof(float),
                                   cudaMemcpyDeviceToHost, st));
    GPB_CHECK_CUDA(cudaMemcpyAsync(bh.data(), S.hist_b.ptr, bh.size() * sizeof(float),
                                   cudaMemcpyDeviceToHost, st));
  }
  GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  out.diag.assign(t, {});
  out.offdiag.assign(t, {});
  bool update = true;
  for (int k = 0; k < size && update; ++k) {
    float max_off = 0.f;
    for (int c = 0; c < t; ++c) {
      const float ak = ah[(size_t)k * t + c];
      const float ar = ak < 1e-10f ? 1.f : 1.f / ak;
      float dv = ar;
      if (k > 0) {
        const float akm = ah[(size_t)(k - 1) * t + c];
        const float prev = akm < 1e-10f ? 1.f : 1.f / akm;
        float bkm = bh[(size_t)(k - 1) * t + c];
        dv += bkm * prev;
        if (bkm < 0.f) bkm = 0.f;
        const float off = std::sqrt(bkm) * prev;
        out.offdiag[c].push_back(off);
        max_off = std::max(max_off, off);
      }
      out.diag[c].push_back(dv);
    }
    if (k > 0 && max_off < 1e-6f) update = false;
  }
  return GPB_OK;
}

// ------------------------------------------------------------------ BBMM
int bbmm_step(Engine& E, Precond* P, BBMMState& S, int num_probes, int max_cg, int max_tridiag,
              float tol, int iteration, bool recycle, BBMMResult& R) {
  const int t = 1 + num_probes;
  const int64_t nl = E.nl;
  cudaStream_t st = E.st;
  gpb_provider* p = E.p;
  const bool use_p = P && P->rank > 0;
  float* norms_dev = S.scal.f() + 3 * t;  // rhs norms [t], probe norms [num_probes]
  float* pnorms_dev = norms_dev + t;
  const uint64_t seed = (uint64_t)iteration * 104729ull + 42ull;

  // 1. probes ~ N(0, P) or N(0, I), normalised (kept with their norms).
  float* sampled = S.sampled.f();
  if (use_p)
    GPB_TRY(precond_sample(E, *P, num_probes, seed, sampled));
  else if (E.op)
    GPB_TRY(E.op->gaussian(sampled, num_probes, seed, st));
  else
    GPB_TRY(k_gaussian(sampled, num_probes, nl, nl, E.n, E.r0, seed, st));
  float* probes = S.probes.f();
  GPB_TRY(k_copy(probes, sampled, (int64_t)num_probes * nl, st));
  std::vector<float> pnorms, rnorms;
  GPB_TRY(column_norms(E, probes, num_probes, pnorms, pnorms_dev, true));

  // 2. rhs = [y | Z] with every column normalised.
  float* rhs = S.rhs.f();
  GPB_TRY(k_copy(rhs, S.yc.f(), nl, st));
  GPB_TRY(k_copy(rhs + nl, probes, (int64_t)num_probes * nl, st));
  GPB_TRY(column_norms(E, rhs, t, rnorms, norms_dev, true));
  const bool warm = recycle && iteration > 0 && S.have_x;
  if (warm) GPB_TRY(k_fill(S.x.f() + nl, (int64_t)num_probes * nl, 0.f, st));

  // 3. mBCG.
  CGResult cg;
  GPB_TRY(cg_solve(E, P, S, rhs, t, max_cg, max_tridiag, tol, warm, cg));
  S.have_x = true;
  R.cg_iters = cg.iters;

  // Solution un-normalised: sol = x * rhs_norms.
  float* sol = S.sol.f();
  GPB_TRY(k_copy(sol, S.x.f(), (int64_t)t * nl, st));
  GPB_TRY(k_scale_cols(sol, nl, nl, t, norms_dev, 0, st));

  // 4. inv_quad = y . alpha ; sum(alpha) for the mean gradient.
  {
    const float* a[2] = {S.yc.f(), sol};
    const float* b[2] = {sol, S.ones.f()};
    GPB_TRY(E.coldots(2, a, b, nl, 1, true));
    R.inv_quad = E.host_sums[0];
    R.sum_alpha = E.host_sums[1];
  }
  // 5. log|K| = SLQ over the probe tridiagonals + log|P|.
  std::vector<std::vector<double>> dg, od;
  for (int c = 1; c < t; ++c) {
    dg.emplace_back(cg.diag[c].begin(), cg.diag[c].end());
    od.emplace_back(cg.offdiag[c].begin(), cg.offdiag[c].end());
  }
  R.logdet = slq_logdet(dg, od, E.n) + (use_p ? P->logdet : 0.0);
  const double n = (double)E.n;
  const double PI32 = (double)3.14159265358979323846f;
  R.nll = (0.5 * R.inv_quad + 0.5 * R.logdet + 0.5 * n * std::log(2.0 * PI32)) / n;

  // 6. Gradients: a = [alpha | u_j * |z_j|], b = [alpha | P^{-1} z_j].
  float* A = sol;  // probe columns scaled by probe norms in place
  GPB_TRY(k_scale_cols(A + nl, nl, nl, num_probes, pnorms_dev, 0, st));
  float* B = S.rf.f();
  GPB_TRY(k_copy(B, sol, nl, st));
  if (use_p)
    GPB_TRY(precond_apply(E, *P, sampled, B + nl, num_probes));
  else
    GPB_TRY(k_copy(B + nl, sampled, (int64_t)num_probes * nl, st));
  // LMC: the right factors are P^{-1} z (z when unpreconditioned), as in the
  // single-output path.
  if (E.op) return lmc_bbmm_gradients(E, S, A, B + nl, num_probes, R);
  const int P_ = p->dk.nparams;
  std::vector<double> data(P_, 0.0), trace(P_, 0.0);
  {
    // The column side of the bilinear form needs all rows of B.
    float* Bfull = B;
    if (E.dist.world > 1) {
      GPB_TRY(S.bfull.ensure((size_t)t * E.n * sizeof(float)));
      GPB_TRY(E.allgather_cols(B, nl, t, S.bfull.f()));
      Bfull = S.bfull.f();
    }
    GPB_TRY(provider_bilinear_rows(p, A, nl, Bfull, t, E.r0, E.r1, data.data(),
                                       trace.data(), st));
    if (E.dist.world > 1) {
      std::vector<double> both(2 * P_);
      for (int q = 0; q < P_; ++q) {
        both[q] = data[q];
        both[P_ + q] = trace[q];
      }
      GPB_TRY(S.gbuf.ensure(both.size() * sizeof(double)));
      GPB_CHECK_CUDA(cudaMemcpyAsync(S.gbuf.ptr, both.data(), both.size() * sizeof(double),
                                     cudaMemcpyHostToDevice, st));
      GPB_TRY(E.allreduce_sum(S.gbuf.d(), both.size()));
      GPB_CHECK_CUDA(cudaMemcpyAsync(both.data(), S.gbuf.ptr, both.size() * sizeof(double),
                                     cudaMemcpyDeviceToHost, st));
      GPB_CHECK_CUDA(cudaStreamSynchronize(st));
      for (int q = 0; q < P_; ++q) {
        data[q] = both[q];
        trace[q] = both[P_ + q];
      }
    }
  }
  R.grads.assign(P_ + 1, 0.0);
  for (int q = 0; q < P_; ++q) {
    const float dt = -0.5f * (float)data[q];
    const float ct = 0.5f * (float)trace[q] / (float)num_probes;
    float g = (dt + ct) / (float)n;
    if (!std::isfinite(g)) g = 0.f;
    R.grads[q] = g;
  }
  // Noise gradient: (-0.5 |alpha|^2 + 0.5 sum_j u_j . w_j / P) / n.
  {
    const float* a[2] = {A, A + nl};
    const float* b[2] = {A, B + nl};
    GPB_TRY(E.coldots(1, a, b, nl, 1, true));
    const double an = E.host_sums[0];
    GPB_TRY(E.coldots(1, a + 1, b + 1, nl, num_probes, true));
    double tr = 0.0;
    for (int c = 0; c < num_probes; ++c) tr += (float)E.host_sums[c];
    float g = (-0.5f * (float)an + 0.5f * (float)tr / (float)num_probes) / (float)n;
    if (!std::isfinite(g)) g = 0.f;
    R.grads[P_] = g;
  }
  return GPB_OK;
}

// ------------------------------------------------------------ train loop
int train_loop(Engine& E, const float* y_host_local, const gpb_train_options& o,
               gpb_train_result& res) {
  gpb_provider* p = E.p;
  cudaStream_t st = E.st;
  const int P_ = p->dk.nparams;
  const int t = 1 + o.num_probes;
  BBMMState S;
  GPB_TRY(S.ensure(E, t, o.max_tridiag_iter));
  DBuf y_dev;
  GPB_TRY(y_dev.ensure(sizeof(float) * std::max<int64_t>(E.nl, 1)));
  GPB_CHECK_CUDA(cudaMemcpyAsync(y_dev.ptr, y_host_local, E.nl * sizeof(float),
                                 cudaMemcpyHostToDevice, st));
  std::vector<float> init(P_);
  for (int q = 0; q < P_; ++q) init[q] = p->dk.params[q];
  const float initial_noise = p->noise;
  std::vector<float> raw(P_ + 1), m(P_ + 1, 0.f), v(P_ + 1, 0.f);
  for (int q = 0; q < P_; ++q) raw[q] = inv_softplus(init[q]);
  raw[P_] = inv_softplus(initial_noise);
  int adam_t = 0;
  float raw_mean = o.init_mean, m_mean = 0.f, v_mean = 0.f;
  std::vector<float> best_raw(raw), best_m(m), best_v(v);
  float best_raw_mean = raw_mean, best_m_mean = 0.f, best_v_mean = 0.f;
  int best_t = 0;
  float best_nll_seen = 1e30f, best_nll_es = 1e30f;
  int no_improve = 0;
  float lr = o.learning_rate;
  std::vector<float> last_rebuild(init);
  float last_rebuild_noise = initial_noise;
  bool alpha_valid = false;
  std::vector<float> best_alpha;
  Precond P;
  int builds = 0;
  double build_ms = 0.0;
  const bool use_p = o.use_preconditioner && o.precond_rank > 0;
  auto build = [&]() -> int {
    auto t0 = std::chrono::steady_clock::now();
    int s = precond_build(E, use_p ? o.precond_rank : 0, P);
    build_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    ++builds;
    return s;
  };
  GPB_TRY(build());
  int iters = 0;
  bool converged = false;
  for (int it = 0; it < o.max_iterations; ++it) {
    const auto t0 = std::chrono::steady_clock::now();
    iters = it + 1;
    std::vector<float> cons(P_);
    for (int q = 0; q < P_; ++q) cons[q] = softplus(raw[q]);
    const float noise = o.learn_noise ? softplus(raw[P_]) : 0.f;
    for (int q = 0; q < P_; ++q) p->dk.params[q] = cons[q];
    GPB_TRY(provider_plan(p));
    p->noise = noise;
    if (it > 0) {
      float max_rel = 0.f;
      for (int q = 0; q < P_; ++q)
        max_rel = std::max(max_rel, std::fabs(cons[q] - last_rebuild[q]) /
                                        std::max(std::fabs(last_rebuild[q]), 1e-8f));
      if (o.learn_noise)
        max_rel = std::max(max_rel, std::fabs(noise - last_rebuild_noise) /
                                        std::max(std::fabs(last_rebuild_noise), 1e-8f));
      if (max_rel > o.precond_rebuild_threshold) {
        GPB_TRY(build());
        last_rebuild = cons;
        last_rebuild_noise = noise;
      }
    }
    // centre y by the current mean
    GPB_TRY(k_copy(S.yc.f(), y_dev.f(), E.nl, st));
    GPB_TRY(k_fill(S.ones.f(), E.nl, 1.f, st));
    GPB_TRY(k_sub_scalar(S.yc.f(), E.nl, raw_mean, st));
    BBMMResult R;
    GPB_TRY(bbmm_step(E, use_p ? &P : nullptr, S, o.num_probes, o.max_cg_iter, o.max_tridiag_iter,
                      o.cg_tol, it, it > 0, R));
    const float nll = (float)R.nll;
    if (res.cg_iterations) res.cg_iterations[it] = R.cg_iters;
    if (res.tile_layouts) res.tile_layouts[it] = kv_layout(p->eval, p->DP, 16, p->gram_ok);
    if (nll != nll) {
      lr *= 0.5f;
      if (o.verbose) std::printf("  NaN NLL at iteration %d - halving LR to %g\n", it, lr);
      raw = best_raw;
      m = best_m;
      v = best_v;
      m_mean = best_m_mean;
      v_mean = best_v_mean;
      adam_t = best_t;
      raw_mean = best_raw_mean;
      for (int q = 0; q < P_; ++q) {
        p->dk.params[q] = softplus(raw[q]);
        last_rebuild[q] = p->dk.params[q];
      }
      GPB_TRY(provider_plan(p));
      p->noise = o.learn_noise ? softplus(raw[P_]) : 0.f;
      last_rebuild_noise = p->noise;
      GPB_TRY(build());
      if (res.nll_history) res.nll_history[it] = nll;
      if (res.iter_times_ms)
        res.iter_times_ms[it] =
            std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
      continue;
    }
    if (nll < best_nll_seen) {
      best_nll_seen = nll;
      best_raw = raw;
      best_raw_mean = raw_mean;
      best_m = m;
      best_v = v;
      best_m_mean = m_mean;
      best_v_mean = v_mean;
      best_t = adam_t;
      if (res.alpha) {
        best_alpha.resize(E.nl);
        GPB_CHECK_CUDA(cudaMemcpyAsync(best_alpha.data(), S.sol.ptr, E.nl * sizeof(float),
                                       cudaMemcpyDeviceToHost, st));
        GPB_CHECK_CUDA(cudaStreamSynchronize(st));
      }
      alpha_valid = true;
    }
    const float eff_lr = o.use_cosine_lr ? cosine_lr(o.learning_rate, it, o.max_iterations) : lr;
    std::vector<float> g(P_ + 1);
    for (int q = 0; q < P_; ++q)
      g[q] = (o.trainable_mask && !o.trainable_mask[q]) ? 0.f : (float)R.grads[q];
    g[P_] = o.learn_noise ? (float)R.grads[P_] : 0.f;
    // Adam (training_utils.mojo:214-315): clip, chain rule through softplus,
    // bias-corrected moments, raw clamp to [-20, 20].
    adam_t += 1;
    for (int q = 0; q <= P_; ++q) {
      const float gr = clip_gradient(g[q]) * softplus_derivative(raw[q]);
      m[q] = 0.9f * m[q] + 0.1f * gr;
      v[q] = 0.999f * v[q] + 0.001f * gr * gr;
    }
    for (int q = 0; q <= P_; ++q) {
      const float mh = m[q] / (1.f - powi(0.9f, adam_t));
      const float vh = v[q] / (1.f - powi(0.999f, adam_t));
      float nr = raw[q] - eff_lr * mh / (std::sqrt(vh) + 1e-8f);
      raw[q] = std::max(-20.f, std::min(20.f, nr));
    }
    // Constant mean (jit_training.mojo:810-848).
    float mg = clip_gradient(-(float)R.sum_alpha / (float)E.n);
    m_mean = 0.9f * m_mean + 0.1f * mg;
    v_mean = 0.999f * v_mean + 0.001f * mg * mg;
    const float mhm = m_mean / (1.f - powi(0.9f, adam_t));
    const float vhm = v_mean / (1.f - powi(0.999f, adam_t));
    raw_mean -= eff_lr * mhm / (std::sqrt(vhm) + 1e-8f);
    if (raw_mean != raw_mean || raw_mean > 1000.f || raw_mean < -1000.f) raw_mean = o.init_mean;
    if (o.verbose && (it % 10 == 0 || it == o.max_iterations - 1))
      std::printf("Iter %d : NLL = %g , noise = %g , mean = %g\n", it, nll, noise, raw_mean);
    if (res.nll_history) res.nll_history[it] = nll;
    if (res.iter_times_ms)
      res.iter_times_ms[it] =
          std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (o.enable_early_stopping) {
      if (nll < best_nll_es - o.early_stop_tol) {
        best_nll_es = nll;
        no_improve = 0;
      } else if (++no_improve >= o.early_stop_patience) {
        converged = true;
        break;
      }
    }
  }
  // Restore best parameters.
  raw = best_raw;
  raw_mean = best_raw_mean;
  for (int q = 0; q < P_; ++q) {
    p->dk.params[q] = softplus(raw[q]);
    if (res.params) res.params[q] = p->dk.params[q];
  }
  GPB_TRY(provider_plan(p));
  p->noise = o.learn_noise ? softplus(raw[P_]) : 0.f;
  res.final_nll = best_nll_seen;
  res.noise = p->noise;
  res.mean = raw_mean;
  res.iterations = iters;
  res.converged = converged;
  res.alpha_valid = alpha_valid && res.alpha != nullptr;
  if (res.alpha && alpha_valid) std::copy(best_alpha.begin(), best_alpha.end(), res.alpha);
  res.precond_build_count = builds;
  res.precond_build_ms = build_ms;
  res.precond_rank = P.rank;
  return provider_check_device_error(p);
}

}  // namespace gpb

using namespace gpb;

namespace gpb {
int engine_from_comm(gpb_provider* p, gpb_comm* comm, Engine& E) {
  Dist d;
  if (comm) {
    d = comm->dist;
    GPB_REQUIRE(comm->device == p->device, GPB_ERR_INVALID,
                "communicator device %d != provider device %d", comm->device, p->device);
  }
  return E.init(p, d);
}
}  // namespace gpb

extern "C" {

int gpb_comm_unique_id(uint8_t* id_out) {
  GPB_REQUIRE(id_out, GPB_ERR_INVALID, "null id");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  GPB_REQUIRE(r == ncclSuccess, GPB_ERR_NCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  static_assert(sizeof(ncclUniqueId) == GPB_COMM_ID_BYTES, "nccl id size");
  std::memcpy(id_out, &id, sizeof(id));
  return GPB_OK;
}

int gpb_comm_init(const uint8_t* id, int32_t world, int32_t rank, int32_t device, gpb_comm** out) {
  GPB_REQUIRE(id && out && world >= 1 && rank >= 0 && rank < world, GPB_ERR_INVALID,
              "bad communicator arguments");
  GPB_CHECK_CUDA(cudaSetDevice(device));
  gpb_comm* c = new gpb_comm();
  c->device = device;
  c->dist.rank = rank;
  c->dist.world = world;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = ncclCommInitRank(&c->dist.comm, world, uid, rank);
  if (r != ncclSuccess) {
    set_error("ncclCommInitRank: %s", ncclGetErrorString(r));
    delete c;
    return GPB_ERR_NCCL;
  }
  if (cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->buf, 4096 * sizeof(double)) != cudaSuccess) {
    set_error("communicator scratch setup failed");
    ncclCommDestroy(c->dist.comm);
    delete c;
    return GPB_ERR_CUDA;
  }
  *out = c;
  return GPB_OK;
}

int gpb_comm_destroy(gpb_comm* c) {
  if (!c) return GPB_OK;
  cudaSetDevice(c->device);
  if (c->st) cudaStreamSynchronize(c->st);
  if (c->dist.comm) ncclCommDestroy(c->dist.comm);
  if (c->buf) cudaFree(c->buf);
  if (c->st) cudaStreamDestroy(c->st);
  delete c;
  return GPB_OK;
}

static int comm_host_reduce(gpb_comm* c, double* vals, int64_t count, ncclRedOp_t op) {
  GPB_REQUIRE(c && (vals || count == 0) && count >= 0, GPB_ERR_INVALID, "bad reduce arguments");
  GPB_CHECK_CUDA(cudaSetDevice(c->device));
  // The communicator's staging buffer holds 4096 doubles: larger arrays go
  // through it in pieces.
  for (int64_t off = 0; off < count; off += 4096) {
    const int64_t m = std::min<int64_t>(4096, count - off);
    GPB_CHECK_CUDA(cudaMemcpyAsync(c->buf, vals + off, m * sizeof(double), cudaMemcpyHostToDevice,
                                   c->st));
    ncclResult_t r = ncclAllReduce(c->buf, c->buf, m, ncclDouble, op, c->dist.comm, c->st);
    GPB_REQUIRE(r == ncclSuccess, GPB_ERR_NCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
    GPB_CHECK_CUDA(cudaMemcpyAsync(vals + off, c->buf, m * sizeof(double), cudaMemcpyDeviceToHost,
                                   c->st));
  }
  GPB_CHECK_CUDA(cudaStreamSynchronize(c->st));
  return GPB_OK;
}

int gpb_comm_allreduce_max_f64(gpb_comm* c, double* value_inout) {
  return comm_host_reduce(c, value_inout, 1, ncclMax);
}
int gpb_comm_allreduce_sum_f64(gpb_comm* c, double* values_inout, int64_t count) {
  return comm_host_reduce(c, values_inout, count, ncclSum);
}
int gpb_comm_barrier(gpb_comm* c) {
  double z = 0.0;
  return comm_host_reduce(c, &z, 1, ncclSum);
}

int gpb_train(gpb_provider* p, gpb_comm* comm, const float* y_host, int64_t n,
              const gpb_train_options* opt, gpb_train_result* res) {
  clear_error();
  GPB_REQUIRE(p && y_host && opt && res, GPB_ERR_INVALID, "null argument");
  GPB_REQUIRE(n == p->n, GPB_ERR_INVALID, "y has %lld rows, provider has %lld", (long long)n,
              (long long)p->n);
  GPB_REQUIRE(opt->max_iterations >= 0 && opt->num_probes >= 1 && opt->max_cg_iter >= 1 &&
                  opt->max_tridiag_iter >= 0,
              GPB_ERR_INVALID, "invalid training options");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  Engine E;
  GPB_TRY(engine_from_comm(p, comm, E));
  return train_loop(E, y_host + E.r0, *opt, *res);
}

int gpb_bbmm(gpb_provider* p, gpb_comm* comm, const float* y_centered_host, int64_t n,
             int32_t num_probes, int32_t max_cg_iter, int32_t max_tridiag_iter, float cg_tol,
             int32_t precond_rank, int32_t iteration, double* nll_out, double* grads_out,
             double* logdet_out, double* inv_quad_out, int32_t* cg_iters_out) {
  clear_error();
  GPB_REQUIRE(p && y_centered_host && nll_out && grads_out, GPB_ERR_INVALID, "null argument");
  GPB_REQUIRE(n == p->n && num_probes >= 1, GPB_ERR_INVALID, "bad sizes");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  Engine E;
  GPB_TRY(engine_from_comm(p, comm, E));
  BBMMState S;
  GPB_TRY(S.ensure(E, 1 + num_probes, max_tridiag_iter));
  GPB_CHECK_CUDA(cudaMemcpyAsync(S.yc.ptr, y_centered_host + E.r0, E.nl * sizeof(float),
                                 cudaMemcpyHostToDevice, E.st));
  Precond P;
  GPB_TRY(precond_build(E, precond_rank, P));
  BBMMResult R;
  GPB_TRY(bbmm_step(E, precond_rank > 0 ? &P : nullptr, S, num_probes, max_cg_iter,
                    max_tridiag_iter, cg_tol, iteration, false, R));
  *nll_out = R.nll;
  for (int q = 0; q <= p->dk.nparams; ++q) grads_out[q] = R.grads[q];
  if (logdet_out) *logdet_out = R.logdet;
  if (inv_quad_out) *inv_quad_out = R.inv_quad;
  if (cg_iters_out) *cg_iters_out = R.cg_iters;
  return provider_check_device_error(p);
}

int gpb_precond_pivots(gpb_provider* p, gpb_comm* comm, int32_t rank, int64_t* pivots_out,
                       float* values_out, int32_t* actual_rank_out) {
  clear_error();
  GPB_REQUIRE(p && pivots_out && actual_rank_out && rank >= 1, GPB_ERR_INVALID, "bad arguments");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  Engine E;
  GPB_TRY(engine_from_comm(p, comm, E));
  Precond P;
  GPB_TRY(precond_build(E, rank, P, false));
  const int rmax = (int)std::min<int64_t>(rank, E.n);
  const int got = std::min(P.rank, rmax);
  std::vector<int64_t> piv(rmax);
  std::vector<float> val(rmax);
  GPB_CHECK_CUDA(cudaMemcpyAsync(piv.data(), P.piv.ptr, rmax * sizeof(int64_t),
                                 cudaMemcpyDeviceToHost, E.st));
  GPB_CHECK_CUDA(cudaMemcpyAsync(val.data(), (const int64_t*)P.piv.ptr + rmax,
                                 rmax * sizeof(float), cudaMemcpyDeviceToHost, E.st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(E.st));
  // The termination rule may report rank 1 with no accepted pivot (a zero
  // kernel); only picks the kernel accepted are returned.
  int accepted = 0;
  for (int m = 0; m < got; ++m) {
    if (!(val[m] >= 1e-10f)) break;
    pivots_out[m] = piv[m];
    if (values_out) values_out[m] = val[m];
    ++accepted;
  }
  *actual_rank_out = accepted;
  return provider_check_device_error(p);
}

int gpb_matvec_sharded(gpb_provider* p, gpb_comm* comm, float* out_local_dev,
                       const float* v_local_dev, int64_t ncols) {
  clear_error();
  GPB_REQUIRE(p && out_local_dev && v_local_dev && ncols >= 1, GPB_ERR_INVALID, "bad arguments");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  Engine E;
  GPB_TRY(engine_from_comm(p, comm, E));
  // Engine::matvec packs from its column argument, so stage the caller's
  // (read-only) block in a local copy.
  DBuf vloc;
  GPB_TRY(vloc.ensure(E.blk((int)ncols) + 16));
  GPB_TRY(k_copy(vloc.f(), v_local_dev, (int64_t)ncols * E.nl, E.st));
  GPB_TRY(E.matvec(vloc.f(), E.nl, (int)ncols, out_local_dev, E.nl));
  return provider_check_device_error(p);
}

int gpb_benchmark_forward_sharded(gpb_provider* p, gpb_comm* c, const float* v_dev, int64_t ncols,
                                  int32_t warmup, int32_t steps, int32_t flush_l2,
                                  double* step_ms_out, double* kernel_ms_out,
                                  int64_t* launches_out) {
  GPB_REQUIRE(p && v_dev && ncols >= 1 && steps >= 1 && warmup >= 0 && step_ms_out &&
                  kernel_ms_out && launches_out,
              GPB_ERR_INVALID, "bad benchmark arguments");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  Engine E;
  GPB_TRY(engine_from_comm(p, c, E));
  // Local row block of V and of the output.
  DBuf vloc, out, flush;
  GPB_TRY(vloc.ensure(E.blk((int)ncols) + 16));
  GPB_TRY(out.ensure(E.blk((int)ncols) + 16));
  for (int64_t col = 0; col < ncols; ++col)
    GPB_TRY(k_copy(vloc.f() + col * E.nl, v_dev + col * E.n + E.r0, E.nl, E.st));
  const size_t flush_bytes = (size_t)256 << 20;
  if (flush_l2) GPB_TRY(flush.ensure(flush_bytes));
  cudaEvent_t e0, e1, k0, k1;
  GPB_CHECK_CUDA(cudaEventCreate(&e0));
  GPB_CHECK_CUDA(cudaEventCreate(&e1));
  GPB_CHECK_CUDA(cudaEventCreate(&k0));
  GPB_CHECK_CUDA(cudaEventCreate(&k1));
  int status = GPB_OK;
  for (int it = 0; it < warmup + steps && status == GPB_OK; ++it) {
    if (flush_l2) cudaMemsetAsync(flush.ptr, it & 0xff, flush_bytes, E.st);
    if (c) {
      // barrier on the stream: a zero-byte style all-reduce keeps ranks in step
      ncclAllReduce(c->buf, c->buf, 1, ncclDouble, ncclSum, c->dist.comm, E.st);
    }
    const bool timed = it >= warmup;
    if (timed) {
      p->launches = 0;
      // Tile-kernel events (recorded by the first and last chunk's launch):
      // the rest of the step is packing and the NCCL exchange.
      p->tile_ev[0] = k0;
      p->tile_ev[1] = k1;
      cudaEventRecord(e0, E.st);
    }
    status = E.matvec(vloc.f(), E.nl, (int)ncols, out.f(), E.nl);
    p->tile_ev[0] = p->tile_ev[1] = nullptr;
    if (timed) {
      cudaEventRecord(e1, E.st);
      if (cudaEventSynchronize(e1) != cudaSuccess) {
        set_error("benchmark step failed: %s", cudaGetErrorString(cudaGetLastError()));
        status = GPB_ERR_CUDA;
        break;
      }
      float ms = 0.f, kms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      cudaEventElapsedTime(&kms, k0, k1);
      step_ms_out[it - warmup] = ms;
      kernel_ms_out[it - warmup] = kms;
      launches_out[it - warmup] = p->launches;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaEventDestroy(k0);
  cudaEventDestroy(k1);
  if (status != GPB_OK) return status;
  return provider_check_device_error(p);
}

}  // extern "C"
