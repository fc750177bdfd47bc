// Pivoted-Cholesky preconditioner state and operations (see precond.cu).
#pragma once

#include "engine.cuh"

namespace gpb {

struct LmcPrecond;  // sum-of-Kronecker Woodbury preconditioner (lmc.cu)

struct Precond {
  int rank = 0;        // actual rank; 0 = no preconditioner
  float noise = 0.f;
  double logdet = 0.0;  // log|L L^T + noise I|
  DBuf L;               // [rank][nl] (column k of L over this rank's rows)
  DBuf Minv;            // [rank][rank] float
  DBuf u;               // [t][rank] work
  DBuf diag, mask, scratch, keys;
  DBuf piv;             // [rank] int64 pivot indices in pick order, then [rank] float
                        // residual diagonal at each pick
  LmcPrecond* lmc = nullptr;  // when set, apply / sample / logdet are the LMC ones
};

// Greedy pivoted Cholesky of the provider's kernel; `finalize` = false stops
// after the factor L (no Woodbury inverse, no log-determinant).
int precond_build(Engine& E, int rank_req, Precond& P, bool finalize = true);
int precond_finalize(Engine& E, Precond& P);
int precond_apply(Engine& E, Precond& P, const float* v, float* out, int t);
int precond_sample(Engine& E, Precond& P, int num, uint64_t seed, float* out);
int lmc_precond_apply(Engine& E, LmcPrecond& P, const float* v, float* out, int t);
int lmc_precond_sample(Engine& E, LmcPrecond& P, int num, uint64_t seed, float* out);

}  // namespace gpb
