// Host float64 numerics used by the engine (see numerics.cpp).
#pragma once

#include <cstdint>
#include <vector>

namespace gpb {

// Eigen-decomposition of a symmetric tridiagonal matrix (diag m, offdiag m-1).
// evals ascending; evecs row-major m x m with column k the k-th eigenvector.
// Returns false if the iteration budget ran out (results are then approximate).
bool tridiag_eig(const double* diag, const double* offdiag, int m, double* evals, double* evecs);

// Stochastic Lanczos quadrature log-determinant from per-probe tridiagonals.
double slq_logdet(const std::vector<std::vector<double>>& diags,
                  const std::vector<std::vector<double>>& offdiags, int64_t n);

bool cholesky_lower(const double* A, int m, double* Lo);
// Inverse of a small SPD matrix (Cholesky; LU fallback) and its log-determinant.
bool spd_inverse(const double* A, int m, double* Ainv, double* logdet);

}  // namespace gpb
