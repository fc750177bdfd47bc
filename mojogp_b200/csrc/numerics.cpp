// Small dense host numerics in float64: symmetric tridiagonal eigensolver
// (implicit QL with Wilkinson shifts, the textbook method of the EISPACK
// tql2 family), Cholesky factor / inverse / log-determinant of small SPD
// matrices, and the SLQ log-determinant from CG tridiagonals.
//
// These replace the reference's native host routines
// (mojogp/kernels/native_numerics.mojo:271-518, 724-849;
//  kernels/pivoted_cholesky.mojo:1083-1207, 1411-1517).
#include "numerics.h"

#include <algorithm>
#include <cmath>
#include <vector>

namespace gpb {

static double hyp(double a, double b) {
  const double aa = std::fabs(a), bb = std::fabs(b);
  if (aa > bb) return aa * std::sqrt(1.0 + (bb / aa) * (bb / aa));
  if (bb == 0.0) return 0.0;
  return bb * std::sqrt(1.0 + (aa / bb) * (aa / bb));
}

bool tridiag_eig(const double* diag, const double* offdiag, int m, double* evals, double* evecs) {
  if (m <= 0) return true;
  std::vector<double> d(diag, diag + m), e(m, 0.0);
  for (int i = 0; i + 1 < m; ++i) e[i] = offdiag[i];
  // evecs: row-major m x m, column k = eigenvector k.
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < m; ++j) evecs[i * m + j] = (i == j) ? 1.0 : 0.0;
  const double eps = 2.220446049250313e-16;
  bool converged = true;
  for (int l = 0; l < m; ++l) {
    int iter = 0;
    while (true) {
      int mm = l;
      for (; mm < m - 1; ++mm) {
        const double dd = std::fabs(d[mm]) + std::fabs(d[mm + 1]);
        if (std::fabs(e[mm]) <= eps * dd) break;
      }
      if (mm == l) break;
      if (++iter > 60 * m) {
        converged = false;
        break;
      }
      double g = (d[l + 1] - d[l]) / (2.0 * e[l]);
      double r = hyp(g, 1.0);
      g = d[mm] - d[l] + e[l] / (g + (g >= 0 ? std::fabs(r) : -std::fabs(r)));
      double s = 1.0, c = 1.0, p = 0.0;
      int i = mm - 1;
      bool early = false;
      for (; i >= l; --i) {
        double f = s * e[i];
        const double b = c * e[i];
        r = hyp(f, g);
        e[i + 1] = r;
        if (r == 0.0) {
          d[i + 1] -= p;
          e[mm] = 0.0;
          early = true;
          break;
        }
        s = f / r;
        c = g / r;
        g = d[i + 1] - p;
        r = (d[i] - g) * s + 2.0 * c * b;
        p = s * r;
        d[i + 1] = g + p;
        g = c * r - b;
        for (int k = 0; k < m; ++k) {
          f = evecs[k * m + i + 1];
          evecs[k * m + i + 1] = s * evecs[k * m + i] + c * f;
          evecs[k * m + i] = c * evecs[k * m + i] - s * f;
        }
      }
      if (early) continue;
      d[l] -= p;
      e[l] = g;
      e[mm] = 0.0;
    }
  }
  // sort ascending with eigenvectors
  std::vector<int> idx(m);
  for (int i = 0; i < m; ++i) idx[i] = i;
  std::sort(idx.begin(), idx.end(), [&](int a, int b) { return d[a] < d[b]; });
  std::vector<double> v(evecs, evecs + (size_t)m * m);
  for (int k = 0; k < m; ++k) {
    evals[k] = d[idx[k]];
    for (int i = 0; i < m; ++i) evecs[i * m + k] = v[i * m + idx[k]];
  }
  return converged;
}

double slq_logdet(const std::vector<std::vector<double>>& diags,
                  const std::vector<std::vector<double>>& offdiags, int64_t n) {
  // Reference: native_numerics.mojo:403-518. Per probe: eigen-decompose T,
  // sum_i V[0,i]^2 log(lambda_i) over eigenvalues >= max(lambda_max,1e-10)*1e-6
  // and >= 0; probes with NaN/Inf entries are skipped; mean over valid probes
  // times n.
  double total = 0.0;
  int valid = 0;
  for (size_t p = 0; p < diags.size(); ++p) {
    const int m = (int)diags[p].size();
    if (m == 0) continue;
    bool bad = false;
    for (double v : diags[p])
      if (!std::isfinite(v)) bad = true;
    for (int i = 0; i + 1 < m; ++i)
      if (!std::isfinite(offdiags[p][i])) bad = true;
    if (bad) continue;
    std::vector<double> ev(m), V((size_t)m * m);
    tridiag_eig(diags[p].data(), offdiags[p].data(), m, ev.data(), V.data());
    double max_eig = 1e-10;
    for (int i = 0; i < m; ++i) max_eig = std::max(max_eig, ev[i]);
    const double clamp = max_eig * 1e-6;
    double term = 0.0;
    for (int i = 0; i < m; ++i) {
      const double lam = ev[i];
      if (lam < 0.0 || lam < clamp) continue;
      term += V[i] * V[i] * std::log(lam);
    }
    total += term;
    ++valid;
  }
  if (valid == 0) return 0.0;
  return (double)n * total / valid;
}

bool cholesky_lower(const double* A, int m, double* Lo) {
  for (int i = 0; i < m * m; ++i) Lo[i] = 0.0;
  for (int i = 0; i < m; ++i) {
    for (int j = 0; j <= i; ++j) {
      double s = A[i * m + j];
      for (int k = 0; k < j; ++k) s -= Lo[i * m + k] * Lo[j * m + k];
      if (i == j) {
        if (!(s > 0.0)) return false;
        Lo[i * m + i] = std::sqrt(s);
      } else {
        Lo[i * m + j] = s / Lo[j * m + j];
      }
    }
  }
  return true;
}

bool spd_inverse(const double* A, int m, double* Ainv, double* logdet) {
  std::vector<double> Lo((size_t)m * m), Li((size_t)m * m, 0.0);
  if (!cholesky_lower(A, m, Lo.data())) {
    // LU with partial pivoting fallback (matrix_inv_native / slogdet analogue).
    std::vector<double> a(A, A + (size_t)m * m), inv((size_t)m * m, 0.0);
    for (int i = 0; i < m; ++i) inv[i * m + i] = 1.0;
    double ld = 0.0;
    for (int c = 0; c < m; ++c) {
      int piv = c;
      for (int r = c + 1; r < m; ++r)
        if (std::fabs(a[r * m + c]) > std::fabs(a[piv * m + c])) piv = r;
      if (a[piv * m + c] == 0.0) return false;
      if (piv != c)
        for (int k = 0; k < m; ++k) {
          std::swap(a[c * m + k], a[piv * m + k]);
          std::swap(inv[c * m + k], inv[piv * m + k]);
        }
      const double dv = a[c * m + c];
      ld += std::log(std::fabs(dv));
      for (int k = 0; k < m; ++k) {
        a[c * m + k] /= dv;
        inv[c * m + k] /= dv;
      }
      for (int r = 0; r < m; ++r)
        if (r != c) {
          const double f = a[r * m + c];
          if (f != 0.0)
            for (int k = 0; k < m; ++k) {
              a[r * m + k] -= f * a[c * m + k];
              inv[r * m + k] -= f * inv[c * m + k];
            }
        }
    }
    std::copy(inv.begin(), inv.end(), Ainv);
    if (logdet) *logdet = ld;
    return true;
  }
  // Li = Lo^{-1} by forward substitution; Ainv = Li^T Li.
  for (int i = 0; i < m; ++i) {
    Li[i * m + i] = 1.0 / Lo[i * m + i];
    for (int j = 0; j < i; ++j) {
      double s = 0.0;
      for (int k = j; k < i; ++k) s += Lo[i * m + k] * Li[k * m + j];
      Li[i * m + j] = -s / Lo[i * m + i];
    }
  }
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < m; ++j) {
      double s = 0.0;
      for (int k = std::max(i, j); k < m; ++k) s += Li[k * m + i] * Li[k * m + j];
      Ainv[i * m + j] = s;
    }
  if (logdet) {
    double ld = 0.0;
    for (int i = 0; i < m; ++i) ld += std::log(Lo[i * m + i]);
    *logdet = 2.0 * ld;
  }
  return true;
}

}  // namespace gpb

extern "C" int gpb_slq_logdet(const double* diags, const double* offdiags, int32_t m,
                              int32_t num_probes, int64_t n, double* out) {
  if (!diags || !out || m < 0 || num_probes < 0 || (m > 1 && !offdiags)) return -1;
  std::vector<std::vector<double>> d(num_probes), e(num_probes);
  for (int p = 0; p < num_probes; ++p) {
    d[p].assign(diags + (size_t)p * m, diags + (size_t)(p + 1) * m);
    if (m > 1) e[p].assign(offdiags + (size_t)p * (m - 1), offdiags + (size_t)(p + 1) * (m - 1));
  }
  *out = gpb::slq_logdet(d, e, n);
  return 0;
}

extern "C" int gpb_tridiag_eig(const double* diag, const double* offdiag, int32_t m, double* evals,
                               double* evecs) {
  if (!diag || !evals || !evecs || m < 0 || (m > 1 && !offdiag)) return -1;
  return gpb::tridiag_eig(diag, offdiag, m, evals, evecs) ? 0 : -7;
}
