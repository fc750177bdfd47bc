// Engine: device-resident mBCG / BBMM, greedy pivoted-Cholesky preconditioner,
// LOVE, on one GPU or row-sharded over several GPUs of one box (NCCL).
//
// Row sharding: rank g owns training rows [r0, r1) of every n-length vector
// (x, r, z, p, Ap, L rows, Lanczos vectors). X is replicated (the provider
// holds all rows). Each matvec packs the local rows of the right-hand side
// into TMA tile rows and all-gathers the packed tiles, so every rank streams
// the full column side from its own HBM; column dot products are local
// partial sums followed by an all-reduce of t doubles.
#pragma once

#include <nccl.h>

#include <vector>

#include "provider.cuh"

namespace gpb {

struct Dist {
  ncclComm_t comm = nullptr;
  int rank = 0;
  int world = 1;
};

inline void shard_bounds(int64_t n, int world, int rank, int64_t* r0, int64_t* r1) {
  *r0 = n * rank / world;
  *r1 = n * (rank + 1) / world;
}

// Device buffer owned by the engine.
struct DBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  int ensure(size_t b);
  void release();
  float* f() const { return (float*)ptr; }
  double* d() const { return (double*)ptr; }
  ~DBuf() { release(); }
};

// Scratch shared by the reduction kernels.
struct Reducer {
  DBuf partial;  // doubles [blocks][k]
  DBuf counter;  // unsigned, reset by the last block
  DBuf sums;     // doubles [k]
  int ensure(int max_blocks, int k);
};

// Linear operator other than a single provider's K + noise (the LMC sum of
// Kronecker products); when set, Engine::matvec delegates to it.
struct LinOp {
  virtual ~LinOp() = default;
  // out = A v for [t][ld] blocks over this rank's rows.
  virtual int apply(const float* v, int64_t ld, int t, float* out, cudaStream_t st) = 0;
  // t probe columns ~ N(0, I) over this rank's rows, indexed so that every
  // sharding draws the same numbers.
  virtual int gaussian(float* out, int t, uint64_t seed, cudaStream_t st) = 0;
};

struct Engine {
  gpb_provider* p = nullptr;
  LinOp* op = nullptr;
  Dist dist;
  cudaStream_t st = nullptr;
  int64_t n = 0, r0 = 0, r1 = 0, nl = 0, nl_pad = 0;
  DBuf xv;          // packed column tiles [world * nl_pad][W]
  Reducer red;
  std::vector<double> host_sums;

  int init(gpb_provider* prov, const Dist& d);
  // Column-major local block [t][nl] helpers.
  size_t blk(int t) const { return (size_t)t * nl * sizeof(float); }

  // out = (K + noise) v for local rows; v_local [t][ld]; if `update_beta`
  // is non-null, first p = z + beta p (reference freeze rules) in place.
  int matvec(float* v_local, int64_t v_ld, int t, float* out, int64_t out_ld,
             const float* update_z = nullptr, const float* update_beta = nullptr);
  // sums[q*t + c] over global rows of a_q[c] . b_q[c] (npairs <= 3), left in
  // red.sums (device, doubles) and, if `to_host`, in host_sums.
  int coldots(int npairs, const float* const* a, const float* const* b, int64_t ld, int t,
              bool to_host);
  int allreduce_sum(double* dev, size_t count);
  int allreduce_sum_f(float* dev, size_t count);
  int allgather_cols(const float* local, int64_t ld_local, int t, float* full);
};

// Kernel launchers (engine_kernels.cu).
int k_fill(float* p, int64_t count, float v, cudaStream_t st);
int k_gaussian_tasks(float* out, int cols, int T, int64_t nl, int64_t n, int64_t r0, uint64_t seed,
                     cudaStream_t st);
int k_copy(float* dst, const float* src, int64_t count, cudaStream_t st);
int k_gaussian(float* out, int t, int64_t nl, int64_t ld, int64_t n_global, int64_t row0,
               uint64_t seed, cudaStream_t st);
int k_scale_cols(float* v, int64_t ld, int64_t nl, int t, const float* scale, int inverse,
                 cudaStream_t st);
int k_pack(const float* xs, int DP, float* v, int64_t v_ld, int c0, int tcols, int T, int64_t nl,
           int64_t nl_pad, float* dst, const float* upd_z, const float* upd_beta,
           cudaStream_t st, int layout = 0);
int k_coldots(int npairs, const float* const* a, const float* const* b, int64_t ld, int64_t nl,
              int t, Reducer& red, cudaStream_t st);
int k_cg_alpha(const float* rz_old, const double* pap, float* alpha, float* alpha_hist, int t,
               cudaStream_t st);
int k_cg_beta(float* rz_old, const double* rz_new, float* beta, float* beta_hist, int t,
              cudaStream_t st);
int k_cg_update(const float* alpha, const float* p, const float* Ap, float* x, float* r,
                int64_t nl, int64_t ld, int t, cudaStream_t st);
int k_sub(float* r, const float* a, int64_t count, cudaStream_t st);
int k_set_rz(float* rz, const double* sums, int t, cudaStream_t st);
// p = z + beta p with the reference's freeze rules (in place), [t][ld].
int k_update_p(float* p, const float* z, const float* beta, int64_t nl, int64_t ld, int t,
               cudaStream_t st);

// Preconditioner kernels.
int k_ltv(const float* L, int64_t nl, int rank, const float* v, int64_t ld, int t, Reducer& red,
          cudaStream_t st);  // red.sums[c*rank + k]
int k_woodbury_out(const float* v, int64_t ld, const float* L, int64_t nl, int rank,
                   const float* u, int t, float inv_noise, float* out, cudaStream_t st);
int k_minv_apply(const float* Minv, int rank, const double* w, int t, float* u, cudaStream_t st);
int k_ltl(const float* L, int64_t nl, int rank, Reducer& red, cudaStream_t st);
// out[c][i] = add_coef * src[c][i] + lu_coef * sum_k L[k][i] u[c][k]
int k_l_times_u(const float* L, int64_t nl, int rank, const float* u, int t, const float* src,
                int64_t ld, float add_coef, float lu_coef, float* out, cudaStream_t st);
int k_lz_plus_noise(const float* L, int64_t nl, int rank, const float* zr, int t,
                    const float* zn, float sqrt_noise, float* out, cudaStream_t st);

}  // namespace gpb
