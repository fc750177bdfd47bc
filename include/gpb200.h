/*
 * gpb200 — B200-native exact Gaussian-process hot path, C ABI.
 *
 * This is the drop-in boundary for MojoGP's JIT kernel-module / engine slot.
 * The reference splits the hot path into a per-kernel "provider" module whose
 * init_provider() returns a dict of raw function pointers
 * (mojogp/codegen_engine/emit/fn_ptr_module.py:998-1169) and an engine module
 * that consumes them (mojogp/kernels/jit/jit_engine_bindings.mojo:123-1234).
 * Each entry point below names the reference function-pointer or binding it
 * replaces. Conventions:
 *   - every function returns an int status (GPB_OK == 0, negative on error);
 *     gpb_last_error() returns the thread's last message;
 *   - "_dev" pointers are device pointers on the provider's device, "_host"
 *     pointers are host memory;
 *   - column blocks are column-major [ncols][n]: element (i, c) at c*n + i,
 *     matching the reference layout (gpu_kernel.py:225-228, 257-258);
 *   - X is row-major [n][d] float32;
 *   - calls on one provider are ordered on that provider's CUDA stream; call
 *     gpb_provider_synchronize() before reading results on the host.
 */
#ifndef GPB200_H
#define GPB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define GPB_OK 0
#define GPB_ERR_INVALID (-1)   /* bad argument (shape, null pointer, range) */
#define GPB_ERR_CUDA (-2)      /* CUDA runtime error */
#define GPB_ERR_NOMEM (-3)     /* device allocation failed */
#define GPB_ERR_UNSUPPORTED (-4)
#define GPB_ERR_DEVICE (-5)    /* a kernel reported a device-side error word */
#define GPB_ERR_NCCL (-6)
#define GPB_ERR_NUMERIC (-7)

/* ----------------------------------------------------------- kernel spec
 * A kernel tree is passed as a flat int32 program in post-order, replacing
 * the reference's SymPy -> Mojo codegen of the same tree
 * (mojogp/codegen_engine/expressions.py:77-650):
 *   word 0: GPB_SPEC_VERSION
 *   word 1: number of kernel parameters P (engine layout, see below)
 *   word 2: number of nodes
 *   then per node:
 *     leaf : GPB_NODE_LEAF, type, ard, param_offset, ndims, dims[ndims]
 *     sum  : GPB_NODE_SUM
 *     prod : GPB_NODE_PRODUCT
 *     scale: GPB_NODE_SCALE, param_index
 * Parameter layout per leaf follows mojogp/kernel.py:324-460
 * (get_param_names): ARD stationary [l_0..l_{k-1}, (period|alpha), os],
 * isotropic [ls, (period|alpha), os], linear [variance | var_0..var_{k-1}, os],
 * polynomial [degree, offset, os] (isotropic; degree is a fixed integer).
 * A scale node's parameter follows its child's parameters (kernel.py:553-556).
 */
#define GPB_SPEC_VERSION 1
#define GPB_NODE_LEAF 1
#define GPB_NODE_SUM 2
#define GPB_NODE_PRODUCT 3
#define GPB_NODE_SCALE 4

#define GPB_KERNEL_RBF 0
#define GPB_KERNEL_MATERN12 1
#define GPB_KERNEL_MATERN32 2
#define GPB_KERNEL_MATERN52 3
#define GPB_KERNEL_RQ 4
#define GPB_KERNEL_PERIODIC 5
#define GPB_KERNEL_LINEAR 6
#define GPB_KERNEL_POLYNOMIAL 7

#define GPB_MAX_LEAVES 8
#define GPB_MAX_NODES 16
#define GPB_MAX_PARAMS 96
#define GPB_MAX_DIM 64

/* noise modes (reference fn_ptr_module.py:297-322, modes 0 and 1) */
#define GPB_NOISE_SCALAR 0
#define GPB_NOISE_FIXED_VECTOR 1

typedef struct gpb_provider gpb_provider;

/* ---------------------------------------------------------------- library */
const char* gpb_version(void);
/* Copies the calling thread's last error message into buf (NUL-terminated). */
int gpb_last_error(char* buf, int64_t buf_len);
int gpb_device_count(int32_t* count_out);
/* Free and total device memory in bytes (cudaMemGetInfo) on `device`; no
 * reference counterpart (memory planning for row shards and for callers that
 * budget device memory up front). */
int gpb_device_mem_info(int32_t device, int64_t* free_out, int64_t* total_out);

/* Plain device-memory helpers so a NumPy host (no torch) can own device
 * buffers for the provider calls. */
int gpb_device_alloc(int32_t device, int64_t bytes, void** ptr_out);
int gpb_device_free(int32_t device, void* ptr);
int gpb_memcpy_h2d(int32_t device, void* dst_dev, const void* src_host, int64_t bytes);
int gpb_memcpy_d2h(int32_t device, void* dst_host, const void* src_dev, int64_t bytes);
int gpb_memset_d(int32_t device, void* dst_dev, int32_t value, int64_t bytes);
/* Page-lock (pin) / unpin an existing host buffer (cudaHostRegister /
 * cudaHostUnregister) so copies to and from it run at full PCIe/C2C rate and
 * stay asynchronous; no reference counterpart (the reference's host arrays
 * are NumPy-owned and pageable). */
int gpb_host_register(void* host_ptr, int64_t bytes);
int gpb_host_unregister(void* host_ptr);

/* ---------------------------------------------------------------- provider
 * Replaces init_provider() (fn_ptr_module.py:998-1115): copies X to the
 * device and keeps params/noise. noise_vec_host may be NULL (scalar noise);
 * otherwise it holds n fixed per-row noise variances (noise mode 1).
 */
int gpb_provider_create(const float* X_host, int64_t n, int32_t d, const int32_t* spec,
                        int32_t spec_len, const float* params_host, int32_t num_params,
                        float noise, const float* noise_vec_host, int32_t device,
                        gpb_provider** out);
/* Replaces destroy_provider() (fn_ptr_module.py:1183-1196). */
int gpb_provider_destroy(gpb_provider* p);
int gpb_provider_synchronize(gpb_provider* p);
/* Replaces impl_update_params (fn_ptr_module.py:651-664): host params, P floats. */
int gpb_update_params(gpb_provider* p, const float* params_host, int32_t num_params);
/* Replaces update_noise / get_noise / get_noise_mode. */
int gpb_update_noise(gpb_provider* p, float noise);
int gpb_get_noise(gpb_provider* p, float* noise_out);
int gpb_get_noise_mode(gpb_provider* p, int32_t* mode_out);
int gpb_get_num_params(gpb_provider* p, int32_t* num_out);
int gpb_get_params(gpb_provider* p, float* params_host, int32_t num_params);
/* Replaces get_diagonal_value (k(x,x) for a stationary kernel). */
int gpb_get_diagonal_value(gpb_provider* p, float* value_out);
/* Device pointer of the provider's X [n][d] (x_ptr in the provider dict). */
int gpb_get_x_ptr(gpb_provider* p, const float** x_dev_out);

/* Replaces impl_forward_matvec (fn_ptr_module.py:391-490):
 * out = K(X,X) V + sigma^2 V (scalar noise) or + diag(noise_vec) V. */
int gpb_forward_matvec(gpb_provider* p, float* out_dev, const float* v_dev, int64_t ncols);
/* Same, restricted to output rows [row_begin, row_end) (row-sharded matvec):
 * out has (row_end-row_begin) rows per column, v has all n rows. */
int gpb_forward_matvec_rows(gpb_provider* p, float* out_dev, const float* v_dev, int64_t ncols,
                            int64_t row_begin, int64_t row_end);
/* Host-buffer variant: copies V in, runs the matvec, copies out back. */
int gpb_forward_matvec_host(gpb_provider* p, float* out_host, const float* v_host,
                            int64_t ncols);
/* Replaces impl_cross_matvec (fn_ptr_module.py:576-616): out = K(X*, X) V,
 * xtest_dev row-major [n_test][d], out [ncols][n_test]. No noise term. */
int gpb_cross_matvec(gpb_provider* p, float* out_dev, const float* xtest_dev, const float* v_dev,
                     int64_t n_test, int64_t ncols);
/* Replaces impl_extract_diagonal / impl_extract_diagonal_test: k(x_i, x_i). */
int gpb_extract_diagonal(gpb_provider* p, float* diag_dev);
int gpb_extract_diagonal_test(gpb_provider* p, float* diag_dev, const float* xtest_dev,
                              int64_t n_test);
/* Kernel row K(X, x_piv) for one training index (no noise). */
int gpb_kernel_column(gpb_provider* p, float* out_dev, int64_t pivot);

/* Replaces impl_gradient_matvec (fn_ptr_module.py:511-540 single param) and
 * impl_fused_gradient_matvec: out[p][c][i] = sum_j dK_ij/dtheta_p V[j,c]
 * (all P params, layout [P][ncols][n]) — constrained-parameter derivatives. */
int gpb_gradient_matvec(gpb_provider* p, float* out_dev, const float* v_dev, int64_t ncols,
                        int32_t param_index);
int gpb_fused_gradient_matvec(gpb_provider* p, float* out_dev, const float* v_dev,
                              int64_t ncols);
/* Fused bilinear gradient reduction (no [P][t][n] intermediate). With a and b
 * column-major [ncols][n]:
 *   data_out[p]  = sum_ij a[0,i] dK_ij/dtheta_p b[0,j]
 *   trace_out[p] = sum_{c>=1} sum_ij a[c,i] dK_ij/dtheta_p b[c,j]
 * These are exactly the dot products the reference forms after its two fused
 * gradient matvecs (combined_inv_quad_logdet.mojo:740-785). Outputs are host
 * arrays of P floats; the call synchronizes. */
int gpb_gradient_bilinear(gpb_provider* p, const float* a_dev, const float* b_dev, int64_t ncols,
                          double* data_out, double* trace_out);

/* Replaces benchmark_provider_ops (jit_engine_bindings.mojo:439-567) for the
 * forward op: runs warmup + steps matvecs on the provider's stream and
 * reports, per timed step, the CUDA-event time of the whole step and of the
 * tiled kernel(s) alone, and the number of kernels launched. With flush_l2
 * a 256 MB buffer is rewritten before every step (outside the timed events). */
int gpb_benchmark_forward(gpb_provider* p, const float* v_dev, float* out_dev, int64_t ncols,
                          int32_t warmup, int32_t steps, int32_t flush_l2, double* step_ms_out,
                          double* kernel_ms_out, int64_t* launches_out);

/* FP32 (FFMA) throughput probe on `device`: the measured denominator of the
 * matvec roofline. No reference counterpart (measurement utility). */
int gpb_measure_fp32_peak(int32_t device, double* tflops_out, double* ms_out);

/* ------------------------------------------------------- multi-GPU comm
 * One communicator per process-per-GPU (NCCL over NVLink/NVSwitch). The
 * 128-byte unique id is created on rank 0 (gpb_comm_unique_id) and shared
 * with the other ranks by the host (any transport), then every rank calls
 * gpb_comm_init. No reference counterpart: MojoGP is single-GPU. */
typedef struct gpb_comm gpb_comm;
#define GPB_COMM_ID_BYTES 128
int gpb_comm_unique_id(uint8_t* id_out /* GPB_COMM_ID_BYTES */);
int gpb_comm_init(const uint8_t* id, int32_t world, int32_t rank, int32_t device, gpb_comm** out);
int gpb_comm_destroy(gpb_comm* c);
/* Host-value collectives for harness use (timing max, barriers). */
int gpb_comm_allreduce_max_f64(gpb_comm* c, double* value_inout);
int gpb_comm_allreduce_sum_f64(gpb_comm* c, double* values_inout, int64_t count);
int gpb_comm_barrier(gpb_comm* c);
/* One row-sharded (K + noise I) V product, as every mBCG iteration runs it
 * (no reference counterpart; the reference is single-GPU): each rank passes
 * its rows [n*rank/world, n*(rank+1)/world) of the ncols columns
 * (v_local_dev [ncols][n_local]) and receives the same rows of the product
 * (out_local_dev [ncols][n_local]); the column side is all-gathered over
 * NCCL. comm NULL = one GPU (n_local = n). */
int gpb_matvec_sharded(gpb_provider* p, gpb_comm* comm, float* out_local_dev,
                       const float* v_local_dev, int64_t ncols);
/* Row-sharded forward matvec benchmark: each rank computes rows
 * [n*rank/world, n*(rank+1)/world) of (K + noise) V and all-gathers the packed
 * output blocks, i.e. one CG-iteration matvec. Same outputs as
 * gpb_benchmark_forward. */
int gpb_benchmark_forward_sharded(gpb_provider* p, gpb_comm* c, const float* v_dev, int64_t ncols,
                                  int32_t warmup, int32_t steps, int32_t flush_l2,
                                  double* step_ms_out, double* kernel_ms_out,
                                  int64_t* launches_out);

/* ------------------------------------------------------------- training
 * Replaces engine.train (jit_engine_bindings.mojo:123-432 ->
 * jit_training.mojo:274-1008): Adam over softplus-raw kernel params, noise and
 * a constant mean; per iteration one BBMM step (probes, mBCG with tridiagonal
 * capture, SLQ log-det, fused gradient reduction) with a greedy pivoted-
 * Cholesky preconditioner rebuilt when parameters move by more than
 * precond_rebuild_threshold. With comm != NULL the rows are sharded. */
typedef struct {
  int32_t max_iterations;
  float learning_rate;
  int32_t num_probes;
  int32_t max_cg_iter;
  float cg_tol;
  int32_t precond_rank;
  int32_t max_tridiag_iter;
  float precond_rebuild_threshold;
  int32_t use_cosine_lr;
  int32_t use_preconditioner;
  int32_t learn_noise;
  float init_mean;
  int32_t enable_early_stopping;
  int32_t early_stop_patience;
  float early_stop_tol;
  int32_t verbose;
  const uint8_t* trainable_mask; /* num_params entries (1 = train) or NULL */
} gpb_train_options;

typedef struct {
  float final_nll;       /* best NLL seen (per sample) */
  float noise;
  float mean;
  int32_t iterations;
  int32_t converged;
  float* params;         /* [num_params], caller-allocated */
  float* nll_history;    /* [max_iterations] */
  double* iter_times_ms; /* [max_iterations] */
  int32_t* cg_iterations;/* [max_iterations] */
  float* alpha;          /* [n] best-iteration (K + noise)^{-1}(y - mean), or NULL */
  int32_t alpha_valid;
  int32_t precond_build_count;
  double precond_build_ms;
  int32_t precond_rank;
  int32_t* tile_layouts; /* [max_iterations] tile kernel of the 16-column K.V chunks in each
                            iteration (gpb_matvec_layout codes), or NULL */
} gpb_train_result;

int gpb_train(gpb_provider* p, gpb_comm* comm, const float* y_host, int64_t n,
              const gpb_train_options* opt, gpb_train_result* res);

/* One BBMM evaluation at the provider's current parameters (no optimizer
 * step): NLL and gradients w.r.t. the constrained kernel params and noise.
 * Replaces bbmm_with_precond (combined_inv_quad_logdet.mojo:452-1136). grads
 * has num_params + 1 entries (noise last). */
int gpb_bbmm(gpb_provider* p, gpb_comm* comm, const float* y_centered_host, int64_t n,
             int32_t num_probes, int32_t max_cg_iter, int32_t max_tridiag_iter, float cg_tol,
             int32_t precond_rank, int32_t iteration, double* nll_out, double* grads_out,
             double* logdet_out, double* inv_quad_out, int32_t* cg_iters_out);

/* The greedy pivoted-Cholesky pivots at the provider's current parameters:
 * the preconditioner build of gpb_bbmm / gpb_train (precond_method 0,
 * pivoted_cholesky.mojo:772-1050 with the argmax of 500-609: largest residual
 * diagonal among unused rows, lowest index on ties, stop when it falls below
 * 1e-10) run alone. pivots_out / values_out (values_out may be NULL) receive,
 * in pick order, up to `rank` global row indices and the residual diagonal
 * each was picked at; *actual_rank_out = how many were accepted. The
 * reference keeps its pivots internal; this entry point exists so callers and
 * tests can compare pivot lists. With comm != NULL the rows are sharded and
 * every rank returns the same list. */
int gpb_precond_pivots(gpb_provider* p, gpb_comm* comm, int32_t rank, int64_t* pivots_out,
                       float* values_out, int32_t* actual_rank_out);

/* Host-only numerics exposed for testing (no GPU needed): the SLQ
 * log-determinant from per-probe tridiagonals (diags [num_probes][m],
 * offdiags [num_probes][m-1]; native_numerics.mojo:403-518) and the
 * symmetric tridiagonal eigensolver (native_numerics.mojo:724-849). */
int gpb_slq_logdet(const double* diags, const double* offdiags, int32_t m, int32_t num_probes,
                   int64_t n, double* out);
int gpb_tridiag_eig(const double* diag, const double* offdiag, int32_t m, double* evals,
                    double* evecs);

/* Replaces kernel_gpu_gaussian (pivoted_cholesky.mojo:51-86): counter-hash
 * Box-Muller normals for indices [0, count) with `seed`, copied to host. */
int gpb_hash_gaussian(int32_t device, float* out_host, int64_t count, uint64_t seed);

/* ----------------------------------------------------------- prediction
 * Replaces the engine's alpha solve (jit_prediction.mojo:681-806): CG on
 * (K + noise I) alpha = y - mean with the relative-residual stop rule.
 * alpha_host_out has n entries (all rows, also when sharded). */
int gpb_compute_alpha(gpb_provider* p, gpb_comm* comm, const float* y_centered_host, int64_t n,
                      int32_t max_cg_iter, float cg_tol, float* alpha_host_out,
                      int32_t* iters_out);

/* Replaces prepare_prediction_cache / predict_with_cache /
 * destroy_prediction_cache (jit_engine_bindings.mojo:636-942): holds alpha and
 * the LOVE inverse root S ([love_rank][n], S S^T ~ (K + noise I)^{-1},
 * jit_prediction.mojo:974-1177) on the device. root_host may supply a
 * previously exported root; NULL computes it (Lanczos with full
 * re-orthogonalisation). love_rank 0 = mean only. */
typedef struct gpb_prediction_cache gpb_prediction_cache;
int gpb_prediction_cache_create(gpb_provider* p, gpb_comm* comm, const float* alpha_host,
                                float mean, int32_t love_rank, const float* root_host,
                                gpb_prediction_cache** out);
int gpb_prediction_cache_root(gpb_prediction_cache* c, float* root_host_out);
/* mean = K(X*, X) alpha + mean; var = max(k** - |K(X*, X) S|^2, 1e-10) + noise
 * (jit_prediction.mojo:211-232, 1236-1344, 2048-2051). var_out may be NULL. */
int gpb_predict_with_cache(gpb_prediction_cache* c, const float* xtest_host, int64_t n_test,
                           float* mean_out, float* var_out);
int gpb_prediction_cache_destroy(gpb_prediction_cache* c);
/* Replaces predict_variance_exact_jit (jit_prediction.mojo:1352-1788) with the
 * noise add of predict_from_alpha (2048-2051): per block of block_cols (<= 0:
 * min(n_test, 512)) test points, K(X, X*) is filled, (K + noise I) V = K(X, X*)
 * is solved by batched CG (pivoted-Cholesky preconditioner of rank
 * precond_rank when > 0, relative stop cg_tol), and
 * var = max(k(x*, x*) - K(x*, X) v, 1e-10) + noise. Training rows are sharded
 * over comm (NULL = one GPU); every rank returns all n_test variances. */
int gpb_predict_exact_variance(gpb_provider* p, gpb_comm* comm, const float* xtest_host,
                               int64_t n_test, int32_t block_cols, int32_t max_cg_iter,
                               float cg_tol, int32_t precond_rank, float* var_out,
                               int32_t* cg_iters_out);

/* ------------------------------------------------------------------ LMC
 * Linear model of coregionalisation over R latent providers (same X, n, device):
 * K_full = sum_s (A_s (x) K_s) + diag(noise_t (x) 1_n) on task-blocked vectors
 * (element (t, i) at t*n + i). Replaces JITLMCGradientAdapter
 * (jit_lmc.mojo:131-540) and the LMC kernels (lmc_provider.mojo:45-267).
 * Latent providers contribute K_s without their own noise. */
typedef struct gpb_lmc gpb_lmc;
int gpb_lmc_create(gpb_provider* const* providers, int32_t num_latents, int32_t num_tasks,
                   gpb_lmc** out);
/* Row-sharded LMC (no reference counterpart): rank g owns data rows
 * [n g / W, n (g+1) / W) of every task, so device-side column blocks
 * (gpb_lmc_matvec, gpb_lmc_precond_apply / _sample) are this rank's
 * [ncols][T][n_local]; host-side y / alpha / rhs stay full [T][n] on every
 * rank. comm NULL = one GPU (same as gpb_lmc_create). */
int gpb_lmc_create_sharded(gpb_provider* const* providers, int32_t num_latents, int32_t num_tasks,
                           gpb_comm* comm, gpb_lmc** out);
int gpb_lmc_destroy(gpb_lmc* h);
/* A [R][T][T] (symmetric PSD coregionalisation matrices), noise [T]. */
int gpb_lmc_set_coregion(gpb_lmc* h, const float* A, const float* noise);
/* out = K_full v for ncols task-blocked columns [ncols][T][n] (device). */
int gpb_lmc_matvec(gpb_lmc* h, float* out_dev, const float* v_dev, int64_t ncols);
/* One BBMM evaluation on the LMC operator (combined_inv_quad_logdet.mojo:452
 * with jit_lmc.mojo:582-691 gradients): NLL per nT, gradients w.r.t. every
 * latent's kernel params (concatenated), A_s [R][T][T], per-task noise [T],
 * per-task sum(alpha) [T]; alpha_out [T*n] optional. recycle != 0 warm-starts
 * from the previous call's solution. */
int gpb_lmc_bbmm(gpb_lmc* h, const float* y_centered_host, int32_t num_probes, int32_t max_cg_iter,
                 int32_t max_tridiag_iter, float cg_tol, int32_t iteration, int32_t recycle,
                 double* nll_out, double* kernel_grads_out, double* grad_A_out,
                 double* grad_noise_out, double* sum_alpha_out, float* alpha_out,
                 int32_t* cg_iters_out);
/* Sum-of-Kronecker Woodbury preconditioner (lmc_preconditioner.mojo:143-470,
 * built as in jit_lmc.mojo:848-900): P = sum_s A_s (x) L_s L_s^T + D with L_s
 * the rank-`rank` pivoted-Cholesky factor of K_s, from the current A_s and
 * noise. Once built, gpb_lmc_bbmm preconditions with it (probes ~ N(0, P),
 * log|P| added) until rebuilt; rank <= 0 removes it. ranks_out [R] (actual
 * per-latent ranks) and logdet_out (log|P|) may be NULL. */
int gpb_lmc_build_precond(gpb_lmc* h, int32_t rank, int32_t* ranks_out, double* logdet_out);
/* out = P^{-1} v for ncols task-blocked device columns (apply_precond,
 * lmc_preconditioner.mojo:397-560). */
int gpb_lmc_precond_apply(gpb_lmc* h, float* out_dev, const float* v_dev, int64_t ncols);
/* num probes ~ N(0, P): D^{1/2} eps + U omega with counter-hash Gaussians
 * (omega seed `seed`, eps seed `seed + 1e6`) in place of the reference's host
 * generator (sample_probes, lmc_preconditioner.mojo:567-719). */
int gpb_lmc_precond_sample(gpb_lmc* h, float* out_dev, int32_t num, uint64_t seed);
/* K_full^{-1} rhs by CG (relative-residual stop), rhs and x [T*n] host. */
int gpb_lmc_solve(gpb_lmc* h, const float* rhs_host, int32_t max_cg_iter, float cg_tol,
                  float* x_host_out, int32_t* iters_out);

/* Exact LMC posterior variance (_predict_lmc_full_exact_variance_backend,
 * mojogp/multi_output_gp.py:4360-4519): var[c][t] = max(sum_s A_s[t][t]
 * k_s(x*_c, x*_c) - r^T K_full^{-1} r + noise_t, 1e-10) with
 * r = sum_s k_s(X, x*_c) (x) A_s[:, t]. Test points are solved in blocks of
 * block_cols / T points (block_cols <= 0: 512) x all T tasks by batched CG
 * (relative stop cg_tol; the LMC preconditioner when built). xtest [n_test][d]
 * host, var_out [n_test][T] host. Every rank of a sharded handle returns all. */
int gpb_lmc_predict_exact_variance(gpb_lmc* h, const float* xtest_host, int64_t n_test,
                                   int32_t block_cols, int32_t max_cg_iter, float cg_tol,
                                   float* var_out, int32_t* cg_iters_out);

/* Tensor-core self-test (no reference counterpart): one 128x16x8 tcgen05
 * kind::tf32 MMA from shared-memory operands, A [128][8], B [16][8] row-major
 * host arrays, D = A B^T [128][16]. variant 0 = the operand layout the
 * library's tensor-core kernels use; variant 2 reads A from TMEM. */
int gpb_tc_selftest(int32_t device, int32_t variant, const float* a_host, const float* b_host,
                    float* d_host);

/* Tile kernel the forward matvec uses for its first 16 columns (no reference
 * counterpart; diagnostics and tests): 0 scalar FFMA, 1 paired-row FFMA2,
 * 2 tensor-core contraction, 3 Gram form on tf32 operands (both contractions
 * on the tensor core, chosen only for bounded prescaled input norms, when
 * GPB_KV_GRAMH=0, and by default for the Matern and RQ leaves), 4 narrow Gram form (tensor-core distances, fp32 CUDA-core
 * contraction; 1-column chunks), 5 Gram form on fp16 operands (the default
 * for RBF where 3 applies; every Gram leaf with GPB_KV_GRAMH=2). */
int gpb_matvec_layout(gpb_provider* p, int64_t ncols, int32_t* layout);

/* Same result as gpb_forward_matvec, on the same tile kernel, but the call
 * allocates no device memory: all scratch lives in one fixed 32 MiB array
 * compiled into the library, held on every GPU that uses it until the process
 * exits. For callers that must not allocate while they run (an external
 * memory pool or arena, or code where an allocation's implicit
 * synchronisation is not allowed). No counterpart in the reference.
 * Limit: 64 + S + round_up(n, 128) * W floats must fit in 8 Mi floats, where
 * W is the widest packed row over the call's 16-column chunks for either
 * outcome of the Gram norm check (48 at d <= 16, t = 16; 80 at d 17..32 when
 * a 5..8-column chunk follows)
 * and S = n * DP (DP = padded input dims) only when the provider's prescaled
 * inputs are stale (no product since the last parameter update). That is
 * about 174k rows at d = 16, t = 16 (131k when stale) and 104k rows at d = 32
 * (75k when stale); larger n is rejected with GPB_ERR_INVALID. A stale call
 * reduces the input norms itself, with one stream synchronisation. The first
 * call on a device loads the array's module, so make that first call before
 * any stream capture. Calls share the array: calls that overlap on the GPU
 * race and must be ordered by the caller. */
int gpb_forward_matvec_noalloc(gpb_provider* p, float* out_dev, const float* v_dev, int64_t ncols);

#ifdef __cplusplus
}
#endif

#endif /* GPB200_H */
