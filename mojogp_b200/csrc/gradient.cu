// Gradient matvecs.
//
// 1. gpb_gradient_matvec / gpb_fused_gradient_matvec keep the reference
//    layout out[p][c][i] = sum_j dK_ij/dtheta_p v[c][j]
//    (codegen_engine/emit/gpu_kernel.py:382-484, 878) for API parity; they
//    use the generic tree evaluator and are not on the training hot path.
// 2. gpb_gradient_bilinear is the training path: it fuses the two gradient
//    matvecs and the strided dot products that follow them in
//    combined_inv_quad_logdet.mojo:740-785 into one tiled pass that forms,
//    per parameter, sum_ij a_i dK_ij b_j directly, so the [P][t][n]
//    intermediate (1.1 GB at n=1e6, d=16, t=16) is never written.
#include <vector>

#include "provider.cuh"
#include "gradient_gram.cuh"

namespace gpb {

// ------------------------------------------------------------------ layout
__global__ void grad_matvec_ref_kernel(const float* __restrict__ X, int64_t n, int d,
                                       const float* __restrict__ v, int64_t ncols, int param_index,
                                       const __grid_constant__ DevKernel K, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float xi[GPB_MAX_DIM], xj[GPB_MAX_DIM], g[GPB_MAX_PARAMS];
  for (int k = 0; k < d; ++k) xi[k] = X[i * d + k];
  const int P = K.nparams;
  const int p_lo = param_index >= 0 ? param_index : 0;
  const int p_hi = param_index >= 0 ? param_index + 1 : P;
  for (int64_t c = 0; c < ncols; ++c) {
    float acc[GPB_MAX_PARAMS];
    for (int q = p_lo; q < p_hi; ++q) acc[q] = 0.f;
    for (int64_t j = 0; j < n; ++j) {
      for (int k = 0; k < d; ++k) xj[k] = X[j * d + k];
      tree_eval<true>(K, xi, xj, g);
      const float vj = v[c * n + j];
      for (int q = p_lo; q < p_hi; ++q) acc[q] = fmaf(g[q], vj, acc[q]);
    }
    for (int q = p_lo; q < p_hi; ++q) {
      const int64_t slot = param_index >= 0 ? 0 : q;
      out[(slot * ncols + c) * n + i] = acc[q];
    }
  }
}

// -------------------------------------------------------------- bilinear
// Accumulator layout per block: [2][NACC] (data, trace); NACC = DP + 2 for
// the fast leaves (A_k per dim, B = kernel value, C = RQ alpha term) and P
// for the generic evaluator.

template <int LEAF>
__device__ __forceinline__ void fast_value_and_phi(float u, const FastParams& fp, float& kap,
                                                   float& phi, float& h) {
  h = 0.f;
  if constexpr (LEAF == GPB_KERNEL_RBF) {
    kap = ex2_approx(-u);
    phi = kap * (2.f * kLn2);
  } else if constexpr (LEAF == GPB_KERNEL_MATERN12) {
    const float uu = fmaxf(u + fp.a1, fp.a1);
    const float rinv = rsqrtf(uu);
    const float r = uu * rinv;
    const float a = fp.a0 != 0.f ? fmaxf(-r, -20.f) : -r;
    kap = exp_fast(a);
    phi = kap * rinv;
  } else if constexpr (LEAF == GPB_KERNEL_MATERN32) {
    const float uu = fmaxf(u + fp.a1, fp.a1);
    const float r = uu * rsqrtf(uu);
    const float e = exp_fast(fmaxf(-r, -20.f));
    kap = (1.f + r) * e;
    phi = e;
  } else if constexpr (LEAF == GPB_KERNEL_MATERN52) {
    const float uu = fmaxf(u + fp.a1, fp.a1);
    const float r = uu * rsqrtf(uu);
    const float e = exp_fast(fmaxf(-r, -20.f));
    kap = (1.f + r + u * (1.f / 3.f)) * e;
    phi = (1.f + r) * e * (1.f / 3.f);
  } else {  // RQ
    const float base = fmaf(u, fp.a1, 1.f);
    const float lg = lg2_approx(base);
    kap = ex2_approx(-fp.a0 * lg);
    phi = kap / base;
    const float z = base - 1.f;
    h = z / base - lg * kLn2;
  }
}

template <int N>
__device__ __forceinline__ void block_reduce_store(float (&vals)[N], float* __restrict__ dst) {
  __shared__ float red[N][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
#pragma unroll
  for (int q = 0; q < N; ++q) {
    float x = vals[q];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) red[q][warp] = x;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < N; q += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < nwarps; ++w) s += red[q][w];
    dst[q] = s;
  }
}

template <int DP, int T, int LEAF>
__global__ void __launch_bounds__(128) bilinear_fast_kernel(
    const float* __restrict__ xrow, const float* __restrict__ a, int64_t nrow, int64_t a_ld,
    const float* __restrict__ xv, int ntiles_total, int tiles_per_split, FastParams fp, int tcols,
    int has_data, float* __restrict__ partial, int* err) {
  constexpr int R = 2;
  constexpr int BLK = 128;
  constexpr int W = packed_width(DP, T);
  constexpr int NACC = DP + 2;
  extern __shared__ __align__(128) float smem[];
  __shared__ __align__(8) uint64_t bars[kStages];
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  TileRing ring{smem, bars, xv, t0, ntiles, (uint32_t)(kJT * W)};
  ring.start();

  const int64_t row0 = (int64_t)blockIdx.x * (BLK * R) + threadIdx.x;
  float xi[R][DP], ai[R][T];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t i = row0 + (int64_t)r * BLK;
    const bool ok = i < nrow;
#pragma unroll
    for (int k = 0; k < DP; ++k) xi[r][k] = ok ? xrow[i * DP + k] : 0.f;
#pragma unroll
    for (int c = 0; c < T; ++c) ai[r][c] = (ok && c < tcols) ? a[c * a_ld + i] : 0.f;
  }
  float accd[NACC], acct[NACC];
#pragma unroll
  for (int q = 0; q < NACC; ++q) accd[q] = acct[q] = 0.f;

  const int nd = has_data;  // leading data columns in this chunk
  for (int kt = 0; kt < ntiles; ++kt) {
    const float* buf = ring.acquire(kt);
    if (buf == nullptr) {
      ring.fail(err);
      return;
    }
#pragma unroll 1
    for (int j = 0; j < kJT; ++j) {
      const float* rowp = buf + j * W;
      float xj[DP], bj[T];
#pragma unroll
      for (int k = 0; k < DP; ++k) xj[k] = rowp[k];
#pragma unroll
      for (int c = 0; c < T; ++c) bj[c] = rowp[DP + c];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float sq[DP];
        float u = 0.f;
#pragma unroll
        for (int k = 0; k < DP; ++k) {
          const float df = xi[r][k] - xj[k];
          sq[k] = df * df;
          u += sq[k];
        }
        float kap, phi, h;
        fast_value_and_phi<LEAF>(u, fp, kap, phi, h);
        float wd = 0.f, wt = 0.f;
#pragma unroll
        for (int c = 0; c < T; ++c) {
          if (c < nd)
            wd = fmaf(ai[r][c], bj[c], wd);
          else
            wt = fmaf(ai[r][c], bj[c], wt);
        }
        const float pd = phi * wd, pt = phi * wt;
#pragma unroll
        for (int k = 0; k < DP; ++k) {
          accd[k] = fmaf(pd, sq[k], accd[k]);
          acct[k] = fmaf(pt, sq[k], acct[k]);
        }
        accd[DP] = fmaf(kap, wd, accd[DP]);
        acct[DP] = fmaf(kap, wt, acct[DP]);
        if constexpr (LEAF == GPB_KERNEL_RQ) {
          const float kh = kap * h;
          accd[DP + 1] = fmaf(kh, wd, accd[DP + 1]);
          acct[DP + 1] = fmaf(kh, wt, acct[DP + 1]);
        }
      }
    }
    ring.release(kt);
  }
  float vals[2 * NACC];
#pragma unroll
  for (int q = 0; q < NACC; ++q) {
    vals[q] = accd[q];
    vals[NACC + q] = acct[q];
  }
  const int64_t bid = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
  block_reduce_store<2 * NACC>(vals, partial + bid * (2 * NACC));
}

// Generic bilinear: one row per thread; P-wide accumulators.
template <int DP, int T>
__global__ void __launch_bounds__(128) bilinear_generic_kernel(
    const float* __restrict__ xrow, const float* __restrict__ a, int64_t nrow, int64_t a_ld,
    const float* __restrict__ xv, int ntiles_total, int tiles_per_split,
    const __grid_constant__ DevKernel K, int tcols, int has_data, float* __restrict__ partial,
    int* err) {
  constexpr int BLK = 128;
  constexpr int W = packed_width(DP, T);
  extern __shared__ __align__(128) float smem[];
  __shared__ __align__(8) uint64_t bars[kStages];
  __shared__ float red[4 * 2 * GPB_MAX_PARAMS];
  const int split = blockIdx.y;
  const int t0 = split * tiles_per_split;
  const int ntiles = max(0, min(ntiles_total, t0 + tiles_per_split) - t0);
  TileRing ring{smem, bars, xv, t0, ntiles, (uint32_t)(kJT * W)};
  ring.start();
  const int P = K.nparams;

  const int64_t i = (int64_t)blockIdx.x * BLK + threadIdx.x;
  const bool ok = i < nrow;
  float xi[DP], ai[T];
  for (int k = 0; k < DP; ++k) xi[k] = ok ? xrow[i * DP + k] : 0.f;
  for (int c = 0; c < T; ++c) ai[c] = (ok && c < tcols) ? a[c * a_ld + i] : 0.f;
  float gd[GPB_MAX_PARAMS], gt[GPB_MAX_PARAMS], g[GPB_MAX_PARAMS];
  for (int q = 0; q < P; ++q) gd[q] = gt[q] = 0.f;
  const int nd = has_data;
  for (int kt = 0; kt < ntiles; ++kt) {
    const float* buf = ring.acquire(kt);
    if (buf == nullptr) {
      ring.fail(err);
      return;
    }
    for (int j = 0; j < kJT; ++j) {
      const float* rowp = buf + j * W;
      float xj[DP];
      for (int k = 0; k < DP; ++k) xj[k] = rowp[k];
      float wd = 0.f, wt = 0.f;
      for (int c = 0; c < T; ++c) {
        if (c < nd)
          wd = fmaf(ai[c], rowp[DP + c], wd);
        else
          wt = fmaf(ai[c], rowp[DP + c], wt);
      }
      tree_eval<true>(K, xi, xj, g);
      for (int q = 0; q < P; ++q) {
        gd[q] = fmaf(g[q], wd, gd[q]);
        gt[q] = fmaf(g[q], wt, gt[q]);
      }
    }
    ring.release(kt);
  }
  __syncthreads();
  // Fixed-order block reduction: each warp reduces with shuffles and writes
  // its own slot; thread q then sums the four warp slots in order.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int q = 0; q < 2 * P; ++q) {
    float x = (q < P) ? gd[q] : gt[q - P];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) red[warp * 2 * GPB_MAX_PARAMS + q] = x;
  }
  __syncthreads();
  const int64_t bid = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
  for (int q = threadIdx.x; q < 2 * P; q += BLK) {
    float s = 0.f;
    for (int w = 0; w < BLK / 32; ++w) s += red[w * 2 * GPB_MAX_PARAMS + q];
    partial[bid * (2 * P) + q] = s;
  }
}

__global__ void sum_partials_kernel(const float* __restrict__ partial, int64_t nblocks, int nacc,
                                    double* __restrict__ out) {
  // one thread per accumulator, fixed order over blocks
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nacc) return;
  double s = 0.0;
  for (int64_t b = 0; b < nblocks; ++b) s += (double)partial[b * nacc + q];
  out[q] = s;
}

template <int DP, int T, int LEAF>
int bilinear_fast_launch(const float* xrow, const float* a, int64_t nrow, int64_t a_ld,
                         const float* xv, int ntiles, const FastParams& fp, int tcols, int has_data,
                         float* partial, int64_t partial_cap, int* err, cudaStream_t st,
                         int64_t* nblocks_out) {
  auto kern = bilinear_fast_kernel<DP, T, LEAF>;
  constexpr int W = packed_width(DP, T);
  const size_t smem = (size_t)kStages * kJT * W * sizeof(float);
  static bool init = false;
  static int resident = 1, sms = 148;
  if (!init) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    GPB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kern, 128, smem));
    int dev = 0;
    GPB_CHECK_CUDA(cudaGetDevice(&dev));
    GPB_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (resident < 1) resident = 1;
    init = true;
  }
  const int64_t row_blocks = ceil_div(nrow, 256);
  int splits = kv_choose_splits(row_blocks, ntiles, resident, sms);
  constexpr int NACC2 = 2 * (DP + 2);
  while (splits > 1 && row_blocks * splits * NACC2 > partial_cap) --splits;
  const int tps = (int)ceil_div(ntiles, splits);
  splits = (int)ceil_div(ntiles, tps);
  GPB_REQUIRE(row_blocks * splits * NACC2 <= partial_cap, GPB_ERR_INVALID, "partial buffer too small");
  kern<<<dim3((unsigned)row_blocks, (unsigned)splits), 128, smem, st>>>(
      xrow, a, nrow, a_ld, xv, ntiles, tps, fp, tcols, has_data, partial, err);
  GPB_CHECK_CUDA(cudaGetLastError());
  *nblocks_out = row_blocks * splits;
  return GPB_OK;
}

template <int DP, int LEAF>
int bilinear_fast_t(int T, const float* xrow, const float* a, int64_t nrow, int64_t a_ld,
                    const float* xv, int ntiles, const FastParams& fp, int tcols, int has_data,
                    float* partial, int64_t cap, int* err, cudaStream_t st, int64_t* nb) {
  if (T == 4)
    return bilinear_fast_launch<DP, 4, LEAF>(xrow, a, nrow, a_ld, xv, ntiles, fp, tcols, has_data,
                                             partial, cap, err, st, nb);
  return bilinear_fast_launch<DP, 16, LEAF>(xrow, a, nrow, a_ld, xv, ntiles, fp, tcols, has_data,
                                            partial, cap, err, st, nb);
}

template <int LEAF>
int bilinear_fast_dp(int DP, int T, const float* xrow, const float* a, int64_t nrow, int64_t a_ld,
                     const float* xv, int ntiles, const FastParams& fp, int tcols, int has_data,
                     float* partial, int64_t cap, int* err, cudaStream_t st, int64_t* nb) {
#define GPB_BL_CASE(D)                                                                         \
  case D:                                                                                      \
    return bilinear_fast_t<D, LEAF>(T, xrow, a, nrow, a_ld, xv, ntiles, fp, tcols, has_data,   \
                                    partial, cap, err, st, nb);
  switch (DP) {
    GPB_BL_CASE(1)
    GPB_BL_CASE(2)
    GPB_BL_CASE(4)
    GPB_BL_CASE(8)
    GPB_BL_CASE(16)
    GPB_BL_CASE(32)
  }
#undef GPB_BL_CASE
  set_error("bilinear gradient: unsupported DP=%d", DP);
  return GPB_ERR_UNSUPPORTED;
}

template <int DP, int T>
int bilinear_generic_launch(const float* xrow, const float* a, int64_t nrow, int64_t a_ld,
                            const float* xv, int ntiles, const DevKernel& K, int tcols,
                            int has_data, float* partial, int64_t cap, int* err, cudaStream_t st,
                            int64_t* nb) {
  auto kern = bilinear_generic_kernel<DP, T>;
  constexpr int W = packed_width(DP, T);
  const size_t smem = (size_t)kStages * kJT * W * sizeof(float);
  static bool init = false;
  if (!init) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    init = true;
  }
  const int64_t row_blocks = ceil_div(nrow, 128);
  int splits = kv_choose_splits(row_blocks, ntiles, 2, 148);
  const int P2 = 2 * K.nparams;
  while (splits > 1 && row_blocks * splits * P2 > cap) --splits;
  const int tps = (int)ceil_div(ntiles, splits);
  splits = (int)ceil_div(ntiles, tps);
  GPB_REQUIRE(row_blocks * splits * P2 <= cap, GPB_ERR_INVALID, "partial buffer too small");
  kern<<<dim3((unsigned)row_blocks, (unsigned)splits), 128, smem, st>>>(
      xrow, a, nrow, a_ld, xv, ntiles, tps, K, tcols, has_data, partial, err);
  GPB_CHECK_CUDA(cudaGetLastError());
  *nb = row_blocks * splits;
  return GPB_OK;
}

int bilinear_generic_dp(int DP, int T, const float* xrow, const float* a, int64_t nrow, int64_t a_ld,
                        const float* xv, int ntiles, const DevKernel& K, int tcols, int has_data,
                        float* partial, int64_t cap, int* err, cudaStream_t st, int64_t* nb) {
#define GPB_BG_CASE(D)                                                                        \
  case D:                                                                                     \
    return T == 4 ? bilinear_generic_launch<D, 4>(xrow, a, nrow, a_ld, xv, ntiles, K, tcols,  \
                                                  has_data, partial, cap, err, st, nb)        \
                  : bilinear_generic_launch<D, 16>(xrow, a, nrow, a_ld, xv, ntiles, K, tcols, \
                                                   has_data, partial, cap, err, st, nb);
  switch (DP) {
    GPB_BG_CASE(4)
    GPB_BG_CASE(8)
    GPB_BG_CASE(16)
    GPB_BG_CASE(32)
    GPB_BG_CASE(64)
  }
#undef GPB_BG_CASE
  set_error("bilinear gradient: unsupported DP=%d", DP);
  return GPB_ERR_UNSUPPORTED;
}

// ------------------------------------------------- tensor-core RBF reduction
// Column tiles for gb_kernel: the Gram K.V B part, b (columns col0 .. col0 +
// ncol - 1 of the 16, the others zero) split into tf32 hi / lo, and
// B' = [1 | z | z^2] hi / lo along N (gradient_gram.cuh).
__global__ void pack_gb_kernel(const float* __restrict__ xs, int DP, const float* __restrict__ b,
                               int64_t b_ld, int col0, int ncol, int64_t n, int64_t npad,
                               float* __restrict__ dst) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= npad) return;
  float* base = dst + (j / 128) * gb_tile_floats(DP);
  const int jt = (int)(j % 128);
  const int KA = gram_kaug(DP);
  const bool live = j < n;
  float y[16];
  for (int q = 0; q < DP; ++q) y[q] = live ? xs[j * DP + q] : 0.f;
  for (int q = 0; q < DP; ++q) {
    const float bv = -2.f * y[q];
    const float hi = tf32_hi(bv);
    base[gram_xoff(jt, q)] = hi;
    base[128 * KA + gram_xoff(jt, q)] = bv - hi;
  }
  float e[8] = {1.f, 1.f, 1.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  gram_split3(gram_sqnorm(y, DP), e[3], e[4], e[5]);
  for (int q = 0; q < 8; ++q) base[gram_xoff(jt, DP + q)] = e[q];
  float* bb = base + gb_b_offset(DP);
  for (int c = 0; c < 16; ++c) {
    const float v = (live && c >= col0 && c < col0 + ncol) ? b[(int64_t)c * b_ld + j] : 0.f;
    const float hi = tf32_hi(v);
    bb[gram_xoff(jt, c)] = hi;
    bb[2048 + gram_xoff(jt, c)] = v - hi;
  }
  float* bp = base + gb_bp_offset(DP) + (jt / 8) * (8 * kGBN);
  const int k = jt % 8;
  for (int nn = 0; nn < 40; ++nn) {
    float f = 0.f;
    if (live) {
      if (nn == 0)
        f = 1.f;
      else if (nn <= DP)
        f = y[nn - 1];
      else if (nn <= 2 * DP)
        f = y[nn - 1 - DP] * y[nn - 1 - DP];
    }
    const float hi = tf32_hi(f);
    bp[gb_bp_off(nn, k)] = hi;
    bp[gb_bp_off(40 + nn, k)] = f - hi;
  }
}

bool gb_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("GPB_GRAD_TC");
    v = (e && e[0] == '0') ? 1 : 0;
  }
  return v == 1;
}

// One pass (data or probe columns) of the tensor-core reduction; adds the
// DP + 2 accumulators to acc_half.
template <int DP>
int gb_pass(gpb_provider* p, const float* xrow, const float* a, int64_t nrow, int64_t a_ld,
            const float* b, int col0, int ncol, double* acc_half, cudaStream_t st) {
  constexpr int NACC = DP + 2;
  const int64_t npad = round_up(std::max<int64_t>(p->n, 1), kJT);
  const int ntiles = (int)(npad / kJT);
  void* xv = nullptr;
  GPB_TRY(p->ws.get(WS_XV, (size_t)ntiles * gb_tile_floats(DP) * sizeof(float), &xv));
  pack_gb_kernel<<<(unsigned)ceil_div(npad, 128), 128, 0, st>>>(p->Xs_d, DP, b, p->n, col0, ncol,
                                                               p->n, npad, (float*)xv);
  GPB_CHECK_CUDA(cudaGetLastError());
  auto kern = gb_kernel<DP>;
  const size_t smem = (size_t)kGBStages * gb_tile_floats(DP) * sizeof(float);
  static bool init = false;
  static int sms = 148;
  if (!init) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int dev = 0, res = 0;
    GPB_CHECK_CUDA(cudaGetDevice(&dev));
    GPB_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    GPB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&res, kern, kGBThreads, smem));
    // The kernel allocates all 512 TMEM columns: two CTAs must never share an SM.
    GPB_REQUIRE(res == 1, GPB_ERR_UNSUPPORTED, "gradient tile kernel: %d CTAs per SM", res);
    init = true;
  }
  const int64_t row_blocks = ceil_div(nrow, kGBEpi);
  int splits = kv_choose_splits(row_blocks, ntiles, 1, sms);
  const int tps = (int)ceil_div(ntiles, splits);
  splits = (int)ceil_div(ntiles, tps);
  const int64_t nb = row_blocks * splits;
  void* part = nullptr;
  GPB_TRY(p->ws.get(WS_GRAD, (size_t)nb * NACC * sizeof(float) + 4096, &part));
  kern<<<dim3((unsigned)row_blocks, (unsigned)splits), kGBThreads, smem, st>>>(
      xrow, a, nrow, a_ld, col0, ncol, (const float*)xv, ntiles, tps, (float*)part, p->err_d);
  GPB_CHECK_CUDA(cudaGetLastError());
  p->launches += 2;
  void* sums = nullptr;
  GPB_TRY(p->ws.get(WS_MISC, (size_t)NACC * sizeof(double), &sums));
  sum_partials_kernel<<<1, 128, 0, st>>>((float*)part, nb, NACC, (double*)sums);
  GPB_CHECK_CUDA(cudaGetLastError());
  double tmp[NACC];
  GPB_CHECK_CUDA(cudaMemcpyAsync(tmp, sums, NACC * sizeof(double), cudaMemcpyDeviceToHost, st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  for (int q = 0; q < NACC; ++q) acc_half[q] += tmp[q];
  return GPB_OK;
}

// Sum over row range [row_begin, row_end) of the bilinear forms; results are
// accumulated (added) into data_out/trace_out (P doubles each, host).
int provider_bilinear_rows(gpb_provider* p, const float* a_dev, int64_t a_ld, const float* b_dev,
                           int64_t ncols, int64_t row_begin, int64_t row_end, double* data_out,
                           double* trace_out, cudaStream_t st) {
  return provider_bilinear_rows_nd(p, a_dev, a_ld, b_dev, ncols, row_begin, row_end, 1, data_out,
                                   trace_out, st);
}

int provider_bilinear_rows_nd(gpb_provider* p, const float* a_dev, int64_t a_ld, const float* b_dev,
                              int64_t ncols, int64_t row_begin, int64_t row_end, int64_t ndata,
                              double* data_out, double* trace_out, cudaStream_t st) {
  const int P = p->dk.nparams;
  for (int q = 0; q < P; ++q) data_out[q] = trace_out[q] = 0.0;
  const int64_t nrow = row_end - row_begin;
  if (nrow <= 0 || ncols <= 0) return GPB_OK;
  GPB_TRY(provider_refresh_xs(p));
  const int64_t npad = round_up(p->n, kJT);
  const int ntiles = (int)(npad / kJT);
  const bool fast = p->eval != kEvalGeneric;
  const int nacc = fast ? 2 * (p->DP + 2) : 2 * P;
  // Generic evaluator reads raw (unscaled) inputs: its plan's prescale is identity.
  const float* xrow = p->Xs_d + row_begin * p->DP;
  std::vector<double> acc(nacc, 0.0), tmp(nacc);
  // Tensor-core route: RBF on the Gram path (bounded prescaled norms), one
  // pass for the data columns and one for the probe columns of each chunk.
  const bool tc = p->eval == GPB_KERNEL_RBF && p->gram_ok && (p->DP == 8 || p->DP == 16) &&
                  !kv_tc_disabled() && !gb_disabled();
  for (int64_t c0 = 0; tc && c0 < ncols; c0 += 16) {
    const int tcols = (int)std::min<int64_t>(ncols - c0, 16);
    const int nd = (int)std::max<int64_t>(0, std::min<int64_t>(ndata - c0, tcols));
    const float* a_chunk = a_dev + c0 * a_ld;
    const float* b_chunk = b_dev + c0 * p->n;
    for (int half = 0; half < 2; ++half) {
      const int col0 = half == 0 ? 0 : nd, nc = half == 0 ? nd : tcols - nd;
      if (nc <= 0) continue;
      double* dst = acc.data() + half * (p->DP + 2);
      GPB_TRY(p->DP == 8 ? gb_pass<8>(p, xrow, a_chunk, nrow, a_ld, b_chunk, col0, nc, dst, st)
                         : gb_pass<16>(p, xrow, a_chunk, nrow, a_ld, b_chunk, col0, nc, dst, st));
    }
  }
  for (int64_t c0 = 0; !tc && c0 < ncols; c0 += 16) {
    const int64_t rem = ncols - c0;
    const int T = rem > 4 ? 16 : 4;
    const int tcols = (int)std::min<int64_t>(rem, T);
    const int W = packed_width(p->DP, T);
    void* xv = nullptr;
    GPB_TRY(p->ws.get(WS_XV, (size_t)npad * W * sizeof(float), &xv));
    GPB_TRY(launch_pack(p->Xs_d, p->DP, b_dev + c0 * p->n, p->n, tcols, T, p->n, npad, (float*)xv,
                        st));
    const int64_t cap = std::max<int64_t>((int64_t)ceil_div(nrow, 128) * 32 * nacc, 1 << 16);
    void* part = nullptr;
    GPB_TRY(p->ws.get(WS_GRAD, (size_t)cap * sizeof(float) + 4096, &part));
    int64_t nb = 0;
    // number of leading data columns inside this 16-column chunk
    const int has_data = (int)std::max<int64_t>(0, std::min<int64_t>(ndata - c0, tcols));
    const float* a_chunk = a_dev + c0 * a_ld;  // a_dev points at row_begin
    int s;
    switch (p->eval) {
      case GPB_KERNEL_RBF:
        s = bilinear_fast_dp<GPB_KERNEL_RBF>(p->DP, T, xrow, a_chunk, nrow, a_ld, (float*)xv, ntiles,
                                            p->fp, tcols, has_data, (float*)part, cap, p->err_d, st,
                                            &nb);
        break;
      case GPB_KERNEL_MATERN12:
        s = bilinear_fast_dp<GPB_KERNEL_MATERN12>(p->DP, T, xrow, a_chunk, nrow, a_ld, (float*)xv,
                                                 ntiles, p->fp, tcols, has_data, (float*)part, cap,
                                                 p->err_d, st, &nb);
        break;
      case GPB_KERNEL_MATERN32:
        s = bilinear_fast_dp<GPB_KERNEL_MATERN32>(p->DP, T, xrow, a_chunk, nrow, a_ld, (float*)xv,
                                                 ntiles, p->fp, tcols, has_data, (float*)part, cap,
                                                 p->err_d, st, &nb);
        break;
      case GPB_KERNEL_MATERN52:
        s = bilinear_fast_dp<GPB_KERNEL_MATERN52>(p->DP, T, xrow, a_chunk, nrow, a_ld, (float*)xv,
                                                 ntiles, p->fp, tcols, has_data, (float*)part, cap,
                                                 p->err_d, st, &nb);
        break;
      case GPB_KERNEL_RQ:
        s = bilinear_fast_dp<GPB_KERNEL_RQ>(p->DP, T, xrow, a_chunk, nrow, a_ld, (float*)xv, ntiles,
                                           p->fp, tcols, has_data, (float*)part, cap, p->err_d, st,
                                           &nb);
        break;
      default:
        s = bilinear_generic_dp(p->DP, T, xrow, a_chunk, nrow, a_ld, (float*)xv, ntiles, p->dk,
                                tcols, has_data, (float*)part, cap, p->err_d, st, &nb);
    }
    GPB_TRY(s);
    void* sums = nullptr;
    GPB_TRY(p->ws.get(WS_MISC, (size_t)nacc * sizeof(double), &sums));
    sum_partials_kernel<<<(unsigned)ceil_div(nacc, 128), 128, 0, st>>>((float*)part, nb, nacc,
                                                                       (double*)sums);
    GPB_CHECK_CUDA(cudaGetLastError());
    GPB_CHECK_CUDA(cudaMemcpyAsync(tmp.data(), sums, nacc * sizeof(double), cudaMemcpyDeviceToHost, st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(st));
    for (int q = 0; q < nacc; ++q) acc[q] += tmp[q];
  }
  if (!fast) {
    for (int q = 0; q < P; ++q) {
      data_out[q] = acc[q];
      trace_out[q] = acc[P + q];
    }
    return GPB_OK;
  }
  // Map fast accumulators to parameters.
  const DevKernel& K = p->dk;
  const LeafDesc& L = K.leaf[K.node_arg[0]];
  const float* prm = K.params + L.pofs;
  const int nl = L.ard ? L.ndims : 1;
  const int os_idx = L.pofs + ((L.type == GPB_KERNEL_RQ) ? nl + 1 : nl);
  const double M = p->os_eff;
  const int NA = p->DP + 2;
  for (int half = 0; half < 2; ++half) {
    const double* A = acc.data() + half * NA;
    double* dst = half == 0 ? data_out : trace_out;
    if (L.ard) {
      for (int k = 0; k < L.ndims; ++k) dst[L.pofs + k] = M * A[k] / prm[k];
    } else {
      double s = 0.0;
      for (int k = 0; k < L.ndims; ++k) s += A[k];
      dst[L.pofs] = M * s / prm[0];
    }
    dst[os_idx] = M / prm[os_idx - L.pofs] * A[p->DP];
    if (L.type == GPB_KERNEL_RQ) dst[L.pofs + nl] = M * A[p->DP + 1];
    if (K.nnodes == 2) {
      const int sc = K.node_arg[1];
      dst[sc] = M / K.params[sc] * A[p->DP];
    }
  }
  return GPB_OK;
}

}  // namespace gpb

using namespace gpb;

extern "C" {

int gpb_gradient_matvec(gpb_provider* p, float* out_dev, const float* v_dev, int64_t ncols,
                        int32_t param_index) {
  GPB_REQUIRE(p && out_dev && v_dev && ncols >= 0, GPB_ERR_INVALID, "bad arguments");
  GPB_REQUIRE(param_index >= -1 && param_index < p->dk.nparams, GPB_ERR_INVALID,
              "param_index %d out of range", param_index);
  if (ncols == 0) return GPB_OK;
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  grad_matvec_ref_kernel<<<(unsigned)ceil_div(p->n, 64), 64, 0, p->stream>>>(
      p->X_d, p->n, p->d, v_dev, ncols, param_index, p->dk, out_dev);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int gpb_fused_gradient_matvec(gpb_provider* p, float* out_dev, const float* v_dev, int64_t ncols) {
  return gpb_gradient_matvec(p, out_dev, v_dev, ncols, -1);
}

int gpb_gradient_bilinear(gpb_provider* p, const float* a_dev, const float* b_dev, int64_t ncols,
                          double* data_out, double* trace_out) {
  GPB_REQUIRE(p && a_dev && b_dev && data_out && trace_out && ncols >= 1, GPB_ERR_INVALID,
              "bad arguments");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  GPB_TRY(provider_bilinear_rows(p, a_dev, p->n, b_dev, ncols, 0, p->n, data_out, trace_out,
                                 p->stream));  // a at row 0
  return provider_check_device_error(p);
}

}  // extern "C"
