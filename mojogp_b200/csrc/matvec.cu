// Matvec plumbing: split selection, deterministic split reduction, input
// prescaling and column packing for the tiled K·V kernels.
#include "kv_launch.cuh"
#include "matvec.cuh"
#include "kv_tiles_tc.cuh"
#include "kv_tiles_gram.cuh"
#include "kv_tiles_gramh.cuh"

#include <cstdlib>

namespace gpb {

int launch_kv(const KvLaunch& L) {
  switch (L.eval) {
    case GPB_KERNEL_RBF: return launch_kv_rbf(L);
    case GPB_KERNEL_MATERN12: return launch_kv_m12(L);
    case GPB_KERNEL_MATERN32: return launch_kv_m32(L);
    case GPB_KERNEL_MATERN52: return launch_kv_m52(L);
    case GPB_KERNEL_RQ: return launch_kv_rq(L);
    case kEvalGeneric: return launch_kv_generic(L);
  }
  set_error("unknown evaluator %d", L.eval);
  return GPB_ERR_INVALID;
}

int kv_choose_splits(int64_t row_blocks, int ntiles, int resident_per_sm, int num_sms) {
  const int64_t slots = (int64_t)resident_per_sm * num_sms;
  // Each split should still stream a handful of tiles through the TMA ring.
  const int max_by_tiles = ntiles / 4 > 1 ? ntiles / 4 : 1;
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= 32 && s <= max_by_tiles; ++s) {
    const int64_t blocks = row_blocks * s;
    const int64_t waves = ceil_div(blocks, slots);
    // time ~ waves * (work per block) ~ waves / s; small penalty per split
    // for the partial-sum traffic and reduction.
    const double cost = (double)waves / s * (1.0 + 0.004 * (s - 1));
    if (cost < best_cost * 0.995) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

__global__ void kv_reduce_kernel(const float* __restrict__ part, int splits, int T, int tcols,
                                 int64_t nrow, TileEpilogue ep) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)tcols * nrow;
  if (idx >= total) return;
  const int c = (int)(idx / nrow);
  const int64_t i = idx - (int64_t)c * nrow;
  float s = 0.f;
  for (int sp = 0; sp < splits; ++sp) s += part[((int64_t)sp * T + c) * nrow + i];
  float o = ep.scale * s;
  if (ep.noise_v) {
    const float nz = ep.noise_vec ? ep.noise_vec[i] : ep.noise;
    o = fmaf(nz, ep.noise_v[c * ep.noise_ld + i], o);
  }
  ep.out[c * ep.out_ld + i] = o;
}

int launch_kv_reduce(const KvLaunch& L, int splits) {
  const int64_t total = (int64_t)L.tcols * L.nrow;
  if (total == 0) return GPB_OK;
  const int bs = 256;
  kv_reduce_kernel<<<(unsigned)ceil_div(total, bs), bs, 0, L.stream>>>(L.partial, splits, L.T,
                                                                      L.tcols, L.nrow, L.ep);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// xs[i][k] = X[i][dims[k]] * scale[k] for k < nd, 0 for nd <= k < DP.
__global__ void prescale_kernel(const float* __restrict__ X, int64_t n, int d, PrescaleSpec ps,
                                float* __restrict__ xs) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = n * ps.DP;
  if (idx >= total) return;
  const int64_t i = idx / ps.DP;
  const int k = (int)(idx - i * ps.DP);
  xs[idx] = (k < ps.nd) ? X[i * d + ps.dims[k]] * ps.scale[k] : 0.f;
}

int launch_prescale(const float* X, int64_t n, int d, const PrescaleSpec& ps, float* xs,
                    cudaStream_t stream) {
  const int64_t total = n * ps.DP;
  if (total == 0) return GPB_OK;
  prescale_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, stream>>>(X, n, d, ps, xs);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// Packed column rows: xv[j] = [xs[j][0..DP), v[c0+c][j] for c < tcols, 0...]
// for j < n, zero rows for n <= j < npad (their v = 0, so they add nothing).
__global__ void pack_kernel(const float* __restrict__ xs, int DP, const float* __restrict__ v,
                            int64_t v_ld, int tcols, int64_t n, int64_t npad, int W,
                            float* __restrict__ xv) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= npad) return;
  float* row = xv + j * W;
  if (j < n) {
    for (int k = 0; k < DP; ++k) row[k] = xs[j * DP + k];
    for (int c = 0; c < W - DP; ++c) row[DP + c] = (c < tcols) ? v[c * v_ld + j] : 0.f;
  } else {
    for (int k = 0; k < W; ++k) row[k] = 0.f;
  }
}

// Paired-row layout: every value twice, x' negated (kv_tiles_x2.cuh).
__global__ void pack_dup_kernel(const float* __restrict__ xs, int DP, const float* __restrict__ v,
                                int64_t v_ld, int tcols, int T, int64_t n, int64_t npad,
                                float* __restrict__ xv) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= npad) return;
  const int W = 2 * (DP + T);
  float2* row = reinterpret_cast<float2*>(xv + j * W);
  if (j < n) {
    for (int k = 0; k < DP; ++k) {
      const float x = -xs[j * DP + k];
      row[k] = make_float2(x, x);
    }
    for (int c = 0; c < T; ++c) {
      const float a = (c < tcols) ? v[c * v_ld + j] : 0.f;
      row[DP + c] = make_float2(a, a);
    }
  } else {
    for (int k = 0; k < DP + T; ++k) row[k] = make_float2(0.f, 0.f);
  }
}

bool kv_tc_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("GPB_KV_TC");
    v = (e && e[0] == '0') ? 1 : 0;  // default on; GPB_KV_TC=0 selects the FFMA2 kernel
  }
  return v == 1;
}

// Tensor-core tile layout (kv_tiles_tc.cuh): per 128-row tile
// [-x' 128 x DP][V hi: 16 k-steps x 128][V lo: 16 k-steps x 128].
__global__ void pack_tc_kernel(const float* __restrict__ xs, int DP, float* __restrict__ v,
                               int64_t v_ld, int c0, int tcols, int64_t n, int64_t npad,
                               float* __restrict__ dst, const float* __restrict__ upd_z,
                               const float* __restrict__ upd_beta) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= npad) return;
  const int TILE = 128 * DP + 2 * 16 * 128;
  float* base = dst + (j / 128) * TILE;
  const int jt = (int)(j % 128);
  const int ks = jt / 8, k = jt % 8;
  float* bh = base + 128 * DP + ks * 128;
  float* bl = bh + 16 * 128;
  for (int q = 0; q < DP; ++q) base[jt * DP + q] = (j < n) ? -xs[j * DP + q] : 0.f;  // negated x'
  for (int c = 0; c < 16; ++c) {
    float val = 0.f;
    if (j < n && c < tcols) {
      const int64_t off = (int64_t)(c0 + c) * v_ld + j;
      val = v[off];
      if (upd_beta) {
        const float b = upd_beta[c0 + c];
        const float zz = upd_z[off];
        val = (b == 0.f || b != b || val != val) ? zz : fmaf(b, val, zz);
        v[off] = val;
      }
    }
    const float hi = tf32_hi(val);
    bh[tc_b_offset(c, k)] = hi;
    bl[tc_b_offset(c, k)] = val - hi;
  }
}

int launch_pack_tc(const float* xs, int DP, float* v, int64_t v_ld, int c0, int tcols, int64_t n,
                   int64_t npad, float* xv, const float* upd_z, const float* upd_beta,
                   cudaStream_t stream) {
  if (npad == 0) return GPB_OK;
  pack_tc_kernel<<<(unsigned)ceil_div(npad, 256), 256, 0, stream>>>(xs, DP, v, v_ld, c0, tcols, n,
                                                                   npad, xv, upd_z, upd_beta);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// Gram tile packing: per 128 columns [B hi | B lo | V hi | V lo] with
// B = [-2y | 1 1 1 | |y|^2 in three exact tf32 parts | 0 0]
// (kv_tiles_gram.cuh), with the same optional p = z + beta p update.
__global__ void pack_gram_kernel(const float* __restrict__ xs, int DP, float* __restrict__ v,
                                 int64_t v_ld, int c0, int tcols, int64_t n, int64_t npad,
                                 float* __restrict__ dst, const float* __restrict__ upd_z,
                                 const float* __restrict__ upd_beta) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= npad) return;
  float* base = dst + (j / 128) * gram_tile_floats(DP);
  const int jt = (int)(j % 128);
  const int KA = gram_kaug(DP);
  float y[32];
  for (int q = 0; q < DP; ++q) y[q] = (j < n) ? xs[j * DP + q] : 0.f;
  for (int q = 0; q < DP; ++q) {
    const float b = -2.f * y[q];
    const float hi = tf32_hi(b);
    base[gram_xoff(jt, q)] = hi;
    base[128 * KA + gram_xoff(jt, q)] = b - hi;
  }
  float e[8] = {1.f, 1.f, 1.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  gram_split3(gram_sqnorm(y, DP), e[3], e[4], e[5]);
  for (int q = 0; q < 8; ++q) base[gram_xoff(jt, DP + q)] = e[q];
  // V block per 8-column k-step: N = 32 rows (n < 16: V hi, n >= 16: V lo),
  // core matrices 8 n x 4 k, K-adjacent at 512 B, N-adjacent at 128 B.
  float* vb = base + gram_v_offset(DP) + (jt / 8) * 256;
  const int k = jt % 8;
  auto voff = [k](int nn) { return (k / 4) * 128 + (nn / 8) * 32 + (nn % 8) * 4 + (k % 4); };
  for (int c = 0; c < 16; ++c) {
    float val = 0.f;
    if (j < n && c < tcols) {
      const int64_t off = (int64_t)(c0 + c) * v_ld + j;
      val = v[off];
      if (upd_beta) {
        const float b = upd_beta[c0 + c];
        const float zz = upd_z[off];
        val = (b == 0.f || b != b || val != val) ? zz : fmaf(b, val, zz);
        v[off] = val;
      }
    }
    const float hi = tf32_hi(val);
    vb[voff(c)] = hi;
    vb[voff(16 + c)] = val - hi;
  }
}

// Narrow Gram tile packing: per 128 columns [B hi | B lo | V : 128 x NV fp32]
// (kv_tile_gram1_kernel), B as above, with the same optional p = z + beta p update.
__global__ void pack_gram1_kernel(const float* __restrict__ xs, int DP, int NV,
                                  float* __restrict__ v, int64_t v_ld, int c0, int tcols, int64_t n,
                                  int64_t npad, float* __restrict__ dst,
                                  const float* __restrict__ upd_z,
                                  const float* __restrict__ upd_beta) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= npad) return;
  float* base = dst + (j / 128) * gram1_tile_floats(DP, NV);
  const int jt = (int)(j % 128);
  const int KA = gram_kaug(DP);
  float y[32];
  for (int q = 0; q < DP; ++q) y[q] = (j < n) ? xs[j * DP + q] : 0.f;
  for (int q = 0; q < DP; ++q) {
    const float b = -2.f * y[q];
    const float hi = tf32_hi(b);
    base[gram_xoff(jt, q)] = hi;
    base[128 * KA + gram_xoff(jt, q)] = b - hi;
  }
  float e[8] = {1.f, 1.f, 1.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  gram_split3(gram_sqnorm(y, DP), e[3], e[4], e[5]);
  for (int q = 0; q < 8; ++q) base[gram_xoff(jt, DP + q)] = e[q];
  float* vb = base + 128 * (2 * DP + 8) + jt * NV;
  for (int c = 0; c < NV; ++c) {
    float val = 0.f;
    if (j < n && c < tcols) {
      const int64_t off = (int64_t)(c0 + c) * v_ld + j;
      val = v[off];
      if (upd_beta) {
        const float b = upd_beta[c0 + c];
        const float zz = upd_z[off];
        val = (b == 0.f || b != b || val != val) ? zz : fmaf(b, val, zz);
        v[off] = val;
      }
    }
    vb[c] = val;
  }
}

int launch_pack_gram1(const float* xs, int DP, int NV, float* v, int64_t v_ld, int c0, int tcols,
                      int64_t n, int64_t npad, float* xv, const float* upd_z,
                      const float* upd_beta, cudaStream_t stream) {
  if (npad == 0) return GPB_OK;
  GPB_REQUIRE((DP == 8 || DP == 16) && (NV == 1 || NV == 2 || NV == 4 || NV == 8), GPB_ERR_INVALID,
              "narrow Gram packing needs DP in {8,16}, NV in {1,2,4,8}");
  pack_gram1_kernel<<<(unsigned)ceil_div(npad, 128), 128, 0, stream>>>(
      xs, DP, NV, v, v_ld, c0, tcols, n, npad, xv, upd_z, upd_beta);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int launch_pack_gram(const float* xs, int DP, float* v, int64_t v_ld, int c0, int tcols, int64_t n,
                     int64_t npad, float* xv, const float* upd_z, const float* upd_beta,
                     cudaStream_t stream) {
  if (npad == 0) return GPB_OK;
  GPB_REQUIRE(DP % 8 == 0 && DP <= 32, GPB_ERR_INVALID, "Gram packing needs DP in {8,16,24,32}");
  pack_gram_kernel<<<(unsigned)ceil_div(npad, 128), 128, 0, stream>>>(xs, DP, v, v_ld, c0, tcols, n,
                                                                     npad, xv, upd_z, upd_beta);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

// ---------------------------------------------------------- fp16 Gram tiles
// Column value of the packed right-hand side, with the optional in-place
// p = z + beta p update of the CG direction (not written back here).
__device__ __forceinline__ float gramh_col_value(const float* v, int64_t v_ld, int c0, int c,
                                                 int64_t j, const float* upd_z,
                                                 const float* upd_beta) {
  const int64_t off = (int64_t)(c0 + c) * v_ld + j;
  float val = v[off];
  if (upd_beta) {
    const float b = upd_beta[c0 + c];
    const float zz = upd_z[off];
    val = (b == 0.f || b != b || val != val) ? zz : fmaf(b, val, zz);
  }
  return val;
}

// maxbits[c] = max over rows j < n of |column c| (float bit patterns; the
// caller zeroes them). NaN maps above every finite value.
__global__ void gramh_colmax_kernel(const float* __restrict__ v, int64_t v_ld, int c0, int tcols,
                                    int64_t n, const float* __restrict__ upd_z,
                                    const float* __restrict__ upd_beta,
                                    unsigned* __restrict__ maxbits) {
  float m[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) m[c] = 0.f;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x) {
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      if (c >= tcols) break;
      const float a = fabsf(gramh_col_value(v, v_ld, c0, c, j, upd_z, upd_beta));
      m[c] = (a != a) ? a : fmaxf(m[c], a);
    }
  }
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    if (c >= tcols) break;
    unsigned b = __float_as_uint(m[c]);
    if (m[c] != m[c]) b = 0x7FC00000u;
    for (int o = 16; o > 0; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
    if ((threadIdx.x & 31) == 0 && b) atomicMax(&maxbits[c], b);
  }
}

// One packed fp16 Gram tile row per column j (see kv_tiles_gramh.cuh).
__global__ void pack_gramh_kernel(const float* __restrict__ xs, int DP, float* __restrict__ v,
                                  int64_t v_ld, int c0, int tcols, int64_t n, int64_t npad,
                                  float* __restrict__ dst, const float* __restrict__ upd_z,
                                  const float* __restrict__ upd_beta,
                                  const unsigned* __restrict__ maxbits) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= npad) return;
  const int TILE = DP == 16 ? gramh_tile_floats(16) : gramh_tile_floats(8);
  float* base = dst + (j / 128) * TILE;
  const int jt = (int)(j % 128);
  __half* hb = reinterpret_cast<__half*>(base);
  float y[16];
  for (int q = 0; q < DP; ++q) y[q] = (j < n) ? kGHInScale * xs[j * DP + q] : 0.f;
  // Norm row of the column side: 2^-8 against the row's |x''|^2 parts, |y'|^2
  // = |y''|^2 / 256 in three parts against the row's ones, -12 against its
  // last one (MMA1 then yields u - 12).
  float m3[3];
  gramh_split3(gram_sqnorm(y, DP) * (1.f / 256.f), m3[0], m3[1], m3[2]);
  const float c8 = 1.f / 256.f;
  const float ny[8] = {c8, c8, c8, m3[0], m3[1], m3[2], -kGHUShift, 0.f};
  auto put = [&](int blk, int k, float val) {
    hb[blk * 2048 + gramh_boff(jt, k, 2048) / 2] = __float2half_rn(val);
  };
  for (int q = 0; q < DP; ++q) {
    const float b = y[q] * (-2.f / 256.f);  // -2 y'' / 256 = -2 y' / 16
    const float bh = __half2float(__float2half_rn(b));
    const float bl = b - bh;
    if (DP == 16) {
      put(0, q, bh);
      put(1, q, bl);
    } else {
      put(0, q, bh);
      put(0, 8 + q, bh);
      put(1, q, bl);
    }
  }
  if (DP == 16) {
    for (int k = 0; k < 16; ++k) put(2, k, k < 8 ? ny[k] : 0.f);
  } else {
    for (int k = 0; k < 8; ++k) put(1, 8 + k, ny[k]);
  }
  // V block of chunk jt / 16: rows [V hi (16) | V lo (16)], k = jt % 16.
  __half* vb = hb + 2 * gramh_v_offset(DP) + (jt / 16) * 512;
  const int k = jt % 16;
  for (int c = 0; c < 16; ++c) {
    float val = 0.f;
    if (j < n && c < tcols) {
      val = gramh_col_value(v, v_ld, c0, c, j, upd_z, upd_beta);
      if (upd_beta) v[(int64_t)(c0 + c) * v_ld + j] = val;
    }
    const float sv = val * gramh_col_scale(__uint_as_float(maxbits[c]));
    const __half h = __float2half_rn(sv);
    vb[gramh_boff(c, k, 512) / 2] = h;
    vb[gramh_boff(16 + c, k, 512) / 2] = __float2half_rn(sv - __half2float(h));
  }
  base[gramh_max_offset(DP) + jt] = jt < 16 ? __uint_as_float(maxbits[jt]) : 0.f;
}

int launch_gramh_colmax(float* v, int64_t v_ld, int c0, int tcols, int64_t n, float* dst,
                        const float* upd_z, const float* upd_beta, int DP, cudaStream_t stream) {
  unsigned* maxbits = reinterpret_cast<unsigned*>(dst + gramh_max_offset(DP));
  GPB_CHECK_CUDA(cudaMemsetAsync(maxbits, 0, 16 * sizeof(unsigned), stream));
  if (n <= 0) return GPB_OK;
  const unsigned blocks = (unsigned)std::min<int64_t>(ceil_div(n, 256), 4 * 148);
  gramh_colmax_kernel<<<blocks, 256, 0, stream>>>(v, v_ld, c0, tcols, n, upd_z, upd_beta, maxbits);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int launch_pack_gramh(const float* xs, int DP, float* v, int64_t v_ld, int c0, int tcols,
                      int64_t n, int64_t npad, float* xv, const float* upd_z,
                      const float* upd_beta, cudaStream_t stream, bool colmax) {
  if (npad == 0) return GPB_OK;
  GPB_REQUIRE(DP == 8 || DP == 16, GPB_ERR_INVALID, "fp16 Gram packing needs DP in {8,16}");
  if (colmax)
    GPB_TRY(launch_gramh_colmax(v, v_ld, c0, tcols, n, xv, upd_z, upd_beta, DP, stream));
  // Every block reads the maxima from tile 0's tail; block 0 rewrites the same
  // values there.
  const unsigned* maxbits = reinterpret_cast<const unsigned*>(xv + gramh_max_offset(DP));
  pack_gramh_kernel<<<(unsigned)ceil_div(npad, 128), 128, 0, stream>>>(
      xs, DP, v, v_ld, c0, tcols, n, npad, xv, upd_z, upd_beta, maxbits);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int kv_gramh_mode() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("GPB_KV_GRAMH");
    v = (e && (e[0] == '0' || e[0] == '2')) ? e[0] - '0' : 1;
  }
  return v;
}

bool kv_gram1_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("GPB_KV_GRAM1");
    v = (e && e[0] == '0') ? 1 : 0;
  }
  return v == 1;
}

bool kv_gram_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("GPB_KV_GRAM");
    v = (e && e[0] == '0') ? 1 : 0;
  }
  return v == 1;
}

bool kv_x2_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("GPB_KV_SCALAR");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

int launch_pack(const float* xs, int DP, const float* v, int64_t v_ld, int tcols, int T, int64_t n,
                int64_t npad, float* xv, cudaStream_t stream, int layout) {
  const int W = packed_width(DP, T);
  if (npad == 0) return GPB_OK;
  if (layout == KV_TC)
    return launch_pack_tc(xs, DP, const_cast<float*>(v), v_ld, 0, tcols, n, npad, xv, nullptr,
                          nullptr, stream);
  if (layout == KV_GRAM)
    return launch_pack_gram(xs, DP, const_cast<float*>(v), v_ld, 0, tcols, n, npad, xv, nullptr,
                            nullptr, stream);
  if (layout == KV_GRAM1)
    return launch_pack_gram1(xs, DP, T, const_cast<float*>(v), v_ld, 0, tcols, n, npad, xv,
                             nullptr, nullptr, stream);
  if (layout == KV_GRAMH)
    return launch_pack_gramh(xs, DP, const_cast<float*>(v), v_ld, 0, tcols, n, npad, xv, nullptr,
                             nullptr, stream, true);
  if (layout == KV_X2) {
    pack_dup_kernel<<<(unsigned)ceil_div(npad, 256), 256, 0, stream>>>(xs, DP, v, v_ld, tcols, T,
                                                                      n, npad, xv);
    GPB_CHECK_CUDA(cudaGetLastError());
    return GPB_OK;
  }
  pack_kernel<<<(unsigned)ceil_div(npad, 256), 256, 0, stream>>>(xs, DP, v, v_ld, tcols, n, npad,
                                                                W, xv);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

}  // namespace gpb
