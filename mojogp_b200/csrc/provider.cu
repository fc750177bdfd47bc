// Provider lifecycle and the matvec entry points of the C ABI.
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <new>

#include "provider.cuh"
#include "kv_tiles_gram.cuh"

namespace gpb {

// ------------------------------------------------------------------ errors
static thread_local char g_err[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
void clear_error() { g_err[0] = 0; }

// --------------------------------------------------------------- workspace
int Workspace::get(int slot, size_t bytes, void** out) {
  if ((int)ptr.size() <= slot) {
    ptr.resize(slot + 1, nullptr);
    cap.resize(slot + 1, 0);
  }
  if (cap[slot] < bytes) {
    if (ptr[slot]) cudaFree(ptr[slot]);
    ptr[slot] = nullptr;
    cap[slot] = 0;
    const size_t want = bytes + bytes / 8 + 256;
    cudaError_t e = cudaMalloc(&ptr[slot], want);
    if (e != cudaSuccess) {
      set_error("workspace allocation of %zu bytes failed: %s", want, cudaGetErrorString(e));
      ptr[slot] = nullptr;
      return GPB_ERR_NOMEM;
    }
    cap[slot] = want;
  }
  *out = ptr[slot];
  return GPB_OK;
}

void Workspace::release() {
  for (void* q : ptr)
    if (q) cudaFree(q);
  ptr.clear();
  cap.clear();
}

// ------------------------------------------------------------------ spec
int parse_spec(const int32_t* spec, int32_t len, int32_t d, DevKernel* k) {
  GPB_REQUIRE(spec != nullptr && len >= 3, GPB_ERR_INVALID, "kernel spec is empty");
  GPB_REQUIRE(spec[0] == GPB_SPEC_VERSION, GPB_ERR_INVALID, "kernel spec version %d != %d", spec[0],
              GPB_SPEC_VERSION);
  std::memset(k, 0, sizeof(*k));
  k->nparams = spec[1];
  k->nnodes = spec[2];
  k->d = d;
  GPB_REQUIRE(k->nparams > 0 && k->nparams <= GPB_MAX_PARAMS, GPB_ERR_INVALID,
              "kernel has %d parameters (max %d)", k->nparams, GPB_MAX_PARAMS);
  GPB_REQUIRE(k->nnodes > 0 && k->nnodes <= GPB_MAX_NODES, GPB_ERR_INVALID,
              "kernel has %d nodes (max %d)", k->nnodes, GPB_MAX_NODES);
  int pos = 3, depth = 0;
  std::vector<int> used(k->nparams, 0);
  for (int nidx = 0; nidx < k->nnodes; ++nidx) {
    GPB_REQUIRE(pos < len, GPB_ERR_INVALID, "kernel spec truncated at node %d", nidx);
    const int op = spec[pos++];
    k->node_op[nidx] = op;
    if (op == GPB_NODE_LEAF) {
      GPB_REQUIRE(pos + 4 <= len, GPB_ERR_INVALID, "truncated leaf");
      GPB_REQUIRE(k->nleaves < GPB_MAX_LEAVES, GPB_ERR_INVALID, "more than %d leaves",
                  GPB_MAX_LEAVES);
      LeafDesc& L = k->leaf[k->nleaves];
      L.type = spec[pos++];
      L.ard = spec[pos++] != 0;
      L.pofs = spec[pos++];
      L.ndims = spec[pos++];
      GPB_REQUIRE(L.type >= GPB_KERNEL_RBF && L.type <= GPB_KERNEL_POLYNOMIAL, GPB_ERR_INVALID,
                  "unknown kernel type %d", L.type);
      GPB_REQUIRE(L.ndims >= 1 && L.ndims <= GPB_MAX_DIM && pos + L.ndims <= len, GPB_ERR_INVALID,
                  "leaf has %d active dims", L.ndims);
      for (int q = 0; q < L.ndims; ++q) {
        L.dims[q] = spec[pos++];
        GPB_REQUIRE(L.dims[q] >= 0 && L.dims[q] < d, GPB_ERR_INVALID,
                    "active dim %d out of range for d=%d", L.dims[q], d);
      }
      const int np = leaf_num_params(L.type, L.ard, L.ndims);
      GPB_REQUIRE(L.pofs >= 0 && L.pofs + np <= k->nparams, GPB_ERR_INVALID,
                  "leaf parameters [%d, %d) exceed P=%d", L.pofs, L.pofs + np, k->nparams);
      for (int q = 0; q < np; ++q) used[L.pofs + q]++;
      k->node_arg[nidx] = k->nleaves++;
      ++depth;
    } else if (op == GPB_NODE_SCALE) {
      GPB_REQUIRE(pos < len, GPB_ERR_INVALID, "truncated scale node");
      const int pi = spec[pos++];
      GPB_REQUIRE(pi >= 0 && pi < k->nparams, GPB_ERR_INVALID, "scale parameter %d out of range",
                  pi);
      GPB_REQUIRE(depth >= 1, GPB_ERR_INVALID, "scale node without operand");
      used[pi]++;
      k->node_arg[nidx] = pi;
    } else if (op == GPB_NODE_SUM || op == GPB_NODE_PRODUCT) {
      GPB_REQUIRE(depth >= 2, GPB_ERR_INVALID, "binary node without two operands");
      k->node_arg[nidx] = 0;
      --depth;
    } else {
      set_error("unknown node op %d", op);
      return GPB_ERR_INVALID;
    }
  }
  GPB_REQUIRE(depth == 1, GPB_ERR_INVALID, "kernel program leaves %d values on the stack", depth);
  GPB_REQUIRE(pos == len, GPB_ERR_INVALID, "kernel spec has %d trailing words", len - pos);
  for (int q = 0; q < k->nparams; ++q)
    GPB_REQUIRE(used[q] == 1, GPB_ERR_INVALID, "parameter %d used %d times", q, used[q]);
  return GPB_OK;
}

// ------------------------------------------------------------------ plan
int provider_plan(gpb_provider* p) {
  const DevKernel& K = p->dk;
  for (int l = 0; l < K.nleaves; ++l) {
    const LeafDesc& L = K.leaf[l];
    if (L.type == GPB_KERNEL_POLYNOMIAL) {
      const float deg = K.params[L.pofs + (L.ard ? L.ndims : 0)];
      GPB_REQUIRE(deg >= 1.f && std::fabs(deg - std::nearbyint(deg)) <= 1e-5f, GPB_ERR_INVALID,
                  "Polynomial kernel degree must be a fixed positive integer, got %g", (double)deg);
    }
  }
  // Fast path: one stationary leaf, optionally under a scale node.
  int leaf_node = -1, scale_param = -1;
  if (K.nnodes == 1 && K.node_op[0] == GPB_NODE_LEAF) leaf_node = 0;
  if (K.nnodes == 2 && K.node_op[0] == GPB_NODE_LEAF && K.node_op[1] == GPB_NODE_SCALE) {
    leaf_node = 0;
    scale_param = K.node_arg[1];
  }
  bool fast = false;
  if (leaf_node >= 0) {
    const LeafDesc& L = K.leaf[K.node_arg[leaf_node]];
    fast = is_stationary(L.type) && kv_pick_dp(L.type, L.ndims) > 0;
  }
  PrescaleSpec& ps = p->ps;
  std::memset(&ps, 0, sizeof(ps));
  if (fast) {
    const LeafDesc& L = K.leaf[K.node_arg[leaf_node]];
    const float* prm = K.params + L.pofs;
    const int nl = L.ard ? L.ndims : 1;
    float c2 = 1.f;
    switch (L.type) {
      case GPB_KERNEL_RBF: c2 = 0.5f * kLog2e; break;
      case GPB_KERNEL_MATERN32: c2 = 3.f; break;
      case GPB_KERNEL_MATERN52: c2 = 5.f; break;
      default: c2 = 1.f;
    }
    const float c = std::sqrt(c2);
    p->eval = L.type;
    p->DP = kv_pick_dp(L.type, L.ndims);
    // 3-8 input dims on a leaf the Gram tensor-core kernels take: pad to 8
    // (zero dims change no distance) so that those kernels can run.
    if (gram_leaf(L.type) && L.ndims >= 3 && L.ndims <= 8) p->DP = 8;
    ps.DP = p->DP;
    ps.nd = L.ndims;
    for (int q = 0; q < L.ndims; ++q) {
      const float ell = L.ard ? prm[q] : prm[0];
      GPB_REQUIRE(ell > 0.f && std::isfinite(ell), GPB_ERR_INVALID, "lengthscale %g must be > 0",
                  (double)ell);
      ps.dims[q] = L.dims[q];
      ps.scale[q] = c / ell;
    }
    float os = (L.type == GPB_KERNEL_RQ) ? prm[nl + 1] : prm[nl];
    if (scale_param >= 0) os *= K.params[scale_param];
    p->os_eff = os;
    p->fp = FastParams{0.f, 0.f};
    if (L.type == GPB_KERNEL_MATERN12) {
      p->fp.a0 = L.ard ? 1.f : 0.f;
      p->fp.a1 = 1e-20f * c2;
    } else if (L.type == GPB_KERNEL_MATERN32 || L.type == GPB_KERNEL_MATERN52) {
      p->fp.a1 = 1e-20f * c2;
    } else if (L.type == GPB_KERNEL_RQ) {
      const float alpha = prm[nl];
      GPB_REQUIRE(alpha > 0.f, GPB_ERR_INVALID, "RQ alpha must be > 0");
      p->fp.a0 = alpha;
      p->fp.a1 = 1.f / (2.f * alpha);
    }
  } else {
    p->eval = kEvalGeneric;
    p->DP = kv_pick_dp(kEvalGeneric, p->d);
    GPB_REQUIRE(p->DP > 0, GPB_ERR_UNSUPPORTED, "input dimension %d exceeds %d", p->d,
                GPB_MAX_DIM);
    ps.DP = p->DP;
    ps.nd = p->d;
    for (int q = 0; q < p->d; ++q) {
      ps.dims[q] = q;
      ps.scale[q] = 1.f;
    }
    p->os_eff = 1.f;
  }
  p->xs_dirty = true;
  return GPB_OK;
}

__global__ void max_sqnorm_kernel(const float* __restrict__ xs, int64_t n, int DP,
                                  unsigned* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float s = 0.f;
  if (i < n) s = gram_sqnorm(xs + i * DP, DP);
  for (int o = 16; o > 0; o >>= 1) s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, o));
  // Non-negative floats order like their bit patterns; NaN maps above every finite value.
  if ((threadIdx.x & 31) == 0) atomicMax(out, s != s ? 0xFFFFFFFFu : __float_as_uint(s));
}

int launch_max_sqnorm(const float* xs, int64_t n, int DP, unsigned* word, cudaStream_t st) {
  if (n <= 0) return GPB_OK;
  max_sqnorm_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(xs, n, DP, word);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int provider_refresh_xs(gpb_provider* p) {
  if (!p->xs_dirty) return GPB_OK;
  if (p->Xs_d) cudaFree(p->Xs_d);
  p->Xs_d = nullptr;
  GPB_CHECK_CUDA(cudaMalloc(&p->Xs_d, (size_t)std::max<int64_t>(p->n, 1) * p->DP * sizeof(float)));
  GPB_TRY(launch_prescale(p->X_d, p->n, p->d, p->ps, p->Xs_d, p->stream));
  p->gram_ok = false;
  if (p->eval != kEvalGeneric && gram_leaf(p->eval) && (p->DP == 8 || p->DP == 16) && p->n > 0) {
    if (!p->sqnorm_d) GPB_CHECK_CUDA(cudaMalloc(&p->sqnorm_d, sizeof(unsigned)));
    GPB_CHECK_CUDA(cudaMemsetAsync(p->sqnorm_d, 0, sizeof(unsigned), p->stream));
    max_sqnorm_kernel<<<(unsigned)ceil_div(p->n, 256), 256, 0, p->stream>>>(p->Xs_d, p->n, p->DP,
                                                                            p->sqnorm_d);
    GPB_CHECK_CUDA(cudaGetLastError());
    unsigned h = 0;
    GPB_CHECK_CUDA(cudaMemcpyAsync(&h, p->sqnorm_d, sizeof(unsigned), cudaMemcpyDeviceToHost,
                                   p->stream));
    GPB_CHECK_CUDA(cudaStreamSynchronize(p->stream));
    float hf = 0.f;
    std::memcpy(&hf, &h, sizeof(hf));
    p->gram_ok = h != 0xFFFFFFFFu && hf <= kGramMaxSqNorm;
    p->launches += 1;
  }
  p->xs_dirty = false;
  return GPB_OK;
}

// *ok = max_i |xs_i|^2 over nrow prescaled rows is within the Gram bound.
static int rows_sqnorm_bounded(gpb_provider* p, const float* xs, int64_t nrow, cudaStream_t stream,
                               bool* ok) {
  *ok = false;
  if (!p->sqnorm_d) GPB_CHECK_CUDA(cudaMalloc(&p->sqnorm_d, sizeof(unsigned)));
  GPB_CHECK_CUDA(cudaMemsetAsync(p->sqnorm_d, 0, sizeof(unsigned), stream));
  max_sqnorm_kernel<<<(unsigned)ceil_div(nrow, 256), 256, 0, stream>>>(xs, nrow, p->DP,
                                                                      p->sqnorm_d);
  GPB_CHECK_CUDA(cudaGetLastError());
  unsigned h = 0;
  GPB_CHECK_CUDA(cudaMemcpyAsync(&h, p->sqnorm_d, sizeof(unsigned), cudaMemcpyDeviceToHost, stream));
  GPB_CHECK_CUDA(cudaStreamSynchronize(stream));
  float hf = 0.f;
  std::memcpy(&hf, &h, sizeof(hf));
  *ok = h != 0xFFFFFFFFu && hf <= kGramMaxSqNorm;
  p->launches += 1;
  return GPB_OK;
}

int provider_prescale_rows(gpb_provider* p, const float* x_raw, int64_t nrow, int slot,
                           const float** out, cudaStream_t stream) {
  void* buf = nullptr;
  GPB_TRY(p->ws.get(slot, (size_t)std::max<int64_t>(nrow, 1) * p->DP * sizeof(float), &buf));
  GPB_TRY(launch_prescale(x_raw, nrow, p->d, p->ps, (float*)buf, stream));
  *out = (const float*)buf;
  return GPB_OK;
}

int provider_check_device_error(gpb_provider* p) {
  int h = 0;
  GPB_CHECK_CUDA(cudaMemcpyAsync(&h, p->err_d, sizeof(int), cudaMemcpyDeviceToHost, p->stream));
  GPB_CHECK_CUDA(cudaStreamSynchronize(p->stream));
  if (h != 0) {
    cudaMemsetAsync(p->err_d, 0, sizeof(int), p->stream);
    set_error("device error word %d (bounded wait gave up in a tiled kernel)", h);
    return GPB_ERR_DEVICE;
  }
  return GPB_OK;
}

int provider_kv(gpb_provider* p, const float* xrow, int64_t nrow, const float* v, int64_t v_ld,
                int64_t ncols, float* out, int64_t out_ld, bool add_noise, int64_t noise_row0,
                cudaStream_t stream) {
  if (nrow == 0 || ncols == 0) return GPB_OK;
  GPB_TRY(provider_refresh_xs(p));
  // The Gram path needs bounded prescaled norms on both sides: the training
  // rows were checked when Xs was built; other rows (test points) are checked here.
  bool gram = p->gram_ok;
  if (gram && !(xrow >= p->Xs_d && xrow < p->Xs_d + std::max<int64_t>(p->n, 1) * p->DP))
    GPB_TRY(rows_sqnorm_bounded(p, xrow, nrow, stream, &gram));
  const int64_t npad = round_up(std::max<int64_t>(p->n, 1), kJT);
  const int ntiles = (int)(npad / kJT);
  for (int64_t c0 = 0; c0 < ncols; c0 += 16) {
    const int64_t rem = ncols - c0;
    const int T = kv_chunk_t(p->eval, p->DP, rem, gram);
    const int tcols = (int)std::min<int64_t>(rem, T);
    const int W = kv_packed_width(p->eval, p->DP, T, gram);
    void* xv = nullptr;
    GPB_TRY(p->ws.get(WS_XV, (size_t)npad * W * sizeof(float), &xv));
    GPB_TRY(launch_pack(p->Xs_d, p->DP, v + c0 * v_ld, v_ld, tcols, T, p->n, npad, (float*)xv,
                        stream, kv_layout(p->eval, p->DP, T, gram)));
    p->launches += 1;
    const int64_t part_floats = std::min<int64_t>((int64_t)32 * T * nrow, (int64_t)1 << 29);
    void* part = nullptr;
    GPB_TRY(p->ws.get(WS_PARTIAL, (size_t)part_floats * sizeof(float), &part));
    KvLaunch L{};
    L.eval = p->eval;
    L.DP = p->DP;
    L.T = T;
    L.xrow = xrow;
    L.nrow = nrow;
    L.xv = (const float*)xv;
    L.ntiles = ntiles;
    L.fp = p->fp;
    L.dk = &p->dk;
    L.ep.out = out + c0 * out_ld;
    L.ep.out_ld = out_ld;
    L.ep.scale = p->os_eff;
    if (add_noise) {
      L.ep.noise_v = v + c0 * v_ld + noise_row0;
      L.ep.noise_ld = v_ld;
      L.ep.noise = p->noise;
      L.ep.noise_vec = p->noise_vec_d ? p->noise_vec_d + noise_row0 : nullptr;
    }
    L.tcols = tcols;
    L.partial = (float*)part;
    L.partial_capacity = part_floats;
    L.err = p->err_d;
    L.stream = stream;
    L.launches = &p->launches;
    L.gram_ok = gram;
    if (c0 == 0) L.ev_begin = p->tile_ev[0];
    if (c0 + 16 >= ncols) L.ev_end = p->tile_ev[1];
    GPB_TRY(launch_kv(L));
  }
  return GPB_OK;
}

// ---------------------------------------------------------- small kernels
__global__ void diag_kernel(const float* __restrict__ X, int64_t n, int d,
                            const __grid_constant__ DevKernel K, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float xi[GPB_MAX_DIM];
  for (int k = 0; k < d; ++k) xi[k] = X[i * d + k];
  out[i] = tree_eval<false>(K, xi, xi, nullptr);
}

__global__ void column_kernel(const float* __restrict__ X, int64_t n, int d, int64_t piv,
                              const __grid_constant__ DevKernel K, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float xi[GPB_MAX_DIM], xp[GPB_MAX_DIM];
  for (int k = 0; k < d; ++k) {
    xi[k] = X[i * d + k];
    xp[k] = X[piv * d + k];
  }
  out[i] = tree_eval<false>(K, xi, xp, nullptr);
}

}  // namespace gpb

using namespace gpb;

// ================================================================== C ABI
extern "C" {

const char* gpb_version(void) { return "gpb200 0.1.0 (sm_100a)"; }

int gpb_last_error(char* buf, int64_t buf_len) {
  if (!buf || buf_len <= 0) return GPB_ERR_INVALID;
  std::strncpy(buf, g_err, (size_t)buf_len - 1);
  buf[buf_len - 1] = 0;
  return GPB_OK;
}

int gpb_device_count(int32_t* count_out) {
  GPB_REQUIRE(count_out, GPB_ERR_INVALID, "null count_out");
  int c = 0;
  cudaError_t e = cudaGetDeviceCount(&c);
  if (e != cudaSuccess) {
    cudaGetLastError();
    c = 0;
  }
  *count_out = c;
  return GPB_OK;
}

int gpb_device_mem_info(int32_t device, int64_t* free_out, int64_t* total_out) {
  GPB_REQUIRE(free_out && total_out, GPB_ERR_INVALID, "null output");
  GPB_CHECK_CUDA(cudaSetDevice(device));
  size_t f = 0, t = 0;
  GPB_CHECK_CUDA(cudaMemGetInfo(&f, &t));
  *free_out = (int64_t)f;
  *total_out = (int64_t)t;
  return GPB_OK;
}

int gpb_device_alloc(int32_t device, int64_t bytes, void** ptr_out) {
  GPB_REQUIRE(ptr_out && bytes >= 0, GPB_ERR_INVALID, "bad alloc arguments");
  GPB_CHECK_CUDA(cudaSetDevice(device));
  *ptr_out = nullptr;
  cudaError_t e = cudaMalloc(ptr_out, (size_t)std::max<int64_t>(bytes, 1));
  if (e != cudaSuccess) {
    set_error("cudaMalloc(%lld) failed: %s", (long long)bytes, cudaGetErrorString(e));
    return GPB_ERR_NOMEM;
  }
  return GPB_OK;
}

int gpb_device_free(int32_t device, void* ptr) {
  GPB_CHECK_CUDA(cudaSetDevice(device));
  if (ptr) GPB_CHECK_CUDA(cudaFree(ptr));
  return GPB_OK;
}

int gpb_memcpy_h2d(int32_t device, void* dst_dev, const void* src_host, int64_t bytes) {
  GPB_REQUIRE(bytes >= 0 && (bytes == 0 || (dst_dev && src_host)), GPB_ERR_INVALID, "bad copy");
  GPB_CHECK_CUDA(cudaSetDevice(device));
  if (bytes) GPB_CHECK_CUDA(cudaMemcpy(dst_dev, src_host, (size_t)bytes, cudaMemcpyHostToDevice));
  return GPB_OK;
}

int gpb_memcpy_d2h(int32_t device, void* dst_host, const void* src_dev, int64_t bytes) {
  GPB_REQUIRE(bytes >= 0 && (bytes == 0 || (dst_host && src_dev)), GPB_ERR_INVALID, "bad copy");
  GPB_CHECK_CUDA(cudaSetDevice(device));
  if (bytes) GPB_CHECK_CUDA(cudaMemcpy(dst_host, src_dev, (size_t)bytes, cudaMemcpyDeviceToHost));
  return GPB_OK;
}

int gpb_host_register(void* host_ptr, int64_t bytes) {
  GPB_REQUIRE(host_ptr && bytes > 0, GPB_ERR_INVALID, "bad host buffer");
  GPB_CHECK_CUDA(cudaHostRegister(host_ptr, (size_t)bytes, cudaHostRegisterPortable));
  return GPB_OK;
}

int gpb_host_unregister(void* host_ptr) {
  GPB_REQUIRE(host_ptr, GPB_ERR_INVALID, "null host buffer");
  GPB_CHECK_CUDA(cudaHostUnregister(host_ptr));
  return GPB_OK;
}

int gpb_memset_d(int32_t device, void* dst_dev, int32_t value, int64_t bytes) {
  GPB_REQUIRE(bytes >= 0 && (bytes == 0 || dst_dev), GPB_ERR_INVALID, "bad memset");
  GPB_CHECK_CUDA(cudaSetDevice(device));
  if (bytes) GPB_CHECK_CUDA(cudaMemset(dst_dev, value, (size_t)bytes));
  return GPB_OK;
}

int gpb_provider_create(const float* X_host, int64_t n, int32_t d, const int32_t* spec,
                        int32_t spec_len, const float* params_host, int32_t num_params,
                        float noise, const float* noise_vec_host, int32_t device,
                        gpb_provider** out) {
  clear_error();
  GPB_REQUIRE(out, GPB_ERR_INVALID, "null output handle");
  *out = nullptr;
  GPB_REQUIRE(n >= 1 && d >= 1 && d <= GPB_MAX_DIM, GPB_ERR_INVALID,
              "invalid shape n=%lld d=%d (need n>=1, 1<=d<=%d)", (long long)n, d, GPB_MAX_DIM);
  GPB_REQUIRE(X_host && params_host, GPB_ERR_INVALID, "null X or params");
  DevKernel dk;
  GPB_TRY(parse_spec(spec, spec_len, d, &dk));
  GPB_REQUIRE(num_params == dk.nparams, GPB_ERR_INVALID,
              "params has %d entries, kernel expects %d", num_params, dk.nparams);
  for (int q = 0; q < num_params; ++q) dk.params[q] = params_host[q];
  GPB_REQUIRE(std::isfinite(noise) && noise >= 0.f, GPB_ERR_INVALID, "noise must be >= 0");

  gpb_provider* p = new (std::nothrow) gpb_provider();
  GPB_REQUIRE(p, GPB_ERR_NOMEM, "host allocation failed");
  p->device = device;
  p->n = n;
  p->d = d;
  p->dk = dk;
  p->noise = noise;
  auto fail = [&](int code) {
    gpb_provider_destroy(p);
    return code;
  };
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    set_error("cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
    delete p;
    return GPB_ERR_CUDA;
  }
  if ((e = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaMalloc(&p->X_d, (size_t)n * d * sizeof(float))) != cudaSuccess ||
      (e = cudaMalloc(&p->err_d, sizeof(int))) != cudaSuccess) {
    set_error("provider setup: %s", cudaGetErrorString(e));
    return fail(GPB_ERR_CUDA);
  }
  if ((e = cudaMemcpy(p->X_d, X_host, (size_t)n * d * sizeof(float), cudaMemcpyHostToDevice)) !=
          cudaSuccess ||
      (e = cudaMemset(p->err_d, 0, sizeof(int))) != cudaSuccess) {
    set_error("provider upload: %s", cudaGetErrorString(e));
    return fail(GPB_ERR_CUDA);
  }
  if (noise_vec_host) {
    p->noise_mode = GPB_NOISE_FIXED_VECTOR;
    if ((e = cudaMalloc(&p->noise_vec_d, (size_t)n * sizeof(float))) != cudaSuccess ||
        (e = cudaMemcpy(p->noise_vec_d, noise_vec_host, (size_t)n * sizeof(float),
                        cudaMemcpyHostToDevice)) != cudaSuccess) {
      set_error("noise vector upload: %s", cudaGetErrorString(e));
      return fail(GPB_ERR_CUDA);
    }
  }
  int s = provider_plan(p);
  if (s != GPB_OK) return fail(s);
  *out = p;
  return GPB_OK;
}

int gpb_provider_destroy(gpb_provider* p) {
  if (!p) return GPB_OK;
  cudaSetDevice(p->device);
  if (p->stream) cudaStreamSynchronize(p->stream);
  p->ws.release();
  if (p->X_d) cudaFree(p->X_d);
  if (p->Xs_d) cudaFree(p->Xs_d);
  if (p->noise_vec_d) cudaFree(p->noise_vec_d);
  if (p->err_d) cudaFree(p->err_d);
  if (p->sqnorm_d) cudaFree(p->sqnorm_d);
  if (p->stream) cudaStreamDestroy(p->stream);
  delete p;
  return GPB_OK;
}

int gpb_provider_synchronize(gpb_provider* p) {
  GPB_REQUIRE(p, GPB_ERR_INVALID, "null provider");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  GPB_CHECK_CUDA(cudaStreamSynchronize(p->stream));
  return provider_check_device_error(p);
}

int gpb_update_params(gpb_provider* p, const float* params_host, int32_t num_params) {
  GPB_REQUIRE(p && params_host, GPB_ERR_INVALID, "null argument");
  GPB_REQUIRE(num_params == p->dk.nparams, GPB_ERR_INVALID, "params has %d entries, expected %d",
              num_params, p->dk.nparams);
  for (int q = 0; q < num_params; ++q) {
    GPB_REQUIRE(std::isfinite(params_host[q]), GPB_ERR_INVALID, "parameter %d is not finite", q);
    p->dk.params[q] = params_host[q];
  }
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  return provider_plan(p);
}

int gpb_update_noise(gpb_provider* p, float noise) {
  GPB_REQUIRE(p, GPB_ERR_INVALID, "null provider");
  GPB_REQUIRE(std::isfinite(noise) && noise >= 0.f, GPB_ERR_INVALID, "noise must be >= 0");
  p->noise = noise;
  return GPB_OK;
}

int gpb_get_noise(gpb_provider* p, float* noise_out) {
  GPB_REQUIRE(p && noise_out, GPB_ERR_INVALID, "null argument");
  *noise_out = p->noise;
  return GPB_OK;
}

int gpb_get_noise_mode(gpb_provider* p, int32_t* mode_out) {
  GPB_REQUIRE(p && mode_out, GPB_ERR_INVALID, "null argument");
  *mode_out = p->noise_mode;
  return GPB_OK;
}

int gpb_get_num_params(gpb_provider* p, int32_t* num_out) {
  GPB_REQUIRE(p && num_out, GPB_ERR_INVALID, "null argument");
  *num_out = p->dk.nparams;
  return GPB_OK;
}

int gpb_get_params(gpb_provider* p, float* params_host, int32_t num_params) {
  GPB_REQUIRE(p && params_host && num_params == p->dk.nparams, GPB_ERR_INVALID, "bad arguments");
  for (int q = 0; q < num_params; ++q) params_host[q] = p->dk.params[q];
  return GPB_OK;
}

int gpb_get_diagonal_value(gpb_provider* p, float* value_out) {
  GPB_REQUIRE(p && value_out, GPB_ERR_INVALID, "null argument");
  // k(x, x) for the first training row (constant for stationary kernels).
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  void* buf = nullptr;
  GPB_TRY(p->ws.get(WS_MISC, sizeof(float), &buf));
  diag_kernel<<<1, 32, 0, p->stream>>>(p->X_d, 1, p->d, p->dk, (float*)buf);
  GPB_CHECK_CUDA(cudaGetLastError());
  GPB_CHECK_CUDA(cudaMemcpyAsync(value_out, buf, sizeof(float), cudaMemcpyDeviceToHost, p->stream));
  GPB_CHECK_CUDA(cudaStreamSynchronize(p->stream));
  return GPB_OK;
}

int gpb_get_x_ptr(gpb_provider* p, const float** x_dev_out) {
  GPB_REQUIRE(p && x_dev_out, GPB_ERR_INVALID, "null argument");
  *x_dev_out = p->X_d;
  return GPB_OK;
}

int gpb_forward_matvec_rows(gpb_provider* p, float* out_dev, const float* v_dev, int64_t ncols,
                            int64_t row_begin, int64_t row_end) {
  GPB_REQUIRE(p && out_dev && v_dev, GPB_ERR_INVALID, "null argument");
  GPB_REQUIRE(ncols >= 0 && row_begin >= 0 && row_begin <= row_end && row_end <= p->n,
              GPB_ERR_INVALID, "bad row range [%lld, %lld) for n=%lld", (long long)row_begin,
              (long long)row_end, (long long)p->n);
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  GPB_TRY(provider_refresh_xs(p));
  return provider_kv(p, p->Xs_d + row_begin * p->DP, row_end - row_begin, v_dev, p->n, ncols,
                     out_dev, row_end - row_begin, true, row_begin, p->stream);
}

int gpb_matvec_layout(gpb_provider* p, int64_t ncols, int32_t* layout) {
  GPB_REQUIRE(p && layout && ncols > 0, GPB_ERR_INVALID, "bad arguments");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  GPB_TRY(provider_refresh_xs(p));
  const int T = kv_chunk_t(p->eval, p->DP, ncols, p->gram_ok);
  *layout = kv_layout(p->eval, p->DP, T, p->gram_ok);
  return GPB_OK;
}

int gpb_forward_matvec(gpb_provider* p, float* out_dev, const float* v_dev, int64_t ncols) {
  GPB_REQUIRE(p, GPB_ERR_INVALID, "null provider");
  return gpb_forward_matvec_rows(p, out_dev, v_dev, ncols, 0, p->n);
}

int gpb_forward_matvec_host(gpb_provider* p, float* out_host, const float* v_host,
                            int64_t ncols) {
  GPB_REQUIRE(p && out_host && v_host && ncols >= 0, GPB_ERR_INVALID, "bad arguments");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  const size_t bytes = (size_t)p->n * ncols * sizeof(float);
  void *vd = nullptr, *od = nullptr;
  GPB_TRY(p->ws.get(WS_VTMP, bytes + 16, &vd));
  GPB_TRY(p->ws.get(WS_OTMP, bytes + 16, &od));
  GPB_CHECK_CUDA(cudaMemcpyAsync(vd, v_host, bytes, cudaMemcpyHostToDevice, p->stream));
  GPB_TRY(gpb_forward_matvec(p, (float*)od, (const float*)vd, ncols));
  GPB_CHECK_CUDA(cudaMemcpyAsync(out_host, od, bytes, cudaMemcpyDeviceToHost, p->stream));
  return gpb_provider_synchronize(p);
}

int gpb_cross_matvec(gpb_provider* p, float* out_dev, const float* xtest_dev, const float* v_dev,
                     int64_t n_test, int64_t ncols) {
  GPB_REQUIRE(p && out_dev && xtest_dev && v_dev, GPB_ERR_INVALID, "null argument");
  GPB_REQUIRE(n_test >= 0 && ncols >= 0, GPB_ERR_INVALID, "negative size");
  if (n_test == 0 || ncols == 0) return GPB_OK;
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  const float* xt = nullptr;
  GPB_TRY(provider_prescale_rows(p, xtest_dev, n_test, WS_XTEST, &xt, p->stream));
  return provider_kv(p, xt, n_test, v_dev, p->n, ncols, out_dev, n_test, false, 0, p->stream);
}

int gpb_extract_diagonal(gpb_provider* p, float* diag_dev) {
  GPB_REQUIRE(p && diag_dev, GPB_ERR_INVALID, "null argument");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  diag_kernel<<<(unsigned)ceil_div(p->n, 128), 128, 0, p->stream>>>(p->X_d, p->n, p->d, p->dk,
                                                                    diag_dev);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int gpb_extract_diagonal_test(gpb_provider* p, float* diag_dev, const float* xtest_dev,
                              int64_t n_test) {
  GPB_REQUIRE(p && diag_dev && xtest_dev && n_test >= 0, GPB_ERR_INVALID, "bad arguments");
  if (n_test == 0) return GPB_OK;
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  diag_kernel<<<(unsigned)ceil_div(n_test, 128), 128, 0, p->stream>>>(xtest_dev, n_test, p->d,
                                                                      p->dk, diag_dev);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int gpb_kernel_column(gpb_provider* p, float* out_dev, int64_t pivot) {
  GPB_REQUIRE(p && out_dev, GPB_ERR_INVALID, "null argument");
  GPB_REQUIRE(pivot >= 0 && pivot < p->n, GPB_ERR_INVALID, "pivot %lld out of range",
              (long long)pivot);
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  column_kernel<<<(unsigned)ceil_div(p->n, 128), 128, 0, p->stream>>>(p->X_d, p->n, p->d, pivot,
                                                                      p->dk, out_dev);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int gpb_benchmark_forward(gpb_provider* p, const float* v_dev, float* out_dev, int64_t ncols,
                          int32_t warmup, int32_t steps, int32_t flush_l2, double* step_ms_out,
                          double* kernel_ms_out, int64_t* launches_out) {
  GPB_REQUIRE(p && v_dev && out_dev && ncols >= 1 && warmup >= 0 && steps >= 1 && step_ms_out &&
                  kernel_ms_out && launches_out,
              GPB_ERR_INVALID, "bad benchmark arguments");
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  cudaEvent_t e0, e1, k0, k1;
  GPB_CHECK_CUDA(cudaEventCreate(&e0));
  GPB_CHECK_CUDA(cudaEventCreate(&e1));
  GPB_CHECK_CUDA(cudaEventCreate(&k0));
  GPB_CHECK_CUDA(cudaEventCreate(&k1));
  void* flush = nullptr;
  const size_t flush_bytes = (size_t)256 << 20;  // 2x the 126 MB L2
  int status = GPB_OK;
  if (flush_l2) status = p->ws.get(WS_MISC + 1, flush_bytes, &flush);
  for (int it = 0; status == GPB_OK && it < warmup + steps; ++it) {
    if (flush) cudaMemsetAsync(flush, it & 0xff, flush_bytes, p->stream);
    const bool timed = it >= warmup;
    if (timed) {
      p->tile_ev[0] = k0;
      p->tile_ev[1] = k1;
      cudaEventRecord(e0, p->stream);
      p->launches = 0;
    }
    status = gpb_forward_matvec(p, out_dev, v_dev, ncols);
    if (timed) {
      cudaEventRecord(e1, p->stream);
      p->tile_ev[0] = p->tile_ev[1] = nullptr;
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
  p->tile_ev[0] = p->tile_ev[1] = nullptr;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaEventDestroy(k0);
  cudaEventDestroy(k1);
  if (status != GPB_OK) return status;
  return provider_check_device_error(p);
}

}  // extern "C"
