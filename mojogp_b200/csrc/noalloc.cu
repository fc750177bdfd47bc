// Forward matvec that performs no device allocation.
//
// Some callers cannot call cudaMalloc at the moment they need a product: code
// running under a caller-owned memory pool or arena that forbids outside
// allocations, latency-critical loops where an allocation's implicit
// synchronisation is not allowed, or hosts that must know all device memory
// up front. gpb_forward_matvec may grow the provider's workspace (prescaled
// inputs, packed column tiles, split partial sums). This variant keeps all of
// that scratch in one fixed file-scope device array instead.
//
// The array is loaded with the library: every GPU the library is used on
// holds its kNoAllocScratchFloats floats (32 MiB) until the process exits.
// All calls share it, so two calls whose work overlaps on the GPU (different
// streams, or different providers on the same device) race; callers must
// order them. Every region a call reads is written earlier in the same call,
// so nothing has to be cleared between calls.
#include "provider.cuh"

namespace gpb {

constexpr int64_t kNoAllocScratchFloats = (int64_t)8 << 20;  // 32 MiB

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of g_noalloc_scratch per device, looked up once per device
// (with that device current). In host code the symbol name is only a host
// stand-in and must never be handed to a kernel.
static float* g_scratch_addr[64] = {nullptr};

static int noalloc_scratch(int device, float** out) {
  GPB_REQUIRE(device >= 0 && device < 64, GPB_ERR_INVALID, "device %d out of range", device);
  if (!g_scratch_addr[device]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      set_error("cudaGetSymbolAddress(no-alloc scratch) failed on device %d: %s", device,
                cudaGetErrorString(e));
      return GPB_ERR_CUDA;
    }
    g_scratch_addr[device] = (float*)ptr;
  }
  *out = g_scratch_addr[device];
  return GPB_OK;
}

}  // namespace gpb

using namespace gpb;

extern "C" int gpb_forward_matvec_noalloc(gpb_provider* p, float* out_dev, const float* v_dev,
                                          int64_t ncols) {
  GPB_REQUIRE(p && out_dev && v_dev && ncols >= 0, GPB_ERR_INVALID, "bad arguments");
  if (ncols == 0) return GPB_OK;
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  const int64_t n = p->n;
  const int DP = p->DP;
  const int64_t npad = round_up(n, kJT);
  const int Tmax = kv_pick_t(ncols);
  const int64_t xs_floats = round_up(n * DP, 64);
  const int64_t xv_floats = round_up(npad * kv_packed_width(p->eval, DP, Tmax), 64);
  const int64_t need = xs_floats + xv_floats;
  GPB_REQUIRE(need <= kNoAllocScratchFloats, GPB_ERR_INVALID,
              "gpb_forward_matvec_noalloc: n=%lld needs %lld scratch floats but the fixed "
              "scratch holds %lld (use gpb_forward_matvec for this size)",
              (long long)n, (long long)need, (long long)kNoAllocScratchFloats);
  float* scratch = nullptr;
  GPB_TRY(noalloc_scratch(p->device, &scratch));
  float* xs = scratch;
  float* xv = scratch + xs_floats;
  float* partial = scratch + need;
  const int64_t partial_floats = kNoAllocScratchFloats - need;
  cudaStream_t st = p->stream;
  GPB_TRY(launch_prescale(p->X_d, n, p->d, p->ps, xs, st));
  for (int64_t c0 = 0; c0 < ncols; c0 += 16) {
    const int64_t rem = ncols - c0;
    const int T = kv_pick_t(rem);
    const int tcols = (int)std::min<int64_t>(rem, T);
    GPB_TRY(launch_pack(xs, DP, v_dev + c0 * n, n, tcols, T, n, npad, xv, st,
                        kv_layout(p->eval, DP, T)));
    KvLaunch L{};
    L.eval = p->eval;
    L.DP = DP;
    L.T = T;
    L.xrow = xs;
    L.nrow = n;
    L.xv = xv;
    L.ntiles = (int)(npad / kJT);
    L.fp = p->fp;
    L.dk = &p->dk;
    L.ep.out = out_dev + c0 * n;
    L.ep.out_ld = n;
    L.ep.scale = p->os_eff;
    L.ep.noise_v = v_dev + c0 * n;
    L.ep.noise_ld = n;
    L.ep.noise = p->noise;
    L.ep.noise_vec = p->noise_vec_d;
    L.tcols = tcols;
    L.partial = partial_floats > 0 ? partial : nullptr;
    L.partial_capacity = partial_floats;
    L.err = p->err_d;
    L.stream = st;
    GPB_TRY(launch_kv(L));
  }
  return GPB_OK;
}
