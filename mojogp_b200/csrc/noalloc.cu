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
#include <algorithm>
#include <cstring>

#include "provider.cuh"

namespace gpb {

constexpr int64_t kNoAllocScratchFloats = (int64_t)8 << 20;  // 32 MiB

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of g_noalloc_scratch on the current device. In host code the
// symbol name is only a host-side stand-in and must never be handed to a
// kernel. The lookup runs on every call (it is cheap), so the address stays
// right if the device's context is torn down and the module reloaded.
static int noalloc_scratch(int device, float** out) {
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    set_error("cudaGetSymbolAddress(no-alloc scratch) failed on device %d: %s", device,
              cudaGetErrorString(e));
    return GPB_ERR_CUDA;
  }
  *out = (float*)ptr;
  return GPB_OK;
}

// Packed width of the widest column chunk of an ncols-column product. Chunks
// after the first can run at a narrower T on a different layout whose width
// is larger (at DP = 32: T = 16 packs 64 floats per row on the tensor-core
// layout, T = 8 packs 80 on the paired-row layout), so the first chunk's width
// is not an upper bound.
static int64_t noalloc_max_width(int eval, int DP, int64_t ncols, bool gram) {
  int64_t w = 0;
  for (int64_t c0 = 0; c0 < ncols; c0 += 16)
    w = std::max<int64_t>(w, kv_packed_width(eval, DP, kv_chunk_t(eval, DP, ncols - c0, gram),
                                             gram));
  return w;
}

// max_i |xs_i|^2 over n prescaled rows within the Gram bound, reduced into a
// word of the fixed scratch (one small kernel and one stream synchronisation).
static int noalloc_gram_bounded(const float* xs, int64_t n, int DP, unsigned* word,
                                cudaStream_t st, bool* ok) {
  *ok = false;
  GPB_CHECK_CUDA(cudaMemsetAsync(word, 0, sizeof(unsigned), st));
  GPB_TRY(launch_max_sqnorm(xs, n, DP, word, st));
  unsigned h = 0;
  GPB_CHECK_CUDA(cudaMemcpyAsync(&h, word, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  float hf = 0.f;
  std::memcpy(&hf, &h, sizeof(hf));
  *ok = h != 0xFFFFFFFFu && hf <= kGramMaxSqNorm;
  return GPB_OK;
}

}  // namespace gpb

using namespace gpb;

// Scratch layout, in floats: [64: max-norm word][xs: n*DP, only when the
// provider's prescaled inputs are stale][xv: npad * widest packed width]
// [partial sums: the rest]. When the provider's prescaled inputs are current
// (the usual case after any earlier product on this provider) the call reads
// them and their Gram-bound flag in place, so it runs the same tile kernel as
// gpb_forward_matvec; otherwise it prescales into the array and checks the
// bound itself.
extern "C" int gpb_forward_matvec_noalloc(gpb_provider* p, float* out_dev, const float* v_dev,
                                          int64_t ncols) {
  GPB_REQUIRE(p && out_dev && v_dev && ncols >= 0, GPB_ERR_INVALID, "bad arguments");
  if (ncols == 0) return GPB_OK;
  GPB_CHECK_CUDA(cudaSetDevice(p->device));
  const int64_t n = p->n;
  const int DP = p->DP;
  const int64_t npad = round_up(n, kJT);
  const bool fresh = !p->xs_dirty && p->Xs_d != nullptr;
  const int64_t word_floats = 64;
  const int64_t xs_floats = fresh ? 0 : round_up(n * DP, 64);
  // Size the packed region for either layout choice, so the size check does
  // not depend on the norm reduction that runs later.
  const int64_t W = std::max(noalloc_max_width(p->eval, DP, ncols, false),
                             noalloc_max_width(p->eval, DP, ncols, fresh ? p->gram_ok : true));
  const int64_t xv_floats = round_up(npad * W, 64);
  const int64_t need = word_floats + xs_floats + xv_floats;
  GPB_REQUIRE(need <= kNoAllocScratchFloats, GPB_ERR_INVALID,
              "gpb_forward_matvec_noalloc: n=%lld, ncols=%lld needs %lld scratch floats but the "
              "fixed scratch holds %lld (use gpb_forward_matvec for this size)",
              (long long)n, (long long)ncols, (long long)need, (long long)kNoAllocScratchFloats);
  float* scratch = nullptr;
  GPB_TRY(noalloc_scratch(p->device, &scratch));
  unsigned* word = (unsigned*)scratch;
  float* xv = scratch + word_floats + xs_floats;
  float* partial = scratch + need;
  const int64_t partial_floats = kNoAllocScratchFloats - need;
  cudaStream_t st = p->stream;
  const float* xs = p->Xs_d;
  bool gram = p->gram_ok;
  if (!fresh) {
    float* xs_w = scratch + word_floats;
    GPB_TRY(launch_prescale(p->X_d, n, p->d, p->ps, xs_w, st));
    xs = xs_w;
    gram = false;
    if (p->eval != kEvalGeneric && gram_leaf(p->eval) && (DP == 8 || DP == 16) && n > 0)
      GPB_TRY(noalloc_gram_bounded(xs, n, DP, word, st, &gram));
  }
  for (int64_t c0 = 0; c0 < ncols; c0 += 16) {
    const int64_t rem = ncols - c0;
    const int T = kv_chunk_t(p->eval, DP, rem, gram);
    const int tcols = (int)std::min<int64_t>(rem, T);
    GPB_TRY(launch_pack(xs, DP, v_dev + c0 * n, n, tcols, T, n, npad, xv, st,
                        kv_layout(p->eval, DP, T, gram)));
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
    L.gram_ok = gram;
    GPB_TRY(launch_kv(L));
  }
  return GPB_OK;
}
