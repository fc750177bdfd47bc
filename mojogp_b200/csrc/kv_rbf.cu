// Tiled K·V instantiations for the fast RBF evaluator.
#include "kv_impl.cuh"

namespace gpb {
int launch_kv_rbf(const KvLaunch& L) { return kv_launch_fast<FastEval<GPB_KERNEL_RBF>>(L); }
}  // namespace gpb

#ifdef GPB_GRAM_PROFILE
// Diagnostic build only: role / wait cycle counters of the RBF Gram kernel.
extern "C" int gpb_debug_gram_prof(unsigned long long* out, int reset) {
  cudaMemcpyFromSymbol(out, gpb::g_gram_prof, 16 * sizeof(unsigned long long));
  if (reset) {
    unsigned long long z[16] = {0};
    cudaMemcpyToSymbol(gpb::g_gram_prof, z, sizeof(z));
  }
  return 0;
}
#endif
