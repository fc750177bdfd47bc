// Tiled K·V instantiations for the composite-tree (generic) evaluator.
#include "kv_impl.cuh"

namespace gpb {
int launch_kv_generic(const KvLaunch& L) {
  switch (L.DP) {
    case 4: return kv_launch_t<4, GenericEval>(L);
    case 8: return kv_launch_t<8, GenericEval>(L);
    case 16: return kv_launch_t<16, GenericEval>(L);
    case 32: return kv_launch_t<32, GenericEval>(L);
    case 64: return kv_launch_t<64, GenericEval>(L);
  }
  set_error("unsupported padded dimension DP=%d for composite kernels", L.DP);
  return GPB_ERR_UNSUPPORTED;
}
}  // namespace gpb
