// Tiled K·V instantiations for the fast RBF evaluator.
#include "kv_impl.cuh"

namespace gpb {
int launch_kv_rbf(const KvLaunch& L) { return kv_launch_fast<FastEval<GPB_KERNEL_RBF>>(L); }
}  // namespace gpb
