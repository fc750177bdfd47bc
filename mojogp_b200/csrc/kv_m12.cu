// Tiled K·V instantiations for the fast MATERN12 evaluator.
#include "kv_impl.cuh"

namespace gpb {
int launch_kv_m12(const KvLaunch& L) { return kv_launch_fast<FastEval<GPB_KERNEL_MATERN12>>(L); }
}  // namespace gpb
