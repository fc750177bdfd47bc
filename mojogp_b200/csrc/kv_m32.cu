// Tiled K·V instantiations for the fast MATERN32 evaluator.
#include "kv_impl.cuh"

namespace gpb {
int launch_kv_m32(const KvLaunch& L) { return kv_launch_fast<FastEval<GPB_KERNEL_MATERN32>>(L); }
}  // namespace gpb
