// Tiled K·V instantiations for the fast MATERN52 evaluator.
#include "kv_impl.cuh"

namespace gpb {
int launch_kv_m52(const KvLaunch& L) { return kv_launch_fast<FastEval<GPB_KERNEL_MATERN52>>(L); }
}  // namespace gpb
