// Tiled K·V instantiations for the fast RQ evaluator.
#include "kv_impl.cuh"

namespace gpb {
int launch_kv_rq(const KvLaunch& L) { return kv_launch_fast<FastEval<GPB_KERNEL_RQ>>(L); }
}  // namespace gpb
