// Host-side matvec helpers shared by the provider and the engine.
#pragma once

#include "kv_launch.cuh"

namespace gpb {

struct PrescaleSpec {
  int DP;
  int nd;
  int dims[GPB_MAX_DIM];
  float scale[GPB_MAX_DIM];
};

int launch_prescale(const float* X, int64_t n, int d, const PrescaleSpec& ps, float* xs,
                    cudaStream_t stream);
// dup = paired-row layout ([-x, -x, ..., v, v, ...], width 2 (DP + T)).
int launch_pack(const float* xs, int DP, const float* v, int64_t v_ld, int tcols, int T, int64_t n,
                int64_t npad, float* xv, cudaStream_t stream, bool dup = false);

}  // namespace gpb
