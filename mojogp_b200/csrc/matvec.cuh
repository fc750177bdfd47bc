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
// layout = KvLayout: scalar rows, paired rows ([-x, -x, ..., v, v, ...]) or
// tensor-core tiles ([x' | V hi | V lo] per 128 rows).
int launch_pack(const float* xs, int DP, const float* v, int64_t v_ld, int tcols, int T, int64_t n,
                int64_t npad, float* xv, cudaStream_t stream, int layout = 0);
// Tensor-core tile packing with optional in-place p = z + beta p update
// (columns c0 .. c0+tcols of v).
int launch_pack_tc(const float* xs, int DP, float* v, int64_t v_ld, int c0, int tcols, int64_t n,
                   int64_t npad, float* xv, const float* upd_z, const float* upd_beta,
                   cudaStream_t stream);
// Gram tile packing (KV_GRAM), same arguments.
int launch_pack_gram(const float* xs, int DP, float* v, int64_t v_ld, int c0, int tcols, int64_t n,
                     int64_t npad, float* xv, const float* upd_z, const float* upd_beta,
                     cudaStream_t stream);
// Narrow Gram tile packing (KV_GRAM1, NV = T columns in fp32), same arguments.
int launch_pack_gram1(const float* xs, int DP, int NV, float* v, int64_t v_ld, int c0, int tcols,
                      int64_t n, int64_t npad, float* xv, const float* upd_z,
                      const float* upd_beta, cudaStream_t stream);

// fp16 Gram tile packing (KV_GRAMH), same arguments. With `colmax` the
// column maxima are first reduced into tile 0's tail; without it the caller
// has put them there (the sharded engine all-reduces them between the two).
int launch_pack_gramh(const float* xs, int DP, float* v, int64_t v_ld, int c0, int tcols,
                      int64_t n, int64_t npad, float* xv, const float* upd_z,
                      const float* upd_beta, cudaStream_t stream, bool colmax);
// Zeroes dst's tile-0 column-maximum slots and reduces max |v_c| into them.
int launch_gramh_colmax(float* v, int64_t v_ld, int c0, int tcols, int64_t n, float* dst,
                        const float* upd_z, const float* upd_beta, int DP, cudaStream_t stream);

}  // namespace gpb
