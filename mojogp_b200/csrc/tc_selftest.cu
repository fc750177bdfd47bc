// Self-test of the tcgen05 building blocks: one 128 x 16 x 8 kind::tf32 MMA
// from shared-memory operands in the no-swizzle K-major layout, accumulator
// read back from TMEM. Used by the tests before any tensor-core kernel runs.
#include "tcgen05.cuh"

namespace gpb {

// A [128][8] and B [16][8] (row = M or N index, 8 = K) in global memory;
// D [128][16] out. `variant` 1 swaps the LBO / SBO roles (diagnostic);
// `variant` 2 stages A in TMEM (tcgen05.st, one column per k) instead of
// shared memory; `variant` 3 does the same with A left in full fp32 (the
// tensor core reads the top 19 bits: truncation to tf32).
__global__ void __launch_bounds__(128) tc_selftest_kernel(const float* __restrict__ A,
                                                          const float* __restrict__ B,
                                                          float* __restrict__ D, int variant,
                                                          int* err) {
  __shared__ __align__(1024) float sA[8192];  // 32 KB: room for either offset reading
  __shared__ __align__(1024) float sB[1024];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tslot;
  const int tid = threadIdx.x;
  for (int q = tid; q < 8192; q += 128) sA[q] = 0.f;
  for (int q = tid; q < 1024; q += 128) sB[q] = 0.f;
  __syncthreads();
  // A: offset(m, k) = (k/4)*2048 + (m/8)*128 + (m%8)*16 + (k%4)*4 bytes
  for (int k = 0; k < 8; ++k)
    sA[((k / 4) * 2048 + (tid / 8) * 128 + (tid % 8) * 16 + (k % 4) * 4) / 4] = to_tf32(A[tid * 8 + k]);
  // B: offset(n, k) = (k/4)*256 + (n/8)*128 + (n%8)*16 + (k%4)*4 bytes
  if (tid < 16)
    for (int k = 0; k < 8; ++k)
      sB[((k / 4) * 256 + (tid / 8) * 128 + (tid % 8) * 16 + (k % 4) * 4) / 4] = to_tf32(B[tid * 8 + k]);
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (tid < 32) tmem_alloc(&tslot, 64);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = tslot;
  if (variant == 2 || variant == 3) {
    uint32_t r[8];
    for (int k = 0; k < 8; ++k)
      r[k] = __float_as_uint(variant == 2 ? to_tf32(A[tid * 8 + k]) : A[tid * 8 + k]);
    tmem_st8(taddr + 32 + ((uint32_t)((tid / 32) * 32) << 16), r);
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint64_t bd = make_smem_desc(sB, 256, 128);
      mma_tf32_tmem_a(taddr, taddr + 32, bd, make_idesc_tf32(128, 16), 0);
      mma_commit(&bar);
    }
  } else if (tid == 0) {
    const uint32_t lboA = variant ? 128 : 2048, sboA = variant ? 2048 : 128;
    const uint32_t lboB = variant ? 128 : 256, sboB = variant ? 256 : 128;
    const uint64_t ad = make_smem_desc(sA, lboA, sboA);
    const uint64_t bd = make_smem_desc(sB, lboB, sboB);
    mma_tf32(taddr, ad, bd, make_idesc_tf32(128, 16), 0);
    mma_commit(&bar);
  }
  const bool ok = mbar_wait_bounded(&bar, 0, 1000000000ull);
  tc_fence_after();
  if (ok) {
    float v[16];
    tmem_ld16(taddr + ((uint32_t)((tid / 32) * 32) << 16), v);
    for (int c = 0; c < 16; ++c) D[tid * 16 + c] = v[c];
  } else if (tid == 0) {
    atomicExch(err, DEV_WAIT_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(taddr, 64);
}

}  // namespace gpb

using namespace gpb;

extern "C" int gpb_tc_selftest(int32_t device, int32_t variant, const float* a_host,
                               const float* b_host, float* d_host) {
  GPB_REQUIRE(a_host && b_host && d_host, GPB_ERR_INVALID, "null argument");
  GPB_CHECK_CUDA(cudaSetDevice(device));
  float *a = nullptr, *b = nullptr, *dd = nullptr;
  int* err = nullptr;
  GPB_CHECK_CUDA(cudaMalloc(&a, 128 * 8 * sizeof(float)));
  GPB_CHECK_CUDA(cudaMalloc(&b, 16 * 8 * sizeof(float)));
  GPB_CHECK_CUDA(cudaMalloc(&dd, 128 * 16 * sizeof(float)));
  GPB_CHECK_CUDA(cudaMalloc(&err, sizeof(int)));
  cudaMemset(err, 0, sizeof(int));
  cudaMemset(dd, 0, 128 * 16 * sizeof(float));
  cudaMemcpy(a, a_host, 128 * 8 * sizeof(float), cudaMemcpyHostToDevice);
  cudaMemcpy(b, b_host, 16 * 8 * sizeof(float), cudaMemcpyHostToDevice);
  tc_selftest_kernel<<<1, 128>>>(a, b, dd, variant, err);
  cudaError_t e = cudaDeviceSynchronize();
  int herr = 0;
  if (e == cudaSuccess) {
    cudaMemcpy(d_host, dd, 128 * 16 * sizeof(float), cudaMemcpyDeviceToHost);
    cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost);
  }
  cudaFree(a);
  cudaFree(b);
  cudaFree(dd);
  cudaFree(err);
  if (e != cudaSuccess) {
    set_error("tc self-test: %s", cudaGetErrorString(e));
    return GPB_ERR_CUDA;
  }
  if (herr) {
    set_error("tc self-test: MMA completion wait timed out");
    return GPB_ERR_DEVICE;
  }
  return GPB_OK;
}
