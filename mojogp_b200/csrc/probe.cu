// FP32 throughput probe: the denominator for the matvec roofline.
// A grid of blocks runs independent FFMA chains (8 per thread) for a fixed
// number of iterations; achieved FLOP/s = 2 * FMAs / CUDA-event time.
#include "gpb_common.cuh"

namespace gpb {

__global__ void __launch_bounds__(256) ffma_probe_kernel(const float* __restrict__ seed, int iters,
                                                         float* __restrict__ sink) {
  float a0 = seed[0] + threadIdx.x, a1 = a0 + 1, a2 = a0 + 2, a3 = a0 + 3;
  float a4 = a0 + 4, a5 = a0 + 5, a6 = a0 + 6, a7 = a0 + 7;
  const float b = seed[1], c = seed[2];
#pragma unroll 4
  for (int i = 0; i < iters; ++i) {
    a0 = fmaf(a0, b, c); a1 = fmaf(a1, b, c); a2 = fmaf(a2, b, c); a3 = fmaf(a3, b, c);
    a4 = fmaf(a4, b, c); a5 = fmaf(a5, b, c); a6 = fmaf(a6, b, c); a7 = fmaf(a7, b, c);
  }
  const float s = a0 + a1 + a2 + a3 + a4 + a5 + a6 + a7;
  if (s == 12345.678f) sink[threadIdx.x] = s;  // practically never taken; keeps the chains live
}

}  // namespace gpb

using namespace gpb;

extern "C" int gpb_measure_fp32_peak(int32_t device, double* tflops_out, double* ms_out) {
  GPB_REQUIRE(tflops_out && ms_out, GPB_ERR_INVALID, "null output");
  GPB_CHECK_CUDA(cudaSetDevice(device));
  int sms = 0;
  GPB_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  float* buf = nullptr;
  GPB_CHECK_CUDA(cudaMalloc(&buf, 1024 * sizeof(float)));
  const float h[3] = {0.5f, 0.999999f, 1e-7f};
  GPB_CHECK_CUDA(cudaMemcpy(buf, h, sizeof(h), cudaMemcpyHostToDevice));
  const int blocks = sms * 8, threads = 256, iters = 1 << 16;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  ffma_probe_kernel<<<blocks, threads>>>(buf, 1024, buf + 16);  // warm-up
  float best = 1e30f;
  for (int rep = 0; rep < 3; ++rep) {
    cudaEventRecord(e0);
    ffma_probe_kernel<<<blocks, threads>>>(buf, iters, buf + 16);
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    if (ms < best) best = ms;
  }
  cudaError_t err = cudaGetLastError();
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(buf);
  if (err != cudaSuccess) {
    set_error("fp32 probe: %s", cudaGetErrorString(err));
    return GPB_ERR_CUDA;
  }
  const double flops = 2.0 * 8.0 * (double)iters * blocks * threads;
  *ms_out = best;
  *tflops_out = flops / (best * 1e-3) / 1e12;
  return GPB_OK;
}
