// The provider object: device-resident training inputs, kernel program,
// parameters and noise, plus a grow-only scratch workspace. It plays the role
// of the reference's JITProvider struct (fn_ptr_module.py:159-210).
#pragma once

#include <vector>

#include "kernel_program.cuh"
#include "matvec.cuh"

namespace gpb {

// Grow-only device scratch, one buffer per slot.
struct Workspace {
  std::vector<void*> ptr;
  std::vector<size_t> cap;
  int get(int slot, size_t bytes, void** out);
  void release();
};

enum WsSlot : int {
  WS_XV = 0,       // packed column tiles
  WS_PARTIAL,      // split partial sums
  WS_XTEST,        // prescaled test rows
  WS_VTMP,         // host-variant staging (v)
  WS_OTMP,         // host-variant staging (out)
  WS_GRAD,         // gradient scratch
  WS_MISC,
  WS_NUM_SLOTS
};

}  // namespace gpb

struct gpb_provider {
  int device = 0;
  cudaStream_t stream = nullptr;
  int64_t n = 0;
  int32_t d = 0;
  gpb::DevKernel dk{};          // program + current params
  float noise = 0.f;
  int32_t noise_mode = GPB_NOISE_SCALAR;
  float* noise_vec_d = nullptr;  // fixed per-row noise (mode 1)
  float* X_d = nullptr;          // raw training inputs [n][d]

  // Evaluation plan derived from the program and params.
  int eval = gpb::kEvalGeneric;  // fast leaf id or kEvalGeneric
  int DP = 0;
  float os_eff = 1.f;            // outputscale applied in the epilogue (fast path)
  gpb::FastParams fp{};
  gpb::PrescaleSpec ps{};
  float* Xs_d = nullptr;         // prescaled/padded training inputs [n][DP]
  bool xs_dirty = true;
  bool gram_ok = false;          // max_i |Xs_i|^2 <= kGramMaxSqNorm (Gram tile path allowed)
  unsigned* sqnorm_d = nullptr;  // device word for that reduction

  int* err_d = nullptr;          // device error word
  int64_t launches = 0;          // kernels launched by this provider (diagnostics)
  cudaEvent_t tile_ev[2] = {nullptr, nullptr};  // set only while benchmarking
  gpb::Workspace ws;
};

namespace gpb {

// Rebuild eval plan (fast vs generic, prescale) from dk.params.
int provider_plan(gpb_provider* p);
// Ensure Xs_d matches the current params.
int provider_refresh_xs(gpb_provider* p);
// atomicMax of the bit patterns of |xs_i|^2 over n prescaled rows into *word
// (which the caller zeroes first; NaN maps to 0xFFFFFFFF).
int launch_max_sqnorm(const float* xs, int64_t n, int DP, unsigned* word, cudaStream_t st);
// Check and clear the device error word (synchronizes the stream).
int provider_check_device_error(gpb_provider* p);
// out[c][i] = k(x_{r0 + i}, x*_c) for i < nl, c < m (raw inputs; xt_dev [m][d] on the device).
int cross_fill(gpb_provider* p, int64_t r0, int64_t nl, const float* xt_dev, int m, float* out,
               cudaStream_t st);

// out[c*out_ld + i] = scale * sum_j k(xrow_i, x_j) v[c*v_ld + j]  (+ noise * v for
// the training rows when add_noise). `xrow_prescaled` holds nrow rows already
// prescaled for the provider's plan; `noise_row0` is the global index of the
// first row (for the noise term).
int provider_kv(gpb_provider* p, const float* xrow_prescaled, int64_t nrow, const float* v,
                int64_t v_ld, int64_t ncols, float* out, int64_t out_ld, bool add_noise,
                int64_t noise_row0, cudaStream_t stream);

// Prescale arbitrary rows (e.g. test inputs) for the provider's plan into ws slot.
int provider_prescale_rows(gpb_provider* p, const float* x_raw, int64_t nrow, int slot,
                           const float** out, cudaStream_t stream);

// Bilinear gradient sums over rows [row_begin, row_end) (see gradient.cu).
// a_dev points at row row_begin (column stride a_ld); b_dev holds all n rows.
int provider_bilinear_rows(gpb_provider* p, const float* a_dev, int64_t a_ld, const float* b_dev,
                           int64_t ncols, int64_t row_begin, int64_t row_end, double* data_out,
                           double* trace_out, cudaStream_t st);
// Same with the first `ndata` columns as data columns (the rest are trace
// columns): data_out = sum_{c<ndata} a_c' dK b_c, trace_out over c >= ndata.
int provider_bilinear_rows_nd(gpb_provider* p, const float* a_dev, int64_t a_ld, const float* b_dev,
                              int64_t ncols, int64_t row_begin, int64_t row_end, int64_t ndata,
                              double* data_out, double* trace_out, cudaStream_t st);

}  // namespace gpb
