// Instantiation helper: compiles the tile kernel for every supported (DP, T)
// of one evaluator and launches the requested one.
#pragma once

#include "kv_launch.cuh"
#include "kv_tiles_x2.cuh"
#include "kv_tiles_tc.cuh"
#include "kv_tiles_gram.cuh"

namespace gpb {

template <int DP, int T, class Ev, bool kX2>
int kv_launch_impl(const KvLaunch& L);

template <class Ev>
constexpr int leaf_of() {
  if constexpr (Ev::kGeneric) {
    return -1;
  } else {
    return Ev::kLeaf;
  }
}

template <int DP, int LEAF>
int kv_launch_tc(const KvLaunch& L) {
  auto kern = kv_tile_tc_kernel<DP, LEAF>;
  const size_t smem = (size_t)kTcStages * tc_tile_floats(DP) * sizeof(float) + 2 * kTcAStageBytes;
  int dev = 0;
  GPB_CHECK_CUDA(cudaGetDevice(&dev));
  static int resident[64];
  static bool init[64] = {false};
  static int num_sms[64];
  if (dev < 0 || dev >= 64) dev = 0;
  if (!init[dev]) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    GPB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident[dev], kern, kTcThreads + 32, smem));
    GPB_CHECK_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    if (resident[dev] < 1) resident[dev] = 1;
    init[dev] = true;
  }
  const int64_t row_blocks = ceil_div(L.nrow, 128 * kTcRows);
  if (row_blocks == 0 || L.ntiles == 0) return GPB_OK;
  int splits = kv_choose_splits(row_blocks, L.ntiles, resident[dev], num_sms[dev]);
  if (splits > 1) {
    const int64_t need_per_split = (int64_t)16 * L.nrow;
    const int64_t cap = L.partial ? L.partial_capacity / need_per_split : 0;
    if (cap < splits) splits = (int)(cap >= 2 ? cap : 1);
  }
  int tiles_per_split = (int)ceil_div(L.ntiles, splits);
  splits = (int)ceil_div(L.ntiles, tiles_per_split);
  TileEpilogue ep = L.ep;
  ep.tcols = L.tcols;
  if (splits > 1) {
    ep.out = L.partial;
    ep.out_ld = L.nrow;
  }
  if (L.ev_begin) GPB_CHECK_CUDA(cudaEventRecord(L.ev_begin, L.stream));
  kern<<<dim3((unsigned)row_blocks, (unsigned)splits), kTcThreads + 32, smem, L.stream>>>(
      L.xrow, L.nrow, L.xv, L.ntiles, tiles_per_split, L.fp, ep, L.err);
  GPB_CHECK_CUDA(cudaGetLastError());
  if (L.launches) *L.launches += 1;
  if (splits > 1) {
    GPB_TRY(launch_kv_reduce(L, splits));
    if (L.launches) *L.launches += 1;
  }
  if (L.ev_end) GPB_CHECK_CUDA(cudaEventRecord(L.ev_end, L.stream));
  return GPB_OK;
}

template <int DP, int LEAF>
int kv_launch_gram(const KvLaunch& L) {
  auto kern = kv_tile_gram_kernel<DP, LEAF>;
  constexpr int kThreads = kGThreads;
  constexpr int kRows = kGEpiThreads;
  const size_t smem = ((size_t)kGStages * gram_tile_floats(DP)) * sizeof(float);
  int dev = 0;
  GPB_CHECK_CUDA(cudaGetDevice(&dev));
  static int resident[64];
  static bool init[64] = {false};
  static int num_sms[64];
  if (dev < 0 || dev >= 64) dev = 0;
  if (!init[dev]) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    GPB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident[dev], kern, kThreads, smem));
    GPB_CHECK_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    if (resident[dev] < 1) resident[dev] = 1;
    // The kernel allocates all 512 TMEM columns: two CTAs must never share an SM.
    GPB_REQUIRE(resident[dev] == 1, GPB_ERR_UNSUPPORTED, "Gram tile kernel: %d CTAs per SM",
                resident[dev]);
    init[dev] = true;
  }
  const int64_t row_blocks = ceil_div(L.nrow, kRows);
  if (row_blocks == 0 || L.ntiles == 0) return GPB_OK;
  int splits = kv_choose_splits(row_blocks, L.ntiles, resident[dev], num_sms[dev]);
  if (splits > 1) {
    const int64_t need_per_split = (int64_t)16 * L.nrow;
    const int64_t cap = L.partial ? L.partial_capacity / need_per_split : 0;
    if (cap < splits) splits = (int)(cap >= 2 ? cap : 1);
  }
  int tiles_per_split = (int)ceil_div(L.ntiles, splits);
  splits = (int)ceil_div(L.ntiles, tiles_per_split);
  TileEpilogue ep = L.ep;
  ep.tcols = L.tcols;
  if (splits > 1) {
    ep.out = L.partial;
    ep.out_ld = L.nrow;
  }
  if (L.ev_begin) GPB_CHECK_CUDA(cudaEventRecord(L.ev_begin, L.stream));
  kern<<<dim3((unsigned)row_blocks, (unsigned)splits), kThreads, smem, L.stream>>>(
      L.xrow, L.nrow, L.xv, L.ntiles, tiles_per_split, L.fp, ep, L.err);
  GPB_CHECK_CUDA(cudaGetLastError());
  if (L.launches) *L.launches += 1;
  if (splits > 1) {
    GPB_TRY(launch_kv_reduce(L, splits));
    if (L.launches) *L.launches += 1;
  }
  if (L.ev_end) GPB_CHECK_CUDA(cudaEventRecord(L.ev_end, L.stream));
  return GPB_OK;
}

template <int DP, int LEAF>
int kv_launch_gramh(const KvLaunch& L) {
  auto kern = kv_tile_gramh_kernel<DP, LEAF>;
  constexpr int kThreads = kGHThreads;
  constexpr int kRows = kGHEpiThreads;
  const size_t smem = ((size_t)kGStages * gramh_tile_floats(DP)) * sizeof(float);
  int dev = 0;
  GPB_CHECK_CUDA(cudaGetDevice(&dev));
  static int resident[64];
  static bool init[64] = {false};
  static int num_sms[64];
  if (dev < 0 || dev >= 64) dev = 0;
  if (!init[dev]) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    GPB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident[dev], kern, kThreads, smem));
    GPB_CHECK_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    if (resident[dev] < 1) resident[dev] = 1;
    // The kernel allocates all 512 TMEM columns: two CTAs must never share an SM.
    GPB_REQUIRE(resident[dev] == 1, GPB_ERR_UNSUPPORTED, "Gram tile kernel: %d CTAs per SM",
                resident[dev]);
    init[dev] = true;
  }
  const int64_t row_blocks = ceil_div(L.nrow, kRows);
  if (row_blocks == 0 || L.ntiles == 0) return GPB_OK;
  int splits = kv_choose_splits(row_blocks, L.ntiles, resident[dev], num_sms[dev]);
  if (splits > 1) {
    const int64_t need_per_split = (int64_t)16 * L.nrow;
    const int64_t cap = L.partial ? L.partial_capacity / need_per_split : 0;
    if (cap < splits) splits = (int)(cap >= 2 ? cap : 1);
  }
  int tiles_per_split = (int)ceil_div(L.ntiles, splits);
  splits = (int)ceil_div(L.ntiles, tiles_per_split);
  TileEpilogue ep = L.ep;
  ep.tcols = L.tcols;
  if (splits > 1) {
    ep.out = L.partial;
    ep.out_ld = L.nrow;
  }
  if (L.ev_begin) GPB_CHECK_CUDA(cudaEventRecord(L.ev_begin, L.stream));
  kern<<<dim3((unsigned)row_blocks, (unsigned)splits), kThreads, smem, L.stream>>>(
      L.xrow, L.nrow, L.xv, L.ntiles, tiles_per_split, L.fp, ep, L.err);
  GPB_CHECK_CUDA(cudaGetLastError());
  if (L.launches) *L.launches += 1;
  if (splits > 1) {
    GPB_TRY(launch_kv_reduce(L, splits));
    if (L.launches) *L.launches += 1;
  }
  if (L.ev_end) GPB_CHECK_CUDA(cudaEventRecord(L.ev_end, L.stream));
  return GPB_OK;
}


template <int DP, int LEAF, int NV>
int kv_launch_gram1(const KvLaunch& L) {
  auto kern = kv_tile_gram1_kernel<DP, LEAF, NV>;
  // At least 120 KB of shared memory with the ring: the kernel holds all 512
  // TMEM columns, so two CTAs must never share an SM.
  const size_t ring = (size_t)kG1Stages * gram1_tile_floats(DP, NV) * sizeof(float);
  const size_t smem = ring > 120 * 1024 ? ring : 120 * 1024;
  int dev = 0;
  GPB_CHECK_CUDA(cudaGetDevice(&dev));
  static int resident[64];
  static bool init[64] = {false};
  static int num_sms[64];
  if (dev < 0 || dev >= 64) dev = 0;
  if (!init[dev]) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    GPB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident[dev], kern, kG1Threads, smem));
    GPB_CHECK_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    if (resident[dev] < 1) resident[dev] = 1;
    GPB_REQUIRE(resident[dev] == 1, GPB_ERR_UNSUPPORTED, "narrow Gram kernel: %d CTAs per SM",
                resident[dev]);
    init[dev] = true;
  }
  const int64_t row_blocks = ceil_div(L.nrow, kG1EpiThreads);
  if (row_blocks == 0 || L.ntiles == 0) return GPB_OK;
  int splits = kv_choose_splits(row_blocks, L.ntiles, resident[dev], num_sms[dev]);
  if (splits > 1) {
    const int64_t need_per_split = (int64_t)NV * L.nrow;
    const int64_t cap = L.partial ? L.partial_capacity / need_per_split : 0;
    if (cap < splits) splits = (int)(cap >= 2 ? cap : 1);
  }
  int tiles_per_split = (int)ceil_div(L.ntiles, splits);
  splits = (int)ceil_div(L.ntiles, tiles_per_split);
  TileEpilogue ep = L.ep;
  ep.tcols = L.tcols;
  if (splits > 1) {
    ep.out = L.partial;
    ep.out_ld = L.nrow;
  }
  if (L.ev_begin) GPB_CHECK_CUDA(cudaEventRecord(L.ev_begin, L.stream));
  kern<<<dim3((unsigned)row_blocks, (unsigned)splits), kG1Threads, smem, L.stream>>>(
      L.xrow, L.nrow, L.xv, L.ntiles, tiles_per_split, L.fp, ep, L.err);
  GPB_CHECK_CUDA(cudaGetLastError());
  if (L.launches) *L.launches += 1;
  if (splits > 1) {
    GPB_TRY(launch_kv_reduce(L, splits));
    if (L.launches) *L.launches += 1;
  }
  if (L.ev_end) GPB_CHECK_CUDA(cudaEventRecord(L.ev_end, L.stream));
  return GPB_OK;
}

template <int DP, int T, class Ev>
int kv_launch_one(const KvLaunch& L) {
  if constexpr (!Ev::kGeneric && T == 1 && (DP == 8 || DP == 16)) {
    if constexpr (gram_leaf(Ev::kLeaf)) {
      if (kv_layout(L.eval, DP, T, L.gram_ok) == KV_GRAM1)
        return kv_launch_gram1<DP, Ev::kLeaf, T>(L);
    }
  }
  if constexpr (!Ev::kGeneric && T == 16 && (DP == 8 || DP == 16)) {
    if constexpr (gram_leaf(Ev::kLeaf)) {
      if (kv_layout(L.eval, DP, T, L.gram_ok) == KV_GRAMH) return kv_launch_gramh<DP, Ev::kLeaf>(L);
      if (kv_layout(L.eval, DP, T, L.gram_ok) == KV_GRAM) return kv_launch_gram<DP, Ev::kLeaf>(L);
    }
  }
  if constexpr (!Ev::kGeneric && T == 16 && DP % 4 == 0 && DP <= 32) {
    if (kv_layout(L.eval, DP, T, L.gram_ok) == KV_TC) return kv_launch_tc<DP, Ev::kLeaf>(L);
  }
  if constexpr (!Ev::kGeneric && DP % 2 == 0 && T >= 4) {
    if (kv_layout(L.eval, DP, T, L.gram_ok) == KV_X2) return kv_launch_impl<DP, T, Ev, true>(L);
  }
  return kv_launch_impl<DP, T, Ev, false>(L);
}

template <int DP, int T, class Ev, bool kX2>
int kv_launch_impl(const KvLaunch& L) {
  constexpr bool kGen = Ev::kGeneric;
  constexpr int R = kv_rows_per_thread(DP, T, kGen);
  constexpr int W = kX2 ? packed_width_x2(DP, T) : packed_width(DP, T);
  constexpr int S = kX2 ? kStagesX2 : kStages;
  auto kern = [] {
    if constexpr (kX2) {
      return kv_tile_x2_kernel<DP, T, R, kKvBlock, leaf_of<Ev>()>;
    } else {
      return kv_tile_kernel<DP, T, R, kKvBlock, Ev>;
    }
  }();
  // Ring stages plus the per-thread fold slots (R * T floats per thread).
  const size_t smem = (size_t)S * kJT * W * sizeof(float) + (size_t)R * T * kKvBlock * sizeof(float);

  int dev = 0;
  GPB_CHECK_CUDA(cudaGetDevice(&dev));
  static int resident[64];
  static bool init[64] = {false};
  static int num_sms[64];
  if (dev < 0 || dev >= 64) dev = 0;
  if (!init[dev]) {
    GPB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    GPB_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident[dev], kern, kKvBlock, smem));
    GPB_CHECK_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    if (resident[dev] < 1) resident[dev] = 1;
    init[dev] = true;
  }
  const int64_t rows_per_block = (int64_t)kKvBlock * R;
  const int64_t row_blocks = ceil_div(L.nrow, rows_per_block);
  if (row_blocks == 0 || L.ntiles == 0) return GPB_OK;
  GPB_REQUIRE(row_blocks < (1ll << 31), GPB_ERR_INVALID, "too many rows for one launch: %lld",
              (long long)L.nrow);
  int splits = kv_choose_splits(row_blocks, L.ntiles, resident[dev], num_sms[dev]);
  if (splits > 1) {
    const int64_t need_per_split = (int64_t)T * L.nrow;
    const int64_t cap = L.partial ? L.partial_capacity / need_per_split : 0;
    if (cap < splits) splits = (int)(cap >= 2 ? cap : 1);
  }
  int tiles_per_split = (int)ceil_div(L.ntiles, splits);
  splits = (int)ceil_div(L.ntiles, tiles_per_split);

  TileEpilogue ep = L.ep;
  ep.tcols = L.tcols;
  if (splits > 1) {
    ep.out = L.partial;
    ep.out_ld = L.nrow;
  }
  dim3 grid((unsigned)row_blocks, (unsigned)splits);
  typename Ev::Params params;
  if constexpr (kGen) {
    params = *L.dk;
  } else {
    params = L.fp;
  }
  if (L.ev_begin) GPB_CHECK_CUDA(cudaEventRecord(L.ev_begin, L.stream));
  kern<<<grid, kKvBlock, smem, L.stream>>>(L.xrow, L.nrow, L.xv, L.ntiles, tiles_per_split, params,
                                           ep, L.err);
  GPB_CHECK_CUDA(cudaGetLastError());
  if (L.launches) *L.launches += 1;
  if (splits > 1) {
    GPB_TRY(launch_kv_reduce(L, splits));
    if (L.launches) *L.launches += 1;
  }
  if (L.ev_end) GPB_CHECK_CUDA(cudaEventRecord(L.ev_end, L.stream));
  return GPB_OK;
}

template <int DP, class Ev>
int kv_launch_t(const KvLaunch& L) {
  switch (L.T) {
    case 1: return kv_launch_one<DP, 1, Ev>(L);
    case 4: return kv_launch_one<DP, 4, Ev>(L);
    case 8: return kv_launch_one<DP, 8, Ev>(L);
    case 16: return kv_launch_one<DP, 16, Ev>(L);
  }
  set_error("unsupported rhs tile width T=%d", L.T);
  return GPB_ERR_UNSUPPORTED;
}

template <class Ev>
int kv_launch_fast(const KvLaunch& L) {
  switch (L.DP) {
    case 1: return kv_launch_t<1, Ev>(L);
    case 2: return kv_launch_t<2, Ev>(L);
    case 4: return kv_launch_t<4, Ev>(L);
    case 8: return kv_launch_t<8, Ev>(L);
    case 16: return kv_launch_t<16, Ev>(L);
    case 32: return kv_launch_t<32, Ev>(L);
  }
  set_error("unsupported padded dimension DP=%d", L.DP);
  return GPB_ERR_UNSUPPORTED;
}

}  // namespace gpb
