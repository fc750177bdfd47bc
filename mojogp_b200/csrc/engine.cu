// Engine plumbing: buffers, sharded matvec with packed all-gather, column
// dot products with cross-rank all-reduce.
#include "engine.cuh"

namespace gpb {

int DBuf::ensure(size_t b) {
  if (bytes >= b && ptr) return GPB_OK;
  release();
  const size_t want = std::max<size_t>(b, 16);
  cudaError_t e = cudaMalloc(&ptr, want);
  if (e != cudaSuccess) {
    ptr = nullptr;
    set_error("device allocation of %zu bytes failed: %s", want, cudaGetErrorString(e));
    return GPB_ERR_NOMEM;
  }
  bytes = want;
  return GPB_OK;
}

void DBuf::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
}

int Engine::init(gpb_provider* prov, const Dist& d) {
  p = prov;
  dist = d;
  st = prov->stream;
  n = prov->n;
  shard_bounds(n, dist.world, dist.rank, &r0, &r1);
  nl = r1 - r0;
  int64_t maxl = 0;
  for (int g = 0; g < dist.world; ++g) {
    int64_t a, b;
    shard_bounds(n, dist.world, g, &a, &b);
    maxl = std::max(maxl, b - a);
  }
  nl_pad = round_up(std::max<int64_t>(maxl, 1), kJT);
  return GPB_OK;
}

int Engine::allreduce_sum(double* dev, size_t count) {
  if (dist.world <= 1 || count == 0) return GPB_OK;
  ncclResult_t r = ncclAllReduce(dev, dev, count, ncclDouble, ncclSum, dist.comm, st);
  GPB_REQUIRE(r == ncclSuccess, GPB_ERR_NCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
  return GPB_OK;
}

int Engine::allreduce_sum_f(float* dev, size_t count) {
  if (dist.world <= 1 || count == 0) return GPB_OK;
  ncclResult_t r = ncclAllReduce(dev, dev, count, ncclFloat, ncclSum, dist.comm, st);
  GPB_REQUIRE(r == ncclSuccess, GPB_ERR_NCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
  return GPB_OK;
}

__global__ void scatter_shards_kernel(const float* staged, int64_t nl_pad, int t, int world,
                                      int64_t n, float* full) {
  // staged [world][t][nl_pad] -> full [t][n]
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)t * n) return;
  const int c = (int)(idx / n);
  const int64_t i = idx - (int64_t)c * n;
  // owner of row i: largest g with r0(g) <= i
  int g = (int)((i * world) / n);
  while (g + 1 < world && (n * (g + 1)) / world <= i) ++g;
  while (g > 0 && (n * g) / world > i) --g;
  const int64_t r0 = (n * g) / world;
  full[idx] = staged[((int64_t)g * t + c) * nl_pad + (i - r0)];
}

int Engine::allgather_cols(const float* local, int64_t ld_local, int t, float* full) {
  if (dist.world <= 1) {
    if (ld_local == n) return k_copy(full, local, (int64_t)t * n, st);
    for (int c = 0; c < t; ++c) GPB_TRY(k_copy(full + (int64_t)c * n, local + c * ld_local, n, st));
    return GPB_OK;
  }
  DBuf& stage = xv;  // reuse the packed buffer as staging
  GPB_TRY(stage.ensure((size_t)dist.world * t * nl_pad * sizeof(float)));
  float* mine = stage.f() + (int64_t)dist.rank * t * nl_pad;
  for (int c = 0; c < t; ++c) GPB_TRY(k_copy(mine + (int64_t)c * nl_pad, local + c * ld_local, nl, st));
  ncclResult_t r = ncclAllGather(mine, stage.f(), (size_t)t * nl_pad, ncclFloat, dist.comm, st);
  GPB_REQUIRE(r == ncclSuccess, GPB_ERR_NCCL, "ncclAllGather: %s", ncclGetErrorString(r));
  const int64_t total = (int64_t)t * n;
  scatter_shards_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(stage.f(), nl_pad, t,
                                                                       dist.world, n, full);
  GPB_CHECK_CUDA(cudaGetLastError());
  return GPB_OK;
}

int Engine::coldots(int npairs, const float* const* a, const float* const* b, int64_t ld, int t,
                    bool to_host) {
  GPB_TRY(k_coldots(npairs, a, b, ld, nl, t, red, st));
  GPB_TRY(allreduce_sum(red.sums.d(), (size_t)npairs * t));
  if (to_host) {
    host_sums.resize((size_t)npairs * t);
    GPB_CHECK_CUDA(cudaMemcpyAsync(host_sums.data(), red.sums.ptr,
                                   host_sums.size() * sizeof(double), cudaMemcpyDeviceToHost, st));
    GPB_CHECK_CUDA(cudaStreamSynchronize(st));
  }
  return GPB_OK;
}

int Engine::matvec(float* v_local, int64_t v_ld, int t, float* out, int64_t out_ld,
                   const float* update_z, const float* update_beta) {
  if (op) {
    GPB_REQUIRE(v_ld == nl && out_ld == nl, GPB_ERR_UNSUPPORTED,
                "operator matvec needs dense column blocks");
    if (update_beta) GPB_TRY(k_update_p(v_local, update_z, update_beta, nl, v_ld, t, st));
    return op->apply(v_local, v_ld, t, out, st);
  }
  GPB_TRY(provider_refresh_xs(p));
  const int world = dist.world;
  const int64_t rows_total = (int64_t)world * nl_pad;
  const int ntiles = (int)(rows_total / kJT);
  for (int c0 = 0; c0 < t; c0 += 16) {
    const int rem = t - c0;
    const int T = kv_chunk_t(p->eval, p->DP, rem, p->gram_ok);
    const int tcols = std::min(rem, T);
    const int layout = kv_layout(p->eval, p->DP, T, p->gram_ok);
    const int W = kv_packed_width(p->eval, p->DP, T, p->gram_ok);
    GPB_TRY(xv.ensure((size_t)rows_total * W * sizeof(float)));
    float* mine = xv.f() + (int64_t)dist.rank * nl_pad * W;
    if (layout == KV_GRAMH) {
      // Column scales from the maxima over every rank's rows.
      GPB_TRY(launch_gramh_colmax(v_local, v_ld, c0, tcols, nl, mine, update_z, update_beta,
                                  p->DP, st));
      if (world > 1) {
        unsigned* mx = reinterpret_cast<unsigned*>(mine + gramh_max_offset(p->DP));
        ncclResult_t r = ncclAllReduce(mx, mx, 16, ncclUint32, ncclMax, dist.comm, st);
        GPB_REQUIRE(r == ncclSuccess, GPB_ERR_NCCL, "ncclAllReduce(max): %s",
                    ncclGetErrorString(r));
      }
      GPB_TRY(launch_pack_gramh(p->Xs_d + r0 * p->DP, p->DP, v_local, v_ld, c0, tcols, nl, nl_pad,
                                mine, update_z, update_beta, st, false));
      p->launches += 1;
    } else {
      GPB_TRY(k_pack(p->Xs_d + r0 * p->DP, p->DP, v_local, v_ld, c0, tcols, T, nl, nl_pad, mine,
                     update_z, update_beta, st, layout));
    }
    p->launches += 1;
    if (world > 1) {
      ncclResult_t r = ncclAllGather(mine, xv.f(), (size_t)nl_pad * W, ncclFloat, dist.comm, st);
      GPB_REQUIRE(r == ncclSuccess, GPB_ERR_NCCL, "ncclAllGather: %s", ncclGetErrorString(r));
    }
    const int64_t part_floats = std::min<int64_t>((int64_t)32 * T * std::max<int64_t>(nl, 1),
                                                  (int64_t)1 << 29);
    void* part = nullptr;
    GPB_TRY(p->ws.get(WS_PARTIAL, (size_t)part_floats * sizeof(float), &part));
    KvLaunch L{};
    L.eval = p->eval;
    L.DP = p->DP;
    L.T = T;
    L.xrow = p->Xs_d + r0 * p->DP;
    L.nrow = nl;
    L.xv = xv.f();
    L.ntiles = ntiles;
    L.fp = p->fp;
    L.dk = &p->dk;
    L.ep.out = out + (int64_t)c0 * out_ld;
    L.ep.out_ld = out_ld;
    L.ep.scale = p->os_eff;
    L.ep.noise_v = v_local + (int64_t)c0 * v_ld;
    L.ep.noise_ld = v_ld;
    L.ep.noise = p->noise;
    L.ep.noise_vec = p->noise_vec_d ? p->noise_vec_d + r0 : nullptr;
    L.tcols = tcols;
    L.partial = (float*)part;
    L.partial_capacity = part_floats;
    L.err = p->err_d;
    L.stream = st;
    L.launches = &p->launches;
    L.gram_ok = p->gram_ok;
    if (c0 == 0) L.ev_begin = p->tile_ev[0];
    if (c0 + 16 >= t) L.ev_end = p->tile_ev[1];
    GPB_TRY(launch_kv(L));
  }
  return GPB_OK;
}

}  // namespace gpb
