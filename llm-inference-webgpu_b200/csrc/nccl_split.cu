// Split-KV decode over NCCL behind the C ABI (b2a_split_kv_decode_nccl): the
// collective form beside the in-kernel exchange of b2a_attention_decode_split.
// Each rank holds a contiguous slice of every sequence's positions; a step is
//   1. the rank's unnormalised partials (o, m, l) for every (sequence, layer,
//      head), written by b2a_attention_decode_partial_layers straight into the
//      rank's slot of a [world][rows][heads][head_dim + 4] buffer,
//   2. ncclAllGather of that buffer in place, on the context's stream,
//   3. b2a_lse_combine of the world slots in ascending rank order into `out`
//      (the same bits on every rank).
// NCCL is resolved at the first call with dlopen: the libnccl.so.2 the process
// has loaded already (the one that made the communicator), else the system's.
// The library itself does not link against NCCL, so hosts without it still
// load libb2a; only this entry point then reports B2A_ENCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "b2a_internal.cuh"

using namespace b2a;

namespace {

using AllGatherFn = ncclResult_t (*)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
using ErrorStringFn = const char* (*)(ncclResult_t);

struct NcclApi {
  AllGatherFn all_gather = nullptr;
  ErrorStringFn error_string = nullptr;
};

const NcclApi* nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) return;
    api.all_gather = reinterpret_cast<AllGatherFn>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<ErrorStringFn>(dlsym(h, "ncclGetErrorString"));
  });
  return api.all_gather != nullptr ? &api : nullptr;
}

// The gathered partials of the last call, grown on demand (one per context).
struct GatherBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_mu;
std::vector<std::pair<b2a_ctx*, GatherBuf>> g_bufs;

b2a_status gather_buffer(b2a_ctx* ctx, size_t need, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  GatherBuf* gb = nullptr;
  for (auto& e : g_bufs) {
    if (e.first == ctx) gb = &e.second;
  }
  if (gb == nullptr) {
    g_bufs.emplace_back(ctx, GatherBuf{});
    gb = &g_bufs.back().second;
  }
  if (need > gb->bytes) {
    if (gb->ptr != nullptr) {
      const cudaError_t e = cudaFree(gb->ptr);   // waits for work that may still use it
      gb->ptr = nullptr;
      gb->bytes = 0;
      if (e != cudaSuccess) return cuda_fail(e, "freeing the gather buffer");
    }
    const size_t bytes = need + need / 4 + 4096;
    const cudaError_t e = cudaMalloc(&gb->ptr, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "allocating the gather buffer");
    gb->bytes = bytes;
  }
  *out = gb->ptr;
  return B2A_OK;
}

}  // namespace

namespace b2a {
// b2a_destroy: the context's gather buffer goes with it.
void nccl_split_release(b2a_ctx* ctx) {
  std::lock_guard<std::mutex> lock(g_mu);
  for (size_t i = 0; i < g_bufs.size(); i++) {
    if (g_bufs[i].first == ctx) {
      if (g_bufs[i].second.ptr != nullptr) cudaFree(g_bufs[i].second.ptr);
      g_bufs.erase(g_bufs.begin() + static_cast<long>(i));
      return;
    }
  }
}
}  // namespace b2a

extern "C" {

b2a_status b2a_split_kv_decode_nccl(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope, int layer_begin,
                                    int num_layers, int num_heads, const void* q, const void* k_new,
                                    const void* v_new, b2a_dtype in_dtype, const int32_t* q_positions,
                                    void* nccl_comm, int world, int rank, void* out, b2a_dtype out_dtype,
                                    int flags) {
  if (ctx == nullptr || cache == nullptr || rope == nullptr || q == nullptr || q_positions == nullptr ||
      out == nullptr || nccl_comm == nullptr) {
    return fail(B2A_EINVAL, "null argument");
  }
  if (flags != B2A_DEVICE) return fail(B2A_EINVAL, "the NCCL split-KV decode takes device pointers (B2A_DEVICE)");
  if (world < 1 || rank < 0 || rank >= world) return fail(B2A_EINVAL, "rank %d of world %d", rank, world);
  if (num_layers < 1 || num_heads < 1) return fail(B2A_EINVAL, "layers %d, heads %d", num_layers, num_heads);
  const NcclApi* api = nccl_api();
  if (api == nullptr) return fail(B2A_ENCCL, "libnccl.so.2 (ncclAllGather) could not be loaded");
  const int64_t rows = static_cast<int64_t>(cache->batch) * num_layers;   // (sequence, layer) rows
  const size_t slot_floats = static_cast<size_t>(rows) * num_heads * (cache->head_dim + 4);
  void* buf = nullptr;
  if (!ctx_acquire(ctx)) return busy_fail(ctx);
  b2a_status s = gather_buffer(ctx, static_cast<size_t>(world) * slot_floats * 4, &buf);
  ctx_release(ctx);
  if (s != B2A_OK) return s;
  float* gathered = static_cast<float*>(buf);
  float* mine = gathered + static_cast<size_t>(rank) * slot_floats;
  // the new token's key and value belong to the slice that ends the sequence
  const bool last = rank == world - 1;
  s = b2a_attention_decode_partial_layers(ctx, cache, rope, layer_begin, num_layers, num_heads, q,
                                          last ? k_new : nullptr, last ? v_new : nullptr, in_dtype, q_positions,
                                          mine, B2A_DEVICE);
  if (s != B2A_OK) return s;
  if (!ctx_acquire(ctx)) return busy_fail(ctx);
  cudaSetDevice(ctx->device);
  const ncclResult_t r = api->all_gather(mine, gathered, slot_floats, ncclFloat32,
                                         static_cast<ncclComm_t>(nccl_comm), ctx->stream);
  ctx_release(ctx);
  if (r != ncclSuccess) {
    return fail(B2A_ENCCL, "ncclAllGather: %s", api->error_string ? api->error_string(r) : "error");
  }
  return b2a_lse_combine(ctx, gathered, world, static_cast<int>(rows), num_heads, cache->head_dim, out, out_dtype,
                         B2A_DEVICE);
}

}  // extern "C"
