// b2a_attention_decode_noalloc: the single-token decode of
// b2a_attention_decode, for callers that cannot allocate device memory.
//
// Who cannot allocate, and why:
//  - A serving process that sizes its own pools (KV caches, activations) to
//    fill the GPU's memory at start-up. After that, a cudaMalloc from inside
//    the attention call can fail, or can only succeed by pushing the caller's
//    own allocator out of memory it planned for.
//  - A caller that keeps several streams busy at once. cudaMalloc and cudaFree
//    may synchronize the device, so one attention call that grows its scratch
//    buffer stalls every other stream of the process.
// b2a_attention_decode grows a per-context scratch buffer with cudaMalloc the
// first time a shape needs more room; this entry point never does.
//
// Instead, the split-KV partials live in one file-scope device array of
// B2A_NOALLOC_SCRATCH_BYTES bytes. The CUDA runtime loads a module's device
// code and variables lazily, on first use, and loading allocates device
// memory. So b2a_init, when it creates a context, calls noalloc_prepare below
// for the context's device: that looks up the array's address (which makes
// the runtime create the array) and loads every kernel this decode launches.
// From then on the GPU holds the array until the process exits, and calls of
// b2a_attention_decode_noalloc on that device allocate nothing. A host that
// cannot allocate later should therefore create its contexts before it hands
// the GPU's memory to its own pools. All calls on a device share that one
// array, and it keeps whatever the previous call left in it: nothing in it has
// to start at zero, because every partial the merge step reads is written
// earlier in the same call. Two calls whose work overlaps on the GPU (on
// different streams, or from different contexts on one device) would write
// the same array at the same time and corrupt each other's results; callers
// must order such calls, for example by issuing them on one stream.
//
// Host code cannot pass the array's name to a kernel: in host code that name
// is only a host-side stand-in, not a device address. The set-up looks up the
// array's device address with cudaGetSymbolAddress, once per device and with
// that device current, and keeps it; the decode passes that address to the
// kernels. Because the set-up runs in b2a_init, stream capture that begins
// after the context exists never sees it.
#include <cmath>
#include <mutex>

#include "b2a_internal.cuh"

namespace {

// The one shared scratch array (split-KV partials, f32).
static __device__ __align__(256) unsigned char g_noalloc_scratch[B2A_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Looks up (once per device, with that device current) the device address of
// g_noalloc_scratch.
b2a_status scratch_address(int device, void** out) {
  if (device < 0 || device >= kMaxDevices) return b2a::fail(B2A_ENODEV, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_addr[device] == nullptr) {
    int current = -1;
    cudaError_t e = cudaGetDevice(&current);
    if (e == cudaSuccess && current != device) e = cudaSetDevice(device);
    void* ptr = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      return b2a::cuda_fail(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                            "looking up the device address of the no-alloc scratch array");
    }
    g_scratch_addr[device] = ptr;
  }
  *out = g_scratch_addr[device];
  return B2A_OK;
}

bool valid_dtype(int d) { return d == B2A_F32 || d == B2A_F16 || d == B2A_BF16; }

}  // namespace

namespace b2a {

b2a_status noalloc_prepare(int device) {
  void* ptr = nullptr;
  b2a_status s = scratch_address(device, &ptr);
  if (s != B2A_OK) return s;
  cudaError_t e = preload_attn_mma();
  if (e == cudaSuccess) e = preload_attn_simt();
  if (e == cudaSuccess) e = preload_pages();
  if (e != cudaSuccess) return cuda_fail(e, "loading the decode kernels onto the device");
  return B2A_OK;
}

}  // namespace b2a

extern "C" b2a_status b2a_attention_decode_noalloc(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope,
                                                   int layer_begin, int num_layers, int num_heads, const void* q,
                                                   const void* k_new, const void* v_new, b2a_dtype in_dtype,
                                                   void* out, b2a_dtype out_dtype) {
  using namespace b2a;
  if (ctx == nullptr || c == nullptr || rope == nullptr) return fail(B2A_EINVAL, "null context, cache or rope table");
  if (q == nullptr || out == nullptr) return fail(B2A_EINVAL, "null q or out");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(B2A_EINVAL, "give both new keys and values, or neither");
  if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype)) return fail(B2A_EINVAL, "unknown dtype");
  if (num_heads <= 0 || num_heads % c->kv_heads != 0 || num_heads / c->kv_heads > 8) {
    return fail(B2A_EINVAL, "num_heads %d does not group evenly (at most 8 per KV head) over %d KV heads", num_heads,
                c->kv_heads);
  }
  if (c->head_dim != 64 || rope->head_dim != c->head_dim) return fail(B2A_EINVAL, "head_dim must be 64");
  if (layer_begin < 0 || num_layers < 1 || layer_begin + num_layers > c->layers) {
    return fail(B2A_EINVAL, "layers [%d, %d) outside the cache's %d", layer_begin, layer_begin + num_layers, c->layers);
  }
  int max_keys = 0;
  for (int b = 0; b < c->batch; b++) {
    const int past = c->len[b];
    if (past + 1 > c->capacity) {
      return fail(B2A_ERANGE, "cache holds %d of %d positions; cannot add 1 more", past, c->capacity);
    }
    if (past + 1 > rope->max_positions) {
      return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", past + 1, rope->max_positions);
    }
    if (past + 1 > max_keys) max_keys = past + 1;
  }

  AttnParams p{};
  fill_cache_params(p, c);
  p.seq_begin = 0;
  p.batch = c->batch;
  p.num_layers = num_layers;
  p.layer_begin = layer_begin;
  p.tokens = 1;
  p.heads = num_heads;
  p.kv_heads = c->kv_heads;
  p.group = num_heads / c->kv_heads;
  p.head_dim = c->head_dim;
  p.q = q;
  p.k_new = k_new;
  p.v_new = v_new;
  p.in_dtype = static_cast<int>(in_dtype);
  p.horizon_extra = 1;
  p.rope_cos = rope->d_cos;
  p.rope_sin = rope->d_sin;
  p.rope_cos32 = rope->d_cos32;
  p.rope_sin32 = rope->d_sin32;
  p.rope_max = rope->max_positions;
  p.err = ctx->d_err;
  if (c->has_tmaps) {
    p.tmap_k = &c->tmap_k;
    p.tmap_v = &c->tmap_v;
  }

  // Chunking: the tensor-core path keeps the default planning (many chunks for
  // load balance) when its partials fit; otherwise it takes longer chunks until
  // they do. The CUDA-core path works in chunks of 256 positions.
  const int64_t rows = static_cast<int64_t>(p.batch) * p.num_layers * p.heads;
  const int64_t row_bytes = (p.head_dim + 4) * static_cast<int64_t>(sizeof(float));
  const int64_t cap_rows = B2A_NOALLOC_SCRATCH_BYTES / row_bytes;   // (row, chunk) slots that fit
  const bool mma = attn_mma_supported(p);
  int64_t items = 0;
  bool fits = false;
  if (mma) {
    const int64_t want = 12LL * ctx->sm_count;
    int best = 0;
    for (int chunk : {4096, 2048, 1024, 512, 256}) {
      if (rows * ((max_keys + chunk - 1) / chunk) > cap_rows) break;   // shorter chunks need more room
      p.chunk = chunk;
      items = attn_mma_items(p, c->len.data());
      best = chunk;
      if (items >= want) break;
    }
    if (best == 0) {   // even 4096-position chunks overflow: try longer ones
      for (int chunk : {8192, 16384, 32768, 65536, 131072}) {
        if (rows * ((max_keys + chunk - 1) / chunk) <= cap_rows) {
          p.chunk = chunk;
          items = attn_mma_items(p, c->len.data());
          best = chunk;
          break;
        }
      }
    }
    fits = best != 0;
    if (fits) p.chunk = best;
  } else {
    p.chunk = 256;
    fits = rows * ((max_keys + 255) / 256) <= cap_rows;
  }
  if (!fits) {
    return fail(B2A_ERANGE,
                "decode of %lld query rows over up to %d positions needs more split-KV scratch than the %d-byte "
                "no-alloc array holds; use b2a_attention_decode, or fewer sequences or layers per call",
                static_cast<long long>(rows), max_keys, static_cast<int>(B2A_NOALLOC_SCRATCH_BYTES));
  }
  p.nchunks = (max_keys + p.chunk - 1) / p.chunk;

  int expected = 0;
  if (!ctx->busy.compare_exchange_strong(expected, 1)) {
    return fail(B2A_EBUSY, "a call is already running on this context; wait for it first");
  }
  struct Release {
    b2a_ctx* ctx;
    ~Release() { ctx->busy.store(0); }
  } release{ctx};
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return cuda_fail(e, "selecting the device");
  void* scratch = nullptr;
  b2a_status s = scratch_address(ctx->device, &scratch);
  if (s != B2A_OK) return s;
  p.partial = static_cast<float*>(scratch);
  // a paged cache backs the new slot of every sequence first (host page
  // tables and a by-value table update: no device allocation)
  if ((s = cache_reserve_all(c, 1)) != B2A_OK) return s;

  e = mma ? launch_attn_mma(p, items, ctx->stream) : launch_attn_simt(p, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "launching the attention kernel");
  CombineParams cp{};
  cp.partial = p.partial;
  cp.rows = rows;
  cp.nchunks = p.nchunks;
  cp.head_dim = p.head_dim;
  cp.part_stride_rows = 0;
  cp.out = out;
  cp.out_dtype = static_cast<int>(out_dtype);
  cp.mode = 0;
  cp.len = p.len;
  cp.seq_begin = p.seq_begin;
  cp.chunk = p.chunk;
  cp.extra = p.horizon_extra;
  cp.tokens = p.tokens;
  cp.heads = p.heads;
  cp.num_layers = p.num_layers;
  e = launch_combine(cp, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "launching the split-KV combine");
  return B2A_OK;
}
