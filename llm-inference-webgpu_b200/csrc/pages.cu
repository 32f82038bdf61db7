// Paged KV caches: the host page allocator (b2a_pagepool), the device page
// table it keeps in step, and the reserve / release calls every cache
// operation that adds positions goes through.
//
// The reference's KVCache (src/cpu/cache.js:18-119) gives each sequence one
// block of `capacity` positions; allocate(count) only checks that the block
// has room (cache.js:53-58). A paged cache keeps that per-sequence bound but
// backs a sequence's positions with pages taken from one pool as it grows, so
// the pool is sized for the positions the batch holds. Page tables live on the
// host (the truth, read by the host-side copies) and on the device (read by the
// kernels through kv_elem); the device table is written by a kernel whose
// entries travel by value, so an update is ordered on the stream before the
// launches that read it and no host buffer has to outlive the call.
#include <algorithm>
#include <new>

#include "b2a_internal.cuh"

struct b2a_pagepool {
  int num_pages = 0, page_size = 0, page_shift = 0, batch = 0, max_pages = 0, capacity = 0;
  std::vector<int32_t> table;   // [batch][max_pages]; unmapped entries hold num_pages (the scratch page)
  std::vector<int32_t> mapped;  // pages mapped per sequence: always a prefix of its row
  std::vector<int32_t> free;    // free pages; the next one handed out is at the back
};

namespace b2a {

namespace {

__global__ void k_page_table_update(int32_t* table, PageUpdate u) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < u.n) table[u.idx[i]] = u.page[i];
}

int pages_for(const b2a_pagepool* pool, int64_t positions) {
  return static_cast<int>((positions + pool->page_size - 1) >> pool->page_shift);
}

// Pages sequences first..first+n-1 still need so that positions[i] are backed.
int64_t pages_needed(const b2a_pagepool* pool, int first, int n, const int32_t* positions) {
  int64_t need = 0;
  for (int i = 0; i < n; i++) {
    const int want = pages_for(pool, positions[i]);
    if (want > pool->mapped[first + i]) need += want - pool->mapped[first + i];
  }
  return need;
}

b2a_status exhausted(const b2a_pagepool* pool, int seq, int64_t need) {
  const int used = pool->num_pages - static_cast<int>(pool->free.size());
  return fail(B2A_ERANGE, "page pool exhausted: %d of %d pages in use; sequence %d needs %lld more", used,
              pool->num_pages, seq, static_cast<long long>(need));
}

// Maps the pages; the caller checked that the pool covers them. Each new
// (entry, page) pair is passed to `emit`.
template <class Emit>
void map_pages(b2a_pagepool* pool, int first, int n, const int32_t* positions, Emit&& emit) {
  for (int i = 0; i < n; i++) {
    const int b = first + i;
    const int want = pages_for(pool, positions[i]);
    while (pool->mapped[b] < want) {
      const int32_t page = pool->free.back();
      pool->free.pop_back();
      const int k = pool->mapped[b]++;
      pool->table[static_cast<size_t>(b) * pool->max_pages + k] = page;
      emit(b * pool->max_pages + k, page);
    }
  }
}

// Unmaps one sequence's pages, last page first, so that the free stack hands
// them out again in their old order.
template <class Emit>
void unmap_pages(b2a_pagepool* pool, int b, Emit&& emit) {
  while (pool->mapped[b] > 0) {
    const int k = --pool->mapped[b];
    int32_t& e = pool->table[static_cast<size_t>(b) * pool->max_pages + k];
    pool->free.push_back(e);
    e = pool->num_pages;
    emit(b * pool->max_pages + k, pool->num_pages);
  }
}

// Collects table writes and launches them in batches of kPageUpdateMax.
struct UpdateBatch {
  int32_t* table;
  cudaStream_t st;
  PageUpdate u;
  cudaError_t err = cudaSuccess;
  UpdateBatch(int32_t* t, cudaStream_t s) : table(t), st(s) { u.n = 0; }
  void add(int idx, int32_t page) {
    u.idx[u.n] = idx;
    u.page[u.n] = page;
    if (++u.n == kPageUpdateMax) flush();
  }
  void flush() {
    if (u.n > 0 && err == cudaSuccess) err = launch_page_table_update(table, u, st);
    u.n = 0;
  }
};

}  // namespace

cudaError_t preload_pages() {
  cudaFuncAttributes a;
  return cudaFuncGetAttributes(&a, k_page_table_update);
}

cudaError_t launch_page_table_update(int32_t* table, const PageUpdate& u, cudaStream_t st) {
  if (u.n <= 0) return cudaSuccess;
  k_page_table_update<<<(u.n + 127) / 128, 128, 0, st>>>(table, u);
  return cudaGetLastError();
}

int pool_mapped(const b2a_pagepool* pool, int seq) { return pool->mapped[seq]; }
const int32_t* pool_row(const b2a_pagepool* pool, int seq) {
  return pool->table.data() + static_cast<size_t>(seq) * pool->max_pages;
}

b2a_status cache_reserve(b2a_kvcache* c, int first, int n, const int32_t* positions) {
  if (c->pool == nullptr || n <= 0) return B2A_OK;
  b2a_pagepool* pool = c->pool;
  if (first < 0 || first + n > pool->batch) return fail(B2A_EINVAL, "sequences [%d, %d) out of range", first, first + n);
  for (int i = 0; i < n; i++) {   // callers check capacity first; a table row must never overflow
    if (positions[i] < 0 || positions[i] > pool->capacity) {
      return fail(B2A_ERANGE, "cannot back %d positions of a %d-position sequence", positions[i], pool->capacity);
    }
  }
  const int64_t need = pages_needed(pool, first, n, positions);
  if (need == 0) return B2A_OK;
  if (need > static_cast<int64_t>(pool->free.size())) {
    // name the first sequence that cannot be backed once the ones before it are
    int64_t left = static_cast<int64_t>(pool->free.size());
    for (int i = 0; i < n; i++) {
      const int64_t k = std::max(0, pages_for(pool, positions[i]) - pool->mapped[first + i]);
      if (k > left) return exhausted(pool, first + i, k);
      left -= k;
    }
    return exhausted(pool, first, need);
  }
  UpdateBatch ub(c->d_pages, c->ctx->stream);
  map_pages(pool, first, n, positions, [&](int idx, int32_t page) { ub.add(idx, page); });
  ub.flush();
  if (ub.err != cudaSuccess) return cuda_fail(ub.err, "updating the device page table");
  return B2A_OK;
}

b2a_status cache_reserve_all(b2a_kvcache* c, int extra) {
  if (c->pool == nullptr) return B2A_OK;
  std::vector<int32_t> want(c->batch);
  for (int b = 0; b < c->batch; b++) want[b] = c->len[b] + extra;
  return cache_reserve(c, 0, c->batch, want.data());
}

b2a_status cache_release(b2a_kvcache* c, int seq) {
  if (c->pool == nullptr) return B2A_OK;
  UpdateBatch ub(c->d_pages, c->ctx->stream);
  for (int b = 0; b < c->batch; b++) {
    if (seq >= 0 && b != seq) continue;
    unmap_pages(c->pool, b, [&](int idx, int32_t page) { ub.add(idx, page); });
  }
  ub.flush();
  if (ub.err != cudaSuccess) return cuda_fail(ub.err, "updating the device page table");
  return B2A_OK;
}

}  // namespace b2a

// ------------------------------------------------------------------ C ABI --

extern "C" {

b2a_status b2a_pagepool_create(int num_pages, int page_size, int batch, int capacity, b2a_pagepool** out) {
  using namespace b2a;
  if (out == nullptr) return fail(B2A_EINVAL, "null output pointer");
  *out = nullptr;
  if (capacity < 1) return fail(B2A_ERANGE, "cache capacity must be a positive integer, got %d", capacity);
  if (page_size < 128 || (page_size & (page_size - 1)) != 0) {
    return fail(B2A_EINVAL, "page size must be a power of two of at least 128 positions, got %d", page_size);
  }
  if (num_pages < 1 || batch < 1) {
    return fail(B2A_EINVAL, "a page pool needs at least one page and one sequence (pages %d, batch %d)", num_pages,
                batch);
  }
  b2a_pagepool* p = new (std::nothrow) b2a_pagepool();
  if (p == nullptr) return fail(B2A_EINVAL, "out of host memory");
  p->num_pages = num_pages;
  p->page_size = page_size;
  while ((1 << p->page_shift) < page_size) p->page_shift++;
  p->batch = batch;
  p->capacity = capacity;
  p->max_pages = static_cast<int>((static_cast<int64_t>(capacity) + page_size - 1) / page_size);
  p->table.assign(static_cast<size_t>(batch) * p->max_pages, num_pages);
  p->mapped.assign(batch, 0);
  p->free.resize(num_pages);
  for (int i = 0; i < num_pages; i++) p->free[i] = num_pages - 1 - i;   // page 0 is handed out first
  *out = p;
  return B2A_OK;
}

b2a_status b2a_pagepool_destroy(b2a_pagepool* pool) {
  delete pool;
  return B2A_OK;
}

b2a_status b2a_pagepool_reserve(b2a_pagepool* pool, int seq_idx, int positions) {
  using namespace b2a;
  if (pool == nullptr) return fail(B2A_EINVAL, "null page pool");
  if (seq_idx < 0 || seq_idx >= pool->batch) {
    return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, pool->batch);
  }
  if (positions < 0 || positions > pool->capacity) {
    return fail(B2A_ERANGE, "cannot back %d positions of a %d-position sequence", positions, pool->capacity);
  }
  const int32_t pos = positions;
  const int64_t need = pages_needed(pool, seq_idx, 1, &pos);
  if (need > static_cast<int64_t>(pool->free.size())) return exhausted(pool, seq_idx, need);
  map_pages(pool, seq_idx, 1, &pos, [](int, int32_t) {});
  return B2A_OK;
}

b2a_status b2a_pagepool_release(b2a_pagepool* pool, int seq_idx) {
  using namespace b2a;
  if (pool == nullptr) return fail(B2A_EINVAL, "null page pool");
  if (seq_idx < -1 || seq_idx >= pool->batch) return fail(B2A_EINVAL, "sequence %d out of range", seq_idx);
  for (int b = 0; b < pool->batch; b++) {
    if (seq_idx >= 0 && b != seq_idx) continue;
    unmap_pages(pool, b, [](int, int32_t) {});
  }
  return B2A_OK;
}

b2a_status b2a_pagepool_table(const b2a_pagepool* pool, int seq_idx, int32_t* pages_out, int max_entries,
                              int* mapped) {
  using namespace b2a;
  if (pool == nullptr) return fail(B2A_EINVAL, "null page pool");
  if (seq_idx < 0 || seq_idx >= pool->batch) {
    return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, pool->batch);
  }
  const int m = pool->mapped[seq_idx];
  if (mapped != nullptr) *mapped = m;
  if (pages_out != nullptr) {
    const int32_t* row = pool_row(pool, seq_idx);
    for (int k = 0; k < m && k < max_entries; k++) pages_out[k] = row[k];
  }
  return B2A_OK;
}

b2a_status b2a_pagepool_free_pages(const b2a_pagepool* pool, int* free_pages) {
  using namespace b2a;
  if (pool == nullptr || free_pages == nullptr) return fail(B2A_EINVAL, "null argument");
  *free_pages = static_cast<int>(pool->free.size());
  return B2A_OK;
}

b2a_status b2a_kvcache_page_table(const b2a_kvcache* cache, int seq_idx, int32_t* pages_out, int max_entries,
                                  int* mapped) {
  using namespace b2a;
  if (cache == nullptr) return fail(B2A_EINVAL, "null cache");
  if (seq_idx < 0 || seq_idx >= cache->batch) {
    return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, cache->batch);
  }
  if (cache->pool == nullptr) {
    if (mapped != nullptr) *mapped = 0;
    return B2A_OK;
  }
  return b2a_pagepool_table(cache->pool, seq_idx, pages_out, max_entries, mapped);
}

b2a_status b2a_kvcache_free_pages(const b2a_kvcache* cache, int* free_pages) {
  using namespace b2a;
  if (cache == nullptr || free_pages == nullptr) return fail(B2A_EINVAL, "null argument");
  if (cache->pool == nullptr) {
    *free_pages = 0;
    return B2A_OK;
  }
  return b2a_pagepool_free_pages(cache->pool, free_pages);
}

}  // extern "C"
