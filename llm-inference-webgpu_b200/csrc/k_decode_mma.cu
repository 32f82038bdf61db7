// Split-KV flash-decode on the tensor cores, for f16 / bf16 caches with
// head_dim 64 and up to 8 query heads per KV head (Qwen2.5: 7).
//
// One CTA owns one work item (sequence b, layer, KV head g, chunk of
// positions). A producer warp streams 64-position K and V tiles of the
// head-major cache into shared memory with 2D TMA (128-byte swizzle, one
// tensor map over the whole pool) through a 4-stage mbarrier ring; four
// consumer warps each take 16 positions of every tile:
//
//   S^T[16 pos x 8 heads] = K[16 x 64] . Q^T[64 x 8]       (4 x mma m16n8k16)
//   online softmax per head (a head's column lives in 8 lanes of one warp)
//   O^T[64 x 8]         += V^T[64 x 16] . P^T[16 x 8]       (4 x mma m16n8k16)
//
// K is the A operand, so the 7 query heads of a group fill the n=8 side of the
// MMA instead of padding a 16-row tile. P^T reaches B-fragment layout with two
// movmatrix transposes, and V^T is read with ldmatrix.trans. For bf16 the
// query and the probabilities are split into a bf16 high part and a bf16
// residual (two MMAs each), which keeps ~16 mantissa bits on both products.
// At the end the four warps' (m, l, O) merge in shared memory into one
// unnormalised partial per query head; k_combine (k_attn_simt.cu) merges the
// chunks. RoPE(q) happens in the prologue in f32 (its operand is rounded to
// 16 bits next); the fused append of the new token's K/V rotates in f64 from
// the host-built table, as every cache write does.
#include <cuda.h>
#include <math_constants.h>

#include <type_traits>

#include "b2a_internal.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {

constexpr int kD = 64;
constexpr int kTile = 64;                 // positions per TMA box
constexpr int kStages = 4;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kTileBytes = kTile * kD * 2;          // 8 KiB per K or V tile
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kSmemRing = kStages * kStageBytes;   // 64 KiB
constexpr float kLog2e = 1.4426950408889634f;
constexpr long long kWaitCycles = 4000000000LL;     // ~2 s at 1.9 GHz, then give up
constexpr int kErrTimeout = 1;
constexpr int kMaxFusedChunks = 64;                 // chunks the fused merge takes (two per lane)

struct __align__(16) MergeSmem {
  float o[kConsumerWarps][8][kD];
  float m[kConsumerWarps][8];
  float l[kConsumerWarps][8];
  int item[4];
};

constexpr int kSmemTotal = kSmemRing + static_cast<int>(sizeof(MergeSmem)) + (2 * kStages + 2) * 8 + 1024;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~2 s, records the timeout in the error word and
// returns false; the caller carries on so no thread of the CTA can hang.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      if (err) atomicOr(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Untiled bulk copy global -> shared (both 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two floats packed as the MMA input type (RNE), low half = first.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<__half2*>(&v));
}
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
}

constexpr long long kPeerWaitNs = 1000000000LL;     // exchange waits give up after ~1 s
constexpr int kErrPeerTimeout = 4;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* a) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint64_t* a, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
// fuse_mode 2: counts this CTA as finished; the launch's last CTA advances the
// exchange's step counter (every CTA that reads it has done so before counting).
__device__ __forceinline__ void exchange_done(const AttnParams& p) {
  if (atomicAdd(p.x_done, 1) == static_cast<int>(gridDim.x) - 1) {
    *p.x_done = 0;
    atomicAdd(p.x_epoch, 1);
  }
}

// Byte offset of (row, 16-byte chunk) in a 128-byte-swizzled tile of 128-byte rows.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kThreads, 3)
    k_decode_mma(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                 AttnParams p) {
  constexpr bool kSplit = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  MergeSmem& ms = *reinterpret_cast<MergeSmem*>(smem + kSmemRing);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSmemRing + sizeof(MergeSmem));
  uint64_t* empty = full + kStages;
  uint64_t* qbar = empty + kStages;   // the query tile and its rotation row landed
  uint64_t* pbar = qbar + 1;          // the fused merge's partials landed

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Programmatic dependent launch: the next kernel in the stream may begin its
  // prologue once every CTA of this grid is resident, and this grid's own
  // reads of anything an earlier kernel writes (lengths, q, k/v, the cache)
  // wait for that kernel to finish. With lengths passed by value the work-item
  // lookup below runs before the wait.
  asm volatile("griddepcontrol.launch_dependents;");
  if (p.n_len_inline == 0) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the earlier kernel's generic-proxy stores are read below by tensor loads (async proxy)
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }

  // ---- which work item: items are numbered sequence-major, each sequence
  // contributing num_layers * kv_heads * chunks(b) of them.
  if (warp == 0) {
    const int item = blockIdx.x;
    int base = 0;
    int found_b = -1, found_off = 0, found_cnt = 0;
    for (int b0 = 0; b0 < p.batch && found_b < 0; b0 += 32) {
      const int b = b0 + lane;
      int cnt = 0;
      if (b < p.batch) {
        const int nk = len_of(p, b) + p.horizon_extra;
        cnt = nk > 0 ? (nk + p.chunk - 1) / p.chunk : 1;
      }
      int items = cnt * p.num_layers * p.kv_heads;
      int incl = items;
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int excl = incl - items;
      const bool mine = b < p.batch && item >= base + excl && item < base + incl;
      const unsigned mask = __ballot_sync(0xffffffffu, mine);
      if (mask) {
        const int src = __ffs(mask) - 1;
        found_b = __shfl_sync(0xffffffffu, b, src);
        found_off = item - base - __shfl_sync(0xffffffffu, excl, src);
        found_cnt = __shfl_sync(0xffffffffu, cnt, src);
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      ms.item[0] = found_b;
      ms.item[1] = found_off;
      ms.item[2] = found_cnt;
    }
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init(qbar, 1);
    mbar_init(pbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (p.n_len_inline != 0) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  __syncthreads();
  const int b = ms.item[0];
  if (b < 0) return;   // grid larger than the item count (cannot happen with the host's count)
  const int off = ms.item[1];
  const int cnt = ms.item[2];
  const int c = off % cnt;
  const int gl = off / cnt;
  const int g = gl % p.kv_heads;
  const int l = gl / p.kv_heads;
  const int G = p.group;
  const int bc = p.seq_begin + b;

  const int past = len_of(p, b);
  const int pos_q = p.q_pos ? p.q_pos[b] : past;
  const int n_keys = past + p.horizon_extra;
  const int p0 = c * p.chunk;
  const int p1 = min(p0 + p.chunk, n_keys);
  const int layer = p.layer_begin + l;
  const double* cosr = p.rope_cos + static_cast<int64_t>(pos_q) * (kD / 2);
  const double* sinr = p.rope_sin + static_cast<int64_t>(pos_q) * (kD / 2);

  // The group's queries and the position's f32 rotation row reach shared
  // memory by bulk copies that the producer issues ahead of the ring fills
  // (plain loads issued beside them wait behind the whole grid's first fills);
  // so do, in the CTA whose chunk holds the new token's slot, the new key and
  // value rows and the f64 rotation row of the fused append. That CTA writes
  // the appended row to the cache and patches it into the shared-memory tile
  // that holds the slot, so its stream starts with everyone else's instead of
  // after the append. Blocks that are not 16-byte aligned take per-element
  // loads, with the append done before the stream starts.
  const int ntiles = (p1 - p0 + kTile - 1) / kTile;
  const bool has_append = p.k_new != nullptr && past >= p0 && past < p1;
  const int in_es = p.in_dtype == DT_F32 ? 4 : 2;
  const int64_t qbase = ((static_cast<int64_t>(b) * p.num_layers + l) * p.heads + g * G) * kD;
  const int64_t nsrc = ((static_cast<int64_t>(b) * p.num_layers + l) * p.kv_heads + g) * kD;
  const unsigned char* qsrc = static_cast<const unsigned char*>(p.q) + qbase * in_es;
  const uint32_t qbytes = static_cast<uint32_t>(G * kD * in_es);
  const uint32_t row_bytes = static_cast<uint32_t>(kD * in_es);
  const float* c32 = p.rope_cos32 + static_cast<int64_t>(pos_q) * (kD / 2);
  const float* s32 = p.rope_sin32 + static_cast<int64_t>(pos_q) * (kD / 2);
  const unsigned char* ksrc = has_append ? static_cast<const unsigned char*>(p.k_new) + nsrc * in_es : nullptr;
  const unsigned char* vsrc = has_append ? static_cast<const unsigned char*>(p.v_new) + nsrc * in_es : nullptr;
  uintptr_t amask = reinterpret_cast<uintptr_t>(qsrc) | reinterpret_cast<uintptr_t>(c32) |
                    reinterpret_cast<uintptr_t>(s32);
  if (has_append) {
    amask |= reinterpret_cast<uintptr_t>(ksrc) | reinterpret_cast<uintptr_t>(vsrc) |
             reinterpret_cast<uintptr_t>(cosr) | reinterpret_cast<uintptr_t>(sinr);
  }
  const bool staged = (amask & 15) == 0;
  // staging areas in the merge area (free until the tile loop ends)
  float* q_raw = &ms.o[2][0][0];                    // raw queries [G][64], <= 2 KiB
  float* stg = &ms.o[3][0][0];                      // 2 KiB:
  float* cs_raw = stg;                              //   f32 cos[32], sin[32]      (256 B)
  unsigned char* k_raw = reinterpret_cast<unsigned char*>(stg + 64);    // new key row  (<= 256 B)
  unsigned char* v_raw = reinterpret_cast<unsigned char*>(stg + 128);   // new value row (<= 256 B)
  double* cs64 = reinterpret_cast<double*>(stg + 192);                  // f64 cos[32], sin[32] (512 B)
  // the tile and the consumer warp whose 16 positions hold the slot
  const int a_tile = (past - p0) / kTile, a_row = (past - p0) % kTile, a_warp = a_row / 16;

  // ---- fused append, unstaged form: before the stream starts
  if (has_append && !staged) {
    if (tid < kD / 2) {
      const int j = tid;
      const int64_t dst = kv_elem(p, bc, layer, g, past);
      float lo, hi;
      rope_pair_f64(ld_as_f32(p.k_new, nsrc + j, p.in_dtype), ld_as_f32(p.k_new, nsrc + j + kD / 2, p.in_dtype),
                    cosr[j], sinr[j], lo, hi);
      st_from_f32(p.kc_w, dst + j, p.cache_dtype, lo);
      st_from_f32(p.kc_w, dst + j + kD / 2, p.cache_dtype, hi);
      convert_elem(p.v_new, nsrc + j, p.in_dtype, p.vc_w, dst + j, p.cache_dtype);
      convert_elem(p.v_new, nsrc + j + kD / 2, p.in_dtype, p.vc_w, dst + j + kD / 2, p.cache_dtype);
      // the tensor-memory-access (async proxy) loads below must see these stores
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncthreads();
  }

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (staged) {
        mbar_arrive_expect_tx(qbar, qbytes + 256 + (has_append ? 2 * row_bytes + 512 : 0));
        bulk_g2s(q_raw, qsrc, qbytes, qbar);
        bulk_g2s(cs_raw, c32, 128, qbar);
        bulk_g2s(cs_raw + 32, s32, 128, qbar);
        if (has_append) {
          bulk_g2s(k_raw, ksrc, row_bytes, qbar);
          bulk_g2s(v_raw, vsrc, row_bytes, qbar);
          bulk_g2s(cs64, cosr, 256, qbar);
          bulk_g2s(cs64 + 32, sinr, 256, qbar);
        }
      }
      for (int i = 0; i < ntiles; i++) {
        const int s = i % kStages;
        if (i >= kStages) mbar_wait(&empty[s], ((i / kStages) - 1) & 1, p.err);
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        unsigned char* st = smem + s * kStageBytes;
        // a 64-position tile starting at a multiple of 64 lies in one page
        const int y = static_cast<int>(kv_elem(p, bc, layer, g, p0 + i * kTile) / kD);
        tma_load_2d(st, &tmap_k, &full[s], 0, y);
        tma_load_2d(st + kTileBytes, &tmap_v, &full[s], 0, y);
      }
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int gq = lane >> 2, tq = lane & 3;
  // RoPE(q) of the group's G heads, staged once in shared memory (the merge
  // area is free until the tile loop ends): every global load is issued before
  // the first use, the rotation runs in f32 (the operand is rounded to 16 bits
  // next, or split into two bf16 parts that keep ~16 bits).
  {
    float* qs = &ms.o[0][0][0];   // [G][64] rotated queries
    constexpr int kPairsPerThread = 2;   // 8 heads x 32 pairs over 128 consumer threads
    float x0[kPairsPerThread], x1[kPairsPerThread], cv[kPairsPerThread], sv[kPairsPerThread];
    if (staged) mbar_wait(qbar, 0, p.err);
#pragma unroll
    for (int r = 0; r < kPairsPerThread; r++) {
      const int idx = tid + r * kConsumerWarps * 32;
      const int h = idx >> 5, j = idx & 31;
      x0[r] = x1[r] = cv[r] = sv[r] = 0.f;
      if (h < G) {
        if (staged) {
          x0[r] = ld_as_f32(q_raw, h * kD + j, p.in_dtype);
          x1[r] = ld_as_f32(q_raw, h * kD + j + 32, p.in_dtype);
          cv[r] = cs_raw[j];
          sv[r] = cs_raw[32 + j];
        } else {
          x0[r] = ld_as_f32(p.q, qbase + h * kD + j, p.in_dtype);
          x1[r] = ld_as_f32(p.q, qbase + h * kD + j + 32, p.in_dtype);
          cv[r] = c32[j];
          sv[r] = s32[j];
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kPairsPerThread; r++) {
      const int idx = tid + r * kConsumerWarps * 32;
      const int h = idx >> 5, j = idx & 31;
      if (h < G) {
        qs[h * kD + j] = fmaf(x0[r], cv[r], -(x1[r] * sv[r]));
        qs[h * kD + j + 32] = fmaf(x1[r], cv[r], x0[r] * sv[r]);
      }
    }
  }
  // ---- fused append, staged form, by the warp that owns the slot's row: the
  // row to the cache, and kept in registers (lane j: dims j and j + 32 of k
  // and v) to be patched into the tile; same arithmetic as the unstaged form
  uint32_t a_k = 0, a_v = 0;   // packed (dim j, dim j + 32) 16-bit codes
  if (has_append && staged && warp == a_warp) {
    const int j = lane;
    const int64_t dst = kv_elem(p, bc, layer, g, past);
    float lo, hi;
    rope_pair_f64(ld_as_f32(k_raw, j, p.in_dtype), ld_as_f32(k_raw, j + kD / 2, p.in_dtype), cs64[j], cs64[32 + j],
                  lo, hi);
    const bool bf = p.cache_dtype == DT_BF16;
    const uint32_t k0 = bf ? f32_to_bf16_bits(lo) : f32_to_f16_bits(lo);
    const uint32_t k1 = bf ? f32_to_bf16_bits(hi) : f32_to_f16_bits(hi);
    uint32_t v0, v1;
    if (p.in_dtype == p.cache_dtype) {
      v0 = reinterpret_cast<const uint16_t*>(v_raw)[j];
      v1 = reinterpret_cast<const uint16_t*>(v_raw)[j + kD / 2];
    } else {
      const float x0v = ld_as_f32(v_raw, j, p.in_dtype), x1v = ld_as_f32(v_raw, j + kD / 2, p.in_dtype);
      v0 = bf ? f32_to_bf16_bits(x0v) : f32_to_f16_bits(x0v);
      v1 = bf ? f32_to_bf16_bits(x1v) : f32_to_f16_bits(x1v);
    }
    uint16_t* kc = static_cast<uint16_t*>(p.kc_w);
    uint16_t* vc = static_cast<uint16_t*>(p.vc_w);
    kc[dst + j] = static_cast<uint16_t>(k0);
    kc[dst + j + kD / 2] = static_cast<uint16_t>(k1);
    vc[dst + j] = static_cast<uint16_t>(v0);
    vc[dst + j + kD / 2] = static_cast<uint16_t>(v1);
    a_k = k0 | (k1 << 16);
    a_v = v0 | (v1 << 16);
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  // Q^T B-fragments for head gq (zero for padding heads): b0 = dims 16ks+2tq..+1,
  // b1 = dims 16ks+8+2tq..+1; ks 0-1 are dims 0..31, ks 2-3 dims 32..63.
  uint32_t qb[4][2];
  uint32_t qlo[4][2];
  {
    const float* qh = &ms.o[0][0][0] + gq * kD;
    const bool valid = gq < G;
#pragma unroll
    for (int ks = 0; ks < 4; ks++) {
      float qv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) qv[e] = valid ? qh[16 * ks + (e >> 1) * 8 + 2 * tq + (e & 1)] : 0.f;
      qb[ks][0] = pack2<T>(qv[0], qv[1]);
      qb[ks][1] = pack2<T>(qv[2], qv[3]);
      if (kSplit) {
        const float2 h0 = unpack2<T>(qb[ks][0]), h1 = unpack2<T>(qb[ks][1]);
        qlo[ks][0] = pack2<T>(qv[0] - h0.x, qv[1] - h0.y);
        qlo[ks][1] = pack2<T>(qv[2] - h1.x, qv[3] - h1.y);
      }
    }
  }
  // every consumer has its fragments before any warp reuses the merge area
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");

  const float sc = rsqrtf(static_cast<float>(kD)) * kLog2e;   // score -> base-2 exponent
  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F;                // raw-score max, heads 2tq, 2tq+1
  float l0 = 0.f, l1 = 0.f;                                    // this thread's share of the sums
  float o[4][4];
#pragma unroll
  for (int mb = 0; mb < 4; mb++)
#pragma unroll
    for (int e = 0; e < 4; e++) o[mb][e] = 0.f;

  const uint32_t ring = smem_u32(smem);
  for (int i = 0; i < ntiles; i++) {
    const int s = i % kStages;
    mbar_wait(&full[s], (i / kStages) & 1, p.err);
    const int valid = min(kTile, p1 - (p0 + i * kTile)) - 16 * warp;   // positions of my 16 that exist
    // the appended row, when it lies in my 16 positions of this tile: lane j
    // writes dims j and j + 32 of k and v over what the tile load brought
    const bool patch = has_append && staged && i == a_tile && warp == a_warp;
    if (patch) {
      unsigned char* kt0 = smem + s * kStageBytes;
      const int j = lane;
      const uint32_t o0 = swz(a_row, j >> 3) + 2 * (j & 7), o1 = swz(a_row, (j + kD / 2) >> 3) + 2 * (j & 7);
      *reinterpret_cast<uint16_t*>(kt0 + o0) = static_cast<uint16_t>(a_k);
      *reinterpret_cast<uint16_t*>(kt0 + o1) = static_cast<uint16_t>(a_k >> 16);
      *reinterpret_cast<uint16_t*>(kt0 + kTileBytes + o0) = static_cast<uint16_t>(a_v);
      *reinterpret_cast<uint16_t*>(kt0 + kTileBytes + o1) = static_cast<uint16_t>(a_v >> 16);
      __syncwarp();
    }
    if (valid > 0) {
      const uint32_t kt = ring + s * kStageBytes;
      const uint32_t vt = kt + kTileBytes;
      if (valid < 16) {
        // zero V rows past the end so 0 * (stale bits) cannot make NaN
        unsigned char* vrow = smem + s * kStageBytes + kTileBytes + (16 * warp + valid) * 128;
        for (int x = lane; x < (16 - valid) * 8; x += 32) reinterpret_cast<uint4*>(vrow)[x] = make_uint4(0, 0, 0, 0);
        __syncwarp();
      }
      // S^T = K . Q^T
      float st[4] = {0.f, 0.f, 0.f, 0.f};
      const int r = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int ks = 0; ks < 4; ks++) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kt + swz(r, 2 * ks + (lane >> 4)), a0, a1, a2, a3);
        mma16816<T>(st, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
        if (kSplit) mma16816<T>(st, a0, a1, a2, a3, qlo[ks][0], qlo[ks][1]);
      }
      if (valid < 16) {
        if (gq >= valid) st[0] = st[1] = -CUDART_INF_F;
        if (gq + 8 >= valid) st[2] = st[3] = -CUDART_INF_F;
      }
      // online softmax, heads 2tq (st[0], st[2]) and 2tq+1 (st[1], st[3])
      float t0 = fmaxf(st[0], st[2]), t1 = fmaxf(st[1], st[3]);
#pragma unroll
      for (int x = 4; x < 32; x <<= 1) {
        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, x));
        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, x));
      }
      const float n0 = fmaxf(m0, t0), n1 = fmaxf(m1, t1);
      const float a0s = (m0 == -CUDART_INF_F) ? 0.f : exp2f((m0 - n0) * sc);
      const float a1s = (m1 == -CUDART_INF_F) ? 0.f : exp2f((m1 - n1) * sc);
      m0 = n0;
      m1 = n1;
      const float nb0 = -n0 * sc, nb1 = -n1 * sc;
      const float p00 = exp2f(fmaf(st[0], sc, nb0)), p01 = exp2f(fmaf(st[1], sc, nb1));
      const float p10 = exp2f(fmaf(st[2], sc, nb0)), p11 = exp2f(fmaf(st[3], sc, nb1));
      l0 = fmaf(l0, a0s, p00 + p10);
      l1 = fmaf(l1, a1s, p01 + p11);
#pragma unroll
      for (int mb = 0; mb < 4; mb++) {
        o[mb][0] *= a0s;
        o[mb][2] *= a0s;
        o[mb][1] *= a1s;
        o[mb][3] *= a1s;
      }
      // P^T as B fragments: transpose [pos][head] 8x8 blocks into [head][pos]
      const uint32_t pk0 = pack2<T>(p00, p01), pk1 = pack2<T>(p10, p11);
      const uint32_t pb0 = movmatrix_t(pk0), pb1 = movmatrix_t(pk1);
      uint32_t pl0 = 0, pl1 = 0;
      if (kSplit) {
        const float2 h0 = unpack2<T>(pk0), h1 = unpack2<T>(pk1);
        pl0 = movmatrix_t(pack2<T>(p00 - h0.x, p01 - h0.y));
        pl1 = movmatrix_t(pack2<T>(p10 - h1.x, p11 - h1.y));
      }
      // O^T += V^T . P^T
      const int vr = 16 * warp + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
      for (int mb = 0; mb < 4; mb++) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vt + swz(vr, 2 * mb + ((lane >> 3) & 1)), a0, a1, a2, a3);
        mma16816<T>(o[mb], a0, a1, a2, a3, pb0, pb1);
        if (kSplit) mma16816<T>(o[mb], a0, a1, a2, a3, pl0, pl1);
      }
      if (valid < 16 || patch) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- merge the four warps: per head h, m* = max m_w, scale, sum
#pragma unroll
  for (int x = 4; x < 32; x <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, x);
    l1 += __shfl_xor_sync(0xffffffffu, l1, x);
  }
  if (gq == 0) {
    ms.m[warp][2 * tq] = m0;
    ms.m[warp][2 * tq + 1] = m1;
    ms.l[warp][2 * tq] = l0;
    ms.l[warp][2 * tq + 1] = l1;
  }
#pragma unroll
  for (int mb = 0; mb < 4; mb++) {
    ms.o[warp][2 * tq][16 * mb + gq] = o[mb][0];
    ms.o[warp][2 * tq + 1][16 * mb + gq] = o[mb][1];
    ms.o[warp][2 * tq][16 * mb + 8 + gq] = o[mb][2];
    ms.o[warp][2 * tq + 1][16 * mb + 8 + gq] = o[mb][3];
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));   // consumers only

  const int64_t row0 = (static_cast<int64_t>(b) * p.num_layers + l) * p.heads + g * G;
  const int64_t part_row = static_cast<int64_t>(p.nchunks) * (kD + 4);
  float* part_base = p.partial + row0 * part_row;            // chunk 0 of head 0 of this group
  float* part = part_base + c * (kD + 4);
  // A group whose keys fit in one chunk writes its final result directly
  // (except across ranks, where every group goes through the exchange).
  const bool direct = p.fuse_out != nullptr && cnt == 1 && p.fuse_mode != 2;
  for (int idx = tid; idx < G * kD; idx += kConsumerWarps * 32) {
    const int h = idx / kD, d = idx % kD;
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) mx = fmaxf(mx, ms.m[w][h]);
    float acc = 0.f, ls = 0.f;
    if (mx != -CUDART_INF_F) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; w++) {
        const float mw = ms.m[w][h];
        if (mw != -CUDART_INF_F) {
          const float sw = exp2f((mw - mx) * sc);
          acc = fmaf(sw, ms.o[w][h][d], acc);
          ls = fmaf(sw, ms.l[w][h], ls);
        }
      }
    }
    const float m2 = mx == -CUDART_INF_F ? -CUDART_INF_F : mx * sc;
    if (direct) {
      if (p.fuse_mode == 0) {
        st_from_f32(p.fuse_out, (row0 + h) * kD + d, p.fuse_dtype, acc / ls);
      } else {
        float* o = static_cast<float*>(p.fuse_out) + (row0 + h) * (kD + 4);
        o[d] = acc;
        if (d == 0) {
          o[kD] = m2;
          o[kD + 1] = ls;
          o[kD + 2] = 0.f;
          o[kD + 3] = 0.f;
        }
      }
    } else {
      part[h * part_row + d] = acc;
      if (d == 0) {
        part[h * part_row + kD] = m2;
        part[h * part_row + kD + 1] = ls;
      }
    }
  }
  if (p.fuse_out == nullptr || direct) return;

  // ---- fused merge: the last CTA of this (sequence, layer, KV head) to finish
  // merges the group's `cnt` chunk partials. The barrier orders every thread's
  // partial stores before thread 0's acquire-release add (cumulative at GPU
  // scope); in the last CTA the same add acquires every other CTA's stores.
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  if (tid == 0) {
    int32_t* ctr = p.counters + (static_cast<int64_t>(b) * p.num_layers + l) * p.kv_heads + g;
    int prev;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(ctr) : "memory");
    const bool last = prev == cnt - 1;
    if (last) *ctr = 0;   // ready for the next launch
    ms.item[3] = last ? 1 : 0;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  if (ms.item[3] == 0) {
    if (p.fuse_mode == 2 && tid == 0) exchange_done(p);
    return;
  }
  float* wts = &ms.o[0][0][0];   // two-pass merge: [8 heads][kMaxFusedChunks] chunk weights
  float* xs = wts + 8 * kMaxFusedChunks;   // fuse_mode 2: the group's merged partial [G][D+4]
  float* hinv = &ms.l[0][0];     // per head: 1/L (or L), and m* in ms.m
  // one merged element of head h, dim d (unnormalised sum v)
  auto put = [&](int h, int d, float v) {
    if (p.fuse_mode == 0) {
      st_from_f32(p.fuse_out, (row0 + h) * kD + d, p.fuse_dtype, v * hinv[h]);
      return;
    }
    float* o = p.fuse_mode == 2 ? xs + h * (kD + 4) : static_cast<float*>(p.fuse_out) + (row0 + h) * (kD + 4);
    o[d] = v;
    if (d == 0) {
      o[kD] = ms.m[0][h];
      o[kD + 1] = hinv[h];
      o[kD + 2] = 0.f;
      o[kD + 3] = 0.f;
    }
  };
  // the group's partials, [G][cnt][D+4], into the (drained) ring with one bulk
  // copy per head when they fit: one round trip to L2 instead of two passes
  const uint32_t head_bytes = static_cast<uint32_t>(cnt * (kD + 4) * 4);
  const bool pbulk = G * head_bytes <= static_cast<uint32_t>(kSmemRing);
  if (pbulk) {
    if (tid == 0) {
      // the acquire above made the other CTAs' partial stores visible to this
      // thread; order them, and the consumers' reads of the ring, before the
      // async-proxy copies
      asm volatile("fence.proxy.async.global;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(pbar, G * head_bytes);
      for (int h = 0; h < G; h++) bulk_g2s(smem + h * head_bytes, part_base + h * part_row, head_bytes, pbar);
    }
    mbar_wait(pbar, 0, p.err);
    const float* pv = reinterpret_cast<const float*>(smem);   // [G][cnt][D+4]
    for (int h = warp; h < G; h += kConsumerWarps) {
      const float* ph = pv + h * cnt * (kD + 4);
      float mi[2], li[2];
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const int cc = lane + 32 * u;
        mi[u] = -CUDART_INF_F;
        li[u] = 0.f;
        if (cc < cnt) {
          mi[u] = ph[cc * (kD + 4) + kD];
          li[u] = ph[cc * (kD + 4) + kD + 1];
        }
        if (li[u] > 0.f) mx = fmaxf(mx, mi[u]);
      }
      for (int x = 16; x > 0; x >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
      float L = 0.f;
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const float w = li[u] > 0.f ? exp2f(mi[u] - mx) : 0.f;
        wts[h * kMaxFusedChunks + lane + 32 * u] = w;
        L = fmaf(w, li[u], L);
      }
      for (int x = 16; x > 0; x >>= 1) L += __shfl_xor_sync(0xffffffffu, L, x);
      if (lane == 0) {
        hinv[h] = p.fuse_mode == 0 ? 1.f / L : L;
        ms.m[0][h] = mx;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
    for (int t = tid; t < G * (kD / 4); t += kConsumerWarps * 32) {
      const int h = t / (kD / 4), d4 = t % (kD / 4);
      const float4* src = reinterpret_cast<const float4*>(pv + h * cnt * (kD + 4)) + d4;
      constexpr int kRowVec = (kD + 4) / 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c2 = 0; c2 < cnt; c2++) {
        const float w = wts[h * kMaxFusedChunks + c2];
        const float4 v = src[c2 * kRowVec];
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
      }
      put(h, 4 * d4, acc.x);
      put(h, 4 * d4 + 1, acc.y);
      put(h, 4 * d4 + 2, acc.z);
      put(h, 4 * d4 + 3, acc.w);
    }
  } else {
    // two passes over the partials (L2): per head (one warp each, a lane per
    // chunk and chunk + 32) the chunk weights 2^(m_c - m*) into shared memory,
    // then the weighted sum with a thread per (head, 4 dims), whose loads are
    // coalesced across the warp
    for (int h = warp; h < G; h += kConsumerWarps) {
      const float* ph = part_base + h * part_row;
      float mi[2], li[2];
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const int cc = lane + 32 * u;
        mi[u] = -CUDART_INF_F;
        li[u] = 0.f;
        if (cc < cnt) {
          mi[u] = __ldcg(ph + cc * (kD + 4) + kD);
          li[u] = __ldcg(ph + cc * (kD + 4) + kD + 1);
        }
        if (li[u] > 0.f) mx = fmaxf(mx, mi[u]);
      }
      for (int x = 16; x > 0; x >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
      float L = 0.f;
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const float w = li[u] > 0.f ? exp2f(mi[u] - mx) : 0.f;
        wts[h * kMaxFusedChunks + lane + 32 * u] = w;
        L = fmaf(w, li[u], L);
      }
      for (int x = 16; x > 0; x >>= 1) L += __shfl_xor_sync(0xffffffffu, L, x);
      if (lane == 0) {
        hinv[h] = p.fuse_mode == 0 ? 1.f / L : L;
        ms.m[0][h] = mx;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
    // a thread per (head, 4 dims), 32 chunk loads in flight at a time
    for (int t = tid; t < G * (kD / 4); t += kConsumerWarps * 32) {
      const int h = t / (kD / 4), d4 = t % (kD / 4);
      const float4* src = reinterpret_cast<const float4*>(part_base + h * part_row) + d4;
      constexpr int kRowVec = (kD + 4) / 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c0 = 0; c0 < cnt; c0 += 32) {
        float4 v[32];
#pragma unroll
        for (int u = 0; u < 32; u++)
          v[u] = c0 + u < cnt ? __ldcg(src + (c0 + u) * kRowVec) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 32; u++) {
          const float w = wts[h * kMaxFusedChunks + c0 + u];   // 0 past cnt
          acc.x = fmaf(w, v[u].x, acc.x);
          acc.y = fmaf(w, v[u].y, acc.y);
          acc.z = fmaf(w, v[u].z, acc.z);
          acc.w = fmaf(w, v[u].w, acc.w);
        }
      }
      put(h, 4 * d4, acc.x);
      put(h, 4 * d4 + 1, acc.y);
      put(h, 4 * d4 + 2, acc.z);
      put(h, 4 * d4 + 3, acc.w);
    }
  }
  if (p.fuse_mode != 2) return;

  // ---- exchange across ranks: store this group's merged partial into every
  // rank's buffer (peer stores over NVLink) as 64-bit words (value, step), then
  // read every rank's words here until all carry this step, and combine the
  // ranks in ascending order. A 64-bit aligned store is seen whole or not at
  // all, so the step half vouches for the value half: no flag, no fence.
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");   // xs complete
  const int epoch = __ldcg(p.x_epoch) + 1;
  const int parity = epoch & 1;
  const uint64_t tag = static_cast<uint64_t>(static_cast<uint32_t>(epoch)) << 32;
  const int nwords = G * (kD + 4);
  for (int i = tid; i < p.x_world * nwords; i += kConsumerWarps * 32) {
    const int r = i / nwords, k = i % nwords;
    uint64_t* dst = p.x_peer[r] + ((static_cast<int64_t>(parity) * p.x_world + p.x_rank) * p.x_rows + row0) * (kD + 4) + k;
    st_relaxed_sys(dst, tag | __float_as_uint(xs[k]));
  }
  // read every rank's words until all carry this step: first each rank's
  // (m, l) per head (a thread per (rank, head)), then each rank's outputs (a
  // thread per (head, 4 dims)), every load of a pass in flight together
  const unsigned long long t0 = globaltimer_ns();
  bool gave_up = false;
  auto timed_out = [&]() {
    if (!gave_up && globaltimer_ns() - t0 > kPeerWaitNs) {
      atomicOr(p.err, kErrPeerTimeout);
      gave_up = true;
    }
    return gave_up;
  };
  const int64_t rank_stride = static_cast<int64_t>(p.x_rows) * (kD + 4);   // words between ranks' slots
  const uint64_t* slot0 = p.x_local + (static_cast<int64_t>(parity) * p.x_world * p.x_rows + row0) * (kD + 4);
  float* mlx = xs + 16 * (kD + 4);   // [world][G] weights 2^(m_r - m*) of head h, then 1/L per head
  if (tid < G) {
    const uint64_t* src = slot0 + tid * (kD + 4);
    float mr[kMaxWorld], lr[kMaxWorld];
    while (true) {
      bool ready = true;
#pragma unroll
      for (int r = 0; r < kMaxWorld; r++) {
        mr[r] = -CUDART_INF_F;
        lr[r] = 0.f;
        if (r < p.x_world) {
          const uint64_t wm = ld_relaxed_sys(src + r * rank_stride + kD);
          const uint64_t wl = ld_relaxed_sys(src + r * rank_stride + kD + 1);
          ready &= static_cast<uint32_t>(wm >> 32) == static_cast<uint32_t>(epoch) &&
                   static_cast<uint32_t>(wl >> 32) == static_cast<uint32_t>(epoch);
          mr[r] = __uint_as_float(static_cast<uint32_t>(wm));
          lr[r] = __uint_as_float(static_cast<uint32_t>(wl));
        }
      }
      if (ready || timed_out()) break;
      __nanosleep(64);
    }
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int r = 0; r < kMaxWorld; r++)
      if (lr[r] > 0.f) mx = fmaxf(mx, mr[r]);
    float L = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxWorld; r++) {
      const float w = lr[r] > 0.f ? exp2f(mr[r] - mx) : 0.f;
      if (r < p.x_world) mlx[r * G + tid] = w;
      L = fmaf(w, lr[r], L);
    }
    mlx[kMaxWorld * G + tid] = 1.f / L;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
  for (int t = tid; t < G * (kD / 4); t += kConsumerWarps * 32) {
    const int h = t / (kD / 4), d4 = t % (kD / 4);
    const uint64_t* src = slot0 + h * (kD + 4) + 4 * d4;
    float ov[kMaxWorld][4];
    while (true) {
      bool ready = true;
#pragma unroll
      for (int r = 0; r < kMaxWorld; r++) {
        ov[r][0] = ov[r][1] = ov[r][2] = ov[r][3] = 0.f;
        if (r < p.x_world) {
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const uint64_t wd = ld_relaxed_sys(src + r * rank_stride + e);
            ready &= static_cast<uint32_t>(wd >> 32) == static_cast<uint32_t>(epoch);
            ov[r][e] = __uint_as_float(static_cast<uint32_t>(wd));
          }
        }
      }
      if (ready || timed_out()) break;
      __nanosleep(64);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < kMaxWorld; r++) {
      if (r < p.x_world) {
        const float w = mlx[r * G + h];
#pragma unroll
        for (int e = 0; e < 4; e++) acc[e] = fmaf(w, ov[r][e], acc[e]);
      }
    }
    const float inv = mlx[kMaxWorld * G + h];
#pragma unroll
    for (int e = 0; e < 4; e++) st_from_f32(p.fuse_out, (row0 + h) * kD + 4 * d4 + e, p.fuse_dtype, acc[e] * inv);
  }
  if (tid == 0) exchange_done(p);
}

int attn_mma_max_fused_chunks() { return kMaxFusedChunks; }

bool attn_mma_supported(const AttnParams& p) {
  return p.tmap_k != nullptr && p.tmap_v != nullptr && p.tokens == 1 && p.head_dim == kD && p.group <= 8 &&
         (p.cache_dtype == DT_F16 || p.cache_dtype == DT_BF16);
}

int64_t attn_mma_items(const AttnParams& p, const int32_t* host_len) {
  int64_t items = 0;
  for (int b = 0; b < p.batch; b++) {
    const int nk = host_len[p.seq_begin + b] + p.horizon_extra;
    const int cnt = nk > 0 ? (nk + p.chunk - 1) / p.chunk : 1;
    items += static_cast<int64_t>(cnt) * p.num_layers * p.kv_heads;
  }
  return items;
}

// Loads both instantiations onto the current device (the runtime otherwise
// loads a kernel's code lazily, at its first launch, which allocates device
// memory for it).
cudaError_t preload_attn_mma() {
  cudaFuncAttributes a;
  cudaError_t e = cudaFuncGetAttributes(&a, k_decode_mma<__half>);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, k_decode_mma<__nv_bfloat16>);
  return e;
}

cudaError_t launch_attn_mma(const AttnParams& p, int64_t items, cudaStream_t st) {
  if (!attn_mma_supported(p) || p.chunk % kTile != 0) return cudaErrorInvalidValue;
  if (items == 0) return cudaSuccess;
  if (items > 0x7fffffff) return cudaErrorInvalidValue;
  const CUtensorMap* mk = static_cast<const CUtensorMap*>(p.tmap_k);
  const CUtensorMap* mv = static_cast<const CUtensorMap*>(p.tmap_v);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_f16[64] = {}, attr_bf16[64] = {};
  const bool f16 = p.cache_dtype == DT_F16;
  void (*kern)(const CUtensorMap, const CUtensorMap, AttnParams) = f16 ? k_decode_mma<__half> : k_decode_mma<__nv_bfloat16>;
  bool* attr = f16 ? attr_f16 : attr_bf16;
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal);
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(items));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemTotal;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, *mk, *mv, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace b2a
