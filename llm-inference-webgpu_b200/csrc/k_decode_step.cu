// One decode step of the whole decoder (every layer, the final norm, the tied
// output projection and the greedy pick) as ONE cooperative kernel with one
// CTA per SM: the batch-1 token loop of src/cpu/model.js:165-186, where the
// layered path's ~8 launches per layer cost more than the weights take to read.
//
// Work split. Every matrix is split by output rows: CTA i owns rows
// [i*R/G, (i+1)*R/G) of each projection (G = CTAs; gate/up by row pairs), so
// its share of every matrix is one contiguous byte range and every output
// element has exactly one writer (no atomics: run-to-run identical results).
// Phases, separated by grid barriers (a monotonic arrival counter in global
// memory, bounded spin):
//   A  rmsnorm(x) -> q/k/v rows (+bias)                         -> qkv scratch
//   B  attention items (head, chunk of 128 keys): RoPE of q and the new key,
//      the append of the new key/value (one item per KV head), scores, exp,
//      the chunk's partial (o, m, l)                              -> partials
//   C  merge the partials per head -> o_proj rows, x += (owner rows)
//   D  rmsnorm(x) -> interleaved gate/up row pairs -> silu(g)*u   -> h scratch
//   E  down rows, x += (owner rows)
//   ... (every layer) ...
//   F  final rmsnorm -> output-projection rows (logits) -> argmax word
//      (atomicMax of a packed (value, -index)); the last CTA to finish writes
//      the token.
//
// Weight streaming. A producer warp walks the same plan as the compute warps
// and streams this CTA's rows of every matrix, in order, through a ring of
// shared-memory stages with bulk async copies (cp.async.bulk with mbarrier
// complete_tx; no multicast). It never waits for a grid barrier, only for a
// free stage, so the next phases' weights are on chip while the grid
// synchronises. A phase's scales, gains and cached attention keys/values
// (which do not depend on this step) are loaded by warps 1-7 while thread 0
// waits at the barrier.
//
// Dot products in integers. The activation vector is expanded once per phase
// into three int8 digits, x ~= s * (d0 + d1/128 + d2/16384) with
// s = max|x|/127 (error <= 2.4e-7 * max|x|), and each weight row is multiplied
// with dp4a (int8 x int8 -> int32, exact): three dp4a per four weights, no
// per-weight conversion. A row's result is scale_row * s * (A0 + A1/128 +
// A2/16384). A warp takes up to four rows of a chunk at once (independent
// dp4a chains and one interleaved shuffle reduction); products against the
// hidden vector keep the digits in registers, the down projection (K =
// intermediate) spreads each chunk over the whole CTA with digits in shared
// memory.
#include <cfloat>
#include <climits>

#include "b2a_internal.cuh"
#include "k_sm100.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {

using namespace sm100;

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;      // + the producer warp
constexpr int kStages = 8;
constexpr int kStageBytes = 16384;
constexpr int kMaxHidden = 1024;
constexpr int kMaxInter = 8192;
constexpr int kMaxOutRows = 2048;               // output-projection rows per CTA
constexpr int kMaxRows = 128;                   // q/k/v rows or gate/up rows per CTA
constexpr int kMaxOwnRows = 16;                 // hidden rows per CTA
constexpr int kDownBatch = 8;                   // down-projection rows per pass
constexpr int kAttnChunk = 128;                 // keys per attention item
constexpr int kPartPitch = 68;                  // o[64], m, l, pad
constexpr int kErrBarrier = 32;                 // error word: a grid barrier gave up
constexpr int kErrStepToken = 16;               // = kErrBadToken

struct StepSmem {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  // phase B: the item's cached keys [128][64] and values [128][64] (f16)
  union {
    float act[kMaxInter];
    uint16_t kv[2][kAttnChunk][64];
  };
  union {
    int32_t dig[3][kMaxInter / 4];        // digits of a K = intermediate activation
    float scores[kAttnChunk];
  };
  int32_t hdig[3][kMaxHidden / 4];        // digits of a K = hidden activation (read into registers)
  float gain[kMaxHidden];                 // rmsnorm gain of the phase
  float rowscale[kMaxOutRows];            // per-row scales of the phase's rows (f32)
  float rowbias[kMaxRows];                // q/k/v bias of the phase's rows
  float xown[kMaxOwnRows];                // this CTA's rows of the residual stream
  float down_part[kConsumerWarps][8];     // down projection: per-warp row sums
  double rope_c[32], rope_s[32];          // cos/sin of this step's position
  float aq[64], ak[64], av[64];           // attention: rotated q, rotated k_new, v_new
  uint16_t k16[64], v16[64];              // the new key/value as stored in the cache
  float ao[kConsumerWarps][64];           // attention: per-warp partial o
  float redf[2][kConsumerWarps];
  double redd[kConsumerWarps];
  int abort;
  float best_v[kConsumerWarps];
  int best_i[kConsumerWarps];
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile_i(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kConsumers) : "memory"); }

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ int part_begin(int i, int G, int R) {
  return static_cast<int>((static_cast<int64_t>(i) * R) / G);
}

// Orderable word of the greedy pick: larger value first, then the smaller
// index; NaN below every number (never picked while a number is present).
__device__ __forceinline__ unsigned long long pick_key(float v, int idx) {
  const uint32_t u = __float_as_uint(v);
  uint32_t ord;
  if (v != v) ord = 0u;
  else ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) | static_cast<uint32_t>(0xffffffffu - static_cast<uint32_t>(idx));
}
__device__ __forceinline__ float key_value(unsigned long long key) {
  const uint32_t ord = static_cast<uint32_t>(key >> 32);
  const uint32_t u = (ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord;
  return __uint_as_float(u);
}

// ---- the plan: the weight stream of one CTA ------------------------------------
// Per layer: 0 qkv rows, 1 o rows, 2 gate/up row pairs, 3 down rows; then the
// output projection. Chunks are whole rows (whole row pairs for gate/up).
struct Seg {
  const int8_t* base;   // row 0 of the matrix
  int r0, r1, K, rpc;   // this CTA's rows, row bytes, rows per chunk
};
constexpr int kSegsPerLayer = 4;

__device__ __forceinline__ Seg plan_seg(const StepParams& p, int layer, int kind, int cta, int G) {
  Seg s;
  s.K = p.hidden;
  if (layer == p.num_layers) {
    s.base = p.emb;
    s.r0 = part_begin(cta, G, p.vocab);
    s.r1 = part_begin(cta + 1, G, p.vocab);
  } else {
    const StepLayer& L = p.layers[layer];
    const int H = p.hidden, I = p.inter, Q = p.hidden + 2 * p.kv_heads * 64;
    switch (kind) {
      case 0:
        s.base = L.qkv;
        s.r0 = part_begin(cta, G, Q);
        s.r1 = part_begin(cta + 1, G, Q);
        break;
      case 1:
        s.base = L.o;
        s.r0 = part_begin(cta, G, H);
        s.r1 = part_begin(cta + 1, G, H);
        break;
      case 2:
        s.base = L.gu;
        s.r0 = 2 * part_begin(cta, G, I);
        s.r1 = 2 * part_begin(cta + 1, G, I);
        break;
      default:
        s.base = L.down;
        s.r0 = part_begin(cta, G, H);
        s.r1 = part_begin(cta + 1, G, H);
        s.K = I;
        break;
    }
  }
  s.rpc = max(1, kStageBytes / s.K);
  const bool in_layer = layer < p.num_layers;
  if (!(in_layer && kind == 3)) s.rpc = min(s.rpc, 4 * kConsumerWarps);   // a warp takes <= 4 rows of a chunk
  if (in_layer && kind == 2) s.rpc = max(2, s.rpc & ~1);                  // whole gate/up pairs
  if (in_layer && kind == 3) s.rpc = min(s.rpc, 4);                       // the CTA-wide down chunk: <= 4 rows
  return s;
}

// ---- the producer warp -------------------------------------------------------
__device__ void producer(const StepParams& p, StepSmem& sm, unsigned char* ring, int cta, int G) {
  if ((threadIdx.x & 31) != 0) return;
  bool dead = false;
  uint32_t iter = 0;
  for (int layer = 0; layer <= p.num_layers && !dead; layer++) {
    const int kinds = layer == p.num_layers ? 1 : kSegsPerLayer;
    for (int kind = 0; kind < kinds && !dead; kind++) {
      const Seg sg = plan_seg(p, layer, kind, cta, G);
      for (int r = sg.r0; r < sg.r1; r += sg.rpc) {
        if (*reinterpret_cast<volatile int*>(&sm.abort)) {
          dead = true;
          break;
        }
        const int s = iter % kStages;
        if (iter >= kStages) mbar_wait(&sm.empty[s], ((iter / kStages) - 1) & 1, p.err, dead);
        if (dead) break;
        const uint32_t bytes = static_cast<uint32_t>(min(sg.rpc, sg.r1 - r) * sg.K);
        mbar_arrive_expect_tx(&sm.full[s], bytes);
        bulk_copy(ring + static_cast<size_t>(s) * kStageBytes, sg.base + static_cast<int64_t>(r) * sg.K, bytes,
                  &sm.full[s]);
        iter++;
      }
    }
  }
  // no copy may still be landing when the CTA exits: wait for the last
  // stage-full of every stage this warp filled (complete already when the
  // consumers took them)
  bool d2 = false;
  for (uint32_t j = iter > kStages ? iter - kStages : 0; j < iter; j++) {
    mbar_wait(&sm.full[j % kStages], (j / kStages) & 1, p.err, d2);
  }
}

// ---- compute-warp helpers ---------------------------------------------------------

// Three int8 digits of t (|t| <= 127): d0 + d1/128 + d2/16384.
__device__ __forceinline__ void digits3(float t, int& d0, int& d1, int& d2) {
  const float r0 = rintf(t);
  const float t1 = (t - r0) * 128.f;
  const float r1 = rintf(t1);
  const float r2 = rintf((t1 - r1) * 128.f);
  d0 = static_cast<int>(r0);
  d1 = static_cast<int>(r1);
  d2 = static_cast<int>(r2);
}
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | ((static_cast<uint32_t>(d) & 0xffu) << 24);
}
// The packed digits of four values times inv -> dst[k * pitch + g], k = 0..2.
__device__ __forceinline__ void store_digits4(int32_t* dst, int pitch, int g, float4 v, float inv) {
  int a[4], b[4], c[4];
  digits3(v.x * inv, a[0], b[0], c[0]);
  digits3(v.y * inv, a[1], b[1], c[1]);
  digits3(v.z * inv, a[2], b[2], c[2]);
  digits3(v.w * inv, a[3], b[3], c[3]);
  dst[g] = static_cast<int32_t>(pack4(a[0], a[1], a[2], a[3]));
  dst[pitch + g] = static_cast<int32_t>(pack4(b[0], b[1], b[2], b[3]));
  dst[2 * pitch + g] = static_cast<int32_t>(pack4(c[0], c[1], c[2], c[3]));
}
__device__ __forceinline__ float max4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// Block-wide (consumer threads) sum of a double and max of a float, one round.
__device__ __forceinline__ void block_sum_max(StepSmem& sm, double& s, float& m) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  }
  if ((tid & 31) == 0) {
    sm.redd[tid >> 5] = s;
    sm.redf[0][tid >> 5] = m;
  }
  consumers_sync();
  s = 0.0;
  m = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; i++) {
    s = __dadd_rn(s, sm.redd[i]);
    m = fmaxf(m, sm.redf[0][i]);
  }
}
// One-round block max / sum; `slot` alternates between consecutive reductions
// so a slot is never rewritten before every thread has read it.
__device__ __forceinline__ float block_max(StepSmem& sm, float m, int slot) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) sm.redf[slot][tid >> 5] = m;
  consumers_sync();
  m = sm.redf[slot][0];
#pragma unroll
  for (int i = 1; i < kConsumerWarps; i++) m = fmaxf(m, sm.redf[slot][i]);
  return m;
}
__device__ __forceinline__ float block_sum(StepSmem& sm, float v, int slot) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((tid & 31) == 0) sm.redf[slot][tid >> 5] = v;
  consumers_sync();
  v = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; i++) v += sm.redf[slot][i];
  return v;
}

// This lane's digits of a K <= 1024 activation: 16-byte units u = lane + 32 j.
struct RegDigits {
  int4 d[2][3];
};
__device__ __forceinline__ void load_reg_digits(const StepSmem& sm, int K, RegDigits& rd) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int u = lane + 32 * j;
#pragma unroll
    for (int k = 0; k < 3; k++) {
      rd.d[j][k] = 16 * u < K ? *reinterpret_cast<const int4*>(&sm.hdig[k][4 * u]) : make_int4(0, 0, 0, 0);
    }
  }
}

// Digits of a K = hidden vector given as one float4 per thread (threads
// t < K/4 hold elements 4t..4t+3), with the vector's max |value|; returns the
// digit scale. Ends with the digits in every warp's registers.
__device__ __forceinline__ float hidden_digits(StepSmem& sm, int K, float4 v, float mx, RegDigits& rd) {
  const int tid = threadIdx.x;
  const float inv = mx > 0.f ? 127.f / mx : 0.f;
  if (4 * tid < K) store_digits4(&sm.hdig[0][0], kMaxHidden / 4, tid, v, inv);
  consumers_sync();
  load_reg_digits(sm, K, rd);
  return mx / 127.f;
}

// rmsnorm (src/core/ops.js:17-24, f64 as k_rmsnorm) of a K = hidden vector
// given as one float4 per thread, gain in sm.gain; then its digits.
__device__ __forceinline__ float norm_digits(StepSmem& sm, int K, float4 x, double eps, RegDigits& rd) {
  const int tid = threadIdx.x;
  double ss = 0.0;
  float mg = 0.f;
  float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
  if (4 * tid < K) {
    g = *reinterpret_cast<const float4*>(&sm.gain[4 * tid]);
    ss = __dadd_rn(__dadd_rn(__dmul_rn(x.x, x.x), __dmul_rn(x.y, x.y)),
                   __dadd_rn(__dmul_rn(x.z, x.z), __dmul_rn(x.w, x.w)));
    mg = max4(make_float4(x.x * g.x, x.y * g.y, x.z * g.z, x.w * g.w));
  }
  block_sum_max(sm, ss, mg);
  const double scale = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, static_cast<double>(K)), eps)));
  float4 n;
  n.x = __double2float_rn(__dmul_rn(__dmul_rn(static_cast<double>(x.x), scale), static_cast<double>(g.x)));
  n.y = __double2float_rn(__dmul_rn(__dmul_rn(static_cast<double>(x.y), scale), static_cast<double>(g.y)));
  n.z = __double2float_rn(__dmul_rn(__dmul_rn(static_cast<double>(x.z), scale), static_cast<double>(g.z)));
  n.w = __double2float_rn(__dmul_rn(__dmul_rn(static_cast<double>(x.w), scale), static_cast<double>(g.w)));
  // the normalised maximum, raised a hair so that no digit exceeds 127
  const float mx = static_cast<float>(static_cast<double>(mg) * scale) * (1.f + 1e-6f);
  return hidden_digits(sm, K, n, mx, rd);
}

__device__ __forceinline__ float combine3(int a0, int a1, int a2) {
  return static_cast<float>(a0) + static_cast<float>(a1) * (1.f / 128.f) + static_cast<float>(a2) * (1.f / 16384.f);
}

// Up to four rows (cnt of them valid; the rest repeat row 0) of K <= 1024
// against the register digits; every lane gets the sums, in digit units.
template <int R>
__device__ __forceinline__ void dot_rows(const unsigned char* base, const uint32_t (&ro)[R], int cnt, int K,
                                         const RegDigits& rd, float (&y)[R]) {
  const int lane = threadIdx.x & 31;
  int a[R][3];
#pragma unroll
  for (int r = 0; r < R; r++) a[r][0] = a[r][1] = a[r][2] = 0;
  // rows in groups of four (four 16-byte weight loads in flight at a time)
#pragma unroll
  for (int g = 0; g < R; g += 4) {
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int u = lane + 32 * j;
      if (16 * u < K) {
        int4 w[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
          if (g + r < cnt) w[r] = *reinterpret_cast<const int4*>(base + ro[g + r] + 16 * u);
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
          if (g + r < cnt) {
#pragma unroll
            for (int k = 0; k < 3; k++) {
              a[g + r][k] = __dp4a(w[r].x, rd.d[j][k].x, a[g + r][k]);
              a[g + r][k] = __dp4a(w[r].y, rd.d[j][k].y, a[g + r][k]);
              a[g + r][k] = __dp4a(w[r].z, rd.d[j][k].z, a[g + r][k]);
              a[g + r][k] = __dp4a(w[r].w, rd.d[j][k].w, a[g + r][k]);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) y[r] = combine3(a[r][0], a[r][1], a[r][2]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int r = 0; r < R; r++) y[r] += __shfl_xor_sync(0xffffffffu, y[r], o);
  }
}

// The state one consumer thread carries through the kernel.
struct Walk {
  uint32_t iter = 0;       // chunks taken from the ring
  unsigned target = 0;     // grid-barrier arrival count to wait for
  bool dead = false;
};

// Phase-prologue loads that do not depend on this step (scales, gains, cached
// keys), run by warps 1-7 while thread 0 waits at the barrier.
__device__ __forceinline__ int pf_index() { return threadIdx.x - 32; }
constexpr int kPf = kConsumers - 32;

// Grid barrier among the consumer warps of every CTA: once this CTA's phase
// outputs are written, thread 0 arrives (release) and spins (acquire,
// bounded) while warps 1-7 run pf(). Returns false once any CTA gave up.
template <typename PF>
__device__ bool grid_sync(const StepParams& p, StepSmem& sm, Walk& w, PF&& pf) {
  consumers_sync();
  w.target += gridDim.x;
  if (threadIdx.x >= 32) pf();
  if (threadIdx.x == 0) {
    red_release_add(p.bar, 1u);
    int ab = 0;
    const long long t0 = clock64();
    for (uint32_t spin = 1;; spin++) {
      if (static_cast<int>(ld_acquire(p.bar) - w.target) >= 0) break;
      if ((spin & 15) == 0) {
        if ((ab = ld_volatile_i(p.abort)) != 0) break;
        if (clock64() - t0 > kWaitCycles) {
          atomicOr(p.err, kErrBarrier);
          atomicExch(p.abort, 1);
          ab = 1;
          break;
        }
      }
    }
    sm.abort = ab;
  }
  consumers_sync();
  return sm.abort == 0;
}

// Walks a K <= 1024 segment: per chunk, waits for it, hands warp w the rows
// (or row pairs, pairs = 2) w, w+8, ... of the chunk as one group of up to
// four rows, fn(chunk_first_row, first, stride, cnt, y[4]) with the sums in
// digit units (row k of the group: first + (k / pairs) * stride + k % pairs),
// then frees the stage.
template <typename F>
__device__ __forceinline__ void walk_rows(const StepParams& p, StepSmem& sm, const unsigned char* ring, const Seg& sg,
                                          const RegDigits& rd, Walk& w, int pairs, F&& fn) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stride = kConsumerWarps * pairs;
  const int first = warp * pairs;
  for (int r = sg.r0; r < sg.r1; r += sg.rpc) {
    const int s = w.iter % kStages;
    mbar_wait(&sm.full[s], (w.iter / kStages) & 1, p.err, w.dead);
    const int n = min(sg.rpc, sg.r1 - r);
    const unsigned char* st = ring + static_cast<size_t>(s) * kStageBytes;
    const int cnt = first < n ? min(4, pairs * ((n - first + stride - 1) / stride)) : 0;
    if (cnt > 0) {
      uint32_t ro[4];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int row = k < cnt ? first + (k / pairs) * stride + (k % pairs) : first;
        ro[k] = static_cast<uint32_t>(row * sg.K);
      }
      float y[4];
      dot_rows<4>(st, ro, cnt, sg.K, rd, y);
      fn(r, first, stride, cnt, y);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
    w.iter++;
  }
}

// The down segment (a few rows of K = intermediate, in at most kStages
// stages) is taken whole: wait for every stage, run its rows as one batch of
// independent dot products with one CTA reduction, free every stage at the
// end. (Taking the gate/up segment whole measured slower than its chunk walk:
// its later stages are still landing when the phase starts.)
__device__ __forceinline__ int seg_stages(const Seg& sg) { return (sg.r1 - sg.r0 + sg.rpc - 1) / sg.rpc; }
__device__ __forceinline__ void seg_wait(const StepParams& p, StepSmem& sm, Walk& w, int nst) {
  for (int k = 0; k < nst; k++) {
    const uint32_t it = w.iter + k;
    mbar_wait(&sm.full[it % kStages], (it / kStages) & 1, p.err, w.dead);
  }
}
// Byte offset in the ring of row i (0-based in the segment) of a segment
// waited for with seg_wait.
__device__ __forceinline__ uint32_t seg_off(const Seg& sg, const Walk& w, int i) {
  const int k = i / sg.rpc;
  return static_cast<uint32_t>(((w.iter + k) % kStages) * kStageBytes + (i - k * sg.rpc) * sg.K);
}

__device__ __forceinline__ void seg_free(StepSmem& sm, Walk& w, int nst) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    for (int k = 0; k < nst; k++) mbar_arrive(&sm.empty[(w.iter + k) % kStages]);
  }
  w.iter += nst;
}

__device__ __forceinline__ void pf_scales(StepSmem& sm, const void* scales, int dt, int r0, int r1) {
  for (int i = pf_index(); i < r1 - r0; i += kPf) sm.rowscale[i] = ld_as_f32(scales, r0 + i, dt);
}
__device__ __forceinline__ void pf_gain(StepSmem& sm, const float* g, int n) {
  for (int i = pf_index(); i < n; i += kPf) sm.gain[i] = __ldg(g + i);
}

// ---- phase B: attention ---------------------------------------------------------
__device__ __forceinline__ void item_range(const StepParams& p, int it, int& h, int& c, int& p0, int& p1) {
  h = it / p.attn_nchunks;
  c = it % p.attn_nchunks;
  p0 = c * p.attn_chunk;
  p1 = min(p.past + 1, p0 + p.attn_chunk);
}
__device__ __forceinline__ int64_t cache_base(const StepParams& p, int layer, int g) {
  return static_cast<int64_t>(layer) * p.s_layer + static_cast<int64_t>(g) * p.s_head;
}
// The cached keys and values [p0, p0 + n) of an item -> sm.kv, 16-byte async
// copies by the threads t, t + nt, ... of the consumers.
__device__ __forceinline__ void load_item_kv(const StepParams& p, StepSmem& sm, int64_t cb, int p0, int n, int t,
                                             int nt) {
  for (int i = t; i < 2 * n * 8; i += nt) {
    const int which = i / (n * 8), rest = i - which * n * 8, q = rest >> 3, part = rest & 7;
    cp_async16(&sm.kv[which][q][8 * part], (which ? p.vc : p.kc) + cb + static_cast<int64_t>(p0 + q) * 64 + 8 * part);
  }
}

// During phase B's barrier: this CTA's first item's cached keys and values
// (positions below past) into shared memory, and the position's cos/sin.
__device__ void attention_prefetch(const StepParams& p, StepSmem& sm, int layer, int cta) {
  if (cta >= p.heads * p.attn_nchunks) return;
  int h, c, p0, p1;
  item_range(p, cta, h, c, p0, p1);
  const int g = h / (p.heads / p.kv_heads);
  load_item_kv(p, sm, cache_base(p, layer, g), p0, max(0, min(p1, p.past) - p0), pf_index(), kPf);
  if (pf_index() < 32) {
    sm.rope_c[pf_index()] = p.rope_cos[static_cast<int64_t>(p.past) * 32 + pf_index()];
    sm.rope_s[pf_index()] = p.rope_sin[static_cast<int64_t>(p.past) * 32 + pf_index()];
  }
}

// One attention item (query head h, keys [p0, p1) of the past+1),
// src/core/attention.js:42-63 split-KV style: the chunk's partial (o
// unnormalised, m, l). first: the item whose keys attention_prefetch loaded.
__device__ void attention_item(const StepParams& p, StepSmem& sm, int layer, int it, bool first) {
  const int tid = threadIdx.x;
  int h, c, p0, p1;
  item_range(p, it, h, c, p0, p1);
  const int H = p.hidden, KV = p.kv_heads * 64, group = p.heads / p.kv_heads, g = h / group;
  const int pos = p.past;
  const int64_t cb = cache_base(p, layer, g);
  if (!first) {   // a further item of this CTA (long contexts): load its keys now
    load_item_kv(p, sm, cb, p0, max(0, min(p1, pos) - p0), tid, kConsumers);
    if (tid < 32) {
      sm.rope_c[tid] = p.rope_cos[static_cast<int64_t>(pos) * 32 + tid];
      sm.rope_s[tid] = p.rope_sin[static_cast<int64_t>(pos) * 32 + tid];
    }
    consumers_sync();
  }
  // q (f16 input, rotated in f64 and kept in f32), the new key (rotated, then
  // f16 as stored) and value (f16), src/cpu/model.js:108-116
  if (tid < 32) {
    const double cs = sm.rope_c[tid], sn = sm.rope_s[tid];
    const float qlo = __half2float(__float2half_rn(__ldcg(p.qkv + h * 64 + tid)));
    const float qhi = __half2float(__float2half_rn(__ldcg(p.qkv + h * 64 + tid + 32)));
    float olo, ohi;
    rope_pair_f64(qlo, qhi, cs, sn, olo, ohi);
    sm.aq[tid] = olo;
    sm.aq[tid + 32] = ohi;
  } else if (tid < 64) {
    const int d = tid - 32;
    const double cs = sm.rope_c[d], sn = sm.rope_s[d];
    const float klo = __half2float(__float2half_rn(__ldcg(p.qkv + H + g * 64 + d)));
    const float khi = __half2float(__float2half_rn(__ldcg(p.qkv + H + g * 64 + d + 32)));
    float olo, ohi;
    rope_pair_f64(klo, khi, cs, sn, olo, ohi);
    const uint16_t b0 = f32_to_f16_bits(olo), b1 = f32_to_f16_bits(ohi);
    sm.k16[d] = b0;
    sm.k16[d + 32] = b1;
    sm.ak[d] = __half2float(__ushort_as_half(b0));
    sm.ak[d + 32] = __half2float(__ushort_as_half(b1));
  } else if (tid < 128) {
    const int d = tid - 64;
    const uint16_t b = f32_to_f16_bits(__ldcg(p.qkv + H + KV + g * 64 + d));
    sm.v16[d] = b;
    sm.av[d] = __half2float(__ushort_as_half(b));
  }
  cp_async_wait_all();
  consumers_sync();
  // the append (one item per KV head: the group's first head, last chunk)
  if (h % group == 0 && p1 == pos + 1 && tid < 64) {
    p.kc[cb + static_cast<int64_t>(pos) * 64 + tid] = sm.k16[tid];
    p.vc[cb + static_cast<int64_t>(pos) * 64 + tid] = sm.v16[tid];
  }
  // scores: two threads per key (32 dims each), f32 dot times 1/sqrt(64)
  const int n = p1 - p0;
  float s = -INFINITY;
  {
    const int q = tid >> 1, half = tid & 1;
    float dot = 0.f;
    if (q < n) {
      if (p0 + q < pos) {
        const uint4* kr = reinterpret_cast<const uint4*>(&sm.kv[0][q][32 * half]);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const uint4 u = kr[j];
          const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[e]));
            dot = fmaf(sm.aq[32 * half + 8 * j + 2 * e], f.x, dot);
            dot = fmaf(sm.aq[32 * half + 8 * j + 2 * e + 1], f.y, dot);
          }
        }
      } else {
#pragma unroll 8
        for (int d = 0; d < 32; d++) dot = fmaf(sm.aq[32 * half + d], sm.ak[32 * half + d], dot);
      }
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    if (q < n) s = dot * 0.125f;
  }
  const float mx = block_max(sm, s, 0);
  float e = 0.f;
  if ((tid >> 1) < n && (tid & 1) == 0) {
    e = __expf(s - mx);
    sm.scores[tid >> 1] = e;
  }
  const float l = block_sum(sm, e, 1);
  // o: thread (subset ps, dims 2dp, 2dp+1) over keys ps, ps+8, ...
  const int dp = tid & 31, ps = tid >> 5;
  float o0 = 0.f, o1 = 0.f;
  for (int q = ps; q < n; q += kConsumerWarps) {
    const float wq = sm.scores[q];
    float2 v;
    if (p0 + q < pos) v = __half22float2(*reinterpret_cast<const __half2*>(&sm.kv[1][q][2 * dp]));
    else v = make_float2(sm.av[2 * dp], sm.av[2 * dp + 1]);
    o0 = fmaf(wq, v.x, o0);
    o1 = fmaf(wq, v.y, o1);
  }
  sm.ao[ps][2 * dp] = o0;
  sm.ao[ps][2 * dp + 1] = o1;
  consumers_sync();
  float* out = p.part + (static_cast<int64_t>(h) * p.attn_nchunks + c) * kPartPitch;
  if (tid < 64) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kConsumerWarps; k++) t += sm.ao[k][tid];
    out[tid] = t;
  } else if (tid == 64) {
    out[64] = mx;
    out[65] = l;
  }
  consumers_sync();
}

// ---- the compute warps ---------------------------------------------------------
__device__ void consumer(const StepParams& p, StepSmem& sm, const unsigned char* ring, int cta, int G) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = p.hidden, I = p.inter;
  const int sdt = p.scale_dtype;
  Walk w;
  w.target = p.bar_base;
  const int own0 = part_begin(cta, G, H), own1 = part_begin(cta + 1, G, H);
  const bool xthread = 4 * tid < H;   // holds x[4 tid .. 4 tid + 3] in the prologues

  // the token: its embedding row starts the residual stream (every CTA
  // widens the whole row itself: hidden bytes from L2)
  float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
  {
    int tok = __ldcg(p.token_in);
    if (tok < 0 || tok >= p.vocab) {
      if (tid == 0) atomicOr(p.err, kErrStepToken);
      tok = 0;
    }
    const float es = ld_as_f32(p.s_emb, tok, sdt);
    if (xthread) {
      const char4 cv = reinterpret_cast<const char4*>(p.emb + static_cast<int64_t>(tok) * H)[tid];
      xv = make_float4(static_cast<float>(cv.x) * es, static_cast<float>(cv.y) * es, static_cast<float>(cv.z) * es,
                       static_cast<float>(cv.w) * es);
      *reinterpret_cast<float4*>(&sm.act[4 * tid]) = xv;
    }
    consumers_sync();
    if (tid < own1 - own0) sm.xown[tid] = sm.act[own0 + tid];
  }

  RegDigits rd;
  for (int layer = 0; layer < p.num_layers; layer++) {
    const StepLayer& L = p.layers[layer];
    // ---- A: rmsnorm -> q/k/v rows
    {
      const Seg sg = plan_seg(p, layer, 0, cta, G);
      auto pf = [&] {
        pf_scales(sm, L.s_qkv, sdt, sg.r0, sg.r1);
        for (int i = pf_index(); i < sg.r1 - sg.r0; i += kPf) sm.rowbias[i] = __ldg(L.b_qkv + sg.r0 + i);
        pf_gain(sm, L.n_in, H);
      };
      if (layer > 0) {
        if (!grid_sync(p, sm, w, pf)) return;
        if (xthread) xv = __ldcg(reinterpret_cast<const float4*>(p.x) + tid);
      } else {
        if (tid >= 32) pf();
        consumers_sync();
      }
      const float sx = norm_digits(sm, H, xv, p.eps, rd);
      walk_rows(p, sm, ring, sg, rd, w, 1, [&](int r, int first, int stride, int cnt, const float (&y)[4]) {
        if (lane < cnt) {
          const float yl = lane == 0 ? y[0] : lane == 1 ? y[1] : lane == 2 ? y[2] : y[3];
          const int i = r + first + lane * stride - sg.r0;
          p.qkv[sg.r0 + i] = fmaf(yl * sx, sm.rowscale[i], sm.rowbias[i]);
        }
      });
    }
    // ---- B: attention items
    {
      if (!grid_sync(p, sm, w, [&] { attention_prefetch(p, sm, layer, cta); })) return;
      const int items = p.heads * p.attn_nchunks;
      for (int it = cta; it < items; it += G) attention_item(p, sm, layer, it, it == cta);
    }
    // ---- C: merge -> o_proj rows, residual
    {
      const Seg sg = plan_seg(p, layer, 1, cta, G);
      if (!grid_sync(p, sm, w, [&] { pf_scales(sm, L.s_o, sdt, sg.r0, sg.r1); })) return;
      // thread t: outputs 4t..4t+3 (of head 4t/64), one pass over the chunks
      // in order, rescaled by the running maximum
      float4 ov = make_float4(0.f, 0.f, 0.f, 0.f);
      float omax = 0.f;
      if (xthread) {
        const int h = (4 * tid) >> 6, d = (4 * tid) & 63;
        const int nch = p.attn_nchunks;
        const float* pr = p.part + static_cast<int64_t>(h) * nch * kPartPitch;
        float m = -INFINITY, lsum = 0.f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < nch; c++) {
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(pr + c * kPartPitch + 64));
          const float4 oc = __ldcg(reinterpret_cast<const float4*>(pr + c * kPartPitch + d));
          const float mn = fmaxf(m, ml.x);
          const float fo = __expf(m - mn), fc = __expf(ml.x - mn);
          lsum = lsum * fo + ml.y * fc;
          o.x = o.x * fo + oc.x * fc;
          o.y = o.y * fo + oc.y * fc;
          o.z = o.z * fo + oc.z * fc;
          o.w = o.w * fo + oc.w * fc;
          m = mn;
        }
        ov = make_float4(o.x / lsum, o.y / lsum, o.z / lsum, o.w / lsum);
        omax = max4(ov);
      }
      omax = block_max(sm, omax, 0);
      const float sx = hidden_digits(sm, H, ov, omax, rd);
      walk_rows(p, sm, ring, sg, rd, w, 1, [&](int r, int first, int stride, int cnt, const float (&y)[4]) {
        if (lane < cnt) {
          const float yl = lane == 0 ? y[0] : lane == 1 ? y[1] : lane == 2 ? y[2] : y[3];
          const int row = r + first + lane * stride;
          const float xn = sm.xown[row - own0] + yl * sx * sm.rowscale[row - sg.r0];
          sm.xown[row - own0] = xn;
          p.x[row] = xn;
        }
      });
    }
    // ---- D: rmsnorm -> gate/up row pairs -> silu(g) * u
    {
      const Seg sg = plan_seg(p, layer, 2, cta, G);
      if (!grid_sync(p, sm, w, [&] {
            pf_scales(sm, L.s_gu, sdt, sg.r0, sg.r1);
            pf_gain(sm, L.n_post, H);
          })) {
        return;
      }
      if (xthread) xv = __ldcg(reinterpret_cast<const float4*>(p.x) + tid);
      const float sx = norm_digits(sm, H, xv, p.eps, rd);
      // rows come as (gate, up) pairs: lanes 0 and 1 keep pairs 0 and 1 of
      // the chunk (in shared memory); silu(g) * u of every pair once the
      // segment is done, off the chunks' path
      walk_rows(p, sm, ring, sg, rd, w, 2, [&](int r, int first, int stride, int cnt, const float (&y)[4]) {
        if (2 * lane < cnt) {
          const int row = r + first + lane * stride - sg.r0;   // even: the gate row
          sm.act[row] = (lane == 0 ? y[0] : y[2]) * sx * sm.rowscale[row];
          sm.act[row + 1] = (lane == 0 ? y[1] : y[3]) * sx * sm.rowscale[row + 1];
        }
      });
      consumers_sync();
      for (int j = tid; 2 * j < sg.r1 - sg.r0; j += kConsumers) {
        // silu in f32 here (the per-layer kernel keeps the reference's f64)
        const float gv = sm.act[2 * j], uv = sm.act[2 * j + 1];
        p.h[(sg.r0 >> 1) + j] = __fdividef(gv, 1.f + __expf(-gv)) * uv;
      }
    }
    // ---- E: down rows (K = intermediate), residual
    {
      const Seg sg = plan_seg(p, layer, 3, cta, G);
      if (!grid_sync(p, sm, w, [&] { pf_scales(sm, L.s_down, sdt, sg.r0, sg.r1); })) return;
      // h (f32) -> digits in shared memory; a thread takes float4 units t, t+256, ...
      constexpr int kUnitsPerThread = kMaxInter / 4 / kConsumers;
      const int units = I / 4;
      float4 hv[kUnitsPerThread];
      float hmax = 0.f;
#pragma unroll
      for (int k = 0; k < kUnitsPerThread; k++) {
        const int u = tid + k * kConsumers;
        hv[k] = u < units ? __ldcg(reinterpret_cast<const float4*>(p.h) + u) : make_float4(0.f, 0.f, 0.f, 0.f);
        hmax = fmaxf(hmax, max4(hv[k]));
      }
      hmax = block_max(sm, hmax, 1);
      const float inv = hmax > 0.f ? 127.f / hmax : 0.f;
#pragma unroll
      for (int k = 0; k < kUnitsPerThread; k++) {
        const int u = tid + k * kConsumers;
        if (u < units) store_digits4(&sm.dig[0][0], kMaxInter / 4, u, hv[k], inv);
      }
      consumers_sync();
      const float sx = hmax / 127.f;
      // the whole segment at once, eight rows per pass: thread t takes the
      // 16-byte units t, t+256, ... of every row of the pass
      const int urow = I / 16;
      const int nst = seg_stages(sg);
      const int nrow = sg.r1 - sg.r0;
      seg_wait(p, sm, w, nst);
      for (int r0 = 0; r0 < nrow; r0 += kDownBatch) {
        const int nb = min(kDownBatch, nrow - r0);
        uint32_t ro[kDownBatch];
#pragma unroll
        for (int k = 0; k < kDownBatch; k++) ro[k] = seg_off(sg, w, r0 + (k < nb ? k : 0));
        int a[kDownBatch][3] = {};
        for (int u = tid; u < urow; u += kConsumers) {
          const int4 d0 = *reinterpret_cast<const int4*>(&sm.dig[0][4 * u]);
          const int4 d1 = *reinterpret_cast<const int4*>(&sm.dig[1][4 * u]);
          const int4 d2 = *reinterpret_cast<const int4*>(&sm.dig[2][4 * u]);
#pragma unroll
          for (int g = 0; g < kDownBatch; g += 4) {   // four weight loads in flight at a time
            int4 wv[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
              if (g + k < nb) wv[k] = *reinterpret_cast<const int4*>(ring + ro[g + k] + 16 * u);
            }
#pragma unroll
            for (int k = 0; k < 4; k++) {
              if (g + k < nb) {
                int* ak = a[g + k];
                ak[0] = __dp4a(wv[k].w, d0.w, __dp4a(wv[k].z, d0.z, __dp4a(wv[k].y, d0.y, __dp4a(wv[k].x, d0.x, ak[0]))));
                ak[1] = __dp4a(wv[k].w, d1.w, __dp4a(wv[k].z, d1.z, __dp4a(wv[k].y, d1.y, __dp4a(wv[k].x, d1.x, ak[1]))));
                ak[2] = __dp4a(wv[k].w, d2.w, __dp4a(wv[k].z, d2.z, __dp4a(wv[k].y, d2.y, __dp4a(wv[k].x, d2.x, ak[2]))));
              }
            }
          }
        }
        float y[kDownBatch];
#pragma unroll
        for (int k = 0; k < kDownBatch; k++) y[k] = combine3(a[k][0], a[k][1], a[k][2]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
          for (int k = 0; k < kDownBatch; k++) y[k] += __shfl_xor_sync(0xffffffffu, y[k], o);
        }
        if (lane == 0) {
#pragma unroll
          for (int k = 0; k < kDownBatch; k++) sm.down_part[warp][k] = y[k];
        }
        consumers_sync();
        if (tid < nb) {
          float t = 0.f;
#pragma unroll
          for (int k = 0; k < kConsumerWarps; k++) t += sm.down_part[k][tid];
          const int row = sg.r0 + r0 + tid;
          const float xn = sm.xown[row - own0] + t * sx * sm.rowscale[row - sg.r0];
          sm.xown[row - own0] = xn;
          p.x[row] = xn;
        }
        consumers_sync();
      }
      seg_free(sm, w, nst);
    }
  }
  // ---- F: final rmsnorm -> output projection rows -> greedy pick
  {
    const Seg sg = plan_seg(p, p.num_layers, 0, cta, G);
    if (!grid_sync(p, sm, w, [&] {
          pf_scales(sm, p.s_emb, sdt, sg.r0, sg.r1);
          pf_gain(sm, p.n_final, H);
        })) {
      return;
    }
    if (xthread) xv = __ldcg(reinterpret_cast<const float4*>(p.x) + tid);
    const float sx = norm_digits(sm, H, xv, p.eps, rd);
    float bv = -INFINITY;
    int bi = INT_MAX;
    walk_rows(p, sm, ring, sg, rd, w, 1, [&](int r, int first, int stride, int cnt, const float (&y)[4]) {
      if (lane < cnt) {
        const float yl = lane == 0 ? y[0] : lane == 1 ? y[1] : lane == 2 ? y[2] : y[3];
        const int row = r + first + lane * stride;
        const float v = yl * sx * sm.rowscale[row - sg.r0];
        p.logits[row] = v;
        if (v > bv) {   // a lane's rows ascend: strict > keeps the first
          bv = v;
          bi = row;
        }
      }
    });
    // the warp's first maximum, then the CTA's
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      sm.best_v[warp] = bv;
      sm.best_i[warp] = bi;
    }
    consumers_sync();
    if (tid == 0) {
      unsigned long long key = 0ull;
      for (int k = 0; k < kConsumerWarps; k++) {
        if (sm.best_i[k] != INT_MAX) {
          const unsigned long long kk = pick_key(sm.best_v[k], sm.best_i[k]);
          key = kk > key ? kk : key;
        }
      }
      if (key) atomicMax(p.key, key);
      __threadfence();
      // the last CTA to arrive turns the word into the token
      const unsigned final_target = w.target + gridDim.x;
      const unsigned old = atomicAdd(p.bar, 1u);
      if (old == final_target - 1u) {
        __threadfence();
        const unsigned long long k = atomicMax(p.key, 0ull);
        // no number among the logits: the reference's pick stays at index 0
        const int idx = k ? static_cast<int>(0xffffffffu - static_cast<uint32_t>(k)) : 0;
        *p.token_out = idx;
        if (p.best_out) *p.best_out = k ? key_value(k) : __ldcg(p.logits);
        if (p.len) *p.len = p.past + 1;
      }
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) k_decode_step(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StepSmem& sm = *reinterpret_cast<StepSmem*>(smem_raw);
  unsigned char* ring = smem_raw + ((sizeof(StepSmem) + 127) / 128) * 128;
  const int cta = blockIdx.x, G = gridDim.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x >= kConsumers) {
    producer(p, sm, ring, cta, G);
  } else {
    consumer(p, sm, ring, cta, G);
  }
}

size_t decode_step_smem_bytes() {
  return ((sizeof(StepSmem) + 127) / 128) * 128 + static_cast<size_t>(kStages) * kStageBytes;
}

int decode_step_barriers(int num_layers) { return 5 * num_layers; }

int decode_step_attn_chunk() { return kAttnChunk; }

bool decode_step_supported(int hidden, int inter, int q_rows, int vocab, int ctas) {
  if (ctas < 1) return false;
  auto per = [ctas](int rows) { return (rows + ctas - 1) / ctas; };
  // the down segment is taken whole: its stages must fit the ring
  const int rpc_down = min(kStageBytes / max(inter, 1), 4);
  if (rpc_down < 1 || (per(hidden) + rpc_down - 1) / rpc_down > kStages) return false;
  return hidden % 64 == 0 && hidden <= kMaxHidden && inter % 16 == 0 && inter <= kMaxInter &&
         per(hidden) <= kMaxOwnRows && per(q_rows) <= kMaxRows && 2 * per(inter) <= kMaxRows &&
         per(vocab) <= kMaxOutRows && inter <= kStageBytes && decode_step_smem_bytes() <= 227 * 1024;
}

cudaError_t launch_decode_step(const StepParams& p, int ctas, cudaStream_t st) {
  const size_t smem = decode_step_smem_bytes();
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[64] = {};
  if (dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_decode_step, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_decode_step, p);
}

int decode_step_max_ctas() {
  int dev = 0, sms = 0, per = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = decode_step_smem_bytes();
  if (smem > 227 * 1024) return 0;
  cudaFuncSetAttribute(k_decode_step, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_decode_step, kThreads, smem) != cudaSuccess) return 0;
  return sms * (per > 0 ? 1 : 0);
}

}  // namespace b2a
