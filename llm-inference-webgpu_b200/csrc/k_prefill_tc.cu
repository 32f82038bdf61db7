// Causal prefill attention on the 5th-generation tensor cores (tcgen05, TMEM,
// TMA), head_dim 64, for f16 or bf16 KV caches.
//
// One CTA computes one tile of 128 query rows of one query head against every
// KV tile its rows can see. Six warps:
//   warp 0      producer: 128-position K and V tiles of the (already rotated
//               and appended) cache into a 3-stage shared-memory ring, by 2D
//               TMA with the 128-byte swizzle (two 64-row boxes per tile).
//   warp 1      allocates 512 TMEM columns and issues every MMA from one lane:
//                 S_j = Q . K_j^T      M=128 N=128 K=64   (SS, f32 accum in TMEM)
//                 O  += P_j . V_j      M=128 N=64  K=128  (A = P from TMEM)
//               S is double-buffered in TMEM, so S_{j+1} runs while the
//               softmax of tile j does.
//   warps 2-5   softmax: TMEM lane = query row, so thread r owns row r and
//               every row statistic stays in registers. The running max is
//               raised lazily (only when a tile's max exceeds it by more than
//               2^8), so O in TMEM is rescaled rarely. P is written back into
//               the S buffer's columns (it aliases the consumed S).
// RoPE(q) is applied while the softmax warps stage the Q tile into swizzled
// shared memory (f64 rotation from the host table, as every kernel here does).
// With a bf16 cache the rotated query and P are each split into a bf16 high
// part and a bf16 residual (two MMAs each): a single bf16 rounding of either
// puts the output about 5e-3 off the f32 reference, the split keeps it ~1e-6.
// With an f16 cache one f16 rounding of each is already within ~7e-4.
#include <cuda.h>
#include <math_constants.h>

#include <type_traits>

#include "b2a_internal.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {

constexpr int kD = 64;
constexpr int kBM = 128;                       // query rows per CTA
constexpr int kBN = 128;                       // KV positions per tile
constexpr int kStages = 3;
constexpr int kThreads = 192;
constexpr int kQBytes = kBM * kD * 2;          // 16 KiB
constexpr int kKVBytes = kBN * kD * 2;         // 16 KiB per K or V tile
constexpr int kStageBytes = 2 * kKVBytes;
constexpr int kTmemCols = 512;                 // S0 [0,128) S1 [128,256) O [256,320)
constexpr int kOCol = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;      // log2 units
constexpr long long kWaitCycles = 1000000000LL;
constexpr int kErrTimeout = 2;

// smem layout (offsets from a 1024-aligned base)
constexpr int kOffQHi = 0;
constexpr int kOffQLo = kOffQHi + kQBytes;
constexpr int kOffRing = kOffQLo + kQBytes;
constexpr int kOffBars = kOffRing + kStages * kStageBytes;
constexpr int kNumBars = 2 * kStages + 2 /*s_full*/ + 2 /*p_full*/ + 1 /*o_done*/ + 1 /*q_ready*/;
constexpr int kSmemTotal = kOffBars + kNumBars * 8 + 16 + 1024;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait (~0.5 s): on timeout, record it in the error word, mark this
// thread dead and carry on; a dead thread skips every later wait, so a broken
// pipeline ends the CTA quickly instead of hanging.
__device__ __forceinline__ void mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err, bool& dead) {
  if (dead || mbar_try_wait(bar, parity)) return;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      if (err) atomicOr(err, kErrTimeout);
      dead = true;
      return;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---- tcgen05 wrappers -------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFF) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: f32 accumulate, A/B type (0 f16, 1 bf16),
// B major-ness (0 K-major, 1 MN-major), shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int ab_type, int b_mn_major, int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(ab_type) << 7) | (static_cast<uint32_t>(ab_type) << 10) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define B2A_REG8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                    "=r"(r[i + 6]), "=r"(r[i + 7])
#define B2A_IREG8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                     "r"(r[i + 6]), "r"(r[i + 7])

// 32 consecutive TMEM columns of this thread's lane -> r[0..31]
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : B2A_REG8(0), B2A_REG8(8), B2A_REG8(16), B2A_REG8(24)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      B2A_IREG8(0), B2A_IREG8(8), B2A_IREG8(16), B2A_IREG8(24)
      : "memory");
}
// 2^x on the multi-function unit (flushes subnormal results to zero, which for
// softmax weights below 2^-126 is harmless).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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

// Splits two floats into bf16 (high, truncated) and bf16 residual parts:
// x = hi + lo exactly up to the residual's own rounding (~2^-17 relative).
__device__ __forceinline__ void split2_bf16(float a, float b, uint32_t& hi, uint32_t& lo) {
  const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
  hi = __byte_perm(ua, ub, 0x7632);   // upper halves: a -> low 16 bits, b -> high 16 bits
  const float ra = a - __uint_as_float(ua & 0xffff0000u);
  const float rb = b - __uint_as_float(ub & 0xffff0000u);
  lo = pack2<__nv_bfloat16>(ra, rb);
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    k_prefill_tc(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                 AttnParams p) {
  constexpr bool kSplit = std::is_same<T, __nv_bfloat16>::value;
  constexpr int kAB = kSplit ? 1 : 0;
  constexpr uint32_t kIdescS = idesc_f16(kAB, 0, kBM, kBN);
  constexpr uint32_t kIdescPV = idesc_f16(kAB, 1, kBM, kD);

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + kStages;
  uint64_t* s_full = bars + 2 * kStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* q_ready = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  bool dead = false;   // set once a bounded wait of this thread gave up
  const int n_qtiles = (p.tokens + kBM - 1) / kBM;
  const int qt = n_qtiles - 1 - static_cast<int>(blockIdx.x);   // heaviest (latest) tiles first
  const int h = blockIdx.y;
  const int g = h / p.group;
  const int bc = p.seq_begin;
  const int past = p.len[bc];
  const int q0 = qt * kBM;
  const int q_last = min(q0 + kBM, p.tokens) - 1;               // last valid query of this tile
  const int n_keys = past + q_last + 1;
  const int n_kv = (n_keys + kBN - 1) / kBN;
  const int64_t cache_base = bc * p.s_seq + static_cast<int64_t>(p.layer_begin) * p.s_layer + g * p.s_head;
  const int row_base = static_cast<int>(cache_base / kD);

  if (tid == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
    }
    mbar_init(o_done, 1);
    mbar_init(q_ready, 128);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int j = 0; j < n_kv; j++) {
        const int s = j % kStages;
        if (j >= kStages) mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, p.err, dead);
        mbar_arrive_expect_tx(&kv_full[s], kStageBytes);
        const uint32_t st = smem_u32(smem + kOffRing + s * kStageBytes);
        const int y = row_base + j * kBN;
        tma_load_2d(st, &tmap_k, &kv_full[s], 0, y);
        tma_load_2d(st + kKVBytes / 2, &tmap_k, &kv_full[s], 0, y + 64);
        tma_load_2d(st + kKVBytes, &tmap_v, &kv_full[s], 0, y);
        tma_load_2d(st + kKVBytes + kKVBytes / 2, &tmap_v, &kv_full[s], 0, y + 64);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t q_hi = smem_u32(smem + kOffQHi), q_lo = smem_u32(smem + kOffQLo);
      mbar_wait(q_ready, 0, p.err, dead);
      tc_fence_after();
      auto issue_s = [&](int j) {
        const int s = j % kStages;
        mbar_wait(&kv_full[s], (j / kStages) & 1, p.err, dead);
        tc_fence_after();
        const uint32_t kt = smem_u32(smem + kOffRing + s * kStageBytes);
        const uint32_t d = tmem + (j & 1) * kBN;
#pragma unroll
        for (int kk = 0; kk < kD / 16; kk++) {
          mma_ss(d, sdesc_sw128(q_hi + kk * 32), sdesc_sw128(kt + kk * 32), kIdescS, kk > 0);
        }
        if (kSplit) {
#pragma unroll
          for (int kk = 0; kk < kD / 16; kk++) {
            mma_ss(d, sdesc_sw128(q_lo + kk * 32), sdesc_sw128(kt + kk * 32), kIdescS, 1);
          }
        }
        mma_commit(&s_full[j & 1]);
      };
      issue_s(0);
      for (int j = 0; j < n_kv; j++) {
        if (j + 1 < n_kv) {
          // S_{j+1} reuses the buffer of S_{j-1}/P_{j-1}: wait for PV_{j-1}
          if (j >= 1) mbar_wait(o_done, (j - 1) & 1, p.err, dead);
          issue_s(j + 1);
        }
        mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.err, dead);
        tc_fence_after();
        const int s = j % kStages;
        const uint32_t vt = smem_u32(smem + kOffRing + s * kStageBytes + kKVBytes);
        const uint32_t pcol = tmem + (j & 1) * kBN;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; kk++) {
          mma_ts(tmem + kOCol, pcol + kk * 8, sdesc_sw128(vt + kk * 2048), kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        if (kSplit) {
#pragma unroll
          for (int kk = 0; kk < kBN / 16; kk++) {
            mma_ts(tmem + kOCol, pcol + 64 + kk * 8, sdesc_sw128(vt + kk * 2048), kIdescPV, 1u);
          }
        }
        mma_commit(&kv_empty[s]);
        mma_commit(o_done);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;                  // TMEM lanes this warp may touch
    const int r = quarter * 32 + lane;             // query row within the tile
    const int t = q0 + r;                          // token index within this call
    const int a = past + t;                        // absolute position
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    // stage RoPE(q) into Q_hi (and Q_lo), 128-byte-swizzled K-major rows
    {
      const double* cosr = p.rope_cos + static_cast<int64_t>(a) * (kD / 2);
      const double* sinr = p.rope_sin + static_cast<int64_t>(a) * (kD / 2);
      const int64_t qrow = (static_cast<int64_t>(t) * p.heads + h) * kD;
      unsigned char* rh = smem + kOffQHi + r * 128;
      unsigned char* rl = smem + kOffQLo + r * 128;
      const bool vec = p.in_dtype != DT_F32 && (reinterpret_cast<uintptr_t>(p.q) & 15) == 0;
#pragma unroll
      for (int c = 0; c < 4; c++) {         // chunk c holds dims 8c..8c+7; chunk c+4 dims 32+8c..
        float lo[8], hi[8];
        float x0[8], x1[8];
        double cs[8], sn[8];
        if (t < p.tokens) {
          if (vec) {   // one 16-byte load per 8 elements
            const uint4 u0 = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.q) + qrow + 8 * c);
            const uint4 u1 = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.q) + qrow + 8 * c + 32);
            const uint16_t* h0 = reinterpret_cast<const uint16_t*>(&u0);
            const uint16_t* h1 = reinterpret_cast<const uint16_t*>(&u1);
#pragma unroll
            for (int e = 0; e < 8; e++) {
              x0[e] = p.in_dtype == DT_F16 ? __half2float(__ushort_as_half(h0[e]))
                                           : __bfloat162float(__ushort_as_bfloat16(h0[e]));
              x1[e] = p.in_dtype == DT_F16 ? __half2float(__ushort_as_half(h1[e]))
                                           : __bfloat162float(__ushort_as_bfloat16(h1[e]));
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; e++) {
              x0[e] = ld_as_f32(p.q, qrow + 8 * c + e, p.in_dtype);
              x1[e] = ld_as_f32(p.q, qrow + 8 * c + e + 32, p.in_dtype);
            }
          }
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const double2 c2 = *reinterpret_cast<const double2*>(cosr + 8 * c + e);
            const double2 s2 = *reinterpret_cast<const double2*>(sinr + 8 * c + e);
            cs[e] = c2.x;
            cs[e + 1] = c2.y;
            sn[e] = s2.x;
            sn[e + 1] = s2.y;
          }
        }
#pragma unroll
        for (int e = 0; e < 8; e++) {
          lo[e] = hi[e] = 0.f;
          if (t < p.tokens) rope_pair_f64(x0[e], x1[e], cs[e], sn[e], lo[e], hi[e]);
        }
        uint4 vh0, vh1, vl0, vl1;
        uint32_t* ph0 = reinterpret_cast<uint32_t*>(&vh0);
        uint32_t* ph1 = reinterpret_cast<uint32_t*>(&vh1);
        uint32_t* pl0 = reinterpret_cast<uint32_t*>(&vl0);
        uint32_t* pl1 = reinterpret_cast<uint32_t*>(&vl1);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          if (kSplit) {
            split2_bf16(lo[2 * e], lo[2 * e + 1], ph0[e], pl0[e]);
            split2_bf16(hi[2 * e], hi[2 * e + 1], ph1[e], pl1[e]);
          } else {
            ph0[e] = pack2<T>(lo[2 * e], lo[2 * e + 1]);
            ph1[e] = pack2<T>(hi[2 * e], hi[2 * e + 1]);
          }
        }
        *reinterpret_cast<uint4*>(rh + ((c ^ (r & 7)) << 4)) = vh0;
        *reinterpret_cast<uint4*>(rh + (((c + 4) ^ (r & 7)) << 4)) = vh1;
        if (kSplit) {
          *reinterpret_cast<uint4*>(rl + ((c ^ (r & 7)) << 4)) = vl0;
          *reinterpret_cast<uint4*>(rl + (((c + 4) ^ (r & 7)) << 4)) = vl1;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(q_ready);
    }

    const float sc = rsqrtf(static_cast<float>(kD)) * kLog2e;
    float m_used = -CUDART_INF_F;   // log2 units
    float l = 0.f;
    for (int j = 0; j < n_kv; j++) {
      mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.err, dead);
      tc_fence_after();
      const uint32_t scol = tmem + lane_addr + (j & 1) * kBN;
      uint32_t sr[4][32];
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++) tmem_ld32(scol + q4 * 32, sr[q4]);
      tmem_wait_ld();
      // causal / end-of-sequence mask: key k visible iff k <= a
      const int kbase = j * kBN;
      const bool need_mask = kbase + kBN - 1 > past + q0;
      if (need_mask) {
        const int lim = a - kbase;   // columns > lim are masked
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++)
#pragma unroll
          for (int e = 0; e < 32; e++)
            if (q4 * 32 + e > lim) sr[q4][e] = __float_as_uint(-CUDART_INF_F);
      }
      // row max with 8 independent chains (a single chain is latency-bound)
      float mxs[8];
#pragma unroll
      for (int x = 0; x < 8; x++) mxs[x] = -CUDART_INF_F;
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++)
#pragma unroll
        for (int e = 0; e < 32; e++) mxs[e & 7] = fmaxf(mxs[e & 7], __uint_as_float(sr[q4][e]));
      const float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                             fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
      const float tmx = mx * sc;
      const bool grow = tmx > m_used + kRescaleThreshold;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = fmaxf(m_used, tmx);
        const float alpha = (m_used == -CUDART_INF_F) ? 0.f : ex2_approx(m_used - m_new);
        l *= alpha;
        if (j > 0) {
          // O holds the sum through PV_{j-1}: rescale it in place
          mbar_wait(o_done, (j - 1) & 1, p.err, dead);
          tc_fence_after();
          const uint32_t ocol = tmem + lane_addr + kOCol;
          uint32_t ov[2][32];
          tmem_ld32(ocol, ov[0]);
          tmem_ld32(ocol + 32, ov[1]);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 2; x++)
#pragma unroll
            for (int e = 0; e < 32; e++) ov[x][e] = __float_as_uint(__uint_as_float(ov[x][e]) * alpha);
          tmem_st32(ocol, ov[0]);
          tmem_st32(ocol + 32, ov[1]);
          tmem_wait_st();
        }
        m_used = m_new;
      }
      const float nb = -m_used;
      // P = 2^(s*sc - m), written over this S buffer's columns
      float sums[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t ph[2][32];   // 64 columns of packed pairs; lo parts reuse sr storage
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(sr[q4][e]), sc, nb));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sr[q4][e + 1]), sc, nb));
          sums[(e >> 1) & 3] += p0 + p1;
          const int col = q4 * 16 + e / 2;   // packed column 0..63
          if (kSplit) {
            uint32_t hi, lo;
            split2_bf16(p0, p1, hi, lo);
            ph[col >> 5][col & 31] = hi;
            sr[col >> 5][col & 31] = lo;   // columns 0..31 of sr[0], sr[1] are dead by now
          } else {
            ph[col >> 5][col & 31] = pack2<T>(p0, p1);
          }
        }
      }
      l += (sums[0] + sums[1]) + (sums[2] + sums[3]);
      // the last KV tile: zero V rows past the sequence end (0 * stale bits must not give NaN)
      if (j == n_kv - 1) {
        const int valid_rows = (past + p.tokens) - kbase;
        if (r >= valid_rows && r < kBN) {
          uint4* vrow = reinterpret_cast<uint4*>(smem + kOffRing + (j % kStages) * kStageBytes + kKVBytes + r * 128);
#pragma unroll
          for (int x = 0; x < 8; x++) vrow[x] = make_uint4(0, 0, 0, 0);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      tmem_st32(scol, ph[0]);
      tmem_st32(scol + 32, ph[1]);
      if (kSplit) {
        tmem_st32(scol + 64, sr[0]);
        tmem_st32(scol + 96, sr[1]);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    // epilogue: O / l -> out rows
    mbar_wait(o_done, (n_kv - 1) & 1, p.err, dead);
    tc_fence_after();
    uint32_t ov[2][32];
    const uint32_t ocol = tmem + lane_addr + kOCol;
    tmem_ld32(ocol, ov[0]);
    tmem_ld32(ocol + 32, ov[1]);
    tmem_wait_ld();
    if (t < p.tokens) {
      const float inv = 1.f / l;
      const int64_t orow = (static_cast<int64_t>(t) * p.heads + h) * kD;
      void* out = p.partial;   // the output pointer travels in the partial slot for this kernel
      const int odt = p.nchunks;   // and its dtype in nchunks
      if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) {
#pragma unroll
        for (int x = 0; x < 2; x++)
#pragma unroll
          for (int e = 0; e < 32; e++) st_from_f32(out, orow + x * 32 + e, odt, __uint_as_float(ov[x][e]) * inv);
      } else if (odt == DT_F32) {
        float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(out) + orow);
#pragma unroll
        for (int x = 0; x < 16; x++) {
          const int e = 4 * x;
          o4[x] = make_float4(__uint_as_float(ov[e >> 5][e & 31]) * inv, __uint_as_float(ov[e >> 5][(e & 31) + 1]) * inv,
                              __uint_as_float(ov[e >> 5][(e & 31) + 2]) * inv,
                              __uint_as_float(ov[e >> 5][(e & 31) + 3]) * inv);
        }
      } else {
        uint4* o4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + orow);
#pragma unroll
        for (int x = 0; x < 8; x++) {
          uint32_t w[4];
#pragma unroll
          for (int y = 0; y < 4; y++) {
            const int e = 8 * x + 2 * y;
            const float f0 = __uint_as_float(ov[e >> 5][e & 31]) * inv;
            const float f1 = __uint_as_float(ov[e >> 5][(e & 31) + 1]) * inv;
            const uint32_t b0 = odt == DT_F16 ? f32_to_f16_bits(f0) : f32_to_bf16_bits(f0);
            const uint32_t b1 = odt == DT_F16 ? f32_to_f16_bits(f1) : f32_to_bf16_bits(f1);
            w[y] = b0 | (b1 << 16);
          }
          o4[x] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

bool prefill_tc_supported(const AttnParams& p) {
  return p.tmap_k != nullptr && p.tmap_v != nullptr && p.batch == 1 && p.num_layers == 1 && p.head_dim == kD &&
         p.k_new == nullptr && (p.cache_dtype == DT_F16 || p.cache_dtype == DT_BF16);
}

cudaError_t launch_prefill_tc(const AttnParams& p, void* out, int out_dtype, cudaStream_t st) {
  if (!prefill_tc_supported(p)) return cudaErrorInvalidValue;
  if (p.tokens <= 0) return cudaSuccess;
  AttnParams q = p;
  q.partial = static_cast<float*>(out);
  q.nchunks = out_dtype;
  const dim3 grid((p.tokens + kBM - 1) / kBM, p.heads);
  const CUtensorMap* mk = static_cast<const CUtensorMap*>(p.tmap_k);
  const CUtensorMap* mv = static_cast<const CUtensorMap*>(p.tmap_v);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_f16[64] = {}, attr_bf16[64] = {};
  if (p.cache_dtype == DT_F16) {
    if (dev < 64 && !attr_f16[dev]) {
      cudaFuncSetAttribute(k_prefill_tc<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal);
      attr_f16[dev] = true;
    }
    k_prefill_tc<__half><<<grid, kThreads, kSmemTotal, st>>>(*mk, *mv, q);
  } else {
    if (dev < 64 && !attr_bf16[dev]) {
      cudaFuncSetAttribute(k_prefill_tc<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal);
      attr_bf16[dev] = true;
    }
    k_prefill_tc<__nv_bfloat16><<<grid, kThreads, kSmemTotal, st>>>(*mk, *mv, q);
  }
  return cudaGetLastError();
}

}  // namespace b2a
