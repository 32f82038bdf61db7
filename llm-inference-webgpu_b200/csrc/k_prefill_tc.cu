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
// RoPE(q): with an f16 cache the append kernel before this one writes the
// rotated queries as f16 rows and the producer loads the Q tile by TMA (one
// box, 128-byte swizzle); with a bf16 cache the softmax warps rotate and stage
// the Q tile (and its residual) into swizzled shared memory themselves. Both
// rotate in f32 and round the operand to 16 bits next.
// The kernel is launched as a programmatic dependent of the RoPE(K) + append
// kernel before it: barriers, TMEM allocation (and, with a bf16 cache, the Q
// staging) overlap that kernel, and the producer waits on the grid dependency
// before its first TMA load (the rotated Q tile with an f16 cache, then the
// cache).
// With a bf16 cache the rotated query and P are each split into a bf16 high
// part and a bf16 residual (two MMAs each): a single bf16 rounding of either
// puts the output about 5e-3 off the f32 reference, the split keeps it ~1e-6.
// With an f16 cache one f16 rounding of each is already within ~7e-4.
#include <cuda.h>
#include <math_constants.h>

#include <type_traits>

#include "b2a_internal.cuh"
#include "k_sm100.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {

using namespace sm100;

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

// smem layout (offsets from a 1024-aligned base)
constexpr int kOffQHi = 0;
constexpr int kOffQLo = kOffQHi + kQBytes;
constexpr int kOffRing = kOffQLo + kQBytes;
constexpr int kOffBars = kOffRing + kStages * kStageBytes;
constexpr int kNumBars = 2 * kStages + 2 /*s_full*/ + 2 /*p_full*/ + 1 /*o_done*/ + 1 /*q_ready*/ + 1 /*o_final*/;
constexpr int kSmemTotal = kOffBars + kNumBars * 8 + 16 + 1024;

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
                 const __grid_constant__ CUtensorMap tmap_q, AttnParams p) {
  constexpr bool kSplit = std::is_same<T, __nv_bfloat16>::value;
  // the Q tile by TMA from the rotated rows (f16 cache, rows written)
  const bool q_tma = !kSplit && p.q_rot != nullptr;
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
  // completes once, when the last PV has: the epilogue waits on it, not on
  // o_done, because a softmax warp can reach the epilogue while o_done is still
  // two phases short (it never waits for the previous tile's PV), where a
  // parity wait on o_done cannot tell "two short" from "done"
  uint64_t* o_final = q_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  bool dead = false;   // set once a bounded wait of this thread gave up
  const int n_qtiles = (p.tokens + kBM - 1) / kBM;
  // blocks are dispatched in linear order (x fastest): with the query tile in z,
  // every head and sequence of the heaviest (latest) tile starts before any
  // lighter tile, so a second wave never holds a heavy tile
  const int qt = n_qtiles - 1 - static_cast<int>(blockIdx.z);
  const int h = blockIdx.x;
  const int g = h / p.group;
  const int sb = blockIdx.y;                                    // sequence of a batched call
  const int bc = p.seq_begin + sb;
  const int past = p.len[bc];
  const int q0 = qt * kBM;
  const int q_last = min(q0 + kBM, p.tokens) - 1;               // last valid query of this tile
  const int n_keys = past + q_last + 1;
  const int n_kv = (n_keys + kBN - 1) / kBN;

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
    mbar_init(q_ready, q_tma ? 1 : 128);
    mbar_init(o_final, 1);
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
      // the cache rows come from the preceding append kernel
      asm volatile("griddepcontrol.wait;" ::: "memory");
      // the append kernel stored the new rows (and the rotated queries) through
      // the generic proxy; the tensor loads below read them through the async proxy
      asm volatile("fence.proxy.async.global;" ::: "memory");
      if (q_tma) {
        mbar_arrive_expect_tx(q_ready, kQBytes);
        tma_load_2d(smem_u32(smem + kOffQHi), &tmap_q, q_ready, h * kD, sb * p.tokens + q0);
      }
      for (int j = 0; j < n_kv; j++) {
        const int s = j % kStages;
        if (j >= kStages) mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, p.err, dead);
        mbar_arrive_expect_tx(&kv_full[s], kStageBytes);
        const uint32_t st = smem_u32(smem + kOffRing + s * kStageBytes);
        // a 128-position tile starting at a multiple of 128 lies in one page
        const int y = static_cast<int>(kv_elem(p, bc, p.layer_begin, g, j * kBN) / kD);
        tma_load_2d(st, &tmap_k, &kv_full[s], 0, y);
        tma_load_2d(st + kKVBytes / 2, &tmap_k, &kv_full[s], 0, y + 64);
        tma_load_2d(st + kKVBytes, &tmap_v, &kv_full[s], 0, y);
        tma_load_2d(st + kKVBytes + kKVBytes / 2, &tmap_v, &kv_full[s], 0, y + 64);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop and its waits; one elected lane issues and
    // commits (a converged warp issues tcgen05.mma faster than a lone lane).
    {
      const uint32_t q_hi = smem_u32(smem + kOffQHi), q_lo = smem_u32(smem + kOffQLo);
      mbar_wait(q_ready, 0, p.err, dead);
      tc_fence_after();
      auto issue_s = [&](int j) {
        const int s = j % kStages;
        mbar_wait(&kv_full[s], (j / kStages) & 1, p.err, dead);
        tc_fence_after();
        const uint32_t kt = smem_u32(smem + kOffRing + s * kStageBytes);
        const uint32_t d = tmem + (j & 1) * kBN;
        if (elect_one()) {
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
        }
        __syncwarp();
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
        if (elect_one()) {
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
        __syncwarp();
      }
      // tracks every MMA the elected lane issued, the last PV included
      if (elect_one()) mma_commit(o_final);
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;                  // TMEM lanes this warp may touch
    const int r = quarter * 32 + lane;             // query row within the tile
    const int t = q0 + r;                          // token index within this call
    const int a = past + t;                        // absolute position
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    // stage RoPE(q) into Q_hi (and Q_lo), 128-byte-swizzled K-major rows.
    // Every global load of the row (q, cos, sin) is issued before the first
    // use so the thread pays one memory latency, not one per chunk. The
    // rotation runs in f32 from the f32 table: its error (~2^-24) is far below
    // the 16-bit rounding of the MMA operand that follows.
    if (!q_tma) {
      float x[kD], cs[kD / 2], sn[kD / 2];
      if (t < p.tokens) {
        const int64_t qrow = ((static_cast<int64_t>(sb) * p.tokens + t) * p.heads + h) * kD;
        const float4* c4 = reinterpret_cast<const float4*>(p.rope_cos32 + static_cast<int64_t>(a) * (kD / 2));
        const float4* s4 = reinterpret_cast<const float4*>(p.rope_sin32 + static_cast<int64_t>(a) * (kD / 2));
        if (p.in_dtype != DT_F32 && (reinterpret_cast<uintptr_t>(p.q) & 15) == 0) {
          uint4 u[8];   // one 16-byte load per 8 elements
          const uint4* q4 = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.q) + qrow);
#pragma unroll
          for (int i = 0; i < 8; i++) u[i] = q4[i];
#pragma unroll
          for (int i = 0; i < 8; i++) {
            reinterpret_cast<float4*>(cs)[i] = c4[i];
            reinterpret_cast<float4*>(sn)[i] = s4[i];
          }
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const uint16_t* hw = reinterpret_cast<const uint16_t*>(&u[i]);
#pragma unroll
            for (int e = 0; e < 8; e++)
              x[8 * i + e] = p.in_dtype == DT_F16 ? __half2float(__ushort_as_half(hw[e]))
                                                  : __bfloat162float(__ushort_as_bfloat16(hw[e]));
          }
        } else {
#pragma unroll
          for (int e = 0; e < kD; e++) x[e] = ld_as_f32(p.q, qrow + e, p.in_dtype);
#pragma unroll
          for (int i = 0; i < 8; i++) {
            reinterpret_cast<float4*>(cs)[i] = c4[i];
            reinterpret_cast<float4*>(sn)[i] = s4[i];
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < kD; e++) x[e] = 0.f;
#pragma unroll
        for (int e = 0; e < kD / 2; e++) cs[e] = sn[e] = 0.f;
      }
      unsigned char* rh = smem + kOffQHi + r * 128;
      unsigned char* rl = smem + kOffQLo + r * 128;
#pragma unroll
      for (int c = 0; c < 4; c++) {         // chunk c holds dims 8c..8c+7; chunk c+4 dims 32+8c..
        float lo[8], hi[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int d = 8 * c + e;
          lo[e] = fmaf(x[d], cs[d], -(x[d + 32] * sn[d]));
          hi[e] = fmaf(x[d + 32], cs[d], x[d] * sn[d]);
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
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++) tmem_ld_fence(sr[q4]);
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
      // row max: eight independent chains of three-input max
      float mxs[8];
#pragma unroll
      for (int x = 0; x < 8; x++) mxs[x] = -CUDART_INF_F;
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++)
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          mxs[(e >> 1) & 7] = max3f(mxs[(e >> 1) & 7], __uint_as_float(sr[q4][e]), __uint_as_float(sr[q4][e + 1]));
      const float mx = max3f(max3f(mxs[0], mxs[1], mxs[2]), max3f(mxs[3], mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7]));
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
          tmem_ld_fence(ov[0]);
          tmem_ld_fence(ov[1]);
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
      // (the scale-and-shift and the row sums run as packed f32 pairs)
      const uint64_t sc2 = f2_pack(sc, sc), nb2 = f2_pack(nb, nb);
      uint64_t sums[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t ph[2][32];   // 64 columns of packed pairs; lo parts reuse sr storage
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[q4][e]), __uint_as_float(sr[q4][e + 1])), sc2, nb2), x0, x1);
          const float p0 = ex2_approx(x0);
          const float p1 = ex2_approx(x1);
          sums[(e >> 1) & 3] = f2_add(sums[(e >> 1) & 3], f2_pack(p0, p1));
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
      {
        float a0, a1;
        f2_unpack(f2_add(f2_add(sums[0], sums[1]), f2_add(sums[2], sums[3])), a0, a1);
        l += a0 + a1;
      }
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
    mbar_wait(o_final, 0, p.err, dead);
    tc_fence_after();
    uint32_t ov[2][32];
    const uint32_t ocol = tmem + lane_addr + kOCol;
    tmem_ld32(ocol, ov[0]);
    tmem_ld32(ocol + 32, ov[1]);
    tmem_wait_ld();
    tmem_ld_fence(ov[0]);
    tmem_ld_fence(ov[1]);
    if (t < p.tokens) {
      const float inv = 1.f / l;
      const int64_t orow = ((static_cast<int64_t>(sb) * p.tokens + t) * p.heads + h) * kD;
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
  // grid (heads, batch, query tiles): y and z are limited to 65535
  return p.tmap_k != nullptr && p.tmap_v != nullptr && p.batch >= 1 && p.batch <= 65535 &&
         (p.tokens + kBM - 1) / kBM <= 65535 && p.num_layers == 1 && p.head_dim == kD &&
         p.k_new == nullptr && (p.cache_dtype == DT_F16 || p.cache_dtype == DT_BF16);
}

cudaError_t launch_prefill_tc(const AttnParams& p, void* out, int out_dtype, cudaStream_t st) {
  if (!prefill_tc_supported(p)) return cudaErrorInvalidValue;
  if (p.tokens <= 0) return cudaSuccess;
  AttnParams q = p;
  q.partial = static_cast<float*>(out);
  q.nchunks = out_dtype;
  const dim3 grid(p.heads, p.batch, (p.tokens + kBM - 1) / kBM);
  const CUtensorMap* mk = static_cast<const CUtensorMap*>(p.tmap_k);
  const CUtensorMap* mv = static_cast<const CUtensorMap*>(p.tmap_v);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_f16[64] = {}, attr_bf16[64] = {};
  const bool f16 = p.cache_dtype == DT_F16;
  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, AttnParams) =
      f16 ? k_prefill_tc<__half> : k_prefill_tc<__nv_bfloat16>;
  // the rotated-query map travels with the rows it covers; absent (bf16
  // cache, or the rows not written) the kernel stages its own Q tile
  CUtensorMap mq = {};
  if (f16 && p.q_rot != nullptr && p.tmap_q != nullptr) mq = *static_cast<const CUtensorMap*>(p.tmap_q);
  else q.q_rot = nullptr;
  bool* attr = f16 ? attr_f16 : attr_bf16;
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal);
    attr[dev] = true;
  }
  // programmatic dependent launch: may start while the append kernel runs
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemTotal;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, *mk, *mv, mq, q);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace b2a
