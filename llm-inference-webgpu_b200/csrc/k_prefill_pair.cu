// Causal prefill attention for f16 KV caches on the tcgen05 tensor cores,
// head_dim 64: two 128-row query tiles per CTA that share every K/V tile.
//
// The two tiles are the same 128 positions of two query heads of one KV group
// (heads 2k and 2k+1 of the group; an odd group leaves one CTA per tile row
// with a single head), so both see exactly the same keys and one K/V stream
// feeds both. Twelve warps:
//   warp 0      producer: after waiting on the append kernel's grid, the
//               CTA's query tiles (RoPE(q) as f16, written by that kernel)
//               and then K and V tiles (128 positions) of the rotated,
//               appended cache into a 4-stage ring, all by 2D TMA (128-byte
//               swizzle). Rows of a query tile past its sequence's tokens
//               hold the next sequence's queries (or zeros past the last);
//               their outputs are never stored.
//   warp 1      allocates the 512 TMEM columns and issues every MMA:
//                 S_w = Q_w . K_j^T    M=128 N=128 K=64  into S_w
//                 O_w += P_w . V_j     M=128 N=64  K=128 (A = P_w from TMEM)
//               S_w(j+1) is issued as soon as softmax w has read S_w(j) into
//               registers, so it runs under that tile's exponentials. The
//               whole warp runs the loop and waits; one elected lane issues
//               (a converged warp issues tcgen05.mma markedly faster than a
//               lone lane: the S/PV issue no longer trails the softmax).
//   warps 2-3   idle after setup.
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1: TMEM lane =
//               query row, thread r owns row r. Two softmax warps per SM
//               sub-partition share its exponential unit; with no hand-over
//               between them the two tiles settle about a third of a KV step
//               apart (tile 1's first S starts a fixed 800 cycles after tile
//               0's, so they do not start together), and one tile's TMEM
//               traffic, row max and P store run under the other's
//               exponentials.
// TMEM columns: S_0 [0,128) S_1 [128,256) O_0 [256,320) O_1 [320,384)
// P_0 [384,448) P_1 [448,512) (P as packed f16 pairs, separate from S so the
// next S can be written while P is still being produced or consumed).
// The running max is raised lazily (only past 2^8 growth), so O is rescaled
// rarely; bf16 inputs are exact in the f16 cache and one f16 rounding of the
// rotated query and of P keeps the output within ~7e-4 of the f32 reference.
#include <cuda.h>
#include <math_constants.h>

#include "b2a_internal.cuh"
#include "k_sm100.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {

using namespace sm100;

constexpr int kD = 64;
constexpr int kBM = 128;                       // query rows per tile
constexpr int kBN = 128;                       // KV positions per tile
constexpr int kStages = 4;
constexpr int kThreads = 384;
constexpr int kQBytes = kBM * kD * 2;          // 16 KiB per query tile
constexpr int kKVBytes = kBN * kD * 2;         // 16 KiB per K or V tile
constexpr int kStageBytes = 2 * kKVBytes;
constexpr int kTmemCols = 512;
constexpr int kColS = 0;                       // + 128 w
constexpr int kColO = 256;                     // + 64 w
constexpr int kColP = 384;                     // + 64 w
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;      // log2 units
constexpr long long kTile1Delay = 800;         // cycles between the two tiles' first S (600-1000 measured alike)

// smem layout (offsets from a 1024-aligned base)
constexpr int kOffQ = 0;                       // + w * kQBytes
constexpr int kOffRing = 2 * kQBytes;
constexpr int kOffBars = kOffRing + kStages * kStageBytes;
// kv_full[kStages], kv_empty[kStages], then per tile: s_full, s_free, p_full, pv_done, q_ready
constexpr int kNumBars = 2 * kStages + 2 * 5 + 2;   // + out_full[tile]
constexpr int kSmemTotal = kOffBars + kNumBars * 8 + 16 + 1024;

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    k_prefill_pair(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                   const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_o,
                   AttnParams p, int tma_out) {
  constexpr uint32_t kIdescS = idesc_f16(0, 0, kBM, kBN);
  constexpr uint32_t kIdescPV = idesc_f16(0, 1, kBM, kD);

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + kStages;
  uint64_t* s_full = bars + 2 * kStages;   // [2]
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* q_ready = pv_done + 2;         // the CTA's query tiles are in Q_0 (and Q_1)
  uint64_t* out_full = q_ready + 2;        // [tile]: the tile's output rows are in Q_w
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(out_full + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  bool dead = false;   // set once a bounded wait of this thread gave up
  const int n_qtiles = (p.tokens + kBM - 1) / kBM;
  // blocks are dispatched in linear order (x fastest): with the query tile in z,
  // every head pair and sequence of the heaviest (latest) tile starts first
  const int qt = n_qtiles - 1 - static_cast<int>(blockIdx.z);
  const int pairs = (p.group + 1) >> 1;                          // CTAs per KV group and query tile
  const int g = blockIdx.x / pairs;
  const int first = 2 * (blockIdx.x % pairs);                    // first head of the pair within its group
  const int h0 = g * p.group + first;
  const int ntile = first + 1 < p.group ? 2 : 1;
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
    for (int w = 0; w < 2; w++) {
      mbar_init(&s_full[w], 1);
      mbar_init(&s_free[w], 128);
      mbar_init(&p_full[w], 128);
      mbar_init(&pv_done[w], 1);

    }
    mbar_init(q_ready, 1);
    mbar_init(&out_full[0], 128);
    mbar_init(&out_full[1], 128);
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
  const uint32_t ring = smem_u32(smem + kOffRing);

  if (warp < 4) {
  // producer and MMA warpgroup: few registers, the softmax warpgroups get the
  // rest (launch: 384 x 168 = 128 x 56 + 256 x 224)
  asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // the cache rows come from the preceding append kernel
      asm volatile("griddepcontrol.wait;" ::: "memory");
      // the append kernel stored the new rows and the rotated queries through
      // the generic proxy; the tensor loads below read them through the async proxy
      asm volatile("fence.proxy.async.global;" ::: "memory");
      // the query tiles: RoPE(q) as f16 rows, 128-byte swizzled as the MMAs read them
      mbar_arrive_expect_tx(q_ready, static_cast<uint32_t>(ntile * kQBytes));
      for (int w = 0; w < ntile; w++) {
        tma_load_2d(smem_u32(smem + kOffQ + w * kQBytes), &tmap_q, q_ready, (h0 + w) * kD, sb * p.tokens + q0);
      }
      for (int j = 0; j < n_kv; j++) {
        const int s = j % kStages;
        if (j >= kStages) mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, p.err, dead);
        mbar_arrive_expect_tx(&kv_full[s], kStageBytes);
        const uint32_t st = ring + s * kStageBytes;
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
    // Every lane runs the loop and its waits (a lane whose bounded wait gave
    // up skips its later waits but keeps the same sequence of elect.sync
    // calls, so the warp stays converged); the elected lane issues and commits.
    {
      const uint32_t q_base = smem_u32(smem + kOffQ);
      mbar_wait(q_ready, 0, p.err, dead);
      auto issue_s = [&](int w, int j) {
        const uint32_t kt = ring + (j % kStages) * kStageBytes;
        const uint32_t qw = q_base + w * kQBytes;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < kD / 16; kk++) {
            mma_ss(tmem + kColS + w * kBN, sdesc_sw128(qw + kk * 32), sdesc_sw128(kt + kk * 32), kIdescS, kk > 0);
          }
          mma_commit(&s_full[w]);
        }
        __syncwarp();
      };
      mbar_wait(&kv_full[0], 0, p.err, dead);
      tc_fence_after();
      // Tile 1's first S goes in kTile1Delay cycles after tile 0's, so the two
      // tiles' first exponentials do not collide on the sub-partitions'
      // exponential units; later steps keep that offset on their own (left to
      // themselves the tiles start together and settle ~900 cycles apart only
      // after a few steps). A fixed count of cycles: no wait on anything.
      issue_s(0, 0);
      if (ntile > 1) {
        const long long t0 = clock64();
        while (clock64() - t0 < kTile1Delay) {
        }
        issue_s(1, 0);
      }
      for (int j = 0; j < n_kv; j++) {
        const int s = j % kStages;
        if (j + 1 < n_kv) mbar_wait(&kv_full[(j + 1) % kStages], ((j + 1) / kStages) & 1, p.err, dead);
        const uint32_t vt = ring + s * kStageBytes + kKVBytes;
        // per tile: the next S as soon as softmax w has read this one, then this
        // tile's PV once its P is in TMEM (the tiles run about half a step apart)
        for (int w = 0; w < ntile; w++) {
          if (j + 1 < n_kv) {
            mbar_wait(&s_free[w], j & 1, p.err, dead);
            tc_fence_after();
            issue_s(w, j + 1);
          }
          mbar_wait(&p_full[w], j & 1, p.err, dead);
          tc_fence_after();
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < kBN / 16; kk++) {
              mma_ts(tmem + kColO + w * kD, tmem + kColP + w * (kBN / 2) + kk * 8, sdesc_sw128(vt + kk * 2048),
                     kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(&pv_done[w]);
          }
          __syncwarp();
        }
        if (elect_one()) mma_commit(&kv_empty[s]);
        __syncwarp();
      }
    }
  }
  } else {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 224;" ::: "memory");
  if ((warp - 4) / 4 < ntile) {
    // ------------------------------------------------------------ softmax
    const int w = (warp - 4) >> 2;                 // query tile (head h0 + w)
    const int h = h0 + w;
    const int quarter = warp & 3;                  // TMEM lanes this warp may touch
    const int r = quarter * 32 + lane;             // query row within the tile
    const int t = q0 + r;                          // token index within this call
    const int a = past + t;                        // absolute position
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t scol = tmem + lane_addr + kColS + w * kBN;
    const uint32_t ocol = tmem + lane_addr + kColO + w * kD;
    const uint32_t pcol = tmem + lane_addr + kColP + w * (kBN / 2);
    const float sc = rsqrtf(static_cast<float>(kD)) * kLog2e;
    float m_used = -CUDART_INF_F;   // log2 units
    float l = 0.f;
    for (int j = 0; j < n_kv; j++) {
      mbar_wait(&s_full[w], j & 1, p.err, dead);
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++) tmem_ld32(scol + q4 * 32, sr[q4]);
      tmem_wait_ld();
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++) tmem_ld_fence(sr[q4]);
      // S_w is in registers: the next S may be written over it
      tc_fence_before();
      mbar_arrive(&s_free[w]);
      // causal / end-of-sequence mask: key k visible iff k <= a
      const int kbase = j * kBN;
      if (kbase + kBN - 1 > past + q0) {
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
          // O_w holds the sum through PV_w(j-1): rescale it in place
          mbar_wait(&pv_done[w], (j - 1) & 1, p.err, dead);
          tc_fence_after();
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
      // P = 2^(s*sc - m) as f16 pairs, packed in place: pair c lands in word
      // c of sr[0..1], whose S values were consumed before it is written
      // (the scale-and-shift and the row sums run as packed f32 pairs)
      const uint64_t sc2 = f2_pack(sc, sc), nb2 = f2_pack(nb, nb);
      uint64_t sums[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[q4][e]), __uint_as_float(sr[q4][e + 1])), sc2, nb2), x0, x1);
          const float p0 = ex2_approx(x0);
          const float p1 = ex2_approx(x1);
          sums[(e >> 1) & 3] = f2_add(sums[(e >> 1) & 3], f2_pack(p0, p1));
          const int col = q4 * 16 + e / 2;
          sr[col >> 5][col & 31] = pack_f16x2(p0, p1);
        }
      }
      {
        float a0, a1;
        f2_unpack(f2_add(f2_add(sums[0], sums[1]), f2_add(sums[2], sums[3])), a0, a1);
        l += a0 + a1;
      }
      // the last KV tile: zero V rows past the sequence end (0 * stale bits
      // must not give NaN). Tile 0's rows do it; PV_1 of this tile is issued
      // after PV_0, which waits for tile 0's P.
      if (j == n_kv - 1 && w == 0) {
        const int valid_rows = (past + p.tokens) - kbase;
        if (r >= valid_rows && r < kBN) {
          uint4* vrow = reinterpret_cast<uint4*>(smem + kOffRing + (j % kStages) * kStageBytes + kKVBytes + r * 128);
#pragma unroll
          for (int x = 0; x < 8; x++) vrow[x] = make_uint4(0, 0, 0, 0);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      // P_w is free once PV_w(j-1) has completed
      if (j > 0) mbar_wait(&pv_done[w], (j - 1) & 1, p.err, dead);
      tc_fence_after();
      tmem_st32(pcol, sr[0]);
      tmem_st32(pcol + 32, sr[1]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[w]);
    }
    // epilogue: O / l -> out rows
    mbar_wait(&pv_done[w], (n_kv - 1) & 1, p.err, dead);
    tc_fence_after();
    uint32_t ov[2][32];
    tmem_ld32(ocol, ov[0]);
    tmem_ld32(ocol + 32, ov[1]);
    tmem_wait_ld();
    tmem_ld_fence(ov[0]);
    tmem_ld_fence(ov[1]);
    if (tma_out) {
      // 16-bit output: the tile's rows go into Q_w (its S MMAs are all done),
      // 128-byte swizzled, and leave by one TMA store (rows past the
      // sequence's tokens are clipped by the map); thread-per-row stores would
      // touch 32 rows per warp instruction
      const float inv = 1.f / l;
      const int odt = p.nchunks;   // the output dtype travels in nchunks
      unsigned char* orow = smem + kOffQ + w * kQBytes + r * 128;
#pragma unroll
      for (int x = 0; x < 8; x++) {
        uint32_t wd[4];
#pragma unroll
        for (int y = 0; y < 4; y++) {
          const int e = 8 * x + 2 * y;
          const float f0 = __uint_as_float(ov[e >> 5][e & 31]) * inv;
          const float f1 = __uint_as_float(ov[e >> 5][(e & 31) + 1]) * inv;
          const uint32_t b0 = odt == DT_F16 ? f32_to_f16_bits(f0) : f32_to_bf16_bits(f0);
          const uint32_t b1 = odt == DT_F16 ? f32_to_f16_bits(f1) : f32_to_bf16_bits(f1);
          wd[y] = b0 | (b1 << 16);
        }
        *reinterpret_cast<uint4*>(orow + ((x ^ (r & 7)) << 4)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&out_full[w]);
      if (r == 0) {
        mbar_wait(&out_full[w], 0, p.err, dead);
        if (!dead) {
          asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                           reinterpret_cast<uint64_t>(&tmap_o)),
                       "r"(smem_u32(smem + kOffQ + w * kQBytes)), "r"(h * kD), "r"(q0), "r"(sb)
                       : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          // the shared rows must stay until the store has read them
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        }
      }
    } else if (t < p.tokens) {
      const float inv = 1.f / l;
      const int64_t orow = ((static_cast<int64_t>(sb) * p.tokens + t) * p.heads + h) * kD;
      void* out = p.partial;       // the output pointer travels in the partial slot for this kernel
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
          uint32_t wd[4];
#pragma unroll
          for (int y = 0; y < 4; y++) {
            const int e = 8 * x + 2 * y;
            const float f0 = __uint_as_float(ov[e >> 5][e & 31]) * inv;
            const float f1 = __uint_as_float(ov[e >> 5][(e & 31) + 1]) * inv;
            const uint32_t b0 = odt == DT_F16 ? f32_to_f16_bits(f0) : f32_to_bf16_bits(f0);
            const uint32_t b1 = odt == DT_F16 ? f32_to_f16_bits(f1) : f32_to_bf16_bits(f1);
            wd[y] = b0 | (b1 << 16);
          }
          o4[x] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
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

bool prefill_pair_supported(const AttnParams& p) {
  // grid (heads, batch, query tiles): y and z are limited to 65535
  return p.tmap_k != nullptr && p.tmap_v != nullptr && p.tmap_q != nullptr && p.batch >= 1 && p.batch <= 65535 &&
         (p.tokens + kBM - 1) / kBM <= 65535 && p.num_layers == 1 && p.head_dim == kD &&
         p.k_new == nullptr && p.cache_dtype == DT_F16 && p.group >= 1;
}

cudaError_t launch_prefill_pair(const AttnParams& p, void* out, int out_dtype, cudaStream_t st) {
  if (!prefill_pair_supported(p)) return cudaErrorInvalidValue;
  if (p.tokens <= 0) return cudaSuccess;
  AttnParams q = p;
  q.partial = static_cast<float*>(out);
  q.nchunks = out_dtype;
  const int pairs = (p.group + 1) / 2;
  const dim3 grid(p.kv_heads * pairs, p.batch, (p.tokens + kBM - 1) / kBM);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[64] = {};
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(k_prefill_pair, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal);
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
  // 16-bit output with a map: the epilogue's TMA store
  const int tma_out = p.tmap_o != nullptr && (out_dtype == DT_F16 || out_dtype == DT_BF16) ? 1 : 0;
  CUtensorMap omap = {};
  if (tma_out) omap = *static_cast<const CUtensorMap*>(p.tmap_o);
  return cudaLaunchKernelEx(&cfg, k_prefill_pair, *static_cast<const CUtensorMap*>(p.tmap_k),
                            *static_cast<const CUtensorMap*>(p.tmap_v), *static_cast<const CUtensorMap*>(p.tmap_q), omap,
                            q, tma_out);
}

}  // namespace b2a
