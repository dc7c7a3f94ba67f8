// Non-causal, unmasked scaled-dot-product attention for head_dim 64 on sm_100a.
//
// Replaces the SDPA call of the reference's self-attention path
// (layers/attention/backends/sdpa.py:56-80, called from
// models/dits/eraserdit_attention.py:287-289): out = softmax(Q K^T * scale) V
// per (batch, head), BF16 in / BF16 out, FP32 softmax state and accumulation.
//
// Design (one CTA per pair of 128-row query tiles of one (batch, head)):
//   warp 8      TMA producer: Q pair once, then K / V tiles through a ring of
//               shared-memory stages (128 x 64 BF16, 128-byte swizzle).
//   warp 9      MMA issuer (one thread): S = Q K^T into TMEM (M=128, N=128,
//               K=64), then O += P V with P read from TMEM (M=128, N=64, K=128).
//   warps 0-7   two softmax warpgroups, one per query tile; thread r owns
//               query row r: reads its S row from TMEM, keeps the running
//               max / sum, writes P (BF16) to TMEM, rescales its O row when
//               the running max grows by more than 2^8, and finally writes
//               O / l to global memory.
// TMEM columns: S_A [0,128) S_B [128,256) O_A [256,320) O_B [320,384)
//               P_A [384,448) P_B [448,512).
//
// The key / value sequence may be split into `nseg` segments held in slots of
// `seg_len` tokens, segment s holding seg_lens[s] <= seg_len valid tokens
// (the layout the Ulysses all-to-all delivers: one segment per source rank).
// Tiles never straddle a segment; rows past a segment's end are masked (and
// zero-filled by TMA past the slot).  Queries use the same tiling, and output
// rows are scattered back with the caller's strides.
//
// The block-sparse instantiation (kSparse) replaces the mask-STA kernel
// (layers/attention/backends/csrc/mask_sta/core.cu, driven by
// layers/attention/backends/mask_sta.py:134-194).  Each CTA reads one schedule
// row {query tile A, query tile B or -1, first entry, entries} and walks that
// list of key tiles instead of all of them.  An entry is
//   key tile | (64-token halves tile A attends) << 24 | (halves of B) << 26;
// a softmax warpgroup masks the halves its tile does not attend (and writes
// P = 0 for a key tile it skips entirely), so the two tiles of a CTA may have
// different lists and the CTA computes their union.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <math_constants.h>

#include "host_common.h"
#include "sm100_ptx.cuh"
#include "tmem_io.cuh"

namespace erd {

constexpr int kBlockM = 128;  // query rows per tile
constexpr int kBlockN = 128;  // key / value rows per tile
constexpr int kHeadDim = 64;
constexpr int kStages = 3;  // K and V ring depth
constexpr int kTileBytes = kBlockM * kHeadDim * 2;  // 16 KB
constexpr int kThreads = 320;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale only if max grows > 2^8
// Of every 8 consecutive column pairs of a P row, this many are exponentiated
// with the FMA-pipe polynomial and the rest with MUFU ex2.  One in eight
// measured 1-1.5 % faster than two in eight (and than all-MUFU) at
// configuration 1: the polynomial costs about five more issue slots per pair
// than MUFU, and issue slots are shared with the other softmax warpgroup.
#ifndef ERD_POLY_EVERY8
#define ERD_POLY_EVERY8 1
#endif
constexpr int kPolyPairsPer8 = ERD_POLY_EVERY8;

constexpr int kMaxSegments = 16;
constexpr int kMaxCrossBatch = 16;  // batch entries with their own key count (cross-attention)

struct AttnParams {
  int seg_lens[kMaxSegments];  // tokens of each segment (<= seg_len, the slot length)
  int seg_len;
  int nseg;
  int tiles_per_seg;
  int q_tiles;
  float scale_log2;
  __nv_bfloat16* out;
  long long o_rs, o_hs, o_bs, o_ss;
  int* status;
  // block-sparse instantiation only
  const int4* sched;         // per CTA: query tile A, query tile B (or -1), first entry, entries
  const uint32_t* entries;   // key tile | A halves << 24 | B halves << 26
  long long n_entries;
  const int* out_rows;       // optional (one segment): output token of each query row
  // Optional per-segment output bases (another rank's return buffer); when set
  // they replace out + segment * o_ss.
  __nv_bfloat16* seg_out[kMaxSegments];
  // Key / value tiling: the query tiling for self-attention; its own length for
  // cross-attention, where kv_valid[batch] (kv_per_batch != 0) counts the
  // attended keys of each batch entry (the text mask's unpadded prefix).
  int kv_tiles, kv_tiles_per_seg;
  int kv_per_batch;
  int kv_valid[kMaxCrossBatch];
  // Valid tokens of each key / value segment (the query's seg_lens for
  // self-attention; a ring piece's own lengths otherwise).
  int kv_seg_lens[kMaxSegments];
  // Carried softmax state (kState instantiation only): per query tile, O as
  // 64 x 128 fp32 (column-major: column c of row r at c * 128 + r), then the
  // running max (log2 domain) and sum of its 128 rows.  state_mode bits:
  // kStateRead starts from it, kStateWrite stores it instead of the output.
  float* state;
  int state_mode;
};

constexpr int kStateRead = 1;
constexpr int kStateWrite = 2;
constexpr int kStateFloatsPerTile = kHeadDim * kBlockM + 2 * kBlockM;

constexpr uint32_t kEntryTileMask = (1u << 24) - 1;

struct __align__(8) AttnBarriers {
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done[2];
  uint64_t mma_drain;
  uint32_t tmem_base;
  int abort;
};

constexpr int kSmemQ = 0;
constexpr int kSmemK = kSmemQ + 2 * kTileBytes;
constexpr int kSmemV = kSmemK + kStages * kTileBytes;
constexpr int kSmemBar = kSmemV + kStages * kTileBytes;
constexpr int kSmemBytes = kSmemBar + 1024;
// +1024 for aligning the dynamic shared memory base to the swizzle atom.
constexpr int kSmemLaunchBytes = kSmemBytes + 1024;
static_assert(kSmemLaunchBytes <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ void tile_coords(int tile, int tiles_per_seg, int& seg, int& l0) {
  seg = tile / tiles_per_seg;
  l0 = (tile - seg * tiles_per_seg) * kBlockN;
}

template <bool kSparse, bool kState>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_bf16_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_v, const AttnParams p) {
  static_assert(!(kSparse && kState), "the carried state serves dense pieces only");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  AttnBarriers* bars = reinterpret_cast<AttnBarriers*>(smem + kSmemBar);
  const uint32_t sQ = smem_u32(smem + kSmemQ);
  const uint32_t sK = smem_u32(smem + kSmemK);
  const uint32_t sV = smem_u32(smem + kSmemV);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  // Query tiles of the two softmax warpgroups and the key tiles to visit: all
  // of them (the same tiling is used for keys and queries), or a list.
  int q_tile_a = 2 * static_cast<int>(blockIdx.x), q_tile_b = q_tile_a + 1;
  int n_kv = p.kv_tiles;
  const uint32_t* list = nullptr;
  if (kSparse) {
    const int4 row = p.sched[blockIdx.x];
    q_tile_a = row.x;
    q_tile_b = row.y;
    n_kv = row.w;
    // A malformed row is skipped by the whole CTA (its outputs stay unwritten).
    if (n_kv <= 0 || row.z < 0 || static_cast<long long>(row.z) + n_kv > p.n_entries ||
        q_tile_a < 0 || q_tile_a >= p.q_tiles)
      return;
    list = p.entries + row.z;
  }
  volatile int* abort = &bars->abort;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars->q_full), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars->k_full[s]), 1);
      mbar_init(smem_u32(&bars->k_empty[s]), 1);
      mbar_init(smem_u32(&bars->v_full[s]), 1);
      mbar_init(smem_u32(&bars->v_empty[s]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&bars->s_full[t]), 1);
      mbar_init(smem_u32(&bars->p_full[t]), kBlockM);
      mbar_init(smem_u32(&bars->o_done[t]), 1);
    }
    mbar_init(smem_u32(&bars->mma_drain), 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(smem_u32(&bars->tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      const int qa = q_tile_a;
      const int qb = (q_tile_b < 0 || q_tile_b >= p.q_tiles) ? qa : q_tile_b;
      int seg, l0;
      const uint32_t qbar = smem_u32(&bars->q_full);
      mbar_arrive_expect_tx(qbar, 2 * kTileBytes);
      tile_coords(qa, p.tiles_per_seg, seg, l0);
      tma_load_5d(sQ, &tmap_q, qbar, 0, l0, head, batch, seg);
      tile_coords(qb, p.tiles_per_seg, seg, l0);
      tma_load_5d(sQ + kTileBytes, &tmap_q, qbar, 0, l0, head, batch, seg);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        // Key tiles past the last one read as zeros (TMA fills out-of-range
        // boxes) and are masked by the softmax.
        const int kv = kSparse ? static_cast<int>(__ldg(list + j) & kEntryTileMask) : j;
        tile_coords(kv, p.kv_tiles_per_seg, seg, l0);
        if (!mbar_wait(smem_u32(&bars->k_empty[s]), ph ^ 1, abort, p.status,
                       kStatusTimeoutProducer))
          break;
        mbar_arrive_expect_tx(smem_u32(&bars->k_full[s]), kTileBytes);
        tma_load_5d(sK + s * kTileBytes, &tmap_k, smem_u32(&bars->k_full[s]), 0, l0, head, batch,
                    seg);
        if (!mbar_wait(smem_u32(&bars->v_empty[s]), ph ^ 1, abort, p.status,
                       kStatusTimeoutProducer))
          break;
        mbar_arrive_expect_tx(smem_u32(&bars->v_full[s]), kTileBytes);
        tma_load_5d(sV + s * kTileBytes, &tmap_v, smem_u32(&bars->v_full[s]), 0, l0, head, batch,
                    seg);
      }
      if (*abort) {
        // Let every load this thread may have started land before the CTA
        // exits (on the normal path the consumers have already seen them).
        mbar_wait_drain(qbar, 0);
        for (int j = (n_kv > kStages ? n_kv - kStages : 0); j < n_kv; ++j) {
          const int s = j % kStages;
          const uint32_t ph = (j / kStages) & 1;
          mbar_wait_drain(smem_u32(&bars->k_full[s]), ph);
          mbar_wait_drain(smem_u32(&bars->v_full[s]), ph);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(kBlockM, kBlockN, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(kBlockM, kHeadDim, false, true);
      const uint32_t tS[2] = {tmem + 0, tmem + 128};
      const uint32_t tO[2] = {tmem + 256, tmem + 320};
      const uint32_t tP[2] = {tmem + 384, tmem + 448};
      auto issue_qk = [&](int t, int s) {
        const uint32_t qa = sQ + t * kTileBytes;
        const uint32_t ka = sK + s * kTileBytes;
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          mma_bf16_ss(tS[t], sdesc_sw128(qa + k * 32, 16, 1024), sdesc_sw128(ka + k * 32, 16, 1024),
                      idesc_qk, k > 0);
        }
      };
      auto issue_pv = [&](int t, int s, bool accumulate) {
        const uint32_t va = sV + s * kTileBytes;
#pragma unroll
        for (int k = 0; k < kBlockN / 16; ++k) {
          mma_bf16_ts(tO[t], tP[t] + k * 8, sdesc_sw128(va + k * 2048, 1024, 1024), idesc_pv,
                      (accumulate || k > 0) ? 1u : 0u);
        }
      };
      // With a carried state O starts from the stored rows (written to TMEM by
      // the softmax warps before their first P), so every P V accumulates.
      const bool acc_first = kState && (p.state_mode & kStateRead);
      bool ok = mbar_wait(smem_u32(&bars->q_full), 0, abort, p.status, kStatusTimeoutMma) &&
                mbar_wait(smem_u32(&bars->k_full[0]), 0, abort, p.status, kStatusTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        mma_commit(smem_u32(&bars->s_full[0]));
        issue_qk(1, 0);
        mma_commit(smem_u32(&bars->s_full[1]));
        mma_commit(smem_u32(&bars->k_empty[0]));
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        const int s1 = (j + 1) % kStages;
        const uint32_t ph1 = ((j + 1) / kStages) & 1;
        const bool more = j + 1 < n_kv;
        // Operand waits first (normally long complete), so that once a
        // softmax hands over its P the products are issued without delay.
        if (more && !mbar_wait(smem_u32(&bars->k_full[s1]), ph1, abort, p.status, kStatusTimeoutMma))
          break;
        if (!mbar_wait(smem_u32(&bars->v_full[s]), ph, abort, p.status, kStatusTimeoutMma)) break;
        // query tile A
        if (!mbar_wait(smem_u32(&bars->p_full[0]), j & 1, abort, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        if (more) {
          issue_qk(0, s1);
          mma_commit(smem_u32(&bars->s_full[0]));
        }
        issue_pv(0, s, j > 0 || acc_first);
        mma_commit(smem_u32(&bars->o_done[0]));
        // query tile B
        if (!mbar_wait(smem_u32(&bars->p_full[1]), j & 1, abort, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        if (more) {
          issue_qk(1, s1);
          mma_commit(smem_u32(&bars->s_full[1]));
          mma_commit(smem_u32(&bars->k_empty[s1]));
        }
        issue_pv(1, s, j > 0 || acc_first);
        mma_commit(smem_u32(&bars->o_done[1]));
        mma_commit(smem_u32(&bars->v_empty[s]));
      }
      // Every MMA this thread issued completes before TMEM is released.
      mma_commit(smem_u32(&bars->mma_drain));
      mbar_wait_drain(smem_u32(&bars->mma_drain), 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;             // query tile of this warpgroup
    const int row = threadIdx.x & 127;   // query row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_off;
    const uint32_t tO = tmem + 256 + t * 64 + lane_off;
    const uint32_t tP = tmem + 384 + t * 64 + lane_off;
    const float c = p.scale_log2;
    float m_run = -CUDART_INF_F;  // running max of S * c (log2 domain)
    float l_run = 0.f;
    bool ok = true;
    // Carried state of this thread's query row (kState).  The warpgroup of an
    // odd tile count's missing B tile starts from zeros and never writes.
    float* st_o = nullptr;
    const bool state_in = kState && (p.state_mode & kStateRead);
    if (kState) {
      const int qt_own = t == 0 ? q_tile_a : q_tile_b;
      const bool own_valid = qt_own >= 0 && qt_own < p.q_tiles;
      const long long tile = (static_cast<long long>(batch) * gridDim.y + head) * p.q_tiles +
                             (own_valid ? qt_own : 0);
      st_o = p.state + tile * kStateFloatsPerTile;
      if (state_in) {
        if (own_valid) {
          m_run = st_o[kHeadDim * kBlockM + row];
          l_run = st_o[kHeadDim * kBlockM + kBlockM + row];
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t o[32];
#pragma unroll
          for (int i = 0; i < 32; ++i)
            o[i] = own_valid ? __float_as_uint(st_o[(h * 32 + i) * kBlockM + row]) : 0u;
          tmem_st32(tO + h * 32, o);
        }
        tmem_wait_st();
      }
    }
    for (int j = 0; j < n_kv; ++j) {
      // The list entry is read before the wait, which hides its latency.
      const uint32_t entry = kSparse ? __ldg(list + j) : 0u;
      // Wait results are made warp-uniform: tcgen05.ld/st are .sync.aligned.
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->s_full[t]), j & 1, abort, p.status,
                                             kStatusTimeoutSoftmax))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Columns [lo, hi) of this key tile are attended by this query tile.
      int lo = 0, hi;
      if (kSparse) {
        const int kv = static_cast<int>(entry & kEntryTileMask);
        const uint32_t halves = (entry >> (24 + 2 * t)) & 3u;
        hi = 0;
        if (halves != 0 && kv < p.kv_tiles) {
          int seg, l0;
          tile_coords(kv, p.kv_tiles_per_seg, seg, l0);
          hi = min(kBlockN, (p.kv_per_batch ? p.kv_valid[batch] : p.kv_seg_lens[seg]) - l0);
          if (!(halves & 2u)) hi = min(hi, kBlockN / 2);
          if (!(halves & 1u)) lo = kBlockN / 2;
        }
      } else {
        int seg, l0;
        tile_coords(j, p.kv_tiles_per_seg, seg, l0);
        hi = min(kBlockN, (p.kv_per_batch ? p.kv_valid[batch] : p.kv_seg_lens[seg]) - l0);
      }
      // Pass 1: row max over the whole S row (registers released afterwards).
      // A key tile this query tile does not attend at all (sparse lists only)
      // contributes P = 0 and leaves the running max and sum alone.
      float mx0 = -CUDART_INF_F, mx1 = -CUDART_INF_F, mx2 = -CUDART_INF_F, mx3 = -CUDART_INF_F;
      if (!kSparse || hi > lo) {
        uint32_t sr[128];
        tmem_ld_wait_128(tS, sr);
        if (lo > 0 || hi < kBlockN) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i < lo || i >= hi) sr[i] = __float_as_uint(-CUDART_INF_F);
        }
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          mx0 = fmax3(mx0, __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
          mx1 = fmax3(mx1, __uint_as_float(sr[32 + i]), __uint_as_float(sr[33 + i]));
          mx2 = fmax3(mx2, __uint_as_float(sr[64 + i]), __uint_as_float(sr[65 + i]));
          mx3 = fmax3(mx3, __uint_as_float(sr[96 + i]), __uint_as_float(sr[97 + i]));
        }
      }
      const float m_tile = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c;
      float m_new = m_run;
      bool rescale = false;
      if (m_tile > m_run + kRescaleThreshold) {
        m_new = m_tile;
        rescale = j > 0 || state_in;
      }
      if (j > 0) {
        // P_t and O_t are free once the previous P V product has completed.
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->o_done[t]), (j - 1) & 1, abort,
                                               p.status, kStatusTimeoutSoftmax))) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // The O row update is done by the whole warp when any of its rows needs
      // it (rows that do not need it scale by 1).
      if (__any_sync(0xffffffffu, rescale)) {
        const float alpha = rescale ? ex2_approx(m_run - m_new) : 1.0f;
        l_run *= alpha;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t o[32];
          tmem_ld_wait_32(tO + h * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + h * 32, o);
        }
      }
      m_run = m_new;
      const float neg_m = -m_new;
      float sum0 = 0.f, sum1 = 0.f;
      // Pass 2: P = 2^(S c - m) in BF16, written to TMEM 64 S columns at a time.
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
        if (kSparse && (h * 64 >= hi || h * 64 + 64 <= lo)) {
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = 0u;
          tmem_st32(tP + h * 32, pk);
          continue;
        }
        uint32_t sr[64];
        tmem_ld_wait_64(tS + h * 64, sr);
        if (lo > 0 || hi < kBlockN) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (h * 64 + i < lo || h * 64 + i >= hi) sr[i] = __float_as_uint(-CUDART_INF_F);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x0, x1, p0, p1;
          fma2(x0, x1, __uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1]), c, c, neg_m,
               neg_m);
          if ((i & 7) < kPolyPairsPer8) {
            exp2_poly2(x0, x1, p0, p1);
          } else {
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          add2(sum0, sum1, sum0, sum1, p0, p1);
          pk[i] = pack_bf16x2(p0, p1);
        }
        tmem_st32(tP + h * 32, pk);
      }
      l_run += sum0 + sum1;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&bars->p_full[t]));
    }
    // ------------------------------------------------------------ epilogue
    if (ok && __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->o_done[t]), (n_kv - 1) & 1, abort,
                                                p.status, kStatusTimeoutEpilogue))) {
      tc_fence_after();
      uint32_t oflat[64];
      tmem_ld_wait_64(tO, oflat);
      uint32_t(&o)[2][32] = *reinterpret_cast<uint32_t(*)[2][32]>(oflat);
      const int qt = t == 0 ? q_tile_a : q_tile_b;
      if (kState && (p.state_mode & kStateWrite)) {
        if (qt >= 0 && qt < p.q_tiles) {
          // one fp32 column per store: 128 contiguous bytes per warp
#pragma unroll
          for (int i = 0; i < kHeadDim; ++i) st_o[i * kBlockM + row] = __uint_as_float(oflat[i]);
          st_o[kHeadDim * kBlockM + row] = m_run;
          st_o[kHeadDim * kBlockM + kBlockM + row] = l_run;
        }
      } else if (qt >= 0 && qt < p.q_tiles) {
        int seg, l0;
        tile_coords(qt, p.tiles_per_seg, seg, l0);
        const int tok = l0 + row;
        if (tok < p.seg_lens[seg]) {
          const float inv_l = 1.0f / l_run;
          const long long out_tok = (kSparse && p.out_rows != nullptr) ? __ldg(p.out_rows + tok) : tok;
          __nv_bfloat16* seg_base = p.seg_out[seg] != nullptr ? p.seg_out[seg] : p.out + seg * p.o_ss;
          __nv_bfloat16* dst = seg_base + batch * p.o_bs + head * p.o_hs + out_tok * p.o_rs;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[h][8 * v + 0]) * inv_l,
                                __uint_as_float(o[h][8 * v + 1]) * inv_l);
              w.y = pack_bf16x2(__uint_as_float(o[h][8 * v + 2]) * inv_l,
                                __uint_as_float(o[h][8 * v + 3]) * inv_l);
              w.z = pack_bf16x2(__uint_as_float(o[h][8 * v + 4]) * inv_l,
                                __uint_as_float(o[h][8 * v + 5]) * inv_l);
              w.w = pack_bf16x2(__uint_as_float(o[h][8 * v + 6]) * inv_l,
                                __uint_as_float(o[h][8 * v + 7]) * inv_l);
              *reinterpret_cast<uint4*>(dst + h * 32 + v * 8) = w;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace erd

using namespace erd;

namespace {

// Rank-5 tensor map {d, token, head, batch, segment} over a BF16 operand with
// a 64 x 128 box and the 128-byte swizzle the MMA descriptors expect.
int make_operand_map(CUtensorMap* map, const void* base, int seg_len, int heads, int batch,
                     int nseg, int64_t ts, int64_t hs, int64_t bs, int64_t ss) {
  const uint64_t dims[5] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(seg_len),
                            static_cast<uint64_t>(heads), static_cast<uint64_t>(batch),
                            static_cast<uint64_t>(nseg)};
  // Unused (size-1) dimensions still need a valid 16-byte-multiple stride.
  auto stride = [](int64_t s, uint64_t n) -> uint64_t {
    return n > 1 ? static_cast<uint64_t>(s) * 2 : 16;
  };
  const uint64_t strides[4] = {stride(ts, dims[1]), stride(hs, dims[2]), stride(bs, dims[3]),
                               stride(ss, dims[4])};
  const uint32_t box[5] = {kHeadDim, kBlockN, 1, 1, 1};
  return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims,
                           strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool strides_ok(int64_t a, int64_t b, int64_t c, int64_t d) {
  return a >= 0 && b >= 0 && c >= 0 && d >= 0 && ((a | b | c | d) & 7) == 0;
}

// Argument checks, tensor maps and parameters shared by the dense and the
// block-sparse entry points.
struct Launch {
  CUtensorMap tq, tk, tv;
  AttnParams p;
};

int prepare(const void* q, const void* k, const void* v, int64_t q_token_stride,
            int64_t q_head_stride, int64_t q_batch_stride, int64_t q_seg_stride,
            int64_t k_token_stride, int64_t k_head_stride, int64_t k_batch_stride,
            int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
            int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len,
            int nseg, const int32_t* seg_lens, int head_dim, float softmax_scale, void* out,
            int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride,
            int64_t o_seg_stride, int* status, Launch* L) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) return kErrNullPointer;
  if (head_dim != kHeadDim || batch <= 0 || heads <= 0 || seg_len <= 0 || nseg <= 0 ||
      nseg > kMaxSegments || batch > 65535 || heads > 65535)
    return kErrBadShape;
  if (seg_lens != nullptr) {
    for (int s = 0; s < nseg; ++s)
      if (seg_lens[s] <= 0 || seg_lens[s] > seg_len) return kErrBadShape;
  }
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return kErrMisaligned;
  if (!strides_ok(q_token_stride, q_head_stride, q_batch_stride, q_seg_stride) ||
      !strides_ok(k_token_stride, k_head_stride, k_batch_stride, k_seg_stride) ||
      !strides_ok(v_token_stride, v_head_stride, v_batch_stride, v_seg_stride) ||
      !strides_ok(o_token_stride, o_head_stride, o_batch_stride, o_seg_stride))
    return kErrMisaligned;
  if (int rc = check_device_sm100()) return rc;

  const int tiles_per_seg = (seg_len + kBlockN - 1) / kBlockN;
  const long long q_tiles = static_cast<long long>(tiles_per_seg) * nseg;
  if (q_tiles > (1LL << 24)) return kErrTooLarge;

  if (make_operand_map(&L->tq, q, seg_len, heads, batch, nseg, q_token_stride, q_head_stride,
                       q_batch_stride, q_seg_stride) ||
      make_operand_map(&L->tk, k, seg_len, heads, batch, nseg, k_token_stride, k_head_stride,
                       k_batch_stride, k_seg_stride) ||
      make_operand_map(&L->tv, v, seg_len, heads, batch, nseg, v_token_stride, v_head_stride,
                       v_batch_stride, v_seg_stride))
    return kErrTensorMap;

  AttnParams& p = L->p;
  for (int s = 0; s < kMaxSegments; ++s)
    p.seg_lens[s] = (s < nseg) ? (seg_lens != nullptr ? seg_lens[s] : seg_len) : 0;
  p.seg_len = seg_len;
  p.nseg = nseg;
  p.tiles_per_seg = tiles_per_seg;
  p.q_tiles = static_cast<int>(q_tiles);
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_rs = o_token_stride;
  p.o_hs = o_head_stride;
  p.o_bs = o_batch_stride;
  p.o_ss = o_seg_stride;
  p.status = status;
  p.sched = nullptr;
  p.entries = nullptr;
  p.n_entries = 0;
  p.out_rows = nullptr;
  for (int s = 0; s < kMaxSegments; ++s) p.seg_out[s] = nullptr;
  p.kv_tiles = p.q_tiles;
  p.kv_tiles_per_seg = tiles_per_seg;
  p.kv_per_batch = 0;
  for (int b = 0; b < kMaxCrossBatch; ++b) p.kv_valid[b] = 0;
  for (int s = 0; s < kMaxSegments; ++s) p.kv_seg_lens[s] = p.seg_lens[s];
  p.state = nullptr;
  p.state_mode = 0;
  return kErrOk;
}

template <bool kSparse, bool kState = false>
int launch(const Launch& L, unsigned ctas, int heads, int batch, void* stream) {
  cudaError_t e = cudaFuncSetAttribute(attn_fwd_bf16_kernel<kSparse, kState>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSmemLaunchBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  const dim3 grid(ctas, static_cast<unsigned>(heads), static_cast<unsigned>(batch));
  attn_fwd_bf16_kernel<kSparse, kState><<<grid, kThreads, kSmemLaunchBytes,
                                          static_cast<cudaStream_t>(stream)>>>(L.tq, L.tk, L.tv,
                                                                               L.p);
  return static_cast<int>(cudaGetLastError());
}

long long ring_state_floats(int batch, int heads, int seg_len, int q_nseg) {
  const long long tiles_per_seg = (seg_len + kBlockN - 1) / kBlockN;
  return static_cast<long long>(batch) * heads * tiles_per_seg * q_nseg * kStateFloatsPerTile;
}

}  // namespace

extern "C" int erd_attn_fwd_bf16(const void* q, const void* k, const void* v,
                                 int64_t q_token_stride, int64_t q_head_stride,
                                 int64_t q_batch_stride, int64_t q_seg_stride,
                                 int64_t k_token_stride, int64_t k_head_stride,
                                 int64_t k_batch_stride, int64_t k_seg_stride,
                                 int64_t v_token_stride, int64_t v_head_stride,
                                 int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads,
                                 int seg_len, int nseg, const int32_t* seg_lens, int head_dim,
                                 float softmax_scale,
                                 void* out, int64_t o_token_stride, int64_t o_head_stride,
                                 int64_t o_batch_stride, int64_t o_seg_stride, int* status,
                                 void* stream) {
  Launch L;
  if (int rc = prepare(q, k, v, q_token_stride, q_head_stride, q_batch_stride, q_seg_stride,
                       k_token_stride, k_head_stride, k_batch_stride, k_seg_stride,
                       v_token_stride, v_head_stride, v_batch_stride, v_seg_stride, batch, heads,
                       seg_len, nseg, seg_lens, head_dim, softmax_scale, out, o_token_stride,
                       o_head_stride, o_batch_stride, o_seg_stride, status, &L))
    return rc;
  return launch<false>(L, static_cast<unsigned>((L.p.q_tiles + 1) / 2), heads, batch, stream);
}

extern "C" int erd_attn_fwd_sparse_bf16(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int nseg,
    const int32_t* seg_lens, int head_dim, float softmax_scale, void* out, int64_t o_token_stride,
    int64_t o_head_stride, int64_t o_batch_stride, int64_t o_seg_stride, const int32_t* schedule,
    int n_schedule, const uint32_t* entries, int64_t n_entries, const int32_t* out_rows,
    int* status, void* stream) {
  if (schedule == nullptr || entries == nullptr) return kErrNullPointer;
  if (n_schedule <= 0 || n_schedule > (1 << 30) || n_entries <= 0) return kErrBadShape;
  if ((reinterpret_cast<uintptr_t>(schedule) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(entries) & 3) != 0 ||
      (reinterpret_cast<uintptr_t>(out_rows) & 3) != 0)
    return kErrMisaligned;
  if (out_rows != nullptr && nseg != 1) return kErrBadShape;
  Launch L;
  if (int rc = prepare(q, k, v, q_token_stride, q_head_stride, q_batch_stride, q_seg_stride,
                       k_token_stride, k_head_stride, k_batch_stride, k_seg_stride,
                       v_token_stride, v_head_stride, v_batch_stride, v_seg_stride, batch, heads,
                       seg_len, nseg, seg_lens, head_dim, softmax_scale, out, o_token_stride,
                       o_head_stride, o_batch_stride, o_seg_stride, status, &L))
    return rc;
  L.p.sched = reinterpret_cast<const int4*>(schedule);
  L.p.entries = entries;
  L.p.n_entries = n_entries;
  L.p.out_rows = out_rows;
  return launch<true>(L, static_cast<unsigned>(n_schedule), heads, batch, stream);
}

extern "C" int erd_attn_fwd_bf16_peer(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int nseg,
    const int32_t* seg_lens, int head_dim, float softmax_scale, void* const* seg_out,
    int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride, int* status,
    void* stream) {
  if (seg_out == nullptr) return kErrNullPointer;
  if (nseg <= 0 || nseg > kMaxSegments) return kErrBadShape;
  for (int s = 0; s < nseg; ++s) {
    if (seg_out[s] == nullptr) return kErrNullPointer;
    if (!aligned16(seg_out[s])) return kErrMisaligned;
  }
  Launch L;
  if (int rc = prepare(q, k, v, q_token_stride, q_head_stride, q_batch_stride, q_seg_stride,
                       k_token_stride, k_head_stride, k_batch_stride, k_seg_stride,
                       v_token_stride, v_head_stride, v_batch_stride, v_seg_stride, batch, heads,
                       seg_len, nseg, seg_lens, head_dim, softmax_scale, seg_out[0],
                       o_token_stride, o_head_stride, o_batch_stride, 0, status, &L))
    return rc;
  for (int s = 0; s < nseg; ++s) L.p.seg_out[s] = static_cast<__nv_bfloat16*>(seg_out[s]);
  return launch<false>(L, static_cast<unsigned>((L.p.q_tiles + 1) / 2), heads, batch, stream);
}

extern "C" int erd_attn_fwd_sparse_bf16_peer(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int nseg,
    const int32_t* seg_lens, int head_dim, float softmax_scale, void* const* seg_out,
    int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride,
    const int32_t* schedule, int n_schedule, const uint32_t* entries, int64_t n_entries,
    int* status, void* stream) {
  if (seg_out == nullptr || schedule == nullptr || entries == nullptr) return kErrNullPointer;
  if (nseg <= 0 || nseg > kMaxSegments || n_schedule <= 0 || n_schedule > (1 << 30) ||
      n_entries <= 0)
    return kErrBadShape;
  for (int s = 0; s < nseg; ++s) {
    if (seg_out[s] == nullptr) return kErrNullPointer;
    if (!aligned16(seg_out[s])) return kErrMisaligned;
  }
  if ((reinterpret_cast<uintptr_t>(schedule) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(entries) & 3) != 0)
    return kErrMisaligned;
  Launch L;
  if (int rc = prepare(q, k, v, q_token_stride, q_head_stride, q_batch_stride, q_seg_stride,
                       k_token_stride, k_head_stride, k_batch_stride, k_seg_stride,
                       v_token_stride, v_head_stride, v_batch_stride, v_seg_stride, batch, heads,
                       seg_len, nseg, seg_lens, head_dim, softmax_scale, seg_out[0],
                       o_token_stride, o_head_stride, o_batch_stride, 0, status, &L))
    return rc;
  L.p.sched = reinterpret_cast<const int4*>(schedule);
  L.p.entries = entries;
  L.p.n_entries = n_entries;
  for (int s = 0; s < nseg; ++s) L.p.seg_out[s] = static_cast<__nv_bfloat16*>(seg_out[s]);
  return launch<true>(L, static_cast<unsigned>(n_schedule), heads, batch, stream);
}

extern "C" int erd_attn_fwd_cross_bf16(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t k_token_stride, int64_t k_head_stride, int64_t k_batch_stride,
    int64_t v_token_stride, int64_t v_head_stride, int64_t v_batch_stride, int batch, int heads,
    int q_len, int kv_len, const int32_t* kv_valid, int head_dim, float softmax_scale, void* out,
    int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride, int* status,
    void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) return kErrNullPointer;
  if (head_dim != kHeadDim || batch <= 0 || batch > kMaxCrossBatch || heads <= 0 ||
      heads > 65535 || q_len <= 0 || kv_len <= 0)
    return kErrBadShape;
  if (kv_valid != nullptr) {
    for (int b = 0; b < batch; ++b)
      if (kv_valid[b] <= 0 || kv_valid[b] > kv_len) return kErrBadShape;
  }
  // Queries through the common checks (their own tiling); keys get their own maps.
  Launch L;
  if (int rc = prepare(q, q, q, q_token_stride, q_head_stride, q_batch_stride, 0, q_token_stride,
                       q_head_stride, q_batch_stride, 0, q_token_stride, q_head_stride,
                       q_batch_stride, 0, batch, heads, q_len, 1, nullptr, head_dim,
                       softmax_scale, out, o_token_stride, o_head_stride, o_batch_stride, 0,
                       status, &L))
    return rc;
  if (!aligned16(k) || !aligned16(v) ||
      !strides_ok(k_token_stride, k_head_stride, k_batch_stride, 0) ||
      !strides_ok(v_token_stride, v_head_stride, v_batch_stride, 0))
    return kErrMisaligned;
  if (make_operand_map(&L.tk, k, kv_len, heads, batch, 1, k_token_stride, k_head_stride,
                       k_batch_stride, 0) ||
      make_operand_map(&L.tv, v, kv_len, heads, batch, 1, v_token_stride, v_head_stride,
                       v_batch_stride, 0))
    return kErrTensorMap;
  L.p.kv_tiles_per_seg = (kv_len + kBlockN - 1) / kBlockN;
  L.p.kv_tiles = L.p.kv_tiles_per_seg;
  L.p.kv_per_batch = 1;
  for (int b = 0; b < kMaxCrossBatch; ++b)
    L.p.kv_valid[b] = b < batch ? (kv_valid != nullptr ? kv_valid[b] : kv_len) : 0;
  return launch<false>(L, static_cast<unsigned>((L.p.q_tiles + 1) / 2), heads, batch, stream);
}

extern "C" size_t erd_ring_state_bytes(int batch, int heads, int seg_len, int q_nseg) {
  if (batch <= 0 || heads <= 0 || seg_len <= 0 || q_nseg <= 0 || q_nseg > kMaxSegments) return 0;
  return static_cast<size_t>(ring_state_floats(batch, heads, seg_len, q_nseg)) * sizeof(float);
}

extern "C" int erd_attn_fwd_ring_bf16(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int q_nseg,
    const int32_t* q_seg_lens, int kv_seg_len, int kv_nseg, const int32_t* kv_seg_lens,
    int head_dim, float softmax_scale, void* out, int64_t o_token_stride, int64_t o_head_stride,
    int64_t o_batch_stride, int64_t o_seg_stride, void* const* seg_out, void* state,
    size_t state_bytes, int state_mode, int* status, void* stream) {
  if (state_mode < 0 || state_mode > (kStateRead | kStateWrite)) return kErrBadShape;
  const bool writes_output = (state_mode & kStateWrite) == 0;
  if (kv_seg_lens == nullptr) return kErrNullPointer;
  if (kv_nseg <= 0 || kv_nseg > kMaxSegments || q_nseg <= 0 || q_nseg > kMaxSegments ||
      kv_seg_len <= 0)
    return kErrBadShape;
  for (int s = 0; s < kv_nseg; ++s)
    if (kv_seg_lens[s] <= 0 || kv_seg_lens[s] > kv_seg_len) return kErrBadShape;
  if (writes_output && out == nullptr && seg_out == nullptr) return kErrNullPointer;
  if (seg_out != nullptr) {
    for (int s = 0; s < q_nseg; ++s) {
      if (seg_out[s] == nullptr) return kErrNullPointer;
      if (!aligned16(seg_out[s])) return kErrMisaligned;
    }
  }
  // The output pointer goes through the common checks; with the state written
  // instead (or per-segment bases) it is never dereferenced.
  const void* out_checked = out != nullptr ? out : (seg_out != nullptr ? seg_out[0] : q);
  Launch L;
  if (int rc = prepare(q, k, v, q_token_stride, q_head_stride, q_batch_stride, q_seg_stride,
                       k_token_stride, k_head_stride, k_batch_stride, k_seg_stride,
                       v_token_stride, v_head_stride, v_batch_stride, v_seg_stride, batch, heads,
                       seg_len, q_nseg, q_seg_lens, head_dim, softmax_scale,
                       const_cast<void*>(out_checked), o_token_stride, o_head_stride,
                       o_batch_stride, o_seg_stride, status, &L))
    return rc;
  if (make_operand_map(&L.tk, k, kv_seg_len, heads, batch, kv_nseg, k_token_stride,
                       k_head_stride, k_batch_stride, k_seg_stride) ||
      make_operand_map(&L.tv, v, kv_seg_len, heads, batch, kv_nseg, v_token_stride,
                       v_head_stride, v_batch_stride, v_seg_stride))
    return kErrTensorMap;
  const long long kv_tiles_per_seg = (kv_seg_len + kBlockN - 1) / kBlockN;
  if (kv_tiles_per_seg * kv_nseg > (1LL << 24)) return kErrTooLarge;
  L.p.kv_tiles_per_seg = static_cast<int>(kv_tiles_per_seg);
  L.p.kv_tiles = static_cast<int>(kv_tiles_per_seg * kv_nseg);
  for (int s = 0; s < kMaxSegments; ++s) L.p.kv_seg_lens[s] = s < kv_nseg ? kv_seg_lens[s] : 0;
  if (seg_out != nullptr)
    for (int s = 0; s < q_nseg; ++s) L.p.seg_out[s] = static_cast<__nv_bfloat16*>(seg_out[s]);
  const unsigned ctas = static_cast<unsigned>((L.p.q_tiles + 1) / 2);
  if (state_mode == 0) return launch<false>(L, ctas, heads, batch, stream);
  if (state == nullptr) return kErrNullPointer;
  if (!aligned16(state)) return kErrMisaligned;
  if (state_bytes < erd_ring_state_bytes(batch, heads, seg_len, q_nseg)) return kErrTooLarge;
  L.p.state = static_cast<float*>(state);
  L.p.state_mode = state_mode;
  return launch<false, true>(L, ctas, heads, batch, stream);
}
