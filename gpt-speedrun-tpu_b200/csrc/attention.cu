// Causal flash attention (head_dim 64) on the Blackwell tensor cores.
//
// Both kernels are persistent: one CTA per SM walks a list of work items and
// keeps its shared-memory rings and TMEM handshakes running from one item into
// the next (see the item comments at each kernel).
// Forward (attn_fwd_tc): work item = (pair of 128-query tiles, batch*head).
// 11 warps, all of TMEM: warp 0 loads both Q tiles of an item (two item
// slots) and 128-key K/V blocks into a 4-stage ring (4-D tensor maps over
// (e, t, h, b), so any [b, t, h, e] strides work and rows past the sequence
// end arrive as zeros); one MMA thread per tile issues S_x = Q_x K^T (128x128
// fp32 in TMEM) and O_x += P_x V (P_x read from TMEM, V an MN-major shared
// operand); two softmax warpgroups own one tile each (thread = query row =
// TMEM lane) and turn S_x into bf16 P_x in TMEM, so the two tiles ping-pong:
// while one warpgroup exponentiates, the tensor core runs the other tile's
// MMAs.
// Backward (attn_bwd_tc): work item = (128-key tile, batch*head), looping over
// 64-query tiles from the diagonal down. 23 warps: TMA (K, V per item in two
// slots; Q/dO into a 4-stage ring with the tile's lse/delta copied in by
// cp.async), a scores MMA thread (S^T = K Q^T and dP^T = V dO^T into one
// of three 128-column TMEM buffers, as far ahead as the buffers allow), a
// gradient MMA thread (dV += P^T dO and dK += dS^T Q with P^T / dS^T read
// straight from TMEM; dQ = dS K per pair of tiles, dS^T read MN-major from a
// shared-memory ring), 16 softmax warps that take every tile together
// (thread = key row, 16 query columns per warp: P^T = exp2(S^T c - lse),
// dS^T = P^T (dP^T - delta), written over the warp's own S^T columns as bf16
// pairs), and four dQ warps. Two issuing threads keep the tensor pipe fed
// while either waits on a barrier. The dQ warps read each pair's dQ out of
// TMEM as soon as its MMA completes and reduce it into an fp32 accumulator by
// TMA; at the end of an item they also write dK and dV.
// q and k arrive already rotated (RoPE runs in the QKV projection epilogue);
// with RoPE tables the backward rotates dq and dk back so they are gradients
// of the unrotated inputs.
// Every mbarrier wait is bounded (common.cuh). Semantics follow
// rig/kernels/tpu_flash_attention.py:171-207 (fp32 statistics, bf16 P).
#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace gptb200 {

static __device__ int g_attn_error;


constexpr int HD = 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnParams {
  int B, H, T;
  float scale;
  // output / saved tensors
  bf16* o;
  int64_t osb, osh, ost;
  float* lse;          // [B, H, T], natural log
  const bf16* dout;
  const float* delta;  // [B, H, T]
  float* dq_acc;       // [B, H, T, 64] fp32
  bf16* dk;
  bf16* dv;
  int64_t sb, sh, st;  // q/k/v (and dq/dk/dv) strides
  const bf16* rcos;    // RoPE tables [T, 32] or null
  const bf16* rsin;
  const int* seg;      // document segment ids [B, T] or null (causal only)
  unsigned* sched;     // this launch's work counter {next item, finished CTAs}
};

__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return (uint32_t)(row * 128 + (((chunk ^ (row & 7)) & 7) << 4));
}

// Rotates 4 interleaved pairs (one 16-byte chunk holding elements 8c..8c+7 of
// position t) by the transpose of the RoPE rotation.
__device__ __forceinline__ void rope_back(float* v, const bf16* rcos, const bf16* rsin, int t,
                                          int c) {
  const bf16* cs = rcos + (int64_t)t * (HD / 2) + c * 4;
  const bf16* sn = rsin + (int64_t)t * (HD / 2) + c * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float cv = __bfloat162float(cs[j]), sv = __bfloat162float(sn[j]);
    float ge = v[2 * j], go = v[2 * j + 1];
    v[2 * j] = ge * cv + go * sv;
    v[2 * j + 1] = -ge * sv + go * cv;
  }
}

// ------------------------------------------------------------------ segments
// Document masking (rig/kernels/tpu_flash_attention.py:171-207 with segment
// ids): a query sees a key only if the key is not later and both carry the same
// segment id. Each CTA first reduces the ids of every 64-position chunk of its
// sequence to a (min, max) range in shared memory; a key block and a query tile
// whose ranges are disjoint never meet, and when both ranges are one and the
// same single id no per-element test is needed. Both hold for any ids; with the
// nondecreasing ids of document_segments (rig/attention.py:205-208) the blocks
// before a query tile's first document are exactly the ones skipped.
constexpr int kSegChunk = 64;
constexpr int kMaxSegChunks = 1024;  // segment ids are supported up to T = 65536

__device__ __forceinline__ int2 rng_merge(int2 a, int2 b) {
  return make_int2(min(a.x, b.x), max(a.y, b.y));
}
__device__ __forceinline__ bool rng_meet(int2 a, int2 b) { return a.x <= b.y && b.x <= a.y; }
__device__ __forceinline__ bool rng_single(int2 a, int2 b) {
  return a.x == a.y && b.x == b.y && a.x == b.x;
}

// tab[c - c0] = (min, max) id of positions [64c, 64c + 64) of seg_row for
// chunks c0 <= c < c1; positions past T are ignored (an empty chunk is
// (INT_MAX, INT_MIN)). Every thread of the CTA takes part.
__device__ void seg_chunk_ranges(const int* __restrict__ seg_row, int T, int c0, int c1,
                                 int2* tab) {
  const int warps = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = c0 + w; c < c1; c += warps) {
    int mn = INT_MAX, mx = INT_MIN;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int t = c * kSegChunk + u * 32 + lane;
      if (t < T) {
        const int v = seg_row[t];
        mn = min(mn, v);
        mx = max(mx, v);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) tab[c - c0] = make_int2(mn, mx);
  }
}

// Range of the ids in table entries [c, c + n) (entries at or past nch are empty).
__device__ __forceinline__ int2 seg_range(const int2* tab, int nch, int c, int n) {
  int2 r = make_int2(INT_MAX, INT_MIN);
  for (int i = c; i < c + n && i < nch; ++i) r = rng_merge(r, tab[i]);
  return r;
}

// Dynamic work distribution of the persistent kernels: the TMA warp of each
// CTA takes the next item index from a per-launch counter (the items are laid
// out head by head, heaviest first within a head, so the items in flight at
// once cover a few heads whose K/V or Q/dO tiles come from DRAM about once and
// are then served from L2, and a CTA that finishes early takes more work).
// The counters live in a small device array of slots; each launch gets its own
// slot (so launches that overlap on the GPU do not share one) and the last CTA
// to finish puts the slot back to zero.
constexpr int kSchedSlots = 64;
__device__ unsigned g_attn_sched[2][kSchedSlots][2];

// Called by the whole producer warp: the next item index (lane 0 fetches).
__device__ __forceinline__ int next_item(unsigned* sched, int lane) {
  int v = 0;
  if (lane == 0) v = (int)atomicAdd(sched, 1u);
  return __shfl_sync(0xffffffffu, v, 0);
}

// Called by thread 0 of each CTA after all of the CTA's work: the last CTA
// resets the launch's counter slot.
__device__ __forceinline__ void sched_finish(unsigned* sched) {
  __threadfence();
  if (atomicAdd(sched + 1, 1u) == gridDim.x - 1) {
    sched[0] = 0;
    sched[1] = 0;
    __threadfence();
  }
}

// ------------------------------------------------------------------ forward
// Persistent: one CTA per SM walks work items (pair of 128-query tiles pr,
// batch*head bh), item = bh * npair + (npair-1-pr), handed out by next_item.
// Every role keeps running
// counters across items, so the K/V ring and the per-tile S/P/O handshakes
// flow from one item into the next; Q tiles are double-buffered per item.
constexpr int FQ = 128;                 // queries per tile (TMEM lanes); two tiles per item
constexpr int FK = 128;                 // keys per K/V block
constexpr int Q_BYTES = FQ * 128;       // 128 rows x 64 bf16
constexpr int KV_BYTES = FK * 128;      // 128 rows x 64 bf16
constexpr int kKvStages = 4;
constexpr int kFwdMma1Warp = 10;       // MMA thread of tile 1 (warp 1 serves tile 0)
constexpr int kFwdThreads = 32 * 11;
constexpr int kFwdItemUsers = 2 + 8;   // both MMA threads, the 8 softmax warps

// Item slot written by the TMA warp: pair, batch*head, key blocks the pair
// visits (tile 0 the first n0 of them), whether tile 1 lies inside the sequence.
struct FwdItem {
  int pr, bh, nkv, n0, has1, pad0, pad1, pad2;
};

template <bool SEG>
struct FwdSmem {
  static constexpr int Q = 0;                                 // 2 item slots x 2 tiles
  static constexpr int K = Q + 4 * Q_BYTES;                   // kKvStages
  static constexpr int V = K + kKvStages * KV_BYTES;          // kKvStages
  static constexpr int ITEM = V + kKvStages * KV_BYTES;       // 2 FwdItem slots
  // segment ids only: per slot, (min, max) id per 64-position chunk and the
  // key blocks the pair visits; per tile, two buffers of a block's key ids
  static constexpr int SEGTAB = ITEM + 64;
  static constexpr int BLOCKS = SEGTAB + (SEG ? 2 * kMaxSegChunks * 8 : 0);
  static constexpr int KSEG = BLOCKS + (SEG ? 2 * (kMaxSegChunks / 2) * 4 : 0);
  static constexpr int BAR = KSEG + (SEG ? 2 * 2 * FK * 4 : 0);
  // the dynamic shared memory base is 1024-byte aligned (checked at entry)
  static constexpr int TOTAL = BAR + 256;
};

template <bool SEG>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using L = FwdSmem<SEG>;
  extern __shared__ __align__(1024) uint8_t smem_fwd[];
  uint8_t* sm = smem_fwd;
  if (smem_u32(sm) & 1023) {  // the layout needs 1024-byte aligned tiles: give up, flagged
    if (threadIdx.x == 0) {
      atomicCAS(&g_attn_error, 0, kErrSmemAlign);
      sched_finish(p.sched);
    }
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* q_full = bars + 0;                 // [2 item slots]
  uint64_t* q_empty = bars + 2;                // [2]
  uint64_t* kv_full = bars + 4;                // [kKvStages]
  uint64_t* kv_empty = kv_full + kKvStages;    // [kKvStages]
  uint64_t* s_full = kv_empty + kKvStages;     // [2 tiles]: S of the current block is in TMEM
  uint64_t* p_full = s_full + 2;               // [2]: P written to TMEM
  uint64_t* pv_done = p_full + 2;              // [2]: the tile's P.V MMA has completed
  uint64_t* s_free = pv_done + 2;              // [2]: S has been loaded into registers
  uint64_t* kseg_full = s_free + 2;            // [2 tiles][2]: a block's key ids are in smem
  uint64_t* item_full = kseg_full + 4;         // [2]
  uint64_t* item_empty = item_full + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  FwdItem* items = reinterpret_cast<FwdItem*>(sm + L::ITEM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int npair = (p.T + 2 * FQ - 1) / (2 * FQ);
  const int n_items = npair * BH;  // item = bh * npair + (npair - 1 - pair)
  int* err = &g_attn_error;
  auto segtab_of = [&](int slot) {
    return reinterpret_cast<int2*>(sm + L::SEGTAB) + slot * kMaxSegChunks;
  };
  // key block of list entry j of the item in `slot`
  auto kblock = [&](int slot, int j) -> int {
    if constexpr (SEG)
      return reinterpret_cast<const int*>(sm + L::BLOCKS)[slot * (kMaxSegChunks / 2) + j];
    else
      return j;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 2);  // released by each tile's MMA thread
      mbar_init(&item_full[s], 1);
      mbar_init(&item_empty[s], kFwdItemUsers);
    }
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 2);  // released by each tile's MMA thread
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);
      mbar_init(&pv_done[x], 1);
      mbar_init(&s_free[x], 4);
      mbar_init(&kseg_full[2 * x], FQ);
      mbar_init(&kseg_full[2 * x + 1], FQ);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // TMEM columns: S[2] (128 fp32 each) | O[2] (64 fp32) | P[2] (128 keys as bf16 pairs)
  const uint32_t tmem = *tmem_slot;
  auto tS = [&](int x) { return tmem + 128 * x; };
  auto tO = [&](int x) { return tmem + 256 + 64 * x; };
  auto tP = [&](int x) { return tmem + 384 + 64 * x; };

  if (warp == 0) {
    // Item producer: publishes each item's slot (with segment ids also the
    // chunk ranges and the key-block list), then loads its two Q tiles and its
    // K/V blocks into the ring.
    bool ok = true;
    int gk = 0;
    for (int ii = 0; ok; ++ii) {
      const int slot = ii & 1;
      const int item = next_item(p.sched, lane);
      if (!(ok = mbar_wait(&item_empty[slot], ((ii >> 1) & 1) ^ 1, abort_flag, err))) break;
      if (item >= n_items) {  // no more work: an empty slot ends every role's loop
        if (lane == 0) {
          items[slot].nkv = -1;
          mbar_arrive(&item_full[slot]);
        }
        break;
      }
      const int bh = item / npair, pr = npair - 1 - (item - bh * npair);
      const int b = bh / p.H, h = bh - b * p.H;
      const int q0 = pr * 2 * FQ;
      // tile x's diagonal key block is d0 + x; tile 1 of the last pair may lie
      // wholly past the sequence end
      const int d0 = q0 / FK;
      const int has1 = q0 + FQ < p.T;
      const int dmax = has1 ? d0 + 1 : d0;
      int nkv = dmax + 1, n0 = d0 + 1;
      if constexpr (SEG) {
        // The key blocks 0..dmax either query tile can see, in order. Both
        // tiles walk this one list (tile 0 its prefix up to d0); a block only
        // the other tile needs is fully masked for a tile, at most costing its
        // exps.
        const int* segrow = p.seg + (int64_t)b * p.T;
        int2* tab = segtab_of(slot);
        const int nch = min((p.T + kSegChunk - 1) / kSegChunk, 2 * (dmax + 1));
        for (int c = 0; c < nch; ++c) {
          int mn = INT_MAX, mx = INT_MIN;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int t = c * kSegChunk + u * 32 + lane;
            if (t < p.T) {
              const int v = segrow[t];
              mn = min(mn, v);
              mx = max(mx, v);
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          }
          if (lane == 0) tab[c] = make_int2(mn, mx);
        }
        __syncwarp();
        if (lane == 0) {
          int* bl = reinterpret_cast<int*>(sm + L::BLOCKS) + slot * (kMaxSegChunks / 2);
          const int2 qr0 = seg_range(tab, nch, 2 * d0, 2);
          const int2 qr1 = seg_range(tab, nch, 2 * d0 + 2, 2);
          int n = 0, n_le0 = 0;
          for (int j = 0; j <= dmax; ++j) {
            const int2 kr = seg_range(tab, nch, 2 * j, 2);
            if ((j <= d0 && rng_meet(kr, qr0)) || (has1 && rng_meet(kr, qr1))) {
              bl[n++] = j;
              if (j <= d0) ++n_le0;
            }
          }
          nkv = n;
          n0 = n_le0;
        }
        nkv = __shfl_sync(0xffffffffu, nkv, 0);
        n0 = __shfl_sync(0xffffffffu, n0, 0);
      }
      if (lane == 0) {
        items[slot] = FwdItem{pr, bh, nkv, n0, has1, 0, 0, 0};
        mbar_arrive(&item_full[slot]);
        if ((ok = mbar_wait(&q_empty[slot], ((ii >> 1) & 1) ^ 1, abort_flag, err))) {
          uint8_t* qd = sm + L::Q + slot * 2 * Q_BYTES;
          mbar_arrive_expect_tx(&q_full[slot], 2 * Q_BYTES);
          tma_load_4d(qd, &tmQ, &q_full[slot], 0, q0, h, b);
          tma_load_4d(qd + Q_BYTES, &tmQ, &q_full[slot], 0, q0 + FQ, h, b);
        }
        for (int j = 0; ok && j < nkv; ++j, ++gk) {
          const int s = gk % kKvStages;
          if (!(ok = mbar_wait(&kv_empty[s], ((gk / kKvStages) & 1) ^ 1, abort_flag, err))) break;
          mbar_arrive_expect_tx(&kv_full[s], 2 * KV_BYTES);
          const int key0 = kblock(slot, j) * FK;
          tma_load_4d(sm + L::K + s * KV_BYTES, &tmK, &kv_full[s], 0, key0, h, b);
          tma_load_4d(sm + L::V + s * KV_BYTES, &tmV, &kv_full[s], 0, key0, h, b);
        }
      }
      ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
    }
  } else if (warp == 1 || warp == kFwdMma1Warp) {
    // One MMA thread per tile: S_x = Q_x K_j^T (128 x 128 fp32) for the next
    // block as soon as the softmax holds S_x in registers, O_x += P_x V_j
    // once P_x is in TMEM. The two tiles progress independently; each walks
    // every block of the item's list and releases the ones it does not use.
    const int x = warp == 1 ? 0 : 1;
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc_bf16(128, FK, 0, 0);
      constexpr uint32_t idO = umma_idesc_bf16(128, HD, 0, 1);  // A = P in TMEM, B = V MN-major
      bool ok = true;
      int gk = 0, jx = 0, ii = 0;  // ring block, this tile's running block, item
      for (; ok; ++ii) {
        const int slot = ii & 1;
        if (!(ok = mbar_wait(&item_full[slot], (ii >> 1) & 1, abort_flag, err))) break;
        const FwdItem inf = items[slot];
        if (inf.nkv < 0) break;  // no more items
        const int nb = x == 0 ? inf.n0 : (inf.has1 ? inf.nkv : 0);
        const uint32_t sQ = smem_u32(sm + L::Q + (slot * 2 + x) * Q_BYTES);
        auto issue_s = [&](int s) {
          const uint32_t sK = smem_u32(sm + L::K + s * KV_BYTES);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k)
            umma_bf16(tS(x), umma_smem_desc(sQ + k * 32, 16, 1024),
                      umma_smem_desc(sK + k * 32, 16, 1024), idS, k > 0);
          umma_commit(&s_full[x]);
        };
        if (nb > 0) {
          // S of the item's first block: Q loaded, the block loaded, and the
          // previous item's last S taken out of TMEM by the softmax
          ok = mbar_wait(&q_full[slot], (ii >> 1) & 1, abort_flag, err) &&
               mbar_wait(&kv_full[gk % kKvStages], (gk / kKvStages) & 1, abort_flag, err) &&
               (jx == 0 || mbar_wait(&s_free[x], (jx - 1) & 1, abort_flag, err));
          if (!ok) break;
          tc_fence_after();
          issue_s(gk % kKvStages);
        }
        for (int j = 0; ok && j < inf.nkv; ++j) {
          const int s = (gk + j) % kKvStages;
          if (j >= nb) {  // a block this tile skips: release it once it has arrived
            if (!(ok = mbar_wait(&kv_full[s], ((gk + j) / kKvStages) & 1, abort_flag, err))) break;
            mbar_arrive(&kv_empty[s]);
            continue;
          }
          const int jj = jx + j;  // running block index of this tile
          if (j + 1 < nb) {
            const int s1 = (gk + j + 1) % kKvStages;
            if (!(ok = mbar_wait(&kv_full[s1], ((gk + j + 1) / kKvStages) & 1, abort_flag, err)) ||
                !(ok = mbar_wait(&s_free[x], jj & 1, abort_flag, err)))
              break;
            tc_fence_after();
            issue_s(s1);
          }
          if (!(ok = mbar_wait(&p_full[x], jj & 1, abort_flag, err))) break;
          tc_fence_after();
          const uint32_t sV = smem_u32(sm + L::V + s * KV_BYTES);
          // O_x += P_x V_j, P read from TMEM (keys 16k..16k+15 at column 8k)
#pragma unroll
          for (int k = 0; k < FK / 16; ++k)
            umma_bf16_ts(tO(x), tP(x) + k * 8, umma_smem_desc(sV + k * 2048, KV_BYTES, 1024), idO,
                         (j > 0 || k > 0));
          umma_commit(&pv_done[x]);
          umma_commit(&kv_empty[s]);
        }
        if (!ok) break;
        // the item's Q tile is free once its last S MMA has completed
        if (nb > 0)
          umma_commit(&q_empty[slot]);
        else
          mbar_arrive(&q_empty[slot]);
        mbar_arrive(&item_empty[slot]);
        gk += inf.nkv;
        jx += nb;
      }
    }
  } else if (warp < kFwdMma1Warp) {
    // Softmax warpgroup x (warps 2-5: tile 0, 6-9: tile 1); thread = query
    // row r of the tile (TMEM lane r). Per block: the S row into registers,
    // its max, then exp + row sum + P, with a running max that is only raised
    // when the row max grows by more than 2^8; O is then rescaled in TMEM.
    // Otherwise the stale max is exact because O and the row sum share it.
    const int x = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float c = p.scale * kLog2e;
    int* kseg = reinterpret_cast<int*>(sm + L::KSEG) + x * 2 * FK;
    int nseg = 0;  // blocks of this tile that needed the per-element test so far
    bool ok = true;
    int jx = 0, ii = 0;
    for (; ok; ++ii) {
      const int slot = ii & 1;
      if (!(ok = mbar_wait(&item_full[slot], (ii >> 1) & 1, abort_flag, err))) break;
      const FwdItem inf = items[slot];
      if (inf.nkv < 0) break;  // no more items
      const int nb = x == 0 ? inf.n0 : (inf.has1 ? inf.nkv : 0);
      const int bh = inf.bh, b = bh / p.H, h = bh - b * p.H;
      const int q0 = inf.pr * 2 * FQ;
      const int d0 = q0 / FK;
      const int qrow = q0 + x * FQ + r;
      const int* segrow = SEG ? p.seg + (int64_t)b * p.T : nullptr;
      const int2* segtab = SEG ? segtab_of(slot) : nullptr;
      const int nch = min((p.T + kSegChunk - 1) / kSegChunk, 2 * (d0 + inf.has1 + 1));
      // this row's segment id (rows past T take an id no key has)
      const int sq = segrow ? (qrow < p.T ? segrow[qrow] : INT_MIN) : 0;
      const int2 qrng = segrow ? seg_range(segtab, nch, 2 * (d0 + x), 2) : make_int2(0, 0);
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nb && ok; ++j) {
        const int jj = jx + j;
        if (!(ok = mbar_wait(&s_full[x], jj & 1, abort_flag, err))) break;
        tc_fence_after();
        const int jb = kblock(slot, j);
        const bool diag = (jb == d0 + x);  // keys past the query (and past T) are masked
        // Per-element segment test unless keys and queries all share one id;
        // the block's key ids then come through shared memory (double-buffered,
        // one mbarrier handshake across the warpgroup).
        const bool segmask = segrow && !rng_single(seg_range(segtab, nch, 2 * jb, 2), qrng);
        const int* ks = kseg + (nseg & 1) * FK;
        if (segmask) {
          const int key = jb * FK + r;
          kseg[(nseg & 1) * FK + r] = key < p.T ? segrow[key] : INT_MAX;
          mbar_arrive(&kseg_full[2 * x + (nseg & 1)]);
          if (!(ok = mbar_wait(&kseg_full[2 * x + (nseg & 1)], (nseg >> 1) & 1, abort_flag, err)))
            break;
          ++nseg;
        }
        // The whole 128-column S row in one batch of TMEM loads, then S_x is
        // handed back so the next block's scores overlap this block's exps.
        uint32_t v[FK];
#pragma unroll
        for (int cc = 0; cc < FK / 32; ++cc) tmem_ld32_nw(tS(x) + lane_off + cc * 32, v + 32 * cc);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[x]);
        // Row max of the raw scores (c > 0 commutes with the max), eight
        // independent chains; on the diagonal block keys past the query are out.
        float m8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) m8[u] = -INFINITY;
        auto visible = [&](int i) { return (!diag || i <= r) && (!segmask || ks[i] == sq); };
        if (diag || segmask) {
#pragma unroll
          for (int i = 0; i < FK; i += 2)
            m8[(i >> 1) & 7] = fmax3(m8[(i >> 1) & 7], visible(i) ? __uint_as_float(v[i]) : -INFINITY,
                                     visible(i + 1) ? __uint_as_float(v[i + 1]) : -INFINITY);
        } else {
#pragma unroll
          for (int i = 0; i < FK; i += 2)
            m8[(i >> 1) & 7] =
                fmax3(m8[(i >> 1) & 7], __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
        }
        const float mx =
            fmaxf(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], fmaxf(m8[5], fmaxf(m8[6], m8[7])))) * c;
        // The rescale decision is made per warp: the TMEM loads/stores of O are
        // warp-collective and must not run in a divergent branch. Rows whose
        // max did not move rescale by exactly 1.
        const bool rescale = __any_sync(0xffffffffu, mx > m_used + 8.0f);
        float alpha = 1.f;
        if (rescale) {
          // 0 on a row's first visible block (m_used = -inf); a row with no
          // visible key yet (document masking) keeps its -inf max and alpha 1
          const float m_new = fmaxf(m_used, mx);
          alpha = m_new == -INFINITY ? 1.f : ex2(m_used - m_new);
          m_used = m_new;
        }
        // P = exp2(s*c - m) packed to bf16 pairs in registers (the S registers
        // die as P is produced); four packed partial row sums.
        const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_used, -m_used);
        float2 acc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[u] = make_float2(0.f, 0.f);
        uint32_t pk[FK / 2];
#pragma unroll
        for (int i = 0; i < FK; i += 2) {
          const float2 t = ffma2(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), c2, nm2);
          float p0 = ex2(t.x), p1 = ex2(t.y);
          if (diag || segmask) {
            if (!visible(i)) p0 = 0.f;
            if (!visible(i + 1)) p1 = 0.f;
          }
          acc[(i >> 1) & 3] = fadd2(acc[(i >> 1) & 3], make_float2(p0, p1));
          pk[i / 2] = pack_bf16x2(p0, p1);
        }
        const float2 s01 = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
        const float sum = s01.x + s01.y;
        // P and O of the previous block must have been consumed by its P.V
        // MMA (the previous item's last block was waited for at its end).
        if (j > 0) {
          if (!(ok = mbar_wait(&pv_done[x], (jj - 1) & 1, abort_flag, err))) break;
          tc_fence_after();
        }
#pragma unroll
        for (int g = 0; g < FK / 16; ++g) tmem_st8_nw(tP(x) + lane_off + g * 8, pk + 8 * g);
        l = l * alpha + sum;
        if (rescale && j > 0) {
          float o[32];
#pragma unroll
          for (int cc = 0; cc < HD / 32; ++cc) {
            tmem_ld32(tO(x) + lane_off + cc * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO(x) + lane_off + cc * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
      if (ok && nb > 0) {
        if (!(ok = mbar_wait(&pv_done[x], (jx + nb - 1) & 1, abort_flag, err))) break;
        tc_fence_after();
        const float inv = 1.f / l;
        float o[32];
        bf16* orow = p.o + b * p.osb + h * p.osh + (int64_t)qrow * p.ost;
#pragma unroll
        for (int cc = 0; cc < HD / 32; ++cc) {
          tmem_ld32(tO(x) + lane_off + cc * 32, o);
          if (qrow < p.T) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 q;
              q.x = pack_bf16x2(o[8 * g] * inv, o[8 * g + 1] * inv);
              q.y = pack_bf16x2(o[8 * g + 2] * inv, o[8 * g + 3] * inv);
              q.z = pack_bf16x2(o[8 * g + 4] * inv, o[8 * g + 5] * inv);
              q.w = pack_bf16x2(o[8 * g + 6] * inv, o[8 * g + 7] * inv);
              *reinterpret_cast<uint4*>(orow + cc * 32 + 8 * g) = q;
            }
          }
        }
        if (qrow < p.T) p.lse[(int64_t)bh * p.T + qrow] = (m_used + __log2f(l)) * kLn2;
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
      jx += nb;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) sched_finish(p.sched);
}

// ------------------------------------------------------------------ backward
// Persistent: one CTA per SM walks work items (key tile kt, batch*head bh),
// item = bh * nkt + kt, handed out by next_item. Every role
// walks the same item list and keeps running tile / query-pair counters across
// items, so the rings (Q/dO stages, TMEM score buffers, dS^T slots, dQ pairs)
// flow from one item into the next without draining: while the last tiles of
// an item finish, the TMA warp already holds the next item's K/V (two K/V
// slots) and the scores MMA thread computes its first scores.
constexpr int BT = 128;                 // keys per item (TMEM lanes)
constexpr int BQ = 64;                  // queries per inner tile
constexpr int BT_BYTES = BT * 128;      // 128 rows x 64 bf16
constexpr int BQ_BYTES = BQ * 128;      // 64 rows x 64 bf16
constexpr int kBwdSmWarps = 16;         // softmax warps: four per TMEM lane quadrant
// The softmax warps form GROUPS groups (a kernel template parameter) that take
// alternate tiles; a warp of a group covers 64 / (group warps / 4) query
// columns of its tile. One group (every warp on every tile) has the shortest
// latency per tile and wins at T = 1024, where items are a few tiles long;
// two groups overlap consecutive tiles and win on long sequences.
constexpr int kBwdScoreWarp = 2 + kBwdSmWarps;  // issues the S^T / dP^T MMAs
constexpr int kBwdFlushWarp = kBwdScoreWarp + 1;  // first of four dQ read-out warps
constexpr int kBwdThreads = 32 * (kBwdFlushWarp + 4);
// Arrivals that release an item slot: both MMA threads, the softmax warps and
// the dQ warps.
constexpr int kBwdItemUsers = 2 + kBwdSmWarps + 4;

// Item slot written by the TMA warp: key tile, batch*head, number of 64-query
// tiles (always even: an odd count gets one tile past the sequence end, whose
// rows load as zeros and carry no probability, so query pairs never straddle
// two items).
struct BwdItem {
  int kt, bh, nq, pad;
};

template <bool SEG>
struct BwdSmem {
  static constexpr int kQStages = SEG ? 2 : 4;          // Q / dO tile ring
  static constexpr int kStatBytes = SEG ? 768 : 512;    // per stage: lse, delta (, segment ids)
  static constexpr int KV = 0;                          // 2 slots x (K, V)
  static constexpr int Q = KV + 4 * BT_BYTES;           // kQStages tiles
  static constexpr int DO = Q + kQStages * BQ_BYTES;    // kQStages tiles
  static constexpr int DST = DO + kQStages * BQ_BYTES;  // ring of 4 dS^T tiles [128 keys x 64 queries]
  static constexpr int DQS = DST + 4 * BT_BYTES;        // dQ staging: 4 warps x 2 x (32 x 32 fp32)
  // per Q/dO stage, the tile's query statistics copied in by the producer
  // warp: 64 x lse, 64 x delta, 64 segment ids (zeros past the sequence end)
  static constexpr int STAT = DQS + 8 * 4096;
  static constexpr int ITEM = STAT + kQStages * kStatBytes;  // 2 BwdItem slots
  // segment ids only: per slot, (min, max) id per 64-position chunk from k0
  // and the list of query tiles that can see the key tile
  static constexpr int SEGTAB = ITEM + 32;
  static constexpr int QLIST = SEGTAB + (SEG ? 2 * kMaxSegChunks * 8 : 0);
  static constexpr int BAR = QLIST + (SEG ? 2 * kMaxSegChunks * 4 : 0);
  // the dynamic shared memory base is 1024-byte aligned (checked at entry)
  static constexpr int TOTAL = BAR + 272;
};

template <bool SEG, int GROUPS>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                const __grid_constant__ CUtensorMap tmDQ, const AttnParams p) {
  using L = BwdSmem<SEG>;
  constexpr int kQS = L::kQStages;
  constexpr int kBwdSmGroups = GROUPS;
  constexpr int kBwdGroupWarps = kBwdSmWarps / kBwdSmGroups;
  constexpr int kBwdWarpCols = 64 / (kBwdGroupWarps / 4);
  extern __shared__ __align__(1024) uint8_t smem_bwd[];
  uint8_t* sm = smem_bwd;
  if (smem_u32(sm) & 1023) {  // the layout needs 1024-byte aligned tiles: give up, flagged
    if (threadIdx.x == 0) {
      atomicCAS(&g_attn_error, 0, kErrSmemAlign);
      sched_finish(p.sched);
    }
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* kv_full = bars + 0;       // [2] K/V slot loaded
  uint64_t* kv_empty = bars + 2;      // [2] every MMA of the slot's item has completed
  uint64_t* q_full = bars + 4;        // [4]
  uint64_t* q_empty = bars + 8;       // [4]
  uint64_t* s_full = bars + 12;       // [3]: S^T and dP^T of a tile are in TMEM buffer b
  uint64_t* p_full = bars + 15;       // [3]: P^T, dS^T of a tile written (TMEM buffer b, smem ring)
  uint64_t* done = bars + 18;         // [4]: every MMA issued up to the end of tile g has completed
  uint64_t* dq_full = bars + 22;      // [2]: dQ of query pair J is in TMEM
  uint64_t* dq_free = bars + 24;      // [2]: ... and has been read out
  uint64_t* fin = bars + 26;          // an item's dK / dV are complete in TMEM
  uint64_t* acc_free = bars + 27;     // ... and have been read out
  uint64_t* item_full = bars + 28;    // [2]
  uint64_t* item_empty = bars + 30;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 32);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  BwdItem* items = reinterpret_cast<BwdItem*>(sm + L::ITEM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int n_items = ((p.T + BT - 1) / BT) * BH;  // item = bh * nkt + kt
  int* err = &g_attn_error;
  // query tile (64-position index past k0) of list entry `it` of the item in `slot`
  auto qtile = [&](int slot, int it) -> int {
    if constexpr (SEG)
      return reinterpret_cast<const int*>(sm + L::QLIST)[slot * kMaxSegChunks + it];
    else
      return it;
  };
  auto segtab_of = [&](int slot) {
    return reinterpret_cast<int2*>(sm + L::SEGTAB) + slot * kMaxSegChunks;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&item_full[s], 1);
      mbar_init(&item_empty[s], kBwdItemUsers);
      mbar_init(&dq_full[s], 1);
      mbar_init(&dq_free[s], 4);
    }
    for (int s = 0; s < kQS; ++s) {
      mbar_init(&q_full[s], 33);  // the Q/dO TMA and the 32 lanes' statistics copies
      mbar_init(&q_empty[s], 2);  // the scores MMAs and the gradient MMAs of the tile
    }
    for (int s = 0; s < 3; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], kBwdGroupWarps);
    }
    for (int s = 0; s < 4; ++s) mbar_init(&done[s], 1);
    mbar_init(fin, 1);
    mbar_init(acc_free, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // TMEM columns: three tile buffers of 128 columns, then dV | dK. In buffer
  // b, columns [0, 64) receive S^T and [64, 128) dP^T (fp32, lane = key). The
  // softmax writes P^T and dS^T as bf16 pairs over the S^T half (query group
  // cg = 16 queries: columns 16 cg + [0, 8) for P^T, 16 cg + [8, 16) for
  // dS^T); the dP^T half then holds dQ when the tile closes a query pair.
  const uint32_t tmem = *tmem_slot;
  const uint32_t tDV = tmem + 384, tDK = tmem + 448;
  auto tBuf = [&](int bb) { return tmem + 128 * bb; };

  if (warp == 0) {
    // Item producer: publishes each item's slot (and, with segment ids, its
    // chunk ranges and query-tile list), then loads its K/V and Q/dO tiles.
    bool ok = true;
    int g = 0;
    for (int ii = 0; ok; ++ii) {
      const int slot = ii & 1;
      const int item = next_item(p.sched, lane);
      if (!(ok = mbar_wait(&item_empty[slot], ((ii >> 1) & 1) ^ 1, abort_flag, err))) break;
      if (item >= n_items) {  // no more work: an empty slot ends every role's loop
        if (lane == 0) {
          items[slot].nq = -1;
          mbar_arrive(&item_full[slot]);
        }
        break;
      }
      const int nkt = (p.T + BT - 1) / BT;
      const int bh = item / nkt, kt = item - bh * nkt;
      const int b = bh / p.H, h = bh - b * p.H;
      const int k0 = kt * BT;
      const int nq_all = (p.T - k0 + BQ - 1) / BQ;  // 64-query tiles from the diagonal on
      int nq = nq_all;
      if constexpr (SEG) {
        // (min, max) segment id per 64-position chunk from k0, then the query
        // tiles whose ids can meet this key tile's, in order
        const int* segrow = p.seg + (int64_t)b * p.T;
        int2* tab = segtab_of(slot);
        const int nch = (p.T + kSegChunk - 1) / kSegChunk - 2 * kt;
        for (int c = 0; c < nch; ++c) {
          int mn = INT_MAX, mx = INT_MIN;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int t = (2 * kt + c) * kSegChunk + u * 32 + lane;
            if (t < p.T) {
              const int v = segrow[t];
              mn = min(mn, v);
              mx = max(mx, v);
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          }
          if (lane == 0) tab[c] = make_int2(mn, mx);
        }
        __syncwarp();
        if (lane == 0) {
          int* ql = reinterpret_cast<int*>(sm + L::QLIST) + slot * kMaxSegChunks;
          const int2 kr = seg_range(tab, nch, 0, 2);
          int n = 0;
          for (int it = 0; it < nq_all; ++it)
            if (rng_meet(seg_range(tab, nch, it, 1), kr)) ql[n++] = it;
          if (n & 1) ql[n++] = nq_all;  // past the sequence end: no probability
          nq = n;
        }
        nq = __shfl_sync(0xffffffffu, nq, 0);
      } else {
        nq += nq & 1;
      }
      if (lane == 0) {
        items[slot] = BwdItem{kt, bh, nq, 0};
        mbar_arrive(&item_full[slot]);
        const int kvs = ii & 1;
        ok = mbar_wait(&kv_empty[kvs], ((ii >> 1) & 1) ^ 1, abort_flag, err);
        if (ok) {
          uint8_t* kv = sm + L::KV + kvs * 2 * BT_BYTES;
          mbar_arrive_expect_tx(&kv_full[kvs], 2 * BT_BYTES);
          tma_load_4d(kv, &tmK, &kv_full[kvs], 0, k0, h, b);
          tma_load_4d(kv + BT_BYTES, &tmV, &kv_full[kvs], 0, k0, h, b);
        }
      }
      ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
      const float* Lg = p.lse + (int64_t)bh * p.T;
      const float* Dg = p.delta + (int64_t)bh * p.T;
      for (int it = 0; ok && it < nq; ++it, ++g) {
        const int s = g % kQS;
        const int qq = k0 + qtile(slot, it) * BQ;
        if (lane == 0) {
          ok = mbar_wait(&q_empty[s], ((g / kQS) & 1) ^ 1, abort_flag, err);
          if (ok) {
            mbar_arrive_expect_tx(&q_full[s], 2 * BQ_BYTES);
            tma_load_4d(sm + L::Q + s * BQ_BYTES, &tmQ, &q_full[s], 0, qq, h, b);
            tma_load_4d(sm + L::DO + s * BQ_BYTES, &tmDO, &q_full[s], 0, qq, h, b);
          }
        }
        if (!(ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0)) break;
        // the tile's statistics, copied asynchronously (each lane arrives on
        // the stage's barrier once its copies have landed)
        float* st = reinterpret_cast<float*>(sm + L::STAT + s * L::kStatBytes);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int cidx = lane + 32 * u, t = qq + cidx;
          const uint32_t nb = t < p.T ? 4u : 0u;
          const int tc = min(t, p.T - 1);
          cp_async_4(st + cidx, Lg + tc, nb);
          cp_async_4(st + 64 + cidx, Dg + tc, nb);
          if constexpr (SEG) cp_async_4(st + 128 + cidx, p.seg + (int64_t)b * p.T + tc, nb);
        }
        cp_async_mbar_arrive(&q_full[s]);
      }
    }
  } else if (warp == 1) {
    // Gradient MMAs of tile g once its softmax is done. This thread and the
    // scores thread (warp 18) issue independently: a thread that stops at a
    // barrier leaves the tensor pipe to the other one.
    if (lane == 0) {
      constexpr uint32_t idKN = umma_idesc_bf16(128, 64, 0, 1);  // dV, dK: A in TMEM, B MN-major
      constexpr uint32_t idMN = umma_idesc_bf16(128, 64, 1, 1);  // dQ: A, B MN-major
      bool ok = true;
      int g = 0, ii = 0;
      for (; ok; ++ii) {
        const int slot = ii & 1, kvs = ii & 1;
        if (!(ok = mbar_wait(&item_full[slot], (ii >> 1) & 1, abort_flag, err))) break;
        const int nq = items[slot].nq;
        if (nq < 0) break;  // no more items
        // dV / dK of the previous item have been read out of TMEM
        if (ii > 0 && !(ok = mbar_wait(acc_free, (ii - 1) & 1, abort_flag, err))) break;
        const uint32_t sK = smem_u32(sm + L::KV + kvs * 2 * BT_BYTES);
        for (int it = 0; it < nq; ++it, ++g) {
          const int bb = g % 3, s = g % kQS;
          if (!(ok = mbar_wait(&p_full[bb], (g / 3) & 1, abort_flag, err))) break;
          tc_fence_after();
          const uint32_t sQ = smem_u32(sm + L::Q + s * BQ_BYTES);
          const uint32_t sDO = smem_u32(sm + L::DO + s * BQ_BYTES);
          // dV += P^T dO and dK += dS^T Q with the A operands read from TMEM:
          // queries 16k..16k+15 sit at column 16k of the buffer (P^T, bf16
          // pairs), 8 further on for dS^T.
#pragma unroll
          for (int k = 0; k < BQ / 16; ++k) {
            const uint32_t acol = tBuf(bb) + k * 16;
            umma_bf16_ts(tDV, acol, umma_smem_desc(sDO + k * 2048, BQ_BYTES, 1024), idKN,
                         (it > 0 || k > 0));
            umma_bf16_ts(tDK, acol + 8, umma_smem_desc(sQ + k * 2048, BQ_BYTES, 1024), idKN,
                         (it > 0 || k > 0));
          }
          umma_commit(&q_empty[s]);
          if (it & 1) {
            // dQ of query pair J (tiles g-1, g) = dS K into the dP^T half of
            // this buffer: A = the pair's two dS^T tiles of the ring read
            // MN-major (M = 128 queries, 16 KB apart), B = K tile MN-major.
            const int J = g >> 1;
            const uint32_t sd = smem_u32(sm + L::DST + ((g - 1) & 3) * BT_BYTES);
#pragma unroll
            for (int k = 0; k < BT / 16; ++k)
              umma_bf16(tBuf(bb) + 64, umma_smem_desc(sd + k * 2048, BT_BYTES, 1024),
                        umma_smem_desc(sK + k * 2048, BT_BYTES, 1024), idMN, k > 0);
            umma_commit(&dq_full[J & 1]);
          }
          umma_commit(&done[g & 3]);
        }
        if (!ok) break;
        umma_commit(fin);
        umma_commit(&kv_empty[kvs]);
        mbar_arrive(&item_empty[slot]);
      }
    }
  } else if (warp == kBwdScoreWarp) {
    // S^T = K Q^T and dP^T = V dO^T of each tile into TMEM buffer g % 3, as
    // far ahead as the buffers allow. The buffer last served tile g-3: read by
    // that tile's dV / dK MMAs and, when g-3 closed a query pair, holding that
    // pair's dQ until the dQ warps have read it out.
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc_bf16(128, BQ, 0, 0);
      bool ok = true;
      int g = 0, ii = 0;
      for (; ok; ++ii) {
        const int slot = ii & 1, kvs = ii & 1;
        if (!(ok = mbar_wait(&item_full[slot], (ii >> 1) & 1, abort_flag, err))) break;
        const int nq = items[slot].nq;
        if (nq < 0) break;  // no more items
        if (!(ok = mbar_wait(&kv_full[kvs], (ii >> 1) & 1, abort_flag, err))) break;
        const uint32_t sK = smem_u32(sm + L::KV + kvs * 2 * BT_BYTES), sV = sK + BT_BYTES;
        for (int it = 0; it < nq; ++it, ++g) {
          const int s = g % kQS;
          if (g >= 3) {
            const int o = g - 3;
            if (!(ok = mbar_wait(&done[o & 3], (o >> 2) & 1, abort_flag, err))) break;
            if ((o & 1) && !(ok = mbar_wait(&dq_free[(o >> 1) & 1], (o >> 2) & 1, abort_flag, err)))
              break;
          }
          if (!(ok = mbar_wait(&q_full[s], (g / kQS) & 1, abort_flag, err))) break;
          tc_fence_after();
          const uint32_t sQ = smem_u32(sm + L::Q + s * BQ_BYTES);
          const uint32_t sDO = smem_u32(sm + L::DO + s * BQ_BYTES);
          const uint32_t tb = tBuf(g % 3);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            umma_bf16(tb, umma_smem_desc(sK + k * 32, 16, 1024),
                      umma_smem_desc(sQ + k * 32, 16, 1024), idS, k > 0);
            umma_bf16(tb + 64, umma_smem_desc(sV + k * 32, 16, 1024),
                      umma_smem_desc(sDO + k * 32, 16, 1024), idS, k > 0);
          }
          umma_commit(&s_full[g % 3]);
          umma_commit(&q_empty[s]);
        }
        if (!ok) break;
        mbar_arrive(&item_empty[slot]);
      }
    }
  } else if (warp < 2 + kBwdSmWarps) {
    // Softmax group wg takes the tiles it = wg, wg + kBwdSmGroups, ... of
    // each item. Warp w reads TMEM lanes of quadrant w % 4 (key rows) and
    // kBwdWarpCols query columns of the tile, in 16-column groups cg, and
    // writes P^T and dS^T (bf16 pairs) over exactly those S^T columns, so no
    // warp overwrites scores another warp has yet to read. The tile's
    // statistics come from the shared memory of its Q/dO stage (cp.async).
    const int quad = warp & 3;
    const int wg = (warp - 2) / kBwdGroupWarps;
    const int cg0 = (((warp - 2) % kBwdGroupWarps) >> 2) * (kBwdWarpCols / 16);
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float c = p.scale * kLog2e;
    bool ok = true;
    int g = 0, ii = 0;
    for (; ok; ++ii) {
      const int slot = ii & 1;
      if (!(ok = mbar_wait(&item_full[slot], (ii >> 1) & 1, abort_flag, err))) break;
      const BwdItem inf = items[slot];
      if (inf.nq < 0) break;  // no more items
      const int nq = inf.nq;
      const int b = inf.bh / p.H;
      const int k0 = inf.kt * BT;
      const int key = k0 + r;
      const int* segrow = SEG ? p.seg + (int64_t)b * p.T : nullptr;
      const int2* segtab = SEG ? segtab_of(slot) : nullptr;
      const int nch = (p.T + kSegChunk - 1) / kSegChunk - 2 * inf.kt;
      // this key row's segment id (rows past T take an id no query has)
      const int sk = segrow ? (key < p.T ? segrow[key] : INT_MAX) : 0;
      const int2 krng = segrow ? seg_range(segtab, nch, 0, 2) : make_int2(0, 0);
      for (int it = wg; it < nq; it += kBwdSmGroups) {
        const int gt = g + it;  // running tile index
        const int bb = gt % 3;
        const uint32_t tb = tBuf(bb);
        const int qt = qtile(slot, it);  // query tile index (64 positions) past k0
        if (!(ok = mbar_wait(&s_full[bb], (gt / 3) & 1, abort_flag, err))) break;
        if (!(ok = mbar_wait(&q_full[gt % kQS], (gt / kQS) & 1, abort_flag, err))) break;
        // The dS^T ring slot of this tile was last read by the dQ MMA of the
        // pair closed by tile gt-3.
        if (gt >= 4 && !(ok = mbar_wait(&done[(gt - 3) & 3], ((gt - 3) >> 2) & 1, abort_flag, err)))
          break;
        tc_fence_after();
        uint8_t* sd = sm + L::DST + (gt & 3) * BT_BYTES;
#pragma unroll
        for (int sub = 0; sub < kBwdWarpCols / 16; ++sub) {
        const int cg = cg0 + sub;
        // this 16-column group's statistics; the scores of the tile exist only
        // after its Q/dO stage (statistics included) was full
        const float* stat =
            reinterpret_cast<const float*>(sm + L::STAT + (gt % kQS) * L::kStatBytes) + cg * 16;
        const int* stat_seg = reinterpret_cast<const int*>(stat) + 128;
        uint32_t sraw[16], draw[16];
        tmem_ld16_nw(tb + lane_off + cg * 16, sraw);
        tmem_ld16_nw(tb + 64 + lane_off + cg * 16, draw);
        tmem_wait_ld();
        const int qbase = qt * BQ + cg * 16;  // query index relative to k0
        const bool diag = (qt < 2);           // key r > query masks only near the diagonal
        const int tail = p.T - k0 - qbase;    // columns j >= tail lie past the sequence end
        const bool mask = diag || tail < 16;
        // per-element segment test unless this key tile and query tile share one id
        const bool segmask = segrow && !rng_single(seg_range(segtab, nch, qt, 1), krng);
        // P^T = exp2(S^T c - lse log2e) and dS^T = P^T (dP^T - delta), two
        // columns per packed f32x2 instruction; the causal and end-of-sequence
        // tests run only on tiles that need them and the segment test only
        // when the tiles' ids differ.
        uint32_t pk[8], dk[8];
        auto softmax_cols = [&](auto mask_tag) {
          constexpr bool kMask = decltype(mask_tag)::value;
          const float2 c2 = make_float2(c, c);
          const float2 nlog2e = make_float2(-kLog2e, -kLog2e);
          const float2 m1 = make_float2(-1.f, -1.f);
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            const float4 l4 = reinterpret_cast<const float4*>(stat)[j4];
            const float4 d4 = reinterpret_cast<const float4*>(stat + 64)[j4];
            const float2 x01 = ffma2(make_float2(__uint_as_float(sraw[4 * j4]),
                                                 __uint_as_float(sraw[4 * j4 + 1])),
                                     c2, fmul2(make_float2(l4.x, l4.y), nlog2e));
            const float2 x23 = ffma2(make_float2(__uint_as_float(sraw[4 * j4 + 2]),
                                                 __uint_as_float(sraw[4 * j4 + 3])),
                                     c2, fmul2(make_float2(l4.z, l4.w), nlog2e));
            float pv[4] = {ex2(x01.x), ex2(x01.y), ex2(x23.x), ex2(x23.y)};
            // dP^T - delta as fma(delta, -1, dP^T): one rounding, as a subtraction
            const float2 g01 = ffma2(make_float2(d4.x, d4.y), m1,
                                     make_float2(__uint_as_float(draw[4 * j4]),
                                                 __uint_as_float(draw[4 * j4 + 1])));
            const float2 g23 = ffma2(make_float2(d4.z, d4.w), m1,
                                     make_float2(__uint_as_float(draw[4 * j4 + 2]),
                                                 __uint_as_float(draw[4 * j4 + 3])));
            float2 dv01 = fmul2(make_float2(pv[0], pv[1]), g01);
            float2 dv23 = fmul2(make_float2(pv[2], pv[3]), g23);
            float dvs[4] = {dv01.x, dv01.y, dv23.x, dv23.y};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int j = 4 * j4 + u;
              bool off = false;
              if (kMask) off = (diag && r > qbase + j) || j >= tail;
              if (SEG && segmask && stat_seg[j] != sk) off = true;
              if (off) pv[u] = dvs[u] = 0.f;
            }
            dv01 = make_float2(dvs[0], dvs[1]);
            dv23 = make_float2(dvs[2], dvs[3]);
            pk[2 * j4] = pack_bf16x2(pv[0], pv[1]);
            pk[2 * j4 + 1] = pack_bf16x2(pv[2], pv[3]);
            dk[2 * j4] = pack_bf16x2(dv01.x, dv01.y);
            dk[2 * j4 + 1] = pack_bf16x2(dv23.x, dv23.y);
          }
        };
        if (mask)
          softmax_cols(std::integral_constant<bool, true>());
        else
          softmax_cols(std::integral_constant<bool, false>());
        tmem_st8_nw(tb + lane_off + cg * 16, pk);
        tmem_st8_nw(tb + lane_off + cg * 16 + 8, dk);
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2)
          *reinterpret_cast<uint4*>(sd + swz128(r, cg * 2 + q2)) =
              make_uint4(dk[4 * q2], dk[4 * q2 + 1], dk[4 * q2 + 2], dk[4 * q2 + 3]);
        }
        tmem_wait_st();
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[bb]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
      g += nq;
    }
  } else {
    // dQ read-out: warp kBwdFlushWarp + i serves TMEM lane quadrant
    // (kBwdFlushWarp + i) % 4. For each query pair (list entries 2j, 2j+1 of
    // an item; TMEM lane m is row m of the pair, quadrants 0-1 the first tile,
    // 2-3 the second) it loads its 32 rows x 64 fp32 columns as soon as the
    // pair's dQ MMA has completed, releases the TMEM buffer, stages the rows
    // in two 128-byte swizzled [32 x 32] boxes of its own and reduces them
    // into dq_acc with TMA reduce-adds (rows past the sequence end are clipped
    // by the map; a box that starts past it is skipped). At the end of an
    // item the same warps write dK and dV. The softmax warps never wait for
    // this.
    const int quad = warp & 3;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    uint8_t* stage = sm + L::DQS + (warp - kBwdFlushWarp) * 8192;
    bool ok = true;
    int g = 0, ii = 0;
    for (; ok; ++ii) {
      const int slot = ii & 1;
      if (!(ok = mbar_wait(&item_full[slot], (ii >> 1) & 1, abort_flag, err))) break;
      const BwdItem inf = items[slot];
      if (inf.nq < 0) break;  // no more items
      const int k0 = inf.kt * BT;
      for (int j = 0; j < inf.nq / 2; ++j) {
        const int J = (g >> 1) + j;  // running pair index
        if (!(ok = mbar_wait(&dq_full[J & 1], (J >> 1) & 1, abort_flag, err))) break;
        tc_fence_after();
        const int bb = (g + 2 * j + 1) % 3;  // buffer of the pair's closing tile
        float v[64];
        tmem_ld32(tBuf(bb) + 64 + lane_off, v);
        tmem_ld32(tBuf(bb) + 96 + lane_off, v + 32);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dq_free[J & 1]);
        const int row0 = k0 + qtile(slot, 2 * j + (quad >> 1)) * BQ + (quad & 1) * 32;
        if (row0 < p.T) {  // warp-uniform
          if (lane == 0) bulk_wait_read();  // the previous reduce has read the staging boxes
          __syncwarp();
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
              *reinterpret_cast<float4*>(stage + hh * 4096 + swz128(lane, ch)) =
                  make_float4(v[32 * hh + 4 * ch], v[32 * hh + 4 * ch + 1],
                              v[32 * hh + 4 * ch + 2], v[32 * hh + 4 * ch + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_3d(&tmDQ, stage, 0, row0, inf.bh);
            tma_reduce_add_3d(&tmDQ, stage + 4096, 32, row0, inf.bh);
            bulk_commit();
          }
        }
      }
      if (!ok) break;
      // dK (times the softmax scale, rotated back by RoPE) and dV of the
      // item's 128 keys, this warp's 32 rows. All four 32-column chunks leave
      // TMEM first (dK parked in this warp's staging area, dV in registers) so
      // the next item's gradient MMAs can start; then the rows are written.
      if (!(ok = mbar_wait(fin, ii & 1, abort_flag, err))) break;
      tc_fence_after();
      {
        const int key = k0 + quad * 32 + lane;
        const int bi = inf.bh / p.H, hi = inf.bh - bi * p.H;
        if (lane == 0) bulk_wait_read();  // the last dQ reduce has read the staging area
        __syncwarp();
        float* park = reinterpret_cast<float*>(stage);  // [32 rows][64] fp32, 16-byte chunks xor-swizzled
        auto park_at = [&](int chunk) { return park + lane * 64 + ((chunk ^ (lane & 15)) << 2); };
        {
          float t64[64];
          tmem_ld32_nw(tDK + lane_off, reinterpret_cast<uint32_t*>(t64));
          tmem_ld32_nw(tDK + lane_off + 32, reinterpret_cast<uint32_t*>(t64) + 32);
          tmem_wait_ld();
#pragma unroll
          for (int c4 = 0; c4 < 16; ++c4)
            *reinterpret_cast<float4*>(park_at(c4)) =
                make_float4(t64[4 * c4], t64[4 * c4 + 1], t64[4 * c4 + 2], t64[4 * c4 + 3]);
        }
        float dvv[64];
        tmem_ld32_nw(tDV + lane_off, reinterpret_cast<uint32_t*>(dvv));
        tmem_ld32_nw(tDV + lane_off + 32, reinterpret_cast<uint32_t*>(dvv) + 32);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_free);
        if (key < p.T) {
          bf16* vrow = p.dv + bi * p.sb + hi * p.sh + (int64_t)key * p.st;
          bf16* krow = p.dk + bi * p.sb + hi * p.sh + (int64_t)key * p.st;
#pragma unroll
          for (int q8 = 0; q8 < 8; ++q8) {
            const float* gv = dvv + 8 * q8;
            uint4 o;
            o.x = pack_bf16x2(gv[0], gv[1]);
            o.y = pack_bf16x2(gv[2], gv[3]);
            o.z = pack_bf16x2(gv[4], gv[5]);
            o.w = pack_bf16x2(gv[6], gv[7]);
            *reinterpret_cast<uint4*>(vrow + 8 * q8) = o;
          }
#pragma unroll 2
          for (int q8 = 0; q8 < 8; ++q8) {
            const float4 a4 = *reinterpret_cast<const float4*>(park_at(2 * q8));
            const float4 b4 = *reinterpret_cast<const float4*>(park_at(2 * q8 + 1));
            float gv[8] = {a4.x, a4.y, a4.z, a4.w, b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) gv[i] *= p.scale;
            if (p.rcos) rope_back(gv, p.rcos, p.rsin, key, q8);
            uint4 o;
            o.x = pack_bf16x2(gv[0], gv[1]);
            o.y = pack_bf16x2(gv[2], gv[3]);
            o.z = pack_bf16x2(gv[4], gv[5]);
            o.w = pack_bf16x2(gv[6], gv[7]);
            *reinterpret_cast<uint4*>(krow + 8 * q8) = o;
          }
        }
        __syncwarp();  // the park area is read before the next dQ staging writes
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
      g += inf.nq;
    }
    if (lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) sched_finish(p.sched);
}

// delta[bh, t] = sum_e dO * O, and zero the dQ accumulator row. Eight lanes
// per row (16-byte loads), four rows per warp.
__global__ void attn_delta_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dout,
                                  int64_t osb, int64_t osh, int64_t ost, int B, int H, int T,
                                  float* __restrict__ delta, float* __restrict__ dq_acc) {
  const int64_t rows = (int64_t)B * H * T;
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
  const int seg = threadIdx.x & 7;
  const bool valid = r < rows;  // no early return: the 8-lane shuffles below span the warp
  const int64_t rr = valid ? r : 0;
  const int64_t bh = rr / T;
  const int t = (int)(rr - bh * T);
  const int b = (int)(bh / H), h = (int)(bh - (int64_t)b * H);
  const int64_t off = b * osb + h * osh + (int64_t)t * ost + seg * 8;
  const uint4 qo = *reinterpret_cast<const uint4*>(o + off);
  const uint4 qg = *reinterpret_cast<const uint4*>(dout + off);
  const uint32_t* wo = &qo.x;
  const uint32_t* wg = &qg.x;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float o0, o1, g0, g1;
    unpack_bf16x2(wo[j], o0, o1);
    unpack_bf16x2(wg[j], g0, g1);
    s += o0 * g0 + o1 * g1;
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  if (!valid) return;
  if (seg == 0) delta[r] = s;
  float4* z = reinterpret_cast<float4*>(dq_acc + r * HD + seg * 8);
  z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// dq = bf16(scale * dq_acc), rotated back by RoPE when tables are given.
__global__ void attn_dq_store_kernel(const float* __restrict__ dq_acc, bf16* __restrict__ dq,
                                     int64_t sb, int64_t sh, int64_t st, int B, int H, int T,
                                     float scale, const bf16* rcos, const bf16* rsin) {
  const int64_t chunks = (int64_t)B * H * T * (HD / 8);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i >> 3;
    const int c = (int)(i & 7);
    const int64_t bh = row / T;
    const int t = (int)(row - bh * T);
    const int b = (int)(bh / H), h = (int)(bh - (int64_t)b * H);
    const float4* src = reinterpret_cast<const float4*>(dq_acc + row * HD + c * 8);
    float4 a = src[0], e = src[1];
    float v[8] = {a.x * scale, a.y * scale, a.z * scale, a.w * scale,
                  e.x * scale, e.y * scale, e.z * scale, e.w * scale};
    if (rcos) rope_back(v, rcos, rsin, t, c);
    uint4 q;
    q.x = pack_bf16x2(v[0], v[1]);
    q.y = pack_bf16x2(v[2], v[3]);
    q.z = pack_bf16x2(v[4], v[5]);
    q.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(dq + b * sb + h * sh + (int64_t)t * st + c * 8) = q;
  }
}

int attention_read_error(int clear) {
  int hv = 0;
  cudaMemcpyFromSymbol(&hv, g_attn_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_attn_error, &z, sizeof(int));
  }
  return hv;
}

// ------------------------------------------------------------------ host
// A counter slot of g_attn_sched for one launch of kernel `which` (0 forward,
// 1 backward) on the current device: slots rotate per device, so up to
// kSchedSlots launches may be in flight at once.
static unsigned* sched_slot(int which) {
  static unsigned* base[64] = {};
  static std::atomic<unsigned> next[64][2];
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return nullptr;
  if (!base[dev]) {
    std::lock_guard<std::mutex> lock(mu);
    if (!base[dev]) {
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_attn_sched) != cudaSuccess) return nullptr;
      base[dev] = reinterpret_cast<unsigned*>(ptr);
    }
  }
  const unsigned k = next[dev][which].fetch_add(1) % kSchedSlots;
  return base[dev] + ((size_t)which * kSchedSlots + k) * 2;
}
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 4-D map over a [b, t, h, e] tensor with element strides (sb, st, sh), box
// 64 (e) x box_rows (t), 128-byte swizzle.
static bool make_map4(CUtensorMap* m, const void* base, int B, int H, int T, int64_t sb,
                      int64_t sh, int64_t st, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {HD, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {HD, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gptb200

using namespace gptb200;

// 3-D fp32 map over dq_acc [B*H, T, 64], box 32 x 32 x 1, 128-byte swizzle
// (the bwd kernel's TMA reduce-add target).
static bool make_dq_map(CUtensorMap* m, float* base, int BH, int T) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {HD, (cuuint64_t)T, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)HD * 4, (cuuint64_t)T * HD * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int check_attn(const void* q, const void* k, const void* v, int64_t sb, int64_t sh,
                      int64_t st, int64_t osb, int64_t osh, int64_t ost, int64_t batch,
                      int64_t heads, int64_t seq, int64_t hd) {
  if (!q || !k || !v) return GPTB200_EINVAL;
  if (batch <= 0 || heads <= 0 || seq <= 0) return GPTB200_EINVAL;
  if (hd != HD) return GPTB200_EUNSUPPORTED;
  if (batch * heads > 65535 || seq > (1 << 24)) return GPTB200_ESHAPE;
  if ((sb | sh | st | osb | osh | ost) % 8) return GPTB200_ESHAPE;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v)) & 15)
    return GPTB200_ESHAPE;
  return 0;
}

extern "C" int gptb200_attention_fwd(const void* q, const void* k, const void* v, int64_t stride_b,
                                     int64_t stride_h, int64_t stride_t, void* o,
                                     int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_t,
                                     float* lse, int64_t batch, int64_t heads, int64_t seq,
                                     int64_t head_dim, float softmax_scale,
                                     const int32_t* segment_ids, void* stream) {
  int s = check_attn(q, k, v, stride_b, stride_h, stride_t, o_stride_b, o_stride_h, o_stride_t,
                     batch, heads, seq, head_dim);
  if (s) return s;
  if (!o || !lse || !(softmax_scale > 0.f)) return GPTB200_EINVAL;
  if (segment_ids && seq > (int64_t)kMaxSegChunks * kSegChunk) return GPTB200_EUNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(segment_ids) & 3) return GPTB200_ESHAPE;
  if (reinterpret_cast<uintptr_t>(o) & 15) return GPTB200_ESHAPE;
  CUtensorMap mq, mk, mv;
  if (!make_map4(&mq, q, (int)batch, (int)heads, (int)seq, stride_b, stride_h, stride_t, FQ) ||
      !make_map4(&mk, k, (int)batch, (int)heads, (int)seq, stride_b, stride_h, stride_t, FK) ||
      !make_map4(&mv, v, (int)batch, (int)heads, (int)seq, stride_b, stride_h, stride_t, FK))
    return GPTB200_ESHAPE;
  AttnParams p = {};
  p.B = (int)batch;
  p.H = (int)heads;
  p.T = (int)seq;
  p.scale = softmax_scale;
  p.o = reinterpret_cast<bf16*>(o);
  p.osb = o_stride_b;
  p.osh = o_stride_h;
  p.ost = o_stride_t;
  p.lse = lse;
  p.seg = segment_ids;
  p.sched = sched_slot(0);
  if (!p.sched) return GPTB200_EUNSUPPORTED;
  static bool cfg[64][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int seg = segment_ids != nullptr;
  auto kern = seg ? attn_fwd_tc<true> : attn_fwd_tc<false>;
  const int smem = seg ? FwdSmem<true>::TOTAL : FwdSmem<false>::TOTAL;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 64 || !cfg[dev][seg]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return -static_cast<int>(e);
    if (dev < 64) cfg[dev][seg] = true;
  }
  // persistent: one CTA per SM (or per item, when there are fewer items)
  const int64_t items = (seq + 2 * FQ - 1) / (2 * FQ) * batch * heads;
  const unsigned grid = (unsigned)std::min<int64_t>(items, sms);
  kern<<<grid, kFwdThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(mq, mk, mv, p);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" size_t gptb200_attention_bwd_workspace_size(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  const int64_t rows = batch * heads * seq;
  return (size_t)((rows * 4 + 255) / 256 * 256 + rows * HD * 4);
}

extern "C" int gptb200_attention_bwd(const void* q, const void* k, const void* v, int64_t stride_b,
                                     int64_t stride_h, int64_t stride_t, const void* o,
                                     const void* dout, int64_t o_stride_b, int64_t o_stride_h,
                                     int64_t o_stride_t, const float* lse, void* dq, void* dk,
                                     void* dv, int64_t batch, int64_t heads, int64_t seq,
                                     int64_t head_dim, float softmax_scale, const void* rope_cos,
                                     const void* rope_sin, const int32_t* segment_ids,
                                     void* workspace, void* stream) {
  int s = check_attn(q, k, v, stride_b, stride_h, stride_t, o_stride_b, o_stride_h, o_stride_t,
                     batch, heads, seq, head_dim);
  if (s) return s;
  if (!o || !dout || !lse || !dq || !dk || !dv || !workspace || !(softmax_scale > 0.f))
    return GPTB200_EINVAL;
  if (segment_ids && seq > (int64_t)kMaxSegChunks * kSegChunk) return GPTB200_EUNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(segment_ids) & 3) return GPTB200_ESHAPE;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return GPTB200_EINVAL;
  if ((reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(dq) |
       reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv) |
       reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(workspace)) & 15)
    return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  const int B = (int)batch, H = (int)heads, T = (int)seq;
  CUtensorMap mq, mk, mv, mdo;
  if (!make_map4(&mq, q, B, H, T, stride_b, stride_h, stride_t, BQ) ||
      !make_map4(&mk, k, B, H, T, stride_b, stride_h, stride_t, BT) ||
      !make_map4(&mv, v, B, H, T, stride_b, stride_h, stride_t, BT) ||
      !make_map4(&mdo, dout, B, H, T, o_stride_b, o_stride_h, o_stride_t, BQ))
    return GPTB200_ESHAPE;
  const int64_t rows = batch * heads * seq;
  float* delta = reinterpret_cast<float*>(workspace);
  float* dq_acc = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                           (rows * 4 + 255) / 256 * 256);
  attn_delta_kernel<<<(unsigned)((rows * 8 + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const bf16*>(o), reinterpret_cast<const bf16*>(dout), o_stride_b,
      o_stride_h, o_stride_t, B, H, T, delta, dq_acc);
  GPTB200_CHECK_LAUNCH();
  AttnParams p = {};
  p.B = B;
  p.H = H;
  p.T = T;
  p.scale = softmax_scale;
  p.lse = const_cast<float*>(lse);
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dk = reinterpret_cast<bf16*>(dk);
  p.dv = reinterpret_cast<bf16*>(dv);
  p.sb = stride_b;
  p.sh = stride_h;
  p.st = stride_t;
  p.rcos = reinterpret_cast<const bf16*>(rope_cos);
  p.rsin = reinterpret_cast<const bf16*>(rope_sin);
  p.seg = segment_ids;
  p.sched = sched_slot(1);
  if (!p.sched) return GPTB200_EUNSUPPORTED;
  static bool cfg[64][4] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int seg = segment_ids != nullptr;
  const int groups = seq >= 2048 ? 2 : 1;
  auto kern = seg ? (groups == 2 ? attn_bwd_tc<true, 2> : attn_bwd_tc<true, 1>)
                  : (groups == 2 ? attn_bwd_tc<false, 2> : attn_bwd_tc<false, 1>);
  const int smem = seg ? BwdSmem<true>::TOTAL : BwdSmem<false>::TOTAL;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ci = seg * 2 + (groups - 1);
  if (dev >= 64 || !cfg[dev][ci]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return -static_cast<int>(e);
    if (dev < 64) cfg[dev][ci] = true;
  }
  // persistent: one CTA per SM (or per item, when there are fewer items)
  const int64_t items = (seq + BT - 1) / BT * batch * heads;
  const unsigned grid = (unsigned)std::min<int64_t>(items, sms);
  CUtensorMap mdq;
  if (!make_dq_map(&mdq, dq_acc, B * H, T)) return GPTB200_ESHAPE;
  kern<<<grid, kBwdThreads, smem, st>>>(mq, mk, mv, mdo, mdq, p);
  GPTB200_CHECK_LAUNCH();
  const int64_t chunks = rows * (HD / 8);
  int blocks = (int)std::min<int64_t>((chunks + 255) / 256, (int64_t)sms * 8);
  attn_dq_store_kernel<<<blocks, 256, 0, st>>>(dq_acc, reinterpret_cast<bf16*>(dq), stride_b,
                                               stride_h, stride_t, B, H, T, softmax_scale,
                                               reinterpret_cast<const bf16*>(rope_cos),
                                               reinterpret_cast<const bf16*>(rope_sin));
  GPTB200_CHECK_LAUNCH();
  return 0;
}
