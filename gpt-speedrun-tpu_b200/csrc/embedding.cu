// Token-embedding gradient (the backward of the gather of
// recipes/reference/train.py:1107), reproducible bit for bit.
//
// dtable[v, :] += sum over rows r with tokens[r] == v of dout[r, :].
// A scatter with fp32 atomics would add each vocabulary row's terms in
// whatever order the rows arrive, so two runs could differ in the last bits.
// Here the rows are first put in a fixed order, (token, row index), by a
// stable LSD radix sort (8-bit digits, one pass per byte of the largest id),
// and then every token's rows are added in that order:
//
//   radix_upsweep    per 2048-row tile: how many keys of each digit
//   radix_scan       exclusive scan of those counts, digit-major (one block)
//   radix_downsweep  stable scatter: the rank of a key among equal digits is
//                    (tile base) + (earlier warps of the tile) + (earlier
//                    batches of the warp) + (earlier lanes, __match_any_sync)
//   embed_segsum     each block adds a fixed run of 128 sorted positions; a
//                    token whose rows all lie inside the block is written
//                    directly, the head and tail of a token that crosses a
//                    block boundary are stored as partials
//   embed_fixup      the block where a crossing token starts adds its tail and
//                    the heads of the following blocks, in block order
//
// Every step is deterministic (integer counts, fixed fp32 addition order).
// Token ids outside [0, vocab) are sorted to the end and contribute nothing.
#include <algorithm>

#include "common.cuh"

namespace gptb200 {

constexpr int kTile = 2048;        // keys per radix tile (256 threads x 8)
constexpr int kSortThreads = 256;
constexpr int kSeg = 128;          // sorted positions per segmented-sum block
constexpr int kSegThreads = 128;   // 8 columns per thread

static int64_t rup(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Initial key of row i: the token id, or `vocab` (sorts last) when invalid.
__device__ __forceinline__ uint32_t first_key(const int32_t* tok, int64_t i, int64_t vocab) {
  const int32_t t = tok[i];
  return (t >= 0 && t < vocab) ? (uint32_t)t : (uint32_t)vocab;
}

__global__ void __launch_bounds__(kSortThreads) radix_upsweep(const int32_t* __restrict__ tok,
                                                              const uint32_t* __restrict__ keys,
                                                              int64_t n, int64_t vocab, int shift,
                                                              int tiles, int* __restrict__ hist) {
  __shared__ int cnt[256];
  cnt[threadIdx.x] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kTile;
  for (int j = threadIdx.x; j < kTile; j += kSortThreads) {
    const int64_t i = base + j;
    if (i >= n) break;
    const uint32_t k = keys ? keys[i] : first_key(tok, i, vocab);
    atomicAdd(&cnt[(k >> shift) & 255u], 1);
  }
  __syncthreads();
  hist[(int64_t)threadIdx.x * tiles + blockIdx.x] = cnt[threadIdx.x];
}

// In-place exclusive scan of `total` ints with one block of 1024 threads:
// the counts go through shared memory in coalesced chunks of 8192, each
// thread scans 8 consecutive entries, the 1024 sums are scanned by warps.
constexpr int kScanChunk = 8192;

__global__ void __launch_bounds__(1024) radix_scan(int* __restrict__ h, int64_t total) {
  __shared__ int buf[kScanChunk];
  __shared__ int wsum[32];
  __shared__ int carry_s;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry_s = 0;
  for (int64_t base = 0; base < total; base += kScanChunk) {
    const int n = (int)min(total - base, (int64_t)kScanChunk);
    for (int i = threadIdx.x; i < kScanChunk; i += 1024) buf[i] = i < n ? h[base + i] : 0;
    __syncthreads();
    int v[8], s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = buf[threadIdx.x * 8 + j];
      s += v[j];
    }
    // inclusive warp scan of the per-thread sums
    int x = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int t = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      wsum[lane] = t;  // inclusive over warps
    }
    __syncthreads();
    int run = carry_s + (w ? wsum[w - 1] : 0) + x - s;  // exclusive prefix of this thread
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      buf[threadIdx.x * 8 + j] = run;
      run += v[j];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += 1024) h[base + i] = buf[i];
    if (threadIdx.x == 0) carry_s += wsum[31];
    __syncthreads();
  }
}

// Stable scatter of one tile. Warp w owns keys [w*256, w*256+256) of the tile,
// taken as 8 batches of 32 consecutive keys, so (warp, batch, lane) order is
// the original order.
__global__ void __launch_bounds__(kSortThreads) radix_downsweep(
    const int32_t* __restrict__ tok, const uint32_t* __restrict__ keys_in,
    const int32_t* __restrict__ vals_in, uint32_t* __restrict__ keys_out,
    int32_t* __restrict__ vals_out, int64_t n, int64_t vocab, int shift, int tiles,
    const int* __restrict__ hist) {
  __shared__ int wcnt[kSortThreads / 32][256];
  __shared__ int tbase[256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned lt = (1u << lane) - 1u;
  for (int w = 0; w < kSortThreads / 32; ++w) wcnt[w][threadIdx.x] = 0;
  tbase[threadIdx.x] = hist[(int64_t)threadIdx.x * tiles + blockIdx.x];
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kTile + warp * 256;
  uint32_t key[8];
  int32_t val[8];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const int64_t i = base + b * 32 + lane;
    if (i < n) {
      key[b] = keys_in ? keys_in[i] : first_key(tok, i, vocab);
      val[b] = keys_in ? vals_in[i] : (int32_t)i;
    } else {
      key[b] = 0xffffffffu;  // past the end: digit 256, never written
      val[b] = 0;
    }
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const int dig = key[b] == 0xffffffffu ? 256 : (int)((key[b] >> shift) & 255u);
    const unsigned peers = __match_any_sync(0xffffffffu, dig);
    if (dig < 256 && lane == __ffs(peers) - 1) wcnt[warp][dig] += __popc(peers);
    __syncwarp();  // the next batch's leader may be another lane
  }
  __syncthreads();
  {  // exclusive prefix over the warps, per digit
    int run = 0;
    for (int w = 0; w < kSortThreads / 32; ++w) {
      const int t = wcnt[w][threadIdx.x];
      wcnt[w][threadIdx.x] = run;
      run += t;
    }
  }
  __syncthreads();
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const int dig = key[b] == 0xffffffffu ? 256 : (int)((key[b] >> shift) & 255u);
    const unsigned peers = __match_any_sync(0xffffffffu, dig);
    int before = 0;
    if (dig < 256) before = wcnt[warp][dig];
    __syncwarp();
    if (dig < 256) {
      const int pos = tbase[dig] + before + __popc(peers & lt);
      keys_out[pos] = key[b];
      vals_out[pos] = val[b];
      if (lane == __ffs(peers) - 1) wcnt[warp][dig] = before + __popc(peers);
    }
    __syncwarp();
  }
}

__device__ __forceinline__ void add_bf16x8(float* acc, uint4 q) {
  float a, b;
  unpack_bf16x2(q.x, a, b);
  acc[0] += a;
  acc[1] += b;
  unpack_bf16x2(q.y, a, b);
  acc[2] += a;
  acc[3] += b;
  unpack_bf16x2(q.z, a, b);
  acc[4] += a;
  acc[5] += b;
  unpack_bf16x2(q.w, a, b);
  acc[6] += a;
  acc[7] += b;
}

__device__ __forceinline__ void add_to_row(float* dst, const float* acc) {
  float4* d4 = reinterpret_cast<float4*>(dst);
  float4 x = d4[0], y = d4[1];
  d4[0] = make_float4(x.x + acc[0], x.y + acc[1], x.z + acc[2], x.w + acc[3]);
  d4[1] = make_float4(y.x + acc[4], y.y + acc[5], y.z + acc[6], y.w + acc[7]);
}

__device__ __forceinline__ void store_row(float* dst, const float* acc) {
  float4* d4 = reinterpret_cast<float4*>(dst);
  d4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  d4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// Thread t of block (x, y) owns columns [8c, 8c + 8), c = y * 128 + t, and adds
// the rows of sorted positions [x * 128, x * 128 + 128) token by token.
__global__ void __launch_bounds__(kSegThreads) embed_segsum(
    const uint32_t* __restrict__ keys, const int32_t* __restrict__ rows,
    const bf16* __restrict__ dout, int64_t n, int d, int64_t vocab, float* __restrict__ dtable,
    float* __restrict__ head, float* __restrict__ tail) {
  const int c8 = (blockIdx.y * kSegThreads + threadIdx.x) * 8;
  if (c8 >= d) return;
  const int64_t p0 = (int64_t)blockIdx.x * kSeg, p1 = min(n, p0 + kSeg);
  const uint32_t before = p0 > 0 ? keys[p0 - 1] : 0xffffffffu;
  const uint32_t after = p1 < n ? keys[p1] : 0xffffffffu;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  uint32_t cur = keys[p0];
  auto flush = [&](uint32_t k, bool first_run, bool crosses_end) {
    if (k >= (uint32_t)vocab) return;
    if (first_run && k == before)
      store_row(head + blockIdx.x * (int64_t)d + c8, acc);  // continues a run of earlier blocks
    else if (crosses_end)
      store_row(tail + blockIdx.x * (int64_t)d + c8, acc);  // finished by embed_fixup
    else
      add_to_row(dtable + (int64_t)k * d + c8, acc);
  };
  bool first_run = true;
  for (int64_t p = p0; p < p1; p += 8) {
    uint32_t k8[8];
    uint4 q8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      k8[j] = p + j < p1 ? keys[p + j] : 0xffffffffu;
      const int32_t r = p + j < p1 ? rows[p + j] : 0;
      q8[j] = (k8[j] < (uint32_t)vocab)
                  ? *reinterpret_cast<const uint4*>(dout + (int64_t)r * d + c8)
                  : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (k8[j] == 0xffffffffu) break;
      if (k8[j] != cur) {
        flush(cur, first_run, false);
        first_run = false;
        cur = k8[j];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      }
      add_bf16x8(acc, q8[j]);
    }
  }
  flush(cur, first_run, cur == after);
}

// Block x finishes the token whose rows start in block x and run past its
// end: it adds its tail and the heads of the following blocks the token
// covers, in block order. The block's threads first find how many blocks the
// token covers (each thread tests its own candidates), so that the head rows
// can then be loaded independently of one another.
__global__ void __launch_bounds__(kSegThreads) embed_fixup(const uint32_t* __restrict__ keys,
                                                           int64_t n, int d, int64_t vocab,
                                                           const float* __restrict__ head,
                                                           const float* __restrict__ tail,
                                                           float* __restrict__ dtable) {
  __shared__ int last_s;
  const int64_t p0 = (int64_t)blockIdx.x * kSeg, p1 = min(n, p0 + kSeg);
  if (p1 >= n) return;
  const uint32_t k = keys[p1 - 1];
  if (k >= (uint32_t)vocab || keys[p1] != k) return;          // nothing crosses the end
  if (keys[p0] == k && p0 > 0 && keys[p0 - 1] == k) return;  // started earlier: not the owner
  // blocks x > blockIdx.x that the token reaches: those whose first key is k
  const int64_t nblocks = (n + kSeg - 1) / kSeg;
  if (threadIdx.x == 0) last_s = (int)blockIdx.x + 1;
  __syncthreads();
  for (int64_t base = blockIdx.x + 1;; base += kSegThreads) {
    const int64_t x = base + threadIdx.x;
    const bool reach = x < nblocks && keys[x * kSeg] == k;
    if (reach) atomicMax(&last_s, (int)x);
    if (!__syncthreads_or(x < nblocks && !reach) && base + kSegThreads < nblocks) continue;
    break;
  }
  __syncthreads();
  const int last = last_s;
  const int c8 = (blockIdx.y * kSegThreads + threadIdx.x) * 8;
  if (c8 >= d) return;
  float acc[8];
  const float4* t4 = reinterpret_cast<const float4*>(tail + blockIdx.x * (int64_t)d + c8);
  float4 a = t4[0], b = t4[1];
  acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w;
  acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
  for (int x = (int)blockIdx.x + 1; x <= last; x += 4) {
    float4 hv[4][2];
#pragma unroll
    for (int u = 0; u < 4; ++u) {  // independent loads, then the adds in block order
      const float4* h4 = reinterpret_cast<const float4*>(head + (int64_t)(x + u) * d + c8);
      if (x + u <= last) {
        hv[u][0] = h4[0];
        hv[u][1] = h4[1];
      } else {
        hv[u][0] = hv[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (x + u > last) break;
      acc[0] += hv[u][0].x; acc[1] += hv[u][0].y; acc[2] += hv[u][0].z; acc[3] += hv[u][0].w;
      acc[4] += hv[u][1].x; acc[5] += hv[u][1].y; acc[6] += hv[u][1].z; acc[7] += hv[u][1].w;
    }
  }
  add_to_row(dtable + (int64_t)k * d + c8, acc);
}

struct EmbedBwdLayout {
  int64_t tiles, blocks, passes;
  size_t keys0, vals0, keys1, vals1, hist, head, tail, total;
};

static EmbedBwdLayout embed_bwd_layout(int64_t n, int64_t d, int64_t vocab) {
  EmbedBwdLayout L;
  L.tiles = (n + kTile - 1) / kTile;
  L.blocks = (n + kSeg - 1) / kSeg;
  int bits = 1;
  while (bits < 31 && (int64_t(1) << bits) <= vocab) ++bits;  // keys are <= vocab
  L.passes = (bits + 7) / 8;
  size_t off = 0;
  auto take = [&](int64_t bytes) {
    size_t o = off;
    off += (size_t)rup(bytes, 256);
    return o;
  };
  L.keys0 = take(n * 4);
  L.vals0 = take(n * 4);
  L.keys1 = take(n * 4);
  L.vals1 = take(n * 4);
  L.hist = take(256 * L.tiles * 4);
  L.head = take(L.blocks * d * 4);
  L.tail = take(L.blocks * d * 4);
  L.total = off;
  return L;
}

}  // namespace gptb200

using namespace gptb200;

extern "C" size_t gptb200_embedding_bwd_workspace_size(int64_t n, int64_t d, int64_t vocab) {
  if (n <= 0 || d <= 0 || vocab <= 0) return 0;
  return embed_bwd_layout(n, d, vocab).total;
}

extern "C" int gptb200_embedding_bwd(const int32_t* tokens, const void* dout, float* dtable,
                                     int64_t n, int64_t d, int64_t vocab, void* workspace,
                                     void* stream) {
  if (!tokens || !dout || !dtable || !workspace || n <= 0 || d <= 0 || vocab <= 0)
    return GPTB200_EINVAL;
  if (d % 8 || ((reinterpret_cast<uintptr_t>(dtable) | reinterpret_cast<uintptr_t>(dout) |
                 reinterpret_cast<uintptr_t>(workspace)) & 15))
    return GPTB200_ESHAPE;
  if (n > INT32_MAX || vocab >= INT32_MAX || 256 * ((n + kTile - 1) / kTile) > INT32_MAX)
    return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  const EmbedBwdLayout L = embed_bwd_layout(n, d, vocab);
  char* ws = reinterpret_cast<char*>(workspace);
  uint32_t* keys[2] = {reinterpret_cast<uint32_t*>(ws + L.keys0),
                       reinterpret_cast<uint32_t*>(ws + L.keys1)};
  int32_t* vals[2] = {reinterpret_cast<int32_t*>(ws + L.vals0),
                      reinterpret_cast<int32_t*>(ws + L.vals1)};
  int* hist = reinterpret_cast<int*>(ws + L.hist);
  const int tiles = (int)L.tiles;
  int cur = -1;  // -1: keys come from `tokens`
  for (int pass = 0; pass < L.passes; ++pass) {
    const int shift = 8 * pass;
    const uint32_t* kin = cur < 0 ? nullptr : keys[cur];
    const int32_t* vin = cur < 0 ? nullptr : vals[cur];
    const int out = cur < 0 ? 0 : 1 - cur;
    radix_upsweep<<<tiles, kSortThreads, 0, st>>>(tokens, kin, n, vocab, shift, tiles, hist);
    GPTB200_CHECK_LAUNCH();
    radix_scan<<<1, 1024, 0, st>>>(hist, 256 * (int64_t)tiles);
    GPTB200_CHECK_LAUNCH();
    radix_downsweep<<<tiles, kSortThreads, 0, st>>>(tokens, kin, vin, keys[out], vals[out], n,
                                                    vocab, shift, tiles, hist);
    GPTB200_CHECK_LAUNCH();
    cur = out;
  }
  float* head = reinterpret_cast<float*>(ws + L.head);
  float* tail = reinterpret_cast<float*>(ws + L.tail);
  dim3 grid((unsigned)L.blocks, (unsigned)((d / 8 + kSegThreads - 1) / kSegThreads));
  embed_segsum<<<grid, kSegThreads, 0, st>>>(keys[cur], vals[cur],
                                             reinterpret_cast<const bf16*>(dout), n, (int)d,
                                             vocab, dtable, head, tail);
  GPTB200_CHECK_LAUNCH();
  embed_fixup<<<grid, kSegThreads, 0, st>>>(keys[cur], n, (int)d, vocab, head, tail, dtable);
  GPTB200_CHECK_LAUNCH();
  return 0;
}
