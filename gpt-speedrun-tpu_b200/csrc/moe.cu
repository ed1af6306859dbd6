// Top-k routed MLP (recipes/reference_moe/train.py:1230-1345, routed_mlp_local)
// around the tcgen05 GEMM: routing, dropless dispatch into expert segments,
// gather / combine and their backward, router backward, per-expert bias
// gradients and the balance-loss statistics.
//
// Layout of one layer's routed buffers (N tokens, k = top-k, E experts):
//   assignment a = i * k + j (token i, choice j); the assignments are stably
//   sorted by expert into one row buffer where expert e owns the segment
//   [seg[e].x, seg[e].x + seg[e].y), seg[e].y = its count rounded up to 128
//   (padding rows hold zeros on the way in and are ignored on the way out), so
//   every 128-row GEMM tile belongs to one expert and the expert GEMMs take
//   their bounds from `seg` on the device (GemmParams::range).
#include <algorithm>

#include "common.cuh"

namespace gptb200 {

constexpr int kMoeMaxE = 16;
constexpr int kMoeMaxK = 4;
constexpr int kDispatchBlock = 1024;  // assignments per dispatch block

// Per layer statistics, fp32: [0, E) router probability sums, [E, 2E) counts,
// 2E entropy sum, 2E+1 top-1 gate sum, 2E+2 sum of squared logits.
__host__ __device__ constexpr int moe_stat_width(int E) { return 2 * E + 3; }

// ------------------------------------------------------------------ routing
// logits = x(fp32) . W_router (fp32) -- the reference promotes the bf16
// activations to fp32 -- softmax probabilities, the top-k logits (ties: lower
// expert first, like lax.top_k) and the gates (softmax of the chosen logits).
// EP = E rounded up to a power of two (at least 4), TPG = 32 / EP tokens per
// warp step. Lane l owns the 8-feature chunks l, l + 32, ... of the step's
// TPG tokens and accumulates all TPG x EP dot products (each chunk of W read
// once from shared memory for the whole step); one transposing butterfly
// reduction (31 shuffles) then leaves lane l with the logit of token l / EP,
// expert l % EP, so each group of EP lanes finishes one token (softmax,
// entropy, top-k by group arg-max) with shuffles inside the group.
// Statistics are accumulated per lane, combined per block in warp order and
// added to `stats` with one atomic per block.

// Arg-max over the aligned groups of `width` lanes; ties go to the lower index.
template <int width>
__device__ __forceinline__ void group_argmax(float& v, int& i) {
#pragma unroll
  for (int o = width / 2; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}
template <int width>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = width / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <int width>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = width / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <int EP>
__global__ void __launch_bounds__(256) moe_route_kernel(
    const bf16* __restrict__ x, const float* __restrict__ w, int64_t n, int d, int E, int k,
    float* __restrict__ logits, int* __restrict__ chosen, float* __restrict__ gate,
    float* __restrict__ stats) {
  constexpr int TPG = 32 / EP;
  // Router weights as float4 [EP][2][d / 8] (experts past E are zero): expert
  // e's features 8c..8c+3 at [e][0][c], 8c+4..8c+7 at [e][1][c], so the 32
  // lanes of a warp (chunks c, c+1, ...) read 32 consecutive 16-byte words;
  // then [8 warps][stat width] statistics.
  extern __shared__ float wsm[];
  const int width = moe_stat_width(E);
  const int nch = d / 8;
  float* wst = wsm + (size_t)d * EP;
  for (int i = threadIdx.x; i < d * EP; i += blockDim.x) {
    const int f = i / EP, e = i - f * EP;
    wsm[(((size_t)e * 2 + ((f >> 2) & 1)) * nch + (f >> 3)) * 4 + (f & 3)] =
        e < E ? w[(size_t)f * E + e] : 0.f;
  }
  const float4* w4 = reinterpret_cast<const float4*>(wsm);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int my_e = lane % EP, my_j = lane / EP;
  // per-lane statistics: expert my_e's probability sum and count; the entropy,
  // top-1 gate and squared-logit sums in the lanes with my_e == 0
  float st_prob = 0.f, st_cnt = 0.f, st_ent = 0.f, st_top1 = 0.f, st_sq = 0.f;
  __syncthreads();
  const int64_t groups = (n + TPG - 1) / TPG;
  for (int64_t gi = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp; gi < groups;
       gi += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t t0 = gi * TPG;
    float acc[TPG * EP];
#pragma unroll
    for (int i = 0; i < TPG * EP; ++i) acc[i] = 0.f;
    for (int c = lane; c < nch; c += 32) {
      float a[TPG][8];
#pragma unroll
      for (int j = 0; j < TPG; ++j) {
        const int64_t t = t0 + j < n ? t0 + j : n - 1;
        const uint4 q = *reinterpret_cast<const uint4*>(x + t * d + c * 8);
        const uint32_t* qw = &q.x;
#pragma unroll
        for (int h = 0; h < 4; ++h) unpack_bf16x2(qw[h], a[j][2 * h], a[j][2 * h + 1]);
      }
#pragma unroll
      for (int e = 0; e < EP; ++e) {
        const float4 w0 = w4[(size_t)(e * 2) * nch + c], w1 = w4[(size_t)(e * 2 + 1) * nch + c];
#pragma unroll
        for (int j = 0; j < TPG; ++j) {
          float s = acc[j * EP + e];
          s = fmaf(a[j][0], w0.x, s);
          s = fmaf(a[j][1], w0.y, s);
          s = fmaf(a[j][2], w0.z, s);
          s = fmaf(a[j][3], w0.w, s);
          s = fmaf(a[j][4], w1.x, s);
          s = fmaf(a[j][5], w1.y, s);
          s = fmaf(a[j][6], w1.z, s);
          s = fmaf(a[j][7], w1.w, s);
          acc[j * EP + e] = s;
        }
      }
    }
    // transposing butterfly: after the step with offset o, a lane keeps the
    // half of its values whose index bit o matches its own lane bit
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < o; ++i) {
        const float send = upper ? acc[i] : acc[i + o];
        const float keep = upper ? acc[i + o] : acc[i];
        acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    const int64_t t = t0 + my_j;
    const bool tok = t < n;
    const bool live = tok && my_e < E;
    const float lg = live ? acc[0] : -INFINITY;
    if (live) logits[t * E + my_e] = lg;
    const float mx = group_max<EP>(lg);
    const float ex = live ? expf(lg - mx) : 0.f;
    const float z = group_sum<EP>(ex);
    const float pr = tok ? ex / z : 0.f;
    const float ent = group_sum<EP>(live ? -pr * logf(pr + 1.0e-9f) : 0.f);
    const float sq = group_sum<EP>(live ? lg * lg : 0.f);
    // top-k by repeated group arg-max; the first (lowest) expert wins ties
    float cur = lg;
    float l0 = 0.f, gz = 0.f, mygate_logit = -INFINITY;
    int mysel = -1;
    for (int jj = 0; jj < k; ++jj) {
      float v = cur;
      int i = live ? my_e : 1 << 30;
      group_argmax<EP>(v, i);
      if (jj == 0) l0 = v;
      gz += expf(v - l0);
      if (my_e == jj) {
        mysel = i;
        mygate_logit = v;
      }
      if (my_e == i) {
        cur = -INFINITY;
        if (live) st_cnt += 1.f;
      }
    }
    // lanes my_e = 0..k-1 hold choice my_e; the first choice has the largest gate
    if (tok && my_e < k) {
      chosen[t * k + my_e] = mysel;
      gate[t * k + my_e] = expf(mygate_logit - l0) / gz;
    }
    if (live) st_prob += pr;
    if (tok && my_e == 0) {
      st_ent += ent;
      st_top1 += 1.f / gz;  // the first gate, exp(0) / gz
      st_sq += sq;
    }
  }
  // lanes with the same expert combine, then per warp, then the warps in order
#pragma unroll
  for (int o = EP; o < 32; o <<= 1) {
    st_prob += __shfl_xor_sync(0xffffffffu, st_prob, o);
    st_cnt += __shfl_xor_sync(0xffffffffu, st_cnt, o);
    st_ent += __shfl_xor_sync(0xffffffffu, st_ent, o);
    st_top1 += __shfl_xor_sync(0xffffffffu, st_top1, o);
    st_sq += __shfl_xor_sync(0xffffffffu, st_sq, o);
  }
  float* mine = wst + warp * width;
  if (lane < E) {
    mine[lane] = st_prob;
    mine[E + lane] = st_cnt;
  }
  if (lane == 0) {
    mine[2 * E] = st_ent;
    mine[2 * E + 1] = st_top1;
    mine[2 * E + 2] = st_sq;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    float s = 0.f;
    for (int w8 = 0; w8 < (int)(blockDim.x >> 5); ++w8) s += wst[w8 * width + i];
    atomicAdd(&stats[i], s);
  }
}

// ------------------------------------------------------------------ dispatch
// Stable counting sort of the assignments by expert. Pass 1: per-block
// counts. Pass 2 (one block): segment offsets (counts rounded up to 128) and
// each block's starting rank per expert. Pass 3: per-warp ballots give each
// assignment its rank among equal experts in flat order.
__global__ void __launch_bounds__(256) moe_count_kernel(const int* __restrict__ chosen,
                                                        int64_t na, int E,
                                                        int* __restrict__ block_counts) {
  __shared__ int c[kMoeMaxE];
  if (threadIdx.x < E) c[threadIdx.x] = 0;
  __syncthreads();
  const int64_t a0 = (int64_t)blockIdx.x * kDispatchBlock;
  for (int64_t a = a0 + threadIdx.x; a < min(na, a0 + kDispatchBlock); a += blockDim.x)
    atomicAdd(&c[chosen[a]], 1);
  __syncthreads();
  if (threadIdx.x < E) block_counts[(int64_t)blockIdx.x * E + threadIdx.x] = c[threadIdx.x];
}

__global__ void moe_offsets_kernel(int* __restrict__ block_counts, int nblocks, int E,
                                   int2* __restrict__ seg, int* __restrict__ total) {
  // thread e scans expert e's column of block counts (in place: exclusive)
  __shared__ int cnt[kMoeMaxE];
  const int e = threadIdx.x;
  if (e < E) {
    int run = 0;
    for (int b = 0; b < nblocks; ++b) {
      const int v = block_counts[(int64_t)b * E + e];
      block_counts[(int64_t)b * E + e] = run;
      run += v;
    }
    cnt[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0;
    for (int x = 0; x < E; ++x) {
      const int padded = (cnt[x] + 127) / 128 * 128;
      seg[x] = make_int2(off, padded);
      off += padded;
    }
    *total = off;
  }
}

__global__ void __launch_bounds__(kDispatchBlock) moe_place_kernel(
    const int* __restrict__ chosen, int64_t na, int E, int k,
    const int* __restrict__ block_base, const int2* __restrict__ seg, int* __restrict__ pos,
    int* __restrict__ src) {
  __shared__ int wc[kDispatchBlock / 32][kMoeMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t a = (int64_t)blockIdx.x * kDispatchBlock + threadIdx.x;
  const int ex = a < na ? chosen[a] : -1;
  int rank = 0;
  for (int e = 0; e < E; ++e) {
    const unsigned m = __ballot_sync(0xffffffffu, ex == e);
    if (ex == e) rank = __popc(m & ((1u << lane) - 1u));
    if (lane == 0) wc[warp][e] = __popc(m);
  }
  __syncthreads();
  if (threadIdx.x < E) {  // exclusive scan over the block's warps, expert = thread
    int run = 0;
    for (int w = 0; w < kDispatchBlock / 32; ++w) {
      const int v = wc[w][threadIdx.x];
      wc[w][threadIdx.x] = run;
      run += v;
    }
  }
  __syncthreads();
  if (ex >= 0) {
    const int p = seg[ex].x + block_base[(int64_t)blockIdx.x * E + ex] + wc[warp][ex] + rank;
    pos[a] = p;
    src[p] = (int)(a / k);
  }
}

// grouped[r] = x[src[r]] (zeros on padding rows), rows < total.
__global__ void moe_gather_kernel(const bf16* __restrict__ x, const int* __restrict__ src,
                                  const int* __restrict__ total, int d, bf16* __restrict__ out) {
  const int64_t rows = *total;
  const int nch = d / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * nch;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nch;
    const int c = (int)(i - r * nch);
    const int s = src[r];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (s >= 0) v = *reinterpret_cast<const uint4*>(x + (int64_t)s * d + c * 8);
    *reinterpret_cast<uint4*>(out + r * d + c * 8) = v;
  }
}

// ------------------------------------------------------------------ combine
// x_out[i] = resid[i] + alpha * sum_j bf16(out[pos(i,j)] * bf16(gate(i,j))),
// each product and sum rounded to bf16 as the reference's bf16 scatter-add.
__global__ void moe_combine_kernel(const bf16* __restrict__ out, const int* __restrict__ pos,
                                   const float* __restrict__ gate, const bf16* __restrict__ resid,
                                   float alpha, int64_t n, int d, int k,
                                   bf16* __restrict__ x_out) {
  const int nch = d / 8;
  const uint32_t al = pack_bf16x2(alpha, alpha);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n * nch;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nch;
    const int c = (int)(i - t * nch);
    uint32_t acc[4] = {0u, 0u, 0u, 0u};
    for (int j = 0; j < k; ++j) {
      const float g = gate[t * k + j];
      const uint32_t gb = pack_bf16x2(g, g);
      const uint4 o = *reinterpret_cast<const uint4*>(out + (int64_t)pos[t * k + j] * d + c * 8);
      const uint32_t* ow = &o.x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w = hmul2_bf16(ow[q], gb);
        acc[q] = j == 0 ? w : hadd2_bf16(acc[q], w);
      }
    }
    const uint4 rq = *reinterpret_cast<const uint4*>(resid + t * d + c * 8);
    const uint32_t* rw = &rq.x;
    uint4 res;
    uint32_t* ow = &res.x;
#pragma unroll
    for (int q = 0; q < 4; ++q) ow[q] = hadd2_bf16(rw[q], hmul2_bf16(acc[q], al));
    *reinterpret_cast<uint4*>(x_out + t * d + c * 8) = res;
  }
}

// Backward of the combine: d_mlp = bf16(alpha * dx); d_out[pos(i,j)] =
// bf16(d_mlp * bf16(gate)); d_gate(i,j) = bf16-rounded sum_d d_mlp * out.
// One warp per token; a lane owns the 8-column chunks lane, lane + 32, ...,
// taken kCbChunks at a time with all their row reads issued before the math.
// Padding rows of d_out are zeroed by moe_zero_pad_kernel.
constexpr int kCbChunks = 3;
__global__ void __launch_bounds__(256) moe_combine_bwd_kernel(
    const bf16* __restrict__ dx, float alpha, const bf16* __restrict__ out,
    const int* __restrict__ pos, const float* __restrict__ gate, int64_t n, int d, int k,
    bf16* __restrict__ d_out, float* __restrict__ d_gate) {
  const int lane = threadIdx.x & 31;
  const int nch = d / 8;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const uint32_t al = pack_bf16x2(alpha, alpha);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < n;
       t += warps) {
    int64_t r[kMoeMaxK];
    uint32_t gb[kMoeMaxK];
    float dg[kMoeMaxK];
#pragma unroll
    for (int j = 0; j < kMoeMaxK; ++j) {
      dg[j] = 0.f;
      if (j < k) {
        r[j] = pos[t * k + j];
        const float g = gate[t * k + j];
        gb[j] = pack_bf16x2(g, g);
      }
    }
    for (int cb = 0; cb < nch; cb += 32 * kCbChunks) {
    uint4 q[kCbChunks], o[kCbChunks][kMoeMaxK];
#pragma unroll
    for (int i = 0; i < kCbChunks; ++i) {
      const int c = cb + lane + 32 * i;
      if (c < nch) {
        q[i] = *reinterpret_cast<const uint4*>(dx + t * d + c * 8);
#pragma unroll
        for (int j = 0; j < kMoeMaxK; ++j)
          if (j < k) o[i][j] = *reinterpret_cast<const uint4*>(out + r[j] * d + c * 8);
      }
    }
#pragma unroll
    for (int i = 0; i < kCbChunks; ++i) {
      const int c = cb + lane + 32 * i;
      if (c >= nch) break;
      const uint32_t* qw = &q[i].x;
      uint32_t dm[4];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) dm[q4] = hmul2_bf16(qw[q4], al);
#pragma unroll
      for (int j = 0; j < kMoeMaxK; ++j) {
        if (j >= k) break;
        const uint32_t* ow = &o[i][j].x;
        uint4 w;
        uint32_t* ww = &w.x;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          ww[q4] = hmul2_bf16(dm[q4], gb[j]);
          float a0, a1, b0, b1;
          unpack_bf16x2(dm[q4], a0, a1);
          unpack_bf16x2(ow[q4], b0, b1);
          dg[j] = fmaf(a0, b0, fmaf(a1, b1, dg[j]));
        }
        *reinterpret_cast<uint4*>(d_out + r[j] * d + c * 8) = w;
      }
    }
    }
#pragma unroll
    for (int j = 0; j < kMoeMaxK; ++j) {
      if (j >= k) break;
      const float s = warp_sum(dg[j]);
      if (lane == 0) d_gate[t * k + j] = bf16r(s);
    }
  }
}

// Zeroes the padding rows (src < 0) of a grouped buffer: one thread per row.
__global__ void moe_zero_pad_kernel(const int* __restrict__ src, const int* __restrict__ total,
                                    int d, bf16* __restrict__ buf) {
  const int64_t rows = *total;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows;
       r += (int64_t)gridDim.x * blockDim.x) {
    if (src[r] >= 0) continue;
    uint4* row = reinterpret_cast<uint4*>(buf + r * d);
    for (int c = 0; c < d / 8; ++c) row[c] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// ------------------------------------------------------------------ router backward
// d_logits from the gates (softmax of the chosen logits) and from the balance
// loss through the router probabilities (d prob_e = bal[e], the same for every
// token); then d_x = bf16(bf16(sum_j d_grouped[pos(i,j)]) + bf16(d_logits . W^T))
// and d_W += x^T d_logits. Tokens go in chunks of 64: the first 64 threads
// form the chunk's d_logits in shared memory (a thread per token); then thread (stream s,
// group g) owns features [FPT g, FPT g + FPT) -- their weights and d_W
// partials in registers -- and takes tokens s, s + S, ... of the chunk with
// 8- or 16-byte row reads. At the end the S streams' d_W partials are added in
// stream order in shared memory and the block adds them with one atomic each.
constexpr int kRbChunk = 64;
constexpr int kRbMaxThreads = 512;  // 128 registers a thread
// tokens whose row reads a thread has in flight (fewer for wider rows, so the
// weights and partials stay in registers)
__host__ __device__ constexpr int rb_unroll(int fpt) { return fpt == 2 ? 4 : (fpt == 4 ? 3 : 2); }

template <int FPT>
struct RbVec;
template <>
struct RbVec<8> {
  using T = uint4;
};
template <>
struct RbVec<4> {
  using T = uint2;
};
template <>
struct RbVec<2> {
  using T = uint32_t;
};

template <int FPT>
__device__ __forceinline__ void rb_unpack(const typename RbVec<FPT>::T& q, float* f) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&q);
#pragma unroll
  for (int h = 0; h < FPT / 2; ++h) unpack_bf16x2(w[h], f[2 * h], f[2 * h + 1]);
}

template <int E, int FPT>
__global__ void __launch_bounds__(kRbMaxThreads, 1) moe_route_bwd_kernel(
    const bf16* __restrict__ x, const float* __restrict__ w, const float* __restrict__ logits,
    const int* __restrict__ chosen, const float* __restrict__ gate,
    const float* __restrict__ d_gate, const float* __restrict__ bal,
    const bf16* __restrict__ d_grouped, const int* __restrict__ pos, int64_t n, int d, int k,
    int streams, float* __restrict__ d_w, bf16* __restrict__ d_x) {
  using Vec = typename RbVec<FPT>::T;
  extern __shared__ float dwsum[];  // [d][E] d_W partial of the block
  __shared__ float dl[kRbChunk][E];
  __shared__ int ps[kRbChunk][kMoeMaxK];
  const int groups = d / FPT;
  const int stream = threadIdx.x / groups, g = threadIdx.x - stream * groups;
  const bool active = stream < streams;
  const int f0 = g * FPT;
  float wreg[FPT][E], acc[FPT][E];
#pragma unroll
  for (int i = 0; i < FPT; ++i)
#pragma unroll
    for (int e = 0; e < E; ++e) {
      wreg[i][e] = active ? w[(int64_t)(f0 + i) * E + e] : 0.f;
      acc[i][e] = 0.f;
    }
  for (int64_t c0 = (int64_t)blockIdx.x * kRbChunk; c0 < n; c0 += (int64_t)gridDim.x * kRbChunk) {
    const int nt = (int)(n - c0 < kRbChunk ? n - c0 : kRbChunk);
    // (a) d_logits of the chunk: one thread per token, all experts in registers
    for (int tt = threadIdx.x; tt < nt; tt += blockDim.x) {
      const int64_t t = c0 + tt;
      float lg[E], pr[E];
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        lg[e] = logits[t * E + e];
        mx = fmaxf(mx, lg[e]);
      }
      float z = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        pr[e] = expf(lg[e] - mx);
        z += pr[e];
      }
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        pr[e] = pr[e] / z;
        dot += pr[e] * bal[e];
      }
      float gt[kMoeMaxK], dgt[kMoeMaxK];
      int ch[kMoeMaxK];
      float gd = 0.f;
#pragma unroll
      for (int j = 0; j < kMoeMaxK; ++j) {
        if (j < k) {
          gt[j] = gate[t * k + j];
          dgt[j] = d_gate[t * k + j];
          ch[j] = chosen[t * k + j];
          ps[tt][j] = pos[t * k + j];
          gd += gt[j] * dgt[j];
        }
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float gg = pr[e] * (bal[e] - dot);
#pragma unroll
        for (int j = 0; j < kMoeMaxK; ++j)
          if (j < k && ch[j] == e) gg += gt[j] * (dgt[j] - gd);
        dl[tt][e] = gg;
      }
    }
    __syncthreads();
    // (b) d_W partials and d_x, FPT features of one token per step; a thread
    // issues the row reads of rb_unroll(FPT) of its tokens before their math (the
    // tokens still enter the partials in order s, s + S, s + 2S, ...)
    if (active) {
      for (int tb = stream; tb < nt; tb += streams * rb_unroll(FPT)) {
        constexpr int U = rb_unroll(FPT);
        Vec xq[U], gq[U][kMoeMaxK];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int tt = tb + u * streams;
          if (tt < nt) {
            const int64_t t = c0 + tt;
            xq[u] = *reinterpret_cast<const Vec*>(x + t * d + f0);
#pragma unroll
            for (int j = 0; j < kMoeMaxK; ++j)
              if (j < k) gq[u][j] = *reinterpret_cast<const Vec*>(d_grouped + (int64_t)ps[tt][j] * d + f0);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int tt = tb + u * streams;
          if (tt >= nt) break;
          const int64_t t = c0 + tt;
          float xv[FPT];
          rb_unpack<FPT>(xq[u], xv);
          Vec g0 = gq[u][0];
#pragma unroll
          for (int j = 1; j < kMoeMaxK; ++j) {
            if (j >= k) break;
            uint32_t* a32 = reinterpret_cast<uint32_t*>(&g0);
            const uint32_t* o32 = reinterpret_cast<const uint32_t*>(&gq[u][j]);
#pragma unroll
            for (int h = 0; h < FPT / 2; ++h) a32[h] = hadd2_bf16(a32[h], o32[h]);
          }
          float v[FPT];
#pragma unroll
          for (int i = 0; i < FPT; ++i) v[i] = 0.f;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const float de = dl[tt][e];
#pragma unroll
            for (int i = 0; i < FPT; ++i) {
              acc[i][e] = fmaf(xv[i], de, acc[i][e]);
              v[i] = fmaf(de, wreg[i][e], v[i]);
            }
          }
          Vec out;
          uint32_t* o32 = reinterpret_cast<uint32_t*>(&out);
          const uint32_t* g32 = reinterpret_cast<const uint32_t*>(&g0);
#pragma unroll
          for (int h = 0; h < FPT / 2; ++h)
            o32[h] = hadd2_bf16(g32[h], pack_bf16x2(v[2 * h], v[2 * h + 1]));
          *reinterpret_cast<Vec*>(d_x + t * d + f0) = out;
        }
      }
    }
    __syncthreads();
  }
  // d_W: the streams' partials added in stream order, then one atomic each
  for (int s = 0; s < streams; ++s) {
    if (active && stream == s) {
#pragma unroll
      for (int i = 0; i < FPT; ++i)
#pragma unroll
        for (int e = 0; e < E; ++e) {
          float* dst = &dwsum[(f0 + i) * E + e];
          *dst = s == 0 ? acc[i][e] : *dst + acc[i][e];
        }
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < d * E; i += blockDim.x) atomicAdd(&d_w[i], dwsum[i]);
}

// out[e][c] += sum of buf rows [seg[e].x, seg[e].x + seg[e].y), column c.
// A thread owns 8 consecutive columns (16-byte row reads, four rows in flight)
// of one of gridDim.z row chunks of the segment; the chunk's sums (rows added
// in order) go to `out` with one atomic per column. width % 8 == 0.
__global__ void __launch_bounds__(128) moe_seg_colsum_kernel(const bf16* __restrict__ buf,
                                                             const int2* __restrict__ seg, int w,
                                                             float* __restrict__ out) {
  const int e = blockIdx.y;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= w) return;
  const int2 sg = seg[e];
  const int chunk = (sg.y + gridDim.z - 1) / gridDim.z;
  const int r0 = sg.x + blockIdx.z * chunk, r1 = min(sg.x + sg.y, r0 + chunk);
  float s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = 0.f;
  int r = r0;
  for (; r + 4 <= r1; r += 4) {
    uint4 q[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) q[u] = *reinterpret_cast<const uint4*>(buf + (int64_t)(r + u) * w + c0);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t* qw = &q[u].x;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float a, b;
        unpack_bf16x2(qw[h], a, b);
        s[2 * h] += a;
        s[2 * h + 1] += b;
      }
    }
  }
  for (; r < r1; ++r) {
    const uint4 q = *reinterpret_cast<const uint4*>(buf + (int64_t)r * w + c0);
    const uint32_t* qw = &q.x;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      float a, b;
      unpack_bf16x2(qw[h], a, b);
      s[2 * h] += a;
      s[2 * h + 1] += b;
    }
  }
  if (r1 > r0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(&out[(int64_t)e * w + c0 + j], s[j]);
  }
}

// ------------------------------------------------------------------ statistics
// After the per-rank statistics have been summed over ranks: per layer load
// = count / (tokens * k), mean probability = prob sum / tokens, balance =
// E * sum(load * mean prob) (recipes/reference_moe/train.py:1347-1372), the
// backward coefficient of each router probability, the router history row
// (train.py:1881-1915) and loss += coef * mean balance.
__global__ void moe_finalize_kernel(const float* __restrict__ stats, int layers, int E,
                                    float tokens, int k, float coef, float bwd_scale,
                                    float* __restrict__ bal_grad, float* __restrict__ loss,
                                    float* __restrict__ history, int history_rows,
                                    const int* __restrict__ step) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  // this step's row: the optimizer's step counter before its increment
  const int s = *step;
  float scratch[6 + 64 * (3 + kMoeMaxE)];
  const int width = 6 + layers * (3 + E);
  float* row = (s >= 0 && s < history_rows) ? history + (int64_t)s * width : scratch;
  if (row == scratch && layers > 64) return;
  const int W = moe_stat_width(E);
  float bal_sum = 0.f, lmax = -INFINITY, lmin = INFINITY, sm0 = 0.f, sm1 = 0.f, sm2 = 0.f;
  for (int l = 0; l < layers; ++l) {
    const float* s = stats + (size_t)l * W;
    float b = 0.f;
    for (int e = 0; e < E; ++e) {
      const float load = s[E + e] / (tokens * (float)k);
      const float mp = s[e] / tokens;
      b += load * mp;
      lmax = fmaxf(lmax, load);
      lmin = fminf(lmin, load);
      bal_grad[l * E + e] = coef / (float)layers * (float)E * load * bwd_scale;
    }
    bal_sum += (float)E * b;
    const float ent = s[2 * E] / tokens, top1 = s[2 * E + 1] / tokens;
    const float rms = sqrtf(s[2 * E + 2] / (tokens * (float)E));
    sm0 += ent;
    sm1 += top1;
    sm2 += rms;
    float* pl = row + 6 + l * (3 + E);
    pl[0] = ent;
    pl[1] = top1;
    pl[2] = rms;
    for (int e = 0; e < E; ++e) pl[3 + e] = s[E + e] / (tokens * (float)k);
  }
  const float balance = bal_sum / (float)layers;
  row[0] = balance;
  row[1] = lmax;
  row[2] = lmin;
  row[3] = sm0 / (float)layers;
  row[4] = sm1 / (float)layers;
  row[5] = sm2 / (float)layers;
  if (coef != 0.f) *loss += coef * balance;
}

}  // namespace gptb200

using namespace gptb200;

extern "C" size_t gptb200_moe_rows(int64_t tokens, int32_t top_k, int32_t experts) {
  if (tokens <= 0 || top_k <= 0 || experts <= 0) return 0;
  return (size_t)((tokens * top_k + (int64_t)experts * 127 + 127) / 128 * 128);
}

extern "C" size_t gptb200_moe_dispatch_workspace_size(int64_t tokens, int32_t top_k,
                                                      int32_t experts) {
  if (tokens <= 0 || top_k <= 0 || experts <= 0) return 0;
  const int64_t nblocks = (tokens * top_k + kDispatchBlock - 1) / kDispatchBlock;
  return (size_t)(nblocks * experts * 4 + 256);
}

extern "C" int gptb200_moe_route(const void* x, const float* router_w, int64_t tokens,
                                 int64_t d, int32_t experts, int32_t top_k, float* logits,
                                 int32_t* chosen, float* gate, float* stats, void* stream) {
  if (!x || !router_w || !logits || !chosen || !gate || !stats || tokens <= 0) return GPTB200_EINVAL;
  if (experts < 1 || experts > kMoeMaxE || top_k < 1 || top_k > kMoeMaxK || top_k > experts)
    return GPTB200_EUNSUPPORTED;
  const int ep = experts <= 4 ? 4 : (experts <= 8 ? 8 : 16);
  const size_t smem = (size_t)(d * ep + 8 * moe_stat_width(experts)) * 4;
  if (d % 8 || smem > 200 * 1024) return GPTB200_ESHAPE;
  if (reinterpret_cast<uintptr_t>(x) & 15) return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tpg = 32 / ep;
  const int blocks = (int)std::min<int64_t>((tokens + 8 * tpg - 1) / (8 * tpg), (int64_t)sms * 4);
  auto run = [&](auto kern) -> int {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return -static_cast<int>(e);
    }
    kern<<<blocks, 256, smem, st>>>(reinterpret_cast<const bf16*>(x), router_w, tokens, (int)d,
                                    experts, top_k, logits, chosen, gate, stats);
    return 0;
  };
  const int status = ep == 4 ? run(moe_route_kernel<4>)
                             : (ep == 8 ? run(moe_route_kernel<8>) : run(moe_route_kernel<16>));
  if (status) return status;
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" int gptb200_moe_dispatch(const int32_t* chosen, int64_t tokens, int32_t top_k,
                                    int32_t experts, const void* x, int64_t d, int32_t* seg,
                                    int32_t* total, int32_t* pos, int32_t* src, void* grouped,
                                    void* workspace, void* stream) {
  if (!chosen || !x || !seg || !total || !pos || !src || !grouped || !workspace || tokens <= 0)
    return GPTB200_EINVAL;
  if (experts < 1 || experts > kMoeMaxE || top_k < 1 || top_k > kMoeMaxK) return GPTB200_EUNSUPPORTED;
  if (d % 8) return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t na = tokens * top_k;
  const int nblocks = (int)((na + kDispatchBlock - 1) / kDispatchBlock);
  int* bc = reinterpret_cast<int*>(workspace);
  const int64_t rows = (int64_t)gptb200_moe_rows(tokens, top_k, experts);
  cudaError_t e = cudaMemsetAsync(src, 0xff, (size_t)rows * 4, st);  // -1: padding
  if (e != cudaSuccess) return -static_cast<int>(e);
  moe_count_kernel<<<nblocks, 256, 0, st>>>(chosen, na, experts, bc);
  GPTB200_CHECK_LAUNCH();
  moe_offsets_kernel<<<1, 32, 0, st>>>(bc, nblocks, experts, reinterpret_cast<int2*>(seg), total);
  GPTB200_CHECK_LAUNCH();
  moe_place_kernel<<<nblocks, kDispatchBlock, 0, st>>>(chosen, na, experts, top_k, bc,
                                                       reinterpret_cast<const int2*>(seg), pos,
                                                       src);
  GPTB200_CHECK_LAUNCH();
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  moe_gather_kernel<<<sms * 8, 256, 0, st>>>(reinterpret_cast<const bf16*>(x), src, total, (int)d,
                                             reinterpret_cast<bf16*>(grouped));
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" int gptb200_moe_combine(const void* out, const int32_t* pos, const float* gate,
                                   const void* residual, float alpha, int64_t tokens, int64_t d,
                                   int32_t top_k, void* x_out, void* stream) {
  if (!out || !pos || !gate || !residual || !x_out || tokens <= 0) return GPTB200_EINVAL;
  if (top_k < 1 || top_k > kMoeMaxK) return GPTB200_EUNSUPPORTED;
  if (d % 8) return GPTB200_ESHAPE;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  moe_combine_kernel<<<sms * 8, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const bf16*>(out), pos, gate, reinterpret_cast<const bf16*>(residual),
      alpha, tokens, (int)d, top_k, reinterpret_cast<bf16*>(x_out));
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" int gptb200_moe_combine_bwd(const void* dx, float alpha, const void* out,
                                       const int32_t* pos, const float* gate,
                                       const int32_t* src, const int32_t* total, int64_t tokens,
                                       int64_t d, int32_t top_k, void* d_out, float* d_gate,
                                       void* stream) {
  if (!dx || !out || !pos || !gate || !src || !total || !d_out || !d_gate || tokens <= 0)
    return GPTB200_EINVAL;
  if (top_k < 1 || top_k > kMoeMaxK) return GPTB200_EUNSUPPORTED;
  if (d % 8) return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  moe_combine_bwd_kernel<<<sms * 4, 256, 0, st>>>(
      reinterpret_cast<const bf16*>(dx), alpha, reinterpret_cast<const bf16*>(out), pos, gate,
      tokens, (int)d, top_k, reinterpret_cast<bf16*>(d_out), d_gate);
  GPTB200_CHECK_LAUNCH();
  moe_zero_pad_kernel<<<sms * 4, 256, 0, st>>>(src, total, (int)d, reinterpret_cast<bf16*>(d_out));
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" int gptb200_moe_route_bwd(const void* x, const float* router_w, const float* logits,
                                     const int32_t* chosen, const float* gate,
                                     const float* d_gate, const float* bal_grad,
                                     const void* d_grouped, const int32_t* pos, int64_t tokens,
                                     int64_t d, int32_t experts, int32_t top_k, float* d_router_w,
                                     void* d_x, void* stream) {
  if (!x || !router_w || !logits || !chosen || !gate || !d_gate || !bal_grad || !d_grouped ||
      !pos || !d_router_w || !d_x || tokens <= 0)
    return GPTB200_EINVAL;
  if (experts < 1 || experts > kMoeMaxE || top_k < 1 || top_k > kMoeMaxK) return GPTB200_EUNSUPPORTED;
  if (d % 8 || d > 2048) return GPTB200_ESHAPE;
  // Instantiated for every expert count 1..16 with 8, 4 or 2 features per
  // thread (up to 4, 8, 16 experts) so that a thread's weights and partials
  // (2 x features x experts floats) stay in registers.
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int fpt = experts <= 4 ? 8 : (experts <= 8 ? 4 : 2);
  const int groups = (int)(d / fpt);
  const int streams = std::max(1, std::min(8, kRbMaxThreads / groups));
  const int threads = (groups * streams + 31) / 32 * 32;
  const int blocks = (int)std::min<int64_t>((tokens + kRbChunk - 1) / kRbChunk, (int64_t)sms);
  const size_t smem = (size_t)d * experts * sizeof(float);
  auto st = reinterpret_cast<cudaStream_t>(stream);
  int status = GPTB200_OK;
  auto run = [&](auto kern) {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
      if (e != cudaSuccess) {
        status = -static_cast<int>(e);
        return;
      }
    }
    kern<<<blocks, threads, smem, st>>>(reinterpret_cast<const bf16*>(x), router_w, logits, chosen,
                                        gate, d_gate, bal_grad,
                                        reinterpret_cast<const bf16*>(d_grouped), pos, tokens,
                                        (int)d, top_k, streams, d_router_w,
                                        reinterpret_cast<bf16*>(d_x));
  };
  switch (experts) {
#define GPTB200_ROUTE_BWD_CASE(E) \
  case E: run(moe_route_bwd_kernel<E, (E <= 4 ? 8 : (E <= 8 ? 4 : 2))>); break;
    GPTB200_ROUTE_BWD_CASE(1) GPTB200_ROUTE_BWD_CASE(2) GPTB200_ROUTE_BWD_CASE(3)
    GPTB200_ROUTE_BWD_CASE(4) GPTB200_ROUTE_BWD_CASE(5) GPTB200_ROUTE_BWD_CASE(6)
    GPTB200_ROUTE_BWD_CASE(7) GPTB200_ROUTE_BWD_CASE(8) GPTB200_ROUTE_BWD_CASE(9)
    GPTB200_ROUTE_BWD_CASE(10) GPTB200_ROUTE_BWD_CASE(11) GPTB200_ROUTE_BWD_CASE(12)
    GPTB200_ROUTE_BWD_CASE(13) GPTB200_ROUTE_BWD_CASE(14) GPTB200_ROUTE_BWD_CASE(15)
    GPTB200_ROUTE_BWD_CASE(16)
#undef GPTB200_ROUTE_BWD_CASE
    default: return GPTB200_EUNSUPPORTED;
  }
  if (status) return status;
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" int gptb200_moe_segment_colsum(const void* buf, const int32_t* seg, int32_t experts,
                                          int64_t width, float* out, void* stream) {
  if (!buf || !seg || !out || width <= 0) return GPTB200_EINVAL;
  if (experts < 1 || experts > kMoeMaxE) return GPTB200_EUNSUPPORTED;
  if (width % 8 || (reinterpret_cast<uintptr_t>(buf) & 15)) return GPTB200_ESHAPE;
  dim3 grid((unsigned)((width / 8 + 127) / 128), (unsigned)experts, 128);
  moe_seg_colsum_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const bf16*>(buf), reinterpret_cast<const int2*>(seg), (int)width, out);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" int gptb200_moe_finalize(const float* stats, int32_t layers, int32_t experts,
                                    int64_t tokens, int32_t top_k, float coefficient,
                                    float bwd_scale, float* bal_grad, float* loss,
                                    float* history, int32_t history_rows, const int32_t* step,
                                    void* stream) {
  if (!stats || !bal_grad || !loss || !history || !step || layers <= 0 || tokens <= 0)
    return GPTB200_EINVAL;
  if (experts < 1 || experts > kMoeMaxE || layers > 64) return GPTB200_EUNSUPPORTED;
  moe_finalize_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      stats, layers, experts, (float)tokens, top_k, coefficient, bwd_scale, bal_grad, loss,
      history, history_rows, step);
  GPTB200_CHECK_LAUNCH();
  return 0;
}
