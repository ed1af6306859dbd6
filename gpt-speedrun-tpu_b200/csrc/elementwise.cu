// Memory-bound kernels of the step: RMSNorm forward/backward, embedding
// gather (the scatter is in embedding.cu), RoPE tables, bias-gradient column sums and the fp32->bf16
// cast. All of them move 16-byte vectors (8 bf16 / 4 fp32) per thread access,
// reduce with warp shuffles and size their grids from the SM count.
#include <algorithm>

#include "common.cuh"

namespace gptb200 {

static int sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

__device__ __forceinline__ void ld8(const bf16* p, float* v) {
  uint4 q = *reinterpret_cast<const uint4*>(p);
  unpack_bf16x2(q.x, v[0], v[1]);
  unpack_bf16x2(q.y, v[2], v[3]);
  unpack_bf16x2(q.z, v[4], v[5]);
  unpack_bf16x2(q.w, v[6], v[7]);
}
__device__ __forceinline__ void st8(bf16* p, const float* v) {
  uint4 q;
  q.x = pack_bf16x2(v[0], v[1]);
  q.y = pack_bf16x2(v[2], v[3]);
  q.z = pack_bf16x2(v[4], v[5]);
  q.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = q;
}

// ------------------------------------------------------------------ RMSNorm
// One warp per row; each lane keeps CH 8-element chunks of the row in
// registers (CH = ceil(d / 256)), so x is read once. A warp takes two rows
// (r and r + warps) per iteration and issues both rows' loads before either
// reduction, so twice as many bytes are in flight per warp.
template <int CH>
__global__ void __launch_bounds__(256, (CH <= 3 ? 4 : 1)) rms_fwd_kernel(const bf16* __restrict__ x,
                                                      const bf16* __restrict__ scale,
                                                      bf16* __restrict__ y,
                                                      float* __restrict__ rstd_out, int64_t rows,
                                                      int d) {
  constexpr int R = CH <= 3 ? 2 : 1;  // wider rows already have enough bytes in flight
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nch = d >> 3;
  for (int64_t r0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r0 < rows;
       r0 += R * warps) {
    uint4 xq[R][CH];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const int64_t r = r0 + u * warps;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int ch = lane + 32 * c;
        xq[u][c] = (r < rows && ch < nch)
                       ? *reinterpret_cast<const uint4*>(x + r * d + ch * 8)
                       : make_uint4(0, 0, 0, 0);
      }
    }
    float ss[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      ss[u] = 0.f;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const uint32_t* w = &xq[u][c].x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float a0, a1;
          unpack_bf16x2(w[j], a0, a1);
          ss[u] += a0 * a0;  // same fma order as a sequential sum over the row
          ss[u] += a1 * a1;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int u = 0; u < R; ++u) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
    }
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const int64_t r = r0 + u * warps;
      if (r >= rows) break;  // warp-uniform
      const float rstd = rsqrtf(ss[u] / (float)d + 1.0e-5f);
      if (lane == 0) rstd_out[r] = rstd;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int ch = lane + 32 * c;
        if (ch < nch) {
          float v[8], sc[8], o[8];
          const uint32_t* w = &xq[u][c].x;
#pragma unroll
          for (int j = 0; j < 4; ++j) unpack_bf16x2(w[j], v[2 * j], v[2 * j + 1]);
          ld8(scale + ch * 8, sc);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = bf16r(v[j] * rstd) * sc[j];
          st8(y + r * d + ch * 8, o);
        }
      }
    }
  }
}

// Backward: dn = dy*scale; xhat = x*rstd;
// dx = rstd * (dn - xhat * mean(dn * xhat)); dscale += dy * bf16(xhat).
// x and dy stay packed (bf16) in registers between the two passes, which keeps
// the register count low enough for full occupancy (the kernel is latency-bound
// on its three input streams); each warp accumulates its dscale partial in its
// own shared-memory row instead of registers.
// A warp takes two of its rows (r and r + warps) per iteration and loads both
// before computing either, so twice the bytes are in flight; the rows still
// enter the per-warp partials in the same order (r, r + warps, r + 2 warps ...).
template <int CH>
__global__ void __launch_bounds__(128, (CH <= 3 ? 4 : 1)) rms_bwd_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ scale, const float* __restrict__ rstd_in,
    const bf16* __restrict__ dy, const bf16* dx_in, bf16* dx_out, float* __restrict__ part,
    bool want_col, int64_t rows, int d) {
  extern __shared__ float red[];  // [2][warps_per_block][d]: dscale, then column sums of dx_out
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int wpb = blockDim.x >> 5;
  const int64_t warps = (int64_t)gridDim.x * wpb;
  const int nch = d >> 3;
  float* myred = red + wib * d;
  float* mycol = red + (wpb + wib) * d;
  for (int i = lane; i < d; i += 32) myred[i] = mycol[i] = 0.f;
  __syncwarp();
  uint4 sc[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int ch = lane + 32 * c;
    sc[c] = (ch < nch) ? *reinterpret_cast<const uint4*>(scale + ch * 8) : make_uint4(0, 0, 0, 0);
  }

  constexpr int R = CH <= 3 ? 2 : 1;
  for (int64_t r0 = (int64_t)blockIdx.x * wpb + wib; r0 < rows; r0 += R * warps) {
    uint4 xq2[R][CH], gq2[R][CH], pq2[R][CH];
    float rstd2[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const int64_t r = r0 + u * warps;
      const bool live = r < rows;
      rstd2[u] = live ? rstd_in[r] : 0.f;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int ch = lane + 32 * c;
        if (live && ch < nch) {
          xq2[u][c] = *reinterpret_cast<const uint4*>(x + r * d + ch * 8);
          gq2[u][c] = *reinterpret_cast<const uint4*>(dy + r * d + ch * 8);
          pq2[u][c] = dx_in ? *reinterpret_cast<const uint4*>(dx_in + r * d + ch * 8)
                            : make_uint4(0, 0, 0, 0);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < R; ++u) {
    const int64_t r = r0 + u * warps;
    if (r >= rows) break;  // warp-uniform
    const float rstd = rstd2[u];
    const uint4* xq = xq2[u];
    const uint4* gq = gq2[u];
    const uint4* pq = pq2[u];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int ch = lane + 32 * c;
      if (ch < nch) {
        const uint32_t* xw = &xq[c].x;
        const uint32_t* gw = &gq[c].x;
        const uint32_t* sw = &sc[c].x;
        float4* acc = reinterpret_cast<float4*>(myred + ch * 8);
        const float4 a0 = acc[0], a1 = acc[1];
        float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float x0, x1, g0, g1, s0, s1;
          unpack_bf16x2(xw[j], x0, x1);
          unpack_bf16x2(gw[j], g0, g1);
          unpack_bf16x2(sw[j], s0, s1);
          const float h0 = x0 * rstd, h1 = x1 * rstd;
          av[2 * j] += g0 * bf16r(h0);
          av[2 * j + 1] += g1 * bf16r(h1);
          dot += g0 * s0 * h0 + g1 * s1 * h1;
        }
        acc[0] = make_float4(av[0], av[1], av[2], av[3]);
        acc[1] = make_float4(av[4], av[5], av[6], av[7]);
      }
    }
    dot = warp_sum(dot) / (float)d;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int ch = lane + 32 * c;
      if (ch < nch) {
        const uint32_t* xw = &xq[c].x;
        const uint32_t* gw = &gq[c].x;
        const uint32_t* sw = &sc[c].x;
        const uint32_t* pw = &pq[c].x;
        uint4 o;
        uint32_t* ow = &o.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float x0, x1, g0, g1, s0, s1, p0, p1;
          unpack_bf16x2(xw[j], x0, x1);
          unpack_bf16x2(gw[j], g0, g1);
          unpack_bf16x2(sw[j], s0, s1);
          unpack_bf16x2(pw[j], p0, p1);
          const float v0 = p0 + bf16r(rstd * (g0 * s0 - x0 * rstd * dot));
          const float v1 = p1 + bf16r(rstd * (g1 * s1 - x1 * rstd * dot));
          ow[j] = pack_bf16x2(v0, v1);
        }
        *reinterpret_cast<uint4*>(dx_out + r * d + ch * 8) = o;
        if (want_col) {  // column sums of the stored (bf16) gradient, for a bias gradient
          float4* cs = reinterpret_cast<float4*>(mycol + ch * 8);
          float4 c0 = cs[0], c1 = cs[1];
          float f[8];
          unpack_bf16x2(ow[0], f[0], f[1]);
          unpack_bf16x2(ow[1], f[2], f[3]);
          unpack_bf16x2(ow[2], f[4], f[5]);
          unpack_bf16x2(ow[3], f[6], f[7]);
          cs[0] = make_float4(c0.x + f[0], c0.y + f[1], c0.z + f[2], c0.w + f[3]);
          cs[1] = make_float4(c1.x + f[4], c1.y + f[5], c1.z + f[6], c1.w + f[7]);
        }
      }
    }
    }
  }
  // Reduce the per-warp partials inside the block (warp order) and store the
  // block's row: part[block][0][:] = dscale partial, part[block][1][:] = column
  // sums. colred_kernel adds the rows in block order, so the result does not
  // depend on which block finished first.
  __syncthreads();
  float* prow = part + (int64_t)blockIdx.x * 2 * d;
  for (int col = threadIdx.x; col < d; col += blockDim.x) {
    float s = 0.f, c = 0.f;
    for (int w = 0; w < wpb; ++w) {
      s += red[w * d + col];
      c += red[(wpb + w) * d + col];
    }
    prow[col] = s;
    prow[d + col] = c;
  }
}

// out_j[c] += alpha_j * sum_p part[p * pstride + j * n + c] for j < nout,
// summed in a fixed order: thread row y adds partials y, y + 16, ... in turn,
// then the 16 row sums are added in y order. Block = 32 columns x 16 rows.
__global__ void __launch_bounds__(512) colred_kernel(const float* __restrict__ part, int nparts,
                                                     int64_t pstride, int n, float* out0,
                                                     float alpha0, float* out1, float alpha1) {
  __shared__ float red[16][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  const int j = blockIdx.y;  // 0: out0, 1: out1
  float s = 0.f;
  if (c < n) {
    const float* src = part + (int64_t)j * n + c;
    int p = threadIdx.y;
#pragma unroll 4
    for (; p < nparts; p += 16) s += __ldg(src + (int64_t)p * pstride);
  }
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < n) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 16; ++y) t += red[y][threadIdx.x];
    if (j == 0) out0[c] += alpha0 * t;
    else out1[c] += alpha1 * t;
  }
}

static int colred_launch(const float* part, int nparts, int64_t pstride, int n, float* out0,
                         float alpha0, float* out1, float alpha1, cudaStream_t st) {
  dim3 grid((n + 31) / 32, out1 ? 2 : 1), block(32, 16);
  colred_kernel<<<grid, block, 0, st>>>(part, nparts, pstride, n, out0, alpha0, out1, alpha1);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

// Blocks of the RMSNorm backward: each ends in one row of 2 x d partials.
static int64_t rms_bwd_blocks(int64_t rows) {
  return std::min<int64_t>((rows + 3) / 4, (int64_t)sms() * 4);
}

template <int CH>
static int rms_fwd_launch(const bf16* x, const bf16* s, bf16* y, float* rstd, int64_t rows, int d,
                          cudaStream_t st) {
  int64_t blocks = std::min<int64_t>((rows + 15) / 16, (int64_t)sms() * 4);
  rms_fwd_kernel<CH><<<(int)blocks, 256, 0, st>>>(x, s, y, rstd, rows, d);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

template <int CH>
static int rms_bwd_launch(const bf16* x, const bf16* s, const float* rstd, const bf16* dy,
                          const bf16* dxi, bf16* dxo, float* dscale, float* dcol, float col_alpha,
                          int64_t rows, int d, float* part, cudaStream_t st) {
  const int threads = 128;
  const int64_t blocks = rms_bwd_blocks(rows);
  size_t smem = 2 * (size_t)(threads / 32) * d * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(rms_bwd_kernel<CH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return -static_cast<int>(e);
  }
  rms_bwd_kernel<CH><<<(int)blocks, threads, smem, st>>>(x, s, rstd, dy, dxi, dxo, part,
                                                       dcol != nullptr, rows, d);
  GPTB200_CHECK_LAUNCH();
  return colred_launch(part, (int)blocks, 2 * (int64_t)d, d, dscale, 1.f, dcol, col_alpha, st);
}

}  // namespace gptb200

using namespace gptb200;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int gptb200_rms_norm_fwd(const void* x, const void* scale, void* y, float* rstd,
                                    int64_t rows, int64_t d, void* stream) {
  if (!x || !scale || !y || !rstd || rows <= 0 || d <= 0) return GPTB200_EINVAL;
  if (d % 8 || d > 4096 || !aligned16(x) || !aligned16(y) || !aligned16(scale)) return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  auto X = reinterpret_cast<const bf16*>(x);
  auto S = reinterpret_cast<const bf16*>(scale);
  auto Y = reinterpret_cast<bf16*>(y);
  int ch = (int)((d / 8 + 31) / 32);
  if (ch <= 1) return rms_fwd_launch<1>(X, S, Y, rstd, rows, (int)d, st);
  if (ch <= 2) return rms_fwd_launch<2>(X, S, Y, rstd, rows, (int)d, st);
  if (ch <= 3) return rms_fwd_launch<3>(X, S, Y, rstd, rows, (int)d, st);
  if (ch <= 4) return rms_fwd_launch<4>(X, S, Y, rstd, rows, (int)d, st);
  if (ch <= 8) return rms_fwd_launch<8>(X, S, Y, rstd, rows, (int)d, st);
  return rms_fwd_launch<16>(X, S, Y, rstd, rows, (int)d, st);
}

extern "C" size_t gptb200_rms_norm_bwd_workspace_size(int64_t rows, int64_t d) {
  if (rows <= 0 || d <= 0) return 0;
  return (size_t)rms_bwd_blocks(rows) * 2 * (size_t)d * sizeof(float);
}

extern "C" int gptb200_rms_norm_bwd(const void* x, const void* scale, const float* rstd,
                                    const void* dy, const void* dx_in, void* dx_out,
                                    float* dscale, float* dx_colsum, float colsum_alpha,
                                    int64_t rows, int64_t d, void* workspace, void* stream) {
  if (!x || !scale || !rstd || !dy || !dx_out || !dscale || !workspace || rows <= 0 || d <= 0)
    return GPTB200_EINVAL;
  if (d % 8 || d > 2048 || !aligned16(x) || !aligned16(dy) || !aligned16(dx_out) ||
      (dx_in && !aligned16(dx_in)))
    return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  auto X = reinterpret_cast<const bf16*>(x);
  auto S = reinterpret_cast<const bf16*>(scale);
  auto DY = reinterpret_cast<const bf16*>(dy);
  auto DXI = reinterpret_cast<const bf16*>(dx_in);
  auto DXO = reinterpret_cast<bf16*>(dx_out);
  auto W = reinterpret_cast<float*>(workspace);
  int ch = (int)((d / 8 + 31) / 32);
  if (ch <= 1) return rms_bwd_launch<1>(X, S, rstd, DY, DXI, DXO, dscale, dx_colsum, colsum_alpha, rows, (int)d, W, st);
  if (ch <= 2) return rms_bwd_launch<2>(X, S, rstd, DY, DXI, DXO, dscale, dx_colsum, colsum_alpha, rows, (int)d, W, st);
  if (ch <= 3) return rms_bwd_launch<3>(X, S, rstd, DY, DXI, DXO, dscale, dx_colsum, colsum_alpha, rows, (int)d, W, st);
  if (ch <= 4) return rms_bwd_launch<4>(X, S, rstd, DY, DXI, DXO, dscale, dx_colsum, colsum_alpha, rows, (int)d, W, st);
  return rms_bwd_launch<8>(X, S, rstd, DY, DXI, DXO, dscale, dx_colsum, colsum_alpha, rows, (int)d, W, st);
}

// ------------------------------------------------------------------ document segments
// out[b, t] = number of boundary tokens in tokens[b, 0..t] (rig/attention.py:
// 205-208): one block per sequence, each thread a contiguous run of positions,
// a block-wide exclusive scan of the run counts, then the running count.
__global__ void __launch_bounds__(256) doc_segments_kernel(const int* __restrict__ tokens,
                                                           int64_t seq, int boundary,
                                                           int* __restrict__ out) {
  __shared__ int part[256];
  const int64_t row = blockIdx.x;
  const int64_t per = (seq + blockDim.x - 1) / blockDim.x;
  const int64_t t0 = threadIdx.x * per, t1 = min(seq, t0 + per);
  const int* tk = tokens + row * seq;
  int n = 0;
  for (int64_t t = t0; t < t1; ++t) n += tk[t] == boundary;
  part[threadIdx.x] = n;
  __syncthreads();
  // inclusive Hillis-Steele scan over the 256 run counts
  for (int o = 1; o < (int)blockDim.x; o <<= 1) {
    const int v = threadIdx.x >= o ? part[threadIdx.x - o] : 0;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  int run = part[threadIdx.x] - n;
  int* o = out + row * seq;
  for (int64_t t = t0; t < t1; ++t) {
    run += tk[t] == boundary;
    o[t] = run;
  }
}

extern "C" int gptb200_document_segments(const int32_t* tokens, int64_t batch, int64_t seq,
                                         int32_t boundary_token, int32_t* out, void* stream) {
  if (!tokens || !out || batch <= 0 || seq <= 0 || batch > INT32_MAX) return GPTB200_EINVAL;
  doc_segments_kernel<<<(unsigned)batch, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      tokens, seq, boundary_token, out);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

// ------------------------------------------------------------------ embedding
static __device__ int g_embed_error;

__global__ void embed_fwd_kernel(const int32_t* __restrict__ tok, const bf16* __restrict__ table,
                                 bf16* __restrict__ out, int64_t n, int d, int64_t vocab) {
  const int nch = d >> 3;
  const int64_t total = n * nch;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / nch;
    int c = (int)(i - r * nch);
    int64_t t = tok[r];
    if (t < 0 || t >= vocab) {
      if (c == 0) atomicCAS(&g_embed_error, 0, kErrTokenRange);
      t = t < 0 ? 0 : vocab - 1;
    }
    *reinterpret_cast<uint4*>(out + r * d + c * 8) =
        *reinterpret_cast<const uint4*>(table + t * d + c * 8);
  }
}

extern "C" int gptb200_embedding_fwd(const int32_t* tokens, const void* table, void* out, int64_t n,
                                     int64_t d, int64_t vocab, void* stream) {
  if (!tokens || !table || !out || n <= 0 || d <= 0 || vocab <= 0) return GPTB200_EINVAL;
  if (d % 8 || !aligned16(table) || !aligned16(out)) return GPTB200_ESHAPE;
  int64_t total = n * (d / 8);
  int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sms() * 16);
  embed_fwd_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      tokens, reinterpret_cast<const bf16*>(table), reinterpret_cast<bf16*>(out), n, (int)d, vocab);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

// ------------------------------------------------------------------ RoPE tables
__global__ void rope_tables_kernel(bf16* cos_out, bf16* sin_out, int64_t seq, int half, int hd) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= seq * half) return;
  int64_t t = i / half;
  int k = (int)(i - t * half);
  // fraction = arange(0, hd, 2) / hd ; inv = 10000^-fraction ; angle = t * inv (all fp32)
  float fraction = (float)(2 * k) / (float)hd;
  float inv = powf(10000.0f, -fraction);
  float angle = (float)t * inv;
  cos_out[i] = __float2bfloat16(cosf(angle));
  sin_out[i] = __float2bfloat16(sinf(angle));
}

extern "C" int gptb200_rope_tables(void* cos_out, void* sin_out, int64_t seq, int64_t head_dim,
                                   void* stream) {
  if (!cos_out || !sin_out || seq <= 0 || head_dim <= 0 || head_dim % 2) return GPTB200_EINVAL;
  int half = (int)(head_dim / 2);
  int64_t total = seq * half;
  rope_tables_kernel<<<(int)((total + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<bf16*>(cos_out), reinterpret_cast<bf16*>(sin_out), seq, half, (int)head_dim);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

// ------------------------------------------------------------------ column sums
// Block = 8 warps. Lane l of every warp owns columns [8l, 8l+8) of a 256-wide
// strip; the warps of the block split the rows of the block's row range
// (blockIdx.y). Each block stores its strip's sums as row blockIdx.y of the
// partials; colred_kernel adds the rows in order (deterministic).
__global__ void __launch_bounds__(256) colsum_kernel(const bf16* __restrict__ x, int64_t rows,
                                                     int n, int64_t rows_per_block,
                                                     float* __restrict__ part) {
  __shared__ float red[8][256];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int col = blockIdx.x * 256 + lane * 8;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
  const int64_t r1 = min(rows, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (col < n) {
    for (int64_t r = r0 + w; r < r1; r += 8) {
      float v[8];
      ld8(x + r * n + col, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[w][lane * 8 + j] = acc[j];
  __syncthreads();
  int c = threadIdx.x;  // 256 threads -> 256 columns of the strip
  if (blockIdx.x * 256 + c < n) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k][c];
    part[(int64_t)blockIdx.y * n + blockIdx.x * 256 + c] = s;
  }
}

// Row split of gptb200_colsum: about 4 blocks per SM, >= 64 rows per block.
static void colsum_split(int64_t rows, int64_t n, int64_t* rpb, int* ysplit) {
  const int strips = (int)((n + 255) / 256);
  const int64_t want = std::max<int64_t>(1, (int64_t)sms() * 4 / strips);
  *rpb = std::max<int64_t>(64, (rows + want - 1) / want);
  *ysplit = (int)((rows + *rpb - 1) / *rpb);
}

extern "C" size_t gptb200_colsum_workspace_size(int64_t rows, int64_t n) {
  if (rows <= 0 || n <= 0) return 0;
  int64_t rpb;
  int ysplit;
  colsum_split(rows, n, &rpb, &ysplit);
  return (size_t)ysplit * (size_t)n * sizeof(float);
}

extern "C" int gptb200_colsum(const void* x, int64_t rows, int64_t n, float alpha, float* out,
                              void* workspace, void* stream) {
  if (!x || !out || !workspace || rows <= 0 || n <= 0) return GPTB200_EINVAL;
  if (n % 8 || !aligned16(x)) return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  int64_t rpb;
  int ysplit;
  colsum_split(rows, n, &rpb, &ysplit);
  dim3 grid((int)((n + 255) / 256), ysplit);
  float* part = reinterpret_cast<float*>(workspace);
  colsum_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const bf16*>(x), rows, (int)n, rpb, part);
  GPTB200_CHECK_LAUNCH();
  return colred_launch(part, ysplit, n, (int)n, out, alpha, nullptr, 0.f, st);
}

// ------------------------------------------------------------------ cast
__global__ void cast_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, int64_t n) {
  int64_t n4 = n >> 2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(src)[i];
    uint2 q;
    q.x = pack_bf16x2(v.x, v.y);
    q.y = pack_bf16x2(v.z, v.w);
    reinterpret_cast<uint2*>(dst)[i] = q;
  }
  int64_t tail = (n4 << 2) + blockIdx.x * blockDim.x + threadIdx.x;
  if (tail < n && blockIdx.x == 0) dst[tail] = __float2bfloat16(src[tail]);
}

extern "C" int gptb200_cast_bf16(const float* src, void* dst, int64_t n, void* stream) {
  if (!src || !dst || n <= 0) return GPTB200_EINVAL;
  if (!aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7)) return GPTB200_ESHAPE;
  int blocks = (int)std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t)sms() * 16);
  cast_bf16_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      src, reinterpret_cast<bf16*>(dst), n);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

// ------------------------------------------------------------------ standalone RoPE
// One thread per 8-element chunk (4 interleaved pairs) of a [b, t, h, 64] view.
__global__ void rope_apply_kernel(bf16* __restrict__ x, int64_t sb, int64_t st, int64_t sh, int B,
                                  int T, int H, int hd, const bf16* __restrict__ rcos,
                                  const bf16* __restrict__ rsin, int inverse) {
  const int cph = hd / 8;
  const int64_t total = (int64_t)B * T * H * cph;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / cph;
    const int c = (int)(i - r * cph);
    const int h = (int)(r % H);
    r /= H;
    const int t = (int)(r % T);
    const int b = (int)(r / T);
    bf16* p = x + b * sb + (int64_t)t * st + h * sh + c * 8;
    float v[8];
    ld8(p, v);
    const bf16* cs = rcos + (int64_t)t * (hd / 2) + c * 4;
    const bf16* sn = rsin + (int64_t)t * (hd / 2) + c * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float cv = __bfloat162float(cs[j]);
      const float sv = inverse ? -__bfloat162float(sn[j]) : __bfloat162float(sn[j]);
      const float e = v[2 * j], o = v[2 * j + 1];
      v[2 * j] = e * cv - o * sv;
      v[2 * j + 1] = e * sv + o * cv;
    }
    st8(p, v);
  }
}

extern "C" int gptb200_rope_apply(void* x, int64_t stride_b, int64_t stride_t, int64_t stride_h,
                                  int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                                  const void* rope_cos, const void* rope_sin, int inverse,
                                  void* stream) {
  if (!x || !rope_cos || !rope_sin || batch <= 0 || seq <= 0 || heads <= 0 || head_dim <= 0)
    return GPTB200_EINVAL;
  if (head_dim % 8 || (stride_b | stride_t | stride_h) % 8 || !aligned16(x)) return GPTB200_ESHAPE;
  const int64_t total = batch * seq * heads * (head_dim / 8);
  int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sms() * 16);
  rope_apply_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<bf16*>(x), stride_b, stride_t, stride_h, (int)batch, (int)seq, (int)heads,
      (int)head_dim, reinterpret_cast<const bf16*>(rope_cos), reinterpret_cast<const bf16*>(rope_sin),
      inverse);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

namespace gptb200 {
int embed_read_error(int clear) {
  int h = 0;
  cudaMemcpyFromSymbol(&h, g_embed_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_embed_error, &z, sizeof(int));
  }
  return h;
}
}  // namespace gptb200
