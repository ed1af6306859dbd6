// Fused linear cross-entropy over a tied embedding, built on the tcgen05 GEMM.
//
// Forward: logits tiles (128 tokens x 256 vocab, fp32 in TMEM) are reduced in
// the GEMM epilogue to per-(token, vocab-tile) (max, sum exp) partials and the
// target logit, so the [n, vocab] logits never reach HBM. A combine kernel
// merges the partials into the log-sum-exp and the per-token loss, and a
// one-block kernel forms the mean.
//
// Backward, per chunk of token rows: the logits tile is recomputed and the
// epilogue writes G = (softmax - onehot) * cotangent in bf16 (the logits
// themselves are never stored); then dH = G · E and dE += Gᵀ · H run as two
// more tcgen05 GEMMs. Semantics follow rig/kernels/linear_cross_entropy.py:
// 115-302 (invalid targets: +inf loss and no gradient; rows >= the semantic
// vocabulary get no probability mass and no gradient).
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"

namespace gptb200 {

static int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Partial (max, sum-exp) pairs per row: one per 256-wide vocabulary tile.
static int64_t lce_tiles_n(int64_t v_storage) {
  return (round_up(v_storage, 8) + gemm_tile_n() - 1) / gemm_tile_n();
}

// Rows per backward chunk: bounds the G scratch to chunk * vocab bf16.
static int64_t lce_bwd_chunk(int64_t n) { return std::min<int64_t>(n, 16384); }

__global__ void lce_combine_kernel(const float2* __restrict__ part, int tiles,
                                   const float* __restrict__ tgt, const int32_t* __restrict__ targets,
                                   int64_t n, int v_sem, float* __restrict__ losses,
                                   float* __restrict__ lse_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n) return;
  float m = -INFINITY, s = 0.f;
  const float kLog2e = 1.4426950408889634f;
  for (int t = lane; t < tiles; t += 32) {
    float2 q = part[row * tiles + t];
    if (q.x == -INFINITY) continue;
    float nm = fmaxf(m, q.x);
    s = s * exp2f((m - nm) * kLog2e) + q.y * exp2f((q.x - nm) * kLog2e);
    m = nm;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float om = __shfl_xor_sync(0xffffffffu, m, o);
    float os = __shfl_xor_sync(0xffffffffu, s, o);
    float nm = fmaxf(m, om);
    if (nm == -INFINITY) continue;
    s = s * exp2f((m - nm) * kLog2e) + os * exp2f((om - nm) * kLog2e);
    m = nm;
  }
  if (lane == 0) {
    float lse = m + logf(s);
    lse_out[row] = lse;
    int t = targets[row];
    losses[row] = (t >= 0 && t < v_sem) ? lse - tgt[row] : INFINITY;
  }
}

// Mean of n fp32 values in one block (deterministic order).
__global__ void __launch_bounds__(1024) mean_kernel(const float* __restrict__ x, int64_t n,
                                                    float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) *out = t / (float)n;
  }
}

// out[0] = sum(losses * mask), out[1] = sum(mask), fp32, one block (fixed
// summation order, so repeated evaluations agree bit for bit).
__global__ void __launch_bounds__(1024) masked_sum_kernel(const float* __restrict__ losses,
                                                          const float* __restrict__ mask,
                                                          int64_t n, float* __restrict__ out) {
  __shared__ float red[2][32];
  float s = 0.f, c = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float m = mask[i];
    s += losses[i] * m;
    c += m;
  }
  s = warp_sum(s);
  c = warp_sum(c);
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = s;
    red[1][threadIdx.x >> 5] = c;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const bool live = threadIdx.x < (blockDim.x >> 5);
    float t = live ? red[0][threadIdx.x] : 0.f;
    float u = live ? red[1][threadIdx.x] : 0.f;
    t = warp_sum(t);
    u = warp_sum(u);
    if (threadIdx.x == 0) {
      out[0] = t;
      out[1] = u;
    }
  }
}

}  // namespace gptb200

using namespace gptb200;

extern "C" int gptb200_masked_loss_sum(const float* losses, const float* mask, int64_t n,
                                       float* out, void* stream) {
  if (!losses || !mask || !out || n <= 0) return GPTB200_EINVAL;
  masked_sum_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(losses, mask, n, out);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" size_t gptb200_lce_fwd_workspace_size(int64_t n, int64_t v_storage) {
  if (n <= 0 || v_storage <= 0) return 0;
  return (size_t)round_up(n * lce_tiles_n(v_storage) * (int64_t)sizeof(float2), 256) +
         (size_t)round_up(n * (int64_t)sizeof(float), 256);
}

extern "C" int gptb200_lce_fwd(const void* hidden, const void* embedding, const int32_t* targets,
                               int64_t n, int64_t d, int64_t v_storage, int64_t v_semantic,
                               float* losses, float* lse, float* mean_loss, void* workspace,
                               void* stream) {
  if (!hidden || !embedding || !targets || !losses || !lse || !workspace) return GPTB200_EINVAL;
  if (n <= 0 || d <= 0 || v_storage <= 0) return GPTB200_EINVAL;
  if (v_semantic <= 0 || v_semantic > v_storage) return GPTB200_EINVAL;
  if (d % 8) return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t tiles = lce_tiles_n(v_storage);
  float2* part = reinterpret_cast<float2*>(workspace);
  float* tgt = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                        round_up(n * tiles * (int64_t)sizeof(float2), 256));
  GemmParams p = {};
  p.C = part;  // not stored through; must be non-null and aligned
  p.ldc = round_up(v_storage, 8);
  p.alpha = 1.f;
  p.targets = targets;
  p.partial = part;
  p.tgt_logit = tgt;
  p.v_sem = (int)v_semantic;
  int s = gemm_launch(hidden, 0, d, embedding, 0, d, n, round_up(v_storage, 8), d, EPI_LCE_FWD_, p,
                      st);
  if (s) return s;
  const int wpb = 8;
  lce_combine_kernel<<<(int)((n + wpb - 1) / wpb), wpb * 32, 0, st>>>(
      part, (int)tiles, tgt, targets, n, (int)v_semantic, losses, lse);
  GPTB200_CHECK_LAUNCH();
  if (mean_loss) {
    mean_kernel<<<1, 1024, 0, st>>>(losses, n, mean_loss);
    GPTB200_CHECK_LAUNCH();
  }
  return 0;
}

// ------------------------------------------------------------------ allocation-free forward
// Scratch of gptb200_lce_fwd_noalloc: the per-(row, vocabulary tile) partials
// and the target logits, in a fixed device array instead of a caller
// workspace. Every GPU that loads this library holds these 8 MiB until the
// process exits.
constexpr int64_t kNoAllocPartials = int64_t(1) << 20;   // float2 entries: rows x vocab tiles
constexpr int64_t kNoAllocRows = 16384;                  // target logits
constexpr int64_t kNoAllocBytes = kNoAllocPartials * 8 + kNoAllocRows * 4;
static __device__ __align__(256) unsigned char g_lce_noalloc_scratch[kNoAllocBytes];

// Device address of the scratch array for the current device. In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device (with that device current) and cached.
static void* noalloc_scratch_address(int* status) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *status = -static_cast<int>(e);
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    *status = GPTB200_EUNSUPPORTED;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_lce_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      *status = e != cudaSuccess ? -static_cast<int>(e) : GPTB200_EDEVICE;
      return nullptr;
    }
    addr[dev] = p;
  }
  *status = GPTB200_OK;
  return addr[dev];
}

extern "C" int gptb200_lce_fwd_noalloc(const void* hidden, const void* embedding,
                                       const int32_t* targets, int64_t n, int64_t d,
                                       int64_t v_storage, int64_t v_semantic, float* losses,
                                       float* lse, float* mean_loss, void* stream) {
  if (n <= 0 || v_storage <= 0) return GPTB200_EINVAL;
  const int64_t tiles = lce_tiles_n(v_storage);
  if (n > kNoAllocRows || n * tiles > kNoAllocPartials) return GPTB200_ETOOLARGE;
  int status = GPTB200_OK;
  void* scratch = noalloc_scratch_address(&status);
  if (!scratch) return status;
  // Same layout as the workspace of gptb200_lce_fwd: partials, then (256-byte
  // aligned) the target logits. Both are fully rewritten by every call before
  // they are read, so nothing needs clearing between calls.
  static_assert(kNoAllocPartials * 8 % 256 == 0, "target logits must stay 256-byte aligned");
  return gptb200_lce_fwd(hidden, embedding, targets, n, d, v_storage, v_semantic, losses, lse,
                         mean_loss, scratch, stream);
}

extern "C" size_t gptb200_lce_bwd_workspace_size(int64_t n, int64_t v_storage) {
  if (n <= 0 || v_storage <= 0) return 0;
  return (size_t)round_up(lce_bwd_chunk(n) * round_up(v_storage, 8) * 2, 256);
}

extern "C" int gptb200_lce_bwd(const void* hidden, const void* embedding, const int32_t* targets,
                               const float* lse, const float* dlosses, int64_t n, int64_t d,
                               int64_t v_storage, int64_t v_semantic, void* dhidden,
                               float* dembedding, void* workspace, void* stream) {
  if (!hidden || !embedding || !targets || !lse || !dlosses || !dhidden || !dembedding ||
      !workspace)
    return GPTB200_EINVAL;
  if (n <= 0 || d <= 0 || v_storage <= 0) return GPTB200_EINVAL;
  if (v_semantic <= 0 || v_semantic > v_storage) return GPTB200_EINVAL;
  if (d % 8) return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t vp = round_up(v_storage, 8);
  const int64_t chunk = lce_bwd_chunk(n);
  bf16* G = reinterpret_cast<bf16*>(workspace);
  const bf16* H = reinterpret_cast<const bf16*>(hidden);
  bf16* dH = reinterpret_cast<bf16*>(dhidden);
  for (int64_t r0 = 0; r0 < n; r0 += chunk) {
    const int64_t rows = std::min(chunk, n - r0);
    // 1. G = (softmax(H E^T) - onehot) * cot   [rows, vp] bf16
    GemmParams pg = {};
    pg.C = G;
    pg.ldc = vp;
    pg.alpha = 1.f;
    pg.targets = targets + r0;
    pg.lse = lse + r0;
    pg.cot = dlosses + r0;
    pg.v_sem = (int)v_semantic;
    int s = gemm_launch(H + r0 * d, 0, d, embedding, 0, d, rows, vp, d, EPI_LCE_BWD_, pg, st);
    if (s) return s;
    // 2. dH = G · E     (B = E stored [K=vocab, N=d])
    GemmParams ph = {};
    ph.C = dH + r0 * d;
    ph.ldc = d;
    ph.alpha = 1.f;
    s = gemm_launch(G, 0, vp, embedding, 1, d, rows, d, vp, EPI_BF16_, ph, st);
    if (s) return s;
    // 3. dE += G^T · H  (A = G stored [K=rows, M=vocab], B = H stored [K=rows, N=d])
    GemmParams pe = {};
    pe.C = dembedding;
    pe.ldc = d;
    pe.alpha = 1.f;
    pe.accumulate = 1;
    s = gemm_launch(G, 1, vp, H + r0 * d, 1, d, v_storage, d, rows, EPI_F32_, pe, st);
    if (s) return s;
  }
  return 0;
}
