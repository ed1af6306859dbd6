// CompleteP AdamW over one flat fp32 parameter buffer (three launches):
//   1. sqnorm_partial : per-block partial sums of grad^2 (fixed grid, deterministic)
//   2. adamw_scalars  : one block -> global grad norm, step+1, learning rate
//                       (warmup + cosine, train.py:1219-1236), bias
//                       corrections, clip scale, history row
//   3. adamw_update   : the element-wise m/v/param update with per-tensor
//                       lr/eps/decay multipliers looked up from the group
//                       table, plus the bf16 compute copy of the new params.
// The step counter lives on the device, so a captured CUDA graph of the whole
// step replays correctly.
#include <algorithm>

#include "common.cuh"

namespace gptb200 {

constexpr int kNormBlocks = 1184;  // 8 x 148
constexpr int kNormThreads = 512;

struct AdamScalars {
  float lr;
  float bc1;
  float bc2;
  float gscale;     // grad_scale * clip scale
  float grad_norm;
  int step;
};

__global__ void __launch_bounds__(kNormThreads) sqnorm_partial_kernel(const float* __restrict__ g,
                                                                      int64_t n,
                                                                      double* __restrict__ part) {
  __shared__ double red[kNormThreads / 32];
  double acc = 0.0;
  float accf = 0.f;
  const int64_t n4 = n >> 2;
  int cnt = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(g)[i];
    accf += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    if (++cnt == 64) {
      acc += accf;
      accf = 0.f;
      cnt = 0;
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    float t = g[(n4 << 2) + threadIdx.x];
    accf += t * t;
  }
  acc += accf;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < kNormThreads / 32; ++w) s += red[w];
    part[blockIdx.x] = s;
  }
}

static __device__ int g_optim_error;

__global__ void adamw_scalars_kernel(const double* __restrict__ part, int nparts,
                                     const gptb200_adamw_config cfg, int32_t* step_io,
                                     const float* loss, float* history, AdamScalars* out) {
  __shared__ double red[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += part[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x != 0) return;
  double tot = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
  // Gradients are scaled by grad_scale before the norm (1.0 for the reference step).
  const float gs = cfg.grad_scale;
  const float grad_norm = (float)sqrt(tot) * gs;
  float clip = 1.0f;
  if (cfg.grad_clip > 0.f) clip = fminf(1.0f, cfg.grad_clip / (grad_norm + 1.0e-6f));
  const int step = *step_io + 1;
  const float stepf = (float)step;
  float warm = 1.0f;
  if (cfg.warmup_steps > 0) warm = fminf(1.0f, stepf / (float)cfg.warmup_steps);
  const int span = max(1, cfg.total_steps - cfg.warmup_steps);
  float prog = (stepf - (float)cfg.warmup_steps) / (float)span;
  prog = fminf(fmaxf(prog, 0.0f), 1.0f);
  const float cosine = 0.5f * (1.0f + cosf(3.14159265358979323846f * prog));
  const float mult = cfg.min_lr_ratio + (1.0f - cfg.min_lr_ratio) * cosine;
  const float lr = (cfg.learning_rate * cfg.horizon_lr_scale) * warm * mult;
  AdamScalars a;
  a.lr = lr;
  a.bc1 = 1.0f - powf(cfg.beta1, stepf);
  a.bc2 = 1.0f - powf(cfg.beta2, stepf);
  a.gscale = gs * clip;
  a.grad_norm = grad_norm;
  a.step = step;
  *out = a;
  *step_io = step;
  // A non-finite loss or gradient norm is the reference's FloatingPointError
  // (rig/mesh.py finite_metric); record it for gptb200_device_error().
  if (!isfinite(grad_norm) || (loss && !isfinite(*loss))) g_optim_error = kErrNonFinite;
  if (history && step >= 1 && step <= cfg.total_steps) {
    float* row = history + (int64_t)(step - 1) * 3;
    row[0] = loss ? *loss : 0.f;
    row[1] = lr;
    row[2] = grad_norm;
  }
}

// Finds the tensor group holding element e (offsets increasing); -1 for the
// padding between tensors. `gi` is the caller's cached guess.
__device__ __forceinline__ int find_group(const gptb200_tensor_group* sg, int ngroups, int gi,
                                          int64_t e) {
  if (gi >= 0 && gi < ngroups && e >= sg[gi].offset && e < sg[gi].offset + sg[gi].size) return gi;
  int lo = 0, hi = ngroups - 1, f = -1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (sg[mid].offset <= e) {
      f = mid;
      lo = mid + 1;
    } else {
      hi = mid - 1;
    }
  }
  return (f < 0 || e >= sg[f].offset + sg[f].size) ? -1 : f;
}

// AdamW on the float4 at element e0 (elements [e0, min(e0 + 4, lim))) of
// tensor group G; returns the sum of squares of the (unscaled) gradients.
__device__ __forceinline__ float adamw_quad(float* __restrict__ p, float* __restrict__ m,
                                            float* __restrict__ v, const float* __restrict__ g,
                                            bf16* __restrict__ pbf, int64_t e0, int64_t lim,
                                            const gptb200_tensor_group& G,
                                            const gptb200_adamw_config& cfg,
                                            const AdamScalars& s) {
  const float b1 = cfg.beta1, b2 = cfg.beta2;
  const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
  const float lr = s.lr * G.lr_mult;
  const float eps = cfg.eps * cfg.eps_horizon_scale * G.eps_mult;
  const float wd = G.decay ? cfg.weight_decay * cfg.wd_horizon_scale * G.wd_mult : 0.f;
  const int cnt = (int)((lim - e0) < 4 ? (lim - e0) : 4);
  float sq = 0.f;
  if (cnt == 4) {
    const int64_t q = e0 >> 2;
    float4 P = reinterpret_cast<float4*>(p)[q];
    float4 M = reinterpret_cast<float4*>(m)[q];
    float4 V = reinterpret_cast<float4*>(v)[q];
    const float4 Gr = reinterpret_cast<const float4*>(g)[q];
    float* pp = &P.x;
    float* mm = &M.x;
    float* vv = &V.x;
    const float* gg = &Gr.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sq += gg[j] * gg[j];
      const float gr = gg[j] * s.gscale;
      mm[j] = b1 * mm[j] + omb1 * gr;
      vv[j] = b2 * vv[j] + omb2 * (gr * gr);
      const float adam = (mm[j] / s.bc1) / (sqrtf(vv[j] / s.bc2) + eps);
      pp[j] = pp[j] - lr * (adam + wd * pp[j]);
    }
    reinterpret_cast<float4*>(p)[q] = P;
    reinterpret_cast<float4*>(m)[q] = M;
    reinterpret_cast<float4*>(v)[q] = V;
    if (pbf) {
      uint2 o;
      o.x = pack_bf16x2(P.x, P.y);
      o.y = pack_bf16x2(P.z, P.w);
      reinterpret_cast<uint2*>(pbf)[q] = o;
    }
  } else {
    for (int j = 0; j < cnt; ++j) {
      const int64_t e = e0 + j;
      sq += g[e] * g[e];
      const float gr = g[e] * s.gscale;
      const float mj = b1 * m[e] + omb1 * gr;
      const float vj = b2 * v[e] + omb2 * (gr * gr);
      const float adam = (mj / s.bc1) / (sqrtf(vj / s.bc2) + eps);
      const float pj = p[e] - lr * (adam + wd * p[e]);
      m[e] = mj;
      v[e] = vj;
      p[e] = pj;
      if (pbf) pbf[e] = __float2bfloat16(pj);
    }
  }
  return sq;
}

__global__ void __launch_bounds__(256) adamw_update_kernel(
    float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
    const float* __restrict__ g, int64_t n, const gptb200_tensor_group* __restrict__ groups,
    int ngroups, const gptb200_adamw_config cfg, const AdamScalars* __restrict__ sc,
    bf16* __restrict__ pbf) {
  extern __shared__ gptb200_tensor_group sg[];
  for (int i = threadIdx.x; i < ngroups; i += blockDim.x) sg[i] = groups[i];
  __syncthreads();
  const AdamScalars s = *sc;
  const int64_t n4 = (n + 3) >> 2;
  int gi = 0;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
       q += (int64_t)gridDim.x * blockDim.x) {
    // Groups start on multiples of 4 elements, so a float4 never straddles two.
    const int64_t e0 = q << 2;
    gi = find_group(sg, ngroups, gi, e0);
    if (gi < 0) {
      gi = 0;
      continue;  // padding between tensors
    }
    const gptb200_tensor_group G = sg[gi];
    adamw_quad(p, m, v, g, pbf, e0, min(n, G.offset + G.size), G, cfg, s);
  }
}

// ------------------------------------------------------------------ bucketed update
// The same update split into ranges that can run as soon as their gradients
// are final (each bucket right after its all-reduce), possible when the step
// does not clip: the learning rate and bias corrections do not depend on the
// global gradient norm then. adamw_begin advances the step and computes the
// scalars; each range's update also stores, per block, the sum of squares of
// its gradients in slot `slot`; adamw_end adds every slot in order (slot,
// block: deterministic) into the logged gradient norm.
constexpr int kRangeBlocks = 1184;  // fixed grid of the ranged update (8 x 148)
constexpr int kMaxSlots = 256;

__global__ void adamw_begin_kernel(const gptb200_adamw_config cfg, int32_t* step_io,
                                   AdamScalars* out) {
  const int step = *step_io + 1;
  const float stepf = (float)step;
  float warm = 1.0f;
  if (cfg.warmup_steps > 0) warm = fminf(1.0f, stepf / (float)cfg.warmup_steps);
  const int span = max(1, cfg.total_steps - cfg.warmup_steps);
  float prog = (stepf - (float)cfg.warmup_steps) / (float)span;
  prog = fminf(fmaxf(prog, 0.0f), 1.0f);
  const float cosine = 0.5f * (1.0f + cosf(3.14159265358979323846f * prog));
  const float mult = cfg.min_lr_ratio + (1.0f - cfg.min_lr_ratio) * cosine;
  AdamScalars a;
  a.lr = (cfg.learning_rate * cfg.horizon_lr_scale) * warm * mult;
  a.bc1 = 1.0f - powf(cfg.beta1, stepf);
  a.bc2 = 1.0f - powf(cfg.beta2, stepf);
  a.gscale = cfg.grad_scale;
  a.grad_norm = 0.f;
  a.step = step;
  *out = a;
  *step_io = step;
}

__global__ void __launch_bounds__(256) adamw_range_kernel(
    float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
    const float* __restrict__ g, int64_t begin, int64_t end,
    const gptb200_tensor_group* __restrict__ groups, int ngroups, const gptb200_adamw_config cfg,
    const AdamScalars* __restrict__ sc, bf16* __restrict__ pbf, double* __restrict__ part) {
  extern __shared__ gptb200_tensor_group sg[];
  __shared__ double red[8];
  for (int i = threadIdx.x; i < ngroups; i += blockDim.x) sg[i] = groups[i];
  __syncthreads();
  const AdamScalars s = *sc;
  double acc = 0.0;
  float accf = 0.f;
  int cnt = 0, gi = 0;
  for (int64_t q = (begin >> 2) + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; (q << 2) < end;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = q << 2;
    gi = find_group(sg, ngroups, gi, e0);
    if (gi < 0) {
      gi = 0;
      continue;
    }
    const gptb200_tensor_group G = sg[gi];
    accf += adamw_quad(p, m, v, g, pbf, e0, min(end, G.offset + G.size), G, cfg, s);
    if (++cnt == 64) {
      acc += accf;
      accf = 0.f;
      cnt = 0;
    }
  }
  acc += accf;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(1024) adamw_end_kernel(const double* __restrict__ part,
                                                         int nparts, const int32_t* step_io,
                                                         const gptb200_adamw_config cfg,
                                                         const float* loss, float* history) {
  __shared__ double red[32];
  // fixed association: thread t adds parts t, t + 1024, ...; then warps, then the 32 sums
  double s = 0.0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += part[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x != 0) return;
  double tot = 0.0;
  for (int w = 0; w < 32; ++w) tot += red[w];
  const float grad_norm = (float)sqrt(tot) * cfg.grad_scale;
  const int step = *step_io;
  if (history && step >= 1 && step <= cfg.total_steps) {
    float* row = history + (int64_t)(step - 1) * 3;
    row[0] = loss ? *loss : 0.f;
    // the learning rate of this step, recomputed as adamw_begin did
    const float stepf = (float)step;
    float warm = 1.0f;
    if (cfg.warmup_steps > 0) warm = fminf(1.0f, stepf / (float)cfg.warmup_steps);
    const int span = max(1, cfg.total_steps - cfg.warmup_steps);
    float prog = (stepf - (float)cfg.warmup_steps) / (float)span;
    prog = fminf(fmaxf(prog, 0.0f), 1.0f);
    const float cosine = 0.5f * (1.0f + cosf(3.14159265358979323846f * prog));
    row[1] = (cfg.learning_rate * cfg.horizon_lr_scale) * warm *
             (cfg.min_lr_ratio + (1.0f - cfg.min_lr_ratio) * cosine);
    row[2] = grad_norm;
  }
  if (!isfinite(grad_norm) || (loss && !isfinite(*loss))) g_optim_error = kErrNonFinite;
}

}  // namespace gptb200

using namespace gptb200;

// Workspace: [kNormBlocks] doubles of the one-shot norm, the AdamScalars
// (256 bytes), then kMaxSlots x kRangeBlocks doubles of the ranged update.
constexpr size_t kScalarsOffset = kNormBlocks * sizeof(double);
constexpr size_t kSlotsOffset = kScalarsOffset + 256;

extern "C" size_t gptb200_adamw_workspace_size(int64_t n) {
  (void)n;
  return kSlotsOffset + (size_t)kMaxSlots * kRangeBlocks * sizeof(double);
}

extern "C" int gptb200_adamw_step(float* params, float* m, float* v, const float* grads, int64_t n,
                                  const gptb200_tensor_group* groups, int32_t n_groups,
                                  const gptb200_adamw_config* cfg, int32_t* step, const float* loss,
                                  float* history, void* params_bf16, void* workspace,
                                  void* stream) {
  if (!params || !m || !v || !grads || !groups || !cfg || !step || !workspace || n <= 0 ||
      n_groups <= 0)
    return GPTB200_EINVAL;
  if (n_groups > 4096) return GPTB200_EUNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(m) |
        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(grads) |
        reinterpret_cast<uintptr_t>(workspace)) & 15) ||
      (params_bf16 && (reinterpret_cast<uintptr_t>(params_bf16) & 7)))
    return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  double* part = reinterpret_cast<double*>(workspace);
  AdamScalars* sc = reinterpret_cast<AdamScalars*>(reinterpret_cast<char*>(workspace) +
                                                   kScalarsOffset);
  sqnorm_partial_kernel<<<kNormBlocks, kNormThreads, 0, st>>>(grads, n, part);
  GPTB200_CHECK_LAUNCH();
  adamw_scalars_kernel<<<1, 1024, 0, st>>>(part, kNormBlocks, *cfg, step, loss, history, sc);
  GPTB200_CHECK_LAUNCH();
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t n4 = (n + 3) / 4;
  int blocks = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)sms * 8);
  size_t smem = (size_t)n_groups * sizeof(gptb200_tensor_group);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(adamw_update_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return -static_cast<int>(e);
  }
  adamw_update_kernel<<<blocks, 256, smem, st>>>(params, m, v, grads, n, groups, n_groups, *cfg, sc,
                                                 reinterpret_cast<bf16*>(params_bf16));
  GPTB200_CHECK_LAUNCH();
  return 0;
}

namespace gptb200 {
int optim_read_error(int clear) {
  int h = 0;
  cudaMemcpyFromSymbol(&h, g_optim_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_optim_error, &z, sizeof(int));
  }
  return h;
}
}  // namespace gptb200

extern "C" int gptb200_adamw_begin(const gptb200_adamw_config* cfg, int32_t* step, void* workspace,
                                   void* stream) {
  if (!cfg || !step || !workspace) return GPTB200_EINVAL;
  if (cfg->grad_clip > 0.f) return GPTB200_EUNSUPPORTED;  // clipping needs the norm first
  auto sc = reinterpret_cast<AdamScalars*>(reinterpret_cast<char*>(workspace) + kScalarsOffset);
  adamw_begin_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*cfg, step, sc);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" int gptb200_adamw_update_range(float* params, float* m, float* v, const float* grads,
                                          int64_t begin, int64_t end,
                                          const gptb200_tensor_group* groups, int32_t n_groups,
                                          const gptb200_adamw_config* cfg, int32_t slot,
                                          void* params_bf16, void* workspace, void* stream) {
  if (!params || !m || !v || !grads || !groups || !cfg || !workspace || n_groups <= 0)
    return GPTB200_EINVAL;
  if (begin < 0 || end <= begin || (begin & 3) || slot < 0 || slot >= kMaxSlots)
    return GPTB200_EINVAL;
  if (n_groups > 4096 || cfg->grad_clip > 0.f) return GPTB200_EUNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(m) |
        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(grads) |
        reinterpret_cast<uintptr_t>(workspace)) & 15) ||
      (params_bf16 && (reinterpret_cast<uintptr_t>(params_bf16) & 7)))
    return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(workspace);
  auto sc = reinterpret_cast<const AdamScalars*>(ws + kScalarsOffset);
  auto part = reinterpret_cast<double*>(ws + kSlotsOffset) + (int64_t)slot * kRangeBlocks;
  size_t smem = (size_t)n_groups * sizeof(gptb200_tensor_group);
  if (smem > 40 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(adamw_range_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return -static_cast<int>(e);
  }
  adamw_range_kernel<<<kRangeBlocks, 256, smem, st>>>(params, m, v, grads, begin, end, groups,
                                                      n_groups, *cfg, sc,
                                                      reinterpret_cast<bf16*>(params_bf16), part);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" int gptb200_adamw_end(int32_t n_slots, const gptb200_adamw_config* cfg,
                                 const int32_t* step, const float* loss, float* history,
                                 void* workspace, void* stream) {
  if (!cfg || !step || !workspace || n_slots <= 0 || n_slots > kMaxSlots) return GPTB200_EINVAL;
  auto part = reinterpret_cast<const double*>(reinterpret_cast<char*>(workspace) + kSlotsOffset);
  adamw_end_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      part, n_slots * kRangeBlocks, step, *cfg, loss, history);
  GPTB200_CHECK_LAUNCH();
  return 0;
}
