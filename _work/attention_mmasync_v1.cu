// Causal flash attention (head_dim 64) with RoPE applied on the Q/K loads.
//
// Forward: one CTA per (128-query block, batch*head); 8 warps x 16 query rows.
// K/V tiles of 64 keys stream through double-buffered, XOR-swizzled shared
// memory with cp.async; RoPE rotates the Q tile and every K tile in shared
// memory right after arrival (interleaved pairs, bf16 cos/sin tables). Scores,
// online softmax (fp32, base-2 exponent) and P·V (bf16 P) stay in registers.
// Output O and the natural-log LSE per row are written for the backward.
//
// Backward: delta = rowsum(dO ∘ O); a dK/dV kernel (one CTA per 64-key block,
// looping over the query blocks at or below the diagonal) and a dQ kernel (one
// CTA per 64-query block, looping over key blocks up to the diagonal) recompute
// P from the LSE, so no atomics are needed. Gradients of rotated q/k are
// rotated back (transpose of the RoPE rotation) before the bf16 store.
//
// The tensor-core instructions are warp-level mma.sync m16n8k16 (bf16 in,
// fp32 accumulate). Semantics: rig/kernels/tpu_flash_attention.py:171-207
// (reference_causal_attention) and rig/nn.py:36-52 (apply_rotary).
#include <algorithm>

#include "common.cuh"

namespace gptb200 {

static __device__ int g_attn_error;

constexpr int HD = 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnArgs {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  int64_t sb, sh, st;
  const bf16* o;
  bf16* o_out;
  const bf16* dout;
  int64_t osb, osh, ost;
  float* lse_out;
  const float* lse;
  const float* delta;
  bf16* dq;
  bf16* dk;
  bf16* dv;
  int B, H, T;
  float scale;
  const bf16* rcos;
  const bf16* rsin;
};

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 128 + (((chunk ^ (row & 7)) & 7) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Asynchronously copies `rows` x 64 bf16 rows (row r at base + (r0+r)*stride)
// into a swizzled tile; rows at or beyond T are zero-filled.
__device__ __forceinline__ void load_tile_async(uint8_t* s, const bf16* base, int64_t stride, int r0,
                                                int rows, int T, int tid, int nthreads) {
  const uint32_t sa = smem_u32(s);
  for (int i = tid; i < rows * 8; i += nthreads) {
    int r = i >> 3, c = i & 7;
    if (r0 + r < T) {
      cp_async16(sa + swz(r, c), base + (int64_t)(r0 + r) * stride + c * 8);
    } else {
      *reinterpret_cast<uint4*>(s + swz(r, c)) = make_uint4(0, 0, 0, 0);
    }
  }
}

// Rotates a swizzled tile in place: pair i of row r at position r0+r.
__device__ __forceinline__ void rope_tile(uint8_t* s, const bf16* rcos, const bf16* rsin, int r0,
                                          int rows, int T, int tid, int nthreads) {
  for (int i = tid; i < rows * 8; i += nthreads) {
    int r = i >> 3, c = i & 7;
    int t = r0 + r;
    if (t >= T) continue;
    uint4* p = reinterpret_cast<uint4*>(s + swz(r, c));
    uint4 q = *p;
    uint32_t* w = &q.x;
    const bf16* cs = rcos + (int64_t)t * (HD / 2) + c * 4;
    const bf16* sn = rsin + (int64_t)t * (HD / 2) + c * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float e, o;
      unpack_bf16x2(w[j], e, o);
      float cv = __bfloat162float(cs[j]), sv = __bfloat162float(sn[j]);
      w[j] = pack_bf16x2(e * cv - o * sv, e * sv + o * cv);
    }
    *p = q;
  }
}

// Loads the A fragments (16 rows x 64 dims, 4 k-steps) of rows [row0, row0+16)
// of a swizzled 64-wide tile.
__device__ __forceinline__ void load_a_frags(const uint8_t* s, int row0, int lane, uint32_t (*a)[4]) {
  const uint32_t sa = smem_u32(s);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    int r = row0 + (lane & 7) + 8 * ((lane >> 3) & 1);
    int c = kk * 2 + (lane >> 4);
    ldsm_x4(sa + swz(r, c), a[kk][0], a[kk][1], a[kk][2], a[kk][3]);
  }
}

// acc[16 x 64] (8 n-tiles) += A[16 x 64] · Tile^T, where Tile is 64 rows
// (the n dimension) x 64 dims (the k dimension), non-transposed ldmatrix.
__device__ __forceinline__ void mma_a_tileT(float (*acc)[4], const uint32_t (*a)[4], const uint8_t* s,
                                            int lane) {
  const uint32_t sa = smem_u32(s);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b0, b1, b2, b3;
      int r = np * 16 + (lane & 7) + 8 * (lane >> 4);
      int c = kk * 2 + ((lane >> 3) & 1);
      ldsm_x4(sa + swz(r, c), b0, b1, b2, b3);
      mma16816(acc[2 * np], a[kk], b0, b1);
      mma16816(acc[2 * np + 1], a[kk], b2, b3);
    }
  }
}

// acc[16 x 64 dims] += P[16 x 64 rows-of-tile] · Tile, where Tile is 64 rows
// (the k dimension) x 64 dims (the n dimension), transposed ldmatrix. P is
// given as fp32 accumulator fragments (8 n-tiles) and rounded to bf16 here.
__device__ __forceinline__ void mma_p_tile(float (*acc)[4], const float (*p)[4], const uint8_t* s,
                                           int lane) {
  const uint32_t sa = smem_u32(s);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4];
    a[0] = pack_bf16x2(p[2 * kk][0], p[2 * kk][1]);
    a[1] = pack_bf16x2(p[2 * kk][2], p[2 * kk][3]);
    a[2] = pack_bf16x2(p[2 * kk + 1][0], p[2 * kk + 1][1]);
    a[3] = pack_bf16x2(p[2 * kk + 1][2], p[2 * kk + 1][3]);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b0, b1, b2, b3;
      int r = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
      int c = np * 2 + (lane >> 4);
      ldsm_x4_t(sa + swz(r, c), b0, b1, b2, b3);
      mma16816(acc[2 * np], a, b0, b1);
      mma16816(acc[2 * np + 1], a, b2, b3);
    }
  }
}

// Writes a warp's 16 x 64 fp32 accumulator (scaled) as bf16 rows into a
// swizzled smem tile, optionally rotating pairs back (inverse RoPE) for
// positions pos0 + row.
__device__ __forceinline__ void stage_rows(uint8_t* s, int row0, const float (*acc)[4], float mul,
                                           int lane) {
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    int col = nt * 8 + (lane & 3) * 2;
    int r = row0 + (lane >> 2);
    uint32_t off0 = swz(r, col >> 3) + (col & 7) * 2;
    uint32_t off1 = swz(r + 8, col >> 3) + (col & 7) * 2;
    *reinterpret_cast<uint32_t*>(s + off0) = pack_bf16x2(acc[nt][0] * mul, acc[nt][1] * mul);
    *reinterpret_cast<uint32_t*>(s + off1) = pack_bf16x2(acc[nt][2] * mul, acc[nt][3] * mul);
  }
}

// Copies `rows` swizzled smem rows to global (row r -> base + (r0+r)*stride),
// skipping rows >= T; with rcos != NULL applies the transpose RoPE rotation
// (d_even = g_e*c + g_o*s, d_odd = -g_e*s + g_o*c) on the way out.
__device__ __forceinline__ void store_tile(const uint8_t* s, bf16* base, int64_t stride, int r0,
                                           int rows, int T, const bf16* rcos, const bf16* rsin,
                                           int tid, int nthreads) {
  for (int i = tid; i < rows * 8; i += nthreads) {
    int r = i >> 3, c = i & 7;
    int t = r0 + r;
    if (t >= T) continue;
    uint4 q = *reinterpret_cast<const uint4*>(s + swz(r, c));
    if (rcos) {
      uint32_t* w = &q.x;
      const bf16* cs = rcos + (int64_t)t * (HD / 2) + c * 4;
      const bf16* sn = rsin + (int64_t)t * (HD / 2) + c * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float ge, go;
        unpack_bf16x2(w[j], ge, go);
        float cv = __bfloat162float(cs[j]), sv = __bfloat162float(sn[j]);
        w[j] = pack_bf16x2(ge * cv + go * sv, -ge * sv + go * cv);
      }
    }
    *reinterpret_cast<uint4*>(base + (int64_t)t * stride + c * 8) = q;
  }
}

// ------------------------------------------------------------------ forward
constexpr int FWD_BR = 128, FWD_BC = 64, FWD_THREADS = 256;
constexpr int TILE_BYTES = 64 * 128;  // 64 rows x 64 bf16

__global__ void __launch_bounds__(FWD_THREADS, 2) attn_fwd_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;                        // 128 rows
  uint8_t* sK = sm + 2 * TILE_BYTES;       // 2 buffers
  uint8_t* sV = sK + 2 * TILE_BYTES;       // 2 buffers
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nqb = (a.T + FWD_BR - 1) / FWD_BR;
  const int qb = nqb - 1 - blockIdx.x;  // heaviest blocks first
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh - b * a.H;
  const int q0 = qb * FWD_BR;
  const bf16* Q = a.q + b * a.sb + h * a.sh;
  const bf16* K = a.k + b * a.sb + h * a.sh;
  const bf16* V = a.v + b * a.sb + h * a.sh;

  load_tile_async(sQ, Q, a.st, q0, FWD_BR, a.T, tid, FWD_THREADS);
  cp_commit();
  const int kv_end = min(a.T, q0 + FWD_BR);
  const int ntiles = (kv_end + FWD_BC - 1) / FWD_BC;
  load_tile_async(sK, K, a.st, 0, FWD_BC, a.T, tid, FWD_THREADS);
  load_tile_async(sV, V, a.st, 0, FWD_BC, a.T, tid, FWD_THREADS);
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  if (a.rcos) {
    rope_tile(sQ, a.rcos, a.rsin, q0, FWD_BR, a.T, tid, FWD_THREADS);
    __syncthreads();
  }
  uint32_t qf[4][4];
  load_a_frags(sQ, warp * 16, lane, qf);

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = a.scale * kLog2e;
  const int row_a = q0 + warp * 16 + (lane >> 2);
  const int row_b = row_a + 8;

  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < ntiles) {
      load_tile_async(sK + (buf ^ 1) * TILE_BYTES, K, a.st, (j + 1) * FWD_BC, FWD_BC, a.T, tid,
                      FWD_THREADS);
      load_tile_async(sV + (buf ^ 1) * TILE_BYTES, V, a.st, (j + 1) * FWD_BC, FWD_BC, a.T, tid,
                      FWD_THREADS);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    uint8_t* kt = sK + buf * TILE_BYTES;
    uint8_t* vt = sV + buf * TILE_BYTES;
    if (a.rcos) {
      rope_tile(kt, a.rcos, a.rsin, j * FWD_BC, FWD_BC, a.T, tid, FWD_THREADS);
      __syncthreads();
    }
    const int k0 = j * FWD_BC;
    if (k0 <= q0 + warp * 16 + 15) {  // the warp sees at least one key of this tile
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      mma_a_tileT(s, qf, kt, lane);
      const bool diag = k0 + FWD_BC - 1 > q0 + warp * 16;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          int key = k0 + nt * 8 + (lane & 3) * 2 + e;
          float va = s[nt][e] * sl2, vb = s[nt][2 + e] * sl2;
          if (diag) {
            if (key > row_a) va = -INFINITY;
            if (key > row_b) vb = -INFINITY;
          }
          s[nt][e] = va;
          s[nt][2 + e] = vb;
          mx0 = fmaxf(mx0, va);
          mx1 = fmaxf(mx1, vb);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
      const float c0 = (nm0 == -INFINITY) ? 0.f : nm0;
      const float c1 = (nm1 == -INFINITY) ? 0.f : nm1;
      const float al0 = exp2f(m0 - c0), al1 = exp2f(m1 - c1);
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][0] = exp2f(s[nt][0] - c0);
        s[nt][1] = exp2f(s[nt][1] - c0);
        s[nt][2] = exp2f(s[nt][2] - c1);
        s[nt][3] = exp2f(s[nt][3] - c1);
        rs0 += s[nt][0] + s[nt][1];
        rs1 += s[nt][2] + s[nt][3];
      }
      l0 = l0 * al0 + rs0;
      l1 = l1 * al1 + rs1;
      m0 = nm0;
      m1 = nm1;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        o[nt][0] *= al0;
        o[nt][1] *= al0;
        o[nt][2] *= al1;
        o[nt][3] *= al1;
      }
      mma_p_tile(o, s, vt, lane);
    }
    __syncthreads();
  }
  // Finish: row sums across the quad, normalize, LSE.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    o[nt][0] *= inv0;
    o[nt][1] *= inv0;
    o[nt][2] *= inv1;
    o[nt][3] *= inv1;
  }
  if ((lane & 3) == 0) {
    float* L = a.lse_out + (int64_t)bh * a.T;
    if (row_a < a.T) L[row_a] = (m0 + log2f(l0)) * kLn2;
    if (row_b < a.T) L[row_b] = (m1 + log2f(l1)) * kLn2;
  }
  // Stage O through shared memory (the Q tile is no longer needed).
  stage_rows(sQ, warp * 16, o, 1.f, lane);
  __syncthreads();
  store_tile(sQ, a.o_out + b * a.osb + h * a.osh, a.ost, q0, FWD_BR, a.T, nullptr, nullptr, tid,
             FWD_THREADS);
}

// ------------------------------------------------------------------ backward
__global__ void attn_delta_kernel(const AttnArgs a) {
  // One warp per row: delta = sum_e dO * O (fp32).
  const int64_t rows = (int64_t)a.B * a.H * a.T;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int64_t bh = r / a.T;
  const int t = (int)(r - bh * a.T);
  const int b = (int)(bh / a.H), h = (int)(bh - (int64_t)b * a.H);
  const int64_t off = b * a.osb + h * a.osh + (int64_t)t * a.ost + lane * 2;
  float o0, o1, g0, g1;
  unpack_bf16x2(*reinterpret_cast<const uint32_t*>(a.o + off), o0, o1);
  unpack_bf16x2(*reinterpret_cast<const uint32_t*>(a.dout + off), g0, g1);
  float s = warp_sum(o0 * g0 + o1 * g1);
  if (lane == 0) const_cast<float*>(a.delta)[r] = s;
}

constexpr int BWD_B = 64, BWD_THREADS = 128;

// dK, dV for one 64-key block. Warp w owns keys [k0 + 16w, k0 + 16w + 16).
__global__ void __launch_bounds__(BWD_THREADS) attn_bwd_dkdv_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sK = sm;                    // K block (rotated), later dK staging
  uint8_t* sV = sK + TILE_BYTES;       // V block, later dV staging
  uint8_t* sQ = sV + TILE_BYTES;       // 2 buffers
  uint8_t* sD = sQ + 2 * TILE_BYTES;   // dO, 2 buffers
  float* sL = reinterpret_cast<float*>(sD + 2 * TILE_BYTES);  // lse (log2 units), 2 x 64
  float* sDl = sL + 2 * BWD_B;                                  // delta, 2 x 64
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nkb = (a.T + BWD_B - 1) / BWD_B;
  const int kb = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh - b * a.H;
  const int k0 = kb * BWD_B;
  const bf16* Q = a.q + b * a.sb + h * a.sh;
  const bf16* K = a.k + b * a.sb + h * a.sh;
  const bf16* V = a.v + b * a.sb + h * a.sh;
  const bf16* dO = a.dout + b * a.osb + h * a.osh;
  const float* L = a.lse + (int64_t)bh * a.T;
  const float* Dl = a.delta + (int64_t)bh * a.T;

  load_tile_async(sK, K, a.st, k0, BWD_B, a.T, tid, BWD_THREADS);
  load_tile_async(sV, V, a.st, k0, BWD_B, a.T, tid, BWD_THREADS);
  cp_commit();
  auto load_q = [&](int qi, int buf) {
    const int q0 = qi * BWD_B;
    load_tile_async(sQ + buf * TILE_BYTES, Q, a.st, q0, BWD_B, a.T, tid, BWD_THREADS);
    load_tile_async(sD + buf * TILE_BYTES, dO, a.ost, q0, BWD_B, a.T, tid, BWD_THREADS);
    for (int i = tid; i < BWD_B; i += BWD_THREADS) {
      int t = q0 + i;
      sL[buf * BWD_B + i] = (t < a.T) ? L[t] * kLog2e : 0.f;
      sDl[buf * BWD_B + i] = (t < a.T) ? Dl[t] : 0.f;
    }
  };
  load_q(kb, 0);
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  if (a.rcos) {
    rope_tile(sK, a.rcos, a.rsin, k0, BWD_B, a.T, tid, BWD_THREADS);
    __syncthreads();
  }
  uint32_t kf[4][4], vf[4][4];
  load_a_frags(sK, warp * 16, lane, kf);
  load_a_frags(sV, warp * 16, lane, vf);

  float dk[8][4], dv[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;
  const float sl2 = a.scale * kLog2e;
  const int key_a = k0 + warp * 16 + (lane >> 2);
  const int key_b = key_a + 8;

  for (int qi = kb; qi < nkb; ++qi) {
    const int buf = (qi - kb) & 1;
    if (qi + 1 < nkb) {
      load_q(qi + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    uint8_t* qt = sQ + buf * TILE_BYTES;
    uint8_t* dt = sD + buf * TILE_BYTES;
    const int q0 = qi * BWD_B;
    if (a.rcos) {
      rope_tile(qt, a.rcos, a.rsin, q0, BWD_B, a.T, tid, BWD_THREADS);
      __syncthreads();
    }
    const float* lq = sL + buf * BWD_B;
    const float* dq = sDl + buf * BWD_B;
    // S^T = K_w Q^T  (rows = keys, cols = queries)
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
    mma_a_tileT(s, kf, qt, lane);
    mma_a_tileT(dp, vf, dt, lane);
    const bool diag = (qi == kb);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int qc = nt * 8 + (lane & 3) * 2 + e;
        const int query = q0 + qc;
        const float lv = lq[qc], dl = dq[qc];
        float pa = exp2f(s[nt][e] * sl2 - lv);
        float pb = exp2f(s[nt][2 + e] * sl2 - lv);
        if ((diag && key_a > query) || query >= a.T) pa = 0.f;
        if ((diag && key_b > query) || query >= a.T) pb = 0.f;
        s[nt][e] = pa;
        s[nt][2 + e] = pb;
        dp[nt][e] = pa * (dp[nt][e] - dl);
        dp[nt][2 + e] = pb * (dp[nt][2 + e] - dl);
      }
    }
    mma_p_tile(dv, s, dt, lane);   // dV += P^T dO
    mma_p_tile(dk, dp, qt, lane);  // dK += dS^T Q
    __syncthreads();
  }
  // Stage and store: dK (scaled, inverse RoPE), dV.
  stage_rows(sK, warp * 16, dk, a.scale, lane);
  stage_rows(sV, warp * 16, dv, 1.f, lane);
  __syncthreads();
  store_tile(sK, a.dk + b * a.sb + h * a.sh, a.st, k0, BWD_B, a.T, a.rcos, a.rsin, tid, BWD_THREADS);
  store_tile(sV, a.dv + b * a.sb + h * a.sh, a.st, k0, BWD_B, a.T, nullptr, nullptr, tid,
             BWD_THREADS);
}

// dQ for one 64-query block. Warp w owns queries [q0 + 16w, q0 + 16w + 16).
__global__ void __launch_bounds__(BWD_THREADS) attn_bwd_dq_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;                   // Q block (rotated), later dQ staging
  uint8_t* sD = sQ + TILE_BYTES;      // dO block
  uint8_t* sK = sD + TILE_BYTES;      // 2 buffers
  uint8_t* sV = sK + 2 * TILE_BYTES;  // 2 buffers
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nqb = (a.T + BWD_B - 1) / BWD_B;
  const int qb = nqb - 1 - blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh - b * a.H;
  const int q0 = qb * BWD_B;
  const bf16* Q = a.q + b * a.sb + h * a.sh;
  const bf16* K = a.k + b * a.sb + h * a.sh;
  const bf16* V = a.v + b * a.sb + h * a.sh;
  const bf16* dO = a.dout + b * a.osb + h * a.osh;

  load_tile_async(sQ, Q, a.st, q0, BWD_B, a.T, tid, BWD_THREADS);
  load_tile_async(sD, dO, a.ost, q0, BWD_B, a.T, tid, BWD_THREADS);
  cp_commit();
  load_tile_async(sK, K, a.st, 0, BWD_B, a.T, tid, BWD_THREADS);
  load_tile_async(sV, V, a.st, 0, BWD_B, a.T, tid, BWD_THREADS);
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  if (a.rcos) {
    rope_tile(sQ, a.rcos, a.rsin, q0, BWD_B, a.T, tid, BWD_THREADS);
    __syncthreads();
  }
  uint32_t qf[4][4], df[4][4];
  load_a_frags(sQ, warp * 16, lane, qf);
  load_a_frags(sD, warp * 16, lane, df);
  const int row_a = q0 + warp * 16 + (lane >> 2);
  const int row_b = row_a + 8;
  const float* L = a.lse + (int64_t)bh * a.T;
  const float* Dl = a.delta + (int64_t)bh * a.T;
  const float la = (row_a < a.T) ? L[row_a] * kLog2e : 0.f;
  const float lb = (row_b < a.T) ? L[row_b] * kLog2e : 0.f;
  const float da = (row_a < a.T) ? Dl[row_a] : 0.f;
  const float db = (row_b < a.T) ? Dl[row_b] : 0.f;
  const float sl2 = a.scale * kLog2e;

  float dq[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  for (int j = 0; j <= qb; ++j) {
    const int buf = j & 1;
    if (j + 1 <= qb) {
      load_tile_async(sK + (buf ^ 1) * TILE_BYTES, K, a.st, (j + 1) * BWD_B, BWD_B, a.T, tid,
                      BWD_THREADS);
      load_tile_async(sV + (buf ^ 1) * TILE_BYTES, V, a.st, (j + 1) * BWD_B, BWD_B, a.T, tid,
                      BWD_THREADS);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    uint8_t* kt = sK + buf * TILE_BYTES;
    uint8_t* vt = sV + buf * TILE_BYTES;
    const int k0 = j * BWD_B;
    if (a.rcos) {
      rope_tile(kt, a.rcos, a.rsin, k0, BWD_B, a.T, tid, BWD_THREADS);
      __syncthreads();
    }
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
    mma_a_tileT(s, qf, kt, lane);
    mma_a_tileT(dp, df, vt, lane);
    const bool diag = (j == qb);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = k0 + nt * 8 + (lane & 3) * 2 + e;
        float pa = exp2f(s[nt][e] * sl2 - la);
        float pb = exp2f(s[nt][2 + e] * sl2 - lb);
        if (diag && key > row_a) pa = 0.f;
        if (diag && key > row_b) pb = 0.f;
        s[nt][e] = pa * (dp[nt][e] - da);
        s[nt][2 + e] = pb * (dp[nt][2 + e] - db);
      }
    }
    mma_p_tile(dq, s, kt, lane);  // dQ += dS K
    __syncthreads();
  }
  stage_rows(sQ, warp * 16, dq, a.scale, lane);
  __syncthreads();
  store_tile(sQ, a.dq + b * a.sb + h * a.sh, a.st, q0, BWD_B, a.T, a.rcos, a.rsin, tid,
             BWD_THREADS);
}

int attention_read_error(int clear) {
  int h = 0;
  cudaMemcpyFromSymbol(&h, g_attn_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_attn_error, &z, sizeof(int));
  }
  return h;
}

}  // namespace gptb200

using namespace gptb200;

static int check_attn(const void* q, const void* k, const void* v, int64_t sb, int64_t sh,
                      int64_t st, int64_t osb, int64_t osh, int64_t ost, int64_t batch,
                      int64_t heads, int64_t seq, int64_t hd) {
  if (!q || !k || !v) return GPTB200_EINVAL;
  if (batch <= 0 || heads <= 0 || seq <= 0) return GPTB200_EINVAL;
  if (hd != HD) return GPTB200_EUNSUPPORTED;
  if (batch * heads > 65535 * 1024LL || seq > (1 << 24)) return GPTB200_ESHAPE;
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
                                     int64_t head_dim, float softmax_scale, const void* rope_cos,
                                     const void* rope_sin, void* stream) {
  int s = check_attn(q, k, v, stride_b, stride_h, stride_t, o_stride_b, o_stride_h, o_stride_t,
                     batch, heads, seq, head_dim);
  if (s) return s;
  if (!o || !lse || !(softmax_scale > 0.f)) return GPTB200_EINVAL;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return GPTB200_EINVAL;
  AttnArgs a = {};
  a.q = reinterpret_cast<const bf16*>(q);
  a.k = reinterpret_cast<const bf16*>(k);
  a.v = reinterpret_cast<const bf16*>(v);
  a.sb = stride_b;
  a.sh = stride_h;
  a.st = stride_t;
  a.o_out = reinterpret_cast<bf16*>(o);
  a.osb = o_stride_b;
  a.osh = o_stride_h;
  a.ost = o_stride_t;
  a.lse_out = lse;
  a.B = (int)batch;
  a.H = (int)heads;
  a.T = (int)seq;
  a.scale = softmax_scale;
  a.rcos = reinterpret_cast<const bf16*>(rope_cos);
  a.rsin = reinterpret_cast<const bf16*>(rope_sin);
  const int smem = 6 * TILE_BYTES;
  static bool cfg = false;
  if (!cfg) {
    cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cfg = true;
  }
  dim3 grid((unsigned)((seq + FWD_BR - 1) / FWD_BR), (unsigned)(batch * heads));
  attn_fwd_kernel<<<grid, FWD_THREADS, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  GPTB200_CHECK_LAUNCH();
  return 0;
}

extern "C" size_t gptb200_attention_bwd_workspace_size(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  return (size_t)((batch * heads * seq * 4 + 255) / 256 * 256);
}

extern "C" int gptb200_attention_bwd(const void* q, const void* k, const void* v, int64_t stride_b,
                                     int64_t stride_h, int64_t stride_t, const void* o,
                                     const void* dout, int64_t o_stride_b, int64_t o_stride_h,
                                     int64_t o_stride_t, const float* lse, void* dq, void* dk,
                                     void* dv, int64_t batch, int64_t heads, int64_t seq,
                                     int64_t head_dim, float softmax_scale, const void* rope_cos,
                                     const void* rope_sin, void* workspace, void* stream) {
  int s = check_attn(q, k, v, stride_b, stride_h, stride_t, o_stride_b, o_stride_h, o_stride_t,
                     batch, heads, seq, head_dim);
  if (s) return s;
  if (!o || !dout || !lse || !dq || !dk || !dv || !workspace || !(softmax_scale > 0.f))
    return GPTB200_EINVAL;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return GPTB200_EINVAL;
  if ((reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(dq) |
       reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15)
    return GPTB200_ESHAPE;
  auto st = reinterpret_cast<cudaStream_t>(stream);
  AttnArgs a = {};
  a.q = reinterpret_cast<const bf16*>(q);
  a.k = reinterpret_cast<const bf16*>(k);
  a.v = reinterpret_cast<const bf16*>(v);
  a.sb = stride_b;
  a.sh = stride_h;
  a.st = stride_t;
  a.o = reinterpret_cast<const bf16*>(o);
  a.dout = reinterpret_cast<const bf16*>(dout);
  a.osb = o_stride_b;
  a.osh = o_stride_h;
  a.ost = o_stride_t;
  a.lse = lse;
  a.delta = reinterpret_cast<float*>(workspace);
  a.dq = reinterpret_cast<bf16*>(dq);
  a.dk = reinterpret_cast<bf16*>(dk);
  a.dv = reinterpret_cast<bf16*>(dv);
  a.B = (int)batch;
  a.H = (int)heads;
  a.T = (int)seq;
  a.scale = softmax_scale;
  a.rcos = reinterpret_cast<const bf16*>(rope_cos);
  a.rsin = reinterpret_cast<const bf16*>(rope_sin);
  const int64_t rows = batch * heads * seq;
  attn_delta_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(a);
  GPTB200_CHECK_LAUNCH();
  const int smem_kv = 6 * TILE_BYTES + 4 * BWD_B * (int)sizeof(float);
  const int smem_q = 6 * TILE_BYTES;
  static bool cfg = false;
  if (!cfg) {
    cudaFuncSetAttribute(attn_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_kv);
    cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_q);
    cfg = true;
  }
  dim3 grid((unsigned)((seq + BWD_B - 1) / BWD_B), (unsigned)(batch * heads));
  attn_bwd_dkdv_kernel<<<grid, BWD_THREADS, smem_kv, st>>>(a);
  GPTB200_CHECK_LAUNCH();
  attn_bwd_dq_kernel<<<grid, BWD_THREADS, smem_q, st>>>(a);
  GPTB200_CHECK_LAUNCH();
  return 0;
}
