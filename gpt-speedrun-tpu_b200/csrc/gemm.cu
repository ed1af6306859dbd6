// Persistent, warp-specialized tcgen05 GEMM for sm_100a.
//
//   C[M,N] = epilogue( sum_k A[m,k] B[n,k] )   bf16 operands, fp32 accumulation in TMEM
//
// One CTA per SM loops over output tiles (128 x BN) and, for weight gradients,
// over K splits. Roles inside the CTA (576 threads):
//   warp 0  lane 0 : TMA producer. Each pipeline stage holds a 128x64 A tile and
//                    a BNx64 B tile in 128-byte-swizzled shared memory. K-major
//                    operands are one box; MN-major operands are 64-wide boxes.
//   warp 1  lane 0 : MMA issuer. 4 tcgen05.mma (K=16 each) per stage into one of
//                    two TMEM accumulators (2 x BN fp32 columns), so the
//                    epilogue of tile i overlaps the main loop of tile i+1.
//   warps 2-17     : epilogue. Each warp owns the 32 TMEM lanes (= tile rows) of
//                    its quadrant (warp % 4) and a quarter of the tile's columns,
//                    pulls them out of TMEM with tcgen05.ld (releasing the
//                    accumulator right away) and applies the fused epilogue
//                    (bias, branch multiplier, residual, RoPE, GELU, dGELU, fp32
//                    store or atomic add, and the two cross-entropy epilogues
//                    used by lce.cu).
// Every wait is bounded (common.cuh); a wait that runs out raises the CTA's
// abort flag so all roles leave their loops, TMEM is freed and the error is
// visible through gptb200_device_error().
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace gptb200 {

static __device__ int g_gemm_error;

constexpr int BM = 128;
constexpr int BK = 64;
// Epilogue warps: 16 (four per TMEM lane quadrant, a quarter of the tile's
// columns each) or 8 (two per quadrant, half the columns each, in two passes);
// a kernel has 64 + 32 x that many threads (TMA warp + MMA warp + epilogue).

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // Per epilogue warp a 2 KB staging tile (32 rows x 32 bf16, 64-byte swizzle)
  // for the TMA stores of bf16 outputs; the LCE forward reuses it for its
  // 4 x 128 float2 row partials.
  static constexpr int STAGE_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int STAGE_TILE = 2048;
  static constexpr int RED_OFFSET = STAGE_OFFSET;
  static constexpr int BAR_OFFSET = STAGE_OFFSET + 16 * STAGE_TILE;
  static constexpr int TOTAL = BAR_OFFSET + 256 + 1023;  // + alignment slack
};

// Tensor maps of the bf16 outputs (C and the GELU pre-activation), box 32 x 32.
struct EpiMaps {
  CUtensorMap c;
  CUtensorMap aux;
};

struct TileCoord {
  int tm, tn, ks;
};

// Work unit u -> (M tile, N tile, K split). Within a split the tiles are
// rastered in groups of group_m M tiles: consecutive units walk down the
// group's M tiles, then to the next N tile. The CTAs in flight at any moment
// then share a few A stripes and a few B panels, which stay in L2, instead of
// all sweeping the full width of B (re-fetched from DRAM for every M tile).
__device__ __forceinline__ TileCoord decode_unit(const GemmParams& p, int u) {
  TileCoord c;
  const int per_split = p.tiles_m * p.tiles_n;
  c.ks = u / per_split;
  const int r = u - c.ks * per_split;
  const int per_group = p.group_m * p.tiles_n;
  const int g = r / per_group;
  const int first_m = g * p.group_m;
  const int gm = min(p.group_m, p.tiles_m - first_m);
  const int w = r - g * per_group;
  c.tm = first_m + w % gm;
  c.tn = w / gm;
  return c;
}

// ------------------------------------------------------------------ epilogues
template <int EPI>
struct EpilogueRowState {
  float run_max = -INFINITY;
  float run_sum = 0.f;
};

// Writes 8 consecutive bf16 values (one 16-byte store).
__device__ __forceinline__ void store_bf16x8(bf16* dst, const float* v) {
  uint4 q;
  q.x = pack_bf16x2(v[0], v[1]);
  q.y = pack_bf16x2(v[2], v[3]);
  q.z = pack_bf16x2(v[4], v[5]);
  q.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(dst) = q;
}

__device__ __forceinline__ void load_bf16x8(const bf16* src, float* v) {
  uint4 q = *reinterpret_cast<const uint4*>(src);
  unpack_bf16x2(q.x, v[0], v[1]);
  unpack_bf16x2(q.y, v[2], v[3]);
  unpack_bf16x2(q.z, v[4], v[5]);
  unpack_bf16x2(q.w, v[6], v[7]);
}

template <int EPI>
constexpr bool kStagedEpi = EPI == EPI_BF16_ || EPI == EPI_BIAS_ROPE_ || EPI == EPI_BIAS_GELU_ ||
                            EPI == EPI_DGELU_ || EPI == EPI_LCE_BWD_;

// Global operands of the bf16-output epilogues for 8 columns [c0, c0+8) of
// one row: bias, the residual / saved GELU derivative row, RoPE tables.
// Addresses are clamped into the matrix (N is a multiple of 8 whenever these
// are read), so a chunk's loads can all be issued before any of its math.
struct EpiOperands {
  uint4 b, x;
  uint2 cs, sn;
};

template <int EPI>
__device__ __forceinline__ EpiOperands epi_load8(const GemmParams& p, int row, int c0) {
  EpiOperands o;
  o.b = o.x = make_uint4(0u, 0u, 0u, 0u);
  o.cs = o.sn = make_uint2(0u, 0u);
  const int cc = min(c0, p.N - 8);
  const int64_t rr = min(row, p.M - 1);
  if constexpr (EPI == EPI_BF16_) {
    if (p.bias) o.b = *reinterpret_cast<const uint4*>(p.bias + cc);
    if (p.resid) o.x = *reinterpret_cast<const uint4*>(p.resid + rr * p.ld_resid + cc);
  } else if constexpr (EPI == EPI_BIAS_ROPE_) {
    o.b = *reinterpret_cast<const uint4*>(p.bias + cc);
    if (cc < p.rope_cols) {
      const int64_t pos = rr % p.rope_seq;
      const int pair0 = (cc & 63) >> 1;
      o.cs = *reinterpret_cast<const uint2*>(p.rope_cos + pos * 32 + pair0);
      o.sn = *reinterpret_cast<const uint2*>(p.rope_sin + pos * 32 + pair0);
    }
  } else if constexpr (EPI == EPI_BIAS_GELU_) {
    o.b = *reinterpret_cast<const uint4*>(p.bias + cc);
  } else if constexpr (EPI == EPI_DGELU_) {
    o.x = *reinterpret_cast<const uint4*>(p.aux + rr * p.ld_aux + cc);
  }
  return o;
}

// Packed bf16 outputs for 8 consecutive columns [c0, c0+8) of one row of the
// bf16-output epilogues: o0 = C, o1 = the GELU derivative (EPI_BIAS_GELU only).
// Each operation rounds where the reference's bf16 op does: bf16(acc), then
// bias / branch-multiplier / residual as bf16x2 ops with one rounding each.
// Rows and columns outside the matrix produce zeros (the TMA store clips them).
template <int EPI>
__device__ __forceinline__ void epi_pack8(const GemmParams& p, int row, int c0, const float* a,
                                          const EpiOperands& op, uint32_t* o0, uint32_t* o1,
                                          int target, float lse, float cot) {
  if (row >= p.M || c0 >= p.N) {
#pragma unroll
    for (int j = 0; j < 4; ++j) o0[j] = o1[j] = 0u;
    return;
  }
  uint32_t t[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) t[j] = pack_bf16x2(a[2 * j], a[2 * j + 1]);
  if constexpr (EPI == EPI_BF16_) {
    if (p.bias) {
      const uint32_t* bw = &op.b.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) t[j] = hadd2_bf16(t[j], bw[j]);
    }
    if (p.alpha != 1.0f) {
      const uint32_t al = pack_bf16x2(p.alpha, p.alpha);
#pragma unroll
      for (int j = 0; j < 4; ++j) t[j] = hmul2_bf16(t[j], al);
    }
    if (p.resid) {
      const uint32_t* rw = &op.x.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) t[j] = hadd2_bf16(rw[j], t[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o0[j] = t[j];
  } else if constexpr (EPI == EPI_BIAS_ROPE_) {
    // bias, then the interleaved RoPE rotation of q/k columns at this row's
    // position (rig/nn.py:36-52), one bf16 rounding per value as in the reference.
    const uint32_t* bw = &op.b.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = hadd2_bf16(t[j], bw[j]);
    if (c0 < p.rope_cols) {
      float cs[4], sn[4];
      unpack_bf16x2(op.cs.x, cs[0], cs[1]);
      unpack_bf16x2(op.cs.y, cs[2], cs[3]);
      unpack_bf16x2(op.sn.x, sn[0], sn[1]);
      unpack_bf16x2(op.sn.y, sn[2], sn[3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float e, d;
        unpack_bf16x2(t[j], e, d);
        t[j] = pack_bf16x2(e * cs[j] - d * sn[j], e * sn[j] + d * cs[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o0[j] = t[j];
  } else if constexpr (EPI == EPI_BIAS_GELU_) {
    const uint32_t* bw = &op.b.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 u, g, d;
      unpack_bf16x2(hadd2_bf16(t[j], bw[j]), u.x, u.y);
      gelu_tanh_fwd_grad2(u, g, d);
      o0[j] = pack_bf16x2(g.x, g.y);
      o1[j] = pack_bf16x2(d.x, d.y);
    }
  } else if constexpr (EPI == EPI_DGELU_) {
    // du = bf16(alpha * acc) * gelu'(u), the derivative saved by the forward epilogue
    const uint32_t* gw = &op.x.x;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o0[j] = hmul2_bf16(pack_bf16x2(p.alpha * a[2 * j], p.alpha * a[2 * j + 1]), gw[j]);
  } else if constexpr (EPI == EPI_LCE_BWD_) {
    // G = (softmax - onehot(target)) * cotangent
    const float kLog2e = 1.4426950408889634f;
    float g[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = c0 + j;
      const float pr = (c < p.v_sem) ? ex2((a[j] - lse) * kLog2e) : 0.f;
      g[j] = (pr - (c == target ? 1.f : 0.f)) * cot;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o0[j] = pack_bf16x2(g[2 * j], g[2 * j + 1]);
  }
}

// Applies the fp32 / cross-entropy-forward epilogues to 32 accumulator
// columns [col, col+32) of one row (bf16 outputs go through epi_value8).
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int row, int col, int ks,
                                               float* v, EpilogueRowState<EPI>& st, int target,
                                               float lse, float cot) {
  const bool row_ok = row < p.M;
  if constexpr (kStagedEpi<EPI>) {
    return;
  } else if constexpr (EPI == EPI_F32_SPLITK_) {
    // One split: C += alpha * acc directly. Several: this split's raw partial
    // goes to its own slab; splitk_reduce_kernel adds the slabs in split order.
    if (!row_ok) return;
    const bool direct = p.splits == 1;
    float* dst_row = direct ? reinterpret_cast<float*>(p.C) + (int64_t)row * p.ldc
                            : p.slab + ((int64_t)ks * p.M + row) * p.N;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      int c0 = col + 4 * g;
      if (c0 >= p.N) break;
      float4* dst = reinterpret_cast<float4*>(dst_row + c0);
      if (direct) {
        float4 o = *dst;
        *dst = make_float4(o.x + p.alpha * v[4 * g], o.y + p.alpha * v[4 * g + 1],
                           o.z + p.alpha * v[4 * g + 2], o.w + p.alpha * v[4 * g + 3]);
      } else {
        *dst = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
      }
    }
  } else if constexpr (EPI == EPI_F32_) {
    if (!row_ok) return;
    float* C = reinterpret_cast<float*>(p.C);
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      int c0 = col + 4 * g;
      if (c0 >= p.N) break;
      float4* dst = reinterpret_cast<float4*>(C + (int64_t)row * p.ldc + c0);
      float4 w = make_float4(p.alpha * v[4 * g], p.alpha * v[4 * g + 1], p.alpha * v[4 * g + 2],
                             p.alpha * v[4 * g + 3]);
      if (p.accumulate) {
        float4 o = *dst;
        w.x += o.x;
        w.y += o.y;
        w.z += o.z;
        w.w += o.w;
      }
      *dst = w;
    }
  } else if constexpr (EPI == EPI_F32_ATOMIC_) {
    if (!row_ok) return;
    float* C = reinterpret_cast<float*>(p.C);
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      int c0 = col + 4 * g;
      if (c0 >= p.N) break;
      float4* dst = reinterpret_cast<float4*>(C + (int64_t)row * p.ldc + c0);
      atomicAdd(dst, make_float4(p.alpha * v[4 * g], p.alpha * v[4 * g + 1],
                                 p.alpha * v[4 * g + 2], p.alpha * v[4 * g + 3]));
    }
  } else if constexpr (EPI == EPI_LCE_FWD_) {
    // Online log-sum-exp over the semantic vocabulary, plus the target logit.
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (col + j >= p.v_sem) v[j] = -INFINITY;
      m = fmaxf(m, v[j]);
    }
    if (target >= col && target < col + 32) {
      float tv = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j == target) tv = v[j];
      if (row_ok) p.tgt_logit[row] = tv;
    }
    if (m == -INFINITY) return;
    float nm = fmaxf(st.run_max, m);
    const float kLog2e = 1.4426950408889634f;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) s += exp2f((v[j] - nm) * kLog2e);
    st.run_sum = st.run_sum * exp2f((st.run_max - nm) * kLog2e) + s;
    st.run_max = nm;
  }
}

// ------------------------------------------------------------------ kernel
template <int BN, int STAGES, int EPIW, int EPI, int A_MN, int B_MN>
__global__ void __launch_bounds__(64 + 32 * EPIW, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ EpiMaps maps, const GemmParams p) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPIW);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  int* err = &g_gemm_error;
  // device-side M or K range (see GemmParams::range)
  int m_off = 0, tiles_m_eff = p.tiles_m, k_off = 0, kb_eff = p.num_kb;
  if (p.range) {
    const int2 rg = *p.range;
    if (p.range_dim == 1) {
      m_off = rg.x;
      tiles_m_eff = min(p.tiles_m, rg.y / BM);
    } else {
      k_off = rg.x;
      kb_eff = min(p.num_kb, rg.y / BK);
    }
  }
  auto unit_kb = [&](const TileCoord& tc, int& kb0, int& kb1) {
    kb0 = tc.ks * p.kb_per_split;
    kb1 = min(kb_eff, kb0 + p.kb_per_split);
    return tc.tm < tiles_m_eff && kb0 < kb1;  // false: nothing to do in this unit
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
        TileCoord tc = decode_unit(p, u);
        int kb0, kb1;
        if (!unit_kb(tc, kb0, kb1)) continue;
        const int m0 = m_off + tc.tm * BM, n0 = tc.tn * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err)) goto producer_done;
          uint8_t* sa = smem + stage * L::STAGE_BYTES;
          uint8_t* sb = sa + L::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
          const int k0 = k_off + kb * BK;
          if constexpr (!A_MN) {
            tma_load_2d(sa, &tmA, &full[stage], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(sa + j * 64 * BK * 2, &tmA, &full[stage], m0 + 64 * j, k0);
          }
          if constexpr (!B_MN) {
            tma_load_2d(sb, &tmB, &full[stage], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * 64 * BK * 2, &tmB, &full[stage], n0 + 64 * j, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
        TileCoord tc = decode_unit(p, u);
        int kb0, kb1;
        if (!unit_kb(tc, kb0, kb1)) continue;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t dtmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
          for (int ki = 0; ki < BK / 16; ++ki) {
            // K-major SW128: rows of 128 B, 8-row atoms 1024 B apart; a K step
            // of 16 bf16 advances the start address by 32 B inside the atom.
            // MN-major SW128: 64-wide MN blocks (LBO apart), 8-k-row atoms
            // 1024 B apart (SBO); a K step of 16 rows advances 2048 B.
            const uint64_t ad = A_MN ? umma_smem_desc(sa + ki * 2048, 64 * BK * 2, 1024)
                                     : umma_smem_desc(sa + ki * 32, 16, 1024);
            const uint64_t bd = B_MN ? umma_smem_desc(sb + ki * 2048, 64 * BK * 2, 1024)
                                     : umma_smem_desc(sb + ki * 32, 16, 1024);
            umma_bf16(dtmem, ad, bd, idesc, (kb > kb0 || ki > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ---------------- epilogue warps 2..17: warp w reads the TMEM lanes of
    // quadrant w % 4 and one quarter (BN / 4 columns) of the tile. Both 32-column
    // loads are issued before one wait, and the accumulator is handed back to
    // the MMA warp as soon as it is in registers.
    constexpr int COLS = BN / 4;
    constexpr int PASSES = 16 / EPIW;  // column quarters a warp takes in turn
    const int quad = warp & 3;
    const int wpart = (warp - 2) >> 2;
    const int r_in_tile = quad * 32 + lane;
    float2* red = reinterpret_cast<float2*>(smem + L::RED_OFFSET);  // [4][128] LCE partials
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
      TileCoord tc = decode_unit(p, u);
      int kb0, kb1;
      if (!unit_kb(tc, kb0, kb1)) continue;
      const int row = m_off + tc.tm * BM + r_in_tile;
      for (int vp = 0; vp < PASSES; ++vp) {
      const int part = wpart * PASSES + vp;
      const int n0 = tc.tn * BN + part * COLS;
      if constexpr (EPI == EPI_BF16_) {
        // The residual rows of this thread's slice of the NEXT tile go to L2
        // now, a whole epilogue ahead of their loads (measured: the K = 768
        // projection with a residual 10% faster; the same prefetch of the
        // saved GELU derivative made the dGELU class 5% slower, so it has none).
        const int un = u + gridDim.x;
        if (p.resid && un < p.num_units) {
          const TileCoord tn = decode_unit(p, un);
          const int rn = m_off + tn.tm * BM + r_in_tile;
          const int cn = tn.tn * BN + part * COLS;
          const bf16* src = nullptr;
          if (rn < p.M && cn < p.N) src = p.resid + (int64_t)rn * p.ld_resid + cn;
          if (src) {
#pragma unroll
            for (int c = 0; c < COLS * 2; c += 128) prefetch_l2(reinterpret_cast<const char*>(src) + c);
          }
        }
      }
      if (vp == 0) {
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, err)) goto epi_done;
        tc_fence_after();
      }
      int target = -1;
      float lse = 0.f, cot = 0.f;
      if constexpr (EPI == EPI_LCE_FWD_ || EPI == EPI_LCE_BWD_) {
        if (row < p.M) {
          target = p.targets[row];
          if (target < 0 || target >= p.v_sem) target = -1;
          if constexpr (EPI == EPI_LCE_BWD_) {
            lse = p.lse[row];
            cot = (target >= 0) ? p.cot[row] : 0.f;
          }
        }
      }
      uint32_t raw[COLS];
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + part * COLS;
#pragma unroll
      for (int c = 0; c < COLS / 32; ++c) tmem_ld32_nw(taddr + c * 32, raw + c * 32);
      tmem_wait_ld();
      if (vp == PASSES - 1) {  // the whole slice is in registers: hand the accumulator back
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      }
      EpilogueRowState<EPI> st;
      if constexpr (kStagedEpi<EPI>) {
        // bf16 outputs: 32x32 sub-tiles through the warp's swizzled staging
        // tile, written by TMA stores (full 128-byte lines, clipped to M x N).
        uint8_t* stage = smem + L::STAGE_OFFSET + (warp - 2) * L::STAGE_TILE;
        constexpr int NOUT = (EPI == EPI_BIAS_GELU_) ? 2 : 1;
#pragma unroll
        for (int c = 0; c < COLS / 32; ++c) {
          uint32_t out0[16], out1[16];
          // operand loads of PRE groups at a time are issued before their math
          constexpr int PRE = (EPI == EPI_BF16_ || EPI == EPI_BIAS_ROPE_) ? 2 : 4;
#pragma unroll
          for (int g0 = 0; g0 < 4; g0 += PRE) {
            EpiOperands op[PRE];
#pragma unroll
            for (int g = 0; g < PRE; ++g) op[g] = epi_load8<EPI>(p, row, n0 + c * 32 + (g0 + g) * 8);
#pragma unroll
            for (int g = 0; g < PRE; ++g) {
              float a8[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) a8[j] = __uint_as_float(raw[c * 32 + (g0 + g) * 8 + j]);
              epi_pack8<EPI>(p, row, n0 + c * 32 + (g0 + g) * 8, a8, op[g], out0 + 4 * (g0 + g),
                             out1 + 4 * (g0 + g), target, lse, cot);
            }
          }
#pragma unroll
          for (int o = 0; o < NOUT; ++o) {
            const uint32_t* w = o ? out1 : out0;
            if (lane == 0) bulk_wait_read();
            __syncwarp();
#pragma unroll
            for (int g = 0; g < 4; ++g)
              *reinterpret_cast<uint4*>(stage + lane * 64 + ((g ^ ((lane >> 1) & 3)) << 4)) =
                  make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(o ? &maps.aux : &maps.c, stage, n0 + c * 32, m_off + tc.tm * BM + quad * 32);
              bulk_commit();
            }
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < COLS / 32; ++c) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[c * 32 + i]);
          epilogue_chunk<EPI>(p, row, n0 + c * 32, tc.ks, v, st, target, lse, cot);
        }
      }
      if constexpr (EPI == EPI_LCE_FWD_) red[part * BM + r_in_tile] = make_float2(st.run_max, st.run_sum);
      }  // passes
      if constexpr (EPI == EPI_LCE_FWD_) {
        // combine the four column quarters of each row, one partial per tile
        named_bar_sync(1, 32 * EPIW);
        if (wpart == 0 && row < p.M) {
          const float kLog2e = 1.4426950408889634f;
          float m = -INFINITY, sum = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 e = red[q * BM + r_in_tile];
            if (e.x == -INFINITY) continue;
            const float nm = fmaxf(m, e.x);
            sum = sum * exp2f((m - nm) * kLog2e) + e.y * exp2f((e.x - nm) * kLog2e);
            m = nm;
          }
          p.partial[(int64_t)row * p.tiles_n + tc.tn] = make_float2(m, sum);
        }
        named_bar_sync(1, 32 * EPIW);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

epi_done:
  if constexpr (kStagedEpi<EPI>) {
    if (warp >= 2 && lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// C[r, c] += alpha * (((slab_0 + slab_1) + slab_2) + ...)[r, c]: the K splits of
// an EPI_F32_SPLITK_ product, added in split order so that the result is the
// same whichever CTA finished first. One float4 of C per thread.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ slab,
                                                            int splits, int64_t M, int N,
                                                            float* __restrict__ C, int64_t ldc,
                                                            float alpha) {
  const int64_t per = M * (int64_t)N;
  const int64_t n4 = per >> 2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i << 2;
    const int64_t r = e / N;
    const int c = (int)(e - r * N);
    float4 s = __ldcs(reinterpret_cast<const float4*>(slab + e));
    for (int k = 1; k < splits; ++k) {
      const float4 t = __ldcs(reinterpret_cast<const float4*>(slab + k * per + e));
      s.x += t.x;
      s.y += t.y;
      s.z += t.z;
      s.w += t.w;
    }
    float4* dst = reinterpret_cast<float4*>(C + r * ldc + c);
    const float4 o = *dst;
    *dst = make_float4(o.x + alpha * s.x, o.y + alpha * s.y, o.z + alpha * s.z, o.w + alpha * s.w);
  }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor map: `inner` contiguous elements per row, `outer` rows,
// row stride `ld` elements, box {64, box_outer}, 128-byte swizzle.
static bool make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t ld,
                     int box_outer) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Store map of a bf16 [outer, inner] output (row stride ld): box 32 x 32 with
// 64-byte swizzle, matching the epilogue staging tiles.
static bool make_store_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer,
                           int64_t ld) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cache[64] = {0};
  if (dev < 64 && cache[dev]) return cache[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cache[dev] = n;
  return n;
}

// Epilogue warps by kind: the heavy per-element epilogues (GELU and its
// derivative, RoPE, the two cross-entropy epilogues) use 8, the others 16.
template <int EPI>
constexpr int kEpiWarpsFor = (EPI == EPI_BIAS_GELU_ || EPI == EPI_DGELU_ || EPI == EPI_BIAS_ROPE_ ||
                              EPI == EPI_LCE_BWD_ || EPI == EPI_LCE_FWD_)
                                 ? 8
                                 : 16;

template <int BN, int STAGES, int EPI, int A_MN, int B_MN>
static int launch_variant(const CUtensorMap& ta, const CUtensorMap& tb, const EpiMaps& em,
                          const GemmParams& p, cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  constexpr int EPIW = kEpiWarpsFor<EPI>;
  auto kern = gemm_tc_kernel<BN, STAGES, EPIW, EPI, A_MN, B_MN>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
    if (e != cudaSuccess) return -static_cast<int>(e);
    if (dev < 64) configured[dev] = true;
  }
  int grid = std::min<int64_t>(p.num_units, sm_count());
  kern<<<grid, 64 + 32 * EPIW, L::TOTAL, stream>>>(ta, tb, em, p);
  GPTB200_CHECK_LAUNCH();
  return GPTB200_OK;
}

constexpr int kBN = 256;
constexpr int kStages = 4;

template <int EPI>
static int dispatch_layout(int a_mn, int b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                           const EpiMaps& em, const GemmParams& p, cudaStream_t s) {
  if (a_mn == 0 && b_mn == 0) return launch_variant<kBN, kStages, EPI, 0, 0>(ta, tb, em, p, s);
  if (a_mn == 0 && b_mn == 1) return launch_variant<kBN, kStages, EPI, 0, 1>(ta, tb, em, p, s);
  if (a_mn == 1 && b_mn == 0) return launch_variant<kBN, kStages, EPI, 1, 0>(ta, tb, em, p, s);
  return launch_variant<kBN, kStages, EPI, 1, 1>(ta, tb, em, p, s);
}

static int gemm_split_request(int64_t M, int64_t N, int64_t K);

int gemm_launch(const void* a, int a_mn, int64_t lda, const void* b, int b_mn, int64_t ldb,
                int64_t M, int64_t N, int64_t K, int epi, GemmParams p, cudaStream_t stream) {
  if (!a || !b || !p.C) return GPTB200_EINVAL;
  if (M <= 0 || N <= 0 || K <= 0) return GPTB200_EINVAL;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return GPTB200_ESHAPE;
  if ((lda % 8) || (ldb % 8) || (N % 8)) return GPTB200_ESHAPE;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
       reinterpret_cast<uintptr_t>(p.C)) & 15)
    return GPTB200_ESHAPE;
  if (a_mn ? lda < M : lda < K) return GPTB200_ESHAPE;
  if (b_mn ? ldb < N : ldb < K) return GPTB200_ESHAPE;
  if (p.ldc < N || (p.ldc % 8)) return GPTB200_ESHAPE;

  CUtensorMap ta, tb;
  bool ok = a_mn ? make_map(&ta, a, M, K, lda, BK) : make_map(&ta, a, K, M, lda, BM);
  ok = ok && (b_mn ? make_map(&tb, b, N, K, ldb, BK) : make_map(&tb, b, K, N, ldb, kBN));
  if (!ok) return GPTB200_ESHAPE;
  EpiMaps em;
  memset(&em, 0, sizeof(em));
  if (epi == EPI_BF16_ || epi == EPI_BIAS_ROPE_ || epi == EPI_BIAS_GELU_ || epi == EPI_DGELU_ ||
      epi == EPI_LCE_BWD_) {
    if (!make_store_map(&em.c, p.C, N, M, p.ldc)) return GPTB200_ESHAPE;
    if (epi == EPI_BIAS_GELU_ && !make_store_map(&em.aux, p.aux, N, M, p.ld_aux))
      return GPTB200_ESHAPE;
  }

  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.tiles_m = (int)((M + BM - 1) / BM);
  p.tiles_n = (int)((N + kBN - 1) / kBN);
  p.num_kb = (int)((K + BK - 1) / BK);
  int splits = 1;
  if (epi == EPI_F32_ATOMIC_ || epi == EPI_F32_SPLITK_) splits = gemm_split_request(M, N, K);
  // Raster groups: enough M tiles that a wave of CTAs spans few N tiles, with
  // the group's A stripe (group_m x BM rows of K) at most ~16 MB of L2.
  {
    const int64_t stripe = (int64_t)BM * K * 2;
    int g = (int)std::max<int64_t>(1, std::min<int64_t>(32, (16ll << 20) / stripe));
    p.group_m = std::min(g, p.tiles_m);
  }
  p.kb_per_split = (p.num_kb + splits - 1) / splits;
  p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
  p.num_units = p.tiles_m * p.tiles_n * p.splits;

  switch (epi) {
    case EPI_BF16_: return dispatch_layout<EPI_BF16_>(a_mn, b_mn, ta, tb, em, p, stream);
    case EPI_F32_: return dispatch_layout<EPI_F32_>(a_mn, b_mn, ta, tb, em, p, stream);
    case EPI_F32_ATOMIC_: return dispatch_layout<EPI_F32_ATOMIC_>(a_mn, b_mn, ta, tb, em, p, stream);
    case EPI_F32_SPLITK_: {
      if (p.splits > 1 && !p.slab) return GPTB200_EINVAL;
      int s = dispatch_layout<EPI_F32_SPLITK_>(a_mn, b_mn, ta, tb, em, p, stream);
      if (s || p.splits == 1) return s;
      const int64_t n4 = (int64_t)p.M * p.N / 4;
      const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)sm_count() * 8);
      splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(p.slab, p.splits, p.M, p.N,
                                                      reinterpret_cast<float*>(p.C), p.ldc,
                                                      p.alpha);
      GPTB200_CHECK_LAUNCH();
      return GPTB200_OK;
    }
    case EPI_BIAS_ROPE_:
      if (a_mn || !b_mn) return GPTB200_EUNSUPPORTED;
      return launch_variant<kBN, kStages, EPI_BIAS_ROPE_, 0, 1>(ta, tb, em, p, stream);
    case EPI_BIAS_GELU_:
      if (a_mn || !b_mn) return GPTB200_EUNSUPPORTED;
      return launch_variant<kBN, kStages, EPI_BIAS_GELU_, 0, 1>(ta, tb, em, p, stream);
    case EPI_DGELU_:
      if (a_mn || b_mn) return GPTB200_EUNSUPPORTED;
      return launch_variant<kBN, kStages, EPI_DGELU_, 0, 0>(ta, tb, em, p, stream);
    case EPI_LCE_FWD_:
      if (a_mn || b_mn) return GPTB200_EUNSUPPORTED;
      return launch_variant<kBN, kStages, EPI_LCE_FWD_, 0, 0>(ta, tb, em, p, stream);
    case EPI_LCE_BWD_:
      if (a_mn || b_mn) return GPTB200_EUNSUPPORTED;
      return launch_variant<kBN, kStages, EPI_LCE_BWD_, 0, 0>(ta, tb, em, p, stream);
    default: return GPTB200_EUNSUPPORTED;
  }
}

int gemm_tile_n() { return kBN; }

static int gemm_split_request(int64_t M, int64_t N, int64_t K) {
  // The split count with the shortest main-loop critical path, in k-blocks
  // per CTA: waves of units over the SMs x k-blocks per unit. Ties go to the
  // fewer splits (less fp32 partial traffic: every unit ends in a BM x BN
  // slab write that the ordered reduction reads back). A unit keeps >= 32
  // k-blocks (2048 of K) so its write-out hides behind the next unit's loop,
  // and at most 256 (16,384 of K): the accumulation error of the fp32 TMEM
  // accumulator grows with the length it runs over (measured relative error
  // ~1.1e-9 x K per unit), while the slabs are added in exact fp32.
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + kBN - 1) / kBN);
  const int64_t num_kb = (K + BK - 1) / BK;
  const int64_t sms = sm_count();
  int s0 = 1;
  while (s0 < 64 && (num_kb + s0 - 1) / s0 > 256) s0 *= 2;
  int best_s = s0;
  int64_t best = INT64_MAX;
  for (int s = s0; s <= 64 && (s == s0 || num_kb / s >= 32); s *= 2) {
    const int64_t waves = (tiles * s + sms - 1) / sms;
    const int64_t cost = waves * ((num_kb + s - 1) / s);
    if (cost < best) {
      best = cost;
      best_s = s;
    }
  }
  return best_s;
}

// Splits that actually run: k-blocks are dealt in runs of ceil(num_kb / request).
int gemm_splits(int64_t M, int64_t N, int64_t K) {
  const int64_t num_kb = (K + BK - 1) / BK;
  const int64_t per = (num_kb + gemm_split_request(M, N, K) - 1) / gemm_split_request(M, N, K);
  return (int)((num_kb + per - 1) / per);
}

int gemm_read_error(int clear) {
  int h = 0;
  cudaMemcpyFromSymbol(&h, g_gemm_error, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemm_error, &z, sizeof(int));
  }
  return h;
}

}  // namespace gptb200

extern "C" int gptb200_gemm(const void* a, int a_mn_major, int64_t lda, const void* b,
                            int b_mn_major, int64_t ldb, void* c, int64_t ldc, int64_t m,
                            int64_t n, int64_t k, const gptb200_epilogue* e, void* stream) {
  using namespace gptb200;
  if (!e) return GPTB200_EINVAL;
  GemmParams p = {};
  p.C = c;
  p.ldc = ldc;
  p.alpha = e->alpha;
  p.accumulate = e->accumulate;
  p.bias = reinterpret_cast<const bf16*>(e->bias);
  p.resid = reinterpret_cast<const bf16*>(e->residual);
  p.ld_resid = e->ld_residual;
  p.aux = reinterpret_cast<bf16*>(e->aux);
  p.ld_aux = e->ld_aux;
  int kind;
  switch (e->kind) {
    case GPTB200_EPI_BF16: kind = EPI_BF16_; break;
    case GPTB200_EPI_BIAS_GELU:
      if (!e->bias || !e->aux || e->ld_aux < n || (e->ld_aux % 8)) return GPTB200_EINVAL;
      kind = EPI_BIAS_GELU_;
      break;
    case GPTB200_EPI_DGELU:
      if (!e->aux || e->ld_aux < n || (e->ld_aux % 8)) return GPTB200_EINVAL;
      kind = EPI_DGELU_;
      break;
    case GPTB200_EPI_BIAS_ROPE:
      if (!e->bias || !e->rope_cos || !e->rope_sin || e->rope_seq <= 0 || e->rope_cols < 0 ||
          (e->rope_cols % 64) || e->rope_cols > n)
        return GPTB200_EINVAL;
      kind = EPI_BIAS_ROPE_;
      p.rope_cos = reinterpret_cast<const bf16*>(e->rope_cos);
      p.rope_sin = reinterpret_cast<const bf16*>(e->rope_sin);
      p.rope_seq = (int)e->rope_seq;
      p.rope_cols = (int)e->rope_cols;
      break;
    case GPTB200_EPI_F32: kind = EPI_F32_; break;
    case GPTB200_EPI_F32_ATOMIC: kind = EPI_F32_ATOMIC_; break;
    case GPTB200_EPI_F32_SPLITK:
      kind = EPI_F32_SPLITK_;
      p.slab = reinterpret_cast<float*>(e->workspace);
      if (e->row_range) return GPTB200_EUNSUPPORTED;
      if (e->workspace && (reinterpret_cast<uintptr_t>(e->workspace) & 15)) return GPTB200_ESHAPE;
      break;
    default: return GPTB200_EUNSUPPORTED;
  }
  if (e->residual && (e->ld_residual < n || (e->ld_residual % 8))) return GPTB200_EINVAL;
  if (e->range_dim < 0 || e->range_dim > 2 || (e->range_dim != 0) != (e->row_range != nullptr))
    return GPTB200_EINVAL;
  if (e->range_dim == 2 && !(a_mn_major && b_mn_major)) return GPTB200_EUNSUPPORTED;
  if (e->range_dim == 1 && a_mn_major) return GPTB200_EUNSUPPORTED;
  p.range = reinterpret_cast<const int2*>(e->row_range);
  p.range_dim = e->range_dim;
  // bias / residual / derivative rows are read in 16-byte groups of 8 columns
  if ((e->bias || e->residual || kind == EPI_BIAS_GELU_ || kind == EPI_DGELU_) && (n % 8))
    return GPTB200_ESHAPE;
  if (kind == EPI_F32_ || kind == EPI_F32_ATOMIC_ || kind == EPI_F32_SPLITK_) {
    if (ldc % 4) return GPTB200_ESHAPE;
  }
  return gemm_launch(a, a_mn_major, lda, b, b_mn_major, ldb, m, n, k, kind, p,
                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t gptb200_gemm_workspace_size(int64_t m, int64_t n, int64_t k, int kind) {
  if (m <= 0 || n <= 0 || k <= 0 || kind != GPTB200_EPI_F32_SPLITK) return 0;
  const int splits = gptb200::gemm_splits(m, n, k);
  return splits > 1 ? (size_t)splits * (size_t)m * (size_t)n * sizeof(float) : 0;
}
