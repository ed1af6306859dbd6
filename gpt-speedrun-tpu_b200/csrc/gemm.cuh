// Internal interface of the tcgen05 GEMM (gemm.cu), shared with lce.cu.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gptb200 {

enum {
  EPI_BF16_ = 0,
  EPI_BIAS_GELU_ = 1,
  EPI_DGELU_ = 2,
  EPI_F32_ = 3,
  EPI_F32_ATOMIC_ = 4,
  EPI_BIAS_ROPE_ = 5,
  EPI_F32_SPLITK_ = 6,  // C fp32 += alpha * acc, K splits reduced in a fixed order
  EPI_LCE_FWD_ = 10,  // per (row, N-tile) partial (max, sum exp) + target logit
  EPI_LCE_BWD_ = 11,  // bf16 (softmax - onehot) * cotangent
};

struct GemmParams {
  // filled by gemm_launch
  int M, N, K;
  int tiles_m, tiles_n, num_kb, kb_per_split, splits, num_units;
  int group_m;  // M tiles per raster group (consecutive units sweep a group's N tiles)
  // Optional device-side row range {offset, count} (count a multiple of 128)
  // read at kernel start: range_dim 1 restricts the M rows (A and C rows
  // offset, tiles past the count do nothing), 2 the K rows of MN-major
  // operands. Lets a segment of a buffer whose bounds live on the device (an
  // expert's tokens) be multiplied without a host round trip.
  const int2* range;
  int range_dim;
  // output + generic epilogue operands
  void* C;
  int64_t ldc;
  float alpha;
  int accumulate;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* resid;
  int64_t ld_resid;
  __nv_bfloat16* aux;
  int64_t ld_aux;
  // RoPE epilogue
  const __nv_bfloat16* rope_cos;
  const __nv_bfloat16* rope_sin;
  int rope_seq;
  int rope_cols;
  // cross-entropy epilogues
  const int32_t* targets;
  const float* lse;
  const float* cot;
  float2* partial;    // [M, tiles_n]
  float* tgt_logit;   // [M]
  int v_sem;
  // EPI_F32_SPLITK_: per-split fp32 partial products [splits][M][N]
  float* slab;
};

// Validates shapes, encodes the TMA maps and launches the persistent kernel.
int gemm_launch(const void* a, int a_mn, int64_t lda, const void* b, int b_mn, int64_t ldb,
                int64_t M, int64_t N, int64_t K, int epi, GemmParams p, cudaStream_t stream);
int gemm_tile_n();
// K splits the weight-gradient epilogues use for an M x N x K product.
int gemm_splits(int64_t M, int64_t N, int64_t K);
int gemm_read_error(int clear);

}  // namespace gptb200
