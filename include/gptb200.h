/*
 * libgptb200 — C ABI of the B200 (sm_100a) kernels behind the GPT training step
 * of the GPT-speedrun rig (recipes/reference/train.py, train_step at :1460-1472).
 *
 * Conventions (every entry point):
 *   - Pointers are device pointers unless the parameter says "host".
 *   - bf16 tensors are passed as `void*` (IEEE bfloat16, row-major).
 *   - `stream` is a cudaStream_t passed as `void*` (NULL = legacy stream).
 *   - Return value: 0 on success, a positive GPTB200_E* code for an argument or
 *     shape error (checked before anything is launched), or the negated
 *     cudaError_t of a failed launch. Nothing throws across this boundary.
 *   - No entry point allocates device memory. Scratch space that a kernel needs
 *     is passed in as `workspace`, sized by the matching *_workspace_size().
 *   - All work is stream-ordered and asynchronous; entry points are reentrant.
 *
 * Each declaration names the reference interface it replaces (file:line within
 * the reference project honglu2875/GPT-speedrun-TPU).
 */
#ifndef GPTB200_H_
#define GPTB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GPTB200_OK 0
#define GPTB200_EINVAL 1       /* bad argument: null pointer, non-positive size */
#define GPTB200_ESHAPE 2       /* unsupported shape / alignment */
#define GPTB200_EUNSUPPORTED 3 /* unsupported combination of options */
#define GPTB200_EDEVICE 4      /* a kernel reported a device-side error (bounded wait ran out) */
#define GPTB200_ERANGE 5       /* token id outside the vocabulary */
#define GPTB200_ETOOLARGE 6    /* size exceeds the fixed scratch of an allocation-free entry point */

/* Library identification; no reference counterpart. */
const char* gptb200_version(void);
const char* gptb200_status_string(int status);

/* Reads (and with clear != 0 resets) the device-side error flags of every
 * kernel family on the current device. Returns 0 when no kernel reported an
 * error, else GPTB200_EDEVICE. Synchronizes the device. */
int gptb200_device_error(int clear);

/* The same flags as a bit mask (0: none). Synchronizes the device. */
#define GPTB200_DEVERR_GEMM 1         /* a GEMM / cross-entropy wait ran out of time */
#define GPTB200_DEVERR_ATTENTION 2    /* an attention wait ran out of time */
#define GPTB200_DEVERR_TOKEN_RANGE 4  /* the embedding gather saw an id outside [0, vocab) */
#define GPTB200_DEVERR_NONFINITE 8    /* the optimizer saw a NaN/inf loss or gradient norm */
int gptb200_device_error_flags(int clear);

/* Number of kernels this library has launched in this process (all devices).
 * Used by the benchmark to report how many native launches a step makes; no
 * reference counterpart. */
uint64_t gptb200_launch_count(void);

/* ------------------------------------------------------------------ GEMM
 * C[M,N] = epilogue( sum_k A[m,k] * B[n,k] ), bf16 operands, fp32 accumulate
 * in tensor memory (tcgen05.mma, TMA-fed).
 *   a_mn_major = 0: A stored [M, K] (row stride lda >= K)
 *   a_mn_major = 1: A stored [K, M] (row stride lda >= M)
 *   b_mn_major = 0: B stored [N, K] (row stride ldb >= K)
 *   b_mn_major = 1: B stored [K, N] (row stride ldb >= N)
 * Replaces rig/nn.py:55-56 (`linear`: einsum("...d,df->...f", x, W) + b) and
 * the projections of recipes/reference/train.py:1136,1164-1166,1170-1174, with
 * their XLA-generated transposes for the backward pass. Leading dimensions and
 * N must be multiples of 8 elements; pointers 16-byte aligned.
 */
#define GPTB200_EPI_BF16 0       /* C bf16 = resid + alpha*(bf16(acc) + bias), each step rounded to bf16 */
#define GPTB200_EPI_BIAS_GELU 1  /* u = bf16(bf16(acc)+bias); C bf16 = gelu_tanh(u);
                                    aux bf16 = gelu_tanh'(u) (saved for the backward) */
#define GPTB200_EPI_DGELU 2      /* C bf16 = bf16(alpha*acc) * aux, aux from EPI_BIAS_GELU */
#define GPTB200_EPI_F32 3        /* C fp32 = alpha*acc (accumulate=1: C += alpha*acc) */
#define GPTB200_EPI_F32_ATOMIC 4 /* C fp32 += alpha*acc with atomics; K may be split across CTAs */
#define GPTB200_EPI_BIAS_ROPE 5  /* C bf16 = bf16(acc)+bias, then columns < rope_cols rotated by
                                    RoPE at position (row % rope_seq), pairs (2i, 2i+1) within
                                    each 64-wide head (the QKV projection + apply_rotary) */
#define GPTB200_EPI_F32_SPLITK 6 /* C fp32 += alpha*acc; K may be split across CTAs, each split
                                    writing its partial product to its own slab of `workspace`
                                    (gptb200_gemm_workspace_size bytes, 0 when K is not split),
                                    the slabs then added in split order: bit-reproducible.
                                    Calls sharing a workspace must not overlap on the GPU. */

typedef struct gptb200_epilogue {
  int kind;              /* GPTB200_EPI_* */
  int accumulate;        /* EPI_F32 only */
  float alpha;           /* 1.0f for none */
  const void* bias;      /* bf16 [N] or NULL (EPI_BF16, required for EPI_BIAS_GELU) */
  const void* residual;  /* bf16 [M, ld_residual] or NULL (EPI_BF16) */
  int64_t ld_residual;
  void* aux;             /* bf16 [M, ld_aux]: written by BIAS_GELU, read by DGELU */
  int64_t ld_aux;
  const void* rope_cos;  /* EPI_BIAS_ROPE: bf16 [rope_seq, 32] tables (gptb200_rope_tables) */
  const void* rope_sin;
  int64_t rope_seq;      /* rows are token positions row % rope_seq */
  int64_t rope_cols;     /* columns [0, rope_cols) are rotated (q and k: 2 * d_model) */
  /* Optional device-resident row range: int32 {offset, count} with count a
   * multiple of 128, read when the kernel starts. range_dim 1: only rows
   * [offset, offset + count) of A and C take part (m = the buffer's rows);
   * range_dim 2: only K rows [offset, offset + count) of MN-major A and B
   * (k = the buffer's rows). 0: no range. Used for per-expert segments of a
   * token buffer whose sizes are only known on the device. */
  const int32_t* row_range;
  int range_dim;
  void* workspace;       /* EPI_F32_SPLITK: scratch of gptb200_gemm_workspace_size bytes */
} gptb200_epilogue;

/* Scratch bytes gptb200_gemm needs for an m x n x k product with epilogue
 * `kind` on the current device (0 for every kind but EPI_F32_SPLITK, and for
 * that one when K is not split). */
size_t gptb200_gemm_workspace_size(int64_t m, int64_t n, int64_t k, int kind);

int gptb200_gemm(const void* a, int a_mn_major, int64_t lda, const void* b, int b_mn_major,
                 int64_t ldb, void* c, int64_t ldc, int64_t m, int64_t n, int64_t k,
                 const gptb200_epilogue* epilogue, void* stream);

/* ------------------------------------------------------------------ RMSNorm
 * y = bf16(x * rsqrt(mean(x^2) + 1e-5)) * scale   (fp32 statistics)
 * Replaces rig/nn.py:26-33 (`rms_norm`). x, y, scale bf16; rstd fp32 [rows]
 * (saved for the backward pass). d must be a multiple of 8 and <= 4096
 * (<= 2048 for the backward).
 */
int gptb200_rms_norm_fwd(const void* x, const void* scale, void* y, float* rstd, int64_t rows,
                         int64_t d, void* stream);

/* Backward of rms_norm. dx_out (bf16) = dx_in (bf16 residual-stream gradient,
 * may be NULL for zero, may alias dx_out) + d(rms_norm)/dx · dy.
 * dscale (fp32 [d]) is accumulated into (+=). With dx_colsum != NULL the column
 * sums of dx_out times colsum_alpha are accumulated into dx_colsum (fp32 [d]):
 * the bias gradient of the residual branch that consumed this gradient.
 * Both column reductions add per-block partials (kept in `workspace`, sized by
 * gptb200_rms_norm_bwd_workspace_size) in a fixed order: repeated calls give
 * bit-identical results. Replaces the XLA autodiff of rig/nn.py:26-33. */
size_t gptb200_rms_norm_bwd_workspace_size(int64_t rows, int64_t d);
int gptb200_rms_norm_bwd(const void* x, const void* scale, const float* rstd, const void* dy,
                         const void* dx_in, void* dx_out, float* dscale, float* dx_colsum,
                         float colsum_alpha, int64_t rows, int64_t d, void* workspace,
                         void* stream);

/* ------------------------------------------------------------------ embedding
 * out[i, :] = bf16(table[tokens[i], :]); Replaces recipes/reference/train.py:1107
 * (`params["token_embedding"][tokens].astype(dtype)`). table bf16 [vocab, d].
 * Token ids outside [0, vocab) are clamped (the step validates ids on the host,
 * rig/tokens.py:262-268). */
int gptb200_embedding_fwd(const int32_t* tokens, const void* table, void* out, int64_t n,
                          int64_t d, int64_t vocab, void* stream);
/* dtable[tokens[i], :] += dout[i, :] (fp32). Backward of the gather. The rows
 * are sorted by (token, row) on the device and each token's rows are added in
 * that order, so the result is bit-identical from run to run (no atomics).
 * Tokens outside [0, vocab) contribute nothing. d must be a multiple of 8;
 * workspace of gptb200_embedding_bwd_workspace_size bytes, 16-byte aligned. */
size_t gptb200_embedding_bwd_workspace_size(int64_t n, int64_t d, int64_t vocab);
int gptb200_embedding_bwd(const int32_t* tokens, const void* dout, float* dtable, int64_t n,
                          int64_t d, int64_t vocab, void* workspace, void* stream);

/* ------------------------------------------------------------------ RoPE
 * Tables of the interleaved base-10000 rotary embedding of rig/nn.py:36-52:
 * angle[t, i] = t * 10000^(-2i/head_dim) in fp32, cos/sin rounded to bf16.
 * cos_out, sin_out: bf16 [seq, head_dim/2]. */
int gptb200_rope_tables(void* cos_out, void* sin_out, int64_t seq, int64_t head_dim,
                        void* stream);

/* Applies (inverse = 0) or undoes (inverse = 1, the transpose rotation, i.e.
 * the backward of apply_rotary) the interleaved RoPE in place on a
 * [batch, seq, heads, head_dim] bf16 view with element strides (stride_b,
 * stride_t, stride_h) and a contiguous head dimension. Replaces rig/nn.py:36-52
 * (`apply_rotary`) when q/k are not produced by a GEMM with EPI_BIAS_ROPE. */
int gptb200_rope_apply(void* x, int64_t stride_b, int64_t stride_t, int64_t stride_h,
                       int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                       const void* rope_cos, const void* rope_sin, int inverse, void* stream);

/* Document ids for attention masking (rig/attention.py:205-208): out[b, t] =
 * count of boundary_token in tokens[b, 0..t] (int32 [batch, seq] both). */
int gptb200_document_segments(const int32_t* tokens, int64_t batch, int64_t seq,
                              int32_t boundary_token, int32_t* out, void* stream);

/* ------------------------------------------------------------------ attention
 * Causal softmax attention on tcgen05 tensor cores, fp32 statistics, bf16 P
 * before P·V. q and k are taken as given (already rotated: in the training
 * step RoPE runs in the QKV projection epilogue, GPTB200_EPI_BIAS_ROPE).
 * Tensors are addressed as base + b*stride_b + h*stride_h + t*stride_t + e
 * (element strides); q, k, v share (stride_b, stride_h, stride_t), o and do
 * share (o_stride_*). lse: fp32 [batch, heads, seq] (natural-log units of the
 * scaled scores). head_dim must be 64; strides multiples of 8 elements.
 * segment_ids: NULL (causal only) or int32 [batch, seq] document ids: a query
 * then sees a key only if both carry the same id (block-diagonal over
 * documents on top of the causal mask, reference_causal_attention's
 * segment_ids); key blocks whose id range misses a query tile's are skipped.
 * With segment ids, seq <= 65536 (GPTB200_EUNSUPPORTED otherwise).
 * Replaces rig/kernels/tpu_flash_attention.py:236-348 (forward kernel) behind
 * make_causal_attention (:962-1164); semantics of reference_causal_attention
 * (:171-207).
 */
int gptb200_attention_fwd(const void* q, const void* k, const void* v, int64_t stride_b,
                          int64_t stride_h, int64_t stride_t, void* o, int64_t o_stride_b,
                          int64_t o_stride_h, int64_t o_stride_t, float* lse, int64_t batch,
                          int64_t heads, int64_t seq, int64_t head_dim, float softmax_scale,
                          const int32_t* segment_ids, void* stream);

size_t gptb200_attention_bwd_workspace_size(int64_t batch, int64_t heads, int64_t seq);

/* Backward: dq, dk, dv are written (not accumulated) with the q/k/v strides.
 * segment_ids: as in the forward (the same ids, or NULL).
 * With rope tables (the ones q and k were rotated with), dq and dk are rotated
 * back, i.e. they are gradients with respect to the unrotated q and k.
 * Replaces rig/kernels/tpu_flash_attention.py:479-575 (dQ) and :578-701 (dK/dV). */
int gptb200_attention_bwd(const void* q, const void* k, const void* v, int64_t stride_b,
                          int64_t stride_h, int64_t stride_t, const void* o, const void* dout,
                          int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_t,
                          const float* lse, void* dq, void* dk, void* dv, int64_t batch,
                          int64_t heads, int64_t seq, int64_t head_dim, float softmax_scale,
                          const void* rope_cos, const void* rope_sin, const int32_t* segment_ids,
                          void* workspace, void* stream);

/* ------------------------------------------------------------------ routed MLP (MoE)
 * recipes/reference_moe/train.py:1230-1372 (routed_mlp_local, load_balance_loss)
 * as kernels around gptb200_gemm. Assignment a = token * top_k + choice; the
 * assignments are stably sorted by expert into one row buffer of
 * gptb200_moe_rows() rows, expert e owning rows [seg[2e], seg[2e] + seg[2e+1])
 * (its count rounded up to 128; padding rows are zero on the way in and
 * ignored on the way out). The expert GEMMs read seg[2e..2e+1] on the device
 * (gptb200_epilogue.row_range), so no host synchronisation is needed.
 * stats (fp32, per layer, accumulated): [0, E) router-probability sums,
 * [E, 2E) assignment counts, entropy sum, top-1 gate sum, sum of squared
 * logits. 1 <= E <= 16, 1 <= top_k <= min(4, E). */
size_t gptb200_moe_rows(int64_t tokens, int32_t top_k, int32_t experts);
size_t gptb200_moe_dispatch_workspace_size(int64_t tokens, int32_t top_k, int32_t experts);
/* logits fp32 [tokens, E] = x (bf16 [tokens, d], promoted to fp32) . router_w
 * (fp32 [d, E]); chosen/gate [tokens, top_k]: top-k experts (ties: lower
 * index first) and the softmax of their logits. */
int gptb200_moe_route(const void* x, const float* router_w, int64_t tokens, int64_t d,
                      int32_t experts, int32_t top_k, float* logits, int32_t* chosen, float* gate,
                      float* stats, void* stream);
/* seg int32 [E, 2], total int32 [1] (rows in use), pos int32 [tokens, top_k]
 * (row of each assignment), src int32 [rows] (token of each row, -1 padding),
 * grouped bf16 [rows, d] = x[src]. */
int gptb200_moe_dispatch(const int32_t* chosen, int64_t tokens, int32_t top_k, int32_t experts,
                         const void* x, int64_t d, int32_t* seg, int32_t* total, int32_t* pos,
                         int32_t* src, void* grouped, void* workspace, void* stream);
/* x_out = residual + alpha * sum_j bf16(out[pos(t, j)] * bf16(gate(t, j))) (bf16). */
int gptb200_moe_combine(const void* out, const int32_t* pos, const float* gate,
                        const void* residual, float alpha, int64_t tokens, int64_t d,
                        int32_t top_k, void* x_out, void* stream);
/* Backward of the combine for dx = d x_out: d_out rows (zero on padding) and
 * d_gate fp32 [tokens, top_k]. */
int gptb200_moe_combine_bwd(const void* dx, float alpha, const void* out, const int32_t* pos,
                            const float* gate, const int32_t* src, const int32_t* total,
                            int64_t tokens, int64_t d, int32_t top_k, void* d_out, float* d_gate,
                            void* stream);
/* Router backward: d_logits from the gates and from the balance loss (bal_grad
 * fp32 [E]: d loss / d router probability, equal for every token); d_router_w
 * += x^T d_logits (fp32); d_x = bf16(sum_j d_grouped[pos] + d_logits router_w^T). */
int gptb200_moe_route_bwd(const void* x, const float* router_w, const float* logits,
                          const int32_t* chosen, const float* gate, const float* d_gate,
                          const float* bal_grad, const void* d_grouped, const int32_t* pos,
                          int64_t tokens, int64_t d, int32_t experts, int32_t top_k,
                          float* d_router_w, void* d_x, void* stream);
/* out fp32 [E, width] += column sums of buf (bf16 [rows, width], 16-byte
 * aligned, width % 8 == 0) over each expert's segment (per-expert bias
 * gradients). */
int gptb200_moe_segment_colsum(const void* buf, const int32_t* seg, int32_t experts,
                               int64_t width, float* out, void* stream);
/* From the (rank-summed) stats of all layers: balance loss per layer, the
 * backward coefficients bal_grad [layers, E] (= coefficient / layers * E * load
 * * bwd_scale), loss += coefficient * mean balance, and the router history row
 * (train.py:1881-1915: balance, max load, min load, mean entropy / top-1 gate /
 * logit RMS, then per layer those three and the load vector) written to row
 * *step of history [history_rows, 6 + layers * (3 + E)]. */
int gptb200_moe_finalize(const float* stats, int32_t layers, int32_t experts, int64_t tokens,
                         int32_t top_k, float coefficient, float bwd_scale, float* bal_grad,
                         float* loss, float* history, int32_t history_rows, const int32_t* step,
                         void* stream);

/* ------------------------------------------------------------------ linear cross-entropy
 * Tied-embedding cross entropy without materializing [n, vocab] logits:
 * loss[i] = logsumexp_{v < v_semantic}(h_i · E_v) - h_i · E_{target_i}
 * (+inf for a target outside [0, v_semantic)). hidden bf16 [n, d], embedding
 * bf16 [v_storage, d], targets int32 [n]. Outputs: losses fp32 [n], lse fp32
 * [n] (saved for the backward), mean_loss fp32 [1] = mean(losses).
 * Replaces rig/kernels/linear_cross_entropy.py:115-179 and :349-368
 * (`tiled_tied_cross_entropy` / `_losses`).
 */
size_t gptb200_lce_fwd_workspace_size(int64_t n, int64_t v_storage);
int gptb200_lce_fwd(const void* hidden, const void* embedding, const int32_t* targets, int64_t n,
                    int64_t d, int64_t v_storage, int64_t v_semantic, float* losses, float* lse,
                    float* mean_loss, void* workspace, void* stream);

/* Allocation-free variant of gptb200_lce_fwd, for callers that cannot allocate
 * device memory or own a workspace: for example an XLA custom-call handler,
 * whose device memory is owned by XLA's allocator, or code recording a CUDA
 * graph, where cudaMalloc is not allowed. Same arguments and results as
 * gptb200_lce_fwd without `workspace`: the scratch lives in a fixed 8 MiB
 * device array inside this library, held by every GPU that loads it until the
 * process exits. Limits: n <= 16384 rows and n * ceil(v_storage / 256) <=
 * 1,048,576 (about 5,300 rows at vocabulary 50,304); larger sizes return
 * GPTB200_ETOOLARGE before anything is launched. The first call on a device
 * looks up the array's device address (a one-time set-up), so make it before
 * any stream capture. All calls share the one array: calls that overlap on the
 * GPU (different streams, or devices sharing nothing but this process) race.
 * No counterpart in the reference. */
int gptb200_lce_fwd_noalloc(const void* hidden, const void* embedding, const int32_t* targets,
                            int64_t n, int64_t d, int64_t v_storage, int64_t v_semantic,
                            float* losses, float* lse, float* mean_loss, void* stream);

/* Backward with per-token cotangent dlosses (fp32 [n]; for the mean this is
 * 1/n everywhere). dhidden bf16 [n, d] is written; dembedding fp32
 * [v_storage, d] is accumulated into (+=); rows >= v_semantic receive nothing.
 * Targets outside [0, v_semantic) contribute no gradient.
 * Replaces rig/kernels/linear_cross_entropy.py:220-302. */
size_t gptb200_lce_bwd_workspace_size(int64_t n, int64_t v_storage);
int gptb200_lce_bwd(const void* hidden, const void* embedding, const int32_t* targets,
                    const float* lse, const float* dlosses, int64_t n, int64_t d,
                    int64_t v_storage, int64_t v_semantic, void* dhidden, float* dembedding,
                    void* workspace, void* stream);

/* ------------------------------------------------------------------ reductions
 * Evaluation reduction of recipes/reference/train.py:1494-1525 (eval_step):
 * out[0] = sum(losses * mask), out[1] = sum(mask), both fp32, over n per-token
 * losses (from gptb200_lce_fwd) and an fp32 mask. Deterministic (one block). */
int gptb200_masked_loss_sum(const float* losses, const float* mask, int64_t n, float* out,
                            void* stream);

/* out[j] += alpha * sum_i x[i, j] for bf16 x [rows, n] (the bias gradients of
 * recipes/reference/train.py's projections, XLA's reduction of the bias
 * cotangent). Per-block partials in `workspace` (gptb200_colsum_workspace_size
 * bytes) are added in a fixed order: bit-identical from run to run. */
size_t gptb200_colsum_workspace_size(int64_t rows, int64_t n);
int gptb200_colsum(const void* x, int64_t rows, int64_t n, float alpha, float* out,
                   void* workspace, void* stream);

/* ------------------------------------------------------------------ optimizer
 * CompleteP AdamW over one flat fp32 parameter buffer, replacing
 * recipes/reference/train.py:1362-1457 (`_apply_training_update` after the
 * gradients: global grad norm, optional clip, m/v update, bias correction,
 * per-tensor lr/eps/decay multipliers of :1274-1333, history row).
 */
typedef struct gptb200_tensor_group {
  int64_t offset;        /* first element in the flat buffers */
  int64_t size;          /* element count */
  float lr_mult;
  float eps_mult;
  float wd_mult;
  int32_t decay;         /* 1 when weight decay applies (train.py:1252-1271) */
} gptb200_tensor_group;

typedef struct gptb200_adamw_config {
  float learning_rate;       /* base lr (config.learning_rate) */
  float horizon_lr_scale;    /* sqrt(batch_multiplier / data_multiplier) */
  float min_lr_ratio;
  int32_t warmup_steps;
  int32_t total_steps;
  float beta1, beta2;        /* effective betas (train.py:1336-1345) */
  float eps;                 /* config.adam_epsilon */
  float eps_horizon_scale;   /* sqrt(data_multiplier / batch_multiplier) */
  float weight_decay;
  float wd_horizon_scale;    /* sqrt(batch_multiplier / data_multiplier) */
  float grad_clip;           /* <= 0: disabled */
  float grad_scale;          /* gradients are multiplied by this first (1.0) */
} gptb200_adamw_config;

/* Device scalars of the optimizer: step (int32, incremented by the update),
 * plus the per-step values written for the history row. */
size_t gptb200_adamw_workspace_size(int64_t n);

/* One update. groups: DEVICE array of n_groups gptb200_tensor_group covering
 * [0, n) in increasing offset order. step: device int32 (read, then +1).
 * loss: device fp32 scalar (the step's mean loss) for the history row.
 * history: device fp32 [total_steps, 3] rows (loss, lr, grad_norm); may be NULL.
 * params_bf16: optional bf16 mirror of params written after the update. */
int gptb200_adamw_step(float* params, float* m, float* v, const float* grads, int64_t n,
                       const gptb200_tensor_group* groups, int32_t n_groups,
                       const gptb200_adamw_config* cfg, int32_t* step, const float* loss,
                       float* history, void* params_bf16, void* workspace, void* stream);

/* The same update in parts, so that each gradient bucket can be updated as
 * soon as it is final (right after its all-reduce) while the backward pass
 * goes on, for configurations without gradient clipping (grad_clip <= 0: the
 * learning rate and bias corrections then do not depend on the global norm;
 * GPTB200_EUNSUPPORTED otherwise). One step is:
 *   gptb200_adamw_begin         advances *step, computes this step's scalars
 *   gptb200_adamw_update_range  per bucket: elements [begin, end) (begin a
 *                               multiple of 4); stores the bucket's squared
 *                               gradient sums in slot `slot` (0 <= slot < 256,
 *                               one slot per bucket)
 *   gptb200_adamw_end           gradient norm from slots [0, n_slots) in slot
 *                               order (deterministic), history row, and the
 *                               non-finite flag.
 * Same workspace as gptb200_adamw_step; the results equal its results except
 * for the summation order of the logged gradient norm. Replaces the update
 * of recipes/reference/train.py:1362-1457 like gptb200_adamw_step. */
int gptb200_adamw_begin(const gptb200_adamw_config* cfg, int32_t* step, void* workspace,
                        void* stream);
int gptb200_adamw_update_range(float* params, float* m, float* v, const float* grads,
                               int64_t begin, int64_t end, const gptb200_tensor_group* groups,
                               int32_t n_groups, const gptb200_adamw_config* cfg, int32_t slot,
                               void* params_bf16, void* workspace, void* stream);
int gptb200_adamw_end(int32_t n_slots, const gptb200_adamw_config* cfg, const int32_t* step,
                      const float* loss, float* history, void* workspace, void* stream);

/* fp32 -> bf16 copy of n elements (the compute-dtype cast of train.py's
 * `weight.astype(dtype)`). */
int gptb200_cast_bf16(const float* src, void* dst, int64_t n, void* stream);

/* ------------------------------------------------------------------ data loader (host)
 * Native core of rig/tokens.py:171-272 (`ShuffledEpochBatchStream`). All
 * pointers in this section are HOST pointers; these functions run on the CPU.
 */
/* SplitMix64 avalanche of rig/tokens.py:127-133. */
uint64_t gptb200_mix_uint64(uint64_t value);
/* Keyed bounded Feistel permutation of rig/tokens.py:136-168. Returns the
 * image of `value` in [0, size), or UINT64_MAX for value >= size. */
uint64_t gptb200_permute_bounded(uint64_t value, uint64_t size, uint64_t key);
/* Element types of token shards. */
#define GPTB200_TOKENS_U8 0
#define GPTB200_TOKENS_U16 1
#define GPTB200_TOKENS_I32 2
#define GPTB200_TOKENS_U32 3
#define GPTB200_TOKENS_I64 4
/* Windows first .. first + rows - 1 of epoch `epoch` of the shuffled stream
 * (rig/tokens.py:221-254), each seq_len + 1 tokens, into out (int32
 * [rows, seq_len + 1]). shards/lengths: n_shards host arrays of element type
 * `dtype`; order: the epoch's shard order (int64 permutation of
 * 0..n_shards-1, the caller's numpy PCG64 draw of rig/tokens.py:222-227).
 * Computes the epoch's window table, the epoch key mix(seed ^ mix(epoch)),
 * the keyed permutation of each window ordinal and the copy. The ordinals
 * must lie inside the epoch. Returns 0, GPTB200_ERANGE if a token lies
 * outside [0, vocab) (the window is still copied), or GPTB200_EINVAL. */
int gptb200_epoch_windows(const void* const* shards, const int64_t* lengths, int64_t n_shards,
                          int dtype, const int64_t* order, int64_t seq_len, uint64_t seed,
                          int64_t epoch, int64_t first, int64_t rows, int64_t vocab,
                          int32_t* out);

#ifdef __cplusplus
}
#endif

#endif /* GPTB200_H_ */
