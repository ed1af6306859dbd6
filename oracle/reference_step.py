"""CPU restatement of the reference GPT training step — TEST INFRASTRUCTURE ONLY.

This module is the parity oracle for the B200 step. Only tests/, the smoke()
check of __graft_entry__.py and the `cpu_baseline` / `--impl reference` legs of
bench.py may import it; the product path (rig_b200) never does.

It restates, in PyTorch on the CPU, the arithmetic of the reference JAX step
(honglu2875/GPT-speedrun-TPU) with the same dtype flow: bf16 activations and
bf16 residual stream, fp32 statistics, bf16 operands with fp32 accumulation
for every contraction, fp32 master parameters and AdamW.

    rms_norm            rig/nn.py:26-33
    apply_rotary        rig/nn.py:36-52
    linear              rig/nn.py:55-56
    init_params         recipes/reference/train.py:865-901 (draw order)
    gpt_hidden          recipes/reference/train.py:1096-1176
    attention           rig/kernels/tpu_flash_attention.py:171-207
                        (reference_causal_attention: fp32 softmax, bf16 P)
    tiled LCE + VJP     rig/kernels/linear_cross_entropy.py:115-302
    learning_rate       recipes/reference/train.py:1219-1236
    decay mask          recipes/reference/train.py:1252-1271
    CompleteP trees     recipes/reference/train.py:1274-1333
    betas               recipes/reference/train.py:1336-1345
    AdamW update        recipes/reference/train.py:1362-1457

Third-party semantics restated: `jax.nn.gelu(approximate=True)` is the tanh
form; an XLA dot of bf16 operands accumulates in fp32 and rounds its output to
bf16; fused elementwise chains round once at their output.

Parity status: JAX is not installable in this container (no network), so the
restatement itself cannot be executed side by side with the reference step.
It is pinned by the reference's own invariants that run without JAX (see
tests/test_oracle.py); absolute step-level parity against JAX is UNPINNED.
"""

from __future__ import annotations

import math
from typing import Any

import numpy as np
import torch
import torch.nn.functional as F

BF16 = torch.bfloat16
F32 = torch.float32
BLOCK_FIELDS = (
    "ln1_scale", "qkv_w", "qkv_b", "attn_w", "attn_b",
    "ln2_scale", "mlp_up_w", "mlp_up_b", "mlp_down_w", "mlp_down_b",
)


# ------------------------------------------------------------------ layer math
def rms_norm(x: torch.Tensor, scale: torch.Tensor, dtype=BF16) -> torch.Tensor:
    x32 = x.to(F32)
    normalized = x32 * torch.rsqrt((x32 * x32).mean(-1, keepdim=True) + 1.0e-5)
    return normalized.to(dtype) * scale.to(dtype)


def rope_tables(length: int, head_dim: int, dtype=BF16):
    fraction = torch.arange(0, head_dim, 2, dtype=F32) / float(head_dim)
    inverse_frequency = torch.pow(torch.tensor(10000.0, dtype=F32), -fraction)
    angle = torch.arange(length, dtype=F32)[:, None] * inverse_frequency[None, :]
    return torch.cos(angle).to(dtype), torch.sin(angle).to(dtype)


def apply_rotary(x: torch.Tensor) -> torch.Tensor:
    """Interleaved base-10000 RoPE of one BTHD tensor (one rounding per output)."""

    length, head_dim = x.shape[1], x.shape[-1]
    cos, sin = rope_tables(length, head_dim, x.dtype)
    cos = cos[None, :, None, :].to(F32)
    sin = sin[None, :, None, :].to(F32)
    even = x[..., 0::2].to(F32)
    odd = x[..., 1::2].to(F32)
    out = torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1)
    return out.reshape(x.shape).to(x.dtype)


def bf16_dot(a: torch.Tensor, b: torch.Tensor, dtype=BF16) -> torch.Tensor:
    """XLA dot of `dtype` operands: fp32 accumulation, output rounded to `dtype`."""

    return (a.to(dtype).to(F32) @ b.to(dtype).to(F32)).to(dtype)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, dtype=BF16):
    return bf16_dot(x, weight, dtype) + bias.to(dtype)


def causal_attention(q, k, v, scale: float, segment_ids=None) -> torch.Tensor:
    """reference_causal_attention on BHSD tensors
    (rig/kernels/tpu_flash_attention.py:171-207): with segment_ids [B, T], a
    query sees only keys of its own segment, on top of the causal mask."""

    t = q.shape[2]
    scores = (q.to(F32) @ k.to(F32).transpose(-1, -2)) * scale
    visible = torch.ones(t, t, dtype=torch.bool).tril()
    if segment_ids is not None:
        seg = torch.as_tensor(segment_ids)
        same = seg[:, None, :, None] == seg[:, None, None, :]
        visible = visible[None, None] & same
    scores = torch.where(visible, scores, torch.tensor(-0.7 * torch.finfo(F32).max))
    probabilities = torch.softmax(scores, dim=-1).to(v.dtype)
    return (probabilities.to(F32) @ v.to(F32)).to(q.dtype)


# ------------------------------------------------------------------ tiled LCE
class TiledLinearCrossEntropy(torch.autograd.Function):
    """Per-token losses of the tied head with the reference's custom VJP.

    Forward: log-sum-exp over the semantic vocabulary of fp32 logits from bf16
    operands; target logit by a separate fp32-accumulated dot; +inf for an
    invalid target. Backward: G = (softmax - onehot) * cotangent (zero for an
    invalid target), dH = G·E accumulated in fp32 and cast to hidden's dtype,
    dE = Gᵀ·H in fp32 (cast to the embedding's dtype, fp32 here).
    """

    @staticmethod
    def forward(ctx, hidden, embedding, targets, semantic_vocab_size: int, dtype=BF16):
        h = hidden.reshape(-1, hidden.shape[-1]).to(dtype).to(F32)
        e = embedding.to(dtype).to(F32)
        logits = h @ e.T
        vocab = embedding.shape[0]
        valid_cols = torch.arange(vocab) < semantic_vocab_size
        logits = torch.where(valid_cols[None, :], logits, torch.tensor(-math.inf))
        lse = torch.logsumexp(logits, dim=-1)
        t = targets.reshape(-1).long()
        valid = (t >= 0) & (t < semantic_vocab_size)
        safe = t.clamp(0, semantic_vocab_size - 1)
        target_logits = (h * e[safe]).sum(-1)
        losses = torch.where(valid, lse - target_logits, torch.tensor(math.inf))
        ctx.save_for_backward(hidden, embedding, targets, lse)
        ctx.semantic_vocab_size = semantic_vocab_size
        ctx.dtype = dtype
        return losses.reshape(targets.shape)

    @staticmethod
    def backward(ctx, cot):
        hidden, embedding, targets, lse = ctx.saved_tensors
        dtype = ctx.dtype
        sv = ctx.semantic_vocab_size
        h = hidden.reshape(-1, hidden.shape[-1]).to(dtype).to(F32)
        e = embedding.to(dtype).to(F32)
        t = targets.reshape(-1).long()
        valid = (t >= 0) & (t < sv)
        c = torch.where(valid, cot.reshape(-1).to(F32), torch.zeros(()))
        logits = h @ e.T
        vocab = embedding.shape[0]
        cols = torch.arange(vocab)
        probs = torch.where((cols < sv)[None, :], torch.exp(logits - lse[:, None]), torch.zeros(()))
        onehot = (t[:, None] == cols[None, :]).to(F32)
        g = (probs - onehot) * c[:, None]
        g16 = g.to(dtype).to(F32)
        dh = (g16 @ e).to(hidden.dtype).reshape(hidden.shape)
        de = (g16.T @ h).to(embedding.dtype)
        return dh, de, None, None, None


def tiled_tied_cross_entropy(hidden, embedding, targets, semantic_vocab_size, dtype=BF16):
    losses = TiledLinearCrossEntropy.apply(hidden, embedding, targets, semantic_vocab_size, dtype)
    return losses.to(F32).mean()


# ------------------------------------------------------------------ model
def document_segments(tokens, boundary_token: int):
    """rig/attention.py:205-208: each token's document index inside its window
    (cumulative count of boundary tokens, the boundary opening a new document)."""

    return np.cumsum(np.asarray(tokens) == boundary_token, axis=1).astype(np.int32)


def init_params(cfg: Any, seed: int) -> dict[str, np.ndarray]:
    """train.py:865-901 with rig/nn.py:20-23's normal()."""

    rng = np.random.default_rng(seed)
    d, hidden = cfg.d_model, cfg.mlp_mult * cfg.d_model
    width = cfg.d_model / float(cfg.base_width)
    hidden_scale = (cfg.init_std / math.sqrt(width)
                    if cfg.parameterization == "completep_fixed_tpp_v1" else 0.02)

    def normal(shape, scale):
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)

    out: dict[str, np.ndarray] = {}
    for b in range(cfg.layers):
        out[f"blocks/{b}/ln1_scale"] = np.ones((d,), np.float32)
        out[f"blocks/{b}/qkv_w"] = normal((d, 3 * d), hidden_scale)
        out[f"blocks/{b}/qkv_b"] = np.zeros((3 * d,), np.float32)
        out[f"blocks/{b}/attn_w"] = normal((d, d), hidden_scale)
        out[f"blocks/{b}/attn_b"] = np.zeros((d,), np.float32)
        out[f"blocks/{b}/ln2_scale"] = np.ones((d,), np.float32)
        experts = getattr(cfg, "experts", 0)
        if experts:  # recipes/reference_moe/train.py:905-931 (router, then experts)
            eh = cfg.expert_mult * d
            out[f"blocks/{b}/router_w"] = normal((d, experts), hidden_scale)
            out[f"blocks/{b}/expert_up_w"] = normal((experts, d, eh), hidden_scale)
            out[f"blocks/{b}/expert_up_b"] = np.zeros((experts, eh), np.float32)
            out[f"blocks/{b}/expert_down_w"] = normal((experts, eh, d), hidden_scale)
            out[f"blocks/{b}/expert_down_b"] = np.zeros((experts, d), np.float32)
            continue
        out[f"blocks/{b}/mlp_up_w"] = normal((d, hidden), hidden_scale)
        out[f"blocks/{b}/mlp_up_b"] = np.zeros((hidden,), np.float32)
        out[f"blocks/{b}/mlp_down_w"] = normal((hidden, d), hidden_scale)
        out[f"blocks/{b}/mlp_down_b"] = np.zeros((d,), np.float32)
    out["token_embedding"] = normal((cfg.vocab_size, d), cfg.init_std)
    out["final_ln_scale"] = np.ones((d,), np.float32)
    if cfg.embeddings != "tied":
        out["output_embedding"] = normal((cfg.vocab_size, d), cfg.init_std / width)
    return out


def softmax_scale(cfg) -> float:
    head_dim = cfg.d_model // cfg.heads
    return 1.0 / head_dim if cfg.attention_scale == "inverse_head_dim" else head_dim ** -0.5


def routed_mlp(x, router_w, up_w, up_b, down_w, down_b, experts: int, top_k: int, dtype=BF16):
    """recipes/reference_moe/train.py:1230-1311 (routed_mlp_local, one device):
    fp32 router logits, softmax probabilities, top-k logits and their softmax
    gates, stable sort of the assignments by expert, per-expert bf16 matmuls
    with fp32 accumulation (megablox.gmm), bias, tanh GELU, bias, gate weighting
    in bf16 and a bf16 scatter-add back to the tokens. Returns the output and
    the per-expert mean probability, load and (entropy, top-1 gate, logit RMS)."""

    batch, length, width = x.shape
    n = batch * length
    flat = x.reshape(n, width)
    logits = flat.to(F32) @ router_w.to(F32)
    probabilities = torch.softmax(logits, dim=-1)
    chosen_logits, chosen = torch.topk(logits, top_k, dim=-1)
    gate = torch.softmax(chosen_logits, dim=-1)
    assignments = chosen.reshape(-1)
    order = torch.argsort(assignments, stable=True)
    sorted_assignments = assignments[order]
    counts = torch.bincount(assignments, minlength=experts)
    rows = torch.arange(n).repeat_interleave(top_k)[order]
    grouped = flat[rows].to(dtype)
    hidden_parts, out_parts = [], []
    start = 0
    for e in range(experts):
        seg = grouped[start:start + int(counts[e])]
        hidden_parts.append(bf16_dot(seg, up_w[e], dtype))
        start += int(counts[e])
    hidden = torch.cat(hidden_parts) + up_b[sorted_assignments].to(dtype)
    hidden = F.gelu(hidden.to(F32), approximate="tanh").to(dtype)
    start = 0
    for e in range(experts):
        out_parts.append(bf16_dot(hidden[start:start + int(counts[e])], down_w[e], dtype))
        start += int(counts[e])
    out = torch.cat(out_parts) + down_b[sorted_assignments].to(dtype)
    weighted = out * gate.reshape(-1)[order][:, None].to(dtype)
    combined = torch.zeros(n, width, dtype=dtype).index_add(0, rows, weighted)
    mean_probability = probabilities.mean(dim=0)
    load = counts.to(F32) / float(n * top_k)
    entropy = -(probabilities * torch.log(probabilities + 1.0e-9)).sum(-1).mean()
    summary = torch.stack((entropy, gate.max(dim=-1).values.mean(),
                           torch.sqrt(torch.mean(logits * logits))))
    return combined.reshape(batch, length, width), mean_probability, load, summary


def load_balance_loss(mean_probability, load):
    """recipes/reference_moe/train.py:1347-1372: E * sum(load * mean probability)."""

    return float(load.shape[0]) * torch.sum(load * mean_probability)


def gpt_hidden(params: dict[str, torch.Tensor], tokens: torch.Tensor, cfg, dtype=BF16,
               router_out: list | None = None):
    batch, length = tokens.shape
    heads = cfg.heads
    head_dim = cfg.d_model // heads
    mult = (cfg.layers / float(cfg.base_depth)) ** (-cfg.depth_alpha)
    scale = softmax_scale(cfg)
    segments = (document_segments(tokens.numpy(), cfg.document_boundary_token)
                if getattr(cfg, "document_masking", False) else None)  # train.py:1127-1131
    x = params["token_embedding"][tokens.long()].to(dtype)
    for b in range(cfg.layers):
        p = {k: v for k, v in ((f.split("/")[-1], params[f]) for f in params
                                if f.startswith(f"blocks/{b}/"))}
        residual = x
        xn = rms_norm(x, p["ln1_scale"], dtype)
        qkv = linear(xn, p["qkv_w"], p["qkv_b"], dtype)
        q, k, v = torch.split(qkv, cfg.d_model, dim=-1)
        q = apply_rotary(q.reshape(batch, length, heads, head_dim))
        k = apply_rotary(k.reshape(batch, length, heads, head_dim))
        v = v.reshape(batch, length, heads, head_dim)
        att = causal_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale,
                               segments)
        att = att.transpose(1, 2).reshape(batch, length, cfg.d_model)
        x = residual + mult * linear(att, p["attn_w"], p["attn_b"], dtype)
        residual = x
        xn = rms_norm(x, p["ln2_scale"], dtype)
        if getattr(cfg, "experts", 0):
            mlp_out, mean_p, load, summary = routed_mlp(
                xn, p["router_w"], p["expert_up_w"], p["expert_up_b"], p["expert_down_w"],
                p["expert_down_b"], cfg.experts, cfg.expert_top_k, dtype)
            if router_out is not None:
                router_out.append((mean_p, load, summary))
            x = residual + mult * mlp_out
            continue
        hidden = linear(xn, p["mlp_up_w"], p["mlp_up_b"], dtype)
        hidden = F.gelu(hidden.to(F32), approximate="tanh").to(dtype)
        x = residual + mult * linear(hidden, p["mlp_down_w"], p["mlp_down_b"], dtype)
    return rms_norm(x, params["final_ln_scale"], dtype)


def loss_fn(params, x, y, cfg, dtype=BF16):
    """recipes/reference/train.py:1194-1216; for routed models plus the
    coefficient times the layer-mean balance loss
    (recipes/reference_moe/train.py:1562-1602)."""

    router: list = []
    hidden = gpt_hidden(params, x, cfg, dtype, router)
    emb = params.get("output_embedding", params["token_embedding"])
    loss = tiled_tied_cross_entropy(hidden, emb, y, cfg.semantic_vocab_size, dtype)
    if router and cfg.router_aux_coefficient:
        balance = torch.stack([load_balance_loss(mp, ld) for mp, ld, _ in router]).mean()
        loss = loss + cfg.router_aux_coefficient * balance
    return loss


def loss_and_grads(params_np: dict[str, np.ndarray], x, y, cfg, dtype=BF16):
    params = {k: torch.tensor(v, dtype=F32, requires_grad=True) for k, v in params_np.items()}
    loss = loss_fn(params, torch.as_tensor(x), torch.as_tensor(y), cfg, dtype)
    loss.backward()
    grads = {k: p.grad.detach().to(F32).numpy() for k, p in params.items()}
    return float(loss.detach()), grads


# ------------------------------------------------------------------ optimizer
def eval_step(params_np: dict[str, np.ndarray], x, y, mask, cfg, dtype=BF16) -> tuple[float, float]:
    """recipes/reference/train.py:1494-1525 (tiled loss backend): the masked
    per-token loss sum and the mask sum, both fp32."""

    params = {k: torch.from_numpy(np.asarray(v, np.float32)) for k, v in params_np.items()}
    with torch.no_grad():
        hidden = gpt_hidden(params, torch.as_tensor(x), cfg, dtype)
        emb = params.get("output_embedding", params["token_embedding"])
        losses = TiledLinearCrossEntropy.apply(hidden, emb, torch.as_tensor(y),
                                               cfg.semantic_vocab_size, dtype).to(F32)
        m = torch.as_tensor(mask).to(F32)
        return float((losses * m).sum()), float(m.sum())


def learning_rate(step: int, cfg) -> float:
    s = np.float32(step)
    if cfg.warmup_steps:
        warmup = np.minimum(np.float32(1.0), s / np.float32(cfg.warmup_steps))
    else:
        warmup = np.float32(1.0)
    span = max(1, cfg.steps - cfg.warmup_steps)
    progress = np.clip((s - np.float32(cfg.warmup_steps)) / np.float32(span), 0.0, 1.0)
    cosine = np.float32(0.5) * (np.float32(1.0) + np.cos(np.float32(np.pi) * progress))
    mult = np.float32(cfg.min_lr_ratio) + np.float32(1.0 - cfg.min_lr_ratio) * cosine
    horizon = math.sqrt(cfg.batch_multiplier / cfg.data_multiplier)
    return float(np.float32(cfg.learning_rate * horizon) * warmup * mult)


def multipliers(name: str, cfg) -> tuple[float, float, float, bool]:
    """(lr, eps, decay multipliers, decay flag) of a flat parameter name."""

    leaf = name.rsplit("/", 1)[-1]
    if leaf in {"token_embedding", "output_embedding"} or leaf.endswith("_w"):
        decay = True
    elif leaf.endswith(("_b", "_bias", "_scale")):
        decay = False
    else:
        raise ValueError(f"no decay rule for {leaf!r}")
    if cfg.parameterization != "completep_fixed_tpp_v1":
        return 1.0, 1.0, 1.0, decay
    width = cfg.d_model / float(cfg.base_width)
    depth = cfg.layers / float(cfg.base_depth)
    alpha = cfg.depth_alpha
    if name.startswith("blocks/"):
        lr = width ** -1 * depth ** (alpha - 1.0) if leaf.endswith("_w") else depth ** (alpha - 1.0)
        return lr, width ** -1 * depth ** -alpha, (width if leaf.endswith("_w") else 1.0), decay
    if leaf == "token_embedding":
        return 1.0, width ** -1, 1.0, decay
    if leaf == "output_embedding":
        return width ** -1, 1.0, width, decay
    return 1.0, 1.0, 1.0, decay


def adamw_update(params, m, v, grads, step: int, cfg) -> tuple[dict, dict, dict, float, float]:
    """One CompleteP AdamW update in fp32 (train.py:1362-1457). Returns
    (params, m, v, lr, grad_norm); `step` is the new (1-based) step."""

    ratio = cfg.batch_multiplier / cfg.data_multiplier
    beta1 = 1.0 - (1.0 - cfg.beta1) * ratio
    beta2 = 1.0 - (1.0 - cfg.beta2) * ratio
    grad_norm = float(np.sqrt(sum(float(np.sum(np.square(g, dtype=np.float64))) for g in grads.values())))
    clip = min(1.0, cfg.grad_clip / (grad_norm + 1.0e-6)) if cfg.grad_clip > 0 else 1.0
    lr = learning_rate(step, cfg)
    bc1 = np.float32(1.0) - np.float32(beta1) ** np.float32(step)
    bc2 = np.float32(1.0) - np.float32(beta2) ** np.float32(step)
    eps_h = math.sqrt(cfg.data_multiplier / cfg.batch_multiplier)
    wd_h = math.sqrt(cfg.batch_multiplier / cfg.data_multiplier)
    new_p, new_m, new_v = {}, {}, {}
    for k in params:
        g = grads[k].astype(np.float32) * np.float32(clip)
        mk = np.float32(beta1) * m[k] + np.float32(1.0 - beta1) * g
        vk = np.float32(beta2) * v[k] + np.float32(1.0 - beta2) * np.square(g)
        lr_m, eps_m, wd_m, decay = multipliers(k, cfg)
        eps = np.float32(cfg.adam_epsilon * eps_h * eps_m)
        adam = (mk / bc1) / (np.sqrt(vk / bc2) + eps)
        dec = np.float32(cfg.weight_decay * wd_h * wd_m) * params[k] if decay else np.float32(0.0)
        new_p[k] = (params[k] - np.float32(lr) * np.float32(lr_m) * (adam + dec)).astype(np.float32)
        new_m[k] = mk.astype(np.float32)
        new_v[k] = vk.astype(np.float32)
    return new_p, new_m, new_v, lr, grad_norm


class OracleTrainer:
    """The whole reference step on the CPU: loss, grads, AdamW, history."""

    def __init__(self, cfg, params: dict[str, np.ndarray], dtype=BF16):
        self.cfg = cfg
        self.dtype = dtype
        self.params = {k: v.astype(np.float32).copy() for k, v in params.items()}
        self.m = {k: np.zeros_like(v) for k, v in self.params.items()}
        self.v = {k: np.zeros_like(v) for k, v in self.params.items()}
        self.step = 0
        self.history: list[tuple[float, float, float]] = []

    def train_step(self, x, y) -> float:
        loss, grads = loss_and_grads(self.params, x, y, self.cfg, self.dtype)
        self.step += 1
        self.params, self.m, self.v, lr, gn = adamw_update(
            self.params, self.m, self.v, grads, self.step, self.cfg)
        self.history.append((loss, lr, gn))
        return loss
