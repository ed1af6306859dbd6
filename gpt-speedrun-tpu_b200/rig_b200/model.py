"""The GPT training step on one GPU (and its data-parallel replicas).

`GPTTrainer` replaces the reference's jitted ``train_step``
(recipes/reference/train.py:1460-1472, wiring of `gpt_hidden` :1096-1176,
loss :1194-1216, update :1362-1457). It owns:

* one flat fp32 buffer each for parameters, gradients and the two Adam
  moments, with every tensor at a 64-element-aligned offset (so any tensor
  view is 16-byte aligned for TMA and 128-bit accesses), plus a bf16 mirror
  of the parameters that the update kernel rewrites every step (the
  ``weight.astype(dtype)`` of rig/nn.py:56);
* every activation the backward pass reads, preallocated once for the local
  batch (the step is static-shaped, so nothing is allocated per step);
* the explicit forward/backward kernel schedule below. There is no autograd
  on the hot path: each launch is a libgptb200 kernel on the current stream.

Forward, per block (activations bf16, rows = local tokens):
  rms_norm -> GEMM(+bias, RoPE on the q/k columns) -> qkv -> attention ->
  GEMM(+bias, x branch multiplier, + residual) -> rms_norm -> GEMM(+bias, GELU,
  saving gelu'(u)) -> GEMM(+bias, x multiplier, + residual); then the final
  rms_norm and the fused linear cross-entropy (no logits in HBM).
Backward mirrors it with dgrad GEMMs (dGELU fused), weight-gradient GEMMs that
accumulate into the fp32 gradient buffer with split-K atomics, bias-gradient
column sums, RMSNorm backward fused with the residual-gradient add, and the
attention backward writing dq/dk/dv straight into the packed qkv gradient.
With data parallelism each block's gradient slice is all-reduced on NCCL as
soon as its backward has been enqueued, overlapping the remaining backward.
"""

from __future__ import annotations

import ctypes
import dataclasses
from typing import Iterable

import numpy as np
import torch

from . import _lib, ops
from .config import (
    Config,
    decay_for_name,
    effective_adam_betas,
    horizon_scales,
    tensor_multipliers,
)

BLOCK_FIELDS = (
    "ln1_scale", "qkv_w", "qkv_b", "attn_w", "attn_b",
    "ln2_scale", "mlp_up_w", "mlp_up_b", "mlp_down_w", "mlp_down_b",
)
# A routed block (recipes/reference_moe/train.py:905-931), in its init order.
MOE_BLOCK_FIELDS = (
    "ln1_scale", "qkv_w", "qkv_b", "attn_w", "attn_b", "ln2_scale",
    "router_w", "expert_up_w", "expert_up_b", "expert_down_w", "expert_down_b",
)
ALIGN = 64


def block_fields(config: Config) -> tuple[str, ...]:
    return MOE_BLOCK_FIELDS if config.experts else BLOCK_FIELDS


def block_shapes(config: Config) -> dict[str, tuple[int, ...]]:
    d, h = config.d_model, config.hidden
    E, eh = config.experts, config.expert_mult * config.d_model
    return {
        "ln1_scale": (d,),
        "qkv_w": (d, 3 * d),
        "qkv_b": (3 * d,),
        "attn_w": (d, d),
        "attn_b": (d,),
        "ln2_scale": (d,),
        "mlp_up_w": (d, h),
        "mlp_up_b": (h,),
        "mlp_down_w": (h, d),
        "mlp_down_b": (d,),
        "router_w": (d, E),
        "expert_up_w": (E, d, eh),
        "expert_up_b": (E, eh),
        "expert_down_w": (E, eh, d),
        "expert_down_b": (E, d),
    }


@dataclasses.dataclass(frozen=True)
class Slot:
    name: str          # "blocks/3/qkv_w", "token_embedding", ...
    leaf: str          # "qkv_w"
    block: int         # -1 outside the blocks
    shape: tuple[int, ...]
    offset: int

    @property
    def size(self) -> int:
        return int(np.prod(self.shape))


class ParamLayout:
    """Flat layout: blocks 0..L-1, then final_ln_scale, token/output embedding."""

    def __init__(self, config: Config):
        self.config = config
        slots: list[Slot] = []
        off = 0

        def add(name, leaf, block, shape):
            nonlocal off
            slots.append(Slot(name, leaf, block, tuple(shape), off))
            off += int(np.prod(shape))
            off = (off + ALIGN - 1) // ALIGN * ALIGN

        shapes = block_shapes(config)
        self.block_ranges: list[tuple[int, int]] = []
        for b in range(config.layers):
            start = off
            for leaf in block_fields(config):
                add(f"blocks/{b}/{leaf}", leaf, b, shapes[leaf])
            self.block_ranges.append((start, off))
        tail = off
        add("final_ln_scale", "final_ln_scale", -1, (config.d_model,))
        add("token_embedding", "token_embedding", -1, (config.vocab_size, config.d_model))
        if not config.tied:
            add("output_embedding", "output_embedding", -1, (config.vocab_size, config.d_model))
        self.tail_range = (tail, off)
        self.slots = slots
        self.by_name = {s.name: s for s in slots}
        self.numel = off

    def parameter_count(self) -> int:
        return sum(s.size for s in self.slots)


def init_params(config: Config, seed: int) -> dict[str, np.ndarray]:
    """Initial parameters with the reference's draw order (train.py:865-901).

    numpy PCG64 `default_rng(seed)`; per block qkv_w, attn_w, mlp_up_w,
    mlp_down_w ~ N(0, sigma_h) (rig/nn.py:20-23: float32 standard normal times
    float32 scale), biases 0, scales 1; then token_embedding ~ N(0, init_std),
    then output_embedding ~ N(0, init_std / m_N) when untied.
    """

    rng = np.random.default_rng(seed)
    hidden_scale = (
        config.init_std / np.sqrt(config.width_multiplier)
        if config.parameterization == "completep_fixed_tpp_v1"
        else 0.02
    )

    def normal(shape, scale):
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)

    shapes = block_shapes(config)
    out: dict[str, np.ndarray] = {}
    for b in range(config.layers):
        for leaf in block_fields(config):
            shape = shapes[leaf]
            if leaf.endswith("_scale"):
                value = np.ones(shape, dtype=np.float32)
            elif leaf.endswith("_b"):
                value = np.zeros(shape, dtype=np.float32)
            else:
                value = normal(shape, hidden_scale)
            out[f"blocks/{b}/{leaf}"] = value
    out["token_embedding"] = normal((config.vocab_size, config.d_model), config.init_std)
    out["final_ln_scale"] = np.ones((config.d_model,), dtype=np.float32)
    if not config.tied:
        out["output_embedding"] = normal(
            (config.vocab_size, config.d_model), config.init_std / config.width_multiplier
        )
    return out


class _Block:
    """Views of one block's parameters, bf16 mirrors and gradients."""

    def __init__(self, trainer: "GPTTrainer", b: int):
        for leaf in block_fields(trainer.config):
            name = f"blocks/{b}/{leaf}"
            setattr(self, leaf, trainer.param_view(name, bf16=True))
            setattr(self, "g_" + leaf, trainer.grad_view(name))
        if trainer.config.experts:  # the router computes in fp32 (train.py:1258-1263)
            self.router_w32 = trainer.param_view(f"blocks/{b}/router_w")


# Parts the tail gradient bucket is all-reduced and updated in (see backward).
TAIL_PARTS = 4


def tail_parts(start: int, end: int, parts: int = TAIL_PARTS) -> list[tuple[int, int]]:
    """[start, end) cut into `parts` contiguous ranges whose inner boundaries
    are start + multiples of 1024 elements (one range if it is too short)."""

    if end - start < parts * 4096:
        return [(start, end)]
    cuts = [start + (end - start) * i // parts // 1024 * 1024 for i in range(parts)] + [end]
    return [(cuts[i], cuts[i + 1]) for i in range(parts)]


class GPTTrainer:
    """Holds the model state on one GPU and runs the training step."""

    def __init__(
        self,
        config: Config,
        local_batch: int,
        device: torch.device | str = "cuda",
        *,
        process_group=None,
        world_size: int = 1,
        history_steps: int | None = None,
        deterministic: bool = True,
        overlap_optimizer: bool | None = None,
    ):
        if config.dtype_name != "bfloat16":
            raise ValueError("the B200 step computes in bfloat16")
        if config.head_dim != 64:
            raise ValueError("the attention kernels need head_dim 64")
        self.config = config
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("GPTTrainer needs a CUDA device (there is no CPU path)")
        self.B = int(local_batch)
        self.T = config.seq_len
        self.N = self.B * self.T
        self.world_size = int(world_size)
        self.pg = process_group
        # Bit-reproducible gradients: weight gradients split over K are summed
        # from per-split slabs in a fixed order (EPI_F32_SPLITK) instead of with
        # fp32 atomics. The other reductions of the step are always ordered.
        self.deterministic = bool(deterministic)
        self.wgrad_kind = _lib.EPI_F32_SPLITK if deterministic else _lib.EPI_F32_ATOMIC
        # Without gradient clipping the AdamW update of a bucket does not wait
        # for the global norm, so with data parallelism each bucket is updated
        # on a side stream as soon as its all-reduce completes, overlapping the
        # rest of the backward pass. On one GPU the update only competes with
        # the backward for HBM bandwidth (measured: no gain), so it stays off.
        if overlap_optimizer is None:
            overlap_optimizer = config.grad_clip <= 0.0 and self.world_size > 1
        if overlap_optimizer and config.grad_clip > 0.0:
            raise ValueError("overlap_optimizer needs grad_clip <= 0 (clipping needs the global norm)")
        self.overlap_optimizer = bool(overlap_optimizer)
        self.layout = ParamLayout(config)
        if (config.declared_parameters is not None
                and self.layout.parameter_count() != config.declared_parameters):
            # recipes/reference/train.py:1672-1678
            raise ValueError(f"tier {config.tier} declares {config.declared_parameters:,} "
                             f"parameters, but initialized {self.layout.parameter_count():,}")
        dev = self.device
        n = self.layout.numel
        self.params = torch.zeros(n, dtype=torch.float32, device=dev)
        self.grads = torch.zeros(n, dtype=torch.float32, device=dev)
        self.m = torch.zeros(n, dtype=torch.float32, device=dev)
        self.v = torch.zeros(n, dtype=torch.float32, device=dev)
        self.params_bf16 = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        self.step_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        self.history = torch.zeros(max(1, history_steps or config.steps), 3,
                                   dtype=torch.float32, device=dev)
        self.blocks = [_Block(self, b) for b in range(config.layers)]
        self.final_scale = self.param_view("final_ln_scale", bf16=True)
        self.g_final_scale = self.grad_view("final_ln_scale")
        self.tok_emb = self.param_view("token_embedding", bf16=True)
        self.g_tok_emb = self.grad_view("token_embedding")
        if config.tied:
            self.out_emb, self.g_out_emb = self.tok_emb, self.g_tok_emb
        else:
            self.out_emb = self.param_view("output_embedding", bf16=True)
            self.g_out_emb = self.grad_view("output_embedding")
        self._alloc_activations()
        self._build_optimizer()
        self.opt_stream = torch.cuda.Stream(self.device) if self.overlap_optimizer else None
        self.rope = ops.rope_tables(self.T, config.head_dim, dev)

    # ------------------------------------------------------------ state views
    def param_view(self, name: str, bf16: bool = False) -> torch.Tensor:
        s = self.layout.by_name[name]
        buf = self.params_bf16 if bf16 else self.params
        return buf[s.offset : s.offset + s.size].view(s.shape)

    def grad_view(self, name: str) -> torch.Tensor:
        s = self.layout.by_name[name]
        return self.grads[s.offset : s.offset + s.size].view(s.shape)

    def load_params(self, values: dict[str, np.ndarray]) -> None:
        for s in self.layout.slots:
            arr = np.asarray(values[s.name], dtype=np.float32).reshape(s.shape)
            self.params[s.offset : s.offset + s.size].copy_(
                torch.from_numpy(np.ascontiguousarray(arr)).reshape(-1))
        ops.cast_bf16(self.params, self.params_bf16)
        self.m.zero_()
        self.v.zero_()
        self.step_dev.zero_()

    def export(self, buf: torch.Tensor | None = None) -> dict[str, np.ndarray]:
        buf = self.params if buf is None else buf
        host = buf.detach().float().cpu().numpy()
        return {s.name: host[s.offset : s.offset + s.size].reshape(s.shape).copy()
                for s in self.layout.slots}

    # ------------------------------------------------------------ buffers
    def _alloc_activations(self) -> None:
        c, dev, N = self.config, self.device, self.N
        d, h, L = c.d_model, c.hidden, c.layers
        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.x = [torch.empty(N, d, **bf) for _ in range(L + 1)]
        self.ln1 = [torch.empty(N, d, **bf) for _ in range(L)]
        self.rstd1 = [torch.empty(N, **f32) for _ in range(L)]
        self.qkv = [torch.empty(N, 3 * d, **bf) for _ in range(L)]
        self.att = [torch.empty(N, d, **bf) for _ in range(L)]
        self.lse = [torch.empty(self.B, c.heads, self.T, **f32) for _ in range(L)]
        self.xm = [torch.empty(N, d, **bf) for _ in range(L)]
        self.ln2 = [torch.empty(N, d, **bf) for _ in range(L)]
        self.rstd2 = [torch.empty(N, **f32) for _ in range(L)]
        if c.experts:
            self._alloc_moe()
        else:
            self.gelu_grad = [torch.empty(N, h, **bf) for _ in range(L)]  # gelu'(u), saved
            self.g = [torch.empty(N, h, **bf) for _ in range(L)]
        self.lnf = torch.empty(N, d, **bf)
        self.rstdf = torch.empty(N, **f32)
        self.losses = torch.empty(N, **f32)
        self.segments = (torch.empty(self.B, self.T, dtype=torch.int32, device=dev)
                         if c.document_masking else None)
        self.lse_ce = torch.empty(N, **f32)
        self.loss = torch.zeros(1, **f32)
        self.cot = torch.full((N,), 1.0 / (N * self.world_size), **f32)
        # backward scratch
        self.dx = torch.empty(N, d, **bf)
        self.dln = torch.empty(N, d, **bf)
        self.du = None if c.experts else torch.empty(N, h, **bf)
        self.datt = torch.empty(N, d, **bf)
        self.dqkv = torch.empty(N, 3 * d, **bf)
        self.attn_ws = ops.attention_workspace(self.B, c.heads, self.T, dev)
        self.lce_fwd_ws = ops.lce_fwd_workspace(N, c.vocab_size, dev)
        self.lce_bwd_ws = ops.lce_bwd_workspace(N, c.vocab_size, dev)
        self.tokens = torch.empty(self.B, self.T, dtype=torch.int32, device=dev)
        self.targets = torch.empty(self.B, self.T, dtype=torch.int32, device=dev)
        # One scratch buffer shared by the backward's ordered reductions (they
        # run one after another on the step's stream).
        wgrad_shapes = [(d, 3 * d), (d, d)] + ([] if c.experts else [(d, h), (h, d)])
        need = [ops.rms_norm_bwd_workspace_size(N, d),
                ops.embedding_bwd_workspace_size(N, d, c.vocab_size)]
        need += [ops.colsum_workspace_size(N, w) for w in (3 * d, h)]
        self.scratch = torch.empty(max(need), dtype=torch.uint8, device=dev)
        # per-split partial slabs of the ordered split-K weight gradients
        self.splitk_ws = ops.splitk_workspace(
            max(ops.gemm_workspace_size(m, n, N, self.wgrad_kind) for m, n in wgrad_shapes), dev)

    def _alloc_moe(self) -> None:
        """Per-layer routed buffers (kept for the backward) and shared scratch."""

        c, dev, N, L = self.config, self.device, self.N, self.config.layers
        d, E, k, eh = c.d_model, c.experts, c.expert_top_k, c.expert_mult * c.d_model
        R = ops.moe_rows(N, k, E)
        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.moe_R = R
        self.m_logits = [torch.empty(N, E, **f32) for _ in range(L)]
        self.m_chosen = [torch.empty(N, k, **i32) for _ in range(L)]
        self.m_gate = [torch.empty(N, k, **f32) for _ in range(L)]
        self.m_pos = [torch.empty(N, k, **i32) for _ in range(L)]
        self.m_src = [torch.empty(R, **i32) for _ in range(L)]
        self.m_seg = [torch.zeros(E, 2, **i32) for _ in range(L)]
        self.m_total = [torch.zeros(1, **i32) for _ in range(L)]
        self.m_grouped = [torch.empty(R, d, **bf) for _ in range(L)]
        self.m_hidden = [torch.empty(R, eh, **bf) for _ in range(L)]
        self.m_gelu = [torch.empty(R, eh, **bf) for _ in range(L)]
        self.m_out = [torch.empty(R, d, **bf) for _ in range(L)]
        width = 2 * E + 3
        self.m_stats = torch.zeros(L, width, **f32)
        self.m_bal = torch.zeros(L, E, **f32)
        self.m_dout = torch.empty(R, d, **bf)
        self.m_dhidden = torch.empty(R, eh, **bf)
        self.m_dgrouped = torch.empty(R, d, **bf)
        self.m_dgate = torch.empty(N, k, **f32)
        self.m_ws = ops.moe_dispatch_workspace(N, k, E, dev)
        self.router_history = torch.zeros(self.history.shape[0], 6 + L * (3 + E), **f32)

    def _moe_forward(self, l: int, blk) -> None:
        """Routed MLP of block l (recipes/reference_moe/train.py:1230-1311):
        route, dispatch into padded expert segments, per-expert up (bias + GELU)
        and down GEMMs over the device-side segment bounds, gate-weighted combine
        with the residual branch."""

        c = self.config
        E, eh, d = c.experts, c.expert_mult * c.d_model, c.d_model
        ops.moe_route(self.ln2[l], blk.router_w32, self.m_logits[l], self.m_chosen[l],
                      self.m_gate[l], self.m_stats[l])
        ops.moe_dispatch(self.m_chosen[l], self.ln2[l], E, self.m_seg[l], self.m_total[l],
                         self.m_pos[l], self.m_src[l], self.m_grouped[l], self.m_ws)
        R = self.moe_R
        for e in range(E):
            rr = self.m_seg[l][e]
            ops.gemm(self.m_grouped[l], blk.expert_up_w[e], self.m_hidden[l], b_mn_major=True,
                     m=R, n=eh, k=d, kind=_lib.EPI_BIAS_GELU, bias=blk.expert_up_b[e],
                     aux=self.m_gelu[l], row_range=rr, range_dim=1)
        for e in range(E):
            rr = self.m_seg[l][e]
            ops.gemm(self.m_hidden[l], blk.expert_down_w[e], self.m_out[l], b_mn_major=True,
                     m=R, n=d, k=eh, bias=blk.expert_down_b[e], row_range=rr, range_dim=1)
        ops.moe_combine(self.m_out[l], self.m_pos[l], self.m_gate[l], self.xm[l],
                        c.branch_scale, self.x[l + 1])

    def _moe_backward(self, l: int, blk, dx: torch.Tensor) -> None:
        """Backward of _moe_forward: dx (gradient of the block output) in,
        self.dln (gradient of the routed MLP's input) out; expert, router and
        bias gradients accumulated."""

        c = self.config
        E, eh, d, R = c.experts, c.expert_mult * c.d_model, c.d_model, self.moe_R
        ops.moe_combine_bwd(dx, c.branch_scale, self.m_out[l], self.m_pos[l], self.m_gate[l],
                            self.m_src[l], self.m_total[l], self.m_dout, self.m_dgate)
        for e in range(E):
            rr = self.m_seg[l][e]
            # d_hidden = dGELU(d_out . W_down[e]^T)
            ops.gemm(self.m_dout, blk.expert_down_w[e], self.m_dhidden, m=R, n=eh, k=d,
                     kind=_lib.EPI_DGELU, aux=self.m_gelu[l], row_range=rr, range_dim=1)
            # dW_down[e] += hidden^T d_out over the expert's rows
            ops.gemm(self.m_hidden[l], self.m_dout, blk.g_expert_down_w[e], a_mn_major=True,
                     b_mn_major=True, m=eh, n=d, k=R, kind=_lib.EPI_F32_ATOMIC, row_range=rr,
                     range_dim=2)
        ops.moe_segment_colsum(self.m_dout, self.m_seg[l], E, blk.g_expert_down_b)
        for e in range(E):
            rr = self.m_seg[l][e]
            ops.gemm(self.m_dhidden, blk.expert_up_w[e], self.m_dgrouped, m=R, n=d, k=eh,
                     row_range=rr, range_dim=1)
            ops.gemm(self.m_grouped[l], self.m_dhidden, blk.g_expert_up_w[e], a_mn_major=True,
                     b_mn_major=True, m=d, n=eh, k=R, kind=_lib.EPI_F32_ATOMIC, row_range=rr,
                     range_dim=2)
        ops.moe_segment_colsum(self.m_dhidden, self.m_seg[l], E, blk.g_expert_up_b)
        ops.moe_route_bwd(self.ln2[l], blk.router_w32, self.m_logits[l], self.m_chosen[l],
                          self.m_gate[l], self.m_dgate, self.m_bal[l], self.m_dgrouped,
                          self.m_pos[l], blk.g_router_w, self.dln)

    def _moe_finalize(self) -> None:
        """Balance loss and router statistics over all ranks (the reference
        pmeans them, train.py:1302-1305), added to the loss; backward
        coefficients of the router probabilities."""

        c = self.config
        if self.world_size > 1:
            import torch.distributed as dist

            dist.all_reduce(self.m_stats, op=dist.ReduceOp.SUM, group=self.pg)
        ops.moe_finalize(self.m_stats, c.layers, c.experts, self.N * self.world_size,
                         c.expert_top_k, c.router_aux_coefficient,
                         1.0 / (self.N * self.world_size), self.m_bal, self.loss,
                         self.router_history, self.step_dev)

    def _build_optimizer(self) -> None:
        c = self.config
        groups = []
        for s in self.layout.slots:
            lr_m, eps_m, wd_m = tensor_multipliers(s.leaf, s.block >= 0, c)
            groups.append(_lib.TensorGroup(
                offset=s.offset, size=s.size, lr_mult=lr_m, eps_mult=eps_m, wd_mult=wd_m,
                decay=int(decay_for_name(s.leaf))))
        arr = (_lib.TensorGroup * len(groups))(*groups)
        raw = bytes(arr)
        self.groups_dev = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.device)
        self.n_groups = len(groups)
        b1, b2 = effective_adam_betas(c)
        lr_h, eps_h, wd_h = horizon_scales(c)
        self.adam_cfg = _lib.AdamWConfig(
            learning_rate=c.learning_rate, horizon_lr_scale=lr_h, min_lr_ratio=c.min_lr_ratio,
            warmup_steps=c.warmup_steps, total_steps=c.steps, beta1=b1, beta2=b2,
            eps=c.adam_epsilon, eps_horizon_scale=eps_h, weight_decay=c.weight_decay,
            wd_horizon_scale=wd_h, grad_clip=c.grad_clip, grad_scale=1.0)
        self.adam_ws = ops.adamw_workspace(self.layout.numel, self.device)

    # ------------------------------------------------------------ views
    def _qkv_views(self, buf: torch.Tensor):
        c = self.config
        t5 = buf.view(self.B, self.T, 3, c.heads, c.head_dim)
        return t5[:, :, 0], t5[:, :, 1], t5[:, :, 2]

    def _bthd(self, buf: torch.Tensor):
        c = self.config
        return buf.view(self.B, self.T, c.heads, c.head_dim)

    # ------------------------------------------------------------ step
    def set_batch(self, x: torch.Tensor, y: torch.Tensor) -> None:
        """Copies a [B, T] int32 batch (host pinned or device) into the step's buffers."""

        self.tokens.copy_(x, non_blocking=True)
        self.targets.copy_(y, non_blocking=True)

    def forward(self) -> torch.Tensor:
        c = self.config
        d, h, N = c.d_model, c.hidden, self.N
        a = c.branch_scale
        ops.embedding_fwd(self.tokens.view(-1), self.tok_emb, self.x[0])
        if c.experts:
            self.m_stats.zero_()
        if self.segments is not None:  # document masking (train.py:1127-1131)
            ops.document_segments(self.tokens.view(self.B, self.T), c.document_boundary_token,
                                  self.segments)
        for l, blk in enumerate(self.blocks):
            ops.rms_norm_fwd(self.x[l], blk.ln1_scale, self.ln1[l], self.rstd1[l])
            # QKV projection with bias and RoPE on the q/k columns in the epilogue
            ops.matmul(self.ln1[l], blk.qkv_w, bias=blk.qkv_b, out=self.qkv[l],
                       kind=_lib.EPI_BIAS_ROPE, rope=self.rope, rope_cols=2 * d)
            q, k, v = self._qkv_views(self.qkv[l])
            ops.attention_fwd(q, k, v, self._bthd(self.att[l]), self.lse[l], scale=c.softmax_scale,
                              layout="bthd", segment_ids=self.segments)
            ops.matmul(self.att[l], blk.attn_w, bias=blk.attn_b, alpha=a, residual=self.x[l],
                       out=self.xm[l])
            ops.rms_norm_fwd(self.xm[l], blk.ln2_scale, self.ln2[l], self.rstd2[l])
            if c.experts:
                self._moe_forward(l, blk)
                continue
            ops.matmul(self.ln2[l], blk.mlp_up_w, bias=blk.mlp_up_b, kind=_lib.EPI_BIAS_GELU,
                       aux=self.gelu_grad[l], out=self.g[l])
            ops.matmul(self.g[l], blk.mlp_down_w, bias=blk.mlp_down_b, alpha=a,
                       residual=self.xm[l], out=self.x[l + 1])
        ops.rms_norm_fwd(self.x[c.layers], self.final_scale, self.lnf, self.rstdf)
        ops.lce_fwd(self.lnf, self.out_emb, self.targets.view(-1), c.semantic_vocab_size,
                    self.losses, self.lse_ce, self.loss, workspace=self.lce_fwd_ws)
        if c.experts:
            self._moe_finalize()
        return self.loss

    def _wgrad(self, act: torch.Tensor, dy: torch.Tensor, gview: torch.Tensor, alpha: float):
        """gview[K_in, N_out] += alpha * act^T dy (fp32; K split over CTAs, the
        splits summed in a fixed order unless the trainer runs with atomics)."""

        m, n = act.shape[1], dy.shape[1]
        ops.gemm(act, dy, gview, a_mn_major=True, b_mn_major=True, m=m, n=n, k=self.N,
                 kind=self.wgrad_kind, alpha=alpha, workspace=self.splitk_ws)

    def _dgrad(self, dy: torch.Tensor, w: torch.Tensor, out: torch.Tensor, **kw):
        """out[N, in] = epilogue(dy[N, out] @ w[in, out]^T)."""

        ops.gemm(dy, w, out, m=self.N, n=w.shape[0], k=w.shape[1], **kw)

    def backward(self, reduce_hook=None) -> None:
        c = self.config
        a = c.branch_scale
        self.grads.zero_()
        ops.lce_bwd(self.lnf, self.out_emb, self.targets.view(-1), self.lse_ce, self.cot,
                    c.semantic_vocab_size, self.dln, self.g_out_emb, workspace=self.lce_bwd_ws)
        # The residual-stream gradient each RMSNorm backward produces is also the
        # gradient of the bias of the branch below it; its column sums are fused.
        # (a routed MLP's biases are per expert: their sums come from moe_segment_colsum)
        mlp_bias = (lambda l: None) if c.experts else (lambda l: self.blocks[l].g_mlp_down_b)
        ops.rms_norm_bwd(self.x[c.layers], self.final_scale, self.rstdf, self.dln, None, self.dx,
                         self.g_final_scale, mlp_bias(c.layers - 1), a, workspace=self.scratch)
        dx = self.dx
        for l in reversed(range(c.layers)):
            blk = self.blocks[l]
            if c.experts:
                self._moe_backward(l, blk, dx)
            else:
                # MLP: x[l+1] = xm + a * (gelu(ln2 Wu + bu) Wd + bd)
                self._dgrad(dx, blk.mlp_down_w, self.du, kind=_lib.EPI_DGELU, alpha=a,
                            aux=self.gelu_grad[l])
                self._wgrad(self.g[l], dx, blk.g_mlp_down_w, a)
                self._wgrad(self.ln2[l], self.du, blk.g_mlp_up_w, 1.0)
                ops.colsum(self.du, blk.g_mlp_up_b, 1.0, workspace=self.scratch)
                self._dgrad(self.du, blk.mlp_up_w, self.dln)
            ops.rms_norm_bwd(self.xm[l], blk.ln2_scale, self.rstd2[l], self.dln, dx, dx,
                             blk.g_ln2_scale, blk.g_attn_b, a, workspace=self.scratch)
            # attention: xm = x + a * (att Wo + bo)
            self._dgrad(dx, blk.attn_w, self.datt, alpha=a)
            self._wgrad(self.att[l], dx, blk.g_attn_w, a)
            q, k, v = self._qkv_views(self.qkv[l])
            dq, dk, dv = self._qkv_views(self.dqkv)
            ops.attention_bwd(q, k, v, self._bthd(self.att[l]), self._bthd(self.datt), self.lse[l],
                              dq, dk, dv, scale=c.softmax_scale, layout="bthd", rope=self.rope,
                              workspace=self.attn_ws, segment_ids=self.segments)
            self._wgrad(self.ln1[l], self.dqkv, blk.g_qkv_w, 1.0)
            ops.colsum(self.dqkv, blk.g_qkv_b, 1.0, workspace=self.scratch)
            self._dgrad(self.dqkv, blk.qkv_w, self.dln)
            below = mlp_bias(l - 1) if l > 0 else None
            ops.rms_norm_bwd(self.x[l], blk.ln1_scale, self.rstd1[l], self.dln, dx, dx,
                             blk.g_ln1_scale, below, a, workspace=self.scratch)
            if reduce_hook is not None:
                reduce_hook(*self.layout.block_ranges[l])
        ops.embedding_bwd(self.tokens.view(-1), dx, self.g_tok_emb, workspace=self.scratch)
        if reduce_hook is not None:
            # The tail bucket (final norm + embeddings, about a third of the
            # parameters) is final only after the last backward kernel, so it
            # goes in parts: each part's update overlaps the next part's
            # all-reduce instead of waiting for the whole bucket.
            for part in tail_parts(*self.layout.tail_range):
                reduce_hook(*part)

    def optimizer_step(self) -> None:
        ops.adamw_step(self.params, self.m, self.v, self.grads, self.groups_dev, self.n_groups,
                       self.adam_cfg, self.step_dev, self.loss, self.history, self.params_bf16,
                       self.adam_ws)

    def capture(self) -> None:
        """Records one whole step (forward, backward, AdamW) as a CUDA graph.

        The step is static-shaped and allocates nothing, so after one eager
        warm-up step (which also sets every kernel's shared-memory attribute)
        the graph replays the identical launch sequence; the batch is read from
        `self.tokens` / `self.targets` and the step counter lives on the device.
        With data parallelism the bucketed NCCL all-reduces and the optimizer
        stream's per-bucket updates are recorded with the kernels (every rank
        records the same sequence, so replays stay matched across ranks).
        Release the graph (`self.graph = None`) before the process group is
        destroyed.
        """

        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        graph = torch.cuda.CUDAGraph()
        before = ops.launch_count()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                self._eager_step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.graph = graph
        self.graph_launches = ops.launch_count() - before

    def eval_step(self, x: torch.Tensor, y: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        """recipes/reference/train.py:1494-1525: [sum(loss * mask), sum(mask)]
        over the global batch (fp32, on the device; summed over data-parallel
        ranks). The forward runs through the same kernels as the training step
        (tiled cross-entropy losses, never materialized logits); parameters and
        optimizer state are untouched."""

        if tuple(x.shape) != (self.B, self.T) or tuple(mask.shape) != (self.B, self.T):
            raise ValueError(f"eval batch must be [{self.B}, {self.T}]; got x {tuple(x.shape)}, "
                             f"mask {tuple(mask.shape)}")
        self.set_batch(x, y)
        self.forward()
        m = mask.to(device=self.device, dtype=torch.float32)
        out = ops.masked_loss_sum(self.losses, m.reshape(-1))
        if self.world_size > 1:
            import torch.distributed as dist

            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.pg)
        return out

    def checked_metrics(self, step: int) -> dict[str, float]:
        """Synchronizes, then checks and returns step `step`'s history row.

        Raises GptB200Error when a kernel set a device-side error flag (a wait
        that ran out, a token id outside the vocabulary, a non-finite gradient
        norm), and FloatingPointError when the loss or gradient norm is not
        finite or the learning rate is negative, as the reference's logging
        path does through finite_metric (rig/mesh.py:214-223). Call it on log
        steps; it costs one device synchronisation."""

        from .mesh import finite_metric

        flags = _lib.load().gptb200_device_error_flags(1)
        if flags:
            raise _lib.GptB200Error(f"device-side error flags 0x{flags:x} after step {step}")
        if not 1 <= step <= self.history.shape[0]:
            raise ValueError(f"step {step} is outside the history (1..{self.history.shape[0]})")
        loss, lr, gn = (float(v) for v in self.history[step - 1].tolist())
        return {"train_loss": finite_metric("train_loss", loss),
                "learning_rate": finite_metric("learning_rate", lr),
                "grad_norm": finite_metric("grad_norm", gn)}

    # ------------------------------------------------------------ artifacts
    def training_history(self, final_step: int) -> np.ndarray:
        """Rows 1..final_step of the on-device (loss, lr, grad_norm) history,
        followed for a routed model by that step's router statistics row
        (the column order of `runlog.training_log_columns`)."""

        rows = self.history[:final_step]
        if self.config.experts:
            rows = torch.cat((rows, self.router_history[:final_step]), dim=1)
        return rows.detach().cpu().numpy().astype(np.float32)

    def save_checkpoint(self, output_dir, seed: int) -> None:
        """checkpoint.npz in the rig's layout (fp32 master parameters)."""

        from . import runlog

        tree = runlog.nest_params(self.export(), self.config.layers)
        runlog.save_checkpoint(output_dir, tree, runlog.checkpoint_metadata(self.config, seed))

    def write_training_log(self, output_dir, final_step: int, flops_per_token: float | None = None):
        """training.riglog: one record per optimizer step 1..final_step."""

        from . import runlog

        c = self.config
        columns = runlog.training_log_columns(c.layers if c.experts else 0, c.experts)
        runlog.write_training_log(output_dir, self.training_history(final_step),
                                  tokens_per_step=c.batch_size * self.T,
                                  final_step=final_step, flops_per_token=flops_per_token,
                                  columns=columns)

    graph: "torch.cuda.CUDAGraph | None" = None
    graph_launches: int = 0  # libgptb200 kernels inside one replay

    def train_step(self, x: torch.Tensor | None = None, y: torch.Tensor | None = None) -> None:
        """One full step: forward, backward, (all-reduce), AdamW. Asynchronous."""

        if x is not None:
            self.set_batch(x, y)
        if self.graph is not None:
            self.graph.replay()
            return
        self._eager_step()

    def _eager_step(self) -> None:
        self.forward()
        if self.overlap_optimizer:
            self._overlapped_backward_and_update()
            return
        if self.world_size > 1:
            from .mesh import GradientReducer

            reducer = GradientReducer(self.grads, self.pg)
            self.backward(reduce_hook=reducer.launch)
            reducer.finish(self.loss)
        else:
            self.backward()
        self.optimizer_step()

    def _overlapped_backward_and_update(self) -> None:
        """Backward with each bucket (a block's parameters, then the final norm
        and embeddings) updated on the optimizer stream once its gradient is
        final: right after its all-reduce with data parallelism, right after
        its backward kernels on one GPU. The compute stream waits for the
        optimizer stream before the next step reads the new parameters."""

        compute = torch.cuda.current_stream(self.device)
        opt = self.opt_stream
        ops.adamw_begin(self.adam_cfg, self.step_dev, self.adam_ws)
        opt.wait_stream(compute)  # the step's scalars
        slots = []

        def update(start: int, end: int, work=None) -> None:
            if work is None:
                opt.wait_stream(compute)
            with torch.cuda.stream(opt):
                if work is not None:
                    work.wait()
                ops.adamw_update_range(self.params, self.m, self.v, self.grads, start, end,
                                       self.groups_dev, self.n_groups, self.adam_cfg, len(slots),
                                       self.params_bf16, self.adam_ws)
            slots.append((start, end))

        if self.world_size > 1:
            from .mesh import GradientReducer

            reducer = GradientReducer(self.grads, self.pg, on_reduced=update)
            self.backward(reduce_hook=reducer.launch)
            reducer.finish(self.loss)
        else:
            self.backward(reduce_hook=update)
        opt.wait_stream(compute)  # the (all-reduced) loss for the history row
        with torch.cuda.stream(opt):
            ops.adamw_end(len(slots), self.adam_cfg, self.step_dev, self.loss, self.history,
                          self.adam_ws)
        compute.wait_stream(opt)
