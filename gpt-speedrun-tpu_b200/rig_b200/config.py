"""Run configuration of the training step, resolved like the reference recipe.

Mirrors the subset of recipes/reference/train.py that decides the numbers the
step uses: the typed YAML document (schema 6, :177-562), `resolve_config`
(:688-862: steps, warmup, batch/data multipliers), the CompleteP multipliers
(`optimizer_hyperparameter_trees`, :1274-1333), `effective_adam_betas`
(:1336-1345), `weight_decay_mask` (:1252-1271) and `learning_rate`
(:1219-1236). Field names follow the reference `Config` dataclass.
"""

from __future__ import annotations

import dataclasses
import math
import pathlib
from typing import Any, Mapping

import yaml

CONFIG_DIR = pathlib.Path(__file__).resolve().parent.parent / "configs"


@dataclasses.dataclass(frozen=True)
class Config:
    steps: int
    batch_size: int
    seq_len: int
    layers: int
    heads: int
    d_model: int
    mlp_mult: int
    vocab_size: int
    semantic_vocab_size: int
    parameterization: str
    base_width: int
    base_depth: int
    depth_alpha: float
    init_std: float
    attention_scale: str
    embeddings: str
    data_multiplier: float
    batch_multiplier: float
    learning_rate: float
    min_lr_ratio: float
    warmup_steps: int
    weight_decay: float
    adam_epsilon: float
    beta1: float
    beta2: float
    grad_clip: float
    vocab_tile_size: int
    dtype_name: str
    sampling: str = "shuffled_epochs"
    tier: str = ""
    normalization: str = "rms_norm"
    position_encoding: str = "rope_base_10000"
    mlp_activation: str = "gelu"
    document_masking: bool = False        # the context preset's document-attention policy
    document_boundary_token: int = 50256  # recipes/reference/train.py:234-235
    # routed MLP (recipes/reference_moe/train.py:242-245); experts = 0: dense MLP
    experts: int = 0
    expert_top_k: int = 2
    expert_mult: int = 2
    router_aux_coefficient: float = 0.01
    # fixed tokens-per-parameter horizon (train.py:745-751): the tier's declared
    # parameter denominator and the requested TPP; None for a fixed-step run
    declared_parameters: int | None = None
    target_tokens_per_parameter: float | None = None

    @property
    def width_multiplier(self) -> float:
        return self.d_model / float(self.base_width)

    @property
    def depth_multiplier(self) -> float:
        return self.layers / float(self.base_depth)

    @property
    def tokens_per_parameter(self) -> float | None:
        """Achieved full-schedule TPP after rounding to whole steps (train.py:255-266)."""

        if self.declared_parameters is None:
            return None
        return self.steps * self.batch_size * self.seq_len / float(self.declared_parameters)

    @property
    def head_dim(self) -> int:
        return self.d_model // self.heads

    @property
    def hidden(self) -> int:
        return self.mlp_mult * self.d_model

    @property
    def branch_scale(self) -> float:
        """Residual-branch multiplier m_L^-alpha (train.py:1164,1172)."""

        return self.depth_multiplier ** (-self.depth_alpha)

    @property
    def softmax_scale(self) -> float:
        """`attention_softmax_scale` (rig/attention.py:55-62)."""

        if self.attention_scale == "inverse_head_dim":
            return 1.0 / float(self.head_dim)
        if self.attention_scale == "inverse_sqrt_head_dim":
            return self.head_dim ** -0.5
        raise ValueError(f"unsupported attention scale {self.attention_scale!r}")

    @property
    def tied(self) -> bool:
        return self.embeddings == "tied"

    def replace(self, **kw: Any) -> "Config":
        return dataclasses.replace(self, **kw)


def _require(mapping: Mapping[str, Any], key: str, where: str) -> Any:
    if key not in mapping:
        raise ValueError(f"{where} is missing {key!r}")
    return mapping[key]


def tpp_parameters(model: Mapping[str, Any]) -> int:
    """Parameter denominator of the fixed-TPP ladder (train.py:355-364): two
    vocabulary tables, per block 12 d^2 + 11 d, and the final norm."""

    d, layers, vocab = int(model["d_model"]), int(model["layers"]), int(model["vocab_size"])
    return 2 * vocab * d + layers * (12 * d * d + 11 * d) + d


def resolve_config(
    document: Mapping[str, Any],
    *,
    tier: str | None = None,
    context: str | None = None,
    batch_size: int | None = None,
    tokens_per_parameter: float | None = None,
) -> Config:
    """Resolves a schema-6 experiment document into a step Config.

    The duration is either a fixed step count (``run.training.duration.steps``)
    or a fixed tokens-per-parameter horizon (``tokens_per_parameter``): then
    steps = max(1, floor(tpp_parameters * tpp / tokens_per_step + 0.5)) and the
    CompleteP data multiplier is the tier's tpp_parameters over the base
    tier's (train.py:745-751, 792-800). `tokens_per_parameter` overrides the
    document's horizon like the reference's --tokens-per-parameter flag.
    """

    if int(_require(document, "schema_version", "config")) != 6:
        raise ValueError("only schema_version 6 documents are supported")
    family = _require(document, "family", "config")
    run = _require(document, "run", "config")
    tier_name = tier or family["default_tier"]
    context_name = context or family["default_context"]
    tiers = family["tiers"]
    if tier_name not in tiers:
        raise ValueError(f"unknown tier {tier_name!r}")
    model = tiers[tier_name]["model"]
    ctx = family["contexts"][context_name]
    param = family["parameterization"]
    base = tiers[param["base_tier"]]["model"]
    training = run["training"]
    optimizer = run["optimizer"]
    kernels = run["kernels"]
    if model.get("normalization", "rms_norm") != "rms_norm":
        raise ValueError("only rms_norm is supported (train.py:323)")
    _check_routing(model, tier_name)

    batch = int(batch_size or ctx["reference_batch_size"])
    seq_len = int(ctx["seq_len"])
    duration = training["duration"]
    fixed_steps = duration.get("steps")
    doc_tpp = duration.get("tokens_per_parameter")
    if (fixed_steps is None) == (doc_tpp is None):
        raise ValueError("run.training.duration must define exactly one of steps and "
                         "tokens_per_parameter")
    declared = None
    requested_tpp = None
    if fixed_steps is not None:
        if tokens_per_parameter is not None:
            raise ValueError("tokens_per_parameter cannot override a fixed-step configuration")
        steps = int(fixed_steps)
        data_multiplier = 1.0
    else:
        requested_tpp = float(tokens_per_parameter if tokens_per_parameter is not None else doc_tpp)
        if not math.isfinite(requested_tpp) or requested_tpp <= 0.0:
            raise ValueError(f"tokens_per_parameter must be positive and finite, got {requested_tpp}")
        declared = tpp_parameters(model)
        steps = max(1, int(math.floor(declared * requested_tpp / (batch * seq_len) + 0.5)))
        data_multiplier = declared / float(tpp_parameters(base))
    warmup = int(math.floor(steps * float(optimizer["warmup_ratio"]) + 0.5))
    warmup = min(warmup, steps - 1) if steps > 1 else 0
    return Config(
        steps=steps,
        batch_size=batch,
        seq_len=seq_len,
        layers=int(model["layers"]),
        heads=int(model["heads"]),
        d_model=int(model["d_model"]),
        mlp_mult=int(model["mlp_mult"]),
        vocab_size=int(model["vocab_size"]),
        semantic_vocab_size=int(model["semantic_vocab_size"]),
        parameterization=str(param["name"]),
        base_width=int(base["d_model"]),
        base_depth=int(base["layers"]),
        depth_alpha=float(param["depth_alpha"]),
        init_std=float(param["init_std"]),
        attention_scale=str(param["attention_scale"]),
        embeddings=str(param["embeddings"]),
        data_multiplier=data_multiplier,
        batch_multiplier=batch / float(ctx["reference_batch_size"]),
        learning_rate=float(optimizer["learning_rate"]),
        min_lr_ratio=float(optimizer["min_lr_ratio"]),
        warmup_steps=warmup,
        weight_decay=float(optimizer["weight_decay"]),
        adam_epsilon=float(optimizer["adam_epsilon"]),
        beta1=float(optimizer["beta1"]),
        beta2=float(optimizer["beta2"]),
        grad_clip=float(optimizer["grad_clip"]),
        vocab_tile_size=int(kernels.get("vocab_tile_size", 2048)),
        dtype_name=str(training["dtype"]),
        sampling=str(training.get("sampling", "shuffled_epochs")),
        tier=tier_name,
        document_masking=bool(ctx.get("document_masking", False)),
        experts=int(model.get("experts", 0)),
        expert_top_k=int(model.get("expert_top_k", 2)),
        expert_mult=int(model.get("expert_mult", 2)),
        router_aux_coefficient=float(model.get("router_aux_coefficient", 0.01)),
        declared_parameters=declared,
        target_tokens_per_parameter=requested_tpp,
    )


MOE_MAX_EXPERTS = 16  # gptb200_moe_* kernels: 1 <= experts <= 16, top_k <= min(4, experts)
MOE_MAX_TOP_K = 4


def _check_routing(model: Mapping[str, Any], label: str) -> None:
    """The routed tier's rules (recipes/reference_moe/train.py:362-371) plus
    the limits of the routing kernels, checked before anything is built."""

    experts = int(model.get("experts", 0))
    if not experts:
        return
    top_k = int(model.get("expert_top_k", 2))
    mult = int(model.get("expert_mult", 2))
    if top_k > experts:
        raise ValueError(f"{label}.expert_top_k must not exceed experts")
    if top_k * mult != int(model["mlp_mult"]):
        raise ValueError(f"{label} must satisfy expert_top_k * expert_mult == mlp_mult so active "
                         "MLP FLOPs match the dense tier")
    if experts > MOE_MAX_EXPERTS or top_k > MOE_MAX_TOP_K:
        raise ValueError(f"{label}: the routing kernels support up to {MOE_MAX_EXPERTS} experts "
                         f"and top-{MOE_MAX_TOP_K}, got {experts} experts top-{top_k}")


def load_config(name_or_path: str | pathlib.Path, **overrides: Any) -> Config:
    """Loads `configs/<name>.yaml` (or a path) and resolves it."""

    path = pathlib.Path(name_or_path)
    if not path.suffix:
        path = CONFIG_DIR / f"{name_or_path}.yaml"
    with open(path, "r", encoding="utf-8") as handle:
        document = yaml.safe_load(handle)
    return resolve_config(document, **overrides)


# ----------------------------------------------------------------- optimizer policy
def decay_for_name(name: str) -> bool:
    """`weight_decay_mask` (train.py:1252-1271): decide decay from the leaf name."""

    if name in {"token_embedding", "output_embedding"} or name.endswith("_w"):
        return True
    if name.endswith(("_b", "_bias", "_scale")):
        return False
    raise ValueError(f"weight-decay policy has no rule for parameter {name!r}")


def tensor_multipliers(name: str, in_block: bool, config: Config) -> tuple[float, float, float]:
    """(lr, eps, decay) multipliers of one tensor (train.py:1274-1333)."""

    if config.parameterization != "completep_fixed_tpp_v1":
        return 1.0, 1.0, 1.0
    width, depth, alpha = config.width_multiplier, config.depth_multiplier, config.depth_alpha
    if in_block:
        lr = (width ** -1 * depth ** (alpha - 1.0)) if name.endswith("_w") else depth ** (alpha - 1.0)
        eps = width ** -1 * depth ** -alpha
        wd = width if name.endswith("_w") else 1.0
        return lr, eps, wd
    if name == "token_embedding":
        return 1.0, width ** -1, 1.0
    if name == "final_ln_scale":
        return 1.0, 1.0, 1.0
    if name == "output_embedding":
        return width ** -1, 1.0, width
    raise ValueError(f"no CompleteP multipliers for {name!r}")


def effective_adam_betas(config: Config) -> tuple[float, float]:
    ratio = config.batch_multiplier / config.data_multiplier
    beta1 = 1.0 - (1.0 - config.beta1) * ratio
    beta2 = 1.0 - (1.0 - config.beta2) * ratio
    if not 0.0 <= beta1 < 1.0 or not 0.0 <= beta2 < 1.0:
        raise ValueError("fixed-TPP batch/data scaling produced invalid Adam momenta")
    return beta1, beta2


def horizon_scales(config: Config) -> tuple[float, float, float]:
    """(lr, eps, decay) horizon scales: sqrt(m_B/m_D), sqrt(m_D/m_B), sqrt(m_B/m_D)."""

    ratio = config.batch_multiplier / config.data_multiplier
    return math.sqrt(ratio), math.sqrt(1.0 / ratio), math.sqrt(ratio)


def learning_rate(step: int, config: Config) -> float:
    """Host restatement of train.py:1219-1236 (fp64; the device uses fp32)."""

    step_float = float(step)
    warmup = min(1.0, step_float / config.warmup_steps) if config.warmup_steps else 1.0
    span = max(1, config.steps - config.warmup_steps)
    progress = min(max((step_float - config.warmup_steps) / span, 0.0), 1.0)
    cosine = 0.5 * (1.0 + math.cos(math.pi * progress))
    multiplier = config.min_lr_ratio + (1.0 - config.min_lr_ratio) * cosine
    return config.learning_rate * horizon_scales(config)[0] * warmup * multiplier
