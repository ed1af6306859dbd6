#!/usr/bin/env python
"""Benchmark of the B200 GPT training step (BASELINE metric: train tokens/s and
MFU of the 125M tier, bf16, seq 1024, global batch 128, at 1/2/4/8 GPUs).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    python bench.py --op attention|lce|gemm|gelu_gemm   (op configurations, 1 GPU)

One process per GPU (torchrun for N > 1). A "step" is one full training step
(forward, backward, gradient all-reduce, AdamW) over the rank's share of the
128 x 1024-token global batch (strong scaling: the global batch is fixed).

Printed by rank 0 as one JSON line:
  value        whole-job tokens/s with the step's inputs already in HBM
  e2e          the same through the public API with the batch copied from
               pinned host memory and the loss read back every step
  roofline     the GEMM kernel family (the dominant kernel) timed with CUDA
               events around its launches in instrumented steps
  cpu_baseline the CPU restatement of the reference step (oracle/) on this
               host's cores, on a bounded sample (rank 0, N = 1 only)
`--impl reference` times that CPU restatement alone as the reference arm (the
reference itself is JAX, which this image does not have).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gpt-speedrun-tpu_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "train tokens/sec + MFU, GPT-125M bf16 seq1024"
UNIT = "tokens/s"
NOMINAL_BF16_TFLOPS = 2250.0


def flops_per_token(cfg) -> int:
    """Reference MFU convention (docs/FLOPS.md:9-24 of the rig): 6 x matmul
    parameters (incl. the tied head) + full-square attention 12*L*H*T*Dh."""

    d, L = cfg.d_model, cfg.layers
    if cfg.experts:  # active parameters: top_k experts of width expert_mult*d, plus the router
        mlp = 2 * cfg.expert_top_k * d * cfg.expert_mult * d + d * cfg.experts
    else:
        mlp = 2 * d * cfg.mlp_mult * d
    return (6 * (L * (4 * d * d + mlp) + cfg.vocab_size * d)
            + 12 * L * cfg.heads * cfg.seq_len * cfg.head_dim)


def gemm_traffic_estimate(cfg, local_batch: int, launches: int):
    """DRAM bytes per GEMM launch of the matmul family, from the committed ncu
    capture of one reduced step (profiles/gemm_traffic_125m_batch16.md, the
    JSON block), scaled by the tokens per GPU. Only for the dense 125M tier
    with the captured launch count; (None, reason) otherwise."""

    path = ROOT / "profiles" / "gemm_traffic_125m_batch16.md"
    if cfg.experts or cfg.tier != "125m_768_tied" or not path.exists():
        return None, "no committed capture of this configuration's GEMM traffic"
    text = path.read_text()
    block = json.loads(text.split("```json", 1)[1].split("```", 1)[0])
    if launches != block["matmul_launches"]:
        return None, f"launch count {launches} differs from the capture's {block['matmul_launches']}"
    scale = local_batch * cfg.seq_len / block["tokens"]
    per_launch = (block["dram_read_bytes"] + block["dram_write_bytes"]) / launches * scale
    return per_launch, (f"ncu capture at {block['tokens']} tokens (profiles/gemm_traffic_125m_batch16.md) "
                        f"scaled x{scale:g} to {local_batch * cfg.seq_len} tokens per GPU")


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16": data["bf16_tflops"],
                "bf16_sustained": data["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock/throttle samples every 50 ms, kept for the timed window.

    Started before the warm-up steps; `wait_ready` blocks until the first sample
    exists, and `stop(t0, t1)` keeps the samples whose timestamps fall inside the
    host-time window [t0, t1] of the timed region (a region shorter than one
    sampling interval keeps the single nearest sample, and says so)."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def wait_ready(self, timeout_s: float = 10.0) -> None:
        t_end = time.time() + timeout_s
        while self.proc is not None and time.time() < t_end:
            if os.path.getsize(self.file.name) > 0:
                return
            time.sleep(0.02)

    @staticmethod
    def _ts(text: str) -> float:
        try:
            return datetime.datetime.strptime(text, "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return float("nan")

    def stop(self, t0: float, t1: float) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.flush()
        rows = []
        for line in pathlib.Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                rows.append((self._ts(parts[0]), parts[1:]))
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        inside = [r for t, r in rows if t0 <= t <= t1]
        note = None
        if not inside:
            mid = 0.5 * (t0 + t1)
            inside = [min(rows, key=lambda tr: abs(tr[0] - mid) if tr[0] == tr[0] else 1e30)[1]]
            note = "timed region shorter than the sampling interval: nearest sample"
        sm = [float(r[1]) for r in inside if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in inside if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in inside for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        out = {"sm_mhz": statistics.median(sm) if sm else None,
               "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(inside)}
        if note:
            out["note"] = note
        return out


def make_stream(cfg, rank: int, world: int, steps: int, seed: int):
    """Synthetic Zipf(1.1) tokens (seed 3) in an llm.c shard, read through the
    shuffled-epoch stream like the reference trainer (stream seed = seed + 1)."""

    from rig_b200.tokens import (ShardedTokens, ShuffledEpochBatchStream, load_token_file,
                                 write_llmc_shard, zipf_tokens)

    n_tokens = (steps + 2) * cfg.batch_size * (cfg.seq_len + 1)
    path = pathlib.Path(tempfile.gettempdir()) / f"gptb200_zipf_s{seed}_{n_tokens}_r{rank}.bin"
    if not path.exists():
        write_llmc_shard(path, zipf_tokens(n_tokens, cfg.vocab_size, seed))
    shard = np.ascontiguousarray(load_token_file(path, data_format="llmc"))
    return ShuffledEpochBatchStream(ShardedTokens([shard]), global_batch_size=cfg.batch_size,
                                    seq_len=cfg.seq_len, vocab_size=cfg.vocab_size, seed=seed + 1,
                                    process_index=rank, process_count=world)


def cpu_oracle_rate(cfg, tokens: int, steps: int, threads: int) -> tuple[float, str]:
    """Tokens/s of the CPU restatement of the reference step on `tokens`-token
    samples (one sequence each), `steps` timed steps after one warm-up."""

    from oracle import reference_step as ref
    from rig_b200.tokens import zipf_tokens

    torch.set_num_threads(threads)
    seqs = max(1, tokens // cfg.seq_len)
    small = cfg.replace(batch_size=seqs)
    params = ref.init_params(small, 3)
    trainer = ref.OracleTrainer(small, params)
    toks = zipf_tokens((steps + 1) * seqs * (cfg.seq_len + 1), cfg.vocab_size, 7).astype(np.int32)
    w = toks.reshape(steps + 1, seqs, cfg.seq_len + 1)
    trainer.train_step(w[0][:, :-1], w[0][:, 1:])
    t0 = time.perf_counter()
    for i in range(1, steps + 1):
        trainer.train_step(w[i][:, :-1], w[i][:, 1:])
    dt = time.perf_counter() - t0
    sample = (f"{steps} step(s) of {seqs} x {cfg.seq_len} tokens of the {cfg.tier} step "
              "(forward, backward, AdamW over all parameters)")
    return steps * seqs * cfg.seq_len / dt, sample


def run_reference(args, cfg, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    rate, sample = cpu_oracle_rate(cfg, cfg.seq_len, max(1, args.steps), threads)
    line = {
        "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * cfg.seq_len / rate,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic Zipf(1.1) tokens", "impl": "reference",
        "config": {"workload": f"{cfg.tier} training step, CPU restatement", "seq_len": cfg.seq_len},
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference is JAX (not installable offline); its step is timed as the "
                "oracle/ CPU restatement",
    }
    print(json.dumps(line), flush=True)


def run_op(args) -> None:
    """Op-level configurations of the same kernels (one GPU, rank 0):

    * attention: benchmark config 3 -- q, k, v, dO [16, 12, 1024, 64] bf16 ~ N(0, 1)
      (seeds 0..2), RoPE on q and k, scale 1/64; one step = forward + backward;
      algorithmic FLOPs (causal) 6 B H T^2 D = 7.73e10 per step.
    * lce: config 2 -- hidden [65536, 768] bf16 ~ N(0, 1), embedding
      [50304, 768] bf16 ~ N(0, 0.02), Zipf(1.1) labels (seed 1); one step = mean
      loss + dH + dE; algorithmic FLOPs 6 N V D = 1.519e13 per step.
    * gemm: the MLP down projection of the step (M = 131072, K = 3072,
      N = 768) with the plain bf16 epilogue.
    * gelu_gemm: the MLP up projection of the step (M = 131072, K = 768,
      N = 3072) with the bias + GELU epilogue (writes g and gelu').
    Each timed iteration is bracketed by CUDA events on the launching stream;
    a 256 MB buffer is rewritten between iterations (outside the events) so no
    input is served from the 126 MB L2.
    """

    from rig_b200 import _lib, ops
    from rig_b200.tokens import zipf_tokens

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    gen = lambda seed: torch.Generator(device="cpu").manual_seed(seed)  # noqa: E731
    if args.op == "attention":
        b, h, t, d = 16, 12, 1024, 64
        q, k, v = (torch.randn(b, h, t, d, generator=gen(i)).bfloat16().to(dev) for i in range(3))
        do = torch.randn(b, h, t, d, generator=gen(2)).bfloat16().to(dev)
        rope = ops.rope_tables(t, d, dev)
        ops.rope_apply(q.transpose(1, 2), rope)
        ops.rope_apply(k.transpose(1, 2), rope)
        o, lse = torch.empty_like(q), torch.empty(b, h, t, device=dev)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ws = ops.attention_workspace(b, h, t, dev)
        fwd = lambda: ops.attention_fwd(q, k, v, o, lse, scale=1 / 64)  # noqa: E731
        bwd = lambda: ops.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, scale=1 / 64,  # noqa
                                        rope=rope, workspace=ws)
        # causal algorithmic FLOPs: forward 2 B H T^2 D, backward 4 B H T^2 D
        parts = {"fwd": (fwd, 2.0 * b * h * t * t * d), "bwd": (bwd, 4.0 * b * h * t * t * d)}
        config = {"workload": "config 3: causal attention fwd+bwd", "batch": b, "heads": h,
                  "seq_len": t, "head_dim": d, "rope": True, "scale": "1/64"}
    elif args.op == "lce":
        n, vocab, d = 65536, 50304, 768
        hid = torch.randn(n, d, generator=gen(0)).bfloat16().to(dev)
        emb = (0.02 * torch.randn(vocab, d, generator=gen(1))).bfloat16().to(dev)
        tgt = torch.from_numpy(zipf_tokens(n, vocab, 1).astype("int32")).to(dev)
        losses, lse = torch.empty(n, device=dev), torch.empty(n, device=dev)
        mean = torch.empty(1, device=dev)
        cot = torch.full((n,), 1.0 / n, device=dev)
        dh = torch.empty_like(hid)
        de = torch.zeros(vocab, d, device=dev)
        fws, bws = ops.lce_fwd_workspace(n, vocab, dev), ops.lce_bwd_workspace(n, vocab, dev)
        fwd = lambda: ops.lce_fwd(hid, emb, tgt, vocab, losses, lse, mean, workspace=fws)  # noqa
        bwd = lambda: ops.lce_bwd(hid, emb, tgt, lse, cot, vocab, dh, de, workspace=bws)  # noqa
        parts = {"fwd": (fwd, 2.0 * n * vocab * d), "bwd": (bwd, 4.0 * n * vocab * d)}
        config = {"workload": "config 2: tied linear cross-entropy loss + dH + dE", "tokens": n,
                  "vocab": vocab, "d_model": d}
    elif args.op == "gemm":
        m, kk, nn = 131072, 3072, 768
        x = torch.randn(m, kk, generator=gen(0)).bfloat16().to(dev)
        w = (0.02 * torch.randn(kk, nn, generator=gen(1))).bfloat16().to(dev)
        out = torch.empty(m, nn, dtype=torch.bfloat16, device=dev)
        run = lambda: ops.matmul(x, w, out=out)  # noqa: E731
        parts = {"gemm": (run, 2.0 * m * nn * kk)}
        config = {"workload": "MLP down projection, plain bf16 epilogue", "M": m, "K": kk, "N": nn}
    elif args.op == "gelu_gemm":
        m, kk, nn = 131072, 768, 3072
        x = torch.randn(m, kk, generator=gen(0)).bfloat16().to(dev)
        w = (0.02 * torch.randn(kk, nn, generator=gen(1))).bfloat16().to(dev)
        bias = torch.zeros(nn, dtype=torch.bfloat16, device=dev)
        g, gp = (torch.empty(m, nn, dtype=torch.bfloat16, device=dev) for _ in range(2))
        run = lambda: ops.matmul(x, w, bias=bias, out=g, kind=_lib.EPI_BIAS_GELU, aux=gp)  # noqa
        parts = {"gemm": (run, 2.0 * m * nn * kk)}
        config = {"workload": "MLP up projection + bias + GELU (writes g and gelu')", "M": m,
                  "K": kk, "N": nn}
    else:
        raise SystemExit(f"unknown --op {args.op}")

    for _ in range(args.warmup):
        for fn, _fl in parts.values():
            fn()
    torch.cuda.synchronize()
    times = {name: 0.0 for name in parts}
    for _ in range(args.steps):
        for name, (fn, _fl) in parts.items():
            flush.fill_(1)
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record()
            fn()
            en.record()
            torch.cuda.synchronize()
            times[name] += st.elapsed_time(en)
    if ops.device_error() != 0:
        raise RuntimeError("device-side error flag set during the benchmark")
    ms = sum(times.values()) / args.steps
    flops = sum(fl for _fn, fl in parts.values())
    peaks = measured_peaks()
    tflops = flops / (ms / 1e3) / 1e12
    print(json.dumps({
        "metric": f"{args.op} TFLOP/s (algorithmic)", "value": tflops, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, shapes and distributions of the op configuration)",
        "config": {**config, "l2": "256 MB buffer rewritten between timed iterations"},
        "parts_ms": {k: v / args.steps for k, v in times.items()},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": peaks["bf16"],
                     "unit": "TFLOP/s", "frac": tflops / peaks["bf16"],
                     "peak_source": f"{peaks['source']} bf16 burst (kernel timed alone)"},
    }), flush=True)


def run_kernels(args) -> None:
    """Memory-bound kernels of the step, one entry point at a time, at the
    shapes of the 125M step on one GPU (N = 131,072 tokens, d 768, hidden
    3072, vocabulary 50,304, 123.7 M parameters) and of a routed layer of the
    same width (8 experts, top-2, expert width 1536). Each timed call is
    bracketed by CUDA events on the launching stream after a 256 MB L2 flush;
    achieved GB/s = the entry point's algorithmic bytes (stated per case:
    every input read once, every output written once) / its mean time,
    against the measured HBM copy bandwidth. One JSON line per case, then a
    summary line."""

    from rig_b200 import _lib, ops
    from rig_b200.config import load_config
    from rig_b200.model import ParamLayout
    from rig_b200.tokens import zipf_tokens

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks = measured_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    N, d, h, V = 131072, 768, 3072, 50304
    g = torch.Generator(device="cpu").manual_seed(0)
    bf = lambda *shape: torch.randn(*shape, generator=g).bfloat16().to(dev)  # noqa: E731
    x, dy, dxi = bf(N, d), bf(N, d), bf(N, d)
    scale = (1 + 0.1 * torch.randn(d, generator=g)).bfloat16().to(dev)
    y, dx = torch.empty_like(x), torch.empty_like(x)
    rstd = torch.empty(N, device=dev)
    dscale, dcol = torch.zeros(d, device=dev), torch.zeros(d, device=dev)
    ops.rms_norm_fwd(x, scale, y, rstd)
    rws = ops._scratch(ops.rms_norm_bwd_workspace_size(N, d), dev)
    u = bf(N, h)
    bgrad = torch.zeros(h, device=dev)
    cws = ops._scratch(ops.colsum_workspace_size(N, h), dev)
    tok = torch.from_numpy(zipf_tokens(N, V, 3).astype(np.int32)).to(dev)
    table = bf(V, d)
    emb = torch.empty(N, d, dtype=torch.bfloat16, device=dev)
    dtable = torch.zeros(V, d, device=dev)
    ews = ops._scratch(ops.embedding_bwd_workspace_size(N, d, V), dev)
    uniq = int(torch.unique(tok).numel())
    cfg = load_config("baseline_125m")
    layout = ParamLayout(cfg)
    P = layout.numel
    params = (0.02 * torch.randn(P, generator=g)).to(dev)
    grads = (1e-3 * torch.randn(P, generator=g)).to(dev)
    m1, v1 = torch.zeros_like(params), torch.zeros_like(params)
    pbf = torch.empty(P, dtype=torch.bfloat16, device=dev)
    groups = (_lib.TensorGroup * 1)(_lib.TensorGroup(offset=0, size=P, lr_mult=1.0, eps_mult=1.0,
                                                      wd_mult=1.0, decay=1))
    groups_dev = torch.frombuffer(bytearray(bytes(groups)), dtype=torch.uint8).to(dev)
    adam_cfg = _lib.AdamWConfig(learning_rate=2 ** -8, horizon_lr_scale=1.0, min_lr_ratio=0.1,
                                warmup_steps=10, total_steps=10 ** 6, beta1=0.9, beta2=0.95,
                                eps=1e-8, eps_horizon_scale=1.0, weight_decay=0.1,
                                wd_horizon_scale=1.0, grad_clip=0.0, grad_scale=1.0)
    step = torch.zeros(1, dtype=torch.int32, device=dev)
    aws = ops.adamw_workspace(P, dev)
    # split-K reduction of the QKV weight gradient (768 x 2304 over K = N)
    slabs = ops.gemm_workspace_size(d, 3 * d, N, _lib.EPI_F32_SPLITK) // (d * 3 * d * 4)
    # routed layer: 8 experts, top-2, expert width 1536
    E, k, eh = 8, 2, 2 * d
    R = ops.moe_rows(N, k, E)
    router_w = (0.02 * torch.randn(d, E, generator=g)).to(dev)
    logits = torch.empty(N, E, device=dev)
    chosen = torch.empty(N, k, dtype=torch.int32, device=dev)
    gate = torch.empty(N, k, device=dev)
    stats = torch.zeros(2 * E + 3, device=dev)
    seg = torch.zeros(E, 2, dtype=torch.int32, device=dev)
    total = torch.zeros(1, dtype=torch.int32, device=dev)
    pos = torch.empty(N, k, dtype=torch.int32, device=dev)
    src = torch.empty(R, dtype=torch.int32, device=dev)
    grouped = torch.empty(R, d, dtype=torch.bfloat16, device=dev)
    mws = ops.moe_dispatch_workspace(N, k, E, dev)
    ops.moe_route(x, router_w, logits, chosen, gate, stats)
    ops.moe_dispatch(chosen, x, E, seg, total, pos, src, grouped, mws)
    out_rows = bf(R, d)
    xo = torch.empty_like(x)
    dout_rows = torch.empty(R, d, dtype=torch.bfloat16, device=dev)
    dgate = torch.empty(N, k, device=dev)
    bal = torch.zeros(E, device=dev)
    dgrouped = bf(R, d)
    drw = torch.zeros(d, E, device=dev)
    dxr = torch.empty_like(x)
    hid = bf(R, eh)
    bexp = torch.zeros(E, eh, device=dev)

    B2 = 2  # bf16 bytes
    cases = [
        ("rms_norm_fwd", lambda: ops.rms_norm_fwd(x, scale, y, rstd), 2 * N * d * B2 + 4 * N,
         "read x, write y + rstd"),
        ("rms_norm_bwd", lambda: ops.rms_norm_bwd(x, scale, rstd, dy, dxi, dx, dscale, dcol, 1.0,
                                                  workspace=rws), 4 * N * d * B2 + 4 * N,
         "read x, dy, dx_in, rstd; write dx (dscale and column sums fused)"),
        ("colsum", lambda: ops.colsum(u, bgrad, 1.0, workspace=cws), N * h * B2,
         "read the [N, 3072] bias-gradient source once"),
        ("embedding_fwd", lambda: ops.embedding_fwd(tok, table, emb), 2 * N * d * B2 + 4 * N,
         "gather N rows, write N rows"),
        ("embedding_bwd", lambda: ops.embedding_bwd(tok, dy, dtable, workspace=ews),
         N * d * B2 + 4 * N + 2 * uniq * d * 4,
         f"read dout and ids, read+write the {uniq} touched fp32 rows"),
        ("adamw_step", lambda: ops.adamw_step(params, m1, v1, grads, groups_dev, 1, adam_cfg, step,
                                              None, None, pbf, aws), 30 * P,
         "p, m, v read+write, g read (fp32), bf16 mirror write: 30 B/param"),
        ("cast_bf16", lambda: ops.cast_bf16(params, pbf), 6 * P, "fp32 read, bf16 write"),
        ("moe_route", lambda: ops.moe_route(x, router_w, logits, chosen, gate, stats),
         N * d * B2 + N * E * 4 + N * k * 8, "read x; write logits, choices, gates"),
        ("moe_dispatch", lambda: ops.moe_dispatch(chosen, x, E, seg, total, pos, src, grouped, mws),
         N * k * 4 + N * d * B2 * k + R * d * B2 + N * k * 4 + R * 4,
         "read choices and x rows (k per token); write grouped rows, positions, sources"),
        ("moe_combine", lambda: ops.moe_combine(out_rows, pos, gate, x, 1.0, xo),
         N * k * d * B2 + 2 * N * d * B2 + N * k * 8, "read k expert rows + residual, write x"),
        ("moe_combine_bwd", lambda: ops.moe_combine_bwd(dy, 1.0, out_rows, pos, gate, src, total,
                                                        dout_rows, dgate),
         N * d * B2 + 2 * R * d * B2 + N * k * 12, "read dx and expert rows, write d_out rows"),
        ("moe_route_bwd", lambda: ops.moe_route_bwd(x, router_w, logits, chosen, gate, dgate, bal,
                                                    dgrouped, pos, drw, dxr),
         2 * N * d * B2 + N * k * d * B2 + N * E * 4, "read x, logits, k grouped-gradient rows; write dx"),
        ("moe_segment_colsum", lambda: ops.moe_segment_colsum(hid, seg, E, bexp), R * eh * B2,
         "read the [rows, 1536] expert buffer once"),
    ]
    results = []
    for name, fn, nbytes, what in cases:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        t = 0.0
        for _ in range(args.steps):
            flush.fill_(1)
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record()
            fn()
            en.record()
            torch.cuda.synchronize()
            t += st.elapsed_time(en)
        ms = t / args.steps
        gbs = nbytes / (ms / 1e3) / 1e9
        results.append({"kernel": name, "ms": ms, "bytes": nbytes, "bytes_are": what,
                        "achieved_gbs": gbs, "frac": gbs / peaks["hbm_gbs"]})
        print(json.dumps(results[-1]), flush=True)
    if ops.device_error() != 0:
        raise RuntimeError("device-side error flag set during the kernel benchmark")
    print(json.dumps({
        "metric": "memory-bound kernels, achieved HBM GB/s", "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "peak": peaks["hbm_gbs"],
        "peak_source": f"{peaks['source']} HBM copy", "splitk_slabs_qkv_wgrad": slabs,
        "config": {"workload": "125M step shapes: N 131072, d 768, hidden 3072, V 50304; "
                               "routed layer 8 experts top-2 width 1536",
                   "l2": "256 MB buffer rewritten between timed calls"},
        "kernels": {r["kernel"]: round(r["achieved_gbs"], 1) for r in results},
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", default="baseline_125m")
    ap.add_argument("--tier", default=None, help="tier of the config (default: its default tier)")
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--batch", type=int, default=None,
                    help="global batch override (reduced cases for profiling; default: the "
                         "config's 128)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="no CUDA graph replay")
    ap.add_argument("--dp-graph", action="store_true",
                    help="capture the data-parallel step as a CUDA graph also above 2 GPUs")
    ap.add_argument("--single-update", action="store_true",
                    help="one AdamW pass after the backward instead of per-bucket updates")
    ap.add_argument("--atomic-wgrad", action="store_true",
                    help="fp32 atomics for split-K weight gradients (not bit-reproducible)")
    ap.add_argument("--op", choices=["step", "attention", "lce", "gemm", "gelu_gemm", "kernels"],
                    default="step",
                    help="op-level configuration instead of the training step (1 GPU)")
    args = ap.parse_args()
    if args.op == "kernels":
        run_kernels(args)
        return
    if args.op != "step":
        run_op(args)
        return

    from rig_b200.config import load_config
    from rig_b200.mesh import initialize_distributed_runtime

    cfg = load_config(args.config, batch_size=args.batch, tier=args.tier)
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, cfg, rank, int(os.environ.get("WORLD_SIZE", "1")))
        return

    import torch.distributed as dist

    from rig_b200 import ops
    from rig_b200.model import GPTTrainer, init_params

    rank, world, local = initialize_distributed_runtime("nccl")
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    local_batch = cfg.batch_size // world
    total_steps = args.warmup + 2 * args.steps + 1
    stream = make_stream(cfg, rank, world, total_steps, args.seed)
    batches = [stream.next_batch() for _ in range(total_steps)]
    pinned = [(torch.from_numpy(x).pin_memory(), torch.from_numpy(y).pin_memory())
              for x, y in batches]
    dev_batches = [(x.to(device), y.to(device)) for x, y in pinned[: args.warmup + args.steps]]

    trainer = GPTTrainer(cfg, local_batch, device, process_group=None, world_size=world,
                         history_steps=max(cfg.steps, total_steps + 1),
                         deterministic=not args.atomic_wgrad,
                         overlap_optimizer=False if args.single_update else None)
    trainer.load_params(init_params(cfg, args.seed))
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(ms: float) -> float:
        if world == 1:
            return ms
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local)
    for i in range(args.warmup):
        trainer.train_step(*dev_batches[i])
        if i == 0 and not args.eager and (world <= 2 or args.dp_graph):
            # after one eager step; replays the same launches. Measured and
            # checked at 1 and 2 GPUs; with more ranks NCCL may take another
            # algorithm (NVLink SHARP) whose buffer registration inside a
            # capture is unchecked here, so those runs stay eager unless asked.
            trainer.capture()
    clocks.wait_ready()
    barrier()

    # ---- value: inputs resident in HBM
    launches0 = ops.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    t_host0 = time.time()
    start.record()
    for i in range(args.steps):
        trainer.train_step(*dev_batches[args.warmup + i])
    end.record()
    barrier()
    t_host1 = time.time()
    launches = ops.launch_count() - launches0
    if trainer.graph is not None:  # replays do not pass through the host launch counter
        launches += trainer.graph_launches * args.steps
    clock_info = clocks.stop(t_host0, t_host1)
    ms = max_over_ranks(start.elapsed_time(end))
    global_tokens = cfg.batch_size * cfg.seq_len
    value = global_tokens * args.steps / (ms / 1000.0)

    # ---- e2e: H2D of each step's batch from pinned host memory + D2H of the loss
    loss_host = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    off = args.warmup + args.steps
    barrier()
    start.record()
    for i in range(args.steps):
        x, y = pinned[off + i]
        trainer.set_batch(x, y)
        trainer.train_step()
        loss_host[i : i + 1].copy_(trainer.loss, non_blocking=True)
    end.record()
    barrier()
    ms_e2e = max_over_ranks(start.elapsed_time(end))
    e2e_value = global_tokens * args.steps / (ms_e2e / 1000.0)
    if not np.all(np.isfinite(loss_host.numpy())):
        raise FloatingPointError(f"non-finite loss during the benchmark: {loss_host.tolist()}")

    # ---- roofline of the dominant kernel family (tcgen05 GEMM), instrumented steps
    peaks = measured_peaks()
    graph, trainer.graph = trainer.graph, None  # instrumented step runs eagerly
    ops.gemm_timer = []
    gstart, gend = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gstart.record()
    trainer.train_step(*dev_batches[-1])
    gend.record()
    torch.cuda.synchronize()
    timed = ops.gemm_timer
    ops.gemm_timer = None
    trainer.graph = graph
    gemm_ms = sum(s.elapsed_time(e) for s, e, _, _ in timed)
    gemm_flops = sum(f for _, _, f, _ in timed)
    gemm_bytes = sum(b for _, _, _, b in timed)
    step_ms_instr = gstart.elapsed_time(gend)
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12
    traffic, traffic_note = gemm_traffic_estimate(cfg, local_batch, len(timed))
    roofline = {
        "bound": "tensor", "kernel": "gemm_tc_kernel (tcgen05 GEMM, all launches of one step)",
        "achieved": achieved, "peak": peaks["bf16_sustained"], "unit": "TFLOP/s",
        "frac": achieved / peaks["bf16_sustained"],
        "peak_source": f"{peaks['source']} sustained bf16 (kernel timed inside a long step)",
        "traffic": traffic, "traffic_unit": "DRAM bytes read + written per launch",
        "traffic_note": traffic_note,
        "algorithmic_bytes_per_launch": gemm_bytes / max(len(timed), 1),
        "launches_per_step": len(timed), "share_of_step": gemm_ms / step_ms_instr,
        "algorithmic_flops_per_step": gemm_flops,
    }

    fpt = flops_per_token(cfg)
    mfu = value * fpt / (world * peaks["bf16"] * 1e12)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: Zipf(s=1.1) token ids (seed 3) in an llm.c uint16 shard, read "
                "through the shuffled-epoch stream; random-init weights (CompleteP init)",
        "config": {"workload": f"{cfg.tier} training step (fwd+bwd+allreduce+AdamW)",
                   "model": f"GPT {cfg.layers}L/{cfg.d_model}d/{cfg.heads}H "
                            + ("tied" if cfg.tied else "untied") + f" vocab {cfg.vocab_size}"
                            + (f", {cfg.experts} experts top-{cfg.expert_top_k}"
                               if cfg.experts else ""), "global_batch": cfg.batch_size,
                   "seq_len": cfg.seq_len, "parallelism": f"dp{world}",
                   "bit_reproducible": trainer.deterministic,
                   "optimizer": "per-bucket AdamW overlapped with the backward"
                                if trainer.overlap_optimizer else "one AdamW pass after the backward",
                   "l2": "working set (activations ~40 GB/GPU at dp1) far larger than L2"},
        "mfu": mfu, "mfu_peak_tflops": peaks["bf16"], "mfu_peak_source": peaks["source"],
        "mfu_vs_nominal_2250": value * fpt / (world * NOMINAL_BF16_TFLOPS * 1e12),
        "flops_per_token": fpt,
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": 2 * local_batch * cfg.seq_len * 4,
                "d2h_bytes_per_step": 4, "ms_per_step": ms_e2e / args.steps},
        "roofline": roofline,
        "clocks": clock_info,
        "gpu_launches": int(launches),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, sample = cpu_oracle_rate(cfg, cfg.seq_len, 1, threads)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    # The captured step holds references to the NCCL communicator: release it
    # before the process group goes away.
    trainer.graph = None
    del graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
