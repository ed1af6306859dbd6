"""Routed MLP (recipes/reference_moe/train.py:1230-1372) in the training step
against the CPU restatement: loss including the balance term, every gradient
(router, expert and bias tensors included), and the router statistics row."""

import numpy as np
import pytest
import torch

from oracle import reference_step as ref
from rig_b200 import ops
from rig_b200.config import load_config
from rig_b200.model import GPTTrainer, init_params
from rig_b200.tokens import zipf_tokens

pytestmark = pytest.mark.gpu


def _cfg():
    return load_config("smoke_parity").replace(experts=4, expert_top_k=2, expert_mult=2,
                                               router_aux_coefficient=0.01)


def _batch(cfg, seed):
    b, t = cfg.batch_size, cfg.seq_len
    w = zipf_tokens(b * (t + 1), cfg.vocab_size, seed).astype(np.int32).reshape(b, t + 1)
    return np.ascontiguousarray(w[:, :-1]), np.ascontiguousarray(w[:, 1:])


def test_moe_loss_and_grads(cuda):
    cfg = _cfg()
    params = init_params(cfg, 0)
    x, y = _batch(cfg, 3)
    loss_ref, grads_ref = ref.loss_and_grads(params, x, y, cfg)
    tr = GPTTrainer(cfg, cfg.batch_size, cuda)
    tr.load_params(params)
    tr.set_batch(torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda))
    tr.forward()
    tr.backward()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    loss = tr.loss.item()
    assert abs(loss - loss_ref) / abs(loss_ref) < 1e-3, (loss, loss_ref)
    grads = tr.export(tr.grads)
    worst = {}
    for k, g_ref in grads_ref.items():
        denom = np.linalg.norm(g_ref)
        worst[k] = np.linalg.norm(grads[k] - g_ref) / denom if denom > 0 else np.linalg.norm(grads[k])
    # Router and expert tensors: a token whose two largest router logits are
    # nearly tied can pick a different expert pair on the two sides (bf16-level
    # differences of the hidden state, growing with depth: 1 to 12 of 2048
    # tokens per layer here), which changes its expert and router gradients
    # wholesale. The routed MLP itself is held to 1e-2 on identical inputs in
    # test_routed_mlp_op; here the routed tensors (and the norm scale in front
    # of them) get 8e-2, the rest 2e-2.
    def tol(k):
        return 8e-2 if ("router" in k or "expert" in k or "ln2" in k) else 2e-2
    bad = {k: v for k, v in worst.items() if v > tol(k)}
    assert not bad, sorted(bad.items(), key=lambda kv: -kv[1])[:6]


def test_router_statistics_row(cuda):
    cfg = _cfg()
    params = init_params(cfg, 1)
    x, y = _batch(cfg, 4)
    tparams = {k: torch.tensor(v) for k, v in params.items()}
    router = []
    with torch.no_grad():
        ref.gpt_hidden(tparams, torch.as_tensor(x), cfg, router_out=router)
    tr = GPTTrainer(cfg, cfg.batch_size, cuda)
    tr.load_params(params)
    tr.set_batch(torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda))
    tr.forward()
    row = tr.router_history[0].cpu().numpy()
    E, L = cfg.experts, cfg.layers
    bal = np.mean([float(ref.load_balance_loss(mp, ld)) for mp, ld, _ in router])
    loads = np.stack([ld.numpy() for _, ld, _ in router])
    summ = np.stack([s.numpy() for _, _, s in router])
    # A few near-tied tokens per layer route differently on the two sides (see
    # test_moe_loss_and_grads): loads may differ by up to 16 of the 4096
    # assignments of a layer, everything else is a mean over all tokens.
    flip = 16.0 / (cfg.batch_size * cfg.seq_len * cfg.expert_top_k)
    assert abs(row[0] - bal) < 2e-3 * bal
    assert abs(row[1] - loads.max()) <= flip and abs(row[2] - loads.min()) <= flip
    np.testing.assert_allclose(row[3:6], summ.mean(0), rtol=5e-3)
    for layer in range(L):
        per = row[6 + layer * (3 + E): 6 + (layer + 1) * (3 + E)]
        np.testing.assert_allclose(per[:3], summ[layer], rtol=5e-3)
        np.testing.assert_allclose(per[3:], loads[layer], atol=flip)
        assert abs(per[3:].sum() - 1.0) < 1e-6  # every assignment counted once


def test_moe_steps_train(cuda, tmp_path):
    """A few optimizer steps stay finite and the loss drops (graph capture too);
    the training log carries the router statistics columns of every step."""

    cfg = _cfg()
    tr = GPTTrainer(cfg, cfg.batch_size, cuda)
    tr.load_params(init_params(cfg, 0))
    x, y = _batch(cfg, 7)
    xd, yd = torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda)
    tr.train_step(xd, yd)
    tr.capture()
    for _ in range(5):
        tr.train_step(xd, yd)
    torch.cuda.synchronize()
    h = tr.history[:6, 0].cpu().numpy()
    assert np.all(np.isfinite(h)) and h[-1] < h[0], h
    assert ops.device_error() == 0
    from rig_b200 import logpack, runlog

    tr.write_training_log(tmp_path, 6)
    log = logpack.read_log(tmp_path / runlog.TRAINING_LOG_NAME)
    assert log.columns == runlog.training_log_columns(cfg.layers, cfg.experts)
    want = np.concatenate((tr.history[:6].cpu().numpy(), tr.router_history[:6].cpu().numpy()), 1)
    np.testing.assert_array_equal(log.values, want)
    assert np.all(log.values[:, 3] > 0)  # the balance loss of every step
    E = cfg.experts
    for layer in range(cfg.layers):
        c0 = 9 + layer * (3 + E) + 3
        np.testing.assert_allclose(log.values[:, c0:c0 + E].sum(1), 1.0, atol=1e-5)


@pytest.mark.parametrize("experts", [4, 3, 8, 12, 16])
def test_routed_mlp_op(cuda, experts):
    """One routed block on identical inputs: the forward output and the input,
    router, expert and bias gradients match the restatement's autograd (the
    routing is identical here, so the bound is tight). Expert counts cover
    every register layout of the router backward (8, 4 and 2 features a
    thread) and counts that are not powers of two."""

    cfg = _cfg().replace(layers=1, experts=experts)
    params = init_params(cfg, 2)
    n, d = cfg.batch_size * cfg.seq_len, cfg.d_model
    g = torch.Generator().manual_seed(9)
    xn = torch.randn(cfg.batch_size, cfg.seq_len, d, generator=g).bfloat16()
    resid = torch.randn(cfg.batch_size, cfg.seq_len, d, generator=g).bfloat16()
    dx = (0.01 * torch.randn(cfg.batch_size, cfg.seq_len, d, generator=g)).bfloat16()
    names = ["router_w", "expert_up_w", "expert_up_b", "expert_down_w", "expert_down_b"]
    tp = {k: torch.tensor(params[f"blocks/0/{k}"], requires_grad=True) for k in names}
    xr = xn.float().requires_grad_(True)
    out, mean_p, load, _ = ref.routed_mlp(xr.bfloat16(), tp["router_w"], tp["expert_up_w"],
                                          tp["expert_up_b"], tp["expert_down_w"],
                                          tp["expert_down_b"], cfg.experts, cfg.expert_top_k)
    mult = cfg.branch_scale
    x_out = resid + mult * out
    aux = cfg.router_aux_coefficient * ref.load_balance_loss(mean_p, load)
    ((x_out.float() * dx.float()).sum() + aux).backward()

    tr = GPTTrainer(cfg, cfg.batch_size, cuda)
    tr.load_params(params)
    blk = tr.blocks[0]
    tr.ln2[0].copy_(xn.reshape(n, d).to(cuda))
    tr.xm[0].copy_(resid.reshape(n, d).to(cuda))
    tr.m_stats.zero_()
    tr.grads.zero_()
    tr._moe_forward(0, blk)
    tr._moe_finalize()
    tr._moe_backward(0, blk, dx.reshape(n, d).to(cuda))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    def rel(a, b):
        a, b = a.detach().float(), b.detach().float()
        return float((a - b).norm() / b.norm())
    assert rel(tr.x[1].cpu(), x_out.reshape(n, d)) < 5e-3
    assert rel(tr.dln.cpu(), xr.grad.reshape(n, d)) < 1e-2
    for k in names:
        got = tr.grad_view(f"blocks/0/{k}").cpu()
        assert rel(got, tp[k].grad) < 1e-2, (k, rel(got, tp[k].grad))
