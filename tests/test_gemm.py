"""tcgen05 GEMM vs a plain fp32 PyTorch reference, every operand layout and epilogue."""

import pytest
import torch

from rig_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _operands(m, n, k, a_mn, b_mn, dev, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(dev).bfloat16()
    b = torch.randn(n, k, generator=g).to(dev).bfloat16()
    a_st = a.t().contiguous() if a_mn else a
    b_st = b.t().contiguous() if b_mn else b
    return a, b, a_st, b_st


def _rel(x, ref):
    return ((x.float() - ref).norm() / ref.norm()).item()


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("shape", [(128, 256, 64), (256, 512, 128), (1024, 768, 768),
                                   (384, 264, 200), (136, 40, 24)])
def test_layouts_bf16(cuda, a_mn, b_mn, shape):
    m, n, k = shape
    a, b, a_st, b_st = _operands(m, n, k, a_mn, b_mn, cuda)
    c = torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
    ops.gemm(a_st, b_st, c, a_mn_major=bool(a_mn), b_mn_major=bool(b_mn), m=m, n=n, k=k)
    ref = a.float() @ b.float().t()
    assert _rel(c, ref) < 4e-3
    assert ops.device_error() == 0


def test_bias_alpha_residual(cuda):
    m, n, k = 300, 768, 256
    a, b, _, b_st = _operands(m, n, k, 0, 1, cuda, 1)
    bias = torch.randn(n, device=cuda).bfloat16()
    res = torch.randn(m, n, device=cuda).bfloat16()
    c = torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
    ops.gemm(a, b_st, c, b_mn_major=True, m=m, n=n, k=k, bias=bias, alpha=0.25, residual=res)
    t = (a.float() @ b.float().t()).bfloat16().float()
    t = (t + bias.float()).bfloat16().float()
    t = (0.25 * t).bfloat16().float()
    ref = res.float() + t
    assert _rel(c, ref) < 4e-3


def test_gelu_and_dgelu(cuda):
    """Forward: C = gelu(u), aux = gelu'(u) with u = bf16(bf16(acc) + bias).
    Backward: C = bf16(alpha * acc) * aux."""

    m, n, k = 512, 1024, 256
    a, b, _, b_st = _operands(m, n, k, 0, 1, cuda, 2)
    bias = (0.1 * torch.randn(n, device=cuda)).bfloat16()
    gp = torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
    g = torch.empty_like(gp)
    ops.gemm(a, b_st, g, b_mn_major=True, m=m, n=n, k=k, kind=_lib.EPI_BIAS_GELU, bias=bias, aux=gp)
    u = ((a.float() @ b.float().t()).bfloat16().float() + bias.float()).bfloat16().float()
    x = u.clone().requires_grad_(True)
    g_ref = torch.nn.functional.gelu(x, approximate="tanh")
    g_ref.sum().backward()
    assert _rel(g, g_ref.detach()) < 4e-3
    assert _rel(gp, x.grad) < 4e-3
    dy = torch.randn(m, 256, device=cuda).bfloat16()
    w = torch.randn(n, 256, device=cuda).bfloat16()  # [N, K] K-major
    du = torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
    ops.gemm(dy, w, du, m=m, n=n, k=256, kind=_lib.EPI_DGELU, alpha=0.5, aux=gp)
    up = (0.5 * (dy.float() @ w.float().t())).bfloat16().float()
    assert _rel(du, up * gp.float()) < 5e-3


@pytest.mark.parametrize("k", [64, 4096, 20000])
def test_f32_atomic_split_k(cuda, k):
    m, n = 768, 2304
    a, b, a_st, b_st = _operands(m, n, k, 1, 1, cuda, 3)
    c = torch.ones(m, n, device=cuda)
    ops.gemm(a_st, b_st, c, a_mn_major=True, b_mn_major=True, m=m, n=n, k=k,
             kind=_lib.EPI_F32_ATOMIC, alpha=0.5)
    ref = 1.0 + 0.5 * (a.float() @ b.float().t())
    assert _rel(c, ref) < 1e-5


@pytest.mark.parametrize("m,n,k", [(768, 2304, 64), (768, 2304, 4096), (768, 768, 131072),
                                   (3072, 768, 16384), (200, 136, 9000)])
def test_f32_splitk_ordered(cuda, m, n, k):
    """Weight-gradient epilogue with K split over CTAs: each split's partial
    goes to its own slab and the slabs are added in split order, so the result
    equals the fp32 product and repeats bit for bit."""

    a, b, a_st, b_st = _operands(m, n, k, 1, 1, cuda, 7)
    size = ops.gemm_workspace_size(m, n, k, _lib.EPI_F32_SPLITK)
    if k >= 4096 * 2:
        assert size >= 2 * m * n * 4  # K is split
    ws = ops.splitk_workspace(size, cuda)  # one workspace reused by every call below
    outs = []
    for _ in range(3):
        c = torch.ones(m, n, device=cuda)
        ops.gemm(a_st, b_st, c, a_mn_major=True, b_mn_major=True, m=m, n=n, k=k,
                 kind=_lib.EPI_F32_SPLITK, alpha=0.5, workspace=ws)
        outs.append(c)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = 1.0 + 0.5 * (a.float() @ b.float().t())
    # Each split accumulates up to 16,384 of K in the fp32 TMEM accumulator,
    # whose relative error grows with that length (measured ~1.1e-9 per unit
    # of K: 4.4e-6 at 4,096, 9.1e-6 at 8,192, 1.9e-5 at 16,384 against an fp64
    # product); the slabs themselves are added in plain fp32.
    splits = max(1, size // (m * n * 4))
    assert _rel(outs[0], ref) < max(1e-5, 1.5e-9 * k / splits)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_f32_store_and_accumulate(cuda):
    m, n, k = 600, 768, 512
    a, b, a_st, b_st = _operands(m, n, k, 1, 1, cuda, 4)
    c = torch.full((m, n), 2.0, device=cuda)
    ops.gemm(a_st, b_st, c, a_mn_major=True, b_mn_major=True, m=m, n=n, k=k, kind=_lib.EPI_F32,
             accumulate=True)
    ref = 2.0 + a.float() @ b.float().t()
    assert _rel(c, ref) < 1e-5
    ops.gemm(a_st, b_st, c, a_mn_major=True, b_mn_major=True, m=m, n=n, k=k, kind=_lib.EPI_F32)
    assert _rel(c, ref - 2.0) < 1e-5


def test_rejects_bad_arguments(cuda):
    a = torch.zeros(64, 60, device=cuda, dtype=torch.bfloat16)  # lda % 8 != 0
    b = torch.zeros(64, 60, device=cuda, dtype=torch.bfloat16)
    c = torch.zeros(64, 64, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(_lib.GptB200Error):
        ops.gemm(a, b, c, m=64, n=64, k=60)


def test_device_row_range(cuda):
    """M rows (range_dim 1) and K rows (range_dim 2) bounded by an int32
    {offset, count} pair that lives on the device: rows outside stay untouched."""

    g = torch.Generator().manual_seed(5)
    R, K, N = 1024, 192, 256
    a = torch.randn(R, K, generator=g).bfloat16().to(cuda)
    b = (0.1 * torch.randn(K, N, generator=g)).bfloat16().to(cuda)  # [K, N]: MN-major operand
    c = torch.full((R, N), 7.0, device=cuda).bfloat16()
    rr = torch.tensor([256, 384], dtype=torch.int32, device=cuda)
    ops.gemm(a, b, c, b_mn_major=True, m=R, n=N, k=K, row_range=rr, range_dim=1)
    ref = (a.float() @ b.float())
    assert _rel(c[256:640], ref[256:640]) < 4e-3
    assert torch.all(c[:256] == 7.0) and torch.all(c[640:] == 7.0)
    # K range: out[M, N] = A[K rows]^T B[K rows] with A, B MN-major [R, M] / [R, N]
    am = torch.randn(R, 128, generator=g).bfloat16().to(cuda)
    bm = torch.randn(R, N, generator=g).bfloat16().to(cuda)
    out = torch.zeros(128, N, device=cuda)
    kr = torch.tensor([128, 512], dtype=torch.int32, device=cuda)
    ops.gemm(am, bm, out, a_mn_major=True, b_mn_major=True, m=128, n=N, k=R,
             kind=_lib.EPI_F32_ATOMIC, row_range=kr, range_dim=2)
    want = am[128:640].float().t() @ bm[128:640].float()
    assert _rel(out, want) < 4e-3
    empty = torch.tensor([0, 0], dtype=torch.int32, device=cuda)
    c2 = torch.full((R, N), 3.0, device=cuda).bfloat16()
    ops.gemm(a, b, c2, b_mn_major=True, m=R, n=N, k=K, row_range=empty, range_dim=1)
    torch.cuda.synchronize()
    assert torch.all(c2 == 3.0) and ops.device_error() == 0
