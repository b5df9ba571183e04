"""The fp16 and fp8 e5m2 boundary formats on the sm_100a kernels: the
standalone quantiser, the LayerNorm prologue and backward reading each
format, the residual epilogue reading each format and writing fp16, and the
quantising epilogue writing e5m2. Each is compared with a plain PyTorch fp32
restatement of the same op; the quantisers also bit for bit with the host
restatement (same scale rule, same round-to-nearest-even cast).

Would fail if a kernel read or wrote a format with the wrong element size,
the wrong scale exponent (2^(e-15) for e5m2) or the wrong fp8 interpretation.
"""

import pytest
import torch
import torch.nn.functional as F

from elysium_wan_b200 import ops

pytestmark = pytest.mark.gpu

FORMATS = ["bf16", "fp16", "fp8_e4m3_b128", "fp8_e5m2_b128"]


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda")


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def bf(*shape, dev, scale=1.0):
    return (torch.randn(*shape, device=dev) * scale).to(torch.bfloat16)


def as_format(x, fmt):
    """(tensor, scales or None, its fp32 value) of bf16 x in a boundary format."""
    q8 = ops.q8_dtype(fmt)
    if q8 is not None:
        q, s = ops.quant_q8(x, q8)
        return q, s, ops.dequant_q8(q, s, torch.float32)
    if fmt == "fp16":
        h = x.to(torch.float16)
        return h, None, h.float()
    return x, None, x.float()


def test_e5m2_quantiser_matches_host_bitwise(cuda):
    torch.manual_seed(21)
    y = bf(64, 1024, dev=cuda, scale=30.0)
    y[3] = 0  # an all-zero row keeps scale 1
    for dt in (ops.E4M3, ops.E5M2):
        q, s = ops.quant_q8(y, dt)
        qc, sc = ops.quant_q8(y.cpu(), dt)
        assert q.dtype == dt
        assert torch.equal(s.cpu(), sc)
        assert torch.equal(q.cpu().view(torch.uint8), qc.view(torch.uint8))
        back = ops.dequant_q8(q, s, torch.float32)
        assert rel_err(back, y) < (0.07 if dt == ops.E5M2 else 0.04)
    # e5m2 scale rule: |x| / scale < 2^15 for every block
    q, s = ops.quant_q8(y, ops.E5M2)
    amax = y.float().view(64, 8, 128).abs().amax(-1)
    live = amax > 0
    assert torch.all(amax[live] / s[live] < 2.0 ** 15)
    assert torch.all(amax[live] / s[live] >= 2.0 ** 14)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("d", [512, 5120])
def test_layernorm_reads_every_format(cuda, fmt, d):
    torch.manual_seed(22)
    T = 260
    x = bf(T, d, dev=cuda, scale=3.0)
    xin, xs, xf = as_format(x, fmt)
    gamma, beta = torch.randn(d, device=cuda), torch.randn(d, device=cuda)
    y, mean, rstd = ops.layernorm_fwd(xin, xs, gamma, beta)
    assert rel_err(y, F.layer_norm(xf, (d,), gamma, beta, 1e-5)) < 8e-3
    xr = xf.clone().requires_grad_(True)
    g_, b_ = gamma.clone().requires_grad_(True), beta.clone().requires_grad_(True)
    dy, dres = bf(T, d, dev=cuda), bf(T, d, dev=cuda)
    F.layer_norm(xr, (d,), g_, b_, 1e-5).backward(dy.float())
    dg, db = torch.zeros(d, device=cuda), torch.zeros(d, device=cuda)
    dx = ops.layernorm_bwd(dy, xin, xs, mean, rstd, gamma, dres, dg, db, accumulate=True)
    assert rel_err(dx, xr.grad + dres.float()) < 1e-2
    assert rel_err(dg, g_.grad) < 1e-4
    assert rel_err(db, b_.grad) < 1e-4


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("N", [5120, 640])
def test_residual_epilogue_reads_every_format_and_writes_fp16(cuda, fmt, N):
    torch.manual_seed(23)
    M, K = 384, 256
    x, w = bf(M, K, dev=cuda), bf(N, K, dev=cuda, scale=0.05)
    b = torch.randn(N, device=cuda)
    acc = x.float() @ w.float().t() + b
    r, rs, rf = as_format(bf(M, N, dev=cuda), fmt)
    for out_dtype in (torch.bfloat16, torch.float16):
        y = ops.linear_fwd(x, w, b, epi="resid", resid=r, resid_scale=rs, out_dtype=out_dtype)
        assert y.dtype == out_dtype
        assert rel_err(y, acc + rf) < 8e-3


@pytest.mark.parametrize("fmt", FORMATS)
def test_quantising_epilogue_writes_e5m2(cuda, fmt):
    torch.manual_seed(24)
    M, N, K = 512, 1024, 384
    x, w = bf(M, K, dev=cuda), bf(N, K, dev=cuda, scale=0.05)
    b = torch.randn(N, device=cuda)
    r, rs, rf = as_format(bf(M, N, dev=cuda), fmt)
    want = x.float() @ w.float().t() + b + rf
    q, s = ops.linear_fwd(x, w, b, epi="resid_q8", resid=r, resid_scale=rs, q8=ops.E5M2)
    assert q.dtype == ops.E5M2
    assert rel_err(ops.dequant_q8(q, s, torch.float32), want) < 0.07
    # the block scales follow the e5m2 rule on the epilogue's own fp32 sums:
    # recomputing them from the fp32 reference agrees almost everywhere
    _, s_ref = ops.quant_q8(want.cpu(), ops.E5M2)
    assert (s.cpu() == s_ref).float().mean().item() > 0.95
