"""Hot ops of the framework, one function per op, no autograd.

CUDA tensors run the hand-written sm_100a kernels of ``elysium_wan_b200._C``
(tcgen05 GEMM with fused epilogues, attention, LayerNorm, cross-entropy,
embedding, AdamW, fp8 boundary quantisation). CPU tensors run a plain fp32
torch restatement of the same math; that path serves the CPU/gloo plumbing
configuration and is the oracle of the kernel tests.

Reference ops being replaced (all PyTorch library calls in the reference):
``F.linear``/``SplitLinear`` (src/wantrain/model/wgrad.py:193-265),
``nn.LayerNorm`` and SDPA (src/wantrain/model/gpt.py:346-418),
``F.cross_entropy`` (gpt.py:556), ``torch.optim.AdamW``
(src/wantrain/runtime/optim.py:45), the fp8 boundary (src/wantrain/model/fp8.py).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ._ext import ext, launch_count  # noqa: F401

E4M3 = torch.float8_e4m3fn
E5M2 = torch.float8_e5m2
# fp8 boundary formats: torch dtype, exponent offset of the 1x128 block scale
# (scale = 2^(e - offset) with amax = f 2^e, f in [0.5, 1), so |x| / scale <
# 2^offset stays inside the format: 256 <= 448 for e4m3, 32768 <= 57344 for
# e5m2) and the largest finite value.
Q8_FORMATS = {"fp8_e4m3_b128": (E4M3, 8, 448.0), "fp8_e5m2_b128": (E5M2, 15, 57344.0)}
_Q8_BY_DTYPE = {dt: (off, mx) for dt, off, mx in Q8_FORMATS.values()}


def q8_dtype(boundary: str):
    """The fp8 dtype of an fp8 boundary recipe, else None."""
    f = Q8_FORMATS.get(boundary)
    return f[0] if f else None


def act_dtype(boundary: str, cuda: bool):
    """dtype of a dense boundary activation: fp16 for the fp16 recipe and bf16
    otherwise on the GPU; fp32 (holding the recipe's rounded values) on the
    host path. Gradients stay in the compute dtype whatever the recipe."""
    if not cuda:
        return torch.float32
    return torch.float16 if boundary == "fp16" else torch.bfloat16

# Epilogue kinds of the GEMM (mirrors csrc/gemm.h).
EPI_BF16, EPI_GELU, EPI_RESID, EPI_RESID_Q8, EPI_ACC_F32, EPI_DGELU, EPI_F32 = range(7)


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


# ----------------------------------------------------------------------------- fp8 boundary
def q8_block_scale_ref(amax: torch.Tensor, dtype=E4M3) -> torch.Tensor:
    """Power-of-two scale 2^(e - offset) with amax = f * 2^e, f in [0.5, 1); 1
    where amax == 0 (offset 8 for e4m3, 15 for e5m2)."""
    off, _ = _Q8_BY_DTYPE[dtype]
    _, e = torch.frexp(amax)
    s = torch.ldexp(torch.ones_like(amax), e - off)
    return torch.where(amax > 0, s, torch.ones_like(amax))


def e4m3_block_scale_ref(amax: torch.Tensor) -> torch.Tensor:
    return q8_block_scale_ref(amax, E4M3)


def quant_q8(x: torch.Tensor, dtype=E4M3):
    """1x128 block-scaled fp8 (e4m3 or e5m2): returns (q [T,d], scale [T,d/128] fp32)."""
    T, d = x.shape
    assert d % 128 == 0, "fp8 boundary needs d_model % 128 == 0"
    if _cuda(x):
        q = torch.empty((T, d), dtype=dtype, device=x.device)
        s = torch.empty((T, d // 128), dtype=torch.float32, device=x.device)
        ext().quant_q8(x.to(torch.bfloat16).contiguous(), q, s)
        return q, s
    _, mx = _Q8_BY_DTYPE[dtype]
    xf = x.float().view(T, d // 128, 128)
    s = q8_block_scale_ref(xf.abs().amax(dim=2), dtype)
    q = (xf / s[..., None]).clamp(-mx, mx).to(dtype).view(T, d)
    return q, s


def quant_e4m3(x: torch.Tensor):
    return quant_q8(x, E4M3)


def dequant_q8(q: torch.Tensor, s: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    T, d = q.shape
    if _cuda(q) and dtype == torch.bfloat16:
        y = torch.empty((T, d), dtype=torch.bfloat16, device=q.device)
        ext().dequant_q8(q.contiguous(), s.contiguous(), y)
        return y
    return (q.float().view(T, d // 128, 128) * s[..., None]).view(T, d).to(dtype)


dequant_e4m3 = dequant_q8


# ----------------------------------------------------------------------------- GEMM
def gemm(a, b, out, epi=EPI_BF16, *, a_mn=False, b_mn=False, bias=None, resid=None,
         resid_scale=None, aux=None, scale_out=None, beta=0.0, bn=0):
    """out[m, n] (epi)= sum_k A[m, k] B[n, k] on the tcgen05 kernel (CUDA only).

    A is [M, K] (a_mn=False) or stored transposed [K, M]; B is [N, K] or [K, N].
    """
    ext().gemm(a, a_mn, b, b_mn, out, epi, bias, resid, resid_scale, aux, scale_out, float(beta),
               int(bn))
    return out


def _resid_value(resid, resid_scale):
    if resid.dtype in _Q8_BY_DTYPE:
        return dequant_q8(resid, resid_scale, torch.float32)
    return resid.float()


def linear_fwd(x, w, bias=None, *, epi="none", resid=None, resid_scale=None, out=None,
               q8=E4M3, out_dtype=torch.bfloat16):
    """Y = X W^T (+ b) with a fused epilogue.

    epi: "none" -> Y; "gelu" -> (gelu(U), U) with U = XW^T+b kept for the
    backward; "resid" -> resid + XW^T + b (out_dtype bf16 or fp16 on the GPU);
    "resid_q8" -> fp8 (q8: e4m3 or e5m2) + 1x128 scales of that.
    """
    T = x.shape[0]
    N = w.shape[0]
    if _cuda(x):
        dev = x.device
        if epi == "none":
            out = out if out is not None else torch.empty((T, N), dtype=torch.bfloat16, device=dev)
            return gemm(x, w, out, EPI_BF16, bias=bias)
        if epi == "gelu":
            u = torch.empty((T, N), dtype=torch.bfloat16, device=dev)
            g = out if out is not None else torch.empty((T, N), dtype=torch.bfloat16, device=dev)
            gemm(x, w, g, EPI_GELU, bias=bias, aux=u)
            return g, u
        if epi == "resid":
            out = out if out is not None else torch.empty((T, N), dtype=out_dtype, device=dev)
            return gemm(x, w, out, EPI_RESID, bias=bias, resid=resid, resid_scale=resid_scale)
        if epi == "resid_q8":
            q = torch.empty((T, N), dtype=q8, device=dev)
            s = torch.empty((T, N // 128), dtype=torch.float32, device=dev)
            gemm(x, w, q, EPI_RESID_Q8, bias=bias, resid=resid, resid_scale=resid_scale,
                 scale_out=s)
            return q, s
        if epi == "f32":
            out = out if out is not None else torch.empty((T, N), dtype=torch.float32, device=dev)
            return gemm(x, w, out, EPI_F32, bias=bias)
        raise ValueError(epi)
    # CPU restatement (fp32)
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    if epi == "none" or epi == "f32":
        return y.to(x.dtype) if epi == "none" else y
    if epi == "gelu":
        return F.gelu(y), y
    if epi == "resid":
        return _resid_value(resid, resid_scale) + y
    if epi == "resid_q8":
        return quant_q8(_resid_value(resid, resid_scale) + y, q8)
    raise ValueError(epi)


def linear_dx(dy, w, *, gelu_u=None, out=None):
    """dX = dY W (B pass); with gelu_u, returns dY W * gelu'(u) (fc1's input grad of GELU)."""
    T = dy.shape[0]
    K = w.shape[1]
    if _cuda(dy):
        out = out if out is not None else torch.empty((T, K), dtype=torch.bfloat16, device=dy.device)
        if gelu_u is not None:
            return gemm(dy, w, out, EPI_DGELU, b_mn=True, aux=gelu_u)
        return gemm(dy, w, out, EPI_BF16, b_mn=True)
    g = dy.float() @ w.float()
    if gelu_u is not None:
        u = gelu_u.float()
        cdf = 0.5 * (1.0 + torch.erf(u * (1.0 / math.sqrt(2.0))))
        pdf = torch.exp(-0.5 * u * u) / math.sqrt(2.0 * math.pi)
        g = g * (cdf + u * pdf)
    return g


def linear_dw_pair(dy1, x1, dy2, x2, grad, accumulate: bool):
    """grad (+)= dY1^T X1 + dY2^T X2 as ONE reduction over the two microbatches'
    tokens (K = T1 + T2), folded into grad once: half the fp32 read-modify-write
    of two separate folds. The sum order differs from two folds, so a run pairs
    its weight gradients only as its recipe declares (`w_pair`)."""
    if _cuda(dy1):
        ext().gemm_pair(dy1, x1, dy2, x2, grad, 1.0 if accumulate else 0.0, 0)
        return grad
    g = torch.cat([dy1.float(), dy2.float()]).t() @ torch.cat([x1.float(), x2.float()])
    if accumulate:
        grad.add_(g)
    else:
        grad.copy_(g)
    return grad


def linear_dw(dy, x, grad, accumulate: bool):
    """grad (+)= dY^T X (W pass): the deferred weight gradient, folded in call order."""
    if _cuda(dy):
        return gemm(dy, x, grad, EPI_ACC_F32, a_mn=True, b_mn=True,
                    beta=1.0 if accumulate else 0.0)
    g = dy.float().t() @ x.float()
    if accumulate:
        grad.add_(g)
    else:
        grad.copy_(g)
    return grad


def colsum(x, grad, accumulate: bool):
    """grad (+)= sum over rows of x (bias gradients), fixed order."""
    if _cuda(x):
        part = torch.empty((ext().colsum_chunks(x.shape[0]), x.shape[1]), dtype=torch.float32,
                           device=x.device)
        ext().colsum(x, part, grad, accumulate)
        return grad
    s = x.float().sum(0)
    if accumulate:
        grad.add_(s)
    else:
        grad.copy_(s)
    return grad


# ----------------------------------------------------------------------------- LayerNorm
def layernorm_fwd(x, x_scale, gamma, beta, eps=1e-5):
    """Returns (y bf16/fp32, mean, rstd). x may be e4m3 with 1x128 scales
    (dequant prologue). beta None = RMSNorm (mean 0, no shift)."""
    T, d = x.shape
    if _cuda(x):
        y = torch.empty((T, d), dtype=torch.bfloat16, device=x.device)
        mean = torch.empty(T, dtype=torch.float32, device=x.device)
        rstd = torch.empty(T, dtype=torch.float32, device=x.device)
        ext().layernorm_fwd(x, x_scale, gamma, beta, y, mean, rstd, eps)
        return y, mean, rstd
    xf = _resid_value(x, x_scale)
    if beta is None:
        mean = torch.zeros(T, dtype=torch.float32)
        rstd = torch.rsqrt((xf * xf).mean(dim=1) + eps)
        return xf * rstd[:, None] * gamma, mean, rstd
    mean = xf.mean(dim=1)
    var = ((xf - mean[:, None]) ** 2).mean(dim=1)
    rstd = torch.rsqrt(var + eps)
    y = (xf - mean[:, None]) * rstd[:, None] * gamma + beta
    return y, mean, rstd


def layernorm_bwd(dy, x, x_scale, mean, rstd, gamma, dres, dgamma, dbeta, accumulate: bool):
    """dx (+ dres); dgamma/dbeta (+)= their row sums (fixed order). dbeta None
    = RMSNorm."""
    T, d = x.shape
    rms = dbeta is None
    if _cuda(x):
        dx = torch.empty((T, d), dtype=torch.bfloat16, device=x.device)
        chunks = ext().layernorm_bwd_chunks(T)
        pg = torch.empty((chunks, d), dtype=torch.float32, device=x.device)
        pb = None if rms else torch.empty((chunks, d), dtype=torch.float32, device=x.device)
        ext().layernorm_bwd(dy, x, x_scale, mean, rstd, gamma, dres, dx, pg, pb, dgamma, dbeta,
                            accumulate)
        return dx
    xf = _resid_value(x, x_scale)
    xh = (xf - mean[:, None]) * rstd[:, None]
    dyf = dy.float()
    g = dyf * gamma
    centre = 0.0 if rms else g.mean(1, keepdim=True)
    dx = rstd[:, None] * (g - centre - xh * (g * xh).mean(1, keepdim=True))
    if dres is not None:
        dx = dx + dres.float()
    pg = (dyf * xh).sum(0)
    if accumulate:
        dgamma.add_(pg)
    else:
        dgamma.copy_(pg)
    if not rms:
        pb = dyf.sum(0)
        if accumulate:
            dbeta.add_(pb)
        else:
            dbeta.copy_(pb)
    return dx


# ----------------------------------------------------------------------------- attention
def _split_qkv(qkv, B, S, H, hd, Hkv):
    """(q, k, v) as fp32 [B, heads, S, hd] from the fused [q | k | v] rows."""
    d, dkv = H * hd, Hkv * hd
    x = qkv.float().view(B, S, d + 2 * dkv)
    q = x[..., :d].reshape(B, S, H, hd).transpose(1, 2)
    k = x[..., d:d + dkv].reshape(B, S, Hkv, hd).transpose(1, 2)
    v = x[..., d + dkv:].reshape(B, S, Hkv, hd).transpose(1, 2)
    return q, k, v


def attention_fwd(qkv, B, S, H, hd, Hkv=None):
    """Causal attention on the fused buffer [B*S, (H + 2*Hkv)*hd] (q | k | v;
    Hkv < H is grouped-query attention) -> (o [B*S, H*hd], lse base 2)."""
    d = H * hd
    Hkv = Hkv or H
    scale = 1.0 / math.sqrt(hd)
    if _cuda(qkv):
        o = torch.empty((B * S, d), dtype=torch.bfloat16, device=qkv.device)
        lse = torch.empty((B, H, S), dtype=torch.float32, device=qkv.device)
        ext().attention_fwd(qkv, o, lse, B, S, H, hd, scale, Hkv)
        return o, lse
    q, k, v = _split_qkv(qkv, B, S, H, hd, Hkv)
    rep = H // Hkv
    k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
    att = (q @ k.transpose(-2, -1)) * scale
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
    att = att.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(att, dim=-1) * (1.0 / math.log(2.0))
    o = (torch.softmax(att, dim=-1) @ v).transpose(1, 2).reshape(B * S, d)
    return o, lse


def attention_bwd(qkv, o, dout, lse, B, S, H, hd, Hkv=None):
    """Gradient of causal attention w.r.t. the fused qkv buffer (same layout).
    With grouped-query attention a kv head's gradient sums its group's query
    heads in head order."""
    d = H * hd
    Hkv = Hkv or H
    scale = 1.0 / math.sqrt(hd)
    if _cuda(qkv):
        dqkv = torch.empty_like(qkv)
        D = torch.empty((B, H, S), dtype=torch.float32, device=qkv.device)
        ext().attention_bwd(qkv, o, dout, lse, D, dqkv, B, S, H, hd, scale, Hkv)
        return dqkv
    q, k, v = _split_qkv(qkv, B, S, H, hd, Hkv)
    rep = H // Hkv
    kr, vr = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
    do = dout.float().view(B, S, H, hd).transpose(1, 2)
    att = (q @ kr.transpose(-2, -1)) * scale
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
    p = torch.softmax(att.masked_fill(mask, float("-inf")), dim=-1)
    dv = p.transpose(-2, -1) @ do
    dp = do @ vr.transpose(-2, -1)
    ds = p * (dp - (dp * p).sum(-1, keepdim=True))
    dq = ds @ kr * scale
    dk = ds.transpose(-2, -1) @ q * scale
    dk = dk.view(B, Hkv, rep, S, hd).sum(2)
    dv = dv.view(B, Hkv, rep, S, hd).sum(2)
    rows = lambda t: t.transpose(1, 2).reshape(B * S, -1)  # noqa: E731
    return torch.cat([rows(dq), rows(dk), rows(dv)], dim=1)


# ----------------------------------------------------------------------------- Llama family
_ROPE_TABLES: dict = {}


def rope_tables(S, hd, theta, device):
    """(cos, sin) fp32 [S, hd/2] of p * theta^(-2i/hd), computed once in fp64
    on the host so every device type uses the same table."""
    key = (S, hd, float(theta), str(device))
    t = _ROPE_TABLES.get(key)
    if t is None:
        inv = 1.0 / (float(theta) ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
        ang = torch.outer(torch.arange(S, dtype=torch.float64), inv)
        t = (torch.cos(ang).float().to(device).contiguous(),
             torch.sin(ang).float().to(device).contiguous())
        _ROPE_TABLES[key] = t
    return t


def rope(x, S, ncols, hd, theta, inverse=False):
    """Rotate adjacent column pairs of columns [0, ncols) of each row in place
    (q heads then k heads); row r is at position r % S. inverse rotates back
    (the backward)."""
    cos, sin = rope_tables(S, hd, theta, x.device)
    if _cuda(x):
        ext().rope(x, S, ncols, hd, cos, sin, bool(inverse))
        return x
    T = x.shape[0]
    v = x[:, :ncols].reshape(T, ncols // hd, hd // 2, 2)
    pos = torch.arange(T) % S
    c, s_ = cos[pos][:, None, :], sin[pos][:, None, :]
    if inverse:
        s_ = -s_
    x1, x2 = v[..., 0].clone(), v[..., 1].clone()
    v[..., 0] = x1 * c - x2 * s_
    v[..., 1] = x1 * s_ + x2 * c
    return x


def swiglu_fwd(gu):
    """h = silu(gu[:, :f]) * gu[:, f:]."""
    T, f2 = gu.shape
    f = f2 // 2
    if _cuda(gu):
        h = torch.empty((T, f), dtype=torch.bfloat16, device=gu.device)
        ext().swiglu_fwd(gu, h)
        return h
    g, u = gu[:, :f].float(), gu[:, f:].float()
    return g * torch.sigmoid(g) * u


def swiglu_bwd(dh, gu):
    """d(gu) from dh: [dh * u * silu'(g) | dh * silu(g)]."""
    T, f2 = gu.shape
    f = f2 // 2
    if _cuda(gu):
        dgu = torch.empty_like(gu)
        ext().swiglu_bwd(dh, gu, dgu)
        return dgu
    g, u, d = gu[:, :f].float(), gu[:, f:].float(), dh.float()
    s = torch.sigmoid(g)
    return torch.cat([d * u * s * (1 + g * (1 - s)), d * g * s], dim=1)


def residual_add(x, y):
    """x + y rounded to x's dtype, y first rounded to x's dtype (the block's
    `x + mlp(h).to(x.dtype)`)."""
    return x + y.to(x.dtype)


# ----------------------------------------------------------------------------- cross-entropy
def cross_entropy(logits, V, targets, grad_scale, want_grad=True, ld_grad=None):
    """Mean CE over rows of fp32 logits; returns (loss scalar tensor, dlogits or None).

    dlogits = (softmax - onehot) * grad_scale, bf16 with row length ld_grad
    (a multiple of 8 so it can feed TMA), pad columns zero.
    """
    T = logits.shape[0]
    if _cuda(logits):
        rows = torch.empty(T, dtype=torch.float32, device=logits.device)
        dl = None
        if want_grad:
            ldg = ld_grad or ((V + 7) // 8) * 8
            dl = torch.empty((T, ldg), dtype=torch.bfloat16, device=logits.device)
        ext().cross_entropy(logits, V, targets, rows, dl, grad_scale)
        loss = torch.empty(1, dtype=torch.float32, device=logits.device)
        ext().mean_reduce(rows, loss)
        return loss[0], dl
    lg = logits[:, :V].float()
    loss = F.cross_entropy(lg, targets)
    dl = None
    if want_grad:
        p = torch.softmax(lg, dim=-1)
        p[torch.arange(T), targets] -= 1.0
        dl = p * grad_scale
    return loss, dl


def head_ce(h, w, targets, V, grad_scale):
    """Fused head logits + mean cross-entropy on the GPU: (loss scalar tensor,
    dlogits bf16 [T][ld], ld = V rounded up to 8, pad columns zero).

    The logits GEMM's epilogue keeps, per row and 256-wide vocabulary tile,
    the tile max and the sum of exp(x - max) (and the target's logit), and
    writes exp(x - tile max) in fp16 where the gradient will go; a second
    kernel combines the tiles' partials in a fixed order into the row's
    log-sum-exp and loss and turns those values into the bf16 gradient in
    place. The fp32 logits are never stored (reference op: logits.float()
    then F.cross_entropy, src/wantrain/model/gpt.py:410-418,556-557)."""
    T = h.shape[0]
    ld = (V + 7) // 8 * 8
    nt = (V + 255) // 256
    dev = h.device
    buf = torch.empty((T, ld), dtype=torch.bfloat16, device=dev)
    part = torch.empty((T, nt, 2), dtype=torch.float32, device=dev)
    tgt_logit = torch.empty(T, dtype=torch.float32, device=dev)
    targets = targets.reshape(-1).contiguous()
    ext().gemm_lse(h, w, buf[:, :V], V, targets, part, tgt_logit)
    rows = torch.empty(T, dtype=torch.float32, device=dev)
    ext().ce_lse_finalize(part, tgt_logit, targets, V, buf, grad_scale, rows)
    loss = torch.empty(1, dtype=torch.float32, device=dev)
    ext().mean_reduce(rows, loss)
    return loss[0], buf


# ----------------------------------------------------------------------------- embedding
def embed_fwd(idx, wte, wpe, S, q8=None, out_dtype=torch.bfloat16):
    """x = wte[idx] (+ wpe[pos] when learned positions) in a boundary format:
    (fp8, scales) when q8 names an fp8 dtype, else a dense out_dtype tensor
    (bf16 / fp16 on the GPU)."""
    T = idx.numel()
    d = wte.shape[1]
    if _cuda(idx):
        if q8 is not None:
            q = torch.empty((T, d), dtype=q8, device=idx.device)
            s = torch.empty((T, d // 128), dtype=torch.float32, device=idx.device)
            ext().embed_fwd(idx, wte, wpe, S, q, s)
            return q, s
        x = torch.empty((T, d), dtype=out_dtype, device=idx.device)
        ext().embed_fwd(idx, wte, wpe, S, x, None)
        return x
    flat = idx.reshape(-1)
    x = wte[flat]
    if wpe is not None:
        x = x + wpe[torch.arange(T) % S]
    if q8 is not None:
        return quant_q8(x, q8)
    return x.to(out_dtype)


def embed_bwd(idx, dx, S, dwte, dwpe):
    """dwte[tok] += rows of dx in position order; dwpe[s] += rows in batch order."""
    if _cuda(idx):
        order = torch.empty(idx.numel(), dtype=torch.int32, device=idx.device)
        ext().embed_bwd(idx.reshape(-1), dx, S, order, dwte, dwpe)
        return
    flat = idx.reshape(-1)
    T = flat.numel()
    dxf = dx.float()
    dwte.index_add_(0, flat, dxf)
    if dwpe is not None:
        dwpe.add_(dxf.view(T // S, S, -1).sum(0))


# ----------------------------------------------------------------------------- AdamW
def adamw(p, m, v, g, p_bf16, lr, b1, b2, eps, wd, step):
    """One AdamW step on flat fp32 state (torch AdamW update order)."""
    if _cuda(p):
        ext().adamw(p, m, v, g, p_bf16, lr, b1, b2, eps, wd, step)
        return
    bc1 = 1.0 - b1 ** step
    bc2 = 1.0 - b2 ** step
    m.mul_(b1).add_(g, alpha=1.0 - b1)
    v.mul_(b2).addcmul_(g, g, value=1.0 - b2)
    if wd != 0.0:
        p.mul_(1.0 - lr * wd)
    denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
    p.addcdiv_(m, denom, value=-lr / bc1)
    if p_bf16 is not None:
        p_bf16.copy_(p)
