"""CPU restatement of the reference's attention operator.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): never imported by the product.

Three entry points:
  attention_ops   -- the operator surface of app/gpu/ops.js:103-149 on flat float32 arrays,
                     computed in float64: per head h, S = Q_h K_h^T * scale (+ bias[h])
                     (app/gpu/kernels.js:34, app/gpu/kernels.js:262-264), row softmax
                     (app/gpu/kernels.js:46-62), O_h = P V_h, written with row stride H*D at
                     oOff (app/gpu/ops.js:104-105,114-115,139-144).
  attention_heads -- the same on [Lq, H*D]-shaped arrays (no offsets), float64.
  sdpa_port       -- the reference's own CPU oracle restated: tools/reference.py:72-79
                     (view -> transpose -> torch scaled_dot_product_attention in float32 ->
                     back), used as the timed CPU baseline.
"""

from __future__ import annotations

import math

import numpy as np


def _gather(buf, off, rows, ld, h, D):
    """Rows of head h: buf[off + i*ld + h*D + d] (app/gpu/ops.js:104-105)."""
    idx = off + np.arange(rows, dtype=np.int64)[:, None] * ld + h * D + np.arange(D, dtype=np.int64)[None, :]
    return np.asarray(buf, dtype=np.float32)[idx].astype(np.float64)


def _softmax_rows(s):
    """Row softmax: max pass, exp/sum pass, normalise (app/gpu/kernels.js:53-62)."""
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    return e / e.sum(axis=-1, keepdims=True)


def attention_ops(q, k, v, Lq, Lk, H, D, ldq, ldk, ldv, qOff=0, kOff=0, vOff=0, oOff=0,
                  scale=None, bias=None, out=None):
    """ops.attention (app/gpu/ops.js:109) on flat arrays. Returns the flat float32 `out`.

    scale defaults to 1/sqrt(D) (app/gpu/ops.js:109). bias is the flat [H, Lq, Lk] additive
    score bias (app/gpu/ops.js:106). If out is None a zero buffer of Lq*H*D floats is made,
    like gpu.empty([Lq, H*D]) (app/gpu/ops.js:110).
    """
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = np.zeros(oOff + Lq * H * D, dtype=np.float32)
    b = None if bias is None else np.asarray(bias, dtype=np.float32).reshape(-1)
    for h in range(H):
        Q = _gather(q, qOff, Lq, ldq, h, D)
        K = _gather(k, kOff, Lk, ldk, h, D)
        V = _gather(v, vOff, Lk, ldv, h, D)
        s = (Q @ K.T) * np.float64(np.float32(scale))
        if b is not None:
            s = s + b[h * Lq * Lk:(h + 1) * Lq * Lk].reshape(Lq, Lk).astype(np.float64)
        O = _softmax_rows(s) @ V
        idx = oOff + np.arange(Lq, dtype=np.int64)[:, None] * (H * D) + h * D + np.arange(D, dtype=np.int64)[None, :]
        out[idx] = O.astype(np.float32)
    return out


def attention_heads(q, k, v, H, scale=None, bias=None):
    """q [Lq, H*D], k/v [Lk, H*D] (any float dtype) -> [Lq, H*D] float64."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    Lq, C = q.shape
    Lk = k.shape[0]
    D = C // H
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    Qh = q.reshape(Lq, H, D).transpose(1, 0, 2)
    Kh = k.reshape(Lk, H, D).transpose(1, 0, 2)
    Vh = v.reshape(Lk, H, D).transpose(1, 0, 2)
    s = np.einsum("hid,hjd->hij", Qh, Kh) * np.float64(np.float32(scale))
    if bias is not None:
        s = s + np.asarray(bias, dtype=np.float64).reshape(H, Lq, Lk)
    O = np.einsum("hij,hjd->hid", _softmax_rows(s), Vh)
    return O.transpose(1, 0, 2).reshape(Lq, C)


def sdpa_port(q, k, v, heads, mask=None):
    """tools/reference.py:72-79 restated: q [B, N, C], k/v [B, M, C] torch float32 tensors.

    Splits C into `heads` heads, runs torch's scaled_dot_product_attention (default scale
    1/sqrt(C/heads)) with an optional boolean key mask [B, M], and merges the heads back.
    """
    import torch
    import torch.nn.functional as F

    B, N, C = q.shape
    M = k.shape[1]
    qh = q.view(B, N, heads, C // heads).transpose(1, 2)
    kh = k.view(B, M, heads, C // heads).transpose(1, 2)
    vh = v.view(B, M, heads, C // heads).transpose(1, 2)
    am = None if mask is None else mask.bool()[:, None, None, :]
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=am)
    return o.transpose(1, 2).reshape(B, N, C)


def t5_sdpa_port(q, k, v, bias, heads):
    """T5 encoder self-attention in torch float32 on the CPU (the timed CPU baseline of the T5 call
    site, app/models/t5.js:80): q, k, v [L, C] torch float32, bias [heads, L, L] (positionBias,
    app/models/t5.js:55-65). The arithmetic of transformers' T5Attention.forward (an unvendored
    dependency of tools/reference.py:129, version 5.5.0 in this image, models/t5/modeling_t5.py):
    scores = Q K^T with NO 1/sqrt(d) scaling (:308), plus the position bias (:327-328), softmax in
    float (:331), times V (:334); heads split and merged as C = heads x d."""
    import torch.nn.functional as F

    L, C = q.shape
    M = k.shape[0]
    qh = q.view(L, heads, C // heads).transpose(0, 1)
    kh = k.view(M, heads, C // heads).transpose(0, 1)
    vh = v.view(M, heads, C // heads).transpose(0, 1)
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=bias.view(heads, L, M), scale=1.0)
    return o.transpose(0, 1).reshape(L, C)


def rel_l2(got, ref):
    """Relative L2 error, the reference's parity metric (tools/check.js:31-44)."""
    g = np.asarray(got, dtype=np.float64).reshape(-1)
    r = np.asarray(ref, dtype=np.float64).reshape(-1)
    return float(np.sqrt(((g - r) ** 2).sum() / max((r ** 2).sum(), 1e-30)))


def max_rel(got, ref):
    """max|got - ref| / max|ref| over one output tensor (normwise max-relative error)."""
    g = np.asarray(got, dtype=np.float64).reshape(-1)
    r = np.asarray(ref, dtype=np.float64).reshape(-1)
    return float(np.abs(g - r).max() / max(np.abs(r).max(), 1e-30))
