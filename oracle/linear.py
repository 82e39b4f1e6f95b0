"""CPU restatement of the reference's linear layer and the cross-attention K/V preparation.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): never imported by the product.

  linear           -- ops.linear (app/gpu/ops.js:35-43): y = x @ W^T (+ bias) with W in the
                      reference's [N, K] layout, on flat float32 arrays with row strides and
                      element offsets, computed in float64.
  prepare_context  -- DiT.prepareContext (app/models/dit.js:137-144): p = ctx_proj(ctx), then
                      each block's kv projection of p ([L, 1152]: K at columns 0..575, V at
                      576..1151), as tools/reference.py:92,99 computes them.
  groupnorm        -- ops.groupnorm (app/gpu/ops.js:82-92, app/gpu/kernels.js:117-162).
  vae_attention_block -- VAE.attention (app/models/vae.js:77-94): GroupNorm, q/k/v, attention,
                      output projection, residual.
  layernorm        -- ops.layernorm (app/gpu/ops.js:71-79, app/gpu/kernels.js:87-114), with the
                      optional adaLN modulation LN(x) * (1 + scale) + shift.
  activation       -- ops.linear's act (app/gpu/gemm.js:28-36): gelu (erf form), gelu_tanh, silu.
  dit_block        -- one DiT block (app/models/dit.js:161-194; tools/reference.py:96-102).
  gated_residual   -- ops.linear with { out, resid: true, gate, gOff } (app/gpu/gemm.js:10,135):
                      out = out + gate[gOff + n] * (x W^T + bias), the DiT blocks' projections
                      (app/models/dit.js:175,187,193; tools/reference.py:98,100,102).
"""

from __future__ import annotations

import numpy as np


def linear(x, w, M, N, K, bias=None, ldx=None, ldw=None, ldy=None, x_off=0, y_off=0, out=None):
    """Flat-array ops.linear; returns the flat float32 `out` (allocated [M, N] when None)."""
    ldx = K if ldx is None else ldx
    ldw = K if ldw is None else ldw
    ldy = N if ldy is None else ldy
    xa = np.asarray(x, dtype=np.float32).reshape(-1)
    wa = np.asarray(w, dtype=np.float32).reshape(-1)
    rows = x_off + np.arange(M, dtype=np.int64)[:, None] * ldx + np.arange(K, dtype=np.int64)[None, :]
    wrows = np.arange(N, dtype=np.int64)[:, None] * ldw + np.arange(K, dtype=np.int64)[None, :]
    y = xa[rows].astype(np.float64) @ wa[wrows].astype(np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float64).reshape(-1)[:N][None, :]
    if out is None:
        out = np.zeros(y_off + (M - 1) * ldy + N if M else 1, dtype=np.float32)
    if M:
        idx = y_off + np.arange(M, dtype=np.int64)[:, None] * ldy + np.arange(N, dtype=np.int64)[None, :]
        out[idx] = y.astype(np.float32)
    return out


def prepare_context(ctx, w_proj, b_proj, w_kv, b_kv):
    """ctx [L, Kc]; w_proj [D, Kc], b_proj [D]; w_kv / b_kv lists of [2D, D] / [2D] per block.
    Returns (p [L, D], [kv_b [L, 2D] for each block]) in float32."""
    ctx = np.asarray(ctx, dtype=np.float64)
    p = ctx @ np.asarray(w_proj, dtype=np.float64).T + np.asarray(b_proj, dtype=np.float64)[None, :]
    kvs = [(p @ np.asarray(w, dtype=np.float64).T + np.asarray(b, dtype=np.float64)[None, :]).astype(np.float32)
           for w, b in zip(w_kv, b_kv)]
    return p.astype(np.float32), kvs


def groupnorm(x, gamma, beta, groups, eps=1e-6, silu=False):
    """ops.groupnorm (app/gpu/ops.js:82-92; app/gpu/kernels.js:117-162) of one NHWC image
    x [pixels, C]: per group of C/groups channels the mean, then the variance around it (biased),
    y = (x - mean) * (var + eps)^-1/2 * gamma[c] + beta[c], then SiLU if asked. float64."""
    x = np.asarray(x, dtype=np.float64)
    P, Cn = x.shape
    cg = Cn // groups
    xg = x.reshape(P, groups, cg)
    mean = xg.mean(axis=(0, 2), keepdims=True)
    var = ((xg - mean) ** 2).mean(axis=(0, 2), keepdims=True)
    y = ((xg - mean) / np.sqrt(var + eps)).reshape(P, Cn) * np.asarray(gamma, np.float64) + np.asarray(beta, np.float64)
    if silu:
        y = y / (1.0 + np.exp(-y))
    return y


def vae_attention_block(x, gn_gamma, gn_beta, wq, bq, wk, bk, wv, bv, wo, bo, groups=32, eps=1e-6):
    """VAE.attention (app/models/vae.js:77-94) on one image x [hw, C]: GroupNorm (no SiLU), q/k/v
    projections, single-head attention with scale 1/sqrt(C) (app/gpu/ops.js:109), output
    projection, residual add. float64 throughout; returns float32 [hw, C]."""
    x64 = np.asarray(x, dtype=np.float64)
    n = groupnorm(x64, gn_gamma, gn_beta, groups, eps)
    f = lambda a, w, b: a @ np.asarray(w, np.float64).T + np.asarray(b, np.float64)
    q, k, v = f(n, wq, bq), f(n, wk, bk), f(n, wv, bv)
    s = q @ k.T / np.sqrt(q.shape[1])
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return (x64 + f(p @ v, wo, bo)).astype(np.float32)


def gated_residual(out, x, w, M, N, K, bias=None, gate=None, g_off=0):
    """out [M, N] + gate[g_off + n] * (x [M, K] @ W^T + bias) in float64, returned as float32
    [M, N]; gate None is the ungated residual (app/gpu/gemm.js:135 stores C[ci] = C[ci] + r)."""
    y = np.asarray(x, np.float64).reshape(M, K) @ np.asarray(w, np.float64).reshape(N, K).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64).reshape(-1)[:N][None, :]
    if gate is not None:
        y = y * np.asarray(gate, np.float64).reshape(-1)[g_off:g_off + N][None, :]
    return (np.asarray(out, np.float64).reshape(M, N) + y).astype(np.float32)


def layernorm(x, mod=None, shift_off=0, scale_off=0, eps=1e-6):
    """ops.layernorm (app/gpu/ops.js:71-79; app/gpu/kernels.js:101-113) of x [rows, cols]: per row
    the mean, then the variance around it (biased), (x - mean) / sqrt(var + eps), then
    * (1 + mod[scale_off + c]) + mod[shift_off + c] when mod is given. float64."""
    x = np.asarray(x, dtype=np.float64)
    cols = x.shape[1]
    mean = x.mean(axis=1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=1, keepdims=True)
    y = (x - mean) / np.sqrt(var + eps)
    if mod is not None:
        m = np.asarray(mod, dtype=np.float64).reshape(-1)
        y = y * (1.0 + m[scale_off:scale_off + cols]) + m[shift_off:shift_off + cols]
    return y


def activation(x, act):
    """ops.linear's act (app/gpu/gemm.js:28-36) in float64: "gelu" = 0.5 x (1 + erf(x / sqrt 2)),
    "gelu_tanh" = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), "silu" = x / (1 + e^-x)."""
    from math import erf, pi, sqrt

    x = np.asarray(x, dtype=np.float64)
    if act == "gelu":
        return 0.5 * x * (1.0 + np.vectorize(erf)(x / sqrt(2.0)))
    if act == "gelu_tanh":
        return 0.5 * x * (1.0 + np.tanh(sqrt(2.0 / pi) * (x + 0.044715 * x ** 3)))
    if act == "silu":
        return x / (1.0 + np.exp(-x))
    raise ValueError(act)


def dit_block(x, mod, w, kv, heads=9):
    """One DiT block on one image (app/models/dit.js:161-194; tools/reference.py:96-102), float64:
    x [N, D]; mod the step's modulation vector [6D] (shift, scale, gate for the attention, then for
    the MLP); w dict of [out, in] weights and biases qkv, proj, q, cproj, fc1, fc2; kv [L, 2D] the
    prompt's cross-attention K|V. Returns (x after self attention, after cross attention, after
    the MLP) as float32 [N, D]."""
    from .attention import attention_heads

    x = np.asarray(x, dtype=np.float64)
    D = x.shape[1]
    m = np.asarray(mod, dtype=np.float64).reshape(-1)
    f = lambda a, nm: a @ np.asarray(w[nm], np.float64).T + np.asarray(w["b" + nm], np.float64)
    qkv = f(layernorm(x, m, 0, D), "qkv")
    x1 = x + m[2 * D:3 * D] * f(attention_heads(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], heads), "proj")
    kv = np.asarray(kv, dtype=np.float64)
    c = attention_heads(f(layernorm(x1), "q"), kv[:, :D], kv[:, D:], heads)
    x2 = x1 + f(c, "cproj")
    h = activation(f(layernorm(x2, m, 3 * D, 4 * D), "fc1"), "gelu_tanh")
    x3 = x2 + m[5 * D:6 * D] * f(h, "fc2")
    return tuple(t.astype(np.float32) for t in (x1, x2, x3))
