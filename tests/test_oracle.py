"""Pins the CPU oracle against the golden vectors made from the reference's own oracles.

The golden outputs come from tools/reference.py:72-79 (DiT and VAE shapes) and from Hugging
Face's T5Attention (T5 with relative-position bias); see tests/golden/make_golden.py.
"""

import hashlib

import numpy as np
import pytest

import oracle

# oracle (float64) vs the reference's float32 torch CPU outputs: the gap is torch's own fp32
# rounding (largest for T5, whose scores are unscaled), 2x tighter than the kernels' 1e-5 bar
TOL = 5e-6


def test_dit_self_interleaved(golden):
    c = golden.cases["dit_self"]
    B, N, H, D = c["B"], c["N"], c["H"], c["D"]
    qkv = golden("dit_self_qkv").reshape(-1)
    ref = golden("dit_self_out")
    out = np.zeros(B * N * H * D, dtype=np.float32)
    for b in range(B):  # app/models/dit.js:170-173
        r = b * N * 3 * H * D
        oracle.attention_ops(qkv, qkv, qkv, N, N, H, D, 3 * H * D, 3 * H * D, 3 * H * D,
                             qOff=r, kOff=r + H * D, vOff=r + 2 * H * D, oOff=b * N * H * D, out=out)
    assert oracle.max_rel(out, ref) < TOL
    assert oracle.rel_l2(out, ref) < TOL


def test_dit_self_config1(golden):
    import torch

    meta = golden.meta("dit_self_cfg1_out")
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(2, 256, 1728, generator=g)
    assert hashlib.sha256(qkv.numpy().astype("<f4").tobytes()).hexdigest() == meta["input_sha256"]
    ref = golden("dit_self_cfg1_out")
    for b in range(2):
        o = oracle.attention_heads(qkv[b, :, :576].numpy(), qkv[b, :, 576:1152].numpy(), qkv[b, :, 1152:].numpy(), 9)
        assert oracle.max_rel(o, ref[b]) < TOL


def test_dit_cross_ragged(golden):
    c = golden.cases["dit_cross"]
    q = golden("dit_cross_q")
    ref = golden("dit_cross_out")
    for b, L in enumerate(c["Ls"]):
        kv = golden(f"dit_cross_kv{b}")
        assert kv.shape == (L, 1152)
        qf = q[b].reshape(-1)
        kvf = kv.reshape(-1)
        out = oracle.attention_ops(qf, kvf, kvf, c["N"], L, 9, 64, 576, 1152, 1152, kOff=0, vOff=576)
        assert oracle.max_rel(out, ref[b]) < TOL


def test_ragged_equals_masked_padding(golden):
    # the reference's only evidence that true-length K/V equals masked padding (tools/check.js:130-131)
    a = golden("dit_cross_out")
    b = golden("dit_cross_out_masked")
    assert oracle.rel_l2(a, b) < 1e-6


@pytest.mark.parametrize("L", [1, 5, 37, 128])
def test_t5_bias_and_attention(golden, L):
    table = golden("t5_table")
    bias = oracle.position_bias(table, L, 12)
    np.testing.assert_array_equal(bias.reshape(12, L, L), golden(f"t5_L{L}_bias"))  # bit-exact
    q, k, v = (golden(f"t5_L{L}_{n}").reshape(-1) for n in "qkv")
    out = oracle.attention_ops(q, k, v, L, L, 12, 64, 768, 768, 768, scale=1.0, bias=bias)
    ref = golden(f"t5_L{L}_out")
    assert oracle.max_rel(out, ref) < TOL


@pytest.mark.parametrize("L", [1, 5, 37, 128])
def test_t5_torch_port(golden, L):
    """The torch fp32 T5 attention timed as the T5 call site's CPU baseline, against the goldens
    from transformers' T5Attention."""
    import torch

    bias = torch.from_numpy(golden(f"t5_L{L}_bias").reshape(12, L, L).copy())
    q, k, v = (torch.from_numpy(golden(f"t5_L{L}_{n}").reshape(L, 768).copy()) for n in "qkv")
    out = oracle.t5_sdpa_port(q, k, v, bias, 12).numpy()
    assert oracle.max_rel(out, golden(f"t5_L{L}_out")) < TOL


@pytest.mark.parametrize("nb,md", [(32, 128), (32, 64), (16, 32), (64, 256)])
def test_relative_bucket_matches_hf(golden, nb, md):
    ref = golden(f"bucket_{nb}_{md}").astype(np.int64)
    got = np.array([oracle.relative_bucket(r, nb, md) for r in range(-1000, 1001)])
    np.testing.assert_array_equal(got, ref)


def test_vae_single_head(golden):
    c = golden.cases["vae_small"]
    T = c["T"]
    q, k, v = (golden(f"vae_small_{n}").reshape(-1) for n in "qkv")
    out = oracle.attention_ops(q, k, v, T, T, 1, 512, 512, 512, 512)  # default scale 1/sqrt(512)
    assert oracle.max_rel(out, golden("vae_small_out")) < TOL


def test_known_answers():
    rng = np.random.default_rng(0)
    # L = 1: the output is V exactly
    q = rng.standard_normal(7 * 64).astype(np.float32)
    k = rng.standard_normal(64).astype(np.float32)
    v = rng.standard_normal(64).astype(np.float32)
    out = oracle.attention_ops(q, k, v, 7, 1, 1, 64, 64, 64, 64)
    np.testing.assert_allclose(out.reshape(7, 64), np.tile(v, (7, 1)), rtol=0, atol=0)
    # uniform scores (q = 0): the mean of V
    kk = rng.standard_normal(9 * 64).astype(np.float32)
    vv = rng.standard_normal(9 * 64).astype(np.float32)
    out = oracle.attention_ops(np.zeros(3 * 64, np.float32), kk, vv, 3, 9, 1, 64, 64, 64, 64)
    np.testing.assert_allclose(out.reshape(3, 64), np.tile(vv.reshape(9, 64).mean(0), (3, 1)), rtol=1e-6, atol=1e-6)
    # a dominant bias selects one key
    bias = np.full(3 * 9, -1e4, np.float32)
    bias[[4, 9 + 2, 18 + 8]] = 0
    out = oracle.attention_ops(np.zeros(3 * 64, np.float32), kk, vv, 3, 9, 1, 64, 64, 64, 64, bias=bias)
    np.testing.assert_allclose(out.reshape(3, 64), vv.reshape(9, 64)[[4, 2, 8]], rtol=1e-6, atol=1e-6)


def test_sdpa_port_matches_golden(golden):
    import torch

    qkv = torch.from_numpy(golden("dit_self_qkv").copy())
    B, N = qkv.shape[:2]
    v3 = qkv.view(B, N, 3, 576)
    out = oracle.sdpa_port(v3[:, :, 0], v3[:, :, 1], v3[:, :, 2], 9)
    assert oracle.max_rel(out.numpy(), golden("dit_self_out")) < 1e-6


def test_context_preparation(golden):
    """oracle.prepare_context / oracle.linear against the reference's own linear (ctx_proj, then
    each block's cross_attn.kv) and the cross attention on block 1's K/V."""
    from conftest import ctxprep_inputs

    x = ctxprep_inputs()
    sha = lambda a: hashlib.sha256(np.asarray(a, dtype="<f4").tobytes()).hexdigest()
    assert sha(x["flat"]) == golden.meta("ctxprep_p")["input_sha256"]
    assert sha(x["q_flat"]) == golden.meta("ctxprep_cross_out")["q_sha256"]
    p, kvs = oracle.prepare_context(x["ctx"], x["wp"], x["bp"], x["wkv"], x["bkv"])
    assert oracle.max_rel(p, golden("ctxprep_p")) <= TOL
    for i, kv in enumerate(kvs):
        assert oracle.max_rel(kv, golden(f"ctxprep_kv{i}")) <= TOL
    # the flat-array operator with offsets and strides gives the same
    L = x["L"]
    y = oracle.linear(np.concatenate([np.zeros(8, np.float32), x["ctx"].reshape(-1)]), x["wp"], L, 576, 768,
                      bias=x["bp"], x_off=8, ldy=600)
    yy = y[np.arange(L)[:, None] * 600 + np.arange(576)[None, :]]
    assert oracle.max_rel(yy, golden("ctxprep_p")) <= TOL
    kv1 = kvs[1]
    out = oracle.attention_heads(x["q"], kv1[:, :576], kv1[:, 576:], 9)
    assert oracle.max_rel(out, golden("ctxprep_cross_out")) <= TOL


def test_vae_attention_block(golden):
    """oracle.vae_attention_block (GroupNorm, q/k/v, attention, projection, residual) against the
    reference's linear and attention around torch's group_norm."""
    from conftest import vae_block_inputs

    x = vae_block_inputs()
    assert hashlib.sha256(np.asarray(x["flat"], dtype="<f4").tobytes()).hexdigest() == \
        golden.meta("vae_block_out")["input_sha256"]
    got = oracle.vae_attention_block(x["x"], x["gamma"], x["beta"], x["wq"], x["bq"], x["wk"], x["bk"], x["wv"],
                                     x["bv"], x["wo"], x["bo"])
    assert oracle.max_rel(got, golden("vae_block_out")) <= TOL


def test_dit_block_projections(golden):
    """oracle.gated_residual around oracle.attention_heads against the reference's dit_forward
    lines for the gated self-attention projection and the ungated cross projection."""
    from conftest import dit_proj_inputs

    x = dit_proj_inputs()
    assert hashlib.sha256(np.asarray(x["flat"], dtype="<f4").tobytes()).hexdigest() == \
        golden.meta("dit_proj_x1")["input_sha256"]
    B, N, D = x["B"], x["N"], x["D"]
    x1, x2 = [], []
    for b in range(B):
        qkv = x["qkv"][b]
        a = oracle.attention_heads(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], 9)
        x1.append(oracle.gated_residual(x["x0"][b], a, x["wp"], N, D, D, bias=x["bp"], gate=x["mod"], g_off=2 * D))
        x2.append(oracle.gated_residual(x1[-1], x["c"][b], x["wc"], N, D, D, bias=x["bc"]))
    assert oracle.max_rel(np.stack(x1), golden("dit_proj_x1")) <= TOL
    assert oracle.max_rel(np.stack(x2), golden("dit_proj_x2")) <= TOL


def test_dit_block(golden):
    """oracle.dit_block (LayerNorm with adaLN modulation, q/k/v, self attention, gated projection,
    LayerNorm, cross attention, projection, modulated LayerNorm, fc1 + GELU(tanh), gated fc2)
    against the reference's dit_forward pieces on one whole block."""
    from conftest import dit_block_inputs

    x = dit_block_inputs()
    assert hashlib.sha256(np.asarray(x["flat"], dtype="<f4").tobytes()).hexdigest() == \
        golden.meta("dit_block_x1")["input_sha256"]
    outs = [oracle.dit_block(x["x0"][b], x["mod"], x["w"], x["kv"][b]) for b in range(x["B"])]
    for i in range(3):
        assert oracle.max_rel(np.stack([o[i] for o in outs]), golden(f"dit_block_x{i + 1}")) <= TOL


def test_layernorm_and_activations():
    """oracle.layernorm / oracle.activation against torch's layer_norm and GELU / SiLU."""
    import torch
    import torch.nn.functional as F

    rng = np.random.default_rng(4)
    x = rng.standard_normal((7, 50)) * 3 + 1
    mod = rng.standard_normal(200)
    t = F.layer_norm(torch.from_numpy(x), (50,), eps=1e-6).numpy()
    assert np.abs(oracle.layernorm(x) - t).max() < 1e-12
    want = t * (1 + mod[100:150]) + mod[20:70]
    assert np.abs(oracle.layernorm(x, mod, 20, 100) - want).max() < 1e-12
    xt = torch.from_numpy(x)
    for act, ref in [("gelu", F.gelu(xt)), ("gelu_tanh", F.gelu(xt, approximate="tanh")), ("silu", F.silu(xt))]:
        assert np.abs(oracle.activation(x, act) - ref.numpy()).max() < 1e-12, act
