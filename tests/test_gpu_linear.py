"""The linear operator (ops.linear, app/gpu/ops.js:35-43) and the cross-attention K/V preparation
(app/models/dit.js:137-144) through the C ABI, against the float64 oracle and the golden
vectors of the reference's own linear (tools/reference.py:67-68,92,99).

FP32 bar: max|got - ref| / max|ref| <= 1e-5 and rel-L2 <= 1e-5 per output tensor.
"""

import numpy as np
import pytest

import oracle
from conftest import ctxprep_inputs

pytestmark = pytest.mark.gpu
TOL = 1e-5


def dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32)).reshape(-1)).cuda()


def host(t):
    return t.detach().cpu().numpy().reshape(-1)


def assert_close(got, ref, tol=TOL):
    mr, rl = oracle.max_rel(got, ref), oracle.rel_l2(got, ref)
    assert mr <= tol and rl <= tol, f"max_rel={mr:.3e} rel_l2={rl:.3e} (tol {tol})"


def test_context_preparation_golden(gpu, golden):
    """ctx_proj, then the blocks' kv projections as ONE product with the stacked weights, then a
    cross attention that reads block 1's K/V in place (ld = 3*1152) -- against the reference."""
    import supra_attn

    x = ctxprep_inputs()
    L, nb = x["L"], len(x["wkv"])
    ctx, wp, bp = dev(x["ctx"]), dev(x["wp"]), dev(x["bp"])
    wkv = dev(np.concatenate(x["wkv"], 0))   # [3*1152, 576]
    bkv = dev(np.concatenate(x["bkv"], 0))
    p = supra_attn.linear(gpu, ctx, wp, N=576, K=768, bias=bp)
    kv = supra_attn.linear(gpu, p, wkv, N=nb * 1152, K=576, bias=bkv)  # records behind p (hazard-ordered)
    q = dev(x["q"])
    o = supra_attn.attention(gpu, q=q, k=kv, v=kv, Lq=48, Lk=L, H=9, D=64, ldq=576, ldk=nb * 1152, ldv=nb * 1152,
                             kOff=1152, vOff=1152 + 576)
    got_p = gpu.read(p).reshape(L, 576)
    got_kv = gpu.read(kv).reshape(L, nb * 1152)
    assert_close(got_p, golden("ctxprep_p"))
    for i in range(nb):
        assert_close(got_kv[:, 1152 * i:1152 * (i + 1)], golden(f"ctxprep_kv{i}"))
    assert_close(gpu.read(o), golden("ctxprep_cross_out"))
    for t in (p, kv, o):
        t.release()


@pytest.mark.parametrize(
    "M,N,K,bias",
    [(1, 1, 1, False), (1, 1152, 576, True), (37, 576, 768, True), (130, 129, 33, True), (257, 1000, 64, False),
     (128, 128, 16, True), (300, 16128, 576, True), (1000, 7, 3, True),
     # the 128-column tile form (one 288-tile wave), and the 64-column form chosen for the DiT
     # blocks' N = 576 products (576 tiles against 320); the smaller cases above take the 64-column
     # form too (one wave either way, the narrower tile cheaper)
     (2048, 2304, 64, True), (2048, 2301, 33, False), (8192, 576, 64, True), (8192, 570, 33, False)],
)
def test_linear_shapes(gpu, M, N, K, bias):
    import supra_attn

    rng = np.random.default_rng(M * 31 + N * 7 + K)
    xa = rng.standard_normal(M * K).astype(np.float32)
    wa = (rng.standard_normal(N * K) / np.sqrt(K)).astype(np.float32)
    ba = rng.standard_normal(N).astype(np.float32) if bias else None
    xd, wd, bd = dev(xa), dev(wa), (dev(ba) if bias else None)  # alive until the flush runs
    y = supra_attn.linear(gpu, xd, wd, N=N, K=K, bias=bd)
    got = gpu.read(y)
    y.release()
    assert_close(got, oracle.linear(xa, wa, M, N, K, bias=ba))


@pytest.mark.parametrize("aligned", [True, False])
def test_linear_strides_and_offsets(gpu, aligned):
    """Row strides and element offsets on x and y; misaligned ones take the 4-byte copy path."""
    import supra_attn

    rng = np.random.default_rng(5 + aligned)
    M, N, K = 70, 90, 52 if aligned else 51
    ldx, ldw, ldy, xo, yo = (60, 56, 100, 8, 12) if aligned else (61, 53, 97, 3, 5)
    xa = rng.standard_normal(xo + M * ldx).astype(np.float32)
    wa = rng.standard_normal(N * ldw).astype(np.float32)
    ba = rng.standard_normal(N).astype(np.float32)
    out = dev(np.full(yo + M * ldy, 7.0))
    xd, wd, bd = dev(xa), dev(wa), dev(ba)
    supra_attn.linear(gpu, xd, wd, M=M, N=N, K=K, bias=bd, out=out, ldx=ldx, ldw=ldw, ldy=ldy, xOff=xo, yOff=yo)
    gpu.sync()
    got = host(out)
    ref = oracle.linear(xa, wa, M, N, K, bias=ba, ldx=ldx, ldw=ldw, ldy=ldy, x_off=xo, y_off=yo,
                        out=np.full(yo + M * ldy, 7.0, dtype=np.float32))
    assert np.all(got[:yo] == 7.0)
    gap = np.ones(ldy, bool)
    gap[:N] = False
    assert np.all(got[yo:].reshape(M, ldy)[:, gap] == 7.0), "wrote between rows"
    assert_close(got, ref)


def test_linear_batch_one_launch(gpu):
    """Many recorded problems (different M, N, K, some with bias) go out as one launch."""
    import supra_attn

    rng = np.random.default_rng(9)
    shapes = [(int(rng.integers(1, 300)), int(rng.integers(1, 700)), int(rng.integers(1, 200))) for _ in range(40)]
    xs = [rng.standard_normal(m * k).astype(np.float32) for m, n, k in shapes]
    ws = [rng.standard_normal(n * k).astype(np.float32) for m, n, k in shapes]
    bs = [rng.standard_normal(n).astype(np.float32) for m, n, k in shapes]
    n0 = gpu.launch_count()
    gpu.profile(True)
    gpu.profile_reset()
    ops = [(dev(xs[i]), dev(ws[i]), dev(bs[i])) for i in range(len(shapes))]  # alive until the flush runs
    outs = [supra_attn.linear(gpu, ops[i][0], ops[i][1], N=n, K=k, bias=ops[i][2])
            for i, (m, n, k) in enumerate(shapes)]
    gpu.flush()
    gpu.sync()
    names = [r["name"] for r in gpu.profile_report()]
    gpu.profile_reset()
    gpu.profile(False)
    assert names == ["linear_fp32_bias"], names
    groups = len({k % 4 == 0 for m, n, k in shapes})  # 16-byte rows or not: one launch form each
    assert gpu.launch_count() - n0 == 2 * groups  # staging + linear per group
    for i, (m, n, k) in enumerate(shapes):
        assert_close(gpu.read(outs[i]), oracle.linear(xs[i], ws[i], m, n, k, bias=bs[i]))
        outs[i].release()


# ---- VAE mid-block attention, fused (app/models/vae.js:77-94) --------------------------------------
def vae_block(gpu, x, p, nimg, hw, C, stacked):
    """GroupNorm folded into the stacked q/k/v product, attention reading q/k/v in place, and the
    residual folded into the output projection: three launches (plus the statistics)."""
    import supra_attn

    qkv = supra_attn.linear(gpu, x, stacked["w"], N=3 * C, K=C, bias=stacked["b"],
                            groupnorm=dict(gamma=p["gamma"], beta=p["beta"], groups=32, rows_per_image=hw))
    a = gpu.empty([nimg * hw, C])
    for i in range(nimg):
        r = i * hw
        supra_attn.attention(gpu, q=qkv, k=qkv, v=qkv, Lq=hw, Lk=hw, H=1, D=C, ldq=3 * C, ldk=3 * C, ldv=3 * C,
                             qOff=r * 3 * C, kOff=r * 3 * C + C, vOff=r * 3 * C + 2 * C, oOff=r * C, out=a)
    out = supra_attn.linear(gpu, a, p["wo"], N=C, K=C, bias=p["bo"], resid=x)
    return out, (qkv, a)


def stack_qkv(x):
    return {"w": dev(np.concatenate([x["wq"], x["wk"], x["wv"]], 0)), "b": dev(np.concatenate([x["bq"], x["bk"], x["bv"]]))}


def test_vae_block_golden(gpu, golden):
    from conftest import vae_block_inputs

    x = vae_block_inputs()
    p = {k: dev(x[k]) for k in ("gamma", "beta", "wo", "bo")}
    xd = dev(x["x"])
    out, tmp = vae_block(gpu, xd, p, 1, x["hw"], x["C"], stack_qkv(x))
    assert_close(gpu.read(out), golden("vae_block_out"))
    for t in (out,) + tmp:
        t.release()


def test_vae_block_full_size_batch(gpu):
    """Two 32x32 images (1024 tokens x 512 channels) in one flush: per-image GroupNorm statistics,
    against the float64 oracle."""
    rng = np.random.default_rng(77)
    hw, C, nimg = 1024, 512, 2
    x = rng.standard_normal((nimg * hw, C)).astype(np.float32)
    prm = {"gamma": (1 + 0.1 * rng.standard_normal(C)).astype(np.float32),
           "beta": (0.1 * rng.standard_normal(C)).astype(np.float32)}
    for nm in "qkvo":
        prm["w" + nm] = (rng.standard_normal((C, C)) / np.sqrt(C)).astype(np.float32)
        prm["b" + nm] = (0.1 * rng.standard_normal(C)).astype(np.float32)
    p = {k: dev(prm[k]) for k in ("gamma", "beta", "wo", "bo")}
    xd = dev(x)
    out, tmp = vae_block(gpu, xd, p, nimg, hw, C, stack_qkv(prm))
    got = gpu.read(out).reshape(nimg, hw, C)
    for i in range(nimg):
        ref = oracle.vae_attention_block(x[i * hw:(i + 1) * hw], prm["gamma"], prm["beta"], prm["wq"], prm["bq"],
                                         prm["wk"], prm["bk"], prm["wv"], prm["bv"], prm["wo"], prm["bo"])
        assert_close(got[i], ref)
    for t in (out,) + tmp:
        t.release()


def test_linear_groupnorm_silu_and_residual(gpu):
    """The two fusions on their own, with SiLU, against oracle.groupnorm + oracle.linear."""
    import supra_attn

    rng = np.random.default_rng(88)
    M, K, N, rows = 3 * 40, 96, 70, 40
    x = rng.standard_normal((M, K)).astype(np.float32)
    gamma, beta = rng.standard_normal(K).astype(np.float32), rng.standard_normal(K).astype(np.float32)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    r = rng.standard_normal((M, N + 3)).astype(np.float32)
    xd, gd, bd, wd, rd = dev(x), dev(gamma), dev(beta), dev(w), dev(r)
    y = supra_attn.linear(gpu, xd, wd, N=N, K=K, resid=rd, ldr=N + 3,
                          groupnorm=dict(gamma=gd, beta=bd, groups=8, rows_per_image=rows, silu=True))
    got = gpu.read(y).reshape(M, N)
    for i in range(M // rows):
        sl = slice(i * rows, (i + 1) * rows)
        n = oracle.groupnorm(x[sl], gamma, beta, 8, silu=True).astype(np.float32)
        ref = oracle.linear(n, w, rows, N, K).reshape(rows, N) + r[sl, :N]
        assert_close(got[sl], ref)
    y.release()


# ---- DiT block projections around the attention (app/models/dit.js:161-187) -----------------------
def test_dit_block_projections_golden(gpu, golden):
    """The residual stream x updated in place, as the reference's DiT block does: self attention
    into a, x += g1 * proj(a) with g1 = mod[2D:3D] (gated), then x += cproj(c) (ungated); both
    recorded behind the attention and flushed together, against the reference's outputs."""
    import supra_attn
    from conftest import dit_proj_inputs

    x = dit_proj_inputs()
    B, N, D = x["B"], x["N"], x["D"]
    xs = dev(x["x0"])
    qkv, mod, c = dev(x["qkv"]), dev(x["mod"]), dev(x["c"])
    wp, bp, wc, bc = dev(x["wp"]), dev(x["bp"]), dev(x["wc"]), dev(x["bc"])
    a = gpu.empty([B * N, D])
    for b in range(B):
        r = b * N * 3 * D
        supra_attn.attention(gpu, q=qkv, k=qkv, v=qkv, Lq=N, Lk=N, H=9, D=64, ldq=3 * D, ldk=3 * D, ldv=3 * D,
                             qOff=r, kOff=r + D, vOff=r + 2 * D, oOff=b * N * D, out=a)
    supra_attn.linear(gpu, a, wp, N=D, K=D, bias=bp, out=xs, resid=True, gate=mod, gOff=2 * D)
    gpu.sync()
    assert_close(host(xs), golden("dit_proj_x1"))
    supra_attn.linear(gpu, c, wc, N=D, K=D, bias=bc, out=xs, resid=True)
    gpu.sync()
    assert_close(host(xs), golden("dit_proj_x2"))
    a.release()


@pytest.mark.parametrize("aligned", [True, False])
def test_linear_gated_in_place_strided(gpu, aligned):
    """In-place gated residual on a strided y with offsets (rows of ldy, first at yOff): only the
    M x N block changes, each element to y + gate[gOff + n] * (x W^T + b)."""
    import supra_attn

    rng = np.random.default_rng(31 + aligned)
    M, N, K = 150, 200, 64 if aligned else 61
    ldy, yo, go = (208, 16, 40) if aligned else (203, 5, 7)
    y0 = rng.standard_normal(yo + M * ldy).astype(np.float32)
    xa = rng.standard_normal((M, K)).astype(np.float32)
    wa = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    ba = rng.standard_normal(N).astype(np.float32)
    ga = rng.standard_normal(go + N + 3).astype(np.float32)
    yd, xd, wd, bd, gd = dev(y0), dev(xa), dev(wa), dev(ba), dev(ga)
    supra_attn.linear(gpu, xd, wd, M=M, N=N, K=K, bias=bd, out=yd, ldy=ldy, yOff=yo, resid=True, gate=gd, gOff=go)
    gpu.sync()
    got = host(yd)
    idx = yo + np.arange(M)[:, None] * ldy + np.arange(N)[None, :]
    keep = np.ones(got.size, bool)
    keep[idx.reshape(-1)] = False
    np.testing.assert_array_equal(got[keep], y0[keep])
    ref = oracle.gated_residual(y0[idx], xa, wa, M, N, K, bias=ba, gate=ga, g_off=go)
    assert_close(got[idx], ref)


def test_linear_in_place_is_ordered_after_readers(gpu):
    """x is read by an attention recorded before the in-place update of x: the update waits for
    it (write-after-read hazard), and a reader recorded after sees the updated x."""
    import supra_attn

    rng = np.random.default_rng(12)
    L, D = 80, 576
    xa = rng.standard_normal(L * D).astype(np.float32)
    ca = rng.standard_normal(L * D).astype(np.float32)
    wa = (rng.standard_normal((D, D)) / np.sqrt(D)).astype(np.float32)
    xd, cd, wd = dev(xa), dev(ca), dev(wa)
    o1 = supra_attn.attention(gpu, q=xd, k=xd, v=xd, Lq=L, Lk=L, H=9, D=64, ldq=D, ldk=D, ldv=D)
    supra_attn.linear(gpu, cd, wd, N=D, K=D, out=xd, resid=True)
    o2 = supra_attn.attention(gpu, q=xd, k=xd, v=xd, Lq=L, Lk=L, H=9, D=64, ldq=D, ldk=D, ldv=D)
    gpu.sync()
    x1 = oracle.gated_residual(xa, ca, wa, L, D, D).reshape(-1)
    assert_close(gpu.read(o1), oracle.attention_ops(xa, xa, xa, L, L, 9, 64, D, D, D))
    assert_close(host(xd), x1)
    assert_close(gpu.read(o2), oracle.attention_ops(x1, x1, x1, L, L, 9, 64, D, D, D))
    for t in (o1, o2):
        t.release()


# ---- one whole DiT block (app/models/dit.js:161-194) -----------------------------------------------
def dit_block(gpu, x, mod, w, kvs, Ls, B, N, D=576):
    """The reference's block with its LayerNorms folded into the products that follow them and its
    residual updates done in place: 8 recorded products and attentions, no other op."""
    import supra_attn

    qkv = supra_attn.linear(gpu, x, w["qkv"], N=3 * D, K=D, bias=w["bqkv"],
                            layernorm=dict(mod=mod, shiftOff=0, scaleOff=D))
    a = gpu.empty([B * N, D])
    for b in range(B):
        r = b * N * 3 * D
        supra_attn.attention(gpu, q=qkv, k=qkv, v=qkv, Lq=N, Lk=N, H=9, D=64, ldq=3 * D, ldk=3 * D, ldv=3 * D,
                             qOff=r, kOff=r + D, vOff=r + 2 * D, oOff=b * N * D, out=a)
    supra_attn.linear(gpu, a, w["proj"], N=D, K=D, bias=w["bproj"], out=x, resid=True, gate=mod, gOff=2 * D)
    q = supra_attn.linear(gpu, x, w["q"], N=D, K=D, bias=w["bq"], layernorm={})
    c = gpu.empty([B * N, D])
    for b in range(B):
        supra_attn.attention(gpu, q=q, k=kvs[b], v=kvs[b], Lq=N, Lk=Ls[b], H=9, D=64, ldq=D, ldk=2 * D, ldv=2 * D,
                             qOff=b * N * D, kOff=0, vOff=D, oOff=b * N * D, out=c)
    supra_attn.linear(gpu, c, w["cproj"], N=D, K=D, bias=w["bcproj"], out=x, resid=True)
    f = supra_attn.linear(gpu, x, w["fc1"], N=4 * D, K=D, bias=w["bfc1"], act="gelu_tanh",
                          layernorm=dict(mod=mod, shiftOff=3 * D, scaleOff=4 * D))
    supra_attn.linear(gpu, f, w["fc2"], N=D, K=4 * D, bias=w["bfc2"], out=x, resid=True, gate=mod, gOff=5 * D)
    return (qkv, a, q, c, f)


def test_dit_block_golden(gpu, golden):
    """One whole DiT block through the library against the reference's dit_forward pieces."""
    from conftest import dit_block_inputs

    x = dit_block_inputs()
    B, N, D = x["B"], x["N"], x["D"]
    w = {k: dev(v) for k, v in x["w"].items()}
    mod, kvs = dev(x["mod"]), [dev(t) for t in x["kv"]]
    xs = dev(x["x0"])
    gpu.profile(True)
    gpu.profile_reset()
    tmp = dit_block(gpu, xs, mod, w, kvs, x["Ls"], B, N)
    gpu.sync()
    names = {r["name"] for r in gpu.profile_report()}
    gpu.profile_reset()
    gpu.profile(False)
    assert {"layernorm_stats", "linear_fp32_bias"} <= names, names
    assert_close(host(xs), golden("dit_block_x3"))
    for t in tmp:
        t.release()


def test_dit_block_full_size(gpu):
    """Four images of 256 tokens (the DiT step's shape, ragged prompts up to 128 tokens) against the
    float64 oracle, each residual stage checked."""
    rng = np.random.default_rng(1234)
    B, N, D = 4, 256, 576
    Ls = [1, 37, 128, 77]
    wn = {}
    for nm, (o, i) in [("qkv", (3 * D, D)), ("proj", (D, D)), ("q", (D, D)), ("cproj", (D, D)),
                       ("fc1", (4 * D, D)), ("fc2", (D, 4 * D))]:
        wn[nm] = (rng.standard_normal((o, i)) / np.sqrt(i)).astype(np.float32)
        wn["b" + nm] = (0.1 * rng.standard_normal(o)).astype(np.float32)
    x0 = rng.standard_normal((B, N, D)).astype(np.float32)
    modn = (0.5 * rng.standard_normal(6 * D)).astype(np.float32)
    kvn = [rng.standard_normal((L, 2 * D)).astype(np.float32) for L in Ls]
    w = {k: dev(v) for k, v in wn.items()}
    mod, kvs = dev(modn), [dev(t) for t in kvn]
    xs = dev(x0)
    tmp = dit_block(gpu, xs, mod, w, kvs, Ls, B, N)
    gpu.sync()  # the last product is recorded until a flush; x is read outside the library
    got = host(xs).reshape(B, N, D)
    for b in range(B):
        assert_close(got[b], oracle.dit_block(x0[b], modn, wn, kvn[b])[2])
    for t in tmp:
        t.release()


@pytest.mark.parametrize("act", ["gelu", "gelu_tanh", "silu"])
def test_linear_activations(gpu, act):
    import supra_attn

    rng = np.random.default_rng(len(act))
    M, N, K = 140, 300, 72
    xa = (2 * rng.standard_normal((M, K))).astype(np.float32)
    wa = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    ba = rng.standard_normal(N).astype(np.float32)
    xd, wd, bd = dev(xa), dev(wa), dev(ba)
    y = supra_attn.linear(gpu, xd, wd, N=N, K=K, bias=bd, act=act)
    got = gpu.read(y).reshape(M, N)
    y.release()
    ref = oracle.activation(oracle.linear(xa, wa, M, N, K, bias=ba).reshape(M, N).astype(np.float64), act)
    assert_close(got, ref)


@pytest.mark.parametrize("K", [61, 576])
def test_linear_layernorm(gpu, K):
    """Plain and modulated LayerNorm prologues on rows that do not fill a tile, K ragged or not."""
    import supra_attn

    rng = np.random.default_rng(K)
    M, N = 333, 150
    xa = (rng.standard_normal((M, K)) * 2 + 0.5).astype(np.float32)
    wa = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    modn = rng.standard_normal(3 * K + 5).astype(np.float32)
    xd, wd, md = dev(xa), dev(wa), dev(modn)
    y1 = supra_attn.linear(gpu, xd, wd, N=N, K=K, layernorm={})
    y2 = supra_attn.linear(gpu, xd, wd, N=N, K=K, layernorm=dict(mod=md, shiftOff=5, scaleOff=2 * K + 3))
    got1, got2 = gpu.read(y1).reshape(M, N), gpu.read(y2).reshape(M, N)
    w64 = wa.astype(np.float64)
    assert_close(got1, oracle.layernorm(xa) @ w64.T)
    assert_close(got2, oracle.layernorm(xa, modn, 5, 2 * K + 3) @ w64.T)
    for t in (y1, y2):
        t.release()
