"""The linear operator on the tensor cores (variants "tf32x3" and "tf32", K >= 32) through the C
ABI: tf32x3 (every operand split into a TF32 part and its remainder, three products) is held to
the FP32 bar, max_rel and rel-L2 <= 1e-5; tf32 to rel-L2 <= 2e-3 (max <= 5e-3). Against the
float64 oracle and the reference's golden vectors."""

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL = {"tf32x3": (1e-5, 1e-5), "tf32": (2e-3, 5e-3)}  # (rel-L2, normwise max)


def dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32)).reshape(-1)).cuda()


def host(t):
    return t.detach().cpu().numpy().reshape(-1)


def check(got, ref, variant):
    rl_tol, mr_tol = TOL[variant]
    mr, rl = oracle.max_rel(got, ref), oracle.rel_l2(got, ref)
    assert rl <= rl_tol and mr <= mr_tol, f"{variant}: max_rel={mr:.3e} rel_l2={rl:.3e}"


def names_of(gpu):
    return {r["name"] for r in gpu.profile_report()}


@pytest.mark.parametrize("variant", ["tf32x3", "tf32"])
@pytest.mark.parametrize(
    "M,N,K,bias",
    [(1, 1, 32, False), (1, 1152, 576, True), (37, 576, 768, True), (130, 129, 33, True), (257, 1000, 64, False),
     (300, 16128, 576, True), (1000, 7, 35, True), (128, 128, 2304, True), (513, 300, 1000, False)],
)
def test_shapes(gpu, variant, M, N, K, bias):
    import supra_attn

    rng = np.random.default_rng(M * 31 + N * 7 + K)
    xa = rng.standard_normal(M * K).astype(np.float32)
    wa = (rng.standard_normal(N * K) / np.sqrt(K)).astype(np.float32)
    ba = rng.standard_normal(N).astype(np.float32) if bias else None
    xd, wd, bd = dev(xa), dev(wa), (dev(ba) if bias else None)
    gpu.profile(True)
    gpu.profile_reset()
    y = supra_attn.linear(gpu, xd, wd, N=N, K=K, bias=bd, variant=variant)
    got = gpu.read(y)
    names = names_of(gpu)
    gpu.profile_reset()
    gpu.profile(False)
    y.release()
    assert f"linear_tc_{variant}" in names, names
    check(got, oracle.linear(xa, wa, M, N, K, bias=ba), variant)


def test_shallow_products_run_the_ffma_kernel(gpu):
    """K < 32 (one k-block would be mostly padding): the FFMA kernel, at the FP32 bar."""
    import supra_attn

    rng = np.random.default_rng(3)
    M, N, K = 70, 50, 7
    xa, wa = rng.standard_normal(M * K).astype(np.float32), rng.standard_normal(N * K).astype(np.float32)
    xd, wd = dev(xa), dev(wa)
    gpu.profile(True)
    gpu.profile_reset()
    y = supra_attn.linear(gpu, xd, wd, N=N, K=K, variant="tf32x3")
    got = gpu.read(y)
    names = names_of(gpu)
    gpu.profile_reset()
    gpu.profile(False)
    y.release()
    assert names == {"linear_fp32"}, names
    check(got, oracle.linear(xa, wa, M, N, K), "tf32x3")


def test_strides_offsets_and_epilogue(gpu):
    """Strided x with an offset, strided y, in-place gated residual, GELU(tanh) (tf32x3)."""
    import supra_attn

    rng = np.random.default_rng(17)
    M, N, K = 150, 200, 61
    ldx, xo, ldy, yo, go = 67, 5, 203, 7, 11
    xa = rng.standard_normal(xo + M * ldx).astype(np.float32)
    wa = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    ba = rng.standard_normal(N).astype(np.float32)
    ga = rng.standard_normal(go + N).astype(np.float32)
    y0 = rng.standard_normal(yo + M * ldy).astype(np.float32)
    xd, wd, bd, gd, yd = dev(xa), dev(wa), dev(ba), dev(ga), dev(y0)
    supra_attn.linear(gpu, xd, wd, M=M, N=N, K=K, bias=bd, ldx=ldx, xOff=xo, out=yd, ldy=ldy, yOff=yo, resid=True,
                      gate=gd, gOff=go, act="gelu_tanh", variant="tf32x3")
    gpu.sync()
    got = host(yd)
    idx = yo + np.arange(M)[:, None] * ldy + np.arange(N)[None, :]
    keep = np.ones(got.size, bool)
    keep[idx.reshape(-1)] = False
    np.testing.assert_array_equal(got[keep], y0[keep])
    xr = xa[xo + np.arange(M)[:, None] * ldx + np.arange(K)[None, :]].astype(np.float64)
    pre = oracle.activation(xr @ wa.astype(np.float64).T + ba, "gelu_tanh")
    ref = y0[idx] + ga[go:go + N][None, :] * pre
    check(got[idx], ref, "tf32x3")


def test_norm_prologues(gpu):
    """GroupNorm (+ SiLU) and modulated LayerNorm applied before the split (tf32x3)."""
    import supra_attn

    rng = np.random.default_rng(19)
    rows, M, K, N = 64, 3 * 64, 96, 130
    x = (rng.standard_normal((M, K)) * 2 + 0.5).astype(np.float32)
    gamma, beta = rng.standard_normal(K).astype(np.float32), rng.standard_normal(K).astype(np.float32)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    mod = rng.standard_normal(3 * K).astype(np.float32)
    xd, gd, bd, wd, md = dev(x), dev(gamma), dev(beta), dev(w), dev(mod)
    y1 = supra_attn.linear(gpu, xd, wd, N=N, K=K, variant="tf32x3",
                           groupnorm=dict(gamma=gd, beta=bd, groups=8, rows_per_image=rows, silu=True))
    y2 = supra_attn.linear(gpu, xd, wd, N=N, K=K, variant="tf32x3", layernorm=dict(mod=md, shiftOff=K, scaleOff=2 * K))
    g1, g2 = gpu.read(y1).reshape(M, N), gpu.read(y2).reshape(M, N)
    w64 = w.astype(np.float64)
    for i in range(M // rows):
        sl = slice(i * rows, (i + 1) * rows)
        check(g1[sl], oracle.groupnorm(x[sl], gamma, beta, 8, silu=True) @ w64.T, "tf32x3")
    check(g2, oracle.layernorm(x, mod, K, 2 * K) @ w64.T, "tf32x3")
    for t in (y1, y2):
        t.release()


def test_batch_shares_weights(gpu):
    """Many problems with the same weights (split once per flush) and one with other weights."""
    import supra_attn

    rng = np.random.default_rng(23)
    K, N = 576, 1152
    wa = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    w2 = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    ba = rng.standard_normal(N).astype(np.float32)
    wd, w2d, bd = dev(wa), dev(w2), dev(ba)
    Ms = [5, 77, 128, 1, 300]
    xs = [rng.standard_normal((m, K)).astype(np.float32) for m in Ms]
    xds = [dev(x) for x in xs]
    gpu.sync()
    n0 = gpu.launch_count()
    gpu.profile(True)
    gpu.profile_reset()
    ys = [supra_attn.linear(gpu, xds[i], wd if i != 2 else w2d, N=N, K=K, bias=bd, variant="tf32x3")
          for i in range(len(Ms))]
    gpu.flush()
    gpu.sync()
    rep = {r["name"]: r for r in gpu.profile_report()}
    gpu.profile_reset()
    gpu.profile(False)
    assert rep["linear_tc_tf32x3"]["count"] == 1 and rep["linear_split"]["count"] == 1
    # one split launch (every x and the 2 distinct w), one product launch, one descriptor staging
    assert gpu.launch_count() - n0 == 3
    for i, m in enumerate(Ms):
        check(gpu.read(ys[i]), oracle.linear(xs[i], wa if i != 2 else w2, m, N, K, bias=ba), "tf32x3")
        ys[i].release()


def test_dit_block_golden_tf32x3(gpu, golden):
    """The whole DiT block with every product and attention in the split-precision form, against
    the reference's dit_forward pieces at the FP32 bar."""
    import supra_attn
    from conftest import dit_block_inputs

    x = dit_block_inputs()
    B, N, D = x["B"], x["N"], x["D"]
    w = {k: dev(v) for k, v in x["w"].items()}
    mod, kvs = dev(x["mod"]), [dev(t) for t in x["kv"]]
    xs = dev(x["x0"])
    V = "tf32x3"
    qkv = supra_attn.linear(gpu, xs, w["qkv"], N=3 * D, K=D, bias=w["bqkv"], variant=V,
                            layernorm=dict(mod=mod, shiftOff=0, scaleOff=D))
    a = gpu.empty([B * N, D])
    for b in range(B):
        r = b * N * 3 * D
        supra_attn.attention(gpu, q=qkv, k=qkv, v=qkv, Lq=N, Lk=N, H=9, D=64, ldq=3 * D, ldk=3 * D, ldv=3 * D,
                             qOff=r, kOff=r + D, vOff=r + 2 * D, oOff=b * N * D, out=a, variant=V)
    supra_attn.linear(gpu, a, w["proj"], N=D, K=D, bias=w["bproj"], out=xs, resid=True, gate=mod, gOff=2 * D,
                      variant=V)
    q = supra_attn.linear(gpu, xs, w["q"], N=D, K=D, bias=w["bq"], layernorm={}, variant=V)
    c = gpu.empty([B * N, D])
    for b in range(B):
        supra_attn.attention(gpu, q=q, k=kvs[b], v=kvs[b], Lq=N, Lk=x["Ls"][b], H=9, D=64, ldq=D, ldk=2 * D,
                             ldv=2 * D, qOff=b * N * D, kOff=0, vOff=D, oOff=b * N * D, out=c, variant=V)
    supra_attn.linear(gpu, c, w["cproj"], N=D, K=D, bias=w["bcproj"], out=xs, resid=True, variant=V)
    f = supra_attn.linear(gpu, xs, w["fc1"], N=4 * D, K=D, bias=w["bfc1"], act="gelu_tanh", variant=V,
                          layernorm=dict(mod=mod, shiftOff=3 * D, scaleOff=4 * D))
    supra_attn.linear(gpu, f, w["fc2"], N=D, K=4 * D, bias=w["bfc2"], out=xs, resid=True, gate=mod, gOff=5 * D,
                      variant=V)
    gpu.sync()
    check(host(xs), golden("dit_block_x3"), "tf32x3")
    for t in (qkv, a, q, c, f):
        t.release()


def test_gates_folded_into_weights(gpu):
    """Gated residuals without an activation (the DiT block's proj / fc2): two problems on the same
    weights with different gates, in place on strided outputs with offsets, one flush (tf32x3)."""
    import supra_attn

    rng = np.random.default_rng(29)
    M, N, K = 300, 576, 576
    ldy, yo = 580, 8
    wa = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    ba = rng.standard_normal(N).astype(np.float32)
    mod = rng.standard_normal(6 * N).astype(np.float32)
    xs = [rng.standard_normal((M, K)).astype(np.float32) for _ in range(2)]
    y0s = [rng.standard_normal(yo + M * ldy).astype(np.float32) for _ in range(2)]
    wd, bd, md = dev(wa), dev(ba), dev(mod)
    xds, yds = [dev(x) for x in xs], [dev(y) for y in y0s]
    goffs = [2 * N, 5 * N]
    for i in range(2):
        supra_attn.linear(gpu, xds[i], wd, M=M, N=N, K=K, bias=bd, out=yds[i], ldy=ldy, yOff=yo, resid=True, gate=md,
                          gOff=goffs[i], variant="tf32x3")
    gpu.sync()
    idx = yo + np.arange(M)[:, None] * ldy + np.arange(N)[None, :]
    for i in range(2):
        got = host(yds[i])
        keep = np.ones(got.size, bool)
        keep[idx.reshape(-1)] = False
        np.testing.assert_array_equal(got[keep], y0s[i][keep])
        ref = oracle.gated_residual(y0s[i][idx], xs[i], wa, M, N, K, bias=ba, gate=mod, g_off=goffs[i])
        check(got[idx], ref, "tf32x3")


def test_tf32_operands_read_in_place(gpu):
    """The TF32 form reads 16-byte aligned operands (row strides a multiple of 4 floats) in place:
    no split launch. An x at an odd offset is split first. Both at the TF32 bar; the split form
    always splits."""
    import supra_attn

    rng = np.random.default_rng(41)
    M, N, K = 200, 300, 576
    xa = rng.standard_normal(1 + M * K).astype(np.float32)
    wa = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    xd, wd = dev(xa), dev(wa)
    for xo, variant, split in ((0, "tf32", False), (1, "tf32", True), (0, "tf32x3", True)):
        gpu.profile(True)
        gpu.profile_reset()
        y = supra_attn.linear(gpu, xd, wd, M=M, N=N, K=K, xOff=xo, variant=variant)
        got = gpu.read(y)
        names = names_of(gpu)
        gpu.profile_reset()
        gpu.profile(False)
        y.release()
        assert f"linear_tc_{variant}" in names and ("linear_split" in names) == split, (xo, variant, names)
        check(got, oracle.linear(xa[xo:xo + M * K], wa, M, N, K), variant)
