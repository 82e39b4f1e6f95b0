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
     (128, 128, 16, True), (300, 16128, 576, True), (1000, 7, 3, True)],
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
