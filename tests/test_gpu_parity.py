"""CUDA kernels (through the C ABI) against the pinned CPU oracle and the golden vectors.

FP32 bar: normwise max-relative error max|got - ref| / max|ref| <= 1e-5 and rel-L2 <= 1e-5 per
output tensor (the reference's rel-L2 metric, tools/check.js:31-44).
"""

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _torch():
    import torch

    return torch


def dev(a):
    return _torch().from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32)).reshape(-1)).cuda()


def host(t):
    return t.detach().cpu().numpy().reshape(-1)


def assert_close(got, ref, tol=TOL):
    mr, rl = oracle.max_rel(got, ref), oracle.rel_l2(got, ref)
    assert mr <= tol and rl <= tol, f"max_rel={mr:.3e} rel_l2={rl:.3e} (tol {tol})"


def attn(gpu, **kw):
    import supra_attn

    return supra_attn.attention(gpu, **kw)


# ---- the four call sites against the reference's golden outputs --------------------------------
def test_dit_self_golden(gpu, golden):
    c = golden.cases["dit_self"]
    B, N, H, D = c["B"], c["N"], c["H"], c["D"]
    qkv = dev(golden("dit_self_qkv"))
    out = dev(np.zeros(B * N * H * D))
    for b in range(B):  # one call per sample, as app/models/dit.js:170-173
        r = b * N * 3 * H * D
        attn(gpu, q=qkv, k=qkv, v=qkv, Lq=N, Lk=N, H=H, D=D, ldq=3 * H * D, ldk=3 * H * D, ldv=3 * H * D,
             qOff=r, kOff=r + H * D, vOff=r + 2 * H * D, oOff=b * N * H * D, out=out)
    assert gpu.pending() == B
    gpu.sync()
    assert_close(host(out), golden("dit_self_out"))


def test_dit_self_config1(gpu, golden):
    torch = _torch()
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(2, 256, 1728, generator=g).reshape(-1).cuda()
    out = torch.zeros(2 * 256 * 576, device="cuda")
    for b in range(2):
        r = b * 256 * 1728
        attn(gpu, q=qkv, k=qkv, v=qkv, Lq=256, Lk=256, H=9, D=64, ldq=1728, ldk=1728, ldv=1728, qOff=r,
             kOff=r + 576, vOff=r + 1152, oOff=b * 256 * 576, out=out)
    gpu.sync()
    assert_close(host(out), golden("dit_self_cfg1_out"))


def test_dit_cross_ragged_golden(gpu, golden):
    c = golden.cases["dit_cross"]
    N = c["N"]
    q = dev(golden("dit_cross_q"))
    out = dev(np.zeros(len(c["Ls"]) * N * 576))
    kvs = []
    for b, L in enumerate(c["Ls"]):  # app/models/dit.js:182-185, K/V cached per prompt [L, 1152]
        kv = dev(golden(f"dit_cross_kv{b}"))
        kvs.append(kv)
        attn(gpu, q=q, k=kv, v=kv, Lq=N, Lk=L, H=9, D=64, ldq=576, ldk=1152, ldv=1152, qOff=b * N * 576, kOff=0,
             vOff=576, oOff=b * N * 576, out=out)
    gpu.sync()
    assert_close(host(out), golden("dit_cross_out"))


@pytest.mark.parametrize("L", [1, 5, 37, 128])
def test_t5_golden(gpu, golden, L):
    import supra_attn

    table = dev(golden("t5_table"))
    bias = supra_attn.position_bias(gpu, table, L, H=12, buckets=32, max_distance=128)
    q, k, v = (dev(golden(f"t5_L{L}_{n}")) for n in "qkv")
    o = attn(gpu, q=q, k=k, v=v, Lq=L, Lk=L, H=12, D=64, ldq=768, ldk=768, ldv=768, scale=1.0, bias=bias)
    got = gpu.read(o)
    np.testing.assert_array_equal(gpu.read(bias), golden(f"t5_L{L}_bias").reshape(-1))  # bit-exact
    assert_close(got, golden(f"t5_L{L}_out"))
    o.release()
    bias.release()


@pytest.mark.parametrize("L", [1, 5, 37, 128])
def test_t5_table_golden(gpu, golden, L):
    """The T5 call site with the [32, 12] table in place of the expanded bias: the kernel forms
    the bias itself and gives the same bits as the expanded-bias call."""
    import supra_attn

    table = dev(golden("t5_table"))
    bias = supra_attn.position_bias(gpu, table, L, H=12, buckets=32, max_distance=128)
    q, k, v = (dev(golden(f"t5_L{L}_{n}")) for n in "qkv")
    kw = dict(q=q, k=k, v=v, Lq=L, Lk=L, H=12, D=64, ldq=768, ldk=768, ldv=768, scale=1.0)
    o_tab = attn(gpu, t5_table=table, t5_buckets=32, t5_max_distance=128, **kw)
    o_exp = attn(gpu, bias=bias, **kw)
    got = gpu.read(o_tab)
    np.testing.assert_array_equal(got, gpu.read(o_exp))
    assert_close(got, golden(f"t5_L{L}_out"))
    for t in (o_tab, o_exp, bias):
        t.release()


@pytest.mark.parametrize("L,H,D", [(300, 12, 64), (70, 2, 128), (70, 2, 512)])
def test_t5_table_long_and_wide(gpu, L, H, D):
    """Relative positions beyond max_distance (the bucket saturates; the kernels clamp) and the
    D = 128 and D = 512 kernels, against the float64 oracle and the expanded-bias call."""
    import supra_attn

    rng = np.random.default_rng(L + D)
    table = (0.5 * rng.standard_normal(32 * H)).astype(np.float32)
    q, k, v = (rng.standard_normal(L * H * D).astype(np.float32) for _ in range(3))
    scale = (64.0 / D) ** 0.5
    ref_bias = oracle.position_bias(table, L, H, 32, 128).reshape(-1)
    ref = oracle.attention_ops(q, k, v, L, L, H, D, H * D, H * D, H * D, scale=scale, bias=ref_bias)
    td = dev(table)
    kw = dict(q=dev(q), k=dev(k), v=dev(v), Lq=L, Lk=L, H=H, D=D, ldq=H * D, ldk=H * D, ldv=H * D, scale=scale)
    o_tab = attn(gpu, t5_table=td, **kw)
    bias = supra_attn.position_bias(gpu, td, L, H=H, buckets=32, max_distance=128)
    o_exp = attn(gpu, bias=bias, **kw)
    got = gpu.read(o_tab)
    assert_close(got, ref)
    np.testing.assert_array_equal(got, gpu.read(o_exp))
    for t in (o_tab, o_exp, bias):
        t.release()


@pytest.mark.parametrize("L", [65, 100, 128, 300])
def test_t5_bias_on_the_persistent_kernel(gpu, L):
    """Lq > 64 with a bias (the T5 encoder, app/models/t5.js:80) runs the bias form of the
    persistent FP32 kernel, table and expanded forms bit-identical to each other; L = 100 and 300
    leave query rows past Lq in a tile (warps wholly past Lq skip the arithmetic)."""
    import supra_attn

    rng = np.random.default_rng(L)
    H = 12
    table = (0.5 * rng.standard_normal(32 * H)).astype(np.float32)
    q, k, v = (rng.standard_normal(L * H * 64).astype(np.float32) for _ in range(3))
    ref = oracle.attention_ops(q, k, v, L, L, H, 64, H * 64, H * 64, H * 64, scale=1.0,
                               bias=oracle.position_bias(table, L, H, 32, 128).reshape(-1))
    td = dev(table)
    kw = dict(q=dev(q), k=dev(k), v=dev(v), Lq=L, Lk=L, H=H, D=64, ldq=H * 64, ldk=H * 64, ldv=H * 64, scale=1.0)
    bias = supra_attn.position_bias(gpu, td, L, H=H, buckets=32, max_distance=128)
    gpu.sync()
    gpu.profile(True)
    gpu.profile_reset()
    o_tab = attn(gpu, t5_table=td, **kw)
    gpu.flush()
    o_exp = attn(gpu, bias=bias, **kw)
    got = gpu.read(o_tab)
    rep = {r["name"]: r["count"] for r in gpu.profile_report()}
    gpu.profile(False)
    assert rep == {"attn_fp32_d64_tma_bias": 2}, rep
    assert_close(got, ref)
    np.testing.assert_array_equal(got, gpu.read(o_exp))
    for t in (o_tab, o_exp, bias):
        t.release()


def test_expanded_bias_scaled_on_the_persistent_kernel(gpu):
    """A [H, Lq, Lk] bias with scale 1/8 and Lq != Lk (ragged last key block, a partial last
    query tile) on the persistent FP32 kernel's bias form, against the oracle."""
    rng = np.random.default_rng(9)
    Lq, Lk, H = 200, 150, 3
    q = rng.standard_normal(Lq * H * 64).astype(np.float32)
    k, v = (rng.standard_normal(Lk * H * 64).astype(np.float32) for _ in range(2))
    b = rng.standard_normal(H * Lq * Lk).astype(np.float32)
    ref = oracle.attention_ops(q, k, v, Lq, Lk, H, 64, H * 64, H * 64, H * 64, scale=0.125, bias=b)
    gpu.profile(True)
    gpu.profile_reset()
    o = attn(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=64, ldq=H * 64, ldk=H * 64, ldv=H * 64,
             scale=0.125, bias=dev(b))
    got = gpu.read(o)
    names = [r["name"] for r in gpu.profile_report()]
    gpu.profile(False)
    o.release()
    assert names == ["attn_fp32_d64_tma_bias"], names
    assert_close(got, ref)


def test_t5_table_ragged_batch(gpu):
    """256 prompts of ragged length (config 3) in one flush, table mode, against the oracle."""
    import supra_attn

    rng = np.random.default_rng(33)
    Ls = rng.integers(1, 129, 256)
    table = (0.1 * rng.standard_normal(32 * 12)).astype(np.float32)
    offs = np.concatenate([[0], np.cumsum(Ls * 768)]).astype(np.int64)
    q, k, v = (rng.standard_normal(int(offs[-1])).astype(np.float32) for _ in range(3))
    qd, kd, vd, td = dev(q), dev(k), dev(v), dev(table)
    out = dev(np.zeros(int(offs[-1])))
    descs = (supra_attn.Desc * 256)()
    for i, L in enumerate(Ls):
        descs[i] = supra_attn.make_desc(q=qd, k=kd, v=vd, out=out, Lq=int(L), Lk=int(L), H=12, D=64, ldq=768, ldk=768,
                                        ldv=768, qOff=int(offs[i]), kOff=int(offs[i]), vOff=int(offs[i]),
                                        oOff=int(offs[i]), scale=1.0, t5_table=td)
    gpu.enqueue_batch(descs)
    gpu.sync()
    got = host(out)
    for i in range(256):  # every prompt against the float64 oracle
        L, a, b = int(Ls[i]), int(offs[i]), int(offs[i + 1])
        bias = oracle.position_bias(table, L, 12, 32, 128).reshape(-1)
        assert_close(got[a:b], oracle.attention_ops(q[a:b], k[a:b], v[a:b], L, L, 12, 64, 768, 768, 768, scale=1.0,
                                                    bias=bias))


def test_t5_tables_mixed_in_one_flush(gpu):
    """T5 table problems with different tables, bucket counts, max distances and head counts in
    one flush of the persistent kernel (each distinct (table, buckets, max distance, H) gets its
    own bias-by-relative-position array), relative positions past max_distance included, against
    the float64 oracle."""
    import supra_attn

    rng = np.random.default_rng(35)
    cfgs = [(12, 32, 128), (4, 16, 40), (12, 32, 128), (4, 8, 20), (12, 16, 40)]
    tables = {}
    for H, nb, md in cfgs:
        if (H, nb) not in tables:
            tables[(H, nb)] = (0.3 * rng.standard_normal(nb * H)).astype(np.float32)
    tdev = {key: dev(t) for key, t in tables.items()}
    probs = []
    for i in range(20):
        H, nb, md = cfgs[i % len(cfgs)]
        L = int(rng.integers(65, 200))
        q, k, v = (rng.standard_normal(L * H * 64).astype(np.float32) for _ in range(3))
        probs.append((H, nb, md, L, q, k, v, dev(q), dev(k), dev(v), dev(np.zeros(L * H * 64))))
    descs = (supra_attn.Desc * len(probs))()
    for i, (H, nb, md, L, q, k, v, qd, kd, vd, od) in enumerate(probs):
        descs[i] = supra_attn.make_desc(q=qd, k=kd, v=vd, out=od, Lq=L, Lk=L, H=H, D=64, ldq=H * 64, ldk=H * 64,
                                        ldv=H * 64, scale=1.0, t5_table=tdev[(H, nb)], t5_buckets=nb,
                                        t5_max_distance=md)
    gpu.profile(True)
    gpu.profile_reset()
    gpu.enqueue_batch(descs)
    gpu.sync()
    names = sorted(r["name"] for r in gpu.profile_report())
    gpu.profile(False)
    assert names == ["attn_fp32_d64_tma_bias"], names
    for H, nb, md, L, q, k, v, qd, kd, vd, od in probs:
        bias = oracle.position_bias(tables[(H, nb)], L, H, nb, md).reshape(-1)
        assert_close(host(od), oracle.attention_ops(q, k, v, L, L, H, 64, H * 64, H * 64, H * 64, scale=1.0,
                                                    bias=bias))


@pytest.mark.parametrize("variant", ["fp32", "tf32x3"])
def test_tensor_map_table_refills_and_grows(gpu, variant):
    """Flushes whose problems each bring their own buffers (distinct base pointers: new tensor
    maps every flush). The context's device table of maps fills up, starts over (maps staged
    again into reused slots while earlier launches may still be queued) and, for one flush that
    needs more maps than it holds, grows; sampled outputs of every flush against the float64
    oracle."""
    import supra_attn

    rng = np.random.default_rng(41)
    H, D, ld = 2, 64, 128
    pool = rng.standard_normal(12 * 14000 + 70 * ld + 64).astype(np.float32)
    pd = dev(pool)
    tol = TOL if variant == "fp32" else 1e-5

    def run(first, n, L):
        # problem i: q, k, v start 0, 4 and 8 floats after base 12 * (first + i) of the pool
        # (overlapping reads, 16-byte aligned, each its own tensor map)
        out = _torch().zeros(n * L * ld, device="cuda")
        descs = (supra_attn.Desc * n)()
        for i in range(n):
            b = 12 * (first + i)
            d = supra_attn.make_desc(q=pd, k=pd, v=pd, out=out, Lq=L, Lk=L, H=H, D=D, ldq=ld, ldk=ld, ldv=ld,
                                     oOff=i * L * ld, variant=variant)
            for name, off in (("q", b), ("k", b + 4), ("v", b + 8)):
                setattr(d, name, pd.data_ptr() + 4 * off)
                setattr(d, name + "_size", L * ld)
            descs[i] = d
        gpu.enqueue_batch(descs)
        return out

    outs = []
    first = 0
    for f in range(9):  # 700 problems x 3 new maps per flush: the 16384-slot table starts over
        outs.append((first, 700, 65 + f % 3, run(first, 700, 65 + f % 3)))
        gpu.flush()
        first += 700
    outs.append((first, 4200, 65, run(first, 4200, 65)))  # 12600 maps in one flush: the table grows
    gpu.sync()
    for first, n, L, out in outs:
        got = host(out)
        for i in sorted(set([0, n - 1] + list(rng.integers(0, n, 6)))):
            b = 12 * (first + i)
            q, k, v = (pool[o:o + L * ld] for o in (b, b + 4, b + 8))
            ref = oracle.attention_ops(q, k, v, L, L, H, D, ld, ld, ld)
            assert_close(got[i * L * ld:(i + 1) * L * ld], ref, tol)


def test_t5_expanded_bias_ragged_batch(gpu):
    """Config 3 as the T5 call site issues it (app/models/t5.js:73-80): 256 prompts of ragged
    length L ~ U{1..128} in one flush, each with its own expanded [12, L, L] bias from
    positionBias, scale 1, on the persistent kernel's bias form (L > 64) and the block kernel
    (L <= 64); every prompt against the float64 oracle."""
    import supra_attn

    rng = np.random.default_rng(34)
    Ls = rng.integers(1, 129, 256)
    table = (0.1 * rng.standard_normal(32 * 12)).astype(np.float32)
    offs = np.concatenate([[0], np.cumsum(Ls * 768)]).astype(np.int64)
    boffs = np.concatenate([[0], np.cumsum(12 * Ls * Ls)]).astype(np.int64)
    q, k, v = (rng.standard_normal(int(offs[-1])).astype(np.float32) for _ in range(3))
    biases = np.concatenate([oracle.position_bias(table, int(L), 12, 32, 128).reshape(-1) for L in Ls])
    qd, kd, vd, bd = dev(q), dev(k), dev(v), dev(biases)
    out = dev(np.zeros(int(offs[-1])))
    descs = (supra_attn.Desc * 256)()
    for i, L in enumerate(Ls):
        descs[i] = supra_attn.make_desc(q=qd, k=kd, v=vd, out=out, Lq=int(L), Lk=int(L), H=12, D=64, ldq=768, ldk=768,
                                        ldv=768, qOff=int(offs[i]), kOff=int(offs[i]), vOff=int(offs[i]),
                                        oOff=int(offs[i]), scale=1.0)
        # the bias of prompt i starts at boffs[i]; the descriptor addresses it by pointer
        descs[i].bias = bd.data_ptr() + 4 * int(boffs[i])
        descs[i].bias_size = 12 * int(L) * int(L)
    gpu.profile(True)
    gpu.profile_reset()
    gpu.enqueue_batch(descs)
    gpu.sync()
    names = sorted(r["name"] for r in gpu.profile_report())
    gpu.profile(False)
    assert "attn_fp32_d64_tma_bias" in names, names
    got = host(out)
    for i in range(256):
        L, a, b = int(Ls[i]), int(offs[i]), int(offs[i + 1])
        ref = oracle.attention_ops(q[a:b], k[a:b], v[a:b], L, L, 12, 64, 768, 768, 768, scale=1.0,
                                   bias=biases[boffs[i]:boffs[i + 1]])
        assert_close(got[a:b], ref)


def test_vae_golden(gpu, golden):
    T = golden.cases["vae_small"]["T"]
    q, k, v = (dev(golden(f"vae_small_{n}")) for n in "qkv")
    o = attn(gpu, q=q, k=k, v=v, Lq=T, Lk=T, H=1, D=512, ldq=512, ldk=512, ldv=512)  # app/models/vae.js:86
    assert_close(gpu.read(o), golden("vae_small_out"))
    o.release()


def vae_inputs(n_img, seed):
    """Config 4: x ~ N(0,1) per channel, Q/K/V = x W^T + b, W Xavier-uniform, b ~ U(+-1/sqrt(512))."""
    rng = np.random.default_rng(seed)
    bound = (6.0 / 1024) ** 0.5
    W = [rng.uniform(-bound, bound, (512, 512)).astype(np.float32) for _ in range(3)]
    bv = [rng.uniform(-1 / 512 ** 0.5, 1 / 512 ** 0.5, 512).astype(np.float32) for _ in range(3)]
    x = rng.standard_normal((n_img, 1024, 512)).astype(np.float32)
    return [(x @ w.T + b).astype(np.float32) for w, b in zip(W, bv)]


@pytest.mark.parametrize("n_img,checked", [(2, (0, 1)), (8, tuple(range(8))), (64, (0, 9, 27, 45, 63))])
def test_vae_full_size(gpu, n_img, checked):
    """Config 4 at batch 2, 8 (every image checked) and 64 (a sample of images checked), one call
    per image (app/models/vae.js:86) grouped into one flush, FP32 FFMA score path: from 8 images
    on (enough tiles for two CTAs per SM) S = Q K^T and O = P V run on the FFMA linear, the
    latter reading V as W [Lk, D]."""
    q, k, v = vae_inputs(n_img, 4)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = dev(np.zeros(n_img * 1024 * 512))
    gpu.profile(True)
    gpu.profile_reset()
    for i in range(n_img):
        o = i * 1024 * 512
        attn(gpu, q=qd, k=kd, v=vd, Lq=1024, Lk=1024, H=1, D=512, ldq=512, ldk=512, ldv=512, qOff=o, kOff=o, vOff=o,
             oOff=o, out=out)
    gpu.sync()
    names = {r["name"] for r in gpu.profile_report()}
    gpu.profile(False)
    assert names == ({"attn_gemm_qk_lin", "attn_softmax_rows", "attn_gemm_pv_lin"} if n_img >= 8
                     else {"attn_gemm_qk", "attn_softmax_rows", "attn_gemm_pv"}), names
    got = host(out).reshape(n_img, 1024, 512)
    for i in checked:
        assert_close(got[i], oracle.attention_heads(q[i], k[i], v[i], 1))


def test_score_path_on_linear_ragged(gpu):
    """The score path's products on the FFMA linear (S = Q K^T, and O = P V reading V as W [Lk, D])
    at sizes that are not multiples of any tile: 9 problems of 2 heads, Lq = 700, Lk = 900, D = 192,
    each in its own buffers with padded row strides; every problem against the oracle."""
    import supra_attn

    rng = np.random.default_rng(41)
    H, D, Lq, Lk = 2, 192, 700, 900
    ld = H * D + 8
    gpu.profile(True)
    gpu.profile_reset()
    cases = []
    for _ in range(9):
        q = rng.standard_normal(Lq * ld).astype(np.float32)
        k = rng.standard_normal(Lk * ld).astype(np.float32)
        v = rng.standard_normal(Lk * ld).astype(np.float32)
        qd, kd, vd = dev(q), dev(k), dev(v)  # (kept alive until the flush)
        o = supra_attn.attention(gpu, q=qd, k=kd, v=vd, Lq=Lq, Lk=Lk, H=H, D=D, ldq=ld, ldk=ld, ldv=ld)
        cases.append((q, k, v, o, (qd, kd, vd)))
    gpu.sync()
    names = {r["name"] for r in gpu.profile_report()}
    gpu.profile(False)
    assert {"attn_gemm_qk_lin", "attn_gemm_pv_lin"} <= names, names
    for q, k, v, o, _ in cases:
        got = gpu.read(o).reshape(Lq, H * D)
        ref = oracle.attention_heads(q.reshape(Lq, ld)[:, : H * D], k.reshape(Lk, ld)[:, : H * D],
                                     v.reshape(Lk, ld)[:, : H * D], H)
        assert_close(got, ref)
        o.release()


# ---- edge cases ---------------------------------------------------------------------------------
def rand_problem(rng, Lq, Lk, H, D, ldq=None, ldk=None, ldv=None, qOff=0, kOff=0, vOff=0, oOff=0, bias=False):
    ldq = ldq or H * D
    ldk = ldk or H * D
    ldv = ldv or H * D
    q = rng.standard_normal(qOff + (Lq - 1) * ldq + H * D if Lq else 1).astype(np.float32)
    k = rng.standard_normal(kOff + (Lk - 1) * ldk + H * D).astype(np.float32)
    v = rng.standard_normal(vOff + (Lk - 1) * ldv + H * D).astype(np.float32)
    b = rng.standard_normal(H * Lq * Lk).astype(np.float32) if bias else None
    return dict(q=q, k=k, v=v, bias=b, Lq=Lq, Lk=Lk, H=H, D=D, ldq=ldq, ldk=ldk, ldv=ldv, qOff=qOff, kOff=kOff,
                vOff=vOff, oOff=oOff)


def run_and_check(gpu, p, scale=None, tol=TOL):
    q, k, v = dev(p["q"]), dev(p["k"]), dev(p["v"])
    bias = dev(p["bias"]) if p["bias"] is not None else None
    n_out = p["oOff"] + p["Lq"] * p["H"] * p["D"]
    out = dev(np.full(max(n_out, 1), 7.0))
    kw = {kk: p[kk] for kk in ("Lq", "Lk", "H", "D", "ldq", "ldk", "ldv", "qOff", "kOff", "vOff", "oOff")}
    attn(gpu, q=q, k=k, v=v, bias=bias, out=out, scale=scale, **kw)
    gpu.sync()
    ref = np.full(max(n_out, 1), 7.0, dtype=np.float32)
    oracle.attention_ops(p["q"], p["k"], p["v"], scale=scale, bias=p["bias"], out=ref, **kw)
    got = host(out)
    assert np.all(got[: p["oOff"]] == 7.0), "wrote before oOff"
    assert_close(got, ref, tol)


@pytest.mark.parametrize(
    "Lq,Lk,H,D",
    [
        (1, 1, 1, 64), (1, 300, 2, 64), (63, 65, 3, 64), (64, 64, 1, 64), (65, 129, 2, 64), (129, 63, 1, 64),
        (200, 1000, 2, 64), (256, 4096, 1, 64), (17, 33, 2, 16), (40, 40, 2, 32), (50, 70, 3, 60),
        (70, 130, 2, 96), (100, 100, 2, 128), (33, 77, 1, 192), (130, 260, 2, 256), (64, 96, 1, 512),
        # warp-pipelined D<=64 kernel: idle warps (Lq % 128), partial key blocks, head-dim padding,
        # single key, many ring refills
        (100, 50, 2, 32), (97, 31, 3, 48), (130, 1, 1, 64), (300, 97, 2, 64), (129, 33, 2, 64),
        (160, 2000, 1, 64), (65, 8, 4, 8),
        # persistent TMA kernel: ragged last blocks with 1, 2, 3 and 4 key groups of 8
        (100, 37, 2, 64), (100, 44, 2, 64), (100, 52, 2, 64), (100, 60, 2, 64), (257, 31, 3, 64),
    ],
)
def test_shapes(gpu, Lq, Lk, H, D):
    rng = np.random.default_rng(Lq * 1000 + Lk * 10 + D)
    run_and_check(gpu, rand_problem(rng, Lq, Lk, H, D))


@pytest.mark.parametrize("D", [64, 128, 512])
def test_strided_and_unaligned(gpu, D):
    rng = np.random.default_rng(D)
    H = 2
    # 16-byte aligned strides/offsets (bulk-copy path) with padding between rows
    run_and_check(gpu, rand_problem(rng, 70, 90, H, D, ldq=H * D + 4, ldk=H * D + 8, ldv=H * D + 12, qOff=4, kOff=8,
                                    vOff=12, oOff=4))
    # misaligned offsets and strides (the reference's own unfused fallback case, app/gpu/ops.js:111)
    run_and_check(gpu, rand_problem(rng, 70, 90, H, D, ldq=H * D + 1, ldk=H * D + 3, ldv=H * D + 5, qOff=1, kOff=3,
                                    vOff=5, oOff=1))


@pytest.mark.parametrize("D", [64, 128, 512])
@pytest.mark.parametrize("Lq,Lk", [(1, 1), (37, 37), (65, 130)])
def test_bias(gpu, D, Lq, Lk):
    # T5 runs unscaled at D = 64 (app/models/t5.js:80); wider heads keep the same score spread
    # (N(0,1) inputs at D = 512 and scale 1 give scores of std 22, where fp32 accumulation alone
    # is ~1e-5 off float64)
    rng = np.random.default_rng(D + Lq)
    run_and_check(gpu, rand_problem(rng, Lq, Lk, 3, D, bias=True), scale=(64.0 / D) ** 0.5)


def test_custom_scale_and_lq_zero(gpu):
    rng = np.random.default_rng(5)
    run_and_check(gpu, rand_problem(rng, 33, 45, 2, 64), scale=0.37)
    run_and_check(gpu, rand_problem(rng, 100, 70, 2, 64), scale=-0.2)  # non-positive scales
    run_and_check(gpu, rand_problem(rng, 100, 70, 2, 64), scale=0.0)
    p = rand_problem(rng, 0, 5, 1, 64)
    torch = _torch()
    out = torch.zeros(1, device="cuda")
    attn(gpu, q=dev(p["q"]), k=dev(p["k"]), v=dev(p["v"]), Lq=0, Lk=5, H=1, D=64, ldq=64, ldk=64, ldv=64, out=out)
    assert gpu.pending() == 0
    gpu.sync()


def test_known_answers(gpu):
    rng = np.random.default_rng(7)
    v = rng.standard_normal(64).astype(np.float32)
    q = rng.standard_normal(5 * 64).astype(np.float32)
    k = rng.standard_normal(64).astype(np.float32)
    o = attn(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=5, Lk=1, H=1, D=64, ldq=64, ldk=64, ldv=64)
    np.testing.assert_array_equal(gpu.read(o).reshape(5, 64), np.tile(v, (5, 1)))  # L = 1: exactly V
    vv = rng.standard_normal(9 * 64).astype(np.float32)
    o2 = attn(gpu, q=dev(np.zeros(3 * 64)), k=dev(rng.standard_normal(9 * 64)), v=dev(vv), Lq=3, Lk=9, H=1, D=64,
              ldq=64, ldk=64, ldv=64)
    np.testing.assert_allclose(gpu.read(o2).reshape(3, 64), np.tile(vv.reshape(9, 64).mean(0), (3, 1)), atol=2e-6)


def test_hazard_ordering(gpu):
    """A call that reads an earlier recorded call's output sees it (auto-flush on the hazard)."""
    rng = np.random.default_rng(11)
    q = rng.standard_normal(40 * 128).astype(np.float32)
    k = rng.standard_normal(50 * 128).astype(np.float32)
    v = rng.standard_normal(50 * 128).astype(np.float32)
    qd, kd, vd = dev(q), dev(k), dev(v)
    o1 = dev(np.zeros(40 * 128))
    o2 = dev(np.zeros(40 * 128))
    attn(gpu, q=qd, k=kd, v=vd, Lq=40, Lk=50, H=2, D=64, ldq=128, ldk=128, ldv=128, out=o1)
    attn(gpu, q=o1, k=kd, v=vd, Lq=40, Lk=50, H=2, D=64, ldq=128, ldk=128, ldv=128, out=o2)
    gpu.sync()
    r1 = oracle.attention_ops(q, k, v, 40, 50, 2, 64, 128, 128, 128)
    r2 = oracle.attention_ops(r1, k, v, 40, 50, 2, 64, 128, 128, 128)
    assert_close(host(o2), r2)


def test_invalid_call_raises_and_records_nothing(gpu):
    rng = np.random.default_rng(3)
    q = dev(rng.standard_normal(64))
    before = gpu.pending()
    with pytest.raises(ValueError):
        attn(gpu, q=q, k=q, v=q, Lq=2, Lk=1, H=1, D=64, ldq=64, ldk=64, ldv=64)  # q too short for Lq=2
    assert gpu.pending() == before


def test_determinism_and_profile(gpu):
    rng = np.random.default_rng(9)
    p = rand_problem(rng, 256, 256, 9, 64)
    q, k, v = dev(p["q"]), dev(p["k"]), dev(p["v"])
    gpu.profile(True)
    gpu.profile_reset()
    n0 = gpu.launch_count()
    outs = []
    for _ in range(2):
        o = attn(gpu, q=q, k=k, v=v, Lq=256, Lk=256, H=9, D=64, ldq=576, ldk=576, ldv=576)
        outs.append(gpu.read(o))
        o.release()
    np.testing.assert_array_equal(outs[0], outs[1])
    rep = gpu.profile_report()
    gpu.profile(False)
    # per flush: descriptor staging + the attention kernel; the first flush also stages its new
    # tensor maps into the context's table, which the second reuses
    assert gpu.launch_count() - n0 == 5
    names = [r["name"] for r in rep]
    assert names == ["attn_fp32_d64_tma"], names  # the persistent TMA kernel serves the DiT shapes


# ---- persistent FP32 kernel (TMA boxes, K/V ring across tiles) ------------------------------------
def test_fp32_tma_nan_past_lengths(gpu):
    """Whole 32-row boxes read rows past Lq and Lk. Fill those rows with NaN/inf: no output may
    change (scores past Lk are replaced by -inf, V rows past Lk are not read, rows past Lq are
    not stored)."""
    rng = np.random.default_rng(21)
    H, D, Lq, Lk = 3, 64, 200, 45  # 200 = 128 + 72 rows; 45 keys = 1 block + 13 (a ragged group of 1)
    ld = H * D
    q = rng.standard_normal((Lq + 40) * ld).astype(np.float32)
    k = rng.standard_normal((Lk + 40) * ld).astype(np.float32)
    v = rng.standard_normal((Lk + 40) * ld).astype(np.float32)
    q[Lq * ld:] = np.nan
    k[Lk * ld:] = np.inf
    v[Lk * ld:] = np.nan
    out = dev(np.full((Lq + 40) * ld, 7.0))
    gpu.profile(True)
    gpu.profile_reset()
    attn(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=D, ldq=ld, ldk=ld, ldv=ld, out=out)
    gpu.sync()
    names = [r["name"] for r in gpu.profile_report()]
    gpu.profile(False)
    assert names == ["attn_fp32_d64_tma"], names
    got = host(out)
    ref = oracle.attention_ops(q[: Lq * ld], k[: Lk * ld], v[: Lk * ld], Lq, Lk, H, D, ld, ld, ld)
    assert_close(got[: Lq * ld], ref)
    assert np.all(got[Lq * ld:] == 7.0), "wrote past Lq"


def test_fp32_tma_many_ragged_tiles(gpu):
    """600 problems with 1..70 keys (1-3 key blocks per tile): every CTA runs several tiles and the
    K/V ring carries blocks of the next tiles; one launch."""
    torch = _torch()
    import supra_attn

    g = torch.Generator().manual_seed(22)
    n, H, D, Lq = 600, 2, 64, 130
    Ls = torch.randint(1, 71, (n,), generator=g).tolist()
    q = torch.randn(n * Lq * H * D, generator=g)
    kv_off = np.concatenate([[0], np.cumsum([L * 2 * H * D for L in Ls])]).astype(np.int64)
    kv = torch.randn(int(kv_off[-1]), generator=g)
    qd, kvd = q.cuda(), kv.cuda()
    out = torch.zeros(n * Lq * H * D, device="cuda")
    descs = (supra_attn.Desc * n)()
    for b, L in enumerate(Ls):
        descs[b] = supra_attn.make_desc(q=qd, k=kvd, v=kvd, out=out, Lq=Lq, Lk=L, H=H, D=D, ldq=H * D,
                                        ldk=2 * H * D, ldv=2 * H * D, qOff=b * Lq * H * D, kOff=int(kv_off[b]),
                                        vOff=int(kv_off[b]) + H * D, oOff=b * Lq * H * D)
    n0 = gpu.launch_count()
    gpu.enqueue_batch(descs)
    gpu.sync()
    # descriptor staging + one attention launch, and the staging of the batch's tensor maps (new
    # buffers) into the context's table
    assert gpu.launch_count() - n0 == 3
    got = host(out).reshape(n, Lq, H * D)
    qn, kvn = q.numpy().reshape(n, Lq, H * D), kv.numpy()
    for b in list(range(0, n, 37)) + [n - 1]:
        x = kvn[kv_off[b]: kv_off[b + 1]].reshape(-1, 2 * H * D)
        assert_close(got[b], oracle.attention_heads(qn[b], x[:, : H * D], x[:, H * D:], H))
    for b in range(n):  # every row a convex combination of its V rows
        x = kvn[kv_off[b]: kv_off[b + 1]].reshape(-1, 2 * H * D)[:, H * D:]
        assert np.all(got[b] >= x.min(0) - 1e-5) and np.all(got[b] <= x.max(0) + 1e-5)


# ---- BASELINE config sizes --------------------------------------------------------------------
def test_config2_cross_full(gpu):
    """Config 2: 128 sequences, L ~ U{1..128}, Q [128, 256, 576], K/V packed [L, 1152] per sequence."""
    torch = _torch()
    g = torch.Generator().manual_seed(2)
    Ls = torch.randint(1, 129, (128,), generator=g).tolist()
    q = torch.randn(128 * 256 * 576, generator=g)
    kvs = [torch.randn(L * 1152, generator=g) for L in Ls]
    qd = q.cuda()
    kvd = [x.cuda() for x in kvs]
    out = torch.zeros(128 * 256 * 576, device="cuda")
    import supra_attn

    descs = (supra_attn.Desc * 128)()
    for b, L in enumerate(Ls):
        descs[b] = supra_attn.make_desc(q=qd, k=kvd[b], v=kvd[b], out=out, Lq=256, Lk=L, H=9, D=64, ldq=576,
                                        ldk=1152, ldv=1152, qOff=b * 256 * 576, kOff=0, vOff=576, oOff=b * 256 * 576)
    gpu.enqueue_batch(descs)
    gpu.sync()
    got = host(out).reshape(128, 256, 576)
    qn = q.numpy().reshape(128, 256, 576)
    for b in range(128):  # every sequence against the float64 oracle
        kv = kvs[b].numpy().reshape(-1, 1152)
        assert_close(got[b], oracle.attention_heads(qn[b], kv[:, :576], kv[:, 576:], 9))


# ---- key splits of the persistent FP32 kernel (launches with few (head, query tile) groups) -----
@pytest.mark.parametrize("Lq,Lk,H,bias", [
    (256, 256, 9, None),      # 18 groups: 8 splits of one key block
    (200, 37, 3, None),       # 6 groups, 2 key blocks (ragged last) -> 2 splits; a partial query tile
    (128, 300, 2, None),      # 2 groups, 10 blocks -> splits of 2 blocks, the last one ragged
    (65, 4096, 2, None),      # two groups of 65 query rows, 128 key blocks in 8 splits each
    (100, 100, 12, "table"),  # one T5 prompt (app/models/t5.js:80): 12 groups, 4 splits, table bias
    (150, 200, 3, "expanded"),
])
def test_fp32_key_splits(gpu, Lq, Lk, H, bias):
    """A launch with at most half as many groups as CTA slots splits each group's key blocks
    across CTAs and combines the partial rows in the kernel; against the float64 oracle, with
    NaN/inf planted past Lq and Lk (boxes read those rows; nothing there may reach the output)."""
    import supra_attn

    rng = np.random.default_rng(Lq * 7 + Lk)
    D = 64
    ld = H * D
    q = rng.standard_normal((Lq + 40) * ld).astype(np.float32)
    k = rng.standard_normal((Lk + 40) * ld).astype(np.float32)
    v = rng.standard_normal((Lk + 40) * ld).astype(np.float32)
    q[Lq * ld:] = np.nan
    k[Lk * ld:] = np.inf
    v[Lk * ld:] = np.nan
    kw = dict(q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=D, ldq=ld, ldk=ld, ldv=ld)
    scale, b_ref = None, None
    if bias == "table":
        table = (0.5 * rng.standard_normal(32 * H)).astype(np.float32)
        kw.update(t5_table=dev(table), scale=1.0)
        scale, b_ref = 1.0, oracle.position_bias(table, Lq, H, 32, 128).reshape(-1)
    elif bias == "expanded":
        b_ref = rng.standard_normal(H * Lq * Lk).astype(np.float32)
        kw.update(bias=dev(b_ref), scale=0.125)
        scale = 0.125
    out = dev(np.full((Lq + 40) * ld, 7.0))
    gpu.profile(True)
    gpu.profile_reset()
    attn(gpu, out=out, **kw)
    gpu.sync()
    names = [r["name"] for r in gpu.profile_report()]
    gpu.profile(False)
    assert names == ["attn_fp32_d64_tma" + ("_bias" if bias else "")], names
    got = host(out)
    ref = oracle.attention_ops(q[: Lq * ld], k[: Lk * ld], v[: Lk * ld], Lq, Lk, H, D, ld, ld, ld, scale=scale,
                               bias=b_ref)
    assert_close(got[: Lq * ld], ref)
    assert np.all(got[Lq * ld:] == 7.0), "wrote past Lq"


def test_fp32_key_splits_deterministic_and_unsplit_batch(gpu):
    """Split results are the same on every run (the combine sums the splits in a fixed order), and
    a batch of the same problems large enough not to split gives the same values to the FP32 bar."""
    import supra_attn

    rng = np.random.default_rng(77)
    n, Lq, Lk, H, D = 40, 256, 256, 9, 64
    q = rng.standard_normal(n * Lq * H * D).astype(np.float32)
    kv = rng.standard_normal(n * Lk * 2 * H * D).astype(np.float32)
    qd, kvd = dev(q), dev(kv)
    outs = []
    for _ in range(2):  # problem 0 alone: 18 groups, split
        o = dev(np.zeros(Lq * H * D))
        attn(gpu, q=qd, k=kvd, v=kvd, out=o, Lq=Lq, Lk=Lk, H=H, D=D, ldq=H * D, ldk=2 * H * D, ldv=2 * H * D, kOff=0,
             vOff=H * D)
        gpu.sync()
        outs.append(host(o))
    np.testing.assert_array_equal(outs[0], outs[1])
    big = dev(np.zeros(n * Lq * H * D))
    descs = (supra_attn.Desc * n)()
    for b in range(n):  # 720 groups: not split
        descs[b] = supra_attn.make_desc(q=qd, k=kvd, v=kvd, out=big, Lq=Lq, Lk=Lk, H=H, D=D, ldq=H * D, ldk=2 * H * D,
                                        ldv=2 * H * D, qOff=b * Lq * H * D, kOff=b * Lk * 2 * H * D,
                                        vOff=b * Lk * 2 * H * D + H * D, oOff=b * Lq * H * D)
    gpu.enqueue_batch(descs)
    gpu.sync()
    got = host(big)
    assert_close(got[: Lq * H * D], outs[0])
    x = kv[: Lk * 2 * H * D].reshape(Lk, 2 * H * D)
    assert_close(outs[0], oracle.attention_heads(q[: Lq * H * D].reshape(Lq, H * D), x[:, : H * D], x[:, H * D:], H))


def test_batch_hazards_fall_back_to_ordered_recording(gpu):
    """supra_attn_enqueue_batch records a conflict-free batch in one merge; a batch whose problems
    depend on each other is recorded in order with a flush at each hazard, as single calls are:
    (1) problem 1 reads problem 0's output (read after write), (2) problems 0 and 2 write the same
    output (the later one wins), (3) a batch reading an output still queued from an earlier call."""
    import supra_attn

    rng = np.random.default_rng(12)
    H, D, L = 2, 64, 70
    ld = H * D
    q, k, v = (rng.standard_normal(L * ld).astype(np.float32) for _ in range(3))
    k2 = rng.standard_normal(L * ld).astype(np.float32)
    qd, kd, vd, k2d = dev(q), dev(k), dev(v), dev(k2)
    o1, o2, o3 = (dev(np.zeros(L * ld)) for _ in range(3))
    kw = dict(Lq=L, Lk=L, H=H, D=D, ldq=ld, ldk=ld, ldv=ld)
    r1 = oracle.attention_ops(q, k, v, L, L, H, D, ld, ld, ld)
    r2 = oracle.attention_ops(r1, k, v, L, L, H, D, ld, ld, ld)
    r3 = oracle.attention_ops(q, k2, v, L, L, H, D, ld, ld, ld)
    # (1) and (2) in one batch: o1 = A(q); o2 = A(o1); o1 = A(q, k2) (overwrites o1 after o2 read it)
    descs = (supra_attn.Desc * 3)(supra_attn.make_desc(q=qd, k=kd, v=vd, out=o1, **kw),
                                  supra_attn.make_desc(q=o1, k=kd, v=vd, out=o2, **kw),
                                  supra_attn.make_desc(q=qd, k=k2d, v=vd, out=o1, **kw))
    gpu.enqueue_batch(descs)
    gpu.sync()
    assert_close(host(o2), r2)
    assert_close(host(o1), r3)
    # (3) a queued single call, then a batch that reads its output and a conflict-free problem
    attn(gpu, q=qd, k=kd, v=vd, out=o3, **kw)
    descs = (supra_attn.Desc * 2)(supra_attn.make_desc(q=o3, k=kd, v=vd, out=o2, **kw),
                                  supra_attn.make_desc(q=qd, k=k2d, v=vd, out=o1, **kw))
    gpu.enqueue_batch(descs)
    gpu.sync()
    assert_close(host(o2), r2)
    assert_close(host(o1), r3)
    # (4) a conflict-free batch (its ranges recorded unsorted), then a single call reading its
    # output and a batch writing what the first batch read: both must see the batch's ranges
    descs = (supra_attn.Desc * 2)(supra_attn.make_desc(q=qd, k=k2d, v=vd, out=o3, **kw),
                                  supra_attn.make_desc(q=qd, k=kd, v=vd, out=o1, **kw))
    gpu.enqueue_batch(descs)
    attn(gpu, q=o1, k=kd, v=vd, out=o2, **kw)  # reads o1 (read after write)
    descs = (supra_attn.Desc * 1)(supra_attn.make_desc(q=o3, k=kd, v=vd, out=k2d, **kw))  # writes k2 (after read)
    gpu.enqueue_batch(descs)
    gpu.sync()
    assert_close(host(o3), r3)
    assert_close(host(o1), r1)
    assert_close(host(o2), r2)
    assert_close(host(k2d), oracle.attention_ops(r3, k, v, L, L, H, D, ld, ld, ld))


@pytest.mark.parametrize("Lq,Lk,H,D,bias", [
    (1024, 2048, 1, 256, False),  # 8 x 16 tiles of 128 rows: 64-row tiles (256 of them)
    (1000, 2000, 1, 192, True),   # the same with a bias and a ragged last row tile
    (1024, 1024, 1, 512, False),  # one VAE image: 32-row tiles
])
def test_score_path_small_launch_tiles(gpu, Lq, Lk, H, D, bias):
    """The FFMA score path (head dims above 128) takes 64- or 32-row tiles when a launch has
    fewer 128-row Q K^T tiles than SMs; against the float64 oracle."""
    rng = np.random.default_rng(Lq + D)
    run_and_check(gpu, rand_problem(rng, Lq, Lk, H, D, bias=bias), scale=(64.0 / D) ** 0.5 if bias else None)
