"""TF32 tensor-core kernel (tcgen05) through the C ABI against the oracle and golden vectors.

TF32 bar (its own stated tolerance, "<= 2e-3 relative on attention output"): rel-L2 <= 2e-3 per
output tensor, the reference's own parity metric (tools/check.js:31-44), plus a sanity bound of
5e-3 on the normwise max error max|got - ref| / max|ref| (TF32 operands carry 2^-11 relative
rounding; T5's unscaled scores of standard deviation 8 turn that into ~2e-3 normwise max error). Head dims above 128 run the score path's two products on the tensor-core linear (TF32 bar).
Other requests the tensor-core attention kernel does not cover (head dims up to 128 other than 64,
rows that are not whole buffer rows) run the FP32 kernels and are held to the FP32 bar (1e-5).
"""

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL_TF32 = 2e-3      # rel-L2
TOL_TF32_MAX = 5e-3  # normwise max error, sanity bound
TOL_FP32 = 1e-5


def dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32)).reshape(-1)).cuda()


def host(t):
    return t.detach().cpu().numpy().reshape(-1)


def check(got, ref, tol):
    mr, rl = oracle.max_rel(got, ref), oracle.rel_l2(got, ref)
    max_tol = TOL_TF32_MAX if tol == TOL_TF32 else tol
    assert rl <= tol and mr <= max_tol, f"max_rel={mr:.3e} rel_l2={rl:.3e} (tol {tol}, max {max_tol})"
    return mr, rl


def kernel_names(gpu):
    return {r["name"] for r in gpu.profile_report()}


def test_dit_self_config1_tf32(gpu, golden):
    import torch

    import supra_attn

    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(2, 256, 1728, generator=g).reshape(-1).cuda()
    out = torch.zeros(2 * 256 * 576, device="cuda")
    gpu.profile(True)
    gpu.profile_reset()
    for b in range(2):
        r = b * 256 * 1728
        supra_attn.attention(gpu, q=qkv, k=qkv, v=qkv, Lq=256, Lk=256, H=9, D=64, ldq=1728, ldk=1728, ldv=1728,
                             qOff=r, kOff=r + 576, vOff=r + 1152, oOff=b * 256 * 576, out=out, variant="tf32")
    gpu.sync()
    names = kernel_names(gpu)
    gpu.profile(False)
    assert "attn_tf32_d64" in names, names
    check(host(out), golden("dit_self_cfg1_out"), TOL_TF32)


def test_dit_cross_ragged_tf32(gpu, golden):
    import supra_attn

    c = golden.cases["dit_cross"]
    N = c["N"]
    q = dev(golden("dit_cross_q"))
    out = dev(np.zeros(len(c["Ls"]) * N * 576))
    kvs = [dev(golden(f"dit_cross_kv{b}")) for b in range(len(c["Ls"]))]
    for b, L in enumerate(c["Ls"]):
        supra_attn.attention(gpu, q=q, k=kvs[b], v=kvs[b], Lq=N, Lk=L, H=9, D=64, ldq=576, ldk=1152, ldv=1152,
                             qOff=b * N * 576, kOff=0, vOff=576, oOff=b * N * 576, out=out, variant="tf32")
    gpu.sync()
    ref = golden("dit_cross_out")
    got = host(out).reshape(ref.shape)
    for b in range(len(c["Ls"])):
        check(got[b], ref[b], TOL_TF32)


@pytest.mark.parametrize(
    "Lq,Lk,H",
    [(1, 1, 1), (100, 63, 2), (128, 64, 1), (129, 65, 3), (256, 256, 9), (300, 1000, 2), (64, 4096, 1), (7, 200, 4)],
)
def test_shapes_tf32(gpu, Lq, Lk, H):
    import supra_attn

    rng = np.random.default_rng(Lq * 7 + Lk)
    HD = H * 64
    q = rng.standard_normal(Lq * HD).astype(np.float32)
    k = rng.standard_normal(Lk * HD).astype(np.float32)
    v = rng.standard_normal(Lk * HD).astype(np.float32)
    o = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=64, ldq=HD, ldk=HD, ldv=HD,
                             variant="tf32")
    got = gpu.read(o)
    o.release()
    check(got, oracle.attention_ops(q, k, v, Lq, Lk, H, 64, HD, HD, HD), TOL_TF32)


def test_tf32_requests_outside_the_tensor_core_kernel_run_fp32(gpu):
    """Head dim 32 and a last row shorter than ld run the FP32 kernels (1e-5)."""
    import supra_attn

    rng = np.random.default_rng(3)
    gpu.profile(True)
    gpu.profile_reset()
    # head dim 32
    q, k, v = (rng.standard_normal(n).astype(np.float32) for n in (70 * 64, 90 * 64, 90 * 64))
    o = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=70, Lk=90, H=2, D=32, ldq=64, ldk=64, ldv=64,
                             variant="tf32")
    check(gpu.read(o), oracle.attention_ops(q, k, v, 70, 90, 2, 32, 64, 64, 64), TOL_FP32)
    # padded rows with a short last row (buffer of (Lq-1)*ld + H*D floats)
    q = rng.standard_normal(69 * 132 + 128).astype(np.float32)
    k = rng.standard_normal(89 * 132 + 128).astype(np.float32)
    v = rng.standard_normal(89 * 132 + 128).astype(np.float32)
    o3 = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=70, Lk=90, H=2, D=64, ldq=132, ldk=132, ldv=132,
                              variant="tf32")
    check(gpu.read(o3), oracle.attention_ops(q, k, v, 70, 90, 2, 64, 132, 132, 132), TOL_FP32)
    names = kernel_names(gpu)
    gpu.profile(False)
    assert not any(n.startswith("attn_tf32") for n in names), names
    for t in (o, o3):
        t.release()


@pytest.mark.parametrize("Lq,Lk", [(1, 1), (70, 90), (129, 200), (256, 64)])
def test_bias_tf32(gpu, Lq, Lk):
    import supra_attn

    rng = np.random.default_rng(Lq + Lk)
    H = 3
    b = (rng.standard_normal(H * Lq * Lk) * 2).astype(np.float32)
    q, k, v = (rng.standard_normal(n).astype(np.float32) for n in (Lq * H * 64, Lk * H * 64, Lk * H * 64))
    gpu.profile(True)
    gpu.profile_reset()
    o = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=64, ldq=H * 64, ldk=H * 64,
                             ldv=H * 64, bias=dev(b), scale=0.125, variant="tf32")
    got = gpu.read(o)
    names = kernel_names(gpu)
    gpu.profile(False)
    assert "attn_tf32_d64_bias" in names, names
    check(got, oracle.attention_ops(q, k, v, Lq, Lk, H, 64, H * 64, H * 64, H * 64, scale=0.125, bias=b), TOL_TF32)
    o.release()


@pytest.mark.parametrize("L", [1, 5, 37, 128])
def test_t5_golden_tf32(gpu, golden, L):
    """The T5 call site (unscaled scores, relative-position bias) through the tensor cores."""
    import supra_attn

    table = dev(golden("t5_table"))
    bias = supra_attn.position_bias(gpu, table, L, H=12)
    q, k, v = (dev(golden(f"t5_L{L}_{n}")) for n in "qkv")
    o = supra_attn.attention(gpu, q=q, k=k, v=v, Lq=L, Lk=L, H=12, D=64, ldq=768, ldk=768, ldv=768, scale=1.0,
                             bias=bias, variant="tf32")
    check(gpu.read(o), golden(f"t5_L{L}_out"), TOL_TF32)
    o.release()
    bias.release()


@pytest.mark.parametrize("L", [5, 128, 300])
def test_t5_table_tf32(gpu, golden, L):
    """The T5 table in place of the expanded bias on the tensor-core kernel: same bits as the
    expanded-bias call, and within the TF32 bar of the oracle (L = 300 clamps beyond max_distance)."""
    import supra_attn

    rng = np.random.default_rng(L)
    table = golden("t5_table").reshape(-1).astype(np.float32)
    q, k, v = (rng.standard_normal(L * 768).astype(np.float32) for _ in range(3))
    td = dev(table)
    kw = dict(q=dev(q), k=dev(k), v=dev(v), Lq=L, Lk=L, H=12, D=64, ldq=768, ldk=768, ldv=768, scale=0.125,
              variant="tf32")
    gpu.profile(True)
    gpu.profile_reset()
    o_tab = supra_attn.attention(gpu, t5_table=td, **kw)
    got = gpu.read(o_tab)
    names = [r["name"] for r in gpu.profile_report()]
    gpu.profile(False)
    assert names == ["attn_tf32_d64_bias"], names
    bias = supra_attn.position_bias(gpu, td, L, H=12)
    o_exp = supra_attn.attention(gpu, bias=bias, **kw)
    np.testing.assert_array_equal(got, gpu.read(o_exp))
    ref_bias = oracle.position_bias(table, L, 12, 32, 128).reshape(-1)
    check(got, oracle.attention_ops(q, k, v, L, L, 12, 64, 768, 768, 768, scale=0.125, bias=ref_bias), TOL_TF32)
    for t in (o_tab, o_exp, bias):
        t.release()


def test_tf32_determinism(gpu):
    import supra_attn

    rng = np.random.default_rng(8)
    q, k, v = (dev(rng.standard_normal(300 * 576)) for _ in range(3))
    outs = []
    for _ in range(2):
        o = supra_attn.attention(gpu, q=q, k=k, v=v, Lq=300, Lk=300, H=9, D=64, ldq=576, ldk=576, ldv=576,
                                 variant="tf32")
        outs.append(gpu.read(o))
        o.release()
    np.testing.assert_array_equal(outs[0], outs[1])


def test_config2_cross_tf32(gpu):
    """Config 2 at full size through the TF32 kernel: 128 ragged sequences, 2304 tiles, so every
    persistent CTA runs several tiles back to back with key blocks flowing across tile boundaries."""
    import torch

    import supra_attn

    g = torch.Generator().manual_seed(12)
    Ls = torch.randint(1, 129, (128,), generator=g).tolist()
    q = torch.randn(128 * 256 * 576, generator=g)
    kvs = [torch.randn(L * 1152, generator=g) for L in Ls]
    qd = q.cuda()
    kvd = [x.cuda() for x in kvs]
    out = torch.zeros(128 * 256 * 576, device="cuda")
    descs = (supra_attn.Desc * 128)()
    for b, L in enumerate(Ls):
        descs[b] = supra_attn.make_desc(q=qd, k=kvd[b], v=kvd[b], out=out, Lq=256, Lk=L, H=9, D=64, ldq=576,
                                        ldk=1152, ldv=1152, qOff=b * 256 * 576, kOff=0, vOff=576, oOff=b * 256 * 576,
                                        variant="tf32")
    gpu.enqueue_batch(descs)
    gpu.sync()
    got = host(out).reshape(128, 256, 576)
    qn = q.numpy().reshape(128, 256, 576)
    for b in range(0, 128, 7):
        kv = kvs[b].numpy().reshape(-1, 1152)
        check(got[b], oracle.attention_heads(qn[b], kv[:, :576], kv[:, 576:], 9), TOL_TF32)


@pytest.mark.parametrize("Lq,Lk,H,D", [(64, 96, 1, 512), (33, 77, 1, 192), (130, 260, 2, 256), (70, 70, 2, 130)])
def test_score_path_on_tensor_cores_tf32(gpu, Lq, Lk, H, D):
    """Head dims above 128 (the VAE mid-block, app/models/vae.js:86) run S = Q K^T and O = P V on
    the tensor-core linear with TF32 operands (Q, K and P read in place where 16-byte aligned) and
    the row softmax between them, held to the TF32 bar."""
    import supra_attn

    rng = np.random.default_rng(Lq + Lk + D)
    HD = H * D
    q = rng.standard_normal(Lq * HD).astype(np.float32)
    k = rng.standard_normal(Lk * HD).astype(np.float32)
    v = rng.standard_normal(Lk * HD).astype(np.float32)
    gpu.profile(True)
    gpu.profile_reset()
    o = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=D, ldq=HD, ldk=HD, ldv=HD,
                             variant="tf32")
    got = gpu.read(o)
    names = kernel_names(gpu)
    gpu.profile(False)
    o.release()
    check(got, oracle.attention_ops(q, k, v, Lq, Lk, H, D, HD, HD, HD), TOL_TF32)
    assert "linear_tc_tf32" in names and "attn_gemm_qk" not in names, names
