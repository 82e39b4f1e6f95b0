"""Split-precision tensor-core kernel (variant "tf32x3": every operand split into a TF32 part and
its remainder, each product formed from three tcgen05 TF32 products) through the C ABI, held to
the FP32 bar: max|got - ref| / max|ref| <= 1e-5 and rel-L2 <= 1e-5 per output tensor, against
the oracle and the reference's golden vectors."""

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-5


def dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32)).reshape(-1)).cuda()


def host(t):
    return t.detach().cpu().numpy().reshape(-1)


def check(got, ref, tol=TOL):
    mr, rl = oracle.max_rel(got, ref), oracle.rel_l2(got, ref)
    assert mr <= tol and rl <= tol, f"max_rel={mr:.3e} rel_l2={rl:.3e} (tol {tol})"


def names_of(gpu):
    return {r["name"] for r in gpu.profile_report()}


def test_dit_self_config1(gpu, golden):
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
                             qOff=r, kOff=r + 576, vOff=r + 1152, oOff=b * 256 * 576, out=out, variant="tf32x3")
    gpu.sync()
    names = names_of(gpu)
    gpu.profile_reset()
    gpu.profile(False)
    assert names == {"attn_tf32x3_d64"}, names
    check(host(out), golden("dit_self_cfg1_out"))


def test_dit_cross_ragged(gpu, golden):
    import supra_attn

    c = golden.cases["dit_cross"]
    N = c["N"]
    q = dev(golden("dit_cross_q"))
    out = dev(np.zeros(len(c["Ls"]) * N * 576))
    kvs = [dev(golden(f"dit_cross_kv{b}")) for b in range(len(c["Ls"]))]
    for b, L in enumerate(c["Ls"]):
        supra_attn.attention(gpu, q=q, k=kvs[b], v=kvs[b], Lq=N, Lk=L, H=9, D=64, ldq=576, ldk=1152, ldv=1152,
                             qOff=b * N * 576, kOff=0, vOff=576, oOff=b * N * 576, out=out, variant="tf32x3")
    gpu.sync()
    ref = golden("dit_cross_out")
    got = host(out).reshape(ref.shape)
    for b in range(len(c["Ls"])):
        check(got[b], ref[b])


@pytest.mark.parametrize(
    "Lq,Lk,H",
    [(1, 1, 1), (100, 63, 2), (128, 64, 1), (129, 65, 3), (256, 256, 9), (300, 1000, 2), (64, 4096, 1), (7, 200, 4)],
)
def test_shapes(gpu, Lq, Lk, H):
    import supra_attn

    rng = np.random.default_rng(Lq * 7 + Lk + 1)
    HD = H * 64
    q = rng.standard_normal(Lq * HD).astype(np.float32)
    k = rng.standard_normal(Lk * HD).astype(np.float32)
    v = rng.standard_normal(Lk * HD).astype(np.float32)
    o = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=64, ldq=HD, ldk=HD, ldv=HD,
                             variant="tf32x3")
    got = gpu.read(o)
    o.release()
    check(got, oracle.attention_ops(q, k, v, Lq, Lk, H, 64, HD, HD, HD))


def test_large_scores(gpu):
    """Scores of standard deviation ~16 (inputs scaled by 4, scale 1/8): the softmax is sharp, and
    the split still holds the FP32 bar."""
    import supra_attn

    rng = np.random.default_rng(21)
    Lq, Lk, H = 200, 300, 3
    HD = H * 64
    q, k, v = ((rng.standard_normal(n) * s).astype(np.float32) for n, s in ((Lq * HD, 4), (Lk * HD, 4), (Lk * HD, 1)))
    o = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=64, ldq=HD, ldk=HD, ldv=HD,
                             variant="tf32x3")
    got = gpu.read(o)
    o.release()
    check(got, oracle.attention_ops(q, k, v, Lq, Lk, H, 64, HD, HD, HD))


@pytest.mark.parametrize("L", [1, 5, 37, 128])
def test_t5_golden(gpu, golden, L):
    """T5 (unscaled scores of standard deviation ~8, relative-position bias) at the FP32 bar."""
    import supra_attn

    table = dev(golden("t5_table"))
    q, k, v = (dev(golden(f"t5_L{L}_{n}")) for n in "qkv")
    gpu.profile(True)
    gpu.profile_reset()
    o = supra_attn.attention(gpu, q=q, k=k, v=v, Lq=L, Lk=L, H=12, D=64, ldq=768, ldk=768, ldv=768, scale=1.0,
                             t5_table=table, variant="tf32x3")
    got = gpu.read(o)
    names = names_of(gpu)
    gpu.profile_reset()
    gpu.profile(False)
    assert names == {"attn_tf32x3_d64_bias"}, names
    check(got, golden(f"t5_L{L}_out"))
    o.release()


def test_expanded_bias(gpu):
    import supra_attn

    rng = np.random.default_rng(6)
    Lq, Lk, H = 129, 200, 3
    b = (rng.standard_normal(H * Lq * Lk) * 2).astype(np.float32)
    q, k, v = (rng.standard_normal(n).astype(np.float32) for n in (Lq * H * 64, Lk * H * 64, Lk * H * 64))
    o = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=64, ldq=H * 64, ldk=H * 64,
                             ldv=H * 64, bias=dev(b), scale=0.125, variant="tf32x3")
    got = gpu.read(o)
    o.release()
    check(got, oracle.attention_ops(q, k, v, Lq, Lk, H, 64, H * 64, H * 64, H * 64, scale=0.125, bias=b))


def test_determinism_and_nan_rows_past_lengths(gpu):
    """Bit-identical on a rerun; NaNs in buffer rows past Lk (another sequence's rows) reach no output."""
    import supra_attn

    rng = np.random.default_rng(8)
    Lq, Lk, ld = 300, 77, 576
    q = dev(rng.standard_normal(Lq * ld))
    kvh = rng.standard_normal(128 * ld).astype(np.float32)
    kvh[Lk * ld:] = np.nan
    k = dev(kvh)
    outs = []
    for _ in range(2):
        o = supra_attn.attention(gpu, q=q, k=k, v=k, Lq=Lq, Lk=Lk, H=9, D=64, ldq=ld, ldk=ld, ldv=ld,
                                 variant="tf32x3")
        outs.append(gpu.read(o))
        o.release()
    np.testing.assert_array_equal(outs[0], outs[1])
    assert np.isfinite(outs[0]).all()
    check(outs[0], oracle.attention_ops(host(q), kvh, kvh, Lq, Lk, 9, 64, ld, ld, ld))


def test_config2_cross_full_size(gpu):
    """128 ragged sequences (2304 tiles): every persistent CTA runs many tiles back to back."""
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
                                        variant="tf32x3")
    gpu.enqueue_batch(descs)
    gpu.sync()
    got = host(out).reshape(128, 256, 576)
    qn = q.numpy().reshape(128, 256, 576)
    for b in range(0, 128, 7):
        kv = kvs[b].numpy().reshape(-1, 1152)
        check(got[b], oracle.attention_heads(qn[b], kv[:, :576], kv[:, 576:], 9))


def vae_like(rng, T, nimg):
    """Config 4's value distribution: x ~ N(0,1), Q/K/V = x W^T with W Xavier-uniform (512 x 512),
    so scores q.k / sqrt(512) have standard deviation ~1."""
    bound = (6.0 / 1024) ** 0.5
    x = rng.standard_normal((nimg * T, 512)).astype(np.float32)
    return [(x @ rng.uniform(-bound, bound, (512, 512)).astype(np.float32).T).reshape(-1) for _ in range(3)]


@pytest.mark.parametrize(
    "Lq,Lk,H,D",
    [(64, 96, 1, 512), (33, 77, 1, 192), (130, 260, 2, 256), (70, 70, 2, 130), (70, 70, 4, 134), (200, 70, 2, 258),
     (300, 31, 1, 512)],
)
def test_score_path_on_tensor_cores(gpu, Lq, Lk, H, D):
    """Head dims above 128 (the VAE mid-block's one head of 512, app/models/vae.js:86) run the
    score path's two products, S = Q K^T and O = P V, on the tensor-core linear with the split
    operands, and the row softmax (which applies the scale and writes P split) between them;
    ragged Lk (ld of the scores a multiple of 4 above Lk) and several heads included; head dims
    that are not a multiple of 4 put a head's first columns in the 16-byte chunk of the previous
    head's last ones. Lk < 32 stays on the FFMA GEMMs."""
    import supra_attn

    rng = np.random.default_rng(Lq * 3 + Lk * 5 + D)
    HD = H * D
    q = rng.standard_normal(Lq * HD).astype(np.float32)
    k = rng.standard_normal(Lk * HD).astype(np.float32)
    v = rng.standard_normal(Lk * HD).astype(np.float32)
    gpu.profile(True)
    gpu.profile_reset()
    o = supra_attn.attention(gpu, q=dev(q), k=dev(k), v=dev(v), Lq=Lq, Lk=Lk, H=H, D=D, ldq=HD, ldk=HD, ldv=HD,
                             variant="tf32x3")
    got = gpu.read(o)
    names = names_of(gpu)
    gpu.profile(False)
    o.release()
    check(got, oracle.attention_ops(q, k, v, Lq, Lk, H, D, HD, HD, HD))
    if Lk >= 32:
        assert "linear_tc_tf32x3" in names and "attn_softmax_rows" in names, names
        assert "attn_gemm_qk" not in names and "attn_gemm_pv" not in names, names
    else:
        assert "attn_gemm_qk" in names, names


def test_vae_full_size_on_tensor_cores(gpu):
    """Config 4 at full size: 2 images of 32 x 32 latents (Lq = Lk = 1024, H = 1, D = 512) in one
    flush, each image's rows at its own offset, at the FP32 bar per image."""
    import supra_attn

    rng = np.random.default_rng(4)
    T, nimg = 1024, 2
    q, k, v = vae_like(rng, T, nimg)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = dev(np.zeros(nimg * T * 512))
    for i in range(nimg):
        o = i * T * 512
        supra_attn.attention(gpu, q=qd, k=kd, v=vd, Lq=T, Lk=T, H=1, D=512, ldq=512, ldk=512, ldv=512, qOff=o,
                             kOff=o, vOff=o, oOff=o, out=out, variant="tf32x3")
    got = gpu.read(out)
    for i in range(nimg):
        s = slice(i * T * 512, (i + 1) * T * 512)
        check(got[s], oracle.attention_ops(q[s], k[s], v[s], T, T, 1, 512, 512, 512, 512))
