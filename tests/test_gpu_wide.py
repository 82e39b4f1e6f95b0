"""The 256-row persistent FP32 kernel (csrc/attn_fp32_wide.cu) against the float64 oracle.

Unbiased D = 64 launches that hold at least one 256-row tile per SM run on it (the DiT self- and
cross-attention batches, app/models/dit.js:172,184); smaller ones on the 128-row kernel. The bar is
the FP32 one: max_rel and rel_l2 <= 1e-5 per problem.
"""

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _torch():
    import torch

    return torch


def assert_close(got, ref, tol=TOL):
    mr, rl = oracle.max_rel(got, ref), oracle.rel_l2(got, ref)
    assert mr <= tol and rl <= tol, f"max_rel={mr:.3e} rel_l2={rl:.3e} (tol {tol})"


def _run(gpu, descs):
    gpu.profile(True)
    gpu.profile_reset()
    gpu.enqueue_batch(descs)
    gpu.sync()
    names = [r["name"] for r in gpu.profile_report()]
    gpu.profile(False)
    return names


def test_wide_dit_self_batch_deterministic(gpu):
    """40 DiT self-attention sequences (Lq = Lk = 256, 9 x 64 heads, packed qkv rows of 1728): 360
    tiles of 256 rows, every sequence against the oracle, and a second launch bit-identical."""
    torch = _torch()
    import supra_attn

    n = 40
    g = torch.Generator().manual_seed(31)
    qkv = torch.randn(n * 256 * 1728, generator=g)
    qkvd = qkv.cuda()
    outs = []
    for _ in range(2):
        out = torch.full((n * 256 * 576,), 7.0, device="cuda")
        descs = (supra_attn.Desc * n)()
        for b in range(n):
            r = b * 256 * 1728
            descs[b] = supra_attn.make_desc(q=qkvd, k=qkvd, v=qkvd, out=out, Lq=256, Lk=256, H=9, D=64, ldq=1728,
                                            ldk=1728, ldv=1728, qOff=r, kOff=r + 576, vOff=r + 1152,
                                            oOff=b * 256 * 576)
        assert _run(gpu, descs) == ["attn_fp32_d64_wide"]
        outs.append(out.cpu().numpy())
    np.testing.assert_array_equal(outs[0], outs[1])
    got = outs[0].reshape(n, 256, 576)
    x = qkv.numpy().reshape(n, 256, 1728)
    for b in range(n):
        assert_close(got[b], oracle.attention_heads(x[b, :, :576], x[b, :, 576:1152], x[b, :, 1152:], 9))


# key lengths around every block edge: 32-key halves, 64-key blocks, several blocks
_EDGE_LK = [1, 2, 3, 4, 5, 31, 32, 33, 36, 63, 64, 65, 95, 96, 97, 127, 128, 129, 160, 191, 192, 193, 255, 256,
            257, 300, 383, 384, 385, 511, 512, 513, 640, 700, 1000, 1023]


def test_wide_ragged_lengths_nan_past_ends(gpu):
    """36 problems (Lq = 200, so the last warp's rows all lie past Lq and the one before it holds
    8 rows) with the key lengths around every 32/64-key edge; rows past Lq in Q and past Lk in K/V
    hold NaN/inf. No output may change and nothing past Lq may be written."""
    torch = _torch()
    import supra_attn

    rng = np.random.default_rng(32)
    H, D, Lq, pad = 9, 64, 200, 40
    C = H * D
    n = len(_EDGE_LK)
    q = rng.standard_normal((n, Lq + pad, C)).astype(np.float32)
    q[:, Lq:] = np.nan
    kv_off = np.concatenate([[0], np.cumsum([(L + pad) * 2 * C for L in _EDGE_LK])]).astype(np.int64)
    kv = rng.standard_normal(int(kv_off[-1])).astype(np.float32)
    for b, L in enumerate(_EDGE_LK):
        x = kv[kv_off[b]: kv_off[b + 1]].reshape(L + pad, 2 * C)
        x[L:, :C] = np.inf  # K rows past Lk
        x[L:, C:] = np.nan  # V rows past Lk
    qd = torch.from_numpy(q.reshape(-1)).cuda()
    kvd = torch.from_numpy(kv).cuda()
    out = torch.full((n * (Lq + pad) * C,), 7.0, device="cuda")
    descs = (supra_attn.Desc * n)()
    for b, L in enumerate(_EDGE_LK):
        descs[b] = supra_attn.make_desc(q=qd, k=kvd, v=kvd, out=out, Lq=Lq, Lk=L, H=H, D=D, ldq=C, ldk=2 * C,
                                        ldv=2 * C, qOff=b * (Lq + pad) * C, kOff=int(kv_off[b]),
                                        vOff=int(kv_off[b]) + C, oOff=b * (Lq + pad) * C)
    assert _run(gpu, descs) == ["attn_fp32_d64_wide"]
    got = out.cpu().numpy().reshape(n, Lq + pad, C)
    for b, L in enumerate(_EDGE_LK):
        x = kv[kv_off[b]: kv_off[b + 1]].reshape(L + pad, 2 * C)
        assert_close(got[b, :Lq], oracle.attention_heads(q[b, :Lq], x[:L, :C], x[:L, C:], H))
        assert np.all(got[b, Lq:] == 7.0), f"problem {b} (Lk {L}) wrote past Lq"


def test_wide_mixed_heads_and_scales(gpu):
    """Problems of 9 and 4 heads (tile counts differ per problem, so tiles map to problems by search),
    Lq 256 and 240, explicit scales, and query/key/value in separate buffers with their own row
    strides and offsets."""
    torch = _torch()
    import supra_attn

    rng = np.random.default_rng(33)
    specs = [(9 if b % 3 else 4, 256 if b % 2 else 240, int(rng.integers(1, 300)), float(rng.uniform(0.05, 0.3)))
             for b in range(60)]
    D = 64
    descs = (supra_attn.Desc * len(specs))()
    keep, outs = [], []
    for b, (H, Lq, Lk, scale) in enumerate(specs):
        C = H * D
        ldq, ldk, ldv = C + 16, C + 8, C + 20  # padded row strides; each offset + H * D fits in a row
        q = rng.standard_normal(Lq * ldq + 16).astype(np.float32)
        k = rng.standard_normal(Lk * ldk + 8).astype(np.float32)
        v = rng.standard_normal(Lk * ldv + 20).astype(np.float32)
        qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
        out = torch.full((Lq * C + 4,), 7.0, device="cuda")
        keep.append((qd, kd, vd, out))
        outs.append(out)
        descs[b] = supra_attn.make_desc(q=qd, k=kd, v=vd, out=out, Lq=Lq, Lk=Lk, H=H, D=D, ldq=ldq, ldk=ldk,
                                        ldv=ldv, qOff=16, kOff=8, vOff=20, oOff=4, scale=scale)
        specs[b] = (H, Lq, Lk, scale, q, k, v)
    tiles = sum(H for H, *_ in specs)
    assert tiles >= 2 * 148
    assert _run(gpu, descs) == ["attn_fp32_d64_wide"]
    for b, (H, Lq, Lk, scale, q, k, v) in enumerate(specs):
        C = H * D
        ldq, ldk, ldv = C + 16, C + 8, C + 20
        qm = q[16: 16 + Lq * ldq].reshape(Lq, ldq)[:, :C]
        km = k[8: 8 + Lk * ldk].reshape(Lk, ldk)[:, :C]
        vm = v[20: 20 + Lk * ldv].reshape(Lk, ldv)[:, :C]
        got = outs[b].cpu().numpy()
        assert np.all(got[:4] == 7.0)
        assert_close(got[4:], oracle.attention_heads(qm, km, vm, H, scale=scale).reshape(-1))


@pytest.mark.parametrize("n,Lq,expect", [
    (16, 256, "attn_fp32_d64_tma"),   # 144 tiles: under one per SM
    (17, 256, "attn_fp32_d64_wide"),  # 153 tiles
    (32, 256, "attn_fp32_d64_wide"),  # 288 tiles (the DiT block of 32 images)
    (40, 300, "attn_fp32_d64_tma"),   # 300 rows: 512 rows in 256-row tiles against 384 in 128-row ones
    (40, 129, "attn_fp32_d64_wide"),  # 129 rows: 256 either way
])
def test_wide_selection(gpu, n, Lq, expect):
    torch = _torch()
    import supra_attn

    g = torch.Generator().manual_seed(34)
    q = torch.randn(n * Lq * 576, generator=g)
    kv = torch.randn(n * 77 * 1152, generator=g)
    qd, kvd = q.cuda(), kv.cuda()
    out = torch.zeros(n * Lq * 576, device="cuda")
    descs = (supra_attn.Desc * n)()
    for b in range(n):
        descs[b] = supra_attn.make_desc(q=qd, k=kvd, v=kvd, out=out, Lq=Lq, Lk=77, H=9, D=64, ldq=576, ldk=1152,
                                        ldv=1152, qOff=b * Lq * 576, kOff=b * 77 * 1152, vOff=b * 77 * 1152 + 576,
                                        oOff=b * Lq * 576)
    assert _run(gpu, descs) == [expect]
    got = out.cpu().numpy().reshape(n, Lq, 576)
    qn, kvn = q.numpy().reshape(n, Lq, 576), kv.numpy().reshape(n, 77, 1152)
    for b in (0, n // 2, n - 1):
        assert_close(got[b], oracle.attention_heads(qn[b], kvn[b, :, :576], kvn[b, :, 576:], 9))


@pytest.mark.parametrize("Lq,Lk", [(512, 300), (1000, 77)])
def test_wide_several_query_tiles(gpu, Lq, Lk):
    """Problems of several 256-row tiles (the last one partial at Lq = 1000), each tile claimed on
    its own; sampled problems against the oracle, and nothing written past Lq."""
    torch = _torch()
    import supra_attn

    n, H, C = 20, 9, 576
    g = torch.Generator().manual_seed(35)
    q = torch.randn(n * (Lq + 8) * C, generator=g)
    kv = torch.randn(n * Lk * 2 * C, generator=g)
    qd, kvd = q.cuda(), kv.cuda()
    out = torch.full((n * (Lq + 8) * C,), 7.0, device="cuda")
    descs = (supra_attn.Desc * n)()
    for b in range(n):
        descs[b] = supra_attn.make_desc(q=qd, k=kvd, v=kvd, out=out, Lq=Lq, Lk=Lk, H=H, D=64, ldq=C, ldk=2 * C,
                                        ldv=2 * C, qOff=b * (Lq + 8) * C, kOff=b * Lk * 2 * C,
                                        vOff=b * Lk * 2 * C + C, oOff=b * (Lq + 8) * C)
    assert _run(gpu, descs) == ["attn_fp32_d64_wide"]
    got = out.cpu().numpy().reshape(n, Lq + 8, C)
    qn, kvn = q.numpy().reshape(n, Lq + 8, C), kv.numpy().reshape(n, Lk, 2 * C)
    for b in (0, 7, n - 1):
        assert_close(got[b, :Lq], oracle.attention_heads(qn[b, :Lq], kvn[b, :, :C], kvn[b, :, C:], H))
    assert np.all(got[:, Lq:] == 7.0)
