"""supra_attn_attention_noalloc: attention for callers that cannot allocate device memory.

Such callers are hosts whose allocator has reserved the GPU's memory up front, and code on a
latency-critical path that must not call cudaMalloc/cudaFree because those can synchronise
the device. The entry point keeps its score scratch in a fixed 16 MiB static device array
instead of allocating it. These tests call it through the C ABI and check that two calls
in a row give the same results, within the FP32 tolerance, as the regular recorded entry
point (supra_attn_enqueue + sync) on the same inputs. The file is named to be collected last.
"""

import ctypes as C

import numpy as np
import pytest

import oracle
import supra_attn
from supra_attn import _lib

TOL = 1e-5


def noalloc(desc, stream):
    msg = C.create_string_buffer(256)
    st = _lib.lib.supra_attn_attention_noalloc(C.byref(desc), C.c_void_p(stream), msg, 256)
    return st, msg.value.decode()


def test_noalloc_rejects_rows_longer_than_the_scratch():
    # one score row of Lk floats must fit the 16 MiB array; this returns before any CUDA call
    d = _lib.Desc()
    d.q = d.k = d.v = 0x7F0000000000
    d.out = 0x7F8000000000
    Lk = 4194305
    d.Lq, d.Lk, d.H, d.D = 1, Lk, 1, 64
    d.ldq = d.ldk = d.ldv = 64
    d.q_size = 64
    d.k_size = d.v_size = Lk * 64
    d.out_size = 64
    d.flags = _lib.F_DEFAULT_SCALE
    st, msg = noalloc(d, 0)
    assert st == _lib.EINVAL and "Lk too large" in msg, msg


@pytest.mark.gpu
def test_noalloc_matches_regular_entry_point_on_two_calls():
    import torch

    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    handle = stream.cuda_stream or 1  # torch's default stream as cudaStreamLegacy
    gpu = supra_attn.GPU(0, stream=stream)
    rng = np.random.default_rng(123)
    # 1) the VAE mid-block shape: one 512-wide head over 1024 tokens (one 4 MiB unit)
    # 2) a problem whose scores (4 heads x 1000 x 4100 floats) need several passes over the scratch
    cases = [dict(Lq=1024, Lk=1024, H=1, D=512, scale=None), dict(Lq=1000, Lk=4100, H=4, D=64, scale=0.2)]
    outs = []
    for c in cases:
        HD = c["H"] * c["D"]
        q = torch.from_numpy(rng.standard_normal(c["Lq"] * HD).astype(np.float32)).cuda()
        k = torch.from_numpy(rng.standard_normal(c["Lk"] * HD).astype(np.float32)).cuda()
        v = torch.from_numpy(rng.standard_normal(c["Lk"] * HD).astype(np.float32)).cuda()
        o_ref = torch.full((c["Lq"] * HD,), 3.0, device="cuda")
        o_na = torch.full((c["Lq"] * HD,), 3.0, device="cuda")
        kw = dict(q=q, k=k, v=v, Lq=c["Lq"], Lk=c["Lk"], H=c["H"], D=c["D"], ldq=HD, ldk=HD, ldv=HD,
                  scale=c["scale"])
        supra_attn.attention(gpu, out=o_ref, **kw)  # regular entry point (recorded, flushed at sync)
        gpu.sync()
        outs.append((supra_attn.make_desc(out=o_na, **kw), o_ref, o_na, (q, k, v)))
    # two no-alloc calls in a row on one stream, no synchronisation between them
    for desc, _, _, _ in outs:
        st, msg = noalloc(desc, handle)
        assert st == _lib.OK, msg
    torch.cuda.synchronize()
    for desc, o_ref, o_na, _ in outs:
        a = o_na.cpu().numpy()
        b = o_ref.cpu().numpy()
        mr, rl = oracle.max_rel(a, b), oracle.rel_l2(a, b)
        assert mr <= TOL and rl <= TOL, f"max_rel={mr:.3e} rel_l2={rl:.3e}"
    gpu.close()


@pytest.mark.gpu
def test_noalloc_bias_unaligned_and_oracle():
    """Cases beyond the aligned bias-free ones, each against the float64 oracle at the FP32 bar,
    run twice in a row on one stream (the second call overwrites the shared scratch and unit table
    the first left behind):
      1) an expanded [H, Lq, Lk] bias whose scores span several passes over the scratch
         (4 heads x 1000 x 4100 floats: units of 896 and 104 rows, one head's two units per chunk,
         four chunks), so the bias rows are indexed from each unit's first row across chunks;
      2) a misaligned layout (D = 30, odd row strides and offsets), which takes the 4-byte copy
         path of the score kernels;
      3) the VAE mid-block shape (one 512-wide head over 1024 tokens)."""
    import torch

    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    handle = stream.cuda_stream or 1
    rng = np.random.default_rng(321)
    cases = [
        dict(Lq=1000, Lk=4100, H=4, D=64, ldq=256, ldk=256, ldv=256, qOff=0, kOff=0, vOff=0, oOff=0, scale=0.125,
             bias=True),
        dict(Lq=700, Lk=2000, H=3, D=30, ldq=91, ldk=93, ldv=97, qOff=1, kOff=3, vOff=2, oOff=5, scale=None,
             bias=False),
        dict(Lq=1024, Lk=1024, H=1, D=512, ldq=512, ldk=512, ldv=512, qOff=0, kOff=0, vOff=0, oOff=0, scale=None,
             bias=False),
    ]
    prepared = []
    for c in cases:
        H, D, Lq, Lk = c["H"], c["D"], c["Lq"], c["Lk"]
        qh = rng.standard_normal(c["qOff"] + Lq * c["ldq"]).astype(np.float32)
        kh = rng.standard_normal(c["kOff"] + Lk * c["ldk"]).astype(np.float32)
        vh = rng.standard_normal(c["vOff"] + Lk * c["ldv"]).astype(np.float32)
        bh = (rng.standard_normal(H * Lq * Lk) * 0.5).astype(np.float32) if c["bias"] else None
        ref = oracle.attention_ops(qh, kh, vh, Lq, Lk, H, D, c["ldq"], c["ldk"], c["ldv"], qOff=c["qOff"],
                                   kOff=c["kOff"], vOff=c["vOff"], oOff=c["oOff"], scale=c["scale"], bias=bh,
                                   out=np.full(c["oOff"] + Lq * H * D, 3.0, dtype=np.float32))
        q, k, v = (torch.from_numpy(a).cuda() for a in (qh, kh, vh))
        b = torch.from_numpy(bh).cuda() if bh is not None else None
        o = torch.full((c["oOff"] + Lq * H * D,), 3.0, device="cuda")
        desc = supra_attn.make_desc(q=q, k=k, v=v, out=o, bias=b, Lq=Lq, Lk=Lk, H=H, D=D, ldq=c["ldq"], ldk=c["ldk"],
                                    ldv=c["ldv"], qOff=c["qOff"], kOff=c["kOff"], vOff=c["vOff"], oOff=c["oOff"],
                                    scale=c["scale"])
        prepared.append((desc, o, ref, (q, k, v, b)))
    for rep in range(2):
        for desc, o, _, _ in prepared:
            o.fill_(3.0)
            st, msg = noalloc(desc, handle)
            assert st == _lib.OK, msg
        torch.cuda.synchronize()
        for i, (desc, o, ref, _) in enumerate(prepared):
            got = o.cpu().numpy()
            mr, rl = oracle.max_rel(got, ref), oracle.rel_l2(got, ref)
            assert mr <= TOL and rl <= TOL, f"call {rep} case {i}: max_rel={mr:.3e} rel_l2={rl:.3e}"
