"""CPU-side checks of the C ABI: the library loads, exports every declared symbol, and its pure
host functions (descriptor validation, the T5 bucket function) behave like the reference."""

import ctypes as C
import os
import re

import numpy as np
import pytest

import supra_attn
from supra_attn import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "supra_attn.h")


def header_functions():
    txt = open(HEADER).read()
    return set(re.findall(r"SUPRA_ATTN_API\s+[\w\s\*]+?\b(supra_attn_\w+)\s*\(", txt))


def test_exports_every_declared_symbol():
    declared = header_functions()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(_lib.lib, name), name
    assert {s[0] for s in _lib.SIGNATURES} == declared


def test_library_path_is_in_tree():
    assert os.path.exists(_lib.LIB_PATH)
    assert "supra2-img-web_b200" in os.path.abspath(_lib.LIB_PATH)


def test_status_strings():
    for st in range(7):
        assert _lib.lib.supra_attn_status_string(st).decode()


@pytest.mark.parametrize("nb,md", [(32, 128), (32, 64), (16, 32), (64, 256)])
def test_relative_bucket_matches_hf(golden, nb, md):
    ref = golden(f"bucket_{nb}_{md}").astype(np.int64)
    got = np.array([supra_attn.relative_bucket(r, nb, md) for r in range(-1000, 1001)])
    np.testing.assert_array_equal(got, ref)


def test_relative_bucket_rejects_bad_config():
    assert _lib.lib.supra_attn_relative_bucket(3, 3, 128) == -1
    assert _lib.lib.supra_attn_relative_bucket(3, 2, 128) == -1
    assert _lib.lib.supra_attn_relative_bucket(3, 32, 8) == -1
    with pytest.raises(ValueError):
        supra_attn.relative_bucket(1, 31, 128)


# ---- descriptor validation (pure host; fake, never dereferenced device addresses) ----------------
BASE_Q = 0x7F0000000000
BASE_O = 0x7F1000000000
BASE_B = 0x7F2000000000


def dit_self_desc(**kw):
    """DiT self-attention for sample b=1 of B=2 (app/models/dit.js:172)."""
    d = _lib.Desc()
    d.q = d.k = d.v = BASE_Q
    d.out = BASE_O
    d.q_size = d.k_size = d.v_size = 2 * 256 * 1728
    d.out_size = 2 * 256 * 576
    d.ldq = d.ldk = d.ldv = 1728
    r = 256 * 1728
    d.q_off, d.k_off, d.v_off, d.o_off = r, r + 576, r + 1152, 256 * 576
    d.Lq, d.Lk, d.H, d.D = 256, 256, 9, 64
    d.flags = _lib.F_DEFAULT_SCALE
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def check(d):
    msg = C.create_string_buffer(512)
    st = _lib.lib.supra_attn_check_desc(C.byref(d), msg, 512)
    return st, msg.value.decode()


def test_valid_descriptors():
    assert check(dit_self_desc()) == (_lib.OK, "")
    # T5 with bias
    d = dit_self_desc(q_off=0, k_off=0, v_off=0, o_off=0, ldq=768, ldk=768, ldv=768, Lq=37, Lk=37, H=12, D=64)
    d.q_size = d.k_size = d.v_size = 37 * 768
    d.out_size = 37 * 768
    d.bias = BASE_B
    d.bias_size = 12 * 37 * 37
    d.flags = 0
    d.scale = 1.0
    assert check(d)[0] == _lib.OK
    # Lq = 0 records nothing and is valid
    assert check(dit_self_desc(Lq=0))[0] == _lib.OK
    # the three numeric variants (FP32 FFMA, TF32, split-precision TF32X3); 3 is not one
    for v in (_lib.FP32, _lib.TF32, _lib.TF32X3):
        assert check(dit_self_desc(variant=v))[0] == _lib.OK
    st, msg = check(dit_self_desc(variant=3))
    assert st == _lib.EINVAL and "variant" in msg
    # the Python mirror's names for them
    assert supra_attn.ops.VARIANTS == {"fp32": _lib.FP32, "tf32": _lib.TF32, "tf32x3": _lib.TF32X3}


@pytest.mark.parametrize(
    "kw,needle",
    [
        (dict(Lk=0), "Lk"),
        (dict(H=0), "H="),
        (dict(D=0), "D="),
        (dict(Lq=-1), "Lq"),
        (dict(q_off=-4), "offset"),
        (dict(ldq=-1), "leading"),
        (dict(v_size=2 * 256 * 1728 - 1), "v out of bounds"),  # v's last read is the buffer's last float
        (dict(q_size=511 * 1728 + 575), "q out of bounds"),
        (dict(out_size=2 * 256 * 576 - 1), "out out of bounds"),
        (dict(o_off=256 * 576 + 4), "out out of bounds"),
        (dict(flags=0x10), "flag"),
        (dict(variant=7), "variant"),
        (dict(q=0), "non-NULL"),
        (dict(q=BASE_Q + 2, k=BASE_Q + 2, v=BASE_Q + 2), "aligned"),
        (dict(flags=0, scale=float("inf")), "finite"),
    ],
)
def test_invalid_descriptors(kw, needle):
    st, msg = check(dit_self_desc(**kw))
    assert st == _lib.EINVAL
    assert needle in msg, msg


def test_bias_too_small():
    d = dit_self_desc()
    d.bias = BASE_B
    d.bias_size = 9 * 256 * 256 - 1
    st, msg = check(d)
    assert st == _lib.EINVAL and "bias" in msg


def t5_table_desc(**kw):
    """T5 encoder attention (app/models/t5.js:80) with the [32, 12] table in place of the bias."""
    d = dit_self_desc(q_off=0, k_off=0, v_off=0, o_off=0, ldq=768, ldk=768, ldv=768, Lq=37, Lk=37, H=12, D=64)
    d.q_size = d.k_size = d.v_size = 37 * 768
    d.out_size = 37 * 768
    d.bias = BASE_B
    d.bias_size = 32 * 12
    d.flags = _lib.F_T5_TABLE
    d.bias_param = 32 | (128 << 16)
    d.scale = 1.0
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def test_t5_table_descriptors():
    assert check(t5_table_desc()) == (_lib.OK, "")
    assert check(t5_table_desc(flags=_lib.F_T5_TABLE | _lib.F_DEFAULT_SCALE))[0] == _lib.OK
    cases = [
        (dict(bias=0), "table"),                             # the flag needs the table pointer
        (dict(bias_size=32 * 12 - 1), "buckets*H"),          # table too small
        (dict(bias_param=31 | (128 << 16)), "buckets"),      # odd bucket count
        (dict(bias_param=32 | (8 << 16)), "max_distance"),   # max_distance <= buckets/4
        (dict(flags=0), "bias_param"),                       # parameters without the flag
    ]
    for kw, needle in cases:
        st, msg = check(t5_table_desc(**kw))
        assert st == _lib.EINVAL and needle in msg, (kw, msg)


def test_out_may_not_alias_inputs():
    d = dit_self_desc()
    d.out = BASE_Q  # writes over rows that q/k/v of this call read
    d.out_size = d.q_size
    d.o_off = 256 * 1728
    st, msg = check(d)
    assert st == _lib.EINVAL and "overlaps" in msg


def test_create_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ctx = C.c_void_p()
    st = _lib.lib.supra_attn_create(0, C.byref(ctx))
    assert st != _lib.OK and not ctx.value
    with pytest.raises(supra_attn.SupraAttnError):
        supra_attn.GPU(0)


# ---- linear descriptors (pure host) ----------------------------------------------------------
def linear_desc(**kw):
    """ctx_proj of one prompt (app/models/dit.js:139): x [37, 768], W [576, 768], bias [576]."""
    d = _lib.LinearDesc()
    d.x, d.w, d.bias, d.y = BASE_Q, BASE_B, BASE_B + 4 * 576 * 768, BASE_O
    d.x_size, d.w_size, d.bias_size, d.y_size = 37 * 768, 576 * 768, 576, 37 * 576
    d.ldx, d.ldw, d.ldy = 768, 768, 576
    d.M, d.N, d.K = 37, 576, 768
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def check_linear(d):
    msg = C.create_string_buffer(512)
    st = _lib.lib.supra_attn_check_linear_desc(C.byref(d), msg, 512)
    return st, msg.value.decode()


def test_linear_descriptors():
    assert check_linear(linear_desc()) == (_lib.OK, "")
    assert check_linear(linear_desc(bias=0, bias_size=0))[0] == _lib.OK
    assert check_linear(linear_desc(M=0))[0] == _lib.OK  # nothing to do
    cases = [
        (dict(N=0), "N="),
        (dict(K=0), "K="),
        (dict(M=-1), "M="),
        (dict(ldx=700), "ldx >= K"),
        (dict(ldy=500), "ldy >= N"),
        (dict(x_size=37 * 768 - 1), "x out of bounds"),
        (dict(w_size=576 * 768 - 1), "w out of bounds"),
        (dict(bias_size=575), "bias"),
        (dict(y_size=37 * 576 - 1), "y out of bounds"),
        (dict(x_off=-4), "offset"),
        (dict(flags=1), "flags"),
        (dict(variant=9), "variant"),
        (dict(w=0), "non-NULL"),
        (dict(x=BASE_Q + 2), "aligned"),
        (dict(y=BASE_Q, y_size=37 * 768), "overlaps"),
    ]
    for kw, needle in cases:
        st, msg = check_linear(linear_desc(**kw))
        assert st == _lib.EINVAL and needle in msg, (kw, msg)


def test_linear_groupnorm_and_residual_descriptors():
    gn = _lib.GroupNorm()
    gn.gamma, gn.beta, gn.groups, gn.rows_per_image, gn.eps = BASE_B + 4 * 600000, BASE_B + 4 * 700000, 32, 37, 1e-6
    assert check_linear(linear_desc(gn=C.pointer(gn)))[0] == _lib.OK
    for field, value, needle in [("groups", 7, "groups"), ("rows_per_image", 5, "rows_per_image"),
                                 ("eps", -1.0, "eps"), ("gamma", 0, "gamma")]:
        bad = _lib.GroupNorm()
        C.pointer(bad)[0] = gn
        setattr(bad, field, value)
        st, msg = check_linear(linear_desc(gn=C.pointer(bad)))
        assert st == _lib.EINVAL and needle in msg, (field, msg)
    st, msg = check_linear(linear_desc(gn=C.pointer(gn), x_off=4, x_size=37 * 768 + 4))
    assert st == _lib.EINVAL and "contiguous" in msg
    ok = linear_desc(resid=BASE_O + 4 * 10 ** 6, resid_size=37 * 576, ldr=576)
    assert check_linear(ok)[0] == _lib.OK
    st, msg = check_linear(linear_desc(resid=BASE_O + 4 * 10 ** 6, resid_size=37 * 576 - 1, ldr=576))
    assert st == _lib.EINVAL and "resid" in msg
    # resid == y row for row is the in-place residual (app/models/dit.js:187); any other overlap is not
    assert check_linear(linear_desc(resid=BASE_O, resid_size=37 * 576, ldr=576))[0] == _lib.OK
    st, msg = check_linear(linear_desc(resid=BASE_O, resid_size=37 * 576 + 1, ldr=576, r_off=1))
    assert st == _lib.EINVAL and "overlaps" in msg
    st, msg = check_linear(linear_desc(resid=BASE_O, resid_size=38 * 580, ldr=580, ldy=580, y_size=38 * 580,
                                       r_off=0, y_off=0))
    assert st == _lib.OK, msg


def test_linear_gate_descriptors():
    """The gated residual of the DiT blocks (app/gpu/gemm.js:135): gate[g_off + n], needs resid."""
    gate = BASE_B + 4 * 800000
    ok = dict(resid=BASE_O, resid_size=37 * 576, ldr=576, gate=gate, gate_size=6 * 576, g_off=2 * 576)
    assert check_linear(linear_desc(**ok))[0] == _lib.OK
    for kw, needle in [(dict(resid=0, resid_size=0), "needs resid"), (dict(g_off=5 * 576 + 1), "gate out of bounds"),
                       (dict(g_off=-1), "gate out of bounds"), (dict(gate=gate + 2), "gate must be")]:
        st, msg = check_linear(linear_desc(**{**ok, **kw}))
        assert st == _lib.EINVAL and needle in msg, (kw, msg)


def test_linear_python_argument_checks():
    """ops.linear's own checks, made before anything is recorded: an in-place residual needs out,
    and a gate needs a residual (app/gpu/gemm.js:135 only gates the residual form)."""
    with pytest.raises(ValueError, match="pass out"):
        supra_attn.linear(None, BASE_Q, BASE_B, N=4, K=4, M=1, resid=True)
    with pytest.raises(ValueError, match="needs resid"):
        supra_attn.linear(None, BASE_Q, BASE_B, N=4, K=4, M=1, out=BASE_O, gate=BASE_B)


def test_linear_layernorm_and_act_descriptors():
    """LayerNorm prologue (ops.layernorm's mod/shiftOff/scaleOff) and the act epilogue."""
    ln = _lib.LayerNorm()
    ln.eps = 1e-6
    assert check_linear(linear_desc(ln=C.pointer(ln)))[0] == _lib.OK  # plain
    mod = BASE_B + 4 * 900000
    ln.mod, ln.mod_size, ln.shift_off, ln.scale_off = mod, 6 * 768, 0, 768
    assert check_linear(linear_desc(ln=C.pointer(ln)))[0] == _lib.OK
    for field, value, needle in [("scale_off", 5 * 768 + 1, "mod out of bounds"), ("shift_off", -1, "mod out of bounds"),
                                 ("eps", float("nan"), "eps"), ("reserved", 1, "reserved"), ("mod", mod + 1, "aligned")]:
        bad = _lib.LayerNorm()
        C.pointer(bad)[0] = ln
        setattr(bad, field, value)
        st, msg = check_linear(linear_desc(ln=C.pointer(bad)))
        assert st == _lib.EINVAL and needle in msg, (field, msg)
    st, msg = check_linear(linear_desc(ln=C.pointer(ln), ldx=800, x_size=37 * 800))
    assert st == _lib.EINVAL and "contiguous" in msg
    gn = _lib.GroupNorm()
    gn.gamma, gn.beta, gn.groups, gn.rows_per_image, gn.eps = BASE_B + 4 * 600000, BASE_B + 4 * 700000, 32, 37, 1e-6
    st, msg = check_linear(linear_desc(ln=C.pointer(ln), gn=C.pointer(gn)))
    assert st == _lib.EINVAL and "exclusive" in msg
    for a in range(4):
        assert check_linear(linear_desc(act=a))[0] == _lib.OK
    st, msg = check_linear(linear_desc(act=4))
    assert st == _lib.EINVAL and "act" in msg
    with pytest.raises(ValueError, match="act"):
        supra_attn.make_linear_desc(x=BASE_Q, w=BASE_B, y=BASE_O, M=1, N=4, K=4, act="relu")
