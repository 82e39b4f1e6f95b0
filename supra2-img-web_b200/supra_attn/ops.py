"""Python mirror of the reference's attention operator surface over libsupra_attn.

  GPU / Tensor      -- the device half of app/gpu/device.js (empty, fromArray, read, flush,
                       sync, Tensor.release, the Profiler), one libsupra_attn context each.
  attention()       -- ops.attention (app/gpu/ops.js:103-149): same keyword arguments, same
                       defaults (scale = 1/sqrt(D), out allocated as [Lq, H*D] when omitted),
                       a synchronous ValueError where the reference throws.
  linear()          -- ops.linear (app/gpu/ops.js:35-43): y = x @ W^T (+ bias), the projections
                       beside the attention (the cross-attention K/V preparation,
                       app/models/dit.js:137-144).
  relative_bucket() -- relativeBucket (app/models/t5.js:14-23).
  position_bias()   -- T5Encoder.positionBias + upload (app/models/t5.js:55-65,73), on the device.

Operands may be Tensors of a GPU or CUDA float32 torch tensors (contiguous); in the latter
case run the GPU on torch's current stream (GPU(stream=torch.cuda.current_stream())) so the
work is ordered with torch's. Every call goes through the C ABI; nothing computes on the CPU.
"""

from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import _lib
from ._lib import Desc, GroupNorm, LayerNorm, LinearDesc, ProfileEntry, check, lib

VARIANTS = {"fp32": _lib.FP32, "tf32": _lib.TF32, "tf32x3": _lib.TF32X3}
ACTS = {None: 0, "gelu": 1, "gelu_tanh": 2, "silu": 3}  # SUPRA_ATTN_ACT_*


class Tensor:
    """app/gpu/device.js:41-55 — {buf, shape, size, release()} over a device address."""

    def __init__(self, gpu: "GPU", buf: int, shape, capacity: int, owned: bool = True, keepalive=None):
        self.gpu = gpu
        self.buf = buf
        self.shape = list(shape)
        self.capacity = capacity  # floats addressable at buf (bounds for every call)
        self.owned = owned
        self._keep = keepalive

    @property
    def size(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    def release(self):
        if self.buf and self.owned:
            check(lib.supra_attn_tensor_free(self.gpu.ctx, C.c_void_p(self.buf)), self.gpu.ctx)
        self.buf = None
        self._keep = None


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream as an explicit handle


def _stream_handle(stream) -> int:
    """None -> 0 (the context's own stream); an int is passed through; a torch stream object
    maps to its handle, with torch's default stream (handle 0) mapped to cudaStreamLegacy."""
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    h = int(getattr(stream, "cuda_stream"))
    return h if h != 0 else CUDA_STREAM_LEGACY


class GPU:
    """A libsupra_attn context bound to one CUDA device (GPU.create, app/gpu/device.js:92-118)."""

    def __init__(self, device: int = 0, stream=None):
        ctx = C.c_void_p()
        st = lib.supra_attn_create(int(device), C.byref(ctx))
        if st != _lib.OK:
            raise _lib.SupraAttnError(st, f"supra_attn_create(device={device}) failed "
                                          "(needs an sm_100 GPU and the CUDA driver)")
        self.ctx = ctx
        self.device = int(device)
        if stream is not None:
            self.set_stream(stream)

    # ---- lifetime -------------------------------------------------------------------------------
    def close(self):
        if self.ctx:
            lib.supra_attn_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream):
        check(lib.supra_attn_set_stream(self.ctx, C.c_void_p(_stream_handle(stream))), self.ctx)

    # ---- tensors ----------------------------------------------------------------------------------
    def empty(self, shape) -> Tensor:
        n = 1
        for s in shape:
            n *= int(s)
        p = C.c_void_p()
        check(lib.supra_attn_tensor_alloc(self.ctx, n, C.byref(p)), self.ctx)
        return Tensor(self, p.value, shape, n)

    def from_array(self, arr, shape=None) -> Tensor:
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32)).reshape(-1)
        t = self.empty(list(shape) if shape is not None else [a.size])
        if t.size != a.size:
            t.release()
            raise ValueError(f"from_array: {a.size} values for shape {shape}")
        check(lib.supra_attn_upload(self.ctx, C.c_void_p(t.buf), a.ctypes.data_as(C.c_void_p), a.size), self.ctx)
        return t

    fromArray = from_array

    def write(self, t: Tensor, arr, offset: int = 0):
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32)).reshape(-1)
        if offset < 0 or offset + a.size > t.capacity:
            raise ValueError("write: out of bounds")
        check(lib.supra_attn_upload(self.ctx, C.c_void_p(t.buf + 4 * offset), a.ctypes.data_as(C.c_void_p), a.size),
              self.ctx)

    def read(self, t, count: int | None = None) -> np.ndarray:
        buf, cap = _as_buf(t)
        n = cap if count is None and not isinstance(t, Tensor) else (t.size if count is None else int(count))
        if n > cap:
            raise ValueError("read: count exceeds the tensor")
        out = np.empty(n, dtype=np.float32)
        check(lib.supra_attn_download(self.ctx, out.ctypes.data_as(C.c_void_p), C.c_void_p(buf), n), self.ctx)
        return out

    def wrap(self, x, shape=None) -> Tensor:
        """A non-owning Tensor over a CUDA float32 torch tensor (kept alive by the Tensor)."""
        buf, cap = _as_buf(x)
        return Tensor(self, buf, shape if shape is not None else list(x.shape), cap, owned=False, keepalive=x)

    # ---- execution ----------------------------------------------------------------------------------
    def enqueue(self, desc: Desc):
        check(lib.supra_attn_enqueue(self.ctx, C.byref(desc)), self.ctx)

    def enqueue_batch(self, descs):
        """descs: a ctypes array of Desc (see make_desc); recorded all-or-none."""
        check(lib.supra_attn_enqueue_batch(self.ctx, descs, len(descs)), self.ctx)

    def flush(self):
        check(lib.supra_attn_flush(self.ctx), self.ctx)

    def sync(self) -> int:
        st = C.c_int32(0)
        check(lib.supra_attn_sync(self.ctx, C.byref(st)), self.ctx)
        return st.value

    def pending(self) -> int:
        n = C.c_int32(0)
        check(lib.supra_attn_pending(self.ctx, C.byref(n)), self.ctx)
        return n.value

    def launch_count(self) -> int:
        n = C.c_int64(0)
        check(lib.supra_attn_launch_count(self.ctx, C.byref(n)), self.ctx)
        return n.value

    # ---- profiler (app/gpu/device.js:272-325) -------------------------------------------------------
    def profile(self, on: bool = True):
        check(lib.supra_attn_profile_enable(self.ctx, 1 if on else 0), self.ctx)

    def profile_report(self):
        arr = (ProfileEntry * 64)()
        n = C.c_int32(0)
        check(lib.supra_attn_profile_report(self.ctx, arr, 64, C.byref(n)), self.ctx)
        return [{"name": e.name.decode(), "count": e.launches, "ms": e.ms, "flops": e.flops, "bytes": e.bytes}
                for e in arr[: n.value]]

    def profile_reset(self):
        check(lib.supra_attn_profile_reset(self.ctx), self.ctx)


def _as_buf(x):
    """(device address, capacity in floats) of a Tensor or a CUDA float32 torch tensor."""
    if isinstance(x, Tensor):
        if not x.buf:
            raise ValueError("tensor was released")
        return x.buf, x.capacity
    if hasattr(x, "data_ptr") and hasattr(x, "is_cuda"):
        import torch

        if not x.is_cuda:
            raise ValueError("torch tensors must live on a CUDA device")
        if x.dtype != torch.float32:
            raise ValueError("torch tensors must be float32")
        if not x.is_contiguous():
            raise ValueError("torch tensors must be contiguous")
        return x.data_ptr(), x.numel()
    raise TypeError(f"unsupported operand type {type(x).__name__}")


def make_desc(*, q, k, v, out, Lq, Lk, H, D, ldq, ldk, ldv, qOff=0, kOff=0, vOff=0, oOff=0, scale=None,
              bias=None, t5_table=None, t5_buckets=32, t5_max_distance=128, variant="fp32") -> Desc:
    """Packs one ops.attention call into a supra_attn_desc (no validation; the library does it).

    t5_table (instead of bias): T5's [buckets, H] relative-attention-bias table; the kernels form
    the [H, Lq, Lk] bias from it (SUPRA_ATTN_F_T5_TABLE)."""
    if t5_table is not None and bias is not None:
        raise ValueError("pass either bias or t5_table, not both")
    d = Desc()
    d.q, d.q_size = _as_buf(q)
    d.k, d.k_size = _as_buf(k)
    d.v, d.v_size = _as_buf(v)
    d.out, d.out_size = _as_buf(out)
    if bias is not None:
        d.bias, d.bias_size = _as_buf(bias)
    if t5_table is not None:
        d.bias, d.bias_size = _as_buf(t5_table)
        if not (0 <= int(t5_buckets) < 1 << 16 and 0 <= int(t5_max_distance) < 1 << 16):
            raise ValueError("t5_buckets and t5_max_distance must fit in 16 bits")
        d.bias_param = int(t5_buckets) | (int(t5_max_distance) << 16)
    d.ldq, d.ldk, d.ldv = int(ldq), int(ldk), int(ldv)
    d.q_off, d.k_off, d.v_off, d.o_off = int(qOff), int(kOff), int(vOff), int(oOff)
    d.Lq, d.Lk, d.H, d.D = int(Lq), int(Lk), int(H), int(D)
    if scale is None:
        d.flags = _lib.F_DEFAULT_SCALE
        d.scale = 0.0
    else:
        d.scale = float(scale)
    if t5_table is not None:
        d.flags |= _lib.F_T5_TABLE
    if variant not in VARIANTS:
        raise ValueError(f"variant must be one of {sorted(VARIANTS)}")
    d.variant = VARIANTS[variant]
    return d


def attention(gpu: GPU, *, q, k, v, Lq, Lk, H, D, ldq, ldk, ldv, qOff=0, kOff=0, vOff=0, oOff=0, scale=None,
              bias=None, out=None, variant="fp32", t5_table=None, t5_buckets=32, t5_max_distance=128):
    """ops.attention (app/gpu/ops.js:109): records the call and returns the output tensor.

    q: [Lq, ldq] with head h at column qOff + h*D; k, v: [Lk, ldk] / [Lk, ldv] with head h at
    kOff / vOff + h*D. The output rows [Lq, H*D] are written at element offset oOff of `out`
    (allocated as gpu.empty([Lq, H*D]) when omitted). scale defaults to 1/sqrt(D). bias is an
    additive score bias [H, Lq, Lk]. Alternatively t5_table, T5's [buckets, H] relative-bias
    table, makes the kernels form that bias themselves (bias[h, i, j] = table[bucket(j - i), h],
    app/models/t5.js:55-65) instead of reading an expanded one. Work runs at the next
    flush/sync/read.
    """
    o = out if out is not None else gpu.empty([Lq, H * D])
    try:
        d = make_desc(q=q, k=k, v=v, out=o, Lq=Lq, Lk=Lk, H=H, D=D, ldq=ldq, ldk=ldk, ldv=ldv, qOff=qOff, kOff=kOff,
                      vOff=vOff, oOff=oOff, scale=scale, bias=bias, t5_table=t5_table, t5_buckets=t5_buckets,
                      t5_max_distance=t5_max_distance, variant=variant)
        gpu.enqueue(d)
    except Exception:
        if out is None:
            o.release()
        raise
    return o


def make_linear_desc(*, x, w, y, M, N, K, bias=None, ldx=None, ldw=None, ldy=None, xOff=0, yOff=0,
                     groupnorm=None, layernorm=None, resid=None, ldr=None, rOff=0, gate=None, gOff=0, act=None,
                     variant="fp32") -> LinearDesc:
    """Packs one linear call y = resid + gate * (x W^T + bias) (resid, gate and bias optional) into
    a supra_attn_linear_desc (validated by the library). resid=True is the reference's in-place
    residual: resid is y itself, same rows. groupnorm: dict(gamma, beta, groups, rows_per_image,
    eps=1e-6, silu=False) to GroupNorm x on the way in; layernorm: dict(mod=None, shiftOff=0,
    scaleOff=0, eps=1e-6) to LayerNorm each row of x on the way in, modulated by mod when given
    (ops.layernorm's arguments, app/gpu/ops.js:71). act: None, "gelu", "gelu_tanh" or "silu" on
    x W^T + bias (app/gpu/gemm.js:130-134). The returned descriptor keeps the norm blocks alive."""
    if act not in ACTS:
        raise ValueError(f"act must be one of {sorted(a for a in ACTS if a)} or None")
    d = LinearDesc()
    if groupnorm is not None:
        gnb = GroupNorm()
        gnb.gamma = _as_buf(groupnorm["gamma"])[0]
        gnb.beta = _as_buf(groupnorm["beta"])[0]
        gnb.groups = int(groupnorm["groups"])
        gnb.rows_per_image = int(groupnorm["rows_per_image"])
        gnb.eps = float(groupnorm.get("eps", 1e-6))
        gnb.silu = 1 if groupnorm.get("silu", False) else 0
        d._gn = gnb
        d.gn = C.pointer(gnb)
    if layernorm is not None:
        lnb = LayerNorm()
        mod = layernorm.get("mod")
        if mod is not None:
            lnb.mod, lnb.mod_size = _as_buf(mod)
            lnb.shift_off = int(layernorm.get("shiftOff", 0))
            lnb.scale_off = int(layernorm.get("scaleOff", 0))
        lnb.eps = float(layernorm.get("eps", 1e-6))
        d._ln = lnb
        d.ln = C.pointer(lnb)
    if resid is True:  # in place on y (app/gpu/gemm.js:135 reads C[ci] before it writes it)
        resid, ldr, rOff = y, (N if ldy is None else ldy), yOff
    if resid is not None and resid is not False:
        d.resid, d.resid_size = _as_buf(resid)
        d.ldr = int(N if ldr is None else ldr)
        d.r_off = int(rOff)
    if gate is not None:
        d.gate, d.gate_size = _as_buf(gate)
        d.g_off = int(gOff)
    d.x, d.x_size = _as_buf(x)
    d.w, d.w_size = _as_buf(w)
    d.y, d.y_size = _as_buf(y)
    if bias is not None:
        d.bias, d.bias_size = _as_buf(bias)
    d.M, d.N, d.K = int(M), int(N), int(K)
    d.ldx = int(K if ldx is None else ldx)
    d.ldw = int(K if ldw is None else ldw)
    d.ldy = int(N if ldy is None else ldy)
    d.x_off, d.y_off = int(xOff), int(yOff)
    if variant not in VARIANTS:
        raise ValueError(f"variant must be one of {sorted(VARIANTS)}")
    d.variant = VARIANTS[variant]
    d.act = ACTS[act]
    return d


def linear(gpu: GPU, x, w, *, N, K, M=None, bias=None, out=None, ldx=None, ldw=None, ldy=None, xOff=0, yOff=0,
           groupnorm=None, layernorm=None, resid=None, ldr=None, rOff=0, gate=None, gOff=0, act=None,
           variant="fp32"):
    """ops.linear (app/gpu/ops.js:35-43): y = x @ W^T (+ bias), recorded; returns y.

    x: M rows of K floats (row stride ldx, first row at xOff; M defaults to x.size / K as in the
    reference); w: [N, K] row-major weights; bias: N floats. y is allocated as gpu.empty([M, N])
    when `out` is omitted. groupnorm (dict, see make_linear_desc) normalises x on the way in
    (ops.groupnorm, app/gpu/ops.js:82-92), layernorm (dict(mod, shiftOff, scaleOff), or {} for the
    plain norm) LayerNorms each row of x on the way in (ops.layernorm, app/gpu/ops.js:71-79, with
    the adaLN modulation of app/models/dit.js:164,189); resid is added to y (the residual add of
    app/models/vae.js:91). resid=True with `out` is the reference's in-place residual
    `{ out: x, resid: true }` (app/models/dit.js:187), and gate/gOff scale the product per output
    column first, out = out + gate[gOff + n] * (x W^T + bias) (app/gpu/gemm.js:10,135,
    app/models/dit.js:175,193). act ("gelu", "gelu_tanh", "silu") applies to x W^T + bias before
    the gate and the residual (app/gpu/gemm.js:130-135). fp32 FFMA; runs at the next
    flush/sync/read.
    """
    if resid is True and out is None:
        raise ValueError("resid=True accumulates into out: pass out")
    if gate is not None and (resid is None or resid is False):
        raise ValueError("gate needs resid (the gated residual)")
    if M is None:  # the reference's x.size / W.K (app/gpu/ops.js:36), from the logical size
        n = x.size if isinstance(x, Tensor) else _as_buf(x)[1]
        M = (n - int(xOff)) // int(K)
    y = out if out is not None else gpu.empty([int(M), int(N)])
    try:
        d = make_linear_desc(x=x, w=w, y=y, M=M, N=N, K=K, bias=bias, ldx=ldx, ldw=ldw, ldy=ldy, xOff=xOff,
                             yOff=yOff, groupnorm=groupnorm, layernorm=layernorm, resid=resid, ldr=ldr, rOff=rOff,
                             gate=gate, gOff=gOff, act=act, variant=variant)
        check(lib.supra_attn_enqueue_linear(gpu.ctx, C.byref(d)), gpu.ctx)
    except Exception:
        if out is None:
            y.release()
        raise
    return y


def relative_bucket(rel: int, buckets: int = 32, max_distance: int = 128) -> int:
    """relativeBucket (app/models/t5.js:14-23)."""
    b = lib.supra_attn_relative_bucket(int(rel), int(buckets), int(max_distance))
    if b < 0:
        raise ValueError("buckets must be even and >= 4, and max_distance > buckets/4")
    return b


def position_bias(gpu: GPU, table, L: int, H: int = 12, buckets: int = 32, max_distance: int = 128, out=None):
    """T5Encoder.positionBias(L) uploaded as [H, L, L] (app/models/t5.js:55-65,73), built on the device.

    table: device [buckets, H] (Tensor or CUDA torch tensor).
    """
    tb, tcap = _as_buf(table)
    if tcap < buckets * H:
        raise ValueError("table must hold buckets*H floats")
    o = out if out is not None else gpu.empty([H, L, L])
    ob, ocap = _as_buf(o)
    try:
        check(lib.supra_attn_position_bias(gpu.ctx, C.c_void_p(tb), int(tcap), int(buckets), int(max_distance), int(H), int(L),
                                           C.c_void_p(ob), int(ocap)), gpu.ctx)
    except Exception:
        if out is None:
            o.release()
        raise
    return o


def default_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)
