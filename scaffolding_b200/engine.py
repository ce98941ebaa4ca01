"""Thin Python layer over the engine's C ABI: device buffers, streams,
workspaces and the GEMM / softmax / elementwise launches.

Everything here is plumbing around ``libsf_engine.so``; no arithmetic runs
in Python and there is no CPU path.  ``_cuda_ops`` builds the reference's
drop-in surface on top of these helpers.
"""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np

from . import _lib
from ._lib import (ACT_GELU_TANH, ACT_NONE, ACT_SILU, DT_BF16, DT_F16, DT_F32, Batch,
                   Epilogue, check, lib)

try:  # bf16 host storage (NumPy has none; the reference maps bf16 to fp32, dtype.py:31)
    import ml_dtypes as _mld
    bfloat16 = np.dtype(_mld.bfloat16)
except ImportError:  # pragma: no cover - ml_dtypes ships with this image
    bfloat16 = None

_ACTS = {"none": ACT_NONE, None: ACT_NONE, "silu": ACT_SILU, "gelu_tanh": ACT_GELU_TANH,
         "gelu": ACT_GELU_TANH}


def dtype_code(dtype) -> int:
    dt = np.dtype(dtype)
    if dt == np.float32:
        return DT_F32
    if dt == np.float16:
        return DT_F16
    if bfloat16 is not None and dt == bfloat16:
        return DT_BF16
    raise TypeError(f"unsupported dtype for the matmul engine: {dt}")


def code_dtype(code: int) -> np.dtype:
    return {DT_F32: np.dtype(np.float32), DT_F16: np.dtype(np.float16), DT_BF16: bfloat16}[code]


def act_code(act) -> int:
    try:
        return _ACTS[act]
    except KeyError:
        raise ValueError(f"unknown activation {act!r} (none | silu | gelu_tanh)") from None


# ───────────────────────────── devices ─────────────────────────────

def device_count() -> int:
    n = C.c_int32()
    check(lib.sf_device_count(C.byref(n)), "sf_device_count")
    return n.value


def current_device() -> int:
    d = C.c_int32()
    check(lib.sf_get_device(C.byref(d)), "sf_get_device")
    return d.value


def set_device(dev: int) -> None:
    check(lib.sf_set_device(int(dev)), "sf_set_device")


class on_device:
    """Run a block with ``dev`` current, restoring the previous device after
    (the ``_make_buffer`` pattern of ``_cuda_ops.pyx:463-470``)."""

    def __init__(self, dev: int):
        self.dev = int(dev)
        self.prev = None

    def __enter__(self):
        cur = current_device()
        if cur != self.dev:
            self.prev = cur
            set_device(self.dev)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            set_device(self.prev)
        return False


# ───────────────────────────── streams ─────────────────────────────
# The engine launches on a per-device "current stream"; None means the
# legacy default stream, as in the reference (_cuda_ops.pyx:680).

_streams: dict[int, int] = {}


def get_stream(dev: int) -> int | None:
    return _streams.get(dev)


def set_stream(dev: int, stream_ptr: int | None) -> None:
    if stream_ptr:
        _streams[dev] = int(stream_ptr)
    else:
        _streams.pop(dev, None)


# ───────────────────────────── buffers ─────────────────────────────

class DeviceBuffer:
    """Owning handle to engine-allocated device memory (caching allocator)."""

    __slots__ = ("ptr", "nbytes", "device_id", "owns", "__weakref__")

    def __init__(self, ptr: int, nbytes: int, device_id: int, owns: bool):
        self.ptr = int(ptr or 0)
        self.nbytes = int(nbytes)
        self.device_id = int(device_id)
        self.owns = bool(owns)

    @classmethod
    def alloc(cls, nbytes: int, device_id: int) -> "DeviceBuffer":
        p = C.c_void_p()
        check(lib.sf_malloc(int(device_id), int(nbytes), C.byref(p)), "sf_malloc")
        return cls(p.value or 0, nbytes, device_id, True)

    def free(self) -> None:
        if self.owns and self.ptr:
            lib.sf_free(self.device_id, C.c_void_p(self.ptr), self.nbytes)
            self.ptr = 0
            self.owns = False

    def __del__(self):
        try:
            self.free()
        except Exception:  # interpreter shutdown
            pass


class PinnedHostBuffer:
    """Page-locked host memory viewed as a NumPy array."""

    def __init__(self, nbytes: int):
        p = C.c_void_p()
        check(lib.sf_host_alloc_pinned(int(nbytes), C.byref(p)), "sf_host_alloc_pinned")
        self.ptr = p.value
        self.nbytes = int(nbytes)

    def array(self, shape, dtype) -> np.ndarray:
        dt = np.dtype(dtype)
        n = int(np.prod(shape)) * dt.itemsize
        assert n <= self.nbytes
        raw = (C.c_uint8 * n).from_address(self.ptr)
        return np.frombuffer(raw, dtype=np.uint8, count=n).view(dt).reshape(shape)

    def __del__(self):
        try:
            if self.ptr:
                lib.sf_host_free_pinned(C.c_void_p(self.ptr))
                self.ptr = None
        except Exception:
            pass


def memcpy(dst: int, src: int, nbytes: int, kind: int, stream: int | None = None) -> None:
    check(lib.sf_memcpy(C.c_void_p(dst), C.c_void_p(src), int(nbytes), kind,
                        C.c_void_p(stream) if stream else None), "sf_memcpy")


def stream_sync(stream: int | None) -> None:
    check(lib.sf_stream_synchronize(C.c_void_p(stream) if stream else None),
          "sf_stream_synchronize")


# ───────────────────────────── workspaces ─────────────────────────────

_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], DeviceBuffer] = {}


def workspace(dev: int, stream: int | None, nbytes: int) -> DeviceBuffer | None:
    """Per-(device, stream) scratch buffer, grown on demand.  Launches on one
    stream are ordered, so reusing it across calls on that stream is safe."""
    if nbytes <= 0:
        return None
    key = (dev, int(stream or 0))
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.nbytes < nbytes:
            if buf is not None:
                stream_sync(stream)
                buf.free()
            buf = DeviceBuffer.alloc(nbytes, dev)
            _workspaces[key] = buf
        return buf


def release_workspaces() -> None:
    with _ws_lock:
        for b in _workspaces.values():
            b.free()
        _workspaces.clear()


# ───────────────────────────── launches ─────────────────────────────

def make_epilogue(alpha=1.0, bias_ptr=0, bias_dt=DT_F32, act=ACT_NONE, residual_ptr=0,
                  residual_dt=DT_F32, ldr=0, beta=1.0, r_stride0=0, r_stride1=0) -> Epilogue:
    e = Epilogue()
    e.alpha = float(alpha)
    e.beta = float(beta)
    e.bias = bias_ptr or None
    e.bias_dtype = int(bias_dt)
    e.activation = int(act)
    e.residual = residual_ptr or None
    e.residual_dtype = int(residual_dt)
    e.ldr = int(ldr)
    e.r_stride0 = int(r_stride0)
    e.r_stride1 = int(r_stride1)
    return e


def make_batch(count0, count1=1, a=(0, 0), b=(0, 0), c=(0, 0)) -> Batch:
    bt = Batch()
    bt.count0, bt.count1 = int(count0), int(count1)
    bt.a_stride0, bt.a_stride1 = int(a[0]), int(a[1])
    bt.b_stride0, bt.b_stride1 = int(b[0]), int(b[1])
    bt.c_stride0, bt.c_stride1 = int(c[0]), int(c[1])
    return bt


def gemm(M, N, K, A, lda, trans_a, B, ldb, trans_b, Cp, ldc, in_dt, out_dt, *,
         epi: Epilogue | None = None, batch: Batch | None = None, device: int | None = None,
         stream: int | None = None) -> None:
    """Launch ``sf_gemm`` / ``sf_gemm_batched`` with a managed workspace."""
    dev = current_device() if device is None else device
    if stream is None:
        stream = get_stream(dev)
    need = C.c_size_t()
    check(lib.sf_gemm_workspace_size(C.byref(batch) if batch is not None else None,
                                     M, N, K, trans_a, trans_b, in_dt, out_dt, C.byref(need)),
          "sf_gemm_workspace_size")
    ws = workspace(dev, stream, need.value)
    wsp = C.c_void_p(ws.ptr) if ws else None
    wsb = ws.nbytes if ws else 0
    ep = C.byref(epi) if epi is not None else None
    sp = C.c_void_p(stream) if stream else None
    if batch is None:
        st = lib.sf_gemm(M, N, K, C.c_void_p(A), lda, trans_a, C.c_void_p(B), ldb, trans_b,
                         C.c_void_p(Cp), ldc, in_dt, out_dt, ep, wsp, wsb, sp)
        check(st, "sf_gemm")
    else:
        st = lib.sf_gemm_batched(C.byref(batch), M, N, K, C.c_void_p(A), lda, trans_a,
                                 C.c_void_p(B), ldb, trans_b, C.c_void_p(Cp), ldc, in_dt, out_dt,
                                 ep, wsp, wsb, sp)
        check(st, "sf_gemm_batched")


def softmax_rows(x, x_dt, ldx, y, y_dt, ldy, rows, cols, scale=1.0, stream=None, device=None):
    dev = current_device() if device is None else device
    if stream is None:
        stream = get_stream(dev)
    check(lib.sf_softmax_rows(C.c_void_p(x), x_dt, ldx, C.c_void_p(y), y_dt, ldy, rows, cols,
                              float(scale), C.c_void_p(stream) if stream else None),
          "sf_softmax_rows")


def attention(batch, heads, q_len, kv_len, q, ldq, q_bstride, k, ldk, k_bstride, v, ldv,
              v_bstride, o, ldo, o_bstride, scale, dtype=DT_BF16, head_dim=64, stream=None,
              device=None):
    """Fused attention forward (sf_attention_fwd): pointers are device
    addresses, strides in elements; head h of Q at column h * head_dim."""
    dev = current_device() if device is None else device
    s = get_stream(dev) if stream is None else stream
    check(lib.sf_attention_fwd(batch, heads, q_len, kv_len, head_dim, C.c_void_p(q), ldq,
                               q_bstride, C.c_void_p(k), ldk, k_bstride, C.c_void_p(v), ldv,
                               v_bstride, C.c_void_p(o), ldo, o_bstride, float(scale), dtype,
                               C.c_void_p(s) if s else None),
          "sf_attention_fwd")


def attention_launch_count(batch, heads, q_len, kv_len, skip_lo=None, skip_hi=None,
                           device=None):
    """Kernel launches of one attention / attention_partial call of these
    sizes, keys [skip_lo, skip_hi) skipped (sf_attention_launch_count): 1;
    with a stream-K tail, the whole units' kernel, the tail kernel and the
    merge kernel (2 when every unit is in the tail)."""
    lo = kv_len if skip_lo is None else skip_lo
    hi = kv_len if skip_hi is None else skip_hi
    prev = current_device()
    if device is not None and device != prev:
        set_device(device)
    try:
        n = C.c_int32()
        check(lib.sf_attention_launch_count(batch, heads, q_len, kv_len, lo, hi, C.byref(n)),
              "sf_attention_launch_count")
        return n.value
    finally:
        if device is not None and device != prev:
            set_device(prev)


def attention_partial(batch, heads, q_len, kv_len, q, ldq, q_bstride, k, ldk, k_bstride, v, ldv,
                      v_bstride, o, ldo, o_bstride, scale, skip_lo, skip_hi, part_o, part_ml,
                      part_mode, dtype=DT_BF16, head_dim=64, stream=None, device=None):
    """sf_attention_fwd_partial: attention over keys [0, kv_len) minus
    [skip_lo, skip_hi); part_mode 1 writes the partial result to part_o /
    part_ml, 2 merges it and writes o."""
    dev = current_device() if device is None else device
    s = get_stream(dev) if stream is None else stream
    check(lib.sf_attention_fwd_partial(batch, heads, q_len, kv_len, head_dim, C.c_void_p(q), ldq,
                                       q_bstride, C.c_void_p(k), ldk, k_bstride, C.c_void_p(v),
                                       ldv, v_bstride, C.c_void_p(o), ldo, o_bstride, float(scale),
                                       dtype, skip_lo, skip_hi, C.c_void_p(part_o),
                                       C.c_void_p(part_ml), part_mode,
                                       C.c_void_p(s) if s else None),
          "sf_attention_fwd_partial")


def unary(x, x_dt, y, y_dt, n, alpha=1.0, act=ACT_NONE, stream=None, device=None):
    dev = current_device() if device is None else device
    if stream is None:
        stream = get_stream(dev)
    check(lib.sf_unary(C.c_void_p(x), x_dt, C.c_void_p(y), y_dt, n, float(alpha), int(act),
                       C.c_void_p(stream) if stream else None), "sf_unary")


def device_error_status(dev: int, clear: bool = False) -> int:
    code = C.c_int32()
    check(lib.sf_device_error_status(int(dev), C.byref(code), 1 if clear else 0),
          "sf_device_error_status")
    return code.value


__all__ = [n for n in dir() if not n.startswith("_")] + ["_lib"]
