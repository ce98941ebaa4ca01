"""Drop-in replacement for the hot-path surface of ``scaffolding._cuda_ops``.

The reference's callers (``tensor.py:37``, ``nn/layers.py:12``,
``nn/functional.py:11``, ``nn/parallel.py:23``) import
``scaffolding._cuda_ops`` and call the names below; this module exports the
same names with the same signatures and argument meaning, backed by the
sm_100a engine (``libsf_engine.so``) instead of cuBLAS:

* ``GpuTensor`` / ``CudaBuffer`` and the NumPy transfer helpers
  (``_cuda_ops.pyx:307-341``, ``:807-875``);
* the matmul family ``dev_matmul``, ``dev_matmul_nt``, ``dev_batched_matmul``,
  ``dev_batched_matmul_nt``, ``dev_linear_forward`` (``_cuda_ops.pyx:1088-1302``)
  and the host-array ``cuda_*`` variants (``:2120-2230``, ``:2453-2471``);
* the glue the attention path uses: ``dev_muls``, ``dev_softmax``, ``dev_silu``,
  ``dev_gelu``, ``dev_reshape``, ``dev_unsqueeze``, ``dev_squeeze``;
* ``dev_layer_norm`` and the DiT blocks' adaptive norm ``dev_ada_layer_norm``
  (the bandwidth step in front of the QKV and FFN-up GEMMs);
* runtime: devices, caching allocator, streams, events, peer access.

Differences from the reference, all deliberate:
* dtype-aware: bf16 (``ml_dtypes.bfloat16`` on the host) and fp16 tensors
  are computed as such with fp32 accumulation and returned in their own
  dtype; fp32 tensors behave exactly as before (fp32 in, fp32 out).  The
  reference read every buffer as ``float*`` (``_cuda_ops.pyx:1095-1102``).
* ``dev_linear_forward`` fuses bias and an optional activation into the GEMM
  epilogue (the reference launched SGEMM, then a bias kernel on the NULL
  stream, then the activation separately).
* ``dev_batched_matmul_nt`` is one launch (the reference looped over the
  batch on the host, ``_cuda_ops.pyx:1181-1187``).
* every op runs on the device that holds its inputs, and allocates there
  (the reference used the current device in ``dev_muls`` / ``dev_softmax``).
* ``gputensor_to_device`` copies ``numel * itemsize`` bytes (the reference
  assumed 4-byte elements, ``_cuda_ops.pyx:868-870``).

Operations outside the matmul path (RMS norm, cross-entropy, AdamW, ...)
raise ``NotImplementedError`` naming the op.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import engine as E
from ._lib import (ACT_GELU_TANH, ACT_NONE, ACT_SILU, COPY_D2D, COPY_D2H, COPY_H2D,
                   DT_F32, FP32_ACCURATE, FP32_TF32, DeviceProps, check, lib)

bfloat16 = E.bfloat16


# ───────────────────────────── buffers / tensors ─────────────────────────────

class CudaBuffer(E.DeviceBuffer):
    """Device allocation from the engine's caching allocator
    (``_cuda_ops.pyx:307-341``)."""

    __slots__ = ()

    @property
    def data_ptr(self) -> int:
        return self.ptr

    @property
    def size(self) -> int:
        return self.nbytes

    def __reduce__(self):
        # Pickle the raw bytes (the reference pickled as float32 regardless
        # of the element type, _cuda_ops.pyx:333-341).
        arr = np.empty(self.nbytes, dtype=np.uint8)
        if self.ptr and self.nbytes:
            with E.on_device(self.device_id):
                E.memcpy(arr.ctypes.data, self.ptr, self.nbytes, COPY_D2H)
                E.stream_sync(None)
        return (_rebuild_cuda_buffer, (arr, self.device_id))


def _rebuild_cuda_buffer(arr: np.ndarray, device_id: int = 0):
    buf = _make_buffer(arr.nbytes, device_id)
    with E.on_device(device_id):
        E.memcpy(buf.ptr, arr.ctypes.data, arr.nbytes, COPY_H2D)
        E.stream_sync(None)
    return buf


def _make_buffer(nbytes: int, device_id: int) -> CudaBuffer:
    p = C.c_void_p()
    check(lib.sf_malloc(int(device_id), int(nbytes), C.byref(p)), "sf_malloc")
    return CudaBuffer(p.value or 0, nbytes, device_id, True)


class GpuTensor:
    """GPU-resident tensor: CudaBuffer + shape + NumPy dtype + device id
    (``_cuda_ops.pyx:807-819``), contiguous row-major."""

    __slots__ = ("buffer", "shape", "dtype", "numel", "device_id")

    def __init__(self, buffer, shape: tuple, dtype, device_id: int = -1):
        self.buffer = buffer
        self.shape = tuple(int(s) for s in shape)
        self.dtype = np.dtype(dtype)
        self.device_id = device_id if device_id >= 0 else buffer.device_id
        n = 1
        for s in self.shape:
            n *= s
        self.numel = n

    @property
    def ptr(self) -> int:
        return self.buffer.ptr

    @property
    def ndim(self) -> int:
        return len(self.shape)

    def matmul(self, other: "GpuTensor", *, trans_b: bool = False, out_dtype=None) -> "GpuTensor":
        """``self @ other`` (``trans_b``: ``self @ other^T``, ``other`` in the
        ``nn.Linear`` weight layout).  2-D or batched, like ``sf.matmul`` /
        ``sf.matmul_nt`` (``tensor.py:1480-1539``)."""
        if self.ndim == 2 and other.ndim == 2:
            return _matmul2d(self, other, trans_b, out_dtype)
        return _batched(self, other, trans_b, out_dtype)

    def __matmul__(self, other: "GpuTensor") -> "GpuTensor":
        return self.matmul(other)

    def __repr__(self) -> str:
        return f"GpuTensor(shape={self.shape}, dtype={self.dtype}, device={self.device_id})"


def _alloc(shape, dtype, dev) -> GpuTensor:
    dt = np.dtype(dtype)
    n = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
    return GpuTensor(_make_buffer(n * dt.itemsize, dev), tuple(shape), dt, dev)


# ───────────────────────────── NumPy <-> GPU ─────────────────────────────

def gputensor_from_numpy(arr: np.ndarray, device_id: int = -1) -> GpuTensor:
    """Upload a NumPy array (``_cuda_ops.pyx:822-840``)."""
    flat = np.ascontiguousarray(arr)
    dev = device_id if device_id >= 0 else E.current_device()
    gt = _alloc(flat.shape, flat.dtype, dev)
    if flat.nbytes:
        with E.on_device(dev):
            E.memcpy(gt.ptr, flat.ctypes.data, flat.nbytes, COPY_H2D)
            E.stream_sync(E.get_stream(dev))
    return gt


def gputensor_to_numpy(gt: GpuTensor) -> np.ndarray:
    """Download a GpuTensor synchronously (``_cuda_ops.pyx:843-858``)."""
    out = np.empty(gt.shape, dtype=gt.dtype)
    if out.nbytes:
        with E.on_device(gt.device_id):
            stream = E.get_stream(gt.device_id)
            E.stream_sync(stream)
            E.memcpy(out.ctypes.data, gt.ptr, out.nbytes, COPY_D2H, stream)
            E.stream_sync(stream)
    return out


def gputensor_to_device(gt: GpuTensor, target_dev: int) -> GpuTensor:
    """Copy to another device (``_cuda_ops.pyx:861-875``), ``numel*itemsize`` bytes."""
    if gt.device_id == target_dev:
        return gt
    out = _alloc(gt.shape, gt.dtype, target_dev)
    nbytes = gt.numel * gt.dtype.itemsize
    if nbytes:
        with E.on_device(gt.device_id):
            E.stream_sync(E.get_stream(gt.device_id))
        check(lib.sf_memcpy_peer(C.c_void_p(out.ptr), int(target_dev), C.c_void_p(gt.ptr),
                                 int(gt.device_id), nbytes, None), "sf_memcpy_peer")
        E.stream_sync(None)
    return out


def gputensor_astype(gt: GpuTensor, dtype) -> GpuTensor:
    """Copy of ``gt`` converted to ``dtype`` on its device (fp32 / bf16 / fp16,
    round to nearest even), e.g. fp32 weights stored as bf16 after upload.
    New: the reference uploads fp32 only (``nn/layers.py:18-35``)."""
    dt = np.dtype(dtype)
    if dt == gt.dtype:
        return gt
    out = _alloc(gt.shape, dt, gt.device_id)
    if gt.numel:
        with E.on_device(gt.device_id):
            E.unary(gt.ptr, E.dtype_code(gt.dtype), out.ptr, E.dtype_code(dt), gt.numel, 1.0,
                    ACT_NONE, device=gt.device_id)
    return out


def numpy_to_gpu(arr: np.ndarray, stream=None):
    gt = gputensor_from_numpy(arr)
    return gt.buffer, arr.shape, arr.dtype


def gpu_to_numpy(buf: CudaBuffer, shape, dtype, stream=None) -> np.ndarray:
    return gputensor_to_numpy(GpuTensor(buf, tuple(shape), dtype, buf.device_id))


# ───────────────────────────── matmul family ─────────────────────────────

def _out_dtype(a: GpuTensor, out_dtype) -> np.dtype:
    return np.dtype(out_dtype) if out_dtype is not None else a.dtype


def _check_pair(a: GpuTensor, b: GpuTensor) -> None:
    if a.dtype != b.dtype:
        raise TypeError(f"matmul operands must share a dtype ({a.dtype} vs {b.dtype})")
    if a.device_id != b.device_id:
        raise ValueError(f"operands on different devices ({a.device_id} vs {b.device_id})")


def _matmul2d(a: GpuTensor, b: GpuTensor, trans_b: bool, out_dtype=None, epi=None) -> GpuTensor:
    _check_pair(a, b)
    M, K = a.shape
    if trans_b:
        N, Kb = b.shape
    else:
        Kb, N = b.shape
    if K != Kb:
        raise ValueError(f"matmul shape mismatch: {a.shape} x {b.shape}{'^T' if trans_b else ''}")
    odt = _out_dtype(a, out_dtype)
    dev = a.device_id
    c = _alloc((M, N), odt, dev)
    with E.on_device(dev):
        E.gemm(M, N, K, a.ptr, K, 0, b.ptr, K if trans_b else N, 1 if trans_b else 0,
               c.ptr, N, E.dtype_code(a.dtype), E.dtype_code(odt), epi=epi, device=dev)
    return c


def _batched(a: GpuTensor, b: GpuTensor, trans_b: bool, out_dtype=None, epi=None) -> GpuTensor:
    _check_pair(a, b)
    if a.ndim < 2 or b.ndim < 2:
        raise ValueError("batched matmul needs operands of rank >= 2")
    M, K = a.shape[-2:]
    if trans_b:
        N, Kb = b.shape[-2:]
    else:
        Kb, N = b.shape[-2:]
    if K != Kb:
        raise ValueError(f"matmul shape mismatch: {a.shape} x {b.shape}{'^T' if trans_b else ''}")
    lead = a.shape[:-2]
    batch = int(np.prod(lead, dtype=np.int64)) if lead else 1
    b_batch = int(np.prod(b.shape[:-2], dtype=np.int64)) if b.ndim > 2 else 1
    if b_batch not in (1, batch):
        raise ValueError(f"batch dims differ: {a.shape} vs {b.shape}")
    odt = _out_dtype(a, out_dtype)
    dev = a.device_id
    c = _alloc(lead + (M, N), odt, dev)
    ldb = K if trans_b else N
    with E.on_device(dev):
        if b.ndim == 2 or b_batch == 1:
            # Shared right operand: one GEMM over the stacked rows of A.
            E.gemm(batch * M, N, K, a.ptr, K, 0, b.ptr, ldb, 1 if trans_b else 0, c.ptr, N,
                   E.dtype_code(a.dtype), E.dtype_code(odt), epi=epi, device=dev)
        elif b_batch == batch:
            bt = E.make_batch(batch, 1, a=(M * K, 0), b=(N * K, 0), c=(M * N, 0))
            E.gemm(M, N, K, a.ptr, K, 0, b.ptr, ldb, 1 if trans_b else 0, c.ptr, N,
                   E.dtype_code(a.dtype), E.dtype_code(odt), epi=epi, batch=bt, device=dev)
        else:
            raise ValueError(f"batch dims differ: {a.shape} vs {b.shape}")
    return c


def dev_matmul(gt_a: GpuTensor, gt_b: GpuTensor) -> GpuTensor:
    """C = A @ B; A (M,K), B (K,N) (``_cuda_ops.pyx:1088-1102``)."""
    return _matmul2d(gt_a, gt_b, False)


def dev_matmul_nt(gt_a: GpuTensor, gt_b: GpuTensor) -> GpuTensor:
    """C = A @ B^T; A (M,K), B (N,K) (``_cuda_ops.pyx:1105-1119``)."""
    return _matmul2d(gt_a, gt_b, True)


def dev_batched_matmul(gt_a: GpuTensor, gt_b: GpuTensor) -> GpuTensor:
    """(..., M, K) @ (..., K, N) (``_cuda_ops.pyx:1122-1149``); B may also be
    2-D (shared across the batch)."""
    return _batched(gt_a, gt_b, False)


def dev_batched_matmul_nt(gt_a: GpuTensor, gt_b: GpuTensor) -> GpuTensor:
    """(..., M, K) @ (..., N, K)^T in one launch (``_cuda_ops.pyx:1152-1190``)."""
    return _batched(gt_a, gt_b, True)


def dev_linear_forward(gt_x: GpuTensor, gt_weight: GpuTensor, gt_bias: GpuTensor | None = None,
                       activation: str = "none", out_dtype=None) -> GpuTensor:
    """y = act(x @ W^T + bias) with bias and activation fused into the GEMM
    epilogue (``_cuda_ops.pyx:1278-1302``; activation was a separate launch,
    ``nn/functional.py:37-40``)."""
    _check_pair(gt_x, gt_weight)
    K = gt_x.shape[-1]
    M = int(np.prod(gt_x.shape[:-1], dtype=np.int64))
    N, Kw = gt_weight.shape
    if Kw != K:
        raise ValueError(f"linear shape mismatch: x {gt_x.shape}, W {gt_weight.shape}")
    odt = _out_dtype(gt_x, out_dtype)
    dev = gt_x.device_id
    y = _alloc(gt_x.shape[:-1] + (N,), odt, dev)
    bias_ptr, bias_dt = 0, DT_F32
    if gt_bias is not None:
        if gt_bias.numel != N:
            raise ValueError(f"bias has {gt_bias.numel} elements, expected {N}")
        bias_ptr, bias_dt = gt_bias.ptr, E.dtype_code(gt_bias.dtype)
    epi = E.make_epilogue(bias_ptr=bias_ptr, bias_dt=bias_dt, act=E.act_code(activation))
    with E.on_device(dev):
        E.gemm(M, N, K, gt_x.ptr, K, 0, gt_weight.ptr, K, 1, y.ptr, N,
               E.dtype_code(gt_x.dtype), E.dtype_code(odt), epi=epi, device=dev)
    return y


# ───────────────────────────── attention glue ─────────────────────────────

def _unary(gt: GpuTensor, alpha: float, act: int) -> GpuTensor:
    dev = gt.device_id
    out = _alloc(gt.shape, gt.dtype, dev)
    code = E.dtype_code(gt.dtype)
    with E.on_device(dev):
        E.unary(gt.ptr, code, out.ptr, code, gt.numel, alpha, act, device=dev)
    return out


def dev_muls(gt: GpuTensor, scalar: float) -> GpuTensor:
    """y = scalar * x (``_cuda_ops.pyx:990-998``)."""
    return _unary(gt, float(scalar), ACT_NONE)


def dev_silu(gt: GpuTensor) -> GpuTensor:
    """SiLU (``_cuda_ops.pyx:944-945``)."""
    return _unary(gt, 1.0, ACT_SILU)


def dev_gelu(gt: GpuTensor) -> GpuTensor:
    """GELU, tanh form (``_cuda_ops.pyx:947-948``)."""
    return _unary(gt, 1.0, ACT_GELU_TANH)


def dev_softmax(gt: GpuTensor, dim: int = -1) -> GpuTensor:
    """Softmax over the last dimension (``_cuda_ops.pyx:1016-1034``)."""
    nd = len(gt.shape)
    if nd == 0:
        raise ValueError("softmax of a 0-d tensor")
    if dim not in (-1, nd - 1):
        raise NotImplementedError("dev_softmax supports the last dimension only")
    cols = gt.shape[-1]
    rows = gt.numel // cols if cols else 0
    dev = gt.device_id
    out = _alloc(gt.shape, gt.dtype, dev)
    code = E.dtype_code(gt.dtype)
    with E.on_device(dev):
        E.softmax_rows(gt.ptr, code, cols, out.ptr, code, cols, rows, cols, 1.0, device=dev)
    return out


def _norm_launch(gt: GpuTensor, gamma, beta, eps: float, mod=None, group_rows: int = 1,
                 out_dtype=None) -> GpuTensor:
    cols = gt.shape[-1]
    rows = gt.numel // cols if cols else 0
    dev = gt.device_id
    odt = np.dtype(out_dtype) if out_dtype is not None else gt.dtype
    out = _alloc(gt.shape, odt, dev)
    for t, name in ((gamma, "gamma"), (beta, "beta")):
        if t is not None and (t.dtype != np.float32 or t.numel != cols):
            raise ValueError(f"layer norm {name} must be fp32 with {cols} elements")
    if (gamma is None) != (beta is None):
        raise ValueError("layer norm gamma and beta go together")
    mod_ptr, mod_dt, ld_mod = None, DT_F32, 0
    if mod is not None:
        if mod.shape[-1] != 2 * cols:
            raise ValueError(f"modulation rows must hold 2 x {cols} values, got {mod.shape}")
        mod_ptr, mod_dt, ld_mod = C.c_void_p(mod.ptr), E.dtype_code(mod.dtype), 2 * cols
    with E.on_device(dev):
        s = E.get_stream(dev)
        check(lib.sf_layernorm_modulate(rows, cols, C.c_void_p(gt.ptr), E.dtype_code(gt.dtype), cols,
                                        C.c_void_p(gamma.ptr) if gamma is not None else None,
                                        C.c_void_p(beta.ptr) if beta is not None else None,
                                        float(eps), mod_ptr, mod_dt, ld_mod, int(group_rows),
                                        C.c_void_p(out.ptr), E.dtype_code(odt), cols,
                                        C.c_void_p(s) if s else None), "sf_layernorm_modulate")
    return out


def dev_layer_norm(gt: GpuTensor, gt_gamma: GpuTensor | None = None,
                   gt_beta: GpuTensor | None = None, eps: float = 1e-5) -> GpuTensor:
    """LayerNorm over the last dimension (``dev_layer_norm`` behind
    ``nn/layers.py:470-493``; kernel ``_cuda_kernels.cu:1070-1093``), fp32 /
    bf16 / fp16 in and out, fp32 gamma and beta."""
    return _norm_launch(gt, gt_gamma, gt_beta, eps)


def dev_ada_layer_norm(gt: GpuTensor, gt_params: GpuTensor, gt_gamma: GpuTensor | None = None,
                       gt_beta: GpuTensor | None = None, eps: float = 1e-5,
                       out_dtype=None) -> GpuTensor:
    """AdaLayerNorm (``diffusion/models.py:478-487``) of ``x [B, N, C]`` with
    the modulation linear's output ``params [B, 2C]``: LayerNorm, then
    ``h * (1 + params[b, :C]) + params[b, C:]`` for every token of sample b,
    in one kernel.  New (the reference modulates on the host)."""
    if gt.ndim != 3 or gt_params.ndim != 2 or gt_params.shape[0] != gt.shape[0]:
        raise ValueError(f"adaLN shapes: x {gt.shape}, params {gt_params.shape}")
    return _norm_launch(gt, gt_gamma, gt_beta, eps, gt_params, gt.shape[1], out_dtype)


def dev_unsqueeze(gt: GpuTensor, dim: int) -> GpuTensor:
    shape = list(gt.shape)
    if dim < 0:
        dim = len(shape) + 1 + dim
    shape.insert(dim, 1)
    return GpuTensor(gt.buffer, tuple(shape), gt.dtype, gt.device_id)


def dev_squeeze(gt: GpuTensor, dim=None) -> GpuTensor:
    shape = list(gt.shape)
    if dim is not None:
        if dim < 0:
            dim = len(shape) + dim
        if 0 <= dim < len(shape) and shape[dim] == 1:
            shape.pop(dim)
    else:
        shape = [s for s in shape if s != 1]
    return GpuTensor(gt.buffer, tuple(shape), gt.dtype, gt.device_id)


def dev_reshape(gt: GpuTensor, new_shape) -> GpuTensor:
    new_shape = tuple(int(s) for s in new_shape)
    if -1 in new_shape:
        known = int(np.prod([s for s in new_shape if s != -1], dtype=np.int64))
        new_shape = tuple(gt.numel // known if s == -1 else s for s in new_shape)
    if int(np.prod(new_shape, dtype=np.int64)) != gt.numel:
        raise ValueError(f"cannot reshape {gt.shape} to {new_shape}")
    return GpuTensor(gt.buffer, new_shape, gt.dtype, gt.device_id)


# ───────────────────────────── host-array variants ─────────────────────────────

def _host_dtype(*arrs):
    dt = np.result_type(*[a.dtype for a in arrs])
    if dt not in (np.float16, np.float32) and not (bfloat16 is not None and dt == bfloat16):
        dt = np.dtype(np.float32)
    return dt


def cuda_matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Host C = A @ B through the device (``_cuda_ops.pyx:2120-2147``)."""
    dt = _host_dtype(a, b)
    ga = gputensor_from_numpy(np.ascontiguousarray(a, dtype=dt))
    gb = gputensor_from_numpy(np.ascontiguousarray(b, dtype=dt))
    return gputensor_to_numpy(dev_matmul(ga, gb))


def cuda_matmul_nt(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Host C = A @ B^T (``_cuda_ops.pyx:2150-2177``)."""
    dt = _host_dtype(a, b)
    ga = gputensor_from_numpy(np.ascontiguousarray(a, dtype=dt))
    gb = gputensor_from_numpy(np.ascontiguousarray(b, dtype=dt))
    return gputensor_to_numpy(dev_matmul_nt(ga, gb))


def cuda_batched_matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Host batched (..., M, K) @ (..., K, N) (``_cuda_ops.pyx:2180-2225``)."""
    dt = _host_dtype(a, b)
    ga = gputensor_from_numpy(np.ascontiguousarray(a, dtype=dt))
    gb = gputensor_from_numpy(np.ascontiguousarray(b, dtype=dt))
    return gputensor_to_numpy(dev_batched_matmul(ga, gb))


def cuda_linear_forward(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None = None,
                        activation: str = "none") -> np.ndarray:
    """Host y = x @ W^T + bias (``_cuda_ops.pyx:2453-2471``), bias fused on the
    device instead of added in NumPy."""
    dt = _host_dtype(x, weight)
    K = x.shape[-1]
    gx = gputensor_from_numpy(np.ascontiguousarray(x.reshape(-1, K), dtype=dt))
    gw = gputensor_from_numpy(np.ascontiguousarray(weight, dtype=dt))
    gb = gputensor_from_numpy(np.ascontiguousarray(bias, dtype=dt).ravel()) if bias is not None else None
    y = gputensor_to_numpy(dev_linear_forward(gx, gw, gb, activation))
    return y.reshape(x.shape[:-1] + (weight.shape[0],))


def _host_unary(x: np.ndarray, fn) -> np.ndarray:
    """Host array -> device -> ``fn`` -> host, in the array's dtype (fp32 for
    anything the engine does not store), shape kept."""
    dt = _host_dtype(x)
    g = gputensor_from_numpy(np.ascontiguousarray(x, dtype=dt))
    return gputensor_to_numpy(fn(g)).reshape(np.shape(x))


def cuda_muls(a: np.ndarray, scalar: float) -> np.ndarray:
    """Host ``scalar * a`` through the device (``_cuda_ops.pyx:1926-1944``)."""
    return _host_unary(a, lambda g: dev_muls(g, scalar))


def cuda_silu(x: np.ndarray) -> np.ndarray:
    """Host SiLU through the device (``_cuda_ops.pyx:1954-1955``): the path
    ``F.silu`` takes for a ``cuda`` tensor without device data."""
    return _host_unary(x, dev_silu)


def cuda_gelu(x: np.ndarray) -> np.ndarray:
    """Host GELU-tanh through the device (``_cuda_ops.pyx:1957-1958``)."""
    return _host_unary(x, dev_gelu)


def cuda_softmax(x: np.ndarray, dim: int = -1) -> np.ndarray:
    """Host softmax over the last dimension (``_cuda_ops.pyx:2011-2040``)."""
    return _host_unary(x, lambda g: dev_softmax(g, -1))


def cuda_layer_norm(x: np.ndarray, gamma: np.ndarray | None, beta: np.ndarray | None,
                    eps: float = 1e-5) -> np.ndarray:
    """Host LayerNorm of an (N, D) array (``_cuda_ops.pyx:2231-2270``)."""
    g = gputensor_from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    gg = gputensor_from_numpy(np.ascontiguousarray(gamma, dtype=np.float32)) if gamma is not None else None
    gb = gputensor_from_numpy(np.ascontiguousarray(beta, dtype=np.float32)) if beta is not None else None
    return gputensor_to_numpy(dev_layer_norm(g, gg, gb, eps))


def set_tf32_enabled(enable: bool) -> None:
    """``allow_tf32``: True permits single-pass TF32 for fp32 GEMMs; False
    (default) keeps fp32 accuracy via 3xTF32 (``_cuda_ops.pyx:2474-2477``)."""
    check(lib.sf_set_fp32_mode(FP32_TF32 if enable else FP32_ACCURATE), "sf_set_fp32_mode")


# ───────────────────────────── runtime ─────────────────────────────

def get_device_count() -> int:
    return E.device_count()


def set_device(device: int) -> None:
    E.set_device(device)


def get_current_device() -> int:
    return E.current_device()


def device_synchronize() -> None:
    check(lib.sf_device_synchronize(), "sf_device_synchronize")


def get_device_properties(device: int) -> dict:
    p = DeviceProps()
    check(lib.sf_device_properties(int(device), C.byref(p)), "sf_device_properties")
    return {
        "name": p.name.decode(errors="replace"),
        "total_memory": int(p.total_memory),
        "major": p.major,
        "minor": p.minor,
        "multi_processor_count": p.multi_processor_count,
        "shared_mem_per_block": int(p.shared_mem_per_block),
        "max_threads_per_block": p.max_threads_per_block,
        "warp_size": p.warp_size,
        "max_threads_per_mp": p.max_threads_per_mp,
        "l2_cache_size": int(p.l2_cache_size),
    }


def get_device_capability(device: int = 0) -> tuple[int, int]:
    p = get_device_properties(device)
    return (p["major"], p["minor"])


def get_device_name(device: int = 0) -> str:
    return get_device_properties(device)["name"]


def mem_info() -> tuple[int, int]:
    f, t = C.c_size_t(), C.c_size_t()
    check(lib.sf_mem_info(C.byref(f), C.byref(t)), "sf_mem_info")
    return (f.value, t.value)


def empty_cache(device: int = -1) -> None:
    E.release_workspaces()
    check(lib.sf_empty_cache(int(device)), "sf_empty_cache")


def gpu_malloc(nbytes: int) -> CudaBuffer:
    return _make_buffer(nbytes, E.current_device())


def gpu_free(buf: CudaBuffer) -> None:
    buf.free()


def can_access_peer(device: int, peer_device: int) -> bool:
    c = C.c_int32()
    check(lib.sf_can_access_peer(int(device), int(peer_device), C.byref(c)), "sf_can_access_peer")
    return bool(c.value)


def init_p2p() -> None:
    check(lib.sf_enable_peer_access_all(), "sf_enable_peer_access_all")


def init_all_devices() -> None:
    """Touch every device (engine state is created lazily) and enable P2P."""
    prev = E.current_device()
    for d in range(E.device_count()):
        E.set_device(d)
        E.device_error_status(d)
    E.set_device(prev)
    init_p2p()


class CudaStream:
    """Owned CUDA stream (``_cuda_ops.pyx:608-643``)."""

    def __init__(self, device_id: int = 0, non_blocking: bool = True):
        p = C.c_void_p()
        check(lib.sf_stream_create(int(device_id), 1 if non_blocking else 0, C.byref(p)),
              "sf_stream_create")
        self._stream = p.value
        self._device_id = device_id

    def synchronize(self) -> None:
        E.stream_sync(self._stream)

    def wait_event(self, event: "CudaEvent") -> None:
        check(lib.sf_stream_wait_event(C.c_void_p(self._stream), C.c_void_p(event._event)),
              "sf_stream_wait_event")

    @property
    def cuda_stream(self) -> int:
        return self._stream

    @property
    def device_id(self) -> int:
        return self._device_id

    def __del__(self):
        try:
            if self._stream:
                lib.sf_stream_destroy(C.c_void_p(self._stream))
                self._stream = None
        except Exception:
            pass


class CudaEvent:
    """CUDA event for timing / sync (``_cuda_ops.pyx:646-673``)."""

    def __init__(self, enable_timing: bool = True):
        p = C.c_void_p()
        check(lib.sf_event_create(1 if enable_timing else 0, C.byref(p)), "sf_event_create")
        self._event = p.value

    def record(self, stream: CudaStream | None = None) -> None:
        s = stream._stream if stream is not None else E.get_stream(E.current_device())
        check(lib.sf_event_record(C.c_void_p(self._event), C.c_void_p(s) if s else None),
              "sf_event_record")

    def synchronize(self) -> None:
        check(lib.sf_event_synchronize(C.c_void_p(self._event)), "sf_event_synchronize")

    def elapsed_time(self, end: "CudaEvent") -> float:
        ms = C.c_float()
        check(lib.sf_event_elapsed_ms(C.c_void_p(self._event), C.c_void_p(end._event),
                                      C.byref(ms)), "sf_event_elapsed_ms")
        return ms.value

    def __del__(self):
        try:
            if self._event:
                lib.sf_event_destroy(C.c_void_p(self._event))
                self._event = None
        except Exception:
            pass


def cublas_set_stream(stream: CudaStream | None = None) -> None:
    """Route subsequent engine launches on the current device to ``stream``
    (the reference set the cuBLAS handle's stream, ``_cuda_ops.pyx:725-729``)."""
    E.set_stream(E.current_device(), stream._stream if stream is not None else None)


# ───────────────────────────── out of scope ─────────────────────────────

_OUT_OF_SCOPE = {
    "dev_exp", "dev_log", "dev_sqrt", "dev_rsqrt", "dev_sigmoid", "dev_tanh", "dev_sin",
    "dev_cos", "dev_neg", "dev_abs", "dev_relu", "dev_add", "dev_sub", "dev_mul", "dev_div",
    "dev_adds", "dev_clamp", "dev_log_softmax", "dev_cross_entropy",
    "dev_rms_norm", "dev_dropout", "dev_embedding", "dev_adamw_step", "dev_sum", "dev_fill",
    "dev_copy", "dev_transpose_2d", "dev_pow_scalar", "dev_expand", "dev_slice", "dev_cat",
    "dev_stack", "dev_chunk", "dev_cumsum", "dev_mean_dim", "dev_sum_dim", "dev_sum_tensor",
    "dev_mean_tensor", "cuda_exp", "cuda_log", "cuda_sqrt", "cuda_rsqrt", "cuda_sigmoid",
    "cuda_tanh", "cuda_sin", "cuda_cos", "cuda_neg", "cuda_abs", "cuda_add", "cuda_sub",
    "cuda_mul", "cuda_div", "cuda_adds", "cuda_relu",
    "cuda_silu_fwd", "cuda_clamp", "cuda_log_softmax", "cuda_cross_entropy",
    "cuda_rms_norm", "cuda_adamw_step", "cuda_dropout", "cuda_embedding",
    "cuda_transpose_2d", "cuda_sum", "cuda_fill",
}


def __getattr__(name: str):
    if name in _OUT_OF_SCOPE:
        def _missing(*_a, **_k):
            raise NotImplementedError(
                f"_cuda_ops.{name} is outside the B200 engine's matmul path "
                "(only the GEMM / linear / attention-product surface is provided)")
        _missing.__name__ = name
        return _missing
    raise AttributeError(name)
