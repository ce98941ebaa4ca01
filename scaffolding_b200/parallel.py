"""``DataParallel`` over the GPUs of one process, rows moved device to device.

Mirrors ``nn/parallel.py:45-290`` of the reference -- same constructor
(``module, device_ids=None, output_device=None, dim=0``), same split rule
(``chunk = ceil(batch / n_devices)`` rows per device in device order, devices
past the end of the batch get nothing, ``:118-131``), parameters replicated
once per device with ``gputensor_to_device`` and cached (``:149-200``), one
forward per device with that device current (``:202-227``) and the outputs
concatenated along ``dim`` 0 on ``output_device`` (``:229-267``) -- with the
data path rebuilt for NVLink:

* scatter: each device's rows are copied from the input's device with one
  ``cudaMemcpyPeerAsync`` (copy engines over NVLink, no host round trip);
  the input device's own rows are used in place.  The reference downloaded
  the batch to the host and re-uploaded every chunk (``:128-132``).
* forward: every replica launches on its own device; launches are
  asynchronous, so all devices compute at once.
* gather: the replicas' outputs are copied peer to peer into one tensor on
  ``output_device`` (the reference went through host NumPy, ``:245-266``).

The wrapped module is any callable taking and returning a ``GpuTensor``
whose parameters are ``GpuTensor`` attributes (directly, or inside lists,
tuples or dicts, or nested modules): ``nn.Linear``, ``nn.Sequential`` and
``dit.DitBlock`` are.  Outputs must keep the input's rows (row i of the
output depends on row i of the input only), as the reference's gather
assumes.  Only ``dim`` 0 is supported.
"""
from __future__ import annotations

import copy
import ctypes as C

import numpy as np

from . import _cuda_ops as ops
from . import engine as E
from ._cuda_ops import GpuTensor
from ._lib import check, lib


def split_rows(batch: int, n_devices: int) -> list[tuple[int, int]]:
    """Row range [start, end) of each device, the reference's scatter rule
    (``nn/parallel.py:118-131``): ``ceil(batch / n)`` rows per device in
    device order; a device whose start is past the batch gets an empty range."""
    if n_devices < 1:
        raise ValueError("need at least one device")
    chunk = (batch + n_devices - 1) // n_devices
    out = []
    for i in range(n_devices):
        start = min(i * chunk, batch)
        out.append((start, min(start + chunk, batch)))
    return out


class _RowView:
    """Device memory inside another buffer (a row range); keeps the parent alive."""

    __slots__ = ("ptr", "nbytes", "device_id", "parent")

    def __init__(self, parent, offset: int, nbytes: int, device_id: int):
        self.parent = parent
        self.ptr = parent.ptr + offset
        self.nbytes = nbytes
        self.device_id = device_id


def row_slice(t: GpuTensor, start: int, end: int) -> GpuTensor:
    """Rows [start, end) of ``t`` along dim 0, without a copy."""
    row_bytes = (t.numel // t.shape[0]) * t.dtype.itemsize if t.shape[0] else 0
    view = _RowView(t.buffer, start * row_bytes, (end - start) * row_bytes, t.device_id)
    return GpuTensor(view, (end - start,) + t.shape[1:], t.dtype, t.device_id)


def _wait_device(dev: int) -> None:
    """Host wait for the work queued on ``dev``'s engine stream."""
    with E.on_device(dev):
        E.stream_sync(E.get_stream(dev))


class DataParallel:
    """Split-batch data parallelism across the GPUs of one process
    (``nn/parallel.py:45-290``)."""

    def __init__(self, module, device_ids: list[int] | None = None,
                 output_device: int | None = None, dim: int = 0):
        if dim != 0:
            raise NotImplementedError("DataParallel splits along dim 0 only")
        if device_ids is None:
            device_ids = list(range(ops.get_device_count())) or [0]
        self.module = module
        self.device_ids = list(device_ids)
        self.output_device = self.device_ids[0] if output_device is None else int(output_device)
        self.dim = dim
        self._param_cache: dict[tuple[int, int], GpuTensor] = {}
        self._replicas: dict[int, object] = {}
        if len(set(self.device_ids)) > 1:
            check(lib.sf_enable_peer_access_all(), "sf_enable_peer_access_all")

    # ── replication (nn/parallel.py:149-200)
    def _copy_value(self, v, dev: int, src_dev: int):
        if isinstance(v, GpuTensor):
            if v.device_id == dev:
                return v
            key = (id(v), dev)
            if key not in self._param_cache:
                self._param_cache[key] = ops.gputensor_to_device(v, dev)
            return self._param_cache[key]
        if isinstance(v, list):
            return [self._copy_value(x, dev, src_dev) for x in v]
        if isinstance(v, tuple):
            return tuple(self._copy_value(x, dev, src_dev) for x in v)
        if isinstance(v, dict):
            return {k: self._copy_value(x, dev, src_dev) for k, x in v.items()}
        if hasattr(v, "__dict__") and _holds_tensors(v):
            return self._replicate(v, dev, src_dev)
        return v

    def _replicate(self, module, dev: int, src_dev: int):
        rep = copy.copy(module)
        for name, v in vars(module).items():
            setattr(rep, name, self._copy_value(v, dev, src_dev))
        if hasattr(rep, "dev"):
            rep.dev = dev
        return rep

    def replica(self, dev: int):
        """The module with its parameters on ``dev`` (built once, cached)."""
        if dev not in self._replicas:
            src = _module_device(self.module)
            self._replicas[dev] = (self.module if src in (None, dev)
                                   else self._replicate(self.module, dev, src))
        return self._replicas[dev]

    def clear_cache(self) -> None:
        """Drop the replicated parameters (after the module's weights change)."""
        self._param_cache.clear()
        self._replicas.clear()

    # ── forward (nn/parallel.py:93-108)
    def forward(self, x: GpuTensor) -> GpuTensor:
        if len(self.device_ids) <= 1:
            return self.replica(self.device_ids[0] if self.device_ids else x.device_id)(x)
        ranges = split_rows(x.shape[0], len(self.device_ids))
        src = x.device_id
        row_bytes = (x.numel // x.shape[0]) * x.dtype.itemsize if x.shape[0] else 0
        _wait_device(src)  # the input is complete before other devices read it
        # scatter + forward: every device launches its share without waiting
        outs = []
        for dev, (r0, r1) in zip(self.device_ids, ranges):
            if r1 <= r0:
                continue
            if dev == src:
                part = row_slice(x, r0, r1)
            else:
                part = ops._alloc((r1 - r0,) + x.shape[1:], x.dtype, dev)
                with E.on_device(dev):
                    check(lib.sf_memcpy_peer(C.c_void_p(part.ptr), dev,
                                             C.c_void_p(x.ptr + r0 * row_bytes), src,
                                             (r1 - r0) * row_bytes,
                                             C.c_void_p(E.get_stream(dev) or 0) or None),
                          "sf_memcpy_peer")
            with E.on_device(dev):
                y = self.replica(dev)(part)
            if y.shape[0] != r1 - r0:
                raise ValueError("DataParallel needs outputs with the input's rows")
            outs.append((dev, r0, r1, y))
        # gather on the output device (nn/parallel.py:229-267), peer to peer
        y0 = outs[0][3]
        out = ops._alloc((x.shape[0],) + y0.shape[1:], y0.dtype, self.output_device)
        orow = (y0.numel // y0.shape[0]) * y0.dtype.itemsize
        for dev, r0, r1, y in outs:
            _wait_device(dev)
        with E.on_device(self.output_device):
            s = E.get_stream(self.output_device)
            for dev, r0, r1, y in outs:
                check(lib.sf_memcpy_peer(C.c_void_p(out.ptr + r0 * orow), self.output_device,
                                         C.c_void_p(y.ptr), dev, (r1 - r0) * orow,
                                         C.c_void_p(s) if s else None), "sf_memcpy_peer")
            E.stream_sync(s)
        return out

    __call__ = forward


def _holds_tensors(obj, depth: int = 0) -> bool:
    if depth > 4:
        return False
    for v in vars(obj).values():
        if isinstance(v, GpuTensor):
            return True
        if isinstance(v, (list, tuple)) and any(isinstance(x, GpuTensor) or
                                                (hasattr(x, "__dict__") and _holds_tensors(x, depth + 1))
                                                for x in v):
            return True
        if isinstance(v, dict) and any(isinstance(x, GpuTensor) for x in v.values()):
            return True
        if hasattr(v, "__dict__") and not isinstance(v, type) and _holds_tensors(v, depth + 1):
            return True
    return False


def _module_device(obj, depth: int = 0):
    """Device of the first GpuTensor parameter found in ``obj``, or None."""
    if depth > 4 or not hasattr(obj, "__dict__"):
        return None
    for v in vars(obj).values():
        if isinstance(v, GpuTensor):
            return v.device_id
        items = v if isinstance(v, (list, tuple)) else (v.values() if isinstance(v, dict) else [v])
        for x in items:
            if isinstance(x, GpuTensor):
                return x.device_id
            if hasattr(x, "__dict__") and not isinstance(x, (type, np.ndarray)):
                d = _module_device(x, depth + 1)
                if d is not None:
                    return d
    return None
