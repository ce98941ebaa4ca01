"""``nn.Linear`` / ``nn.functional`` mirror for GPU-resident tensors.

Mirrors the GPU branches of the reference's modules, with the same names,
argument meaning and error behaviour:

* ``Linear`` -- ``nn/layers.py:59-146``: weight ``[out, in]`` and bias
  ``[out]`` drawn U(-1/sqrt(in), 1/sqrt(in)) (Kaiming-uniform, ``:66-74``);
  ``forward`` moves parameters to the input's device on first use
  (``:89-105``) and calls ``dev_linear_forward`` (``:108-110``).  New: an
  optional fused ``activation`` and a storage ``dtype`` (bf16 / fp16).
* ``functional.linear`` -- ``nn/functional.py:374-395``.
* ``functional.scaled_dot_product_attention`` -- GPU path of
  ``nn/functional.py:310-321``: QK^T (one batched launch, scale fused in
  its epilogue), row softmax, P.V.
* ``functional.silu`` / ``gelu`` / ``softmax`` -- ``nn/functional.py:37-145``.
"""
from __future__ import annotations

import math
import types

import numpy as np

from . import _cuda_ops as ops
from . import engine as E
from ._cuda_ops import GpuTensor


class Linear:
    """y = act(x W^T + b) on the GPU (``nn/layers.py:59-146``)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None,
                 dtype=np.float32, rng: np.random.Generator | None = None):
        self.in_features = in_features
        self.out_features = out_features
        dev = _device_index(device)
        k = 1.0 / math.sqrt(in_features)
        gen = rng if rng is not None else np.random
        w = gen.uniform(-k, k, (out_features, in_features)).astype(np.float32)
        self.weight = ops.gputensor_from_numpy(w.astype(dtype), dev)
        if bias:
            b = gen.uniform(-k, k, (out_features,)).astype(np.float32)
            self.bias = ops.gputensor_from_numpy(b.astype(dtype), dev)
        else:
            self.bias = None

    def _to(self, dev: int) -> None:
        if self.weight.device_id != dev:
            self.weight = ops.gputensor_to_device(self.weight, dev)
        if self.bias is not None and self.bias.device_id != dev:
            self.bias = ops.gputensor_to_device(self.bias, dev)

    def forward(self, x: GpuTensor, activation: str = "none") -> GpuTensor:
        self._to(x.device_id)
        ops.set_device(x.device_id)
        return ops.dev_linear_forward(x, self.weight, self.bias, activation)

    __call__ = forward


def _device_index(device) -> int:
    if device is None:
        return E.current_device()
    if isinstance(device, int):
        return device
    s = str(device)
    if s.startswith("cuda"):
        return int(s.split(":")[1]) if ":" in s else 0
    raise ValueError(f"not a CUDA device: {device!r}")


def _linear(input: GpuTensor, weight: GpuTensor, bias: GpuTensor | None = None,
            activation: str = "none") -> GpuTensor:
    """``F.linear`` (``nn/functional.py:374-395``) plus an optional fused activation."""
    return ops.dev_linear_forward(input, weight, bias, activation)


def _silu(input: GpuTensor) -> GpuTensor:
    return ops.dev_silu(input)


def _gelu(input: GpuTensor) -> GpuTensor:
    return ops.dev_gelu(input)


def _softmax(input: GpuTensor, dim: int = -1) -> GpuTensor:
    return ops.dev_softmax(input, dim)


def _sdpa(q: GpuTensor, k: GpuTensor, v: GpuTensor, attn_mask=None, dropout_p: float = 0.0,
          scale: float | None = None, score_dtype=np.float32) -> GpuTensor:
    """GPU path of ``F.scaled_dot_product_attention`` (``nn/functional.py:298-321``).

    ``scores = (Q K^T) * scale`` in fp32 (scale applied in the GEMM epilogue,
    bit-identical to the separate ``dev_muls``), row softmax in fp32 written
    in the value dtype, then ``P V``.  Masks and dropout are not part of the
    GPU path in the reference either (it falls back to the host for a mask).
    """
    if attn_mask is not None:
        raise NotImplementedError("attention masks are not supported on the GPU path")
    if dropout_p:
        raise NotImplementedError("attention dropout is not supported on the GPU path")
    d = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if q.ndim < 2 or q.shape[:-2] != k.shape[:-2] or k.shape != v.shape or k.shape[-1] != d:
        raise ValueError(f"sdpa shapes: q {q.shape}, k {k.shape}, v {v.shape}")
    M, S = q.shape[-2], k.shape[-2]
    lead = q.shape[:-2]
    batch = int(np.prod(lead, dtype=np.int64)) if lead else 1
    dev = q.device_id
    code = E.dtype_code(q.dtype)
    scores = ops._alloc(lead + (M, S), score_dtype, dev)
    probs = ops._alloc(lead + (M, S), q.dtype, dev)
    out = ops._alloc(lead + (M, d), q.dtype, dev)
    with E.on_device(dev):
        bt = E.make_batch(batch, 1, a=(M * d, 0), b=(S * d, 0), c=(M * S, 0))
        E.gemm(M, S, d, q.ptr, d, 0, k.ptr, d, 1, scores.ptr, S, code,
               E.dtype_code(score_dtype), epi=E.make_epilogue(alpha=scale), batch=bt, device=dev)
        E.softmax_rows(scores.ptr, E.dtype_code(score_dtype), S, probs.ptr, code, S, batch * M, S,
                       1.0, device=dev)
        bt2 = E.make_batch(batch, 1, a=(M * S, 0), b=(S * d, 0), c=(M * d, 0))
        E.gemm(M, d, S, probs.ptr, S, 0, v.ptr, d, 0, out.ptr, d, code, code, batch=bt2,
               device=dev)
    return out


functional = types.SimpleNamespace(
    linear=_linear, silu=_silu, gelu=_gelu, softmax=_softmax,
    scaled_dot_product_attention=_sdpa,
)
