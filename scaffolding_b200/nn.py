"""``nn.Linear`` / ``nn.functional`` mirror for GPU-resident tensors.

Mirrors the GPU branches of the reference's modules, with the same names,
argument meaning and error behaviour:

* ``Linear`` -- ``nn/layers.py:59-146``: weight ``[out, in]`` and bias
  ``[out]`` drawn U(-1/sqrt(in), 1/sqrt(in)) (Kaiming-uniform, ``:66-74``);
  ``forward`` moves parameters to the input's device on first use
  (``:89-105``) and calls ``dev_linear_forward`` (``:108-110``).  New: an
  optional fused ``activation`` and a storage ``dtype`` (bf16 / fp16);
  ``to(device, dtype)`` (``Module.to``, ``nn/module.py:208-235``) and
  ``from_weights`` convert fp32 weights to bf16 / fp16 on the device at load.
* ``functional.linear`` -- ``nn/functional.py:374-395``.
* ``functional.scaled_dot_product_attention`` -- GPU path of
  ``nn/functional.py:310-321``: for bf16/fp16 with head_dim 64 the fused
  attention kernel (one launch, scores never leave the SM); otherwise QK^T
  (one batched launch, scale fused in its epilogue), row softmax, P.V.
* ``functional.silu`` / ``gelu`` / ``softmax`` -- ``nn/functional.py:37-145``.
* ``Sequential`` -- the container the reference's models stack layers in.
* ``LayerNorm`` (``nn/layers.py:443-521``) and ``AdaLayerNorm``
  (``diffusion/models.py:470-487``), the norms in front of the DiT linears.
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

    @classmethod
    def from_weights(cls, weight: np.ndarray, bias: np.ndarray | None = None, device=None,
                     dtype=np.float32) -> "Linear":
        """A layer holding the given host weights (``[out, in]``, ``[out]``):
        each array is uploaded in fp32 as the reference's ``_param_to_device``
        does (``nn/layers.py:18-35``) and converted to ``dtype`` on the device
        (bf16 / fp16 storage for the 16-bit GEMM paths), one parameter at a
        time."""
        out_f, in_f = weight.shape
        lin = cls.__new__(cls)
        lin.in_features, lin.out_features = in_f, out_f
        dev = _device_index(device)
        lin.weight = ops.gputensor_astype(
            ops.gputensor_from_numpy(np.ascontiguousarray(weight, dtype=np.float32), dev), dtype)
        lin.bias = None
        if bias is not None:
            lin.bias = ops.gputensor_astype(
                ops.gputensor_from_numpy(np.ascontiguousarray(bias, dtype=np.float32), dev), dtype)
        return lin

    def to(self, device=None, dtype=None) -> "Linear":
        """``Module.to`` (``nn/module.py:208-235``): move the parameters to
        ``device`` and/or convert them to ``dtype`` on the device, one at a
        time (the old buffers return to the pool before the next one)."""
        if device is not None:
            self._to(_device_index(device))
        if dtype is not None:
            self.weight = ops.gputensor_astype(self.weight, dtype)
            if self.bias is not None:
                self.bias = ops.gputensor_astype(self.bias, dtype)
        return self

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


class LayerNorm:
    """``nn.LayerNorm`` (``nn/layers.py:443-521``) over the last dimension:
    fp32 weight (ones) and bias (zeros) on the device, GPU forward through
    ``dev_layer_norm``."""

    def __init__(self, normalized_shape, eps: float = 1e-5, elementwise_affine: bool = True,
                 device=None):
        if isinstance(normalized_shape, int):
            normalized_shape = (normalized_shape,)
        self.normalized_shape = tuple(normalized_shape)
        self.eps = eps
        dev = _device_index(device)
        C = self.normalized_shape[-1]
        if elementwise_affine:
            self.weight = ops.gputensor_from_numpy(np.ones(C, np.float32), dev)
            self.bias = ops.gputensor_from_numpy(np.zeros(C, np.float32), dev)
        else:
            self.weight = self.bias = None

    def forward(self, x: GpuTensor) -> GpuTensor:
        return ops.dev_layer_norm(x, self.weight, self.bias, self.eps)

    __call__ = forward


class AdaLayerNorm:
    """``AdaLayerNorm`` (``diffusion/models.py:470-487``): LayerNorm of
    ``x [B, N, C]`` modulated per sample by ``linear(cond)`` (``[B, 2C]``:
    scale ``+ 1`` then shift), the modulation applied in the norm kernel."""

    def __init__(self, dim: int, cond_dim: int, device=None, dtype=np.float32,
                 rng: np.random.Generator | None = None):
        self.norm = LayerNorm(dim, device=device)
        self.linear = Linear(cond_dim, dim * 2, device=device, dtype=dtype, rng=rng)

    def forward(self, x: GpuTensor, cond: GpuTensor) -> GpuTensor:
        params = self.linear(cond)
        return ops.dev_ada_layer_norm(x, params, self.norm.weight, self.norm.bias, self.norm.eps)

    __call__ = forward


class Sequential:
    """Modules applied in order (``nn/module.py:345``): each
    takes and returns a GpuTensor."""

    def __init__(self, *modules):
        self.layers = list(modules)

    def forward(self, x: GpuTensor) -> GpuTensor:
        for m in self.layers:
            x = m(x)
        return x

    def to(self, device=None, dtype=None) -> "Sequential":
        for m in self.layers:
            if hasattr(m, "to"):
                m.to(device, dtype)
        return self

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
    if d == 64 and code != E.DT_F32 and q.dtype == k.dtype == v.dtype:
        return _sdpa_fused(q, k, v, float(scale), lead, batch, M, S, code, dev)
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


# Calls of scaled_dot_product_attention served by the fused kernel.
sdpa_fused_calls = 0

# The fused kernel's grid holds at most 65535 batch items per launch.
_FUSED_MAX_BATCH = 65535


def _sdpa_fused(q, k, v, scale, lead, batch, M, S, code, dev) -> GpuTensor:
    """16-bit, head_dim 64: one fused launch (QK^T, online softmax and P.V on
    chip, ``sf_attention_fwd``) per 65535 batch items instead of the three
    launches and the [.., M, S] score and probability buffers of the chain
    below.  Each (…, M, 64) matrix is one batch item with a single head."""
    global sdpa_fused_calls
    out = ops._alloc(lead + (M, 64), q.dtype, dev)
    with E.on_device(dev):
        for b0 in range(0, batch, _FUSED_MAX_BATCH):
            nb = min(_FUSED_MAX_BATCH, batch - b0)
            off = b0 * 2
            E.attention(nb, 1, M, S, q.ptr + off * M * 64, 64, M * 64, k.ptr + off * S * 64, 64,
                        S * 64, v.ptr + off * S * 64, 64, S * 64, out.ptr + off * M * 64, 64,
                        M * 64, scale, dtype=code, head_dim=64, device=dev)
    sdpa_fused_calls += 1
    return out


functional = types.SimpleNamespace(
    linear=_linear, silu=_silu, gelu=_gelu, softmax=_softmax,
    scaled_dot_product_attention=_sdpa,
)
