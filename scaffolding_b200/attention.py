"""GPU-resident multi-head attention of the DiT-family blocks.

The reference computes these attentions on the host after downloading the
projections and transposing them to ``(B, H, N, D)``:

* ``CrossAttentionBlock._attn`` (``diffusion/models.py:123-133``), used for
  its self-attention over the fused ``to_qkv`` projection (``:145-154``) and
  its cross-attention over text context (``:161-176``), and the DiT block's
  attention (``diffusion/models.py:529-536``);
* ``SpatialTemporalAttention.forward`` (``nn/video.py:345-432``): the same
  split of a fused QKV projection into heads (``:363-372``), then
  ``F.scaled_dot_product_attention`` for self- (``:373``) and
  cross-attention (``:405``).

Here the projections stay on the device in their natural ``[B, N, C]``
row layout (C = heads * head_dim, head h in columns ``[h*D, (h+1)*D)``) and
the attention reads every head in place, writing ``[B, N, C]`` -- the
``transpose(0, 2, 1, 3).reshape(B, N, C)`` the reference performs after its
attention.  bf16/fp16 with head_dim 64 runs the fused tcgen05 kernel
(``sf_attention_fwd``: QK^T, online softmax and P.V on chip); other dtypes
or head sizes run the engine's unfused chain (one batched QK^T launch with
the scale in its epilogue, fp32 row softmax, one batched P.V launch).
"""
from __future__ import annotations

import math

import numpy as np

from . import _cuda_ops as ops
from . import engine as E
from ._cuda_ops import GpuTensor

# Calls that took the fused kernel (for tests and launch accounting).
fused_calls = 0


def _check_rows(t: GpuTensor, name: str) -> tuple[int, int, int]:
    if t.ndim != 3:
        raise ValueError(f"{name} must be [batch, tokens, channels], got {t.shape}")
    return t.shape


def _run(B: int, H: int, N: int, S: int, D: int, q_ptr: int, ldq: int, q_bs: int, k_ptr: int,
         ldk: int, k_bs: int, v_ptr: int, ldv: int, v_bs: int, out: GpuTensor, scale: float,
         dtype, dev: int) -> None:
    """softmax(scale q k^T) v for every (batch, head), heads packed in rows."""
    global fused_calls
    C = H * D
    code = E.dtype_code(dtype)
    with E.on_device(dev):
        if D == 64 and code != E.DT_F32:
            E.attention(B, H, N, S, q_ptr, ldq, q_bs, k_ptr, ldk, k_bs, v_ptr, ldv, v_bs, out.ptr,
                        C, N * C, scale, dtype=code, head_dim=D, device=dev)
            fused_calls += 1
            return
        scores = ops._alloc((B, H, N, S), np.float32, dev)
        probs = ops._alloc((B, H, N, S), dtype, dev)
        # batch index: head (count0, stride D), sample (count1)
        bt = E.make_batch(H, B, a=(D, q_bs), b=(D, k_bs), c=(N * S, H * N * S))
        E.gemm(N, S, D, q_ptr, ldq, 0, k_ptr, ldk, 1, scores.ptr, S, code, E.DT_F32,
               epi=E.make_epilogue(alpha=scale), batch=bt, device=dev)
        E.softmax_rows(scores.ptr, E.DT_F32, S, probs.ptr, code, S, B * H * N, S, 1.0, device=dev)
        bt2 = E.make_batch(H, B, a=(N * S, H * N * S), b=(D, v_bs), c=(D, N * C))
        E.gemm(N, D, S, probs.ptr, S, 0, v_ptr, ldv, 0, out.ptr, C, code, code, batch=bt2,
               device=dev)


def self_attention(qkv: GpuTensor, heads: int, scale: float | None = None) -> GpuTensor:
    """Multi-head self-attention over a fused ``[B, N, 3C]`` QKV projection
    (q, k, v in column blocks ``[0, C)``, ``[C, 2C)``, ``[2C, 3C)``, head h at
    ``h*D`` inside each block); returns ``[B, N, C]``."""
    B, N, C3 = _check_rows(qkv, "qkv")
    if C3 % 3 or (C3 // 3) % heads:
        raise ValueError(f"qkv width {C3} does not split into 3 x {heads} heads")
    C = C3 // 3
    D = C // heads
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    out = ops._alloc((B, N, C), qkv.dtype, qkv.device_id)
    es = np.dtype(qkv.dtype).itemsize
    base = qkv.ptr
    _run(B, heads, N, N, D, base, C3, N * C3, base + C * es, C3, N * C3, base + 2 * C * es, C3,
         N * C3, out, scale, qkv.dtype, qkv.device_id)
    return out


def cross_attention(q: GpuTensor, k: GpuTensor, v: GpuTensor, heads: int,
                    scale: float | None = None) -> GpuTensor:
    """Multi-head attention of ``q [B, N, C]`` over ``k, v [B, S, C]`` (S may
    differ from N, e.g. text context); returns ``[B, N, C]``."""
    B, N, C = _check_rows(q, "q")
    Bk, S, Ck = _check_rows(k, "k")
    if k.shape != v.shape or Bk != B or Ck != C:
        raise ValueError(f"attention shapes: q {q.shape}, k {k.shape}, v {v.shape}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("q, k and v must share a dtype")
    if len({q.device_id, k.device_id, v.device_id}) != 1:
        raise ValueError("q, k and v must be on one device")
    if C % heads:
        raise ValueError(f"{C} channels do not split into {heads} heads")
    D = C // heads
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    out = ops._alloc((B, N, C), q.dtype, q.device_id)
    _run(B, heads, N, S, D, q.ptr, C, N * C, k.ptr, C, S * C, v.ptr, C, S * C, out, scale,
         q.dtype, q.device_id)
    return out
