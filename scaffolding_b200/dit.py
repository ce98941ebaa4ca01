"""DiT transformer-block workloads on the engine (benchmark configs 4 and 5).

Shapes follow the reference ``DiTBlock`` (``diffusion/models.py:490-590``):
fused ``to_qkv`` (dim -> 3*dim, no bias, ``:508``), ``self_out``
(dim -> dim, ``:509``), FFN dim -> 4*dim -> dim (``:522-527``; GELU-tanh as
the benchmark configuration specifies).  Adaptive LayerNorm modulation is not
part of the matmul path and is omitted.

Block linears (config 4), per token shard x[m, C]:
    qkv = x . Wqkv^T                              [m, 3C]
    h   = qkv[:, :C] . Wo^T + bo + x              [m, C]   (stands in for the
                                                           attention output)
    f   = gelu_tanh(h . W1^T + b1)                [m, 4C]
    y   = f . W2^T + b2 + h                       [m, C]
Bias, activation and residual are fused into the GEMM epilogues, so the
block is exactly four tcgen05 GEMM launches.
"""
from __future__ import annotations

import numpy as np

from . import _cuda_ops as ops
from . import engine as E
from ._lib import ACT_GELU_TANH, ACT_NONE, DT_BF16

HIDDEN = 1920
HEADS = 30
HEAD_DIM = 64
TOKENS = 17776
BATCH = 2


def block_flops(m: int, C: int = HIDDEN) -> float:
    """Algorithmic FLOPs of the four block linears on m token rows."""
    return 2.0 * m * C * (3 * C + C + 4 * C + 4 * C)


class DitLinears:
    """Device-resident bf16 weights of one block plus activation buffers for
    an m-row token shard."""

    def __init__(self, weights: dict, m: int, device: int):
        bf = E.bfloat16
        self.C = weights["out_w"].shape[0]
        self.m = m
        self.dev = device
        up = lambda a: ops.gputensor_from_numpy(np.ascontiguousarray(a).astype(bf), device)  # noqa: E731
        self.w = {k: up(v) for k, v in weights.items()}
        C = self.C
        self.qkv = ops._alloc((m, 3 * C), bf, device)
        self.h = ops._alloc((m, C), bf, device)
        self.f = ops._alloc((m, 4 * C), bf, device)
        self.y = ops._alloc((m, C), bf, device)

    def launches(self, x_ptr: int):
        """The four GEMM launches of one block as (name, kwargs) for engine.gemm."""
        C, m, w = self.C, self.m, self.w
        bf = DT_BF16
        return [
            ("qkv", dict(M=m, N=3 * C, K=C, A=x_ptr, lda=C, trans_a=0, B=w["qkv_w"].ptr, ldb=C,
                         trans_b=1, Cp=self.qkv.ptr, ldc=3 * C, in_dt=bf, out_dt=bf, epi=None)),
            ("out", dict(M=m, N=C, K=C, A=self.qkv.ptr, lda=3 * C, trans_a=0, B=w["out_w"].ptr,
                         ldb=C, trans_b=1, Cp=self.h.ptr, ldc=C, in_dt=bf, out_dt=bf,
                         epi=E.make_epilogue(bias_ptr=w["out_b"].ptr, bias_dt=bf, act=ACT_NONE,
                                             residual_ptr=x_ptr, residual_dt=bf, ldr=C))),
            ("up", dict(M=m, N=4 * C, K=C, A=self.h.ptr, lda=C, trans_a=0, B=w["up_w"].ptr,
                        ldb=C, trans_b=1, Cp=self.f.ptr, ldc=4 * C, in_dt=bf, out_dt=bf,
                        epi=E.make_epilogue(bias_ptr=w["up_b"].ptr, bias_dt=bf,
                                            act=ACT_GELU_TANH))),
            ("down", dict(M=m, N=C, K=4 * C, A=self.f.ptr, lda=4 * C, trans_a=0,
                          B=w["down_w"].ptr, ldb=4 * C, trans_b=1, Cp=self.y.ptr, ldc=C,
                          in_dt=bf, out_dt=bf,
                          epi=E.make_epilogue(bias_ptr=w["down_b"].ptr, bias_dt=bf, act=ACT_NONE,
                                              residual_ptr=self.h.ptr, residual_dt=bf, ldr=C))),
        ]

    def run(self, x_ptr: int, stream: int | None = None, timer=None) -> None:
        for name, kw in self.launches(x_ptr):
            if timer is not None:
                timer.start(name)
            E.gemm(kw["M"], kw["N"], kw["K"], kw["A"], kw["lda"], kw["trans_a"], kw["B"],
                   kw["ldb"], kw["trans_b"], kw["Cp"], kw["ldc"], kw["in_dt"], kw["out_dt"],
                   epi=kw["epi"], device=self.dev, stream=stream)
            if timer is not None:
                timer.stop(name)

