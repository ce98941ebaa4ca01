"""NumPy restatement of the reference's CPU matmul path (TEST INFRASTRUCTURE).

Every function names the reference file:line it restates.  Paths are relative
to the reference project root (pictofeed/scaffolding).  On Linux the
reference's CPU path *is* NumPy/OpenBLAS: its Cython CPU extensions are built
only on macOS (``setup.py:306-352``), so ``_USE_CYTHON``/``_USE_MPS`` are
False and every branch below is the one the reference itself executes.

Reduced-precision inputs: the reference has no bf16 storage
(``dtype.py:31`` maps bfloat16 to float32), so the bf16/fp16 oracle is the
same fp32 NumPy code applied to inputs rounded to bf16/fp16 with
round-to-nearest-even ("an fp32 reference computed on identically rounded
inputs").

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import this module.
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "round_bf16", "round_f16", "round_to", "bf16_bits", "bf16_from_bits",
    "linear", "silu", "gelu_tanh", "activation", "linear_act",
    "matmul", "matmul_nt", "batched_matmul", "batched_matmul_nt",
    "softmax_rows", "sdpa", "layer_norm", "ada_layer_norm", "block_attention", "heads_split", "heads_merge",
    "dit_attention_chunked", "dit_layer", "dit_block_linears",
    "config1_inputs", "square_inputs", "skinny_inputs", "dit_weights",
    "rel_frobenius", "elementwise_rel_check", "abs_product", "ACT_NONE", "ACT_SILU",
    "ACT_GELU_TANH",
]

ACT_NONE = "none"
ACT_SILU = "silu"
ACT_GELU_TANH = "gelu_tanh"


# ───────────────────────── rounding helpers ──────────────────────────────

def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); return fp32.

    The reference cannot hold bf16 (``dtype.py:31``); this produces the
    "identically rounded inputs" the bf16 parity bar is defined on.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)).astype(np.uint32)
    nan = np.isnan(x)
    out = r.view(np.float32).copy()
    if nan.any():
        out[nan] = np.nan
    return out


def round_f16(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to fp16 (IEEE round-to-nearest-even); return fp32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round to the storage dtype named by ``dtype`` ('f32', 'bf16', 'f16')."""
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Raw bf16 bit patterns (uint16) of ``round_bf16(x)``."""
    return (round_bf16(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    """Widen raw bf16 bit patterns (uint16) to fp32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32)
            << np.uint32(16)).view(np.float32)


# ───────────────────────── elementwise ops ───────────────────────────────

def silu(z: np.ndarray) -> np.ndarray:
    """SiLU, as ``nn/functional.py:57-59``: ``sig = 1/(1+exp(-x)); x*sig``."""
    sig = 1.0 / (1.0 + np.exp(-z))
    return z * sig


def gelu_tanh(z: np.ndarray) -> np.ndarray:
    """GELU (tanh form), as ``nn/functional.py:79-82``."""
    return 0.5 * z * (1 + np.tanh(
        math.sqrt(2.0 / math.pi) * (z + 0.044715 * z ** 3)))


def activation(z: np.ndarray, act: str) -> np.ndarray:
    if act == ACT_NONE:
        return z
    if act == ACT_SILU:
        return silu(z)
    if act == ACT_GELU_TANH:
        return gelu_tanh(z)
    raise ValueError(f"unknown activation {act!r}")


# ───────────────────────── matmul family ─────────────────────────────────

def linear(x: np.ndarray, W: np.ndarray, b: np.ndarray | None = None) -> np.ndarray:
    """``nn.Linear`` CPU branch, ``nn/layers.py:129-131``: ``x @ W.T`` then ``+ b``.

    ``F.linear`` (``nn/functional.py:388-391``) is the same arithmetic via
    ``np.matmul(input, weight.T)``.
    """
    y = x @ W.T
    if b is not None:
        y = y + b
    return y


def linear_act(x, W, b=None, act: str = ACT_NONE):
    """``Linear`` followed by the separate activation call the reference's
    callers make (e.g. ``F.silu(lin(x))``: ``nn/layers.py:129-131`` then
    ``nn/functional.py:57-59``)."""
    return activation(linear(x, W, b), act)


def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """``sf.matmul`` CPU branch, ``tensor.py:1516-1519``: ``np.matmul``."""
    return np.matmul(a, b)


def matmul_nt(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """``sf.matmul_nt`` fallback, ``tensor.py:1538-1539``: ``matmul(a, b^T)``."""
    return np.matmul(a, np.swapaxes(b, -2, -1))


def batched_matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Batched NN product (``dev_batched_matmul`` semantics,
    ``_cuda_ops.pyx:1122-1149``; CPU arithmetic is ``np.matmul``)."""
    return np.matmul(a, b)


def batched_matmul_nt(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Batched NT product (``dev_batched_matmul_nt``, ``_cuda_ops.pyx:1152-1190``)."""
    return np.matmul(a, np.swapaxes(b, -2, -1))


def softmax_rows(x: np.ndarray) -> np.ndarray:
    """Row softmax, ``nn/functional.py:131-136``: max-subtract, exp, sum, divide."""
    x_max = x.max(axis=-1, keepdims=True)
    e = np.exp(x - x_max)
    e_sum = e.sum(axis=-1, keepdims=True)
    np.divide(e, e_sum, out=e)
    return e


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray,
         scale: float | None = None) -> np.ndarray:
    """``F.scaled_dot_product_attention`` CPU branch, ``nn/functional.py:323-357``
    (no mask, no dropout)."""
    d = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    k_T = np.swapaxes(k, -2, -1)
    scores = np.matmul(q, k_T)
    scores *= scale
    s_max = scores.max(axis=-1, keepdims=True)
    scores -= s_max
    np.exp(scores, out=scores)
    s_sum = scores.sum(axis=-1, keepdims=True)
    np.divide(scores, s_sum, out=scores)
    return np.matmul(scores, v)


def layer_norm(x: np.ndarray, gamma: np.ndarray | None = None, beta: np.ndarray | None = None,
               eps: float = 1e-5) -> np.ndarray:
    """``LayerNorm.forward`` NumPy path, ``nn/layers.py:512-521``: mean and
    (population) variance over the last axis, ``(x - mean) / sqrt(var + eps)``,
    then ``* weight + bias``."""
    x = np.asarray(x, np.float32)
    mean = np.mean(x, axis=-1, keepdims=True)
    var = np.var(x, axis=-1, keepdims=True)
    y = (x - mean) / np.sqrt(var + eps)
    if gamma is not None:
        y = y * gamma + beta
    return y.astype(np.float32)


def ada_layer_norm(x: np.ndarray, params: np.ndarray, gamma=None, beta=None,
                   eps: float = 1e-5) -> np.ndarray:
    """``AdaLayerNorm.forward`` (``diffusion/models.py:478-487``): LayerNorm,
    then ``h * (params[..., :C] + 1) + params[..., C:]`` with ``params`` the
    modulation linear's output for each sample.  ``x`` is ``(B, N, C)`` and
    ``params`` ``(B, 2C)``; each sample's row of params modulates all of its
    tokens (``params[:, None, :]``).  The reference broadcasts ``(B, C)``
    against ``(B, N, C)`` directly, which is the same for B = 1 (the case its
    golden vectors pin) and misaligned for B > 1."""
    h = layer_norm(x, gamma, beta, eps)
    C = h.shape[-1]
    p = np.asarray(params, np.float32)
    if p.ndim == 2 and h.ndim == 3:
        p = p[:, None, :]
    return (h * (p[..., :C] + 1.0) + p[..., C:]).astype(np.float32)


def block_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """``CrossAttentionBlock._attn`` (``diffusion/models.py:123-133``) on
    ``(B, H, N, D)`` / ``(B, H, S, D)`` arrays: einsum scores scaled by
    ``1/sqrt(D)``, max-subtracted exp, division by ``sum + 1e-9``, einsum
    with v."""
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D)
    scores = np.einsum('bhnd,bhmd->bhnm', q, k) * scale
    scores -= scores.max(axis=-1, keepdims=True)
    exp_s = np.exp(scores)
    attn = exp_s / (exp_s.sum(axis=-1, keepdims=True) + 1e-9)
    return np.einsum('bhnm,bhmd->bhnd', attn, v)


def heads_split(x: np.ndarray, heads: int) -> np.ndarray:
    """``[B, N, C] -> (B, H, N, D)``: the reference's
    ``reshape(B, N, H, D).transpose(0, 2, 1, 3)`` (``diffusion/models.py:148-151``,
    ``:167-169``; ``nn/video.py:364-371``)."""
    B, N, C = x.shape
    return x.reshape(B, N, heads, C // heads).transpose(0, 2, 1, 3).copy()


def heads_merge(x: np.ndarray) -> np.ndarray:
    """``(B, H, N, D) -> [B, N, C]``: ``transpose(0, 2, 1, 3).reshape(B, N, C)``
    (``diffusion/models.py:153``, ``:174``; ``nn/video.py:376``, ``:408``)."""
    B, H, N, D = x.shape
    return x.transpose(0, 2, 1, 3).reshape(B, N, H * D).copy()


def dit_attention_chunked(qkv: np.ndarray, batch: int, heads: int,
                          head_dim: int, chunk: int = 2048,
                          p_dtype: str = "f32", return_absprod: bool = False):
    """Attention over a fused QKV activation, in query chunks.

    ``qkv`` is ``[batch*tokens, 3*heads*head_dim]`` laid out as the reference
    ``DiTBlock`` slices it (``diffusion/models.py:546-549``: q, k, v are
    column blocks of ``to_qkv``'s output, head h at columns
    ``h*head_dim:(h+1)*head_dim``).  Per (b, h) and query chunk:
    ``S = (Q K^T) * scale``, row softmax in fp32, ``O = P V`` -- the SDPA
    sequence of ``nn/functional.py:314-320`` / ``:323-357``.  ``p_dtype``
    rounds P to the storage type the device path keeps it in.
    Returns ``[batch*tokens, heads*head_dim]`` (and, with ``return_absprod``,
    the matching ``|P| |V|`` error scale of the P.V products).
    """
    rows, width = qkv.shape
    C = heads * head_dim
    assert width == 3 * C and rows % batch == 0
    N = rows // batch
    scale = 1.0 / math.sqrt(head_dim)
    out = np.empty((rows, C), dtype=np.float32)
    absprod = np.empty((rows, C), dtype=np.float64) if return_absprod else None
    for b in range(batch):
        blk = qkv[b * N:(b + 1) * N]
        for h in range(heads):
            q = blk[:, h * head_dim:(h + 1) * head_dim]
            k = blk[:, C + h * head_dim:C + (h + 1) * head_dim]
            v = blk[:, 2 * C + h * head_dim:2 * C + (h + 1) * head_dim]
            for c0 in range(0, N, chunk):
                c1 = min(c0 + chunk, N)
                s = (q[c0:c1] @ k.T).astype(np.float32)
                s *= np.float32(scale)
                p = softmax_rows(s)
                p = round_to(p, p_dtype)
                out[b * N + c0:b * N + c1, h * head_dim:(h + 1) * head_dim] = p @ v
                if absprod is not None:
                    absprod[b * N + c0:b * N + c1, h * head_dim:(h + 1) * head_dim] = \
                        abs_product(p, v.T)
    return (out, absprod) if return_absprod else out


def _bf16_neighbours(p: np.ndarray, p_dtype: str):
    """The two representable ``p_dtype`` values around ``p`` (p >= 0)."""
    if p_dtype == "bf16":
        bits = np.asarray(p, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)
        lo = bits.view(np.float32)
        hi = (bits + np.uint32(0x10000)).view(np.float32)
        return lo, hi
    if p_dtype == "f16":
        lo = np.asarray(p, np.float32).astype(np.float16)
        lo = np.where(lo.astype(np.float32) > p, np.nextafter(lo, np.float16(0)), lo)
        hi = np.nextafter(lo, np.float16(np.inf))
        return lo.astype(np.float32), hi.astype(np.float32)
    return p, p


def flash_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
                    block: int = 128, p_dtype: str = "bf16", flip_tol: float = 2.0 ** -12,
                    return_allowance: bool = False, integer_base: bool = False):
    """Attention ``softmax(scale * q k^T) v`` for one head, restated in the
    online (blockwise) form the fused device kernel computes, so that the
    P.V operand is rounded where the device rounds it.

    The result equals ``sdpa`` (``nn/functional.py:323-357``) up to that
    rounding.  Keys are taken in blocks of ``block``; with the running row
    maximum ``m`` kept in the log2 domain (``c = scale * log2 e``):
    ``m' = max(m, c * max_j s_ij)``, ``alpha = 2^(m - m')``,
    ``p_ij = 2^(c s_ij - m')`` (fp32), ``l = alpha l + sum_j p_ij``,
    ``o = alpha o + round(p) v_block``; finally ``o / l``.  ``p_dtype`` is the
    storage type of the P operand (the device's 16-bit MMA input).

    ``integer_base`` rounds each row's base up to an integer
    (``m' = max(m, ceil(c * max_j s_ij))``).  With integer bases the rounding
    of ``2^(c s - m)`` does not depend on which base is used (a change of base
    scales every p by an exact power of two), so this also stands for the
    device kernel, which sets a row's base from its first block and raises
    it (to ``ceil(c * block max)``) only when a block's ``p`` under the
    current base sum to ``2^8`` or more.

    With ``return_allowance`` it also returns, per output element, the
    change that rounding p the other way could cause for every p lying
    within ``flip_tol`` (relative) of a rounding midpoint: scores computed
    in a different summation order shift such p across the midpoint, so no
    restatement can fix which neighbour the device picks.
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    n = q.shape[0]
    c = np.float32(scale * 1.4426950408889634)
    m = np.full(n, -np.inf, np.float32)
    l = np.zeros(n, np.float32)
    o = np.zeros((n, v.shape[1]), np.float32)
    a = np.zeros((n, v.shape[1]), np.float64)
    for j0 in range(0, k.shape[0], block):
        s = (q @ k[j0:j0 + block].T).astype(np.float32)
        cand = s.max(axis=1) * c
        if integer_base:
            cand = np.ceil(cand)
        m_new = np.maximum(m, cand)
        alpha = np.exp2(m - m_new).astype(np.float32)
        p = np.exp2(s * c - m_new[:, None]).astype(np.float32)
        l = l * alpha + p.sum(axis=1, dtype=np.float32)
        o = o * alpha[:, None] + round_to(p, p_dtype) @ v[j0:j0 + block]
        if return_allowance:
            lo, hi = _bf16_neighbours(p, p_dtype)
            mid = 0.5 * (lo.astype(np.float64) + hi)
            near = np.abs(p - mid) <= flip_tol * np.maximum(p, 1e-30)
            flip = np.where(near, hi.astype(np.float64) - lo, 0.0)
            a = a * alpha[:, None] + flip @ np.abs(v[j0:j0 + block].astype(np.float64))
        m = m_new
    out = (o / l[:, None]).astype(np.float32)
    if return_allowance:
        return out, a / l[:, None]
    return out


def dit_layer(x: np.ndarray, w: dict, batch: int, heads: int, head_dim: int,
              chunk: int = 2048, dtype: str = "bf16") -> np.ndarray:
    """One DiT layer as the B200 engine runs it (no adaLN / LayerNorm).

    Follows ``DiTBlock.forward`` (``diffusion/models.py:538-590``) minus the
    adaptive norms: ``qkv = to_qkv(x)`` (no bias, ``:508``), attention,
    ``x = x + self_out(attn)``, ``x = x + ff_down(gelu(ff_up(x)))``.  The FFN
    activation is GELU-tanh, as the benchmark configuration specifies (the
    reference block's own FFN uses SiLU, ``:522-527``).  Intermediate
    activations are rounded to ``dtype`` at the points where the device path
    stores them.
    """
    r = lambda a: round_to(a, dtype)  # noqa: E731
    qkv = r(linear(x, w["qkv_w"]))
    attn = r(dit_attention_chunked(qkv, batch, heads, head_dim, chunk, p_dtype=dtype))
    h = r(linear(attn, w["out_w"], w["out_b"]) + x)
    f = r(gelu_tanh(linear(h, w["up_w"], w["up_b"])))
    return r(linear(f, w["down_w"], w["down_b"]) + h)


def dit_block_linears(x: np.ndarray, w: dict, dtype: str = "bf16") -> np.ndarray:
    """The four DiT block linears as the benchmark's config-4 step chains them
    (``diffusion/models.py:508-527`` shapes; bias, GELU-tanh and residual as
    the device epilogues apply them):
    ``qkv = x Wqkv^T``; ``h = qkv[:, :C] Wo^T + bo + x``;
    ``f = gelu(h W1^T + b1)``; ``y = f W2^T + b2 + h``.  Intermediates are
    rounded to ``dtype`` where the device stores them."""
    C = w["out_w"].shape[0]
    r = lambda a: round_to(a, dtype)  # noqa: E731
    qkv = r(linear(x, w["qkv_w"]))
    h = r(linear(qkv[:, :C], w["out_w"], w["out_b"]) + x)
    f = r(gelu_tanh(linear(h, w["up_w"], w["up_b"])))
    return r(linear(f, w["down_w"], w["down_b"]) + h)


# ───────────────────────── seeded inputs ─────────────────────────────────
# Draw order and distributions follow the benchmark configurations: one
# ``np.random.default_rng(seed)`` stream, x then W then b, drawn in fp32 and
# then rounded to the storage dtype.

def config1_inputs(seed: int = 0, M: int = 512, K: int = 1024, N: int = 4096):
    """Config 1: x ~ N(0,1); W, b ~ U(-1/sqrt(K), 1/sqrt(K)) -- the
    ``nn.Linear`` Kaiming-uniform bound of ``nn/layers.py:66-74``."""
    rng = np.random.default_rng(seed)
    k = 1.0 / math.sqrt(K)
    x = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.uniform(-k, k, (N, K)).astype(np.float32)
    b = rng.uniform(-k, k, (N,)).astype(np.float32)
    return x, W, b


def square_inputs(n: int, dtype: str = "bf16", seed: int = 0, m: int | None = None,
                  k: int | None = None):
    """Config 2: A [M,K], B [N,K] (``nn.Linear`` weight layout), ~N(0,1)/sqrt(K)."""
    m = n if m is None else m
    k = n if k is None else k
    rng = np.random.default_rng(seed)
    s = np.float32(1.0 / math.sqrt(k))
    A = rng.standard_normal((m, k), dtype=np.float32) * s
    B = rng.standard_normal((n, k), dtype=np.float32) * s
    return round_to(A, dtype), round_to(B, dtype)


def skinny_inputs(M: int, N: int, K: int = 4096, seed: int = 0, dtype: str = "bf16"):
    """Config 3: x ~ N(0,1) [M,K], W ~ N(0,0.02) [N,K], b ~ N(0,0.02) [N]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    b = rng.standard_normal((N,), dtype=np.float32) * np.float32(0.02)
    return round_to(x, dtype), round_to(W, dtype), round_to(b, dtype)


def dit_weights(hidden: int = 1920, seed: int = 1, dtype: str = "bf16",
                zero_bias: bool = True) -> dict:
    """Config 4/5 block weights: W ~ N(0, 0.02), biases 0 (or N(0,0.02))."""
    rng = np.random.default_rng(seed)
    C = hidden

    def w(n, k):
        return round_to(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02), dtype)

    def b(n):
        if zero_bias:
            return np.zeros((n,), np.float32)
        return round_to(rng.standard_normal((n,), dtype=np.float32) * np.float32(0.02), dtype)

    return {
        "qkv_w": w(3 * C, C),
        "out_w": w(C, C), "out_b": b(C),
        "up_w": w(4 * C, C), "up_b": b(4 * C),
        "down_w": w(C, 4 * C), "down_b": b(C),
    }


# ───────────────────────── tolerance checks ──────────────────────────────

def rel_frobenius(out: np.ndarray, ref: np.ndarray) -> float:
    """``||out - ref||_F / ||ref||_F`` in float64 (the fp32 parity bar, 1e-5)."""
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(r)
    num = np.linalg.norm(o - r)
    return float(num / den) if den > 0 else float(num)


def abs_product(a: np.ndarray, b_t: np.ndarray) -> np.ndarray:
    """``|a| @ |b_t|^T`` in float64: the sum of absolute products behind each
    output of ``a @ b_t^T`` (the scale of its rounding error)."""
    return np.abs(np.asarray(a, np.float64)) @ np.abs(np.asarray(b_t, np.float64)).T


def elementwise_rel_check(out: np.ndarray, ref: np.ndarray, rtol: float = 1e-2,
                          tau: float = 1e-2, absprod: np.ndarray | None = None,
                          kappa: float = 1e-2, allowance: np.ndarray | None = None):
    """Per-element relative check for bf16/fp16 outputs (bar: 1e-2).

    An element passes when ``|out - ref| <= rtol * max(|ref|, tau * rms(ref row),
    kappa * absprod)``.  The floors only matter where the exact value cancels
    to nearly zero, where a relative error is undefined in practice:
    ``tau * rms(row)`` (1 % of the row's RMS) and, when ``absprod`` -- the
    sum of absolute products ``(|A| |B|)_ij`` behind each output -- is given,
    ``kappa * absprod``.  The second is the standard error scale of a dot
    product; with rtol = kappa = 1e-2 it allows an error of 1e-4 of the
    absolute sum, the accumulation precision of the tensor cores' fp32
    accumulators (measured ~2^-15 of the absolute sum on cancelling sums).  Returns ``(ok, stats)`` with the worst pure
    relative error, the worst error against the floored denominator, and the
    number of elements that needed the floor.  ``allowance`` (optional) is an
    absolute per-element slack added to the bar: the rounding decisions the
    oracle cannot reproduce (``flash_attention``'s flip allowance).
    """
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    if r.ndim == 0:
        r = r.reshape(1)
        o = o.reshape(1)
    rr = r.reshape(-1, r.shape[-1]) if r.ndim > 1 else r.reshape(1, -1)
    oo = o.reshape(rr.shape)
    rms = np.sqrt(np.mean(rr * rr, axis=1, keepdims=True))
    absr = np.abs(rr)
    den = np.maximum(absr, tau * rms)
    if absprod is not None:
        den = np.maximum(den, kappa * np.asarray(absprod, np.float64).reshape(rr.shape))
    den = np.where(den > 0, den, 1.0)
    err = np.abs(oo - rr)
    if allowance is not None:
        # an allowance of A widens the bar rtol*den by A: scale it into err
        err = np.maximum(err - np.asarray(allowance, np.float64).reshape(rr.shape), 0.0)
    floored = err / den
    finite = np.isfinite(oo).all()
    pure = err / np.where(absr > 0, absr, np.inf)
    needed_floor = int(np.count_nonzero((pure > rtol) & (floored <= rtol)))
    worst = float(floored.max()) if floored.size else 0.0
    # Which floor each passing element relied on (first that suffices, in
    # the order row RMS, |A||B|, rounding-flip allowance).
    raw = np.abs(oo - rr)
    ok_final = floored <= rtol
    ok_pure = raw <= rtol * absr
    ok_row = raw <= rtol * np.maximum(absr, tau * rms)
    ok_abs = raw <= rtol * den
    stats = {
        "max_rel_floored": worst,
        "max_rel_pure": float(np.nanmax(pure)) if pure.size else 0.0,
        "n_needed_floor": needed_floor,
        "n_row_floor": int(np.count_nonzero(ok_final & ~ok_pure & ok_row)),
        "n_absprod_floor": int(np.count_nonzero(ok_final & ~ok_row & ok_abs)),
        "n_allowance": int(np.count_nonzero(ok_final & ~ok_abs)),
        "n": int(rr.size),
        "tau": tau,
        "rtol": rtol,
        "finite": bool(finite),
    }
    return bool(finite and worst <= rtol), stats
