"""Attention of the DiT-family blocks on the device, and the fused kernel
behind the SDPA drop-in (-m gpu).

* ``functional.scaled_dot_product_attention`` (the GPU path of
  ``nn/functional.py:310-321``) dispatches bf16/fp16 head_dim-64 calls to
  the fused kernel (one launch; asserted through the dispatch counter) and
  everything else to the unfused chain.
* ``attention.self_attention`` / ``cross_attention`` replace the host
  attention of ``CrossAttentionBlock._attn`` (``diffusion/models.py:123-133``)
  and ``SpatialTemporalAttention`` (``nn/video.py:345-432``): checked against
  the oracle's restatement of ``_attn`` on the reference's head split.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import (assert_close_16bit, assert_close_fp32, attn_oracle_opts, device_error,
                            np_dtype, to_device, to_host32)

pytestmark = pytest.mark.gpu


def _check_fused_heads(out, q, k, v, scale, dt, what):
    """Per (batch, head) against the oracle restating the fused kernel's
    blockwise softmax, with the rounding-flip allowance and |P||V| floor."""
    for idx in np.ndindex(*q.shape[:-2]):
        qi, ki, vi = q[idx], k[idx], v[idx]
        ref, allow = O.flash_attention(qi, ki, vi, scale, p_dtype=dt, return_allowance=True,
                                       **attn_oracle_opts())
        p = O.softmax_rows((qi @ ki.T * np.float32(scale)).astype(np.float32))
        assert_close_16bit(out[idx], ref, f"{what} {idx}", absprod=O.abs_product(p, vi.T),
                           allowance=allow)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("lead,M,S", [((2, 3), 300, 300), ((4,), 77, 1000), ((1,), 129, 64)])
def test_sdpa_dispatches_fused_kernel(gpu, ops, dt, lead, M, S):
    from scaffolding_b200 import nn
    rng = np.random.default_rng(M + S)
    gq, q = to_device(ops, rng.standard_normal(lead + (M, 64), dtype=np.float32), dt)
    gk, k = to_device(ops, rng.standard_normal(lead + (S, 64), dtype=np.float32), dt)
    gv, v = to_device(ops, rng.standard_normal(lead + (S, 64), dtype=np.float32), dt)
    before = nn.sdpa_fused_calls
    out = to_host32(ops, nn.functional.scaled_dot_product_attention(gq, gk, gv))
    assert nn.sdpa_fused_calls == before + 1, "16-bit head_dim-64 SDPA must take the fused kernel"
    assert out.shape == lead + (M, 64)
    _check_fused_heads(out, q, k, v, 0.125, dt, f"sdpa {dt}")
    # and the reference's own (fp32, exact softmax) SDPA on the rounded inputs
    assert O.rel_frobenius(out, O.sdpa(q, k, v)) < 1e-2
    assert device_error(0) == 0


def test_sdpa_unfused_path_other_head_dims(gpu, ops):
    """head_dim 32 (fp16) and fp32 inputs stay on the three-launch chain."""
    from scaffolding_b200 import nn
    rng = np.random.default_rng(9)
    before = nn.sdpa_fused_calls
    gq, q = to_device(ops, rng.standard_normal((2, 200, 32), dtype=np.float32), "f16")
    gk, k = to_device(ops, rng.standard_normal((2, 150, 32), dtype=np.float32), "f16")
    gv, v = to_device(ops, rng.standard_normal((2, 150, 32), dtype=np.float32), "f16")
    out = to_host32(ops, nn.functional.scaled_dot_product_attention(gq, gk, gv))
    s = O.batched_matmul_nt(q, k) * np.float32(1 / np.sqrt(32))
    ref = O.batched_matmul(O.round_f16(O.softmax_rows(s)), v)
    assert_close_16bit(out, ref, "sdpa f16 d32")
    q32, k32, v32 = (rng.standard_normal((3, 100, 64), dtype=np.float32) for _ in range(3))
    out32 = ops.gputensor_to_numpy(nn.functional.scaled_dot_product_attention(
        ops.gputensor_from_numpy(q32), ops.gputensor_from_numpy(k32), ops.gputensor_from_numpy(v32)))
    assert_close_fp32(out32, O.sdpa(q32, k32, v32), "sdpa fp32 d64")
    assert nn.sdpa_fused_calls == before


@pytest.mark.parametrize("dt,heads,D", [("bf16", 2, 64), ("f16", 3, 64), ("f32", 4, 16),
                                        ("f32", 2, 64)])
def test_self_attention_from_fused_qkv(gpu, ops, dt, heads, D):
    """Self-attention over a fused [B, N, 3C] to_qkv projection, heads read in
    place; against CrossAttentionBlock._attn on the reference's head split
    (diffusion/models.py:145-154, the same split as nn/video.py:363-376)."""
    from scaffolding_b200 import attention as A
    rng = np.random.default_rng(heads * D)
    B, N = 2, 300
    C = heads * D
    gqkv, qkv = to_device(ops, rng.standard_normal((B, N, 3 * C), dtype=np.float32), dt)
    before = A.fused_calls
    out = to_host32(ops, A.self_attention(gqkv, heads))
    assert out.shape == (B, N, C)
    q, k, v = (O.heads_split(qkv[:, :, i * C:(i + 1) * C], heads) for i in range(3))
    ref = O.heads_merge(O.block_attention(q, k, v))
    if dt == "f32":
        assert A.fused_calls == before
        assert_close_fp32(out, ref, f"self-attention fp32 D={D}")
    else:
        assert A.fused_calls == before + 1
        _check_fused_heads(O.heads_split(out, heads), q, k, v, 1 / np.sqrt(D), dt,
                           f"self-attention {dt}")
        assert O.rel_frobenius(out, ref) < 1e-2
    assert device_error(0) == 0


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_cross_attention_text_context(gpu, ops, dt):
    """Cross-attention of N = 300 latent tokens over S = 77 context tokens
    (CrossAttentionBlock, diffusion/models.py:161-176; SpatialTemporalAttention,
    nn/video.py:380-408)."""
    from scaffolding_b200 import attention as A
    rng = np.random.default_rng(77)
    B, N, S, heads = 2, 300, 77, 3
    C = heads * 64
    gq, q = to_device(ops, rng.standard_normal((B, N, C), dtype=np.float32), dt)
    gk, k = to_device(ops, rng.standard_normal((B, S, C), dtype=np.float32), dt)
    gv, v = to_device(ops, rng.standard_normal((B, S, C), dtype=np.float32), dt)
    out = to_host32(ops, A.cross_attention(gq, gk, gv, heads))
    qh, kh, vh = (O.heads_split(t, heads) for t in (q, k, v))
    ref = O.heads_merge(O.block_attention(qh, kh, vh))
    if dt == "f32":
        assert_close_fp32(out, ref, "cross-attention fp32")
    else:
        _check_fused_heads(O.heads_split(out, heads), qh, kh, vh, 0.125, dt, "cross-attention")
        assert O.rel_frobenius(out, ref) < 1e-2
    assert device_error(0) == 0
