"""Pin the CPU oracle against golden vectors produced by the reference's own
code (tests/golden/make_golden.py).  CPU only."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))


def _same_blas():
    meta = json.load(open(os.path.join(HERE, "golden", "golden_meta.json")))
    try:
        blas = np.show_config(mode="dicts")["Build Dependencies"]["blas"]
    except Exception:
        return False
    return (meta["numpy"] == np.__version__ and meta["blas"] and
            meta["blas"].get("version") == blas.get("version"))


def _match(out, ref, exact):
    if exact:
        np.testing.assert_array_equal(out, ref)
    else:
        assert O.rel_frobenius(out, ref) < 1e-6


def test_config1_linear_silu_matches_reference(golden):
    x, W, b = O.config1_inputs(seed=0)
    y = O.linear_act(x, W, b, O.ACT_SILU)
    assert y.dtype == np.float32 and y.shape == tuple(golden["cfg1_y_shape"])
    _match(y[::8], golden["cfg1_y_rows"], _same_blas())
    np.testing.assert_allclose(y.astype(np.float64).sum(), float(golden["cfg1_y_sum"]), rtol=1e-6)
    np.testing.assert_allclose((y.astype(np.float64) ** 2).sum(), float(golden["cfg1_y_sumsq"]),
                               rtol=1e-6)


@pytest.mark.parametrize("tag", ["mm_a", "mm_b", "mm_c"])
def test_matmul_2d(golden, tag):
    exact = _same_blas()
    _match(O.matmul(golden[f"{tag}_a"], golden[f"{tag}_b"]), golden[f"{tag}_nn"], exact)
    _match(O.matmul_nt(golden[f"{tag}_a"], golden[f"{tag}_bt"]), golden[f"{tag}_nt"], exact)


def test_batched(golden):
    exact = _same_blas()
    _match(O.batched_matmul(golden["bmm_a"], golden["bmm_b"]), golden["bmm_nn"], exact)
    _match(O.batched_matmul_nt(golden["bmm_a"], golden["bmm_bt"]), golden["bmm_nt"], exact)


@pytest.mark.parametrize("tag,act", [("lin_silu_f32", "silu"), ("lin_gelu_f32", "gelu_tanh"),
                                     ("lin_none_f32", "none"), ("lin_gelu_bf16", "gelu_tanh"),
                                     ("lin_silu_f16", "silu")])
def test_linear_act(golden, tag, act):
    y = O.linear_act(golden[f"{tag}_x"], golden[f"{tag}_w"], golden[f"{tag}_b"], act)
    _match(y, golden[f"{tag}_y"], _same_blas())
    _match(golden[f"{tag}_yf"], golden[f"{tag}_y"], _same_blas())


def test_activations_bit_exact(golden):
    z = golden["act_z"]
    np.testing.assert_array_equal(O.silu(z), golden["act_silu"])
    np.testing.assert_array_equal(O.gelu_tanh(z), golden["act_gelu"])


@pytest.mark.parametrize("tag", ["sm1", "sm2"])
def test_softmax_bit_exact(golden, tag):
    np.testing.assert_array_equal(O.softmax_rows(golden[f"{tag}_x"]), golden[f"{tag}_y"])


def test_sdpa(golden):
    exact = _same_blas()
    _match(O.sdpa(golden["sdpa_q"], golden["sdpa_k"], golden["sdpa_v"]), golden["sdpa_o"], exact)
    _match(O.sdpa(golden["sdpa8_q"], golden["sdpa8_k"], golden["sdpa8_v"], scale=0.125),
           golden["sdpa8_o"], exact)


def test_dit_chunked_attention_equals_sdpa():
    rng = np.random.default_rng(3)
    B, N, H, D = 2, 70, 3, 16
    qkv = rng.standard_normal((B * N, 3 * H * D), dtype=np.float32)
    out = O.dit_attention_chunked(qkv, B, H, D, chunk=32)
    C = H * D
    for b in range(B):
        blk = qkv[b * N:(b + 1) * N]
        for h in range(H):
            q, k, v = (blk[:, s * C + h * D:s * C + (h + 1) * D] for s in range(3))
            ref = O.sdpa(q[None], k[None], v[None])[0]
            np.testing.assert_allclose(out[b * N:(b + 1) * N, h * D:(h + 1) * D], ref,
                                       rtol=1e-5, atol=1e-6)


def test_bf16_rounding_rne():
    # ties to even: 1 + 2^-8 lies halfway between bf16 neighbours 1 and 1 + 2^-7
    x = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, -2.5, 0.0, np.inf, 3.0e38],
                 dtype=np.float32)
    r = O.round_bf16(x)
    assert r[0] == 1.0 and r[1] == 1.0 + 2.0 ** -6
    assert r[2] == -2.5 and r[3] == 0.0 and np.isinf(r[4])
    bits = O.bf16_bits(x)
    np.testing.assert_array_equal(O.bf16_from_bits(bits), r)
    try:
        import ml_dtypes
        np.testing.assert_array_equal(
            x.astype(ml_dtypes.bfloat16).astype(np.float32)[:5], r[:5])
    except ImportError:
        pass


def test_elementwise_check_floor():
    ref = np.array([[1.0, -1.0, 1e-6, 2.0]], dtype=np.float32)
    out = ref + np.array([[0.005, 0.0, 1e-4, -0.01]], dtype=np.float32)
    ok, st = O.elementwise_rel_check(out, ref, rtol=1e-2, tau=1e-2)
    assert ok and st["n_needed_floor"] == 1
    ok, _ = O.elementwise_rel_check(ref * 1.02, ref)
    assert not ok


def test_elementwise_check_absprod_floor():
    # an output that cancels to ~0 is judged against the size of its terms
    a = np.array([[1.0, -1.0, 1e-3]], np.float32)
    b = np.array([[1.0, 1.0, 1.0]], np.float32)
    ref = a @ b.T
    ap = O.abs_product(a, b)
    assert abs(ap[0, 0] - 2.001) < 1e-6
    out = ref + np.float32(1e-4)
    assert not O.elementwise_rel_check(out, ref)[0]
    assert O.elementwise_rel_check(out, ref, absprod=ap)[0]


def test_seeded_inputs_deterministic():
    a1, b1 = O.square_inputs(64, "bf16", seed=5)
    a2, b2 = O.square_inputs(64, "bf16", seed=5)
    np.testing.assert_array_equal(a1, a2)
    np.testing.assert_array_equal(b1, b2)
    np.testing.assert_array_equal(O.round_bf16(a1), a1)


def test_flash_attention_matches_sdpa():
    """The blockwise (online-softmax) restatement equals the reference SDPA
    when P is not rounded, for ragged key counts and large logits."""
    rng = np.random.default_rng(9)
    for n_q, n_k in [(5, 7), (130, 300), (64, 128)]:
        q = rng.standard_normal((n_q, 64), dtype=np.float32) * np.float32(3)
        k = rng.standard_normal((n_k, 64), dtype=np.float32) * np.float32(3)
        v = rng.standard_normal((n_k, 64), dtype=np.float32)
        ref = O.sdpa(q[None], k[None], v[None], scale=0.125)[0]
        np.testing.assert_allclose(O.flash_attention(q, k, v, 0.125, p_dtype="f32"), ref,
                                   rtol=2e-5, atol=2e-6)


def test_flash_allowance_covers_flips_only():
    """The flip allowance is zero when no p lies near a rounding midpoint
    and otherwise bounded by the 16-bit spacing of the p that may flip."""
    rng = np.random.default_rng(2)
    q = rng.standard_normal((40, 64), dtype=np.float32)
    k = rng.standard_normal((200, 64), dtype=np.float32)
    v = rng.standard_normal((200, 64), dtype=np.float32)
    _, a0 = O.flash_attention(q, k, v, 0.125, return_allowance=True, flip_tol=0.0)
    assert np.count_nonzero(a0) <= a0.size // 100  # only exact midpoints
    ref, a = O.flash_attention(q, k, v, 0.125, return_allowance=True)
    p = O.softmax_rows((q @ k.T * np.float32(0.125)).astype(np.float32))
    assert (a <= 2.0 ** -7 * O.abs_product(p, v.T) + 1e-12).all()
    # a change larger than the allowance still fails the check
    bad = ref + np.float32(0.05)
    assert not O.elementwise_rel_check(bad, ref, allowance=a)[0]


def test_layer_norm_and_adaln_match_reference_golden(golden):
    """LayerNorm / AdaLayerNorm restatements against the reference's own
    modules (B = 1, where its broadcast of the modulation is per sample)."""
    x, g, b = golden["adaln_x"], golden["adaln_gamma"], golden["adaln_beta"]
    np.testing.assert_array_equal(O.layer_norm(x, g, b), golden["adaln_ln"])
    params = O.linear(golden["adaln_cond"], golden["adaln_w"], golden["adaln_b"])
    np.testing.assert_array_equal(params, golden["adaln_params"])
    np.testing.assert_array_equal(O.ada_layer_norm(x, params, g, b), golden["adaln_y"])


def test_block_attention_matches_reference_golden(golden):
    o = O.block_attention(golden["battn_q"], golden["battn_k"], golden["battn_v"])
    np.testing.assert_array_equal(o, golden["battn_o"])
