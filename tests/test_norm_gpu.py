"""LayerNorm and the DiT blocks' adaptive LayerNorm on the device (-m gpu):
sf_layernorm_modulate behind dev_layer_norm / dev_ada_layer_norm /
nn.LayerNorm / nn.AdaLayerNorm, against the reference's own outputs
(golden, B = 1) and the oracle (nn/layers.py:512-521,
diffusion/models.py:478-487) on every kernel path: register-resident rows
(16-byte vectors), the generic loop (odd widths, strided rows), fp32 and
16-bit in and out, per-sample modulation for B > 1."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import (assert_close_16bit, assert_close_fp32, device_error, np_dtype,
                            to_device, to_host32)

pytestmark = pytest.mark.gpu


def test_layer_norm_and_adaln_golden(gpu, ops, golden):
    x, g, b = golden["adaln_x"], golden["adaln_gamma"], golden["adaln_beta"]
    gx, gg, gb = (ops.gputensor_from_numpy(t) for t in (x, g, b))
    ln = ops.gputensor_to_numpy(ops.dev_layer_norm(gx, gg, gb, 1e-5))
    assert_close_fp32(ln, golden["adaln_ln"], "LayerNorm vs reference", tol=1e-6)
    gp = ops.gputensor_from_numpy(golden["adaln_params"])
    y = ops.gputensor_to_numpy(ops.dev_ada_layer_norm(gx, gp, gg, gb, 1e-5))
    assert_close_fp32(y, golden["adaln_y"], "AdaLayerNorm (given params) vs reference", tol=1e-6)


def test_nn_ada_layer_norm_module_golden(gpu, ops, golden):
    """nn.AdaLayerNorm end to end: the modulation linear (fp32, 3xTF32 GEMM)
    then the fused norm + modulation, with the reference module's weights."""
    from scaffolding_b200 import nn
    m = nn.AdaLayerNorm(64, 32, device=0)
    m.norm.weight = ops.gputensor_from_numpy(golden["adaln_gamma"])
    m.norm.bias = ops.gputensor_from_numpy(golden["adaln_beta"])
    m.linear.weight = ops.gputensor_from_numpy(golden["adaln_w"])
    m.linear.bias = ops.gputensor_from_numpy(golden["adaln_b"])
    y = ops.gputensor_to_numpy(m(ops.gputensor_from_numpy(golden["adaln_x"]),
                                 ops.gputensor_from_numpy(golden["adaln_cond"])))
    assert_close_fp32(y, golden["adaln_y"], "nn.AdaLayerNorm vs reference")


@pytest.mark.parametrize("dt_in,dt_out", [("bf16", "bf16"), ("f16", "f16"), ("f32", "f32"),
                                          ("bf16", "f32")])
@pytest.mark.parametrize("C", [64, 1920, 3000, 100, 8200])
def test_adaln_per_sample_modulation(gpu, ops, dt_in, dt_out, C):
    """B = 3 samples of N = 37 tokens: each sample's scale / shift applies to
    its own tokens only.  C = 64 / 1920 / 3000 take the register-resident
    kernel (16-bit in and out), 100 and 8200 (and mixed dtypes) the generic
    loop."""
    rng = np.random.default_rng(C)
    B, N = 3, 37
    gx, x = to_device(ops, rng.standard_normal((B, N, C), dtype=np.float32) * np.float32(1.5) +
                      np.float32(0.3), dt_in)
    params = rng.standard_normal((B, 2 * C), dtype=np.float32) * np.float32(0.2)
    gp = ops.gputensor_from_numpy(params)
    gamma = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    gg, gb = ops.gputensor_from_numpy(gamma), ops.gputensor_from_numpy(beta)
    y = to_host32(ops, ops.dev_ada_layer_norm(gx, gp, gg, gb, 1e-5, out_dtype=np_dtype(dt_out)))
    ref = O.ada_layer_norm(x, params, gamma, beta)
    if dt_out == "f32":
        assert_close_fp32(y, ref, f"adaLN {dt_in}->{dt_out} C={C}", tol=2e-6)
    else:
        assert_close_16bit(y.reshape(-1, C), ref.reshape(-1, C), f"adaLN {dt_in}->{dt_out} C={C}")
    assert device_error(0) == 0


def test_layer_norm_dit_shape_and_no_affine(gpu, ops):
    """The DiT activation shape (35552 x 1920, bf16) on sampled rows, and a
    LayerNorm without the affine parameters."""
    from scaffolding_b200 import nn
    M, C = 35552, 1920
    gx, x = to_device(ops, np.random.default_rng(3).standard_normal((M, C), dtype=np.float32), "bf16")
    ln = nn.LayerNorm(C, elementwise_affine=False, device=0)
    y = to_host32(ops, ln(gx))
    rows = np.random.default_rng(4).choice(M, 64, replace=False)
    assert_close_16bit(y[rows], O.layer_norm(x[rows]), "LayerNorm 35552x1920 bf16")
    assert np.isfinite(y).all()
    assert device_error(0) == 0
