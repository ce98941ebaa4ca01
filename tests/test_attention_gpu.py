"""Row softmax and the attention products (QK^T, softmax, P.V) on the GPU
against the oracle (-m gpu)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import assert_close_16bit, assert_close_fp32, np_dtype, to_device, to_host32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cols", [1, 300, 1500, 4097, 17776, 40000])
@pytest.mark.parametrize("out_dt", ["f32", "bf16"])
def test_softmax_rows(gpu, ops, cols, out_dt):
    from scaffolding_b200 import engine as E
    rng = np.random.default_rng(cols)
    rows = 37
    x = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(6)
    gx = ops.gputensor_from_numpy(x)
    y = ops._alloc((rows, cols), np_dtype(out_dt), 0)
    E.softmax_rows(gx.ptr, 0, cols, y.ptr, E.dtype_code(np_dtype(out_dt)), cols, rows, cols, 0.125)
    ref = O.softmax_rows(x * np.float32(0.125))
    out = to_host32(ops, y)
    if out_dt == "f32":
        np.testing.assert_allclose(out, ref, rtol=2e-6, atol=1e-9)
        np.testing.assert_allclose(out.sum(axis=1), 1.0, rtol=1e-5)
    else:
        assert_close_16bit(out, ref, "softmax bf16")


def test_dev_softmax_golden(gpu, ops, golden):
    for tag in ("sm1", "sm2"):
        y = ops.gputensor_to_numpy(ops.dev_softmax(ops.gputensor_from_numpy(golden[f"{tag}_x"])))
        np.testing.assert_allclose(y, golden[f"{tag}_y"], rtol=2e-6, atol=1e-9)


def test_sdpa_fp32_golden(gpu, ops, golden):
    from scaffolding_b200.nn import functional as F
    q, k, v = (ops.gputensor_from_numpy(golden[f"sdpa_{s}"]) for s in "qkv")
    o = ops.gputensor_to_numpy(F.scaled_dot_product_attention(q, k, v))
    assert_close_fp32(o, golden["sdpa_o"], "sdpa fp32")


def _sdpa_p_rounded(q, k, v, scale):
    """Oracle SDPA with the probabilities rounded to bf16, the storage type
    the device keeps P in before the P.V product (its bf16 operand)."""
    s = O.batched_matmul_nt(q, k) * np.float32(scale)
    p = O.round_bf16(O.softmax_rows(s))
    return O.batched_matmul(p, v)


def test_sdpa_bf16_golden(gpu, ops, golden):
    """bf16 SDPA.  Per-element bar (1e-2) against the oracle on identically
    rounded GEMM operands (Q, K, V and the stored bf16 P); against the
    reference's fp32-P output the bf16 rounding of P is visible on outputs
    that cancel to ~0, so that comparison uses the aggregate bar."""
    from scaffolding_b200.nn import functional as F
    bf = np_dtype("bf16")
    qh, kh, vh = (golden[f"sdpa8_{s}"] for s in "qkv")
    q, k, v = (ops.gputensor_from_numpy(t.astype(bf)) for t in (qh, kh, vh))
    o = to_host32(ops, F.scaled_dot_product_attention(q, k, v, scale=0.125))
    assert_close_16bit(o, _sdpa_p_rounded(qh, kh, vh, 0.125), "sdpa bf16 vs P-rounded oracle")
    assert O.rel_frobenius(o, golden["sdpa8_o"]) < 1e-2


def test_dev_muls_silu_gelu(gpu, ops, golden):
    z = golden["act_z"]
    gz = ops.gputensor_from_numpy(z)
    np.testing.assert_allclose(ops.gputensor_to_numpy(ops.dev_silu(gz)), golden["act_silu"],
                               rtol=2e-6, atol=1e-7)
    # 1 + tanh(u) cancels for u << 0: the reference's own formula carries an
    # absolute error of ~|z| * eps(fp32) there, hence the absolute floor.
    np.testing.assert_allclose(ops.gputensor_to_numpy(ops.dev_gelu(gz)), golden["act_gelu"],
                               rtol=2e-6, atol=1e-6)
    np.testing.assert_array_equal(ops.gputensor_to_numpy(ops.dev_muls(gz, 0.125)), z * np.float32(0.125))
