"""Parity at the benchmark configurations' full sizes and through every
drop-in entry point (-m gpu).

* Config 2 (square sweep, ``C = A B^T`` with B in the nn.Linear layout) at
  every size 1024 ... 16384 in bf16, fp16 and fp32 (3xTF32), plus FFMA at
  the small sizes.  16-bit: per-element bar on sampled rows; fp32: relative
  Frobenius error <= 1e-5 over 64 full rows against the reference's own
  NumPy fp32 product (``tensor.py:1516-1519``).
* Config 4 (the four DiT block linears) at M = 35552 on sampled rows: every
  linear is row-local, so the oracle chain on the sampled rows of x is the
  exact restatement of those output rows.
* The drop-in surface: ``GpuTensor.matmul`` / ``@``, ``nn.Linear`` (fp32 and
  bf16 weights), ``gputensor_to_device``, the host-array ``cuda_*``
  variants, and ``trans_a = 1`` of ``sf_gemm``.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import (assert_close_16bit, assert_close_fp32, device_error, fp32_mode,
                            np_dtype, to_device, to_host32)

pytestmark = pytest.mark.gpu

SQUARE = [1024, 2048, 4096, 8192, 16384]


def _sample_rows(n, k=62, seed=0):
    rows = np.random.default_rng(seed).choice(n, k, replace=False)
    return np.unique(np.concatenate([rows, [0, n - 1]]))


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("n", SQUARE)
def test_config2_square_16bit(gpu, ops, n, dt):
    a, b = O.square_inputs(n, dt, seed=n + 1)
    d = np_dtype(dt)
    ga, gb = ops.gputensor_from_numpy(a.astype(d)), ops.gputensor_from_numpy(b.astype(d))
    c = ops.dev_matmul_nt(ga, gb)
    assert c.dtype == d and c.shape == (n, n)
    out = to_host32(ops, c)
    rows = _sample_rows(n, seed=n)
    assert_close_16bit(out[rows], O.matmul_nt(a[rows], b), f"config 2 {dt} n={n} sampled rows")
    assert np.isfinite(out).all()
    assert device_error(0) == 0


@pytest.mark.parametrize("n", SQUARE)
def test_config2_square_fp32_accurate(gpu, ops, n):
    """3xTF32 (the default fp32 arithmetic) against the reference's fp32
    NumPy product: relative Frobenius error over 64 full rows <= 1e-5."""
    fp32_mode(0)
    a, b = O.square_inputs(n, "f32", seed=n + 2)
    c = ops.gputensor_to_numpy(ops.dev_matmul_nt(ops.gputensor_from_numpy(a),
                                                 ops.gputensor_from_numpy(b)))
    rows = _sample_rows(n, seed=n + 5)
    ref = O.matmul_nt(a[rows], b)
    exact = a[rows].astype(np.float64) @ b.T.astype(np.float64)
    err = O.rel_frobenius(c[rows], ref)
    assert err <= 1e-5, (f"n={n}: rel Frobenius {err:.3e} vs NumPy fp32 "
                         f"(device vs fp64 {O.rel_frobenius(c[rows], exact):.3e}, "
                         f"NumPy vs fp64 {O.rel_frobenius(ref, exact):.3e})")
    assert np.isfinite(c).all()
    assert device_error(0) == 0


@pytest.mark.parametrize("n", [1024, 2048])
def test_config2_square_fp32_ffma(gpu, ops, n):
    """The IEEE fp32 SIMT (FFMA) mode at the small sweep sizes, full output."""
    fp32_mode(1)
    try:
        a, b = O.square_inputs(n, "f32", seed=n + 3)
        c = ops.gputensor_to_numpy(ops.dev_matmul_nt(ops.gputensor_from_numpy(a),
                                                     ops.gputensor_from_numpy(b)))
    finally:
        fp32_mode(0)
    assert_close_fp32(c, O.matmul_nt(a, b), f"FFMA n={n}")


def test_config4_block_linears_full_size(gpu, ops):
    """The config-4 block (M = 35552 tokens, hidden 1920, bf16, zero biases)
    through dit.DitLinears, checked on 64 sampled token rows stage by stage."""
    from scaffolding_b200 import dit
    from scaffolding_b200 import engine as E
    M, C = dit.BATCH * dit.TOKENS, dit.HIDDEN
    w = O.dit_weights(C, seed=4)
    x = O.round_bf16(np.random.default_rng(44).standard_normal((M, C), dtype=np.float32))
    gx = ops.gputensor_from_numpy(x.astype(E.bfloat16))
    lin = dit.DitLinears(w, M, 0)
    lin.run(gx.ptr)
    ops.device_synchronize()
    rows = _sample_rows(M, seed=45)
    xs = x[rows]
    qkv = O.round_bf16(O.linear(xs, w["qkv_w"]))
    h = O.round_bf16(O.linear(qkv[:, :C], w["out_w"], w["out_b"]) + xs)
    f = O.round_bf16(O.gelu_tanh(O.linear(h, w["up_w"], w["up_b"])))
    y = O.linear(f, w["down_w"], w["down_b"]) + h
    got = {k: to_host32(ops, getattr(lin, k))[rows] for k in ("qkv", "h", "f", "y")}
    assert_close_16bit(got["qkv"], O.linear(xs, w["qkv_w"]), "config 4 QKV")
    assert_close_16bit(got["h"], O.linear(got["qkv"][:, :C], w["out_w"], w["out_b"]) + xs,
                       "config 4 out-proj + residual")
    assert_close_16bit(got["f"], O.gelu_tanh(O.linear(got["h"], w["up_w"], w["up_b"])),
                       "config 4 FFN-up + GELU")
    assert_close_16bit(got["y"], O.linear(got["f"], w["down_w"], w["down_b"]) + got["h"],
                       "config 4 FFN-down + residual")
    # the whole chain against the oracle chain on the same rows
    assert O.rel_frobenius(got["y"], y) < 1e-2
    assert device_error(0) == 0


# ───────────────────────────── drop-in entry points ─────────────────────────────

@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_gputensor_matmul_and_operator(gpu, ops, dt):
    """GpuTensor.matmul / @ (the sf.matmul / sf.matmul_nt dispatch of
    tensor.py:1480-1539): 2-D NN and NT, batched with a shared and with a
    batched right operand, and a wider output dtype."""
    rng = np.random.default_rng(3)
    check = assert_close_fp32 if dt == "f32" else assert_close_16bit
    ga, a = to_device(ops, rng.standard_normal((200, 96), dtype=np.float32), dt)
    gb, b = to_device(ops, rng.standard_normal((96, 130), dtype=np.float32), dt)
    gbt, bt = to_device(ops, rng.standard_normal((130, 96), dtype=np.float32), dt)
    check(to_host32(ops, ga @ gb), O.matmul(a, b), f"@ {dt}")
    check(to_host32(ops, ga.matmul(gbt, trans_b=True)), O.matmul_nt(a, bt), f"matmul NT {dt}")
    g3, a3 = to_device(ops, rng.standard_normal((2, 3, 40, 96), dtype=np.float32), dt)
    check(to_host32(ops, g3 @ gb), O.matmul(a3, b), f"batched @ shared B {dt}")
    gb3, b3 = to_device(ops, rng.standard_normal((2, 3, 96, 24), dtype=np.float32), dt)
    check(to_host32(ops, g3.matmul(gb3)), O.batched_matmul(a3, b3), f"batched @ batched B {dt}")
    if dt != "f32":
        wide = ga.matmul(gb, out_dtype=np.float32)
        assert wide.dtype == np.float32
        assert_close_16bit(ops.gputensor_to_numpy(wide), O.matmul(a, b), "bf16 -> fp32 output")


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_nn_linear_forward(gpu, ops, dt):
    """nn.Linear (nn/layers.py:59-146): Kaiming-uniform parameters uploaded in
    the storage dtype, forward = dev_linear_forward with the fused bias and an
    optional fused activation."""
    from scaffolding_b200 import nn
    rng = np.random.default_rng(12)
    lin = nn.Linear(256, 384, device=0, dtype=np_dtype(dt), rng=rng)
    W = to_host32(ops, lin.weight)
    b = to_host32(ops, lin.bias)
    assert np.abs(W).max() <= 1 / 16 + 1e-6  # bound 1/sqrt(in_features)
    gx, x = to_device(ops, rng.standard_normal((3, 70, 256), dtype=np.float32), dt)
    for act in ("none", "silu"):
        y = lin(gx, activation=act)
        assert y.shape == (3, 70, 384)
        ref = O.linear_act(x.reshape(-1, 256), W, b, act).reshape(3, 70, 384)
        if dt == "f32":
            assert_close_fp32(ops.gputensor_to_numpy(y), ref, f"Linear fp32 {act}")
        else:
            assert_close_16bit(to_host32(ops, y), ref, f"Linear bf16 {act}")
    y2 = nn.functional.linear(gx, lin.weight, lin.bias)
    assert_close_16bit(to_host32(ops, y2), O.linear(x.reshape(-1, 256), W, b).reshape(3, 70, 384),
                       "F.linear")


def test_gputensor_to_device_copies_bytes_of_the_dtype(gpu, ops):
    """gputensor_to_device (_cuda_ops.pyx:861-875) copies numel * itemsize
    bytes (the reference assumed 4-byte elements): a bf16 tensor round-trips
    bit for bit; to the same device it is returned as is."""
    bf = np_dtype("bf16")
    x = O.round_bf16(np.random.default_rng(1).standard_normal((333, 77), dtype=np.float32))
    g = ops.gputensor_from_numpy(x.astype(bf))
    assert ops.gputensor_to_device(g, g.device_id) is g
    n = ops.get_device_count()
    if n < 2:
        pytest.skip("the peer copy needs a second GPU")
    ops.init_p2p()
    g1 = ops.gputensor_to_device(g, 1)
    assert g1.device_id == 1 and g1.dtype == bf and g1.shape == g.shape
    back = ops.gputensor_to_numpy(g1)
    assert np.array_equal(back.view(np.uint16), x.astype(bf).view(np.uint16))


def test_host_array_variants(gpu, ops):
    """cuda_matmul / cuda_matmul_nt / cuda_batched_matmul / cuda_linear_forward
    (_cuda_ops.pyx:2120-2225, :2453-2471): NumPy in, NumPy out, fp32."""
    rng = np.random.default_rng(6)
    a = rng.standard_normal((150, 64), dtype=np.float32)
    b = rng.standard_normal((64, 90), dtype=np.float32)
    bt = rng.standard_normal((90, 64), dtype=np.float32)
    assert_close_fp32(ops.cuda_matmul(a, b), O.matmul(a, b), "cuda_matmul")
    assert_close_fp32(ops.cuda_matmul_nt(a, bt), O.matmul_nt(a, bt), "cuda_matmul_nt")
    a3 = rng.standard_normal((4, 30, 64), dtype=np.float32)
    b3 = rng.standard_normal((4, 64, 20), dtype=np.float32)
    assert_close_fp32(ops.cuda_batched_matmul(a3, b3), O.batched_matmul(a3, b3), "cuda_batched")
    x = rng.standard_normal((2, 5, 64), dtype=np.float32)
    bias = rng.standard_normal((90,), dtype=np.float32)
    y = ops.cuda_linear_forward(x, bt, bias)
    assert y.shape == (2, 5, 90)
    assert_close_fp32(y, O.linear(x.reshape(-1, 64), bt, bias).reshape(2, 5, 90),
                      "cuda_linear_forward")


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_trans_a(gpu, ops, dt):
    """sf_gemm with trans_a = 1 (A stored [K, M]), the cuda_sgemm transA
    mapping of _cuda_kernels.cu:1175-1220; both B layouts."""
    from scaffolding_b200 import engine as E
    rng = np.random.default_rng(15)
    M, N, K = 130, 96, 72
    gat, at = to_device(ops, rng.standard_normal((K, M), dtype=np.float32), dt)
    gb, b = to_device(ops, rng.standard_normal((K, N), dtype=np.float32), dt)
    gbt, bt = to_device(ops, rng.standard_normal((N, K), dtype=np.float32), dt)
    code = E.dtype_code(np_dtype(dt))
    check = assert_close_fp32 if dt == "f32" else assert_close_16bit
    for trans_b, bb, ref in ((0, gb, at.T @ b), (1, gbt, at.T @ bt.T)):
        c = ops._alloc((M, N), np_dtype(dt), 0)
        E.gemm(M, N, K, gat.ptr, M, 1, bb.ptr, K if trans_b else N, trans_b, c.ptr, N, code, code)
        check(to_host32(ops, c), ref, f"trans_a {dt} trans_b={trans_b}")
    assert device_error(0) == 0


def test_weights_converted_to_bf16_at_load(gpu, ops):
    """fp32 weights uploaded as the reference does (nn/layers.py:18-35) and
    converted to bf16 on the device (Linear.from_weights, Linear.to): the
    stored bits are the round-to-nearest-even bf16 of the fp32 weights, and
    the layer then runs the bf16 GEMM path."""
    from scaffolding_b200 import nn
    bf = np_dtype("bf16")
    rng = np.random.default_rng(31)
    W = rng.standard_normal((384, 256), dtype=np.float32) * np.float32(0.05)
    b = rng.standard_normal((384,), dtype=np.float32) * np.float32(0.05)
    lin = nn.Linear.from_weights(W, b, device=0, dtype=bf)
    assert lin.weight.dtype == bf and lin.bias.dtype == bf
    assert np.array_equal(ops.gputensor_to_numpy(lin.weight).view(np.uint16),
                          W.astype(bf).view(np.uint16))
    lin32 = nn.Linear.from_weights(W, b, device=0).to(0, bf)
    assert np.array_equal(ops.gputensor_to_numpy(lin32.weight).view(np.uint16),
                          ops.gputensor_to_numpy(lin.weight).view(np.uint16))
    gx, x = to_device(ops, rng.standard_normal((100, 256), dtype=np.float32), "bf16")
    y = lin(gx, activation="gelu_tanh")
    assert y.dtype == bf
    ref = O.linear_act(x, O.round_bf16(W), O.round_bf16(b), O.ACT_GELU_TANH)
    assert_close_16bit(to_host32(ops, y), ref, "bf16-loaded Linear")
