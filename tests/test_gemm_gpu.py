"""Parity of the sm_100a GEMM paths against the CPU oracle (-m gpu).

bf16/fp16: per-element relative error <= 1e-2 against the oracle's fp32
result on identically rounded inputs (floor: 1% of the row RMS, see
oracle.elementwise_rel_check).  fp32: relative Frobenius error <= 1e-5.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import (assert_close_16bit, assert_close_fp32, device_error, fp32_mode,
                            kernel_override, np_dtype, to_device, to_host32)

pytestmark = pytest.mark.gpu


def _rand(rng, *shape, scale=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))


def test_bounded_wait_selftest(gpu, ops):
    """An mbarrier wait nobody satisfies expires, records code 6 and returns;
    the context stays usable afterwards."""
    import ctypes as C

    from scaffolding_b200._lib import lib
    code = C.c_int32(-1)
    assert lib.sf_selftest_bounded_wait(50_000_000, C.byref(code), None) == 0
    assert code.value == 6
    a = ops.gputensor_from_numpy(np.ones((4, 4), np.float32))
    np.testing.assert_array_equal(ops.gputensor_to_numpy(ops.dev_muls(a, 2.0)), 2 * np.ones((4, 4)))


# N = 160 and 192 take the 192-wide tile (one tile covers N), the others 256 or narrower
NT_SHAPES = [(128, 256, 64), (256, 512, 512), (300, 200, 136), (129, 257, 72), (512, 16, 64),
             (64, 4096, 8), (1000, 1000, 1000), (777, 333, 264), (300, 160, 136),
             (777, 192, 264)]


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K", NT_SHAPES)
def test_matmul_nt_16bit(gpu, ops, dt, M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    ga, a = to_device(ops, _rand(rng, M, K), dt)
    gb, b = to_device(ops, _rand(rng, N, K), dt)
    out = ops.dev_matmul_nt(ga, gb)
    assert out.dtype == np_dtype(dt) and out.shape == (M, N)
    assert_close_16bit(to_host32(ops, out), O.matmul_nt(a, b), f"nt {dt} {M}x{N}x{K}")


NN_SHAPES = [(256, 64, 512), (300, 136, 200), (128, 256, 64), (1024, 1024, 1024), (70, 64, 1000)]


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K", NN_SHAPES)
def test_matmul_nn_16bit(gpu, ops, dt, M, N, K):
    """B stored [K, N] row-major: MN-major B operand on the tensor cores."""
    rng = np.random.default_rng(M + N + K)
    ga, a = to_device(ops, _rand(rng, M, K), dt)
    gb, b = to_device(ops, _rand(rng, K, N), dt)
    out = ops.dev_matmul(ga, gb)
    assert_close_16bit(to_host32(ops, out), O.matmul(a, b), f"nn {dt} {M}x{N}x{K}")


@pytest.mark.parametrize("path", ["pair", "swap"])
@pytest.mark.parametrize("M", [1, 8, 64, 226])
@pytest.mark.parametrize("N", [4096, 11008])
def test_skinny_linear_bias_gelu(gpu, ops, M, N, path, monkeypatch):
    """Benchmark config 3: bf16 x[M,4096] W[N,4096] b[N], bias + GELU-tanh, on
    the skinny CTA-pair path and on the swap-AB path."""
    if path == "swap":
        monkeypatch.setenv("SF_SKINNY_PAIR", "0")
    else:
        monkeypatch.setenv("SF_SKINNY_PAIR_MIN_M", "5")  # M = 1 stays on the GEMV
        monkeypatch.setenv("SF_SKINNY_PAIR_MIN_N", "1")
    x, W, b = O.skinny_inputs(M, N, seed=M + N)
    bf = np_dtype("bf16")
    gx, gw, gb = (ops.gputensor_from_numpy(t.astype(bf)) for t in (x, W, b))
    y = ops.dev_linear_forward(gx, gw, gb, activation="gelu_tanh")
    ref = O.linear_act(x, W, b, O.ACT_GELU_TANH)
    assert_close_16bit(to_host32(ops, y), ref, f"skinny M={M} N={N}")


def test_config1_fp32_linear_silu_accurate(gpu, ops, golden):
    """Benchmark config 1 through dev_linear_forward in fp32 (3xTF32)."""
    fp32_mode(0)
    x, W, b = O.config1_inputs(seed=0)
    gx, gw, gb = (ops.gputensor_from_numpy(t) for t in (x, W, b))
    y = ops.gputensor_to_numpy(ops.dev_linear_forward(gx, gw, gb, activation="silu"))
    assert y.dtype == np.float32
    assert_close_fp32(y[::8], golden["cfg1_y_rows"], "config 1 vs reference golden rows")
    assert_close_fp32(y, O.linear_act(x, W, b, O.ACT_SILU), "config 1 vs oracle")


@pytest.mark.parametrize("mode,tol", [(0, 1e-5), (1, 1e-5), (2, 3e-3)])
@pytest.mark.parametrize("nt", [True, False])
def test_fp32_modes(gpu, ops, mode, tol, nt):
    """fp32: 3xTF32 (accurate), FFMA and single TF32, NT and NN."""
    fp32_mode(mode)
    try:
        rng = np.random.default_rng(11)
        M, N, K = 333, 517, 1029
        a = _rand(rng, M, K)
        b = _rand(rng, N, K) if nt else _rand(rng, K, N)
        ga, gb = ops.gputensor_from_numpy(a), ops.gputensor_from_numpy(b)
        out = ops.dev_matmul_nt(ga, gb) if nt else ops.dev_matmul(ga, gb)
        ref = O.matmul_nt(a, b) if nt else O.matmul(a, b)
        assert_close_fp32(ops.gputensor_to_numpy(out), ref, f"fp32 mode {mode}", tol)
    finally:
        fp32_mode(0)


@pytest.mark.parametrize("tag", ["mm_a", "mm_b", "mm_c"])
def test_golden_matmuls_fp32(gpu, ops, golden, tag):
    a, b, bt = golden[f"{tag}_a"], golden[f"{tag}_b"], golden[f"{tag}_bt"]
    ga, gb, gbt = (ops.gputensor_from_numpy(t) for t in (a, b, bt))
    assert_close_fp32(ops.gputensor_to_numpy(ops.dev_matmul(ga, gb)), golden[f"{tag}_nn"], tag)
    assert_close_fp32(ops.gputensor_to_numpy(ops.dev_matmul_nt(ga, gbt)), golden[f"{tag}_nt"], tag)


@pytest.mark.parametrize("tag,act,dt", [("lin_silu_f32", "silu", "f32"),
                                        ("lin_gelu_f32", "gelu_tanh", "f32"),
                                        ("lin_none_f32", "none", "f32"),
                                        ("lin_gelu_bf16", "gelu_tanh", "bf16"),
                                        ("lin_silu_f16", "silu", "f16")])
def test_golden_linear(gpu, ops, golden, tag, act, dt):
    d = np_dtype(dt)
    gx, gw, gb = (ops.gputensor_from_numpy(golden[f"{tag}_{s}"].astype(d)) for s in "xwb")
    y = to_host32(ops, ops.dev_linear_forward(gx, gw, gb, activation=act))
    if dt == "f32":
        assert_close_fp32(y, golden[f"{tag}_y"], tag)
    else:
        assert_close_16bit(y, golden[f"{tag}_y"], tag)


def test_golden_batched_fp32(gpu, ops, golden):
    ga, gb, gbt = (ops.gputensor_from_numpy(golden[k]) for k in ("bmm_a", "bmm_b", "bmm_bt"))
    assert_close_fp32(ops.gputensor_to_numpy(ops.dev_batched_matmul(ga, gb)), golden["bmm_nn"], "bmm")
    assert_close_fp32(ops.gputensor_to_numpy(ops.dev_batched_matmul_nt(ga, gbt)),
                      golden["bmm_nt"], "bmm_nt")


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_batched_16bit(gpu, ops, dt):
    rng = np.random.default_rng(5)
    ga, a = to_device(ops, _rand(rng, 2, 3, 136, 64), dt)
    gk, k = to_device(ops, _rand(rng, 2, 3, 200, 64), dt)
    gv, v = to_device(ops, _rand(rng, 2, 3, 200, 64), dt)
    s = ops.dev_batched_matmul_nt(ga, gk)
    assert s.shape == (2, 3, 136, 200)
    assert_close_16bit(to_host32(ops, s), O.batched_matmul_nt(a, k), "bmm_nt")
    gp, p = to_device(ops, _rand(rng, 2, 3, 136, 200), dt)
    o = ops.dev_batched_matmul(gp, gv)
    assert_close_16bit(to_host32(ops, o), O.batched_matmul(p, v), "bmm_nn")


def test_two_level_batch_strided_heads(gpu, ops):
    """Per-(batch, head) QK^T reading q/k straight out of a fused QKV
    activation [B*N, 3*H*D] (two-level batch, head stride = D elements)."""
    from scaffolding_b200 import engine as E
    rng = np.random.default_rng(9)
    B, N, H, D = 2, 333, 3, 64
    Cw = H * D
    gqkv, qkv = to_device(ops, _rand(rng, B * N, 3 * Cw), "bf16")
    out = ops._alloc((B, H, N, N), np.float32, 0)
    bt = E.make_batch(H, B, a=(D, N * 3 * Cw), b=(D, N * 3 * Cw), c=(N * N, H * N * N))
    E.gemm(N, N, D, gqkv.ptr, 3 * Cw, 0, gqkv.ptr + Cw * 2, 3 * Cw, 1, out.ptr, N, 2, 0,
           epi=E.make_epilogue(alpha=0.125), batch=bt)
    s = ops.gputensor_to_numpy(out)
    for b in range(B):
        blk = qkv[b * N:(b + 1) * N]
        for h in range(H):
            q = blk[:, h * D:(h + 1) * D]
            k = blk[:, Cw + h * D:Cw + (h + 1) * D]
            ref = (q @ k.T) * np.float32(0.125)
            assert_close_fp32(s[b, h], ref, f"b{b} h{h}", tol=1e-5)


def test_epilogue_residual_alpha_bias(gpu, ops):
    from scaffolding_b200 import engine as E
    rng = np.random.default_rng(21)
    M, N, K = 300, 384, 256
    gx, x = to_device(ops, _rand(rng, M, K), "bf16")
    gw, w = to_device(ops, _rand(rng, N, K, scale=0.05), "bf16")
    gb, bias = to_device(ops, _rand(rng, N), "bf16")
    gr, res = to_device(ops, _rand(rng, M, N), "bf16")
    out = ops._alloc((M, N), np_dtype("bf16"), 0)
    epi = E.make_epilogue(alpha=0.5, bias_ptr=gb.ptr, bias_dt=2, act=2, residual_ptr=gr.ptr,
                          residual_dt=2, ldr=N, beta=1.0)
    E.gemm(M, N, K, gx.ptr, K, 0, gw.ptr, K, 1, out.ptr, N, 2, 2, epi=epi)
    ref = O.gelu_tanh(0.5 * (x @ w.T) + bias) + res
    assert_close_16bit(to_host32(ops, out), ref, "epilogue")


def test_simt_path_matches_tcgen05(gpu, ops):
    rng = np.random.default_rng(4)
    ga, a = to_device(ops, _rand(rng, 257, 192), "bf16")
    gb, b = to_device(ops, _rand(rng, 300, 192), "bf16")
    tc = to_host32(ops, ops.dev_matmul_nt(ga, gb))
    kernel_override(2)
    try:
        simt = to_host32(ops, ops.dev_matmul_nt(ga, gb))
    finally:
        kernel_override(0)
    ref = O.matmul_nt(a, b)
    assert_close_16bit(tc, ref, "tcgen05")
    assert_close_16bit(simt, ref, "simt")


def test_unaligned_rows_take_simt_path(gpu, ops):
    """K = 53 bf16 rows are not 16-byte multiples: TMA cannot describe them."""
    rng = np.random.default_rng(8)
    ga, a = to_device(ops, _rand(rng, 37, 53), "bf16")
    gb, b = to_device(ops, _rand(rng, 29, 53), "bf16")
    assert_close_16bit(to_host32(ops, ops.dev_matmul_nt(ga, gb)), O.matmul_nt(a, b), "odd K")


@pytest.mark.parametrize("n", [4096, 8192])
def test_large_square_bf16_sampled(gpu, ops, n):
    """Benchmark config 2 sizes; the oracle checks a sample of output rows."""
    a, b = O.square_inputs(n, "bf16", seed=n)
    bf = np_dtype("bf16")
    ga, gb = ops.gputensor_from_numpy(a.astype(bf)), ops.gputensor_from_numpy(b.astype(bf))
    c = to_host32(ops, ops.dev_matmul_nt(ga, gb))
    rows = np.random.default_rng(0).choice(n, 96, replace=False)
    rows = np.concatenate([rows, [0, n - 1]])
    assert_close_16bit(c[rows], a[rows] @ b.T, f"square {n} sampled rows")
    assert np.isfinite(c).all()


def test_zero_k_gives_bias_only(gpu, ops):
    x = ops.gputensor_from_numpy(np.zeros((5, 0), np.float32))
    w = ops.gputensor_from_numpy(np.zeros((7, 0), np.float32))
    b = ops.gputensor_from_numpy(np.arange(7, dtype=np.float32))
    y = ops.gputensor_to_numpy(ops.dev_linear_forward(x, w, b))
    np.testing.assert_array_equal(y, np.tile(np.arange(7, dtype=np.float32), (5, 1)))


def test_no_device_errors_recorded(gpu):
    assert device_error(0) == 0


def test_graph_capture_replays_gemm(gpu, ops):
    """A GEMM captured into a CUDA graph and replayed gives the same result as
    the direct launch (used for launch-bound skinny shapes)."""
    import ctypes as C

    from scaffolding_b200 import engine as E
    from scaffolding_b200._lib import lib
    rng = np.random.default_rng(77)
    M, N, K = 8, 4096, 4096
    ga, a = to_device(ops, _rand(rng, M, K), "bf16")
    gb, b = to_device(ops, _rand(rng, N, K, scale=0.02), "bf16")
    sp = C.c_void_p()
    assert lib.sf_stream_create(0, 1, C.byref(sp)) == 0
    s = sp.value
    y1 = ops._alloc((M, N), np_dtype("bf16"), 0)
    y2 = ops._alloc((M, N), np_dtype("bf16"), 0)
    E.gemm(M, N, K, ga.ptr, K, 0, gb.ptr, K, 1, y1.ptr, N, 2, 2, stream=s)  # sizes the workspace
    E.stream_sync(s)
    g = C.c_void_p()
    assert lib.sf_graph_begin(C.c_void_p(s)) == 0
    E.gemm(M, N, K, ga.ptr, K, 0, gb.ptr, K, 1, y2.ptr, N, 2, 2, stream=s)
    assert lib.sf_graph_end(C.c_void_p(s), C.byref(g)) == 0
    for _ in range(3):
        assert lib.sf_graph_launch(g, C.c_void_p(s)) == 0
    E.stream_sync(s)
    assert lib.sf_graph_destroy(g) == 0
    lib.sf_stream_destroy(C.c_void_p(s))
    r1, r2 = to_host32(ops, y1), to_host32(ops, y2)
    assert_close_16bit(r2, O.matmul_nt(a, b), "graph replay")
    assert_close_16bit(r1, r2, "direct vs graph")


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("K", [1024, 776])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_gemv_small_m(gpu, ops, M, K, dt, monkeypatch):
    """Small M runs on the GEMV kernels (balanced one for K % 256 == 0, up to
    M = 8 here; row-per-warp one otherwise): ragged N, bias + GELU and a
    residual, against the oracle."""
    from scaffolding_b200 import engine as E
    monkeypatch.setenv("SF_GEMV_MAX_M", "8")
    rng = np.random.default_rng(90 + M + K)
    N = 1003
    gx, x = to_device(ops, _rand(rng, M, K), dt)
    gw, w = to_device(ops, _rand(rng, N, K, scale=0.03), dt)
    gb, b = to_device(ops, _rand(rng, N, scale=0.1), dt)
    gr, res = to_device(ops, _rand(rng, M, N), dt)
    out = ops._alloc((M, N), np_dtype(dt), 0)
    code = E.dtype_code(np_dtype(dt))
    epi = E.make_epilogue(bias_ptr=gb.ptr, bias_dt=code, act=2, residual_ptr=gr.ptr,
                          residual_dt=code, ldr=N)
    E.gemm(M, N, K, gx.ptr, K, 0, gw.ptr, K, 1, out.ptr, N, code, code, epi=epi)
    ref = O.gelu_tanh(O.linear(x, w, b)) + res
    assert_close_16bit(to_host32(ops, out), ref, f"gemv M={M} {dt}")


# M >= 1024, K >= 256, N > 64: the CTA-pair (cta_group::2) kernel.  Ragged M
# (not a multiple of the 256-row pair tile), ragged N and K, and both
# pair tile widths.
PAIR_SHAPES = [(1024, 256, 256), (1100, 1000, 300), (2048, 1920, 1920), (1536, 384, 512),
               (1280, 200, 264), (1030, 5760, 640)]


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
def test_pair_kernel_nt(gpu, ops, dt, M, N, K, monkeypatch):
    rng = np.random.default_rng(M + 5 * N + 11 * K)
    ga, a = to_device(ops, _rand(rng, M, K), dt)
    gb, b = to_device(ops, _rand(rng, N, K), dt)
    monkeypatch.setenv("SF_PAIR", "1")  # every eligible GEMM on the pair kernel
    pair = to_host32(ops, ops.dev_matmul_nt(ga, gb))
    monkeypatch.delenv("SF_PAIR")
    kernel_override(3)  # SF_KERNEL_TCGEN05_1CTA
    try:
        single = to_host32(ops, ops.dev_matmul_nt(ga, gb))
    finally:
        kernel_override(0)
    ref = O.matmul_nt(a, b)
    assert_close_16bit(pair, ref, f"pair {dt} {M}x{N}x{K}")
    assert_close_16bit(single, ref, f"1-CTA {dt} {M}x{N}x{K}")
    assert device_error(0) == 0


def test_pair_kernel_fused_epilogue_and_batch(gpu, ops, monkeypatch):
    """Bias + GELU + scaled residual on the pair kernel, and a batched pair GEMM."""
    from scaffolding_b200 import engine as E
    monkeypatch.setenv("SF_PAIR", "1")
    rng = np.random.default_rng(123)
    M, N, K = 1300, 768, 384
    gx, x = to_device(ops, _rand(rng, M, K), "bf16")
    gw, w = to_device(ops, _rand(rng, N, K, scale=0.05), "bf16")
    gb, bias = to_device(ops, _rand(rng, N, scale=0.1), "bf16")
    gr, res = to_device(ops, _rand(rng, M, N), "bf16")
    out = ops._alloc((M, N), np_dtype("bf16"), 0)
    epi = E.make_epilogue(alpha=0.5, bias_ptr=gb.ptr, bias_dt=2, act=2, residual_ptr=gr.ptr,
                          residual_dt=2, ldr=N, beta=1.0)
    E.gemm(M, N, K, gx.ptr, K, 0, gw.ptr, K, 1, out.ptr, N, 2, 2, epi=epi)
    ref = O.gelu_tanh(0.5 * (x @ w.T) + bias) + res
    assert_close_16bit(to_host32(ops, out), ref, "pair epilogue")

    B = 3
    ga, a = to_device(ops, _rand(rng, B, 1024, 256), "bf16")
    gbb, bb = to_device(ops, _rand(rng, B, 320, 256), "bf16")
    c = to_host32(ops, ops.dev_batched_matmul_nt(ga, gbb))
    assert_close_16bit(c, O.batched_matmul_nt(a, bb), "pair batched")
    assert device_error(0) == 0


@pytest.mark.parametrize("M,N,K", [(5, 1024, 64), (17, 3000, 200), (128, 4100, 520), (129, 2048, 256),
                                   (256, 1536, 1024), (200, 11008, 4096)])
def test_skinny_pair_ragged(gpu, ops, M, N, K, monkeypatch):
    """Skinny CTA-pair path: A boxes of round_up(M, 8) rows, the odd CTA idle
    when M <= 128, ragged N tiles and K, fp16 and bf16."""
    monkeypatch.setenv("SF_SKINNY_PAIR_MIN_M", "1")
    monkeypatch.setenv("SF_SKINNY_PAIR_MIN_N", "1")
    for dt in ("bf16", "f16"):
        rng = np.random.default_rng(M * 31 + N + K)
        ga, a = to_device(ops, _rand(rng, M, K), dt)
        gb, b = to_device(ops, _rand(rng, N, K, scale=0.05), dt)
        out = to_host32(ops, ops.dev_matmul_nt(ga, gb))
        assert_close_16bit(out, O.matmul_nt(a, b), f"skinny pair {dt} {M}x{N}x{K}")
    assert device_error(0) == 0


@pytest.mark.parametrize("M,N,K", [(8, 4096, 4096), (33, 1000, 777), (200, 3000, 1000), (5, 300, 4160),
                                   (64, 11008, 4096)])
def test_swap_ab_path(gpu, ops, M, N, K, monkeypatch):
    """Swap-AB skinny GEMM (k-blocks split so that every SM streams the same
    share of the weights, partial slices summed by the finaliser), with a
    bias + GELU + residual epilogue; the split count differs per shape."""
    from scaffolding_b200 import engine as E
    monkeypatch.setenv("SF_SKINNY_PAIR", "0")
    rng = np.random.default_rng(M * 3 + N + K)
    gx, x = to_device(ops, _rand(rng, M, K), "bf16")
    gw, w = to_device(ops, _rand(rng, N, K, scale=0.03), "bf16")
    gb, b = to_device(ops, _rand(rng, N, scale=0.1), "bf16")
    gr, res = to_device(ops, _rand(rng, M, N), "bf16")
    out = ops._alloc((M, N), np_dtype("bf16"), 0)
    epi = E.make_epilogue(bias_ptr=gb.ptr, bias_dt=2, act=2, residual_ptr=gr.ptr, residual_dt=2,
                          ldr=N)
    E.gemm(M, N, K, gx.ptr, K, 0, gw.ptr, K, 1, out.ptr, N, 2, 2, epi=epi)
    ref = O.gelu_tanh(O.linear(x, w, b)) + res
    assert_close_16bit(to_host32(ops, out), ref, f"swap-AB {M}x{N}x{K}")
    assert device_error(0) == 0
