"""sf_linear_skinny_noalloc against the allocating path (-m gpu).

The no-alloc entry point serves callers that cannot allocate device memory
(a process that owns all of the GPU's memory through its own allocator, or
one that must not call cudaMalloc on its latency path), so it cannot be
handed a workspace: its split-K partial sums live in a fixed 4 MiB array
inside the library.  This file checks, through the C ABI, that two calls in
a row (the second one reusing the array the first one left behind) give the
same results as sf_gemm with a workspace, within the bf16 bar the other
tests use, and that oversize problems are rejected.  It sits in a file of
its own, collected last.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import assert_close_16bit, device_error, np_dtype, to_host32

pytestmark = pytest.mark.gpu

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
ACT_NONE, ACT_GELU = 0, 2


def _upload(ops, *arrays):
    bf = np_dtype("bf16")
    return [ops.gputensor_from_numpy(a.astype(bf)) for a in arrays]


def _noalloc(lib, M, N, K, gx, gw, gb, gy):
    return lib.sf_linear_skinny_noalloc(M, N, K, C.c_void_p(gx.ptr), K, C.c_void_p(gw.ptr), K,
                                        C.c_void_p(gb.ptr), DT_BF16, C.c_void_p(gy.ptr), N,
                                        DT_BF16, DT_BF16, ACT_GELU, None)


def test_noalloc_matches_workspace_path_two_calls(gpu, ops):
    from scaffolding_b200._lib import lib
    # Two calls in a row on shapes that both take the split-K route: the
    # second must not see the partial sums the first left in the array.
    for M, N, seed in [(8, 4096, 31), (226, 4096, 32)]:
        K = 4096
        x, W, b = O.skinny_inputs(M, N, K=K, seed=seed)
        gx, gw, gb = _upload(ops, x, W, b)
        ref = to_host32(ops, ops.dev_linear_forward(gx, gw, gb, activation="gelu_tanh"))
        gy = ops._alloc((M, N), np_dtype("bf16"), 0)
        assert _noalloc(lib, M, N, K, gx, gw, gb, gy) == 0, lib.sf_last_error()
        ops.device_synchronize()
        out = to_host32(ops, gy)
        assert_close_16bit(out, ref, f"no-alloc vs sf_gemm M={M} N={N}")
        assert_close_16bit(out, O.linear_act(x, W, b, O.ACT_GELU_TANH), f"no-alloc vs oracle M={M}")
    # a bounded wait that expired inside these kernels would show up here
    assert device_error(0) == 0


def test_noalloc_repeat_is_stable(gpu, ops):
    from scaffolding_b200._lib import lib
    M, N, K = 64, 4096, 4096
    x, W, b = O.skinny_inputs(M, N, K=K, seed=33)
    gx, gw, gb = _upload(ops, x, W, b)
    ref = to_host32(ops, ops.dev_linear_forward(gx, gw, gb, activation="gelu_tanh"))
    outs = []
    for _ in range(2):
        gy = ops._alloc((M, N), np_dtype("bf16"), 0)
        assert _noalloc(lib, M, N, K, gx, gw, gb, gy) == 0, lib.sf_last_error()
        outs.append(to_host32(ops, gy))
    for out in outs:
        assert_close_16bit(out, ref, "no-alloc repeat")
    assert np.isfinite(outs[1]).all()


def test_noalloc_rejects_sizes_beyond_scratch(gpu, ops):
    from scaffolding_b200._lib import SF_ERR_INVALID_ARGUMENT, lib
    M, N, K = 256, 8192, 64  # M*N = 2^21 > 2^20 fp32 values of scratch
    gx, gw, gb = _upload(ops, np.zeros((M, K), np.float32), np.zeros((N, K), np.float32),
                         np.zeros((N,), np.float32))
    gy = ops._alloc((M, N), np_dtype("bf16"), 0)
    assert _noalloc(lib, M, N, K, gx, gw, gb, gy) == SF_ERR_INVALID_ARGUMENT
    assert b"exceeds the fixed scratch" in lib.sf_last_error()


def test_noalloc_single_split_and_fp16_fp32_out(gpu, ops):
    """The paths the bf16 split-K cases above do not reach, each twice in a row:
    K = 64 (one k-block, so no split: the epilogue stores straight from the
    accumulator), and fp16 inputs with an fp32 output and no bias."""
    from scaffolding_b200._lib import lib
    # (M, N, K, input dtype, output dtype, with bias, activation)
    cases = [(8, 4096, 64, "bf16", "bf16", True, ACT_GELU),
             (40, 2048, 1024, "f16", "f32", False, ACT_NONE)]
    codes = {"f32": DT_F32, "f16": DT_F16, "bf16": DT_BF16}
    for M, N, K, din, dout, with_bias, act in cases:
        x, W, b = O.skinny_inputs(M, N, K=K, seed=M + K)
        x, W, b = (O.round_to(t, din) for t in (x, W, b))
        gx, gw, gb = (ops.gputensor_from_numpy(t.astype(np_dtype(din))) for t in (x, W, b))
        act_name = "gelu_tanh" if act == ACT_GELU else "none"
        ref = to_host32(ops, ops.dev_linear_forward(gx, gw, gb if with_bias else None,
                                                    activation=act_name,
                                                    out_dtype=np_dtype(dout)))
        bias_ptr = C.c_void_p(gb.ptr) if with_bias else None
        want = O.linear_act(x, W, b if with_bias else None,
                            O.ACT_GELU_TANH if act == ACT_GELU else O.ACT_NONE)
        for call in range(2):
            gy = ops._alloc((M, N), np_dtype(dout), 0)
            st = lib.sf_linear_skinny_noalloc(M, N, K, C.c_void_p(gx.ptr), K, C.c_void_p(gw.ptr), K,
                                              bias_ptr, codes[din], C.c_void_p(gy.ptr), N,
                                              codes[din], codes[dout], act, None)
            assert st == 0, lib.sf_last_error()
            out = to_host32(ops, gy)
            what = f"no-alloc M={M} K={K} {din}->{dout} call {call}"
            assert_close_16bit(out, ref, what + " vs sf_gemm")
            assert_close_16bit(out, want, what + " vs oracle")
    assert device_error(0) == 0
