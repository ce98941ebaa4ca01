"""The C ABI library loads, exports every symbol include/sf_engine.h declares,
and rejects bad arguments before touching a device.  CPU only."""
import ctypes as C
import inspect
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sf_engine.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int32_t|const char\s*\*)\s*(sf_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from scaffolding_b200 import _lib
    names = _declared()
    assert len(names) >= 40
    for n in names:
        assert hasattr(_lib.lib, n), f"{n} declared but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signature table out of sync with header"


def test_library_loaded_from_tree():
    from scaffolding_b200 import _lib
    assert os.path.dirname(_lib.LIB_PATH) == os.path.join(ROOT, "scaffolding_b200")
    assert _lib.lib.sf_version().decode().startswith("scaffolding-b200")


def test_struct_layouts_match_header():
    from scaffolding_b200 import _lib
    # sf_epilogue: 2 floats, ptr, 2 int32, ptr, 2 int32, 3 int64 = 64 bytes on LP64
    assert C.sizeof(_lib.Epilogue) == 64
    assert C.sizeof(_lib.Batch) == 64
    assert C.sizeof(_lib.DeviceProps) == 256 + 8 + 4 * 6 + 8 * 3 + 4 * 4


def test_invalid_arguments_rejected():
    from scaffolding_b200._lib import SF_ERR_INVALID_ARGUMENT, lib
    st = lib.sf_gemm(-1, 4, 4, None, 4, 0, None, 4, 1, None, 4, 2, 2, None, None, 0, None)
    assert st == SF_ERR_INVALID_ARGUMENT
    assert b"negative" in lib.sf_last_error()
    st = lib.sf_gemm(4, 4, 4, None, 4, 0, None, 4, 1, None, 4, 9, 2, None, None, 0, None)
    assert st == SF_ERR_INVALID_ARGUMENT
    st = lib.sf_gemm(4, 4, 4, None, 4, 3, None, 4, 1, None, 4, 2, 2, None, None, 0, None)
    assert st == SF_ERR_INVALID_ARGUMENT
    assert lib.sf_set_fp32_mode(7) == SF_ERR_INVALID_ARGUMENT
    assert lib.sf_softmax_rows(None, 0, 4, None, 0, 4, -1, 4, 1.0, None) == SF_ERR_INVALID_ARGUMENT
    # zero-sized problems are no-ops, even without a device
    assert lib.sf_gemm(0, 4, 4, None, 4, 0, None, 4, 1, None, 4, 2, 2, None, None, 0, None) == 0


def test_workspace_sizes():
    from scaffolding_b200._lib import lib
    sz = C.c_size_t()

    def ws(M, N, K, ta, tb, dt):
        assert lib.sf_gemm_workspace_size(None, M, N, K, ta, tb, dt, dt, C.byref(sz)) == 0
        return sz.value

    # bf16 large GEMM: direct tcgen05, no workspace
    assert ws(4096, 4096, 4096, 0, 1, 2) == 0
    # fp32 accurate (3xTF32): K-concatenated hi/lo panels for A and B
    assert ws(512, 4096, 1024, 0, 1, 0) == (512 + 4096) * 3 * 1024 * 4
    # skinny bf16, M <= 32: swap-AB; the k-blocks are split so that every SM
    # streams the same share of the weights, one fp32 partial slice per split
    # (148 SMs: 32 tiles x 13 splits of 5 k-blocks; 86 tiles x 5 splits)
    assert ws(8, 4096, 4096, 0, 1, 2) == 13 * 8 * 4096 * 4
    assert ws(8, 11008, 4096, 0, 1, 2) == 5 * 8 * 11008 * 4
    # M = 33..128 (and up to 256 at N < 8192) on the swap-AB path too
    assert ws(64, 4096, 4096, 0, 1, 2) == 4 * 64 * 4096 * 4
    # wide outputs with M = 129..256 on CTA pairs (one pair tile holds all M
    # rows): no workspace
    assert ws(226, 11008, 4096, 0, 1, 2) == 0
    # the same shape on the swap-AB path: too many partial bytes to split
    os.environ["SF_SKINNY_PAIR"] = "0"
    try:
        assert ws(226, 11008, 4096, 0, 1, 2) == 0
    finally:
        del os.environ["SF_SKINNY_PAIR"]


def test_fp32_mode_roundtrip():
    from scaffolding_b200._lib import lib
    m = C.c_int32()
    for mode in (1, 2, 0):
        assert lib.sf_set_fp32_mode(mode) == 0
        assert lib.sf_get_fp32_mode(C.byref(m)) == 0 and m.value == mode


def test_drop_in_surface_signatures(ops):
    """Hot-path names exist with the reference's parameter names."""
    expect = {
        "dev_matmul": ["gt_a", "gt_b"],
        "dev_matmul_nt": ["gt_a", "gt_b"],
        "dev_batched_matmul": ["gt_a", "gt_b"],
        "dev_batched_matmul_nt": ["gt_a", "gt_b"],
        "dev_linear_forward": ["gt_x", "gt_weight", "gt_bias"],
        "gputensor_from_numpy": ["arr", "device_id"],
        "gputensor_to_numpy": ["gt"],
        "gputensor_to_device": ["gt", "target_dev"],
        "dev_muls": ["gt", "scalar"],
        "dev_softmax": ["gt", "dim"],
        "cuda_matmul": ["a", "b"],
        "cuda_matmul_nt": ["a", "b"],
        "cuda_batched_matmul": ["a", "b"],
        "cuda_linear_forward": ["x", "weight", "bias"],
        "set_tf32_enabled": ["enable"],
    }
    for name, params in expect.items():
        sig = list(inspect.signature(getattr(ops, name)).parameters)
        assert sig[:len(params)] == params, (name, sig)
    for name in ["set_device", "get_device_count", "get_current_device", "device_synchronize",
                 "get_device_properties", "get_device_capability", "get_device_name", "mem_info",
                 "empty_cache", "init_all_devices", "init_p2p", "can_access_peer", "CudaStream",
                 "CudaEvent", "cublas_set_stream", "dev_silu", "dev_gelu", "dev_reshape",
                 "dev_unsqueeze", "dev_squeeze", "GpuTensor", "CudaBuffer"]:
        assert hasattr(ops, name), name


def test_out_of_scope_ops_raise(ops):
    with pytest.raises(NotImplementedError, match="dev_rms_norm"):
        ops.dev_rms_norm(None, None, None)
    with pytest.raises(AttributeError):
        ops.definitely_not_an_op


def _fake(ops, shape, dtype=np.float32, dev=0):
    buf = ops.CudaBuffer(0, 0, dev, False)
    return ops.GpuTensor(buf, shape, dtype, dev)


def test_shape_and_dtype_validation_precedes_launch(ops):
    a = _fake(ops, (4, 8))
    with pytest.raises(ValueError, match="shape mismatch"):
        ops.dev_matmul(a, _fake(ops, (9, 3)))
    with pytest.raises(ValueError, match="shape mismatch"):
        ops.dev_matmul_nt(a, _fake(ops, (3, 9)))
    with pytest.raises(TypeError, match="share a dtype"):
        ops.dev_matmul(a, _fake(ops, (8, 3), np.float16))
    with pytest.raises(ValueError, match="different devices"):
        ops.dev_matmul(a, _fake(ops, (8, 3), np.float32, dev=1))
    with pytest.raises(ValueError, match="linear shape mismatch"):
        ops.dev_linear_forward(_fake(ops, (2, 3, 8)), _fake(ops, (16, 7)))
    with pytest.raises(ValueError, match="batch dims differ"):
        ops.dev_batched_matmul(_fake(ops, (2, 3, 4, 8)), _fake(ops, (5, 8, 6)))


def test_reshape_family_is_metadata_only(ops):
    t = _fake(ops, (2, 3, 4))
    assert ops.dev_reshape(t, (6, -1)).shape == (6, 4)
    assert ops.dev_unsqueeze(t, 0).shape == (1, 2, 3, 4)
    assert ops.dev_squeeze(ops.dev_unsqueeze(t, -1)).shape == (2, 3, 4)
    with pytest.raises(ValueError):
        ops.dev_reshape(t, (5, 5))


def test_dtype_codes():
    from scaffolding_b200 import engine as E
    assert E.dtype_code(np.float32) == 0 and E.dtype_code(np.float16) == 1
    assert E.dtype_code(E.bfloat16) == 2
    with pytest.raises(TypeError):
        E.dtype_code(np.float64)
    with pytest.raises(ValueError):
        E.act_code("relu")
