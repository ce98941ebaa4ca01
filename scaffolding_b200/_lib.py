"""ctypes binding of ``libsf_engine.so`` (declared in ``include/sf_engine.h``).

The library is built in-tree by ``scaffolding_b200.build``.  There is no
fallback: if the shared library is missing or fails to load, importing this
module raises ``ImportError`` naming the build command.  ctypes releases the
GIL around every foreign call, so GPU launches never hold it (the reference
held it around its SGEMM calls, ``_cuda_ops.pyx:1098``).
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libsf_engine.so")

SF_OK = 0
SF_ERR_INVALID_ARGUMENT = -1
SF_ERR_UNSUPPORTED = -2
SF_ERR_CUDA = -3
SF_ERR_OUT_OF_MEMORY = -4
SF_ERR_WORKSPACE = -5
SF_ERR_DEVICE_TIMEOUT = -6
SF_ERR_NCCL = -7

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
ACT_NONE, ACT_SILU, ACT_GELU_TANH = 0, 1, 2
FP32_ACCURATE, FP32_FFMA, FP32_TF32 = 0, 1, 2
KERNEL_AUTO, KERNEL_TCGEN05, KERNEL_SIMT = 0, 1, 2
COPY_H2D, COPY_D2H, COPY_D2D, COPY_DEFAULT = 0, 1, 2, 3


class Epilogue(C.Structure):
    _fields_ = [
        ("alpha", C.c_float), ("beta", C.c_float),
        ("bias", C.c_void_p), ("bias_dtype", C.c_int32), ("activation", C.c_int32),
        ("residual", C.c_void_p), ("residual_dtype", C.c_int32), ("reserved", C.c_int32),
        ("ldr", C.c_int64), ("r_stride0", C.c_int64), ("r_stride1", C.c_int64),
    ]


class Batch(C.Structure):
    _fields_ = [
        ("count0", C.c_int64), ("count1", C.c_int64),
        ("a_stride0", C.c_int64), ("a_stride1", C.c_int64),
        ("b_stride0", C.c_int64), ("b_stride1", C.c_int64),
        ("c_stride0", C.c_int64), ("c_stride1", C.c_int64),
    ]


class DeviceProps(C.Structure):
    _fields_ = [
        ("name", C.c_char * 256), ("total_memory", C.c_uint64),
        ("major", C.c_int32), ("minor", C.c_int32),
        ("multi_processor_count", C.c_int32), ("max_threads_per_block", C.c_int32),
        ("max_threads_per_mp", C.c_int32), ("warp_size", C.c_int32),
        ("shared_mem_per_block", C.c_uint64), ("shared_mem_per_block_optin", C.c_uint64),
        ("l2_cache_size", C.c_uint64), ("clock_rate_khz", C.c_int32),
        ("memory_clock_rate_khz", C.c_int32), ("memory_bus_width", C.c_int32),
        ("reserved", C.c_int32),
    ]


_i32, _i64, _vp, _sz = C.c_int32, C.c_int64, C.c_void_p, C.c_size_t
_P = C.POINTER

# name -> argtypes (all return int32 status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "sf_gemm": [_i64, _i64, _i64, _vp, _i64, _i32, _vp, _i64, _i32, _vp, _i64, _i32, _i32,
                _P(Epilogue), _vp, _sz, _vp],
    "sf_gemm_batched": [_P(Batch), _i64, _i64, _i64, _vp, _i64, _i32, _vp, _i64, _i32, _vp, _i64,
                        _i32, _i32, _P(Epilogue), _vp, _sz, _vp],
    "sf_linear_skinny_noalloc": [_i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _i32, _vp, _i64,
                                 _i32, _i32, _i32, _vp],
    "sf_gemm_workspace_size": [_P(Batch), _i64, _i64, _i64, _i32, _i32, _i32, _i32, _P(_sz)],
    "sf_set_fp32_mode": [_i32],
    "sf_get_fp32_mode": [_P(_i32)],
    "sf_set_kernel_override": [_i32],
    "sf_softmax_rows": [_vp, _i32, _i64, _vp, _i32, _i64, _i64, _i64, C.c_float, _vp],
    "sf_attention_fwd": [_i32, _i32, _i32, _i32, _i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp,
                         _i64, _i64, _vp, _i64, _i64, C.c_float, _i32, _vp],
    "sf_attention_fwd_partial": [_i32, _i32, _i32, _i32, _i32, _vp, _i64, _i64, _vp, _i64, _i64,
                                 _vp, _i64, _i64, _vp, _i64, _i64, C.c_float, _i32, _i32, _i32,
                                 _vp, _vp, _i32, _vp],
    "sf_attention_launch_count": [_i32, _i32, _i32, _i32, _i32, _i32, _P(_i32)],
    "sf_unary": [_vp, _i32, _vp, _i32, _i64, C.c_float, _i32, _vp],
    "sf_layernorm_modulate": [_i64, _i64, _vp, _i32, _i64, _vp, _vp, C.c_float, _vp, _i32, _i64,
                              _i64, _vp, _i32, _i64, _vp],
    "sf_device_count": [_P(_i32)],
    "sf_set_device": [_i32],
    "sf_get_device": [_P(_i32)],
    "sf_device_synchronize": [],
    "sf_device_properties": [_i32, _P(DeviceProps)],
    "sf_mem_info": [_P(_sz), _P(_sz)],
    "sf_malloc": [_i32, _sz, _P(_vp)],
    "sf_free": [_i32, _vp, _sz],
    "sf_empty_cache": [_i32],
    "sf_pool_stats": [_i32, _P(_sz), _P(_sz)],
    "sf_set_pool_cap": [_sz],
    "sf_host_alloc_pinned": [_sz, _P(_vp)],
    "sf_host_free_pinned": [_vp],
    "sf_memcpy": [_vp, _vp, _sz, _i32, _vp],
    "sf_memcpy_peer": [_vp, _i32, _vp, _i32, _sz, _vp],
    "sf_ipc_alloc": [_sz, _P(_vp)],
    "sf_ipc_free": [_vp],
    "sf_ipc_handle": [_vp, _P(C.c_uint8)],
    "sf_ipc_open": [_P(C.c_uint8), _P(_vp)],
    "sf_ipc_close": [_vp],
    "sf_flag_store": [_P(_vp), _i32, _i32, _vp],
    "sf_flag_wait": [_vp, _i32, _i32, _i32, _i32, _i64, _vp],
    "sf_memset": [_vp, _i32, _sz, _vp],
    "sf_stream_create": [_i32, _i32, _P(_vp)],
    "sf_stream_create_priority": [_i32, _i32, _i32, _P(_vp)],
    "sf_stream_destroy": [_vp],
    "sf_stream_synchronize": [_vp],
    "sf_stream_wait_event": [_vp, _vp],
    "sf_event_create": [_i32, _P(_vp)],
    "sf_event_destroy": [_vp],
    "sf_event_record": [_vp, _vp],
    "sf_event_synchronize": [_vp],
    "sf_event_elapsed_ms": [_vp, _vp, _P(C.c_float)],
    "sf_graph_begin": [_vp],
    "sf_graph_end": [_vp, _P(_vp)],
    "sf_graph_launch": [_vp, _vp],
    "sf_graph_destroy": [_vp],
    "sf_can_access_peer": [_i32, _i32, _P(_i32)],
    "sf_enable_peer_access_all": [],
    "sf_device_error_status": [_i32, _P(_i32), _i32],
    "sf_selftest_bounded_wait": [_i64, _P(_i32), _vp],
    "sf_fill_normal": [_vp, _i32, _i64, C.c_uint64, C.c_float, C.c_float, _vp],
    "sf_last_error": [],
    "sf_version": [],
    "sf_comm_unique_id": [_P(C.c_uint8)],
    "sf_comm_init": [_P(_vp), _i32, _i32, _P(C.c_uint8)],
    "sf_comm_split": [_vp, _i32, _i32, _P(_vp)],
    "sf_comm_allgather": [_vp, _vp, _vp, _sz, _vp],
    "sf_comm_allreduce_f32": [_vp, _P(C.c_float), _sz, _i32, _vp],
    "sf_comm_async_error": [_vp, _P(_i32)],
    "sf_comm_abort": [_vp],
    "sf_comm_destroy": [_vp],
}
_RESTYPES = {"sf_last_error": C.c_char_p, "sf_version": C.c_char_p}


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"scaffolding_b200: engine library {LIB_PATH} is missing; build it with "
            "`python -m scaffolding_b200.build` (there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, C.c_int32)
    return lib


lib = _load()


class EngineError(RuntimeError):
    """Raised for a nonzero engine status (the reference raised RuntimeError
    for CUDA failures, ``_cuda_ops.pyx:292-300``)."""

    def __init__(self, status: int, where: str):
        msg = lib.sf_last_error().decode(errors="replace")
        super().__init__(f"{where}: engine status {status}: {msg}")
        self.status = status


def check(status: int, where: str) -> None:
    if status != SF_OK:
        raise EngineError(status, where)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
