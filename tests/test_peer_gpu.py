"""Peer flags of the copy-engine K/V exchange on one GPU (-m gpu): the
release-store and bounded acquire-wait kernels (sf_flag_store /
sf_flag_wait) and the IPC buffer calls that need no second process.

The expired wait is made on a flag that nothing stores, with a 1 ms limit:
the kernel records code 7 in the device error word and returns, and the
stream keeps working (no fault, no hang)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ipc_alloc(lib, nbytes):
    p = C.c_void_p()
    assert lib.sf_ipc_alloc(nbytes, C.byref(p)) == 0
    return p.value


def _read_i32(ops, lib, ptr, n):
    out = np.empty(n, np.int32)
    assert lib.sf_memcpy(C.c_void_p(out.ctypes.data), C.c_void_p(ptr), 4 * n, 1, None) == 0
    return out


def test_flag_store_then_wait(gpu, ops):
    from scaffolding_b200._lib import lib
    from tests.gpu_util import device_error
    flags = _ipc_alloc(lib, 64)
    assert np.array_equal(_read_i32(ops, lib, flags, 16), np.zeros(16, np.int32))  # zeroed
    ptrs = (C.c_void_p * 3)(flags, flags + 8, flags + 12)
    assert lib.sf_flag_store(ptrs, 3, 5, None) == 0
    # flags 0, 2, 3 hold 5; flag 1 (skipped) holds 0
    assert lib.sf_flag_wait(C.c_void_p(flags), 4, 1, 1, 5, 0, None) == 0
    # stride 2 reads flags 0 and 2
    assert lib.sf_flag_wait(C.c_void_p(flags), 2, 2, -1, 4, 0, None) == 0
    assert lib.sf_device_synchronize() == 0
    assert list(_read_i32(ops, lib, flags, 4)) == [5, 0, 5, 5]
    assert device_error(0) == 0
    assert lib.sf_ipc_free(C.c_void_p(flags)) == 0


def test_flag_wait_expires_with_status(gpu, ops):
    """A flag nothing stores: the bounded wait gives up after its limit,
    records 7 and the stream goes on with the next operation."""
    from scaffolding_b200._lib import lib
    flags = _ipc_alloc(lib, 16)
    assert lib.sf_flag_wait(C.c_void_p(flags), 1, 1, -1, 1, 1_000_000, None) == 0
    ptrs = (C.c_void_p * 1)(flags + 4)
    assert lib.sf_flag_store(ptrs, 1, 9, None) == 0  # runs after the expired wait
    assert lib.sf_device_synchronize() == 0
    code = C.c_int32()
    assert lib.sf_device_error_status(0, C.byref(code), 1) == 0
    assert code.value == 7
    assert list(_read_i32(ops, lib, flags, 2)) == [0, 9]
    assert lib.sf_device_error_status(0, C.byref(code), 0) == 0 and code.value == 0
    assert lib.sf_ipc_free(C.c_void_p(flags)) == 0


def test_ipc_handle_and_argument_checks(gpu, ops):
    from scaffolding_b200._lib import SF_ERR_INVALID_ARGUMENT, lib
    buf = _ipc_alloc(lib, 4096)
    h = (C.c_uint8 * 64)()
    assert lib.sf_ipc_handle(C.c_void_p(buf), h) == 0
    assert any(bytes(h))
    ptrs = (C.c_void_p * 9)(*([buf] * 9))
    assert lib.sf_flag_store(ptrs, 9, 1, None) == SF_ERR_INVALID_ARGUMENT  # at most 8
    bad = (C.c_void_p * 1)(buf + 2)
    assert lib.sf_flag_store(bad, 1, 1, None) == SF_ERR_INVALID_ARGUMENT  # misaligned
    assert lib.sf_flag_wait(C.c_void_p(buf), 1, 0, -1, 1, 0, None) == SF_ERR_INVALID_ARGUMENT
    assert lib.sf_flag_wait(C.c_void_p(buf), 1, 1, -1, 1, -5, None) == SF_ERR_INVALID_ARGUMENT
    assert lib.sf_ipc_alloc(0, C.byref(C.c_void_p())) == SF_ERR_INVALID_ARGUMENT
    assert lib.sf_ipc_free(C.c_void_p(buf)) == 0
