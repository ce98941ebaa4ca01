"""Helpers shared by the GPU parity tests (import only from -m gpu tests)."""
import ctypes as C

import numpy as np

from oracle import oracle as O

RTOL_16BIT = 1e-2     # bf16/fp16 (fp32 accumulate): per-element relative, with row-RMS floor
TAU_16BIT = 1e-2      # floor = TAU * rms(row of the exact result)
RTOL_FP32 = 1e-5      # fp32: relative Frobenius error


def np_dtype(name):
    from scaffolding_b200 import engine as E
    return {"f32": np.dtype(np.float32), "f16": np.dtype(np.float16), "bf16": E.bfloat16}[name]


def to_device(ops, x32, dt):
    """Round fp32 data to `dt` and upload; returns (GpuTensor, rounded fp32 copy)."""
    r = O.round_to(x32, dt)
    return ops.gputensor_from_numpy(r.astype(np_dtype(dt))), r


def to_host32(ops, gt):
    return ops.gputensor_to_numpy(gt).astype(np.float32)


KAPPA_16BIT = 1e-2    # floor = KAPPA * (|A| |B|)_ij when the absolute product is supplied


# Every per-element 16-bit check of the session, for the floor audit that
# tests/conftest.py prints at the end of the run.
FLOOR_AUDIT: list = []


def record_floor_stats(what, st):
    FLOOR_AUDIT.append((what, st))


def assert_close_16bit(out, ref, what="", absprod=None, allowance=None):
    ok, st = O.elementwise_rel_check(out, ref, rtol=RTOL_16BIT, tau=TAU_16BIT, absprod=absprod,
                                     kappa=KAPPA_16BIT, allowance=allowance)
    record_floor_stats(what, st)
    assert ok, f"{what}: {st}"
    return st


def assert_close_fp32(out, ref, what="", tol=RTOL_FP32):
    err = O.rel_frobenius(out, ref)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    assert err <= tol, f"{what}: rel Frobenius {err:.3e} > {tol:.1e}"
    return err


def device_error(dev=0):
    from scaffolding_b200 import engine as E
    return E.device_error_status(dev)


def kernel_override(kind):
    from scaffolding_b200._lib import check, lib
    check(lib.sf_set_kernel_override(kind), "sf_set_kernel_override")


def fp32_mode(mode):
    from scaffolding_b200._lib import check, lib
    check(lib.sf_set_fp32_mode(mode), "sf_set_fp32_mode")


def attn_oracle_opts():
    """oracle.flash_attention settings that restate the fused-attention
    kernel: 64-key blocks and integer row bases."""
    return {"block": 64, "integer_base": True}
