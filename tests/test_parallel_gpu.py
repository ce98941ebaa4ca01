"""parallel.DataParallel on the device (-m gpu): scatter by peer copy,
replicas on every device, peer-to-peer gather (nn/parallel.py:45-290).

Rows of a linear stack do not depend on each other and every share here
takes the same GEMM kernel as the whole batch, so the split result equals
the one-device result bit for bit.  With one GPU the devices are [0, 0]:
the same scatter / replicate / gather path (device-to-device copies).
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import assert_close_16bit, device_error, np_dtype, to_device, to_host32

pytestmark = pytest.mark.gpu


def _devices(ops, n):
    have = ops.get_device_count()
    return list(range(n)) if have >= n else [0] * n


def _bits(ops, t):
    return ops.gputensor_to_numpy(t).view(np.uint16 if t.dtype.itemsize == 2 else np.uint32)


@pytest.mark.parametrize("n", [2, 3])
@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_data_parallel_linear_stack_bit_equal(gpu, ops, n, dt):
    from scaffolding_b200 import nn
    from scaffolding_b200.parallel import DataParallel
    rng = np.random.default_rng(20 + n)
    model = nn.Sequential(nn.Linear(256, 512, device=0, dtype=np_dtype(dt), rng=rng),
                          nn.Linear(512, 256, device=0, dtype=np_dtype(dt), rng=rng))
    gx, x = to_device(ops, rng.standard_normal((2 * 1030, 256), dtype=np.float32), dt)
    whole = model(gx)
    dp = DataParallel(model, device_ids=_devices(ops, n))
    split = dp(gx)
    assert split.shape == whole.shape and split.device_id == 0
    assert np.array_equal(_bits(ops, split), _bits(ops, whole))
    again = dp(gx)  # replicas and parameter copies are cached
    assert np.array_equal(_bits(ops, again), _bits(ops, whole))
    assert device_error(0) == 0


def test_data_parallel_dit_block(gpu, ops):
    """The config-4 block linears through DataParallel at M = 35552: every
    output row against the single-device block within the bf16 bar (shares of
    35552 / n rows may take a different GEMM tile shape than the whole), and
    sampled rows against the oracle chain."""
    from scaffolding_b200 import dit
    from scaffolding_b200.parallel import DataParallel
    n = min(4, max(2, ops.get_device_count()))
    M, C = dit.BATCH * dit.TOKENS, dit.HIDDEN
    w = O.dit_weights(C, seed=8)
    x = O.round_bf16(np.random.default_rng(81).standard_normal((M, C), dtype=np.float32))
    gx = ops.gputensor_from_numpy(x.astype(np_dtype("bf16")))
    block = dit.DitBlock(w, 0)
    whole = to_host32(ops, block(gx))
    got = to_host32(ops, DataParallel(block, device_ids=_devices(ops, n))(gx))
    rows = np.random.default_rng(82).choice(M, 48, replace=False)
    assert_close_16bit(got[rows], whole[rows], f"DataParallel DiT block ({n} shares)")
    assert O.rel_frobenius(got, whole) < 1e-3
    ref = O.dit_block_linears(x[rows], w)
    assert O.rel_frobenius(got[rows], ref) < 1e-2
    assert device_error(0) == 0
