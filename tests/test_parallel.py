"""Host logic of parallel.DataParallel on CPU: the row split rule of the
reference's scatter (nn/parallel.py:118-131) and, on two gloo ranks standing
in for two devices, scatter -> per-rank forward -> gather in device order
reproducing the unsplit result.  No GPU."""
import os
import tempfile

import numpy as np
import pytest
import torch.distributed as td
import torch.multiprocessing as mp

from oracle import oracle as O


def _reference_scatter(batch, n):
    """The reference's scatter loop, restated: chunk = ceil(batch / n); device
    i gets [i*chunk, min(i*chunk + chunk, batch)), nothing when it starts past
    the batch."""
    chunk = (batch + n - 1) // n
    out = []
    for i in range(n):
        start = i * chunk
        if start >= batch:
            out.append(None)
            continue
        out.append((start, min(start + chunk, batch)))
    return out


@pytest.mark.parametrize("batch", [1, 2, 5, 7, 8, 35552, 17777])
@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_split_rows_matches_reference_scatter(batch, n):
    from scaffolding_b200.parallel import split_rows
    got = split_rows(batch, n)
    ref = _reference_scatter(batch, n)
    assert len(got) == n
    for g, r in zip(got, ref):
        if r is None:
            assert g[0] == g[1]  # empty range: the device gets no rows
        else:
            assert g == r
    covered = np.zeros(batch, np.int32)
    for a, b in got:
        covered[a:b] += 1
    assert (covered == 1).all()


def _rank_main(rank, world, batch, init_file, q):
    import torch

    from scaffolding_b200.parallel import split_rows
    td.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    rng = np.random.default_rng(8)
    C = 48
    x = rng.standard_normal((batch, C), dtype=np.float32)
    w1 = rng.standard_normal((2 * C, C), dtype=np.float32) * np.float32(0.1)
    w2 = rng.standard_normal((C, 2 * C), dtype=np.float32) * np.float32(0.1)
    r0, r1 = split_rows(batch, world)[rank]
    y = O.linear(O.silu(O.linear(x[r0:r1], w1)), w2)  # this "device's" replica forward
    # gather in device order; ragged shares travel padded to the chunk size
    chunk = (batch + world - 1) // world
    pad = np.zeros((chunk, C), np.float32)
    pad[:r1 - r0] = y
    parts = [torch.empty((chunk, C)) for _ in range(world)]
    td.all_gather(parts, torch.from_numpy(pad))
    if rank == 0:
        full = np.concatenate([p.numpy()[:b - a] for p, (a, b) in zip(parts, split_rows(batch, world))])
        ref = O.linear(O.silu(O.linear(x, w1)), w2)
        q.put(bool(np.array_equal(full, ref)))
    td.destroy_process_group()


@pytest.mark.parametrize("batch", [10, 7])
def test_scatter_forward_gather_on_two_ranks(batch):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(2, batch, os.path.join(d, "init"), q), nprocs=2,
                           join=True, start_method="spawn")
    assert q.get()
