"""Host-side logic of the token-sharded path on CPU ranks (gloo, world 2).

Each rank owns the rows ShardPlan assigns it, computes its part of one DiT
layer with the NumPy oracle, exchanges K/V inside its sample's group and
all-gathers the output -- the same plan and gather order the GPU path uses.
Rank 0 checks the result against the unsharded oracle layer.  No GPU.
"""
import os
import tempfile

import numpy as np
import pytest
import torch.distributed as td
import torch.multiprocessing as mp

from oracle import oracle as O


def _rank_main(rank, world, batch, tokens, init_file, q):
    import torch

    from scaffolding_b200.dit import ShardPlan
    td.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    Cw, H = 64, 2
    D = Cw // H
    w = O.dit_weights(hidden=Cw, seed=5, dtype="f32", zero_bias=False)
    x = np.random.default_rng(6).standard_normal((batch * tokens, Cw), dtype=np.float32)
    plan = ShardPlan(batch, tokens, world, rank)
    r0, r1 = plan.rows()
    xl = x[r0:r1]
    qkv_l = O.linear(xl, w["qkv_w"])
    q_l, kv_l = qkv_l[:, :Cw], np.ascontiguousarray(qkv_l[:, Cw:])
    # every rank creates every K/V group, in the same order (new_group is collective)
    colors = sorted({ShardPlan(batch, tokens, world, r).group_color for r in range(world)})
    groups = {c: [r for r in range(world) if ShardPlan(batch, tokens, world, r).group_color == c]
              for c in colors}
    handles = {c: td.new_group(ranks=groups[c]) for c in colors}
    if plan.kv_exchange:
        ranks = groups[plan.group_color]
        parts = [torch.empty_like(torch.from_numpy(kv_l)) for _ in ranks]
        td.all_gather(parts, torch.from_numpy(kv_l), group=handles[plan.group_color])
        kv_full = torch.cat(parts).numpy()
    else:
        kv_full = kv_l
    attn = np.empty_like(xl)
    for s in range(plan.samples_per_rank):
        if plan.whole_samples:
            qs = slice(s * tokens, (s + 1) * tokens)
            keys = kv_full[s * tokens:(s + 1) * tokens]
        else:
            qs = slice(0, plan.m)
            keys = kv_full
        for h in range(H):
            attn[qs, h * D:(h + 1) * D] = O.sdpa(q_l[qs, h * D:(h + 1) * D][None],
                                                 keys[:, h * D:(h + 1) * D][None],
                                                 keys[:, Cw + h * D:Cw + (h + 1) * D][None])[0]
    hh = O.linear(attn, w["out_w"], w["out_b"]) + xl
    y_l = O.linear(O.gelu_tanh(O.linear(hh, w["up_w"], w["up_b"])), w["down_w"], w["down_b"]) + hh
    parts = [torch.empty_like(torch.from_numpy(y_l)) for _ in range(world)]
    td.all_gather(parts, torch.from_numpy(np.ascontiguousarray(y_l)))
    if rank == 0:
        full = torch.cat(parts).numpy()
        ref = O.dit_layer(x, w, batch, H, D, chunk=tokens, dtype="f32")
        q.put(float(O.rel_frobenius(full, ref)))
    td.destroy_process_group()


@pytest.mark.parametrize("batch,tokens", [(2, 48), (1, 48)])
def test_sharded_layer_matches_unsharded(batch, tokens):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(2, batch, tokens, os.path.join(d, "init"), q), nprocs=2,
                           join=True, start_method="spawn")
    err = q.get()
    assert err < 1e-5, err


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plan_covers_rows_once(world):
    from scaffolding_b200.dit import ShardPlan
    B, N = 2, 17776
    seen = np.zeros(B * N, np.int32)
    groups = {}
    for r in range(world):
        p = ShardPlan(B, N, world, r)
        a, b = p.rows()
        seen[a:b] += 1
        groups.setdefault(p.group_color, []).append(r)
        if p.kv_exchange:
            assert p.row0 // N == p.sample0 and (p.row0 + p.m - 1) // N == p.sample0
    assert (seen == 1).all()
    if world > B:
        assert all(len(v) == world // B for v in groups.values())
    with pytest.raises(ValueError):
        ShardPlan(2, 17776, 3, 0)
