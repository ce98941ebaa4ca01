"""DiT stack (benchmark config 5) on the GPU against the oracle (-m gpu)."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import attn_oracle_opts, assert_close_16bit, np_dtype, to_host32

pytestmark = pytest.mark.gpu


def _weights(layers, hidden, seed):
    return [O.dit_weights(hidden=hidden, seed=seed + i, dtype="bf16", zero_bias=False)
            for i in range(layers)]


def _upload_x(ops, x):
    return ops.gputensor_from_numpy(x.astype(np_dtype("bf16")))


def _host(ops, t, shape=None):
    if shape is not None:
        t = ops.GpuTensor(t.buffer, shape, t.dtype, t.device_id)
    return to_host32(ops, t)


def _lin(x, w, b=None):
    """Oracle linear and the |x| |W|^T (+ |b|) error scale of its outputs."""
    y = O.linear(x, w, b)
    ap = O.abs_product(x, w)
    if b is not None:
        ap = ap + np.abs(b)
    return y, ap


def _attention_stages(ops, st, q, kv, B, N, H, D, what):
    """Stage-wise check of one attention pass held entirely in the S/P
    buffers (one query chunk per sample): S against Q K^T / sqrt(D) on the
    device's Q/K, P against the softmax of the device's S, O against the
    device's P times V."""
    Cw = H * D
    S = _host(ops, st.S, (B, H, N, N))
    P = _host(ops, st.P, (B, H, N, N))
    attn = _host(ops, st.attn)
    scale = np.float32(1.0 / np.sqrt(D))
    for b in range(B):
        for h in range(H):
            qh = q[b * N:(b + 1) * N, h * D:(h + 1) * D]
            kh = kv[b * N:(b + 1) * N, h * D:(h + 1) * D]
            vh = kv[b * N:(b + 1) * N, Cw + h * D:Cw + (h + 1) * D]
            assert_close_16bit(S[b, h], (qh @ kh.T) * scale, f"{what} S b{b}h{h}",
                               O.abs_product(qh, kh) * float(scale))
            assert_close_16bit(P[b, h], O.softmax_rows(S[b, h]), f"{what} P b{b}h{h}")
            assert_close_16bit(attn[b * N:(b + 1) * N, h * D:(h + 1) * D], P[b, h] @ vh,
                               f"{what} O b{b}h{h}", O.abs_product(P[b, h], vh.T))
    return attn


def test_stack_small_matches_oracle(gpu, ops):
    """Two layers, 2 samples x 200 tokens, 4 heads x 64.  Every stage -- the
    q / kv / out / ffn GEMMs, S = QK^T, P = softmax(S), O = PV -- is checked
    against the oracle on the device's own (identically rounded) stage inputs
    with the per-element bf16 bar; the two-layer output against the pure
    oracle composition with the aggregate bar (bf16 intermediates re-rounded
    at every stage make one-ulp flips unavoidable where outputs cancel).  A
    second stack with ragged query chunks of 64 must reproduce the attention
    bit for bit."""
    from scaffolding_b200 import dit
    B, N, Cw, H, L = 2, 200, 256, 4, 2
    D = Cw // H
    ws = _weights(L, Cw, 40)
    x = O.round_bf16(np.random.default_rng(41).standard_normal((B * N, Cw), dtype=np.float32))
    plan = dit.ShardPlan(B, N, 1, 0)
    st = dit.DitStack(plan, Cw, H, L, 0, chunk=256, weights=ws, fused=False)
    chunked = dit.DitStack(plan, Cw, H, L, 0, chunk=64, weights=ws, fused=False)
    gx = _upload_x(ops, x)
    cur_ptr, cur = gx.ptr, x
    for li in range(L):
        w = ws[li]
        st.qkv(li, cur_ptr)
        q, kv = _host(ops, st.q), _host(ops, st.kv_local)
        rq, aq = _lin(cur, w["qkv_w"][:Cw])
        rkv, akv = _lin(cur, w["qkv_w"][Cw:])
        assert_close_16bit(q, rq, f"L{li} q", aq)
        assert_close_16bit(kv, rkv, f"L{li} kv", akv)
        st._attention(None, None)
        attn = _attention_stages(ops, st, q, kv, B, N, H, D, f"L{li}")
        chunked.qkv(li, cur_ptr)
        chunked._attention(None, None)
        np.testing.assert_array_equal(_host(ops, chunked.attn), attn)
        out = st.y[li % 2]
        st.post(li, cur_ptr, out.ptr)
        h, f, y = _host(ops, st.h), _host(ops, st.f), _host(ops, out)
        rh, ah = _lin(attn, w["out_w"], w["out_b"])
        assert_close_16bit(h, rh + cur, f"L{li} out-proj", ah + np.abs(cur))
        ru, au = _lin(h, w["up_w"], w["up_b"])
        assert_close_16bit(f, O.gelu_tanh(ru), f"L{li} ffn-up", au)
        rd, ad = _lin(f, w["down_w"], w["down_b"])
        assert_close_16bit(y, rd + h, f"L{li} ffn-down", ad + np.abs(h))
        cur_ptr, cur = out.ptr, y
    ref = x
    for li in range(L):
        ref = O.dit_layer(ref, ws[li], B, H, D, chunk=64, dtype="bf16")
    assert O.rel_frobenius(cur, ref) < 1e-2
    # forward() runs the same launches end to end
    gy = st.forward(gx.ptr)
    assert gy == st.y[(L - 1) % 2].ptr
    np.testing.assert_array_equal(_host(ops, st.y[(L - 1) % 2]), cur)


@pytest.mark.parametrize("mode", ["unfused", "fused", "fused_split"])
def test_sliced_ranks_equal_whole_sample(gpu, ops, mode, monkeypatch):
    """Four emulated ranks holding half a sample each (K/V exchanged between
    the two ranks of a sample) reproduce the one-rank result: bit for bit
    when every row goes through the same kernels over the same keys (shards
    of 300 rows take the same GEMM path as the whole 1200-row batch; the
    fused attention computes each query row from its own scores only), and
    within the bf16 bar when the fused attention is split into the rank's
    own keys and the gathered ones (the overlapped exchange: another fp32
    summation order)."""
    from scaffolding_b200 import dit
    from scaffolding_b200 import engine as E
    fused = mode != "unfused"
    monkeypatch.setenv("SF_KV_OVERLAP", "1" if mode == "fused_split" else "0")
    B, N, Cw, H, chunk = 2, 600, 256, 4, 160
    ws = _weights(1, Cw, 50)
    x = O.round_bf16(np.random.default_rng(51).standard_normal((B * N, Cw), dtype=np.float32))
    gx = _upload_x(ops, x)
    whole = dit.DitStack(dit.ShardPlan(B, N, 1, 0), Cw, H, 1, 0, chunk=chunk, weights=ws,
                         fused=fused)
    whole.forward(gx.ptr)
    ref = _host(ops, whole.y[0])
    world = 4
    ranks = [dit.DitStack(dit.ShardPlan(B, N, world, r), Cw, H, 1, 0, chunk=chunk, weights=ws,
                          fused=fused)
             for r in range(world)]
    assert all(st.overlap == (mode == "fused_split") for st in ranks)
    outs = []
    for r, st in enumerate(ranks):
        st.qkv(0, gx.ptr + st.plan.row0 * Cw * 2)
    for st in ranks:  # emulate the K/V all-gather inside each sample's group
        p = st.plan
        peers = [o for o in ranks if o.plan.group_color == p.group_color]
        for q, o in enumerate(sorted(peers, key=lambda s: s.plan.rank)):
            nbytes = o.plan.m * 2 * Cw * 2
            E.memcpy(st.kv_full.ptr + q * nbytes, o.kv_local.ptr, nbytes, 2)
    for r, st in enumerate(ranks):
        st._attention(None, None)
        st.post(0, gx.ptr + st.plan.row0 * Cw * 2, st.y[0].ptr)
        outs.append(_host(ops, st.y[0]))
    got = np.concatenate(outs)
    if mode == "fused_split":
        # one layer: attention differs in fp32 order, then three bf16 linears
        assert np.abs(got - ref).max() <= 2.0 ** -5 * np.abs(ref).max()
        assert O.rel_frobenius(got, ref) < 2e-3
    else:
        np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("fused", [False, True])
def test_full_size_attention_sampled_rows(gpu, ops, fused):
    """Config 5 attention at full size (2 x 17776 tokens, 30 heads; unfused in
    9 query chunks of <= 2048, or fused): the oracle recomputes sampled query
    rows (including the ragged last chunk / block) from the device's own
    bf16 Q/K/V -- for the fused kernel in its blockwise form with the
    rounding-flip allowance."""
    from scaffolding_b200 import dit
    B, N, Cw, H = 2, 17776, 1920, 30
    D = Cw // H
    plan = dit.ShardPlan(B, N, 1, 0)
    st = dit.DitStack(plan, Cw, H, 1, 0, chunk=2048, seed=3, fused=fused)
    xt = ops._alloc((B * N, Cw), np_dtype("bf16"), 0)
    from scaffolding_b200._lib import lib
    assert lib.sf_fill_normal(C.c_void_p(xt.ptr), 2, B * N * Cw, 5, 0.0, 1.0, None) == 0
    st.qkv(0, xt.ptr)
    st._attention(None, None)
    q = to_host32(ops, st.q)
    kv = to_host32(ops, st.kv_full)
    attn = to_host32(ops, st.attn)
    rng = np.random.default_rng(0)
    rows = np.concatenate([rng.choice(B * N, 20, replace=False), [0, N - 1, N, 16384, N + 16390]])
    for r in rows:
        b = r // N
        keys = kv[b * N:(b + 1) * N]
        ref = np.empty(Cw, np.float32)
        allow = np.zeros(Cw)
        absprod = np.zeros(Cw)
        for h in range(H):
            qh, kh, vh = (q[r, h * D:(h + 1) * D][None], keys[:, h * D:(h + 1) * D],
                          keys[:, Cw + h * D:Cw + (h + 1) * D])
            s = (qh @ kh.T) * np.float32(0.125)
            if fused:
                o, a = O.flash_attention(qh, kh, vh, 0.125, return_allowance=True,
                                         **attn_oracle_opts())
                ref[h * D:(h + 1) * D], allow[h * D:(h + 1) * D] = o[0], a[0]
                absprod[h * D:(h + 1) * D] = O.abs_product(O.softmax_rows(s), vh.T)[0]
            else:
                p = O.round_bf16(O.softmax_rows(s))[0]
                ref[h * D:(h + 1) * D] = p @ vh
        if fused:
            assert_close_16bit(attn[r][None], ref[None], f"fused attention row {r}",
                               absprod=absprod[None], allowance=allow[None])
        else:
            assert_close_16bit(attn[r][None], ref[None], f"attention row {r}")
    assert np.isfinite(attn).all()


def test_stack_small_fused_matches_oracle(gpu, ops):
    """The fused-attention stack: the attention output of each layer against
    the blockwise oracle on the device's own Q/K/V (with the rounding-flip
    allowance), the linears stage-wise, and forward() bit for bit equal to
    the stage-by-stage run."""
    from scaffolding_b200 import dit
    B, N, Cw, H, L = 2, 200, 256, 4, 2
    D = Cw // H
    ws = _weights(L, Cw, 60)
    x = O.round_bf16(np.random.default_rng(61).standard_normal((B * N, Cw), dtype=np.float32))
    st = dit.DitStack(dit.ShardPlan(B, N, 1, 0), Cw, H, L, 0, weights=ws, fused=True)
    from scaffolding_b200 import engine as E
    n_attn = E.attention_launch_count(B, H, N, N)
    assert st.S is None and st.launches_per_forward() == (5 + n_attn) * L
    gx = _upload_x(ops, x)
    cur_ptr, cur = gx.ptr, x
    for li in range(L):
        w = ws[li]
        st.qkv(li, cur_ptr)
        q, kv = _host(ops, st.q), _host(ops, st.kv_local)
        st._attention(None, None)
        attn = _host(ops, st.attn)
        for b in range(B):
            for h in range(H):
                rs = slice(b * N, (b + 1) * N)
                qh, kh = q[rs, h * D:(h + 1) * D], kv[rs, h * D:(h + 1) * D]
                vh = kv[rs, Cw + h * D:Cw + (h + 1) * D]
                ref, allow = O.flash_attention(qh, kh, vh, 1.0 / np.sqrt(D), return_allowance=True,
                                               **attn_oracle_opts())
                p = O.softmax_rows((qh @ kh.T * np.float32(1.0 / np.sqrt(D))).astype(np.float32))
                assert_close_16bit(attn[rs, h * D:(h + 1) * D], ref, f"L{li} b{b} h{h}",
                                   absprod=O.abs_product(p, vh.T), allowance=allow)
        out = st.y[li % 2]
        st.post(li, cur_ptr, out.ptr)
        h_, y = _host(ops, st.h), _host(ops, out)
        rh, ah = _lin(attn, w["out_w"], w["out_b"])
        assert_close_16bit(h_, rh + cur, f"L{li} out-proj", ah + np.abs(cur))
        cur_ptr, cur = out.ptr, y
    gy = st.forward(gx.ptr)
    np.testing.assert_array_equal(_host(ops, st.y[(L - 1) % 2]), cur)
    assert gy == st.y[(L - 1) % 2].ptr
