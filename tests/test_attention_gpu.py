"""Row softmax and the attention products (QK^T, softmax, P.V) on the GPU
against the oracle (-m gpu)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import (assert_close_16bit, assert_close_fp32, attn_oracle_opts, np_dtype,
                            to_device, to_host32)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cols", [1, 300, 1500, 4097, 17776, 40000])
@pytest.mark.parametrize("out_dt", ["f32", "bf16"])
def test_softmax_rows(gpu, ops, cols, out_dt):
    from scaffolding_b200 import engine as E
    rng = np.random.default_rng(cols)
    rows = 37
    x = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(6)
    gx = ops.gputensor_from_numpy(x)
    y = ops._alloc((rows, cols), np_dtype(out_dt), 0)
    E.softmax_rows(gx.ptr, 0, cols, y.ptr, E.dtype_code(np_dtype(out_dt)), cols, rows, cols, 0.125)
    ref = O.softmax_rows(x * np.float32(0.125))
    out = to_host32(ops, y)
    if out_dt == "f32":
        np.testing.assert_allclose(out, ref, rtol=2e-6, atol=1e-9)
        np.testing.assert_allclose(out.sum(axis=1), 1.0, rtol=1e-5)
    else:
        assert_close_16bit(out, ref, "softmax bf16")


def test_dev_softmax_golden(gpu, ops, golden):
    for tag in ("sm1", "sm2"):
        y = ops.gputensor_to_numpy(ops.dev_softmax(ops.gputensor_from_numpy(golden[f"{tag}_x"])))
        np.testing.assert_allclose(y, golden[f"{tag}_y"], rtol=2e-6, atol=1e-9)


def test_sdpa_fp32_golden(gpu, ops, golden):
    from scaffolding_b200.nn import functional as F
    q, k, v = (ops.gputensor_from_numpy(golden[f"sdpa_{s}"]) for s in "qkv")
    o = ops.gputensor_to_numpy(F.scaled_dot_product_attention(q, k, v))
    assert_close_fp32(o, golden["sdpa_o"], "sdpa fp32")


def test_sdpa_bf16_golden(gpu, ops, golden):
    """bf16 SDPA (head_dim 64: the fused kernel).  Per-element bar (1e-2) per
    (batch, head) against the oracle restating the fused kernel's blockwise
    softmax on identically rounded Q, K, V (with its rounding-flip allowance);
    against the reference's fp32-P output the bf16 rounding of P is visible
    on outputs that cancel to ~0, so that comparison uses the aggregate bar."""
    from scaffolding_b200.nn import functional as F
    bf = np_dtype("bf16")
    qh, kh, vh = (golden[f"sdpa8_{s}"] for s in "qkv")
    q, k, v = (ops.gputensor_from_numpy(t.astype(bf)) for t in (qh, kh, vh))
    o = to_host32(ops, F.scaled_dot_product_attention(q, k, v, scale=0.125))
    for idx in np.ndindex(*qh.shape[:-2]):
        ref, allow = O.flash_attention(qh[idx], kh[idx], vh[idx], 0.125, return_allowance=True,
                                       **attn_oracle_opts())
        p = O.softmax_rows((qh[idx] @ kh[idx].T * np.float32(0.125)).astype(np.float32))
        _check_attn(o[idx], ref, O.abs_product(p, vh[idx].T), allow, f"sdpa bf16 {idx}")
    assert O.rel_frobenius(o, golden["sdpa8_o"]) < 1e-2


def test_dev_muls_silu_gelu(gpu, ops, golden):
    z = golden["act_z"]
    gz = ops.gputensor_from_numpy(z)
    np.testing.assert_allclose(ops.gputensor_to_numpy(ops.dev_silu(gz)), golden["act_silu"],
                               rtol=2e-6, atol=1e-7)
    # 1 + tanh(u) cancels for u << 0: the reference's own formula carries an
    # absolute error of ~|z| * eps(fp32) there, hence the absolute floor.
    np.testing.assert_allclose(ops.gputensor_to_numpy(ops.dev_gelu(gz)), golden["act_gelu"],
                               rtol=2e-6, atol=1e-6)
    np.testing.assert_array_equal(ops.gputensor_to_numpy(ops.dev_muls(gz, 0.125)), z * np.float32(0.125))


# Fused attention rounds the unnormalised block probabilities 2^(c s - m)
# to 16 bits as the P.V operand; the oracle restates that (flash_attention).
# Scores summed in another order can move a p across a 16-bit rounding
# midpoint; flash_attention's allowance adds, per output, the change such a
# flip could cause for every p within 2^-12 of a midpoint.
def _check_attn(out, ref, absprod, allowance, what):
    assert_close_16bit(out, ref, what, absprod=absprod, allowance=allowance)


def _fused(ops, batch, heads, q_len, kv_len, q, k, v, ldq, ldk, ldv, q_bs, k_bs, v_bs, scale,
           dt="bf16"):
    """Run sf_attention_fwd on device copies; returns O as fp32 [batch*q_len, heads*64]."""
    from scaffolding_b200 import engine as E
    o = ops._alloc((batch * q_len, heads * 64), np_dtype(dt), 0)
    E.attention(batch, heads, q_len, kv_len, q.ptr, ldq, q_bs, k.ptr, ldk, k_bs, v.ptr, ldv, v_bs,
                o.ptr, heads * 64, q_len * heads * 64, scale, dtype=E.dtype_code(np_dtype(dt)))
    return to_host32(ops, o)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("batch,tokens,heads", [(2, 300, 3), (1, 128, 1), (1, 2048, 2), (2, 1000, 4)])
def test_fused_attention_dit_layout(gpu, ops, dt, batch, tokens, heads):
    """Fused attention reading Q, K, V in place from a fused [B*N, 3C] QKV
    activation (the DiT layout), ragged last query and key blocks; against
    the oracle's exact-softmax attention with the |P||V| error floor."""
    from tests.gpu_util import device_error
    rng = np.random.default_rng(tokens + heads)
    C = heads * 64
    qkv32 = rng.standard_normal((batch * tokens, 3 * C), dtype=np.float32)
    g, qkv = to_device(ops, qkv32, dt)
    base = g.ptr
    out = _fused(ops, batch, heads, tokens, tokens,
                 type("P", (), {"ptr": base})(), type("P", (), {"ptr": base + C * 2})(),
                 type("P", (), {"ptr": base + 2 * C * 2})(), 3 * C, 3 * C, 3 * C,
                 tokens * 3 * C, tokens * 3 * C, tokens * 3 * C, 0.125, dt)
    for b in range(batch):
        X = qkv[b * tokens:(b + 1) * tokens]
        for h in range(heads):
            q, k, v = (X[:, s * C + h * 64:s * C + (h + 1) * 64] for s in range(3))
            ref, allow = O.flash_attention(q, k, v, 0.125, p_dtype=dt, return_allowance=True,
                                           **attn_oracle_opts())
            p = O.softmax_rows((q @ k.T * np.float32(0.125)).astype(np.float32))
            _check_attn(out[b * tokens:(b + 1) * tokens, h * 64:(h + 1) * 64], ref,
                        O.abs_product(p, v.T), allow, f"fused {dt} B={batch} N={tokens} b{b} h{h}")
    assert device_error(0) == 0


def test_fused_attention_separate_qkv_lengths(gpu, ops):
    """Separate Q / K / V buffers, q_len != kv_len (ragged both), large
    logits (online-softmax rescaling), against per-head oracle SDPA."""
    from tests.gpu_util import device_error
    rng = np.random.default_rng(5)
    B, H, Lq, Lk = 2, 2, 200, 517
    q32 = rng.standard_normal((B, Lq, H * 64), dtype=np.float32) * np.float32(3)
    k32 = rng.standard_normal((B, Lk, H * 64), dtype=np.float32) * np.float32(3)
    v32 = rng.standard_normal((B, Lk, H * 64), dtype=np.float32)
    gq, q = to_device(ops, q32, "bf16")
    gk, k = to_device(ops, k32, "bf16")
    gv, v = to_device(ops, v32, "bf16")
    out = _fused(ops, B, H, Lq, Lk, gq, gk, gv, H * 64, H * 64, H * 64, Lq * H * 64, Lk * H * 64,
                 Lk * H * 64, 0.125)
    for b in range(B):
        for h in range(H):
            sl = slice(h * 64, (h + 1) * 64)
            s = q[b][:, sl] @ k[b][:, sl].T * np.float32(0.125)
            p = O.softmax_rows(s.astype(np.float32))
            ref, allow = O.flash_attention(q[b][:, sl], k[b][:, sl], v[b][:, sl], 0.125,
                                           return_allowance=True, **attn_oracle_opts())
            ap = O.abs_product(p, v[b][:, sl].T)
            _check_attn(out[b * Lq:(b + 1) * Lq, sl], ref, ap, allow, f"b{b} h{h}")
    assert device_error(0) == 0


@pytest.mark.parametrize("split", ["2", "0"])
@pytest.mark.parametrize("B,H,Lq,Lk", [(1, 2, 300, 641), (1, 3, 128, 64), (2, 1, 129, 700),
                                      (1, 2, 257, 65), (2, 3, 700, 1500)])
def test_fused_attention_grid_shapes(gpu, ops, monkeypatch, B, H, Lq, Lk, split):
    """Ragged query units (one or both tiles of a 256-row unit holding rows,
    the second tile a single row), ragged and single key blocks, q_len !=
    kv_len and large logits, against the oracle restating the kernel's key
    block and row bases; with the last wave run as a stream-K tail
    (SF_ATTN_SPLIT=2 forces it; at 2x3x700x1500 its 27 CTAs of 16 key blocks
    split every unit, so CTAs run two segments and a merge kernel combines
    the parts) and with one CTA per unit (SF_ATTN_SPLIT=0)."""
    from scaffolding_b200 import engine as E
    from tests.gpu_util import device_error
    monkeypatch.setenv("SF_ATTN_SPLIT", split)
    if split == "0" or Lk <= 64:
        assert E.attention_launch_count(B, H, Lq, Lk) == 1
    else:
        assert E.attention_launch_count(B, H, Lq, Lk) == 2
    rng = np.random.default_rng(Lq * 7 + Lk)
    q32 = rng.standard_normal((B, Lq, H * 64), dtype=np.float32) * np.float32(3)
    k32 = rng.standard_normal((B, Lk, H * 64), dtype=np.float32) * np.float32(3)
    v32 = rng.standard_normal((B, Lk, H * 64), dtype=np.float32)
    gq, q = to_device(ops, q32, "bf16")
    gk, k = to_device(ops, k32, "bf16")
    gv, v = to_device(ops, v32, "bf16")
    out = _fused(ops, B, H, Lq, Lk, gq, gk, gv, H * 64, H * 64, H * 64, Lq * H * 64, Lk * H * 64,
                 Lk * H * 64, 0.125)
    for b in range(B):
        for h in range(H):
            sl = slice(h * 64, (h + 1) * 64)
            p = O.softmax_rows((q[b][:, sl] @ k[b][:, sl].T * np.float32(0.125)).astype(np.float32))
            ref, allow = O.flash_attention(q[b][:, sl], k[b][:, sl], v[b][:, sl], 0.125,
                                           return_allowance=True, **attn_oracle_opts())
            _check_attn(out[b * Lq:(b + 1) * Lq, sl], ref, O.abs_product(p, v[b][:, sl].T), allow,
                        f"B{B} H{H} {Lq}x{Lk} b{b} h{h} split={split}")
    assert device_error(0) == 0


def test_fused_attention_two_streams(gpu, ops, monkeypatch):
    """Stream-K tail calls on two streams at once (each stream has its own
    workspace for the parts) give the same bits as the same calls run one by
    one."""
    import ctypes as C

    from scaffolding_b200 import engine as E
    from scaffolding_b200._lib import lib
    from tests.gpu_util import device_error
    monkeypatch.setenv("SF_ATTN_SPLIT", "2")
    B, H, L = 1, 3, 700
    W = H * 64
    assert E.attention_launch_count(B, H, L, L) == 2
    bf = np_dtype("bf16")
    ins, outs = [], []
    for seed in (71, 72):
        rng = np.random.default_rng(seed)
        g, _ = to_device(ops, rng.standard_normal((L, 3 * W), dtype=np.float32), "bf16")
        ins.append(g)
        outs.append([ops._alloc((L, W), bf, 0), ops._alloc((L, W), bf, 0)])

    def call(i, o, stream):
        base = ins[i].ptr
        E.attention(B, H, L, L, base, 3 * W, L * 3 * W, base + W * 2, 3 * W, L * 3 * W,
                    base + 2 * W * 2, 3 * W, L * 3 * W, o.ptr, W, L * W, 0.125, stream=stream)

    for i in (0, 1):  # one by one on the default stream
        call(i, outs[i][0], None)
    E.check(lib.sf_device_synchronize(), "sync")
    streams = []
    for _ in (0, 1):
        sp = C.c_void_p()
        E.check(lib.sf_stream_create(0, 1, C.byref(sp)), "sf_stream_create")
        streams.append(sp.value)
    for _ in range(3):  # interleaved on two streams
        for i in (0, 1):
            call(i, outs[i][1], streams[i])
    E.check(lib.sf_device_synchronize(), "sync")
    for i in (0, 1):
        a, b = (ops.gputensor_to_numpy(t).view(np.uint16) for t in outs[i])
        assert np.array_equal(a, b), f"stream {i}"
    for sp in streams:
        lib.sf_stream_destroy(C.c_void_p(sp))
    assert device_error(0) == 0


def test_fused_attention_rejects_bad_arguments(gpu, ops):
    from scaffolding_b200._lib import SF_ERR_INVALID_ARGUMENT, SF_ERR_UNSUPPORTED, lib
    import ctypes as C
    buf = ops._alloc((256, 3 * 64), np_dtype("bf16"), 0)
    p = C.c_void_p(buf.ptr)
    # head_dim other than 64
    assert lib.sf_attention_fwd(1, 1, 8, 8, 32, p, 192, 0, p, 192, 0, p, 192, 0, p, 192, 0,
                                1.0, 2, None) == SF_ERR_UNSUPPORTED
    # misaligned stride (ld * 2 bytes not a multiple of 16)
    assert lib.sf_attention_fwd(1, 1, 8, 8, 64, p, 65, 0, p, 192, 0, p, 192, 0, p, 192, 0,
                                1.0, 2, None) == SF_ERR_INVALID_ARGUMENT
    # zero keys
    assert lib.sf_attention_fwd(1, 1, 8, 0, 64, p, 192, 0, p, 192, 0, p, 192, 0, p, 192, 0,
                                1.0, 2, None) == SF_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("lo,hi,Lq,Lk,split", [(300, 500, 200, 700, "1"), (0, 256, 200, 700, "1"),
                                              (520, 700, 200, 700, "1"),
                                              (1000, 3200, 300, 5000, "2"),
                                              (0, 2400, 300, 5000, "2"),
                                              (2600, 5000, 300, 5000, "2")])
def test_fused_attention_split_keys_merge(gpu, ops, monkeypatch, lo, hi, Lq, Lk, split):
    """Two-pass attention as the sharded DiT stack runs it: keys [lo, hi)
    from their own buffer (partial result written), then every other key
    (skip [lo, hi)) merged with it.  Equals the one-pass kernel up to fp32
    summation order, and the oracle with its usual bar.  The 5000-key cases
    force the stream-K tail (SF_ATTN_SPLIT=2) on all three calls: tail CTAs
    of 16 key blocks split units whose keys straddle the skipped range, and
    the merge kernel writes the partial result (mode 1) or merges it
    (mode 2)."""
    import ctypes as C

    from scaffolding_b200 import engine as E
    from tests.gpu_util import device_error
    monkeypatch.setenv("SF_ATTN_SPLIT", split)
    rng = np.random.default_rng(lo + hi)
    B, H = 2, 3
    if split == "2":
        assert E.attention_launch_count(B, H, Lq, hi - lo) == 2
        assert E.attention_launch_count(B, H, Lq, Lk, lo, hi) == 2
    W = H * 64
    gq, q = to_device(ops, rng.standard_normal((B, Lq, W), dtype=np.float32), "bf16")
    gk, k = to_device(ops, rng.standard_normal((B, Lk, W), dtype=np.float32), "bf16")
    gv, v = to_device(ops, rng.standard_normal((B, Lk, W), dtype=np.float32), "bf16")
    bf = np_dtype("bf16")
    one = ops._alloc((B * Lq, W), bf, 0)
    E.attention(B, H, Lq, Lk, gq.ptr, W, Lq * W, gk.ptr, W, Lk * W, gv.ptr, W, Lk * W,
                one.ptr, W, Lq * W, 0.125)
    part_o = ops._alloc((B * Lq * H * 64,), np.float32, 0)
    part_ml = ops._alloc((B * Lq * H * 2,), np.float32, 0)
    two = ops._alloc((B * Lq, W), bf, 0)
    off = lo * W * 2  # the slice [lo, hi) as its own K/V buffer
    E.attention_partial(B, H, Lq, hi - lo, gq.ptr, W, Lq * W, gk.ptr + off, W, Lk * W,
                        gv.ptr + off, W, Lk * W, two.ptr, W, Lq * W, 0.125, hi - lo, hi - lo,
                        part_o.ptr, part_ml.ptr, 1)
    E.attention_partial(B, H, Lq, Lk, gq.ptr, W, Lq * W, gk.ptr, W, Lk * W, gv.ptr, W, Lk * W,
                        two.ptr, W, Lq * W, 0.125, lo, hi, part_o.ptr, part_ml.ptr, 2)
    a, b2 = to_host32(ops, one), to_host32(ops, two)
    # one 16-bit ulp at most where the two summation orders round differently
    assert np.abs(a - b2).max() <= 2.0 ** -7 * np.abs(a).max()
    for b in range(B):
        for h in range(H):
            sl = slice(h * 64, (h + 1) * 64)
            ref, allow = O.flash_attention(q[b][:, sl], k[b][:, sl], v[b][:, sl], 0.125,
                                           return_allowance=True, **attn_oracle_opts())
            p = O.softmax_rows((q[b][:, sl] @ k[b][:, sl].T * np.float32(0.125)).astype(np.float32))
            _check_attn(b2[b * Lq:(b + 1) * Lq, sl], ref, O.abs_product(p, v[b][:, sl].T), allow,
                        f"split [{lo},{hi}) b{b} h{h}")
    assert device_error(0) == 0
    from scaffolding_b200._lib import SF_ERR_INVALID_ARGUMENT, lib
    assert lib.sf_attention_fwd_partial(B, H, Lq, Lk, 64, C.c_void_p(gq.ptr), W, Lq * W,
                                        C.c_void_p(gk.ptr), W, Lk * W, C.c_void_p(gv.ptr), W,
                                        Lk * W, C.c_void_p(two.ptr), W, Lq * W, 0.125, 2, 10, 1,
                                        None, None, 1, None) == SF_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("jump", [12.0, 60.0, 140.0, 250.0])
def test_fused_attention_base_raises(gpu, ops, dt, jump):
    """The row base after the first key block: rows whose later scores climb
    above it, one key `jump` log2 units above everything before it (blocks
    after the first whose p sum reaches 2^8 raise the base by a power of two
    read off the sum; a sum past 2^120, 2^15 for f16 P, or infinite takes the
    row max and recomputes), and a steady climb that raises the base in
    block after block.  Against the oracle's blockwise restatement."""
    from tests.gpu_util import device_error
    rng = np.random.default_rng(int(jump) + (7 if dt == "f16" else 0))
    Lq, Lk, scale = 130, 700, 0.125
    c = scale * 1.4426950408889634
    q32 = rng.standard_normal((Lq, 64), dtype=np.float32) * np.float32(0.5)
    k32 = rng.standard_normal((Lk, 64), dtype=np.float32) * np.float32(0.2)
    v32 = rng.standard_normal((Lk, 64), dtype=np.float32)
    q32[:, 0] = 8.0
    # rows 0..63: one key (index 333, block 5) `jump` log2 units up
    k32[333, 0] = np.float32(jump / c / 8.0)
    # rows 64..129: a steady climb through every block (another head)
    q2 = q32.copy()
    k2 = k32.copy()
    k2[:, 0] = np.linspace(0.0, 40.0 / c / 8.0, Lk, dtype=np.float32)
    k2[333, 0] = 0.0
    qh = np.concatenate([q32, q2], axis=1)       # [Lq, 2 heads * 64]
    kh = np.concatenate([k32, k2], axis=1)
    vh = np.concatenate([v32, v32[::-1]], axis=1)
    gq, q = to_device(ops, qh, dt)
    gk, k = to_device(ops, kh, dt)
    gv, v = to_device(ops, vh, dt)
    out = _fused(ops, 1, 2, Lq, Lk, gq, gk, gv, 128, 128, 128, Lq * 128, Lk * 128, Lk * 128, scale,
                 dt=dt)
    for h in range(2):
        sl = slice(h * 64, (h + 1) * 64)
        p = O.softmax_rows((q[:, sl] @ k[:, sl].T * np.float32(scale)).astype(np.float32))
        ref, allow = O.flash_attention(q[:, sl], k[:, sl], v[:, sl], scale, p_dtype=dt,
                                       return_allowance=True, **attn_oracle_opts())
        assert np.isfinite(out[:, sl]).all()
        _check_attn(out[:, sl], ref, O.abs_product(p, v[:, sl].T), allow,
                    f"{dt} jump {jump} head {h}")
    assert device_error(0) == 0


def test_fused_attention_graph_keeps_captured_workspace(gpu, ops, monkeypatch):
    """A stream-K attention call captured into a CUDA graph keeps using the
    tail workspace it was captured with: a later direct call on the same
    stream that needs a larger workspace retires the captured buffer instead
    of freeing it, so replaying the graph afterwards gives the same bits as
    the direct call of the captured shape."""
    import ctypes as C

    from scaffolding_b200 import engine as E
    from scaffolding_b200._lib import lib
    from tests.gpu_util import device_error
    monkeypatch.setenv("SF_ATTN_SPLIT", "2")
    bf = np_dtype("bf16")
    rng = np.random.default_rng(91)

    def inputs(B, H, L):
        W = H * 64
        g, _ = to_device(ops, rng.standard_normal((B * L, 3 * W), dtype=np.float32), "bf16")
        return g, W

    def call(g, B, H, L, W, out, stream):
        base = g.ptr
        E.attention(B, H, L, L, base, 3 * W, L * 3 * W, base + W * 2, 3 * W, L * 3 * W,
                    base + 2 * W * 2, 3 * W, L * 3 * W, out.ptr, W, L * W, 0.125, stream=stream)

    sp = C.c_void_p()
    assert lib.sf_stream_create(0, 1, C.byref(sp)) == 0
    s = sp.value
    # small shape: 6 units, all in the tail (a small workspace)
    Ba, Ha, La = 1, 2, 700
    ga, Wa = inputs(Ba, Ha, La)
    assert E.attention_launch_count(Ba, Ha, La, La) == 2
    direct = ops._alloc((Ba * La, Wa), bf, 0)
    replay = ops._alloc((Ba * La, Wa), bf, 0)
    call(ga, Ba, Ha, La, Wa, direct, s)  # sizes the workspace
    E.stream_sync(s)
    g = C.c_void_p()
    assert lib.sf_graph_begin(C.c_void_p(s)) == 0
    call(ga, Ba, Ha, La, Wa, replay, s)
    assert lib.sf_graph_end(C.c_void_p(s), C.byref(g)) == 0
    # a larger shape on the same stream grows the workspace (128 units, 256 tail CTAs)
    Bb, Hb, Lb = 2, 8, 2000
    gb, Wb = inputs(Bb, Hb, Lb)
    big = ops._alloc((Bb * Lb, Wb), bf, 0)
    call(gb, Bb, Hb, Lb, Wb, big, s)
    E.stream_sync(s)
    for _ in range(2):
        assert lib.sf_graph_launch(g, C.c_void_p(s)) == 0
    E.stream_sync(s)
    assert lib.sf_graph_destroy(g) == 0
    lib.sf_stream_destroy(C.c_void_p(s))
    a = ops.gputensor_to_numpy(direct).view(np.uint16)
    b = ops.gputensor_to_numpy(replay).view(np.uint16)
    assert np.array_equal(a, b)
    assert device_error(0) == 0


def test_fused_attention_full_wave_plus_tail(gpu, ops):
    """More units than CTA slots: a full wave of whole units (one kernel,
    launched behind the tail kernel) plus a stream-K tail of 34 units, whose
    split parts the merge kernel combines after both.  The tail units are the
    last ones (the last heads); every row of those heads is checked against
    the oracle, and one head of whole units beside them."""
    from scaffolding_b200 import engine as E
    from tests.gpu_util import device_error
    B, H, L = 1, 30, 2600                     # 11 units per head, 330 units
    assert E.attention_launch_count(B, H, L, L) == 3
    rng = np.random.default_rng(2600)
    W = H * 64
    gq, q = to_device(ops, rng.standard_normal((L, W), dtype=np.float32), "bf16")
    gk, k = to_device(ops, rng.standard_normal((L, W), dtype=np.float32), "bf16")
    gv, v = to_device(ops, rng.standard_normal((L, W), dtype=np.float32), "bf16")
    out = _fused(ops, B, H, L, L, gq, gk, gv, W, W, W, L * W, L * W, L * W, 0.125)
    for h in (0, 26, 27, 28, 29):
        sl = slice(h * 64, (h + 1) * 64)
        p = O.softmax_rows((q[:, sl] @ k[:, sl].T * np.float32(0.125)).astype(np.float32))
        ref, allow = O.flash_attention(q[:, sl], k[:, sl], v[:, sl], 0.125, return_allowance=True,
                                       **attn_oracle_opts())
        _check_attn(out[:, sl], ref, O.abs_product(p, v[:, sl].T), allow, f"wave+tail head {h}")
    assert device_error(0) == 0
