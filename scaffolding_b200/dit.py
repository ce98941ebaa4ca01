"""DiT transformer-block workloads on the engine (benchmark configs 4 and 5).

Shapes follow the reference ``DiTBlock`` (``diffusion/models.py:490-590``):
fused ``to_qkv`` (dim -> 3*dim, no bias, ``:508``), ``self_out``
(dim -> dim, ``:509``), FFN dim -> 4*dim -> dim (``:522-527``; GELU-tanh as
the benchmark configuration specifies).  The adaptive LayerNorm modulation
(``:470-487``) is optional in ``DitStack`` (``adaln=True``).

Block linears (config 4), per token shard x[m, C]:
    qkv = x . Wqkv^T                              [m, 3C]
    h   = qkv[:, :C] . Wo^T + bo + x              [m, C]   (stands in for the
                                                           attention output)
    f   = gelu_tanh(h . W1^T + b1)                [m, 4C]
    y   = f . W2^T + b2 + h                       [m, C]
Bias, activation and residual are fused into the GEMM epilogues, so the
block is exactly four tcgen05 GEMM launches.
"""
from __future__ import annotations

import math
import os

import numpy as np

from . import _cuda_ops as ops
from . import engine as E
from ._lib import ACT_GELU_TANH, ACT_NONE, DT_BF16

HIDDEN = 1920
HEADS = 30
HEAD_DIM = 64
TOKENS = 17776
BATCH = 2


def block_flops(m: int, C: int = HIDDEN) -> float:
    """Algorithmic FLOPs of the four block linears on m token rows."""
    return 2.0 * m * C * (3 * C + C + 4 * C + 4 * C)


def _block_launches(C: int, m: int, w: dict, x_ptr: int, qkv: int, h: int, f: int, y: int):
    """The four GEMM launches of one block on m token rows as (name, kwargs)
    for engine.gemm; w holds the device weights, the rest are device pointers."""
    bf = DT_BF16
    return [
        ("qkv", dict(M=m, N=3 * C, K=C, A=x_ptr, lda=C, trans_a=0, B=w["qkv_w"].ptr, ldb=C,
                     trans_b=1, Cp=qkv, ldc=3 * C, in_dt=bf, out_dt=bf, epi=None)),
        ("out", dict(M=m, N=C, K=C, A=qkv, lda=3 * C, trans_a=0, B=w["out_w"].ptr,
                     ldb=C, trans_b=1, Cp=h, ldc=C, in_dt=bf, out_dt=bf,
                     epi=E.make_epilogue(bias_ptr=w["out_b"].ptr, bias_dt=bf, act=ACT_NONE,
                                         residual_ptr=x_ptr, residual_dt=bf, ldr=C))),
        ("up", dict(M=m, N=4 * C, K=C, A=h, lda=C, trans_a=0, B=w["up_w"].ptr,
                    ldb=C, trans_b=1, Cp=f, ldc=4 * C, in_dt=bf, out_dt=bf,
                    epi=E.make_epilogue(bias_ptr=w["up_b"].ptr, bias_dt=bf,
                                        act=ACT_GELU_TANH))),
        ("down", dict(M=m, N=C, K=4 * C, A=f, lda=4 * C, trans_a=0,
                      B=w["down_w"].ptr, ldb=4 * C, trans_b=1, Cp=y, ldc=C,
                      in_dt=bf, out_dt=bf,
                      epi=E.make_epilogue(bias_ptr=w["down_b"].ptr, bias_dt=bf, act=ACT_NONE,
                                          residual_ptr=h, residual_dt=bf, ldr=C))),
    ]


def _run_launches(launches, dev: int, stream=None, timer=None) -> None:
    for name, kw in launches:
        if timer is not None:
            timer.start(name)
        E.gemm(kw["M"], kw["N"], kw["K"], kw["A"], kw["lda"], kw["trans_a"], kw["B"],
               kw["ldb"], kw["trans_b"], kw["Cp"], kw["ldc"], kw["in_dt"], kw["out_dt"],
               epi=kw["epi"], device=dev, stream=stream)
        if timer is not None:
            timer.stop(name)


def _upload_weights(weights: dict, device: int) -> dict:
    bf = E.bfloat16
    return {k: (v if isinstance(v, ops.GpuTensor)
                else ops.gputensor_from_numpy(np.ascontiguousarray(v).astype(bf), device))
            for k, v in weights.items()}


class DitLinears:
    """Device-resident bf16 weights of one block plus activation buffers for
    an m-row token shard."""

    def __init__(self, weights: dict, m: int, device: int):
        bf = E.bfloat16
        self.C = weights["out_w"].shape[0]
        self.m = m
        self.dev = device
        self.w = _upload_weights(weights, device)
        C = self.C
        self.qkv = ops._alloc((m, 3 * C), bf, device)
        self.h = ops._alloc((m, C), bf, device)
        self.f = ops._alloc((m, 4 * C), bf, device)
        self.y = ops._alloc((m, C), bf, device)

    def launches(self, x_ptr: int):
        """The four GEMM launches of one block as (name, kwargs) for engine.gemm."""
        return _block_launches(self.C, self.m, self.w, x_ptr, self.qkv.ptr, self.h.ptr,
                               self.f.ptr, self.y.ptr)

    def run(self, x_ptr: int, stream: int | None = None, timer=None) -> None:
        _run_launches(self.launches(x_ptr), self.dev, stream, timer)


class DitBlock:
    """The block linears as a module (the config-4 workload): ``forward(x)``
    on ``[m, C]`` bf16 token rows returns ``y [m, C]`` (QKV projection,
    out projection + bias + residual, FFN-up + GELU, FFN-down + bias +
    residual; four fused-epilogue GEMM launches).  Every output row depends
    on its own input row only, so ``parallel.DataParallel`` can split the
    rows over GPUs."""

    def __init__(self, weights: dict, device: int):
        self.dev = device
        self.w = _upload_weights(weights, device)
        self.C = self.w["out_w"].shape[0]

    def forward(self, x: "ops.GpuTensor") -> "ops.GpuTensor":
        if x.ndim != 2 or x.shape[1] != self.C:
            raise ValueError(f"DitBlock expects [m, {self.C}] rows, got {x.shape}")
        m, C, dev, bf = x.shape[0], self.C, x.device_id, E.bfloat16
        qkv = ops._alloc((m, 3 * C), bf, dev)
        h = ops._alloc((m, C), bf, dev)
        f = ops._alloc((m, 4 * C), bf, dev)
        y = ops._alloc((m, C), bf, dev)
        with E.on_device(dev):
            _run_launches(_block_launches(C, m, self.w, x.ptr, qkv.ptr, h.ptr, f.ptr, y.ptr), dev)
        return y

    __call__ = forward



# ───────────────────────────── peer K/V exchange ─────────────────────────────

class PeerKV:
    """Copy-engine K/V exchange inside one K/V group of a token-sharded stack
    (one process per GPU on one node).

    Every rank of the group owns a ``[tokens, 2C]`` key buffer shared with
    the others through CUDA IPC; its K/V projection writes its own rows
    there (rows ``group_rank * m ..``) and side streams, one per peer, push
    those rows into the peers' buffers with ``cudaMemcpyAsync`` (copy
    engines over NVLink: no SMs taken from the attention that runs
    meanwhile).  Order is kept with int32 sequence flags in each rank's flag
    buffer (``ready[g]`` then ``consumed[g]``), one sequence number per layer:

    * push to peer p: wait until p has consumed the previous layer
      (``consumed[p] >= seq - 1`` here), copy, store ``p.ready[r] = seq``;
    * before the attention over the peers' keys: ``ready[q] >= seq`` for all
      peers q (bounded wait, ``sf_flag_wait``);
    * after it: store ``p.consumed[r] = seq`` on every peer p;
    * before the next K/V projection overwrites the own rows: the pushes of
      the previous layer are done (stream events).

    Each wait depends only on stores made by other GPUs.  Replaces the NCCL
    all-gather of the K/V rows, whose kernels took SMs from the overlapped
    attention; handles are swapped once over the group's NCCL communicator.
    """

    def __init__(self, plan: "ShardPlan", kv_comm, row_bytes: int, device: int):
        import ctypes as C

        from ._lib import check, lib
        self.g, self.r, self.m = plan.group_size, plan.group_rank, plan.m
        self.row_bytes, self.dev, self.kv_comm = row_bytes, device, kv_comm
        self.seq = 0
        self._lib, self._C, self._check = lib, C, check
        with E.on_device(device):
            self._setup(plan)

    def _setup(self, plan: "ShardPlan") -> None:
        C, lib, check, device = self._C, self._lib, self._check, self.dev
        row_bytes = self.row_bytes
        self.kv_full = self._ipc_alloc(plan.tokens * row_bytes)
        self.flags = self._ipc_alloc(8 * self.g)
        # swap (key buffer, flag buffer) handles inside the group
        hb = 2 * 64
        mine = np.zeros(hb, np.uint8)
        for i, ptr in enumerate((self.kv_full, self.flags)):
            h = (C.c_uint8 * 64)()
            check(lib.sf_ipc_handle(C.c_void_p(ptr), h), "sf_ipc_handle")
            mine[i * 64:(i + 1) * 64] = np.frombuffer(bytes(h), np.uint8)
        allh = self._allgather_host(mine)
        self.peer_kv, self.peer_flags = {}, {}
        for p in range(self.g):
            if p == self.r:
                continue
            opened = []
            for i in range(2):
                h = (C.c_uint8 * 64).from_buffer_copy(allh[p * hb + i * 64:p * hb + (i + 1) * 64].tobytes())
                ptr = C.c_void_p()
                check(lib.sf_ipc_open(h, C.byref(ptr)), "sf_ipc_open")
                opened.append(ptr.value)
            self.peer_kv[p], self.peer_flags[p] = opened
        self.streams, self.ev_push = {}, {}
        for p in self.peer_kv:
            sp, ev = C.c_void_p(), C.c_void_p()
            check(lib.sf_stream_create(device, 1, C.byref(sp)), "sf_stream_create")
            check(lib.sf_event_create(0, C.byref(ev)), "sf_event_create")
            self.streams[p], self.ev_push[p] = sp.value, ev.value
        ev = C.c_void_p()
        check(lib.sf_event_create(0, C.byref(ev)), "sf_event_create")
        self.ev_kv = ev.value
        self.closed = False

    def _ipc_alloc(self, nbytes: int) -> int:
        p = self._C.c_void_p()
        self._check(self._lib.sf_ipc_alloc(int(nbytes), self._C.byref(p)), "sf_ipc_alloc")
        return p.value

    def _allgather_host(self, buf: np.ndarray) -> np.ndarray:
        """All-gather a small host byte array over the group communicator."""
        C, lib, check = self._C, self._lib, self._check
        n = buf.nbytes
        src = E.DeviceBuffer.alloc(n, self.dev)
        dst = E.DeviceBuffer.alloc(n * self.g, self.dev)
        host = np.ascontiguousarray(buf)
        check(lib.sf_memcpy(C.c_void_p(src.ptr), C.c_void_p(host.ctypes.data), n, 0, None),
              "sf_memcpy")
        check(lib.sf_comm_allgather(C.c_void_p(self.kv_comm), C.c_void_p(src.ptr),
                                    C.c_void_p(dst.ptr), n, None), "sf_comm_allgather")
        check(lib.sf_device_synchronize(), "sf_device_synchronize")
        out = np.empty(n * self.g, np.uint8)
        check(lib.sf_memcpy(C.c_void_p(out.ctypes.data), C.c_void_p(dst.ptr), n * self.g, 1,
                            None), "sf_memcpy")
        return out

    def _store(self, ptrs, stream) -> None:
        C = self._C
        arr = (C.c_void_p * len(ptrs))(*ptrs)
        self._check(self._lib.sf_flag_store(arr, len(ptrs), self.seq,
                                            C.c_void_p(stream) if stream else None),
                    "sf_flag_store")

    def own_rows(self) -> int:
        """Device address of this rank's rows in its key buffer."""
        return self.kv_full + self.r * self.m * self.row_bytes

    def before_kv(self, stream) -> None:
        """The pushes of the previous layer have read the own rows."""
        C = self._C
        for p, ev in self.ev_push.items():
            self._check(self._lib.sf_stream_wait_event(C.c_void_p(stream) if stream else None,
                                                       C.c_void_p(ev)), "sf_stream_wait_event")

    def push(self, stream) -> None:
        """After the K/V projection: push the own rows to every peer."""
        C, lib, check = self._C, self._lib, self._check
        self.seq += 1
        s = C.c_void_p(stream) if stream else None
        check(lib.sf_event_record(C.c_void_p(self.ev_kv), s), "sf_event_record")
        off = self.r * self.m * self.row_bytes
        nbytes = self.m * self.row_bytes
        for p, ps in self.streams.items():
            check(lib.sf_stream_wait_event(C.c_void_p(ps), C.c_void_p(self.ev_kv)),
                  "sf_stream_wait_event")
            check(lib.sf_flag_wait(C.c_void_p(self.flags + 4 * (self.g + p)), 1, 1, -1,
                                   self.seq - 1, 0, C.c_void_p(ps)), "sf_flag_wait")
            check(lib.sf_memcpy(C.c_void_p(self.peer_kv[p] + off), C.c_void_p(self.kv_full + off),
                                nbytes, 3, C.c_void_p(ps)), "sf_memcpy")
            self._store([self.peer_flags[p] + 4 * self.r], ps)
            check(lib.sf_event_record(C.c_void_p(self.ev_push[p]), C.c_void_p(ps)),
                  "sf_event_record")

    def wait_ready(self, stream) -> None:
        """Every peer's rows of this layer have landed in the key buffer."""
        C = self._C
        self._check(self._lib.sf_flag_wait(C.c_void_p(self.flags), self.g, 1, self.r, self.seq, 0,
                                           C.c_void_p(stream) if stream else None),
                    "sf_flag_wait")

    def consumed(self, stream) -> None:
        """After the attention over the peers' keys: they may push the next layer."""
        self._store([self.peer_flags[p] + 4 * (self.g + self.r) for p in self.peer_flags], stream)

    def launches_per_layer(self) -> int:
        """Kernels of the exchange per layer: a flag wait and store on the main
        stream, a flag wait and store per peer on the push streams."""
        return 2 + 2 * len(self.peer_kv)

    def close(self) -> None:
        """Unmap the peers' buffers, then free the own ones once every peer
        has unmapped them (two group barriers)."""
        if self.closed:
            return
        with E.on_device(self.dev):
            self._close()

    def _close(self) -> None:
        C, lib, check = self._C, self._lib, self._check
        check(lib.sf_device_synchronize(), "sf_device_synchronize")
        self._allgather_host(np.zeros(4, np.uint8))
        for p in self.peer_kv:
            check(lib.sf_ipc_close(C.c_void_p(self.peer_kv[p])), "sf_ipc_close")
            check(lib.sf_ipc_close(C.c_void_p(self.peer_flags[p])), "sf_ipc_close")
        self._allgather_host(np.zeros(4, np.uint8))
        for p in self.streams:
            lib.sf_stream_destroy(C.c_void_p(self.streams[p]))
            lib.sf_event_destroy(C.c_void_p(self.ev_push[p]))
        lib.sf_event_destroy(C.c_void_p(self.ev_kv))
        check(lib.sf_ipc_free(C.c_void_p(self.kv_full)), "sf_ipc_free")
        check(lib.sf_ipc_free(C.c_void_p(self.flags)), "sf_ipc_free")
        self.closed = True


# ───────────────────────────── token sharding ─────────────────────────────

class ShardPlan:
    """Token (M) sharding of a ``[batch * tokens, hidden]`` activation over
    ``world`` ranks, one process per GPU, contiguous row blocks.

    * ``world <= batch``: every rank holds whole samples; attention needs no
      exchange (keys and queries of a sample live on the same rank).
    * ``world > batch``: every rank holds a slice of one sample; the ranks of
      a sample form a K/V group that all-gathers its K/V rows once per layer.

    Replaces ``DataParallel``'s host scatter (``nn/parallel.py:111-147``):
    rows never leave the device.
    """

    def __init__(self, batch: int, tokens: int, world: int, rank: int):
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside world {world}")
        M = batch * tokens
        if M % world:
            raise ValueError(f"{M} token rows do not split over {world} ranks")
        self.batch, self.tokens, self.world, self.rank = batch, tokens, world, rank
        self.m = M // world
        self.row0 = rank * self.m
        if world <= batch:
            if batch % world:
                raise ValueError(f"batch {batch} does not split over {world} ranks")
            self.samples_per_rank = batch // world
            self.whole_samples = True
            self.kv_exchange = False
            self.sample0 = rank * self.samples_per_rank
            self.group_color, self.group_size, self.group_rank = rank, 1, 0
            self.token0 = 0
        else:
            if world % batch or tokens % (world // batch):
                raise ValueError(f"{world} ranks do not tile {batch} samples of {tokens} tokens")
            self.samples_per_rank = 1
            self.whole_samples = False
            self.kv_exchange = True
            self.group_size = world // batch
            self.sample0 = self.row0 // tokens
            self.token0 = self.row0 % tokens
            self.group_color = self.sample0
            self.group_rank = rank % self.group_size

    def rows(self) -> tuple[int, int]:
        return self.row0, self.row0 + self.m


class DitStack:
    """The benchmark's config 5: ``layers`` DiT layers (attention + block
    linears) over a token shard, bf16 storage, fp32 accumulation.

    Per layer (all on one stream):
      q  = x Wq^T, kv = x Wkv^T          (Wq, Wkv = row blocks of to_qkv)
      [kv all-gather inside the K/V group when the sample is split]
      attention, either fused (``fused=True``, the default for head_dim 64:
      one sf_attention_fwd launch, S and P never leave the SM) or unfused,
      per query chunk of <= ``chunk`` rows, for every (sample, head):
        S = (Q K^T) / sqrt(d)  fp32   -- one batched GEMM, scale in the epilogue
        P = softmax(S)         bf16   -- row softmax in fp32
        O = P V                       -- one batched GEMM, V read MN-major in place
      h = O Wo^T + bo + x
      y = gelu(h W1^T + b1) W2^T + b2 + h
    The reference runs the same sequence with separate scale / softmax /
    bmm launches and the attention on the host (``nn/functional.py:310-321``,
    ``diffusion/models.py:529-590``).

    ``adaln=True`` adds the block's adaptive LayerNorms (norm1 before the QKV
    projection, norm3 before FFN-up, ``diffusion/models.py:470-487``): per
    layer two modulation linears on the per-sample condition vector and two
    fused norm + modulation kernels (``sf_layernorm_modulate``).  Benchmark
    config 5 specifies the linears and attention without them, so it is off
    by default.
    """

    def __init__(self, plan: ShardPlan, hidden: int, heads: int, layers: int, device: int,
                 chunk: int = 2048, weights: list | None = None, seed: int = 1,
                 kv_comm=None, world_comm=None, fused: bool | None = None,
                 adaln: bool = False):
        import ctypes as C

        from ._lib import check, lib
        self.plan, self.C, self.H, self.L = plan, hidden, heads, layers
        self.D = hidden // heads
        self.dev = device
        self.chunk = chunk
        if fused is None:
            fused = self.D == 64 and os.environ.get("SF_ATTN_FUSED", "1") != "0"
        self.fused = bool(fused)
        self.kv_comm, self.world_comm = kv_comm, world_comm
        bf = E.bfloat16
        m, Cw = plan.m, hidden
        shapes = {"qkv_w": (3 * Cw, Cw), "out_w": (Cw, Cw), "out_b": (Cw,),
                  "up_w": (4 * Cw, Cw), "up_b": (4 * Cw,), "down_w": (Cw, 4 * Cw),
                  "down_b": (Cw,)}
        self.w = []
        for li in range(layers):
            if weights is not None:
                self.w.append({k: ops.gputensor_from_numpy(np.ascontiguousarray(v).astype(bf), device)
                               for k, v in weights[li].items()})
                continue
            lw = {}
            for j, (k, shp) in enumerate(shapes.items()):
                t = ops._alloc(shp, bf, device)
                if k.endswith("_b"):
                    check(lib.sf_memset(C.c_void_p(t.ptr), 0, t.numel * 2, None), "sf_memset")
                else:
                    check(lib.sf_fill_normal(C.c_void_p(t.ptr), DT_BF16, t.numel,
                                             seed * 1000003 + li * 16 + j, 0.0, 0.02, None),
                          "sf_fill_normal")
                lw[k] = t
            self.w.append(lw)
        spr = plan.samples_per_rank
        keys = plan.tokens
        self.q = ops._alloc((m, Cw), bf, device)
        # K/V exchange inside a split sample's rank group: copy-engine pushes
        # into the peers' key buffers (PeerKV), or the NCCL all-gather (test
        # hook SF_KV_EXCHANGE=nccl).
        self.peer = None
        if (plan.kv_exchange and kv_comm is not None
                and os.environ.get("SF_KV_EXCHANGE", "ce") != "nccl"):
            self.peer = PeerKV(plan, kv_comm, 2 * Cw * 2, device)
            full = E.DeviceBuffer(self.peer.kv_full, keys * 2 * Cw * 2, device, False)
            own = E.DeviceBuffer(self.peer.own_rows(), m * 2 * Cw * 2, device, False)
            self.kv_full = ops.GpuTensor(full, (keys, 2 * Cw), bf, device)
            self.kv_local = ops.GpuTensor(own, (m, 2 * Cw), bf, device)
        else:
            self.kv_local = ops._alloc((m, 2 * Cw), bf, device)
            self.kv_full = (ops._alloc((keys, 2 * Cw), bf, device) if plan.kv_exchange
                            else self.kv_local)
        q_rows = plan.tokens if plan.whole_samples else m
        crow = min(chunk, q_rows)
        self.S = self.P = None
        if not self.fused:
            self.S = ops._alloc((spr, heads, crow, keys), np.float32, device)
            self.P = ops._alloc((spr, heads, crow, keys), bf, device)
        self.attn = ops._alloc((m, Cw), bf, device)
        # Adaptive LayerNorm in front of the QKV and FFN-up GEMMs (DiTBlock's
        # norm1 / norm3, diffusion/models.py:470-487, 555, 584): per layer
        # two modulation linears (cond [B, C] -> [B, 2C]) and the fused
        # norm + modulation kernel; cond is one [B, C] vector per sample.
        self.adaln = bool(adaln)
        self.xn = self.cond = None
        self.mod = []
        if self.adaln:
            B = plan.batch
            self.xn = ops._alloc((m, Cw), bf, device)
            self.cond = ops._alloc((B, Cw), bf, device)
            check(lib.sf_fill_normal(C.c_void_p(self.cond.ptr), DT_BF16, B * Cw, seed * 7 + 3,
                                     0.0, 1.0, None), "sf_fill_normal")
            for li in range(layers):
                lm = {}
                for j, name in enumerate(("mod1", "mod3")):
                    wt = ops._alloc((2 * Cw, Cw), bf, device)
                    check(lib.sf_fill_normal(C.c_void_p(wt.ptr), DT_BF16, wt.numel,
                                             seed * 1000003 + li * 16 + 8 + j, 0.0, 0.02, None),
                          "sf_fill_normal")
                    lm[name + "_w"] = wt
                    lm[name + "_p"] = ops._alloc((B, 2 * Cw), bf, device)
                self.mod.append(lm)
        self.h = ops._alloc((m, Cw), bf, device)
        self.f = ops._alloc((m, 4 * Cw), bf, device)
        self.y = [ops._alloc((m, Cw), bf, device), ops._alloc((m, Cw), bf, device)]
        self.out_full = (ops._alloc((plan.batch * plan.tokens, Cw), bf, device)
                         if plan.world > 1 else None)
        # Overlap of the K/V all-gather with attention over the rank's own keys
        # (fused TMEM-accumulator kernel only): attention over kv_local writes a
        # partial result while the gather runs on a side stream; attention over
        # the gathered keys (minus the local slice) merges it.
        self.overlap = (self.fused and plan.kv_exchange
                        and os.environ.get("SF_KV_OVERLAP", "1") != "0")
        self.part_o = self.part_ml = None
        self.comm_stream = self.ev_kv = self.ev_gather = None
        if self.overlap:
            self.part_o = ops._alloc((m, Cw), np.float32, device)
            self.part_ml = ops._alloc((m, heads, 2), np.float32, device)
            if kv_comm is not None and self.peer is None:
                sp, e1, e2 = C.c_void_p(), C.c_void_p(), C.c_void_p()
                # high priority: the gather's kernel is scheduled onto SMs as
                # soon as attention blocks retire instead of after them all
                check(lib.sf_stream_create_priority(device, 1, 1, C.byref(sp)),
                      "sf_stream_create_priority")
                check(lib.sf_event_create(0, C.byref(e1)), "sf_event_create")
                check(lib.sf_event_create(0, C.byref(e2)), "sf_event_create")
                self.comm_stream, self.ev_kv, self.ev_gather = sp.value, e1.value, e2.value

    # ── launches
    def _gemm(self, name, timer, stream, *args, **kw):
        if timer is not None:
            timer.start(name)
        E.gemm(*args, device=self.dev, stream=stream, **kw)
        if timer is not None:
            timer.stop(name)

    def _attention(self, stream, timer):
        p, Cw, H, D = self.plan, self.C, self.H, self.D
        keys = p.tokens
        spr = p.samples_per_rank
        q_rows = p.tokens if p.whole_samples else p.m
        scale = 1.0 / math.sqrt(D)
        bf = DT_BF16
        if self.overlap:
            import ctypes as C

            from ._lib import check, lib
            m = p.m
            if timer is not None:
                timer.start("attn")
            # own keys (kv_local) -> partial result
            E.attention_partial(1, H, m, m, self.q.ptr, Cw, m * Cw, self.kv_local.ptr, 2 * Cw,
                                m * 2 * Cw, self.kv_local.ptr + Cw * 2, 2 * Cw, m * 2 * Cw,
                                self.attn.ptr, Cw, m * Cw, scale, m, m, self.part_o.ptr,
                                self.part_ml.ptr, 1, dtype=bf, head_dim=D, stream=stream,
                                device=self.dev)
            s = stream if stream else E.get_stream(self.dev)
            if self.peer is not None:
                self.peer.wait_ready(s)
            elif self.comm_stream is not None:
                check(lib.sf_stream_wait_event(C.c_void_p(s), C.c_void_p(self.ev_gather)),
                      "sf_stream_wait_event")
            # the group's other keys (the local slice skipped), merged
            E.attention_partial(1, H, m, keys, self.q.ptr, Cw, m * Cw, self.kv_full.ptr, 2 * Cw,
                                keys * 2 * Cw, self.kv_full.ptr + Cw * 2, 2 * Cw, keys * 2 * Cw,
                                self.attn.ptr, Cw, m * Cw, scale, p.token0, p.token0 + m,
                                self.part_o.ptr, self.part_ml.ptr, 2, dtype=bf, head_dim=D,
                                stream=stream, device=self.dev)
            if self.peer is not None:
                self.peer.consumed(s)
            if timer is not None:
                timer.stop("attn")
            return
        if self.peer is not None:
            self.peer.wait_ready(stream if stream else E.get_stream(self.dev))
            self._attention_local(stream, timer)
            self.peer.consumed(stream if stream else E.get_stream(self.dev))
            return
        self._attention_local(stream, timer)

    def _attention_local(self, stream, timer):
        """Attention of the rank's query rows over the keys in kv_full."""
        p, Cw, H, D = self.plan, self.C, self.H, self.D
        keys = p.tokens
        spr = p.samples_per_rank
        q_rows = p.tokens if p.whole_samples else p.m
        scale = 1.0 / math.sqrt(D)
        bf = DT_BF16
        if self.fused:
            # Q rows of each local sample; K and V in place in the [keys, 2C]
            # rows of kv_full (K at column 0, V at column C, head h at h*64).
            if timer is not None:
                timer.start("attn")
            E.attention(spr, H, q_rows, keys, self.q.ptr, Cw, q_rows * Cw, self.kv_full.ptr,
                        2 * Cw, keys * 2 * Cw, self.kv_full.ptr + Cw * 2, 2 * Cw, keys * 2 * Cw,
                        self.attn.ptr, Cw, q_rows * Cw, scale, dtype=bf, head_dim=D,
                        stream=stream, device=self.dev)
            if timer is not None:
                timer.stop("attn")
            return
        for c0 in range(0, q_rows, self.chunk):
            rows = min(self.chunk, q_rows - c0)
            s_batch = rows * keys
            bt = E.make_batch(H, spr, a=(D, keys * Cw), b=(D, keys * 2 * Cw),
                              c=(s_batch, H * s_batch))
            self._gemm("qk", timer, stream, rows, keys, D, self.q.ptr + c0 * Cw * 2, Cw, 0,
                       self.kv_full.ptr, 2 * Cw, 1, self.S.ptr, keys, bf, 0,
                       epi=E.make_epilogue(alpha=scale), batch=bt)
            if timer is not None:
                timer.start("softmax")
            E.softmax_rows(self.S.ptr, 0, keys, self.P.ptr, bf, keys, spr * H * rows, keys, 1.0,
                           stream=stream, device=self.dev)
            if timer is not None:
                timer.stop("softmax")
            bt2 = E.make_batch(H, spr, a=(s_batch, H * s_batch), b=(D, keys * 2 * Cw),
                               c=(D, keys * Cw))
            self._gemm("pv", timer, stream, rows, D, keys, self.P.ptr, keys, 0,
                       self.kv_full.ptr + Cw * 2, 2 * Cw, 0, self.attn.ptr + c0 * Cw * 2, Cw,
                       bf, bf, batch=bt2)

    def _adaln(self, li: int, which: str, x_ptr: int, stream, timer) -> int:
        """Modulation linear of ``which`` (mod1 / mod3) for layer ``li``, then
        LayerNorm + per-sample scale / shift of the rank's rows into ``xn``;
        returns the pointer of the normalised rows."""
        import ctypes as C

        from ._lib import check, lib
        p, Cw, lm = self.plan, self.C, self.mod[li]
        B, bf = p.batch, DT_BF16
        prm = lm[which + "_p"]
        self._gemm(which, timer, stream, B, 2 * Cw, Cw, self.cond.ptr, Cw, 0, lm[which + "_w"].ptr,
                   Cw, 1, prm.ptr, 2 * Cw, bf, bf)
        # the rank's rows: whole samples (group = tokens) or one sample's slice
        group = p.tokens if p.whole_samples else p.m
        s = stream if stream else E.get_stream(self.dev)
        if timer is not None:
            timer.start("adaln")
        check(lib.sf_layernorm_modulate(p.m, Cw, C.c_void_p(x_ptr), bf, Cw, None, None, 1e-5,
                                        C.c_void_p(prm.ptr + p.sample0 * 2 * Cw * 2), bf, 2 * Cw,
                                        group, C.c_void_p(self.xn.ptr), bf, Cw,
                                        C.c_void_p(s) if s else None), "sf_layernorm_modulate")
        if timer is not None:
            timer.stop("adaln")
        return self.xn.ptr

    def _qkv_input(self, li: int, x_ptr: int, stream, timer) -> int:
        """The rows the QKV projection reads: x, or norm1(x) with adaLN."""
        return self._adaln(li, "mod1", x_ptr, stream, timer) if self.adaln else x_ptr

    def _q(self, li: int, x_ptr: int, stream, timer) -> None:
        p, Cw, w = self.plan, self.C, self.w[li]
        self._gemm("q", timer, stream, p.m, Cw, Cw, x_ptr, Cw, 0, w["qkv_w"].ptr, Cw, 1,
                   self.q.ptr, Cw, DT_BF16, DT_BF16)

    def _kv(self, li: int, x_ptr: int, stream, timer) -> None:
        p, Cw, w = self.plan, self.C, self.w[li]
        if self.peer is not None:
            # the previous layer's pushes have read the rows this overwrites
            self.peer.before_kv(stream if stream else E.get_stream(self.dev))
        self._gemm("kv", timer, stream, p.m, 2 * Cw, Cw, x_ptr, Cw, 0,
                   w["qkv_w"].ptr + Cw * Cw * 2, Cw, 1, self.kv_local.ptr, 2 * Cw, DT_BF16,
                   DT_BF16)

    def qkv(self, li: int, x_ptr: int, stream=None, timer=None) -> None:
        """q and the local K/V rows of layer ``li``."""
        x_in = self._qkv_input(li, x_ptr, stream, timer)
        self._q(li, x_in, stream, timer)
        self._kv(li, x_in, stream, timer)

    def exchange(self, stream=None, timer=None) -> None:
        """All-gather the K/V rows of this rank's sample inside its K/V group."""
        import ctypes as C

        from ._lib import check, lib
        p = self.plan
        if not p.kv_exchange:
            return
        if self.peer is not None:
            self.peer.push(stream if stream else E.get_stream(self.dev))
            return
        if self.comm_stream is not None:
            # gather on the side stream once the K/V projection is done; the
            # attention over the gathered keys waits for ev_gather
            s = stream if stream else E.get_stream(self.dev)
            check(lib.sf_event_record(C.c_void_p(self.ev_kv), C.c_void_p(s)), "sf_event_record")
            check(lib.sf_stream_wait_event(C.c_void_p(self.comm_stream), C.c_void_p(self.ev_kv)),
                  "sf_stream_wait_event")
            check(lib.sf_comm_allgather(C.c_void_p(self.kv_comm), C.c_void_p(self.kv_local.ptr),
                                        C.c_void_p(self.kv_full.ptr), p.m * 2 * self.C * 2,
                                        C.c_void_p(self.comm_stream)), "sf_comm_allgather")
            check(lib.sf_event_record(C.c_void_p(self.ev_gather), C.c_void_p(self.comm_stream)),
                  "sf_event_record")
            return
        if timer is not None:
            timer.start("kv_allgather")
        check(lib.sf_comm_allgather(C.c_void_p(self.kv_comm), C.c_void_p(self.kv_local.ptr),
                                    C.c_void_p(self.kv_full.ptr), p.m * 2 * self.C * 2,
                                    C.c_void_p(stream) if stream else None),
              "sf_comm_allgather")
        if timer is not None:
            timer.stop("kv_allgather")

    def post(self, li: int, x_ptr: int, out_ptr: int, stream=None, timer=None) -> None:
        """Output projection + residual, FFN + residual."""
        p, Cw, w = self.plan, self.C, self.w[li]
        m, bf = p.m, DT_BF16
        self._gemm("out", timer, stream, m, Cw, Cw, self.attn.ptr, Cw, 0, w["out_w"].ptr, Cw, 1,
                   self.h.ptr, Cw, bf, bf,
                   epi=E.make_epilogue(bias_ptr=w["out_b"].ptr, bias_dt=bf, residual_ptr=x_ptr,
                                       residual_dt=bf, ldr=Cw))
        up_in = self._adaln(li, "mod3", self.h.ptr, stream, timer) if self.adaln else self.h.ptr
        self._gemm("up", timer, stream, m, 4 * Cw, Cw, up_in, Cw, 0, w["up_w"].ptr, Cw, 1,
                   self.f.ptr, 4 * Cw, bf, bf,
                   epi=E.make_epilogue(bias_ptr=w["up_b"].ptr, bias_dt=bf, act=ACT_GELU_TANH))
        self._gemm("down", timer, stream, m, Cw, 4 * Cw, self.f.ptr, 4 * Cw, 0, w["down_w"].ptr,
                   4 * Cw, 1, out_ptr, Cw, bf, bf,
                   epi=E.make_epilogue(bias_ptr=w["down_b"].ptr, bias_dt=bf,
                                       residual_ptr=self.h.ptr, residual_dt=bf, ldr=Cw))

    def layer(self, li: int, x_ptr: int, out_ptr: int, stream=None, timer=None) -> None:
        x_in = self._qkv_input(li, x_ptr, stream, timer)
        if self.comm_stream is not None or self.peer is not None:
            # K/V first, so that their gather on the side stream runs during
            # the Q projection as well as the attention over the own keys
            self._kv(li, x_in, stream, timer)
            self.exchange(stream, timer)
            self._q(li, x_in, stream, timer)
        else:
            self._q(li, x_in, stream, timer)
            self._kv(li, x_in, stream, timer)
            self.exchange(stream, timer)
        self._attention(stream, timer)
        self.post(li, x_ptr, out_ptr, stream, timer)

    def forward(self, x_ptr: int, stream=None, timer=None) -> int:
        """Run all layers on the local rows starting from ``x_ptr``; return the
        device pointer of the output (the gathered ``[batch*tokens, C]`` on
        multi-rank runs, the local rows otherwise)."""
        import ctypes as C

        from ._lib import check, lib
        cur = x_ptr
        for li in range(self.L):
            out = self.y[li % 2].ptr
            self.layer(li, cur, out, stream, timer)
            cur = out
        if self.out_full is not None:
            if timer is not None:
                timer.start("out_allgather")
            check(lib.sf_comm_allgather(C.c_void_p(self.world_comm), C.c_void_p(cur),
                                        C.c_void_p(self.out_full.ptr),
                                        self.plan.m * self.C * 2,
                                        C.c_void_p(stream) if stream else None),
                  "sf_comm_allgather")
            if timer is not None:
                timer.stop("out_allgather")
            return self.out_full.ptr
        return cur

    def launches_per_forward(self) -> int:
        p = self.plan
        q_rows = p.tokens if p.whole_samples else p.m
        if self.fused:
            # five linears, then the attention call(s): a split last wave adds a merge launch
            if self.overlap:
                n_attn = (E.attention_launch_count(1, self.H, p.m, p.m, device=self.dev)
                          + E.attention_launch_count(1, self.H, p.m, p.tokens, p.token0,
                                                     p.token0 + p.m, device=self.dev))
            else:
                n_attn = E.attention_launch_count(p.samples_per_rank, self.H, q_rows, p.tokens,
                                                  device=self.dev)
            n_peer = self.peer.launches_per_layer() if self.peer is not None else 0
            return self.L * (5 + n_attn + n_peer + self._adaln_launches())
        chunks = (q_rows + self.chunk - 1) // self.chunk
        n_peer = self.peer.launches_per_layer() if self.peer is not None else 0
        return self.L * (5 + 3 * chunks + n_peer + self._adaln_launches())

    def close(self) -> None:
        """Release the peer key buffers (collective over the K/V group: every
        rank of the group calls it)."""
        if self.peer is not None:
            self.peer.close()

    def _adaln_launches(self) -> int:
        """Per layer: two modulation linears and two norm kernels (a linear
        whose split-K needs a workspace is two launches)."""
        if not self.adaln:
            return 0
        import ctypes as C

        from ._lib import check, lib
        need = C.c_size_t()
        check(lib.sf_gemm_workspace_size(None, self.plan.batch, 2 * self.C, self.C, 0, 1, DT_BF16,
                                         DT_BF16, C.byref(need)), "sf_gemm_workspace_size")
        return 2 * (2 if need.value else 1) + 2


def stack_flops(batch: int, tokens: int, hidden: int, heads: int, layers: int) -> float:
    """Algorithmic FLOPs of one forward: block linears + QK^T and P.V."""
    M = batch * tokens
    attn = 2 * (2.0 * batch * heads * tokens * tokens * (hidden // heads))
    return layers * (block_flops(M, hidden) + attn)
