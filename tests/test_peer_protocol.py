"""The copy-engine K/V exchange of the token-sharded DiT stack (dit.PeerKV),
checked on the CPU: four ranks of one sample's group run as threads of this
process against an in-memory stand-in for the C ABI calls PeerKV makes.
Device buffers are byte arrays at fake addresses; an IPC mapping is the
peer's own array (one address space); sf_memcpy and sf_flag_store act at
once; sf_flag_wait asserts that its condition already holds when it is
enqueued (the ranks move in lock step, so it must), which checks the flag
indices, the sequence numbers and the row offsets of every push: after each
layer's exchange every rank's key buffer must hold every peer's rows of that
layer."""
import bisect
import ctypes as C
import threading

import numpy as np
import pytest

from scaffolding_b200 import dit
from scaffolding_b200 import engine as E

BASE = 1 << 60  # above every user-space host address


class FakeMem:
    def __init__(self):
        self.lock = threading.Lock()
        self.bases, self.bufs, self.next = [], {}, BASE

    def alloc(self, n):
        with self.lock:
            a = self.next
            self.next += (n + 4095) // 4096 * 4096 + 4096
            self.bases.append(a)
            self.bufs[a] = np.zeros(n, np.uint8)
            return a

    def free(self, a):
        with self.lock:
            del self.bufs[a]
            self.bases.remove(a)

    def view(self, addr, n):
        """The n bytes at a fake device address, or at a real host address."""
        if addr < BASE:
            return np.ctypeslib.as_array((C.c_uint8 * n).from_address(addr))
        with self.lock:
            i = bisect.bisect_right(self.bases, addr) - 1
            base = self.bases[i]
            buf = self.bufs[base]
        off = addr - base
        assert 0 <= off and off + n <= buf.size, "access outside a buffer"
        return buf[off:off + n]


def _val(x):
    return x.value if isinstance(x, C.c_void_p) else (0 if x is None else int(x))


class FakeLib:
    """The calls of PeerKV; the communicator argument is a FakeGroup."""

    def __init__(self, mem, groups):
        self.mem, self.groups = mem, groups
        self.ids = 0
        self.flag_waits = []
        self.ipc_live = set()

    def _out(self, ref, value):
        ref._obj.value = value
        return 0

    def sf_ipc_alloc(self, n, ref):
        a = self.mem.alloc(int(n))
        self.ipc_live.add(a)
        return self._out(ref, a)

    def sf_ipc_free(self, p):
        self.ipc_live.remove(_val(p))
        self.mem.free(_val(p))
        return 0

    def sf_ipc_handle(self, p, h):
        C.memmove(h, int(_val(p)).to_bytes(8, "little") + bytes(56), 64)
        return 0

    def sf_ipc_open(self, h, ref):
        return self._out(ref, int.from_bytes(bytes(h)[:8], "little"))

    def sf_ipc_close(self, p):
        return 0

    def sf_stream_create(self, dev, nb, ref):
        self.ids += 1
        return self._out(ref, self.ids)

    def sf_event_create(self, timing, ref):
        self.ids += 1
        return self._out(ref, self.ids)

    def sf_stream_destroy(self, s):
        return 0

    def sf_event_destroy(self, e):
        return 0

    def sf_event_record(self, e, s):
        return 0

    def sf_stream_wait_event(self, s, e):
        return 0

    def sf_device_synchronize(self):
        return 0

    def sf_memcpy(self, dst, src, n, kind, stream):
        n = int(n)
        self.mem.view(_val(dst), n)[:] = self.mem.view(_val(src), n)
        return 0

    def sf_comm_allgather(self, comm, send, recv, n, stream):
        return self.groups[_val(comm)].allgather(self.mem, _val(send), _val(recv), int(n))

    def sf_flag_store(self, arr, count, value, stream):
        for i in range(count):
            self.mem.view(_val(arr[i]), 4).view(np.int32)[0] = value
        return 0

    def sf_flag_wait(self, flags, count, stride, skip, value, timeout, stream):
        base = _val(flags)
        for i in range(count):
            if i == skip:
                continue
            got = int(self.mem.view(base + 4 * i * stride, 4).view(np.int32)[0])
            assert got >= value, f"flag {i} holds {got}, waiting for {value}"
        self.flag_waits.append((base, count, skip, value))
        return 0


class FakeGroup:
    """An all-gather among `n` threads (one per rank, `rank_of` by thread)."""

    def __init__(self, n):
        self.n = n
        self.barrier = threading.Barrier(n)
        self.slots = [None] * n
        self.rank_of = {}

    def allgather(self, mem, send, recv, nbytes):
        r = self.rank_of[threading.get_ident()]
        self.slots[r] = bytes(mem.view(send, nbytes))
        self.barrier.wait()
        out = mem.view(recv, nbytes * self.n)
        for i in range(self.n):
            out[i * nbytes:(i + 1) * nbytes] = np.frombuffer(self.slots[i], np.uint8)
        self.barrier.wait()
        return 0


class _Buf:
    def __init__(self, mem, n):
        self.ptr = mem.alloc(n)


@pytest.mark.parametrize("batch,world", [(1, 4), (2, 8), (1, 2)])
def test_peer_exchange_protocol(monkeypatch, batch, world):
    tokens, row_bytes, layers = 96, 48, 4
    mem = FakeMem()
    groups = {}
    lib = FakeLib(mem, groups)
    from scaffolding_b200 import _lib
    monkeypatch.setattr(_lib, "lib", lib)
    monkeypatch.setattr(E.DeviceBuffer, "alloc", classmethod(lambda cls, n, dev: _Buf(mem, n)))

    class _Dev:
        def __init__(self, dev):
            pass

        def __enter__(self):
            return self

        def __exit__(self, *a):
            return False

    monkeypatch.setattr(E, "on_device", _Dev)
    plans = [dit.ShardPlan(batch, tokens, world, r) for r in range(world)]
    g = plans[0].group_size
    for c in range(batch):
        groups[1000 + c] = FakeGroup(g)
    stacks = [None] * world
    step = threading.Barrier(world)
    errors = []

    def rank(r):
        try:
            p = plans[r]
            grp = groups[1000 + p.group_color]
            grp.rank_of[threading.get_ident()] = p.group_rank
            kv = dit.PeerKV(p, 1000 + p.group_color, row_bytes, 0)
            stacks[r] = kv
            m = p.m
            own = mem.view(kv.own_rows(), m * row_bytes)
            assert kv.own_rows() == kv.kv_full + p.group_rank * m * row_bytes
            for layer in range(layers):
                step.wait()
                kv.before_kv(None)
                own[:] = (layer * 16 + r) & 0xff        # this layer's K/V rows of rank r
                kv.push(None)
                step.wait()                            # every rank has pushed
                kv.wait_ready(None)
                full = mem.view(kv.kv_full, tokens * row_bytes).reshape(tokens, row_bytes)
                for q in range(g):
                    peer = p.sample0 * g + q if batch > 1 else q
                    rows = full[q * m:(q + 1) * m]
                    assert (rows == ((layer * 16 + peer) & 0xff)).all(), (r, layer, q)
                step.wait()                            # every rank has read its keys
                kv.consumed(None)
            step.wait()
            kv.close()
        except BaseException as exc:  # reported by the main thread
            errors.append((r, exc))
            step.abort()
            for grp in groups.values():
                grp.barrier.abort()

    threads = [threading.Thread(target=rank, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(60)
    assert not errors, errors
    assert all(s is not None and s.closed for s in stacks)
    assert all(s.seq == layers for s in stacks)
    # per layer: one ready wait per rank, one consumed wait per (rank, peer)
    assert len(lib.flag_waits) == world * layers * g
    assert not lib.ipc_live, "shared buffers left allocated"
