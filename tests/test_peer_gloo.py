"""sharded.PeerSum's host-side logic on CPU ranks (gloo), against a stand-in
for the library.

The stand-in keeps every "device allocation" in memory shared by the
processes (one slot array per rank in a multiprocessing array) and runs the
peer all-reduce's algorithm on the host: write this rank's value and the
generation into every rank's slots, wait for every rank's generation in its
own, add in rank order.  What is checked is PeerSum's own logic — the IPC
handle exchange over torch.distributed, the mapping of every rank's array
in rank order, the generation numbering (1, 2, 3, ... on every rank) and
the teardown order (close the mappings, then free) — and that the values
every rank gets are the rank-order sums.  The device kernel itself is
tested on GPUs by tests/test_peer_gpu.py.
"""
import ctypes
import os
import socket
import struct
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from rusttorch_b200 import _native as N
from rusttorch_b200 import sharded


def _ok():
    r = N.RtcResult()
    r.success = True
    r.code = N.OK
    return r


class FakeLib:
    """The entry points PeerSum calls, on shared host memory.  Allocation
    "addresses" are small integers: 1000 * (rank + 1) for rank's slot array,
    2000000 + k for opened mappings (remembering which rank's array they
    map)."""

    def __init__(self, rank, world, shared, log):
        self.rank, self.world, self.shared, self.log = rank, world, shared, log
        self.mapped = {}          # fake peer pointer -> rank whose array it maps
        self.values = {}          # fake device f64 pointers -> value

    def rtc_peer_slot_bytes(self, world):
        return 2 * world * 16

    def rtc_malloc(self, device, nbytes, out):
        out._obj.value = 1000 * (self.rank + 1)
        self.log.append(("malloc", nbytes))
        return _ok()

    def rtc_memcpy_h2d(self, device, dst, src, nbytes):
        if dst.value == 1000 * (self.rank + 1):   # zeroing the slot array
            base = self.rank * 2 * self.world * 2
            for i in range(2 * self.world * 2):
                self.shared[base + i] = 0.0
        return _ok()

    def rtc_ipc_handle(self, device, ptr, handle):
        payload = struct.pack("<q", ptr.value).ljust(N.IPC_HANDLE_BYTES, b"\0")
        ctypes.memmove(handle, payload, N.IPC_HANDLE_BYTES)
        return _ok()

    def rtc_ipc_open(self, device, handle, out):
        owner_ptr = struct.unpack("<q", bytes(handle)[:8])[0]
        owner = owner_ptr // 1000 - 1
        fake = 2000000 + owner
        self.mapped[fake] = owner
        out._obj.value = fake
        self.log.append(("open", owner))
        return _ok()

    def _owner(self, ptr):
        return self.rank if ptr == 1000 * (self.rank + 1) else self.mapped[ptr]

    def rtc_peer_allreduce_sum_f64(self, device, local, slots, world, rank, gen, out):
        owners = [self._owner(slots[p]) for p in range(world)]
        self.log.append(("allreduce", gen, owners))
        par = gen & 1
        v = self.values[local.value]
        stride = 2 * world * 2            # floats per rank's array: [2][world] {value, gen}
        for p in range(world):
            at = owners[p] * stride + (par * world + rank) * 2
            self.shared[at] = v
        for p in range(world):
            at = owners[p] * stride + (par * world + rank) * 2
            self.shared[at + 1] = float(gen)
        mine = owners[rank] * stride + par * world * 2
        t0 = time.time()
        for q in range(world):
            while self.shared[mine + 2 * q + 1] != float(gen):
                if time.time() - t0 > 20:
                    raise TimeoutError("rank never arrived")
                time.sleep(0.001)
        s = 0.0
        for q in range(world):
            s = s + self.shared[mine + 2 * q]
        self.values[out.value] = s
        return _ok()

    def rtc_synchronize(self):
        return _ok()

    def rtc_ipc_close(self, device, ptr):
        self.log.append(("close", self.mapped.pop(ptr.value)))
        return _ok()

    def rtc_free(self, device, ptr):
        self.log.append(("free", ptr.value))
        return _ok()


def _rank(rank, world, port, shared, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        log = []
        lib = FakeLib(rank, world, shared, log)
        peer = sharded.PeerSum(lib, rank, world, device=0)
        got = []
        for step in range(4):
            vals = [0.25 * (r + 1) + step * 1e-3 + 2.0 ** (-45 + r) for r in range(world)]
            lib.values[111] = vals[rank]
            peer.allreduce(111, 222)
            want = 0.0
            for v in vals:
                want = want + v
            got.append((lib.values[222], want))
        peer.close()
        dist.destroy_process_group()
        q.put((rank, got, log, None))
    except Exception as ex:
        q.put((rank, None, None, repr(ex)))


@pytest.mark.parametrize("world", [2, 3])
def test_peer_sum_host_logic(world):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    shared = ctx.Array("d", world * 2 * world * 2, lock=False)
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, shared, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, got, log, err = q.get(timeout=120)
        results[rank] = (got, log, err)
    for p in procs:
        p.join(timeout=30)
    for rank, (got, log, err) in results.items():
        assert err is None, (rank, err)
        for value, want in got:
            assert value == want, (rank, value, want)
        # every other rank's array mapped once, in rank order in each call
        assert [e[1] for e in log if e[0] == "open"] == [p for p in range(world) if p != rank]
        calls = [e for e in log if e[0] == "allreduce"]
        assert [c[1] for c in calls] == [1, 2, 3, 4]
        assert all(c[2] == list(range(world)) for c in calls)
        # teardown: the mappings closed before this rank's array is freed
        tail = [e[0] for e in log[-world:]]
        assert tail == ["close"] * (world - 1) + ["free"]
