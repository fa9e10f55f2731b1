"""Global reductions over a tensor sharded across processes (one per GPU).

Each rank summarises its shard on its own GPU (rtc_shard_summary_local), the
32-byte summaries are all-gathered with torch.distributed (NCCL over
NVLink/NVSwitch on GPUs, gloo on CPU), and every rank folds them in rank
order with rtc_shard_combine, so every rank returns the reference's
sum/mean/max/min of the concatenated tensor.  That all-gather is the only
communication of the hot path.
"""
from __future__ import annotations

import ctypes
from ctypes import c_double

from . import _native as N


ShardSummary = N.ShardSummary

SUMMARY_BYTES = ctypes.sizeof(ShardSummary)


def _bind(lib):
    """Binds the two summary entry points on a library loaded elsewhere
    (N.lib() already binds them)."""
    lib.rtc_shard_summary_local.restype = N.RtcResult
    lib.rtc_shard_summary_local.argtypes = [ctypes.POINTER(N.RtcTensor),
                                            ctypes.POINTER(ShardSummary)]
    lib.rtc_shard_combine.restype = N.RtcResult
    lib.rtc_shard_combine.argtypes = [ctypes.POINTER(ShardSummary), ctypes.c_size_t,
                                      ctypes.POINTER(c_double)]


def combine(summaries: list[ShardSummary], lib=None) -> tuple[float, float, float, float]:
    """(sum, mean, max, min) of the concatenation of the shards, in order."""
    lib = lib or N.lib()
    _bind(lib)
    arr = (ShardSummary * max(1, len(summaries)))(*summaries)
    out = (c_double * 4)()
    N.check(lib.rtc_shard_combine(arr, len(summaries), out))
    return tuple(out)


class ShardedReducer:
    """sum/mean/max/min of a tensor sharded over the ranks of the default
    process group (torch.distributed must be initialised).

    `timeout_s` bounds the exchange: if the other ranks' summaries have not
    all arrived after that many seconds (a rank left between steps, or never
    reached this step), exchange() raises RusttorchError (BackendError)
    instead of waiting for the process group's own timeout.  After that the
    process group is not usable for further collectives: destroy it."""

    def __init__(self, lib, rank: int, world: int, timeout_s: float | None = None):
        import torch

        self.lib, self.rank, self.world = lib, rank, world
        self.timeout_s = timeout_s
        _bind(lib)
        dev = "cuda" if torch.cuda.is_available() else "cpu"
        self._send = torch.empty(SUMMARY_BYTES, dtype=torch.uint8, device=dev)
        self._recv = torch.empty(SUMMARY_BYTES * world, dtype=torch.uint8, device=dev)
        self._host = torch.empty(SUMMARY_BYTES, dtype=torch.uint8, pin_memory=dev == "cuda")

    def local(self, desc) -> ShardSummary:
        s = ShardSummary()
        N.check(self.lib.rtc_shard_summary_local(desc.ref, ctypes.byref(s)))
        return s

    def exchange(self, s: ShardSummary) -> list[ShardSummary]:
        import torch.distributed as dist

        ctypes.memmove(self._host.data_ptr(), ctypes.addressof(s), SUMMARY_BYTES)
        self._send.copy_(self._host, non_blocking=True)
        if self.timeout_s is None:
            dist.all_gather_into_tensor(self._recv, self._send)
        else:
            from datetime import timedelta

            work = dist.all_gather_into_tensor(self._recv, self._send, async_op=True)
            try:
                done = work.wait(timeout=timedelta(seconds=self.timeout_s))
            except Exception as e:   # the backend's timeout or a lost peer
                raise N.RusttorchError(
                    f"sharded stats: the shard summaries of all {self.world} ranks did not "
                    f"arrive within {self.timeout_s} s: {e}", N.BACKEND_ERROR) from e
            if done is False:
                raise N.RusttorchError(
                    f"sharded stats: the shard summaries of all {self.world} ranks did not "
                    f"arrive within {self.timeout_s} s", N.BACKEND_ERROR)
        raw = self._recv.cpu().numpy().tobytes()
        return [ShardSummary.from_buffer_copy(raw, i * SUMMARY_BYTES) for i in range(self.world)]

    def stats(self, desc) -> tuple[float, float, float, float]:
        return combine(self.exchange(self.local(desc)), self.lib)

    def sum(self, desc) -> float:
        return self.stats(desc)[0]

    def close(self) -> None:
        pass


class PeerSum:
    """The sum of one f64 per rank (each rank's partial of a sharded sum),
    over peer memory: every rank's library writes its partial into a slot on
    every rank's GPU through a CUDA IPC mapping and adds the slots in rank
    order (rtc_peer_allreduce_sum_f64) — one kernel, no NCCL call, no host
    round trip.  Construct on every rank of the default process group (one
    process per GPU, all on one node); the IPC handles travel once, through
    torch.distributed.  Call close() on every rank before the process group
    is destroyed."""

    def __init__(self, lib, rank: int, world: int, device: int):
        import torch.distributed as dist

        if world > N.PEER_MAX_RANKS:
            raise ValueError(f"at most {N.PEER_MAX_RANKS} ranks")
        self.lib, self.rank, self.world, self.device = lib, rank, world, device
        self.generation = 0
        nbytes = lib.rtc_peer_slot_bytes(world)
        own = ctypes.c_void_p()
        N.check(lib.rtc_malloc(device, nbytes, ctypes.byref(own)))
        self._own = own
        zero = (ctypes.c_char * nbytes)()
        N.check(lib.rtc_memcpy_h2d(device, own, zero, nbytes))
        handle = (ctypes.c_char * N.IPC_HANDLE_BYTES)()
        N.check(lib.rtc_ipc_handle(device, own, handle))
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle))
        self._opened = []
        ptrs = (ctypes.c_void_p * world)()
        for p in range(world):
            if p == rank:
                ptrs[p] = own.value
                continue
            h = (ctypes.c_char * N.IPC_HANDLE_BYTES).from_buffer_copy(handles[p])
            mapped = ctypes.c_void_p()
            N.check(lib.rtc_ipc_open(device, h, ctypes.byref(mapped)))
            self._opened.append(mapped)
            ptrs[p] = mapped.value
        self._ptrs = ptrs
        dist.barrier()   # every rank's slots are zeroed and mapped

    def allreduce(self, local_ptr: int, out_ptr: int) -> None:
        """Queues *out = sum over ranks of *local (device f64 pointers) on the
        library's stream of the calling thread."""
        self.generation += 1
        N.check(self.lib.rtc_peer_allreduce_sum_f64(
            self.device, ctypes.c_void_p(local_ptr), self._ptrs, self.world, self.rank,
            self.generation, ctypes.c_void_p(out_ptr)))

    def close(self) -> None:
        """Unmaps the other ranks' slots and frees this rank's (after a
        barrier, so no rank still writes into them)."""
        import torch.distributed as dist

        if self._own is None:
            return
        N.check(self.lib.rtc_synchronize())
        dist.barrier()
        for m in self._opened:
            N.check(self.lib.rtc_ipc_close(self.device, m))
        self._opened = []
        dist.barrier()
        N.check(self.lib.rtc_free(self.device, self._own))
        self._own = None
