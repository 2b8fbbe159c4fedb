"""Host-side orchestration of the N-sharded GEMM across ranks (one process
per GPU, torch.distributed for the plumbing).

The kernel side is aegis_gemm_bf16_nsharded (include/aegis.h): rank r
computes its column shard of C and stores every finished tile into the C of
every rank. What the host must do around it lives here, written against a
small "memory backend" interface so the same code runs with CUDA IPC on a
GPU node and with POSIX shared memory in the CPU tests (gloo ranks):

  1. shard_columns: which columns rank r owns (N divisible by nranks);
  2. exchange_handles: every rank exports its C buffer, all-gathers the
     handles, and opens its peers' (the others' C becomes addressable);
  3. after each launch, a cross-rank barrier ordered after it on the stream,
     before anyone reads C;
  4. close the peers' mappings before the buffers are freed.
No counterpart in the reference (it has no multi-GPU code).
"""
from __future__ import annotations

from dataclasses import dataclass


def shard_columns(N: int, nranks: int, rank: int) -> tuple[int, int]:
    """(first column, width) of rank's shard of N columns."""
    if nranks < 1 or not 0 <= rank < nranks:
        raise ValueError(f"rank {rank} of {nranks}")
    if N % nranks:
        raise ValueError(f"N = {N} does not divide evenly over {nranks} ranks")
    ns = N // nranks
    return rank * ns, ns


@dataclass
class PeerMap:
    """Every rank's C as an address valid in this process (own first-class)."""
    rank: int
    nranks: int
    addrs: list          # addrs[i]: rank i's C in this process
    opened: list         # indices this process opened (to close later)


def exchange_handles(backend, own_addr: int, group=None) -> PeerMap:
    """All-gather the export handle of each rank's C and open the peers'.
    `backend` provides export(addr) -> bytes, open(handle) -> addr,
    close(addr); torch.distributed carries the handles."""
    import torch.distributed as dist
    rank, nranks = dist.get_rank(group), dist.get_world_size(group)
    mine = backend.export(own_addr)
    handles = [None] * nranks
    dist.all_gather_object(handles, mine, group=group)
    addrs, opened = [], []
    for i, h in enumerate(handles):
        if i == rank:
            addrs.append(own_addr)
        else:
            addrs.append(backend.open(h))
            opened.append(i)
    return PeerMap(rank, nranks, addrs, opened)


def close_peers(backend, pm: PeerMap) -> None:
    for i in pm.opened:
        backend.close(pm.addrs[i])
    pm.opened = []


class CudaIpcBackend:
    """CUDA IPC through the C ABI (aegis_ipc_get_handle / open / close)."""

    def __init__(self, ctx):
        self.ctx = ctx

    def export(self, addr: int) -> bytes:
        return self.ctx.ipc_get_handle(addr)

    def open(self, handle: bytes) -> int:
        return self.ctx.ipc_open_handle(handle)

    def close(self, addr: int) -> None:
        self.ctx.ipc_close_handle(addr)
