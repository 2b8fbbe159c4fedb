"""Host-side logic of the N-sharded GEMM with real ranks on CPU: two gloo
processes run the same orchestration code as bench.py (aegis_dist:
shard_columns, exchange_handles, close_peers) with POSIX shared memory
standing in for CUDA IPC. Each rank "stores" its column shard of C into every
rank's C, as the fused epilogue does, then a barrier; every rank's C must be
the full product. Failure detection is made on the host: a rank that never
joins, and a rank that leaves before the exchange, end the other rank's wait
with an error inside its process-group timeout."""
import multiprocessing as mp
import os
import socket
import time
from datetime import timedelta
from multiprocessing import shared_memory

import numpy as np
import pytest

import aegis_dist as ad


class ShmBackend:
    """export/open/close over POSIX shared memory; an "address" is a key."""

    def __init__(self):
        self.arrays, self.shms, self.next = {}, {}, 1

    def create(self, nbytes):
        shm = shared_memory.SharedMemory(create=True, size=nbytes)
        return self._add(shm)

    def _add(self, shm):
        key = self.next
        self.next += 1
        self.shms[key] = shm
        self.arrays[key] = np.ndarray((shm.size // 8,), dtype=np.float64, buffer=shm.buf)
        return key

    def export(self, addr):
        return self.shms[addr].name.encode()

    def open(self, handle):
        return self._add(shared_memory.SharedMemory(name=handle.decode()))

    def close(self, addr):
        self.arrays.pop(addr)
        self.shms.pop(addr).close()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, mode, q):
    import torch.distributed as dist
    try:
        if mode == "never_joins" and rank == 1:
            q.put((rank, "left", 0.0))
            return
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=8))
        if mode == "leaves" and rank == 1:
            q.put((rank, "left", 0.0))
            q.close()
            q.join_thread()  # the message is delivered before the abrupt exit
            os._exit(0)  # gone before the handle exchange, no clean shutdown
        M, N, K = 8, 24, 12
        rng = np.random.RandomState(5)
        A, B = rng.randn(M, K), rng.randn(K, N)
        c0, ns = ad.shard_columns(N, world, rank)
        be = ShmBackend()
        own = be.create(M * N * 8)
        be.arrays[own][:] = np.nan
        t0 = time.time()
        pm = ad.exchange_handles(be, own)
        Cr = A @ B[:, c0:c0 + ns]
        for addr in pm.addrs:  # the fused epilogue: this rank's tile into every rank's C
            be.arrays[addr].reshape(M, N)[:, c0:c0 + ns] = Cr
        dist.barrier()  # after it, every rank's C is complete
        ok = np.array_equal(be.arrays[own].reshape(M, N), A @ B) or np.allclose(be.arrays[own].reshape(M, N), A @ B)
        dist.barrier()
        ad.close_peers(be, pm)
        dist.barrier()
        be.shms[own].close()
        be.shms[own].unlink()
        dist.destroy_process_group()
        q.put((rank, "ok" if ok else "wrong", time.time() - t0))
    except Exception as e:  # noqa: BLE001 - report any failure to the parent
        q.put((rank, "error: " + type(e).__name__, 0.0))


def run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, mode, q)) for r in range(world)]
    t0 = time.time()
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, _ = q.get(timeout=120)
        out[r] = status
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out, time.time() - t0


@pytest.mark.parametrize("world", [2, 3])
def test_ranks_assemble_the_full_product(world):
    out, _ = run(world, "normal")
    assert all(v == "ok" for v in out.values()), out


def test_rank_that_never_joins_is_detected():
    out, secs = run(2, "never_joins")
    assert out[1] == "left" and out[0].startswith("error"), out
    assert secs < 90


def test_rank_that_leaves_before_the_exchange_is_detected():
    out, secs = run(2, "leaves")
    assert out[1] == "left" and out[0].startswith("error"), out
    assert secs < 90


def test_shard_columns():
    assert ad.shard_columns(16384, 8, 3) == (6144, 2048)
    assert ad.shard_columns(10, 1, 0) == (0, 10)
    with pytest.raises(ValueError):
        ad.shard_columns(10, 4, 0)
    with pytest.raises(ValueError):
        ad.shard_columns(16, 4, 4)
