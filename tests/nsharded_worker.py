"""One rank of the multi-GPU N-sharded check (run by torchrun from
tests/test_nsharded_multigpu.py): real CUDA-IPC peers over NVLink. Each rank
computes its column shard with aegis_gemm_bf16_nsharded, storing into every
rank's C; after the barrier its C must equal the single-GPU GEMM bit for bit."""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, os.path.join(ROOT, "aegis-core_b200"))
import aegis_capi as ac  # noqa: E402
import aegis_dist as ad  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", local))
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    ctx = ac.Context(local)
    ctx.set_stream(s.cuda_stream)
    M, N, K = 640, 2048, 1536
    g = ac.Generator(99)
    A, B = g.uniform(M * K, "bf16"), g.uniform(K * N, "bf16")
    c0, ns = ad.shard_columns(N, world, rank)
    dA = torch.from_numpy(A.view(np.int16)).cuda()
    dBfull = torch.from_numpy(B.view(np.int16)).cuda()
    dB = torch.from_numpy(np.ascontiguousarray(B.reshape(K, N)[:, c0:c0 + ns]).view(np.int16).reshape(-1)).cuda()
    import ctypes
    cptr = ctypes.c_void_p()
    ac.check(ctx.lib.aegis_device_alloc(ctx.ptr, M * N * 2, ctypes.byref(cptr)), "alloc")
    be = ad.CudaIpcBackend(ctx)
    pm = ad.exchange_handles(be, cptr.value)
    full = torch.zeros(M * N, dtype=torch.int16, device="cuda")
    ctx.gemm(dA.data_ptr(), dBfull.data_ptr(), full.data_ptr(), M, N, K, ac.DTYPE_BF16)
    ok = True
    for rep in range(3):
        ctx.nsharded(M, N, K, dA.data_ptr(), K, dB.data_ptr(), ns, pm.addrs, N, world, rank, ac.DTYPE_BF16)
        dist.all_reduce(torch.zeros(1, device="cuda"))  # barrier after the fused all-gather
        torch.cuda.synchronize()
        mine = np.empty(M * N, dtype=np.int16)
        ac.check(ctx.lib.aegis_copy_to_host(ctx.ptr, mine.ctypes.data, cptr.value, M * N * 2), "d2h")
        ok &= np.array_equal(mine, full.cpu().numpy())
    ctx.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    ad.close_peers(be, pm)
    dist.barrier()
    ac.check(ctx.lib.aegis_device_free(ctx.ptr, cptr), "free")
    print(f"rank {rank}: {'ok' if ok else 'MISMATCH'}", flush=True)
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
