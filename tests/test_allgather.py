"""Column-parallel FP8 GEMV with its all-gather fused into the epilogue
(cek_gemv_fp8_allgather, cek_comm_barrier), the N > 1 form of BASELINE
config 1: each rank streams its rows of W and pushes them into every rank's
full output over NVLink peer memory.

CPU: the row split and its reassembly on two gloo ranks against the
unsharded oracle.  One GPU: the push epilogue with two comm regions on the
same device (two "ranks" run one after the other; no barrier, whose ranks
must run concurrently) and the one-rank barrier.  Two GPUs: the full path
across processes (skipped on a one-GPU box)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from esimd_learning_b200.chain import shard_rows
from esimd_learning_b200.workloads import gemv_case
from oracle import oracle as O


@pytest.mark.parametrize("n", [1, 7, 8, 4096, 6143])
def test_shard_rows_partition(n):
    for world in (1, 2, 3, 4, 8):
        spans = [shard_rows(n, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    M, N, K = 3, 1000, 256
    x, wq, s = gemv_case(M, N, K, seed=4)
    r0, r1 = shard_rows(N, rank, world)
    part = O.gemv_fp8(x, wq[r0:r1], s[r0:r1], out_dtype=torch.float32)
    parts = [None] * world
    dist.all_gather_object(parts, (r0, part.numpy().copy()))
    y = torch.cat([torch.from_numpy(p) for _, p in sorted(parts, key=lambda t: t[0])], dim=1)
    q.put((rank, y.half().numpy().copy()))
    dist.destroy_process_group()


def test_column_parallel_reassembly_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, wq, s = gemv_case(3, 1000, 256, seed=4)
    ref = O.gemv_fp8(x, wq, s)
    for _, y in got:
        assert torch.equal(torch.from_numpy(y), ref)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 6144, 4096), (8, 4096, 14336), (5, 1000, 512), (20, 2048, 1024),
                                   (4, 2048, 14336), (1, 1024, 14336)])
def test_allgather_push_two_regions_one_gpu(ext, cuda_device, M, N, K):
    """Both ranks' shards pushed into two comm regions on one GPU; the last
    two shapes' shards (1024 and 512 rows of K = 14336) take the cluster K
    split, whose leader CTAs run the push epilogue."""
    import ctypes
    from esimd_learning_b200 import cabi
    L = cabi.lib()
    nbytes = cabi.CEK_COMM_SYNC_BYTES + 256 + M * N * 2
    regions = []
    for _ in range(2):
        p = ctypes.c_void_p()
        cabi.call("cek_comm_alloc", nbytes, ctypes.byref(p))
        regions.append(p.value)
    try:
        peers = torch.tensor(regions, dtype=torch.int64, device=cuda_device)
        x, wq, s = gemv_case(M, N, K, seed=M)
        xd = x.to(cuda_device)
        for rank in range(2):
            r0, r1 = shard_rows(N, rank, 2)
            w = wq[r0:r1].contiguous().to(cuda_device)
            sc = s[r0:r1].contiguous().to(cuda_device)
            cabi.call("cek_gemv_fp8_allgather", cabi.ptr(xd), cabi.ptr(w), cabi.ptr(sc), M, r1 - r0, K, r0, N, 256,
                      cabi.CEK_F16, cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, cabi.ptr(peers), regions[rank], nbytes,
                      rank, 2, 0, cabi.current_stream())
        torch.cuda.synchronize()
        ref = O.gemv_fp8(x, wq, s)
        for reg in regions:
            class _View:  # zero-copy view of the region's output
                __cuda_array_interface__ = {"shape": (M * N * 2,), "typestr": "|u1", "version": 3, "strides": None,
                                            "data": (reg + cabi.CEK_COMM_SYNC_BYTES + 256, False)}
            y = torch.as_tensor(_View(), device=cuda_device).view(torch.float16).view(M, N)
            O.assert_parity(y, ref, f"region M={M} N={N} K={K}")
        assert L.cek_gemv_fp8_allgather(cabi.ptr(xd), 16, 16, M, N, K, 1, N, 256, 0, 0, 1, cabi.ptr(peers),
                                        regions[0], nbytes, 0, 2, 0, None) == cabi.CEK_ERR_INVALID_ARG
    finally:
        for r in regions:
            L.cek_comm_free(r)


@pytest.mark.gpu
def test_allgather_one_rank_with_barrier(ext, cuda_device):
    from esimd_learning_b200.chain import TPComm, gemv_fp8_allgather
    M, N, K = 4, 4096, 4096
    comm = TPComm(0, 0, 1, cuda_device, data_bytes=M * N * 2)
    try:
        x, wq, s = gemv_case(M, N, K, seed=9, device=cuda_device)
        gemv_fp8_allgather(comm, x, wq, s, 0, N, 0)
        comm.barrier()
        torch.cuda.synchronize()
        O.assert_parity(comm.data_tensor(0, (M, N)), O.gemv_fp8(x.cpu(), wq.cpu(), s.cpu()), "one rank")
        assert comm.errors() == 0
    finally:
        comm.close()


@pytest.mark.gpu
def test_allgather_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    worker = Path(__file__).resolve().parent / "allgather_worker.py"
    for _ in range(3):  # a free port can be taken between the probe and the rendezvous: retry
        r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                            "--master-addr", "127.0.0.1", "--master-port", str(_port()), str(worker)],
                           capture_output=True, text=True, timeout=600, env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
        if "EADDRINUSE" not in r.stderr:
            break
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
