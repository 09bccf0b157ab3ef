"""Worker for tests/test_allgather.py::test_allgather_two_gpus: one rank of
the column-parallel GEMV with its fused all-gather (cek_gemv_fp8_allgather +
cek_comm_barrier) on its own GPU, eager and as CUDA-graph replays alternating
two output buffers; every rank's gathered output must equal the unsharded CPU
oracle and agree bit for bit across ranks.  Launched by torch.distributed.run."""
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from esimd_learning_b200.chain import TPComm, gemv_fp8_allgather, shard_rows  # noqa: E402
from esimd_learning_b200.workloads import gemv_case  # noqa: E402
from oracle import oracle as O  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    # the last case's shards (1024 rows of K = 14336) take the cluster K split
    cases = [(1, 6144, 4096), (8, 4096, 14336), (3, 1000, 512), (16, 2048, 1024), (8, 2048, 14336)]
    ybytes = [M * N * 2 for M, N, K in cases]
    offs = [sum(ybytes[:i]) for i in range(len(cases))]
    total = (sum(ybytes) + 255) // 256 * 256
    comm = TPComm(0, rank, world, dev, data_bytes=2 * total)
    data = []
    for i, (M, N, K) in enumerate(cases):
        x, wq, s = gemv_case(M, N, K, seed=10 + i)
        r0, r1 = shard_rows(N, rank, world)
        data.append((x.to(dev), wq[r0:r1].contiguous().to(dev), s[r0:r1].contiguous().to(dev), r0,
                     O.gemv_fp8(x, wq, s)))

    def step(parity):
        for i, (M, N, K) in enumerate(cases):
            x, w, s, r0, _ = data[i]
            gemv_fp8_allgather(comm, x, w, s, r0, N, parity * total + offs[i], early_weights=True)
        comm.barrier()

    def check(parity, what):
        for i, (M, N, K) in enumerate(cases):
            y = comm.data_tensor(parity * total + offs[i], (M, N)).clone()
            O.assert_parity(y, data[i][4], f"rank {rank} {what} case {i}")
            g = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(g, y)
            assert all(torch.equal(t, y) for t in g), f"{what}: ranks disagree"

    step(0)
    torch.cuda.synchronize()
    check(0, "eager")
    st = torch.cuda.Stream(dev)
    with torch.cuda.stream(st):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            step(1)
            step(0)
        for _ in range(3):
            graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    check(0, "graph")
    check(1, "graph")
    assert comm.errors() == 0, "a bounded wait ran out"
    comm.close()
    dist.destroy_process_group()
    print(f"rank {rank} ok")


if __name__ == "__main__":
    main()
