"""Worker for tests/test_chain_tp.py::test_chain_tp_nccl_gpu: one rank of the
tensor-parallel decode step on its GPU (NCCL), checked against the unsharded
CPU oracle.  Launched by torch.distributed.run; exits non-zero on mismatch."""
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from esimd_learning_b200.chain import SMALL, DecodeChain, TPComm, full_weights, shard_weights  # noqa: E402
from oracle import oracle as O  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    shape, M = SMALL, 4
    full = full_weights(shape, seed=0)
    shards = shard_weights(full, shape, rank, world)
    comm = TPComm(16 * shape.hidden, rank, world, dev)
    g = torch.Generator().manual_seed(5)
    h, r, a = (torch.randn(M, shape.hidden, generator=g).half() for _ in range(3))
    pos = torch.randint(0, shape.max_position, (M,), generator=g)
    ref_out, _, ref_r = O.decode_chain(full, shape, h, r, a, pos)
    for mode in ("nccl", "fused", "fused-graph"):
        chain = DecodeChain(shards, shape, M, dev, world=world, comm=None if mode == "nccl" else comm)
        rd = r.to(dev)
        hd, ad, pd = h.to(dev), a.to(dev), pos.to(dev)
        if mode == "fused-graph":
            chain.capture(hd, rd, ad, pd)
            for _ in range(3):  # replays advance the device-side epoch
                rd.copy_(r.to(dev))
                chain.graph.replay()
            out = chain.out
        else:
            out, _ = chain.step(hd, rd, ad, pd)
        torch.cuda.synchronize()
        assert torch.equal(rd.cpu(), ref_r), f"{mode}: residual"
        O.assert_parity(out, ref_out, f"rank {rank} TP={world} {mode} out")
        # ranks must agree bit for bit after the all-reduce
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        for t in gathered:
            assert torch.equal(t, out), f"{mode}: ranks disagree"
    assert comm.errors() == 0, "a bounded wait ran out"
    comm.close()
    dist.destroy_process_group()
    print(f"rank {rank} ok")


if __name__ == "__main__":
    main()
