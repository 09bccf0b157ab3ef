"""Worker for tests/test_chain_tp.py::test_chain_tp_nccl_gpu: one rank of the
tensor-parallel decode step on its GPU (NCCL), checked against the unsharded
CPU oracle.  Launched by torch.distributed.run; exits non-zero on mismatch."""
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from esimd_learning_b200.chain import SMALL, DecodeChain, full_weights, shard_weights  # noqa: E402
from oracle import oracle as O  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    shape, M = SMALL, 4
    full = full_weights(shape, seed=0)
    chain = DecodeChain(shard_weights(full, shape, rank, world), shape, M, dev, world=world)
    g = torch.Generator().manual_seed(5)
    h, r, a = (torch.randn(M, shape.hidden, generator=g).half() for _ in range(3))
    pos = torch.randint(0, shape.max_position, (M,), generator=g)
    ref_out, _, ref_r = O.decode_chain(full, shape, h, r, a, pos)
    rd = r.to(dev)
    out, _ = chain.step(h.to(dev), rd, a.to(dev), pos.to(dev))
    torch.cuda.synchronize()
    assert torch.equal(rd.cpu(), ref_r), "residual"
    O.assert_parity(out, ref_out, f"rank {rank} TP={world} out")
    # ranks must agree bit for bit after the all-reduce
    gathered = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(gathered, out)
    for t in gathered:
        assert torch.equal(t, out), "ranks disagree"
    dist.destroy_process_group()
    print(f"rank {rank} ok")


if __name__ == "__main__":
    main()
