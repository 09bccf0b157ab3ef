"""Failure detection without faulting a GPU.

* GPU: the tensor-parallel reduce kernel's bounded wait.  One process plays
  rank 0 of a world of 2 whose second rank never arrives (its region is
  mapped but nothing raises its ready flag).  The wait gives up after its
  poll limit (about a second), the kernel returns, bit 0 of the comm
  region's error word is set, and the context stays usable.
* Host: a gloo rank that leaves before a collective makes the surviving
  rank's collective fail within the process-group timeout instead of
  hanging.
"""
import ctypes
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from esimd_learning_b200 import cabi
from esimd_learning_b200.workloads import gemv_case
from oracle import oracle as O


@pytest.mark.gpu
def test_allreduce_wait_times_out_and_reports(cuda_device):
    L = cabi.lib()
    M, N, K = 1, 256, 512
    slot = M * N
    nbytes = L.cek_tp_comm_bytes(slot, 2)
    regions = []
    for _ in range(2):
        p = ctypes.c_void_p()
        cabi.call("cek_comm_alloc", nbytes, ctypes.byref(p))
        regions.append(p.value)
    try:
        peers = torch.tensor(regions, dtype=torch.int64, device=cuda_device)
        x, wq, s = gemv_case(M, N, K, seed=3, device=cuda_device)
        out = torch.zeros(M, N, dtype=torch.float16, device=cuda_device)
        cabi.call("cek_gemv_fp8_allreduce", cabi.ptr(x), cabi.ptr(wq), cabi.ptr(s), cabi.ptr(out), M, N, K,
                  cabi.CEK_F16, cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, cabi.ptr(peers), regions[0], slot, 0, 2,
                  0, cabi.current_stream())
        torch.cuda.synchronize()  # returns: the wait is bounded
        err = ctypes.c_uint32(0)
        cabi.call("cek_comm_errors", regions[0], ctypes.byref(err))
        assert err.value & 1, "the missing rank was not reported"
        # recovery: the reset clears the sticky error word
        cabi.call("cek_comm_reset", regions[0], nbytes)
        cabi.call("cek_comm_errors", regions[0], ctypes.byref(err))
        assert err.value == 0
        # the context is still healthy
        y = torch.zeros(M, N, dtype=torch.float16, device=cuda_device)
        cabi.call("cek_gemv_fp8", cabi.ptr(x), cabi.ptr(wq), cabi.ptr(s), cabi.ptr(y), M, N, K, cabi.CEK_F16,
                  cabi.CEK_F16, cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, 0, cabi.current_stream())
        torch.cuda.synchronize()
        O.assert_parity(y, O.gemv_fp8(x.cpu(), wq.cpu(), s.cpu()), "after timeout")
    finally:
        for r in regions:
            L.cek_comm_free(r)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)  # both ranks healthy here
    if rank == 1:
        os._exit(0)  # leaves between steps, no collective in flight
    try:
        dist.all_reduce(t)
        q.put(("no error", None))
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        q.put(("error", type(e).__name__))


def test_departed_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    status, kind = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert status == "error", "the surviving rank's collective did not fail"
