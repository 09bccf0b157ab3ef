"""Tensor-parallel decode step of a 70B-shaped layer built from the custom ops
hidden 8192, 64 q / 8 kv heads of 128, MLP 28672.

One step, on every rank (rank r of TP):

1. ``esimd_fused_add_rms_norm_batched_fp8``: residual += hidden; RMSNorm
   (replicated, every rank holds the full hidden row); the QKV GEMV over this
   rank's heads (column-parallel, 10240 / TP output rows laid out as
   [q heads | k heads | v heads] of the shard).
2. ``esimd_qkv_norm_rope`` on the local heads (per-head RMSNorm of q and k,
   RoPE theta 500000 at the token positions).  Attention itself is outside
   this path.
3. ``esimd_fused_add_rms_norm_gelu_mul_fp8`` for the MLP block: residual
   += attention output (given as an input), RMSNorm, the gate_up GEMV over
   this rank's [gate | up] rows (column-parallel, 57344 / TP rows) with
4. GeLU(tanh)-and-mul in its epilogue: the local activation [M, 28672 / TP]
   in one launch of the gated bulk GEMV (M > 16: the GEMV, then
   ``esimd_gelu_and_mul``).
5. The down GEMV on this rank's K-slice of the down weight (row-parallel,
   K = 28672 / TP) with the full per-channel scale: a partial sum of the
   output.
6. The all-reduce (sum) of the fp16 [M, 8192] partials: fused into the down
   GEMV over peer memory (``TPComm``) or NCCL; at TP = 1 it is skipped.

All weights are e4m3 with per-output-channel fp32 scales computed on the
full (unsharded) matrix, so the sharded step equals the unsharded one up to
the order of the final fp16 sums.  The step is a sequence of kernels on one
stream with no host synchronisation, so it captures in one CUDA graph
(``DecodeChain.capture``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ChainShape:
    hidden: int = 8192
    num_q_heads: int = 64
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 28672
    rope_theta: float = 500000.0
    max_position: int = 8192
    eps: float = 1e-6

    @property
    def qkv_rows(self) -> int:
        return (self.num_q_heads + 2 * self.num_kv_heads) * self.head_dim

    def weight_bytes(self) -> int:
        """FP8 weight bytes of one full (unsharded) step."""
        h = self.hidden
        return self.qkv_rows * h + 2 * self.intermediate * h + h * self.intermediate


SMALL = ChainShape(hidden=1024, num_q_heads=8, num_kv_heads=2, head_dim=128, intermediate=2048,
                   max_position=512)


def _quantize_rows(w: torch.Tensor):
    """Per-output-row e4m3 quantisation: scale = rowabsmax / 448 (fp32)."""
    wf = w.float()
    s = wf.abs().amax(dim=1).clamp(min=1e-12) / 448.0
    return (wf / s[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn), s


def full_weights(shape: ChainShape, seed: int = 0, device="cpu"):
    """The unsharded weights of one layer: dict of (e4m3 [N, K], fp32 [N]) plus
    the norm weights (gamma = 1 + 0.1 N(0,1) in fp16)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    h, f = shape.hidden, shape.intermediate

    def w(n, k):
        return _quantize_rows(torch.randn(n, k, generator=gen, device=device) * 0.02)

    out = {"qkv": w(shape.qkv_rows, h), "gate_up": w(2 * f, h), "down": w(h, f)}
    out["gamma_attn"] = (1 + 0.1 * torch.randn(h, generator=gen, device=device)).half()
    out["gamma_mlp"] = (1 + 0.1 * torch.randn(h, generator=gen, device=device)).half()
    out["q_norm"] = (1 + 0.1 * torch.randn(shape.head_dim, generator=gen, device=device)).half()
    out["k_norm"] = (1 + 0.1 * torch.randn(shape.head_dim, generator=gen, device=device)).half()
    return out


def shard_weights(full: dict, shape: ChainShape, rank: int, world: int) -> dict:
    """This rank's shards.  QKV by heads (q heads, then k heads, then v heads
    of the shard), gate_up by matching gate/up rows, down by K columns."""
    hq, hkv, d, f = shape.num_q_heads, shape.num_kv_heads, shape.head_dim, shape.intermediate
    if hq % world or hkv % world or f % world:
        raise ValueError(f"TP={world} must divide q heads {hq}, kv heads {hkv} and intermediate {f}")
    lq, lkv, lf = hq // world, hkv // world, f // world
    wq, sq = full["qkv"]
    qrows = torch.arange(rank * lq * d, (rank + 1) * lq * d)
    krows = hq * d + torch.arange(rank * lkv * d, (rank + 1) * lkv * d)
    vrows = (hq + hkv) * d + torch.arange(rank * lkv * d, (rank + 1) * lkv * d)
    rows = torch.cat([qrows, krows, vrows]).to(wq.device)
    wgu, sgu = full["gate_up"]
    gu_rows = torch.cat([torch.arange(rank * lf, (rank + 1) * lf),
                         f + torch.arange(rank * lf, (rank + 1) * lf)]).to(wgu.device)
    wd, sd = full["down"]
    return {
        "qkv": (wq.view(torch.uint8)[rows].contiguous().view(torch.float8_e4m3fn), sq[rows].contiguous()),
        "gate_up": (wgu.view(torch.uint8)[gu_rows].contiguous().view(torch.float8_e4m3fn),
                    sgu[gu_rows].contiguous()),
        "down": (wd.view(torch.uint8)[:, rank * lf:(rank + 1) * lf].contiguous().view(torch.float8_e4m3fn),
                 sd.contiguous()),
        "gamma_attn": full["gamma_attn"], "gamma_mlp": full["gamma_mlp"],
        "q_norm": full["q_norm"], "k_norm": full["k_norm"],
        "local_q_heads": lq, "local_kv_heads": lkv, "local_intermediate": lf,
    }


def rope_cache(shape: ChainShape, device) -> torch.Tensor:
    """fp32 [max_position, head_dim] cos | sin (vLLM layout)."""
    d = shape.head_dim
    inv = 1.0 / (shape.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    t = torch.arange(shape.max_position, dtype=torch.float32)
    fr = torch.outer(t, inv)
    return torch.cat([fr.cos(), fr.sin()], dim=-1).to(device)


class TPComm:
    """Peer-memory plumbing for the fused down-projection all-reduce
    (cek_gemv_fp8_allreduce): this rank's comm region (cek_comm_alloc), its
    CUDA IPC handle exchanged over `group`, the peers' regions mapped into
    this process, and a device array of all regions' addresses.  Set-up only
    (allocates, maps, synchronises); the per-step call does neither."""

    def __init__(self, slot_elems: int, rank: int, world: int, device, group=None, data_bytes: int | None = None):
        """slot_elems sizes the all-reduce receive slots; data_bytes, when
        given, sizes the data area directly (all-gather outputs)."""
        import ctypes

        import torch.distributed as dist

        from esimd_learning_b200 import cabi

        self.cabi, self.rank, self.world, self.slot_elems = cabi, rank, world, slot_elems
        self.group, self.device = group, device
        L = cabi.lib()
        nbytes = (cabi.CEK_COMM_SYNC_BYTES + int(data_bytes) if data_bytes is not None
                  else L.cek_tp_comm_bytes(slot_elems, world))
        if nbytes <= 0:
            raise ValueError("bad comm size")
        self.nbytes = nbytes
        mine = ctypes.c_void_p()
        cabi.call("cek_comm_alloc", nbytes, ctypes.byref(mine))
        self.mine = mine.value
        handle = ctypes.create_string_buffer(64)
        cabi.call("cek_ipc_get_handle", self.mine, handle)
        handles = [handle.raw]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle.raw, group=group)
        self.opened = []
        addrs = []
        for r, h in enumerate(handles):
            if r == rank:
                addrs.append(self.mine)
            else:
                p = ctypes.c_void_p()
                cabi.call("cek_ipc_open_handle", h, ctypes.byref(p))
                self.opened.append(p.value)
                addrs.append(p.value)
        self.peers = torch.tensor(addrs, dtype=torch.int64, device=device)
        if world > 1:
            dist.barrier(group=group)

    def data_tensor(self, byte_offset: int, shape, dtype=torch.float16) -> torch.Tensor:
        """A zero-copy tensor over this rank's data area at byte_offset."""
        n = 1
        for d in shape:
            n *= d
        esz = torch.empty((), dtype=dtype).element_size()
        if byte_offset < 0 or self.cabi.CEK_COMM_SYNC_BYTES + byte_offset + n * esz > self.nbytes:
            raise ValueError("view outside the comm region")

        class _View:
            __cuda_array_interface__ = {
                "shape": (n * esz,), "typestr": "|u1", "version": 3, "strides": None,
                "data": (self.mine + self.cabi.CEK_COMM_SYNC_BYTES + byte_offset, False)}

        return torch.as_tensor(_View(), device=self.device).view(dtype).view(*shape)

    def barrier(self, stream=None):
        """cek_comm_barrier on the current stream: every rank's earlier pushes
        into this region become visible here."""
        cb = self.cabi
        cb.call("cek_comm_barrier", cb.ptr(self.peers), self.mine, self.rank, self.world,
                stream if stream is not None else cb.current_stream())

    def errors(self) -> int:
        import ctypes
        v = ctypes.c_uint32(0)
        self.cabi.call("cek_comm_errors", self.mine, ctypes.byref(v))
        return v.value

    def reset(self):
        """Recovery after a reported timeout: every rank calls this with no
        call in flight on any rank (the group barriers on both sides)."""
        import torch.distributed as dist
        dist.barrier(group=self.group)
        self.cabi.call("cek_comm_reset", self.mine, self.cabi.lib().cek_tp_comm_bytes(self.slot_elems, self.world))
        dist.barrier(group=self.group)

    def close(self):
        for p in self.opened:
            self.cabi.lib().cek_ipc_close_handle(p)
        self.opened = []
        if self.mine:
            self.cabi.lib().cek_comm_free(self.mine)
            self.mine = None


def shard_rows(n: int, rank: int, world: int) -> tuple[int, int]:
    """Column-parallel split of n output rows: rank r owns [n r / W, n (r + 1) / W)."""
    return n * rank // world, n * (rank + 1) // world


def gemv_fp8_allgather(comm: TPComm, x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, row0: int,
                       n_full: int, y_off: int, early_weights: bool = False) -> None:
    """Column-parallel FP8 GEMV with its all-gather fused into the epilogue
    (cek_gemv_fp8_allgather): this rank's rows [row0, row0 + w.shape[0]) of
    y = x @ deq(W)^T * scale are stored into every rank's y [M, n_full] at
    byte offset y_off of the comm data area.  Follow the step's calls with
    comm.barrier()."""
    cb = comm.cabi
    M, K = x.shape
    fmt = cb.CEK_E5M2 if w.dtype == torch.float8_e5m2 else cb.CEK_E4M3
    sk = cb.CEK_SCALE_PERT_F32 if scale.numel() == 1 else (
        cb.CEK_SCALE_PERN_F16 if scale.dtype == torch.float16 else cb.CEK_SCALE_PERN_F32)
    cb.call("cek_gemv_fp8_allgather", cb.ptr(x), cb.ptr(w), cb.ptr(scale), M, w.shape[0], K, row0, n_full, y_off,
            cb.io_dtype(x), fmt, sk, cb.ptr(comm.peers), comm.mine, comm.nbytes, comm.rank, comm.world,
            cb.CEK_GEMV_EARLY_WEIGHTS if early_weights else 0, cb.current_stream())


class DecodeChain:
    """One rank's executor of the decode step (module docstring).  `group`
    is the torch.distributed process group of the TP ranks (None at TP=1).
    With `comm` (a TPComm) the down projection and its all-reduce run as the
    fused peer-memory pair of cek_gemv_fp8_allreduce instead of a GEMV
    followed by an NCCL all-reduce."""

    def __init__(self, shards: dict, shape: ChainShape, M: int, device, group=None, world: int = 1,
                 comm: "TPComm | None" = None):
        import esimd_learning_b200 as ops

        self.ops, self.shape, self.M, self.dev, self.group, self.world = ops, shape, M, device, group, world
        self.comm = comm
        self.w = {k: (tuple(t.to(device) for t in v) if isinstance(v, tuple) else
                      (v.to(device) if torch.is_tensor(v) else v)) for k, v in shards.items()}
        lq, lkv, lf = shards["local_q_heads"], shards["local_kv_heads"], shards["local_intermediate"]
        d, h = shape.head_dim, shape.hidden
        self.lq, self.lkv, self.lf = lq, lkv, lf
        self.cos_sin = rope_cache(shape, device)
        f16 = dict(dtype=torch.float16, device=device)
        self.qkv = torch.empty(M, (lq + 2 * lkv) * d, **f16)
        self.act = torch.empty(M, lf, **f16)
        self.out = torch.empty(M, h, **f16)
        self.graph = None

    def step(self, hidden, residual, attn_out, positions):
        """Runs the step on the current stream; returns (out [M, hidden] fp16,
        qkv [M, local qkv] fp16 after norm+RoPE).  residual is updated in place."""
        o, s, w = self.ops, self.shape, self.w
        o.esimd_fused_add_rms_norm_batched_fp8(hidden, residual, w["gamma_attn"], s.eps, *w["qkv"], self.qkv)
        o.esimd_qkv_norm_rope(self.qkv, positions, w["q_norm"], w["k_norm"], self.cos_sin, self.lq, self.lkv,
                              s.head_dim, s.eps, True)
        o.esimd_fused_add_rms_norm_gelu_mul_fp8(attn_out, residual, w["gamma_mlp"], s.eps, *w["gate_up"], self.act)
        wd, sd = w["down"]
        if self.world > 1 and self.comm is not None:
            c, cb = self.comm, self.comm.cabi
            cb.call("cek_gemv_fp8_allreduce", cb.ptr(self.act), cb.ptr(wd), cb.ptr(sd), cb.ptr(self.out),
                    self.M, s.hidden, self.lf, cb.CEK_F16, cb.CEK_E4M3, cb.CEK_SCALE_PERN_F32, cb.ptr(c.peers),
                    c.mine, c.slot_elems, c.rank, c.world, 0, cb.current_stream())
            return self.out, self.qkv
        o.esimd_gemv_fp8_pern(self.act, wd, sd, self.out, s.hidden, self.lf)
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(self.out, group=self.group)
        return self.out, self.qkv

    def capture(self, hidden, residual, attn_out, positions, stream=None):
        """Capture one step into a CUDA graph over these (static) input tensors."""
        st = stream or torch.cuda.Stream(self.dev)
        with torch.cuda.stream(st):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                self.step(hidden, residual, attn_out, positions)
        self.graph = g
        return g
