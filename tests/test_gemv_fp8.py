"""FP8 GEMV on the GPU against the CPU oracle.

Mirrors the reference's tests/test_gemv_fp8.py (shapes, data distributions,
per-N / per-tensor / e5m2 cases, pert-vs-pern consistency) with the stricter
max-abs <= 1e-2 * ||ref||_inf and mean-rel <= 2e-3
(oracle.MAX_ABS_FRAC / oracle.MEAN_REL).  Every case runs through the C ABI
(esimd_learning_b200.cabi) and through the torch op.
"""
import pytest
import torch

from esimd_learning_b200 import cabi
from esimd_learning_b200.workloads import CONFIG1_MS, CONFIG1_SHAPES, gemv_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu

# reference tests/test_gemv_fp8.py:20-21, 48, 337-338, 396
REF_SHAPES_BASIC = [(3072, 2560), (2560, 2048), (20480, 2560), (2560, 10240),
                    (256, 2560), (2048, 128), (3072, 2048), (16, 2048)]
REF_SHAPES_SCALE = [(3072, 2560), (2560, 2048), (20480, 2560), (2560, 10240), (128, 2048),
                    (2560, 10752)]
REF_SHAPES_PERT = [(1024, 1024), (2560, 2048), (512, 2048), (3072, 2048), (128, 2048), (16, 2048),
                   (2048, 512)]


FLAGS = [0, cabi.CEK_GEMV_EARLY_WEIGHTS]


def cabi_gemv(x, w, scale, y, per_tensor=False, flags=0):
    """Call cek_gemv_fp8 through the C ABI."""
    M, K = x.shape
    N = w.shape[0]
    cabi.call("cek_gemv_fp8", cabi.ptr(x), cabi.ptr(w), cabi.ptr(scale), cabi.ptr(y), M, N, K,
              cabi.io_dtype(x), cabi.io_dtype(y), cabi.fp8_format(w),
              cabi.scale_kind(scale, N, per_tensor), flags, cabi.current_stream())
    return y


@pytest.mark.parametrize("flags", FLAGS)
def test_golden_vectors_through_cabi(cuda_device, golden_cases, flags):
    n = 0
    for c in golden_cases:
        if c["kind"] not in ("gemv_pern", "gemv_pert", "gemm_pert"):
            continue
        x = c["input"].to(cuda_device)
        w = c["weight"].to(cuda_device)
        s = c["scale"].to(cuda_device).reshape(-1)
        y = torch.zeros(x.shape[0], c["N"], dtype=x.dtype, device=cuda_device)
        cabi_gemv(x, w, s, y, per_tensor=c["kind"] != "gemv_pern", flags=flags)
        torch.cuda.synchronize()
        O.assert_parity(y, c["ref"], f"{c['kind']} N={c['N']} K={c['K']}")
        n += 1
    assert n >= 20


@pytest.mark.parametrize("N,K", REF_SHAPES_BASIC)
def test_correctness_basic(ext, cuda_device, N, K):
    torch.manual_seed(0)
    weight_fp8 = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(torch.float8_e4m3fn)
    scale = torch.ones(N, dtype=torch.float16)
    x = torch.randn(1, K, dtype=torch.float16) * 0.1
    out = torch.zeros(1, N, dtype=torch.float16, device=cuda_device)
    ext.esimd_gemv_fp8_pern(x.to(cuda_device), weight_fp8.to(cuda_device), scale.to(cuda_device),
                            out, N, K)
    O.assert_parity(out, O.gemv_fp8(x, weight_fp8, scale), f"N={N} K={K}")


@pytest.mark.parametrize("N,K", REF_SHAPES_SCALE)
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_correctness_with_scale(ext, cuda_device, N, K, io):
    torch.manual_seed(1)
    weight_fp8 = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(torch.float8_e4m3fn)
    scale = torch.randn(N, dtype=torch.float16) * 0.1
    x = (torch.rand(1, K, dtype=torch.float16) * 0.1).to(io)
    out = torch.zeros(1, N, dtype=io, device=cuda_device)
    ext.esimd_gemv_fp8_pern(x.to(cuda_device), weight_fp8.to(cuda_device), scale.to(cuda_device),
                            out, N, K)
    O.assert_parity(out, O.gemv_fp8(x, weight_fp8, scale), f"N={N} K={K} {io}")


@pytest.mark.parametrize("N,K", REF_SHAPES_PERT)
def test_pert_correctness(ext, cuda_device, N, K):
    torch.manual_seed(2)
    weight_fp8 = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(torch.float8_e4m3fn)
    scale_t = torch.tensor(0.05 + torch.rand(1).item() * 0.1, dtype=torch.float32)
    x = torch.randn(1, K, dtype=torch.float16) * 0.1
    out = torch.zeros(1, N, dtype=torch.float16, device=cuda_device)
    ext.esimd_gemv_fp8_pert(x.to(cuda_device), weight_fp8.to(cuda_device), scale_t.to(cuda_device),
                            out)
    O.assert_parity(out, O.gemv_fp8(x, weight_fp8, scale_t), f"N={N} K={K}")


@pytest.mark.parametrize("N,K", [(2560, 2048), (512, 2048), (128, 2048)])
def test_pert_vs_pern(ext, cuda_device, N, K):
    """reference tests/test_gemv_fp8.py:361-388 (rel < 0.01)."""
    torch.manual_seed(3)
    w = (torch.randn(N, K, dtype=torch.float16, device=cuda_device) * 0.1).to(torch.float8_e4m3fn)
    x = torch.randn(1, K, dtype=torch.float16, device=cuda_device) * 0.1
    sp = torch.full((N,), 0.073, dtype=torch.float16, device=cuda_device)
    st = torch.tensor(0.073, dtype=torch.float32, device=cuda_device)
    a = torch.zeros(1, N, dtype=torch.float16, device=cuda_device)
    b = torch.zeros(1, N, dtype=torch.float16, device=cuda_device)
    ext.esimd_gemv_fp8_pern(x, w, sp, a, N, K)
    ext.esimd_gemv_fp8_pert(x, w, st, b)
    rel = (a.float() - b.float()).abs().max().item() / a.float().abs().max().item()
    assert rel < 0.01


@pytest.mark.parametrize("N,K", [(1024, 1024), (2560, 2048), (512, 2048), (128, 2048), (16, 2048)])
@pytest.mark.parametrize("per_tensor", [False, True])
def test_e5m2_correctness(ext, cuda_device, N, K, per_tensor):
    torch.manual_seed(4)
    w = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(torch.float8_e5m2)
    x = torch.randn(1, K, dtype=torch.float16) * 0.1
    s = torch.tensor(0.08) if per_tensor else torch.randn(N, dtype=torch.float16) * 0.1
    out = torch.zeros(1, N, dtype=torch.float16, device=cuda_device)
    if per_tensor:
        ext.esimd_gemv_fp8_pert(x.to(cuda_device), w.to(cuda_device), s.to(cuda_device), out)
    else:
        ext.esimd_gemv_fp8_pern(x.to(cuda_device), w.to(cuda_device), s.to(cuda_device), out, N, K)
    O.assert_parity(out, O.gemv_fp8(x, w, s), f"e5m2 N={N} K={K}")


def test_config0_north_star(cuda_device):
    """x ~ N(0,1) [1,4096], W per-row e4m3 (rowabsmax/448), seed 0."""
    x, wq, s = gemv_case(1, 4096, 4096, seed=0)
    y = torch.zeros(1, 4096, dtype=torch.float16, device=cuda_device)
    cabi_gemv(x.to(cuda_device), wq.to(cuda_device), s.to(cuda_device), y)
    torch.cuda.synchronize()
    O.assert_parity(y, O.gemv_fp8(x, wq, s), "config 0")


@pytest.mark.parametrize("flags", FLAGS)
@pytest.mark.parametrize("name", list(CONFIG1_SHAPES))
@pytest.mark.parametrize("M", CONFIG1_MS)
def test_config1_batched(cuda_device, name, M, flags):
    """batched GEMV, M in {1,2,4,8}; down (K=14336) is the split-K case."""
    N, K = CONFIG1_SHAPES[name]
    x, wq, s = gemv_case(M, N, K, seed=0)
    y = torch.zeros(M, N, dtype=torch.float16, device=cuda_device)
    cabi_gemv(x.to(cuda_device), wq.to(cuda_device), s.to(cuda_device), y, flags=flags)
    torch.cuda.synchronize()
    O.assert_parity(y, O.gemv_fp8(x, wq, s), f"config1 {name} M={M} flags={flags}")


@pytest.mark.parametrize("flags", FLAGS)
@pytest.mark.parametrize("M,N,K", [(3, 17, 16), (5, 1, 48), (16, 33, 80), (9, 200, 1040),
                                   (17, 64, 256), (40, 100, 512), (1, 8, 4096), (2, 31, 3088),
                                   (1, 5000, 16384), (8, 300, 9216), (4, 4096, 1040)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_ragged_shapes(cuda_device, M, N, K, io, flags):
    """N not a multiple of the 16-row group, K not a multiple of the 64-k chunk,
    M across token-tile boundaries, mixed fp32 [N] scale."""
    x, wq, s = gemv_case(M, N, K, seed=M * 1000 + N, dtype=io)
    y = torch.full((M, N), float("nan"), dtype=io, device=cuda_device)
    cabi_gemv(x.to(cuda_device), wq.to(cuda_device), s.to(cuda_device), y, flags=flags)
    torch.cuda.synchronize()
    O.assert_parity(y, O.gemv_fp8(x, wq, s), f"M={M} N={N} K={K}")


@pytest.mark.parametrize("flags", FLAGS)
@pytest.mark.parametrize("M,N,K", [(1, 17, 64), (3, 200, 1024), (8, 1001, 512), (7, 33, 2048),
                                   (2, 2371, 14336), (1, 150, 7168), (5, 4096, 4096), (1, 1, 128),
                                   (6, 148 * 16 + 5, 3072), (8, 777, 14336), (4, 4096, 14336),
                                   (9, 1000, 4096), (12, 333, 2048), (16, 4096, 14336), (16, 2049, 8192),
                                   (11, 57, 28672)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_bulk_path_shapes(cuda_device, M, N, K, io, flags):
    """Shapes the bulk-copy GEMV takes (M <= 16, K % 64 == 0): ragged row
    ranges per CTA, partial 16-row blocks, K cut into row pieces (K = 7168,
    14336, 28672), grids smaller than the SM count, one and two token groups,
    x in shared memory, tensor memory and L2.  No bounded wait may give
    up."""
    import ctypes
    x, wq, s = gemv_case(M, N, K, seed=M * 7919 + N, dtype=io)
    y = torch.full((M, N), float("nan"), dtype=io, device=cuda_device)
    cabi_gemv(x.to(cuda_device), wq.to(cuda_device), s.to(cuda_device), y, flags=flags)
    torch.cuda.synchronize()
    O.assert_parity(y, O.gemv_fp8(x, wq, s), f"M={M} N={N} K={K}")
    n = ctypes.c_uint64(99)
    cabi.call("cek_gemv_fp8_timeouts", ctypes.byref(n))
    assert n.value == 0


@pytest.mark.parametrize("flags", FLAGS)
@pytest.mark.parametrize("M,N,K", [(1, 512, 14336), (8, 512, 14336), (1, 1024, 14336), (4, 1, 16384),
                                   (6, 333, 28672), (3, 700, 12288), (8, 1184, 14336), (2, 100, 14336),
                                   (5, 1280, 8192), (7, 40, 8192), (3, 768, 4096)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("per_tensor", [False, True])
def test_cluster_k_split_shapes(cuda_device, M, N, K, io, flags, per_tensor):
    """Shapes with fewer 16-row blocks than SMs and K >= 12288 take the
    cluster K split (4-8 CTAs per row block, 6 at K = 12288, partial sums
    reduced in the leader's shared memory): short shards of tensor-parallel
    weights, ragged last blocks, N = 1; the last three shapes stay on the
    plain bulk path.  Against the oracle; no bounded
    wait may give up; two calls agree bit for bit."""
    import ctypes
    x, wq, s = gemv_case(M, N, K, seed=M * 104729 + N, dtype=io)
    if per_tensor:
        s = s[:1].clone()
    xd, wd, sd = x.to(cuda_device), wq.to(cuda_device), s.to(cuda_device)
    y = torch.full((M, N), float("nan"), dtype=io, device=cuda_device)
    cabi_gemv(xd, wd, sd, y, per_tensor=per_tensor, flags=flags)
    y2 = torch.full((M, N), float("nan"), dtype=io, device=cuda_device)
    cabi_gemv(xd, wd, sd, y2, per_tensor=per_tensor, flags=flags)
    torch.cuda.synchronize()
    ref = O.gemv_fp8(x, wq, s)
    O.assert_parity(y, ref, f"M={M} N={N} K={K}")
    assert torch.equal(y, y2)
    n = ctypes.c_uint64(99)
    cabi.call("cek_gemv_fp8_timeouts", ctypes.byref(n))
    assert n.value == 0


def test_mixed_io_dtypes_cabi(cuda_device):
    """The C ABI allows input and output dtypes to differ (the reference host
    code instantiates all four combinations, fp8_GEMV_v2.h:181-190)."""
    x, wq, s = gemv_case(2, 256, 1024, seed=5)
    for xi, yo in ((torch.float16, torch.bfloat16), (torch.bfloat16, torch.float16)):
        xx = x.to(xi)
        y = torch.zeros(2, 256, dtype=yo, device=cuda_device)
        cabi_gemv(xx.to(cuda_device), wq.to(cuda_device), s.to(cuda_device), y)
        torch.cuda.synchronize()
        O.assert_parity(y, O.gemv_fp8(xx, wq, s, out_dtype=yo), f"{xi}->{yo}")


@pytest.mark.parametrize("flags", FLAGS)
def test_deterministic(cuda_device, flags):
    x, wq, s = gemv_case(4, 4096, 14336, seed=7)
    x, wq, s = x.to(cuda_device), wq.to(cuda_device), s.to(cuda_device)
    a = torch.zeros(4, 4096, dtype=torch.float16, device=cuda_device)
    b = torch.zeros_like(a)
    cabi_gemv(x, wq, s, a, flags=flags)
    cabi_gemv(x, wq, s, b, flags=flags)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_early_weights_back_to_back(ext, cuda_device):
    """With weight prefetch on, a chain of GEMVs where each consumes the
    previous output (only activations depend on the preceding kernel) gives
    the same bits as with prefetch off."""
    dims = [4096, 1024, 2048, 4096]
    ws = [gemv_case(2, dims[i + 1], dims[i], seed=i, device=cuda_device)[1:] for i in range(3)]
    x0 = torch.randn(2, dims[0], device=cuda_device).half()
    outs = []
    for prefetch in (False, True):
        old = ext.esimd_set_weight_prefetch(prefetch)
        try:
            x = x0
            for (wq, s), n, k in zip(ws, dims[1:], dims[:-1]):
                y = torch.empty(2, n, dtype=torch.float16, device=cuda_device)
                ext.esimd_gemv_fp8_pern(x, wq, s, y, n, k)
                x = y
            outs.append(x.clone())
        finally:
            ext.esimd_set_weight_prefetch(old)
    assert torch.equal(outs[0], outs[1])
    assert torch.isfinite(outs[0].float()).all()


def test_reference_dtype_errors(ext, cuda_device):
    """Reference TORCH_CHECK messages (esimd_kernel.sycl:26-37)."""
    x = torch.zeros(1, 64, dtype=torch.float32, device=cuda_device)
    w = torch.zeros(16, 64, dtype=torch.float8_e4m3fn, device=cuda_device)
    s = torch.ones(16, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="input must be fp16 or bf16"):
        ext.esimd_gemv_fp8_pern(x, w, s, torch.zeros(1, 16, dtype=torch.float16, device=cuda_device),
                                16, 64)
    with pytest.raises(RuntimeError, match="same dtype"):
        ext.esimd_gemv_fp8_pern(x.half(), w, s,
                                torch.zeros(1, 16, dtype=torch.bfloat16, device=cuda_device), 16, 64)
    with pytest.raises(RuntimeError, match="invalid argument"):
        ext.esimd_gemv_fp8_pern(torch.zeros(1, 24, dtype=torch.float16, device=cuda_device),
                                torch.zeros(16, 24, dtype=torch.float8_e4m3fn, device=cuda_device), s,
                                torch.zeros(1, 16, dtype=torch.float16, device=cuda_device), 16, 24)


def test_cuda_graph_capture(ext, cuda_device):
    """The op allocates nothing and never syncs: it captures into a CUDA graph."""
    x, wq, s = gemv_case(1, 4096, 4096, seed=0, device=cuda_device)
    y = torch.zeros(1, 4096, dtype=torch.float16, device=cuda_device)
    ext.esimd_gemv_fp8_pern(x, wq, s, y, 4096, 4096)
    ref = y.clone()
    y.zero_()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            ext.esimd_gemv_fp8_pern(x, wq, s, y, 4096, 4096)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)



# reference benchmark_fused cases (tests/test_gemv_fp8.py:299-303) plus ragged ones
MULTI_CASES = [[(3072, 2048), (16, 2048)], [(512, 2048), (512, 2048)], [(128, 2048), (128, 2048)],
               [(100, 1024), (33, 1024), (2000, 1024), (16, 1024)]]


@pytest.mark.parametrize("shapes", MULTI_CASES)
@pytest.mark.parametrize("M", [1, 4, 12])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_fused_multi_gemv(ext, cuda_device, shapes, M, io):
    """esimd_gemv_fp8_pern_fused == the per-matrix oracle GEMVs."""
    K = shapes[0][1]
    torch.manual_seed(M)
    x = (torch.randn(M, K) * 0.5).to(io)
    ws, ss, ys = [], [], []
    for i, (N, _) in enumerate(shapes):
        _, wq, s = gemv_case(1, N, K, seed=100 + i)
        ws.append(wq)
        ss.append(s.half())  # the reference's fp16 per-N scale
        ys.append(torch.zeros(M, N, dtype=io, device=cuda_device))
    ext.esimd_gemv_fp8_pern_fused(x.to(cuda_device), [w.to(cuda_device) for w in ws],
                                  [s.to(cuda_device) for s in ss], ys)
    for wq, s, y in zip(ws, ss, ys):
        O.assert_parity(y, O.gemv_fp8(x, wq, s), f"multi N={wq.shape[0]} M={M}")


def test_fused_multi_gemv_cabi(cuda_device):
    import ctypes
    K, M = 512, 3
    Ns = [64, 200]
    x, _, _ = gemv_case(M, 16, K, seed=1, device=cuda_device)
    parts = [gemv_case(1, N, K, seed=N, device=cuda_device)[1:] for N in Ns]
    ys = [torch.zeros(M, N, dtype=torch.float16, device=cuda_device) for N in Ns]
    P = ctypes.c_void_p * 2
    cabi.call("cek_gemv_fp8_multi", cabi.ptr(x), P(*[cabi.ptr(w) for w, _ in parts]),
              P(*[cabi.ptr(s) for _, s in parts]), P(*[cabi.ptr(y) for y in ys]), (ctypes.c_int64 * 2)(*Ns), 2,
              M, K, cabi.CEK_F16, cabi.CEK_F16, cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, 0, cabi.current_stream())
    torch.cuda.synchronize()
    for (w, s), y in zip(parts, ys):
        O.assert_parity(y, O.gemv_fp8(x.cpu(), w.cpu(), s.cpu()), "cabi multi")
