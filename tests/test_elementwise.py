"""GeLU(tanh)-and-mul, q/k-norm + RoPE and per-token e4m3 quantisation on the
GPU against the oracle (BASELINE config 4 shapes)."""
import pytest
import torch

from esimd_learning_b200 import cabi
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,d", [(1, 28672), (16, 3584), (7, 8), (3, 1000)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_gelu_and_mul(ext, cuda_device, M, d, io):
    torch.manual_seed(0)
    x = (torch.randn(M, 2 * d) * 2).to(io)
    out = torch.zeros(M, d, dtype=io, device=cuda_device)
    ext.esimd_gelu_and_mul(x.to(cuda_device), out)
    O.assert_parity(out, O.gelu_and_mul(x), f"M={M} d={d}")


@pytest.mark.parametrize("hq,hkv,D", [(64, 8, 128), (8, 1, 128), (16, 4, 64), (4, 2, 256)])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_qkv_norm_rope(ext, cuda_device, hq, hkv, D, neox, io):
    torch.manual_seed(1)
    M = 5
    qkv = torch.randn(M, (hq + 2 * hkv) * D).to(io)
    pos = torch.randint(0, 8192, (M,), dtype=torch.int64)
    qw = (1 + 0.1 * torch.randn(D)).to(io)
    kw = (1 + 0.1 * torch.randn(D)).to(io)
    cs = O.rope_cos_sin_cache(8192, D, 500000.0)
    ref = O.qkv_norm_rope(qkv, pos, qw, kw, cs, hq, hkv, D, 1e-6, neox)
    qd = qkv.to(cuda_device)
    ext.esimd_qkv_norm_rope(qd, pos.to(cuda_device), qw.to(cuda_device), kw.to(cuda_device),
                            cs.to(cuda_device), hq, hkv, D, 1e-6, neox)
    qc = qd.cpu()
    v0 = (hq + hkv) * D
    assert torch.equal(qc[:, v0:], qkv[:, v0:])
    O.assert_parity(qc[:, :v0], ref[:, :v0], f"hq={hq} hkv={hkv} D={D} neox={neox}")


@pytest.mark.parametrize("M,K", [(1, 4096), (2048, 4096), (5, 8), (33, 1000), (7, 8192), (3, 16384)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_quant_fp8_per_token_bit_exact(ext, cuda_device, M, K, io):
    torch.manual_seed(2)
    a = torch.randn(M, K).to(io)
    a[0, :] = 0 if M > 3 else a[0, :]
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=cuda_device)
    s = torch.empty(M, dtype=torch.float32, device=cuda_device)
    ext.esimd_quant_fp8_per_token(a.to(cuda_device), q, s)
    rq, rs = O.quant_fp8_per_token(a)
    assert torch.equal(s.cpu(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


def test_quant_through_cabi(cuda_device):
    a = torch.randn(4, 512, dtype=torch.float16, device=cuda_device)
    q = torch.empty(4, 512, dtype=torch.float8_e4m3fn, device=cuda_device)
    s = torch.empty(4, dtype=torch.float32, device=cuda_device)
    cabi.call("cek_quant_fp8_per_token", cabi.ptr(a), cabi.ptr(q), cabi.ptr(s), 4, 512, cabi.CEK_F16,
              cabi.current_stream())
    torch.cuda.synchronize()
    rq, rs = O.quant_fp8_per_token(a.cpu())
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
