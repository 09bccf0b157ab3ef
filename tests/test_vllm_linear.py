"""The vLLM-shaped W8A16 linear method (esimd_learning_b200.vllm_linear)
against the oracle: every dispatch branch (GEMV family for M <= 64, the
tcgen05 W8A16 GEMM for M > 64, shapes the GEMM does not take), per-channel
and per-tensor scales, bias, leading batch dims."""
import pytest
import torch

from esimd_learning_b200.vllm_linear import EsimdFp8LinearMethod
from esimd_learning_b200.workloads import make_fp8_weight
from oracle import oracle as O


def _layer(N, K, per_tensor, seed=0):
    m = EsimdFp8LinearMethod()
    layer = torch.nn.Module()
    m.create_weights(layer, K, [N // 2, N - N // 2], K, N, torch.float16, per_tensor=per_tensor)
    gen = torch.Generator().manual_seed(seed)
    wq, sc = make_fp8_weight(N, K, gen)
    if per_tensor:
        sc = torch.tensor([0.07])
    layer.weight.data = wq
    layer.weight_scale.data = sc
    m.process_weights_after_loading(layer)
    return m, layer, wq, sc


def test_create_weights_shapes():
    m = EsimdFp8LinearMethod()
    layer = torch.nn.Module()
    m.create_weights(layer, 256, [128, 64], 256, 192, torch.bfloat16)
    assert layer.weight.shape == (192, 256) and layer.weight.dtype == torch.float8_e4m3fn
    assert layer.weight_scale.shape == (192,) and layer.logical_widths == [128, 64]
    with pytest.raises(ValueError):
        EsimdFp8LinearMethod(torch.float16)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 5, 33, 200])
@pytest.mark.parametrize("per_tensor", [False, True])
@pytest.mark.parametrize("N,K", [(512, 1024), (1000, 576)])
def test_apply_matches_oracle(cuda_device, M, per_tensor, N, K):
    m, layer, wq, sc = _layer(N, K, per_tensor, seed=M)
    layer.to(cuda_device)
    gen = torch.Generator().manual_seed(M + 1)
    x = torch.randn(M, K, generator=gen).half()
    bias = torch.randn(N, generator=gen).half()
    y = m.apply(layer, x.to(cuda_device), bias.to(cuda_device))
    torch.cuda.synchronize()
    ref = (O.gemv_fp8(x, wq, sc).float() + bias.float()).half()
    O.assert_parity(y, ref, f"M={M} N={N} K={K} per_tensor={per_tensor}")


@pytest.mark.gpu
def test_apply_batch_dims_bf16(cuda_device):
    m, layer, wq, sc = _layer(256, 512, False, seed=3)
    layer.to(cuda_device)
    x = torch.randn(2, 3, 512).bfloat16()
    y = m.apply(layer, x.to(cuda_device))
    assert y.shape == (2, 3, 256)
    O.assert_parity(y.reshape(6, 256), O.gemv_fp8(x.reshape(6, 512), wq, sc), "batch dims")
