"""Child process of tests/test_vllm_layer.py: registers the "esimd_fp8"
quantization method with vLLM, builds vLLM ReplicatedLinear layers with it,
loads FP8 weights through the layer's own weight_loader and runs forward at
decode and prefill token counts, checking each output against the CPU
oracle.  Prints one JSON line; exits non-zero on a mismatch."""
import json
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "python"))
sys.path.insert(0, str(ROOT))

from esimd_learning_b200 import vllm_plugin  # noqa: E402
from esimd_learning_b200.workloads import make_fp8_weight  # noqa: E402
from oracle import oracle as O  # noqa: E402


def main():
    from vllm.config import VllmConfig, set_current_vllm_config
    from vllm.model_executor.layers.linear import ReplicatedLinear
    from vllm.model_executor.layers.quantization import get_quantization_config

    cfg_cls = vllm_plugin.register()
    assert get_quantization_config(vllm_plugin.NAME) is cfg_cls
    dev = torch.device("cuda", 0)
    res = {}
    with set_current_vllm_config(VllmConfig()):
        for per_tensor in (False, True):
            N, K = 2048, 1024
            qc = cfg_cls.from_config({"fmt": "e4m3", "per_tensor": per_tensor})
            layer = ReplicatedLinear(K, N, bias=True, params_dtype=torch.float16, quant_config=qc,
                                     disable_tp=True, return_bias=False).to(dev)
            gen = torch.Generator().manual_seed(3)
            wq, sc = make_fp8_weight(N, K, gen)
            if per_tensor:
                sc = torch.tensor([0.02])
            bias = (torch.randn(N, generator=gen) * 0.1).half()
            layer.weight_loader(layer.weight, wq.to(dev))
            layer.weight_loader(layer.weight_scale, sc.to(dev))
            layer.weight_loader(layer.bias, bias.to(dev))
            layer.quant_method.process_weights_after_loading(layer)
            for M in (1, 8, 100, 300):
                x = torch.randn(M, K, generator=gen).half()
                y = layer(x.to(dev))
                torch.cuda.synchronize()
                ref = (O.gemv_fp8(x, wq, sc, out_dtype=torch.float32) + bias.float()).half()
                m = O.assert_parity(y, ref, f"vLLM layer per_tensor={per_tensor} M={M}")
                res[f"{'pert' if per_tensor else 'pern'}_M{M}"] = round(m["max_abs_frac"], 6)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
