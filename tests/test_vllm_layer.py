"""A real vLLM 0.22 linear layer (ReplicatedLinear) built with this package's
quantization method ("esimd_fp8", esimd_learning_b200.vllm_plugin): weights
loaded by vLLM's own weight_loader, forward at decode (GEMV family) and
prefill (tcgen05 W8A16 GEMM, with and without the dequantised-weight
workspace) token counts, against the oracle.  Runs in a child process
(tests/vllm_layer_worker.py) so vLLM's import stays out of the test process."""
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu


def test_vllm_replicated_linear_on_esimd_kernels(cuda_device):
    worker = Path(__file__).resolve().parent / "vllm_layer_worker.py"
    r = subprocess.run([sys.executable, str(worker)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert any(l.startswith("{") for l in r.stdout.splitlines())
