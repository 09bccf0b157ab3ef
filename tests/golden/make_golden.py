"""Generate tests/golden/reference_vectors.pt from the reference's own test oracles.

The reference (jilongW/esimd_learning) ships no golden vectors and its kernels
need an Intel GPU, but its tests compute their expected values on the host
with plain torch.  This script runs exactly those expressions, taken from the
reference test sources with `ast` (never copied into this repository), on
small seeded CPU inputs drawn the way the reference tests draw them, and
stores inputs and expected outputs:

  gemv_pern  tests/test_gemv_fp8.py:58-59   (fp16 per-N scale, e4m3)
             tests/test_gemv_fp8.py:406-407 (fp16 per-N scale, e5m2)
  gemv_pert  tests/test_gemv_fp8.py:349-350 (fp32 per-tensor scale)
  gemm_pert  tests/test_gemm_fp8.py:35-36   (M x K input, per-tensor scale)
  rmsnorm    tests/test_fused_add_rms_norm_batched_fp8.py:7-27
             (ref_fused_add_rms_norm_batched_fp16, called as a function)

Usage: python tests/golden/make_golden.py [REFERENCE_ROOT]
(default REFERENCE_ROOT: the CEK_REFERENCE_ROOT environment variable).  Only
needed when the fixture is regenerated; the tests read the committed .pt file.
"""
from __future__ import annotations

import ast
import os
import sys
from pathlib import Path

import torch

OUT = Path(__file__).resolve().parent / "reference_vectors.pt"


def _stmt_source(path: Path, lineno: int) -> str:
    """Source of the statement that starts at `lineno` in `path`."""
    src = path.read_text()
    tree = ast.parse(src)
    for node in ast.walk(tree):
        if isinstance(node, ast.stmt) and getattr(node, "lineno", None) == lineno:
            return ast.get_source_segment(src, node)
    raise LookupError(f"no statement at {path}:{lineno}")


def _function(path: Path, name: str):
    src = path.read_text()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            ns = {"torch": torch}
            exec(compile(ast.Module(body=[node], type_ignores=[]), str(path), "exec"), ns)
            return ns[name]
    raise LookupError(f"{name} not in {path}")


def _run(stmts: list[str], ns: dict) -> dict:
    for s in stmts:
        exec(s, {"torch": torch}, ns)
    return ns


def main(ref_root: Path) -> None:
    tg = ref_root / "tests" / "test_gemv_fp8.py"
    tm = ref_root / "tests" / "test_gemm_fp8.py"
    tr = ref_root / "tests" / "test_fused_add_rms_norm_batched_fp8.py"
    pern = [_stmt_source(tg, 58), _stmt_source(tg, 59)]
    pern_e5 = [_stmt_source(tg, 406), _stmt_source(tg, 407)]
    pert = [_stmt_source(tg, 349), _stmt_source(tg, 350)]
    gemm = [_stmt_source(tm, 35), _stmt_source(tm, 36)]
    ref_norm = _function(tr, "ref_fused_add_rms_norm_batched_fp16")

    torch.manual_seed(1234)
    cases = []
    for fmt, stmts in ((torch.float8_e4m3fn, pern), (torch.float8_e5m2, pern_e5)):
        for N, K in ((64, 2048), (96, 512), (16, 2048), (40, 1024)):
            w = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(fmt)
            scale = torch.randn(N, dtype=torch.float16) * 0.1
            x = torch.rand(1, K, dtype=torch.float16) * 0.1
            ns = _run(stmts, {"input_t": x, "weight_fp8": w, "scale": scale})
            cases.append({"kind": "gemv_pern", "input": x, "weight": w, "scale": scale,
                          "N": N, "K": K, "ref": ns["ref"].float()})
    for N, K in ((64, 2048), (128, 512), (16, 2048)):
        w = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(torch.float8_e4m3fn)
        scale_val = 0.05 + torch.rand(1).item() * 0.1
        x = torch.randn(1, K, dtype=torch.float16) * 0.1
        ns = _run(pert, {"input_t": x, "weight_fp8": w, "scale_val": scale_val})
        cases.append({"kind": "gemv_pert", "input": x, "weight": w,
                      "scale": torch.tensor(scale_val, dtype=torch.float32),
                      "N": N, "K": K, "ref": ns["ref"].float()})
    for io in (torch.float16, torch.bfloat16):
        for fmt in (torch.float8_e4m3fn, torch.float8_e5m2):
            for M, N, K in ((1, 64, 512), (4, 48, 1024), (16, 64, 256), (64, 32, 512)):
                w = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(fmt)
                scale_val = 0.05 + torch.rand(1).item() * 0.1
                x = torch.randn(M, K, dtype=io) * 0.1
                ns = _run(gemm, {"input_t": x, "weight_fp8": w, "scale_val": scale_val})
                cases.append({"kind": "gemm_pert", "input": x, "weight": w,
                              "scale": torch.tensor(scale_val, dtype=torch.float32),
                              "N": N, "K": K, "ref": ns["ref"].float()})
    torch.manual_seed(42)
    for M in (1, 3):
        for K in (512, 1024, 2048, 4096):
            h = torch.randn(M, K, dtype=torch.float16)
            r = torch.randn(M, K, dtype=torch.float16)
            w = torch.randn(K, dtype=torch.float16) * 0.1 + (1.0 if M == 3 else 0.0)
            ref_r, ref_n = ref_norm(h, r, w, 1e-6)
            cases.append({"kind": "rmsnorm", "hidden": h, "residual": r, "weight": w, "eps": 1e-6,
                          "K": K, "ref_residual": ref_r, "ref_normed": ref_n})
    torch.save({"source": "reference tests' host-side oracle expressions", "cases": cases}, OUT)
    print(f"wrote {len(cases)} cases to {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CEK_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (or set CEK_REFERENCE_ROOT)")
    main(Path(root))
