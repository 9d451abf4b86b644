"""Run the reference's own benchmark driver with this build's model.

The reference measures its hot path with two programs: the benchmark script
torch_transformer_benchmark.py (`main`, torch_transformer_benchmark.py:
5135-5320: builds BaselineTransformer and UserOptimizedTransformer, copies the
weights, checks accuracy, times both, prints "baseline : median=... ms",
"optimized: median=... ms", "speedup : ...x" and "summary: PASS | ...") and
the suite driver run_bench.py, which runs that script once per case as a
subprocess and parses those lines (run_bench.py:254-258, 261-314).

This module lets both run unchanged against a checkout of the reference:

    python -m transformer_optimization_b200.reference_harness run-bench \\
        --reference-dir REF [run_bench.py arguments, e.g. --suite user_matrix]

imports REF/run_bench.py, points its SCRIPT at this file and its PEAK_TFLOPS at
B200 figures, and calls its main(). run_bench then starts this file as the
per-case script; in that role it imports REF/torch_transformer_benchmark.py,
puts this package's UserOptimizedTransformer in place of the reference's
class, and calls the reference's main() with the same arguments, so the
printed lines are the reference's own. For an fp32 model the class reports
the precision it computes in (fp16 tensor cores) with the reference's
"-> ENABLE fp16-GEMM" line when TJ_DEBUG_GATE is set, which run_bench uses to
pick the peak its MFU divides by (run_bench.py:271-281, 363-369).

A single case runs the same way without run_bench:

    TFB_REFERENCE_DIR=REF python transformer_optimization_b200/reference_harness.py [script arguments]
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path
from types import ModuleType
from typing import List, Optional

import torch

_HERE = Path(__file__).resolve()
_ROOT = _HERE.parent.parent
ENV_REFERENCE_DIR = "TFB_REFERENCE_DIR"

# Dense per-GPU peaks by model dtype (TFLOP/s), the denominators run_bench's
# MFU uses. fp16/bf16: the measured cuBLAS bf16 GEMM rate of this pool's B200s
# when MEASURED_PEAKS.json is present (the fp16 and bf16 tensor rates are the
# same), else NVIDIA's dense 2250. float32: NVIDIA's dense TF32 figure (the
# reference's fp32 baseline runs on TF32 tensor cores when they are enabled).
B200_NOMINAL_TFLOPS = {"float32": 1100.0, "float16": 2250.0, "bfloat16": 2250.0}


def b200_peak_tflops(measured: Optional[Path] = None) -> dict:
    peaks = dict(B200_NOMINAL_TFLOPS)
    path = measured if measured is not None else _ROOT / "MEASURED_PEAKS.json"
    try:
        bf16 = float(json.loads(Path(path).read_text())["bf16_tflops"])
        peaks["float16"] = peaks["bfloat16"] = bf16
    except (OSError, KeyError, ValueError, TypeError):
        pass
    return peaks


def _load(name: str, path: Path) -> ModuleType:
    if not path.is_file():
        raise FileNotFoundError(f"{path} not found: pass the directory of a reference checkout")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _reporting_class(base):
    """The package's UserOptimizedTransformer plus the reference's precision
    report: for an fp32 model on CUDA, one stderr line per input shape in the
    reference's format when TJ_DEBUG_GATE is set (no parameters or buffers
    are added, so the state_dict contract is unchanged)."""

    class UserOptimizedTransformer(base):
        def forward(self, x, valid_token_mask=None):
            if os.environ.get("TJ_DEBUG_GATE") and x.dtype.is_floating_point and x.is_cuda:
                seen = self.__dict__.setdefault("_tfb_reported", set())
                key = (tuple(x.shape), self.config.causal, valid_token_mask is not None)
                if key not in seen and next(self.parameters()).dtype == torch.float32:
                    print(f"[fp16-gemm-policy] shape={tuple(x.shape)} causal={self.config.causal} "
                          f"mask_active={valid_token_mask is not None} -> ENABLE fp16-GEMM", file=sys.stderr)
                    seen.add(key)
            return super().forward(x, valid_token_mask)

    UserOptimizedTransformer.__qualname__ = base.__qualname__
    return UserOptimizedTransformer


def run_reference_script(reference_dir: Path, argv: List[str]) -> int:
    """The reference's benchmark script with this package's model class."""
    if str(_ROOT) not in sys.path:
        sys.path.insert(0, str(_ROOT))
    from transformer_optimization_b200 import UserOptimizedTransformer

    reference_dir = Path(reference_dir)
    sys.path.insert(0, str(reference_dir))
    ref = _load("torch_transformer_benchmark", reference_dir / "torch_transformer_benchmark.py")
    ref.UserOptimizedTransformer = _reporting_class(UserOptimizedTransformer)
    sys.argv = [str(reference_dir / "torch_transformer_benchmark.py"), *argv]
    return int(ref.main() or 0)


# BASELINE's configs that the reference's eager fp32 model can run densely
# on one B200 (c4 and c5 need its query-tiled / streamed protocols), as
# run_bench case arguments in the reference's own flag vocabulary
# (torch_transformer_benchmark.py:5028-5034); added to run_bench's suites as
# "b200_baseline".
B200_SUITE = {
    "c1": ["--batch-size", "2", "--seq-len", "128", "--d-model", "256", "--heads", "4", "--ffn-dim", "1024",
           "--layers", "2"],
    "c2": ["--batch-size", "1", "--seq-len", "64", "--d-model", "512", "--heads", "8", "--ffn-dim", "2048",
           "--layers", "6"],
    "c3": ["--batch-size", "8", "--seq-len", "2048", "--d-model", "1024", "--heads", "16", "--ffn-dim", "4096",
           "--layers", "12"],
}


def run_bench(reference_dir: Path, argv: List[str]) -> int:
    """The reference's suite driver with this file as its per-case script and
    B200 peaks for its MFU, plus the "b200_baseline" suite (B200_SUITE).
    run_bench writes its results JSON beside its per-case script, i.e. under
    this package's agent/results/ (run_bench.py:527-530)."""
    reference_dir = Path(reference_dir).resolve()
    os.environ[ENV_REFERENCE_DIR] = str(reference_dir)
    rb = _load("run_bench", reference_dir / "run_bench.py")
    rb.SCRIPT = _HERE
    rb.PEAK_TFLOPS = b200_peak_tflops()
    if hasattr(rb, "SUITES"):
        rb.SUITES["b200_baseline"] = {k: list(v) for k, v in B200_SUITE.items()}
    sys.argv = [str(reference_dir / "run_bench.py"), *argv]
    return int(rb.main() or 0)


def main(argv: Optional[List[str]] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "run-bench":
        rest = argv[1:]
        if "--reference-dir" not in rest:
            raise SystemExit("run-bench needs --reference-dir <reference checkout>")
        i = rest.index("--reference-dir")
        if i + 1 >= len(rest):
            raise SystemExit("--reference-dir needs a value")
        ref_dir = rest[i + 1]
        return run_bench(Path(ref_dir), rest[:i] + rest[i + 2:])
    ref_dir = os.environ.get(ENV_REFERENCE_DIR)
    if not ref_dir:
        raise SystemExit(f"set {ENV_REFERENCE_DIR} to the reference checkout (or use the run-bench mode)")
    return run_reference_script(Path(ref_dir), argv)


if __name__ == "__main__":
    raise SystemExit(main())
