"""Host-side checks of the reference-driver bridge (reference_harness.py) on
stand-ins for the reference's two programs: the benchmark script gets this
package's model class, the suite driver gets this file as its per-case script
and B200 peaks. (The real programs need a CUDA device and the reference
checkout; the bridge's own logic is what is tested here.)"""

import json
import subprocess
import sys
import textwrap

from transformer_optimization_b200 import reference_harness as rh
from transformer_optimization_b200.model import UserOptimizedTransformer as Ours

FAKE_SCRIPT = textwrap.dedent("""
    import sys
    class BaselineTransformer: pass
    class UserOptimizedTransformer: pass
    def main():
        base = UserOptimizedTransformer.__mro__[1]
        print("args", " ".join(sys.argv[1:]))
        print("class", base.__module__, base.__name__)
        print("optimized: median=1.25 ms")
        return 0
""")

FAKE_RUN_BENCH = textwrap.dedent("""
    import subprocess, sys
    from pathlib import Path
    SCRIPT = Path(__file__).parent / "torch_transformer_benchmark.py"
    PEAK_TFLOPS = {"float32": 24.7, "float16": 48.8, "bfloat16": 49.4}
    SUITES = {"quick": {"default_fp32": []}}
    def main():
        print("suites", ",".join(sorted(SUITES)))
        print("c3args", " ".join(SUITES.get("b200_baseline", {}).get("c3", [])))
        out = subprocess.run([sys.executable, str(SCRIPT), "--batch-size", "2"], capture_output=True, text=True)
        print("script", SCRIPT)
        print("peak16", PEAK_TFLOPS["float16"])
        print(out.stdout.strip())
        print(out.stderr.strip()[-400:])
        return out.returncode
""")


def _fake_reference(tmp_path):
    (tmp_path / "torch_transformer_benchmark.py").write_text(FAKE_SCRIPT)
    (tmp_path / "run_bench.py").write_text(FAKE_RUN_BENCH)
    return tmp_path


def test_script_gets_this_model(tmp_path, capsys):
    ref = _fake_reference(tmp_path)
    assert rh.run_reference_script(ref, ["--batch-size", "4", "--causal"]) == 0
    out = capsys.readouterr().out
    assert "args --batch-size 4 --causal" in out
    assert f"class {Ours.__module__} UserOptimizedTransformer" in out
    assert "optimized: median=1.25 ms" in out


def test_run_bench_uses_this_script_and_b200_peaks(tmp_path):
    ref = _fake_reference(tmp_path)
    code = ("import sys; from transformer_optimization_b200 import reference_harness as rh; "
            f"sys.exit(rh.main(['run-bench', '--reference-dir', {str(ref)!r}]))")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=str(rh._ROOT))
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"script {rh._HERE}" in r.stdout
    assert f"peak16 {rh.b200_peak_tflops()['float16']}" in r.stdout
    assert f"class {Ours.__module__} UserOptimizedTransformer" in r.stdout  # the per-case run went through us
    assert "optimized: median=1.25 ms" in r.stdout
    # BASELINE's c1-c3 shapes are offered as the driver's "b200_baseline" suite
    assert "suites b200_baseline,quick" in r.stdout
    assert ("c3args --batch-size 8 --seq-len 2048 --d-model 1024 --heads 16 --ffn-dim 4096 --layers 12"
            in r.stdout)


def test_b200_peaks(tmp_path):
    m = tmp_path / "peaks.json"
    m.write_text(json.dumps({"bf16_tflops": 1671.5}))
    p = rh.b200_peak_tflops(m)
    assert p["float16"] == p["bfloat16"] == 1671.5 and p["float32"] == 1100.0
    assert rh.b200_peak_tflops(tmp_path / "missing.json")["float16"] == 2250.0
