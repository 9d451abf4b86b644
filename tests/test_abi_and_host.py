"""CPU-only checks of the boundary and the host logic (no kernel launches).

* the C-ABI library loads and exports every function include/tfb200.h
  declares, with the argument count the ctypes binding uses;
* the module tree / state_dict contract with the reference
  (torch_transformer_benchmark.py:135-248, 4328-4338);
* TransformerConfig validation (torch_transformer_benchmark.py:52-70) and the
  reference's FLOP convention (run_bench.py:102-113);
* the product path refuses CPU tensors instead of falling back.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

from oracle import reference_model as om
from transformer_optimization_b200 import (NAMED_CONFIGS, BaselineTransformer, TransformerConfig,
                                           UserOptimizedTransformer, copy_model_weights, count_causal_flops,
                                           count_dense_flops)
from transformer_optimization_b200 import _abi

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "tfb200.h"


def _declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(?:int64_t|int|const char\s*\*)\s*(tf_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a for a in m.group(2).split(",") if a.strip() and a.strip() != "void"]
        out[m.group(1)] = len(args)
    return out


@pytest.fixture(scope="module")
def lib():
    if not _abi.LIB_PATH.exists():
        from transformer_optimization_b200 import build
        build.build()
    return _abi.load()


def test_header_symbols_exported(lib):
    declared = _declared()
    assert set(declared) == set(_abi.SIGNATURES), "ctypes binding and header disagree"
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (tf_\w+)", nm))
    for name, nargs in declared.items():
        assert name in exported, f"{name} not exported"
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)
        assert len(_abi.SIGNATURES[name][0]) == nargs, f"{name}: header has {nargs} args"


def test_abi_version_and_error_string(lib):
    assert lib.tf_abi_version() == 11
    assert isinstance(lib.tf_last_error(), bytes)


def test_missing_library_is_loud(tmp_path):
    with pytest.raises(RuntimeError, match="missing"):
        _abi.load(tmp_path / "nope.so")


def test_state_dict_contract():
    cfg = TransformerConfig(2, 16, 64, 4, 128, 3, False)
    torch.manual_seed(0)
    opt = UserOptimizedTransformer(cfg)
    p = om.init_params(cfg, 0)
    sd = opt.state_dict()
    assert list(sd) == list(p)
    assert all(torch.equal(sd[k], p[k]) for k in p)  # same init draws under the same seed
    opt.load_state_dict(p, strict=True)
    base = BaselineTransformer(cfg)
    copy_model_weights(opt, base, strict=True)
    # no parameters or buffers beyond the reference's
    assert len(list(opt.buffers())) == 0
    assert sum(1 for _ in opt.parameters()) == sum(1 for _ in base.parameters())


def test_product_refuses_cpu():
    cfg = NAMED_CONFIGS["c1"]
    m = UserOptimizedTransformer(cfg)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(2, 128, 256))
    with pytest.raises(NotImplementedError):
        BaselineTransformer(cfg)(torch.randn(2, 128, 256))


def test_config_validation():
    with pytest.raises(ValueError, match="divisible"):
        TransformerConfig(1, 8, 30, 4, 8, 1, False).validate()
    for bad in ((0, 8, 32, 4, 8, 1), (1, 0, 32, 4, 8, 1), (1, 8, 32, 4, 0, 1), (1, 8, 32, 4, 8, 0)):
        with pytest.raises(ValueError):
            TransformerConfig(*bad, False).validate()


def test_flop_convention():
    # run_bench.py:102-113 numbers for the BASELINE configs
    assert count_dense_flops(NAMED_CONFIGS["c1"]) == 872415232
    assert abs(count_dense_flops(NAMED_CONFIGS["c3"]) / 1e12 - 6.597) < 1e-3
    assert abs(count_dense_flops(NAMED_CONFIGS["c4"]) / 1e12 - 422.2) < 0.1
    assert abs(count_dense_flops(NAMED_CONFIGS["c5"]) / 1e12 - 173.9) < 0.1
    c = TransformerConfig(1, 100, 64, 2, 64, 1, True)
    assert count_causal_flops(c) < count_dense_flops(c)


def test_mask_resolution_memoised(monkeypatch):
    m = UserOptimizedTransformer(NAMED_CONFIGS["c1"])
    mask = torch.ones(2, 128, dtype=torch.bool)
    calls = []
    real_all = torch.all
    monkeypatch.setattr(torch, "all", lambda t: calls.append(1) or real_all(t))
    assert m._resolve_mask_active(mask) is False
    assert m._resolve_mask_active(mask) is False
    assert len(calls) == 1
    mask2 = mask.clone()
    mask2[1, 100:] = False
    assert m._resolve_mask_active(mask2) is True
    assert m._resolve_mask_active(None) is False


def test_splitk_choice():
    """Few-row projections take the split-K form (fewer than a quarter of the
    SMs would get a 128x64 tile, K >= 256); the c3-sized ones do not."""
    from transformer_optimization_b200.model import _splitk
    assert _splitk(64, 512, 2048, 148) == 0      # c2 FFN-out
    assert _splitk(256, 256, 1024, 148) == 0     # c1 FFN-out
    assert _splitk(256, 768, 256, 148) == 0      # c1 QKV
    assert _splitk(256, 768, 128, 148) is None   # K too short to split
    assert _splitk(16384, 3072, 1024, 148) is None
    assert _splitk(64, 512, 2048, 16) is None    # few SMs: enough tiles already


def test_bench_algorithmic_bytes():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    cfg = NAMED_CONFIGS["c3"]
    m, d, f = 16384, 1024, 4096
    expect = (2 * (m * d + 3 * d * d + 3 * m * d) + 2 * (m * d + f * d + m * f)
              + 2 * (m * d + d * d) + 8 * m * d + 2 * (m * f + d * f) + 8 * m * d) / 4
    assert bench.algo_bytes_per_gemm(cfg) == expect
    assert 140e6 < bench.C3_GEMM_DRAM_BYTES_PER_LAUNCH < expect  # measured DRAM bytes below algorithmic


def _record_schedule(monkeypatch, cfg, m_rows, chunk_budget=None, overlap_ln=True):
    """Run the model's per-layer schedule with the kernel wrappers replaced
    by recorders (no GPU): returns [(wrapper, kwargs)] in call order."""
    import types
    from transformer_optimization_b200 import kernels as K
    calls = []

    def rec(name, ret):
        def f(*a, **kw):
            calls.append((name, kw))
            return ret(*a, **kw)
        return f

    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda dev: types.SimpleNamespace(multi_processor_count=148,
                                                          total_memory=183359 * 2**20))
    monkeypatch.setattr(K, "splitk_workspace_bytes", lambda m, n, k, splits=0: 1024)
    monkeypatch.setattr(K, "ln_residual", rec("ln", lambda x, *a, **kw: (x, torch.zeros(1))))
    monkeypatch.setattr(K, "linear", rec("linear", lambda *a, **kw: None))
    monkeypatch.setattr(K, "flash_attention", rec("flash", lambda *a, **kw: (None, None)))
    monkeypatch.setattr(K, "linear_residual", rec("res", lambda a, w, b, x_in, x_out, *r, **kw: x_out))
    monkeypatch.setattr(K, "linear_residual_ln",
                        rec("res_ln", lambda a, w, b, x_in, x_out, *r, **kw: (x_out, torch.zeros(1))))
    monkeypatch.setattr(K, "ln_ready", rec("ln_ready", lambda x, *a, **kw: torch.zeros(1)))
    monkeypatch.setattr(K, "ready_counters", lambda rows, dev: torch.zeros((rows + 7) // 8 + 2, dtype=torch.int32))
    model = UserOptimizedTransformer(cfg)
    model.ffn_chunk_budget_bytes = chunk_budget
    model.overlap_ln = overlap_ln
    model._forward_core(torch.zeros(1, m_rows, cfg.d_model), None, False)
    return calls


def test_forward_schedule_few_rows(monkeypatch):
    """c2 (64 rows): every projection takes the split-K form and each
    residual site runs the following LayerNorm in its reduce kernel (the next
    layer's norm1, the final norm after the last layer, fp32 out)."""
    cfg = NAMED_CONFIGS["c2"]
    calls = _record_schedule(monkeypatch, cfg, 64)
    names = [c[0] for c in calls]
    assert names == ["ln"] + ["linear", "flash", "res_ln", "linear", "res_ln"] * cfg.num_layers
    assert all(kw.get("splits") == 0 for n, kw in calls if n in ("linear", "res_ln"))
    assert calls[-1][1]["out_dtype"] == torch.float32 and calls[-1][1]["mask_out"] is False


def test_forward_schedule_many_rows(monkeypatch):
    """c3-sized rows: no split-K; residual sites in the GEMM epilogue, each
    followed by a LayerNorm that overlaps the GEMM's tail through the same
    ready counters (norm2, the next layer's norm1, the final norm in fp32)."""
    cfg = TransformerConfig(8, 2048, 1024, 16, 4096, 2, False)
    calls = _record_schedule(monkeypatch, cfg, 8 * 2048)  # the 16 384 rows as one sequence
    names = [c[0] for c in calls]
    assert names == ["ln"] + ["linear", "flash", "res", "ln_ready", "linear", "res", "ln_ready"] * cfg.num_layers
    assert all(kw.get("splits") is None for n, kw in calls if n == "linear")
    readies = [kw["ready"] for n, kw in calls if n == "res"]
    assert all(r is readies[0] and r.numel() == 8 * 2048 // 8 + 2 for r in readies)
    assert calls[-1][1]["out_dtype"] == torch.float32 and calls[-1][1]["mask_out"] is False


def test_forward_schedule_many_rows_no_overlap(monkeypatch):
    """overlap_ln = False: each LayerNorm runs after its GEMM has finished."""
    cfg = TransformerConfig(8, 2048, 1024, 16, 4096, 2, False)
    calls = _record_schedule(monkeypatch, cfg, 8 * 2048, overlap_ln=False)
    names = [c[0] for c in calls]
    assert names == ["ln", "linear", "flash", "res", "ln", "linear", "res"] * cfg.num_layers + ["ln"]
    assert all(kw.get("ready") is None for n, kw in calls if n == "res")


def test_ffn_chunk_decision():
    """The FFN runs in row chunks only when the [rows, ffn_dim] hidden would
    exceed the budget (torch_transformer_benchmark.py:3886-3908): chunks
    are a power of two of rows that fits, at least 256, at most all rows."""
    from transformer_optimization_b200.model import FFN_CHUNK_BUDGET_FRAC, ffn_chunk_rows
    b200 = int(183359 * 2**20 * FFN_CHUNK_BUDGET_FRAC)
    for name in ("c1", "c2", "c3", "c4", "c5"):  # BASELINE's configs never chunk on a B200
        c = NAMED_CONFIGS[name]
        assert ffn_chunk_rows(c.batch_size * c.seq_len, c.ffn_dim, 2, b200) is None
    assert ffn_chunk_rows(1000, 1024, 2, 300 * 1024 * 2) == 256
    assert ffn_chunk_rows(1000, 1024, 2, 600 * 1024 * 2) == 512
    assert ffn_chunk_rows(1000, 1024, 2, 10) == 256          # floor
    assert ffn_chunk_rows(200, 1024, 2, 10) == 200           # never more than the rows
    assert ffn_chunk_rows(1000, 1024, 2, 1000 * 1024 * 2) is None
    # the reference's row-14 shape on a 16 GB card would chunk; on a B200 it does not
    assert ffn_chunk_rows(32 * 100000, 1024, 2, b200) is None
    assert ffn_chunk_rows(32 * 100000, 1024, 2, int(16e9 * FFN_CHUNK_BUDGET_FRAC)) == 1 << 20


def test_forward_schedule_chunked_ffn(monkeypatch):
    """Over budget: each layer's FFN becomes FFN-in + FFN-out per row chunk,
    in place on the residual stream, followed by the next LayerNorm site."""
    cfg = TransformerConfig(1, 1000, 256, 4, 1024, 2, False)
    calls = _record_schedule(monkeypatch, cfg, 1000, chunk_budget=300 * 1024 * 2)
    names = [c[0] for c in calls]
    # (1000 rows: the out-projection takes the split-K form, whose reduce runs norm2)
    assert names == (["ln", "linear", "flash", "res_ln"] + ["linear", "res"] * 4) * cfg.num_layers + ["ln"]


C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "tfb200.h"

int main(void) {
  printf("abi %d\n", tf_abi_version());
  /* null operands: refused with a status code and a message, whether or not
     a GPU is present (no device: TF_ERR_DEVICE; device: a shape/alignment code) */
  int rc = tf_gemm(NULL, 64, NULL, 64, NULL, NULL, 64, 64, 64, 64, TF_EPI_BIAS, NULL);
  const char* msg = tf_last_error();
  printf("rc %d msg_len %d\n", rc, (int)strlen(msg));
  return (rc != TF_OK && strlen(msg) > 0) ? 0 : 1;
}
"""


def test_c_program_binds_the_abi(lib, tmp_path):
    """The header is plain C: a C program compiled by gcc against
    include/tfb200.h links libtfb200.so and gets a refused call's status code
    and message (the binding a C, cgo or other FFI host would use)."""
    import shutil
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    src = tmp_path / "abi_smoke.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "abi_smoke"
    libdir = _abi.LIB_PATH.parent
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src), "-o", str(exe),
                    f"-L{libdir}", "-l:libtfb200.so", f"-Wl,-rpath,{libdir}"], check=True, capture_output=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert f"abi {lib.tf_abi_version()}" in res.stdout
