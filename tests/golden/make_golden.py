"""Generate the golden fixtures that pin the oracle to the real reference.

Run in the build container, where the reference checkout is importable:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own `torch_transformer_benchmark` module and, for
each case below, builds the model exactly as the benchmark definition says
(`torch.manual_seed(seed)`, construct `BaselineTransformer` or
`QueryTiledBaselineTransformer`, then `x = torch.randn(B, S, D)` on the CPU),
runs the reference's own eager forward in fp32 on the CPU, and stores:

* checksums of the reference's state_dict and of x (so a test can prove the
  oracle's `init_params`/`seeded_case` rebuild the same weights and input),
* the key-padding mask where the case has one,
* the full output for tiny cases and a fixed strided subset for larger ones.

The output file `golden_cases.pt` is small (<1 MB) and committed; the tests
never need the reference checkout.

`golden_half_cases.pt` holds the same records for half-precision models: the
reference's model and input converted with `.to(dtype)` (fp16 or bf16, as the
harness converts both before the accuracy check) and its eager forward run in
that type on the CPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle.reference_model import padded_mask  # noqa: E402

# name: (B, S, D, H, F, L, causal, padding_ratio, query_tile or None, seed)
CASES = {
    "tiny": (2, 32, 64, 2, 128, 2, False, 0.0, None, 0),
    "tiny_causal": (2, 32, 64, 2, 128, 2, True, 0.0, None, 0),
    "tiny_padded": (3, 40, 64, 4, 96, 2, False, 0.4, None, 7),
    "tiny_padded_causal": (3, 40, 64, 4, 96, 2, True, 0.4, None, 7),
    "ragged_hd128": (1, 100, 256, 2, 512, 1, False, 0.0, None, 3),
    "qtiled_causal": (1, 300, 128, 2, 256, 2, True, 0.0, 64, 5),
    "c1": (2, 128, 256, 4, 1024, 2, False, 0.0, None, 0),
    "c1_causal": (2, 128, 256, 4, 1024, 2, True, 0.0, None, 0),
}

# name: (B, S, D, H, F, L, causal, padding_ratio, seed, dtype)
HALF_CASES = {
    "tiny_fp16": (2, 32, 64, 2, 128, 2, False, 0.0, 0, torch.float16),
    "tiny_causal_bf16": (2, 32, 64, 2, 128, 2, True, 0.0, 0, torch.bfloat16),
    "tiny_padded_fp16": (3, 40, 64, 4, 96, 2, False, 0.4, 7, torch.float16),
    "tiny_padded_causal_bf16": (3, 40, 64, 4, 96, 2, True, 0.4, 7, torch.bfloat16),
    "c1_fp16": (2, 128, 256, 4, 1024, 2, False, 0.0, 0, torch.float16),
    "c1_bf16": (2, 128, 256, 4, 1024, 2, False, 0.0, 0, torch.bfloat16),
}

FULL_LIMIT = 20000  # store the whole output below this many elements


def sd_checksum(sd):
    tot = torch.zeros((), dtype=torch.float64)
    wsum = torch.zeros((), dtype=torch.float64)
    for i, (k, v) in enumerate(sd.items()):
        v = v.double()
        tot += v.sum()
        wsum += (v.flatten()[:: max(1, v.numel() // 97)] * (i + 1)).sum()
    return torch.stack([tot, wsum])


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import torch_transformer_benchmark as ttb  # the reference itself

    torch.set_num_threads(8)
    out = {"torch_version": torch.__version__, "cases": {}}
    for name, (b, s, d, h, f, l, causal, pad, qtile, seed) in CASES.items():
        cfg = ttb.TransformerConfig(b, s, d, h, f, l, causal)
        torch.manual_seed(seed)
        model = ttb.BaselineTransformer(cfg)
        x = torch.randn(b, s, d)
        if qtile is not None:
            # The query-tiled model draws extra weights while it is built
            # (its base class builds layers twice), so give it the plain
            # model's weights, as copy_model_weights does in the harness.
            tiled = ttb.QueryTiledBaselineTransformer(cfg, query_tile_size=qtile)
            ttb.copy_model_weights(model, tiled, strict=True)
            model = tiled
        mask = padded_mask(cfg, pad, seed + 1000) if pad > 0 else None
        if mask is not None:
            x = x.masked_fill(~mask[..., None], 0)
        model.eval()
        with torch.inference_mode():
            y = model(x, mask)
        rec = {
            "shape": (b, s, d, h, f, l, causal, pad, qtile, seed),
            "sd_checksum": sd_checksum(model.state_dict()),
            "x_checksum": torch.stack([x.double().sum(), (x.double() ** 2).sum()]),
            "mask": mask,
        }
        if y.numel() <= FULL_LIMIT:
            rec["y"] = y.clone()
            rec["y_index"] = None
        else:
            # a fixed strided subset of tokens: every 9th token of each row
            idx = torch.arange(0, s, 9)
            rec["y"] = y[:, idx, :].clone()
            rec["y_index"] = idx
        rec["y_checksum"] = torch.stack([y.double().sum(), y.double().abs().sum()])
        out["cases"][name] = rec
        print(name, tuple(y.shape), float(y.double().sum()))
    torch.save(out, HERE / "golden_cases.pt")

    half = {"torch_version": torch.__version__, "cases": {}}
    for name, (b, s, d, h, f, l, causal, pad, seed, dtype) in HALF_CASES.items():
        cfg = ttb.TransformerConfig(b, s, d, h, f, l, causal)
        torch.manual_seed(seed)
        model = ttb.BaselineTransformer(cfg)
        x = torch.randn(b, s, d)
        mask = padded_mask(cfg, pad, seed + 1000) if pad > 0 else None
        if mask is not None:
            x = x.masked_fill(~mask[..., None], 0)
        sd32 = sd_checksum(model.state_dict())
        model = model.to(dtype).eval()
        xt = x.to(dtype)
        with torch.inference_mode():
            y = model(xt, mask)
        assert y.dtype == dtype
        rec = {"shape": (b, s, d, h, f, l, causal, pad, seed), "dtype": dtype, "sd_checksum": sd32,
               "mask": mask}
        if y.numel() <= FULL_LIMIT:
            rec["y"], rec["y_index"] = y.clone(), None
        else:
            idx = torch.arange(0, s, 9)
            rec["y"], rec["y_index"] = y[:, idx, :].clone(), idx
        half["cases"][name] = rec
        print(name, tuple(y.shape), float(y.double().sum()))
    torch.save(half, HERE / "golden_half_cases.pt")

    # the harness's random inputs (generate_random_case) on the CPU
    cases = {}
    for name, (b, s, d, h, f, l, seed, pad, scale) in {
        "c1_seed1234": (2, 128, 256, 4, 1024, 2, 1234, 0.0, 1.0),
        "c1_seed1236_pad": (2, 128, 256, 4, 1024, 2, 1236, 0.4, 1.0),
        "c2_seed1235_pad_scaled": (1, 64, 512, 8, 2048, 6, 1235, 0.5, 3.0),
    }.items():
        cfg = ttb.TransformerConfig(b, s, d, h, f, l, False)
        x, mask = ttb.generate_random_case(cfg, torch.device("cpu"), torch.float32, seed, pad, scale)
        xd = x.double().flatten()
        w = torch.arange(1, xd.numel() + 1, dtype=torch.float64) % 97
        cases[name] = {"args": (b, s, d, h, f, l, seed, pad, scale), "x_head": x.flatten()[:64].clone(),
                       "x_checksum": torch.stack([xd.sum(), (xd * xd).sum(), (xd * w).sum()]),
                       "mask": mask.clone()}
    torch.save({"torch_version": torch.__version__, "cases": cases}, HERE / "golden_harness_inputs.pt")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <directory of the reference checkout>")
    main(sys.argv[1])
