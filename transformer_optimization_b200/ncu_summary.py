"""Summarise Nsight Compute output into the short text kept under profiles/.

    python -m transformer_optimization_b200.ncu_summary launches LAUNCHES.csv
        per kernel: launches, total device time, share (from an
        `ncu --metrics gpu__time_duration.sum --clock-control none --csv
        --log-file` capture)
    python -m transformer_optimization_b200.ncu_summary report REPORT.ncu-rep
        the figures the roofline needs from a `--set full --clock-control
        none` capture:
        duration, DRAM bytes and throughput, tensor-pipe activity, warp
        stall reasons, registers (reads the report with `ncu -i --page raw`)

Every capture is taken with `--clock-control none`: without it ncu locks
the GPU's clocks, and a capture that is interrupted can leave them locked.
Counters only; nothing here reads instruction-level output.
"""

from __future__ import annotations

import csv
import io
import re
import subprocess
import sys
from collections import defaultdict


def _short(name: str) -> str:
    name = re.sub(r"\(.*", "", name)
    name = re.sub(r"^void\s+", "", name)
    return name.replace("tfb::", "")


def launches(path: str) -> str:
    rows = list(csv.reader(open(path, newline="")))
    # the csv log starts with ==PROF== lines; find the header
    start = next(i for i, r in enumerate(rows) if r and r[0] == "ID")
    hdr = rows[start]
    idx = {k: i for i, k in enumerate(hdr)}
    per = defaultdict(lambda: [0, 0.0])
    unit = "ns"
    for r in rows[start + 1:]:
        if len(r) != len(hdr) or r[idx["Metric Name"]] != "gpu__time_duration.sum":
            continue
        unit = r[idx["Metric Unit"]]
        v = float(r[idx["Metric Value"]].replace(",", ""))
        k = _short(r[idx["Kernel Name"]])
        per[k][0] += 1
        per[k][1] += v
    scale = {"ns": 1e-3, "usecond": 1.0, "us": 1.0, "msecond": 1e3, "ms": 1e3}.get(unit, 1e-3)
    total = sum(t for _, t in per.values())
    out = io.StringIO()
    out.write(f"{'kernel':60s} {'launches':>8s} {'total_us':>12s} {'share':>7s}\n")
    for k, (n, t) in sorted(per.items(), key=lambda kv: -kv[1][1]):
        out.write(f"{k[:60]:60s} {n:8d} {t * scale:12.1f} {t / total:7.1%}\n")
    out.write(f"{'total':60s} {sum(n for n, _ in per.values()):8d} {total * scale:12.1f}\n")
    return out.getvalue()


REPORT_METRICS = [
    "gpu__time_duration.sum",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "dram__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active",
    "smsp__issue_active.avg.pct_of_peak_sustained_active",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "lts__throughput.avg.pct_of_peak_sustained_elapsed",
    "launch__registers_per_thread",
    "launch__grid_size",
    "launch__block_size",
]


def report(path: str) -> str:
    raw = subprocess.run(["ncu", "-i", path, "--page", "raw", "--csv"], capture_output=True, text=True).stdout
    rows = list(csv.reader(io.StringIO(raw)))
    hdr, units = rows[0], rows[1]
    out = io.StringIO()
    for r in rows[2:]:
        d = dict(zip(hdr, r))
        u = dict(zip(hdr, units))
        out.write(f"kernel: {_short(d.get('Kernel Name', '?'))}\n")
        for m in REPORT_METRICS:
            if m in d:
                out.write(f"  {m:66s} {d[m]:>16s} {u.get(m, '')}\n")
        stalls = sorted(((float(d[k] or 0), k) for k in hdr
                         if k.startswith("smsp__average_warps_issue_stalled_")
                         and k.endswith("_per_issue_active.ratio")), reverse=True)[:6]
        out.write("  top warp stall reasons (warps per issue):\n")
        for v, k in stalls:
            out.write(f"    {k[len('smsp__average_warps_issue_stalled_'):-len('_per_issue_active.ratio')]:28s} {v:6.2f}\n")
    return out.getvalue()


if __name__ == "__main__":
    kind, path = sys.argv[1], sys.argv[2]
    print(launches(path) if kind == "launches" else report(path), end="")
