"""Summaries of ncu output for profiles/.

    python profiling.py launches launches.csv [N]
        per-kernel launches, total device time and share of a
        `ncu --metrics gpu__time_duration.sum --csv` launch list (N: only
        the N launches after the bench's pre-timing spin kernel)
    python profiling.py report prof.ncu-rep
        the headline metrics of an `ncu --set full` capture
    python profiling.py traffic sweep_ncu.csv
        per-launch duration and DRAM bytes of a `--metrics` capture
"""
from __future__ import annotations

import collections
import csv
import io
import subprocess
import sys

UNIT_NS = {"ns": 1.0, "nsecond": 1.0, "us": 1e3, "usecond": 1e3, "ms": 1e6, "msecond": 1e6}


def launches(path: str, foreign: str = "at::", window: int = 0) -> str:
    """Per-kernel launches, device time and share; kernels whose name
    contains `foreign` (PyTorch's own helper kernels, e.g. the spin kernel
    the bench runs before its timed region) are listed apart and left out of
    the shares.  window > 0: only the first `window` launches of this
    library after the first foreign launch (the bench's timed steps)."""
    text = open(path).read().splitlines()
    start = next(i for i, line in enumerate(text) if line.startswith('"ID"'))
    rows = list(csv.reader(text[start:]))
    hdr = rows[0]
    ki, mi, ui, vi = (hdr.index(k) for k in ("Kernel Name", "Metric Name", "Metric Unit", "Metric Value"))
    agg = collections.defaultdict(lambda: [0, 0.0])
    seen_foreign, taken = window == 0, 0
    for r in rows[1:]:
        if len(r) <= vi or r[mi] != "gpu__time_duration.sum":
            continue
        name = r[ki].split("(")[0].replace("(anonymous namespace)::", "")
        if window:
            if foreign in name:
                if seen_foreign:
                    continue
                seen_foreign = True
            elif not seen_foreign or taken >= window:
                continue
            else:
                taken += 1
        agg[name][0] += 1
        agg[name][1] += float(r[vi].replace(",", "")) * UNIT_NS.get(r[ui], 1.0)
    ours = {k: v for k, v in agg.items() if foreign not in k}
    other = {k: v for k, v in agg.items() if foreign in k}
    total = sum(v[1] for v in ours.values())
    out = [f"{sum(v[0] for v in ours.values())} launches of this library, {total / 1e6:.2f} ms total "
           "(cold-cache, serialised)", "", "| kernel | launches | total ms | share |", "|---|---:|---:|---:|"]
    for name, (n, t) in sorted(ours.items(), key=lambda kv: -kv[1][1]):
        short = name.replace("tysor::", "").replace("<unnamed>::", "").replace("unnamed>::", "")
        out.append(f"| `{short}` | {n} | {t / 1e6:.3f} | "
                   f"{100 * t / total:.1f}% |")
    for name, (n, t) in other.items():
        out.append(f"\nNot counted (not this library's): `{name}` x{n}, {t / 1e6:.3f} ms.")
    return "\n".join(out)


REPORT_KEYS = [
    "gpu__time_duration.sum", "sm__cycles_elapsed.avg.per_second",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "dram__bytes_read.sum", "dram__bytes_write.sum",
    "dram__throughput.avg.pct_of_peak_sustained_elapsed",
    "lts__t_sector_hit_rate.pct", "l1tex__throughput.avg.pct_of_peak_sustained_active",
    "launch__registers_per_thread", "launch__occupancy_limit_shared_mem",
    "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
]


def report(path: str) -> str:
    raw = subprocess.run(["ncu", "-i", path, "--page", "raw", "--csv"], capture_output=True, text=True,
                         check=True).stdout
    rows = list(csv.reader(io.StringIO(raw)))
    hdr, units = rows[0], rows[1]
    out = []
    for vals in rows[2:]:
        name = vals[hdr.index("Kernel Name")] if "Kernel Name" in hdr else "kernel"
        out.append(f"kernel: `{name.split('(')[0]}`")
        for k in REPORT_KEYS:
            if k in hdr:
                i = hdr.index(k)
                out.append(f"- {k}: {vals[i]} {units[i]}")
    return "\n".join(out)


def traffic(path: str) -> str:
    """Per launch of a `ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,
    dram__bytes_write.sum --csv` log: duration, DRAM bytes read and written,
    and the DRAM bandwidth they imply."""
    text = open(path).read().splitlines()
    start = next(i for i, line in enumerate(text) if line.startswith('"ID"'))
    rows = list(csv.reader(text[start:]))
    hdr = rows[0]
    ii, ki, mi, ui, vi = (hdr.index(k) for k in ("ID", "Kernel Name", "Metric Name", "Metric Unit", "Metric Value"))
    per = collections.OrderedDict()
    for r in rows[1:]:
        if len(r) <= vi:
            continue
        name = r[ki].split("(")[0].replace("(anonymous namespace)::", "")
        scale = UNIT_NS.get(r[ui], 1.0) if r[mi] == "gpu__time_duration.sum" else \
            {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}.get(r[ui], 1.0)
        per.setdefault((r[ii], name), {})[r[mi]] = float(r[vi].replace(",", "")) * scale
    out = ["| launch | kernel | time us | DRAM read MB | DRAM write MB | DRAM GB/s |", "|---:|---|---:|---:|---:|---:|"]
    for (lid, name), m in per.items():
        t = m.get("gpu__time_duration.sum", 0.0)
        rd = m.get("dram__bytes_read.sum", 0.0)
        wr = m.get("dram__bytes_write.sum", 0.0)
        bw = (rd + wr) / t if t else 0.0
        out.append(f"| {lid} | `{name}` | {t / 1e3:.1f} | {rd / 1e6:.1f} | {wr / 1e6:.1f} | {bw:.0f} |")
    return "\n".join(out)


if __name__ == "__main__":
    kind, path = sys.argv[1], sys.argv[2]
    if kind == "launches" and len(sys.argv) > 3:
        print(launches(path, window=int(sys.argv[3])))
    else:
        print({"launches": launches, "report": report, "traffic": traffic}[kind](path))
