"""Summarise an ncu launch list (CSV) into a per-kernel table.

Input: the CSV that `ncu --metrics gpu__time_duration.sum[,dram__bytes_read.sum,
dram__bytes_write.sum] --csv --log-file F <cmd>` writes (one row per launch and
metric).  Output (markdown): per kernel (template arguments kept, argument
lists dropped) its launches, summed device time, share of the summed time and,
when DRAM metrics are present, MB per launch and the achieved fraction of HBM
while it runs.  With --marker NAME the table covers only the launches from the
last --steps occurrences of kernel NAME on (one occurrence per training step),
so warm-up and set-up launches drop out.

Per-launch times under ncu are serialised and cold-cache: compare shares, not
absolute times, with a run outside the profiler.

  python -m malus_b200.profsum launches.csv [--marker k_embed2 --steps 2] [--peak-gbs G]
"""
from __future__ import annotations

import argparse
import csv
import json
import re
from collections import OrderedDict, defaultdict
from pathlib import Path

_TIME = {"nsecond": 1e-6, "ns": 1e-6, "usecond": 1e-3, "us": 1e-3, "msecond": 1.0, "ms": 1.0,
         "second": 1e3, "s": 1e3}
_BYTES = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "B": 1.0, "KB": 1e3, "MB": 1e6, "GB": 1e9}


def short_name(name: str) -> str:
    """Kernel name without its argument list, return type and namespaces."""
    # ncu writes anonymous namespaces as "(anonymous namespace)::", "<unnamed>::"
    # or, truncated, "unnamed>::"; drop them before the argument list, whose
    # "(" would otherwise match the namespace's
    n = re.sub(r"\(anonymous namespace\)::|<?unnamed>::", "", name)
    n = re.sub(r"\(.*$", "", n)
    n = re.sub(r"^void ", "", n.strip())
    n = re.sub(r"malus::", "", n)
    return n.strip()


def read_launches(path: str | Path) -> list[dict]:
    """One dict per launch: name, ms, bytes (None when no DRAM metric)."""
    with open(path) as f:
        lines = [ln for ln in f if ln.startswith('"')]
    launches: "OrderedDict[str, dict]" = OrderedDict()
    for r in csv.DictReader(lines):
        d = launches.setdefault(r["ID"], {"name": short_name(r["Kernel Name"]), "ms": 0.0, "bytes": None})
        v = float(r["Metric Value"].replace(",", ""))
        unit = r["Metric Unit"]
        if r["Metric Name"] == "gpu__time_duration.sum":
            d["ms"] = v * _TIME[unit]
        elif r["Metric Name"].startswith("dram__bytes"):
            d["bytes"] = (d["bytes"] or 0.0) + v * _BYTES[unit]
    return list(launches.values())


def window(launches: list[dict], marker: str | None, steps: int) -> list[dict]:
    if not marker:
        return launches
    starts = [i for i, d in enumerate(launches) if d["name"].startswith(marker)]
    if len(starts) < steps:
        return launches
    return launches[starts[-steps]:]


def summarise(launches: list[dict], peak_gbs: float) -> tuple[list[dict], dict]:
    agg: dict = defaultdict(lambda: {"launches": 0, "ms": 0.0, "bytes": None})
    for d in launches:
        a = agg[d["name"]]
        a["launches"] += 1
        a["ms"] += d["ms"]
        if d["bytes"] is not None:
            a["bytes"] = (a["bytes"] or 0.0) + d["bytes"]
    total_ms = sum(a["ms"] for a in agg.values())
    rows = []
    for name, a in sorted(agg.items(), key=lambda kv: -kv[1]["ms"]):
        row = {"kernel": name, "launches": a["launches"], "ms": a["ms"],
               "share": a["ms"] / total_ms if total_ms else 0.0}
        if a["bytes"] is not None:
            row["mb_per_launch"] = a["bytes"] / a["launches"] / 1e6
            gbs = a["bytes"] / (a["ms"] * 1e-3) / 1e9 if a["ms"] else 0.0
            row["gbs"] = gbs
            row["of_hbm"] = gbs / peak_gbs
        rows.append(row)
    tot = {"launches": len(launches), "ms": total_ms,
           "bytes": sum(a["bytes"] or 0.0 for a in agg.values())}
    return rows, tot


def markdown(rows: list[dict], tot: dict) -> str:
    dram = any("gbs" in r for r in rows)
    out = [f"launches {tot['launches']}, summed device time {tot['ms']:.3f} ms"
           + (f", DRAM {tot['bytes'] / 1e9:.2f} GB" if dram else "")]
    if dram:
        out.append("| kernel | launches | total ms | share | MB / launch | achieved GB/s | of HBM |")
        out.append("|---|---:|---:|---:|---:|---:|---:|")
    else:
        out.append("| kernel | launches | total ms | share |")
        out.append("|---|---:|---:|---:|")
    for r in rows:
        line = f"| {r['kernel']} | {r['launches']} | {r['ms']:.3f} | {100 * r['share']:.1f}% |"
        if dram:
            line += (f" {r.get('mb_per_launch', 0.0):.1f} | {r.get('gbs', 0.0):.0f} | "
                     f"{r.get('of_hbm', 0.0):.2f} |")
        out.append(line)
    return "\n".join(out)


def _default_peak() -> float:
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"])
    return 6650.0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("csv")
    ap.add_argument("--marker", default=None, help="kernel that starts each step")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--peak-gbs", type=float, default=None)
    a = ap.parse_args(argv)
    rows, tot = summarise(window(read_launches(a.csv), a.marker, a.steps), a.peak_gbs or _default_peak())
    print(markdown(rows, tot))


if __name__ == "__main__":
    main()
