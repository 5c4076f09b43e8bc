"""Per-kernel summary of an ncu launch list, normalised per step.

    ncu --metrics gpu__time_duration.sum --clock-control none --csv \\
        --log-file launches.csv python bench.py --steps 2 --warmup 1 ...
    python -m kernelswift_b200.ncu_summary launches.csv --steps 17

Prints a markdown table: per kernel (templates and namespaces shortened) the
launch count, total and mean microseconds, the share of all kernel time and
the share of the step (kernels named by --setup, one-time work such as weight
initialisation, weight preparation and the L2 flush of bench.py, are left
out of the step share), and with --steps the launches and microseconds per
step. ncu serialises launches and runs them with cold caches, so the shares
are what compares with a live run, not the absolute times.
"""
from __future__ import annotations

import argparse
import collections
import csv
import sys

SCALE_US = {"ns": 1e-3, "nsecond": 1e-3, "us": 1.0, "usecond": 1.0, "ms": 1e3,
            "msecond": 1e3, "s": 1e6, "second": 1e6}
DEFAULT_SETUP = ("distribution_elementwise", "prep_cast", "prep_fp8", "prep_i8", "FillFunctor",
                 "reduce_kernel", "copy_kernel")


def short_name(name: str, width: int = 80) -> str:
    for junk in ("ksw::<unnamed>::", "(anonymous namespace)::", "ksw::"):
        name = name.replace(junk, "")
    return name.split("(")[0][:width]


def summarize(rows, setup=DEFAULT_SETUP):
    """rows: dicts with 'Kernel Name', 'Metric Name', 'Metric Value', 'Metric
    Unit'. Returns [(kernel, launches, total_us, is_setup)] by total time."""
    agg = collections.OrderedDict()
    for r in rows:
        if r.get("Metric Name") != "gpu__time_duration.sum":
            continue
        us = float(str(r["Metric Value"]).replace(",", "")) * SCALE_US[r["Metric Unit"]]
        k = short_name(r["Kernel Name"])
        a = agg.setdefault(k, [0, 0.0])
        a[0] += 1
        a[1] += us
    out = [(k, n, t, any(s in k for s in setup)) for k, (n, t) in agg.items()]
    return sorted(out, key=lambda x: -x[2])


def read_csv(path):
    with open(path, newline="") as f:
        lines = f.read().splitlines()
    start = next(i for i, line in enumerate(lines) if "Kernel Name" in line)
    return list(csv.DictReader(lines[start:]))


def markdown(summary, steps: int | None = None) -> str:
    total = sum(t for _, _, t, _ in summary)
    step_total = sum(t for _, _, t, s in summary if not s)
    head = "| kernel | launches | total us | mean us | share all | share/step |"
    sep = "|---|---:|---:|---:|---:|---:|"
    if steps:
        head += " launches/step | us/step |"
        sep += "---:|---:|"
    lines = [head, sep]
    for k, n, t, is_setup in summary:
        share = "" if is_setup else f"{100 * t / step_total:.1f}%"
        line = (f"| `{k}` | {n} | {t:.1f} | {t / n:.1f} | {100 * t / total:.1f}% | {share} |")
        if steps:
            line += "  |  |" if is_setup else f" {n / steps:.2f} | {t / steps:.1f} |"
        lines.append(line)
    return "\n".join(lines)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("csv")
    ap.add_argument("--steps", type=int, default=0, help="steps the capture covered")
    ap.add_argument("--setup", default=",".join(DEFAULT_SETUP),
                    help="comma-separated name fragments of one-time kernels")
    a = ap.parse_args()
    summary = summarize(read_csv(a.csv), tuple(s for s in a.setup.split(",") if s))
    sys.stdout.write(markdown(summary, a.steps or None) + "\n")


if __name__ == "__main__":
    main()
