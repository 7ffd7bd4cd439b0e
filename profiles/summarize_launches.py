"""Summarise an ncu `--metrics gpu__time_duration.sum --csv` launch list by kernel.

Usage: python profiles/summarize_launches.py <launches.csv>
Prints launches, total device time and share per kernel (cold-cache, serialised timings).
"""
import collections
import csv
import sys

SCALE = {"ns": 1e-6, "nsecond": 1e-6, "us": 1e-3, "usecond": 1e-3, "ms": 1.0,
         "msecond": 1.0, "s": 1e3, "second": 1e3}


def main(path):
    rows = list(csv.reader(open(path)))
    hi = next(i for i, r in enumerate(rows) if "Kernel Name" in r)
    hdr, data = rows[hi], rows[hi + 1:]
    ki, mi = hdr.index("Kernel Name"), hdr.index("Metric Name")
    vi, ui = hdr.index("Metric Value"), hdr.index("Metric Unit")
    agg = collections.defaultdict(lambda: [0, 0.0])
    for r in data:
        if len(r) <= vi or r[mi] != "gpu__time_duration.sum":
            continue
        name = r[ki].split("(")[0].strip()
        agg[name][0] += 1
        agg[name][1] += float(r[vi].replace(",", "")) * SCALE[r[ui]]
    tot = sum(v[1] for v in agg.values())
    print(f"{'kernel':62s} {'launches':>8s} {'total ms':>10s} {'share':>7s}")
    for k, (n, t) in sorted(agg.items(), key=lambda x: -x[1][1]):
        print(f"{k[:62]:62s} {n:8d} {t:10.2f} {100 * t / tot:6.2f}%")
    print(f"{'all':62s} {sum(v[0] for v in agg.values()):8d} {tot:10.2f}")


if __name__ == "__main__":
    main(sys.argv[1])
