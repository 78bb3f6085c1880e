"""Writes a TNCCL_TUNING_FILE from measured all-reduce sweeps.

Reads the JSON lines of benchmarks/allreduce_sweep.py (one record per
implementation and size; the records of the library's own algorithms,
`oneshot`, `twoshot`, `ring`, `nvls`, are used) and writes, per rank count,
the fastest algorithm for each measured size, merged into runs:

    <nranks> <max_bytes> <algo>

A message of b bytes uses the line with the smallest max_bytes >= b for its
rank count; the last run of a rank count extends to every larger size.

    python benchmarks/make_tuning_table.py sweep8.jsonl sweep4.jsonl -o tuning.txt
    TNCCL_TUNING_FILE=tuning.txt python ...
"""
from __future__ import annotations

import argparse
import collections
import json
import sys

ALGOS = ("oneshot", "twoshot", "ring", "nvls")
UNBOUNDED = (1 << 64) - 1


def best_runs(records):
    """{nranks: [(max_bytes, algo), ...]} from sweep records."""
    best = collections.defaultdict(dict)  # nranks -> bytes -> (busbw, algo)
    for r in records:
        impl = r.get("impl")
        if impl not in ALGOS or r.get("busbw_gbs") is None:
            continue
        key = (int(r["n_gpus"]), int(r["bytes"]))
        cur = best[key[0]].get(key[1])
        if cur is None or r["busbw_gbs"] > cur[0]:
            best[key[0]][key[1]] = (float(r["busbw_gbs"]), impl)
    out = {}
    for nranks, by_size in best.items():
        sizes = sorted(by_size)
        runs = []
        for i, s in enumerate(sizes):
            algo = by_size[s][1]
            last = i + 1 == len(sizes)
            if last or by_size[sizes[i + 1]][1] != algo:
                runs.append((UNBOUNDED if last else s, algo))
        out[nranks] = runs
    return out


def render(runs) -> str:
    lines = ["# TNCCL_TUNING_FILE: <nranks> <max_bytes> <algo>, written by "
             "benchmarks/make_tuning_table.py"]
    for nranks in sorted(runs):
        for max_bytes, algo in runs[nranks]:
            lines.append(f"{nranks} {max_bytes} {algo}")
    return "\n".join(lines) + "\n"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("sweeps", nargs="+", help="allreduce_sweep.py JSON-lines files")
    ap.add_argument("-o", "--out", default="-")
    args = ap.parse_args(argv)
    records = []
    for path in args.sweeps:
        with open(path) as f:
            records += [json.loads(line) for line in f if line.strip()]
    text = render(best_runs(records))
    if args.out == "-":
        sys.stdout.write(text)
    else:
        with open(args.out, "w") as f:
            f.write(text)


if __name__ == "__main__":
    main()
