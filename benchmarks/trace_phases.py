"""Per-phase timing of the all-reduce kernels from the device tracer.

With TNCCL_TRACE=1 every channel records {globaltimer, (family, phase, tile)}
at each phase boundary. This script runs a few all-reduces of one size and
algorithm on every rank and prints, per phase transition, the mean and the
spread of the time channel 0..C-1 spend between consecutive marks.

    TNCCL_TRACE=1 python -m torch.distributed.run --nproc-per-node 2 \
        --master-addr 127.0.0.1 benchmarks/trace_phases.py --algo twoshot --bytes 64M

`--chrome trace.json` also writes the marks of every rank as one Chrome /
Perfetto trace (process = rank, thread = channel; team busy intervals as
spans, the other marks as instants). A `--dump` file converts offline, no
GPU needed:

    python benchmarks/trace_phases.py --convert dump.rank0.json --algo twoshot \
        --chrome trace.json
"""
from __future__ import annotations

import argparse
import collections
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

NAMES = {
    2: {0: "pushed+published", 1: "RS arrived", 2: "reduced+AG published",
        4: "AG arrived", 5: "copied out"},
    1: {0: "tile start", 1: "slot free", 2: "pushed+published", 3: "peers arrived",
        4: "reduced+acked"},
    3: {1: "copied in", 2: "all copied in", 3: "switch reduce+store counted",
        4: "all stored", 5: "copied out"},
    4: {1: "all entered", 2: "reduced+stored", 3: "all stored"},
}
FAMILY = {"ring": 0, "oneshot": 1, "twoshot": 2, "nvls": 3, "nvls_zc": 4}

# Warp-specialised kernels: each team marks its own phases. (start mark,
# end mark) pairs give a team's busy time per tile; (end of tile t-1, start
# of tile t) its wait. The push / copy-in team marks once per tile (period).
TEAMS = {
    2: {"push": (None, 0), "reduce": (1, 2), "gather": (4, 5)},
    3: {"copy-in": (None, 1), "switch": (2, 3), "copy-out": (4, 5)},
}


def team_stats(raw: dict, fam: int) -> dict:
    """Mean busy / wait / period per team over every channel's last call."""
    out = {}
    acc = {}
    for ev in raw.values():
        ts = [e[0] for e in ev]
        if len(ts) < 2:
            continue
        gap, i = max((ts[k + 1] - ts[k], k) for k in range(len(ts) - 1))
        last = ev[i + 1:] if gap > 50_000 else ev  # keep the final call
        by = collections.defaultdict(dict)
        for t, p, tile in last:
            by[p][tile] = t
        for team, (s, e) in TEAMS.get(fam, {}).items():
            for tile in by[e]:
                if s is None:
                    if tile - 1 in by[e]:
                        acc.setdefault((team, "period"), []).append(by[e][tile] - by[e][tile - 1])
                    continue
                if tile in by[s]:
                    acc.setdefault((team, "busy"), []).append(by[e][tile] - by[s][tile])
                if tile in by[s] and tile - 1 in by[e]:
                    acc.setdefault((team, "wait"), []).append(by[s][tile] - by[e][tile - 1])
    for (team, kind), v in acc.items():
        out[f"{team} {kind}"] = {"mean_us": sum(v) / len(v) / 1e3, "n": len(v)}
    return out


def chrome_events(raw: dict, fam: int, rank: int) -> list:
    """Trace Event Format events of one rank's marks: raw maps a channel to
    its [(globaltimer ns, phase, tile)] list. Timestamps are microseconds
    from the rank's first mark."""
    marks = [t for ev in raw.values() for t, _, _ in ev]
    if not marks:
        return []
    t0 = min(marks)
    names = NAMES.get(fam, {})
    spans = {e: (team, s) for team, (s, e) in TEAMS.get(fam, {}).items() if s is not None}
    out = [{"ph": "M", "name": "process_name", "pid": rank, "args": {"name": f"rank {rank}"}}]
    for c, ev in sorted(raw.items(), key=lambda kv: int(kv[0])):
        c = int(c)
        out.append({"ph": "M", "name": "thread_name", "pid": rank, "tid": c,
                    "args": {"name": f"channel {c}"}})
        start = {}
        for t, p, tile in ev:
            us = (t - t0) / 1e3
            if p in spans and (spans[p][1], tile) in start:
                b = start.pop((spans[p][1], tile))
                out.append({"ph": "X", "name": spans[p][0], "pid": rank, "tid": c, "ts": b,
                            "dur": max(us - b, 0.0), "args": {"tile": tile}})
            else:
                start[(p, tile)] = us
                out.append({"ph": "i", "s": "t", "name": names.get(p, f"phase {p}"),
                            "pid": rank, "tid": c, "ts": us, "args": {"tile": tile}})
    return out


def write_chrome(path: str, events: list) -> None:
    with open(path, "w") as f:
        json.dump({"traceEvents": events, "displayTimeUnit": "ns"}, f)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--algo", default="twoshot")
    ap.add_argument("--bytes", default="64M")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--out", default="")
    ap.add_argument("--dump", default="", help="write every channel's raw events (JSON) here")
    ap.add_argument("--chrome", default="", help="write a Chrome / Perfetto trace here")
    ap.add_argument("--convert", default="", help="a --dump file to convert (no run)")
    args = ap.parse_args()
    if args.convert:
        with open(args.convert) as f:
            raw = {int(c): [tuple(e) for e in ev] for c, ev in json.load(f).items()}
        write_chrome(args.chrome or args.convert + ".trace.json",
                     chrome_events(raw, FAMILY[args.algo], 0))
        return
    assert os.environ.get("TNCCL_TRACE") == "1", "run with TNCCL_TRACE=1"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    import tiny_nccl_b200 as tn

    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    size = int(args.bytes[:-1]) * mult[args.bytes[-1]]
    comm = tn.init_from_torch_distributed(device=rank)
    x = torch.randn(size // 4, device=dev)
    y = torch.empty_like(x)
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for _ in range(args.iters):
            comm.all_reduce(x, y, algo=args.algo)
    torch.cuda.synchronize()
    fam = FAMILY[args.algo]
    deltas = collections.defaultdict(list)
    spans = []
    raw = {}
    for c in range(128):
        rec = comm._c.trace_read(c, 1 << 16)
        if not rec:
            continue
        ev = [(rec[2 * i], rec[2 * i + 1]) for i in range(len(rec) // 2)]
        ev = [(t, (tag >> 16) & 0xFF, tag & 0xFFFF) for t, tag in ev if (tag >> 24) == fam]
        if not ev:
            continue
        raw[c] = ev
        spans.append(ev[-1][0] - ev[0][0])
        for (t0, p0, _), (t1, p1, _) in zip(ev, ev[1:]):
            deltas[(p0, p1)].append(t1 - t0)
    summary = {f"{NAMES.get(fam, {}).get(a, a)} -> {NAMES.get(fam, {}).get(b, b)}":
               {"mean_us": sum(v) / len(v) / 1e3, "n": len(v)} for (a, b), v in sorted(deltas.items())}
    rec = {"rank": rank, "algo": args.algo, "bytes": size, "phases": summary,
           "teams": team_stats(raw, fam),
           "channel_span_us_mean": sum(spans) / max(1, len(spans)) / 1e3}
    if args.dump:
        with open(f"{args.dump}.rank{rank}.json", "w") as f:
            json.dump(raw, f)
    allrec = [None] * world
    dist.all_gather_object(allrec, rec)
    if args.chrome:
        events = [None] * world
        dist.all_gather_object(events, chrome_events(raw, fam, rank))
        if rank == 0:
            write_chrome(args.chrome, [e for ev in events for e in ev])
    if rank == 0:
        for r in allrec:
            print(json.dumps(r))
        if args.out:
            with open(args.out, "a") as f:
                for r in allrec:
                    f.write(json.dumps(r) + "\n")
    torch.cuda.synchronize()
    comm.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
