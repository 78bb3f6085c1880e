"""``python -m tiny_nccl_b200``: what a run of this library depends on.

Prints the library and extension versions and paths, the CUDA devices with
their SM count and memory, the peer matrix the communicator checks at init
(P2P access and native peer atomics for every pair), multicast (NVLS)
support, and the ``TNCCL_*`` variables set in the environment, as one JSON
document (``--text`` for a table). Measured results quote these facts
beside the numbers. Works without a GPU (it then lists none).
"""
from __future__ import annotations

import argparse
import json
import os
import sys


def _peer_matrix(n: int):
    """[i][j] = {"p2p": bool, "atomics": bool | None} from the CUDA runtime;
    native atomics need cuda-python and are None without it."""
    import torch

    try:
        from cuda.bindings import runtime as rt
    except ImportError:  # pragma: no cover - cuda-python is optional
        rt = None
    out = []
    for i in range(n):
        row = []
        for j in range(n):
            if i == j:
                row.append(None)
                continue
            p2p = bool(torch.cuda.can_device_access_peer(i, j))
            atomics = None
            if rt is not None:
                err, v = rt.cudaDeviceGetP2PAttribute(
                    rt.cudaDeviceP2PAttr.cudaDevP2PAttrNativeAtomicSupported, i, j)
                if err == rt.cudaError_t.cudaSuccess:
                    atomics = bool(v)
            row.append({"p2p": p2p, "atomics": atomics})
        out.append(row)
    return out


def _multicast(i: int):
    try:
        from cuda.bindings import driver as drv
    except ImportError:  # pragma: no cover
        return None
    drv.cuInit(0)
    err, dev = drv.cuDeviceGet(i)
    if err != drv.CUresult.CUDA_SUCCESS:
        return None
    err, v = drv.cuDeviceGetAttribute(
        drv.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev)
    return bool(v) if err == drv.CUresult.CUDA_SUCCESS else None


def report() -> dict:
    import torch

    import tiny_nccl_b200 as tn

    info = {
        "tnccl_version": tn.load().version(),
        "package_version": tn.__version__,
        "library": tn.library_path(),
        "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "nccl": ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available()
        else None,
        "env": {k: v for k, v in sorted(os.environ.items()) if k.startswith("TNCCL_")},
        "devices": [],
        "peers": [],
    }
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        info["devices"].append({
            "index": i, "name": p.name, "sm": f"{p.major}.{p.minor}",
            "sms": p.multi_processor_count, "memory_gib": round(p.total_memory / 2**30, 1),
            "multicast": _multicast(i),
        })
    if n > 1:
        info["peers"] = _peer_matrix(n)
    return info


def _text(info: dict) -> str:
    lines = [f"tnccl {info['tnccl_version']} (package {info['package_version']}), "
             f"torch {info['torch']}, CUDA {info['cuda_runtime']}, NCCL {info['nccl']}",
             f"library: {info['library']}"]
    for d in info["devices"]:
        lines.append(f"GPU {d['index']}: {d['name']} sm_{d['sm'].replace('.', '')}, "
                     f"{d['sms']} SMs, {d['memory_gib']} GiB, multicast {d['multicast']}")
    if not info["devices"]:
        lines.append("no CUDA device visible")
    if info["peers"]:
        lines.append("peer access / native atomics (row -> column):")
        for i, row in enumerate(info["peers"]):
            cells = ["  - " if c is None else
                     f" {'P' if c['p2p'] else '.'}{'A' if c['atomics'] else '.'} " for c in row]
            lines.append(f"  {i}: " + "".join(cells))
    for k, v in info["env"].items():
        lines.append(f"{k}={v}")
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m tiny_nccl_b200", description=__doc__.split("\n")[0])
    ap.add_argument("--text", action="store_true", help="a table instead of JSON")
    args = ap.parse_args(argv)
    info = report()
    sys.stdout.write((_text(info) if args.text else json.dumps(info, indent=1)) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
