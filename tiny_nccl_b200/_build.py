"""In-tree native build for tiny_nccl_b200.

Builds three shared objects next to this file (``lib/``), all for sm_100a:

* ``libtnccl.so``      - the collective library (C API of ``include/tnccl.h``):
                         bootstrap, communicator, transport and the all-reduce
                         kernels. Links the CUDA runtime statically and resolves
                         driver entry points at run time, so it loads on hosts
                         without a GPU driver.
* ``libtnccl_ops.so``  - the framework's model kernels (``csrc/ops``) behind a
                         plain C launcher interface.
* ``_C.*.so``          - the PyTorch binding (``csrc/torch``), compiled with g++
                         only and linked against the two libraries above.
* ``checked/libtnccl.so`` - the collective library again, with the kernels'
                         debug protocol checks compiled in (-DTNCCL_DEVICE_CHECKS=1).
                         Both collective libraries carry the SONAME
                         ``libtnccl.so``, so a process that preloads the checked
                         one (LD_PRELOAD) runs the binding on it.

A build is skipped when a stamp file records the same source/flag hash, so the
``.so`` files that travel with the repository are reused as they are.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = Path(__file__).resolve().parent
LIB = PKG / "lib"
OBJ = ROOT / "build" / "obj"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXXFLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter"]
NVCCFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                    "--expt-relaxed-constexpr", "-diag-suppress", "177"]
# TNCCL_DEVICE_CHECKS=1 at build time compiles the kernels' debug protocol
# checks in (plan capacities, exact ring sequence numbers; device.cuh).
if os.environ.get("TNCCL_DEVICE_CHECKS") == "1":
    NVCCFLAGS.append("-DTNCCL_DEVICE_CHECKS=1")

TNCCL_SRC = ROOT / "csrc" / "tnccl"
OPS_SRC = ROOT / "csrc" / "ops"
TORCH_SRC = ROOT / "csrc" / "torch"
INCLUDES = [f"-I{ROOT / 'include'}", f"-I{TNCCL_SRC}", f"-I{CUDA_HOME / 'include'}"]
TORCH_EXTRA_INC = [f"-I{TNCCL_SRC}"]


def _hash(paths, extra: str) -> str:
    h = hashlib.sha256(extra.encode())
    for p in sorted(paths):
        h.update(str(p.relative_to(ROOT)).encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def _run(cmd, cwd=ROOT):
    r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build command failed ({r.returncode}):\n{' '.join(map(str, cmd))}\n"
                           f"{r.stdout}\n{r.stderr}")
    return r


def _compile(src: Path, obj: Path, extra_inc=(), defines=()):
    obj.parent.mkdir(parents=True, exist_ok=True)
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCCFLAGS, *defines, *INCLUDES, *extra_inc, "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXXFLAGS, *defines, *INCLUDES, *extra_inc, "-c", str(src), "-o", str(obj)]
    _run(cmd)
    return obj


def _headers(d: Path):
    return [p for p in d.rglob("*") if p.suffix in (".h", ".cuh", ".hpp")]


def _build_shared(name: str, srcs, deps, link_extra=(), extra_inc=(), jobs=8,
                  subdir: str = "", defines=()) -> Path:
    outdir = LIB / subdir if subdir else LIB
    out = outdir / name
    stamp = outdir / (name + ".stamp")
    key = _hash(list(srcs) + list(deps),
                " ".join(NVCCFLAGS + list(defines) + CXXFLAGS + list(link_extra)))
    if out.exists() and stamp.exists() and stamp.read_text() == key:
        return out
    outdir.mkdir(parents=True, exist_ok=True)
    objdir = OBJ / (subdir + "_" + name if subdir else name)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, objdir / (s.stem + s.suffix.replace(".", "_") + ".o"),
                                              extra_inc, defines), srcs))
    tmp = out.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
           "-Xlinker", "-rpath,$ORIGIN", "-Xlinker", f"-soname,{name}", *link_extra,
           "-lpthread", "-ldl", "-lrt"]
    _run(cmd)
    os.replace(tmp, out)
    stamp.write_text(key)
    return out


def build_tnccl() -> Path:
    srcs = sorted(TNCCL_SRC.glob("*.cc")) + sorted(TNCCL_SRC.glob("*.cu"))
    deps = _headers(TNCCL_SRC) + [ROOT / "include" / "tnccl.h"]
    return _build_shared("libtnccl.so", srcs, deps)


def build_tnccl_checked() -> Path:
    """libtnccl.so with the device protocol checks, in lib/checked/."""
    srcs = sorted(TNCCL_SRC.glob("*.cc")) + sorted(TNCCL_SRC.glob("*.cu"))
    deps = _headers(TNCCL_SRC) + [ROOT / "include" / "tnccl.h"]
    return _build_shared("libtnccl.so", srcs, deps, subdir="checked",
                         defines=["-DTNCCL_DEVICE_CHECKS=1"])


def build_ops() -> Path | None:
    srcs = sorted(OPS_SRC.glob("*.cu"))
    if not srcs:
        return None
    deps = _headers(OPS_SRC)
    return _build_shared("libtnccl_ops.so", srcs, deps, extra_inc=[f"-I{OPS_SRC}"])


def _ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def build_torch_ext() -> Path:
    import torch.utils.cpp_extension as ce  # noqa: WPS433 (build-time only)

    srcs = sorted(TORCH_SRC.glob("*.cpp"))
    name = "_C" + _ext_suffix()
    out = PKG / name
    stamp = LIB / "_C.stamp"
    import torch
    deps = _headers(TORCH_SRC) + [ROOT / "include" / "tnccl.h"] + _headers(OPS_SRC)
    key = _hash(list(srcs) + deps, "torch-" + torch.__version__ + " ".join(CXXFLAGS))
    if out.exists() and stamp.exists() and stamp.read_text() == key:
        return out
    inc = [f"-I{p}" for p in ce.include_paths()] + [f"-I{sysconfig.get_paths()['include']}",
                                                   f"-I{OPS_SRC}"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    flags = [*CXXFLAGS, "-Wno-missing-field-initializers", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
             "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    objdir = OBJ / "_C"
    objdir.mkdir(parents=True, exist_ok=True)

    def comp(s: Path) -> Path:
        o = objdir / (s.stem + ".o")
        _run(["g++", *flags, *INCLUDES, *inc, "-c", str(s), "-o", str(o)])
        return o

    with cf.ThreadPoolExecutor(max_workers=8) as ex:
        objs = list(ex.map(comp, srcs))
    libdirs = ce.library_paths()
    tmp = out.with_suffix(".tmp")
    cmd = ["g++", "-shared", "-o", str(tmp), *map(str, objs), f"-L{LIB}", "-ltnccl",
           "-ltnccl_ops" if (LIB / "libtnccl_ops.so").exists() else "",
           *[f"-L{d}" for d in libdirs], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_cuda", "-ltorch_python",
           f"-Wl,-rpath,$ORIGIN/lib", *[f"-Wl,-rpath,{d}" for d in libdirs]]
    _run([c for c in cmd if c])
    os.replace(tmp, out)
    stamp.write_text(key)
    return out


BIN = ROOT / "build" / "bin"

# C++ programs: (source, needs CUDA headers/runtime)
PROGRAMS = {
    "tnccl_allreduce": ROOT / "examples" / "allreduce.cc",
    "allreduce_gpu_test": ROOT / "tests" / "cpp" / "allreduce_gpu_test.cc",
    "bootstrap_test": ROOT / "tests" / "cpp" / "bootstrap_test.cc",
    "rank_model_test": ROOT / "tests" / "cpp" / "rank_model_test.cc",
    # socket ring edges: connection set-up, proxy thread, ring over sockets
    "net_proxy_test": ROOT / "tests" / "cpp" / "net_proxy_test.cc",
    # mbarrier hand-offs of the tcgen05 GEMM pipelines, as threads
    "gemm_pipeline_model_test": ROOT / "tests" / "cpp" / "gemm_pipeline_model_test.cc",
    # launch geometry and schedule of the row-group LayerNorm backward
    "ln_plan_test": ROOT / "tests" / "cpp" / "ln_plan_test.cc",
    # host configuration / partition checks, built with the library's config code
    "config_test": (ROOT / "tests" / "cpp" / "config_test.cc", TNCCL_SRC / "common.cc"),
}


# C++ tests built from sources with g++ alone (no libtnccl, no CUDA runtime:
# they bring their own fakes of the CUDA calls the sources make).
STANDALONE = {
    # registered buffers: forked ranks, real bootstrap, fake driver
    "register_test": [ROOT / "tests" / "cpp" / "register_test.cc", TNCCL_SRC / "register.cc",
                      TNCCL_SRC / "enqueue.cc", TNCCL_SRC / "bootstrap.cc",
                      TNCCL_SRC / "sockio.cc", TNCCL_SRC / "common.cc"],
}


def build_standalone() -> list[Path]:
    BIN.mkdir(parents=True, exist_ok=True)
    outs = []
    for name, srcs in STANDALONE.items():
        out = BIN / name
        stamp = BIN / (name + ".stamp")
        deps = srcs + _headers(ROOT / "tests" / "cpp") + _headers(TNCCL_SRC) + \
            [ROOT / "include" / "tnccl.h"]
        key = _hash(deps, "standalone " + " ".join(CXXFLAGS))
        if not (out.exists() and stamp.exists() and stamp.read_text() == key):
            _run(["g++", *CXXFLAGS, "-O1", *INCLUDES, f"-I{ROOT / 'tests' / 'cpp'}",
                  *[str(s) for s in srcs], "-o", str(out), "-lpthread", "-ldl"])
            stamp.write_text(key)
        outs.append(out)
    return outs


def build_programs() -> list[Path]:
    """Builds the example and the C++ test programs into build/bin."""
    lib = build_tnccl()
    BIN.mkdir(parents=True, exist_ok=True)
    outs = []
    for name, entry in PROGRAMS.items():
        srcs = list(entry) if isinstance(entry, tuple) else [entry]
        if not srcs[0].exists():
            continue
        out = BIN / name
        stamp = BIN / (name + ".stamp")
        deps = srcs + _headers(ROOT / "tests" / "cpp") + _headers(TNCCL_SRC) + \
            _headers(OPS_SRC) + [ROOT / "include" / "tnccl.h"]
        key = _hash(deps, "prog " + " ".join(CXXFLAGS) + str(lib.stat().st_size))
        if not (out.exists() and stamp.exists() and stamp.read_text() == key):
            objs = []
            for k, src in enumerate(srcs):
                obj = OBJ / "bin" / f"{name}.{k}.o"
                obj.parent.mkdir(parents=True, exist_ok=True)
                _run(["g++", *CXXFLAGS, "-O2", *INCLUDES, f"-I{ROOT / 'tests' / 'cpp'}",
                      f"-I{OPS_SRC}", "-c", str(src), "-o", str(obj)])
                objs.append(str(obj))
            _run([NVCC, *ARCH, "-o", str(out), *objs, f"-L{LIB}", "-ltnccl",
                  "-Xlinker", f"-rpath,{LIB}", "-Xlinker", "-rpath,$ORIGIN/../../tiny_nccl_b200/lib",
                  "-lpthread"])
            stamp.write_text(key)
        outs.append(out)
    return outs


def build_all(verbose: bool = False) -> None:
    paths = [build_tnccl(), build_tnccl_checked(), build_ops(), build_torch_ext(),
             *build_programs(), *build_standalone()]
    if verbose:
        for p in paths:
            if p is not None:
                print(f"built {p.relative_to(ROOT)}", file=sys.stderr)


if __name__ == "__main__":
    build_all(verbose=True)
