"""In-tree builds of the native modules.

* ``_vbplan`` — the schedule compiler and CPU interpreter (C++17, pybind11,
  built with g++; no CUDA needed).
* ``_vbcuda`` — the sm_100a kernels, the symmetric heap and the launch path
  (a PyTorch CUDA extension built with nvcc for ``compute_100a/sm_100a``).
* ``libvericcl_b200.so`` and ``vericcl-native`` — the C API and its driver.

Outputs live next to the package (``vericcl_b200/_native/``) so they travel
with a source snapshot; a stamp file holding the hash of sources and flags
decides whether a rebuild is needed.
(reference counterparts: runtime/build_runtime.py:72, runtime/build_probes.py:45 and
runtime/build_native.py:46, which build the patched MSCCL, the probe binary and the native driver).
"""
from __future__ import annotations

import fcntl
import functools
import hashlib
import os
import threading
import subprocess
import sys
import sysconfig
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
CSRC = ROOT / "csrc"
OUT = ROOT / "vericcl_b200" / "_native"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
EXT = sysconfig.get_config_var("EXT_SUFFIX") or ".so"

PLAN_SOURCES = ["plan/xml_parse.cc", "plan/compile.cc", "plan/cpu_interp.cc"]
RUNTIME_SOURCES = ["runtime/contract.cc", "runtime/control_transport.cc", "runtime/trace_io.cc"]


_build_guard = threading.RLock()
_build_depth = 0


def _serialized(fn):
    """Run a build function under an exclusive lock on a file in the output folder.

    Every rank of a multi-GPU job imports the extension at the same moment; when
    the in-tree module is stale, the first process to take the lock rebuilds it
    and the others, once they get the lock, find it fresh instead of compiling
    and renaming over the same files at once.  Nested builds (``build_all``)
    take the lock once.
    """
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        global _build_depth
        with _build_guard:
            if _build_depth:
                _build_depth += 1
                try:
                    return fn(*args, **kwargs)
                finally:
                    _build_depth -= 1
            OUT.mkdir(parents=True, exist_ok=True)
            with open(OUT / ".build.lock", "a") as lock:
                fcntl.flock(lock, fcntl.LOCK_EX)
                _build_depth = 1
                try:
                    return fn(*args, **kwargs)
                finally:
                    _build_depth = 0
                    fcntl.flock(lock, fcntl.LOCK_UN)
    return wrapper


def _digest(paths, flags) -> str:
    h = hashlib.sha256()
    for p in sorted(paths):
        h.update(str(Path(p).relative_to(ROOT)).encode())
        h.update(Path(p).read_bytes())
    for f in flags:
        h.update(f.replace(str(ROOT), "<root>").encode())
    for header in sorted((CSRC / "include").rglob("*.h")):
        h.update(header.read_bytes())
    return h.hexdigest()


def _fresh(target: Path, stamp: str) -> bool:
    s = target.with_suffix(target.suffix + ".stamp")
    return target.exists() and s.exists() and s.read_text() == stamp


def _mark(target: Path, stamp: str) -> None:
    target.with_suffix(target.suffix + ".stamp").write_text(stamp)


def _run(cmd, what):
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError("%s failed (%d):\n%s\n%s" % (what, proc.returncode, " ".join(map(str, cmd)),
                                                        proc.stdout[-8000:]))
    return proc.stdout


def pybind_includes():
    import pybind11
    return [pybind11.get_include(), sysconfig.get_paths()["include"]]


@_serialized
def build_plan_module(force: bool = False) -> Path:
    OUT.mkdir(parents=True, exist_ok=True)
    target = OUT / ("_vbplan" + EXT)
    sources = [CSRC / s for s in PLAN_SOURCES] + [CSRC / "plan" / "bindings.cc"]
    flags = ["-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wno-unused-function"]
    stamp = _digest(sources, flags)
    if not force and _fresh(target, stamp):
        return target
    cmd = ["g++", *flags, "-I", str(CSRC / "include")]
    for inc in pybind_includes():
        cmd += ["-I", inc]
    cmd += [str(s) for s in sources] + ["-o", str(target) + ".tmp"]
    _run(cmd, "g++ build of _vbplan")
    os.replace(str(target) + ".tmp", target)
    _mark(target, stamp)
    return target


def torch_flags():
    import torch.utils.cpp_extension as ext
    inc = ext.include_paths(device_type="cuda") if "device_type" in ext.include_paths.__code__.co_varnames \
        else ext.include_paths(cuda=True)
    libs = ext.library_paths(device_type="cuda") if "device_type" in ext.library_paths.__code__.co_varnames \
        else ext.library_paths(cuda=True)
    return inc, libs


CUDA_SOURCES = ["cuda/interp.cu", "cuda/oneshot.cu", "cuda/helpers.cu", "cuda/probes.cu", "cuda/push.cu",
                "cuda/fp8.cu", "runtime/symheap.cc", "runtime/cuda_ext.cc"]


@_serialized
def build_cuda_module(force: bool = False, jobs: int | None = None) -> Path:
    """nvcc/g++ build of the PyTorch CUDA extension ``_vbcuda`` for sm_100a."""
    OUT.mkdir(parents=True, exist_ok=True)
    target = OUT / ("_vbcuda" + EXT)
    sources = [CSRC / s for s in CUDA_SOURCES + PLAN_SOURCES]
    inc, libs = torch_flags()
    import torch
    abi = "-D_GLIBCXX_USE_CXX11_ABI=%d" % int(torch._C._GLIBCXX_USE_CXX11_ABI)
    common = ["-O3", "-std=c++17", abi, "-DTORCH_EXTENSION_NAME=_vbcuda", "-DTORCH_API_INCLUDE_EXTENSION_H",
              "-I", str(CSRC / "include")] + sum((["-I", i] for i in inc + pybind_includes()), [])
    nvflags = ARCH_FLAGS + ["-lineinfo", "--use_fast_math", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                            "-Xptxas", "-v", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__"]
    ccflags = ["-fPIC", "-Wall", "-Wno-unused-function", "-I", str(CUDA_HOME / "include")]
    stamp = _digest(sources, common + nvflags + ccflags)
    if not force and _fresh(target, stamp):
        return target
    objdir = ROOT / "build" / "vbcuda"
    objdir.mkdir(parents=True, exist_ok=True)
    objects, logs = [], []
    from concurrent.futures import ThreadPoolExecutor

    def compile_one(src: Path):
        obj = objdir / (src.name + ".o")
        if src.suffix == ".cu":
            cmd = [str(CUDA_HOME / "bin" / "nvcc"), "-c", str(src), "-o", str(obj), *common, *nvflags]
        else:
            cmd = ["g++", "-c", str(src), "-o", str(obj), *common, *ccflags]
        out = _run(cmd, "compile " + src.name)
        return obj, out

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 2)) as pool:
        for obj, out in pool.map(compile_one, sources):
            objects.append(obj)
            logs.append(out)
    (objdir / "ptxas.log").write_text("\n".join(logs))
    link = ["g++", "-shared", "-o", str(target) + ".tmp", *map(str, objects)]
    for lib in libs:
        link += ["-L", lib, "-Wl,-rpath," + lib]
    link += ["-L", str(CUDA_HOME / "lib64"), "-Wl,-rpath," + str(CUDA_HOME / "lib64"),
             "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart", "-lcuda"]
    stubs = CUDA_HOME / "lib64" / "stubs"
    if stubs.exists():
        link += ["-L", str(stubs)]
    _run(link, "link _vbcuda")
    os.replace(str(target) + ".tmp", target)
    _mark(target, stamp)
    return target


CAPI_SOURCES = ["runtime/capi.cc"]


@_serialized
def build_capi(force: bool = False) -> Path:
    """Standalone C API library ``libvericcl_b200.so`` (C ABI, no Python)."""
    OUT.mkdir(parents=True, exist_ok=True)
    target = OUT / "libvericcl_b200.so"
    sources = [CSRC / s for s in CAPI_SOURCES + RUNTIME_SOURCES + PLAN_SOURCES] + \
        [CSRC / "cuda" / "interp.cu", CSRC / "cuda" / "helpers.cu", CSRC / "cuda" / "noalloc.cu",
         CSRC / "runtime" / "symheap.cc"]
    existing = [s for s in sources if s.exists()]
    if len(existing) != len(sources):
        raise FileNotFoundError("C API sources missing: %s" % [str(s) for s in sources if not s.exists()])
    flags = ARCH_FLAGS + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared", "-DVB_NO_TORCH",
                          "-I", str(CSRC / "include")]
    stamp = _digest(sources, flags)
    if not force and _fresh(target, stamp):
        return target
    stubs = CUDA_HOME / "lib64" / "stubs"
    cmd = [str(CUDA_HOME / "bin" / "nvcc"), *flags, *map(str, sources), "-o", str(target) + ".tmp"]
    if stubs.exists():
        cmd += ["-L", str(stubs)]
    cmd += ["-lcuda", "-lpthread"]
    _run(cmd, "nvcc build of libvericcl_b200")
    os.replace(str(target) + ".tmp", target)
    _mark(target, stamp)
    return target


@_serialized
def build_driver(force: bool = False) -> Path:
    """``vericcl-native``: one rank of a schedule through the C API, with a JSON receipt."""
    lib = build_capi(force)
    target = OUT / "vericcl-native"
    sources = [CSRC / "runtime" / "driver.cc"]
    flags = ["-O2", "-std=c++17", "-I", str(CSRC / "include"), "-I", str(CUDA_HOME / "include")]
    stamp = _digest(sources + [lib], flags)
    if not force and _fresh(target, stamp):
        return target
    cmd = ["g++", *flags, str(sources[0]), "-o", str(target) + ".tmp", "-L", str(OUT), "-lvericcl_b200",
           "-Wl,-rpath,$ORIGIN", "-L", str(CUDA_HOME / "lib64"), "-Wl,-rpath," + str(CUDA_HOME / "lib64"), "-lcudart",
           "-L", str(CUDA_HOME / "lib64" / "stubs"), "-lcuda"]
    _run(cmd, "driver build")
    os.replace(str(target) + ".tmp", target)
    _mark(target, stamp)
    return target


@_serialized
def build_native_tests(force: bool = False) -> Path:
    """CPU-only tests of the contract utilities and the control plane (g++, no CUDA)."""
    OUT.mkdir(parents=True, exist_ok=True)
    target = OUT / "native_cpu_tests"
    sources = [CSRC / s for s in RUNTIME_SOURCES] + [ROOT / "tests" / "native" / "test_control_and_contract.cc"]
    flags = ["-O1", "-std=c++17", "-pthread", "-I", str(CSRC / "include")]
    stamp = _digest(sources, flags)
    if not force and _fresh(target, stamp):
        return target
    _run(["g++", *flags, *map(str, sources), "-o", str(target) + ".tmp"], "native test build")
    os.replace(str(target) + ".tmp", target)
    _mark(target, stamp)
    return target


@_serialized
def build_capi_cpu_tests(force: bool = False) -> Path:
    """The C API's execute path built with g++ against host stand-ins of the CUDA runtime and the heap."""
    OUT.mkdir(parents=True, exist_ok=True)
    target = OUT / "capi_cpu_tests"
    stubs = ROOT / "tests" / "native" / "cpu_stubs"
    sources = [CSRC / s for s in CAPI_SOURCES + RUNTIME_SOURCES] + [CSRC / "plan" / "xml_parse.cc",
                                                                     CSRC / "plan" / "compile.cc"] + \
        [stubs / "stubs.cc", ROOT / "tests" / "native" / "test_capi_cpu.cc"]
    headers = [stubs / "cuda_runtime.h", stubs / "cuda.h"]
    flags = ["-O1", "-std=c++17", "-pthread", "-I", str(stubs), "-I", str(CSRC / "include")]
    stamp = _digest(sources + headers, flags)
    if not force and _fresh(target, stamp):
        return target
    _run(["g++", *flags, *map(str, sources), "-o", str(target) + ".tmp"], "C API CPU test build")
    os.replace(str(target) + ".tmp", target)
    _mark(target, stamp)
    return target


@_serialized
def build_all(force: bool = False) -> dict:
    out = {"plan": str(build_plan_module(force))}
    out["cuda"] = str(build_cuda_module(force))
    out["capi"] = str(build_capi(force))
    out["driver"] = str(build_driver(force))
    out["native_tests"] = str(build_native_tests(force))
    out["capi_cpu_tests"] = str(build_capi_cpu_tests(force))
    return out


if __name__ == "__main__":
    if "-h" in sys.argv or "--help" in sys.argv:
        print("usage: python -m vericcl_b200.ops.build [--force]\n"
              "builds the in-tree native modules (sm_100a CUDA extension, schedule compiler, C API, driver, "
              "CPU test binaries) that are out of date, or all of them with --force")
        sys.exit(0)
    print(build_all(force="--force" in sys.argv))
