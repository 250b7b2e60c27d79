"""Build the reference's own GPU runtime for B200 (sm_100), unmodified, for ``bench.py --impl reference``.

1. Install the reference package into ``baseline/_ref`` (offline wheelhouse; the
   ``--no-deps`` form, because ``argcomplete`` is not in the wheelhouse).
2. Run the reference's runtime builder, runtime/build_runtime.py:24-69, with
   ``--arch 100``: it copies third_party/msccl (MSCCL 0.1 on NCCL 2.12.12),
   applies its ten trace patches, verifies their hashes and runs
   ``make src.build NVCC_GENCODE=-gencode=arch=compute_100,code=sm_100``.
3. Copy ``libnccl.so*`` and ``nccl.h`` into ``baseline/_ref/lib`` / ``include``.
4. Compile the reference's helper kernels (runtime/execution/gpu_operations.cu:
   fill_input, scale_output, check_output, sample_timer) into
   ``baseline/_ref/lib/libvericcl_gpuops.so`` with the same ``-gencode`` the
   reference's native build uses (runtime/build_native.py:78-95).

The outcome (commands, return codes, first compiler error) goes to
``baseline/_ref/lib/build.json``; ``bench.py --impl reference`` reads it when
the library is missing.  Usage: ``python baseline/build_reference.py [--jobs 8]``.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")
SHARE = os.path.join(REF, "share", "vericcl")
LIB = os.path.join(REF, "lib")
INC = os.path.join(REF, "include")
SOURCE = "/root/reference"


def run(cmd, log, **kw):
    t = time.monotonic()
    p = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, **kw)
    log.append({"argv": cmd, "rc": p.returncode, "seconds": round(time.monotonic() - t, 1),
                "tail": p.stdout[-3000:]})
    return p


def first_error(text: str) -> str:
    for line in text.splitlines():
        if " error" in line or "error:" in line:
            return line.strip()[:300]
    return text.strip().splitlines()[-1][:300] if text.strip() else "unknown"


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--arch", type=int, default=100)
    ap.add_argument("--cuda-home", default=os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    ap.add_argument("--timeout-s", type=float, default=7200)
    ap.add_argument("--from-build", default=None,
                    help="output directory of an earlier run of the reference's build_runtime.py to reuse")
    args = ap.parse_args()
    log: list = []
    record = {"arch": args.arch, "steps": log}
    os.makedirs(LIB, exist_ok=True)
    os.makedirs(INC, exist_ok=True)
    try:
        if not os.path.isdir(os.path.join(REF, "vericcl")):
            with tempfile.TemporaryDirectory() as tmp:
                copy = os.path.join(tmp, "reference")
                shutil.copytree(SOURCE, copy)
                p = run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                         "--find-links", "/opt/wheelhouse", "--target", REF, copy], log)
                if p.returncode:
                    raise RuntimeError("pip install of the reference failed: " + first_error(p.stdout))
        if args.from_build:
            out = os.path.abspath(args.from_build)
            rc = 0
        else:
            out = tempfile.mkdtemp(prefix="vb_refbuild_")
            os.rmdir(out)   # the reference's builder wants a directory that does not exist yet
            env = dict(os.environ, PYTHONPATH=REF)
            p = run([sys.executable, os.path.join(SHARE, "runtime", "build_runtime.py"), "--output-dir", out,
                     "--cuda-home", args.cuda_home, "--arch", str(args.arch), "--jobs", str(args.jobs),
                     "--timeout-s", str(args.timeout_s)], log, env=env)
            rc = p.returncode
        built = os.path.join(out, "build")
        record["output_dir"] = out
        if rc or not os.path.isfile(os.path.join(built, "lib", "libnccl.so")):
            err = ""
            for name in ("stderr.log", "stdout.log"):
                f = os.path.join(out, "process", "jobs", "compile", name)
                if os.path.isfile(f):
                    with open(f, errors="replace") as fh:
                        text = fh.read()
                    if "error" in text:
                        err = first_error(text)
                        break
            raise RuntimeError("reference runtime build failed: " + (err or "no libnccl.so in " + built))
        for name in os.listdir(os.path.join(built, "lib")):
            if name.startswith("libnccl.so"):
                src = os.path.join(built, "lib", name)
                dst = os.path.join(LIB, name)
                if os.path.lexists(dst):
                    os.remove(dst)
                if os.path.islink(src):
                    os.symlink(os.readlink(src), dst)
                else:
                    shutil.copy2(src, dst)
        shutil.copy2(os.path.join(built, "include", "nccl.h"), os.path.join(INC, "nccl.h"))
        nvcc = os.path.join(args.cuda_home, "bin", "nvcc")
        p = run([nvcc, "-std=c++17", "-O2", "-shared", "-Xcompiler=-fPIC",
                 "-gencode=arch=compute_{0},code=sm_{0}".format(args.arch),
                 "-I" + INC, "-I" + os.path.join(SHARE, "runtime", "include"),
                 "-I" + os.path.join(SHARE, "runtime", "execution"),
                 os.path.join(SHARE, "runtime", "execution", "gpu_operations.cu"),
                 "-o", os.path.join(LIB, "libvericcl_gpuops.so")], log)
        if p.returncode:
            raise RuntimeError("gpu_operations.cu build failed: " + first_error(p.stdout))
        record["ok"] = True
    except Exception as e:   # recorded for the bench's unavailable line
        record["ok"] = False
        record["error"] = str(e)
    with open(os.path.join(LIB, "build.json"), "w") as f:
        json.dump(record, f, indent=1)
    print(json.dumps({k: v for k, v in record.items() if k != "steps"}))
    return 0 if record["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
