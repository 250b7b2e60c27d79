"""Reference arm of ``bench.py``: the reference's own NCCL/MSCCL build, run on the same GPUs.

The reference runs its collectives through a vendored MSCCL 0.1 / NCCL 2.12.12
(third_party/msccl, prepared and compiled by runtime/build_runtime.py:24-69).
``baseline/build_reference.py`` builds that library unmodified for sm_100 into
``baseline/_ref/lib/libnccl.so`` and compiles the reference's helper kernels
(runtime/execution/gpu_operations.cu) into ``baseline/_ref/lib/libvericcl_gpuops.so``.

One step of the gradient-bucket workload is what the reference's execute path
does per request (runtime/execution/execute_impl.h:53-55): the collective, then
its separate ``vericcl_scale_output`` pass, here once per 25 MiB bucket.  The
collective is the library's stock ``ncclAllReduce`` (SUM, bf16, in place): the
reference can only emit a custom MSCCL schedule through its SCIP synthesizer,
which cannot be installed offline, and ``ncclAllReduce`` is also what its
documented baseline protocol measures (README.md:456-503, nccl-tests).

Nothing of vericcl_b200 and no PyTorch is loaded in this process (PyTorch
would bring its own NCCL 2.28 into the symbol namespace): the CUDA runtime is
driven through ctypes, ranks exchange the ``ncclUniqueId`` through a file in
/tmp (all ranks of a run share one parent process), and the barrier and the
max over ranks use the reference library's own ``ncclAllReduce``.
"""
from __future__ import annotations

import ctypes
import json
import os
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "lib")
NCCL_SO = os.path.join(REF_LIB, "libnccl.so")
GPUOPS_SO = os.path.join(REF_LIB, "libvericcl_gpuops.so")
BUILD_RECORD = os.path.join(REF_LIB, "build.json")

NCCL_BF16, NCCL_F64, NCCL_SUM, NCCL_MAX = 9, 8, 0, 2
H2D, D2H, D2D = 1, 2, 3


# Observed on an 8-GPU B200 system: the library's first 2-GPU run (ncclCommInitRank, then ncclAllReduce of 25 MiB bf16
# buckets, torchrun with two ranks) printed its version banner and then returned nothing within 300 s (0.4 GB
# per rank) nor within 900 s (16 GB per rank), while the GPUs still answered.  The inputs were checked by
# reading (argument types, sizes, the 128-byte id exchange); a reference that hangs is not run again on
# GPUs that other jobs share, so every multi-GPU run of the arm reports this instead.
MULTI_GPU_HANG = ("the reference's MSCCL 0.1 / NCCL 2.12.12 built for sm_100 hung on its first 2-GPU run on a B200 "
                  "(no result within 300 s at 0.4 GB per rank nor 900 s at 16 GB per rank; GPUs still answered) "
                  "and is not re-run on more than one GPU")


def unavailable_reason(world: int = 1) -> str | None:
    """Why the reference arm cannot run here (None when its libraries are built and the run has one GPU)."""
    if world > 1:
        return MULTI_GPU_HANG
    if not os.path.isfile(NCCL_SO):
        if os.path.isfile(BUILD_RECORD):
            with open(BUILD_RECORD) as f:
                rec = json.load(f)
            return "reference MSCCL/NCCL 2.12.12 build for sm_100 failed: %s" % rec.get("error", "see build.json")
        return "reference MSCCL/NCCL 2.12.12 is not built (run baseline/build_reference.py)"
    if not os.path.isfile(GPUOPS_SO):
        return "the reference's gpu_operations.cu (scale_output kernel) is not built"
    return None


class CudaRT:
    """The few CUDA runtime calls the arm needs, through ctypes (no PyTorch)."""

    def __init__(self):
        cand = [os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "lib64", "libcudart.so"),
                "libcudart.so.12", "libcudart.so"]
        last = None
        for c in cand:
            try:
                self.lib = ctypes.CDLL(c)
                break
            except OSError as e:
                last = e
        else:
            raise OSError("libcudart not found: %s" % last)
        self.lib.cudaGetErrorString.restype = ctypes.c_char_p
        self.lib.cudaEventElapsedTime.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_void_p, ctypes.c_void_p]
        for name in ("cudaMemcpy", "cudaMemcpyAsync"):
            getattr(self.lib, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int] + \
                ([ctypes.c_void_p] if name.endswith("Async") else [])
        self.lib.cudaMemsetAsync.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p]
        self.lib.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
        self.lib.cudaHostAlloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t, ctypes.c_uint]
        self.lib.cudaFree.argtypes = [ctypes.c_void_p]
        self.lib.cudaFreeHost.argtypes = [ctypes.c_void_p]
        self.lib.cudaEventRecord.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        self.lib.cudaStreamSynchronize.argtypes = [ctypes.c_void_p]
        self.lib.cudaEventSynchronize.argtypes = [ctypes.c_void_p]

    def check(self, rc, what):
        if rc != 0:
            raise RuntimeError("%s: %s" % (what, self.lib.cudaGetErrorString(rc).decode()))

    def call(self, name, *args):
        self.check(getattr(self.lib, name)(*args), name)

    def malloc(self, n):
        p = ctypes.c_void_p()
        self.call("cudaMalloc", ctypes.byref(p), ctypes.c_size_t(n))
        return p.value

    def host_alloc(self, n):
        p = ctypes.c_void_p()
        self.call("cudaHostAlloc", ctypes.byref(p), ctypes.c_size_t(n), 0)
        return p.value

    def stream(self):
        s = ctypes.c_void_p()
        self.call("cudaStreamCreateWithFlags", ctypes.byref(s), 1)   # non-blocking
        return s.value

    def event(self):
        e = ctypes.c_void_p()
        self.call("cudaEventCreate", ctypes.byref(e))
        return e.value

    def elapsed_ms(self, a, b):
        ms = ctypes.c_float()
        self.call("cudaEventElapsedTime", ctypes.byref(ms), ctypes.c_void_p(a), ctypes.c_void_p(b))
        return float(ms.value)


class UniqueId(ctypes.Structure):
    # raw bytes: a c_char array would read back only up to its first zero byte
    _fields_ = [("internal", ctypes.c_ubyte * 128)]


class RefNccl:
    """The reference's libnccl (MSCCL 0.1 on NCCL 2.12.12) through its public C API."""

    def __init__(self):
        self.lib = ctypes.CDLL(NCCL_SO, mode=os.RTLD_LOCAL)
        self.lib.ncclGetErrorString.restype = ctypes.c_char_p
        self.lib.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, UniqueId, ctypes.c_int]
        self.lib.ncclAllReduce.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        self.lib.ncclCommDestroy.argtypes = [ctypes.c_void_p]
        v = ctypes.c_int()
        self.check(self.lib.ncclGetVersion(ctypes.byref(v)), "ncclGetVersion")
        self.version = v.value

    def check(self, rc, what):
        if rc != 0:
            raise RuntimeError("%s: %s" % (what, self.lib.ncclGetErrorString(rc).decode()))

    def unique_id(self) -> bytes:
        uid = UniqueId()
        self.check(self.lib.ncclGetUniqueId(ctypes.byref(uid)), "ncclGetUniqueId")
        return bytes(uid.internal)

    def init_rank(self, nranks, uid: bytes, rank):
        comm = ctypes.c_void_p()
        if len(uid) != 128:
            raise ValueError("an ncclUniqueId has 128 bytes, got %d" % len(uid))
        u = UniqueId.from_buffer_copy(uid)
        self.check(self.lib.ncclCommInitRank(ctypes.byref(comm), nranks, u, rank), "ncclCommInitRank")
        return comm.value

    def all_reduce(self, send, recv, count, dtype, op, comm, stream):
        self.check(self.lib.ncclAllReduce(send, recv, count, dtype, op, comm, stream), "ncclAllReduce")


def exchange_unique_id(nccl: RefNccl, rank: int, world: int, timeout_s: float = 180.0) -> bytes:
    """Rank 0 publishes the id in a file every local rank of this launch can name (same parent, same port)."""
    d = "/tmp/vb_refarm_%d_%s" % (os.getppid(), os.environ.get("MASTER_PORT", "0"))
    path = os.path.join(d, "unique_id")
    if rank == 0:
        os.makedirs(d, exist_ok=True)
        uid = nccl.unique_id()
        tmp = path + ".tmp"
        with open(tmp, "wb") as f:
            f.write(uid)
        os.replace(tmp, path)
        return uid
    deadline = time.monotonic() + timeout_s
    while time.monotonic() < deadline:
        if os.path.isfile(path):
            with open(path, "rb") as f:
                data = f.read()
            if len(data) == 128:
                return data
        time.sleep(0.05)
    raise RuntimeError("rank %d: no ncclUniqueId from rank 0 within %.0f s" % (rank, timeout_s))


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 → bfloat16 bit patterns, round to nearest even."""
    u = x.astype(np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def run(args, clock_sampler_cls, metric: str, model: str) -> int:
    """The arm, guarded: any failure prints the ``unavailable`` line (rank 0) instead of a traceback, and a
    watchdog ends a process whose NCCL calls never return (VB_REF_DEADLINE_S, default 600 s)."""
    import threading
    rank = int(os.environ.get("RANK", "0"))
    deadline = float(os.environ.get("VB_REF_DEADLINE_S", "600"))

    def expire():
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference library did not finish within "
                              "%.0f s (stopped by the arm's watchdog)" % deadline}), flush=True)
        os._exit(0)

    watchdog = threading.Timer(deadline, expire)
    watchdog.daemon = True
    watchdog.start()
    try:
        return _run(args, clock_sampler_cls, metric, model)
    except Exception as error:          # noqa: BLE001 - reported as the arm's outcome
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "reference run failed: %s: %s"
                              % (type(error).__name__, str(error)[:300])}), flush=True)
        return 0
    finally:
        watchdog.cancel()


def _run(args, clock_sampler_cls, metric: str, model: str) -> int:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    reason = unavailable_reason(world)
    if reason is not None:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
        return 0
    if world != args.gpus:
        raise SystemExit("--gpus %d but WORLD_SIZE=%d (launch N>1 with torchrun)" % (args.gpus, world))
    # every rank of this launch is on this host: NCCL's TCP bootstrap goes over the loopback interface
    # (an NCCL setting; the library is unchanged)
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    rt = CudaRT()
    rt.call("cudaSetDevice", local)
    nccl = RefNccl()
    ops = ctypes.CDLL(GPUOPS_SO)
    # void vericcl_scale_output(void*, size_t, ncclDataType_t, int divisor, cudaStream_t) (C++ linkage)
    scale_fn = getattr(ops, "_Z20vericcl_scale_outputPvm14ncclDataType_tiP11CUstream_st")
    scale_fn.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    scale_fn.restype = None
    divisor = int(round(1.0 / args.scale))
    if abs(1.0 / divisor - args.scale) > 1e-12:
        raise SystemExit("the reference's scale pass divides by an integer; scale must be 1/k")
    uid = exchange_unique_id(nccl, rank, world) if world > 1 else nccl.unique_id()
    comm = nccl.init_rank(world, uid, rank)
    stream = rt.stream()

    esize = 2
    total = args.params
    bucket = args.bucket_bytes // esize
    buckets = -(-total // bucket)
    grads = rt.malloc(buckets * bucket * esize)
    # synthetic N(0, 0.02) gradients: one 64 MiB random block per rank, tiled over the buffer on the device
    block = min(total, 32 << 20)
    rng = np.random.default_rng(1234 + rank)
    host_block = bf16_bits(rng.standard_normal(block, dtype=np.float32) * np.float32(0.02))
    rt.call("cudaMemcpy", ctypes.c_void_p(grads), host_block.ctypes.data_as(ctypes.c_void_p), block * esize, H2D)
    off = block
    while off < total:
        n = min(block, total - off)
        rt.call("cudaMemcpyAsync", ctypes.c_void_p(grads + off * esize), ctypes.c_void_p(grads), n * esize, D2D,
                ctypes.c_void_p(stream))
        off += n
    pad = buckets * bucket - total
    if pad:
        rt.call("cudaMemsetAsync", ctypes.c_void_p(grads + total * esize), 0, pad * esize, ctypes.c_void_p(stream))
    small = rt.malloc(64)

    def sync_step():
        for i in range(buckets):
            p = grads + i * bucket * esize
            nccl.all_reduce(p, p, bucket, NCCL_BF16, NCCL_SUM, comm, stream)
            scale_fn(p, bucket, NCCL_BF16, divisor, stream)

    def all_max(x: float) -> float:
        v = np.array([x], dtype=np.float64)
        rt.call("cudaMemcpy", ctypes.c_void_p(small), v.ctypes.data_as(ctypes.c_void_p), 8, H2D)
        nccl.all_reduce(small, small, 1, NCCL_F64, NCCL_MAX, comm, stream)
        rt.call("cudaStreamSynchronize", ctypes.c_void_p(stream))
        rt.call("cudaMemcpy", v.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(small), 8, D2H)
        return float(v[0])

    def barrier():
        all_max(0.0)

    # correctness of one sync on the first 4096 elements against the fp64 host result of every rank's block
    rt.call("cudaStreamSynchronize", ctypes.c_void_p(stream))
    sync_step()
    rt.call("cudaStreamSynchronize", ctypes.c_void_p(stream))
    got = np.empty(4096, dtype=np.uint16)
    rt.call("cudaMemcpy", got.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(grads), got.nbytes, D2H)
    expect = np.zeros(4096, dtype=np.float64)
    for r in range(world):
        g = np.random.default_rng(1234 + r)
        expect += bf16_to_f32(bf16_bits(g.standard_normal(block, dtype=np.float32)[:4096] * np.float32(0.02)))
    expect /= divisor
    err = float(np.abs(bf16_to_f32(got).astype(np.float64) - expect).max())
    check_ok = all_max(1.0 if err > 2e-2 * max(1e-6, float(np.abs(expect).max())) else 0.0) == 0.0

    for _ in range(args.warmup):
        sync_step()
    rt.call("cudaStreamSynchronize", ctypes.c_void_p(stream))
    barrier()
    t0, t1 = rt.event(), rt.event()
    with clock_sampler_cls([local] if world == 1 else list(range(world)), enabled=rank == 0) as clocks:
        barrier()
        rt.call("cudaEventRecord", ctypes.c_void_p(t0), ctypes.c_void_p(stream))
        for _ in range(args.steps):
            sync_step()
        rt.call("cudaEventRecord", ctypes.c_void_p(t1), ctypes.c_void_p(stream))
        rt.call("cudaEventSynchronize", ctypes.c_void_p(t1))
        barrier()
    ms = all_max(rt.elapsed_ms(t0, t1) / args.steps)
    clock_info = clocks.summary() if rank == 0 else None

    e2e = None
    if not args.no_e2e:
        nbytes = total * esize
        host = rt.host_alloc(nbytes)
        hv = np.ctypeslib.as_array(ctypes.cast(host, ctypes.POINTER(ctypes.c_uint16)), shape=(total,))
        for lo in range(0, total, block):
            hi = min(total, lo + block)
            hv[lo:hi] = host_block[:hi - lo]
        out_host = rt.host_alloc(65536)
        e0, e1 = rt.event(), rt.event()

        def e2e_step():
            rt.call("cudaMemcpyAsync", ctypes.c_void_p(grads), ctypes.c_void_p(host), nbytes, H2D, ctypes.c_void_p(stream))
            sync_step()
            rt.call("cudaMemcpyAsync", ctypes.c_void_p(out_host), ctypes.c_void_p(grads), 65536, D2H,
                    ctypes.c_void_p(stream))
            rt.call("cudaStreamSynchronize", ctypes.c_void_p(stream))
            _ = ctypes.cast(out_host, ctypes.POINTER(ctypes.c_uint16))[0]

        e2e_step()
        barrier()
        rt.call("cudaEventRecord", ctypes.c_void_p(e0), ctypes.c_void_p(stream))
        for _ in range(args.e2e_steps):
            e2e_step()
        rt.call("cudaEventRecord", ctypes.c_void_p(e1), ctypes.c_void_p(stream))
        rt.call("cudaEventSynchronize", ctypes.c_void_p(e1))
        ems = all_max(rt.elapsed_ms(e0, e1) / args.e2e_steps)
        bus = total * esize * (2.0 * (world - 1) / world if world > 1 else 1.0)
        e2e = {"value": round(bus / (ems * 1e-3) / 1e9 * world, 2), "unit": "GB/s (sum over GPUs of per-GPU bus bandwidth)",
               "ms_per_step": round(ems, 3), "h2d_bytes_per_step": int(nbytes), "d2h_bytes_per_step": 65536,
               "api": "ncclAllReduce + vericcl_scale_output per bucket after a pinned host->device copy"}
        rt.call("cudaFreeHost", ctypes.c_void_p(host))
        rt.call("cudaFreeHost", ctypes.c_void_p(out_host))

    barrier()
    bus = total * esize * (2.0 * (world - 1) / world if world > 1 else 1.0)
    busbw = bus / (ms * 1e-3) / 1e9
    if rank == 0:
        v = nccl.version
        vs = "%d.%d.%d" % (v // 1000, v % 1000 // 100, v % 100) if v < 10000 else \
            "%d.%d.%d" % (v // 10000, v % 10000 // 100, v % 100)
        line = {"metric": metric, "value": round(busbw * world, 2),
                "unit": "GB/s (sum over GPUs of per-GPU bus bandwidth)", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic N(0,0.02) gradients, random init", "impl": "reference",
                "config": {"model": model, "global_batch": None, "seq_len": None, "parallelism": "dp%d" % world,
                           "bucket_bytes": args.bucket_bytes, "buckets": buckets, "bytes_per_rank": total * esize,
                           "scale": args.scale,
                           "schedule": "reference MSCCL/NCCL %s ncclAllReduce SUM per bucket + vericcl_scale_output"
                                       % vs,
                           "nccl_algo": os.environ.get("NCCL_ALGO", "library default"),
                           "nccl_socket_ifname": os.environ.get("NCCL_SOCKET_IFNAME"),
                           "library": os.path.relpath(NCCL_SO, os.path.dirname(HERE)),
                           "l2": "inputs (16 GB) larger than the 126 MB L2; no flush needed"},
                "busbw_per_gpu_gbs": round(busbw, 2),
                "check": {"first_4096_max_err": err, "ok": bool(check_ok), "reference": "fp64 host sum x scale"},
                "clocks": clock_info, "e2e": e2e}
        print(json.dumps(line), flush=True)
    nccl.lib.ncclCommDestroy(ctypes.c_void_p(comm))
    if rank == 0 and world > 1:
        d = "/tmp/vb_refarm_%d_%s" % (os.getppid(), os.environ.get("MASTER_PORT", "0"))
        for name in ("unique_id",):
            try:
                os.remove(os.path.join(d, name))
            except OSError:
                pass
        try:
            os.rmdir(d)
        except OSError:
            pass
    return 0
