"""The allocation-free AllReduce entry point, called through its exported C symbol.

``vb_allreduce_local_noalloc`` (libvericcl_b200.so, declared in
csrc/include/vericcl_b200_noalloc.h) serves callers that must not allocate
device memory on their call path: it runs the single-rank AllReduce schedule
with its fused scale through the interpreter kernel, taking all of the
kernel's working memory from a fixed static device array.  This test checks
it on two calls in a row against the regular entry point (the PyTorch
collective engine, which stages through heap memory) and against a plain fp32
PyTorch computation of the same result, reads the kernel status after each
call, covers in == out, and checks that oversized requests are refused.  It lives in its own file, collected last, so a
failing run that stops at the first failure has already run every other test.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from vericcl_b200.ops.build import build_capi
    handle = ctypes.CDLL(str(build_capi()))
    handle.vb_allreduce_local_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                                  ctypes.c_float, ctypes.c_void_p]
    handle.vb_allreduce_local_noalloc.restype = ctypes.c_int
    handle.vb_noalloc_last_error.restype = ctypes.c_char_p
    handle.vb_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
    handle.vb_noalloc_status.restype = ctypes.c_int
    return handle


def kernel_status(lib):
    status, detail = ctypes.c_int(-1), (ctypes.c_int * 4)()
    assert lib.vb_noalloc_status(ctypes.byref(status), detail) == 0, lib.vb_noalloc_last_error()
    return status.value


@pytest.fixture(scope="module")
def engine():
    from vericcl_b200.models import CollectiveEngine
    from vericcl_b200.parallel import Communicator
    comm = Communicator(heap_bytes=64 << 20)
    yield CollectiveEngine(comm)
    comm.close()


CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
TOL = {torch.float32: 1e-6, torch.bfloat16: 1e-2, torch.float16: 1e-3}


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_matches_regular_entry_point_on_two_calls(lib, engine, dtype):
    stream = torch.cuda.current_stream()
    for call, (count, scale) in enumerate([(300_001, 0.125), (1 << 20, 0.5)]):
        x = torch.randn(count, device="cuda").to(dtype)
        expected = x.clone()
        engine.all_reduce(expected, scale=scale)
        out = torch.empty_like(x)
        rc = lib.vb_allreduce_local_noalloc(x.data_ptr(), out.data_ptr(), count, CODES[dtype], scale,
                                            stream.cuda_stream)
        assert rc == 0, lib.vb_noalloc_last_error()
        torch.cuda.synchronize()
        assert kernel_status(lib) == 0
        tol = dict(atol=TOL[dtype], rtol=TOL[dtype])
        assert torch.allclose(out.float(), expected.float(), **tol), "call %d vs engine" % call
        assert torch.allclose(out.float(), x.float() * scale, **tol), "call %d vs fp32 torch" % call


def test_in_place_call(lib):
    """``in`` and ``out`` may be the same buffer."""
    stream = torch.cuda.current_stream()
    x = torch.randn(123_457, device="cuda")
    ref = x.clone() * 0.25
    for _ in range(2):
        rc = lib.vb_allreduce_local_noalloc(x.data_ptr(), x.data_ptr(), x.numel(), 0, 0.5, stream.cuda_stream)
        assert rc == 0, lib.vb_noalloc_last_error()
    torch.cuda.synchronize()
    assert kernel_status(lib) == 0
    assert torch.allclose(x, ref, atol=1e-6, rtol=1e-6)


def test_rejects_requests_beyond_the_static_buffer(lib):
    x = torch.empty(1, device="cuda")
    too_many = (8 << 20) // 4 + 1
    rc = lib.vb_allreduce_local_noalloc(x.data_ptr(), x.data_ptr(), too_many, 0, 1.0, None)
    assert rc == 2
    assert b"exceeds" in lib.vb_noalloc_last_error()
