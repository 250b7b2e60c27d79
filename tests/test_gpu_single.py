"""Single-GPU numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comm():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from vericcl_b200.parallel import Communicator
    c = Communicator(heap_bytes=256 << 20)
    yield c
    c.close()


def test_extension_loaded_from_tree():
    from vericcl_b200.ops import native
    mod = native.cuda()
    assert "vericcl_b200/_native/_vbcuda" in mod.__file__


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("lanes,iters", [(1, 1), (37, 3), (148, 1)])
def test_single_rank_allreduce_scale_matches_reference(comm, dtype, lanes, iters):
    from vericcl_b200.synthesis import schedule_xml
    dname = str(dtype).split(".")[-1]
    plan = comm.compile(schedule_xml("allreduce", 1, 1, inplace=False, datatype=dname), nlanes=lanes, niters=iters)
    n = 1 << 18
    x = comm.empty(n, dtype)
    y = comm.empty(n, dtype)
    x.copy_(torch.randn(n, device="cuda"))
    comm.run(plan, x, y, scale=0.37)
    torch.cuda.synchronize()
    comm.check_status()
    ref = x.float() * 0.37
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert torch.allclose(y.float(), ref, atol=tol, rtol=tol)
    comm.free(x)
    comm.free(y)


def test_batched_launch_covers_every_instance(comm):
    from vericcl_b200.synthesis import schedule_xml
    plan = comm.compile(schedule_xml("allreduce", 1, 1, inplace=True, datatype="bfloat16"), nlanes=64)
    per, nb = 8192, 5
    buf = comm.empty(per * nb, torch.bfloat16)
    src = torch.randn(per * nb, device="cuda").to(torch.bfloat16)
    buf.copy_(src)
    comm.run(plan, buf[:per], buf[:per], scale=0.5, nbatch=nb, in_stride=per, out_stride=per)
    torch.cuda.synchronize()
    comm.check_status()
    assert torch.allclose(buf.float(), src.float() * 0.5, atol=1e-2)


def test_engine_all_reduce_non_heap_tensor(comm):
    from vericcl_b200.models import CollectiveEngine
    eng = CollectiveEngine(comm)
    t = torch.randn(10001, device="cuda")   # not in the heap, not a multiple of the vector width
    ref = t.clone() * 0.25
    eng.all_reduce(t, scale=0.25)
    torch.cuda.synchronize()
    assert torch.allclose(t, ref, atol=1e-6)


def test_helper_kernels(comm):
    mod = comm._mod
    x = torch.empty(4096, device="cuda")
    mod.fill(x, 0, 3, 0)
    i = torch.arange(4096, device="cuda")
    assert torch.equal(x, 1.0 + ((9 + i) % 5).float())
    y = torch.empty_like(x)
    mod.scale(y, x, 2.0)
    assert torch.equal(y, 2 * x)
    # a 1-rank AllReduce of pattern 0 is the pattern itself: the analytic checker finds no error
    mod.fill(x, 0, 0, 0)
    assert int(mod.check(x, 0, 0, 1, 0, 4096, 0.0, 0.0).item()) == 0
    x[7] += 1
    assert int(mod.check(x, 0, 0, 1, 0, 4096, 0.0, 0.0).item()) == 1
    t = torch.zeros(1, dtype=torch.int64, device="cuda")
    mod.read_timer(t)
    torch.cuda.synchronize()
    assert int(t.item()) > 0


@pytest.mark.parametrize("dtype,rows,cols,pitch", [(torch.float32, 37, 64, 100), (torch.bfloat16, 5, 8, 8),
                                                    (torch.float16, 129, 3, 7), (torch.uint8, 9, 33, 40)])
def test_strided_copy_matches_torch(comm, dtype, rows, cols, pitch):
    """The 2D pitched copy (16/8/4/1-byte paths) against torch's own copy of the same views."""
    base = (torch.arange(rows * pitch, device="cuda") % 251).to(dtype).view(rows, pitch)
    src = base[:, 1:1 + cols] if pitch > cols else base
    dst_store = torch.full((rows, pitch + 3), 7, device="cuda").to(dtype)
    before = dst_store.clone()
    dst = dst_store[:, :cols]
    comm._mod.strided_copy(dst, src)
    torch.cuda.synchronize()
    assert torch.equal(dst, src)
    assert torch.equal(dst_store[:, cols:], before[:, cols:])      # nothing written past the rows
    flat = torch.empty(rows, cols, device="cuda").to(dtype)
    comm._mod.strided_copy(flat, src)
    assert torch.equal(flat, src.contiguous())


def test_engine_collectives_on_strided_views(comm):
    """A column slice of a matrix goes through the engine without a contiguous copy by the caller."""
    from vericcl_b200.models import CollectiveEngine
    eng = CollectiveEngine(comm)
    m = torch.randn(64, 96, device="cuda")
    view = m[:, 16:80]
    expect = view.clone() * 0.5
    keep = m[:, :16].clone()
    eng.all_reduce(view, scale=0.5)
    torch.cuda.synchronize()
    assert torch.allclose(view, expect, atol=1e-6) and torch.equal(m[:, :16], keep)
    out = torch.zeros(64, 200, device="cuda")[:, 10:74]
    eng.all_gather(view, out)                      # one rank: out = input
    torch.cuda.synchronize()
    assert torch.equal(out, view)


def test_trace_capture(comm):
    from vericcl_b200.online.trace import analyze_trace_causality, capture_once
    from vericcl_b200.synthesis import schedule_xml
    plan = comm.compile(schedule_xml("allreduce", 1, 1), nlanes=8, niters=2)
    x, y = comm.empty(1 << 16), comm.empty(1 << 16)
    x.fill_(1.0)
    out = capture_once(comm, plan, x, y)
    assert out["records"], "the traced launch recorded no steps"
    report = analyze_trace_causality({0: out["records"]}, {0: out["clock"]})
    assert report["global_span_us"] > 0


def test_device_timeout_is_reported_not_hung(comm):
    """A wait on a flag nothing sets gives up after its limit and reports ST_TIMEOUT (no fault, no hang)."""
    status = comm._mod.wait_probe(comm.heap, 0.2)
    torch.cuda.synchronize()
    assert status["status"] == 1
    comm.heap.clear_status()
    # the context stays usable afterwards
    x = comm.empty(4096)
    x.fill_(2.0)
    torch.cuda.synchronize()
    assert float(x.sum()) == 8192.0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fp8_block_quantization_matches_torch(comm, dtype):
    mod = comm._mod
    n, block = 4096 + 77, 128
    x = (torch.randn(n, device="cuda") * 3).to(dtype)
    nb = -(-n // block)
    q = torch.empty(n, dtype=torch.uint8, device="cuda")
    s = torch.empty(nb, dtype=torch.float32, device="cuda")
    mod.quantize_fp8(x, q, s, block)
    xf = torch.nn.functional.pad(x.float(), (0, nb * block - n)).view(nb, block)
    ref_s = xf.abs().amax(dim=1) / 448.0
    ref_s[ref_s == 0] = 1.0
    assert torch.allclose(s, ref_s, rtol=1e-6)
    ref_q = (xf / ref_s[:, None]).to(torch.float8_e4m3fn).view(-1)[:n].view(torch.uint8)
    assert (q != ref_q).sum().item() <= n // 1000 + 1
    out = torch.empty(n, dtype=dtype, device="cuda")
    mod.dequantize_fp8(q, s, out, block)
    rel = ((out.float() - x.float()).abs() / xf.abs().amax(dim=1).repeat_interleave(block)[:n].clamp_min(1e-6))
    assert rel.max().item() < 0.07          # e4m3 keeps 3 mantissa bits


def test_engine_all_gather_fp8_single_rank(comm):
    from vericcl_b200.models import CollectiveEngine
    eng = CollectiveEngine(comm)
    x = torch.randn(10240, device="cuda")
    out = torch.empty_like(x)
    eng.all_gather_fp8(x, out)
    torch.cuda.synchronize()
    assert torch.allclose(out, x, atol=0.07 * x.abs().max().item())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [4096, 10240 + 48, 1 << 20])
def test_fused_fp8_all_gather_matches_three_pass_path(comm, dtype, n):
    """One rank: the fused kernel (quantize, publish, dequantize) gives the three-pass path's values."""
    from vericcl_b200.models import CollectiveEngine
    eng = CollectiveEngine(comm)
    x = (torch.randn(n, device="cuda") * 2).to(dtype)
    slow = torch.empty_like(x)
    eng.all_gather_fp8(x, slow, fused=False)
    for _ in range(3):                                  # both staging parities, then the first again
        out = torch.full_like(x, float("nan"))
        eng.all_gather_fp8(x, out, fused=True)
        torch.cuda.synchronize()
        comm.check_status()
        assert not torch.isnan(out.float()).any()
        xf = torch.nn.functional.pad(x.float(), (0, (-n) % 128)).view(-1, 128)
        amax = xf.abs().amax(dim=1).repeat_interleave(128)[:n]
        assert ((out.float() - x.float()).abs() / amax.clamp_min(1e-6)).max().item() < 0.07
        assert (out.float() - slow.float()).abs().max().item() <= 1e-2 * float(amax.max()) / 448


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_oneshot_kernel_single_rank(comm, dtype):
    """The one-shot kernel on one rank: AllReduce is the scaled copy, AllGather the copy; the tag counter advances."""
    n = 4096
    plan_ar = comm.oneshot_plan("allreduce", 64 << 10)
    plan_ag = comm.oneshot_plan("allgather", 64 << 10)
    x = comm.empty(n, dtype)
    y = comm.empty(n, dtype)
    src = torch.randn(n, device="cuda").to(dtype)
    seq0 = comm.status()["ll_seq"]
    for rep in range(3):
        x.copy_(src)
        comm.run(plan_ar, x, y, scale=0.25)
        comm.run(plan_ag, x, x)
        torch.cuda.synchronize()
        comm.check_status()
        tol = 1e-6 if dtype == torch.float32 else 1e-2
        assert torch.allclose(y.float(), src.float() * 0.25, atol=tol, rtol=tol)
        assert torch.equal(x, src)
    assert comm.status()["ll_seq"] == seq0 + 6
    comm.free(x)
    comm.free(y)


def test_bound_launch_follows_the_tensor_size(comm):
    """The same plan and pointers with a longer view must not replay the shorter launch."""
    from vericcl_b200.synthesis import schedule_xml
    plan = comm.compile(schedule_xml("allreduce", 1, 1, inplace=False, datatype="float32"), nlanes=8)
    n = 1 << 14
    x = comm.empty(2 * n, torch.float32)
    y = comm.empty(2 * n, torch.float32)
    x.copy_(torch.randn(2 * n, device="cuda"))
    y.zero_()
    comm.run(plan, x[:n], y[:n], scale=2.0)
    comm.run(plan, x, y, scale=2.0)
    torch.cuda.synchronize()
    comm.check_status()
    assert torch.allclose(y, x * 2.0)
    comm.free(x)
    comm.free(y)


REDOPS = {"sum": 0, "prod": 1, "min": 2, "max": 3}


def _reference(stack: torch.Tensor, op: str) -> torch.Tensor:
    x = stack.float()
    if op == "sum":
        return x.sum(0)
    if op == "prod":
        return x.prod(0)
    return x.amin(0) if op == "min" else x.amax(0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("op", ["sum", "prod", "min", "max"])
@pytest.mark.parametrize("k", [1, 2, 3, 4, 5, 6, 7, 8, 9, 12])
def test_local_multi_source_reduce_matches_fp32_reference(comm, dtype, op, k):
    """The interpreter's K-source move paths (fixed K = 1..8, generic above) for every reduction and dtype."""
    n = 3 * 4096 + 64
    gen = torch.Generator(device="cuda").manual_seed(100 * k + REDOPS[op])
    if op == "prod":
        srcs = (0.5 + torch.rand(k, n, device="cuda", generator=gen)).to(dtype)
    else:
        srcs = torch.randn(k, n, device="cuda", generator=gen).to(dtype)
    dst = torch.empty(n, device="cuda", dtype=dtype)
    scale = 0.37 if op == "sum" else 1.0
    ws = comm._mod.local_reduce(dst, srcs, REDOPS[op], scale, op == "sum", 7, 2, False)
    torch.cuda.synchronize()
    assert int(ws[12:16].view(torch.int32).item()) == 0          # the control block's status word
    ref = _reference(srcs, op) * scale
    tol = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 2e-3}[dtype]
    assert torch.allclose(dst.float(), ref, atol=tol * max(1.0, k ** 0.5), rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("k", [1, 2, 3, 8])
def test_lean_instance_local_reduce(comm, dtype, k):
    """The register-lean interpreter instance (sum and copies) on the same one-step programs."""
    n = 1 << 16
    srcs = torch.randn(k, n, device="cuda").to(dtype)
    dst = torch.empty(n, device="cuda", dtype=dtype)
    ws = comm._mod.local_reduce(dst, srcs, 0, 0.5, True, 64, 1, True)
    torch.cuda.synchronize()
    assert int(ws[12:16].view(torch.int32).item()) == 0
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert torch.allclose(dst.float(), srcs.float().sum(0) * 0.5, atol=tol * 2, rtol=tol)


@pytest.mark.parametrize("k", [1, 2, 5, 8])
def test_reduce_probe_matches_torch(comm, k):
    n = 1 << 18
    srcs = [torch.randn(n, device="cuda") for _ in range(k)]
    dst = torch.empty(n, device="cuda")
    comm._mod.reduce_probe(dst.data_ptr(), [s.data_ptr() for s in srcs], n * 4, 64, 256)
    torch.cuda.synchronize()
    assert torch.allclose(dst, torch.stack(srcs).sum(0), atol=1e-5, rtol=1e-5)


def test_copy_probe_matches_source(comm):
    n = 1 << 18
    src = torch.randn(n, device="cuda")
    dst = torch.zeros_like(src)
    comm._mod.copy_probe(dst.data_ptr(), src.data_ptr(), n * 4, 32, 256, 4)
    torch.cuda.synchronize()
    assert torch.equal(dst, src)


def test_push_allgather_kernel_single_rank(comm):
    """One rank: the push kernel copies the chunk into part 0 of the heap output; its counter advances."""
    mod = comm._mod
    ctas = max(1, min(mod.push_allgather_max_ctas(), 148))
    flags = comm.empty(4 * (ctas + 1), torch.float16)
    flags.zero_()
    x = torch.randn(4096 * 3 + 4, device="cuda")
    out = comm.empty(x.numel())
    before = comm.heap.status()
    for fanout in (False, False, True, True):
        out.zero_()
        mod.push_allgather(comm.heap, x.data_ptr(), comm.offset_of(out), x.numel() * 4, comm.offset_of(flags), ctas,
                           10.0, fanout)
        torch.cuda.synchronize()
        comm.check_status()
        assert torch.equal(out, x)
    comm.free(out)
    comm.free(flags)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("op", ["sum", "prod", "min", "max"])
@pytest.mark.parametrize("k", [1, 2, 3, 5, 8, 12])
def test_tma_staged_reduce_matches_fp32_reference(comm, dtype, op, k):
    """The TMA-staged instance: sources reach shared memory by cp.async.bulk (several tiles per piece, a partial
    last tile), are combined in fp32 and stored; same results as the fp32 reference."""
    n = (1 << 20) + 96
    gen = torch.Generator(device="cuda").manual_seed(7 * k + REDOPS[op])
    if op == "prod":
        srcs = (0.9 + 0.2 * torch.rand(k, n, device="cuda", generator=gen)).to(dtype)
    else:
        srcs = torch.randn(k, n, device="cuda", generator=gen).to(dtype)
    dst = torch.full((n,), float("nan"), device="cuda", dtype=dtype)
    scale = 0.37 if op == "sum" else 1.0
    ws = comm._mod.local_reduce(dst, srcs, REDOPS[op], scale, op == "sum", 4, 2, False, 1)
    torch.cuda.synchronize()
    assert int(ws[12:16].view(torch.int32).item()) == 0
    ref = _reference(srcs, op) * scale
    tol = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 2e-3}[dtype]
    assert torch.allclose(dst.float(), ref, atol=tol * max(1.0, k ** 0.5), rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tma_staged_single_rank_allreduce_through_the_engine(comm, dtype):
    from vericcl_b200.synthesis import schedule_xml
    dname = str(dtype).split(".")[-1]
    plan = comm.compile(schedule_xml("allreduce", 1, 1, inplace=False, datatype=dname), nlanes=16, niters=2)
    n = 1 << 22
    x, y = comm.empty(n, dtype), comm.empty(n, dtype)
    x.copy_(torch.randn(n, device="cuda"))
    saved, comm.bulk = comm.bulk, 1
    try:
        for _ in range(2):
            y.fill_(float("nan"))
            comm.run(plan, x, y, scale=0.25)
            torch.cuda.synchronize()
            comm.check_status()
            tol = 1e-6 if dtype == torch.float32 else 1e-2
            assert torch.allclose(y.float(), x.float() * 0.25, atol=tol, rtol=tol)
    finally:
        comm.bulk = saved
        comm.free(x)
        comm.free(y)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [(1 << 20) + 96, 3 * (1 << 16) + 8])
def test_tma_store_copy_is_exact(comm, dtype, n):
    """Staged plain copy written back by TMA bulk stores (mode 3): bit-exact, twice in a row on one workspace."""
    gen = torch.Generator(device="cuda").manual_seed(n)
    src = torch.randn(1, n, device="cuda", generator=gen).to(dtype)
    for _ in range(2):
        dst = torch.full((n,), float("nan"), device="cuda", dtype=dtype)
        ws = comm._mod.local_reduce(dst, src, 0, 1.0, False, 8, 2, False, 3)
        torch.cuda.synchronize()
        assert int(ws[12:16].view(torch.int32).item()) == 0
        assert torch.equal(dst, src[0])


def test_tma_store_engine_allgather_single_rank(comm):
    """A one-rank AllGather through the engine with TMA loads and stores: the output equals the input."""
    from vericcl_b200.synthesis import schedule_xml
    plan = comm.compile(schedule_xml("allgather", 1, 1, inplace=False, datatype="bfloat16"), nlanes=16, niters=2)
    n = 1 << 22
    x, y = comm.empty(n, torch.bfloat16), comm.empty(n, torch.bfloat16)
    x.copy_(torch.randn(n, device="cuda"))
    saved, comm.bulk = comm.bulk, 3
    try:
        for _ in range(2):
            y.fill_(float("nan"))
            comm.run(plan, x, y)
            torch.cuda.synchronize()
            comm.check_status()
            assert torch.equal(y, x)
    finally:
        comm.bulk = saved
        comm.free(x)
        comm.free(y)


def test_gradient_sync_from_host_matches_scaled_input(comm):
    """sync_from_host: bucket groups copied in from pinned memory, each AllReduced (one rank: scaled) after its copy."""
    from vericcl_b200.models import GradBucketAllReduce
    numel = 5 * 65536 + 1000                    # a partial last bucket
    ar = GradBucketAllReduce(comm, numel, dtype=torch.bfloat16, bucket_bytes=131072, scale=0.25)
    host = torch.randn(numel).to(torch.bfloat16).pin_memory()
    for step in range(2):
        ar.grads.fill_(float("nan"))
        ar.grads[numel:].zero_()
        launches = ar.sync_from_host(host, groups=3)
        torch.cuda.synchronize()
        comm.check_status()
        assert launches == 3
        ref = host.float() * 0.25
        assert torch.allclose(ar.flat.float().cpu(), ref, atol=1e-2, rtol=1e-2)
    comm.free(ar.grads)
