"""gpuos_ew_batch_noalloc: the element-wise batch entry point that allocates no device memory.

Called through the C ABI with ctypes.  Its outputs must equal, bit for bit, those of the
allocating path (gpuos_rt_submit_ew + gpuos_rt_flush) on the same inputs, on two calls in a
row: the second call shows that nothing left in the shared scratch array by the first one
leaks into it.  The file is named to run last; it also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

from oracle.reference_semantics import same_bits
from tests._items import LIB_PATH, operand

pytestmark = pytest.mark.gpu

GPUOS_FLUSH_SYNC = 1
GPUOS_ERR_INVALID = 1
MAX_TILES = 16384  # GPUOS_NOALLOC_MAX_TILES
ADD, MUL, EXP, GELU, ADD_ALPHA = 0, 1, 11, 17, 28


class EwRequest(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int), ("b_is_scalar", ctypes.c_int), ("nparams", ctypes.c_int),
                ("_pad", ctypes.c_int), ("b_scalar", ctypes.c_double), ("a", ctypes.c_void_p),
                ("b", ctypes.c_void_p), ("out", ctypes.c_void_p), ("params", ctypes.c_float * 4)]


assert ctypes.sizeof(EwRequest) == 64


def _lib():
    lib = ctypes.CDLL(LIB_PATH)
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.gpuos_ew_batch_noalloc.argtypes = [P, I, I, P]
    lib.gpuos_ew_batch_noalloc.restype = I
    lib.gpuos_rt_get.argtypes = [I]
    lib.gpuos_rt_get.restype = P
    lib.gpuos_rt_submit_ew.argtypes = [P, I, P, P, I, ctypes.c_double, P, P, I]
    lib.gpuos_rt_submit_ew.restype = I
    lib.gpuos_rt_flush.argtypes = [P, I, P, P]
    lib.gpuos_rt_flush.restype = I
    lib.gpuos_rt_last_error.restype = ctypes.c_char_p
    return lib


def _workload(seed):
    """Requests covering the tiled contiguous path, broadcast and strided operands, a 16-bit
    dtype, op parameters, a scalar operand and a read-after-write dependency."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(4096, 4096, generator=g).cuda()            # 4096 tiles of float32
    y = torch.randn(4096, 4096, generator=g).cuda()
    row = torch.randn(4096, generator=g).cuda()
    h = torch.randn(3, 1000, 517, generator=g).to(torch.bfloat16).cuda()
    t = torch.randn(600, 900, generator=g).cuda().t()          # transposed: strided input
    ins = dict(x=x, y=y, row=row, h=h, t=t)
    shapes = dict(s=(4096, 4096), m=(4096, 4096), e=h.shape, g=(900, 600), d=(4096, 4096))
    dtypes = dict(s=torch.float32, m=torch.float32, e=torch.bfloat16, g=torch.float32, d=torch.float32)
    # (op, a, b | float scalar | None, out, params); "d" reads "s" written earlier in the batch
    reqs = [(ADD, "x", "y", "s", []), (MUL, "x", "row", "m", []), (EXP, "h", None, "e", []),
            (GELU, "t", None, "g", []), (ADD_ALPHA, "s", "x", "d", [0.75])]
    return ins, shapes, dtypes, reqs


def _outputs(shapes, dtypes):
    # garbage (NaN) everywhere: an untouched element shows up as a mismatch
    return {k: torch.full(shapes[k], float("nan"), dtype=dtypes[k], device="cuda") for k in shapes}


def _ops(ins, outs, reqs):
    keep = []
    plan = []
    for op, a, b, o, params in reqs:
        A = operand(ins.get(a, outs.get(a)))
        B = operand(ins.get(b, outs.get(b))) if isinstance(b, str) else None
        O = operand(outs[o])
        keep += [A, B, O]
        plan.append((op, A, B, O, params))
    return plan, keep


def _run_existing(lib, ins, outs, reqs):
    rt = lib.gpuos_rt_get(0)
    assert rt, "runtime not initialised"
    plan, keep = _ops(ins, outs, reqs)
    for op, A, B, O, params in plan:
        pa = (ctypes.c_float * 4)(*params)
        rc = lib.gpuos_rt_submit_ew(rt, op, ctypes.byref(A), ctypes.byref(B) if B is not None else None,
                                    0, 0.0, ctypes.byref(O), pa, len(params))
        assert rc == 0, lib.gpuos_rt_last_error()
    rc = lib.gpuos_rt_flush(rt, GPUOS_FLUSH_SYNC, None, None)
    assert rc == 0, lib.gpuos_rt_last_error()


def _run_noalloc(lib, ins, outs, reqs, stream, flags=GPUOS_FLUSH_SYNC):
    plan, keep = _ops(ins, outs, reqs)
    arr = (EwRequest * len(plan))()
    for r, (op, A, B, O, params) in zip(arr, plan):
        r.op = op
        r.a = ctypes.addressof(A)
        r.b = ctypes.addressof(B) if B is not None else None
        r.out = ctypes.addressof(O)
        r.nparams = len(params)
        for i, v in enumerate(params):
            r.params[i] = v
    rc = lib.gpuos_ew_batch_noalloc(arr, len(plan), flags, ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.gpuos_rt_last_error()


def test_noalloc_matches_allocating_path_twice(rt):
    lib = _lib()
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    for call, seed in enumerate((11, 12)):
        ins, shapes, dtypes, reqs = _workload(seed)
        want = _outputs(shapes, dtypes)
        _run_existing(lib, ins, want, reqs)
        got = _outputs(shapes, dtypes)
        torch.cuda.synchronize()
        # the second call is asynchronous and is read after a stream synchronisation
        _run_noalloc(lib, ins, got, reqs, stream, flags=GPUOS_FLUSH_SYNC if call == 0 else 0)
        stream.synchronize()
        for k in shapes:
            assert not torch.isnan(want[k].float()).any(), f"allocating path left {k} unwritten"
            assert same_bits(got[k].cpu(), want[k].cpu()), f"call {call}: output {k} differs"
        # the dependent request ("d" reads "s") saw the finished result of "s": s = x + y exactly
        x = ins["x"].cpu()
        s = x + ins["y"].cpu()
        assert same_bits(got["s"].cpu(), s)
        # d = s + 0.75 x with one rounding (fused), within one rounding step of the operands
        err = (got["d"].cpu().double() - (s.double() + 0.75 * x.double())).abs()
        assert bool((err <= 2.0 ** -24 * (s.double().abs() + 0.75 * x.double().abs()) + 1e-30).all())


def test_noalloc_rejects_batches_beyond_the_limit(rt):
    lib = _lib()
    stream = torch.cuda.Stream()
    x = torch.zeros(MAX_TILES * 4096 + 1, device="cuda")   # one element more than the tiles hold
    A = operand(x)
    r = EwRequest(op=ADD)
    r.a = r.b = r.out = ctypes.addressof(A)
    rc = lib.gpuos_ew_batch_noalloc(ctypes.byref(r), 1, GPUOS_FLUSH_SYNC, ctypes.c_void_p(stream.cuda_stream))
    assert rc == GPUOS_ERR_INVALID
    assert b"GPUOS_NOALLOC_MAX_TILES" in lib.gpuos_rt_last_error()
    assert not bool(x.any())
    assert lib.gpuos_ew_batch_noalloc(ctypes.byref(r), 1, 4, ctypes.c_void_p(stream.cuda_stream)) == GPUOS_ERR_INVALID


def test_noalloc_allocates_no_device_memory(rt):
    """After a first call (which resolves the array's address), further calls change neither the
    device's free memory nor the caching allocator's reservation; an empty synchronous call is a
    status query that reports no earlier device error."""
    lib = _lib()
    stream = torch.cuda.Stream()
    ins, shapes, dtypes, reqs = _workload(13)
    got = _outputs(shapes, dtypes)
    _run_noalloc(lib, ins, got, reqs, stream)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    reserved0 = torch.cuda.memory_reserved()
    for flags in (GPUOS_FLUSH_SYNC, 0, 0, GPUOS_FLUSH_SYNC):
        _run_noalloc(lib, ins, got, reqs, stream, flags=flags)
    rc = lib.gpuos_ew_batch_noalloc(None, 0, GPUOS_FLUSH_SYNC, ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.gpuos_rt_last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_reserved() == reserved0
