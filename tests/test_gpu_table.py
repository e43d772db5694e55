"""Op table: reference-layout Tasks dispatched through g_op_alias/g_op_table at dequeue time
(src/persistent_kernel.cu:184-193): online switch of slot 0 (test/online_switch.cpp), dual-
slot switch and rollback (test/dual_slot_switch.cpp), registered reductions
(pytorch_ext/gpuos_ext.cpp:1003-1045) and the reference's Task-ring worker C ABI."""
import ctypes
import hashlib
import json
import os
import time

import numpy as np
import pytest
import torch

from oracle.reference_semantics import same_bits
from tests._items import LIB_PATH

pytestmark = pytest.mark.gpu
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_known_answers.json")))


def digest(t):
    return hashlib.sha256(t.cpu().numpy().astype(np.float32).tobytes()).hexdigest()


def run_tasks(rt, slot, a, b, out, count):
    for _ in range(count):
        rt.submit_binary(slot, a, b, out)
    rt.flush(sync=True)


def test_online_switch_slot0(rt):
    g = GOLD["online_switch"]
    n = g["n"]
    i = torch.arange(n, dtype=torch.float32)
    A = (0.5 * i).cuda()
    B = (1.0 + (torch.arange(n) % 5).float()).cuda()
    c_add, c_mul = torch.zeros_like(A), torch.zeros_like(A)
    add_addr = rt.get_slot(0)
    mul_addr = rt.builtin_op_address(1)
    try:
        run_tasks(rt, 0, A, B, c_add, 128)      # slot 0 = add
        rt.set_slot(0, mul_addr)                 # online switch: slot 0 now multiplies
        run_tasks(rt, 0, A, B, c_mul, 128)
    finally:
        rt.set_slot(0, add_addr)
    assert digest(c_add) == g["c_add_sha256"]
    assert digest(c_mul) == g["c_mul_sha256"]


def test_dual_slot_switch_and_rollback(rt):
    g = GOLD["dual_slot"]
    n = g["n"]
    i = torch.arange(n, dtype=torch.float32)
    A = (0.3 * i).cuda()
    B = (2.0 + (torch.arange(n) % 9).float()).cuda()
    c1, c2, c3 = (torch.zeros_like(A) for _ in range(3))
    assert rt.get_alias(0) == 0
    try:
        run_tasks(rt, 0, A, B, c1, 96)
        rt.set_alias(0, 1)          # logical 0 -> physical 1 (mul)
        run_tasks(rt, 0, A, B, c2, 96)
        rt.set_alias(0, 0)          # rollback
        run_tasks(rt, 0, A, B, c3, 96)
    finally:
        rt.set_alias(0, 0)
    assert digest(c1) == g["c1_sha256"]
    assert digest(c2) == g["c2_sha256"]
    assert digest(c3) == g["c3_sha256"]


def test_registered_reductions(rt):
    x = torch.randn(64, 128)
    xd = x.cuda()
    s_sum = rt.register_reduce("reduce_sum|axes=[1]|keep=1", "sum")
    s_mean = rt.register_reduce("reduce_mean|axes=[1]|keep=0", "mean")
    assert s_sum >= 20 and s_mean >= 20 and s_sum != s_mean
    y = torch.empty(64, 1, device="cuda")
    z = torch.empty(64, device="cuda")
    rt.submit_reduce(s_sum, xd, y, [1], True)
    rt.submit_reduce(s_mean, xd, z, [1], False)
    rt.flush(sync=True)
    assert torch.allclose(y.cpu(), x.sum(1, keepdim=True), rtol=1e-5, atol=1e-4)
    assert torch.allclose(z.cpu(), x.mean(1), rtol=1e-5, atol=1e-5)
    w = torch.randn(8, 16, 32)
    s2 = rt.register_reduce("reduce_sum|axes=[0,1]|keep=0", "sum")
    o = torch.empty(32, device="cuda")
    rt.submit_reduce(s2, w.cuda(), o, [0, 1], False)
    rt.flush(sync=True)
    assert torch.allclose(o.cpu(), w.sum((0, 1)), rtol=1e-5, atol=1e-4)


def test_register_elementwise_exact_expressions(rt):
    a = torch.randn(3000)
    b = torch.randn(3000)
    s_add = rt.register_elementwise("k_add", "(A + B)", 2)
    s_exp = rt.register_elementwise("k_exp", "expf(A)", 1)
    assert rt.register_elementwise("k_add", "(A + B)", 2) == s_add
    o1 = torch.empty(3000, device="cuda")
    o2 = torch.empty(3000, device="cuda")
    rt.submit_binary(s_add, a.cuda(), b.cuda(), o1)
    rt.submit_unary(s_exp, a.cuda(), o2)
    rt.flush(sync=True)
    assert same_bits(o1.cpu(), a + b)
    assert torch.allclose(o2.cpu(), torch.exp(a), rtol=3e-7, atol=0)


def test_task_broadcast_middle_dim(rt):
    # broadcast in a middle dim through the Task path (the reference decode drops it)
    a = torch.randn(2, 3, 4)
    b = torch.randn(2, 1, 4)
    o = torch.empty(2, 3, 4, device="cuda")
    rt.submit_binary(0, a.cuda(), b.cuda(), o)
    rt.flush(sync=True)
    assert same_bits(o.cpu(), a + b)


class TensorRef(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
                ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8)]


class Task(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int), ("flags", ctypes.c_int), ("ndim", ctypes.c_int), ("numel", ctypes.c_int64),
                ("rrank", ctypes.c_int), ("r_axes", ctypes.c_int * 8), ("r_keepdim", ctypes.c_int),
                ("in0", TensorRef), ("in1", TensorRef), ("out0", TensorRef)]


class WorkQueue(ctypes.Structure):
    _fields_ = [("tasks", ctypes.c_void_p), ("capacity", ctypes.c_int), ("head", ctypes.c_void_p),
                ("tail", ctypes.c_void_p), ("quit", ctypes.c_void_p), ("sync", ctypes.c_void_p)]


def test_reference_task_ring_worker_c_abi(rt):
    """launch_persistent_worker over a reference WorkQueue (test/dual_slot_switch.cpp)."""
    assert ctypes.sizeof(Task) == 496
    lib = ctypes.CDLL(LIB_PATH)
    stream = torch.cuda.Stream()
    s = ctypes.c_void_p(stream.cuda_stream)
    n, cap, ntask = 1 << 12, 512, 96
    A = (0.3 * torch.arange(n, dtype=torch.float32)).cuda()
    B = (2.0 + (torch.arange(n) % 9).float()).cuda()
    outs = [torch.zeros(n, device="cuda") for _ in range(3)]
    ring = torch.zeros(cap * 496, dtype=torch.uint8, device="cuda")
    ctl = torch.zeros(3, dtype=torch.int32, device="cuda")  # head, tail, quit
    sync = torch.zeros(64, dtype=torch.uint8).pin_memory()
    q = WorkQueue(ring.data_ptr(), cap, ctl.data_ptr(), ctl.data_ptr() + 4, ctl.data_ptr() + 8, sync.data_ptr())

    def ref(t):
        r = TensorRef(t.data_ptr(), 0, 1)
        r.sizes[0] = n
        r.strides[0] = 1
        return r

    def tasks_bytes(out, start):
        buf = bytearray()
        for _ in range(ntask):
            t = Task(op=0, ndim=1, numel=n, in0=ref(A), in1=ref(B), out0=ref(out))
            buf += bytes(t)
        return buf

    assert lib.gpuos_ring_set_idle_limit_ms(5000, s) == 0
    mul_addr = rt.builtin_op_address(1)
    lib.gpu_set_alias_async.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    proc = ctypes.c_ulonglong(0)
    lib.gpu_get_processed_count_async(ctypes.byref(proc), s)
    stream.synchronize()
    base = proc.value
    # The ring is filled and tail/quit are published with copies from pinned host memory on
    # a second stream: copies need no kernel, and a kernel that is not loaded yet could wait
    # for the running ring worker under lazy module loading.
    side = torch.cuda.Stream()
    word = torch.zeros(1, dtype=torch.int32).pin_memory()

    def publish(index, value):
        word[0] = value
        with torch.cuda.stream(side):
            ctl[index:index + 1].copy_(word, non_blocking=True)
        side.synchronize()

    try:
        assert lib.launch_persistent_worker(q, 8, 128, s) == 0
        tail = 0
        side_s = ctypes.c_void_p(side.cuda_stream)
        for phase, out in enumerate(outs):
            # the ring worker resolves Tasks through the reference C ABI's table
            # (test/dual_slot_switch.cpp:151, 158); the copy runs beside the running worker
            if phase == 1:
                assert lib.gpu_set_alias_async(0, 1, side_s) == 0
                side.synchronize()
            if phase == 2:
                assert lib.gpu_set_alias_async(0, 0, side_s) == 0
                side.synchronize()
            host = torch.frombuffer(bytearray(tasks_bytes(out, tail)), dtype=torch.uint8).pin_memory()
            with torch.cuda.stream(side):
                ring[(tail % cap) * 496:(tail % cap) * 496 + ntask * 496].copy_(host, non_blocking=True)
            side.synchronize()
            tail += ntask
            publish(1, tail)
            deadline = 0
            while True:
                pv = int(torch.frombuffer(bytearray(bytes(sync[:8])), dtype=torch.int64)[0])
                if pv - base >= tail or deadline > 20000:
                    break
                time.sleep(0.0005)
                deadline += 1
            if pv - base < tail:
                dbg = torch.cuda.Stream()
                pc = ctypes.c_ulonglong(0)
                lib.gpu_get_processed_count_async(ctypes.byref(pc), ctypes.c_void_p(dbg.cuda_stream))
                dbg.synchronize()
                raise AssertionError(f"phase {phase}: sync.processed={pv} device processed={pc.value} "
                                     f"ring_stream_done={stream.query()}")
    finally:
        publish(2, 1)  # quit
        stream.synchronize()
        lib.gpu_set_alias_async(0, 0, s)
        stream.synchronize()
    assert mul_addr != 0
    Ac, Bc = A.cpu(), B.cpu()
    assert same_bits(outs[0].cpu(), Ac + Bc)
    assert same_bits(outs[1].cpu(), Ac * Bc)
    assert same_bits(outs[2].cpu(), Ac + Bc)
