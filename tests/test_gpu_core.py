"""Persistent runtime on the GPU: the batched add/mul path (config 1 at full size), the
reference's known answers, ordering of dependent requests, stream dependencies and
completion accounting.  Parity oracle: PyTorch CPU eager, bit-exact."""
import json
import os

import numpy as np
import pytest
import torch

from oracle.reference_semantics import same_bits

pytestmark = pytest.mark.gpu
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_known_answers.json")))


def test_config1_full_size_bit_exact(rt):
    # 4096 independent fp32 requests of 4096 elements, U(-1,1), op 50/50 add/mul
    g = torch.Generator().manual_seed(1234 + 1)
    n_req, n = 4096, 4096
    A = (torch.rand(n_req, n, generator=g) * 2 - 1)
    B = (torch.rand(n_req, n, generator=g) * 2 - 1)
    ops = torch.randint(0, 2, (n_req,), generator=g)
    a, b = A.cuda(), B.cuda()
    out = torch.empty_like(a)
    for i in range(n_req):
        (rt.submit_add if ops[i] == 0 else rt.submit_mul)(a[i], b[i], out[i])
    rt.flush(sync=True)
    ref = torch.where(ops[:, None] == 0, A + B, A * B)
    assert same_bits(out.cpu(), ref)


def test_known_answer_test_py_in_order(rt):
    # test/test.py: add, mul, sub, div into the same c in one flush -> c = a / b
    a = torch.arange(16, device="cuda", dtype=torch.float32)
    b = 2 * torch.ones_like(a)
    c = torch.empty_like(a)
    rt.submit_add(a, b, c)
    rt.submit_mul(a, b, c)
    rt.submit_sub(a, b, c)
    rt.submit_div(a, b, c)
    rt.flush(sync=True)
    assert c.cpu().tolist() == GOLD["test_py"]["c"]
    assert c[:4].tolist() == [0.0, 0.5, 1.0, 1.5]


def test_known_answer_full_sync(rt):
    g = GOLD["full_sync"]
    rng = np.random.default_rng(g["seed"])
    a = torch.from_numpy(rng.standard_normal(g["n"]).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal(g["n"]).astype(np.float32)).cuda()
    c = torch.empty_like(a)
    before = rt.sync_poll_processed()
    rt.submit_add(a, b, c)
    rt.flush(sync=False)
    rt.sync_wait(before + 1, 5000)
    assert rt.sync_poll_processed() >= before + 1
    rt.submit_mul(a, b, c)
    rt.flush(sync=True)
    for _ in range(5):
        rt.submit_add(a, b, c)
    rt.flush(sync=True)
    assert same_bits(c.cpu(), (a.cpu() + b.cpu()))
    st = rt.peek_queue()
    assert st["sync_enabled"] and st["processed"] >= before + 7


def test_dependent_chain_within_one_flush(rt):
    # each request reads the previous output: RAW hazards inside one flush
    x = torch.randn(5000, device="cuda")
    y = torch.randn(5000, device="cuda")
    bufs = [torch.empty_like(x) for _ in range(8)]
    rt.submit_add(x, y, bufs[0])
    for k in range(1, 8):
        rt.submit_mul(bufs[k - 1], y, bufs[k])
    rt.flush(sync=True)
    r = x.cpu() + y.cpu()
    for _ in range(7):
        r = r * y.cpu()
    assert same_bits(bufs[7].cpu(), r)


def test_dependent_across_async_flushes(rt):
    x = torch.randn(70_000, device="cuda")
    y = torch.randn(70_000, device="cuda")
    t = torch.empty_like(x)
    u = torch.empty_like(x)
    rt.submit_add(x, y, t)
    rt.flush(sync=False)
    rt.submit_mul(t, y, u)  # reads the output of the previous (possibly running) flush
    rt.flush(sync=True)
    assert same_bits(u.cpu(), (x.cpu() + y.cpu()) * y.cpu())


def test_inputs_from_pending_torch_work(rt):
    # inputs produced by torch kernels still queued on the current stream
    big = torch.randn(64 << 20, device="cuda")
    a = big.mul(2.0).narrow(0, 0, 4096).clone()
    b = torch.full((4096,), 3.0, device="cuda")
    out = torch.empty_like(a)
    rt.submit_add(a, b, out)
    rt.flush(sync=True)
    assert same_bits(out.cpu(), a.cpu() + 3.0)


def test_many_small_flushes_and_tickets(rt):
    a = torch.randn(256, device="cuda")
    outs = [torch.empty_like(a) for _ in range(300)]
    seqs = []
    for k, o in enumerate(outs):
        rt.submit_mul(a, a, o) if k % 2 else rt.submit_add(a, a, o)
        seqs.append(rt.flush(sync=False))
    assert seqs == sorted(seqs) and len(set(seqs)) == len(seqs)
    rt.wait(seqs[-1])
    assert rt.completed() >= seqs[-1]
    t0, t1 = rt.flush_times(seqs[-1])
    assert t1 >= t0 > 0
    ac = a.cpu()
    for k, o in enumerate(outs):
        assert same_bits(o.cpu(), ac * ac if k % 2 else ac + ac)


def test_quiesce_and_relaunch(rt):
    a = torch.randn(1000, device="cuda")
    o = torch.empty_like(a)
    rt.quiesce()
    assert not rt.worker_alive()
    n0 = rt.launches()
    rt.submit_add(a, a, o)
    rt.flush(sync=True)
    assert rt.launches() == n0 + 1
    assert same_bits(o.cpu(), a.cpu() * 2)


def test_drain_mode_each_flush_launches(rt):
    # drain mode: the worker exits once the ring is drained, the next flush relaunches it
    import time
    a = torch.randn(3000, device="cuda")
    o = torch.empty_like(a)
    rt.set_idle_quiesce_ms(0)
    try:
        rt.quiesce()
        n0 = rt.launches()
        for _ in range(3):
            rt.submit_mul(a, a, o)
            rt.flush(sync=True)
            t0 = time.time()
            while rt.worker_alive() and time.time() - t0 < 5:
                time.sleep(0.001)
            assert not rt.worker_alive()
        assert rt.launches() == n0 + 3
        assert same_bits(o.cpu(), a.cpu() * a.cpu())
    finally:
        rt.set_idle_quiesce_ms(200)


def test_errors_are_exceptions(rt):
    a = torch.randn(4, device="cuda")
    with pytest.raises(ValueError):
        rt.submit_add(a, torch.randn(5, device="cuda"), torch.empty(5, device="cuda"))
    with pytest.raises(ValueError):
        rt.submit_add(a.double(), a.double(), a.double())
    with pytest.raises(RuntimeError, match="CUDA"):
        rt.submit_add(a.cpu(), a.cpu(), a.cpu())


def test_inputs_from_kernels_queued_behind_a_full_worker(rt):
    # At 448 compute threads one worker CTA holds every register of its SM, so a PyTorch kernel
    # queued after the worker started cannot run before the worker stops.  A flush whose
    # inputs come from such a kernel must stop the worker itself, and an idle worker must stop
    # even while requests wait unflushed, or the caller's stream never drains.
    import time as _t

    def drained(limit_s=5.0):
        t0 = _t.monotonic()
        while not torch.cuda.current_stream().query():
            if _t.monotonic() - t0 > limit_s:
                return False
            _t.sleep(0.001)
        return True

    rt.shutdown()
    try:
        rt.init(capacity=8192, threads_per_block=448)
        x = torch.randn(1 << 16, device="cuda")  # queued behind the resident worker
        y = torch.empty_like(x)
        t0 = _t.monotonic()
        rt.submit_add(x, x, y)
        rt.flush(sync=True)
        assert _t.monotonic() - t0 < 5.0
        assert drained()
        assert torch.equal(y.cpu(), x.cpu() + x.cpu())
        z = torch.randn(1 << 16, device="cuda")
        rt.submit_mul(z, z, y)  # pending, not flushed: the idle worker still stops
        assert drained()
        rt.flush(sync=True)
        assert torch.equal(y.cpu(), z.cpu() * z.cpu())
    finally:
        rt.shutdown()
        rt.init(capacity=8192, threads_per_block=256)


def test_submit_ew_new_allocates_the_output(rt):
    """submit_ew_new returns a new contiguous output like `a` holding op(a, b): a tensor or a
    number as b, the two operator parameters, a non-contiguous a (the output is contiguous)."""
    g = torch.Generator().manual_seed(21)
    x = torch.randn(33, 257, generator=g)
    y = torch.randn(33, 257, generator=g)
    xd, yd = x.cuda(), y.cuda()
    o1 = rt.submit_ew_new(rt.EW_MUL, xd, yd)
    o2 = rt.submit_ew_new(rt.EW_ADD, xd, 0.5)
    o3 = rt.submit_ew_new(rt.EW_LEAKY_RELU, xd, None, 0.2)
    o4 = rt.submit_ew_new(rt.EW_CLAMP, xd.t(), None, -0.5, 0.25)
    rt.flush(sync=True)
    assert o4.is_contiguous() and o4.shape == (257, 33) and o1.dtype == torch.float32
    assert same_bits(o1.cpu(), x * y)
    assert same_bits(o2.cpu(), x + 0.5)
    assert same_bits(o3.cpu(), torch.nn.functional.leaky_relu(x, 0.2))
    assert same_bits(o4.cpu(), torch.clamp(x.t(), -0.5, 0.25))
