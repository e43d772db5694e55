"""The C++ dispatcher intercept of scheduler_context (csrc/intercept.cpp) without a GPU: with no
runtime every op is left to PyTorch, results are PyTorch's own, the counters name ops as the
Python dispatch mode does (an op PyTorch decomposes at the autograd level counts as its parts),
only the entering thread is intercepted, and autograd still works underneath.
Reference: pytorch_ext/scheduler.py:162-373 (the intercept), :399-466 (stats via the mode)."""
import threading

import torch
import torch.nn.functional as F

from gpuos_b200 import gpuos_ext as E


def _run(fn):
    E.intercept_enable(1 << 16)
    try:
        out = fn()
        return out, E.intercept_stats()
    finally:
        E.intercept_disable()


def test_cpu_ops_pass_through_and_are_counted():
    x, y = torch.ones(5), torch.full((5,), 2.0)

    def body():
        with torch.no_grad():
            return torch.relu(x + y)

    w, st = _run(body)
    assert torch.equal(w, torch.full((5,), 3.0))
    assert st["scheduled"] == 0 and st["scheduled_ops"] == {}
    assert st["fallback_ops"] == {"aten::add.Tensor": 1, "aten::relu": 1}
    assert st["fallbacks"] == 2
    assert not E.intercept_enabled()


def test_composite_ops_count_as_their_parts():
    """relu6 and linear decompose at the autograd level: the intercept sees hardtanh, t and mm,
    as a dispatch mode below autograd does."""
    g = torch.Generator().manual_seed(3)
    x, w = torch.randn(4, 6, generator=g), torch.randn(3, 6, generator=g)

    def body():
        with torch.no_grad():
            return F.relu6(x * 4), F.linear(x, w)

    (a, b), st = _run(body)
    assert torch.equal(a, F.relu6(x * 4)) and torch.allclose(b, x @ w.t())
    ops = st["fallback_ops"]
    assert ops.get("aten::hardtanh") == 1 and ops.get("aten::mul.Tensor") == 1
    assert "aten::relu6" not in ops and "aten::linear" not in ops
    assert ops.get("aten::t") == 1 and ops.get("aten::mm") == 1


def test_enable_resets_the_counters():
    x = torch.ones(3)
    _run(lambda: x + x)
    _, st = _run(lambda: x * x)
    assert st["fallback_ops"] == {"aten::mul.Tensor": 1}


def test_only_the_entering_thread_is_intercepted():
    x = torch.ones(3)
    seen = {}

    def other():
        seen["enabled"] = E.intercept_enabled()
        seen["out"] = x - x

    def body():
        t = threading.Thread(target=other)
        t.start()
        t.join()
        return x + x

    out, st = _run(body)
    assert seen["enabled"] is False and torch.equal(seen["out"], torch.zeros(3))
    assert torch.equal(out, torch.full((3,), 2.0))
    assert st["fallback_ops"] == {"aten::add.Tensor": 1}


def test_autograd_runs_underneath():
    """The key sits above autograd; with grad mode on nothing is scheduled and the graph is
    recorded as usual."""
    w = torch.tensor([1.0, -2.0, 3.0], requires_grad=True)

    def body():
        loss = (torch.tanh(w) * 2).sum()
        loss.backward()
        return loss.detach()

    loss, st = _run(body)
    assert torch.allclose(w.grad, 2 * (1 - torch.tanh(w.detach()) ** 2))
    assert torch.allclose(loss, (torch.tanh(w.detach()) * 2).sum())
    assert st["scheduled"] == 0 and st["fallback_ops"].get("aten::tanh") == 1


def test_errors_of_the_op_reach_the_caller():
    a, b = torch.ones(3), torch.ones(4)

    def body():
        try:
            a + b
        except RuntimeError as e:
            return str(e)
        return ""

    msg, st = _run(body)
    assert "size of tensor a (3)" in msg
    assert st["fallback_ops"] == {"aten::add.Tensor": 1}


def test_routes_match_the_python_mode():
    """The C++ intercept routes exactly the ops the Python dispatch mode routes, to the same
    runtime operators (kinds: 1 binary, 2 unary, 3 parametric unary, 4 reduction, 5 top-k)."""
    from gpuos_b200 import scheduler as S
    want = {}
    for name, op in S._BINARY.items():
        want[name] = (1, op)
    for name, op in S._UNARY.items():
        want[name] = (2, op)
    for name in S._PARAMETRIC:
        want[name] = (3, 0)
    for name in S._REDUCE:
        want[name] = (4, E.RED_MEAN if "mean" in name else E.RED_SUM)
    want["aten::topk"] = (5, 0)
    assert E.intercept_routes() == want


def test_models_and_ops_of_every_argument_kind_pass_through():
    """Tensor lists, optional-tensor lists (indexing), tuple returns, in-place writes, views and
    a small convolutional model give PyTorch's own results with the intercept on; so does a
    training step (grad mode on: nothing is scheduled, autograd records as usual)."""
    import torch.nn as nn

    torch.manual_seed(0)
    model = nn.Sequential(nn.Conv2d(3, 8, 3, padding=1), nn.BatchNorm2d(8), nn.ReLU(), nn.Flatten(),
                          nn.Linear(8 * 8 * 8, 16), nn.LayerNorm(16), nn.GELU(), nn.Linear(16, 4)).eval()
    x = torch.randn(2, 3, 8, 8)

    def work():
        with torch.no_grad():
            y = model(x)
            z = x[torch.tensor([0, 1]), :, None, 1:5]
            c = torch.cat([y, y * 2], dim=1)
            s = torch.softmax(c, -1)
            v, i = torch.sort(s, dim=-1)
            a = torch.where(s > 0.1, s, torch.zeros_like(s))
            q = s.clone()
            q.add_(1.0)
            q[0, 0] = 5.0
            u = torch.stack(torch.chunk(c, 2, dim=1))
            m = torch.einsum("ij,kj->ik", y, y)
        return [y, z, c, s, v, i, a, q, u, m]

    ref = work()
    got, st = _run(work)
    assert all(torch.equal(r, g) for r, g in zip(ref, got))
    assert st["scheduled"] == 0 and st["fallback_ops"]["aten::index.Tensor"] == 1

    def train(intercept):
        torch.manual_seed(1)
        lin = nn.Linear(5, 3)
        opt = torch.optim.SGD(lin.parameters(), lr=0.1)
        xb = torch.randn(4, 5)

        def step():
            loss = F.mse_loss(lin(xb), torch.ones(4, 3))
            opt.zero_grad()
            loss.backward()
            opt.step()

        _run(step) if intercept else step()
        return lin.weight.detach().clone(), lin.bias.detach().clone()

    w0, b0 = train(False)
    w1, b1 = train(True)
    assert torch.equal(w0, w1) and torch.equal(b0, b1)


def test_other_dispatch_modes_and_autocast_still_work():
    """A user's TorchDispatchMode (as profilers and tracers use) still sees every op under the
    intercept, and CPU autocast still changes the dtype: calls with those keys are not plain
    dense ones, so they pass through unchanged."""
    from torch.utils._python_dispatch import TorchDispatchMode

    class Count(TorchDispatchMode):
        def __init__(self):
            super().__init__()
            self.names = []

        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            self.names.append(func.name())
            return func(*args, **(kwargs or {}))

    x = torch.randn(8, 8)

    def body():
        with Count() as m:
            y = torch.relu(x) + 1.0
        with torch.autocast("cpu", dtype=torch.bfloat16):
            z = x @ x
        return m.names, y, z

    (names, y, z), st = _run(body)
    assert names == ["aten::relu", "aten::add.Tensor"]
    assert torch.equal(y, torch.relu(x) + 1.0)
    assert z.dtype == torch.bfloat16
    assert st["scheduled"] == 0
