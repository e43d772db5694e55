"""Host-side logic of scheduler_context that needs no GPU: the exact float literals and nested
operator expressions of fused chains, the parametric ops' (code, p0, p1), and the per-op
counters.  Reference: pytorch_ext/scheduler.py:145-160, 192-290 (the expressions and parameters
the reference generated for the same ops)."""
import struct

import torch

from gpuos_b200 import gpuos_ext as E
from gpuos_b200 import scheduler as S


def _f32(v):
    return struct.unpack("f", struct.pack("f", v))[0]


def test_float_literals_are_exact():
    for v in (0.1, -0.5, 1e-40, 3.0e38, 0.0, -0.0, 2):
        lit = S._f32_literal(v)
        assert lit.endswith("f")
        assert float.fromhex(lit[:-1]) == _f32(float(v))
    assert S._f32_literal(float("inf")) is None
    assert S._f32_literal(float("nan")) is None


def test_chain_expressions_nest_in_order():
    a = torch.empty(4)
    out0, out1, out2 = torch.empty(4), torch.empty(4), torch.empty(4)
    c = S._Chain(a, None, f"gpuos::ew_apply<{E.EW_ABS}>(A, 0.f, 0x0.0p+0f, 0x0.0p+0f)", (E.EW_ABS, None, 0.0, 0.0),
                 out0)
    c.extend(E.EW_MUL, S._f32_literal(0.5), "0.f", "0.f", out1)
    c.extend(E.EW_LEAKY_RELU, "0.f", S._f32_literal(0.01), "0.f", out2)
    assert c.out is out2 and c.arity == 1 and len(c.steps) == 3
    last = c.steps[-1][0]
    assert last.startswith(f"gpuos::ew_apply<{E.EW_LEAKY_RELU}>(gpuos::ew_apply<{E.EW_MUL}>(gpuos::ew_apply<{E.EW_ABS}>(A")
    # every prefix is the expression of that step's own result
    assert c.steps[1][0] in last and c.steps[0][0] in c.steps[1][0]
    assert c.steps[0][2]() is out0 and c.steps[1][2]() is out1


def _mode():
    return S._GPUOSSchedulerMode(size_threshold=1 << 16, auto_flush_ms=None, pending=set())


def test_parametric_codes_follow_pytorch_defaults():
    m = _mode()
    x = torch.empty(3)
    assert m._parametric_code("aten::gelu", (x,), {}) == (E.EW_GELU, 0.0, 0.0)
    assert m._parametric_code("aten::gelu", (x,), {"approximate": "tanh"})[0] == E.EW_GELU_TANH
    assert m._parametric_code("aten::leaky_relu", (x,), {}) == (E.EW_LEAKY_RELU, 0.01, 0.0)
    assert m._parametric_code("aten::leaky_relu", (x, 0.2), {}) == (E.EW_LEAKY_RELU, 0.2, 0.0)
    assert m._parametric_code("aten::hardtanh", (x,), {}) == (E.EW_CLAMP, -1.0, 1.0)
    assert m._parametric_code("aten::elu", (x, 1.5), {}) == (E.EW_ELU, 1.5, 0.0)
    assert m._parametric_code("aten::elu", (x, 1.0, 2.0), {}) is None          # scale != 1: PyTorch
    assert m._parametric_code("aten::softplus", (x,), {}) == (E.EW_SOFTPLUS, 1.0, 20.0)
    assert m._parametric_code("aten::clamp", (x, -0.5, 0.5), {}) == (E.EW_CLAMP, -0.5, 0.5)
    assert m._parametric_code("aten::clamp", (x,), {"min": 0.25}) == (E.EW_CLAMP_MIN, 0.25, 0.0)
    assert m._parametric_code("aten::clamp", (x, None, 0.75), {}) == (E.EW_CLAMP_MAX, 0.75, 0.0)
    assert m._parametric_code("aten::clamp", (x,), {}) is None
    assert m._parametric_code("aten::clamp", (x, torch.zeros(3)), {}) is None   # tensor bound: PyTorch
    m.close()


def test_cpu_tensors_fall_back_and_are_counted():
    """Inside the mode, an op on CPU tensors is not scheduled: PyTorch runs it and the per-op
    fallback counter records it (the runtime is never called)."""
    m = _mode()
    x, y = torch.ones(5), torch.full((5,), 2.0)
    with torch.no_grad(), m:
        z = x + y
        w = torch.relu(z)
    assert torch.equal(w, torch.full((5,), 3.0))
    assert m.fallback_ops == {"aten::add.Tensor": 1, "aten::relu": 1}
    assert m.scheduled == 0
    m.close()


def test_auto_flusher_runs_and_stops(monkeypatch):
    """The periodic asynchronous flush shared by both intercepts (scheduler.py:40-51): it calls
    flush(sync=False) every period and stops within one period of close()."""
    import time
    calls = []
    monkeypatch.setattr(S.gpuos_ext, "flush", lambda sync=False: calls.append(sync))
    f = S._AutoFlusher(5.0)
    time.sleep(0.08)
    t0 = time.perf_counter()
    f.close()
    assert time.perf_counter() - t0 < 0.5
    n = len(calls)
    assert n >= 3 and not any(calls)
    time.sleep(0.03)
    assert len(calls) == n
    assert S._AutoFlusher(None)._bg is None and S._AutoFlusher(0)._bg is None


def test_python_mode_when_the_intercept_is_unavailable(monkeypatch):
    """If the C++ intercept cannot be enabled, the context warns and routes through the Python
    dispatch mode (runtime calls stubbed: no device is touched)."""
    import pytest
    for name in ("init", "shutdown"):
        monkeypatch.setattr(S.gpuos_ext, name, lambda *a, **k: None)
    monkeypatch.setattr(S.gpuos_ext, "flush", lambda sync=False: 0)

    def taken(_):
        raise RuntimeError("intercept unavailable: the dispatcher key already has a fallback")

    monkeypatch.setattr(S.gpuos_ext, "intercept_enable", taken)
    x = torch.ones(3)
    with pytest.warns(RuntimeWarning, match="Python dispatch mode"):
        with S.scheduler_context(auto_flush_ms=None) as s:
            assert s.native is False
            z = x + x
            st = s.stats
    assert torch.equal(z, torch.full((3,), 2.0))
    assert st["fallback_ops"] == {"aten::add.Tensor": 1}


def test_native_context_lifecycle(monkeypatch):
    """The C++ intercept is on exactly inside the context (also when the body raises), its
    counters are the context's stats, and the runtime calls happen in order (stubbed here)."""
    import pytest
    calls = []
    monkeypatch.setattr(S.gpuos_ext, "init", lambda *a, **k: calls.append("init"))
    monkeypatch.setattr(S.gpuos_ext, "shutdown", lambda *a, **k: calls.append("shutdown"))
    monkeypatch.setattr(S.gpuos_ext, "flush", lambda sync=False: calls.append(("flush", sync)) or 0)
    x = torch.ones(4)
    with S.scheduler_context(auto_flush_ms=None, native=True) as s:
        assert s.native is True and E.intercept_enabled()
        y = torch.relu(x * 2.0)
        st = s.stats
    assert not E.intercept_enabled()
    assert torch.equal(y, torch.full((4,), 2.0))
    assert st["scheduled"] == 0 and st["fallback_ops"] == {"aten::mul.Tensor": 1, "aten::relu": 1}
    assert st["fused_chains"] == 0
    assert calls == ["init", ("flush", True), "shutdown"]
    with pytest.raises(ValueError, match="boom"):
        with S.scheduler_context(auto_flush_ms=None, native=True):
            raise ValueError("boom")
    assert not E.intercept_enabled()
