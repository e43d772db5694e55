"""Fusion in scheduler_context (GPUOS_SCHEDULER_DISABLE_JIT=0, as in the reference): a chain of
fp32 element-wise ops, each applied to the previous op's result, becomes one operator compiled
by NVRTC for sm_100a and linked into the worker; its result lands in the tensor returned for the
chain's last op, and earlier results that are still referenced are written too.
Reference: pytorch_ext/scheduler.py:145-160 (fused nodes), :376-396 (flush_fused)."""
import pytest
import torch
import torch.nn.functional as F

from oracle.reference_semantics import same_bits, ulp_diff

pytestmark = pytest.mark.gpu


@pytest.fixture()
def fused(rt, monkeypatch):
    rt.shutdown()
    monkeypatch.setenv("GPUOS_SCHEDULER_DISABLE_JIT", "0")
    from gpuos_b200.scheduler import scheduler_context
    yield scheduler_context
    rt.init(capacity=8192, threads_per_block=256)


def _inputs(seed, shape=(3, 1000)):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * 2, torch.randn(*shape, generator=g) * 2


def test_four_op_chain_is_one_operator_and_bit_exact(fused):
    a, b = _inputs(11)
    ad, bd = a.cuda(), b.cuda()
    with torch.no_grad(), fused(auto_flush_ms=None) as s:
        out = F.leaky_relu(torch.clamp(torch.abs(ad * bd), 0.1, 0.9), 0.2)
        s.flush(sync=True)
        st = s.stats
    assert st["fused_chains"] == 1 and st["fused_ops"] == 4
    assert st["fallback_ops"] == {}
    assert same_bits(out.cpu(), F.leaky_relu(torch.clamp(torch.abs(a * b), 0.1, 0.9), 0.2))


def test_chain_ending_in_a_transcendental_within_2_ulp(fused):
    a, b = _inputs(12)
    with torch.no_grad(), fused(auto_flush_ms=None) as s:
        ad, bd = a.cuda(), b.cuda()
        out = torch.sigmoid(F.hardswish(torch.relu(ad + bd)))
        s.flush(sync=True)
        st = s.stats
    assert st["fused_chains"] == 1 and st["fused_ops"] == 4
    ref = torch.sigmoid(F.hardswish(torch.relu(a + b)))
    assert int(ulp_diff(out.cpu(), ref).max()) <= 2


def test_chain_with_scalar_operands_and_referenced_intermediates(fused):
    """y and z stay referenced: the fused operator writes w, and y and z are written as well."""
    a, b = _inputs(13)
    with torch.no_grad(), fused(auto_flush_ms=None) as s:
        ad, bd = a.cuda(), b.cuda()
        y = ad * bd
        z = torch.tanh(y * 0.5)
        w = torch.clamp(z + 0.25, -0.5, 0.75)
        s.flush(sync=True)
        st = s.stats
    assert st["fused_chains"] == 1 and st["fused_ops"] == 5
    yr = a * b
    zr = torch.tanh(yr * 0.5)
    assert same_bits(y.cpu(), yr)
    assert int(ulp_diff(z.cpu(), zr).max()) <= 2
    # w is computed from the runtime's own z (tanh within 2 ulp), then exact ops
    assert same_bits(w.cpu(), torch.clamp(z.cpu() + 0.25, -0.5, 0.75))


def test_consumers_see_the_chain_complete(fused):
    """A reduction, an unscheduled op and an in-place write after a chain all see its result."""
    a, b = _inputs(14)
    with torch.no_grad(), fused(auto_flush_ms=None) as s:
        ad, bd = a.cuda(), b.cuda()
        c = torch.relu(torch.exp(ad - bd))
        total = c.sum(-1)            # scheduled reduction of the chain's result
        m = c @ c.t()                # not scheduled
        ad.add_(1.0)                 # in-place write to the chain's input after the chain
        s.flush(sync=True)
    cr = torch.relu(torch.exp(a - b))
    assert int(ulp_diff(c.cpu(), cr).max()) <= 2
    assert torch.allclose(total.cpu(), cr.sum(-1), rtol=1e-5)
    assert torch.allclose(m.cpu(), cr @ cr.t(), rtol=1e-4)
    assert same_bits(ad.cpu(), a + 1.0)


def test_non_fp32_and_broadcast_ops_are_not_fused(fused):
    a, b = _inputs(15)
    with torch.no_grad(), fused(auto_flush_ms=None) as s:
        ah = a.cuda().half()
        r = torch.relu(torch.sigmoid(ah))           # fp16: submitted op by op
        row = b[0].cuda()
        q = torch.relu(a.cuda() + row)              # broadcast root: not a chain root
        s.flush(sync=True)
        st = s.stats
    assert st["fused_chains"] == 0
    assert int((r.cpu().float() - torch.relu(torch.sigmoid(a.half())).float()).abs().max() * 1024) <= 2
    assert same_bits(q.cpu(), torch.relu(a + b[0]))
