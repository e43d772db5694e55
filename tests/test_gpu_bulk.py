"""submit_many: many element-wise requests in one call (a bulk submitter beside the
reference's one-call-per-op submit_*, pytorch_ext/gpuos_ext.cpp:638-672).  Results must equal
the per-op submissions bit for bit, and a call with an invalid request submits nothing."""
import pytest
import torch

from oracle.reference_semantics import same_bits

pytestmark = pytest.mark.gpu


def test_submit_many_matches_per_op_submits(rt):
    g = torch.Generator().manual_seed(11)
    R, N = 300, 4096
    a = (torch.rand(R, N, generator=g) * 2 - 1).cuda()
    b = (torch.rand(R, N, generator=g) * 2 - 1).cuda()
    ops = torch.randint(0, 6, (R,), generator=g).tolist()  # add, mul, sub, div, maximum, minimum
    bulk, single = torch.empty_like(a), torch.empty_like(a)
    rt.submit_many(ops, list(a.unbind(0)), list(b.unbind(0)), list(bulk.unbind(0)))
    rt.flush(sync=True)
    for i, op in enumerate(ops):
        rt.submit_elementwise(op, a[i], b[i], single[i])
    rt.flush(sync=True)
    assert same_bits(bulk.cpu(), single.cpu())
    # one op code for every request, and unary requests without b
    out = torch.empty_like(a)
    rt.submit_many(rt.EW_MUL, list(a.unbind(0)), list(b.unbind(0)), list(out.unbind(0)))
    rt.flush(sync=True)
    assert same_bits(out.cpu(), a.cpu() * b.cpu())
    rt.submit_many(rt.EW_RELU, list(a.unbind(0)), None, list(out.unbind(0)))
    rt.flush(sync=True)
    assert same_bits(out.cpu(), torch.relu(a.cpu()))


def test_submit_many_dependencies_and_errors(rt):
    x = torch.randn(8, 1000, device="cuda")
    y = torch.empty_like(x)
    rows_x, rows_y = list(x.unbind(0)), list(y.unbind(0))
    # the second half reads what the first half writes, in the same call
    rt.submit_many(rt.EW_ADD, rows_x, rows_x, rows_y)
    rt.submit_many(rt.EW_MUL, rows_y, rows_y, rows_y)
    rt.flush(sync=True)
    assert same_bits(y.cpu(), (x.cpu() + x.cpu()) * (x.cpu() + x.cpu()))
    before = y.clone()
    with pytest.raises(ValueError, match="same length"):
        rt.submit_many(rt.EW_ADD, rows_x, rows_x[:3], rows_y)
    with pytest.raises(ValueError):  # a binary op without b: nothing is submitted
        rt.submit_many(rt.EW_ADD, rows_x, None, rows_y)
    with pytest.raises(TypeError):
        rt.submit_many(rt.EW_ADD, rows_x, rows_x[:7] + [3.0], rows_y)
    rt.flush(sync=True)
    assert torch.equal(y, before)
    rt.submit_many(rt.EW_ADD, [], [], [])  # empty call: nothing to do
