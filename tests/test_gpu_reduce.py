"""Batched last-dim and general reductions on the GPU (config 4 shapes) against PyTorch
CPU eager with fp32 accumulation: error <= 1e-5 * sum|x| (fp32 output) or
1e-2 * max(|ref|, sum|x|) (bf16 output), sum|x| taken over the reduced elements (divided
by the reduced count for mean)."""
import math

import pytest
import torch

from oracle.reference_semantics import reduce_torch

pytestmark = pytest.mark.gpu


def check(rt, x_cpu, axes, keepdim, mean, x_dev=None):
    x_dev = x_cpu.cuda() if x_dev is None else x_dev
    ax = sorted(a % x_cpu.dim() for a in axes) if axes else list(range(x_cpu.dim()))
    shape = list(x_cpu.shape)
    out_shape = [1 if i in ax else s for i, s in enumerate(shape)] if keepdim else \
        [s for i, s in enumerate(shape) if i not in ax]
    out = torch.empty(out_shape, device="cuda", dtype=x_cpu.dtype)
    rt.submit_reduction(rt.RED_MEAN if mean else rt.RED_SUM, x_dev, out, axes, keepdim)
    rt.flush(sync=True)
    ref = reduce_torch(x_cpu, ax, keepdim, mean)
    red = math.prod(shape[a] for a in ax) if ax else 1
    scale = x_cpu.float().abs().sum(dim=ax, keepdim=keepdim) / (red if mean else 1)
    got = out.cpu().float()
    if x_cpu.dtype == torch.float32:
        bound = 1e-5 * scale + 1e-30
    else:
        bound = 1e-2 * torch.maximum(ref.float().abs(), scale) + 1e-30
    err = (got - ref.float()).abs()
    assert (err <= bound).all(), float((err / bound).max())


def test_config4_sample(rt):
    g = torch.Generator().manual_seed(1234 + 4)
    for k in range(96):
        R = int(math.exp(torch.rand(1, generator=g).item() * math.log(1024)))
        C = int(math.exp(math.log(32) + torch.rand(1, generator=g).item() * (math.log(4096) - math.log(32))))
        dt = torch.float32 if k % 2 == 0 else torch.bfloat16
        keep = bool(torch.randint(0, 2, (1,), generator=g))
        mean = bool(torch.randint(0, 2, (1,), generator=g))
        if (k // 2) % 2 == 0:
            buf = torch.randn(R, 2 * C, generator=g).to(dt)
            x = buf[:, ::2]
            xd = buf.cuda()[:, ::2]
        else:
            x = torch.randn(R, C, generator=g).to(dt)
            xd = x.cuda()
        check(rt, x, [-1], keep, mean, xd)


def test_reduce_demo_cases(rt):
    # examples/pytorch_reduce_demo.py:29-52
    x = torch.randn(64, 128)
    check(rt, x, [-1], True, False)
    check(rt, x, [-1], False, True)
    xT = x.t().contiguous().t()
    check(rt, xT, [-1], False, False, xT.cuda().t().contiguous().t())
    w = torch.randn(8, 16, 32)
    check(rt, w, [0, 1], False, False)


def test_long_rows_and_edge_shapes(rt):
    check(rt, torch.randn(3, 50_000), [-1], False, False)   # row longer than a stage
    check(rt, torch.randn(1, 1), [-1], True, True)
    check(rt, torch.randn(4, 0), [-1], False, False)        # empty reduction -> 0
    check(rt, torch.randn(2, 3, 4), [1], True, True)
    check(rt, torch.randn(5, 7), [], False, False)          # empty dim list: full reduction
