"""Top-k on the persistent worker (the batched replacement of the torch::topk call behind
submit_topk, pytorch_ext/gpuos_ext.cpp:1050-1071): rows staged like reduction row groups,
k selection rounds per row.  Values must equal PyTorch CPU topk bit for bit and, for
distinct values, so must the indices; NaN counts as the largest value."""
import pytest
import torch

from oracle.reference_semantics import same_bits

pytestmark = pytest.mark.gpu


def run(rt, x, k, largest):
    v = torch.empty(x.shape[:-1] + (k,), dtype=x.dtype, device="cuda")
    i = torch.empty(x.shape[:-1] + (k,), dtype=torch.int64, device="cuda")
    rt.submit_topk_rows(x.cuda(), v, i, k, largest)
    rt.flush(sync=True)
    return v.cpu(), i.cpu()


def distinct(rows, n, dtype, g):
    # integers are exact in every dtype up to 256 (bf16); wider rows use float32 halves
    if dtype == torch.float32:
        vals = torch.stack([torch.randperm(n, generator=g) for _ in range(rows)]).float() * 0.5 - n / 4
    else:
        assert n <= 256
        vals = torch.stack([torch.randperm(n, generator=g) for _ in range(rows)]).float() - 128
    return vals.to(dtype)


@pytest.mark.parametrize("dtype,rows,n", [
    (torch.float32, 1, 1), (torch.float32, 3, 7), (torch.float32, 64, 1000), (torch.float32, 5, 8192),
    (torch.float32, 2, 20000),        # a row longer than a stage: read from global memory
    (torch.float16, 100, 256), (torch.bfloat16, 33, 200)])
@pytest.mark.parametrize("largest", [True, False])
def test_topk_rows_match_torch(rt, dtype, rows, n, largest):
    g = torch.Generator().manual_seed(rows * 7919 + n)
    x = distinct(rows, n, dtype, g)
    for k in sorted({1, min(n, 5), min(n, 32)}):
        v, i = run(rt, x, k, largest)
        rv, ri = torch.topk(x, k, dim=-1, largest=largest, sorted=True)
        assert same_bits(v, rv), (k, largest)
        assert torch.equal(i, ri), (k, largest)


def test_topk_large_k_and_leading_dims(rt):
    g = torch.Generator().manual_seed(5)
    x = distinct(24, 600, torch.float32, g).view(2, 3, 4, 600)
    v, i = run(rt, x, 256, True)
    rv, ri = torch.topk(x, 256)
    assert same_bits(v, rv) and torch.equal(i, ri)


def test_topk_ties_and_nan(rt):
    g = torch.Generator().manual_seed(6)
    x = torch.randint(0, 5, (16, 300), generator=g).float()      # many equal values
    v, i = run(rt, x, 20, True)
    rv, _ = torch.topk(x, 20)
    assert torch.equal(v, rv)
    assert torch.equal(torch.gather(x, 1, i), v)                  # indices point at the values
    assert all(len(set(r.tolist())) == 20 for r in i)             # no position taken twice
    # equal values: the lower position first
    for r in range(16):
        for q in range(19):
            if v[r, q] == v[r, q + 1]:
                assert i[r, q] < i[r, q + 1]
    y = torch.randn(4, 50, generator=g)
    y[0, 3] = float("nan")
    y[2, 10] = float("nan")
    y[2, 40] = float("nan")
    v, i = run(rt, y, 6, True)
    rv, ri = torch.topk(y, 6)
    assert torch.equal(torch.isnan(v), torch.isnan(rv))
    assert torch.equal(v[~torch.isnan(v)], rv[~torch.isnan(rv)])
    v, i = run(rt, y, 6, False)                                   # smallest: NaN never chosen
    rv, _ = torch.topk(y, 6, largest=False)
    assert same_bits(v, rv) and not torch.isnan(v).any()


def test_topk_rejects_bad_requests(rt):
    x = torch.randn(4, 300, device="cuda")
    v = torch.empty(4, 300, device="cuda")
    i = torch.empty(4, 300, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError, match="k must be"):
        rt.submit_topk_rows(x, v, i, 300, True)                  # above 256
    with pytest.raises(ValueError, match="int64"):
        rt.submit_topk_rows(x, v[:, :5].contiguous(), i[:, :5].int().contiguous(), 5, True)
    with pytest.raises(ValueError, match="contiguous"):
        rt.submit_topk_rows(x.t(), v[:, :5].contiguous(), i[:, :5].contiguous(), 5, True)


@pytest.mark.parametrize("native", [True, False], ids=["native", "python"])
def test_scheduler_routes_topk(rt, native):
    rt.shutdown()
    from gpuos_b200.scheduler import scheduler_context
    g = torch.Generator().manual_seed(7)
    x = distinct(32, 500, torch.float32, g)
    xd = x.cuda()
    try:
        with torch.no_grad(), scheduler_context(size_threshold=1 << 16, native=native) as s:
            assert s.native is native
            before = s.stats["scheduled"]
            v, i = torch.topk(xd, 10)
            v2, i2 = torch.topk(xd * 2, 7, largest=False)
            s.flush(sync=True)
            assert s.stats["scheduled"] >= before + 3   # two top-k and the multiply
    finally:
        rt.init(capacity=8192, threads_per_block=256)
    rv, ri = torch.topk(x, 10)
    assert same_bits(v.cpu(), rv) and torch.equal(i.cpu(), ri)
    rv2, ri2 = torch.topk(x * 2, 7, largest=False)
    assert same_bits(v2.cpu(), rv2) and torch.equal(i2.cpu(), ri2)
