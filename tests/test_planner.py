"""Host planner (no GPU): broadcast alignment, dimension coalescing and tiling of requests
into work items, checked by executing the planned items on the CPU and comparing with
PyTorch CPU eager (bit-exact for add/mul/sub/div/max/min)."""
import pytest
import torch

from oracle.reference_semantics import EW, ew_torch, reduce_torch, same_bits
from tests._items import (IF_A_BCAST, IF_A_T, IF_B_BCAST, IF_B_SCALAR, IF_B_T, IF_UNSTAGED, IK_EW_2D, IK_EW_2DT,
                          IK_EW_CONTIG, IK_EW_GENERIC, IK_RED_GENERIC, IK_ROW_REDUCE, Memory, plan_ew,
                          plan_reduce, run_items)


def op_fn(op, a, b, p0, p1):
    return ew_torch(op, a, b, p0, p1).float()


def check_ew(op, a, b, out_dtype, p0=0.0, p1=0.0):
    shape = torch.broadcast_shapes(a.shape, b.shape) if isinstance(b, torch.Tensor) else a.shape
    out = torch.empty(shape, dtype=out_dtype)
    items, lay = plan_ew(op, a, b, out, p0, p1)
    run_items(items, lay, Memory(a, b, out), op_fn)
    ref = ew_torch(op, a.float(), b.float() if isinstance(b, torch.Tensor) else b, p0, p1).to(out_dtype)
    assert same_bits(out, ref), (op, a.shape, out_dtype)
    return items


def test_c1_request_is_one_contiguous_tile():
    a, b = torch.rand(4096) * 2 - 1, torch.rand(4096) * 2 - 1
    items = check_ew(EW["ADD"], a, b, torch.float32)
    assert len(items) == 1 and items[0]["kind"] == IK_EW_CONTIG and items[0]["count"] == 4096


def test_large_request_is_tiled():
    a, b = torch.randn(100_003), torch.randn(100_003)
    items = check_ew(EW["MUL"], a, b, torch.float32)
    assert len(items) == -(-100_003 // 4096)
    assert all(it["kind"] == IK_EW_CONTIG for it in items)
    # 16-bit inputs: 8192 elements per tile
    items = check_ew(EW["MUL"], a.half(), b.half(), torch.float16)
    assert len(items) == -(-100_003 // 8192)


@pytest.mark.parametrize("dt,shift", [(torch.float32, 1), (torch.float32, 3), (torch.float16, 5), (torch.bfloat16, 1)])
def test_misaligned_operand_tiles_fit_a_stage_half(dt, shift):
    # a view that starts off a 16-byte boundary: every tile's 16-byte-aligned span must fit
    # the 16 KB stage half, or the tile would not be staged
    base = torch.randn(30_001 + shift).to(dt)
    a, b = base[shift:], torch.randn(30_001).to(dt)
    items = check_ew(EW["ADD"], a, b, dt)
    es = base.element_size()
    for it in items:
        for addr in (int(it["a"]), int(it["b"])):
            span = ((addr + int(it["count"]) * es + 15) & ~15) - (addr & ~15)
            assert span <= 16384
    assert int(items[0]["count"]) == (16384 - 32) // es


def test_transposed_fp16_with_broadcast_bf16_is_staged_transpose_blocks():
    # C3: a = transpose of [512,64] fp16 viewed [64,512]; b = [512] bf16; out fp32.  A block of
    # all 64 rows x 64 columns of a is one contiguous 8 KiB span (staged by one bulk copy).
    a = torch.randn(512, 64).half().t()
    b = torch.randn(512).bfloat16()
    items = check_ew(EW["ADD"], a, b, torch.float32)
    assert all(it["kind"] == IK_EW_2DT for it in items)
    assert len(items) == 512 // 64
    assert all((int(it["count"]) >> 16) == 64 and (int(it["count"]) & 0xFFFF) == 64 for it in items)
    assert all(int(it["x"]) & 0xFFFFFFFF == 6 for it in items)      # log2 of the column width
    check_ew(EW["MAXIMUM"], a, b, torch.float32)
    check_ew(EW["RELU"], a, None, torch.float32)   # unary through the same blocks


@pytest.mark.parametrize("R,C,dt", [(2, 5000, torch.float16), (17, 333, torch.bfloat16), (256, 40, torch.float16),
                                    (100, 77, torch.float32), (128, 1000, torch.float32), (3, 9, torch.float32)])
def test_staged_transpose_blocks_fit_a_stage_half(R, C, dt):
    a = torch.randn(C, R).to(dt).t()
    items = check_ew(EW["MUL"], a, torch.randn(C).bfloat16(), torch.float32)
    es = a.element_size()
    for it in items:
        assert it["kind"] == IK_EW_2DT
        nr, nc, w = int(it["count"]) >> 16, int(it["count"]) & 0xFFFF, 1 << (int(it["x"]) & 0xFFFFFFFF)
        assert nr == R and 1 <= nc <= w and nr * w <= 4096 and w >= 8
        assert ((w - 1) * R + R) * es + 32 <= 16384
    check_ew(EW["SUB"], a, torch.randn(R, C), torch.float16)    # b read element by element


@pytest.mark.parametrize("R,C", [(1, 300), (15, 17), (16, 256), (17, 257), (40, 1000), (300, 9)])
def test_2d_blocks_cover_ragged_shapes(R, C):
    a = torch.randn(C, R).t()                      # transposed
    b = torch.randn(R, C)                          # contiguous
    check_ew(EW["SUB"], a, b, torch.float32)
    check_ew(EW["SUB"], b, a, torch.float32)       # transposed second operand
    items = check_ew(EW["MUL"], a, a, torch.float32)  # both transposed
    if R > 1:
        assert all(it["flags"] & IF_A_T and it["flags"] & IF_B_T for it in items)
    check_ew(EW["ADD"], b, torch.randn(C), torch.float32)        # row broadcast: row mode
    check_ew(EW["ADD"], b, torch.randn(R, 1), torch.float32)     # column broadcast: row mode
    big = torch.randn(R, 2 * C)
    check_ew(EW["MAXIMUM"], big[:, ::2], b, torch.float16)       # stride-2 rows, 16-bit out


def test_row_mode_long_rows_are_split():
    a = torch.randn(3, 20000)
    items = check_ew(EW["ADD"], a, torch.randn(20000), torch.float32)
    assert all(it["kind"] == IK_EW_2D and not it["flags"] & (IF_A_T | IF_B_T) for it in items)
    assert len(items) == 3 * 3  # 8192-column pieces of each row


def test_transposed_output_is_walked_in_its_own_order():
    out = torch.empty(30, 50).t()                  # [50, 30] view of a column-major buffer
    a, b = torch.randn(50, 30), torch.randn(30)
    items, lay = plan_ew(EW["ADD"], a, b, out)
    run_items(items, lay, Memory(a, b, out), op_fn)
    assert same_bits(out, a + b)
    assert int(lay["so"][1]) == 1                  # columns follow the output's contiguous dim


def test_broadcast_row_and_scalar_operands():
    a = torch.randn(33, 17)
    items = check_ew(EW["SUB"], a, torch.randn(1), torch.float32)  # one-element tensor
    assert items[0]["kind"] == IK_EW_CONTIG and items[0]["flags"] & IF_B_BCAST
    items = check_ew(EW["DIV"], a, 3.0, torch.float32)  # Python scalar
    assert items[0]["flags"] & IF_B_SCALAR
    items = check_ew(EW["MUL"], torch.randn(1), a, torch.float32)
    assert items[0]["flags"] & IF_A_BCAST
    check_ew(EW["ADD"], a, torch.randn(17), torch.float32)  # row broadcast -> generic
    check_ew(EW["ADD"], torch.randn(5, 1, 7), torch.randn(4, 1), torch.float32)  # middle broadcast


def test_coalescing_merges_contiguous_dims():
    a = torch.randn(8, 16, 32)
    items = check_ew(EW["ADD"], a, torch.randn(8, 16, 32), torch.float32)
    assert all(it["kind"] == IK_EW_CONTIG for it in items)
    # a slice with a gap stays strided
    big = torch.randn(8, 40)
    items = check_ew(EW["ADD"], big[:, :32], torch.randn(8, 32), torch.float32)
    assert items[0]["kind"] == IK_EW_2D
    # three dims that do not merge stay on the generic path
    cube = torch.randn(6, 7, 9)
    items = check_ew(EW["ADD"], cube[:, :5, ::2], torch.randn(6, 5, 5), torch.float32)
    assert items[0]["kind"] == IK_EW_GENERIC


@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
def test_unary_params_and_dtypes(dt):
    x = (torch.randn(3001) * 3).to(dt)
    check_ew(EW["LEAKY_RELU"], x, None, dt, 0.01)
    check_ew(EW["CLAMP"], x, None, dt, -0.5, 0.5)
    check_ew(EW["HARDSWISH"], x, None, dt)
    check_ew(EW["RELU"], x, None, torch.float32)


def test_empty_and_invalid_requests():
    items, _ = plan_ew(EW["ADD"], torch.randn(0), torch.randn(0), torch.empty(0))
    assert len(items) == 0
    with pytest.raises(ValueError, match="broadcast"):
        plan_ew(EW["ADD"], torch.randn(3), torch.randn(4), torch.empty(4))
    with pytest.raises(ValueError, match="dtype"):
        plan_ew(EW["ADD"], torch.randn(3).double(), torch.randn(3), torch.empty(3))


def check_reduce(x, axes, keepdim, mean, expect_kind=None):
    shape = list(x.shape)
    ax = sorted(a % x.dim() for a in axes)
    if keepdim:
        out_shape = [1 if i in ax else s for i, s in enumerate(shape)]
    else:
        out_shape = [s for i, s in enumerate(shape) if i not in ax]
    out = torch.empty(out_shape, dtype=x.dtype)
    items, lay = plan_reduce(1 if mean else 0, x, out, list(axes), keepdim)
    run_items(items, lay, Memory(x, out), op_fn)
    ref = reduce_torch(x, ax, keepdim, mean)
    tol = 1e-5 if x.dtype == torch.float32 else 1e-2
    scale = x.float().abs().sum(dim=ax, keepdim=keepdim)
    if mean:
        scale = scale / max(1, int(torch.tensor([shape[a] for a in ax]).prod()))
    assert ((out.float() - ref.float()).abs() <= tol * scale + 1e-6).all()
    if expect_kind is not None:
        assert all(int(it["kind"]) == expect_kind for it in items)
    return items


def test_row_reductions_contiguous_and_stride2():
    # C4 shapes: contiguous rows, and stride-2 views of a [R, 2C] buffer
    check_reduce(torch.randn(37, 1000), [-1], False, False, IK_ROW_REDUCE)
    items = check_reduce(torch.randn(1024, 32), [-1], True, True, IK_ROW_REDUCE)
    assert all(not (it["flags"] & IF_UNSTAGED) for it in items)
    buf = torch.randn(64, 2 * 300)
    check_reduce(buf[:, ::2], [-1], False, True, IK_ROW_REDUCE)
    check_reduce(torch.randn(5, 4096).bfloat16(), [1], False, False, IK_ROW_REDUCE)
    items = check_reduce(torch.randn(3, 20000), [-1], False, False, IK_ROW_REDUCE)
    assert all(it["flags"] & IF_UNSTAGED for it in items)


def test_generic_reductions():
    check_reduce(torch.randn(8, 16, 32), [0, 1], False, False, IK_RED_GENERIC)
    check_reduce(torch.randn(64, 128).t(), [-1], False, True)
    check_reduce(torch.randn(6, 5, 4), [1], True, True, IK_RED_GENERIC)
