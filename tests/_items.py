"""Test helpers: ctypes access to the device-free planning hooks of libgpuos_b200.so and a
numpy executor of the planned work items (test infrastructure)."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(ROOT, "gpuos_b200", "lib", "libgpuos_b200.so")

ITEM_DT = np.dtype([("kind", "u1"), ("op", "u1"), ("dt_a", "u1"), ("dt_b", "u1"), ("dt_o", "u1"),
                    ("flags", "u1"), ("batch", "<u2"), ("count", "<u4"), ("aux", "<u4"), ("a", "<u8"),
                    ("b", "<u8"), ("o", "<u8"), ("x", "<u8"), ("wait_items", "<u8"),
                    ("batch_items", "<u4"), ("batch_seq", "<u4")])
assert ITEM_DT.itemsize == 64
LAYOUT_DT = np.dtype([("ndim", "<i4"), ("rdim", "<i4"), ("params", "<f4", 4), ("sizes", "<i8", 8),
                      ("sa", "<i8", 8), ("sb", "<i8", 8), ("so", "<i8", 8), ("rsizes", "<i8", 8),
                      ("rsa", "<i8", 8), ("rtotal", "<i8"), ("pad", "<i8"), ("pad2", "<i8")])
assert LAYOUT_DT.itemsize == 432

IK_EW_CONTIG, IK_EW_GENERIC, IK_ROW_REDUCE, IK_RED_GENERIC, IK_TASK, IK_EW_2D = 1, 2, 3, 4, 5, 6
IK_EW_2DT = 8
IF_B_PRESENT, IF_B_SCALAR, IF_A_BCAST, IF_B_BCAST, IF_UNSTAGED, IF_MEAN = 1, 2, 4, 8, 16, 32
IF_A_T, IF_B_T = 64, 128
CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.float64: 4, torch.int32: 3}
TDT = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}
ES = {0: 4, 1: 2, 2: 2}


class Operand(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
                ("sizes", ctypes.c_int64 * 8), ("strides", ctypes.c_int64 * 8)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.gpuos_rt_last_error.restype = ctypes.c_char_p
        P, I = ctypes.c_void_p, ctypes.c_int
        _lib.gpuos_plan_ew.argtypes = [I, P, P, I, ctypes.c_double, P, P, I, P, I, P, P]
        _lib.gpuos_plan_ew.restype = I
        _lib.gpuos_plan_reduce.argtypes = [I, P, P, P, I, I, P, I, P, P]
        _lib.gpuos_plan_reduce.restype = I
    return _lib


def operand(t: torch.Tensor) -> Operand:
    o = Operand()
    o.data = t.data_ptr()
    o.dtype = CODE[t.dtype]
    o.ndim = t.dim()
    for d in range(t.dim()):
        o.sizes[d] = t.shape[d]
        o.strides[d] = t.stride(d)
    return o


def plan_ew(op, a, b, out, p0=0.0, p1=0.0, max_items=1 << 16):
    items = np.zeros(max_items, ITEM_DT)
    lay = np.zeros(512, np.uint8)
    n = ctypes.c_int(0)
    params = (ctypes.c_float * 2)(p0, p1)
    oa, oo = operand(a), operand(out)
    if isinstance(b, torch.Tensor):
        ob = operand(b)
        st = lib().gpuos_plan_ew(op, ctypes.byref(oa), ctypes.byref(ob), 0, ctypes.c_double(0.0), ctypes.byref(oo),
                                 params, 2, items.ctypes.data, max_items, lay.ctypes.data, ctypes.byref(n))
    elif b is None:
        st = lib().gpuos_plan_ew(op, ctypes.byref(oa), None, 0, ctypes.c_double(0.0), ctypes.byref(oo), params, 2,
                                 items.ctypes.data, max_items, lay.ctypes.data, ctypes.byref(n))
    else:
        st = lib().gpuos_plan_ew(op, ctypes.byref(oa), None, 1, ctypes.c_double(float(b)), ctypes.byref(oo), params,
                                 2, items.ctypes.data, max_items, lay.ctypes.data, ctypes.byref(n))
    if st != 0:
        raise ValueError(lib().gpuos_rt_last_error().decode())
    return items[: n.value], lay[:432].view(LAYOUT_DT)[0]


def plan_reduce(op, x, out, axes, keepdim, max_items=1 << 16):
    items = np.zeros(max_items, ITEM_DT)
    lay = np.zeros(512, np.uint8)
    n = ctypes.c_int(0)
    ax = (ctypes.c_int * max(1, len(axes)))(*axes)
    ox, oo = operand(x), operand(out)
    st = lib().gpuos_plan_reduce(op, ctypes.byref(ox), ctypes.byref(oo), ax, len(axes), int(keepdim),
                                 items.ctypes.data, max_items, lay.ctypes.data, ctypes.byref(n))
    if st != 0:
        raise ValueError(lib().gpuos_rt_last_error().decode())
    return items[: n.value], lay[:432].view(LAYOUT_DT)[0]


class Memory:
    """Maps absolute addresses in planned items back to CPU tensors' storage."""

    def __init__(self, *tensors):
        self.bufs = []
        for t in tensors:
            if isinstance(t, torch.Tensor):
                st = t.untyped_storage()
                self.bufs.append((st.data_ptr(), st.nbytes(), st))

    def view(self, addr: int, dtype_code: int, count: int) -> torch.Tensor:
        """A 1-D tensor of `count` elements starting at address addr (strided access uses
        element offsets on top of this base)."""
        for base, nbytes, st in self.bufs:
            if base <= addr < base + max(nbytes, 1):
                off = addr - base
                es = ES[dtype_code]
                assert off % es == 0
                full = torch.empty(0, dtype=TDT[dtype_code]).set_(st, 0, (nbytes // es,), (1,))
                return full[off // es: off // es + count] if count >= 0 else full[off // es:]
        raise AssertionError(f"address {addr:#x} outside every buffer")


def run_items(items, layout, mem: Memory, op_fn):
    """Execute planned items on CPU.  op_fn(op, a_vals, b_vals_or_scalar, p0, p1) -> float32."""
    for it in items:
        kind = int(it["kind"])
        dta, dtb, dto = int(it["dt_a"]), int(it["dt_b"]), int(it["dt_o"])
        if kind in (IK_EW_CONTIG, IK_EW_GENERIC):
            n = int(it["count"])
            if kind == IK_EW_CONTIG:
                a = mem.view(int(it["a"]), dta, 1 if it["flags"] & IF_A_BCAST else n).float()
                if it["flags"] & IF_A_BCAST:
                    a = a.expand(n)
                if it["flags"] & IF_B_SCALAR:
                    b = float(np.uint32(it["b"] & 0xFFFFFFFF).view(np.float32))
                elif it["flags"] & IF_B_PRESENT:
                    b = mem.view(int(it["b"]), dtb, 1 if it["flags"] & IF_B_BCAST else n).float()
                    if it["flags"] & IF_B_BCAST:
                        b = b.expand(n)
                else:
                    b = None
                p0 = float(np.uint32(int(it["x"]) & 0xFFFFFFFF).view(np.float32))
                p1 = float(np.uint32(int(it["x"]) >> 32).view(np.float32))
                r = op_fn(int(it["op"]), a, b, p0, p1)
                mem.view(int(it["o"]), dto, n).copy_(r.to(TDT[dto]))
            else:
                L = layout
                nd = int(L["ndim"])
                idx = torch.arange(int(it["x"]), int(it["x"]) + n, dtype=torch.int64)
                oa = torch.zeros(n, dtype=torch.int64)
                ob = torch.zeros(n, dtype=torch.int64)
                oo = torch.zeros(n, dtype=torch.int64)
                rem = idx.clone()
                for d in range(nd - 1, -1, -1):
                    sz = int(L["sizes"][d])
                    c = rem % sz
                    rem = rem // sz
                    oa += c * int(L["sa"][d])
                    ob += c * int(L["sb"][d])
                    oo += c * int(L["so"][d])
                a = mem.view(int(it["a"]), dta, -1).float()[oa]
                if it["flags"] & IF_B_SCALAR:
                    b = float(np.uint32(it["b"] & 0xFFFFFFFF).view(np.float32))
                elif it["flags"] & IF_B_PRESENT:
                    b = mem.view(int(it["b"]), dtb, -1).float()[ob]
                else:
                    b = None
                r = op_fn(int(it["op"]), a, b, float(L["params"][0]), float(L["params"][1]))
                mem.view(int(it["o"]), dto, -1)[oo] = r.to(TDT[dto])
        elif kind in (IK_EW_2D, IK_EW_2DT):
            # block rows [r0, r0 + nr) x columns [c0, c0 + nc) of the 2-D layout (EW_2DT: every
            # row, the low 32 bits of x hold the log2 of the block's column width)
            L = layout
            r0, c0 = (0 if kind == IK_EW_2DT else int(it["x"]) & 0xFFFFFFFF), int(it["x"]) >> 32
            nr, nc = int(it["count"]) >> 16, int(it["count"]) & 0xFFFF
            rr = (torch.arange(nr, dtype=torch.int64) + r0).unsqueeze(1)
            cc = (torch.arange(nc, dtype=torch.int64) + c0).unsqueeze(0)

            def offs(st):
                return (rr * int(st[0]) + cc * int(st[1])).reshape(-1)
            a = mem.view(int(it["a"]), dta, -1).float()[offs(L["sa"])]
            if it["flags"] & IF_B_SCALAR:
                b = float(np.uint32(it["b"] & 0xFFFFFFFF).view(np.float32))
            elif it["flags"] & IF_B_PRESENT:
                b = mem.view(int(it["b"]), dtb, -1).float()[offs(L["sb"])]
            else:
                b = None
            r = op_fn(int(it["op"]), a, b, float(L["params"][0]), float(L["params"][1]))
            mem.view(int(it["o"]), dto, -1)[offs(L["so"])] = r.to(TDT[dto])
        elif kind == IK_ROW_REDUCE:
            rows, C, rs, es_ = int(it["count"]), int(it["aux"]), int(it["x"]), int(it["b"])
            base = mem.view(int(it["a"]), dta, -1).float()
            r = torch.arange(rows).unsqueeze(1) * rs + torch.arange(C).unsqueeze(0) * es_
            s = base[r].sum(dim=1)
            if it["flags"] & IF_MEAN:
                s = s / C
            mem.view(int(it["o"]), dto, rows).copy_(s.to(TDT[dto]))
        elif kind == IK_RED_GENERIC:
            L = layout
            n = int(it["count"])
            base = mem.view(int(it["a"]), dta, -1).float()
            outv = mem.view(int(it["o"]), dto, -1)
            for k in range(n):
                li = int(it["x"]) + k
                ia = oo = 0
                rem = li
                for d in range(int(L["ndim"]) - 1, -1, -1):
                    c = rem % int(L["sizes"][d])
                    rem //= int(L["sizes"][d])
                    ia += c * int(L["sa"][d])
                    oo += c * int(L["so"][d])
                offs = torch.zeros(1, dtype=torch.int64)
                for d in range(int(L["rdim"])):
                    offs = (offs.unsqueeze(1) + torch.arange(int(L["rsizes"][d])) * int(L["rsa"][d])).reshape(-1)
                s = base[ia + offs].sum() if int(L["rtotal"]) > 0 else torch.tensor(0.0)
                if it["flags"] & IF_MEAN:
                    s = s / int(L["rtotal"])
                outv[oo] = s.to(TDT[dto])
        else:
            raise AssertionError(f"unexpected item kind {kind}")
