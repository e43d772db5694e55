"""CPU oracle for the persistent micro-op path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (its CPU baseline leg and
``--impl reference``) may import this module; the runtime never does.

Two layers:

1. A numpy restatement of the reference's own device semantics, used to pin the oracle
   against the reference's known answers and to document where the reference deviates
   from PyTorch:
     * ``linear_to_offset``   src/persistent_kernel.cu:20-31
     * ``ld_as_float`` / ``st_from_float``   src/persistent_kernel.cu:60-78
     * ``op_batch``           src/persistent_kernel.cu:81-112 (sub-tasks in order; op codes
                              0 add, 1 mul, 2 sub, 3 div with ``B != 0 ? A / B : 0``)
     * ``fill_tensorref``     pytorch_ext/gpuos_ext.cpp:260-278 (right-aligned broadcast,
                              stride 0 where the input size is 1)
     * ``reduce_task``        pytorch_ext/gpuos_ext.cpp:915-995 (sum/mean over r_axes,
                              keepdim axis skipping)
2. ``ew_torch`` / ``reduce_torch``: the same requests evaluated by PyTorch CPU eager, the
   parity oracle named by the task (bit-exact for add/sub/mul/div/max/min/clamp and the
   other non-transcendental ops; ulp-bounded for transcendentals).
"""
from __future__ import annotations

import numpy as np
import torch

F32, F16, BF16 = 0, 1, 2
TORCH_DTYPE = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}

# Element-wise op codes (include/gpuos_b200.h, GpuosEwOp); 0..3 are the reference's
# op_batch sub-op codes (src/persistent_kernel.cu:101-106).
EW = dict(ADD=0, MUL=1, SUB=2, DIV=3, MAXIMUM=4, MINIMUM=5, POW=6, COPY=7, RELU=8, SIGMOID=9,
          TANH=10, EXP=11, LOG=12, SQRT=13, ABS=14, HARDSIGMOID=15, HARDSWISH=16, GELU=17,
          GELU_TANH=18, SIN=19, COS=20, LEAKY_RELU=21, CLAMP=22, CLAMP_MIN=23, CLAMP_MAX=24,
          ELU=25, SOFTPLUS=26, NEG=27, ADD_ALPHA=28, SUB_ALPHA=29)
BINARY = {EW[k] for k in ("ADD", "MUL", "SUB", "DIV", "MAXIMUM", "MINIMUM", "POW", "ADD_ALPHA", "SUB_ALPHA")}
TRANSCENDENTAL = {EW[k] for k in ("POW", "SIGMOID", "TANH", "EXP", "LOG", "GELU", "GELU_TANH", "SIN",
                                  "COS", "ELU", "SOFTPLUS")}


# ---------------------------------------------------------------------------------------
# 1. reference device semantics
# ---------------------------------------------------------------------------------------
def linear_to_offset(sizes, strides, idx: int) -> int:
    """src/persistent_kernel.cu:20-31: decode a linear output index with the operand's own
    sizes (size <= 0 treated as 1) and accumulate idx_d * stride_d."""
    off = 0
    for d in range(len(sizes) - 1, -1, -1):
        dim = sizes[d] if sizes[d] > 0 else 1
        off += (idx % dim) * strides[d]
        idx //= dim
    return off


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 (round to nearest even) -> float32, as __float2bfloat16_rn."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    out[nan] = np.float32("nan")
    return out


def st_from_float(v: np.ndarray, dtype: int) -> np.ndarray:
    """src/persistent_kernel.cu:70-78: fp32 value stored as f32 / f16 (RN) / bf16 (RN)."""
    v = np.asarray(v, dtype=np.float32)
    if dtype == F16:
        return v.astype(np.float16).astype(np.float32)
    if dtype == BF16:
        return bf16_round(v)
    return v


def fill_tensorref(in_sizes, in_strides, out_sizes):
    """pytorch_ext/gpuos_ext.cpp:260-278: right-align the input against the output dims;
    missing dims get size 1 / stride 0, size-1 dims get stride 0."""
    nd = len(out_sizes)
    sizes, strides = [0] * nd, [0] * nd
    for d in range(nd):
        od, i = nd - 1 - d, len(in_sizes) - 1 - d
        size_in = in_sizes[i] if i >= 0 else 1
        stride_in = in_strides[i] if i >= 0 else 0
        sizes[od] = size_in
        strides[od] = 0 if size_in == 1 else stride_in
    return sizes, strides


def op_batch(subtasks):
    """src/persistent_kernel.cu:81-112.  ``subtasks`` is a list of dicts with keys op, a, b
    (flat float32 numpy arrays, b may be None), out (flat array, written in place) and numel.
    Sub-tasks run in order, so later ones see earlier writes."""
    for u in subtasks:
        n = u["numel"]
        A = u["a"][:n].astype(np.float32)
        B = u["b"][:n].astype(np.float32) if u.get("b") is not None else np.zeros(n, np.float32)
        op = u["op"]
        with np.errstate(all="ignore"):
            if op == 0:
                R = A + B
            elif op == 1:
                R = A * B
            elif op == 2:
                R = A - B
            elif op == 3:
                R = np.where(B != 0, A / np.where(B != 0, B, 1), np.float32(0))
            else:
                R = A
        u["out"][:n] = R.astype(np.float32)


def reduce_task(x: np.ndarray, axes, keepdim: bool, mean: bool) -> np.ndarray:
    """pytorch_ext/gpuos_ext.cpp:915-995: float32 accumulation over the reduced axes."""
    axes = tuple(sorted(a % x.ndim for a in axes))
    acc = np.add.reduce(x.astype(np.float32), axis=axes, keepdims=keepdim, dtype=np.float32)
    if mean:
        red = int(np.prod([x.shape[a] for a in axes])) if axes else 1
        acc = acc / np.float32(red)
    return acc


# ---------------------------------------------------------------------------------------
# 2. PyTorch CPU eager (parity oracle)
# ---------------------------------------------------------------------------------------
def ew_torch(op: int, a: torch.Tensor, b=None, p0: float = 0.0, p1: float = 0.0,
             out_dtype=None) -> torch.Tensor:
    """Evaluate element-wise op ``op`` with PyTorch CPU eager.  ``b`` may be a tensor or a
    Python number; inputs are promoted as torch does and the result cast to out_dtype."""
    a = a.cpu()
    if isinstance(b, torch.Tensor):
        b = b.cpu()
    F = torch.nn.functional
    if op == EW["ADD"]:
        r = torch.add(a, b)
    elif op == EW["MUL"]:
        r = torch.mul(a, b)
    elif op == EW["SUB"]:
        r = torch.sub(a, b)
    elif op == EW["DIV"]:
        r = torch.div(a, b)
    elif op == EW["MAXIMUM"]:
        r = torch.maximum(a, b if isinstance(b, torch.Tensor) else torch.tensor(b, dtype=a.dtype))
    elif op == EW["MINIMUM"]:
        r = torch.minimum(a, b if isinstance(b, torch.Tensor) else torch.tensor(b, dtype=a.dtype))
    elif op == EW["POW"]:
        r = torch.pow(a, b)
    elif op == EW["COPY"]:
        r = a.clone()
    elif op == EW["RELU"]:
        r = torch.relu(a)
    elif op == EW["SIGMOID"]:
        r = torch.sigmoid(a)
    elif op == EW["TANH"]:
        r = torch.tanh(a)
    elif op == EW["EXP"]:
        r = torch.exp(a)
    elif op == EW["LOG"]:
        r = torch.log(a)
    elif op == EW["SQRT"]:
        r = torch.sqrt(a)
    elif op == EW["ABS"]:
        r = torch.abs(a)
    elif op == EW["HARDSIGMOID"]:
        r = F.hardsigmoid(a)
    elif op == EW["HARDSWISH"]:
        r = F.hardswish(a)
    elif op == EW["GELU"]:
        r = F.gelu(a)
    elif op == EW["GELU_TANH"]:
        r = F.gelu(a, approximate="tanh")
    elif op == EW["SIN"]:
        r = torch.sin(a)
    elif op == EW["COS"]:
        r = torch.cos(a)
    elif op == EW["LEAKY_RELU"]:
        r = F.leaky_relu(a, p0)
    elif op == EW["CLAMP"]:
        r = torch.clamp(a, p0, p1)
    elif op == EW["CLAMP_MIN"]:
        r = torch.clamp_min(a, p0)
    elif op == EW["CLAMP_MAX"]:
        r = torch.clamp_max(a, p0)
    elif op == EW["ELU"]:
        r = F.elu(a, p0)
    elif op == EW["SOFTPLUS"]:
        r = F.softplus(a, p0, p1)
    elif op == EW["NEG"]:
        r = torch.neg(a)
    elif op == EW["ADD_ALPHA"]:
        r = torch.add(a, b, alpha=p0)
    elif op == EW["SUB_ALPHA"]:
        r = torch.sub(a, b, alpha=p0)
    else:
        raise ValueError(f"unknown op {op}")
    return r.to(out_dtype) if out_dtype is not None else r


def reduce_torch(x: torch.Tensor, axes, keepdim: bool, mean: bool, out_dtype=None) -> torch.Tensor:
    """sum/mean over axes with float32 accumulation, result cast to out_dtype (the input
    dtype by default, pytorch_ext/scheduler.py:338)."""
    xf = x.cpu().float()
    r = xf.mean(dim=list(axes), keepdim=keepdim) if mean else xf.sum(dim=list(axes), keepdim=keepdim)
    return r.to(out_dtype if out_dtype is not None else x.dtype)


# ---------------------------------------------------------------------------------------
# comparison helpers
# ---------------------------------------------------------------------------------------
def ulp_diff(got: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    """Distance in float32 ulps (monotone integer mapping); NaN==NaN counts as 0, NaN vs
    number as 2**31."""
    g = got.detach().cpu().float().contiguous().view(torch.int32).long()
    r = ref.detach().cpu().float().contiguous().view(torch.int32).long()
    g = torch.where(g < 0, -(g & 0x7FFFFFFF), g)
    r = torch.where(r < 0, -(r & 0x7FFFFFFF), r)
    d = (g - r).abs()
    gn, rn = torch.isnan(got.detach().cpu().float()), torch.isnan(ref.detach().cpu().float())
    d = torch.where(gn & rn, torch.zeros_like(d), d)
    d = torch.where(gn ^ rn, torch.full_like(d, 2 ** 31), d)
    return d


def same_bits(got: torch.Tensor, ref: torch.Tensor) -> bool:
    """Bit-exact equality with every NaN treated as equal to every NaN."""
    g = got.detach().cpu()
    r = ref.detach().cpu()
    if g.dtype != r.dtype or g.shape != r.shape:
        return False
    gn, rn = torch.isnan(g.float()), torch.isnan(r.float())
    if not torch.equal(gn, rn):
        return False
    w = {torch.float32: torch.int32, torch.float16: torch.int16, torch.bfloat16: torch.int16}[g.dtype]
    gb = g.contiguous().view(w)[~gn]
    rb = r.contiguous().view(w)[~rn]
    return torch.equal(gb, rb)
