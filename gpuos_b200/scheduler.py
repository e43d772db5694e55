"""scheduler_context — the PyTorch plugin that routes small pointwise and reduction ops to the
persistent runtime (the reference's pytorch_ext/scheduler.py API), intercepting ATen calls in
C++ (default) or in a TorchDispatchMode.

Same public surface as the reference: ``scheduler_context(*, capacity=8192,
threads_per_block=256, size_threshold=1 << 16, auto_flush_ms=2.0)``, ``GPUOSScheduler`` and
``_GPUOSSchedulerMode`` (scheduler.py:22-466).  Differences, all deliberate:

* Every in-scope op runs on the GPU through a built-in operator of the runtime; nothing
  needs an NVRTC compile, so the reference's ``GPUOS_SCHEDULER_DISABLE_JIT`` switch
  (scheduler.py:19, default on, which sent everything except add/sub/mul/div back to
  eager) no longer gates which ops are scheduled.  With ``GPUOS_SCHEDULER_DISABLE_JIT=0`` it
  turns on fusion, as in the reference (scheduler.py:145-160, 376-396): a chain of fp32
  element-wise ops, each taking the previous one's result, is compiled into one NVRTC operator
  (the built-in operators' own math, so the chain rounds as the unfused ops do) and written
  into the tensor returned for the chain's last op; results of the chain that are still
  referenced when it is submitted are written too (the reference wrote into a fresh tensor and
  lost them).
* Results are written into the tensor returned to the caller (the reference's fused path
  wrote into a fresh tensor and lost them, scheduler.py:380).
* Dependencies: the runtime orders scheduled requests that read or write the same memory
  (inside and across flushes), so chains of scheduled ops need no flush.  Any op that is
  not scheduled and touches memory a pending request reads or writes triggers a sync
  flush first (the reference only tracked outputs, and skipped "fusible" ops, so a chain
  of pending adds never flushed, scheduler.py:53-98).  An op that is not scheduled and launches
  a kernel on CUDA tensors also stops the resident worker first, which would otherwise hold
  every SM until its idle stop.
* Semantics follow PyTorch: alpha of add/sub, positional clamp bounds (scheduler.py:270
  read kwargs only), NaN-propagating maximum/minimum, erf GELU, expm1 ELU, softplus
  threshold.
* Operands: CUDA float32/float16/bfloat16 tensors (any strides, broadcast) or Python
  numbers; anything else (integer tensors, grad mode, CPU tensors, tensors above
  ``size_threshold`` elements) is left to PyTorch, as in the reference.
* Two interchangeable intercepts (``native=``): the C++ one (a boxed fallback on a dispatcher
  key included for the entering thread, csrc/intercept.cpp; the default) routes the same ops
  by the same rules as the Python ``TorchDispatchMode`` below without a Python call per op.
  Fusion (``GPUOS_SCHEDULER_DISABLE_JIT=0``) is built on the Python mode, which it then selects.
"""
from __future__ import annotations

import collections
import contextlib
import math
import os
import struct
import threading
import warnings
import weakref
from typing import Any, Optional, Set

import torch
from torch.utils._python_dispatch import TorchDispatchMode

from . import gpuos_ext

_DISABLE_JIT = os.environ.get("GPUOS_SCHEDULER_DISABLE_JIT", "1") not in ("0", "false", "False")
_FLOATS = (torch.float32, torch.float16, torch.bfloat16)
_E = gpuos_ext

_BINARY = {
    "aten::add.Tensor": _E.EW_ADD, "aten::sub.Tensor": _E.EW_SUB, "aten::mul.Tensor": _E.EW_MUL,
    "aten::div.Tensor": _E.EW_DIV, "aten::maximum": _E.EW_MAXIMUM, "aten::minimum": _E.EW_MINIMUM,
    "aten::pow.Tensor_Tensor": _E.EW_POW, "aten::pow.Tensor_Scalar": _E.EW_POW,
}
_UNARY = {
    "aten::relu": _E.EW_RELU, "aten::sigmoid": _E.EW_SIGMOID, "aten::tanh": _E.EW_TANH,
    "aten::exp": _E.EW_EXP, "aten::log": _E.EW_LOG, "aten::sqrt": _E.EW_SQRT, "aten::abs": _E.EW_ABS,
    "aten::hardsigmoid": _E.EW_HARDSIGMOID, "aten::hardswish": _E.EW_HARDSWISH, "aten::sin": _E.EW_SIN,
    "aten::cos": _E.EW_COS, "aten::neg": _E.EW_NEG,
}
_PARAMETRIC = {"aten::gelu", "aten::leaky_relu", "aten::hardtanh", "aten::elu", "aten::softplus",
               "aten::clamp", "aten::clamp_min", "aten::clamp_max"}
_REDUCE = {"aten::sum.dim_IntList", "aten::mean.dim", "aten::sum", "aten::mean"}
# allocations that launch no kernel (views are recognised by func.is_view)
_NO_KERNEL = {"aten::empty.memory_format", "aten::empty_like", "aten::empty_strided", "aten::new_empty",
              "aten::new_empty_strided"}


def _storage_key(t: torch.Tensor) -> int:
    """Base address of the tensor's storage (a view's data pointer minus its offset), without
    building a storage object on every call."""
    return t.data_ptr() - t.storage_offset() * t.element_size()


def _f32_literal(v) -> Optional[str]:
    """Exact C++ literal of a Python number rounded to float32 (None for inf / nan)."""
    f = struct.unpack("f", struct.pack("f", float(v)))[0]
    if not math.isfinite(f):
        return None
    return float(f).hex() + "f"


class _Chain:
    """A deferred chain of fp32 element-wise ops: the root reads A (and B), every later op the
    previous result.  `steps` holds (expression of the value after the step, built-in op of a
    one-op chain, weak reference to the step's result tensor)."""

    def __init__(self, a, b, expr: str, single, out):
        self.a, self.b = a, b
        self.arity = 2 if b is not None else 1
        self.out = out
        self.steps = [(expr, single, weakref.ref(out))]

    def extend(self, code: int, b_lit: str, p0: str, p1: str, out) -> None:
        prev = self.steps[-1][0]
        self.steps.append((f"gpuos::ew_apply<{code}>({prev}, {b_lit}, {p0}, {p1})", None, weakref.ref(out)))
        self.out = out


_MAX_CHAIN = 16

def _submit_new(op: int, a, b):
    """Submit op(a[, b]) into a new contiguous tensor like a, allocated by the extension."""
    return gpuos_ext.submit_ew_new(op, a, b)


def _same_layout_operands(a, b, size_threshold: int) -> bool:
    """Both CUDA tensors of one floating dtype, shape and device, contiguous, within the size
    threshold."""
    return (type(a) is torch.Tensor and type(b) is torch.Tensor and a.is_cuda and a.dtype is b.dtype
            and a.dtype in _FLOATS and a.shape == b.shape and a.numel() <= size_threshold
            and a.is_contiguous() and b.is_contiguous() and a.device == b.device)


def _has_cuda_tensor(args, kwargs) -> bool:
    """Whether a CUDA tensor is among the arguments (lists and tuples included)."""
    def walk(o) -> bool:
        if isinstance(o, torch.Tensor):
            return o.is_cuda
        if isinstance(o, (list, tuple)):
            return any(walk(i) for i in o)
        return False
    return walk(args) or any(walk(v) for v in kwargs.values())


def _one_operand(x, size_threshold: int) -> bool:
    """A CUDA tensor of a floating dtype within the size threshold and the rank limit."""
    return (type(x) is torch.Tensor and x.is_cuda and x.dtype in _FLOATS and x.numel() <= size_threshold
            and x.dim() <= 8)


# op overload -> (route, name): 1 binary, 2 unary, 3 parametric unary, 4 reduction, 5 top-k,
# 0 not ours
_ROUTES: dict = {}


def _route(func):
    r = _ROUTES.get(func)
    if r is None:
        name = func.name()
        kind = (1 if name in _BINARY else 2 if name in _UNARY else 3 if name in _PARAMETRIC
                else 4 if name in _REDUCE else 5 if name == "aten::topk" else 0)
        r = _ROUTES[func] = (kind, name)
    return r


class _AutoFlusher:
    """Periodic asynchronous flush of pending requests (scheduler.py:40-51), for either intercept."""

    def __init__(self, period_ms: Optional[float]):
        self._stop = threading.Event()
        self._bg: Optional[threading.Thread] = None
        if period_ms and period_ms > 0:
            self._bg = threading.Thread(target=self._run, args=(period_ms / 1000.0,), daemon=True)
            self._bg.start()

    def _run(self, period: float):
        while not self._stop.wait(period):
            try:
                gpuos_ext.flush(sync=False)
            except Exception:
                pass

    def close(self):
        self._stop.set()
        if self._bg:
            self._bg.join(timeout=1.0)


class _GPUOSSchedulerMode(TorchDispatchMode):
    @classmethod
    def _should_skip_dynamo(cls) -> bool:
        # PyTorch otherwise wraps __torch_dispatch__ in a per-call guard that keeps torch.compile
        # from tracing into it (about 3 us of every op's ~8.5 us here); nothing compiled runs
        # through this mode
        return False

    def __init__(self, *, size_threshold: int, auto_flush_ms: Optional[float], pending: Set[int]):
        super().__init__()
        self.size_threshold = size_threshold
        self.auto_flush_ms = auto_flush_ms
        self.pending = pending  # storages read or written by requests not yet known complete
        self.fused = {}  # kept for API compatibility (the chain being fused is self.chain)
        self.scheduled = 0
        self.fallbacks = 0
        # per aten op name: requests submitted to the runtime / ops left to PyTorch
        self.scheduled_ops: collections.Counter = collections.Counter()
        self.fallback_ops: collections.Counter = collections.Counter()
        # fusion (GPUOS_SCHEDULER_DISABLE_JIT=0): the chain being built, not yet submitted
        self.fuse = _fusion_requested()
        self.chain: Optional[_Chain] = None
        self.fused_chains = 0
        self.fused_ops = 0
        self._flusher = _AutoFlusher(auto_flush_ms)

    def close(self):
        self._flusher.close()

    # -- dependency tracking ----------------------------------------------------------
    def _touches_pending(self, args, kwargs) -> bool:
        if not self.pending:
            return False

        def walk(o: Any) -> bool:
            if isinstance(o, torch.Tensor):
                return o.is_cuda and _storage_key(o) in self.pending
            if isinstance(o, (list, tuple)):
                return any(walk(i) for i in o)
            if isinstance(o, dict):
                return any(walk(v) for v in o.values())
            return False

        return walk(args) or walk(kwargs)

    def _sync_flush(self):
        self.flush_fused()
        gpuos_ext.flush(sync=True)
        self.pending.clear()

    def _mark(self, *tensors):
        for t in tensors:
            if isinstance(t, torch.Tensor):
                self.pending.add(_storage_key(t))

    # -- eligibility --------------------------------------------------------------------
    def _ok_tensor(self, t) -> bool:
        return (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype in _FLOATS
                and t.numel() <= self.size_threshold and t.dim() <= 8)

    @staticmethod
    def _ok_scalar(v) -> bool:
        return isinstance(v, (float, int, bool)) and not isinstance(v, complex)

    # -- scheduling ---------------------------------------------------------------------
    def _try_schedule_binary(self, name, a, b, *, alpha=None, out=None):
        op = _BINARY[name]
        a_t, b_t = isinstance(a, torch.Tensor), isinstance(b, torch.Tensor)
        if not a_t or not self._ok_tensor(a):
            return None
        if b_t:
            if b.dim() == 0 and not b.is_cuda:
                b = b.item()
                b_t = False
            elif not self._ok_tensor(b) or b.get_device() != a.get_device():
                return None
        if not b_t and not self._ok_scalar(b):
            return None
        p0 = 0.0
        if alpha is not None and alpha != 1:
            if name not in ("aten::add.Tensor", "aten::sub.Tensor") or not self._ok_scalar(alpha):
                return None
            op = _E.EW_ADD_ALPHA if name == "aten::add.Tensor" else _E.EW_SUB_ALPHA
            p0 = float(alpha)
            if not b_t:  # a + alpha * scalar folds to a scalar operand
                op = _E.EW_ADD if name == "aten::add.Tensor" else _E.EW_SUB
                b = float(b) * p0
        if b_t:
            shape = a.shape
            if b.shape != shape:
                try:
                    shape = torch.broadcast_shapes(shape, b.shape)
                except RuntimeError:
                    return None
            dtype = a.dtype if b.dtype == a.dtype else torch.result_type(a, b)
        else:
            shape = a.shape
            dtype = a.dtype  # a floating tensor keeps its dtype against a Python number
        if dtype not in _FLOATS:
            return None
        ours = out is None
        if out is None:
            if shape == a.shape and dtype == a.dtype and a.is_contiguous():
                out = torch.empty_like(a)  # the same contiguous tensor, allocated faster
            else:
                out = torch.empty(shape, dtype=dtype, device=a.device)
        elif not (isinstance(out, torch.Tensor) and out.is_cuda and out.dtype in _FLOATS):
            return None
        if (self.fuse and ours and dtype == torch.float32 and a.dtype == torch.float32 and p0 == 0.0
                and (b.dtype == torch.float32 and b.shape == a.shape if b_t else name != "aten::pow.Tensor_Scalar")):
            lit = "B" if b_t else _f32_literal(b)
            if lit is not None:
                # the root of a chain: submitted when the chain ends
                self.chain = _Chain(a, b if b_t else None, f"gpuos::ew_apply<{op}>(A, {lit}, 0.f, 0.f)",
                                    (op, b if b_t else float(b), 0.0, 0.0), out)
                self._mark(a, b if b_t else None, out)
                self.scheduled += 1
                return out
        gpuos_ext.submit_elementwise(op, a, b if b_t else float(b), out, p0, 0.0)
        self._mark(a, b if b_t else None, out)
        self.scheduled += 1
        return out

    def _schedule_unary(self, op, x, p0=0.0, p1=0.0):
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
        if self.fuse and x.dtype == torch.float32:
            l0, l1 = _f32_literal(p0), _f32_literal(p1)
            if l0 is not None and l1 is not None:
                self.chain = _Chain(x, None, f"gpuos::ew_apply<{op}>(A, 0.f, {l0}, {l1})", (op, None, p0, p1), out)
                self._mark(x, out)
                self.scheduled += 1
                return out
        gpuos_ext.submit_elementwise(op, x, None, out, p0, p1)
        self._mark(x, out)
        self.scheduled += 1
        return out

    # -- fusion ---------------------------------------------------------------------------
    def _unary_code(self, kind, name, args, kwargs):
        """(op code, p0, p1) of a unary or parametric op on args[0], or None."""
        if kind == 2:
            return _UNARY[name], 0.0, 0.0
        return self._parametric_code(name, args, kwargs)

    def _try_extend(self, kind, name, args, kwargs):
        """Append this op to the chain when it is an fp32 element-wise op of the chain's last
        result (the very tensor returned for it) and nothing else; returns its result or None."""
        c = self.chain
        if (not args or args[0] is not c.out or len(c.steps) >= _MAX_CHAIN or torch.is_grad_enabled()
                or kwargs.get("out") is not None):
            return None
        if kind in (2, 3):
            rc = self._unary_code(kind, name, args, kwargs)
            if rc is None:
                return None
            op, p0, p1 = rc
            lits = ("0.f", _f32_literal(p0), _f32_literal(p1))
        elif kind == 1 and len(args) >= 2 and name != "aten::pow.Tensor_Scalar":
            b = args[1]
            if isinstance(b, torch.Tensor):
                if b.dim() != 0 or b.is_cuda:
                    return None
                b = b.item()
            alpha = kwargs.get("alpha")
            if not self._ok_scalar(b) or (alpha is not None and alpha != 1):
                return None
            op = _BINARY[name]
            lits = (_f32_literal(b), "0.f", "0.f")
        else:
            return None
        if any(v is None for v in lits):
            return None
        out = torch.empty_like(c.out)
        c.extend(op, *lits, out)
        self._mark(out)
        self.scheduled += 1
        return out

    def _submit_steps(self, c: _Chain, k: int, out) -> None:
        """Submit the value after step k of chain c into `out`."""
        expr, single, _ = c.steps[k]
        if k == 0:
            op, b, p0, p1 = single
            gpuos_ext.submit_elementwise(op, c.a, b, out, p0, p1)
            return
        slot = gpuos_ext.register_elementwise(f"fused|{c.arity}|{expr}", expr, c.arity, backend="nvrtc",
                                              device=out.device)
        if c.arity == 2:
            gpuos_ext.submit_binary(slot, c.a, c.b, out)
        else:
            gpuos_ext.submit_unary(slot, c.a, out)

    def flush_fused(self):
        """Submit the chain being built: its last result, plus every earlier result of it that
        is still referenced."""
        c, self.chain = self.chain, None
        if c is None:
            return
        last = len(c.steps) - 1
        self._submit_steps(c, last, c.out)
        for k in range(last):
            t = c.steps[k][2]()
            if t is not None:
                self._submit_steps(c, k, t)
        if last > 0:
            self.fused_chains += 1
            self.fused_ops += last + 1

    def _try_parametric(self, name, args, kwargs):
        code = self._parametric_code(name, args, kwargs)
        return None if code is None else self._schedule_unary(code[0], args[0], code[1], code[2])

    def _parametric_code(self, name, args, kwargs):
        """(op code, p0, p1) of a parametric unary op, or None when its arguments are not ours."""
        kw = kwargs or {}

        def arg(i, key, default):
            if key in kw:
                return kw[key]
            return args[i] if len(args) > i else default

        if name == "aten::gelu":
            approx = arg(1, "approximate", "none")
            return (_E.EW_GELU_TANH if approx == "tanh" else _E.EW_GELU, 0.0, 0.0)
        if name == "aten::leaky_relu":
            return (_E.EW_LEAKY_RELU, float(arg(1, "negative_slope", 0.01)), 0.0)
        if name == "aten::hardtanh":
            return (_E.EW_CLAMP, float(arg(1, "min_val", -1.0)), float(arg(2, "max_val", 1.0)))
        if name == "aten::elu":
            alpha, scale, iscale = arg(1, "alpha", 1.0), arg(2, "scale", 1), arg(3, "input_scale", 1)
            if scale != 1 or iscale != 1:
                return None
            return (_E.EW_ELU, float(alpha), 0.0)
        if name == "aten::softplus":
            return (_E.EW_SOFTPLUS, float(arg(1, "beta", 1.0)), float(arg(2, "threshold", 20.0)))
        if name == "aten::clamp":
            lo, hi = arg(1, "min", None), arg(2, "max", None)
            if isinstance(lo, torch.Tensor) or isinstance(hi, torch.Tensor):
                return None
            if lo is not None and hi is not None:
                return (_E.EW_CLAMP, float(lo), float(hi))
            if lo is not None:
                return (_E.EW_CLAMP_MIN, float(lo), 0.0)
            if hi is not None:
                return (_E.EW_CLAMP_MAX, float(hi), 0.0)
            return None
        if name == "aten::clamp_min":
            v = arg(1, "min", None)
            return None if isinstance(v, torch.Tensor) or v is None else (_E.EW_CLAMP_MIN, float(v), 0.0)
        if name == "aten::clamp_max":
            v = arg(1, "max", None)
            return None if isinstance(v, torch.Tensor) or v is None else (_E.EW_CLAMP_MAX, float(v), 0.0)
        return None

    def _try_reduce(self, name, args, kwargs):
        x = args[0]
        kw = kwargs or {}
        if kw.get("dtype") is not None and kw.get("dtype") != x.dtype:
            return None
        if name in ("aten::sum", "aten::mean"):
            dims, keepdim = [], False
            if len(args) > 1 and args[1] is not None:
                return None  # sum(x, dtype) positional form
        else:
            dims = kw.get("dim", args[1] if len(args) > 1 else None)
            keepdim = bool(kw.get("keepdim", args[2] if len(args) > 2 else False))
            if dims is None:
                dims = []
            if isinstance(dims, int):
                dims = [dims]
            dims = list(dims)
        nd = x.dim()
        norm = []
        for d in dims:
            d = int(d)
            d = d + nd if d < 0 else d
            if d < 0 or d >= nd:
                return None
            norm.append(d)
        norm = sorted(set(norm))
        red = norm if norm else list(range(nd))
        if keepdim:
            shape = [1 if i in red else s for i, s in enumerate(x.shape)]
        else:
            shape = [s for i, s in enumerate(x.shape) if i not in red]
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
        op = _E.RED_MEAN if "mean" in name else _E.RED_SUM
        gpuos_ext.submit_reduction(op, x, out, red, keepdim)
        self._mark(x, out)
        self.scheduled += 1
        return out

    def _try_topk(self, args, kwargs):
        """aten::topk(self, k, dim=-1, largest=True, sorted=True) along the last dim of a
        contiguous tensor, k <= min(n, 256): the runtime's batched top-k (the reference sends
        topk to torch::topk, scheduler.py:346-370).  The values come preferred first, which
        also satisfies sorted=False."""
        x = args[0]

        def arg(i, key, default):
            return kwargs[key] if key in kwargs else (args[i] if len(args) > i else default)

        k, dim, largest = arg(1, "k", None), arg(2, "dim", -1), arg(3, "largest", True)
        if not isinstance(k, int) or x.dim() == 0 or not x.is_contiguous():
            return None
        n = x.shape[-1]
        if (dim if dim >= 0 else dim + x.dim()) != x.dim() - 1 or not (1 <= k <= min(n, 256)):
            return None
        shape = tuple(x.shape[:-1]) + (k,)
        values = torch.empty(shape, dtype=x.dtype, device=x.device)
        indices = torch.empty(shape, dtype=torch.int64, device=x.device)
        gpuos_ext.submit_topk_rows(x, values, indices, k, bool(largest))
        self._mark(x, values, indices)
        self.scheduled += 1
        return values, indices

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kind, name = _route(func)
        # fast path: a tensor-tensor op with operands of one dtype, shape and device, both
        # contiguous (the mixed-op stream's common case): no broadcasting, promotion or keyword
        # handling
        if kind == 1 and not kwargs and self.chain is None and not self.fuse and len(args) == 2:
            a, b = args
            if _same_layout_operands(a, b, self.size_threshold) and not torch.is_grad_enabled():
                out = _submit_new(_BINARY[name], a, b)
                pend = self.pending
                pend.add(a.data_ptr() - a.storage_offset() * a.element_size())
                pend.add(b.data_ptr() - b.storage_offset() * b.element_size())
                pend.add(out.data_ptr())
                self.scheduled += 1
                self.scheduled_ops[name] += 1
                return out
        elif kind == 3 and self.chain is None and not self.fuse and args:
            x = args[0]
            if _one_operand(x, self.size_threshold) and not torch.is_grad_enabled():
                code = self._parametric_code(name, args, kwargs or {})
                if code is not None:
                    out = gpuos_ext.submit_ew_new(code[0], x, None, code[1], code[2])
                    pend = self.pending
                    pend.add(x.data_ptr() - x.storage_offset() * x.element_size())
                    pend.add(out.data_ptr())
                    self.scheduled += 1
                    self.scheduled_ops[name] += 1
                    return out
        elif kind == 2 and not kwargs and self.chain is None and not self.fuse and len(args) == 1:
            x = args[0]
            if _one_operand(x, self.size_threshold) and not torch.is_grad_enabled():
                out = _submit_new(_UNARY[name], x, None)
                pend = self.pending
                pend.add(x.data_ptr() - x.storage_offset() * x.element_size())
                pend.add(out.data_ptr())
                self.scheduled += 1
                self.scheduled_ops[name] += 1
                return out
        kwargs = kwargs or {}
        if self.chain is not None:
            res = self._try_extend(kind, name, args, kwargs) if kind in (1, 2, 3) else None
            if res is not None:
                self.scheduled_ops[name] += 1
                return res
            self.flush_fused()  # anything else sees the chain's results in place
        res = None
        if kind and not torch.is_grad_enabled():
            if kind == 1:
                if len(args) >= 2:
                    res = self._try_schedule_binary(name, args[0], args[1], alpha=kwargs.get("alpha"),
                                                    out=kwargs.get("out"))
            elif args and self._ok_tensor(args[0]):
                if kind == 2:
                    res = self._schedule_unary(_UNARY[name], args[0])
                elif kind == 3:
                    res = self._try_parametric(name, args, kwargs)
                elif kind == 4:
                    res = self._try_reduce(name, args, kwargs)
                else:
                    res = self._try_topk(args, kwargs)
        if res is not None:
            self.scheduled_ops[name] += 1
            return res
        # Not scheduled: make sure no pending request reads or writes what this op touches.
        if self._touches_pending(args, kwargs):
            self._sync_flush()
        if (not func.is_view and name not in _NO_KERNEL and (self.pending or gpuos_ext.worker_alive())
                and _has_cuda_tensor(args, kwargs)):
            # A kernel of this op may need SMs that the resident worker holds; left alone, the
            # worker gives them back only at its idle stop (200 ms).  Finish the runtime's work and
            # stop the worker now: the next flush relaunches it (tens of microseconds).
            self._sync_flush()
            gpuos_ext.quiesce()
        self.fallbacks += 1
        self.fallback_ops[name] += 1
        return func(*args, **kwargs)



def _fusion_requested() -> bool:
    return os.environ.get("GPUOS_SCHEDULER_DISABLE_JIT", "1") in ("0", "false", "False")


class GPUOSScheduler:
    """``native``: True routes ops through the C++ intercept, False through the Python
    ``TorchDispatchMode``; None (default) takes the C++ one unless fusion is requested.  If the
    C++ intercept cannot be enabled (its dispatcher key taken in this process) the Python mode
    is used and a RuntimeWarning says so."""

    def __init__(self, *, capacity: int = 8192, threads_per_block: int = 256, size_threshold: int = 1 << 16,
                 auto_flush_ms: Optional[float] = 2.0, native: Optional[bool] = None):
        self.capacity = capacity
        self.threads_per_block = threads_per_block
        self.size_threshold = size_threshold
        self.auto_flush_ms = auto_flush_ms
        if native and _fusion_requested():
            raise ValueError("fusion (GPUOS_SCHEDULER_DISABLE_JIT=0) runs on the Python dispatch mode: native=False")
        self.native = (not _fusion_requested()) if native is None else bool(native)
        self._mode: Optional[_GPUOSSchedulerMode] = None
        self._flusher: Optional[_AutoFlusher] = None
        self._pending: Set[int] = set()

    def __enter__(self):
        gpuos_ext.init(self.capacity, self.threads_per_block)
        if self.native:
            try:
                gpuos_ext.intercept_enable(self.size_threshold)
            except RuntimeError as e:
                warnings.warn(f"scheduler_context: {e}; using the Python dispatch mode", RuntimeWarning)
                self.native = False
        if self.native:
            self._flusher = _AutoFlusher(self.auto_flush_ms)
        else:
            self._mode = _GPUOSSchedulerMode(size_threshold=self.size_threshold, auto_flush_ms=self.auto_flush_ms,
                                             pending=self._pending)
            self._cm = self._mode.__enter__()
        return self

    def flush(self, sync: bool = False):
        if self._mode is not None:
            self._mode.flush_fused()
        gpuos_ext.flush(sync=sync)
        if sync:
            self._pending.clear()
            if self.native:
                gpuos_ext.intercept_clear_pending()

    @property
    def stats(self):
        """Totals plus per-op counts: ``scheduled_ops`` / ``fallback_ops`` map an aten op name
        (``"aten::gelu"``) to the requests submitted to the runtime / the calls left to PyTorch."""
        if self.native:
            st = gpuos_ext.intercept_stats()
            st.update(fused_chains=0, fused_ops=0)
            return st
        m = self._mode
        return {"scheduled": m.scheduled if m else 0, "fallbacks": m.fallbacks if m else 0,
                "scheduled_ops": dict(m.scheduled_ops) if m else {},
                "fallback_ops": dict(m.fallback_ops) if m else {},
                "fused_chains": m.fused_chains if m else 0, "fused_ops": m.fused_ops if m else 0}

    def __exit__(self, exc_type, exc, tb):
        try:
            if self.native:
                if self._flusher is not None:
                    self._flusher.close()
                gpuos_ext.intercept_disable()
            elif self._mode is not None:
                self._mode.close()
                self._mode.__exit__(exc_type, exc, tb)
                self._mode.flush_fused()
        finally:
            gpuos_ext.flush(sync=True)
            self._pending.clear()
            if self.native:
                gpuos_ext.intercept_clear_pending()
            gpuos_ext.shutdown()

    def flush_fused(self):
        if self._mode is not None:
            self._mode.flush_fused()


@contextlib.contextmanager
def scheduler_context(*, capacity: int = 8192, threads_per_block: int = 256, size_threshold: int = 1 << 16,
                      auto_flush_ms: Optional[float] = 2.0, native: Optional[bool] = None):
    sched = GPUOSScheduler(capacity=capacity, threads_per_block=threads_per_block, size_threshold=size_threshold,
                           auto_flush_ms=auto_flush_ms, native=native)
    with sched:
        yield sched
