"""scheduler_context — TorchDispatchMode plugin that routes small pointwise and reduction
ops to the persistent runtime (the reference's pytorch_ext/scheduler.py API).

Same public surface as the reference: ``scheduler_context(*, capacity=8192,
threads_per_block=256, size_threshold=1 << 16, auto_flush_ms=2.0)``, ``GPUOSScheduler`` and
``_GPUOSSchedulerMode`` (scheduler.py:22-466).  Differences, all deliberate:

* Every in-scope op runs on the GPU through a built-in operator of the runtime; nothing
  needs an NVRTC compile, so the reference's ``GPUOS_SCHEDULER_DISABLE_JIT`` switch
  (scheduler.py:19, default on, which sent everything except add/sub/mul/div back to
  eager) no longer gates which ops are scheduled.
* Results are written into the tensor returned to the caller (the reference's fused path
  wrote into a fresh tensor and lost them, scheduler.py:380).
* Dependencies: the runtime orders scheduled requests that read or write the same memory
  (inside and across flushes), so chains of scheduled ops need no flush.  Any op that is
  not scheduled and touches memory a pending request reads or writes triggers a sync
  flush first (the reference only tracked outputs, and skipped "fusible" ops, so a chain
  of pending adds never flushed, scheduler.py:53-98).
* Semantics follow PyTorch: alpha of add/sub, positional clamp bounds (scheduler.py:270
  read kwargs only), NaN-propagating maximum/minimum, erf GELU, expm1 ELU, softplus
  threshold.
* Operands: CUDA float32/float16/bfloat16 tensors (any strides, broadcast) or Python
  numbers; anything else (integer tensors, grad mode, CPU tensors, tensors above
  ``size_threshold`` elements) is left to PyTorch, as in the reference.
"""
from __future__ import annotations

import contextlib
import os
import threading
import time
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


def _storage_key(t: torch.Tensor) -> int:
    """Base address of the tensor's storage (a view's data pointer minus its offset), without
    building a storage object on every call."""
    return t.data_ptr() - t.storage_offset() * t.element_size()


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


class _GPUOSSchedulerMode(TorchDispatchMode):
    def __init__(self, *, size_threshold: int, auto_flush_ms: Optional[float], pending: Set[int]):
        super().__init__()
        self.size_threshold = size_threshold
        self.auto_flush_ms = auto_flush_ms
        self.pending = pending  # storages read or written by requests not yet known complete
        self.fused = {}  # kept for API compatibility (expression fusion is not used)
        self.scheduled = 0
        self.fallbacks = 0
        self._stop = False
        self._bg: Optional[threading.Thread] = None
        if auto_flush_ms and auto_flush_ms > 0:
            self._bg = threading.Thread(target=self._flusher, daemon=True)
            self._bg.start()

    def close(self):
        self._stop = True
        if self._bg:
            self._bg.join(timeout=1.0)

    def _flusher(self):
        # periodic asynchronous flush of pending requests (scheduler.py:40-51)
        while not self._stop:
            time.sleep(self.auto_flush_ms / 1000.0)
            try:
                gpuos_ext.flush(sync=False)
            except Exception:
                pass

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
        if out is None:
            if shape == a.shape and dtype == a.dtype and a.is_contiguous():
                out = torch.empty_like(a)  # the same contiguous tensor, allocated faster
            else:
                out = torch.empty(shape, dtype=dtype, device=a.device)
        elif not (isinstance(out, torch.Tensor) and out.is_cuda and out.dtype in _FLOATS):
            return None
        gpuos_ext.submit_elementwise(op, a, b if b_t else float(b), out, p0, 0.0)
        self._mark(a, b if b_t else None, out)
        self.scheduled += 1
        return out

    def _schedule_unary(self, op, x, p0=0.0, p1=0.0):
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
        gpuos_ext.submit_elementwise(op, x, None, out, p0, p1)
        self._mark(x, out)
        self.scheduled += 1
        return out

    def _try_parametric(self, name, args, kwargs):
        x = args[0]
        kw = kwargs or {}

        def arg(i, key, default):
            if key in kw:
                return kw[key]
            return args[i] if len(args) > i else default

        if name == "aten::gelu":
            approx = arg(1, "approximate", "none")
            return self._schedule_unary(_E.EW_GELU_TANH if approx == "tanh" else _E.EW_GELU, x)
        if name == "aten::leaky_relu":
            return self._schedule_unary(_E.EW_LEAKY_RELU, x, float(arg(1, "negative_slope", 0.01)))
        if name == "aten::hardtanh":
            return self._schedule_unary(_E.EW_CLAMP, x, float(arg(1, "min_val", -1.0)), float(arg(2, "max_val", 1.0)))
        if name == "aten::elu":
            alpha, scale, iscale = arg(1, "alpha", 1.0), arg(2, "scale", 1), arg(3, "input_scale", 1)
            if scale != 1 or iscale != 1:
                return None
            return self._schedule_unary(_E.EW_ELU, x, float(alpha))
        if name == "aten::softplus":
            return self._schedule_unary(_E.EW_SOFTPLUS, x, float(arg(1, "beta", 1.0)), float(arg(2, "threshold", 20.0)))
        if name == "aten::clamp":
            lo, hi = arg(1, "min", None), arg(2, "max", None)
            if isinstance(lo, torch.Tensor) or isinstance(hi, torch.Tensor):
                return None
            if lo is not None and hi is not None:
                return self._schedule_unary(_E.EW_CLAMP, x, float(lo), float(hi))
            if lo is not None:
                return self._schedule_unary(_E.EW_CLAMP_MIN, x, float(lo))
            if hi is not None:
                return self._schedule_unary(_E.EW_CLAMP_MAX, x, float(hi))
            return None
        if name == "aten::clamp_min":
            v = arg(1, "min", None)
            return None if isinstance(v, torch.Tensor) or v is None else self._schedule_unary(_E.EW_CLAMP_MIN, x, float(v))
        if name == "aten::clamp_max":
            v = arg(1, "max", None)
            return None if isinstance(v, torch.Tensor) or v is None else self._schedule_unary(_E.EW_CLAMP_MAX, x, float(v))
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
        kwargs = kwargs or {}
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
            return res
        # Not scheduled: make sure no pending request reads or writes what this op touches.
        if self._touches_pending(args, kwargs):
            self._sync_flush()
        self.fallbacks += 1
        return func(*args, **kwargs)

    def flush_fused(self):
        """Kept for API compatibility: requests are submitted as they are dispatched."""
        self.fused.clear()


class GPUOSScheduler:
    def __init__(self, *, capacity: int = 8192, threads_per_block: int = 256, size_threshold: int = 1 << 16,
                 auto_flush_ms: Optional[float] = 2.0):
        self.capacity = capacity
        self.threads_per_block = threads_per_block
        self.size_threshold = size_threshold
        self.auto_flush_ms = auto_flush_ms
        self._mode: Optional[_GPUOSSchedulerMode] = None
        self._pending: Set[int] = set()

    def __enter__(self):
        gpuos_ext.init(self.capacity, self.threads_per_block)
        self._mode = _GPUOSSchedulerMode(size_threshold=self.size_threshold, auto_flush_ms=self.auto_flush_ms,
                                         pending=self._pending)
        self._cm = self._mode.__enter__()
        return self

    def flush(self, sync: bool = False):
        gpuos_ext.flush(sync=sync)
        if sync:
            self._pending.clear()

    @property
    def stats(self):
        m = self._mode
        return {"scheduled": m.scheduled if m else 0, "fallbacks": m.fallbacks if m else 0}

    def __exit__(self, exc_type, exc, tb):
        try:
            if self._mode is not None:
                self._mode.close()
                self._mode.__exit__(exc_type, exc, tb)
        finally:
            gpuos_ext.flush(sync=True)
            self._pending.clear()
            gpuos_ext.shutdown()

    def flush_fused(self):
        if self._mode is not None:
            self._mode.flush_fused()


@contextlib.contextmanager
def scheduler_context(*, capacity: int = 8192, threads_per_block: int = 256, size_threshold: int = 1 << 16,
                      auto_flush_ms: Optional[float] = 2.0):
    sched = GPUOSScheduler(capacity=capacity, threads_per_block=threads_per_block, size_threshold=size_threshold,
                           auto_flush_ms=auto_flush_ms)
    with sched:
        yield sched
