"""gpuos_ext — the reference's Python module API (pytorch_ext/gpuos_ext.cpp:1093-1142) on the
B200 runtime.

Every function of the reference module is here with the same name, defaults and argument
meaning.  The compiled binding (``_gpuos_ext``) provides the hot calls directly; this file
adds the registry-style calls that the reference implements next to them:

* ``register_elementwise(key, expr, arity)`` (gpuos_ext.cpp:814-881): expressions with
  the exact semantics of a built-in operator map to that operator's reference-ABI device
  function; any other C float expression is compiled by NVRTC for sm_100a, linked into the
  worker and installed in a slot (``register_jit``).  ``backend="interp"`` runs it on the
  worker's expression interpreter instead, which loads nothing and never stops the worker.
* ``register_reduce(key, op_name)`` (gpuos_ext.cpp:1003-1014): built-in sum/mean.
* ``register_topk`` / ``submit_topk`` (gpuos_ext.cpp:1050-1071): slot 42; top-k along the
  last dimension of a contiguous tensor runs on the persistent worker, other cases through
  ``torch.topk`` as in the reference.
* ``load_and_register_custom(ptx, entry_name, slot)`` (gpuos_ext.cpp:1079-1088): PTX that
  defines ``extern "C" __device__ void entry_name(const Task&)`` is linked into the worker
  and the function's device address goes into ``slot``.

Importing this module without the compiled extension raises ImportError: there is no CPU
or PyTorch fallback for the runtime itself.
"""
from __future__ import annotations

import re
import threading

import torch  # noqa: F401  (loads libtorch / libc10 before the binding)

try:
    from . import _gpuos_ext as _ext
except ImportError as e:  # pragma: no cover - exercised only on broken installs
    raise ImportError(
        "gpuos_b200 extension not built; run `python -m gpuos_b200.build` "
        f"(original error: {e})") from e

from ._gpuos_ext import *  # noqa: F401,F403  (init, submit_add, flush, ...)

_reg_lock = threading.Lock()
_slots: dict[tuple[int, str], int] = {}

# Expressions whose meaning is exactly a built-in operator (whitespace-insensitive).
_EXACT_EXPR = {
    "(A+B)": _ext.EW_ADD,
    "(A-B)": _ext.EW_SUB,
    "(A*B)": _ext.EW_MUL,
    "(A/B)": _ext.EW_DIV,
    "powf(A,B)": _ext.EW_POW,
    "(A)": _ext.EW_COPY,
    "expf(A)": _ext.EW_EXP,
    "logf(A)": _ext.EW_LOG,
    "sqrtf(A)": _ext.EW_SQRT,
    "fabsf(A)": _ext.EW_ABS,
    "tanhf(A)": _ext.EW_TANH,
    "sinf(A)": _ext.EW_SIN,
    "cosf(A)": _ext.EW_COS,
    "1.f/(1.f+expf(-A))": _ext.EW_SIGMOID,
}


def _norm(expr: str) -> str:
    return re.sub(r"\s+", "", expr)


def _device_key(device=None) -> int:
    if device is None:
        return torch.cuda.current_device()
    return torch.device(device).index if not isinstance(device, int) else device


def register_elementwise(key: str, expr: str, arity: int, *, slot: int = -1, device=None,
                         backend: str = "auto") -> int:
    """Register an element-wise operator ``R = expr(A[, B])`` and return its table slot.

    backend: "auto" (a built-in operator when ``expr`` means exactly one and no slot is given,
    otherwise NVRTC), "nvrtc", "builtin" or "interp" (the worker's expression interpreter)."""
    if arity not in (1, 2):
        raise ValueError("arity must be 1 or 2")
    if backend not in ("auto", "nvrtc", "builtin", "interp"):
        raise ValueError("backend must be 'auto', 'nvrtc', 'builtin' or 'interp'")
    dev = _device_key(device)
    with _reg_lock:
        hit = _slots.get((dev, key))
        if hit is not None and slot < 0:
            return hit
        op = _EXACT_EXPR.get(_norm(expr))
        if backend == "builtin" or (backend == "auto" and op is not None and slot < 0):
            if op is None:
                raise ValueError(f"{expr!r} is not a built-in operator")
            s = _ext.register_builtin("elementwise", op, device=dev)
            if slot >= 0:
                _ext.set_slot(slot, _ext.get_slot(s, device=dev), device=dev)
                s = slot
        elif backend == "interp":
            s = _ext.register_expr(key, expr, arity, slot, device=dev)
        else:
            s = _ext.register_jit(expr, arity, slot, device=dev)
        _slots[(dev, key)] = s
        return s


def register_reduce(key: str, op_name: str, *, device=None) -> int:
    """Register a sum/mean reduction operator and return its table slot."""
    names = {"sum": _ext.RED_SUM, "mean": _ext.RED_MEAN}
    if op_name not in names:
        raise ValueError(f"unknown reduction {op_name!r} (sum, mean)")
    dev = _device_key(device)
    with _reg_lock:
        hit = _slots.get((dev, key))
        if hit is not None:
            return hit
        s = _ext.register_builtin("reduce", names[op_name], device=dev)
        _slots[(dev, key)] = s
        return s


TOPK_SLOT = 42  # gpuos_ext.cpp:1052


def register_topk(key: str, k: int, dim: int, largest: bool, sorted: bool) -> int:  # noqa: A002
    return TOPK_SLOT


def submit_topk(slot: int, x, values, indices, k: int, dim: int, largest: bool, sorted: bool) -> None:  # noqa: A002
    """Top-k of x along dim into values/indices, complete when this call returns (the reference
    runs torch::topk on the calling thread, gpuos_ext.cpp:1050-1071).  Along the last dimension
    of a contiguous float tensor with k <= 256 it runs on the persistent worker (sorted, ties to
    the lower position); other cases use torch.topk as the reference does."""
    nd = x.dim()
    d = dim + nd if dim < 0 else dim
    if (nd >= 1 and d == nd - 1 and x.is_cuda and x.is_contiguous() and x.numel() > 0
            and x.dtype in (torch.float32, torch.float16, torch.bfloat16) and 1 <= k <= min(x.shape[-1], 256)
            and values.is_contiguous() and indices.is_contiguous() and values.dtype == x.dtype
            and indices.dtype == torch.int64 and tuple(values.shape) == tuple(x.shape[:-1]) + (k,)
            and tuple(indices.shape) == tuple(values.shape)):
        n = x.shape[-1]
        _ext.submit_topk_rows(x.view(-1, n), values.view(-1, k), indices.view(-1, k), k, bool(largest))
        _ext.flush(True, device=x.device.index)
        return
    v, i = torch.topk(x, k, dim, largest, sorted)
    values.copy_(v)
    indices.copy_(i)


def load_and_register_custom(ptx: str, entry_name: str, slot: int) -> int:
    """Link PTX that defines ``extern "C" __device__ void entry_name(const Task&)`` (the
    reference operator ABI) into the worker and install the function in ``slot``.  The
    reference stores the host handle of a kernel in the slot instead (gpuos_ext.cpp:347-354,
    1079-1088)."""
    return _ext.load_custom(ptx, entry_name, slot)


def reset_registry() -> None:
    """Forget cached key -> slot registrations (after shutdown)."""
    with _reg_lock:
        _slots.clear()


_shutdown_native = _ext.shutdown


def shutdown(device=None) -> None:  # noqa: F811
    _shutdown_native(device=device)
    if device is None:
        reset_registry()
