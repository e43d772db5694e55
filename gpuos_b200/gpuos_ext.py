"""gpuos_ext — the reference's Python module API (pytorch_ext/gpuos_ext.cpp:1093-1142) on the
B200 runtime.

Every function of the reference module is here with the same name, defaults and argument
meaning.  The compiled binding (``_gpuos_ext``) provides the hot calls directly; this file
adds the registry-style calls that the reference implements next to them:

* ``register_elementwise(key, expr, arity)`` (gpuos_ext.cpp:870-881): expressions with
  the exact semantics of a built-in operator map to that operator's reference-ABI device
  function; any other C float expression is compiled on the host into a program for the
  worker's expression interpreter (``register_expr``), so registering never loads a module
  next to the running worker.
* ``register_reduce(key, op_name)`` (gpuos_ext.cpp:1003-1014): built-in sum/mean.
* ``register_topk`` / ``submit_topk`` (gpuos_ext.cpp:1050-1071): slot 42; values are
  produced by ``torch.topk`` as in the reference (top-k is not on the batched path).
* ``load_and_register_custom(ptx, entry_name, slot)`` (gpuos_ext.cpp:1079-1088): not
  provided; raises NotImplementedError.

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


def register_elementwise(key: str, expr: str, arity: int, *, slot: int = -1, device=None) -> int:
    """Register an element-wise operator ``R = expr(A[, B])`` and return its table slot."""
    if arity not in (1, 2):
        raise ValueError("arity must be 1 or 2")
    dev = _device_key(device)
    with _reg_lock:
        hit = _slots.get((dev, key))
        if hit is not None and slot < 0:
            return hit
        op = _EXACT_EXPR.get(_norm(expr))
        if op is not None and slot < 0:
            s = _ext.register_builtin("elementwise", op, device=dev)
        else:
            s = _ext.register_expr(key, expr, arity, slot, device=dev)
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
    v, i = torch.topk(x, k, dim, largest, sorted)
    values.copy_(v)
    indices.copy_(i)


def load_and_register_custom(ptx: str, entry_name: str, slot: int) -> None:
    """Not provided.  Calling an operator of a separately loaded module from the persistent
    worker hung the worker on B200 in this build's tests, so operators are not injected as
    machine code; use ``register_elementwise`` with an expression instead."""
    raise NotImplementedError("custom PTX operators are not supported; register an expression with "
                              "register_elementwise instead")


def reset_registry() -> None:
    """Forget cached key -> slot registrations (after shutdown)."""
    with _reg_lock:
        _slots.clear()


_shutdown_native = _ext.shutdown


def shutdown(device=None) -> None:  # noqa: F811
    _shutdown_native(device=device)
    if device is None:
        reset_registry()
