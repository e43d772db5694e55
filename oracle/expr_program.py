"""CPU evaluator of expression-operator programs (test infrastructure only, never the product
path): restates the stack machine of gpuos_b200/csrc/device/expr.cuh in numpy float32 so that
CPU tests can check what the host compiler (gpuos_expr_compile) emits for an expression.

The expressions themselves follow the reference's elementwise operator sources
(pytorch_ext/gpuos_ext.cpp:814-868, `R = expr(A[, B])`, expressions from
pytorch_ext/scheduler.py:145-153, 192-205, 244-290)."""
from __future__ import annotations

import math

import numpy as np

OPS = ["END", "A", "B", "CONST", "NEG", "NOT", "ADD", "SUB", "MUL", "DIV", "LT", "LE", "GT", "GE", "EQ",
       "NE", "AND", "OR", "SELECT", "EXP", "LOG", "LOG1P", "EXPM1", "SQRT", "RSQRT", "ABS", "TANH", "SIN",
       "COS", "TAN", "ERF", "FLOOR", "CEIL", "TRUNC", "ROUND", "EXP2", "LOG2", "LOG10", "SINH", "COSH",
       "ASIN", "ACOS", "ATAN", "MIN", "MAX", "POW", "FMOD", "ATAN2", "COPYSIGN"]
PROG_DT = np.dtype([("code", "u1", 64), ("imm", "<f4", 64), ("len", "<i4"), ("arity", "<i4"),
                    ("depth", "<i4"), ("pad", "<i4")])
assert PROG_DT.itemsize == 336

f32 = np.float32
_erf = np.vectorize(math.erf, otypes=[np.float64])


def _round_half_away(x):
    return np.where(x >= 0, np.floor(x + f32(0.5)), np.ceil(x - f32(0.5))).astype(f32)


UNARY = {
    "NEG": lambda x: -x, "NOT": lambda x: (x == 0).astype(f32), "EXP": np.exp, "LOG": np.log,
    "LOG1P": np.log1p, "EXPM1": np.expm1, "SQRT": np.sqrt, "RSQRT": lambda x: f32(1) / np.sqrt(x),
    "ABS": np.abs, "TANH": np.tanh, "SIN": np.sin, "COS": np.cos, "TAN": np.tan,
    "ERF": lambda x: _erf(x.astype(np.float64)).astype(f32), "FLOOR": np.floor, "CEIL": np.ceil,
    "TRUNC": np.trunc, "ROUND": _round_half_away, "EXP2": np.exp2, "LOG2": np.log2, "LOG10": np.log10,
    "SINH": np.sinh, "COSH": np.cosh, "ASIN": np.arcsin, "ACOS": np.arccos, "ATAN": np.arctan,
}
BINARY = {
    "ADD": np.add, "SUB": np.subtract, "MUL": np.multiply, "DIV": np.divide,
    "LT": lambda x, y: (x < y).astype(f32), "LE": lambda x, y: (x <= y).astype(f32),
    "GT": lambda x, y: (x > y).astype(f32), "GE": lambda x, y: (x >= y).astype(f32),
    "EQ": lambda x, y: (x == y).astype(f32), "NE": lambda x, y: (x != y).astype(f32),
    "AND": lambda x, y: ((x != 0) & (y != 0)).astype(f32), "OR": lambda x, y: ((x != 0) | (y != 0)).astype(f32),
    "MIN": np.fmin, "MAX": np.fmax, "POW": np.power, "FMOD": np.fmod, "ATAN2": np.arctan2,
    "COPYSIGN": np.copysign,
}


def disassemble(prog: bytes) -> list[str]:
    p = np.frombuffer(prog, dtype=PROG_DT)[0]
    out = []
    for i in range(int(p["len"])):
        name = OPS[p["code"][i]]
        out.append(f"{name}({float(p['imm'][i])!r})" if name == "CONST" else name)
    return out


def evaluate(prog: bytes, A: np.ndarray, B: np.ndarray | None = None) -> np.ndarray:
    """Run a program over float32 arrays A (and B) element-wise, as the worker does."""
    p = np.frombuffer(prog, dtype=PROG_DT)[0]
    A = np.asarray(A, dtype=f32)
    B = np.zeros_like(A) if B is None else np.asarray(B, dtype=f32)
    st: list[np.ndarray] = []
    with np.errstate(all="ignore"):
        for i in range(int(p["len"])):
            name = OPS[p["code"][i]]
            if name == "A":
                st.append(A)
            elif name == "B":
                st.append(B)
            elif name == "CONST":
                st.append(np.full_like(A, p["imm"][i]))
            elif name == "SELECT":
                y, x, c = st.pop(), st.pop(), st.pop()
                st.append(np.where(c != 0, x, y).astype(f32))
            elif name in BINARY:
                y, x = st.pop(), st.pop()
                st.append(np.asarray(BINARY[name](x, y), dtype=f32))
            else:
                st.append(np.asarray(UNARY[name](st.pop()), dtype=f32))
    assert len(st) == 1
    return st[0]
