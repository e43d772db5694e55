"""Host compiler of expression operators (gpuos_expr_compile, no device): the expressions the
reference's scheduler emits (pytorch_ext/scheduler.py:145-153, 192-205, 244-290) compile, the
programs compute what the expressions say (checked with the CPU evaluator in oracle/), C
precedence holds, and malformed expressions are rejected with a message."""
import ctypes

import numpy as np
import pytest

from oracle.expr_program import disassemble, evaluate
from tests._items import LIB_PATH

f32 = np.float32


@pytest.fixture(scope="module")
def lib():
    l = ctypes.CDLL(LIB_PATH)
    l.gpuos_expr_compile.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
    l.gpuos_rt_last_error.restype = ctypes.c_char_p
    return l


def compile_expr(lib, expr, arity):
    buf = ctypes.create_string_buffer(336)
    rc = lib.gpuos_expr_compile(expr.encode(), arity, buf, 336)
    assert rc == 0, lib.gpuos_rt_last_error()
    return buf.raw


RNG = np.random.default_rng(3)
A = RNG.standard_normal(4096).astype(f32) * f32(3)
B = RNG.standard_normal(4096).astype(f32) * f32(3)
P = np.abs(A) + f32(0.1)

# (expression, arity, numpy reference, input for A)
CASES = [
    ("A > 0 ? A : 0", 1, lambda a, b: np.where(a > 0, a, f32(0)), A),
    ("1.f/(1.f+expf(-A))", 1, lambda a, b: f32(1) / (f32(1) + np.exp(-a)), A),
    ("tanhf(A)", 1, lambda a, b: np.tanh(a), A),
    ("logf(A)", 1, lambda a, b: np.log(a), P),
    ("sqrtf(A)", 1, lambda a, b: np.sqrt(a), P),
    ("fabsf(A)", 1, lambda a, b: np.abs(a), A),
    ("A*fminf(fmaxf(A/6.f+0.5f, 0.f), 1.f)", 1,
     lambda a, b: a * np.fmin(np.fmax(a / f32(6) + f32(0.5), f32(0)), f32(1)), A),
    ("A >= 0 ? A : 0.01f*A", 1, lambda a, b: np.where(a >= 0, a, f32(0.01) * a), A),
    ("A > 0 ? A : 1.0f*(expf(A)-1.f)", 1, lambda a, b: np.where(a > 0, a, f32(1) * (np.exp(a) - f32(1))), A),
    ("log1pf(expf(1.0f*A))/1.0f", 1, lambda a, b: np.log1p(np.exp(f32(1) * a)) / f32(1), A),
    ("(A > B ? A : B)", 2, lambda a, b: np.where(a > b, a, b), A),
    ("powf(A, B)", 2, lambda a, b: np.power(a, b), P),
    ("A - B * 2 + -A / 4e-1f", 2, lambda a, b: a - b * f32(2) + (-a) / f32(0.4), A),
    ("!(A < 0) && B != 0 || A == B", 2, lambda a, b: (((a >= 0) & (b != 0)) | (a == b)).astype(f32), A),
    ("(float)A * (float)(B)", 2, lambda a, b: a * b, A),
]


@pytest.mark.parametrize("expr,arity,ref,a", CASES)
def test_programs_compute_the_expression(lib, expr, arity, ref, a):
    prog = compile_expr(lib, expr, arity)
    with np.errstate(all="ignore"):
        want = ref(a, B).astype(f32)
        got = evaluate(prog, a, B if arity == 2 else None)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    np.testing.assert_allclose(got[ok], want[ok], rtol=2e-6, atol=0)


def test_c_precedence_and_shape_of_programs(lib):
    assert disassemble(compile_expr(lib, "A+B*2", 2)) == ["A", "B", "CONST(2.0)", "MUL", "ADD"]
    assert disassemble(compile_expr(lib, "A-B-1", 2)) == ["A", "B", "SUB", "CONST(1.0)", "SUB"]
    assert disassemble(compile_expr(lib, "A>0?A:B>0?B:0", 2)) == [
        "A", "CONST(0.0)", "GT", "A", "B", "CONST(0.0)", "GT", "B", "CONST(0.0)", "SELECT", "SELECT"]
    assert disassemble(compile_expr(lib, "-expf(A)", 1)) == ["A", "EXP", "NEG"]


@pytest.mark.parametrize("expr,arity,msg", [
    ("A +* B", 2, b"unexpected"), ("B", 1, b"one-operand"), ("foo(A)", 1, b"unknown function"),
    ("fmaxf(A)", 1, b"two arguments"), ("(A", 1, b"expected ')'"), ("A ? B", 2, b"expected ':'"),
    ("", 1, b"ends early"), ("A A", 1, b"unexpected"),
    ("+".join(["A"] * 40), 1, b"longer than"), ("A+(" * 20 + "A" + ")" * 20, 1, b"deeper than"),
])
def test_malformed_expressions_rejected(lib, expr, arity, msg):
    assert lib.gpuos_expr_compile(expr.encode(), arity, None, 0) == 1
    assert msg in lib.gpuos_rt_last_error()


def test_bad_arity(lib):
    assert lib.gpuos_expr_compile(b"A", 3, None, 0) == 1
