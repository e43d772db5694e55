"""Run-time operator compilation without a device: NVRTC compiles an element-wise operator for
sm_100a as relocatable code within the worker's register budget and nvJitLink links it with the
worker's relocatable code (the step gpuos_rt_register_jit runs before it loads the module).
Reference: pytorch_ext/gpuos_ext.cpp:316-345 (NVRTC), :814-868 (operator source)."""
import pytest

from gpuos_b200 import _gpuos_ext as ext


def test_toolkit_nvrtc_is_used():
    # the toolkit's NVRTC (the one the worker was built with), not the older copy PyTorch loads
    assert ext.jit_nvrtc_version() >= 12090


@pytest.mark.parametrize("expr,arity", [
    ("A * B + 1.0f", 2),
    ("A > 0.f ? A : 0.01f * A", 1),
    ("expf(-A * A) / (1.f + fabsf(A)) + powf(A, 2.0f) + tanhf(A)", 1),
])
def test_expression_compiles_and_links_with_the_worker(expr, arity):
    assert ext.jit_check_expr(expr, arity) > 1 << 20   # the linked image carries the whole worker


@pytest.mark.parametrize("expr,arity,err,match", [
    ("A;}", 1, ValueError, "outside C expression syntax"),
    ('A + "x"', 1, ValueError, "outside C expression syntax"),
    ("B + 1.f", 1, RuntimeError, "identifier \"B\" is undefined"),
    ("frobf(A)", 1, RuntimeError, "frobf"),
    ("A + B", 3, ValueError, "arity"),
])
def test_bad_expressions_are_rejected(expr, arity, err, match):
    with pytest.raises(err, match=match):
        ext.jit_check_expr(expr, arity)


def test_compile_outputs():
    src = 'struct Task; extern "C" __device__ void my_op(const Task& t) {}'
    ptx = ext.jit_compile(src, ptx=True)
    cubin = ext.jit_compile(src)
    assert isinstance(ptx, str) and len(ptx) > 0
    assert isinstance(cubin, bytes) and len(cubin) > 0
    with pytest.raises(RuntimeError, match="NVRTC"):
        ext.jit_compile("this is not CUDA")
