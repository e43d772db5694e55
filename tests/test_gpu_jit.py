"""Operators compiled at run time by NVRTC for sm_100a and linked into the worker
(register_elementwise / load_and_register_custom; pytorch_ext/gpuos_ext.cpp:316-363, 814-881,
1079-1088).

The reference's known answers are reproduced with an NVRTC-compiled multiply installed in slot 0
(test/online_switch.cpp:170-228) and in physical slot 1 behind the alias table with a rollback
(test/dual_slot_switch.cpp:139-168).  The checks run in a child process under a time limit; the
last test installs an operator in the session runtime, so every later test file runs on the
linked worker module."""
import json
import os
import subprocess
import sys
import textwrap

import pytest
import torch

from oracle.reference_semantics import same_bits, ulp_diff

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent(r'''
    import hashlib, json, os, time
    import numpy as np, torch
    from gpuos_b200 import gpuos_ext as g
    from oracle.reference_semantics import same_bits, ulp_diff

    GOLD = json.load(open(os.path.join("tests", "golden", "reference_known_answers.json")))
    def digest(t):
        return hashlib.sha256(t.cpu().numpy().astype(np.float32).tobytes()).hexdigest()
    def run(slot, a, b, out, count):
        for _ in range(count):
            g.submit_binary(slot, a, b, out)
        g.flush(sync=True)

    g.init(4096, 256)
    g.set_device_wait_ms(2000)
    x = torch.randn(1 << 16, device="cuda"); o = torch.empty_like(x)
    g.submit_add(x, x, o); g.flush(sync=True)
    assert torch.equal(o.cpu(), x.cpu() * 2)
    assert g.jit_ops() == 0

    # 1. an expression compiled by NVRTC: bit-exact arithmetic, broadcast, 16-bit storage
    t0 = time.time()
    s1 = g.register_elementwise("j_fma_free", "A * B + 1.0f", 2)
    t_install = time.time() - t0
    assert s1 >= 20 and g.jit_ops() == 1
    a = torch.randn(300, 257); b = torch.randn(257)
    out = torch.empty(300, 257, device="cuda")
    g.submit_binary(s1, a.cuda(), b.cuda(), out); g.flush(sync=True)
    assert same_bits(out.cpu(), a * b + 1.0), "A*B+1"
    ah, bh = a.to(torch.float16), b.to(torch.float16)
    oh = torch.empty(300, 257, device="cuda", dtype=torch.float16)
    g.submit_binary(s1, ah.cuda(), bh.cuda(), oh); g.flush(sync=True)
    assert same_bits(oh.cpu(), (ah.float() * bh.float() + 1.0).to(torch.float16)), "f16"

    # 2. batched requests on the linked worker
    A = torch.randn(64, 4096, device="cuda"); B = torch.randn(64, 4096, device="cuda")
    O = torch.empty_like(A)
    for i in range(64):
        (g.submit_add if i % 2 == 0 else g.submit_mul)(A[i], B[i], O[i])
    g.flush(sync=True)
    ref = torch.where((torch.arange(64) % 2 == 0)[:, None], A.cpu() + B.cpu(), A.cpu() * B.cpu())
    assert same_bits(O.cpu(), ref), "batched after install"

    # 3. online switch of slot 0 to an NVRTC multiply (test/online_switch.cpp)
    go = GOLD["online_switch"]; n = go["n"]
    i = torch.arange(n, dtype=torch.float32)
    A1 = (0.5 * i).cuda(); B1 = (1.0 + (torch.arange(n) % 5).float()).cuda()
    c_add, c_mul, c_back = (torch.zeros_like(A1) for _ in range(3))
    add_addr = g.get_slot(0)
    run(0, A1, B1, c_add, 128)
    g.register_elementwise("op_mul", "A * B", 2, slot=0, backend="nvrtc")   # slot 0 now multiplies
    run(0, A1, B1, c_mul, 128)
    g.set_slot(0, add_addr)                                                # roll back
    run(0, A1, B1, c_back, 8)
    assert digest(c_add) == go["c_add_sha256"], "online add"
    assert digest(c_mul) == go["c_mul_sha256"], "online mul"
    assert digest(c_back) == go["c_add_sha256"], "online rollback"

    # 4. dual-slot switch and rollback through the alias table (test/dual_slot_switch.cpp)
    gd = GOLD["dual_slot"]; n = gd["n"]
    i = torch.arange(n, dtype=torch.float32)
    A2 = (0.3 * i).cuda(); B2 = (2.0 + (torch.arange(n) % 9).float()).cuda()
    c1, c2, c3 = (torch.zeros_like(A2) for _ in range(3))
    mul1 = g.get_slot(1)
    run(0, A2, B2, c1, 96)
    g.register_elementwise("op_mul_phys1", "B * A", 2, slot=1, backend="nvrtc")  # JIT mul -> slot 1
    g.set_alias(0, 1)
    run(0, A2, B2, c2, 96)
    g.set_alias(0, 0)
    run(0, A2, B2, c3, 96)
    g.set_slot(1, mul1)
    assert digest(c1) == gd["c1_sha256"] and digest(c2) == gd["c2_sha256"] and digest(c3) == gd["c3_sha256"], "dual"

    # 5. custom PTX through the fixed load_and_register_custom
    src = """
    struct TR { void* data; int dtype; int ndim; long long sizes[8]; long long strides[8]; };
    struct Task { int op; int flags; int ndim; long long numel; int rrank; int r_axes[8]; int r_keepdim;
                  TR in0; TR in1; TR out0; };
    extern "C" __device__ void triple_plus_one(const Task& t) {
      const float* a = (const float*)t.in0.data; float* o = (float*)t.out0.data;
      for (long long i = threadIdx.x; i < t.numel; i += blockDim.x) o[i] = a[i] * 3.0f + 1.0f;
    }
    """
    ptx = g.jit_compile(src, ptx=True)
    s5 = g.load_and_register_custom(ptx, "triple_plus_one", -1)
    z = torch.randn(5000); oz = torch.empty(5000, device="cuda")
    g.submit_unary(s5, z.cuda(), oz); g.flush(sync=True)
    assert same_bits(oz.cpu(), z * 3.0 + 1.0), "custom ptx"

    # 6. operators installed earlier keep working after later installs (table carried over)
    g.submit_binary(s1, a.cuda(), b.cuda(), out); g.flush(sync=True)
    assert same_bits(out.cpu(), a * b + 1.0), "carried over"
    si = g.register_elementwise("j_interp_after", "A * 2.f - B", 2, backend="interp")
    g.submit_binary(si, a.cuda(), b.cuda(), out); g.flush(sync=True)
    assert same_bits(out.cpu(), a * 2.0 - b), "interpreter on the linked module"
    assert g.jit_ops() == 4

    # 7. a malformed expression is an error, the runtime keeps working
    try:
        g.register_elementwise("j_bad", "frobf(A)", 1)
        raise SystemExit("expected a compile error")
    except RuntimeError as e:
        assert "frobf" in str(e), str(e)
    g.submit_mul(x, x, o); g.flush(sync=True)
    assert torch.equal(o.cpu(), x.cpu() * x.cpu())
    g.shutdown()
    print("JIT-OK install_s=%.2f" % t_install)
''')


def test_nvrtc_operators_in_child_process():
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    assert "JIT-OK" in r.stdout


FUNCS = [  # (expression, float64 reference, input)
    ("expf(A)", torch.exp, lambda x: x * 4),
    ("logf(A)", torch.log, lambda x: x.abs() + 1e-3),
    ("tanhf(A)", torch.tanh, lambda x: x * 3),
    ("sinf(A) * cosf(A)", lambda x: torch.sin(x).float().double() * torch.cos(x).float().double(), lambda x: x * 3),
    ("powf(A, B)", torch.pow, lambda x: x.abs() + 0.1),
]


def test_nvrtc_functions_in_session_runtime(rt):
    """Installs operators in the session runtime (every later test file then runs on the linked
    worker).  A single transcendental is within 1 ulp of the float64 value; a product of two is
    the product of the two rounded values, rounded once."""
    g = torch.Generator().manual_seed(5)
    for expr, fn, dom in FUNCS:
        x = dom(torch.randn(1 << 15, generator=g))
        y = torch.rand(1 << 15, generator=g) * 1.5 + 0.5
        two = "B" in expr
        s = rt.register_elementwise("js_" + expr, expr, 2 if two else 1, backend="nvrtc")
        o = torch.empty(1 << 15, device="cuda")
        if two:
            rt.submit_binary(s, x.cuda(), y.cuda(), o)
            ref = fn(x.double(), y.double()).float()
        else:
            rt.submit_unary(s, x.cuda(), o)
            ref = fn(x.double()).float()
        rt.flush(sync=True)
        assert int(ulp_diff(o.cpu(), ref).max()) <= 1, expr
    assert rt.jit_ops() >= len(FUNCS)
    a = torch.randn(1 << 20, device="cuda")
    out = torch.empty_like(a)
    rt.submit_mul(a, a, out)
    rt.flush(sync=True)
    assert same_bits(out.cpu(), a.cpu() * a.cpu())
