"""Expression operators run by the worker's interpreter (register_elementwise(...,
backend="interp"); the reference compiles them with NVRTC, pytorch_ext/gpuos_ext.cpp:814-896):
results against PyTorch, single transcendental functions within 1 ulp of the float64 value, an
expression operator switched into slot 0 while Tasks flow (test/online_switch.cpp), and
registration while the persistent worker keeps running."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle.reference_semantics import same_bits, ulp_diff

pytestmark = pytest.mark.gpu
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_known_answers.json")))


def digest(t):
    return hashlib.sha256(t.cpu().numpy().astype(np.float32).tobytes()).hexdigest()


def test_expression_operators_match_torch(rt):
    g = torch.Generator().manual_seed(7)
    a = torch.randn(300, 257, generator=g)
    b = torch.randn(257, generator=g)                       # broadcast along dim 0
    s_leaky = rt.register_elementwise("x_leaky", "A > 0.f ? A : 0.1f * A", 1, backend="interp")
    s_maxh = rt.register_elementwise("x_maxhalf", "fmaxf(A, B) * 0.5f", 2, backend="interp")
    s_sqb = rt.register_elementwise("x_sq_plus", "A * A + B", 2, backend="interp")
    s_sig = rt.register_elementwise("x_sigmoid_like", "1.f / (1.f + expf(-A)) - B", 2, backend="interp")
    assert len({s_leaky, s_maxh, s_sqb, s_sig}) == 4 and min(s_leaky, s_maxh, s_sqb, s_sig) >= 20
    outs = [torch.empty(300, 257, device="cuda") for _ in range(4)]
    ad, bd = a.cuda(), b.cuda()
    rt.submit_unary(s_leaky, ad, outs[0])
    rt.submit_binary(s_maxh, ad, bd, outs[1])
    rt.submit_binary(s_sqb, ad, bd, outs[2])
    rt.submit_binary(s_sig, ad, bd, outs[3])
    rt.flush(sync=True)
    assert same_bits(outs[0].cpu(), torch.where(a > 0, a, a * 0.1))
    assert same_bits(outs[1].cpu(), torch.maximum(a, b) * 0.5)
    assert same_bits(outs[2].cpu(), a * a + b)              # two roundings, as the program runs them
    sig = 1.0 / (1.0 + torch.exp(-a.double()))
    err = (outs[3].cpu().double() - (sig - b.double())).abs()
    # four float roundings (exp, add, divide, subtract), each at most half an ulp of its result
    assert bool((err <= 2.0 ** -23 * (2 * sig.abs() + b.double().abs())).all())
    assert int(ulp_diff(outs[0].cpu(), torch.where(a > 0, a, a * 0.1)).max()) == 0
    # 16-bit storage: computed in float32, rounded once on store
    ah, bh = a.to(torch.bfloat16), b.to(torch.bfloat16)
    o = torch.empty(300, 257, device="cuda", dtype=torch.bfloat16)
    rt.submit_binary(s_maxh, ah.cuda(), bh.cuda(), o)
    rt.flush(sync=True)
    assert same_bits(o.cpu(), (torch.maximum(ah.float(), bh.float()) * 0.5).to(torch.bfloat16))


def test_expression_operator_switched_into_slot0_online(rt):
    g = GOLD["online_switch"]
    n = g["n"]
    i = torch.arange(n, dtype=torch.float32)
    A = (0.5 * i).cuda()
    B = (1.0 + (torch.arange(n) % 5).float()).cuda()
    c_add, c_mul, c_back = (torch.zeros_like(A) for _ in range(3))
    s = rt.register_elementwise("x_mul_for_switch", "(A) * (B)", 2, backend="interp")  # not a built-in spelling
    x_mul = rt.get_slot(s)
    add_addr = rt.get_slot(0)
    try:
        for _ in range(64):
            rt.submit_binary(0, A, B, c_add)
        rt.flush(sync=True)
        rt.set_slot(0, x_mul)                   # online switch: slot 0 now runs the expression
        for _ in range(64):
            rt.submit_binary(0, A, B, c_mul)
        rt.flush(sync=True)
    finally:
        rt.set_slot(0, add_addr)                # roll back
    for _ in range(8):
        rt.submit_binary(0, A, B, c_back)
    rt.flush(sync=True)
    assert digest(c_add) == g["c_add_sha256"]
    assert digest(c_mul) == g["c_mul_sha256"]
    assert digest(c_back) == g["c_add_sha256"]


def test_registration_does_not_stop_the_worker(rt):
    a = torch.randn(1 << 16, device="cuda")
    o = torch.empty_like(a)
    rt.submit_add(a, a, o)
    rt.flush(sync=True)
    launches = rt.launches()
    s = rt.register_elementwise("x_while_running", "A * 3.f - B", 2, backend="interp")
    rt.submit_binary(s, a, a, o)
    rt.flush(sync=True)
    assert rt.launches() == launches            # the worker that was running did the work
    assert same_bits(o.cpu(), a.cpu() * 3.0 - a.cpu())


def test_malformed_expression_raises(rt):
    with pytest.raises(ValueError, match="unknown function"):
        rt.register_elementwise("x_bad", "frobf(A)", 1, backend="interp")


FUNCS = [  # (expression, float64 reference, input)
    ("expf(A)", torch.exp, lambda x: x * 4),
    ("logf(A)", torch.log, lambda x: x.abs() + 1e-3),
    ("log1pf(A)", torch.log1p, lambda x: x.abs()),
    ("expm1f(A)", torch.expm1, lambda x: x),
    ("tanhf(A)", torch.tanh, lambda x: x * 3),
    ("sinf(A)", torch.sin, lambda x: x * 3),
    ("cosf(A)", torch.cos, lambda x: x * 3),
    ("erff(A)", torch.erf, lambda x: x),
    ("sinhf(A)", torch.sinh, lambda x: x * 2),
    ("atanf(A)", torch.atan, lambda x: x * 5),
    ("powf(A, B)", torch.pow, lambda x: x.abs() + 0.1),
]


@pytest.mark.parametrize("expr,fn,dom", FUNCS, ids=[f[0] for f in FUNCS])
def test_interpreter_functions_within_one_ulp(rt, expr, fn, dom):
    g = torch.Generator().manual_seed(11)
    x = dom(torch.randn(1 << 15, generator=g))
    y = torch.rand(1 << 15, generator=g) * 1.5 + 0.5
    two = "B" in expr
    s = rt.register_elementwise("xi_" + expr, expr, 2 if two else 1, backend="interp")
    o = torch.empty(1 << 15, device="cuda")
    if two:
        rt.submit_binary(s, x.cuda(), y.cuda(), o)
        ref = fn(x.double(), y.double()).float()
    else:
        rt.submit_unary(s, x.cuda(), o)
        ref = fn(x.double()).float()
    rt.flush(sync=True)
    assert int(ulp_diff(o.cpu(), ref).max()) <= 1
