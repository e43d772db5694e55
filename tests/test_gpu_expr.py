"""Expression operators on the device (register_elementwise with expressions that are not a
built-in operator; pytorch_ext/gpuos_ext.cpp:814-896): results against PyTorch, an expression
operator switched into slot 0 while Tasks flow (test/online_switch.cpp), and registration
while the persistent worker keeps running."""
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
    s_leaky = rt.register_elementwise("x_leaky", "A > 0.f ? A : 0.1f * A", 1)
    s_maxh = rt.register_elementwise("x_maxhalf", "fmaxf(A, B) * 0.5f", 2)
    s_sqb = rt.register_elementwise("x_sq_plus", "A * A + B", 2)
    s_sig = rt.register_elementwise("x_sigmoid_like", "1.f / (1.f + expf(-A)) - B", 2)
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
    # expf (a few ulp) and three roundings, bounded on the operands' scale
    assert bool((err <= 2.0 ** -20 * (sig.abs() + b.double().abs())).all())
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
    s = rt.register_elementwise("x_mul_for_switch", "(A) * (B)", 2)  # not a built-in spelling
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
    s = rt.register_elementwise("x_while_running", "A * 3.f - B", 2)
    rt.submit_binary(s, a, a, o)
    rt.flush(sync=True)
    assert rt.launches() == launches            # the worker that was running did the work
    assert same_bits(o.cpu(), a.cpu() * 3.0 - a.cpu())


def test_malformed_expression_raises(rt):
    with pytest.raises(ValueError, match="unknown function"):
        rt.register_elementwise("x_bad", "frobf(A)", 1)
