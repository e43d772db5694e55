"""Pin the oracle: the reference's known answers (tests/golden) reproduced by the
numpy restatement, and the documented reference-vs-PyTorch divergences."""
import hashlib
import json
import os

import numpy as np
import torch

from oracle.reference_semantics import (EW, BINARY, bf16_round, ew_torch, fill_tensorref,
                                        linear_to_offset, op_batch, reduce_task, reduce_torch,
                                        same_bits, st_from_float, ulp_diff)

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_known_answers.json")))


def digest(x):
    return hashlib.sha256(np.ascontiguousarray(x, dtype=np.float32).tobytes()).hexdigest()


def test_test_py_known_answer():
    # test/test.py:1-13: add, mul, sub, div into c in one flush -> c = a / b
    a = np.arange(16, dtype=np.float32)
    b = np.full(16, 2.0, np.float32)
    c = np.zeros(16, np.float32)
    op_batch([{"op": k, "a": a, "b": b, "out": c, "numel": 16} for k in range(4)])
    assert c[:4].tolist() == GOLD["test_py"]["c_head4"] == [0.0, 0.5, 1.0, 1.5]
    assert c.tolist() == GOLD["test_py"]["c"]


def test_switch_known_answers():
    g = GOLD["online_switch"]
    n = g["n"]
    i = np.arange(n, dtype=np.float32)
    A = (np.float32(0.5) * i).astype(np.float32)
    B = (1 + (np.arange(n) % 5)).astype(np.float32)
    assert digest(A + B) == g["c_add_sha256"] and digest(A * B) == g["c_mul_sha256"]
    # the reference spot check: 5 elements within 1e-4
    assert np.allclose((A + B)[:5], g["c_add_head"][:5], atol=1e-4)
    g = GOLD["dual_slot"]
    A = (np.float32(0.3) * i).astype(np.float32)
    B = (2 + (np.arange(n) % 9)).astype(np.float32)
    assert digest(A + B) == g["c1_sha256"] == g["c3_sha256"]
    assert digest(A * B) == g["c2_sha256"]


def test_full_sync_known_answer():
    g = GOLD["full_sync"]
    rng = np.random.default_rng(g["seed"])
    a = rng.standard_normal(g["n"]).astype(np.float32)
    b = rng.standard_normal(g["n"]).astype(np.float32)
    assert digest(a) == g["a_sha256"] and digest(a + b) == g["c_sha256"]


def test_linear_to_offset_and_broadcast_fill():
    # out [2,3,4], input [3,1] -> right-aligned sizes [1,3,1], strides [0,1,0]
    sizes, strides = fill_tensorref([3, 1], [1, 1], [2, 3, 4])
    assert sizes == [1, 3, 1] and strides == [0, 1, 0]
    # The reference decodes with the input's own sizes: for out [2,3,4] and an input
    # [2,1,4] (broadcast in the middle dim) the output element (1,1,0) = linear 16 maps to
    # offset 0 instead of 4 (documented divergence; the runtime decodes with output sizes).
    assert linear_to_offset([2, 1, 4], [4, 0, 1], 16) == 0
    assert linear_to_offset([2, 3, 4], [4, 0, 1], 16) == 4


def test_reference_div_by_zero_diverges_from_torch():
    a = np.array([1.0, -1.0, 0.0], np.float32)
    b = np.zeros(3, np.float32)
    c = np.zeros(3, np.float32)
    op_batch([{"op": 3, "a": a, "b": b, "out": c, "numel": 3}])
    assert c.tolist() == [0.0, 0.0, 0.0]  # reference rule
    t = ew_torch(EW["DIV"], torch.from_numpy(a), torch.from_numpy(b))
    assert torch.isinf(t[0]) and torch.isinf(t[1]) and torch.isnan(t[2])  # PyTorch rule (followed)


def test_bf16_rounding_matches_torch():
    x = torch.randn(1 << 16) * 100
    assert torch.equal(torch.from_numpy(bf16_round(x.numpy())), x.to(torch.bfloat16).float())
    assert torch.equal(torch.from_numpy(st_from_float(x.numpy(), 1)), x.half().float())


def test_reduce_oracles_agree():
    x = torch.randn(7, 33, 5)
    for axes, keep in [((2,), False), ((1, 2), True), ((0,), False)]:
        a = torch.from_numpy(reduce_task(x.numpy(), axes, keep, mean=True))
        b = reduce_torch(x, axes, keep, mean=True)
        assert torch.allclose(a, b, rtol=1e-5, atol=1e-6)


def test_ew_oracle_covers_every_op_and_comparators():
    x = torch.randn(64)
    y = torch.rand(64) + 0.5
    for name, op in EW.items():
        r = ew_torch(op, x.abs() + 0.1 if name in ("LOG", "SQRT", "POW") else x,
                     y if op in BINARY else None, 0.1 if name != "CLAMP" else -0.5,
                     0.5 if name == "CLAMP" else 20.0)
        assert r.shape == x.shape
    assert same_bits(torch.tensor([float("nan"), 1.0]), torch.tensor([float("nan"), 1.0]))
    assert not same_bits(torch.tensor([0.0]), torch.tensor([-0.0]))
    assert int(ulp_diff(torch.tensor([1.0]), torch.tensor([1.0000001])).max()) == 1
