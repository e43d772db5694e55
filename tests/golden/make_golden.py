"""Regenerate tests/golden/reference_known_answers.json.

The reference ships no golden data files; its known answers are the expectations written
in its test programs.  This script restates those inputs and expectations and evaluates
them with the oracle's restatement of the reference semantics (sub-tasks of one flush run
in order, src/persistent_kernel.cu:81-112):

* test/online_switch.cpp:146-153, 219-228 — N = 1<<15, A[i] = 0.5 i, B[i] = 1 + (i % 5);
  128 op-0 Tasks with slot 0 = add -> C_add = A + B; slot 0 switched to a multiply ->
  C_mul = A * B; spot-checked on i < 5 with tolerance 1e-4.
* test/dual_slot_switch.cpp:127-128, 139-168 — A[i] = 0.3 i, B[i] = 2 + (i % 9); alias 0->0
  (add) -> C1, alias 0->1 (mul) -> C2, rollback 0->0 -> C3 = A + B.
* test/test.py:1-13 — a = arange(16), b = 2; add, mul, sub, div all into c, one flush:
  c = a / b, c[:4] = [0, 0.5, 1, 1.5].
* test_full_sync.py:40-124 — a, b ~ N(0,1) of 10000 (seeded here); add (async flush),
  mul (sync flush), 5 x add (sync flush); final c == a + b.

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.reference_semantics import op_batch  # noqa: E402


def digest(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x, dtype=np.float32).tobytes()).hexdigest()


def main() -> None:
    out = {}
    n = 1 << 15
    i = np.arange(n, dtype=np.float32)
    # online switch
    A = (np.float32(0.5) * i).astype(np.float32)
    B = (np.float32(1.0) + (np.arange(n) % 5).astype(np.float32)).astype(np.float32)
    c_add, c_mul = np.zeros(n, np.float32), np.zeros(n, np.float32)
    op_batch([{"op": 0, "a": A, "b": B, "out": c_add, "numel": n}])
    op_batch([{"op": 1, "a": A, "b": B, "out": c_mul, "numel": n}])
    out["online_switch"] = {
        "n": n, "a": "0.5*i", "b": "1+(i%5)", "tol": 1e-4,
        "c_add_head": c_add[:8].tolist(), "c_mul_head": c_mul[:8].tolist(),
        "c_add_sha256": digest(c_add), "c_mul_sha256": digest(c_mul)}
    # dual slot
    A = (np.float32(0.3) * i).astype(np.float32)
    B = (np.float32(2.0) + (np.arange(n) % 9).astype(np.float32)).astype(np.float32)
    c1, c2, c3 = (np.zeros(n, np.float32) for _ in range(3))
    op_batch([{"op": 0, "a": A, "b": B, "out": c1, "numel": n}])
    op_batch([{"op": 1, "a": A, "b": B, "out": c2, "numel": n}])
    op_batch([{"op": 0, "a": A, "b": B, "out": c3, "numel": n}])
    out["dual_slot"] = {
        "n": n, "a": "0.3*i", "b": "2+(i%9)", "tol": 1e-4,
        "c1_head": c1[:8].tolist(), "c2_head": c2[:8].tolist(), "c3_head": c3[:8].tolist(),
        "c1_sha256": digest(c1), "c2_sha256": digest(c2), "c3_sha256": digest(c3)}
    # test.py: four sub-tasks into one output, run in order
    a = np.arange(16, dtype=np.float32)
    b = np.full(16, 2.0, np.float32)
    c = np.zeros(16, np.float32)
    op_batch([{"op": k, "a": a, "b": b, "out": c, "numel": 16} for k in (0, 1, 2, 3)])
    out["test_py"] = {"a": "arange(16)", "b": "2", "c": c.tolist(), "c_head4": [0.0, 0.5, 1.0, 1.5]}
    # test_full_sync.py
    rng = np.random.default_rng(20240611)
    a = rng.standard_normal(10000).astype(np.float32)
    b = rng.standard_normal(10000).astype(np.float32)
    c = np.zeros(10000, np.float32)
    op_batch([{"op": 0, "a": a, "b": b, "out": c, "numel": 10000}])
    op_batch([{"op": 1, "a": a, "b": b, "out": c, "numel": 10000}])
    op_batch([{"op": 0, "a": a, "b": b, "out": c, "numel": 10000} for _ in range(5)])
    out["full_sync"] = {"seed": 20240611, "n": 10000, "c_sha256": digest(c),
                        "a_sha256": digest(a), "b_sha256": digest(b), "c_head": c[:8].tolist()}
    path = os.path.join(HERE, "reference_known_answers.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
