"""The config-5 pattern on one GPU: dependent chains of element-wise requests (each request
reads the previous request's output of its chain, within a flush and across flushes) run
while op slot 0 is switched online to multiply and then routed through the alias table and
rolled back (test/online_switch.cpp, test/dual_slot_switch.cpp; the full workload spreads the
chains over up to 8 GPUs, one runtime each, in bench.py --workload c5).  Probe Tasks through slot 0 in every phase must show
that phase's operator (no misdispatch) and every chain must end exactly at its PyTorch CPU
value (no lost or reordered request)."""
import pytest
import torch

import bench
from oracle.reference_semantics import same_bits

pytestmark = pytest.mark.gpu


def test_chains_with_online_switch_and_alias_rollback(rt):
    g = torch.Generator().manual_seed(1234 + 5)
    n_chain, depth, n = 64, 32, 4096
    y0 = torch.rand(n_chain, n, generator=g) * 2 - 1
    consts = torch.rand(n_chain, depth, n, generator=g) + 0.5          # U(0.5, 1.5)
    kinds = torch.randint(0, 4, (n_chain, depth), generator=g).tolist()
    host_ops = [torch.add, torch.sub, torch.mul, torch.maximum]
    dev_ops = [rt.submit_add, rt.submit_sub, rt.submit_mul,
               lambda a, b, o: rt.submit_elementwise(rt.EW_MAXIMUM, a, b, o)]

    i = torch.arange(n, dtype=torch.float32)
    A = (0.5 * i).cuda()
    B = (1.0 + (torch.arange(n) % 5).float()).cuda()
    add_ref, mul_ref = (A + B).cpu(), (A * B).cpu()
    probes = {phase: [torch.full_like(A, -1.0) for _ in range(8)] for phase in range(4)}

    y = y0.cuda()
    c = consts.cuda()
    rows = list(y.unbind(0))
    add_addr, mul_addr = rt.get_slot(0), rt.builtin_op_address(1)
    phase_at = {8: 1, 16: 2, 24: 3}
    try:
        phase = 0
        for k in range(depth):
            if k in phase_at:
                rt.flush(sync=True)  # every probe of the previous phase has run
                phase = phase_at[k]
                if phase == 1:
                    rt.set_slot(0, mul_addr)     # online switch of slot 0
                elif phase == 2:
                    rt.set_slot(0, add_addr)     # undo it, then route 0 -> physical slot 1 (mul)
                    rt.set_alias(0, 1)
                elif phase == 3:
                    rt.set_alias(0, 0)           # rollback
            for ch in range(n_chain):
                dev_ops[kinds[ch][k]](rows[ch], c[ch, k], rows[ch])
            if k % 2 == 0:
                for out in probes[phase][(k % 8) // 2 * 2:(k % 8) // 2 * 2 + 2]:
                    rt.submit_binary(0, A, B, out)
            if k % 4 == 3:
                rt.flush(sync=(k % 8 == 7))
        rt.flush(sync=True)
    finally:
        rt.set_alias(0, 0)
        rt.set_slot(0, add_addr)

    expect = y0.clone()
    for k in range(depth):
        for ch in range(n_chain):
            expect[ch] = host_ops[kinds[ch][k]](expect[ch], consts[ch, k])
    assert same_bits(y.cpu(), expect)
    for phase, outs in probes.items():
        ref = add_ref if phase in (0, 3) else mul_ref
        for out in outs:
            assert same_bits(out.cpu(), ref), phase


def test_config5_full_size_one_gpu(rt):
    """Config 5 at its full size on one runtime: 2048 chains x 32 dependent requests over the 19
    config-2 operators, an NVRTC-compiled multiply committed into slot 0 at request 50000, the
    dual-slot switch at 55000 and the rollback at 60000.  Every one of the 65536 requests is
    checked against PyTorch CPU applied to its own GPU input (bit-exact or within 2 ulp), a
    request that never ran keeps the sentinel value of its output (lost), and every probe Task
    through op 0 must show its phase's operator (misdispatched)."""
    r = bench.c5_run(rt, 0, 1, lambda: None)
    assert r["requests"] == 2048 * 32
    summary = {k: r[k] for k in ("lost", "wrong", "misdispatched", "wrong_by_op", "wrong_examples")}
    assert r["lost"] == 0 and r["wrong"] == 0 and r["misdispatched"] == 0, summary
    assert all(p > 0 for p in r["probes_per_phase"]), r["probes_per_phase"]
    assert rt.get_slot(0) == rt.builtin_op_address(0) and rt.get_alias(0) == 0
