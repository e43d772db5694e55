"""Failure detection without a GPU fault: a work item whose dependency barrier never opens
makes the worker's bounded wait expire; the worker records the error in mapped memory and
exits, the host raises on the pending flush, and shutdown/re-init still work.  Runs in a
child process so the session runtime is untouched."""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import torch, time
    from gpuos_b200 import gpuos_ext as g
    g.init(1024, 256)
    g.set_device_wait_ms(300)
    a = torch.randn(4096, device="cuda"); o = torch.empty_like(a)
    g.submit_add(a, a, o); g.flush(sync=True)
    assert torch.equal(o.cpu(), a.cpu() * 2)
    g.debug_inject_stall()
    t0 = time.time()
    try:
        g.flush(sync=True)
        raise SystemExit("expected an error")
    except RuntimeError as e:
        msg = str(e)
    assert "dependency barrier" in msg, msg
    assert time.time() - t0 < 10
    try:
        g.submit_add(a, a, o); g.flush(sync=True)
        raise SystemExit("runtime should stay failed")
    except RuntimeError:
        pass
    g.shutdown()
    g.init(1024, 256)
    g.submit_mul(a, a, o); g.flush(sync=True)
    assert torch.equal(o.cpu(), a.cpu() * a.cpu())
    g.shutdown()
    print("FAILURE-PATH-OK", msg)
""")


def test_bounded_device_wait_reports_error():
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAILURE-PATH-OK" in r.stdout
