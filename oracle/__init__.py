"""CPU oracle of the persistent micro-op path — test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU baseline leg; never by the
runtime (gpuos_b200/), which fails loudly when its CUDA extension is missing.
"""
