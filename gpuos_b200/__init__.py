"""B200-native persistent micro-op runtime (drop-in for the gpuos_ext / scheduler_context
API of jwgale/GPUOS).

    from gpuos_b200 import gpuos_ext
    from gpuos_b200.scheduler import scheduler_context

The compiled extension (gpuos_b200/_gpuos_ext*.so over gpuos_b200/lib/libgpuos_b200.so) is
required; build it with ``python -m gpuos_b200.build``.  There is no CPU or PyTorch fallback.
"""
import os as _os

# The persistent worker occupies one hardware work queue of the device for as long as it
# runs; kernels on other streams that the driver maps to the same queue wait behind it
# (until the worker's idle stop).  More queues make that sharing rare.  Only effective
# when this package is imported before CUDA is initialised in the process.
_os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

LIB_PATH = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "lib", "libgpuos_b200.so")

__all__ = ["gpuos_ext", "scheduler", "LIB_PATH"]
