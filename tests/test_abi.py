"""C-ABI boundary: the library loads without a GPU, exports every symbol include/*.h
declares, and keeps the reference's descriptor layout (src/common.h:24-74)."""
import ctypes
import glob
import os
import re

import pytest

from tests._items import LIB_PATH, ROOT

REFERENCE_MODULE_FUNCS = [  # pytorch_ext/gpuos_ext.cpp:1093-1142
    "init", "shutdown", "abi_version", "set_debug_level", "set_verbose_level", "peek_queue",
    "set_yield_every", "worker_alive", "submit_add", "submit_mul", "submit_sub", "submit_div",
    "flush", "register_elementwise", "submit_unary", "submit_binary", "register_reduce",
    "submit_reduce", "register_topk", "submit_topk", "load_and_register_custom",
    "sync_poll_processed", "sync_poll_heartbeat", "sync_poll_ready", "sync_wait", "sync_enabled"]

REFERENCE_C_ABI = [  # src/persistent_kernel.cu:233-269
    "launch_init_builtin_ops", "launch_persistent_worker", "gpu_get_processed_count_async",
    "gpu_set_op_table_async", "gpu_set_alias_async", "gpu_get_heartbeat_async",
    "gpu_set_debug_level_async", "gpu_set_yield_every_async"]


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w]*\s*\**\s+\**(\w+)\s*\([^;]*\);", src, re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB_PATH)
    names = declared_functions()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_reference_c_abi_present():
    lib = ctypes.CDLL(LIB_PATH)
    for n in REFERENCE_C_ABI:
        assert hasattr(lib, n), n
    assert set(REFERENCE_C_ABI) <= set(declared_functions())


def test_descriptor_layout_matches_reference():
    lib = ctypes.CDLL(LIB_PATH)
    buf = (ctypes.c_int64 * 16)()
    n = lib.gpuos_abi_sizes(buf, 16)
    v = list(buf)[:n]
    # TensorRef 144, Task 496, in0@64, in1@208, out0@352, SyncState 64, WorkQueue 48
    assert v[:7] == [144, 496, 64, 208, 352, 64, 48]
    assert v[7] == 64  # work item


def test_python_module_has_reference_functions():
    from gpuos_b200 import gpuos_ext
    missing = [f for f in REFERENCE_MODULE_FUNCS if not callable(getattr(gpuos_ext, f, None))]
    assert not missing, missing
    assert gpuos_ext.abi_version() == 1


def test_runtime_calls_fail_cleanly_without_init():
    from gpuos_b200 import gpuos_ext
    with pytest.raises(RuntimeError):
        gpuos_ext.sync_poll_processed()
    with pytest.raises(RuntimeError):
        gpuos_ext.peek_queue()


def test_error_codes_without_device():
    lib = ctypes.CDLL(LIB_PATH)
    lib.gpuos_rt_last_error.restype = ctypes.c_char_p
    # NULL runtime -> GPUOS_ERR_NOT_INIT, message set, no crash
    assert lib.gpuos_rt_flush(None, 1, None, None) == 5
    assert b"not initialized" in lib.gpuos_rt_last_error()
    assert lib.gpuos_rt_submit_task(None, None) == 5
