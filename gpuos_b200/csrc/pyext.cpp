// pyext.cpp — CPython binding of libgpuos_b200.so with the reference module's API.
//
// Reference: the pybind11 module gpuos_ext (pytorch_ext/gpuos_ext.cpp:1093-1142).  Same
// function names, defaults and argument meaning; differences:
//   * tensors are kept alive until the flush that reads/writes them has completed (the
//     reference borrows raw data_ptr values);
//   * errors raise (RuntimeError / ValueError / TimeoutError) instead of exit();
//   * a blocking wait releases the GIL;
//   * requests go to the runtime of the tensors' device (the reference uses device 0);
//   * extra entry points for the scheduler (submit_elementwise, submit_reduction) and for
//     op-table control (set_slot, set_alias, ...).
// The hot calls (submit_add/mul/sub/div) use METH_FASTCALL and read the tensors through
// THPVariable_Unpack without creating intermediate objects.
#include <Python.h>

#include <ATen/core/Tensor.h>
#include <ATen/ops/empty_like.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/python_variable.h>

#include <cmath>
#include <cstring>
#include <deque>
#include <string>
#include <utility>
#include <atomic>
#include <chrono>
#include <thread>
#include <vector>

#include "gpuos_b200.h"
#include "intercept.h"

namespace {

constexpr int kMaxDev = gpuos_py::kMaxDev;

struct DevRefs {
  std::vector<PyObject*> pending;
  std::deque<std::pair<uint64_t, std::vector<PyObject*>>> inflight;
};

gpuos_rt* g_rt[kMaxDev] = {nullptr};
// Calls that run with the GIL released while they use a runtime; shutdown waits for them.
std::atomic<int> g_busy[kMaxDev];
struct Busy {
  int d;
  explicit Busy(int dev) : d(dev) { g_busy[d].fetch_add(1); }
  ~Busy() { g_busy[d].fetch_sub(1); }
};
DevRefs g_refs[kMaxDev];
int g_verbose = 0;

PyObject* raise_status(int st) {
  const char* msg = gpuos_rt_last_error();
  PyObject* exc = PyExc_RuntimeError;
  if (st == GPUOS_ERR_INVALID) exc = PyExc_ValueError;
  else if (st == GPUOS_ERR_TIMEOUT) exc = PyExc_TimeoutError;
  else if (st == GPUOS_ERR_UNSUPPORTED) exc = PyExc_NotImplementedError;
  PyErr_SetString(exc, (msg && *msg) ? msg : "gpuos error");
  return nullptr;
}

// Dropping a reference can run arbitrary Python code (finalizers, weakref callbacks, the
// garbage collector) and let another thread run, which may flush and touch g_refs.  So the
// references are first taken out of the shared lists, and dropped afterwards.
void drop_refs(std::vector<PyObject*>& v) {
  for (PyObject* o : v) Py_DECREF(o);
}

void release_completed(int dev) {
  gpuos_rt* rt = g_rt[dev];
  const uint64_t done = rt ? gpuos_rt_completed(rt) : ~0ull;
  gpuos_py::intercept_release(dev, done);  // tensors held by the dispatcher intercept's requests
  DevRefs& R = g_refs[dev];
  if (R.inflight.empty()) return;
  std::vector<PyObject*> dead;
  while (!R.inflight.empty() && R.inflight.front().first <= done) {
    auto& v = R.inflight.front().second;
    dead.insert(dead.end(), v.begin(), v.end());
    R.inflight.pop_front();
  }
  drop_refs(dead);
}

void release_all(int dev) {
  gpuos_py::intercept_release_all(dev);
  DevRefs& R = g_refs[dev];
  std::vector<PyObject*> dead;
  dead.swap(R.pending);
  while (!R.inflight.empty()) {
    auto& v = R.inflight.front().second;
    dead.insert(dead.end(), v.begin(), v.end());
    R.inflight.pop_front();
  }
  drop_refs(dead);
}

int dtype_code(c10::ScalarType st) {
  switch (st) {
    case c10::ScalarType::Float: return kF32;
    case c10::ScalarType::Half: return kF16;
    case c10::ScalarType::BFloat16: return kBF16;
    default: return -1;
  }
}

// Fill a GpuosOperand from a CUDA tensor.  Returns the device index or -1 with an error set.
int to_operand(PyObject* o, GpuosOperand* op, const char* name) {
  if (!THPVariable_Check(o)) {
    PyErr_Format(PyExc_TypeError, "%s must be a torch.Tensor", name);
    return -1;
  }
  const at::Tensor& t = THPVariable_Unpack(o);
  if (!t.is_cuda()) {
    PyErr_SetString(PyExc_RuntimeError, "tensors must be CUDA");
    return -1;
  }
  const int dt = dtype_code(t.scalar_type());
  if (dt < 0) {
    PyErr_Format(PyExc_ValueError, "%s: unsupported dtype (float32, float16, bfloat16 only)", name);
    return -1;
  }
  const int nd = (int)t.dim();
  if (nd > GPUOS_MAX_NDIM) {
    PyErr_Format(PyExc_ValueError, "%s: more than %d dimensions", name, GPUOS_MAX_NDIM);
    return -1;
  }
  op->data = t.data_ptr();
  op->dtype = dt;
  op->ndim = nd;
  const auto sz = t.sizes();
  const auto st = t.strides();
  for (int d = 0; d < nd; ++d) {
    op->sizes[d] = sz[d];
    op->strides[d] = st[d];
  }
  const int dev = t.get_device();
  if (dev < 0 || dev >= kMaxDev) {
    PyErr_SetString(PyExc_RuntimeError, "device index out of range");
    return -1;
  }
  return dev;
}

gpuos_rt* rt_for(int dev) {
  gpuos_rt* rt = g_rt[dev];
  if (!rt) PyErr_SetString(PyExc_RuntimeError, "gpuos not initialized");
  return rt;
}

void keep(int dev, PyObject* o) {
  Py_INCREF(o);
  g_refs[dev].pending.push_back(o);
}

// After a publish with ticket seq: pending refs belong to flushes <= seq.
void move_pending(int dev, uint64_t seq) {
  DevRefs& R = g_refs[dev];
  if (R.pending.empty()) return;
  if (seq == 0) seq = ~0ull >> 1;
  if (!R.inflight.empty() && R.inflight.back().first == seq) {
    auto& v = R.inflight.back().second;
    v.insert(v.end(), R.pending.begin(), R.pending.end());
    R.pending.clear();
  } else {
    R.inflight.emplace_back(seq, std::move(R.pending));
    R.pending = std::vector<PyObject*>();
  }
}

// Second operand: CUDA tensor, Python number, 0-dim CPU tensor, or None.
int parse_b(PyObject* o, GpuosOperand* op, int* is_scalar, double* val, bool* present) {
  *is_scalar = 0;
  *val = 0.0;
  *present = false;
  if (o == nullptr || o == Py_None) return 0;
  *present = true;
  if (PyFloat_Check(o) || PyLong_Check(o) || PyBool_Check(o)) {
    *is_scalar = 1;
    *val = PyFloat_AsDouble(o);
    return PyErr_Occurred() ? -1 : 0;
  }
  if (THPVariable_Check(o)) {
    const at::Tensor& t = THPVariable_Unpack(o);
    if (!t.is_cuda() && t.dim() == 0) {
      *is_scalar = 1;
      *val = t.item<double>();
      return 0;
    }
  }
  return to_operand(o, op, "b") < 0 ? -1 : 1;
}

// ---- submit_add / mul / sub / div (gpuos_ext.cpp:638-672) -------------------------------
PyObject* submit_binary_builtin(PyObject* const* args, Py_ssize_t nargs, int op) {
  if (nargs != 3) {
    PyErr_SetString(PyExc_TypeError, "expected (a, b, out)");
    return nullptr;
  }
  GpuosOperand a, b, out;
  const int da = to_operand(args[0], &a, "a");
  if (da < 0) return nullptr;
  const int db = to_operand(args[1], &b, "b");
  if (db < 0) return nullptr;
  const int dout = to_operand(args[2], &out, "out");
  if (dout < 0) return nullptr;
  if (da != dout || db != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  gpuos_rt* rt = rt_for(dout);
  if (!rt) return nullptr;
  const int st = gpuos_rt_submit_ew(rt, op, &a, &b, 0, 0.0, &out, nullptr, 0);
  if (st) return raise_status(st);
  keep(dout, args[0]);
  keep(dout, args[1]);
  keep(dout, args[2]);
  Py_RETURN_NONE;
}

PyObject* py_submit_add(PyObject*, PyObject* const* a, Py_ssize_t n) { return submit_binary_builtin(a, n, GPUOS_EW_ADD); }
PyObject* py_submit_mul(PyObject*, PyObject* const* a, Py_ssize_t n) { return submit_binary_builtin(a, n, GPUOS_EW_MUL); }
PyObject* py_submit_sub(PyObject*, PyObject* const* a, Py_ssize_t n) { return submit_binary_builtin(a, n, GPUOS_EW_SUB); }
PyObject* py_submit_div(PyObject*, PyObject* const* a, Py_ssize_t n) { return submit_binary_builtin(a, n, GPUOS_EW_DIV); }

// submit_elementwise(op, a, b, out, p0=0.0, p1=0.0) — any built-in element-wise op, b may be
// a tensor, a number or None.
PyObject* py_submit_elementwise(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs < 4 || nargs > 6) {
    PyErr_SetString(PyExc_TypeError, "expected (op, a, b, out[, p0[, p1]])");
    return nullptr;
  }
  const long op = PyLong_AsLong(args[0]);
  if (op == -1 && PyErr_Occurred()) return nullptr;
  GpuosOperand a, b, out;
  const int da = to_operand(args[1], &a, "a");
  if (da < 0) return nullptr;
  int b_scalar = 0;
  double b_val = 0.0;
  bool b_present = false;
  const int bt = parse_b(args[2], &b, &b_scalar, &b_val, &b_present);
  if (bt < 0) return nullptr;
  const int dout = to_operand(args[3], &out, "out");
  if (dout < 0) return nullptr;
  if (da != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  float params[2] = {0.f, 0.f};
  for (int i = 0; i < 2 && 4 + i < nargs; ++i) {
    params[i] = (float)PyFloat_AsDouble(args[4 + i]);
    if (PyErr_Occurred()) return nullptr;
  }
  gpuos_rt* rt = rt_for(dout);
  if (!rt) return nullptr;
  const int st = gpuos_rt_submit_ew(rt, (int)op, &a, bt == 1 ? &b : nullptr, b_scalar, b_val, &out, params, 2);
  if (st) return raise_status(st);
  keep(dout, args[1]);
  if (bt == 1) keep(dout, args[2]);
  keep(dout, args[3]);
  Py_RETURN_NONE;
}

// submit_ew_new(op, a, b_or_None_or_number[, p0[, p1]]) -> out: an element-wise request whose output is a new
// contiguous tensor like `a` (same dtype, shape and device), allocated here.  The scheduler's
// common case (operands of one dtype and shape) in one call: allocating from Python through the
// dispatcher costs about as much as the rest of the dispatch.
PyObject* py_submit_ew_new(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs < 3 || nargs > 5) {
    PyErr_SetString(PyExc_TypeError, "expected (op, a, b[, p0[, p1]])");
    return nullptr;
  }
  const long op = PyLong_AsLong(args[0]);
  if (op == -1 && PyErr_Occurred()) return nullptr;
  if (!THPVariable_Check(args[1])) {
    PyErr_SetString(PyExc_TypeError, "a must be a tensor");
    return nullptr;
  }
  GpuosOperand a, b, out;
  const int da = to_operand(args[1], &a, "a");
  if (da < 0) return nullptr;
  int b_scalar = 0;
  double b_val = 0.0;
  bool b_present = false;
  const int bt = parse_b(args[2], &b, &b_scalar, &b_val, &b_present);
  if (bt < 0) return nullptr;
  PyObject* o = THPVariable_Wrap(at::empty_like(THPVariable_Unpack(args[1]), at::MemoryFormat::Contiguous));
  if (!o) return nullptr;
  const int dout = to_operand(o, &out, "out");
  if (dout < 0) {
    Py_DECREF(o);
    return nullptr;
  }
  gpuos_rt* rt = rt_for(dout);
  if (!rt) {
    Py_DECREF(o);
    return nullptr;
  }
  float params[2] = {0.f, 0.f};
  for (int i = 0; i < 2 && 3 + i < nargs; ++i) {
    params[i] = (float)PyFloat_AsDouble(args[3 + i]);
    if (PyErr_Occurred()) {
      Py_DECREF(o);
      return nullptr;
    }
  }
  const int st = gpuos_rt_submit_ew(rt, (int)op, &a, bt == 1 ? &b : nullptr, b_scalar, b_val, &out, params, 2);
  if (st) {
    Py_DECREF(o);
    return raise_status(st);
  }
  keep(dout, args[1]);
  if (bt == 1) keep(dout, args[2]);
  keep(dout, o);
  return o;
}

bool parse_axes(PyObject* seq, std::vector<int>* axes) {
  axes->clear();
  if (PyLong_Check(seq)) {
    axes->push_back((int)PyLong_AsLong(seq));
    return !PyErr_Occurred();
  }
  PyObject* fast = PySequence_Fast(seq, "axes must be a sequence of ints");
  if (!fast) return false;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fast);
  for (Py_ssize_t i = 0; i < n; ++i) {
    const long v = PyLong_AsLong(PySequence_Fast_GET_ITEM(fast, i));
    if (v == -1 && PyErr_Occurred()) {
      Py_DECREF(fast);
      return false;
    }
    axes->push_back((int)v);
  }
  Py_DECREF(fast);
  return true;
}

// submit_reduction(op, x, out, axes, keepdim) — batched sum/mean.
PyObject* py_submit_reduction(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs != 5) {
    PyErr_SetString(PyExc_TypeError, "expected (op, x, out, axes, keepdim)");
    return nullptr;
  }
  const long op = PyLong_AsLong(args[0]);
  if (op == -1 && PyErr_Occurred()) return nullptr;
  GpuosOperand x, out;
  const int dx = to_operand(args[1], &x, "x");
  if (dx < 0) return nullptr;
  const int dout = to_operand(args[2], &out, "out");
  if (dout < 0) return nullptr;
  if (dx != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  std::vector<int> axes;
  if (!parse_axes(args[3], &axes)) return nullptr;
  const int keepdim = PyObject_IsTrue(args[4]);
  if (keepdim < 0) return nullptr;
  gpuos_rt* rt = rt_for(dout);
  if (!rt) return nullptr;
  const int st = gpuos_rt_submit_reduce(rt, (int)op, &x, &out, axes.data(), (int)axes.size(), keepdim);
  if (st) return raise_status(st);
  keep(dout, args[1]);
  keep(dout, args[2]);
  Py_RETURN_NONE;
}

// ---- flush (gpuos_ext.cpp:675-811) ------------------------------------------------------
int flush_device(int dev, bool sync, uint64_t* seq_out) {
  gpuos_rt* rt = g_rt[dev];
  if (!rt) return 0;
  cudaStream_t dep = c10::cuda::getCurrentCUDAStream((c10::DeviceIndex)dev).stream();
  uint64_t seq = 0;
  // through the intercept: its references are tied to this flush in the same step
  int st = gpuos_py::intercept_flush(dev, rt, GPUOS_FLUSH_DEP, dep, &seq);
  if (st) return st;
  move_pending(dev, seq);
  if (sync && seq) {
    Busy busy(dev);
    Py_BEGIN_ALLOW_THREADS st = gpuos_rt_wait(rt, seq, 30000);
    Py_END_ALLOW_THREADS
  }
  if (seq_out) *seq_out = seq;
  release_completed(dev);
  return st;
}

PyObject* py_flush(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"sync", "device", nullptr};
  int sync = 0;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|pO", const_cast<char**>(kwlist), &sync, &devobj)) return nullptr;
  uint64_t last = 0;
  if (devobj != Py_None) {
    const long d = PyLong_AsLong(devobj);
    if (d < 0 || d >= kMaxDev) return PyErr_Format(PyExc_ValueError, "bad device %ld", d);
    const int st = flush_device((int)d, sync != 0, &last);
    if (st) return raise_status(st);
    return PyLong_FromUnsignedLongLong(last);
  }
  for (int d = 0; d < kMaxDev; ++d) {
    if (!g_rt[d]) continue;
    uint64_t s = 0;
    const int st = flush_device(d, sync != 0, &s);
    if (st) return raise_status(st);
    if (s) last = s;
  }
  return PyLong_FromUnsignedLongLong(last);
}

// ---- lifecycle ----------------------------------------------------------------------------
int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int parse_device(PyObject* devobj, int* dev) {
  if (devobj == nullptr || devobj == Py_None) {
    *dev = current_device();
    return 0;
  }
  if (PyLong_Check(devobj)) {
    *dev = (int)PyLong_AsLong(devobj);
  } else {
    PyObject* idx = PyObject_GetAttrString(devobj, "index");
    if (!idx) return -1;
    *dev = idx == Py_None ? current_device() : (int)PyLong_AsLong(idx);
    Py_DECREF(idx);
  }
  if (*dev < 0 || *dev >= kMaxDev) {
    PyErr_SetString(PyExc_ValueError, "device index out of range");
    return -1;
  }
  return 0;
}

PyObject* py_init(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"capacity", "threads_per_block", "device", nullptr};
  int capacity = 4096, tpb = 256;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|iiO", const_cast<char**>(kwlist), &capacity, &tpb, &devobj))
    return nullptr;
  int dev;
  if (parse_device(devobj, &dev)) return nullptr;
  if (g_rt[dev]) Py_RETURN_NONE;
  gpuos_rt* rt = nullptr;
  int st;
  Py_BEGIN_ALLOW_THREADS st = gpuos_rt_init(dev, capacity, tpb, &rt);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  g_rt[dev] = rt;
  Py_RETURN_NONE;
}

int shutdown_device(int dev) {
  gpuos_rt* rt = g_rt[dev];
  if (!rt) return 0;
  g_rt[dev] = nullptr;  // later calls see "not initialized"; calls in flight finish first
  move_pending(dev, 0);
  int st;
  Py_BEGIN_ALLOW_THREADS
  while (g_busy[dev].load() > 0) std::this_thread::sleep_for(std::chrono::microseconds(50));
  st = gpuos_rt_shutdown(rt);
  Py_END_ALLOW_THREADS
  release_all(dev);
  return st;
}

PyObject* py_shutdown(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  int first_err = 0;
  if (devobj != Py_None) {
    int dev;
    if (parse_device(devobj, &dev)) return nullptr;
    first_err = shutdown_device(dev);
  } else {
    for (int d = 0; d < kMaxDev; ++d) {
      const int st = shutdown_device(d);
      if (st && !first_err) first_err = st;
    }
  }
  if (first_err) return raise_status(first_err);
  Py_RETURN_NONE;
}

// Runtime selected by an optional device argument (default: first initialised runtime).
gpuos_rt* rt_arg(PyObject* devobj, int* dev_out) {
  if (devobj && devobj != Py_None) {
    int dev;
    if (parse_device(devobj, &dev)) return nullptr;
    if (dev_out) *dev_out = dev;
    return rt_for(dev);
  }
  const int cur = current_device();
  if (g_rt[cur]) {
    if (dev_out) *dev_out = cur;
    return g_rt[cur];
  }
  for (int d = 0; d < kMaxDev; ++d)
    if (g_rt[d]) {
      if (dev_out) *dev_out = d;
      return g_rt[d];
    }
  PyErr_SetString(PyExc_RuntimeError, "gpuos not initialized");
  return nullptr;
}

PyObject* py_abi_version(PyObject*, PyObject*) { return PyLong_FromLong(1); }

PyObject* py_set_debug_level(PyObject*, PyObject* args) {
  int lvl;
  if (!PyArg_ParseTuple(args, "i", &lvl)) return nullptr;
  for (int d = 0; d < kMaxDev; ++d)
    if (g_rt[d]) {
      const int st = gpuos_rt_set_debug_level(g_rt[d], lvl);
      if (st) return raise_status(st);
    }
  Py_RETURN_NONE;
}

PyObject* py_set_verbose_level(PyObject*, PyObject* args) {
  if (!PyArg_ParseTuple(args, "i", &g_verbose)) return nullptr;
  Py_RETURN_NONE;
}

PyObject* py_set_yield_every(PyObject*, PyObject* args) {
  unsigned long long every;
  if (!PyArg_ParseTuple(args, "K", &every)) return nullptr;
  for (int d = 0; d < kMaxDev; ++d)
    if (g_rt[d]) {
      const int st = gpuos_rt_set_yield_every(g_rt[d], every);
      if (st) return raise_status(st);
    }
  Py_RETURN_NONE;
}

PyObject* py_set_idle_quiesce_ms(PyObject*, PyObject* args) {
  int ms;
  if (!PyArg_ParseTuple(args, "i", &ms)) return nullptr;
  for (int d = 0; d < kMaxDev; ++d)
    if (g_rt[d]) {
      const int st = gpuos_rt_set_idle_quiesce_ms(g_rt[d], ms);
      if (st) return raise_status(st);
    }
  Py_RETURN_NONE;
}

PyObject* py_worker_alive(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  if (devobj == Py_None) {
    bool any = false;
    for (int d = 0; d < kMaxDev; ++d) any |= (g_rt[d] && gpuos_rt_worker_alive(g_rt[d]));
    return PyBool_FromLong(any);
  }
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  return PyBool_FromLong(gpuos_rt_worker_alive(rt));
}

PyObject* py_quiesce(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"timeout_ms", "device", nullptr};
  int timeout_ms = 30000;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|iO", const_cast<char**>(kwlist), &timeout_ms, &devobj)) return nullptr;
  for (int d = 0; d < kMaxDev; ++d) {
    if (!g_rt[d]) continue;
    if (devobj != Py_None) {
      int dev;
      if (parse_device(devobj, &dev)) return nullptr;
      if (dev != d) continue;
    }
    int st;
    gpuos_rt* rt = g_rt[d];
    Busy busy(d);
    Py_BEGIN_ALLOW_THREADS st = gpuos_rt_quiesce(rt, timeout_ms);
    Py_END_ALLOW_THREADS
    if (st) return raise_status(st);
  }
  Py_RETURN_NONE;
}

PyObject* py_peek_queue(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  int64_t v[32];
  const int st = gpuos_rt_stats(rt, v, 32);
  if (st) return raise_status(st);
  PyObject* d = PyDict_New();
  std::string names = gpuos_rt_stat_names();
  size_t pos = 0;
  int i = 0;
  while (pos <= names.size() && i < 32) {
    size_t c = names.find(',', pos);
    if (c == std::string::npos) c = names.size();
    const std::string key = names.substr(pos, c - pos);
    PyObject* val = PyLong_FromLongLong(v[i++]);
    PyDict_SetItemString(d, key.c_str(), val);
    Py_DECREF(val);
    pos = c + 1;
  }
  PyObject* t = Py_True;
  PyDict_SetItemString(d, "sync_enabled", t);
  PyObject* sv = PyUnicode_FromString("mapped");
  PyDict_SetItemString(d, "staging", sv);
  Py_DECREF(sv);
  PyObject* dv = PyLong_FromLong(dev);
  PyDict_SetItemString(d, "device", dv);
  Py_DECREF(dv);
  return d;
}

// ---- zero-copy sync API (gpuos_ext.cpp:1125-1141) ---------------------------------------
PyObject* py_sync_poll_processed(PyObject*, PyObject*) {
  uint64_t total = 0;
  bool any = false;
  for (int d = 0; d < kMaxDev; ++d)
    if (g_rt[d]) {
      total += gpuos_rt_poll_processed(g_rt[d]);
      release_completed(d);
      any = true;
    }
  if (!any) {
    PyErr_SetString(PyExc_RuntimeError, "gpuos not initialized");
    return nullptr;
  }
  return PyLong_FromUnsignedLongLong(total);
}

PyObject* py_sync_poll_heartbeat(PyObject*, PyObject*) {
  gpuos_rt* rt = rt_arg(nullptr, nullptr);
  if (!rt) return nullptr;
  return PyLong_FromUnsignedLongLong(gpuos_rt_poll_heartbeat(rt));
}

PyObject* py_sync_poll_ready(PyObject*, PyObject*) {
  gpuos_rt* rt = rt_arg(nullptr, nullptr);
  if (!rt) return nullptr;
  return PyBool_FromLong(gpuos_rt_poll_ready(rt));
}

PyObject* py_sync_enabled(PyObject*, PyObject*) {
  for (int d = 0; d < kMaxDev; ++d)
    if (g_rt[d]) Py_RETURN_TRUE;
  Py_RETURN_FALSE;
}

// ---- the dispatcher intercept of scheduler_context (intercept.cpp) ------------------------
PyObject* py_intercept_enable(PyObject*, PyObject* args) {
  long long thr;
  if (!PyArg_ParseTuple(args, "L", &thr)) return nullptr;
  std::string err;
  bool ok = false;
  try {
    ok = gpuos_py::intercept_enable(thr, &err);
  } catch (const std::exception& e) {
    err = e.what();
  }
  if (!ok) return PyErr_Format(PyExc_RuntimeError, "intercept unavailable: %s", err.c_str());
  Py_RETURN_NONE;
}

PyObject* py_intercept_disable(PyObject*, PyObject*) {
  gpuos_py::intercept_disable();
  Py_RETURN_NONE;
}

PyObject* py_intercept_enabled(PyObject*, PyObject*) { return PyBool_FromLong(gpuos_py::intercept_enabled()); }

PyObject* py_intercept_clear_pending(PyObject*, PyObject*) {
  gpuos_py::intercept_clear_pending();
  Py_RETURN_NONE;
}

PyObject* counts_dict(const std::vector<std::pair<std::string, int64_t>>& v) {
  PyObject* d = PyDict_New();
  if (!d) return nullptr;
  for (const auto& kv : v) {
    PyObject* n = PyLong_FromLongLong(kv.second);
    if (!n || PyDict_SetItemString(d, kv.first.c_str(), n) < 0) {
      Py_XDECREF(n);
      Py_DECREF(d);
      return nullptr;
    }
    Py_DECREF(n);
  }
  return d;
}

PyObject* py_intercept_routes(PyObject*, PyObject*) {
  PyObject* d = PyDict_New();
  if (!d) return nullptr;
  for (const auto& kv : gpuos_py::intercept_routes()) {
    PyObject* v = Py_BuildValue("(ii)", kv.second.first, kv.second.second);
    if (!v || PyDict_SetItemString(d, kv.first.c_str(), v) < 0) {
      Py_XDECREF(v);
      Py_DECREF(d);
      return nullptr;
    }
    Py_DECREF(v);
  }
  return d;
}

PyObject* py_intercept_stats(PyObject*, PyObject*) {
  const gpuos_py::InterceptStats s = gpuos_py::intercept_stats();
  PyObject* so = counts_dict(s.scheduled_ops);
  PyObject* fo = so ? counts_dict(s.fallback_ops) : nullptr;
  if (!fo) {
    Py_XDECREF(so);
    return nullptr;
  }
  return Py_BuildValue("{s:L,s:L,s:N,s:N}", "scheduled", (long long)s.scheduled, "fallbacks", (long long)s.fallbacks,
                       "scheduled_ops", so, "fallback_ops", fo);
}

PyObject* py_sync_wait(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"target", "timeout_ms", nullptr};
  unsigned long long target;
  int timeout_ms = 30000;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "K|i", const_cast<char**>(kwlist), &target, &timeout_ms)) return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(nullptr, &dev);
  if (!rt) return nullptr;
  int st;
  Busy busy(dev);
  Py_BEGIN_ALLOW_THREADS st = gpuos_rt_sync_wait(rt, target, timeout_ms);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  Py_RETURN_NONE;
}

PyObject* py_wait(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"seq", "timeout_ms", "device", nullptr};
  unsigned long long seq;
  int timeout_ms = 30000;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "K|iO", const_cast<char**>(kwlist), &seq, &timeout_ms, &devobj))
    return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  int st;
  Busy busy(dev);
  Py_BEGIN_ALLOW_THREADS st = gpuos_rt_wait(rt, seq, timeout_ms);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  release_completed(dev);
  Py_RETURN_NONE;
}

PyObject* py_completed(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  const uint64_t c = gpuos_rt_completed(rt);
  release_completed(dev);
  return PyLong_FromUnsignedLongLong(c);
}

PyObject* py_flush_times(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"seq", "device", nullptr};
  unsigned long long seq;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "K|O", const_cast<char**>(kwlist), &seq, &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  uint64_t t0 = 0, t1 = 0;
  const int st = gpuos_rt_flush_times(rt, seq, &t0, &t1);
  if (st) return raise_status(st);
  return Py_BuildValue("(KK)", (unsigned long long)t0, (unsigned long long)t1);
}

PyObject* py_kernel_stream(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  return PyLong_FromVoidPtr(reinterpret_cast<void*>(gpuos_rt_kernel_stream(rt)));
}

PyObject* py_set_device_wait_ms(PyObject*, PyObject* args) {
  int ms;
  if (!PyArg_ParseTuple(args, "i", &ms)) return nullptr;
  for (int d = 0; d < kMaxDev; ++d)
    if (g_rt[d]) {
      const int st = gpuos_rt_set_device_wait_ms(g_rt[d], ms);
      if (st) return raise_status(st);
    }
  Py_RETURN_NONE;
}

PyObject* py_debug_inject_stall(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  const int st = gpuos_rt_debug_inject_stall(rt);
  if (st) return raise_status(st);
  Py_RETURN_NONE;
}

PyObject* py_debug_counters(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  // one row per worker CTA (fewer than 512) plus the launch timeline row
  std::vector<uint64_t> buf(513 * 12, ~0ull);
  int ctas = gpuos_rt_debug_counters(rt, buf.data(), (int)buf.size());
  if (ctas < 0) return raise_status(-ctas);
  if (ctas > 512) ctas = 512;
  PyObject* rows = PyList_New(ctas);
  for (int c = 0; c < ctas; ++c) {
    PyObject* row = PyList_New(12);
    for (int k = 0; k < 12; ++k) PyList_SET_ITEM(row, k, PyLong_FromUnsignedLongLong(buf[c * 12 + k]));
    PyList_SET_ITEM(rows, c, row);
  }
  return rows;
}

PyObject* py_debug_timeline(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  std::vector<uint64_t> buf(513 * 12, ~0ull);
  int ctas = gpuos_rt_debug_counters(rt, buf.data(), (int)buf.size());
  if (ctas < 0) return raise_status(-ctas);
  if (ctas > 511) ctas = 511;
  PyObject* row = PyList_New(12);
  for (int k = 0; k < 12; ++k) PyList_SET_ITEM(row, k, PyLong_FromUnsignedLongLong(buf[ctas * 12 + k]));
  return row;
}

PyObject* py_set_launch_timing(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"on", "device", nullptr};
  int on = 1;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "p|O", const_cast<char**>(kwlist), &on, &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  const int st = gpuos_rt_set_launch_timing(rt, on);
  if (st) return raise_status(st);
  Py_RETURN_NONE;
}

PyObject* py_launch_times(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  std::vector<float> buf(4096);
  int n;
  Busy busy(dev);
  Py_BEGIN_ALLOW_THREADS
  n = gpuos_rt_launch_times(rt, buf.data(), (int)buf.size());
  Py_END_ALLOW_THREADS
  if (n < 0) return raise_status(-n);
  PyObject* out = PyList_New(n);
  for (int i = 0; i < n; ++i) PyList_SET_ITEM(out, i, PyFloat_FromDouble(buf[i]));
  return out;
}

PyObject* py_launches(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  return PyLong_FromUnsignedLongLong(gpuos_rt_launches(rt));
}

// ---- op table: slots, aliases, built-in registrations -------------------------------------
PyObject* py_set_slot(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"slot", "fn", "device", nullptr};
  int slot;
  unsigned long long fn;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "iK|O", const_cast<char**>(kwlist), &slot, &fn, &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  const int st = gpuos_rt_set_slot(rt, slot, fn);
  if (st) return raise_status(st);
  Py_RETURN_NONE;
}

PyObject* py_get_slot(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"slot", "device", nullptr};
  int slot;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "i|O", const_cast<char**>(kwlist), &slot, &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  OpPtrInt fn = 0;
  const int st = gpuos_rt_get_slot(rt, slot, &fn);
  if (st) return raise_status(st);
  return PyLong_FromUnsignedLongLong(fn);
}

PyObject* py_set_alias(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"logical", "physical", "device", nullptr};
  int lg, ph;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "ii|O", const_cast<char**>(kwlist), &lg, &ph, &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  const int st = gpuos_rt_set_alias(rt, lg, ph);
  if (st) return raise_status(st);
  Py_RETURN_NONE;
}

PyObject* py_get_alias(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"logical", "device", nullptr};
  int lg;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "i|O", const_cast<char**>(kwlist), &lg, &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  int ph = -1;
  const int st = gpuos_rt_get_alias(rt, lg, &ph);
  if (st) return raise_status(st);
  return PyLong_FromLong(ph);
}

PyObject* py_builtin_op_address(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"code", "device", nullptr};
  int code;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "i|O", const_cast<char**>(kwlist), &code, &devobj)) return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  // the address in the worker module the runtime of this device currently runs
  OpPtrInt addr = 0;
  const int st = gpuos_rt_builtin_op(rt, code, &addr);
  if (st) return raise_status(st);
  return PyLong_FromUnsignedLongLong(addr);
}

// ---- operators compiled at run time (NVRTC for sm_100a, linked into the worker) ---------------
PyObject* py_register_jit(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"expr", "arity", "slot", "device", nullptr};
  const char* expr;
  int arity, slot = -1;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "si|iO", const_cast<char**>(kwlist), &expr, &arity, &slot, &devobj))
    return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  int out = -1, st;
  Busy busy(dev);
  Py_BEGIN_ALLOW_THREADS st = gpuos_rt_register_jit(rt, expr, arity, slot, &out);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  return PyLong_FromLong(out);
}

PyObject* py_load_custom(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"ptx", "entry", "slot", "device", nullptr};
  const char* ptx;  // PTX is text: no embedded NUL
  const char* entry;
  int slot = -1;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "ss|iO", const_cast<char**>(kwlist), &ptx, &entry, &slot, &devobj))
    return nullptr;
  const size_t n = std::strlen(ptx);
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  int out = -1, st;
  Busy busy(dev);
  Py_BEGIN_ALLOW_THREADS st = gpuos_rt_load_custom(rt, ptx, (size_t)n, entry, slot, &out);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  return PyLong_FromLong(out);
}

// Staged operator: a capsule that frees the staged image when dropped.
void staged_free(PyObject* cap) {
  void* p = PyCapsule_GetPointer(cap, "gpuos_jit_staged");
  if (p) gpuos_rt_jit_discard(static_cast<gpuos_jit_staged*>(p));
}

PyObject* py_jit_stage(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"expr", "arity", "device", nullptr};
  const char* expr;
  int arity;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "si|O", const_cast<char**>(kwlist), &expr, &arity, &devobj))
    return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  gpuos_jit_staged* st = nullptr;
  int e;
  Busy busy(dev);
  Py_BEGIN_ALLOW_THREADS e = gpuos_rt_jit_stage(rt, expr, arity, &st);
  Py_END_ALLOW_THREADS
  if (e) return raise_status(e);
  return PyCapsule_New(st, "gpuos_jit_staged", staged_free);
}

PyObject* py_jit_commit(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"staged", "slot", "device", nullptr};
  PyObject* cap;
  int slot = -1;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "O|iO", const_cast<char**>(kwlist), &cap, &slot, &devobj)) return nullptr;
  auto* st = static_cast<gpuos_jit_staged*>(PyCapsule_GetPointer(cap, "gpuos_jit_staged"));
  if (!st) return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  int out = -1, e;
  Busy busy(dev);
  Py_BEGIN_ALLOW_THREADS e = gpuos_rt_jit_commit(rt, st, slot, &out);
  Py_END_ALLOW_THREADS
  if (e) return raise_status(e);
  return PyLong_FromLong(out);
}

PyObject* py_jit_ops(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"device", nullptr};
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "|O", const_cast<char**>(kwlist), &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  const int n = gpuos_rt_jit_ops(rt);
  if (n < 0) return raise_status(-n);
  return PyLong_FromLong(n);
}

// Device-free: NVRTC output (relocatable sm_100a code, or PTX) of a CUDA source.
PyObject* py_jit_compile(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"src", "ptx", nullptr};
  const char* src;
  int ptx = 0;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "s|p", const_cast<char**>(kwlist), &src, &ptx)) return nullptr;
  size_t n = 0;
  int st;
  Py_BEGIN_ALLOW_THREADS st = gpuos_jit_compile(src, ptx, nullptr, 0, &n);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  std::string buf(n, '\0');
  Py_BEGIN_ALLOW_THREADS st = gpuos_jit_compile(src, ptx, &buf[0], n, &n);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  if (ptx) {
    while (!buf.empty() && buf.back() == '\0') buf.pop_back();
    return PyUnicode_FromStringAndSize(buf.data(), (Py_ssize_t)buf.size());
  }
  return PyBytes_FromStringAndSize(buf.data(), (Py_ssize_t)n);
}

// Device-free: compile an expression operator and link it with the worker; returns the size of
// the linked image.
PyObject* py_jit_check_expr(PyObject*, PyObject* args) {
  const char* expr;
  int arity;
  if (!PyArg_ParseTuple(args, "si", &expr, &arity)) return nullptr;
  size_t n = 0;
  int st;
  Py_BEGIN_ALLOW_THREADS st = gpuos_jit_check_expr(expr, arity, &n);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  return PyLong_FromSize_t(n);
}

PyObject* py_jit_nvrtc_version(PyObject*, PyObject*) { return PyLong_FromLong(gpuos_jit_nvrtc_version()); }

PyObject* py_register_builtin(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"kind", "op", "device", nullptr};
  const char* kind;
  int op;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "si|O", const_cast<char**>(kwlist), &kind, &op, &devobj)) return nullptr;
  gpuos_rt* rt = rt_arg(devobj, nullptr);
  if (!rt) return nullptr;
  int slot = -1;
  int st;
  if (std::strcmp(kind, "reduce") == 0) st = gpuos_rt_register_builtin_reduce(rt, op, &slot);
  else if (std::strcmp(kind, "elementwise") == 0) st = gpuos_rt_register_builtin_ew(rt, op, &slot);
  else return PyErr_Format(PyExc_ValueError, "kind must be 'reduce' or 'elementwise'");
  if (st) return raise_status(st);
  return PyLong_FromLong(slot);
}

PyObject* py_register_expr(PyObject*, PyObject* args, PyObject* kw) {
  static const char* kwlist[] = {"key", "expr", "arity", "slot", "device", nullptr};
  const char *key, *expr;
  int arity, slot = -1;
  PyObject* devobj = Py_None;
  if (!PyArg_ParseTupleAndKeywords(args, kw, "ssi|iO", const_cast<char**>(kwlist), &key, &expr, &arity, &slot, &devobj))
    return nullptr;
  int dev = 0;
  gpuos_rt* rt = rt_arg(devobj, &dev);
  if (!rt) return nullptr;
  int out = -1, st;
  Busy busy(dev);
  Py_BEGIN_ALLOW_THREADS st = gpuos_rt_register_expr(rt, key, expr, arity, slot, &out);
  Py_END_ALLOW_THREADS
  if (st) return raise_status(st);
  return PyLong_FromLong(out);
}

// ---- reference-layout Tasks (gpuos_ext.cpp:280-314, 884-896, 1016-1045) --------------------
void fill_ref(TensorRef& tr, const GpuosOperand& t) {
  std::memset(&tr, 0, sizeof(tr));
  tr.data = t.data;
  tr.dtype = t.dtype;
  tr.ndim = t.ndim;
  for (int d = 0; d < t.ndim; ++d) {
    tr.sizes[d] = t.sizes[d];
    tr.strides[d] = t.strides[d];
  }
}

// Input aligned to the output dims: broadcast dims carry the output size and stride 0, so
// decoding an output index with the input's own sizes gives the right coordinates.
bool fill_ref_bcast(TensorRef& tr, const GpuosOperand& in, const GpuosOperand& out) {
  std::memset(&tr, 0, sizeof(tr));
  tr.data = in.data;
  tr.dtype = in.dtype;
  tr.ndim = out.ndim;
  for (int d = 0; d < out.ndim; ++d) {
    const int id = in.ndim - out.ndim + d;
    const int64_t sz = id >= 0 ? in.sizes[id] : 1;
    tr.sizes[d] = out.sizes[d];
    if (sz == out.sizes[d]) tr.strides[d] = out.sizes[d] == 1 ? 0 : in.strides[id];
    else if (sz == 1) tr.strides[d] = 0;
    else return false;
  }
  return true;
}

PyObject* submit_task_common(int dev, const Task& t, PyObject* const* keep_objs, int nkeep) {
  gpuos_rt* rt = rt_for(dev);
  if (!rt) return nullptr;
  int st = gpuos_rt_submit_task(rt, &t);
  if (st) return raise_status(st);
  for (int i = 0; i < nkeep; ++i) keep(dev, keep_objs[i]);
  // The reference enqueues these Tasks directly (no flush needed): publish now.
  uint64_t seq = 0;
  st = flush_device(dev, false, &seq);
  if (st) return raise_status(st);
  Py_RETURN_NONE;
}

PyObject* py_submit_unary(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs != 3) {
    PyErr_SetString(PyExc_TypeError, "expected (slot, a, out)");
    return nullptr;
  }
  const long slot = PyLong_AsLong(args[0]);
  if (slot == -1 && PyErr_Occurred()) return nullptr;
  GpuosOperand a, out;
  const int da = to_operand(args[1], &a, "a");
  if (da < 0) return nullptr;
  const int dout = to_operand(args[2], &out, "out");
  if (dout < 0) return nullptr;
  if (da != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  Task t;
  std::memset(&t, 0, sizeof(t));
  t.op = (int)slot;
  t.ndim = out.ndim;
  t.numel = 1;
  for (int d = 0; d < out.ndim; ++d) t.numel *= out.sizes[d];
  fill_ref(t.out0, out);
  if (!fill_ref_bcast(t.in0, a, out)) return PyErr_Format(PyExc_ValueError, "a does not broadcast to out");
  t.in1.data = nullptr;
  t.in1.dtype = t.in0.dtype;
  t.in1.ndim = out.ndim;
  for (int d = 0; d < out.ndim; ++d) t.in1.sizes[d] = 1;
  PyObject* ks[2] = {args[1], args[2]};
  return submit_task_common(dout, t, ks, 2);
}

PyObject* py_submit_binary(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs != 4) {
    PyErr_SetString(PyExc_TypeError, "expected (slot, a, b, out)");
    return nullptr;
  }
  const long slot = PyLong_AsLong(args[0]);
  if (slot == -1 && PyErr_Occurred()) return nullptr;
  GpuosOperand a, b, out;
  const int da = to_operand(args[1], &a, "a");
  if (da < 0) return nullptr;
  const int db = to_operand(args[2], &b, "b");
  if (db < 0) return nullptr;
  const int dout = to_operand(args[3], &out, "out");
  if (dout < 0) return nullptr;
  if (da != dout || db != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  Task t;
  std::memset(&t, 0, sizeof(t));
  t.op = (int)slot;
  t.ndim = out.ndim;
  t.numel = 1;
  for (int d = 0; d < out.ndim; ++d) t.numel *= out.sizes[d];
  fill_ref(t.out0, out);
  if (!fill_ref_bcast(t.in0, a, out) || !fill_ref_bcast(t.in1, b, out))
    return PyErr_Format(PyExc_ValueError, "operands do not broadcast to out");
  PyObject* ks[3] = {args[1], args[2], args[3]};
  return submit_task_common(dout, t, ks, 3);
}

PyObject* py_submit_reduce(PyObject*, PyObject* args) {
  int slot, keepdim;
  PyObject *xo, *oo, *axes_obj;
  if (!PyArg_ParseTuple(args, "iOOOp", &slot, &xo, &oo, &axes_obj, &keepdim)) return nullptr;
  GpuosOperand x, out;
  const int dx = to_operand(xo, &x, "x");
  if (dx < 0) return nullptr;
  const int dout = to_operand(oo, &out, "out");
  if (dout < 0) return nullptr;
  if (dx != dout) {
    PyErr_SetString(PyExc_RuntimeError, "device mismatch");
    return nullptr;
  }
  std::vector<int> axes;
  if (!parse_axes(axes_obj, &axes)) return nullptr;
  if ((int)axes.size() > GPUOS_MAX_NDIM) return PyErr_Format(PyExc_ValueError, "too many axes");
  Task t;
  std::memset(&t, 0, sizeof(t));
  t.op = slot;
  t.ndim = out.ndim;
  t.numel = 1;
  for (int d = 0; d < out.ndim; ++d) t.numel *= out.sizes[d];
  t.rrank = (int)axes.size();
  for (size_t i = 0; i < axes.size(); ++i) {
    int ax = axes[i] < 0 ? axes[i] + x.ndim : axes[i];
    if (ax < 0 || ax >= x.ndim) return PyErr_Format(PyExc_ValueError, "axis %d out of range", axes[i]);
    t.r_axes[i] = ax;
  }
  t.r_keepdim = keepdim;
  fill_ref(t.in0, x);
  fill_ref(t.out0, out);
  t.in1.data = nullptr;
  t.in1.ndim = out.ndim;
  for (int d = 0; d < out.ndim; ++d) t.in1.sizes[d] = 1;
  PyObject* ks[2] = {xo, oo};
  return submit_task_common(dout, t, ks, 2);
}

// submit_topk_rows(x, values, indices, k, largest) — top-k of every row of a contiguous x
// [..., n] into contiguous values [..., k] (x's dtype) and int64 indices [..., k]; pending
// until flush like the other batched requests.
static bool row_major(const at::Tensor& t) { return t.is_contiguous(); }

PyObject* py_submit_topk_rows(PyObject*, PyObject* args) {
  PyObject *xo, *vo, *io;
  int k = 0, largest = 1;
  if (!PyArg_ParseTuple(args, "OOOip", &xo, &vo, &io, &k, &largest)) return nullptr;
  GpuosOperand x, v;
  const int dx = to_operand(xo, &x, "x");
  if (dx < 0) return nullptr;
  const int dv = to_operand(vo, &v, "values");
  if (dv < 0) return nullptr;
  if (!THPVariable_Check(io)) return PyErr_Format(PyExc_TypeError, "indices must be a torch.Tensor");
  const at::Tensor& xt = THPVariable_Unpack(xo);
  const at::Tensor& vt = THPVariable_Unpack(vo);
  const at::Tensor& it = THPVariable_Unpack(io);
  if (!it.is_cuda() || it.get_device() != dx || dv != dx)
    return PyErr_Format(PyExc_RuntimeError, "x, values and indices must be on the same CUDA device");
  if (it.scalar_type() != at::kLong) return PyErr_Format(PyExc_ValueError, "indices must be int64");
  if (vt.scalar_type() != xt.scalar_type()) return PyErr_Format(PyExc_ValueError, "values must have x's dtype");
  if (xt.dim() < 1 || !row_major(xt) || !row_major(vt) || !row_major(it))
    return PyErr_Format(PyExc_ValueError, "x, values and indices must be contiguous");
  const int64_t n = xt.size(-1);
  const int64_t rows = n > 0 ? xt.numel() / n : 0;
  if (vt.numel() != rows * k || it.numel() != rows * k)
    return PyErr_Format(PyExc_ValueError, "values and indices must hold k elements per row of x");
  gpuos_rt* rt = rt_for(dx);
  if (!rt) return nullptr;
  const int st = gpuos_rt_submit_topk(rt, x.data, x.dtype, rows, n, v.data, static_cast<int64_t*>(it.data_ptr()),
                                      k, largest);
  if (st) return raise_status(st);
  keep(dx, xo);
  keep(dx, vo);
  keep(dx, io);
  Py_RETURN_NONE;
}

// submit_many(ops, a, b, out) — many element-wise requests in one call: a, b and out are
// sequences of tensors of one length (b may be None when every op is unary), ops one op code
// or a sequence of codes.  Nothing is submitted if any request is invalid.
struct FastSeq {
  PyObject* o = nullptr;
  ~FastSeq() { Py_XDECREF(o); }
};

PyObject* py_submit_many(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
  if (nargs != 4) {
    PyErr_SetString(PyExc_TypeError, "expected (ops, a, b, out)");
    return nullptr;
  }
  FastSeq fa, fb, fo, fops;
  if (!(fa.o = PySequence_Fast(args[1], "a must be a sequence of tensors"))) return nullptr;
  if (args[2] != Py_None && !(fb.o = PySequence_Fast(args[2], "b must be a sequence of tensors or None")))
    return nullptr;
  if (!(fo.o = PySequence_Fast(args[3], "out must be a sequence of tensors"))) return nullptr;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fa.o);
  if (PySequence_Fast_GET_SIZE(fo.o) != n || (fb.o && PySequence_Fast_GET_SIZE(fb.o) != n))
    return PyErr_Format(PyExc_ValueError, "a, b and out must have the same length");
  long op_all = -1;
  if (PyLong_Check(args[0])) {
    op_all = PyLong_AsLong(args[0]);
  } else {
    if (!(fops.o = PySequence_Fast(args[0], "ops must be an op code or a sequence of op codes"))) return nullptr;
    if (PySequence_Fast_GET_SIZE(fops.o) != n) return PyErr_Format(PyExc_ValueError, "ops must have one code per request");
  }
  if (n == 0) Py_RETURN_NONE;
  static thread_local std::vector<GpuosOperand> va, vb, vo;
  static thread_local std::vector<int> vops;
  va.resize((size_t)n);
  vb.resize((size_t)n);
  vo.resize((size_t)n);
  vops.resize((size_t)n);
  PyObject** ia = PySequence_Fast_ITEMS(fa.o);
  PyObject** ib = fb.o ? PySequence_Fast_ITEMS(fb.o) : nullptr;
  PyObject** io = PySequence_Fast_ITEMS(fo.o);
  int dev = -1;
  for (Py_ssize_t i = 0; i < n; ++i) {
    if (fops.o) {
      const long v = PyLong_AsLong(PySequence_Fast_GET_ITEM(fops.o, i));
      if (v == -1 && PyErr_Occurred()) return nullptr;
      vops[(size_t)i] = (int)v;
    } else {
      vops[(size_t)i] = (int)op_all;
    }
    const int d1 = to_operand(ia[i], &va[(size_t)i], "a");
    if (d1 < 0) return nullptr;
    const int d3 = to_operand(io[i], &vo[(size_t)i], "out");
    if (d3 < 0) return nullptr;
    int d2 = d1;
    if (ib && (d2 = to_operand(ib[i], &vb[(size_t)i], "b")) < 0) return nullptr;
    if (dev < 0) dev = d1;
    if (d1 != dev || d2 != dev || d3 != dev) return PyErr_Format(PyExc_RuntimeError, "device mismatch");
  }
  gpuos_rt* rt = rt_for(dev);
  if (!rt) return nullptr;
  const int st = gpuos_rt_submit_ew_many(rt, (int)n, vops.data(), va.data(), ib ? vb.data() : nullptr, vo.data());
  if (st) return raise_status(st);
  for (Py_ssize_t i = 0; i < n; ++i) {
    keep(dev, ia[i]);
    if (ib) keep(dev, ib[i]);
    keep(dev, io[i]);
  }
  Py_RETURN_NONE;
}

PyMethodDef kMethods[] = {
    {"init", (PyCFunction)(void (*)(void))py_init, METH_VARARGS | METH_KEYWORDS,
     "init(capacity=4096, threads_per_block=256, device=None)"},
    {"shutdown", (PyCFunction)(void (*)(void))py_shutdown, METH_VARARGS | METH_KEYWORDS, "shutdown(device=None)"},
    {"abi_version", py_abi_version, METH_NOARGS, "extension ABI version"},
    {"set_debug_level", py_set_debug_level, METH_VARARGS, "device debug print level"},
    {"set_verbose_level", py_set_verbose_level, METH_VARARGS, "host verbose level"},
    {"peek_queue", (PyCFunction)(void (*)(void))py_peek_queue, METH_VARARGS | METH_KEYWORDS, "queue state dict"},
    {"set_yield_every", py_set_yield_every, METH_VARARGS, "worker exits after every N items (0 = never)"},
    {"set_idle_quiesce_ms", py_set_idle_quiesce_ms, METH_VARARGS, "stop an idle worker after ms (0 = after every drain, -1 = never)"},
    {"worker_alive", (PyCFunction)(void (*)(void))py_worker_alive, METH_VARARGS | METH_KEYWORDS, "worker kernel running"},
    {"quiesce", (PyCFunction)(void (*)(void))py_quiesce, METH_VARARGS | METH_KEYWORDS, "drain and stop the worker"},
    {"submit_add", (PyCFunction)(void (*)(void))py_submit_add, METH_FASTCALL, "out = a + b (pending until flush)"},
    {"submit_mul", (PyCFunction)(void (*)(void))py_submit_mul, METH_FASTCALL, "out = a * b (pending until flush)"},
    {"submit_sub", (PyCFunction)(void (*)(void))py_submit_sub, METH_FASTCALL, "out = a - b (pending until flush)"},
    {"submit_div", (PyCFunction)(void (*)(void))py_submit_div, METH_FASTCALL, "out = a / b (pending until flush)"},
    {"submit_ew_new", (PyCFunction)(void (*)(void))py_submit_ew_new, METH_FASTCALL,
     "submit_ew_new(op, a, b[, p0[, p1]]) -> out: element-wise request into a new contiguous tensor like a"},
    {"submit_elementwise", (PyCFunction)(void (*)(void))py_submit_elementwise, METH_FASTCALL,
     "submit_elementwise(op, a, b, out, p0=0.0, p1=0.0)"},
    {"submit_topk_rows", py_submit_topk_rows, METH_VARARGS,
     "submit_topk_rows(x, values, indices, k, largest): top-k of each row of x (pending until flush)"},
    {"submit_many", (PyCFunction)(void (*)(void))py_submit_many, METH_FASTCALL,
     "submit_many(ops, a, b, out): many element-wise requests in one call (pending until flush)"},
    {"submit_reduction", (PyCFunction)(void (*)(void))py_submit_reduction, METH_FASTCALL,
     "submit_reduction(op, x, out, axes, keepdim)"},
    {"flush", (PyCFunction)(void (*)(void))py_flush, METH_VARARGS | METH_KEYWORDS, "flush(sync=False, device=None) -> ticket"},
    {"wait", (PyCFunction)(void (*)(void))py_wait, METH_VARARGS | METH_KEYWORDS, "wait(seq, timeout_ms=30000, device=None)"},
    {"completed", (PyCFunction)(void (*)(void))py_completed, METH_VARARGS | METH_KEYWORDS, "highest completed ticket"},
    {"flush_times", (PyCFunction)(void (*)(void))py_flush_times, METH_VARARGS | METH_KEYWORDS,
     "device (t_start_ns, t_end_ns) of a completed flush"},
    {"kernel_stream", (PyCFunction)(void (*)(void))py_kernel_stream, METH_VARARGS | METH_KEYWORDS,
     "raw handle of the worker kernel's stream"},
    {"launches", (PyCFunction)(void (*)(void))py_launches, METH_VARARGS | METH_KEYWORDS, "worker launches so far"},
    {"set_device_wait_ms", py_set_device_wait_ms, METH_VARARGS, "bound of the worker's in-grid waits"},
    {"debug_timeline", (PyCFunction)(void (*)(void))py_debug_timeline, METH_VARARGS | METH_KEYWORDS,
     "debug_timeline(device=None) -> [12 %globaltimer stamps of the last launch's first events]"},
    {"set_launch_timing", (PyCFunction)(void (*)(void))py_set_launch_timing, METH_VARARGS | METH_KEYWORDS,
     "set_launch_timing(on, device=None): bracket every worker launch with CUDA events"},
    {"launch_times", (PyCFunction)(void (*)(void))py_launch_times, METH_VARARGS | METH_KEYWORDS,
     "launch_times(device=None) -> [ms of each finished timed launch, oldest first]"},
    {"debug_counters", (PyCFunction)(void (*)(void))py_debug_counters, METH_VARARGS | METH_KEYWORDS,
     "per-CTA cycle counters of the last worker launch"},
    {"debug_inject_stall", (PyCFunction)(void (*)(void))py_debug_inject_stall, METH_VARARGS | METH_KEYWORDS,
     "publish an item whose dependency barrier never opens (failure-path test)"},
    {"submit_unary", (PyCFunction)(void (*)(void))py_submit_unary, METH_FASTCALL, "submit_unary(slot, a, out)"},
    {"submit_binary", (PyCFunction)(void (*)(void))py_submit_binary, METH_FASTCALL, "submit_binary(slot, a, b, out)"},
    {"submit_reduce", py_submit_reduce, METH_VARARGS, "submit_reduce(slot, x, out, axes, keepdim)"},
    {"set_slot", (PyCFunction)(void (*)(void))py_set_slot, METH_VARARGS | METH_KEYWORDS, "write a device function address into a slot"},
    {"get_slot", (PyCFunction)(void (*)(void))py_get_slot, METH_VARARGS | METH_KEYWORDS, "read a slot"},
    {"set_alias", (PyCFunction)(void (*)(void))py_set_alias, METH_VARARGS | METH_KEYWORDS, "route logical op to a physical slot"},
    {"get_alias", (PyCFunction)(void (*)(void))py_get_alias, METH_VARARGS | METH_KEYWORDS, "read an alias"},
    {"builtin_op_address", (PyCFunction)(void (*)(void))py_builtin_op_address, METH_VARARGS | METH_KEYWORDS,
     "device address of a built-in reference-ABI operator"},
    {"register_builtin", (PyCFunction)(void (*)(void))py_register_builtin, METH_VARARGS | METH_KEYWORDS,
     "register_builtin(kind, op) -> slot"},
    {"register_expr", (PyCFunction)(void (*)(void))py_register_expr, METH_VARARGS | METH_KEYWORDS,
     "register_expr(key, expr, arity, slot=-1): expression operator run by the worker's interpreter"},
    {"register_jit", (PyCFunction)(void (*)(void))py_register_jit, METH_VARARGS | METH_KEYWORDS,
     "register_jit(expr, arity, slot=-1): NVRTC-compile an expression operator for sm_100a, link it "
     "into the worker, install it in a slot"},
    {"load_custom", (PyCFunction)(void (*)(void))py_load_custom, METH_VARARGS | METH_KEYWORDS,
     "load_custom(ptx, entry, slot=-1): link PTX holding extern \"C\" __device__ void entry(const Task&) "
     "into the worker, install entry in a slot"},
    {"jit_stage", (PyCFunction)(void (*)(void))py_jit_stage, METH_VARARGS | METH_KEYWORDS,
     "jit_stage(expr, arity) -> staged operator (compiled and linked; the worker keeps running)"},
    {"jit_commit", (PyCFunction)(void (*)(void))py_jit_commit, METH_VARARGS | METH_KEYWORDS,
     "jit_commit(staged, slot=-1) -> slot (stops the worker, loads the module, installs the operator)"},
    {"jit_ops", (PyCFunction)(void (*)(void))py_jit_ops, METH_VARARGS | METH_KEYWORDS,
     "operators compiled at run time installed on the device"},
    {"jit_compile", (PyCFunction)(void (*)(void))py_jit_compile, METH_VARARGS | METH_KEYWORDS,
     "jit_compile(src, ptx=False): NVRTC output for sm_100a (no device needed)"},
    {"jit_check_expr", py_jit_check_expr, METH_VARARGS,
     "jit_check_expr(expr, arity) -> linked image bytes (no device needed)"},
    {"jit_nvrtc_version", py_jit_nvrtc_version, METH_NOARGS, "NVRTC version in use (major*1000+minor*10)"},
    {"sync_poll_processed", py_sync_poll_processed, METH_NOARGS, "completed requests (zero-copy)"},
    {"sync_poll_heartbeat", py_sync_poll_heartbeat, METH_NOARGS, "worker heartbeat (zero-copy)"},
    {"sync_poll_ready", py_sync_poll_ready, METH_NOARGS, "worker ready (zero-copy)"},
    {"sync_wait", (PyCFunction)(void (*)(void))py_sync_wait, METH_VARARGS | METH_KEYWORDS,
     "sync_wait(target, timeout_ms=30000)"},
    {"sync_enabled", py_sync_enabled, METH_NOARGS, "zero-copy sync available"},
    {"intercept_enable", py_intercept_enable, METH_VARARGS,
     "intercept_enable(size_threshold): route this thread's ATen calls through the C++ scheduler intercept"},
    {"intercept_disable", py_intercept_disable, METH_NOARGS, "stop intercepting this thread's ATen calls"},
    {"intercept_enabled", py_intercept_enabled, METH_NOARGS, "whether this thread's ATen calls are intercepted"},
    {"intercept_stats", py_intercept_stats, METH_NOARGS,
     "intercept counters: scheduled, fallbacks, scheduled_ops, fallback_ops"},
    {"intercept_routes", py_intercept_routes, METH_NOARGS,
     "the intercept's routing table: aten op name -> (kind, op code)"},
    {"intercept_clear_pending", py_intercept_clear_pending, METH_NOARGS,
     "forget the intercept's pending storages (after a synchronous flush)"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_gpuos_ext", "B200 persistent micro-op runtime binding", -1,
                       kMethods};

}  // namespace

namespace gpuos_py {
gpuos_rt* runtime(int dev) { return dev >= 0 && dev < kMaxDev ? g_rt[dev] : nullptr; }
void busy_add(int dev, int delta) { g_busy[dev].fetch_add(delta); }
}  // namespace gpuos_py

PyMODINIT_FUNC PyInit__gpuos_ext(void) {
  PyObject* m = PyModule_Create(&kModule);
  if (!m) return nullptr;
  struct {
    const char* n;
    int v;
  } consts[] = {{"EW_ADD", GPUOS_EW_ADD},
                {"EW_MUL", GPUOS_EW_MUL},
                {"EW_SUB", GPUOS_EW_SUB},
                {"EW_DIV", GPUOS_EW_DIV},
                {"EW_MAXIMUM", GPUOS_EW_MAXIMUM},
                {"EW_MINIMUM", GPUOS_EW_MINIMUM},
                {"EW_POW", GPUOS_EW_POW},
                {"EW_COPY", GPUOS_EW_COPY},
                {"EW_RELU", GPUOS_EW_RELU},
                {"EW_SIGMOID", GPUOS_EW_SIGMOID},
                {"EW_TANH", GPUOS_EW_TANH},
                {"EW_EXP", GPUOS_EW_EXP},
                {"EW_LOG", GPUOS_EW_LOG},
                {"EW_SQRT", GPUOS_EW_SQRT},
                {"EW_ABS", GPUOS_EW_ABS},
                {"EW_HARDSIGMOID", GPUOS_EW_HARDSIGMOID},
                {"EW_HARDSWISH", GPUOS_EW_HARDSWISH},
                {"EW_GELU", GPUOS_EW_GELU},
                {"EW_GELU_TANH", GPUOS_EW_GELU_TANH},
                {"EW_SIN", GPUOS_EW_SIN},
                {"EW_COS", GPUOS_EW_COS},
                {"EW_LEAKY_RELU", GPUOS_EW_LEAKY_RELU},
                {"EW_CLAMP", GPUOS_EW_CLAMP},
                {"EW_CLAMP_MIN", GPUOS_EW_CLAMP_MIN},
                {"EW_CLAMP_MAX", GPUOS_EW_CLAMP_MAX},
                {"EW_ELU", GPUOS_EW_ELU},
                {"EW_SOFTPLUS", GPUOS_EW_SOFTPLUS},
                {"EW_NEG", GPUOS_EW_NEG},
                {"EW_ADD_ALPHA", GPUOS_EW_ADD_ALPHA},
                {"EW_SUB_ALPHA", GPUOS_EW_SUB_ALPHA},
                {"EW_NUM_OPS", GPUOS_EW_NUM_OPS},
                {"RED_SUM", GPUOS_RED_SUM},
                {"RED_MEAN", GPUOS_RED_MEAN},
                {"GPUOS_MAX_OPS", GPUOS_MAX_OPS}};
  for (auto& c : consts) PyModule_AddIntConstant(m, c.n, c.v);
  return m;
}
