// intercept.cpp — scheduler_context's op intercept as a boxed dispatcher fallback in C++.
//
// Reference: pytorch_ext/scheduler.py:162-373, a Python TorchDispatchMode that sends small
// pointwise ops, sum/mean and topk to the runtime and everything else to PyTorch.  The Python
// mode in gpuos_b200/scheduler.py keeps that form; this file routes the same ops by the same
// rules without a Python call per op:
//
//   * A boxed fallback is registered (once, on first use) for the dispatcher key
//     TESTING_ONLY_GenericMode, and scheduler_context includes that key in the entering
//     thread's thread-local dispatch key set.  It is the one functionality key above the backend
//     kernels that a library can switch on per thread without taking one PyTorch itself drives
//     (Python, PreDispatch, functorch, autocast); if another library in the process has already
//     registered a fallback for it, enabling fails and the Python mode is used instead.
//   * The key sits above autograd.  Ops are scheduled only with grad mode off (as the Python
//     mode) and only when every key of the call is a plain dense one (no tensor subclass,
//     Python mode, functorch transform, autocast, conjugate/negative view, sparse layout).
//     Ops that PyTorch decomposes at the autograd level (CompositeImplicitAutograd) pass
//     through with the key kept, so their parts come back here one by one, as the Python mode
//     (which sits below autograd) sees them; every other op that is not scheduled runs below
//     this key with the key excluded, so the kernels it calls internally are not intercepted.
//   * Scheduled requests keep their tensors (at::Tensor references) until the flush that
//     carries them completes, and mark their storages pending.  An op left to PyTorch that
//     touches a pending storage first flushes and waits; a non-view op that launches a kernel
//     and reads or writes CUDA memory also stops the resident worker (it holds every SM until
//     its idle stop), exactly as the Python mode does.
//   * PyTorch's bindings release the GIL before dispatching, so nothing here touches Python
//     objects; the binding's auto-flush thread may flush concurrently (intercept_flush).
#include "intercept.h"

#include <ATen/ExpandUtils.h>
#include <ATen/core/Tensor.h>
#include <ATen/core/dispatch/Dispatcher.h>
#include <ATen/core/stack.h>
#include <ATen/cuda/EmptyTensor.h>
#include <ATen/ops/result_type.h>
#include <c10/core/GradMode.h>
#include <c10/core/impl/LocalDispatchKeySet.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <algorithm>
#include <atomic>
#include <deque>
#include <mutex>
#include <unordered_map>
#include <unordered_set>

namespace gpuos_py {
namespace {

constexpr c10::DispatchKey kKey = c10::DispatchKey::TESTING_ONLY_GenericMode;
const c10::DispatchKeySet kBelow(c10::DispatchKeySet::FULL_AFTER, kKey);

enum Kind : uint8_t { K_NONE, K_BINARY, K_UNARY, K_PARAM, K_REDUCE, K_TOPK };

// Per-operator routing, built the first time an operator comes through.
struct Route {
  std::string name;        // "aten::add.Tensor", "aten::relu" (the Python mode's func.name())
  Kind kind = K_NONE;
  int code = 0;            // element-wise op (binary, unary) or reduction op
  bool add_sub = false;    // add.Tensor / sub.Tensor (the alpha argument)
  bool composite = false;  // CompositeImplicitAutograd: decomposed at the autograd level
  bool no_kernel = false;  // a view or an allocation: launches nothing, needs no SM
  int64_t scheduled = 0;   // counters since the intercept was enabled (under g_mu)
  int64_t fallbacks = 0;
};

struct DevRefs {
  std::vector<at::Tensor> pending;                                // requests not yet flushed
  std::deque<std::pair<uint64_t, std::vector<at::Tensor>>> inflight;  // by flush ticket
};

std::mutex g_mu;  // guards everything below
std::unordered_map<c10::OperatorHandle, Route*> g_routes;  // entries live as long as the process
std::unordered_set<uintptr_t> g_pending;  // storages read or written by requests not known complete
DevRefs g_refs[kMaxDev];
int64_t g_scheduled = 0, g_fallbacks = 0;
std::atomic<int64_t> g_threshold{int64_t(1) << 16};
torch::Library* g_lib = nullptr;

// Same tables as the Python mode (gpuos_b200/scheduler.py _BINARY/_UNARY/_PARAMETRIC/_REDUCE).
const std::unordered_map<std::string, std::pair<Kind, int>>& route_table() {
  static const std::unordered_map<std::string, std::pair<Kind, int>> table = {
      {"aten::add.Tensor", {K_BINARY, GPUOS_EW_ADD}},
      {"aten::sub.Tensor", {K_BINARY, GPUOS_EW_SUB}},
      {"aten::mul.Tensor", {K_BINARY, GPUOS_EW_MUL}},
      {"aten::div.Tensor", {K_BINARY, GPUOS_EW_DIV}},
      {"aten::maximum", {K_BINARY, GPUOS_EW_MAXIMUM}},
      {"aten::minimum", {K_BINARY, GPUOS_EW_MINIMUM}},
      {"aten::pow.Tensor_Tensor", {K_BINARY, GPUOS_EW_POW}},
      {"aten::pow.Tensor_Scalar", {K_BINARY, GPUOS_EW_POW}},
      {"aten::relu", {K_UNARY, GPUOS_EW_RELU}},
      {"aten::sigmoid", {K_UNARY, GPUOS_EW_SIGMOID}},
      {"aten::tanh", {K_UNARY, GPUOS_EW_TANH}},
      {"aten::exp", {K_UNARY, GPUOS_EW_EXP}},
      {"aten::log", {K_UNARY, GPUOS_EW_LOG}},
      {"aten::sqrt", {K_UNARY, GPUOS_EW_SQRT}},
      {"aten::abs", {K_UNARY, GPUOS_EW_ABS}},
      {"aten::hardsigmoid", {K_UNARY, GPUOS_EW_HARDSIGMOID}},
      {"aten::hardswish", {K_UNARY, GPUOS_EW_HARDSWISH}},
      {"aten::sin", {K_UNARY, GPUOS_EW_SIN}},
      {"aten::cos", {K_UNARY, GPUOS_EW_COS}},
      {"aten::neg", {K_UNARY, GPUOS_EW_NEG}},
      {"aten::gelu", {K_PARAM, 0}},
      {"aten::leaky_relu", {K_PARAM, 0}},
      {"aten::hardtanh", {K_PARAM, 0}},
      {"aten::elu", {K_PARAM, 0}},
      {"aten::softplus", {K_PARAM, 0}},
      {"aten::clamp", {K_PARAM, 0}},
      {"aten::clamp_min", {K_PARAM, 0}},
      {"aten::clamp_max", {K_PARAM, 0}},
      {"aten::sum.dim_IntList", {K_REDUCE, GPUOS_RED_SUM}},
      {"aten::mean.dim", {K_REDUCE, GPUOS_RED_MEAN}},
      {"aten::sum", {K_REDUCE, GPUOS_RED_SUM}},
      {"aten::mean", {K_REDUCE, GPUOS_RED_MEAN}},
      {"aten::topk", {K_TOPK, 0}},
  };
  return table;
}

void classify(Route* r) {
  const auto& table = route_table();
  // allocations that launch no kernel (views are recognised from the schema)
  static const std::unordered_set<std::string> alloc = {
      "aten::empty.memory_format", "aten::empty_like", "aten::empty_strided", "aten::new_empty",
      "aten::new_empty_strided"};
  auto it = table.find(r->name);
  if (it != table.end()) {
    r->kind = it->second.first;
    r->code = it->second.second;
  }
  r->add_sub = r->name == "aten::add.Tensor" || r->name == "aten::sub.Tensor";
  r->no_kernel = alloc.count(r->name) != 0;
}

Route* route_of(const c10::OperatorHandle& op) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_routes.find(op);
  if (it != g_routes.end()) return it->second;
  Route* r = new Route();
  const c10::OperatorName& on = op.operator_name();
  r->name = on.overload_name.empty() ? on.name : on.name + "." + on.overload_name;
  classify(r);
  r->composite = op.hasKernelForDispatchKey(c10::DispatchKey::CompositeImplicitAutograd);
  const auto& rets = op.schema().returns();
  if (!rets.empty() && rets[0].alias_info() != nullptr && !rets[0].alias_info()->isWrite()) r->no_kernel = true;
  g_routes.emplace(op, r);
  return r;
}

// Every key of the call is a plain dense one (see the file comment).
bool plain(c10::DispatchKeySet ks) {
  for (c10::DispatchKey k : ks) {
    switch (c10::toFunctionalityKey(k)) {
      case kKey:
      case c10::DispatchKey::Dense:
      case c10::DispatchKey::BackendSelect:
      case c10::DispatchKey::ADInplaceOrView:
      case c10::DispatchKey::AutogradFunctionality:
        break;
      default:
        return false;
    }
  }
  return true;
}

int dtype_code(c10::ScalarType st) {
  switch (st) {
    case c10::ScalarType::Float: return kF32;
    case c10::ScalarType::Half: return kF16;
    case c10::ScalarType::BFloat16: return kBF16;
    default: return -1;
  }
}

// A CUDA tensor of a floating dtype within the size threshold and the rank limit.
bool ok_tensor(const at::Tensor& t, int64_t thr) {
  return t.defined() && t.is_cuda() && dtype_code(t.scalar_type()) >= 0 && t.numel() <= thr &&
         t.dim() <= GPUOS_MAX_NDIM;
}

void to_operand(const at::Tensor& t, GpuosOperand* o) {
  o->data = const_cast<void*>(t.const_data_ptr());
  o->dtype = dtype_code(t.scalar_type());
  o->ndim = (int)t.dim();
  const auto sz = t.sizes();
  const auto st = t.strides();
  for (int d = 0; d < o->ndim; ++d) {
    o->sizes[d] = sz[d];
    o->strides[d] = st[d];
  }
}

// Base address of the tensor's storage (the Python mode's data_ptr - offset * itemsize).
uintptr_t storage_key(const at::Tensor& t) { return reinterpret_cast<uintptr_t>(t.storage().data()); }

// A real number argument (Python's float(v) of an int, float or bool); false otherwise.
bool number(const c10::IValue& v, double* out) {
  if (v.isDouble()) *out = v.toDouble();
  else if (v.isInt()) *out = (double)v.toInt();
  else if (v.isBool()) *out = v.toBool() ? 1.0 : 0.0;
  else return false;
  return true;
}

// The value of a 0-dim CPU tensor (a wrapped Python number), as the Python mode's b.item().
bool cpu_scalar(const at::Tensor& t, double* v) {
  const void* p = t.const_data_ptr();
  switch (t.scalar_type()) {
    case c10::ScalarType::Double: *v = *static_cast<const double*>(p); return true;
    case c10::ScalarType::Float: *v = *static_cast<const float*>(p); return true;
    case c10::ScalarType::Half: *v = static_cast<float>(*static_cast<const c10::Half*>(p)); return true;
    case c10::ScalarType::BFloat16: *v = static_cast<float>(*static_cast<const c10::BFloat16*>(p)); return true;
    case c10::ScalarType::Long: *v = (double)*static_cast<const int64_t*>(p); return true;
    case c10::ScalarType::Int: *v = (double)*static_cast<const int32_t*>(p); return true;
    case c10::ScalarType::Short: *v = (double)*static_cast<const int16_t*>(p); return true;
    case c10::ScalarType::Char: *v = (double)*static_cast<const int8_t*>(p); return true;
    case c10::ScalarType::Byte: *v = (double)*static_cast<const uint8_t*>(p); return true;
    case c10::ScalarType::Bool: *v = *static_cast<const bool*>(p) ? 1.0 : 0.0; return true;
    default: return false;  // complex and the rest: not a number the runtime takes
  }
}

// A new contiguous CUDA tensor: the allocation at::empty's CUDA kernel makes (the caching
// allocator on the current stream), without the dispatcher's hops to reach it.
at::Tensor new_cuda(c10::IntArrayRef sizes, c10::ScalarType dt, c10::Device dev) {
  return at::Tensor(at::detail::empty_cuda(sizes, dt, dev, at::MemoryFormat::Contiguous));
}

struct BusyGuard {
  int d;
  explicit BusyGuard(int dev) : d(dev) { busy_add(d, 1); }
  ~BusyGuard() { busy_add(d, -1); }
};

// f(dev, rt) for every device with a runtime, each call under the device's busy count (the
// runtime is read again after the count is raised: shutdown clears it first, then waits).
template <typename F>
void each_runtime(F&& f) {
  for (int d = 0; d < kMaxDev; ++d) {
    if (!runtime(d)) continue;
    BusyGuard busy(d);
    gpuos_rt* rt = runtime(d);
    if (rt && !f(d, rt)) return;
  }
}

void check(int st) {
  if (st) {
    const char* msg = gpuos_rt_last_error();
    TORCH_CHECK(false, "gpuos: ", (msg && *msg) ? msg : "runtime error");
  }
}

// Record a submitted request: references until its flush completes, storages pending.
void record(Route* r, int dev, std::initializer_list<const at::Tensor*> ts) {
  DevRefs& R = g_refs[dev];
  for (const at::Tensor* t : ts) {
    R.pending.push_back(*t);
    g_pending.insert(storage_key(*t));
  }
  ++g_scheduled;
  ++r->scheduled;
}

// Replace the call's arguments on the stack by its results.
void finish(torch::jit::Stack* stack, size_t nargs, at::Tensor out) {
  torch::jit::drop(*stack, nargs);
  torch::jit::push(*stack, std::move(out));
}

// An element-wise request into `out`; false (nothing submitted) when the runtime declines it.
bool submit_ew(Route* r, int op, const at::Tensor& a, const at::Tensor* b, bool b_scalar, double b_val,
               const at::Tensor& out, float p0, float p1) {
  const int dev = out.get_device();
  if (dev < 0 || dev >= kMaxDev) return false;
  GpuosOperand A, B, O;
  to_operand(a, &A);
  if (b) to_operand(*b, &B);
  to_operand(out, &O);
  const float params[2] = {p0, p1};
  BusyGuard busy(dev);
  gpuos_rt* rt = runtime(dev);
  if (!rt) return false;
  std::lock_guard<std::mutex> lk(g_mu);
  if (gpuos_rt_submit_ew(rt, op, &A, b ? &B : nullptr, b_scalar ? 1 : 0, b_val, &O, params, 2)) return false;
  if (b) record(r, dev, {&a, b, &out});
  else record(r, dev, {&a, &out});
  return true;
}

// aten::add.Tensor(self, other, *, alpha) and the other binary ops (scheduler.py:221-290).
bool try_binary(Route* r, c10::IValue* args, size_t nargs, torch::jit::Stack* stack, int64_t thr) {
  if (nargs < 2 || !args[0].isTensor()) return false;
  const at::Tensor& a = args[0].toTensor();
  if (!ok_tensor(a, thr)) return false;
  at::Tensor b;
  bool b_t = false;
  double bv = 0.0;
  if (args[1].isTensor()) {
    const at::Tensor& bt = args[1].toTensor();
    if (bt.dim() == 0 && !bt.is_cuda()) {
      if (!cpu_scalar(bt, &bv)) return false;
    } else {
      if (!ok_tensor(bt, thr) || bt.get_device() != a.get_device()) return false;
      b = bt;
      b_t = true;
    }
  } else if (!number(args[1], &bv)) {
    return false;
  }
  int op = r->code;
  double p0 = 0.0;
  if (r->add_sub && nargs >= 3) {
    double al;
    if (!number(args[2], &al)) return false;
    if (al != 1.0) {
      const bool add = r->code == GPUOS_EW_ADD;
      if (b_t) {
        op = add ? GPUOS_EW_ADD_ALPHA : GPUOS_EW_SUB_ALPHA;
        p0 = al;
      } else {
        bv *= al;  // a + alpha * scalar folds into a scalar operand
      }
    }
  }
  c10::ScalarType dt = a.scalar_type();
  std::vector<int64_t> shape;
  bool same_shape = true;
  if (b_t) {
    if (!b.sizes().equals(a.sizes())) {
      try {
        shape = at::infer_size(a.sizes(), b.sizes());
      } catch (const c10::Error&) {
        return false;
      }
      same_shape = c10::IntArrayRef(shape).equals(a.sizes());
    }
    if (b.scalar_type() != dt) dt = at::result_type(a, b);
  }
  if (dtype_code(dt) < 0) return false;
  at::Tensor out = new_cuda(same_shape ? a.sizes() : c10::IntArrayRef(shape), dt, a.device());
  if (!submit_ew(r, op, a, b_t ? &b : nullptr, !b_t, bv, out, (float)p0, 0.f)) return false;
  finish(stack, nargs, std::move(out));
  return true;
}

// Parametric unary ops: (op code, p0, p1) from the arguments (scheduler.py:244-290).
bool param_code(const Route* r, const c10::IValue* args, size_t nargs, int* op, double* p0, double* p1) {
  const std::string& n = r->name;
  auto num = [&](size_t i, double* v) { return i < nargs && number(args[i], v); };
  *p0 = *p1 = 0.0;
  if (n == "aten::gelu") {
    const bool tanh = nargs > 1 && args[1].isString() && args[1].toStringRef() == "tanh";
    *op = tanh ? GPUOS_EW_GELU_TANH : GPUOS_EW_GELU;
    return true;
  }
  if (n == "aten::leaky_relu") {
    *op = GPUOS_EW_LEAKY_RELU;
    return num(1, p0);
  }
  if (n == "aten::hardtanh") {
    *op = GPUOS_EW_CLAMP;
    return num(1, p0) && num(2, p1);
  }
  if (n == "aten::elu") {
    double scale, iscale;
    if (!num(1, p0) || !num(2, &scale) || !num(3, &iscale) || scale != 1.0 || iscale != 1.0) return false;
    *op = GPUOS_EW_ELU;
    return true;
  }
  if (n == "aten::softplus") {
    *op = GPUOS_EW_SOFTPLUS;
    return num(1, p0) && num(2, p1);
  }
  if (n == "aten::clamp") {
    const bool lo = nargs > 1 && !args[1].isNone(), hi = nargs > 2 && !args[2].isNone();
    if (lo && hi) {
      *op = GPUOS_EW_CLAMP;
      return num(1, p0) && num(2, p1);
    }
    if (lo) {
      *op = GPUOS_EW_CLAMP_MIN;
      return num(1, p0);
    }
    if (hi) {
      *op = GPUOS_EW_CLAMP_MAX;
      return num(2, p0);
    }
    return false;
  }
  if (n == "aten::clamp_min") {
    *op = GPUOS_EW_CLAMP_MIN;
    return num(1, p0);
  }
  if (n == "aten::clamp_max") {
    *op = GPUOS_EW_CLAMP_MAX;
    return num(1, p0);
  }
  return false;
}

// Unary and parametric unary ops into a new contiguous tensor like x.
bool try_unary(Route* r, c10::IValue* args, size_t nargs, torch::jit::Stack* stack, int64_t thr) {
  if (nargs < 1 || !args[0].isTensor()) return false;
  const at::Tensor& x = args[0].toTensor();
  if (!ok_tensor(x, thr)) return false;
  int op = r->code;
  double p0 = 0.0, p1 = 0.0;
  if (r->kind == K_PARAM && !param_code(r, args, nargs, &op, &p0, &p1)) return false;
  at::Tensor out = new_cuda(x.sizes(), x.scalar_type(), x.device());
  if (!submit_ew(r, op, x, nullptr, false, 0.0, out, (float)p0, (float)p1)) return false;
  finish(stack, nargs, std::move(out));
  return true;
}

// sum / mean over dims (scheduler.py:292-344).
bool try_reduce(Route* r, c10::IValue* args, size_t nargs, torch::jit::Stack* stack, int64_t thr) {
  if (nargs < 1 || !args[0].isTensor()) return false;
  const at::Tensor& x = args[0].toTensor();
  if (!ok_tensor(x, thr)) return false;
  const bool all = r->name == "aten::sum" || r->name == "aten::mean";
  // dtype: the last argument of every overload; None or x's own dtype
  const c10::IValue& dtv = args[nargs - 1];
  if (!dtv.isNone() && (!dtv.isInt() || dtv.toScalarType() != x.scalar_type())) return false;
  std::vector<int64_t> dims;
  bool keepdim = false;
  if (!all) {
    if (nargs < 4) return false;
    if (args[1].isIntList()) dims = args[1].toIntVector();
    else if (!args[1].isNone()) return false;
    if (!args[2].isBool()) return false;
    keepdim = args[2].toBool();
  }
  const int64_t nd = x.dim();
  std::vector<int> red;
  for (int64_t d : dims) {
    const int64_t e = d < 0 ? d + nd : d;
    if (e < 0 || e >= nd) return false;
    red.push_back((int)e);
  }
  std::sort(red.begin(), red.end());
  red.erase(std::unique(red.begin(), red.end()), red.end());
  if (red.empty())
    for (int d = 0; d < nd; ++d) red.push_back(d);
  std::vector<int64_t> shape;
  for (int64_t d = 0; d < nd; ++d) {
    const bool reduced = std::binary_search(red.begin(), red.end(), (int)d);
    if (!reduced) shape.push_back(x.size(d));
    else if (keepdim) shape.push_back(1);
  }
  at::Tensor out = new_cuda(shape, x.scalar_type(), x.device());
  const int dev = x.get_device();
  if (dev < 0 || dev >= kMaxDev) return false;
  GpuosOperand X, O;
  to_operand(x, &X);
  to_operand(out, &O);
  {
    BusyGuard busy(dev);
    gpuos_rt* rt = runtime(dev);
    if (!rt) return false;
    std::lock_guard<std::mutex> lk(g_mu);
    if (gpuos_rt_submit_reduce(rt, r->code, &X, &O, red.data(), (int)red.size(), keepdim ? 1 : 0)) return false;
    record(r, dev, {&x, &out});
  }
  finish(stack, nargs, std::move(out));
  return true;
}

// topk(self, k, dim=-1, largest=True, sorted=True) along the last dim of a contiguous tensor,
// 1 <= k <= min(n, 256) (scheduler.py:346-370 sends topk to torch::topk).
bool try_topk(Route* r, c10::IValue* args, size_t nargs, torch::jit::Stack* stack, int64_t thr) {
  if (nargs < 4 || !args[0].isTensor() || !args[1].isInt() || !args[2].isInt() || !args[3].isBool()) return false;
  const at::Tensor& x = args[0].toTensor();
  if (!ok_tensor(x, thr) || x.dim() == 0 || !x.is_contiguous()) return false;
  const int64_t k = args[1].toInt(), n = x.size(-1);
  int64_t dim = args[2].toInt();
  if (dim < 0) dim += x.dim();
  if (dim != x.dim() - 1 || k < 1 || k > std::min<int64_t>(n, 256)) return false;
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  shape.back() = k;
  at::Tensor values = new_cuda(shape, x.scalar_type(), x.device());
  at::Tensor indices = new_cuda(shape, at::kLong, x.device());
  const int dev = x.get_device();
  if (dev < 0 || dev >= kMaxDev) return false;
  {
    BusyGuard busy(dev);
    gpuos_rt* rt = runtime(dev);
    if (!rt) return false;
    std::lock_guard<std::mutex> lk(g_mu);
    if (gpuos_rt_submit_topk(rt, x.const_data_ptr(), dtype_code(x.scalar_type()), x.numel() / n, n,
                             values.data_ptr(), indices.data_ptr<int64_t>(), (int)k, args[3].toBool() ? 1 : 0))
      return false;
    record(r, dev, {&x, &values, &indices});
  }
  torch::jit::drop(*stack, nargs);
  torch::jit::push(*stack, std::move(values));
  torch::jit::push(*stack, std::move(indices));
  return true;
}

// ---- ops left to PyTorch ---------------------------------------------------------------

template <typename F>
void each_tensor(const c10::IValue& v, F&& f) {
  if (v.isTensor()) {
    f(v.toTensor());
  } else if (v.isTensorList()) {
    for (const at::Tensor& t : v.toTensorVector()) f(t);
  } else if (v.isList()) {
    for (const c10::IValue& e : v.toListRef()) each_tensor(e, f);
  } else if (v.isTuple()) {
    for (const c10::IValue& e : v.toTupleRef().elements()) each_tensor(e, f);
  }
}

// Publish and wait for every device's requests, drop what they held, forget pending storages.
void sync_flush_all() {
  each_runtime([](int d, gpuos_rt* rt) {
    uint64_t seq = 0;
    check(intercept_flush(d, rt, GPUOS_FLUSH_DEP, c10::cuda::getCurrentCUDAStream((c10::DeviceIndex)d).stream(), &seq));
    if (seq) check(gpuos_rt_wait(rt, seq, 30000));
    intercept_release(d, gpuos_rt_completed(rt));
    return true;
  });
  std::lock_guard<std::mutex> lk(g_mu);
  g_pending.clear();
}

bool any_worker_alive() {
  bool alive = false;
  each_runtime([&](int, gpuos_rt* rt) {
    alive = gpuos_rt_worker_alive(rt) != 0;
    return !alive;
  });
  return alive;
}

void quiesce_all() {
  each_runtime([](int, gpuos_rt* rt) {
    check(gpuos_rt_quiesce(rt, 30000));
    return true;
  });
}

// scheduler.py's "not scheduled" branch: order the op after pending requests it touches, stop
// the resident worker before a kernel that may need its SMs, count, run below this key.
void leave_to_pytorch(Route* r, const c10::OperatorHandle& op, c10::DispatchKeySet ks, torch::jit::Stack* stack,
                      size_t nargs) {
  bool cuda = false, touches = false, pending = false;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    pending = !g_pending.empty();
    const c10::IValue* args = stack->data() + (stack->size() - nargs);
    for (size_t i = 0; i < nargs; ++i)
      each_tensor(args[i], [&](const at::Tensor& t) {
        if (!t.defined() || !t.is_cuda()) return;
        cuda = true;
        if (!pending || touches || !t.has_storage()) return;
        try {
          touches = g_pending.count(storage_key(t)) != 0;
        } catch (const c10::Error&) {
          // a tensor whose data pointer cannot be read (a fake tensor): no request of ours holds it
        }
      });
    ++g_fallbacks;
    ++r->fallbacks;
  }
  if (touches) {
    sync_flush_all();
    pending = false;
  }
  if (cuda && !r->no_kernel && (pending || any_worker_alive())) {
    sync_flush_all();
    quiesce_all();
  }
  c10::impl::ExcludeDispatchKeyGuard below(kKey);
  op.redispatchBoxed(ks & kBelow, stack);
}

void intercept_fallback(const c10::OperatorHandle& op, c10::DispatchKeySet ks, torch::jit::Stack* stack) {
  Route* r = route_of(op);
  if (r->kind == K_NONE && r->composite) {
    // decomposed at the autograd level: its parts come back through here one by one
    op.redispatchBoxed(ks & kBelow, stack);
    return;
  }
  const size_t nargs = op.schema().arguments().size();
  if (r->kind != K_NONE && !c10::GradMode::is_enabled() && plain(ks)) {
    c10::impl::ExcludeDispatchKeyGuard below(kKey);  // allocations made here are not intercepted
    c10::IValue* args = stack->data() + (stack->size() - nargs);
    const int64_t thr = g_threshold.load(std::memory_order_relaxed);
    bool done = false;
    switch (r->kind) {
      case K_BINARY: done = try_binary(r, args, nargs, stack, thr); break;
      case K_UNARY:
      case K_PARAM: done = try_unary(r, args, nargs, stack, thr); break;
      case K_REDUCE: done = try_reduce(r, args, nargs, stack, thr); break;
      case K_TOPK: done = try_topk(r, args, nargs, stack, thr); break;
      default: break;
    }
    if (done) return;
  }
  leave_to_pytorch(r, op, ks, stack, nargs);
}

}  // namespace

bool intercept_enable(int64_t size_threshold, std::string* err) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_lib) {
    if (c10::Dispatcher::singleton().hasBackendFallbackForDispatchKey(kKey)) {
      *err = "the dispatcher key TESTING_ONLY_GenericMode already has a fallback in this process";
      return false;
    }
    g_lib = new torch::Library(torch::Library::IMPL, "_", std::make_optional(kKey), __FILE__, __LINE__);
    g_lib->fallback(torch::CppFunction::makeFromBoxedFunction<&intercept_fallback>());
  }
  g_threshold.store(size_threshold);
  g_scheduled = g_fallbacks = 0;
  for (auto& kv : g_routes) kv.second->scheduled = kv.second->fallbacks = 0;
  g_pending.clear();
  c10::impl::tls_set_dispatch_key_included(kKey, true);
  return true;
}

void intercept_disable() { c10::impl::tls_set_dispatch_key_included(kKey, false); }

bool intercept_enabled() { return c10::impl::tls_is_dispatch_key_included(kKey); }

InterceptStats intercept_stats() {
  std::lock_guard<std::mutex> lk(g_mu);
  InterceptStats s;
  s.scheduled = g_scheduled;
  s.fallbacks = g_fallbacks;
  for (const auto& kv : g_routes) {
    if (kv.second->scheduled) s.scheduled_ops.emplace_back(kv.second->name, kv.second->scheduled);
    if (kv.second->fallbacks) s.fallback_ops.emplace_back(kv.second->name, kv.second->fallbacks);
  }
  return s;
}

std::vector<std::pair<std::string, std::pair<int, int>>> intercept_routes() {
  std::vector<std::pair<std::string, std::pair<int, int>>> v;
  for (const auto& kv : route_table()) v.emplace_back(kv.first, std::make_pair((int)kv.second.first, kv.second.second));
  return v;
}

void intercept_clear_pending() {
  std::lock_guard<std::mutex> lk(g_mu);
  g_pending.clear();
}

int intercept_flush(int dev, gpuos_rt* rt, int flags, cudaStream_t dep, uint64_t* seq_out) {
  std::lock_guard<std::mutex> lk(g_mu);
  uint64_t seq = 0;
  const int st = gpuos_rt_flush(rt, flags, dep, &seq);
  if (seq_out) *seq_out = seq;
  if (st || seq == 0 || dev < 0 || dev >= kMaxDev) return st;  // nothing published: refs wait for the next flush
  DevRefs& R = g_refs[dev];
  if (R.pending.empty()) return st;
  if (!R.inflight.empty() && R.inflight.back().first == seq) {
    auto& v = R.inflight.back().second;
    v.insert(v.end(), std::make_move_iterator(R.pending.begin()), std::make_move_iterator(R.pending.end()));
    R.pending.clear();
  } else {
    R.inflight.emplace_back(seq, std::move(R.pending));
    R.pending = std::vector<at::Tensor>();
  }
  return st;
}

void intercept_release(int dev, uint64_t completed) {
  if (dev < 0 || dev >= kMaxDev) return;
  std::vector<at::Tensor> dead;  // dropped after the lock: a drop may need the GIL
  {
    std::lock_guard<std::mutex> lk(g_mu);
    DevRefs& R = g_refs[dev];
    while (!R.inflight.empty() && R.inflight.front().first <= completed) {
      auto& v = R.inflight.front().second;
      dead.insert(dead.end(), std::make_move_iterator(v.begin()), std::make_move_iterator(v.end()));
      R.inflight.pop_front();
    }
  }
}

void intercept_release_all(int dev) {
  if (dev < 0 || dev >= kMaxDev) return;
  std::vector<at::Tensor> dead;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    DevRefs& R = g_refs[dev];
    dead.swap(R.pending);
    while (!R.inflight.empty()) {
      auto& v = R.inflight.front().second;
      dead.insert(dead.end(), std::make_move_iterator(v.begin()), std::make_move_iterator(v.end()));
      R.inflight.pop_front();
    }
  }
}

}  // namespace gpuos_py
