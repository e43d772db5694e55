// jit.cpp — operators compiled at run time (NVRTC, sm_100a) and linked into the worker.
//
// Reference: pytorch_ext/gpuos_ext.cpp:316-363 (NVRTC compile to PTX, module load, operator
// address read through a __device__ pointer), :814-881 (element-wise operator source), and
// :1079-1088 (custom PTX).  Differences, and why:
//   * operators are compiled to relocatable sm_100a code with the worker's register budget
//     (-maxrregcount=128) and linked with the worker's relocatable code by nvJitLink, so the
//     worker calls them within one module; the reference calls into a separately loaded
//     module, whose code reads its own module's constant banks and globals under a kernel of
//     another module, and whose register use nothing checks against the caller's launch;
//   * NVRTC and nvJitLink are opened by absolute path from the CUDA toolkit the worker was
//     built with: PyTorch loads its own (older) copies under the same library names, and a
//     linker older than the compiler of its inputs rejects them;
//   * transcendental functions in an expression are evaluated in double precision and
//     rounded once to float (at most one float rounding error per call).
#include "jit.h"

#include <cuda.h>
#include <dlfcn.h>
#include <nvJitLink.h>
#include <nvrtc.h>
#include <stdio.h>
#include <stdlib.h>

#include <fstream>
#include <iterator>
#include <mutex>

#include "gpuos_b200.h"

namespace gpuos {
namespace jit {
namespace {

// ---- libraries -----------------------------------------------------------------------------
struct Nvrtc {
  void* h = nullptr;
  nvrtcResult (*Version)(int*, int*) = nullptr;
  nvrtcResult (*CreateProgram)(nvrtcProgram*, const char*, const char*, int, const char* const*,
                               const char* const*) = nullptr;
  nvrtcResult (*CompileProgram)(nvrtcProgram, int, const char* const*) = nullptr;
  nvrtcResult (*GetProgramLogSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*GetProgramLog)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*GetCUBINSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*GetCUBIN)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*GetPTXSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*GetPTX)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*DestroyProgram)(nvrtcProgram*) = nullptr;
  const char* (*GetErrorString)(nvrtcResult) = nullptr;
};

struct JitLink {
  void* h = nullptr;
  nvJitLinkResult (*Create)(nvJitLinkHandle*, uint32_t, const char**) = nullptr;
  nvJitLinkResult (*Destroy)(nvJitLinkHandle*) = nullptr;
  nvJitLinkResult (*AddData)(nvJitLinkHandle, nvJitLinkInputType, const void*, size_t, const char*) = nullptr;
  nvJitLinkResult (*Complete)(nvJitLinkHandle) = nullptr;
  nvJitLinkResult (*GetLinkedCubinSize)(nvJitLinkHandle, size_t*) = nullptr;
  nvJitLinkResult (*GetLinkedCubin)(nvJitLinkHandle, void*) = nullptr;
  nvJitLinkResult (*GetErrorLogSize)(nvJitLinkHandle, size_t*) = nullptr;
  nvJitLinkResult (*GetErrorLog)(nvJitLinkHandle, char*) = nullptr;
};

struct Driver {
  bool ok = false;
  CUresult (*ModuleLoadData)(CUmodule*, const void*) = nullptr;
  CUresult (*ModuleUnload)(CUmodule) = nullptr;
  CUresult (*ModuleGetFunction)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*FuncSetAttribute)(CUfunction, CUfunction_attribute, int) = nullptr;
  CUresult (*FuncLoad)(CUfunction) = nullptr;  // optional (driver >= 12.4)
  CUresult (*LaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                           CUstream, void**, void**) = nullptr;
  CUresult (*Occupancy)(int*, CUfunction, int, size_t) = nullptr;
  CUresult (*GetErrorString)(CUresult, const char**) = nullptr;
};

std::mutex g_mu;
Nvrtc g_nvrtc;
JitLink g_link;
Driver g_drv;
std::vector<char> g_worker;  // relocatable worker code (read once)
std::string g_lib_error;

std::string cuda_home() {
  const char* e = getenv("CUDA_HOME");
  return e && *e ? std::string(e) : std::string("/usr/local/cuda");
}

template <typename F>
bool sym(void* h, const char* name, F* out, std::string* err) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  if (!*out) {
    *err = std::string("missing symbol ") + name;
    return false;
  }
  return true;
}

bool open_nvrtc(std::string* err) {
  if (g_nvrtc.h) return true;
  const std::string path = cuda_home() + "/lib64/libnvrtc.so.12";
  void* h = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    *err = "cannot open " + path + ": " + dlerror();
    return false;
  }
  Nvrtc n;
  n.h = h;
  bool ok = sym(h, "nvrtcVersion", &n.Version, err) && sym(h, "nvrtcCreateProgram", &n.CreateProgram, err) &&
            sym(h, "nvrtcCompileProgram", &n.CompileProgram, err) &&
            sym(h, "nvrtcGetProgramLogSize", &n.GetProgramLogSize, err) &&
            sym(h, "nvrtcGetProgramLog", &n.GetProgramLog, err) && sym(h, "nvrtcGetCUBINSize", &n.GetCUBINSize, err) &&
            sym(h, "nvrtcGetCUBIN", &n.GetCUBIN, err) && sym(h, "nvrtcGetPTXSize", &n.GetPTXSize, err) &&
            sym(h, "nvrtcGetPTX", &n.GetPTX, err) && sym(h, "nvrtcDestroyProgram", &n.DestroyProgram, err) &&
            sym(h, "nvrtcGetErrorString", &n.GetErrorString, err);
  if (!ok) return false;
  g_nvrtc = n;
  return true;
}

// nvJitLink exports one entry point per toolkit release it understands; use the one of the
// release whose headers this file was compiled against.
#define GPUOS_JL_STR2(x) #x
#define GPUOS_JL_STR(x) GPUOS_JL_STR2(x)
#define GPUOS_JL_NAME(fn) "__nvJitLink" #fn "_" GPUOS_JL_STR(CUDA_VERSION_MAJOR_) "_" GPUOS_JL_STR(CUDA_VERSION_MINOR_)
#define CUDA_VERSION_MAJOR_ 12
#define CUDA_VERSION_MINOR_ 9
static_assert(CUDA_VERSION / 1000 == CUDA_VERSION_MAJOR_ && (CUDA_VERSION % 1000) / 10 == CUDA_VERSION_MINOR_,
              "nvJitLink entry points are named for the toolkit release of cuda.h");

bool open_link(std::string* err) {
  if (g_link.h) return true;
  const std::string path = cuda_home() + "/lib64/libnvJitLink.so.12";
  void* h = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    *err = "cannot open " + path + ": " + dlerror();
    return false;
  }
  JitLink l;
  l.h = h;
  bool ok = sym(h, GPUOS_JL_NAME(Create), &l.Create, err) && sym(h, GPUOS_JL_NAME(Destroy), &l.Destroy, err) &&
            sym(h, GPUOS_JL_NAME(AddData), &l.AddData, err) && sym(h, GPUOS_JL_NAME(Complete), &l.Complete, err) &&
            sym(h, GPUOS_JL_NAME(GetLinkedCubinSize), &l.GetLinkedCubinSize, err) &&
            sym(h, GPUOS_JL_NAME(GetLinkedCubin), &l.GetLinkedCubin, err) &&
            sym(h, GPUOS_JL_NAME(GetErrorLogSize), &l.GetErrorLogSize, err) &&
            sym(h, GPUOS_JL_NAME(GetErrorLog), &l.GetErrorLog, err);
  if (!ok) return false;
  g_link = l;
  return true;
}

template <typename F>
bool drv(const char* name, F* out, bool required, std::string* err) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) {
    *out = nullptr;
    if (required) *err = std::string("driver entry point ") + name + " unavailable";
    return !required;
  }
  *out = reinterpret_cast<F>(p);
  return true;
}

bool open_driver(std::string* err) {
  if (g_drv.ok) return true;
  Driver d;
  bool ok = drv("cuModuleLoadData", &d.ModuleLoadData, true, err) && drv("cuModuleUnload", &d.ModuleUnload, true, err) &&
            drv("cuModuleGetFunction", &d.ModuleGetFunction, true, err) &&
            drv("cuFuncSetAttribute", &d.FuncSetAttribute, true, err) && drv("cuFuncLoad", &d.FuncLoad, false, err) &&
            drv("cuLaunchKernel", &d.LaunchKernel, true, err) &&
            drv("cuOccupancyMaxActiveBlocksPerMultiprocessor", &d.Occupancy, true, err) &&
            drv("cuGetErrorString", &d.GetErrorString, true, err);
  if (!ok) return false;
  d.ok = true;
  g_drv = d;
  return true;
}

std::string drv_msg(const char* what, CUresult r) {
  const char* s = nullptr;
  if (g_drv.GetErrorString) g_drv.GetErrorString(r, &s);
  return std::string(what) + ": " + (s ? s : "unknown driver error");
}

// The worker's relocatable code lives next to this library (built with it).
bool load_worker_code(std::string* err) {
  if (!g_worker.empty()) return true;
  Dl_info info;
  if (!dladdr(reinterpret_cast<void*>(&load_worker_code), &info) || !info.dli_fname) {
    *err = "cannot locate libgpuos_b200.so";
    return false;
  }
  std::string path(info.dli_fname);
  const size_t slash = path.rfind('/');
  path = (slash == std::string::npos ? std::string(".") : path.substr(0, slash)) + "/gpuos_worker_rdc.cubin";
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    *err = "missing " + path + " (rebuild with python -m gpuos_b200.build)";
    return false;
  }
  g_worker.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  if (g_worker.empty()) {
    *err = "empty " + path;
    return false;
  }
  return true;
}

// Expression characters: identifiers, numbers, operators, parentheses, commas, ?:, blanks.
bool expr_chars_ok(const std::string& e) {
  if (e.empty()) return false;
  for (char c : e) {
    const bool ok = (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_' ||
                    c == '.' || c == '+' || c == '-' || c == '*' || c == '/' || c == '%' || c == '<' || c == '>' ||
                    c == '=' || c == '!' || c == '&' || c == '|' || c == '?' || c == ':' || c == '(' || c == ')' ||
                    c == ',' || c == ' ' || c == '\t';
    if (!ok) return false;
  }
  return true;
}

bool ident_ok(const std::string& s) {
  if (s.empty() || s.size() > 200 || (s[0] >= '0' && s[0] <= '9')) return false;
  for (char c : s)
    if (!((c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_')) return false;
  return true;
}

// Reference descriptor layout (src/common.h:22-46), checked at compile time, plus the element
// access of the reference's operators (persistent_kernel.cu:20-31, 60-78): offsets from
// per-dimension sizes and strides (broadcast dims carry stride 0), f32/f16/bf16 storage, math
// in float, round-to-nearest-even stores.
// The built-in operators' math (the same text the worker is compiled from), so that an operator
// compiled here can call gpuos::ew_apply<GPUOS_EW_...>(a, b, p0, p1) and round exactly as the
// built-in operator does (fused chains).  It goes ahead of the prelude's macros, which would
// otherwise turn its float math functions into double-precision ones.
#define GPUOS_EW_MATH(...) #__VA_ARGS__
const char* const kEwMath =
#include "device/ew_math.inc"
    ;
#undef GPUOS_EW_MATH

std::string ew_math_source() {
  std::string s;
#define GX_CODE(n) s += "constexpr int GPUOS_EW_" #n " = " + std::to_string((int)GPUOS_EW_##n) + ";\n";
  GX_CODE(ADD) GX_CODE(MUL) GX_CODE(SUB) GX_CODE(DIV) GX_CODE(MAXIMUM) GX_CODE(MINIMUM) GX_CODE(POW)
  GX_CODE(COPY) GX_CODE(RELU) GX_CODE(SIGMOID) GX_CODE(TANH) GX_CODE(EXP) GX_CODE(LOG) GX_CODE(SQRT)
  GX_CODE(ABS) GX_CODE(HARDSIGMOID) GX_CODE(HARDSWISH) GX_CODE(GELU) GX_CODE(GELU_TANH) GX_CODE(SIN)
  GX_CODE(COS) GX_CODE(LEAKY_RELU) GX_CODE(CLAMP) GX_CODE(CLAMP_MIN) GX_CODE(CLAMP_MAX) GX_CODE(ELU)
  GX_CODE(SOFTPLUS) GX_CODE(NEG) GX_CODE(ADD_ALPHA) GX_CODE(SUB_ALPHA)
#undef GX_CODE
  s += "namespace gpuos {\n";
  s += kEwMath;
  s += "\n}  // namespace gpuos\n";
  return s;
}

const char* kPrelude = R"PRELUDE(
typedef long long gx_i64;
struct TensorRef { void* data; int dtype; int ndim; gx_i64 sizes[8]; gx_i64 strides[8]; };
struct TaskHead { int op; int flags; int ndim; gx_i64 numel; int rrank; int r_axes[8]; int r_keepdim; };
struct Task { int op; int flags; int ndim; gx_i64 numel; int rrank; int r_axes[8]; int r_keepdim;
              TensorRef in0; TensorRef in1; TensorRef out0; };
// in0 at 64, in1 at 208, out0 at 352
static_assert(sizeof(TensorRef) == 144 && sizeof(TaskHead) == 64 && sizeof(Task) == 496, "reference Task layout");
namespace gx {
__device__ __forceinline__ gx_i64 offset(const TensorRef& r, gx_i64 i) {
  gx_i64 off = 0;
  for (int d = r.ndim - 1; d >= 0; --d) {
    const gx_i64 n = r.sizes[d] > 0 ? r.sizes[d] : 1;
    off += (i % n) * r.strides[d];
    i /= n;
  }
  return off;
}
__device__ __forceinline__ float load(const TensorRef& r, gx_i64 off) {
  if (r.dtype == 1) {
    const unsigned short h = static_cast<const unsigned short*>(r.data)[off];
    float f;
    asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
    return f;
  }
  if (r.dtype == 2) return __uint_as_float((unsigned)static_cast<const unsigned short*>(r.data)[off] << 16);
  return static_cast<const float*>(r.data)[off];
}
__device__ __forceinline__ void store(const TensorRef& r, gx_i64 off, float v) {
  if (r.dtype == 1 || r.dtype == 2) {
    unsigned short h;
    if (r.dtype == 1) asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(v));
    else asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(v));
    static_cast<unsigned short*>(r.data)[off] = h;
    return;
  }
  static_cast<float*>(r.data)[off] = v;
}
// one rounding to float per transcendental call
#define GX_D1(n) __device__ __forceinline__ float d_##n(float x) { return (float)::n((double)x); }
GX_D1(exp) GX_D1(log) GX_D1(log1p) GX_D1(expm1) GX_D1(tanh) GX_D1(sin) GX_D1(cos) GX_D1(tan) GX_D1(erf)
GX_D1(exp2) GX_D1(log2) GX_D1(log10) GX_D1(sinh) GX_D1(cosh) GX_D1(asin) GX_D1(acos) GX_D1(atan)
#undef GX_D1
__device__ __forceinline__ float d_rsqrt(float x) { return (float)(1.0 / ::sqrt((double)x)); }
__device__ __forceinline__ float d_pow(float x, float y) { return (float)::pow((double)x, (double)y); }
__device__ __forceinline__ float d_atan2(float x, float y) { return (float)::atan2((double)x, (double)y); }
}  // namespace gx
#define expf(x) gx::d_exp(x)
#define exp(x) gx::d_exp(x)
#define logf(x) gx::d_log(x)
#define log(x) gx::d_log(x)
#define log1pf(x) gx::d_log1p(x)
#define log1p(x) gx::d_log1p(x)
#define expm1f(x) gx::d_expm1(x)
#define expm1(x) gx::d_expm1(x)
#define tanhf(x) gx::d_tanh(x)
#define tanh(x) gx::d_tanh(x)
#define sinf(x) gx::d_sin(x)
#define sin(x) gx::d_sin(x)
#define cosf(x) gx::d_cos(x)
#define cos(x) gx::d_cos(x)
#define tanf(x) gx::d_tan(x)
#define tan(x) gx::d_tan(x)
#define erff(x) gx::d_erf(x)
#define erf(x) gx::d_erf(x)
#define exp2f(x) gx::d_exp2(x)
#define exp2(x) gx::d_exp2(x)
#define log2f(x) gx::d_log2(x)
#define log2(x) gx::d_log2(x)
#define log10f(x) gx::d_log10(x)
#define log10(x) gx::d_log10(x)
#define sinhf(x) gx::d_sinh(x)
#define sinh(x) gx::d_sinh(x)
#define coshf(x) gx::d_cosh(x)
#define cosh(x) gx::d_cosh(x)
#define asinf(x) gx::d_asin(x)
#define asin(x) gx::d_asin(x)
#define acosf(x) gx::d_acos(x)
#define acos(x) gx::d_acos(x)
#define atanf(x) gx::d_atan(x)
#define atan(x) gx::d_atan(x)
#define rsqrtf(x) gx::d_rsqrt(x)
#define rsqrt(x) gx::d_rsqrt(x)
#define powf(x, y) gx::d_pow(x, y)
#define pow(x, y) gx::d_pow(x, y)
#define atan2f(x, y) gx::d_atan2(x, y)
#define atan2(x, y) gx::d_atan2(x, y)
)PRELUDE";

std::string nvrtc_log(nvrtcProgram p) {
  size_t n = 0;
  if (g_nvrtc.GetProgramLogSize(p, &n) != NVRTC_SUCCESS || n <= 1) return std::string();
  std::string log(n, '\0');
  g_nvrtc.GetProgramLog(p, &log[0]);
  while (!log.empty() && (log.back() == '\0' || log.back() == '\n')) log.pop_back();
  return log;
}

}  // namespace

int ew_source(int id, const std::string& expr, int arity, std::string* src, std::string* err) {
  if (arity != 1 && arity != 2) {
    *err = "arity must be 1 or 2";
    return GPUOS_ERR_INVALID;
  }
  if (!expr_chars_ok(expr) || expr.size() > 4000) {
    *err = "expression holds characters outside C expression syntax";
    return GPUOS_ERR_INVALID;
  }
  const std::string n = std::to_string(id);
  std::string s = ew_math_source();
  s += kPrelude;
  s += "extern \"C\" __device__ void gpuos_jit_op_" + n + "(const Task& t) {\n";
  s += "  const gx_i64 N = t.numel;\n";
  s += "  for (gx_i64 i = threadIdx.x; i < N; i += blockDim.x) {\n";
  s += "    const float A = gx::load(t.in0, gx::offset(t.in0, i));\n";
  if (arity == 2) s += "    const float B = gx::load(t.in1, gx::offset(t.in1, i));\n";
  s += "    const float R = (float)(" + expr + ");\n";
  s += "    gx::store(t.out0, gx::offset(t.out0, i), R);\n";
  s += "  }\n}\n";
  s += "extern \"C\" __global__ void gpuos_jit_addr_" + n + "(unsigned long long* out) {\n";
  s += "  out[0] = reinterpret_cast<unsigned long long>(&gpuos_jit_op_" + n + ");\n";
  // a call site keeps the operator in this kernel's call graph (never taken: out is valid)
  s += "  if (out == nullptr) gpuos_jit_op_" + n + "(*reinterpret_cast<const Task*>(out + 1));\n}\n";
  *src = s;
  return GPUOS_OK;
}

int bridge_source(int id, const std::string& entry, std::string* src, std::string* err) {
  if (!ident_ok(entry)) {
    *err = "entry name must be a C identifier";
    return GPUOS_ERR_INVALID;
  }
  const std::string n = std::to_string(id);
  std::string s;
  s += "struct Task;\n";
  s += "extern \"C\" __device__ void " + entry + "(const Task& t);\n";
  s += "extern \"C\" __global__ void gpuos_jit_addr_" + n + "(unsigned long long* out) {\n";
  s += "  out[0] = reinterpret_cast<unsigned long long>(&" + entry + ");\n";
  s += "  if (out == nullptr) " + entry + "(*reinterpret_cast<const Task*>(out + 1));\n}\n";
  *src = s;
  return GPUOS_OK;
}

int compile(const std::string& src, const char* name, const char* output, std::vector<char>* out,
            std::string* err) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!open_nvrtc(err)) return GPUOS_ERR_UNSUPPORTED;
  const bool ptx = std::string(output) == "ptx";
  nvrtcProgram p = nullptr;
  nvrtcResult r = g_nvrtc.CreateProgram(&p, src.c_str(), name, 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) {
    *err = std::string("nvrtcCreateProgram: ") + g_nvrtc.GetErrorString(r);
    return GPUOS_ERR_NVRTC;
  }
  // relocatable code within the worker's register budget (512 threads per CTA)
  const char* opts_cubin[] = {"-arch=sm_100a", "-rdc=true", "-maxrregcount=128", "-std=c++17", "-fmad=false"};
  const char* opts_ptx[] = {"-arch=compute_100a", "-rdc=true", "-maxrregcount=128", "-std=c++17", "-fmad=false"};
  r = g_nvrtc.CompileProgram(p, 5, ptx ? opts_ptx : opts_cubin);
  if (r != NVRTC_SUCCESS) {
    *err = std::string("NVRTC: ") + g_nvrtc.GetErrorString(r) + "\n" + nvrtc_log(p);
    g_nvrtc.DestroyProgram(&p);
    return GPUOS_ERR_NVRTC;
  }
  size_t n = 0;
  r = ptx ? g_nvrtc.GetPTXSize(p, &n) : g_nvrtc.GetCUBINSize(p, &n);
  if (r == NVRTC_SUCCESS) {
    out->assign(n, 0);
    r = ptx ? g_nvrtc.GetPTX(p, out->data()) : g_nvrtc.GetCUBIN(p, out->data());
  }
  g_nvrtc.DestroyProgram(&p);
  if (r != NVRTC_SUCCESS) {
    *err = std::string("NVRTC output: ") + g_nvrtc.GetErrorString(r);
    return GPUOS_ERR_NVRTC;
  }
  return GPUOS_OK;
}

int link(const std::vector<Op>& ops, std::vector<char>* image, std::string* err) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!open_link(err) || !load_worker_code(err)) return GPUOS_ERR_UNSUPPORTED;
  nvJitLinkHandle h = nullptr;
  const char* opts[] = {"-arch=sm_100a", "-maxrregcount=128"};
  nvJitLinkResult r = g_link.Create(&h, 2, opts);
  if (r != NVJITLINK_SUCCESS) {
    *err = "nvJitLinkCreate failed (" + std::to_string((int)r) + ")";
    return GPUOS_ERR_NVRTC;
  }
  auto log = [&]() {
    size_t n = 0;
    std::string s;
    if (g_link.GetErrorLogSize(h, &n) == NVJITLINK_SUCCESS && n > 1) {
      s.assign(n, '\0');
      g_link.GetErrorLog(h, &s[0]);
      while (!s.empty() && (s.back() == '\0' || s.back() == '\n')) s.pop_back();
    }
    return s;
  };
  r = g_link.AddData(h, NVJITLINK_INPUT_CUBIN, g_worker.data(), g_worker.size(), "gpuos_worker");
  for (const Op& op : ops) {
    for (const Object& o : op.objs) {
      if (r != NVJITLINK_SUCCESS) break;
      r = g_link.AddData(h, o.ptx ? NVJITLINK_INPUT_PTX : NVJITLINK_INPUT_CUBIN, o.bytes.data(), o.bytes.size(),
                         o.name.c_str());
    }
  }
  if (r == NVJITLINK_SUCCESS) r = g_link.Complete(h);
  if (r != NVJITLINK_SUCCESS) {
    *err = "nvJitLink (" + std::to_string((int)r) + "): " + log();
    g_link.Destroy(&h);
    return GPUOS_ERR_NVRTC;
  }
  size_t n = 0;
  r = g_link.GetLinkedCubinSize(h, &n);
  if (r == NVJITLINK_SUCCESS) {
    image->assign(n, 0);
    r = g_link.GetLinkedCubin(h, image->data());
  }
  g_link.Destroy(&h);
  if (r != NVJITLINK_SUCCESS) {
    *err = "nvJitLink output (" + std::to_string((int)r) + ")";
    return GPUOS_ERR_NVRTC;
  }
  return GPUOS_OK;
}

int load(const std::vector<char>& image, const std::vector<Op>& ops, Module* m, std::string* err) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!open_driver(err)) return GPUOS_ERR_UNSUPPORTED;
  CUmodule mod = nullptr;
  CUresult r = g_drv.ModuleLoadData(&mod, image.data());
  if (r != CUDA_SUCCESS) {
    *err = drv_msg("cuModuleLoadData", r);
    return GPUOS_ERR_CUDA;
  }
  auto fail = [&](const char* what) {
    *err = drv_msg(what, r);
    g_drv.ModuleUnload(mod);
    return GPUOS_ERR_CUDA;
  };
  CUfunction w = nullptr, a = nullptr;
  r = g_drv.ModuleGetFunction(&w, mod, "gpuos_batch_worker");
  if (r != CUDA_SUCCESS) return fail("worker kernel");
  r = g_drv.ModuleGetFunction(&a, mod, "gpuos_module_addrs");
  if (r != CUDA_SUCCESS) return fail("address kernel");
  std::vector<void*> fns;
  for (const Op& op : ops) {
    CUfunction f = nullptr;
    r = g_drv.ModuleGetFunction(&f, mod, op.addr_kernel.c_str());
    if (r != CUDA_SUCCESS) return fail("operator address kernel");
    fns.push_back(f);
  }
  // load every kernel now: a lazy load at the first launch could wait for running kernels
  if (g_drv.FuncLoad) {
    r = g_drv.FuncLoad(w);
    if (r == CUDA_SUCCESS) r = g_drv.FuncLoad(a);
    for (void* f : fns)
      if (r == CUDA_SUCCESS) r = g_drv.FuncLoad(static_cast<CUfunction>(f));
    if (r != CUDA_SUCCESS) return fail("cuFuncLoad");
  }
  m->mod = mod;
  m->worker = w;
  m->addrs = a;
  m->op_addr = fns;
  return GPUOS_OK;
}

void unload(Module* m) {
  if (m && m->mod && g_drv.ok) g_drv.ModuleUnload(static_cast<CUmodule>(m->mod));
  if (m) *m = Module();
}

int launch(void* fn, unsigned grid, unsigned block, size_t smem, cudaStream_t s, void** args, std::string* err) {
  CUresult r = g_drv.LaunchKernel(static_cast<CUfunction>(fn), grid, 1, 1, block, 1, 1, (unsigned)smem,
                                  reinterpret_cast<CUstream>(s), args, nullptr);
  if (r != CUDA_SUCCESS) {
    *err = drv_msg("cuLaunchKernel", r);
    return GPUOS_ERR_CUDA;
  }
  return GPUOS_OK;
}

int set_smem(void* fn, size_t smem, std::string* err) {
  CUresult r = g_drv.FuncSetAttribute(static_cast<CUfunction>(fn), CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                      (int)smem);
  if (r != CUDA_SUCCESS) {
    *err = drv_msg("cuFuncSetAttribute", r);
    return GPUOS_ERR_CUDA;
  }
  return GPUOS_OK;
}

int occupancy(void* fn, int threads, size_t smem, int* blocks, std::string* err) {
  CUresult r = g_drv.Occupancy(blocks, static_cast<CUfunction>(fn), threads, smem);
  if (r != CUDA_SUCCESS) {
    *err = drv_msg("cuOccupancyMaxActiveBlocksPerMultiprocessor", r);
    return GPUOS_ERR_CUDA;
  }
  return GPUOS_OK;
}

int nvrtc_version() {
  std::lock_guard<std::mutex> lk(g_mu);
  std::string err;
  if (!open_nvrtc(&err)) return 0;
  int ma = 0, mi = 0;
  if (g_nvrtc.Version(&ma, &mi) != NVRTC_SUCCESS) return 0;
  return ma * 1000 + mi * 10;
}

}  // namespace jit
}  // namespace gpuos
