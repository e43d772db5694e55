// jit.h — operators compiled at run time and linked into the worker (internal to the runtime).
//
// The reference compiles each registered expression with NVRTC into a module of its own and
// writes the operator's address into the op table that the running worker calls through
// (pytorch_ext/gpuos_ext.cpp:316-363, 814-881).  A function pointer is only safe to call from
// code of the module it belongs to: each module binds its own constant banks and globals, and
// a separately compiled callee is held to no register budget of the caller.  Here every
// operator compiled at run time is linked (nvJitLink) together with the worker's relocatable
// device code, capped at the worker's register budget, and the worker is relaunched from the
// linked module; the op table then only holds addresses of that module.
#pragma once
#include <stdint.h>

#include <string>
#include <vector>

#include <cuda_runtime_api.h>

namespace gpuos {
namespace jit {

// One input of a link: relocatable sm_100a code (NVRTC output) or PTX.
struct Object {
  bool ptx = false;
  std::string name;
  std::vector<char> bytes;
};

// An operator compiled at run time: its objects and the name of the kernel that writes its
// address (one unsigned long long) into device memory.
struct Op {
  std::vector<Object> objs;
  std::string addr_kernel;
};

// Loaded worker module (opaque driver handles).
struct Module {
  void* mod = nullptr;     // CUmodule
  void* worker = nullptr;  // CUfunction gpuos_batch_worker
  void* addrs = nullptr;   // CUfunction gpuos_module_addrs
  std::vector<void*> op_addr;  // CUfunction per operator, in Op order
};

// Status codes are GpuosStatus values; *err receives the NVRTC / linker / driver message.
// Translation unit of an element-wise operator `gpuos_jit_op_<id>`: out[i] = expr(A[, B]) over
// a reference-layout Task.  Characters outside C expression syntax are rejected.
int ew_source(int id, const std::string& expr, int arity, std::string* src, std::string* err);
// Translation unit that takes the address of `entry` (a reference-ABI device function defined
// in other linked code) for operator `id`.
int bridge_source(int id, const std::string& entry, std::string* src, std::string* err);
// NVRTC: relocatable sm_100a code (output == "cubin") or PTX (output == "ptx").
int compile(const std::string& src, const char* name, const char* output, std::vector<char>* out,
            std::string* err);
// nvJitLink: the worker's relocatable code + `ops`, linked for sm_100a.
int link(const std::vector<Op>& ops, std::vector<char>* image, std::string* err);
// Driver: load an image into the current context and look up the worker and address kernels.
int load(const std::vector<char>& image, const std::vector<Op>& ops, Module* m, std::string* err);
void unload(Module* m);
// Launch helpers on `s` (current context).
int launch(void* fn, unsigned grid, unsigned block, size_t smem, cudaStream_t s, void** args, std::string* err);
int set_smem(void* fn, size_t smem, std::string* err);
int occupancy(void* fn, int threads, size_t smem, int* blocks, std::string* err);
// Version of the NVRTC library in use (major * 1000 + minor * 10), 0 if it cannot be loaded.
int nvrtc_version();

}  // namespace jit
}  // namespace gpuos
