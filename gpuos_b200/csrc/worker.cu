// worker.cu — device tables, kernels and the reference C ABI of libgpuos_b200.so.
//
// Reference counterparts: src/persistent_kernel.cu (globals :9-15, init_builtin_ops
// :115-130, persistent_worker :138-231, C-ABI shim :233-269).
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>

#include "internal.h"
#include "device/ptx.cuh"
#include "device/ops.cuh"
#include "device/tiles.cuh"
#include "device/refops.cuh"
#include "device/expr.cuh"
#include "device/worker.cuh"

namespace gpuos {

// ---- tables (persistent_kernel.cu:9-15) -------------------------------------------------
// The op table holds device function addresses (reference ABI); the alias maps a logical
// op id to a physical slot.  The worker reads both when it dequeues a Task, so a slot or
// alias write is an online switch for every Task dequeued afterwards.
__device__ OpFn g_op_table[GPUOS_MAX_OPS];
__device__ int g_op_alias[GPUOS_MAX_OPS];
__device__ unsigned long long g_processed_count = 0ull;  // Task-ring worker completions
__device__ unsigned long long g_heartbeat = 0ull;        // Task-ring worker idle polls
__device__ int g_debug_level = 0;
__device__ unsigned long long g_yield_every = 0ull;
__device__ unsigned long long g_ring_idle_limit_ns = 30ull * 1000 * 1000 * 1000;

// Built-in reference-ABI operators that can occupy a slot.
constexpr int kBatchSlot = 10;  // persistent_kernel.cu:17
__device__ OpFn g_builtin_ref_ops[GPUOS_EW_NUM_OPS + 2] = {
    ref_ew<0>,  ref_ew<1>,  ref_ew<2>,  ref_ew<3>,  ref_ew<4>,  ref_ew<5>,  ref_ew<6>,  ref_ew<7>,
    ref_ew<8>,  ref_ew<9>,  ref_ew<10>, ref_ew<11>, ref_ew<12>, ref_ew<13>, ref_ew<14>, ref_ew<15>,
    ref_ew<16>, ref_ew<17>, ref_ew<18>, ref_ew<19>, ref_ew<20>, ref_ew<21>, ref_ew<22>, ref_ew<23>,
    ref_ew<24>, ref_ew<25>, ref_ew<26>, ref_ew<27>, ref_ew<28>, ref_ew<29>, op_reduce_sum,
    op_reduce_mean};

#ifndef GPUOS_JIT_WORKER
// persistent_kernel.cu:115-130: null table, identity alias, add@0, mul@1, batch@10.
__global__ void init_builtin_ops_kernel() {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx < GPUOS_MAX_OPS) {
    g_op_table[idx] = nullptr;
    g_op_alias[idx] = idx;
  }
  if (idx == 0) g_op_table[0] = op_add;
  if (idx == 1) g_op_table[1] = op_mul;
  if (idx == kBatchSlot) g_op_table[kBatchSlot] = op_batch;
}

#endif  // GPUOS_JIT_WORKER

// Operator addresses of the expression programs (one per program index).
__device__ OpFn g_expr_fns[kExprPrograms] = {
    op_expr<0>,  op_expr<1>,  op_expr<2>,  op_expr<3>,  op_expr<4>,  op_expr<5>,  op_expr<6>,  op_expr<7>,
    op_expr<8>,  op_expr<9>,  op_expr<10>, op_expr<11>, op_expr<12>, op_expr<13>, op_expr<14>, op_expr<15>,
    op_expr<16>, op_expr<17>, op_expr<18>, op_expr<19>, op_expr<20>, op_expr<21>, op_expr<22>, op_expr<23>,
    op_expr<24>, op_expr<25>, op_expr<26>, op_expr<27>, op_expr<28>, op_expr<29>, op_expr<30>, op_expr<31>};

// Every built-in operator address of this module, in the order of ModuleAddr, and the address
// of this module's expression-program table.  The runtime keeps one such list per loaded
// worker module (this library's own, and each module linked with run-time compiled
// operators) and translates op-table entries between them when it switches modules.
extern "C" __global__ void gpuos_module_addrs(unsigned long long* out) {
  const int i = threadIdx.x;
  if (i == 0) {
    out[MA_ADD] = reinterpret_cast<unsigned long long>(&op_add);
    out[MA_MUL] = reinterpret_cast<unsigned long long>(&op_mul);
    out[MA_BATCH] = reinterpret_cast<unsigned long long>(&op_batch);
    out[MA_EXPR_PROGS] = reinterpret_cast<unsigned long long>(&g_expr_progs[0]);
  }
  if (i < GPUOS_EW_NUM_OPS + 2) out[MA_REF_OPS + i] = reinterpret_cast<unsigned long long>(g_builtin_ref_ops[i]);
  if (i < kExprPrograms) out[MA_EXPR_FNS + i] = reinterpret_cast<unsigned long long>(g_expr_fns[i]);
}

#ifndef GPUOS_JIT_WORKER
__global__ void builtin_addr_kernel(int which, unsigned long long* out) {
  if (which == -1) *out = reinterpret_cast<unsigned long long>(&op_add);
  else if (which == -2) *out = reinterpret_cast<unsigned long long>(&op_mul);
  else if (which == -3) *out = reinterpret_cast<unsigned long long>(&op_batch);
  else if (which >= 0 && which < GPUOS_EW_NUM_OPS + 2)
    *out = reinterpret_cast<unsigned long long>(g_builtin_ref_ops[which]);
  else if (which >= 1000 && which < 1000 + kExprPrograms)
    *out = reinterpret_cast<unsigned long long>(g_expr_fns[which - 1000]);
  else *out = 0ull;
}

#endif  // GPUOS_JIT_WORKER

extern "C" __global__ void __launch_bounds__(kMaxComputeThreads + 64, 1) gpuos_batch_worker(const __grid_constant__ WorkerParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  batch_worker_body(P, smem_raw);
}

#ifndef GPUOS_JIT_WORKER
// ---- Task-ring worker (persistent_kernel.cu:138-231) --------------------------------------
// Same protocol as the reference (CAS claim of q.head < q.tail, dispatch through the alias
// and op table at dequeue time, completion counted after a system fence) with three
// changes: the idle wait is bounded (g_ring_idle_limit_ns), quit is polled once per claim
// by thread 0 instead of by every thread, and the mapped SyncState is written by block 0
// only (single writer: a mirror of the device counters) instead of system atomics on host
// memory.
__global__ void ring_worker_kernel(WorkQueue q) {
  if (q.capacity == 0) return;
  __shared__ Task s_task;
  __shared__ int s_state;  // 0 idle, 1 work, 2 exit
  __shared__ OpFn s_fn;
  if (threadIdx.x == 0 && blockIdx.x == 0 && q.sync != nullptr) {
    __threadfence_system();
    *reinterpret_cast<volatile int*>(&q.sync->ready) = 1;
  }
  uint64_t idle_since = ptx::now_ns();
  uint32_t idle_sleep = 64;
  while (true) {
    if (threadIdx.x == 0) {
      s_state = 0;
      volatile int* quit = q.quit;
      if (*quit != 0) {
        s_state = 2;
      } else {
        for (int attempt = 0; attempt < 1024; ++attempt) {
          const int h = atomicAdd(q.head, 0);
          const int t = atomicAdd(q.tail, 0);
          if (h >= t) break;
          if (atomicCAS(q.head, h, h + 1) == h) {
            const volatile Task* src = q.tasks + (h % q.capacity);
            const volatile uint4* s4 = reinterpret_cast<const volatile uint4*>(src);
            uint4* d4 = reinterpret_cast<uint4*>(&s_task);
            for (int k = 0; k < (int)(sizeof(Task) / 16); ++k) {
              uint4 v;
              v.x = s4[k].x; v.y = s4[k].y; v.z = s4[k].z; v.w = s4[k].w;
              d4[k] = v;
            }
            s_state = 1;
            if (g_debug_level > 0)
              printf("[worker] picked idx=%d tail=%d op=%d numel=%lld\n", h, t, s_task.op, (long long)s_task.numel);
            break;
          }
        }
        const uint64_t now = ptx::now_ns();
        if (s_state == 1) {
          idle_since = now;
          idle_sleep = 64;
          OpFn fn = nullptr;
          const int op = s_task.op;
          if (op >= 0 && op < GPUOS_MAX_OPS) {
            const int phys = *reinterpret_cast<volatile int*>(&g_op_alias[op]);
            if (phys >= 0 && phys < GPUOS_MAX_OPS)
              fn = reinterpret_cast<OpFn>(*reinterpret_cast<volatile unsigned long long*>(&g_op_table[phys]));
          }
          s_fn = fn;
        } else {
          if (blockIdx.x == 0) {
            const unsigned long long hb = atomicAdd(&g_heartbeat, 1ull) + 1;
            if (q.sync != nullptr) {
              q.sync->heartbeat = hb;
              q.sync->processed = atomicAdd(&g_processed_count, 0ull);
            }
          }
          if (ptx::elapsed(now, idle_since) > g_ring_idle_limit_ns) s_state = 2;
        }
      }
    }
    __syncthreads();
    const int state = s_state;
    if (state == 2) break;
    if (state == 0) {
      __nanosleep(idle_sleep);
      if (idle_sleep < 1024) idle_sleep <<= 1;
      continue;
    }
    OpFn fn = s_fn;
    if (fn) fn(s_task);
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned long long pc = atomicAdd(&g_processed_count, 1ull) + 1;
      if (blockIdx.x == 0 && q.sync != nullptr) q.sync->processed = pc;
      const unsigned long long ye = *reinterpret_cast<volatile unsigned long long*>(&g_yield_every);
      if (ye > 0ull && (pc % ye) == 0ull) atomicExch(q.quit, 1);
    }
    __syncthreads();
  }
  __syncthreads();
  if (threadIdx.x == 0 && blockIdx.x == 0 && q.sync != nullptr) {
    __threadfence_system();
    q.sync->processed = atomicAdd(&g_processed_count, 0ull);
  }
}

#endif  // GPUOS_JIT_WORKER
}  // namespace gpuos

using namespace gpuos;

#ifndef GPUOS_JIT_WORKER

// ---- reference C ABI (persistent_kernel.cu:233-269) --------------------------------------
extern "C" cudaError_t launch_init_builtin_ops(cudaStream_t stream) {
  init_builtin_ops_kernel<<<(GPUOS_MAX_OPS + 127) / 128, 128, 0, stream>>>();
  return cudaGetLastError();
}

// Under CUDA's default lazy module loading a kernel is loaded on its first launch, and that
// load can wait for kernels already running on the device.  A persistent worker never
// finishes on its own, so every kernel of this library is loaded before a worker starts.
extern "C" cudaError_t gpuos_internal_preload_kernels() {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, init_builtin_ops_kernel);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, builtin_addr_kernel);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, gpuos_batch_worker);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, ring_worker_kernel);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, gpuos_module_addrs);
  return e;
}

// Built-in operator addresses of this library's module (MA_COUNT values) into device memory.
extern "C" cudaError_t gpuos_internal_module_addrs(unsigned long long* d_out, cudaStream_t s) {
  gpuos_module_addrs<<<1, 64, 0, s>>>(d_out);
  return cudaGetLastError();
}

extern "C" cudaError_t launch_persistent_worker(WorkQueue q, int blocks, int threads, cudaStream_t stream) {
  if (blocks <= 0 || threads <= 0 || threads > 1024) return cudaErrorInvalidValue;
  cudaError_t e = gpuos_internal_preload_kernels();
  if (e != cudaSuccess) return e;
  ring_worker_kernel<<<blocks, threads, 0, stream>>>(q);
  return cudaGetLastError();
}

extern "C" cudaError_t gpu_get_processed_count_async(unsigned long long* out, cudaStream_t s) {
  return cudaMemcpyFromSymbolAsync(out, g_processed_count, sizeof(*out), 0, cudaMemcpyDeviceToHost, s);
}

extern "C" cudaError_t gpu_set_op_table_async(int index, OpPtrInt fn, cudaStream_t s) {
  if (index < 0 || index >= GPUOS_MAX_OPS) return cudaErrorInvalidValue;
  static thread_local OpPtrInt staged[GPUOS_MAX_OPS];
  staged[index] = fn;
  return cudaMemcpyToSymbolAsync(g_op_table, &staged[index], sizeof(fn), index * sizeof(OpFn),
                                 cudaMemcpyHostToDevice, s);
}

extern "C" cudaError_t gpu_set_alias_async(int logical_id, int physical_slot, cudaStream_t s) {
  if (logical_id < 0 || logical_id >= GPUOS_MAX_OPS || physical_slot < 0 || physical_slot >= GPUOS_MAX_OPS)
    return cudaErrorInvalidValue;
  static thread_local int staged[GPUOS_MAX_OPS];
  staged[logical_id] = physical_slot;
  return cudaMemcpyToSymbolAsync(g_op_alias, &staged[logical_id], sizeof(int), logical_id * sizeof(int),
                                 cudaMemcpyHostToDevice, s);
}

extern "C" cudaError_t gpu_get_heartbeat_async(unsigned long long* out, cudaStream_t s) {
  return cudaMemcpyFromSymbolAsync(out, g_heartbeat, sizeof(*out), 0, cudaMemcpyDeviceToHost, s);
}

extern "C" cudaError_t gpu_set_debug_level_async(int level, cudaStream_t s) {
  static thread_local int staged;
  staged = level;
  return cudaMemcpyToSymbolAsync(g_debug_level, &staged, sizeof(int), 0, cudaMemcpyHostToDevice, s);
}

extern "C" cudaError_t gpu_set_yield_every_async(unsigned long long every, cudaStream_t s) {
  static thread_local unsigned long long staged;
  staged = every;
  return cudaMemcpyToSymbolAsync(g_yield_every, &staged, sizeof(staged), 0, cudaMemcpyHostToDevice, s);
}

extern "C" cudaError_t gpuos_ring_set_idle_limit_ms(unsigned int ms, cudaStream_t s) {
  static thread_local unsigned long long staged;
  staged = (unsigned long long)ms * 1000ull * 1000ull;
  return cudaMemcpyToSymbolAsync(g_ring_idle_limit_ns, &staged, sizeof(staged), 0, cudaMemcpyHostToDevice, s);
}

// Built-in operator addresses: slot 0/1/10 codes map to add/mul/batch, codes 100+k to
// g_builtin_ref_ops[k] (element-wise op k, then reduce sum, reduce mean).
extern "C" cudaError_t gpu_get_builtin_op_async(int slot, OpPtrInt* out, cudaStream_t s) {
  int which;
  if (slot == 0) which = -1;
  else if (slot == 1) which = -2;
  else if (slot == kBatchSlot) which = -3;
  else if (slot >= 100 && slot < 100 + GPUOS_EW_NUM_OPS + 2) which = slot - 100;
  else if (slot >= 200 && slot < 200 + kExprPrograms) which = 1000 + (slot - 200);
  else which = -100;
  unsigned long long* d = nullptr;
  cudaError_t e = cudaMallocAsync(&d, sizeof(*d), s);
  if (e != cudaSuccess) return e;
  builtin_addr_kernel<<<1, 1, 0, s>>>(which, d);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, d, sizeof(*d), cudaMemcpyDeviceToHost, s);
  cudaError_t e2 = cudaFreeAsync(d, s);
  return e != cudaSuccess ? e : e2;
}

// ---- launch glue used by the host runtime (runtime.cpp) ------------------------------------
extern "C" cudaError_t gpuos_internal_launch_batch_worker(const WorkerParams* p, int blocks, int threads,
                                                          size_t smem, cudaStream_t s) {
  gpuos_batch_worker<<<blocks, threads, smem, s>>>(*p);
  return cudaGetLastError();
}

// Raise (never lower) the worker's dynamic shared-memory limit on the current device: the
// runtime and the no-allocation entry point may size their launches differently.
extern "C" cudaError_t gpuos_internal_set_worker_smem(size_t smem) {
  static std::mutex mu;
  static size_t limit[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && limit[dev] >= smem) return cudaSuccess;
  e = cudaFuncSetAttribute(gpuos_batch_worker, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess && dev >= 0 && dev < 64) limit[dev] = smem;
  return e;
}

// Worker CTAs of `threads` threads and `smem` dynamic shared memory that fit on one SM.
extern "C" cudaError_t gpuos_internal_worker_occupancy(int threads, size_t smem, int* blocks) {
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, gpuos_batch_worker, threads, smem);
}

extern "C" cudaError_t gpuos_internal_table_ptrs(void** table, void** alias) {
  cudaError_t e = cudaGetSymbolAddress(table, g_op_table);
  if (e != cudaSuccess) return e;
  return cudaGetSymbolAddress(alias, g_op_alias);
}

extern "C" size_t gpuos_internal_smem_header_bytes() { return (sizeof(SmemHeader) + 127) & ~size_t(127); }

// ---- fixed scratch of the no-allocation entry point ------------------------------------------
// gpuos_ew_batch_noalloc serves callers that may not allocate device memory, so the control
// words, ticket, layouts and tile descriptors of its one-shot worker launch live in this array,
// which every device that loads the library holds until the process exits.  In host code the
// name stands in for the array only; its device address comes from cudaGetSymbolAddress.
static_assert(StaticScratch::kBytes == 1142528, "the documented scratch size has changed");
static __device__ __align__(256) unsigned char g_noalloc_scratch[StaticScratch::kBytes];

namespace {
constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxScratchDevices];
}  // namespace

// Device address of the scratch array on the current device.  The first call on a device
// resolves the address, loads this library's kernels and sets the worker's shared-memory
// limit to `smem`; later calls return the cached address.
extern "C" cudaError_t gpuos_internal_noalloc_scratch(size_t smem, void** ptr, size_t* bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxScratchDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    e = gpuos_internal_preload_kernels();
    if (e != cudaSuccess) return e;
    e = gpuos_internal_set_worker_smem(smem);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  *bytes = StaticScratch::kBytes;
  return cudaSuccess;
}
#endif  // GPUOS_JIT_WORKER
