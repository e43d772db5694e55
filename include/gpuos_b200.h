/*
 * gpuos_b200.h — C ABI of the B200 persistent micro-op runtime.
 *
 * Two groups of entry points live in libgpuos_b200.so:
 *
 *  1. The reference's own C ABI (src/persistent_kernel.cu:233-269 of jwgale/GPUOS,
 *     prototypes repeated in pytorch_ext/gpuos_ext.cpp:23-30 and src/host.cpp:19-22).
 *     Same names, argument meaning and return type (cudaError_t).  They drive the
 *     reference-layout Task ring (WorkQueue) with the device op table.
 *
 *  2. The runtime ABI (gpuos_rt_*): the host runtime that the reference implements
 *     inside its pybind module (pytorch_ext/gpuos_ext.cpp:448-1088), exposed here with
 *     plain pointers and sizes so that any host language can bind it.  The Python
 *     module gpuos_b200.gpuos_ext is a thin binding over these calls.
 *
 * Descriptor types keep the reference layout byte for byte (src/common.h:14-74):
 * sizeof(TensorRef)=144, sizeof(Task)=496 (in0@64, in1@208, out0@352),
 * sizeof(SyncState)=64, so operators written against the reference ABI
 * (extern "C" __device__ void op(const Task&)) receive the same struct.
 */
#ifndef GPUOS_B200_H_
#define GPUOS_B200_H_

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference descriptor ABI (src/common.h:8-74) ---------------------- */
#ifndef GPUOS_MAX_OPS
#define GPUOS_MAX_OPS 128 /* src/common.h:9-11 */
#endif
#define GPUOS_MAX_NDIM 8 /* src/common.h:22 (MAX_NDIM) */

/* DType codes, src/common.h:14-20 */
enum GpuosDType { kF32 = 0, kF16 = 1, kBF16 = 2, kI32 = 3, kF64 = 4 };

/* src/common.h:25-31: data pointer + dtype + ndim + sizes/strides in elements */
typedef struct TensorRef {
  void* data;
  int dtype;
  int ndim;
  int64_t sizes[GPUOS_MAX_NDIM];
  int64_t strides[GPUOS_MAX_NDIM];
} TensorRef;

/* src/common.h:34-46: one operator invocation */
typedef struct Task {
  int op;
  int flags;
  int ndim;
  int64_t numel;
  int rrank;
  int r_axes[GPUOS_MAX_NDIM];
  int r_keepdim;
  TensorRef in0;
  TensorRef in1;
  TensorRef out0;
} Task;

/* src/common.h:52-58: zero-copy completion state in mapped pinned memory */
typedef struct SyncState {
  volatile unsigned long long processed;
  volatile unsigned long long submitted;
  volatile unsigned long long heartbeat;
  volatile int ready;
  char _pad[32];
} SyncState;

/* src/common.h:61-68: Task ring consumed by launch_persistent_worker */
typedef struct WorkQueue {
  Task* tasks;
  int capacity;
  int* head;
  int* tail;
  int* quit;
  SyncState* sync;
} WorkQueue;

typedef unsigned long long OpPtrInt; /* src/common.h:74 */

/* ---- reference C ABI (src/persistent_kernel.cu:233-269) ------------------ */

/* persistent_kernel.cu:234-239 — null the table, identity alias, install the
 * built-in operators (add@0, mul@1, batch@10) on the current device. */
cudaError_t launch_init_builtin_ops(cudaStream_t stream);

/* persistent_kernel.cu:241-244 — launch the Task-ring worker over q.  The worker
 * consumes q.tasks[head % capacity] while head < tail, dispatches each Task through
 * g_op_alias/g_op_table and counts completions in q.sync->processed.  Unlike the
 * reference, every wait is bounded: the worker exits by itself after
 * gpuos_ring_set_idle_limit_ms() of idleness (default 30000 ms). */
cudaError_t launch_persistent_worker(WorkQueue q, int blocks, int threads, cudaStream_t stream);

/* persistent_kernel.cu:247-249 — completed Task count of the ring worker. */
cudaError_t gpu_get_processed_count_async(unsigned long long* out, cudaStream_t s);

/* persistent_kernel.cu:251-253 — write a device function address into table slot. */
cudaError_t gpu_set_op_table_async(int index, OpPtrInt fn, cudaStream_t s);

/* persistent_kernel.cu:255-257 — route logical op id to physical slot. */
cudaError_t gpu_set_alias_async(int logical_id, int physical_slot, cudaStream_t s);

/* persistent_kernel.cu:259-261 — idle heartbeat counter of the ring worker. */
cudaError_t gpu_get_heartbeat_async(unsigned long long* out, cudaStream_t s);

/* persistent_kernel.cu:263-265 — device debug level (0 silent). */
cudaError_t gpu_set_debug_level_async(int level, cudaStream_t s);

/* persistent_kernel.cu:267-269 — ring worker exits after every `every` Tasks. */
cudaError_t gpu_set_yield_every_async(unsigned long long every, cudaStream_t s);

/* Device address of a built-in operator (0 if none): codes 0, 1, 10 are the operators
 * launch_init_builtin_ops installs (add, mul, batch); 100+k the reference-ABI element-wise
 * operator k, then sum and mean; 200+k the operator of expression program k.  The
 * reference tests obtain such addresses through NVRTC modules
 * (test/dual_slot_switch.cpp:78-102); this returns the built-in ones so a slot can be
 * refilled after a swap. */
cudaError_t gpu_get_builtin_op_async(int slot, OpPtrInt* out, cudaStream_t s);

/* Bound for the ring worker's idle wait (reference worker: unbounded,
 * persistent_kernel.cu:171-181). */
cudaError_t gpuos_ring_set_idle_limit_ms(unsigned int ms, cudaStream_t s);

/* ---- runtime ABI ------------------------------------------------------- */

/* Status codes returned by gpuos_rt_* (0 = success). */
enum GpuosStatus {
  GPUOS_OK = 0,
  GPUOS_ERR_INVALID = 1,     /* bad argument (dtype, shape, pointer, slot) */
  GPUOS_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
  GPUOS_ERR_TIMEOUT = 3,     /* a bounded host wait expired */
  GPUOS_ERR_DEVICE = 4,      /* the worker reported an error (bounded device wait expired) */
  GPUOS_ERR_NOT_INIT = 5,    /* runtime not initialised for this device */
  GPUOS_ERR_UNSUPPORTED = 6, /* operator / layout outside the supported set */
  GPUOS_ERR_NVRTC = 7,       /* NVRTC compile of an injected operator failed */
  GPUOS_ERR_FULL = 8         /* a fixed-size table is exhausted */
};

/* Element-wise operator codes of the batched path.  0..3 keep the sub-op codes of
 * the reference's aggregated operator (persistent_kernel.cu:101-106). */
enum GpuosEwOp {
  GPUOS_EW_ADD = 0, GPUOS_EW_MUL = 1, GPUOS_EW_SUB = 2, GPUOS_EW_DIV = 3,
  GPUOS_EW_MAXIMUM = 4, GPUOS_EW_MINIMUM = 5, GPUOS_EW_POW = 6, GPUOS_EW_COPY = 7,
  GPUOS_EW_RELU = 8, GPUOS_EW_SIGMOID = 9, GPUOS_EW_TANH = 10, GPUOS_EW_EXP = 11,
  GPUOS_EW_LOG = 12, GPUOS_EW_SQRT = 13, GPUOS_EW_ABS = 14, GPUOS_EW_HARDSIGMOID = 15,
  GPUOS_EW_HARDSWISH = 16, GPUOS_EW_GELU = 17, GPUOS_EW_GELU_TANH = 18, GPUOS_EW_SIN = 19,
  GPUOS_EW_COS = 20, GPUOS_EW_LEAKY_RELU = 21, GPUOS_EW_CLAMP = 22, GPUOS_EW_CLAMP_MIN = 23,
  GPUOS_EW_CLAMP_MAX = 24, GPUOS_EW_ELU = 25, GPUOS_EW_SOFTPLUS = 26, GPUOS_EW_NEG = 27,
  GPUOS_EW_ADD_ALPHA = 28, GPUOS_EW_SUB_ALPHA = 29,
  GPUOS_EW_NUM_OPS = 30
};

/* Reduction operator codes (reference: build_reduce_src op_name "sum"|"mean",
 * pytorch_ext/gpuos_ext.cpp:899-1001). */
enum GpuosRedOp { GPUOS_RED_SUM = 0, GPUOS_RED_MEAN = 1 };

/* An operand: the TensorRef of the reference without the fixed ndim coupling. */
typedef struct GpuosOperand {
  void* data;
  int dtype; /* GpuosDType; only kF32/kF16/kBF16 are computed */
  int ndim;  /* 0..8 */
  int64_t sizes[GPUOS_MAX_NDIM];
  int64_t strides[GPUOS_MAX_NDIM]; /* in elements */
} GpuosOperand;

typedef struct gpuos_rt gpuos_rt; /* one runtime per device */

/* gpuos_ext.init (pytorch_ext/gpuos_ext.cpp:448-540): allocate the ring and
 * control state on `device`, launch the persistent worker (one CTA per SM, each
 * `threads_per_block` compute threads, a multiple of 32 in [64, 448], plus a dequeue
 * warp and a completion warp). */
int gpuos_rt_init(int device, int capacity, int threads_per_block, gpuos_rt** out);

/* gpuos_ext.shutdown (gpuos_ext.cpp:542-592): drain, stop the worker, free. */
int gpuos_rt_shutdown(gpuos_rt* rt);

/* Runtime of `device` created by gpuos_rt_init (NULL if none). */
gpuos_rt* gpuos_rt_get(int device);

/* Batched element-wise request: out = op(a[, b]) with right-aligned broadcast of a
 * and b against out (gpuos_ext.cpp:260-297).  b may be NULL (unary) and is ignored
 * when b_is_scalar != 0, in which case `b_scalar` is the second operand.  params
 * holds op parameters (slope, bounds, alpha, beta/threshold), up to 4.  Requests
 * are kept pending until gpuos_rt_flush (gpuos_ext.cpp:638-672). */
int gpuos_rt_submit_ew(gpuos_rt* rt, int op, const GpuosOperand* a, const GpuosOperand* b,
                       int b_is_scalar, double b_scalar, const GpuosOperand* out,
                       const float* params, int nparams);

/* Batched top-k (replaces the torch::topk call behind submit_topk, gpuos_ext.cpp:1050-1071, on
 * the persistent worker): for every row of x [rows, n] (contiguous, dtype a GpuosDtype float
 * code) writes the k largest (largest != 0) or smallest elements, preferred first, to values
 * [rows, k] (x's dtype) and their positions to indices [rows, k] (int64), both contiguous.  NaN
 * counts as the largest value (as PyTorch's topk); equal values take the lower position first.
 * 1 <= k <= min(n, 256).  Pending until gpuos_rt_flush, ordered against other requests that
 * touch the same memory. */
int gpuos_rt_submit_topk(gpuos_rt* rt, const void* x, int dtype, int64_t rows, int64_t n, void* values,
                         int64_t* indices, int k, int largest);

/* Bulk form of gpuos_rt_submit_ew for n requests: request i is ops[i] on a[i], b[i] (b may be
 * NULL when every op is unary) and out[i], parameters 0.  A bulk submitter beside the
 * reference's one-call-per-op submit_* (gpuos_ext.cpp:638-672): every request is validated
 * before any is submitted, and all are appended under one lock acquisition. */
int gpuos_rt_submit_ew_many(gpuos_rt* rt, int n, const int* ops, const GpuosOperand* a, const GpuosOperand* b,
                            const GpuosOperand* out);

/* Batched reduction: out = sum|mean of x over `axes` (gpuos_ext.cpp:1016-1045). */
int gpuos_rt_submit_reduce(gpuos_rt* rt, int red_op, const GpuosOperand* x,
                           const GpuosOperand* out, const int* axes, int naxes, int keepdim);

/* Reference-layout Task dispatched through g_op_alias/g_op_table at dequeue time
 * (gpuos_ext.cpp:884-896, 1040-1045).  Large Tasks are split along their leading
 * output dimension into Tasks that are each valid on their own. */
int gpuos_rt_submit_task(gpuos_rt* rt, const Task* task);

/* Flags of gpuos_rt_flush. */
#define GPUOS_FLUSH_SYNC 1 /* return once this flush (and every earlier one) has completed */
#define GPUOS_FLUSH_DEP 2  /* work already enqueued on dep_stream (which may be the legacy
                              default stream, handle 0) finishes before the requests run */

/* Publish every pending request (gpuos_ext.cpp:675-811).  *seq_out (optional) receives
 * the flush ticket (0 when nothing was pending). */
int gpuos_rt_flush(gpuos_rt* rt, int flags, cudaStream_t dep_stream, uint64_t* seq_out);

/* Wait until flush ticket `seq` and every earlier flush have completed, at most timeout_ms
 * (flushes can finish out of order on the device). */
int gpuos_rt_wait(gpuos_rt* rt, uint64_t seq, int timeout_ms);

/* Highest ticket t such that every flush with ticket <= t has completed. */
uint64_t gpuos_rt_completed(gpuos_rt* rt);

/* Zero-copy polls (gpuos_ext.cpp:134-150): completed requests, worker heartbeat,
 * worker ready flag.  No CUDA call is made. */
uint64_t gpuos_rt_poll_processed(gpuos_rt* rt);
uint64_t gpuos_rt_poll_heartbeat(gpuos_rt* rt);
int gpuos_rt_poll_ready(gpuos_rt* rt);

/* Wait until the processed count reaches target (gpuos_ext.cpp:160-212). */
int gpuos_rt_sync_wait(gpuos_rt* rt, uint64_t target, int timeout_ms);

/* Worker liveness (gpuos_ext.cpp:241-248) and relaunch (gpuos_ext.cpp:214-239). */
int gpuos_rt_worker_alive(gpuos_rt* rt);
int gpuos_rt_ensure_worker(gpuos_rt* rt);

/* Drain and stop the worker without freeing anything; the next flush relaunches it. */
int gpuos_rt_quiesce(gpuos_rt* rt, int timeout_ms);

/* Control knobs (gpuos_ext.cpp:594-604). */
int gpuos_rt_set_debug_level(gpuos_rt* rt, int level);
int gpuos_rt_set_yield_every(gpuos_rt* rt, uint64_t every);
/* Host-side idle time after which the worker is stopped (0: stop after every drain; -1:
 * never; default 200, env GPUOS_IDLE_QUIESCE_MS).  The worker is idle when nothing flushed
 * is in flight (requests not yet flushed do not keep it).  A resident worker holds most of
 * every SM (all of its registers at 448 compute threads), so kernels on other streams that
 * do not fit beside it wait until it stops.  A flush whose inputs come from such a kernel
 * stops the worker itself and relaunches it.  With -1 other waits last until
 * gpuos_rt_quiesce or shutdown: a blocking CUDA call that waits for such a kernel (a
 * synchronous copy, a stream synchronize) does not return before then. */
int gpuos_rt_set_idle_quiesce_ms(gpuos_rt* rt, int ms);
/* Bound (ms) of the worker's in-grid waits (default 5000, env GPUOS_DEVICE_WAIT_MS).  A
 * worker reads the bound when it is launched, so a running worker is stopped first
 * (gpuos_rt_quiesce) and the next flush launches one with the new bound. */
int gpuos_rt_set_device_wait_ms(gpuos_rt* rt, int ms);
/* Failure-path test hook: publish one item whose dependency barrier never opens.  The
 * worker's bounded wait expires, it reports "dependency barrier wait expired" and exits;
 * the runtime then fails every later call until shutdown.  No GPU fault is involved. */
int gpuos_rt_debug_inject_stall(gpuos_rt* rt);

/* Queue state for peek_queue (gpuos_ext.cpp:606-635).  Fills `vals` with up to n
 * values in the order named by gpuos_rt_stat_names() (comma separated). */
int gpuos_rt_stats(gpuos_rt* rt, int64_t* vals, int n);
const char* gpuos_rt_stat_names(void);

/* Op table control of the runtime (gpuos_ext.cpp:361-363, persistent_kernel.cu:251-257).
 * The runtime's table starts as launch_init_builtin_ops sets the reference one (add@0, mul@1,
 * batch@10, identity alias).  Writes take effect for Tasks dequeued after the call returns
 * (online switch / dual-slot switch / rollback).  An address of this library's module (from
 * gpu_get_builtin_op_async) is taken to mean the same operator of the module the worker runs. */
int gpuos_rt_set_slot(gpuos_rt* rt, int slot, OpPtrInt fn);
int gpuos_rt_get_slot(gpuos_rt* rt, int slot, OpPtrInt* fn);
int gpuos_rt_set_alias(gpuos_rt* rt, int logical, int physical);
int gpuos_rt_get_alias(gpuos_rt* rt, int logical, int* physical);

/* Built-in reference-ABI operators that can be placed in a slot: reduce sum/mean
 * (gpuos_ext.cpp:899-1001) and the built-in element-wise ops of GpuosEwOp with
 * zero parameters.  Returns the allocated slot (>= 20) in *slot. */
int gpuos_rt_register_builtin_reduce(gpuos_rt* rt, int red_op, int* slot);
int gpuos_rt_register_builtin_ew(gpuos_rt* rt, int ew_op, int* slot);

/* register_elementwise through the worker's expression interpreter (the alternative to
 * gpuos_rt_register_jit that loads nothing and never stops the worker;
 * gpuos_ext.cpp:814-881 compiles with NVRTC): `expr` is a C float expression in A (and B when
 * arity == 2) — literals, + - * /, comparisons, ! && ||, ?:, (float) casts and the float
 * functions exp log log1p expm1 sqrt rsqrt fabs tanh sin cos tan erf floor ceil trunc round
 * exp2 log2 log10 sinh cosh asin acos atan fmin fmax pow fmod atan2 copysign (with or
 * without the f suffix).  It is compiled on the host into a program for the worker's stack
 * machine (at most 64 steps, 16 stack slots) and becomes a reference-ABI operator: element i
 * of out = expr of element i of in0/in1 under the Task's broadcast strides, computed in float
 * (transcendental functions in double, rounded once) and stored as out's dtype.  Up to 32 expressions per device; the operator goes to `slot`
 * (< 0: next free slot >= 20), *slot_out receives the slot.  No module is loaded, so a
 * running worker keeps running. */
int gpuos_rt_register_expr(gpuos_rt* rt, const char* key, const char* expr, int arity,
                           int slot, int* slot_out);

/* Compile-only check of a gpuos_rt_register_expr expression (no device needed).  With
 * prog_out non-NULL (prog_bytes >= 336) the program is copied out: code[64] (uint8 opcodes),
 * imm[64] (float constants), then int32 len, arity, depth. */
int gpuos_expr_compile(const char* expr, int arity, void* prog_out, int prog_bytes);

/* ---- operators compiled at run time ---------------------------------------------------------
 * Replaces the reference's NVRTC path (pytorch_ext/gpuos_ext.cpp:316-363 compile + load +
 * address read, :814-881 register_elementwise, :1079-1088 load_and_register_custom).  There
 * each operator is a module of its own whose address the running worker calls; here each
 * operator is compiled by NVRTC as relocatable sm_100a code held to the worker's register
 * budget, linked (nvJitLink) with the worker's relocatable code and every operator installed
 * before it, and the worker runs from the linked module: the call stays inside one module.
 * Installing stops the worker (published work drains first), loads the linked module (a module
 * load waits for kernels running on the device), carries the op table and expression programs
 * over to the new module's addresses and lets the next flush relaunch the worker.  Queued
 * requests are not lost.  Each runtime resolves Tasks through its own op table (gpuos_rt_set_slot,
 * gpuos_rt_set_alias); the table of the reference C ABI (gpu_set_op_table_async, read by
 * launch_persistent_worker) is separate and only ever holds addresses of this library's module.
 * NVRTC and nvJitLink are opened from $CUDA_HOME/lib64 (default /usr/local/cuda).  Up to 64
 * operators per device. */

/* register_elementwise (gpuos_ext.cpp:814-881): element i of out = expr(A[, B]) over a
 * reference-layout Task, A and B read with the Task's sizes/strides and dtypes, computed in
 * float with every transcendental function evaluated in double and rounded once, stored as
 * out's dtype (round to nearest even).  expr is a C float expression (no ';', braces or
 * quotes).  Goes to `slot` (< 0: next free slot >= 20); *slot_out receives it. */
int gpuos_rt_register_jit(gpuos_rt* rt, const char* expr, int arity, int slot, int* slot_out);

/* load_and_register_custom (gpuos_ext.cpp:1079-1088, fixed): `ptx` (ptx_len bytes) holds
 * extern "C" __device__ void <entry>(const Task&) (the reference operator ABI, src/common.h:71);
 * it is linked into the worker and entry's device address goes to `slot` (the reference stores
 * a host CUfunction handle there). */
int gpuos_rt_load_custom(gpuos_rt* rt, const char* ptx, size_t ptx_len, const char* entry, int slot,
                         int* slot_out);

/* The two halves of gpuos_rt_register_jit / gpuos_rt_load_custom, so that the slow half can run
 * ahead of a switch point: gpuos_rt_jit_stage[_ptx] compiles and links (seconds; no device
 * work, the worker keeps running), gpuos_rt_jit_commit stops the worker, loads the staged module
 * and installs the operator in `slot` (milliseconds).  A staged operator can be committed only
 * while no other operator was installed on the device after it was staged
 * (GPUOS_ERR_INVALID otherwise: stage again).  gpuos_rt_jit_discard frees a staged operator
 * (committed or not). */
typedef struct gpuos_jit_staged gpuos_jit_staged;
int gpuos_rt_jit_stage(gpuos_rt* rt, const char* expr, int arity, gpuos_jit_staged** staged);
int gpuos_rt_jit_stage_ptx(gpuos_rt* rt, const char* ptx, size_t ptx_len, const char* entry,
                           gpuos_jit_staged** staged);
int gpuos_rt_jit_commit(gpuos_rt* rt, gpuos_jit_staged* staged, int slot, int* slot_out);
void gpuos_rt_jit_discard(gpuos_jit_staged* staged);

/* Operators compiled at run time installed on the runtime's device (negative: -status). */
int gpuos_rt_jit_ops(gpuos_rt* rt);

/* Address of a built-in operator (codes as gpu_get_builtin_op_async) in the worker module the
 * runtime currently runs: what a slot must hold to run that operator. */
int gpuos_rt_builtin_op(gpuos_rt* rt, int code, OpPtrInt* addr);

/* Device-free checks (no CUDA device needed).  gpuos_jit_compile: NVRTC output of `src` for
 * sm_100a (relocatable code, or PTX when ptx != 0); *size_out receives its size, copied to out
 * when out != NULL and cap is large enough.  gpuos_jit_check_expr: compile a
 * gpuos_rt_register_jit operator and link it with the worker; *image_bytes receives the size
 * of the linked image.  gpuos_jit_nvrtc_version: major*1000 + minor*10, 0 if NVRTC cannot be
 * opened. */
int gpuos_jit_compile(const char* src, int ptx, void* out, size_t cap, size_t* size_out);
int gpuos_jit_check_expr(const char* expr, int arity, size_t* image_bytes);
int gpuos_jit_nvrtc_version(void);

/* Device %globaltimer stamps of a completed flush: start of its first item and end
 * of its last item (ns).  Returns GPUOS_ERR_INVALID if `seq` is not complete or has
 * been recycled (only the most recent 1024 flushes are kept). */
int gpuos_rt_flush_times(gpuos_rt* rt, uint64_t seq, uint64_t* t_start, uint64_t* t_end);

/* The stream the worker kernel is launched on, and the number of worker launches so
 * far (for CUDA events around launches and launch counting). */
cudaStream_t gpuos_rt_kernel_stream(gpuos_rt* rt);
uint64_t gpuos_rt_launches(gpuos_rt* rt);

/* Launch timing: while on, every worker launch is bracketed by two CUDA events recorded on
 * the worker's stream right before and after the launch.  gpuos_rt_launch_times writes the
 * durations (ms) of up to `max` finished launches, oldest first, drops them, and returns
 * their number (negative status on error). */
int gpuos_rt_set_launch_timing(gpuos_rt* rt, int on);
int gpuos_rt_launch_times(gpuos_rt* rt, float* ms_out, int max);

/* Per-CTA cycle counters of the last worker launch (valid once it has exited, e.g.
 * after gpuos_rt_quiesce): rows of 12 counters (stage wait, claim, idle, descriptor
 * fetch, staging, items staged, fill wait, tile, completer wait, completion, bulk-copy
 * issue, total cycles), one row per CTA, followed by one row of %globaltimer stamps (ns)
 * of the launch's first events: launch initialised, first claim, first staging, first bulk
 * copies, first tile start and end, first completion accounting, first exit round, first
 * gather, exit verdict, first and last CTA finished (~0 where an event did not happen).
 * Copies min(n, (ctas+1)*12) values into out and returns the number of CTAs (negative
 * status on error). */
int gpuos_rt_debug_counters(gpuos_rt* rt, uint64_t* out, int n);

/* Device-free planning hooks (no CUDA call): the 64-byte work items (and, for strided
 * requests, the 432-byte layout record) a request would be split into.  Used to test
 * broadcast, dimension coalescing and tiling on hosts without a GPU.  items_out holds
 * max_items * 64 bytes; layout_out (may be NULL) 512 bytes. */
int gpuos_plan_ew(int op, const GpuosOperand* a, const GpuosOperand* b, int b_is_scalar, double b_scalar,
                  const GpuosOperand* out, const float* params, int nparams, void* items_out,
                  int max_items, void* layout_out, int* n_items);
int gpuos_plan_reduce(int red_op, const GpuosOperand* x, const GpuosOperand* out, const int* axes,
                      int naxes, int keepdim, void* items_out, int max_items, void* layout_out,
                      int* n_items);

/* ---- element-wise batch without device allocation ----------------------------------------
 * No counterpart in the reference: the reference allocates its queue and control state with
 * cudaMalloc/cudaHostAlloc at init.  Some callers may not allocate device memory where they
 * run: an execute hook inside a host engine that owns every byte of device memory and forbids
 * allocation while it executes, or a latency-critical path that cannot afford cudaMalloc's
 * implicit device synchronisation.  gpuos_ew_batch_noalloc runs the same worker kernel as
 * gpuos_rt_submit_ew + gpuos_rt_flush, once, on `stream`, over `nreq` element-wise requests,
 * with all of its scratch (control words, completion ticket, tile descriptors, strided
 * layouts) in one fixed array of device memory that is part of this library: 1,142,528 bytes
 * (1.09 MiB) per device, held by every device that loads the library until the process exits.  It calls
 * no cudaMalloc, cudaFree or other allocating routine.
 *
 * Limits: the requests together may be split into at most GPUOS_NOALLOC_MAX_TILES tiles
 * (16 KiB of one operand each: 4096 float32 or 8192 16-bit elements), of which at most
 * GPUOS_NOALLOC_MAX_STRIDED requests may need the strided/broadcast path; larger batches are
 * rejected with GPUOS_ERR_INVALID before anything runs.
 *
 * The work runs on the current device, in stream order on `stream`: requests see earlier
 * work on `stream`, later work on `stream` sees their results, and requests of one call that
 * overlap in memory run in submission order.  Without GPUOS_FLUSH_SYNC the call returns once
 * the work is enqueued; with it, the call waits for `stream` (at most GPUOS_NOALLOC_WAIT_MS,
 * default 60000 ms, then GPUOS_ERR_TIMEOUT) and reports a device-side error (GPUOS_ERR_DEVICE).
 * The first device-side error of a call made without GPUOS_FLUSH_SYNC is kept in the array and
 * reported, then cleared, by the next call made with it on that device; a call with nreq == 0
 * and GPUOS_FLUSH_SYNC only does that (a status query).  Every call shares the one scratch
 * array and resets it: calls that overlap on the GPU (issued on different streams, or from
 * different threads) race and corrupt each other.  The first call on a device resolves the array's address and sets up
 * the kernel; make that first call before any stream capture is begun.  The launch puts one
 * CTA on every SM and its CTAs coordinate with one another, so all of them must be resident at
 * once: kernels on other streams that hold SMs for longer than GPUOS_DEVICE_WAIT_MS (default
 * 5000 ms) make it fail with a device-side error instead of running.  The persistent worker of
 * gpuos_rt_init, while running on the same device, holds those SMs, so the launch starts once
 * that worker has gone idle (GPUOS_IDLE_QUIESCE_MS); with the idle stop disabled
 * (gpuos_rt_set_idle_quiesce_ms(rt, -1)) it starts only after gpuos_rt_quiesce or shutdown, and a
 * synchronous call returns GPUOS_ERR_TIMEOUT meanwhile. */
#define GPUOS_NOALLOC_MAX_TILES 16384
#define GPUOS_NOALLOC_MAX_STRIDED 64

typedef struct GpuosEwRequest {
  int op;                  /* GpuosEwOp */
  int b_is_scalar;         /* nonzero: b is ignored and b_scalar is the second operand */
  int nparams;             /* entries of params in use (0..4) */
  int _pad;
  double b_scalar;
  const GpuosOperand* a;   /* as gpuos_rt_submit_ew */
  const GpuosOperand* b;   /* may be NULL for unary ops */
  const GpuosOperand* out;
  float params[4];
} GpuosEwRequest;

int gpuos_ew_batch_noalloc(const GpuosEwRequest* reqs, int nreq, int flags, cudaStream_t stream);

/* Last error message of this thread (never NULL). */
const char* gpuos_rt_last_error(void);

/* sizeof() of the ABI structs, for binding-side layout checks. */
int gpuos_abi_sizes(int64_t* out, int n);

#ifdef __cplusplus
}
#endif
#endif /* GPUOS_B200_H_ */
