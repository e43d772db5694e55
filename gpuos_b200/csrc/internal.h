// internal.h — descriptors shared by the host runtime and the device worker.
//
// The reference publishes one 496-byte Task per ring slot and aggregates micro
// requests into "batch" Tasks whose sub-tasks one CTA walks serially
// (src/persistent_kernel.cu:81-112, pytorch_ext/gpuos_ext.cpp:755-778).  Here a flush is
// split into 64-byte work items (a tile of one request, a group of reduction rows,
// or one reference-layout Task) that every CTA of the persistent grid claims from a
// ring in mapped pinned memory.  Items are self-contained for the contiguous case so
// the dequeue warp needs a single 64-byte read per item.
#pragma once
#include <stdint.h>
#include "gpuos_b200.h"

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
#define GPUOS_HD __host__ __device__
#else
#define GPUOS_HD
#endif

namespace gpuos {

// ---- item kinds -----------------------------------------------------------------
enum ItemKind : uint8_t {
  IK_NONE = 0,
  IK_EW_CONTIG = 1,   // 1-D contiguous element-wise tile (operands staged by TMA bulk copy)
  IK_EW_GENERIC = 2,  // strided / broadcast element-wise tile (layout record)
  IK_ROW_REDUCE = 3,  // group of rows reduced over the last (possibly strided) axis
  IK_RED_GENERIC = 4, // arbitrary-axes reduction, one output element per thread
  IK_TASK = 5,        // reference-layout Task dispatched through g_op_alias/g_op_table
  IK_EW_2D = 6,       // element-wise block of a 2-D strided / broadcast layout (layout record)
  IK_TOPK = 7,        // top-k of each row of a group of contiguous rows (staged like a row group)
  IK_EW_2DT = 8,      // 2-D block of every row x a column range whose operand a runs along rows:
                      // a's block is one contiguous span, staged by one bulk copy and transposed
                      // in shared memory (layout record)
  IK_EXIT = 255       // in-CTA sentinel (never in the ring)
};

enum ItemFlags : uint8_t {
  IF_B_PRESENT = 1,   // binary op: operand b exists
  IF_B_SCALAR = 2,    // b is an immediate float held in the low 32 bits of WorkItem::b
  IF_A_BCAST = 4,     // EW_CONTIG: a is one element broadcast over the tile
  IF_B_BCAST = 8,     // EW_CONTIG: b is one element (in memory) broadcast over the tile
  IF_UNSTAGED = 16,   // ROW_REDUCE: rows read directly from global memory
  IF_MEAN = 32,       // reductions: divide by the reduced extent
  IF_A_T = 64,        // EW_2D: a is contiguous along rows; read through a shared-memory transpose
  IF_B_T = 128        // EW_2D: the same for b
};

// One work item (64 bytes).  Field use per kind:
//   EW_CONTIG   a,b,o = operand addresses of the tile's first element; count = elements;
//               x = two float params (p0 low, p1 high); aux = layout index when the op
//               needs more than two params (else 0xffffffff).
//   EW_GENERIC  a,b,o = base addresses; x = first output linear index; count = elements;
//               aux = layout index.
//   ROW_REDUCE  a = first element of the first row; o = first output; count = rows;
//               aux = row length C; x = row stride (elements); b = element stride.
//   RED_GENERIC a,o = base addresses; x = first output linear index; count = outputs;
//               aux = layout index.
//   TASK        aux = task ring index; op = logical op id (low 8 bits of Task::op).
//   EW_2DT      a,b,o = base addresses; count = (rows << 16) | columns; x = log2 of the block's
//               power-of-two column width (low 32 bits) | first column << 32; aux = layout index.
struct alignas(64) WorkItem {
  uint8_t kind;
  uint8_t op;
  uint8_t dt_a;
  uint8_t dt_b;
  uint8_t dt_o;
  uint8_t flags;
  uint16_t batch;        // ticket slot of the flush this item belongs to
  uint32_t count;
  uint32_t aux;
  uint64_t a;
  uint64_t b;
  uint64_t o;
  uint64_t x;
  uint64_t wait_items;   // start only once items_done >= wait_items (dependency barrier)
  uint32_t batch_items;  // number of items of this flush
  uint32_t batch_seq;    // low 32 bits of the flush ticket
};
static_assert(sizeof(WorkItem) == 64, "WorkItem must be 64 bytes");

// Strided layout for EW_GENERIC / RED_GENERIC (coalesced dims, in elements).
struct alignas(16) Layout {
  int32_t ndim;        // output dims
  int32_t rdim;        // reduced dims (RED_GENERIC)
  float params[4];
  int64_t sizes[GPUOS_MAX_NDIM];
  int64_t sa[GPUOS_MAX_NDIM];
  int64_t sb[GPUOS_MAX_NDIM];
  int64_t so[GPUOS_MAX_NDIM];
  int64_t rsizes[GPUOS_MAX_NDIM];
  int64_t rsa[GPUOS_MAX_NDIM];
  int64_t rtotal;
  int64_t _pad;
};
static_assert(sizeof(Layout) <= 512, "Layout must fit the stage extension area");

// ---- control blocks ----------------------------------------------------------------
// Host-written, device-read (mapped pinned memory).
struct alignas(128) HostCtl {
  volatile uint64_t tail;            // items published (global monotonic index)
  volatile uint64_t quit_epoch;      // workers with epoch <= quit_epoch exit once drained
  volatile uint64_t host_beat;       // incremented by the host keeper thread
  volatile uint64_t safety_idle_ns;  // exit if idle and host_beat unchanged this long
  volatile uint64_t yield_every;     // exit after this many completed items (0: never)
  volatile uint32_t debug_level;
  volatile uint32_t spin_ns;         // idle poll back-off of the leader
  volatile uint64_t wait_limit_ns;   // bound of the worker's in-grid waits
  uint64_t _pad[9];
};

// Device-written, host-read (mapped pinned memory).  Every field has one writer.
enum WorkerState : uint64_t { WS_NONE = 0, WS_RUNNING = 1, WS_EXITING = 2, WS_EXITED = 3 };
struct alignas(128) DevReport {
  volatile uint64_t ready_epoch;     // epoch of the last worker that came up
  volatile uint64_t heartbeat;       // leader idle-poll counter
  volatile uint64_t state;           // (epoch << 8) | WorkerState
  volatile uint64_t exit_tail;       // items < exit_tail were processed when it exited
  volatile uint64_t error;           // (code << 32) | detail; 0 = no error
  volatile uint64_t error_item;      // item index involved in the error
  volatile uint64_t head_mirror;     // dequeue position (for peek_queue)
  volatile uint64_t items_done;      // completed items (mirror)
  // diagnostics (leader / last CTA)
  volatile uint64_t t_launch;        // %globaltimer when CTA 0 initialised the launch
  volatile uint64_t t_exit;          // %globaltimer when the last CTA left
  volatile uint64_t park_rounds;     // exit rounds started by the leader (this launch)
  volatile uint64_t park_timeouts;   // rounds abandoned because not every CTA parked in time
  volatile uint64_t park_work;       // rounds abandoned because work arrived
  volatile uint64_t host_read_ns_max;  // slowest leader read of the host tail
  volatile uint64_t host_read_ns_avg;  // average leader read of the host tail
  volatile uint64_t parked_seen;     // CTAs parked when the last round was abandoned
};

enum DeviceError : uint32_t {
  DE_NONE = 0,
  DE_WAIT_EMPTY = 1,    // dequeue warp: compute warps did not release a stage in time
  DE_WAIT_FULL = 2,     // compute warps: dequeue warp stopped feeding
  DE_WAIT_BARRIER = 3,  // dependency barrier did not open in time
  DE_WAIT_PARK = 4,     // grid exit coordination timed out
  DE_WAIT_START = 5,    // grid start coordination timed out
  DE_BAD_ITEM = 6,      // malformed item (kind / slot / ndim out of range)
  DE_NULL_OP = 7,       // table slot resolved to a null function
  DE_HOST_LOST = 8,     // host heartbeat stopped while idle
  DE_WAIT_DONE = 9      // completer: compute warps did not finish a stage in time
};

// Completion ticket of one flush (mapped pinned memory, one writer).
struct alignas(32) Ticket {
  volatile uint64_t seq;       // flush ticket once complete
  volatile uint64_t t_start;   // %globaltimer when its first item started
  volatile uint64_t t_end;     // %globaltimer when its last item completed
  volatile uint64_t tseq;      // flush whose t_start/t_end are written (after seq)
};

constexpr int kNumBatchSlots = 1024;

// ---- registered expression operators ------------------------------------------------
// register_elementwise(key, expr, arity) compiles `expr` (a C float expression in A and B)
// on the host into a postfix program for a small stack machine; the worker evaluates it per
// element.  Installing an operator writes a program into a device table: no module is
// loaded while the persistent worker runs.
constexpr int kExprMaxCode = 64;   // instructions per program
constexpr int kExprMaxStack = 16;  // evaluation stack depth
constexpr int kExprPrograms = 32;  // programs per device (each gets its own operator address)
enum ExprOp : uint8_t {
  XO_END = 0,
  XO_A, XO_B, XO_CONST,                                        // push A, B, imm[pc]
  XO_NEG, XO_NOT,                                              // unary operators
  XO_ADD, XO_SUB, XO_MUL, XO_DIV,                              // arithmetic
  XO_LT, XO_LE, XO_GT, XO_GE, XO_EQ, XO_NE, XO_AND, XO_OR,     // comparisons, logic (1 / 0)
  XO_SELECT,                                                   // c ? x : y  (pops y, x, c)
  XO_EXP, XO_LOG, XO_LOG1P, XO_EXPM1, XO_SQRT, XO_RSQRT, XO_ABS, XO_TANH, XO_SIN, XO_COS,
  XO_TAN, XO_ERF, XO_FLOOR, XO_CEIL, XO_TRUNC, XO_ROUND, XO_EXP2, XO_LOG2, XO_LOG10,
  XO_SINH, XO_COSH, XO_ASIN, XO_ACOS, XO_ATAN,                 // one-argument functions
  XO_MIN, XO_MAX, XO_POW, XO_FMOD, XO_ATAN2, XO_COPYSIGN,      // two-argument functions
  XO_NUM
};
struct ExprProg {
  uint8_t code[kExprMaxCode];
  float imm[kExprMaxCode];  // constant of an XO_CONST at the same index
  int32_t len;
  int32_t arity;
  int32_t depth;            // stack slots the program needs
  int32_t _pad;
};
static_assert(sizeof(ExprProg) == 336, "ExprProg layout");

// ---- worker modules -------------------------------------------------------------------
// The worker runs from this library's module until an operator compiled at run time is
// installed; from then on it runs from a module that links the worker's relocatable code with
// every such operator (function pointers are only called within the module they belong to).
// gpuos_module_addrs writes each module's built-in operator addresses in this order.
enum ModuleAddr : int {
  MA_ADD = 0,                                      // op_add (slot 0 at init)
  MA_MUL = 1,                                      // op_mul (slot 1 at init)
  MA_BATCH = 2,                                    // op_batch (slot 10 at init)
  MA_REF_OPS = 3,                                  // reference-ABI element-wise ops, then sum, mean
  MA_EXPR_FNS = MA_REF_OPS + GPUOS_EW_NUM_OPS + 2, // expression-program operators
  MA_EXPR_PROGS = MA_EXPR_FNS + kExprPrograms,     // address of the module's program table
  MA_COUNT
};
constexpr int kMaxJitOps = 64;  // run-time compiled operators per device

// Per-CTA cycle counters (clock64) of one launch, written when the CTA exits.
enum DiagSlot {
  DG_P_WAIT_EMPTY = 0,  // dequeue warp: waiting for a free stage
  DG_P_CLAIM,           // dequeue warp: ticket atomics
  DG_P_IDLE,            // dequeue warp: waiting for publication (idle / park)
  DG_P_DESC,            // dequeue warp: descriptor fetch from the mapped ring
  DG_P_STAGE,           // dequeue warp: staging (barrier check, TMA issue, Task run)
  DG_P_ITEMS,           // items staged
  DG_C_WAIT_FULL,       // compute thread 0: waiting for a filled stage
  DG_C_TILE,            // compute thread 0: tile function
  DG_C_BAR,             // compute thread 0: compute-warp barrier after the tile
  DG_C_COMPLETE,        // compute thread 0: completion accounting
  DG_C_FILL,            // compute thread 0: from the bulk-copy issue of an item to seeing it staged (summed)
  DG_CYCLES,            // total cycles of the CTA
  kDiagSlots = 12
};
constexpr int kDiagCtas = 512;  // worker CTAs per launch stay below this (one row per CTA + timeline)

// Launch timeline: %globaltimer stamps of the first occurrence of each event in the last
// worker launch, kept in diag row gridDim.x (the row after the last CTA's).
enum TimelineSlot {
  TL_INIT = 0,    // CTA 0 initialised the launch
  TL_CLAIM,       // first ticket claim
  TL_STAGE,       // first item staging began
  TL_TMA,         // first bulk copies issued
  TL_TILE0,       // first tile started
  TL_TILE1,       // first tile finished
  TL_ACCOUNT,     // first completion accounting
  TL_ROUND,       // leader opened the first exit round
  TL_GATHER,      // leader's first gather ended (all parked, work, or timeout)
  TL_VERDICT,     // leader published the exit verdict
  TL_EXIT_FIRST,  // first CTA finished
  TL_EXIT_LAST    // last CTA finished
};

// Device-memory control block (cudaMalloc, zeroed at init).
struct alignas(128) DevCtl {
  unsigned long long head;         // next item ticket
  unsigned long long items_done;   // completed items (dependency barriers)
  unsigned long long tail_mirror;  // leader's copy of HostCtl::tail
  unsigned long long launch_epoch; // set by CTA 0 once the launch is initialised
  unsigned long long exit_tail;    // head value for the next launch
  unsigned long long closing;      // leader requests grid exit (round number)
  unsigned long long verdict;      // (round << 2) | 1 resume | 2 exit
  unsigned long long park_min;     // lowest held ticket among parked CTAs
  unsigned long long err_wait;      // first expired wait: (waited us << 32) | bound ms
  unsigned int abort;              // a CTA hit an error: everybody exits
  unsigned int exited;             // CTAs that left the current launch
  unsigned long long yield_base;   // items_done at launch (yield accounting)
  // HostCtl words as CTA 0 read them at launch: every other CTA takes them from here, so a
  // launch reads host memory from one thread only
  unsigned long long p_wait_limit_ns, p_safety_idle_ns, p_yield_every, p_quit_epoch, p_spin_ns;
  unsigned long long parked[kDiagCtas];  // per CTA: the exit round it last parked in
  unsigned int batch_done[kNumBatchSlots];
  unsigned long long batch_t0[kNumBatchSlots];
  unsigned long long diag[kDiagCtas][kDiagSlots];  // per-CTA cycle counters of the last launch
};

// ---- worker launch parameters ---------------------------------------------------------
typedef void (*OpFn)(const Task&);

struct WorkerParams {
  HostCtl* hc;
  DevReport* rep;
  Ticket* tickets;
  const WorkItem* items;
  const Task* tasks;
  const Layout* layouts;
  DevCtl* dc;
  OpFn* op_table;
  int* op_alias;
  uint64_t item_mask;     // item ring capacity - 1 (power of two)
  uint32_t task_mask;
  uint32_t layout_mask;
  uint64_t epoch;
  uint32_t stages;
  uint32_t stage_bytes;   // operand buffer bytes per stage
  uint32_t compute_threads;
  uint32_t account_every;  // completions accounted per gpu-scope fence while work is staged (0: 8)
  uint32_t load_hint;      // nonzero: operand bulk loads carry an L2 evict-first policy
  uint32_t _pad;
  uint64_t wait_limit_ns;  // bound of the launch-start wait (HostCtl::wait_limit_ns at launch)
  // optional: the first error of the launch is also recorded here (if still 0), in memory that
  // outlives the launch's report (the no-allocation entry point's sticky error word)
  unsigned long long* sticky_error;
};

// Per-stage bookkeeping in shared memory.
struct alignas(64) StageMeta {
  WorkItem item;
  uint32_t a_off;       // byte offset of the first a element inside the staged buffer
  uint32_t b_off;
  uint32_t staged;      // bit0: a staged, bit1: b staged
  uint32_t _pad;
  unsigned long long t_issue;  // clock64 when the item's copies were issued (diagnostics)
  union {
    Task task;
    Layout layout;
    unsigned char raw[512];
  } ext;
};

// Worker shared-memory header (stage buffers follow, 128-byte aligned).
constexpr int kMaxStages = 8;
// Dequeue-warp state used off the per-item path (leader polling, exit rounds, diagnostics);
// kept in shared memory so the per-item state stays in registers.
struct ProdCold {
  uint64_t seen_round;  // last closing round handled
  uint64_t round;       // leader: current closing round
  uint64_t beat_val;    // leader: last observed host beat
  uint64_t beat_t;      // leader: when it changed
  uint64_t polls;
  uint64_t quit_epoch, yield_every, safety_ns;  // leader: host control words (refreshed while idle)
  uint64_t spin_ns;
  uint64_t read_sum, read_n, read_max;          // leader: host tail read latency
  uint64_t mirrored;                            // leader: last value stored to DevCtl::tail_mirror
  uint64_t rounds, timeouts, work_resumes, parked_seen;
  unsigned long long dg[7];  // DG_P_WAIT_EMPTY .. DG_P_ITEMS, then the bulk-copy issue cycles
};

struct alignas(128) SmemHeader {
  unsigned long long full[kMaxStages];   // dequeue warp -> compute warps (+ TMA bytes)
  unsigned long long empty[kMaxStages];  // completer -> dequeue warp
  unsigned long long done[kMaxStages];   // compute warps -> completer
  unsigned long long prod_alive;   // %globaltimer stamp of the dequeue warp
  unsigned long long full_wait_ns; // compute warps' bound on a silent dequeue warp
  unsigned long long wait_limit_ns; // bound of the CTA's other waits (launch copy of HostCtl)
  unsigned int exit_flag;
  unsigned int armed;              // uses staged so far by the dequeue warp (low 32 bits)
  StageMeta meta[kMaxStages];
  WorkItem dcache[2][8];           // descriptors of the current / next chunk (ticket & 7)
  ProdCold cold;
  // the layout record last copied from the ring: every tile of a request shares its layout,
  // so later tiles copy it from here instead of over PCIe (key: the item's aux, which holds
  // the layout's unmasked ring sequence number)
  Layout lay_cache;
  uint32_t lay_key;
  uint32_t lay_valid;
};

// Compute threads per worker CTA at most (plus the dequeue and completer warps): 512 threads
// leave each thread 128 registers.
constexpr int kMaxComputeThreads = 448;
constexpr uint32_t kStageBytesDefault = 32768 + 128;  // two 16 KB operand halves + slack
constexpr uint32_t kHalfBytes = 16384;                // one operand tile
// EW_2D geometry: transpose-mode blocks are 16 rows x 256 columns (a float [16][256] tile
// per transposed operand fills one stage half); row-mode blocks hold about 8192 elements.
constexpr int64_t k2dBlockRows = 16, k2dBlockCols = 256, k2dRowTile = 8192;
// EW_2DT: rows per block at most (every row in one block) and elements per block at most (the
// float transpose buffer is one stage half)
constexpr int64_t k2dtMaxRows = 256, k2dtElems = 4096;
// Top-k on the batched path: k rounds of a warp-wide selection per row, so k is bounded.
constexpr int kTopkMaxK = 256;

// ---- fixed device scratch of gpuos_ew_batch_noalloc ----------------------------------
// One statically sized block per device holds everything a one-shot worker launch needs
// besides the caller's operands: control words, the completion ticket, strided layouts
// and the tile descriptors.  Offsets are bytes from the start of the block.
constexpr size_t round_up256(size_t x) { return (x + 255) & ~size_t(255); }
struct StaticScratch {
  static constexpr uint64_t kMaxItems = GPUOS_NOALLOC_MAX_TILES;     // power of two
  static constexpr uint32_t kMaxLayouts = GPUOS_NOALLOC_MAX_STRIDED;  // power of two
  static constexpr size_t kHostCtl = 0;
  static constexpr size_t kReport = 128;
  static constexpr size_t kDevCtl = 256;
  static constexpr size_t kTickets = round_up256(kDevCtl + sizeof(DevCtl));
  static constexpr size_t kLayouts = kTickets + 256;  // tickets of batch slots 0..7
  // ticket slot 7 (never used: every call is flush 1) holds the sticky error word, which the
  // per-call image copy leaves alone
  static constexpr size_t kSticky = kTickets + 7 * 32;
  static constexpr size_t kItems = round_up256(kLayouts + kMaxLayouts * sizeof(Layout));
  static constexpr size_t kBytes = kItems + kMaxItems * sizeof(WorkItem);
};
static_assert((StaticScratch::kMaxItems & (StaticScratch::kMaxItems - 1)) == 0, "tile capacity: power of two");
static_assert((StaticScratch::kMaxLayouts & (StaticScratch::kMaxLayouts - 1)) == 0, "layout capacity: power of two");

GPUOS_HD inline int dtype_size(int dt) {
  return dt == kF32 ? 4 : (dt == kF16 || dt == kBF16) ? 2 : dt == kF64 ? 8 : 4;
}

// Number of tensor inputs an element-wise op reads (1 or 2).
GPUOS_HD inline int ew_arity(int op) {
  switch (op) {
    case GPUOS_EW_ADD: case GPUOS_EW_MUL: case GPUOS_EW_SUB: case GPUOS_EW_DIV:
    case GPUOS_EW_MAXIMUM: case GPUOS_EW_MINIMUM: case GPUOS_EW_POW:
    case GPUOS_EW_ADD_ALPHA: case GPUOS_EW_SUB_ALPHA:
      return 2;
    default:
      return 1;
  }
}

}  // namespace gpuos
