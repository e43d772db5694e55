// runtime.cpp — host runtime of the persistent micro-op worker (C ABI: gpuos_rt_*).
//
// Reference: pytorch_ext/gpuos_ext.cpp.  The reference keeps one global queue on device 0,
// appends 496-byte Tasks to a vector, and at flush copies them to the device with a
// blocking cudaMemcpy, hashes them (FNV-1a over the whole array), enqueues 512-request
// shards with ~3 CUDA calls each and waits until a global completion count reaches
// "before + shards" (gpuos_ext.cpp:675-811).  This runtime:
//   * keeps one instance per device (queue, control blocks, worker);
//   * plans each request into 64-byte work items as it is submitted, written straight
//     into a ring in mapped pinned memory, so a flush is a single store of the tail
//     (no CUDA call unless the worker has to be (re)launched);
//   * orders dependent requests inside and across flushes with segment barriers
//     derived from the byte ranges the requests read and write;
//   * tracks completion per flush with a ticket the device writes, so sync flushes wait
//     for exactly their own work;
//   * never calls exit(): every failure is a status code plus a message.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "internal.h"
#include "jit.h"

using namespace gpuos;

extern "C" cudaError_t gpuos_internal_launch_batch_worker(const WorkerParams* p, int blocks, int threads,
                                                          size_t smem, cudaStream_t s);
extern "C" cudaError_t gpuos_internal_set_worker_smem(size_t smem);
extern "C" cudaError_t gpuos_internal_table_ptrs(void** table, void** alias);
extern "C" cudaError_t gpuos_internal_preload_kernels();
extern "C" cudaError_t gpuos_internal_worker_occupancy(int threads, size_t smem, int* blocks);
extern "C" cudaError_t gpuos_internal_module_addrs(unsigned long long* d_out, cudaStream_t s);
namespace gpuos {
int expr_compile(const char* expr, int arity, ExprProg* out, std::string* err);
}
extern "C" size_t gpuos_internal_smem_header_bytes();

// ---- errors -----------------------------------------------------------------------------
static thread_local std::string t_last_error;

static int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

#define CK(expr)                                                                              \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess)                                                                    \
      return fail(GPUOS_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__); \
  } while (0)

extern "C" const char* gpuos_rt_last_error(void) { return t_last_error.c_str(); }

static uint64_t mono_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

static inline void cpu_relax() {
#if defined(__x86_64__)
  __builtin_ia32_pause();
#else
  std::this_thread::yield();
#endif
}

static uint64_t pow2_at_least(uint64_t v) {
  uint64_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

static int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  return std::atoi(v);
}

// =========================================================================================
// Planner (no CUDA calls)
// =========================================================================================
namespace {

struct Dims {
  int nd = 0;
  int64_t size[GPUOS_MAX_NDIM];
  int64_t st[3][GPUOS_MAX_NDIM];
};

struct Range {
  uint64_t lo = 0, hi = 0;
  bool empty() const { return hi <= lo; }
};

bool dtype_ok(int dt) { return dt == kF32 || dt == kF16 || dt == kBF16; }

Range operand_range(const void* data, int dtype, int ndim, const int64_t* sizes, const int64_t* strides) {
  Range r;
  int64_t lo = 0, hi = 0;
  for (int d = 0; d < ndim; ++d) {
    if (sizes[d] == 0) return r;
    const int64_t ext = (sizes[d] - 1) * strides[d];
    if (ext < 0) lo += ext;
    else hi += ext;
  }
  const int es = dtype_size(dtype);
  r.lo = (uint64_t)((int64_t)(uintptr_t)data + lo * es);
  r.hi = (uint64_t)((int64_t)(uintptr_t)data + (hi + 1) * es);
  return r;
}

Range operand_range(const GpuosOperand& t) { return operand_range(t.data, t.dtype, t.ndim, t.sizes, t.strides); }

int64_t numel_of(int ndim, const int64_t* sizes) {
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) n *= sizes[d];
  return n;
}

// Right-aligned broadcast of `in` against the output dims (gpuos_ext.cpp:260-278).
bool align_operand(const GpuosOperand& in, const GpuosOperand& out, int64_t* st, std::string* err) {
  const int nd = out.ndim;
  if (in.ndim > nd) {
    for (int d = 0; d < in.ndim - nd; ++d)
      if (in.sizes[d] != 1) {
        *err = "operand has more dimensions than the output";
        return false;
      }
  }
  for (int d = 0; d < nd; ++d) {
    const int id = in.ndim - nd + d;
    if (id < 0) {
      st[d] = 0;
      continue;
    }
    if (in.sizes[id] == out.sizes[d]) {
      st[d] = out.sizes[d] == 1 ? 0 : in.strides[id];
    } else if (in.sizes[id] == 1) {
      st[d] = 0;
    } else {
      *err = "operand shape does not broadcast to the output shape";
      return false;
    }
  }
  return true;
}

void coalesce(Dims* d, int nops) {
  Dims r;
  r.nd = 0;
  for (int i = 0; i < d->nd; ++i) {
    if (d->size[i] == 1) continue;
    r.size[r.nd] = d->size[i];
    for (int k = 0; k < nops; ++k) r.st[k][r.nd] = d->st[k][i];
    ++r.nd;
  }
  // merge right to left
  Dims m;
  m.nd = 0;
  for (int i = 0; i < r.nd; ++i) {
    if (m.nd > 0) {
      bool ok = true;
      // previous (outer) dim m.nd-1 merges with inner dim i when outer stride == inner stride * inner size
      for (int k = 0; k < nops; ++k)
        if (m.st[k][m.nd - 1] != r.st[k][i] * r.size[i]) ok = false;
      if (ok) {
        m.size[m.nd - 1] *= r.size[i];
        for (int k = 0; k < nops; ++k) m.st[k][m.nd - 1] = r.st[k][i];
        continue;
      }
    }
    m.size[m.nd] = r.size[i];
    for (int k = 0; k < nops; ++k) m.st[k][m.nd] = r.st[k][i];
    ++m.nd;
  }
  *d = m;
}

struct EwReq {
  int op;
  const GpuosOperand* a;
  const GpuosOperand* b;  // tensor operand or null
  bool b_imm;
  float b_val;
  const GpuosOperand* out;
  float params[4];
};

struct Plan {
  std::vector<WorkItem> items;
  bool has_layout = false;
  Layout layout;
  Range reads[2];
  int nreads = 0;
  Range write;
  Range write2;  // a second output (top-k indices), empty otherwise
};

constexpr uint32_t kGenericTile = 8192;

// Elements per contiguous tile.  A tile is staged as the 16-byte-aligned span around its
// bytes, so an operand that starts off a 16-byte boundary gets tiles 32 bytes shorter than
// the stage half (a multiple of 16 bytes, so every tile keeps the operand's misalignment).
static uint32_t stage_tile(uint32_t half_bytes, int es, bool misaligned) {
  return (misaligned ? half_bytes - 32 : half_bytes) / (uint32_t)es;
}

// Row-major dense (every size > 1 dim has the contiguous stride).
static bool dense(const GpuosOperand& t) {
  int64_t expect = 1;
  for (int d = t.ndim - 1; d >= 0; --d) {
    if (t.sizes[d] != 1 && t.strides[d] != expect) return false;
    expect *= t.sizes[d];
  }
  return true;
}

static bool same_shape(const GpuosOperand& x, const GpuosOperand& y) {
  if (x.ndim != y.ndim) return false;
  for (int d = 0; d < x.ndim; ++d)
    if (x.sizes[d] != y.sizes[d]) return false;
  return true;
}

int plan_ew(const EwReq& r, uint32_t half_bytes, Plan* p) {
  if (r.op < 0 || r.op >= GPUOS_EW_NUM_OPS) return fail(GPUOS_ERR_INVALID, "unknown element-wise op %d", r.op);
  const GpuosOperand& out = *r.out;
  if (!r.a || !dtype_ok(r.a->dtype) || !dtype_ok(out.dtype))
    return fail(GPUOS_ERR_INVALID, "unsupported dtype (only float32, float16 and bfloat16 are computed)");
  const bool binary = ew_arity(r.op) == 2;
  if (binary && !r.b && !r.b_imm) return fail(GPUOS_ERR_INVALID, "binary op without a second operand");
  const GpuosOperand* b = binary ? r.b : nullptr;
  if (b && !dtype_ok(b->dtype)) return fail(GPUOS_ERR_INVALID, "unsupported dtype for the second operand");
  if (out.ndim < 0 || out.ndim > GPUOS_MAX_NDIM || r.a->ndim < 0 || r.a->ndim > GPUOS_MAX_NDIM ||
      (b && (b->ndim < 0 || b->ndim > GPUOS_MAX_NDIM)))
    return fail(GPUOS_ERR_INVALID, "at most %d dimensions are supported", GPUOS_MAX_NDIM);
  for (int d = 0; d < out.ndim; ++d)
    if (out.sizes[d] < 0 || out.strides[d] < 0) return fail(GPUOS_ERR_INVALID, "negative size or stride");
  const int64_t n = numel_of(out.ndim, out.sizes);
  p->items.clear();
  p->has_layout = false;
  p->nreads = 0;
  if (n == 0) return GPUOS_OK;
  if (!out.data || !r.a->data || (b && !b->data)) return fail(GPUOS_ERR_INVALID, "null data pointer");

  const int esa = dtype_size(r.a->dtype), eso = dtype_size(out.dtype);
  const int esb = b ? dtype_size(b->dtype) : 4;
  uint8_t base_flags = 0;
  if (binary) base_flags |= IF_B_PRESENT;
  if (binary && r.b_imm && !b) base_flags |= IF_B_SCALAR;
  uint32_t bimm_u;
  std::memcpy(&bimm_u, &r.b_val, 4);
  const uint64_t bimm_bits = bimm_u;
  WorkItem proto;
  std::memset(&proto, 0, sizeof(proto));
  proto.op = (uint8_t)r.op;
  proto.dt_a = (uint8_t)r.a->dtype;
  proto.dt_b = (uint8_t)(b ? b->dtype : kF32);
  proto.dt_o = (uint8_t)out.dtype;
  proto.aux = 0xffffffffu;

  // Fast path: operands of the output's shape, all dense (the common case): one 1-D
  // contiguous run, no broadcast, no dimension bookkeeping.
  if (same_shape(*r.a, out) && dense(*r.a) && dense(out) && (!b || (same_shape(*b, out) && dense(*b)))) {
    const int es_max = std::max(esa, b ? esb : 1);
    const bool misaligned = (((uintptr_t)r.a->data | (b ? (uintptr_t)b->data : 0)) & 15) != 0;
    const uint32_t tile = stage_tile(half_bytes, es_max, misaligned);
    uint32_t p0u, p1u;
    std::memcpy(&p0u, &r.params[0], 4);
    std::memcpy(&p1u, &r.params[1], 4);
    proto.kind = IK_EW_CONTIG;
    proto.x = (uint64_t)p0u | ((uint64_t)p1u << 32);
    proto.flags = base_flags;
    const uint64_t A = (uint64_t)(uintptr_t)r.a->data, O = (uint64_t)(uintptr_t)out.data;
    const uint64_t B = b ? (uint64_t)(uintptr_t)b->data : (r.b_imm ? bimm_bits : 0);
    p->reads[p->nreads++] = Range{A, A + (uint64_t)n * esa};
    if (b) p->reads[p->nreads++] = Range{B, B + (uint64_t)n * esb};
    p->write = Range{O, O + (uint64_t)n * eso};
    for (int64_t s = 0; s < n; s += tile) {
      WorkItem it = proto;
      it.count = (uint32_t)std::min<int64_t>(tile, n - s);
      it.a = A + (uint64_t)s * esa;
      it.b = b ? B + (uint64_t)s * esb : B;
      it.o = O + (uint64_t)s * eso;
      p->items.push_back(it);
    }
    return GPUOS_OK;
  }

  std::string err;
  Dims d;
  d.nd = out.ndim;
  for (int i = 0; i < out.ndim; ++i) {
    d.size[i] = out.sizes[i];
    d.st[2][i] = out.sizes[i] == 1 ? 0 : out.strides[i];
  }
  if (!align_operand(*r.a, out, d.st[0], &err)) return fail(GPUOS_ERR_INVALID, "%s", err.c_str());
  if (b) {
    if (!align_operand(*b, out, d.st[1], &err)) return fail(GPUOS_ERR_INVALID, "%s", err.c_str());
  } else {
    for (int i = 0; i < out.ndim; ++i) d.st[1][i] = 0;
  }
  // output must not overlap itself (a broadcast output cannot be written element-wise)
  for (int i = 0; i < out.ndim; ++i)
    if (out.sizes[i] > 1 && out.strides[i] == 0) return fail(GPUOS_ERR_INVALID, "output has a zero stride");
  coalesce(&d, 3);
  if (d.nd == 0) {
    d.nd = 1;
    d.size[0] = 1;
    d.st[0][0] = 0;
    d.st[1][0] = 0;
    d.st[2][0] = 1;
  }
  p->reads[p->nreads++] = operand_range(*r.a);
  if (b) p->reads[p->nreads++] = operand_range(*b);
  p->write = operand_range(out);

  const bool contig = d.nd == 1 && d.st[2][0] == 1 && (d.st[0][0] == 1 || d.st[0][0] == 0) &&
                      (!b || d.st[1][0] == 1 || d.st[1][0] == 0);
  if (contig) {
    const bool a_vec = d.st[0][0] == 1;
    const bool b_vec = b && d.st[1][0] == 1;
    int es_max = 1;
    if (a_vec) es_max = std::max(es_max, esa);
    if (b_vec) es_max = std::max(es_max, esb);
    if (!a_vec && !b_vec) es_max = 4;
    const bool misaligned =
        (((a_vec ? (uintptr_t)r.a->data : 0) | (b_vec ? (uintptr_t)b->data : 0)) & 15) != 0;
    const uint32_t tile = stage_tile(half_bytes, es_max, misaligned);
    uint32_t p0u, p1u;
    std::memcpy(&p0u, &r.params[0], 4);
    std::memcpy(&p1u, &r.params[1], 4);
    proto.kind = IK_EW_CONTIG;
    proto.x = (uint64_t)p0u | ((uint64_t)p1u << 32);
    proto.flags = base_flags | (a_vec ? 0 : IF_A_BCAST) | ((b && !b_vec) ? IF_B_BCAST : 0);
    const uint64_t A = (uint64_t)(uintptr_t)r.a->data, B = b ? (uint64_t)(uintptr_t)b->data : bimm_bits,
                   O = (uint64_t)(uintptr_t)out.data;
    for (int64_t s = 0; s < n; s += tile) {
      WorkItem it = proto;
      it.count = (uint32_t)std::min<int64_t>(tile, n - s);
      it.a = A + (a_vec ? (uint64_t)s * esa : 0);
      it.b = b ? (B + (b_vec ? (uint64_t)s * esb : 0)) : (r.b_imm ? bimm_bits : 0);
      it.o = O + (uint64_t)s * eso;
      p->items.push_back(it);
    }
    return GPUOS_OK;
  }
  // strided / broadcast layouts of at most two dims: row x column blocks (EW_2D).  Element
  // offsets of every operand stay below 2^31 (the device computes them in 32 bits).
  auto extent_ok = [&]() {
    for (int k = 0; k < 3; ++k) {
      int64_t e = 0;
      for (int i = 0; i < d.nd; ++i) e += (d.size[i] - 1) * std::llabs(d.st[k][i]);
      if (e >= (int64_t(1) << 31)) return false;
    }
    return true;
  };
  if (d.nd <= 2 && n < (int64_t(1) << 31) && extent_ok()) {
    int64_t R = 1, C = d.size[0], st[3][2];
    for (int k = 0; k < 3; ++k) {
      st[k][0] = d.nd == 2 ? d.st[k][0] : 0;
      st[k][1] = d.nd == 2 ? d.st[k][1] : d.st[k][0];
    }
    if (d.nd == 2) {
      R = d.size[0];
      C = d.size[1];
    }
    // walk the output in its memory order: its smaller stride is the column dimension
    if (R > 1 && st[2][0] < st[2][1]) {
      std::swap(R, C);
      for (int k = 0; k < 3; ++k) std::swap(st[k][0], st[k][1]);
    }
    // an input that runs contiguously along rows (a transposed view) is read through shared memory
    auto along_rows = [&](int k) {
      return R > 1 && st[k][0] != 0 && st[k][1] != 0 && std::llabs(st[k][0]) < std::llabs(st[k][1]);
    };
    const bool at = along_rows(0), bt = b && along_rows(1);
    p->has_layout = true;
    Layout& L = p->layout;
    std::memset(&L, 0, sizeof(L));
    L.ndim = 2;
    L.sizes[0] = R;
    L.sizes[1] = C;
    L.sa[0] = st[0][0];
    L.sa[1] = st[0][1];
    L.sb[0] = st[1][0];
    L.sb[1] = st[1][1];
    L.so[0] = st[2][0];
    L.so[1] = st[2][1];
    for (int i = 0; i < 4; ++i) L.params[i] = r.params[i];
    proto.kind = IK_EW_2D;
    proto.flags = base_flags | (at ? IF_A_T : 0) | (bt ? IF_B_T : 0);
    proto.a = (uint64_t)(uintptr_t)r.a->data;
    proto.b = b ? (uint64_t)(uintptr_t)b->data : (r.b_imm ? bimm_bits : 0);
    proto.o = (uint64_t)(uintptr_t)out.data;
    auto block = [&](int64_t r0, int64_t c0, int64_t nr, int64_t nc) {
      WorkItem it = proto;
      it.x = (uint64_t)r0 | ((uint64_t)c0 << 32);
      it.count = (uint32_t)((nr << 16) | nc);
      p->items.push_back(it);
    };
    // a runs along rows with unit stride and every row fits one block: a block of all rows x a
    // power-of-two column range is one contiguous span of a (plus the column stride's gaps),
    // staged by one bulk copy and transposed in shared memory (at most k2dtElems elements, so the
    // float transpose buffer fills one stage half)
    if (at && !bt && st[0][0] == 1 && st[0][1] >= R && R <= k2dtMaxRows) {
      const int64_t esa = dtype_size(r.a->dtype);
      auto span = [&](int lg) { return (((int64_t(1) << lg) - 1) * st[0][1] + R) * esa; };
      int lg = 0;
      while ((int64_t(2) << lg) * R <= k2dtElems) ++lg;
      while (lg > 3 && span(lg) + 32 > (int64_t)half_bytes) --lg;
      if (lg >= 3 && span(lg) + 32 <= (int64_t)half_bytes) {  // at least 8 columns per block
        proto.kind = IK_EW_2DT;
        proto.flags = base_flags;
        const int64_t w = int64_t(1) << lg;
        for (int64_t c0 = 0; c0 < C; c0 += w) {
          WorkItem it = proto;
          it.x = (uint64_t)lg | ((uint64_t)c0 << 32);
          it.count = (uint32_t)((R << 16) | std::min<int64_t>(w, C - c0));
          p->items.push_back(it);
        }
        return GPUOS_OK;
      }
    }
    if (at || bt) {
      for (int64_t r0 = 0; r0 < R; r0 += k2dBlockRows)
        for (int64_t c0 = 0; c0 < C; c0 += k2dBlockCols)
          block(r0, c0, std::min<int64_t>(k2dBlockRows, R - r0), std::min<int64_t>(k2dBlockCols, C - c0));
    } else if (C >= k2dRowTile) {
      for (int64_t r0 = 0; r0 < R; ++r0)
        for (int64_t c0 = 0; c0 < C; c0 += k2dRowTile) block(r0, c0, 1, std::min<int64_t>(k2dRowTile, C - c0));
    } else {
      const int64_t rows = std::max<int64_t>(1, k2dRowTile / C);
      for (int64_t r0 = 0; r0 < R; r0 += rows) block(r0, 0, std::min<int64_t>(rows, R - r0), C);
    }
    return GPUOS_OK;
  }
  // strided / broadcast of more dims: layout record shared by the request's tiles
  p->has_layout = true;
  Layout& L = p->layout;
  std::memset(&L, 0, sizeof(L));
  L.ndim = d.nd;
  for (int i = 0; i < d.nd; ++i) {
    L.sizes[i] = d.size[i];
    L.sa[i] = d.st[0][i];
    L.sb[i] = d.st[1][i];
    L.so[i] = d.st[2][i];
  }
  for (int i = 0; i < 4; ++i) L.params[i] = r.params[i];
  proto.kind = IK_EW_GENERIC;
  proto.flags = base_flags;
  for (int64_t s = 0; s < n; s += kGenericTile) {
    WorkItem it = proto;
    it.count = (uint32_t)std::min<int64_t>(kGenericTile, n - s);
    it.a = (uint64_t)(uintptr_t)r.a->data;
    it.b = b ? (uint64_t)(uintptr_t)b->data : (r.b_imm ? bimm_bits : 0);
    it.o = (uint64_t)(uintptr_t)out.data;
    it.x = (uint64_t)s;
    p->items.push_back(it);
  }
  return GPUOS_OK;
}

int plan_reduce(int rop, const GpuosOperand& x, const GpuosOperand& out, const int* axes, int naxes, int keepdim,
                uint32_t stage_bytes, Plan* p) {
  if (rop != GPUOS_RED_SUM && rop != GPUOS_RED_MEAN) return fail(GPUOS_ERR_INVALID, "unknown reduction %d", rop);
  if (!dtype_ok(x.dtype) || !dtype_ok(out.dtype))
    return fail(GPUOS_ERR_INVALID, "unsupported dtype (only float32, float16 and bfloat16 are computed)");
  if (x.ndim < 0 || x.ndim > GPUOS_MAX_NDIM || out.ndim < 0 || out.ndim > GPUOS_MAX_NDIM)
    return fail(GPUOS_ERR_INVALID, "at most %d dimensions are supported", GPUOS_MAX_NDIM);
  bool red[GPUOS_MAX_NDIM] = {false};
  if (naxes == 0) {
    for (int d = 0; d < x.ndim; ++d) red[d] = true;
  }
  for (int i = 0; i < naxes; ++i) {
    int a = axes[i];
    if (a < 0) a += x.ndim;
    if (a < 0 || a >= x.ndim) return fail(GPUOS_ERR_INVALID, "reduction axis %d out of range", axes[i]);
    if (red[a]) return fail(GPUOS_ERR_INVALID, "duplicate reduction axis %d", axes[i]);
    red[a] = true;
  }
  // expected output shape
  int64_t exp_sizes[GPUOS_MAX_NDIM];
  int exp_nd = 0;
  for (int d = 0; d < x.ndim; ++d) {
    if (red[d]) {
      if (keepdim) exp_sizes[exp_nd++] = 1;
    } else {
      exp_sizes[exp_nd++] = x.sizes[d];
    }
  }
  if (exp_nd != out.ndim) return fail(GPUOS_ERR_INVALID, "output rank %d does not match reduction result rank %d", out.ndim, exp_nd);
  for (int d = 0; d < exp_nd; ++d)
    if (exp_sizes[d] != out.sizes[d]) return fail(GPUOS_ERR_INVALID, "output shape does not match the reduction result");
  p->items.clear();
  p->has_layout = false;
  p->nreads = 0;
  const int64_t nout = numel_of(out.ndim, out.sizes);
  if (nout == 0) return GPUOS_OK;
  if (!out.data || (!x.data && numel_of(x.ndim, x.sizes) != 0)) return fail(GPUOS_ERR_INVALID, "null data pointer");

  Dims kept, rd;
  kept.nd = 0;
  rd.nd = 0;
  int od = 0;
  for (int d = 0; d < x.ndim; ++d) {
    if (red[d]) {
      rd.size[rd.nd] = x.sizes[d];
      rd.st[0][rd.nd] = x.strides[d];
      ++rd.nd;
      if (keepdim) ++od;
    } else {
      kept.size[kept.nd] = x.sizes[d];
      kept.st[0][kept.nd] = x.strides[d];
      kept.st[1][kept.nd] = out.strides[od];
      ++kept.nd;
      ++od;
    }
  }
  coalesce(&kept, 2);
  coalesce(&rd, 1);
  int64_t rtotal = 1;
  for (int i = 0; i < rd.nd; ++i) rtotal *= rd.size[i];
  p->reads[p->nreads++] = operand_range(x);
  p->write = operand_range(out);
  const int es = dtype_size(x.dtype);

  WorkItem proto;
  std::memset(&proto, 0, sizeof(proto));
  proto.op = (uint8_t)rop;
  proto.dt_a = (uint8_t)x.dtype;
  proto.dt_o = (uint8_t)out.dtype;
  proto.flags = rop == GPUOS_RED_MEAN ? IF_MEAN : 0;
  proto.aux = 0xffffffffu;

  // Row case: one reduced dim, at most one kept dim with a contiguous output, and rows that
  // do not interleave.
  if (rd.nd == 1 && kept.nd <= 1 && (kept.nd == 0 || kept.st[1][0] == 1)) {
    const int64_t C = rd.size[0], is = rd.st[0][0];
    const int64_t rows = kept.nd ? kept.size[0] : 1;
    const int64_t rs = kept.nd ? kept.st[0][0] : 0;
    if (C > 0 && is >= 1 && (rows == 1 || C * is <= rs) && C <= 0x7fffffff) {
      const int64_t row_span = ((C - 1) * is + 1) * es;
      int64_t rows_per;
      uint8_t fl = proto.flags;
      const bool gaps = rows > 1 && rs * es > 2 * row_span;
      if (row_span + 32 <= (int64_t)stage_bytes && !gaps) {
        rows_per = rows > 1 ? 1 + ((int64_t)stage_bytes - 32 - row_span) / (rs * es) : 1;
      } else {
        fl |= IF_UNSTAGED;
        rows_per = std::max<int64_t>(1, 16384 / C);
      }
      rows_per = std::max<int64_t>(1, std::min<int64_t>(rows_per, 1 << 16));
      proto.kind = IK_ROW_REDUCE;
      proto.flags = fl;
      proto.aux = (uint32_t)C;
      const int eso = dtype_size(out.dtype);
      for (int64_t r0 = 0; r0 < rows; r0 += rows_per) {
        WorkItem it = proto;
        it.count = (uint32_t)std::min<int64_t>(rows_per, rows - r0);
        it.a = (uint64_t)(uintptr_t)x.data + (uint64_t)(r0 * rs * es);
        it.o = (uint64_t)(uintptr_t)out.data + (uint64_t)(r0 * eso);
        it.x = (uint64_t)rs;
        it.b = (uint64_t)is;
        p->items.push_back(it);
      }
      return GPUOS_OK;
    }
  }
  p->has_layout = true;
  Layout& L = p->layout;
  std::memset(&L, 0, sizeof(L));
  L.ndim = kept.nd;
  for (int i = 0; i < kept.nd; ++i) {
    L.sizes[i] = kept.size[i];
    L.sa[i] = kept.st[0][i];
    L.so[i] = kept.st[1][i];
  }
  L.rdim = rd.nd;
  for (int i = 0; i < rd.nd; ++i) {
    L.rsizes[i] = rd.size[i];
    L.rsa[i] = rd.st[0][i];
  }
  L.rtotal = rtotal;
  proto.kind = IK_RED_GENERIC;
  const int64_t per = std::max<int64_t>(1, std::min<int64_t>(8192, 262144 / std::max<int64_t>(rtotal, 1)));
  for (int64_t s = 0; s < nout; s += per) {
    WorkItem it = proto;
    it.count = (uint32_t)std::min<int64_t>(per, nout - s);
    it.a = (uint64_t)(uintptr_t)x.data;
    it.o = (uint64_t)(uintptr_t)out.data;
    it.x = (uint64_t)s;
    p->items.push_back(it);
  }
  return GPUOS_OK;
}

// ---- hazard tracking --------------------------------------------------------------------
// Byte ranges read and written by the requests of the current segment, bucketed by
// 64 KiB block.  A request that reads a range written in the segment, or writes a range
// read or written in the segment, starts a new segment whose items wait for every
// earlier item (WorkItem::wait_items).
class HazardMap {
 public:
  HazardMap() : table_(1 << 16) {}

  void clear() {
    ++gen_;
    pool_.clear();
    large_.clear();
    pending_.clear();
    rbox_ = wbox_ = Range();
  }
  size_t size() const { return pool_.size() + large_.size() + pending_.size(); }

  // true if r (read when !write) conflicts with the segment.  The bounding boxes of the
  // segment's reads and writes answer most queries; the ranges are hashed into 64 KiB
  // buckets only once a query falls inside a box.
  bool conflicts(const Range& r, bool write) {
    if (r.empty()) return false;
    const bool in_w = box_overlap(wbox_, r), in_r = write && box_overlap(rbox_, r);
    if (!in_w && !in_r) return false;
    index_pending();
    for (const Ent& e : large_)
      if ((write || e.write) && overlap(e, r)) return true;
    const uint64_t b0 = r.lo >> kShift, b1 = (r.hi - 1) >> kShift;
    if (b1 - b0 > kMaxBlocks) {
      // scan everything for a huge range
      for (const Ent& e : pool_)
        if ((write || e.write) && overlap(e, r)) return true;
      return false;
    }
    for (uint64_t blk = b0; blk <= b1; ++blk) {
      const Slot* s = find(blk);
      if (!s) continue;
      for (int32_t i = s->head; i >= 0; i = pool_[i].next)
        if ((write || pool_[i].write) && overlap(pool_[i], r)) return true;
    }
    return false;
  }

  void insert(const Range& r, bool write) {
    if (r.empty()) return;
    Range& box = write ? wbox_ : rbox_;
    if (box.empty()) {
      box = r;
    } else {
      box.lo = std::min(box.lo, r.lo);
      box.hi = std::max(box.hi, r.hi);
    }
    pending_.push_back(Ent{r.lo, r.hi, write, -1});
  }

 private:
  void index_pending() {
    for (const Ent& e : pending_) index(Range{e.lo, e.hi}, e.write);
    pending_.clear();
  }
  static bool box_overlap(const Range& box, const Range& r) { return !box.empty() && box.lo < r.hi && r.lo < box.hi; }

  // A range already among the last entries of a block's chain (a write covers a read of the same
  // range) is not added again: a tensor read by many requests of a segment would otherwise grow
  // its blocks' chains by one entry per request, and every later query in those blocks would
  // scan them (quadratic in the segment's requests).
  bool recent(int32_t i, const Range& r, bool write) const {
    for (int k = 0; i >= 0 && k < 8; ++k, i = pool_[i].next)
      if (pool_[i].lo == r.lo && pool_[i].hi == r.hi && (pool_[i].write || !write)) return true;
    return false;
  }

  void index(const Range& r, bool write) {
    const uint64_t b0 = r.lo >> kShift, b1 = (r.hi - 1) >> kShift;
    if (b1 - b0 > kMaxBlocks) {
      for (size_t k = large_.size(), n = 0; k > 0 && n < 8; --k, ++n) {
        const Ent& e = large_[k - 1];
        if (e.lo == r.lo && e.hi == r.hi && (e.write || !write)) return;
      }
      large_.push_back(Ent{r.lo, r.hi, write, -1});
      return;
    }
    for (uint64_t blk = b0; blk <= b1; ++blk) {
      Slot* s = find_or_add(blk);
      if (recent(s->head, r, write)) continue;
      pool_.push_back(Ent{r.lo, r.hi, write, s->head});
      s->head = (int32_t)pool_.size() - 1;
    }
  }

  static constexpr int kShift = 16;
  static constexpr uint64_t kMaxBlocks = 64;
  struct Ent {
    uint64_t lo, hi;
    bool write;
    int32_t next;
  };
  struct Slot {
    uint64_t key = 0;
    uint32_t gen = 0;
    int32_t head = -1;
  };
  static bool overlap(const Ent& e, const Range& r) { return e.lo < r.hi && r.lo < e.hi; }
  static uint64_t hash(uint64_t k) {
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdull;
    k ^= k >> 33;
    return k;
  }
  const Slot* find(uint64_t key) const {
    const size_t mask = table_.size() - 1;
    for (size_t i = hash(key) & mask;; i = (i + 1) & mask) {
      const Slot& s = table_[i];
      if (s.gen != gen_) return nullptr;
      if (s.key == key) return &s;
    }
  }
  Slot* find_or_add(uint64_t key) {
    if (used_gen_ != gen_) {
      used_ = 0;
      used_gen_ = gen_;
    }
    if (used_ * 2 >= table_.size()) grow();
    const size_t mask = table_.size() - 1;
    for (size_t i = hash(key) & mask;; i = (i + 1) & mask) {
      Slot& s = table_[i];
      if (s.gen != gen_) {
        s.gen = gen_;
        s.key = key;
        s.head = -1;
        ++used_;
        return &s;
      }
      if (s.key == key) return &s;
    }
  }
  void grow() {
    std::vector<Slot> old;
    old.swap(table_);
    table_.assign(old.size() * 2, Slot());
    const size_t mask = table_.size() - 1;
    for (const Slot& s : old) {
      if (s.gen != gen_) continue;
      for (size_t i = hash(s.key) & mask;; i = (i + 1) & mask)
        if (table_[i].gen != gen_) {
          table_[i] = s;
          break;
        }
    }
  }
  std::vector<Slot> table_;
  std::vector<Ent> pool_;
  std::vector<Ent> large_;
  std::vector<Ent> pending_;  // inserted since the last query that needed the index
  Range rbox_, wbox_;         // bounding boxes of the segment's reads and writes
  uint32_t gen_ = 1;
  uint32_t used_gen_ = 0;
  size_t used_ = 0;
};

}  // namespace

// =========================================================================================
// Runtime
// =========================================================================================
struct BatchInfo {
  uint64_t seq;
  uint64_t first_item, n_items;
  uint64_t n_reqs;
  uint64_t task_end, layout_end;
  bool done;
};

struct gpuos_rt {
  int device = 0;
  int capacity = 0;
  int tpb = 0;
  int sm_count = 0;
  uint32_t stages = 4;
  uint32_t stage_bytes = kStageBytesDefault;
  size_t smem = 0;
  cudaStream_t kstream = nullptr, cstream = nullptr;
  // CUDA events around worker launches (gpuos_rt_set_launch_timing): pairs in launch order
  bool time_launches = false;
  std::deque<std::pair<cudaEvent_t, cudaEvent_t>> launch_events;
  std::vector<cudaEvent_t> spare_events;

  // mapped pinned block
  void* host_block = nullptr;
  HostCtl* hc = nullptr;
  DevReport* rep = nullptr;
  SyncState* sync = nullptr;
  Ticket* tickets = nullptr;
  WorkItem* items = nullptr;
  Task* tasks = nullptr;
  Layout* layouts = nullptr;
  uint64_t item_cap = 0, task_cap = 0, layout_cap = 0;
  DevCtl* dc = nullptr;
  // this runtime's op table and alias (device memory; the worker resolves Tasks through them at
  // dequeue time).  The reference C ABI's table (launch_persistent_worker) stays separate: it
  // only ever holds addresses of this library's module.
  void* op_table = nullptr;  // OpPtrInt[GPUOS_MAX_OPS], followed by int alias[GPUOS_MAX_OPS]
  void* op_alias = nullptr;

  std::mutex mu;
  // producer cursors
  uint64_t item_w = 0;    // next item index to write
  uint64_t item_pub = 0;  // items published (tail)
  uint64_t task_w = 0, layout_w = 0;
  uint64_t pend_reqs = 0;
  uint64_t seg_wait = 0;  // wait_items of new items
  HazardMap hz;
  // batches
  uint64_t last_seq = 0;
  std::deque<BatchInfo> inflight;
  uint64_t completed_seq = 0;  // every seq <= completed_seq done
  uint64_t processed = 0;      // completed requests
  uint64_t submitted = 0;      // submitted requests
  uint64_t oldest_item = 0, oldest_task = 0, oldest_layout = 0;
  // worker
  uint64_t epoch = 0;
  bool launched = false;
  int idle_quiesce_ms = 200;
  uint64_t last_activity_ns = 0;
  bool failed = false;
  std::string fail_msg;
  // keeper
  std::thread keeper;
  std::atomic<bool> stop{false};
  int next_slot = 20;
  int next_expr = 0;  // expression programs installed on this device
  // Worker module: this library's until an operator compiled at run time is installed, then
  // the module that links the worker with every such operator (jit_mod.worker != nullptr).
  jit::Module jit_mod;
  std::vector<jit::Module> old_mods;  // earlier linked modules, kept loaded until shutdown
  std::vector<jit::Op> jit_ops;       // operators of the current linked module, in install order
  std::vector<uint64_t> addr_map;     // current module: MA_COUNT built-in addresses, then one per jit op
  std::vector<uint64_t> static_map;   // this library's module
  std::vector<ExprProg> expr_progs;   // host copies of the installed expression programs
  unsigned long long* addr_dev = nullptr;  // device output of the address kernels
  std::mutex jit_mu;                  // one operator install at a time
  int ctas_per_sm = 1;  // worker CTAs resident per SM (each with its own dequeue warp)
  int grid = 0;         // worker CTAs per launch
  int cta_threads = 0;  // compute threads per worker CTA
  int verbose = 0;
};

// Stages of the worker's ring: as many as shared memory holds (GPUOS_STAGES caps it), 2 to
// kMaxStages.  Every staged item keeps its operand loads in flight, so more stages keep more
// bytes in flight per SM.
static uint32_t pick_stages(size_t smem_cap, size_t stage_bytes) {
  const int want = std::max(2, std::min(kMaxStages, env_int("GPUOS_STAGES", kMaxStages)));
  uint32_t S = (uint32_t)want;
  while (S > 2 && gpuos_internal_smem_header_bytes() + S * stage_bytes > smem_cap) --S;
  return S;
}

static std::mutex g_rt_mu;
static std::map<int, gpuos_rt*> g_rts;

extern "C" gpuos_rt* gpuos_rt_get(int device) {
  std::lock_guard<std::mutex> lk(g_rt_mu);
  auto it = g_rts.find(device);
  return it == g_rts.end() ? nullptr : it->second;
}

// ---- completion reaping -------------------------------------------------------------------
static void reap_locked(gpuos_rt* rt) {
  for (BatchInfo& b : rt->inflight) {
    if (!b.done) {
      const Ticket& tk = rt->tickets[b.seq % kNumBatchSlots];
      if (tk.seq == (uint32_t)b.seq) b.done = true;
    }
  }
  while (!rt->inflight.empty() && rt->inflight.front().done) {
    const BatchInfo& b = rt->inflight.front();
    rt->completed_seq = b.seq;
    rt->processed += b.n_reqs;
    rt->oldest_item = b.first_item + b.n_items;
    rt->oldest_task = b.task_end;
    rt->oldest_layout = b.layout_end;
    rt->inflight.pop_front();
  }
  if (rt->inflight.empty()) {
    rt->oldest_item = rt->item_pub;
    if (rt->pend_reqs == 0 && rt->item_w == rt->item_pub) {
      // nothing outstanding: every earlier range is complete
      rt->hz.clear();
      rt->oldest_task = rt->task_w;
      rt->oldest_layout = rt->layout_w;
    }
  }
  if (rt->sync) rt->sync->processed = rt->processed;
}

static int check_device_error_locked(gpuos_rt* rt) {
  const uint64_t e = rt->rep->error;
  if (e == 0) return GPUOS_OK;
  static const char* names[] = {"none",
                                "dequeue warp: stage release wait expired",
                                "compute warps: stage fill wait expired",
                                "dependency barrier wait expired",
                                "exit coordination wait expired",
                                "start coordination wait expired",
                                "malformed work item",
                                "task dispatched to an empty op-table slot",
                                "host heartbeat lost",
                                "completer: compute warps did not finish a stage in time"};
  const uint32_t code = (uint32_t)(e >> 32);
  rt->failed = true;
  // how long the expired wait lasted against which bound (device memory, read on this error path)
  unsigned long long ew = 0;
  if (cudaSetDevice(rt->device) == cudaSuccess)
    cudaMemcpy(&ew, &rt->dc->err_wait, sizeof(ew), cudaMemcpyDeviceToHost);
  char buf[320];
  snprintf(buf, sizeof(buf), "worker error: %s (block %u, item %llu%s%llu us of a %llu ms bound)",
           code < 10 ? names[code] : "unknown", (unsigned)(e & 0xffffffffu), (unsigned long long)rt->rep->error_item,
           ew ? "; waited " : "; ", ew >> 32, ew & 0xffffffffull);
  rt->fail_msg = buf;
  return fail(GPUOS_ERR_DEVICE, "%s", buf);
}

// ---- worker launch --------------------------------------------------------------------------
static int launch_worker_locked(gpuos_rt* rt) {
  const uint64_t ep = ++rt->epoch;
  if (rt->idle_quiesce_ms == 0) rt->hc->quit_epoch = ep;  // drain mode: exit once drained
  WorkerParams P;
  std::memset(&P, 0, sizeof(P));
  P.hc = rt->hc;
  P.rep = rt->rep;
  P.tickets = rt->tickets;
  P.items = rt->items;
  P.tasks = rt->tasks;
  P.layouts = rt->layouts;
  P.dc = rt->dc;
  P.op_table = reinterpret_cast<OpFn*>(rt->op_table);
  P.op_alias = reinterpret_cast<int*>(rt->op_alias);
  P.item_mask = rt->item_cap - 1;
  P.task_mask = (uint32_t)(rt->task_cap - 1);
  P.layout_mask = (uint32_t)(rt->layout_cap - 1);
  P.epoch = ep;
  P.stages = rt->stages;
  P.stage_bytes = rt->stage_bytes;
  P.compute_threads = (uint32_t)rt->cta_threads;
  // while more work is staged, completions are accounted 32 at a time (each account is a
  // gpu-scope fence that waits for the tiles' stores); operands are read once, so their bulk
  // loads carry an L2 evict-first policy.  Measured on 8 steps of 4096 fp32 tiles per launch:
  // 0.333 ms -> 0.299 ms per launch.
  P.account_every = (uint32_t)std::max(1, env_int("GPUOS_ACCOUNT_EVERY", 32));
  P.load_hint = (uint32_t)env_int("GPUOS_LOAD_HINT", 1);
  P.wait_limit_ns = rt->hc->wait_limit_ns;
  CK(cudaSetDevice(rt->device));
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  if (rt->time_launches) {
    for (cudaEvent_t* ev : {&ev0, &ev1}) {
      if (!rt->spare_events.empty()) {
        *ev = rt->spare_events.back();
        rt->spare_events.pop_back();
      } else {
        CK(cudaEventCreate(ev));
      }
    }
    CK(cudaEventRecord(ev0, rt->kstream));
  }
  // one dequeue warp + one completer warp + threads_per_block compute threads
  if (rt->jit_mod.worker) {
    void* args[] = {&P};
    std::string err;
    const int st = jit::launch(rt->jit_mod.worker, (unsigned)rt->grid, (unsigned)(rt->cta_threads + 64), rt->smem,
                               rt->kstream, args, &err);
    if (st) return fail(st, "worker launch: %s", err.c_str());
  } else {
    CK(gpuos_internal_launch_batch_worker(&P, rt->grid, rt->cta_threads + 64, rt->smem, rt->kstream));
  }
  if (rt->time_launches) {
    CK(cudaEventRecord(ev1, rt->kstream));
    rt->launch_events.emplace_back(ev0, ev1);
  }
  rt->launched = true;
  return GPUOS_OK;
}

// Make sure a worker will process the published tail (after the tail store + fence).
static int ensure_worker_locked(gpuos_rt* rt) {
  if (!rt->launched) return launch_worker_locked(rt);
  const uint64_t st = rt->rep->state;
  const uint64_t ep = st >> 8, code = st & 0xff;
  if (ep == rt->epoch && (code == WS_EXITING || code == WS_EXITED)) return launch_worker_locked(rt);
  if (ep < rt->epoch) return GPUOS_OK;  // current launch queued behind the previous one
  return GPUOS_OK;
}

// Publish pending items as one flush.  *seq_out = its ticket (0 if nothing was pending).
static int publish_locked(gpuos_rt* rt, uint64_t* seq_out) {
  if (seq_out) *seq_out = 0;
  if (rt->failed) return fail(GPUOS_ERR_DEVICE, "%s", rt->fail_msg.c_str());
  const uint64_t n = rt->item_w - rt->item_pub;
  if (n == 0 && rt->pend_reqs == 0) return GPUOS_OK;
  const uint64_t seq = ++rt->last_seq;
  // the ticket slot of seq - kNumBatchSlots must be free
  if (!rt->inflight.empty() && rt->inflight.front().seq + kNumBatchSlots <= seq) {
    const uint64_t t0 = mono_ns();
    while (!rt->inflight.empty() && rt->inflight.front().seq + kNumBatchSlots <= seq) {
      reap_locked(rt);
      int e = check_device_error_locked(rt);
      if (e) return e;
      if (mono_ns() - t0 > 30ull * 1000 * 1000 * 1000) return fail(GPUOS_ERR_TIMEOUT, "ticket ring full");
      cpu_relax();
    }
  }
  const uint16_t slot = (uint16_t)(seq % kNumBatchSlots);
  for (uint64_t i = rt->item_pub; i < rt->item_w; ++i) {
    WorkItem& it = rt->items[i & (rt->item_cap - 1)];
    it.batch = slot;
    it.batch_items = (uint32_t)n;
    it.batch_seq = (uint32_t)seq;
  }
  BatchInfo b;
  b.seq = seq;
  b.first_item = rt->item_pub;
  b.n_items = n;
  b.n_reqs = rt->pend_reqs;
  b.task_end = rt->task_w;
  b.layout_end = rt->layout_w;
  b.done = (n == 0);
  rt->inflight.push_back(b);
  rt->submitted += rt->pend_reqs;
  rt->pend_reqs = 0;
  rt->last_activity_ns = mono_ns();
  if (seq_out) *seq_out = seq;
  if (n == 0) {
    reap_locked(rt);
    return GPUOS_OK;
  }
  if (rt->idle_quiesce_ms != 0 && rt->hc->quit_epoch >= rt->epoch && rt->epoch > 0) {
    rt->hc->quit_epoch = rt->epoch - 1;  // withdraw an idle-quiesce request
  }
  std::atomic_thread_fence(std::memory_order_seq_cst);
  rt->hc->tail = rt->item_w;
  rt->item_pub = rt->item_w;
  std::atomic_thread_fence(std::memory_order_seq_cst);
  if (rt->sync) rt->sync->submitted = rt->submitted;
  return ensure_worker_locked(rt);
}

// Make room for `items` more items (and tasks/layouts) in the rings.
static int reserve_locked(gpuos_rt* rt, uint64_t items, uint64_t tasks, uint64_t layouts) {
  if (items > rt->item_cap / 2 || tasks > rt->task_cap / 2 || layouts > rt->layout_cap / 2)
    return fail(GPUOS_ERR_INVALID, "request too large for the ring (%llu items)", (unsigned long long)items);
  const uint64_t t0 = mono_ns();
  bool published = false;
  while (true) {
    reap_locked(rt);
    const bool ok = rt->item_w + items - rt->oldest_item <= rt->item_cap &&
                    rt->task_w + tasks - rt->oldest_task <= rt->task_cap &&
                    rt->layout_w + layouts - rt->oldest_layout <= rt->layout_cap;
    if (ok) return GPUOS_OK;
    if (!published) {
      // pending requests occupy the ring: publish them so the worker can drain
      int e = publish_locked(rt, nullptr);
      if (e) return e;
      published = true;
    }
    int e = check_device_error_locked(rt);
    if (e) return e;
    if (mono_ns() - t0 > 30ull * 1000 * 1000 * 1000) return fail(GPUOS_ERR_TIMEOUT, "ring full: worker not draining");
    std::this_thread::yield();
  }
}

// Append a planned request.
static int append_plan_locked(gpuos_rt* rt, const Plan& p, const Task* task) {
  if (rt->failed) return fail(GPUOS_ERR_DEVICE, "%s", rt->fail_msg.c_str());
  const uint64_t nitems = p.items.size();
  int e = reserve_locked(rt, nitems, task ? 1 : 0, p.has_layout ? 1 : 0);
  if (e) return e;
  // hazards against the current segment
  bool hazard = false;
  for (int i = 0; i < p.nreads && !hazard; ++i) hazard = rt->hz.conflicts(p.reads[i], false);
  if (!hazard) hazard = rt->hz.conflicts(p.write, true);
  if (!hazard) hazard = rt->hz.conflicts(p.write2, true);
  if (hazard || rt->hz.size() > (1u << 20)) {
    rt->hz.clear();
    rt->seg_wait = rt->item_w;
  }
  for (int i = 0; i < p.nreads; ++i) rt->hz.insert(p.reads[i], false);
  rt->hz.insert(p.write, true);
  rt->hz.insert(p.write2, true);

  // items carry the layout's unmasked sequence number (the worker masks it to a ring slot and
  // uses the full value as the key of its cached copy, so a reused slot never looks cached)
  uint32_t layout_idx = 0, task_idx = 0;
  if (p.has_layout) {
    rt->layouts[rt->layout_w & (rt->layout_cap - 1)] = p.layout;
    layout_idx = (uint32_t)rt->layout_w;
    ++rt->layout_w;
  }
  if (task) {
    task_idx = (uint32_t)(rt->task_w & (rt->task_cap - 1));
    std::memcpy(&rt->tasks[task_idx], task, sizeof(Task));
    ++rt->task_w;
  }
  const uint64_t mask = rt->item_cap - 1;
  for (uint64_t i = 0; i < nitems; ++i) {
    WorkItem it = p.items[i];
    it.wait_items = rt->seg_wait;
    if (p.has_layout) it.aux = layout_idx;
    if (task) it.aux = task_idx;
    rt->items[(rt->item_w + i) & mask] = it;
  }
  rt->item_w += nitems;
  rt->pend_reqs += 1;
  return GPUOS_OK;
}

// ---- keeper thread: host heartbeat, completion reaping, idle quiesce ------------------------
static void keeper_main(gpuos_rt* rt) {
  while (!rt->stop.load(std::memory_order_relaxed)) {
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
    std::lock_guard<std::mutex> lk(rt->mu);
    rt->hc->host_beat = rt->hc->host_beat + 1;
    reap_locked(rt);
    // idle: nothing published is in flight (requests not yet flushed do not need the worker,
    // and their flush relaunches it), so kernels on other streams get the SMs back
    if (rt->launched && rt->idle_quiesce_ms > 0 && rt->inflight.empty() && rt->hc->quit_epoch < rt->epoch &&
        mono_ns() - rt->last_activity_ns > (uint64_t)rt->idle_quiesce_ms * 1000000ull) {
      rt->hc->quit_epoch = rt->epoch;
    }
  }
}

// =========================================================================================
// C ABI
// =========================================================================================
extern "C" int gpuos_rt_init(int device, int capacity, int threads_per_block, gpuos_rt** out) {
  if (out) *out = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_rt_mu);
    auto it = g_rts.find(device);
    if (it != g_rts.end()) {  // gpuos_ext.cpp:450: init is idempotent
      if (out) *out = it->second;
      return GPUOS_OK;
    }
  }
  if (capacity <= 0) capacity = 4096;
  if (threads_per_block <= 0) threads_per_block = 256;
  if (threads_per_block % 32 != 0 || threads_per_block < 64 || threads_per_block > kMaxComputeThreads)
    return fail(GPUOS_ERR_INVALID, "threads_per_block must be a multiple of 32 in [64, %d]", kMaxComputeThreads);
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(GPUOS_ERR_INVALID, "device %d out of range (%d devices)", device, ndev);
  CK(cudaSetDevice(device));
  CK(cudaFree(0));
  gpuos_rt* rt = new gpuos_rt();
  rt->device = device;
  rt->capacity = capacity;
  rt->tpb = threads_per_block;
  rt->verbose = env_int("GPUOS_VERBOSE", 0);
  rt->idle_quiesce_ms = env_int("GPUOS_IDLE_QUIESCE_MS", 200);
  auto cleanup = [&](int code) {
    if (rt->host_block) cudaFreeHost(rt->host_block);
    if (rt->dc) cudaFree(rt->dc);
    if (rt->addr_dev) cudaFree(rt->addr_dev);
    if (rt->op_table) cudaFree(rt->op_table);
    if (rt->kstream) cudaStreamDestroy(rt->kstream);
    if (rt->cstream) cudaStreamDestroy(rt->cstream);
    delete rt;
    return code;
  };
  cudaError_t e = cudaDeviceGetAttribute(&rt->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return cleanup(fail(GPUOS_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e)));
  int smem_optin = 0, smem_sm = 0, smem_reserved = 0;
  cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device);
  cudaDeviceGetAttribute(&smem_reserved, cudaDevAttrReservedSharedMemoryPerBlock, device);
  // Worker CTAs per SM (GPUOS_CTAS_PER_SM, 1 or 2): with 2, each CTA gets half of the compute
  // threads and half of the shared memory, and every SM runs two dequeue warps.
  rt->ctas_per_sm = std::max(1, std::min(2, env_int("GPUOS_CTAS_PER_SM", 1)));
  if (rt->ctas_per_sm == 2 && (threads_per_block / 2) % 32 != 0) rt->ctas_per_sm = 1;
  rt->cta_threads = threads_per_block / rt->ctas_per_sm;
  rt->grid = rt->sm_count * rt->ctas_per_sm;
  if (rt->grid >= kDiagCtas) return cleanup(fail(GPUOS_ERR_UNSUPPORTED, "%d worker CTAs exceed %d", rt->grid, kDiagCtas - 1));
  const size_t smem_cap = std::min<size_t>((size_t)smem_optin, (size_t)smem_sm / rt->ctas_per_sm - smem_reserved);
  rt->stages = pick_stages(smem_cap, rt->stage_bytes);
  rt->smem = gpuos_internal_smem_header_bytes() + (size_t)rt->stages * rt->stage_bytes;
  if (rt->smem > smem_cap) return cleanup(fail(GPUOS_ERR_UNSUPPORTED, "worker needs %zu bytes of shared memory", rt->smem));
  rt->item_cap = pow2_at_least(std::max<uint64_t>((uint64_t)capacity * 8, 1u << 16));
  rt->task_cap = pow2_at_least(std::max<uint64_t>((uint64_t)capacity, 1024));
  rt->layout_cap = pow2_at_least(std::max<uint64_t>((uint64_t)capacity, 1024));
  const size_t off_hc = 0, off_rep = 128, off_sync = 256, off_tk = 512;
  const size_t off_items = off_tk + sizeof(Ticket) * kNumBatchSlots;
  const size_t off_tasks = off_items + sizeof(WorkItem) * rt->item_cap;
  const size_t off_lay = off_tasks + ((sizeof(Task) * rt->task_cap + 127) & ~size_t(127));
  const size_t total = off_lay + sizeof(Layout) * rt->layout_cap;
  e = cudaHostAlloc(&rt->host_block, total, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) return cleanup(fail(GPUOS_ERR_CUDA, "cudaHostAlloc(%zu): %s", total, cudaGetErrorString(e)));
  std::memset(rt->host_block, 0, total);
  void* dev_block = nullptr;
  e = cudaHostGetDevicePointer(&dev_block, rt->host_block, 0);
  if (e != cudaSuccess || dev_block != rt->host_block)
    return cleanup(fail(GPUOS_ERR_CUDA, "mapped memory needs unified addressing (%s)", cudaGetErrorString(e)));
  unsigned char* hb = static_cast<unsigned char*>(rt->host_block);
  rt->hc = reinterpret_cast<HostCtl*>(hb + off_hc);
  rt->rep = reinterpret_cast<DevReport*>(hb + off_rep);
  rt->sync = reinterpret_cast<SyncState*>(hb + off_sync);
  rt->tickets = reinterpret_cast<Ticket*>(hb + off_tk);
  rt->items = reinterpret_cast<WorkItem*>(hb + off_items);
  rt->tasks = reinterpret_cast<Task*>(hb + off_tasks);
  rt->layouts = reinterpret_cast<Layout*>(hb + off_lay);
  rt->hc->safety_idle_ns = (uint64_t)env_int("GPUOS_SAFETY_IDLE_MS", 10000) * 1000000ull;
  rt->hc->spin_ns = (uint32_t)env_int("GPUOS_SPIN_NS", 32);
  rt->hc->wait_limit_ns = (uint64_t)env_int("GPUOS_DEVICE_WAIT_MS", 5000) * 1000000ull;
  rt->hc->debug_level = (uint32_t)env_int("GPUOS_DEBUG", 0);

  e = cudaMalloc(&rt->dc, sizeof(DevCtl));
  if (e == cudaSuccess) e = cudaMemset(rt->dc, 0, sizeof(DevCtl));
  if (e == cudaSuccess) e = cudaMemset(rt->dc->batch_t0, 0xff, sizeof(rt->dc->batch_t0));
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&rt->kstream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&rt->cstream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = launch_init_builtin_ops(rt->cstream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->cstream);
  // built-in operator addresses of this library's module
  if (e == cudaSuccess) e = cudaMalloc(&rt->addr_dev, sizeof(unsigned long long) * (MA_COUNT + kMaxJitOps));
  if (e == cudaSuccess) e = gpuos_internal_module_addrs(rt->addr_dev, rt->cstream);
  rt->static_map.assign(MA_COUNT, 0);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(rt->static_map.data(), rt->addr_dev, sizeof(uint64_t) * MA_COUNT, cudaMemcpyDeviceToHost,
                        rt->cstream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->cstream);
  rt->addr_map = rt->static_map;
  // the runtime's table as launch_init_builtin_ops sets the reference one
  // (persistent_kernel.cu:115-130): empty slots, identity alias, add@0, mul@1, batch@10
  static thread_local OpPtrInt init_table[GPUOS_MAX_OPS];
  static thread_local int init_alias[GPUOS_MAX_OPS];
  for (int i = 0; i < GPUOS_MAX_OPS; ++i) {
    init_table[i] = 0;
    init_alias[i] = i;
  }
  init_table[0] = rt->static_map[MA_ADD];
  init_table[1] = rt->static_map[MA_MUL];
  init_table[10] = rt->static_map[MA_BATCH];
  if (e == cudaSuccess) e = cudaMalloc(&rt->op_table, sizeof(init_table) + sizeof(init_alias));
  if (e == cudaSuccess) {
    rt->op_alias = static_cast<unsigned char*>(rt->op_table) + sizeof(init_table);
    e = cudaMemcpyAsync(rt->op_table, init_table, sizeof(init_table), cudaMemcpyHostToDevice, rt->cstream);
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(rt->op_alias, init_alias, sizeof(init_alias), cudaMemcpyHostToDevice, rt->cstream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->cstream);
  rt->expr_progs.assign(kExprPrograms, ExprProg());
  if (e == cudaSuccess) e = gpuos_internal_set_worker_smem(rt->smem);
  if (e == cudaSuccess) e = gpuos_internal_preload_kernels();
  int resident = 0;
  if (e == cudaSuccess) e = gpuos_internal_worker_occupancy(rt->cta_threads + 64, rt->smem, &resident);
  if (e != cudaSuccess) return cleanup(fail(GPUOS_ERR_CUDA, "runtime setup: %s", cudaGetErrorString(e)));
  // every worker CTA must be resident at once (the grid coordinates its exit)
  if (resident < rt->ctas_per_sm)
    return cleanup(fail(GPUOS_ERR_UNSUPPORTED, "%d worker CTAs per SM requested, %d fit", rt->ctas_per_sm, resident));
  rt->last_activity_ns = mono_ns();
  {
    std::lock_guard<std::mutex> lk(rt->mu);
    int st = launch_worker_locked(rt);
    if (st) return cleanup(st);
  }
  // wait for the worker to come up (gpuos_ext.cpp:495-511: 1 s cap, then proceed)
  const uint64_t t0 = mono_ns();
  while (rt->rep->ready_epoch < rt->epoch && mono_ns() - t0 < 2000ull * 1000 * 1000) std::this_thread::yield();
  rt->keeper = std::thread(keeper_main, rt);
  {
    std::lock_guard<std::mutex> lk(g_rt_mu);
    g_rts[device] = rt;
  }
  if (out) *out = rt;
  return GPUOS_OK;
}

static int wait_seq_locked(gpuos_rt* rt, std::unique_lock<std::mutex>& lk, uint64_t seq, int timeout_ms);

extern "C" int gpuos_rt_shutdown(gpuos_rt* rt) {
  if (!rt) return GPUOS_OK;
  {
    std::lock_guard<std::mutex> lk(g_rt_mu);
    auto it = g_rts.find(rt->device);
    if (it == g_rts.end() || it->second != rt) return fail(GPUOS_ERR_NOT_INIT, "runtime not registered");
    g_rts.erase(it);
  }
  rt->stop.store(true);
  if (rt->keeper.joinable()) rt->keeper.join();
  int status = GPUOS_OK;
  cudaSetDevice(rt->device);
  {
    std::unique_lock<std::mutex> lk(rt->mu);
    if (!rt->failed) {
      uint64_t seq = 0;
      status = publish_locked(rt, &seq);
      if (!status && rt->last_seq) status = wait_seq_locked(rt, lk, rt->last_seq, 30000);
    }
    rt->hc->quit_epoch = rt->epoch;
  }
  // The worker exits once drained; a bounded wait before the stream sync.
  const uint64_t t0 = mono_ns();
  while (rt->launched && mono_ns() - t0 < 20ull * 1000 * 1000 * 1000) {
    const uint64_t st = rt->rep->state;
    if ((st >> 8) == rt->epoch && (st & 0xff) == WS_EXITED) break;
    if (cudaStreamQuery(rt->kstream) != cudaErrorNotReady) break;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  cudaError_t e = cudaStreamSynchronize(rt->kstream);
  if (e != cudaSuccess && !status) status = fail(GPUOS_ERR_CUDA, "worker: %s", cudaGetErrorString(e));
  cudaStreamSynchronize(rt->cstream);
  for (auto& pr : rt->launch_events) {
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  for (cudaEvent_t ev : rt->spare_events) cudaEventDestroy(ev);
  cudaStreamDestroy(rt->kstream);
  cudaStreamDestroy(rt->cstream);
  jit::unload(&rt->jit_mod);
  for (jit::Module& m : rt->old_mods) jit::unload(&m);
  cudaFree(rt->addr_dev);
  cudaFree(rt->op_table);
  cudaFree(rt->dc);
  cudaFreeHost(rt->host_block);
  delete rt;
  return status;
}

extern "C" int gpuos_rt_submit_ew(gpuos_rt* rt, int op, const GpuosOperand* a, const GpuosOperand* b, int b_is_scalar,
                                  double b_scalar, const GpuosOperand* out, const float* params, int nparams) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (!a || !out) return fail(GPUOS_ERR_INVALID, "null operand");
  EwReq r;
  r.op = op;
  r.a = a;
  r.b = b_is_scalar ? nullptr : b;
  r.b_imm = b_is_scalar != 0;
  r.b_val = (float)b_scalar;
  r.out = out;
  for (int i = 0; i < 4; ++i) r.params[i] = (params && i < nparams) ? params[i] : 0.f;
  static thread_local Plan plan;
  int e = plan_ew(r, kHalfBytes, &plan);
  if (e) return e;
  std::lock_guard<std::mutex> lk(rt->mu);
  return append_plan_locked(rt, plan, nullptr);
}

// Several element-wise requests in one call: every request is planned (and validated) before
// any is appended, then all are appended under one acquisition of the runtime lock.
extern "C" int gpuos_rt_submit_ew_many(gpuos_rt* rt, int n, const int* ops, const GpuosOperand* a,
                                       const GpuosOperand* b, const GpuosOperand* out) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (n < 0) return fail(GPUOS_ERR_INVALID, "negative request count");
  if (n == 0) return GPUOS_OK;
  if (!ops || !a || !out) return fail(GPUOS_ERR_INVALID, "null operand array");
  static thread_local std::vector<Plan> plans;
  if ((int)plans.size() < n) plans.resize((size_t)n);
  for (int i = 0; i < n; ++i) {
    EwReq r;
    r.op = ops[i];
    r.a = &a[i];
    r.b = b ? &b[i] : nullptr;
    r.b_imm = false;
    r.b_val = 0.f;
    r.out = &out[i];
    for (int k = 0; k < 4; ++k) r.params[k] = 0.f;
    const int e = plan_ew(r, kHalfBytes, &plans[(size_t)i]);
    if (e) return e;
  }
  std::lock_guard<std::mutex> lk(rt->mu);
  for (int i = 0; i < n; ++i) {
    const int e = append_plan_locked(rt, plans[(size_t)i], nullptr);
    if (e) return e;
  }
  return GPUOS_OK;
}

extern "C" int gpuos_rt_submit_reduce(gpuos_rt* rt, int red_op, const GpuosOperand* x, const GpuosOperand* out,
                                      const int* axes, int naxes, int keepdim) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (!x || !out) return fail(GPUOS_ERR_INVALID, "null operand");
  static thread_local Plan plan;
  int e = plan_reduce(red_op, *x, *out, axes, naxes, keepdim, rt->stage_bytes, &plan);
  if (e) return e;
  std::lock_guard<std::mutex> lk(rt->mu);
  return append_plan_locked(rt, plan, nullptr);
}

// Top-k of every row of x [rows, n] (contiguous): values [rows, k] in x's dtype and int64
// indices [rows, k], both contiguous, largest or smallest first.  Rows are grouped so that a
// group fits one stage (a row longer than a stage is read from global memory).
extern "C" int gpuos_rt_submit_topk(gpuos_rt* rt, const void* x, int dtype, int64_t rows, int64_t n, void* values,
                                    int64_t* indices, int k, int largest) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (!dtype_ok(dtype)) return fail(GPUOS_ERR_INVALID, "unsupported dtype (only float32, float16 and bfloat16)");
  if (rows < 0 || n <= 0 || n >= (int64_t(1) << 31)) return fail(GPUOS_ERR_INVALID, "bad row count or row length");
  if (k < 1 || k > n || k > kTopkMaxK) return fail(GPUOS_ERR_INVALID, "k must be in [1, min(n, %d)]", kTopkMaxK);
  if (rows == 0) return GPUOS_OK;
  if (!x || !values || !indices) return fail(GPUOS_ERR_INVALID, "null data pointer");
  const int es = dtype_size(dtype);
  static thread_local Plan p;
  p.items.clear();
  p.has_layout = false;
  p.nreads = 0;
  WorkItem proto;
  std::memset(&proto, 0, sizeof(proto));
  proto.kind = IK_TOPK;
  proto.dt_a = proto.dt_o = (uint8_t)dtype;
  proto.dt_b = kF32;
  proto.aux = (uint32_t)n;
  proto.x = (uint64_t)(uint32_t)k | ((uint64_t)(largest ? 1 : 0) << 32);
  const int64_t row_bytes = n * es;
  const int64_t rows_per = std::min<int64_t>(4096, std::max<int64_t>(1, ((int64_t)rt->stage_bytes - 32) / row_bytes));
  const uint64_t X = (uint64_t)(uintptr_t)x, V = (uint64_t)(uintptr_t)values, I = (uint64_t)(uintptr_t)indices;
  for (int64_t r0 = 0; r0 < rows; r0 += rows_per) {
    WorkItem it = proto;
    it.count = (uint32_t)std::min<int64_t>(rows_per, rows - r0);
    it.a = X + (uint64_t)(r0 * row_bytes);
    it.o = V + (uint64_t)(r0 * k * es);
    it.b = I + (uint64_t)(r0 * k * 8);
    p.items.push_back(it);
  }
  p.reads[p.nreads++] = Range{X, X + (uint64_t)(rows * row_bytes)};
  p.write = Range{V, V + (uint64_t)(rows * k * es)};
  p.write2 = Range{I, I + (uint64_t)(rows * k * 8)};
  std::lock_guard<std::mutex> lk(rt->mu);
  return append_plan_locked(rt, p, nullptr);
}

static Range tensorref_range(const TensorRef& t) {
  if (!t.data) return Range();
  return operand_range(t.data, t.dtype, t.ndim, t.sizes, t.strides);
}

extern "C" int gpuos_rt_submit_task(gpuos_rt* rt, const Task* task) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (!task) return fail(GPUOS_ERR_INVALID, "null task");
  if (task->op < 0 || task->op >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_INVALID, "task op %d out of range", task->op);
  if (task->in0.ndim > GPUOS_MAX_NDIM || task->in1.ndim > GPUOS_MAX_NDIM || task->out0.ndim > GPUOS_MAX_NDIM)
    return fail(GPUOS_ERR_INVALID, "task rank above %d", GPUOS_MAX_NDIM);
  Plan p;
  WorkItem it;
  std::memset(&it, 0, sizeof(it));
  it.kind = IK_TASK;
  it.op = (uint8_t)task->op;
  p.items.push_back(it);
  p.reads[p.nreads++] = tensorref_range(task->in0);
  p.reads[p.nreads++] = tensorref_range(task->in1);
  p.write = tensorref_range(task->out0);
  std::lock_guard<std::mutex> lk(rt->mu);
  return append_plan_locked(rt, p, task);
}

static int wait_seq_locked(gpuos_rt* rt, std::unique_lock<std::mutex>& lk, uint64_t seq, int timeout_ms) {
  const uint64_t t0 = mono_ns();
  const uint64_t limit = (uint64_t)(timeout_ms < 0 ? 30000 : timeout_ms) * 1000000ull;
  uint32_t spins = 0;
  while (true) {
    // flushes may finish out of order; the wait ends once `seq` and every earlier flush are done
    reap_locked(rt);
    if (rt->completed_seq >= seq) return GPUOS_OK;
    int e = check_device_error_locked(rt);
    if (e) return e;
    if ((++spins & 1023u) == 0) {
      // a worker that exited (yield, idle) with work outstanding is relaunched
      const uint64_t st = rt->rep->state;
      if ((st >> 8) == rt->epoch && (st & 0xff) == WS_EXITED && rt->item_pub > rt->rep->exit_tail) {
        e = launch_worker_locked(rt);
        if (e) return e;
      }
    }
    const uint64_t el = mono_ns() - t0;
    if (el > limit) return fail(GPUOS_ERR_TIMEOUT, "timed out waiting for flush %llu", (unsigned long long)seq);
    if (spins < 4096) {
      cpu_relax();
    } else {
      lk.unlock();
      std::this_thread::sleep_for(std::chrono::microseconds(spins < 16384 ? 5 : 100));
      lk.lock();
    }
  }
}

extern "C" int gpuos_rt_flush(gpuos_rt* rt, int flags, cudaStream_t dep_stream, uint64_t* seq_out) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (seq_out) *seq_out = 0;
  const bool sync = (flags & GPUOS_FLUSH_SYNC) != 0;
  // Work already enqueued on dep_stream (e.g. the kernels that produced the inputs) must
  // finish before the worker reads the inputs.
  if (flags & GPUOS_FLUSH_DEP) {
    CK(cudaSetDevice(rt->device));
    cudaError_t q = cudaStreamQuery(dep_stream);
    if (q == cudaErrorNotReady) {
      const uint64_t t0 = mono_ns();
      bool asked = false;
      while ((q = cudaStreamQuery(dep_stream)) == cudaErrorNotReady) {
        if (!asked && mono_ns() - t0 > 50ull * 1000) {
          // The kernels on the caller's stream may need the SM resources the resident worker
          // holds (all of them at 448 compute threads): stop the worker (work already
          // published drains first); this flush's publish relaunches it.
          std::lock_guard<std::mutex> lk(rt->mu);
          if (rt->launched && rt->hc->quit_epoch < rt->epoch) rt->hc->quit_epoch = rt->epoch;
          asked = true;
        }
        if (mono_ns() - t0 > 30ull * 1000 * 1000 * 1000) return fail(GPUOS_ERR_TIMEOUT, "dependency stream did not drain");
        std::this_thread::yield();
      }
    }
    if (q != cudaSuccess) return fail(GPUOS_ERR_CUDA, "dependency stream: %s", cudaGetErrorString(q));
  }
  std::unique_lock<std::mutex> lk(rt->mu);
  uint64_t seq = 0;
  int e = publish_locked(rt, &seq);
  if (e) return e;
  if (seq_out) *seq_out = seq ? seq : rt->last_seq;
  if (sync) {
    const uint64_t target = rt->last_seq;  // this flush and everything before it
    if (target) return wait_seq_locked(rt, lk, target, 30000);
  }
  return GPUOS_OK;
}

extern "C" int gpuos_rt_wait(gpuos_rt* rt, uint64_t seq, int timeout_ms) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::unique_lock<std::mutex> lk(rt->mu);
  if (seq > rt->last_seq) return fail(GPUOS_ERR_INVALID, "flush %llu was never issued", (unsigned long long)seq);
  return wait_seq_locked(rt, lk, seq, timeout_ms);
}

extern "C" uint64_t gpuos_rt_completed(gpuos_rt* rt) {
  if (!rt) return 0;
  std::lock_guard<std::mutex> lk(rt->mu);
  reap_locked(rt);
  return rt->completed_seq;
}

extern "C" int gpuos_rt_flush_times(gpuos_rt* rt, uint64_t seq, uint64_t* t_start, uint64_t* t_end) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::lock_guard<std::mutex> lk(rt->mu);
  reap_locked(rt);
  const Ticket& tk = rt->tickets[seq % kNumBatchSlots];
  if (seq == 0 || seq > rt->last_seq || seq + kNumBatchSlots <= rt->last_seq || tk.seq != (uint32_t)seq)
    return fail(GPUOS_ERR_INVALID, "flush %llu not complete or recycled", (unsigned long long)seq);
  // the worker writes the stamps just after the ticket
  const uint64_t t0 = mono_ns();
  while (tk.tseq != (uint32_t)seq) {
    if (mono_ns() - t0 > 100ull * 1000 * 1000)
      return fail(GPUOS_ERR_TIMEOUT, "time stamps of flush %llu not written", (unsigned long long)seq);
    cpu_relax();
  }
  if (t_start) *t_start = tk.t_start;
  if (t_end) *t_end = tk.t_end;
  return GPUOS_OK;
}

extern "C" cudaStream_t gpuos_rt_kernel_stream(gpuos_rt* rt) { return rt ? rt->kstream : nullptr; }

extern "C" int gpuos_rt_set_launch_timing(gpuos_rt* rt, int on) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::lock_guard<std::mutex> lk(rt->mu);
  rt->time_launches = on != 0;
  return GPUOS_OK;
}

extern "C" int gpuos_rt_launch_times(gpuos_rt* rt, float* ms_out, int max) {
  if (!rt) return -fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::lock_guard<std::mutex> lk(rt->mu);
  int n = 0;
  while (!rt->launch_events.empty() && n < max) {
    auto pr = rt->launch_events.front();
    const cudaError_t q = cudaEventQuery(pr.second);
    if (q == cudaErrorNotReady) break;
    if (q != cudaSuccess) return -fail(GPUOS_ERR_CUDA, "launch timing: %s", cudaGetErrorString(q));
    float ms = 0.f;
    const cudaError_t e = cudaEventElapsedTime(&ms, pr.first, pr.second);
    if (e != cudaSuccess) return -fail(GPUOS_ERR_CUDA, "launch timing: %s", cudaGetErrorString(e));
    if (ms_out) ms_out[n] = ms;
    ++n;
    rt->launch_events.pop_front();
    rt->spare_events.push_back(pr.first);
    rt->spare_events.push_back(pr.second);
  }
  return n;
}

extern "C" uint64_t gpuos_rt_launches(gpuos_rt* rt) {
  if (!rt) return 0;
  std::lock_guard<std::mutex> lk(rt->mu);
  return rt->epoch;
}

extern "C" uint64_t gpuos_rt_poll_processed(gpuos_rt* rt) {
  if (!rt) return 0;
  std::lock_guard<std::mutex> lk(rt->mu);
  reap_locked(rt);
  return rt->processed;
}

extern "C" uint64_t gpuos_rt_poll_heartbeat(gpuos_rt* rt) { return rt ? rt->rep->heartbeat : 0; }

extern "C" int gpuos_rt_poll_ready(gpuos_rt* rt) {
  if (!rt) return 0;
  const uint64_t st = rt->rep->state;
  return (rt->rep->ready_epoch >= 1 && (st & 0xff) == WS_RUNNING) ? 1 : 0;
}

extern "C" int gpuos_rt_sync_wait(gpuos_rt* rt, uint64_t target, int timeout_ms) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::unique_lock<std::mutex> lk(rt->mu);
  const uint64_t t0 = mono_ns();
  const uint64_t limit = (uint64_t)(timeout_ms < 0 ? 30000 : timeout_ms) * 1000000ull;
  while (true) {
    reap_locked(rt);
    if (rt->processed >= target) return GPUOS_OK;
    int e = check_device_error_locked(rt);
    if (e) return e;
    if (mono_ns() - t0 > limit)
      return fail(GPUOS_ERR_TIMEOUT, "sync_wait: processed=%llu target=%llu", (unsigned long long)rt->processed,
                  (unsigned long long)target);
    lk.unlock();
    std::this_thread::sleep_for(std::chrono::microseconds(5));
    lk.lock();
  }
}

extern "C" int gpuos_rt_worker_alive(gpuos_rt* rt) {
  if (!rt || !rt->launched) return 0;
  return cudaStreamQuery(rt->kstream) == cudaErrorNotReady ? 1 : 0;
}

extern "C" int gpuos_rt_ensure_worker(gpuos_rt* rt) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::lock_guard<std::mutex> lk(rt->mu);
  if (rt->failed) return fail(GPUOS_ERR_DEVICE, "%s", rt->fail_msg.c_str());
  if (cudaStreamQuery(rt->kstream) == cudaSuccess) {
    if (rt->idle_quiesce_ms != 0 && rt->hc->quit_epoch >= rt->epoch) rt->hc->quit_epoch = rt->epoch;
    return launch_worker_locked(rt);
  }
  return GPUOS_OK;
}

extern "C" int gpuos_rt_quiesce(gpuos_rt* rt, int timeout_ms) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  uint64_t ep;
  {
    std::lock_guard<std::mutex> lk(rt->mu);
    if (!rt->launched) return GPUOS_OK;
    rt->hc->quit_epoch = rt->epoch;
    ep = rt->epoch;
  }
  const uint64_t t0 = mono_ns();
  const uint64_t limit = (uint64_t)(timeout_ms < 0 ? 30000 : timeout_ms) * 1000000ull;
  while (true) {
    const uint64_t st = rt->rep->state;
    if ((st >> 8) == ep && (st & 0xff) == WS_EXITED) break;
    if (rt->rep->error) {
      std::lock_guard<std::mutex> lk(rt->mu);
      return check_device_error_locked(rt);
    }
    if (mono_ns() - t0 > limit) return fail(GPUOS_ERR_TIMEOUT, "worker did not exit");
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  CK(cudaStreamSynchronize(rt->kstream));
  return GPUOS_OK;
}

extern "C" int gpuos_rt_set_debug_level(gpuos_rt* rt, int level) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  rt->hc->debug_level = (uint32_t)level;
  CK(cudaSetDevice(rt->device));
  CK(gpu_set_debug_level_async(level, rt->cstream));
  CK(cudaStreamSynchronize(rt->cstream));
  return GPUOS_OK;
}

extern "C" int gpuos_rt_set_yield_every(gpuos_rt* rt, uint64_t every) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  rt->hc->yield_every = every;
  return GPUOS_OK;
}

extern "C" int gpuos_rt_debug_counters(gpuos_rt* rt, uint64_t* out, int n) {
  if (!rt) return -fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  const int ctas = std::min(rt->grid, kDiagCtas);
  const int rows = std::min(ctas + 1, kDiagCtas);  // + the launch timeline row
  std::vector<unsigned long long> buf((size_t)rows * kDiagSlots);
  cudaError_t e = cudaSetDevice(rt->device);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(buf.data(), rt->dc->diag, buf.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                        rt->cstream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->cstream);
  if (e != cudaSuccess) return -fail(GPUOS_ERR_CUDA, "debug_counters: %s", cudaGetErrorString(e));
  const int m = std::min<int>(n, (int)buf.size());
  for (int i = 0; i < m; ++i) out[i] = buf[i];
  return ctas;
}

extern "C" int gpuos_rt_set_device_wait_ms(gpuos_rt* rt, int ms) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (ms <= 0) return fail(GPUOS_ERR_INVALID, "device wait bound must be positive");
  rt->hc->wait_limit_ns = (uint64_t)ms * 1000000ull;
  // a running worker keeps the bound it was launched with: stop it so the next launch
  // (on the next flush) takes the new one
  return gpuos_rt_quiesce(rt, 30000);
}

// Publish one item whose dependency barrier never opens: the dequeue warp's bounded wait
// expires, the worker records DE_WAIT_BARRIER and exits.  The item is never executed.
extern "C" int gpuos_rt_debug_inject_stall(gpuos_rt* rt) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::lock_guard<std::mutex> lk(rt->mu);
  int e = reserve_locked(rt, 1, 0, 0);
  if (e) return e;
  WorkItem it;
  std::memset(&it, 0, sizeof(it));
  it.kind = IK_EW_CONTIG;
  it.op = GPUOS_EW_COPY;
  it.count = 0;
  it.aux = 0xffffffffu;
  it.wait_items = ~0ull >> 1;
  rt->items[rt->item_w & (rt->item_cap - 1)] = it;
  rt->item_w += 1;
  rt->pend_reqs += 1;
  return publish_locked(rt, nullptr);
}

extern "C" int gpuos_rt_set_idle_quiesce_ms(gpuos_rt* rt, int ms) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::lock_guard<std::mutex> lk(rt->mu);
  rt->idle_quiesce_ms = ms < 0 ? -1 : ms;
  if (ms == 0) rt->hc->quit_epoch = rt->epoch;
  return GPUOS_OK;
}

extern "C" const char* gpuos_rt_stat_names(void) {
  return "head,tail,in_flight,capacity,processed,heartbeat,quit,host_tail_shadow,host_pending,"
         "item_capacity,sync_processed,sync_heartbeat,sync_ready,sync_submitted,epoch,state,error,items_done,"
         "completed_seq,last_seq,t_launch_ns,t_exit_ns,park_rounds,park_timeouts,park_work,host_read_ns_max,"
         "host_read_ns_avg,parked_seen";
}

extern "C" int gpuos_rt_stats(gpuos_rt* rt, int64_t* v, int n) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::lock_guard<std::mutex> lk(rt->mu);
  reap_locked(rt);
  int64_t vals[28];
  vals[0] = (int64_t)rt->rep->head_mirror;
  vals[1] = (int64_t)rt->item_pub;
  vals[2] = (int64_t)(rt->item_pub - std::min(rt->item_pub, (uint64_t)rt->rep->items_done));
  vals[3] = rt->capacity;
  vals[4] = (int64_t)rt->processed;
  vals[5] = (int64_t)rt->rep->heartbeat;
  vals[6] = rt->hc->quit_epoch >= rt->epoch ? 1 : 0;
  vals[7] = (int64_t)rt->item_pub;
  vals[8] = (int64_t)rt->pend_reqs;
  vals[9] = (int64_t)rt->item_cap;
  vals[10] = (int64_t)rt->processed;
  vals[11] = (int64_t)rt->rep->heartbeat;
  vals[12] = gpuos_rt_poll_ready(rt);
  vals[13] = (int64_t)rt->submitted;
  vals[14] = (int64_t)rt->epoch;
  vals[15] = (int64_t)(rt->rep->state & 0xff);
  vals[16] = (int64_t)rt->rep->error;
  vals[17] = (int64_t)rt->rep->items_done;
  vals[18] = (int64_t)rt->completed_seq;
  vals[19] = (int64_t)rt->last_seq;
  vals[20] = (int64_t)rt->rep->t_launch;
  vals[21] = (int64_t)rt->rep->t_exit;
  vals[22] = (int64_t)rt->rep->park_rounds;
  vals[23] = (int64_t)rt->rep->park_timeouts;
  vals[24] = (int64_t)rt->rep->park_work;
  vals[25] = (int64_t)rt->rep->host_read_ns_max;
  vals[26] = (int64_t)rt->rep->host_read_ns_avg;
  vals[27] = (int64_t)rt->rep->parked_seen;
  for (int i = 0; i < n && i < 28; ++i) v[i] = vals[i];
  return GPUOS_OK;
}

// ---- op table control --------------------------------------------------------------------
static uint64_t translate_addr(const std::vector<uint64_t>& from, const std::vector<uint64_t>& to, uint64_t a,
                               bool* found);

extern "C" int gpuos_rt_set_slot(gpuos_rt* rt, int slot, OpPtrInt fn) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (slot < 0 || slot >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_INVALID, "slot %d out of range", slot);
  {
    // once the worker runs from a linked module, an address of this library's module (from
    // gpu_get_builtin_op_async) names the same operator of the linked module
    std::lock_guard<std::mutex> lk(rt->mu);
    if (rt->jit_mod.worker) {
      bool found = false;
      fn = translate_addr(rt->static_map, rt->addr_map, fn, &found);
    }
  }
  CK(cudaSetDevice(rt->device));
  static thread_local OpPtrInt staged;
  staged = fn;
  CK(cudaMemcpyAsync(static_cast<OpPtrInt*>(rt->op_table) + slot, &staged, sizeof(OpPtrInt), cudaMemcpyHostToDevice,
                     rt->cstream));
  CK(cudaStreamSynchronize(rt->cstream));
  return GPUOS_OK;
}

extern "C" int gpuos_rt_get_slot(gpuos_rt* rt, int slot, OpPtrInt* fn) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (slot < 0 || slot >= GPUOS_MAX_OPS || !fn) return fail(GPUOS_ERR_INVALID, "slot %d out of range", slot);
  CK(cudaSetDevice(rt->device));
  CK(cudaMemcpyAsync(fn, static_cast<OpPtrInt*>(rt->op_table) + slot, sizeof(OpPtrInt), cudaMemcpyDeviceToHost,
                     rt->cstream));
  CK(cudaStreamSynchronize(rt->cstream));
  return GPUOS_OK;
}

extern "C" int gpuos_rt_set_alias(gpuos_rt* rt, int logical, int physical) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (logical < 0 || logical >= GPUOS_MAX_OPS || physical < 0 || physical >= GPUOS_MAX_OPS)
    return fail(GPUOS_ERR_INVALID, "alias %d -> %d out of range", logical, physical);
  CK(cudaSetDevice(rt->device));
  static thread_local int staged;
  staged = physical;
  CK(cudaMemcpyAsync(static_cast<int*>(rt->op_alias) + logical, &staged, sizeof(int), cudaMemcpyHostToDevice,
                     rt->cstream));
  CK(cudaStreamSynchronize(rt->cstream));
  return GPUOS_OK;
}

extern "C" int gpuos_rt_get_alias(gpuos_rt* rt, int logical, int* physical) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (logical < 0 || logical >= GPUOS_MAX_OPS || !physical) return fail(GPUOS_ERR_INVALID, "logical %d out of range", logical);
  CK(cudaSetDevice(rt->device));
  CK(cudaMemcpyAsync(physical, static_cast<int*>(rt->op_alias) + logical, sizeof(int), cudaMemcpyDeviceToHost,
                     rt->cstream));
  CK(cudaStreamSynchronize(rt->cstream));
  return GPUOS_OK;
}

// Address of built-in operator `code` in the worker module the runtime currently runs
// (codes as gpu_get_builtin_op_async: 0, 1, 10, 100+k, 200+k), 0 if there is none.
static uint64_t builtin_addr_locked(gpuos_rt* rt, int code) {
  int i = -1;
  if (code == 0) i = MA_ADD;
  else if (code == 1) i = MA_MUL;
  else if (code == 10) i = MA_BATCH;
  else if (code >= 100 && code < 100 + GPUOS_EW_NUM_OPS + 2) i = MA_REF_OPS + (code - 100);
  else if (code >= 200 && code < 200 + kExprPrograms) i = MA_EXPR_FNS + (code - 200);
  return i < 0 ? 0 : rt->addr_map[i];
}

// An address of this library's module (or of an earlier linked module) names the same operator
// in the current module; anything else is kept as written.
static uint64_t translate_addr(const std::vector<uint64_t>& from, const std::vector<uint64_t>& to, uint64_t a,
                               bool* found) {
  if (a == 0) return 0;
  for (size_t i = 0; i < from.size() && i < to.size(); ++i) {
    if (i == (size_t)MA_EXPR_PROGS) continue;
    if (from[i] == a) {
      *found = true;
      return to[i];
    }
  }
  return a;
}

extern "C" int gpuos_rt_builtin_op(gpuos_rt* rt, int code, OpPtrInt* addr) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (!addr) return fail(GPUOS_ERR_INVALID, "null output");
  std::lock_guard<std::mutex> lk(rt->mu);
  *addr = builtin_addr_locked(rt, code);
  if (!*addr) return fail(GPUOS_ERR_INVALID, "no built-in operator %d", code);
  return GPUOS_OK;
}

static int register_builtin_code(gpuos_rt* rt, int code, int* slot) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  OpPtrInt addr = 0;
  int s;
  {
    std::lock_guard<std::mutex> lk(rt->mu);
    addr = builtin_addr_locked(rt, code);
    if (!addr) return fail(GPUOS_ERR_INVALID, "no built-in operator %d", code);
    if (rt->next_slot >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_FULL, "op table full (%d slots)", GPUOS_MAX_OPS);
    s = rt->next_slot++;
  }
  int e = gpuos_rt_set_slot(rt, s, addr);
  if (e) return e;
  if (slot) *slot = s;
  return GPUOS_OK;
}

extern "C" int gpuos_rt_register_builtin_reduce(gpuos_rt* rt, int red_op, int* slot) {
  if (red_op != GPUOS_RED_SUM && red_op != GPUOS_RED_MEAN) return fail(GPUOS_ERR_INVALID, "unknown reduction %d", red_op);
  return register_builtin_code(rt, 100 + GPUOS_EW_NUM_OPS + red_op, slot);
}

extern "C" int gpuos_rt_register_builtin_ew(gpuos_rt* rt, int ew_op, int* slot) {
  if (ew_op < 0 || ew_op >= GPUOS_EW_NUM_OPS) return fail(GPUOS_ERR_INVALID, "unknown element-wise op %d", ew_op);
  return register_builtin_code(rt, 100 + ew_op, slot);
}

// register_elementwise through the expression interpreter: compile the expression into a
// program, write the program into the next free program entry of the running worker module,
// then point `slot` at that entry's operator.  Nothing is loaded and the worker keeps running.
extern "C" int gpuos_rt_register_expr(gpuos_rt* rt, const char* key, const char* expr, int arity, int slot,
                                      int* slot_out) {
  (void)key;  // the key -> slot registry lives with the caller (the Python module caches it)
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (slot >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_INVALID, "slot %d out of range", slot);
  ExprProg prog;
  std::string err;
  int e = expr_compile(expr, arity, &prog, &err);
  if (e) return fail(e, "expression '%s': %s", expr ? expr : "", err.c_str());
  std::lock_guard<std::mutex> jl(rt->jit_mu);  // the worker module does not change meanwhile
  int k, s;
  uint64_t progs, addr;
  {
    std::lock_guard<std::mutex> lk(rt->mu);
    if (rt->next_expr >= kExprPrograms)
      return fail(GPUOS_ERR_FULL, "all %d expression operators of this device are in use", kExprPrograms);
    if (slot < 0 && rt->next_slot >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_FULL, "op table full (%d slots)", GPUOS_MAX_OPS);
    k = rt->next_expr++;
    s = slot >= 0 ? slot : rt->next_slot++;
    rt->expr_progs[k] = prog;
    progs = rt->addr_map[MA_EXPR_PROGS];
    addr = rt->addr_map[MA_EXPR_FNS + k];
  }
  CK(cudaSetDevice(rt->device));
  CK(cudaMemcpyAsync(reinterpret_cast<void*>(progs + (uint64_t)k * sizeof(ExprProg)), &prog, sizeof(ExprProg),
                     cudaMemcpyHostToDevice, rt->cstream));
  CK(cudaStreamSynchronize(rt->cstream));
  if (!addr) return fail(GPUOS_ERR_CUDA, "expression operator %d has no address", k);
  e = gpuos_rt_set_slot(rt, s, addr);
  if (e) return e;
  if (slot_out) *slot_out = s;
  return GPUOS_OK;
}

// ---- operators compiled at run time ---------------------------------------------------------
// Stop the worker (published work drains first) and wait for it to leave the device.
static int stop_worker_locked(gpuos_rt* rt, int timeout_ms) {
  if (rt->failed) return fail(GPUOS_ERR_DEVICE, "%s", rt->fail_msg.c_str());
  if (!rt->launched) return GPUOS_OK;
  const uint64_t ep = rt->epoch;
  if (rt->hc->quit_epoch < ep) rt->hc->quit_epoch = ep;
  const uint64_t t0 = mono_ns();
  while (true) {
    const uint64_t st = rt->rep->state;
    if ((st >> 8) == ep && (st & 0xff) == WS_EXITED) break;
    if (rt->rep->error) return check_device_error_locked(rt);
    if (mono_ns() - t0 > (uint64_t)timeout_ms * 1000000ull) return fail(GPUOS_ERR_TIMEOUT, "worker did not stop");
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  CK(cudaStreamSynchronize(rt->kstream));
  return GPUOS_OK;
}

// An operator compiled and linked, not yet installed: the linked image holds the worker, every
// operator installed before it (`id` of them) and this one.
struct gpuos_jit_staged {
  int device = -1;
  int id = 0;
  jit::Op op;
  std::vector<jit::Op> ops;
  std::vector<char> image;
};

// Compile nothing, link `op` with the worker and the operators installed so far.
static int stage_jit_op(gpuos_rt* rt, int id, jit::Op op, gpuos_jit_staged** out) {
  auto* st = new gpuos_jit_staged();
  st->device = rt->device;
  st->id = id;
  st->op = std::move(op);
  {
    std::lock_guard<std::mutex> jl(rt->jit_mu);
    if ((int)rt->jit_ops.size() != id) {
      delete st;
      return fail(GPUOS_ERR_INVALID, "another operator was installed meanwhile; stage again");
    }
    if (id >= kMaxJitOps) {
      delete st;
      return fail(GPUOS_ERR_FULL, "all %d run-time compiled operators of this device are in use", kMaxJitOps);
    }
    st->ops = rt->jit_ops;
  }
  st->ops.push_back(st->op);
  std::string err;
  const int e = jit::link(st->ops, &st->image, &err);
  if (e) {
    delete st;
    return fail(e, "%s", err.c_str());
  }
  *out = st;
  return GPUOS_OK;
}

// Stop the worker, load the staged module, carry the op table and the expression programs over
// to it, and run the worker from it from the next publish on.  *addr_out = the new operator's
// address.  On failure the runtime keeps its previous module (the worker restarts from it with
// the next publish).
static int commit_jit_op(gpuos_rt* rt, const gpuos_jit_staged& st, uint64_t* addr_out) {
  std::lock_guard<std::mutex> jl(rt->jit_mu);
  if (st.device != rt->device) return fail(GPUOS_ERR_INVALID, "staged for device %d", st.device);
  if ((int)rt->jit_ops.size() != st.id)
    return fail(GPUOS_ERR_INVALID, "another operator was installed after this one was staged; stage again");
  const std::vector<jit::Op>& ops = st.ops;
  std::string err;
  CK(cudaSetDevice(rt->device));
  std::lock_guard<std::mutex> lk(rt->mu);
  // a module load waits for kernels running on the device: load with the worker stopped
  int e = stop_worker_locked(rt, 30000);
  if (e) return e;
  jit::Module m;
  e = jit::load(st.image, ops, &m, &err);
  if (e) return fail(e, "%s", err.c_str());
  auto undo = [&](int code, const char* what) {
    jit::unload(&m);
    return fail(code, "%s: %s", what, err.c_str());
  };
  if (jit::set_smem(m.worker, rt->smem, &err)) return undo(GPUOS_ERR_CUDA, "linked worker");
  int resident = 0;
  if (jit::occupancy(m.worker, rt->cta_threads + 64, rt->smem, &resident, &err)) return undo(GPUOS_ERR_CUDA, "linked worker");
  if (resident < rt->ctas_per_sm) {
    err = std::to_string(resident) + " CTAs per SM fit";
    return undo(GPUOS_ERR_UNSUPPORTED, "linked worker");
  }
  // built-in and operator addresses of the linked module
  void* a0[] = {&rt->addr_dev};
  if (jit::launch(m.addrs, 1, 64, 0, rt->cstream, a0, &err)) return undo(GPUOS_ERR_CUDA, "address kernel");
  std::vector<unsigned long long*> outs(ops.size());
  for (size_t j = 0; j < ops.size(); ++j) {
    outs[j] = rt->addr_dev + MA_COUNT + j;
    void* a1[] = {&outs[j]};
    if (jit::launch(m.op_addr[j], 1, 1, 0, rt->cstream, a1, &err)) return undo(GPUOS_ERR_CUDA, "operator address kernel");
  }
  std::vector<uint64_t> nmap(MA_COUNT + ops.size(), 0);
  std::vector<uint64_t> table(GPUOS_MAX_OPS, 0);
  cudaError_t ce = cudaMemcpyAsync(nmap.data(), rt->addr_dev, sizeof(uint64_t) * nmap.size(), cudaMemcpyDeviceToHost,
                                   rt->cstream);
  if (ce == cudaSuccess)
    ce = cudaMemcpyAsync(table.data(), rt->op_table, sizeof(uint64_t) * GPUOS_MAX_OPS, cudaMemcpyDeviceToHost,
                         rt->cstream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(rt->cstream);
  if (ce != cudaSuccess) {
    err = cudaGetErrorString(ce);
    return undo(GPUOS_ERR_CUDA, "module addresses");
  }
  for (size_t j = 0; j < ops.size(); ++j)
    if (nmap[MA_COUNT + j] == 0) return undo(GPUOS_ERR_CUDA, "operator without an address");
  // op table: every entry that names an operator of the previous module names the same one here
  for (uint64_t& t : table) {
    bool found = false;
    uint64_t v = translate_addr(rt->addr_map, nmap, t, &found);
    if (!found) v = translate_addr(rt->static_map, nmap, t, &found);
    t = v;
  }
  ce = cudaMemcpyAsync(rt->op_table, table.data(), sizeof(uint64_t) * GPUOS_MAX_OPS, cudaMemcpyHostToDevice,
                       rt->cstream);
  // expression programs installed so far
  if (ce == cudaSuccess && rt->next_expr > 0)
    ce = cudaMemcpyAsync(reinterpret_cast<void*>(nmap[MA_EXPR_PROGS]), rt->expr_progs.data(),
                         sizeof(ExprProg) * rt->next_expr, cudaMemcpyHostToDevice, rt->cstream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(rt->cstream);
  if (ce != cudaSuccess) {
    err = cudaGetErrorString(ce);
    return undo(GPUOS_ERR_CUDA, "op table");
  }
  if (rt->jit_mod.mod) rt->old_mods.push_back(rt->jit_mod);
  rt->jit_mod = m;
  rt->jit_ops = ops;
  rt->addr_map = nmap;
  if (addr_out) *addr_out = nmap[MA_COUNT + ops.size() - 1];
  return GPUOS_OK;
}

static int next_slot_for(gpuos_rt* rt, int slot, int* s) {
  std::lock_guard<std::mutex> lk(rt->mu);
  if (slot >= 0) {
    *s = slot;
    return GPUOS_OK;
  }
  if (rt->next_slot >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_FULL, "op table full (%d slots)", GPUOS_MAX_OPS);
  *s = rt->next_slot++;
  return GPUOS_OK;
}

static int current_jit_id(gpuos_rt* rt) {
  std::lock_guard<std::mutex> jl(rt->jit_mu);
  return (int)rt->jit_ops.size();
}

extern "C" int gpuos_rt_jit_stage(gpuos_rt* rt, const char* expr, int arity, gpuos_jit_staged** staged) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (!expr || !staged) return fail(GPUOS_ERR_INVALID, "null argument");
  *staged = nullptr;
  const int id = current_jit_id(rt);
  std::string src, err;
  int e = jit::ew_source(id, expr, arity, &src, &err);
  if (e) return fail(e, "expression '%s': %s", expr, err.c_str());
  jit::Op op;
  op.objs.resize(1);
  op.objs[0].name = "gpuos_jit_op_" + std::to_string(id);
  e = jit::compile(src, (op.objs[0].name + ".cu").c_str(), "cubin", &op.objs[0].bytes, &err);
  if (e) return fail(e, "expression '%s': %s", expr, err.c_str());
  op.addr_kernel = "gpuos_jit_addr_" + std::to_string(id);
  return stage_jit_op(rt, id, std::move(op), staged);
}

extern "C" int gpuos_rt_jit_stage_ptx(gpuos_rt* rt, const char* ptx, size_t ptx_len, const char* entry,
                                      gpuos_jit_staged** staged) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (!ptx || ptx_len == 0 || !entry || !staged) return fail(GPUOS_ERR_INVALID, "empty PTX or entry name");
  *staged = nullptr;
  const int id = current_jit_id(rt);
  std::string src, err;
  int e = jit::bridge_source(id, entry, &src, &err);
  if (e) return fail(e, "entry '%s': %s", entry, err.c_str());
  jit::Op op;
  op.objs.resize(2);
  op.objs[0].ptx = true;
  op.objs[0].name = "gpuos_custom_" + std::to_string(id) + ".ptx";
  op.objs[0].bytes.assign(ptx, ptx + ptx_len);
  if (op.objs[0].bytes.back() != '\0') op.objs[0].bytes.push_back('\0');
  op.objs[1].name = "gpuos_jit_bridge_" + std::to_string(id);
  e = jit::compile(src, (op.objs[1].name + ".cu").c_str(), "cubin", &op.objs[1].bytes, &err);
  if (e) return fail(e, "bridge for '%s': %s", entry, err.c_str());
  op.addr_kernel = "gpuos_jit_addr_" + std::to_string(id);
  return stage_jit_op(rt, id, std::move(op), staged);
}

extern "C" int gpuos_rt_jit_commit(gpuos_rt* rt, gpuos_jit_staged* staged, int slot, int* slot_out) {
  if (!rt) return fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  if (!staged) return fail(GPUOS_ERR_INVALID, "nothing staged");
  if (slot >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_INVALID, "slot %d out of range", slot);
  uint64_t addr = 0;
  int e = commit_jit_op(rt, *staged, &addr);
  if (e) return e;
  int s = -1;
  e = next_slot_for(rt, slot, &s);
  if (e) return e;
  e = gpuos_rt_set_slot(rt, s, addr);
  if (e) return e;
  if (slot_out) *slot_out = s;
  return GPUOS_OK;
}

extern "C" void gpuos_rt_jit_discard(gpuos_jit_staged* staged) { delete staged; }

extern "C" int gpuos_rt_register_jit(gpuos_rt* rt, const char* expr, int arity, int slot, int* slot_out) {
  if (slot >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_INVALID, "slot %d out of range", slot);
  gpuos_jit_staged* st = nullptr;
  int e = gpuos_rt_jit_stage(rt, expr, arity, &st);
  if (e) return e;
  e = gpuos_rt_jit_commit(rt, st, slot, slot_out);
  delete st;
  return e;
}

extern "C" int gpuos_rt_load_custom(gpuos_rt* rt, const char* ptx, size_t ptx_len, const char* entry, int slot,
                                    int* slot_out) {
  if (slot >= GPUOS_MAX_OPS) return fail(GPUOS_ERR_INVALID, "slot %d out of range", slot);
  gpuos_jit_staged* st = nullptr;
  int e = gpuos_rt_jit_stage_ptx(rt, ptx, ptx_len, entry, &st);
  if (e) return e;
  e = gpuos_rt_jit_commit(rt, st, slot, slot_out);
  delete st;
  return e;
}

extern "C" int gpuos_rt_jit_ops(gpuos_rt* rt) {
  if (!rt) return -fail(GPUOS_ERR_NOT_INIT, "gpuos not initialized");
  std::lock_guard<std::mutex> jl(rt->jit_mu);
  return (int)rt->jit_ops.size();
}

// ---- device-free checks of the run-time compile path -----------------------------------------
extern "C" int gpuos_jit_compile(const char* src, int ptx, void* out, size_t cap, size_t* size_out) {
  if (!src) return fail(GPUOS_ERR_INVALID, "null source");
  std::vector<char> bytes;
  std::string err;
  const int e = jit::compile(src, "user.cu", ptx ? "ptx" : "cubin", &bytes, &err);
  if (e) return fail(e, "%s", err.c_str());
  if (size_out) *size_out = bytes.size();
  if (out) {
    if (cap < bytes.size()) return fail(GPUOS_ERR_INVALID, "output buffer of %zu bytes, %zu needed", cap, bytes.size());
    std::memcpy(out, bytes.data(), bytes.size());
  }
  return GPUOS_OK;
}

extern "C" int gpuos_jit_check_expr(const char* expr, int arity, size_t* image_bytes) {
  if (!expr) return fail(GPUOS_ERR_INVALID, "null expression");
  std::string src, err;
  int e = jit::ew_source(0, expr, arity, &src, &err);
  if (e) return fail(e, "expression '%s': %s", expr, err.c_str());
  std::vector<jit::Op> ops(1);
  ops[0].objs.resize(1);
  ops[0].objs[0].name = "gpuos_jit_op_0";
  e = jit::compile(src, "gpuos_jit_op_0.cu", "cubin", &ops[0].objs[0].bytes, &err);
  if (e) return fail(e, "expression '%s': %s", expr, err.c_str());
  std::vector<char> image;
  e = jit::link(ops, &image, &err);
  if (e) return fail(e, "%s", err.c_str());
  if (image_bytes) *image_bytes = image.size();
  return GPUOS_OK;
}

extern "C" int gpuos_jit_nvrtc_version(void) { return jit::nvrtc_version(); }

extern "C" int gpuos_expr_compile(const char* expr, int arity, void* prog_out, int prog_bytes) {
  if (prog_out && prog_bytes < (int)sizeof(ExprProg)) return fail(GPUOS_ERR_INVALID, "program buffer smaller than %zu bytes", sizeof(ExprProg));
  ExprProg prog;
  std::string err;
  const int e = expr_compile(expr, arity, &prog, &err);
  if (e) return fail(e, "expression '%s': %s", expr ? expr : "", err.c_str());
  if (prog_out) std::memcpy(prog_out, &prog, sizeof(prog));
  return GPUOS_OK;
}

// ---- planning hooks -----------------------------------------------------------------------
static int copy_plan(const Plan& p, void* items_out, int max_items, void* layout_out, int* n_items) {
  if (n_items) *n_items = (int)p.items.size();
  if ((int)p.items.size() > max_items) return fail(GPUOS_ERR_FULL, "plan has %zu items", p.items.size());
  if (items_out && !p.items.empty()) std::memcpy(items_out, p.items.data(), p.items.size() * sizeof(WorkItem));
  if (layout_out) {
    std::memset(layout_out, 0, 512);
    if (p.has_layout) std::memcpy(layout_out, &p.layout, sizeof(Layout));
  }
  return GPUOS_OK;
}

extern "C" int gpuos_plan_ew(int op, const GpuosOperand* a, const GpuosOperand* b, int b_is_scalar, double b_scalar,
                             const GpuosOperand* out, const float* params, int nparams, void* items_out, int max_items,
                             void* layout_out, int* n_items) {
  if (!a || !out) return fail(GPUOS_ERR_INVALID, "null operand");
  EwReq r;
  r.op = op;
  r.a = a;
  r.b = b_is_scalar ? nullptr : b;
  r.b_imm = b_is_scalar != 0;
  r.b_val = (float)b_scalar;
  r.out = out;
  for (int i = 0; i < 4; ++i) r.params[i] = (params && i < nparams) ? params[i] : 0.f;
  Plan p;
  int e = plan_ew(r, kHalfBytes, &p);
  if (e) return e;
  return copy_plan(p, items_out, max_items, layout_out, n_items);
}

extern "C" int gpuos_plan_reduce(int red_op, const GpuosOperand* x, const GpuosOperand* out, const int* axes, int naxes,
                                 int keepdim, void* items_out, int max_items, void* layout_out, int* n_items) {
  if (!x || !out) return fail(GPUOS_ERR_INVALID, "null operand");
  Plan p;
  int e = plan_reduce(red_op, *x, *out, axes, naxes, keepdim, kStageBytesDefault, &p);
  if (e) return e;
  return copy_plan(p, items_out, max_items, layout_out, n_items);
}

extern "C" int gpuos_abi_sizes(int64_t* out, int n) {
  const int64_t v[] = {(int64_t)sizeof(TensorRef), (int64_t)sizeof(Task),       (int64_t)offsetof(Task, in0),
                       (int64_t)offsetof(Task, in1), (int64_t)offsetof(Task, out0), (int64_t)sizeof(SyncState),
                       (int64_t)sizeof(WorkQueue), (int64_t)sizeof(WorkItem),   (int64_t)sizeof(Layout),
                       (int64_t)sizeof(GpuosOperand)};
  const int m = (int)(sizeof(v) / sizeof(v[0]));
  for (int i = 0; i < n && i < m; ++i) out[i] = v[i];
  return m;
}

// =========================================================================================
// gpuos_ew_batch_noalloc: one drain-mode launch of the batch worker over a fixed scratch array
// =========================================================================================
// For callers that may not allocate device memory where they run.  Everything the launch needs
// besides the caller's operands -- control words, the completion ticket, layouts and tile
// descriptors -- is written into the library's fixed scratch array (StaticScratch) with one
// stream-ordered copy, and the worker runs once in drain mode (it exits when the last tile
// is done).  Device memory is never allocated; host staging buffers are per thread and reused.
extern "C" cudaError_t gpuos_internal_noalloc_scratch(size_t smem, void** ptr, size_t* bytes);

// Wait for `stream` with a bound (GPUOS_NOALLOC_WAIT_MS, default 60000) instead of blocking for
// good: the launch needs every SM at once, and other work can keep them.
static int noalloc_wait(cudaStream_t stream) {
  const uint64_t limit = (uint64_t)std::max(1, env_int("GPUOS_NOALLOC_WAIT_MS", 60000)) * 1000000ull;
  const uint64_t t0 = mono_ns();
  uint32_t spins = 0;
  while (true) {
    const cudaError_t q = cudaStreamQuery(stream);
    if (q == cudaSuccess) return GPUOS_OK;
    if (q != cudaErrorNotReady) return fail(GPUOS_ERR_CUDA, "stream: %s", cudaGetErrorString(q));
    if (mono_ns() - t0 > limit)
      return fail(GPUOS_ERR_TIMEOUT, "the stream did not finish within %llu ms (the launch needs every SM)",
                  (unsigned long long)(limit / 1000000ull));
    if (++spins < 256) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// Read and clear the sticky error word (the first device error of any call since it was last
// cleared), stream-ordered on `stream`; *err receives it (0: none).
static int noalloc_take_sticky(unsigned char* base, cudaStream_t stream, unsigned long long* err) {
  static thread_local unsigned long long word;
  word = 0;
  CK(cudaMemcpyAsync(&word, base + StaticScratch::kSticky, sizeof(word), cudaMemcpyDeviceToHost, stream));
  CK(cudaMemsetAsync(base + StaticScratch::kSticky, 0, sizeof(word), stream));
  const int e = noalloc_wait(stream);
  if (e) return e;
  *err = word;
  return GPUOS_OK;
}

extern "C" int gpuos_ew_batch_noalloc(const GpuosEwRequest* reqs, int nreq, int flags, cudaStream_t stream) {
  using SS = StaticScratch;
  if (nreq < 0 || (nreq > 0 && !reqs)) return fail(GPUOS_ERR_INVALID, "null request array");
  if (flags & ~GPUOS_FLUSH_SYNC) return fail(GPUOS_ERR_INVALID, "unsupported flags 0x%x (only GPUOS_FLUSH_SYNC)", flags);

  struct Staging {
    Plan plan;
    HazardMap hz;
    std::vector<WorkItem> items;
    std::vector<Layout> layouts;
    std::vector<unsigned char> image;
  };
  static thread_local Staging h;
  h.items.clear();
  h.layouts.clear();
  h.hz.clear();
  uint64_t seg_wait = 0;
  for (int i = 0; i < nreq; ++i) {
    const GpuosEwRequest& q = reqs[i];
    if (!q.a || !q.out) return fail(GPUOS_ERR_INVALID, "request %d: null operand", i);
    EwReq r;
    r.op = q.op;
    r.a = q.a;
    r.b = q.b_is_scalar ? nullptr : q.b;
    r.b_imm = q.b_is_scalar != 0;
    r.b_val = (float)q.b_scalar;
    r.out = q.out;
    for (int k = 0; k < 4; ++k) r.params[k] = k < q.nparams ? q.params[k] : 0.f;
    int e = plan_ew(r, kHalfBytes, &h.plan);
    if (e) return fail(e, "request %d: %s", i, gpuos_rt_last_error());
    const Plan& p = h.plan;
    if (h.items.size() + p.items.size() > SS::kMaxItems)
      return fail(GPUOS_ERR_INVALID,
                  "batch needs more than %llu tiles (request %d brings the total to %llu); "
                  "gpuos_ew_batch_noalloc takes at most GPUOS_NOALLOC_MAX_TILES = %llu",
                  (unsigned long long)SS::kMaxItems, i, (unsigned long long)(h.items.size() + p.items.size()),
                  (unsigned long long)SS::kMaxItems);
    if (p.has_layout && h.layouts.size() + 1 > SS::kMaxLayouts)
      return fail(GPUOS_ERR_INVALID,
                  "batch has more than %u strided or broadcast requests; gpuos_ew_batch_noalloc takes at most "
                  "GPUOS_NOALLOC_MAX_STRIDED = %u",
                  SS::kMaxLayouts, SS::kMaxLayouts);
    // requests that touch memory an earlier request of this call writes (or writes memory it
    // reads) start a new segment: its tiles wait until every earlier tile has completed
    bool hazard = false;
    for (int k = 0; k < p.nreads && !hazard; ++k) hazard = h.hz.conflicts(p.reads[k], false);
    if (!hazard) hazard = h.hz.conflicts(p.write, true);
    if (hazard) {
      h.hz.clear();
      seg_wait = h.items.size();
    }
    for (int k = 0; k < p.nreads; ++k) h.hz.insert(p.reads[k], false);
    h.hz.insert(p.write, true);
    const uint32_t layout_idx = (uint32_t)h.layouts.size();
    if (p.has_layout) h.layouts.push_back(p.layout);
    for (const WorkItem& src : p.items) {
      WorkItem it = src;
      it.wait_items = seg_wait;
      if (p.has_layout) it.aux = layout_idx;
      h.items.push_back(it);
    }
  }
  const uint64_t n = h.items.size();
  int dev = 0, sm_count = 0, smem_optin = 0;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev));
  CK(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  // same stage rule as gpuos_rt_init with one worker CTA per SM
  const uint32_t stages = pick_stages((size_t)smem_optin, kStageBytesDefault);
  const size_t smem = gpuos_internal_smem_header_bytes() + (size_t)stages * kStageBytesDefault;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  CK(gpuos_internal_noalloc_scratch(smem, &scratch, &scratch_bytes));
  unsigned char* base = static_cast<unsigned char*>(scratch);
  if (n == 0) {
    if (!(flags & GPUOS_FLUSH_SYNC)) return GPUOS_OK;
    unsigned long long sticky = 0;
    const int e = noalloc_take_sticky(base, stream, &sticky);
    if (e) return e;
    if (sticky)
      return fail(GPUOS_ERR_DEVICE, "an earlier call without GPUOS_FLUSH_SYNC failed on the device: worker error code "
                  "%llu detail %llu", sticky >> 32, sticky & 0xffffffffull);
    return GPUOS_OK;
  }
  void *op_table = nullptr, *op_alias = nullptr;
  CK(gpuos_internal_table_ptrs(&op_table, &op_alias));

  // host image of the scratch block up to the last tile descriptor; all of it is rewritten
  // by every call, so nothing of an earlier call survives into this one
  const uint64_t seq = 1;
  const uint16_t slot = (uint16_t)(seq % kNumBatchSlots);
  const size_t image_bytes = SS::kItems + n * sizeof(WorkItem);
  h.image.assign(image_bytes, 0);
  unsigned char* img = h.image.data();
  HostCtl* hc = reinterpret_cast<HostCtl*>(img + SS::kHostCtl);
  hc->tail = n;
  hc->quit_epoch = 1;  // drain mode: the launch of epoch 1 exits once every tile is done
  hc->safety_idle_ns = (uint64_t)env_int("GPUOS_SAFETY_IDLE_MS", 10000) * 1000000ull;
  hc->spin_ns = (uint32_t)env_int("GPUOS_SPIN_NS", 32);
  hc->wait_limit_ns = (uint64_t)env_int("GPUOS_DEVICE_WAIT_MS", 5000) * 1000000ull;
  DevCtl* dc_img = reinterpret_cast<DevCtl*>(img + SS::kDevCtl);
  std::memset(dc_img->batch_t0, 0xff, sizeof(dc_img->batch_t0));
  if (!h.layouts.empty())
    std::memcpy(img + SS::kLayouts, h.layouts.data(), h.layouts.size() * sizeof(Layout));
  WorkItem* items = reinterpret_cast<WorkItem*>(img + SS::kItems);
  for (uint64_t i = 0; i < n; ++i) {
    WorkItem it = h.items[i];
    it.batch = slot;
    it.batch_items = (uint32_t)n;
    it.batch_seq = seq;
    items[i] = it;
  }
  // everything but the sticky error word, which keeps a failed asynchronous call's error
  CK(cudaMemcpyAsync(base, img, SS::kSticky, cudaMemcpyHostToDevice, stream));
  CK(cudaMemcpyAsync(base + SS::kSticky + 32, img + SS::kSticky + 32, image_bytes - SS::kSticky - 32,
                     cudaMemcpyHostToDevice, stream));

  WorkerParams P;
  std::memset(&P, 0, sizeof(P));
  P.hc = reinterpret_cast<HostCtl*>(base + SS::kHostCtl);
  P.rep = reinterpret_cast<DevReport*>(base + SS::kReport);
  P.tickets = reinterpret_cast<Ticket*>(base + SS::kTickets);
  P.items = reinterpret_cast<const WorkItem*>(base + SS::kItems);
  P.tasks = nullptr;  // element-wise requests produce no Task items
  P.layouts = reinterpret_cast<const Layout*>(base + SS::kLayouts);
  P.dc = reinterpret_cast<DevCtl*>(base + SS::kDevCtl);
  P.op_table = reinterpret_cast<OpFn*>(op_table);
  P.op_alias = reinterpret_cast<int*>(op_alias);
  P.item_mask = SS::kMaxItems - 1;
  P.task_mask = 0;
  P.layout_mask = SS::kMaxLayouts - 1;
  P.epoch = 1;
  P.stages = stages;
  P.stage_bytes = kStageBytesDefault;
  P.compute_threads = 256;
  P.wait_limit_ns = hc->wait_limit_ns;
  P.sticky_error = reinterpret_cast<unsigned long long*>(base + SS::kSticky);
  CK(gpuos_internal_launch_batch_worker(&P, sm_count, 256 + 64, smem, stream));
  if (!(flags & GPUOS_FLUSH_SYNC)) return GPUOS_OK;

  static thread_local DevReport rep;
  static thread_local Ticket tk;
  CK(cudaMemcpyAsync(&rep, base + SS::kReport, sizeof(rep), cudaMemcpyDeviceToHost, stream));
  CK(cudaMemcpyAsync(&tk, base + SS::kTickets + slot * sizeof(Ticket), sizeof(tk), cudaMemcpyDeviceToHost, stream));
  unsigned long long sticky = 0;
  const int we = noalloc_take_sticky(base, stream, &sticky);
  if (we) return we;
  if (rep.error != 0)
    return fail(GPUOS_ERR_DEVICE, "worker error code %llu detail %llu at tile %llu",
                (unsigned long long)(rep.error >> 32), (unsigned long long)(rep.error & 0xffffffffull),
                (unsigned long long)rep.error_item);
  if (sticky)
    return fail(GPUOS_ERR_DEVICE, "an earlier call without GPUOS_FLUSH_SYNC failed on the device: worker error code "
                "%llu detail %llu", sticky >> 32, sticky & 0xffffffffull);
  if (rep.items_done != n || tk.seq != seq)
    return fail(GPUOS_ERR_DEVICE, "worker exited after %llu of %llu tiles", (unsigned long long)rep.items_done,
                (unsigned long long)n);
  return GPUOS_OK;
}
