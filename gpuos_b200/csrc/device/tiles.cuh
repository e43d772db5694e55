// tiles.cuh — per-item compute bodies of the batched path.
//
// The reference aggregates sub-tasks in one device function that one CTA walks
// serially, decoding every element with three int64 stride walks
// (src/persistent_kernel.cu:20-31, 81-112).  Here each work item is one tile; the
// dequeue warp has staged its contiguous operands in shared memory with a TMA bulk
// copy, and the compute warps run one tile function reached through a device
// function-pointer table (one indirect call per tile, not per element).
#pragma once
#include <type_traits>

#include "ptx.cuh"
#include "ops.cuh"

namespace gpuos {

struct TileCtx {
  const StageMeta* m;
  const unsigned char* sa;  // stage buffer for operand a (shared memory)
  const unsigned char* sb;  // stage buffer for operand b (shared memory)
  uint32_t tid;             // compute-thread index
  uint32_t nt;              // compute-thread count (multiple of 32)
};
typedef void (*TileFn)(const TileCtx&);

__device__ __forceinline__ float item_p0(const WorkItem& it) { return __uint_as_float((uint32_t)it.x); }
__device__ __forceinline__ float item_p1(const WorkItem& it) { return __uint_as_float((uint32_t)(it.x >> 32)); }

template <int OP>
__device__ __forceinline__ float4 ew_apply4(float4 a, float4 b, float p0, float p1) {
  return make_float4(ew_apply<OP>(a.x, b.x, p0, p1), ew_apply<OP>(a.y, b.y, p0, p1),
                     ew_apply<OP>(a.z, b.z, p0, p1), ew_apply<OP>(a.w, b.w, p0, p1));
}

// The ops whose fp32 contiguous tiles run inlined (the cases of f32_staged_tile's switch).
constexpr uint32_t kF32InlineOps =
    (1u << GPUOS_EW_ADD) | (1u << GPUOS_EW_MUL) | (1u << GPUOS_EW_SUB) | (1u << GPUOS_EW_DIV) |
    (1u << GPUOS_EW_MAXIMUM) | (1u << GPUOS_EW_MINIMUM) | (1u << GPUOS_EW_COPY) | (1u << GPUOS_EW_RELU) |
    (1u << GPUOS_EW_ABS) | (1u << GPUOS_EW_NEG) | (1u << GPUOS_EW_ADD_ALPHA) | (1u << GPUOS_EW_SUB_ALPHA) |
    (1u << GPUOS_EW_CLAMP) | (1u << GPUOS_EW_CLAMP_MIN) | (1u << GPUOS_EW_CLAMP_MAX) | (1u << GPUOS_EW_LEAKY_RELU) |
    (1u << GPUOS_EW_SQRT) | (1u << GPUOS_EW_HARDSIGMOID) | (1u << GPUOS_EW_HARDSWISH) | (1u << GPUOS_EW_EXP) |
    (1u << GPUOS_EW_LOG) | (1u << GPUOS_EW_TANH) | (1u << GPUOS_EW_ELU) | (1u << GPUOS_EW_SOFTPLUS) |
    (1u << GPUOS_EW_GELU);

// The ops of kSharedOps on four values, the op chosen at run time: one copy of the staged
// transpose block's loops then serves all of them (OP = kDynOp).  Per-op copies of the loops
// missed in the instruction cache whenever consecutive blocks had different ops (on a stream of
// transposed fp16 / broadcast bf16 requests with four ops interleaved, "no instruction" was the
// largest stall reason, 32 % of stalls).
// Division keeps a body per op: its IEEE slow path needs registers that make the shared body
// spill.  (Two shared bodies, simple ops and float-math ops, spilled less but measured slower
// on the mixed stream: consecutive tiles alternating between the two bodies miss again.)
constexpr int kDynOp = -1;
constexpr uint32_t kSharedOps = kF32InlineOps & ~(1u << GPUOS_EW_DIV);
__device__ __forceinline__ void ew_apply4_sw(uint32_t op, const float* a, const float* b, float p0, float p1,
                                             float* v) {
  switch (op) {
#define GPUOS_SW(k)                                                    \
  case k: {                                                            \
    _Pragma("unroll") for (int t = 0; t < 4; ++t) v[t] = ew_apply<k>(a[t], b[t], p0, p1); \
  } break;
    GPUOS_SW(GPUOS_EW_ADD) GPUOS_SW(GPUOS_EW_MUL) GPUOS_SW(GPUOS_EW_SUB)
    GPUOS_SW(GPUOS_EW_MAXIMUM) GPUOS_SW(GPUOS_EW_MINIMUM) GPUOS_SW(GPUOS_EW_COPY) GPUOS_SW(GPUOS_EW_RELU)
    GPUOS_SW(GPUOS_EW_ABS) GPUOS_SW(GPUOS_EW_NEG) GPUOS_SW(GPUOS_EW_ADD_ALPHA) GPUOS_SW(GPUOS_EW_SUB_ALPHA)
    GPUOS_SW(GPUOS_EW_CLAMP) GPUOS_SW(GPUOS_EW_CLAMP_MIN) GPUOS_SW(GPUOS_EW_CLAMP_MAX) GPUOS_SW(GPUOS_EW_LEAKY_RELU)
    GPUOS_SW(GPUOS_EW_SQRT) GPUOS_SW(GPUOS_EW_HARDSIGMOID) GPUOS_SW(GPUOS_EW_HARDSWISH) GPUOS_SW(GPUOS_EW_EXP)
    GPUOS_SW(GPUOS_EW_LOG) GPUOS_SW(GPUOS_EW_TANH) GPUOS_SW(GPUOS_EW_ELU) GPUOS_SW(GPUOS_EW_SOFTPLUS)
    GPUOS_SW(GPUOS_EW_GELU)
#undef GPUOS_SW
    default:
#pragma unroll
      for (int t = 0; t < 4; ++t) v[t] = a[t];
  }
}


// ---- 16-bit vector helpers: 8 elements per 16 bytes ----------------------------------
__device__ __forceinline__ void unpack8(uint4 raw, int dt, float* f) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (dt == kF16) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
      float2 v = __half22float2(h);
      f[2 * k] = v.x;
      f[2 * k + 1] = v.y;
    } else {
      f[2 * k] = __uint_as_float(w[k] << 16);
      f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  }
}

__device__ __forceinline__ uint4 pack8(const float* f, int dt) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (dt == kF16) {
      __half2 h = __floats2half2_rn(f[2 * k], f[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Load 8 consecutive elements starting at element i (16-byte aligned for 16-bit
// types, 32-byte span for fp32) as floats.
__device__ __forceinline__ void load8(const unsigned char* base, int dt, uint32_t i, float* f) {
  if (dt == kF32) {
    const float4* p = reinterpret_cast<const float4*>(base) + 2 * (i >> 3);
    float4 v0 = p[0], v1 = p[1];
    f[0] = v0.x; f[1] = v0.y; f[2] = v0.z; f[3] = v0.w;
    f[4] = v1.x; f[5] = v1.y; f[6] = v1.z; f[7] = v1.w;
  } else {
    uint4 raw = reinterpret_cast<const uint4*>(base)[i >> 3];
    unpack8(raw, dt, f);
  }
}

__device__ __forceinline__ void store8(unsigned char* base, int dt, uint32_t i, const float* f) {
  if (dt == kF32) {
    float4* p = reinterpret_cast<float4*>(base) + 2 * (i >> 3);
    ptx::st_cs_v4(p, make_float4(f[0], f[1], f[2], f[3]));
    ptx::st_cs_v4(p + 1, make_float4(f[4], f[5], f[6], f[7]));
  } else {
    uint4 v = pack8(f, dt);
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(reinterpret_cast<uint4*>(base) + (i >> 3)),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  }
}

// ---- EW_CONTIG -------------------------------------------------------------------------
template <int OP>
__device__ __forceinline__ void ew_contig(const TileCtx& c) {
  const WorkItem& it = c.m->item;
  const uint32_t n = it.count;
  const float p0 = item_p0(it), p1 = item_p1(it);
  const int dta = it.dt_a, dtb = it.dt_b, dto = it.dt_o;
  const bool has_b = (it.flags & IF_B_PRESENT) != 0;
  const bool b_imm = (it.flags & IF_B_SCALAR) != 0;
  const bool a_bc = (it.flags & IF_A_BCAST) != 0;
  const bool b_bc = (it.flags & IF_B_BCAST) != 0;
  const unsigned char* A = (c.m->staged & 1) ? c.sa + c.m->a_off : reinterpret_cast<const unsigned char*>(it.a);
  const unsigned char* B = (c.m->staged & 2) ? c.sb + c.m->b_off : reinterpret_cast<const unsigned char*>(it.b);
  unsigned char* O = reinterpret_cast<unsigned char*>(it.o);

  float bscal = 0.f;
  if (has_b) {
    if (b_imm) bscal = __uint_as_float((uint32_t)it.b);
    else if (b_bc) bscal = ld_elem(B, dtb, 0);
  }
  const bool b_vec = has_b && !b_imm && !b_bc;
  float ascal = a_bc ? ld_elem(A, dta, 0) : 0.f;

  // Vector body: 8 elements per step when every vector operand is 16-byte aligned.
  const bool a_al = a_bc || ((reinterpret_cast<uintptr_t>(A) & 15) == 0);
  const bool b_al = !b_vec || ((reinterpret_cast<uintptr_t>(B) & 15) == 0);
  const bool o_al = (reinterpret_cast<uintptr_t>(O) & 15) == 0;
  uint32_t done = 0;
  if (a_al && b_al && o_al) {
    const uint32_t n8 = n >> 3;
    if (dta == kF32 && dto == kF32 && (!b_vec || dtb == kF32) && !a_bc) {
      // fp32 fast path: two float4 per step.
      const float4* A4 = reinterpret_cast<const float4*>(A);
      const float4* B4 = reinterpret_cast<const float4*>(B);
      float4* O4 = reinterpret_cast<float4*>(O);
      const float4 bsv = make_float4(bscal, bscal, bscal, bscal);
      const uint32_t n4 = n >> 2;
      for (uint32_t i = c.tid; i < n4; i += c.nt) {
        float4 av = A4[i];
        float4 bv = b_vec ? B4[i] : bsv;
        ptx::st_cs_v4(O4 + i, ew_apply4<OP>(av, bv, p0, p1));
      }
      done = n4 << 2;
    } else {
      for (uint32_t v = c.tid; v < n8; v += c.nt) {
        float fa[8], fb[8], fo[8];
        if (a_bc) {
#pragma unroll
          for (int k = 0; k < 8; ++k) fa[k] = ascal;
        } else {
          load8(A, dta, v << 3, fa);
        }
        if (b_vec) {
          load8(B, dtb, v << 3, fb);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) fb[k] = bscal;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) fo[k] = ew_apply<OP>(fa[k], fb[k], p0, p1);
        store8(O, dto, v << 3, fo);
      }
      done = n8 << 3;
    }
  }
  for (uint32_t i = done + c.tid; i < n; i += c.nt) {
    float av = a_bc ? ascal : ld_elem(A, dta, i);
    float bv = b_vec ? ld_elem(B, dtb, i) : bscal;
    st_elem(O, dto, i, ew_apply<OP>(av, bv, p0, p1));
  }
}

// ---- fp32 contiguous tiles of the simple ops, inlined into the compute loop -------------
// A tile function reached through the table is an indirect call, and every indirect call
// saves and restores the callee-saved registers of all compute threads through local memory
// (about 36 KB of extra L2 writes per tile at 256 threads).  The fp32 tiles of the ops whose
// arithmetic is a few instructions, with a staged (and b staged, scalar or absent), run here
// instead, through the same ew_apply arithmetic.
template <int OP>
__device__ __forceinline__ void f32_staged_loop(uint32_t sA, uint32_t sB, bool b_vec, float bscal, float* O,
                                                uint32_t n, uint32_t tid, uint32_t nt, float p0, float p1) {
  const uint32_t n4 = n >> 2;
  const float4 bsv = make_float4(bscal, bscal, bscal, bscal);
  float4* O4 = reinterpret_cast<float4*>(O);
  for (uint32_t i = tid; i < n4; i += nt) {
    const float4 av = ptx::ld_shared_v4f(sA + i * 16u);
    const float4 bv = b_vec ? ptx::ld_shared_v4f(sB + i * 16u) : bsv;
    ptx::st_cs_v4(O4 + i, ew_apply4<OP>(av, bv, p0, p1));
  }
  for (uint32_t i = (n4 << 2) + tid; i < n; i += nt) {
    const float av = ptx::ld_shared_f(sA + i * 4u);
    const float bv = b_vec ? ptx::ld_shared_f(sB + i * 4u) : bscal;
    O[i] = ew_apply<OP>(av, bv, p0, p1);
  }
}

// Whether an item is one of those tiles: fp32 a and out, contiguous (no broadcast), a staged
// (and b staged, scalar or absent), 16-byte aligned.
__device__ __forceinline__ bool f32_inline_ok(const StageMeta& m) {
  const WorkItem& it = m.item;
  const uint32_t flags = it.flags;
  if (it.kind != IK_EW_CONTIG || it.op >= 32 || !((kF32InlineOps >> it.op) & 1u)) return false;
  if (it.dt_a != kF32 || it.dt_o != kF32 || (flags & (IF_A_BCAST | IF_B_BCAST)) || !(m.staged & 1)) return false;
  const bool b_vec = (flags & IF_B_PRESENT) && !(flags & IF_B_SCALAR);
  if (b_vec && (it.dt_b != kF32 || !(m.staged & 2))) return false;
  return !((m.a_off & 15u) || (b_vec && (m.b_off & 15u)) || (it.o & 15ull));
}

// Runs the tile and returns true when it qualifies (f32_inline_ok); false leaves it to the table.
__device__ __forceinline__ bool f32_staged_tile(const StageMeta& m, const unsigned char* sa,
                                                const unsigned char* sb, uint32_t tid, uint32_t nt) {
  if (!f32_inline_ok(m)) return false;
  const WorkItem& it = m.item;
  const uint32_t flags = it.flags;
  const bool b_imm = (flags & IF_B_SCALAR) != 0;
  const bool b_vec = (flags & IF_B_PRESENT) && !b_imm;
  const float bscal = ((flags & IF_B_PRESENT) && b_imm) ? __uint_as_float((uint32_t)it.b) : 0.f;
  const uint32_t sA = ptx::smem_addr(sa + m.a_off);
  const uint32_t sB = b_vec ? ptx::smem_addr(sb + m.b_off) : 0u;
  float* O = reinterpret_cast<float*>(it.o);
  const uint32_t n = it.count;
  const float p0 = item_p0(it), p1 = item_p1(it);
  // one body per op: a body shared by all ops (the op switched per four values, as the staged
  // transpose blocks do) measured slower here (a stream of 16384 fp32 requests over 19 ops:
  // 0.64 -> 0.78 ms)
  switch (it.op) {
#define GPUOS_F32_CASE(OPC) \
  case OPC:                 \
    f32_staged_loop<OPC>(sA, sB, b_vec, bscal, O, n, tid, nt, p0, p1); \
    return true;
    GPUOS_F32_CASE(GPUOS_EW_ADD)
    GPUOS_F32_CASE(GPUOS_EW_MUL)
    GPUOS_F32_CASE(GPUOS_EW_SUB)
    GPUOS_F32_CASE(GPUOS_EW_DIV)
    GPUOS_F32_CASE(GPUOS_EW_MAXIMUM)
    GPUOS_F32_CASE(GPUOS_EW_MINIMUM)
    GPUOS_F32_CASE(GPUOS_EW_COPY)
    GPUOS_F32_CASE(GPUOS_EW_RELU)
    GPUOS_F32_CASE(GPUOS_EW_ABS)
    GPUOS_F32_CASE(GPUOS_EW_NEG)
    GPUOS_F32_CASE(GPUOS_EW_ADD_ALPHA)
    GPUOS_F32_CASE(GPUOS_EW_SUB_ALPHA)
    GPUOS_F32_CASE(GPUOS_EW_CLAMP)
    GPUOS_F32_CASE(GPUOS_EW_CLAMP_MIN)
    GPUOS_F32_CASE(GPUOS_EW_CLAMP_MAX)
    GPUOS_F32_CASE(GPUOS_EW_LEAKY_RELU)
    GPUOS_F32_CASE(GPUOS_EW_SQRT)
    GPUOS_F32_CASE(GPUOS_EW_HARDSIGMOID)
    GPUOS_F32_CASE(GPUOS_EW_HARDSWISH)
    GPUOS_F32_CASE(GPUOS_EW_EXP)
    GPUOS_F32_CASE(GPUOS_EW_LOG)
    GPUOS_F32_CASE(GPUOS_EW_TANH)
    GPUOS_F32_CASE(GPUOS_EW_ELU)
    GPUOS_F32_CASE(GPUOS_EW_SOFTPLUS)
    GPUOS_F32_CASE(GPUOS_EW_GELU)
#undef GPUOS_F32_CASE
    default:
      return false;
  }
}

// ---- EW_GENERIC: strided / broadcast operands -----------------------------------------
__device__ __noinline__ void ew_generic(const TileCtx& c) {
  const int OP = c.m->item.op;
  const WorkItem& it = c.m->item;
  const Layout& L = c.m->ext.layout;
  const int nd = L.ndim;
  const bool has_b = (it.flags & IF_B_PRESENT) != 0;
  const bool b_imm = (it.flags & IF_B_SCALAR) != 0;
  const float bscal = b_imm ? __uint_as_float((uint32_t)it.b) : 0.f;
  const float p0 = L.params[0], p1 = L.params[1];
  const void* A = reinterpret_cast<const void*>(it.a);
  const void* B = reinterpret_cast<const void*>(it.b);
  void* O = reinterpret_cast<void*>(it.o);
  const int64_t start = (int64_t)it.x;
  const int64_t n = it.count;
  for (int64_t k = c.tid; k < n; k += c.nt) {
    int64_t rem = start + k;
    int64_t oa = 0, ob = 0, oo = 0;
    for (int d = nd - 1; d >= 0; --d) {
      const int64_t sz = L.sizes[d];
      const int64_t idx = rem % sz;
      rem /= sz;
      oa += idx * L.sa[d];
      ob += idx * L.sb[d];
      oo += idx * L.so[d];
    }
    const float av = ld_elem(A, it.dt_a, oa);
    const float bv = has_b ? (b_imm ? bscal : ld_elem(B, it.dt_b, ob)) : 0.f;
    st_elem(O, it.dt_o, oo, ew_apply_dyn(OP, av, bv, p0, p1));
  }
}

// ---- EW_2D: a block of a 2-D strided / broadcast layout ------------------------------
// The layout is [rows, cols] with the output's inner dimension last.  An item covers rows
// [r0, r0 + nr) x columns [c0, c0 + nc) (x = r0 | c0 << 32, count = nr << 16 | nc); offsets
// are row * stride0 + col * stride1 in 32 bits, so no element index is ever divided.
//   row mode: warp w takes rows w, w + nwarps, ...; lanes take consecutive columns.
//   transpose mode (IF_A_T / IF_B_T, nr <= 16, nc <= 256): an operand that is contiguous
//   along rows is first read 16 rows per column (coalesced in its own memory order) into
//   the stage buffer, which these blocks do not use for staging, as float [16][256] with
//   the column index XOR 2*row (no bank conflicts in either phase); then thread j computes
//   column j for every row, so the output is written coalesced along its columns.
constexpr uint32_t kBarBlock = 1;  // named barrier of the compute warps (transpose mode)
static_assert(k2dBlockRows == 16 && k2dBlockCols == 256, "the transpose tile below is float [16][256]");
static_assert(16 * 256 * 4 <= kStageBytesDefault / 2, "a transpose tile fills at most one stage half");

// Loads of a batch of kBatch elements go into registers before any store: a store through a
// generic pointer may alias the next load, so a load-compute-store loop would wait a full
// memory latency per element.
constexpr uint32_t kBatch = 8;

// Storage type <-> float, and f(T{}) called with the storage type of a dtype code, so a loop
// is compiled once per dtype instead of branching on the dtype for every element.
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename F>
__device__ __forceinline__ void with_dtype(int dt, F&& f) {
  if (dt == kF16) f(__half{});
  else if (dt == kBF16) f(__nv_bfloat16{});
  else f(float{});
}

// apply(a, b) is the element operation (its parameters captured).
template <typename F>
__device__ __forceinline__ void ew_2d_body(const TileCtx& c, F&& apply) {
  const WorkItem& it = c.m->item;
  const Layout& L = c.m->ext.layout;
  const uint32_t nr = it.count >> 16, nc = it.count & 0xffffu;
  const int64_t r0 = (int64_t)(uint32_t)it.x, c0 = (int64_t)(it.x >> 32);
  const int32_t a0s = (int32_t)L.sa[0], a1s = (int32_t)L.sa[1], b0s = (int32_t)L.sb[0], b1s = (int32_t)L.sb[1];
  const int32_t o0s = (int32_t)L.so[0], o1s = (int32_t)L.so[1];
  const int dta = it.dt_a, dtb = it.dt_b, dto = it.dt_o;
  const uint32_t flags = it.flags;
  const bool has_b = (flags & IF_B_PRESENT) != 0;
  const bool b_imm = (flags & IF_B_SCALAR) != 0;
  const bool b_mem = has_b && !b_imm;
  const float bscal = b_imm ? __uint_as_float((uint32_t)it.b) : 0.f;
  const unsigned char* A =
      reinterpret_cast<const unsigned char*>(it.a) + (r0 * L.sa[0] + c0 * L.sa[1]) * dtype_size(dta);
  const unsigned char* B =
      b_mem ? reinterpret_cast<const unsigned char*>(it.b) + (r0 * L.sb[0] + c0 * L.sb[1]) * dtype_size(dtb) : nullptr;
  unsigned char* O = reinterpret_cast<unsigned char*>(it.o) + (r0 * L.so[0] + c0 * L.so[1]) * dtype_size(dto);
  const bool a_t = (flags & IF_A_T) != 0, b_t = b_mem && (flags & IF_B_T) != 0;

  if (!a_t && !b_t) {
    // row mode: warp w takes rows w, w + nw, ...; lane l takes columns l, l + 32, ...; each
    // step loads kBatch columns of one row before it stores them
    const uint32_t warp = c.tid >> 5, lane = c.tid & 31, nw = c.nt >> 5;
    with_dtype(dto, [&](auto otag) {
      using TO = decltype(otag);
      for (uint32_t r = warp; r < nr; r += nw) {
        const unsigned char* Ar = A + (int64_t)((int32_t)r * a0s) * dtype_size(dta);
        const unsigned char* Br = b_mem ? B + (int64_t)((int32_t)r * b0s) * dtype_size(dtb) : nullptr;
        TO* Or = reinterpret_cast<TO*>(O) + (int32_t)r * o0s;
        for (uint32_t j0 = lane; j0 < nc; j0 += 32 * kBatch) {
          float va[kBatch], vb[kBatch];
#pragma unroll
          for (uint32_t u = 0; u < kBatch; ++u) {
            const uint32_t j = j0 + 32 * u;
            va[u] = j < nc ? ld_elem(Ar, dta, (int32_t)j * a1s) : 0.f;
            vb[u] = (b_mem && j < nc) ? ld_elem(Br, dtb, (int32_t)j * b1s) : bscal;
          }
#pragma unroll
          for (uint32_t u = 0; u < kBatch; ++u) {
            const uint32_t j = j0 + 32 * u;
            if (j < nc) Or[(int32_t)j * o1s] = from_f<TO>(apply(va[u], vb[u]));
          }
        }
      }
    });
    return;
  }
  // transpose mode
  const uint32_t sta = ptx::smem_addr(c.sa), stb = ptx::smem_addr(c.sb);
  const uint32_t total = 16u * nc;
  auto fill = [&](auto tag, const unsigned char* X, int32_t x0, int32_t x1, uint32_t dst) {
    using T = decltype(tag);
    const T* Xp = reinterpret_cast<const T*>(X);
    for (uint32_t e0 = c.tid; e0 < total; e0 += c.nt * kBatch) {
      float v[kBatch];
#pragma unroll
      for (uint32_t u = 0; u < kBatch; ++u) {
        const uint32_t e = e0 + c.nt * u, r = e & 15u, j = e >> 4;
        v[u] = (e < total && r < nr) ? to_f<T>(Xp[(int32_t)r * x0 + (int32_t)j * x1]) : 0.f;
      }
#pragma unroll
      for (uint32_t u = 0; u < kBatch; ++u) {
        const uint32_t e = e0 + c.nt * u, r = e & 15u, j = e >> 4;
        if (e < total && r < nr) ptx::st_shared_f(dst + 4u * (r * 256u + (j ^ (r << 1))), v[u]);
      }
    }
  };
  if (a_t) with_dtype(dta, [&](auto t) { fill(t, A, a0s, a1s, sta); });
  if (b_t) with_dtype(dtb, [&](auto t) { fill(t, B, b0s, b1s, stb); });
  ptx::named_bar_sync(kBarBlock, c.nt);
  // thread j computes column j for every row of the block
  const bool b_col = b_mem && !b_t && b0s == 0;  // b constant down a column (row broadcast)
  with_dtype(dto, [&](auto otag) {
    using TO = decltype(otag);
    for (uint32_t j = c.tid; j < nc; j += c.nt) {
      const float bj = b_col ? ld_elem(B, dtb, (int32_t)j * b1s) : bscal;
      TO* oc = reinterpret_cast<TO*>(O) + (int32_t)j * o1s;
      for (uint32_t r = 0; r < nr; ++r) {
        const uint32_t k = 4u * (r * 256u + (j ^ (r << 1)));
        const float av = a_t ? ptx::ld_shared_f(sta + k) : ld_elem(A, dta, (int32_t)r * a0s + (int32_t)j * a1s);
        const float bv = b_t ? ptx::ld_shared_f(stb + k)
                             : ((b_mem && !b_col) ? ld_elem(B, dtb, (int32_t)r * b0s + (int32_t)j * b1s) : bj);
        oc[(int32_t)r * o0s] = from_f<TO>(apply(av, bv));
      }
    }
  });
  // the stage buffer is next filled by bulk copies (async proxy) after these generic writes
  ptx::fence_proxy_async_smem();
}

template <int OP>
__device__ __forceinline__ void ew_2d(const TileCtx& c) {
  const float p0 = c.m->ext.layout.params[0], p1 = c.m->ext.layout.params[1];
  ew_2d_body(c, [=](float a, float b) { return ew_apply<OP>(a, b, p0, p1); });
}


// ---- EW_2DT: staged transpose blocks ----------------------------------------------------
// A block is every row (nr) x nc columns of a 2-D layout whose operand a runs along rows with
// unit stride; w = 2^lg >= nc, w >= 8 and nr * w <= 4096.  The dequeue warp staged a's block in
// stage half A exactly as it lies in memory: element (r, j) at a_off + (j * sa1 + r) * es.
// Phase 1 gives each thread one row r and a quad of columns 4jq..4jq+3: four 16- or 32-bit shared
// loads (consecutive threads take consecutive rows: consecutive addresses) and one 16-byte store
// of the four floats into the transpose buffer T in stage half B.  T holds row r as cw = w / 4
// 16-byte chunks, chunk jq at r * cw + (jq ^ f(r)), f(r) = (r >> ksh) & swm with
// ksh = log2(max(1, 8 / cw)) and swm = min(cw, 8) - 1: the eight chunks a quarter-warp writes (or
// reads) fall in eight different 16-byte bank groups.  Phase 2 gives each thread a row and a
// column quad with consecutive threads on consecutive quads: one 16-byte shared load, four
// results, one 16-byte store when the output allows it (coalesced either way).
// jq = q / nr in phase 1 uses a multiply by ceil(2^32 / nr), exact for q, nr <= 4096.
struct T2d {
  uint32_t nr, nc, lg, cw;  // rows, valid columns, log2 and quads (cw = w / 4) of the width
  uint32_t ksh, swm;        // swizzle of the chunk index
};

__device__ __forceinline__ T2d t2d_geom(uint32_t nr, uint32_t nc, uint32_t lg) {
  T2d g;
  g.nr = nr;
  g.nc = nc;
  g.lg = lg;
  g.cw = 1u << (lg - 2);
  g.ksh = lg >= 5 ? 0u : 5u - lg;
  g.swm = (lg >= 5 ? 8u : g.cw) - 1u;
  return g;
}

// Byte offset in T of chunk jq of row r.
__device__ __forceinline__ uint32_t t2d_chunk(const T2d& g, uint32_t r, uint32_t jq) {
  return ((r << (g.lg - 2)) + (jq ^ ((r >> g.ksh) & g.swm))) << 4;
}

// Phase 1 for one storage type; TSRC: 0 float, 1 half, 2 bfloat16.  Columns at or beyond nc
// are not read (their T entries are never used).
template <int TSRC>
__device__ __forceinline__ void t2d_fill(const T2d& g, uint32_t src, uint32_t tbuf, uint32_t sa1, uint32_t tid,
                                         uint32_t nt) {
  constexpr uint32_t es = TSRC == 0 ? 4u : 2u;
  const uint32_t nq = (g.nc + 3u) >> 2;
  const uint32_t total = g.nr * nq;
  // ceil(2^32 / nr) = floor((2^32 - 1) / nr) + 1 for nr >= 2: a 32-bit division (a 64-bit one is a
  // long software routine, run by every thread of every block)
  const uint32_t mg = g.nr > 1 ? 0xffffffffu / g.nr + 1u : 0u;
  const uint32_t cstep = sa1 * es;  // bytes from one column to the next
  for (uint32_t q = tid; q < total; q += nt) {
    const uint32_t jq = g.nr > 1 ? __umulhi(q, mg) : q;
    const uint32_t r = q - jq * g.nr;
    const uint32_t j0 = jq << 2;
    const uint32_t a = src + (j0 * sa1 + r) * es;
    float v[4];
#pragma unroll
    for (uint32_t t = 0; t < 4; ++t) {
      const uint32_t at = a + t * cstep;
      if (j0 + t < g.nc) {
        if constexpr (TSRC == 0) v[t] = ptx::ld_shared_f(at);
        else if constexpr (TSRC == 1) v[t] = __half2float(__ushort_as_half((unsigned short)ptx::ld_shared_u16(at)));
        else v[t] = __uint_as_float(ptx::ld_shared_u16(at) << 16);
      } else {
        v[t] = 0.f;
      }
    }
    ptx::st_shared_v4f(tbuf + t2d_chunk(g, r, jq), make_float4(v[0], v[1], v[2], v[3]));
  }
}

// Phase 1 when a's block could not be staged (the planner keeps spans within a stage half, so
// this only guards the layout): read a from global memory.
__device__ __forceinline__ void t2d_fill_global(const T2d& g, const unsigned char* A, int dta, uint32_t tbuf,
                                                uint32_t sa1, uint32_t tid, uint32_t nt) {
  const uint32_t nq = (g.nc + 3u) >> 2;
  for (uint32_t q = tid; q < g.nr * nq; q += nt) {
    const uint32_t jq = q / g.nr, r = q - jq * g.nr;
    float v[4];
#pragma unroll
    for (uint32_t t = 0; t < 4; ++t)
      v[t] = (jq * 4 + t < g.nc) ? ld_elem(A, dta, (int64_t)(jq * 4 + t) * sa1 + r) : 0.f;
    ptx::st_shared_v4f(tbuf + t2d_chunk(g, r, jq), make_float4(v[0], v[1], v[2], v[3]));
  }
}

// Four results of one output quad into row r, columns j0..j0+3 (those below nc).
template <typename TO>
__device__ __forceinline__ void t2d_store4(TO* O, int32_t o0s, int32_t o1s, uint32_t r, uint32_t j0, uint32_t nc,
                                           bool vec, const float* v) {
  TO* p = O + (int32_t)r * o0s + (int32_t)j0 * o1s;
  if (vec && j0 + 4 <= nc) {
    if constexpr (sizeof(TO) == 4) {
      *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      const TO h0 = from_f<TO>(v[0]), h1 = from_f<TO>(v[1]), h2 = from_f<TO>(v[2]), h3 = from_f<TO>(v[3]);
      uint2 u;
      const unsigned short* b0 = reinterpret_cast<const unsigned short*>(&h0);
      const unsigned short* b1 = reinterpret_cast<const unsigned short*>(&h1);
      const unsigned short* b2 = reinterpret_cast<const unsigned short*>(&h2);
      const unsigned short* b3 = reinterpret_cast<const unsigned short*>(&h3);
      u.x = (uint32_t)*b0 | ((uint32_t)*b1 << 16);
      u.y = (uint32_t)*b2 | ((uint32_t)*b3 << 16);
      *reinterpret_cast<uint2*>(p) = u;
    }
    return;
  }
#pragma unroll
  for (uint32_t t = 0; t < 4; ++t)
    if (j0 + t < nc) p[(int32_t)t * o1s] = from_f<TO>(v[t]);
}

// Phase 2 for one output type.  bmode: 0 none or scalar (bscal), 1 constant down a column
// (b[(c0 + j) * b1s]), 2 any stride (b[r * b0s + (c0 + j) * b1s]).  vec: the output's column
// stride is 1 and every quad starts on a 16-byte (float) or 8-byte (16-bit) boundary.
template <int OP, typename TO>
__device__ __forceinline__ void t2d_out(const T2d& g, uint32_t tbuf, TO* O, int32_t o0s, int32_t o1s, bool vec,
                                        const void* B, int dtb, int bmode, int32_t b0s, int32_t b1s,
                                        const float* bpre, bool have_b, float p0, float p1, uint32_t tid,
                                        uint32_t nt, uint32_t dop) {
  const uint32_t qsh = g.lg - 2, total = g.nr << qsh;
  // with cw dividing nt every quad of a thread is in the same column quad: a column broadcast
  // operand is read once per thread (before phase 1, `bpre`, when `have_b`)
  const bool fixed = (nt & (g.cw - 1u)) == 0u;
  uint32_t jqb = have_b ? (tid & (g.cw - 1u)) : 0xffffffffu;
  float bq[4] = {bpre[0], bpre[1], bpre[2], bpre[3]};
  for (uint32_t q = tid; q < total; q += nt) {
    const uint32_t jq = q & (g.cw - 1u), r = q >> qsh, j0 = jq << 2;
    if (j0 >= g.nc) continue;
    const float4 a4 = ptx::ld_shared_v4f(tbuf + t2d_chunk(g, r, jq));
    const float av[4] = {a4.x, a4.y, a4.z, a4.w};
    if (bmode == 1 && (!fixed || jq != jqb)) {
#pragma unroll
      for (uint32_t t = 0; t < 4; ++t) bq[t] = j0 + t < g.nc ? ld_elem(B, dtb, (int64_t)(j0 + t) * b1s) : 0.f;
      jqb = jq;
    } else if (bmode == 2) {
#pragma unroll
      for (uint32_t t = 0; t < 4; ++t)
        bq[t] = j0 + t < g.nc ? ld_elem(B, dtb, (int64_t)r * b0s + (int64_t)(j0 + t) * b1s) : 0.f;
    }
    float v[4];
    if constexpr (OP == kDynOp) {
      ew_apply4_sw(dop, av, bq, p0, p1, v);
    } else {
#pragma unroll
      for (uint32_t t = 0; t < 4; ++t) v[t] = ew_apply<OP>(av[t], bq[t], p0, p1);
    }
    t2d_store4<TO>(O, o0s, o1s, r, j0, g.nc, vec, v);
  }
}

template <int OP>
__device__ __forceinline__ void ew_2dt(const TileCtx& c) {
  const StageMeta& m = *c.m;
  const WorkItem& it = m.item;
  const Layout& L = m.ext.layout;
  const T2d g = t2d_geom(it.count >> 16, it.count & 0xffffu, (uint32_t)it.x);
  const uint32_t c0 = (uint32_t)(it.x >> 32);
  const uint32_t sa1 = (uint32_t)L.sa[1];
  const int dta = it.dt_a, dtb = it.dt_b, dto = it.dt_o;
  const uint32_t tbuf = ptx::smem_addr(c.sb);
  const uint32_t flags = it.flags;
  const bool b_imm = (flags & IF_B_SCALAR) != 0;
  const bool b_mem = (flags & IF_B_PRESENT) && !b_imm;
  const int32_t b0s = (int32_t)L.sb[0], b1s = (int32_t)L.sb[1];
  const int bmode = !b_mem ? 0 : (b0s == 0 ? 1 : 2);
  const float bscal = b_imm ? __uint_as_float((uint32_t)it.b) : 0.f;
  const void* B = b_mem ? reinterpret_cast<const unsigned char*>(it.b) + (int64_t)c0 * b1s * dtype_size(dtb)
                        : nullptr;
  // a broadcast row operand: each thread's four columns are fixed (cw divides nt), so their
  // loads are issued now and land while phase 1 runs
  // (raw bits: converting here would wait for the loads before phase 1)
  uint32_t braw[4] = {0u, 0u, 0u, 0u};
  bool have_b = false;
  if (bmode == 1 && (c.nt & (g.cw - 1u)) == 0u) {
    const uint32_t j0 = (c.tid & (g.cw - 1u)) << 2;
    if (dtb == kF32) {
#pragma unroll
      for (uint32_t t = 0; t < 4; ++t)
        if (j0 + t < g.nc) braw[t] = reinterpret_cast<const uint32_t*>(B)[(int64_t)(j0 + t) * b1s];
    } else {
#pragma unroll
      for (uint32_t t = 0; t < 4; ++t)
        if (j0 + t < g.nc) braw[t] = reinterpret_cast<const unsigned short*>(B)[(int64_t)(j0 + t) * b1s];
    }
    have_b = true;
  }
  if (m.staged & 1) {
    const uint32_t src = ptx::smem_addr(c.sa) + m.a_off;
    if (dta == kF16) t2d_fill<1>(g, src, tbuf, sa1, c.tid, c.nt);
    else if (dta == kBF16) t2d_fill<2>(g, src, tbuf, sa1, c.tid, c.nt);
    else t2d_fill<0>(g, src, tbuf, sa1, c.tid, c.nt);
  } else {
    const unsigned char* A = reinterpret_cast<const unsigned char*>(it.a) + (int64_t)c0 * sa1 * dtype_size(dta);
    t2d_fill_global(g, A, dta, tbuf, sa1, c.tid, c.nt);
  }
  ptx::named_bar_sync(kBarBlock, c.nt);
  const int32_t o0s = (int32_t)L.so[0], o1s = (int32_t)L.so[1];
  const int eso = dtype_size(dto);
  unsigned char* O = reinterpret_cast<unsigned char*>(it.o) + (int64_t)c0 * o1s * eso;
  // quads start at columns 4k: vector stores need unit column stride, and the block start and the
  // row stride on a 4-element boundary of 16 (float) or 8 (16-bit) bytes
  const bool vec = o1s == 1 && (o0s & 3) == 0 && ((reinterpret_cast<uintptr_t>(O) & (uintptr_t)(4 * eso - 1)) == 0);
  const float p0 = L.params[0], p1 = L.params[1];
  float bpre[4] = {bscal, bscal, bscal, bscal};
  if (have_b) {
#pragma unroll
    for (uint32_t t = 0; t < 4; ++t)
      bpre[t] = dtb == kF32 ? __uint_as_float(braw[t])
                : dtb == kBF16 ? __uint_as_float(braw[t] << 16)
                               : __half2float(__ushort_as_half((unsigned short)braw[t]));
  }
  if (dto == kF16)
    t2d_out<OP, __half>(g, tbuf, reinterpret_cast<__half*>(O), o0s, o1s, vec, B, dtb, bmode, b0s, b1s, bpre, have_b, p0,
                        p1, c.tid, c.nt, it.op);
  else if (dto == kBF16)
    t2d_out<OP, __nv_bfloat16>(g, tbuf, reinterpret_cast<__nv_bfloat16*>(O), o0s, o1s, vec, B, dtb, bmode, b0s, b1s,
                               bpre, have_b, p0, p1, c.tid, c.nt, it.op);
  else
    t2d_out<OP, float>(g, tbuf, reinterpret_cast<float*>(O), o0s, o1s, vec, B, dtb, bmode, b0s, b1s, bpre, have_b,
                       p0, p1, c.tid, c.nt, it.op);
  // the stage is next filled by bulk copies (async proxy) after these generic writes of T
  ptx::fence_proxy_async_smem();
}

// ---- reductions ------------------------------------------------------------------------

// Elements of a row group, as float: staged rows by 32-bit shared-memory addresses (a group
// never exceeds its stage), rows left in place by global pointers.
template <typename T>
struct StagedRows {
  uint32_t base, rs, is;  // shared address of row 0; row and element strides in bytes
  __device__ __forceinline__ float operator()(uint32_t r, int64_t j) const {
    const uint32_t a = base + r * rs + (uint32_t)j * is;
    if constexpr (sizeof(T) == 4) return ptx::ld_shared_f(a);
    else if constexpr (std::is_same<T, __half>::value)
      return __half2float(__ushort_as_half((unsigned short)ptx::ld_shared_u16(a)));
    else return __uint_as_float(ptx::ld_shared_u16(a) << 16);
  }
};
template <typename T>
struct GlobalRows {
  const T* X;
  int64_t rs, is;  // in elements
  __device__ __forceinline__ float operator()(uint32_t r, int64_t j) const { return to_f<T>(X[(int64_t)r * rs + j * is]); }
};

// One lane's sum over the 128-element chunks of row r that start at j - lane, j - lane + step,
// ... below C: two chunks (eight loads) per step, then a last whole chunk, then the rest of
// the last chunk (the chunk after it starts beyond C).  Four partial sums, added in an order
// that depends only on C, step and the first chunk.
template <typename L>
__device__ __forceinline__ float chunk_sum(const L& ld, uint32_t r, int64_t j, int64_t C, int64_t step) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  for (; j + step + 96 < C; j += 2 * step) {
    const float v0 = ld(r, j), v1 = ld(r, j + 32), v2 = ld(r, j + 64), v3 = ld(r, j + 96);
    const float v4 = ld(r, j + step), v5 = ld(r, j + step + 32), v6 = ld(r, j + step + 64),
                v7 = ld(r, j + step + 96);
    s0 = __fadd_rn(__fadd_rn(s0, v0), v4);
    s1 = __fadd_rn(__fadd_rn(s1, v1), v5);
    s2 = __fadd_rn(__fadd_rn(s2, v2), v6);
    s3 = __fadd_rn(__fadd_rn(s3, v3), v7);
  }
  if (j + 96 < C) {
    const float v0 = ld(r, j), v1 = ld(r, j + 32), v2 = ld(r, j + 64), v3 = ld(r, j + 96);
    s0 = __fadd_rn(s0, v0);
    s1 = __fadd_rn(s1, v1);
    s2 = __fadd_rn(s2, v2);
    s3 = __fadd_rn(s3, v3);
    j += step;
  }
  for (; j < C; j += 32) s0 = __fadd_rn(s0, ld(r, j));
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

__device__ __forceinline__ void row_store(void* out, int dto, uint32_t r, float s, bool mean, int64_t C) {
  st_elem(out, dto, r, mean ? __fdiv_rn(s, (float)C) : s);
}

// Rows of one item; every row is read by all 32 lanes of a warp on consecutive elements (no
// bank conflicts on staged rows).  Rows of 128 elements or more: a warp takes two rows per
// step, eight loads in flight per lane and the two rows' shuffle reductions interleaved; when
// the item has fewer rows than there are compute warps, each row is split over wpr warps (the
// largest power of two with rows * wpr <= warps): part p of a row takes its 128-element chunks
// p, p + wpr, ..., and the row's first warp adds the parts' sums in order after a block
// barrier.  Shorter rows: four rows per warp step, one partial sum per lane and row, the four
// rows' shuffle reductions interleaved.  The order of additions depends only on C and the
// item's row count, so the result is deterministic.  Inlined in the compute loop (no call
// through the tile table), loads specialised by dtype and by where the rows are.
template <typename L>
__device__ __forceinline__ void row_reduce_rows(const TileCtx& c, const L& ld, uint32_t rows, int64_t C, bool mean,
                                                void* out, int dto) {
  const uint32_t warp = c.tid >> 5, lane = c.tid & 31, nw = c.nt >> 5;
  if (C >= 128 && rows * 2 <= nw) {
    uint32_t lw = 1;  // log2 of the warps per row
    while ((rows << (lw + 1)) <= nw && lw < 3) ++lw;
    const uint32_t wpr = 1u << lw, r = warp >> lw, part = warp & (wpr - 1u);
    // partial sums of the parts meet in the stage's descriptor extension, which nothing
    // reads for a row-reduction item until the stage is handed back
    float* parts = reinterpret_cast<float*>(const_cast<StageMeta*>(c.m)->ext.raw);
    if (r < rows) {
      float s = chunk_sum(ld, r, (int64_t)part * 128 + lane, C, (int64_t)128 << lw);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
      if (lane == 0) parts[warp] = s;
    }
    ptx::named_bar_sync(kBarBlock, c.nt);
    if (r < rows && part == 0 && lane == 0) {
      float s = parts[warp];
      for (uint32_t k = 1; k < wpr; ++k) s = __fadd_rn(s, parts[warp + k]);
      row_store(out, dto, r, s, mean, C);
    }
    return;
  }
  if (C >= 128) {
    for (uint32_t r = warp; r < rows; r += 2 * nw) {
      const uint32_t r2 = r + nw;
      float a = chunk_sum(ld, r, lane, C, 128);
      float b = r2 < rows ? chunk_sum(ld, r2, lane, C, 128) : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        b = __fadd_rn(b, __shfl_xor_sync(0xffffffffu, b, o));
      }
      if (lane == 0) row_store(out, dto, r, a, mean, C);
      if (lane == 1 && r2 < rows) row_store(out, dto, r2, b, mean, C);
    }
    return;
  }
  const int32_t c32 = (int32_t)C;
  for (uint32_t rb = warp * 4; rb < rows; rb += nw * 4) {
    float s[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      s[q] = 0.f;
      if (rb + q < rows)
        for (int32_t j = lane; j < c32; j += 32) s[q] = __fadd_rn(s[q], ld(rb + q, j));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int q = 0; q < 4; ++q) s[q] = __fadd_rn(s[q], __shfl_xor_sync(0xffffffffu, s[q], o));
    }
    if (lane < 4 && rb + lane < rows) {
      const float v = lane == 0 ? s[0] : lane == 1 ? s[1] : lane == 2 ? s[2] : s[3];
      row_store(out, dto, rb + lane, v, mean, C);
    }
  }
}

__device__ __forceinline__ void row_reduce_body(const TileCtx& c) {
  const WorkItem& it = c.m->item;
  const uint32_t rows = it.count;
  const int64_t C = it.aux;
  const int64_t rs = (int64_t)it.x;
  const int64_t is = (int64_t)it.b;
  const bool mean = (it.flags & IF_MEAN) != 0;
  void* out = reinterpret_cast<void*>(it.o);
  const int dto = it.dt_o;
  const bool staged = (c.m->staged & 1) != 0;
  with_dtype(it.dt_a, [&](auto tag) {
    using T = decltype(tag);
    if (staged) {
      const StagedRows<T> ld{ptx::smem_addr(c.sa) + c.m->a_off, (uint32_t)(rs * (int64_t)sizeof(T)),
                             (uint32_t)(is * (int64_t)sizeof(T))};
      row_reduce_rows(c, ld, rows, C, mean, out, dto);
    } else {
      const GlobalRows<T> ld{reinterpret_cast<const T*>(it.a), rs, is};
      row_reduce_rows(c, ld, rows, C, mean, out, dto);
    }
  });
}


// Arbitrary reduced axes: one output element per thread, serial over the reduced extent.
__device__ __forceinline__ void red_generic_tile(const TileCtx& c) {
  const WorkItem& it = c.m->item;
  const Layout& L = c.m->ext.layout;
  const void* A = reinterpret_cast<const void*>(it.a);
  void* O = reinterpret_cast<void*>(it.o);
  const bool mean = (it.flags & IF_MEAN) != 0;
  const int64_t start = (int64_t)it.x;
  for (int64_t k = c.tid; k < (int64_t)it.count; k += c.nt) {
    int64_t rem = start + k, ia = 0, oo = 0;
    for (int d = L.ndim - 1; d >= 0; --d) {
      const int64_t idx = rem % L.sizes[d];
      rem /= L.sizes[d];
      ia += idx * L.sa[d];
      oo += idx * L.so[d];
    }
    float acc = 0.f;
    for (int64_t rv = 0; rv < L.rtotal; ++rv) {
      int64_t t = rv, off = 0;
      for (int d = L.rdim - 1; d >= 0; --d) {
        const int64_t idx = t % L.rsizes[d];
        t /= L.rsizes[d];
        off += idx * L.rsa[d];
      }
      acc = __fadd_rn(acc, ld_elem(A, it.dt_a, ia + off));
    }
    if (mean) acc = __fdiv_rn(acc, (float)L.rtotal);
    st_elem(O, it.dt_o, oo, acc);
  }
}

// ---- top-k of rows ----------------------------------------------------------------------
// Preference key of a value: larger is preferred.  IEEE order as unsigned integers, NaN above
// every number for largest-first (PyTorch's topk orders NaN as the largest value) and below
// every number for smallest-first.
__device__ __forceinline__ uint32_t topk_key(float v, bool largest) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  if (v != v) return largest ? 0xffffffffu : 0u;
  return largest ? key : ~key;
}

// Warp w takes rows w, w + nwarps, ...  Every candidate has a distinct packed value
// (key << 32 | ~index, so equal values prefer the lower index); round q takes the warp-wide
// maximum below round q-1's winner, so k rounds give the k preferred elements in order and
// nothing has to be marked.  Values are copied bit for bit (they keep x's dtype).
__device__ __forceinline__ void topk_tile(const TileCtx& c) {
  const WorkItem& it = c.m->item;
  const uint32_t rows = it.count, n = it.aux, k = (uint32_t)it.x;
  const bool largest = ((it.x >> 32) & 1u) != 0;
  const int dt = it.dt_a;
  const int es = dtype_size(dt);
  const unsigned char* base =
      (c.m->staged & 1) ? c.sa + c.m->a_off : reinterpret_cast<const unsigned char*>(it.a);
  unsigned char* vals = reinterpret_cast<unsigned char*>(it.o);
  int64_t* idx = reinterpret_cast<int64_t*>(it.b);
  const uint32_t warp = c.tid >> 5, lane = c.tid & 31, nw = c.nt >> 5;
  for (uint32_t r = warp; r < rows; r += nw) {
    const unsigned char* row = base + (int64_t)r * n * es;
    unsigned long long last = ~0ull;
    for (uint32_t q = 0; q < k; ++q) {
      unsigned long long best = 0;
      for (uint32_t j = lane; j < n; j += 32) {
        const unsigned long long pk =
            ((unsigned long long)topk_key(ld_elem(row, dt, j), largest) << 32) | (0xffffffffu - j);
        if (pk < last && pk > best) best = pk;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      last = best;
      if (lane == 0) {
        const uint32_t j = 0xffffffffu - (uint32_t)best;
        const int64_t o = (int64_t)r * k + q;
        if (es == 4) reinterpret_cast<uint32_t*>(vals)[o] = reinterpret_cast<const uint32_t*>(row)[j];
        else reinterpret_cast<uint16_t*>(vals)[o] = reinterpret_cast<const uint16_t*>(row)[j];
        idx[o] = j;
      }
    }
  }
}


}  // namespace gpuos
