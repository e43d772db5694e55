// expr.cuh — the stack machine that runs registered expression operators.
//
// Reference: pytorch_ext/gpuos_ext.cpp:814-868 builds one NVRTC module per expression,
// `R = expr(A[, B])` with generic indexing, and loads it next to the running persistent
// kernel.  Here the expression arrives as a postfix program (ExprProg, compiled on the host)
// and one interpreter evaluates it per element; each of the kExprPrograms table entries has
// its own operator address (op_expr<K>), so slots and aliases switch between them exactly as
// between compiled operators.  Every thread runs the same instruction sequence (no
// divergence); the stack lives in thread-local memory.  Transcendental functions are evaluated
// in double precision and rounded once to float, like the built-in operators, so each call
// contributes at most one float rounding error.
#pragma once
#include "refops.cuh"

namespace gpuos {

__device__ ExprProg g_expr_progs[kExprPrograms];

// Evaluates one element.  The host compiler emits only programs with a balanced stack no
// deeper than kExprMaxStack; every push and pop is still checked, and a program that breaks
// the discipline yields NaN instead of touching memory outside the stack.
__device__ __forceinline__ float expr_run(const ExprProg& p, float A, float B) {
  float st[kExprMaxStack];
  int sp = 0;
  const int len = p.len;
  const float bad = __int_as_float(0x7fc00000);
  for (int pc = 0; pc < len; ++pc) {
    const int op = p.code[pc];
    if (op == XO_A || op == XO_B || op == XO_CONST) {
      if (sp >= kExprMaxStack) return bad;
      st[sp++] = op == XO_A ? A : op == XO_B ? B : p.imm[pc];
      continue;
    }
    if (op == XO_SELECT) {
      if (sp < 3) return bad;
      const float y = st[--sp], x = st[--sp], c = st[--sp];
      st[sp++] = c != 0.f ? x : y;
      continue;
    }
    if (op >= XO_MIN && op < XO_NUM) {  // two-argument functions
      if (sp < 2) return bad;
      const float y = st[--sp], x = st[--sp];
      float r;
      switch (op) {
        case XO_MIN: r = fminf(x, y); break;
        case XO_MAX: r = fmaxf(x, y); break;
        case XO_POW: r = (float)pow((double)x, (double)y); break;
        case XO_FMOD: r = fmodf(x, y); break;
        case XO_ATAN2: r = (float)atan2((double)x, (double)y); break;
        default: r = copysignf(x, y); break;
      }
      st[sp++] = r;
      continue;
    }
    if (op >= XO_ADD && op <= XO_OR) {
      if (sp < 2) return bad;
      const float y = st[--sp], x = st[--sp];
      float r;
      switch (op) {
        case XO_ADD: r = __fadd_rn(x, y); break;
        case XO_SUB: r = __fsub_rn(x, y); break;
        case XO_MUL: r = __fmul_rn(x, y); break;
        case XO_DIV: r = __fdiv_rn(x, y); break;
        case XO_LT: r = x < y ? 1.f : 0.f; break;
        case XO_LE: r = x <= y ? 1.f : 0.f; break;
        case XO_GT: r = x > y ? 1.f : 0.f; break;
        case XO_GE: r = x >= y ? 1.f : 0.f; break;
        case XO_EQ: r = x == y ? 1.f : 0.f; break;
        case XO_NE: r = x != y ? 1.f : 0.f; break;
        case XO_AND: r = (x != 0.f && y != 0.f) ? 1.f : 0.f; break;
        default: r = (x != 0.f || y != 0.f) ? 1.f : 0.f; break;
      }
      st[sp++] = r;
      continue;
    }
    if (sp < 1 || op < XO_NEG || op >= XO_MIN) return bad;  // one argument, in place
    const float x = st[sp - 1];
    float r;
    switch (op) {
      case XO_NEG: r = -x; break;
      case XO_NOT: r = x == 0.f ? 1.f : 0.f; break;
      case XO_EXP: r = (float)exp((double)x); break;
      case XO_LOG: r = (float)log((double)x); break;
      case XO_LOG1P: r = (float)log1p((double)x); break;
      case XO_EXPM1: r = (float)expm1((double)x); break;
      case XO_SQRT: r = sqrtf(x); break;
      case XO_RSQRT: r = (float)(1.0 / sqrt((double)x)); break;
      case XO_ABS: r = fabsf(x); break;
      case XO_TANH: r = (float)tanh((double)x); break;
      case XO_SIN: r = (float)sin((double)x); break;
      case XO_COS: r = (float)cos((double)x); break;
      case XO_TAN: r = (float)tan((double)x); break;
      case XO_ERF: r = (float)erf((double)x); break;
      case XO_FLOOR: r = floorf(x); break;
      case XO_CEIL: r = ceilf(x); break;
      case XO_TRUNC: r = truncf(x); break;
      case XO_ROUND: r = roundf(x); break;
      case XO_EXP2: r = (float)exp2((double)x); break;
      case XO_LOG2: r = (float)log2((double)x); break;
      case XO_LOG10: r = (float)log10((double)x); break;
      case XO_SINH: r = (float)sinh((double)x); break;
      case XO_COSH: r = (float)cosh((double)x); break;
      case XO_ASIN: r = (float)asin((double)x); break;
      case XO_ACOS: r = (float)acos((double)x); break;
      default: r = (float)atan((double)x); break;
    }
    st[sp - 1] = r;
  }
  return sp == 1 ? st[0] : bad;
}

// Reference-ABI operator body for program k: out[i] = expr(in0[i], in1[i]) over the Task,
// with the Task's own sizes/strides (broadcast inputs carry stride 0) and the reference's
// dtype casts.  Programs that fail the host-side checks never reach the table; the checks
// are repeated here so that a corrupted program cannot index outside the stack.
__device__ __noinline__ void expr_task(int k, const Task& t) {
  // private copy read from L2: a program is written once, after other programs whose bytes
  // may share its cache lines were already read through this SM's (non-coherent) L1
  ExprProg p;
  const uint4* src = reinterpret_cast<const uint4*>(&g_expr_progs[k]);
  uint4* dst = reinterpret_cast<uint4*>(&p);
#pragma unroll
  for (int i = 0; i < (int)(sizeof(ExprProg) / 16); ++i) dst[i] = __ldcg(src + i);
  if (p.len <= 0 || p.len > kExprMaxCode || p.depth <= 0 || p.depth > kExprMaxStack) return;
  const int64_t N = t.numel;
  const bool two = p.arity == 2 && t.in1.data != nullptr;
  for (int64_t li = threadIdx.x; li < N; li += blockDim.x) {
    const float A = ld_elem(t.in0.data, t.in0.dtype, ref_offset(t.in0, li));
    const float B = two ? ld_elem(t.in1.data, t.in1.dtype, ref_offset(t.in1, li)) : 0.f;
    st_elem(t.out0.data, t.out0.dtype, ref_offset(t.out0, li), expr_run(p, A, B));
  }
}

template <int K>
__device__ void op_expr(const Task& t) {
  expr_task(K, t);
}

}  // namespace gpuos
