// ops.cuh — element-wise operator math and dtype conversion (fp32 compute).
//
// Semantics follow PyTorch CPU eager (the parity oracle); where the reference's
// expressions differ (pytorch_ext/scheduler.py:192-205, 244-290: tanh-GELU for gelu,
// expf-1 for elu, no softplus threshold, NaN-dropping max/min; src/persistent_kernel.cu:105
// div-by-zero -> 0) the PyTorch form is used:
//   relu(x)        = x < 0 ? +0 : x                      (keeps -0 and NaN)
//   maximum(a,b)   = NaN if either is NaN, else (a < b ? b : a)
//   minimum(a,b)   = NaN if either is NaN, else (b < a ? b : a)
//   clamp(x,lo,hi) = min(max(x,lo),hi) with max(x,y) = x < y ? y : x, min(x,y) = y < x ? y : x
//   hardsigmoid    = clamp(x + 3, 0, 6) / 6
//   hardswish      = x * clamp(x + 3, 0, 6) / 6
//   gelu           = x * 0.5 * (1 + erf(x * sqrt(1/2)))
//   gelu(tanh)     = 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 * x^3)))
//   elu            = x > 0 ? x : expm1(x) * alpha
//   softplus       = x * beta > threshold ? x : log1p(exp(x * beta)) / beta
//   leaky_relu     = x > 0 ? x : x * slope
//   div            = IEEE a / b (inf / nan on zero divisors)
// Non-transcendental arithmetic is IEEE round-to-nearest float; the build disables FMA
// contraction so products and sums round exactly as on the CPU.
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace gpuos {

__device__ __forceinline__ float ld_elem(const void* base, int dt, int64_t i) {
  if (dt == kF32) return reinterpret_cast<const float*>(base)[i];
  if (dt == kF16) return __half2float(reinterpret_cast<const __half*>(base)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
}

__device__ __forceinline__ void st_elem(void* base, int dt, int64_t i, float v) {
  if (dt == kF32) {
    reinterpret_cast<float*>(base)[i] = v;
  } else if (dt == kF16) {
    reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
  } else {
    reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  }
}

__device__ __forceinline__ float qnan() { return __int_as_float(0x7fc00000); }
__device__ __forceinline__ float max_std(float x, float y) { return x < y ? y : x; }
__device__ __forceinline__ float min_std(float x, float y) { return y < x ? y : x; }

// Transcendental cores are evaluated in double precision and rounded once to float, so
// the fp32 result is within about 0.5 ulp of the true value; PyTorch CPU's own results are
// within about 1 ulp, which keeps the difference inside the 2-ulp parity bound.  The
// non-transcendental ops are single IEEE float operations (bit-exact).
template <int OP>
__device__ __forceinline__ float ew_apply(float a, float b, float p0, float p1) {
  if constexpr (OP == GPUOS_EW_ADD) return __fadd_rn(a, b);
  else if constexpr (OP == GPUOS_EW_MUL) return __fmul_rn(a, b);
  else if constexpr (OP == GPUOS_EW_SUB) return __fsub_rn(a, b);
  else if constexpr (OP == GPUOS_EW_DIV) return __fdiv_rn(a, b);
  else if constexpr (OP == GPUOS_EW_MAXIMUM) return (a != a || b != b) ? qnan() : (a < b ? b : a);
  else if constexpr (OP == GPUOS_EW_MINIMUM) return (a != a || b != b) ? qnan() : (b < a ? b : a);
  else if constexpr (OP == GPUOS_EW_POW) return (float)pow((double)a, (double)b);
  else if constexpr (OP == GPUOS_EW_COPY) return a;
  else if constexpr (OP == GPUOS_EW_RELU) return a < 0.f ? 0.f : a;
  else if constexpr (OP == GPUOS_EW_SIGMOID) {
    // PyTorch CPU forms 1 / (1 + exp(-x)) in float: where exp(-x) overflows float (x below about
    // -88.72) the result is 0, not the (denormal) true value
    const double e = exp(-(double)a);
    return isinf((float)e) ? 0.f : (float)(1.0 / (1.0 + e));
  }
  else if constexpr (OP == GPUOS_EW_TANH) return (float)tanh((double)a);
  else if constexpr (OP == GPUOS_EW_EXP) return (float)exp((double)a);
  else if constexpr (OP == GPUOS_EW_LOG) return (float)log((double)a);
  else if constexpr (OP == GPUOS_EW_SQRT) return __fsqrt_rn(a);
  else if constexpr (OP == GPUOS_EW_ABS) return fabsf(a);
  else if constexpr (OP == GPUOS_EW_HARDSIGMOID)
    return __fdiv_rn(min_std(max_std(__fadd_rn(a, 3.f), 0.f), 6.f), 6.f);
  else if constexpr (OP == GPUOS_EW_HARDSWISH)
    return __fdiv_rn(__fmul_rn(a, min_std(max_std(__fadd_rn(a, 3.f), 0.f), 6.f)), 6.f);
  else if constexpr (OP == GPUOS_EW_GELU) {
    // PyTorch CPU (its vectorised kernel, which every tensor of 8 or more elements takes) gives NaN
    // for +-inf and overflows to +inf once x (1 + erf(x / sqrt 2)) does in float (x >= 2^127)
    if (isinf(a)) return qnan();
    if (a >= 1.7014118346046923e38f) return __int_as_float(0x7f800000);
    const double x = a;
    return (float)(x * 0.5 * (1.0 + erf(x * 0.70710678118654752440)));
  } else if constexpr (OP == GPUOS_EW_GELU_TANH) {
    const double x = a;
    const double inner = 0.79788456080286535588 * (x + 0.044715 * x * x * x);
    return (float)(0.5 * x * (1.0 + tanh(inner)));
  } else if constexpr (OP == GPUOS_EW_SIN) return (float)sin((double)a);
  else if constexpr (OP == GPUOS_EW_COS) return (float)cos((double)a);
  else if constexpr (OP == GPUOS_EW_LEAKY_RELU) return a > 0.f ? a : __fmul_rn(a, p0);
  else if constexpr (OP == GPUOS_EW_CLAMP) return min_std(max_std(a, p0), p1);
  else if constexpr (OP == GPUOS_EW_CLAMP_MIN) return max_std(a, p0);
  else if constexpr (OP == GPUOS_EW_CLAMP_MAX) return min_std(a, p0);
  else if constexpr (OP == GPUOS_EW_ELU) return a > 0.f ? a : (float)(expm1((double)a) * (double)p0);
  else if constexpr (OP == GPUOS_EW_SOFTPLUS) {
    const float xb = __fmul_rn(a, p0);
    return xb > p1 ? a : (float)(log1p(exp((double)xb)) / (double)p0);
  } else if constexpr (OP == GPUOS_EW_NEG) return -a;
  else if constexpr (OP == GPUOS_EW_ADD_ALPHA) return __fmaf_rn(p0, b, a);
  else if constexpr (OP == GPUOS_EW_SUB_ALPHA) return __fmaf_rn(-p0, b, a);
  else return a;
}

// Runtime-selected op (generic and reference-ABI paths; the contiguous tile path is
// instantiated per op).
__device__ __noinline__ float ew_apply_dyn(int op, float a, float b, float p0, float p1) {
  switch (op) {
#define GPUOS_CASE(k) case k: return ew_apply<k>(a, b, p0, p1);
    GPUOS_CASE(0) GPUOS_CASE(1) GPUOS_CASE(2) GPUOS_CASE(3) GPUOS_CASE(4) GPUOS_CASE(5)
    GPUOS_CASE(6) GPUOS_CASE(7) GPUOS_CASE(8) GPUOS_CASE(9) GPUOS_CASE(10) GPUOS_CASE(11)
    GPUOS_CASE(12) GPUOS_CASE(13) GPUOS_CASE(14) GPUOS_CASE(15) GPUOS_CASE(16) GPUOS_CASE(17)
    GPUOS_CASE(18) GPUOS_CASE(19) GPUOS_CASE(20) GPUOS_CASE(21) GPUOS_CASE(22) GPUOS_CASE(23)
    GPUOS_CASE(24) GPUOS_CASE(25) GPUOS_CASE(26) GPUOS_CASE(27) GPUOS_CASE(28) GPUOS_CASE(29)
#undef GPUOS_CASE
    default: return a;
  }
}

}  // namespace gpuos
