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

#define GPUOS_EW_MATH(...) __VA_ARGS__
#include "ew_math.inc"
#undef GPUOS_EW_MATH

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
