// Shared device helpers for the SlottedGLU kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "sg_abi.h"

#define SG_VERSION 1

namespace sg {

// ------------------------------------------------------------------ bf16 bits
__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }
// low / high bf16 of a packed 32-bit word, widened to fp32 exactly
__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// ------------------------------------------------------------------ exp
// e^x for x <= 0, the routing exp shared bit-for-bit with the CPU oracle:
// Cody-Waite reduction x = n*ln2 + r (ln2 split into a 15-bit head and a tail,
// so n*LN2_HI is exact for |n| <= 127) and the degree-7 Taylor polynomial of
// e^r in Horner form.  Every step is one IEEE-rounded fp32 multiply or add
// (__fmul_rn / __fadd_rn are never contracted into FMAs).
__device__ __forceinline__ float routing_exp(float x) {
  const float kLog2e = __uint_as_float(0x3FB8AA3Bu);
  const float kLn2Hi = __uint_as_float(0x3F317200u);
  const float kLn2Lo = __uint_as_float(0x35BFBE8Eu);
  float n = rintf(__fmul_rn(x, kLog2e));
  if (n < -126.0f) return 0.0f;
  float r = __fsub_rn(x, __fmul_rn(n, kLn2Hi));
  r = __fsub_rn(r, __fmul_rn(n, kLn2Lo));
  // Taylor coefficients 1/7! .. 1/0! as exact fp32 bit patterns
  float p = __uint_as_float(0x39500D01u);
  p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(0x3AB60B61u));
  p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(0x3C088889u));
  p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(0x3D2AAAABu));
  p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(0x3E2AAAABu));
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  int ni = static_cast<int>(n);
  if (ni > 127) ni = 127;
  float scale = __uint_as_float(static_cast<uint32_t>(ni + 127) << 23);
  return __fmul_rn(p, scale);
}

// logistic function used by SwiGLU and the shared-expert gate (tolerance-checked)
__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }

// SwiGLU with the reference's bf16 rounding points: silu(g) * u,
// silu(g) = g * sigmoid(g), every elementwise result rounded to bf16.
__device__ __forceinline__ uint16_t swiglu_bf16(float gate_acc, float up_acc) {
  float g = round_bf16(gate_acc);
  float u = round_bf16(up_acc);
  float sg = round_bf16(sigmoidf_(g));
  float silu = round_bf16(g * sg);
  return f32_to_bf16(silu * u);
}

// ------------------------------------------------------------------ warp utils
__device__ __forceinline__ float warp_fold_sum(float v) {
  // pairwise fold 16, 8, 4, 2, 1 -- identical value in every lane
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

}  // namespace sg

#define SG_CUDA_TRY(expr)                                  \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) return SG_ERR_CUDA;             \
  } while (0)

#define SG_LAUNCH_CHECK() SG_CUDA_TRY(cudaGetLastError())
