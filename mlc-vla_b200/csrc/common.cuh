// Shared device helpers for the π0.5 B200 kernels: element-type traits, warp-level MMA and
// shared-memory load wrappers, cp.async, and the rounding helpers that pin where the model
// dtype rounds (the reference keeps every Linear output, residual and activation in the model
// dtype and every norm / RoPE / softmax statistic in fp32).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pi0 {

template <typename T>
struct Tr;

template <>
struct Tr<__half> {
  using T2 = __half2;
  static __device__ __forceinline__ float f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half t(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ float r(float x) { return __half2float(__float2half_rn(x)); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr bool kBf16 = false;
};

template <>
struct Tr<__nv_bfloat16> {
  using T2 = __nv_bfloat162;
  static __device__ __forceinline__ float f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 t(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float r(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr bool kBf16 = true;
};

// ------------------------------------------------------------------------------------------
// cp.async (Ampere-style 16-byte async copies, used by the v1 tiles)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte copy global -> shared; src_bytes = 0 zero-fills the destination.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ------------------------------------------------------------------------------------------
// ldmatrix / mma.sync
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

template <typename T>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, const uint32_t* b);

template <>
__device__ __forceinline__ void mma16816<__half>(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* c, const uint32_t* a,
                                                       const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// tf32 m16n8k8 (fp32 operands rounded to tf32 with cvt.rna), fp32 accumulate.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void mma1688_tf32(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// ------------------------------------------------------------------------------------------
// programmatic dependent launch: every kernel of the chain waits for its predecessor's results
// with griddepcontrol.wait before touching them (a no-op when launched without the attribute)
// and lets its own dependents get scheduled early.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// math
// ------------------------------------------------------------------------------------------
// GELU, tanh approximation, 0.5·x·(1 + tanh(u)) with u = √(2/π)·(x + 0.044715·x³), in fp32.
// Evaluated through the identity 1 + tanh(u) = 2 / (1 + e^(−2u)) as x / (1 + e^(−2u)): nothing
// cancels for either sign of u, and CUDA's fast exponential and division keep the relative error
// near 2e-6, far below the rounding step of the 16-bit result (fp16 2.4e-4, bf16 2e-3). Limits:
// e^(−2u) overflows to +inf for x ≪ 0 and the quotient is 0; x → +inf gives x.
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return __fdividef(x, 1.0f + __expf(-2.0f * u));
}
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// L1 prefetch hint for an epilogue operand that is read later in the kernel
__device__ __forceinline__ void pf_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// a / b, correctly rounded, given rb = the correctly rounded reciprocal of b (__frcp_rn(b)):
// q0 = RN(a·rb) is within one ulp of a/b, the remainder a − q0·b is exact in one fma, and the
// corrected RN(q0 + rem·rb) equals RN(a/b) (Markstein's theorem; P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. R&D 34(1), 1990). Valid
// for normal, finite operands without overflow or underflow, i.e. the RMS-norm quotient x / den
// with den = sqrt(mean(x²) + eps) ≥ sqrt(eps). A zero, infinite or NaN first quotient (x = ±0,
// ±inf or NaN) is returned as it is, which keeps IEEE division's signed zero and specials. A few
// instructions instead of the general division sequence; pi0_div_check compares it with IEEE
// division bit for bit.
__device__ __forceinline__ float div_by_rcp(float a, float b, float rb) {
  const float q0 = __fmul_rn(a, rb);
  const float rem = fmaf(-q0, b, a);
  return (fabsf(q0) < INFINITY && q0 != 0.f) ? fmaf(rem, rb, q0) : q0;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace pi0
