// Register-level helpers of the fused attention kernels: byte packing,
// 3-input max, register reallocation, and the K-major shared-memory
// descriptor choice (packed f32x2 arithmetic is in common.cuh).  Included by
// attention.cu.
//
// Per-score arithmetic of the ExpCast encoders (no conversion-unit work):
//   float(raw) = as_float(raw + 0x4B400000) - 1.5*2^23    (exact, |raw| < 2^22)
//   u          = fma(logit-domain value, A, B)
//   byte       = sat_u8(bits(u * 2^-149))                    (RNE on the denormal grid)
#pragma once

// (c[15:0] << 16) | (sat_u8(a) << 8) | sat_u8(b), a and b read as s32.
__device__ __forceinline__ uint32_t pack_u8x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

constexpr float kBias = 12582912.0f;   // 1.5 * 2^23: the score preset, bits 0x4B400000

template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  if constexpr (D == 128) return smem_desc_sw128(saddr);
  else return smem_desc_sw64(saddr);
}
