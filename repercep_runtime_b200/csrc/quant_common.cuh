// Per-element steps of the bf16 / fp16 -> e4m3 quantizer, shared by the
// quantize kernels (quantize.cu) and the FP8 GEMM's fused-quantize epilogue
// (gemm.cu), so both produce the same bytes and scales.
//
// Semantics (bit-exact with the reference's eager PyTorch quantizer,
// kernels/triton_kernels/fp8_flash_attn_hopper.py:374-398):
//   amax   = max |x| over the scale group, taken in bf16 (NaN propagates)
//   amax   = max(amax, bf16(1e-6))                         (clamp in bf16)
//   scale  = bf16_rne(float(amax) / 425.6f)   -> dequant scale, stored f32
//   q_mul  = 1 / scale                          (IEEE round-to-nearest)
//   y      = clamp(float(x) * q_mul, -448, 448)
//   byte   = e4m3fn_rne(y)                      (NaN -> 0x7F | sign)
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "ptx.cuh"

namespace rp {
namespace quant {

constexpr float kScaleDiv = 425.6f;  // float(0.95 * 448)

// The two 16-bit input formats: bits -> float, the amax floor (the format's
// value nearest 1e-6), the +inf pattern, and RNE rounding of a float.
template <bool F16>
struct Fmt;
template <>
struct Fmt<false> {  // bf16
  static constexpr uint32_t kFloor = 0x3586u;
  static constexpr uint32_t kInf = 0x7F80u;
  __device__ static __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
  __device__ static __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
  __device__ static __forceinline__ float of(uint32_t bits) { return __uint_as_float(bits << 16); }
  __device__ static __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};
template <>
struct Fmt<true> {  // fp16
  static constexpr uint32_t kFloor = 0x0011u;
  static constexpr uint32_t kInf = 0x7C00u;
  __device__ static __forceinline__ float lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
  }
  __device__ static __forceinline__ float hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  }
  __device__ static __forceinline__ float of(uint32_t bits) { return lo(bits); }
  __device__ static __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
};

template <bool F16>
__device__ __forceinline__ float scale_from_amax_bits(uint32_t amax_bits) {
  using T = Fmt<F16>;
  uint32_t b = amax_bits;
  // Clamp to the floor; NaN (bits above +inf) is kept, like torch.clamp.
  if (b <= T::kInf && b < T::kFloor) b = T::kFloor;
  return T::round(__fdiv_rn(T::of(b), kScaleDiv));
}

__device__ __forceinline__ uint32_t quant_byte(float x, float qm) {
  float y = __fmul_rn(x, qm);
  y = (y > 448.f) ? 448.f : y;   // comparisons keep NaN
  y = (y < -448.f) ? -448.f : y;
  if (y != y) return 0x7Fu | ((__float_as_uint(y) >> 24) & 0x80u);
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3));
}

// 8 16-bit values (one 16-byte vector) -> 8 e4m3 bytes.
template <bool F16>
__device__ __forceinline__ uint2 quant8(uint4 v, float qm) {
  using T = Fmt<F16>;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t a = w[2 * i], b = w[2 * i + 1];
    const uint32_t b0 = quant_byte(T::lo(a), qm);
    const uint32_t b1 = quant_byte(T::hi(a), qm);
    const uint32_t b2 = quant_byte(T::lo(b), qm);
    const uint32_t b3 = quant_byte(T::hi(b), qm);
    o[i] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
  }
  return make_uint2(o[0], o[1]);
}

// quant8 for a finite scale, two elements per instruction: packed fp32
// multiply, then the paired e4m3 conversion, whose saturation is the clamp
// to +-448 (every |y| between 448 and 464 rounds to 448 as well).  With a
// finite scale no product is NaN (x is at most amax, and qm is finite and
// nonzero), so the bytes equal quant8's; a NaN or infinite amax (NaN
// products) takes quant8.
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
  const __nv_fp8x2_storage_t r = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE,
                                                          __NV_E4M3);
  return static_cast<uint32_t>(r);
}

template <bool F16>
__device__ __forceinline__ uint2 quant8_fast(uint4 v, float qm) {
  using T = Fmt<F16>;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const uint64_t q2 = pack_f32x2(qm, qm);
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float y0, y1;
    unpack_f32x2(fmul2(pack_f32x2(T::lo(w[i]), T::hi(w[i])), q2), y0, y1);
    h[i] = e4m3x2(y0, y1);
  }
  return make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
}

template <bool F16>
__device__ __forceinline__ uint2 quant8_any(uint4 v, float qm, bool fast) {
  return fast ? quant8_fast<F16>(v, qm) : quant8<F16>(v, qm);
}

// max of |x| bit patterns held in a 16-byte vector (bf16 and fp16 alike:
// non-negative values of both order like their bits, NaN above +inf).
__device__ __forceinline__ uint32_t absmax8(uint4 v) {
  uint32_t m = __vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu);
  m = __vmaxu2(m, v.z & 0x7FFF7FFFu);
  m = __vmaxu2(m, v.w & 0x7FFF7FFFu);
  return max(m & 0xFFFFu, m >> 16);
}

}  // namespace quant
}  // namespace rp
