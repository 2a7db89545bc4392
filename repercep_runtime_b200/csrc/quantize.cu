// bf16 -> e4m3 quantization with amax scales.
//
// Semantics (bit-exact with the reference's eager PyTorch quantizer,
// kernels/triton_kernels/fp8_flash_attn_hopper.py:374-398):
//   amax   = max |x| over the scale group, taken in bf16 (NaN propagates)
//   amax   = max(amax, bf16(1e-6))                         (clamp in bf16)
//   scale  = bf16_rne(float(amax) / 425.6f)   -> dequant scale, stored f32
//   q_mul  = 1 / scale                          (IEEE round-to-nearest)
//   y      = clamp(float(x) * q_mul, -448, 448)
//   byte   = e4m3fn_rne(y)                      (NaN -> 0x7F | sign)
// 425.6f is float(0.95 * 448).  For every bf16 amax, the fp32 quotient and
// the fp32 product with the rounded reciprocal (PyTorch's CUDA path) round
// to the same bf16, so one formula covers both of the reference's devices.
//
// Scale groups: one per (b,h) (the reference) or one per 128-token block of
// each (b,h) (the per-block extension; the last block of a ragged S is short).
//
// fp16 inputs follow the same steps in fp16: amax and its 1e-6 floor in fp16
// (fp16(1e-6) = 0x0011, a subnormal), scale = fp16_rne(float(amax)/425.6f).
//
// The input is read through arbitrary (b,h,s) element strides with d
// unit-stride, so BHSD and BSHD (diffusers) tensors need no transposing copy.
// Output rows are out_ld bytes apart (out_ld >= D; bytes D..out_ld-1 of every
// row are written as zero), rows contiguous: (B*H, S, out_ld).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "internal.h"
#include "ptx.cuh"
#include "quant_common.cuh"

namespace rp {

namespace {

using namespace quant;

__device__ __forceinline__ uint32_t block_max(uint32_t v, uint32_t* red) {
  v = __reduce_max_sync(0xffffffffu, v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < kQuantThreads / 32; ++i) m = max(m, red[i]);
  return m;
}

// One CTA = one 128-token block of one (b,h) of one job.  D/8 vectors per
// row, 128 rows: each thread holds D/16 vectors in registers.
template <int D, bool F16>
struct BlockTile {
  static constexpr int kVpr = D / 8;
  static constexpr int kPer = kQuantRows * kVpr / kQuantThreads;
  uint4 v[kPer];

  __device__ __forceinline__ uint32_t load(const QuantJob& j, int b, int h, int s0, int rows) {
    const uint16_t* base = j.x + b * j.sB + h * j.sH;
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int idx = threadIdx.x + k * kQuantThreads;
      const int r = idx / kVpr, c = idx % kVpr;
      if (r < rows) {
        v[k] = __ldcs(reinterpret_cast<const uint4*>(base + (int64_t)(s0 + r) * j.sS + c * 8));
        m = max(m, absmax8(v[k]));
      } else {
        v[k] = make_uint4(0, 0, 0, 0);
      }
    }
    return m;
  }

  __device__ __forceinline__ void store(const QuantJob& j, int bh, int S, int ld, int s0,
                                        int rows, float sc) {
    uint8_t* out = j.out + ((int64_t)bh * S + s0) * ld;
    const float qm = __frcp_rn(sc);
    const bool fast = isfinite(sc);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int idx = threadIdx.x + k * kQuantThreads;
      const int r = idx / kVpr, c = idx % kVpr;
      if (r < rows)
        __stcs(reinterpret_cast<uint2*>(out + (int64_t)r * ld + c * 8),
               quant8_any<F16>(v[k], qm, fast));
    }
    // zero padding of rows wider than D
    const int pad = (ld - D) / 8;
    for (int idx = threadIdx.x; idx < rows * pad; idx += kQuantThreads) {
      const int r = idx / pad, c = idx % pad;
      __stcs(reinterpret_cast<uint2*>(out + (int64_t)r * ld + D + c * 8), make_uint2(0, 0));
    }
  }
};

template <int D, bool F16>
__global__ void __launch_bounds__(kQuantThreads) quant_block_kernel(const QuantArgs a) {
  // A dependent kernel (the shared-prefix decode) may start its prologue now;
  // it waits for this grid's completion before reading what it writes.
  griddep_launch();
  __shared__ uint32_t red[kQuantThreads / 32];
  const QuantJob& j = a.job[blockIdx.z];
  const int blk = blockIdx.x, bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int s0 = blk * kQuantRows;
  const int rows = min(kQuantRows, a.S - s0);
  BlockTile<D, F16> t;
  const uint32_t m = block_max(t.load(j, b, h, s0, rows), red);
  const float sc = scale_from_amax_bits<F16>(m);
  if (threadIdx.x == 0) j.scales[(int64_t)bh * a.nblk + blk] = sc;
  t.store(j, bh, a.S, a.out_ld, s0, rows, sc);
}

// Per-(b,h) pass 1: partial amax of one 128-row chunk.
template <int D, bool F16>
__global__ void __launch_bounds__(kQuantThreads) amax_chunk_kernel(const QuantArgs a) {
  __shared__ uint32_t red[kQuantThreads / 32];
  const QuantJob& j = a.job[blockIdx.z];
  const int blk = blockIdx.x, bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int s0 = blk * kQuantRows;
  const int rows = min(kQuantRows, a.S - s0);
  const uint16_t* base = j.x + b * j.sB + h * j.sH;
  constexpr int kVpr = D / 8;
  uint32_t m = 0;
  for (int idx = threadIdx.x; idx < rows * kVpr; idx += kQuantThreads) {
    const int r = idx / kVpr, c = idx % kVpr;
    m = max(m, absmax8(__ldg(reinterpret_cast<const uint4*>(base + (int64_t)(s0 + r) * j.sS + c * 8))));
  }
  m = block_max(m, red);
  if (threadIdx.x == 0)
    a.partial[((int64_t)blockIdx.z * gridDim.y + bh) * a.npart + blk] = m;
}

// Per-(b,h) pass 2: reduce the npart partials of this (b,h), quantize one chunk.
template <int D, bool F16>
__global__ void __launch_bounds__(kQuantThreads) quant_bh_kernel(const QuantArgs a) {
  __shared__ uint32_t red[kQuantThreads / 32];
  const QuantJob& j = a.job[blockIdx.z];
  const int blk = blockIdx.x, bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const uint32_t* part = a.partial + ((int64_t)blockIdx.z * gridDim.y + bh) * a.npart;
  uint32_t m = 0;
  for (int i = threadIdx.x; i < a.npart; i += kQuantThreads) m = max(m, part[i]);
  m = block_max(m, red);
  const float sc = scale_from_amax_bits<F16>(m);
  if (blk == 0 && threadIdx.x == 0) j.scales[bh] = sc;
  const int s0 = blk * kQuantRows;
  const int rows = min(kQuantRows, a.S - s0);
  BlockTile<D, F16> t;
  t.load(j, b, h, s0, rows);
  t.store(j, bh, a.S, a.out_ld, s0, rows, sc);
}

// Row-wise scales for the linear operands: one scale group per row of an
// (rows, cols) matrix (a token of the activations, an output channel of a
// weight), with the steps above.  TPR threads share a row and hold it in
// registers (VPT 16-byte vectors each, all loads in flight at once), so the
// row is read from HBM once and quantized from registers.
template <bool F16, int TPR, int VPT>
__global__ void __launch_bounds__(kQuantThreads) quant_rows_kernel(const QuantRowsArgs a) {
  static_assert(TPR % 32 == 0 && kQuantThreads % TPR == 0, "whole warps per row");
  constexpr int kWarpsPerRow = TPR / 32;
  __shared__ uint32_t red[kQuantThreads / 32];
  const int grp = threadIdx.x / TPR, t = threadIdx.x % TPR;
  const int64_t row = (int64_t)blockIdx.x * (kQuantThreads / TPR) + grp;
  const bool live = row < a.rows;
  const int nv = a.cols / 8;
  const uint4* x = reinterpret_cast<const uint4*>(a.x + (live ? row : 0) * a.ldx);
  uint4 v[VPT];
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = t + i * TPR;
    v[i] = (live && idx < nv) ? __ldcs(x + idx) : make_uint4(0, 0, 0, 0);
    m = max(m, absmax8(v[i]));
  }
  m = __reduce_max_sync(0xffffffffu, m);
  if constexpr (kWarpsPerRow > 1) {
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = m;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kWarpsPerRow; ++w) m = max(m, red[grp * kWarpsPerRow + w]);
  }
  if (!live) return;
  const float sc = scale_from_amax_bits<F16>(m);
  if (t == 0) a.scales[row] = sc;
  const float qm = __frcp_rn(sc);
  const bool fast = isfinite(sc);
  uint2* o = reinterpret_cast<uint2*>(a.out + row * a.ldo);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = t + i * TPR;
    if (idx < nv) __stcs(o + idx, quant8_any<F16>(v[i], qm, fast));
  }
}

// Rows longer than the register-resident forms hold: one warp per row, the
// second pass re-reads the row (from L2).
template <bool F16>
__global__ void __launch_bounds__(kQuantThreads) quant_long_rows_kernel(const QuantRowsArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kQuantThreads / 32) + warp;
  if (row >= a.rows) return;
  const uint4* x = reinterpret_cast<const uint4*>(a.x + row * a.ldx);
  const int nv = a.cols / 8;
  uint32_t m = 0;
  for (int i = lane; i < nv; i += 32) m = max(m, absmax8(__ldg(x + i)));
  m = __reduce_max_sync(0xffffffffu, m);
  const float sc = scale_from_amax_bits<F16>(m);
  if (lane == 0) a.scales[row] = sc;
  const float qm = __frcp_rn(sc);
  const bool fast = isfinite(sc);
  uint2* o = reinterpret_cast<uint2*>(a.out + row * a.ldo);
  for (int i = lane; i < nv; i += 32) __stcs(o + i, quant8_any<F16>(__ldg(x + i), qm, fast));
}

template <bool F16, int TPR, int VPT>
cudaError_t launch_rows_t(const QuantRowsArgs& a, cudaStream_t st) {
  constexpr int kRowsPerCta = kQuantThreads / TPR;
  const int64_t grid = (a.rows + kRowsPerCta - 1) / kRowsPerCta;
  if (grid > 0x7FFFFFFF) return cudaErrorInvalidValue;
  quant_rows_kernel<F16, TPR, VPT><<<static_cast<unsigned>(grid), kQuantThreads, 0, st>>>(a);
  return cudaGetLastError();
}

template <bool F16>
cudaError_t launch_rows_f(const QuantRowsArgs& a, cudaStream_t st) {
  const int nv = a.cols / 8;  // 16-byte vectors per row
  if (nv <= 32 * 4) return launch_rows_t<F16, 32, 4>(a, st);      // cols <= 1024
  if (nv <= 128 * 4) return launch_rows_t<F16, 128, 4>(a, st);    // cols <= 4096
  if (nv <= 256 * 8) return launch_rows_t<F16, 256, 8>(a, st);    // cols <= 16384
  if (nv <= 256 * 16) return launch_rows_t<F16, 256, 16>(a, st);  // cols <= 32768
  const int64_t grid = (a.rows + kQuantThreads / 32 - 1) / (kQuantThreads / 32);
  if (grid > 0x7FFFFFFF) return cudaErrorInvalidValue;
  quant_long_rows_kernel<F16><<<static_cast<unsigned>(grid), kQuantThreads, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quant_rows(const QuantRowsArgs& a, cudaStream_t st) {
  return a.in_f16 ? launch_rows_f<true>(a, st) : launch_rows_f<false>(a, st);
}

#define RP_DISPATCH_DF(KERNEL, F16)                                               \
  switch (a.D) {                                                                     \
    case 32: KERNEL<32, F16><<<grid, kQuantThreads, 0, st>>>(a); break;             \
    case 64: KERNEL<64, F16><<<grid, kQuantThreads, 0, st>>>(a); break;             \
    case 128: KERNEL<128, F16><<<grid, kQuantThreads, 0, st>>>(a); break;           \
    case 256: KERNEL<256, F16><<<grid, kQuantThreads, 0, st>>>(a); break;           \
    default: return cudaErrorInvalidValue;                                           \
  }
#define RP_DISPATCH_D(KERNEL)        \
  if (a.in_f16) {                    \
    RP_DISPATCH_DF(KERNEL, true)     \
  } else {                           \
    RP_DISPATCH_DF(KERNEL, false)    \
  }

cudaError_t launch_quant_block(const QuantArgs& a, int njobs, cudaStream_t st) {
  const dim3 grid(a.nblk, a.B * a.H, njobs);
  RP_DISPATCH_D(quant_block_kernel)
  return cudaGetLastError();
}

cudaError_t launch_quant_bh(const QuantArgs& a, int njobs, cudaStream_t st, int phases) {
  const dim3 grid(a.nblk, a.B * a.H, njobs);
  if (phases & 1) {
    RP_DISPATCH_D(amax_chunk_kernel)
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (phases & 2) {
    RP_DISPATCH_D(quant_bh_kernel)
  }
  return cudaGetLastError();
}

#undef RP_DISPATCH_D

}  // namespace rp
