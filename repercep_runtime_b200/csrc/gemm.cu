// FP8 (e4m3) GEMM for the DiT linears, sm_100a.
//
//   C[m, n] = out( acc[m, n] * (sa_m * sb_n) + bias[n] ),  acc[m, n] = sum_k A[m, k] * B(k, n)
//
// A is (M, K) e4m3 with K contiguous.  B is either (K, N) with N contiguous --
// the layout of the reference's proof-of-life kernel,
// kernels/hip/fp8_attn/fp8_gemm.hip:79-156 -- or (N, K) with K contiguous (an
// nn.Linear weight).  The accumulator is fp32.  sa_m / sb_n are per-row /
// per-column dequant scales or one scalar each; the reference's kernel is the
// scalar case, C = bf16(acc * (a_scale * b_scale)) (fp8_gemm.hip:145-153):
// the two scales are multiplied first, then the accumulator, then the bias is
// added (three fp32 roundings) and the sum is rounded to bf16 / fp16 (RNE).
//
// Kernel: persistent, one CTA per SM, 128 x 256 output tiles in a grouped
// raster (group_m row tiles share each column tile while it is hot in L2).
//   warp 0     TMA producer: per 128-byte K block an A box (128 rows) and a B
//              box (256 rows, K-major) or two (128 K rows x 128 N bytes,
//              N-major), 128-byte swizzle, into a 4-stage ring of 48 KB;
//   warp 1     MMA issuer (one thread): four tcgen05.mma kind::f8f6f4 M128
//              N256 K32 per stage into one of two TMEM accumulators (2 x 256
//              columns), so tile t+1's MMAs run while the epilogue drains t;
//   warps 2-9  epilogue: two warps per TMEM lane quarter, one per 128-column
//              half; each stages its columns' scales and bias in its own slice
//              of shared memory before the accumulator is ready, then
//              tcgen05.ld 2 x 32 columns in flight, scale, bias, round,
//              16-byte global stores (each thread owns one row).
// K, M and N tails need no special case: the TMA unit fills out-of-range box
// elements with zeros (they add nothing to acc) and the epilogue masks rows
// and columns past M and N.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "internal.h"
#include "ptx.cuh"

namespace rp {

namespace {

constexpr int kBM = 128;  // output rows per tile (TMEM lanes)
constexpr int kBN = 256;  // output columns per tile (TMEM columns per accumulator)
constexpr int kBK = 128;  // K bytes per stage (one 128-byte swizzle row)
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK;                 // 16 KB
constexpr int kBBytes = kBN * kBK;                 // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;     // 48 KB
constexpr int kHalfB = kBBytes / 2;                // one 128-column N-major box
constexpr int kTmaWarp = 0, kMmaWarp = 1;          // warps 2..9: epilogue
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kEpiCols = kBN / 2;                  // columns per epilogue warp
constexpr int kTmemCols = 2 * kBN;                 // two accumulators
// Per epilogue warp: kEpiCols column scales then kEpiCols bias values (fp32).
constexpr int kOffCol = kStages * kStageBytes;
constexpr int kColBytes = kEpiWarps * 2 * kEpiCols * 4;
constexpr int kOffBar = kOffCol + kColBytes;
constexpr int kNumBars = 2 * kStages + 2 + 2 + 1;  // full, empty, acc_full, acc_empty, fin
constexpr int kSmemBytes = 1024 + kOffBar + kNumBars * 8 + 16;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

enum : int {
  kErrGemmFull = 0x201,
  kErrGemmEmpty = 0x202,
  kErrGemmAccFull = 0x203,
  kErrGemmAccEmpty = 0x204,
};

struct GemmBars {
  uint64_t* full;       // [kStages] TMA bytes landed
  uint64_t* empty;      // [kStages] MMAs reading the stage are done
  uint64_t* acc_full;   // [2] accumulator complete (commit after a tile's last MMA)
  uint64_t* acc_empty;  // [2] epilogue has read the accumulator (one arrive per warp)
  uint64_t* fin;        // every MMA of this CTA done (teardown)
  volatile int* abort_flag;
  uint32_t* tmem_slot;
};

__device__ __forceinline__ GemmBars carve_gemm_bars(uint8_t* s) {
  uint64_t* b = reinterpret_cast<uint64_t*>(s);
  GemmBars r;
  r.full = b;
  r.empty = b + kStages;
  r.acc_full = b + 2 * kStages;
  r.acc_empty = r.acc_full + 2;
  r.fin = r.acc_empty + 2;
  r.abort_flag = reinterpret_cast<volatile int*>(b + kNumBars);
  r.tmem_slot = reinterpret_cast<uint32_t*>(b + kNumBars) + 1;
  return r;
}

__device__ __forceinline__ void drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles / 4) return;
  }
}

struct TileCoord {
  int m, n;
};

// Tile t of the grouped raster: group_m row tiles (M fastest) per column tile.
__device__ __forceinline__ TileCoord tile_coord(const GemmParams& p, int t) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group;
  const int first = g * p.group_m;
  const int rows = min(p.group_m, p.tiles_m - first);
  const int r = t - g * per_group;
  return {first + r % rows, r / rows};
}

template <bool BKM>
__device__ void gemm_producer(const CUtensorMap* ta, const CUtensorMap* tb, const GemmParams& p,
                              const GemmBars& bar, uint8_t* smem) {
  int g = 0;
  bool ok = true;
  for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x) {
    const TileCoord c = tile_coord(p, t);
    for (int kb = 0; kb < p.n_kb; ++kb, ++g) {
      const int s = g % kStages;
      if (!mbar_wait(bar.empty + s, ((g / kStages) & 1) ^ 1, bar.abort_flag, p.status,
                     kErrGemmEmpty)) {
        ok = false;
        break;
      }
      uint8_t* sa = smem + s * kStageBytes;
      uint8_t* sb = sa + kABytes;
      mbar_arrive_expect_tx(bar.full + s, kStageBytes);
      tma_load_4d(sa, ta, bar.full + s, kb * kBK, c.m * kBM, 0, 0);
      if constexpr (BKM) {
        tma_load_4d(sb, tb, bar.full + s, kb * kBK, c.n * kBN, 0, 0);
      } else {
        tma_load_4d(sb, tb, bar.full + s, c.n * kBN, kb * kBK, 0, 0);
        tma_load_4d(sb + kHalfB, tb, bar.full + s, c.n * kBN + 128, kb * kBK, 0, 0);
      }
    }
  }
  if (!ok) {
    // Loads still in flight write this CTA's shared memory: let them land.
    for (int s = 0; s < kStages; ++s) {
      if (s >= g) break;
      const int last = g - 1 - ((g - 1 - s) % kStages);  // last fill of stage s
      drain(bar.full + s, (last / kStages) & 1);
    }
  }
}

template <bool BKM>
__device__ void gemm_mma(const GemmParams& p, const GemmBars& bar, uint32_t sbase,
                         uint32_t tmem) {
  constexpr uint32_t idesc = make_idesc_e4m3(kBM, kBN, 0, BKM ? 0 : 1);
  int g = 0, it = 0;
  bool ok = true;
  for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++it) {
    const int buf = it & 1;
    if (!mbar_wait(bar.acc_empty + buf, ((it >> 1) & 1) ^ 1, bar.abort_flag, p.status,
                   kErrGemmAccEmpty)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t d = tmem + buf * kBN;
    for (int kb = 0; kb < p.n_kb; ++kb, ++g) {
      const int s = g % kStages;
      if (!mbar_wait(bar.full + s, (g / kStages) & 1, bar.abort_flag, p.status, kErrGemmFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a_addr = sbase + s * kStageBytes;
      const uint64_t ad = make_sw128_desc(a_addr, 16, 1024);
      // K-major B: 8-row groups 1024 B apart, K step 32 B.  N-major B: the
      // two 128-column boxes kHalfB apart (LBO), 8-K-row groups 1024 B apart
      // (SBO), K step 32 rows = 4096 B.
      const uint64_t bd = BKM ? make_sw128_desc(a_addr + kABytes, 16, 1024)
                              : make_sw128_desc(a_addr + kABytes, kHalfB, 1024);
#pragma unroll
      for (int k = 0; k < kBK / 32; ++k)
        mma_f8(d, ad + 2 * k, bd + (BKM ? 2 * k : 256 * k), idesc, (kb | k) ? 1u : 0u);
      mma_commit(bar.empty + s);
    }
    if (!ok) break;
    mma_commit(bar.acc_full + buf);
  }
  // Everything this thread issued must finish before TMEM is released.
  mma_commit(bar.fin);
  drain(bar.fin, 0);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool f16) {
  if (f16) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}

__device__ __forceinline__ float bias_at(const uint16_t* bias, int n, bool f16) {
  const uint16_t b = bias[n];
  return f16 ? __half2float(__ushort_as_half(b)) : __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Scale, bias and round 32 accumulator columns of one row and store them.
// cs / cb: this chunk's 32 column scales / bias values in shared memory.
template <bool F16OUT>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, const uint32_t (&r)[32],
                                               const float* cs, const float* cb, float sa,
                                               bool col_scale, bool has_bias, uint16_t* crow,
                                               int n0) {
  const bool full = (n0 + 32 <= p.N);
  const uint64_t sa2 = pack_f32x2(sa, sa);
  const uint64_t sb2 = pack_f32x2(p.b_scale, p.b_scale);
  uint32_t o[16];
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    float4 sc = make_float4(0.f, 0.f, 0.f, 0.f), bi = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col_scale) sc = *reinterpret_cast<const float4*>(cs + j);
    if (has_bias) bi = *reinterpret_cast<const float4*>(cb + j);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // s = sa * sb, y = acc * s, y += bias: three fp32 roundings, in that order
      const uint64_t s2 =
          col_scale ? fmul2(sa2, h ? pack_f32x2(sc.z, sc.w) : pack_f32x2(sc.x, sc.y))
                    : fmul2(sa2, sb2);
      uint64_t y2 = fmul2(
          pack_f32x2(__uint_as_float(r[j + 2 * h]), __uint_as_float(r[j + 2 * h + 1])), s2);
      if (has_bias) y2 = fadd2(y2, h ? pack_f32x2(bi.z, bi.w) : pack_f32x2(bi.x, bi.y));
      float y0, y1;
      unpack_f32x2(y2, y0, y1);
      o[j / 2 + h] = pack2(y0, y1, F16OUT);
    }
  }
  if (full && p.vec_store) {
    uint4* dst = reinterpret_cast<uint4*>(crow + n0);
#pragma unroll
    for (int v = 0; v < 4; ++v)
      dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < p.N) crow[n0 + j] = static_cast<uint16_t>(o[j / 2] >> (16 * (j & 1)));
  }
}

template <bool F16OUT>
__device__ void gemm_epilogue(const GemmParams& p, const GemmBars& bar, uint32_t tmem,
                              float* colbuf) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ew = warp - 2;                // epilogue warp 0..7
  const int q = warp & 3;                 // TMEM lane quarter this warp may access
  const int half = ew / 4;                // column half of the tile
  const bool col_scale = p.sb != nullptr, has_bias = p.bias != nullptr;
  float* cs = colbuf + ew * 2 * kEpiCols;  // this warp's column scales, then bias
  float* cb = cs + kEpiCols;
  int it = 0;
  for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++it) {
    const int buf = it & 1;
    const TileCoord c = tile_coord(p, t);
    const int ncol0 = c.n * kBN + half * kEpiCols;
    // Column data for this tile, fetched while the MMAs run (the previous
    // tile's reads of this slice are done: same warp, program order).
    if (col_scale || has_bias) {
      __syncwarp();
#pragma unroll
      for (int i = 0; i < kEpiCols / 32; ++i) {
        const int n = ncol0 + i * 32 + lane;
        const bool in = n < p.N;
        if (col_scale) cs[i * 32 + lane] = in ? __ldg(p.sb + (int64_t)n * p.sb_stride) : 0.f;
        if (has_bias) cb[i * 32 + lane] = in ? bias_at(p.bias, n, F16OUT) : 0.f;
      }
      __syncwarp();
    }
    const int m = c.m * kBM + q * 32 + lane;
    const bool row_ok = m < p.M;
    const float sa = p.sa ? (row_ok ? __ldg(p.sa + (int64_t)m * p.sa_stride) : 0.f) : p.a_scale;
    uint16_t* crow = static_cast<uint16_t*>(p.C) + (int64_t)(row_ok ? m : 0) * p.ldc;
    if (!mbar_wait(bar.acc_full + buf, (it >> 1) & 1, bar.abort_flag, p.status, kErrGemmAccFull))
      return;
    tc_fence_after();
    const uint32_t taddr =
        tmem + buf * kBN + half * kEpiCols + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
    for (int pr = 0; pr < kEpiCols / 64; ++pr) {
      uint32_t r0[32], r1[32];
      if (p.n_kb > 0) {
        tmem_ld32(taddr + pr * 64, r0);
        tmem_ld32(taddr + pr * 64 + 32, r1);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r0[j] = r1[j] = 0u;
      }
      if (pr == kEpiCols / 64 - 1) {
        // The accumulator may be overwritten once every warp's loads are done.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar.acc_empty + buf);
      }
      const int n0 = ncol0 + pr * 64;
      if (row_ok && n0 < p.N)
        epilogue_chunk<F16OUT>(p, r0, cs + pr * 64, cb + pr * 64, sa, col_scale, has_bias, crow,
                               n0);
      if (row_ok && n0 + 32 < p.N)
        epilogue_chunk<F16OUT>(p, r1, cs + pr * 64 + 32, cb + pr * 64 + 32, sa, col_scale,
                               has_bias, crow, n0 + 32);
    }
  }
}

template <bool BKM, bool F16OUT>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_b, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const GemmBars bar = carve_gemm_bars(smem + kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar.full + s, 1);
      mbar_init(bar.empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar.acc_full + b, 1);
      mbar_init(bar.acc_empty + b, kEpiWarps);
    }
    mbar_init(bar.fin, 1);
    *bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(bar.tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0 && p.n_kb > 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tmem_slot;

  if (warp == kTmaWarp) {
    if (lane == 0) gemm_producer<BKM>(&tm_a, &tm_b, p, bar, smem);
  } else if (warp == kMmaWarp) {
    if (lane == 0) gemm_mma<BKM>(p, bar, smem_u32(smem), tmem);
  } else {
    gemm_epilogue<F16OUT>(p, bar, tmem, reinterpret_cast<float*>(smem + kOffCol));
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool BKM, bool F16OUT>
cudaError_t launch_gemm_variant(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p,
                                int grid, cudaStream_t st) {
  auto kern = fp8_gemm_kernel<BKM, F16OUT>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_release);
  }
  kern<<<grid, kThreads, kSmemBytes, st>>>(a, b, p);
  return cudaGetLastError();
}

int sm_count() {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace

int gemm_tile_m() { return kBM; }
int gemm_tile_n() { return kBN; }

cudaError_t launch_fp8_gemm(const CUtensorMap& a, const CUtensorMap& b, GemmParams p,
                            bool b_kmajor, bool out_f16, cudaStream_t st) {
  p.tiles_m = (p.M + kBM - 1) / kBM;
  p.tiles_n = (p.N + kBN - 1) / kBN;
  p.tiles = p.tiles_m * p.tiles_n;
  p.n_kb = (p.K + kBK - 1) / kBK;
  if (p.group_m <= 0) p.group_m = 16;
  if (p.group_m > p.tiles_m) p.group_m = p.tiles_m;
  const int grid = p.tiles < sm_count() ? p.tiles : sm_count();
  if (b_kmajor)
    return out_f16 ? launch_gemm_variant<true, true>(a, b, p, grid, st)
                   : launch_gemm_variant<true, false>(a, b, p, grid, st);
  return out_f16 ? launch_gemm_variant<false, true>(a, b, p, grid, st)
                 : launch_gemm_variant<false, false>(a, b, p, grid, st);
}

}  // namespace rp
