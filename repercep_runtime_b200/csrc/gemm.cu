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
// Kernel: persistent, 256 x 256 output tiles in a grouped raster (group_m
// row tiles share each column tile while it is hot in L2), one tile per pair
// of CTAs on the two SMs of a TPC (a cluster of 2):
//   warp 0     TMA producer: per 128-byte K block this CTA's 128 A rows and
//              128 B rows (K-major) or columns (N-major), 128-byte swizzle,
//              into a 6-stage ring of 32 KB; the bytes of both CTAs complete
//              on rank 0's barrier;
//   warp 1     MMA issuer (one thread of rank 0): four tcgen05.mma
//              cta_group::2 kind::f8f6f4 M256 N256 K32 per stage, reading
//              both CTAs' shared memory, into one of two accumulators (2 x
//              256 TMEM columns in each CTA: its 128 rows), so tile t+1's MMAs
//              run while the epilogue drains t;
//   warps 2-9  epilogue (both CTAs): two warps per TMEM lane quarter, one per
//              128-column half; each stages its columns' scales and bias in
//              its own slice of shared memory before the accumulator is ready,
//              then tcgen05.ld 2 x 32 columns in flight, scale, bias, round,
//              16-byte global stores (each thread owns one row).
// Splitting B across the pair halves what each SM pulls from L2 per MMA
// (32 KB instead of 48 KB per 128-deep K block).  REPERCEP_B200_GEMM_PAIR=0
// selects the single-CTA form: 128 x 256 tiles, one CTA per SM, a 4-stage
// ring of 48 KB (A 128 rows, B 256).
// K, M and N tails need no special case: the TMA unit fills out-of-range box
// elements with zeros (they add nothing to acc) and the epilogue masks rows
// and columns past M and N.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <cstdlib>

#include "internal.h"
#include "ptx.cuh"
#include "quant_common.cuh"

namespace rp {

namespace {

constexpr int kBK = 128;  // K bytes per stage (one 128-byte swizzle row)
constexpr int kCtaRows = 128;  // A rows (TMEM lanes) per CTA
constexpr int kTileN = 256;    // output columns per tile (TMEM columns per accumulator)
constexpr int kABytes = kCtaRows * kBK;  // 16 KB
constexpr int kTmaWarp = 0, kMmaWarp = 1;  // warps 2..9: epilogue
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kEpiCols = kTileN / 2;       // columns per epilogue warp
constexpr int kTmemCols = 2 * kTileN;      // two accumulators
// Per epilogue warp: kEpiCols column scales then kEpiCols bias values (fp32).
constexpr int kColBytes = kEpiWarps * 2 * kEpiCols * 4;

template <bool PAIR>
struct GCfg {
  static constexpr int kTileM = PAIR ? 2 * kCtaRows : kCtaRows;  // output rows per tile
  static constexpr int kBRows = PAIR ? kTileN / 2 : kTileN;      // B rows (N) per CTA
  static constexpr int kBBytes = kBRows * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;           // 32 / 48 KB
  static constexpr int kStages = PAIR ? 6 : 4;
  static constexpr int kOffCol = kStages * kStageBytes;
  // fused QKV quantize: per-warp block amax, [2 tile parities][2 halves][4 lane quarters]
  static constexpr int kOffAmax = kOffCol + kColBytes;
  static constexpr int kOffBar = kOffAmax + 2 * 2 * 4 * 4;
  static constexpr int kNumBars = 2 * kStages + 2 + 2 + 1;  // full, empty, acc_full, acc_empty, fin
  static constexpr int kSmemBytes = 1024 + kOffBar + kNumBars * 8 + 16;
  // acc_empty arrivals: every epilogue warp of the pair
  static constexpr int kAccEmptyCount = (PAIR ? 2 : 1) * kEpiWarps;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

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

template <bool PAIR>
__device__ __forceinline__ GemmBars carve_gemm_bars(uint8_t* s) {
  constexpr int kStages = GCfg<PAIR>::kStages, kNumBars = GCfg<PAIR>::kNumBars;
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

// Tile loop position of this CTA (PAIR: of its pair).
template <bool PAIR>
__device__ __forceinline__ int tile_unit() {
  return PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
}
template <bool PAIR>
__device__ __forceinline__ int tile_units() {
  return PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
}

// First A row of this CTA's part of row tile cm: tiles in row order, or (fused
// QKV quantize) per batch -- the tile's rows within its batch of qkv_S tokens,
// offset by the batch (rows past the batch are masked by the epilogue).
template <bool PAIR>
__device__ __forceinline__ int tile_row0(const GemmParams& p, int cm, uint32_t rank) {
  using C = GCfg<PAIR>;
  if (p.qkv_S > 0) {
    const int b = cm / p.qkv_per_b;
    return b * p.qkv_S + (cm - b * p.qkv_per_b) * C::kTileM + static_cast<int>(rank) * kCtaRows;
  }
  return cm * C::kTileM + static_cast<int>(rank) * kCtaRows;
}

template <bool PAIR>
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, const GemmBars& b,
                                         int* status, int code) {
  return PAIR ? mbar_wait_cluster(bar, parity, b.abort_flag, status, code)
              : mbar_wait(bar, parity, b.abort_flag, status, code);
}

template <bool PAIR, bool BKM>
__device__ void gemm_producer(const CUtensorMap* ta, const CUtensorMap* tb, const GemmParams& p,
                              const GemmBars& bar, uint8_t* smem, uint32_t rank) {
  using C = GCfg<PAIR>;
  int g = 0;
  bool ok = true;
  for (int t = tile_unit<PAIR>(); ok && t < p.tiles; t += tile_units<PAIR>()) {
    const TileCoord c = tile_coord(p, t);
    const int m0 = tile_row0<PAIR>(p, c.m, rank);
    const int n0 = c.n * kTileN + static_cast<int>(rank) * C::kBRows;
    for (int kb = 0; kb < p.n_kb; ++kb, ++g) {
      const int s = g % C::kStages;
      if (!wait_bar<PAIR>(bar.empty + s, ((g / C::kStages) & 1) ^ 1, bar, p.status,
                          kErrGemmEmpty)) {
        ok = false;
        break;
      }
      uint8_t* sa = smem + s * C::kStageBytes;
      uint8_t* sb = sa + kABytes;
      if constexpr (PAIR) {
        // Both CTAs' bytes complete on rank 0's barrier, which rank 0 arms.
        if (rank == 0) mbar_arrive_expect_tx(bar.full + s, 2 * C::kStageBytes);
        const uint32_t fb = mapa_shared(smem_u32(bar.full + s), 0);
        tma_load_4d_pair(sa, ta, fb, kb * kBK, m0, 0, 0);
        if constexpr (BKM)
          tma_load_4d_pair(sb, tb, fb, kb * kBK, n0, 0, 0);
        else
          tma_load_4d_pair(sb, tb, fb, n0, kb * kBK, 0, 0);
      } else {
        mbar_arrive_expect_tx(bar.full + s, C::kStageBytes);
        tma_load_4d(sa, ta, bar.full + s, kb * kBK, m0, 0, 0);
        if constexpr (BKM) {
          tma_load_4d(sb, tb, bar.full + s, kb * kBK, n0, 0, 0);
        } else {
          tma_load_4d(sb, tb, bar.full + s, n0, kb * kBK, 0, 0);
          tma_load_4d(sb + C::kBBytes / 2, tb, bar.full + s, n0 + 128, kb * kBK, 0, 0);
        }
      }
    }
  }
  if (!ok) {
    // Loads still in flight write this CTA's shared memory: let them land.
    if (PAIR && rank != 0) {
      // (their bytes complete on rank 0's barriers): a fixed grace period
      const long long t0 = clock64();
      while (clock64() - t0 < 2000000) {
      }
    } else {
      for (int s = 0; s < C::kStages; ++s) {
        if (s >= g) break;
        const int last = g - 1 - ((g - 1 - s) % C::kStages);  // last fill of stage s
        drain(bar.full + s, (last / C::kStages) & 1);
      }
    }
  }
}

// Signals `bar` (same offset in both CTAs for PAIR) when the MMAs issued so
// far are done.
template <bool PAIR>
__device__ __forceinline__ void commit_both(uint64_t* bar) {
  if constexpr (PAIR) {
    mma_commit_pair_to(bar, 0x3);
  } else {
    mma_commit(bar);
  }
}

template <bool PAIR, bool BKM>
__device__ void gemm_mma(const GemmParams& p, const GemmBars& bar, uint32_t sbase,
                         uint32_t tmem) {
  using C = GCfg<PAIR>;
  constexpr uint32_t idesc = make_idesc_e4m3(C::kTileM, kTileN, 0, BKM ? 0 : 1);
  int g = 0, it = 0;
  bool ok = true;
  for (int t = tile_unit<PAIR>(); ok && t < p.tiles; t += tile_units<PAIR>(), ++it) {
    const int buf = it & 1;
    if (!wait_bar<PAIR>(bar.acc_empty + buf, ((it >> 1) & 1) ^ 1, bar, p.status,
                        kErrGemmAccEmpty)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t d = tmem + buf * kTileN;
    for (int kb = 0; kb < p.n_kb; ++kb, ++g) {
      const int s = g % C::kStages;
      if (!wait_bar<PAIR>(bar.full + s, (g / C::kStages) & 1, bar, p.status, kErrGemmFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a_addr = sbase + s * C::kStageBytes;
      const uint64_t ad = make_sw128_desc(a_addr, 16, 1024);
      // K-major B: 8-row groups 1024 B apart, K step 32 B.  N-major B: 128-
      // column boxes C::kBBytes / 2 apart (LBO; one box per CTA when PAIR),
      // 8-K-row groups 1024 B apart (SBO), K step 32 rows = 4096 B.
      const uint64_t bd = BKM ? make_sw128_desc(a_addr + kABytes, 16, 1024)
                              : make_sw128_desc(a_addr + kABytes, C::kBBytes / 2, 1024);
#pragma unroll
      for (int k = 0; k < kBK / 32; ++k) {
        const uint64_t bk = bd + (BKM ? 2 * k : 256 * k);
        if constexpr (PAIR)
          mma_f8_pair(d, ad + 2 * k, bk, idesc, (kb | k) ? 1u : 0u);
        else
          mma_f8(d, ad + 2 * k, bk, idesc, (kb | k) ? 1u : 0u);
      }
      commit_both<PAIR>(bar.empty + s);
    }
    if (!ok) break;
    commit_both<PAIR>(bar.acc_full + buf);
  }
  // Everything this thread issued must finish before TMEM is released.
  if constexpr (PAIR)
    mma_commit_pair(bar.fin);
  else
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

// Scale, bias and round 32 accumulator columns of one row into 16 packed
// pairs (first column in the low half).  cs / cb: this chunk's 32 column
// scales / bias values in shared memory.
template <bool F16OUT>
__device__ __forceinline__ void epilogue_values(const GemmParams& p, const uint32_t (&r)[32],
                                                const float* cs, const float* cb, float sa,
                                                bool col_scale, bool has_bias, uint32_t* o) {
  const uint64_t sa2 = pack_f32x2(sa, sa);
  const uint64_t sb2 = pack_f32x2(p.b_scale, p.b_scale);
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
}

// epilogue_values for 32 columns of one row, stored to C.
template <bool F16OUT>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, const uint32_t (&r)[32],
                                               const float* cs, const float* cb, float sa,
                                               bool col_scale, bool has_bias, uint16_t* crow,
                                               int n0) {
  const bool full = (n0 + 32 <= p.N);
  uint32_t o[16];
  epilogue_values<F16OUT>(p, r, cs, cb, sa, col_scale, has_bias, o);
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

template <bool PAIR, bool F16OUT>
__device__ void gemm_epilogue(const GemmParams& p, const GemmBars& bar, uint32_t tmem,
                              float* colbuf, uint32_t rank) {
  using C = GCfg<PAIR>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ew = warp - 2;                // epilogue warp 0..7
  const int q = warp & 3;                 // TMEM lane quarter this warp may access
  const int half = ew / 4;                // column half of the tile
  const bool col_scale = p.sb != nullptr, has_bias = p.bias != nullptr;
  float* cs = colbuf + ew * 2 * kEpiCols;  // this warp's column scales, then bias
  float* cb = cs + kEpiCols;
  int it = 0;
  for (int t = tile_unit<PAIR>(); t < p.tiles; t += tile_units<PAIR>(), ++it) {
    const int buf = it & 1;
    const TileCoord c = tile_coord(p, t);
    const int ncol0 = c.n * kTileN + half * kEpiCols;
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
    const int m = c.m * C::kTileM + static_cast<int>(rank) * kCtaRows + q * 32 + lane;
    const bool row_ok = m < p.M;
    const float sa = p.sa ? (row_ok ? __ldg(p.sa + (int64_t)m * p.sa_stride) : 0.f) : p.a_scale;
    uint16_t* crow = static_cast<uint16_t*>(p.C) + (int64_t)(row_ok ? m : 0) * p.ldc;
    if (!wait_bar<PAIR>(bar.acc_full + buf, (it >> 1) & 1, bar, p.status, kErrGemmAccFull))
      return;
    tc_fence_after();
    const uint32_t taddr =
        tmem + buf * kTileN + half * kEpiCols + (static_cast<uint32_t>(q * 32) << 16);
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
        if (lane == 0) {
          if constexpr (PAIR)
            mbar_arrive_cluster(mapa_shared(smem_u32(bar.acc_empty + buf), 0));
          else
            mbar_arrive(bar.acc_empty + buf);
        }
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

// Fused QKV quantize epilogue (p.qkv_S > 0).  A CTA's 128 rows are one
// 128-token block of one batch and each half of the tile's 256 columns is one
// head of Q, K or V, so the four warps of a half (one per TMEM lane quarter)
// hold exactly one scale group of the per-block quantizer: 128 tokens x 128
// head dims of one (batch, head).  Each thread keeps its row's 128 bf16
// values (the bf16 C the plain epilogue would store, bit for bit), the four
// warps combine their block amax through shared memory and a named barrier,
// and every thread quantizes its row with the quantizer's own steps
// (quant_common.cuh) and writes its 128 e4m3 bytes into the attention
// kernel's (B * H, S, 128) layout; one thread writes the block's scale.
template <bool PAIR>
__device__ void gemm_epilogue_qkv(const GemmParams& p, const GemmBars& bar, uint32_t tmem,
                                  float* colbuf, uint32_t* amax_slots, uint32_t rank) {
  using C = GCfg<PAIR>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ew = warp - 2;
  const int q = warp & 3;
  const int half = ew / 4;
  const bool col_scale = p.sb != nullptr, has_bias = p.bias != nullptr;
  float* cs = colbuf + ew * 2 * kEpiCols;
  float* cb = cs + kEpiCols;
  const int H = p.qkv_H, S = p.qkv_S;
  int it = 0;
  for (int t = tile_unit<PAIR>(); t < p.tiles; t += tile_units<PAIR>(), ++it) {
    const int buf = it & 1;
    const TileCoord c = tile_coord(p, t);
    const int b = c.m / p.qkv_per_b;
    const int s0 = (c.m - b * p.qkv_per_b) * C::kTileM + static_cast<int>(rank) * kCtaRows;
    const int cblk = c.n * 2 + half;  // 128-column block: which * H + head
    const bool blk_ok = cblk < 3 * H && s0 < S;
    const int ncol0 = c.n * kTileN + half * kEpiCols;
    if (col_scale || has_bias) {
      __syncwarp();
#pragma unroll
      for (int i = 0; i < kEpiCols / 32; ++i) {
        const int n = ncol0 + i * 32 + lane;
        const bool in = n < p.N;
        if (col_scale) cs[i * 32 + lane] = in ? __ldg(p.sb + (int64_t)n * p.sb_stride) : 0.f;
        if (has_bias) cb[i * 32 + lane] = in ? bias_at(p.bias, n, false) : 0.f;
      }
      __syncwarp();
    }
    const int s = s0 + q * 32 + lane;  // this thread's token
    const bool row_ok = blk_ok && s < S;
    const int64_t m = (int64_t)b * S + s;
    const float sa = p.sa ? (row_ok ? __ldg(p.sa + m * p.sa_stride) : 0.f) : p.a_scale;
    if (!wait_bar<PAIR>(bar.acc_full + buf, (it >> 1) & 1, bar, p.status, kErrGemmAccFull))
      return;
    tc_fence_after();
    const uint32_t taddr =
        tmem + buf * kTileN + half * kEpiCols + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t y[kEpiCols / 2];  // the row's 128 bf16 values, packed pairs
#pragma unroll
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
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR)
            mbar_arrive_cluster(mapa_shared(smem_u32(bar.acc_empty + buf), 0));
          else
            mbar_arrive(bar.acc_empty + buf);
        }
      }
      epilogue_values<false>(p, r0, cs + pr * 64, cb + pr * 64, sa, col_scale, has_bias, y + pr * 32);
      epilogue_values<false>(p, r1, cs + pr * 64 + 32, cb + pr * 64 + 32, sa, col_scale, has_bias,
                             y + pr * 32 + 16);
    }
    // block amax: |bf16| bit patterns (NaN above +inf), valid rows only
    uint32_t am = 0;
    if (row_ok) {
      uint32_t a2 = 0;
#pragma unroll
      for (int i = 0; i < kEpiCols / 2; ++i) a2 = __vmaxu2(a2, y[i] & 0x7FFF7FFFu);
      am = max(a2 & 0xFFFFu, a2 >> 16);
    }
    am = __reduce_max_sync(0xffffffffu, am);
    uint32_t* slots = amax_slots + (buf * 2 + half) * 4;
    if (lane == 0) slots[q] = am;
    named_bar_sync(1 + half, 128);
    const uint32_t bm = max(max(slots[0], slots[1]), max(slots[2], slots[3]));
    if (blk_ok) {
      const float sc = quant::scale_from_amax_bits<false>(bm);
      const float qm = __frcp_rn(sc);
      const bool fast = isfinite(sc);
      const int which = cblk / H, h = cblk - which * H;
      if (row_ok) {
        // (conditional picks, not a dynamic index into the parameter struct)
        uint8_t* out8 = which == 0 ? p.qkv_out[0] : (which == 1 ? p.qkv_out[1] : p.qkv_out[2]);
        uint4* dst = reinterpret_cast<uint4*>(out8 + ((int64_t)(b * H + h) * S + s) * 128);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const uint2 lo = quant::quant8_any<false>(
              make_uint4(y[8 * v], y[8 * v + 1], y[8 * v + 2], y[8 * v + 3]), qm, fast);
          const uint2 hi = quant::quant8_any<false>(
              make_uint4(y[8 * v + 4], y[8 * v + 5], y[8 * v + 6], y[8 * v + 7]), qm, fast);
          dst[v] = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
      }
      if (q == 0 && lane == 0) {
        float* sd = which == 0 ? p.qkv_scales[0] : (which == 1 ? p.qkv_scales[1] : p.qkv_scales[2]);
        sd[(int64_t)(b * H + h) * p.qkv_nblk + s0 / kCtaRows] = sc;
      }
    }
  }
}

template <bool PAIR, bool BKM, bool F16OUT, bool QKV = false>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_b, const GemmParams p) {
  using C = GCfg<PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const GemmBars bar = carve_gemm_bars<PAIR>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar.full + s, 1);
      mbar_init(bar.empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar.acc_full + b, 1);
      mbar_init(bar.acc_empty + b, C::kAccEmptyCount);
    }
    mbar_init(bar.fin, 1);
    *bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    if constexpr (PAIR) {
      tmem_alloc_pair(bar.tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(bar.tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  if (warp == kTmaWarp && lane == 0 && p.n_kb > 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  tc_fence_before();
  // Both CTAs' barriers must be initialised before either signals the other's.
  if constexpr (PAIR)
    cluster_sync();
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tmem_slot;

  if (warp == kTmaWarp) {
    if (lane == 0) gemm_producer<PAIR, BKM>(&tm_a, &tm_b, p, bar, smem, rank);
  } else if (warp == kMmaWarp) {
    if (lane == 0 && rank == 0) gemm_mma<PAIR, BKM>(p, bar, smem_u32(smem), tmem);
  } else {
    if constexpr (QKV)
      gemm_epilogue_qkv<PAIR>(p, bar, tmem, reinterpret_cast<float*>(smem + C::kOffCol),
                              reinterpret_cast<uint32_t*>(smem + C::kOffAmax), rank);
    else
      gemm_epilogue<PAIR, F16OUT>(p, bar, tmem, reinterpret_cast<float*>(smem + C::kOffCol), rank);
  }
  __syncwarp();

  tc_fence_before();
  // Rank 0's MMAs read rank 1's shared memory and write its TMEM: neither CTA
  // releases either until both are done.
  if constexpr (PAIR)
    cluster_sync();
  else
    __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, kTmemCols);
    else
      tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool PAIR, bool BKM, bool F16OUT, bool QKV = false>
cudaError_t launch_gemm_variant(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p,
                                int units, cudaStream_t st) {
  using C = GCfg<PAIR>;
  auto kern = fp8_gemm_kernel<PAIR, BKM, F16OUT, QKV>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_release);
  }
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * units, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, b, p);
  } else {
    kern<<<units, kThreads, C::kSmemBytes, st>>>(a, b, p);
    return cudaGetLastError();
  }
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

// 2-SM pairs (1, default) or single-CTA tiles (0).  REPERCEP_B200_GEMM_PAIR
// overrides (read once).
bool gemm_pair_setting() {
  static const bool v = [] {
    const char* e = std::getenv("REPERCEP_B200_GEMM_PAIR");
    return !(e && std::atoi(e) == 0);
  }();
  return v;
}

// Row tiles per raster group (0: the kernel's default).  REPERCEP_B200_GEMM_GROUP
// overrides (read once).
int gemm_group_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_GEMM_GROUP");
    const int x = e ? std::atoi(e) : 0;
    return (x > 0 && x <= 1024) ? x : 0;
  }();
  return v;
}

int gemm_b_box_rows(bool b_kmajor) {
  if (!b_kmajor) return 128;  // N-major: 128 K rows x 128 N bytes per box
  return gemm_pair_setting() ? GCfg<true>::kBRows : GCfg<false>::kBRows;
}

template <bool PAIR>
cudaError_t launch_fp8_gemm_t(const CUtensorMap& a, const CUtensorMap& b, GemmParams p,
                              bool b_kmajor, bool out_f16, cudaStream_t st) {
  using C = GCfg<PAIR>;
  if (p.qkv_S > 0) {
    if (!b_kmajor || out_f16 || p.qkv_S <= 0 || p.M % p.qkv_S != 0) return cudaErrorInvalidValue;
    p.qkv_per_b = (p.qkv_S + C::kTileM - 1) / C::kTileM;
    p.tiles_m = (p.M / p.qkv_S) * p.qkv_per_b;
  } else {
    p.tiles_m = (p.M + C::kTileM - 1) / C::kTileM;
  }
  p.tiles_n = (p.N + kTileN - 1) / kTileN;
  p.tiles = p.tiles_m * p.tiles_n;
  p.n_kb = (p.K + kBK - 1) / kBK;
  if (p.group_m <= 0) p.group_m = gemm_group_setting();
  if (p.group_m <= 0) p.group_m = PAIR ? 8 : 16;
  if (p.group_m > p.tiles_m) p.group_m = p.tiles_m;
  const int slots = PAIR ? sm_count() / 2 : sm_count();
  const int units = p.tiles < slots ? p.tiles : slots;
  if (p.qkv_S > 0) return launch_gemm_variant<PAIR, true, false, true>(a, b, p, units, st);
  if (b_kmajor)
    return out_f16 ? launch_gemm_variant<PAIR, true, true>(a, b, p, units, st)
                   : launch_gemm_variant<PAIR, true, false>(a, b, p, units, st);
  return out_f16 ? launch_gemm_variant<PAIR, false, true>(a, b, p, units, st)
                 : launch_gemm_variant<PAIR, false, false>(a, b, p, units, st);
}

cudaError_t launch_fp8_gemm(const CUtensorMap& a, const CUtensorMap& b, GemmParams p,
                            bool b_kmajor, bool out_f16, cudaStream_t st) {
  return gemm_pair_setting() ? launch_fp8_gemm_t<true>(a, b, p, b_kmajor, out_f16, st)
                             : launch_fp8_gemm_t<false>(a, b, p, b_kmajor, out_f16, st);
}

}  // namespace rp
