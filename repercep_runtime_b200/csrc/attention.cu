// FP8 (e4m3) flash-attention forward for sm_100a: TMA-fed, tcgen05/TMEM,
// warp-specialised.  Restates the algorithm of the reference's fused kernel
// (kernels/triton_kernels/fp8_flash_attn_hopper.py:197-338): per-tile
// S = Q K^T in fp32 scaled by softmax_scale * q_scale * k_scale, an online
// softmax, P quantised to e4m3 against a fixed 448 range (:322), O += P V
// scaled by v_scale / 448 (:323-327), O /= l (:332).
//
// CTA layout (NQ query tiles of 128 rows share each K/V tile):
//   warps [0, 4*NQ)   softmax warpgroups, warpgroup t owns query tile t; a
//                     thread owns one query row == one TMEM lane
//   warp  4*NQ        TMA producer (Q once, then a ring of K and V tiles)
//   warp  4*NQ + 1    MMA issuer (one thread issues every tcgen05.mma)
// TMEM: S[t] at columns [128 t, 128 t + 128), O[t] at [128 (NQ + DB t), ...) (128 DB wide).
// SMEM (1024-byte aligned, 128-byte swizzle everywhere):
//   Q[NQ] | K[3] | V[3] | P[NQ][PBUF] (hi [+ lo] planes) | mbarriers
// Operand majors: Q, K, P are K-major; V is MN-major (its natural [kv][d]
// layout), which tcgen05 accepts for e4m3.
//
// Scales are generalised from the reference's one-per-(b,h) to any grid of
// 128-row blocks: k_scale / v_scale may change per K/V tile.  v_scale is
// folded into P: P' = e4m3(p * 448 * sv_j / sv_max) so one TMEM accumulator
// serves every tile, and the epilogue multiplies by sv_max / 448 / l.
//
// PMODE 0: P is one e4m3 plane (the reference's precision).
// PMODE 1: P is split into e4m3 hi + lo planes and PV runs twice, which
//          removes almost all of the P rounding error.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <atomic>
#include <cstdlib>

#include "internal.h"
#include "ptx.cuh"

namespace rp {
namespace {

constexpr int kTile = 128;
constexpr int kTileBytes = kTile * kTile;
constexpr int kKSt = 3;
constexpr int kVSt = 3;
constexpr int kDefaultExpPoly = 2;   // with row layouts 1 and 2 (the lane split: 0)
constexpr int kLaneSplitExpPoly = 0;
constexpr int kDefaultRowSplit = 3;  // kLaneSplit
constexpr float kDefaultRescaleTau = 1.0f;
constexpr int kDefaultStagger = 2;

// Pipeline tracing (compiled in only with -DRP_PIPELINE_TRACE): one chosen CTA
// records (SM clock, event << 16 | step) at every barrier hand-off of every
// role, for offline timeline analysis.  The product build has none of it.
#ifdef RP_PIPELINE_TRACE
// Slot (event, step) of the traced CTA; each role reads the target once
// (RP_TRACE_INIT) so recording is a clock read and a plain store.
__device__ uint32_t* g_trace_buf = nullptr;
__device__ int g_trace_x = -1;
__device__ int g_trace_y = -1;
constexpr int kTraceSteps = 1024;  // events < 256
__device__ __forceinline__ uint32_t* trace_target() {
  // (the launch grid is 1-D: cta_x is the CTA index, cta_y must be 0)
  return (g_trace_buf != nullptr && (int)blockIdx.x == g_trace_x && (int)blockIdx.y == g_trace_y)
             ? g_trace_buf
             : nullptr;
}
#define RP_TRACE_INIT() uint32_t* const rp_trace_buf_ = trace_target()
#define RP_TRACE(ev, j)                                                                   \
  do {                                                                                    \
    if (rp_trace_buf_)                                                                    \
      rp_trace_buf_[(ev) * kTraceSteps + ((j) & (kTraceSteps - 1))] =                     \
          static_cast<uint32_t>(clock64());                                               \
  } while (0)
#else
#define RP_TRACE_INIT() ((void)0)
#define RP_TRACE(ev, j) ((void)0)
#endif

enum : int {
  kErrWaitQ = 0x101,
  kErrWaitK = 0x102,
  kErrWaitV = 0x103,
  kErrWaitKEmpty = 0x104,
  kErrWaitVEmpty = 0x105,
  kErrWaitS = 0x106,
  kErrWaitSFree = 0x107,
  kErrWaitP = 0x108,
  kErrWaitO = 0x109,
  kErrWaitEpi = 0x10A,
  kErrWaitOFinal = 0x10B,
  kErrWaitX = 0x10C,
  kErrWaitStag = 0x10D,
};

// Row layouts of the softmax warps (NSPLIT):
//   1  one thread per query row: warp w of a tile holds the 32 rows of TMEM
//      lane quarter w, all 128 columns each (4 warps per tile);
//   2  two warps per lane quarter, each row's columns split between them
//      (64 each): row maxima and sums are swapped through shared memory;
//   3  (kLaneSplit) two warps per lane quarter, 16 rows each, and each row's
//      128 columns split between lanes t and t + 16 of its warp (64 each,
//      tcgen05.ld 16x32bx2): row maxima and sums are combined with a shuffle.
// 2 and 3 give 8 softmax warps per tile.
constexpr int kLaneSplit = 3;

// DB: head dim in 128-column blocks (1: D <= 128, the rows of D = 32 / 64
// zero-padded to 128 bytes; 2: D = 256, one query tile per CTA).
template <int NQ, int PMODE, int NSPLIT = 1, bool TAB = false, int DB = 1>
struct Cfg {
  static constexpr int kRowThreads = (NSPLIT == 1) ? 1 : 2;  // threads per query row
  static constexpr int kNC = kTile / kRowThreads;            // S columns per softmax thread
  static constexpr int kWarpsPerTile = 4 * kRowThreads;
  static constexpr int kSoftmaxWarps = kWarpsPerTile * NQ;
  static constexpr int kTmaWarp = kSoftmaxWarps;
  static constexpr int kMmaWarp = kSoftmaxWarps + 1;
  static constexpr int kThreads = (kSoftmaxWarps + 2) * 32;
  static constexpr int kPBuf = (PMODE == 0) ? 2 : 1;
  static constexpr int kPParts = (PMODE == 0) ? 1 : 2;
  static_assert(NQ * (1 + DB) * kTile <= 512, "TMEM holds S and O of every query tile");
  static_assert(DB == 1 || NSPLIT == 1, "row split only for D <= 128");
  static_assert(NSPLIT >= 1 && NSPLIT <= 3, "row layouts 1, 2, 3");
  static constexpr int kTmemCols = (NQ * (1 + DB) * kTile > 256) ? 512 : 256;
  static constexpr int kSt = (DB == 2) ? 2 : 3;       // K and V ring stages (<= kKSt, kVSt)
  static constexpr int kQBytes = DB * kTileBytes;     // one query tile
  static constexpr int kKVBytes = DB * kTileBytes;    // one K or V stage
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + NQ * kQBytes;
  static constexpr int kOffV = kOffK + kSt * kKVBytes;
  static constexpr int kOffP = kOffV + kSt * kKVBytes;
  static constexpr int kPStride = kPParts * kTileBytes;
  static constexpr int kOffX = kOffP + NQ * kPBuf * kPStride;  // row-max / row-sum exchange
  static constexpr int kXBytes = (NSPLIT == 2) ? NQ * 3 * 2 * kTile * 4 : 0;
  // Per-step constant table (TAB): 64 bytes of reduction scratch, then one
  // float4 per K/V step.
  static constexpr int kOffT = kOffX + kXBytes;
  static constexpr int kTableSteps = TAB ? ((NSPLIT == 2) ? 1536 : 2048) : 0;
  static constexpr int kTabBytes = TAB ? 64 + kTableSteps * 16 : 0;
  static constexpr int kOffBar = kOffT + kTabBytes;
  static constexpr int kNumBars = 1 + 2 * kKSt + 2 * kVSt + 7 * NQ + 1 + 12 * NQ + 32 + NQ;
  static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Bars {
  uint64_t *q_full, *k_full, *k_empty, *v_full, *v_empty;
  uint64_t *s_full, *s_free, *p_full, *o_done, *o_final, *epi, *fin, *xch, *stag, *stag1, *epi2;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

template <int NQ>
__device__ __forceinline__ Bars carve_bars(uint8_t* base) {
  Bars b;
  uint64_t* p = reinterpret_cast<uint64_t*>(base);
  b.q_full = p;
  b.k_full = b.q_full + 1;
  b.k_empty = b.k_full + kKSt;
  b.v_full = b.k_empty + kKSt;
  b.v_empty = b.v_full + kVSt;
  b.s_full = b.v_empty + kVSt;
  b.s_free = b.s_full + NQ;
  b.p_full = b.s_free + NQ;  // [NQ][2]: step j uses p_full[2 t + (j & 1)]
  b.o_done = b.p_full + 2 * NQ;
  b.o_final = b.o_done + NQ;
  b.epi = b.o_final + NQ;
  b.fin = b.epi + NQ;
  b.xch = b.fin + 1;  // [NQ][4 lane quarters][3]: row-max (x2 by step parity), row-sum
  b.stag = b.xch + 12 * NQ;  // [4 lane quarters][4 by step mod 4]: tile 0 exp done
  b.stag1 = b.stag + 16;     // [4 lane quarters][4 by step mod 4]: tile 1 exp done
  b.epi2 = b.stag1 + 16;     // [NQ] (decode) warpgroup's half of the output staged
  b.tmem_slot = reinterpret_cast<uint32_t*>(b.epi2 + NQ);
  b.abort_flag = reinterpret_cast<volatile int*>(b.tmem_slot + 1);
  return b;
}

// Every lane waits on the barrier (one try_wait instruction for the warp;
// the loop stays convergent because all lanes read the same barrier word,
// clock and abort flag), then a vote makes the outcome warp-uniform.  No
// shuffle: on the softmax path every MIO-queue instruction would wait behind
// the other warpgroup's MUFU stream.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, int code) {
  const bool ok = mbar_wait(bar, parity, abort_flag, status, code);
  return __all_sync(0xffffffffu, ok);
}

// Time-bounded wait that ignores the abort flag: used to drain in-flight
// asynchronous work before the CTA releases its shared memory and TMEM.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles / 4) return;
  }
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Four floats to e4m3 (satfinite, round to nearest even), byte i = value i.
// pack_e4m3x4: the two pair conversions write 16-bit halves that one mov
// joins; built from the 16-bit results with a shift and an OR instead
// (pack_e4m3x4_or), the step loop of the all-MUFU kernels ran ~2 % slower
// (extra integer instructions on the softmax warps' issue path).  The
// polynomial-exp and two-part-P kernels keep the OR form: with the joined
// form ptxas spills registers in them.
__device__ __forceinline__ uint32_t pack_e4m3x4_or(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  uint32_t r;
  asm("{\n .reg .b16 lo, hi;\n"
      " cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n"
      " cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n"
      " mov.b32 %0, {lo, hi};\n}"
      : "=r"(r)
      : "f"(a), "f"(b), "f"(c), "f"(d));
  return r;
}

// Residual of four values after their e4m3 rounding in `packed`, re-packed.
__device__ __forceinline__ uint32_t pack_e4m3x4_residual(uint32_t packed, float a, float b,
                                                         float c, float d) {
  const __half2_raw h01 =
      __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(packed & 0xFFFFu), __NV_E4M3);
  const __half2_raw h23 =
      __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(packed >> 16), __NV_E4M3);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  return pack_e4m3x4_or(a - f01.x, b - f01.y, c - f23.x, d - f23.y);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// 2^x for two lanes on the FMA pipe: x = n + f with n = rint(x) (the 1.5*2^23
// addition rounds into the low mantissa bits), 2^f from a cubic fitted on
// [-0.5, 0.5] (csrc/gen_exp2_poly.py, max relative error 7.5e-5), 2^n added to
// the exponent field as an integer.  Inputs are clamped to >= -125 so the
// exponent never wraps; results below 2^-125 are irrelevant to the softmax.
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& y0, float& y1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const uint64_t x = pack_f32x2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t t = fadd2(x, pack_f32x2(kRound, kRound));
  const uint64_t f = fsub2(x, fsub2(t, pack_f32x2(kRound, kRound)));
  uint64_t q = ffma2(pack_f32x2(0.055170513689517975f, 0.055170513689517975f), f,
                     pack_f32x2(0.24260854721069336f, 0.24260854721069336f));
  q = ffma2(q, f, pack_f32x2(0.6932609677314758f, 0.6932609677314758f));
  q = ffma2(q, f, pack_f32x2(0.9999282360076904f, 0.9999282360076904f));
  float q0, q1, t0, t1;
  unpack_f32x2(q, q0, q1);
  unpack_f32x2(t, t0, t1);
  y0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// This CTA's work unit: (b,h) and column (a group of NQ query tiles, or one
// query tile for the split-step form), from the launch's 1-D unit range.
__device__ __forceinline__ int unit_bh(const AttnKernelParams& p) {
  return (p.unit_base + static_cast<int>(blockIdx.x)) / p.units_per_bh;
}
__device__ __forceinline__ int unit_x(const AttnKernelParams& p) {
  const int u = p.unit_base + static_cast<int>(blockIdx.x);
  return u - (u / p.units_per_bh) * p.units_per_bh;
}

// Which K/V tile step j reads: chunk c, tile t within the chunk, valid rows.
__device__ __forceinline__ void step_info(const AttnKernelParams& p, int j, int& c, int& t,
                                          int& valid, bool& extra) {
  if (p.has_extra && j == p.n_main_tiles) {
    extra = true;
    c = 0;
    t = 0;
    valid = kTile;
    return;
  }
  extra = false;
  c = j / p.tiles_per_chunk;
  t = j - c * p.tiles_per_chunk;
  const int len = (c == p.n_chunks - 1) ? p.last_len : p.chunk_len;
  valid = min(kTile, len - t * kTile);
}

// The same (chunk, tile) walk as step_info, one step at a time without a
// division (main tiles only; the extra tile is handled by the caller).
struct StepCursor {
  int c = 0, t = 0;
  __device__ __forceinline__ void next(const AttnKernelParams& p) {
    if (++t == p.tiles_per_chunk) {
      t = 0;
      ++c;
    }
  }
  __device__ __forceinline__ int valid(const AttnKernelParams& p) const {
    const int len = (c == p.n_chunks - 1) ? p.last_len : p.chunk_len;
    return min(kTile, len - t * kTile);
  }
};

// Orders every later use of `r` after the preceding tcgen05.wait::ld: the
// compiler sees the registers redefined here, after the (volatile) wait.
__device__ __forceinline__ void reg_fence(uint32_t (&r)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 8)
    asm volatile("" : "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]), "+r"(r[i + 4]),
                 "+r"(r[i + 5]), "+r"(r[i + 6]), "+r"(r[i + 7]));
}

// ------------------------------------------------------------ TMA producer
template <int NQ, int PMODE, int DB, bool KS = false>
__device__ void producer(const CUtensorMap* tm_q, const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                         const CUtensorMap* tm_kx, const CUtensorMap* tm_vx,
                         const AttnKernelParams& p, const Bars& bar, uint8_t* smem, int n_steps) {
  using C = Cfg<NQ, PMODE, 1, false, DB>;
  RP_TRACE_INIT();
  const int bh = unit_bh(p);
  // KS: one query tile per CTA, read by both tiles' QK MMAs from Q slot 0.
  const int qt0 = KS ? unit_x(p) : unit_x(p) * NQ;
  constexpr int kQTiles = KS ? 1 : NQ;
  auto load_q = [&]() {
    mbar_arrive_expect_tx(bar.q_full, kQTiles * C::kQBytes);
#pragma unroll
    for (int t = 0; t < kQTiles; ++t)
#pragma unroll
      for (int kb = 0; kb < DB; ++kb)
        tma_load_4d(smem + C::kOffQ + t * C::kQBytes + kb * kTileBytes, tm_q, bar.q_full,
                    kb * kTile, (qt0 + t) * kTile, bh, 0);
  };
  // KS (the decode, launched as a programmatic dependent of the launch
  // before it): no global read before that launch has completed -- it may
  // have written any operand, the prefix included.  What overlaps it is this
  // CTA's launch, barrier and TMEM setup.
  if (KS) griddep_wait();
  RP_TRACE(82, 0);
  load_q();
  RP_TRACE(83, 0);

  int nk = 0, nv = 0;
  bool ok = true;
  StepCursor cur;
  for (int j = 0; j < n_steps && ok; ++j) {
    const bool extra = p.has_extra && j == p.n_main_tiles;
    const int c = cur.c, t = cur.t;
    if (!extra) cur.next(p);
    const int ks = j % C::kSt, ku = j / C::kSt;
    if (ku > 0 && !mbar_wait(bar.k_empty + ks, (ku - 1) & 1, bar.abort_flag, p.status,
                             kErrWaitKEmpty)) {
      ok = false;
      break;
    }
    mbar_arrive_expect_tx(bar.k_full + ks, C::kKVBytes);
#pragma unroll
    for (int kb = 0; kb < DB; ++kb) {
      uint8_t* dst = smem + C::kOffK + ks * C::kKVBytes + kb * kTileBytes;
      if (extra)
        tma_load_4d(dst, tm_kx, bar.k_full + ks, kb * kTile, qt0 * kTile, bh, 0);
      else
        tma_load_4d(dst, tm_k, bar.k_full + ks, kb * kTile, t * kTile, bh, c);
    }
    ++nk;
    RP_TRACE(80, j);
    const int vs = j % C::kSt, vu = j / C::kSt;
    if (vu > 0 && !mbar_wait(bar.v_empty + vs, (vu - 1) & 1, bar.abort_flag, p.status,
                             kErrWaitVEmpty)) {
      ok = false;
      break;
    }
    mbar_arrive_expect_tx(bar.v_full + vs, C::kKVBytes);
#pragma unroll
    for (int kb = 0; kb < DB; ++kb) {
      uint8_t* dst = smem + C::kOffV + vs * C::kKVBytes + kb * kTileBytes;
      if (extra)
        tma_load_4d(dst, tm_vx, bar.v_full + vs, kb * kTile, qt0 * kTile, bh, 0);
      else
        tma_load_4d(dst, tm_v, bar.v_full + vs, kb * kTile, t * kTile, bh, c);
    }
    ++nv;
    RP_TRACE(81, j);
  }
  if (!ok) {
    // Abort: let every load already issued land before shared memory goes away.
    mbar_drain(bar.q_full, 0);
    for (int s = 0; s < C::kSt; ++s)
      if (s < nk) mbar_drain(bar.k_full + s, ((nk - 1 - s) / C::kSt) & 1);
    for (int s = 0; s < C::kSt; ++s)
      if (s < nv) mbar_drain(bar.v_full + s, ((nv - 1 - s) / C::kSt) & 1);
  }
}

// -------------------------------------------------------------- MMA issuer
template <int NQ, int PMODE, int DB, bool KS = false>
__device__ __forceinline__ bool issue_pv(const AttnKernelParams& p, const Bars& bar,
                                         uint32_t sbase, uint32_t tmem, int i, bool last) {
  using C = Cfg<NQ, PMODE, 1, false, DB>;
  RP_TRACE_INIT();
  constexpr uint32_t idesc_pv = make_idesc_e4m3(128, 128, 0, 1);
  const int vsl = i % C::kSt;
  if (!mbar_wait(bar.v_full + vsl, (i / C::kSt) & 1, bar.abort_flag, p.status, kErrWaitV))
    return false;
  RP_TRACE(71, i);
#pragma unroll
  for (int tt = 0; tt < (KS ? 1 : NQ); ++tt) {
    // KS: step i belongs to tile i & 1, its li-th step.
    const int t = KS ? (i & 1) : tt;
    const int li = KS ? (i >> 1) : i;
    // Two P_full barriers per tile, alternating by step: a softmax warpgroup
    // that runs ahead can complete step i+1 before this wait for step i, and
    // a single barrier would then be two phases ahead of the parity wait.
    if (!mbar_wait(bar.p_full + 2 * t + (li & 1), (li >> 1) & 1, bar.abort_flag, p.status,
                   kErrWaitP))
      return false;
    RP_TRACE(70 + 2 * t, i);
    tc_fence_after();
    const int pb = (C::kPBuf == 2) ? (li & 1) : 0;
    const uint32_t paddr = sbase + C::kOffP + (t * C::kPBuf + pb) * C::kPStride;
    const uint64_t pd = make_sw128_desc(paddr, 16, 1024);
    // O_t: DB column blocks of 128 after the NQ S tiles; V block nb feeds block nb.
#pragma unroll
    for (int nb = 0; nb < DB; ++nb) {
      const uint64_t vd = make_sw128_desc(
          sbase + C::kOffV + vsl * C::kKVBytes + nb * kTileBytes, kTileBytes, 1024);
      const uint32_t d_tmem = tmem + (NQ + t * DB + nb) * kTile;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_f8(d_tmem, pd + 2 * k, vd + 256 * k, idesc_pv, (li > 0 || k > 0) ? 1u : 0u);
      if constexpr (PMODE == 1) {
        const uint64_t pl = make_sw128_desc(paddr + kTileBytes, 16, 1024);
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f8(d_tmem, pl + 2 * k, vd + 256 * k, idesc_pv, 1u);
      }
    }
    mma_commit(bar.o_done + t);
    if (last) {
      // KS: the other tile's last PV came earlier; both finals follow this one.
      mma_commit(bar.o_final + t);
      if (KS) mma_commit(bar.o_final + (1 - t));
    }
    RP_TRACE(60 + t, i);
  }
  mma_commit(bar.v_empty + vsl);
  return true;
}

template <int NQ, int PMODE, int DB, bool KS = false>
__device__ void mma_issuer(const AttnKernelParams& p, const Bars& bar, uint8_t* smem,
                           uint32_t tmem, int n_steps) {
  using C = Cfg<NQ, PMODE, 1, false, DB>;
  RP_TRACE_INIT();
  constexpr uint32_t idesc_qk = make_idesc_e4m3(128, 128, 0, 0);
  const uint32_t sbase = smem_u32(smem);
  // KS (launched as a programmatic dependent): the bounded waits below start
  // only once the launch before has completed, so a long predecessor cannot
  // use up their time limit.
  if constexpr (KS) griddep_wait();
  bool ok = mbar_wait(bar.q_full, 0, bar.abort_flag, p.status, kErrWaitQ);
  for (int j = 0; ok && j < n_steps; ++j) {
    const int ks = j % C::kSt;
    if (!mbar_wait(bar.k_full + ks, (j / C::kSt) & 1, bar.abort_flag, p.status, kErrWaitK)) {
      ok = false;
      break;
    }
    RP_TRACE(75, j);
#pragma unroll
    for (int tt = 0; tt < (KS ? 1 : NQ); ++tt) {
      const int t = KS ? (j & 1) : tt;
      const int li = KS ? (j >> 1) : j;
      if (li > 0 &&
          !mbar_wait(bar.s_free + t, (li - 1) & 1, bar.abort_flag, p.status, kErrWaitSFree)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // S_t = sum over the DB head-dim blocks of Q_t[kb] K[kb]^T (K = 32 per MMA)
#pragma unroll
      for (int kb = 0; kb < DB; ++kb) {
        const uint64_t kd =
            make_sw128_desc(sbase + C::kOffK + ks * C::kKVBytes + kb * kTileBytes, 16, 1024);
        const uint64_t qd = make_sw128_desc(
            sbase + C::kOffQ + (KS ? 0 : t) * C::kQBytes + kb * kTileBytes, 16, 1024);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f8(tmem + t * kTile, qd + 2 * k, kd + 2 * k, idesc_qk, (kb > 0 || k > 0) ? 1u : 0u);
      }
      mma_commit(bar.s_full + t);
      RP_TRACE(50 + t, j);
    }
    if (!ok) break;
    mma_commit(bar.k_empty + ks);
    // KS: a warpgroup's next S (step j) is issued before its previous PV
    // (step j - 2), so it computes while that warpgroup is still on step
    // j - 2.  The tensor pipe runs in order, so S_full(j) still implies every
    // earlier PV is done (the P buffer reuse rule below holds unchanged).
    if constexpr (KS) {
      if (j >= 2) ok = issue_pv<NQ, PMODE, DB, KS>(p, bar, sbase, tmem, j - 2, false);
    } else {
      if (j > 0) ok = issue_pv<NQ, PMODE, DB, KS>(p, bar, sbase, tmem, j - 1, false);
    }
  }
  if constexpr (KS) {
    for (int i = n_steps >= 2 ? n_steps - 2 : 0; ok && i < n_steps; ++i)
      ok = issue_pv<NQ, PMODE, DB, KS>(p, bar, sbase, tmem, i, i == n_steps - 1);
  } else {
    if (ok && n_steps > 0) issue_pv<NQ, PMODE, DB, KS>(p, bar, sbase, tmem, n_steps - 1, true);
  }
  // Everything this thread issued must finish before TMEM is released.
  mma_commit(bar.fin);
  mbar_drain(bar.fin, 0);
}

// MMA issue order "ahead" (not the decode): S of steps 0 and 1 for every tile
// first; then, for each step i, for each tile t: PV_t(i) (waits for P_t(i)),
// then QK_t(i + 2) (waits for the softmax to have loaded S_t(i + 1)).  Each
// tile thus has its next S computed while its softmax works on the current
// step, and a tile's QK never waits behind another tile's P.  The tensor pipe
// runs in order, so S_full_t(i + 2) still implies PV_t(i) is done: P buffer
// i & 1 is free again when the softmax writes P_t(i + 2) there.
template <int NQ, int PMODE, int DB>
__device__ void mma_issuer_ahead(const AttnKernelParams& p, const Bars& bar, uint8_t* smem,
                                 uint32_t tmem, int n_steps) {
  using C = Cfg<NQ, PMODE, 1, false, DB>;
  constexpr uint32_t idesc_qk = make_idesc_e4m3(128, 128, 0, 0);
  constexpr uint32_t idesc_pv = make_idesc_e4m3(128, 128, 0, 1);
  const uint32_t sbase = smem_u32(smem);
  auto wait_k = [&](int j) -> bool {
    return mbar_wait(bar.k_full + j % C::kSt, (j / C::kSt) & 1, bar.abort_flag, p.status, kErrWaitK);
  };
  // S_t = Q_t K(j)^T, once the softmax has loaded S_t of step j - 1.
  auto qk = [&](int j, int t) -> bool {
    if (j > 0 &&
        !mbar_wait(bar.s_free + t, (j - 1) & 1, bar.abort_flag, p.status, kErrWaitSFree))
      return false;
    tc_fence_after();
    const int ks = j % C::kSt;
#pragma unroll
    for (int kb = 0; kb < DB; ++kb) {
      const uint64_t kd =
          make_sw128_desc(sbase + C::kOffK + ks * C::kKVBytes + kb * kTileBytes, 16, 1024);
      const uint64_t qd = make_sw128_desc(sbase + C::kOffQ + t * C::kQBytes + kb * kTileBytes, 16, 1024);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_f8(tmem + t * kTile, qd + 2 * k, kd + 2 * k, idesc_qk, (kb > 0 || k > 0) ? 1u : 0u);
    }
    mma_commit(bar.s_full + t);
    return true;
  };
  bool ok = mbar_wait(bar.q_full, 0, bar.abort_flag, p.status, kErrWaitQ);
  for (int j = 0; ok && j < n_steps && j < 2; ++j) {
    ok = wait_k(j);
    for (int t = 0; ok && t < NQ; ++t) ok = qk(j, t);
    if (ok) mma_commit(bar.k_empty + j % C::kSt);
  }
  for (int i = 0; ok && i < n_steps; ++i) {
    const int vsl = i % C::kSt;
    if (!mbar_wait(bar.v_full + vsl, (i / C::kSt) & 1, bar.abort_flag, p.status, kErrWaitV)) {
      ok = false;
      break;
    }
    const bool more = i + 2 < n_steps;
#pragma unroll
    for (int t = 0; t < NQ; ++t) {
      if (!mbar_wait(bar.p_full + 2 * t + (i & 1), (i >> 1) & 1, bar.abort_flag, p.status,
                     kErrWaitP)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int pb = (C::kPBuf == 2) ? (i & 1) : 0;
      const uint32_t paddr = sbase + C::kOffP + (t * C::kPBuf + pb) * C::kPStride;
      const uint64_t pd = make_sw128_desc(paddr, 16, 1024);
#pragma unroll
      for (int nb = 0; nb < DB; ++nb) {
        const uint64_t vd = make_sw128_desc(
            sbase + C::kOffV + vsl * C::kKVBytes + nb * kTileBytes, kTileBytes, 1024);
        const uint32_t d_tmem = tmem + (NQ + t * DB + nb) * kTile;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f8(d_tmem, pd + 2 * k, vd + 256 * k, idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
        if constexpr (PMODE == 1) {
          const uint64_t pl = make_sw128_desc(paddr + kTileBytes, 16, 1024);
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_f8(d_tmem, pl + 2 * k, vd + 256 * k, idesc_pv, 1u);
        }
      }
      mma_commit(bar.o_done + t);
      if (i == n_steps - 1) mma_commit(bar.o_final + t);
      if (more) {
        if (t == 0 && !wait_k(i + 2)) {
          ok = false;
          break;
        }
        if (!qk(i + 2, t)) {
          ok = false;
          break;
        }
      }
    }
    if (!ok) break;
    mma_commit(bar.v_empty + vsl);
    if (more) mma_commit(bar.k_empty + (i + 2) % C::kSt);
  }
  // Everything this thread issued must finish before TMEM is released.
  mma_commit(bar.fin);
  mbar_drain(bar.fin, 0);
}

// ----------------------------------------------------------------- softmax
// Row layout NSPLIT (see Cfg): 1, one thread per row owning all columns;
// 2, thread (half, row) owns S columns [half * kNC, half * kNC + kNC) and the
// two halves swap their partial row maxima through shared memory every step
// and their partial row sums once at the end; 3 (kLaneSplit), warp half h of
// lane quarter q holds rows q*32 + 16h + (lane & 15), lane owning columns
// [64 (lane >> 4), +64), combined with a shuffle.
template <int NQ, int PMODE, int EPOLY, int NSPLIT, bool TAB, int DB, bool KS = false>
__device__ void softmax_wg(const CUtensorMap* tm_o, const AttnKernelParams& p, const Bars& bar,
                           uint8_t* smem, uint32_t tmem, int n_steps) {
  using C = Cfg<NQ, PMODE, NSPLIT, TAB, DB>;
  RP_TRACE_INIT();
  constexpr int NC = C::kNC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = warp / C::kWarpsPerTile;
  const int sub = warp % C::kWarpsPerTile;
  const int half = sub >> 2, wq = sub & 3;
  constexpr bool LS = (NSPLIT == kLaneSplit);
  const int row = LS ? wq * 32 + half * 16 + (lane & 15) : wq * 32 + lane;
  const int col0 = LS ? (lane >> 4) * NC : half * NC;
  const bool tracer = (wq == 0 && lane == 0 && half == 0);
  const int bh = unit_bh(p);
  // KS (one query tile, its K/V steps split between the two tiles' warpgroups):
  // warpgroup t takes steps t, t + 2, ... and warpgroup 1 hands its partial
  // row max and sum to warpgroup 0, which merges the two O accumulators.
  static_assert(!KS || (NQ == 2 && (NSPLIT == 1 || NSPLIT == kLaneSplit) && TAB && DB == 1),
                "KS: two tiles, one thread or two lanes per row, table, D 128");
  const int q_tile = KS ? unit_x(p) : unit_x(p) * NQ + t;
  const int j0 = KS ? t : 0;
  constexpr int kStepStride = KS ? 2 : 1;
  const int q_tile_c = min(q_tile, p.n_q_tiles - 1);
  // TMEM addresses: the lane field is the warp's first lane; LS loads put
  // the column offset of the upper 16 threads in the instruction (64).
  const uint32_t lane_base = static_cast<uint32_t>(LS ? wq * 32 + half * 16 : wq * 32) << 16;
  const uint32_t tS = tmem + lane_base + t * kTile + (LS ? 0 : col0);
  const uint32_t tO = tmem + lane_base + (NQ + t * DB) * kTile + (LS ? 0 : col0);
  uint8_t* pbase = smem + C::kOffP + t * C::kPBuf * C::kPStride;
  // exchange slots: [t][parity 0,1 = row max, 2 = row sum][half][row]
  float* xch = reinterpret_cast<float*>(smem + C::kOffX) + t * 3 * 2 * kTile;
  uint64_t* xbar = bar.xch + (t * 4 + wq) * 3;

  // KS (the decode): Q's scale and the suffix scales come from the launch
  // this one may overlap; wait for it before the first read.
  if constexpr (KS) griddep_wait();
  if (tracer) RP_TRACE(210 + t, 0);  // softmax: predecessor complete
  const float sq = p.qs[bh * p.qs_bh + q_tile_c * p.qs_blk];

  // Largest V scale this CTA meets (positive floats order like their bits),
  // and the per-step constants c_j / (sm_scale log2 e sq) = sk_j, log2 K_j
  // and 1/K_j with K_j = 448 * sv_j / sv_max, the P scale.
  float sv_max, inv_svmax;
  float cj = 0.f, log2k = 0.f, invk = 0.f;
  float sk_n = 0.f, sv_n = 1.f;
  StepCursor ahead;  // K/V tile of the next scale load (no table)
  auto load_step = [&](int j, float& sk, float& sv) {
    if (p.has_extra && j == p.n_main_tiles) {
      const int idx = bh * p.kvx_bh + q_tile_c * p.kvx_blk;
      sk = p.ksx[idx];
      sv = p.vsx[idx];
    } else {
      const int64_t idx = ahead.c * p.kv_chunk + bh * p.kv_bh + ahead.t * p.kv_blk;
      sk = p.ks[idx];
      sv = p.vs[idx];
      ahead.next(p);
    }
  };
  auto make_consts = [&](float sk, float sv, float& c_out, float& l_out, float& i_out) {
    const float kj = 448.f * sv * inv_svmax;
    c_out = p.sm_scale_log2 * sq * sk;
    l_out = __log2f(kj);
    i_out = __fdividef(1.f, kj);
  };
  float4* tab = reinterpret_cast<float4*>(smem + C::kOffT + 64);
  float4 cst_n = make_float4(0.f, 0.f, 0.f, 0.f);
  // The decode (KS) with at most 32 steps: every softmax warp builds its own
  // copy of the table, lane j holding step j, so the latency-bound prologue
  // has no barrier across warps; the values are those of the shared table
  // below.  (The long-sequence kernels keep the shared table: the per-warp
  // form costs them registers.)
  static_assert(!TAB || C::kSoftmaxWarps * 32 <= C::kTableSteps, "per-warp tables fit");
  const int qt0c = min(KS ? unit_x(p) : unit_x(p) * NQ, p.n_q_tiles - 1);
  if (KS && n_steps <= 32) {
    float sk = 0.f, sv = 0.f;
    if (lane < n_steps) {
      int c, tt, valid;
      bool extra;
      step_info(p, lane, c, tt, valid, extra);
      if (extra) {
        const int idx = bh * p.kvx_bh + qt0c * p.kvx_blk;
        sk = p.ksx[idx];
        sv = p.vsx[idx];
      } else {
        const int64_t idx = c * p.kv_chunk + bh * p.kv_bh + tt * p.kv_blk;
        sk = p.ks[idx];
        sv = p.vs[idx];
      }
    }
    const uint32_t vb = __reduce_max_sync(0xffffffffu, __float_as_uint(sv));
    if (tracer) RP_TRACE(212 + t, 0);  // scale loads back
    sv_max = __uint_as_float(vb);
    inv_svmax = 1.f / sv_max;
    tab += warp * 32;
    if (lane < n_steps) {
      const float kj = 448.f * sv * inv_svmax;
      tab[lane] = make_float4(p.sm_scale_log2 * sk, __log2f(kj), __fdividef(1.f, kj), 0.f);
    }
    __syncwarp();
    if (n_steps > j0) cst_n = tab[j0];
  } else if constexpr (TAB) {
    // All softmax threads fill the table once (n_steps <= kTableSteps); the
    // extra (decode) tile belongs to the CTA's only query tile (NQ == 1).
    constexpr int kN = C::kSoftmaxWarps * 32;
    float* red = reinterpret_cast<float*>(smem + C::kOffT);
    uint32_t vb = 0;
    for (int j = threadIdx.x; j < n_steps; j += kN) {
      int c, tt, valid;
      bool extra;
      step_info(p, j, c, tt, valid, extra);
      float sk, sv;
      if (extra) {
        const int idx = bh * p.kvx_bh + qt0c * p.kvx_blk;
        sk = p.ksx[idx];
        sv = p.vsx[idx];
      } else {
        const int64_t idx = c * p.kv_chunk + bh * p.kv_bh + tt * p.kv_blk;
        sk = p.ks[idx];
        sv = p.vs[idx];
      }
      tab[j] = make_float4(sk, sv, 0.f, 0.f);
      vb = max(vb, __float_as_uint(sv));
    }
    vb = __reduce_max_sync(0xffffffffu, vb);
    if (tracer) RP_TRACE(212 + t, 0);  // scale loads back
    if (lane == 0) red[warp] = __uint_as_float(vb);
    named_bar_sync(1, kN);
    if (tracer) RP_TRACE(214 + t, 0);
    vb = 0;
#pragma unroll
    for (int w = 0; w < C::kSoftmaxWarps; ++w) vb = max(vb, __float_as_uint(red[w]));
    sv_max = __uint_as_float(vb);
    inv_svmax = 1.f / sv_max;
    for (int j = threadIdx.x; j < n_steps; j += kN) {
      const float4 e = tab[j];
      const float kj = 448.f * e.y * inv_svmax;
      tab[j] = make_float4(p.sm_scale_log2 * e.x, __log2f(kj), __fdividef(1.f, kj), 0.f);
    }
    named_bar_sync(1, kN);
    if (n_steps > j0) cst_n = tab[j0];
  } else {
    uint32_t vbits = 0;
    for (int j = lane; j < p.n_main_tiles; j += 32) {
      int c, tt, valid;
      bool extra;
      step_info(p, j, c, tt, valid, extra);
      vbits = max(vbits, __float_as_uint(p.vs[c * p.kv_chunk + bh * p.kv_bh + tt * p.kv_blk]));
    }
    if (p.has_extra && lane == 0)
      vbits = max(vbits, __float_as_uint(p.vsx[bh * p.kvx_bh + q_tile_c * p.kvx_blk]));
    vbits = __reduce_max_sync(0xffffffffu, vbits);
    sv_max = __uint_as_float(vbits);
    inv_svmax = 1.f / sv_max;
    // Without the table the constants are formed one step ahead, after the
    // exp loop, and their scale loads two steps ahead.
    if (n_steps > 0) {
      float sk0, sv0;
      load_step(0, sk0, sv0);
      make_consts(sk0, sv0, cj, log2k, invk);
    }
    if (n_steps > 1) load_step(1, sk_n, sv_n);
  }

  // Rescale threshold: a row's running max m is only raised (and O, l
  // rescaled) when some row of this warp would grow by more than tau; until
  // then p = 2^(s c - m) may reach 2^tau, so P carries an extra 2^-tau.
  const float tau = p.rescale_tau;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;
  if (tracer) RP_TRACE(202 + t, 0);  // softmax prologue (scale table) done
  StepCursor cur;  // K/V tile of step j
  if (KS && j0 == 1 && n_steps > 0 && !(p.has_extra && p.n_main_tiles == 0)) cur.next(p);
  for (int j = j0; j < n_steps; j += kStepStride) {
    const int li = KS ? (j >> 1) : j;  // this warpgroup's step count
    const bool extra = p.has_extra && j == p.n_main_tiles;
    const int tt = cur.t;
    const int valid = extra ? kTile : cur.valid(p);
    if constexpr (TAB) {
      const float4 cst = cst_n;
      if (j + kStepStride < n_steps) cst_n = tab[j + kStepStride];
      cj = cst.x * sq;
      log2k = cst.y;
      invk = cst.z;
    }
    if (tracer) RP_TRACE(100 + t, j);

    if (!warp_wait(bar.s_full + t, li & 1, bar.abort_flag, p.status, kErrWaitS)) {
      ok = false;
      break;
    }
    if (tracer) RP_TRACE(10 + t, j);
    tc_fence_after();
    uint32_t r[NC / 32][32];
#pragma unroll
    for (int q = 0; q < NC / 32; ++q) {
      if constexpr (LS)
        tmem_ld16x2(tS + 32 * q, r[q]);
      else
        tmem_ld32(tS + 32 * q, r[q]);
    }
    tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < NC / 32; ++q) reg_fence(r[q]);
    if (tracer) RP_TRACE(104 + t, j);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar.s_free + t);

    float s[NC];
#pragma unroll
    for (int i = 0; i < NC; ++i) s[i] = __uint_as_float(r[i >> 5][i & 31]);

    if (!extra && valid < kTile) {
#pragma unroll
      for (int i = 0; i < NC; ++i)
        if (col0 + i >= valid) s[i] = -INFINITY;
    }
    if (p.causal) {
      const int rel = (q_tile * kTile + row) - tt * kTile;  // column i allowed iff i <= rel
      if (rel < kTile - 1) {
#pragma unroll
        for (int i = 0; i < NC; ++i)
          if (col0 + i > rel) s[i] = -INFINITY;
      }
    }
    if (extra) {
      const int g0 = (row / p.extra_group) * p.extra_group;  // own candidate's first token
#pragma unroll
      for (int i = 0; i < NC; ++i)
        if (col0 + i < g0 || col0 + i > row) s[i] = -INFINITY;
    }

    // Row max: independent chains of 3-input max (16 columns each), a short tree.
    constexpr int NCH = NC / 16;
    float ach[NCH];
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      float acc = s[16 * k];
#pragma unroll
      for (int jj = 0; jj < 7; ++jj) acc = fmax3f(acc, s[16 * k + 1 + 2 * jj], s[16 * k + 2 + 2 * jj]);
      ach[k] = fmaxf(acc, s[16 * k + 15]);
    }
    float mx = ach[0];
#pragma unroll
    for (int k = 1; k < NCH; ++k) mx = fmaxf(mx, ach[k]);
    if constexpr (LS) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));  // the row's other half
    if constexpr (NSPLIT == 2) {
      // swap partial maxima with the warp that owns the other half of these rows
      xch[((j & 1) * 2 + half) * kTile + row] = mx;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar + (j & 1));
      if (!warp_wait(xbar + (j & 1), (j >> 1) & 1, bar.abort_flag, p.status, kErrWaitX)) {
        ok = false;
        break;
      }
      mx = fmaxf(mx, xch[((j & 1) * 2 + (1 - half)) * kTile + row]);
    }
    if (tracer) RP_TRACE(106 + t, j);
    // Both warps of a split row pair see the same maxima, so they agree on resc.
    const float m_cand = fmaxf(m_run, mx * cj);
    const bool resc = __any_sync(0xffffffffu, m_cand > m_run + tau);
    const float m_new = resc ? m_cand : m_run;
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = resc ? ex2_approx(m_run - m_use) : 1.f;
    const float noff = log2k - tau - m_use;

    // Stagger: tile 1's exp phase starts after tile 0's of the same step, so
    // the two warps sharing an SM sub-partition alternate MUFU-bound and
    // latency-bound phases.  Tile 0 is at most two steps ahead of tile 1 (its
    // S for step j+3 is issued only after tile 1's P of step j, in either MMA
    // order), so four barriers indexed by step mod 4 never run a phase ahead
    // of their waiter.
    // Stagger 3 (ping-pong) also holds tile 0's exp phase of step j until
    // tile 1's of step j - 1 is done, so the two never overlap.
    const bool stag_step =
        !KS && NQ == 2 && NSPLIT == 1 && (p.stagger >= 2 || (p.stagger == 1 && j == 0));
    if (stag_step && t == 1 &&
        !warp_wait(bar.stag + 4 * wq + (j & 3), (j >> 2) & 1, bar.abort_flag, p.status, kErrWaitStag)) {
      ok = false;
      break;
    }
    if (stag_step && p.stagger == 3 && t == 0 && j > 0 &&
        !warp_wait(bar.stag1 + 4 * wq + ((j - 1) & 3), ((j - 1) >> 2) & 1, bar.abort_flag, p.status,
                   kErrWaitStag)) {
      ok = false;
      break;
    }

    // p' = 2^(s * c_j - m + log2 K_j - tau).  Packed f32x2 FMAs form the
    // exponents; EPOLY of every 8 go through the FMA-pipe polynomial, the
    // rest through MUFU ex2; the row sum runs on four packed accumulators.
    uint32_t pk[NC / 4];
    uint32_t pl[(PMODE == 1) ? NC / 4 : 1];
    const uint64_t c2 = pack_f32x2(cj, cj);
    const uint64_t o2 = pack_f32x2(noff, noff);
    uint64_t sacc[4];
#pragma unroll
    for (int i = 0; i < NC / 8; ++i) {
      float x[8], e[8];
#pragma unroll
      for (int h = 0; h < 4; ++h)
        unpack_f32x2(ffma2(pack_f32x2(s[8 * i + 2 * h], s[8 * i + 2 * h + 1]), c2, o2), x[2 * h],
                     x[2 * h + 1]);
#pragma unroll
      for (int k = 0; k < 8 - EPOLY; ++k) e[k] = ex2_approx(x[k]);
#pragma unroll
      for (int k = 8 - EPOLY; k < 8; k += 2) ex2_poly2(x[k], x[k + 1], e[k], e[k + 1]);
      const uint64_t e8 = fadd2(fadd2(pack_f32x2(e[0], e[1]), pack_f32x2(e[2], e[3])),
                                fadd2(pack_f32x2(e[4], e[5]), pack_f32x2(e[6], e[7])));
      sacc[i & 3] = (i < 4) ? e8 : fadd2(sacc[i & 3], e8);
      if constexpr (EPOLY == 0 && PMODE == 0) {
        pk[2 * i] = pack_e4m3x4(e[0], e[1], e[2], e[3]);
        pk[2 * i + 1] = pack_e4m3x4(e[4], e[5], e[6], e[7]);
      } else {
        pk[2 * i] = pack_e4m3x4_or(e[0], e[1], e[2], e[3]);
        pk[2 * i + 1] = pack_e4m3x4_or(e[4], e[5], e[6], e[7]);
      }
      if constexpr (PMODE == 1) {
        pl[2 * i] = pack_e4m3x4_residual(pk[2 * i], e[0], e[1], e[2], e[3]);
        pl[2 * i + 1] = pack_e4m3x4_residual(pk[2 * i + 1], e[4], e[5], e[6], e[7]);
      }
    }
    if (tracer) RP_TRACE(108 + t, j);
    if (stag_step && t == 0) {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar.stag + 4 * wq + (j & 3));
    }
    if (stag_step && p.stagger == 3 && t == 1) {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar.stag1 + 4 * wq + (j & 3));
    }
    // Next step's constants (their MUFU ops queue behind this step's exps and
    // are consumed a whole step later), then the scale loads for step j+2.
    float cj_n = cj, log2k_n = log2k, invk_n = invk;
    if constexpr (!TAB) {
      if (j + 1 < n_steps) make_consts(sk_n, sv_n, cj_n, log2k_n, invk_n);
      if (j + 2 < n_steps) load_step(j + 2, sk_n, sv_n);
    }
    float sum;
    {
      float u0, u1;
      unpack_f32x2(fadd2(fadd2(sacc[0], sacc[1]), fadd2(sacc[2], sacc[3])), u0, u1);
      sum = u0 + u1;
    }

    if (C::kPBuf == 1 && li > 0) {
      if (!warp_wait(bar.o_done + t, (li - 1) & 1, bar.abort_flag, p.status, kErrWaitO)) {
        ok = false;
        break;
      }
    }
    uint8_t* pb = pbase + ((C::kPBuf == 2) ? (li & 1) : 0) * C::kPStride;
    const uint32_t prow = smem_u32(pb) + row * 128;
    constexpr int kChunks = NC / 16;  // 16-byte P chunks of this thread
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      const int kg = (LS ? (lane >> 4) : half) * kChunks + k;
      st_shared_v4(prow + ((kg ^ (row & 7)) << 4), pk[4 * k], pk[4 * k + 1], pk[4 * k + 2],
                   pk[4 * k + 3]);
    }
    if constexpr (PMODE == 1) {
#pragma unroll
      for (int k = 0; k < kChunks; ++k) {
        const int kg = (LS ? (lane >> 4) : half) * kChunks + k;
        st_shared_v4(prow + kTileBytes + ((kg ^ (row & 7)) << 4), pl[4 * k], pl[4 * k + 1],
                     pl[4 * k + 2], pl[4 * k + 3]);
      }
    }
    fence_proxy_async_smem();
    if (tracer) RP_TRACE(20 + t, j);

    // O is rescaled only when the running max moved; only then must PV(j-1)
    // have finished before O is touched.  (P buffer j&1 is already free:
    // S_full(j) was committed after PV(j-2) was issued.)
    if (li > 0 && resc) {
      if (C::kPBuf == 2 &&
          !warp_wait(bar.o_done + t, (li - 1) & 1, bar.abort_flag, p.status, kErrWaitO)) {
        ok = false;
        break;
      }
      if (tracer) RP_TRACE(30 + t, j);
      tc_fence_after();
      const uint64_t a2 = pack_f32x2(alpha, alpha);
#pragma unroll
      for (int q = 0; q < DB * NC / 32; ++q) {
        uint32_t o[32];
        if constexpr (LS)
          tmem_ld16x2(tO + 32 * q, o);
        else
          tmem_ld32(tO + 32 * q, o);
        tmem_wait_ld();
        reg_fence(o);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float u0, u1;
          unpack_f32x2(fmul2(pack_f32x2(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), a2), u0, u1);
          o[i] = __float_as_uint(u0);
          o[i + 1] = __float_as_uint(u1);
        }
        if constexpr (LS)
          tmem_st16x2(tO + 32 * q, o);
        else
          tmem_st32(tO + 32 * q, o);
      }
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar.p_full + 2 * t + (li & 1));
    if (tracer) RP_TRACE(40 + t, j);
    l_run = l_run * alpha + sum * invk;
    m_run = m_new;
    cj = cj_n;
    log2k = log2k_n;
    invk = invk_n;
    if (!extra) cur.next(p);
    if constexpr (KS) {  // the other warpgroup's step
      if (j + 1 < n_steps && !(p.has_extra && j + 1 == p.n_main_tiles)) cur.next(p);
    }
  }

  // The last PV of this tile signals o_final (single use, so the wait is
  // unambiguous even though o_done phases were skipped above).
  if (ok && n_steps > 0)
    ok = warp_wait(bar.o_final + t, 0, bar.abort_flag, p.status, kErrWaitOFinal);
  if constexpr (LS) {
    if (ok) l_run += __shfl_xor_sync(0xffffffffu, l_run, 16);  // the row's other half
  }
  if (ok && NSPLIT == 2) {  // the two halves' row sums
    xch[(2 * 2 + half) * kTile + row] = l_run;
    __syncwarp();
    if (lane == 0) mbar_arrive(xbar + 2);
    ok = warp_wait(xbar + 2, 0, bar.abort_flag, p.status, kErrWaitX);
    if (ok) l_run += xch[(2 * 2 + (1 - half)) * kTile + row];
  }
  if (!ok) return;

  // KS: the two warpgroups swap their row max (the reference point of their
  // O and l) and row sum through the unused Q slot 1; each then weights the
  // two accumulators by 2^(m_t - max) for half of the output columns (32 of
  // each thread's 64, or of each 64-column box), staged in tile 0's buffers.
  float w0 = 1.f, w1 = 0.f;
  bool has1 = false;
  if constexpr (KS) {
    float* ml = reinterpret_cast<float*>(smem + C::kOffQ + C::kQBytes);  // [t][m, l][row]
    const float mu = (m_run == -INFINITY) ? 0.f : m_run;
    ml[(2 * t) * kTile + row] = mu;
    ml[(2 * t + 1) * kTile + row] = l_run;
    __syncwarp();
    if (lane == 0) mbar_arrive(bar.epi + t);
    if (!warp_wait(bar.epi + (1 - t), 0, bar.abort_flag, p.status, kErrWaitEpi)) return;
    const float m0 = ml[row], l0 = ml[kTile + row];
    has1 = n_steps > 1;  // warpgroup 1 ran at least one step (else its O was never written)
    l_run = l0;
    if (has1) {
      const float m1 = ml[2 * kTile + row], l1 = ml[3 * kTile + row];
      const float mm = fmaxf(m0, m1);
      w0 = ex2_approx(m0 - mm);
      w1 = ex2_approx(m1 - mm);
      l_run = l0 * w0 + l1 * w1;
    }
  }
  // Accumulator columns [col, col + 32) of this thread's row (KS: tile 0's,
  // merged in place with tile 1's, both loads in flight together).
  const uint32_t tOe = KS ? tmem + lane_base + NQ * kTile : tO;
  auto load_o = [&](uint32_t (&o)[32], uint32_t col) {
    uint32_t o1[32];
    if constexpr (LS)
      tmem_ld16x2(tOe + col, o);
    else
      tmem_ld32(tOe + col, o);
    if (KS && has1) {
      if constexpr (LS)  // tile 1's accumulator, this thread's half row
        tmem_ld16x2(tOe + DB * kTile + col, o1);
      else
        tmem_ld32(tOe + DB * kTile + col, o1);
    }
    tmem_wait_ld();
    reg_fence(o);
    if (KS && has1) {
      reg_fence(o1);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        o[i] = __float_as_uint(
            __fmaf_rn(__uint_as_float(o[i]), w0, __fmul_rn(__uint_as_float(o1[i]), w1)));
    }
  };
  if (tracer) RP_TRACE(204 + t, 0);  // last PV done: epilogue starts

  // Epilogue: O * (sv_max / 448) / l -> bf16 or fp16, staged in this tile's
  // (now idle) Q and P buffers (KS: tile 0's) and written by TMA: 2 DB boxes
  // of 64 columns in the 128-byte swizzle, or (out_plain, D <= 64) one
  // unswizzled box of D.
  tc_fence_after();
  const float f = (sv_max / 448.f) / l_run;
  const int ts = KS ? 0 : t;
  uint8_t* const pbase_e = smem + C::kOffP + ts * C::kPBuf * C::kPStride;
  auto stage_of = [&](int box) -> uint8_t* {
    return (box & 1) ? pbase_e + (box >> 1) * kTileBytes
                     : smem + C::kOffQ + ts * C::kQBytes + (box >> 1) * kTileBytes;
  };
  auto pack2 = [&](float a, float b) -> uint32_t {
    return p.out_f16 ? pack_half2(a * f, b * f) : pack_bf16x2(a * f, b * f);
  };
  if (NSPLIT == 1 && p.out_plain) {
    const int ncols = p.out_cols;  // 32 or 64
    const uint32_t srow = smem_u32(stage_of(0)) + row * ncols * 2;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      if (cc * 32 < ncols) {
        uint32_t o[32];
        load_o(o, 32 * cc);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float* v = reinterpret_cast<const float*>(o) + 8 * q;
          st_shared_v4(srow + (cc * 4 + q) * 16, pack2(v[0], v[1]), pack2(v[2], v[3]),
                       pack2(v[4], v[5]), pack2(v[6], v[7]));
        }
      }
    }
  } else {
#pragma unroll
    for (int hh = 0; hh < 2 * DB / C::kRowThreads; ++hh) {
      // 64-column box this thread fills
      const int box = LS ? (lane >> 4) : (NSPLIT == 2) ? half : hh;
      const uint32_t srow = smem_u32(stage_of(box)) + row * 128;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        if (KS && cc != t) continue;  // the other warpgroup's half
        uint32_t o[32];
        // LS: the thread's own 64-column half, 32 at a time
        load_o(o, LS ? 32 * cc : 64 * hh + 32 * cc);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int k = cc * 4 + q;
          const float* v = reinterpret_cast<const float*>(o) + 8 * q;
          st_shared_v4(srow + ((k ^ (row & 7)) << 4), pack2(v[0], v[1]), pack2(v[2], v[3]),
                       pack2(v[4], v[5]), pack2(v[6], v[7]));
        }
      }
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (tracer) RP_TRACE(218 + t, 0);  // this warp's part of the output staged
  if (lane == 0) mbar_arrive(KS ? bar.epi2 + t : bar.epi + t);
  if (wq == 0 && lane == 0 && half == 0 && (!KS || t == 0) && q_tile < p.n_q_tiles) {
    const bool staged =
        KS ? mbar_wait(bar.epi2, 0, bar.abort_flag, p.status, kErrWaitEpi) &&
                 mbar_wait(bar.epi2 + 1, 0, bar.abort_flag, p.status, kErrWaitEpi)
           : mbar_wait(bar.epi + t, 0, bar.abort_flag, p.status, kErrWaitEpi);
    if (staged) {
      const int b = bh / p.H, h = bh % p.H;
      if (NSPLIT == 1 && p.out_plain) {
        tma_store_4d(tm_o, stage_of(0), 0, q_tile * kTile, h, b);
      } else {
#pragma unroll
        for (int box = 0; box < 2 * DB; ++box)
          tma_store_4d(tm_o, stage_of(box), box * 64, q_tile * kTile, h, b);
      }
      tma_store_commit();
      tma_store_wait0();
      if (tracer) RP_TRACE(206 + t, 0);  // output stored
    }
  }
}

template <int NQ, int PMODE, int EPOLY, int NSPLIT, bool TAB, int DB, bool KS = false>
__global__ void __launch_bounds__(Cfg<NQ, PMODE, NSPLIT>::kThreads, 1)
    fa8_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v,
                   const __grid_constant__ CUtensorMap tm_kx,
                   const __grid_constant__ CUtensorMap tm_vx,
                   const __grid_constant__ CUtensorMap tm_o, const AttnKernelParams p) {
  using C = Cfg<NQ, PMODE, NSPLIT, TAB, DB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const Bars bar = carve_bars<NQ>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  RP_TRACE_INIT();
  if (threadIdx.x == 0) RP_TRACE(200, 0);  // kernel entry

  if (warp == 0) {
    // The barriers lie back to back from q_full (carve_bars); one lane
    // initialises every 32nd.  Arrival counts: one per softmax warp of a tile
    // for s_free, p_full, epi and epi2, two for the row-max exchange, else one.
    for (int i = lane; i < C::kNumBars; i += 32) {
      uint64_t* b = bar.q_full + i;
      uint32_t count = 1;
      if ((b >= bar.s_free && b < bar.o_done) || (b >= bar.epi && b < bar.fin) ||
          (b >= bar.epi2 && b < bar.epi2 + NQ))
        count = C::kWarpsPerTile;
      else if (b >= bar.xch && b < bar.stag)
        count = 2;
      mbar_init(b, count);
    }
    if (lane == 0) *bar.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc(bar.tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == C::kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tmem_slot;
  if (threadIdx.x == 0) RP_TRACE(201, 0);  // barriers and TMEM ready

  int n_steps = p.n_main_tiles + (p.has_extra ? 1 : 0);
  if (p.causal) {
    const int q_end = KS ? unit_x(p) + 1 : unit_x(p) * NQ + NQ;
    const int last_row = min(p.Sq, q_end * kTile) - 1;
    n_steps = min(n_steps, last_row / kTile + 1);
  }

  if (warp == C::kTmaWarp) {
    if (lane == 0)
      producer<NQ, PMODE, DB, KS>(&tm_q, &tm_k, &tm_v, &tm_kx, &tm_vx, p, bar, smem, n_steps);
  } else if (warp == C::kMmaWarp) {
    if (lane == 0) {
      if (!KS && p.mma_ahead)
        mma_issuer_ahead<NQ, PMODE, DB>(p, bar, smem, tmem, n_steps);
      else
        mma_issuer<NQ, PMODE, DB, KS>(p, bar, smem, tmem, n_steps);
    }
  } else {
    softmax_wg<NQ, PMODE, EPOLY, NSPLIT, TAB, DB, KS>(&tm_o, p, bar, smem, tmem, n_steps);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// The decode launched as a programmatic dependent of the launch before it
// (1, default) or after it completes (0).  REPERCEP_B200_DECODE_PDL overrides
// (read once).
int decode_pdl_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_DECODE_PDL");
    return (e && std::atoi(e) == 0) ? 0 : 1;
  }();
  return v;
}

template <int NQ, int PMODE, int EPOLY, int NSPLIT, bool TAB, int DB, bool KS = false>
cudaError_t launch_one(const AttnMaps& m, const AttnKernelParams& p, int B, int H,
                       cudaStream_t st) {
  using C = Cfg<NQ, PMODE, NSPLIT, TAB, DB>;
  auto kern = fa8_fwd_kernel<NQ, PMODE, EPOLY, NSPLIT, TAB, DB, KS>;
  // Opt in to the large dynamic shared-memory carve-out once per device.
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
  // 1-D grid over work units (the whole problem unless the caller set a range)
  AttnKernelParams pl = p;
  int units = 0;
  if (pl.units_per_bh == 0) {
    pl.unit_base = 0;
    pl.units_per_bh = KS ? p.n_q_tiles : (p.n_q_tiles + NQ - 1) / NQ;
    units = pl.units_per_bh * B * H;
  } else {
    units = p.unit_count;
  }
  if (units <= 0) return cudaSuccess;
  const dim3 grid(units, 1, 1);
  if (KS && decode_pdl_setting()) {
    // The decode may start while its quantize launch finishes (programmatic
    // dependent launch); its kernel waits for that launch before reading Q
    // and the suffix.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(C::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, m.q, m.k, m.v, m.kx, m.vx, m.o, pl);
  }
  kern<<<grid, C::kThreads, C::kSmemBytes, st>>>(m.q, m.k, m.v, m.kx, m.vx, m.o, pl);
  return cudaGetLastError();
}

// Per-step constant table in shared memory (1, default) or constants formed
// in the step loop (0).  REPERCEP_B200_STEP_TABLE overrides (read once).
int step_table_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_STEP_TABLE");
    return (e && std::atoi(e) == 0) ? 0 : 1;
  }();
  return v;
}

// The per-step constant table variant whenever every step fits in it.
template <int NQ, int PMODE, int EPOLY, int NSPLIT, int DB = 1>
cudaError_t launch_variant(const AttnMaps& m, const AttnKernelParams& p, int B, int H,
                           cudaStream_t st) {
  const int n_steps = p.n_main_tiles + (p.has_extra ? 1 : 0);
  if (step_table_setting() && n_steps <= Cfg<NQ, PMODE, NSPLIT, true, DB>::kTableSteps &&
      !(NQ > 1 && p.has_extra))
    return launch_one<NQ, PMODE, EPOLY, NSPLIT, true, DB>(m, p, B, H, st);
  return launch_one<NQ, PMODE, EPOLY, NSPLIT, false, DB>(m, p, B, H, st);
}

// Elements (of every 8) whose exp2 runs on the FMA pipe instead of MUFU.
// REPERCEP_B200_EXP_POLY in {0, 2, 4} overrides the default (read once);
// -1 = the default of the row layout in use.
int exp_poly_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_EXP_POLY");
    if (!e) return -1;
    const int x = std::atoi(e);
    return (x == 0 || x == 2 || x == 4) ? x : -1;
  }();
  return v;
}

// Shared-prefix decode (one query tile per CTA): its K/V steps split between
// the two softmax warpgroups of the two-tile layout (1, default) or one
// warpgroup taking every step (0).  REPERCEP_B200_DECODE_KSPLIT overrides
// (read once).
int decode_ksplit_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_DECODE_KSPLIT");
    return (e && std::atoi(e) == 0) ? 0 : 1;
  }();
  return v;
}

// Softmax row layout (1, 2 or 3 = kLaneSplit, see Cfg).
// REPERCEP_B200_ROW_SPLIT overrides the default (read once).
int split_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_ROW_SPLIT");
    if (!e) return kDefaultRowSplit;
    const int x = std::atoi(e);
    return (x == 2 || x == kLaneSplit) ? x : 1;
  }();
  return v;
}

// Exp-phase stagger of the two query tiles (0 off, 1 first step only, 2 tile 1
// after tile 0 every step, 3 ping-pong: also tile 0 after tile 1's previous).
// REPERCEP_B200_STAGGER overrides the default (read once).
int stagger_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_STAGGER");
    if (!e) return kDefaultStagger;
    const int x = std::atoi(e);
    return (x >= 0 && x <= 3) ? x : kDefaultStagger;
  }();
  return v;
}

// MMA issue order of the attention kernel (1: each tile's PV(i) then its
// QK(i + 2); 0: every tile's QK(j), then every tile's PV(j - 1)).
// REPERCEP_B200_MMA_AHEAD overrides the default (read once); -1 = the default
// of the row layout in use (1 with the lane split, else 0).
int mma_ahead_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_MMA_AHEAD");
    if (!e) return -1;
    return std::atoi(e) != 0 ? 1 : 0;
  }();
  return v;
}

// Online-softmax rescale threshold in log2 units (0 = rescale on every
// growth of a row max).  REPERCEP_B200_RESCALE_TAU in [0, 8] overrides the
// default (read once).
float rescale_tau_setting() {
  static const float v = [] {
    const char* e = std::getenv("REPERCEP_B200_RESCALE_TAU");
    if (!e) return kDefaultRescaleTau;
    const float x = static_cast<float>(std::atof(e));
    return (x >= 0.f && x <= 8.f) ? x : kDefaultRescaleTau;
  }();
  return v;
}

}  // namespace

float attention_rescale_tau() { return rescale_tau_setting(); }

#ifdef RP_PIPELINE_TRACE
extern "C" int rp_trace_setup(void* buf, int cta_x, int cta_y) {
  uint32_t* b = static_cast<uint32_t*>(buf);
  if (cudaMemcpyToSymbol(g_trace_buf, &b, sizeof(b)) != cudaSuccess) return -1;
  if (cudaMemcpyToSymbol(g_trace_x, &cta_x, sizeof(int)) != cudaSuccess) return -1;
  if (cudaMemcpyToSymbol(g_trace_y, &cta_y, sizeof(int)) != cudaSuccess) return -1;
  return 0;
}
#endif

namespace {

// Ragged-last-wave split (0, default; REPERCEP_B200_TAIL_SPLIT=1 turns it on,
// read once).  Measured on B200 it neither helps nor hurts (Cosmos-shaped
// shards of 8 / 16 / 64 (b,h): -0.5 / +1 / 0 %): a one-tile CTA takes about as
// long as a two-tile one, because each softmax warp's own dependency chain,
// not the SM's issue or pipe capacity, sets the time of a K/V step.
int tail_split_setting() {
  static const int v = [] {
    const char* e = std::getenv("REPERCEP_B200_TAIL_SPLIT");
    return (e && std::atoi(e) == 1) ? 1 : 0;
  }();
  return v;
}

int attn_sm_count() {
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

// The two-tile CTAs of a launch fill whole waves of the GPU's SMs (one CTA per
// SM) except the last; when that last wave is at most half full (r CTAs,
// 0 < 2r <= SMs), its 2r query tiles run instead as one-tile CTAs after the
// whole waves, each taking about half of a two-tile CTA's time.  A one-tile
// CTA walks its K/V steps in the same order with the same per-step constants
// as the tile does inside a two-tile CTA, so the output bits are those of the
// single launch: that holds for non-causal attention (a causal CTA's step
// count depends on its last tile) with one thread per row, and the split is
// only made there.
bool tail_split(const AttnKernelParams& p, int B, int H, int ep, int sp, int p_mode,
                AttnKernelParams* main_p, AttnKernelParams* tail_p) {
  // the two-tile and one-tile instances built for it: one thread per row with
  // the default exp split, or the lane split with every exp on MUFU
  const bool built = (sp == 1 && ep == kDefaultExpPoly) || (sp == kLaneSplit && ep == kLaneSplitExpPoly);
  if (!tail_split_setting() || p.causal || p.has_extra || !built || p.units_per_bh != 0)
    return false;
  const int ppb = (p.n_q_tiles + 1) / 2;
  const int64_t units = (int64_t)ppb * B * H;
  const int sms = attn_sm_count();
  const int r = static_cast<int>(units % sms);
  if (r == 0 || 2 * r > sms) return false;
  (void)p_mode;
  *main_p = p;
  main_p->unit_base = 0;
  main_p->units_per_bh = ppb;
  main_p->unit_count = static_cast<int>(units - r);
  // the tiles of the last r two-tile units, in (b,h)-major tile order
  const int64_t first_tile = (units - r) / ppb * p.n_q_tiles + ((units - r) % ppb) * 2;
  *tail_p = p;
  tail_p->unit_base = static_cast<int>(first_tile);
  tail_p->units_per_bh = p.n_q_tiles;
  tail_p->unit_count = static_cast<int>((int64_t)B * H * p.n_q_tiles - first_tile);
  return true;
}

}  // namespace

cudaError_t launch_attention(const AttnMaps& maps, const AttnKernelParams& params, int B,
                             int H, int nq, int p_mode, int db, cudaStream_t st) {
  // the row splits have no plain-output epilogue, no D = 256 and no hi/lo P form
  const int sp = (params.out_plain || db != 1 || p_mode != 0) ? 1 : split_setting();
  const bool lane_split = (nq == 2 && sp == kLaneSplit);
  // measured defaults (Cosmos / cfg2 shapes on B200): the lane split runs
  // every exp on MUFU and issues each tile's next QK right after its PV
  const int ep_env = exp_poly_setting(), ahead_env = mma_ahead_setting();
  const int ep = ep_env >= 0 ? ep_env : (lane_split ? kLaneSplitExpPoly : kDefaultExpPoly);
  AttnKernelParams p = params;
  p.rescale_tau = rescale_tau_setting();
  p.stagger = stagger_setting();
  p.mma_ahead = ahead_env >= 0 ? ahead_env : (lane_split ? 1 : 0);
  if (nq == 2 && db == 1) {
    AttnKernelParams pm, pt;
    if (tail_split(p, B, H, ep, sp, p_mode, &pm, &pt)) {
      cudaError_t e;
      if (p_mode != 0) {
        e = launch_variant<2, 1, 0, 1>(maps, pm, B, H, st);
        return e != cudaSuccess ? e : launch_variant<1, 1, 0, 1>(maps, pt, B, H, st);
      }
      if (sp == kLaneSplit) {
        e = launch_variant<2, 0, kLaneSplitExpPoly, kLaneSplit>(maps, pm, B, H, st);
        return e != cudaSuccess ? e : launch_variant<1, 0, kLaneSplitExpPoly, kLaneSplit>(maps, pt, B, H, st);
      }
      e = launch_variant<2, 0, kDefaultExpPoly, 1>(maps, pm, B, H, st);
      return e != cudaSuccess ? e : launch_variant<1, 0, kDefaultExpPoly, 1>(maps, pt, B, H, st);
    }
  }
  if (db == 2) {
    if (nq != 1) return cudaErrorInvalidValue;
    return (p_mode == 0) ? launch_variant<1, 0, 2, 1, 2>(maps, p, B, H, st)
                         : launch_variant<1, 1, 0, 1, 2>(maps, p, B, H, st);
  }
  if (nq == 2 && p_mode == 0) {
    if (sp == 2) {
      if (ep == 0) return launch_variant<2, 0, 0, 2>(maps, p, B, H, st);
      if (ep == 4) return launch_variant<2, 0, 4, 2>(maps, p, B, H, st);
      return launch_variant<2, 0, 2, 2>(maps, p, B, H, st);
    }
    if (sp == kLaneSplit) {  // EXP_POLY 4 is not built for it: 2 instead
      if (ep == 0) return launch_variant<2, 0, 0, kLaneSplit>(maps, p, B, H, st);
      return launch_variant<2, 0, 2, kLaneSplit>(maps, p, B, H, st);
    }
    if (ep == 0) return launch_variant<2, 0, 0, 1>(maps, p, B, H, st);
    if (ep == 4) return launch_variant<2, 0, 4, 1>(maps, p, B, H, st);
    return launch_variant<2, 0, 2, 1>(maps, p, B, H, st);
  }
  if (nq == 2 && p_mode == 1) return launch_variant<2, 1, 0, 1>(maps, p, B, H, st);
  if (nq == 1 && p_mode == 0) {
    const int n_steps = p.n_main_tiles + (p.has_extra ? 1 : 0);
    if (decode_ksplit_setting() && step_table_setting() && !p.causal &&
        n_steps <= Cfg<2, 0, 1, true, 1>::kTableSteps) {
      // the lane split (its default: every exp on MUFU) or one thread per row
      if (split_setting() == kLaneSplit && !p.out_plain)
        return launch_one<2, 0, 0, kLaneSplit, true, 1, true>(maps, p, B, H, st);
      return launch_one<2, 0, 2, 1, true, 1, true>(maps, p, B, H, st);
    }
    return launch_variant<1, 0, 2, 1>(maps, p, B, H, st);
  }
  if (nq == 1 && p_mode == 1) return launch_variant<1, 1, 0, 1>(maps, p, B, H, st);
  return cudaErrorInvalidValue;
}

}  // namespace rp
