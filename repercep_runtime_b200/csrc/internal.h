// Host/device declarations shared by the .cu files of librepercep_b200.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace rp {

// Records `fmt` as the calling thread's rp_last_error() message; returns code.
int set_last_error(int code, const char* fmt, ...);

// ------------------------------------------------------------- quantize
constexpr int kQuantRows = 128;     // tokens per scale block / per CTA
constexpr int kQuantThreads = 256;  // threads per quantize CTA
constexpr int kMaxQuantJobs = 3;    // Q, K, V in one launch

struct QuantJob {
  const uint16_t* x;   // bf16 / fp16 input, element (b,h,s,d) at b*sB + h*sH + s*sS + d
  int64_t sB, sH, sS;  // element strides (d is unit-stride)
  uint8_t* out;        // e4m3, (B*H, S) rows of out_ld bytes
  float* scales;       // (B*H,) per-(b,h) or (B*H, nblk) per block
};

struct QuantArgs {
  QuantJob job[kMaxQuantJobs];
  int B, H, S, D;
  int in_f16;          // 0: bf16 input, 1: fp16 input
  int out_ld;          // output row pitch in bytes (>= D, multiple of 16; padding zeroed)
  int nblk;            // ceil(S / 128)
  uint32_t* partial;   // per-(b,h) mode: (njobs, B*H, npart) partial amax bits
  int npart;           // per-(b,h) mode: partial slots per (job, b*h), >= nblk
};

// Launchers (return cudaError_t of the launch).
cudaError_t launch_quant_block(const QuantArgs& a, int njobs, cudaStream_t st);
// phases: 1 = partial amax of each 128-token chunk, 2 = scale from the npart
// partials of each (job, b*h) and quantize, 3 = both.
cudaError_t launch_quant_bh(const QuantArgs& a, int njobs, cudaStream_t st, int phases = 3);

// Row-wise quantizer of a linear operand: one scale per row of (rows, cols).
struct QuantRowsArgs {
  const uint16_t* x;   // bf16 / fp16, row r at x + r * ldx (elements; 16-byte aligned rows)
  int64_t ldx;
  int rows, cols;      // cols a multiple of 8
  int in_f16;
  uint8_t* out;        // e4m3, row r at out + r * ldo (bytes)
  int64_t ldo;
  float* scales;       // (rows,)
};
cudaError_t launch_quant_rows(const QuantRowsArgs& a, cudaStream_t st);

// --------------------------------------------------------------- fp8 GEMM
struct GemmParams {
  int M, N, K;
  int tiles_m, tiles_n, tiles, n_kb;  // filled by launch_fp8_gemm
  int group_m;                        // row tiles per raster group (0: default)
  // Dequant scales: row m uses sa[m * sa_stride] (sa_stride 0: one device
  // scalar) or a_scale when sa is null; columns likewise with sb / b_scale.
  const float* sa;
  int64_t sa_stride;
  float a_scale;
  const float* sb;
  int64_t sb_stride;
  float b_scale;
  const uint16_t* bias;  // (N,) in the output dtype, or null
  void* C;               // 16-bit output, row m at C + m * ldc (elements)
  int64_t ldc;
  int vec_store;         // C and ldc allow 16-byte stores
  int* status;           // device status word (0 = ok)
  // Fused QKV quantize (qkv_S > 0; B (N, K), bf16 rounding): the rows are
  // M / qkv_S batches of qkv_S tokens and the N = 3 * qkv_H * 128 columns are
  // Q, K, V of qkv_H heads.  Instead of writing C, every 128-token block of
  // every (batch, head) of Q, K and V is quantized to e4m3, as the attention
  // quantizer's per-block mode does on C: qkv_out[i] (B * H, S, 128) e4m3 and
  // qkv_scales[i] (B * H, qkv_nblk) fp32.  qkv_per_b (row tiles per batch) is
  // filled by launch_fp8_gemm.
  int qkv_S, qkv_H, qkv_nblk, qkv_per_b;
  uint8_t* qkv_out[3];
  float* qkv_scales[3];
};

// b_kmajor: B is (N, K) with K contiguous; otherwise (K, N) with N contiguous.
// A fused QKV quantize (p.qkv_S > 0) needs b_kmajor and a bf16 rounding.
cudaError_t launch_fp8_gemm(const CUtensorMap& a, const CUtensorMap& b, GemmParams p,
                            bool b_kmajor, bool out_f16, cudaStream_t st);
// Rows of the B box the selected kernel loads per K block (K-major B: the
// N rows of one CTA; N-major B: 128 K rows).
int gemm_b_box_rows(bool b_kmajor);
bool gemm_pair_setting();

// ------------------------------------------------------------ attention
struct AttnKernelParams {
  int H;                 // heads (bh -> (b, h) for the output map)
  int Sq;                // query rows per (b,h)
  int n_q_tiles;         // ceil(Sq / 128)
  // Main K/V source: n_chunks chunks; all but the last hold chunk_len rows
  // (a multiple of 128), the last holds last_len rows.
  int n_chunks, tiles_per_chunk, chunk_len, last_len, n_main_tiles;
  // Extra K/V tile per query tile (shared-prefix decode suffix).
  int has_extra, extra_group;
  // Scales (dequant multipliers).
  const float* qs;
  int qs_bh, qs_blk;
  const float* ks;
  const float* vs;
  int64_t kv_chunk;      // scale index = c*kv_chunk + bh*kv_bh + t*kv_blk
  int kv_bh, kv_blk;
  const float* ksx;
  const float* vsx;
  int kvx_bh, kvx_blk;   // extra scale index = bh*kvx_bh + qtile*kvx_blk
  float sm_scale_log2;   // softmax scale * log2(e)
  // Online-softmax rescale threshold (log2 units, >= 0): O and the row sum
  // are rescaled only when some row's max grows by more than this; P is
  // scaled by 2^-rescale_tau so a stale max never saturates e4m3.
  float rescale_tau;
  // Two-tile exp stagger: 0 off, 1 at the first step only, 2 every step, 3
  // ping-pong (tile 0 also waits for tile 1's exp phase of the previous step).
  int stagger;
  // MMA issue order (not the decode): 1 = per step i, each tile's PV(i) and
  // then that tile's QK(i + 2), so a tile's next S never waits behind another
  // tile's P; 0 = every tile's QK(j), then every tile's PV(j - 1).
  int mma_ahead;
  int causal;
  // Work units of a launch (1-D grid): CTA i takes unit u = unit_base + i,
  // which is column u % units_per_bh (a group of NQ query tiles, or one query
  // tile for the split-step form) of (b,h) u / units_per_bh.  units_per_bh 0:
  // the whole problem (set by launch_attention).
  int unit_base, units_per_bh;
  int unit_count;        // units in this launch (host side)
  // Output: fp16 instead of bf16; out_plain = one unswizzled box of out_cols
  // (32 or 64) columns instead of 64-column swizzled boxes.
  int out_f16, out_plain, out_cols;
  int* status;           // device status word (0 = ok)
};

struct AttnMaps {
  CUtensorMap q, k, v, kx, vx, o;
};

// Rescale threshold the attention launches use (see rp_attn_rescale_tau).
float attention_rescale_tau();

// nq: query tiles per CTA (1 or 2); db: head dim in 128-column blocks (1, or
// 2 for D = 256, which needs nq = 1).
cudaError_t launch_attention(const AttnMaps& maps, const AttnKernelParams& p, int B, int H,
                             int nq, int p_mode, int db, cudaStream_t st);

}  // namespace rp
