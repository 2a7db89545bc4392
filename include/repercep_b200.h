/*
 * repercep_b200.h — C ABI of librepercep_b200.so, the B200 (sm_100a) FP8
 * attention hot path of repercep-runtime.
 *
 * Conventions (every entry point):
 *   - plain pointers and sizes, no framework types; device pointers are CUDA
 *     device memory owned by the caller; `stream` is a cudaStream_t (NULL =
 *     legacy default stream);
 *   - asynchronous and stream-ordered; no host synchronisation, no device
 *     allocation;
 *   - return RP_OK (0) or a negative rp_status; the message of the calling
 *     thread's last failure is available from rp_last_error();
 *   - bf16 inputs/outputs are addressed by element strides with the head
 *     dimension unit-stride, so (B,H,S,D) and (B,S,H,D) tensors both work
 *     without a transposing copy;
 *   - e4m3 tensors produced here are contiguous (B*H, S, D);
 *   - scale tensors are fp32 dequant multipliers: (B*H) for RP_SCALE_PER_BH,
 *     (B*H, ceil(S/128)) for RP_SCALE_PER_BLOCK128.
 *
 * Reference interfaces replaced (paths inside miteshs/repercep-runtime):
 *   rp_quant_fp8_e4m3      <- _per_bh_scale + _quantize,
 *                             kernels/triton_kernels/fp8_flash_attn_hopper.py:374-398
 *   rp_attn_fp8_fwd        <- _fp8_flash_attn_fwd_impl launch inside
 *                             fp8_flash_attention, fp8_flash_attn_hopper.py:432-586
 *   rp_attn_fp8_fwd_chunked<- (no reference counterpart: the reference refuses
 *                             context parallelism, attention/diffusers_backend.py:199-212)
 *   rp_attn_fp8_prefix_decode <- (no reference kernel: the reference expands the
 *                             prompt per candidate, scripts/run_vla_openvla_gpu.py:174-186)
 *   rp_fp8_gemm            <- fp8_gemm_launch, kernels/hip/fp8_attn/fp8_gemm.hip:162-179
 *                             (bound by fp8_gemm, kernels/hip/fp8_attn/binding.cpp:24-61)
 *   rp_fp8_gemm_ex, rp_quant_fp8_rows <- (no reference kernel: FP8 DiT linears are the
 *                             reference's planned use of that GEMM, docs/OPTIMIZATION.md:161-162)
 *   rp_quant_fp8_e4m3_bh_phase <- _per_bh_scale + _quantize split at the amax, for a sequence
 *                             split across devices (the reference has no context parallelism)
 *   rp_fp8_gemm_qkv_quant  <- the QKV projection followed by the eager quantize of Q, K, V,
 *                             fp8_flash_attn_hopper.py:474-480 (per-128-token-block mode)
 */
#ifndef REPERCEP_B200_H_
#define REPERCEP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RP_ABI_VERSION 4

typedef enum rp_status {
  RP_OK = 0,
  RP_ERR_INVALID = -1,     /* bad argument (null pointer, negative size, ...) */
  RP_ERR_UNSUPPORTED = -2, /* shape or mode this build does not implement */
  RP_ERR_ALIGN = -3,       /* pointer or stride alignment the TMA unit rejects */
  RP_ERR_ARCH = -4,        /* current device is not sm_100 */
  RP_ERR_CUDA = -5,        /* CUDA runtime/driver error (see rp_last_error) */
  RP_ERR_WORKSPACE = -6    /* workspace missing or too small */
} rp_status;

typedef enum rp_scale_mode {
  RP_SCALE_PER_BH = 0,       /* one scale per (b,h): the reference's semantics */
  RP_SCALE_PER_BLOCK128 = 1  /* one scale per 128-token block of each (b,h) */
} rp_scale_mode;

typedef enum rp_p_mode {
  RP_P_E4M3 = 0,      /* P rounded once to e4m3 (reference precision) */
  RP_P_E4M3_HILO = 1  /* P split into e4m3 hi + lo planes, two PV MMAs */
} rp_p_mode;

typedef enum rp_dtype {
  RP_DTYPE_BF16 = 0,
  RP_DTYPE_F16 = 1
} rp_dtype;

/* ABI version compiled into the library (RP_ABI_VERSION). */
int rp_abi_version(void);

/* NUL-terminated message of the calling thread's last failed call ("" if none). */
const char* rp_last_error(void);

/* Device status word written by kernels whose internal pipeline timed out
 * (0 = healthy).  Reads it for the current device (synchronises the device);
 * when `reset` is non-zero it is cleared afterwards.  Diagnostic only. */
int rp_device_status(int* status, int reset);

/* Diagnostic: one warp waits, bounded by limit_cycles SM cycles (at most the
 * kernels' own limit), on a barrier nothing arrives on -- the wait every
 * pipeline role uses -- and records 0x1FF in the device status word when it
 * runs out, as a timed-out pipeline would.  Shows that a timeout is reported
 * through rp_device_status and leaves the context usable.  No reference
 * counterpart. */
int rp_selftest_wait_timeout(long long limit_cycles, void* stream);

/* Online-softmax rescale threshold (log2 units) the attention kernels use:
 * O and the row sums are rescaled only when a row max grows by more than
 * this, and P is rounded at 2^-tau of its usual scale meanwhile (0 = rescale
 * on every growth, as the reference kernel does).  Set once per process by
 * REPERCEP_B200_RESCALE_TAU (0..8); default 1.  No reference counterpart. */
float rp_attn_rescale_tau(void);

/* Workspace bytes rp_quant_fp8_e4m3 needs (0 for RP_SCALE_PER_BLOCK128). */
int rp_quant_workspace_bytes(int num_tensors, int B, int H, int S, int D, int scale_mode,
                             size_t* bytes);

/* Quantise `num_tensors` (1..3) bf16 tensors of one shape (B,H,S,D) to e4m3.
 *   x[i]       bf16 input, element (b,h,s,d) at x[i] + b*strides[4i] +
 *              h*strides[4i+1] + s*strides[4i+2] + d (strides[4i+3] must be 1)
 *   out[i]     e4m3 output, contiguous (B*H, S, D)
 *   scales[i]  fp32 dequant scales (layout per scale_mode)
 * Replaces _per_bh_scale/_quantize (fp8_flash_attn_hopper.py:374-398);
 * bytes and scales are bit-identical to them for RP_SCALE_PER_BH. */
int rp_quant_fp8_e4m3(int num_tensors, const void* const* x, const int64_t* strides, int B, int H,
                      int S, int D, int scale_mode, void* const* out, float* const* scales,
                      void* workspace, size_t workspace_bytes, void* stream);

/* rp_quant_fp8_e4m3 for bf16 or fp16 input (in_dtype, an rp_dtype) and
 * e4m3 rows of out_row_bytes (>= D, multiple of 16; bytes D.. of every row are
 * written as zero, which pads D = 32 / 64 to the 128-byte rows the attention
 * kernel reads).  fp16 follows the reference's steps in fp16: amax and its
 * 1e-6 floor in fp16, scale rounded to fp16 (fp8_flash_attn_hopper.py:374-398
 * on an fp16 tensor).  rp_quant_fp8_e4m3 is this with bf16 and out_row_bytes = D. */
int rp_quant_fp8_e4m3_ex(int num_tensors, const void* const* x, const int64_t* strides, int B,
                         int H, int S, int D, int in_dtype, int scale_mode, void* const* out,
                         int out_row_bytes, float* const* scales, void* workspace,
                         size_t workspace_bytes, void* stream);

/* The two phases of the per-(b,h) quantizer, for a sequence split across
 * devices (context parallelism): the reference's per-(b,h) scale
 * (_per_bh_scale, fp8_flash_attn_hopper.py:374-385) is an amax over the whole
 * sequence, so each device computes the partial amax of its own tokens, the
 * devices combine them with an element-wise max, and each quantizes its
 * tokens with the common scale.
 *   RP_QUANT_PHASE_AMAX   writes the |x| max (bit patterns; NaN above +inf) of
 *                         each 128-token chunk of each (tensor, b, h) to
 *                         partials[(i * B*H + bh) * npart + chunk] for chunk <
 *                         ceil(S/128); the other slots are left as they are
 *                         (zero them: 0 is the max's identity);
 *   RP_QUANT_PHASE_APPLY  takes each (tensor, b, h)'s scale from the max of
 *                         its npart slots and quantizes x into out / scales
 *                         exactly as rp_quant_fp8_e4m3_ex (RP_SCALE_PER_BH).
 * Combining the partial arrays of all devices with an element-wise integer
 * max (e.g. an all-reduce MAX on int32) between the phases gives every device
 * the scales of the whole sequence, and bytes identical to quantizing the
 * whole sequence on one device.  npart >= ceil(S/128).  The amax phase reads
 * no out / scales (they may be NULL). */
enum { RP_QUANT_PHASE_AMAX = 1, RP_QUANT_PHASE_APPLY = 2 };
int rp_quant_fp8_e4m3_bh_phase(int phase, int num_tensors, const void* const* x,
                               const int64_t* strides, int B, int H, int S, int D, int in_dtype,
                               uint32_t* partials, int npart, void* const* out, int out_row_bytes,
                               float* const* scales, void* stream);

/* Allocation-free variant of rp_quant_fp8_e4m3 for RP_SCALE_PER_BH (no
 * counterpart in the reference, which always allocates through PyTorch).
 * For callers that cannot provide device memory beyond their inputs and
 * outputs: e.g. a plugin whose host passes it only the tensors it reads and
 * writes and whose memory pool forbids raw cudaMalloc.  The per-(b,h) scratch
 * (one uint32 partial amax per 128-token chunk) lives in a fixed 1 MiB
 * library-owned device array per device (held until exit); shapes needing
 * more than 262144 slots (num_tensors * B * H * ceil(S/128)) are rejected
 * with RP_ERR_WORKSPACE.  All calls on a device share that array: calls whose
 * kernels may overlap on the GPU race and must be serialised (one stream).
 * Each call writes every slot it reads, so no clearing is needed.  The first
 * call on a device looks up the array's device address; make it before any
 * stream capture.  Bytes and scales equal rp_quant_fp8_e4m3's. */
int rp_quant_fp8_e4m3_noalloc(int num_tensors, const void* const* x, const int64_t* strides,
                              int B, int H, int S, int D, void* const* out,
                              float* const* scales, void* stream);

/* FP8 attention forward, non-causal or causal (top-left aligned mask, as the
 * reference's offs_m >= offs_n).  q8 (B*H, Sq, D), k8/v8 (B*H, Skv, D) e4m3
 * contiguous; qs/ks/vs dequant scales in `scale_mode` layout; out bf16
 * (B,H,Sq,D) addressed by out_strides[4] (elements; last must be 1).
 * sm_scale <= 0 selects 1/sqrt(D).  D must be 128 (other head dims: _ex).
 * Replaces the kernel launch of fp8_flash_attention (fp8_flash_attn_hopper.py:432-586). */
int rp_attn_fp8_fwd(const void* q8, const void* k8, const void* v8, const float* qs,
                    const float* ks, const float* vs, int scale_mode, int B, int H, int Sq,
                    int Skv, int D, float sm_scale, int causal, int p_mode, void* out,
                    const int64_t* out_strides, void* stream);

/* rp_attn_fp8_fwd for every head dim the reference's op advertises
 * (fp8_hopper_triton.py:41: 32, 64, 128, 256) and both output dtypes.
 *   qkv_row_bytes  e4m3 row pitch of q8/k8/v8: 128 for D <= 128 (rows of
 *                  D = 32 / 64 zero-padded to 128 bytes, as
 *                  rp_quant_fp8_e4m3_ex(out_row_bytes = 128) writes them),
 *                  256 for D = 256
 *   out_dtype      RP_DTYPE_BF16 or RP_DTYPE_F16 (the reference returns the
 *                  query's dtype, fp8_flash_attn_hopper.py:586); out has D
 *                  columns, strides multiples of 8 elements
 * sm_scale <= 0 selects 1/sqrt(D) for the true D. */
int rp_attn_fp8_fwd_ex(const void* q8, const void* k8, const void* v8, const float* qs,
                       const float* ks, const float* vs, int scale_mode, int B, int H, int Sq,
                       int Skv, int D, int qkv_row_bytes, float sm_scale, int causal, int p_mode,
                       void* out, const int64_t* out_strides, int out_dtype, void* stream);

/* Context-parallel variant: K/V arrive as `n_chunks` chunks (one per rank),
 * laid out (n_chunks, B*H, chunk_rows, D) e4m3; every chunk holds chunk_rows
 * valid rows except the last, which holds last_rows.  chunk_rows must be a
 * multiple of 128 when n_chunks > 1.  Scales are per 128-row block:
 * (n_chunks, B*H, ceil(chunk_rows/128)).  q8/qs as rp_attn_fp8_fwd with
 * RP_SCALE_PER_BLOCK128.  Non-causal. */
int rp_attn_fp8_fwd_chunked(const void* q8, const void* k8, const void* v8, const float* qs,
                            const float* ks, const float* vs, int B, int H, int Sq,
                            int n_chunks, int chunk_rows, int last_rows, int D, float sm_scale,
                            int p_mode, void* out, const int64_t* out_strides, void* stream);

/* Shared-prefix candidate decode.  C candidates x T new tokens per head:
 *   q8   (H, C*T, D)   e4m3, qs (H, ceil(C*T/128)) per-block scales
 *   kp8, vp8 (H, P, D) e4m3 shared prefix, kps/vps (H, ceil(P/128))
 *   kx8, vx8 (H, C*T, D) e4m3 per-candidate suffix, kxs/vxs (H, ceil(C*T/128))
 *   out  bf16 (C*T, H, D) addressed by out_strides[3] = {token, head, d}
 * Candidate c's token i attends to the whole prefix and to its own suffix
 * tokens 0..i.  Every query tile reads each prefix K/V tile once; 128 % T
 * must be 0.  (No reference kernel: the reference duplicates the prefix per
 * candidate, scripts/run_vla_openvla_gpu.py:174-186.) */
int rp_attn_fp8_prefix_decode(const void* q8, const void* kp8, const void* vp8,
                              const void* kx8, const void* vx8, const float* qs,
                              const float* kps, const float* vps, const float* kxs,
                              const float* vxs, int C, int T, int P, int H, int D,
                              float sm_scale, int p_mode, void* out,
                              const int64_t* out_strides, void* stream);

/* ------------------------------------------------------------ FP8 GEMM
 * C = A @ B on the tensor cores with e4m3 operands and an fp32 accumulator.
 *
 * rp_fp8_gemm is the reference's fp8_gemm_launch: A (M, K) and B (K, N)
 * row-major e4m3, C (M, N) row-major bf16, all contiguous,
 *   C = bf16_rne(acc * (a_scale * b_scale)).
 * e4m3 is the OCP e4m3fn encoding (torch.float8_e4m3fn) that B200 computes
 * in; the reference's gfx942 operands are e4m3fnuz.  The TMA unit needs
 * 16-byte row pitches: K and N must be multiples of 16 here
 * (rp_fp8_gemm_ex takes padded pitches). */
typedef enum rp_b_layout {
  RP_B_KN = 0, /* B is (K, N), N contiguous (the reference's layout)       */
  RP_B_NK = 1  /* B is (N, K), K contiguous (an nn.Linear weight)           */
} rp_b_layout;

int rp_fp8_gemm(const void* a, const void* b, void* c, float a_scale, float b_scale, int M,
                int N, int K, void* stream);

/* General form, for FP8 linears:
 *   C[m, n] = out( acc[m, n] * (sa_m * sb_n) + bias[n] )
 *   a      (M, K) e4m3, row m at a + m * lda bytes (lda % 16 == 0)
 *   b      RP_B_KN: (K, N), row k at b + k * ldb bytes; RP_B_NK: (N, K),
 *          row n at b + n * ldb bytes (ldb % 16 == 0)
 *   sa_m   = sa[m * sa_stride] (sa_stride 0: one device scalar), or a_scale
 *            when sa is NULL; sb_n likewise with sb / sb_stride / b_scale
 *   bias   NULL or (N,) in the output dtype
 *   c      (M, N) bf16 or fp16 (out_dtype, an rp_dtype), row m at
 *          c + m * ldc elements
 * The product of the two scales is formed first, then acc times it, then the
 * bias is added (fp32, round to nearest) and the sum rounded to the output
 * dtype.  K may be any size (the tensor map zero-fills past K). */
int rp_fp8_gemm_ex(const void* a, int64_t lda, const void* b, int64_t ldb, int b_layout,
                   const float* sa, int64_t sa_stride, float a_scale, const float* sb,
                   int64_t sb_stride, float b_scale, const void* bias, void* c, int64_t ldc,
                   int out_dtype, int M, int N, int K, void* stream);

/* The QKV projection with the attention quantizer fused into its epilogue.
 * Replaces the reference's eager quantize of Q, K and V right before its
 * kernel (kernels/triton_kernels/fp8_flash_attn_hopper.py:474-480) for the
 * per-128-token-block scale mode: the projection's bf16 output is never
 * written.
 *   a      (B*S, K) e4m3 activations, row m at a + m * lda bytes (lda % 16 == 0);
 *          rows are B batches of S tokens
 *   w      (N, K) e4m3 weight, N = 3 * H * 128 (the Q, K, V projections
 *          stacked, each head-major), row n at w + n * ldw bytes (ldw % 16 == 0)
 *   sa, sa_stride, a_scale, sb, sb_stride, b_scale, bias (bf16 (N,) or NULL)
 *          as in rp_fp8_gemm_ex
 *   q8, k8, v8   (B*H, S, 128) e4m3 each (16-byte aligned)
 *   qs, ks, vs   (B*H, ceil(S/128)) fp32 each
 * The result is bit for bit what rp_fp8_gemm_ex (bf16 output) followed by
 * rp_quant_fp8_e4m3 (RP_SCALE_PER_BLOCK128) on the (B, S, 3, H, 128) view of
 * that output produce. */
int rp_fp8_gemm_qkv_quant(const void* a, int64_t lda, const void* w, int64_t ldw,
                          const float* sa, int64_t sa_stride, float a_scale, const float* sb,
                          int64_t sb_stride, float b_scale, const void* bias, int B, int S,
                          int H, int K, void* q8, void* k8, void* v8, float* qs, float* ks,
                          float* vs, void* stream);

/* Row-wise e4m3 quantizer for linear operands: x (rows, cols) bf16 or fp16
 * (in_dtype), row r at x + r * ldx elements (16-byte aligned rows, cols % 8
 * == 0), to out (rows, cols) e4m3 with row pitch ldo bytes (ldo % 8 == 0)
 * and scales[r] (fp32 dequant multiplier).  Each row is one scale group of
 * rp_quant_fp8_e4m3's recipe (amax, 1e-6 floor, amax/425.6 rounded to the
 * input format, reciprocal, clamp, e4m3 RNE): per-token activation scales
 * for the A operand, per-output-channel weight scales for an RP_B_NK B. */
int rp_quant_fp8_rows(const void* x, int64_t ldx, int in_dtype, int rows, int cols, void* out,
                      int64_t ldo, float* scales, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* REPERCEP_B200_H_ */
