// extern "C" entry points of librepercep_b200.so (declared in
// include/repercep_b200.h): argument checking, TMA descriptor encoding and
// kernel launch.  No exception crosses the boundary; failures return a
// negative rp_status and leave a message for rp_last_error().
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "repercep_b200.h"
#include "internal.h"
#include "ptx.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(RP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Device status word: kernels whose pipeline wait timed out record a code.
__device__ int g_rp_status;

struct DeviceState {
  bool probed = false;
  bool sm100 = false;
  int* status = nullptr;
};
std::mutex g_mu;
DeviceState g_dev[64];

// Checks that the current device is sm_100 and returns its status word.
int device_ready(int** status) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(RP_ERR_INVALID, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (!d.probed) {
    int major = 0, minor = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    d.sm100 = (major == 10 && minor == 0);
    if (d.sm100) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_rp_status);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
      d.status = static_cast<int*>(p);
    }
    d.probed = true;
  }
  if (!d.sm100) return fail(RP_ERR_ARCH, "device %d is not sm_100 (B200); this library is sm_100a only", dev);
  *status = d.status;
  return RP_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                        &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Rank-4 tiled map.  strides[] are byte strides of dims 1..3.  A dimension
// of extent 1 gets a harmless stride so the encoder's checks pass.
int make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, const uint64_t dims[4],
             uint64_t strides[3], const uint32_t box[4], const char* what,
             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return fail(RP_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return fail(RP_ERR_ALIGN, "%s: base address must be 16-byte aligned", what);
  for (int i = 0; i < 3; ++i) {
    if (dims[i + 1] == 1) strides[i] = (i == 0) ? 16 * ((dims[0] * 2 + 15) / 16) : strides[i - 1];
    if (strides[i] % 16 != 0)
      return fail(RP_ERR_ALIGN, "%s: byte stride %llu of dim %d is not a multiple of 16", what,
                  (unsigned long long)strides[i], i + 1);
  }
  const uint32_t elem_strides[4] = {1, 1, 1, 1};
  CUresult r = fn(m, dt, 4, const_cast<void*>(base), dims, strides, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RP_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return RP_OK;
}

// e4m3 operand stored (chunks, rows_per_chunk, bh, row_bytes) with row_bytes
// 128 or 256: 128x128-byte boxes (two per row block when row_bytes = 256).
int make_fp8_map(CUtensorMap* m, const void* base, int rows, int bh, int chunks, const char* what,
                 int row_bytes = 128) {
  const uint64_t rb = static_cast<uint64_t>(row_bytes);
  const uint64_t dims[4] = {rb, (uint64_t)rows, (uint64_t)bh, (uint64_t)chunks};
  uint64_t strides[3] = {rb, (uint64_t)rows * rb, (uint64_t)rows * rb * bh};
  const uint32_t box[4] = {128, 128, 1, 1};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, dims, strides, box, what);
}

// 16-bit output (B, H, S, D) with element strides {sB, sH, sS}: 64-column
// boxes in the 128-byte swizzle per 128-row tile for D >= 128, one
// unswizzled box of all D columns for D = 32 / 64.
int make_out_map(CUtensorMap* m, void* base, int B, int H, int S, int64_t sB, int64_t sH,
                 int64_t sS, int D = 128, bool f16 = false) {
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  uint64_t strides[3] = {(uint64_t)sS * 2, (uint64_t)sH * 2, (uint64_t)sB * 2};
  const bool plain = D < 128;
  const uint32_t box[4] = {plain ? (uint32_t)D : 64u, 128, 1, 1};
  return make_map(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base,
                  dims, strides, box, "out",
                  plain ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B);
}

// e4m3 matrix of `rows` rows of `cols` bytes, `ld` bytes apart: boxes of 128
// bytes x box_rows rows in the 128-byte swizzle (zero fill past the edges).
int make_mat8_map(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int64_t ld,
                  uint32_t box_rows, const char* what) {
  const uint64_t dims[4] = {(uint64_t)cols, (uint64_t)rows, 1, 1};
  uint64_t strides[3] = {(uint64_t)ld, (uint64_t)ld * rows, (uint64_t)ld * rows};
  const uint32_t box[4] = {128, box_rows, 1, 1};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, dims, strides, box, what);
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

int ceil_div(int a, int b) { return (a + b - 1) / b; }

constexpr float kLog2e = 1.4426950408889634f;

}  // namespace

namespace rp {
int set_last_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}
}  // namespace rp

namespace {

constexpr int kSelftestCode = 0x1FF;

// One warp waits, bounded, on an mbarrier nothing ever arrives on: the same
// wait every pipeline role uses, run out on purpose.
__global__ void wait_selftest_kernel(int* status, long long limit) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    rp::mbar_init(&bar, 1);
    abort_flag = 0;
    rp::fence_barrier_init();
  }
  __syncthreads();
  rp::mbar_wait(&bar, 0, &abort_flag, status, kSelftestCode, limit);
  __syncthreads();
}

}  // namespace

extern "C" {

int rp_abi_version(void) { return RP_ABI_VERSION; }

int rp_selftest_wait_timeout(long long limit_cycles, void* stream) {
  if (limit_cycles <= 0 || limit_cycles > rp::kWaitLimitCycles)
    return fail(RP_ERR_INVALID, "limit_cycles must be in (0, %lld]", rp::kWaitLimitCycles);
  int* status = nullptr;
  int rc = device_ready(&status);
  if (rc != RP_OK) return rc;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_cycles);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  return RP_OK;
}

const char* rp_last_error(void) { return g_last_error.c_str(); }

float rp_attn_rescale_tau(void) { return rp::attention_rescale_tau(); }

int rp_device_status(int* status, int reset) {
  if (!status) return fail(RP_ERR_INVALID, "status is null");
  int* dummy = nullptr;
  int rc = device_ready(&dummy);
  if (rc != RP_OK) return rc;
  cudaError_t e = cudaMemcpyFromSymbol(status, g_rp_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_rp_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "reset status");
  }
  return RP_OK;
}

int rp_quant_workspace_bytes(int num_tensors, int B, int H, int S, int D, int scale_mode,
                             size_t* bytes) {
  if (!bytes) return fail(RP_ERR_INVALID, "bytes is null");
  if (num_tensors < 1 || num_tensors > rp::kMaxQuantJobs || B <= 0 || H <= 0 || S <= 0 || D <= 0)
    return fail(RP_ERR_INVALID, "bad quantize shape");
  if (scale_mode == RP_SCALE_PER_BLOCK128) {
    *bytes = 0;
  } else if (scale_mode == RP_SCALE_PER_BH) {
    *bytes = (size_t)num_tensors * B * H * ceil_div(S, rp::kQuantRows) * sizeof(uint32_t);
  } else {
    return fail(RP_ERR_INVALID, "unknown scale_mode %d", scale_mode);
  }
  return RP_OK;
}

int rp_quant_fp8_e4m3(int num_tensors, const void* const* x, const int64_t* strides, int B, int H,
                      int S, int D, int scale_mode, void* const* out, float* const* scales,
                      void* workspace, size_t workspace_bytes, void* stream) {
  return rp_quant_fp8_e4m3_ex(num_tensors, x, strides, B, H, S, D, RP_DTYPE_BF16, scale_mode, out,
                              D, scales, workspace, workspace_bytes, stream);
}

namespace {

// Checks shared by the quantizer entry points; fills `a` (without partials).
int quant_args(int num_tensors, const void* const* x, const int64_t* strides, int B, int H, int S,
               int D, int in_dtype, void* const* out, int out_row_bytes, float* const* scales,
               rp::QuantArgs* a, bool need_out = true) {
  if (in_dtype != RP_DTYPE_BF16 && in_dtype != RP_DTYPE_F16)
    return fail(RP_ERR_UNSUPPORTED, "input dtype %d is neither bf16 nor fp16", in_dtype);
  if (out_row_bytes < D || out_row_bytes % 16)
    return fail(RP_ERR_INVALID, "out_row_bytes %d must be >= D (%d) and a multiple of 16",
                out_row_bytes, D);
  if (num_tensors < 1 || num_tensors > rp::kMaxQuantJobs)
    return fail(RP_ERR_INVALID, "num_tensors must be 1..3 (got %d)", num_tensors);
  if (!x || !strides || (need_out && (!out || !scales)))
    return fail(RP_ERR_INVALID, "null argument array");
  if (B <= 0 || H <= 0 || S <= 0) return fail(RP_ERR_INVALID, "B, H, S must be positive");
  if (D != 32 && D != 64 && D != 128 && D != 256)
    return fail(RP_ERR_UNSUPPORTED, "head_dim %d not in {32,64,128,256}", D);
  if ((int64_t)B * H > 65535) return fail(RP_ERR_UNSUPPORTED, "B*H > 65535");
  *a = rp::QuantArgs{};
  a->B = B;
  a->H = H;
  a->S = S;
  a->D = D;
  a->in_f16 = (in_dtype == RP_DTYPE_F16) ? 1 : 0;
  a->out_ld = out_row_bytes;
  a->nblk = ceil_div(S, rp::kQuantRows);
  a->npart = a->nblk;
  for (int i = 0; i < num_tensors; ++i) {
    const int64_t* st = strides + 4 * i;
    if (!x[i] || (need_out && (!out[i] || !scales[i])))
      return fail(RP_ERR_INVALID, "tensor %d: null pointer", i);
    if (st[3] != 1) return fail(RP_ERR_UNSUPPORTED, "tensor %d: head dim must be unit-stride", i);
    if (!aligned16(x[i]) || (st[0] % 8) || (st[1] % 8) || (st[2] % 8))
      return fail(RP_ERR_ALIGN, "tensor %d: base and strides must be 16-byte multiples", i);
    if (need_out && !aligned16(out[i]))
      return fail(RP_ERR_ALIGN, "tensor %d: output must be 16-byte aligned", i);
    a->job[i].x = static_cast<const uint16_t*>(x[i]);
    a->job[i].sB = st[0];
    a->job[i].sH = st[1];
    a->job[i].sS = st[2];
    a->job[i].out = need_out ? static_cast<uint8_t*>(out[i]) : nullptr;
    a->job[i].scales = need_out ? scales[i] : nullptr;
  }
  return RP_OK;
}

}  // namespace

int rp_quant_fp8_e4m3_ex(int num_tensors, const void* const* x, const int64_t* strides, int B,
                         int H, int S, int D, int in_dtype, int scale_mode, void* const* out,
                         int out_row_bytes, float* const* scales, void* workspace,
                         size_t workspace_bytes, void* stream) {
  rp::QuantArgs a;
  int rc = quant_args(num_tensors, x, strides, B, H, S, D, in_dtype, out, out_row_bytes, scales, &a);
  if (rc != RP_OK) return rc;
  size_t need = 0;
  rc = rp_quant_workspace_bytes(num_tensors, B, H, S, D, scale_mode, &need);
  if (rc != RP_OK) return rc;
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(RP_ERR_WORKSPACE, "workspace of %zu bytes required", need);
  int* status = nullptr;
  rc = device_ready(&status);
  if (rc != RP_OK) return rc;
  a.partial = static_cast<uint32_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = (scale_mode == RP_SCALE_PER_BLOCK128) ? rp::launch_quant_block(a, num_tensors, s)
                                                        : rp::launch_quant_bh(a, num_tensors, s);
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  return RP_OK;
}

int rp_quant_fp8_e4m3_bh_phase(int phase, int num_tensors, const void* const* x,
                               const int64_t* strides, int B, int H, int S, int D, int in_dtype,
                               uint32_t* partials, int npart, void* const* out, int out_row_bytes,
                               float* const* scales, void* stream) {
  if (phase != RP_QUANT_PHASE_AMAX && phase != RP_QUANT_PHASE_APPLY)
    return fail(RP_ERR_INVALID, "unknown phase %d", phase);
  rp::QuantArgs a;
  int rc = quant_args(num_tensors, x, strides, B, H, S, D, in_dtype, out, out_row_bytes, scales, &a,
                      phase == RP_QUANT_PHASE_APPLY);
  if (rc != RP_OK) return rc;
  if (!partials) return fail(RP_ERR_INVALID, "partials is null");
  if (npart < a.nblk)
    return fail(RP_ERR_INVALID, "npart %d is below ceil(S/128) = %d", npart, a.nblk);
  int* status = nullptr;
  rc = device_ready(&status);
  if (rc != RP_OK) return rc;
  a.partial = partials;
  a.npart = npart;
  cudaError_t e = rp::launch_quant_bh(a, num_tensors, static_cast<cudaStream_t>(stream),
                                      phase == RP_QUANT_PHASE_AMAX ? 1 : 2);
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  return RP_OK;
}

namespace {

int check_attn_common(const void* q8, const void* k8, const void* v8, const float* qs,
                      const float* ks, const float* vs, int D, int p_mode, void* out,
                      const int64_t* out_strides, int n_out_strides) {
  if (!q8 || !k8 || !v8 || !qs || !ks || !vs || !out || !out_strides)
    return fail(RP_ERR_INVALID, "null pointer argument");
  if (D != 32 && D != 64 && D != 128 && D != 256)
    return fail(RP_ERR_UNSUPPORTED, "head_dim %d not in {32,64,128,256}", D);
  if (p_mode != RP_P_E4M3 && p_mode != RP_P_E4M3_HILO)
    return fail(RP_ERR_INVALID, "unknown p_mode %d", p_mode);
  if (out_strides[n_out_strides - 1] != 1)
    return fail(RP_ERR_UNSUPPORTED, "output head dim must be unit-stride");
  if (!aligned16(q8) || !aligned16(k8) || !aligned16(v8) || !aligned16(out))
    return fail(RP_ERR_ALIGN, "tensors must be 16-byte aligned");
  return RP_OK;
}

rp::AttnKernelParams base_params(int H, int Sq, float sm_scale, int D, int* status) {
  rp::AttnKernelParams p{};
  p.H = H;
  p.Sq = Sq;
  p.n_q_tiles = ceil_div(Sq, 128);
  p.has_extra = 0;
  p.extra_group = 1;
  const float scale = (sm_scale > 0.f) ? sm_scale : 1.0f / std::sqrt(static_cast<float>(D));
  p.sm_scale_log2 = scale * kLog2e;
  p.out_f16 = 0;
  p.out_plain = 0;
  p.out_cols = 128;
  p.status = status;
  return p;
}

}  // namespace

int rp_attn_fp8_fwd(const void* q8, const void* k8, const void* v8, const float* qs,
                    const float* ks, const float* vs, int scale_mode, int B, int H, int Sq,
                    int Skv, int D, float sm_scale, int causal, int p_mode, void* out,
                    const int64_t* out_strides, void* stream) {
  if (D != 128) return fail(RP_ERR_UNSUPPORTED, "head_dim %d: rp_attn_fp8_fwd takes 128 (see _ex)", D);
  return rp_attn_fp8_fwd_ex(q8, k8, v8, qs, ks, vs, scale_mode, B, H, Sq, Skv, D, 128, sm_scale,
                            causal, p_mode, out, out_strides, RP_DTYPE_BF16, stream);
}

int rp_attn_fp8_fwd_ex(const void* q8, const void* k8, const void* v8, const float* qs,
                       const float* ks, const float* vs, int scale_mode, int B, int H, int Sq,
                       int Skv, int D, int qkv_row_bytes, float sm_scale, int causal, int p_mode,
                       void* out, const int64_t* out_strides, int out_dtype, void* stream) {
  int rc = check_attn_common(q8, k8, v8, qs, ks, vs, D, p_mode, out, out_strides, 4);
  if (rc != RP_OK) return rc;
  const int need_row = (D == 256) ? 256 : 128;
  if (qkv_row_bytes != need_row)
    return fail(RP_ERR_UNSUPPORTED,
                "head_dim %d needs e4m3 rows of %d bytes (zero-padded beyond D), got %d", D,
                need_row, qkv_row_bytes);
  if (out_dtype != RP_DTYPE_BF16 && out_dtype != RP_DTYPE_F16)
    return fail(RP_ERR_UNSUPPORTED, "output dtype %d is neither bf16 nor fp16", out_dtype);
  for (int i = 0; i < 3; ++i)
    if ((out_strides[i] * 2) % 16 != 0)
      return fail(RP_ERR_ALIGN, "output strides must be multiples of 8 elements");
  if (B <= 0 || H <= 0 || Sq <= 0 || Skv <= 0)
    return fail(RP_ERR_INVALID, "B, H, Sq, Skv must be positive");
  if ((int64_t)B * H > 65535) return fail(RP_ERR_UNSUPPORTED, "B*H > 65535");
  if (scale_mode != RP_SCALE_PER_BH && scale_mode != RP_SCALE_PER_BLOCK128)
    return fail(RP_ERR_INVALID, "unknown scale_mode %d", scale_mode);
  int* status = nullptr;
  rc = device_ready(&status);
  if (rc != RP_OK) return rc;

  const int BH = B * H;
  rp::AttnMaps m;
  if ((rc = make_fp8_map(&m.q, q8, Sq, BH, 1, "q", need_row)) != RP_OK) return rc;
  if ((rc = make_fp8_map(&m.k, k8, Skv, BH, 1, "k", need_row)) != RP_OK) return rc;
  if ((rc = make_fp8_map(&m.v, v8, Skv, BH, 1, "v", need_row)) != RP_OK) return rc;
  m.kx = m.k;
  m.vx = m.v;
  const bool f16 = (out_dtype == RP_DTYPE_F16);
  if ((rc = make_out_map(&m.o, out, B, H, Sq, out_strides[0], out_strides[1], out_strides[2], D,
                         f16)) != RP_OK)
    return rc;

  rp::AttnKernelParams p = base_params(H, Sq, sm_scale, D, status);
  p.out_f16 = f16 ? 1 : 0;
  p.out_plain = (D < 128) ? 1 : 0;
  p.out_cols = D;
  const int nq_blk = ceil_div(Sq, 128), nk_blk = ceil_div(Skv, 128);
  p.n_chunks = 1;
  p.tiles_per_chunk = nk_blk;
  p.chunk_len = Skv;
  p.last_len = Skv;
  p.n_main_tiles = nk_blk;
  const bool per_bh = (scale_mode == RP_SCALE_PER_BH);
  p.qs = qs;
  p.qs_bh = per_bh ? 1 : nq_blk;
  p.qs_blk = per_bh ? 0 : 1;
  p.ks = ks;
  p.vs = vs;
  p.kv_chunk = 0;
  p.kv_bh = per_bh ? 1 : nk_blk;
  p.kv_blk = per_bh ? 0 : 1;
  p.ksx = ks;
  p.vsx = vs;
  p.causal = causal ? 1 : 0;
  const int db = (D == 256) ? 2 : 1;
  cudaError_t e = rp::launch_attention(m, p, B, H, db == 2 ? 1 : 2, p_mode, db,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return RP_OK;
}

int rp_attn_fp8_fwd_chunked(const void* q8, const void* k8, const void* v8, const float* qs,
                            const float* ks, const float* vs, int B, int H, int Sq,
                            int n_chunks, int chunk_rows, int last_rows, int D, float sm_scale,
                            int p_mode, void* out, const int64_t* out_strides, void* stream) {
  int rc = check_attn_common(q8, k8, v8, qs, ks, vs, D, p_mode, out, out_strides, 4);
  if (rc != RP_OK) return rc;
  if (D != 128) return fail(RP_ERR_UNSUPPORTED, "head_dim %d: chunked attention takes 128", D);
  if (B <= 0 || H <= 0 || Sq <= 0 || n_chunks <= 0 || chunk_rows <= 0 || last_rows <= 0 ||
      last_rows > chunk_rows)
    return fail(RP_ERR_INVALID, "bad chunked shape");
  if (n_chunks > 1 && chunk_rows % 128 != 0)
    return fail(RP_ERR_UNSUPPORTED, "chunk_rows must be a multiple of 128 when n_chunks > 1");
  if ((int64_t)B * H > 65535 || n_chunks > 65535) return fail(RP_ERR_UNSUPPORTED, "grid too large");
  int* status = nullptr;
  rc = device_ready(&status);
  if (rc != RP_OK) return rc;

  const int BH = B * H;
  rp::AttnMaps m;
  if ((rc = make_fp8_map(&m.q, q8, Sq, BH, 1, "q")) != RP_OK) return rc;
  if ((rc = make_fp8_map(&m.k, k8, chunk_rows, BH, n_chunks, "k")) != RP_OK) return rc;
  if ((rc = make_fp8_map(&m.v, v8, chunk_rows, BH, n_chunks, "v")) != RP_OK) return rc;
  m.kx = m.k;
  m.vx = m.v;
  if ((rc = make_out_map(&m.o, out, B, H, Sq, out_strides[0], out_strides[1], out_strides[2])) != RP_OK)
    return rc;

  rp::AttnKernelParams p = base_params(H, Sq, sm_scale, D, status);
  const int nblk_c = ceil_div(chunk_rows, 128);
  p.n_chunks = n_chunks;
  p.tiles_per_chunk = nblk_c;
  p.chunk_len = chunk_rows;
  p.last_len = last_rows;
  p.n_main_tiles = (n_chunks - 1) * nblk_c + ceil_div(last_rows, 128);
  p.qs = qs;
  p.qs_bh = ceil_div(Sq, 128);
  p.qs_blk = 1;
  p.ks = ks;
  p.vs = vs;
  p.kv_chunk = (int64_t)BH * nblk_c;
  p.kv_bh = nblk_c;
  p.kv_blk = 1;
  p.ksx = ks;
  p.vsx = vs;
  p.causal = 0;
  cudaError_t e = rp::launch_attention(m, p, B, H, 2, p_mode, 1, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return RP_OK;
}

int rp_attn_fp8_prefix_decode(const void* q8, const void* kp8, const void* vp8,
                              const void* kx8, const void* vx8, const float* qs,
                              const float* kps, const float* vps, const float* kxs,
                              const float* vxs, int C, int T, int P, int H, int D,
                              float sm_scale, int p_mode, void* out,
                              const int64_t* out_strides, void* stream) {
  int rc = check_attn_common(q8, kp8, vp8, qs, kps, vps, D, p_mode, out, out_strides, 3);
  if (rc != RP_OK) return rc;
  if (D != 128) return fail(RP_ERR_UNSUPPORTED, "head_dim %d: prefix decode takes 128", D);
  if (!kx8 || !vx8 || !kxs || !vxs) return fail(RP_ERR_INVALID, "null suffix argument");
  if (!aligned16(kx8) || !aligned16(vx8)) return fail(RP_ERR_ALIGN, "suffix must be 16-byte aligned");
  if (C <= 0 || T <= 0 || P <= 0 || H <= 0) return fail(RP_ERR_INVALID, "C, T, P, H must be positive");
  if (128 % T != 0) return fail(RP_ERR_UNSUPPORTED, "tokens per candidate (%d) must divide 128", T);
  if (H > 65535) return fail(RP_ERR_UNSUPPORTED, "H > 65535");
  int* status = nullptr;
  rc = device_ready(&status);
  if (rc != RP_OK) return rc;

  const int rows = C * T;
  rp::AttnMaps m;
  if ((rc = make_fp8_map(&m.q, q8, rows, H, 1, "q")) != RP_OK) return rc;
  if ((rc = make_fp8_map(&m.k, kp8, P, H, 1, "k_prefix")) != RP_OK) return rc;
  if ((rc = make_fp8_map(&m.v, vp8, P, H, 1, "v_prefix")) != RP_OK) return rc;
  if ((rc = make_fp8_map(&m.kx, kx8, rows, H, 1, "k_suffix")) != RP_OK) return rc;
  if ((rc = make_fp8_map(&m.vx, vx8, rows, H, 1, "v_suffix")) != RP_OK) return rc;
  if ((rc = make_out_map(&m.o, out, 1, H, rows, 0, out_strides[1], out_strides[0])) != RP_OK)
    return rc;

  rp::AttnKernelParams p = base_params(H, rows, sm_scale, D, status);
  const int nq_blk = ceil_div(rows, 128), np_blk = ceil_div(P, 128);
  p.n_chunks = 1;
  p.tiles_per_chunk = np_blk;
  p.chunk_len = P;
  p.last_len = P;
  p.n_main_tiles = np_blk;
  p.has_extra = 1;
  p.extra_group = T;
  p.qs = qs;
  p.qs_bh = nq_blk;
  p.qs_blk = 1;
  p.ks = kps;
  p.vs = vps;
  p.kv_chunk = 0;
  p.kv_bh = np_blk;
  p.kv_blk = 1;
  p.ksx = kxs;
  p.vsx = vxs;
  p.kvx_bh = nq_blk;
  p.kvx_blk = 1;
  p.causal = 0;
  cudaError_t e = rp::launch_attention(m, p, 1, H, 1, p_mode, 1, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return RP_OK;
}


int rp_fp8_gemm_ex(const void* a, int64_t lda, const void* b, int64_t ldb, int b_layout,
                   const float* sa, int64_t sa_stride, float a_scale, const float* sb,
                   int64_t sb_stride, float b_scale, const void* bias, void* c, int64_t ldc,
                   int out_dtype, int M, int N, int K, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(RP_ERR_INVALID, "M, N, K must be non-negative");
  if (b_layout != RP_B_KN && b_layout != RP_B_NK)
    return fail(RP_ERR_INVALID, "unknown b_layout %d", b_layout);
  if (out_dtype != RP_DTYPE_BF16 && out_dtype != RP_DTYPE_F16)
    return fail(RP_ERR_UNSUPPORTED, "output dtype %d is neither bf16 nor fp16", out_dtype);
  if (M == 0 || N == 0) return RP_OK;
  if (!c || (K > 0 && (!a || !b)))
    return fail(RP_ERR_INVALID, "a, b and c must be non-null");
  const int64_t b_cols = (b_layout == RP_B_NK) ? K : N;
  if (lda < K || ldb < b_cols || ldc < N)
    return fail(RP_ERR_INVALID, "row pitches lda=%lld ldb=%lld ldc=%lld are shorter than the rows",
                (long long)lda, (long long)ldb, (long long)ldc);
  if (lda % 16 != 0 || ldb % 16 != 0)
    return fail(RP_ERR_ALIGN, "e4m3 row pitches must be multiples of 16 bytes (lda=%lld ldb=%lld)",
                (long long)lda, (long long)ldb);
  if ((sa && sa_stride < 0) || (sb && sb_stride < 0))
    return fail(RP_ERR_INVALID, "scale strides must be non-negative");
  // tile counts are 32-bit in the kernel (128-row tiles bound both forms)
  if (((int64_t)M + 127) / 128 * (((int64_t)N + 255) / 256) > 0x7FFFFFFF)
    return fail(RP_ERR_UNSUPPORTED, "M x N too large (more than 2^31 output tiles)");
  int* status = nullptr;
  int rc = device_ready(&status);
  if (rc != RP_OK) return rc;

  // K = 0: no K blocks, the operands are never read and need no maps.
  CUtensorMap ma{}, mb{};
  if (K > 0) {
    if ((rc = make_mat8_map(&ma, a, K, M, lda, 128, "a")) != RP_OK) return rc;
    if (b_layout == RP_B_NK)
      rc = make_mat8_map(&mb, b, K, N, ldb, rp::gemm_b_box_rows(true), "b");
    else
      rc = make_mat8_map(&mb, b, N, K, ldb, rp::gemm_b_box_rows(false), "b");
    if (rc != RP_OK) return rc;
  }

  rp::GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.group_m = 0;
  p.sa = sa;
  p.sa_stride = sa_stride;
  p.a_scale = a_scale;
  p.sb = sb;
  p.sb_stride = sb_stride;
  p.b_scale = b_scale;
  p.bias = static_cast<const uint16_t*>(bias);
  p.C = c;
  p.ldc = ldc;
  p.vec_store = (aligned16(c) && (ldc * 2) % 16 == 0) ? 1 : 0;
  p.status = status;
  cudaError_t e = rp::launch_fp8_gemm(ma, mb, p, b_layout == RP_B_NK, out_dtype == RP_DTYPE_F16,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fp8 gemm launch");
  return RP_OK;
}

int rp_fp8_gemm_qkv_quant(const void* a, int64_t lda, const void* w, int64_t ldw,
                          const float* sa, int64_t sa_stride, float a_scale, const float* sb,
                          int64_t sb_stride, float b_scale, const void* bias, int B, int S,
                          int H, int K, void* q8, void* k8, void* v8, float* qs, float* ks,
                          float* vs, void* stream) {
  if (B <= 0 || S <= 0 || H <= 0 || K <= 0) return fail(RP_ERR_INVALID, "B, S, H, K must be positive");
  if ((int64_t)B * H > 65535) return fail(RP_ERR_UNSUPPORTED, "B*H > 65535");
  const int64_t M = (int64_t)B * S, N = (int64_t)3 * H * 128;
  if (M > 0x7FFFFFFF || N > 0x7FFFFFFF) return fail(RP_ERR_UNSUPPORTED, "B*S or 3*H*128 too large");
  if (!a || !w || !q8 || !k8 || !v8 || !qs || !ks || !vs)
    return fail(RP_ERR_INVALID, "a, w, the three outputs and their scales must be non-null");
  if (lda < K || ldw < K) return fail(RP_ERR_INVALID, "row pitches are shorter than K");
  if (lda % 16 != 0 || ldw % 16 != 0)
    return fail(RP_ERR_ALIGN, "e4m3 row pitches must be multiples of 16 bytes (lda=%lld ldw=%lld)",
                (long long)lda, (long long)ldw);
  if (!aligned16(q8) || !aligned16(k8) || !aligned16(v8))
    return fail(RP_ERR_ALIGN, "q8, k8 and v8 must be 16-byte aligned");
  if ((sa && sa_stride < 0) || (sb && sb_stride < 0))
    return fail(RP_ERR_INVALID, "scale strides must be non-negative");
  int* status = nullptr;
  int rc = device_ready(&status);
  if (rc != RP_OK) return rc;
  CUtensorMap ma{}, mb{};
  if ((rc = make_mat8_map(&ma, a, K, M, lda, 128, "a")) != RP_OK) return rc;
  if ((rc = make_mat8_map(&mb, w, K, N, ldw, rp::gemm_b_box_rows(true), "w")) != RP_OK) return rc;
  rp::GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = K;
  p.group_m = 0;
  p.sa = sa;
  p.sa_stride = sa_stride;
  p.a_scale = a_scale;
  p.sb = sb;
  p.sb_stride = sb_stride;
  p.b_scale = b_scale;
  p.bias = static_cast<const uint16_t*>(bias);
  p.C = nullptr;
  p.status = status;
  p.qkv_S = S;
  p.qkv_H = H;
  p.qkv_nblk = (S + 127) / 128;
  p.qkv_out[0] = static_cast<uint8_t*>(q8);
  p.qkv_out[1] = static_cast<uint8_t*>(k8);
  p.qkv_out[2] = static_cast<uint8_t*>(v8);
  p.qkv_scales[0] = qs;
  p.qkv_scales[1] = ks;
  p.qkv_scales[2] = vs;
  cudaError_t e = rp::launch_fp8_gemm(ma, mb, p, true, false, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fp8 qkv gemm launch");
  return RP_OK;
}

int rp_fp8_gemm(const void* a, const void* b, void* c, float a_scale, float b_scale, int M,
                int N, int K, void* stream) {
  if (K % 16 != 0 || N % 16 != 0)
    return fail(RP_ERR_ALIGN,
                "contiguous e4m3 rows need K and N to be multiples of 16 (K=%d N=%d); "
                "rp_fp8_gemm_ex takes padded pitches", K, N);
  return rp_fp8_gemm_ex(a, K, b, N, RP_B_KN, nullptr, 0, a_scale, nullptr, 0, b_scale, nullptr,
                        c, N, RP_DTYPE_BF16, M, N, K, stream);
}

int rp_quant_fp8_rows(const void* x, int64_t ldx, int in_dtype, int rows, int cols, void* out,
                      int64_t ldo, float* scales, void* stream) {
  if (rows < 0 || cols < 0) return fail(RP_ERR_INVALID, "rows and cols must be non-negative");
  if (in_dtype != RP_DTYPE_BF16 && in_dtype != RP_DTYPE_F16)
    return fail(RP_ERR_UNSUPPORTED, "input dtype %d is neither bf16 nor fp16", in_dtype);
  if (rows == 0) return RP_OK;
  if (!x || !out || !scales) return fail(RP_ERR_INVALID, "x, out and scales must be non-null");
  if (cols % 8 != 0) return fail(RP_ERR_UNSUPPORTED, "cols (%d) must be a multiple of 8", cols);
  if (ldx < cols || ldo < cols) return fail(RP_ERR_INVALID, "row pitches are shorter than the rows");
  if (!aligned16(x) || ldx % 8 != 0)
    return fail(RP_ERR_ALIGN, "x rows must start on 16-byte boundaries");
  if (reinterpret_cast<uintptr_t>(out) % 8 != 0 || ldo % 8 != 0)
    return fail(RP_ERR_ALIGN, "out rows must start on 8-byte boundaries");
  int* status = nullptr;
  int rc = device_ready(&status);
  if (rc != RP_OK) return rc;
  rp::QuantRowsArgs q{};
  q.x = static_cast<const uint16_t*>(x);
  q.ldx = ldx;
  q.rows = rows;
  q.cols = cols;
  q.in_f16 = (in_dtype == RP_DTYPE_F16) ? 1 : 0;
  q.out = static_cast<uint8_t*>(out);
  q.ldo = ldo;
  q.scales = scales;
  cudaError_t e = rp::launch_quant_rows(q, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "row quantize launch");
  return RP_OK;
}

}  // extern "C"
