// rp_quant_fp8_e4m3_noalloc: the per-(b,h) quantizer with its scratch in a
// fixed, library-owned device array instead of a caller-provided workspace.
//
// Why it exists: some hosts cannot hand this library any extra device memory.
// A plugin loaded into a serving runtime, for instance, may receive only the
// tensors it reads and writes -- its operator ABI has no workspace argument
// and no allocator handle -- while the runtime's own memory pool owns the GPU
// and forbids raw cudaMalloc (a stray allocation breaks the pool's accounting
// and can stall every stream on the device).  The per-(b,h) mode needs
// scratch for one partial amax per 128-token chunk; this entry point keeps
// that scratch in the array below and calls no allocator at all.
//
// Limits and sharing rules:
//   * the array holds kNoAllocSlots partial-amax slots (1 MiB on each device
//     that loads the library, held until the process exits); a call needs
//     num_tensors * B * H * ceil(S / 128) slots and is rejected with
//     RP_ERR_WORKSPACE if that is more;
//   * every call on a device uses the same array.  A call writes every slot it
//     later reads (pass 1 fills them, pass 2 reads them, in stream order), so
//     nothing has to be cleared and the previous call's leftovers are never
//     read -- but two calls whose kernels overlap on the GPU (different
//     streams, no ordering between them) race on the array and corrupt each
//     other's scales.  Serialise such calls on one stream;
//   * the first call on a device looks up the array's device address (the
//     name of a __device__ variable is only a host-side stand-in; passing it
//     to a kernel from host code would read the wrong memory), so make that
//     first call before any stream capture begins.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "internal.h"
#include "repercep_b200.h"

namespace rp {
namespace {

constexpr size_t kNoAllocSlots = 262144;  // 1 MiB of uint32 partial-amax slots

static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocSlots];

std::mutex g_noalloc_mu;
uint32_t* g_noalloc_ptr[64] = {};

// Device address of g_noalloc_scratch on the current device (looked up once
// per device, with that device current).
int noalloc_scratch(uint32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_last_error(RP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_last_error(RP_ERR_INVALID, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    // Compute capability exactly 10.0, like every other entry point: the
    // library holds sm_100a code only, so a 10.x device with x != 0 is
    // rejected here rather than failing at launch.
    int major = 0, minor = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess)
      return set_last_error(RP_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    if (major != 10 || minor != 0)
      return set_last_error(RP_ERR_ARCH, "device %d is not sm_100 (B200); this library is sm_100a only", dev);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_last_error(RP_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return RP_OK;
}

}  // namespace
}  // namespace rp

extern "C" int rp_quant_fp8_e4m3_noalloc(int num_tensors, const void* const* x,
                                         const int64_t* strides, int B, int H, int S, int D,
                                         void* const* out, float* const* scales, void* stream) {
  using namespace rp;
  if (num_tensors < 1 || num_tensors > kMaxQuantJobs)
    return set_last_error(RP_ERR_INVALID, "num_tensors must be 1..3 (got %d)", num_tensors);
  if (!x || !strides || !out || !scales) return set_last_error(RP_ERR_INVALID, "null argument array");
  if (B <= 0 || H <= 0 || S <= 0) return set_last_error(RP_ERR_INVALID, "B, H, S must be positive");
  if (D != 32 && D != 64 && D != 128 && D != 256)
    return set_last_error(RP_ERR_UNSUPPORTED, "head_dim %d not in {32,64,128,256}", D);
  if ((int64_t)B * H > 65535) return set_last_error(RP_ERR_UNSUPPORTED, "B*H > 65535");
  const int nblk = (S + kQuantRows - 1) / kQuantRows;
  const size_t need = (size_t)num_tensors * B * H * nblk;
  if (need > kNoAllocSlots)
    return set_last_error(RP_ERR_WORKSPACE,
                          "shape needs %zu scratch slots (num_tensors*B*H*ceil(S/128)); the "
                          "built-in scratch holds %zu -- use rp_quant_fp8_e4m3 with a workspace",
                          need, kNoAllocSlots);
  QuantArgs a{};
  a.B = B;
  a.H = H;
  a.S = S;
  a.D = D;
  a.in_f16 = 0;
  a.out_ld = D;
  a.nblk = nblk;
  a.npart = nblk;
  for (int i = 0; i < num_tensors; ++i) {
    const int64_t* st = strides + 4 * i;
    if (!x[i] || !out[i] || !scales[i]) return set_last_error(RP_ERR_INVALID, "tensor %d: null pointer", i);
    if (st[3] != 1) return set_last_error(RP_ERR_UNSUPPORTED, "tensor %d: head dim must be unit-stride", i);
    if (reinterpret_cast<uintptr_t>(x[i]) % 16 || (st[0] % 8) || (st[1] % 8) || (st[2] % 8))
      return set_last_error(RP_ERR_ALIGN, "tensor %d: base and strides must be 16-byte multiples", i);
    if (reinterpret_cast<uintptr_t>(out[i]) % 16)
      return set_last_error(RP_ERR_ALIGN, "tensor %d: output must be 16-byte aligned", i);
    a.job[i].x = static_cast<const uint16_t*>(x[i]);
    a.job[i].sB = st[0];
    a.job[i].sH = st[1];
    a.job[i].sS = st[2];
    a.job[i].out = static_cast<uint8_t*>(out[i]);
    a.job[i].scales = scales[i];
  }
  uint32_t* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != RP_OK) return rc;
  a.partial = scratch;
  const cudaError_t e = launch_quant_bh(a, num_tensors, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_last_error(RP_ERR_CUDA, "quantize launch: %s", cudaGetErrorString(e));
  return RP_OK;
}
