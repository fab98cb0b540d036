// PSA Attention forward (bf16) for callers that cannot allocate device memory.
//
// The regular entry point va_psa_attention_fwd_bf16 takes a caller-provided
// workspace.  Some callers cannot provide one: a graph runtime that plans
// every device buffer before it runs (teenygrad's RuntimeOp declares its
// buffers up front through param_shapes) and has no slot for an extra
// workspace, or host code that must not enter a device allocator while it
// runs (a latency-critical serving loop, code running inside an allocator's
// own callbacks).  This entry point uses a scratch area compiled into the
// library instead: a file-scope device array of kScratchBytes, which every GPU
// that loads the library keeps until the process exits.
//
// The device address of the array is looked up once per device, with that
// device current, by the first call made on it (cudaGetSymbolAddress); make
// that first call before any stream capture.  No call allocates or frees
// device memory.  All calls share the one array: calls whose kernels overlap
// on the GPU (different streams, or different host threads) race on it, so
// serialise them.  The array keeps whatever the previous call left; every
// byte a call reads is written earlier in the same call, so nothing has to
// start at zero.
#include <atomic>

#include "va_common.cuh"
#include "va_psa.h"

namespace va {

namespace {

constexpr size_t kScratchBytes = (size_t)VA_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::atomic<void*> g_scratch_ptr[kMaxDevices];

int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(VA_ERR_UNSUPPORTED, "noalloc: device index %d too large", dev);
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(VA_ERR_LAUNCH, "noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return VA_OK;
}

}  // namespace

}  // namespace va

using namespace va;

extern "C" int va_psa_attention_fwd_bf16_noalloc(const va_bf16* x, const va_bf16* w_qkv, const float* b_qkv,
                                                 const va_bf16* w_pe, const float* b_pe, const va_bf16* w_proj,
                                                 const float* b_proj, va_bf16* y, int B, int C, int H, int W,
                                                 int num_heads, int key_dim, va_stream_t stream) {
  VA_CHECK_ARG(B > 0 && C > 0 && H > 0 && W > 0 && num_heads > 0 && key_dim > 0,
               "psa_attention noalloc: non-positive size");
  VA_CHECK_ARG(psa_tc_supported(C, num_heads, key_dim),
               "psa_attention noalloc: needs key_dim 32 and C = 64·num_heads");
  const size_t need = psa_tc_workspace_bytes(B, C, H, W, num_heads);
  if (need > kScratchBytes)
    return set_error(VA_ERR_WORKSPACE,
                     "psa_attention noalloc: B=%d at %dx%d needs %zu bytes of scratch, more than the %zu bytes "
                     "built into the library; split the batch or use va_psa_attention_fwd_bf16 with a workspace",
                     B, H, W, need, kScratchBytes);
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  return psa_attention_fwd_tc((const __nv_bfloat16*)x, (const __nv_bfloat16*)w_qkv, b_qkv,
                              (const __nv_bfloat16*)w_pe, b_pe, (const __nv_bfloat16*)w_proj, b_proj,
                              (__nv_bfloat16*)y, B, C, H, W, num_heads, key_dim, scratch, kScratchBytes,
                              (cudaStream_t)stream, nullptr);
}
