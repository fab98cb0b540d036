// Data-parallel gradient all-reduce over NVLink peer memory, fused with the
// SGD update of the PSA training step.
//
// The step's gradient buffer is small (VA_PSA_GRAD_COUNT = 50,816 f32,
// ≈200 KB), so an NCCL all-reduce of it costs its launch and protocol
// latency, not bandwidth.  Here every rank exports one device allocation
// through CUDA IPC:
//   data  [2][count] f32      the gradients this rank publishes (double buffer
//                             by step parity)
//   flags [kDpBlocks][8] u32  flags[b][src] = the step number up to which rank
//                             src has published slice b (written by src)
// One launch of dp_allreduce_sgd_kernel, on every rank, per step:
//   1. block b copies its slice of the local gradients into data[parity],
//      then (one thread per peer, release at system scope) writes the step
//      number into flags[b][rank] of every peer;
//   2. waits (acquire at system scope, bounded) until every peer's flag for
//      slice b reaches the step number;
//   3. sums the slice over ranks in rank order (plain loads from the peers'
//      data, L1 bypassed) — the same bits on every rank, and for two ranks
//      the same bits as NCCL's sum — writes the sum back into the gradient
//      buffer and applies master -= lr · sum / world with the bf16/f32
//      parameter rewrite of va_psa_sgd_update.
// No barrier ends the step: a rank writes data[parity] again two steps later,
// after its step+1 wait saw every peer's step+1 flag, which a peer raises only
// in a launch that follows (stream order) its step's reads of data[parity].
// The step number lives in device memory (one counter per block, advanced by
// the block itself), so the launch can be captured in a CUDA graph.
//
// The grid is fixed (kDpBlocks, one block per SM at most) so that every rank
// runs the same slices and all blocks are resident together.  A wait that
// passes the comm's time limit (va_dp_comm_create) records 100 + the peer rank
// in the comm's status word and the block returns without updating; blocks
// that got through have already updated their slices, so the rank's weights
// are then partly stepped.  The status word is sticky: every later launch
// reads it first and returns at once, publishing and updating nothing, so a
// failed comm never sums stale peer data; the caller reads it
// (va_dp_comm_status), and a comm whose status is not 0 must be destroyed and
// created anew on every rank, with the weights restored on every rank.
#include <string.h>

#include "va_common.cuh"

namespace va {
namespace {

constexpr int kDpBlocks = 128;
constexpr int kDpThreads = 256;
constexpr int kDpMaxWorld = 8;
constexpr long long kDpDefaultTimeoutNs = 10000000000LL;  // 10 s: room for host-side skew between ranks

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct DpArgs {
  float* grads;                        // local gradients in, rank sum out
  float* data_self;                    // this rank's published buffer [2][count]
  const float* data_peer[kDpMaxWorld]; // peers' published buffers (NULL at own rank)
  const unsigned* flags_self;          // [kDpBlocks][kDpMaxWorld], written by peers
  unsigned* flags_peer[kDpMaxWorld];   // the same array of every peer
  unsigned* epoch;                     // [kDpBlocks] steps done per block (local)
  int* status;
  float* master;
  __nv_bfloat16 *w_qkv, *w_pe, *w_proj;
  float *b_qkv, *b_pe, *b_proj;
  float lr, gscale;
  long long timeout_ns;
  int rank, world, count, slice;
};

__global__ void __launch_bounds__(kDpThreads) dp_allreduce_sgd_kernel(DpArgs a) {
  __shared__ int s_fail;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int lo = b * a.slice, hi = min(lo + a.slice, a.count);
  const unsigned e = a.epoch[b] + 1u;
  const size_t par = (size_t)(e & 1u) * (size_t)a.count;
  // a comm that failed once stays failed: publish nothing, update nothing
  if (tid == 0) s_fail = *static_cast<volatile int*>(a.status) != 0;
  __syncthreads();
  if (s_fail) return;
  for (int i = lo + tid; i < hi; i += kDpThreads) a.data_self[par + i] = a.grads[i];
  __syncthreads();
  const bool peer = tid < a.world && tid != a.rank;
  if (peer) st_release_sys(a.flags_peer[tid] + b * kDpMaxWorld + a.rank, e);
  if (peer) {
    const unsigned* f = a.flags_self + b * kDpMaxWorld + tid;
    const unsigned long long t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys(f) - e) < 0) {
      if ((long long)(globaltimer_ns() - t0) > a.timeout_ns) {
        atomicCAS(a.status, 0, 100 + tid);
        s_fail = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (s_fail) return;
  for (int i = lo + tid; i < hi; i += kDpThreads) {
    float s = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const float v = p == a.rank ? a.grads[i] : __ldcg(a.data_peer[p] + par + i);
      s = p == 0 ? v : s + v;
    }
    a.grads[i] = s;
    const float w = a.master[i] - a.lr * (s * a.gscale);
    a.master[i] = w;
    if (i < VA_PSA_GRAD_WPROJ) a.w_qkv[i] = __float2bfloat16_rn(w);
    else if (i < VA_PSA_GRAD_WPE) a.w_proj[i - VA_PSA_GRAD_WPROJ] = __float2bfloat16_rn(w);
    else if (i < VA_PSA_GRAD_BQKV) a.w_pe[i - VA_PSA_GRAD_WPE] = __float2bfloat16_rn(w);
    else if (i < VA_PSA_GRAD_BPROJ) a.b_qkv[i - VA_PSA_GRAD_BQKV] = w;
    else if (i < VA_PSA_GRAD_BPE) a.b_proj[i - VA_PSA_GRAD_BPROJ] = w;
    else a.b_pe[i - VA_PSA_GRAD_BPE] = w;
  }
  __syncthreads();
  if (tid == 0) a.epoch[b] = e;
}

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace
}  // namespace va

struct va_dp_comm {
  int rank, world, count, device, connected;
  long long timeout_ns;
  void* base;           // exported allocation: data [2][count] f32, then flags
  unsigned* epoch;      // [kDpBlocks]
  int* status;
  void* peer_base[va::kDpMaxWorld];
  size_t flags_off;
};

using namespace va;

extern "C" {

int va_dp_comm_create(int rank, int world, int count, int timeout_ms, va_dp_comm** out, void* handle) {
  clear_error();
  VA_CHECK_ARG(out && handle, "dp comm: null output");
  VA_CHECK_ARG(timeout_ms >= 0, "dp comm: timeout %d ms", timeout_ms);
  VA_CHECK_ARG(world >= 1 && world <= kDpMaxWorld && rank >= 0 && rank < world,
               "dp comm: rank %d / world %d (1..%d ranks)", rank, world, kDpMaxWorld);
  VA_CHECK_ARG(count == VA_PSA_GRAD_COUNT, "dp comm: count %d (the PSA gradient buffer has %d)", count,
               VA_PSA_GRAD_COUNT);
  *out = nullptr;
  va_dp_comm* c = new va_dp_comm();
  c->rank = rank;
  c->world = world;
  c->count = count;
  c->timeout_ns = timeout_ms > 0 ? (long long)timeout_ms * 1000000LL : kDpDefaultTimeoutNs;
  c->flags_off = align256((size_t)2 * count * sizeof(float));
  const size_t bytes = c->flags_off + align256((size_t)kDpBlocks * kDpMaxWorld * sizeof(unsigned));
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->base, bytes);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->epoch), kDpBlocks * sizeof(unsigned) + 256);
  if (e == cudaSuccess) {
    c->status = reinterpret_cast<int*>(reinterpret_cast<char*>(c->epoch) + kDpBlocks * sizeof(unsigned));
    e = cudaMemset(c->base, 0, bytes);
  }
  if (e == cudaSuccess) e = cudaMemset(c->epoch, 0, kDpBlocks * sizeof(unsigned) + 256);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->base);
  if (e != cudaSuccess) {
    if (c->base) cudaFree(c->base);
    if (c->epoch) cudaFree(c->epoch);
    delete c;
    return set_error(VA_ERR_LAUNCH, "dp comm create: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) <= VA_DP_HANDLE_BYTES, "IPC handle size");
  memset(handle, 0, VA_DP_HANDLE_BYTES);
  memcpy(handle, &h, sizeof(h));
  c->connected = world == 1;
  *out = c;
  return VA_OK;
}

int va_dp_comm_connect(va_dp_comm* c, const void* handles) {
  clear_error();
  VA_CHECK_ARG(c && handles, "dp comm connect: null argument");
  VA_CHECK_ARG(!c->connected || c->world == 1, "dp comm connect: already connected");
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + (size_t)p * VA_DP_HANDLE_BYTES, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(&c->peer_base[p], h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < p; ++q)
        if (c->peer_base[q]) {
          cudaIpcCloseMemHandle(c->peer_base[q]);
          c->peer_base[q] = nullptr;
        }
      return set_error(VA_ERR_LAUNCH, "dp comm connect: rank %d: %s", p, cudaGetErrorString(e));
    }
  }
  c->connected = 1;
  return VA_OK;
}

int va_dp_comm_status(va_dp_comm* c, int* status) {
  clear_error();
  VA_CHECK_ARG(c && status, "dp comm status: null argument");
  cudaError_t e = cudaMemcpy(status, c->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "dp comm status: %s", cudaGetErrorString(e));
  return VA_OK;
}

int va_dp_comm_disconnect(va_dp_comm* c) {
  clear_error();
  VA_CHECK_ARG(c, "dp comm disconnect: null comm");
  cudaError_t first = cudaSuccess;
  for (int p = 0; p < c->world; ++p)
    if (c->peer_base[p]) {
      cudaError_t e = cudaIpcCloseMemHandle(c->peer_base[p]);
      if (first == cudaSuccess) first = e;
      c->peer_base[p] = nullptr;
    }
  c->connected = c->world == 1;
  if (first != cudaSuccess) return set_error(VA_ERR_LAUNCH, "dp comm disconnect: %s", cudaGetErrorString(first));
  return VA_OK;
}

int va_dp_comm_destroy(va_dp_comm* c) {
  clear_error();
  if (!c) return VA_OK;
  for (int p = 0; p < c->world; ++p)
    if (c->peer_base[p]) cudaIpcCloseMemHandle(c->peer_base[p]);
  cudaError_t e = cudaFree(c->base);
  cudaError_t e2 = cudaFree(c->epoch);
  delete c;
  if (e == cudaSuccess) e = e2;
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "dp comm destroy: %s", cudaGetErrorString(e));
  return VA_OK;
}

int va_psa_dp_allreduce_sgd(va_dp_comm* c, float* grads, float* master, float lr, va_bf16* w_qkv, float* b_qkv,
                            va_bf16* w_pe, float* b_pe, va_bf16* w_proj, float* b_proj, va_stream_t stream) {
  clear_error();
  VA_CHECK_ARG(c && grads && master && w_qkv && b_qkv && w_pe && b_pe && w_proj && b_proj,
               "psa dp all-reduce: null pointer");
  VA_CHECK_ARG(c->connected, "psa dp all-reduce: comm not connected");
  DpArgs a{};
  a.grads = grads;
  a.data_self = static_cast<float*>(c->base);
  a.flags_self = reinterpret_cast<const unsigned*>(static_cast<char*>(c->base) + c->flags_off);
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank) continue;
    a.data_peer[p] = static_cast<const float*>(c->peer_base[p]);
    a.flags_peer[p] = reinterpret_cast<unsigned*>(static_cast<char*>(c->peer_base[p]) + c->flags_off);
  }
  a.epoch = c->epoch;
  a.status = c->status;
  a.master = master;
  a.w_qkv = reinterpret_cast<__nv_bfloat16*>(w_qkv);
  a.w_pe = reinterpret_cast<__nv_bfloat16*>(w_pe);
  a.w_proj = reinterpret_cast<__nv_bfloat16*>(w_proj);
  a.b_qkv = b_qkv;
  a.b_pe = b_pe;
  a.b_proj = b_proj;
  a.lr = lr;
  a.timeout_ns = c->timeout_ns;
  a.gscale = 1.f / (float)c->world;
  a.rank = c->rank;
  a.world = c->world;
  a.count = c->count;
  a.slice = ceil_div(ceil_div(c->count, kDpBlocks), 4) * 4;
  dp_allreduce_sgd_kernel<<<kDpBlocks, kDpThreads, 0, stream>>>(a);
  return check_launch("psa dp all-reduce");
}

}  // extern "C"
