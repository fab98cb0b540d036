// The per-node flash_attention2_forward on the tensor cores.
//
// The reference graph records the PSA attention as two flash_attention2_forward
// nodes, one per 32-wide V half (FlashAttn2PsaRuntimeOp::new_lo/new_hi,
// src/models/yolo/kernels/attention/psa.rs:930-1004; kernel flash_attn2.rs:54-121),
// each reading q, k, v as [BH][N][32] bf16 slices of the packed buffer and
// writing o [BH][N][32] and the row log-sum-exp l [BH·N].  This entry keeps
// that contract and runs the tcgen05 attention kernel of the fused path:
//   1. pack: q, k → f16 [2][BH][N][32]; v → f16 channel-major [BH·64][Np]
//      (rows 0-31 the V half, rows 32-63 zeros, Np = N rounded up to 8);
//   2. the tensor-core attention over BH sequences (one head each), token-
//      major bf16 output [BH][N][64] and l;
//   3. take channels 0-31 of each output row into o.
// The scratch comes from a caller-provided workspace (a RuntimeOp declares it
// through param_shapes, as it declares the l scratch).  bf16 → f16 is exact for
// |x| < 65504 except below 2^-14, where f16 keeps fewer bits than bf16.
#include "va_common.cuh"
#include "va_psa.h"
#include "visionattn.h"

namespace va {
namespace {

constexpr int kNodeKd = 32, kNodeTok = 32, kNodeThreads = 256;
constexpr long long kNodeSmallRows = 2048;  // bh·N at or below which the FFMA kernel is faster

__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 a) {
  uint32_t w[4] = {a.x, a.y, a.z, a.w}, r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xffff0000u);
    const __half2 h = __floats2half2_rn(lo, hi);
    r[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// One block: 32 tokens of one (b, h) sequence.  q/k/v rows are 64 bytes
// (32 bf16), so the tile of each is 2 KB contiguous: 128 16-byte chunks.
__global__ void __launch_bounds__(kNodeThreads)
node_pack_kernel(const uint4* __restrict__ q, const uint4* __restrict__ k, const uint4* __restrict__ v,
                 uint4* __restrict__ qk16, __half* __restrict__ vt, int BH, int N, int Np) {
  __shared__ float tv[kNodeTok][kNodeKd + 1];
  const int bh = blockIdx.y, t0 = blockIdx.x * kNodeTok, tid = threadIdx.x;
  const int ntok = min(kNodeTok, N - t0);
  const size_t row0 = (size_t)bh * N + t0;  // first row of the tile in [BH][N]
  constexpr int kChunksPerRow = kNodeKd / 8;  // 4
  for (int c = tid; c < kNodeTok * kChunksPerRow; c += kNodeThreads) {
    const int r = c / kChunksPerRow, j = c % kChunksPerRow;
    if (r >= ntok) continue;
    const size_t src = (row0 + r) * kChunksPerRow + j;
    qk16[src] = bf16x8_to_f16x8(q[src]);
    qk16[(size_t)BH * N * kChunksPerRow + src] = bf16x8_to_f16x8(k[src]);
    const uint4 a = v[src];
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      tv[r][8 * j + 2 * i] = __uint_as_float(w[i] << 16);
      tv[r][8 * j + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __syncthreads();
  // V transposed: rows ch of [BH·64][Np]; channels 32-63 are zeros.  Columns
  // t0 … t0 + ntok − 1 (the pad columns past N are never read).
  for (int e = tid; e < 64 * kNodeTok; e += kNodeThreads) {
    const int ch = e / kNodeTok, r = e % kNodeTok;
    if (r >= ntok) continue;
    vt[((size_t)bh * 64 + ch) * Np + t0 + r] = __float2half_rn(ch < kNodeKd ? tv[r][ch] : 0.0f);
  }
}

// o[row][0:32] = otm[row][0:32] (token-major rows of 64 → 32 channels).
__global__ void node_take_half_kernel(const uint4* __restrict__ otm, uint4* __restrict__ o, long long rows) {
  const long long n = rows * 4;  // 16-byte chunks of o
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    o[i] = otm[(i >> 2) * 8 + (i & 3)];
}

size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

struct NodeWs {
  size_t qk, vt, otm, total;
};

NodeWs node_ws(int n, int bh) {
  const size_t Np = ((size_t)n + 7) / 8 * 8;
  NodeWs w;
  w.qk = 0;
  w.vt = align_up((size_t)2 * bh * n * kNodeKd * 2);
  w.otm = w.vt + align_up((size_t)bh * 64 * Np * 2);
  w.total = w.otm + align_up((size_t)bh * n * 64 * 2);
  return w;
}

}  // namespace
}  // namespace va

using namespace va;

extern "C" {

size_t va_flash_attention2_tc_workspace_bytes(int n_ctx, int bh, int head_dim) {
  if (n_ctx <= 0 || bh <= 0 || head_dim != kNodeKd) return 0;
  return node_ws(n_ctx, bh).total;
}

int va_flash_attention2_forward_tc_bf16(const va_bf16* q, const va_bf16* k, const va_bf16* v, va_bf16* o, float* l,
                                        int n_ctx_q, int n_ctx_k, float softmax_scale, float neg_inf, int bh,
                                        int head_dim, void* workspace, size_t ws_bytes, va_stream_t stream) {
  clear_error();
  (void)neg_inf;  // the running maximum starts at −∞ inside the kernel
  VA_CHECK_ARG(q && k && v && o && l, "flash attention (tensor cores): null pointer (q, k, v, o and l are required)");
  VA_CHECK_ARG(head_dim == kNodeKd, "flash attention (tensor cores): head_dim %d (32 only)", head_dim);
  VA_CHECK_ARG(n_ctx_q == n_ctx_k, "flash attention (tensor cores): self-attention only (n_ctx_q %d, n_ctx_k %d)",
               n_ctx_q, n_ctx_k);
  VA_CHECK_ARG(n_ctx_q > 0 && bh > 0 && bh <= 65535, "flash attention (tensor cores): bad sizes");
  VA_CHECK_ARG(softmax_scale > 0.0f, "flash attention (tensor cores): softmax_scale must be positive");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(workspace)) & 15)
    return set_error(VA_ERR_ALIGN, "flash attention (tensor cores): q, k, v, o and the workspace need 16-byte alignment");
  const int N = n_ctx_q, Np = (N + 7) / 8 * 8;
  // A few hundred query rows in all (cfg1's single image: 2 × 400) fill too
  // few CTAs for the repack + tensor-core pipeline; the split-row FFMA kernel
  // finishes them sooner (20 vs 30 µs at 2 × 400).
  if ((long long)bh * N <= kNodeSmallRows)
    return va_flash_attention2_forward_bf16(q, k, v, o, l, n_ctx_q, n_ctx_k, softmax_scale, neg_inf, bh, head_dim,
                                            stream);
  const NodeWs w = node_ws(N, bh);
  if (!workspace || ws_bytes < w.total)
    return set_error(VA_ERR_WORKSPACE, "flash attention (tensor cores): workspace of %zu bytes needed, %zu given",
                     w.total, ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  node_pack_kernel<<<dim3((N + kNodeTok - 1) / kNodeTok, bh), kNodeThreads, 0, st>>>(
      reinterpret_cast<const uint4*>(q), reinterpret_cast<const uint4*>(k), reinterpret_cast<const uint4*>(v),
      reinterpret_cast<uint4*>(ws + w.qk), reinterpret_cast<__half*>(ws + w.vt), bh, N, Np);
  if (int rc = check_launch("flash attention pack")) return rc;
  if (int rc = tc_flash_attention(ws + w.qk, ws + w.vt, ws + w.otm, l, bh, 1, N, kNodeKd, 1, st, softmax_scale))
    return rc;
  const long long rows = (long long)bh * N;
  node_take_half_kernel<<<(int)std::min<long long>((rows * 4 + 255) / 256, 148LL * 16), 256, 0, st>>>(
      reinterpret_cast<const uint4*>(ws + w.otm), reinterpret_cast<uint4*>(o), rows);
  return check_launch("flash attention take half");
}

}  // extern "C"
