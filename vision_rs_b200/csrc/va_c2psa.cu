// PSABlock and C2PSA forward (bf16, BN folded) around the PSA Attention op.
//
// The reference builds them in src/models/yolo/yolo26/blocks/c2psa.rs:
//   psa_block (:123-137):  b = b + attn(b);  out = b + ffn1(ffn0(b))
//     ffn0 = conv 1×1 c→2c + BN + SiLU (`conv`), ffn1 = conv 1×1 2c→c + BN
//     (`conv_bn`, no activation) — conv.rs:31-69
//   c2psa (:150-179):  h = cv1(x) (c1→2c, SiLU);  a, b = split(h);
//     b = psa_block(b) × n;  out = cv2(cat(a, b)) (2c→c1, SiLU);  c = c1/2,
//     num_heads = c/64, key_dim 32.
// Here every 1×1 convolution is the batched tcgen05 GEMM with its bias,
// SiLU and residual fused into the epilogue, and the attention is the
// tensor-core PSA op:
//   cv1 → two GEMMs: a straight into the concat buffer T (rows 0..c, f16),
//         b into a contiguous bf16 buffer (the attention op's input layout);
//   block: t = attn(b) (bf16); y1 = b + t (f16); g = SiLU(W0·y1 + b0) (f16);
//          out = y1 + W1·g + b1 — the residual is the GEMM's epilogue; the
//          last block writes straight into T rows c..2c;
//   cv2 → one GEMM over T with SiLU, bf16 out.
// Intermediates that feed a GEMM are f16 (3 more mantissa bits than bf16);
// the attention op's input and output stay bf16 as its interface defines.
// Images need H·W % 8 == 0 (16-byte aligned token rows for TMA): YOLO26
// places C2PSA at stride 32, 20×20 at 640 and 40×40 at 1280 input.
#include "va_common.cuh"
#include "va_psa.h"

namespace va {
namespace {

constexpr int kKD = 32;

size_t al(size_t n) { return align256(n); }

// bf16 + bf16 → f16, elementwise over n values (n % 8 == 0, 16-byte aligned)
__global__ void add_bf16_to_f16_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b, uint4* __restrict__ y,
                                       long long n8) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const uint4 ua = __ldg(a + i), ub = __ldg(b + i);
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&ua);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&ub);
    uint4 r;
    __half2* pr = reinterpret_cast<__half2*>(&r);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = __bfloat1622float2(pa[e]), fb = __bfloat1622float2(pb[e]);
      pr[e] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
    }
    y[i] = r;
  }
}

__global__ void w_bf16_to_f16_kernel(const __nv_bfloat16* __restrict__ a, __half* __restrict__ b, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    b[i] = __float2half_rn(__bfloat162float(a[i]));
}

int grid_of(long long n) { return (int)std::min<long long>((n + 255) / 256, 148LL * 8); }

int to_f16(const va_bf16* w, __half* out, int n, cudaStream_t st) {
  w_bf16_to_f16_kernel<<<grid_of(n), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(w), out, n);
  return check_launch("c2psa weight f16");
}

// Workspace of one PSABlock on B images of C channels (reused block after block).
struct BlockWs {
  size_t attn, t, y1, g, w0, w1, total;
};
BlockWs block_layout(int B, int C, int H, int W) {
  const size_t N = (size_t)H * W;
  BlockWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += al(bytes); return o; };
  w.attn = take(psa_tc_workspace_bytes(B, C, H, W, C / 64));
  w.t = take((size_t)B * C * N * 2);
  w.y1 = take((size_t)B * C * N * 2);
  w.g = take((size_t)B * 2 * C * N * 2);
  w.w0 = take((size_t)2 * C * C * 2);
  w.w1 = take((size_t)2 * C * C * 2);
  w.total = off;
  return w;
}

int check_block_args(int B, int C, int H, int W) {
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && C >= 64 && C % 64 == 0, "psa block: C=%d must be a multiple of 64", C);
  VA_CHECK_ARG((H * W) % 8 == 0, "psa block: H·W=%d must be a multiple of 8", H * W);
  return VA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace va

namespace va {
namespace {

// One PSABlock: x bf16 [B][C][N] (contiguous) → out (f16 or bf16, channel rows
// out_ld apart, images out_batch apart).  ws holds block_layout(B, C, H, W).
int psa_block(const __nv_bfloat16* x, const va_psa_block_weights& w, void* out, int out_type, long long out_ld,
              long long out_batch, int B, int C, int H, int W, char* ws, cudaStream_t st) {
  const BlockWs L = block_layout(B, C, H, W);
  const int N = H * W, nh = C / 64;
  __nv_bfloat16* t = reinterpret_cast<__nv_bfloat16*>(ws + L.t);
  __half* y1 = reinterpret_cast<__half*>(ws + L.y1);
  __half* g = reinterpret_cast<__half*>(ws + L.g);
  __half* w0 = reinterpret_cast<__half*>(ws + L.w0);
  __half* w1 = reinterpret_cast<__half*>(ws + L.w1);
  // t = attn(x)   (psa_block: `attn(b)`)
  if (int rc = psa_attention_fwd_tc(x, reinterpret_cast<const __nv_bfloat16*>(w.w_qkv), w.b_qkv,
                                    reinterpret_cast<const __nv_bfloat16*>(w.w_pe), w.b_pe,
                                    reinterpret_cast<const __nv_bfloat16*>(w.w_proj), w.b_proj, t, B, C, H, W, nh,
                                    kKD, ws + L.attn, psa_tc_workspace_bytes(B, C, H, W, nh), st, nullptr,
                                    /*overlap_pe=*/true))
    return rc;
  // y1 = x + t   (`elem_add(b, attn(b))`)
  const long long n8 = (long long)B * C * N / 8;
  add_bf16_to_f16_kernel<<<grid_of(n8), 256, 0, st>>>(reinterpret_cast<const uint4*>(x),
                                                       reinterpret_cast<const uint4*>(t), reinterpret_cast<uint4*>(y1),
                                                       n8);
  if (int rc = check_launch("psa block residual")) return rc;
  if (int rc = to_f16(w.w_ffn0, w0, 2 * C * C, st)) return rc;
  if (int rc = to_f16(w.w_ffn1, w1, 2 * C * C, st)) return rc;
  // g = SiLU(W0·y1 + b0)   (ffn.0: conv + BN + SiLU)
  GemmEpilogue e0;
  e0.silu = true;
  if (int rc = tc_gemm_f16(GemmOperand{w0, false, C, 0, true}, GemmOperand{y1, true, N, (long long)C * N, false}, g,
                           2, N, (long long)2 * C * N, 2 * C, N, C, B, st, 1.0f, 1, w.b_ffn0, false, e0))
    return rc;
  // out = y1 + W1·g + b1   (ffn.1: conv + BN, then `elem_add(b, ffn_out)`)
  GemmEpilogue e1;
  e1.res = y1;
  e1.res_type = 2;
  e1.ldr = N;
  e1.r_batch = (long long)C * N;
  return tc_gemm_f16(GemmOperand{w1, false, 2 * C, 0, true}, GemmOperand{g, true, N, (long long)2 * C * N, false}, out,
                     out_type, out_ld, out_batch, C, N, 2 * C, B, st, 1.0f, 1, w.b_ffn1, false, e1);
}

struct C2Ws {
  size_t block, xb0, xb1, t, wcv2, total;
};
C2Ws c2_layout(int B, int C1, int H, int W) {
  const size_t N = (size_t)H * W, c = (size_t)C1 / 2;
  C2Ws w;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += al(bytes); return o; };
  w.block = take(block_layout(B, (int)c, H, W).total);
  w.xb0 = take((size_t)B * c * N * 2);
  w.xb1 = take((size_t)B * c * N * 2);
  w.t = take((size_t)B * 2 * c * N * 2);
  w.wcv2 = take((size_t)C1 * 2 * c * 2);
  w.total = off;
  return w;
}

}  // namespace
}  // namespace va

using namespace va;

extern "C" {

size_t va_psa_block_workspace_bytes(int B, int C, int H, int W) {
  if (B <= 0 || C < 64 || C % 64 || H <= 0 || W <= 0) return 0;
  return block_layout(B, C, H, W).total;
}

int va_psa_block_fwd_bf16(const va_bf16* x, const va_psa_block_weights* w, va_bf16* y, int B, int C, int H, int W,
                          void* ws, size_t ws_bytes, va_stream_t stream) {
  clear_error();
  VA_CHECK_ARG(x && w && y, "psa block: null pointer");
  if (int rc = check_block_args(B, C, H, W)) return rc;
  const size_t need = block_layout(B, C, H, W).total;
  if (!ws || ws_bytes < need) return set_error(VA_ERR_WORKSPACE, "psa block: workspace %zu < %zu bytes", ws_bytes, need);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) || !aligned16(x) || !aligned16(y))
    return set_error(VA_ERR_ALIGN, "psa block: x, y need 16-byte, workspace 256-byte alignment");
  const long long N = (long long)H * W;
  return psa_block(reinterpret_cast<const __nv_bfloat16*>(x), *w, y, 1, N, (long long)C * N, B, C, H, W,
                   static_cast<char*>(ws), (cudaStream_t)stream);
}

size_t va_c2psa_workspace_bytes(int B, int C1, int H, int W, int n_blocks) {
  (void)n_blocks;  // the blocks reuse one block workspace and two ping-pong buffers
  if (B <= 0 || C1 < 128 || C1 % 128 || H <= 0 || W <= 0) return 0;
  return c2_layout(B, C1, H, W).total;
}

int va_c2psa_fwd_bf16(const va_bf16* x, const va_bf16* w_cv1, const float* b_cv1, int n_blocks,
                      const va_psa_block_weights* blocks, const va_bf16* w_cv2, const float* b_cv2, va_bf16* y, int B,
                      int C1, int H, int W, void* ws, size_t ws_bytes, va_stream_t stream) {
  clear_error();
  VA_CHECK_ARG(x && w_cv1 && b_cv1 && w_cv2 && b_cv2 && y && blocks, "c2psa: null pointer");
  VA_CHECK_ARG(n_blocks >= 1, "c2psa: n_blocks=%d (at least one PSABlock)", n_blocks);
  VA_CHECK_ARG(C1 >= 128 && C1 % 128 == 0, "c2psa: C1=%d must be a multiple of 128", C1);
  const int c = C1 / 2;
  if (int rc = check_block_args(B, c, H, W)) return rc;
  const C2Ws L = c2_layout(B, C1, H, W);
  if (!ws || ws_bytes < L.total) return set_error(VA_ERR_WORKSPACE, "c2psa: workspace %zu < %zu bytes", ws_bytes, L.total);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) || !aligned16(x) || !aligned16(y) || !aligned16(w_cv1) || !aligned16(w_cv2))
    return set_error(VA_ERR_ALIGN, "c2psa: x, y, weights need 16-byte, workspace 256-byte alignment");
  const cudaStream_t st = (cudaStream_t)stream;
  char* base = static_cast<char*>(ws);
  const long long N = (long long)H * W;
  __nv_bfloat16* xb[2] = {reinterpret_cast<__nv_bfloat16*>(base + L.xb0), reinterpret_cast<__nv_bfloat16*>(base + L.xb1)};
  __half* T = reinterpret_cast<__half*>(base + L.t);  // cat(a, b): [B][2c][N]
  __half* wcv2 = reinterpret_cast<__half*>(base + L.wcv2);
  // cv1 (conv + BN + SiLU), rows 0..c → a (into T), rows c..2c → b
  GemmEpilogue silu;
  silu.silu = true;
  const GemmOperand xin{x, true, N, (long long)C1 * N, false};
  if (int rc = tc_gemm_f16(GemmOperand{w_cv1, false, C1, 0, true}, xin, T, 2, N, 2LL * c * N, c, (int)N, C1, B, st,
                           1.0f, 1, b_cv1, true, silu))
    return rc;
  if (int rc = tc_gemm_f16(GemmOperand{w_cv1 + (size_t)c * C1, false, C1, 0, true}, xin, xb[0], 1, N, (long long)c * N,
                           c, (int)N, C1, B, st, 1.0f, 1, b_cv1 + c, true, silu))
    return rc;
  // b = PSABlock(b) × n; the last block writes into T rows c..2c
  for (int i = 0; i < n_blocks; ++i) {
    const bool last = i == n_blocks - 1;
    void* out = last ? static_cast<void*>(T + (size_t)c * N) : static_cast<void*>(xb[(i + 1) & 1]);
    if (int rc = psa_block(xb[i & 1], blocks[i], out, last ? 2 : 1, N, last ? 2LL * c * N : (long long)c * N, B, c, H,
                           W, base + L.block, st))
      return rc;
  }
  // cv2 (conv + BN + SiLU) over cat(a, b)
  if (int rc = to_f16(w_cv2, wcv2, C1 * 2 * c, st)) return rc;
  return tc_gemm_f16(GemmOperand{wcv2, false, 2 * c, 0, true}, GemmOperand{T, true, N, 2LL * c * N, false}, y, 1, N,
                     (long long)C1 * N, C1, (int)N, 2 * c, B, st, 1.0f, 1, b_cv2, false, silu);
}

}  // extern "C"
