// PSA Attention forward (bf16) on the tensor cores for every YOLO26 width.
//
// c2psa sets num_heads = c / 64 with key_dim 32 and head dim 64
// (src/models/yolo/yolo26/blocks/c2psa.rs:158-159), so the widths of the
// model family (yolo26/mod.rs) give C = 128 (n), 256 (s, m, l) and 384 (x).
// C = 128 runs the specialised kernels of va_tc_psa.cu (W_qkv resident in
// shared memory, V produced transposed by the tensor core).  Any other
// C = 64·nh runs here, as five steps over one workspace:
//
//  1. qkv = W_qkv·x + b_qkv — the batched tcgen05 GEMM (bf16 operands, f16
//     out), channel-major [B][2C][Np]: the reference's qkv conv output.
//  2. split: Q and K of every head to token-major [2][B·nh][N][32] (the
//     psa_pack_qkv sections the attention reads) and V to [B·C][Np] (the
//     psa_extract_v_nchw layout), through a shared-memory transpose.
//  3. attention — the same tcgen05 flash-attention kernel as C = 128
//     (per (b, h); O channel-major [B·C][Np] f16, the merged layout).
//  4. S = O + dw3×3(V) + b_pe (f16) and W_proj as f16.
//  5. y = W_proj·S + b_proj — the batched GEMM again (f16 operands, bf16 out).
// Steps 1, 3 and 5 are tensor-core work; 2 and 4 stream their operands once.
#include "va_common.cuh"
#include "va_psa.h"

namespace va {
namespace {

constexpr int kWKD = 32, kWHD = 64;  // key dim, head dim

struct WideWs {
  size_t qkv, qk, v, o, s, w16, xpad, total;
};

WideWs wide_layout(int B, int C, int H, int W) {
  const size_t N = (size_t)H * W, Np = (N + 7) / 8 * 8, nh = (size_t)C / kWHD, BH = (size_t)B * nh;
  WideWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  w.qkv = take((size_t)B * 2 * C * Np * 2);
  w.qk = take(2 * BH * N * kWKD * 2);
  w.v = take((size_t)B * C * Np * 2);
  w.o = take((size_t)B * C * Np * 2);
  w.s = take((size_t)B * C * Np * 2);
  w.w16 = take((size_t)C * C * 2);
  w.xpad = (N % 8) ? take((size_t)B * C * Np * 2) : (size_t)-1;
  w.total = off;
  return w;
}

// Block (b·nh + h, 64-token block): the head's 128 qkv rows (q 32 | k 32 | v 64)
// → Q, K token-major rows of 32 channels and V rows of the [B·C][Np] buffer.
// 16-byte loads and stores; Q and K pass through a shared-memory transpose.
__global__ void __launch_bounds__(256) split_qkv_kernel(const __half* __restrict__ qkv, __half* __restrict__ qk,
                                                        __half* __restrict__ v, int N, int Np, int nh, int BH) {
  __shared__ __align__(16) __half t[64][72];  // [q, k channel][token], 144-byte rows
  const int bh = blockIdx.y, n0 = blockIdx.x * 64, tid = threadIdx.x;
  const int b = bh / nh, h = bh % nh, C = nh * kWHD;
  const __half* src = qkv + ((size_t)b * 2 * C + (size_t)h * 128) * Np;
  for (int i = tid; i < 128 * 8; i += 256) {  // 128 rows × 8 chunks of 8 tokens
    const int r = i >> 3, c8 = (i & 7) * 8, n = n0 + c8;
    const __half* sp = src + (size_t)r * Np + n;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (n + 8 <= N) {
      u = __ldg(reinterpret_cast<const uint4*>(sp));
    } else {
      __half* e = reinterpret_cast<__half*>(&u);
      for (int k = 0; k < 8 && n + k < N; ++k) e[k] = sp[k];
    }
    if (r < 64) {
      *reinterpret_cast<uint4*>(&t[r][c8]) = u;
    } else {
      __half* dp = v + ((size_t)bh * kWHD + r - 64) * Np + n;
      if (n + 8 <= N) {
        *reinterpret_cast<uint4*>(dp) = u;
      } else {
        const __half* e = reinterpret_cast<const __half*>(&u);
        for (int k = 0; k < 8 && n + k < N; ++k) dp[k] = e[k];
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < 64 * 2 * 4; i += 256) {  // token × section × 8-channel chunk
    const int n = i >> 3, sec = (i >> 2) & 1, c8 = (i & 3) * 8;
    if (n0 + n >= N) continue;
    uint4 u;
    uint32_t* w = &u.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __half2 hh = __halves2half2(t[sec * kWKD + c8 + 2 * e][n], t[sec * kWKD + c8 + 2 * e + 1][n]);
      w[e] = *reinterpret_cast<const uint32_t*>(&hh);
    }
    *reinterpret_cast<uint4*>(qk + (((size_t)sec * BH + bh) * N + n0 + n) * kWKD + c8) = u;
  }
}

// S = O + dw3×3(V) + b_pe, one thread per output; plane p = b·C + c (images
// whose width is not a multiple of 4).
__global__ void __launch_bounds__(256) pe_add_kernel(const __half* __restrict__ v, const __half* __restrict__ o,
                                                     const __nv_bfloat16* __restrict__ w_pe,
                                                     const float* __restrict__ b_pe, __half* __restrict__ s, int C,
                                                     int H, int W, int Np, long long total) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / (H * W);
    const int n = (int)(i - p * H * W), y = n / W, x = n - y * W, c = (int)(p % C);
    const __half* vp = v + p * Np;
    float acc = b_pe[c];
#pragma unroll
    for (int dy = -1; dy <= 1; ++dy) {
      const int yy = y + dy;
      if (yy < 0 || yy >= H) continue;
#pragma unroll
      for (int dx = -1; dx <= 1; ++dx) {
        const int xx = x + dx;
        if (xx < 0 || xx >= W) continue;
        acc = fmaf(__bfloat162float(w_pe[c * 9 + (dy + 1) * 3 + dx + 1]), __half2float(vp[yy * W + xx]), acc);
      }
    }
    s[p * Np + n] = __float2half_rn(acc + __half2float(o[p * Np + n]));
  }
}

__global__ void bf16_to_f16_kernel(const __nv_bfloat16* __restrict__ a, __half* __restrict__ b, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    b[i] = __float2half_rn(__bfloat162float(a[i]));
}

// x rows whose pitch (N·2 bytes) TMA cannot address are copied to a pitch of Np.
__global__ void pad_x_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ xp, long long rows,
                             int N, int Np) {
  const long long total = rows * Np;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / Np;
    const int n = (int)(i - r * Np);
    xp[i] = n < N ? x[r * N + n] : __float2bfloat16_rn(0.f);
  }
}

int grid_for(long long n) { return (int)std::min<long long>((n + 255) / 256, 148LL * 16); }

}  // namespace

size_t psa_tc_wide_workspace_bytes(int B, int C, int H, int W) { return wide_layout(B, C, H, W).total; }

int psa_attention_fwd_tc_wide(const __nv_bfloat16* x, const __nv_bfloat16* w_qkv, const float* b_qkv,
                              const __nv_bfloat16* w_pe, const float* b_pe, const __nv_bfloat16* w_proj,
                              const float* b_proj, __nv_bfloat16* y, int B, int C, int H, int W, int nh, void* ws,
                              size_t ws_bytes, cudaStream_t st) {
  VA_CHECK_ARG(C % kWHD == 0 && nh * kWHD == C, "psa_attention bf16: C=%d must be 64·num_heads (nh=%d)", C, nh);
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && (long long)B * nh <= 65535, "psa_attention bf16: bad sizes");
  const WideWs L = wide_layout(B, C, H, W);
  if (!ws || ws_bytes < L.total)
    return set_error(VA_ERR_WORKSPACE, "psa_attention bf16: workspace %zu < %zu bytes", ws_bytes, L.total);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w_qkv) & 15))
    return set_error(VA_ERR_ALIGN, "psa_attention bf16: x/w_qkv need 16-byte, workspace 256-byte alignment");
  const int N = H * W, Np = (N + 7) / 8 * 8, BH = B * nh;
  char* base = static_cast<char*>(ws);
  __half* qkv = reinterpret_cast<__half*>(base + L.qkv);
  __half* qk = reinterpret_cast<__half*>(base + L.qk);
  __half* v = reinterpret_cast<__half*>(base + L.v);
  __half* o = reinterpret_cast<__half*>(base + L.o);
  __half* s = reinterpret_cast<__half*>(base + L.s);
  __half* w16 = reinterpret_cast<__half*>(base + L.w16);
  const __nv_bfloat16* xs = x;
  long long ldx = N;
  if (N % 8) {
    __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(base + L.xpad);
    pad_x_kernel<<<grid_for((long long)B * C * Np), 256, 0, st>>>(x, xp, (long long)B * C, N, Np);
    if (int rc = check_launch("psa wide pad")) return rc;
    xs = xp;
    ldx = Np;
  }
  // 1. qkv[b] = W_qkv · x[b] + b_qkv   (M = 2C channels, N tokens, K = C)
  if (int rc = tc_gemm_f16(GemmOperand{w_qkv, false, C, 0, true}, GemmOperand{xs, true, ldx, (long long)C * ldx, false},
                           qkv, 2, Np, (long long)2 * C * Np, 2 * C, N, C, B, st, 1.0f, 1, b_qkv, true))
    return rc;
  // 2. Q, K token-major; V rows
  split_qkv_kernel<<<dim3((N + 63) / 64, BH), 256, 0, st>>>(qkv, qk, v, N, Np, nh, BH);
  if (int rc = check_launch("psa wide split")) return rc;
  // 3. attention (O channel-major [B·C][Np])
  if (int rc = tc_flash_attention(qk, v, o, nullptr, BH, nh, N, kWKD, 0, st)) return rc;
  // 4. S = O + PE, W_proj as f16 (register-window kernel when W % 4 == 0)
  const int pe_rc = pe_dwconv_vec(v, w_pe, b_pe, s, w_proj, w16, B, C, H, W, Np, o, st);
  if (pe_rc == VA_ERR_UNSUPPORTED) {
    pe_add_kernel<<<grid_for((long long)B * C * N), 256, 0, st>>>(v, o, w_pe, b_pe, s, C, H, W, Np,
                                                                   (long long)B * C * N);
    if (int rc = check_launch("psa wide pe")) return rc;
    bf16_to_f16_kernel<<<grid_for((long long)C * C), 256, 0, st>>>(w_proj, w16, C * C);
    if (int rc = check_launch("psa wide w_proj")) return rc;
  } else if (pe_rc) {
    return pe_rc;
  }
  // 5. y[b] = W_proj · S[b] + b_proj   (M = C, N tokens, K = C), bf16 NCHW
  return tc_gemm_f16(GemmOperand{w16, false, C, 0, true}, GemmOperand{s, true, Np, (long long)C * Np, false}, y, 1,
                     N, (long long)C * N, C, N, C, B, st, 1.0f, 1, b_proj, false);
}

}  // namespace va
