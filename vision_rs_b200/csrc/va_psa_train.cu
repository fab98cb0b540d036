// PSA Attention training step (forward + backward, bf16 activations and
// weights, f32 gradients) for the data-parallel configuration: every rank
// runs this on its shard, the caller all-reduces the f32 gradient buffer
// (NCCL), and va_psa_sgd_update applies it to f32 master weights.
//
// Operator (BN folded into conv weight + bias, c2psa.rs:61-116):
//   qkv = W_qkv·x + b_qkv; per head h: q (32), k (32), v (64) channels at
//   h·128; O_h = V_h·softmax(Q_hᵀK_h/√32)ᵀ; PE = dw3×3(V) + b_pe;
//   y = W_proj·(O + PE) + b_proj.  Loss = mean((y − t)²) over the shard.
//
// Backward, in order (all sums over images run per image and are reduced in
// a fixed order — deterministic, no atomics).  It runs on the residual
// r = y − t (O(1) values, well inside the f16 range; dy = 2r/numel would sit
// in f16's subnormals at these batch sizes) and applies σ = 2/numel once, in
// f32, to every gradient it stores:
//   r = y − t                                               (f16, loss_grad_kernel)
//   dW_proj = σ Σ_b (r_b·O_bᵀ + r_b·PE_bᵀ), db_proj = σ Σ r (tcgen05 GEMM partials)
//   dA = W_projᵀ·r  (= dO = dPE, in units of σ)             (tcgen05 GEMM, f32)
//   dV_pe, dW_pe = dw3×3 backward(V, dA); db_pe = σ Σ dA    (f32 SIMT)
//   dQ, dK, dV = attention backward: tcgen05 kernel over the full 64-wide V
//                (N ≤ 512, psa_attn_bwd_tc), else the f32 SIMT kernels once
//                per 32-wide V half (psa_fa2_backward)
//   dqkv = [dQ | dK | dV + dV_pe] per head                  (f16 + f32 copies)
//   dW_qkv = σ Σ_b dqkv_b·x_bᵀ, db_qkv = σ Σ dqkv; dx = σ W_qkvᵀ·dqkv (tcgen05 GEMMs)
//
// Gradient buffer (f32, PyTorch parameter layouts):
//   [dW_qkv 256×128 | dW_proj 128×128 | dW_pe 128×9 | db_qkv 256 | db_proj 128 | db_pe 128]
#include <algorithm>

#include "va_common.cuh"
#include "va_psa.h"

namespace va {

namespace {

constexpr int kC = 128, kQKV = 256, kKD = 32, kHD = 64, kNH = 2;
constexpr int kLossBlocks = 512;

// scale·(y − t) as f16 [B][C][Np] (pad columns zero); per-block Σ(y − t)².
__global__ void loss_grad_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ t,
                                 __half* __restrict__ dy, float* __restrict__ part, long long rows, int N, int Np,
                                 float scale) {
  __shared__ float red[256];
  float acc = 0.f;
  const long long total = rows * Np;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / Np;
    const int n = (int)(i - r * Np);
    float g = 0.f;
    if (n < N) {
      const float d = __bfloat162float(y[r * N + n]) - __bfloat162float(t[r * N + n]);
      acc = fmaf(d, d, acc);
      g = d * scale;
    }
    dy[i] = __float2half_rn(g);
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = red[0];
}

// out[i] = scale · Σ_z in[z·stride + i], z in order (one thread per i).
__global__ void reduce_batches_kernel(const float* __restrict__ in, float* __restrict__ out, int count, int Z,
                                      long long stride, float scale) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int z = 0; z < Z; ++z) s += in[z * stride + i];
    out[i] = s * scale;
  }
}

// out[c] = scale · Σ_b Σ_{n<N} X[b][c][n]  (X pitch `pitch`), fixed-order tree per channel.
template <typename T>
__global__ void rowsum_kernel(const T* __restrict__ x, float* __restrict__ out, int B, int C, int N, int pitch,
                              float scale) {
  __shared__ float red[256];
  const int c = blockIdx.x;
  float acc = 0.f;
  for (int b = 0; b < B; ++b) {
    const T* row = x + ((size_t)b * C + c) * pitch;
    for (int n = threadIdx.x; n < N; n += blockDim.x) acc += (float)row[n];
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[c] = red[0] * scale;
}

__global__ void scale_kernel(float* __restrict__ x, int n, float s) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] *= s;
}

// bf16 [rows][N] → f16 [rows][Np] (pad zero)
__global__ void bf16_to_f16_pad_kernel(const __nv_bfloat16* __restrict__ x, __half* __restrict__ y, long long rows,
                                       int N, int Np) {
  const long long total = rows * Np;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / Np;
    const int n = (int)(i - r * Np);
    y[i] = n < N ? __float2half_rn(__bfloat162float(x[r * N + n])) : __float2half_rn(0.f);
  }
}

// f16 [rows][pitch] → f32 [rows][N]
__global__ void f16_to_f32_kernel(const __half* __restrict__ x, float* __restrict__ y, long long rows, int N,
                                  int pitch) {
  const long long total = rows * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / N;
    y[i] = __half2float(x[r * pitch + (i - r * N)]);
  }
}

__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ y, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = __bfloat162float(x[i]);
}

// channel-major [B][nh·64][pitch] → token-major f32 halves [2][B·nh][N][32]
// (element (half, b·nh + h, n, d) = src[b][h·64 + half·32 + d][n]).
template <typename T>
__global__ void to_fa_halves_kernel(const T* __restrict__ src, float* __restrict__ dst, int B, int N, int pitch) {
  const long long per_half = (long long)B * kNH * N * kKD;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < 2 * per_half;
       i += (long long)gridDim.x * blockDim.x) {
    const int half = (int)(i / per_half);
    long long r = i - half * per_half;
    const int d = (int)(r % kKD);
    r /= kKD;
    const int n = (int)(r % N);
    const int bh = (int)(r / N), b = bh / kNH, h = bh % kNH;
    dst[i] = (float)src[((size_t)b * kC + h * kHD + half * kKD + d) * pitch + n];
  }
}

// dqkv[b][j][n], j = h·128 + r: r < 32 dQ, r < 64 dK, else dV (+ dV_pe);
// written f16 [B][256][Np] (pad zero) and f32 [B][256][N].
__global__ void assemble_dqkv_kernel(const float* __restrict__ dq, const float* __restrict__ dk,
                                     const float* __restrict__ dv_lo, const float* __restrict__ dv_hi,
                                     const float* __restrict__ dv_pe, __half* __restrict__ d16, float* __restrict__ d32,
                                     int B, int N, int Np) {
  const long long total = (long long)B * kQKV * Np;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i % Np);
    const long long bj = i / Np;
    const int j = (int)(bj % kQKV), b = (int)(bj / kQKV);
    float g = 0.f;
    if (n < N) {
      const int h = j / 128, r = j % 128, bh = b * kNH + h;
      if (r < 32) g = dq[((size_t)bh * N + n) * kKD + r];
      else if (r < 64) g = dk[((size_t)bh * N + n) * kKD + r - 32];
      else {
        const int dd = r - 64;
        g = (dd < 32 ? dv_lo[((size_t)bh * N + n) * kKD + dd] : dv_hi[((size_t)bh * N + n) * kKD + dd - 32]) +
            dv_pe[((size_t)b * kC + h * kHD + dd) * N + n];
      }
      d32[((size_t)b * kQKV + j) * N + n] = g;
    }
    d16[i] = __float2half_rn(g);
  }
}

// f32 [rows][N] → f16 [rows][Np] (pad zero)
__global__ void f32_to_f16_pad_kernel(const float* __restrict__ x, __half* __restrict__ y, long long rows, int N,
                                      int Np) {
  const long long total = rows * Np;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / Np;
    const int n = (int)(i - r * Np);
    y[i] = __float2half_rn(n < N ? x[r * N + n] : 0.f);
  }
}

// dqkv from the tensor-core backward: dQ = Σ_j dq_part[j] (j in order), dK
// [B·nh][N][32], dV [B·nh][N][64] (+ dV_pe); same outputs as assemble_dqkv_kernel.
__global__ void assemble_dqkv_tc_kernel(const float* __restrict__ dq_part, int nparts, const float* __restrict__ dk,
                                        const float* __restrict__ dv, const float* __restrict__ dv_pe,
                                        __half* __restrict__ d16, float* __restrict__ d32, int B, int N, int Np) {
  const long long total = (long long)B * kQKV * Np;
  const size_t part = (size_t)B * kNH * N * kKD;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i % Np);
    const long long bj = i / Np;
    const int j = (int)(bj % kQKV), b = (int)(bj / kQKV);
    float g = 0.f;
    if (n < N) {
      const int h = j / 128, r = j % 128, bh = b * kNH + h;
      if (r < 32) {
        for (int pj = 0; pj < nparts; ++pj) g += dq_part[pj * part + ((size_t)bh * N + n) * kKD + r];
      } else if (r < 64) {
        g = dk[((size_t)bh * N + n) * kKD + r - 32];
      } else {
        const int dd = r - 64;
        g = dv[((size_t)bh * N + n) * kHD + dd] + dv_pe[((size_t)b * kC + h * kHD + dd) * N + n];
      }
      d32[((size_t)b * kQKV + j) * N + n] = g;
    }
    d16[i] = __float2half_rn(g);
  }
}

__global__ void sgd_kernel(float* __restrict__ master, const float* __restrict__ g, int n, float lr, float gscale,
                           __nv_bfloat16* __restrict__ w_qkv, float* __restrict__ b_qkv, __nv_bfloat16* __restrict__ w_pe,
                           float* __restrict__ b_pe, __nv_bfloat16* __restrict__ w_proj, float* __restrict__ b_proj) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float w = master[i] - lr * (g[i] * gscale);
    master[i] = w;
    if (i < VA_PSA_GRAD_WPROJ) w_qkv[i] = __float2bfloat16_rn(w);
    else if (i < VA_PSA_GRAD_WPE) w_proj[i - VA_PSA_GRAD_WPROJ] = __float2bfloat16_rn(w);
    else if (i < VA_PSA_GRAD_BQKV) w_pe[i - VA_PSA_GRAD_WPE] = __float2bfloat16_rn(w);
    else if (i < VA_PSA_GRAD_BPROJ) b_qkv[i - VA_PSA_GRAD_BQKV] = w;
    else if (i < VA_PSA_GRAD_BPE) b_proj[i - VA_PSA_GRAD_BPROJ] = w;
    else b_pe[i - VA_PSA_GRAD_BPE] = w;
  }
}

int grid_for(long long n) { return (int)std::min<long long>(std::max<long long>((n + 255) / 256, 1), 148LL * 16); }

struct TrainWs {
  PsaTcOffsets fwd;
  size_t lse, dy, loss_part, dA, part, v32, dvpe, wpe32, fa, dqkv16, dqkv32, x16, wqkv16, do16, total;
};

TrainWs train_layout(int B, int H, int W) {
  const size_t N = (size_t)H * W, Np = (N + 7) / 8 * 8, BH = (size_t)B * kNH;
  TrainWs w;
  w.fwd = psa_tc_offsets(B, H, W, kNH);
  size_t off = w.fwd.total;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  w.lse = take(BH * N * 4);
  w.dy = take((size_t)B * kC * Np * 2);
  w.loss_part = take(kLossBlocks * 4);
  w.dA = take((size_t)B * kC * N * 4);
  w.part = take((size_t)std::max(2 * B * kC * kC, B * kQKV * kC) * 4);
  w.v32 = take((size_t)B * kC * N * 4);
  w.dvpe = take((size_t)B * kC * N * 4);
  w.wpe32 = take((size_t)kC * 9 * 4);
  w.fa = take(12 * BH * N * kKD * 4);  // q, k, v lo/hi, o lo/hi, do lo/hi, dq, dk, dv lo/hi
  w.dqkv16 = take((size_t)B * kQKV * Np * 2);
  w.dqkv32 = take((size_t)B * kQKV * N * 4);
  w.x16 = take((size_t)B * kC * Np * 2);
  w.wqkv16 = take((size_t)kQKV * kC * 2);
  w.do16 = take((size_t)B * kC * Np * 2);
  w.total = off;
  return w;
}

}  // namespace

size_t psa_train_workspace_bytes(int B, int H, int W) {
  if (B <= 0 || H <= 0 || W <= 0) return 0;
  return train_layout(B, H, W).total;
}

int psa_train_fwd_bwd(const __nv_bfloat16* x, const __nv_bfloat16* target, const __nv_bfloat16* w_qkv,
                      const float* b_qkv, const __nv_bfloat16* w_pe, const float* b_pe, const __nv_bfloat16* w_proj,
                      const float* b_proj, __nv_bfloat16* y, __nv_bfloat16* dx, float* grads, float* loss, int B,
                      int C, int H, int W, int nh, int kd, void* ws, size_t ws_bytes, cudaStream_t st) {
  VA_CHECK_ARG(psa_tc_supported(C, nh, kd), "psa train: needs C=128, nh=2, kd=32");
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0, "psa train: bad sizes");
  VA_CHECK_ARG(target && grads && loss && y, "psa train: null target/grads/loss/y");
  const TrainWs L = train_layout(B, H, W);
  if (!ws || ws_bytes < L.total)
    return set_error(VA_ERR_WORKSPACE, "psa train: workspace %zu < %zu bytes", ws_bytes, L.total);
  if (reinterpret_cast<uintptr_t>(ws) & 255) return set_error(VA_ERR_ALIGN, "psa train: workspace needs 256-byte alignment");
  const int N = H * W, Np = (N + 7) / 8 * 8, BH = B * nh;
  char* base = static_cast<char*>(ws);
  auto at = [&](size_t o) { return static_cast<void*>(base + o); };
  float* lse = static_cast<float*>(at(L.lse));
  // forward, keeping Q/K/V/O/PE and the row LSEs
  if (int rc = psa_attention_fwd_tc(x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, y, B, C, H, W, nh, kd, ws,
                                    L.fwd.total, st, lse))
    return rc;
  const __half* qk = static_cast<const __half*>(at(L.fwd.qk));
  const __half* vb = static_cast<const __half*>(at(L.fwd.v));
  const __half* ob = static_cast<const __half*>(at(L.fwd.o));
  const __half* peb = static_cast<const __half*>(at(L.fwd.pe));
  const __half* wp16 = static_cast<const __half*>(at(L.fwd.wproj));
  __half* dy = static_cast<__half*>(at(L.dy));
  float* lpart = static_cast<float*>(at(L.loss_part));
  const long long rows = (long long)B * kC;
  const double numel = (double)rows * N;
  const float sigma = (float)(2.0 / numel);
  loss_grad_kernel<<<kLossBlocks, 256, 0, st>>>(y, target, dy, lpart, rows, N, Np, 1.0f);
  reduce_batches_kernel<<<1, 32, 0, st>>>(lpart, loss, 1, kLossBlocks, 1, (float)(1.0 / numel));
  if (int rc = check_launch("psa train loss")) return rc;

  float* part = static_cast<float*>(at(L.part));
  // dW_proj partials: z < B from O, z ≥ B from PE
  const GemmOperand a_dy{dy, false, Np, (long long)kC * Np, false};
  if (int rc = tc_gemm_f16(a_dy, GemmOperand{ob, false, Np, (long long)kC * Np, false}, part, false, kC,
                           (long long)kC * kC, kC, kC, N, B, st))
    return rc;
  if (int rc = tc_gemm_f16(a_dy, GemmOperand{peb, false, Np, (long long)kC * Np, false}, part + (size_t)B * kC * kC,
                           false, kC, (long long)kC * kC, kC, kC, N, B, st))
    return rc;
  reduce_batches_kernel<<<grid_for(kC * kC), 256, 0, st>>>(part, grads + VA_PSA_GRAD_WPROJ, kC * kC, 2 * B,
                                                           (long long)kC * kC, sigma);
  rowsum_kernel<__half><<<kC, 256, 0, st>>>(dy, grads + VA_PSA_GRAD_BPROJ, B, kC, N, Np, sigma);
  // dA[b][i][n] = Σ_o W_proj[o][i] dy[b][o][n]
  float* dA = static_cast<float*>(at(L.dA));
  if (int rc = tc_gemm_f16(GemmOperand{wp16, true, kC, 0, true}, GemmOperand{dy, true, Np, (long long)kC * Np, false},
                           dA, false, N, (long long)kC * N, kC, N, kC, B, st))
    return rc;
  rowsum_kernel<float><<<kC, 256, 0, st>>>(dA, grads + VA_PSA_GRAD_BPE, B, kC, N, N, sigma);
  // positional encoding backward
  float* v32 = static_cast<float*>(at(L.v32));
  float* dvpe = static_cast<float*>(at(L.dvpe));
  float* wpe32 = static_cast<float*>(at(L.wpe32));
  f16_to_f32_kernel<<<grid_for(rows * N), 256, 0, st>>>(vb, v32, rows, N, Np);
  bf16_to_f32_kernel<<<1, 256, 0, st>>>(w_pe, wpe32, kC * 9);
  if (int rc = check_launch("psa train conversions")) return rc;
  if (int rc = va_dwconv3x3_backward_f32(v32, wpe32, dA, dvpe, grads + VA_PSA_GRAD_WPE, B, kC, H, W, st)) return rc;
  scale_kernel<<<grid_for(kC * 9), 256, 0, st>>>(grads + VA_PSA_GRAD_WPE, kC * 9, sigma);
  // attention backward
  const size_t fsz = (size_t)BH * N * kKD;
  VA_CHECK_ARG(2 * fsz < (size_t)INT32_MAX, "psa train: shard too large");
  float* fa = static_cast<float*>(at(L.fa));
  __half* dq16 = static_cast<__half*>(at(L.dqkv16));
  float* dq32 = static_cast<float*>(at(L.dqkv32));
  const float scale = 1.0f / sqrtf((float)kd);
  if (N <= 512) {  // tensor cores: dK, dV and per-key-tile dQ partials, then dqkv
    __half* do16 = static_cast<__half*>(at(L.do16));
    f32_to_f16_pad_kernel<<<grid_for(rows * Np), 256, 0, st>>>(dA, do16, rows, N, Np);
    if (int rc = check_launch("psa train dO")) return rc;
    float *dk = fa, *dv = fa + fsz, *dqp = fa + 3 * fsz;
    if (int rc = psa_attn_bwd_tc(qk, vb, ob, do16, lse, dk, dv, dqp, B, nh, N, st)) return rc;
    assemble_dqkv_tc_kernel<<<grid_for((long long)B * kQKV * Np), 256, 0, st>>>(dqp, (N + 127) / 128, dk, dv, dvpe,
                                                                               dq16, dq32, B, N, Np);
  } else {  // f32 SIMT kernels, one call per V half (dq and dk accumulate)
    float *q32 = fa, *k32 = fa + fsz, *vh = fa + 2 * fsz, *oh = fa + 4 * fsz, *doh = fa + 6 * fsz;
    float *dq = fa + 8 * fsz, *dk = fa + 9 * fsz, *dvh = fa + 10 * fsz;
    f16_to_f32_kernel<<<grid_for(2 * fsz), 256, 0, st>>>(qk, q32, 1, (int)(2 * fsz), (int)(2 * fsz));
    to_fa_halves_kernel<__half><<<grid_for(2 * fsz), 256, 0, st>>>(vb, vh, B, N, Np);
    to_fa_halves_kernel<__half><<<grid_for(2 * fsz), 256, 0, st>>>(ob, oh, B, N, Np);
    to_fa_halves_kernel<float><<<grid_for(2 * fsz), 256, 0, st>>>(dA, doh, B, N, N);
    if (int rc = check_launch("psa train layouts")) return rc;
    cudaMemsetAsync(dq, 0, 2 * fsz * sizeof(float), st);
    for (int half = 0; half < 2; ++half)
      if (int rc = va_psa_fa2_backward_f32(q32, k32, vh + half * fsz, oh + half * fsz, doh + half * fsz, lse, dq, dk,
                                           dvh + half * fsz, N, scale, BH, kKD, st))
        return rc;
    assemble_dqkv_kernel<<<grid_for((long long)B * kQKV * Np), 256, 0, st>>>(dq, dk, dvh, dvh + fsz, dvpe, dq16,
                                                                              dq32, B, N, Np);
  }
  rowsum_kernel<float><<<kQKV, 256, 0, st>>>(dq32, grads + VA_PSA_GRAD_BQKV, B, kQKV, N, N, sigma);
  // qkv backward
  __half* x16 = static_cast<__half*>(at(L.x16));
  __half* wq16 = static_cast<__half*>(at(L.wqkv16));
  bf16_to_f16_pad_kernel<<<grid_for(rows * Np), 256, 0, st>>>(x, x16, rows, N, Np);
  bf16_to_f16_pad_kernel<<<grid_for(kQKV * kC), 256, 0, st>>>(w_qkv, wq16, kQKV, kC, kC);
  if (int rc = check_launch("psa train qkv prep")) return rc;
  if (int rc = tc_gemm_f16(GemmOperand{dq16, false, Np, (long long)kQKV * Np, false},
                           GemmOperand{x16, false, Np, (long long)kC * Np, false}, part, false, kC,
                           (long long)kQKV * kC, kQKV, kC, N, B, st))
    return rc;
  reduce_batches_kernel<<<grid_for(kQKV * kC), 256, 0, st>>>(part, grads + VA_PSA_GRAD_WQKV, kQKV * kC, B,
                                                             (long long)kQKV * kC, sigma);
  if (dx) {  // dx[b][i][n] = Σ_j W_qkv[j][i] dqkv[b][j][n]
    if (int rc = tc_gemm_f16(GemmOperand{wq16, true, kC, 0, true},
                             GemmOperand{dq16, true, Np, (long long)kQKV * Np, false}, dx, true, N, (long long)kC * N,
                             kC, N, kQKV, B, st, sigma))
      return rc;
  }
  return check_launch("psa train backward");
}

int psa_sgd_update(float* master, const float* grads, float lr, float grad_scale, __nv_bfloat16* w_qkv, float* b_qkv,
                   __nv_bfloat16* w_pe, float* b_pe, __nv_bfloat16* w_proj, float* b_proj, cudaStream_t st) {
  VA_CHECK_ARG(master && grads && w_qkv && b_qkv && w_pe && b_pe && w_proj && b_proj, "psa sgd: null pointer");
  sgd_kernel<<<grid_for(VA_PSA_GRAD_COUNT), 256, 0, st>>>(master, grads, VA_PSA_GRAD_COUNT, lr, grad_scale, w_qkv,
                                                          b_qkv, w_pe, b_pe, w_proj, b_proj);
  return check_launch("psa sgd");
}

}  // namespace va

using namespace va;

extern "C" {

size_t va_psa_train_workspace_bytes(int B, int H, int W) { return psa_train_workspace_bytes(B, H, W); }

int va_psa_train_fwd_bwd_bf16(const va_bf16* x, const va_bf16* target, const va_bf16* w_qkv, const float* b_qkv,
                              const va_bf16* w_pe, const float* b_pe, const va_bf16* w_proj, const float* b_proj,
                              va_bf16* y, va_bf16* dx, float* grads, float* loss, int B, int C, int H, int W,
                              int num_heads, int key_dim, void* workspace, size_t ws_bytes, va_stream_t stream) {
  return psa_train_fwd_bwd((const __nv_bfloat16*)x, (const __nv_bfloat16*)target, (const __nv_bfloat16*)w_qkv, b_qkv,
                           (const __nv_bfloat16*)w_pe, b_pe, (const __nv_bfloat16*)w_proj, b_proj, (__nv_bfloat16*)y,
                           (__nv_bfloat16*)dx, grads, loss, B, C, H, W, num_heads, key_dim, workspace, ws_bytes,
                           (cudaStream_t)stream);
}

int va_psa_sgd_update(float* master, const float* grads, float lr, float grad_scale, va_bf16* w_qkv, float* b_qkv,
                      va_bf16* w_pe, float* b_pe, va_bf16* w_proj, float* b_proj, va_stream_t stream) {
  return psa_sgd_update(master, grads, lr, grad_scale, (__nv_bfloat16*)w_qkv, b_qkv, (__nv_bfloat16*)w_pe, b_pe,
                        (__nv_bfloat16*)w_proj, b_proj, (cudaStream_t)stream);
}

int va_gemm_f16(const void* a, int a_mn, long long lda, long long a_batch, int a_bcast, const void* b, int b_mn,
                long long ldb, long long b_batch, int b_bcast, void* c, int c_bf16, long long ldc, long long c_batch,
                int M, int N, int K, int Z, float alpha, va_stream_t stream) {
  return tc_gemm_f16(GemmOperand{a, a_mn != 0, lda, a_batch, a_bcast != 0},
                     GemmOperand{b, b_mn != 0, ldb, b_batch, b_bcast != 0}, c, c_bf16 != 0, ldc, c_batch, M, N, K, Z,
                     (cudaStream_t)stream, alpha);
}

}  // extern "C"
