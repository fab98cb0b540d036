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
// Backward.  It runs on the residual r = y − t (O(1) values, well inside the
// f16 range; dy = 2r/numel would sit in f16's subnormals at these batch
// sizes) and applies σ = 2/numel once, in f32, when the gradients are stored.
// Every sum over images is taken per image (or per group of images inside one
// GEMM accumulator) and reduced in a fixed order — deterministic, no atomics.
//   loss_rows_kernel   r (f16), Σr and Σr² per (image, channel)
//   tcgen05 GEMMs      dW_proj partials = r·Oᵀ + r·PEᵀ; dA = W_projᵀ·r (f16)
//   attention backward tcgen05 kernel over the full 64-wide V (N ≤ 512,
//                      psa_attn_bwd_tc), else the f32 SIMT kernels once per
//                      32-wide V half (psa_fa2_backward) + a transpose
//   assemble_kernel    per (image, qkv channel): dqkv = [dQ | dK | dV + dV_pe]
//                      (f16 for the GEMMs), its row sum (db_qkv), and on V
//                      channels the positional-encoding backward (dV_pe, and
//                      dW_pe / db_pe partials)
//   tcgen05 GEMMs      dW_qkv partials = dqkv·xᵀ; dx = σ·W_qkvᵀ·dqkv
//   finalize_kernel    every gradient = σ · Σ partials (fixed order), loss
//
// Gradient buffer (f32, PyTorch parameter layouts):
//   [dW_qkv 256×128 | dW_proj 128×128 | dW_pe 128×9 | db_qkv 256 | db_proj 128 | db_pe 128]
#include <algorithm>

#include "va_common.cuh"
#include "va_psa.h"

namespace va {

namespace {

constexpr int kC = 128, kQKV = 256, kKD = 32, kHD = 64, kNH = 2;
constexpr int kRowThreads = 128;
#ifndef VA_TRAIN_ZFOLD
#define VA_TRAIN_ZFOLD 1
#endif
constexpr int kZFold = VA_TRAIN_ZFOLD;  // images per GEMM accumulator in the weight-gradient GEMMs

__device__ __forceinline__ float block_sum(float v, float* red) {  // fixed-order reduction, kRowThreads threads
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) s += red[w];
  return s;
}

// One CTA per (image, output channel) row: r = y − t as f16 [rows][Np] (pad
// zero), Σr and Σr² of the row.
__global__ void __launch_bounds__(kRowThreads)
loss_rows_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ t, __half* __restrict__ r16,
                 float* __restrict__ rsum, float* __restrict__ rsq, int N, int Np, float inv_scale) {
  __shared__ float red[kRowThreads / 32];
  const size_t row = blockIdx.x;
  float s = 0.f, q = 0.f;
  for (int n = threadIdx.x; n < Np; n += kRowThreads) {
    float d = 0.f;
    if (n < N) {
      d = (__bfloat162float(y[row * N + n]) - (t ? __bfloat162float(t[row * N + n]) : 0.0f)) * inv_scale;
      s += d;
      q = fmaf(d, d, q);
    }
    r16[row * Np + n] = __float2half_rn(d);
  }
  s = block_sum(s, red);
  q = block_sum(q, red);
  if (threadIdx.x == 0) {
    rsum[row] = s;
    rsq[row] = q;
  }
}

// Same as loss_rows_kernel for N % 8 == 0 (then Np == N): one warp per row,
// 16-byte loads (8 values) and stores, warp-shuffle sums in a fixed order.
// With t == nullptr (an upstream gradient given) r = y·inv_scale.
__global__ void __launch_bounds__(256)
loss_rows_vec_kernel(const uint4* __restrict__ y, const uint4* __restrict__ t, uint4* __restrict__ r16,
                     float* __restrict__ rsum, float* __restrict__ rsq, int n8, long long rows, float inv_scale) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float s = 0.f, q = 0.f;
  for (int c = lane; c < n8; c += 32) {
    const uint4 uy = __ldg(y + row * n8 + c), ut = t ? __ldg(t + row * n8 + c) : make_uint4(0, 0, 0, 0);
    const uint32_t* py = &uy.x;
    const uint32_t* pt = &ut.x;
    uint4 r;
    uint32_t* pr = &r.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float d0 = (__uint_as_float(py[e] << 16) - __uint_as_float(pt[e] << 16)) * inv_scale;
      const float d1 = (__uint_as_float(py[e] & 0xffff0000u) - __uint_as_float(pt[e] & 0xffff0000u)) * inv_scale;
      s += d0 + d1;
      q = fmaf(d0, d0, fmaf(d1, d1, q));
      const __half2 h = __floats2half2_rn(d0, d1);
      pr[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
    r16[row * n8 + c] = r;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  if (lane == 0) {
    rsum[row] = s;
    rsq[row] = q;
  }
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

// bf16 → f16, 8 elements per thread (16-byte loads and stores); a second
// array (x2 → y2, m8 chunks) rides along in the same launch when given.
__global__ void bf16_to_f16_vec_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, long long n8,
                                       const uint4* __restrict__ x2 = nullptr, uint4* __restrict__ y2 = nullptr,
                                       long long m8 = 0) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8 + m8; i += (long long)gridDim.x * blockDim.x) {
    const bool second = i >= n8;
    const uint4 u = second ? x2[i - n8] : x[i];
    const unsigned w[4] = {u.x, u.y, u.z, u.w};
    unsigned o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __half2 h = __floats2half2_rn(__uint_as_float(w[k] << 16), __uint_as_float(w[k] & 0xffff0000u));
      o[k] = *reinterpret_cast<const unsigned*>(&h);
    }
    (second ? y2[i - n8] : y[i]) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// f16 [count] → f32 [count]
__global__ void f16_to_f32_kernel(const __half* __restrict__ x, float* __restrict__ y, long long count) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = __half2float(x[i]);
}

// channel-major f16 [B][nh·64][pitch] → token-major f32 halves [2][B·nh][N][32]
// (element (half, b·nh + h, n, d) = src[b][h·64 + half·32 + d][n]); the
// layout of the f32 SIMT attention backward.
__global__ void to_fa_halves_kernel(const __half* __restrict__ src, float* __restrict__ dst, int B, int N, int pitch) {
  const long long per_half = (long long)B * kNH * N * kKD;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < 2 * per_half;
       i += (long long)gridDim.x * blockDim.x) {
    const int half = (int)(i / per_half);
    long long r = i - half * per_half;
    const int d = (int)(r % kKD);
    r /= kKD;
    const int n = (int)(r % N);
    const int bh = (int)(r / N), b = bh / kNH, h = bh % kNH;
    dst[i] = __half2float(src[((size_t)b * kC + h * kHD + half * kKD + d) * pitch + n]);
  }
}

// token-major [mats][N][w] → channel-major [mats][w][N] (f32)
__global__ void tm_to_cm_kernel(const float* __restrict__ src, float* __restrict__ dst, int mats, int N, int w) {
  const long long total = (long long)mats * N * w;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i % N);
    const long long mc = i / N;
    const int c = (int)(mc % w), m = (int)(mc / w);
    dst[i] = src[((size_t)m * N + n) * w + c];
  }
}

// One warp per (qkv channel j, image b) row, blockDim.x / 32 rows per CTA
// (kAsmRows, or fewer for large images).  dqkv row:
// dQ = Σ_p dq_part[p] (p in order), dK, or dV + dV_pe, where dV_pe = the
// depthwise 3×3 backward of dA on channel c = h·64 + (j − h·128 − 64).
// Writes the f16 row (pad zero), its sum (db_qkv partial) and, on V channels,
// the dW_pe (9 taps) and db_pe partials of (b, c).  Every sum is a fixed-order
// warp reduction (no block barrier).  Shared memory: per warp the dA and V
// planes of (b, c), f32, each with a one-pixel zero border.
constexpr int kAsmRows = 4;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kAsmRows * 32)
assemble_kernel(const float* __restrict__ dq_part, int nparts, const float* __restrict__ dk, const float* __restrict__ dv,
                const __half* __restrict__ dA, const __half* __restrict__ vb, const __nv_bfloat16* __restrict__ w_pe,
                __half* __restrict__ d16, float* __restrict__ part_bqkv, float* __restrict__ part_wpe,
                float* __restrict__ part_bpe, int B, int H, int W, int Np) {
  extern __shared__ float planes[];  // [rows][2][N]: dA, V
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x * (blockDim.x >> 5) + warp, b = blockIdx.y, N = H * W;
  const int h = j / 128, r = j % 128, bh = b * kNH + h;
  const size_t part = (size_t)B * kNH * kKD * N;
  __half* out = d16 + ((size_t)b * kQKV + j) * Np;
  float rs = 0.f;
  if (r < 64) {
    const float* src = r < 32 ? dq_part + ((size_t)bh * kKD + r) * N : dk + ((size_t)bh * kKD + r - 32) * N;
    const int np_ = r < 32 ? nparts : 1;
    // four tokens per lane per pass (n0 + 32u): their loads are in flight together
    for (int n0 = lane; n0 < Np; n0 += 128) {
      float g[4] = {0.f, 0.f, 0.f, 0.f};
      for (int p = 0; p < np_; ++p)  // partials summed in order p = 0, 1, …
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (n0 + 32 * u < N) g[u] += src[p * part + n0 + 32 * u];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int n = n0 + 32 * u;
        if (n < N) rs += g[u];
        if (n < Np) out[n] = __float2half_rn(g[u]);
      }
    }
    rs = warp_sum(rs);
    if (lane == 0) part_bqkv[(size_t)b * kQKV + j] = rs;
    return;
  }
  const int dd = r - 64, c = h * kHD + dd;
  // dA and V planes with a one-pixel zero border: pixel (y, x) at (y + 1)·Wp + x + 1, so the
  // 3×3 taps need no bounds checks (a border tap adds w·0)
  const int Wp = W + 2, Pp = (H + 2) * Wp;
  float* pa = planes + (size_t)warp * 2 * Pp;
  float* pv = pa + Pp;
  for (int i = lane; i < 2 * Pp; i += 32) pa[i] = 0.f;
  __syncwarp();
  const __half* arow = dA + ((size_t)b * kC + c) * Np;
  const __half* vrow = vb + ((size_t)b * kC + c) * Np;
  const int dy = 32 / W, dx = 32 - dy * W;
  {
    int yy = lane / W, xx = lane - yy * W;
#pragma unroll 4
    for (int n = lane; n < N; n += 32) {
      const int q = (yy + 1) * Wp + xx + 1;
      pa[q] = __half2float(arow[n]);
      pv[q] = __half2float(vrow[n]);
      yy += dy;
      xx += dx;
      if (xx >= W) {
        xx -= W;
        ++yy;
      }
    }
  }
  float w[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) w[k] = __bfloat162float(w_pe[c * 9 + k]);
  __syncwarp();
  const float* dvr = dv + ((size_t)bh * kHD + dd) * N;
  float tw[9] = {}, ab = 0.f;
  int yy = lane / W, xx = lane - yy * W;  // (y, x) of n, advanced by 32 per iteration
#pragma unroll 2
  for (int n = lane; n < Np; n += 32) {
    float g = 0.f;
    if (n < N) {
      const int q = (yy + 1) * Wp + xx + 1;
      const float a = pa[q];
      ab += a;
      float pe = 0.f;
#pragma unroll
      for (int ky = 0; ky < 3; ++ky)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          // forward: PE[y][x] += w[ky][kx]·V[y+ky−1][x+kx−1], so
          // dV[y][x] += w·dA[y−ky+1][x−kx+1] and dW[ky][kx] += dA[y][x]·V[y+ky−1][x+kx−1]
          pe = fmaf(w[ky * 3 + kx], pa[q + (1 - ky) * Wp + (1 - kx)], pe);
          tw[ky * 3 + kx] = fmaf(a, pv[q + (ky - 1) * Wp + (kx - 1)], tw[ky * 3 + kx]);
        }
      g = dvr[n] + pe;
      rs += g;
    }
    out[n] = __float2half_rn(g);
    yy += dy;
    xx += dx;
    if (xx >= W) {
      xx -= W;
      ++yy;
    }
  }
  rs = warp_sum(rs);
  ab = warp_sum(ab);
#pragma unroll
  for (int k = 0; k < 9; ++k) tw[k] = warp_sum(tw[k]);
  if (lane == 0) {
    part_bqkv[(size_t)b * kQKV + j] = rs;
    part_bpe[(size_t)b * kC + c] = ab;
#pragma unroll
    for (int k = 0; k < 9; ++k) part_wpe[((size_t)b * kC + c) * 9 + k] = tw[k];
  }
}

// grads[i] = σ · Σ_p part_i[p] over the partials of each gradient block (p in
// order); block 0 also writes the loss = Σ rsq / numel.
struct FinalizeArgs {
  const float* part_wqkv;  // [Pq][256·128]
  const float* part_wproj; // [Pp][128·128]
  const float* part_wpe;   // [B][128·9]
  const float* part_bqkv;  // [B][256]
  const float* rsum;       // [B][128]
  const float* part_bpe;   // [B][128]
  const float* rsq;        // [B·128]
  int Pq, Pp, B;
  float sigma, inv_numel;
  float* grads;
  float* loss;
};

// Four consecutive gradients per group of 8 lanes (every block boundary and
// partial stride is a multiple of 4): lane j sums partials j, j+8, … with
// 16-byte loads, and the 8 lanes combine with three shuffles (a fixed order).
__global__ void __launch_bounds__(256) finalize_vec_kernel(FinalizeArgs a) {
  const int j = threadIdx.x & 7;
  // warp-uniform loop (the shuffles need every lane): lanes past the end compute nothing
  for (int t0 = (blockIdx.x * blockDim.x + threadIdx.x) & ~31; t0 < VA_PSA_GRAD_COUNT * 2;
       t0 += gridDim.x * blockDim.x) {
    const int i4 = (t0 + (threadIdx.x & 31)) >> 3;
    const bool live = i4 < VA_PSA_GRAD_COUNT / 4;
    const int i = live ? 4 * i4 : 0;
    const float* src;
    int np, off;
    size_t stride;
    if (i < VA_PSA_GRAD_WPROJ) { src = a.part_wqkv; np = a.Pq; off = i; stride = (size_t)kQKV * kC; }
    else if (i < VA_PSA_GRAD_WPE) { src = a.part_wproj; np = a.Pp; off = i - VA_PSA_GRAD_WPROJ; stride = (size_t)kC * kC; }
    else if (i < VA_PSA_GRAD_BQKV) { src = a.part_wpe; np = a.B; off = i - VA_PSA_GRAD_WPE; stride = (size_t)kC * 9; }
    else if (i < VA_PSA_GRAD_BPROJ) { src = a.part_bqkv; np = a.B; off = i - VA_PSA_GRAD_BQKV; stride = kQKV; }
    else if (i < VA_PSA_GRAD_BPE) { src = a.rsum; np = a.B; off = i - VA_PSA_GRAD_BPROJ; stride = kC; }
    else { src = a.part_bpe; np = a.B; off = i - VA_PSA_GRAD_BPE; stride = kC; }
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int p = j; live && p < np; p += 8) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + p * stride + off));
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      s.x += __shfl_xor_sync(0xffffffffu, s.x, o);
      s.y += __shfl_xor_sync(0xffffffffu, s.y, o);
      s.z += __shfl_xor_sync(0xffffffffu, s.z, o);
      s.w += __shfl_xor_sync(0xffffffffu, s.w, o);
    }
    if (live && j == 0)
      *reinterpret_cast<float4*>(a.grads + i) = make_float4(s.x * a.sigma, s.y * a.sigma, s.z * a.sigma, s.w * a.sigma);
  }
  if (blockIdx.x == 0) {
    __shared__ float red[256];
    float s = 0.f;
#pragma unroll 8
    for (int i = threadIdx.x; i < a.B * kC; i += 256) s += a.rsq[i];  // loads in flight, sums in order
    red[threadIdx.x] = s;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
      if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
      __syncthreads();
    }
    if (threadIdx.x == 0) *a.loss = red[0] * a.inv_numel;
  }
}

__global__ void __launch_bounds__(256) finalize_kernel(FinalizeArgs a) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < VA_PSA_GRAD_COUNT; i += gridDim.x * blockDim.x) {
    const float* src;
    int np, off;
    size_t stride;
    if (i < VA_PSA_GRAD_WPROJ) { src = a.part_wqkv; np = a.Pq; off = i; stride = (size_t)kQKV * kC; }
    else if (i < VA_PSA_GRAD_WPE) { src = a.part_wproj; np = a.Pp; off = i - VA_PSA_GRAD_WPROJ; stride = (size_t)kC * kC; }
    else if (i < VA_PSA_GRAD_BQKV) { src = a.part_wpe; np = a.B; off = i - VA_PSA_GRAD_WPE; stride = (size_t)kC * 9; }
    else if (i < VA_PSA_GRAD_BPROJ) { src = a.part_bqkv; np = a.B; off = i - VA_PSA_GRAD_BQKV; stride = kQKV; }
    else if (i < VA_PSA_GRAD_BPE) { src = a.rsum; np = a.B; off = i - VA_PSA_GRAD_BPROJ; stride = kC; }
    else { src = a.part_bpe; np = a.B; off = i - VA_PSA_GRAD_BPE; stride = kC; }
    float s = 0.f;
    for (int p = 0; p < np; ++p) s += src[p * stride + off];
    a.grads[i] = s * a.sigma;
  }
  if (blockIdx.x == 0) {
    __shared__ float red[256];
    float s = 0.f;
#pragma unroll 8
    for (int i = threadIdx.x; i < a.B * kC; i += 256) s += a.rsq[i];  // loads in flight, sums in order
    red[threadIdx.x] = s;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
      if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
      __syncthreads();
    }
    if (threadIdx.x == 0) *a.loss = red[0] * a.inv_numel;
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
  size_t lse, r16, rsum, rsq, dA16, part_wproj, part_wqkv, part_wpe, part_bqkv, part_bpe, fa, dqkv16, x16, wqkv16,
      y16, lossd, total;
};

TrainWs train_layout(int B, int H, int W) {
  const size_t N = (size_t)H * W, Np = (N + 7) / 8 * 8, BH = (size_t)B * kNH;
  const size_t fsz = BH * N * kKD;
  const size_t Pz = (size_t)(B + kZFold - 1) / kZFold;
  TrainWs w;
  w.fwd = psa_tc_offsets(B, H, W, kNH);
  size_t off = w.fwd.total;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  w.lse = take(BH * N * 4);
  w.r16 = take((size_t)B * kC * Np * 2);
  w.rsum = take((size_t)B * kC * 4);
  w.rsq = take((size_t)B * kC * 4);
  w.dA16 = take((size_t)B * kC * Np * 2);
  w.part_wproj = take(2 * Pz * kC * kC * 4);
  w.part_wqkv = take(Pz * kQKV * kC * 4);
  w.part_wpe = take((size_t)B * kC * 9 * 4);
  w.part_bqkv = take((size_t)B * kQKV * 4);
  w.part_bpe = take((size_t)B * kC * 4);
  w.fa = take(16 * fsz * 4);  // tensor-core path: dk, dv (2), dq partials (≤ 4); SIMT path: 12 + 4 (transposes)
  w.dqkv16 = take((size_t)B * kQKV * Np * 2);
  w.x16 = take((size_t)B * kC * Np * 2);
  w.wqkv16 = take((size_t)kQKV * kC * 2);
  w.y16 = take((size_t)B * kC * N * 2);  // the recomputed forward output when only dy is given
  w.lossd = take(4);
  w.total = off;
  return w;
}

}  // namespace

size_t psa_train_workspace_bytes(int B, int H, int W) {
  if (B <= 0 || H <= 0 || W <= 0) return 0;
  return train_layout(B, H, W).total;
}

// Two modes.  Loss mode (target given): loss = mean((y − t)²), r = y − t and
// σ = 2/numel.  Gradient mode (target == nullptr, dy given): the upstream
// gradient ∂L/∂y arrives as dy; r = dy / dy_scale keeps it in f16's normal
// range and σ = dy_scale restores the scale when the gradients are stored;
// y and loss then go to the workspace.
int psa_train_fwd_bwd(const __nv_bfloat16* x, const __nv_bfloat16* target, const __nv_bfloat16* w_qkv,
                      const float* b_qkv, const __nv_bfloat16* w_pe, const float* b_pe, const __nv_bfloat16* w_proj,
                      const float* b_proj, __nv_bfloat16* y, __nv_bfloat16* dx, float* grads, float* loss, int B,
                      int C, int H, int W, int nh, int kd, void* ws, size_t ws_bytes, cudaStream_t st,
                      const __nv_bfloat16* dy = nullptr, float dy_scale = 1.0f) {
  VA_CHECK_ARG(psa_tc_is_n(C, nh, kd), "psa train: needs C=128, nh=2, kd=32");
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && B <= 65535, "psa train: bad sizes");
  const bool grad_mode = target == nullptr;
  if (grad_mode)
    VA_CHECK_ARG(x && dy && grads && dy_scale > 0.0f, "psa attention backward: null x/dy/grads or dy_scale <= 0");
  else
    VA_CHECK_ARG(x && target && grads && loss && y, "psa train: null x/target/grads/loss/y");
  const int N = H * W, Np = (N + 7) / 8 * 8, BH = B * nh;
  VA_CHECK_ARG(2 * (size_t)(H + 2) * (W + 2) * sizeof(float) <= 200 * 1024,
               "psa train: %d tokens per image exceed the staged planes",
               N);
  const TrainWs L = train_layout(B, H, W);
  if (!ws || ws_bytes < L.total)
    return set_error(VA_ERR_WORKSPACE, "psa train: workspace %zu < %zu bytes", ws_bytes, L.total);
  if (reinterpret_cast<uintptr_t>(ws) & 255) return set_error(VA_ERR_ALIGN, "psa train: workspace needs 256-byte alignment");
  char* base = static_cast<char*>(ws);
  auto at = [&](size_t o) { return static_cast<void*>(base + o); };
  if (grad_mode) {
    y = static_cast<__nv_bfloat16*>(at(L.y16));
    loss = static_cast<float*>(at(L.lossd));
  }
  float* lse = static_cast<float*>(at(L.lse));
  // forward, keeping Q/K/V/O/PE and the row LSEs
  // the forward's PE and the backward's side work run on the library's side streams (psa_side_streams)
  const bool overlap = true;
  if (int rc = psa_attention_fwd_tc(x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, y, B, C, H, W, nh, kd, ws,
                                    L.fwd.total, st, lse, overlap))
    return rc;
  const __half* qk = static_cast<const __half*>(at(L.fwd.qk));
  const __half* vb = static_cast<const __half*>(at(L.fwd.v));
  const __half* ob = static_cast<const __half*>(at(L.fwd.o));
  const __half* peb = static_cast<const __half*>(at(L.fwd.pe));
  const __half* wp16 = static_cast<const __half*>(at(L.fwd.wproj));
  const long long rows = (long long)B * kC;
  const double numel = (double)rows * N;
  const float sigma = grad_mode ? dy_scale : (float)(2.0 / numel);
  const __nv_bfloat16* r_src = grad_mode ? dy : y;  // r = (r_src − target)·inv_scale
  const float inv_scale = grad_mode ? 1.0f / dy_scale : 1.0f;
  const int Pz = (B + kZFold - 1) / kZFold;

  __half* r16 = static_cast<__half*>(at(L.r16));
  float* rsum = static_cast<float*>(at(L.rsum));
  float* rsq = static_cast<float*>(at(L.rsq));
  if (N % 8 == 0 && !((reinterpret_cast<uintptr_t>(r_src) | reinterpret_cast<uintptr_t>(target)) & 15))
    loss_rows_vec_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
        reinterpret_cast<const uint4*>(r_src), reinterpret_cast<const uint4*>(target), reinterpret_cast<uint4*>(r16),
        rsum, rsq, N / 8, rows, inv_scale);
  else
    loss_rows_kernel<<<(unsigned)rows, kRowThreads, 0, st>>>(r_src, target, r16, rsum, rsq, N, Np, inv_scale);
  if (int rc = check_launch("psa train loss")) return rc;
  // Fork: the weight-gradient GEMMs of the projection and the f16 copies of x
  // and W_qkv need only r and the forward's buffers, so they run on the
  // lowest-priority side stream beside the attention backward chain (dA →
  // attention backward → dqkv assembly, highest priority); both join `st`
  // before the qkv weight gradient.
  SideStreams* side = nullptr;
  if (overlap) {
    if (int rc = psa_side_streams(&side)) return rc;
    if (side) {
      if (int rc = psa_stream_dep(st, side->hi)) return rc;
      if (int rc = psa_stream_dep(st, side->lo)) return rc;
    }
  }
  SideJoin joiner{side, st};
  const cudaStream_t cs = side ? side->hi : st, ss = side ? side->lo : st;
  // dW_proj partials: Pz from O, then Pz from PE (kZFold images per accumulator)
  float* pwp = static_cast<float*>(at(L.part_wproj));
  const GemmOperand a_r{r16, false, Np, (long long)kC * Np, false};
  if (int rc = tc_gemm_f16(a_r, GemmOperand{ob, false, Np, (long long)kC * Np, false}, pwp, 0, kC,
                           (long long)kC * kC, kC, kC, N, B, ss, 1.0f, kZFold))
    return rc;
  if (int rc = tc_gemm_f16(a_r, GemmOperand{peb, false, Np, (long long)kC * Np, false}, pwp + (size_t)Pz * kC * kC, 0,
                           kC, (long long)kC * kC, kC, kC, N, B, ss, 1.0f, kZFold))
    return rc;
  // dA[b][i][n] = Σ_o W_proj[o][i]·r[b][o][n]  (f16, dO of the attention and dPE)
  __half* dA = static_cast<__half*>(at(L.dA16));
  if (int rc = tc_gemm_f16(GemmOperand{wp16, true, kC, 0, true}, GemmOperand{r16, true, Np, (long long)kC * Np, false},
                           dA, 2, Np, (long long)kC * Np, kC, N, kC, B, cs))
    return rc;
  // attention backward → channel-major dK, dV, dQ partials
  const size_t fsz = (size_t)BH * N * kKD;
  VA_CHECK_ARG(2 * fsz < (size_t)INT32_MAX, "psa train: shard too large");
  float* fa = static_cast<float*>(at(L.fa));
  float *dk = fa, *dv = fa + fsz, *dqp = fa + 3 * fsz;
  int nparts = 1;
  if (N <= 512) {
    float* delta = fa + 7 * fsz;  // [B·nh][N] ≤ fsz floats
    if (int rc = psa_attn_bwd_tc(qk, vb, ob, dA, lse, delta, dk, dv, dqp, B, nh, N, cs)) return rc;
    nparts = (N + 127) / 128;
  } else {  // f32 SIMT kernels, one call per V half (dq and dk accumulate), then channel-major
    float *q32 = fa + 4 * fsz, *k32 = fa + 5 * fsz, *vh = fa + 6 * fsz, *oh = fa + 8 * fsz, *doh = fa + 10 * fsz;
    float *dq = fa + 12 * fsz, *dkt = fa + 13 * fsz, *dvh = fa + 14 * fsz;
    f16_to_f32_kernel<<<grid_for(2 * fsz), 256, 0, cs>>>(qk, q32, (long long)(2 * fsz));
    to_fa_halves_kernel<<<grid_for(2 * fsz), 256, 0, cs>>>(vb, vh, B, N, Np);
    to_fa_halves_kernel<<<grid_for(2 * fsz), 256, 0, cs>>>(ob, oh, B, N, Np);
    to_fa_halves_kernel<<<grid_for(2 * fsz), 256, 0, cs>>>(dA, doh, B, N, Np);
    if (int rc = check_launch("psa train layouts")) return rc;
    cudaMemsetAsync(dq, 0, 2 * fsz * sizeof(float), cs);
    const float scale = 1.0f / sqrtf((float)kd);
    for (int half = 0; half < 2; ++half)
      if (int rc = va_psa_fa2_backward_f32(q32, k32, vh + half * fsz, oh + half * fsz, doh + half * fsz, lse, dq, dkt,
                                           dvh + half * fsz, N, scale, BH, kKD, cs))
        return rc;
    tm_to_cm_kernel<<<grid_for(fsz), 256, 0, cs>>>(dq, dqp, BH, N, kKD);
    tm_to_cm_kernel<<<grid_for(fsz), 256, 0, cs>>>(dkt, dk, BH, N, kKD);
    // dv halves [2][BH][N][32] → [BH][64][N]: channels 0-31 from lo, 32-63 from hi
    tm_to_cm_kernel<<<grid_for(fsz), 256, 0, cs>>>(dvh, q32, BH, N, kKD);            // lo → [BH][32][N]
    tm_to_cm_kernel<<<grid_for(fsz), 256, 0, cs>>>(dvh + fsz, q32 + fsz, BH, N, kKD);  // hi → [BH][32][N]
    for (int half = 0; half < 2; ++half)
      cudaMemcpy2DAsync(dv + (size_t)half * kKD * N, (size_t)kHD * N * sizeof(float), q32 + half * fsz,
                        (size_t)kKD * N * sizeof(float), (size_t)kKD * N * sizeof(float), BH,
                        cudaMemcpyDeviceToDevice, cs);
  }
  // dqkv rows (+ PE backward and the bias partials)
  __half* dq16 = static_cast<__half*>(at(L.dqkv16));
  float* pbq = static_cast<float*>(at(L.part_bqkv));
  float* pwe = static_cast<float*>(at(L.part_wpe));
  float* pbe = static_cast<float*>(at(L.part_bpe));
  static PerDeviceOnce asm_attr;  // the planes of a large image need more than the default 48 KB (per device)
  if (int rc = asm_attr.run([] {
        cudaError_t e = cudaFuncSetAttribute(assemble_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        return e == cudaSuccess ? VA_OK : set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      }))
    return rc;
  int asm_rows = kAsmRows;  // rows (warps) per CTA: a power of two dividing kQKV whose planes fit
  const size_t plane_bytes = 2 * (size_t)(H + 2) * (W + 2) * sizeof(float);  // dA and V with a zero border
  while (asm_rows > 1 && (size_t)asm_rows * plane_bytes > 200 * 1024) asm_rows >>= 1;
  assemble_kernel<<<dim3(kQKV / asm_rows, B), asm_rows * 32, (size_t)asm_rows * plane_bytes, cs>>>(
      dqp, nparts, dk, dv, dA, vb, w_pe, dq16, pbq, pwe, pbe, B, H, W, Np);
  if (int rc = check_launch("psa train assemble")) return rc;
  // qkv backward
  __half* x16 = static_cast<__half*>(at(L.x16));
  __half* wq16 = static_cast<__half*>(at(L.wqkv16));
  if (N == Np && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {  // x and W_qkv in one launch
    bf16_to_f16_vec_kernel<<<grid_for(rows * N / 8 + kQKV * kC / 8), 256, 0, ss>>>(
        reinterpret_cast<const uint4*>(x), reinterpret_cast<uint4*>(x16), rows * N / 8,
        reinterpret_cast<const uint4*>(w_qkv), reinterpret_cast<uint4*>(wq16), kQKV * kC / 8);
  } else {
    bf16_to_f16_pad_kernel<<<grid_for(rows * Np), 256, 0, ss>>>(x, x16, rows, N, Np);
    bf16_to_f16_vec_kernel<<<grid_for(kQKV * kC / 8), 256, 0, ss>>>(reinterpret_cast<const uint4*>(w_qkv),
                                                                    reinterpret_cast<uint4*>(wq16), kQKV * kC / 8);
  }
  if (int rc = check_launch("psa train qkv prep")) return rc;
  if (int rc = joiner.join()) return rc;
  float* pwq = static_cast<float*>(at(L.part_wqkv));
  if (int rc = tc_gemm_f16(GemmOperand{dq16, false, Np, (long long)kQKV * Np, false},
                           GemmOperand{x16, false, Np, (long long)kC * Np, false}, pwq, 0, kC, (long long)kQKV * kC,
                           kQKV, kC, N, B, st, 1.0f, kZFold))
    return rc;
  if (dx) {  // dx[b][i][n] = σ Σ_j W_qkv[j][i] dqkv[b][j][n]
    if (int rc = tc_gemm_f16(GemmOperand{wq16, true, kC, 0, true},
                             GemmOperand{dq16, true, Np, (long long)kQKV * Np, false}, dx, 1, N, (long long)kC * N,
                             kC, N, kQKV, B, st, sigma))
      return rc;
  }
  FinalizeArgs fa_args{pwq, pwp, pwe, pbq, rsum, pbe, rsq, Pz, 2 * Pz, B, sigma, (float)(1.0 / numel), grads, loss};
  if (!(reinterpret_cast<uintptr_t>(grads) & 15))
    finalize_vec_kernel<<<grid_for(VA_PSA_GRAD_COUNT * 2), 256, 0, st>>>(fa_args);
  else
    finalize_kernel<<<grid_for(VA_PSA_GRAD_COUNT), 256, 0, st>>>(fa_args);
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

size_t va_psa_attention_bwd_workspace_bytes(int B, int H, int W) { return psa_train_workspace_bytes(B, H, W); }

int va_psa_attention_bwd_bf16(const va_bf16* x, const va_bf16* dy, float dy_scale, const va_bf16* w_qkv,
                              const float* b_qkv, const va_bf16* w_pe, const float* b_pe, const va_bf16* w_proj,
                              const float* b_proj, va_bf16* dx, float* grads, int B, int C, int H, int W,
                              int num_heads, int key_dim, void* workspace, size_t ws_bytes, va_stream_t stream) {
  return psa_train_fwd_bwd((const __nv_bfloat16*)x, nullptr, (const __nv_bfloat16*)w_qkv, b_qkv,
                           (const __nv_bfloat16*)w_pe, b_pe, (const __nv_bfloat16*)w_proj, b_proj, nullptr,
                           (__nv_bfloat16*)dx, grads, nullptr, B, C, H, W, num_heads, key_dim, workspace, ws_bytes,
                           (cudaStream_t)stream, (const __nv_bfloat16*)dy, dy_scale);
}

int va_psa_sgd_update(float* master, const float* grads, float lr, float grad_scale, va_bf16* w_qkv, float* b_qkv,
                      va_bf16* w_pe, float* b_pe, va_bf16* w_proj, float* b_proj, va_stream_t stream) {
  return psa_sgd_update(master, grads, lr, grad_scale, (__nv_bfloat16*)w_qkv, b_qkv, (__nv_bfloat16*)w_pe, b_pe,
                        (__nv_bfloat16*)w_proj, b_proj, (cudaStream_t)stream);
}

int va_gemm_f16(const void* a, int a_mn, long long lda, long long a_batch, int a_bcast, const void* b, int b_mn,
                long long ldb, long long b_batch, int b_bcast, void* c, int c_type, long long ldc, long long c_batch,
                int M, int N, int K, int Z, float alpha, va_stream_t stream) {
  return tc_gemm_f16(GemmOperand{a, a_mn != 0, lda, a_batch, a_bcast != 0},
                     GemmOperand{b, b_mn != 0, ldb, b_batch, b_bcast != 0}, c, c_type, ldc, c_batch, M, N, K, Z,
                     (cudaStream_t)stream, alpha);
}

}  // extern "C"
