// Flash attention on [BH, N, D] row-major, FFMA (SIMT) path.
//
// This is the f32 path of the reference's flash_attention2_forward /
// _backward_dq / _backward_dkv (src/models/yolo/kernels/attention/flash_attn2.rs)
// and psa_fa2_backward (psa.rs:650-725), which the f32 configuration
// (max-abs 1e-5 against the f32 reference) needs: tensor-core TF32 would not
// meet that bound.  The bf16 tensor-core attention lives in va_tc_psa.cu.
//
// Work split: the reference runs one CTA per (bh, query row) and re-reads all
// K/V rows for every row.  Here a 128-thread CTA owns 128 query rows (one per
// thread) and stages 64-key K/V tiles in shared memory, so each K/V element
// is read from global memory once per 128 rows and then broadcast from smem.
// The backward is atomics-free: dq by query-row threads, dk/dv by key-row
// threads; the reference's atomic accumulation of the lo/hi calls (psa.rs:700,
// :723) becomes an ordered read-modify-write by the owning thread.
#include "va_common.cuh"

namespace va {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T, int D, int DV>
__global__ void __launch_bounds__(128) fa_fwd_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                          const T* __restrict__ v, T* __restrict__ o,
                                                          float* __restrict__ lse, int nq, int nk,
                                                          float scale) {
  constexpr int BK = 64;
  __shared__ __align__(16) float ks[BK][D];
  __shared__ __align__(16) float vs[BK][DV];
  const int bh = blockIdx.y;
  const int row = blockIdx.x * 128 + threadIdx.x;
  const bool valid = row < nq;
  const float sl2 = scale * kLog2e;
  float qr[D];
  const T* qp = q + ((long long)bh * nq + (valid ? row : 0)) * D;
#pragma unroll
  for (int d = 0; d < D; ++d) qr[d] = ldg(qp + d) * sl2;
  float acc[DV];
#pragma unroll
  for (int d = 0; d < DV; ++d) acc[d] = 0.f;
  float m = -INFINITY, lsum = 0.f;
  const T* kb = k + (long long)bh * nk * D;
  const T* vb = v + (long long)bh * nk * DV;
  for (int k0 = 0; k0 < nk; k0 += BK) {
    __syncthreads();
    for (int i = threadIdx.x; i < BK * D; i += 128) {
      int r = i / D, c = i % D;
      ks[r][c] = (k0 + r < nk) ? ldg(kb + (long long)(k0 + r) * D + c) : 0.f;
    }
    for (int i = threadIdx.x; i < BK * DV; i += 128) {
      int r = i / DV, c = i % DV;
      vs[r][c] = (k0 + r < nk) ? ldg(vb + (long long)(k0 + r) * DV + c) : 0.f;
    }
    __syncthreads();
    const int kn = min(BK, nk - k0);
    for (int j0 = 0; j0 < kn; j0 += 16) {
      float s[16];
      float cmax = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) dot = fmaf(qr[d], ks[j0 + jj][d], dot);
        s[jj] = (j0 + jj < kn) ? dot : -INFINITY;
        cmax = fmaxf(cmax, s[jj]);
      }
      const float mnew = fmaxf(m, cmax);
      const float alpha = exp2f(m - mnew);
      lsum *= alpha;
#pragma unroll
      for (int d = 0; d < DV; ++d) acc[d] *= alpha;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const float p = exp2f(s[jj] - mnew);
        lsum += p;
#pragma unroll
        for (int d = 0; d < DV; ++d) acc[d] = fmaf(p, vs[j0 + jj][d], acc[d]);
      }
      m = mnew;
    }
  }
  if (valid) {
    const float inv = 1.f / lsum;
    T* op = o + ((long long)bh * nq + row) * DV;
#pragma unroll
    for (int d = 0; d < DV; ++d) st(op + d, acc[d] * inv);
    lse[(long long)bh * nq + row] = (m + log2f(lsum)) * kLn2;
  }
}

// dQ: one thread per query row (flash_attn2.rs:129-187).  ACC → dq += result.
template <int D, int DV, bool ACC>
__global__ void __launch_bounds__(128) fa_bwd_dq_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                        const float* __restrict__ v, const float* __restrict__ o,
                                                        const float* __restrict__ dout, const float* __restrict__ lse,
                                                        float* __restrict__ dq, int nq, int nk, float scale) {
  constexpr int BK = 64;
  __shared__ __align__(16) float ks[BK][D];
  __shared__ __align__(16) float vs[BK][DV];
  const int bh = blockIdx.y;
  const int row = blockIdx.x * 128 + threadIdx.x;
  const bool valid = row < nq;
  const long long qoff = ((long long)bh * nq + (valid ? row : 0));
  float qr[D], dor[DV], acc[D];
  float Di = 0.f;
#pragma unroll
  for (int d = 0; d < D; ++d) { qr[d] = q[qoff * D + d] * scale * kLog2e; acc[d] = 0.f; }
#pragma unroll
  for (int d = 0; d < DV; ++d) { dor[d] = dout[qoff * DV + d]; Di = fmaf(o[qoff * DV + d], dor[d], Di); }
  const float l2 = lse[qoff] * kLog2e;
  const float* kb = k + (long long)bh * nk * D;
  const float* vb = v + (long long)bh * nk * DV;
  for (int k0 = 0; k0 < nk; k0 += BK) {
    __syncthreads();
    for (int i = threadIdx.x; i < BK * D; i += 128) {
      int r = i / D, c = i % D;
      ks[r][c] = (k0 + r < nk) ? kb[(long long)(k0 + r) * D + c] : 0.f;
    }
    for (int i = threadIdx.x; i < BK * DV; i += 128) {
      int r = i / DV, c = i % DV;
      vs[r][c] = (k0 + r < nk) ? vb[(long long)(k0 + r) * DV + c] : 0.f;
    }
    __syncthreads();
    const int kn = min(BK, nk - k0);
    for (int j = 0; j < kn; ++j) {
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) s = fmaf(qr[d], ks[j][d], s);
#pragma unroll
      for (int d = 0; d < DV; ++d) dp = fmaf(dor[d], vs[j][d], dp);
      const float p = exp2f(s - l2);
      const float ds = p * (dp - Di);
#pragma unroll
      for (int d = 0; d < D; ++d) acc[d] = fmaf(ds, ks[j][d], acc[d]);
    }
  }
  if (valid) {
    float* dp = dq + qoff * D;
#pragma unroll
    for (int d = 0; d < D; ++d) dp[d] = (ACC ? dp[d] : 0.f) + acc[d] * scale;
  }
}

// dK, dV: one thread per key row (flash_attn2.rs:195-260).  ACC_K → dk += result.
template <int D, int DV, bool ACC_K>
__global__ void __launch_bounds__(128) fa_bwd_dkv_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                         const float* __restrict__ v, const float* __restrict__ o,
                                                         const float* __restrict__ dout, const float* __restrict__ lse,
                                                         float* __restrict__ dk, float* __restrict__ dv, int nq,
                                                         int nk, float scale) {
  constexpr int BQ = 64;
  __shared__ __align__(16) float qs[BQ][D];
  __shared__ __align__(16) float dos[BQ][DV];
  __shared__ float l2s[BQ], Ds[BQ];
  const int bh = blockIdx.y;
  const int row = blockIdx.x * 128 + threadIdx.x;
  const bool valid = row < nk;
  const long long koff = ((long long)bh * nk + (valid ? row : 0));
  float kr[D], vr[DV], dka[D], dva[DV];
#pragma unroll
  for (int d = 0; d < D; ++d) { kr[d] = k[koff * D + d] * scale * kLog2e; dka[d] = 0.f; }
#pragma unroll
  for (int d = 0; d < DV; ++d) { vr[d] = v[koff * DV + d]; dva[d] = 0.f; }
  const float* qb = q + (long long)bh * nq * D;
  const float* ob = o + (long long)bh * nq * DV;
  const float* dob = dout + (long long)bh * nq * DV;
  for (int q0 = 0; q0 < nq; q0 += BQ) {
    __syncthreads();
    for (int i = threadIdx.x; i < BQ * D; i += 128) {
      int r = i / D, c = i % D;
      qs[r][c] = (q0 + r < nq) ? qb[(long long)(q0 + r) * D + c] : 0.f;
    }
    for (int i = threadIdx.x; i < BQ * DV; i += 128) {
      int r = i / DV, c = i % DV;
      dos[r][c] = (q0 + r < nq) ? dob[(long long)(q0 + r) * DV + c] : 0.f;
    }
    if (threadIdx.x < BQ) {
      int r = threadIdx.x;
      float dsum = 0.f, l2 = 0.f;
      if (q0 + r < nq) {
        const float* orow = ob + (long long)(q0 + r) * DV;
        const float* drow = dob + (long long)(q0 + r) * DV;
        for (int d = 0; d < DV; ++d) dsum = fmaf(orow[d], drow[d], dsum);
        l2 = lse[(long long)bh * nq + q0 + r] * kLog2e;
      }
      Ds[r] = dsum;
      l2s[r] = l2;
    }
    __syncthreads();
    const int qn = min(BQ, nq - q0);
    for (int i = 0; i < qn; ++i) {
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) s = fmaf(qs[i][d], kr[d], s);
#pragma unroll
      for (int d = 0; d < DV; ++d) dp = fmaf(dos[i][d], vr[d], dp);
      const float p = exp2f(s - l2s[i]);
      const float ds = p * (dp - Ds[i]);
#pragma unroll
      for (int d = 0; d < DV; ++d) dva[d] = fmaf(p, dos[i][d], dva[d]);
#pragma unroll
      for (int d = 0; d < D; ++d) dka[d] = fmaf(ds, qs[i][d], dka[d]);
    }
  }
  if (valid) {
    float* kp = dk + koff * D;
    float* vp = dv + koff * DV;
#pragma unroll
    for (int d = 0; d < D; ++d) kp[d] = (ACC_K ? kp[d] : 0.f) + dka[d] * scale;
#pragma unroll
    for (int d = 0; d < DV; ++d) vp[d] = dva[d];
  }
}

template <typename T>
static int fa_fwd(const T* q, const T* k, const T* v, T* o, float* l, int nq, int nk, float scale, int bh,
                  int hd, cudaStream_t st) {
  VA_CHECK_ARG(nq > 0 && nk > 0 && bh > 0, "flash_attention2_forward: non-positive size");
  VA_CHECK_ARG(bh <= 65535, "flash_attention2_forward: bh=%d exceeds 65535", bh);
  dim3 grid(ceil_div(nq, 128), bh);
  switch (hd) {
    case 16: fa_fwd_simt_kernel<T, 16, 16><<<grid, 128, 0, st>>>(q, k, v, o, l, nq, nk, scale); break;
    case 32: fa_fwd_simt_kernel<T, 32, 32><<<grid, 128, 0, st>>>(q, k, v, o, l, nq, nk, scale); break;
    case 64: fa_fwd_simt_kernel<T, 64, 64><<<grid, 128, 0, st>>>(q, k, v, o, l, nq, nk, scale); break;
    default: return set_error(VA_ERR_SHAPE, "flash_attention2_forward: head_dim %d unsupported (16/32/64)", hd);
  }
  return check_launch("flash_attention2_forward");
}

template <bool ACC>
static int fa_bwd_dq(const float* q, const float* k, const float* v, const float* o, const float* d_o,
                     const float* l, float* dq, int nq, int nk, float scale, int bh, int hd, cudaStream_t st) {
  dim3 grid(ceil_div(nq, 128), bh);
  switch (hd) {
    case 16: fa_bwd_dq_kernel<16, 16, ACC><<<grid, 128, 0, st>>>(q, k, v, o, d_o, l, dq, nq, nk, scale); break;
    case 32: fa_bwd_dq_kernel<32, 32, ACC><<<grid, 128, 0, st>>>(q, k, v, o, d_o, l, dq, nq, nk, scale); break;
    case 64: fa_bwd_dq_kernel<64, 64, ACC><<<grid, 128, 0, st>>>(q, k, v, o, d_o, l, dq, nq, nk, scale); break;
    default: return set_error(VA_ERR_SHAPE, "flash attention backward: head_dim %d unsupported", hd);
  }
  return check_launch("flash_attention2_backward_dq");
}

template <bool ACC>
static int fa_bwd_dkv(const float* q, const float* k, const float* v, const float* o, const float* d_o,
                      const float* l, float* dk, float* dv, int nq, int nk, float scale, int bh, int hd,
                      cudaStream_t st) {
  dim3 grid(ceil_div(nk, 128), bh);
  switch (hd) {
    case 16: fa_bwd_dkv_kernel<16, 16, ACC><<<grid, 128, 0, st>>>(q, k, v, o, d_o, l, dk, dv, nq, nk, scale); break;
    case 32: fa_bwd_dkv_kernel<32, 32, ACC><<<grid, 128, 0, st>>>(q, k, v, o, d_o, l, dk, dv, nq, nk, scale); break;
    case 64: fa_bwd_dkv_kernel<64, 64, ACC><<<grid, 128, 0, st>>>(q, k, v, o, d_o, l, dk, dv, nq, nk, scale); break;
    default: return set_error(VA_ERR_SHAPE, "flash attention backward: head_dim %d unsupported", hd);
  }
  return check_launch("flash_attention2_backward_dkv");
}

int fa_fwd_f32(const float* q, const float* k, const float* v, float* o, float* l, int nq, int nk, float scale,
               int bh, int hd, cudaStream_t st) {
  return fa_fwd(q, k, v, o, l, nq, nk, scale, bh, hd, st);
}
int fa_fwd_bf16(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, __nv_bfloat16* o,
                float* l, int nq, int nk, float scale, int bh, int hd, cudaStream_t st) {
  return fa_fwd(q, k, v, o, l, nq, nk, scale, bh, hd, st);
}

}  // namespace va

using namespace va;

extern "C" {

int va_flash_attention2_forward_f32(const float* q, const float* k, const float* v, float* o, float* l, int nq,
                                    int nk, float scale, float neg_inf, int bh, int hd, va_stream_t s) {
  (void)neg_inf;  // the kernel's running max starts at -inf, as the reference's does with this argument
  return fa_fwd(q, k, v, o, l, nq, nk, scale, bh, hd, (cudaStream_t)s);
}

int va_flash_attention2_forward_bf16(const va_bf16* q, const va_bf16* k, const va_bf16* v, va_bf16* o, float* l,
                                     int nq, int nk, float scale, float neg_inf, int bh, int hd, va_stream_t s) {
  (void)neg_inf;
  return fa_fwd((const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (__nv_bfloat16*)o, l,
                nq, nk, scale, bh, hd, (cudaStream_t)s);
}

int va_flash_attention2_backward_dq_f32(const float* q, const float* k, const float* v, const float* o,
                                        const float* d_o, const float* l, float* dq, int nq, int nk, float scale,
                                        int bh, int hd, va_stream_t s) {
  VA_CHECK_ARG(nq > 0 && nk > 0 && bh > 0 && bh <= 65535, "flash_attention2_backward_dq: bad sizes");
  return fa_bwd_dq<false>(q, k, v, o, d_o, l, dq, nq, nk, scale, bh, hd, (cudaStream_t)s);
}

int va_flash_attention2_backward_dkv_f32(const float* q, const float* k, const float* v, const float* o,
                                         const float* d_o, const float* l, float* dk, float* dv, int nq, int nk,
                                         float scale, int bh, int hd, va_stream_t s) {
  VA_CHECK_ARG(nq > 0 && nk > 0 && bh > 0 && bh <= 65535, "flash_attention2_backward_dkv: bad sizes");
  return fa_bwd_dkv<false>(q, k, v, o, d_o, l, dk, dv, nq, nk, scale, bh, hd, (cudaStream_t)s);
}

int va_psa_fa2_backward_f32(const float* q, const float* k, const float* v, const float* o, const float* d_o,
                            const float* l, float* dq, float* dk, float* dv, int N, float scale, int bh, int hd,
                            va_stream_t s) {
  VA_CHECK_ARG(N > 0 && bh > 0 && bh <= 65535, "psa_fa2_backward: bad sizes");
  int rc = fa_bwd_dq<true>(q, k, v, o, d_o, l, dq, N, N, scale, bh, hd, (cudaStream_t)s);
  if (rc) return rc;
  return fa_bwd_dkv<true>(q, k, v, o, d_o, l, dk, dv, N, N, scale, bh, hd, (cudaStream_t)s);
}

}  // extern "C"
