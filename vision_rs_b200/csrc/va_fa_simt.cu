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

constexpr int kSplitKeys = 256;

// Forward for small problems (few rows per head, few heads): R threads share
// a query row, each taking every R-th key of a shared-memory K/V tile with its
// own running max, sum and accumulator; the R partial states are merged at
// the end with warp shuffles (rescaled to the common max, then summed).  One
// image of cfg1 (2 heads × 400 rows) fills only 7 CTAs of the row-per-thread
// kernel; here it fills 100.  K/V rows are padded to D+4 floats, so the R
// lanes of a row group read R consecutive rows as 16-byte vectors without
// bank conflicts.
// 4 consecutive elements as f32 (one 16-byte load for f32, 8 bytes for bf16).
__device__ __forceinline__ float4 ld4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x), b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}

template <typename T, int D, int DV, int R>
__global__ void __launch_bounds__(256) fa_fwd_split_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                           const T* __restrict__ v, T* __restrict__ o,
                                                           float* __restrict__ lse, int nq, int nk, float scale) {
  static_assert(D % 4 == 0 && DV % 4 == 0 && DV % R == 0 && 32 % R == 0, "shape");
  // BK keys per shared-memory chunk (all of a cfg1 head's keys in two chunks),
  // KPT of them per thread
  constexpr int BK = kSplitKeys, KPT = BK / R, ROWS = 256 / R, PD = D + 4, PV = DV + 4;
  extern __shared__ float4 split_smem[];
  float* ks = reinterpret_cast<float*>(split_smem);
  float* vs = ks + BK * PD;
  const int bh = blockIdx.y, t = threadIdx.x % R;
  const int row = blockIdx.x * ROWS + threadIdx.x / R;
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
    // the chunk's K and V rows, 4 elements per load, all loads of a thread in flight together
    for (int i = threadIdx.x; i < BK * (D / 4); i += 256) {
      const int r = i / (D / 4), c = 4 * (i % (D / 4));
      const float4 x = k0 + r < nk ? ld4(kb + (long long)(k0 + r) * D + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(ks + r * PD + c) = x;
    }
    for (int i = threadIdx.x; i < BK * (DV / 4); i += 256) {
      const int r = i / (DV / 4), c = 4 * (i % (DV / 4));
      const float4 x = k0 + r < nk ? ld4(vb + (long long)(k0 + r) * DV + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(vs + r * PV + c) = x;
    }
    __syncthreads();
  const int kn = min(BK, nk - k0);
    float s[KPT];
    float cmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      const int j = t + R * i;
      const float4* kr = reinterpret_cast<const float4*>(ks + j * PD);
      float dot = 0.f;
#pragma unroll
      for (int d4 = 0; d4 < D / 4; ++d4) {
        const float4 kk = kr[d4];
        dot = fmaf(qr[4 * d4], kk.x, dot);
        dot = fmaf(qr[4 * d4 + 1], kk.y, dot);
        dot = fmaf(qr[4 * d4 + 2], kk.z, dot);
        dot = fmaf(qr[4 * d4 + 3], kk.w, dot);
      }
      s[i] = j < kn ? dot : -INFINITY;
      cmax = fmaxf(cmax, s[i]);
    }
    const float mnew = fmaxf(m, cmax);
    if (mnew == -INFINITY) continue;  // every key of this thread's share lies past nk
    const float alpha = exp2f(m - mnew);
    lsum *= alpha;
#pragma unroll
    for (int d = 0; d < DV; ++d) acc[d] *= alpha;
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      const float p = exp2f(s[i] - mnew);
      lsum += p;
      const float4* vr = reinterpret_cast<const float4*>(vs + (t + R * i) * PV);
#pragma unroll
      for (int d4 = 0; d4 < DV / 4; ++d4) {
        const float4 vv = vr[d4];
        acc[4 * d4] = fmaf(p, vv.x, acc[4 * d4]);
        acc[4 * d4 + 1] = fmaf(p, vv.y, acc[4 * d4 + 1]);
        acc[4 * d4 + 2] = fmaf(p, vv.z, acc[4 * d4 + 2]);
        acc[4 * d4 + 3] = fmaf(p, vv.w, acc[4 * d4 + 3]);
      }
    }
    m = mnew;
  }
  // merge the R partial states of the row (lanes t = 0..R-1 of one row group)
  float mrow = m;
#pragma unroll
  for (int off = R / 2; off > 0; off >>= 1) mrow = fmaxf(mrow, __shfl_xor_sync(0xffffffffu, mrow, off));
  const float f = m == -INFINITY ? 0.f : exp2f(m - mrow);
  lsum *= f;
#pragma unroll
  for (int d = 0; d < DV; ++d) acc[d] *= f;
#pragma unroll
  for (int off = R / 2; off > 0; off >>= 1) {
    lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
#pragma unroll
    for (int d = 0; d < DV; ++d) acc[d] += __shfl_xor_sync(0xffffffffu, acc[d], off);
  }
  if (valid) {
    const float inv = 1.f / lsum;
    T* op = o + ((long long)bh * nq + row) * DV;
    // lane t writes outputs t·DV/R .. +DV/R (constant indices into acc: a predicated unrolled loop)
#pragma unroll
    for (int d = 0; d < DV; ++d)
      if (d / (DV / R) == t) st(op + d, acc[d] * inv);
    if (t == 0) lse[(long long)bh * nq + row] = (mrow + log2f(lsum)) * kLn2;
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
  VA_CHECK_ARG(hd == 16 || hd == 32 || hd == 64, "flash_attention2_forward: head_dim %d unsupported (16, 32, 64)", hd);
  VA_CHECK_ARG(q && k && v && o && l, "flash_attention2_forward: null pointer (q, k, v, o and l are required)");
  VA_CHECK_ARG(nq > 0 && nk > 0 && bh > 0, "flash_attention2_forward: non-positive size");
  VA_CHECK_ARG(bh <= 65535, "flash_attention2_forward: bh=%d exceeds 65535", bh);
  dim3 grid(ceil_div(nq, 128), bh);
  const uintptr_t vec = sizeof(T) * 4 - 1;  // the split kernel reads 4 elements per load
  const bool aligned = !((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & vec);
  if ((long long)grid.x * bh < 2 * 148 && aligned) {
    // few rows in flight: several threads per row (R), chosen so the grid covers the SMs
    int R = 8;
    const int rmax = hd == 16 ? 16 : 32;  // R divides the head dim (each lane writes DV/R outputs)
    while (R < rmax && (long long)ceil_div(nq, 256 / R) * bh < 148) R *= 2;
    const dim3 gs(ceil_div(nq, 256 / R), bh);
    const size_t smem = (size_t)kSplitKeys * (hd + 4) * 2 * sizeof(float);
    int rc = VA_OK;
    auto launch = [&](auto kernel) {
      // the dynamic shared-memory limit is a per-device, per-kernel attribute: set it at every launch
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) {
        rc = set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        return;
      }
      kernel<<<gs, 256, smem, st>>>(q, k, v, o, l, nq, nk, scale);
    };
    switch (hd * 100 + R) {
      case 1608: launch(fa_fwd_split_kernel<T, 16, 16, 8>); break;
      case 1616: launch(fa_fwd_split_kernel<T, 16, 16, 16>); break;
      case 3208: launch(fa_fwd_split_kernel<T, 32, 32, 8>); break;
      case 3216: launch(fa_fwd_split_kernel<T, 32, 32, 16>); break;
      case 3232: launch(fa_fwd_split_kernel<T, 32, 32, 32>); break;
      case 6408: launch(fa_fwd_split_kernel<T, 64, 64, 8>); break;
      case 6416: launch(fa_fwd_split_kernel<T, 64, 64, 16>); break;
      case 6432: launch(fa_fwd_split_kernel<T, 64, 64, 32>); break;
      default: return set_error(VA_ERR_SHAPE, "flash_attention2_forward: head_dim %d unsupported (16/32/64)", hd);
    }
    if (rc) return rc;
    return check_launch("flash_attention2_forward (split rows)");
  }
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
  VA_CHECK_ARG(q && k && v && o && d_o && l && dq, "flash attention backward (dq): null pointer");
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
  VA_CHECK_ARG(q && k && v && o && d_o && l && dk && dv, "flash attention backward (dk, dv): null pointer");
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
