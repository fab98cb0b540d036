// PSA layout kernels: psa_pack_qkv, psa_extract_v_nchw, psa_merge_attn_nchw
// and their backwards (reference: src/models/yolo/kernels/attention/psa.rs).
//
// The reference launches one CTA per (section, bh, token) and reads NCHW with
// a channel stride of H*W per lane, i.e. uncoalesced.  Here every layout
// change is a 32-token × kd-channel tile transpose through shared memory, so
// both the NCHW side (tokens contiguous) and the packed side (kd contiguous)
// are read and written in full 32-element runs.
#include "va_common.cuh"

namespace va {

constexpr int TT = 32;  // tokens per tile

// NCHW channel block → packed [.., N, kd] rows.  One block per
// (tile of 32 tokens, section, bh).  `src_chan0(b,h,s)` picks the channels.
// ACC: accumulate into dst instead of storing (used by the backward scatter).
template <typename T>
__global__ void pack_qkv_kernel(const T* __restrict__ qkv, T* __restrict__ out, int qkv_h, int N,
                                int BH, int nh, int kd) {
  extern __shared__ float tile[];  // [TT][kd+1]
  const int n0 = blockIdx.x * TT;
  const int s = blockIdx.y;  // section 0..3
  const int bh = blockIdx.z;
  const int b = bh / nh, h = bh % nh;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const long long src_base = ((long long)b * qkv_h + h * 4 * kd + s * kd) * N;
  for (int d = ty; d < kd; d += blockDim.y) {
    int n = n0 + tx;
    tile[tx * (kd + 1) + d] = (n < N) ? ldg(qkv + src_base + (long long)d * N + n) : 0.f;
  }
  __syncthreads();
  const long long dst_base = (((long long)s * BH + bh) * N) * kd;
  // write rows: flatten (token, d) over the block
  const int nthr = blockDim.x * blockDim.y, tid = ty * blockDim.x + tx;
  for (int i = tid; i < TT * kd; i += nthr) {
    int t = i / kd, d = i % kd, n = n0 + t;
    if (n < N) st(out + dst_base + (long long)n * kd + d, tile[t * (kd + 1) + d]);
  }
}

// Backward of pack: packed rows → NCHW, accumulated (psa.rs:229-232).
__global__ void pack_qkv_backward_kernel(const float* __restrict__ dp, float* __restrict__ dqkv,
                                         int qkv_h, int N, int BH, int nh, int kd) {
  extern __shared__ float tile[];
  const int n0 = blockIdx.x * TT;
  const int s = blockIdx.y, bh = blockIdx.z;
  const int b = bh / nh, h = bh % nh;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int nthr = blockDim.x * blockDim.y, tid = ty * blockDim.x + tx;
  const long long src_base = (((long long)s * BH + bh) * N) * kd;
  for (int i = tid; i < TT * kd; i += nthr) {
    int t = i / kd, d = i % kd, n = n0 + t;
    tile[t * (kd + 1) + d] = (n < N) ? dp[src_base + (long long)n * kd + d] : 0.f;
  }
  __syncthreads();
  const long long dst_base = ((long long)b * qkv_h + h * 4 * kd + s * kd) * N;
  for (int d = ty; d < kd; d += blockDim.y) {
    int n = n0 + tx;
    if (n < N) dqkv[dst_base + (long long)d * N + n] += tile[tx * (kd + 1) + d];
  }
}

// extract_v: per (b, h) the 2*kd V channels are one contiguous run of
// 2*kd*N elements in both tensors, so this is a strided block copy.
template <typename T, bool ACC>
__global__ void copy_v_kernel(const T* __restrict__ src, T* __restrict__ dst, long long src_stride_b,
                              long long dst_stride_b, long long src_off_h, long long dst_off_h,
                              long long run, int nh, int B) {
  // blockIdx.y = b*nh + h
  const int bh = blockIdx.y, b = bh / nh, h = bh % nh;
  const T* s = src + b * src_stride_b + h * src_off_h;
  T* d = dst + b * dst_stride_b + h * dst_off_h;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < run;
       i += (long long)gridDim.x * blockDim.x) {
    if (ACC) st(d + i, ld(d + i) + ldg(s + i));
    else d[i] = s[i];
  }
}

// merge: lo/hi [BH, N, kd] → NCHW channels h*2kd + {0, kd} + d.
template <typename T>
__global__ void merge_kernel(const T* __restrict__ lo, const T* __restrict__ hi, T* __restrict__ out,
                             int c, int N, int nh, int kd) {
  extern __shared__ float tile[];  // [TT][2kd+1]
  const int n0 = blockIdx.x * TT, bh = blockIdx.y;
  const int b = bh / nh, h = bh % nh;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int nthr = blockDim.x * blockDim.y, tid = ty * blockDim.x + tx;
  const int w = 2 * kd + 1;
  const long long src_base = (long long)bh * N * kd;
  for (int i = tid; i < TT * kd; i += nthr) {
    int t = i / kd, d = i % kd, n = n0 + t;
    bool ok = n < N;
    tile[t * w + d] = ok ? ldg(lo + src_base + (long long)n * kd + d) : 0.f;
    tile[t * w + kd + d] = ok ? ldg(hi + src_base + (long long)n * kd + d) : 0.f;
  }
  __syncthreads();
  const long long dst_base = ((long long)b * c + h * 2 * kd) * N;
  for (int d = ty; d < 2 * kd; d += blockDim.y) {
    int n = n0 + tx;
    if (n < N) st(out + dst_base + (long long)d * N + n, tile[tx * w + d]);
  }
}

__global__ void merge_backward_kernel(const float* __restrict__ dm, float* __restrict__ dlo,
                                      float* __restrict__ dhi, int c, int N, int nh, int kd) {
  extern __shared__ float tile[];
  const int n0 = blockIdx.x * TT, bh = blockIdx.y;
  const int b = bh / nh, h = bh % nh;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int nthr = blockDim.x * blockDim.y, tid = ty * blockDim.x + tx;
  const int w = 2 * kd + 1;
  const long long src_base = ((long long)b * c + h * 2 * kd) * N;
  for (int d = ty; d < 2 * kd; d += blockDim.y) {
    int n = n0 + tx;
    tile[tx * w + d] = (n < N) ? dm[src_base + (long long)d * N + n] : 0.f;
  }
  __syncthreads();
  const long long dst_base = (long long)bh * N * kd;
  for (int i = tid; i < TT * kd; i += nthr) {
    int t = i / kd, d = i % kd, n = n0 + t;
    if (n < N) {
      dlo[dst_base + (long long)n * kd + d] = tile[t * w + d];
      dhi[dst_base + (long long)n * kd + d] = tile[t * w + kd + d];
    }
  }
}

static bool kd_ok(int kd) { return kd == 8 || kd == 16 || kd == 32 || kd == 64; }

template <typename T>
static int pack_qkv(const T* qkv, T* out, int qkv_h, int H, int W, int B, int nh, cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && nh > 0 && qkv_h > 0, "psa_pack_qkv: non-positive size");
  VA_CHECK_ARG(qkv_h % (4 * nh) == 0, "psa_pack_qkv: qkv_h=%d not a multiple of 4*num_heads", qkv_h);
  int kd = qkv_h / (4 * nh), N = H * W;
  VA_CHECK_ARG(kd_ok(kd), "psa_pack_qkv: key_dim %d unsupported (8/16/32/64)", kd);
  dim3 grid(ceil_div(N, TT), 4, B * nh), block(TT, 8);
  pack_qkv_kernel<T><<<grid, block, TT * (kd + 1) * sizeof(float), st>>>(qkv, out, qkv_h, N, B * nh, nh, kd);
  return check_launch("psa_pack_qkv");
}

template <typename T>
static int extract_v(const T* qkv, T* v, int qkv_h, int c, int H, int W, int nh, int B, cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && nh > 0, "psa_extract_v_nchw: non-positive size");
  VA_CHECK_ARG(qkv_h % (4 * nh) == 0 && c * 2 == qkv_h, "psa_extract_v_nchw: need qkv_h = 2c = 4*nh*kd");
  int kd = qkv_h / (4 * nh);
  long long N = (long long)H * W, run = 2LL * kd * N;
  dim3 grid(ceil_div(run, 256 * 4) > 64 ? 64 : ceil_div(run, 256 * 4), B * nh);
  copy_v_kernel<T, false><<<grid, 256, 0, st>>>(qkv + 2LL * kd * N, v, qkv_h * N, c * N, 4LL * kd * N,
                                                 2LL * kd * N, run, nh, B);
  return check_launch("psa_extract_v_nchw");
}

template <typename T>
static int merge(const T* lo, const T* hi, T* out, int c, int H, int W, int nh, int B, cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && nh > 0, "psa_merge_attn_nchw: non-positive size");
  VA_CHECK_ARG(c % (2 * nh) == 0, "psa_merge_attn_nchw: c=%d not a multiple of 2*num_heads", c);
  int kd = c / (2 * nh), N = H * W;
  VA_CHECK_ARG(kd_ok(kd), "psa_merge_attn_nchw: key_dim %d unsupported", kd);
  dim3 grid(ceil_div(N, TT), B * nh), block(TT, 8);
  merge_kernel<T><<<grid, block, TT * (2 * kd + 1) * sizeof(float), st>>>(lo, hi, out, c, N, nh, kd);
  return check_launch("psa_merge_attn_nchw");
}

}  // namespace va

using namespace va;
typedef __nv_bfloat16 bf16;

extern "C" {

int va_psa_pack_qkv_f32(const float* qkv, float* out, int qkv_h, int H, int W, int B, int nh,
                        va_stream_t s) {
  return pack_qkv(qkv, out, qkv_h, H, W, B, nh, (cudaStream_t)s);
}
int va_psa_pack_qkv_bf16(const va_bf16* qkv, va_bf16* out, int qkv_h, int H, int W, int B, int nh,
                         va_stream_t s) {
  return pack_qkv((const bf16*)qkv, (bf16*)out, qkv_h, H, W, B, nh, (cudaStream_t)s);
}

int va_psa_pack_qkv_backward_f32(const float* dp, float* dqkv, int qkv_h, int H, int W, int B, int nh,
                                 va_stream_t s) {
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && nh > 0 && qkv_h % (4 * nh) == 0,
               "psa_pack_qkv_backward: bad sizes");
  int kd = qkv_h / (4 * nh), N = H * W;
  VA_CHECK_ARG(kd_ok(kd), "psa_pack_qkv_backward: key_dim %d unsupported", kd);
  dim3 grid(ceil_div(N, TT), 4, B * nh), block(TT, 8);
  pack_qkv_backward_kernel<<<grid, block, TT * (kd + 1) * sizeof(float), (cudaStream_t)s>>>(
      dp, dqkv, qkv_h, N, B * nh, nh, kd);
  return check_launch("psa_pack_qkv_backward");
}

int va_psa_extract_v_nchw_f32(const float* qkv, float* v, int qkv_h, int c, int H, int W, int nh, int B,
                              va_stream_t s) {
  return extract_v(qkv, v, qkv_h, c, H, W, nh, B, (cudaStream_t)s);
}
int va_psa_extract_v_nchw_bf16(const va_bf16* qkv, va_bf16* v, int qkv_h, int c, int H, int W, int nh,
                               int B, va_stream_t s) {
  return extract_v((const bf16*)qkv, (bf16*)v, qkv_h, c, H, W, nh, B, (cudaStream_t)s);
}

int va_psa_extract_v_backward_f32(const float* dv, float* dqkv, int qkv_h, int c, int H, int W, int nh,
                                  int B, va_stream_t s) {
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && nh > 0, "psa_extract_v_backward: non-positive size");
  VA_CHECK_ARG(qkv_h % (4 * nh) == 0 && c * 2 == qkv_h, "psa_extract_v_backward: need qkv_h = 2c");
  int kd = qkv_h / (4 * nh);
  long long N = (long long)H * W, run = 2LL * kd * N;
  dim3 grid(ceil_div(run, 256 * 4) > 64 ? 64 : ceil_div(run, 256 * 4), B * nh);
  copy_v_kernel<float, true><<<grid, 256, 0, (cudaStream_t)s>>>(dv, dqkv + 2LL * kd * N, c * N, qkv_h * N,
                                                                2LL * kd * N, 4LL * kd * N, run, nh, B);
  return check_launch("psa_extract_v_backward");
}

int va_psa_merge_attn_nchw_f32(const float* lo, const float* hi, float* out, int c, int H, int W, int nh,
                               int B, va_stream_t s) {
  return merge(lo, hi, out, c, H, W, nh, B, (cudaStream_t)s);
}
int va_psa_merge_attn_nchw_bf16(const va_bf16* lo, const va_bf16* hi, va_bf16* out, int c, int H, int W,
                                int nh, int B, va_stream_t s) {
  return merge((const bf16*)lo, (const bf16*)hi, (bf16*)out, c, H, W, nh, B, (cudaStream_t)s);
}

int va_psa_merge_attn_backward_f32(const float* dm, float* dlo, float* dhi, int c, int H, int W, int nh,
                                   int B, va_stream_t s) {
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && nh > 0 && c % (2 * nh) == 0,
               "psa_merge_attn_backward: bad sizes");
  int kd = c / (2 * nh), N = H * W;
  VA_CHECK_ARG(kd_ok(kd), "psa_merge_attn_backward: key_dim %d unsupported", kd);
  dim3 grid(ceil_div(N, TT), B * nh), block(TT, 8);
  merge_backward_kernel<<<grid, block, TT * (2 * kd + 1) * sizeof(float), (cudaStream_t)s>>>(
      dm, dlo, dhi, c, N, nh, kd);
  return check_launch("psa_merge_attn_backward");
}

}  // extern "C"
