// Convolution pieces of the PSA block on the FFMA path: 1×1 conv (+bias,
// optional prologue add) as a tiled SGEMM per image, depthwise 3×3 (+bias)
// and its backward.  Reference nodes: conv_bn (src/models/yolo/yolo26/blocks/
// conv.rs:53-69) for qkv/pe/proj with BN folded (graph.optimise()), and the
// PE add (c2psa.rs:110-111).  The bf16 tensor-core path replaces the 1×1
// convs with tcgen05 GEMMs (va_tc_psa.cu).
#include "va_common.cuh"

namespace va {

// Y[b][o][n] = sum_i W[o][i] * (X[b][i][n] + X2[b][i][n]) + bias[o]
// 64(o) × 64(n) tiles, k-step 16, 256 threads × (4×4) outputs.
template <typename T, typename TW>
__global__ void __launch_bounds__(256) conv1x1_kernel(const T* __restrict__ x, const T* __restrict__ x2,
                                                      const TW* __restrict__ w, const float* __restrict__ bias,
                                                      T* __restrict__ y, int cin, int cout, int HW) {
  __shared__ float Ws[16][64 + 4];
  __shared__ float Xs[16][64 + 4];
  const int b = blockIdx.z;
  const int o0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const T* xb = x + (long long)b * cin * HW;
  const T* x2b = x2 ? x2 + (long long)b * cin * HW : nullptr;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < cin; k0 += 16) {
    {
      int o = tid / 4, i = (tid % 4) * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        int oo = o0 + o, ii = k0 + i + u;
        Ws[i + u][o] = (oo < cout && ii < cin) ? ldg(w + (long long)oo * cin + ii) : 0.f;
      }
    }
    {
      int i = tid / 16, n = (tid % 16) * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        int ii = k0 + i, nn = n0 + n + u;
        float val = 0.f;
        if (ii < cin && nn < HW) {
          val = ldg(xb + (long long)ii * HW + nn);
          if (x2b) val += ldg(x2b + (long long)ii * HW + nn);
        }
        Xs[i][n + u] = val;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], bv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) { a[u] = Ws[kk][ty * 4 + u]; bv[u] = Xs[kk][tx * 4 + u]; }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(a[r], bv[c], acc[r][c]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    int o = o0 + ty * 4 + r;
    if (o >= cout) continue;
    float bo = bias ? bias[o] : 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      int n = n0 + tx * 4 + c;
      if (n < HW) st(y + ((long long)b * cout + o) * HW + n, acc[r][c] + bo);
    }
  }
}

template <typename T, typename TW>
__global__ void dwconv3x3_kernel(const T* __restrict__ x, const TW* __restrict__ w, const float* __restrict__ bias,
                                 T* __restrict__ y, int C, int H, int W, long long total) {
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    int j = idx % W;
    int i = (idx / W) % H;
    long long bc = idx / ((long long)H * W);
    int c = bc % C;
    const T* xp = x + bc * H * W;
    float acc = bias ? bias[c] : 0.f;
#pragma unroll
    for (int di = 0; di < 3; ++di) {
      int ii = i + di - 1;
      if (ii < 0 || ii >= H) continue;
#pragma unroll
      for (int dj = 0; dj < 3; ++dj) {
        int jj = j + dj - 1;
        if (jj < 0 || jj >= W) continue;
        acc = fmaf(ldg(w + c * 9 + di * 3 + dj), ldg(xp + ii * W + jj), acc);
      }
    }
    st(y + idx, acc);
  }
}

__global__ void dwconv3x3_dx_kernel(const float* __restrict__ w, const float* __restrict__ dy,
                                    float* __restrict__ dx, int C, int H, int W, long long total) {
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    int j = idx % W;
    int i = (idx / W) % H;
    long long bc = idx / ((long long)H * W);
    int c = bc % C;
    const float* g = dy + bc * H * W;
    float acc = 0.f;
    // y[i'] uses x[i'+di-1] → x[i] receives from y[i-di+1]
    for (int di = 0; di < 3; ++di) {
      int ii = i - di + 1;
      if (ii < 0 || ii >= H) continue;
      for (int dj = 0; dj < 3; ++dj) {
        int jj = j - dj + 1;
        if (jj < 0 || jj >= W) continue;
        acc = fmaf(w[c * 9 + di * 3 + dj], g[ii * W + jj], acc);
      }
    }
    dx[idx] = acc;
  }
}

// dW[c][di][dj] = sum_{b,i,j} dy[b,c,i,j] * x[b,c,i+di-1,j+dj-1]; one block
// per channel, fixed-order tree reduction (deterministic).
__global__ void __launch_bounds__(256) dwconv3x3_dw_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                                           float* __restrict__ dw, int B, int C, int H, int W) {
  const int c = blockIdx.x;
  float acc[9] = {};
  const long long HW = (long long)H * W;
  for (long long t = threadIdx.x; t < (long long)B * HW; t += blockDim.x) {
    int b = t / HW;
    int n = t % HW;
    int i = n / W, j = n % W;
    const float* xp = x + ((long long)b * C + c) * HW;
    float g = dy[((long long)b * C + c) * HW + n];
#pragma unroll
    for (int di = 0; di < 3; ++di) {
      int ii = i + di - 1;
#pragma unroll
      for (int dj = 0; dj < 3; ++dj) {
        int jj = j + dj - 1;
        if (ii >= 0 && ii < H && jj >= 0 && jj < W) acc[di * 3 + dj] = fmaf(g, xp[ii * W + jj], acc[di * 3 + dj]);
      }
    }
  }
  __shared__ float red[9][256];
#pragma unroll
  for (int u = 0; u < 9; ++u) red[u][threadIdx.x] = acc[u];
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s)
      for (int u = 0; u < 9; ++u) red[u][threadIdx.x] += red[u][threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x < 9) dw[c * 9 + threadIdx.x] = red[threadIdx.x][0];
}

// Weight gradient of the 1×1 conv (conv_bn backward, BN folded):
// dW[o][i] = Σ_b Σ_n dY[b][o][n] · (X[b][i][n] + X2[b][i][n]).  64(o) × 64(i)
// tiles, the (b, n) reduction in 16-token steps through shared memory, in a
// fixed order — deterministic, no atomics.
__global__ void __launch_bounds__(256) conv1x1_dw_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                         const float* __restrict__ x2, float* __restrict__ dw,
                                                         int B, int cin, int cout, int HW) {
  __shared__ float Gs[16][64 + 4];
  __shared__ float Xs[16][64 + 4];
  const int o0 = blockIdx.y * 64, i0 = blockIdx.x * 64;
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  float acc[4][4] = {};
  for (int b = 0; b < B; ++b) {
    const float* gb = dy + (long long)b * cout * HW;
    const float* xb = x + (long long)b * cin * HW;
    const float* x2b = x2 ? x2 + (long long)b * cin * HW : nullptr;
    for (int n0 = 0; n0 < HW; n0 += 16) {
      {  // 64 rows × 16 tokens of dY and of X, one float4-sized strip per thread each
        const int r = tid / 4, n = (tid % 4) * 4;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int nn = n0 + n + u, oo = o0 + r, ii = i0 + r;
          Gs[n + u][r] = (oo < cout && nn < HW) ? gb[(long long)oo * HW + nn] : 0.f;
          float xv = 0.f;
          if (ii < cin && nn < HW) {
            xv = xb[(long long)ii * HW + nn];
            if (x2b) xv += x2b[(long long)ii * HW + nn];
          }
          Xs[n + u][r] = xv;
        }
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        float a[4], bv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) { a[u] = Gs[kk][ty * 4 + u]; bv[u] = Xs[kk][tx * 4 + u]; }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(a[r], bv[c], acc[r][c]);
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int o = o0 + ty * 4 + r;
    if (o >= cout) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = i0 + tx * 4 + c;
      if (i < cin) dw[(long long)o * cin + i] = acc[r][c];
    }
  }
}

// db[o] = Σ_b Σ_n dY[b][o][n]: one warp per channel, lanes stride the tokens,
// then a fixed shuffle tree (deterministic).
__global__ void __launch_bounds__(256) channel_sum_kernel(const float* __restrict__ dy, float* __restrict__ db, int B,
                                                          int C, int HW) {
  const int o = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (o >= C) return;
  float s = 0.f;
  for (int b = 0; b < B; ++b) {
    const float* g = dy + ((long long)b * C + o) * HW;
    for (int n = lane; n < HW; n += 32) s += g[n];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) db[o] = s;
}

// wt[i][o] = w[o][i]
__global__ void transpose_kernel(const float* __restrict__ w, float* __restrict__ wt, int rows, int cols) {
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= (long long)rows * cols) return;
  const int r = (int)(t / cols), c = (int)(t % cols);
  wt[(long long)c * rows + r] = w[t];
}

int conv1x1_dw_f32(const float* dy, const float* x, const float* x2, float* dw, int B, int cin, int cout, int HW,
                   cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && cin > 0 && cout > 0 && HW > 0, "conv1x1 backward: bad sizes");
  conv1x1_dw_kernel<<<dim3(ceil_div(cin, 64), ceil_div(cout, 64)), 256, 0, st>>>(dy, x, x2, dw, B, cin, cout, HW);
  return check_launch("conv1x1 dw");
}

int channel_sum_f32(const float* dy, float* db, int B, int C, int HW, cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && C > 0 && HW > 0, "channel sum: bad sizes");
  channel_sum_kernel<<<ceil_div(C, 8), 256, 0, st>>>(dy, db, B, C, HW);
  return check_launch("channel sum");
}

int transpose_f32(const float* w, float* wt, int rows, int cols, cudaStream_t st) {
  const long long n = (long long)rows * cols;
  transpose_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, wt, rows, cols);
  return check_launch("transpose");
}

template <typename T, typename TW>
int conv1x1(const T* x, const T* x2, const TW* w, const float* bias, T* y, int B, int cin, int cout, int HW,
            cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && cin > 0 && cout > 0 && HW > 0 && B <= 65535, "conv1x1: bad sizes");
  dim3 grid(ceil_div(HW, 64), ceil_div(cout, 64), B);
  conv1x1_kernel<T, TW><<<grid, 256, 0, st>>>(x, x2, w, bias, y, cin, cout, HW);
  return check_launch("conv1x1");
}

template <typename T, typename TW>
int dwconv3x3(const T* x, const TW* w, const float* bias, T* y, int B, int C, int H, int W, cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && C > 0 && H > 0 && W > 0, "dwconv3x3: bad sizes");
  long long total = (long long)B * C * H * W;
  int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
  dwconv3x3_kernel<T, TW><<<blocks, 256, 0, st>>>(x, w, bias, y, C, H, W, total);
  return check_launch("dwconv3x3");
}

template int conv1x1<float, float>(const float*, const float*, const float*, const float*, float*, int, int, int,
                                   int, cudaStream_t);
template int conv1x1<__nv_bfloat16, __nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*,
                                                   const __nv_bfloat16*, const float*, __nv_bfloat16*, int, int,
                                                   int, int, cudaStream_t);
template int dwconv3x3<float, float>(const float*, const float*, const float*, float*, int, int, int, int,
                                     cudaStream_t);
template int dwconv3x3<__nv_bfloat16, __nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, const float*,
                                                     __nv_bfloat16*, int, int, int, int, cudaStream_t);

}  // namespace va

using namespace va;

extern "C" {

int va_conv1x1_bias_f32(const float* x, const float* w, const float* bias, float* y, int B, int cin, int cout,
                        int HW, va_stream_t s) {
  return conv1x1<float, float>(x, nullptr, w, bias, y, B, cin, cout, HW, (cudaStream_t)s);
}

int va_dwconv3x3_bias_f32(const float* x, const float* w, const float* bias, float* y, int B, int C, int H, int W,
                          va_stream_t s) {
  return dwconv3x3<float, float>(x, w, bias, y, B, C, H, W, (cudaStream_t)s);
}

int va_dwconv3x3_backward_f32(const float* x, const float* w, const float* dy, float* dx, float* dw, int B, int C,
                              int H, int W, va_stream_t s) {
  VA_CHECK_ARG(B > 0 && C > 0 && H > 0 && W > 0, "dwconv3x3_backward: bad sizes");
  long long total = (long long)B * C * H * W;
  int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
  if (dx) dwconv3x3_dx_kernel<<<blocks, 256, 0, (cudaStream_t)s>>>(w, dy, dx, C, H, W, total);
  int rc = check_launch("dwconv3x3_backward dx");
  if (rc) return rc;
  if (dw) dwconv3x3_dw_kernel<<<C, 256, 0, (cudaStream_t)s>>>(x, dy, dw, B, C, H, W);
  return check_launch("dwconv3x3_backward dw");
}

}  // extern "C"
