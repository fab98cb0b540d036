// Multi-scale deformable attention (MSDeformAttn, RF-DETR decoder) forward and
// backward.  The reference has no deformable attention; the operator is the
// published multi-scale deformable attention core (Deformable DETR, eq. 3)
// with PyTorch grid_sample(align_corners=False, padding_mode='zeros')
// sampling: pixel coordinates x = loc_x·W − 0.5, y = loc_y·H − 0.5.
//
// Layouts (as the PyTorch op): value [B][S][nh][dh], spatial_shapes [L][2]
// (H, W; int64), level_start [L] (int64), loc [B][Q][nh][L][P][2] (x, y),
// attn [B][Q][nh][L][P] (already softmaxed), out [B][Q][nh·dh].
//
// Forward: a group of G = dh / VEC threads serves one (b, q, h); each thread
// owns VEC channels and reads every bilinear corner as one 16-byte load
// (f32: 4 channels, bf16: 8).  The block's locations and weights are staged
// in shared memory with coalesced loads first.  The op is a gather: its HBM
// floor is one pass over the value map.
//
// Backward, without atomics: pass 1 (same thread groups) recomputes each
// sample, writes grad_attn and grad_loc, and records every corner's
// grad_value contribution (destination pixel, weight A·w) in a slot fixed by
// (b, h, l, q, p, corner).  Pass 2 runs one CTA per (b, h, l): it owns that
// slice of grad_value exclusively, sorts its contributions by (pixel, slot)
// in shared memory (bitonic sort of unique 64-bit keys) and each thread sums
// whole pixel segments in slot order — deterministic results, no atomics.
#include "va_common.cuh"
#include "va_psa.h"

namespace va {

namespace {

constexpr int kMsdaThreads = 256;
constexpr int kMaxLevels = 8;
constexpr int kMaxContrib = 16384;   // contributions per (b, h, l) sorted in shared memory

template <typename T> struct Vec;
template <> struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&v)[4]) {
    const float4 u = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
  }
  __device__ static void store(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};

struct Levels {
  int H[kMaxLevels], W[kMaxLevels], s0[kMaxLevels];
};

__device__ __forceinline__ void load_levels(Levels& lv, const int64_t* shapes, const int64_t* lstart, int L) {
  if (threadIdx.x < L) {
    lv.H[threadIdx.x] = (int)shapes[2 * threadIdx.x];
    lv.W[threadIdx.x] = (int)shapes[2 * threadIdx.x + 1];
    lv.s0[threadIdx.x] = (int)lstart[threadIdx.x];
  }
}

// Bilinear corners of a sample: corner c = dy*2 + dx, weight and validity.
struct Corners {
  int pix[4];
  float w[4];
  bool ok[4];
  float fx, fy;
};

__device__ __forceinline__ Corners corners(float lx, float ly, int H, int W) {
  Corners c;
  const float x = fmaf(lx, (float)W, -0.5f), y = fmaf(ly, (float)H, -0.5f);
  const float xf = floorf(x), yf = floorf(y);
  c.fx = x - xf;
  c.fy = y - yf;
  const int x0 = (int)xf, y0 = (int)yf;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int dx = k & 1, dy = k >> 1;
    const int xi = x0 + dx, yi = y0 + dy;
    c.ok[k] = xi >= 0 && xi < W && yi >= 0 && yi < H;
    c.pix[k] = c.ok[k] ? yi * W + xi : 0;
    c.w[k] = (dy ? c.fy : 1.f - c.fy) * (dx ? c.fx : 1.f - c.fx);
  }
  return c;
}

template <typename TV, int DH>
__global__ void __launch_bounds__(kMsdaThreads)
msda_fwd_kernel(const TV* __restrict__ value, const int64_t* __restrict__ shapes, const int64_t* __restrict__ lstart,
                const float* __restrict__ loc, const float* __restrict__ attn, TV* __restrict__ out, int B, int S,
                int nh, int L, int Q, int P) {
  constexpr int VEC = Vec<TV>::N, G = DH / VEC, ITEMS = kMsdaThreads / G;
  extern __shared__ float sm_f[];
  __shared__ Levels lv;
  const int LP = L * P;
  float* s_loc = sm_f;                 // [ITEMS][LP][2]
  float* s_att = sm_f + ITEMS * LP * 2;  // [ITEMS][LP]
  load_levels(lv, shapes, lstart, L);
  const long long item0 = (long long)blockIdx.x * ITEMS;
  const long long nitems = (long long)B * Q * nh;
  const int nblk = (int)min((long long)ITEMS, nitems - item0);
  for (int i = threadIdx.x; i < nblk * LP * 2; i += kMsdaThreads) s_loc[i] = __ldg(loc + item0 * LP * 2 + i);
  for (int i = threadIdx.x; i < nblk * LP; i += kMsdaThreads) s_att[i] = __ldg(attn + item0 * LP + i);
  __syncthreads();
  const int it = threadIdx.x / G, part = threadIdx.x % G;
  if (it >= nblk) return;
  const long long item = item0 + it;  // = (b*Q + q)*nh + h
  const int h = (int)(item % nh);
  const int b = (int)(item / ((long long)Q * nh));
  float acc[VEC] = {};
  const float* il = s_loc + it * LP * 2;
  const float* ia = s_att + it * LP;
  for (int l = 0; l < L; ++l) {
    const int H = lv.H[l], W = lv.W[l];
    const TV* vbase = value + (((size_t)b * S + lv.s0[l]) * nh + h) * DH + part * VEC;
    for (int p = 0; p < P; ++p) {
      const int s = l * P + p;
      const Corners c = corners(il[2 * s], il[2 * s + 1], H, W);
      const float a = ia[s];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (!c.ok[k]) continue;
        float v[VEC];
        Vec<TV>::load(vbase + (size_t)c.pix[k] * nh * DH, v);
        const float cw = a * c.w[k];
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] = fmaf(cw, v[e], acc[e]);
      }
    }
  }
  Vec<TV>::store(out + item * DH + part * VEC, acc);
}

// Pass 1 of the backward: grad_attn, grad_loc, and the grad_value
// contributions (pixel within the level, weight) in slot order.
template <typename TV, int DH>
__global__ void __launch_bounds__(kMsdaThreads)
msda_bwd_sample_kernel(const TV* __restrict__ value, const int64_t* __restrict__ shapes,
                       const int64_t* __restrict__ lstart, const float* __restrict__ loc,
                       const float* __restrict__ attn, const TV* __restrict__ grad_out, float* __restrict__ grad_loc,
                       float* __restrict__ grad_attn, int* __restrict__ c_pix, float* __restrict__ c_w, int B, int S,
                       int nh, int L, int Q, int P) {
  constexpr int VEC = Vec<TV>::N, G = DH / VEC, ITEMS = kMsdaThreads / G;
  __shared__ Levels lv;
  load_levels(lv, shapes, lstart, L);
  __syncthreads();
  const long long item = (long long)blockIdx.x * ITEMS + threadIdx.x / G;
  const int part = threadIdx.x % G;
  const bool live = item < (long long)B * Q * nh;
  const long long it = live ? item : 0;
  const int h = (int)(it % nh);
  const int q = (int)((it / nh) % Q);
  const int b = (int)(it / ((long long)Q * nh));
  const int LP = L * P;
  float g[VEC];
  Vec<TV>::load(grad_out + it * DH + part * VEC, g);
  for (int l = 0; l < L; ++l) {
    const int H = lv.H[l], W = lv.W[l];
    const TV* vbase = value + (((size_t)b * S + lv.s0[l]) * nh + h) * DH + part * VEC;
    for (int p = 0; p < P; ++p) {
      const int s = l * P + p;
      const float lx = __ldg(loc + (it * LP + s) * 2), ly = __ldg(loc + (it * LP + s) * 2 + 1);
      const float a = __ldg(attn + it * LP + s);
      const Corners c = corners(lx, ly, H, W);
      float gdv[4];  // g · v at each corner (this thread's channels, then the group's)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float d = 0.f;
        if (c.ok[k]) {
          float v[VEC];
          Vec<TV>::load(vbase + (size_t)c.pix[k] * nh * DH, v);
#pragma unroll
          for (int e = 0; e < VEC; ++e) d = fmaf(g[e], v[e], d);
        }
        gdv[k] = d;
      }
#pragma unroll
      for (int off = 1; off < G; off <<= 1)
#pragma unroll
        for (int k = 0; k < 4; ++k) gdv[k] += __shfl_xor_sync(0xffffffffu, gdv[k], off);
      if (live && part == 0) {
        float ga = 0.f, gx = 0.f, gy = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int dx = k & 1, dy = k >> 1;
          ga = fmaf(c.w[k], gdv[k], ga);
          gx = fmaf((dy ? c.fy : 1.f - c.fy) * (dx ? 1.f : -1.f), gdv[k], gx);
          gy = fmaf((dx ? c.fx : 1.f - c.fx) * (dy ? 1.f : -1.f), gdv[k], gy);
        }
        grad_attn[it * LP + s] = ga;
        grad_loc[(it * LP + s) * 2] = a * gx * (float)W;
        grad_loc[(it * LP + s) * 2 + 1] = a * gy * (float)H;
        // slot of (b, h, l, q, p, corner)
        const size_t slot = ((((size_t)b * nh + h) * L + l) * Q + q) * (size_t)(P * 4) + p * 4;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          c_pix[slot + k] = c.ok[k] ? c.pix[k] : -1;
          c_w[slot + k] = a * c.w[k];
        }
      }
    }
  }
}

// Pass 2: CTA (l, h, b) owns grad_value[b, level l pixels, h, :].
template <typename TV, int DH>
__global__ void __launch_bounds__(512)
msda_bwd_value_kernel(const int64_t* __restrict__ shapes, const int64_t* __restrict__ lstart,
                      const TV* __restrict__ grad_out, const int* __restrict__ c_pix, const float* __restrict__ c_w,
                      TV* __restrict__ grad_value, int S, int nh, int L, int Q, int P, int npad) {
  extern __shared__ unsigned long long keys[];  // [npad]
  const int l = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int H = (int)shapes[2 * l], W = (int)shapes[2 * l + 1], s0 = (int)lstart[l];
  const int n = Q * P * 4;
  const size_t base = (((size_t)b * nh + h) * L + l) * (size_t)n;
  for (int i = threadIdx.x; i < npad; i += blockDim.x) {
    unsigned long long k = ~0ull;
    if (i < n) {
      const int px = c_pix[base + i];
      if (px >= 0) k = ((unsigned long long)(unsigned)px << 32) | (unsigned)i;
    }
    keys[i] = k;
  }
  __syncthreads();
  // bitonic sort, ascending
  for (int size = 2; size <= npad; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < npad / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const unsigned long long a = keys[lo], c = keys[hi];
        if ((a > c) == up) {
          keys[lo] = c;
          keys[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  // one thread per destination pixel: sum its segment in slot order
  const TV* go = grad_out + (size_t)h * DH;
  for (int px = threadIdx.x; px < H * W; px += blockDim.x) {
    const unsigned long long key = (unsigned long long)(unsigned)px << 32;
    int lo = 0, hi = npad;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (keys[mid] < key) lo = mid + 1;
      else hi = mid;
    }
    float acc[DH] = {};
    for (int i = lo; i < npad && (keys[i] >> 32) == (unsigned long long)(unsigned)px; ++i) {
      const int slot = (int)(keys[i] & 0xffffffffu);
      const int q = slot / (P * 4);
      const float w = c_w[base + slot];
      const TV* gr = go + ((size_t)b * Q + q) * nh * DH;
#pragma unroll
      for (int e0 = 0; e0 < DH; e0 += Vec<TV>::N) {
        float v[Vec<TV>::N];
        Vec<TV>::load(gr + e0, v);
#pragma unroll
        for (int e = 0; e < Vec<TV>::N; ++e) acc[e0 + e] = fmaf(w, v[e], acc[e0 + e]);
      }
    }
    TV* dst = grad_value + (((size_t)b * S + s0 + px) * nh + h) * DH;
#pragma unroll
    for (int e0 = 0; e0 < DH; e0 += Vec<TV>::N) {
      float v[Vec<TV>::N];
#pragma unroll
      for (int e = 0; e < Vec<TV>::N; ++e) v[e] = acc[e0 + e];
      Vec<TV>::store(dst + e0, v);
    }
  }
}

int check_msda(int B, int S, int nh, int dh, int L, int Q, int P, const void* value, const void* out) {
  VA_CHECK_ARG(B > 0 && S > 0 && nh > 0 && L > 0 && Q > 0 && P > 0, "msdeform_attn: non-positive size");
  VA_CHECK_ARG(L <= kMaxLevels, "msdeform_attn: %d levels > %d", L, kMaxLevels);
  VA_CHECK_ARG(dh == 16 || dh == 32, "msdeform_attn: head dim %d unsupported (16, 32)", dh);
  if ((reinterpret_cast<uintptr_t>(value) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return set_error(VA_ERR_ALIGN, "msdeform_attn: value/out need 16-byte alignment");
  return VA_OK;
}

template <typename TV>
int msda_fwd(const TV* value, const int64_t* shapes, const int64_t* lstart, const float* loc, const float* attn, TV* out,
             int B, int S, int nh, int dh, int L, int Q, int P, cudaStream_t st) {
  if (int rc = check_msda(B, S, nh, dh, L, Q, P, value, out)) return rc;
  const long long items = (long long)B * Q * nh;
  auto launch = [&](auto kernel, int G) {
    const int per = kMsdaThreads / G;
    const size_t smem = (size_t)per * L * P * 3 * sizeof(float);
    const long long blocks = (items + per - 1) / per;
    kernel<<<(unsigned)blocks, kMsdaThreads, smem, st>>>(value, shapes, lstart, loc, attn, out, B, S, nh, L, Q, P);
  };
  constexpr int VEC = Vec<TV>::N;
  if (dh == 16) launch(msda_fwd_kernel<TV, 16>, 16 / VEC);
  else launch(msda_fwd_kernel<TV, 32>, 32 / VEC);
  return check_launch("msdeform_attn forward");
}

size_t msda_ws_bytes(int B, int nh, int L, int Q, int P) {
  const size_t n = (size_t)B * nh * L * Q * P * 4;
  return align256(n * sizeof(int)) + align256(n * sizeof(float));
}

template <typename TV>
int msda_bwd(const TV* value, const int64_t* shapes, const int64_t* lstart, const float* loc, const float* attn,
             const TV* grad_out, TV* grad_value, float* grad_loc, float* grad_attn, int B, int S, int nh, int dh,
             int L, int Q, int P, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (int rc = check_msda(B, S, nh, dh, L, Q, P, value, grad_value)) return rc;
  const int n = Q * P * 4;
  VA_CHECK_ARG(n <= kMaxContrib, "msdeform_attn backward: Q*P*4 = %d contributions per (b,h,l) > %d", n, kMaxContrib);
  const size_t need = msda_ws_bytes(B, nh, L, Q, P);
  if (!ws || ws_bytes < need)
    return set_error(VA_ERR_WORKSPACE, "msdeform_attn backward: workspace %zu < %zu bytes", ws_bytes, need);
  const size_t nall = (size_t)B * nh * L * n;
  int* c_pix = static_cast<int*>(ws);
  float* c_w = reinterpret_cast<float*>(static_cast<char*>(ws) + align256(nall * sizeof(int)));
  const long long items = (long long)B * Q * nh;
  constexpr int VEC = Vec<TV>::N;
  auto pass1 = [&](auto kernel, int G) {
    const int per = kMsdaThreads / G;
    kernel<<<(unsigned)((items + per - 1) / per), kMsdaThreads, 0, st>>>(value, shapes, lstart, loc, attn, grad_out,
                                                                          grad_loc, grad_attn, c_pix, c_w, B, S, nh,
                                                                          L, Q, P);
  };
  if (dh == 16) pass1(msda_bwd_sample_kernel<TV, 16>, 16 / VEC);
  else pass1(msda_bwd_sample_kernel<TV, 32>, 32 / VEC);
  if (int rc = check_launch("msdeform_attn backward (samples)")) return rc;
  int npad = 1;
  while (npad < n) npad <<= 1;
  const size_t smem = (size_t)npad * sizeof(unsigned long long);
  auto pass2 = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kMaxContrib * 8));
    kernel<<<dim3(L, nh, B), 512, smem, st>>>(shapes, lstart, grad_out, c_pix, c_w, grad_value, S, nh, L, Q, P, npad);
  };
  if (dh == 16) pass2(msda_bwd_value_kernel<TV, 16>);
  else pass2(msda_bwd_value_kernel<TV, 32>);
  return check_launch("msdeform_attn backward (value)");
}

}  // namespace

}  // namespace va

using namespace va;
typedef __nv_bfloat16 bf16;

extern "C" {

int va_msdeform_attn_fwd_f32(const float* value, const int64_t* spatial_shapes, const int64_t* level_start,
                             const float* loc, const float* attn, float* out, int B, int S, int nh, int dh, int L,
                             int Q, int P, va_stream_t s) {
  return msda_fwd(value, spatial_shapes, level_start, loc, attn, out, B, S, nh, dh, L, Q, P, (cudaStream_t)s);
}

int va_msdeform_attn_fwd_bf16(const va_bf16* value, const int64_t* spatial_shapes, const int64_t* level_start,
                              const float* loc, const float* attn, va_bf16* out, int B, int S, int nh, int dh, int L,
                              int Q, int P, va_stream_t s) {
  return msda_fwd((const bf16*)value, spatial_shapes, level_start, loc, attn, (bf16*)out, B, S, nh, dh, L, Q, P,
                  (cudaStream_t)s);
}

size_t va_msdeform_attn_bwd_workspace_bytes(int B, int nh, int L, int Q, int P) {
  if (B <= 0 || nh <= 0 || L <= 0 || Q <= 0 || P <= 0) return 0;
  return msda_ws_bytes(B, nh, L, Q, P);
}

int va_msdeform_attn_bwd_f32(const float* value, const int64_t* spatial_shapes, const int64_t* level_start,
                             const float* loc, const float* attn, const float* grad_out, float* grad_value,
                             float* grad_loc, float* grad_attn, int B, int S, int nh, int dh, int L, int Q, int P,
                             void* ws, size_t ws_bytes, va_stream_t s) {
  return msda_bwd(value, spatial_shapes, level_start, loc, attn, grad_out, grad_value, grad_loc, grad_attn, B, S, nh,
                  dh, L, Q, P, ws, ws_bytes, (cudaStream_t)s);
}

int va_msdeform_attn_bwd_bf16(const va_bf16* value, const int64_t* spatial_shapes, const int64_t* level_start,
                              const float* loc, const float* attn, const va_bf16* grad_out, va_bf16* grad_value,
                              float* grad_loc, float* grad_attn, int B, int S, int nh, int dh, int L, int Q, int P,
                              void* ws, size_t ws_bytes, va_stream_t s) {
  return msda_bwd((const bf16*)value, spatial_shapes, level_start, loc, attn, (const bf16*)grad_out,
                  (bf16*)grad_value, grad_loc, grad_attn, B, S, nh, dh, L, Q, P, ws, ws_bytes, (cudaStream_t)s);
}

}  // extern "C"
