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
// owns VEC channels and reads every bilinear corner as one vector load
// (f32: 4 channels in 16 bytes, bf16: 4 channels in 8 bytes).  The block's locations and weights are staged
// in shared memory with coalesced loads first.  The op is a gather: its HBM
// floor is one pass over the value map.
//
// Backward, deterministic: pass 1 (same thread groups) recomputes each
// sample, writes grad_attn and grad_loc, and records the sample's grad_value
// contribution (anchor pixel, the four corner weights A·w) in a slot fixed by
// (b, h, l, q, p).  Pass 2 runs one CTA per (b, h, l): it owns that slice of
// grad_value exclusively, buckets the samples by anchor pixel in shared
// memory, and each thread sums one pixel's contributions in a fixed order —
// deterministic results, no atomics on grad_value.
#include <algorithm>

#include "va_common.cuh"
#include "va_psa.h"

namespace va {

namespace {

constexpr int kMsdaThreads = 256;
constexpr int kMaxLevels = 8;
constexpr int kMaxEntries = 65536;   // corner entries 4·Q·P per (b, h, l) bucketed in shared memory (< 2^16)

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
template <> struct Vec<__nv_bfloat16> {  // bf16 ↔ f32 by bit placement (exact widening, RN narrowing)
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const unsigned w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ static unsigned pack(float lo, float hi) {
    return (unsigned)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
           ((unsigned)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
  }
  __device__ static void store(__nv_bfloat16* p, const float (&v)[8]) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack(v[0], v[1]), pack(v[2], v[3]), pack(v[4], v[5]), pack(v[6], v[7]));
  }
};

// The forward gathers bf16 maps 4 channels (8 bytes) per thread: twice the
// threads of 16-byte loads over the same rows, which the gather's latency
// needs (with 8-channel loads the bf16 forward ran slower than the f32 one).
struct VecBf4 {
  static constexpr int N = 4;
  __device__ static void load(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    v[0] = __uint_as_float(u.x << 16);
    v[1] = __uint_as_float(u.x & 0xffff0000u);
    v[2] = __uint_as_float(u.y << 16);
    v[3] = __uint_as_float(u.y & 0xffff0000u);
  }
  __device__ static void store(__nv_bfloat16* p, const float (&v)[4]) {
    *reinterpret_cast<uint2*>(p) = make_uint2(Vec<__nv_bfloat16>::pack(v[0], v[1]), Vec<__nv_bfloat16>::pack(v[2], v[3]));
  }
};
template <typename TV> struct FwdVec { using type = Vec<TV>; };
template <> struct FwdVec<__nv_bfloat16> { using type = VecBf4; };

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

// PT > 0: the number of points per level is a compile-time constant; all
// PT·4 corner loads of a level are issued before any of them is used (more
// gathers in flight per thread).  PT = 0: any P, one point at a time.
template <typename TV, int DH, int PT>
__global__ void __launch_bounds__(kMsdaThreads)
msda_fwd_kernel(const TV* __restrict__ value, const int64_t* __restrict__ shapes, const int64_t* __restrict__ lstart,
                const float* __restrict__ loc, const float* __restrict__ attn, TV* __restrict__ out, int B, int S,
                int nh, int L, int Q, int P) {
  constexpr int VEC = FwdVec<TV>::type::N, G = DH / VEC, ITEMS = kMsdaThreads / G;
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
    if constexpr (PT > 0) {
      float v[PT][4][VEC], cw[PT][4];
#pragma unroll
      for (int p = 0; p < PT; ++p) {
        const int s = l * PT + p;
        const Corners c = corners(il[2 * s], il[2 * s + 1], H, W);
        const float a = ia[s];
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // out-of-map corners load row 0 and contribute exactly 0
          FwdVec<TV>::type::load(vbase + (size_t)c.pix[k] * nh * DH, v[p][k]);
          cw[p][k] = c.ok[k] ? a * c.w[k] : 0.f;
          if (!c.ok[k]) {
#pragma unroll
            for (int e = 0; e < VEC; ++e) v[p][k][e] = 0.f;
          }
        }
      }
#pragma unroll
      for (int p = 0; p < PT; ++p)
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[e] = fmaf(cw[p][k], v[p][k][e], acc[e]);
    } else {
      for (int p = 0; p < P; ++p) {
        const int s = l * P + p;
        const Corners c = corners(il[2 * s], il[2 * s + 1], H, W);
        const float a = ia[s];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (!c.ok[k]) continue;
          float vv[VEC];
          FwdVec<TV>::type::load(vbase + (size_t)c.pix[k] * nh * DH, vv);
          const float w = a * c.w[k];
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[e] = fmaf(w, vv[e], acc[e]);
        }
      }
    }
  }
  FwdVec<TV>::type::store(out + item * DH + part * VEC, acc);
}

// Pass 1 of the backward: grad_attn, grad_loc, and the grad_value
// contributions (pixel within the level, weight) in slot order.
template <typename TV, int DH>
__global__ void __launch_bounds__(kMsdaThreads)
msda_bwd_sample_kernel(const TV* __restrict__ value, const int64_t* __restrict__ shapes,
                       const int64_t* __restrict__ lstart, const float* __restrict__ loc,
                       const float* __restrict__ attn, const TV* __restrict__ grad_out, float* __restrict__ grad_loc,
                       float* __restrict__ grad_attn, int4* __restrict__ c_pix, float4* __restrict__ c_w, int B, int S,
                       int nh, int L, int Q, int P) {
  constexpr int VEC = FwdVec<TV>::type::N, G = DH / VEC, ITEMS = kMsdaThreads / G;
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
  FwdVec<TV>::type::load(grad_out + it * DH + part * VEC, g);
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
          FwdVec<TV>::type::load(vbase + (size_t)c.pix[k] * nh * DH, v);
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
        *reinterpret_cast<float2*>(grad_loc + (it * LP + s) * 2) = make_float2(a * gx * (float)W, a * gy * (float)H);
        // the sample's grad_value record at (b, h, l, q·P + p): corner pixels (−1
        // outside the map) and corner weights
        const size_t rec = (((size_t)b * nh + h) * L + l) * (size_t)Q * P + (size_t)q * P + p;
        c_pix[rec] = make_int4(c.ok[0] ? c.pix[0] : -1, c.ok[1] ? c.pix[1] : -1, c.ok[2] ? c.pix[2] : -1,
                               c.ok[3] ? c.pix[3] : -1);
        c_w[rec] = make_float4(a * c.w[0], a * c.w[1], a * c.w[2], a * c.w[3]);
      }
    }
  }
}

// Pass 2: CTA (l, h, b) owns grad_value[b, level l pixels, h, :].
// Its 4·Q·P corner entries (entry e = 4·sample + corner) are bucketed by
// pixel with a counting sort in shared memory.  Shared-memory atomics give
// the counts and a first placement inside each bucket; the final position of
// an entry is its bucket start plus the number of entries of its bucket with
// a smaller index, so each bucket ends up in entry order whatever order the
// atomics ran in.  A group of dh/8 lanes per pixel (8 channels each) sums the
// pixel's bucket in entry order and writes its grad_value row (zeros when no
// sample touched it): every sum is taken in a fixed order — deterministic,
// and no atomics on grad_value.
constexpr int kValueThreads = 512;
constexpr int kValueWarps = kValueThreads / 32;

__device__ __forceinline__ void store4(float* p, const float4& v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float4& v) {
  *reinterpret_cast<uint2*>(p) = make_uint2(Vec<__nv_bfloat16>::pack(v.x, v.y), Vec<__nv_bfloat16>::pack(v.z, v.w));
}

// Bucket counters: two 16-bit counters per word (pixel 2k in the low half,
// 2k + 1 in the high half); counts and positions stay below 2^16 because a
// bucket set holds fewer than 2^16 entries.
__device__ __forceinline__ int cnt_get(const unsigned* c, int p) { return (int)((c[p >> 1] >> ((p & 1) * 16)) & 0xffffu); }
__device__ __forceinline__ int cnt_bump(unsigned* c, int p) {
  const int sh = (p & 1) * 16;
  return (int)((atomicAdd(&c[p >> 1], 1u << sh) >> sh) & 0xffffu);
}

template <typename TV, int DH>
__global__ void __launch_bounds__(kValueThreads, 2)
msda_bwd_value_kernel(const int64_t* __restrict__ shapes, const int64_t* __restrict__ lstart,
                      const TV* __restrict__ grad_out, const int* __restrict__ c_pix,
                      const float* __restrict__ c_w, TV* __restrict__ grad_value, int S, int nh, int L, int Q, int P,
                      unsigned long long q_magic) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int wsum[kValueWarps];
  constexpr int GS = DH + 4;  // padded grad_out row: rows of nearby queries start in different banks
  const int l = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int H = (int)shapes[2 * l], W = (int)shapes[2 * l + 1], s0 = (int)lstart[l];
  const int HW = H * W, n = Q * P * 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* gos = reinterpret_cast<float*>(smem);                        // [Q][GS] grad_out rows of (b, h)
  unsigned short* tmp = reinterpret_cast<unsigned short*>(smem);      // [n] first placement, before gos
  const int rows_bytes = max(Q * GS * 4, (n * 2 + 15) & ~15);
  float* bw = reinterpret_cast<float*>(smem + rows_bytes);            // [n] weights in bucket order
  unsigned short* bq = reinterpret_cast<unsigned short*>(bw + n);     // [n] queries in bucket order
  unsigned* cnt = reinterpret_cast<unsigned*>(bq + n);                // [(HW + 2) / 2] packed counters
  const size_t rec0 = (((size_t)b * nh + h) * L + l) * (size_t)n;   // n % 4 == 0
  const int4* pix4 = reinterpret_cast<const int4*>(c_pix + rec0);
  const float4* w4p = reinterpret_cast<const float4*>(c_w + rec0);
  const int nwords = (HW + 2) / 2;
  for (int i = tid; i < nwords; i += kValueThreads) cnt[i] = 0u;
  __syncthreads();
  for (int i = tid; i < n / 4; i += kValueThreads) {
    const int4 p = __ldg(pix4 + i);
    if (p.x >= 0) cnt_bump(cnt, p.x);
    if (p.y >= 0) cnt_bump(cnt, p.y);
    if (p.z >= 0) cnt_bump(cnt, p.z);
    if (p.w >= 0) cnt_bump(cnt, p.w);
  }
  __syncthreads();
  {  // exclusive scan of the counts: thread t takes a contiguous run of whole words
    const int per = (nwords + kValueThreads - 1) / kValueThreads;
    const int lo = min(nwords, tid * per), hi = min(nwords, lo + per);
    int tot = 0;
    for (int i = lo; i < hi; ++i) {
      const unsigned c = cnt[i];
      tot += (int)(c & 0xffffu) + (int)(c >> 16);
    }
    int inc = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += u;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      const int own = lane < kValueWarps ? wsum[lane] : 0;
      int x = own;
#pragma unroll
      for (int o = 1; o < kValueWarps; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += u;
      }
      if (lane < kValueWarps) wsum[lane] = x - own;
    }
    __syncthreads();
    unsigned run = (unsigned)(wsum[warp] + inc - tot);
    for (int i = lo; i < hi; ++i) {
      const unsigned c = cnt[i];
      const unsigned a = run, bb = run + (c & 0xffffu);
      cnt[i] = a | (bb << 16);
      run = bb + (c >> 16);
    }
  }
  __syncthreads();
  for (int i = tid; i < n / 4; i += kValueThreads) {  // first placement
    const int4 p = __ldg(pix4 + i);
    if (p.x >= 0) tmp[cnt_bump(cnt, p.x)] = (unsigned short)(4 * i);
    if (p.y >= 0) tmp[cnt_bump(cnt, p.y)] = (unsigned short)(4 * i + 1);
    if (p.z >= 0) tmp[cnt_bump(cnt, p.z)] = (unsigned short)(4 * i + 2);
    if (p.w >= 0) tmp[cnt_bump(cnt, p.w)] = (unsigned short)(4 * i + 3);
  }
  __syncthreads();
  // counter k now holds the end of bucket k (= start of bucket k + 1).  Final
  // position = bucket start + number of smaller entry ids in the bucket.
  for (int i = tid; i < n / 4; i += kValueThreads) {
    const int4 p4 = __ldg(pix4 + i);
    const float4 w4 = __ldg(w4p + i);
    const int pc[4] = {p4.x, p4.y, p4.z, p4.w};
    const float wc[4] = {w4.x, w4.y, w4.z, w4.w};
    const unsigned short q = (unsigned short)((4u * i * q_magic) >> 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int p = pc[c];
      if (p < 0) continue;
      const unsigned id = 4u * i + c;
      const int lo = p ? cnt_get(cnt, p - 1) : 0, hi = cnt_get(cnt, p);
      int r = 0;
      for (int j = lo; j < hi; ++j) r += tmp[j] < id;
      bq[lo + r] = q;
      bw[lo + r] = wc[c];
    }
  }
  __syncthreads();
  constexpr int RV = DH / Vec<TV>::N;  // grad_out rows over the first-placement area
  for (int i = tid; i < Q * RV; i += kValueThreads) {
    const int q = i / RV, e0 = (i % RV) * Vec<TV>::N;
    float v[Vec<TV>::N];
    Vec<TV>::load(grad_out + (((size_t)b * Q + q) * nh + h) * DH + e0, v);
#pragma unroll
    for (int e = 0; e < Vec<TV>::N; ++e) gos[q * GS + e0 + e] = v[e];
  }
  __syncthreads();
  // G lanes per pixel, 8 channels each: a group reads whole grad_out rows
  constexpr int G = DH / 8, PPW = 32 / G;
  const int gl = lane % G, pg = lane / G;
  TV* gvb = grad_value + (((size_t)b * S + s0) * nh + h) * DH + 8 * gl;
  for (int z = warp * PPW + pg; z - pg < HW; z += kValueWarps * PPW) {
    if (z >= HW) continue;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    const int hi = cnt_get(cnt, z);
    for (int j = z ? cnt_get(cnt, z - 1) : 0; j < hi; ++j) {
      const float w = bw[j];
      const float* g = gos + (unsigned)bq[j] * GS + 8 * gl;
#pragma unroll
      for (int e = 0; e < 8; e += 4) {
        const float4 g4 = *reinterpret_cast<const float4*>(g + e);
        acc[e] = fmaf(w, g4.x, acc[e]);
        acc[e + 1] = fmaf(w, g4.y, acc[e + 1]);
        acc[e + 2] = fmaf(w, g4.z, acc[e + 2]);
        acc[e + 3] = fmaf(w, g4.w, acc[e + 3]);
      }
    }
    TV* d = gvb + (size_t)z * nh * DH;
    store4(d, make_float4(acc[0], acc[1], acc[2], acc[3]));
    store4(d + 4, make_float4(acc[4], acc[5], acc[6], acc[7]));
  }
}

// Dynamic shared memory of the value kernel: the level's pixel count is only
// known on the device, so the bucket table is sized for S rows (≥ H·W).
size_t msda_value_smem(int n, int Q, int dh, int S) {
  const size_t rows = std::max((size_t)Q * (dh + 4) * 4, ((size_t)n * 2 + 15) & ~(size_t)15);  // grad_out rows / first placement
  return rows + (size_t)n * 6 + (size_t)(S + 2) / 2 * 4;
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
  constexpr int VEC = FwdVec<TV>::type::N;
  if (P == 4) {
    if (dh == 16) launch(msda_fwd_kernel<TV, 16, 4>, 16 / VEC);
    else launch(msda_fwd_kernel<TV, 32, 4>, 32 / VEC);
  } else {
    if (dh == 16) launch(msda_fwd_kernel<TV, 16, 0>, 16 / VEC);
    else launch(msda_fwd_kernel<TV, 32, 0>, 32 / VEC);
  }
  return check_launch("msdeform_attn forward");
}

size_t msda_ws_bytes(int B, int nh, int L, int Q, int P) {
  const size_t n = (size_t)B * nh * L * Q * P;  // one record per sample: 4 corner pixels + 4 corner weights
  return align256(n * sizeof(int4)) + align256(n * sizeof(float4));
}

template <typename TV>
int msda_bwd(const TV* value, const int64_t* shapes, const int64_t* lstart, const float* loc, const float* attn,
             const TV* grad_out, TV* grad_value, float* grad_loc, float* grad_attn, int B, int S, int nh, int dh,
             int L, int Q, int P, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (int rc = check_msda(B, S, nh, dh, L, Q, P, value, grad_value)) return rc;
  const long long n_ll = 4LL * Q * P;
  VA_CHECK_ARG(n_ll < kMaxEntries, "msdeform_attn backward: 4*Q*P = %lld corner entries per (b,h,l) > %d", n_ll,
               kMaxEntries);
  const int n = (int)n_ll;
  const size_t need = msda_ws_bytes(B, nh, L, Q, P);
  if (!ws || ws_bytes < need)
    return set_error(VA_ERR_WORKSPACE, "msdeform_attn backward: workspace %zu < %zu bytes", ws_bytes, need);
  const size_t smem = msda_value_smem(n, Q, dh, S);
  VA_CHECK_ARG(smem <= 200 * 1024, "msdeform_attn backward: per-level working set %zu bytes exceeds shared memory",
               smem);
  const size_t nall = (size_t)B * nh * L * Q * P;  // sample records
  int4* c_pix = static_cast<int4*>(ws);
  float4* c_w = reinterpret_cast<float4*>(static_cast<char*>(ws) + align256(nall * sizeof(int4)));
  const long long items = (long long)B * Q * nh;
  constexpr int VEC = FwdVec<TV>::type::N;  // channels per thread in the sample pass, as in the forward
  auto pass1 = [&](auto kernel, int G) {
    const int per = kMsdaThreads / G;
    kernel<<<(unsigned)((items + per - 1) / per), kMsdaThreads, 0, st>>>(value, shapes, lstart, loc, attn, grad_out,
                                                                          grad_loc, grad_attn, c_pix, c_w, B, S, nh,
                                                                          L, Q, P);
  };
  if (dh == 16) pass1(msda_bwd_sample_kernel<TV, 16>, 16 / VEC);
  else pass1(msda_bwd_sample_kernel<TV, 32>, 32 / VEC);
  if (int rc = check_launch("msdeform_attn backward (samples)")) return rc;
  // query of entry e = e / (4P), as a multiply: q_magic = ceil(2^32 / 4P), exact for e, 4P < 2^16
  const unsigned long long q_magic = ((1ull << 32) + 4ull * P - 1) / (4ull * P);
  auto pass2 = [&](auto kernel) -> int {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    kernel<<<dim3(L, nh, B), kValueThreads, smem, st>>>(shapes, lstart, grad_out, reinterpret_cast<const int*>(c_pix),
                                                        reinterpret_cast<const float*>(c_w), grad_value, S, nh, L, Q,
                                                        P, q_magic);
    return check_launch("msdeform_attn backward (value)");
  };
  return dh == 16 ? pass2(msda_bwd_value_kernel<TV, 16>) : pass2(msda_bwd_value_kernel<TV, 32>);
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
