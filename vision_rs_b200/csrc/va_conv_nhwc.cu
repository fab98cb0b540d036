// Convolution + folded BN (+ SiLU) as a tcgen05 implicit GEMM, NHWC bf16.
//
// The reference builds YOLO26 from `conv` (conv + BN + SiLU) and `conv_bn`
// (conv + BN) blocks (src/models/yolo/yolo26/blocks/conv.rs:31-69); its
// docs/optimisation.md:130 puts the convolutions at 84.8% of the model's GPU
// time.  This kernel computes, for kernel size k ∈ {1, 3}, stride s ∈ {1, 2}
// and padding k/2,
//   y[b][oy][ox][o] = act(bias[o] + Σ_{ky,kx,c} w[o][ky][kx][c] ·
//                                   x[b][s·oy + ky − k/2][s·ox + kx − k/2][c])
// with x, w, y bf16 (NHWC activations, OHWI weights), bias f32 (BN folded),
// act = SiLU or none, f32 accumulation in TMEM.
//
// GEMM view: D[pixels][o] = A[pixels][K] · B[o][K]ᵀ with K = (ky, kx, c).
// A CTA owns an output tile of 8 rows × 16 columns (128 pixels, the MMA's M)
// and BN output channels.  The im2col is done by TMA: for each K step (one
// tap (ky, kx) and KB input channels) a 4-D tiled load of x — box (KB
// channels, 16·s columns, 8·s rows, 1 image) with element strides (1, s, s, 1)
// starting at (c0, s·ox0 + kx − k/2, s·oy0 + ky − k/2, b) — lands the 128
// pixels' KB channels as 128 K-major rows; coordinates outside the image read
// as zeros, which is the padding.  The weight tile is a 2-D load of
// w viewed as [o][k·k·Cin].  A producer thread streams both through a 4-stage
// ring, one thread issues the MMAs (M = 128, N = BN, K = 16 per instruction),
// and the 4 warps drain the TMEM accumulator: + bias, SiLU, bf16, one pixel's
// BN channels per thread stored contiguously (NHWC).
//
// Channel counts.  Cin % 8 == 0 (the NHWC pixel stride must be a multiple of
// 16 bytes for TMA).  KB is 64, 32 or 16, the largest dividing Cin; when
// Cin % 16 == 8 the last channel block of each tap reads past Cin, and TMA
// fills those channels of x with zeros, so the weights the 2-D load picks up
// there (the next tap's first channels, or zeros past the end of the row)
// meet zero activations and add nothing.  Cout % 8 == 0: BN is 128, 64, 32 or
// 16 and weight rows past Cout load as zeros; the epilogue stores only
// channels below Cout.  x, w, y 16-byte aligned.  The YOLO26 stem (Cin = 3)
// takes its input padded to 8 channels with zero weights there.
#include <cudaTypedefs.h>

#include <type_traits>

#include "va_common.cuh"
#include "va_psa.h"
#include "va_sm100.cuh"

namespace va {
using namespace sm100;

__device__ int g_conv_status;

namespace {

constexpr int kCvM = 128, kCvTW = 16, kCvTH = 8, kCvStages = 4, kCvThreads = 128;

template <int KB, int BN>
struct ConvSmem {
  uint8_t a[kCvStages][kCvM * KB * 2];  // im2col tile: 128 pixel rows × KB channels, K-major, swizzled
  uint8_t b[kCvStages][BN * KB * 2];    // weight tile: BN rows × KB, K-major, swizzled
  uint64_t full[kCvStages], empty[kCvStages], done;
  uint32_t tmem_base;
  int abort;
};

template <int KB>
struct KbTraits;
template <> struct KbTraits<64> { static constexpr uint32_t swz = SW_128B; static constexpr uint32_t sbo = 1024; };
template <> struct KbTraits<32> { static constexpr uint32_t swz = SW_64B; static constexpr uint32_t sbo = 512; };
template <> struct KbTraits<16> { static constexpr uint32_t swz = SW_32B; static constexpr uint32_t sbo = 256; };

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

template <int KB, int BN>
__global__ void __launch_bounds__(kCvThreads, 1)
conv_nhwc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                 const float* __restrict__ bias, __nv_bfloat16* __restrict__ y, int Ho, int Wo, int Cin, int Cout,
                 int ksize, int stride, int act, int tiles_w) {
  extern __shared__ uint8_t smem_raw[];
  using Sm = ConvSmem<KB, BN>;
  Sm& sm = *reinterpret_cast<Sm*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kTmemCols = BN < 32 ? 32 : BN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ox0 = (blockIdx.x % tiles_w) * kCvTW, oy0 = (blockIdx.x / tiles_w) * kCvTH;
  const int n0 = blockIdx.y * BN, b = blockIdx.z;
  const int pad = ksize / 2, cblocks = (Cin + KB - 1) / KB, nk = ksize * ksize * cblocks;

  if (tid == 0) {
    for (int i = 0; i < kCvStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0 && lane == 0) {  // ── TMA producer ──
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_w);
    int issued = 0;
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int st = kb % kCvStages;
      if (kb >= kCvStages &&
          !(ok = mbar_wait(&sm.empty[st], ((kb / kCvStages) - 1) & 1, &sm.abort, &g_conv_status, 1)))
        break;
      const int tap = kb / cblocks, c0 = (kb - tap * cblocks) * KB, ky = tap / ksize, kx = tap - ky * ksize;
      mbar_arrive_expect_tx(&sm.full[st], (kCvM + BN) * KB * 2);
      tma_load_4d(sm.a[st], &map_x, &sm.full[st], c0, stride * ox0 + kx - pad, stride * oy0 + ky - pad, b);
      tma_load_2d(sm.b[st], &map_w, &sm.full[st], tap * Cin + c0, n0);
      ++issued;
    }
    if (!ok) {  // every load issued here lands (bounded) before the CTA can exit
      for (int kb = max(0, issued - kCvStages); kb < issued; ++kb) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&sm.full[kb % kCvStages], (kb / kCvStages) & 1) && clock64() - t0 < kSpinCycles) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {  // ── MMA issuer ──
    constexpr uint32_t idesc = idesc_f32acc(kCvM, BN, AB_BF16, false, false);
    const uint64_t da0 = sdesc(smem_u32(sm.a[0]), 16, KbTraits<KB>::sbo, KbTraits<KB>::swz);
    const uint64_t db0 = sdesc(smem_u32(sm.b[0]), 16, KbTraits<KB>::sbo, KbTraits<KB>::swz);
    constexpr uint32_t kAStage = (kCvM * KB * 2) >> 4, kBStage = (BN * KB * 2) >> 4;
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int st = kb % kCvStages;
      if (!(ok = mbar_wait(&sm.full[st], (kb / kCvStages) & 1, &sm.abort, &g_conv_status, 2))) break;
      tc_fence_after();
      const uint64_t da = da0 + (uint64_t)(st * kAStage), db = db0 + (uint64_t)(st * kBStage);
#pragma unroll
      for (int s = 0; s < KB / 16; ++s)  // +32 bytes per 16-channel k-step inside the swizzle atom
        mma_ss(tmem, da + 2 * s, db + 2 * s, idesc, (kb > 0 || s > 0) ? 1u : 0u);
      mma_commit(&sm.empty[st]);
    }
    mma_commit(&sm.done);
  }
  __syncwarp();
  // ── epilogue: thread = pixel row (TMEM lane) ──
  const bool ok = mbar_wait(&sm.done, 0, &sm.abort, &g_conv_status, 3) && !sm.abort;
  tc_fence_after();
  if (ok) {
    const int r = warp * 32 + lane, oy = oy0 + r / kCvTW, ox = ox0 + r % kCvTW;
    const bool live = oy < Ho && ox < Wo;
    __nv_bfloat16* dst = y + (((size_t)b * Ho + (live ? oy : 0)) * Wo + (live ? ox : 0)) * Cout + n0;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      uint32_t u[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c, u);
      tmem_ld_wait();
      reg_fence(u);
      const int nv = min(16, Cout - n0 - c);  // 16 or 8 (Cout % 8 == 0), ≤ 0 past Cout
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] = __uint_as_float(u[i]) + (i < nv ? bias[n0 + c + i] : 0.0f);
        if (act) v[i] = v[i] / (1.0f + __expf(-v[i]));
      }
      if (live && nv > 0) {
        uint4* d = reinterpret_cast<uint4*>(dst + c);
        d[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                          pack_bf16x2(v[6], v[7]));
        if (nv > 8)
          d[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                            pack_bf16x2(v[14], v[15]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// OIHW (the reference's conv weight layout) → OHWI, bf16.
__global__ void oihw_to_ohwi_kernel(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst, int Cout,
                                    int Cin, int kk) {
  const long long total = (long long)Cout * Cin * kk;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % Cin);
    const long long t = i / Cin;
    const int tap = (int)(t % kk), o = (int)(t / kk);
    dst[i] = src[((long long)o * Cin + c) * kk + tap];
  }
}

PFN_cuTensorMapEncodeTiled_v12000 conv_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

CUtensorMapSwizzle tma_swizzle(int kb) {
  return kb == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : kb == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
}

}  // namespace
}  // namespace va

namespace va {
namespace {

int conv_nhwc(const __nv_bfloat16* x, const __nv_bfloat16* w, const float* bias, __nv_bfloat16* y, int B, int H, int W,
              int Cin, int Cout, int k, int s, int act, cudaStream_t st) {
  VA_CHECK_ARG(x && w && bias && y, "conv nhwc: null pointer");
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && B <= 65535, "conv nhwc: bad sizes");
  VA_CHECK_ARG(k == 1 || k == 3, "conv nhwc: kernel size %d (1 or 3)", k);
  VA_CHECK_ARG(s == 1 || s == 2, "conv nhwc: stride %d (1 or 2)", s);
  VA_CHECK_ARG(Cin > 0 && Cin % 8 == 0, "conv nhwc: Cin=%d must be a multiple of 8", Cin);
  VA_CHECK_ARG(Cout > 0 && Cout % 8 == 0, "conv nhwc: Cout=%d must be a multiple of 8", Cout);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15)
    return set_error(VA_ERR_ALIGN, "conv nhwc: x, w, y need 16-byte alignment");
  const int pad = k / 2, Ho = (H + 2 * pad - k) / s + 1, Wo = (W + 2 * pad - k) / s + 1;
  const int KB = Cin % 64 == 0 ? 64 : Cin % 32 == 0 ? 32 : 16;
  const int BN = Cout % 128 == 0 ? 128 : Cout % 64 == 0 ? 64 : Cout % 32 == 0 ? 32 : 16;
  auto fn = conv_encode_fn();
  if (!fn) return set_error(VA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap mx, mw;
  {
    const uint64_t d[4] = {(uint64_t)Cin, (uint64_t)W, (uint64_t)H, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)Cin * 2, (uint64_t)W * Cin * 2, (uint64_t)H * W * Cin * 2};
    const uint32_t box[4] = {(uint32_t)KB, (uint32_t)(16 * s), (uint32_t)(8 * s), 1};
    const uint32_t es[4] = {1, (uint32_t)s, (uint32_t)s, 1};
    CUresult r = fn(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<__nv_bfloat16*>(x), d, str, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, tma_swizzle(KB), CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "conv nhwc: tensor map for x rejected (CUresult %d)", (int)r);
  }
  {
    const uint64_t d[2] = {(uint64_t)k * k * Cin, (uint64_t)Cout};
    const uint64_t str[1] = {(uint64_t)k * k * Cin * 2};
    const uint32_t box[2] = {(uint32_t)KB, (uint32_t)BN}, es[2] = {1, 1};
    CUresult r = fn(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(w), d, str, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, tma_swizzle(KB), CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "conv nhwc: tensor map for w rejected (CUresult %d)", (int)r);
  }
  const int tiles_w = (Wo + kCvTW - 1) / kCvTW, tiles_h = (Ho + kCvTH - 1) / kCvTH;
  const dim3 grid((unsigned)(tiles_w * tiles_h), (unsigned)((Cout + BN - 1) / BN), (unsigned)B);
  int rc = VA_ERR_UNSUPPORTED;
  auto launch = [&](auto kb, auto bn) {
    constexpr int KB_ = decltype(kb)::value, BN_ = decltype(bn)::value;
    auto kernel = conv_nhwc_kernel<KB_, BN_>;
    const size_t smem = sizeof(ConvSmem<KB_, BN_>) + 1024;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      rc = set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return;
    }
    kernel<<<grid, kCvThreads, smem, st>>>(mx, mw, bias, y, Ho, Wo, Cin, Cout, k, s, act, tiles_w);
    rc = check_launch("conv nhwc");
  };
  using std::integral_constant;
  auto by_bn = [&](auto kb) {
    switch (BN) {
      case 128: launch(kb, integral_constant<int, 128>{}); break;
      case 64: launch(kb, integral_constant<int, 64>{}); break;
      case 32: launch(kb, integral_constant<int, 32>{}); break;
      default: launch(kb, integral_constant<int, 16>{}); break;
    }
  };
  switch (KB) {
    case 64: by_bn(integral_constant<int, 64>{}); break;
    case 32: by_bn(integral_constant<int, 32>{}); break;
    default: by_bn(integral_constant<int, 16>{}); break;
  }
  return rc;
}

}  // namespace

int conv_status_read(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_conv_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status read: %s", cudaGetErrorString(e));
  return VA_OK;
}

int conv_status_clear(cudaStream_t st) {
  static const int zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_conv_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status clear: %s", cudaGetErrorString(e));
  return VA_OK;
}

}  // namespace va

using namespace va;

extern "C" {

int va_conv_nhwc_bf16(const va_bf16* x, const va_bf16* w_ohwi, const float* bias, va_bf16* y, int B, int H, int W,
                      int Cin, int Cout, int ksize, int stride, int act, va_stream_t stream) {
  clear_error();
  return conv_nhwc(reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(w_ohwi), bias,
                   reinterpret_cast<__nv_bfloat16*>(y), B, H, W, Cin, Cout, ksize, stride, act, (cudaStream_t)stream);
}

int va_conv_weight_ohwi_bf16(const va_bf16* w_oihw, va_bf16* w_ohwi, int Cout, int Cin, int ksize, va_stream_t stream) {
  clear_error();
  VA_CHECK_ARG(w_oihw && w_ohwi && Cout > 0 && Cin > 0 && (ksize == 1 || ksize == 3), "conv weight: bad arguments");
  const long long total = (long long)Cout * Cin * ksize * ksize;
  oihw_to_ohwi_kernel<<<(int)std::min<long long>((total + 255) / 256, 148LL * 8), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(w_oihw), reinterpret_cast<__nv_bfloat16*>(w_ohwi), Cout, Cin,
      ksize * ksize);
  return check_launch("conv weight ohwi");
}

}  // extern "C"
