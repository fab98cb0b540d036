// Batched GEMM on tcgen05 for the training path (weight and input gradients
// of the 1×1 convolutions) and the 1×1 convolutions of the PSA forward at
// widths other than 128:
//
//   C[z][m][n] = act(α · Σ_k A_z(m, k) · B_z(n, k) + bias[m]) (+ R[z][m][n])
//                f16 or bf16 operands (both the same), f32 accumulate, act = SiLU
//                or none, R an optional residual (f32, bf16 or f16)
//
// Each operand is K-major (row m holds its K elements contiguously) or
// MN-major (row k holds its M — or N — elements contiguously), optionally
// shared by every batch entry.  One CTA computes a 128×128 tile: a producer
// thread streams 64-wide K blocks through a 3-stage TMA ring (out-of-range
// rows and columns read as zeros), one thread issues the MMAs into a TMEM
// accumulator, and the four warps store it (f32, bf16 or f16).  A CTA may
// fold `zfold` consecutive batch entries into its K loop (one accumulator),
// so a weight gradient summed over images comes out as ceil(Z/zfold)
// partials that the caller reduces in a fixed order — deterministic.
#include <cudaTypedefs.h>

#include <type_traits>

#include "va_common.cuh"
#include "va_psa.h"
#include "va_sm100.cuh"

namespace va {
using namespace sm100;

__device__ int g_gemm_status;

namespace {

// Three ring stages (96 KB of shared memory) let two CTAs share an SM, so one
// CTA's set-up, pipeline fill and epilogue overlap the other's MMAs.
constexpr int kGM = 128, kGN = 128, kGK = 64, kGStages = 3;

struct GemmSmem {
  uint8_t a[kGStages][kGM * 128];  // 16 KB per stage
  uint8_t b[kGStages][kGN * 128];
  uint64_t full[kGStages], empty[kGStages], done;
  uint32_t tmem_base;
  int abort;
};

constexpr int kOutF32 = 0, kOutBF16 = 1, kOutF16 = 2;

template <bool A_MN, bool B_MN, int OUT>
__global__ void __launch_bounds__(128, 2)
gemm_f16_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, void* __restrict__ c,
                int M, int N, int K, long long ldc, long long c_batch, int a_bcast, int b_bcast, float alpha, int Z,
                int zfold, uint32_t ab_fmt, const float* __restrict__ bias, int act, const void* __restrict__ res,
                int res_type, long long ldr, long long r_batch) {
  extern __shared__ uint8_t smem_raw[];
  GemmSmem& sm = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * kGM, n0 = blockIdx.y * kGN, z = blockIdx.z;
  const int zbeg = z * zfold, nz = min(zfold, Z - zbeg);
  const int nkz = (K + kGK - 1) / kGK, nk = nkz * nz;  // k blocks: batch entries zbeg.. in order

  if (tid == 0) {
    for (int i = 0; i < kGStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem_base, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    int issued = 0;
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int st = kb % kGStages;
      if (kb >= kGStages &&
          !(ok = mbar_wait(&sm.empty[st], ((kb / kGStages) - 1) & 1, &sm.abort, &g_gemm_status, 1)))
        break;
      mbar_arrive_expect_tx(&sm.full[st], kGM * 128 + kGN * 128);
      const int ze = zbeg + kb / nkz, kk = kb % nkz;
      const int za = a_bcast ? 0 : ze, zb = b_bcast ? 0 : ze;
      if (A_MN) {
        tma_load_3d(sm.a[st], &map_a, &sm.full[st], m0, kk * kGK, za);
        tma_load_3d(sm.a[st] + 8192, &map_a, &sm.full[st], m0 + 64, kk * kGK, za);
      } else {
        tma_load_3d(sm.a[st], &map_a, &sm.full[st], kk * kGK, m0, za);
      }
      if (B_MN) {
        tma_load_3d(sm.b[st], &map_b, &sm.full[st], n0, kk * kGK, zb);
        tma_load_3d(sm.b[st] + 8192, &map_b, &sm.full[st], n0 + 64, kk * kGK, zb);
      } else {
        tma_load_3d(sm.b[st], &map_b, &sm.full[st], kk * kGK, n0, zb);
      }
      ++issued;
    }
    if (!ok) {  // every load issued here lands (bounded) before the CTA can exit
      for (int kb = max(0, issued - kGStages); kb < issued; ++kb) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&sm.full[kb % kGStages], (kb / kGStages) & 1) && clock64() - t0 < kSpinCycles) {
        }
      }
    }
  } else if (warp == 1) {  // the whole warp, converged; one elected lane issues each tcgen05 instruction
    const uint32_t idesc = idesc_f32acc(kGM, kGN, ab_fmt, A_MN, B_MN);
    // K-major SW128: 8-row groups 1024 B apart, a 16-wide k step = +32 B.
    // MN-major SW128: two 64-element blocks 8 KB apart (LBO), 8 k-rows per
    // 1024 B (SBO), a 16-row k step = +2048 B.
    const uint64_t da0 = A_MN ? sdesc(smem_u32(sm.a[0]), 8192, 1024, SW_128B) : sdesc(smem_u32(sm.a[0]), 16, 1024, SW_128B);
    const uint64_t db0 = B_MN ? sdesc(smem_u32(sm.b[0]), 8192, 1024, SW_128B) : sdesc(smem_u32(sm.b[0]), 16, 1024, SW_128B);
    constexpr uint32_t kStage = (kGM * 128) >> 4;
    constexpr uint32_t kAStep = A_MN ? (2048 >> 4) : 2, kBStep = B_MN ? (2048 >> 4) : 2;
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int st = kb % kGStages;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&sm.full[st], (kb / kGStages) & 1, &sm.abort, &g_gemm_status, 2))))
        break;
      tc_fence_after();
      const uint64_t da = da0 + (uint64_t)(st * kStage), db = db0 + (uint64_t)(st * kStage);
#pragma unroll
      for (int s = 0; s < kGK / 16; ++s)
        mma_ss_w(tmem, da + s * kAStep, db + s * kBStep, idesc, (kb > 0 || s > 0) ? 1u : 0u);
      mma_commit_w(&sm.empty[st]);
    }
    mma_commit_w(&sm.done);
  }
  __syncwarp();
  const bool ok = mbar_wait(&sm.done, 0, &sm.abort, &g_gemm_status, 3) && !sm.abort;
  tc_fence_after();
  if (ok) {
    const int m = m0 + warp * 32 + lane;
#pragma unroll 1
    for (int ch = 0; ch < kGN / 32; ++ch) {
      uint32_t u[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + ch * 32, u);
      tmem_ld_wait();
      reg_fence(u);
      const float bm = (bias && m < M) ? bias[m] : 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(fmaf(__uint_as_float(u[i]), alpha, bm));
      const int nb = n0 + ch * 32;
      if (m >= M || nb >= N) continue;
      if (act) {  // SiLU: v·σ(v)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float v = __uint_as_float(u[i]);
          u[i] = __float_as_uint(__fdividef(v, 1.0f + __expf(-v)));  // SiLU; → −0 once exp overflows
        }
      }
      if (res) {  // + residual (f32, bf16 or f16 by res_type), columns < N
        const long long ro = z * r_batch + (long long)m * ldr + nb;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (nb + i >= N) continue;
          const float r = res_type == kOutF32 ? static_cast<const float*>(res)[ro + i]
                          : res_type == kOutBF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(res)[ro + i])
                                                 : __half2float(static_cast<const __half*>(res)[ro + i]);
          u[i] = __float_as_uint(__uint_as_float(u[i]) + r);
        }
      }
      if constexpr (OUT != kOutF32) {
        using T = typename std::conditional<OUT == kOutBF16, __nv_bfloat16, __half>::type;
        auto pk = [](float a, float b) { return OUT == kOutBF16 ? pack_bf16x2(a, b) : pack_f16x2(a, b); };
        T* row = static_cast<T*>(c) + z * c_batch + (long long)m * ldc + nb;
        if (nb + 32 <= N && ((reinterpret_cast<uintptr_t>(row) & 15) == 0)) {
          uint4* d = reinterpret_cast<uint4*>(row);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            d[q] = make_uint4(pk(__uint_as_float(u[8 * q]), __uint_as_float(u[8 * q + 1])),
                              pk(__uint_as_float(u[8 * q + 2]), __uint_as_float(u[8 * q + 3])),
                              pk(__uint_as_float(u[8 * q + 4]), __uint_as_float(u[8 * q + 5])),
                              pk(__uint_as_float(u[8 * q + 6]), __uint_as_float(u[8 * q + 7])));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (nb + i < N) {
              const uint32_t h = pk(__uint_as_float(u[i]), 0.f) & 0xffffu;
              reinterpret_cast<unsigned short*>(row)[i] = (unsigned short)h;
            }
        }
      } else {
        float* row = static_cast<float*>(c) + z * c_batch + (long long)m * ldc + nb;
        if (nb + 32 <= N && ((reinterpret_cast<uintptr_t>(row) & 15) == 0)) {
          float4* d = reinterpret_cast<float4*>(row);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            d[q] = make_float4(__uint_as_float(u[4 * q]), __uint_as_float(u[4 * q + 1]), __uint_as_float(u[4 * q + 2]),
                               __uint_as_float(u[4 * q + 3]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (nb + i < N) row[i] = __uint_as_float(u[i]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

PFN_cuTensorMapEncodeTiled_v12000 gemm_encode_fn() {
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

// 3D map over an operand: inner = contiguous extent, outer = rows, z = batch.
int operand_map(CUtensorMap* m, const GemmOperand& op, uint64_t inner, uint64_t outer, uint64_t zdim, uint32_t box_inner,
                uint32_t box_outer, bool bf16, const char* what) {
  auto fn = gemm_encode_fn();
  if (!fn) return set_error(VA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(op.ptr) & 15) || ((op.ld * 2) % 16) || (zdim > 1 && (op.batch_stride * 2) % 16))
    return set_error(VA_ERR_ALIGN, "gemm %s: base, row pitch and batch stride need 16-byte alignment", what);
  const uint64_t d[3] = {inner, outer, zdim};
  const uint64_t s[2] = {(uint64_t)op.ld * 2, (uint64_t)(zdim > 1 ? op.batch_stride : op.ld * outer) * 2};
  const uint32_t bx[3] = {box_inner, box_outer, 1}, es[3] = {1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(op.ptr), d, s, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "tensor map for gemm %s rejected (CUresult %d)", what, (int)r);
  return VA_OK;
}

}  // namespace

int tc_gemm_f16(const GemmOperand& a, const GemmOperand& b, void* c, int c_type, long long ldc, long long c_batch,
                int M, int N, int K, int Z, cudaStream_t st, float alpha, int zfold, const float* bias, bool ab_bf16,
                const GemmEpilogue& epi) {
  VA_CHECK_ARG(M > 0 && N > 0 && K > 0 && Z > 0 && Z <= 65535 && zfold > 0 && (N + kGN - 1) / kGN <= 65535,
               "gemm: bad sizes");
  VA_CHECK_ARG(c_type >= kOutF32 && c_type <= kOutF16, "gemm: output type %d", c_type);
  CUtensorMap ma, mb;
  const uint64_t za = a.broadcast ? 1 : Z, zb = b.broadcast ? 1 : Z;
  if (int rc = a.mn ? operand_map(&ma, a, M, K, za, 64, 64, ab_bf16, "A")
                    : operand_map(&ma, a, K, M, za, 64, kGM, ab_bf16, "A"))
    return rc;
  if (int rc = b.mn ? operand_map(&mb, b, N, K, zb, 64, 64, ab_bf16, "B")
                    : operand_map(&mb, b, K, N, zb, 64, kGN, ab_bf16, "B"))
    return rc;
  const size_t smem = sizeof(GemmSmem) + 1024;
  const dim3 grid((M + kGM - 1) / kGM, (N + kGN - 1) / kGN, (Z + zfold - 1) / zfold);
  auto launch = [&](auto kernel) -> int {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    kernel<<<grid, 128, smem, st>>>(ma, mb, c, M, N, K, ldc, c_batch, a.broadcast ? 1 : 0, b.broadcast ? 1 : 0,
                                    alpha, Z, zfold, ab_bf16 ? (uint32_t)AB_BF16 : (uint32_t)AB_F16, bias, epi.silu ? 1 : 0,
                                    epi.res, epi.res_type, epi.ldr, epi.r_batch);
    return check_launch("gemm");
  };
  auto pick = [&](auto amn, auto bmn) -> int {
    constexpr bool A = decltype(amn)::value, Bm = decltype(bmn)::value;
    if (c_type == kOutBF16) return launch(gemm_f16_kernel<A, Bm, kOutBF16>);
    if (c_type == kOutF16) return launch(gemm_f16_kernel<A, Bm, kOutF16>);
    return launch(gemm_f16_kernel<A, Bm, kOutF32>);
  };
  using T_ = std::true_type;
  using F_ = std::false_type;
  if (a.mn) return b.mn ? pick(T_{}, T_{}) : pick(T_{}, F_{});
  return b.mn ? pick(F_{}, T_{}) : pick(F_{}, F_{});
}

int gemm_status_read(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_gemm_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status read: %s", cudaGetErrorString(e));
  return VA_OK;
}

int gemm_status_clear(cudaStream_t st) {
  static const int zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_gemm_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status clear: %s", cudaGetErrorString(e));
  return VA_OK;
}

}  // namespace va
