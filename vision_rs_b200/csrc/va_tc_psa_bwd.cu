// PSA attention backward on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the reference's psa_fa2_backward pair (psa.rs:650-725: one call
// per 32-wide V half, dQ/dK accumulated with atomic_add) by one kernel over
// the full 64-wide V, with no atomics.  Per (b, h) and scale s = 1/√32:
//   P = exp(s·Q·Kᵀ − lse),  dP = dO·Vᵀ,  Δ = rowsum(dO ⊙ O) (psa_delta_kernel),
//   dS = P ⊙ (dP − Δ),  dV = Pᵀ·dO,  dK = s·dSᵀ·Q,  dQ = s·dS·K.
//
// Work split: one CTA per (key tile j of 128 keys, b·h).  The CTA holds the Q
// tiles and dOᵀ tiles of the whole sequence (N ≤ 512) and its own K_j, V_jᵀ in
// shared memory, and walks the query tiles i:
//   issuer thread : S = Q_i·K_jᵀ and dP = dO_i·V_jᵀ into TMEM
//   8 compute warps: P and dS for 128 query rows × 128 keys (two warps per
//                    row, 64 keys each) → f16 tiles in shared memory
//   issuer thread : dV_j += Pᵀ·dO_i, dK_j += dSᵀ·Q_i, dQ_i = dS·K_j (TMEM)
// S and dP for tile i+1 are issued as soon as the compute warps hold tile i
// in registers.  The P and dS tiles are stored once, swizzled (SW128), and
// read by the MMAs both as M-major operands (Pᵀ, dSᵀ) and as K-major (dS).
// TMEM (512 columns): S 0-127, dP 128-255, dV 256-319, dK 320-351, dQ_i at
// 352 + 32i.  Outputs are channel-major f32: dK [b·h][32][N], dV
// [b·h][64][N], and dQ as per-key-tile partials [j][b·h][32][N] that the
// caller sums in j order (deterministic).
//
// Operands (f16): Q/K [2][B·nh][N][32] (the forward's packed layout), Vᵀ, Oᵀ
// and dOᵀ channel-major [B][nh·64][Np]; lse [B·nh][N] (natural log).
// dS is kept ×256 in f16 (its small entries stay out of the f16 subnormal
// range); dQ and dK take s/256.
#include <cudaTypedefs.h>

#include "va_common.cuh"
#include "va_psa.h"
#include "va_sm100.cuh"

namespace va {
using namespace sm100;

__device__ int g_bwd_status;

namespace {

constexpr int kT = 128, kKD = 32, kHD = 64, kMaxTiles = 4;
constexpr int kBwdThreads = 288;  // 8 compute warps + 1 TMA/MMA warp
constexpr float kDsScale = 256.0f;

struct BwdSmem {
  uint8_t q[kMaxTiles][kT * 64];       // Q tiles [128 q × 32] f16, SW64 (8 KB)
  uint8_t dO[kMaxTiles][2][64 * 128];  // dOᵀ tiles: 2 blocks [64 d × 64 q] f16, SW128 (16 KB)
  uint8_t k[kT * 64];                  // K_j [128 keys × 32], SW64
  uint8_t v[2][64 * 128];              // V_jᵀ: 2 blocks [64 d × 64 keys], SW128
  uint8_t p[2][kT * 128];              // P: 2 key blocks [128 q × 64 keys] f16, SW128 (32 KB)
  uint8_t ds[2][kT * 128];             // dS (×256)
  float delta[kMaxTiles][kT];          // Δ = rowsum(dO ⊙ O)
  float lse2[kMaxTiles][kT];           // lse·log2(e)
  uint64_t load_full, s_full, s_free, p_full, p_free, done;
  uint32_t tmem_base;
  int abort;
};

constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 320, kColDQ = 352;

__device__ __forceinline__ void named_sync_compute() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__global__ void __launch_bounds__(kBwdThreads, 1)
psa_attn_bwd_kernel(const __grid_constant__ CUtensorMap map_qk, const __grid_constant__ CUtensorMap map_v,
                    const __grid_constant__ CUtensorMap map_do, const float* __restrict__ delta,
                    const float* __restrict__ lse, float* __restrict__ dk_out, float* __restrict__ dv_out,
                    float* __restrict__ dq_part, int N, int Np, float scale) {
  extern __shared__ uint8_t smem_raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j = blockIdx.x, bh = blockIdx.y, BH = gridDim.y;
  const int nt = (N + kT - 1) / kT;
  const int vrow = bh * kHD;

  if (tid == 0) {
    mbar_init(&sm.load_full, 1);
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_free, 256);
    mbar_init(&sm.p_full, 256);
    mbar_init(&sm.p_free, 1);
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 8) {
    // ── TMA producer (lane 0) + MMA issuer: the whole warp runs the issue
    // loop converged (waits made warp-uniform), one elected lane issues ──
    if (lane == 0) {
      tma_prefetch_desc(&map_qk);
      tma_prefetch_desc(&map_v);
      tma_prefetch_desc(&map_do);
      mbar_arrive_expect_tx(&sm.load_full, (uint32_t)(nt * (kT * 64 + 2 * 64 * 128) + kT * 64 + 2 * 64 * 128));
      for (int i = 0; i < nt; ++i) {
        tma_load_3d(sm.q[i], &map_qk, &sm.load_full, 0, i * kT, bh);
        tma_load_2d(sm.dO[i][0], &map_do, &sm.load_full, i * kT, vrow);
        tma_load_2d(sm.dO[i][1], &map_do, &sm.load_full, i * kT + 64, vrow);
      }
      tma_load_3d(sm.k, &map_qk, &sm.load_full, 0, j * kT, BH + bh);
      tma_load_2d(sm.v[0], &map_v, &sm.load_full, j * kT, vrow);
      tma_load_2d(sm.v[1], &map_v, &sm.load_full, j * kT + 64, vrow);
    }
    __syncwarp();
    {
      constexpr uint32_t idS = idesc_f32acc(128, 128, AB_F16, false, false);
      constexpr uint32_t idP = idesc_f32acc(128, 128, AB_F16, true, true);
      constexpr uint32_t idV = idesc_f32acc(128, 64, AB_F16, true, false);
      constexpr uint32_t idK = idesc_f32acc(128, 32, AB_F16, true, true);
      constexpr uint32_t idQ = idesc_f32acc(128, 32, AB_F16, false, true);
      // K-major SW64 (32-wide rows of 64 B): 8-row groups 512 B apart, k step +32 B.
      // M/N-major SW64 (the same tiles seen as [k rows][32]): 8 k-rows per 512 B, k step 16 rows = +1024 B.
      // M/N-major SW128: 64-element blocks LBO apart, 8 k-rows per 1024 B, k step +2048 B.
      // K-major SW128: 8-row groups 1024 B apart, k step +32 B, 64-wide k blocks `blk` apart.
      const uint64_t dk_k = sdesc(smem_u32(sm.k), 16, 512, SW_64B);
      const uint64_t dk_mn = sdesc(smem_u32(sm.k), 8192, 512, SW_64B);
      const uint64_t dv_mn = sdesc(smem_u32(sm.v[0]), 8192, 1024, SW_128B);
      const uint64_t dp_mn = sdesc(smem_u32(sm.p[0]), 16384, 1024, SW_128B);
      const uint64_t dds_mn = sdesc(smem_u32(sm.ds[0]), 16384, 1024, SW_128B);
      const uint64_t dds_k = sdesc(smem_u32(sm.ds[0]), 16, 1024, SW_128B);
      auto dq_k = [&](int i) { return sdesc(smem_u32(sm.q[i]), 16, 512, SW_64B); };
      auto dq_mn = [&](int i) { return sdesc(smem_u32(sm.q[i]), 8192, 512, SW_64B); };
      auto ddo_mn = [&](int i) { return sdesc(smem_u32(sm.dO[i][0]), 8192, 1024, SW_128B); };
      auto ddo_k = [&](int i) { return sdesc(smem_u32(sm.dO[i][0]), 16, 1024, SW_128B); };
      auto issue_sdp = [&](int i) {
        const uint64_t a = dq_k(i), b = ddo_mn(i);
#pragma unroll
        for (int s = 0; s < kKD / 16; ++s) mma_ss_w(tmem + kColS, a + 2 * s, dk_k + 2 * s, idS, s > 0);
#pragma unroll
        for (int s = 0; s < kHD / 16; ++s) mma_ss_w(tmem + kColDP, b + 128 * s, dv_mn + 128 * s, idP, s > 0);
      };
      auto issue_grad = [&](int i) {
        const uint64_t bo = ddo_k(i), bq = dq_mn(i);
#pragma unroll
        for (int s = 0; s < kT / 16; ++s) {
          mma_ss_w(tmem + kColDV, dp_mn + 128 * s, bo + (s >> 2) * 512 + (s & 3) * 2, idV, (i > 0 || s > 0));
          mma_ss_w(tmem + kColDK, dds_mn + 128 * s, bq + 64 * s, idK, (i > 0 || s > 0));
          mma_ss_w(tmem + kColDQ + 32 * i, dds_k + (s >> 2) * 1024 + (s & 3) * 2, dk_mn + 64 * s, idQ, s > 0);
        }
      };
      bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.load_full, 0, &sm.abort, &g_bwd_status, 1));
      if (ok) {
        tc_fence_after();
        issue_sdp(0);
        mma_commit_w(&sm.s_full);
      }
      for (int i = 0; ok && i < nt; ++i) {
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_free, i & 1, &sm.abort, &g_bwd_status, 2)))) break;
        tc_fence_after();
        if (i + 1 < nt) {
          issue_sdp(i + 1);
          mma_commit_w(&sm.s_full);
        }
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&sm.p_full, i & 1, &sm.abort, &g_bwd_status, 3)))) break;
        tc_fence_after();
        issue_grad(i);
        mma_commit_w(&sm.p_free);
      }
      if (!ok) {  // the loads issued here land (bounded) before the CTA can exit
        const long long t0 = clock64();
        while (!mbar_try_wait(&sm.load_full, 0) && clock64() - t0 < kSpinCycles) {
        }
      }
      mma_commit_w(&sm.done);
    }
    __syncwarp();
  } else {
    // ── compute warps: row = query row (TMEM lane), hf = key half ──
    const int row = (warp & 3) * 32 + lane, hf = warp >> 2;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const float scale_log2 = scale * 1.4426950408889634f;
    // Δ (computed by psa_delta_kernel) and lse·log2(e) of every query row
    for (int i = hf; i < nt; i += 2) {
      const int q = i * kT + row;
      sm.delta[i][row] = q < N ? delta[(size_t)bh * N + q] : 0.f;
      sm.lse2[i][row] = q < N ? lse[(size_t)bh * N + q] * 1.4426950408889634f : 0.f;
    }
    named_sync_compute();
    const int kvalid = N - j * kT - hf * 64;  // valid keys among this half's 64
    bool ok = true;
    for (int i = 0; i < nt; ++i) {
      if (!(ok = mbar_wait(&sm.s_full, i & 1, &sm.abort, &g_bwd_status, 10))) break;
      tc_fence_after();
      float sv[64], dpv[64];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(tmem + lane_off + kColS + hf * 64, r0);
        tmem_ld32(tmem + lane_off + kColS + hf * 64 + 32, r1);
        tmem_ld_wait();
        reg_fence(r0);
        reg_fence(r1);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          sv[c] = __uint_as_float(r0[c]);
          sv[32 + c] = __uint_as_float(r1[c]);
        }
        tmem_ld32(tmem + lane_off + kColDP + hf * 64, r0);
        tmem_ld32(tmem + lane_off + kColDP + hf * 64 + 32, r1);
        tmem_ld_wait();
        reg_fence(r0);
        reg_fence(r1);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          dpv[c] = __uint_as_float(r0[c]);
          dpv[32 + c] = __uint_as_float(r1[c]);
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.s_free);
      const bool qv = i * kT + row < N;
      const float l2 = sm.lse2[i][row];
      const float dl = sm.delta[i][row];
      if (i > 0 && !(ok = mbar_wait(&sm.p_free, (i - 1) & 1, &sm.abort, &g_bwd_status, 11))) break;
      uint8_t* prow = sm.p[hf] + row * 128;
      uint8_t* drow = sm.ds[hf] + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = keys 8c..8c+7, stored at chunk c ^ (row & 7)
        uint32_t pp[4], dd[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k0 = 8 * c + 2 * e, k1 = k0 + 1;
          const float p0 = (qv && k0 < kvalid) ? ex2(fmaf(sv[k0], scale_log2, -l2)) : 0.f;
          const float p1 = (qv && k1 < kvalid) ? ex2(fmaf(sv[k1], scale_log2, -l2)) : 0.f;
          pp[e] = pack_f16x2(p0, p1);
          dd[e] = pack_f16x2(p0 * (dpv[k0] - dl) * kDsScale, p1 * (dpv[k1] - dl) * kDsScale);
        }
        const int off = ((c ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(prow + off) = make_uint4(pp[0], pp[1], pp[2], pp[3]);
        *reinterpret_cast<uint4*>(drow + off) = make_uint4(dd[0], dd[1], dd[2], dd[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&sm.p_full);
    }
    const bool fin = mbar_wait(&sm.done, 0, &sm.abort, &g_bwd_status, 12);
    tc_fence_after();
    if (ok && fin && !sm.abort) {
      const float sq = scale / kDsScale;
      const int key = j * kT + row;
      {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + kColDV + hf * 32, r);
        tmem_ld_wait();
        reg_fence(r);
        if (key < N) {  // channel-major: lanes store consecutive keys
          float* d = dv_out + ((size_t)bh * kHD + hf * 32) * N + key;
#pragma unroll
          for (int c = 0; c < 32; ++c) d[(size_t)c * N] = __uint_as_float(r[c]);
        }
      }
      {
        uint32_t r[16];
        tmem_ld16(tmem + lane_off + kColDK + hf * 16, r);
        tmem_ld_wait();
        reg_fence(r);
        if (key < N) {
          float* d = dk_out + ((size_t)bh * kKD + hf * 16) * N + key;
#pragma unroll
          for (int c = 0; c < 16; ++c) d[(size_t)c * N] = __uint_as_float(r[c]) * sq;
        }
      }
      for (int i = 0; i < nt; ++i) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_off + kColDQ + 32 * i + hf * 16, r);
        tmem_ld_wait();
        reg_fence(r);
        const int q = i * kT + row;
        if (q < N) {
          float* d = dq_part + (((size_t)j * BH + bh) * kKD + hf * 16) * N + q;
#pragma unroll
          for (int c = 0; c < 16; ++c) d[(size_t)c * N] = __uint_as_float(r[c]) * sq;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// Δ[b·h][n] = Σ_d dO[b][h·64+d][n] · O[b][h·64+d][n]  (f16 channel-major,
// pitch Np): one thread per token, coalesced across threads.
// Δ with 16-byte loads, N % 8 == 0: lane = 8·(token chunk) + (channel group);
// a thread sums its 8 channels for 8 consecutive tokens, and the 8 channel
// groups of a chunk combine with three shuffles (a fixed order).
__global__ void __launch_bounds__(256) psa_delta_vec_kernel(const __half* __restrict__ o,
                                                            const __half* __restrict__ d_o,
                                                            float* __restrict__ delta, int N, int Np) {
  const int cg = threadIdx.x & 7, n = 8 * (blockIdx.x * 32 + (threadIdx.x >> 3)), bh = blockIdx.y;
  const bool live = n < N;
  const size_t base = (size_t)bh * kHD * Np + (live ? n : 0) + (size_t)cg * 8 * Np;
  float acc[8] = {};
#pragma unroll
  for (int d = 0; d < 8; ++d) {
    const uint4 uo = live ? __ldg(reinterpret_cast<const uint4*>(o + base + (size_t)d * Np)) : make_uint4(0, 0, 0, 0);
    const uint4 ud = live ? __ldg(reinterpret_cast<const uint4*>(d_o + base + (size_t)d * Np)) : make_uint4(0, 0, 0, 0);
    const __half2* ho = reinterpret_cast<const __half2*>(&uo);
    const __half2* hd = reinterpret_cast<const __half2*>(&ud);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fo = __half22float2(ho[e]), fd = __half22float2(hd[e]);
      acc[2 * e] = fmaf(fd.x, fo.x, acc[2 * e]);
      acc[2 * e + 1] = fmaf(fd.y, fo.y, acc[2 * e + 1]);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], off);
  if (live && cg == 0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) delta[(size_t)bh * N + n + e] = acc[e];
  }
}

__global__ void psa_delta_kernel(const __half* __restrict__ o, const __half* __restrict__ d_o,
                                 float* __restrict__ delta, int N, int Np) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x, bh = blockIdx.y;
  if (n >= N) return;
  const size_t base = (size_t)bh * kHD * Np + n;
  float acc = 0.f;
#pragma unroll 16
  for (int d = 0; d < kHD; ++d) acc = fmaf(__half2float(d_o[base + (size_t)d * Np]), __half2float(o[base + (size_t)d * Np]), acc);
  delta[(size_t)bh * N + n] = acc;
}

PFN_cuTensorMapEncodeTiled_v12000 bwd_encode_fn() {
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

int bwd_map(CUtensorMap* m, int rank, const void* base, const uint64_t* d, const uint64_t* s, const uint32_t* box,
            CUtensorMapSwizzle swz, const char* what) {
  auto fn = bwd_encode_fn();
  if (!fn) return set_error(VA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  const uint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), d, s, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "tensor map for %s rejected (CUresult %d)", what, (int)r);
  return VA_OK;
}

}  // namespace

int psa_attn_bwd_tc(const void* qk, const void* v, const void* o, const void* d_o, const float* lse, float* delta,
                    float* dk, float* dv, float* dq_part, int B, int nh, int N, cudaStream_t st) {
  VA_CHECK_ARG(nh == 2 && B > 0 && N > 0, "psa attention backward: need nh=2");
  if (N > kMaxTiles * kT) return set_error(VA_ERR_UNSUPPORTED, "psa attention backward: N=%d > %d", N, kMaxTiles * kT);
  const int BH = B * nh, Np = (N + 7) / 8 * 8;
  VA_CHECK_ARG(BH <= 65535, "psa attention backward: too many heads");
  CUtensorMap mqk, mv, mdo;
  {
    const uint64_t d[3] = {(uint64_t)kKD, (uint64_t)N, (uint64_t)2 * BH}, s[2] = {kKD * 2, (uint64_t)N * kKD * 2};
    const uint32_t bx[3] = {kKD, kT, 1};
    if (int rc = bwd_map(&mqk, 3, qk, d, s, bx, CU_TENSOR_MAP_SWIZZLE_64B, "qk")) return rc;
  }
  {
    const uint64_t d[2] = {(uint64_t)N, (uint64_t)BH * kHD}, s[1] = {(uint64_t)Np * 2};
    const uint32_t bx[2] = {64, kHD};
    if (int rc = bwd_map(&mv, 2, v, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "v")) return rc;
    if (int rc = bwd_map(&mdo, 2, d_o, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "dO")) return rc;
  }
  const size_t smem = sizeof(BwdSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(psa_attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const int nt = (N + kT - 1) / kT;
  if (N % 8 == 0)  // Np == N: rows of 16-byte-aligned 8-token chunks
    psa_delta_vec_kernel<<<dim3((N / 8 + 31) / 32, BH), 256, 0, st>>>(static_cast<const __half*>(o),
                                                                      static_cast<const __half*>(d_o), delta, N, Np);
  else
    psa_delta_kernel<<<dim3((N + 127) / 128, BH), 128, 0, st>>>(static_cast<const __half*>(o),
                                                                 static_cast<const __half*>(d_o), delta, N, Np);
  if (int rc = check_launch("psa attention backward (delta)")) return rc;
  psa_attn_bwd_kernel<<<dim3(nt, BH), kBwdThreads, smem, st>>>(mqk, mv, mdo, delta, lse, dk, dv, dq_part, N, Np,
                                                              1.0f / sqrtf((float)kKD));
  return check_launch("psa attention backward");
}

int bwd_status_read(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_bwd_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status read: %s", cudaGetErrorString(e));
  return VA_OK;
}

int bwd_status_clear(cudaStream_t st) {
  static const int zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_bwd_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status clear: %s", cudaGetErrorString(e));
  return VA_OK;
}

}  // namespace va
