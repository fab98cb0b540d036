// DINOv2 backbone attention on the sm_100a tensor cores: the packed QKV
// Linear (hidden → 3·hidden, tcgen05 GEMM fed by TMA) and softmax(Q·Kᵀ/8)·V
// over independent token sequences with head dim 64 (the flash-attention
// kernel shared with the PSA path, tc_flash_attention).
//
// The reference (spinorml/vision-rs) has no DINOv2 code; the operator is the
// published ViT/DINOv2 self-attention (Oquab et al. 2023, Dosovitskiy et al.
// 2021): qkv = x·W_qkvᵀ + b split as [3][heads][64] along the feature axis
// (q, k, v sections of `hidden` features each, head-major inside a section),
// O = softmax(q·kᵀ·64^-½)·v per head, heads concatenated.
//
// Global layers attend over a whole image (1 + H·W tokens, cls first).
// Windowed layers attend inside windows of win×win patches; the cls token
// joins every window as its first token (window sequences of 1 + win² tokens)
// and un-partitioning averages the windows' cls outputs.  BASELINE does not
// fix the cls handling of windowed layers; this is the choice made here.
//
// Kernels:
//  1. dino_qkv_kernel<EPI>  — persistent GEMM over work units of a 128-token
//     tile of one sequence × 192 features (three heads), x and W k blocks
//     streamed through a TMA ring across unit boundaries, two TMEM
//     accumulators so the epilogue overlaps the next unit's MMAs, bias
//     staged in shared memory per unit, output staged in shared memory and
//     written by TMA stores.  EPI kSplitHeads
//     writes Q and K f16 [2][S·heads][n][64] and V f16 transposed
//     [S·heads·64][n_pad] (the flash-attention operands); EPI kPackedRows
//     writes bf16 [S][n][3·hidden] (torch Linear layout).
//  2. window partition / un-partition (bf16 token gathers, 16-byte moves).
#include <cudaTypedefs.h>

#include <algorithm>

#include "va_common.cuh"
#include "va_psa.h"
#include "va_sm100.cuh"

namespace va {
using namespace sm100;

__device__ int g_dino_status;

namespace {

constexpr int kDM = 128;      // tokens per tile (UMMA M)
constexpr int kDN = 192;      // features per N tile (UMMA N): three heads of 64
constexpr int kWStages = 4;   // (x, W) k-block ring
constexpr int kHead = 64;
constexpr int kSplitHeads = 0, kPackedRows = 1;
constexpr int kQkvThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue

struct DinoQkvSmem {
  uint8_t x[kWStages][kDM * 128];     // x block: 128 tokens × 64 features, K-major SW128 (16 KB)
  uint8_t w[kWStages][kDN * 128];     // W block: 192 rows × 64 features (24 KB)
  uint8_t stage[3][kDM * 128];        // epilogue staging: three 16 KB head groups
  float bias[2][kDN];                 // the bias slice of the accumulator being drained
  uint64_t w_full[kWStages], w_empty[kWStages], acc_full[2], acc_empty[2], fin;
  uint64_t stage_free, stage_full;  // staging handshakes between the epilogue warps and the storing thread
  uint64_t bias_full[2];            // bias slot a written by all 128 epilogue threads
  uint32_t tmem_base;
  int abort;
};

// Work unit u = (N tile nt, token tile tt, sequence sq) with nt fastest, so
// the CTAs working at one time share few x tiles (read from L2 once per N
// tile) while W (≤ a few MB) stays L2-resident.
struct DinoUnit {
  int nt, t0, sq;
};
__device__ __forceinline__ DinoUnit dino_unit(int u, int ntiles, int ntt) {
  const int nt = u % ntiles, r = u / ntiles;
  return DinoUnit{nt, (r % ntt) * kDM, r / ntt};
}

// Persistent: CTA b walks the work units b, b + gridDim.x, …  The 64-wide k
// blocks of x and W stream through a 4-stage TMA ring across unit boundaries;
// two TMEM accumulators (192 columns each) let the epilogue of one unit
// overlap the MMAs of the next.  The epilogue adds the bias (staged in shared
// memory per unit), stages the 128 × 192 tile as three 16 KB head groups and
// writes them with TMA stores (rows past the sequence end are not written).
template <int EPI>
__global__ void __launch_bounds__(kQkvThreads, 1)
dino_qkv_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_o1, const __grid_constant__ CUtensorMap map_o2,
                const float* __restrict__ bias, int hidden, int heads, int BH, int ntt, int units) {
  extern __shared__ uint8_t smem_raw[];
  DinoQkvSmem& sm =
      *reinterpret_cast<DinoQkvSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = hidden / 64, ntiles = 3 * hidden / kDN;
  const int my_units = blockIdx.x < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (tid == 0) {
    for (int i = 0; i < kWStages; ++i) {
      mbar_init(&sm.w_full[i], 1);
      mbar_init(&sm.w_empty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], 128);
    }
    mbar_init(&sm.fin, 1);
    mbar_init(&sm.stage_free, 1);
    mbar_init(&sm.stage_full, 128);
    mbar_init(&sm.bias_full[0], 128);
    mbar_init(&sm.bias_full[1], 128);
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

  if (warp == 0) {
    if (lane == 0) {  // ── TMA producer ──
      tma_prefetch_desc(&map_x);
      tma_prefetch_desc(&map_w);
      const int total = my_units * nk;
      int issued = 0;
      bool ok = true;
      int st = 0, kb = 0, u = blockIdx.x;  // ring slot, k block and unit of stage g, kept incrementally
      uint32_t ph = 0;
      DinoUnit w = dino_unit(u, ntiles, ntt);
      for (int g = 0; g < total; ++g) {
        if (g >= kWStages && !(ok = mbar_wait(&sm.w_empty[st], ph ^ 1u, &sm.abort, &g_dino_status, 1))) break;
        mbar_arrive_expect_tx(&sm.w_full[st], kDM * 128 + kDN * 128);
        tma_load_3d(sm.x[st], &map_x, &sm.w_full[st], kb * 64, w.t0, w.sq);
        tma_load_2d(sm.w[st], &map_w, &sm.w_full[st], kb * 64, w.nt * kDN);
        ++issued;
        st = st + 1 == kWStages ? 0 : st + 1;
        ph ^= st == 0 ? 1u : 0u;
        if (++kb == nk) {
          kb = 0;
          u += gridDim.x;
          w = dino_unit(u, ntiles, ntt);
        }
      }
      if (!ok) {  // loads issued here land (bounded) before the CTA can exit
        for (int g = max(0, issued - kWStages); g < issued; ++g) {
          const long long c0 = clock64();
          while (!mbar_try_wait(&sm.w_full[g % kWStages], (g / kWStages) & 1) && clock64() - c0 < kSpinCycles) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ── MMA issuer: the whole warp runs the loop converged (waits made
    // warp-uniform) and one elected lane issues each tcgen05 instruction ──
    constexpr uint32_t idesc = idesc_f32acc(kDM, kDN, AB_BF16, false, false);
    const uint64_t dx0 = sdesc(smem_u32(sm.x[0]), 16, 1024, SW_128B);
    const uint64_t dw0 = sdesc(smem_u32(sm.w[0]), 16, 1024, SW_128B);
    constexpr uint32_t kXS = (kDM * 128) >> 4, kWS = (kDN * 128) >> 4;
    bool ok = true;
    int st = 0;       // ring slot of the next stage
    uint32_t ph = 0;  // its fill parity
    for (int t = 0; ok && t < my_units; ++t) {
      const int a = t & 1;
      if (t >= 2 &&
          !(ok = __all_sync(0xffffffffu,
                            mbar_wait(&sm.acc_empty[a], ((t >> 1) - 1) & 1, &sm.abort, &g_dino_status, 3))))
        break;
      tc_fence_after();
      for (int kb = 0; kb < nk; ++kb) {
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&sm.w_full[st], ph, &sm.abort, &g_dino_status, 4)))) break;
        tc_fence_after();
        const uint64_t da = dx0 + (uint64_t)(st * kXS), db = dw0 + (uint64_t)(st * kWS);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          mma_ss_w(tmem + a * 256, da + 2 * s, db + 2 * s, idesc, (kb > 0 || s > 0) ? 1u : 0u);
        mma_commit_w(&sm.w_empty[st]);
        st = st + 1 == kWStages ? 0 : st + 1;
        ph ^= st == 0 ? 1u : 0u;
      }
      if (ok) mma_commit_w(&sm.acc_full[a]);
    }
    mma_commit_w(&sm.fin);  // every MMA issued here completes before the CTA tears down
    const long long c0 = clock64();
    while (!mbar_try_wait(&sm.fin, 0) && clock64() - c0 < kSpinCycles) {
    }
    __syncwarp();
  } else {
    // ── epilogue warps 2-5: TMEM lane quarter = warp % 4 ──
    const int row = (warp & 3) * 32 + lane, et = tid - 64;  // et: 0..127
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const bool storer = (warp == 2 && lane == 0);
    bool ok = true;
    for (int t = 0; t < my_units; ++t) {
      const int a = t & 1;
      const DinoUnit w = dino_unit(blockIdx.x + t * gridDim.x, ntiles, ntt);
      const int n0 = w.nt * kDN;
      // this unit's bias slice (slot a: the previous unit's epilogue reads slot a ^ 1)
      sm.bias[a][et] = __ldg(bias + n0 + et);
      if (et < kDN - 128) sm.bias[a][128 + et] = __ldg(bias + n0 + 128 + et);
      mbar_arrive(&sm.bias_full[a]);  // release: the slot's values are visible to the waiters
      if (!(ok = mbar_wait(&sm.bias_full[a], (t >> 1) & 1, &sm.abort, &g_dino_status, 8))) break;
      if (!(ok = mbar_wait(&sm.acc_full[a], (t >> 1) & 1, &sm.abort, &g_dino_status, 5))) break;
      tc_fence_after();
      if (storer) {  // the previous unit's stores have read the staging buffer
        tma_store_wait_read();
        mbar_arrive(&sm.stage_free);
      }
      if (!(ok = mbar_wait(&sm.stage_free, t & 1, &sm.abort, &g_dino_status, 6))) break;
      const float* bs = sm.bias[a];
#pragma unroll 2
      for (int c = 0; c < kDN / 32; ++c) {
        uint32_t u[32];
        tmem_ld32(tmem + lane_off + a * 256 + c * 32, u);
        tmem_ld_wait();
        reg_fence(u);
        const int g = c >> 1, half = c & 1;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(u[i]) + bs[c * 32 + i];
        uint8_t* tile = sm.stage[g];
        const bool vsec = EPI == kSplitHeads && (n0 + g * kHead) / hidden == 2;
        if (vsec) {
          __half* tv = reinterpret_cast<__half*>(tile);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            tv[(half * 32 + i) * kDM + row] = __ushort_as_half((unsigned short)(pack_f16x2_sat(v[i], 0.f) & 0xffffu));
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w4;
            if constexpr (EPI == kPackedRows)
              w4 = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                              pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
            else
              w4 = make_uint4(pack_f16x2_sat(v[8 * q], v[8 * q + 1]), pack_f16x2_sat(v[8 * q + 2], v[8 * q + 3]),
                              pack_f16x2_sat(v[8 * q + 4], v[8 * q + 5]), pack_f16x2_sat(v[8 * q + 6], v[8 * q + 7]));
            *reinterpret_cast<uint4*>(tile + sw128_off(row, half * 4 + q)) = w4;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[a]);
      fence_proxy_async_smem();
      mbar_arrive(&sm.stage_full);
      if (storer) {
        if (!(ok = mbar_wait(&sm.stage_full, t & 1, &sm.abort, &g_dino_status, 7))) break;
#pragma unroll 1
        for (int g = 0; g < kDN / kHead; ++g) {
          const int gcol = n0 + g * kHead;
          if constexpr (EPI == kPackedRows) {
            tma_store_3d(&map_o1, sm.stage[g], gcol, w.t0, w.sq);
          } else {
            const int sec = gcol / hidden, hd = (gcol - sec * hidden) / kHead, bh = w.sq * heads + hd;
            if (sec < 2) tma_store_3d(&map_o1, sm.stage[g], 0, w.t0, sec * BH + bh);
            else tma_store_3d(&map_o2, sm.stage[g], w.t0, bh * kHead, 0);
          }
        }
        tma_store_commit();
      }
    }
    if (storer) tma_store_wait_read();
    (void)ok;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ── window partition / un-partition ─────────────────────────────────────────
// x [B][1 + gh·gw][C] (cls first, patches row-major) ↔ xw [B·nw][1 + win²][C]
// (window w = wy·(gw/win) + wx; cls copied to token 0 of every window).
// One thread per 16-byte chunk (32-bit index arithmetic: the element counts
// are checked < 2^31 by the launchers; 64-bit divisions made these copies
// instruction-bound).
__global__ void window_partition_kernel(const uint4* __restrict__ x, uint4* __restrict__ xw, int B, int gh, int gw,
                                        int win, int cv) {
  const unsigned nwx = gw / win, nw = (gh / win) * nwx, tw = 1 + win * win;
  const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (unsigned)B * nw * tw * cv) return;
  const unsigned row = i / cv, c = i - row * cv;
  const unsigned bw = row / tw, tok = row - bw * tw;
  const unsigned b = bw / nw, w = bw - b * nw;
  unsigned src = 0;
  if (tok > 0) {
    const unsigned iy = (tok - 1) / win, ix = (tok - 1) - iy * win;
    const unsigned wy = w / nwx, wx = w - wy * nwx;
    src = 1 + (wy * win + iy) * gw + wx * win + ix;
  }
  xw[i] = x[((size_t)b * (1 + gh * gw) + src) * cv + c];
}

__global__ void window_unpartition_kernel(const __nv_bfloat16* __restrict__ xw, __nv_bfloat16* __restrict__ x, int B,
                                          int gh, int gw, int win, int C) {
  const int nwx = gw / win, nw = (gh / win) * nwx, tw = 1 + win * win, ntok = 1 + gh * gw;
  const unsigned cv = C / 8, i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < (unsigned)B * ntok * cv) {
    const unsigned row = i / cv, c8 = i - row * cv;
    const unsigned b = row / ntok, tok = row - b * ntok;
    uint4 out;
    if (tok == 0) {  // cls: mean of the windows' cls outputs, summed in window order
      float acc[8] = {};
      for (int w = 0; w < nw; ++w) {
        const uint4 u = *reinterpret_cast<const uint4*>(xw + (((size_t)b * nw + w) * tw) * C + c8 * 8);
        const unsigned ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          acc[2 * k] += __uint_as_float(ws[k] << 16);
          acc[2 * k + 1] += __uint_as_float(ws[k] & 0xffff0000u);
        }
      }
      const float inv = 1.0f / (float)nw;
      out = make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                       pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
    } else {
      const int py = (tok - 1) / gw, px = (tok - 1) - py * gw;
      const int w = (py / win) * nwx + px / win, it = 1 + (py % win) * win + px % win;
      out = *reinterpret_cast<const uint4*>(xw + (((size_t)b * nw + w) * tw + it) * C + c8 * 8);
    }
    *reinterpret_cast<uint4*>(x + ((size_t)b * ntok + tok) * C + c8 * 8) = out;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 dino_encode_fn() {
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

int dino_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows, const char* what) {
  auto fn = dino_encode_fn();
  if (!fn) return set_error(VA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  const uint64_t d[2] = {inner, rows}, s[1] = {inner * 2};
  const uint32_t bx[2] = {64, box_rows}, es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), d, s, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "tensor map for %s rejected (CUresult %d)", what, (int)r);
  return VA_OK;
}

int check_dino(int S, int n, int hidden, const void* x, const void* w) {
  VA_CHECK_ARG(S > 0 && n > 0 && hidden > 0 && hidden % kHead == 0 && (3 * hidden) % kDN == 0,
               "dinov2 qkv: hidden %d must be a positive multiple of 64", hidden);
  VA_CHECK_ARG(S <= 65535 && 3 * hidden / kDN <= 65535, "dinov2 qkv: too many sequences");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return set_error(VA_ERR_ALIGN, "dinov2 qkv: x and w_qkv need 16-byte alignment");
  return VA_OK;
}

int map3(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
         uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swz, const char* what) {
  auto fn = dino_encode_fn();
  if (!fn) return set_error(VA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  const uint64_t d[3] = {d0, d1, d2}, s[2] = {s1, s2};
  const uint32_t bx[3] = {b0, b1, 1}, es[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void*>(base), d, s, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "tensor map for %s rejected (CUresult %d)", what, (int)r);
  return VA_OK;
}

// x [S][n][hidden] bf16; EPI kSplitHeads: qk f16 [2][S·heads][n][64], vbuf f16
// [S·heads·64][n_pad]; EPI kPackedRows: out0 bf16 [S][n][3·hidden].
template <int EPI>
int launch_qkv(const __nv_bfloat16* x, const __nv_bfloat16* w, const float* bias, void* out0, __half* vbuf, int S,
               int n, int hidden, int heads, cudaStream_t st) {
  const int BH = S * heads, n_pad = (n + 7) / 8 * 8;
  CUtensorMap mx, mw, mo1, mo2;
  if (int rc = map3(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, hidden, n, S, (uint64_t)hidden * 2,
                    (uint64_t)n * hidden * 2, 64, kDM, CU_TENSOR_MAP_SWIZZLE_128B, "x"))
    return rc;
  if (int rc = dino_map(&mw, w, (uint64_t)hidden, (uint64_t)3 * hidden, kDN, "w_qkv")) return rc;
  if (EPI == kPackedRows) {
    if (int rc = map3(&mo1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, out0, 3 * hidden, n, S, (uint64_t)3 * hidden * 2,
                      (uint64_t)n * 3 * hidden * 2, kHead, kDM, CU_TENSOR_MAP_SWIZZLE_128B, "qkv out"))
      return rc;
    mo2 = mo1;
  } else {
    if (int rc = map3(&mo1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, out0, kHead, n, 2 * (uint64_t)BH, kHead * 2,
                      (uint64_t)n * kHead * 2, kHead, kDM, CU_TENSOR_MAP_SWIZZLE_128B, "qk out"))
      return rc;
    if (int rc = map3(&mo2, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, vbuf, n, (uint64_t)BH * kHead, 1, (uint64_t)n_pad * 2,
                      (uint64_t)n_pad * 2 * BH * kHead, kDM, kHead, CU_TENSOR_MAP_SWIZZLE_NONE, "v out"))
      return rc;
  }
  const size_t smem = sizeof(DinoQkvSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(dino_qkv_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  const int ntt = (n + kDM - 1) / kDM;
  const long long units = (long long)ntt * S * (3 * hidden / kDN);
  VA_CHECK_ARG(units < (1LL << 31), "dinov2 qkv: too many tiles");
  dino_qkv_kernel<EPI><<<(unsigned)std::min<long long>(units, 148), kQkvThreads, smem, st>>>(
      mx, mw, mo1, mo2, bias, hidden, heads, BH, ntt, (int)units);
  return check_launch("dinov2 qkv");
}

struct DinoWs {
  size_t qk, v, total;
};

DinoWs dino_layout(int S, int n, int hidden) {
  const size_t heads = (size_t)hidden / kHead, BH = (size_t)S * heads, np = ((size_t)n + 7) / 8 * 8;
  DinoWs w;
  w.qk = 0;
  w.v = align256(2 * BH * n * kHead * 2);
  w.total = w.v + align256(BH * kHead * np * 2);
  return w;
}

}  // namespace

size_t dino_workspace_bytes(int S, int n, int hidden) {
  if (S <= 0 || n <= 0 || hidden <= 0 || hidden % kHead) return 0;
  return dino_layout(S, n, hidden).total;
}

int dino_qkv_linear(const __nv_bfloat16* x, const __nv_bfloat16* w, const float* b, __nv_bfloat16* qkv, int tokens,
                    int hidden, cudaStream_t st) {
  // the packed Linear sees the tokens as one sequence (rows are independent)
  if (int rc = check_dino(1, tokens, hidden, x, w)) return rc;
  if (reinterpret_cast<uintptr_t>(qkv) & 15) return set_error(VA_ERR_ALIGN, "dinov2 qkv: output needs 16-byte alignment");
  return launch_qkv<kPackedRows>(x, w, b, qkv, nullptr, 1, tokens, hidden, hidden / kHead, st);
}

int dino_attention_fwd(const __nv_bfloat16* x, const __nv_bfloat16* w, const float* b, __nv_bfloat16* o, int S, int n,
                       int hidden, int heads, void* ws, size_t ws_bytes, cudaStream_t st) {
  VA_CHECK_ARG(S > 0 && n > 0 && heads > 0 && heads * kHead == hidden, "dinov2 attention: need heads·64 == hidden");
  VA_CHECK_ARG((long long)S * heads <= 65535, "dinov2 attention: %d sequences × %d heads too many", S, heads);
  if (int rc = check_dino(S, n, hidden, x, w)) return rc;
  if (reinterpret_cast<uintptr_t>(o) & 15) return set_error(VA_ERR_ALIGN, "dinov2 attention: o needs 16-byte alignment");
  const DinoWs L = dino_layout(S, n, hidden);
  if (!ws || ws_bytes < L.total)
    return set_error(VA_ERR_WORKSPACE, "dinov2 attention: workspace %zu < %zu bytes", ws_bytes, L.total);
  if (reinterpret_cast<uintptr_t>(ws) & 255)
    return set_error(VA_ERR_ALIGN, "dinov2 attention: workspace needs 256-byte alignment");
  char* base = static_cast<char*>(ws);
  __half* qk = reinterpret_cast<__half*>(base + L.qk);
  __half* vb = reinterpret_cast<__half*>(base + L.v);
  if (int rc = launch_qkv<kSplitHeads>(x, w, b, qk, vb, S, n, hidden, heads, st)) return rc;
  return tc_flash_attention(qk, vb, o, nullptr, S * heads, heads, n, kHead, 1, st);
}

int dino_window_partition(const __nv_bfloat16* x, __nv_bfloat16* xw, int B, int gh, int gw, int win, int C,
                          cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && gh > 0 && gw > 0 && win > 0 && gh % win == 0 && gw % win == 0 && C > 0 && C % 8 == 0,
               "dinov2 window partition: grid %dx%d not divisible by window %d, or C %% 8", gh, gw, win);
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(xw) & 15))
    return set_error(VA_ERR_ALIGN, "dinov2 window partition: 16-byte alignment needed");
  const long long total = (long long)B * (gh / win) * (gw / win) * (1 + win * win) * (C / 8);
  VA_CHECK_ARG(total < (1LL << 31), "dinov2 window partition: too many elements");
  window_partition_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const uint4*>(x), reinterpret_cast<uint4*>(xw), B, gh, gw, win, C / 8);
  return check_launch("dinov2 window partition");
}

int dino_window_unpartition(const __nv_bfloat16* xw, __nv_bfloat16* x, int B, int gh, int gw, int win, int C,
                            cudaStream_t st) {
  VA_CHECK_ARG(B > 0 && gh > 0 && gw > 0 && win > 0 && gh % win == 0 && gw % win == 0 && C > 0 && C % 8 == 0,
               "dinov2 window unpartition: grid %dx%d not divisible by window %d, or C %% 8", gh, gw, win);
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(xw) & 15))
    return set_error(VA_ERR_ALIGN, "dinov2 window unpartition: 16-byte alignment needed");
  const long long total = (long long)B * (1 + gh * gw) * (C / 8);
  VA_CHECK_ARG(total < (1LL << 31), "dinov2 window unpartition: too many elements");
  window_unpartition_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(xw, x, B, gh, gw, win, C);
  return check_launch("dinov2 window unpartition");
}

int dino_status_read(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_dino_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status read: %s", cudaGetErrorString(e));
  return VA_OK;
}

int dino_status_clear(cudaStream_t st) {
  static const int zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_dino_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status clear: %s", cudaGetErrorString(e));
  return VA_OK;
}

}  // namespace va

using namespace va;

extern "C" {

size_t va_dinov2_attention_workspace_bytes(int num_seqs, int seq_len, int hidden) {
  return dino_workspace_bytes(num_seqs, seq_len, hidden);
}

int va_dinov2_attention_fwd_bf16(const va_bf16* x, const va_bf16* w_qkv, const float* b_qkv, va_bf16* o,
                                 int num_seqs, int seq_len, int hidden, int num_heads, void* workspace,
                                 size_t ws_bytes, va_stream_t stream) {
  return dino_attention_fwd((const __nv_bfloat16*)x, (const __nv_bfloat16*)w_qkv, b_qkv, (__nv_bfloat16*)o, num_seqs,
                            seq_len, hidden, num_heads, workspace, ws_bytes, (cudaStream_t)stream);
}

int va_dinov2_flash_attention_fwd_f16(const void* qk, const void* v, va_bf16* o, int num_seqs, int seq_len,
                                      int num_heads, va_stream_t stream) {
  return tc_flash_attention(qk, v, o, nullptr, num_seqs * num_heads, num_heads, seq_len, kHead, 1,
                            (cudaStream_t)stream);
}

int va_dinov2_qkv_linear_bf16(const va_bf16* x, const va_bf16* w_qkv, const float* b_qkv, va_bf16* qkv, int tokens,
                              int hidden, va_stream_t stream) {
  return dino_qkv_linear((const __nv_bfloat16*)x, (const __nv_bfloat16*)w_qkv, b_qkv, (__nv_bfloat16*)qkv, tokens,
                         hidden, (cudaStream_t)stream);
}

int va_dinov2_window_partition_bf16(const va_bf16* x, va_bf16* xw, int B, int grid_h, int grid_w, int win,
                                    int hidden, va_stream_t stream) {
  return dino_window_partition((const __nv_bfloat16*)x, (__nv_bfloat16*)xw, B, grid_h, grid_w, win, hidden,
                               (cudaStream_t)stream);
}

int va_dinov2_window_unpartition_bf16(const va_bf16* xw, va_bf16* x, int B, int grid_h, int grid_w, int win,
                                      int hidden, va_stream_t stream) {
  return dino_window_unpartition((const __nv_bfloat16*)xw, (__nv_bfloat16*)x, B, grid_h, grid_w, win, hidden,
                                 (cudaStream_t)stream);
}

}  // extern "C"
