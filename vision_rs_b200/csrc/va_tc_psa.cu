// PSA Attention forward on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// The reference graph (src/models/yolo/yolo26/blocks/c2psa.rs:61-116) runs
// 7 nodes: qkv conv+BN, psa_pack_qkv, flash attention ×2 (V split into two
// 32-wide halves, psa.rs:930-944), psa_merge_attn_nchw, psa_extract_v_nchw,
// pe dw-conv+BN, add, proj conv+BN.  Here it is four kernels:
//
//  1. qkv_proj_kernel  — persistent GEMM D[128 tok × 256 ch] = xᵀ·W_qkvᵀ on
//     tcgen05 (x tile is the MN-major A operand read straight from NCHW by
//     TMA, W_qkv resident).  The epilogue adds the folded-BN bias and writes
//     exactly the layouts the next kernels read: Q and K token-major
//     [2][B·nh][N][32] (psa_pack_qkv sections 0/1) and V channel-major
//     [B][C][Np] (psa_extract_v_nchw's output), f16.
//  2. attn_kernel      — flash attention per (b, h, pair of 128-query tiles):
//     S = Q·Kᵀ (TMEM), online softmax in registers (two threads per query
//     row), P → TMEM (f16), O += P·V with the full 64-wide V (no lo/hi
//     split).  O is written channel-major [B][C][Np] — the layout
//     psa_merge_attn_nchw produces.
//  3. pe_dwconv(_vec)_kernel — PE = dw3×3(V) + b_pe, f16 [B][C][Np].
//  4. proj_kernel      — D = (O + PE)ᵀ·W_projᵀ on tcgen05 (the sum formed by
//     accumulating both MMAs into one TMEM tile), + b_proj, y stored NCHW bf16.
//
// Precision: x, weights and y are bf16; the qkv GEMM runs bf16×bf16; the
// attention operands Q, K, V, P, O and the proj A operand are f16 (3 more
// mantissa bits than bf16 for values whose range is small: |qkv| is clamped
// to ±65504, P ∈ [0, 256]); every accumulation is f32 in TMEM or registers.
//
// Every mbarrier wait is bounded (sm100::mbar_wait); a timeout records a code
// in g_tc_status and the kernel unwinds, releasing its TMEM.
#include <cudaTypedefs.h>

#include <functional>
#include <vector>

#include "va_common.cuh"
#include "va_psa.h"
#include "va_sm100.cuh"

namespace va {
using namespace sm100;

__device__ int g_tc_status;

namespace {

constexpr int kC = 128;      // PSA hidden channels supported by the tensor-core path
constexpr int kQKV = 256;    // nh*4*kd
constexpr int kKD = 32;      // key_dim
constexpr int kHD = 64;      // head_dim (V width)
constexpr int kTile = 128;   // tokens per tile (UMMA M)

// ── Kernel 1: qkv projection ────────────────────────────────────────────────
// Persistent: a CTA keeps W_qkv (64 KB) resident and walks the (image, 128-
// token tile) items blockIdx.x, blockIdx.x + gridDim.x, …  Warp 0 streams xᵀ
// tiles (two 64-token boxes of the NCHW input per tile) through a TMA ring.
// Warp 1 issues two GEMMs per tile into one of two TMEM accumulator pairs:
//   Q/K:  D1[128 tokens][128] = xᵀ·W_qkᵀ   (x tile as the MN-major A operand)
//   V:    D2[128 channels][128 tokens] = W_v·x  (x tile as the MN-major B operand)
// so V comes out of the tensor core already channel-major.  Eight epilogue
// warps drain the other pair meanwhile: warps 2-5 write Q and K rows (thread =
// token, 64 contiguous bytes per row); warps 6-9 (thread = channel) stage the
// V tile in shared memory as two SW128 [128 channels][64 tokens] boxes
// (16-byte stores, conflict-free) that one thread writes with TMA stores
// (double-buffered).  W_qkv's rows are regrouped on load: the Q/K rows of both
// heads form one 128-row operand, the V rows the other.
constexpr int kQpStages = 2;
constexpr int kQpEpiWarps = 8;
constexpr int kQpThreads = (2 + kQpEpiWarps) * 32;

struct QkvSmem {
  uint8_t wqk[2][128 * 128];          // K-major SW128: 2 k-blocks × 128 rows (head 0 q,k; head 1 q,k)
  uint8_t wv[2][128 * 128];           // K-major SW128: 2 k-blocks × 128 rows (head 0 v; head 1 v)
  uint8_t a[kQpStages][2][kC * 128];  // x tile: 2 blocks of 64 tokens × 128 channel rows, SW128
  uint8_t vst[2][2][kC * 128];        // V staging [buffer][token half]: 128 channel rows × 64 tokens, SW128
  float bias[kQKV];
  uint64_t w_full, a_full[kQpStages], a_empty[kQpStages], acc_full[2], acc_empty[2], fin;
  uint64_t stage_free[2], stage_full[2];
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(kQpThreads, 1)
qkv_proj_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                const __grid_constant__ CUtensorMap map_vst, const float* __restrict__ bias,
                __half* __restrict__ qk, int N, int nh, int B, int ntile) {
  extern __shared__ uint8_t smem_raw[];
  QkvSmem& sm = *reinterpret_cast<QkvSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = B * ntile;
  const int cnt = (int)blockIdx.x < total ? (total - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  auto tile_of = [&](int i) { return (int)blockIdx.x + i * (int)gridDim.x; };

  if (tid == 0) {
    mbar_init(&sm.w_full, 1);
    for (int s = 0; s < kQpStages; ++s) {
      mbar_init(&sm.a_full[s], 1);
      mbar_init(&sm.a_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], kQpEpiWarps * 32);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(&sm.stage_free[k], 1);
      mbar_init(&sm.stage_full[k], 4 * 32);
    }
    mbar_init(&sm.fin, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  for (int i = tid; i < kQKV; i += kQpThreads) sm.bias[i] = bias[i];
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
      mbar_arrive_expect_tx(&sm.w_full, 4 * 128 * 128);
      for (int kb = 0; kb < 2; ++kb)
        for (int h = 0; h < 2; ++h) {  // 64-row boxes: W rows h·128 + [0,64) → q,k; h·128 + [64,128) → v
          tma_load_2d(sm.wqk[kb] + h * 64 * 128, &map_w, &sm.w_full, kb * 64, h * 128);
          tma_load_2d(sm.wv[kb] + h * 64 * 128, &map_w, &sm.w_full, kb * 64, h * 128 + 64);
        }
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < cnt; ++i) {
        const int s = i % kQpStages, t = tile_of(i), b = t / ntile, n0 = (t - b * ntile) * kTile;
        if (i >= kQpStages &&
            !(ok = mbar_wait(&sm.a_empty[s], ((i / kQpStages) - 1) & 1, &sm.abort, &g_tc_status, 1)))
          break;
        mbar_arrive_expect_tx(&sm.a_full[s], 2 * kC * 128);
        tma_load_2d(sm.a[s][0], &map_x, &sm.a_full[s], n0, b * kC);
        tma_load_2d(sm.a[s][1], &map_x, &sm.a_full[s], n0 + 64, b * kC);
        ++issued;
      }
      // every load issued here lands (bounded) before the CTA can exit
      const long long c0 = clock64();
      while (!mbar_try_wait(&sm.w_full, 0) && clock64() - c0 < kSpinCycles) {
      }
      if (!ok) {
        for (int i = max(0, issued - kQpStages); i < issued; ++i) {
          const long long c1 = clock64();
          while (!mbar_try_wait(&sm.a_full[i % kQpStages], (i / kQpStages) & 1) && clock64() - c1 < kSpinCycles) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ── MMA issuer: the warp waits converged, one elected lane issues ──
    constexpr uint32_t id_qk = idesc_f32acc(128, 128, AB_BF16, /*a_mn=*/true, /*b_mn=*/false);
    constexpr uint32_t id_v = idesc_f32acc(128, 128, AB_BF16, /*a_mn=*/false, /*b_mn=*/true);
    const uint32_t wqk0 = smem_u32(sm.wqk[0]), wv0 = smem_u32(sm.wv[0]);
    bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.w_full, 0, &sm.abort, &g_tc_status, 2));
    for (int i = 0; ok && i < cnt; ++i) {
      const int s = i % kQpStages, a = i & 1;
      if (i >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.acc_empty[a], ((i >> 1) - 1) & 1, &sm.abort, &g_tc_status, 3));
        if (!ok) break;
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.a_full[s], (i / kQpStages) & 1, &sm.abort, &g_tc_status, 4));
      if (!ok) break;
      tc_fence_after();
      const uint32_t x0 = smem_u32(sm.a[s][0]);
#pragma unroll
      for (int k = 0; k < kC / 16; ++k) {
        // x tile, MN-major: 16 channel rows per k-step, the two 64-token blocks 16 KB apart
        const uint64_t xd = sdesc(x0 + k * 16 * 128, /*lbo=*/kC * 128, /*sbo=*/1024, SW_128B);
        const uint32_t wk = (k >> 2) * (128 * 128) + (k & 3) * 32;
        mma_ss_w(tmem + a * 256, xd, sdesc(wqk0 + wk, 16, 1024, SW_128B), id_qk, k > 0 ? 1u : 0u);
        mma_ss_w(tmem + a * 256 + 128, sdesc(wv0 + wk, 16, 1024, SW_128B), xd, id_v, k > 0 ? 1u : 0u);
      }
      mma_commit_w(&sm.a_empty[s]);
      mma_commit_w(&sm.acc_full[a]);
    }
    mma_commit_w(&sm.fin);  // every MMA issued here completes before the CTA tears down
    const long long c0 = clock64();
    while (!mbar_try_wait(&sm.fin, 0) && clock64() - c0 < kSpinCycles) {
    }
    __syncwarp();
  } else {
    // ── epilogue warps 2-9 (TMEM lane quarter = warp % 4) ──
    const int q4 = warp & 3, row = q4 * 32 + lane;
    const bool vwarp = warp >= 6;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int BH = B * nh;
    for (int i = 0; i < cnt; ++i) {
      const int a = i & 1, t = tile_of(i), b = t / ntile, n0 = (t - b * ntile) * kTile;
      if (!mbar_wait(&sm.acc_full[a], (i >> 1) & 1, &sm.abort, &g_tc_status, 5)) break;
      tc_fence_after();
      if (!vwarp) {
        // Q/K: thread = token n0 + row; chunk c = (head c/2, section c%2)
        const int n = n0 + row;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int h = c >> 1, sec = c & 1, bcol = h * 128 + sec * 32;
          uint32_t r[32];
          tmem_ld32(tmem + lane_off + a * 256 + c * 32, r);
          tmem_ld_wait();
          reg_fence(r);
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            v[e] = __uint_as_float(r[e]);
            v[e + 1] = __uint_as_float(r[e + 1]);
            fadd2(v[e], v[e + 1], sm.bias[bcol + e], sm.bias[bcol + e + 1]);
          }
          if (n < N) {  // 32 contiguous f16 in [sec][b*nh+h][n][:]
            uint4* dst = reinterpret_cast<uint4*>(qk + (((size_t)sec * BH + (size_t)b * nh + h) * N + n) * kKD);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              dst[q] = make_uint4(pack_f16x2_sat(v[q * 8 + 0], v[q * 8 + 1]), pack_f16x2_sat(v[q * 8 + 2], v[q * 8 + 3]),
                                  pack_f16x2_sat(v[q * 8 + 4], v[q * 8 + 5]), pack_f16x2_sat(v[q * 8 + 6], v[q * 8 + 7]));
          }
        }
      } else {
        // V: thread = channel row (h·64 + cv, the MMA's M index); chunk c = tokens 32c .. 32c+31 of the tile
        const int k = i & 1, h = row >> 6, cv = row & 63;
        const bool storer = warp == 6 && lane == 0;
        const float bv = sm.bias[h * 128 + 64 + cv];
        if (storer) {  // the V store of tile i-2 has read staging buffer k (tile i-1's may be in flight)
          tma_store_wait_read_1();
          mbar_arrive(&sm.stage_free[k]);
        }
        if (!mbar_wait(&sm.stage_free[k], (i >> 1) & 1, &sm.abort, &g_tc_status, 6)) break;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_off + a * 256 + 128 + c * 32, r);
          tmem_ld_wait();
          reg_fence(r);
          uint8_t* box = sm.vst[k][c >> 1];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              v[e] = __uint_as_float(r[q * 8 + e]);
              v[e + 1] = __uint_as_float(r[q * 8 + e + 1]);
              fadd2(v[e], v[e + 1], bv, bv);
            }
            *reinterpret_cast<uint4*>(box + sw128_off(row, (c & 1) * 4 + q)) =
                make_uint4(pack_f16x2_sat(v[0], v[1]), pack_f16x2_sat(v[2], v[3]), pack_f16x2_sat(v[4], v[5]),
                           pack_f16x2_sat(v[6], v[7]));
          }
        }
        tc_fence_before();
        mbar_arrive(&sm.acc_empty[a]);
        fence_proxy_async_smem();
        mbar_arrive(&sm.stage_full[k]);
        if (storer) {
          if (!mbar_wait(&sm.stage_full[k], (i >> 1) & 1, &sm.abort, &g_tc_status, 7)) break;
          tma_store_2d(&map_vst, sm.vst[k][0], n0, b * kC);  // columns past N are clipped
          tma_store_2d(&map_vst, sm.vst[k][1], n0 + 64, b * kC);
          tma_store_commit();
        }
        continue;
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[a]);
    }
    if (warp == 6 && lane == 0) tma_store_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ── Kernel 2: flash attention ───────────────────────────────────────────────
// One CTA = two 128-query tiles (groups g = 0, 1) of one (b, h), sharing
// every K/V tile.  Each query row is split across two warps: warps
// 8g + 4h + w (h = 0, 1; w = 0..3) handle rows 32w..32w+31 (TMEM lanes) and
// key columns 64h..64h+63 of group g, so 16 softmax warps (4 per SM
// sub-partition) feed the exponential unit.  The two halves of a row sit on
// the same SM sub-partition and combine their row maxima through shared
// memory under a barrier of that row quarter (an mbarrier with a bounded
// wait, so a half that aborts cannot leave its partner blocked).
//   warp 16: TMA producer + MMA issuer for group 0;
//   warp 17: MMA issuer for group 1.
// The issuer warps run their loops converged and one elected lane issues each
// tcgen05.mma (a lone lane-0 thread issues about 1.5× slower; the issue rate,
// not the tensor pipe, bounds these small MMAs).
// The two groups take turns on the exponentials, one token per row quarter
// (mufu[g][q]): on each sub-partition one group's exponentials overlap the
// other group's score loads, row maxima and barrier waits.  The token is
// handed over a few pairs before the end of the last chunk, so the hand-off
// latency overlaps the tail of the exponentials.
// TMEM per group g (256 columns at 256·g): S (f32, 128 cols), P (packed f16,
// 64 cols; the A operand of the P·V MMA) and O (f32, 64 cols).  S(j+1) is
// issued as soon as the softmax has copied S(j) into registers (s_free).  P
// has its own columns: a TMEM A-operand read of one MMA is not ordered
// against a later MMA's accumulator writes, so P is rewritten only after the
// MMA that read it completed (o_done).
constexpr int kStages = 4;
constexpr int kVBlk = kHD * 128;           // one 64-key block of V: [64 channel rows × 128 B] SW128 (8 KB)
constexpr int kSoftWarps = 16;
constexpr int kAttnThreads = (kSoftWarps + 2) * 32;
constexpr int kHalf = kTile / 2;           // key columns per softmax thread
constexpr int kTokenPair = 11;  // release the exponential token after this pair of the last chunk (16: after it)
// Exponential pairs (bit e of 16 per 32-score chunk) computed by the FMA-pipe
// polynomial ex2_poly instead of the MUFU unit, which alone would bound the
// softmax at 16 exponentials per SM clock.
constexpr uint32_t kPolyMask = 0x8080u;

__device__ __forceinline__ uint32_t col_s(int g) { return (uint32_t)g * 256u; }
__device__ __forceinline__ uint32_t col_p(int g) { return (uint32_t)g * 256u + 128u; }
__device__ __forceinline__ uint32_t col_o(int g) { return (uint32_t)g * 256u + 192u; }

// KD = 32 (PSA key_dim): Q/K rows of 64 bytes, K-major SW64; KD = 64 (DINOv2
// head dim): rows of 128 bytes, K-major SW128.
template <int KD>
struct AttnSmem {
  static constexpr int kQK = kTile * KD * 2;  // bytes of one Q or K tile
  uint8_t q[2][kQK];                       // Q tiles [128 rows × KD] f16
  uint8_t k[kStages][kQK];                 // K tiles
  uint8_t v[kStages][2][kVBlk];            // V: stage × key-block
  float xmax[2][2][2][kTile];              // [tile parity][group][half][row] partial row maxima
  float xsum[2][2][kTile];                 // [group][half][row] partial row sums (end of loop)
  uint64_t q_full, kv_full[kStages], kv_empty[kStages], s_full[2], s_free[2], p_full[2], o_done[2], fin[2];
  // Per group and row quarter q (the two warps q, q+4 of a group that share SM
  // sub-partition q with the other group's two warps of that quarter):
  uint64_t mufu[2][4];  // ping-pong token: group g may run the exponentials of its next tile
  uint64_t xbar[2][4], fbar[2][4];  // row-max exchange (per tile), row-sum exchange (end)
  uint32_t tmem_base;
  int abort;
};

template <int KD>
__device__ __forceinline__ void attn_load_kv(AttnSmem<KD>& sm, const CUtensorMap* mqk, const CUtensorMap* mv, int t,
                                             int stage, int BH, int bh, int vrow) {
  mbar_arrive_expect_tx(&sm.kv_full[stage], AttnSmem<KD>::kQK + 2 * kVBlk);
  tma_load_3d(sm.k[stage], mqk, &sm.kv_full[stage], 0, t * kTile, BH + bh);
  tma_load_2d(sm.v[stage][0], mv, &sm.kv_full[stage], t * kTile, vrow);
  tma_load_2d(sm.v[stage][1], mv, &sm.kv_full[stage], t * kTile + 64, vrow);
}

// Output layouts: kOutChannelMajor — f16 [B][nh·64][Np] (PSA: the proj
// kernel's operand); kOutTokenMajor — bf16 [BH/nh][N][nh·64] (DINOv2: the
// input of the attention's output Linear).
constexpr int kOutChannelMajor = 0, kOutTokenMajor = 1;

template <int KD, int OUT>
__global__ void __launch_bounds__(kAttnThreads, 1)
attn_kernel(const __grid_constant__ CUtensorMap map_qk, const __grid_constant__ CUtensorMap map_v,
            void* __restrict__ obuf, float* __restrict__ lse, int N, int Np, int nh, float scale_log2,
            int linear_bh) {
  static_assert(KD == 32 || KD == 64, "key dim 32 or 64");
  constexpr int kQK = AttnSmem<KD>::kQK;
  extern __shared__ uint8_t smem_raw[];
  AttnSmem<KD>& sm =
      *reinterpret_cast<AttnSmem<KD>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // linear_bh = 0: grid (tile pair, b·h).  linear_bh = BH: a 1-D grid holding the two-tile
  // items of every (b, h) first and the one-tile items of an odd tile count last, so the
  // grid's last wave holds the short ones
  int pair = blockIdx.x, bh = blockIdx.y, BH = gridDim.y;
  if (linear_bh) {
    const int nfull = ((N + kTile - 1) / kTile) / 2;
    BH = linear_bh;
    if ((int)blockIdx.x < nfull * BH) {
      pair = blockIdx.x % nfull;
      bh = blockIdx.x / nfull;
    } else {
      pair = nfull;
      bh = blockIdx.x - nfull * BH;
    }
  }
  const int q0 = pair * 2 * kTile, b = bh / nh, h = bh % nh;
  const int nkv = (N + kTile - 1) / kTile;
  const bool has1 = q0 + kTile < N;
  const int vrow = bh * kHD;  // V rows [BH·64][Np]

  if (tid == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], has1 ? 2 : 1);  // one commit per issuer
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&sm.s_full[g], 1);
      mbar_init(&sm.s_free[g], 256);
      mbar_init(&sm.p_full[g], 256);
      mbar_init(&sm.o_done[g], 1);
      mbar_init(&sm.fin[g], 1);
      for (int q = 0; q < 4; ++q) {
        mbar_init(&sm.mufu[g][q], 64);
        mbar_init(&sm.xbar[g][q], 64);
        mbar_init(&sm.fbar[g][q], 64);
      }
    }
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

  if (warp >= kSoftWarps) {
    // ── issuer for group g (issuer 0 also drives TMA) ──
    // The whole warp runs this loop (barrier waits and descriptor arithmetic
    // stay warp-uniform); lane 0 issues TMA, one elected lane issues MMAs.
    const int g = warp - kSoftWarps;
    if (g == 0 || has1) {
      const bool producer = g == 0, leader = lane == 0;
      int issued = 0;
      if (producer) {
        if (leader) {
          tma_prefetch_desc(&map_qk);
          tma_prefetch_desc(&map_v);
          mbar_arrive_expect_tx(&sm.q_full, (has1 ? 2 : 1) * kQK);
          tma_load_3d(sm.q[0], &map_qk, &sm.q_full, 0, q0, bh);
          if (has1) tma_load_3d(sm.q[1], &map_qk, &sm.q_full, 0, q0 + kTile, bh);
          for (int t = 0; t < kStages && t < nkv; ++t) attn_load_kv(sm, &map_qk, &map_v, t, t, BH, bh, vrow);
        }
        issued = min(kStages, nkv);
      }
      constexpr uint32_t idS = idesc_f32acc(128, kTile, AB_F16, false, false);
      constexpr uint32_t idO = idesc_f32acc(128, kHD, AB_F16, false, false);
      // Descriptors are built once; a stage / k-step only moves the start-
      // address field (bits 0-13, address >> 4) — a plain add that cannot
      // carry out of the field for shared-memory addresses.
      constexpr uint32_t kSbo = KD == 32 ? 512 : 1024;  // 8 rows of the swizzle atom
      constexpr uint32_t kSwz = KD == 32 ? SW_64B : SW_128B;
      const uint64_t dq = sdesc(smem_u32(sm.q[g]), 16, kSbo, kSwz);
      const uint64_t dk0 = sdesc(smem_u32(sm.k[0]), 16, kSbo, kSwz);
      const uint64_t dv0 = sdesc(smem_u32(sm.v[0][0]), 16, 1024, SW_128B);
      constexpr uint32_t kKStage = kQK >> 4, kVStage = (2 * kVBlk) >> 4, kVHalf = kVBlk >> 4;
      const uint32_t ds = tmem + col_s(g), dp = tmem + col_p(g), dO = tmem + col_o(g);
      auto issue_s = [&](int stage) {
        const uint64_t kd_ = dk0 + (uint64_t)(stage * kKStage);
        mma_ss_w(ds, dq, kd_, idS, 0u);
#pragma unroll
        for (int s = 1; s < KD / 16; ++s) mma_ss_w(ds, dq + 2 * s, kd_ + 2 * s, idS, 1u);  // +32 bytes per k-step
      };
      auto issue_o = [&](int stage, uint32_t acc) {
        const uint64_t vd = dv0 + (uint64_t)(stage * kVStage);
        mma_ts_w(dO, dp, vd, idO, acc);
#pragma unroll
        for (int s = 1; s < kTile / 16; ++s)
          mma_ts_w(dO, dp + s * 8, vd + (uint64_t)((s >> 2) * kVHalf + (s & 3) * 2), idO, 1u);
      };
      bool ok = mbar_wait(&sm.q_full, 0, &sm.abort, &g_tc_status, 10) &&
                mbar_wait(&sm.kv_full[0], 0, &sm.abort, &g_tc_status, 11);
      ok = __all_sync(0xffffffffu, ok);
      int consumed = ok ? 1 : 0;  // K/V tiles whose full barrier this warp observed
      if (ok) {
        tc_fence_after();
        issue_s(0);
        mma_commit_w(&sm.s_full[g]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j % kStages;
        if (j + 1 < nkv) {
          const int stn = (j + 1) % kStages;
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&sm.kv_full[stn], ((j + 1) / kStages) & 1, &sm.abort, &g_tc_status, 12));
          if (!ok) break;
          consumed = j + 2;
          ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_free[g], j & 1, &sm.abort, &g_tc_status, 13));
          if (!ok) break;
          tc_fence_after();
          issue_s(stn);
          mma_commit_w(&sm.s_full[g]);
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.p_full[g], j & 1, &sm.abort, &g_tc_status, 14));
        if (!ok) break;
        tc_fence_after();
        issue_o(st, j > 0 ? 1u : 0u);
        mma_commit_w(&sm.o_done[g]);
        mma_commit_w(&sm.kv_empty[st]);
        // producer: refill the stage tile j-1 used (both issuers done with it) with tile j+3
        if (producer && j >= 1 && j + kStages - 1 < nkv) {
          const int sp = (j - 1) % kStages;
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&sm.kv_empty[sp], ((j - 1) / kStages) & 1, &sm.abort, &g_tc_status, 15));
          if (!ok) break;
          if (leader) attn_load_kv(sm, &map_qk, &map_v, j + kStages - 1, sp, BH, bh, vrow);
          ++issued;
        }
      }
      // teardown: every TMA load issued here has landed, every MMA issued here completed
      if (producer) {
        for (int t = consumed; t < issued; ++t) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&sm.kv_full[t % kStages], (t / kStages) & 1) && clock64() - t0 < kSpinCycles) {
          }
        }
        if (!ok) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&sm.q_full, 0) && clock64() - t0 < kSpinCycles) {
          }
        }
      }
      mma_commit_w(&sm.fin[g]);
      const long long t0 = clock64();
      while (!mbar_try_wait(&sm.fin[g], 0) && clock64() - t0 < kSpinCycles) {
      }
    }
    __syncwarp();
  } else if (warp < 8 || has1) {
    // ── softmax: group g, key half hf, thread = query row (TMEM lane) ──
    const int g = warp >> 3, hf = (warp >> 2) & 1, qr = warp & 3, row = qr * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t sc = tmem + lane_off + col_s(g) + hf * kHalf;
    const uint32_t pc = tmem + lane_off + col_p(g) + hf * (kHalf / 2);
    const uint32_t oc = tmem + lane_off + col_o(g) + hf * (kHD / 2);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!(ok = mbar_wait(&sm.s_full[g], j & 1, &sm.abort, &g_tc_status, 20 + g))) break;
      tc_fence_after();
      float sv[kHalf];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(sc + 0, r0);
        tmem_ld32(sc + 32, r1);
        tmem_ld_wait();
        reg_fence(r0);
        reg_fence(r1);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sv[i] = __uint_as_float(r0[i]);
          sv[32 + i] = __uint_as_float(r1[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.s_free[g]);  // S columns may now take the next tile's scores
      const int kvalid = N - j * kTile - hf * kHalf;
      if (kvalid < kHalf) {
#pragma unroll
        for (int i = 0; i < kHalf; ++i)
          if (i >= kvalid) sv[i] = -INFINITY;
      }
      // partial row max over this thread's 64 scores, then combine the halves
      float mx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = max3(sv[e], sv[8 + e], sv[16 + e]);
#pragma unroll
      for (int i = 24; i < kHalf - 8; i += 16)
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = max3(mx[e], sv[i + e], sv[i + 8 + e]);
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = fmaxf(mx[e], sv[kHalf - 8 + e]);
      mx[0] = max3(mx[0], mx[1], mx[2]);
      mx[3] = max3(mx[3], mx[4], mx[5]);
      mx[6] = fmaxf(mx[6], mx[7]);
      const float pmax = max3(mx[0], mx[3], mx[6]);
      sm.xmax[j & 1][g][hf][row] = pmax;
      mbar_arrive(&sm.xbar[g][qr]);  // release: the partial max is visible to the other half
      if (!(ok = mbar_wait(&sm.xbar[g][qr], j & 1, &sm.abort, &g_tc_status, 30 + g))) break;
      const float rmax = fmaxf(pmax, sm.xmax[j & 1][g][hf ^ 1][row]);
      const float m_new = fmaxf(m, rmax * scale_log2);
      // Rescale only when the running max grew by more than 2^8 (the stale max
      // keeps P ≤ 256; exact after the final division by the row sum).  Both
      // halves see the same maxima, so they make the same decision.
      const bool resc = (j == 0) || (m_new > m + 8.0f);
      const float m_use = resc ? m_new : m;
      const float alpha = resc ? ex2(m - m_use) : 1.0f;
      if (j > 0) {
        // P·V(j-1) done: the P columns are free and O is stable
        if (!(ok = mbar_wait(&sm.o_done[g], (j - 1) & 1, &sm.abort, &g_tc_status, 22 + g))) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
          for (int c = 0; c < kHD / 32; ++c) {  // this half's 32 output columns
            uint32_t o16[16];
            tmem_ld16(oc + c * 16, o16);
            tmem_ld_wait();
            reg_fence(o16);
#pragma unroll
            for (int i = 0; i < 16; ++i) o16[i] = __float_as_uint(__uint_as_float(o16[i]) * alpha);
            tmem_st16(oc + c * 16, o16);
          }
        }
      }
      // ping-pong: group 0 runs exps of tile j after group 1 finished tile j-1;
      // group 1 after group 0 finished tile j
      const bool pp = has1 && (g == 1 || j > 0);
      if (pp && !(ok = mbar_wait(&sm.mufu[g][qr], (g == 0 ? j - 1 : j) & 1, &sm.abort, &g_tc_status, 28 + g))) break;
      const float nm = -m_use;
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int c = 0; c < kHalf / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float x0, x1;
          ffma2(x0, x1, sv[c * 32 + 2 * e], sv[c * 32 + 2 * e + 1], scale_log2, scale_log2, nm, nm);
          const bool poly = (kPolyMask >> e) & 1u;
          const float p0 = poly ? ex2_poly(x0) : ex2(x0);
          const float p1 = poly ? ex2_poly(x1) : ex2(x1);
          fadd2(ls0, ls1, p0, p1);
          pk[e] = pack_f16x2(p0, p1);
          // hand the exponential unit over shortly before the end: the other
          // group's first exponentials overlap this group's last ones instead
          // of waiting out the hand-off latency
          if (has1 && c == kHalf / 32 - 1 && e == kTokenPair) mbar_arrive(&sm.mufu[g ^ 1][qr]);
        }
        tmem_st16(pc + c * 16, pk);
        if (has1 && c == kHalf / 32 - 1 && kTokenPair >= 16) mbar_arrive(&sm.mufu[g ^ 1][qr]);
      }
      tmem_st_wait();
      l = l * alpha + (ls0 + ls1);
      m = m_use;
      tc_fence_before();
      mbar_arrive(&sm.p_full[g]);
    }
    if (ok) ok = mbar_wait(&sm.o_done[g], (nkv - 1) & 1, &sm.abort, &g_tc_status, 24 + g);
    // combine the halves' row sums (every thread of the group reaches this barrier)
    sm.xsum[g][hf][row] = l;
    mbar_arrive(&sm.fbar[g][qr]);
    if (ok) ok = mbar_wait(&sm.fbar[g][qr], 0, &sm.abort, &g_tc_status, 32 + g);
    const float lt = l + sm.xsum[g][hf ^ 1][row];
    if (ok) {
      tc_fence_after();
      const int n = q0 + g * kTile + row;
      const float inv = 1.0f / lt;
      uint32_t o[32];
      tmem_ld32(oc, o);
      tmem_ld_wait();
      reg_fence(o);
      if (n < N) {
        if constexpr (OUT == kOutChannelMajor) {
          __half* dst = static_cast<__half*>(obuf) + ((size_t)bh * kHD + hf * 32) * Np + n;
#pragma unroll
          for (int i = 0; i < 32; ++i) dst[(size_t)i * Np] = __float2half_rn(__uint_as_float(o[i]) * inv);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(obuf) +
                                                ((size_t)b * N + n) * (nh * kHD) + h * kHD + hf * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * q]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
        }
      }
      if (lse && hf == 0 && n < N) lse[(size_t)bh * N + n] = (m + __log2f(lt)) * 0.6931471805599453f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ── Kernel 2s: attention over many short sequences (N ≤ 128) ───────────────
// A sequence fits one 128-key tile, so there is no online rescale and no K/V
// ring.  The CTA is persistent: its two groups each walk their own stream of
// (sequence, head) items, item i of group g being
// (2·blockIdx.x + g) + i·2·gridDim.x.  Per group, Q/K/V of two consecutive
// items are double-buffered in shared memory.
//   warps 0-15 : softmax, 8 per group, two warps per query row (as attn_kernel)
//   warp 16    : TMA producer
//   warps 17/18: MMA issuer of group 0 / 1
// Per item: S = Q·Kᵀ → softmax (row max and row sum exchanged between the two
// warps of a row) → P (f16, TMEM) → O = P·V → O/l stored.
constexpr int kShortThreads = 19 * 32;

template <int KD>
struct ShortSmem {
  static constexpr int kQK = kTile * KD * 2;
  uint8_t q[2][2][kQK];         // [group][buffer]
  uint8_t k[2][2][kQK];
  uint8_t v[2][2][2][kVBlk];    // [group][buffer][key block]
  float xmax[2][2][2][kTile];   // [item parity][group][half][row]
  float xsum[2][2][2][kTile];
  uint64_t load_full[2][2], buf_free[2][2], s_full[2], p_full[2], o_full[2], o_free[2], xbar[2], sbar[2], fin[2];
  uint32_t tmem_base;
  int abort;
};

template <int KD, int OUT>
__global__ void __launch_bounds__(kShortThreads, 1)
attn_short_kernel(const __grid_constant__ CUtensorMap map_qk, const __grid_constant__ CUtensorMap map_v,
                  void* __restrict__ obuf, float* __restrict__ lse, int N, int Np, int nh, int BH, float scale_log2) {
  constexpr int kQK = ShortSmem<KD>::kQK;
  extern __shared__ uint8_t smem_raw[];
  ShortSmem<KD>& sm =
      *reinterpret_cast<ShortSmem<KD>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  auto item_of = [&](int g, int i) { return (2 * (int)blockIdx.x + g) + i * 2 * (int)gridDim.x; };
  auto count_of = [&](int g) {
    const int first = 2 * (int)blockIdx.x + g, step = 2 * (int)gridDim.x;
    return first < BH ? (BH - first + step - 1) / step : 0;
  };

  if (tid == 0) {
    for (int g = 0; g < 2; ++g) {
      for (int b2 = 0; b2 < 2; ++b2) {
        mbar_init(&sm.load_full[g][b2], 1);
        mbar_init(&sm.buf_free[g][b2], 1);
      }
      mbar_init(&sm.s_full[g], 1);
      mbar_init(&sm.p_full[g], 256);
      mbar_init(&sm.o_full[g], 1);
      mbar_init(&sm.o_free[g], 256);
      mbar_init(&sm.xbar[g], 256);
      mbar_init(&sm.sbar[g], 256);
      mbar_init(&sm.fin[g], 1);
    }
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

  if (warp == 16) {
    if (lane == 0) {  // ── TMA producer: both groups, item by item ──
      tma_prefetch_desc(&map_qk);
      tma_prefetch_desc(&map_v);
      const int n0c = count_of(0), n1c = count_of(1), nmax = max(n0c, n1c);
      int issued[2] = {0, 0};
      bool ok = true;
      for (int i = 0; ok && i < nmax; ++i) {
        for (int g = 0; g < 2; ++g) {
          if (i >= (g ? n1c : n0c)) continue;
          const int bf = i & 1;
          if (i >= 2 && !(ok = mbar_wait(&sm.buf_free[g][bf], ((i >> 1) - 1) & 1, &sm.abort, &g_tc_status, 60)))
            break;
          const int bh = item_of(g, i);
          mbar_arrive_expect_tx(&sm.load_full[g][bf], 2 * kQK + 2 * kVBlk);
          tma_load_3d(sm.q[g][bf], &map_qk, &sm.load_full[g][bf], 0, 0, bh);
          tma_load_3d(sm.k[g][bf], &map_qk, &sm.load_full[g][bf], 0, 0, BH + bh);
          tma_load_2d(sm.v[g][bf][0], &map_v, &sm.load_full[g][bf], 0, bh * kHD);
          tma_load_2d(sm.v[g][bf][1], &map_v, &sm.load_full[g][bf], 64, bh * kHD);
          ++issued[g];
        }
      }
      if (!ok) {  // wait (bounded) for the loads of the last two items of each group
        for (int g = 0; g < 2; ++g)
          for (int i = max(0, issued[g] - 2); i < issued[g]; ++i) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&sm.load_full[g][i & 1], (i >> 1) & 1) && clock64() - t0 < kSpinCycles) {
            }
          }
      }
    }
    __syncwarp();
  } else if (warp >= 17) {
    const int g = warp - 17;
    if (lane == 0) {  // ── MMA issuer of group g ──
      constexpr uint32_t idS = idesc_f32acc(128, kTile, AB_F16, false, false);
      constexpr uint32_t idO = idesc_f32acc(128, kHD, AB_F16, false, false);
      constexpr uint32_t kSbo = KD == 32 ? 512 : 1024;
      constexpr uint32_t kSwz = KD == 32 ? SW_64B : SW_128B;
      constexpr uint32_t kVHalf = kVBlk >> 4;
      const uint32_t ds = tmem + col_s(g), dp = tmem + col_p(g), dO = tmem + col_o(g);
      const int cnt = count_of(g);
      bool ok = true;
      for (int i = 0; i < cnt; ++i) {
        const int bf = i & 1;
        if (!(ok = mbar_wait(&sm.load_full[g][bf], (i >> 1) & 1, &sm.abort, &g_tc_status, 61))) break;
        tc_fence_after();
        const uint64_t dq = sdesc(smem_u32(sm.q[g][bf]), 16, kSbo, kSwz);
        const uint64_t dk = sdesc(smem_u32(sm.k[g][bf]), 16, kSbo, kSwz);
        const uint64_t dv = sdesc(smem_u32(sm.v[g][bf][0]), 16, 1024, SW_128B);
        mma_ss(ds, dq, dk, idS, 0u);
#pragma unroll
        for (int s = 1; s < KD / 16; ++s) mma_ss(ds, dq + 2 * s, dk + 2 * s, idS, 1u);
        mma_commit(&sm.s_full[g]);
        if (!(ok = mbar_wait(&sm.p_full[g], i & 1, &sm.abort, &g_tc_status, 62))) break;
        if (i > 0 && !(ok = mbar_wait(&sm.o_free[g], (i - 1) & 1, &sm.abort, &g_tc_status, 63))) break;
        tc_fence_after();
        mma_ts(dO, dp, dv, idO, 0u);
#pragma unroll
        for (int s = 1; s < kTile / 16; ++s)
          mma_ts(dO, dp + s * 8, dv + (uint64_t)((s >> 2) * kVHalf + (s & 3) * 2), idO, 1u);
        mma_commit(&sm.o_full[g]);
        mma_commit(&sm.buf_free[g][bf]);
      }
      mma_commit(&sm.fin[g]);
      const long long t0 = clock64();
      while (!mbar_try_wait(&sm.fin[g], 0) && clock64() - t0 < kSpinCycles) {
      }
    }
    __syncwarp();
  } else {
    // ── softmax: group g, key half hf, thread = query row (TMEM lane) ──
    const int g = warp >> 3, hf = (warp >> 2) & 1, row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t sc = tmem + lane_off + col_s(g) + hf * kHalf;
    const uint32_t pc = tmem + lane_off + col_p(g) + hf * (kHalf / 2);
    const uint32_t oc = tmem + lane_off + col_o(g) + hf * (kHD / 2);
    const int cnt = count_of(g);
    const int kvalid = N - hf * kHalf;
    bool ok = true;
    for (int i = 0; i < cnt; ++i) {
      const int par = i & 1, bh = item_of(g, i);
      if (!(ok = mbar_wait(&sm.s_full[g], par, &sm.abort, &g_tc_status, 64))) break;
      tc_fence_after();
      float sv[kHalf];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(sc + 0, r0);
        tmem_ld32(sc + 32, r1);
        tmem_ld_wait();
        reg_fence(r0);
        reg_fence(r1);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          sv[c] = __uint_as_float(r0[c]);
          sv[32 + c] = __uint_as_float(r1[c]);
        }
      }
      if (kvalid < kHalf) {
#pragma unroll
        for (int c = 0; c < kHalf; ++c)
          if (c >= kvalid) sv[c] = -INFINITY;
      }
      float mx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = max3(sv[e], sv[8 + e], sv[16 + e]);
#pragma unroll
      for (int c = 24; c < kHalf - 8; c += 16)
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = max3(mx[e], sv[c + e], sv[c + 8 + e]);
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = fmaxf(mx[e], sv[kHalf - 8 + e]);
      const float pmax = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
      sm.xmax[par][g][hf][row] = pmax;
      mbar_arrive(&sm.xbar[g]);
      if (!(ok = mbar_wait(&sm.xbar[g], par, &sm.abort, &g_tc_status, 65))) break;
      const float m = fmaxf(pmax, sm.xmax[par][g][hf ^ 1][row]) * scale_log2;
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int c = 0; c < kHalf / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = ex2(fmaf(sv[c * 32 + 2 * e], scale_log2, -m));
          const float p1 = ex2(fmaf(sv[c * 32 + 2 * e + 1], scale_log2, -m));
          ls0 += p0;
          ls1 += p1;
          pk[e] = pack_f16x2(p0, p1);
        }
        tmem_st16(pc + c * 16, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sm.p_full[g]);
      const float ls = ls0 + ls1;
      sm.xsum[par][g][hf][row] = ls;
      mbar_arrive(&sm.sbar[g]);
      if (!(ok = mbar_wait(&sm.sbar[g], par, &sm.abort, &g_tc_status, 66))) break;
      const float l = ls + sm.xsum[par][g][hf ^ 1][row];
      if (!(ok = mbar_wait(&sm.o_full[g], par, &sm.abort, &g_tc_status, 67))) break;
      tc_fence_after();
      uint32_t o[32];
      tmem_ld32(oc, o);
      tmem_ld_wait();
      reg_fence(o);
      tc_fence_before();
      mbar_arrive(&sm.o_free[g]);
      const float inv = 1.0f / l;
      if (row < N) {
        if constexpr (OUT == kOutChannelMajor) {
          __half* dst = static_cast<__half*>(obuf) + ((size_t)bh * kHD + hf * 32) * Np + row;
#pragma unroll
          for (int c = 0; c < 32; ++c) dst[(size_t)c * Np] = __float2half_rn(__uint_as_float(o[c]) * inv);
        } else {
          const int b = bh / nh, h = bh % nh;
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(obuf) + ((size_t)b * N + row) * (nh * kHD) +
                                                h * kHD + hf * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * q]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
        }
        if (lse && hf == 0) lse[(size_t)bh * N + row] = (m + __log2f(l)) * 0.6931471805599453f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ── Kernel 3: positional encoding (depthwise 3×3 + bias) ───────────────────
// One CTA per (image, group of kPeCh channels).  Each channel plane is read
// with 16-byte loads (all in flight at once), widened to f32 into a zero-
// bordered [H+2][W2] shared-memory plane (odd pitch W2 ≥ W+10).  A thread then
// produces an 8-column × kPeRows-row block of one channel, sliding a 3-row
// window of 10 values down the rows (1.5 shared loads and 9 FMAs per output;
// the item index is decomposed once per block).  PE is stored f16 [B][C][Np],
// the layout the projection kernel reads with TMA.  CTA 0 also converts
// W_proj (bf16) to the f16 operand the projection uses.
constexpr int kPeCh = 4;
constexpr int kPeThreads = 256;
constexpr int kPeRows = 4;
constexpr int kMaxPlane = 12288;   // (H+2)·pitch floats per staged channel

__global__ void __launch_bounds__(kPeThreads)
pe_dwconv_kernel(const __half* __restrict__ vbuf, const __nv_bfloat16* __restrict__ w_pe,
                 const float* __restrict__ b_pe, __half* __restrict__ pebuf,
                 const __nv_bfloat16* __restrict__ w_proj, __half* __restrict__ wproj16, int H, int W, int Np) {
  extern __shared__ float plane[];   // [kPeCh][(H+2)*W2]
  const int tid = threadIdx.x;
  const int N = H * W, W2 = (W + 10) | 1, P2 = (H + 2) * W2;
  const int cg = blockIdx.x, b = blockIdx.y;
  if (cg == 0 && b == 0) {
    for (int i = tid; i < kC * kC / 8; i += kPeThreads) {
      const uint4 src = __ldg(reinterpret_cast<const uint4*>(w_proj) + i);
      const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&src);
      uint4 u;
      uint32_t* uu = &u.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(s2[e]);
        uu[e] = pack_f16x2_sat(f.x, f.y);
      }
      reinterpret_cast<uint4*>(wproj16)[i] = u;
    }
  }
  // border cells (rows 0 and H+1, column 0 and columns W+1.. of the pitch) are
  // zero; they are disjoint from the interior, so one barrier covers both
  for (int c = 0; c < kPeCh; ++c) {
    float* pl = plane + c * P2;
    for (int i = tid; i < W2; i += kPeThreads) {
      pl[i] = 0.f;
      pl[(H + 1) * W2 + i] = 0.f;
    }
    const int nb = W2 - W;  // column 0 plus the W2-W-1 columns right of the image
    for (int i = tid; i < H * nb; i += kPeThreads) {
      const int r = i / nb, k = i - r * nb;
      pl[(r + 1) * W2 + (k == 0 ? 0 : W + k)] = 0.f;
    }
  }
  const int nchunk = Np >> 3;
  const __half* vb = vbuf + ((size_t)b * kC + (size_t)cg * kPeCh) * Np;
  constexpr int kBatch = 4;
  for (int base = tid; base < kPeCh * nchunk; base += kPeThreads * kBatch) {
    uint4 u[kBatch];
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const int i = base + q * kPeThreads;
      if (i < kPeCh * nchunk) {
        const int c = i / nchunk, k = i - c * nchunk;
        u[q] = __ldg(reinterpret_cast<const uint4*>(vb + (size_t)c * Np) + k);
      }
    }
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const int i = base + q * kPeThreads;
      if (i < kPeCh * nchunk) {
        const int c = i / nchunk, k = i - c * nchunk;
        const __half* h = reinterpret_cast<const __half*>(&u[q]);
        const int n = k * 8;
        int r = n / W, j = n - r * W;
        if ((W & 7) == 0) {  // the 8 tokens lie in one image row
          float* dst = plane + c * P2 + (r + 1) * W2 + j + 1;
#pragma unroll
          for (int e = 0; e < 8; ++e) dst[e] = __half2float(h[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (n + e < N) plane[c * P2 + (r + 1) * W2 + j + 1] = __half2float(h[e]);
            if (++j == W) { j = 0; ++r; }
          }
        }
      }
    }
  }
  __syncthreads();
  const int ngrp = (W + 7) >> 3, nrb = (H + kPeRows - 1) / kPeRows;
  const bool vec_store = (W & 7) == 0;
  for (int it = tid; it < kPeCh * ngrp * nrb; it += kPeThreads) {
    const int rb = it % nrb, rest = it / nrb;
    const int g = rest % ngrp, c = rest / ngrp;
    const int ch = cg * kPeCh + c, j0 = g * 8, r0 = rb * kPeRows;
    float w[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) w[t] = __bfloat162float(w_pe[ch * 9 + t]);
    const float bias = b_pe[ch];
    const float* p = plane + c * P2 + r0 * W2 + j0;   // window top-left: image (r0-1, j0-1)
    float xa[10], xb[10];
#pragma unroll
    for (int q = 0; q < 10; ++q) {
      xa[q] = p[q];
      xb[q] = p[W2 + q];
    }
    __half* out = pebuf + ((size_t)b * kC + ch) * Np + (size_t)r0 * W + j0;
#pragma unroll
    for (int rr = 0; rr < kPeRows; ++rr) {
      if (r0 + rr >= H) break;
      float xc[10];
#pragma unroll
      for (int q = 0; q < 10; ++q) xc[q] = p[(rr + 2) * W2 + q];
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float a = fmaf(w[0], xa[e], fmaf(w[1], xa[e + 1], fmaf(w[2], xa[e + 2], bias)));
        a = fmaf(w[3], xb[e], fmaf(w[4], xb[e + 1], fmaf(w[5], xb[e + 2], a)));
        acc[e] = fmaf(w[6], xc[e], fmaf(w[7], xc[e + 1], fmaf(w[8], xc[e + 2], a)));
      }
      if (vec_store) {
        uint4 u;
        u.x = pack_f16x2(acc[0], acc[1]);
        u.y = pack_f16x2(acc[2], acc[3]);
        u.z = pack_f16x2(acc[4], acc[5]);
        u.w = pack_f16x2(acc[6], acc[7]);
        *reinterpret_cast<uint4*>(out) = u;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (j0 + e < W) out[e] = __float2half_rn(acc[e]);
      }
#pragma unroll
      for (int q = 0; q < 10; ++q) {
        xa[q] = xb[q];
        xb[q] = xc[q];
      }
      out += W;
    }
  }
}

// Kernel 3v: the same positional encoding for W % CW == 0 (CW = 8 or 4)
// without shared memory: a thread produces a CW-column × kPevRows-row block of
// one channel (columns j0..j0+CW-1 of rows r0..r0+kPevRows-1) from kPevRows+2
// row loads of 2·CW bytes plus the two edge values of each row (L1 hits:
// neighbouring threads read the same lines), all issued before any
// arithmetic, with packed f32x2 FMAs.  Blocks are numbered over all B·C
// planes, so a launch has no idle tail per plane.  CTA 0 also converts
// W_proj, as above.
constexpr int kPevThreads = 256;
constexpr int kPevRows = 4;

template <int CW> struct PeRow;
template <> struct PeRow<8> {
  using T = uint4;
  __device__ static void unpack(const T& u, float* x) {
    const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h2[e]);
      x[2 * e] = f.x;
      x[2 * e + 1] = f.y;
    }
  }
  __device__ static T pack(const float* a) {
    return make_uint4(pack_f16x2(a[0], a[1]), pack_f16x2(a[2], a[3]), pack_f16x2(a[4], a[5]), pack_f16x2(a[6], a[7]));
  }
};
template <> struct PeRow<4> {
  using T = uint2;
  __device__ static void unpack(const T& u, float* x) {
    const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float2 f = __half22float2(h2[e]);
      x[2 * e] = f.x;
      x[2 * e + 1] = f.y;
    }
  }
  __device__ static T pack(const float* a) { return make_uint2(pack_f16x2(a[0], a[1]), pack_f16x2(a[2], a[3])); }
};

// Also used by the other widths (va_tc_psa_wide.cu) with C channels per image
// and `add` (O): then pebuf receives O + PE.  Block 0 converts W_proj
// [C][C] to f16 on the side.
template <int CW>
__global__ void __launch_bounds__(kPevThreads)
pe_dwconv_vec_kernel(const __half* __restrict__ vbuf, const __nv_bfloat16* __restrict__ w_pe,
                     const float* __restrict__ b_pe, __half* __restrict__ pebuf,
                     const __nv_bfloat16* __restrict__ w_proj, __half* __restrict__ wproj16, int B, int H, int W,
                     int Np, int C, const __half* __restrict__ add) {
  using Row = PeRow<CW>;
  const int tid = threadIdx.x;
  if (blockIdx.x == 0) {
    for (int i = tid; i < C * C / 8; i += kPevThreads) {
      const uint4 src = __ldg(reinterpret_cast<const uint4*>(w_proj) + i);
      const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&src);
      uint4 u;
      uint32_t* uu = &u.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(s2[e]);
        uu[e] = pack_f16x2_sat(f.x, f.y);
      }
      reinterpret_cast<uint4*>(wproj16)[i] = u;
    }
  }
  constexpr int R = kPevRows;
  const unsigned cpr = W / CW, nrb = (H + R - 1) / R, nblk = nrb * cpr;  // per plane
  const unsigned q = blockIdx.x * kPevThreads + tid;  // < 2^31 (checked by the launcher)
  if (q >= (unsigned)B * C * nblk) return;
  const unsigned plane = q / nblk, k = q - plane * nblk;
  const int rb = (int)(k / cpr), j0 = (int)(k - rb * cpr) * CW, r0 = rb * R, ch = (int)(plane % (unsigned)C);
  const __half* src = vbuf + (size_t)plane * Np + j0;
  // rows r0-1 .. r0+R, clamped into the image (masked below)
  typename Row::T u[R + 2];
  __half2 edge[R + 2];
#pragma unroll
  for (int i = 0; i < R + 2; ++i) {
    const int rr = min(max(r0 + i - 1, 0), H - 1);
    const __half* row = src + (size_t)rr * W;
    u[i] = __ldg(reinterpret_cast<const typename Row::T*>(row));
    edge[i] = __halves2half2(__ldg(row + (j0 > 0 ? -1 : 0)), __ldg(row + (j0 + CW < W ? CW : CW - 1)));
  }
  float w[9];
#pragma unroll
  for (int t = 0; t < 9; ++t) w[t] = __bfloat162float(w_pe[ch * 9 + t]);
  const float bias = b_pe[ch];
  float x[R + 2][CW + 2];
#pragma unroll
  for (int i = 0; i < R + 2; ++i) {
    const int rr = r0 + i - 1;
    const bool in = rr >= 0 && rr < H;
    float xv[CW];
    Row::unpack(u[i], xv);
#pragma unroll
    for (int e = 0; e < CW; ++e) x[i][1 + e] = in ? xv[e] : 0.f;
    const float2 ed = __half22float2(edge[i]);
    x[i][0] = in && j0 > 0 ? ed.x : 0.f;
    x[i][CW + 1] = in && j0 + CW < W ? ed.y : 0.f;
  }
  __half* dst = pebuf + (size_t)plane * Np + (size_t)r0 * W + j0;
#pragma unroll
  for (int o = 0; o < R; ++o) {
    if (r0 + o >= H) break;
    float acc[CW];
#pragma unroll
    for (int e = 0; e < CW; ++e) acc[e] = bias;
#pragma unroll
    for (int di = 0; di < 3; ++di) {
      const float* xr = x[o + di];
#pragma unroll
      for (int e = 0; e < CW; e += 2) {
        ffma2(acc[e], acc[e + 1], w[di * 3 + 2], w[di * 3 + 2], xr[e + 2], xr[e + 3], acc[e], acc[e + 1]);
        ffma2(acc[e], acc[e + 1], w[di * 3 + 1], w[di * 3 + 1], xr[e + 1], xr[e + 2], acc[e], acc[e + 1]);
        ffma2(acc[e], acc[e + 1], w[di * 3], w[di * 3], xr[e], xr[e + 1], acc[e], acc[e + 1]);
      }
    }
    if (add) {
      float ov[CW];
      Row::unpack(__ldg(reinterpret_cast<const typename Row::T*>(add + (size_t)plane * Np + (size_t)(r0 + o) * W + j0)),
                  ov);
#pragma unroll
      for (int e = 0; e < CW; ++e) acc[e] += ov[e];
    }
    *reinterpret_cast<typename Row::T*>(dst + (size_t)o * W) = Row::pack(acc);
  }
}


// ── Kernel 4: output projection y = W_proj·(O + PE) + b_proj ───────────────
// Both O and PE tiles arrive by TMA as MN-major operands; the sum O + PE is
// formed by the tensor core itself: D = Oᵀ·W_projᵀ, then D += PEᵀ·W_projᵀ
// into the same TMEM accumulator (16 k-steps).
struct ProjSmem {
  uint8_t o[2][kC * 128];    // Oᵀ tile, MN-major SW128: 2 blocks of 64 tokens × 128 channel rows
  uint8_t pe[2][kC * 128];   // PEᵀ tile, same layout
  uint8_t w[2][kC * 128];    // W_proj f16, K-major SW128: 2 blocks of 64 in-channels × 128 rows
  float bias[kC];
  uint64_t full_bar, mma_bar;
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(128, 1)
proj_kernel(const __grid_constant__ CUtensorMap map_o, const __grid_constant__ CUtensorMap map_pe,
            const __grid_constant__ CUtensorMap map_w, const float* __restrict__ b_proj,
            __nv_bfloat16* __restrict__ y, int N) {
  extern __shared__ uint8_t smem_raw[];
  ProjSmem& sm = *reinterpret_cast<ProjSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kTile, b = blockIdx.y;
  if (tid == 0) {
    mbar_init(&sm.full_bar, 1);
    mbar_init(&sm.mma_bar, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  sm.bias[tid] = b_proj[tid];
  if (warp == 0) {
    tmem_alloc(&sm.tmem_base, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  if (tid == 0) {
    tma_prefetch_desc(&map_o);
    tma_prefetch_desc(&map_pe);
    tma_prefetch_desc(&map_w);
    mbar_arrive_expect_tx(&sm.full_bar, 6 * kC * 128);
    tma_load_2d(sm.o[0], &map_o, &sm.full_bar, n0, b * kC);
    tma_load_2d(sm.o[1], &map_o, &sm.full_bar, n0 + 64, b * kC);
    tma_load_2d(sm.pe[0], &map_pe, &sm.full_bar, n0, b * kC);
    tma_load_2d(sm.pe[1], &map_pe, &sm.full_bar, n0 + 64, b * kC);
    tma_load_2d(sm.w[0], &map_w, &sm.full_bar, 0, 0);
    tma_load_2d(sm.w[1], &map_w, &sm.full_bar, 64, 0);
    if (mbar_wait(&sm.full_bar, 0, &sm.abort, &g_tc_status, 30)) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_f32acc(128, kC, AB_F16, /*a_mn=*/true, /*b_mn=*/false);
      const uint32_t o0 = smem_u32(sm.o[0]), p0 = smem_u32(sm.pe[0]), w0 = smem_u32(sm.w[0]);
#pragma unroll
      for (int s = 0; s < 2 * kC / 16; ++s) {
        const int k = s & 7;
        const uint32_t a0 = s < 8 ? o0 : p0;
        uint64_t ad = sdesc(a0 + k * 16 * 128, kC * 128, 1024, SW_128B);
        uint64_t bd = sdesc(w0 + (k >> 2) * (kC * 128) + (k & 3) * 32, 16, 1024, SW_128B);
        mma_ss(tmem, ad, bd, idesc, s > 0);
      }
    } else {
      const long long t0 = clock64();
      while (!mbar_try_wait(&sm.full_bar, 0) && clock64() - t0 < kSpinCycles) {
      }
    }
    mma_commit(&sm.mma_bar);
  }
  __syncwarp();
  const bool ok = mbar_wait(&sm.mma_bar, 0, &sm.abort, &g_tc_status, 31) && !sm.abort;
  tc_fence_after();
  if (ok) {
    const int n = n0 + warp * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < kC / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c * 32, r);
      tmem_ld_wait();
      reg_fence(r);
      if (n < N) {
        __nv_bfloat16* dst = y + ((size_t)b * kC + c * 32) * N + n;
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[(size_t)i * N] = __float2bfloat16_rn(__uint_as_float(r[i]) + sm.bias[c * 32 + i]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// Kernel 4p: the projection for N % 8 == 0 (y rows TMA-addressable),
// persistent and transposed: D[128 out-channels][128 tokens] = W_proj·O +
// W_proj·PE (W_proj resident as the K-major A operand, the O and PE tiles as
// MN-major B operands straight from their channel-major buffers), so y comes
// out of the tensor core channel-major.  Warp 0 streams (O, PE) tiles through
// a two-stage TMA ring, warp 1 issues the 16 MMAs of a tile into one of two
// TMEM accumulators, warps 2-5 (thread = output channel) add b_proj, stage
// the bf16 tile as two SW128 [128 channels][64 tokens] boxes and one thread
// writes them with TMA stores.
constexpr int kPpStages = 2;
constexpr int kPpThreads = 6 * 32;

struct ProjPSmem {
  uint8_t w[2][kC * 128];                // W_proj f16, K-major SW128: 2 k-blocks × 128 rows
  uint8_t x[kPpStages][2][2][kC * 128];  // [stage][O, PE][token half]: 128 channel rows × 64 tokens, SW128
  uint8_t yst[2][kC * 128];              // y staging [token half]: 128 channel rows × 64 tokens bf16, SW128
  float bias[kC];
  uint64_t w_full, x_full[kPpStages], x_empty[kPpStages], acc_full[2], acc_empty[2], stage_free, stage_full, fin;
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(kPpThreads, 1)
proj_pers_kernel(const __grid_constant__ CUtensorMap map_o, const __grid_constant__ CUtensorMap map_pe,
                 const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_y,
                 const float* __restrict__ b_proj, int B, int ntile) {
  extern __shared__ uint8_t smem_raw[];
  ProjPSmem& sm =
      *reinterpret_cast<ProjPSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = B * ntile;
  const int cnt = (int)blockIdx.x < total ? (total - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  auto tile_of = [&](int i) { return (int)blockIdx.x + i * (int)gridDim.x; };

  if (tid == 0) {
    mbar_init(&sm.w_full, 1);
    for (int s = 0; s < kPpStages; ++s) {
      mbar_init(&sm.x_full[s], 1);
      mbar_init(&sm.x_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.acc_full[a], 1);
      mbar_init(&sm.acc_empty[a], 128);
    }
    mbar_init(&sm.stage_free, 1);
    mbar_init(&sm.stage_full, 128);
    mbar_init(&sm.fin, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  for (int i = tid; i < kC; i += kPpThreads) sm.bias[i] = b_proj[i];
  if (warp == 0) {
    tmem_alloc(&sm.tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0) {  // ── TMA producer ──
      tma_prefetch_desc(&map_o);
      tma_prefetch_desc(&map_pe);
      tma_prefetch_desc(&map_w);
      mbar_arrive_expect_tx(&sm.w_full, 2 * kC * 128);
      tma_load_2d(sm.w[0], &map_w, &sm.w_full, 0, 0);
      tma_load_2d(sm.w[1], &map_w, &sm.w_full, 64, 0);
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < cnt; ++i) {
        const int s = i % kPpStages, t = tile_of(i), b = t / ntile, n0 = (t - b * ntile) * kTile;
        if (i >= kPpStages &&
            !(ok = mbar_wait(&sm.x_empty[s], ((i / kPpStages) - 1) & 1, &sm.abort, &g_tc_status, 40)))
          break;
        mbar_arrive_expect_tx(&sm.x_full[s], 4 * kC * 128);
        tma_load_2d(sm.x[s][0][0], &map_o, &sm.x_full[s], n0, b * kC);
        tma_load_2d(sm.x[s][0][1], &map_o, &sm.x_full[s], n0 + 64, b * kC);
        tma_load_2d(sm.x[s][1][0], &map_pe, &sm.x_full[s], n0, b * kC);
        tma_load_2d(sm.x[s][1][1], &map_pe, &sm.x_full[s], n0 + 64, b * kC);
        ++issued;
      }
      const long long c0 = clock64();
      while (!mbar_try_wait(&sm.w_full, 0) && clock64() - c0 < kSpinCycles) {
      }
      if (!ok) {
        for (int i = max(0, issued - kPpStages); i < issued; ++i) {
          const long long c1 = clock64();
          while (!mbar_try_wait(&sm.x_full[i % kPpStages], (i / kPpStages) & 1) && clock64() - c1 < kSpinCycles) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ── MMA issuer (converged warp, elected lane) ──
    constexpr uint32_t idesc = idesc_f32acc(128, kTile, AB_F16, /*a_mn=*/false, /*b_mn=*/true);
    const uint32_t w0 = smem_u32(sm.w[0]);
    bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.w_full, 0, &sm.abort, &g_tc_status, 41));
    for (int i = 0; ok && i < cnt; ++i) {
      const int s = i % kPpStages, a = i & 1;
      if (i >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&sm.acc_empty[a], ((i >> 1) - 1) & 1, &sm.abort, &g_tc_status, 42));
        if (!ok) break;
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.x_full[s], (i / kPpStages) & 1, &sm.abort, &g_tc_status, 43));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int src = 0; src < 2; ++src) {  // O, then PE into the same accumulator
        const uint32_t x0 = smem_u32(sm.x[s][src][0]);
#pragma unroll
        for (int k = 0; k < kC / 16; ++k) {
          const uint64_t ad = sdesc(w0 + (k >> 2) * (kC * 128) + (k & 3) * 32, 16, 1024, SW_128B);
          const uint64_t bd = sdesc(x0 + k * 16 * 128, /*lbo=*/kC * 128, /*sbo=*/1024, SW_128B);
          mma_ss_w(tmem + a * 128, ad, bd, idesc, (src | k) ? 1u : 0u);
        }
      }
      mma_commit_w(&sm.x_empty[s]);
      mma_commit_w(&sm.acc_full[a]);
    }
    mma_commit_w(&sm.fin);
    const long long c0 = clock64();
    while (!mbar_try_wait(&sm.fin, 0) && clock64() - c0 < kSpinCycles) {
    }
    __syncwarp();
  } else {
    // ── epilogue warps 2-5: thread = output channel (TMEM lane) ──
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const bool storer = warp == 2 && lane == 0;
    const float bv = sm.bias[row];
    for (int i = 0; i < cnt; ++i) {
      const int a = i & 1, t = tile_of(i), b = t / ntile, n0 = (t - b * ntile) * kTile;
      if (!mbar_wait(&sm.acc_full[a], (i >> 1) & 1, &sm.abort, &g_tc_status, 44)) break;
      tc_fence_after();
      if (storer) {  // the previous tile's y store has read the staging tile
        tma_store_wait_read();
        mbar_arrive(&sm.stage_free);
      }
      if (!mbar_wait(&sm.stage_free, i & 1, &sm.abort, &g_tc_status, 45)) break;
#pragma unroll 1
      for (int c = 0; c < kTile / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + a * 128 + c * 32, r);
        tmem_ld_wait();
        reg_fence(r);
        uint8_t* box = sm.yst[c >> 1];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            v[e] = __uint_as_float(r[q * 8 + e]);
            v[e + 1] = __uint_as_float(r[q * 8 + e + 1]);
            fadd2(v[e], v[e + 1], bv, bv);
          }
          *reinterpret_cast<uint4*>(box + sw128_off(row, (c & 1) * 4 + q)) =
              make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                         pack_bf16x2(v[6], v[7]));
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[a]);
      fence_proxy_async_smem();
      mbar_arrive(&sm.stage_full);
      if (storer) {
        if (!mbar_wait(&sm.stage_full, i & 1, &sm.abort, &g_tc_status, 46)) break;
        tma_store_2d(&map_y, sm.yst[0], n0, b * kC);  // columns past N are clipped
        tma_store_2d(&map_y, sm.yst[1], n0 + 64, b * kC);
        tma_store_commit();
      }
    }
    if (storer) tma_store_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// x with a row pitch that TMA cannot address (N*2 bytes not a multiple of 16)
// is first copied into a padded buffer.
__global__ void pad_rows_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ xp, int rows, int N,
                                int Np) {
  const long long total = (long long)rows * Np;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / Np;
    const int n = (int)(i - r * Np);
    xp[i] = n < N ? x[r * N + n] : __float2bfloat16_rn(0.f);
  }
}

// ── host side ───────────────────────────────────────────────────────────────
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz, const char* what) {
  auto fn = encode_fn();
  if (!fn) return set_error(VA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  uint32_t es[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(m, dt, rank, const_cast<void*>(base), dims, strides_bytes, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "tensor map for %s rejected (CUresult %d)", what, (int)r);
  return VA_OK;
}

struct TcWs {
  size_t qk, v, o, pe, wproj, xpad, total;
};

TcWs tc_layout(int B, int H, int W, int nh) {
  const size_t N = (size_t)H * W, Np = (N + 7) / 8 * 8, BH = (size_t)B * nh;
  TcWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  w.qk = take(2 * BH * N * kKD * 2);
  w.v = take((size_t)B * kC * Np * 2);
  w.o = take((size_t)B * kC * Np * 2);
  w.pe = take((size_t)B * kC * Np * 2);
  w.wproj = take((size_t)kC * kC * 2);
  w.xpad = (N % 8) ? take((size_t)B * kC * Np * 2) : (size_t)-1;
  w.total = off;
  return w;
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return VA_OK;
}

// Launch order of the attention grid.  With an odd tile count every (b, h)
// has one one-tile item (≈0.8 of a two-tile item's time: no ping-pong
// partner).  The block scheduler hands blocks to SMs in grid order as SMs
// free up, so the grid's last wave depends on where the short items sit.
// attn_odd_last() models that greedy assignment on the device's SM count for
// the (b, h)-interleaved order and for "all two-tile items, then the one-tile
// items", and takes the latter when the model's makespan is ≥ 3% shorter
// (e.g. 16 × 6 heads × 1601 tokens: 4.8 against 5.0 items; 64 × 2 heads ×
// 1600 tokens: equal, and measured slower).  One entry per host thread caches
// the last shape's decision.
double attn_makespan(int nfull, int BH, int P, bool odd_last) {
  std::vector<double> h((size_t)P, 0.0);  // min-heap of SM free times
  double m = 0.0;
  auto take = [&](double len) {
    std::pop_heap(h.begin(), h.end(), std::greater<double>());
    h.back() += len;
    m = std::max(m, h.back());
    std::push_heap(h.begin(), h.end(), std::greater<double>());
  };
  if (odd_last) {
    for (long long i = 0; i < (long long)nfull * BH; ++i) take(1.0);
    for (int i = 0; i < BH; ++i) take(0.8);
  } else {
    for (int bh = 0; bh < BH; ++bh) {
      for (int i = 0; i < nfull; ++i) take(1.0);
      take(0.8);
    }
  }
  return m;
}

bool attn_odd_last(int ntile, int BH) {
  if (!(ntile & 1) || ntile < 3 || (long long)(ntile / 2 + 1) * BH > 20000) return false;
  thread_local int c_ntile = -1, c_bh = -1, c_dev = -1;
  thread_local bool c_val = false;
  int dev = 0, P = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (ntile == c_ntile && BH == c_bh && dev == c_dev) return c_val;
  if (cudaDeviceGetAttribute(&P, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || P <= 0) return false;
  const int nfull = ntile / 2;
  c_val = attn_makespan(nfull, BH, P, true) < 0.97 * attn_makespan(nfull, BH, P, false);
  c_ntile = ntile;
  c_bh = BH;
  c_dev = dev;
  return c_val;
}

template <int KD, int OUT>
int launch_attn(dim3 grid, const CUtensorMap& mqk, const CUtensorMap& mv, void* o, float* lse, int N, int Np,
                int nh, float sl2, cudaStream_t st) {
  static PerDeviceOnce attr;  // the shared-memory limit is per device
  if (int rc = attr.run([] { return set_smem(attn_kernel<KD, OUT>, sizeof(AttnSmem<KD>) + 1024); })) return rc;
  const int ntile = (N + kTile - 1) / kTile;
  if (attn_odd_last(ntile, (int)grid.y)) {
    const dim3 g1((ntile / 2) * grid.y + grid.y);
    attn_kernel<KD, OUT><<<g1, kAttnThreads, sizeof(AttnSmem<KD>) + 1024, st>>>(mqk, mv, o, lse, N, Np, nh, sl2,
                                                                                (int)grid.y);
    return check_launch("flash attention");
  }
  attn_kernel<KD, OUT><<<grid, kAttnThreads, sizeof(AttnSmem<KD>) + 1024, st>>>(mqk, mv, o, lse, N, Np, nh, sl2, 0);
  return check_launch("flash attention");
}

}  // namespace

// The register-window PE kernel (no shared-memory plane, any image size) takes
// rows of 4 or 8 columns; otherwise the plane-staging kernel runs, which
// holds (H + 2) · pitch floats of a channel in shared memory (kMaxPlane).
bool pe_vec_supported(int B, int C, int H, int W) {
  const int cw = (W & 7) == 0 ? 8 : (W & 3) == 0 ? 4 : 0;
  return cw && (long long)B * C * ((H + kPevRows - 1) / kPevRows) * (W / cw) < (1LL << 31);
}

int pe_dwconv_vec(const __half* v, const __nv_bfloat16* w_pe, const float* b_pe, __half* pe,
                  const __nv_bfloat16* w_proj, __half* wproj16, int B, int C, int H, int W, int Np,
                  const __half* add, cudaStream_t st) {
  const int cw = (W & 7) == 0 ? 8 : (W & 3) == 0 ? 4 : 0;
  const long long blocks = cw ? (long long)B * C * ((H + kPevRows - 1) / kPevRows) * (W / cw) : 0;
  if (!pe_vec_supported(B, C, H, W)) return VA_ERR_UNSUPPORTED;
  const unsigned grid = (unsigned)((blocks + kPevThreads - 1) / kPevThreads);
  if (cw == 8)
    pe_dwconv_vec_kernel<8><<<grid, kPevThreads, 0, st>>>(v, w_pe, b_pe, pe, w_proj, wproj16, B, H, W, Np, C, add);
  else
    pe_dwconv_vec_kernel<4><<<grid, kPevThreads, 0, st>>>(v, w_pe, b_pe, pe, w_proj, wproj16, B, H, W, Np, C, add);
  return check_launch("psa pe");
}

size_t psa_tc_workspace_bytes(int B, int C, int H, int W, int nh) {
  return psa_tc_is_n(C, nh, kKD) ? tc_layout(B, H, W, nh).total : psa_tc_wide_workspace_bytes(B, C, H, W);
}

PsaTcOffsets psa_tc_offsets(int B, int H, int W, int nh) {
  const TcWs L = tc_layout(B, H, W, nh);
  return PsaTcOffsets{L.qk, L.v, L.o, L.pe, L.wproj, L.total};
}

bool psa_tc_supported(int C, int nh, int kd) { return kd == kKD && nh >= 1 && C == nh * kHD; }

// Side streams of one device for the fork/joins inside the library's ops:
// the critical chain (the fused op's attention, the training step's attention
// backward) on the highest stream priority, independent side work (PE, the
// projection's weight gradients) on the lowest, so the block scheduler places
// side blocks only on SMs that no critical block is waiting for — such as
// the tail of the attention grid.  Created once per device.
namespace {
SideStreams g_side[64];
PerDeviceOnce g_side_once;
}  // namespace

int psa_side_streams(SideStreams** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "psa: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) {  // no side streams kept for such devices: the caller runs serially
    *out = nullptr;
    return VA_OK;
  }
  const int rc = g_side_once.run([dev]() -> int {
    int lo = 0, hi = 0;
    if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess ||
        cudaStreamCreateWithPriority(&g_side[dev].hi, cudaStreamNonBlocking, hi) != cudaSuccess ||
        cudaStreamCreateWithPriority(&g_side[dev].lo, cudaStreamNonBlocking, lo) != cudaSuccess) {
      cudaGetLastError();
      return set_error(VA_ERR_LAUNCH, "psa: side stream creation failed");
    }
    return VA_OK;
  });
  if (rc) return rc;
  *out = &g_side[dev];
  return VA_OK;
}

// Records an event on `from` and makes `to` wait for it (the event is
// released at once; CUDA keeps it until the wait is resolved).
int psa_stream_dep(cudaStream_t from, cudaStream_t to) {
  cudaEvent_t e;
  cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  if (r == cudaSuccess) {
    r = cudaEventRecord(e, from);
    if (r == cudaSuccess) r = cudaStreamWaitEvent(to, e, 0);
    cudaEventDestroy(e);
  }
  if (r != cudaSuccess) return set_error(VA_ERR_LAUNCH, "psa: stream dependency: %s", cudaGetErrorString(r));
  return VA_OK;
}

int psa_attention_fwd_tc(const __nv_bfloat16* x, const __nv_bfloat16* w_qkv, const float* b_qkv,
                         const __nv_bfloat16* w_pe, const float* b_pe, const __nv_bfloat16* w_proj,
                         const float* b_proj, __nv_bfloat16* y, int B, int C, int H, int W, int nh, int kd,
                         void* ws, size_t ws_bytes, cudaStream_t st, float* lse_out, bool overlap_pe) {
  VA_CHECK_ARG(psa_tc_supported(C, nh, kd), "psa_attention bf16: tensor-core path needs key_dim 32 and C = 64·num_heads");
  if (!psa_tc_is_n(C, nh, kd))
    return psa_attention_fwd_tc_wide(x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, y, B, C, H, W, nh, ws, ws_bytes, st);
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0 && B <= 65535, "psa_attention bf16: bad sizes");
  VA_CHECK_ARG(pe_vec_supported(B, kC, H, W) || (H + 2) * ((W + 10) | 1) <= kMaxPlane,
               "psa_attention bf16: image %dx%d with W %% 4 != 0 larger than the PE plane staging supports", H, W);
  const TcWs L = tc_layout(B, H, W, nh);
  if (!ws || ws_bytes < L.total)
    return set_error(VA_ERR_WORKSPACE, "psa_attention bf16: workspace %zu < %zu bytes", ws_bytes, L.total);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w_qkv) & 15) || (reinterpret_cast<uintptr_t>(w_proj) & 15))
    return set_error(VA_ERR_ALIGN, "psa_attention bf16: x/w_qkv/w_proj need 16-byte, workspace 256-byte alignment");
  const int N = H * W, Np = (N + 7) / 8 * 8, BH = B * nh;
  char* base = static_cast<char*>(ws);
  __half* qk = reinterpret_cast<__half*>(base + L.qk);
  __half* vb = reinterpret_cast<__half*>(base + L.v);
  __half* ob = reinterpret_cast<__half*>(base + L.o);
  const __nv_bfloat16* xs = x;
  if (N % 8) {
    __nv_bfloat16* xp = reinterpret_cast<__nv_bfloat16*>(base + L.xpad);
    const long long total = (long long)B * kC * Np;
    pad_rows_kernel<<<(int)std::min<long long>((total + 255) / 256, 148LL * 8), 256, 0, st>>>(x, xp, B * kC, N, Np);
    if (int rc = check_launch("psa pad")) return rc;
    xs = xp;
  }
  CUtensorMap mx, mw, mqk, mv, mvst;
  {
    uint64_t d[2] = {(uint64_t)N, (uint64_t)B * kC}, s[1] = {(uint64_t)Np * 2};
    uint32_t bx[2] = {64, kC};
    if (int rc = make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xs, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "x"))
      return rc;
  }
  {
    uint64_t d[2] = {(uint64_t)kC, (uint64_t)kQKV}, s[1] = {(uint64_t)kC * 2};
    uint32_t bx[2] = {64, 64};  // 64-row boxes: the kernel regroups W_qkv's rows on load
    if (int rc = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w_qkv, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B,
                          "w_qkv"))
      return rc;
  }
  {
    uint64_t d[3] = {(uint64_t)kKD, (uint64_t)N, (uint64_t)2 * BH}, s[2] = {(uint64_t)kKD * 2, (uint64_t)N * kKD * 2};
    uint32_t bx[3] = {kKD, kTile, 1};
    if (int rc = make_map(&mqk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, qk, d, s, bx, CU_TENSOR_MAP_SWIZZLE_64B, "qk"))
      return rc;
  }
  {
    uint64_t d[2] = {(uint64_t)N, (uint64_t)B * kC}, s[1] = {(uint64_t)Np * 2};
    uint32_t bx[2] = {64, kHD};
    if (int rc = make_map(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, vb, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "v"))
      return rc;
  }
  {
    // V store: [B·C rows][Np] f16 in SW128 boxes of 64 tokens × 128 channels; inner
    // extent N, so a tile's columns past N are not written
    uint64_t d[2] = {(uint64_t)N, (uint64_t)B * kC}, s[1] = {(uint64_t)Np * 2};
    uint32_t bx[2] = {64, kC};
    if (int rc = make_map(&mvst, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, vb, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "v store"))
      return rc;
  }
  const int ntile = (N + kTile - 1) / kTile;
  const size_t sm1 = sizeof(QkvSmem) + 1024, sm2 = sizeof(AttnSmem<kKD>) + 1024, sm4 = sizeof(ProjSmem) + 1024;
  const size_t sm3 = (size_t)kPeCh * (H + 2) * ((W + 10) | 1) * sizeof(float);
  static PerDeviceOnce attrs;  // the shared-memory limits are per device
  if (int rc = attrs.run([&] {
        if (int r = set_smem(qkv_proj_kernel, sm1)) return r;
        if (int r = set_smem(attn_kernel<kKD, kOutChannelMajor>, sm2)) return r;
        if (int r = set_smem(pe_dwconv_kernel, (size_t)kPeCh * kMaxPlane * sizeof(float))) return r;
        if (int r = set_smem(proj_kernel, sm4)) return r;
        return set_smem(proj_pers_kernel, sizeof(ProjPSmem) + 1024);
      }))
    return rc;
  __half* peb = reinterpret_cast<__half*>(base + L.pe);
  __half* wp16 = reinterpret_cast<__half*>(base + L.wproj);
  CUtensorMap mo, mpe, mwp;
  {
    uint64_t d[2] = {(uint64_t)N, (uint64_t)B * kC}, s[1] = {(uint64_t)Np * 2};
    uint32_t bx[2] = {64, kC};
    if (int rc = make_map(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ob, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "o"))
      return rc;
    if (int rc = make_map(&mpe, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, peb, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "pe"))
      return rc;
  }
  {
    uint64_t d[2] = {(uint64_t)kC, (uint64_t)kC}, s[1] = {(uint64_t)kC * 2};
    uint32_t bx[2] = {64, kC};
    if (int rc = make_map(&mwp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, wp16, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B,
                          "w_proj"))
      return rc;
  }
  qkv_proj_kernel<<<std::min(B * ntile, 148), kQpThreads, sm1, st>>>(mx, mw, mvst, b_qkv, qk, N, nh, B, ntile);
  if (int rc = check_launch("psa qkv_proj")) return rc;
  const float scale_log2 = (1.0f / sqrtf((float)kd)) * 1.4426950408889634f;
  // overlap_pe: attention and PE (both read only V and Q/K) run on the side
  // streams after the qkv GEMM and join before the projection
  SideStreams* side = nullptr;
  if (overlap_pe) {
    if (int rc = psa_side_streams(&side)) return rc;
    if (side) {
      if (int rc = psa_stream_dep(st, side->hi)) return rc;
      if (int rc = psa_stream_dep(st, side->lo)) return rc;
    }
  }
  SideJoin joiner{side, st};
  const cudaStream_t sa = side ? side->hi : st, sp = side ? side->lo : st;
  if (int rc = launch_attn<kKD, kOutChannelMajor>(dim3((ntile + 1) / 2, BH), mqk, mv, ob, lse_out, N, Np, nh,
                                                  scale_log2, sa))
    return rc;
  const int pe_rc = pe_dwconv_vec(vb, w_pe, b_pe, peb, w_proj, wp16, B, kC, H, W, Np, nullptr, sp);
  if (pe_rc == VA_ERR_UNSUPPORTED) {
    pe_dwconv_kernel<<<dim3(kC / kPeCh, B), kPeThreads, sm3, sp>>>(vb, w_pe, b_pe, peb, w_proj, wp16, H, W, Np);
    if (int rc = check_launch("psa pe")) return rc;
  } else if (pe_rc) {
    return pe_rc;
  }
  if (int rc = joiner.join()) return rc;
  if (N % 8 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    CUtensorMap my;
    uint64_t d[2] = {(uint64_t)N, (uint64_t)B * kC}, s[1] = {(uint64_t)N * 2};
    uint32_t bx[2] = {64, kC};
    if (int rc = make_map(&my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "y"))
      return rc;
    proj_pers_kernel<<<std::min(B * ntile, 148), kPpThreads, sizeof(ProjPSmem) + 1024, st>>>(mo, mpe, mwp, my,
                                                                                              b_proj, B, ntile);
  } else {
    proj_kernel<<<dim3(ntile, B), 128, sm4, st>>>(mo, mpe, mwp, b_proj, y, N);
  }
  return check_launch("psa proj");
}

int tc_status_read(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_tc_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status read: %s", cudaGetErrorString(e));
  return VA_OK;
}

int tc_status_clear(cudaStream_t st) {
  static const int zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_tc_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "device status clear: %s", cudaGetErrorString(e));
  return VA_OK;
}

}  // namespace va

namespace va {

int tc_flash_attention(const void* qk, const void* v, void* o, float* lse, int BH, int nh, int N, int kd,
                       int out_token_major, cudaStream_t st, float scale) {
  VA_CHECK_ARG(kd == 32 || kd == 64, "flash attention: key dim %d (32 or 64)", kd);
  VA_CHECK_ARG(BH > 0 && nh > 0 && BH % nh == 0 && N > 0 && BH <= 65535, "flash attention: bad sizes");
  if ((reinterpret_cast<uintptr_t>(qk) & 15) || (reinterpret_cast<uintptr_t>(v) & 15) ||
      (reinterpret_cast<uintptr_t>(o) & 15))
    return set_error(VA_ERR_ALIGN, "flash attention: qk/v/o need 16-byte alignment");
  const int Np = (N + 7) / 8 * 8;
  CUtensorMap mqk, mv;
  {
    uint64_t d[3] = {(uint64_t)kd, (uint64_t)N, (uint64_t)2 * BH}, s[2] = {(uint64_t)kd * 2, (uint64_t)N * kd * 2};
    uint32_t bx[3] = {(uint32_t)kd, kTile, 1};
    if (int rc = make_map(&mqk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, qk, d, s, bx,
                          kd == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, "qk"))
      return rc;
  }
  {
    // inner extent N (not Np): the pad columns of a row read as zeros
    uint64_t d[2] = {(uint64_t)N, (uint64_t)BH * kHD}, s[1] = {(uint64_t)Np * 2};
    uint32_t bx[2] = {64, kHD};
    if (int rc = make_map(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, v, d, s, bx, CU_TENSOR_MAP_SWIZZLE_128B, "v"))
      return rc;
  }
  const float scale_log2 = (scale > 0.0f ? scale : 1.0f / sqrtf((float)kd)) * 1.4426950408889634f;
  if (N <= kTile) {  // one key tile per sequence: persistent short-sequence kernel
    const int ctas = std::min((BH + 1) / 2, 148);
    auto launch_short = [&](auto kernel, size_t smem) -> int {
      if (int rc = set_smem(kernel, smem)) return rc;
      kernel<<<ctas, kShortThreads, smem, st>>>(mqk, mv, o, lse, N, Np, nh, BH, scale_log2);
      return check_launch("short-sequence attention");
    };
    if (kd == 32)
      return out_token_major ? launch_short(attn_short_kernel<32, kOutTokenMajor>, sizeof(ShortSmem<32>) + 1024)
                             : launch_short(attn_short_kernel<32, kOutChannelMajor>, sizeof(ShortSmem<32>) + 1024);
    return out_token_major ? launch_short(attn_short_kernel<64, kOutTokenMajor>, sizeof(ShortSmem<64>) + 1024)
                           : launch_short(attn_short_kernel<64, kOutChannelMajor>, sizeof(ShortSmem<64>) + 1024);
  }
  const dim3 grid(((N + kTile - 1) / kTile + 1) / 2, BH);
  if (kd == 32)
    return out_token_major
               ? launch_attn<32, kOutTokenMajor>(grid, mqk, mv, o, lse, N, Np, nh, scale_log2, st)
               : launch_attn<32, kOutChannelMajor>(grid, mqk, mv, o, lse, N, Np, nh, scale_log2, st);
  return out_token_major ? launch_attn<64, kOutTokenMajor>(grid, mqk, mv, o, lse, N, Np, nh, scale_log2, st)
                         : launch_attn<64, kOutChannelMajor>(grid, mqk, mv, o, lse, N, Np, nh, scale_log2, st);
}

int psa_attention_core_tc(const void* qk, const void* v, void* o, float* lse, int B, int nh, int H, int W,
                          cudaStream_t st) {
  VA_CHECK_ARG(nh >= 1 && B > 0 && H > 0 && W > 0 && (long long)B * nh <= 65535, "psa flash attention: bad sizes");
  return tc_flash_attention(qk, v, o, lse, B * nh, nh, H * W, kKD, 0, st);
}

}  // namespace va
