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

constexpr int kCvM = 128, kCvTW = 16, kCvTH = 8, kCvMaxStages = 32;
constexpr int kCvEpiWarps = 8, kCvThreads = 64 + 32 * kCvEpiWarps;  // producer, MMA, 8 epilogue warps
constexpr int kCvAcc = 4;  // TMEM accumulator buffers (4 × BN ≤ 512 columns)
// 3×3 stride 2: the even input rows 2·oy0 − 1 … 2·oy0 + 15 (9 rows, taps ky = 0 and 2) and the odd
// rows 2·oy0 … 2·oy0 + 16 (9 rows loaded, 8 used, tap ky = 1), 16 strided columns each
constexpr int kHalo2Rows = 9 * kCvTW;

// Barriers and bookkeeping behind the operand ring in dynamic shared memory.
struct ConvCtl {
  uint64_t full[kCvMaxStages], empty[kCvMaxStages];  // operand ring
  uint64_t acc_full[kCvAcc], acc_empty[kCvAcc];      // rotating TMEM accumulators
  uint64_t wfull;                                    // resident weights landed
  uint64_t done;
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

// Geometry of one launch.  linear: a 1×1 stride-1 conv is a plain GEMM over
// the B·H·W pixels, so a tile is 128 consecutive pixels (x is then a 2-D map
// [pixels][Cin]); otherwise a tile is 8 output rows × 16 output columns of
// one image (x a 4-D map, the im2col done by the load's coordinates).
struct ConvGeom {
  int Ho, Wo, Cin, Cout, ksize, stride, act, linear;
  int tiles_w, tiles_h, n_tiles, total_tiles, stages;
  int wres;          // the CTA's whole weight slice [BN][k·k·Cin] stays in shared memory
  int th;            // subtiles per tile: 1, or 2 / 4 (stacked 8-row subtiles) in stride-1 halo mode
  int halo;          // 1: 3×3 stride 1, one (8·th + 2)-row halo load per (channel block, kx) serves every
                     //    subtile and ky = 0, 1, 2;
                     // 2: 3×3 stride 2, an even-row and an odd-row load per (channel block, kx)
  long long pixels;  // B·Ho·Wo
};

// Columns an epilogue warp drains per TMEM read: the whole tile up to 64, else 64 at a time.
template <int BN>
struct ConvCols {
  static constexpr int chunk = BN < 64 ? BN : 64;
};

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* m, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// Tile t → (image, first output row, first output column or first pixel, first channel).
__device__ __forceinline__ void conv_tile(const ConvGeom& g, int t, int bn, int& b, int& oy0, int& ox0, long long& m0,
                                          int& n0) {
  n0 = (t % g.n_tiles) * bn;
  int r = t / g.n_tiles;
  if (g.linear) {
    m0 = (long long)r * kCvM * g.th;
    b = oy0 = ox0 = 0;
    return;
  }
  ox0 = (r % g.tiles_w) * kCvTW;
  r /= g.tiles_w;
  oy0 = (r % g.tiles_h) * (kCvTH * g.th);
  b = r / g.tiles_h;
  m0 = 0;
}

// Persistent, warp-specialised: warp 0 streams operands through the ring with
// TMA, warp 1 issues the MMAs into one of four rotating TMEM accumulators,
// warps 2-9 drain finished accumulators (bias, SiLU, bf16, NHWC stores), so
// the epilogues of earlier tiles overlap the main loop of later ones.  One
// CTA per SM (the launch asks for more than half the shared memory).
// When the CTA's weight slice fits (wres), it is loaded once and only the
// activation tiles stream through the ring; the grid is then a multiple of
// the channel-tile count, so a CTA keeps one channel tile for all its tiles.
template <int KB, int BN>
__global__ void __launch_bounds__(kCvThreads, 1)
conv_nhwc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                 const __grid_constant__ CUtensorMap map_y, const float* __restrict__ bias,
                 __nv_bfloat16* __restrict__ y, const ConvGeom g) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int kABytes = kCvM * KB * 2, kBBytes = BN * KB * 2;
  constexpr int kChunk = ConvCols<BN>::chunk, kRowBytes = 2 * kChunk;
  constexpr uint32_t kTmemCols = 512;  // 4 accumulator slots × th subtiles × BN columns ≤ 512 (one CTA per SM)
  // [staging: 8 warps × 2 × 32 rows × kRowBytes][A ring][B ring or resident slice][barriers]
  uint8_t* stg = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = stg + kCvEpiWarps * 2 * 32 * kRowBytes;
  // A stage: 128 pixel rows, or in halo mode 160 rows (10 input rows × 16 columns).
  const int aBytes = g.halo == 1 ? (kCvTH * g.th + 2) * kCvTW * KB * 2
                   : g.halo == 2 ? 2 * kHalo2Rows * KB * 2 : kABytes * g.th;
  uint8_t* sb = sa + g.stages * aBytes;  // weight ring, or the resident slice
  const int pad = g.ksize / 2, cblocks = (g.Cin + KB - 1) / KB, nk = g.ksize * g.ksize * cblocks;
  const int nq = g.halo ? 3 * cblocks : nk;  // ring stages per tile
  ConvCtl& c = *reinterpret_cast<ConvCtl*>(sb + (g.wres ? nk : g.stages) * kBBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = g.stages;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], 1);
    }
    for (int i = 0; i < kCvAcc; ++i) {
      mbar_init(&c.acc_full[i], 1);
      mbar_init(&c.acc_empty[i], g.th == 1 ? 4 : 8);  // the epilogue warps that drain it
    }
    mbar_init(&c.done, 1);
    mbar_init(&c.wfull, 1);
    c.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&c.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = c.tmem_base;

  if (warp == 0) {  // ── TMA producer ──
    if (lane == 0) {
      tma_prefetch_desc(&map_x);
      tma_prefetch_desc(&map_w);
      tma_prefetch_desc(&map_y);
      long long q = 0;      // operand ring slots filled so far (across tiles)
      int st = 0;           // = q % S, kept incrementally: no 64-bit division per stage
      uint32_t ph = 0;      // = (q / S) & 1
      bool ok = true;
      if (g.wres && (int)blockIdx.x < g.total_tiles) {
        const int n0 = ((int)blockIdx.x % g.n_tiles) * BN;
        mbar_arrive_expect_tx(&c.wfull, nk * kBBytes);
        for (int kb = 0; kb < nk; ++kb) {
          const int tap = kb / cblocks, c0 = (kb - tap * cblocks) * KB;
          tma_load_2d(sb + kb * kBBytes, &map_w, &c.wfull, tap * g.Cin + c0, n0);
        }
      }
      for (int t = blockIdx.x; t < g.total_tiles && ok; t += gridDim.x) {
        int b, oy0, ox0, n0;
        long long m0;
        conv_tile(g, t, BN, b, oy0, ox0, m0, n0);
        for (int kb = 0; kb < nq; ++kb, ++q, st = st + 1 == S ? 0 : st + 1, ph ^= st == 0 ? 1u : 0u) {
          if (q >= S && !(ok = mbar_wait(&c.empty[st], ph ^ 1u, &c.abort, &g_conv_status, 1))) break;
          if (g.halo == 1) {  // stage kb = (channel block kb / 3, kx = kb % 3): input rows oy0 − 1 … oy0 + 8
            const int cb = kb / 3, kx = kb - 3 * cb;
            mbar_arrive_expect_tx(&c.full[st], aBytes);
            tma_load_4d(sa + st * aBytes, &map_x, &c.full[st], cb * KB, ox0 + kx - 1, oy0 - 1, b);
            continue;
          }
          if (g.halo == 2) {  // even rows from 2·oy0 − 1, odd rows from 2·oy0 (element stride 2 in y and x)
            const int cb = kb / 3, kx = kb - 3 * cb;
            mbar_arrive_expect_tx(&c.full[st], aBytes);
            uint8_t* dst = sa + st * aBytes;
            tma_load_4d(dst, &map_x, &c.full[st], cb * KB, 2 * ox0 + kx - 1, 2 * oy0 - 1, b);
            tma_load_4d(dst + kHalo2Rows * KB * 2, &map_x, &c.full[st], cb * KB, 2 * ox0 + kx - 1, 2 * oy0, b);
            continue;
          }
          const int tap = kb / cblocks, c0 = (kb - tap * cblocks) * KB, ky = tap / g.ksize, kx = tap - ky * g.ksize;
          mbar_arrive_expect_tx(&c.full[st], g.wres ? aBytes : aBytes + kBBytes);
          if (g.linear)  // th·128 consecutive pixels
            tma_load_2d(sa + st * aBytes, &map_x, &c.full[st], c0, (int)m0);
          else
            tma_load_4d(sa + st * aBytes, &map_x, &c.full[st], c0, g.stride * ox0 + kx - pad,
                        g.stride * oy0 + ky - pad, b);
          if (!g.wres) tma_load_2d(sb + st * kBBytes, &map_w, &c.full[st], tap * g.Cin + c0, n0);
        }
      }
      if (!ok) {  // every load issued here lands (bounded) before the CTA can exit
        for (long long k = q - S < 0 ? 0 : q - S; k < q; ++k) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&c.full[k % S], (uint32_t)((k / S) & 1)) && clock64() - t0 < kSpinCycles) {
          }
        }
        if (g.wres) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&c.wfull, 0) && clock64() - t0 < kSpinCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {  // ── MMA issuer ──
    // The whole warp runs the loop converged (waits made warp-uniform) and one
    // elected lane issues each tcgen05.mma / commit: a lone diverged lane
    // issues these small MMAs markedly slower.
    constexpr uint32_t idesc = idesc_f32acc(kCvM, BN, AB_BF16, false, false);
    const uint64_t da0 = sdesc(smem_u32(sa), 16, KbTraits<KB>::sbo, KbTraits<KB>::swz);
    const uint64_t db0 = sdesc(smem_u32(sb), 16, KbTraits<KB>::sbo, KbTraits<KB>::swz);
    int st = 0;       // ring slot, = (stages consumed) % S
    uint32_t ph = 0;  // its fill parity
    bool ok = true;
    if (g.wres && (int)blockIdx.x < g.total_tiles)
      ok = __all_sync(0xffffffffu, mbar_wait(&c.wfull, 0, &c.abort, &g_conv_status, 5));
    int i = 0;
    for (int t = blockIdx.x; t < g.total_tiles && ok; t += gridDim.x, ++i) {
      const int buf = i % kCvAcc, use = i / kCvAcc;
      if (use > 0 &&
          !(ok = __all_sync(0xffffffffu,
                            mbar_wait(&c.acc_empty[buf], (uint32_t)((use - 1) & 1), &c.abort, &g_conv_status, 2))))
        break;
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(buf * g.th * BN);
      for (int kb = 0; kb < nq; ++kb, st = st + 1 == S ? 0 : st + 1, ph ^= st == 0 ? 1u : 0u) {
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&c.full[st], ph, &c.abort, &g_conv_status, 3)))) break;
        tc_fence_after();
        const uint64_t da = da0 + (uint64_t)((st * aBytes) >> 4);
        if (g.halo) {
          // Stride 1: output row r of tap (ky, kx) reads halo row r + 16·ky.
          // Stride 2: ky = 0 → even rows from row 0, ky = 2 → even rows from
          // row 16, ky = 1 → the odd rows (144 rows in).  Every start is a
          // whole number of swizzle atoms.
          const int cb = kb / 3, kx = kb - 3 * cb;
          for (int sub = 0; sub < g.th; ++sub) {  // subtile sub: output rows 8·sub … 8·sub + 7 of the tile
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
              const int row0 = g.halo == 1 ? 16 * (8 * sub + ky) : ky == 1 ? kHalo2Rows : 8 * ky;
              const uint64_t dak = da + (uint64_t)((row0 * KB * 2) >> 4);
              const uint64_t db = db0 + (uint64_t)((((ky * 3 + kx) * cblocks + cb) * kBBytes) >> 4);
#pragma unroll
              for (int s = 0; s < KB / 16; ++s)
                mma_ss_w(d + (uint32_t)(sub * BN), dak + 2 * s, db + 2 * s, idesc,
                         (kb > 0 || ky > 0 || s > 0) ? 1u : 0u);
            }
          }
          mma_commit_w(&c.empty[st]);
          continue;
        }
        const uint64_t db = db0 + (uint64_t)(((g.wres ? kb : st) * kBBytes) >> 4);
        for (int sub = 0; sub < g.th; ++sub) {  // linear mode: subtile sub = pixels 128·sub … of the tile
          const uint64_t das = da + (uint64_t)((sub * kABytes) >> 4);
#pragma unroll
          for (int s = 0; s < KB / 16; ++s)  // +32 bytes per 16-channel k-step inside the swizzle atom
            mma_ss_w(d + (uint32_t)(sub * BN), das + 2 * s, db + 2 * s, idesc, (kb > 0 || s > 0) ? 1u : 0u);
        }
        mma_commit_w(&c.empty[st]);
      }
      if (ok) mma_commit_w(&c.acc_full[buf]);
    }
    // Nothing issued here may still be writing TMEM when it is freed.
    mma_commit_w(&c.done);
    const long long t0 = clock64();
    while (!mbar_try_wait(&c.done, 0) && clock64() - t0 < kSpinCycles) {
    }
  } else {
    // ── epilogue: two groups of four warps (2-5, 6-9).  With one subtile per
    // tile they drain alternate tiles, so two accumulators are read out at
    // once; with th subtiles group e drains subtiles e, e + 2, … of every tile.
    // Warp w reads TMEM lane quarter w % 4 (32 pixel rows of a subtile) and all
    // BN columns, kChunk at a time.
    const int quarter = warp & 3, grp = (warp - 2) >> 2, ew = warp - 2;
    const bool alt = g.th == 1;  // alternate tiles between the groups
    // Swizzled row of this lane in the staging tile: 16-byte chunk j lands at
    // chunk j ^ sw, the pattern TMA applies for a kRowBytes-wide swizzle.
    const int sw = ((lane * kRowBytes) >> 7) & (kRowBytes / 16 - 1);
    int nstore = 0;  // staging buffer use count of this warp
    for (int i = alt ? grp : 0;; i += alt ? 2 : 1) {
      const long long tl = (long long)blockIdx.x + (long long)i * gridDim.x;
      if (tl >= g.total_tiles) break;
      const int t = (int)tl, buf = i % kCvAcc, use = i / kCvAcc;
      int b, oy0t, ox0, n0;
      long long m0;
      conv_tile(g, t, BN, b, oy0t, ox0, m0, n0);
      const bool got = mbar_wait(&c.acc_full[buf], (uint32_t)(use & 1), &c.abort, &g_conv_status, 4);
      if (!__all_sync(0xffffffffu, got)) break;  // warp-uniform: the TMEM loads below are warp-collective
      tc_fence_after();
      const int sub0 = alt ? 0 : grp, sstep = alt ? 1 : 2;
#pragma unroll 1
      for (int sub = sub0; sub < g.th; sub += sstep)
#pragma unroll 1
      for (int cb = 0; cb < BN; cb += kChunk) {
        const int oy0 = oy0t + kCvTH * sub;  // first output row of this subtile
        const int nv = g.Cout - n0 - cb;  // live channels of this chunk (multiple of 8)
        float bv[kChunk];
#pragma unroll
        for (int k = 0; k < kChunk; ++k) bv[k] = k < nv ? __ldg(bias + n0 + cb + k) : 0.0f;
        uint32_t u[kChunk];
        const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)((buf * g.th + sub) * BN + cb);
#pragma unroll
        for (int cc = 0; cc < kChunk; cc += 16) tmem_ld16(ta + cc, *reinterpret_cast<uint32_t(*)[16]>(u + cc));
        tmem_ld_wait();
        reg_fence(u);
        if (cb + kChunk >= BN && sub + sstep >= g.th) {  // this warp's last read of the accumulator
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&c.acc_empty[buf]);
        }
        uint4 outv[kRowBytes / 16];  // this lane's pixel: kChunk channels of bf16
#pragma unroll
        for (int j = 0; j < kRowBytes / 16; ++j) {
          uint32_t q4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = 8 * j + 2 * e;
            float v0 = __uint_as_float(u[k]) + bv[k], v1 = __uint_as_float(u[k + 1]) + bv[k + 1];
            if (g.act) {  // SiLU; → −0 once exp overflows
              v0 = __fdividef(v0, 1.0f + __expf(-v0));
              v1 = __fdividef(v1, 1.0f + __expf(-v1));
            }
            q4[e] = pack_bf16x2(v0, v1);
          }
          outv[j] = make_uint4(q4[0], q4[1], q4[2], q4[3]);
        }
        if constexpr (kRowBytes >= 64) {  // staged in shared memory, written by a TMA store
          uint8_t* stage = stg + (ew * 2 + (nstore & 1)) * (32 * kRowBytes);
          ++nstore;
          if (lane == 0) tma_store_wait_read_1();  // this staging buffer's previous store has read it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < kRowBytes / 16; ++j)
            *reinterpret_cast<uint4*>(stage + lane * kRowBytes + ((j ^ sw) << 4)) = outv[j];
          fence_proxy_async_smem();  // the staging writes become visible to the TMA store
          __syncwarp();
          if (lane == 0) {  // 32 rows × kChunk channels; TMA drops what lies outside y
            if (g.linear)
              tma_store_2d(&map_y, stage, n0 + cb, (int)(m0 + kCvM * sub + quarter * 32));
            else
              tma_store_4d(&map_y, stage, n0 + cb, ox0, oy0 + 2 * quarter, b);
            tma_store_commit();
          }
        } else {  // rows of 32 bytes: plain stores from registers beat a TMA store of narrow rows
          const int r = quarter * 32 + lane;
          long long pix;
          bool live;
          if (g.linear) {
            pix = m0 + kCvM * sub + r;
            live = pix < g.pixels;
          } else {
            const int oy = oy0 + r / kCvTW, ox = ox0 + r % kCvTW;
            live = oy < g.Ho && ox < g.Wo;
            pix = ((long long)b * g.Ho + oy) * g.Wo + ox;
          }
          if (live) {
            uint4* o = reinterpret_cast<uint4*>(y + pix * g.Cout + n0 + cb);
#pragma unroll
            for (int j = 0; j < kRowBytes / 16; ++j)
              if (8 * j < nv) o[j] = outv[j];
          }
        }
      }
    }
    if (lane == 0) tma_store_wait_all();
  }
  __syncwarp();  // lanes 1-31 of the producer and MMA warps rejoin lane 0
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

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

int conv_nhwc(const __nv_bfloat16* x, const __nv_bfloat16* w, const float* bias, __nv_bfloat16* y, int B, int H, int W,
              int Cin, int Cout, int k, int s, int act, cudaStream_t st) {
  VA_CHECK_ARG(x && w && bias && y, "conv nhwc: null pointer");
  VA_CHECK_ARG(B > 0 && H > 0 && W > 0, "conv nhwc: bad sizes");
  VA_CHECK_ARG(k == 1 || k == 3, "conv nhwc: kernel size %d (1 or 3)", k);
  VA_CHECK_ARG(s == 1 || s == 2, "conv nhwc: stride %d (1 or 2)", s);
  VA_CHECK_ARG(Cin > 0 && Cin % 8 == 0, "conv nhwc: Cin=%d must be a multiple of 8", Cin);
  VA_CHECK_ARG(Cout > 0 && Cout % 8 == 0, "conv nhwc: Cout=%d must be a multiple of 8", Cout);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15)
    return set_error(VA_ERR_ALIGN, "conv nhwc: x, w, y need 16-byte alignment");
  const int pad = k / 2, Ho = (H + 2 * pad - k) / s + 1, Wo = (W + 2 * pad - k) / s + 1;
  // Channel block: 64 from 40 input channels up, 32 from 24 (the blocks past
  // C_in read zeros); fewer, wider pipeline stages beat exact-fitting narrow ones.
  const int KB = Cin >= 40 ? 64 : Cin >= 24 ? 32 : 16;
  const int BN = Cout % 128 == 0 ? 128 : Cout % 64 == 0 ? 64 : Cout % 32 == 0 ? 32 : 16;
  ConvGeom g{};
  g.Ho = Ho, g.Wo = Wo, g.Cin = Cin, g.Cout = Cout, g.ksize = k, g.stride = s, g.act = act ? 1 : 0;
  g.linear = (k == 1 && s == 1) ? 1 : 0;
  g.pixels = (long long)B * Ho * Wo;
  g.n_tiles = (Cout + BN - 1) / BN;
  g.tiles_w = (Wo + kCvTW - 1) / kCvTW;
  g.th = 1;  // set below for the stride-1 halo mode
  g.tiles_h = (Ho + kCvTH - 1) / kCvTH;
  const long long tiles = g.linear ? (g.pixels + kCvM - 1) / kCvM * g.n_tiles
                                   : (long long)g.tiles_w * g.tiles_h * B * g.n_tiles;
  VA_CHECK_ARG(g.pixels < (1LL << 31) && tiles < (1LL << 31), "conv nhwc: %lld output pixels is too many", g.pixels);
  g.total_tiles = (int)tiles;
  const int nk = k * k * ((Cin + KB - 1) / KB), a_bytes = kCvM * KB * 2, b_bytes = BN * KB * 2;
  const int sms = sm_count();
  // Resident weight slice when it leaves room for the activation ring.
  g.wres = (nk * b_bytes <= 96 * 1024 && g.n_tiles <= sms) ? 1 : 0;
  const int chunk_cols = BN < 64 ? BN : 64, stg_bytes = kCvEpiWarps * 2 * 32 * 2 * chunk_cols;
  g.halo = (k == 3 && g.wres) ? s : 0;
  if (g.linear && BN <= 64 && g.pixels >= 2 * kCvM) {
    // 1×1: two 128-pixel subtiles per tile (one 256-row load, two accumulators)
    g.th = 2;
    g.total_tiles = (int)((g.pixels + 2 * kCvM - 1) / (2 * kCvM) * g.n_tiles);
  }
  if (g.halo == 1) {
    // Narrow convs: stack 2 or 4 subtiles per tile so that each pipeline stage
    // (one halo load, th·3 MMAs) carries more work; 4 slots × th × BN ≤ 512 TMEM
    // columns, and no taller than the map needs.
    g.th = BN <= 16 ? 4 : BN <= 32 ? 2 : 1;
    while (g.th > 1 && kCvTH * g.th / 2 >= Ho) g.th /= 2;
    g.tiles_h = (Ho + kCvTH * g.th - 1) / (kCvTH * g.th);
    const long long t2 = (long long)g.tiles_w * g.tiles_h * B * g.n_tiles;
    g.total_tiles = (int)t2;
  }
  const int ring_budget = 200 * 1024 - stg_bytes - (g.wres ? nk * b_bytes : 0);
  const int stage_bytes = g.halo == 1 ? (kCvTH * g.th + 2) * kCvTW * KB * 2 : g.halo == 2 ? 2 * kHalo2Rows * KB * 2
                        : g.wres ? a_bytes * g.th : a_bytes * g.th + b_bytes;
  g.stages = std::max(2, std::min(kCvMaxStages, ring_budget / stage_bytes));
  auto fn = conv_encode_fn();
  if (!fn) return set_error(VA_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap mx, mw, my;
  CUresult r;
  if (g.linear) {
    const uint64_t d[2] = {(uint64_t)Cin, (uint64_t)g.pixels};
    const uint64_t str[1] = {(uint64_t)Cin * 2};
    const uint32_t box[2] = {(uint32_t)KB, (uint32_t)(kCvM * g.th)}, es[2] = {1, 1};
    r = fn(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(x), d, str, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, tma_swizzle(KB), CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    const uint64_t d[4] = {(uint64_t)Cin, (uint64_t)W, (uint64_t)H, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)Cin * 2, (uint64_t)W * Cin * 2, (uint64_t)H * W * Cin * 2};
    const uint32_t box[4] = {(uint32_t)KB, (uint32_t)(kCvTW * s),
                             (uint32_t)(g.halo == 1 ? kCvTH * g.th + 2 : g.halo == 2 ? 18 : kCvTH * s), 1};
    const uint32_t es[4] = {1, (uint32_t)s, (uint32_t)s, 1};
    r = fn(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<__nv_bfloat16*>(x), d, str, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, tma_swizzle(KB), CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "conv nhwc: tensor map for x rejected (CUresult %d)", (int)r);
  {
    const uint64_t d[2] = {(uint64_t)k * k * Cin, (uint64_t)Cout};
    const uint64_t str[1] = {(uint64_t)k * k * Cin * 2};
    const uint32_t box[2] = {(uint32_t)KB, (uint32_t)BN}, es[2] = {1, 1};
    r = fn(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(w), d, str, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, tma_swizzle(KB), CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "conv nhwc: tensor map for w rejected (CUresult %d)", (int)r);
  }
  // With resident weights a CTA keeps one channel tile: the grid is a multiple of n_tiles.
  {  // y: tiles of 32 output rows × chunk_cols channels, stored from the staging buffers
    const CUtensorMapSwizzle swz = tma_swizzle(chunk_cols);
    if (g.linear) {
      const uint64_t d[2] = {(uint64_t)Cout, (uint64_t)g.pixels};
      const uint64_t str[1] = {(uint64_t)Cout * 2};
      const uint32_t box[2] = {(uint32_t)chunk_cols, 32}, es[2] = {1, 1};
      r = fn(&my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, d, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
      const uint64_t d[4] = {(uint64_t)Cout, (uint64_t)Wo, (uint64_t)Ho, (uint64_t)B};
      const uint64_t str[3] = {(uint64_t)Cout * 2, (uint64_t)Wo * Cout * 2, (uint64_t)Ho * Wo * Cout * 2};
      const uint32_t box[4] = {(uint32_t)chunk_cols, (uint32_t)kCvTW, 2, 1}, es[4] = {1, 1, 1, 1};
      r = fn(&my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, y, d, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return set_error(VA_ERR_ALIGN, "conv nhwc: tensor map for y rejected (CUresult %d)", (int)r);
  }
  const int grid = std::min(g.total_tiles, g.wres ? sms / g.n_tiles * g.n_tiles : sms);
  // At least 116 KB so that two CTAs never share an SM (each holds 4·BN TMEM columns).
  const size_t smem = std::max<size_t>(
      116 * 1024,
      1024 + (size_t)stg_bytes + (size_t)g.stages * stage_bytes + (g.wres ? (size_t)nk * b_bytes : 0) + sizeof(ConvCtl));
  int rc = VA_ERR_UNSUPPORTED;
  auto launch = [&](auto kb, auto bn) {
    constexpr int KB_ = decltype(kb)::value, BN_ = decltype(bn)::value;
    auto kernel = conv_nhwc_kernel<KB_, BN_>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      rc = set_error(VA_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return;
    }
    kernel<<<grid, kCvThreads, smem, st>>>(mx, mw, my, bias, y, g);
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
