// Internal declarations shared between the visionattn translation units.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace va {

size_t psa_workspace_bytes(int B, int C, int H, int W, int nh, int kd, int dtype);
size_t psa_bwd_f32_workspace_bytes(int B, int C, int H, int W, int nh, int kd);
int psa_attention_bwd_f32(const float* x, const float* dy, const float* w_qkv, const float* b_qkv,
                          const float* w_pe, const float* b_pe, const float* w_proj, const float* b_proj, float* dx,
                          float* grads, int B, int C, int H, int W, int nh, int kd, void* ws, size_t ws_bytes,
                          cudaStream_t st);

int psa_attention_fwd_f32(const float* x, const float* w_qkv, const float* b_qkv, const float* w_pe,
                          const float* b_pe, const float* w_proj, const float* b_proj, float* y, int B, int C,
                          int H, int W, int nh, int kd, void* ws, size_t ws_bytes, cudaStream_t st);

int psa_attention_fwd_bf16(const __nv_bfloat16* x, const __nv_bfloat16* w_qkv, const float* b_qkv,
                           const __nv_bfloat16* w_pe, const float* b_pe, const __nv_bfloat16* w_proj,
                           const float* b_proj, __nv_bfloat16* y, int B, int C, int H, int W, int nh, int kd,
                           void* ws, size_t ws_bytes, cudaStream_t st);

int fa_fwd_f32(const float* q, const float* k, const float* v, float* o, float* l, int nq, int nk, float scale,
               int bh, int hd, cudaStream_t st);
int fa_fwd_bf16(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, __nv_bfloat16* o,
                float* l, int nq, int nk, float scale, int bh, int hd, cudaStream_t st);

template <typename T, typename TW>
int conv1x1(const T* x, const T* x2, const TW* w, const float* bias, T* y, int B, int cin, int cout, int HW,
            cudaStream_t st);
template <typename T, typename TW>
int dwconv3x3(const T* x, const TW* w, const float* bias, T* y, int B, int C, int H, int W, cudaStream_t st);
// f32 1×1-conv backward pieces (va_conv.cu): dW = Σ dY·(X + X2)ᵀ, db = Σ dY
// (both stored, fixed-order reductions), and a weight transpose.
int conv1x1_dw_f32(const float* dy, const float* x, const float* x2, float* dw, int B, int cin, int cout, int HW,
                   cudaStream_t st);
int channel_sum_f32(const float* dy, float* db, int B, int C, int HW, cudaStream_t st);
int transpose_f32(const float* w, float* wt, int rows, int cols, cudaStream_t st);

// Workspace of the tensor-core forward (bf16): the specialised C = 128 path
// or, for other widths C = 64·nh, the general one (va_tc_psa_wide.cu).
size_t psa_tc_workspace_bytes(int B, int C, int H, int W, int nh);
size_t psa_tc_wide_workspace_bytes(int B, int C, int H, int W);
// PE = dw3×3(V) + b_pe (+ add, when given) for V f16 [B·C][Np] with rows of W
// (W % 4 == 0; VA_ERR_UNSUPPORTED otherwise, nothing launched), and W_proj
// [C][C] to f16 on the side.
int pe_dwconv_vec(const __half* v, const __nv_bfloat16* w_pe, const float* b_pe, __half* pe,
                  const __nv_bfloat16* w_proj, __half* wproj16, int B, int C, int H, int W, int Np,
                  const __half* add, cudaStream_t st);
int psa_attention_fwd_tc_wide(const __nv_bfloat16* x, const __nv_bfloat16* w_qkv, const float* b_qkv,
                              const __nv_bfloat16* w_pe, const float* b_pe, const __nv_bfloat16* w_proj,
                              const float* b_proj, __nv_bfloat16* y, int B, int C, int H, int W, int nh, void* ws,
                              size_t ws_bytes, cudaStream_t st);
// Byte offsets of the tensor-core forward's intermediates inside its
// workspace: Q/K f16 [2][B·nh][N][32], V, O and PE f16 [B][128][Np], W_proj
// as f16 [128][128].
struct PsaTcOffsets {
  size_t qk, v, o, pe, wproj, total;
};
PsaTcOffsets psa_tc_offsets(int B, int H, int W, int nh);

// One operand of tc_gemm_f16 (f16 or bf16 elements): K-major — row r (an M or N
// index) holds K contiguous elements, `ld` apart; MN-major — row k holds the
// M (or N) elements contiguously.  batch_stride: elements between batch
// entries; broadcast: one matrix for every batch entry.
struct GemmOperand {
  const void* ptr;
  bool mn;
  long long ld;
  long long batch_stride;
  bool broadcast;
};
// C[z'][m][n] = α·Σ_{z in fold z'} Σ_k A_z(m,k)·B_z(n,k) + bias[m], f32
// accumulation; z' = z / zfold (ceil(Z/zfold) outputs); C is f32 (c_type 0),
// bf16 (1) or f16 (2) with row pitch ldc and batch stride c_batch (elements).
// Operands are f16, or bf16 with ab_bf16; bias (f32 [M]) is optional;
// epi adds SiLU and a residual.
// Optional epilogue of tc_gemm_f16: SiLU after the bias, then + res[z][m][n]
// (res_type 0 f32, 1 bf16, 2 f16; row pitch ldr, batch stride r_batch).
struct GemmEpilogue {
  bool silu = false;
  const void* res = nullptr;
  int res_type = 0;
  long long ldr = 0, r_batch = 0;
};
int tc_gemm_f16(const GemmOperand& a, const GemmOperand& b, void* c, int c_type, long long ldc, long long c_batch,
                int M, int N, int K, int Z, cudaStream_t st, float alpha = 1.0f, int zfold = 1,
                const float* bias = nullptr, bool ab_bf16 = false, const GemmEpilogue& epi = GemmEpilogue());
int gemm_status_read(int* out, cudaStream_t st);
// Tensor-core PSA attention backward (nh = 2, kd = 32, N ≤ 512), channel-major
// f32 outputs: dk [B·nh][32][N], dv [B·nh][64][N], dq_part
// [ceil(N/128)][B·nh][32][N] (sum over the first index = dQ).  qk, v, o, d_o
// in the forward's f16 layouts; delta: f32 [B·nh][N] scratch.
int psa_attn_bwd_tc(const void* qk, const void* v, const void* o, const void* d_o, const float* lse, float* delta,
                    float* dk, float* dv, float* dq_part, int B, int nh, int N, cudaStream_t st);
int bwd_status_read(int* out, cudaStream_t st);
int bwd_status_clear(cudaStream_t st);
int gemm_status_clear(cudaStream_t st);
// Status word of the implicit-GEMM convolution kernel (va_conv_nhwc.cu).
int conv_status_read(int* out, cudaStream_t st);
int conv_status_clear(cudaStream_t st);
// Tensor-core forward: any C = 64·nh with key dim 32 (the c2psa widths);
// the C = 128 kernels of the training step: psa_tc_is_n.
bool psa_tc_supported(int C, int nh, int kd);
inline bool psa_tc_is_n(int C, int nh, int kd) { return C == 128 && nh == 2 && kd == 32; }
// Per-device side streams of the library (highest / lowest stream priority),
// created by the first call on a device (*out = nullptr, run serially, on a
// device index ≥ 64); psa_stream_dep(from, to) makes `to` wait for the work
// issued on `from` so far (an event per call).
struct SideStreams {
  cudaStream_t hi = nullptr, lo = nullptr;
};
int psa_side_streams(SideStreams** out);
int psa_stream_dep(cudaStream_t from, cudaStream_t to);
// Joins both side streams back into `st` once: by join(), or when it goes out
// of scope (an early error return), so no library work is left unordered
// against the caller's stream.
struct SideJoin {
  SideStreams* side;
  cudaStream_t st;
  bool done = false;
  int join() {
    done = true;
    if (!side) return 0;
    const int a = psa_stream_dep(side->hi, st), b = psa_stream_dep(side->lo, st);
    return a ? a : b;
  }
  ~SideJoin() {
    if (!done) join();
  }
};
// overlap_pe (C = 128): attention and PE on the library's per-device side
// streams (highest / lowest priority), forked from and joined back to `st`.
int psa_attention_fwd_tc(const __nv_bfloat16* x, const __nv_bfloat16* w_qkv, const float* b_qkv,
                         const __nv_bfloat16* w_pe, const float* b_pe, const __nv_bfloat16* w_proj,
                         const float* b_proj, __nv_bfloat16* y, int B, int C, int H, int W, int nh, int kd,
                         void* ws, size_t ws_bytes, cudaStream_t st, float* lse_out, bool overlap_pe = false);
// Tensor-core flash attention over BH = sequences·nh heads of N tokens:
// qk f16 [2][BH][N][kd] (Q then K), v f16 [BH·64][Np] (Np = N rounded up to 8),
// head dim 64, kd ∈ {32, 64}; o f16 [BH/nh][nh·64][Np] (channel-major) or,
// with out_token_major, bf16 [BH/nh][N][nh·64]; lse (optional) f32 [BH][N].
// scale: softmax scale (0 → 1/√kd).
int tc_flash_attention(const void* qk, const void* v, void* o, float* lse, int BH, int nh, int N, int kd,
                       int out_token_major, cudaStream_t st, float scale = 0.0f);
int psa_attention_core_tc(const void* qk, const void* v, void* o, float* lse, int B, int nh, int H, int W,
                          cudaStream_t st);
int tc_status_read(int* out, cudaStream_t st);
int tc_status_clear(cudaStream_t st);
int dino_status_read(int* out, cudaStream_t st);
int dino_status_clear(cudaStream_t st);

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace va
