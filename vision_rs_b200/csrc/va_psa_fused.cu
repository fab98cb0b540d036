// Fused PSA Attention forward (the graph of src/models/yolo/yolo26/blocks/
// c2psa.rs:61-116 with BN folded):
//   qkv = conv1x1(x)+b → pack → FA(V_lo), FA(V_hi) → merge
//   v = extract_v(qkv) → pe = dw3x3(v)+b → y = conv1x1(merged + pe)+b
//
// f32: the reference's node sequence on the FFMA kernels, intermediates in the
// caller's workspace.  bf16: the tensor-core path in va_tc_psa.cu.
#include "va_common.cuh"
#include "va_psa.h"

extern "C" {
int va_psa_pack_qkv_backward_f32(const float*, float*, int, int, int, int, int, va_stream_t);
int va_psa_extract_v_backward_f32(const float*, float*, int, int, int, int, int, int, va_stream_t);
int va_psa_merge_attn_backward_f32(const float*, float*, float*, int, int, int, int, int, va_stream_t);
int va_psa_fa2_backward_f32(const float*, const float*, const float*, const float*, const float*, const float*,
                            float*, float*, float*, int, float, int, int, va_stream_t);
int va_dwconv3x3_backward_f32(const float*, const float*, const float*, float*, float*, int, int, int, int,
                              va_stream_t);
int va_psa_pack_qkv_f32(const float*, float*, int, int, int, int, int, va_stream_t);
int va_psa_pack_qkv_bf16(const va_bf16*, va_bf16*, int, int, int, int, int, va_stream_t);
int va_psa_extract_v_nchw_f32(const float*, float*, int, int, int, int, int, int, va_stream_t);
int va_psa_extract_v_nchw_bf16(const va_bf16*, va_bf16*, int, int, int, int, int, int, va_stream_t);
int va_psa_merge_attn_nchw_f32(const float*, const float*, float*, int, int, int, int, int, va_stream_t);
int va_psa_merge_attn_nchw_bf16(const va_bf16*, const va_bf16*, va_bf16*, int, int, int, int, int, va_stream_t);
}

namespace va {

namespace {
struct PsaWs {
  size_t qkv, packed, lo, hi, merged, v, pe, lse, total;
};

PsaWs layout(int B, int C, int H, int W, int nh, int kd, size_t esz) {
  const size_t N = (size_t)H * W, qkv_h = (size_t)nh * 4 * kd, BH = (size_t)B * nh;
  PsaWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  w.qkv = take(B * qkv_h * N * esz);
  w.packed = take(4 * BH * N * kd * esz);
  w.lo = take(BH * N * kd * esz);
  w.hi = take(BH * N * kd * esz);
  w.merged = take((size_t)B * C * N * esz);
  w.v = take((size_t)B * C * N * esz);
  w.pe = take((size_t)B * C * N * esz);
  w.lse = take(BH * N * sizeof(float));
  w.total = off;
  return w;
}

int check_common(int B, int C, int H, int W, int nh, int kd, void* ws, size_t ws_bytes, size_t need) {
  VA_CHECK_ARG(B > 0 && C > 0 && H > 0 && W > 0 && nh > 0 && kd > 0, "psa_attention: non-positive size");
  VA_CHECK_ARG(C == nh * 2 * kd, "psa_attention: need C = num_heads*2*key_dim (C=%d nh=%d kd=%d)", C, nh, kd);
  if (!ws || ws_bytes < need)
    return set_error(VA_ERR_WORKSPACE, "psa_attention: workspace %zu bytes < required %zu", ws_bytes, need);
  return VA_OK;
}
}  // namespace

size_t psa_workspace_bytes(int B, int C, int H, int W, int nh, int kd, int dtype) {
  if (dtype == 0) return layout(B, C, H, W, nh, kd, 4).total;
  return psa_tc_supported(C, nh, kd) ? psa_tc_workspace_bytes(B, C, H, W, nh) : 0;
}

#define VA_TRY(expr)          \
  do {                        \
    int _rc = (expr);         \
    if (_rc) return _rc;      \
  } while (0)

namespace {
// The forward node sequence on the FFMA kernels, intermediates at L's offsets
// in ws; y (the projection) only when y != nullptr.
int fwd_f32_nodes(const PsaWs& L, const float* x, const float* w_qkv, const float* b_qkv, const float* w_pe,
                  const float* b_pe, const float* w_proj, const float* b_proj, float* y, int B, int C, int H, int W,
                  int nh, int kd, void* ws, cudaStream_t st) {
  char* base = (char*)ws;
  float* qkv = (float*)(base + L.qkv);
  float* packed = (float*)(base + L.packed);
  float* lo = (float*)(base + L.lo);
  float* hi = (float*)(base + L.hi);
  float* merged = (float*)(base + L.merged);
  float* v = (float*)(base + L.v);
  float* pe = (float*)(base + L.pe);
  float* lse = (float*)(base + L.lse);
  const int N = H * W, qkv_h = nh * 4 * kd, BH = B * nh;
  const size_t sec = (size_t)BH * N * kd;
  const float scale = 1.0f / sqrtf((float)kd);  // psa.rs:986
  va_stream_t s = (va_stream_t)st;
  VA_TRY((conv1x1<float, float>(x, nullptr, w_qkv, b_qkv, qkv, B, C, qkv_h, N, st)));
  VA_TRY(va_psa_pack_qkv_f32(qkv, packed, qkv_h, H, W, B, nh, s));
  VA_TRY(fa_fwd_f32(packed, packed + sec, packed + 2 * sec, lo, lse, N, N, scale, BH, kd, st));
  VA_TRY(fa_fwd_f32(packed, packed + sec, packed + 3 * sec, hi, lse, N, N, scale, BH, kd, st));
  VA_TRY(va_psa_merge_attn_nchw_f32(lo, hi, merged, C, H, W, nh, B, s));
  VA_TRY(va_psa_extract_v_nchw_f32(qkv, v, qkv_h, C, H, W, nh, B, s));
  VA_TRY((dwconv3x3<float, float>(v, w_pe, b_pe, pe, B, C, H, W, st)));
  if (y) VA_TRY((conv1x1<float, float>(merged, pe, w_proj, b_proj, y, B, C, C, N, st)));
  return VA_OK;
}

// Backward buffers after the forward's: dS (= ∂L/∂(merged + pe)), d_lo, d_hi,
// d_packed, dV from the PE conv, d_qkv, and the transposed 1×1 weights.
struct BwdWs {
  PsaWs f;
  size_t ds, dlo, dhi, dpacked, dvpe, dqkv, wprojt, wqkvt, total;
};

BwdWs bwd_layout(int B, int C, int H, int W, int nh, int kd) {
  BwdWs w;
  w.f = layout(B, C, H, W, nh, kd, 4);
  const size_t N = (size_t)H * W, qkv_h = (size_t)nh * 4 * kd, BH = (size_t)B * nh;
  size_t off = w.f.total;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  w.ds = take((size_t)B * C * N * 4);
  w.dlo = take(BH * N * kd * 4);
  w.dhi = take(BH * N * kd * 4);
  w.dpacked = take(4 * BH * N * kd * 4);
  w.dvpe = take((size_t)B * C * N * 4);
  w.dqkv = take(B * qkv_h * N * 4);
  w.wprojt = take((size_t)C * C * 4);
  w.wqkvt = take(qkv_h * C * 4);
  w.total = off;
  return w;
}
}  // namespace

int psa_attention_fwd_f32(const float* x, const float* w_qkv, const float* b_qkv, const float* w_pe,
                          const float* b_pe, const float* w_proj, const float* b_proj, float* y, int B, int C,
                          int H, int W, int nh, int kd, void* ws, size_t ws_bytes, cudaStream_t st) {
  const PsaWs L = layout(B, C, H, W, nh, kd, 4);
  VA_TRY(check_common(B, C, H, W, nh, kd, ws, ws_bytes, L.total));
  return fwd_f32_nodes(L, x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, y, B, C, H, W, nh, kd, ws, st);
}

size_t psa_bwd_f32_workspace_bytes(int B, int C, int H, int W, int nh, int kd) {
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || nh <= 0 || kd <= 0) return 0;
  return bwd_layout(B, C, H, W, nh, kd).total;
}

// Backward of the f32 op for an upstream gradient dy = ∂L/∂y: the forward
// recomputed, then the reference graph's backward nodes in order — proj conv
// (dW, db, dS = W_projᵀ·dy), PE dw-conv (dV_pe, dW_pe; db_pe = Σ dS),
// psa_merge_attn backward (d_lo, d_hi = dS split), psa_fa2_backward for the
// V_lo and V_hi calls (dq, dk accumulated, dv stored; psa.rs:650-725,
// 1039-1042), psa_pack_qkv and psa_extract_v backwards (accumulating into
// d_qkv; psa.rs:201-281), and the qkv conv (dW, db, dx = W_qkvᵀ·d_qkv).
// grads: [w_qkv | w_proj | w_pe | b_qkv | b_proj | b_pe], stored.
int psa_attention_bwd_f32(const float* x, const float* dy, const float* w_qkv, const float* b_qkv,
                          const float* w_pe, const float* b_pe, const float* w_proj, const float* b_proj, float* dx,
                          float* grads, int B, int C, int H, int W, int nh, int kd, void* ws, size_t ws_bytes,
                          cudaStream_t st) {
  VA_CHECK_ARG(x && dy && w_qkv && b_qkv && w_pe && b_pe && w_proj && b_proj && grads,
               "psa_attention backward f32: null input, weight or grads pointer");
  const BwdWs L = bwd_layout(B, C, H, W, nh, kd);
  VA_TRY(check_common(B, C, H, W, nh, kd, ws, ws_bytes, L.total));
  VA_TRY(fwd_f32_nodes(L.f, x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, nullptr, B, C, H, W, nh, kd, ws, st));
  char* base = (char*)ws;
  auto at = [&](size_t o) { return (float*)(base + o); };
  const float *qkv = at(L.f.qkv), *packed = at(L.f.packed), *lo = at(L.f.lo), *hi = at(L.f.hi),
              *merged = at(L.f.merged), *v = at(L.f.v), *pe = at(L.f.pe), *lse = at(L.f.lse);
  (void)qkv;
  float *ds = at(L.ds), *dlo = at(L.dlo), *dhi = at(L.dhi), *dpacked = at(L.dpacked), *dvpe = at(L.dvpe),
        *dqkv = at(L.dqkv), *wprojt = at(L.wprojt), *wqkvt = at(L.wqkvt);
  const int N = H * W, qkv_h = nh * 4 * kd, BH = B * nh;
  const size_t sec = (size_t)BH * N * kd;
  const float scale = 1.0f / sqrtf((float)kd);
  va_stream_t s = (va_stream_t)st;
  float* g_wqkv = grads;
  float* g_wproj = g_wqkv + (size_t)qkv_h * C;
  float* g_wpe = g_wproj + (size_t)C * C;
  float* g_bqkv = g_wpe + (size_t)C * 9;
  float* g_bproj = g_bqkv + qkv_h;
  float* g_bpe = g_bproj + C;
  // accumulation targets of the backward nodes start at zero
  cudaError_t e = cudaMemsetAsync(dpacked, 0, 4 * sec * sizeof(float), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(dqkv, 0, (size_t)B * qkv_h * N * sizeof(float), st);
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "psa_attention backward f32: memset: %s", cudaGetErrorString(e));
  // proj: y = W_proj·(merged + pe) + b_proj
  VA_TRY(transpose_f32(w_proj, wprojt, C, C, st));
  VA_TRY(conv1x1_dw_f32(dy, merged, pe, g_wproj, B, C, C, N, st));
  VA_TRY(channel_sum_f32(dy, g_bproj, B, C, N, st));
  VA_TRY((conv1x1<float, float>(dy, nullptr, wprojt, nullptr, ds, B, C, C, N, st)));
  // pe = dw3x3(v) + b_pe
  VA_TRY(va_dwconv3x3_backward_f32(v, w_pe, ds, dvpe, g_wpe, B, C, H, W, s));
  VA_TRY(channel_sum_f32(ds, g_bpe, B, C, N, st));
  // merged = merge(lo, hi); lo/hi = FA(q, k, V_lo / V_hi)
  VA_TRY(va_psa_merge_attn_backward_f32(ds, dlo, dhi, C, H, W, nh, B, s));
  VA_TRY(va_psa_fa2_backward_f32(packed, packed + sec, packed + 2 * sec, lo, dlo, lse, dpacked, dpacked + sec,
                                 dpacked + 2 * sec, N, scale, BH, kd, s));
  VA_TRY(va_psa_fa2_backward_f32(packed, packed + sec, packed + 3 * sec, hi, dhi, lse, dpacked, dpacked + sec,
                                 dpacked + 3 * sec, N, scale, BH, kd, s));
  // packed = pack(qkv), v = extract_v(qkv)
  VA_TRY(va_psa_pack_qkv_backward_f32(dpacked, dqkv, qkv_h, H, W, B, nh, s));
  VA_TRY(va_psa_extract_v_backward_f32(dvpe, dqkv, qkv_h, C, H, W, nh, B, s));
  // qkv = W_qkv·x + b_qkv
  VA_TRY(conv1x1_dw_f32(dqkv, x, nullptr, g_wqkv, B, C, qkv_h, N, st));
  VA_TRY(channel_sum_f32(dqkv, g_bqkv, B, qkv_h, N, st));
  if (dx) {
    VA_TRY(transpose_f32(w_qkv, wqkvt, qkv_h, C, st));
    VA_TRY((conv1x1<float, float>(dqkv, nullptr, wqkvt, nullptr, dx, B, qkv_h, C, N, st)));
  }
  return VA_OK;
}

int psa_attention_fwd_bf16(const __nv_bfloat16* x, const __nv_bfloat16* w_qkv, const float* b_qkv,
                           const __nv_bfloat16* w_pe, const float* b_pe, const __nv_bfloat16* w_proj,
                           const float* b_proj, __nv_bfloat16* y, int B, int C, int H, int W, int nh, int kd,
                           void* ws, size_t ws_bytes, cudaStream_t st) {
  return psa_attention_fwd_tc(x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, y, B, C, H, W, nh, kd, ws, ws_bytes, st,
                              nullptr, /*overlap_pe=*/true);
}

}  // namespace va
