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

int psa_attention_fwd_f32(const float* x, const float* w_qkv, const float* b_qkv, const float* w_pe,
                          const float* b_pe, const float* w_proj, const float* b_proj, float* y, int B, int C,
                          int H, int W, int nh, int kd, void* ws, size_t ws_bytes, cudaStream_t st) {
  const PsaWs L = layout(B, C, H, W, nh, kd, 4);
  VA_TRY(check_common(B, C, H, W, nh, kd, ws, ws_bytes, L.total));
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
  VA_TRY((conv1x1<float, float>(merged, pe, w_proj, b_proj, y, B, C, C, N, st)));
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
