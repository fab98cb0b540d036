// C-ABI plumbing: error reporting, shape inference (the reference's
// CustomOp::infer_output_shape), BN folding, workspace sizing and the fused
// PSA Attention forward entry points.
#include <math.h>
#include <stdarg.h>
#include <string.h>

#include <atomic>

#include "va_common.cuh"
#include "va_psa.h"

namespace va {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_err[0] = 0; }

static std::atomic<unsigned long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace va

using namespace va;

extern "C" {

int va_version(void) { return 100; }

const char* va_get_last_error_string(void) { return g_err; }

uint64_t va_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

// psa.rs:766-776
int va_psa_pack_qkv_infer_output_shape(const int64_t* in, int rank, int num_heads, int64_t* out) {
  if (rank != 4 || num_heads <= 0) return -1;
  out[0] = in[0];
  out[1] = 4;
  out[2] = num_heads;
  out[3] = (in[2] < 0 || in[3] < 0) ? -1 : in[2] * in[3];
  out[4] = in[1] < 0 ? -1 : in[1] / (num_heads * 4);
  return 5;
}

// psa.rs:809-812
int va_psa_extract_v_infer_output_shape(const int64_t* in, int rank, int64_t* out) {
  if (rank != 4) return -1;
  out[0] = in[0];
  out[1] = in[1] < 0 ? -1 : in[1] / 2;
  out[2] = in[2];
  out[3] = in[3];
  return 4;
}

// psa.rs:853-863
int va_psa_merge_attn_infer_output_shape(const int64_t* in, int rank, int num_heads, int64_t H, int64_t W,
                                         int64_t* out) {
  if (rank != 4 || num_heads <= 0) return -1;
  out[0] = in[0];
  out[1] = in[3] < 0 ? -1 : num_heads * 2 * in[3];
  out[2] = H;
  out[3] = W;
  return 4;
}

// psa.rs:901-905
int va_flash_attention2_infer_output_shape(const int64_t* in, int rank, int64_t* out) {
  if (rank != 5) return -1;
  out[0] = in[0];
  out[1] = in[2];
  out[2] = in[3];
  out[3] = in[4];
  return 4;
}

int va_fold_bn_f32(const float* w, const float* gamma, const float* beta, const float* mean, const float* var,
                   float eps, int c_out, int k_per_out, float* w_out, float* b_out) {
  if (!w || !gamma || !beta || !mean || !var || !w_out || !b_out || c_out <= 0 || k_per_out <= 0)
    return set_error(VA_ERR_SHAPE, "fold_bn: null pointer or non-positive size");
  for (int o = 0; o < c_out; ++o) {
    double s = (double)gamma[o] / sqrt((double)var[o] + (double)eps);
    for (int i = 0; i < k_per_out; ++i) w_out[(size_t)o * k_per_out + i] = (float)(w[(size_t)o * k_per_out + i] * s);
    b_out[o] = (float)((double)beta[o] - (double)mean[o] * s);
  }
  return VA_OK;
}

size_t va_psa_attention_workspace_bytes(int B, int C, int H, int W, int num_heads, int key_dim, int dtype) {
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || num_heads <= 0 || key_dim <= 0) return 0;
  return psa_workspace_bytes(B, C, H, W, num_heads, key_dim, dtype);
}

int va_psa_attention_fwd_f32(const float* x, const float* w_qkv, const float* b_qkv, const float* w_pe,
                             const float* b_pe, const float* w_proj, const float* b_proj, float* y, int B, int C,
                             int H, int W, int num_heads, int key_dim, void* ws, size_t ws_bytes, va_stream_t s) {
  return psa_attention_fwd_f32(x, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, y, B, C, H, W, num_heads, key_dim, ws,
                               ws_bytes, (cudaStream_t)s);
}

size_t va_psa_attention_bwd_f32_workspace_bytes(int B, int C, int H, int W, int num_heads, int key_dim) {
  return psa_bwd_f32_workspace_bytes(B, C, H, W, num_heads, key_dim);
}

int va_psa_attention_bwd_f32(const float* x, const float* dy, const float* w_qkv, const float* b_qkv,
                             const float* w_pe, const float* b_pe, const float* w_proj, const float* b_proj,
                             float* dx, float* grads, int B, int C, int H, int W, int num_heads, int key_dim,
                             void* ws, size_t ws_bytes, va_stream_t s) {
  return psa_attention_bwd_f32(x, dy, w_qkv, b_qkv, w_pe, b_pe, w_proj, b_proj, dx, grads, B, C, H, W, num_heads,
                               key_dim, ws, ws_bytes, (cudaStream_t)s);
}

int va_psa_attention_fwd_bf16(const va_bf16* x, const va_bf16* w_qkv, const float* b_qkv, const va_bf16* w_pe,
                              const float* b_pe, const va_bf16* w_proj, const float* b_proj, va_bf16* y, int B,
                              int C, int H, int W, int num_heads, int key_dim, void* ws, size_t ws_bytes,
                              va_stream_t s) {
  return psa_attention_fwd_bf16((const __nv_bfloat16*)x, (const __nv_bfloat16*)w_qkv, b_qkv,
                                (const __nv_bfloat16*)w_pe, b_pe, (const __nv_bfloat16*)w_proj, b_proj,
                                (__nv_bfloat16*)y, B, C, H, W, num_heads, key_dim, ws, ws_bytes, (cudaStream_t)s);
}

int va_psa_flash_attention_fwd_f16(const void* qk, const void* v, void* o, float* lse, int B, int nh, int H, int W,
                                   va_stream_t s) {
  return psa_attention_core_tc(qk, v, o, lse, B, nh, H, W, (cudaStream_t)s);
}

int va_device_status_read(int* status, va_stream_t s) {  // first non-zero word of the tensor-core kernels
  if (!status) return set_error(VA_ERR_SHAPE, "device_status_read: null output");
  int v[5] = {0, 0, 0, 0, 0};
  if (int rc = tc_status_read(&v[0], (cudaStream_t)s)) return rc;
  if (int rc = dino_status_read(&v[1], (cudaStream_t)s)) return rc;
  if (int rc = gemm_status_read(&v[2], (cudaStream_t)s)) return rc;
  if (int rc = bwd_status_read(&v[3], (cudaStream_t)s)) return rc;
  if (int rc = conv_status_read(&v[4], (cudaStream_t)s)) return rc;
  *status = 0;
  for (int i = 0; i < 5 && !*status; ++i) *status = v[i];
  return VA_OK;
}

int va_device_status_clear(va_stream_t s) {
  if (int rc = tc_status_clear((cudaStream_t)s)) return rc;
  if (int rc = dino_status_clear((cudaStream_t)s)) return rc;
  if (int rc = gemm_status_clear((cudaStream_t)s)) return rc;
  if (int rc = conv_status_clear((cudaStream_t)s)) return rc;
  return bwd_status_clear((cudaStream_t)s);
}

}  // extern "C"
