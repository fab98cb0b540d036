/*
 * visionattn.h — C ABI of the B200-native (sm_100a) attention hot path of
 * spinorml/vision-rs.
 *
 * Drop-in boundary.  In the reference every hot-path node is a teenygrad
 * `RuntimeOp` whose `pack_args` pushes kernel arguments through an
 * `ArgVisitor` and whose `grid()` derives the launch size from the output
 * shape (src/models/yolo/kernels/attention/psa.rs).  Each entry point below
 * takes exactly the pointer/int/float arguments that `pack_args` pushes, in
 * the same order, followed by the sizes that the reference's `grid()` reads
 * from the output shape (batch, head count, head dim), followed by the
 * stream.  A Rust `RuntimeOp` shim therefore replaces
 * `visitor.visit_*(…); launch(grid, block)` by a single call here.
 *
 * Conventions (all entry points):
 *   - device pointers only; the library never allocates, frees or
 *     synchronises inside these calls, and every launch goes on `stream`;
 *   - return 0 (VA_OK) or a VA_ERR_* code; `va_get_last_error_string()`
 *     describes the last failure on the calling thread;
 *   - bf16 tensors are passed as raw 16-bit words (`va_bf16`);
 *   - "accumulates" means `+=` into caller-zeroed memory, as the reference's
 *     backward kernels do with `atomic_add` (psa.rs:232, :279-280, :700, :723).
 */
#ifndef VISIONATTN_H
#define VISIONATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VA_API __attribute__((visibility("default")))
#else
#define VA_API
#endif

typedef uint16_t va_bf16;
typedef struct CUstream_st *va_stream_t;

enum {
  VA_OK = 0,
  VA_ERR_SHAPE = 1,       /* unsupported or inconsistent sizes */
  VA_ERR_LAUNCH = 2,      /* CUDA launch / runtime error */
  VA_ERR_TIMEOUT = 3,     /* a bounded device-side wait gave up */
  VA_ERR_ALIGN = 4,       /* pointer alignment the kernel needs is not met */
  VA_ERR_UNSUPPORTED = 5, /* device or configuration not supported */
  VA_ERR_WORKSPACE = 6,   /* workspace missing or too small */
  VA_ERR_NCCL = 7         /* collective failed or timed out */
};

/* Library identity and diagnostics. */
VA_API int va_version(void);
VA_API const char *va_get_last_error_string(void);
/* Number of kernels this library has launched in this process (all threads). */
VA_API uint64_t va_launch_count(void);

/* ── Shape inference (CustomOp::infer_output_shape). -1 = dynamic dim. ─────
 * Return the output rank, or -1 on a bad input rank. */
/* psa.rs:766-776 — [B,qkv_h,H,W] → [B,4,nh,N,kd] */
VA_API int va_psa_pack_qkv_infer_output_shape(const int64_t *in, int rank, int num_heads, int64_t *out);
/* psa.rs:809-812 — [B,qkv_h,H,W] → [B,qkv_h/2,H,W] */
VA_API int va_psa_extract_v_infer_output_shape(const int64_t *in, int rank, int64_t *out);
/* psa.rs:853-863 — [B,nh,N,kd] → [B,nh*2*kd,H,W] (H, W fixed at construction) */
VA_API int va_psa_merge_attn_infer_output_shape(const int64_t *in, int rank, int num_heads, int64_t H,
                                         int64_t W, int64_t *out);
/* psa.rs:901-905 — [B,4,nh,N,kd] → [B,nh,N,kd] */
VA_API int va_flash_attention2_infer_output_shape(const int64_t *in, int rank, int64_t *out);

/* ── PSA layout kernels ───────────────────────────────────────────────────── */
/* psa_pack_qkv (psa.rs:58-94; args psa.rs:371-377):
 * NCHW [B,qkv_h,H,W] → flat [4, B*nh, H*W, kd], kd = qkv_h/(4*nh). */
VA_API int va_psa_pack_qkv_f32(const float *qkv, float *out, int qkv_h, int H, int W, int B,
                        int num_heads, va_stream_t stream);
VA_API int va_psa_pack_qkv_bf16(const va_bf16 *qkv, va_bf16 *out, int qkv_h, int H, int W, int B,
                         int num_heads, va_stream_t stream);
/* psa_pack_qkv_backward (psa.rs:201-233; args :411-417): accumulates into d_qkv. */
VA_API int va_psa_pack_qkv_backward_f32(const float *d_packed, float *d_qkv, int qkv_h, int H, int W,
                                 int B, int num_heads, va_stream_t stream);
/* psa_extract_v_nchw (psa.rs:105-142; args :472-478; B from grid() :483-488):
 * V channels of each head → NCHW [B,c,H,W], c = nh*2*kd. */
VA_API int va_psa_extract_v_nchw_f32(const float *qkv, float *v, int qkv_h, int c, int H, int W,
                              int num_heads, int B, va_stream_t stream);
VA_API int va_psa_extract_v_nchw_bf16(const va_bf16 *qkv, va_bf16 *v, int qkv_h, int c, int H, int W,
                               int num_heads, int B, va_stream_t stream);
/* psa_extract_v_backward (psa.rs:244-281; args :512-518): accumulates into d_qkv. */
VA_API int va_psa_extract_v_backward_f32(const float *d_v, float *d_qkv, int qkv_h, int c, int H,
                                  int W, int num_heads, int B, va_stream_t stream);
/* psa_merge_attn_nchw (psa.rs:153-189; args :575-581; B from grid() :586-591):
 * two [B*nh, N, kd] halves → NCHW [B,c,H,W]. */
VA_API int va_psa_merge_attn_nchw_f32(const float *lo, const float *hi, float *out, int c, int H, int W,
                               int num_heads, int B, va_stream_t stream);
VA_API int va_psa_merge_attn_nchw_bf16(const va_bf16 *lo, const va_bf16 *hi, va_bf16 *out, int c,
                                int H, int W, int num_heads, int B, va_stream_t stream);
/* psa_merge_attn_backward (psa.rs:292-327; args :614-620): stores d_lo, d_hi. */
VA_API int va_psa_merge_attn_backward_f32(const float *d_merged, float *d_lo, float *d_hi, int c, int H,
                                   int W, int num_heads, int B, va_stream_t stream);

/* ── Flash attention on [BH, N, head_dim] row-major ───────────────────────── */
/* flash_attention2_forward (flash_attn2.rs:54-121; args psa.rs:988-996;
 * grid (n_ctx_q, BH) psa.rs:999-1004).  l = m + ln(sum exp) per query row.
 * q/k/v may be offsets into the packed buffer exactly as psa.rs:982-985
 * computes them.  head_dim ∈ {16, 32, 64}.  The bf16 variant reads bf16
 * q/k/v, writes bf16 o and an f32 l. */
VA_API int va_flash_attention2_forward_f32(const float *q, const float *k, const float *v, float *o,
                                    float *l, int n_ctx_q, int n_ctx_k, float softmax_scale,
                                    float neg_inf, int bh, int head_dim, va_stream_t stream);
VA_API int va_flash_attention2_forward_bf16(const va_bf16 *q, const va_bf16 *k, const va_bf16 *v,
                                     va_bf16 *o, float *l, int n_ctx_q, int n_ctx_k,
                                     float softmax_scale, float neg_inf, int bh, int head_dim,
                                     va_stream_t stream);

/* The same node on the tensor cores (bf16, head_dim 32, n_ctx_q == n_ctx_k as
 * in the PSA graph): q/k/v/o/l exactly as above, plus a workspace of
 * va_flash_attention2_tc_workspace_bytes(n_ctx, bh, 32) bytes that a RuntimeOp
 * declares through param_shapes next to l.  It repacks q, k, v into the
 * tcgen05 attention kernel's layouts (f16), runs it with the given
 * softmax_scale and copies the 32 output channels back.  Inputs must satisfy
 * |x| < 65504 (f16 range).  VA_ERR_SHAPE for other head dims or cross
 * attention, VA_ERR_WORKSPACE when the workspace is missing or short. */
VA_API size_t va_flash_attention2_tc_workspace_bytes(int n_ctx, int bh, int head_dim);
VA_API int va_flash_attention2_forward_tc_bf16(const va_bf16 *q, const va_bf16 *k, const va_bf16 *v,
                                               va_bf16 *o, float *l, int n_ctx_q, int n_ctx_k,
                                               float softmax_scale, float neg_inf, int bh, int head_dim,
                                               void *workspace, size_t ws_bytes, va_stream_t stream);
/* flash_attention2_backward_dq (flash_attn2.rs:129-187): stores dq. */
VA_API int va_flash_attention2_backward_dq_f32(const float *q, const float *k, const float *v,
                                        const float *o, const float *d_o, const float *l,
                                        float *dq, int n_ctx_q, int n_ctx_k, float softmax_scale,
                                        int bh, int head_dim, va_stream_t stream);
/* flash_attention2_backward_dkv (flash_attn2.rs:195-260): stores dk, dv. */
VA_API int va_flash_attention2_backward_dkv_f32(const float *q, const float *k, const float *v,
                                         const float *o, const float *d_o, const float *l,
                                         float *dk, float *dv, int n_ctx_q, int n_ctx_k,
                                         float softmax_scale, int bh, int head_dim,
                                         va_stream_t stream);
/* psa_fa2_backward (psa.rs:650-725; args psa.rs:1044-1054): dq and dk
 * accumulate (the lo and hi calls share them), dv is stored.  Deterministic:
 * no atomics — each output row is owned by one thread. */
VA_API int va_psa_fa2_backward_f32(const float *q, const float *k, const float *v, const float *o,
                            const float *d_o, const float *l, float *dq, float *dk, float *dv,
                            int N, float softmax_scale, int bh, int head_dim, va_stream_t stream);

/* ── Convolution pieces of the PSA block (conv_bn, conv.rs:53-69) ─────────── */
/* Eval-mode BN folded into the conv (host function, no GPU):
 * w_out = w*g/sqrt(var+eps); b_out = beta - mean*g/sqrt(var+eps). */
VA_API int va_fold_bn_f32(const float *w, const float *gamma, const float *beta, const float *mean,
                   const float *var, float eps, int c_out, int k_per_out, float *w_out,
                   float *b_out);
/* 1×1 conv + bias, NCHW: y[b,o,n] = sum_i w[o,i] x[b,i,n] + bias[o]. */
VA_API int va_conv1x1_bias_f32(const float *x, const float *w, const float *bias, float *y, int B,
                        int c_in, int c_out, int HW, va_stream_t stream);
/* depthwise 3×3, stride 1, pad 1, + bias (the PE conv, c2psa.rs:66). */
VA_API int va_dwconv3x3_bias_f32(const float *x, const float *w, const float *bias, float *y, int B,
                          int C, int H, int W, va_stream_t stream);
/* its backward: stores dx; stores dw [C,1,3,3] (deterministic reduction). */
VA_API int va_dwconv3x3_backward_f32(const float *x, const float *w, const float *dy, float *dx,
                              float *dw, int B, int C, int H, int W, va_stream_t stream);

/* ── Fused PSA Attention forward (c2psa.rs:61-116, BN folded) ─────────────── *
 * y = proj(merge(FA(pack(qkv(x)))) + pe(extract_v(qkv(x)))), x/y NCHW [B,C,H,W].
 * Weights: w_qkv [nh*4*kd, C], w_pe [C,1,3,3], w_proj [C, C]; biases f32.
 * f32 variant: f32 everything (SIMT FFMA path, max-abs 1e-5 class).
 * bf16 variant: x, y and weights bf16, biases f32 (tcgen05/TMEM tensor-core
 * path: bf16 qkv GEMM, f16 attention operands, f32 accumulation); it
 * supports every c2psa width, kd = 32 and C = 64*nh (YOLO26 n: 128, s/m/l:
 * 256, x: 384; c2psa.rs:158) and any H, W (returns VA_ERR_SHAPE otherwise);
 * x, w_qkv, w_proj 16-byte aligned, workspace 256-byte aligned.  f32
 * variant: any C = nh*2*kd.
 * `workspace` holds the qkv/attention intermediates; size from
 * va_psa_attention_workspace_bytes().  dtype: 0 = f32, 1 = bf16.
 * bf16 at C = 128 (and the PSABlock / C2PSA entries below): after the qkv
 * GEMM the attention kernel runs on a highest-priority and the PE
 * convolution on a lowest-priority stream of the library's own (ordered
 * after `stream` by events, joined back before the projection), so PE
 * blocks fill the SMs the attention grid leaves idle at its end.  The
 * first such call on a device creates those two streams: make it before
 * any stream capture. */
VA_API size_t va_psa_attention_workspace_bytes(int B, int C, int H, int W, int num_heads, int key_dim,
                                        int dtype);
VA_API int va_psa_attention_fwd_f32(const float *x, const float *w_qkv, const float *b_qkv,
                             const float *w_pe, const float *b_pe, const float *w_proj,
                             const float *b_proj, float *y, int B, int C, int H, int W,
                             int num_heads, int key_dim, void *workspace, size_t ws_bytes,
                             va_stream_t stream);
VA_API int va_psa_attention_fwd_bf16(const va_bf16 *x, const va_bf16 *w_qkv, const float *b_qkv,
                              const va_bf16 *w_pe, const float *b_pe, const va_bf16 *w_proj,
                              const float *b_proj, va_bf16 *y, int B, int C, int H, int W,
                              int num_heads, int key_dim, void *workspace, size_t ws_bytes,
                              va_stream_t stream);

/* ── PSABlock and C2PSA forward (c2psa.rs:123-179, BN folded, bf16) ─────────
 * PSABlock (psa_block, c2psa.rs:123-137): y1 = x + attn(x);
 * y = y1 + ffn1(SiLU(ffn0(y1))) with ffn0 a 1×1 conv C→2C + BN + SiLU and
 * ffn1 a 1×1 conv 2C→C + BN (conv.rs:31-69).  C2PSA (c2psa.rs:150-179):
 * h = SiLU(cv1(x)) (C1→C1, split into a = h[:C1/2], b = h[C1/2:]);
 * b = PSABlock(b) n_blocks times; y = SiLU(cv2(cat(a, b))); C = C1/2,
 * num_heads = C/64, key_dim 32.  Weights bf16 with BN folded ([out][in] for
 * 1×1 convs), biases f32; x, y bf16 NCHW; H*W % 8 == 0; 16-byte aligned
 * pointers, 256-byte aligned workspace.  Tensor-core GEMMs with bias, SiLU
 * and residual in their epilogues around the tensor-core PSA Attention;
 * intermediates f16 except the attention op's bf16 input and output.  No
 * counterpart entry in the reference (its graph records these as separate
 * conv / elem_add nodes); the maths is the reference graph's. */
typedef struct va_psa_block_weights {
  const va_bf16 *w_qkv;  const float *b_qkv;   /* [2C][C], [2C]  qkv conv + BN */
  const va_bf16 *w_pe;   const float *b_pe;    /* [C][1][3][3], [C]  pe dw-conv + BN */
  const va_bf16 *w_proj; const float *b_proj;  /* [C][C], [C]  proj conv + BN */
  const va_bf16 *w_ffn0; const float *b_ffn0;  /* [2C][C], [2C]  ffn.0 conv + BN (SiLU) */
  const va_bf16 *w_ffn1; const float *b_ffn1;  /* [C][2C], [C]  ffn.1 conv + BN */
} va_psa_block_weights;
VA_API size_t va_psa_block_workspace_bytes(int B, int C, int H, int W);
VA_API int va_psa_block_fwd_bf16(const va_bf16 *x, const va_psa_block_weights *w, va_bf16 *y, int B,
                                 int C, int H, int W, void *workspace, size_t ws_bytes,
                                 va_stream_t stream);
VA_API size_t va_c2psa_workspace_bytes(int B, int C1, int H, int W, int n_blocks);
VA_API int va_c2psa_fwd_bf16(const va_bf16 *x, const va_bf16 *w_cv1, const float *b_cv1, int n_blocks,
                             const va_psa_block_weights *blocks, const va_bf16 *w_cv2,
                             const float *b_cv2, va_bf16 *y, int B, int C1, int H, int W,
                             void *workspace, size_t ws_bytes, va_stream_t stream);

/* ── safetensors weights with BN folding (examples/yolo26.rs:3403-3470) ──────
 * Host-side reader of a safetensors checkpoint (u64 header size, JSON header
 * of name → dtype/shape/data_offsets, tensor bytes) replacing the reference's
 * `load_weights_from_safetensors`.  open reads the file and parses the
 * header (malformed files return VA_ERR_SHAPE); tensor_info gives the dtype
 * (VA_ST_*, -1 for others) and shape (up to 8 dims); read_f32 converts an
 * F32/F16/BF16 tensor to f32 (count must equal its element count);
 * fold_conv_bn reads `{prefix}.conv.weight` and `{prefix}.bn.{weight, bias,
 * running_mean, running_var}` and folds them as the reference does
 * (scale = γ/√(var + eps), w·scale, β − mean·scale; eps 1e-3 for YOLO26,
 * conv.rs:39,64) into host buffers w_out [c_out][w_count/c_out], b_out
 * [c_out].  All pointers are host memory. */
#define VA_ST_F32 0
#define VA_ST_F16 1
#define VA_ST_BF16 2
typedef struct va_safetensors va_safetensors;
VA_API int va_safetensors_open(const char *path, va_safetensors **out);
VA_API void va_safetensors_close(va_safetensors *st);
VA_API int va_safetensors_tensor_info(va_safetensors *st, const char *key, int *dtype, int64_t *shape,
                                      int *rank);
VA_API int va_safetensors_read_f32(va_safetensors *st, const char *key, float *dst, size_t count);
VA_API int va_safetensors_fold_conv_bn(va_safetensors *st, const char *prefix, float eps, float *w_out,
                                       float *b_out, size_t w_count, int c_out);

/* ── Convolution + BN (+ SiLU), NHWC, tcgen05 implicit GEMM ─────────────────
 * Replaces the reference's `conv` (Conv2d → BN(eps 1e-3) → SiLU) and
 * `conv_bn` (Conv2d → BN) blocks with groups = 1 (yolo26/blocks/conv.rs:
 * 31-46, 53-69), BN folded into w and bias (va_fold_bn_f32 or
 * va_safetensors_fold_conv_bn):
 *   y[b][oy][ox][o] = act(bias[o] + Σ w[o][ky][kx][c]·x[b][s·oy+ky−k/2][s·ox+kx−k/2][c])
 * x [B][H][W][Cin] and y [B][Ho][Wo][Cout] bf16 NHWC, w [Cout][k][k][Cin]
 * bf16 (OHWI), bias f32 [Cout]; k ∈ {1, 3}, stride ∈ {1, 2}, padding k/2,
 * Ho = (H + 2·(k/2) − k)/stride + 1 (likewise Wo), act 1 = SiLU, 0 = none.
 * Cin and Cout multiples of 16, x/w/y 16-byte aligned (else
 * VA_ERR_SHAPE / VA_ERR_ALIGN).  f32 accumulation, one bf16 rounding of the
 * output.  A stalled pipeline wait sets the device status word
 * (va_device_status_read).  va_conv_weight_ohwi_bf16 permutes the
 * reference's OIHW weight layout to OHWI on the device. */
VA_API int va_conv_nhwc_bf16(const va_bf16 *x, const va_bf16 *w_ohwi, const float *bias, va_bf16 *y,
                             int B, int H, int W, int Cin, int Cout, int ksize, int stride, int act,
                             va_stream_t stream);
VA_API int va_conv_weight_ohwi_bf16(const va_bf16 *w_oihw, va_bf16 *w_ohwi, int Cout, int Cin,
                                    int ksize, va_stream_t stream);

/* ── Multi-scale deformable attention (RF-DETR decoder) ──────────────────────
 * No counterpart in the reference (it has no deformable attention); the
 * published MSDeformAttn core with grid_sample(align_corners=False,
 * padding_mode='zeros') sampling.  Layouts as the PyTorch op: value
 * [B][S][nh][dh], spatial_shapes [L][2] (H, W) and level_start [L] as int64
 * device arrays, loc [B][Q][nh][L][P][2] (x, y in [0,1]), attn
 * [B][Q][nh][L][P] (softmaxed), out [B][Q][nh*dh].  dh ∈ {16, 32}, L ≤ 8.
 * bf16 variants: value, out, grad_out and grad_value bf16; loc, attn and
 * their gradients f32.  The backward writes every element of grad_value,
 * grad_loc and grad_attn (no accumulation, deterministic) and needs a
 * workspace of va_msdeform_attn_bwd_workspace_bytes(); its per-(b, h, level)
 * working set, 24·Q·P + 4·Q·dh + 4·(S+1) bytes, must fit in 200 KiB of shared
 * memory (VA_ERR_SHAPE otherwise). */
VA_API int va_msdeform_attn_fwd_f32(const float *value, const int64_t *spatial_shapes,
                                    const int64_t *level_start, const float *loc, const float *attn,
                                    float *out, int B, int S, int nh, int dh, int L, int Q, int P,
                                    va_stream_t stream);
VA_API int va_msdeform_attn_fwd_bf16(const va_bf16 *value, const int64_t *spatial_shapes,
                                     const int64_t *level_start, const float *loc, const float *attn,
                                     va_bf16 *out, int B, int S, int nh, int dh, int L, int Q, int P,
                                     va_stream_t stream);
VA_API size_t va_msdeform_attn_bwd_workspace_bytes(int B, int nh, int L, int Q, int P);
VA_API int va_msdeform_attn_bwd_f32(const float *value, const int64_t *spatial_shapes,
                                    const int64_t *level_start, const float *loc, const float *attn,
                                    const float *grad_out, float *grad_value, float *grad_loc,
                                    float *grad_attn, int B, int S, int nh, int dh, int L, int Q, int P,
                                    void *workspace, size_t ws_bytes, va_stream_t stream);
VA_API int va_msdeform_attn_bwd_bf16(const va_bf16 *value, const int64_t *spatial_shapes,
                                     const int64_t *level_start, const float *loc, const float *attn,
                                     const va_bf16 *grad_out, va_bf16 *grad_value, float *grad_loc,
                                     float *grad_attn, int B, int S, int nh, int dh, int L, int Q, int P,
                                     void *workspace, size_t ws_bytes, va_stream_t stream);

/* The attention core of the bf16 path on its own (tcgen05, one launch):
 * O = softmax(Q·Kᵀ/√32)·V per (b, head) with the full 64-wide V — the two
 * reference flash_attention2_forward calls (psa.rs:930-944) in one pass.
 * Layouts (f16): qk = [2][B*nh][N][32] (psa_pack_qkv sections 0 and 1),
 * v and o = [B][nh*64][Np] channel-major with row pitch Np = roundup(N, 8)
 * (psa_extract_v_nchw / psa_merge_attn_nchw layouts, padded); lse optional
 * [B*nh][N] f32.  Any number of heads (C = 64·nh). */
VA_API int va_psa_flash_attention_fwd_f16(const void *qk, const void *v, void *o, float *lse, int B,
                                          int num_heads, int H, int W, va_stream_t stream);

/* PSA Attention forward (bf16) that allocates nothing: no counterpart in the
 * reference.  For callers that cannot hand the op a workspace — a graph
 * runtime whose device buffers are all planned before it runs, or host code
 * that must not enter a device allocator mid-run.  Scratch comes from a
 * VA_NOALLOC_SCRATCH_BYTES array built into the library, held on every GPU
 * that loads it until the process exits; larger problems return
 * VA_ERR_WORKSPACE (split the batch, or use the workspace entry above).  The
 * first call on a device looks up that device's scratch address, so make it
 * before any stream capture.  Calls share the scratch: calls that overlap on
 * the GPU race, so serialise them.  Same sizes and results as
 * va_psa_attention_fwd_bf16. */
#define VA_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
VA_API int va_psa_attention_fwd_bf16_noalloc(const va_bf16 *x, const va_bf16 *w_qkv, const float *b_qkv,
                                             const va_bf16 *w_pe, const float *b_pe,
                                             const va_bf16 *w_proj, const float *b_proj, va_bf16 *y,
                                             int B, int C, int H, int W, int num_heads, int key_dim,
                                             va_stream_t stream);

/* ── DINOv2 backbone attention (bf16, tcgen05) ───────────────────────────
 * No counterpart in the reference (it has no DINOv2 code): the published
 * ViT/DINOv2 self-attention.  x [S][n][hidden] bf16 (S sequences of n
 * tokens), w_qkv [3*hidden][hidden] bf16 (nn.Linear weight: q, k, v sections,
 * head-major inside each), b_qkv [3*hidden] f32, o [S][n][hidden] bf16 =
 * concat_heads(softmax(q·kᵀ/8)·v), head dim 64, num_heads*64 == hidden
 * (DINOv2-S: 384, 6).  Global layers: S = images, n = 1 + H·W (cls first).
 * Windowed layers: S = images·windows, n = 1 + win² — the cls token joins
 * every window as token 0 (va_dinov2_window_partition_bf16), and
 * un-partitioning averages the windows' cls outputs. */
VA_API size_t va_dinov2_attention_workspace_bytes(int num_seqs, int seq_len, int hidden);
VA_API int va_dinov2_attention_fwd_bf16(const va_bf16 *x, const va_bf16 *w_qkv, const float *b_qkv,
                                        va_bf16 *o, int num_seqs, int seq_len, int hidden,
                                        int num_heads, void *workspace, size_t ws_bytes,
                                        va_stream_t stream);
/* The attention core alone (one launch), on the operands the fused op keeps
 * in its workspace: qk f16 [2][S*heads][n][64] (Q then K, sequence-major,
 * head-minor), v f16 [S*heads*64][roundup(n, 8)] (transposed); o bf16
 * [S][n][heads*64]. */
VA_API int va_dinov2_flash_attention_fwd_f16(const void *qk, const void *v, va_bf16 *o, int num_seqs,
                                             int seq_len, int num_heads, va_stream_t stream);
/* The packed QKV Linear alone: qkv [tokens][3*hidden] bf16 = x·w_qkvᵀ + b. */
VA_API int va_dinov2_qkv_linear_bf16(const va_bf16 *x, const va_bf16 *w_qkv, const float *b_qkv,
                                     va_bf16 *qkv, int tokens, int hidden, va_stream_t stream);
/* x [B][1 + gh*gw][hidden] ↔ xw [B*(gh/win)*(gw/win)][1 + win*win][hidden];
 * window w = wy*(gw/win) + wx, patches row-major inside a window. */
VA_API int va_dinov2_window_partition_bf16(const va_bf16 *x, va_bf16 *xw, int B, int grid_h,
                                           int grid_w, int win, int hidden, va_stream_t stream);
VA_API int va_dinov2_window_unpartition_bf16(const va_bf16 *xw, va_bf16 *x, int B, int grid_h,
                                             int grid_w, int win, int hidden, va_stream_t stream);

/* ── PSA Attention training step (data-parallel cfg5) ─────────────────────
 * One rank's forward + backward on its shard, bf16 activations and weights,
 * f32 gradients; the caller all-reduces `grads` across ranks and applies
 * va_psa_sgd_update.  The reference trains the same block through its
 * backward kernels (psa_fa2_backward psa.rs:650-725, psa_*_backward
 * psa.rs:201-327, conv BackwardDx/Dw); here BN is folded (conv weight + bias
 * are the parameters).  Loss = mean((y − target)²) over the shard, written to
 * *loss (device).  y [B,C,H,W] bf16 output; dx (optional, may be NULL)
 * bf16; grads f32 [VA_PSA_GRAD_COUNT] in PyTorch parameter layouts at the
 * offsets below (stored, not accumulated).  Deterministic. */
#define VA_PSA_GRAD_WQKV 0         /* [256][128] */
#define VA_PSA_GRAD_WPROJ 32768    /* [128][128] */
#define VA_PSA_GRAD_WPE 49152      /* [128][1][3][3] */
#define VA_PSA_GRAD_BQKV 50304     /* [256] */
#define VA_PSA_GRAD_BPROJ 50560    /* [128] */
#define VA_PSA_GRAD_BPE 50688      /* [128] */
#define VA_PSA_GRAD_COUNT 50816
VA_API size_t va_psa_train_workspace_bytes(int B, int H, int W);
VA_API int va_psa_train_fwd_bwd_bf16(const va_bf16 *x, const va_bf16 *target, const va_bf16 *w_qkv,
                                     const float *b_qkv, const va_bf16 *w_pe, const float *b_pe,
                                     const va_bf16 *w_proj, const float *b_proj, va_bf16 *y,
                                     va_bf16 *dx, float *grads, float *loss, int B, int C, int H,
                                     int W, int num_heads, int key_dim, void *workspace,
                                     size_t ws_bytes, va_stream_t stream);
/* The backward of the fused bf16 op for any loss: given x, the folded weights and dy = ∂L/∂y
 * [B,C,H,W] bf16, recompute the forward and write grads (f32, the layout and
 * offsets above, stored) and, if dx is not NULL, dx = ∂L/∂x (bf16).  The
 * backward runs on dy/dy_scale in f16; pass dy_scale ≈ max|dy| (e.g. 2/numel
 * for a mean-squared loss) so that the scaled values are O(1); the stored
 * gradients carry the full scale.  Same kernels, workspace query
 * (va_psa_attention_bwd_workspace_bytes) and limits as the training step. */
/* The backward of the f32 op (va_psa_attention_fwd_f32) for any loss: the
 * reference graph's backward nodes in f32 on the FFMA kernels
 * (psa_fa2_backward psa.rs:650-725 for the V_lo and V_hi calls, psa_*_backward
 * psa.rs:201-327, the conv_bn backwards with BN folded) after recomputing the
 * forward.  dy = ∂L/∂y [B,C,H,W]; grads (f32, stored) = [w_qkv (nh·4·kd × C) |
 * w_proj (C × C) | w_pe (C × 9) | b_qkv | b_proj | b_pe], the layout of the
 * bf16 entry's gradient buffer (the VA_PSA_GRAD_* offsets at C = 128); dx =
 * ∂L/∂x (optional, may be NULL).  Any C = nh·2·kd; deterministic (no atomics). */
VA_API size_t va_psa_attention_bwd_f32_workspace_bytes(int B, int C, int H, int W, int num_heads,
                                                       int key_dim);
VA_API int va_psa_attention_bwd_f32(const float *x, const float *dy, const float *w_qkv,
                                    const float *b_qkv, const float *w_pe, const float *b_pe,
                                    const float *w_proj, const float *b_proj, float *dx, float *grads,
                                    int B, int C, int H, int W, int num_heads, int key_dim,
                                    void *workspace, size_t ws_bytes, va_stream_t stream);
VA_API size_t va_psa_attention_bwd_workspace_bytes(int B, int H, int W);
VA_API int va_psa_attention_bwd_bf16(const va_bf16 *x, const va_bf16 *dy, float dy_scale,
                                     const va_bf16 *w_qkv, const float *b_qkv, const va_bf16 *w_pe,
                                     const float *b_pe, const va_bf16 *w_proj, const float *b_proj,
                                     va_bf16 *dx, float *grads, int B, int C, int H, int W,
                                     int num_heads, int key_dim, void *workspace, size_t ws_bytes,
                                     va_stream_t stream);
/* master (f32, gradient layout) -= lr·grad_scale·grads; then the bf16
 * weights and f32 biases the forward reads are rewritten from master. */
VA_API int va_psa_sgd_update(float *master, const float *grads, float lr, float grad_scale,
                             va_bf16 *w_qkv, float *b_qkv, va_bf16 *w_pe, float *b_pe,
                             va_bf16 *w_proj, float *b_proj, va_stream_t stream);

/* ── Data-parallel gradient all-reduce over NVLink peer memory ───────────────
 * Replaces the NCCL all-reduce + va_psa_sgd_update pair of the data-parallel
 * step (the reference's trainer all-reduces the gradients between backward
 * and the optimizer step) with one kernel per step on every rank.  Set-up, one
 * process per GPU on one node:
 *   va_dp_comm_create   allocates and zeroes this rank's exported buffer and
 *                       writes its CUDA IPC handle (VA_DP_HANDLE_BYTES) to
 *                       *handle; count must be VA_PSA_GRAD_COUNT; 1..8 ranks;
 *                       timeout_ms bounds each device-side wait for a peer
 *                       (0 = the default, 10 s).
 *   va_dp_comm_connect  opens every peer's buffer from the rank-ordered array
 *                       of all ranks' handles (world × VA_DP_HANDLE_BYTES);
 *                       call on every rank after all have created theirs.
 *   Teardown, in this order on every rank:
 *   va_dp_comm_disconnect  closes this rank's mappings of the peers' buffers;
 *                       call after a barrier that follows every rank's last
 *                       all-reduce;
 *   va_dp_comm_destroy  frees this rank's buffer; call after a second barrier,
 *                       once every peer has disconnected (it also closes any
 *                       mapping still open).
 * va_psa_dp_allreduce_sgd: grads (f32 [VA_PSA_GRAD_COUNT], in place) becomes
 * the sum over ranks, taken in rank order (the same bits on every rank), and
 * master -= lr · sum / world, then the bf16 weights and f32 biases are
 * rewritten from master as in va_psa_sgd_update.  Every rank must call it once
 * per step, in the same order.  A device-side wait that passes timeout_ms
 * records 100 + the peer's rank in the comm's status word, which
 * va_dp_comm_status reads (synchronising); 0 = no failure.  The status word is
 * sticky: once it is set, every later call returns at once without publishing
 * or updating anything.  Blocks whose waits had passed before the failure
 * have already updated their part of master and the weights, so after a
 * non-zero status the weights must be restored on every rank and the comm
 * destroyed and created anew on every rank. */
#define VA_DP_HANDLE_BYTES 64
typedef struct va_dp_comm va_dp_comm;
VA_API int va_dp_comm_create(int rank, int world, int count, int timeout_ms, va_dp_comm **comm,
                             void *handle);
VA_API int va_dp_comm_connect(va_dp_comm *comm, const void *handles);
VA_API int va_dp_comm_status(va_dp_comm *comm, int *status);
VA_API int va_dp_comm_disconnect(va_dp_comm *comm);
VA_API int va_dp_comm_destroy(va_dp_comm *comm);
VA_API int va_psa_dp_allreduce_sgd(va_dp_comm *comm, float *grads, float *master, float lr, va_bf16 *w_qkv,
                                   float *b_qkv, va_bf16 *w_pe, float *b_pe, va_bf16 *w_proj, float *b_proj,
                                   va_stream_t stream);

/* Batched f16 tensor-core GEMM used by the training step (no counterpart in
 * the reference): C[z][m][n] = alpha·Σ_k A_z(m,k)·B_z(n,k), f32 accumulation.
 * An operand is K-major (x_mn = 0: row m holds K elements, row pitch ld) or
 * MN-major (x_mn = 1: row k holds the M or N elements); x_batch = elements
 * between batch entries, x_bcast = 1 to use one matrix for all z.  C is f32
 * (c_type = 0), bf16 (1) or f16 (2), row pitch ldc, batch stride c_batch.  16-byte
 * aligned bases and pitches. */
VA_API int va_gemm_f16(const void *a, int a_mn, long long lda, long long a_batch, int a_bcast,
                       const void *b, int b_mn, long long ldb, long long b_batch, int b_bcast,
                       void *c, int c_type, long long ldc, long long c_batch, int M, int N, int K,
                       int Z, float alpha, va_stream_t stream);

/* Device status word of the tensor-core kernels: 0, or 1000+site of the
 * first bounded wait that gave up.  read: copies it to *status (synchronises
 * `stream`); clear: resets it to 0. */
VA_API int va_device_status_read(int *status, va_stream_t stream);
VA_API int va_device_status_clear(va_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* VISIONATTN_H */
