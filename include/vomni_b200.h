/*
 * vomni_b200.h — C ABI of the B200-native context-parallel self-attention hot path of the
 * Wan2.2-A14B DiT (const-max ring attention, fused adaLN + FP8 row quant, FP8 QKV projection).
 *
 * Plain pointers, sizes and a CUDA stream handle; no framework types. Every entry point is
 * stream-ordered on `stream`, validates its arguments on the host and returns a vomni_status
 * code (never aborts). Device pointers must be CUDA device (or managed) memory of the calling
 * thread's current device. Kernels that wait on barriers bound every wait; a wait that runs out
 * records a device-side code readable with vomni_device_status().
 *
 * Each entry point names the reference interface it replaces, as
 * reecedantin/vllm-omni-neuron path:line.
 */
#ifndef VOMNI_B200_H
#define VOMNI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VOMNI_API __attribute__((visibility("default")))
#else
#define VOMNI_API
#endif

typedef struct CUstream_st* vomni_stream_t; /* same object as cudaStream_t / CUstream */

enum vomni_status {
  VOMNI_OK = 0,
  VOMNI_EINVAL = 1,     /* bad argument (null pointer, unknown flag/mode)                    */
  VOMNI_EBADSHAPE = 2,  /* unsupported shape (e.g. head_dim != 128, empty extent)            */
  VOMNI_EALIGN = 3,     /* pointer / stride not aligned as the TMA engine requires (16 B)    */
  VOMNI_ECUDA = 4,      /* a CUDA runtime / driver call failed                               */
  VOMNI_ENCCL = 5,      /* NCCL failed or is unavailable                                     */
  VOMNI_ETIMEOUT = 6,   /* a bounded device or host wait ran out                             */
  VOMNI_ENOTSUP = 7,    /* not supported on this device (needs sm_100)                       */
  VOMNI_EWORKSPACE = 8, /* workspace too small                                               */
  VOMNI_ESTATE = 9      /* context misuse (wrong rank count, destroyed context, ...)         */
};

/* Device status word values (vomni_device_status): 0 = healthy; 0x1000 + site = a bounded
 * mbarrier wait at `site` ran out. */
#define VOMNI_DEV_TIMEOUT_BASE 0x1000

/* ------------------------------------------------------------------ library */
VOMNI_API int vomni_abi_version(void);
VOMNI_API const char* vomni_strerror(int code);
/* Synchronises the device, copies the status word to *code, optionally clears it. */
VOMNI_API int vomni_device_status(int* code, int clear);

/* Failure-detection self-test (no counterpart in the reference, whose kernels have no runtime
 * waits): one CTA waits on an mbarrier that nothing arrives on, with a budget of budget_us
 * microseconds (<= 2 s). The bounded wait gives up, the kernel ends normally, the device status
 * word reads VOMNI_DEV_TIMEOUT_BASE + 0x7F and *result_host = 0 (1 would mean the wait
 * completed). Synchronises `stream`. */
VOMNI_API int vomni_selftest_bounded_wait(unsigned budget_us, int* result_host, vomni_stream_t stream);
/* Same for the ring's block-ready gate: one CTA waits (budget_us, <= 2 s) for a device word to
 * reach 1. post = 1: the word is first posted on `stream` with the stream memory operation the ring
 * uses (cuStreamWriteValue32), the wait completes, *result_host = 1 and the status stays 0.
 * post = 0: nothing posts it, the wait gives up, *result_host = 0 and the status word reads
 * VOMNI_DEV_TIMEOUT_BASE + 0x7E. Synchronises `stream`. */
VOMNI_API int vomni_selftest_ready_wait(unsigned budget_us, int post, int* result_host, vomni_stream_t stream);
/* Evaluates, for n device floats x, the FMA-pipe exponential 2^x that the attention kernel uses for
 * a share of its softmax probabilities (Cody-Waite range reduction + degree-3 minimax polynomial in
 * packed fp32 pairs; inputs below -126 clamp to about 2^-126) into device y. A test hook so that the
 * method can be checked against exact 2^x; no counterpart in the reference. Stream-ordered. */
VOMNI_API int vomni_selftest_exp2_poly(const float* x, float* y, long long n, vomni_stream_t stream);
/* Stream-ordered 2-D copy (height rows of width bytes; pitches in bytes) between any two of host
 * (pinned) and device memory: the host-resident attention entry streams head groups with it.
 * No counterpart in the reference (its inputs are always device-resident). */
VOMNI_API int vomni_memcpy_2d_async(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                                    size_t height, vomni_stream_t stream);

/* ------------------------------------------------------------------ const-max attention
 * Replaces the NKI kernel ring_attention_const_max_fwd
 * (vllm_omni_neuron/kernels/nkilib/experimental/attention/ring_attention_const_max_fwd.py:958-1404)
 * and its per-step partial _attention_const_max_partial (attention_const_max.py:69-234).
 *
 * Layouts (bf16): q, k, v token-major [b, s, h, d] (d must be 128). out is head-major
 * [b, h, s, d] (the kernel's return layout, ring_attention_const_max_fwd.py:1400) or, with
 * VOMNI_CM_OUT_DMAJOR, d-major [b, h, d, s] (the layout wan_cp_self_attention returns,
 * wan2_2_transformer.py:836). lse (optional, fp32) is [b, h, 128, ceil(s/128)] with
 * lse[.., r, g] for token g*128 + r (ring_attention_const_max_fwd.py:1062-1065).
 */
#define VOMNI_CM_ACC_IN 1     /* add the fp32 partial already in acc_o / acc_l                */
#define VOMNI_CM_FINAL 2      /* normalise and write bf16 out (else write the fp32 partial)   */
#define VOMNI_CM_OUT_DMAJOR 4 /* out is [b, h, d, s] instead of [b, h, s, d]                  */
#define VOMNI_CM_LSE 8        /* also write lse = c + ln(max(sum, 1e-37))                     */
#define VOMNI_CM_OVERLAP 16   /* vomni_cm_attend only: the pass may start while the preceding
                                 const-max pass on the stream still runs (programmatic dependent
                                 launch); only its epilogue waits for that pass. q, k, v, qn2 and
                                 kmax2 must not be written by the preceding kernel.             */

/* Bytes of workspace vomni_cm_attention_local needs (norms, key max, status). */
VOMNI_API size_t vomni_cm_workspace_bytes(int b, int s, int h, int d);

/* Prologue: qn2[b*h, s] = per-token ||q||^2, kmax2[b*h] = max over this rank's tokens of ||k||^2
 * (fp32, from the bf16 values). kmax2 is overwritten (not max-accumulated).
 * Replaces _transpose_qk_pipelined's fused norms (ring_attention_const_max_fwd.py:424-556). */
VOMNI_API int vomni_cm_prologue(const void* q, const void* k, int b, int s, int h, int d, float* qn2, float* kmax2,
                      vomni_stream_t stream);

/* One pass of const-max attention of all query rows against keys [k_start, k_start + n_keys) of
 * k/v (each [b, s_kv, h, d]), with the per-row bound c_i = bf16(scale * sqrt(kmax2[bh] * qn2[bh, i])).
 * Partial sums go to acc_o [b*h, s_q, d] / acc_l [b*h, s_q] (fp32) unless VOMNI_CM_FINAL.
 * Replaces one ring step: _run_partial_step / _run_last_step_and_normalize
 * (ring_attention_const_max_fwd.py:806-955). */
VOMNI_API int vomni_cm_attend(const void* q, const void* k, const void* v, int b, int s_q, int s_kv, int k_start, int n_keys,
                    int h, int d, float softmax_scale, const float* qn2, const float* kmax2, float* acc_o,
                    float* acc_l, int flags, void* out, float* lse, vomni_stream_t stream);

/* Strided forms: q and k/v rows (tokens) are q_stride / kv_stride elements apart (0 = dense h*d;
 * >= h*d, multiple of 8), batch stride s * stride — the token-major views a fused [b, s, 3*h*d]
 * QKV projection hands out (row_mx_modules.py:390-393 tensor_split), read without a copy. */
VOMNI_API int vomni_cm_prologue_strided(const void* q, const void* k, int b, int s, int h, int d, long long q_stride,
                                        long long k_stride, float* qn2, float* kmax2, vomni_stream_t stream);
VOMNI_API int vomni_cm_attend_strided(const void* q, const void* k, const void* v, int b, int s_q, int s_kv, int k_start,
                                      int n_keys, int h, int d, long long q_stride, long long kv_stride,
                                      float softmax_scale, const float* qn2, const float* kmax2, float* acc_o,
                                      float* acc_l, int flags, void* out, float* lse, vomni_stream_t stream);
VOMNI_API int vomni_cm_attention_local_strided(const void* q, const void* k, const void* v, void* out, float* lse, int b,
                                               int s, int h, int d, long long q_stride, long long kv_stride,
                                               float softmax_scale, int flags, void* workspace, size_t workspace_bytes,
                                               vomni_stream_t stream);
/* Cross-attention (keys from another sequence, e.g. the 512-token text context; no ring): the
 * exact attention of _nki_attend / _torch_attend (wan2_2_transformer.py:640-674) over s_kv keys, via
 * the same const-max kernel. q [b, s_q, h, d] and k, v [b, s_kv, h, d] token-major (token pitches
 * q_stride / kv_stride elements, 0 = dense); workspace as vomni_cm_workspace_bytes(b, s_q, h, d). */
VOMNI_API int vomni_cm_attention_cross(const void* q, const void* k, const void* v, void* out, float* lse, int b,
                                       int s_q, int s_kv, int h, int d, long long q_stride, long long kv_stride,
                                       float softmax_scale, int flags, void* workspace, size_t workspace_bytes,
                                       vomni_stream_t stream);

/* Single-rank (num_workers == 1) const-max attention: prologue + one final pass.
 * Replaces ring_attention_const_max_fwd(num_workers=1) (ring_attention_const_max_fwd.py:1306-1327).
 * flags: VOMNI_CM_OUT_DMAJOR / VOMNI_CM_LSE. */
VOMNI_API int vomni_cm_attention_local(const void* q, const void* k, const void* v, void* out, float* lse, int b, int s, int h,
                             int d, float softmax_scale, int flags, void* workspace, size_t workspace_bytes,
                             vomni_stream_t stream);

/* ------------------------------------------------------------------ fused adaLN + FP8 quant
 * Replaces adaln_quant_kernel (kernels/nkilib/experimental/norm/adaln_quant.py:117-810) as called
 * by the bridge adaln_modulate (diffusion/quantization/adaln_kernels.py:87-201):
 *   t = residual + gate * hidden (fp32, rounded to bf16 -> residual_out); xhat = LayerNorm(t) |
 *   RMSNorm(t) | t; y = xhat * mul + add; out = bf16(y) | FP8 row quant | FP8 MX-32.
 * hidden/residual/residual_out: bf16 [rows, h]; mul/add: bf16 [n_mod, h]; gate: fp32 [n_mod, h]
 * (n_mod = rows / rows_per_mod; all optional except hidden). norm_type 0 layer / 1 rms / 2 none.
 * quant 0: out bf16 [rows, h]. quant 1 (row, range 448 if ocp else 240): packed != 0 -> out u8
 * [rows, h + 4] (codes, then the fp32 dequant scale, adaln_quant.py:540-565); packed == 0 -> out u8
 * [rows, h] + out_scale fp32 [rows]. quant 2 (MX-32, adaln_quant_torch.py:151-175): out u8
 * [rows, h] e4m3fn codes + out_scale u8 [rows, h/32] UE8M0 exponents. h <= 16384, h % 8 == 0. */
VOMNI_API int vomni_adaln_modulate(const void* hidden, const void* residual, const void* mul, const void* add,
                                   const float* gate, long long rows, int h, long long rows_per_mod, float eps,
                                   int norm_type, int quant, int ocp, int packed, void* out, void* out_scale,
                                   void* residual_out, vomni_stream_t stream);

/* ------------------------------------------------------------------ FP8 QKV projection
 * Replaces qkv(quantization_type=ROW_MX) -> _qkv_cte_mx_impl (kernels/nkilib/core/qkv/qkv_cte.py:
 * 2725-3993) as called through torch_compatible_row_mx_qkv (kernels/qkv_shim.py:26-77) by
 * row_mx_qkv_proj (diffusion/quantization/row_mx_kernels.py:48-111).
 *
 * vomni_qkv_fp8_gemm: y[t, i] = bf16(sum_h x[t, h] w[i, h] * row_scale[t] * chan_scale[i] + bias[i])
 * (_dequant_row_mx, qkv_cte.py:3996-4021). x_codes: e4m3fn [t, h]; w_codes: e4m3fn [i, h] (K-major);
 * bias bf16 [i] or NULL; y bf16 [t, i]. If sumsq is non-NULL it receives, per row, the sums of
 * squares of the stored bf16 y over each 128-column head of the Q and K segments
 * ([t, (q_dim + kv_dim) / 128] fp32), the input of the across-heads RMS (qkv_cte.py:3870-3898).
 * h % 128 == 0, i % 256 == 0, q_dim % 256 == 0, kv_dim % 256 == 0. */
VOMNI_API int vomni_qkv_fp8_gemm(const void* x_codes, const float* row_scale, const void* w_codes,
                                 const float* chan_scale, const void* bias, int t, int h, int i, int q_dim, int kv_dim,
                                 void* y, float* sumsq, vomni_stream_t stream);
/* In place on y [t, i]: inv = rsqrt(sum(sumsq row segment) / (heads * 128) + eps) for the Q and K
 * segments; x * gamma (bf16 [heads*128], optional); then rotate-half RoPE with inv folded in
 * (cos/sin fp32 [t, 128], optional: without them x * inv) — the apply pass of qkv_cte.py:3903-3991. */
VOMNI_API int vomni_qk_norm_rope(void* y, int t, int i, int q_heads, int kv_heads, int head_dim, const float* sumsq,
                                 float eps, const void* gamma_q, const void* gamma_k, const float* cos, const float* sin,
                                 vomni_stream_t stream);
/* MX-32 mode (block-scaled tcgen05 GEMM, kind::mxf8f6f4.block_scale; the MX-32 format of
 * _mx_dequant, kernels/nkilib/experimental/norm/adaln_quant_torch.py:151-175):
 * y[t, i] = bf16(sum over 32-blocks of (x codes * 2^(sx-127)) . (w codes * 2^(sw-127)) + bias[i]),
 * same sumsq partials as vomni_qkv_fp8_gemm. Scale factors (UE8M0 bytes, [rows, h/32] row-major as
 * vomni_adaln_modulate quant 2 writes them) must first be re-tiled with vomni_mx_pack_scales into
 * vomni_mx_packed_scales_bytes(rows, h) bytes (weights: once, at load time). */
VOMNI_API size_t vomni_mx_packed_scales_bytes(int rows, int k);
VOMNI_API int vomni_mx_pack_scales(const void* sf, int rows, int k, void* out, vomni_stream_t stream);
VOMNI_API int vomni_qkv_mx32_gemm(const void* x_codes, const void* x_sf_packed, const void* w_codes,
                                  const void* w_sf_packed, const void* bias, int t, int h, int i, int q_dim, int kv_dim,
                                  void* y, float* sumsq, vomni_stream_t stream);
/* [t, h + 4] packed rows (adaln ROW output) -> codes [t, h] + scales [t]. */
VOMNI_API int vomni_qkv_unpack_rows(const void* packed, int t, int h, void* codes, float* scales, vomni_stream_t stream);

/* ------------------------------------------------------------------ output projection
 * _wan_o_proj (diffusion/models/wan2_2/wan2_2_transformer.py:246-254) on the d-major attention output
 * attn [b, k, s] bf16 (k = heads*128; s % 8 == 0) and w [k, h] bf16 (h % 32 == 0, k % 64 == 0):
 * y = bf16(bf16(x @ w) + bias) with x[t] = attn[:, :, t], written to out [b, s, h]. With a residual
 * [b, s, h] bf16 the kernel writes the norm2 gated residual t = bf16(residual + gate * y) instead
 * (gate fp32 [b, h] when gate_per_batch, else [h]; NULL = 1), the residual step of
 * adaln_modulate(..., residual=, gate=) (wan2_2_transformer.py:1470-1489). */
VOMNI_API int vomni_oproj_gemm(const void* attn, int b, int k, int s, const void* w, const void* bias, int h,
                               const void* residual, const float* gate, int gate_per_batch, void* out,
                               vomni_stream_t stream);
/* The activation side of row_mx_o_proj (diffusion/quantization/row_mx_kernels.py:114-138, whose NKI
 * kernel output_projection_cte quantises its input internally): per-token ROW FP8 quantisation of the
 * d-major attention output attn [b, k, s] bf16 (s % 8 == 0, k % 64 == 0, k <= 16384 — k <= 8192 when
 * k % 128 != 0 — 16-byte aligned), with the
 * ROW rule of adaln_quant.py:520-536 (scale = max(amax / 448, 1e-6), codes = e4m3fn(x * (1 / scale)),
 * amax over the token's k values). Writes token rows codes [b * s, k] e4m3 (16-byte aligned) and
 * scales [b * s] fp32, the operands of vomni_qkv_fp8_gemm (row scale = scales, q_dim = kv_dim = 0). */
VOMNI_API int vomni_oproj_rowquant(const void* attn, int b, int k, int s, void* codes, float* scales,
                                   vomni_stream_t stream);

/* Wan FFN GEMM step (_wan_mlp, wan2_2_transformer.py:389-410): out [m, n] = x [m, k] @ w [k, n] + bias,
 * rounded to bf16 after the matmul and after the bias add as torch does; act = 1 then applies
 * GELU-tanh (fp32 opmath, bf16 result). With a residual [m, n] (act = 0) the kernel writes the block's
 * closing gated residual bf16(residual + gate * y) instead (wan2_2_transformer.py:1510-1512; gate fp32
 * [m / gate_rows, n], row r using gate row r / gate_rows; NULL = 1). All bf16; k % 64 == 0, n % 32 == 0. */
VOMNI_API int vomni_ffn_gemm(const void* x, long long m, int k, const void* w, const void* bias, int n, int act,
                             const void* residual, const float* gate, long long gate_rows, void* out,
                             vomni_stream_t stream);

/* ROW_MX MLP (FP8 FFN leaf): row_mx_mlp (diffusion/quantization/row_mx_kernels.py:141-198), the
 * nkilib MLP in ROW_MX / CTE mode whose arithmetic kernels/nkilib/core/mlp/mlp_torch.py:401-600 states.
 * Up: x_codes [t, h] e4m3 with row_scale [t] fp32 (the ROW-quantised adaLN output, codes split from
 * the packed [t, h+4] rows), w_codes [i, h] e4m3 (W_up^T, K-major) with chan_scale [i] fp32 and bias
 * [i] bf16 (NULL = 0): v = gelu_tanh(acc * row_scale * chan_scale + bias) in fp32, MX-32 quantised
 * along i (UE8M0 scale = max biased exponent of 32 values - 7, clip [0, 255]; codes e4m3fn,
 * saturating at 448; _mx_quantize, mlp_torch.py:252-271) into inter_codes [t, i] and
 * inter_sf_packed (vomni_mx_packed_scales_bytes(t, i) bytes, the tcgen05 atom layout of
 * vomni_mx_pack_scales). h % 128 == 0, i % 256 == 0. */
VOMNI_API int vomni_ffn_fp8_up(const void* x_codes, const float* row_scale, const void* w_codes,
                               const float* chan_scale, const void* bias, int t, int h, int i, void* inter_codes,
                               void* inter_sf_packed, vomni_stream_t stream);
/* Down: out [t, h] bf16 = bf16(acc * chan_scale + bias) with acc the block-scaled product of the
 * intermediate (inter_codes, inter_sf_packed) and w_codes [h, i] e4m3 (W_down^T, K-major) whose
 * packed block scales w_sf_packed are all 127 (identity; vomni_mx_packed_scales_bytes(h, i) bytes);
 * chan_scale [h] fp32, bias [h] bf16 (NULL = 0). With a residual [t, h] bf16 the kernel writes the
 * block's closing gated residual bf16(residual + gate * y) instead (wan2_2_transformer.py:1510-1512;
 * gate fp32 [t / gate_rows, h], NULL = 1). i % 128 == 0, h % 256 == 0. */
VOMNI_API int vomni_ffn_fp8_down(const void* inter_codes, const void* inter_sf_packed, const void* w_codes,
                                 const void* w_sf_packed, const float* chan_scale, const void* bias, int t, int i,
                                 int h, const void* residual, const float* gate, long long gate_rows, void* out,
                                 vomni_stream_t stream);

/* bf16 projection for the across-heads RMS norm that follows (the bf16 self-attention leaf's
 * qkv_proj + norm_q/norm_k, wan2_2_transformer.py:1097-1109, and the cross-attention's q/k
 * projections, :1232-1248): out [m, n] = bf16(bf16(x @ w) + bias) and sumsq [m, n_norm_heads] = per
 * 128-column head sums of squares of the stored values, the input of vomni_qk_norm_rope. */
VOMNI_API int vomni_linear_sumsq(const void* x, long long m, int k, const void* w, const void* bias, int n,
                                 float* sumsq, int n_norm_heads, void* out, vomni_stream_t stream);

/* ------------------------------------------------------------------ CFG-parallel combine
 * The combine of _cfg_gather_combine (diffusion/distributed/cfg_parallel.py:48-71) after the CFG
 * group's all_gather: out[i] = negative[i] + scale * (positive[i] - negative[i]) over n elements,
 * with torch eager rounding: for dtype VOMNI_CFG_BF16 every step is computed in fp32 and rounded to
 * bf16 (difference, product, sum), for VOMNI_CFG_F32 in fp32 without contraction. out may alias
 * positive or negative. */
#define VOMNI_CFG_F32 0
#define VOMNI_CFG_BF16 1
VOMNI_API int vomni_cfg_combine(const void* positive, const void* negative, void* out, long long n, int dtype,
                                float scale, vomni_stream_t stream);

/* ------------------------------------------------------------------ context-parallel ring
 * Replaces the ring driver of ring_attention_const_max_fwd(num_workers = N > 1)
 * (ring_attention_const_max_fwd.py:1196-1205 all_reduce(max) of the key norm, :1287-1398 K/V
 * rotation and per-step accumulation) and its replica-group registration
 * (diffusion/distributed/parallel_state.py:180-188, 355-415).
 *
 * One vomni_ring per CP group per process (one process per GPU). Creation is collective over the
 * group: every rank calls it with the same NCCL unique id (rank 0 makes it with
 * vomni_nccl_unique_id and the host broadcasts the bytes) and the same (b, s_max, h, d); it creates
 * an NCCL communicator, allocates the registered send buffer (exported to the peers by CUDA IPC),
 * the gather buffer and the workspace. Every call of vomni_ring_attention is collective too, in the
 * same order on every rank. */
typedef struct vomni_ring vomni_ring;

VOMNI_API int vomni_nccl_unique_id(void* out, size_t bytes);
VOMNI_API int vomni_ring_create(vomni_ring** out, int rank, int world, const void* nccl_id, size_t id_bytes, int b,
                                int s_max, int h, int d);
VOMNI_API int vomni_ring_destroy(vomni_ring* ring);
/* VOMNI_OK, or VOMNI_ENCCL / VOMNI_ESTATE once the communicator reported an asynchronous error. */
VOMNI_API int vomni_ring_check(vomni_ring* ring);
/* q, k, v: this rank's token-major [b, s_loc, h, d] shard (s_loc <= s_max). out: head-major
 * [b, h, s_loc, d] or d-major with VOMNI_CM_OUT_DMAJOR; lse with VOMNI_CM_LSE.
 * Stream-ordered on `stream`: publishes K/V (on an internal copy stream, overlapping the norms),
 * runs the norms and the key-max all-reduce, pulls the peers' blocks on an internal copy stream
 * and runs the attention passes; passes after the first start as programmatic dependents of
 * the previous pass and wait inside the kernel (bounded) for the ready words of all their blocks.
 * Before returning (also on an error) `stream` joins the copy streams. */
VOMNI_API int vomni_ring_attention(vomni_ring* ring, const void* q, const void* k, const void* v, void* out, float* lse,
                                   int b, int s_loc, int h, int d, float softmax_scale, int flags,
                                   vomni_stream_t stream);
VOMNI_API int vomni_ring_attention_strided(vomni_ring* ring, const void* q, const void* k, const void* v, void* out,
                                           float* lse, int b, int s_loc, int h, int d, long long q_stride,
                                           long long kv_stride, float softmax_scale, int flags, vomni_stream_t stream);
/* Pass plan (host-only, no GPU): pass 0 is the local block; pass i >= 1 covers gather slots
 * [first[i], first[i] + count[i]) with counts 1, 2, 4, ...; slot j holds ring step j + 1.
 * Returns the number of passes, or a negative status. */
VOMNI_API int vomni_ring_phase_plan(int world, int* first, int* count, int max_phases);
/* Rank whose block ring step `step` consumes on `rank`: (rank - step) mod world (the reference's
 * collective_permute forwards each block to the next rank, ring_attention_const_max_fwd.py:130-144). */
VOMNI_API int vomni_ring_source_rank(int rank, int world, int step);

/* Allocation-free single-rank const-max attention. No counterpart in the reference: it exists for
 * callers that cannot allocate device memory — a plugin running inside a host runtime that owns the
 * whole device heap, or a latency-critical path that must not take cudaMalloc's implicit device
 * synchronisation. Same computation and arguments as vomni_cm_attention_local, but the prologue
 * scratch lives in a library-owned static device array of 8 MiB (held on every device that loads
 * the library until the process exits), so the call allocates nothing; the caller still passes
 * q, k, v, out (and lse). Limit: vomni_cm_workspace_bytes(b, s, h, d) <= 8 MiB (about
 * b*h*s <= 2.09 million query rows); larger shapes return VOMNI_EWORKSPACE.
 * The first call on a device (and the first after a cudaDeviceReset of it) looks up the array's
 * device address with that device current and caches it; make that first call before any stream
 * capture. All calls share the one array and it keeps the last
 * call's contents (the key-max slots are cleared by each call before use): calls that overlap on
 * the GPU (different streams, or threads without ordering) race on it. */
VOMNI_API int vomni_cm_attention_local_noalloc(const void* q, const void* k, const void* v, void* out, float* lse, int b,
                                               int s, int h, int d, float softmax_scale, int flags,
                                               vomni_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* VOMNI_B200_H */
