/*
 * pymsst_b200 — C ABI of the B200 (sm_100a) kernels for the BS-RoFormer /
 * Mel-band RoFormer training hot path.
 *
 * Conventions shared by every entry point:
 *   - Tensor arguments are DEVICE pointers to densely packed row-major data
 *     unless a stride argument says otherwise.  Sizes are int64_t elements.
 *   - Element types are given by dtype codes (PMB_FLOAT32 / PMB_FLOAT16 /
 *     PMB_BFLOAT16).  All arithmetic is carried out in fp32.
 *   - Per-band arguments (widths, per-band parameter pointers) are HOST
 *     arrays; the library packs them into the kernel launch, so no device
 *     pointer tables are uploaded per call.
 *   - The library never allocates or frees device memory.  Outputs and,
 *     where a function needs one, a scratch `workspace` are supplied by the
 *     caller; the matching *_workspace_size() function gives its byte size.
 *   - Work is enqueued on `stream` (a cudaStream_t, NULL = legacy default
 *     stream); nothing synchronises the host, so calls are stream-ordered
 *     and can be captured into CUDA graphs.
 *   - Every function returns PMB_OK (0) or a negative status;
 *     pmb_last_error() then describes the failure for the calling thread.
 *
 * Each declaration names the reference interface it replaces, in
 * baicai-1145/pymsst: src/pymsst/training/cuda/fused_band_split.cpp (the
 * pybind11 bindings, ".cpp") and fused_band_split.cu (".cu").
 */
#ifndef PYMSST_B200_H_
#define PYMSST_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define PMB_API __attribute__((visibility("default")))
#else
#define PMB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define PMB_FLOAT32 0
#define PMB_FLOAT16 1
#define PMB_BFLOAT16 2

/* status codes */
#define PMB_OK 0
#define PMB_ERR_INVALID_ARGUMENT (-1)
#define PMB_ERR_UNSUPPORTED_DTYPE (-2)
#define PMB_ERR_CUDA (-3)
#define PMB_ERR_ALIGNMENT (-4)
#define PMB_ERR_WORKSPACE (-5)

/* activation codes (grouped linear epilogue) */
#define PMB_ACT_NONE 0
#define PMB_ACT_TANH 1

/* Largest band count accepted by the ragged (per-band) kernels. */
#define PMB_MAX_BANDS 128

/* Library version string, e.g. "0.1.0". */
PMB_API const char* pmb_version(void);

/* Message describing the last failed call on this host thread ("" if none). */
PMB_API const char* pmb_last_error(void);

/* Number of kernels this library has launched in the process so far. */
PMB_API uint64_t pmb_launch_count(void);

/*
 * Non-zero if a tensor-core kernel gave up a bounded wait (a pipeline stall
 * that would otherwise hang the GPU); the value encodes the wait site (low
 * 16 bits) and block.  reset != 0 clears it.  Synchronises the device.
 */
PMB_API unsigned int pmb_umma_timeout(int reset);

/* ------------------------------------------------------------------------
 * Dense GEMM on the tcgen05 tensor cores (bf16 / fp16 operands, fp32
 * accumulate):  C[m, n] = act(sum_k A(m, k) B(n, k) + bias[n])
 * A(m, k) = a[m*lda + k] (a_mn_major = 0) or a[k*lda + m] (a_mn_major = 1);
 * B(n, k) likewise.  C is written in c_dtype with row stride ldc; bias
 * (nullable) in bias_dtype.  lda/ldb must give 16-byte aligned rows.
 * Replaces the dense use of the reference's cuBLAS grouped GEMM
 * (.cu:2038-2281).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_gemm_tc(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb, int b_mn_major,
                        void* c, int64_t ldc, int c_dtype, const void* bias, int bias_dtype, int activation,
                        int64_t m, int64_t n, int64_t k, int dtype, void* stream);

/*
 * Weight-gradient GEMM on the tensor cores: C[m, n] = sum_k A[k*lda + m] *
 * B[k*ldb + n] (both operands row-major with K as the row index, e.g. an
 * output gradient and the layer input over the batch rows), written in
 * c_dtype with row stride ldc.  K is split into slices whose fp32 partials
 * are summed in a fixed order (deterministic); workspace of
 * pmb_gemm_tc_wgrad_workspace_size(m, n, k) bytes (0 when no split).
 * Replaces the weight-gradient use of the reference's cuBLAS grouped GEMM
 * (.cu:2038-2281) for dense layers.
 */
PMB_API int64_t pmb_gemm_tc_wgrad_workspace_size(int64_t m, int64_t n, int64_t k);
PMB_API int pmb_gemm_tc_wgrad(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                              int64_t k, void* c, int64_t ldc, int c_dtype, int dtype, void* workspace,
                              int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * RMSNorm over the last dimension (transformer RMSNorm, F.normalize form):
 *   inv_norm[r] = 1 / max(||x[r,:]||_2, 1e-12)
 *   normed[r,d] = x[r,d] * inv_norm[r] * sqrt(dim)
 *   out[r,d]    = normed[r,d] * gamma[d]
 * `normed` may be NULL (the backward can recompute it from x).
 * `normed` is written in out_dtype.  inv_norm is fp32 [rows].
 * Replaces rms_norm_forward / rms_norm_forward_fp32_gamma /
 * rms_norm_forward_mixed (.cpp:434-444, .cpp:469-479, .cpp:500-510;
 * kernels .cu:1211-1249, .cu:1400-1436, .cu:1589-1625).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_rms_norm_forward(const void* x, const void* gamma, void* out, void* normed, float* inv_norm,
                         int64_t rows, int64_t dim, int x_dtype, int gamma_dtype, int out_dtype,
                         void* stream);

/* Scratch bytes needed by pmb_rms_norm_backward for (rows, dim). */
PMB_API int64_t pmb_rms_norm_backward_workspace_size(int64_t rows, int64_t dim);

/*
 * RMSNorm backward.  `saved` is either the saved `normed` tensor
 * (saved_is_input = 0, reference convention) or the forward input x
 * (saved_is_input = 1; normed is recomputed as x * inv_norm * sqrt(dim)).
 *   g        = grad_out * gamma
 *   grad_x   = inv_norm * (g * sqrt(dim) - normed * (sum_d g*normed) / sqrt(dim))
 *   grad_gamma[d] = sum_r grad_out[r,d] * normed[r,d]     (deterministic)
 * grad_out and saved share grad_dtype.  grad_x may be NULL.
 * Replaces rms_norm_backward / _fp32_gamma / _mixed (.cpp:446-458,
 * .cpp:481-498, .cpp:512-537; kernels .cu:1252-1315, .cu:1439-1504,
 * .cu:1628-1691).
 */
PMB_API int pmb_rms_norm_backward(const void* grad_out, const void* saved, int saved_is_input,
                          const float* inv_norm, const void* gamma, void* grad_x, void* grad_gamma,
                          int64_t rows, int64_t dim, int grad_dtype, int gamma_dtype,
                          int grad_x_dtype, int grad_gamma_dtype, void* workspace,
                          int64_t workspace_bytes, void* stream);

/* The same backward for a pre-norm residual block y = x + f(norm(x)):
 *   grad_x += grad_residual   (grad_residual: [rows, dim] in grad_x_dtype, the
 * gradient reaching x through the residual branch; NULL adds nothing), in the
 * pass that writes grad_x, so the two gradients of x are not summed by a
 * separate elementwise pass (the reference's Transformer blocks,
 * fused_roformer.py:793-818 and pymss-core's `x = attn(x) + x; x = ff(x) + x`).
 * grad_x must not be NULL when grad_residual is given, and the two must not
 * overlap. */
PMB_API int pmb_rms_norm_backward_add(const void* grad_out, const void* saved, int saved_is_input,
                                      const float* inv_norm, const void* gamma, const void* grad_residual,
                                      void* grad_x, void* grad_gamma, int64_t rows, int64_t dim, int grad_dtype,
                                      int gamma_dtype, int grad_x_dtype, int grad_gamma_dtype, void* workspace,
                                      int64_t workspace_bytes, void* stream);

/*
 * pmb_rms_norm_backward for callers that cannot allocate device memory for
 * the call (a program binding this C ABI from another language with no
 * device allocator of its own, or a loop that must not allocate mid-step
 * because cudaMalloc / cudaFree synchronise the device).  Same arguments and
 * results as pmb_rms_norm_backward minus the workspace: the grad_gamma
 * partial sums live in a fixed 2.3 MiB array inside the library, held on
 * every GPU that loads it until exit.  dim <= 1024 (larger: PMB_ERR_WORKSPACE).
 * The first call on a device looks up the array's address there; make it
 * before capturing work on the stream.  All calls on a device share the
 * array (it keeps the last call's contents; each call rewrites what it
 * reads), so calls that overlap on the GPU race: issue them in order on one
 * stream.  No counterpart in the reference.
 */
PMB_API int pmb_rms_norm_backward_noalloc(const void* grad_out, const void* saved, int saved_is_input,
                                          const float* inv_norm, const void* gamma, void* grad_x,
                                          void* grad_gamma, int64_t rows, int64_t dim, int grad_dtype,
                                          int gamma_dtype, int grad_x_dtype, int grad_gamma_dtype,
                                          void* stream);

/* ------------------------------------------------------------------------
 * Interleaved-pair rotary embedding on t[B, N, H, D] (bnhd layout):
 *   (t[2i], t[2i+1]) -> (t[2i] c - t[2i+1] s, t[2i+1] c + t[2i] s),
 *   c = cos[n, i], s = sin[n, i] with cos/sin of shape [N, D/2].
 * backward applies the inverse rotation to grad_out.
 * cos/sin share the tensor dtype.  `out` must not overlap `t`.
 * Replaces rotary_forward / rotary_backward (.cpp:390-430; kernels
 * .cu:1077-1128).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_rotary_forward(const void* t, const void* cos, const void* sin, void* out, int64_t batch,
                       int64_t seq_len, int64_t heads, int64_t dim, int dtype, void* stream);
PMB_API int pmb_rotary_backward(const void* grad_out, const void* cos, const void* sin, void* grad_t,
                        int64_t batch, int64_t seq_len, int64_t heads, int64_t dim, int dtype,
                        void* stream);

/* ------------------------------------------------------------------------
 * BandSplit forward: per-band RMSNorm + per-band Linear(I_b -> O).
 * Band b covers features [off_b, off_b + widths[b]) of a row, off_b the
 * prefix sum of widths.  Element (row m, band b, feature i) of x is read at
 * element offset
 *   m*x_stride_row + (off_b + i)*x_stride_feat          if x_stride_band < 0
 *                                                        (ragged layout),
 *   m*x_stride_row + b*x_stride_band + i*x_stride_feat   otherwise (grouped
 *                                                        layout, equal widths).
 * Per band (host arrays of device pointers): gammas[b] [I_b],
 * weights[b] [O, I_b] row-major, biases (array may be NULL; entries may be
 * NULL) [O].  Outputs: out [rows, num_bands, O]; normed [rows, total]
 * (nullable) = x*inv*sqrt(I_b); inv_norm fp32 [rows, num_bands].
 * x, out, normed are in `dtype`; the per-band parameters (and, in the
 * backward, their gradients) are in `param_dtype`, which is `dtype` or fp32
 * (fp32 master weights read directly under mixed precision).
 * Replaces band_split_forward (.cpp:141-170; .cu:14-123) and
 * band_split_ragged_forward (.cpp:271-314; .cu:590-739).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_band_split_forward(const void* x, int64_t rows, int64_t x_stride_row, int64_t x_stride_band,
                                   int64_t x_stride_feat, int num_bands, const int64_t* widths,
                                   const void* const* gammas, const void* const* weights,
                                   const void* const* biases, int64_t out_features, void* out, void* normed,
                                   float* inv_norm, int dtype, int param_dtype, void* stream);

/* Scratch bytes for pmb_band_split_backward (need_grad_x: grad_x requested). */
PMB_API int64_t pmb_band_split_backward_workspace_size(int64_t rows, int num_bands, const int64_t* widths,
                                                       int64_t out_features, int need_grad_x);

/*
 * BandSplit backward from grad_out [rows, num_bands, O], normed
 * [rows, total] and inv_norm [rows, num_bands]:
 *   grad_weights[b] [O, I_b] = grad_out_b^T (normed_b * gamma_b)
 *   grad_gammas[b]  [I_b]    = sum_m (grad_out_b W_b)[m,:] * normed_b[m,:]
 *   grad_biases[b]  [O]      = sum_m grad_out_b[m,:]      (array may be NULL)
 *   grad_x [rows, total]     = RMSNorm input gradient    (nullable: skipped)
 * All reductions are deterministic (no atomics).
 * Replaces band_split_backward / _v2 / _v3 (.cpp:172-269; .cu:126-587) and
 * band_split_ragged_backward (.cpp:316-356; .cu:742-1003).
 */
PMB_API int pmb_band_split_backward(const void* grad_out, const void* normed, const float* inv_norm, int64_t rows,
                                    int num_bands, const int64_t* widths, const void* const* gammas,
                                    const void* const* weights, int64_t out_features, void* grad_x,
                                    void* const* grad_gammas, void* const* grad_weights, void* const* grad_biases,
                                    int dtype, int param_dtype, void* workspace, int64_t workspace_bytes,
                                    void* stream);

/* ------------------------------------------------------------------------
 * For every remaining band-wise entry point, `dtype` types the activations
 * and `param_dtype` the weights / biases and their gradients; param_dtype is
 * `dtype` (reference convention) or fp32 (mixed precision on fp32 masters).
 *
 * Grouped linear, groups of equal shape (MaskEstimator hidden layers):
 *   out[m, g, :] = act(x[m, g, :] W_g^T + bias_g),  act = none | tanh
 * x element (m, g, i) at m*x_stride_row + g*x_stride_group + i*x_stride_feat;
 * weights[g] [O, I], biases[g] [O] (array may be NULL), out [rows, G, O];
 * G <= PMB_MAX_BANDS (per-group pointers, as the per-band Linear modules
 * hold them; a packed [G, O, I] weight is passed as G row pointers).
 * Replaces grouped_linear_forward (.cpp:358-388; .cu:1006-1074), and with
 * activation = PMB_ACT_TANH fuses the hidden-layer Tanh that the reference
 * applies separately (fused_roformer.py:527-553).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_grouped_linear_forward(const void* x, int64_t rows, int64_t groups, int64_t in_features,
                                       int64_t out_features, int64_t x_stride_row, int64_t x_stride_group,
                                       int64_t x_stride_feat, const void* const* weights,
                                       const void* const* biases, void* out, int activation, int dtype,
                                       int param_dtype, void* stream);
PMB_API int64_t pmb_grouped_linear_backward_workspace_size(int64_t rows, int64_t groups, int64_t out_features);
/*
 * Backward of pmb_grouped_linear_forward for contiguous x [rows, G, I]:
 * `out` is the forward output (needed for tanh'), grad_x nullable,
 * grad_weights[g] [O, I], grad_biases (array nullable) [O].  (No reference counterpart: the reference's hidden
 * layers backpropagate through torch einsum, fused_roformer.py:1042-1048.)
 */
PMB_API int pmb_grouped_linear_backward(const void* grad_out, const void* x, const void* out, int64_t rows,
                                        int64_t groups, int64_t in_features, int64_t out_features,
                                        const void* const* weights, void* grad_x, void* const* grad_weights,
                                        void* const* grad_biases, int activation, int dtype, int param_dtype,
                                        void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * MaskEstimator final layer: per-band Linear(H -> 2*I_b) + GLU.
 * x [rows, num_bands, H]; weights[b] [2*I_b, H]; biases[b] [2*I_b]
 * (the reference's flat [2*total] bias is passed as per-band pointers);
 *   pre[m, 2*off_b + j] = x[m,b,:] . W_b[j,:] + bias_b[j]
 *   out[m, off_b + l]   = pre[m, 2*off_b + l] * sigmoid(pre[m, 2*off_b + I_b + l])
 * out [rows, total], pre [rows, 2*total] (saved for the backward).
 * Replaces mask_estimator_final_direct_forward / mask_estimator_final_forward
 * (.cpp:560-693; .cu:2284-2420, .cu:2516-2553, .cu:2706-2760).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_mask_estimator_final_forward(const void* x, int64_t rows, int num_bands, int64_t hidden,
                                             const int64_t* widths, const void* const* weights,
                                             const void* const* biases, void* out, void* pre, int dtype,
                                             int param_dtype, void* stream);
PMB_API int64_t pmb_mask_estimator_final_backward_workspace_size(int64_t rows, int num_bands, const int64_t* widths);
/*
 * Backward: grad_out [rows, total] -> grad_x [rows, num_bands, H],
 * grad_biases[b] [2*I_b], grad_weights[b] [2*I_b, H].
 * Replaces mask_estimator_final_direct_backward / mask_estimator_final_backward
 * (.cpp:591-729; .cu:2556-2704, .cu:2422-2513, .cu:2762-2851).
 */
PMB_API int pmb_mask_estimator_final_backward(const void* grad_out, const void* x, const void* pre, int64_t rows,
                                              int num_bands, int64_t hidden, const int64_t* widths,
                                              const void* const* weights, void* grad_x, void* const* grad_biases,
                                              void* const* grad_weights, int dtype, int param_dtype,
                                              void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Attention output gate (per head):
 *   gate[r, h] = sigmoid(x[r,:] . weight[h,:] + bias[h])      [rows, H]
 *   out[r, h*Dh + d] = attn(r, h, d) * gate[r, h]              [rows, H*Dh]
 * attn element (r, h, d) at
 *   bi*attn_stride_batch + n*attn_stride_seq + h*attn_stride_head + d,
 * with r = (o*seq_len + n)*seq_inner + i and bi = o*seq_inner + i (seq_inner
 * = 1: r = bi*seq_len + n), so the [batch, H, seq, Dh] attention output is
 * read in place and x / out may stay in an axial transformer's other order.
 * x [rows, dim], weight [H, dim], bias [H]; H <= 16.
 * Replaces attention_gate_forward (.cpp:539-561; .cu:1778-1824, .cu:1922-1970).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_attention_gate_forward(const void* attn, int64_t seq_len, int64_t attn_stride_batch,
                                       int64_t attn_stride_seq, int64_t attn_stride_head, const void* x,
                                       const void* weight, const void* bias, int64_t rows, int64_t heads,
                                       int64_t dim_head, int64_t dim, void* out, void* gate, int dtype,
                                       int param_dtype, int64_t seq_inner, void* stream);
PMB_API int64_t pmb_attention_gate_backward_workspace_size(int64_t rows, int64_t heads, int64_t dim);
/*
 * Backward: grad_out [rows, H*Dh] -> grad_attn (written with the attn
 * strides), grad_x [rows, dim], grad_weight [H, dim], grad_bias [H].
 * Replaces attention_gate_backward (.cpp:563-591; .cu:1826-1920, .cu:1972-2036).
 */
PMB_API int pmb_attention_gate_backward(const void* grad_out, const void* attn, int64_t seq_len,
                                        int64_t attn_stride_batch, int64_t attn_stride_seq,
                                        int64_t attn_stride_head, const void* x, const void* weight,
                                        const void* gate, int64_t rows, int64_t heads, int64_t dim_head,
                                        int64_t dim, void* grad_attn, void* grad_x, void* grad_weight,
                                        void* grad_bias, int dtype, int param_dtype, void* workspace,
                                        int64_t workspace_bytes, int64_t seq_inner, void* stream);

/* ------------------------------------------------------------------------
 * Band index kernels between the STFT and the band feature layouts
 * (Mel-band RoFormer overlapping bands; identity index for BS-RoFormer).
 *   stft  fp32 [B, S, F, T, 2]  (torch.stft of [B*S, L] audio, as real)
 *   feats      [B, T, J, 2]     J = pairs, index[j] = f*S + s (int32)
 *   inv_ptr int32 [F*S + 1], inv_idx int32 [J]: CSR inverse of index.
 * gather:    feats[b,t,j,:] = stft[b, s_j, f_j, t, :]; the gather's rows (one
 *            per (b, t)) are x_ld elements apart (0 = 2 J; a multiple of 8
 *            gives the 16-byte rows pmb_band_split_tc_forward reads in place)
 * recombine: out[b,n,s,f,t] = (stft[b,s,f,t] if multiply_stft else 1) *
 *            sum_{j in inv(f*S+s)} mask[b,n,t,j] / max(count, 1e-8)   (complex)
 * (pymss-core MelBandRoformer gather `stft_repr[batch, freq_indices]` and
 * scatter_add_ / num_bands_per_freq average, which have no pymsst CUDA
 * counterpart; reached via fused_roformer.py:827-873.)
 * ---------------------------------------------------------------------- */
PMB_API int pmb_band_gather_forward(const float* stft, const int* index, int64_t batch, int64_t channels,
                                    int64_t freqs, int64_t frames, int64_t pairs, void* x, int64_t x_ld,
                                    int x_dtype, void* stream);
PMB_API int pmb_band_gather_backward(const void* grad_x, const int* inv_ptr, const int* inv_idx, int64_t batch,
                                     int64_t channels, int64_t freqs, int64_t frames, int64_t pairs,
                                     float* grad_stft, int x_dtype, void* stream);
PMB_API int pmb_band_recombine_forward(const void* mask, const float* stft, const int* inv_ptr,
                                       const int* inv_idx, int64_t batch, int64_t stems, int64_t channels,
                                       int64_t freqs, int64_t frames, int64_t pairs, int multiply_stft,
                                       float* out, int mask_dtype, void* stream);
/* grad_mask [B, N, T, J, 2] from grad_out [B, N, S, F, T, 2] (fp32). */
PMB_API int pmb_band_recombine_backward(const float* grad_out, const float* stft, const int* index,
                                        const int* inv_ptr, int64_t batch, int64_t stems, int64_t channels,
                                        int64_t freqs, int64_t frames, int64_t pairs, int multiply_stft,
                                        void* grad_mask, int mask_dtype, void* stream);

/* ------------------------------------------------------------------------
 * Attention input projection split with rotary embedding (training path).
 *   qkv [B*N, 3, H, Dh] (= x W_qkv^T)  ->  q, k, v [B, H, N, Dh]
 * q and k are rotated (if rotate_qk) by cos/sin fp32 [N, Dh/2]:
 *   (e, o) -> (e c - o s, o c + e s)   on interleaved pairs.
 * merge is the backward: grad_q/k/v [B, H, N, Dh] -> grad_qkv [B*N, 3*H*Dh]
 * with the inverse rotation; the three gradients share the element strides
 * (stride_batch, stride_head, stride_seq) with Dh contiguous, so both the
 * [B, H, N, Dh] and the [B, N, H, Dh] layouts are read in place.
 * seq_inner (>= 1, divides B) orders the qkv rows as (outer, position,
 * inner): sequence = outer * seq_inner + inner index.  1 is the plain
 * [B, N] row order; an axial transformer passes the other axis' extent so its
 * activations never need a permuted copy.  Replaces qkv_to_bnhd +
 * rotary_forward / rotary_backward on q and k (fused_roformer.py:710-732,
 * 793-818; .cu:1077-1168) with one pass each way.
 * ---------------------------------------------------------------------- */
PMB_API int pmb_qkv_rotary_split(const void* qkv, const float* cos, const float* sin, int64_t batch,
                                 int64_t seq_len, int64_t heads, int64_t dim_head, void* q, void* k, void* v,
                                 int rotate_qk, int dtype, int64_t seq_inner, void* stream);
PMB_API int pmb_qkv_rotary_merge(const void* grad_q, const void* grad_k, const void* grad_v, const float* cos,
                                 const float* sin, int64_t batch, int64_t seq_len, int64_t heads,
                                 int64_t dim_head, void* grad_qkv, int rotate_qk, int dtype, int64_t stride_batch,
                                 int64_t stride_head, int64_t stride_seq, int64_t seq_inner, void* stream);

/*
 * Attention input projection with the rotary embedding fused into the GEMM
 * epilogue (bf16 / fp16, tcgen05): x [B*N, dim] and weight [3*H*Dh, dim] in
 * the activation dtype; q, k, v each [B*N, H*Dh] (= the [B, N, H, Dh]
 * layout) = the three thirds of x weight^T, q and k rotated as in
 * pmb_qkv_rotary_split (each projection value rounded to the activation
 * dtype before rotation).  The angle tables are TRANSPOSED here:
 * cos_t / sin_t fp32 [Dh/2, N].  x rows follow the seq_inner row order of
 * pmb_qkv_rotary_split; the planes are always [sequence, N, H, Dh].
 * dim % 8 == 0, Dh % 32 == 0.  The backward
 * is pmb_qkv_rotary_merge (which reads this layout in place) plus the two
 * projection GEMMs.  Replaces to_qkv + qkv_to_bnhd + rotary_forward
 * (fused_roformer.py:710-732, 793-818; .cu:1077-1128).
 */
PMB_API int pmb_qkv_linear_rotary_forward(const void* x, const void* weight, const float* cos_t,
                                          const float* sin_t, int64_t batch, int64_t seq_len, int64_t dim,
                                          int64_t heads, int64_t dim_head, void* q, void* k, void* v,
                                          int rotate_qk, int dtype, int64_t seq_inner, void* stream);

/* ------------------------------------------------------------------------
 * GELU (exact erf form of torch.nn.GELU()) and column sums for the
 * transformer feed-forward block, 16-bit or fp32 tensors:
 *   pmb_gelu_forward:  y = x * Phi(x) over n elements (16-byte aligned).
 *   pmb_gelu_backward: grad_in = grad_out * (Phi(x) + x phi(x)) on [rows,
 *     cols]; with grad_bias non-NULL also its column sums (the bias gradient
 *     of the Linear before the GELU) in bias_dtype.
 *   pmb_column_sum:    out[c] = sum_r x[r, c] (a Linear's bias gradient).
 * cols must be a multiple of 16 bytes' worth of elements; workspace of
 * pmb_rows_pass_workspace_size(rows, cols) bytes.  No counterpart in the
 * reference's extension (torch runs GELU and the bias reductions there).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_gelu_forward(const void* x, void* y, int64_t n, int dtype, void* stream);
PMB_API int64_t pmb_rows_pass_workspace_size(int64_t rows, int64_t cols);
PMB_API int pmb_gelu_backward(const void* grad_out, const void* x, void* grad_in, int64_t rows, int64_t cols,
                              void* grad_bias, int bias_dtype, int dtype, void* workspace, int64_t workspace_bytes,
                              void* stream);
PMB_API int pmb_column_sum(const void* x, int64_t rows, int64_t cols, void* out, int out_dtype, int dtype,
                           void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Transformer feed-forward block on the tcgen05 tensor cores (bf16 / fp16
 * activations; parameters fp32 or the activation dtype):
 *   pre = x w1^T + b1,  act = gelu(pre) (exact erf form),  out = act w2^T + b2
 * x [rows, dim]; w1 [hidden, dim] and w2 [dim, hidden] in the activation
 * dtype (operands of the tensor cores); b1, b2 in param_dtype.  pre and act
 * [rows, hidden] are saved for the backward.  The backward writes grad_x
 * (nullable, activation dtype) and the four parameter gradients in
 * param_dtype, using a workspace of
 * pmb_feed_forward_backward_workspace_size bytes.  dim, hidden % 8 == 0.
 * No counterpart in the reference's extension: the reference runs this
 * block of every transformer layer through torch (Linear, GELU, Linear).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_feed_forward_forward(const void* x, const void* w1, const void* b1, const void* w2, const void* b2,
                                     int64_t rows, int64_t dim, int64_t hidden, void* pre, void* act, void* out,
                                     int dtype, int param_dtype, void* stream);
PMB_API int64_t pmb_feed_forward_backward_workspace_size(int64_t rows, int64_t dim, int64_t hidden, int dtype);
PMB_API int pmb_feed_forward_backward(const void* grad_out, const void* x, const void* pre, const void* act,
                                      const void* w1, const void* w2, int64_t rows, int64_t dim, int64_t hidden,
                                      void* grad_x, void* grad_w1, void* grad_b1, void* grad_w2, void* grad_b2,
                                      int dtype, int param_dtype, void* workspace, int64_t workspace_bytes,
                                      void* stream);

/* ------------------------------------------------------------------------
 * BandSplit on the tcgen05 tensor cores (bf16 / fp16 activations; fp32 or
 * activation-dtype parameters), same math as pmb_band_split_forward:
 *   out[m, b, :] = (x_b * inv * sqrt(w_b) * gamma_b) W_b^T + bias_b,
 * computed as s[m, b] * (x_b (W_b * gamma_b)^T) + bias_b with the row scale
 * s = inv * sqrt(w_b) applied in the GEMM epilogue, so x is read in place.
 * x [rows, total] with row stride x_ld: x 16-byte aligned and x_ld a multiple
 * of sizes[2] (8) elements, >= total.  inv_norm [rows, nb] fp32 is written by
 * the forward and read by the backward (with x).  `packed_weights` (sizes[0]
 * bytes) receives W_b * gamma_b in the activation dtype, bands whose columns
 * share one 64-wide k-block packed block-diagonally into one weight group.
 * The backward produces the parameter gradients (grad_biases nullable) and
 * needs a 256-byte aligned workspace of sizes[1] bytes; the band features'
 * own gradient is not produced (use pmb_band_split_backward when the input
 * needs one).  sizes[3] = number of weight groups.  out_features must be a
 * multiple of 64.  Replaces the ragged band split's forward / weight backward
 * (.cu:590-1003).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_band_split_tc_sizes(int64_t rows, int num_bands, const int64_t* widths, int64_t out_features,
                                    int dtype, int64_t* sizes);
PMB_API int pmb_band_split_tc_forward(const void* x, int64_t rows, int64_t x_ld, int num_bands,
                                      const int64_t* widths, const void* const* gammas, const void* const* weights,
                                      const void* const* biases, int64_t out_features, void* packed_weights,
                                      float* inv_norm, void* out, int dtype, int param_dtype, void* stream);
PMB_API int pmb_band_split_tc_backward(const void* grad_out, const void* x, int64_t x_ld, const float* inv_norm,
                                       int64_t rows, int num_bands, const int64_t* widths, const void* const* gammas,
                                       const void* const* weights, int64_t out_features, void* const* grad_gammas,
                                       void* const* grad_weights, void* const* grad_biases, int dtype,
                                       int param_dtype, void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * MaskEstimator MLP on the tcgen05 tensor cores (training path, bf16/fp16
 * activations, fp32 or 16-bit parameters): per band b,
 *   h_1 = tanh(x_b W_{1,b}^T + b_{1,b}), ..., h_L (hidden_layers of them),
 *   pre_b = h_L W_{f,b}^T + b_{f,b}  (2*w_b outputs),  out_b = GLU(pre_b).
 * x [rows, nb, dim]; weights / biases: host arrays of (hidden_layers + 1)*nb
 * per-band device pointers, layer-major (W [out, in], bias [out]).
 * Caller-owned buffers, sized by pmb_mask_estimator_tc_sizes (sizes[0..4] =
 * packed-weight bytes, saved-activation bytes, pre bytes, backward workspace
 * bytes, packed width P): packed_weights (kept for the backward), acts
 * [hidden_layers, rows, nb, hidden], pre [rows, P] (GLU pre-activations in a
 * chunk-interleaved packed layout), out [rows, sum(widths)].
 * The backward writes per-band parameter gradients (fp32 when param_dtype is
 * fp32) and, if grad_x is not NULL, grad_x [rows, nb, dim].
 * Replaces the per-group grouped_linear + mask_estimator_final kernels
 * (fused_roformer.py:527-583; .cu:1006-1074, :2284-2851) with one launch
 * per layer for all bands.
 * ---------------------------------------------------------------------- */
PMB_API int pmb_mask_estimator_tc_sizes(int64_t rows, int num_bands, int64_t dim, int64_t hidden, int hidden_layers,
                                        const int64_t* widths, int64_t* sizes);
PMB_API int pmb_mask_estimator_tc_forward(const void* x, int64_t rows, int num_bands, int64_t dim, int64_t hidden,
                                          int hidden_layers, const int64_t* widths, const void* const* weights,
                                          const void* const* biases, void* packed_weights, void* acts, void* pre,
                                          void* out, int dtype, int param_dtype, void* stream);
PMB_API int pmb_mask_estimator_tc_backward(const void* grad_out, const void* x, const void* acts, const void* pre,
                                           const void* packed_weights, int64_t rows, int num_bands, int64_t dim,
                                           int64_t hidden, int hidden_layers, const int64_t* widths,
                                           void* const* grad_weights, void* const* grad_biases, void* grad_x,
                                           int dtype, int param_dtype, void* workspace, int64_t workspace_bytes,
                                           void* stream);

/* ------------------------------------------------------------------------
 * Attention core of the axial transformers on the tensor cores: softmax(
 * Q K^T * scale) V per (sequence, head), head dim 64, bf16/fp16, no mask, no
 * dropout.  q, k, v, o (and grad_out, grad_q, grad_k, grad_v) are
 * [sequences, seq_len, heads, 64] planes given by a base pointer and three
 * element strides (sequence, position, head) each, all multiples of 8 with
 * the 64 head elements contiguous; `strides` holds them plane by plane
 * (forward: q, k, v, o = 12 values; backward: q, k, v, o, grad_out, grad_q,
 * grad_k, grad_v = 24 values).  lse: fp32 [sequences * heads, ld] with
 * ld = pmb_attention_row_pitch(seq_len) (seq_len rounded up to a multiple of
 * 4), 16-byte aligned: the natural-log row sums written by the forward and
 * read by the backward.  The backward needs
 * pmb_attention_backward_workspace_size bytes of 16-byte aligned workspace
 * (the row sums D = rowsum(grad_out * o), same layout) and is deterministic.
 * Replaces torch.nn.functional.scaled_dot_product_attention in pymss-core's
 * Attention module, whose backend the reference selects with
 * cuda_attention_backend (src/pymsst/training/module.py:96-107, :416-425).
 * ---------------------------------------------------------------------- */
PMB_API int64_t pmb_attention_row_pitch(int64_t seq_len);
PMB_API int pmb_attention_forward(const void* q, const void* k, const void* v, void* o, float* lse,
                                  int64_t sequences, int64_t seq_len, int64_t heads, int64_t dim_head,
                                  const int64_t* strides, float scale, int dtype, void* stream);
PMB_API int64_t pmb_attention_backward_workspace_size(int64_t sequences, int64_t seq_len, int64_t heads);
PMB_API int pmb_attention_backward(const void* q, const void* k, const void* v, const void* o, const void* grad_out,
                                   const float* lse, void* grad_q, void* grad_k, void* grad_v, int64_t sequences,
                                   int64_t seq_len, int64_t heads, int64_t dim_head, const int64_t* strides,
                                   float scale, int dtype, void* workspace, int64_t workspace_bytes, void* stream);
/* The same backward with the rotary embedding's inverse rotation applied to
 * grad_q and grad_k before they are stored: with cos / sin the fp32 angle
 * tables [seq_len, dim_head / 2] (16-byte aligned) the forward rotated q and
 * k with ((e, o) -> (e c - o s, o c + e s) on interleaved pairs), the
 * gradients come out as those of the unrotated projections ((e, o) ->
 * (e c + o s, o c - e s)).  With grad_q / grad_k / grad_v given as strided
 * views of the [rows, 3 * heads * dim_head] projection gradient, this
 * writes that gradient directly, replacing the attention backward plus
 * pmb_qkv_rotary_merge for sequences stored in row order (the reference's
 * rotary backward, src/pymsst/training/cuda/fused_band_split.cu:1104-1128,
 * applied after the attention backward of fused_roformer.py:793-818). */
/* Attention with the BS-/Mel-RoFormer head gate folded in (sequences of up
 * to 64 positions, the band axis): gated = softmax(q k^T scale) v *
 * sigmoid(gate_logits[seq * seq_len + pos, head]) written in place of o
 * (gate_logits: [sequences * seq_len, heads] in the activation type, rows
 * in sequence order).  The backward takes the gated output and its gradient
 * where pmb_attention_backward_rotary takes o and grad_out (dO = gate *
 * grad_gated), writes dQ / dK (rotated back when cos / sin are given; both
 * NULL otherwise) and dV, and the gate logits' gradient
 * grad_logits[row * grad_logits_ld + head] = rowsum(grad_gated * gated) *
 * (1 - gate); all in one pass.  With grad_bias_partials (fp32,
 * pmb_attention_gate_bias_partials(sequences, heads) values, or NULL) it also
 * writes the sums of the stored logit gradients over groups of 32 rows:
 * partial[(pair * heads + head) * 4 + quarter], pair = sequence / 2, whose
 * sum over pairs and quarters is the gate bias gradient of each head.  Replaces the attention core plus the separate
 * gate pass of the patched Attention.forward
 * (src/pymsst/training/fused_roformer.py:793-818; gate kernels
 * cuda/fused_band_split.cu:1778-2036). */
PMB_API int pmb_attention_forward_gated(const void* q, const void* k, const void* v, const void* gate_logits,
                                        void* gated, float* lse, int64_t sequences, int64_t seq_len, int64_t heads,
                                        int64_t dim_head, const int64_t* strides, float scale, int dtype,
                                        void* stream);
PMB_API int64_t pmb_attention_gate_bias_partials(int64_t sequences, int64_t heads);
PMB_API int pmb_attention_backward_gated(const void* q, const void* k, const void* v, const void* gated,
                                         const void* grad_gated, const float* lse, const void* gate_logits,
                                         const float* cos, const float* sin, void* grad_q, void* grad_k,
                                         void* grad_v, void* grad_logits, int64_t grad_logits_ld,
                                         float* grad_bias_partials, int64_t sequences, int64_t seq_len,
                                         int64_t heads, int64_t dim_head, const int64_t* strides, float scale,
                                         int dtype, void* workspace, int64_t workspace_bytes, void* stream);
PMB_API int pmb_attention_backward_rotary(const void* q, const void* k, const void* v, const void* o,
                                          const void* grad_out, const float* lse, const float* cos, const float* sin,
                                          void* grad_q, void* grad_k, void* grad_v, int64_t sequences,
                                          int64_t seq_len, int64_t heads, int64_t dim_head, const int64_t* strides,
                                          float scale, int dtype, void* workspace, int64_t workspace_bytes,
                                          void* stream);

/* ------------------------------------------------------------------------
 * The overlap-add of torch.istft (center=True), after the inverse real FFT
 * of each frame: y[b, i] = sum_t frames[b, k, t] w[k] / env[i + n/2] with
 * k = i + n/2 - t*hop over the frames that cover that position, env the
 * overlap-added squared window, i < length (zeros past the signal's end, as
 * torch.istft pads to `length`).  frames [batch, n_fft, num_frames] fp32 at
 * any element strides (frame_strides = {batch, k, t}: the inverse FFT along
 * the frequency axis of a [F, T] spectrum leaves time fastest), window fp32
 * [n_fft] (zero-padded to n_fft, centred).  The backward writes the frames'
 * gradient grad_frames[b, k, t] (contiguous [batch, n_fft, num_frames]) =
 * grad_y[b, t*hop + k - n/2] w[k] / env (0 outside the trimmed range).  One
 * pass each, replacing the window multiply, the overlap-add, the envelope
 * division, the trim and their backward (pymss-core's torch.istft at the end
 * of the BS-/Mel-RoFormer forward, reached from
 * src/pymsst/training/module.py:221-224). */
PMB_API int pmb_istft_overlap_add_forward(const float* frames, const int64_t* frame_strides, const float* window,
                                          float* y, int64_t batch, int64_t n_fft, int64_t num_frames, int64_t hop,
                                          int64_t length, void* stream);
PMB_API int pmb_istft_overlap_add_backward(const float* grad_y, const float* window, float* grad_frames,
                                           int64_t batch, int64_t n_fft, int64_t num_frames, int64_t hop,
                                           int64_t length, void* stream);

/* ------------------------------------------------------------------------
 * One resolution of the multi-resolution STFT loss: mean |Y_recon - Y_target|
 * over `count` complex values (fp32, interleaved re / im; 16-byte aligned),
 * the F.l1_loss of two onesided spectra.  The forward writes the mean to
 * loss[0] (deterministic: per-CTA partials in the workspace,
 * pmb_spectral_l1_workspace_size bytes, summed in fp64 in a fixed order).
 * The backward writes grad_recon = grad_loss[0] * (Y_recon - Y_target) /
 * |Y_recon - Y_target| / count (0 where they agree) times the inverse real
 * FFT's bin weight (0.5 for bins strictly between 0 and n_fft / 2, `bins` =
 * n_fft / 2 + 1 per row), so an inverse real FFT of it is the gradient of the
 * frames: one pass replaces the elementwise difference, abs, mean, their
 * backward and the rfft backward's bin weighting.  grad_loss is a device
 * pointer.  Replaces F.l1_loss over torch.stft spectra in pymss-core's
 * multi-resolution STFT loss (trained unchanged by the reference,
 * src/pymsst/training/module.py:221-224). */
PMB_API int64_t pmb_spectral_l1_workspace_size(int64_t count);
PMB_API int pmb_spectral_l1_forward(const float* y_recon, const float* y_target, int64_t count, float* loss,
                                    void* workspace, int64_t workspace_bytes, void* stream);
PMB_API int pmb_spectral_l1_backward(const float* y_recon, const float* y_target, int64_t count, int64_t bins,
                                     int64_t n_fft, const float* grad_loss, float* grad_recon, void* stream);

/* ------------------------------------------------------------------------
 * STFT framing of the multi-resolution STFT loss: torch.stft (center=True,
 * reflect padding by n_fft/2) frames x [batch, length] into frames [batch,
 * frames, n_fft] = reflect_pad(x)[f*hop + k] * window[k].  The forward
 * writes those frames (fp32; window and frames 16-byte aligned, n_fft a
 * multiple of 4); the backward, given the frames' gradient (fp32, contiguous) and the window
 * (fp32, n_fft values, zero-padded to n_fft as torch.stft pads it), writes
 * grad_x [batch, length] (fp32): one overlap-add per sample, deterministic.
 * frames must equal 1 + (length + 2*(n_fft/2) - n_fft) / hop.  Replaces
 * torch.stft's index_add / reflection-pad backward in pymss-core's
 * multi_stft_resolution_loss (reached from src/pymsst/training/module.py:221-224).
 * ---------------------------------------------------------------------- */
PMB_API int pmb_stft_frames_forward(const float* x, const float* window, float* frames, int64_t batch,
                                    int64_t length, int64_t n_fft, int64_t hop, int64_t num_frames, void* stream);
PMB_API int pmb_stft_frames_backward(const float* grad_frames, const float* window, float* grad_x, int64_t batch,
                                     int64_t length, int64_t n_fft, int64_t hop, int64_t frames, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PYMSST_B200_H_ */
