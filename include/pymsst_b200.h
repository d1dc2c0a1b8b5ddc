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

/* Largest band count accepted by the ragged (per-band) kernels. */
#define PMB_MAX_BANDS 128

/* Library version string, e.g. "0.1.0". */
PMB_API const char* pmb_version(void);

/* Message describing the last failed call on this host thread ("" if none). */
PMB_API const char* pmb_last_error(void);

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

#ifdef __cplusplus
}
#endif

#endif /* PYMSST_B200_H_ */
