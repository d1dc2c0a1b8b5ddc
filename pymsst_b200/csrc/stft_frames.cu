// STFT framing of the multi-resolution STFT loss, forward and backward.
//
// torch.stft (center=True, reflect padding) frames the signal as
//   xp = reflect_pad(x, n/2),  frame[f, k] = xp[f*hop + k] * w[k]   (k < n)
// and its gradient with respect to x is an overlap-add of the frame
// gradients, folded back through the reflection.  torch computes it with an
// atomic index_add over the frames plus an atomic reflection-pad backward;
// here one thread owns one input sample i and sums, in a fixed order, every
// frame element that read it:
//   grad_x[i] = sum over padded positions p that hold x[i]
//                 (p = i + n/2, and the mirror positions at the two edges)
//               sum over frames f with 0 <= p - f*hop < n
//                 grad_frame[f, p - f*hop] * w[p - f*hop]
// (at most ceil(n / hop) frames per position).  Deterministic, no atomics;
// consecutive threads read consecutive elements of each frame.
// Reference semantics: the loss of pymss-core's BS-/Mel-RoFormer
// (multi_stft_resolution_loss, torch.stft of the prediction), reached from
// src/pymsst/training/module.py:221-224.
#include "common.cuh"

namespace pmb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float frames_sum(const float* __restrict__ g, const float* __restrict__ w, int64_t p,
                                            int n, int hop, int T) {
  int64_t f_lo = p - n + 1 > 0 ? (p - n + hop) / hop : 0;  // ceil((p - n + 1) / hop)
  int64_t f_hi = p / hop;
  if (f_hi > T - 1) f_hi = T - 1;
  float acc = 0.f;
  for (int64_t f = f_lo; f <= f_hi; ++f) {
    const int k = (int)(p - f * hop);
    acc = fmaf(g[f * n + k], w[k], acc);
  }
  return acc;
}

__global__ void __launch_bounds__(kThreads)
    stft_frames_bwd(const float* __restrict__ grad_frames, const float* __restrict__ window, float* __restrict__ grad_x,
                    int64_t batch, int64_t L, int n, int hop, int T) {
  const int64_t pad = n / 2;
  for (int64_t idx = (int64_t)blockIdx.x * kThreads + threadIdx.x; idx < batch * L; idx += (int64_t)gridDim.x * kThreads) {
    const int64_t b = idx / L, i = idx - b * L;
    const float* g = grad_frames + b * (int64_t)T * n;
    float acc = frames_sum(g, window, i + pad, n, hop, T);
    if (i >= 1 && i <= pad) acc += frames_sum(g, window, pad - i, n, hop, T);                       // left mirror
    if (i <= L - 2 && i >= L - 1 - pad) acc += frames_sum(g, window, pad + 2 * (L - 1) - i, n, hop, T);  // right mirror
    grad_x[idx] = acc;
  }
}

// frames[b, t, k] = reflect_pad(x)[t*hop + k] * w[k] for k in a group of 4
// (one 16-byte store); groups where the (zero-padded) window is zero are
// written as zeros without reading x.
__global__ void __launch_bounds__(kThreads)
    stft_frames_fwd(const float* __restrict__ x, const float* __restrict__ window, float* __restrict__ frames,
                    int64_t batch, int64_t L, int n, int hop, int T) {
  const int64_t pad = n / 2, groups = n / 4, per_b = (int64_t)T * groups;
  for (int64_t idx = (int64_t)blockIdx.x * kThreads + threadIdx.x; idx < batch * per_b;
       idx += (int64_t)gridDim.x * kThreads) {
    const int64_t b = idx / per_b, r = idx - b * per_b, t = r / groups;
    const int k0 = (int)(r - t * groups) * 4;
    const float4 w4 = *reinterpret_cast<const float4*>(window + k0);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (w4.x != 0.f || w4.y != 0.f || w4.z != 0.f || w4.w != 0.f) {
      const float* xb = x + b * L;
      float v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        int64_t j = t * hop + k0 + q - pad;
        if (j < 0) j = -j;
        if (j >= L) j = 2 * (L - 1) - j;
        v[q] = xb[j];
      }
      o = make_float4(v[0] * w4.x, v[1] * w4.y, v[2] * w4.z, v[3] * w4.w);
    }
    *reinterpret_cast<float4*>(frames + idx * 4) = o;
  }
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_stft_frames_forward(const float* x, const float* window, float* frames, int64_t batch,
                                       int64_t length, int64_t n_fft, int64_t hop, int64_t num_frames, void* stream) {
  clear_error();
  const char* name = "pmb_stft_frames_forward";
  PMB_REQUIRE(batch >= 0 && length > 0 && n_fft > 0 && hop > 0 && num_frames > 0, "%s: bad shape", name);
  PMB_REQUIRE(n_fft % 4 == 0, "%s: n_fft must be a multiple of 4", name);
  PMB_REQUIRE(n_fft / 2 < length, "%s: reflect padding needs n_fft / 2 < length", name);
  PMB_REQUIRE(num_frames == 1 + (length + 2 * (n_fft / 2) - n_fft) / hop, "%s: frame count does not match", name);
  PMB_REQUIRE(n_fft < (1 << 30) && num_frames < (1 << 30), "%s: too large", name);
  if (batch == 0) return PMB_OK;
  PMB_REQUIRE(x && window && frames, "%s: NULL argument", name);
  PMB_REQUIRE(((reinterpret_cast<uintptr_t>(window) | reinterpret_cast<uintptr_t>(frames)) & 15) == 0,
              "%s: window and frames must be 16-byte aligned", name);
  int64_t g = (batch * num_frames * (n_fft / 4) + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  stft_frames_fwd<<<(unsigned)g, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, window, frames, batch, length, (int)n_fft, (int)hop, (int)num_frames);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

extern "C" int pmb_stft_frames_backward(const float* grad_frames, const float* window, float* grad_x, int64_t batch,
                                        int64_t length, int64_t n_fft, int64_t hop, int64_t frames, void* stream) {
  clear_error();
  const char* name = "pmb_stft_frames_backward";
  PMB_REQUIRE(batch >= 0 && length > 0 && n_fft > 0 && hop > 0 && frames > 0, "%s: bad shape", name);
  PMB_REQUIRE(n_fft / 2 < length, "%s: reflect padding needs n_fft / 2 < length", name);
  PMB_REQUIRE(frames == 1 + (length + 2 * (n_fft / 2) - n_fft) / hop, "%s: frame count does not match", name);
  PMB_REQUIRE(n_fft < (1 << 30) && frames < (1 << 30), "%s: too large", name);
  if (batch == 0) return PMB_OK;
  PMB_REQUIRE(grad_frames && window && grad_x, "%s: NULL argument", name);
  int64_t g = (batch * length + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  stft_frames_bwd<<<(unsigned)g, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      grad_frames, window, grad_x, batch, length, (int)n_fft, (int)hop, (int)frames);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}
