// Backward of the STFT framing used by the multi-resolution STFT loss.
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

}  // namespace
}  // namespace pmb

using namespace pmb;

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
