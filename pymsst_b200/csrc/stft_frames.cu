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

// Sum over the frames f with 0 <= p - f*hop < n of g[f][p - f*hop] * w[.],
// four frames per step with independent accumulators (the loads of a step
// are in flight together).  p, n, hop and the frame offsets fit in 32 bits.
__device__ __forceinline__ float frames_sum(const float* __restrict__ g, const float* __restrict__ w, int p, int n,
                                            int hop, int T) {
  const int f_lo = p - n + 1 > 0 ? (p - n + hop) / hop : 0;  // ceil((p - n + 1) / hop)
  int f_hi = p / hop;
  if (f_hi > T - 1) f_hi = T - 1;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int f = f_lo;
  for (; f + 3 <= f_hi; f += 4) {
    const int k0 = p - f * hop;
    const float g0 = g[f * n + k0], g1 = g[(f + 1) * n + k0 - hop], g2 = g[(f + 2) * n + k0 - 2 * hop],
                g3 = g[(f + 3) * n + k0 - 3 * hop];
    a0 = fmaf(g0, w[k0], a0);
    a1 = fmaf(g1, w[k0 - hop], a1);
    a2 = fmaf(g2, w[k0 - 2 * hop], a2);
    a3 = fmaf(g3, w[k0 - 3 * hop], a3);
  }
  for (; f <= f_hi; ++f) {
    const int k = p - f * hop;
    a0 = fmaf(g[f * n + k], w[k], a0);
  }
  return (a0 + a1) + (a2 + a3);
}

// grid (samples / 256, batch): one thread per input sample
__global__ void __launch_bounds__(kThreads)
    stft_frames_bwd(const float* __restrict__ grad_frames, const float* __restrict__ window, float* __restrict__ grad_x,
                    int L, int n, int hop, int T) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= L) return;
  const int pad = n / 2;
  const float* g = grad_frames + (int64_t)blockIdx.y * T * n;
  float acc = frames_sum(g, window, i + pad, n, hop, T);
  if (i >= 1 && i <= pad) acc += frames_sum(g, window, pad - i, n, hop, T);                    // left mirror
  if (i <= L - 2 && i >= L - 1 - pad) acc += frames_sum(g, window, pad + 2 * (L - 1) - i, n, hop, T);  // right mirror
  grad_x[(int64_t)blockIdx.y * L + i] = acc;
}

// grid (batch * frames, groups / 256): frames[b, t, k] = reflect_pad(x)[t*hop + k] * w[k] for k in a group
// of 4 (one 16-byte store); groups where the (zero-padded) window is zero are written as zeros without
// reading x.
__global__ void __launch_bounds__(kThreads)
    stft_frames_fwd(const float* __restrict__ x, const float* __restrict__ window, float* __restrict__ frames, int L,
                    int n, int hop, int T) {
  const int grp = blockIdx.y * kThreads + threadIdx.x;
  if (grp >= n / 4) return;
  const int bt = blockIdx.x, b = bt / T, t = bt - b * T, k0 = grp * 4;
  const float4 w4 = *reinterpret_cast<const float4*>(window + k0);
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (w4.x != 0.f || w4.y != 0.f || w4.z != 0.f || w4.w != 0.f) {
    const float* xb = x + (int64_t)b * L;
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int j = t * hop + k0 + q - n / 2;
      if (j < 0) j = -j;
      if (j >= L) j = 2 * (L - 1) - j;
      v[q] = xb[j];
    }
    o = make_float4(v[0] * w4.x, v[1] * w4.y, v[2] * w4.z, v[3] * w4.w);
  }
  *reinterpret_cast<float4*>(frames + (int64_t)bt * n + k0) = o;
}

// ------------------------------------------------------------------ iSTFT
// Overlap-add of the inverse-FFT frames of torch.istft (center=True):
//   y[i] = sum_t frames[t][p - t*hop] w[p - t*hop] / env[p],  p = i + n/2,
//   env[p] = sum_t w[p - t*hop]^2   (the overlap-added squared window)
// over the frames t with 0 <= p - t*hop < n, for the trimmed output i < len
// (zeros past the untrimmed end, as torch.istft pads to `length`).  The
// frames are the inverse real FFT along the frequency axis of a [F, T]
// spectrum, element (k, t) of batch b at frames[b * sb + k * sk + t * st]
// (the layout the transform returned).  One thread per output sample; the
// envelope is summed in the same loop (no buffer).
__global__ void __launch_bounds__(kThreads)
    istft_ola_fwd(const float* __restrict__ frames, int64_t sb, int64_t sk, int64_t st,
                  const float* __restrict__ window, float* __restrict__ y, int n, int T, int hop, int len) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  if (i >= len) return;
  const float* fb = frames + (int64_t)blockIdx.y * sb;
  const int p = i + n / 2;
  const int t_lo = p - n + 1 > 0 ? (p - n + hop) / hop : 0;
  int t_hi = p / hop;
  if (t_hi > T - 1) t_hi = T - 1;
  float acc = 0.f, env = 0.f;
  for (int t = t_lo; t <= t_hi; ++t) {
    const int k = p - t * hop;
    const float w = window[k];
    acc = fmaf(fb[k * sk + t * st], w, acc);
    env = fmaf(w, w, env);
  }
  y[(int64_t)blockIdx.y * len + i] = t_lo <= t_hi ? acc / env : 0.f;
}

// Its gradient with respect to the frames: each frame element (k, t) was
// added into exactly one output sample, p = t*hop + k:
//   grad_frames[k * T + t] = grad_y[p - n/2] w[k] / env[p]  (0 outside the trimmed range)
// grid (T / 256, n, batch): consecutive threads take consecutive t of one k (no index division).
__global__ void __launch_bounds__(kThreads)
    istft_ola_bwd(const float* __restrict__ grad_y, const float* __restrict__ window, float* __restrict__ grad_frames,
                  int n, int T, int hop, int len) {
  const int t = blockIdx.x * kThreads + threadIdx.x, k = blockIdx.y;
  if (t >= T) return;
  const int64_t e = (int64_t)k * T + t;
  const int p = t * hop + k, i = p - n / 2;
  float g = 0.f;
  if (i >= 0 && i < len) {
    const int t_lo = p - n + 1 > 0 ? (p - n + hop) / hop : 0;
    int t_hi = p / hop;
    if (t_hi > T - 1) t_hi = T - 1;
    float env = 0.f;
    for (int u = t_lo; u <= t_hi; ++u) {
      const float w = window[p - u * hop];
      env = fmaf(w, w, env);
    }
    g = grad_y[(int64_t)blockIdx.z * len + i] * window[k] / env;
  }
  grad_frames[(int64_t)blockIdx.z * n * T + e] = g;
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_istft_overlap_add_forward(const float* frames, const int64_t* frame_strides, const float* window,
                                             float* y, int64_t batch, int64_t n_fft, int64_t num_frames, int64_t hop,
                                             int64_t length, void* stream) {
  clear_error();
  const char* name = "pmb_istft_overlap_add_forward";
  PMB_REQUIRE(batch >= 0 && n_fft > 0 && num_frames > 0 && hop > 0 && hop <= n_fft && length > 0,
              "%s: bad shape", name);
  PMB_REQUIRE((num_frames + 1) * n_fft < ((int64_t)1 << 31) && length < (1 << 30) && batch <= 65535,
              "%s: too large", name);
  if (batch == 0) return PMB_OK;
  PMB_REQUIRE(frames && frame_strides && window && y, "%s: NULL argument", name);
  PMB_REQUIRE(frame_strides[0] >= 0 && frame_strides[1] >= 0 && frame_strides[2] >= 0, "%s: bad strides", name);
  const dim3 grid((unsigned)((length + kThreads - 1) / kThreads), (unsigned)batch);
  istft_ola_fwd<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      frames, frame_strides[0], frame_strides[1], frame_strides[2], window, y, (int)n_fft, (int)num_frames, (int)hop,
      (int)length);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

extern "C" int pmb_istft_overlap_add_backward(const float* grad_y, const float* window, float* grad_frames,
                                              int64_t batch, int64_t n_fft, int64_t num_frames, int64_t hop,
                                              int64_t length, void* stream) {
  clear_error();
  const char* name = "pmb_istft_overlap_add_backward";
  PMB_REQUIRE(batch >= 0 && n_fft > 0 && num_frames > 0 && hop > 0 && hop <= n_fft && length > 0,
              "%s: bad shape", name);
  // (num_frames + 1) * n_fft bounds the sample index t * hop + k of every frame element in 32 bits
  PMB_REQUIRE((num_frames + 1) * n_fft < ((int64_t)1 << 31) && length < (1 << 30) && batch <= 65535,
              "%s: too large", name);
  if (batch == 0) return PMB_OK;
  PMB_REQUIRE(grad_y && window && grad_frames, "%s: NULL argument", name);
  PMB_REQUIRE(n_fft <= 65535, "%s: n_fft above 65535", name);
  const dim3 grid((unsigned)((num_frames + kThreads - 1) / kThreads), (unsigned)n_fft, (unsigned)batch);
  istft_ola_bwd<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(grad_y, window, grad_frames, (int)n_fft,
                                                                          (int)num_frames, (int)hop, (int)length);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

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
  PMB_REQUIRE(batch * num_frames < ((int64_t)1 << 31) && n_fft / 4 <= 65535LL * kThreads && length < (1 << 30) &&
                  num_frames * n_fft < ((int64_t)1 << 31),
              "%s: too large", name);
  const dim3 grid((unsigned)(batch * num_frames), (unsigned)((n_fft / 4 + kThreads - 1) / kThreads));
  stft_frames_fwd<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, window, frames, (int)length,
                                                                            (int)n_fft, (int)hop, (int)num_frames);
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
  PMB_REQUIRE(batch <= 65535 && length < (1 << 30) && frames * n_fft < ((int64_t)1 << 31), "%s: too large", name);
  const dim3 grid((unsigned)((length + kThreads - 1) / kThreads), (unsigned)batch);
  stft_frames_bwd<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(grad_frames, window, grad_x, (int)length,
                                                                            (int)n_fft, (int)hop, (int)frames);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}
