// Multi-resolution STFT loss term: mean |Y_r - Y_t| over complex spectra
// (fp32, interleaved re / im), forward and backward, each one pass.
//
// Forward: every CTA sums |Y_r - Y_t| over a grid-strided share of the
// elements (two complex values per 16-byte load) into one fp32 partial; one
// CTA then adds the partials in a fixed order in fp64 and divides by the
// element count (deterministic).
// Backward: dL/dY_r = g * (Y_r - Y_t) / |Y_r - Y_t| / count (0 where the two
// agree, as torch's complex abs backward gives), with g the upstream
// gradient read from device memory (no host round trip, so the pass can sit
// in a captured graph), times the inverse-real-FFT bin weight of the caller's
// rfft backward (0.5 for the bins strictly between 0 and n_fft / 2, which an
// inverse real FFT counts twice): the gradient comes out ready for that
// transform, so the loss's backward is this pass plus the c2r FFT.
// Reference semantics: the multi-resolution STFT L1 of pymss-core's
// BS-/Mel-RoFormer loss (F.l1_loss of torch.stft spectra per resolution,
// summed and weighted), which the reference trains through unchanged
// (src/pymsst/training/module.py:221-224).
#include "common.cuh"

namespace pmb {
namespace {

constexpr int kThreads = 256;

inline int loss_grid(int64_t pairs) {
  int64_t g = (pairs + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)num_sms() * 8;
  return (int)(g > cap ? cap : (g < 1 ? 1 : g));
}

// |a - b| for one complex value
__device__ __forceinline__ float cabs_diff(float ar, float ai, float br, float bi) {
  const float dr = ar - br, di = ai - bi;
  return sqrtf(fmaf(dr, dr, di * di));
}

__global__ void __launch_bounds__(kThreads)
    l1_partial(const float4* __restrict__ yr, const float4* __restrict__ yt, int64_t pairs,
               const float2* __restrict__ yr1, const float2* __restrict__ yt1, int odd, float* __restrict__ partial) {
  __shared__ float red[kThreads / 32];
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * kThreads) {
    const float4 a = yr[i], b = yt[i];
    acc += cabs_diff(a.x, a.y, b.x, b.y) + cabs_diff(a.z, a.w, b.z, b.w);
  }
  if (odd && blockIdx.x == 0 && threadIdx.x == 0) {  // the last complex value of an odd count
    const float2 a = yr1[2 * pairs], b = yt1[2 * pairs];
    acc += cabs_diff(a.x, a.y, b.x, b.y);
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) s += red[w];
    partial[blockIdx.x] = s;
  }
}

__global__ void __launch_bounds__(kThreads)
    l1_finish(const float* __restrict__ partial, int n, double inv_count, float* __restrict__ out) {
  __shared__ double red[kThreads];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += kThreads) s += (double)partial[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = kThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[0] = (float)(red[0] * inv_count);
}

// one complex element (frequency bin `bin`) of the gradient
__device__ __forceinline__ float2 l1_grad(float ar, float ai, float br, float bi, float scale, int bin, int n_fft) {
  const float dr = ar - br, di = ai - bi;
  const float m = sqrtf(fmaf(dr, dr, di * di));
  const float w = (bin == 0 || 2 * bin == n_fft) ? 1.0f : 0.5f;
  const float f = m > 0.f ? scale * w / m : 0.f;
  return make_float2(dr * f, di * f);
}

// 32-bit element indices (the host checks count < 2^31)
__global__ void __launch_bounds__(kThreads)
    l1_backward(const float2* __restrict__ yr, const float2* __restrict__ yt, int count, int bins, int n_fft,
                const float* __restrict__ grad_loss, double inv_count, float2* __restrict__ g) {
  const float scale = (float)((double)grad_loss[0] * inv_count);
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < count; i += gridDim.x * kThreads) {
    const float2 a = yr[i], b = yt[i];
    g[i] = l1_grad(a.x, a.y, b.x, b.y, scale, i % bins, n_fft);
  }
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int64_t pmb_spectral_l1_workspace_size(int64_t count) {
  if (count <= 0) return 0;
  return (int64_t)loss_grid(count / 2) * (int64_t)sizeof(float);
}

extern "C" int pmb_spectral_l1_forward(const float* y_recon, const float* y_target, int64_t count, float* loss,
                                       void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_spectral_l1_forward";
  PMB_REQUIRE(count > 0 && y_recon && y_target && loss, "%s: bad arguments", name);
  PMB_REQUIRE(((reinterpret_cast<uintptr_t>(y_recon) | reinterpret_cast<uintptr_t>(y_target)) & 15) == 0,
              "%s: spectra must be 16-byte aligned", name);
  const int64_t pairs = count / 2;
  const int grid = loss_grid(pairs);
  if (workspace == nullptr || workspace_bytes < (int64_t)grid * (int64_t)sizeof(float)) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)grid * 4);
    return PMB_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(workspace);
  l1_partial<<<grid, kThreads, 0, s>>>(reinterpret_cast<const float4*>(y_recon),
                                        reinterpret_cast<const float4*>(y_target), pairs,
                                        reinterpret_cast<const float2*>(y_recon),
                                        reinterpret_cast<const float2*>(y_target), (int)(count & 1), partial);
  PMB_CHECK_LAUNCH(name);
  l1_finish<<<1, kThreads, 0, s>>>(partial, grid, 1.0 / (double)count, loss);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

extern "C" int pmb_spectral_l1_backward(const float* y_recon, const float* y_target, int64_t count, int64_t bins,
                                        int64_t n_fft, const float* grad_loss, float* grad_recon, void* stream) {
  clear_error();
  const char* name = "pmb_spectral_l1_backward";
  PMB_REQUIRE(count > 0 && count < (1ll << 31) && bins > 0 && count % bins == 0 && n_fft > 0 &&
                  bins == n_fft / 2 + 1,
              "%s: bad shape (count %lld, bins %lld, n_fft %lld)", name, (long long)count, (long long)bins,
              (long long)n_fft);
  PMB_REQUIRE(y_recon && y_target && grad_loss && grad_recon, "%s: NULL argument", name);
  PMB_REQUIRE(((reinterpret_cast<uintptr_t>(y_recon) | reinterpret_cast<uintptr_t>(y_target) |
                reinterpret_cast<uintptr_t>(grad_recon)) & 7) == 0,
              "%s: spectra must be 8-byte aligned", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  l1_backward<<<loss_grid(count), kThreads, 0, s>>>(reinterpret_cast<const float2*>(y_recon),
                                                    reinterpret_cast<const float2*>(y_target), (int)count, (int)bins,
                                                    (int)n_fft, grad_loss, 1.0 / (double)count,
                                                    reinterpret_cast<float2*>(grad_recon));
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}
