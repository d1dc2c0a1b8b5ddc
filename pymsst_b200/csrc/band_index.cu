// Integer-indexed band gather / scatter-add-average kernels between the STFT
// and the band-split / mask-estimator feature layouts.
//
// Layouts (S = audio channels, F = frequency bins, J = gathered (freq, chan)
// pairs, c = real/imag):
//   stft  [B, S, F, T, 2]   (torch.stft of the [B*S, L] audio, as real)
//   feats [B, T, J, 2]      band-split input / mask-estimator output
//   out   [B, N, S, F, T, 2] masked STFT, the iSTFT input
// index[j] = f*S + s is the (freq, chan) pair feeding feature j;
// Mel-band RoFormer's bands overlap, so a pair can feed several features;
// the inverse map (inv_ptr/inv_idx, CSR over f*S + s) lists them.
//
// Reference semantics (pymss-core MelBandRoformer, reached through
// src/pymsst/training/fused_roformer.py:827-873; the index table and the
// average follow the published Mel-band RoFormer):
//   gather:    x[b, t, j, c] = stft[b, s_j, f_j, t, c]
//   recombine: m[b,n,f*S+s,t] = sum_{j: index[j]=f*S+s} mask[b,n,t,j] / count(f*S+s)
//              out = stft * m  (complex product)
// For BS-RoFormer the index is the identity (non-overlapping bands).
//
// A CTA covers kTT = 4 consecutive frames so that every global access moves
// at least 32 contiguous bytes (4 frames x 8-byte complex values); the
// recombine stages the 4 mask rows in shared memory and reduces the
// overlapping contributions there.
#include "common.cuh"

namespace pmb {
namespace {

constexpr int kThreads = 256;
constexpr int kTT = 4;

struct Dims {
  int64_t B, S, F, T, J, N;
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
    gather_fwd(const float* __restrict__ stft, const int* __restrict__ index, Dims d, T* __restrict__ x) {
  const int64_t tiles_t = (d.T + kTT - 1) / kTT;
  const int64_t b = blockIdx.x / tiles_t;
  const int64_t t0 = (blockIdx.x % tiles_t) * kTT;
  for (int64_t e = threadIdx.x; e < d.J * kTT; e += kThreads) {
    const int tt = (int)(e % kTT);
    const int64_t j = e / kTT;
    const int64_t t = t0 + tt;
    if (t >= d.T) continue;
    const int fs = index[j];
    const int64_t f = fs / d.S, s = fs % d.S;
    const float2 v = *reinterpret_cast<const float2*>(stft + ((((b * d.S + s) * d.F + f) * d.T + t) << 1));
    T* dst = x + ((b * d.T + t) * d.J + j) * 2;
    dst[0] = Elem<T>::from_f(v.x);
    dst[1] = Elem<T>::from_f(v.y);
  }
}

// grad_stft[b,s,f,t,c] = sum_{j in inv(f*S+s)} grad_x[b,t,j,c]
template <typename T>
__global__ void __launch_bounds__(kThreads)
    gather_bwd(const T* __restrict__ gx, const int* __restrict__ inv_ptr, const int* __restrict__ inv_idx, Dims d,
               float* __restrict__ gstft) {
  extern __shared__ float rows[];  // [kTT][J*2]
  const int64_t tiles_t = (d.T + kTT - 1) / kTT;
  const int64_t b = blockIdx.x / tiles_t;
  const int64_t t0 = (blockIdx.x % tiles_t) * kTT;
  for (int64_t e = threadIdx.x; e < kTT * d.J * 2; e += kThreads) {
    const int64_t tt = e / (d.J * 2), q = e % (d.J * 2);
    rows[e] = (t0 + tt < d.T) ? Elem<T>::to_f(gx[(b * d.T + t0 + tt) * d.J * 2 + q]) : 0.f;
  }
  __syncthreads();
  const int64_t FS = d.F * d.S;
  for (int64_t e = threadIdx.x; e < FS * kTT; e += kThreads) {
    const int tt = (int)(e % kTT);
    const int64_t fs = e / kTT;
    if (t0 + tt >= d.T) continue;
    float re = 0.f, im = 0.f;
    for (int k = inv_ptr[fs]; k < inv_ptr[fs + 1]; ++k) {
      const int j = inv_idx[k];
      re += rows[tt * d.J * 2 + 2 * j];
      im += rows[tt * d.J * 2 + 2 * j + 1];
    }
    const int64_t f = fs / d.S, s = fs % d.S;
    *reinterpret_cast<float2*>(gstft + ((((b * d.S + s) * d.F + f) * d.T + t0 + tt) << 1)) = make_float2(re, im);
  }
}

// out[b,n,s,f,t] = (multiply ? stft[b,s,f,t] : 1) * sum_{j in inv} mask[b,n,t,j] / count
template <typename T>
__global__ void __launch_bounds__(kThreads)
    recombine_fwd(const T* __restrict__ mask, const float* __restrict__ stft, const int* __restrict__ inv_ptr,
                  const int* __restrict__ inv_idx, Dims d, int multiply, float* __restrict__ out) {
  extern __shared__ float rows[];  // [kTT][J*2]
  const int64_t tiles_t = (d.T + kTT - 1) / kTT;
  const int64_t bn = blockIdx.x / tiles_t;  // b * N + n
  const int64_t b = bn / d.N;
  const int64_t t0 = (blockIdx.x % tiles_t) * kTT;
  for (int64_t e = threadIdx.x; e < kTT * d.J * 2; e += kThreads) {
    const int64_t tt = e / (d.J * 2), q = e % (d.J * 2);
    rows[e] = (t0 + tt < d.T) ? Elem<T>::to_f(mask[(bn * d.T + t0 + tt) * d.J * 2 + q]) : 0.f;
  }
  __syncthreads();
  const int64_t FS = d.F * d.S;
  for (int64_t e = threadIdx.x; e < FS * kTT; e += kThreads) {
    const int tt = (int)(e % kTT);
    const int64_t fs = e / kTT;
    const int64_t t = t0 + tt;
    if (t >= d.T) continue;
    const int k0 = inv_ptr[fs], k1 = inv_ptr[fs + 1];
    float mr = 0.f, mi = 0.f;
    for (int k = k0; k < k1; ++k) {
      const int j = inv_idx[k];
      mr += rows[tt * d.J * 2 + 2 * j];
      mi += rows[tt * d.J * 2 + 2 * j + 1];
    }
    const float cnt = fmaxf((float)(k1 - k0), 1.0e-8f);
    mr /= cnt;
    mi /= cnt;
    const int64_t f = fs / d.S, s = fs % d.S;
    float2 o = make_float2(mr, mi);
    if (multiply) {
      const float2 v = *reinterpret_cast<const float2*>(stft + ((((b * d.S + s) * d.F + f) * d.T + t) << 1));
      o = make_float2(v.x * mr - v.y * mi, v.x * mi + v.y * mr);
    }
    *reinterpret_cast<float2*>(out + (((((bn * d.S + s) * d.F + f) * d.T) + t) << 1)) = o;
  }
}

// grad_mask[b,n,t,j] = conj-chain of out = stft * avg:  g_avg = g * conj(stft)
// (or g when multiply == 0), divided by count(index[j]).
template <typename T>
__global__ void __launch_bounds__(kThreads)
    recombine_bwd(const float* __restrict__ gout, const float* __restrict__ stft, const int* __restrict__ index,
                  const int* __restrict__ inv_ptr, Dims d, int multiply, T* __restrict__ gmask) {
  const int64_t tiles_t = (d.T + kTT - 1) / kTT;
  const int64_t bn = blockIdx.x / tiles_t;
  const int64_t b = bn / d.N;
  const int64_t t0 = (blockIdx.x % tiles_t) * kTT;
  for (int64_t e = threadIdx.x; e < d.J * kTT; e += kThreads) {
    const int tt = (int)(e % kTT);
    const int64_t j = e / kTT;
    const int64_t t = t0 + tt;
    if (t >= d.T) continue;
    const int fs = index[j];
    const int64_t f = fs / d.S, s = fs % d.S;
    const float cnt = fmaxf((float)(inv_ptr[fs + 1] - inv_ptr[fs]), 1.0e-8f);
    const float2 g = *reinterpret_cast<const float2*>(gout + (((((bn * d.S + s) * d.F + f) * d.T) + t) << 1));
    float2 r = g;
    if (multiply) {
      const float2 v = *reinterpret_cast<const float2*>(stft + ((((b * d.S + s) * d.F + f) * d.T + t) << 1));
      r = make_float2(g.x * v.x + g.y * v.y, g.y * v.x - g.x * v.y);
    }
    T* dst = gmask + ((bn * d.T + t) * d.J + j) * 2;
    dst[0] = Elem<T>::from_f(r.x / cnt);
    dst[1] = Elem<T>::from_f(r.y / cnt);
  }
}

bool check_dims(const Dims& d) { return d.B >= 0 && d.S > 0 && d.F > 0 && d.T >= 0 && d.J > 0 && d.N > 0; }

int set_smem(const void* fn, size_t bytes, const char* name) {
  if (bytes > 227 * 1024) {
    set_error("%s: %zu bytes of staged rows exceed shared memory (J too large)", name, bytes);
    return PMB_ERR_INVALID_ARGUMENT;
  }
  if (bytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) {
      set_error("%s: cudaFuncSetAttribute failed: %s", name, cudaGetErrorString(e));
      return PMB_ERR_CUDA;
    }
  }
  return PMB_OK;
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_band_gather_forward(const float* stft, const int* index, int64_t batch, int64_t channels,
                                       int64_t freqs, int64_t frames, int64_t pairs, void* x, int x_dtype,
                                       void* stream) {
  clear_error();
  const char* name = "pmb_band_gather_forward";
  Dims d{batch, channels, freqs, frames, pairs, 1};
  PMB_REQUIRE(check_dims(d), "%s: bad shape", name);
  if (batch * frames == 0) return PMB_OK;
  PMB_REQUIRE(stft && index && x, "%s: NULL tensor argument", name);
  PMB_REQUIRE((reinterpret_cast<uintptr_t>(stft) & 7) == 0, "%s: stft must be 8-byte aligned", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t grid = batch * ((frames + kTT - 1) / kTT);
  return PMB_DISPATCH(x_dtype, T, name, [&] {
    gather_fwd<T><<<(unsigned)grid, kThreads, 0, s>>>(stft, index, d, static_cast<T*>(x));
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

extern "C" int pmb_band_gather_backward(const void* grad_x, const int* inv_ptr, const int* inv_idx, int64_t batch,
                                        int64_t channels, int64_t freqs, int64_t frames, int64_t pairs,
                                        float* grad_stft, int x_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_band_gather_backward";
  Dims d{batch, channels, freqs, frames, pairs, 1};
  PMB_REQUIRE(check_dims(d), "%s: bad shape", name);
  if (batch * frames == 0) return PMB_OK;
  PMB_REQUIRE(grad_x && inv_ptr && inv_idx && grad_stft, "%s: NULL tensor argument", name);
  PMB_REQUIRE((reinterpret_cast<uintptr_t>(grad_stft) & 7) == 0, "%s: grad_stft must be 8-byte aligned", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)kTT * pairs * 2 * sizeof(float);
  const int64_t grid = batch * ((frames + kTT - 1) / kTT);
  return PMB_DISPATCH(x_dtype, T, name, [&] {
    int st = set_smem((const void*)gather_bwd<T>, smem, name);
    if (st) return st;
    gather_bwd<T><<<(unsigned)grid, kThreads, smem, s>>>(static_cast<const T*>(grad_x), inv_ptr, inv_idx, d,
                                                          grad_stft);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

extern "C" int pmb_band_recombine_forward(const void* mask, const float* stft, const int* inv_ptr,
                                          const int* inv_idx, int64_t batch, int64_t stems, int64_t channels,
                                          int64_t freqs, int64_t frames, int64_t pairs, int multiply_stft,
                                          float* out, int mask_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_band_recombine_forward";
  Dims d{batch, channels, freqs, frames, pairs, stems};
  PMB_REQUIRE(check_dims(d), "%s: bad shape", name);
  if (batch * frames == 0) return PMB_OK;
  PMB_REQUIRE(mask && inv_ptr && inv_idx && out && (stft || !multiply_stft), "%s: NULL tensor argument", name);
  PMB_REQUIRE((reinterpret_cast<uintptr_t>(out) & 7) == 0 && (reinterpret_cast<uintptr_t>(stft) & 7) == 0,
              "%s: stft/out must be 8-byte aligned", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)kTT * pairs * 2 * sizeof(float);
  const int64_t grid = batch * stems * ((frames + kTT - 1) / kTT);
  return PMB_DISPATCH(mask_dtype, T, name, [&] {
    int st = set_smem((const void*)recombine_fwd<T>, smem, name);
    if (st) return st;
    recombine_fwd<T><<<(unsigned)grid, kThreads, smem, s>>>(static_cast<const T*>(mask), stft, inv_ptr, inv_idx, d,
                                                             multiply_stft, out);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

extern "C" int pmb_band_recombine_backward(const float* grad_out, const float* stft, const int* index,
                                           const int* inv_ptr, int64_t batch, int64_t stems, int64_t channels,
                                           int64_t freqs, int64_t frames, int64_t pairs, int multiply_stft,
                                           void* grad_mask, int mask_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_band_recombine_backward";
  Dims d{batch, channels, freqs, frames, pairs, stems};
  PMB_REQUIRE(check_dims(d), "%s: bad shape", name);
  if (batch * frames == 0) return PMB_OK;
  PMB_REQUIRE(grad_out && index && inv_ptr && grad_mask && (stft || !multiply_stft), "%s: NULL tensor argument", name);
  PMB_REQUIRE((reinterpret_cast<uintptr_t>(grad_out) & 7) == 0 && (reinterpret_cast<uintptr_t>(stft) & 7) == 0,
              "%s: stft/grad_out must be 8-byte aligned", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t grid = batch * stems * ((frames + kTT - 1) / kTT);
  return PMB_DISPATCH(mask_dtype, T, name, [&] {
    recombine_bwd<T><<<(unsigned)grid, kThreads, 0, s>>>(grad_out, stft, index, inv_ptr, d, multiply_stft,
                                                          static_cast<T*>(grad_mask));
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}
