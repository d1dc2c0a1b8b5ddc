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
// The STFT-side tensors are contiguous along frames, the feature-side ones
// along j, so every kernel works on frame-contiguous runs:
//   gather forward / recombine backward (one value per feature j): a CTA
//     stages a 32 (j) x 32 (frame) tile in shared memory -- rows read along
//     frames for each j's (f, s), written back along j -- so both sides move
//     full 128-byte lines;
//   gather backward / recombine forward (a sum over the features j that read
//     pair (f, s)): a warp owns one pair and 32 consecutive frames, walks the
//     pair's feature list (warp-uniform, in CSR order, so the sum order is
//     fixed and the result deterministic) and writes 32 frames contiguously;
//     the feature-side reads are frame-strided but the [B, T, J] features
//     stay resident in the 126 MB L2.
#include "common.cuh"

namespace pmb {
namespace {

constexpr int kThreads = 256;

struct Dims {
  int64_t B, S, F, T, J, N;
};

constexpr int kTile = 32;

// Two consecutive elements (one complex value) stored with one 4- or 8-byte store.
template <typename T>
__device__ __forceinline__ void store_pair(T* dst, float re, float im) {
  if constexpr (sizeof(T) == 2) {
    T v[2] = {Elem<T>::from_f(re), Elem<T>::from_f(im)};
    *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(v);
  } else {
    *reinterpret_cast<float2*>(dst) = make_float2(re, im);
  }
}

// x[b, t, j, :] = stft[b, s_j, f_j, t, :]: CTA = 32 j x 32 frames of one batch item; rows of x (one per (b, t))
// are `ld` elements apart (ld >= 2 J, even).
template <typename T>
__global__ void __launch_bounds__(kThreads)
    gather_fwd(const float* __restrict__ stft, const int* __restrict__ index, Dims d, int64_t ld,
               T* __restrict__ x) {
  __shared__ float2 tile[kTile][kTile + 1];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t j0 = (int64_t)blockIdx.x * kTile, t0 = (int64_t)blockIdx.y * kTile, b = blockIdx.z;
  for (int jj = ty; jj < kTile; jj += kThreads / 32) {
    const int64_t j = j0 + jj, t = t0 + tx;
    if (j < d.J && t < d.T) {
      const int fs = index[j];
      const int64_t f = fs / d.S, s = fs - f * d.S;
      tile[jj][tx] = *reinterpret_cast<const float2*>(stft + ((((b * d.S + s) * d.F + f) * d.T + t) << 1));
    }
  }
  __syncthreads();
  for (int tt = ty; tt < kTile; tt += kThreads / 32) {
    const int64_t t = t0 + tt, j = j0 + tx;
    if (j < d.J && t < d.T) {
      const float2 v = tile[tx][tt];
      store_pair<T>(x + (b * d.T + t) * ld + j * 2, v.x, v.y);
    }
  }
}

// Pair-major sum over a pair's features for 32 frames: warp = one (f, s) pair.
// MODE 0 (gather backward): out = sum_j src[b, t, j].
// MODE 1 (recombine forward): out = (stft *) sum_j src[bn, t, j] / count.
template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads)
    pair_sum(const T* __restrict__ src, const float* __restrict__ stft, const int* __restrict__ inv_ptr,
             const int* __restrict__ inv_idx, Dims d, int multiply, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t FS = d.F * d.S;
  const int64_t fs = (int64_t)blockIdx.y * (kThreads / 32) + (threadIdx.x >> 5);
  const int64_t t = (int64_t)blockIdx.x * 32 + lane;
  const int64_t bn = blockIdx.z;  // b (MODE 0) or b * N + n (MODE 1)
  if (fs >= FS || t >= d.T) return;
  const int k0 = inv_ptr[fs], k1 = inv_ptr[fs + 1];
  const T* row = src + (bn * d.T + t) * d.J * 2;
  float re = 0.f, im = 0.f;
  for (int k = k0; k < k1; ++k) {
    const int j = inv_idx[k];
    re += Elem<T>::to_f(row[2 * j]);
    im += Elem<T>::to_f(row[2 * j + 1]);
  }
  const int64_t f = fs / d.S, s = fs - f * d.S;
  float2 o;
  if (MODE == 0) {
    o = make_float2(re, im);
    *reinterpret_cast<float2*>(out + ((((bn * d.S + s) * d.F + f) * d.T + t) << 1)) = o;
  } else {
    const float cnt = fmaxf((float)(k1 - k0), 1.0e-8f);
    const float mr = re / cnt, mi = im / cnt;
    o = make_float2(mr, mi);
    if (multiply) {
      const int64_t b = bn / d.N;
      const float2 v = *reinterpret_cast<const float2*>(stft + ((((b * d.S + s) * d.F + f) * d.T + t) << 1));
      o = make_float2(v.x * mr - v.y * mi, v.x * mi + v.y * mr);
    }
    *reinterpret_cast<float2*>(out + (((((bn * d.S + s) * d.F + f) * d.T) + t) << 1)) = o;
  }
}

// grad_mask[b,n,t,j] = (g * conj(stft) or g) / count(index[j]), g = grad_out[b,n,s_j,f_j,t]:
// CTA = 32 j x 32 frames, staged like gather_fwd.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    recombine_bwd(const float* __restrict__ gout, const float* __restrict__ stft, const int* __restrict__ index,
                  const int* __restrict__ inv_ptr, Dims d, int multiply, T* __restrict__ gmask) {
  __shared__ float2 tile[kTile][kTile + 1];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t j0 = (int64_t)blockIdx.x * kTile, t0 = (int64_t)blockIdx.y * kTile, bn = blockIdx.z;
  const int64_t b = bn / d.N;
  for (int jj = ty; jj < kTile; jj += kThreads / 32) {
    const int64_t j = j0 + jj, t = t0 + tx;
    if (j < d.J && t < d.T) {
      const int fs = index[j];
      const int64_t f = fs / d.S, s = fs - f * d.S;
      const float cnt = fmaxf((float)(inv_ptr[fs + 1] - inv_ptr[fs]), 1.0e-8f);
      const float2 g = *reinterpret_cast<const float2*>(gout + (((((bn * d.S + s) * d.F + f) * d.T) + t) << 1));
      float2 r = g;
      if (multiply) {
        const float2 v = *reinterpret_cast<const float2*>(stft + ((((b * d.S + s) * d.F + f) * d.T + t) << 1));
        r = make_float2(g.x * v.x + g.y * v.y, g.y * v.x - g.x * v.y);
      }
      tile[jj][tx] = make_float2(r.x / cnt, r.y / cnt);
    }
  }
  __syncthreads();
  for (int tt = ty; tt < kTile; tt += kThreads / 32) {
    const int64_t t = t0 + tt, j = j0 + tx;
    if (j < d.J && t < d.T) {
      const float2 v = tile[tx][tt];
      T* dst = gmask + ((bn * d.T + t) * d.J + j) * 2;
      dst[0] = Elem<T>::from_f(v.x);
      dst[1] = Elem<T>::from_f(v.y);
    }
  }
}

bool check_dims(const Dims& d) { return d.B >= 0 && d.S > 0 && d.F > 0 && d.T >= 0 && d.J > 0 && d.N > 0; }

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_band_gather_forward(const float* stft, const int* index, int64_t batch, int64_t channels,
                                       int64_t freqs, int64_t frames, int64_t pairs, void* x, int64_t x_ld,
                                       int x_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_band_gather_forward";
  Dims d{batch, channels, freqs, frames, pairs, 1};
  PMB_REQUIRE(check_dims(d), "%s: bad shape", name);
  if (x_ld == 0) x_ld = 2 * pairs;
  PMB_REQUIRE(x_ld >= 2 * pairs && x_ld % 2 == 0, "%s: row stride %lld must be even and >= %lld", name,
              (long long)x_ld, (long long)(2 * pairs));
  if (batch * frames == 0) return PMB_OK;
  PMB_REQUIRE(stft && index && x, "%s: NULL tensor argument", name);
  PMB_REQUIRE((reinterpret_cast<uintptr_t>(stft) & 7) == 0, "%s: stft must be 8-byte aligned", name);
  PMB_REQUIRE((reinterpret_cast<uintptr_t>(x) & (2 * dtype_size(x_dtype) - 1)) == 0,
              "%s: x must be aligned to one complex value", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((pairs + kTile - 1) / kTile), (unsigned)((frames + kTile - 1) / kTile), (unsigned)batch);
  return PMB_DISPATCH(x_dtype, T, name, [&] {
    gather_fwd<T><<<grid, kThreads, 0, s>>>(stft, index, d, x_ld, static_cast<T*>(x));
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
  const dim3 grid((unsigned)((frames + 31) / 32), (unsigned)((freqs * channels + kThreads / 32 - 1) / (kThreads / 32)),
                  (unsigned)batch);
  return PMB_DISPATCH(x_dtype, T, name, [&] {
    pair_sum<T, 0><<<grid, kThreads, 0, s>>>(static_cast<const T*>(grad_x), nullptr, inv_ptr, inv_idx, d, 0,
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
  const dim3 grid((unsigned)((frames + 31) / 32), (unsigned)((freqs * channels + kThreads / 32 - 1) / (kThreads / 32)),
                  (unsigned)(batch * stems));
  return PMB_DISPATCH(mask_dtype, T, name, [&] {
    pair_sum<T, 1><<<grid, kThreads, 0, s>>>(static_cast<const T*>(mask), stft, inv_ptr, inv_idx, d, multiply_stft,
                                             out);
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
  const dim3 grid((unsigned)((pairs + kTile - 1) / kTile), (unsigned)((frames + kTile - 1) / kTile),
                  (unsigned)(batch * stems));
  return PMB_DISPATCH(mask_dtype, T, name, [&] {
    recombine_bwd<T><<<grid, kThreads, 0, s>>>(grad_out, stft, index, inv_ptr, d, multiply_stft,
                                               static_cast<T*>(grad_mask));
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}
