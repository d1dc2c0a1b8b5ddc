// Deterministic two-pass column sums: pass 1 reduces a chunk of rows per CTA
// into an fp32 partial row (workspace), pass 2 sums the partial rows.  Used
// for bias and gamma gradients so results do not depend on atomics order.
#pragma once

#include "common.cuh"

namespace pmb {
namespace red {
namespace {  // internal linkage: each translation unit owns its copy

constexpr int kThreads = 256;
constexpr int kRowsPerChunk = 64;

inline int chunks(int64_t rows) { return (int)((rows + kRowsPerChunk - 1) / kRowsPerChunk); }

// partial[chunk][c] = sum over rows in chunk of src[r * ld + c]
template <typename T>
__global__ void __launch_bounds__(kThreads)
    colsum_partial(const T* __restrict__ src, int64_t rows, int64_t cols, int64_t ld, float* __restrict__ partial) {
  const int64_t c = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.y * kRowsPerChunk;
  const int64_t r1 = r0 + kRowsPerChunk < rows ? r0 + kRowsPerChunk : rows;
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += Elem<T>::to_f(src[r * ld + c]);
  partial[(int64_t)blockIdx.y * cols + c] = s;
}

__device__ __forceinline__ void store_dyn(void* p, int64_t i, int code, float v) {
  switch (code) {
    case PMB_FLOAT16:
      static_cast<__half*>(p)[i] = __float2half_rn(v);
      break;
    case PMB_BFLOAT16:
      static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
      break;
    default:
      static_cast<float*>(p)[i] = v;
  }
}

// out[c] = sum_chunk partial[chunk][c]; dense destination.
__global__ void __launch_bounds__(kThreads)
    colsum_finalize(const float* __restrict__ partial, int nchunks, int64_t cols, void* __restrict__ out,
                    int out_code) {
  const int64_t c = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int k = 0; k < nchunks; ++k) s += partial[(int64_t)k * cols + c];
  store_dyn(out, c, out_code, s);
}

// Same, scattering column c to band table destination: band b = band_of(c),
// written at ptr0[b][c - off[b]].  `scale` multiplies the stored widths:
// column c covers band widths * scale (e.g. 2 for GLU pre-activations).
__global__ void __launch_bounds__(kThreads)
    colsum_finalize_bands(const float* __restrict__ partial, int nchunks, int64_t cols, BandTable table,
                          int out_code) {
  const int64_t c = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int k = 0; k < nchunks; ++k) s += partial[(int64_t)k * cols + c];
  const int b = band_of(table, c);
  store_dyn(const_cast<void*>(table.ptr0[b]), c - table.off[b], out_code, s);
}

// Column sums of a [nrows, cols] fp32 partial matrix with many rows: each CTA
// covers 32 columns; its 8 warps stride over the rows (coalesced 128-byte
// row segments) and the per-warp sums are combined in shared memory.
// Launch: grid ceil(cols / 32), 256 threads.  out[c] stored as out_code.
__global__ void __launch_bounds__(kThreads)
    colsum_rows(const float* __restrict__ partial, int nrows, int64_t cols, void* __restrict__ out, int out_code) {
  __shared__ float red_s[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  float s = 0.f;
  if (c < cols)
    for (int r = warp; r < nrows; r += 8) s += partial[(int64_t)r * cols + c];
  red_s[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && c < cols) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red_s[w][lane];
    store_dyn(out, c, out_code, t);
  }
}

}  // namespace
}  // namespace red
}  // namespace pmb
