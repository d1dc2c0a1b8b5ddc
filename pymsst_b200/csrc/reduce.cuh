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
  // eight rows per step with independent loads (one memory round trip per eight rows), fixed summation order
  float s = 0.f;
  int64_t r = r0;
  for (; r + 8 <= r1; r += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = Elem<T>::to_f(src[(r + j) * ld + c]);
    s += ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
  }
  for (; r < r1; ++r) s += Elem<T>::to_f(src[r * ld + c]);
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
// covers 4 columns with 64 row lanes (a warp reads 8 rows x 16 bytes per
// load, four loads in flight per thread), so even a 192-column matrix spreads
// over 48 CTAs; the row lanes are combined in shared memory in a fixed order.
// Launch: grid colsum_rows_grid(cols), 256 threads.  out[c] stored as out_code.
constexpr int kColsumCols = 4;
constexpr int kColsumRowLanes = kThreads / kColsumCols;
inline int colsum_rows_grid(int64_t cols) { return (int)((cols + kColsumCols - 1) / kColsumCols); }

__global__ void __launch_bounds__(kThreads)
    colsum_rows(const float* __restrict__ partial, int nrows, int64_t cols, void* __restrict__ out, int out_code) {
  __shared__ float red_s[kColsumRowLanes][kColsumCols + 1];
  __shared__ float red8[8][kColsumCols];
  const int cl = threadIdx.x % kColsumCols, rl = threadIdx.x / kColsumCols;
  const int64_t c = (int64_t)blockIdx.x * kColsumCols + cl;
  constexpr int R = kColsumRowLanes;
  float s = 0.f;
  if (c < cols) {
    int r = rl;
    for (; r + 3 * R < nrows; r += 4 * R) {
      const float a = partial[(int64_t)r * cols + c], b = partial[(int64_t)(r + R) * cols + c];
      const float d = partial[(int64_t)(r + 2 * R) * cols + c], e = partial[(int64_t)(r + 3 * R) * cols + c];
      s += (a + b) + (d + e);
    }
    for (; r < nrows; r += R) s += partial[(int64_t)r * cols + c];
  }
  red_s[rl][cl] = s;
  __syncthreads();
  // 64 row lanes -> 8 per column in fixed pairs, then the 8 summed by one thread
  if (threadIdx.x < 8 * kColsumCols) {
    const int col = threadIdx.x % kColsumCols, part = threadIdx.x / kColsumCols;
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < R / 8; ++k) t += red_s[part * (R / 8) + k][col];
    red8[part][col] = t;
  }
  __syncthreads();
  if (threadIdx.x < kColsumCols && (int64_t)blockIdx.x * kColsumCols + threadIdx.x < cols) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red8[k][threadIdx.x];
    store_dyn(out, (int64_t)blockIdx.x * kColsumCols + threadIdx.x, out_code, t);
  }
}

}  // namespace
}  // namespace red
}  // namespace pmb
