// FP32-accumulating SIMT tile GEMM shared by the band-wise (grouped / ragged)
// kernels.  It is the exact-fp32 path (fp32 training must match an fp32
// reference to 1e-4, which excludes TF32 tensor cores) and the fallback for
// shapes the tcgen05 kernels do not take.
//
// C[m, n] = sum_k A[m, k] * B[n, k] with arbitrary element strides, so one
// routine serves "x W^T" (both K-contiguous), "dY^T X" (both MN-contiguous)
// and "dY W" layouts.  A CTA of 256 threads computes a BM x BN tile; thread
// (tx, ty) owns rows ty + 16 i and columns tx + 16 j, so epilogue stores of
// consecutive threads hit consecutive columns.
#pragma once

#include "common.cuh"

namespace pmb {
namespace simt {

constexpr int kThreads = 256;
constexpr int BM = 64;
constexpr int BN = 64;
constexpr int BK = 16;
constexpr int TM = BM / 16;
constexpr int TN = BN / 16;

struct Smem {
  float a[BK][BM + 1];
  float b[BK][BN + 1];
  float a_row_scale[BM];
};

template <typename T, int ROWS, bool KCONTIG>
__device__ __forceinline__ void load_tile(float (*dst)[ROWS + 1], const T* __restrict__ base, int64_t s_r,
                                          int64_t s_k, int r0, int r_lim, int k0, int k_lim) {
  constexpr int kPerThread = ROWS * BK / kThreads;
#pragma unroll
  for (int i = 0; i < kPerThread; ++i) {
    const int e = threadIdx.x + i * kThreads;
    int r, k;
    if (KCONTIG) {
      r = e / BK;
      k = e % BK;
    } else {
      r = e % ROWS;
      k = e / ROWS;
    }
    const int gr = r0 + r, gk = k0 + k;
    float v = 0.f;
    if (gr < r_lim && gk < k_lim) v = Elem<T>::to_f(base[(int64_t)gr * s_r + (int64_t)gk * s_k]);
    dst[k][r] = v;
  }
}

// Accumulate one BM x BN tile over k in [0, K).  Optional A transforms:
// a_row_scale (smem, BM entries, multiplies row r) and a_k_scale_ptr (global,
// K entries of type TKS, multiplies column k; NULL = none).
template <typename TA, typename TB, bool A_KCONTIG, bool B_KCONTIG, typename TKS = float>
__device__ __forceinline__ void mainloop(Smem& sm, const TA* __restrict__ A, int64_t sa_m, int64_t sa_k,
                                         const TB* __restrict__ B, int64_t sb_n, int64_t sb_k, int m0, int m_lim,
                                         int n0, int n_lim, int K, bool use_row_scale,
                                         const void* __restrict__ a_k_scale_ptr, float (&acc)[TM][TN]) {
  const TKS* a_k_scale = static_cast<const TKS*>(a_k_scale_ptr);
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += BK) {
    load_tile<TA, BM, A_KCONTIG>(sm.a, A, sa_m, sa_k, m0, m_lim, k0, K);
    load_tile<TB, BN, B_KCONTIG>(sm.b, B, sb_n, sb_k, n0, n_lim, k0, K);
    __syncthreads();
    if (use_row_scale || a_k_scale != nullptr) {
      for (int e = threadIdx.x; e < BK * BM; e += kThreads) {
        const int k = e / BM, r = e % BM;
        float s = use_row_scale ? sm.a_row_scale[r] : 1.f;
        if (a_k_scale != nullptr && k0 + k < K) s *= Elem<TKS>::to_f(a_k_scale[k0 + k]);
        sm.a[k][r] *= s;
      }
      __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = sm.a[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = sm.b[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ int row_of(int i) { return threadIdx.x / 16 + 16 * i; }
__device__ __forceinline__ int col_of(int j) { return threadIdx.x % 16 + 16 * j; }

__host__ __device__ inline int tiles(int64_t n, int t) { return (int)((n + t - 1) / t); }

}  // namespace simt
}  // namespace pmb
