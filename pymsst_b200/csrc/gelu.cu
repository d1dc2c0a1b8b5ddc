// GELU (exact erf form, torch.nn.GELU()) forward and backward for the
// transformer feed-forward block, and column sums of 16-bit matrices (bias
// gradients).  Memory-bound passes with 16-byte vectors:
//   forward:  y = x * Phi(x)
//   backward: gx = gy * (Phi(x) + x * phi(x)), optionally with the column sums
//             of gx (the preceding Linear's bias gradient) from the same pass:
//             each CTA covers 128 rows x 256 columns and writes one fp32
//             partial row; red::colsum_rows sums the partial rows in order.
// The values are computed in fp32 from the stored 16-bit tensors and rounded
// once, as torch's elementwise kernels do; the bias sums add the rounded gx.
// Reference semantics: the nn.GELU() of pymss-core's FeedForward; the
// reference's patch set (src/pymsst/training/fused_roformer.py:256-824:
// BandSplit, rotary, RMSNorm, attention gates, MaskEstimator) leaves the
// feed-forward block on torch.
#include <initializer_list>

#include "common.cuh"
#include "gelu.cuh"
#include "reduce.cuh"

namespace pmb {
namespace {

constexpr int kRowsPerBlock = 128;

template <typename T>
struct V8 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__global__ void __launch_bounds__(256) gelu_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  constexpr int N = V8<T>::N;
  const int64_t nv = n / N;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < nv; i += (int64_t)gridDim.x * 256) {
    uint4 u = reinterpret_cast<const uint4*>(x)[i];
    T* e = reinterpret_cast<T*>(&u);
    // (the packed two-value form measured 2 us slower here than the scalar one: unlike the derivative, the
    // forward has too little arithmetic per value to pay for the register pairing)
    if constexpr (sizeof(T) == 2) {  // outputs rounded in pairs (one conversion instruction per two values)
      uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < N; j += 2)
        w[j / 2] = Elem<T>::pack2(gelu_of<T>(Elem<T>::to_f(e[j])), gelu_of<T>(Elem<T>::to_f(e[j + 1])));
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) e[j] = Elem<T>::from_f(gelu_of<T>(Elem<T>::to_f(e[j])));
    }
    reinterpret_cast<uint4*>(y)[i] = u;
  }
  // tail (n not a multiple of the vector width)
  for (int64_t i = nv * N + (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
    const float v = Elem<T>::to_f(x[i]);
    y[i] = Elem<T>::from_f(gelu_of<T>(v));
  }
}

// One CTA: rows [r0, r0 + 128), columns [c0, c0 + 32 * N): lane l of every
// warp owns the N columns c0 + l*N.., warp w the rows r0 + w, r0 + w + 8, ...
// MODE 0: column sums of x only.  MODE 1: gx = gy * gelu'(x), stored, and
// column sums of the stored gx.  Requires cols % N == 0 and 16-byte aligned
// rows (checked by the host).
template <typename T, int MODE>
__global__ void __launch_bounds__(256, 3)
    rows_pass(const T* __restrict__ gy, const T* __restrict__ x, int64_t rows, int64_t cols, T* __restrict__ gx,
              float* __restrict__ partial) {
  constexpr int N = V8<T>::N;
  __shared__ float red_s[8][32 * N + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 * N + lane * N;
  const int64_t r0 = (int64_t)blockIdx.y * kRowsPerBlock;
  float acc[N];
#pragma unroll
  for (int j = 0; j < N; ++j) acc[j] = 0.f;
  if (c < cols) {
    const int64_t r1 = r0 + kRowsPerBlock < rows ? r0 + kRowsPerBlock : rows;
    constexpr int U = 4;  // rows of this warp in flight before any arithmetic
    for (int64_t rb = r0 + warp; rb < r1; rb += 8 * U) {
      uint4 ux[U], ug[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int64_t r = rb + 8 * k;
        if (r < r1) {
          ux[k] = *reinterpret_cast<const uint4*>(x + r * cols + c);
          if (MODE == 1) ug[k] = *reinterpret_cast<const uint4*>(gy + r * cols + c);
        }
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int64_t r = rb + 8 * k;
        if (r >= r1) break;
        const T* e = reinterpret_cast<const T*>(&ux[k]);
        if (MODE == 0) {
#pragma unroll
          for (int j = 0; j < N; ++j) acc[j] += Elem<T>::to_f(e[j]);
        } else {
          const T* g = reinterpret_cast<const T*>(&ug[k]);
          uint4 uo;
          T* o = reinterpret_cast<T*>(&uo);
          if constexpr (sizeof(T) == 2) {  // two values per packed instruction
#pragma unroll
            for (int j = 0; j < N; j += 2) {
              float d0, d1, q0, q1;
              gelu_grad_fast2(Elem<T>::to_f(e[j]), Elem<T>::to_f(e[j + 1]), d0, d1);
              unpk2(mul2(pk2(Elem<T>::to_f(g[j]), Elem<T>::to_f(g[j + 1])), pk2(d0, d1)), q0, q1);
              reinterpret_cast<uint32_t*>(&uo)[j / 2] = Elem<T>::pack2(q0, q1);  // rounded as a pair
              acc[j] += Elem<T>::to_f(o[j]);
              acc[j + 1] += Elem<T>::to_f(o[j + 1]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < N; ++j) {
              const float v = Elem<T>::to_f(e[j]);
              o[j] = Elem<T>::from_f(Elem<T>::to_f(g[j]) * gelu_grad_of<T>(v));
              acc[j] += Elem<T>::to_f(o[j]);
            }
          }
          *reinterpret_cast<uint4*>(gx + r * cols + c) = uo;
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) red_s[warp][lane * N + j] = acc[j];
  __syncthreads();
  for (int k = threadIdx.x; k < 32 * N; k += 256) {
    const int64_t cc = (int64_t)blockIdx.x * 32 * N + k;
    if (cc >= cols) continue;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red_s[w][k];
    partial[(int64_t)blockIdx.y * cols + cc] = s;
  }
}

int64_t row_blocks(int64_t rows) { return (rows + kRowsPerBlock - 1) / kRowsPerBlock; }

bool vec_ok(int es, int64_t cols, std::initializer_list<const void*> ptrs) {
  if (cols % (16 / es) != 0) return false;
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15) != 0) return false;
  return true;
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_gelu_forward(const void* x, void* y, int64_t n, int dtype, void* stream) {
  clear_error();
  const char* name = "pmb_gelu_forward";
  PMB_REQUIRE(n >= 0, "%s: bad size", name);
  if (n == 0) return PMB_OK;
  PMB_REQUIRE(x && y, "%s: NULL tensor argument", name);
  PMB_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0,
              "%s: tensors must be 16-byte aligned", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH(dtype, T, name, [&] {
    int64_t g = (n / V8<T>::N + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    gelu_fwd_kernel<T><<<(int)g, 256, 0, s>>>(static_cast<const T*>(x), static_cast<T*>(y), n);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

extern "C" int64_t pmb_rows_pass_workspace_size(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return (row_blocks(rows) * cols * 4 + 255) / 256 * 256;
}

extern "C" int pmb_gelu_backward(const void* grad_out, const void* x, void* grad_in, int64_t rows, int64_t cols,
                                 void* grad_bias, int bias_dtype, int dtype, void* workspace, int64_t workspace_bytes,
                                 void* stream) {
  clear_error();
  const char* name = "pmb_gelu_backward";
  PMB_REQUIRE(rows >= 0 && cols > 0, "%s: bad shape", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (grad_bias) PMB_CHECK_CUDA(cudaMemsetAsync(grad_bias, 0, cols * dtype_size(bias_dtype), s), name);
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && x && grad_in, "%s: NULL tensor argument", name);
  const int64_t need = pmb_rows_pass_workspace_size(rows, cols);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  return PMB_DISPATCH(dtype, T, name, [&] {
    if (!vec_ok(sizeof(T), cols, {grad_out, x, grad_in})) {
      set_error("%s: cols must be a multiple of %d and tensors 16-byte aligned", name, (int)V8<T>::N);
      return PMB_ERR_ALIGNMENT;
    }
    float* partial = static_cast<float*>(workspace);
    dim3 g((unsigned)((cols + 32 * V8<T>::N - 1) / (32 * V8<T>::N)), (unsigned)row_blocks(rows));
    rows_pass<T, 1><<<g, 256, 0, s>>>(static_cast<const T*>(grad_out), static_cast<const T*>(x), rows, cols,
                                      static_cast<T*>(grad_in), partial);
    PMB_CHECK_LAUNCH(name);
    if (grad_bias) {
      red::colsum_rows<<<red::colsum_rows_grid(cols), red::kThreads, 0, s>>>(partial, (int)row_blocks(rows), cols,
                                                                             grad_bias, bias_dtype);
      PMB_CHECK_LAUNCH(name);
    }
    return PMB_OK;
  });
}

extern "C" int pmb_column_sum(const void* x, int64_t rows, int64_t cols, void* out, int out_dtype, int dtype,
                              void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_column_sum";
  PMB_REQUIRE(rows >= 0 && cols > 0 && dtype_size(out_dtype) > 0, "%s: bad arguments", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PMB_REQUIRE(out, "%s: NULL output", name);
  if (rows == 0) {
    PMB_CHECK_CUDA(cudaMemsetAsync(out, 0, cols * dtype_size(out_dtype), s), name);
    return PMB_OK;
  }
  PMB_REQUIRE(x, "%s: NULL tensor argument", name);
  const int64_t need = pmb_rows_pass_workspace_size(rows, cols);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  return PMB_DISPATCH(dtype, T, name, [&] {
    if (!vec_ok(sizeof(T), cols, {x})) {
      set_error("%s: cols must be a multiple of %d and x 16-byte aligned", name, (int)V8<T>::N);
      return PMB_ERR_ALIGNMENT;
    }
    float* partial = static_cast<float*>(workspace);
    dim3 g((unsigned)((cols + 32 * V8<T>::N - 1) / (32 * V8<T>::N)), (unsigned)row_blocks(rows));
    rows_pass<T, 0><<<g, 256, 0, s>>>(nullptr, static_cast<const T*>(x), rows, cols, nullptr, partial);
    PMB_CHECK_LAUNCH(name);
    red::colsum_rows<<<red::colsum_rows_grid(cols), red::kThreads, 0, s>>>(partial, (int)row_blocks(rows), cols, out,
                                                                           out_dtype);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}
