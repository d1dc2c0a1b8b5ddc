// MaskEstimator per-band MLP: grouped Linear(+Tanh) hidden layers and the
// ragged final Linear(H -> 2*I_b) + GLU, forward and backward (exact-fp32
// SIMT path).  Reference semantics: src/pymsst/training/cuda/
// fused_band_split.cu:1006-1074 (grouped linear), :2284-2367 (GLU epilogue and
// its backward), :2516-2851 ("direct" final forward/backward); call sites
// src/pymsst/training/fused_roformer.py:527-583, 1087-1133.
//
// Final layer, band b (off_b = prefix sum of widths, w = I_b):
//   pre[m, 2off_b + j] = x[m,b,:] . W_b[j,:] + bias[2off_b + j],  j < 2w
//   out[m, off_b + l]  = pre[m, 2off_b + l] * sigmoid(pre[m, 2off_b + w + l])
// Backward: grad_pre = (g*gate, g*left*gate*(1-gate)), grad_bias = column
// sums of grad_pre, grad_x_b = grad_pre_b W_b, grad_W_b = grad_pre_b^T x_b.
#include "common.cuh"
#include "gemm_simt.cuh"
#include "reduce.cuh"

#include <vector>

namespace pmb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }

// ------------------------------------------------------ final layer (GLU)
// tab.ptr0 = W_b [2w, H]
// tab.ptr1 = bias_b [2w]
template <typename T, typename TP>
__global__ void __launch_bounds__(simt::kThreads)
    final_fwd_gemm(const T* __restrict__ x, int64_t rows, int64_t H, BandTable tab, T* __restrict__ pre) {
  __shared__ simt::Smem sm;
  const int b = blockIdx.y;
  const int64_t w2 = 2 * (tab.off[b + 1] - tab.off[b]);
  const int ntn = simt::tiles(2 * (int64_t)tab.max_width, simt::BN);
  const int m0 = (blockIdx.x / ntn) * simt::BM;
  const int n0 = (blockIdx.x % ntn) * simt::BN;
  if (n0 >= w2) return;
  float acc[simt::TM][simt::TN];
  simt::mainloop<T, TP, true, true>(sm, x + (int64_t)b * H, (int64_t)tab.count * H, 1,
                                     static_cast<const TP*>(tab.ptr0[b]), H, 1, m0, (int)rows, n0, (int)w2, (int)H,
                                     false, nullptr, acc);
  const int64_t c0 = 2 * tab.off[b];
  const int64_t ld = 2 * tab.total;
  const TP* bias = static_cast<const TP*>(tab.ptr1[b]);
#pragma unroll
  for (int i = 0; i < simt::TM; ++i) {
    const int m = m0 + simt::row_of(i);
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < simt::TN; ++j) {
      const int n = n0 + simt::col_of(j);
      if (n >= w2) continue;
      pre[(int64_t)m * ld + c0 + n] = Elem<T>::from_f(acc[i][j] + Elem<TP>::to_f(bias[n]));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    glu_fwd(const T* __restrict__ pre, int64_t rows, BandTable tab, T* __restrict__ out) {
  const int64_t n = rows * tab.total;
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += (int64_t)gridDim.x * kThreads) {
    const int64_t m = e / tab.total, c = e % tab.total;
    const int b = band_of(tab, c);
    const int64_t w = tab.off[b + 1] - tab.off[b];
    const int64_t l = c - tab.off[b];
    const T* p = pre + m * 2 * tab.total + 2 * tab.off[b];
    out[e] = Elem<T>::from_f(Elem<T>::to_f(p[l]) * sigmoidf_(Elem<T>::to_f(p[w + l])));
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    glu_bwd(const T* __restrict__ dy, const T* __restrict__ pre, int64_t rows, BandTable tab, float* __restrict__ gp) {
  const int64_t n = rows * tab.total;
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += (int64_t)gridDim.x * kThreads) {
    const int64_t m = e / tab.total, c = e % tab.total;
    const int b = band_of(tab, c);
    const int64_t w = tab.off[b + 1] - tab.off[b];
    const int64_t l = c - tab.off[b];
    const int64_t base = m * 2 * tab.total + 2 * tab.off[b];
    const float left = Elem<T>::to_f(pre[base + l]);
    const float gate = sigmoidf_(Elem<T>::to_f(pre[base + w + l]));
    const float g = Elem<T>::to_f(dy[e]);
    gp[base + l] = g * gate;
    gp[base + w + l] = g * left * gate * (1.0f - gate);
  }
}

// grad_x[m,b,h] = sum_j gp[m, 2off_b + j] W_b[j, h]
template <typename T, typename TP>
__global__ void __launch_bounds__(simt::kThreads)
    final_bwd_x(const float* __restrict__ gp, int64_t rows, int64_t H, BandTable tab, T* __restrict__ grad_x) {
  __shared__ simt::Smem sm;
  const int b = blockIdx.y;
  const int64_t w2 = 2 * (tab.off[b + 1] - tab.off[b]);
  const int ntn = simt::tiles(H, simt::BN);
  const int m0 = (blockIdx.x / ntn) * simt::BM;
  const int n0 = (blockIdx.x % ntn) * simt::BN;
  float acc[simt::TM][simt::TN];
  simt::mainloop<float, TP, true, false>(sm, gp + 2 * tab.off[b], 2 * tab.total, 1,
                                         static_cast<const TP*>(tab.ptr0[b]), 1, H, m0, (int)rows, n0, (int)H, (int)w2,
                                         false, nullptr, acc);
#pragma unroll
  for (int i = 0; i < simt::TM; ++i) {
    const int m = m0 + simt::row_of(i);
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < simt::TN; ++j) {
      const int h = n0 + simt::col_of(j);
      if (h < H) grad_x[((int64_t)m * tab.count + b) * H + h] = Elem<T>::from_f(acc[i][j]);
    }
  }
}

// grad_W_b[j, h] = sum_m gp[m, 2off_b + j] x[m, b, h];  tab.ptr1 = grad_W_b
template <typename T, typename TP>
__global__ void __launch_bounds__(simt::kThreads)
    final_bwd_w(const float* __restrict__ gp, const T* __restrict__ x, int64_t rows, int64_t H, BandTable tab) {
  __shared__ simt::Smem sm;
  const int b = blockIdx.y;
  const int64_t w2 = 2 * (tab.off[b + 1] - tab.off[b]);
  const int ntn = simt::tiles(H, simt::BN);
  const int m0 = (blockIdx.x / ntn) * simt::BM;
  const int n0 = (blockIdx.x % ntn) * simt::BN;
  if (m0 >= w2) return;
  float acc[simt::TM][simt::TN];
  simt::mainloop<float, T, false, false>(sm, gp + 2 * tab.off[b], 1, 2 * tab.total, x + (int64_t)b * H, 1,
                                         (int64_t)tab.count * H, m0, (int)w2, n0, (int)H, (int)rows, false, nullptr,
                                         acc);
  TP* gW = static_cast<TP*>(const_cast<void*>(tab.ptr1[b]));
#pragma unroll
  for (int i = 0; i < simt::TM; ++i) {
    const int j = m0 + simt::row_of(i);
    if (j >= w2) continue;
#pragma unroll
    for (int jj = 0; jj < simt::TN; ++jj) {
      const int h = n0 + simt::col_of(jj);
      if (h < H) gW[(int64_t)j * H + h] = Elem<TP>::from_f(acc[i][jj]);
    }
  }
}

// ------------------------------------------------------- grouped linear
struct GL {
  int64_t rows, groups, in_f, out_f;
  int64_t xs_m, xs_g, xs_i;
};

// tab.ptr0 = W_g [O, I], tab.ptr1 = bias_g [O] (may be NULL)
template <typename T, typename TP, bool KCONTIG>
__global__ void __launch_bounds__(simt::kThreads)
    grouped_fwd(const T* __restrict__ x, GL p, BandTable tab, T* __restrict__ out, int act) {
  __shared__ simt::Smem sm;
  const int g = blockIdx.y;
  const TP* W = static_cast<const TP*>(tab.ptr0[g]);
  const TP* bias = static_cast<const TP*>(tab.ptr1[g]);
  const int ntn = simt::tiles(p.out_f, simt::BN);
  const int m0 = (blockIdx.x / ntn) * simt::BM;
  const int n0 = (blockIdx.x % ntn) * simt::BN;
  float acc[simt::TM][simt::TN];
  simt::mainloop<T, TP, KCONTIG, true>(sm, x + g * p.xs_g, p.xs_m, p.xs_i, W, p.in_f, 1, m0, (int)p.rows, n0,
                                        (int)p.out_f, (int)p.in_f, false, nullptr, acc);
#pragma unroll
  for (int i = 0; i < simt::TM; ++i) {
    const int m = m0 + simt::row_of(i);
    if (m >= p.rows) continue;
#pragma unroll
    for (int j = 0; j < simt::TN; ++j) {
      const int o = n0 + simt::col_of(j);
      if (o >= p.out_f) continue;
      float v = acc[i][j];
      if (bias != nullptr) v += Elem<TP>::to_f(bias[o]);
      if (act == PMB_ACT_TANH) v = tanhf(v);
      out[((int64_t)m * p.groups + g) * p.out_f + o] = Elem<T>::from_f(v);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    act_bwd(const T* __restrict__ dy, const T* __restrict__ y, int64_t n, int act, float* __restrict__ dpre) {
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += (int64_t)gridDim.x * kThreads) {
    float g = Elem<T>::to_f(dy[e]);
    if (act == PMB_ACT_TANH) {
      const float t = Elem<T>::to_f(y[e]);
      g *= 1.0f - t * t;
    }
    dpre[e] = g;
  }
}

template <typename T, typename TP>
__global__ void __launch_bounds__(simt::kThreads)
    grouped_bwd_x(const float* __restrict__ dpre, GL p, BandTable tab, T* __restrict__ grad_x) {
  __shared__ simt::Smem sm;
  const int g = blockIdx.y;
  const TP* W = static_cast<const TP*>(tab.ptr0[g]);
  const int ntn = simt::tiles(p.in_f, simt::BN);
  const int m0 = (blockIdx.x / ntn) * simt::BM;
  const int n0 = (blockIdx.x % ntn) * simt::BN;
  float acc[simt::TM][simt::TN];
  simt::mainloop<float, TP, true, false>(sm, dpre + g * p.out_f, p.groups * p.out_f, 1, W, 1, p.in_f, m0,
                                         (int)p.rows, n0, (int)p.in_f, (int)p.out_f, false, nullptr, acc);
#pragma unroll
  for (int i = 0; i < simt::TM; ++i) {
    const int m = m0 + simt::row_of(i);
    if (m >= p.rows) continue;
#pragma unroll
    for (int j = 0; j < simt::TN; ++j) {
      const int c = n0 + simt::col_of(j);
      if (c < p.in_f) grad_x[((int64_t)m * p.groups + g) * p.in_f + c] = Elem<T>::from_f(acc[i][j]);
    }
  }
}

template <typename T, typename TP>
__global__ void __launch_bounds__(simt::kThreads)
    grouped_bwd_w(const float* __restrict__ dpre, const T* __restrict__ x, GL p, BandTable tab) {
  __shared__ simt::Smem sm;
  const int g = blockIdx.y;
  TP* grad_w = static_cast<TP*>(const_cast<void*>(tab.ptr2[g]));
  const int ntn = simt::tiles(p.in_f, simt::BN);
  const int m0 = (blockIdx.x / ntn) * simt::BM;  // over o
  const int n0 = (blockIdx.x % ntn) * simt::BN;  // over i
  float acc[simt::TM][simt::TN];
  simt::mainloop<float, T, false, false>(sm, dpre + g * p.out_f, 1, p.groups * p.out_f, x + g * p.xs_g, p.xs_i,
                                         p.xs_m, m0, (int)p.out_f, n0, (int)p.in_f, (int)p.rows, false, nullptr, acc);
#pragma unroll
  for (int i = 0; i < simt::TM; ++i) {
    const int o = m0 + simt::row_of(i);
    if (o >= p.out_f) continue;
#pragma unroll
    for (int j = 0; j < simt::TN; ++j) {
      const int c = n0 + simt::col_of(j);
      if (c < p.in_f) grad_w[(int64_t)o * p.in_f + c] = Elem<TP>::from_f(acc[i][j]);
    }
  }
}

int elementwise_grid(int64_t n) {
  int64_t g = (n + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }

}  // namespace
}  // namespace pmb

using namespace pmb;

// --------------------------------------------------------------- final layer
extern "C" int pmb_mask_estimator_final_forward(const void* x, int64_t rows, int num_bands, int64_t hidden,
                                                const int64_t* widths, const void* const* weights,
                                                const void* const* biases, void* out, void* pre, int dtype,
                                                int param_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_mask_estimator_final_forward";
  BandTable tab;
  int st = make_band_table(tab, num_bands, widths, weights, biases, nullptr, name);
  if (st) return st;
  PMB_REQUIRE(rows >= 0 && hidden > 0, "%s: bad shape", name);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(x && biases && out && pre && weights, "%s: NULL tensor argument", name);
  for (int b = 0; b < num_bands; ++b)
    PMB_REQUIRE(tab.ptr0[b] && tab.ptr1[b], "%s: band %d weight or bias is NULL", name, b);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    dim3 grid(simt::tiles(rows, simt::BM) * simt::tiles(2 * (int64_t)tab.max_width, simt::BN), num_bands);
    final_fwd_gemm<T, TP><<<grid, simt::kThreads, 0, s>>>(static_cast<const T*>(x), rows, hidden, tab,
                                                           static_cast<T*>(pre));
    PMB_CHECK_LAUNCH(name);
    glu_fwd<T><<<elementwise_grid(rows * tab.total), kThreads, 0, s>>>(static_cast<const T*>(pre), rows, tab,
                                                                        static_cast<T*>(out));
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

extern "C" int64_t pmb_mask_estimator_final_backward_workspace_size(int64_t rows, int num_bands,
                                                                    const int64_t* widths) {
  if (rows <= 0 || num_bands <= 0 || widths == nullptr) return 0;
  int64_t total = 0;
  for (int b = 0; b < num_bands; ++b) total += widths[b];
  return align256(rows * 2 * total * 4) + align256((int64_t)red::chunks(rows) * 2 * total * 4);
}

extern "C" int pmb_mask_estimator_final_backward(const void* grad_out, const void* x, const void* pre, int64_t rows,
                                                 int num_bands, int64_t hidden, const int64_t* widths,
                                                 const void* const* weights, void* grad_x, void* const* grad_biases,
                                                 void* const* grad_weights, int dtype, int param_dtype,
                                                 void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_mask_estimator_final_backward";
  BandTable tab, btab;
  int st = make_band_table(tab, num_bands, widths, weights, (const void* const*)grad_weights, nullptr, name);
  if (st) return st;
  PMB_REQUIRE(rows >= 0 && hidden > 0, "%s: bad shape", name);
  PMB_REQUIRE(weights && grad_weights && grad_biases && grad_x, "%s: NULL argument", name);
  {
    std::vector<int64_t> w2(num_bands);
    for (int b = 0; b < num_bands; ++b) w2[b] = 2 * widths[b];
    st = make_band_table(btab, num_bands, w2.data(), (const void* const*)grad_biases, nullptr, nullptr, name);
    if (st) return st;
  }
  for (int b = 0; b < num_bands; ++b)
    PMB_REQUIRE(tab.ptr0[b] && tab.ptr1[b] && btab.ptr0[b], "%s: band %d pointer is NULL", name, b);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int es = dtype_size(param_dtype);
  PMB_REQUIRE(es > 0, "%s: unsupported parameter dtype %d", name, param_dtype);
  if (rows == 0) {
    for (int b = 0; b < num_bands; ++b) {
      PMB_CHECK_CUDA(cudaMemsetAsync(grad_biases[b], 0, 2 * (tab.off[b + 1] - tab.off[b]) * es, s), name);
      PMB_CHECK_CUDA(cudaMemsetAsync(grad_weights[b], 0, 2 * (tab.off[b + 1] - tab.off[b]) * hidden * es, s), name);
    }
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && x && pre, "%s: NULL tensor argument", name);
  const int64_t need = pmb_mask_estimator_final_backward_workspace_size(rows, num_bands, widths);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  float* gp = static_cast<float*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + align256(rows * 2 * tab.total * 4));
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    glu_bwd<T><<<elementwise_grid(rows * tab.total), kThreads, 0, s>>>(static_cast<const T*>(grad_out),
                                                                        static_cast<const T*>(pre), rows, tab, gp);
    PMB_CHECK_LAUNCH(name);
    const int64_t cols = 2 * tab.total;
    dim3 gpart((int)((cols + 255) / 256), red::chunks(rows));
    red::colsum_partial<float><<<gpart, red::kThreads, 0, s>>>(gp, rows, cols, cols, partial);
    PMB_CHECK_LAUNCH(name);
    red::colsum_finalize_bands<<<(int)((cols + 255) / 256), red::kThreads, 0, s>>>(partial, red::chunks(rows), cols,
                                                                                   btab, param_dtype);
    PMB_CHECK_LAUNCH(name);
    dim3 gx(simt::tiles(rows, simt::BM) * simt::tiles(hidden, simt::BN), num_bands);
    final_bwd_x<T, TP><<<gx, simt::kThreads, 0, s>>>(gp, rows, hidden, tab, static_cast<T*>(grad_x));
    PMB_CHECK_LAUNCH(name);
    dim3 gw(simt::tiles(2 * (int64_t)tab.max_width, simt::BM) * simt::tiles(hidden, simt::BN), num_bands);
    final_bwd_w<T, TP><<<gw, simt::kThreads, 0, s>>>(gp, static_cast<const T*>(x), rows, hidden, tab);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

// ------------------------------------------------------------ grouped linear
extern "C" int pmb_grouped_linear_forward(const void* x, int64_t rows, int64_t groups, int64_t in_features,
                                          int64_t out_features, int64_t x_stride_row, int64_t x_stride_group,
                                          int64_t x_stride_feat, const void* const* weights,
                                          const void* const* biases, void* out, int activation, int dtype,
                                          int param_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_grouped_linear_forward";
  PMB_REQUIRE(rows >= 0 && groups > 0 && groups <= kMaxBands && in_features > 0 && out_features > 0,
              "%s: bad shape (groups must be 1..%d)", name, kMaxBands);
  BandTable tab;
  {
    std::vector<int64_t> ow(groups, out_features);
    int st = make_band_table(tab, (int)groups, ow.data(), weights, biases, nullptr, name);
    if (st) return st;
  }
  PMB_REQUIRE(activation == PMB_ACT_NONE || activation == PMB_ACT_TANH, "%s: unknown activation %d", name,
              activation);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(x && weights && out, "%s: NULL tensor argument", name);
  for (int g = 0; g < groups; ++g) PMB_REQUIRE(tab.ptr0[g], "%s: group %d weight is NULL", name, g);
  GL p{rows, groups, in_features, out_features, x_stride_row, x_stride_group, x_stride_feat};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    dim3 grid(simt::tiles(rows, simt::BM) * simt::tiles(out_features, simt::BN), (unsigned)groups);
    if (x_stride_feat == 1)
      grouped_fwd<T, TP, true><<<grid, simt::kThreads, 0, s>>>(static_cast<const T*>(x), p, tab,
                                                               static_cast<T*>(out), activation);
    else
      grouped_fwd<T, TP, false><<<grid, simt::kThreads, 0, s>>>(static_cast<const T*>(x), p, tab,
                                                                static_cast<T*>(out), activation);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

extern "C" int64_t pmb_grouped_linear_backward_workspace_size(int64_t rows, int64_t groups, int64_t out_features) {
  if (rows <= 0 || groups <= 0 || out_features <= 0) return 0;
  const int64_t cols = groups * out_features;
  return align256(rows * cols * 4) + align256((int64_t)red::chunks(rows) * cols * 4);
}

extern "C" int pmb_grouped_linear_backward(const void* grad_out, const void* x, const void* out, int64_t rows,
                                           int64_t groups, int64_t in_features, int64_t out_features,
                                           const void* const* weights, void* grad_x, void* const* grad_weights,
                                           void* const* grad_biases, int activation, int dtype, int param_dtype,
                                           void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_grouped_linear_backward";
  PMB_REQUIRE(rows >= 0 && groups > 0 && groups <= kMaxBands && in_features > 0 && out_features > 0,
              "%s: bad shape (groups must be 1..%d)", name, kMaxBands);
  BandTable tab, btab;
  {
    std::vector<int64_t> ow(groups, out_features);
    int st = make_band_table(tab, (int)groups, ow.data(), weights, nullptr, (const void* const*)grad_weights, name);
    if (st) return st;
    btab.count = 0;
    if (grad_biases != nullptr) {
      st = make_band_table(btab, (int)groups, ow.data(), (const void* const*)grad_biases, nullptr, nullptr, name);
      if (st) return st;
    }
  }
  PMB_REQUIRE(activation == PMB_ACT_NONE || activation == PMB_ACT_TANH, "%s: unknown activation %d", name,
              activation);
  PMB_REQUIRE(weights && grad_weights, "%s: NULL argument", name);
  for (int g = 0; g < groups; ++g)
    PMB_REQUIRE(tab.ptr0[g] && tab.ptr2[g] && (btab.count == 0 || btab.ptr0[g]), "%s: group %d pointer is NULL",
                name, g);
  PMB_REQUIRE(activation != PMB_ACT_TANH || out != nullptr || rows == 0, "%s: tanh backward needs `out`", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int es = dtype_size(param_dtype);
  PMB_REQUIRE(es > 0, "%s: unsupported parameter dtype %d", name, param_dtype);
  const int64_t cols = groups * out_features;
  if (rows == 0) {
    for (int g = 0; g < groups; ++g) {
      PMB_CHECK_CUDA(cudaMemsetAsync(grad_weights[g], 0, out_features * in_features * es, s), name);
      if (btab.count) PMB_CHECK_CUDA(cudaMemsetAsync(grad_biases[g], 0, out_features * es, s), name);
    }
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && x, "%s: NULL tensor argument", name);
  const int64_t need = pmb_grouped_linear_backward_workspace_size(rows, groups, out_features);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  float* dpre = static_cast<float*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + align256(rows * cols * 4));
  GL p{rows, groups, in_features, out_features, groups * in_features, in_features, 1};
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    act_bwd<T><<<elementwise_grid(rows * cols), kThreads, 0, s>>>(static_cast<const T*>(grad_out),
                                                                  static_cast<const T*>(out), rows * cols, activation,
                                                                  dpre);
    PMB_CHECK_LAUNCH(name);
    if (btab.count > 0) {
      dim3 gpart((int)((cols + 255) / 256), red::chunks(rows));
      red::colsum_partial<float><<<gpart, red::kThreads, 0, s>>>(dpre, rows, cols, cols, partial);
      PMB_CHECK_LAUNCH(name);
      red::colsum_finalize_bands<<<(int)((cols + 255) / 256), red::kThreads, 0, s>>>(partial, red::chunks(rows), cols,
                                                                                     btab, param_dtype);
      PMB_CHECK_LAUNCH(name);
    }
    if (grad_x != nullptr) {
      dim3 gx(simt::tiles(rows, simt::BM) * simt::tiles(in_features, simt::BN), (unsigned)groups);
      grouped_bwd_x<T, TP><<<gx, simt::kThreads, 0, s>>>(dpre, p, tab, static_cast<T*>(grad_x));
      PMB_CHECK_LAUNCH(name);
    }
    dim3 gw(simt::tiles(out_features, simt::BM) * simt::tiles(in_features, simt::BN), (unsigned)groups);
    grouped_bwd_w<T, TP><<<gw, simt::kThreads, 0, s>>>(dpre, static_cast<const T*>(x), p, tab);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}
