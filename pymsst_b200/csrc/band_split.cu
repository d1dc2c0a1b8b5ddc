// BandSplit: per-band RMSNorm followed by a per-band Linear(I_b -> O), over
// bands of unequal width (ragged) or equal width (grouped), forward and
// backward.  Reference semantics: src/pymsst/training/cuda/fused_band_split.cu
// :14-247 (grouped), :590-1003 (ragged), pure-torch form
// src/pymsst/training/fused_roformer.py:1265-1271.
//
// Forward (per band b, row m):   inv = 1/max(||x_b||, eps), s = sqrt(I_b)
//   normed = x_b * inv * s;  out[m,b,:] = (x_b * inv * s * gamma_b) W_b^T + bias_b
// The normalisation is applied as a row scale and a column scale of the GEMM
// A operand, so x is read once by the GEMM and the per-row norm pass only
// reads it to produce inv (and `normed`, which the reference API returns).
//
// Backward uses G_b = dY_b^T normed_b  ([O x I_b], reduction over rows):
//   grad_W_b = G_b * gamma_b (column scale),  grad_gamma_b[i] = sum_o W_b[o,i] G_b[o,i]
// which equals the reference's sum_m (dY W)[m,i] normed[m,i]; grad_bias is a
// column sum of dY; grad_x (optional: the STFT input of BandSplit carries no
// gradient in training) needs gs = dY_b W_b and the RMSNorm input gradient
//   grad_x = inv * (gs*gamma*s - normed * (sum_i gs*gamma*normed) / s).
// This file is the exact-fp32 SIMT path used for fp32 and as the fallback.
#include "common.cuh"
#include "gemm_simt.cuh"
#include "reduce.cuh"

#include <vector>

namespace pmb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

struct XLayout {
  int64_t s_row;   // stride between rows
  int64_t s_band;  // stride between bands (grouped layout); < 0 = ragged (column offset off[b])
  int64_t s_feat;  // stride between features of a band
  __device__ __forceinline__ int64_t base(const BandTable& t, int b) const {
    return s_band < 0 ? t.off[b] * s_feat : (int64_t)b * s_band;
  }
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
    band_norm_kernel(const T* __restrict__ x, int64_t rows, XLayout lx, BandTable tab, T* __restrict__ normed,
                     float* __restrict__ inv_norm) {
  const int lane = threadIdx.x & 31;
  const int64_t pairs = rows * tab.count;
  for (int64_t p = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); p < pairs; p += (int64_t)gridDim.x * kWarps) {
    const int64_t r = p / tab.count;
    const int b = (int)(p % tab.count);
    const int64_t w = tab.off[b + 1] - tab.off[b];
    const T* xb = x + r * lx.s_row + lx.base(tab, b);
    float ss = 0.f;
    for (int64_t i = lane; i < w; i += 32) {
      const float v = Elem<T>::to_f(xb[i * lx.s_feat]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / fmaxf(sqrtf(ss), 1.0e-12f);
    if (lane == 0) inv_norm[r * tab.count + b] = inv;
    if (normed != nullptr) {
      const float k = inv * sqrtf((float)w);
      T* nb = normed + r * tab.total + tab.off[b];
      for (int64_t i = lane; i < w; i += 32) nb[i] = Elem<T>::from_f(Elem<T>::to_f(xb[i * lx.s_feat]) * k);
    }
  }
}

// tab.ptr0 = gamma_b [I_b], ptr1 = W_b [O, I_b], ptr2 = bias_b [O] (may be NULL)
template <typename T, typename TP, bool KCONTIG>
__global__ void __launch_bounds__(simt::kThreads)
    band_split_fwd_gemm(const T* __restrict__ x, int64_t rows, XLayout lx, BandTable tab, int64_t O,
                        const float* __restrict__ inv_norm, T* __restrict__ out) {
  __shared__ simt::Smem sm;
  const int b = blockIdx.y;
  const int ntn = simt::tiles(O, simt::BN);
  const int m0 = (blockIdx.x / ntn) * simt::BM;
  const int n0 = (blockIdx.x % ntn) * simt::BN;
  const int64_t w = tab.off[b + 1] - tab.off[b];
  const float s = sqrtf((float)w);
  for (int r = threadIdx.x; r < simt::BM; r += simt::kThreads)
    sm.a_row_scale[r] = (m0 + r < rows) ? inv_norm[(int64_t)(m0 + r) * tab.count + b] * s : 0.f;
  __syncthreads();
  float acc[simt::TM][simt::TN];
  simt::mainloop<T, TP, KCONTIG, true, TP>(sm, x + lx.base(tab, b), lx.s_row, lx.s_feat,
                                           static_cast<const TP*>(tab.ptr1[b]), w, 1, m0, (int)rows, n0, (int)O,
                                           (int)w, true, tab.ptr0[b], acc);
  const TP* bias = static_cast<const TP*>(tab.ptr2[b]);
#pragma unroll
  for (int i = 0; i < simt::TM; ++i) {
    const int m = m0 + simt::row_of(i);
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < simt::TN; ++j) {
      const int n = n0 + simt::col_of(j);
      if (n >= O) continue;
      float v = acc[i][j];
      if (bias != nullptr) v += Elem<TP>::to_f(bias[n]);
      out[((int64_t)m * tab.count + b) * O + n] = Elem<T>::from_f(v);
    }
  }
}

// G-GEMM: G[o, i] = sum_m dY[m,b,o] normed[m, off_b + i].  Epilogue writes
// grad_W = G * gamma and a per-o-tile partial of grad_gamma (fp32 workspace).
// tab.ptr0 = gamma_b, ptr1 = W_b, ptr2 = grad_W_b.
template <typename T, typename TP>
__global__ void __launch_bounds__(simt::kThreads)
    band_split_bwd_weight(const T* __restrict__ dy, const T* __restrict__ normed, int64_t rows, BandTable tab,
                          int64_t O, float* __restrict__ dgamma_partial) {
  __shared__ simt::Smem sm;
  __shared__ float red[16][simt::BN];
  const int b = blockIdx.y;
  const int64_t w = tab.off[b + 1] - tab.off[b];
  const int nti = simt::tiles(tab.max_width, simt::BN);
  const int to = blockIdx.x / nti;
  const int n0 = (blockIdx.x % nti) * simt::BN;  // over i
  if (n0 >= w) return;
  const int m0 = to * simt::BM;  // over o
  const int64_t nbO = (int64_t)tab.count * O;
  float acc[simt::TM][simt::TN];
  simt::mainloop<T, T, false, false, T>(sm, dy + (int64_t)b * O, 1, nbO, normed + tab.off[b], 1, tab.total, m0,
                                        (int)O, n0, (int)w, (int)rows, false, nullptr, acc);
  const TP* gamma = static_cast<const TP*>(tab.ptr0[b]);
  const TP* W = static_cast<const TP*>(tab.ptr1[b]);
  TP* gW = static_cast<TP*>(const_cast<void*>(tab.ptr2[b]));
  float colpart[simt::TN];
#pragma unroll
  for (int j = 0; j < simt::TN; ++j) {
    const int i = n0 + simt::col_of(j);
    colpart[j] = 0.f;
    if (i >= w) continue;
    const float g = Elem<TP>::to_f(gamma[i]);
#pragma unroll
    for (int ii = 0; ii < simt::TM; ++ii) {
      const int o = m0 + simt::row_of(ii);
      if (o >= O) continue;
      gW[(int64_t)o * w + i] = Elem<TP>::from_f(acc[ii][j] * g);
      colpart[j] += Elem<TP>::to_f(W[(int64_t)o * w + i]) * acc[ii][j];
    }
  }
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
#pragma unroll
  for (int j = 0; j < simt::TN; ++j) red[ty][tx + 16 * j] = colpart[j];
  __syncthreads();
  for (int c = threadIdx.x; c < simt::BN; c += simt::kThreads) {
    const int i = n0 + c;
    if (i >= w) continue;
    float s = 0.f;
#pragma unroll
    for (int y = 0; y < 16; ++y) s += red[y][c];
    dgamma_partial[(int64_t)to * tab.total + tab.off[b] + i] = s;
  }
}

// gs[m, off_b + i] = sum_o dY[m,b,o] W_b[o, i]   (fp32 workspace)
template <typename T, typename TP>
__global__ void __launch_bounds__(simt::kThreads)
    band_split_bwd_gs(const T* __restrict__ dy, int64_t rows, BandTable tab, int64_t O, float* __restrict__ gs) {
  __shared__ simt::Smem sm;
  const int b = blockIdx.y;
  const int64_t w = tab.off[b + 1] - tab.off[b];
  const int nti = simt::tiles(tab.max_width, simt::BN);
  const int m0 = (blockIdx.x / nti) * simt::BM;
  const int n0 = (blockIdx.x % nti) * simt::BN;
  if (n0 >= w) return;
  float acc[simt::TM][simt::TN];
  simt::mainloop<T, TP, true, false>(sm, dy + (int64_t)b * O, (int64_t)tab.count * O, 1,
                                     static_cast<const TP*>(tab.ptr1[b]), 1, w, m0, (int)rows, n0, (int)w, (int)O,
                                     false, nullptr, acc);
#pragma unroll
  for (int ii = 0; ii < simt::TM; ++ii) {
    const int m = m0 + simt::row_of(ii);
    if (m >= rows) continue;
#pragma unroll
    for (int j = 0; j < simt::TN; ++j) {
      const int i = n0 + simt::col_of(j);
      if (i < w) gs[(int64_t)m * tab.total + tab.off[b] + i] = acc[ii][j];
    }
  }
}

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads)
    band_split_bwd_input(const float* __restrict__ gs, const T* __restrict__ normed, const float* __restrict__ inv_norm,
                         int64_t rows, BandTable tab, T* __restrict__ grad_x) {
  const int lane = threadIdx.x & 31;
  const int64_t pairs = rows * tab.count;
  for (int64_t p = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); p < pairs; p += (int64_t)gridDim.x * kWarps) {
    const int64_t r = p / tab.count;
    const int b = (int)(p % tab.count);
    const int64_t w = tab.off[b + 1] - tab.off[b];
    const float s = sqrtf((float)w);
    const TP* gamma = static_cast<const TP*>(tab.ptr0[b]);
    const int64_t base = r * tab.total + tab.off[b];
    float dot = 0.f;
    for (int64_t i = lane; i < w; i += 32) dot += gs[base + i] * Elem<TP>::to_f(gamma[i]) * Elem<T>::to_f(normed[base + i]);
    dot = warp_sum(dot);
    const float inv = inv_norm[r * tab.count + b];
    const float ds = dot / s;
    for (int64_t i = lane; i < w; i += 32) {
      const float gn = gs[base + i] * Elem<TP>::to_f(gamma[i]);
      grad_x[base + i] = Elem<T>::from_f(inv * (gn * s - Elem<T>::to_f(normed[base + i]) * ds));
    }
  }
}

struct BwdWorkspace {
  int64_t dgamma_partial_off, db_partial_off, gs_off, total_bytes;
  int o_tiles, row_chunks;
};

BwdWorkspace bwd_layout(int64_t rows, int64_t total, int nb, int64_t O, bool need_grad_x) {
  BwdWorkspace w;
  w.o_tiles = simt::tiles(O, simt::BM);
  w.row_chunks = red::chunks(rows);
  auto align = [](int64_t v) { return (v + 255) & ~(int64_t)255; };
  w.dgamma_partial_off = 0;
  w.db_partial_off = align((int64_t)w.o_tiles * total * 4);
  w.gs_off = w.db_partial_off + align((int64_t)w.row_chunks * nb * O * 4);
  w.total_bytes = w.gs_off + (need_grad_x ? align(rows * total * 4) : 0);
  return w;
}

int grid_pairs(int64_t pairs) {
  int64_t g = (pairs + kWarps - 1) / kWarps;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

template <typename T, typename TP>
int fwd_impl(const void* x, int64_t rows, XLayout lx, const BandTable& tab, int64_t O, void* out, void* normed,
             float* inv_norm, cudaStream_t stream) {
  band_norm_kernel<T><<<grid_pairs(rows * tab.count), kThreads, 0, stream>>>(
      static_cast<const T*>(x), rows, lx, tab, static_cast<T*>(normed), inv_norm);
  PMB_CHECK_LAUNCH("pmb_band_split_forward(norm)");
  dim3 grid(simt::tiles(rows, simt::BM) * simt::tiles(O, simt::BN), tab.count);
  if (lx.s_feat == 1)
    band_split_fwd_gemm<T, TP, true><<<grid, simt::kThreads, 0, stream>>>(static_cast<const T*>(x), rows, lx, tab,
                                                                           O, inv_norm, static_cast<T*>(out));
  else
    band_split_fwd_gemm<T, TP, false><<<grid, simt::kThreads, 0, stream>>>(static_cast<const T*>(x), rows, lx, tab,
                                                                            O, inv_norm, static_cast<T*>(out));
  PMB_CHECK_LAUNCH("pmb_band_split_forward(gemm)");
  return PMB_OK;
}

template <typename T, typename TP>
int bwd_impl(const void* dy, const void* normed, const float* inv_norm, int64_t rows, const BandTable& wtab,
             const BandTable& gtab, const BandTable& btab, int64_t O, void* grad_x, char* ws, const BwdWorkspace& L,
             int pcode, cudaStream_t stream) {
  float* dgp = reinterpret_cast<float*>(ws + L.dgamma_partial_off);
  float* dbp = reinterpret_cast<float*>(ws + L.db_partial_off);
  float* gs = reinterpret_cast<float*>(ws + L.gs_off);
  const int nti = simt::tiles(wtab.max_width, simt::BN);
  dim3 gw(L.o_tiles * nti, wtab.count);
  band_split_bwd_weight<T, TP><<<gw, simt::kThreads, 0, stream>>>(static_cast<const T*>(dy), static_cast<const T*>(normed),
                                                               rows, wtab, O, dgp);
  PMB_CHECK_LAUNCH("pmb_band_split_backward(weight)");
  red::colsum_finalize_bands<<<(int)((wtab.total + 255) / 256), red::kThreads, 0, stream>>>(dgp, L.o_tiles, wtab.total,
                                                                                             gtab, pcode);
  PMB_CHECK_LAUNCH("pmb_band_split_backward(gamma)");
  if (btab.count > 0) {
    const int64_t cols = (int64_t)wtab.count * O;
    dim3 gp((int)((cols + 255) / 256), L.row_chunks);
    red::colsum_partial<T><<<gp, red::kThreads, 0, stream>>>(static_cast<const T*>(dy), rows, cols, cols, dbp);
    PMB_CHECK_LAUNCH("pmb_band_split_backward(bias partial)");
    red::colsum_finalize_bands<<<(int)((cols + 255) / 256), red::kThreads, 0, stream>>>(dbp, L.row_chunks, cols, btab,
                                                                                         pcode);
    PMB_CHECK_LAUNCH("pmb_band_split_backward(bias)");
  }
  if (grad_x != nullptr) {
    dim3 gg(simt::tiles(rows, simt::BM) * nti, wtab.count);
    band_split_bwd_gs<T, TP><<<gg, simt::kThreads, 0, stream>>>(static_cast<const T*>(dy), rows, wtab, O, gs);
    PMB_CHECK_LAUNCH("pmb_band_split_backward(gs)");
    band_split_bwd_input<T, TP><<<grid_pairs(rows * wtab.count), kThreads, 0, stream>>>(
        gs, static_cast<const T*>(normed), inv_norm, rows, wtab, static_cast<T*>(grad_x));
    PMB_CHECK_LAUNCH("pmb_band_split_backward(input)");
  }
  return PMB_OK;
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_band_split_forward(const void* x, int64_t rows, int64_t x_stride_row, int64_t x_stride_band,
                                      int64_t x_stride_feat, int num_bands, const int64_t* widths,
                                      const void* const* gammas, const void* const* weights,
                                      const void* const* biases, int64_t out_features, void* out, void* normed,
                                      float* inv_norm, int dtype, int param_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_band_split_forward";
  BandTable tab;
  int st = make_band_table(tab, num_bands, widths, gammas, weights, biases, name);
  if (st) return st;
  PMB_REQUIRE(rows >= 0 && out_features > 0, "%s: bad shape rows=%lld out_features=%lld", name, (long long)rows,
              (long long)out_features);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(x && out && inv_norm && gammas && weights, "%s: NULL tensor argument", name);
  for (int b = 0; b < num_bands; ++b)
    PMB_REQUIRE(tab.ptr0[b] && tab.ptr1[b], "%s: band %d has a NULL gamma or weight", name, b);
  PMB_REQUIRE(x_stride_band < 0 || (tab.max_width == tab.total / num_bands && tab.max_width * num_bands == tab.total),
              "%s: a band stride requires equal band widths", name);
  XLayout lx{x_stride_row, x_stride_band, x_stride_feat};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name,
                            [&] { return fwd_impl<T, TP>(x, rows, lx, tab, out_features, out, normed, inv_norm, s); });
}

extern "C" int64_t pmb_band_split_backward_workspace_size(int64_t rows, int num_bands, const int64_t* widths,
                                                          int64_t out_features, int need_grad_x) {
  if (num_bands <= 0 || widths == nullptr || rows < 0) return 0;
  int64_t total = 0;
  for (int b = 0; b < num_bands; ++b) total += widths[b];
  return bwd_layout(rows, total, num_bands, out_features, need_grad_x != 0).total_bytes;
}

extern "C" int pmb_band_split_backward(const void* grad_out, const void* normed, const float* inv_norm, int64_t rows,
                                       int num_bands, const int64_t* widths, const void* const* gammas,
                                       const void* const* weights, int64_t out_features, void* grad_x,
                                       void* const* grad_gammas, void* const* grad_weights, void* const* grad_biases,
                                       int dtype, int param_dtype, void* workspace, int64_t workspace_bytes,
                                       void* stream) {
  clear_error();
  const char* name = "pmb_band_split_backward";
  BandTable wtab, gtab, btab;
  int st = make_band_table(wtab, num_bands, widths, gammas, weights, (const void* const*)grad_weights, name);
  if (st) return st;
  st = make_band_table(gtab, num_bands, widths, (const void* const*)grad_gammas, nullptr, nullptr, name);
  if (st) return st;
  btab.count = 0;
  if (grad_biases != nullptr) {
    std::vector<int64_t> ow(num_bands, out_features);
    st = make_band_table(btab, num_bands, ow.data(), (const void* const*)grad_biases, nullptr, nullptr, name);
    if (st) return st;
  }
  PMB_REQUIRE(rows >= 0 && out_features > 0, "%s: bad shape", name);
  PMB_REQUIRE(grad_gammas && grad_weights && gammas && weights, "%s: NULL per-band pointer array", name);
  for (int b = 0; b < num_bands; ++b)
    PMB_REQUIRE(wtab.ptr0[b] && wtab.ptr1[b] && wtab.ptr2[b] && gtab.ptr0[b] && (btab.count == 0 || btab.ptr0[b]),
                "%s: band %d has a NULL parameter or gradient pointer", name, b);
  const BwdWorkspace L = bwd_layout(rows, wtab.total, num_bands, out_features, grad_x != nullptr);
  if (workspace_bytes < L.total_bytes || (L.total_bytes > 0 && workspace == nullptr)) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)L.total_bytes);
    return PMB_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    // Zero-row batch: every gradient is zero.
    const int es = dtype_size(param_dtype);
    PMB_REQUIRE(es > 0, "%s: unsupported parameter dtype %d", name, param_dtype);
    for (int b = 0; b < num_bands; ++b) {
      const int64_t w = wtab.off[b + 1] - wtab.off[b];
      PMB_CHECK_CUDA(cudaMemsetAsync(const_cast<void*>(wtab.ptr2[b]), 0, w * out_features * es, s), name);
      PMB_CHECK_CUDA(cudaMemsetAsync(const_cast<void*>(gtab.ptr0[b]), 0, w * es, s), name);
      if (btab.count) PMB_CHECK_CUDA(cudaMemsetAsync(const_cast<void*>(btab.ptr0[b]), 0, out_features * es, s), name);
    }
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && normed && inv_norm, "%s: NULL tensor argument", name);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    return bwd_impl<T, TP>(grad_out, normed, inv_norm, rows, wtab, gtab, btab, out_features, grad_x,
                           static_cast<char*>(workspace), L, param_dtype, s);
  });
}
