// BandSplit on the tcgen05 tensor cores (bf16 / fp16 activations, fp32 or
// 16-bit parameters): per band b of width w_b,
//   normed_b = x_b * inv * sqrt(w_b),  inv = 1 / max(||x_b||, eps)
//   out[m, b, :] = (normed_b * gamma_b) W_b^T + bias_b
// Reference semantics: src/pymsst/training/cuda/fused_band_split.cu:590-1003
// (ragged band split) and :14-247; pure-torch form
// src/pymsst/training/fused_roformer.py:1265-1271.
//
// Layout.  The band features are ragged (w_b = 8 ... 516), so the norm pass
// writes `normed` in a padded layout P: band b occupies columns
// [poff_b, poff_b + Kp_b) of a [rows, Kp] matrix, Kp_b = w_b rounded up to 64
// (the k-block), zero beyond w_b.  Every band then starts on a 128-byte
// boundary (TMA-aligned) and k-blocks never run into the next band.  The
// packed weight is (W_b * gamma_b) in the activation dtype in the same column
// layout, [O, Kp] (the tensor-core B operand), built once per forward and
// reused by the backward.
//
// Forward:  norm pass (inv, normed P), pack pass, one grouped GEMM (group = band:
//           M = rows, N = O, K = Kp_b) whose epilogue adds the bias and writes
//           out [rows, nb, O].
// Backward (the weight side; BandSplit's input is the STFT, which carries no
// gradient in training, and the row-norm input gradient stays on the exact
// SIMT path):  G_b = dY_b^T normed_b, a grouped GEMM with M = O, N = Kp_b,
//           K = rows (both operands MN-major); its epilogue writes
//           grad_W_b = G_b * gamma_b and per-32-row column partials of
//           sum_o W_b[o, i] G_b[o, i] (= grad_gamma_b); grad_bias is a column
//           sum of dY.
#include <vector>

#include "gemm_umma.cuh"
#include "reduce.cuh"
#include "tma.cuh"

namespace pmb {
unsigned int timeout_flag_band(int reset) { return umma::flag_reader(reset); }

namespace {

constexpr int kThreads = 256;
constexpr int kKp = 64;  // band padding unit (= the GEMM k-block)

struct BandCols {
  int nb;
  int w[kMaxBands];     // true widths
  int off[kMaxBands];   // column offset in the unpadded feature layout
  int poff[kMaxBands];  // column offset in the padded layout P
  int kp[kMaxBands];    // padded width
  int total, total_p;
};

BandCols make_cols(int nb, const int64_t* widths) {
  BandCols c;
  c.nb = nb;
  int off = 0, poff = 0;
  for (int b = 0; b < nb; ++b) {
    c.w[b] = (int)widths[b];
    c.off[b] = off;
    c.poff[b] = poff;
    c.kp[b] = (c.w[b] + kKp - 1) / kKp * kKp;
    off += c.w[b];
    poff += c.kp[b];
  }
  c.total = off;
  c.total_p = poff;
  return c;
}

struct XLayout {
  int64_t s_row, s_band, s_feat;  // s_band < 0: ragged (column offset off[b])
};

// One warp per (row, band): inv and the padded normed row segment.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    norm_padded(const T* __restrict__ x, int64_t rows, XLayout lx, BandCols bc, T* __restrict__ normed_p,
                float* __restrict__ inv_norm) {
  const int lane = threadIdx.x & 31;
  const int64_t pairs = rows * bc.nb;
  for (int64_t p = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); p < pairs;
       p += (int64_t)gridDim.x * (kThreads / 32)) {
    const int64_t r = p / bc.nb;
    const int b = (int)(p - r * bc.nb);
    const int w = bc.w[b];
    const T* xb = x + r * lx.s_row + (lx.s_band < 0 ? (int64_t)bc.off[b] * lx.s_feat : (int64_t)b * lx.s_band);
    float ss = 0.f;
    for (int i = lane; i < w; i += 32) {
      const float v = Elem<T>::to_f(xb[i * lx.s_feat]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / fmaxf(sqrtf(ss), 1.0e-12f);
    if (lane == 0) inv_norm[r * bc.nb + b] = inv;
    const float k = inv * sqrtf((float)w);
    T* nb_ = normed_p + r * bc.total_p + bc.poff[b];
    for (int i = lane; i < bc.kp[b]; i += 32)
      nb_[i] = Elem<T>::from_f(i < w ? Elem<T>::to_f(xb[i * lx.s_feat]) * k : 0.f);
  }
}

// Contiguous features (s_feat == 1, ragged): one CTA per row.  The row is
// staged in shared memory with 4-byte loads (rows need not be 16-byte
// aligned), then warp w handles bands w, w + 8, ...: sum of squares from
// shared memory, and the padded normalised segment written with coalesced
// stores.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    norm_padded_rows(const T* __restrict__ x, int64_t rows, int64_t s_row, BandCols bc, T* __restrict__ normed_p,
                     float* __restrict__ inv_norm) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* xs = reinterpret_cast<T*>(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * s_row;
    // total is even for 16-bit bands of 4-element multiples; copy pairs when aligned
    if ((reinterpret_cast<uintptr_t>(xr) & 3) == 0 && (bc.total & 1) == 0) {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(xr);
      uint32_t* dst = reinterpret_cast<uint32_t*>(xs);
      for (int i = threadIdx.x; i < bc.total / 2; i += kThreads) dst[i] = src[i];
    } else {
      for (int i = threadIdx.x; i < bc.total; i += kThreads) xs[i] = xr[i];
    }
    __syncthreads();
    for (int b = warp; b < bc.nb; b += kThreads / 32) {
      const int w = bc.w[b];
      const T* xb = xs + bc.off[b];
      float ss = 0.f;
      for (int i = lane; i < w; i += 32) {
        const float v = Elem<T>::to_f(xb[i]);
        ss += v * v;
      }
      ss = warp_sum(ss);
      const float inv = 1.0f / fmaxf(sqrtf(ss), 1.0e-12f);
      if (lane == 0) inv_norm[r * bc.nb + b] = inv;
      const float k = inv * sqrtf((float)w);
      T* nb_ = normed_p + r * bc.total_p + bc.poff[b];
      for (int i = lane; i < bc.kp[b]; i += 32) nb_[i] = Elem<T>::from_f(i < w ? Elem<T>::to_f(xb[i]) * k : 0.f);
    }
    __syncthreads();
  }
}

// packed[n, poff_b + k] for band b = blockIdx.y: threads over k, rows n strided.
template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads)
    pack_weights_band(BandTable tab, BandCols bc, int64_t O, T* __restrict__ packed) {
  const int b = blockIdx.y;
  const int w = bc.w[b], kp = bc.kp[b];
  const TP* W = static_cast<const TP*>(tab.ptr1[b]);
  const TP* g = static_cast<const TP*>(tab.ptr0[b]);
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < O * kp; e += (int64_t)gridDim.x * kThreads) {
    const int64_t n = e / kp;
    const int k = (int)(e - n * kp);
    const float v = k < w ? Elem<TP>::to_f(W[n * w + k]) * Elem<TP>::to_f(g[k]) : 0.f;
    packed[n * bc.total_p + bc.poff[b] + k] = Elem<T>::from_f(v);
  }
}

// out[m, b, n] = acc + bias_b[n]
template <typename T, typename TP>
struct BandOutEpi {
  T* out;
  int nb;
  int O;
  const void* bias[kMaxBands];
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    const int lane = threadIdx.x & 31;
    const int64_t ld = (int64_t)nb * O;
    T* base = out + (int64_t)t.row0 * ld + (int64_t)t.group * O + t.n0;
    const TP* bp = static_cast<const TP*>(bias[t.group]);
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BN; c0 += 32 * ugemm::kSubs) {
      if (c0 >= t.n_valid) break;
      const int ncols = min(32, t.n_valid - c0);
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
      const float bl = (bp != nullptr && lane < ncols) ? Elem<TP>::to_f(bp[t.n0 + c0 + lane]) : 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += __shfl_sync(0xffffffffu, bl, j);
      ugemm::warp_store<T>(t.stage, v, base + c0, ld, t.rows_valid, ncols);
    }
  }
};

// G tile (rows o of O, columns i of the band's padded width):
//   grad_W_b[o, i] = G[o, i] * gamma_b[i]   (i < w_b)
//   partial[row0 / 32][poff_b + i] = sum over this warp's 32 rows of W_b[o, i] * G[o, i]
template <typename TP>
struct WGradBandEpi {
  BandCols bc;
  const void* gamma[kMaxBands];
  const void* weight[kMaxBands];
  void* grad_w[kMaxBands];
  float* partial;
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    const int lane = threadIdx.x & 31;
    const int b = t.group;
    const int w = bc.w[b];
    const TP* gm = static_cast<const TP*>(gamma[b]);
    const TP* W = static_cast<const TP*>(weight[b]);
    TP* gW = static_cast<TP*>(grad_w[b]);
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BN; c0 += 32 * ugemm::kSubs) {
      const int i0 = t.n0 + c0;
      if (c0 >= t.n_valid || i0 >= w) break;
      const int ncols = min(32, w - i0);
      float v[32], wv[32];
      umma::tmem_ld32(t.taddr + c0, v);
      ugemm::warp_load<TP>(t.stage, W + (int64_t)t.row0 * w + i0, w, t.rows_valid, ncols, wv);
      const float gl = lane < ncols ? Elem<TP>::to_f(gm[i0 + lane]) : 0.f;
      float* st = reinterpret_cast<float*>(t.stage + lane * ugemm::kStageRowBytes);
#pragma unroll
      for (int j = 0; j < 32; ++j) st[j] = wv[j] * v[j];  // W * G, this lane's row
      __syncwarp();
      float s = 0.f;
      for (int r = 0; r < t.rows_valid; ++r) s += reinterpret_cast<const float*>(t.stage + r * ugemm::kStageRowBytes)[lane];
      if (lane < ncols && t.rows_valid > 0) partial[(int64_t)(t.row0 / 32) * bc.total_p + bc.poff[b] + i0 + lane] = s;
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= __shfl_sync(0xffffffffu, gl, j);
      ugemm::warp_store<TP>(t.stage, v, gW + (int64_t)t.row0 * w + i0, w, t.rows_valid, ncols);
    }
  }
};

// grad_gamma_b[i] = sum_q partial[q][poff_b + i]
template <typename TP>
__global__ void __launch_bounds__(kThreads)
    gamma_finalize(const float* __restrict__ partial, int nq, BandCols bc, BandTable gtab) {
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= bc.total_p) return;
  int lo = 0, hi = bc.nb - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (bc.poff[mid] <= c) lo = mid; else hi = mid - 1;
  }
  const int b = lo, i = c - bc.poff[b];
  if (i >= bc.w[b]) return;
  float s = 0.f;
  for (int q = 0; q < nq; ++q) s += partial[(int64_t)q * bc.total_p + c];
  static_cast<TP*>(const_cast<void*>(gtab.ptr0[b]))[i] = Elem<TP>::from_f(s);
}

int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }

struct Sizes {
  int64_t packed_bytes, normed_bytes, ws_bytes;
  int64_t ws_gpart, ws_bpart;
};

Sizes sizes_of(int64_t rows, const BandCols& bc, int64_t O, int es) {
  Sizes z;
  z.packed_bytes = align256(O * bc.total_p * es);
  z.normed_bytes = align256(rows * bc.total_p * es);
  z.ws_gpart = 0;
  z.ws_bpart = align256(((O + 31) / 32) * bc.total_p * 4);
  z.ws_bytes = z.ws_bpart + align256((int64_t)red::chunks(rows) * bc.nb * O * 4);
  return z;
}

int grid_for(int64_t n, int per) {
  int64_t g = (n + per - 1) / per;
  const int64_t cap = (int64_t)num_sms() * 16;
  return (int)(g > cap ? cap : (g < 1 ? 1 : g));
}

template <int BN, bool A_MN, bool B_MN, class Epi>
int run_gemm(const CUtensorMap& ma, const CUtensorMap& mb, ugemm::Plan& plan, const Epi& epi, int fp16,
             cudaStream_t s, const char* name) {
  constexpr int STAGES = BN == 256 ? 3 : 4;
  const int tiles = ugemm::build_plan(plan, BN);
  if (tiles == 0) return PMB_OK;
  auto kern = ugemm::umma_gemm_kernel<BN, STAGES, A_MN, B_MN, Epi>;
  const int smem = ugemm::smem_bytes<BN, STAGES>();
  PMB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), name);
  kern<<<ugemm::persistent_grid(tiles), ugemm::kThreads, smem, s>>>(ma, mb, plan, epi, fp16);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_band_split_tc_sizes(int64_t rows, int num_bands, const int64_t* widths, int64_t out_features,
                                       int dtype, int64_t* sizes) {
  clear_error();
  PMB_REQUIRE(num_bands > 0 && num_bands <= kMaxBands && widths && sizes && rows >= 0 && out_features > 0,
              "pmb_band_split_tc_sizes: bad arguments");
  for (int b = 0; b < num_bands; ++b) PMB_REQUIRE(widths[b] > 0, "pmb_band_split_tc_sizes: band %d is empty", b);
  const BandCols bc = make_cols(num_bands, widths);
  const Sizes z = sizes_of(rows, bc, out_features, dtype_size(dtype) > 0 ? dtype_size(dtype) : 2);
  sizes[0] = z.packed_bytes;
  sizes[1] = z.normed_bytes;
  sizes[2] = z.ws_bytes;
  sizes[3] = bc.total_p;
  return PMB_OK;
}

extern "C" int pmb_band_split_tc_forward(const void* x, int64_t rows, int64_t x_stride_row, int64_t x_stride_band,
                                         int64_t x_stride_feat, int num_bands, const int64_t* widths,
                                         const void* const* gammas, const void* const* weights,
                                         const void* const* biases, int64_t out_features, void* packed_weights,
                                         void* normed_padded, float* inv_norm, void* out, int dtype,
                                         int param_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_band_split_tc_forward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  BandTable tab;
  int st = make_band_table(tab, num_bands, widths, gammas, weights, biases, name);
  if (st) return st;
  PMB_REQUIRE(rows >= 0 && rows < (1ll << 31) && out_features > 0 && out_features % 8 == 0,
              "%s: bad shape (out_features must be a multiple of 8)", name);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(x && out && inv_norm && packed_weights && normed_padded, "%s: NULL tensor argument", name);
  for (int b = 0; b < num_bands; ++b)
    PMB_REQUIRE(tab.ptr0[b] && tab.ptr1[b], "%s: band %d has a NULL gamma or weight", name, b);
  PMB_REQUIRE(x_stride_band < 0 || (tab.max_width * num_bands == tab.total),
              "%s: a band stride requires equal band widths", name);
  const BandCols bc = make_cols(num_bands, widths);
  XLayout lx{x_stride_row, x_stride_band, x_stride_feat};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fp16 = dtype == PMB_FLOAT16;
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 4) {
      set_error("%s: fp32 activations are not supported", name);
      return PMB_ERR_UNSUPPORTED_DTYPE;
    } else {
      const size_t row_smem = (size_t)bc.total * sizeof(T);
      if (x_stride_band < 0 && x_stride_feat == 1 && row_smem <= 96 * 1024) {
        if (row_smem > 48 * 1024)
          PMB_CHECK_CUDA(cudaFuncSetAttribute(norm_padded_rows<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)row_smem),
                         name);
        const int g = (int)(rows < (int64_t)num_sms() * 8 ? rows : (int64_t)num_sms() * 8);
        norm_padded_rows<T><<<g, kThreads, row_smem, s>>>(static_cast<const T*>(x), rows, x_stride_row, bc,
                                                            static_cast<T*>(normed_padded), inv_norm);
      } else {
        norm_padded<T><<<grid_for(rows * num_bands, kThreads / 32), kThreads, 0, s>>>(
            static_cast<const T*>(x), rows, lx, bc, static_cast<T*>(normed_padded), inv_norm);
      }
      PMB_CHECK_LAUNCH(name);
      {
        int bx = (int)((out_features * 64 + kThreads - 1) / kThreads);
        dim3 pg((unsigned)(bx < 1 ? 1 : bx), (unsigned)num_bands);
        pack_weights_band<T, TP><<<pg, kThreads, 0, s>>>(tab, bc, out_features, static_cast<T*>(packed_weights));
      }
      PMB_CHECK_LAUNCH(name);
      CUtensorMap ma, mb;
      constexpr int BN = 256;
      int st2 = tma::make_map_3d(ma, normed_padded, dtype, bc.total_p, 1, rows, bc.total_p * 2, bc.total_p * 2, 64, 1,
                                 ugemm::BM, name);
      if (st2) return st2;
      st2 = tma::make_map_3d(mb, packed_weights, dtype, bc.total_p, 1, out_features, bc.total_p * 2,
                             bc.total_p * 2, 64, 1, BN, name);
      if (st2) return st2;
      ugemm::Plan plan;
      plan.num_groups = num_bands;
      BandOutEpi<T, TP> epi;
      epi.out = static_cast<T*>(out);
      epi.nb = num_bands;
      epi.O = (int)out_features;
      for (int b = 0; b < num_bands; ++b) {
        plan.g[b] = ugemm::Group{(int)rows, (int)out_features, bc.kp[b], bc.poff[b], 0, 0, bc.poff[b], 0, 0};
        epi.bias[b] = biases ? biases[b] : nullptr;
      }
      return run_gemm<BN, false, false>(ma, mb, plan, epi, fp16, s, name);
    }
  });
}

extern "C" int pmb_band_split_tc_backward(const void* grad_out, const void* normed_padded, int64_t rows,
                                          int num_bands, const int64_t* widths, const void* const* gammas,
                                          const void* const* weights, int64_t out_features,
                                          void* const* grad_gammas, void* const* grad_weights,
                                          void* const* grad_biases, int dtype, int param_dtype, void* workspace,
                                          int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_band_split_tc_backward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  BandTable wtab, gtab;
  int st = make_band_table(wtab, num_bands, widths, gammas, weights, (const void* const*)grad_weights, name);
  if (st) return st;
  st = make_band_table(gtab, num_bands, widths, (const void* const*)grad_gammas, nullptr, nullptr, name);
  if (st) return st;
  PMB_REQUIRE(rows > 0 && rows < (1ll << 31) && out_features > 0 && out_features % 8 == 0, "%s: bad shape", name);
  PMB_REQUIRE(grad_out && normed_padded && grad_gammas && grad_weights && gammas && weights,
              "%s: NULL tensor argument", name);
  for (int b = 0; b < num_bands; ++b)
    PMB_REQUIRE(wtab.ptr0[b] && wtab.ptr1[b] && wtab.ptr2[b] && gtab.ptr0[b] && (!grad_biases || grad_biases[b]),
                "%s: band %d has a NULL parameter or gradient pointer", name, b);
  const BandCols bc = make_cols(num_bands, widths);
  const Sizes z = sizes_of(rows, bc, out_features, dtype_size(dtype));
  if (workspace == nullptr || workspace_bytes < z.ws_bytes) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)z.ws_bytes);
    return PMB_ERR_WORKSPACE;
  }
  float* gpart = reinterpret_cast<float*>(static_cast<char*>(workspace) + z.ws_gpart);
  float* bpart = reinterpret_cast<float*>(static_cast<char*>(workspace) + z.ws_bpart);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fp16 = dtype == PMB_FLOAT16;
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 4) {
      set_error("%s: fp32 activations are not supported", name);
      return PMB_ERR_UNSUPPORTED_DTYPE;
    } else {
      // G_b = dY_b^T normed_b: A(m = o, k = r) = dY[r, b, o], B(n = i, k = r) = normed_p[r, poff_b + i]
      constexpr int BN = 128;
      CUtensorMap ma, mb;
      int st2 = tma::make_map_3d(ma, grad_out, dtype, out_features, num_bands, rows, out_features * 2,
                                 (int64_t)num_bands * out_features * 2, 64, 1, 64, name);
      if (st2) return st2;
      st2 = tma::make_map_3d(mb, normed_padded, dtype, bc.total_p, 1, rows, bc.total_p * 2, bc.total_p * 2, 64, 1, 64,
                             name);
      if (st2) return st2;
      ugemm::Plan plan;
      plan.num_groups = num_bands;
      WGradBandEpi<TP> epi;
      epi.bc = bc;
      epi.partial = gpart;
      for (int b = 0; b < num_bands; ++b) {
        plan.g[b] = ugemm::Group{(int)out_features, bc.kp[b], (int)rows, 0, b, 0, bc.poff[b], 0, 0};
        epi.gamma[b] = gammas[b];
        epi.weight[b] = weights[b];
        epi.grad_w[b] = grad_weights[b];
      }
      st2 = run_gemm<BN, true, true>(ma, mb, plan, epi, fp16, s, name);
      if (st2) return st2;
      gamma_finalize<TP><<<(bc.total_p + kThreads - 1) / kThreads, kThreads, 0, s>>>(
          gpart, (int)((out_features + 31) / 32), bc, gtab);
      PMB_CHECK_LAUNCH(name);
      if (grad_biases != nullptr) {
        BandTable btab;
        std::vector<int64_t> ow(num_bands, out_features);
        st2 = make_band_table(btab, num_bands, ow.data(), (const void* const*)grad_biases, nullptr, nullptr, name);
        if (st2) return st2;
        const int64_t cols = (int64_t)num_bands * out_features;
        dim3 gp((unsigned)((cols + 255) / 256), (unsigned)red::chunks(rows));
        red::colsum_partial<T><<<gp, red::kThreads, 0, s>>>(static_cast<const T*>(grad_out), rows, cols, cols, bpart);
        PMB_CHECK_LAUNCH(name);
        red::colsum_finalize_bands<<<(unsigned)((cols + 255) / 256), red::kThreads, 0, s>>>(
            bpart, red::chunks(rows), cols, btab, Elem<TP>::code);
        PMB_CHECK_LAUNCH(name);
      }
      return PMB_OK;
    }
  });
}
