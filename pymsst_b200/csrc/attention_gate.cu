// Per-head attention output gate: gate[r,h] = sigmoid(x[r,:] . Wg[h,:] + bg[h]),
// out[r, h*Dh + d] = attn[r,h,d] * gate[r,h], forward and backward.
// Reference semantics: src/pymsst/training/cuda/fused_band_split.cu:1778-2036
// (called from src/pymsst/training/fused_roformer.py:793-818, 1228-1262).
//
// attn is addressed with strides so the attention output can be read in the
// [batch, heads, seq, Dh] layout the attention kernel produces: row
// r = bi*seq + n, element (r, h, d) at bi*s_b + n*s_n + h*s_h + d.  The gate
// row product, sigmoid and gating are one warp-per-row pass (the reference
// uses two launches); the backward writes grad_attn with the attn strides.
#include "common.cuh"
#include "reduce.cuh"

namespace pmb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxHeads = 16;
constexpr int kRowsPerChunk = 256;

struct AttnLayout {
  int64_t seq, s_b, s_n, s_h;
  __device__ __forceinline__ int64_t row_base(int64_t r) const { return (r / seq) * s_b + (r % seq) * s_n; }
};

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads)
    gate_fwd(const T* __restrict__ attn, AttnLayout la, const T* __restrict__ x, const TP* __restrict__ W,
             const TP* __restrict__ bias, int64_t rows, int H, int Dh, int dim, T* __restrict__ out,
             T* __restrict__ gate) {
  extern __shared__ float sw[];  // [H][dim]
  for (int e = threadIdx.x; e < H * dim; e += kThreads) sw[e] = Elem<TP>::to_f(W[e]);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * kWarps) {
    float dots[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) dots[h] = 0.f;
    for (int i = lane; i < dim; i += 32) {
      const float xv = Elem<T>::to_f(x[r * dim + i]);
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h < H) dots[h] += xv * sw[h * dim + i];
    }
    float g[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
      if (h < H) {
        const float d = warp_sum(dots[h]);
        g[h] = round_to<T>(sigmoidf_(d + Elem<TP>::to_f(bias[h])));
      } else {
        g[h] = 0.f;
      }
    }
    if (lane < H) {
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h == lane) gate[r * H + h] = Elem<T>::from_f(g[h]);
    }
    const int64_t ab = la.row_base(r);
    for (int e = lane; e < H * Dh; e += 32) {
      const int h = e / Dh, d = e % Dh;
      float gh = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxHeads; ++k)
        if (k == h) gh = g[k];
      out[r * (int64_t)H * Dh + e] = Elem<T>::from_f(Elem<T>::to_f(attn[ab + h * la.s_h + d]) * gh);
    }
  }
}

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads)
    gate_bwd_rows(const T* __restrict__ grad_out, const T* __restrict__ attn, AttnLayout la, const TP* __restrict__ W,
                  const T* __restrict__ gate, int64_t rows, int H, int Dh, int dim, T* __restrict__ grad_attn,
                  T* __restrict__ grad_x, float* __restrict__ ggp) {
  extern __shared__ float sw[];  // [H][dim]
  for (int e = threadIdx.x; e < H * dim; e += kThreads) sw[e] = Elem<TP>::to_f(W[e]);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * kWarps) {
    const int64_t ab = la.row_base(r);
    float gs[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) gs[h] = 0.f;
    for (int e = lane; e < H * Dh; e += 32) {
      const int h = e / Dh, d = e % Dh;
      const float g = Elem<T>::to_f(grad_out[r * (int64_t)H * Dh + e]);
      const float a = Elem<T>::to_f(attn[ab + h * la.s_h + d]);
      const float gv = Elem<T>::to_f(gate[r * H + h]);
      grad_attn[ab + h * la.s_h + d] = Elem<T>::from_f(g * gv);
#pragma unroll
      for (int k = 0; k < kMaxHeads; ++k)
        if (k == h) gs[k] += g * a;
    }
    float gp[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
      if (h < H) {
        const float gv = Elem<T>::to_f(gate[r * H + h]);
        gp[h] = warp_sum(gs[h]) * gv * (1.0f - gv);
      } else {
        gp[h] = 0.f;
      }
    }
    if (lane < H) {
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h == lane) ggp[r * H + h] = gp[h];
    }
    for (int i = lane; i < dim; i += 32) {
      float acc = 0.f;
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h < H) acc += gp[h] * sw[h * dim + i];
      grad_x[r * dim + i] = Elem<T>::from_f(acc);
    }
  }
}

// partial[chunk][h*(dim+1) + i] = sum_{r in chunk} ggp[r,h] * x[r,i]; column dim holds the bias sum.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    gate_bwd_weight_partial(const float* __restrict__ ggp, const T* __restrict__ x, int64_t rows, int H, int dim,
                            float* __restrict__ partial) {
  const int cols = H * (dim + 1);
  const int64_t r0 = (int64_t)blockIdx.y * kRowsPerChunk;
  const int64_t r1 = r0 + kRowsPerChunk < rows ? r0 + kRowsPerChunk : rows;
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  const int h = c / (dim + 1), i = c % (dim + 1);
  float acc = 0.f;
  for (int64_t r = r0; r < r1; ++r) {
    const float g = ggp[r * H + h];
    acc += i == dim ? g : g * Elem<T>::to_f(x[r * dim + i]);
  }
  partial[(int64_t)blockIdx.y * cols + c] = acc;
}

template <typename TP>
__global__ void __launch_bounds__(kThreads)
    gate_bwd_weight_finalize(const float* __restrict__ partial, int chunks, int H, int dim, TP* __restrict__ grad_w,
                             TP* __restrict__ grad_b) {
  const int cols = H * (dim + 1);
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int k = 0; k < chunks; ++k) s += partial[(int64_t)k * cols + c];
  const int h = c / (dim + 1), i = c % (dim + 1);
  if (i == dim)
    grad_b[h] = Elem<TP>::from_f(s);
  else
    grad_w[h * dim + i] = Elem<TP>::from_f(s);
}

int row_grid(int64_t rows) {
  int64_t g = (rows + kWarps - 1) / kWarps;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }
int64_t chunks_of(int64_t rows) { return (rows + kRowsPerChunk - 1) / kRowsPerChunk; }

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_attention_gate_forward(const void* attn, int64_t seq_len, int64_t attn_stride_batch,
                                          int64_t attn_stride_seq, int64_t attn_stride_head, const void* x,
                                          const void* weight, const void* bias, int64_t rows, int64_t heads,
                                          int64_t dim_head, int64_t dim, void* out, void* gate, int dtype,
                                          int param_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_attention_gate_forward";
  PMB_REQUIRE(rows >= 0 && heads > 0 && heads <= kMaxHeads && dim_head > 0 && dim > 0 && seq_len > 0,
              "%s: bad shape (heads must be 1..%d)", name, kMaxHeads);
  PMB_REQUIRE(heads * dim * 4 <= 96 * 1024, "%s: heads*dim too large", name);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(attn && x && weight && bias && out && gate, "%s: NULL tensor argument", name);
  AttnLayout la{seq_len, attn_stride_batch, attn_stride_seq, attn_stride_head};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)heads * dim * sizeof(float);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if (smem > 48 * 1024)
      PMB_CHECK_CUDA(cudaFuncSetAttribute(gate_fwd<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                     name);
    gate_fwd<T, TP><<<row_grid(rows), kThreads, smem, s>>>(
        static_cast<const T*>(attn), la, static_cast<const T*>(x), static_cast<const TP*>(weight),
        static_cast<const TP*>(bias), rows, (int)heads, (int)dim_head, (int)dim, static_cast<T*>(out),
        static_cast<T*>(gate));
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

extern "C" int64_t pmb_attention_gate_backward_workspace_size(int64_t rows, int64_t heads, int64_t dim) {
  if (rows <= 0 || heads <= 0 || dim <= 0) return 0;
  return align256(rows * heads * 4) + align256(chunks_of(rows) * heads * (dim + 1) * 4);
}

extern "C" int pmb_attention_gate_backward(const void* grad_out, const void* attn, int64_t seq_len,
                                           int64_t attn_stride_batch, int64_t attn_stride_seq,
                                           int64_t attn_stride_head, const void* x, const void* weight,
                                           const void* gate, int64_t rows, int64_t heads, int64_t dim_head,
                                           int64_t dim, void* grad_attn, void* grad_x, void* grad_weight,
                                           void* grad_bias, int dtype, int param_dtype, void* workspace,
                                           int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_attention_gate_backward";
  PMB_REQUIRE(rows >= 0 && heads > 0 && heads <= kMaxHeads && dim_head > 0 && dim > 0 && seq_len > 0,
              "%s: bad shape (heads must be 1..%d)", name, kMaxHeads);
  PMB_REQUIRE(heads * dim * 4 <= 96 * 1024, "%s: heads*dim too large", name);
  PMB_REQUIRE(grad_weight && grad_bias, "%s: NULL gradient argument", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int es = dtype_size(param_dtype);
  PMB_REQUIRE(es > 0, "%s: unsupported parameter dtype %d", name, param_dtype);
  if (rows == 0) {
    PMB_CHECK_CUDA(cudaMemsetAsync(grad_weight, 0, heads * dim * es, s), name);
    PMB_CHECK_CUDA(cudaMemsetAsync(grad_bias, 0, heads * es, s), name);
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && attn && x && weight && gate && grad_attn && grad_x, "%s: NULL tensor argument", name);
  const int64_t need = pmb_attention_gate_backward_workspace_size(rows, heads, dim);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  float* ggp = static_cast<float*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + align256(rows * heads * 4));
  AttnLayout la{seq_len, attn_stride_batch, attn_stride_seq, attn_stride_head};
  const size_t smem = (size_t)heads * dim * sizeof(float);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if (smem > 48 * 1024)
      PMB_CHECK_CUDA(
          cudaFuncSetAttribute(gate_bwd_rows<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), name);
    gate_bwd_rows<T, TP><<<row_grid(rows), kThreads, smem, s>>>(
        static_cast<const T*>(grad_out), static_cast<const T*>(attn), la, static_cast<const TP*>(weight),
        static_cast<const T*>(gate), rows, (int)heads, (int)dim_head, (int)dim, static_cast<T*>(grad_attn),
        static_cast<T*>(grad_x), ggp);
    PMB_CHECK_LAUNCH(name);
    const int cols = (int)(heads * (dim + 1));
    const int nch = (int)chunks_of(rows);
    dim3 gp((cols + kThreads - 1) / kThreads, nch);
    gate_bwd_weight_partial<T><<<gp, kThreads, 0, s>>>(ggp, static_cast<const T*>(x), rows, (int)heads, (int)dim,
                                                       partial);
    PMB_CHECK_LAUNCH(name);
    gate_bwd_weight_finalize<TP><<<(cols + kThreads - 1) / kThreads, kThreads, 0, s>>>(
        partial, nch, (int)heads, (int)dim, static_cast<TP*>(grad_weight), static_cast<TP*>(grad_bias));
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}
