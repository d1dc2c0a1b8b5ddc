// Transformer feed-forward block (Linear -> GELU -> Linear) on the tcgen05
// tensor cores, bf16 / fp16 activations, fp32 or 16-bit parameters.
//
// Forward:  pre = x W1^T + b1 (stored, rounded to the activation dtype),
//           act = gelu(pre) (stored), out = act W2^T + b2;
//           bias and GELU are GEMM epilogues.
// Backward: grad_b2 = column sums of grad_out; grad_W2 = grad_out^T act
//           (split-K); d_pre = (grad_out W2) * gelu'(pre) with the GELU
//           derivative and the grad_b1 column partials in the GEMM epilogue;
//           grad_W1 = d_pre^T x (split-K); grad_x = d_pre W1.
// GELU is the exact (erf) form of torch.nn.GELU(): gelu(v) = v * Phi(v),
// gelu'(v) = Phi(v) + v * phi(v), evaluated as in the elementwise passes
// (gelu.cuh: for 16-bit values the logistic fit that rounds to the exact
// GELU).  Intermediate values are rounded to the
// activation dtype where the unfused autocast path stores them (the linear
// outputs and the GELU output), so both paths see the same bf16 tensors.
// The reference runs this block through torch (pymss-core FeedForward,
// called per layer from src/pymsst/training/fused_roformer.py:256-824).
#include "dense_gemm.cuh"
#include "gelu.cuh"
#include "reduce.cuh"

namespace pmb {
unsigned int timeout_flag_ff(int reset) { return umma::flag_reader(reset); }

namespace {

// pre / act = (acc + b1) / gelu(acc + b1), both stored in T (the 16-bit GELU of gelu.cuh, equal to the exact GELU
// after rounding).  With `use_tma` both go out as TMA tile stores ([rows, hidden] maps; hidden is a multiple of 32).
template <typename T, typename TP>
struct GeluEpi {
  T* pre;
  T* act;
  const TP* bias;
  int64_t ld;
  int use_tma;
  CUtensorMap pre_map, act_map;
  using Pre = dense::BiasPre;  // the bias slice, loaded a tile ahead
  __device__ void prefetch(const ugemm::Plan&, const ugemm::TileCtx& t, Pre& p) const {
    dense::prefetch_bias(t, p, [&](int64_t col) { return Elem<TP>::to_f(bias[col]); });
  }
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t, const Pre& bp) const {
    const int64_t base = (int64_t)t.row0 * ld + t.n0;
    int q = 0;
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BN; c0 += 32 * ugemm::kSubs, ++q) {
      if (c0 >= t.n_valid) break;
      const int ncols = min(32, t.n_valid - c0);
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
      const float bl = dense::bias_of(bp, q);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = round_to<T>(v[j] + __shfl_sync(0xffffffffu, bl, j));
      if (use_tma) {
        ugemm::warp_tma_store<T>(t, v, &pre_map, t.n0 + c0, t.row0);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_of<T>(v[j]);
        ugemm::warp_tma_store<T>(t, v, &act_map, t.n0 + c0, t.row0);
        continue;
      }
      ugemm::warp_store<T>(t.stage, v, pre + base + c0, ld, t.rows_valid, ncols);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_of<T>(v[j]);
      ugemm::warp_store<T>(t.stage, v, act + base + c0, ld, t.rows_valid, ncols);
    }
  }
};

// d_pre = round(acc) * gelu'(pre), stored in T; the column sums of the stored
// values over this warp's 32 rows go to partial[row0 / 32][col] (fp32).
template <typename T>
struct DGeluEpi {
  T* dpre;
  const T* pre;
  float* partial;
  int64_t ld;
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    const int lane = threadIdx.x & 31;
    const int64_t base = (int64_t)t.row0 * ld + t.n0;
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BN; c0 += 32 * ugemm::kSubs) {
      if (c0 >= t.n_valid) break;
      const int ncols = min(32, t.n_valid - c0);
      float v[32], p[32];
      umma::tmem_ld32(t.taddr + c0, v);
      ugemm::warp_load<T>(t.stage, pre + base + c0, ld, t.rows_valid, ncols, p);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = round_to<T>(v[j]) * gelu_grad_of<T>(p[j]);
      ugemm::warp_store<T>(t.stage, v, dpre + base + c0, ld, t.rows_valid, ncols);
      // column sums of the staged (rounded) block, rows in order
      float s = 0.f;
      for (int r = 0; r < t.rows_valid; ++r)
        s += Elem<T>::to_f(reinterpret_cast<const T*>(t.stage + r * ugemm::kStageRowBytes)[lane]);
      if (lane < ncols && t.rows_valid > 0) partial[(int64_t)(t.row0 / 32) * ld + t.n0 + c0 + lane] = s;
      __syncwarp();
    }
  }
};

// partial[chunk][c] = column sums of a [rows, cols] 16-bit matrix over
// 64-row chunks, two adjacent columns per thread.
template <typename T>
__global__ void __launch_bounds__(256)
    colsum_chunks(const T* __restrict__ src, int64_t rows, int64_t cols, float* __restrict__ partial) {
  const int64_t c = 2 * ((int64_t)blockIdx.x * 256 + threadIdx.x);
  if (c >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.y * 64;
  const int64_t r1 = r0 + 64 < rows ? r0 + 64 : rows;
  float s0 = 0.f, s1 = 0.f;
  const bool pair = c + 1 < cols && (cols & 1) == 0;
#pragma unroll 4
  for (int64_t r = r0; r < r1; ++r) {
    if (pair) {
      const T* p = src + r * cols + c;
      s0 += Elem<T>::to_f(p[0]);
      s1 += Elem<T>::to_f(p[1]);
    } else {
      s0 += Elem<T>::to_f(src[r * cols + c]);
      if (c + 1 < cols) s1 += Elem<T>::to_f(src[r * cols + c + 1]);
    }
  }
  partial[(int64_t)blockIdx.y * cols + c] = s0;
  if (c + 1 < cols) partial[(int64_t)blockIdx.y * cols + c + 1] = s1;
}

int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }

struct Workspace {
  int64_t dpre, partial, wgrad, bytes;
};

Workspace layout(int64_t rows, int64_t dim, int64_t hidden, int es) {
  Workspace w;
  w.dpre = 0;
  w.partial = align256(rows * hidden * es);
  const int64_t prow = (rows + 31) / 32 > (rows + 63) / 64 ? (rows + 31) / 32 : (rows + 63) / 64;
  const int64_t pcols = hidden > dim ? hidden : dim;
  w.wgrad = w.partial + align256(prow * pcols * 4);
  const int64_t a = dense::wgrad_workspace(dim, hidden, rows), b = dense::wgrad_workspace(hidden, dim, rows);
  w.bytes = w.wgrad + (a > b ? a : b);
  return w;
}

bool shapes_ok(int64_t dim, int64_t hidden) { return dim % 8 == 0 && hidden % 8 == 0; }

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_feed_forward_forward(const void* x, const void* w1, const void* b1, const void* w2, const void* b2,
                                        int64_t rows, int64_t dim, int64_t hidden, void* pre, void* act, void* out,
                                        int dtype, int param_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_feed_forward_forward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  PMB_REQUIRE(rows >= 0 && rows < (1ll << 31) && dim > 0 && hidden > 0 && shapes_ok(dim, hidden),
              "%s: bad shape (dim and hidden must be multiples of 8)", name);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(x && w1 && b1 && w2 && b2 && pre && act && out, "%s: NULL tensor argument", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fp16 = dtype == PMB_FLOAT16;
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 4) {
      set_error("%s: fp32 activations are not supported", name);
      return PMB_ERR_UNSUPPORTED_DTYPE;
    } else {
      const int bn = dense::pick_bn(hidden);
      CUtensorMap ma, mb;
      int st = dense::make_maps(ma, mb, x, dim, false, w1, dim, false, rows, hidden, dim, bn, dtype, name);
      if (st) return st;
      ugemm::Plan plan;
      plan.num_groups = 1;
      plan.g[0] = ugemm::Group{(int)rows, (int)hidden, (int)dim, 0, 0, 0, 0, 0, 0};
      GeluEpi<T, TP> epi{static_cast<T*>(pre), static_cast<T*>(act), static_cast<const TP*>(b1), hidden, 0, {}, {}};
      epi.use_tma = hidden % 32 == 0 &&
                    tma::make_store_map_2d(epi.pre_map, pre, dtype, hidden, rows, hidden * 2, name) == PMB_OK &&
                    tma::make_store_map_2d(epi.act_map, act, dtype, hidden, rows, hidden * 2, name) == PMB_OK;
      if (!epi.use_tma) clear_error();
      st = bn == 256 ? dense::launch<256, false, false>(ma, mb, plan, epi, fp16, s, name)
                     : (bn == 128 ? dense::launch<128, false, false>(ma, mb, plan, epi, fp16, s, name)
                                  : dense::launch<64, false, false>(ma, mb, plan, epi, fp16, s, name));
      if (st) return st;
      return dense::gemm(act, hidden, false, w2, hidden, false, out, dim, dtype, b2, Elem<TP>::code, PMB_ACT_NONE,
                         rows, dim, hidden, dtype, s, name);
    }
  });
}

extern "C" int64_t pmb_feed_forward_backward_workspace_size(int64_t rows, int64_t dim, int64_t hidden, int dtype) {
  const int es = dtype_size(dtype);
  if (rows <= 0 || dim <= 0 || hidden <= 0 || es <= 0) return 0;
  return layout(rows, dim, hidden, es).bytes;
}

extern "C" int pmb_feed_forward_backward(const void* grad_out, const void* x, const void* pre, const void* act,
                                         const void* w1, const void* w2, int64_t rows, int64_t dim, int64_t hidden,
                                         void* grad_x, void* grad_w1, void* grad_b1, void* grad_w2, void* grad_b2,
                                         int dtype, int param_dtype, void* workspace, int64_t workspace_bytes,
                                         void* stream) {
  clear_error();
  const char* name = "pmb_feed_forward_backward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  PMB_REQUIRE(rows >= 0 && rows < (1ll << 31) && dim > 0 && hidden > 0 && shapes_ok(dim, hidden),
              "%s: bad shape (dim and hidden must be multiples of 8)", name);
  PMB_REQUIRE(grad_w1 && grad_b1 && grad_w2 && grad_b2, "%s: NULL gradient argument", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int pes = dtype_size(param_dtype);
  PMB_REQUIRE(pes > 0, "%s: unsupported parameter dtype", name);
  if (rows == 0) {
    PMB_CHECK_CUDA(cudaMemsetAsync(grad_w1, 0, hidden * dim * pes, s), name);
    PMB_CHECK_CUDA(cudaMemsetAsync(grad_b1, 0, hidden * pes, s), name);
    PMB_CHECK_CUDA(cudaMemsetAsync(grad_w2, 0, dim * hidden * pes, s), name);
    PMB_CHECK_CUDA(cudaMemsetAsync(grad_b2, 0, dim * pes, s), name);
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && x && pre && act && w1 && w2, "%s: NULL tensor argument", name);
  const Workspace L = layout(rows, dim, hidden, dtype_size(dtype));
  if (workspace == nullptr || workspace_bytes < L.bytes) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)L.bytes);
    return PMB_ERR_WORKSPACE;
  }
  char* ws = static_cast<char*>(workspace);
  float* partial = reinterpret_cast<float*>(ws + L.partial);
  void* wg = ws + L.wgrad;
  const int64_t wg_bytes = workspace_bytes - L.wgrad;
  const int fp16 = dtype == PMB_FLOAT16;
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 4) {
      set_error("%s: fp32 activations are not supported", name);
      return PMB_ERR_UNSUPPORTED_DTYPE;
    } else {
      // grad_b2: column sums of grad_out
      const int64_t chunks = (rows + 63) / 64;
      dim3 g((unsigned)((dim / 2 + 255) / 256), (unsigned)chunks);
      colsum_chunks<T><<<g, 256, 0, s>>>(static_cast<const T*>(grad_out), rows, dim, partial);
      PMB_CHECK_LAUNCH(name);
      red::colsum_rows<<<red::colsum_rows_grid(dim), red::kThreads, 0, s>>>(partial, (int)chunks, dim, grad_b2,
                                                                            Elem<TP>::code);
      PMB_CHECK_LAUNCH(name);
      // grad_W2 = grad_out^T act
      int st = dense::wgrad(grad_out, dim, act, hidden, dim, hidden, rows, grad_w2, hidden, param_dtype, dtype, wg,
                            wg_bytes, s, name);
      if (st) return st;
      // d_pre = (grad_out W2) * gelu'(pre), grad_b1 partials
      T* dpre = reinterpret_cast<T*>(ws + L.dpre);
      {
        const int bn = dense::pick_bn(hidden);
        CUtensorMap ma, mb;
        st = dense::make_maps(ma, mb, grad_out, dim, false, w2, hidden, true, rows, hidden, dim, bn, dtype, name);
        if (st) return st;
        ugemm::Plan plan;
        plan.num_groups = 1;
        plan.g[0] = ugemm::Group{(int)rows, (int)hidden, (int)dim, 0, 0, 0, 0, 0, 0};
        DGeluEpi<T> epi{dpre, static_cast<const T*>(pre), partial, hidden};
        st = bn == 256 ? dense::launch<256, false, true>(ma, mb, plan, epi, fp16, s, name)
                       : (bn == 128 ? dense::launch<128, false, true>(ma, mb, plan, epi, fp16, s, name)
                                    : dense::launch<64, false, true>(ma, mb, plan, epi, fp16, s, name));
        if (st) return st;
        red::colsum_rows<<<red::colsum_rows_grid(hidden), red::kThreads, 0, s>>>(partial, (int)((rows + 31) / 32),
                                                                                 hidden, grad_b1, Elem<TP>::code);
        PMB_CHECK_LAUNCH(name);
      }
      // grad_W1 = d_pre^T x
      st = dense::wgrad(dpre, hidden, x, dim, hidden, dim, rows, grad_w1, dim, param_dtype, dtype, wg, wg_bytes, s,
                        name);
      if (st) return st;
      // grad_x = d_pre W1
      if (grad_x) {
        st = dense::gemm(dpre, hidden, false, w1, dim, true, grad_x, dim, dtype, nullptr, 0, PMB_ACT_NONE, rows, dim,
                         hidden, dtype, s, name);
        if (st) return st;
      }
      return PMB_OK;
    }
  });
}
