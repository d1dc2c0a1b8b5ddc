// Split of the attention input projection into the attention layout, with the
// rotary embedding applied to q and k on the way (forward), and the inverse
// (backward): one memory pass each, so q/k make no separate rotary round trip.
//
//   qkv [B*N, 3, H, Dh]  (x W_qkv^T, the 'b n (qkv h d)' layout)
//   q, k, v [B, H, N, Dh] (the layout scaled-dot-product attention takes)
//   rotation of interleaved pairs by angle table cos/sin fp32 [N, Dh/2]:
//     (e, o) -> (e c - o s, o c + e s);  backward (e, o) -> (e c + o s, o c - e s)
// Reference semantics: rotary .cu:1077-1128 applied to q/k after
// qkv_to_bnhd (src/pymsst/training/fused_roformer.py:710-732, 793-818);
// the angles follow rotary-embedding-torch: theta_i = n / 10000^(2i/Dh).
#include "common.cuh"

namespace pmb {
namespace {

constexpr int kThreads = 256;

template <typename T, int P>
struct alignas((sizeof(T) * 2 * P) < 16 ? (sizeof(T) * 2 * P) : 16) Chunk {
  T v[2 * P];
};

struct QkvDims {
  int64_t B, N;
  int H, Dh;
  int64_t s_b, s_h, s_n;  // element strides of q / k / v (d contiguous)
  int64_t inner;          // rows ordered (outer, position, inner); sequence = outer * inner + inner index
};

// One warp per row (b, n) of the packed [B*N, 3, H, Dh] projection; lane l
// handles the P-pair chunks c = l, l + 32, ... of the row (c indexes
// (which, h, pair group) in that order).  Index math is 32-bit except the
// per-row bases; the angle table row n is shared by the whole warp.
template <typename T, int P, bool BACKWARD>
__global__ void __launch_bounds__(kThreads)
    qkv_rotary_kernel(T* __restrict__ qkv, const float* __restrict__ cosv, const float* __restrict__ sinv, QkvDims d,
                      T* __restrict__ q, T* __restrict__ k, T* __restrict__ v, int rotate_qk) {
  const int gph = d.Dh / (2 * P);         // chunks per head
  const int cpw = d.H * gph;              // chunks per q / k / v part of a row
  const int cpr = 3 * cpw;                // chunks per row
  const int half = d.Dh / 2;
  const int lane = threadIdx.x & 31;
  const int64_t rows = d.B * d.N;
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  for (int64_t row = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t q_ = row / d.inner, ii = row - q_ * d.inner;
    const int64_t o = q_ / d.N;
    const int n = (int)(q_ - o * d.N);
    const int64_t b = o * d.inner + ii;
    T* prow = qkv + row * (int64_t)cpr * 2 * P;
    const int64_t sbase = b * d.s_b + (int64_t)n * d.s_n;
    const float* crow = cosv + (int64_t)n * half;
    const float* srow = sinv + (int64_t)n * half;
#pragma unroll 2
    for (int c = lane; c < cpr; c += 32) {
      const int which = c / cpw, rem = c - which * cpw;
      const int h = rem / gph, grp = rem - h * gph;
      T* base = which == 0 ? q : (which == 1 ? k : v);
      T* split = base + sbase + (int64_t)h * d.s_h + grp * 2 * P;
      T* packed = prow + c * 2 * P;
      const Chunk<T, P> in = *reinterpret_cast<const Chunk<T, P>*>(BACKWARD ? split : packed);
      Chunk<T, P> out;
      if (which < 2 && rotate_qk) {
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const float cs = crow[grp * P + p];
          const float sn = BACKWARD ? -srow[grp * P + p] : srow[grp * P + p];
          const float e = Elem<T>::to_f(in.v[2 * p]), o = Elem<T>::to_f(in.v[2 * p + 1]);
          out.v[2 * p] = Elem<T>::from_f(e * cs - o * sn);
          out.v[2 * p + 1] = Elem<T>::from_f(o * cs + e * sn);
        }
      } else {
        out = in;
      }
      *reinterpret_cast<Chunk<T, P>*>(BACKWARD ? packed : split) = out;
    }
  }
}

template <typename T, bool BACKWARD>
int launch(void* qkv, const float* cosv, const float* sinv, QkvDims d, void* q, void* k, void* v, int rotate,
           cudaStream_t stream, const char* name) {
  const uintptr_t al = reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(q) |
                       reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v);
  constexpr int P = sizeof(T) == 2 ? 4 : 2;  // 16-byte chunks
  const bool vec = (d.Dh % (2 * P)) == 0 && (al % 16) == 0 && d.s_b % (2 * P) == 0 && d.s_h % (2 * P) == 0 &&
                   d.s_n % (2 * P) == 0;
  int64_t g = (d.B * d.N + kThreads / 32 - 1) / (kThreads / 32);
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  if (vec)
    qkv_rotary_kernel<T, P, BACKWARD><<<(int)g, kThreads, 0, stream>>>(
        static_cast<T*>(qkv), cosv, sinv, d, static_cast<T*>(q), static_cast<T*>(k), static_cast<T*>(v), rotate);
  else
    qkv_rotary_kernel<T, 1, BACKWARD><<<(int)g, kThreads, 0, stream>>>(
        static_cast<T*>(qkv), cosv, sinv, d, static_cast<T*>(q), static_cast<T*>(k), static_cast<T*>(v), rotate);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_qkv_rotary_split(const void* qkv, const float* cos, const float* sin, int64_t batch,
                                    int64_t seq_len, int64_t heads, int64_t dim_head, void* q, void* k, void* v,
                                    int rotate_qk, int dtype, int64_t seq_inner, void* stream) {
  clear_error();
  const char* name = "pmb_qkv_rotary_split";
  PMB_REQUIRE(batch >= 0 && seq_len >= 0 && heads > 0 && dim_head > 0 && dim_head % 2 == 0,
              "%s: bad shape (dim_head must be even)", name);
  if (batch * seq_len == 0) return PMB_OK;
  PMB_REQUIRE(qkv && q && k && v && (!rotate_qk || (cos && sin)), "%s: NULL tensor argument", name);
  PMB_REQUIRE(seq_inner > 0 && batch % seq_inner == 0, "%s: batch must be a multiple of seq_inner", name);
  QkvDims d{batch, seq_len, (int)heads, (int)dim_head, heads * seq_len * dim_head, seq_len * dim_head, dim_head,
            seq_inner};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH(dtype, T, name, [&] {
    return launch<T, false>(const_cast<void*>(qkv), cos, sin, d, q, k, v, rotate_qk, s, name);
  });
}

extern "C" int pmb_qkv_rotary_merge(const void* grad_q, const void* grad_k, const void* grad_v, const float* cos,
                                    const float* sin, int64_t batch, int64_t seq_len, int64_t heads,
                                    int64_t dim_head, void* grad_qkv, int rotate_qk, int dtype, int64_t stride_batch,
                                    int64_t stride_head, int64_t stride_seq, int64_t seq_inner, void* stream) {
  clear_error();
  const char* name = "pmb_qkv_rotary_merge";
  PMB_REQUIRE(batch >= 0 && seq_len >= 0 && heads > 0 && dim_head > 0 && dim_head % 2 == 0,
              "%s: bad shape (dim_head must be even)", name);
  if (batch * seq_len == 0) return PMB_OK;
  PMB_REQUIRE(grad_q && grad_k && grad_v && grad_qkv && (!rotate_qk || (cos && sin)), "%s: NULL tensor argument",
              name);
  PMB_REQUIRE(stride_batch >= 0 && stride_head >= 0 && stride_seq >= 0, "%s: bad strides", name);
  PMB_REQUIRE(seq_inner > 0 && batch % seq_inner == 0, "%s: batch must be a multiple of seq_inner", name);
  QkvDims d{batch, seq_len, (int)heads, (int)dim_head, stride_batch, stride_head, stride_seq, seq_inner};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH(dtype, T, name, [&] {
    return launch<T, true>(grad_qkv, cos, sin, d, const_cast<void*>(grad_q), const_cast<void*>(grad_k),
                           const_cast<void*>(grad_v), rotate_qk, s, name);
  });
}
