// Interleaved-pair rotary embedding on [B, N, H, D] (standalone form of the
// op; the training path fuses the same rotation into the QKV projection
// epilogue).  Each thread rotates P consecutive pairs with vector loads.
// Reference semantics: src/pymsst/training/cuda/fused_band_split.cu:1077-1128.
#include "common.cuh"

namespace pmb {
namespace {

constexpr int kThreads = 256;

template <typename T, int P>
struct alignas((sizeof(T) * 2 * P) < 16 ? (sizeof(T) * 2 * P) : 16) PairPack {
  T v[2 * P];
};
template <typename T, int P>
struct alignas((sizeof(T) * P) < 16 ? (sizeof(T) * P) : 16) HalfPack {
  T v[P];
};

// inverse = 0: forward rotation; inverse = 1: transpose (backward).
template <typename T, int P>
__global__ void __launch_bounds__(kThreads)
    rotary_kernel(const T* __restrict__ t, const T* __restrict__ cosv, const T* __restrict__ sinv,
                  T* __restrict__ out, int64_t seq_len, int64_t heads, int64_t dim, int64_t total_groups,
                  int inverse) {
  const int64_t pairs = dim / 2;
  const int64_t groups_per_vec = pairs / P;  // pair groups per head vector
  for (int64_t gi = (int64_t)blockIdx.x * kThreads + threadIdx.x; gi < total_groups;
       gi += (int64_t)gridDim.x * kThreads) {
    const int64_t grp = gi % groups_per_vec;
    const int64_t vec = gi / groups_per_vec;  // (b, n, h) flattened
    const int64_t n = (vec / heads) % seq_len;
    const int64_t base = vec * dim + grp * 2 * P;
    const PairPack<T, P> x = *reinterpret_cast<const PairPack<T, P>*>(t + base);
    const HalfPack<T, P> c = *reinterpret_cast<const HalfPack<T, P>*>(cosv + n * pairs + grp * P);
    const HalfPack<T, P> s = *reinterpret_cast<const HalfPack<T, P>*>(sinv + n * pairs + grp * P);
    PairPack<T, P> y;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const float e = Elem<T>::to_f(x.v[2 * p]);
      const float o = Elem<T>::to_f(x.v[2 * p + 1]);
      const float cc = Elem<T>::to_f(c.v[p]);
      const float ss = inverse ? -Elem<T>::to_f(s.v[p]) : Elem<T>::to_f(s.v[p]);
      y.v[2 * p] = Elem<T>::from_f(e * cc - o * ss);
      y.v[2 * p + 1] = Elem<T>::from_f(o * cc + e * ss);
    }
    *reinterpret_cast<PairPack<T, P>*>(out + base) = y;
  }
}

template <typename T>
int launch_rotary(const void* t, const void* cosv, const void* sinv, void* out, int64_t batch, int64_t seq_len,
                  int64_t heads, int64_t dim, int inverse, cudaStream_t stream, const char* name) {
  const int64_t pairs = dim / 2;
  const uintptr_t align_t = reinterpret_cast<uintptr_t>(t) | reinterpret_cast<uintptr_t>(out);
  const uintptr_t align_cs = reinterpret_cast<uintptr_t>(cosv) | reinterpret_cast<uintptr_t>(sinv);
  // P pairs per thread: 4 for 16-bit (16 B of t), 2 for fp32 (16 B of t);
  // cos/sin are read as P-element (8 B) vectors.
  constexpr int P = sizeof(T) == 2 ? 4 : 2;
  const bool vec_ok = pairs % P == 0 && (align_t % 16) == 0 && (dim * (int64_t)sizeof(T)) % 16 == 0 &&
                      (align_cs % (sizeof(T) * P)) == 0;
  const int64_t vecs = batch * seq_len * heads;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (vec_ok) {
    const int64_t total = vecs * (pairs / P);
    int64_t grid = (total + kThreads - 1) / kThreads;
    if (grid > cap) grid = cap;
    rotary_kernel<T, P><<<(int)(grid < 1 ? 1 : grid), kThreads, 0, stream>>>(
        static_cast<const T*>(t), static_cast<const T*>(cosv), static_cast<const T*>(sinv), static_cast<T*>(out),
        seq_len, heads, dim, total, inverse);
  } else {
    const int64_t total = vecs * pairs;
    int64_t grid = (total + kThreads - 1) / kThreads;
    if (grid > cap) grid = cap;
    rotary_kernel<T, 1><<<(int)(grid < 1 ? 1 : grid), kThreads, 0, stream>>>(
        static_cast<const T*>(t), static_cast<const T*>(cosv), static_cast<const T*>(sinv), static_cast<T*>(out),
        seq_len, heads, dim, total, inverse);
  }
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

int rotary_entry(const void* t, const void* cosv, const void* sinv, void* out, int64_t batch, int64_t seq_len,
                 int64_t heads, int64_t dim, int dtype, void* stream, int inverse, const char* name) {
  clear_error();
  PMB_REQUIRE(batch >= 0 && seq_len >= 0 && heads >= 0 && dim > 0, "%s: bad shape", name);
  PMB_REQUIRE(dim % 2 == 0, "%s: last dimension %lld must be even", name, (long long)dim);
  if (batch * seq_len * heads == 0) return PMB_OK;
  PMB_REQUIRE(t && cosv && sinv && out, "%s: NULL tensor argument", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH(dtype, T, name, [&] {
    return launch_rotary<T>(t, cosv, sinv, out, batch, seq_len, heads, dim, inverse, s, name);
  });
}

}  // namespace
}  // namespace pmb

extern "C" int pmb_rotary_forward(const void* t, const void* cos, const void* sin, void* out, int64_t batch,
                                  int64_t seq_len, int64_t heads, int64_t dim, int dtype, void* stream) {
  return pmb::rotary_entry(t, cos, sin, out, batch, seq_len, heads, dim, dtype, stream, 0, "pmb_rotary_forward");
}

extern "C" int pmb_rotary_backward(const void* grad_out, const void* cos, const void* sin, void* grad_t,
                                   int64_t batch, int64_t seq_len, int64_t heads, int64_t dim, int dtype,
                                   void* stream) {
  return pmb::rotary_entry(grad_out, cos, sin, grad_t, batch, seq_len, heads, dim, dtype, stream, 1,
                           "pmb_rotary_backward");
}
