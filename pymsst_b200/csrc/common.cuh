// Shared helpers for the pymsst_b200 sm_100a kernels: dtype traits, the
// status/error channel of the C ABI, warp reductions and the per-band
// parameter table that every ragged (band-wise) kernel receives by value.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/pymsst_b200.h"

namespace pmb {

// ---------------------------------------------------------------------------
// Element types.  Every kernel computes in fp32 and converts at the edges.
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static constexpr int code = PMB_FLOAT32;
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};
template <>
struct Elem<__half> {
  static constexpr int code = PMB_FLOAT16;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
  // (a, b) rounded to nearest even in one instruction, a in the low half (memory order)
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int code = PMB_BFLOAT16;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  // (a, b) rounded to nearest even in one instruction, a in the low half (memory order)
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  return Elem<T>::to_f(*p);
}
template <typename T>
__device__ __forceinline__ void st_f(T* p, float v) {
  *p = Elem<T>::from_f(v);
}
// Round a value through T and back (models a tensor materialised in T).
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return Elem<T>::to_f(Elem<T>::from_f(v));
}

inline int dtype_size(int code) {
  switch (code) {
    case PMB_FLOAT32:
      return 4;
    case PMB_FLOAT16:
    case PMB_BFLOAT16:
      return 2;
    default:
      return 0;
  }
}

// ---------------------------------------------------------------------------
// Error channel: every C entry point returns a status and leaves a message
// that pmb_last_error() reports for the calling host thread.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();
// Counts kernel launches made by this library (read by pmb_launch_count()).
void count_launch();

#define PMB_REQUIRE(cond, ...)                  \
  do {                                          \
    if (!(cond)) {                              \
      ::pmb::set_error(__VA_ARGS__);            \
      return PMB_ERR_INVALID_ARGUMENT;          \
    }                                           \
  } while (0)

// Every kernel launch in the library is followed by exactly one of these.
#define PMB_CHECK_LAUNCH(name)                                                        \
  do {                                                                                \
    ::pmb::count_launch();                                                            \
    cudaError_t err__ = cudaGetLastError();                                           \
    if (err__ != cudaSuccess) {                                                       \
      ::pmb::set_error("%s: kernel launch failed: %s", name, cudaGetErrorString(err__)); \
      return PMB_ERR_CUDA;                                                            \
    }                                                                                 \
  } while (0)

#define PMB_CHECK_CUDA(expr, name)                                                 \
  do {                                                                             \
    cudaError_t err__ = (expr);                                                    \
    if (err__ != cudaSuccess) {                                                    \
      ::pmb::set_error("%s: %s failed: %s", name, #expr, cudaGetErrorString(err__)); \
      return PMB_ERR_CUDA;                                                         \
    }                                                                              \
  } while (0)

// Dispatch a dtype code to a C++ type; unsupported codes are reported.
#define PMB_DISPATCH(code, T, name, ...)                               \
  [&]() -> int {                                                       \
    switch (code) {                                                    \
      case PMB_FLOAT32: {                                              \
        using T = float;                                               \
        return __VA_ARGS__();                                          \
      }                                                                \
      case PMB_FLOAT16: {                                              \
        using T = __half;                                              \
        return __VA_ARGS__();                                          \
      }                                                                \
      case PMB_BFLOAT16: {                                             \
        using T = __nv_bfloat16;                                       \
        return __VA_ARGS__();                                          \
      }                                                                \
      default:                                                         \
        ::pmb::set_error("%s: unsupported dtype code %d", name, code); \
        return PMB_ERR_UNSUPPORTED_DTYPE;                              \
    }                                                                  \
  }()

// Dispatch (activation dtype, parameter dtype): parameters either share the
// activation dtype or are fp32 (master weights used directly under mixed
// precision).
#define PMB_DISPATCH_PARAM(code, pcode, T, TP, name, ...)                                     \
  [&]() -> int {                                                                              \
    if ((pcode) != (code) && (pcode) != PMB_FLOAT32) {                                        \
      ::pmb::set_error("%s: parameter dtype %d must equal the activation dtype or be fp32", \
                       name, pcode);                                                          \
      return PMB_ERR_UNSUPPORTED_DTYPE;                                                       \
    }                                                                                         \
    return PMB_DISPATCH(code, T, name, [&] {                                                  \
      if ((pcode) == PMB_FLOAT32) {                                                           \
        using TP = float;                                                                     \
        return __VA_ARGS__();                                                                 \
      }                                                                                       \
      using TP = T;                                                                           \
      return __VA_ARGS__();                                                                   \
    });                                                                                       \
  }()

// ---------------------------------------------------------------------------
// Reductions.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// Per-band parameter table, passed by value as a kernel argument (no device
// side pointer tables, no per-call host->device uploads).  `off` holds the
// prefix sums of the band widths; `ptr0..ptr2` are per-band device pointers
// whose meaning depends on the kernel (gamma / weight / bias ...).
// ---------------------------------------------------------------------------
constexpr int kMaxBands = PMB_MAX_BANDS;

struct BandTable {
  int count;
  int max_width;
  int64_t total;
  int64_t off[kMaxBands + 1];
  const void* ptr0[kMaxBands];
  const void* ptr1[kMaxBands];
  const void* ptr2[kMaxBands];
};

// Fill a BandTable from host-side widths; returns 0 or an error status.
int make_band_table(BandTable& t, int count, const int64_t* widths, const void* const* p0,
                    const void* const* p1, const void* const* p2, const char* name);

__device__ __forceinline__ int band_of(const BandTable& t, int64_t col) {
  // Binary search over the prefix sums: largest b with off[b] <= col.
  int lo = 0, hi = t.count - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (t.off[mid] <= col)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

inline int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

}  // namespace pmb
