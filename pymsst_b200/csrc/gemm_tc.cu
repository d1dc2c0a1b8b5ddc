// Dense bf16/fp16 GEMM on tcgen05 (the grouped engine with one group), and
// the host-side tensor-map helpers shared by the tensor-core ops.
//
//   C[m, n] = sum_k A(m, k) B(n, k)  (+ bias[n])  (activation)
// A(m, k) = A[m*lda + k] (K-major) or A[k*lda + m] (MN-major); same for B.
// Replaces the reference's cuBLAS grouped-GEMM planner for the dense case
// (src/pymsst/training/cuda/fused_band_split.cu:2038-2281).
#include "dense_gemm.cuh"

namespace pmb {
// This unit's tcgen05 timeout flag (see umma.cuh).
unsigned int timeout_flag_gemm(int reset) { return umma::flag_reader(reset); }

namespace tma {

// The encoder is a driver call and needs a current context on the calling
// thread.  A thread that has not used the runtime yet (an autograd worker
// that reaches a backward op first, a thread of another language's FFI) has
// none, so bind the current device's primary context first.
static void bind_context() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) cudaGetLastError();
}

EncodeTiledFn encode_fn() {
  bind_context();
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_map_3d(CUtensorMap& map, const void* base, int dtype, uint64_t inner, uint64_t mid, uint64_t outer,
                uint64_t stride_mid_bytes, uint64_t stride_outer_bytes, uint32_t box_inner, uint32_t box_mid,
                uint32_t box_outer, const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error("%s: cuTensorMapEncodeTiled is unavailable (driver too old or no GPU)", name);
    return PMB_ERR_CUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (stride_mid_bytes & 15) != 0 || (stride_outer_bytes & 15) != 0) {
    set_error("%s: tensor-core operand needs a 16-byte aligned base and row strides (strides %llu, %llu bytes)",
              name, (unsigned long long)stride_mid_bytes, (unsigned long long)stride_outer_bytes);
    return PMB_ERR_ALIGNMENT;
  }
  const cuuint64_t dims[3] = {inner, mid, outer};
  const cuuint64_t strides[2] = {stride_mid_bytes, stride_outer_bytes};
  const cuuint32_t box[3] = {box_inner, box_mid, box_outer};
  const cuuint32_t elem[3] = {1, 1, 1};
  const CUtensorMapDataType t =
      dtype == PMB_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(&map, t, 3, const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d) dims (%llu, %llu, %llu)", name, (int)r,
              (unsigned long long)inner, (unsigned long long)mid, (unsigned long long)outer);
    return PMB_ERR_CUDA;
  }
  return PMB_OK;
}

int make_map_4d(CUtensorMap& map, const void* base, int dtype, const uint64_t (&dims)[4],
                const uint64_t (&stride_bytes)[3], const uint32_t (&box)[4], const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error("%s: cuTensorMapEncodeTiled is unavailable (driver too old or no GPU)", name);
    return PMB_ERR_CUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || ((stride_bytes[0] | stride_bytes[1] | stride_bytes[2]) & 15)) {
    set_error("%s: tensor-core operand needs a 16-byte aligned base and strides", name);
    return PMB_ERR_ALIGNMENT;
  }
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t st[3] = {stride_bytes[0], stride_bytes[1], stride_bytes[2]};
  const cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  const cuuint32_t elem[4] = {1, 1, 1, 1};
  const CUtensorMapDataType t =
      dtype == PMB_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(&map, t, 4, const_cast<void*>(base), d, st, bx, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d) for a 4-D map", name, (int)r);
    return PMB_ERR_CUDA;
  }
  return PMB_OK;
}

int make_store_map_2d(CUtensorMap& map, const void* base, int dtype, uint64_t cols, uint64_t rows, uint64_t ld_bytes,
                      const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error("%s: cuTensorMapEncodeTiled is unavailable (driver too old or no GPU)", name);
    return PMB_ERR_CUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld_bytes & 15) != 0) {
    set_error("%s: output store map needs a 16-byte aligned base and row pitch (pitch %llu bytes)", name,
              (unsigned long long)ld_bytes);
    return PMB_ERR_ALIGNMENT;
  }
  const cuuint64_t d[2] = {cols, rows};
  const cuuint64_t st[1] = {ld_bytes};
  const cuuint32_t bx[2] = {32, 32};
  const cuuint32_t elem[2] = {1, 1};
  const CUtensorMapDataType t =
      dtype == PMB_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(&map, t, 2, const_cast<void*>(base), d, st, bx, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d) for an output store map", name, (int)r);
    return PMB_ERR_CUDA;
  }
  return PMB_OK;
}

int make_map_rows_f32(CUtensorMap& map, const void* base, uint64_t cols, uint64_t rows, uint64_t pitch_bytes,
                      uint32_t box_cols, const char* name) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error("%s: cuTensorMapEncodeTiled is unavailable (driver too old or no GPU)", name);
    return PMB_ERR_CUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch_bytes & 15) != 0) {
    set_error("%s: fp32 row map needs a 16-byte aligned base and pitch", name);
    return PMB_ERR_ALIGNMENT;
  }
  const cuuint64_t d[2] = {cols, rows};
  const cuuint64_t st[1] = {pitch_bytes};
  const cuuint32_t bx[2] = {box_cols, 1};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), d, st, bx, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d) for an fp32 row map", name, (int)r);
    return PMB_ERR_CUDA;
  }
  return PMB_OK;
}

}  // namespace tma

}  // namespace pmb

using namespace pmb;

extern "C" int pmb_gemm_tc(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb, int b_mn_major,
                           void* c, int64_t ldc, int c_dtype, const void* bias, int bias_dtype, int activation,
                           int64_t m, int64_t n, int64_t k, int dtype, void* stream) {
  clear_error();
  const char* name = "pmb_gemm_tc";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: operands must be bf16 or fp16", name);
  PMB_REQUIRE(m >= 0 && n >= 0 && k > 0 && m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "%s: bad shape",
              name);
  PMB_REQUIRE(activation == PMB_ACT_NONE || activation == PMB_ACT_TANH, "%s: unknown activation", name);
  if (m == 0 || n == 0) return PMB_OK;
  PMB_REQUIRE(a && b && c, "%s: NULL tensor argument", name);
  return dense::gemm(a, lda, a_mn_major != 0, b, ldb, b_mn_major != 0, c, ldc, c_dtype, bias, bias_dtype, activation,
                     m, n, k, dtype, static_cast<cudaStream_t>(stream), name);
}

extern "C" int64_t pmb_gemm_tc_wgrad_workspace_size(int64_t m, int64_t n, int64_t k) {
  return dense::wgrad_workspace(m, n, k);
}

extern "C" int pmb_gemm_tc_wgrad(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                                 int64_t k, void* c, int64_t ldc, int c_dtype, int dtype, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_gemm_tc_wgrad";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: operands must be bf16 or fp16", name);
  PMB_REQUIRE(m >= 0 && n >= 0 && k >= 0 && m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "%s: bad shape",
              name);
  PMB_REQUIRE(dtype_size(c_dtype) > 0, "%s: unsupported output dtype %d", name, c_dtype);
  if (m == 0 || n == 0) return PMB_OK;
  PMB_REQUIRE(c && (k == 0 || (a && b)), "%s: NULL tensor argument", name);
  return dense::wgrad(a, lda, b, ldb, m, n, k, c, ldc, c_dtype, dtype, workspace, workspace_bytes,
                      static_cast<cudaStream_t>(stream), name);
}
