// Dense bf16/fp16 GEMM on tcgen05 (the grouped engine with one group), and
// the host-side tensor-map helpers shared by the tensor-core ops.
//
//   C[m, n] = sum_k A(m, k) B(n, k)  (+ bias[n])  (activation)
// A(m, k) = A[m*lda + k] (K-major) or A[k*lda + m] (MN-major); same for B.
// Replaces the reference's cuBLAS grouped-GEMM planner for the dense case
// (src/pymsst/training/cuda/fused_band_split.cu:2038-2281).
#include "gemm_umma.cuh"
#include "tma.cuh"

namespace pmb {
// This unit's tcgen05 timeout flag (see umma.cuh).
unsigned int timeout_flag_gemm(int reset) { return umma::flag_reader(reset); }

namespace tma {

EncodeTiledFn encode_fn() {
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

}  // namespace tma

namespace {

__device__ __forceinline__ void store_dyn(void* p, int64_t i, int code, float v) {
  switch (code) {
    case PMB_FLOAT16:
      static_cast<__half*>(p)[i] = __float2half_rn(v);
      break;
    case PMB_BFLOAT16:
      static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
      break;
    default:
      static_cast<float*>(p)[i] = v;
  }
}

__device__ __forceinline__ float load_dyn(const void* p, int64_t i, int code) {
  switch (code) {
    case PMB_FLOAT16:
      return __half2float(static_cast<const __half*>(p)[i]);
    case PMB_BFLOAT16:
      return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default:
      return static_cast<const float*>(p)[i];
  }
}

struct DenseEpi {
  void* c;
  int64_t ldc;
  int c_dtype;
  const void* bias;
  int bias_dtype;
  int act;
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
      if (!t.row_valid) continue;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = c0 + j;
        if (n >= t.n_valid) break;
        float x = v[j];
        if (bias) x += load_dyn(bias, t.n0 + n, bias_dtype);
        if (act == PMB_ACT_TANH) x = tanhf(x);
        store_dyn(c, (int64_t)t.row * ldc + t.n0 + n, c_dtype, x);
      }
    }
  }
};

template <int BN, int STAGES, bool A_MN, bool B_MN>
int launch_dense(const CUtensorMap& ma, const CUtensorMap& mb, ugemm::Plan& plan, const DenseEpi& epi, int fp16,
                 cudaStream_t stream, const char* name) {
  const int tiles = ugemm::build_plan(plan, BN);
  if (tiles == 0) return PMB_OK;
  auto kern = ugemm::umma_gemm_kernel<BN, STAGES, A_MN, B_MN, DenseEpi>;
  const int smem = ugemm::smem_bytes<BN, STAGES>();
  PMB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), name);
  kern<<<tiles, ugemm::kThreads, smem, stream>>>(ma, mb, plan, epi, fp16);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

template <int BN, int STAGES>
int dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb, ugemm::Plan& plan,
                   const DenseEpi& epi, int fp16, cudaStream_t s, const char* name) {
  if (!a_mn && !b_mn) return launch_dense<BN, STAGES, false, false>(ma, mb, plan, epi, fp16, s, name);
  if (!a_mn && b_mn) return launch_dense<BN, STAGES, false, true>(ma, mb, plan, epi, fp16, s, name);
  if (a_mn && !b_mn) return launch_dense<BN, STAGES, true, false>(ma, mb, plan, epi, fp16, s, name);
  return launch_dense<BN, STAGES, true, true>(ma, mb, plan, epi, fp16, s, name);
}

}  // namespace
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
  const int bn = n >= 128 ? 128 : 64;
  CUtensorMap ma, mb;
  int st;
  if (!a_mn_major)
    st = tma::make_map_3d(ma, a, dtype, k, 1, m, lda * 2, lda * 2, 64, 1, ugemm::BM, name);
  else
    st = tma::make_map_3d(ma, a, dtype, m, 1, k, lda * 2, lda * 2, 64, 1, 64, name);
  if (st) return st;
  if (!b_mn_major)
    st = tma::make_map_3d(mb, b, dtype, k, 1, n, ldb * 2, ldb * 2, 64, 1, bn, name);
  else
    st = tma::make_map_3d(mb, b, dtype, n, 1, k, ldb * 2, ldb * 2, 64, 1, 64, name);
  if (st) return st;
  ugemm::Plan plan;
  plan.num_groups = 1;
  plan.g[0] = ugemm::Group{(int)m, (int)n, (int)k, 0, 0, 0, 0, 0, 0};
  DenseEpi epi{c, ldc, c_dtype, bias, bias_dtype, activation};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fp16 = dtype == PMB_FLOAT16;
  if (bn == 128) return dispatch_major<128, 4>(a_mn_major, b_mn_major, ma, mb, plan, epi, fp16, s, name);
  return dispatch_major<64, 6>(a_mn_major, b_mn_major, ma, mb, plan, epi, fp16, s, name);
}
