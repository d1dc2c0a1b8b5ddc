// Dense GEMMs on the tcgen05 engine (gemm_umma.cuh): tensor maps, tile-width
// choice, the plain epilogue (bias, tanh) and the split-K weight-gradient
// GEMM.  Included by each translation unit that runs dense tensor-core
// GEMMs; everything here has internal linkage.
#pragma once

#include "gemm_umma.cuh"
#include "tma.cuh"

namespace pmb {
namespace dense {
namespace {

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

// Bias values of a tile, loaded one tile ahead through the engine's prefetch hook (gemm_umma.cuh: `Pre`,
// `prefetch`): lane l of a warp holds bias[n0 + c0 + l] for each of the warp's 32-column chunks c0 = 32 * (sub +
// q * kSubs), q < kBiasChunks, so no chunk waits on a global load after its accumulator read.
constexpr int kBiasChunks = (256 / 32 + ugemm::kSubs - 1) / ugemm::kSubs;
struct BiasPre {
  float b[kBiasChunks];
};
template <class Load>
__device__ __forceinline__ void prefetch_bias(const ugemm::TileCtx& t, BiasPre& p, Load&& load) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < kBiasChunks; ++q) {
    const int c = 32 * (t.sub + q * ugemm::kSubs) + lane;  // column within the tile
    p.b[q] = c < t.n_valid ? load(t.n0 + c) : 0.f;
  }
}
// chunk q's value (q < kBiasChunks) without a dynamically indexed register array
__device__ __forceinline__ float bias_of(const BiasPre& p, int q) {
  static_assert(kBiasChunks == 3, "bias_of selects among three chunks");
  return q == 0 ? p.b[0] : (q == 1 ? p.b[1] : p.b[2]);
}

// C = act(acc + bias) in TC, row stride ldc.  With `slices` set, group g of
// the plan writes slice g (slice_elems apart): the split-K partials.  16-bit
// outputs with `use_tma` are written by TMA tile stores through `out_map`
// (tma::make_store_map_2d over C).
template <typename TC>
struct DenseEpi {
  // the resident-B schedule (dense::launch) measured 57.4 -> 51.2 us on [63984 x 192] x [192 x 1536]; epilogues
  // without this member keep the interleaved schedule (the rotary QKV epilogue measured 79.9 -> 88.1 us under it:
  // its rotating N blocks all landed on two thirds of the CTAs)
  // (16-bit outputs only: the fp32 variant spilled 4 bytes under the resident schedule)
  static constexpr bool kResidentB = sizeof(TC) == 2;
  TC* c;
  int64_t ldc;
  const void* bias;
  int bias_dtype;
  int act;
  int64_t slice_elems;
  int use_tma;
  CUtensorMap out_map;
  using Pre = BiasPre;
  __device__ void prefetch(const ugemm::Plan&, const ugemm::TileCtx& t, Pre& p) const {
    prefetch_bias(t, p, [&](int64_t col) { return bias ? load_dyn(bias, col, bias_dtype) : 0.f; });
  }
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t, const Pre& pre) const {
    TC* base = c + (int64_t)t.group * slice_elems + (int64_t)t.row0 * ldc + t.n0;
    int q = 0;
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BN; c0 += 32 * ugemm::kSubs, ++q) {
      if (c0 >= t.n_valid) break;
      const int ncols = min(32, t.n_valid - c0);
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
      if (bias) {
        const float bl = bias_of(pre, q);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += __shfl_sync(0xffffffffu, bl, j);
      }
      if (act == PMB_ACT_TANH) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = tanhf(v[j]);
      }
      if constexpr (sizeof(TC) == 2) {
        if (use_tma) {
          ugemm::warp_tma_store<TC>(t, v, &out_map, t.n0 + c0, t.row0);
          continue;
        }
      }
      ugemm::warp_store<TC>(t.stage, v, base + c0, ldc, t.rows_valid, ncols);
    }
  }
};

// A DenseEpi for a 16-bit C [m, n] (row stride ldc) that stores through TMA when C's base and pitch allow it.
template <typename TC>
inline DenseEpi<TC> dense_epi_tma(TC* c, int64_t ldc, int64_t m, int64_t n, const void* bias, int bias_dtype, int act,
                                  int c_dtype, const char* name) {
  DenseEpi<TC> e{c, ldc, bias, bias_dtype, act, 0, 0, {}};
  if (((reinterpret_cast<uintptr_t>(c) | (uintptr_t)(ldc * 2)) & 15) == 0 &&
      tma::make_store_map_2d(e.out_map, c, c_dtype, (uint64_t)n, (uint64_t)m, (uint64_t)ldc * 2, name) == PMB_OK)
    e.use_tma = 1;
  else
    clear_error();
  return e;
}

// N tile width for an N extent: 256 once N exceeds 128 (the A rows are then
// read once per 256 columns), else 128 / 64.
inline int pick_bn(int64_t n) { return n > 128 ? 256 : (n > 64 ? 128 : 64); }

template <int BN>
constexpr int stages_for() {
  return BN == 256 ? 3 : (BN == 128 ? 4 : 6);
}

// Tensor maps for A (rows m) and B (rows n) with K extent k.
inline int make_maps(CUtensorMap& ma, CUtensorMap& mb, const void* a, int64_t lda, bool a_mn, const void* b,
                     int64_t ldb, bool b_mn, int64_t m, int64_t n, int64_t k, int bn, int dtype, const char* name) {
  int st;
  if (!a_mn)
    st = tma::make_map_3d(ma, a, dtype, k, 1, m, lda * 2, lda * 2, 64, 1, ugemm::BM, name);
  else
    st = tma::make_map_3d(ma, a, dtype, m, 1, k, lda * 2, lda * 2, 64, 1, 64, name);
  if (st) return st;
  if (!b_mn)
    st = tma::make_map_3d(mb, b, dtype, k, 1, n, ldb * 2, ldb * 2, 64, 1, bn, name);
  else
    st = tma::make_map_3d(mb, b, dtype, n, 1, k, ldb * 2, ldb * 2, 64, 1, 64, name);
  return st;
}

// Resident-B variant (gemm_umma.cuh): 256-wide N blocks with K <= 192, the whole B block of a CTA (96 KB) kept
// in shared memory beside a 4-slot ring of A; operand traffic per tile drops from 144 KB to 48 KB at K = 192.
// Taken for epilogues that declare `static constexpr bool kResidentB = true`.
constexpr int kResKB = 3;
constexpr int kResStages = 4;

template <class E, class = void>
struct WantsResidentB : std::false_type {};
template <class E>
struct WantsResidentB<E, std::void_t<decltype(E::kResidentB)>> : std::bool_constant<E::kResidentB> {};

template <int BN, bool A_MN, bool B_MN, class Epi>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, ugemm::Plan& plan, const Epi& epi, int fp16,
           cudaStream_t stream, const char* name) {
  constexpr int STAGES = stages_for<BN>();
  const int tiles = ugemm::build_plan(plan, BN);
  if (tiles == 0) return PMB_OK;
  if constexpr (BN == 256 && WantsResidentB<Epi>::value) {
    // every N block needs a CTA of its own: more N blocks than CTAs keep the interleaved schedule
    const int ntn = (plan.g[0].n + BN - 1) / BN;
    if (plan.num_groups == 1 && plan.g[0].k <= kResKB * ugemm::BK && ntn <= ugemm::persistent_grid(tiles)) {
      auto kern = ugemm::umma_gemm_kernel<BN, kResStages, A_MN, B_MN, Epi, kResKB>;
      const int smem = ugemm::smem_bytes<BN, kResStages, kResKB>();
      PMB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), name);
      kern<<<ugemm::persistent_grid(tiles), ugemm::kThreads, smem, stream>>>(ma, mb, plan, epi, fp16);
      PMB_CHECK_LAUNCH(name);
      return PMB_OK;
    }
  }
  auto kern = ugemm::umma_gemm_kernel<BN, STAGES, A_MN, B_MN, Epi>;
  const int smem = ugemm::smem_bytes<BN, STAGES>();
  PMB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), name);
  kern<<<ugemm::persistent_grid(tiles), ugemm::kThreads, smem, stream>>>(ma, mb, plan, epi, fp16);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

template <int BN, class Epi>
int launch_major(bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb, ugemm::Plan& plan,
                 const Epi& epi, int fp16, cudaStream_t s, const char* name) {
  if (!a_mn && !b_mn) return launch<BN, false, false>(ma, mb, plan, epi, fp16, s, name);
  if (!a_mn && b_mn) return launch<BN, false, true>(ma, mb, plan, epi, fp16, s, name);
  if (a_mn && !b_mn) return launch<BN, true, false>(ma, mb, plan, epi, fp16, s, name);
  return launch<BN, true, true>(ma, mb, plan, epi, fp16, s, name);
}

template <class Epi>
int launch_any(int bn, bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb, ugemm::Plan& plan,
               const Epi& epi, int fp16, cudaStream_t s, const char* name) {
  if (bn == 256) return launch_major<256>(a_mn, b_mn, ma, mb, plan, epi, fp16, s, name);
  if (bn == 128) return launch_major<128>(a_mn, b_mn, ma, mb, plan, epi, fp16, s, name);
  return launch_major<64>(a_mn, b_mn, ma, mb, plan, epi, fp16, s, name);
}

// C[m, n] = act(sum_k A(m, k) B(n, k) + bias[n]) in c_dtype (see pmb_gemm_tc).
inline int gemm(const void* a, int64_t lda, bool a_mn, const void* b, int64_t ldb, bool b_mn, void* c, int64_t ldc,
                int c_dtype, const void* bias, int bias_dtype, int act, int64_t m, int64_t n, int64_t k, int dtype,
                cudaStream_t s, const char* name) {
  if (m == 0 || n == 0) return PMB_OK;
  const int bn = pick_bn(n);
  CUtensorMap ma, mb;
  int st = make_maps(ma, mb, a, lda, a_mn, b, ldb, b_mn, m, n, k, bn, dtype, name);
  if (st) return st;
  ugemm::Plan plan;
  plan.num_groups = 1;
  plan.g[0] = ugemm::Group{(int)m, (int)n, (int)k, 0, 0, 0, 0, 0, 0};
  const int fp16 = dtype == PMB_FLOAT16;
  switch (c_dtype) {
    case PMB_FLOAT32:
      return launch_any(bn, a_mn, b_mn, ma, mb, plan,
                        DenseEpi<float>{static_cast<float*>(c), ldc, bias, bias_dtype, act, 0}, fp16, s, name);
    case PMB_FLOAT16:
      return launch_any(bn, a_mn, b_mn, ma, mb, plan,
                        dense_epi_tma<__half>(static_cast<__half*>(c), ldc, m, n, bias, bias_dtype, act, c_dtype, name),
                        fp16, s, name);
    case PMB_BFLOAT16:
      return launch_any(bn, a_mn, b_mn, ma, mb, plan,
                        dense_epi_tma<__nv_bfloat16>(static_cast<__nv_bfloat16*>(c), ldc, m, n, bias, bias_dtype, act,
                                                     c_dtype, name),
                        fp16, s, name);
    default:
      set_error("%s: unsupported output dtype %d", name, c_dtype);
      return PMB_ERR_UNSUPPORTED_DTYPE;
  }
}

// ------------------------------------------------ split-K weight gradient
// C[m, n] = sum_k A[k, m] B[k, n]: both operands are row-major with K as the
// row index (an activation-gradient matrix and an activation matrix), so
// both are MN-major.  K (the batch rows) is long and M x N small, so K is
// split into S slices; slice s is group s of one launch and writes an fp32
// partial matrix, and a second kernel sums the S partials in slice order.
struct SplitK {
  int slices;
  int64_t slice_k;
};

// Enough slices for about two waves of tiles on a 148-SM part, each slice at
// least 512 rows of K (a multiple of the 64-row k-block), at most 128.
inline SplitK split_for(int64_t m, int64_t n, int64_t k) {
  const int bn = pick_bn(n);
  const int64_t tiles = ((m + ugemm::BM - 1) / ugemm::BM) * ((n + bn - 1) / bn);
  int64_t s = (296 + tiles - 1) / tiles;
  const int64_t by_k = (k + 511) / 512;
  if (s > by_k) s = by_k;
  if (s > 128) s = 128;
  if (s < 1) s = 1;
  int64_t sk = (k + s - 1) / s;
  sk = (sk + 63) / 64 * 64;
  return SplitK{(int)((k + sk - 1) / sk), sk};
}

inline int64_t wgrad_workspace(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const SplitK sp = split_for(m, n, k);
  return sp.slices > 1 ? ((int64_t)sp.slices * m * n * 4 + 255) / 256 * 256 : 0;
}

template <typename TC>
__global__ void __launch_bounds__(256)
    sum_slices(const float* __restrict__ ws, int slices, int64_t m, int64_t n, TC* __restrict__ c, int64_t ldc) {
  const int64_t total = m * n;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < total; i += (int64_t)gridDim.x * 256) {
    float s = 0.f;
    for (int k = 0; k < slices; ++k) s += ws[(int64_t)k * total + i];
    const int64_t r = i / n;
    c[r * ldc + (i - r * n)] = Elem<TC>::from_f(s);
  }
}

inline int wgrad(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n, int64_t k, void* c,
                 int64_t ldc, int c_dtype, int dtype, void* workspace, int64_t workspace_bytes, cudaStream_t s,
                 const char* name) {
  if (m == 0 || n == 0) return PMB_OK;
  const SplitK sp = split_for(m, n, k);
  if (k == 0 || sp.slices <= 1) {
    if (k == 0) {
      for (int64_t r = 0; r < m; ++r)
        PMB_CHECK_CUDA(cudaMemsetAsync(static_cast<char*>(c) + r * ldc * dtype_size(c_dtype), 0,
                                       n * dtype_size(c_dtype), s),
                       name);
      return PMB_OK;
    }
    return gemm(a, lda, true, b, ldb, true, c, ldc, c_dtype, nullptr, 0, PMB_ACT_NONE, m, n, k, dtype, s, name);
  }
  const int64_t need = wgrad_workspace(m, n, k);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  const int bn = pick_bn(n);
  CUtensorMap ma, mb;
  int st = make_maps(ma, mb, a, lda, true, b, ldb, true, m, n, k, bn, dtype, name);
  if (st) return st;
  ugemm::Plan plan;
  plan.num_groups = sp.slices;
  for (int i = 0; i < sp.slices; ++i) {
    const int64_t k0 = (int64_t)i * sp.slice_k;
    const int64_t kl = k - k0 < sp.slice_k ? k - k0 : sp.slice_k;
    plan.g[i] = ugemm::Group{(int)m, (int)n, (int)kl, 0, 0, (int)k0, 0, 0, (int)k0};
  }
  float* ws = static_cast<float*>(workspace);
  st = launch_any(bn, true, true, ma, mb, plan, DenseEpi<float>{ws, n, nullptr, 0, PMB_ACT_NONE, m * n},
                  dtype == PMB_FLOAT16, s, name);
  if (st) return st;
  int64_t blocks = (m * n + 255) / 256;
  if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
  return PMB_DISPATCH(c_dtype, TC, name, [&] {
    sum_slices<TC><<<(int)blocks, 256, 0, s>>>(ws, sp.slices, m, n, static_cast<TC*>(c), ldc);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

}  // namespace
}  // namespace dense
}  // namespace pmb
