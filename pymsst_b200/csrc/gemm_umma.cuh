// Grouped bf16/fp16 GEMM on the 5th-generation tensor cores (tcgen05).
//
//   for each group g:  C_g[m, n] = sum_k A_g(m, k) * B_g(n, k)   (fp32 accumulate)
//
// A and B are read by TMA from 3-D tensor maps (inner, mid, outer) with
// 128-byte swizzle.  A K-major operand uses coordinates (k, mid, m) with a box
// {64, 1, rows}; an MN-major operand uses (m, mid, k) with boxes {64, 1, 64}
// per 64-wide MN chunk.  Groups carry offsets into the maps, so one launch
// covers all bands of a ragged / grouped layer.
//
// CTA = 128 threads.  Warp 0 lane 0 issues TMA into a STAGES-deep shared
// memory ring (full/empty mbarriers); warp 1 lane 0 issues tcgen05.mma
// (M = 128, N = BN, K = 16 per instruction) into a TMEM accumulator of BN
// fp32 columns and commits stage releases; after the last k-block all four
// warps drain the accumulator with tcgen05.ld (warp w owns rows 32w..32w+31,
// one row per thread) and run the epilogue functor.  All waits are bounded
// (umma.cuh); on a timeout the CTA skips the remaining work, frees its TMEM
// and exits, leaving the site in g_umma_timeout.
#pragma once

#include "umma.cuh"

namespace pmb {
namespace ugemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 128;
constexpr int kMaxGroups = PMB_MAX_BANDS;

struct Group {
  int m, n, k;             // problem size of this group
  int a_inner, a_mid, a_outer;  // offsets added to A's TMA coordinates
  int b_inner, b_mid, b_outer;  // offsets added to B's TMA coordinates
};

struct Plan {
  int num_groups;
  int total_tiles;
  int tile_start[kMaxGroups + 1];  // prefix sums of per-group tile counts
  Group g[kMaxGroups];
};

// Host: per-group tile counts for a given BN.
inline int build_plan(Plan& p, int bn) {
  p.total_tiles = 0;
  p.tile_start[0] = 0;
  for (int i = 0; i < p.num_groups; ++i) {
    const Group& g = p.g[i];
    const int t = (g.m <= 0 || g.n <= 0) ? 0 : ((g.m + BM - 1) / BM) * ((g.n + bn - 1) / bn);
    p.total_tiles += t;
    p.tile_start[i + 1] = p.total_tiles;
  }
  return p.total_tiles;
}

template <int BN, bool A_MN, bool B_MN>
struct Config {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t IDESC_BF16 = umma::idesc_f16(true, A_MN, B_MN, BM, BN);
  static constexpr uint32_t IDESC_F16 = umma::idesc_f16(false, A_MN, B_MN, BM, BN);
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
};

template <int BN, int STAGES>
constexpr int smem_bytes() {
  return STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 /*alignment slack*/ + 256 /*barriers*/;
}

// Per-thread view handed to epilogues: the accumulator row this thread owns.
struct TileCtx {
  int group;
  int m0, n0;       // tile origin within the group
  int row;          // m0 + thread's row
  bool row_valid;   // row < group m
  int n_valid;      // columns of this tile inside the group (<= BN)
  uint32_t taddr;   // TMEM address of this thread's row, column 0 of the tile
};

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(kThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ Plan plan, const __grid_constant__ Epi epi, int fp16) {
  using C = Config<BN, A_MN, B_MN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  __shared__ int abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // ---- locate this CTA's tile
  const int tile = blockIdx.x;
  int lo = 0, hi = plan.num_groups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (plan.tile_start[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  const int gi = lo;
  const Group& G = plan.g[gi];
  const int local = tile - plan.tile_start[gi];
  const int ntn = (G.n + BN - 1) / BN;
  const int m0 = (local / ntn) * BM;
  const int n0 = (local % ntn) * BN;
  const int kblocks = (G.k + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      umma::mbar_init(&full[s], 1);
      umma::mbar_init(&empty[s], 1);
    }
    umma::mbar_init(accum, 1);
    umma::fence_barrier_init();
    abort_flag = 0;
    umma::tma_prefetch(&tmA);
    umma::tma_prefetch(&tmB);
  }
  if (warp == 0) umma::tmem_alloc(tmem_slot, C::TMEM_COLS);
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % STAGES;
      const uint32_t round = kb / STAGES;
      if (!umma::mbar_wait(&empty[s], (round & 1) ^ 1, 1)) {
        atomicExch(&abort_flag, 1);
        break;
      }
      uint8_t* a_dst = smem + s * C::STAGE_BYTES;
      uint8_t* b_dst = a_dst + C::A_BYTES;
      umma::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
      const int k0 = kb * BK;
      if (!A_MN) {
        umma::tma_load_3d(a_dst, &tmA, &full[s], k0 + G.a_inner, G.a_mid, m0 + G.a_outer);
      } else {
#pragma unroll
        for (int c = 0; c < BM / 64; ++c)
          umma::tma_load_3d(a_dst + c * 64 * BK * 2, &tmA, &full[s], m0 + c * 64 + G.a_inner, G.a_mid,
                            k0 + G.a_outer);
      }
      if (!B_MN) {
        umma::tma_load_3d(b_dst, &tmB, &full[s], k0 + G.b_inner, G.b_mid, n0 + G.b_outer);
      } else {
#pragma unroll
        for (int c = 0; c < BN / 64; ++c)
          umma::tma_load_3d(b_dst + c * 64 * BK * 2, &tmB, &full[s], n0 + c * 64 + G.b_inner, G.b_mid,
                            k0 + G.b_outer);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    const uint32_t idesc = fp16 ? C::IDESC_F16 : C::IDESC_BF16;
    bool ok = true;
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % STAGES;
      const uint32_t round = kb / STAGES;
      if (!umma::mbar_wait(&full[s], round & 1, 2)) {
        atomicExch(&abort_flag, 1);
        ok = false;
        break;
      }
      umma::tc_fence_after();
      const uint32_t a_base = umma::smem_u32(smem + s * C::STAGE_BYTES);
      const uint32_t b_base = a_base + C::A_BYTES;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        uint64_t da, db;
        if (!A_MN)
          da = umma::smem_desc_sw128(a_base + kk * 32, 16, 1024);
        else
          da = umma::smem_desc_sw128(a_base + kk * 16 * 128, 64 * BK * 2, 1024);
        if (!B_MN)
          db = umma::smem_desc_sw128(b_base + kk * 32, 16, 1024);
        else
          db = umma::smem_desc_sw128(b_base + kk * 16 * 128, 64 * BK * 2, 1024);
        umma::mma_f16(tmem, da, db, idesc, (kb | kk) != 0 ? 1u : 0u);
      }
      umma::mma_commit(&empty[s]);
    }
    if (ok) umma::mma_commit(accum);
    else umma::mbar_arrive(accum);  // release the epilogue; results are discarded
  }
  __syncwarp();

  // ---------------- epilogue (all 4 warps)
  const bool done = umma::mbar_wait(accum, 0, 3);
  umma::tc_fence_after();
  if (!done) atomicExch(&abort_flag, 1);
  __syncthreads();
  if (!abort_flag && kblocks > 0) {
    TileCtx t;
    t.group = gi;
    t.m0 = m0;
    t.n0 = n0;
    t.row = m0 + warp * 32 + lane;
    t.row_valid = t.row < G.m;
    t.n_valid = min(BN, G.n - n0);
    t.taddr = tmem + ((uint32_t)(warp * 32) << 16);
    epi.template run<BN>(plan, t);
  }
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace ugemm
}  // namespace pmb
