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
// Persistent, warp-specialised CTA of 448 threads, one per SM; CTA i takes
// tiles i, i + grid, ... (tiles enumerated group by group, N fastest, so the
// CTAs in flight share their A rows through L2), or, with RES_KB > 0, only
// the tiles of one N block whose B stays in shared memory (resident_step):
//   warp 0 (one lane)   TMA producer into a STAGES-deep shared-memory ring
//                       (full / empty mbarriers, running across tiles);
//   warp 1 (one lane)   tcgen05.mma issuer (M = 128, N = BN, K = 16 per
//                       instruction) into one of two TMEM accumulators of BN
//                       fp32 columns; commits ring-slot releases and, after a
//                       tile's last k-block, the accumulator-full barrier;
//   warps 2..13         epilogue: drain the accumulator with tcgen05.ld (warp
//                       w reads TMEM lanes 32*(w%4).., one row per thread;
//                       the kSubs = 3 warps of a lane quarter take every
//                       third 32-column chunk), run the epilogue functor,
//                       release the accumulator.
// Two accumulators let the epilogue of tile i overlap the mainloop of tile
// i+1.  Epilogues write through a per-warp shared-memory staging block so
// global stores are 16-byte vectors along rows (warp_store below).
//
// All waits are bounded (umma.cuh); on a timeout the CTA stops issuing work,
// frees its TMEM and exits, leaving the site in g_umma_timeout.
#pragma once

#include <type_traits>

#include "umma.cuh"

namespace pmb {
namespace ugemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kSubs = 3;                 // epilogue warps per TMEM lane quarter
constexpr int kEpiWarps = 4 * kSubs;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxGroups = PMB_MAX_BANDS;
// Per-warp staging block: 32 rows x (32 fp32 + 16 bytes of padding) for the
// row-vector stores, or kStoreBufs 2 KB buffers for the TMA tile stores
// (a warp keeps up to kStoreBufs - 1 stores reading shared memory while it
// fills the next buffer).
constexpr int kStageRowBytes = 32 * 4 + 16;
constexpr int kStoreBufs = 2;  // measured: a third buffer changed no GEMM's time
constexpr int kStageWarpBytes = 32 * kStageRowBytes > kStoreBufs * 2048 ? 32 * kStageRowBytes : kStoreBufs * 2048;
static_assert(kStageWarpBytes % 512 == 0 && kStageWarpBytes >= kStoreBufs * 2048,
              "staging blocks hold kStoreBufs 512-byte-aligned 2 KB TMA store buffers");
constexpr int kMaxSmemBytes = 232448;  // per CTA on sm_100a

struct Group {
  int m, n, k;                  // problem size of this group
  int a_inner, a_mid, a_outer;  // offsets added to A's TMA coordinates
  int b_inner, b_mid, b_outer;  // offsets added to B's TMA coordinates
};

struct Plan {
  int num_groups;
  int total_tiles;
  int tile_start[kMaxGroups + 1];  // prefix sums of per-group tile counts
  Group g[kMaxGroups];
};

// Host: per-group tile counts for a given BN (groups with an empty M, N or K
// contribute no tiles; callers clear such outputs themselves).
inline int build_plan(Plan& p, int bn) {
  p.total_tiles = 0;
  p.tile_start[0] = 0;
  for (int i = 0; i < p.num_groups; ++i) {
    const Group& g = p.g[i];
    const int t = (g.m <= 0 || g.n <= 0 || g.k <= 0) ? 0 : ((g.m + BM - 1) / BM) * ((g.n + bn - 1) / bn);
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
  // two accumulators; tcgen05.alloc takes a power of two from 32 to 512 columns
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128
                                      : 2 * BN <= 256 ? 256 : 512;
  static_assert(2 * BN <= 512, "two accumulators must fit the 512 tensor-memory columns");
};

// RES_KB > 0: B resident in shared memory (RES_KB k-blocks of one N block), ring slots hold A only.
template <int BN, int STAGES, int RES_KB = 0>
constexpr int smem_bytes() {
  return STAGES * (BM * BK * 2 + (RES_KB > 0 ? 0 : BN * BK * 2)) + RES_KB * BN * BK * 2 +
         kEpiWarps * kStageWarpBytes + 1024 /*alignment slack*/ + 256 /*barriers*/;
}

// Resident-B schedule: CTA c serves N block c % ntn only (ntn = N blocks of the single group) and walks the M
// tiles of that block; its tiles are c, c + step, ... with step = (CTAs on that block) * ntn, so every tile of
// the plan is covered once.  Every role of the CTA computes the same step.
__device__ __forceinline__ int resident_step(const Plan& plan, int bn) {
  const int ntn = (plan.g[0].n + bn - 1) / bn;
  const int nb = (int)blockIdx.x % ntn;
  return ((int)gridDim.x - nb + ntn - 1) / ntn * ntn;
}

// Per-warp view handed to epilogues.  Each thread owns one accumulator row;
// the warp owns 32 consecutive rows starting at row0.
struct TileCtx {
  int group;
  int sub;         // this warp's share of the columns: 32-column chunks c with c % kSubs == sub
  int m0, n0;      // tile origin within the group
  int row0;        // first row of this warp
  int row;         // this thread's row (row0 + lane)
  bool row_valid;  // row < group m
  int rows_valid;  // rows of this warp inside the group (0..32)
  int n_valid;     // columns of this tile inside the group (<= BN)
  uint32_t taddr;  // TMEM address of this thread's row, column 0 of the tile
  uint8_t* stage;  // this warp's staging block (kStageWarpBytes)
  int* store_seq;  // this thread's count of TMA tile stores issued so far (picks the staging buffer)
};

// Epilogues with per-tile global operands (row scales, bias slices) may
// declare `struct Pre` and `prefetch(plan, ctx, Pre&)`: the epilogue warps
// then issue tile i+1's loads before they drain tile i, and run(plan, ctx,
// pre) receives values loaded an epilogue earlier, so the loads' latency is
// hidden behind the previous tile instead of sitting on every tile.
template <class E, class = void>
struct HasPre : std::false_type {};
template <class E>
struct HasPre<E, std::void_t<typename E::Pre>> : std::true_type {};
template <class E, bool = HasPre<E>::value>
struct PreOf {
  struct type {};
};
template <class E>
struct PreOf<E, true> {
  using type = typename E::Pre;
};

// Locate tile `tile` of the plan: group, M / N origin.
__device__ __forceinline__ void locate(const Plan& plan, int tile, int bn, int& gi, int& m0, int& n0) {
  int lo = 0, hi = plan.num_groups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (plan.tile_start[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  gi = lo;
  const Group& G = plan.g[gi];
  const int local = tile - plan.tile_start[gi];
  const int ntn = (G.n + bn - 1) / bn;
  m0 = (local / ntn) * BM;
  n0 = (local % ntn) * bn;
}

// ------------------------------------------------------- epilogue helpers
// Store a 32 x 32 block held one row per lane (v = this lane's 32 values):
// dst points at the block's (row 0, column 0), rows `ld` elements apart.
// The block is staged in shared memory and written back as 16-byte vectors
// along rows when dst, ld allow it, else element by element (coalesced
// along columns).  Whole warp; rows_valid / cols_valid clip the block.
template <typename T>
__device__ __forceinline__ void warp_store(uint8_t* stage, const float (&v)[32], T* dst, int64_t ld,
                                           int rows_valid, int cols_valid) {
  const int lane = threadIdx.x & 31;
  T* srow = reinterpret_cast<T*>(stage + lane * kStageRowBytes);
  {
    T pack[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) pack[j] = Elem<T>::from_f(v[j]);
#pragma unroll
    for (int q = 0; q < 32 * (int)sizeof(T) / 16; ++q)
      reinterpret_cast<uint4*>(srow)[q] = reinterpret_cast<const uint4*>(pack)[q];
  }
  __syncwarp();
  const bool vec = cols_valid == 32 &&
                   ((reinterpret_cast<uintptr_t>(dst) | (uintptr_t)(ld * (int64_t)sizeof(T))) & 15) == 0;
  if (vec) {
    constexpr int CPR = 32 * sizeof(T) / 16;  // 16-byte chunks per row
#pragma unroll
    for (int i = lane; i < 32 * CPR; i += 32) {
      const int r = i / CPR, q = i % CPR;
      if (r < rows_valid)
        reinterpret_cast<uint4*>(dst + (int64_t)r * ld)[q] =
            *reinterpret_cast<const uint4*>(stage + r * kStageRowBytes + q * 16);
    }
  } else {
#pragma unroll 4
    for (int r = 0; r < rows_valid; ++r)
      if (lane < cols_valid)
        dst[(int64_t)r * ld + lane] = reinterpret_cast<const T*>(stage + r * kStageRowBytes)[lane];
  }
  __syncwarp();
}

// Same, with an arbitrary destination per row: each lane passes the address
// of its own row's first column (nullptr = row skipped).
template <typename T>
__device__ __forceinline__ void warp_store_rows(uint8_t* stage, const float (&v)[32], T* my_row, int cols_valid) {
  const int lane = threadIdx.x & 31;
  T* srow = reinterpret_cast<T*>(stage + lane * kStageRowBytes);
  {
    T pack[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) pack[j] = Elem<T>::from_f(v[j]);
#pragma unroll
    for (int q = 0; q < 32 * (int)sizeof(T) / 16; ++q)
      reinterpret_cast<uint4*>(srow)[q] = reinterpret_cast<const uint4*>(pack)[q];
  }
  __syncwarp();
  const bool vec = __all_sync(0xffffffffu, (reinterpret_cast<uintptr_t>(my_row) & 15) == 0) && cols_valid == 32;
  const unsigned long long mine = reinterpret_cast<unsigned long long>(my_row);
  if (vec) {
    constexpr int CPR = 32 * sizeof(T) / 16;
#pragma unroll
    for (int i = lane; i < 32 * CPR; i += 32) {
      const int r = i / CPR, q = i % CPR;
      T* row = reinterpret_cast<T*>(__shfl_sync(0xffffffffu, mine, r));
      if (row != nullptr)
        reinterpret_cast<uint4*>(row)[q] = *reinterpret_cast<const uint4*>(stage + r * kStageRowBytes + q * 16);
    }
  } else {
#pragma unroll 4
    for (int r = 0; r < 32; ++r) {
      T* row = reinterpret_cast<T*>(__shfl_sync(0xffffffffu, mine, r));
      if (row != nullptr && lane < cols_valid) row[lane] = reinterpret_cast<const T*>(stage + r * kStageRowBytes)[lane];
    }
  }
  __syncwarp();
}

// Load a 32 x 32 block (same addressing as warp_store) and return this lane's
// row as floats; positions outside the clip read 0.
template <typename T>
__device__ __forceinline__ void warp_load(uint8_t* stage, const T* src, int64_t ld, int rows_valid, int cols_valid,
                                          float (&v)[32]) {
  const int lane = threadIdx.x & 31;
  const bool vec = cols_valid == 32 &&
                   ((reinterpret_cast<uintptr_t>(src) | (uintptr_t)(ld * (int64_t)sizeof(T))) & 15) == 0;
  if (vec) {
    constexpr int CPR = 32 * sizeof(T) / 16;
#pragma unroll
    for (int i = lane; i < 32 * CPR; i += 32) {
      const int r = i / CPR, q = i % CPR;
      uint4 u = make_uint4(0, 0, 0, 0);
      if (r < rows_valid) u = reinterpret_cast<const uint4*>(src + (int64_t)r * ld)[q];
      *reinterpret_cast<uint4*>(stage + r * kStageRowBytes + q * 16) = u;
    }
  } else {
#pragma unroll 4
    for (int r = 0; r < 32; ++r)
      reinterpret_cast<T*>(stage + r * kStageRowBytes)[lane] =
          (r < rows_valid && lane < cols_valid) ? src[(int64_t)r * ld + lane] : Elem<T>::from_f(0.f);
  }
  __syncwarp();
  const T* srow = reinterpret_cast<const T*>(stage + lane * kStageRowBytes);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = Elem<T>::to_f(srow[j]);
  __syncwarp();
}

// TMA tile stores (16-bit outputs).  The warp writes its 32 x 32 block into
// one of two 2 KB buffers at the start of its staging block (512-byte
// aligned) in the 64-byte-swizzled layout of the output's tensor map: row r
// at byte 64 r, its 16-byte chunk c at chunk position c ^ ((r >> 1) & 3), so
// the 32 lanes' row writes spread over all banks.  One lane then issues the
// bulk tensor store of the box at (col, row); the tensor map clips rows and
// columns past the output's extent.  Buffers alternate: before rewriting one,
// the lane waits until at most one earlier store is still reading shared
// memory.  This replaces the staged 16-byte global stores (shared-memory
// reads plus LSU stores per lane) with one asynchronous copy per block.
// Every output-store map is {32 columns, 32 rows}, 64-byte swizzle
// (tma::make_store_map_2d).  An epilogue that uses these stores does not use
// warp_store / warp_load (they share the staging block).
template <typename T>
__device__ __forceinline__ void warp_tma_store(const TileCtx& t, const float (&v)[32], const CUtensorMap* map,
                                               int col, int row) {
  static_assert(sizeof(T) == 2, "TMA tile stores take 16-bit outputs");
  const int lane = threadIdx.x & 31;
  const int buf = (*t.store_seq)++ % kStoreBufs;
  uint8_t* box = t.stage + buf * 2048;
  // the store that last used this buffer (kStoreBufs stores ago) has finished reading it
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kStoreBufs - 1) : "memory");
  __syncwarp();
  uint32_t pk[16];  // two values per conversion instruction
#pragma unroll
  for (int j = 0; j < 16; ++j) pk[j] = Elem<T>::pack2(v[2 * j], v[2 * j + 1]);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(box + lane * 64 + ((q ^ sw) << 4)) =
        make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(col), "r"(row), "r"(umma::smem_u32(box))
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
}

// ------------------------------------------------------------------ kernel
// RES_KB > 0 (single-group plans with K <= RES_KB * BK, the host checks): each CTA loads the B block of its N
// block once (resident_step schedule) and the ring streams only A, so a tile moves 128 x K instead of
// (128 + BN) x K operand bytes from L2; for K = 192, BN = 256 a third.
template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int RES_KB = 0>
__global__ void __launch_bounds__(kThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ Plan plan, const __grid_constant__ Epi epi, int fp16) {
  using C = Config<BN, A_MN, B_MN>;
  static_assert(smem_bytes<BN, STAGES, RES_KB>() <= kMaxSmemBytes, "stage ring + staging blocks exceed shared memory");
  constexpr int SLOT = RES_KB > 0 ? C::A_BYTES : C::STAGE_BYTES;  // bytes a ring slot carries
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bres_smem = smem + STAGES * SLOT;  // resident B: RES_KB k-blocks of C::B_BYTES
  uint8_t* staging = bres_smem + RES_KB * C::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + kEpiWarps * kStageWarpBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2] accumulator ready (MMA -> epilogue)
  uint64_t* tempty = tfull + 2;      // [2] accumulator drained (epilogue -> MMA)
  uint64_t* bres = tempty + 2;       // resident B loaded (producer -> MMA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres + 1);
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int step = gridDim.x;  // tile stride of this CTA
  if constexpr (RES_KB > 0) step = resident_step(plan, BN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      umma::mbar_init(&full[s], 1);
      umma::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      umma::mbar_init(&tfull[b], 1);
      umma::mbar_init(&tempty[b], kEpiWarps);
    }
    umma::mbar_init(bres, 1);
    umma::fence_barrier_init();
    abort_flag = 0;
    umma::tma_prefetch(&tmA);
    umma::tma_prefetch(&tmB);
  }
  if (warp == 1) umma::tmem_alloc(tmem_slot, C::TMEM_COLS);
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      // B block (k-block kb at b_dst) of the N block at n0
      auto load_b = [&](uint8_t* b_dst, uint64_t* bar, const Group& G, int k0, int n0) {
        if (!B_MN) {
          umma::tma_load_3d(b_dst, &tmB, bar, k0 + G.b_inner, G.b_mid, n0 + G.b_outer);
        } else {
#pragma unroll
          for (int c = 0; c < BN / 64; ++c)
            umma::tma_load_3d(b_dst + c * 64 * BK * 2, &tmB, bar, n0 + c * 64 + G.b_inner, G.b_mid,
                              k0 + G.b_outer);
        }
      };
      if constexpr (RES_KB > 0) {
        if ((int)blockIdx.x < plan.total_tiles) {
          int gi, m0, n0;
          locate(plan, blockIdx.x, BN, gi, m0, n0);
          const Group& G = plan.g[gi];
          const int kblocks = (G.k + BK - 1) / BK;  // <= RES_KB
          umma::mbar_arrive_expect_tx(bres, kblocks * C::B_BYTES);
          for (int kb = 0; kb < kblocks; ++kb) load_b(bres_smem + kb * C::B_BYTES, bres, G, kb * BK, n0);
        }
      }
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < plan.total_tiles && !abort_flag; tile += step) {
        int gi, m0, n0;
        locate(plan, tile, BN, gi, m0, n0);
        const Group& G = plan.g[gi];
        const int kblocks = (G.k + BK - 1) / BK;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (!umma::mbar_wait(&empty[s], (round & 1) ^ 1, 1)) {
            abort_flag = 1;
            break;
          }
          uint8_t* a_dst = smem + s * SLOT;
          umma::mbar_arrive_expect_tx(&full[s], SLOT);
          const int k0 = kb * BK;
          if (!A_MN) {
            umma::tma_load_3d(a_dst, &tmA, &full[s], k0 + G.a_inner, G.a_mid, m0 + G.a_outer);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              umma::tma_load_3d(a_dst + c * 64 * BK * 2, &tmA, &full[s], m0 + c * 64 + G.a_inner, G.a_mid,
                                k0 + G.a_outer);
          }
          if constexpr (RES_KB == 0) load_b(a_dst + C::A_BYTES, &full[s], G, k0, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc = fp16 ? C::IDESC_F16 : C::IDESC_BF16;
      if constexpr (RES_KB > 0) {
        if ((int)blockIdx.x < plan.total_tiles && !umma::mbar_wait(bres, 0, 5)) abort_flag = 1;
      }
      uint32_t it = 0, local = 0;
      for (int tile = blockIdx.x; tile < plan.total_tiles && !abort_flag; tile += step, ++local) {
        int gi, m0, n0;
        locate(plan, tile, BN, gi, m0, n0);
        const int kblocks = (plan.g[gi].k + BK - 1) / BK;
        const uint32_t buf = local & 1, use = local >> 1;
        if (!umma::mbar_wait(&tempty[buf], (use & 1) ^ 1, 4)) {
          abort_flag = 1;
          break;
        }
        umma::tc_fence_after();
        const uint32_t acc = tmem + buf * BN;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t round = it / STAGES;
          if (!umma::mbar_wait(&full[s], round & 1, 2)) {
            abort_flag = 1;
            ok = false;
            break;
          }
          umma::tc_fence_after();
          const uint32_t a_base = umma::smem_u32(smem + s * SLOT);
          const uint32_t b_base = RES_KB > 0 ? umma::smem_u32(bres_smem + kb * C::B_BYTES) : a_base + C::A_BYTES;
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
            umma::mma_f16(acc, da, db, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma::mma_commit(&empty[s]);
        }
        if (ok)
          umma::mma_commit(&tfull[buf]);
        else
          umma::mbar_arrive(&tfull[buf]);  // release the epilogue; it sees the abort flag
        if (!ok) break;
      }
    }
  } else {
    // ---------------- epilogue warps
    const int quarter = warp & 3;
    const int sub = (warp - 2) / 4;
    uint8_t* stage = staging + (warp - 2) * kStageWarpBytes;
    int store_seq = 0;
    uint32_t local = 0;
    auto ctx_of = [&](int tile, uint32_t buf) {
      int gi, m0, n0;
      locate(plan, tile, BN, gi, m0, n0);
      const Group& G = plan.g[gi];
      TileCtx t;
      t.group = gi;
      t.sub = sub;
      t.m0 = m0;
      t.n0 = n0;
      t.row0 = m0 + quarter * 32;
      t.row = t.row0 + lane;
      t.row_valid = t.row < G.m;
      t.rows_valid = max(0, min(32, G.m - t.row0));
      t.n_valid = min(BN, G.n - n0);
      t.taddr = tmem + buf * BN + ((uint32_t)(quarter * 32) << 16);
      t.stage = stage;
      t.store_seq = &store_seq;
      return t;
    };
    // this tile's prefetched operands and the next tile's (copied over at the end of each tile: no
    // dynamically indexed register arrays)
    typename PreOf<Epi>::type pre_cur, pre_next;
    if constexpr (HasPre<Epi>::value) {
      if ((int)blockIdx.x < plan.total_tiles) epi.prefetch(plan, ctx_of(blockIdx.x, 0), pre_cur);
    }
    for (int tile = blockIdx.x; tile < plan.total_tiles; tile += step, ++local) {
      if (abort_flag) break;
      const uint32_t buf = local & 1, use = local >> 1;
      if constexpr (HasPre<Epi>::value) {  // the next tile's loads, in flight while this one drains
        if (tile + step < plan.total_tiles) epi.prefetch(plan, ctx_of(tile + step, buf ^ 1), pre_next);
      }
      if (!umma::mbar_wait(&tfull[buf], use & 1, 3)) {
        abort_flag = 1;
        break;
      }
      umma::tc_fence_after();
      __syncwarp();
      if (!abort_flag) {
        const TileCtx t = ctx_of(tile, buf);
        if constexpr (HasPre<Epi>::value)
          epi.template run<BN>(plan, t, pre_cur);
        else
          epi.template run<BN>(plan, t);
      }
      if constexpr (HasPre<Epi>::value) pre_cur = pre_next;
      umma::tc_fence_before();
      __syncwarp();
      if (lane == 0) umma::mbar_arrive(&tempty[buf]);
    }
    // TMA tile stores still reading this warp's staging buffers must finish before the CTA releases them
    if (lane == 0 && store_seq > 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  __syncwarp();
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Host: persistent grid for a plan (one CTA per SM at most).
inline int persistent_grid(int tiles) {
  const int sms = num_sms();
  return tiles < sms ? tiles : sms;
}

}  // namespace ugemm
}  // namespace pmb
