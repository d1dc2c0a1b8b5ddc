// Scaled-dot-product attention core of the axial transformers (head dim 64,
// no mask, no dropout), forward and backward on the tcgen05 tensor cores,
// bf16 / fp16 in, fp32 accumulation and softmax.
//
//   S = Q K^T * scale,  P = softmax_rows(S),  O = P V,  lse = log(sum exp S)
//   backward:  D = rowsum(dO * O),  dP = dO V^T,  dS = P * (dP - D),
//              dV = P^T dO,  dQ = scale * dS K,  dK = scale * dS^T Q
//
// Sequences of up to 128 positions (the band axis) take two single-tile
// kernels, described at "forward, short sequences" / "backward, short
// sequences" below: every key of an item fits one 128 x 128 S tile (two
// sequences per item when N <= 64), the backward is one pass for dQ, dK and
// dV.  Longer sequences take three persistent, warp-specialised kernels with
// the same shape: a work item is 128 rows (queries, or keys for dK/dV) of one
// (sequence, head); two CTAs per SM take items blockIdx.x, + gridDim.x, ...:
//   warp 0   TMA producers: lane 0 loads the item's 128-row tiles, lane 1
//            streams the chunks of the other operand through a ring (4-D
//            plane maps: rows >= N read as zeros) -- 64-row chunks in the
//            forward, 32-row chunks in the backward;
//   warp 1   lane 0 issues tcgen05.mma (M 128, K 16 per instruction, fp32
//            accumulators in tensor memory);
//   row warps  the TMEM lane of a thread is its row: softmax / gradient
//            arithmetic on the accumulators, the 16-bit P / dS operand rows
//            written to shared memory in the 128-byte-swizzled K-major
//            layout the MMA reads, and the item's output rows.  The forward
//            has 4 row warps (one thread per row); the backward 8 (two
//            threads per row, half the columns each).
// Each accumulator product uses the staged tiles as they arrive: a K/V, Q or
// dO tile serves as a K-major operand in one product and as an MN-major
// operand (N = head dim) in the other.  Chunks are counted across items, so
// barrier phases run on; every wait is bounded (on a timeout the roles stop,
// tensor memory is freed and the site is left in the attention timeout
// flag).  No atomics: each output row is written by one thread, so results
// are deterministic.  P and dS are rounded to the input type before their
// products, as torch's fused attention kernels do.
//
// Layout: q, k, v, o and their gradients are [sequences, N, H, 64] planes
// with any sequence / position / head element strides (multiples of 8, the
// 64 head elements contiguous); lse and D are fp32 [sequences * H, ld] with
// ld = N rounded up to a multiple of 4 (16-byte rows for TMA).
// Reference semantics: torch.nn.functional.scaled_dot_product_attention with
// the default scale 1/sqrt(64), as called by the BS-/Mel-RoFormer Attention
// module of pymss-core (the attention backend the reference selects with
// cuda_attention_backend, src/pymsst/training/module.py:96-107).
#include "tma.cuh"
#include "umma.cuh"

namespace pmb {
unsigned int timeout_flag_attn(int reset) { return umma::flag_reader(reset); }

namespace {

constexpr int kD = 64;          // head dim
constexpr int BM = 128;         // rows per work item
constexpr int BN = 64;          // rows per streamed chunk
constexpr int kThreads = 192;   // TMA warp, MMA warp, 4 row warps
constexpr int TILE128 = BM * kD * 2;  // 16 KB: 128 rows x 64 16-bit
constexpr int TILE64 = BN * kD * 2;   // 8 KB
constexpr uint32_t kTmemCols = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct Plane {
  int64_t s_b, s_n, s_h;  // element strides of a [sequences, N, H, 64] plane
};

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Byte offset of 16-byte chunk ch (elements 8ch..8ch+7) of row r in a
// 128-byte-swizzled K-major tile of 64-element rows.
__device__ __forceinline__ uint32_t sw128(int r, int ch) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((ch ^ (r & 7)) << 4));
}

// 32 fp32 values -> chunks [c0, c0 + 4) of row r of a 16-bit SW128 tile
template <typename T>
__device__ __forceinline__ void put_row32(uint8_t* tile, int r, int c0, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<uint4*>(tile + sw128(r, c0 + i)) =
        make_uint4(pack2<T>(v[8 * i], v[8 * i + 1]), pack2<T>(v[8 * i + 2], v[8 * i + 3]),
                   pack2<T>(v[8 * i + 4], v[8 * i + 5]), pack2<T>(v[8 * i + 6], v[8 * i + 7]));
}

// 64 fp32 values (times mul) -> one 128-byte row of a global plane
template <typename T>
__device__ __forceinline__ void store_row64(T* dst, const float (&a)[32], const float (&b)[32], float mul) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<uint4*>(dst + 8 * i) =
        make_uint4(pack2<T>(a[8 * i] * mul, a[8 * i + 1] * mul), pack2<T>(a[8 * i + 2] * mul, a[8 * i + 3] * mul),
                   pack2<T>(a[8 * i + 4] * mul, a[8 * i + 5] * mul), pack2<T>(a[8 * i + 6] * mul, a[8 * i + 7] * mul));
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<uint4*>(dst + 32 + 8 * i) =
        make_uint4(pack2<T>(b[8 * i] * mul, b[8 * i + 1] * mul), pack2<T>(b[8 * i + 2] * mul, b[8 * i + 3] * mul),
                   pack2<T>(b[8 * i + 4] * mul, b[8 * i + 5] * mul), pack2<T>(b[8 * i + 6] * mul, b[8 * i + 7] * mul));
}

// D[tmem] (+)= A * B^T over K = 64: A a 128-row K-major SW128 tile; B either
// a K-major tile (its rows are the N index) or an MN-major one (64 rows of K,
// the 64 head elements are the N index).
__device__ __forceinline__ void mma_k64(uint32_t d, uint32_t a_base, uint32_t b_base, bool b_mn, uint32_t idesc,
                                        bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint64_t a = umma::smem_desc_sw128(a_base + kk * 32, 16, 1024);
    const uint64_t b = b_mn ? umma::smem_desc_sw128(b_base + kk * 16 * 128, BN * 128, 1024)
                            : umma::smem_desc_sw128(b_base + kk * 32, 16, 1024);
    umma::mma_f16(d, a, b, idesc, (accumulate || kk) ? 1u : 0u);
  }
}

template <typename T>
struct Idesc {
  static constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  static constexpr uint32_t K = umma::idesc_f16(kBf16, false, false, BM, BN);  // B K-major, N = 64 rows
  static constexpr uint32_t MN = umma::idesc_f16(kBf16, false, true, BM, kD);  // B MN-major, N = head dim
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Arrive once per row warp on `bar` after this thread's shared / tensor
// memory accesses (count 4 barriers).
__device__ __forceinline__ void warp_arrive(uint64_t* bar, bool wrote_smem) {
  if (wrote_smem) umma::fence_proxy_async_smem();
  umma::tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) umma::mbar_arrive(bar);
}

struct Item {
  int bh, blk, b, h;
};

__device__ __forceinline__ Item item_at(int item, int nblk, int H) {
  Item it;
  it.bh = item / nblk;
  it.blk = item - it.bh * nblk;
  it.b = it.bh / H;
  it.h = it.bh - it.b * H;
  return it;
}

// ---------------------------------------------------------------- forward
// Item = 128 queries.  Lane 0 of warp 0 loads Q, lane 1 streams K/V chunks;
// the MMA lane issues S_c = Q K_c^T into TMEM S[c % 2] and, one chunk
// behind, O_c = P_c V_c into TMEM O[c % 2]; the row threads read S_c, keep
// the running max / sum, write P_c and fold O_{c-1} into their fp32 row
// accumulators (rescaled by the change of the max), then write O and lse.
namespace fw {
constexpr int kStages = 3;
constexpr int OFF_KV = TILE128;                        // kStages x (K, V)
constexpr int OFF_P = OFF_KV + kStages * 2 * TILE64;   // 2 x P
constexpr int OFF_BAR = OFF_P + 2 * BM * BN * 2;
constexpr int kBars = 2 + 2 * kStages + 8;
constexpr int SMEM = OFF_BAR + kBars * 8 + 16 + 1024;
constexpr uint32_t kTmemO = 128;
}  // namespace fw

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, T* __restrict__ o, float* __restrict__ lse, Plane po, int N,
                int H, int ldl, int nblk, int total, float scale) {
  using namespace fw;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* o_empty = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBars);
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (N + BN - 1) / BN;
  if (threadIdx.x == 0) {
    umma::mbar_init(q_full, 1);
    umma::mbar_init(q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      umma::mbar_init(&kv_full[s], 1);
      umma::mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      umma::mbar_init(&s_full[b], 1);
      umma::mbar_init(&p_full[b], 4);
      umma::mbar_init(&o_full[b], 1);
      umma::mbar_init(&o_empty[b], 4);
    }
    abort_flag = 0;
    umma::fence_barrier_init();
  }
  if (warp == 0) umma::tmem_alloc(tmem_slot, kTmemCols);
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // Q tiles
      umma::tma_prefetch(&tmQ);
      uint32_t t = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
        const Item it = item_at(item, nblk, H);
        if (!umma::mbar_wait(q_empty, (t & 1) ^ 1, 0x41)) {
          abort_flag = 1;
          break;
        }
        umma::mbar_arrive_expect_tx(q_full, TILE128);
        umma::tma_load_4d(smem, &tmQ, q_full, 0, it.h, it.blk * BM, it.b);
      }
    } else if (lane == 1) {  // K/V chunks
      umma::tma_prefetch(&tmK);
      umma::tma_prefetch(&tmV);
      uint32_t cc = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x) {
        const Item it = item_at(item, nblk, H);
        for (int j = 0; j < nch; ++j, ++cc) {
          const int s = cc % kStages;
          if (!umma::mbar_wait(&kv_empty[s], ((cc / kStages) & 1) ^ 1, 0x42)) {
            abort_flag = 1;
            break;
          }
          uint8_t* dst = smem + OFF_KV + s * 2 * TILE64;
          umma::mbar_arrive_expect_tx(&kv_full[s], 2 * TILE64);
          umma::tma_load_4d(dst, &tmK, &kv_full[s], 0, it.h, j * BN, it.b);
          umma::tma_load_4d(dst + TILE64, &tmV, &kv_full[s], 0, it.h, j * BN, it.b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // O_c = P_c V_c, issued one chunk behind S so that S_{c+1} runs during softmax c
      auto issue_o = [&](uint32_t c) -> bool {
        const int pb = c & 1;
        if (!umma::mbar_wait(&p_full[pb], (c >> 1) & 1, 0x44)) return false;
        if (!umma::mbar_wait(&o_empty[pb], ((c >> 1) & 1) ^ 1, 0x45)) return false;
        umma::tc_fence_after();
        mma_k64(tmem + kTmemO + pb * kD, umma::smem_u32(smem + OFF_P + pb * BM * BN * 2),
                umma::smem_u32(smem + OFF_KV + (c % kStages) * 2 * TILE64 + TILE64), true, Idesc<T>::MN, false);
        umma::mma_commit(&o_full[pb]);
        umma::mma_commit(&kv_empty[c % kStages]);
        return true;
      };
      uint32_t cc = 0, t = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok && !abort_flag; item += gridDim.x, ++t) {
        if (!umma::mbar_wait(q_full, t & 1, 0x43)) {
          ok = false;
          break;
        }
        umma::tc_fence_after();
        for (int j = 0; j < nch; ++j, ++cc) {
          const int s = cc % kStages;
          if (!umma::mbar_wait(&kv_full[s], (cc / kStages) & 1, 0x46)) {
            ok = false;
            break;
          }
          umma::tc_fence_after();
          mma_k64(tmem + (cc & 1) * BN, umma::smem_u32(smem), umma::smem_u32(smem + OFF_KV + s * 2 * TILE64), false,
                  Idesc<T>::K, false);
          umma::mma_commit(&s_full[cc & 1]);
          if (j == nch - 1) umma::mma_commit(q_empty);
          if (cc > 0 && !issue_o(cc - 1)) {
            ok = false;
            break;
          }
        }
      }
      if (ok && cc > 0) ok = issue_o(cc - 1);
      if (!ok) abort_flag = 1;
    }
  } else {
    const int quarter = warp & 3, row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    uint32_t cc = 0;
    for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x) {
      const Item it = item_at(item, nblk, H);
      float m = -INFINITY, l = 0.f, corr_prev = 0.f;
      float acc[kD];
#pragma unroll
      for (int c = 0; c < kD; ++c) acc[c] = 0.f;
      bool ok = true;
      // acc = acc * corr + O_c; release the O buffer
      auto fold_o = [&](uint32_t c, float corr) -> bool {
        const int ob = c & 1;
        if (!umma::mbar_wait(&o_full[ob], (c >> 1) & 1, 0x48)) return false;
        umma::tc_fence_after();
        float v0[32], v1[32];
        umma::tmem_ld32(tmem + lane_off + kTmemO + ob * kD, v0);
        umma::tmem_ld32(tmem + lane_off + kTmemO + ob * kD + 32, v1);
        warp_arrive(&o_empty[ob], false);
#pragma unroll
        for (int c2 = 0; c2 < 32; ++c2) {
          acc[c2] = fmaf(acc[c2], corr, v0[c2]);
          acc[32 + c2] = fmaf(acc[32 + c2], corr, v1[c2]);
        }
        return true;
      };
      for (int j = 0; j < nch; ++j, ++cc) {
        const int sb = cc & 1;
        if (!umma::mbar_wait(&s_full[sb], (cc >> 1) & 1, 0x47)) {
          ok = false;
          break;
        }
        umma::tc_fence_after();
        float s0[32], s1[32];
        umma::tmem_ld32(tmem + lane_off + sb * BN, s0);
        umma::tmem_ld32(tmem + lane_off + sb * BN + 32, s1);
        const int kc = j * BN;
        if (kc + BN > N) {  // keys past the end of the sequence
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            if (kc + c >= N) s0[c] = -INFINITY;
            if (kc + 32 + c >= N) s1[c] = -INFINITY;
          }
        }
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
#pragma unroll
          for (int e = 0; e < 4; ++e) mx4[e] = fmaxf(mx4[e], fmaxf(s0[c + e], s1[c + e]));
        }
        // the scale is positive, so the max of the raw scores gives the max of the scaled ones
        const float mn = fmaxf(m, fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2);  // finite
        const float corr = exp2f(m - mn);
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          s0[c] = exp2f(fmaf(s0[c], sl2, -mn));
          s1[c] = exp2f(fmaf(s1[c], sl2, -mn));
          sum4[c & 3] += s0[c] + s1[c];
        }
        l = fmaf(l, corr, (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
        m = mn;
        uint8_t* ptile = smem + OFF_P + sb * BM * BN * 2;
        put_row32<T>(ptile, row, 0, s0);
        put_row32<T>(ptile, row, 4, s1);
        warp_arrive(&p_full[sb], true);
        if (j > 0 && !fold_o(cc - 1, corr_prev)) {
          ok = false;
          break;
        }
        corr_prev = corr;
      }
      if (ok) ok = fold_o(cc - 1, corr_prev);
      if (!ok) {
        abort_flag = 1;
        break;
      }
      const int r = it.blk * BM + row;
      if (r < N) {
        float a0[32], a1[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          a0[c] = acc[c];
          a1[c] = acc[32 + c];
        }
        store_row64<T>(o + it.b * po.s_b + it.h * po.s_h + (int64_t)r * po.s_n, a0, a1, 1.f / l);
        lse[(int64_t)it.bh * ldl + r] = (m + log2f(l)) * kLn2;
      }
    }
  }
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- backward
// Both backward kernels run 8 row warps: warp w (2..9) reads TMEM lane
// quarter w % 4 and owns columns [32 h, 32 h + 32) of its row, h = (w-2)/4,
// so two threads share each row and every thread's chain is half as long.
constexpr int kRowWarpsBwd = 8;
constexpr int kBwdThreads = 64 + 32 * kRowWarpsBwd;

// 32 columns of this warp's TMEM lane quarter, without waiting: the values
// are valid after tmem_wait(), which also orders their uses after the wait.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Register dependency on all 32 values (an empty statement the compiler
// cannot move the values' uses ahead of).
__device__ __forceinline__ void tie32(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// Wait for this thread's outstanding tcgen05.ld and tie both arrays after it.
__device__ __forceinline__ void tmem_wait2(uint32_t (&a)[32], uint32_t (&b)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  tie32(a);
  tie32(b);
}

// 32 fp32 values (times mul) -> 64 bytes of a global row
template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const uint32_t (&a)[32], float mul) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float* f = reinterpret_cast<const float*>(a) + 8 * i;
    *reinterpret_cast<uint4*>(dst + 8 * i) =
        make_uint4(pack2<T>(f[0] * mul, f[1] * mul), pack2<T>(f[2] * mul, f[3] * mul),
                   pack2<T>(f[4] * mul, f[5] * mul), pack2<T>(f[6] * mul, f[7] * mul));
  }
}

// Head gate sigma(logit) of one (row, head), from the 16-bit logit the gate projection produced.
template <typename T>
__device__ __forceinline__ float gate_of(T logit) {
  return 1.0f / (1.0f + __expf(-Elem<T>::to_f(logit)));
}

// Inverse rotary rotation of a thread's 32 gradient values of position pos
// (interleaved pairs 16 half .. 16 half + 15 of the head): (e, o) ->
// (e c + o s, o c - e s), the transpose of the forward's (e c - o s,
// o c + e s); angles from fp32 tables [N, 32].  The gradient then leaves the
// kernel in the projection's own (unrotated) space.
__device__ __forceinline__ void unrotate32(uint32_t (&a)[32], const float* __restrict__ rc,
                                           const float* __restrict__ rs, int pos, int half) {
  const float4* c4 = reinterpret_cast<const float4*>(rc + (int64_t)pos * 32 + half * 16);
  const float4* s4 = reinterpret_cast<const float4*>(rs + (int64_t)pos * 32 + half * 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 c = __ldg(c4 + i), sn = __ldg(s4 + i);
    const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e_i = 8 * i + 2 * j;
      const float e = __uint_as_float(a[e_i]), o = __uint_as_float(a[e_i + 1]);
      a[e_i] = __float_as_uint(fmaf(e, cc[j], o * ss[j]));
      a[e_i + 1] = __float_as_uint(fmaf(o, cc[j], -e * ss[j]));
    }
  }
}

// 16 columns of this warp's TMEM lane quarter, without waiting (see tmem_wait16).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tie16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}

__device__ __forceinline__ void tmem_wait16(uint32_t (&a)[16], uint32_t (&b)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  tie16(a);
  tie16(b);
}

// 16 fp32 values -> chunks c0, c0 + 1 of row r of a 16-bit SW128 tile
template <typename T>
__device__ __forceinline__ void put_row16(uint8_t* tile, int r, int c0, const float* v) {
#pragma unroll
  for (int i = 0; i < 2; ++i)
    *reinterpret_cast<uint4*>(tile + sw128(r, c0 + i)) =
        make_uint4(pack2<T>(v[8 * i], v[8 * i + 1]), pack2<T>(v[8 * i + 2], v[8 * i + 3]),
                   pack2<T>(v[8 * i + 4], v[8 * i + 5]), pack2<T>(v[8 * i + 6], v[8 * i + 7]));
}

// D[tmem] (+)= A * B^T over K = 16 * ksteps: A a 128-row K-major SW128 tile
// (128-byte rows, the first 32 * ksteps bytes of each used), B K-major (its
// rows are the N index) or MN-major (rows are K, the 64 head elements N).
__device__ __forceinline__ void mma_k(uint32_t d, uint32_t a_base, uint32_t b_base, bool b_mn, uint32_t idesc,
                                      bool accumulate, int ksteps) {
  for (int kk = 0; kk < ksteps; ++kk) {
    const uint64_t a = umma::smem_desc_sw128(a_base + kk * 32, 16, 1024);
    const uint64_t b = b_mn ? umma::smem_desc_sw128(b_base + kk * 16 * 128, BN * 128, 1024)
                            : umma::smem_desc_sw128(b_base + kk * 32, 16, 1024);
    umma::mma_f16(d, a, b, idesc, (accumulate || kk) ? 1u : 0u);
  }
}

// Backward chunks are 32 rows: S / dP (or their transposes) are then 32 TMEM
// columns each, so two buffers of both plus the 64-column accumulators fit in
// 256 columns, and the next chunk's products run while the row threads work
// on the current one.  The row threads' 16-bit operand tile (dS, or P^T and
// dS^T) is single-buffered: a thread writes chunk c's rows only after the
// products that read chunk c-1's have completed (the *_free barriers).
constexpr int CB = 32;                // rows per backward chunk
constexpr int CTILE = CB * kD * 2;    // 4 KB

template <typename T>
struct IdescB {
  static constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  static constexpr uint32_t K32 = umma::idesc_f16(kBf16, false, false, BM, CB);  // N = 32 chunk rows
  static constexpr uint32_t MN = umma::idesc_f16(kBf16, false, true, BM, kD);    // N = head dim
};

// ------------------------------------------------------------ backward: dQ
// Item = 128 queries.  Lane 0 of warp 0 loads the Q and dO tiles, lane 1
// streams 32-key K/V chunks through a 4-deep ring.  The MMA lane keeps S and
// dP one chunk ahead (S_c = Q K_c^T, dP_c = dO V_c^T into TMEM buffer c % 2)
// and, once the row threads have written dS_c, issues dQ += dS_c K_c (K_c as
// the MN-major operand).  The row threads compute D = rowsum(dO * O) for
// their query once per item (two half-row threads combined through shared
// memory; written out for the dK/dV kernel), then per chunk
// P = exp2(S * scale * log2e - lse * log2e) and dS = P (dP - D).
namespace bq {
constexpr int kStages = 4;
constexpr int OFF_DO = TILE128;
constexpr int OFF_KV = 2 * TILE128;                    // kStages x (K 4 KB, V 4 KB)
constexpr int OFF_DS = OFF_KV + kStages * 2 * CTILE;   // dS: 128 rows x 128 bytes (first 64 used)
constexpr int OFF_BAR = OFF_DS + TILE128;
constexpr int kBars = 2 + 2 * kStages + 4 + 2 + 3;
constexpr int OFF_X = OFF_BAR + 256;                   // [2][128] fp32 partial row sums of D
constexpr int SMEM = OFF_X + 2 * BM * 4 + 1024;
constexpr uint32_t kTmemDP = 64, kTmemDQ = 128;       // S[2] at 0, 32; dP[2] at 64, 96
}  // namespace bq

template <typename T>
__global__ void __launch_bounds__(kBwdThreads, 2)
    attn_bwd_dq_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                   const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const T* __restrict__ o, const float* __restrict__ lse, float* __restrict__ delta,
                   T* __restrict__ dq, Plane po, Plane pdq, int N, int H, int ldl, int nblk, int total, float scale,
                   const float* __restrict__ rcos, const float* __restrict__ rsin) {
  using namespace bq;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* qd_full = bars;
  uint64_t* qd_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* sd_full = kv_empty + kStages;  // [2]
  uint64_t* s_free = sd_full + 2;          // [2]
  uint64_t* ds_full = s_free + 2;
  uint64_t* ds_free = ds_full + 1;
  uint64_t* dq_full = ds_free + 1;
  uint64_t* dq_empty = dq_full + 1;
  uint64_t* x_full = dq_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBars);
  float* xs = reinterpret_cast<float*>(smem + OFF_X);
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (N + CB - 1) / CB;
  if (threadIdx.x == 0) {
    umma::mbar_init(qd_full, 1);
    umma::mbar_init(qd_empty, 1 + kRowWarpsBwd);  // MMA commit + the row warps' D reads
    for (int s = 0; s < kStages; ++s) {
      umma::mbar_init(&kv_full[s], 1);
      umma::mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      umma::mbar_init(&sd_full[b], 1);
      umma::mbar_init(&s_free[b], kRowWarpsBwd);
    }
    umma::mbar_init(ds_full, kRowWarpsBwd);
    umma::mbar_init(ds_free, 1);
    umma::mbar_init(dq_full, 1);
    umma::mbar_init(dq_empty, kRowWarpsBwd);
    umma::mbar_init(x_full, kRowWarpsBwd);
    abort_flag = 0;
    umma::fence_barrier_init();
  }
  if (warp == 0) umma::tmem_alloc(tmem_slot, kTmemCols);
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // Q and dO tiles
      umma::tma_prefetch(&tmQ);
      umma::tma_prefetch(&tmDO);
      uint32_t t = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
        const Item it = item_at(item, nblk, H);
        if (!umma::mbar_wait(qd_empty, (t & 1) ^ 1, 0x51)) {
          abort_flag = 1;
          break;
        }
        umma::mbar_arrive_expect_tx(qd_full, 2 * TILE128);
        umma::tma_load_4d(smem, &tmQ, qd_full, 0, it.h, it.blk * BM, it.b);
        umma::tma_load_4d(smem + OFF_DO, &tmDO, qd_full, 0, it.h, it.blk * BM, it.b);
      }
    } else if (lane == 1) {  // K/V chunks
      umma::tma_prefetch(&tmK);
      umma::tma_prefetch(&tmV);
      uint32_t cc = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x) {
        const Item it = item_at(item, nblk, H);
        for (int j = 0; j < nch; ++j, ++cc) {
          const int s = cc % kStages;
          if (!umma::mbar_wait(&kv_empty[s], ((cc / kStages) & 1) ^ 1, 0x52)) {
            abort_flag = 1;
            break;
          }
          uint8_t* dst = smem + OFF_KV + s * 2 * CTILE;
          umma::mbar_arrive_expect_tx(&kv_full[s], 2 * CTILE);
          umma::tma_load_4d(dst, &tmK, &kv_full[s], 0, it.h, j * CB, it.b);
          umma::tma_load_4d(dst + CTILE, &tmV, &kv_full[s], 0, it.h, j * CB, it.b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S_c, dP_c into TMEM buffer c % 2
      auto issue_s = [&](uint32_t c, bool last) -> bool {
        const int s = c % kStages, b = c & 1;
        if (!umma::mbar_wait(&kv_full[s], (c / kStages) & 1, 0x54)) return false;
        if (!umma::mbar_wait(&s_free[b], ((c >> 1) & 1) ^ 1, 0x5b)) return false;
        umma::tc_fence_after();
        const uint32_t k_base = umma::smem_u32(smem + OFF_KV + s * 2 * CTILE);
        mma_k(tmem + b * CB, umma::smem_u32(smem), k_base, false, IdescB<T>::K32, false, 4);                  // S
        mma_k(tmem + kTmemDP + b * CB, umma::smem_u32(smem + OFF_DO), k_base + CTILE, false, IdescB<T>::K32,  // dP
              false, 4);
        umma::mma_commit(&sd_full[b]);
        if (last) umma::mma_commit(qd_empty);
        return true;
      };
      uint32_t cc = 0, t = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok && !abort_flag; item += gridDim.x, ++t) {
        if (!umma::mbar_wait(qd_full, t & 1, 0x53) || !issue_s(cc, nch == 1)) {
          ok = false;
          break;
        }
        for (int j = 0; j < nch; ++j, ++cc) {
          if (j + 1 < nch && !issue_s(cc + 1, j + 2 == nch)) {
            ok = false;
            break;
          }
          if (!umma::mbar_wait(ds_full, cc & 1, 0x55) ||
              (j == 0 && !umma::mbar_wait(dq_empty, (t & 1) ^ 1, 0x56))) {
            ok = false;
            break;
          }
          umma::tc_fence_after();
          const uint32_t k_base = umma::smem_u32(smem + OFF_KV + (cc % kStages) * 2 * CTILE);
          mma_k(tmem + kTmemDQ, umma::smem_u32(smem + OFF_DS), k_base, true, IdescB<T>::MN, j > 0, 2);  // dQ += dS K
          umma::mma_commit(ds_free);
          umma::mma_commit(&kv_empty[cc % kStages]);
          if (j == nch - 1) umma::mma_commit(dq_full);
        }
      }
      if (!ok) abort_flag = 1;
    }
  } else {
    const int quarter = warp & 3, half = (warp - 2) >> 2, row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    uint32_t cc = 0, t = 0;
    for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
      const Item it = item_at(item, nblk, H);
      const int r = it.blk * BM + row;
      const bool valid = r < N;
      // this row's half of O and its lse, loaded while the tiles are still in flight
      uint4 orow[4] = {};
      float lse2 = 0.f;
      if (valid) {
        const T* src = o + it.b * po.s_b + it.h * po.s_h + (int64_t)r * po.s_n + half * 32;
#pragma unroll
        for (int i = 0; i < 4; ++i) orow[i] = *reinterpret_cast<const uint4*>(src + 8 * i);
        lse2 = lse[(int64_t)it.bh * ldl + r] * kLog2e;
      }
      if (!umma::mbar_wait(qd_full, t & 1, 0x57)) {
        abort_flag = 1;
        break;
      }
      float part = 0.f;
      if (valid) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 o4 = orow[i];
          const uint4 d4 = *reinterpret_cast<const uint4*>(smem + OFF_DO + sw128(row, half * 4 + i));
          const T* oe = reinterpret_cast<const T*>(&o4);
          const T* de = reinterpret_cast<const T*>(&d4);
#pragma unroll
          for (int e = 0; e < 8; ++e) part = fmaf(Elem<T>::to_f(oe[e]), Elem<T>::to_f(de[e]), part);
        }
      }
      xs[half * BM + row] = part;
      warp_arrive(x_full, false);
      if (!umma::mbar_wait(x_full, t & 1, 0x5a)) {
        abort_flag = 1;
        break;
      }
      const float dsum = xs[row] + xs[BM + row];
      if (valid && half == 0) delta[(int64_t)it.bh * ldl + r] = dsum;
      warp_arrive(qd_empty, false);
      bool ok = true;
      for (int j = 0; j < nch; ++j, ++cc) {
        const int b = cc & 1;
        if (!umma::mbar_wait(&sd_full[b], (cc >> 1) & 1, 0x58)) {
          ok = false;
          break;
        }
        umma::tc_fence_after();
        uint32_t su[16], du[16];
        tmem_ld16_nowait(tmem + lane_off + b * CB + half * 16, su);
        tmem_ld16_nowait(tmem + lane_off + kTmemDP + b * CB + half * 16, du);
        tmem_wait16(su, du);
        warp_arrive(&s_free[b], false);  // the next-but-one chunk may overwrite this TMEM buffer
        const int k0 = j * CB + half * 16;
        const bool tail = k0 + 16 > N;
        float* ds = reinterpret_cast<float*>(su);  // dS overwrites S in place
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float p = exp2f(fmaf(__uint_as_float(su[c]), sl2, -lse2));
          if (tail && k0 + c >= N) p = 0.f;  // keys past the end
          ds[c] = p * (__uint_as_float(du[c]) - dsum);
        }
        // the dQ product of the previous chunk has read the dS tile
        if (!umma::mbar_wait(ds_free, (cc & 1) ^ 1, 0x5c)) {
          ok = false;
          break;
        }
        put_row16<T>(smem + OFF_DS, row, half * 2, ds);
        warp_arrive(ds_full, true);
      }
      if (!ok || !umma::mbar_wait(dq_full, t & 1, 0x59)) {
        abort_flag = 1;
        break;
      }
      umma::tc_fence_after();
      uint32_t a0[32];
      tmem_ld32_nowait(tmem + lane_off + kTmemDQ + half * 32, a0);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      tie32(a0);
      warp_arrive(dq_empty, false);
      if (valid) {
        if (rcos != nullptr) unrotate32(a0, rcos, rsin, r, half);
        store_row32<T>(dq + it.b * pdq.s_b + it.h * pdq.s_h + (int64_t)r * pdq.s_n + half * 32, a0, scale);
      }
    }
  }
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tmem, kTmemCols);
  }
}

// -------------------------------------------------------- backward: dK, dV
// Item = 128 keys.  Lane 0 of warp 0 loads the K and V tiles, lane 1 streams
// chunks of 32 queries -- Q_c, dO_c and their lse / D slices -- through a
// 4-deep ring.  The MMA lane keeps S^T = K Q_c^T and dP^T = V dO_c^T one
// chunk ahead (TMEM buffer c % 2) and, once the row threads have written
// P^T and dS^T (one key per thread pair), issues dV += P^T dO_c and
// dK += dS^T Q_c (dO_c and Q_c as MN-major operands); the accumulators stay in
// tensor memory for the whole item.
namespace bk {
constexpr int kStages = 4;
constexpr int STAGE = 2 * CTILE + 1024;  // Q, dO, then lse[32] and D[32] (1024-aligned stride)
constexpr int OFF_V = TILE128;
constexpr int OFF_CH = 2 * TILE128;
constexpr int OFF_PT = OFF_CH + kStages * STAGE;  // P^T, dS^T: 128 rows x 128 bytes (first 64 used)
constexpr int OFF_DST = OFF_PT + TILE128;
constexpr int OFF_BAR = OFF_DST + TILE128;
constexpr int kBars = 2 + 2 * kStages + 4 + 4;
constexpr int SMEM = OFF_BAR + kBars * 8 + 16 + 1024;
constexpr uint32_t kTmemDPT = 64, kTmemDV = 128, kTmemDK = 192;  // S^T[2] at 0, 32; dP^T[2] at 64, 96
}  // namespace bk

template <typename T>
__global__ void __launch_bounds__(kBwdThreads, 2)
    attn_bwd_dkdv_tc(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                     const __grid_constant__ CUtensorMap tmL, const __grid_constant__ CUtensorMap tmD,
                     T* __restrict__ dk, T* __restrict__ dv, Plane pdk, Plane pdv, int N, int H, int nblk, int total,
                     float scale, const float* __restrict__ rcos, const float* __restrict__ rsin) {
  using namespace bk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + 1;
  uint64_t* ch_full = bars + 2;
  uint64_t* ch_empty = ch_full + kStages;
  uint64_t* sd_full = ch_empty + kStages;  // [2]
  uint64_t* s_free = sd_full + 2;          // [2]
  uint64_t* ps_full = s_free + 2;
  uint64_t* pt_free = ps_full + 1;
  uint64_t* acc_full = pt_free + 1;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBars);
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (N + CB - 1) / CB;
  if (threadIdx.x == 0) {
    umma::mbar_init(kv_full, 1);
    umma::mbar_init(kv_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      umma::mbar_init(&ch_full[s], 1);
      umma::mbar_init(&ch_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      umma::mbar_init(&sd_full[b], 1);
      umma::mbar_init(&s_free[b], kRowWarpsBwd);
    }
    umma::mbar_init(ps_full, kRowWarpsBwd);
    umma::mbar_init(pt_free, 1);
    umma::mbar_init(acc_full, 1);
    umma::mbar_init(acc_empty, kRowWarpsBwd);
    abort_flag = 0;
    umma::fence_barrier_init();
  }
  if (warp == 0) umma::tmem_alloc(tmem_slot, kTmemCols);
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // K and V tiles
      umma::tma_prefetch(&tmK);
      umma::tma_prefetch(&tmV);
      uint32_t t = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
        const Item it = item_at(item, nblk, H);
        if (!umma::mbar_wait(kv_empty, (t & 1) ^ 1, 0x61)) {
          abort_flag = 1;
          break;
        }
        umma::mbar_arrive_expect_tx(kv_full, 2 * TILE128);
        umma::tma_load_4d(smem, &tmK, kv_full, 0, it.h, it.blk * BM, it.b);
        umma::tma_load_4d(smem + OFF_V, &tmV, kv_full, 0, it.h, it.blk * BM, it.b);
      }
    } else if (lane == 1) {  // query chunks
      umma::tma_prefetch(&tmQ);
      umma::tma_prefetch(&tmDO);
      umma::tma_prefetch(&tmL);
      umma::tma_prefetch(&tmD);
      uint32_t cc = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x) {
        const Item it = item_at(item, nblk, H);
        for (int j = 0; j < nch; ++j, ++cc) {
          const int s = cc % kStages;
          if (!umma::mbar_wait(&ch_empty[s], ((cc / kStages) & 1) ^ 1, 0x62)) {
            abort_flag = 1;
            break;
          }
          uint8_t* dst = smem + OFF_CH + s * STAGE;
          umma::mbar_arrive_expect_tx(&ch_full[s], 2 * CTILE + 2 * CB * 4);
          umma::tma_load_4d(dst, &tmQ, &ch_full[s], 0, it.h, j * CB, it.b);
          umma::tma_load_4d(dst + CTILE, &tmDO, &ch_full[s], 0, it.h, j * CB, it.b);
          umma::tma_load_2d(dst + 2 * CTILE, &tmL, &ch_full[s], j * CB, it.bh);
          umma::tma_load_2d(dst + 2 * CTILE + CB * 4, &tmD, &ch_full[s], j * CB, it.bh);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      auto issue_s = [&](uint32_t c, bool last) -> bool {
        const int s = c % kStages, b = c & 1;
        if (!umma::mbar_wait(&ch_full[s], (c / kStages) & 1, 0x64)) return false;
        if (!umma::mbar_wait(&s_free[b], ((c >> 1) & 1) ^ 1, 0x6b)) return false;
        umma::tc_fence_after();
        const uint32_t q_base = umma::smem_u32(smem + OFF_CH + s * STAGE);
        mma_k(tmem + b * CB, umma::smem_u32(smem), q_base, false, IdescB<T>::K32, false, 4);                 // S^T
        mma_k(tmem + kTmemDPT + b * CB, umma::smem_u32(smem + OFF_V), q_base + CTILE, false, IdescB<T>::K32,  // dP^T
              false, 4);
        umma::mma_commit(&sd_full[b]);
        if (last) umma::mma_commit(kv_empty);
        return true;
      };
      uint32_t cc = 0, t = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok && !abort_flag; item += gridDim.x, ++t) {
        if (!umma::mbar_wait(kv_full, t & 1, 0x63) || !issue_s(cc, nch == 1)) {
          ok = false;
          break;
        }
        for (int j = 0; j < nch; ++j, ++cc) {
          if (j + 1 < nch && !issue_s(cc + 1, j + 2 == nch)) {
            ok = false;
            break;
          }
          if (!umma::mbar_wait(ps_full, cc & 1, 0x65) ||
              (j == 0 && !umma::mbar_wait(acc_empty, (t & 1) ^ 1, 0x66))) {
            ok = false;
            break;
          }
          umma::tc_fence_after();
          const uint32_t q_base = umma::smem_u32(smem + OFF_CH + (cc % kStages) * STAGE);
          mma_k(tmem + kTmemDV, umma::smem_u32(smem + OFF_PT), q_base + CTILE, true, IdescB<T>::MN, j > 0, 2);  // dV
          mma_k(tmem + kTmemDK, umma::smem_u32(smem + OFF_DST), q_base, true, IdescB<T>::MN, j > 0, 2);        // dK
          umma::mma_commit(pt_free);
          umma::mma_commit(&ch_empty[cc % kStages]);
          if (j == nch - 1) umma::mma_commit(acc_full);
        }
      }
      if (!ok) abort_flag = 1;
    }
  } else {
    const int quarter = warp & 3, half = (warp - 2) >> 2, row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    uint32_t cc = 0, t = 0;
    for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
      const Item it = item_at(item, nblk, H);
      bool ok = true;
      for (int j = 0; j < nch; ++j, ++cc) {
        const int s = cc % kStages, b = cc & 1;
        // the lse / D slices are read from the stage: wait for its TMA as well as for the products
        if (!umma::mbar_wait(&ch_full[s], (cc / kStages) & 1, 0x67) ||
            !umma::mbar_wait(&sd_full[b], (cc >> 1) & 1, 0x68)) {
          ok = false;
          break;
        }
        umma::tc_fence_after();
        uint32_t su[16], du[16];
        tmem_ld16_nowait(tmem + lane_off + b * CB + half * 16, su);
        tmem_ld16_nowait(tmem + lane_off + kTmemDPT + b * CB + half * 16, du);
        const float* ls = reinterpret_cast<const float*>(smem + OFF_CH + s * STAGE + 2 * CTILE) + half * 16;
        const float* dd_s = ls + CB;
        const int q0 = j * CB + half * 16;
        const bool tail = q0 + 16 > N;
        tmem_wait16(su, du);
        warp_arrive(&s_free[b], false);
        float* pt = reinterpret_cast<float*>(su);   // P^T overwrites S^T in place
        float* dst = reinterpret_cast<float*>(du);  // dS^T overwrites dP^T in place
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const float4 l4 = *reinterpret_cast<const float4*>(ls + 4 * c4);
          const float4 d4 = *reinterpret_cast<const float4*>(dd_s + 4 * c4);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dd[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = 4 * c4 + e;
            // queries past the end: their lse / D slots hold padding, so select zeros outright
            const bool dead = tail && q0 + c >= N;
            const float p = dead ? 0.f : exp2f(fmaf(__uint_as_float(su[c]), sl2, -lv[e] * kLog2e));
            pt[c] = p;
            dst[c] = dead ? 0.f : p * (__uint_as_float(du[c]) - dd[e]);
          }
        }
        // the dV / dK products of the previous chunk have read the operand tiles
        if (!umma::mbar_wait(pt_free, (cc & 1) ^ 1, 0x6c)) {
          ok = false;
          break;
        }
        put_row16<T>(smem + OFF_PT, row, half * 2, pt);
        put_row16<T>(smem + OFF_DST, row, half * 2, dst);
        warp_arrive(ps_full, true);
      }
      if (!ok || !umma::mbar_wait(acc_full, t & 1, 0x69)) {
        abort_flag = 1;
        break;
      }
      umma::tc_fence_after();
      uint32_t vv[32], kv[32];
      tmem_ld32_nowait(tmem + lane_off + kTmemDV + half * 32, vv);
      tmem_ld32_nowait(tmem + lane_off + kTmemDK + half * 32, kv);
      tmem_wait2(vv, kv);
      warp_arrive(acc_empty, false);
      const int r = it.blk * BM + row;
      if (r < N) {
        store_row32<T>(dv + it.b * pdv.s_b + it.h * pdv.s_h + (int64_t)r * pdv.s_n + half * 32, vv, 1.f);
        if (rcos != nullptr) unrotate32(kv, rcos, rsin, r, half);
        store_row32<T>(dk + it.b * pdk.s_b + it.h * pdk.s_h + (int64_t)r * pdk.s_n + half * 32, kv, scale);
      }
    }
  }
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------- forward, short sequences
// N <= 128: every key of a (sequence, head) fits one 128-column S tile, so
// the softmax needs no running rescale.  Item = one sequence (N > 64) or two
// (N <= 64, rows 0-63 and 64-127, the cross-sequence blocks masked), as in
// the one-pass backward below.  Lane 0 of warp 0 loads Q, K, V (two 64-row
// boxes each) into a 2-deep stage ring; the MMA lane issues S = Q K^T
// (N = 128) and, once the row threads have written P over the stage's Q and
// K tiles (both consumed by S), O = P V (V as the MN-major operand, K = 128
// keys), then the next item's S; the row threads (one query row each) take
// the row max and sum, write P, and write O / l and lse.  2 CTAs per SM.
namespace fs {
constexpr int kStages = 2;
constexpr int OFF_K = TILE128, OFF_V = 2 * TILE128;
constexpr int STAGE = 3 * TILE128;  // Q, K, V; P (two 64-key blocks) later over Q and K
constexpr int OFF_BAR = kStages * STAGE;
constexpr int kBars = 2 * kStages + 6;
constexpr int SMEM = OFF_BAR + 128 + 1024;
constexpr uint32_t kTmemO = 128;  // S: columns 0-127, O: 128-191
}  // namespace fs

template <typename T>
struct IdescF {
  static constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  static constexpr uint32_t S = umma::idesc_f16(kBf16, false, false, BM, BM);  // N = 128 queries or keys, B K-major
  static constexpr uint32_t G = umma::idesc_f16(kBf16, false, true, BM, kD);   // B MN-major, N = head dim
  static constexpr uint32_t Q = umma::idesc_f16(kBf16, true, true, BM, kD);    // A MN-major as well
};

template <typename T, bool kPack>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_short_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, T* __restrict__ o, float* __restrict__ lse, Plane po,
                      int sequences, int N, int H, int ldl, int total, float scale, const T* __restrict__ glogit) {
  using namespace fs;
  constexpr bool pack = kPack;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* s_full = empty + kStages;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_free + 1;
  uint64_t* o_full = p_full + 1;
  uint64_t* o_empty = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBars);
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      umma::mbar_init(&full[s], 1);
      umma::mbar_init(&empty[s], 1);
    }
    umma::mbar_init(s_full, 1);
    umma::mbar_init(s_free, 4);
    umma::mbar_init(p_full, 4);
    umma::mbar_init(o_full, 1);
    umma::mbar_init(o_empty, 4);
    abort_flag = 0;
    umma::fence_barrier_init();
  }
  if (warp == 0) umma::tmem_alloc(tmem_slot, kTmemCols);
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      umma::tma_prefetch(&tmQ);
      umma::tma_prefetch(&tmK);
      umma::tma_prefetch(&tmV);
      uint32_t t = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
        const int st = t % kStages, p = item / H, h = item - p * H;
        if (!umma::mbar_wait(&empty[st], ((t / kStages) & 1) ^ 1, 0x81)) {
          abort_flag = 1;
          break;
        }
        uint8_t* base = smem + st * STAGE;
        umma::mbar_arrive_expect_tx(&full[st], STAGE);
#pragma unroll
        for (int slot = 0; slot < 2; ++slot) {
          const int seq = pack ? 2 * p + slot : p, pos = pack ? 0 : 64 * slot;  // past the end: zeros
          const int off = slot * 64 * 128;
          umma::tma_load_4d(base + off, &tmQ, &full[st], 0, h, pos, seq);
          umma::tma_load_4d(base + OFF_K + off, &tmK, &full[st], 0, h, pos, seq);
          umma::tma_load_4d(base + OFF_V + off, &tmV, &full[st], 0, h, pos, seq);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      auto issue_s = [&](uint32_t t) -> bool {
        const int st = t % kStages;
        if (!umma::mbar_wait(&full[st], (t / kStages) & 1, 0x82)) return false;
        if (!umma::mbar_wait(s_free, (t & 1) ^ 1, 0x83)) return false;
        umma::tc_fence_after();
        const uint32_t base = umma::smem_u32(smem + st * STAGE);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma::mma_f16(tmem, umma::smem_desc_sw128(base + kk * 32, 16, 1024),
                        umma::smem_desc_sw128(base + OFF_K + kk * 32, 16, 1024), IdescF<T>::S, kk ? 1u : 0u);
        umma::mma_commit(s_full);
        return true;
      };
      uint32_t t = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
        if ((t == 0 && !issue_s(0)) || !umma::mbar_wait(p_full, t & 1, 0x84) ||
            !umma::mbar_wait(o_empty, (t & 1) ^ 1, 0x85)) {
          ok = false;
          break;
        }
        umma::tc_fence_after();
        const int st = t % kStages;
        const uint32_t base = umma::smem_u32(smem + st * STAGE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // K = 128 keys: P block kk / 4 sits over Q (0) or K (1)
          umma::mma_f16(tmem + kTmemO, umma::smem_desc_sw128(base + (kk >> 2) * TILE128 + (kk & 3) * 32, 16, 1024),
                        umma::smem_desc_sw128(base + OFF_V + kk * 16 * 128, TILE128, 1024), IdescF<T>::G,
                        kk ? 1u : 0u);
        umma::mma_commit(o_full);
        umma::mma_commit(&empty[st]);
        if (item + (int)gridDim.x < total && !issue_s(t + 1)) {
          ok = false;
          break;
        }
      }
      if (!ok) abort_flag = 1;
    }
  } else {
    const int quarter = warp & 3, row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    const int slot = pack ? row >> 6 : 0, pos = pack ? row & 63 : row;
    uint32_t t = 0;
    for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
      const int st = t % kStages, p = item / H, h = item - p * H;
      const int seq = pack ? 2 * p + slot : p;
      uint8_t* base = smem + st * STAGE;
      if (!umma::mbar_wait(s_full, t & 1, 0x86)) {
        abort_flag = 1;
        break;
      }
      umma::tc_fence_after();
      float m, l;
      if constexpr (pack) {
        // the 64 keys of this row's own sequence; the other block of P is written as zeros
        uint32_t a[32], b[32];
        tmem_ld32_nowait(tmem + lane_off + slot * 64, a);
        tmem_ld32_nowait(tmem + lane_off + slot * 64 + 32, b);
        tmem_wait2(a, b);
        warp_arrive(s_free, false);
        float* s0 = reinterpret_cast<float*>(a);
        float* s1 = reinterpret_cast<float*>(b);
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (c >= N) s0[c] = -INFINITY;  // keys past the end (N >= 1: key 0 always exists)
          if (32 + c >= N) s1[c] = -INFINITY;
          mx4[c & 3] = fmaxf(mx4[c & 3], fmaxf(s0[c], s1[c]));
        }
        m = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;  // scale > 0
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          s0[c] = exp2f(fmaf(s0[c], sl2, -m));
          s1[c] = exp2f(fmaf(s1[c], sl2, -m));
          sum4[c & 3] += s0[c] + s1[c];
        }
        l = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
        uint8_t* own = base + slot * TILE128;
        put_row32<T>(own, row, 0, *reinterpret_cast<float(*)[32]>(s0));
        put_row32<T>(own, row, 4, *reinterpret_cast<float(*)[32]>(s1));
        uint8_t* other = base + (1 - slot) * TILE128;
#pragma unroll
        for (int i = 0; i < 8; ++i) *reinterpret_cast<uint4*>(other + sw128(row, i)) = make_uint4(0, 0, 0, 0);
      } else {
        // 128 keys: the max from a first read of the four 32-column groups, then P from a second read
        float mx = -INFINITY;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
          uint32_t a[32];
          tmem_ld32_nowait(tmem + lane_off + g * 32, a);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          tie32(a);
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (g * 32 + c < N) mx = fmaxf(mx, __uint_as_float(a[c]));
        }
        m = mx * sl2;
        l = 0.f;
#pragma unroll 1
        for (int g = 0; g < 4; ++g) {
          uint32_t a[32];
          tmem_ld32_nowait(tmem + lane_off + g * 32, a);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          tie32(a);
          if (g == 3) warp_arrive(s_free, false);
          float* pv = reinterpret_cast<float*>(a);
          float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            pv[c] = g * 32 + c < N ? exp2f(fmaf(pv[c], sl2, -m)) : 0.f;
            sum4[c & 3] += pv[c];
          }
          l += (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
          put_row32<T>(base + (g >> 1) * TILE128, row, (g & 1) * 4, *reinterpret_cast<float(*)[32]>(pv));
        }
      }
      warp_arrive(p_full, true);
      if (!umma::mbar_wait(o_full, t & 1, 0x87)) {
        abort_flag = 1;
        break;
      }
      umma::tc_fence_after();
      uint32_t oa[32], ob[32];
      tmem_ld32_nowait(tmem + lane_off + kTmemO, oa);
      tmem_ld32_nowait(tmem + lane_off + kTmemO + 32, ob);
      tmem_wait2(oa, ob);
      warp_arrive(o_empty, false);
      if (seq < sequences && pos < N) {
        // with the head gate: gated = o * sigma(logit[seq * N + pos, h]) in place of o
        const float mul = glogit != nullptr ? gate_of(glogit[((int64_t)seq * N + pos) * H + h]) / l : 1.f / l;
        store_row64<T>(o + seq * po.s_b + h * po.s_h + (int64_t)pos * po.s_n,
                       *reinterpret_cast<float(*)[32]>(oa), *reinterpret_cast<float(*)[32]>(ob), mul);
        lse[((int64_t)seq * H + h) * ldl + pos] = (m + log2f(l)) * kLn2;
      }
    }
  }
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tmem, kTmemCols);
  }
}

// ----------------------------------------------- backward, short sequences
// N <= 128: one work item holds every key and every query of one head of
// one sequence -- of two sequences when N <= 64, in rows 0-63 and 64-127, so
// that the 62-position band-axis sequences fill the 128 TMEM lanes -- and one
// CTA computes all three gradients in a single pass over the inputs.  Lane 0
// of warp 0 loads Q, K, V, dO and O (two 64-row boxes each) into a 2-deep
// stage ring.  The MMA lane issues S^T = K Q^T and dP^T = V dO^T (keys are
// the TMEM lanes, the 128 queries the columns) and, once the row threads
// have written P^T and dS^T, dV = P^T dO, dK = dS^T Q and dQ = dS K, then
// the next item's S^T and dP^T (the TMEM columns are free by then) -- the
// last reads the dS^T tile as an MN-major A operand, so dS is never
// transposed.  Row threads: D = rowsum(dO * O) for their query row from the
// staged tiles (two half-row threads combined through shared memory), P^T
// and dS^T for their key over half of its queries, then the three output
// rows of their TMEM lane (dV, dK of a key; dQ of a query).  In a packed
// pair the cross-sequence blocks of P^T and dS^T are zeroed once and never
// written again.
namespace bf {
constexpr int kStages = 2;
constexpr int OFF_K = TILE128, OFF_V = 2 * TILE128, OFF_DO = 3 * TILE128, OFF_O = 4 * TILE128;
constexpr int STAGE = 5 * TILE128;  // Q, K, V, dO, O
constexpr int kBars = 2 * kStages + 6;
constexpr uint32_t kTmemDPT = 128, kTmemDV = 256, kTmemDK = 320, kTmemDQ = 384, kCols = 512;
// P^T and dS^T: 128 keys x 128 queries as two 64-query SW128 blocks, the
// second kBlk bytes after the first.  In a packed pair rows 64-127 of block 0
// and rows 0-63 of block 1 are both the zero cross-sequence part, so the
// blocks overlap there: 24 KB per operand instead of 32, which leaves room
// for a second D / lse buffer (the next item's D is computed while the
// current item's gradient products run).
template <bool kPack>
struct Layout {
  static constexpr int kBlk = kPack ? TILE128 / 2 : TILE128;
  static constexpr int kOp = kBlk + TILE128;
  static constexpr int OFF_PT = kStages * STAGE;
  static constexpr int OFF_DST = OFF_PT + kOp;
  static constexpr int OFF_BAR = OFF_DST + kOp;
  // per buffer: [2][128] partial D, [128] lse * log2e, and (packed pairs) [128] head gates
  static constexpr int OFF_X = OFF_BAR + 128;
  static constexpr int kXBufs = kPack ? 2 : 1;
  static constexpr int kXFloats = (kPack ? 4 : 3) * BM;
  static constexpr int kXBytes = kXFloats * 4;
  static constexpr int SMEM = OFF_X + kXBufs * kXBytes + 1024;
  static_assert(SMEM <= 232448 - 64, "fused backward shared memory");
};

// Packed pairs keep the rotary angles of a thread's own row in the free TMEM
// columns: every item puts position row & 63 in TMEM lane `row`, so lane
// `row` holds cos of pairs 0..31 at columns kTmemRot.. and sin at
// kTmemRot + 32..; a thread's half reads its 16 pairs of each.
constexpr uint32_t kTmemRot = 448;

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

// unrotate32 with the thread's 16 angle pairs already loaded (c, s)
__device__ __forceinline__ void unrotate32_regs(uint32_t (&a)[32], const uint32_t (&c)[16], const uint32_t (&sn)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float cc = __uint_as_float(c[j]), ss = __uint_as_float(sn[j]);
    const float e = __uint_as_float(a[2 * j]), o = __uint_as_float(a[2 * j + 1]);
    a[2 * j] = __float_as_uint(fmaf(e, cc, o * ss));
    a[2 * j + 1] = __float_as_uint(fmaf(o, cc, -e * ss));
  }
}
}  // namespace bf

template <typename T, bool kPack>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_fused_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                      const __grid_constant__ CUtensorMap tmO, const float* __restrict__ lse, T* __restrict__ dq,
                      T* __restrict__ dk, T* __restrict__ dv, Plane pdq, Plane pdk, Plane pdv, int sequences, int N,
                      int H, int ldl, int total, float scale, const float* __restrict__ rcos,
                      const float* __restrict__ rsin, const T* __restrict__ glogit, T* __restrict__ dlogit,
                      int64_t dl_ld, float* __restrict__ dbias) {
  using namespace bf;
  using L = Layout<kPack>;
  constexpr bool pack = kPack;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* sd_full = empty + kStages;
  uint64_t* s_free = sd_full + 1;
  uint64_t* x_full = s_free + 1;
  uint64_t* ps_full = x_full + 1;
  uint64_t* acc_full = ps_full + 1;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBars);
  float* xbuf = reinterpret_cast<float*>(smem + L::OFF_X);
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      umma::mbar_init(&full[s], 1);
      umma::mbar_init(&empty[s], 1);
    }
    umma::mbar_init(sd_full, 1);
    umma::mbar_init(s_free, kRowWarpsBwd);
    umma::mbar_init(x_full, kRowWarpsBwd);
    umma::mbar_init(ps_full, kRowWarpsBwd);
    umma::mbar_init(acc_full, 1);
    umma::mbar_init(acc_empty, kRowWarpsBwd);
    abort_flag = 0;
    umma::fence_barrier_init();
  }
  if (warp == 0) umma::tmem_alloc(tmem_slot, kCols);
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      umma::tma_prefetch(&tmQ);
      umma::tma_prefetch(&tmK);
      umma::tma_prefetch(&tmV);
      umma::tma_prefetch(&tmDO);
      umma::tma_prefetch(&tmO);
      uint32_t t = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
        const int st = t % kStages, p = item / H, h = item - p * H;
        if (!umma::mbar_wait(&empty[st], ((t / kStages) & 1) ^ 1, 0x71)) {
          abort_flag = 1;
          break;
        }
        uint8_t* base = smem + st * STAGE;
        umma::mbar_arrive_expect_tx(&full[st], STAGE);
#pragma unroll
        for (int slot = 0; slot < 2; ++slot) {
          // rows 64 * slot.. of the tiles: the slot's sequence (packed) or positions 64.. (one sequence);
          // a sequence index past the end (odd count, packed) reads zeros
          const int seq = pack ? 2 * p + slot : p, pos = pack ? 0 : 64 * slot;
          const int off = slot * 64 * 128;
          umma::tma_load_4d(base + off, &tmQ, &full[st], 0, h, pos, seq);
          umma::tma_load_4d(base + OFF_K + off, &tmK, &full[st], 0, h, pos, seq);
          umma::tma_load_4d(base + OFF_V + off, &tmV, &full[st], 0, h, pos, seq);
          umma::tma_load_4d(base + OFF_DO + off, &tmDO, &full[st], 0, h, pos, seq);
          umma::tma_load_4d(base + OFF_O + off, &tmO, &full[st], 0, h, pos, seq);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      auto issue_s = [&](uint32_t t) -> bool {  // S^T, dP^T of the item's t-th stage
        const int st = t % kStages;
        if (!umma::mbar_wait(&full[st], (t / kStages) & 1, 0x72)) return false;
        if (!umma::mbar_wait(s_free, (t & 1) ^ 1, 0x73)) return false;
        umma::tc_fence_after();
        const uint32_t base = umma::smem_u32(smem + st * STAGE);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma::mma_f16(tmem, umma::smem_desc_sw128(base + OFF_K + kk * 32, 16, 1024),
                        umma::smem_desc_sw128(base + kk * 32, 16, 1024), IdescF<T>::S, kk ? 1u : 0u);
          umma::mma_f16(tmem + kTmemDPT, umma::smem_desc_sw128(base + OFF_V + kk * 32, 16, 1024),
                        umma::smem_desc_sw128(base + OFF_DO + kk * 32, 16, 1024), IdescF<T>::S, kk ? 1u : 0u);
        }
        umma::mma_commit(sd_full);
        return true;
      };
      const uint32_t pt = umma::smem_u32(smem + L::OFF_PT), dst = umma::smem_u32(smem + L::OFF_DST);
      uint32_t t = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
        if ((t == 0 && !issue_s(0)) || !umma::mbar_wait(ps_full, t & 1, 0x74) ||
            !umma::mbar_wait(acc_empty, (t & 1) ^ 1, 0x75)) {
          ok = false;
          break;
        }
        umma::tc_fence_after();
        const int st = t % kStages;
        const uint32_t base = umma::smem_u32(smem + st * STAGE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // K = 128 queries (dV, dK) or keys (dQ), 16 per instruction
          const uint32_t a_k = (kk >> 2) * L::kBlk + (kk & 3) * 32, b_mn = kk * 16 * 128;
          const uint32_t acc = kk ? 1u : 0u;
          umma::mma_f16(tmem + kTmemDV, umma::smem_desc_sw128(pt + a_k, 16, 1024),
                        umma::smem_desc_sw128(base + OFF_DO + b_mn, TILE128, 1024), IdescF<T>::G, acc);
          umma::mma_f16(tmem + kTmemDK, umma::smem_desc_sw128(dst + a_k, 16, 1024),
                        umma::smem_desc_sw128(base + b_mn, TILE128, 1024), IdescF<T>::G, acc);
          // dS^T as the MN-major A operand: its two 64-query blocks are kBlk apart
          umma::mma_f16(tmem + kTmemDQ, umma::smem_desc_sw128(dst + b_mn, L::kBlk, 1024),
                        umma::smem_desc_sw128(base + OFF_K + b_mn, TILE128, 1024), IdescF<T>::Q, acc);
        }
        umma::mma_commit(acc_full);
        umma::mma_commit(&empty[st]);
        // the next item's S^T / dP^T only now: it waits for that item's tiles, the gradients above must not
        if (item + (int)gridDim.x < total && !issue_s(t + 1)) {
          ok = false;
          break;
        }
      }
      if (!ok) abort_flag = 1;
    }
  } else {
    const int quarter = warp & 3, half = (warp - 2) >> 2, row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    // Row `row` of every tile: sequence slot and position.  Packed pairs never
    // write the other sequence's block of P^T / dS^T (the shared zero part of
    // the two blocks): zero it once.
    const int slot = pack ? row >> 6 : 0, pos = pack ? row & 63 : row;
    if (pack) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t off = (1 - slot) * L::kBlk + sw128(row, half * 4 + i);
        *reinterpret_cast<uint4*>(smem + L::OFF_PT + off) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(smem + L::OFF_DST + off) = make_uint4(0, 0, 0, 0);
      }
      if (rcos != nullptr) {  // this row's angle pairs into its TMEM lane, once for all items
        float cv[16], sv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const bool ok = pos < N;
          cv[j] = ok ? __ldg(rcos + pos * 32 + half * 16 + j) : 1.f;
          sv[j] = ok ? __ldg(rsin + pos * 32 + half * 16 + j) : 0.f;
        }
        tmem_st16(tmem + lane_off + kTmemRot + half * 16, cv);
        tmem_st16(tmem + lane_off + kTmemRot + 32 + half * 16, sv);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      }
    }
    // query columns of this thread: packed, 32 of its own sequence's block; otherwise 64 in two passes
    constexpr int npass = pack ? 1 : 2;
    const int col0 = pack ? slot * 64 + half * 32 : half * 64;
    auto seq_of = [&](int64_t item) { return pack ? 2 * (int)(item / H) + slot : (int)(item / H); };
    // lse of query `row` of an item (half 0 threads), read an item before it is staged
    auto lse_of = [&](int64_t item) -> float {
      const int seq = seq_of(item), h = (int)(item % H);
      return item < total && half == 0 && seq < sequences && pos < N ? lse[((int64_t)seq * H + h) * ldl + pos] : 0.f;
    };
    // D partial of query `row` over head elements [32 half, 32 half + 32) and its lse * log2e into buffer xb
    // (all row warps, then the exchange); returns false on a timeout
    auto stage_d = [&](uint32_t tt, int64_t item, float lse_v, float* xb) -> bool {
      const int st = tt % kStages;
      if (!umma::mbar_wait(&full[st], (tt / kStages) & 1, 0x76)) return false;
      const uint8_t* base = smem + st * STAGE;
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 o4 = *reinterpret_cast<const uint4*>(base + OFF_O + sw128(row, half * 4 + i));
        const uint4 d4 = *reinterpret_cast<const uint4*>(base + OFF_DO + sw128(row, half * 4 + i));
        const T* oe = reinterpret_cast<const T*>(&o4);
        const T* de = reinterpret_cast<const T*>(&d4);
#pragma unroll
        for (int e = 0; e < 8; ++e) part = fmaf(Elem<T>::to_f(oe[e]), Elem<T>::to_f(de[e]), part);
      }
      // With the head gate g of query `row` folded in, the staged "o" / "dO" tiles are the gated output and
      // its gradient: dO = g dGated, so D = rowsum(dO * O) = rowsum(dGated * gated) = part, dP^T's column of
      // this query carries g, and so must the P^T operand of dV = P^T dO.  Staging D / g and
      // lse log2e - log2 g instead of D and lse log2e makes the softmax loop give P^T g and
      // P^T g (dP^T_raw - D / g) = P^T (g dP^T_raw - D) = dS^T unchanged; g itself is kept for dlogit.
      float g = 1.f;
      if constexpr (pack) {
        const int seq = seq_of(item), h = (int)(item % H);
        if (glogit != nullptr && seq < sequences && pos < N)
          g = fmaxf(gate_of(glogit[((int64_t)seq * N + pos) * H + h]), 1e-30f);
        if (half == 0) xb[3 * BM + row] = g;
      }
      xb[half * BM + row] = part / g;
      if (half == 0)
        xb[2 * BM + row] = seq_of(item) < sequences && pos < N ? lse_v * kLog2e - (pack ? log2f(g) : 0.f) : 0.f;
      warp_arrive(x_full, false);
      return umma::mbar_wait(x_full, tt & 1, 0x77);
    };
    float lse_pf = lse_of(blockIdx.x);
    bool ok = true;
    if (pack && (int)blockIdx.x < total) {  // packed: D of item t + 1 is staged while item t's products run
      ok = stage_d(0, blockIdx.x, lse_pf, xbuf);
      lse_pf = lse_of((int64_t)blockIdx.x + gridDim.x);
    }
    uint32_t t = 0;
    for (int item = blockIdx.x; ok && item < total && !abort_flag; item += gridDim.x, ++t) {
      const int h = item % H, seq = seq_of(item);
      const bool valid = seq < sequences && pos < N;  // as a key and as a query
      float* xb = xbuf + (pack ? (t & 1) : 0) * L::kXFloats;
      if (!pack) {
        if (!stage_d(t, item, lse_pf, xb)) {
          ok = false;
          break;
        }
        lse_pf = lse_of((int64_t)item + gridDim.x);
      }
      const float* xs = xb;
      const float* ls = xb + 2 * BM;
      if (!umma::mbar_wait(sd_full, t & 1, 0x78)) {
        ok = false;
        break;
      }
      umma::tc_fence_after();
#pragma unroll
      for (int ps = 0; ps < npass; ++ps) {
        const int q0 = col0 + ps * 32;          // first query column of this pass
        const int qpos0 = pack ? q0 & 63 : q0;  // its position in the sequence
        uint32_t su[32], du[32];
        tmem_ld32_nowait(tmem + lane_off + q0, su);
        tmem_ld32_nowait(tmem + lane_off + kTmemDPT + q0, du);
        tmem_wait2(su, du);
        // after the last pass's loads the next item's S^T / dP^T may overwrite these TMEM columns
        if (ps == npass - 1) warp_arrive(s_free, false);
        float* pv = reinterpret_cast<float*>(su);   // P^T overwrites S^T in place
        float* dsv = reinterpret_cast<float*>(du);  // dS^T overwrites dP^T in place
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 l4 = *reinterpret_cast<const float4*>(ls + q0 + 4 * c4);
          const float4 x0 = *reinterpret_cast<const float4*>(xs + q0 + 4 * c4);
          const float4 x1 = *reinterpret_cast<const float4*>(xs + BM + q0 + 4 * c4);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
          const float dd[4] = {x0.x + x1.x, x0.y + x1.y, x0.z + x1.z, x0.w + x1.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = 4 * c4 + e;
            // the key (this row) and the query must both exist; padding rows give zeros
            const bool live = valid && qpos0 + c < N;
            const float pr = live ? exp2f(fmaf(__uint_as_float(su[c]), sl2, -lv[e])) : 0.f;
            pv[c] = pr;
            dsv[c] = live ? pr * (__uint_as_float(du[c]) - dd[e]) : 0.f;
          }
        }
        // the previous item's gradient products have completed (its acc_full was waited), so the tiles are free
        const int blk = (q0 >> 6) * L::kBlk;
        put_row32<T>(smem + L::OFF_PT + blk, row, (q0 & 63) >> 3, *reinterpret_cast<float(*)[32]>(pv));
        put_row32<T>(smem + L::OFF_DST + blk, row, (q0 & 63) >> 3, *reinterpret_cast<float(*)[32]>(dsv));
      }
      warp_arrive(ps_full, true);
      if (pack && item + (int64_t)gridDim.x < total) {
        // every row warp has finished this item's softmax (ps_full waited by the MMA lane before acc_full, and
        // the other buffer's last readers were item t - 1's): stage the next item's D now
        if (!stage_d(t + 1, (int64_t)item + gridDim.x, lse_pf, xbuf + ((t + 1) & 1) * L::kXFloats)) {
          ok = false;
          break;
        }
        lse_pf = lse_of((int64_t)item + 2 * (int64_t)gridDim.x);
      }
      if (!umma::mbar_wait(acc_full, t & 1, 0x79)) {
        ok = false;
        break;
      }
      umma::tc_fence_after();
      uint32_t gv[32], gk[32], gq[32];
      tmem_ld32_nowait(tmem + lane_off + kTmemDV + half * 32, gv);
      tmem_ld32_nowait(tmem + lane_off + kTmemDK + half * 32, gk);
      tmem_ld32_nowait(tmem + lane_off + kTmemDQ + half * 32, gq);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      tie32(gv);
      tie32(gk);
      tie32(gq);
      warp_arrive(acc_empty, false);
      if (valid) {
        const int64_t rv = seq * pdv.s_b + h * pdv.s_h + (int64_t)pos * pdv.s_n + half * 32;
        store_row32<T>(dv + rv, gv, 1.f);
      }
      if (rcos != nullptr) {
        if constexpr (pack) {
          // tcgen05.ld is warp-collective: every lane loads (rows past the sequence read the
          // identity angles the prologue wrote), only the valid rows store below
          uint32_t cr[16], sr[16];
          tmem_ld16_nowait(tmem + lane_off + kTmemRot + half * 16, cr);
          tmem_ld16_nowait(tmem + lane_off + kTmemRot + 32 + half * 16, sr);
          tmem_wait16(cr, sr);
          unrotate32_regs(gk, cr, sr);
          unrotate32_regs(gq, cr, sr);
        } else if (valid) {
          unrotate32(gk, rcos, rsin, pos, half);
          unrotate32(gq, rcos, rsin, pos, half);
        }
      }
      if (valid) {
        const int64_t rk = seq * pdk.s_b + h * pdk.s_h + (int64_t)pos * pdk.s_n + half * 32;
        const int64_t rq = seq * pdq.s_b + h * pdq.s_h + (int64_t)pos * pdq.s_n + half * 32;
        store_row32<T>(dk + rk, gk, scale);
        store_row32<T>(dq + rq, gq, scale);
      }
      if constexpr (pack) {
        // gradient of the gate logit of query `row`: sum_d dGated * o * g (1 - g) = D (1 - g), D = g * staged;
        // and, per warp, the sum of the stored values over its 32 queries (the gate bias gradient's partial of
        // this item and lane quarter, summed in a fixed order by the caller)
        if (dlogit != nullptr && half == 0) {  // warp-uniform
          float dl = 0.f;
          if (valid) {
            const float g = xs[3 * BM + row];
            const T v = Elem<T>::from_f((xs[row] + xs[BM + row]) * g * (1.f - g));
            dlogit[((int64_t)seq * N + pos) * dl_ld + h] = v;
            dl = Elem<T>::to_f(v);
          }
          if (dbias != nullptr) {
            dl = warp_sum(dl);
            if (lane == 0) dbias[(int64_t)item * 4 + quarter] = dl;
          }
        }
      }
    }
    if (!ok) abort_flag = 1;
  }
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tmem, kCols);
  }
}

// ------------------------------------------------------------------ host
bool plane_ok(const void* p, const Plane& pl) {
  return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && pl.s_b % 8 == 0 && pl.s_n % 8 == 0 &&
         pl.s_h % 8 == 0;
}

Plane plane_at(const int64_t* strides, int i) { return Plane{strides[3 * i], strides[3 * i + 1], strides[3 * i + 2]}; }

int64_t row_pitch(int64_t seq_len) { return (seq_len + 3) / 4 * 4; }

int check_shape(const char* name, int dtype, int64_t sequences, int64_t seq_len, int64_t heads, int64_t dim_head) {
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: bf16 or fp16 only (dtype %d)", name, dtype);
  PMB_REQUIRE(dim_head == kD, "%s: dim_head must be %d (got %lld)", name, kD, (long long)dim_head);
  PMB_REQUIRE(sequences >= 0 && heads > 0 && seq_len > 0 && seq_len <= (1 << 24), "%s: bad shape", name);
  PMB_REQUIRE(sequences * heads * ((seq_len + BM - 1) / BM) < ((int64_t)1 << 31) && sequences * heads < (1 << 30),
              "%s: too many sequences", name);
  return PMB_OK;
}

// Strides of a plane as the TMA map takes them: the stride of a dimension of
// extent 1 is never used, so it is replaced by the extent of the one inside.
Plane tma_strides(const Plane& pl, int64_t sequences, int N, int H) {
  Plane t = pl;
  if (H == 1) t.s_h = kD;
  if (N == 1) t.s_n = (int64_t)H * t.s_h;
  if (sequences == 1) t.s_b = (int64_t)N * t.s_n;
  return t;
}

// The TMA map (64, H, N, sequences) needs strides that do not overlap:
// head >= 64 elements, position >= H heads, sequence >= N positions.
bool plane_order_ok(const Plane& pl, int64_t sequences, int N, int H) {
  const Plane t = tma_strides(pl, sequences, N, H);
  return t.s_h >= kD && t.s_n >= (int64_t)H * t.s_h && t.s_b >= (int64_t)N * t.s_n;
}

// TMA map over one [sequences, N, H, 64] plane: dims (64, H, N, sequences), box (64, 1, rows, 1)
int plane_map(CUtensorMap& map, const void* base, const Plane& pl_in, int dtype, int64_t sequences, int N, int H,
              int rows, const char* name) {
  const Plane pl = tma_strides(pl_in, sequences, N, H);
  const uint64_t dims[4] = {(uint64_t)kD, (uint64_t)H, (uint64_t)N, (uint64_t)sequences};
  const uint64_t strides[3] = {(uint64_t)pl.s_h * 2, (uint64_t)pl.s_n * 2, (uint64_t)pl.s_b * 2};
  const uint32_t box[4] = {(uint32_t)kD, 1, (uint32_t)rows, 1};
  return tma::make_map_4d(map, base, dtype, dims, strides, box, name);
}

int grid_for(int64_t total) {
  int64_t g = (int64_t)num_sms() * 2;
  return (int)(g < total ? g : total);
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int64_t pmb_attention_row_pitch(int64_t seq_len) { return seq_len > 0 ? row_pitch(seq_len) : 0; }

namespace pmb {
namespace {
// The forward of both entry points; glogit (16-bit [sequences * seq_len, heads], or NULL) gates the output.
int attention_forward(const void* q, const void* k, const void* v, void* o, float* lse, int64_t sequences,
                      int64_t seq_len, int64_t heads, int64_t dim_head, const int64_t* strides, float scale, int dtype,
                      const void* glogit, void* stream, const char* name) {
  if (int st = check_shape(name, dtype, sequences, seq_len, heads, dim_head)) return st;
  if (sequences == 0) return PMB_OK;
  PMB_REQUIRE(lse && strides, "%s: NULL argument", name);
  const Plane pq = plane_at(strides, 0), pk = plane_at(strides, 1), pv = plane_at(strides, 2),
              po = plane_at(strides, 3);
  PMB_REQUIRE(plane_ok(q, pq) && plane_ok(k, pk) && plane_ok(v, pv) && plane_ok(o, po),
              "%s: planes must be non-NULL, 16-byte aligned, with strides that are multiples of 8", name);
  const int N = (int)seq_len, H = (int)heads, nblk = (N + BM - 1) / BM;
  const int64_t total = sequences * heads * nblk;
  PMB_REQUIRE(plane_order_ok(pq, sequences, N, H) && plane_order_ok(pk, sequences, N, H) &&
                  plane_order_ok(pv, sequences, N, H),
              "%s: q, k, v strides must not overlap (head >= 64, position >= heads * head, sequence >= seq_len * "
              "position)", name);
  CUtensorMap mq, mk, mv;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (N <= BM) {
    // every key in one S tile; two sequences per item when N <= 64
    const bool pack = N <= 64;
    const int64_t items = (pack ? (sequences + 1) / 2 : sequences) * heads;
    if (int st = plane_map(mq, q, pq, dtype, sequences, N, H, 64, name)) return st;
    if (int st = plane_map(mk, k, pk, dtype, sequences, N, H, 64, name)) return st;
    if (int st = plane_map(mv, v, pv, dtype, sequences, N, H, 64, name)) return st;
    auto run = [&](auto tag) {
      using T = decltype(tag);
      auto kernel = pack ? attn_fwd_short_tc<T, true> : attn_fwd_short_tc<T, false>;
      PMB_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fs::SMEM), name);
      kernel<<<grid_for(items), kThreads, fs::SMEM, s>>>(mq, mk, mv, static_cast<T*>(o), lse, po, (int)sequences, N,
                                                         H, (int)row_pitch(N), (int)items, scale,
                                                         static_cast<const T*>(glogit));
      PMB_CHECK_LAUNCH(name);
      return PMB_OK;
    };
    return dtype == PMB_BFLOAT16 ? run(__nv_bfloat16()) : run(__half());
  }
  if (int st = plane_map(mq, q, pq, dtype, sequences, N, H, BM, name)) return st;
  if (int st = plane_map(mk, k, pk, dtype, sequences, N, H, BN, name)) return st;
  if (int st = plane_map(mv, v, pv, dtype, sequences, N, H, BN, name)) return st;
  auto run = [&](auto tag) {
    using T = decltype(tag);
    PMB_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_tc<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, fw::SMEM), name);
    attn_fwd_tc<T><<<grid_for(total), kThreads, fw::SMEM, s>>>(mq, mk, mv, static_cast<T*>(o), lse, po, N, H,
                                                               (int)row_pitch(N), nblk, (int)total, scale);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  };
  return dtype == PMB_BFLOAT16 ? run(__nv_bfloat16()) : run(__half());
}
}  // namespace
}  // namespace pmb

extern "C" int pmb_attention_forward(const void* q, const void* k, const void* v, void* o, float* lse,
                                     int64_t sequences, int64_t seq_len, int64_t heads, int64_t dim_head,
                                     const int64_t* strides, float scale, int dtype, void* stream) {
  clear_error();
  return attention_forward(q, k, v, o, lse, sequences, seq_len, heads, dim_head, strides, scale, dtype, nullptr,
                           stream, "pmb_attention_forward");
}

extern "C" int pmb_attention_forward_gated(const void* q, const void* k, const void* v, const void* gate_logits,
                                           void* gated, float* lse, int64_t sequences, int64_t seq_len,
                                           int64_t heads, int64_t dim_head, const int64_t* strides, float scale,
                                           int dtype, void* stream) {
  clear_error();
  const char* name = "pmb_attention_forward_gated";
  PMB_REQUIRE(gate_logits != nullptr, "%s: NULL gate logits", name);
  PMB_REQUIRE(seq_len <= 64, "%s: the gated kernels take sequences of up to 64 positions (got %lld)", name,
              (long long)seq_len);
  return attention_forward(q, k, v, gated, lse, sequences, seq_len, heads, dim_head, strides, scale, dtype,
                           gate_logits, stream, name);
}

extern "C" int64_t pmb_attention_backward_workspace_size(int64_t sequences, int64_t seq_len, int64_t heads) {
  if (sequences <= 0 || seq_len <= 0 || heads <= 0) return 0;
  return (sequences * heads * row_pitch(seq_len) * 4 + 255) / 256 * 256;
}

namespace pmb {
namespace {
// The backward of both entry points; rcos / rsin (fp32 [seq_len, 32], or both NULL) rotate dQ and dK back.
int attention_backward(const void* q, const void* k, const void* v, const void* o, const void* grad_out,
                       const float* lse, void* grad_q, void* grad_k, void* grad_v, int64_t sequences, int64_t seq_len,
                       int64_t heads, int64_t dim_head, const int64_t* strides, float scale, int dtype,
                       const float* rcos, const float* rsin, void* workspace, int64_t workspace_bytes, void* stream,
                       const char* name, const void* glogit = nullptr, void* dlogit = nullptr, int64_t dl_ld = 0,
                       float* dbias = nullptr) {
  if (int st = check_shape(name, dtype, sequences, seq_len, heads, dim_head)) return st;
  if (sequences == 0) return PMB_OK;
  PMB_REQUIRE(lse && strides, "%s: NULL argument", name);
  const int64_t need = pmb_attention_backward_workspace_size(sequences, seq_len, heads);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  PMB_REQUIRE((reinterpret_cast<uintptr_t>(lse) & 15) == 0 && (reinterpret_cast<uintptr_t>(workspace) & 15) == 0,
              "%s: lse and workspace must be 16-byte aligned", name);
  const Plane pq = plane_at(strides, 0), pk = plane_at(strides, 1), pv = plane_at(strides, 2),
              po = plane_at(strides, 3), pdo = plane_at(strides, 4), pdq = plane_at(strides, 5),
              pdk = plane_at(strides, 6), pdv = plane_at(strides, 7);
  PMB_REQUIRE(plane_ok(q, pq) && plane_ok(k, pk) && plane_ok(v, pv) && plane_ok(o, po) && plane_ok(grad_out, pdo) &&
                  plane_ok(grad_q, pdq) && plane_ok(grad_k, pdk) && plane_ok(grad_v, pdv),
              "%s: planes must be non-NULL, 16-byte aligned, with strides that are multiples of 8", name);
  const int N = (int)seq_len, H = (int)heads, nblk = (N + BM - 1) / BM;
  const int64_t total = sequences * heads * nblk, ldl = row_pitch(N), rows = sequences * heads;
  PMB_REQUIRE(plane_order_ok(pq, sequences, N, H) && plane_order_ok(pk, sequences, N, H) &&
                  plane_order_ok(pv, sequences, N, H) && plane_order_ok(pdo, sequences, N, H),
              "%s: q, k, v, grad_out strides must not overlap (head >= 64, position >= heads * head, sequence >= "
              "seq_len * position)", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (N <= BM && plane_order_ok(po, sequences, N, H)) {
    // one pass: every key and query of a (sequence, head) -- two sequences when N <= 64 -- in one work item
    const bool pack = N <= 64;
    const int64_t items = (pack ? (sequences + 1) / 2 : sequences) * heads;
    CUtensorMap mq, mk, mv, mdo, mo;
    if (int st = plane_map(mq, q, pq, dtype, sequences, N, H, 64, name)) return st;
    if (int st = plane_map(mk, k, pk, dtype, sequences, N, H, 64, name)) return st;
    if (int st = plane_map(mv, v, pv, dtype, sequences, N, H, 64, name)) return st;
    if (int st = plane_map(mdo, grad_out, pdo, dtype, sequences, N, H, 64, name)) return st;
    if (int st = plane_map(mo, o, po, dtype, sequences, N, H, 64, name)) return st;
    const int grid = (int)(items < num_sms() ? items : num_sms());
    auto run = [&](auto tag) {
      using T = decltype(tag);
      auto kernel = pack ? attn_bwd_fused_tc<T, true> : attn_bwd_fused_tc<T, false>;
      const int smem = pack ? bf::Layout<true>::SMEM : bf::Layout<false>::SMEM;
      PMB_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), name);
      kernel<<<grid, kBwdThreads, smem, s>>>(mq, mk, mv, mdo, mo, lse, static_cast<T*>(grad_q),
                                                 static_cast<T*>(grad_k), static_cast<T*>(grad_v), pdq, pdk, pdv,
                                                 (int)sequences, N, H, (int)ldl, (int)items, scale, rcos, rsin,
                                                 static_cast<const T*>(glogit), static_cast<T*>(dlogit), dl_ld,
                                                 dbias);
      PMB_CHECK_LAUNCH(name);
      return PMB_OK;
    };
    return dtype == PMB_BFLOAT16 ? run(__nv_bfloat16()) : run(__half());
  }
  // the gate is folded into the one-pass kernel only
  PMB_REQUIRE(glogit == nullptr, "%s: the gated output must be laid out like q (non-overlapping plane strides)",
              name);
  float* delta = static_cast<float*>(workspace);
  CUtensorMap mq128, mdo128, mk64, mv64, mk128, mv128, mq64, mdo64, ml, md;  // *64: 32-row chunk maps
  if (int st = plane_map(mq128, q, pq, dtype, sequences, N, H, BM, name)) return st;
  if (int st = plane_map(mdo128, grad_out, pdo, dtype, sequences, N, H, BM, name)) return st;
  if (int st = plane_map(mk64, k, pk, dtype, sequences, N, H, CB, name)) return st;
  if (int st = plane_map(mv64, v, pv, dtype, sequences, N, H, CB, name)) return st;
  if (int st = plane_map(mk128, k, pk, dtype, sequences, N, H, BM, name)) return st;
  if (int st = plane_map(mv128, v, pv, dtype, sequences, N, H, BM, name)) return st;
  if (int st = plane_map(mq64, q, pq, dtype, sequences, N, H, CB, name)) return st;
  if (int st = plane_map(mdo64, grad_out, pdo, dtype, sequences, N, H, CB, name)) return st;
  if (int st = tma::make_map_rows_f32(ml, lse, ldl, rows, ldl * 4, CB, name)) return st;
  if (int st = tma::make_map_rows_f32(md, delta, ldl, rows, ldl * 4, CB, name)) return st;
  const int grid = grid_for(total);
  auto run = [&](auto tag) {
    using T = decltype(tag);
    PMB_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dq_tc<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, bq::SMEM),
                   name);
    PMB_CHECK_CUDA(
        cudaFuncSetAttribute(attn_bwd_dkdv_tc<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, bk::SMEM), name);
    attn_bwd_dq_tc<T><<<grid, kBwdThreads, bq::SMEM, s>>>(mq128, mdo128, mk64, mv64, static_cast<const T*>(o), lse,
                                                        delta, static_cast<T*>(grad_q), po, pdq, N, H, (int)ldl, nblk,
                                                        (int)total, scale, rcos, rsin);
    PMB_CHECK_LAUNCH(name);
    attn_bwd_dkdv_tc<T><<<grid, kBwdThreads, bk::SMEM, s>>>(mk128, mv128, mq64, mdo64, ml, md, static_cast<T*>(grad_k),
                                                          static_cast<T*>(grad_v), pdk, pdv, N, H, nblk, (int)total,
                                                          scale, rcos, rsin);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  };
  return dtype == PMB_BFLOAT16 ? run(__nv_bfloat16()) : run(__half());
}
}  // namespace
}  // namespace pmb

extern "C" int pmb_attention_backward(const void* q, const void* k, const void* v, const void* o,
                                      const void* grad_out, const float* lse, void* grad_q, void* grad_k,
                                      void* grad_v, int64_t sequences, int64_t seq_len, int64_t heads,
                                      int64_t dim_head, const int64_t* strides, float scale, int dtype,
                                      void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  return attention_backward(q, k, v, o, grad_out, lse, grad_q, grad_k, grad_v, sequences, seq_len, heads, dim_head,
                            strides, scale, dtype, nullptr, nullptr, workspace, workspace_bytes, stream,
                            "pmb_attention_backward");
}

extern "C" int pmb_attention_backward_rotary(const void* q, const void* k, const void* v, const void* o,
                                             const void* grad_out, const float* lse, const float* cos,
                                             const float* sin, void* grad_q, void* grad_k, void* grad_v,
                                             int64_t sequences, int64_t seq_len, int64_t heads, int64_t dim_head,
                                             const int64_t* strides, float scale, int dtype, void* workspace,
                                             int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_attention_backward_rotary";
  PMB_REQUIRE(cos && sin && (reinterpret_cast<uintptr_t>(cos) & 15) == 0 && (reinterpret_cast<uintptr_t>(sin) & 15) == 0,
              "%s: angle tables must be non-NULL and 16-byte aligned", name);
  return attention_backward(q, k, v, o, grad_out, lse, grad_q, grad_k, grad_v, sequences, seq_len, heads, dim_head,
                            strides, scale, dtype, cos, sin, workspace, workspace_bytes, stream, name);
}

extern "C" int64_t pmb_attention_gate_bias_partials(int64_t sequences, int64_t heads) {
  return sequences > 0 && heads > 0 ? (sequences + 1) / 2 * heads * 4 : 0;
}

extern "C" int pmb_attention_backward_gated(const void* q, const void* k, const void* v, const void* gated,
                                            const void* grad_gated, const float* lse, const void* gate_logits,
                                            const float* cos, const float* sin, void* grad_q, void* grad_k,
                                            void* grad_v, void* grad_logits, int64_t grad_logits_ld,
                                            float* grad_bias_partials, int64_t sequences, int64_t seq_len,
                                            int64_t heads, int64_t dim_head, const int64_t* strides, float scale,
                                            int dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_attention_backward_gated";
  PMB_REQUIRE(gate_logits && grad_logits && grad_logits_ld >= heads, "%s: gate logits and their gradient needed",
              name);
  PMB_REQUIRE(seq_len <= 64, "%s: the gated kernels take sequences of up to 64 positions (got %lld)", name,
              (long long)seq_len);
  PMB_REQUIRE((cos == nullptr) == (sin == nullptr) &&
                  (reinterpret_cast<uintptr_t>(cos) & 15) == 0 && (reinterpret_cast<uintptr_t>(sin) & 15) == 0,
              "%s: angle tables must both be given (16-byte aligned) or both be NULL", name);
  return attention_backward(q, k, v, gated, grad_gated, lse, grad_q, grad_k, grad_v, sequences, seq_len, heads,
                            dim_head, strides, scale, dtype, cos, sin, workspace, workspace_bytes, stream, name,
                            gate_logits, grad_logits, grad_logits_ld, grad_bias_partials);
}
