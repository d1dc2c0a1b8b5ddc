// Scaled-dot-product attention core of the axial transformers (head dim 64,
// no mask, no dropout), forward and backward, bf16 / fp16 in, fp32 math.
//
//   S = Q K^T * scale,  P = softmax_rows(S),  O = P V,  lse = log(sum exp S)
//   backward:  D = rowsum(dO * O),  dP = dO V^T,  dS = P * (dP - D),
//              dV = P^T dO,  dQ = scale * dS K,  dK = scale * dS^T Q
//
// Forward: attn_fwd_tc, a persistent warp-specialised tcgen05 kernel (TMA
// tiles, S and per-chunk O accumulators in tensor memory, one softmax thread
// per query row); described above the kernel.
// Backward: two kernels over 64-row blocks of one (sequence, head), four
// warps per CTA, each warp owning 16 rows of the block, products on
// mma.sync m16n8k16 (fp32 accumulators) from ldmatrix fragments:
//   attn_bwd_dq    query block; computes D for its rows, then streams K/V
//                  chunks (double-buffered cp.async ring) recomputing P and
//                  dP and accumulating dQ;
//   attn_bwd_dkdv  key block; streams Q/dO chunks (with lse and D) and
//                  accumulates dK and dV for its keys.
// No atomics: every output row is owned by one thread or warp, so results
// are deterministic.  P and dS are rounded to the input type before their
// products, as torch's fused attention kernels do.
//
// Layout: q, k, v, o and their gradients are [sequences, N, H, 64] planes
// with any sequence / position / head element strides (multiples of 8, the
// 64 head elements contiguous); lse and D are fp32 [sequences * H, N].
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
constexpr int kLd = kD + 8;     // shared-memory row pitch in elements (144 bytes)
constexpr int kBlock = 64;      // rows per CTA block and per streamed chunk (backward)
constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kTile = kBlock * kLd;  // elements of one staged 64-row tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct Plane {
  int64_t s_b, s_n, s_h;  // element strides of a [sequences, N, H, 64] plane
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0));
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0));
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }

template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// c += a * b for one m16n8k16 tile (fp32 accumulators)
template <typename T>
__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const T a = Elem<T>::from_f(lo), b = Elem<T>::from_f(hi);
  return (uint32_t)(*reinterpret_cast<const uint16_t*>(&a)) |
         ((uint32_t)(*reinterpret_cast<const uint16_t*>(&b)) << 16);
}

template <int N>
__device__ __forceinline__ void zero(float (&a)[N][4]) {
#pragma unroll
  for (int i = 0; i < N; ++i) a[i][0] = a[i][1] = a[i][2] = a[i][3] = 0.f;
}

// Rows [row0, row0 + 64) of one (sequence, head) of a plane into a staged
// tile (cp.async; rows >= N are zero-filled).  The whole CTA.
template <typename T>
__device__ __forceinline__ void load_tile(T* dst, const T* src, int64_t s_n, int row0, int N) {
#pragma unroll
  for (int i = threadIdx.x; i < kBlock * (kD / 8); i += kThreads) {
    const int r = i >> 3, c = (i & 7) * 8, gr = row0 + r;
    const bool ok = gr < N;
    cp_async16(dst + r * kLd + c, src + (ok ? (int64_t)gr * s_n + c : 0), ok);
  }
}

// A fragments of a 16 x 64 row-major slab of a staged tile: a[k-step][4]
template <typename T>
__device__ __forceinline__ void load_a(uint32_t (&a)[4][4], const T* slab) {
  const int lane = threadIdx.x & 31;
  const int r = (lane & 7) + 8 * ((lane >> 3) & 1), c = 8 * (lane >> 4);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) ldsm_x4(a[ks], slab + r * kLd + ks * 16 + c);
}

// acc[0..2*NP) (16 x 16*NP) += A (16 x 64, fragments a) * rows^T, where rows
// are NP*16 consecutive rows of a staged tile starting at `rows` (the n index
// runs over those rows, k over the 64 columns).
template <typename T, int NP>
__device__ __forceinline__ void mma_rows_t(float (&acc)[2 * NP][4], const uint32_t (&a)[4][4], const T* rows) {
  const int lane = threadIdx.x & 31;
  const int rr = (lane & 7) + 8 * (lane >> 4), cc = 8 * ((lane >> 3) & 1);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int np = 0; np < NP; ++np) {
      uint32_t b[4];
      ldsm_x4(b, rows + (np * 16 + rr) * kLd + ks * 16 + cc);
      mma<T>(acc[2 * np], a[ks], b[0], b[1]);
      mma<T>(acc[2 * np + 1], a[ks], b[2], b[3]);
    }
  }
}

// acc[0..8) (16 x 64) += A (16 x 16*KS, fragments a) * rows, where rows are
// 16*KS consecutive rows of a staged tile (the k index runs over those rows,
// n over the 64 columns).
template <typename T, int KS>
__device__ __forceinline__ void mma_rows(float (&acc)[8][4], const uint32_t (&a)[KS][4], const T* rows) {
  const int lane = threadIdx.x & 31;
  const int rr = (lane & 7) + 8 * ((lane >> 3) & 1), cc = 8 * (lane >> 4);
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm_x4_t(b, rows + (ks * 16 + rr) * kLd + np * 16 + cc);
      mma<T>(acc[2 * np], a[ks], b[0], b[1]);
      mma<T>(acc[2 * np + 1], a[ks], b[2], b[3]);
    }
  }
}

// C fragments of NT 8-column tiles (16 rows) -> A fragments of NT/2 k-steps
template <typename T, int NT>
__device__ __forceinline__ void c_to_a(uint32_t (&a)[NT / 2][4], const float (&c)[NT][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    a[nt >> 1][(nt & 1) * 2 + 0] = pack2<T>(c[nt][0], c[nt][1]);
    a[nt >> 1][(nt & 1) * 2 + 1] = pack2<T>(c[nt][2], c[nt][3]);
  }
}

// A warp's 16 x 64 accumulator (times `mul`) through its own 16 staged rows
// to rows [r0, r0 + 16) of a plane (rows >= N skipped), 16-byte segments.
template <typename T>
__device__ __forceinline__ void store_rows(const float (&acc)[8][4], float mul, T* stage, T* dst, int64_t s_n, int r0,
                                           int N) {
  const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int c = nt * 8 + tig * 2;
    *reinterpret_cast<uint32_t*>(stage + g * kLd + c) = pack2<T>(acc[nt][0] * mul, acc[nt][1] * mul);
    *reinterpret_cast<uint32_t*>(stage + (g + 8) * kLd + c) = pack2<T>(acc[nt][2] * mul, acc[nt][3] * mul);
  }
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 4 + (lane >> 3), c = (lane & 7) * 8;
    if (r0 + r < N)
      *reinterpret_cast<uint4*>(dst + (int64_t)(r0 + r) * s_n + c) = *reinterpret_cast<const uint4*>(stage + r * kLd + c);
  }
}

// ---------------------------------------------------------------- forward
// tcgen05 forward.  Work item = 128 query rows of one (sequence, head);
// persistent CTAs (two per SM) take items blockIdx.x, + gridDim.x, ...
//   warp 0 (one lane)  TMA: the item's Q tile (4-D plane map, rows >= N read
//                      as zeros), then its K/V chunks into a kStages ring;
//   warp 1 (one lane)  tcgen05.mma: S_c = Q K_c^T into TMEM S[c % 2]
//                      (M 128, N 64, K 64), and one chunk behind,
//                      O_c = P_c V_c into TMEM O[c % 2] (V read as an MN-major
//                      operand straight from its TMA tile);
//   warps 2..5         softmax, one query row per thread (TMEM lane = row):
//                      reads S_c, keeps the running max / sum, writes P_c as
//                      bf16/fp16 into shared memory in the 128-byte-swizzled
//                      K-major layout the MMA reads, then folds O_{c-1} into
//                      its fp32 row accumulator (rescaled by the max change)
//                      and finally writes O and the row lse.
// Chunks are counted across items, so every barrier phase runs on.  All
// waits are bounded; on a timeout the roles stop, TMEM is freed and the
// site is left in the attention timeout flag.
namespace tcf {
constexpr int BM = 128;        // query rows per item
constexpr int BN = 64;         // keys per chunk
constexpr int kThreads = 192;  // TMA warp, MMA warp, 4 softmax warps
constexpr int kStages = 3;     // K/V chunk ring
constexpr int Q_BYTES = BM * kD * 2;
constexpr int KV_BYTES = BN * kD * 2;
constexpr int P_BYTES = BM * BN * 2;
constexpr int OFF_KV = Q_BYTES;
constexpr int OFF_P = OFF_KV + kStages * 2 * KV_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr int kBars = 2 + 2 * kStages + 8;
constexpr int SMEM = OFF_BAR + kBars * 8 + 16 + 1024;  // + slack for the 1024-byte alignment
constexpr uint32_t kTmemCols = 256;                     // S[2] at columns 0, 64; O[2] at 128, 192
constexpr uint32_t kTmemO = 128;
}  // namespace tcf

template <typename T>
__global__ void __launch_bounds__(tcf::kThreads, 2)
    attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, T* __restrict__ o, float* __restrict__ lse, Plane po, int N,
                int H, int nqb, int total, float scale) {
  using namespace tcf;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = umma::idesc_f16(kBf16, false, false, BM, BN);
  constexpr uint32_t IDESC_O = umma::idesc_f16(kBf16, false, true, BM, kD);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
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
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      umma::tma_prefetch(&tmQ);
      umma::tma_prefetch(&tmK);
      umma::tma_prefetch(&tmV);
      uint32_t cc = 0, t = 0;
      for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x, ++t) {
        const int bh = item / nqb, qb = item - bh * nqb, b = bh / H, h = bh - b * H;
        if (!umma::mbar_wait(q_empty, (t & 1) ^ 1, 0x41)) {
          abort_flag = 1;
          break;
        }
        umma::mbar_arrive_expect_tx(q_full, Q_BYTES);
        umma::tma_load_4d(smem, &tmQ, q_full, 0, h, qb * BM, b);
        for (int j = 0; j < nch; ++j, ++cc) {
          const int s = cc % kStages;
          if (!umma::mbar_wait(&kv_empty[s], ((cc / kStages) & 1) ^ 1, 0x42)) {
            abort_flag = 1;
            break;
          }
          uint8_t* dst = smem + OFF_KV + s * 2 * KV_BYTES;
          umma::mbar_arrive_expect_tx(&kv_full[s], 2 * KV_BYTES);
          umma::tma_load_4d(dst, &tmK, &kv_full[s], 0, h, j * BN, b);
          umma::tma_load_4d(dst + KV_BYTES, &tmV, &kv_full[s], 0, h, j * BN, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      // O_c = P_c V_c, issued one chunk behind S so that S_{c+1} runs during softmax c
      auto issue_o = [&](uint32_t c) -> bool {
        const int pb = c & 1;
        if (!umma::mbar_wait(&p_full[pb], (c >> 1) & 1, 0x44)) return false;
        if (!umma::mbar_wait(&o_empty[pb], ((c >> 1) & 1) ^ 1, 0x45)) return false;
        umma::tc_fence_after();
        const uint32_t p_base = umma::smem_u32(smem + OFF_P + pb * P_BYTES);
        const uint32_t v_base = umma::smem_u32(smem + OFF_KV + (c % kStages) * 2 * KV_BYTES + KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma::mma_f16(tmem + kTmemO + pb * kD, umma::smem_desc_sw128(p_base + kk * 32, 16, 1024),
                        umma::smem_desc_sw128(v_base + kk * 16 * 128, BN * 128, 1024), IDESC_O, kk != 0);
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
        const uint32_t q_base = umma::smem_u32(smem);
        for (int j = 0; j < nch; ++j, ++cc) {
          const int s = cc % kStages;
          if (!umma::mbar_wait(&kv_full[s], (cc / kStages) & 1, 0x46)) {
            ok = false;
            break;
          }
          umma::tc_fence_after();
          const uint32_t k_base = umma::smem_u32(smem + OFF_KV + s * 2 * KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            umma::mma_f16(tmem + (cc & 1) * BN, umma::smem_desc_sw128(q_base + kk * 32, 16, 1024),
                          umma::smem_desc_sw128(k_base + kk * 32, 16, 1024), IDESC_S, kk != 0);
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
    // ---------------------------------------------------- softmax warps
    const int quarter = warp & 3, row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    uint32_t cc = 0;
    for (int item = blockIdx.x; item < total && !abort_flag; item += gridDim.x) {
      const int bh = item / nqb, qb = item - bh * nqb, b = bh / H, h = bh - b * H;
      float m = -INFINITY, l = 0.f, corr_prev = 0.f;
      float acc[kD];
#pragma unroll
      for (int c = 0; c < kD; ++c) acc[c] = 0.f;
      bool ok = true;
      // fold O of chunk c into acc (acc * corr + O_c), release the O buffer
      auto fold_o = [&](uint32_t c, float corr) -> bool {
        const int ob = c & 1;
        if (!umma::mbar_wait(&o_full[ob], (c >> 1) & 1, 0x48)) return false;
        umma::tc_fence_after();
        float v0[32], v1[32];
        umma::tmem_ld32(tmem + lane_off + kTmemO + ob * kD, v0);
        umma::tmem_ld32(tmem + lane_off + kTmemO + ob * kD + 32, v1);
        umma::tc_fence_before();
        __syncwarp();
        if (lane == 0) umma::mbar_arrive(&o_empty[ob]);
#pragma unroll
        for (int c2 = 0; c2 < 32; ++c2) {
          acc[c2] = acc[c2] * corr + v0[c2];
          acc[32 + c2] = acc[32 + c2] * corr + v1[c2];
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
        float s[BN];
        umma::tmem_ld32(tmem + lane_off + sb * BN, *reinterpret_cast<float(*)[32]>(&s[0]));
        umma::tmem_ld32(tmem + lane_off + sb * BN + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
        const int kc = j * BN;
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const float v = (kc + c < N) ? s[c] * sl2 : -INFINITY;
          s[c] = v;
          mx = fmaxf(mx, v);
        }
        const float mn = fmaxf(m, mx);  // finite: every chunk holds a key < N
        const float corr = exp2f(m - mn);
        float sum = 0.f;
        uint8_t* prow = smem + OFF_P + sb * P_BYTES + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
        for (int ch = 0; ch < BN / 8; ++ch) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p0 = exp2f(s[ch * 8 + 2 * e] - mn), p1 = exp2f(s[ch * 8 + 2 * e + 1] - mn);
            sum += p0 + p1;
            w[e] = pack2<T>(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l = l * corr + sum;
        m = mn;
        umma::fence_proxy_async_smem();
        umma::tc_fence_before();
        __syncwarp();
        if (lane == 0) umma::mbar_arrive(&p_full[sb]);
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
      const int r = qb * BM + row;
      if (r < N) {
        const float inv = 1.f / l;
        T* dst = o + b * po.s_b + h * po.s_h + (int64_t)r * po.s_n;
#pragma unroll
        for (int ch = 0; ch < kD / 8; ++ch) {
          uint4 u;
          u.x = pack2<T>(acc[ch * 8 + 0] * inv, acc[ch * 8 + 1] * inv);
          u.y = pack2<T>(acc[ch * 8 + 2] * inv, acc[ch * 8 + 3] * inv);
          u.z = pack2<T>(acc[ch * 8 + 4] * inv, acc[ch * 8 + 5] * inv);
          u.w = pack2<T>(acc[ch * 8 + 6] * inv, acc[ch * 8 + 7] * inv);
          *reinterpret_cast<uint4*>(dst + ch * 8) = u;
        }
        lse[(int64_t)bh * N + r] = (m + log2f(l)) * kLn2;
      }
    }
  }
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tmem, tcf::kTmemCols);
  }
}

// ------------------------------------------------------------ backward: dQ
template <typename T>
__global__ void __launch_bounds__(kThreads, 4)
    attn_bwd_dq(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ o,
                const T* __restrict__ dout, const float* __restrict__ lse, float* __restrict__ delta,
                T* __restrict__ dq, Plane pq, Plane pk, Plane pv, Plane po, Plane pdo, Plane pdq, int N, int H,
                int nqb, float scale) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* Qs = reinterpret_cast<T*>(smem_raw);
  T* Ds = Qs + kTile;      // dO tile
  T* Ks = Ds + kTile;      // 2 buffers
  T* Vs = Ks + 2 * kTile;  // 2 buffers
  const int qb = blockIdx.x % nqb, bh = blockIdx.x / nqb, b = bh / H, h = bh - b * H;
  const T* kg = k + b * pk.s_b + h * pk.s_h;
  const T* vg = v + b * pv.s_b + h * pv.s_h;
  const int q0 = qb * kBlock, nch = (N + kBlock - 1) / kBlock;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tig = lane & 3;
  const int r0 = q0 + warp * 16;
  const bool active = r0 < N;
  const float sl2 = scale * kLog2e;

  load_tile(Qs, q + b * pq.s_b + h * pq.s_h, pq.s_n, q0, N);
  load_tile(Ds, dout + b * pdo.s_b + h * pdo.s_h, pdo.s_n, q0, N);
  cp_commit();
  load_tile(Ks, kg, pk.s_n, 0, N);
  load_tile(Vs, vg, pv.s_n, 0, N);
  cp_commit();

  uint32_t qa[4][4], da[4][4];
  float lse2[2] = {0.f, 0.f}, dlt[2] = {0.f, 0.f};
  cp_wait<1>();  // Q and dO tiles
  __syncthreads();
  if (active) {
    load_a(qa, Qs + warp * 16 * kLd);
    load_a(da, Ds + warp * 16 * kLd);
    // D = rowsum(dO * O) of this warp's rows: lane pair (2i, 2i+1) sums row i's halves
    const int dr = lane >> 1, dh = (lane & 1) * 32;
    float dpart = 0.f;
    if (r0 + dr < N) {
      const T* orow = o + b * po.s_b + h * po.s_h + (int64_t)(r0 + dr) * po.s_n + dh;
      const T* drow = Ds + (warp * 16 + dr) * kLd + dh;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 o4 = *reinterpret_cast<const uint4*>(orow + i * 8);
        const uint4 d4 = *reinterpret_cast<const uint4*>(drow + i * 8);
        const T* oe = reinterpret_cast<const T*>(&o4);
        const T* de = reinterpret_cast<const T*>(&d4);
#pragma unroll
        for (int e = 0; e < 8; ++e) dpart += Elem<T>::to_f(oe[e]) * Elem<T>::to_f(de[e]);
      }
    }
    dpart += __shfl_xor_sync(0xffffffffu, dpart, 1);
    if (r0 + dr < N && (lane & 1) == 0) delta[(int64_t)bh * N + r0 + dr] = dpart;
    dlt[0] = __shfl_sync(0xffffffffu, dpart, 2 * g);
    dlt[1] = __shfl_sync(0xffffffffu, dpart, 2 * g + 16);
    const float* lb = lse + (int64_t)bh * N;
    lse2[0] = r0 + g < N ? lb[r0 + g] * kLog2e : 0.f;
    lse2[1] = r0 + g + 8 < N ? lb[r0 + g + 8] * kLog2e : 0.f;
  }
  float dqacc[8][4];
  zero(dqacc);
  for (int j = 0; j < nch; ++j) {
    const int buf = j & 1;
    if (j + 1 < nch) {
      load_tile(Ks + (buf ^ 1) * kTile, kg, pk.s_n, (j + 1) * kBlock, N);
      load_tile(Vs + (buf ^ 1) * kTile, vg, pv.s_n, (j + 1) * kBlock, N);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (active) {
      const T* Kc = Ks + buf * kTile;
      const T* Vc = Vs + buf * kTile;
      const int kc = j * kBlock;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {  // 32-key halves of the chunk
        float s[4][4], dp[4][4];
        zero(s);
        zero(dp);
        mma_rows_t<T, 2>(s, qa, Kc + hh * 32 * kLd);
        mma_rows_t<T, 2>(dp, da, Vc + hh * 32 * kLd);
        const bool tail = kc + hh * 32 + 32 > N;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float p = exp2f(s[nt][e] * sl2 - lse2[e >> 1]);
            if (tail && kc + hh * 32 + nt * 8 + tig * 2 + (e & 1) >= N) p = 0.f;
            s[nt][e] = p * (dp[nt][e] - dlt[e >> 1]);  // dS
          }
        }
        uint32_t sa[2][4];
        c_to_a<T, 4>(sa, s);
        mma_rows<T, 2>(dqacc, sa, Kc + hh * 32 * kLd);
      }
    }
    __syncthreads();
  }
  if (!active) return;
  store_rows<T>(dqacc, scale, Qs + warp * 16 * kLd, dq + b * pdq.s_b + h * pdq.s_h, pdq.s_n, r0, N);
}

// -------------------------------------------------------- backward: dK, dV
template <typename T>
__global__ void __launch_bounds__(kThreads, 3)
    attn_bwd_dkdv(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                  const T* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ delta,
                  T* __restrict__ dk, T* __restrict__ dv, Plane pq, Plane pk, Plane pv, Plane pdo, Plane pdk,
                  Plane pdv, int N, int H, int nkb, float scale) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* Ks = reinterpret_cast<T*>(smem_raw);
  T* Vs = Ks + kTile;
  T* Qs = Vs + kTile;      // 2 buffers
  T* Os = Qs + 2 * kTile;  // dO, 2 buffers
  float* Ls = reinterpret_cast<float*>(Os + 2 * kTile);  // [2][64] lse, then [2][64] D
  const int kb = blockIdx.x % nkb, bh = blockIdx.x / nkb, b = bh / H, h = bh - b * H;
  const T* qg = q + b * pq.s_b + h * pq.s_h;
  const T* dog = dout + b * pdo.s_b + h * pdo.s_h;
  const float* lg = lse + (int64_t)bh * N;
  const float* dg = delta + (int64_t)bh * N;
  const int k0 = kb * kBlock, nch = (N + kBlock - 1) / kBlock;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tig = lane & 3;
  const int r0 = k0 + warp * 16;
  const bool active = r0 < N;
  const float sl2 = scale * kLog2e;

  auto load_rowstats = [&](int buf, int row0) {
    const int i = threadIdx.x & 63, which = threadIdx.x >> 6;  // 128 threads: 64 lse + 64 D
    const bool ok = row0 + i < N;
    const float* src = which ? dg : lg;
    cp_async4(Ls + (which * 2 + buf) * kBlock + i, src + (ok ? row0 + i : 0), ok);
  };
  load_tile(Ks, k + b * pk.s_b + h * pk.s_h, pk.s_n, k0, N);
  load_tile(Vs, v + b * pv.s_b + h * pv.s_h, pv.s_n, k0, N);
  load_tile(Qs, qg, pq.s_n, 0, N);
  load_tile(Os, dog, pdo.s_n, 0, N);
  load_rowstats(0, 0);
  cp_commit();

  uint32_t ka[4][4];
  float dkacc[8][4], dvacc[8][4];
  zero(dkacc);
  zero(dvacc);
  for (int j = 0; j < nch; ++j) {
    const int buf = j & 1;
    if (j + 1 < nch) {
      load_tile(Qs + (buf ^ 1) * kTile, qg, pq.s_n, (j + 1) * kBlock, N);
      load_tile(Os + (buf ^ 1) * kTile, dog, pdo.s_n, (j + 1) * kBlock, N);
      load_rowstats(buf ^ 1, (j + 1) * kBlock);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (active) {
      if (j == 0) load_a(ka, Ks + warp * 16 * kLd);
      const T* Qc = Qs + buf * kTile;
      const T* Oc = Os + buf * kTile;
      const float* lc = Ls + buf * kBlock;
      const float* dc = Ls + (2 + buf) * kBlock;
      const int qc = j * kBlock;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {  // 32-query halves of the chunk
        float st[4][4], dpt[4][4];
        zero(st);
        zero(dpt);
        mma_rows_t<T, 2>(st, ka, Qc + hh * 32 * kLd);  // S^T: keys x queries
        {
          uint32_t va[4][4];  // reloaded from the warp's own V rows: keeps registers for the accumulators
          load_a(va, Vs + warp * 16 * kLd);
          mma_rows_t<T, 2>(dpt, va, Oc + hh * 32 * kLd);  // dP^T = V dO^T
        }
        const bool tail = qc + hh * 32 + 32 > N;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int col = hh * 32 + nt * 8 + tig * 2 + e;  // query within the chunk
            const float ls = lc[col] * kLog2e, dd = dc[col];
            const bool dead = tail && qc + col >= N;
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const int idx = rr * 2 + e;
              const float p = dead ? 0.f : exp2f(st[nt][idx] * sl2 - ls);
              st[nt][idx] = p;
              dpt[nt][idx] = p * (dpt[nt][idx] - dd);  // dS^T
            }
          }
        }
        uint32_t pa[2][4], sa[2][4];
        c_to_a<T, 4>(pa, st);
        c_to_a<T, 4>(sa, dpt);
        mma_rows<T, 2>(dvacc, pa, Oc + hh * 32 * kLd);  // dV += P^T dO
        mma_rows<T, 2>(dkacc, sa, Qc + hh * 32 * kLd);  // dK += dS^T Q
      }
    }
    __syncthreads();
  }
  if (!active) return;
  store_rows<T>(dkacc, scale, Ks + warp * 16 * kLd, dk + b * pdk.s_b + h * pdk.s_h, pdk.s_n, r0, N);
  store_rows<T>(dvacc, 1.f, Vs + warp * 16 * kLd, dv + b * pdv.s_b + h * pdv.s_h, pdv.s_n, r0, N);
}

constexpr size_t kDqSmem = (size_t)6 * kTile * 2;
constexpr size_t kDkdvSmem = (size_t)6 * kTile * 2 + 4 * kBlock * 4;

bool plane_ok(const void* p, const Plane& pl) {
  return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && pl.s_b % 8 == 0 && pl.s_n % 8 == 0 &&
         pl.s_h % 8 == 0;
}

Plane plane_at(const int64_t* strides, int i) { return Plane{strides[3 * i], strides[3 * i + 1], strides[3 * i + 2]}; }

int check_shape(const char* name, int dtype, int64_t sequences, int64_t seq_len, int64_t heads, int64_t dim_head) {
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: bf16 or fp16 only (dtype %d)", name, dtype);
  PMB_REQUIRE(dim_head == kD, "%s: dim_head must be %d (got %lld)", name, kD, (long long)dim_head);
  PMB_REQUIRE(sequences >= 0 && heads > 0 && seq_len > 0 && seq_len <= (1 << 24), "%s: bad shape", name);
  PMB_REQUIRE(sequences * heads * ((seq_len + kBlock - 1) / kBlock) < ((int64_t)1 << 31), "%s: grid too large",
              name);
  return PMB_OK;
}

// TMA map over one [sequences, N, H, 64] plane: dims (64, H, N, sequences), box (64, 1, rows, 1)
int plane_map(CUtensorMap& map, const void* base, const Plane& pl, int dtype, int64_t sequences, int N, int H,
              int rows, const char* name) {
  const uint64_t dims[4] = {(uint64_t)kD, (uint64_t)H, (uint64_t)N, (uint64_t)sequences};
  const uint64_t strides[3] = {(uint64_t)pl.s_h * 2, (uint64_t)pl.s_n * 2, (uint64_t)pl.s_b * 2};
  const uint32_t box[4] = {(uint32_t)kD, 1, (uint32_t)rows, 1};
  return tma::make_map_4d(map, base, dtype, dims, strides, box, name);
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_attention_forward(const void* q, const void* k, const void* v, void* o, float* lse,
                                     int64_t sequences, int64_t seq_len, int64_t heads, int64_t dim_head,
                                     const int64_t* strides, float scale, int dtype, void* stream) {
  clear_error();
  const char* name = "pmb_attention_forward";
  if (int st = check_shape(name, dtype, sequences, seq_len, heads, dim_head)) return st;
  if (sequences == 0) return PMB_OK;
  PMB_REQUIRE(lse && strides, "%s: NULL argument", name);
  const Plane pq = plane_at(strides, 0), pk = plane_at(strides, 1), pv = plane_at(strides, 2),
              po = plane_at(strides, 3);
  PMB_REQUIRE(plane_ok(q, pq) && plane_ok(k, pk) && plane_ok(v, pv) && plane_ok(o, po),
              "%s: planes must be non-NULL, 16-byte aligned, with strides that are multiples of 8", name);
  const int N = (int)seq_len, H = (int)heads, nqb = (N + tcf::BM - 1) / tcf::BM;
  const int64_t total = sequences * heads * nqb;
  PMB_REQUIRE(total < ((int64_t)1 << 31), "%s: too many sequences", name);
  CUtensorMap mq, mk, mv;
  if (int st = plane_map(mq, q, pq, dtype, sequences, N, H, tcf::BM, name)) return st;
  if (int st = plane_map(mk, k, pk, dtype, sequences, N, H, tcf::BN, name)) return st;
  if (int st = plane_map(mv, v, pv, dtype, sequences, N, H, tcf::BN, name)) return st;
  int64_t grid = (int64_t)num_sms() * 2;
  if (grid > total) grid = total;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run = [&](auto tag) {
    using T = decltype(tag);
    PMB_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_tc<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, tcf::SMEM), name);
    attn_fwd_tc<T><<<(unsigned)grid, tcf::kThreads, tcf::SMEM, s>>>(mq, mk, mv, static_cast<T*>(o), lse, po, N, H,
                                                                     nqb, (int)total, scale);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  };
  return dtype == PMB_BFLOAT16 ? run(__nv_bfloat16()) : run(__half());
}

extern "C" int64_t pmb_attention_backward_workspace_size(int64_t sequences, int64_t seq_len, int64_t heads) {
  if (sequences <= 0 || seq_len <= 0 || heads <= 0) return 0;
  return (sequences * heads * seq_len * 4 + 255) / 256 * 256;
}

extern "C" int pmb_attention_backward(const void* q, const void* k, const void* v, const void* o,
                                      const void* grad_out, const float* lse, void* grad_q, void* grad_k,
                                      void* grad_v, int64_t sequences, int64_t seq_len, int64_t heads,
                                      int64_t dim_head, const int64_t* strides, float scale, int dtype,
                                      void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_attention_backward";
  if (int st = check_shape(name, dtype, sequences, seq_len, heads, dim_head)) return st;
  if (sequences == 0) return PMB_OK;
  PMB_REQUIRE(lse && strides, "%s: NULL argument", name);
  const int64_t need = pmb_attention_backward_workspace_size(sequences, seq_len, heads);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  const Plane pq = plane_at(strides, 0), pk = plane_at(strides, 1), pv = plane_at(strides, 2),
              po = plane_at(strides, 3), pdo = plane_at(strides, 4), pdq = plane_at(strides, 5),
              pdk = plane_at(strides, 6), pdv = plane_at(strides, 7);
  PMB_REQUIRE(plane_ok(q, pq) && plane_ok(k, pk) && plane_ok(v, pv) && plane_ok(o, po) && plane_ok(grad_out, pdo) &&
                  plane_ok(grad_q, pdq) && plane_ok(grad_k, pdk) && plane_ok(grad_v, pdv),
              "%s: planes must be non-NULL, 16-byte aligned, with strides that are multiples of 8", name);
  const int N = (int)seq_len, nb = (N + kBlock - 1) / kBlock;
  const unsigned grid = (unsigned)(sequences * heads * nb);
  float* delta = static_cast<float*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run = [&](auto tag) {
    using T = decltype(tag);
    PMB_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dq<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDqSmem),
                   name);
    PMB_CHECK_CUDA(
        cudaFuncSetAttribute(attn_bwd_dkdv<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDkdvSmem), name);
    attn_bwd_dq<T><<<grid, kThreads, kDqSmem, s>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(o),
        static_cast<const T*>(grad_out), lse, delta, static_cast<T*>(grad_q), pq, pk, pv, po, pdo, pdq, N,
        (int)heads, nb, scale);
    PMB_CHECK_LAUNCH(name);
    attn_bwd_dkdv<T><<<grid, kThreads, kDkdvSmem, s>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(grad_out),
        lse, delta, static_cast<T*>(grad_k), static_cast<T*>(grad_v), pq, pk, pv, pdo, pdk, pdv, N, (int)heads, nb,
        scale);
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  };
  return dtype == PMB_BFLOAT16 ? run(__nv_bfloat16()) : run(__half());
}
