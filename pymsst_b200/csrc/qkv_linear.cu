// Attention input projection with the rotary embedding in the GEMM epilogue
// (training path, bf16 / fp16 on the tcgen05 tensor cores).
//
//   [q | k | v][r, :] = x[r, :] W^T,  each written as a [B*N, H*Dh] row-major
//   plane (the [B, N, H, Dh] layout; q, k, v are its [B, H, N, Dh] views, which
//   the attention kernel reads in place).
// The epilogue rounds each q / k projection value to the activation dtype (as
// the stored projection of the unfused path) and rotates the interleaved pairs
// by the row's position angle; the angle tables are passed transposed
// ([Dh/2, N]) so the 32 rows of a warp read 32 consecutive positions of one
// pair (coalesced) instead of 32 scattered table rows, and each epilogue warp
// keeps the 16 angle pairs of its head half in registers across the chunks
// it drains (see the chunk map in QkvRotaryEpi).  Where sequences are
// contiguous rows (inner == 1) each warp's 32 x 32 block goes out as one TMA
// tile store; with the row map (inner > 1) the rows of a block are scattered
// over the plane and go out as 16-byte row vectors.  The projection is written once and never re-read for a split
// or rotary pass; the backward is pmb_qkv_rotary_merge plus the two
// projection-gradient GEMMs.
// Reference semantics: to_qkv projection + qkv_to_bnhd + rotary_forward on
// q and k (src/pymsst/training/fused_roformer.py:710-732, 793-818;
// rotary kernels src/pymsst/training/cuda/fused_band_split.cu:1077-1128).
#include "dense_gemm.cuh"

namespace pmb {
unsigned int timeout_flag_qkv(int reset) { return umma::flag_reader(reset); }

namespace {

template <typename T>
struct QkvRotaryEpi {
  T* plane[3];         // q, k, v: [sequences * seq, H*Dh]
  const float* cos_t;  // [Dh/2, seq]
  const float* sin_t;
  int hd, seq, dh, rotate, inner;
  int use_tma;           // inner == 1 and every plane accepts a TMA store map
  CUtensorMap maps[3];   // q, k, v planes as [rows, H*Dh] store maps
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    // x row r = (outer, position, inner index); its plane row is (outer * inner + inner index) * seq + position.
    // Rows past the end still map to a position in [0, seq): table reads stay in bounds.
    const int q_ = t.row / inner, ii = t.row - q_ * inner;
    const int o = q_ / seq, pos = q_ - o * seq;
    const int64_t prow = (int64_t)(o * inner + ii) * seq + pos;
    // Chunk -> warp map: with eight 32-column chunks per tile (BN = 256, 64-wide heads) the first warp of a lane
    // quarter takes the even chunks 0, 2, 4 (pairs 0..15 of a head), the second the odd chunks 1, 3, 5 (pairs
    // 16..31), the third chunks 6 and 7; so the first two read their 32 angle values once per tile and keep them
    // in registers.  Other widths use the round-robin map.
    constexpr int kNch = BN / 32;
    constexpr bool kPaired = kNch == 8;
    const int nmine = kPaired ? (t.sub < 2 ? 3 : 2) : (kNch - t.sub + ugemm::kSubs - 1) / ugemm::kSubs;
    float cc[16], sn[16];
    int cached = -1;
#pragma unroll 1
    for (int q = 0; q < nmine; ++q) {
      const int chunk = kPaired ? (t.sub < 2 ? t.sub + 2 * q : 6 + q) : t.sub + q * ugemm::kSubs;
      const int c0 = 32 * chunk;
      if (c0 >= t.n_valid) continue;
      const int ncols = min(32, t.n_valid - c0);
      const int n = t.n0 + c0;
      const int which = n / hd, col = n - which * hd;
      const bool rot = rotate && which < 2;
      if (rot) {
        const int p0 = (col % dh) / 2;
        if (p0 != cached) {  // angle loads issued before the accumulator read, so their latency overlaps it
          const float* cp = cos_t + (int64_t)p0 * seq + pos;
          const float* sp = sin_t + (int64_t)p0 * seq + pos;
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            cc[u] = cp[(int64_t)u * seq];
            sn[u] = sp[(int64_t)u * seq];
          }
          cached = p0;
        }
      }
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
      if (rot) {
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const float e = round_to<T>(v[2 * u]), od = round_to<T>(v[2 * u + 1]);
          v[2 * u] = e * cc[u] - od * sn[u];
          v[2 * u + 1] = od * cc[u] + e * sn[u];
        }
      }
      if (use_tma) {
        ugemm::warp_tma_store<T>(t, v, &maps[which], col, t.row0);
        continue;
      }
      T* base = which == 0 ? plane[0] : (which == 1 ? plane[1] : plane[2]);
      if (inner == 1) {
        ugemm::warp_store<T>(t.stage, v, base + (int64_t)t.row0 * hd + col, hd, t.rows_valid, ncols);
      } else {
        T* row = t.row_valid ? base + prow * hd + col : nullptr;
        ugemm::warp_store_rows<T>(t.stage, v, row, ncols);
      }
    }
  }
};

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_qkv_linear_rotary_forward(const void* x, const void* weight, const float* cos_t,
                                             const float* sin_t, int64_t batch, int64_t seq_len, int64_t dim,
                                             int64_t heads, int64_t dim_head, void* q, void* k, void* v,
                                             int rotate_qk, int dtype, int64_t seq_inner, void* stream) {
  clear_error();
  const char* name = "pmb_qkv_linear_rotary_forward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  PMB_REQUIRE(batch >= 0 && seq_len >= 0 && dim > 0 && heads > 0 && dim_head > 0, "%s: bad shape", name);
  PMB_REQUIRE(dim_head % 32 == 0, "%s: dim_head must be a multiple of 32", name);
  PMB_REQUIRE(dim % 8 == 0, "%s: dim must be a multiple of 8", name);
  const int64_t rows = batch * seq_len;
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(rows < (1ll << 31) && 3 * heads * dim_head < (1ll << 31), "%s: too large", name);
  PMB_REQUIRE(x && weight && q && k && v && (!rotate_qk || (cos_t && sin_t)), "%s: NULL tensor argument", name);
  PMB_REQUIRE(seq_inner > 0 && batch % seq_inner == 0, "%s: batch must be a multiple of seq_inner", name);
  const int64_t n = 3 * heads * dim_head;
  const int bn = dense::pick_bn(n);
  CUtensorMap ma, mb;
  int st = dense::make_maps(ma, mb, x, dim, false, weight, dim, false, rows, n, dim, bn, dtype, name);
  if (st) return st;
  ugemm::Plan plan;
  plan.num_groups = 1;
  plan.g[0] = ugemm::Group{(int)rows, (int)n, (int)dim, 0, 0, 0, 0, 0, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fp16 = dtype == PMB_FLOAT16;
  auto run = [&](auto tag) {
    using T = decltype(tag);
    QkvRotaryEpi<T> epi{{static_cast<T*>(q), static_cast<T*>(k), static_cast<T*>(v)}, cos_t, sin_t,
                        (int)(heads * dim_head), (int)seq_len, (int)dim_head, rotate_qk, (int)seq_inner, 0, {}};
    if (seq_inner == 1 && (heads * dim_head * 2) % 16 == 0) {
      // planes stored by TMA tiles: rows in x order are plane rows when sequences are contiguous
      int ok = 1;
      for (int i = 0; i < 3 && ok; ++i)
        ok = tma::make_store_map_2d(epi.maps[i], epi.plane[i], dtype, (uint64_t)(heads * dim_head), (uint64_t)rows,
                                    (uint64_t)(heads * dim_head * 2), name) == PMB_OK;
      if (ok)
        epi.use_tma = 1;
      else
        clear_error();
    }
    if (bn == 256) return dense::launch<256, false, false>(ma, mb, plan, epi, fp16, s, name);
    if (bn == 128) return dense::launch<128, false, false>(ma, mb, plan, epi, fp16, s, name);
    return dense::launch<64, false, false>(ma, mb, plan, epi, fp16, s, name);
  };
  return fp16 ? run(__half()) : run(__nv_bfloat16());
}
