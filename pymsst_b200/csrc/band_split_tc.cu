// BandSplit on the tcgen05 tensor cores (bf16 / fp16 activations, fp32 or
// 16-bit parameters): per band b of width w_b,
//   s[m, b] = sqrt(w_b) / max(||x_b[m]||, eps)
//   out[m, b, :] = s[m, b] * (x_b[m] (W_b * gamma_b)^T) + bias_b
// which is the reference's (normalise, scale by gamma, Linear) because the
// per-(row, band) norm is a row scale and commutes with the Linear.
// Reference semantics: src/pymsst/training/cuda/fused_band_split.cu:590-1003
// (ragged band split) and :14-247; pure-torch form
// src/pymsst/training/fused_roformer.py:1265-1271.
//
// Input layout.  x [rows, total] is read in place by TMA: its row stride must
// be a multiple of 8 elements (16 bytes) -- the band gather writes it that
// way -- and each band's k-range starts at its first column rounded down to a
// multiple of 8, so every TMA box starts 16-byte aligned whatever the band
// offsets.  Columns of the box outside the band (the rounding lead, and the
// rest of the last 64-wide k-block) belong to neighbouring bands or lie past
// the row end (TMA fills those with zeros); the packed weight holds zeros at
// those k positions, so they contribute nothing.
//
// Weight groups.  Consecutive bands whose columns fit in one 64-wide k-block
// (the 8- and 16-feature bands of BS-RoFormer) form one group: one A tile
// x[:, a_g : a_g + 64] feeds all of them, the packed weight of the group is
// block-diagonal [n_bands * O, 64], and the group's output columns are
// consecutive columns of out[m, :, :] (bands are adjacent there).  Wider bands
// are groups of one band with K = their k-range rounded up to 64.
//
// Forward (two launches): a prep kernel whose first CTAs compute s[m, b]
// (row staged as 4-element vectors, per-chunk sums of squares reduced per
// band in a fixed order) and whose remaining CTAs pack W_b * gamma_b into the
// grouped weight matrix; then one persistent grouped GEMM (group = weight
// group, M = rows, N = n_bands * O, K = 64-multiple) whose epilogue scales
// each row by s[m, b], adds the bias and writes out [rows, nb, O].
//
// Backward (the parameter side; BandSplit's input is the STFT, which carries
// no gradient in training): a prep kernel writes normed = x * s (same strided
// layout, in the workspace) and per-64-row column partials of dY (bias
// gradient); one grouped GEMM per band, G_b = dY_b^T normed_b (M = O,
// N = the band's k-range, K = rows, both operands MN-major), whose epilogue
// writes grad_W_b = G_b * gamma_b and per-32-row partials of
// sum_o W_b[o, i] G_b[o, i] (= grad_gamma_b); a finalize kernel sums both
// partial sets.  Every sum runs in a fixed order (deterministic).
#include <vector>

#include "gemm_umma.cuh"
#include "reduce.cuh"
#include "tma.cuh"

namespace pmb {
unsigned int timeout_flag_band(int reset) { return umma::flag_reader(reset); }

namespace {

constexpr int kThreads = 256;
constexpr int kRowAlign = 8;     // x row stride alignment in elements (16 bytes)
constexpr int kMaxGroupBands = 8;
constexpr int kMaxGroupN = 1536;
constexpr int kBiasRows = 32;  // rows per bias-gradient partial sum
inline int bias_chunks(int64_t rows) { return (int)((rows + kBiasRows - 1) / kBiasRows); }

struct Layout {
  int nb, ng, O, total, kpmax, n_total;
  int w[kMaxBands];        // band widths
  int off[kMaxBands];      // first feature column of each band
  int first[kMaxBands + 1];  // group g covers bands [first[g], first[g + 1])
  int a[kMaxBands];        // first column of group g's k-range (multiple of 8)
  int kp[kMaxBands];       // k extent of group g (multiple of 64)
  int row[kMaxBands + 1];  // first row of group g in the packed weight [n_total, kpmax]
  int gof[kMaxBands];           // weight group of band b
  int pack_cta[kMaxBands + 1];  // first packing CTA of band b (a CTA packs up to 8 k-chunks of 8 columns)
};

Layout make_layout(int nb, const int64_t* widths, int O) {
  Layout L;
  L.nb = nb;
  L.O = O;
  int off = 0;
  for (int b = 0; b < nb; ++b) {
    L.w[b] = (int)widths[b];
    L.off[b] = off;
    off += L.w[b];
  }
  L.total = off;
  L.ng = 0;
  L.kpmax = 64;
  int rows = 0;
  for (int b = 0; b < nb;) {
    const int a = L.off[b] & ~(kRowAlign - 1);
    int e = b + 1;
    int end = L.off[b] + L.w[b];
    while (e < nb && L.off[e] + L.w[e] - a <= 64 && e - b < kMaxGroupBands && (e - b + 1) * O <= kMaxGroupN) {
      end = L.off[e] + L.w[e];
      ++e;
    }
    const int g = L.ng++;
    L.first[g] = b;
    L.a[g] = a;
    L.kp[g] = (end - a + 63) / 64 * 64;
    L.row[g] = rows;
    rows += (e - b) * O;
    if (L.kp[g] > L.kpmax) L.kpmax = L.kp[g];
    b = e;
  }
  L.first[L.ng] = nb;
  L.row[L.ng] = rows;
  L.n_total = rows;
  L.pack_cta[0] = 0;
  for (int g = 0; g < L.ng; ++g)
    for (int b = L.first[g]; b < L.first[g + 1]; ++b) {
      L.gof[b] = g;
      L.pack_cta[b + 1] = L.pack_cta[b] + (L.kp[g] / 8 + 7) / 8;
    }
  return L;
}

// Elements per vector of the row passes: the largest of 4 / 2 / 1 that
// divides every band offset and width (so no vector straddles two bands).
int chunk_elems(const Layout& L) {
  int g = 4;
  for (int b = 0; b < L.nb; ++b)
    while (g > 1 && ((L.off[b] % g) || (L.w[b] % g))) g >>= 1;
  return g;
}

template <typename T, int CH>
struct Vec;
template <typename T>
struct Vec<T, 4> {
  using U = uint2;
};
template <typename T>
struct Vec<T, 2> {
  using U = uint32_t;
};
template <typename T>
struct Vec<T, 1> {
  using U = uint16_t;
};

// ------------------------------------------------------------- forward prep
// CTAs [0, row_ctas): s for blocks of kPrepRows rows r0 = kPrepRows * blockIdx.x, + kPrepRows * row_ctas, ...
// CTAs [row_ctas, ...): packed[row_g + n, k] = W_b[o, i] * gamma_b[i] (or 0)
// for 8 consecutive k per thread.
// Rows go kPrepRows at a time: every thread's loads of all of them are in
// flight together, and one pass of the per-band warp reductions serves all of
// them (a lane sums the band's chunk partials of every row, the warp reduces
// them in a fixed order, and lanes 0..kPrepRows-1 finish one row each), so
// the reduction overhead and the final reciprocal square roots are shared.
constexpr int kPrepRows = 4;

template <typename T, typename TP, int CH>
__global__ void __launch_bounds__(kThreads)
    bs_prep_forward(const T* __restrict__ x, int64_t rows, int64_t ld, int row_ctas, BandTable tab, Layout L,
                 float* __restrict__ scale_out, T* __restrict__ packed) {
  extern __shared__ float chunk_ss[];  // [kPrepRows][total / CH]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if ((int)blockIdx.x < row_ctas) {
    using U = typename Vec<T, CH>::U;
    const int nchunks = L.total / CH;
    for (int64_t r0 = (int64_t)blockIdx.x * kPrepRows; r0 < rows; r0 += (int64_t)row_ctas * kPrepRows) {
      const int nr = rows - r0 < kPrepRows ? (int)(rows - r0) : kPrepRows;
      for (int c = threadIdx.x; c < nchunks; c += kThreads) {
        U u[kPrepRows];
#pragma unroll
        for (int i = 0; i < kPrepRows; ++i)
          if (i < nr) u[i] = reinterpret_cast<const U*>(x + (r0 + i) * ld)[c];
#pragma unroll
        for (int i = 0; i < kPrepRows; ++i) {
          float ss = 0.f;
          if (i < nr) {
            const T* e = reinterpret_cast<const T*>(&u[i]);
#pragma unroll
            for (int j = 0; j < CH; ++j) {
              const float v = Elem<T>::to_f(e[j]);
              ss = fmaf(v, v, ss);
            }
          }
          chunk_ss[i * nchunks + c] = ss;
        }
      }
      __syncthreads();
      for (int b = warp; b < L.nb; b += kThreads / 32) {
        const int c0 = L.off[b] / CH, c1 = (L.off[b] + L.w[b]) / CH;
        float ss[kPrepRows];
#pragma unroll
        for (int i = 0; i < kPrepRows; ++i) ss[i] = 0.f;
        for (int c = c0 + lane; c < c1; c += 32)
#pragma unroll
          for (int i = 0; i < kPrepRows; ++i) ss[i] += chunk_ss[i * nchunks + c];
        float mine = 0.f;  // lane i ends with row i's band sum
#pragma unroll
        for (int i = 0; i < kPrepRows; ++i) {
          const float t = warp_sum(ss[i]);
          if (lane == i) mine = t;
        }
        // 1 / max(||x||, 1e-12) as min(rsqrt(ss), 1e12) (rsqrt(0) = inf)
        if (lane < nr) scale_out[(r0 + lane) * L.nb + b] = fminf(rsqrtf(mine), 1.0e12f);
      }
      __syncthreads();
    }
    return;
  }
  // packing: CTA = (band b, up to 8 consecutive 8-column k-chunks of its group's k-range); thread = (chunk,
  // one of 32 row lanes) over the band's O weight rows, so a warp reads four 8-column W row segments and
  // writes four 16-byte-aligned 128-byte packed row segments
  const int cta = (int)blockIdx.x - row_ctas;
  int lo = 0, hi = L.nb - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (L.pack_cta[mid] <= cta) lo = mid; else hi = mid - 1;
  }
  const int b = lo, g = L.gof[b];
  const int c = (cta - L.pack_cta[b]) * 8 + (threadIdx.x & 7);
  if (c >= L.kp[g] / 8) return;
  const int wb = L.w[b];
  const int i0 = L.a[g] + 8 * c - L.off[b];  // band feature of this chunk's first column
  const TP* Wb = static_cast<const TP*>(tab.ptr1[b]);
  const TP* gm = static_cast<const TP*>(tab.ptr0[b]);
  T* dst = packed + (int64_t)(L.row[g] + (b - L.first[g]) * L.O) * L.kpmax + 8 * c;
  float gv[8];
  unsigned inb = 0;  // bit j: column j of the chunk is a feature of band b
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const bool in = i0 + j >= 0 && i0 + j < wb;
    inb |= (unsigned)in << j;
    gv[j] = in ? Elem<TP>::to_f(gm[i0 + j]) : 0.f;
  }
  for (int o = threadIdx.x >> 3; o < L.O; o += kThreads / 8) {
    const TP* Wr = Wb + (int64_t)o * wb;
    alignas(16) T vals[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      vals[j] = Elem<T>::from_f((inb >> j) & 1u ? Elem<TP>::to_f(Wr[i0 + j]) * gv[j] : 0.f);
    *reinterpret_cast<uint4*>(dst + (int64_t)o * L.kpmax) = *reinterpret_cast<const uint4*>(vals);
  }
}

// out[m, b, o] = s[m, b] * sqrt(w_b) * acc + bias_b[o] for the group's bands (one band per 32-column chunk).
template <typename T, typename TP>
struct BandOutEpi {
  T* out;
  const float* inv;
  int nb, O;
  int use_tma;          // out stored by TMA tiles through out_map ([rows, nb * O])
  CUtensorMap out_map;
  int first[kMaxBands];
  float sqrt_w[kMaxBands];
  const void* bias[kMaxBands];
  // row scale and bias of every chunk a warp drains (BN <= 256: at most 3 chunks per warp), loaded by the
  // engine one tile ahead (prefetch), so their latency is hidden behind the previous tile's epilogue
  static constexpr int kMaxChunks = (256 / 32 + ugemm::kSubs - 1) / ugemm::kSubs;
  struct Pre {
    float sc[kMaxChunks], bl[kMaxChunks];
  };
  __device__ void prefetch(const ugemm::Plan&, const ugemm::TileCtx& t, Pre& p) const {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int q = 0; q < kMaxChunks; ++q) {
      const int c0 = 32 * (t.sub + q * ugemm::kSubs);
      p.sc[q] = p.bl[q] = 0.f;
      if (c0 < t.n_valid) {
        const int n = t.n0 + c0;
        const int b = first[t.group] + n / O, o0 = n % O;
        const TP* bp = static_cast<const TP*>(bias[b]);
        p.sc[q] = t.row_valid ? inv[(int64_t)t.row * nb + b] * sqrt_w[b] : 0.f;
        p.bl[q] = (bp != nullptr && lane < t.n_valid - c0) ? Elem<TP>::to_f(bp[o0 + lane]) : 0.f;
      }
    }
  }
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t, const Pre& p) const {
    static_assert(BN <= 256, "at most kMaxChunks chunks per warp");
    const int64_t ld = (int64_t)nb * O;
    const float* sc = p.sc;
    const float* bl = p.bl;
#pragma unroll
    for (int q = 0; q < kMaxChunks; ++q) {
      const int c0 = 32 * (t.sub + q * ugemm::kSubs);
      if (c0 >= BN || c0 >= t.n_valid) break;
      const int ncols = min(32, t.n_valid - c0);
      const int n = t.n0 + c0;
      const int b = first[t.group] + n / O, o0 = n % O;
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fmaf(v[j], sc[q], __shfl_sync(0xffffffffu, bl[q], j));
      if (use_tma) {  // O is a multiple of 64: each 32-column chunk lies inside one band
        ugemm::warp_tma_store<T>(t, v, &out_map, b * O + o0, t.row0);
        continue;
      }
      ugemm::warp_store<T>(t.stage, v, out + (int64_t)t.row0 * ld + (int64_t)b * O + o0, ld, t.rows_valid, ncols);
    }
  }
};

// ------------------------------------------------------------ backward prep
// CTAs [0, row_ctas): normed[r, c] = x[r, c] * s[r, band(c)] * sqrt(w_band) for the band columns, kPrepRows
// rows per pass (all of their loads in flight together, one barrier pair per pass).
// CTAs [row_ctas, ...): bias partials bpart[chunk][col] = sum over the chunk's kBiasRows rows of dY[r, col],
// eight adjacent columns per thread (16-byte loads), eight rows in flight.
template <typename T, int CH>
__global__ void __launch_bounds__(kThreads)
    bs_prep_backward(const T* __restrict__ x, int64_t rows, int64_t ld, const float* __restrict__ inv, Layout L,
                  int row_ctas, T* __restrict__ normed, int64_t nld, const T* __restrict__ dy, int64_t cols,
                  float* __restrict__ bpart) {
  extern __shared__ float sc_s[];  // [kPrepRows][nb] scales of the pass's rows, then the chunk -> band map
  if ((int)blockIdx.x < row_ctas) {
    using U = typename Vec<T, CH>::U;
    const int nchunks = L.total / CH;
    int* band_of_chunk = reinterpret_cast<int*>(sc_s + kPrepRows * L.nb);
    for (int c = threadIdx.x; c < nchunks; c += kThreads) {
      int lo = 0, hi = L.nb - 1;
      const int col = c * CH;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (L.off[mid] <= col) lo = mid; else hi = mid - 1;
      }
      band_of_chunk[c] = lo;
    }
    for (int64_t r0 = (int64_t)blockIdx.x * kPrepRows; r0 < rows; r0 += (int64_t)row_ctas * kPrepRows) {
      const int nr = rows - r0 < kPrepRows ? (int)(rows - r0) : kPrepRows;
      __syncthreads();
      for (int k = threadIdx.x; k < nr * L.nb; k += kThreads) {
        const int i = k / L.nb, b = k - i * L.nb;
        sc_s[k] = inv[(r0 + i) * L.nb + b] * sqrtf((float)L.w[b]);
      }
      __syncthreads();
      for (int c = threadIdx.x; c < nchunks; c += kThreads) {
        U u[kPrepRows];
#pragma unroll
        for (int i = 0; i < kPrepRows; ++i)
          if (i < nr) u[i] = reinterpret_cast<const U*>(x + (r0 + i) * ld)[c];
        const int b = band_of_chunk[c];
#pragma unroll
        for (int i = 0; i < kPrepRows; ++i) {
          if (i >= nr) break;
          T* e = reinterpret_cast<T*>(&u[i]);
          const float sc = sc_s[i * L.nb + b];
#pragma unroll
          for (int j = 0; j < CH; ++j) e[j] = Elem<T>::from_f(Elem<T>::to_f(e[j]) * sc);
          reinterpret_cast<U*>(normed + (r0 + i) * nld)[c] = u[i];
        }
      }
    }
    return;
  }
  const int64_t bid = (int64_t)blockIdx.x - row_ctas;
  const int64_t col_blocks = (cols / 8 + kThreads - 1) / kThreads;
  const int64_t chunk = bid / col_blocks;
  const int64_t c = ((bid % col_blocks) * kThreads + threadIdx.x) * 8;
  if (c >= cols) return;
  const int64_t r0 = chunk * kBiasRows;
  const int64_t r1 = r0 + kBiasRows < rows ? r0 + kBiasRows : rows;
  float s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = 0.f;
  int64_t r = r0;
  for (; r + 8 <= r1; r += 8) {
    uint4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = *reinterpret_cast<const uint4*>(dy + (r + k) * cols + c);
    // rows summed pairwise in a fixed order
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float t[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) t[k] = Elem<T>::to_f(reinterpret_cast<const T*>(&v[k])[j]);
      s[j] += ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
    }
  }
  for (; r < r1; ++r) {
    const uint4 v = *reinterpret_cast<const uint4*>(dy + r * cols + c);
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] += Elem<T>::to_f(reinterpret_cast<const T*>(&v)[j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) bpart[chunk * cols + c + j] = s[j];
}

// G tile (rows o of O, columns n of band b's k-range, feature i = n - lead_b):
//   grad_W_b[o, i] = G[o, n] * gamma_b[i]              (0 <= i < w_b)
//   gpart[row0 / 32][off_b + i] = sum over this warp's 32 rows of W_b[o, i] * G[o, n]
template <typename TP>
struct WGradBandEpi {
  int w[kMaxBands], lead[kMaxBands], off[kMaxBands];
  int total;
  const void* gamma[kMaxBands];
  const void* weight[kMaxBands];
  void* grad_w[kMaxBands];
  float* gpart;
  template <int BN>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    const int lane = threadIdx.x & 31;
    const int b = t.group;
    const int wb = w[b], ld = lead[b];
    const TP* gm = static_cast<const TP*>(gamma[b]);
    const TP* W = static_cast<const TP*>(weight[b]);
    TP* gW = static_cast<TP*>(grad_w[b]);
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BN; c0 += 32 * ugemm::kSubs) {
      const int i0 = t.n0 + c0 - ld;  // feature of this chunk's column 0 (may be negative by the lead)
      if (c0 >= t.n_valid || i0 >= wb) break;
      const int i = i0 + lane;
      const bool col_ok = i >= 0 && i < wb;
      {
        // transpose G through the staging block: row r = output o = row0 + r, column lane
        float v[32];
        umma::tmem_ld32(t.taddr + c0, v);
        float* st = reinterpret_cast<float*>(t.stage + lane * ugemm::kStageRowBytes);
#pragma unroll
        for (int j = 0; j < 32; ++j) st[j] = v[j];
      }
      __syncwarp();
      // lane = feature column i: the warp's W rows, 16 loaded together at a time (coalesced along i)
      const float gl = col_ok ? Elem<TP>::to_f(gm[i]) : 0.f;
      float s = 0.f;
#pragma unroll
      for (int h = 0; h < 32; h += 16) {
        float wr[16];
#pragma unroll
        for (int r = 0; r < 16; ++r)
          wr[r] = (col_ok && h + r < t.rows_valid) ? Elem<TP>::to_f(W[(int64_t)(t.row0 + h + r) * wb + i]) : 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const float g = reinterpret_cast<const float*>(t.stage + (h + r) * ugemm::kStageRowBytes)[lane];
          s = fmaf(wr[r], g, s);
          if (col_ok && h + r < t.rows_valid) gW[(int64_t)(t.row0 + h + r) * wb + i] = Elem<TP>::from_f(g * gl);
        }
      }
      if (col_ok && t.rows_valid > 0) gpart[(int64_t)(t.row0 / 32) * total + off[b] + i] = s;
      __syncwarp();
    }
  }
};

// CTAs [0, gamma_ctas): grad_gamma_b[i] = sum_q gpart[q][off_b + i], one column per thread.
// Other CTAs: grad_bias_b[o] = sum over chunks of bpart[chunk][b * O + o]: 32 columns per CTA, eight threads per
// column each summing every eighth chunk, combined in shared memory in a fixed order.
template <typename TP>
__global__ void __launch_bounds__(kThreads)
    bs_finalize(const float* __restrict__ gpart, int nq, const float* __restrict__ bpart, int nchunks, Layout L,
                int gamma_ctas, BandTable gtab, BandTable btab) {
  if ((int)blockIdx.x < gamma_ctas) {
    const int64_t c = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (c >= L.total) return;
    int lo = 0, hi = L.nb - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (L.off[mid] <= c) lo = mid; else hi = mid - 1;
    }
    float s = 0.f;
#pragma unroll 8
    for (int q = 0; q < nq; ++q) s += gpart[(int64_t)q * L.total + c];
    static_cast<TP*>(const_cast<void*>(gtab.ptr0[lo]))[c - L.off[lo]] = Elem<TP>::from_f(s);
    return;
  }
  __shared__ float part[8][33];
  const int64_t cols = (int64_t)L.nb * L.O;
  const int cl = threadIdx.x & 31, pl = threadIdx.x >> 5;
  const int64_t k = ((int64_t)blockIdx.x - gamma_ctas) * 32 + cl;
  float s = 0.f;
  if (k < cols)
    for (int q = pl; q < nchunks; q += 8) s += bpart[(int64_t)q * cols + k];
  part[pl][cl] = s;
  __syncthreads();
  if (pl == 0 && k < cols && btab.ptr0[0] != nullptr) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += part[j][cl];
    const int b = (int)(k / L.O);
    static_cast<TP*>(const_cast<void*>(btab.ptr0[b]))[k - (int64_t)b * L.O] = Elem<TP>::from_f(t);
  }
}

int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }

struct Sizes {
  int64_t packed_bytes, ws_bytes;
  int64_t ws_gpart, ws_bpart;  // offsets of the partial blocks after the normed copy
};

Sizes sizes_of(int64_t rows, const Layout& L, int es) {
  Sizes z;
  z.packed_bytes = align256((int64_t)L.n_total * L.kpmax * es);
  const int64_t ld = (L.total + kRowAlign - 1) / kRowAlign * kRowAlign;
  z.ws_gpart = align256(rows * ld * es);
  z.ws_bpart = z.ws_gpart + align256((int64_t)((L.O + 31) / 32) * L.total * 4);
  z.ws_bytes = z.ws_bpart + align256((int64_t)bias_chunks(rows) * L.nb * L.O * 4);
  return z;
}

template <int BN, bool A_MN, bool B_MN, class Epi>
int run_gemm(const CUtensorMap& ma, const CUtensorMap& mb, ugemm::Plan& plan, const Epi& epi, int fp16,
             cudaStream_t s, const char* name) {
  constexpr int STAGES = 4;
  const int tiles = ugemm::build_plan(plan, BN);
  if (tiles == 0) return PMB_OK;
  auto kern = ugemm::umma_gemm_kernel<BN, STAGES, A_MN, B_MN, Epi>;
  const int smem = ugemm::smem_bytes<BN, STAGES>();
  PMB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), name);
  kern<<<ugemm::persistent_grid(tiles), ugemm::kThreads, smem, s>>>(ma, mb, plan, epi, fp16);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

template <typename T, typename TP, int CH>
int launch_prep_forward(const T* x, int64_t rows, int64_t ld, const BandTable& tab, const Layout& L, float* inv,
                        T* packed, cudaStream_t s, const char* name) {
  const int64_t blocks = (rows + kPrepRows - 1) / kPrepRows;
  const int row_ctas = (int)(blocks < (int64_t)num_sms() * 8 ? blocks : (int64_t)num_sms() * 8);
  const int pack_ctas = L.pack_cta[L.nb];
  const size_t smem = (size_t)kPrepRows * (L.total / CH) * sizeof(float);
  auto kern = bs_prep_forward<T, TP, CH>;
  if (smem > 48 * 1024) PMB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), name);
  kern<<<row_ctas + pack_ctas, kThreads, smem, s>>>(x, rows, ld, row_ctas, tab, L, inv, packed);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

template <typename T, int CH>
int launch_prep_backward(const T* x, int64_t rows, int64_t ld, const float* inv, const Layout& L, T* normed,
                         int64_t nld, const T* dy, float* bpart, cudaStream_t s, const char* name) {
  const int64_t blocks = (rows + kPrepRows - 1) / kPrepRows;
  const int row_ctas = (int)(blocks < (int64_t)num_sms() * 8 ? blocks : (int64_t)num_sms() * 8);
  const int64_t cols = (int64_t)L.nb * L.O;  // a multiple of 64 (O is)
  const int64_t bias_ctas = bpart ? ((cols / 8 + kThreads - 1) / kThreads) * bias_chunks(rows) : 0;
  const size_t smem = (size_t)kPrepRows * L.nb * sizeof(float) + (size_t)(L.total / CH) * sizeof(int);
  auto kern = bs_prep_backward<T, CH>;
  if (smem > 48 * 1024) PMB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), name);
  kern<<<(unsigned)(row_ctas + bias_ctas), kThreads, smem, s>>>(x, rows, ld, inv, L, row_ctas, normed, nld, dy, cols,
                                                                 bpart);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_band_split_tc_sizes(int64_t rows, int num_bands, const int64_t* widths, int64_t out_features,
                                       int dtype, int64_t* sizes) {
  clear_error();
  PMB_REQUIRE(num_bands > 0 && num_bands <= kMaxBands && widths && sizes && rows >= 0 && out_features > 0 &&
                  out_features % 64 == 0 && out_features <= 4096,
              "pmb_band_split_tc_sizes: bad arguments (out_features must be a positive multiple of 64)");
  for (int b = 0; b < num_bands; ++b) PMB_REQUIRE(widths[b] > 0, "pmb_band_split_tc_sizes: band %d is empty", b);
  const Layout L = make_layout(num_bands, widths, (int)out_features);
  const Sizes z = sizes_of(rows, L, dtype_size(dtype) > 0 ? dtype_size(dtype) : 2);
  sizes[0] = z.packed_bytes;
  sizes[1] = z.ws_bytes;
  sizes[2] = kRowAlign;
  sizes[3] = L.ng;
  return PMB_OK;
}

extern "C" int pmb_band_split_tc_forward(const void* x, int64_t rows, int64_t x_ld, int num_bands,
                                         const int64_t* widths, const void* const* gammas,
                                         const void* const* weights, const void* const* biases, int64_t out_features,
                                         void* packed_weights, float* inv_norm, void* out, int dtype, int param_dtype,
                                         void* stream) {
  clear_error();
  const char* name = "pmb_band_split_tc_forward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  BandTable tab;
  int st = make_band_table(tab, num_bands, widths, gammas, weights, biases, name);
  if (st) return st;
  PMB_REQUIRE(rows >= 0 && rows < (1ll << 31) && out_features > 0 && out_features % 64 == 0 && out_features <= 4096,
              "%s: bad shape (out_features must be a positive multiple of 64)", name);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(x && out && inv_norm && packed_weights, "%s: NULL tensor argument", name);
  for (int b = 0; b < num_bands; ++b)
    PMB_REQUIRE(tab.ptr0[b] && tab.ptr1[b], "%s: band %d has a NULL gamma or weight", name, b);
  const Layout L = make_layout(num_bands, widths, (int)out_features);
  if (x_ld < L.total || x_ld % kRowAlign != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(packed_weights) & 15) != 0) {
    set_error("%s: x needs a 16-byte aligned base and a row stride that is a multiple of %d elements and at least "
              "%d (got %lld)", name, kRowAlign, L.total, (long long)x_ld);
    return PMB_ERR_ALIGNMENT;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fp16 = dtype == PMB_FLOAT16;
  const int ch = chunk_elems(L);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 4) {
      set_error("%s: fp32 activations are not supported", name);
      return PMB_ERR_UNSUPPORTED_DTYPE;
    } else {
      const T* xt = static_cast<const T*>(x);
      T* pk = static_cast<T*>(packed_weights);
      int st2 = ch == 4   ? launch_prep_forward<T, TP, 4>(xt, rows, x_ld, tab, L, inv_norm, pk, s, name)
                : ch == 2 ? launch_prep_forward<T, TP, 2>(xt, rows, x_ld, tab, L, inv_norm, pk, s, name)
                          : launch_prep_forward<T, TP, 1>(xt, rows, x_ld, tab, L, inv_norm, pk, s, name);
      if (st2) return st2;
      CUtensorMap ma, mb;
      constexpr int BN = 192;
      st2 = tma::make_map_3d(ma, x, dtype, L.total, 1, rows, x_ld * 2, x_ld * 2, 64, 1, ugemm::BM, name);
      if (st2) return st2;
      st2 = tma::make_map_3d(mb, packed_weights, dtype, L.kpmax, 1, L.n_total, (int64_t)L.kpmax * 2,
                             (int64_t)L.kpmax * 2, 64, 1, BN, name);
      if (st2) return st2;
      ugemm::Plan plan;
      plan.num_groups = L.ng;
      BandOutEpi<T, TP> epi;
      epi.out = static_cast<T*>(out);
      epi.inv = inv_norm;
      epi.nb = num_bands;
      epi.O = (int)out_features;
      epi.use_tma = tma::make_store_map_2d(epi.out_map, out, dtype, (uint64_t)(num_bands * out_features),
                                           (uint64_t)rows, (uint64_t)(num_bands * out_features * 2), name) == PMB_OK;
      if (!epi.use_tma) clear_error();
      for (int b = 0; b < num_bands; ++b) {
        epi.sqrt_w[b] = sqrtf((float)L.w[b]);
        epi.bias[b] = biases ? biases[b] : nullptr;
      }
      for (int g = 0; g < L.ng; ++g) {
        epi.first[g] = L.first[g];
        plan.g[g] = ugemm::Group{(int)rows, L.row[g + 1] - L.row[g], L.kp[g], L.a[g], 0, 0, 0, 0, L.row[g]};
      }
      return run_gemm<BN, false, false>(ma, mb, plan, epi, fp16, s, name);
    }
  });
}

extern "C" int pmb_band_split_tc_backward(const void* grad_out, const void* x, int64_t x_ld, const float* inv_norm,
                                          int64_t rows, int num_bands, const int64_t* widths,
                                          const void* const* gammas, const void* const* weights,
                                          int64_t out_features, void* const* grad_gammas, void* const* grad_weights,
                                          void* const* grad_biases, int dtype, int param_dtype, void* workspace,
                                          int64_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "pmb_band_split_tc_backward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  BandTable wtab, gtab, btab;
  int st = make_band_table(wtab, num_bands, widths, gammas, weights, (const void* const*)grad_weights, name);
  if (st) return st;
  st = make_band_table(gtab, num_bands, widths, (const void* const*)grad_gammas, nullptr, nullptr, name);
  if (st) return st;
  PMB_REQUIRE(rows > 0 && rows < (1ll << 31) && out_features > 0 && out_features % 64 == 0 && out_features <= 4096,
              "%s: bad shape", name);
  PMB_REQUIRE(grad_out && x && inv_norm && grad_gammas && grad_weights && gammas && weights,
              "%s: NULL tensor argument", name);
  for (int b = 0; b < num_bands; ++b)
    PMB_REQUIRE(wtab.ptr0[b] && wtab.ptr1[b] && wtab.ptr2[b] && gtab.ptr0[b] && (!grad_biases || grad_biases[b]),
                "%s: band %d has a NULL parameter or gradient pointer", name, b);
  {
    std::vector<int64_t> ow(num_bands, out_features);
    st = make_band_table(btab, num_bands, ow.data(), (const void* const*)grad_biases, nullptr, nullptr, name);
    if (st) return st;
    if (!grad_biases) btab.ptr0[0] = nullptr;
  }
  const Layout L = make_layout(num_bands, widths, (int)out_features);
  if (x_ld < L.total || x_ld % kRowAlign != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(grad_out) & 15) != 0) {
    set_error("%s: x and grad_out need 16-byte aligned bases and x a row stride that is a multiple of %d "
              "elements (got %lld)", name, kRowAlign, (long long)x_ld);
    return PMB_ERR_ALIGNMENT;
  }
  const Sizes z = sizes_of(rows, L, dtype_size(dtype));
  if (workspace == nullptr || workspace_bytes < z.ws_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required (or not 256-byte aligned)", name,
              (long long)workspace_bytes, (long long)z.ws_bytes);
    return PMB_ERR_WORKSPACE;
  }
  // row stride of the normed copy in the workspace
  const int64_t nld = (L.total + kRowAlign - 1) / kRowAlign * kRowAlign;
  float* gpart = reinterpret_cast<float*>(static_cast<char*>(workspace) + z.ws_gpart);
  float* bpart = reinterpret_cast<float*>(static_cast<char*>(workspace) + z.ws_bpart);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int fp16 = dtype == PMB_FLOAT16;
  const int ch = chunk_elems(L);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 4) {
      set_error("%s: fp32 activations are not supported", name);
      return PMB_ERR_UNSUPPORTED_DTYPE;
    } else {
      const T* xt = static_cast<const T*>(x);
      T* normed = static_cast<T*>(workspace);
      const T* dy = static_cast<const T*>(grad_out);
      float* bp = grad_biases ? bpart : nullptr;
      int st2 = ch == 4   ? launch_prep_backward<T, 4>(xt, rows, x_ld, inv_norm, L, normed, nld, dy, bp, s, name)
                : ch == 2 ? launch_prep_backward<T, 2>(xt, rows, x_ld, inv_norm, L, normed, nld, dy, bp, s, name)
                          : launch_prep_backward<T, 1>(xt, rows, x_ld, inv_norm, L, normed, nld, dy, bp, s, name);
      if (st2) return st2;
      // G_b = dY_b^T normed_b: A(m = o, k = r) = dY[r, b, o], B(n, k = r) = normed[r, a_b + n]
      constexpr int BN = 128;
      CUtensorMap ma, mb;
      st2 = tma::make_map_3d(ma, grad_out, dtype, out_features, num_bands, rows, out_features * 2,
                             (int64_t)num_bands * out_features * 2, 64, 1, 64, name);
      if (st2) return st2;
      st2 = tma::make_map_3d(mb, normed, dtype, L.total, 1, rows, nld * 2, nld * 2, 64, 1, 64, name);
      if (st2) return st2;
      ugemm::Plan plan;
      plan.num_groups = num_bands;
      WGradBandEpi<TP> epi;
      epi.total = L.total;
      epi.gpart = gpart;
      for (int b = 0; b < num_bands; ++b) {
        const int a = L.off[b] & ~(kRowAlign - 1);
        epi.w[b] = L.w[b];
        epi.lead[b] = L.off[b] - a;
        epi.off[b] = L.off[b];
        plan.g[b] = ugemm::Group{(int)out_features, L.off[b] - a + L.w[b], (int)rows, 0, b, 0, a, 0, 0};
        epi.gamma[b] = gammas[b];
        epi.weight[b] = weights[b];
        epi.grad_w[b] = grad_weights[b];
      }
      st2 = run_gemm<BN, true, true>(ma, mb, plan, epi, fp16, s, name);
      if (st2) return st2;
      const int gamma_ctas = (L.total + kThreads - 1) / kThreads;
      const int64_t bias_ctas = grad_biases ? ((int64_t)num_bands * out_features + 31) / 32 : 0;
      bs_finalize<TP><<<(unsigned)(gamma_ctas + bias_ctas), kThreads, 0, s>>>(
          gpart, (int)((out_features + 31) / 32), bpart, bias_chunks(rows), L, gamma_ctas, gtab, btab);
      PMB_CHECK_LAUNCH(name);
      return PMB_OK;
    }
  });
}
