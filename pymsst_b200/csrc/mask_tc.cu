// MaskEstimator per-band MLP on the tcgen05 tensor cores (bf16 / fp16).
//
// Forward, per band b (rows = batch*frames, D -> H hidden -> 2*w_b):
//   h_1 = tanh(x_b W1_b^T + b1_b), ..., pre = h_L Wf_b^T + bf_b,
//   out_b = pre_left * sigmoid(pre_gate)
// Backward: GLU derivative (+ bias sums), dH = gp Wf_b with the tanh
// derivative fused into the GEMM epilogue, dWf_b = gp^T h_L, and the same
// pair of GEMMs for every hidden layer.  All GEMMs run on the grouped
// tcgen05 engine (gemm_umma.cuh); one launch covers all bands.
//
// Packed final layout P: band b owns P_b = 128 * ceil(w_b / 64) rows of the
// packed final weight (and columns of `pre` / grad_pre); its 64-output chunk
// c occupies rows [128c, 128c + 128): 64 left-half rows (outputs 64c..64c+63),
// then the 64 matching gate-half rows, zero-filled past w_b.  A 128-column
// output tile therefore holds a left value and its gate in the same thread,
// so GLU is an epilogue.  fp32 master weights are packed / cast to bf16 once
// per forward (one launch per layer) and reused by the backward.
// Reference semantics: src/pymsst/training/cuda/fused_band_split.cu:1006-1074,
// :2284-2367, :2516-2851; fused_roformer.py:527-583.
#include <algorithm>
#include <vector>

#include "gemm_umma.cuh"
#include "tma.cuh"

namespace pmb {
unsigned int timeout_flag_mask(int reset) { return umma::flag_reader(reset); }

namespace {

constexpr int kThreads = 256;
constexpr int BN = 128;
constexpr int STAGES = 4;
constexpr int kChunk = 64;  // GLU outputs per 128-column tile
constexpr int kGluRows = 4;    // rows per GLU-backward thread
constexpr int kPartRows = 32;  // rows per partial row of the bias-gradient column sums (GLU and hidden layers)
inline int part_chunks(int64_t rows) { return (int)((rows + kPartRows - 1) / kPartRows); }

struct BandInfo {
  int nb;
  int w[kMaxBands];      // outputs per GLU half
  int off[kMaxBands];    // output column offset (prefix sum of w)
  int pbase[kMaxBands];  // packed row / column offset
  const void* bias[kMaxBands];   // final-layer biases (2w, param dtype) or hidden biases (H)
  void* grad[kMaxBands];         // per-band fp32 gradient destinations (weights)
};

// 16-bit activations only, so the hardware approximations (MUFU; relative
// error around 2^-11, below the 2^-8 / 2^-11 spacing of bf16 / fp16 results)
// replace the accurate library calls, which made the epilogues issue-bound:
//   tanh: tanh.approx.f32;   sigmoid(v) = 1 / (1 + 2^(-v log2 e)) with
//   ex2.approx and rcp.approx (2^+inf -> rcp 0, 2^-inf -> 1: saturates).
__device__ __forceinline__ float tanh_fast(float v) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ float sigm(float v) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(v * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return r;
}

template <typename T>
__device__ __forceinline__ float ld(const void* p, int64_t i) {
  return Elem<T>::to_f(static_cast<const T*>(p)[i]);
}

// ------------------------------------------------------------- packing
// Pack per-band fp32/bf16 [R_b, C] weights into a bf16 [rows_total, C]
// buffer.  mode 0: grouped (row p = b*R + r).  mode 1: GLU-chunked final
// layout (see file comment).
template <typename TP, typename T>
__global__ void __launch_bounds__(kThreads)
    pack_rows_kernel(BandTable src, BandInfo info, int mode, int64_t rows_total, int64_t cols, T* __restrict__ dst) {
  const int64_t vec = cols / 8;
  const int64_t n = rows_total * vec;
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += (int64_t)gridDim.x * kThreads) {
    const int64_t p = e / vec, cv = e % vec;
    int b, srow;
    if (mode == 0) {
      const int64_t per = rows_total / info.nb;
      b = (int)(p / per);
      srow = (int)(p % per);
    } else {
      int lo = 0, hi = info.nb - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (info.pbase[mid] <= p) lo = mid; else hi = mid - 1;
      }
      b = lo;
      const int q = (int)(p - info.pbase[b]);
      const int c = q / 128, j = q % 128;
      const int l = c * kChunk + (j % kChunk);
      srow = l < info.w[b] ? (j < kChunk ? l : info.w[b] + l) : -1;
    }
    T out[8];
    if (srow < 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) out[i] = Elem<T>::from_f(0.f);
    } else {
      const TP* s = static_cast<const TP*>(src.ptr0[b]) + (int64_t)srow * cols + cv * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) out[i] = Elem<T>::from_f(Elem<TP>::to_f(s[i]));
    }
    *reinterpret_cast<uint4*>(dst + p * cols + cv * 8) = *reinterpret_cast<uint4*>(out);
  }
}

// ----------------------------------------------------------- epilogues
// Hidden layer: out[m, b, n] = tanh(acc + bias_b[n])  (bf16/fp16 activations)
template <typename T, typename TP>
struct TanhEpi {
  T* out;
  int64_t ld;  // nb * H
  int h;
  const void* bias[kMaxBands];
  int use_tma;          // out stored by TMA tiles through out_map ([rows, nb * H])
  CUtensorMap out_map;
  template <int BNT>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    T* o = out + (int64_t)t.row0 * ld + (int64_t)t.group * h + t.n0;
    const TP* bp = static_cast<const TP*>(bias[t.group]) + t.n0;
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BNT; c0 += 32 * ugemm::kSubs) {
      if (c0 >= t.n_valid) break;
      const int ncols = min(32, t.n_valid - c0);
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
      const float bl = lane < ncols ? Elem<TP>::to_f(bp[c0 + lane]) : 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = tanh_fast(v[j] + __shfl_sync(0xffffffffu, bl, j));
      if (use_tma) {  // hidden widths are multiples of 64: chunks are whole
        ugemm::warp_tma_store<T>(t, v, &out_map, t.group * h + t.n0 + c0, t.row0);
        continue;
      }
      ugemm::warp_store<T>(t.stage, v, o + c0, ld, t.rows_valid, ncols);
    }
  }
};

// Final layer: GLU, writes out [rows, total] and packed pre [rows, P].
template <typename T, typename TP>
struct GluEpi {
  T* out;
  T* pre;
  int64_t ld_out, ld_pre;
  BandInfo info;
  template <int BNT>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    const int b = t.group;
    const int w = info.w[b];
    const int c = t.n0 / 128;
    const int cw = min(kChunk, w - c * kChunk);
    const TP* bias = static_cast<const TP*>(info.bias[b]);
    T* o = out + (int64_t)t.row0 * ld_out + info.off[b] + c * kChunk;
    T* p = pre + (int64_t)t.row0 * ld_pre + info.pbase[b] + c * 128;
    const int lane = threadIdx.x & 31;
    {  // this warp's 32-wide half h of the 64-output chunk
      const int h = t.sub;  // GLU pairs columns h*32.. with 64 + h*32..: two warps of a lane quarter
      if (h >= 2 || h * 32 >= cw) return;
      const int ncols = min(32, cw - h * 32);
      float left[32], gate[32];
      umma::tmem_ld32(t.taddr + h * 32, left);
      umma::tmem_ld32(t.taddr + kChunk + h * 32, gate);
      const int l0 = c * kChunk + h * 32;
      const float bl = lane < ncols ? Elem<TP>::to_f(bias[l0 + lane]) : 0.f;
      const float bg = lane < ncols ? Elem<TP>::to_f(bias[w + l0 + lane]) : 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        left[j] += __shfl_sync(0xffffffffu, bl, j);
        gate[j] += __shfl_sync(0xffffffffu, bg, j);
      }
      ugemm::warp_store<T>(t.stage, left, p + h * 32, ld_pre, t.rows_valid, ncols);
      ugemm::warp_store<T>(t.stage, gate, p + kChunk + h * 32, ld_pre, t.rows_valid, ncols);
#pragma unroll
      for (int j = 0; j < 32; ++j) left[j] *= sigm(gate[j]);
      ugemm::warp_store<T>(t.stage, left, o + h * 32, ld_out, t.rows_valid, ncols);
    }
  }
};

// dH epilogue: dst[m, b, n] = acc * (1 - y^2) (tanh derivative with the
// layer output y) or acc (no activation before this layer).  Each lane loads
// its own row of y (64 bytes) before it reads the accumulator, so the load
// overlaps the tensor-memory wait.  With `partial`, the column sums of the
// stored (rounded) values over this warp's 32 rows go to
// partial[row0 / 32][column] -- the next layer's bias gradient without a
// separate pass over dst; the sums come from a transposing butterfly (31
// shuffles leave column l's sum in lane l, fixed order).  Widths are
// multiples of 64, so every 32-column chunk is whole.
template <typename T>
struct DActEpi {
  T* dst;
  const T* y;        // nullable
  float* partial;    // nullable: [ceil(rows / 32), ld] fp32
  int64_t ld;
  int h;
  int use_tma;       // dst stored by TMA tiles through dst_map ([rows, ld])
  CUtensorMap dst_map;
  template <int BNT>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    const int lane = threadIdx.x & 31;
    const int64_t col0 = (int64_t)t.group * h + t.n0;
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BNT; c0 += 32 * ugemm::kSubs) {
      if (c0 >= t.n_valid) break;
      uint4 u[4];
      if (y != nullptr) {
        const uint4* src = reinterpret_cast<const uint4*>(y + (int64_t)t.row * ld + col0 + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) u[q] = t.row_valid ? src[q] : make_uint4(0, 0, 0, 0);
      }
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
      if (y != nullptr) {
        const T* e = reinterpret_cast<const T*>(u);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float yv = Elem<T>::to_f(e[j]);
          v[j] *= 1.0f - yv * yv;
        }
      }
      if (use_tma)
        ugemm::warp_tma_store<T>(t, v, &dst_map, (int)(col0 + c0), t.row0);
      else
        ugemm::warp_store<T>(t.stage, v, dst + (int64_t)t.row0 * ld + col0 + c0, ld, t.rows_valid, 32);
      if (partial != nullptr) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = t.row_valid ? round_to<T>(v[j]) : 0.f;
#pragma unroll
        for (int s = 0; s < 5; ++s) {
          const int off = 16 >> s;
          const bool upper = (lane & off) != 0;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (j < off) {
              const float send = upper ? v[j] : v[j + off];
              const float keep = upper ? v[j + off] : v[j];
              v[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
          }
        }
        if (t.rows_valid > 0) partial[(int64_t)(t.row0 / 32) * ld + col0 + c0 + lane] = v[0];
      }
    }
  }
};

// Weight-gradient epilogue into per-band fp32/param-dtype tensors.
// mode 0: grouped (row m of group b -> grad_b[m, n]); mode 1: packed GLU rows
// (m = 128c + j -> left/gate source row, skipped past w_b).  A warp's 32 rows
// map to 32 consecutive source rows in both modes.
template <typename TP>
struct WGradEpi {
  int mode;
  int cols;
  BandInfo info;
  template <int BNT>
  __device__ void run(const ugemm::Plan&, const ugemm::TileCtx& t) const {
    const int b = t.group;
    int srow0 = t.row0, nrows = t.rows_valid;
    if (mode == 1) {
      const int c = t.row0 / 128, j0 = t.row0 % 128;
      const int l0 = c * kChunk + (j0 % kChunk);
      srow0 = j0 < kChunk ? l0 : info.w[b] + l0;
      nrows = max(0, min(nrows, info.w[b] - l0));
    }
    if (nrows == 0) return;
    TP* g = static_cast<TP*>(info.grad[b]) + (int64_t)srow0 * cols + t.n0;
#pragma unroll 1
    for (int c0 = 32 * t.sub; c0 < BNT; c0 += 32 * ugemm::kSubs) {
      if (c0 >= t.n_valid) break;
      float v[32];
      umma::tmem_ld32(t.taddr + c0, v);
      ugemm::warp_store<TP>(t.stage, v, g + c0, cols, nrows, min(32, t.n_valid - c0));
    }
  }
};

// GLU backward in the packed layout: gp = (g*sig(gate), g*left*sig'(gate)),
// zero in padding slots; plus column partial sums for the bias gradient.
// Thread = 8 consecutive left slots of one 64-output chunk (their gates sit
// 64 columns further) over kGluRows rows: 16-byte loads of left and gate,
// both results stored from the same thread.  CTA = 32 slot groups x 8 row
// groups = 256 left slots x kPartRows rows; its column sums (fixed order over
// the row groups) are one partial row.
__device__ __forceinline__ int band_of_slot(const BandInfo& info, int64_t q) {
  int lo = 0, hi = info.nb - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (info.pbase[mid] / 2 <= q) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    glu_bwd_packed(const T* __restrict__ dy, const T* __restrict__ pre, int64_t rows, int64_t total, int64_t P,
                   BandInfo info, T* __restrict__ gp, float* __restrict__ partial) {
  static_assert(kThreads == 256 && kPartRows == 8 * kGluRows, "CTA = 32 slot groups x 8 row groups");
  __shared__ float sums[8][32][17];
  __shared__ int64_t slot_col[32];
  const int sgi = threadIdx.x & 31, rgi = threadIdx.x >> 5;
  const int64_t q = ((int64_t)blockIdx.x * 32 + sgi) * 8;  // first left slot of this group (slots = P / 2)
  float sl[8], sg[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) sl[j] = sg[j] = 0.f;
  if (q < P / 2) {
    const int b = band_of_slot(info, q);
    const int qq = (int)(q - info.pbase[b] / 2);
    const int c = qq / kChunk, jj = qq % kChunk;
    const int64_t pl = info.pbase[b] + 128 * c + jj;  // left slot column; its gates at pl + kChunk
    const int l0 = c * kChunk + jj;                   // band output of the first slot
    const int nvalid = max(0, min(8, info.w[b] - l0));
    if (rgi == 0) slot_col[sgi] = pl;
    const T* dyb = dy + info.off[b] + l0;
    const int64_t r0 = (int64_t)blockIdx.y * kPartRows + rgi * kGluRows;
    // every row's loads issued before the first use (one memory round trip per thread)
    uint4 a[kGluRows], gt[kGluRows];
    float g[kGluRows][8];
#pragma unroll
    for (int i = 0; i < kGluRows; ++i) {
      const int64_t r = r0 + i;
      const bool ok = r < rows;
      a[i] = ok ? *reinterpret_cast<const uint4*>(pre + r * P + pl) : make_uint4(0, 0, 0, 0);
      gt[i] = ok ? *reinterpret_cast<const uint4*>(pre + r * P + pl + kChunk) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[i][j] = ok && j < nvalid ? Elem<T>::to_f(dyb[r * total + j]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kGluRows; ++i) {
      const int64_t r = r0 + i;
      if (r >= rows) break;
      const T* ea = reinterpret_cast<const T*>(&a[i]);
      const T* eg = reinterpret_cast<const T*>(&gt[i]);
      alignas(16) T ol[8], og[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float s = sigm(Elem<T>::to_f(eg[j]));
        // padding slots (past w) hold arbitrary values: selected away, never multiplied
        const float vl = j < nvalid ? g[i][j] * s : 0.f;
        const float vg = j < nvalid ? g[i][j] * Elem<T>::to_f(ea[j]) * s * (1.0f - s) : 0.f;
        ol[j] = Elem<T>::from_f(vl);
        og[j] = Elem<T>::from_f(vg);
        sl[j] += vl;
        sg[j] += vg;
      }
      *reinterpret_cast<uint4*>(gp + r * P + pl) = *reinterpret_cast<const uint4*>(ol);
      *reinterpret_cast<uint4*>(gp + r * P + pl + kChunk) = *reinterpret_cast<const uint4*>(og);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sums[rgi][sgi][j] = sl[j];
    sums[rgi][sgi][8 + j] = sg[j];
  }
  __syncthreads();
  for (int k = threadIdx.x; k < 32 * 16; k += kThreads) {
    const int s = k / 16, j = k % 16;
    if (((int64_t)blockIdx.x * 32 + s) * 8 >= P / 2) continue;
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) acc += sums[r][s][j];
    partial[(int64_t)blockIdx.y * P + slot_col[s] + (j < 8 ? j : kChunk + j - 8)] = acc;
  }
}

// bias grad: packed column p -> original bias index (left l, gate w + l).
template <typename TP>
__global__ void __launch_bounds__(kThreads)
    glu_bias_finalize(const float* __restrict__ partial, int chunks, int64_t P, BandInfo info, const BandTable gb) {
  const int64_t p = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (p >= P) return;
  int lo = 0, hi = info.nb - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (info.pbase[mid] <= p) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int q = (int)(p - info.pbase[b]);
  const int c = q / 128, j = q % 128;
  const int l = c * kChunk + (j % kChunk);
  if (l >= info.w[b]) return;
  float s = 0.f;
  int k = 0;
  for (; k + 4 <= chunks; k += 4)
    s += (partial[(int64_t)k * P + p] + partial[(int64_t)(k + 1) * P + p]) +
         (partial[(int64_t)(k + 2) * P + p] + partial[(int64_t)(k + 3) * P + p]);
  for (; k < chunks; ++k) s += partial[(int64_t)k * P + p];
  TP* dst = static_cast<TP*>(const_cast<void*>(gb.ptr0[b]));
  dst[j < kChunk ? l : info.w[b] + l] = Elem<TP>::from_f(s);
}

// Column sums of a [rows, nb*H] activation gradient into per-band biases.
template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads)
    grouped_bias_finalize(const float* __restrict__ partial, int chunks, int nb, int h, BandTable gb) {
  const int64_t c = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (c >= (int64_t)nb * h) return;
  const int64_t cols = (int64_t)nb * h;
  float s = 0.f;
  int k = 0;
  for (; k + 4 <= chunks; k += 4)
    s += (partial[(int64_t)k * cols + c] + partial[(int64_t)(k + 1) * cols + c]) +
         (partial[(int64_t)(k + 2) * cols + c] + partial[(int64_t)(k + 3) * cols + c]);
  for (; k < chunks; ++k) s += partial[(int64_t)k * cols + c];
  TP* dst = static_cast<TP*>(const_cast<void*>(gb.ptr0[c / h]));
  dst[c % h] = Elem<TP>::from_f(s);
}

int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }

struct Layout {
  int nb, L;
  int64_t rows, dim, hidden, total, P;
  int64_t packed_final_elems;
  // byte offsets inside the caller's buffers
  int64_t pk_bytes, acts_bytes, pre_bytes, ws_bytes;
  int64_t ws_gp, ws_da, ws_db, ws_partial;
};

Layout make_layout(int64_t rows, int nb, int64_t dim, int64_t hidden, int L, const int64_t* widths, BandInfo* info) {
  Layout y;
  y.nb = nb;
  y.L = L;
  y.rows = rows;
  y.dim = dim;
  y.hidden = hidden;
  int64_t total = 0, P = 0;
  for (int b = 0; b < nb; ++b) {
    if (info) {
      info->w[b] = (int)widths[b];
      info->off[b] = (int)total;
      info->pbase[b] = (int)P;
    }
    total += widths[b];
    P += 128 * ((widths[b] + kChunk - 1) / kChunk);
  }
  if (info) info->nb = nb;
  y.total = total;
  y.P = P;
  const int64_t hin = L > 0 ? hidden : dim;  // input width of the final layer
  int64_t pk = 0;
  for (int l = 0; l < L; ++l) pk += (int64_t)nb * hidden * (l == 0 ? dim : hidden);
  y.packed_final_elems = P * hin;
  y.pk_bytes = align256((pk + y.packed_final_elems) * 2);
  y.acts_bytes = align256((int64_t)L * rows * nb * hidden * 2);
  y.pre_bytes = align256(rows * P * 2);
  const int64_t wide = hidden > dim ? hidden : dim;
  y.ws_gp = 0;
  y.ws_da = align256(rows * P * 2);
  y.ws_db = y.ws_da + align256(rows * nb * wide * 2);
  y.ws_partial = y.ws_db + align256(rows * nb * wide * 2);
  const int64_t partial_floats = (int64_t)part_chunks(rows) * std::max(P, (int64_t)nb * wide);
  y.ws_bytes = y.ws_partial + align256(partial_floats * 4);
  return y;
}

// N tile width per GEMM: 256 where N is the 768-wide hidden layer (A tiles then read 3 rather than 6 times,
// and the epilogue's 8 column chunks spread 3 / 3 / 2 over the warps of a lane quarter), 192 for the
// 192-wide model dimension, 128 for the GLU layer (one 64-output chunk and its gates per tile).
template <int BNT, class Epi, bool A_MN, bool B_MN>
int run_gemm(const CUtensorMap& ma, const CUtensorMap& mb, ugemm::Plan& plan, const Epi& epi, int fp16,
             cudaStream_t s, const char* name) {
  constexpr int NST = BNT >= 256 ? 3 : STAGES;
  const int tiles = ugemm::build_plan(plan, BNT);
  if (tiles == 0) return PMB_OK;
  auto kern = ugemm::umma_gemm_kernel<BNT, NST, A_MN, B_MN, Epi>;
  const int smem = ugemm::smem_bytes<BNT, NST>();
  PMB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), name);
  kern<<<ugemm::persistent_grid(tiles), ugemm::kThreads, smem, s>>>(ma, mb, plan, epi, fp16);
  PMB_CHECK_LAUNCH(name);
  return PMB_OK;
}

int grid_for(int64_t n) {
  int64_t g = (n + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)num_sms() * 32;
  return (int)(g > cap ? cap : (g < 1 ? 1 : g));
}

// ------------------------------------------------------------ forward
template <typename T, typename TP>
int forward_impl(const void* x, const Layout& y, const void* const* weights, const void* const* biases,
                 const int64_t* widths, void* packed, void* acts, void* pre, void* out, int dtype,
                 cudaStream_t s) {
  const char* name = "pmb_mask_estimator_tc_forward";
  BandInfo info;
  make_layout(y.rows, y.nb, y.dim, y.hidden, y.L, widths, &info);
  T* pk = static_cast<T*>(packed);
  const int fp16 = dtype == PMB_FLOAT16;
  const T* in = static_cast<const T*>(x);
  int64_t in_w = y.dim;
  for (int l = 0; l <= y.L; ++l) {
    const bool final = l == y.L;
    const int64_t out_rows = final ? y.P : (int64_t)y.nb * y.hidden;
    BandTable src;
    std::vector<int64_t> ones(y.nb, 1);
    int st = make_band_table(src, y.nb, ones.data(), weights + (int64_t)l * y.nb, nullptr, nullptr, name);
    if (st) return st;
    pack_rows_kernel<TP, T><<<grid_for(out_rows * in_w / 8), kThreads, 0, s>>>(src, info, final ? 1 : 0, out_rows,
                                                                               in_w, pk);
    PMB_CHECK_LAUNCH(name);
    CUtensorMap ma, mb;
    st = tma::make_map_3d(ma, in, dtype, in_w, y.nb, y.rows, in_w * 2, (int64_t)y.nb * in_w * 2, 64, 1, ugemm::BM, name);
    if (st) return st;
    ugemm::Plan plan;
    plan.num_groups = y.nb;
    if (!final) {
      const int hbn = y.hidden % 256 == 0 ? 256 : BN;
      st = tma::make_map_3d(mb, pk, dtype, in_w, y.nb, y.hidden, y.hidden * in_w * 2, in_w * 2, 64, 1, hbn, name);
      if (st) return st;
      // the packed hidden weight is [nb, H, in_w]: mid = band stride H*in_w, outer = row stride in_w
      for (int b = 0; b < y.nb; ++b) plan.g[b] = ugemm::Group{(int)y.rows, (int)y.hidden, (int)in_w, 0, b, 0, 0, b, 0};
      TanhEpi<T, TP> epi;
      epi.out = static_cast<T*>(acts) + (int64_t)l * y.rows * y.nb * y.hidden;
      epi.ld = (int64_t)y.nb * y.hidden;
      epi.h = (int)y.hidden;
      for (int b = 0; b < y.nb; ++b) epi.bias[b] = biases[(int64_t)l * y.nb + b];
      // hidden widths are multiples of 64, so every 32-column chunk lies inside one band: TMA tile stores
      epi.use_tma = tma::make_store_map_2d(epi.out_map, epi.out, dtype, (uint64_t)(y.nb * y.hidden), (uint64_t)y.rows,
                                           (uint64_t)(y.nb * y.hidden * 2), name) == PMB_OK;
      if (!epi.use_tma) clear_error();
      st = hbn == 256 ? run_gemm<256, TanhEpi<T, TP>, false, false>(ma, mb, plan, epi, fp16, s, name)
                      : run_gemm<BN, TanhEpi<T, TP>, false, false>(ma, mb, plan, epi, fp16, s, name);
      if (st) return st;
      in = epi.out;
      pk += (int64_t)y.nb * y.hidden * in_w;
      in_w = y.hidden;
    } else {
      st = tma::make_map_3d(mb, pk, dtype, in_w, 1, y.P, y.P * in_w * 2, in_w * 2, 64, 1, BN, name);
      if (st) return st;
      for (int b = 0; b < y.nb; ++b) {
        const int pb = 128 * (int)((widths[b] + kChunk - 1) / kChunk);
        plan.g[b] = ugemm::Group{(int)y.rows, pb, (int)in_w, 0, b, 0, 0, 0, info.pbase[b]};
      }
      GluEpi<T, TP> epi;
      epi.out = static_cast<T*>(out);
      epi.pre = static_cast<T*>(pre);
      epi.ld_out = y.total;
      epi.ld_pre = y.P;
      epi.info = info;
      for (int b = 0; b < y.nb; ++b) epi.info.bias[b] = biases[(int64_t)l * y.nb + b];
      st = run_gemm<BN, GluEpi<T, TP>, false, false>(ma, mb, plan, epi, fp16, s, name);
      if (st) return st;
    }
  }
  return PMB_OK;
}

// ----------------------------------------------------------- backward
template <typename T, typename TP>
int backward_impl(const void* grad_out, const void* x, const void* acts, const void* pre, const void* packed,
                  const Layout& y, const int64_t* widths, void* const* grad_weights, void* const* grad_biases,
                  void* grad_x, char* ws, int dtype, cudaStream_t s) {
  const char* name = "pmb_mask_estimator_tc_backward";
  BandInfo info;
  make_layout(y.rows, y.nb, y.dim, y.hidden, y.L, widths, &info);
  const int fp16 = dtype == PMB_FLOAT16;
  T* gp = reinterpret_cast<T*>(ws + y.ws_gp);
  T* buf[2] = {reinterpret_cast<T*>(ws + y.ws_da), reinterpret_cast<T*>(ws + y.ws_db)};
  float* partial = reinterpret_cast<float*>(ws + y.ws_partial);
  const int64_t hin = y.L > 0 ? y.hidden : y.dim;
  const T* h_last = y.L > 0 ? static_cast<const T*>(acts) + (int64_t)(y.L - 1) * y.rows * y.nb * y.hidden
                            : static_cast<const T*>(x);
  // packed weights: hidden layers first, then the final layer
  std::vector<const T*> pk_layer(y.L + 1);
  {
    const T* p = static_cast<const T*>(packed);
    for (int l = 0; l < y.L; ++l) {
      pk_layer[l] = p;
      p += (int64_t)y.nb * y.hidden * (l == 0 ? y.dim : y.hidden);
    }
    pk_layer[y.L] = p;
  }
  // 1) GLU backward + final bias gradient
  {
    dim3 g((unsigned)((y.P / 2 + 255) / 256), part_chunks(y.rows));
    glu_bwd_packed<T><<<g, kThreads, 0, s>>>(static_cast<const T*>(grad_out), static_cast<const T*>(pre), y.rows,
                                             y.total, y.P, info, gp, partial);
    PMB_CHECK_LAUNCH(name);
    BandTable gb;
    std::vector<int64_t> ones(y.nb, 1);
    int st = make_band_table(gb, y.nb, ones.data(), (const void* const*)(grad_biases + (int64_t)y.L * y.nb), nullptr,
                             nullptr, name);
    if (st) return st;
    glu_bias_finalize<TP><<<(unsigned)((y.P + kThreads - 1) / kThreads), kThreads, 0, s>>>(
        partial, part_chunks(y.rows), y.P, info, gb);
    PMB_CHECK_LAUNCH(name);
  }
  // 2) final weight gradient: dWf_b = gp_b^T h_b   (M = packed rows, N = hin, K = rows)
  {
    CUtensorMap ma, mb;
    int st = tma::make_map_3d(ma, gp, dtype, y.P, 1, y.rows, y.P * 2, y.P * 2, 64, 1, 64, name);
    if (st) return st;
    st = tma::make_map_3d(mb, h_last, dtype, hin, y.nb, y.rows, hin * 2, (int64_t)y.nb * hin * 2, 64, 1, 64, name);
    if (st) return st;
    ugemm::Plan plan;
    plan.num_groups = y.nb;
    WGradEpi<TP> epi;
    epi.mode = 1;
    epi.cols = (int)hin;
    epi.info = info;
    for (int b = 0; b < y.nb; ++b) {
      const int pb = 128 * (int)((widths[b] + kChunk - 1) / kChunk);
      plan.g[b] = ugemm::Group{pb, (int)hin, (int)y.rows, info.pbase[b], 0, 0, 0, b, 0};
      epi.info.grad[b] = grad_weights[(int64_t)y.L * y.nb + b];
    }
    st = hin % 256 == 0 ? run_gemm<256, WGradEpi<TP>, true, true>(ma, mb, plan, epi, fp16, s, name)
                        : run_gemm<BN, WGradEpi<TP>, true, true>(ma, mb, plan, epi, fp16, s, name);
    if (st) return st;
  }
  // 3) dH = gp_b Wf_b (M = rows, N = hin, K = packed rows), tanh' fused
  const bool need_x = grad_x != nullptr;
  T* dcur = nullptr;
  if (y.L > 0 || need_x) {
    CUtensorMap ma, mb;
    int st = tma::make_map_3d(ma, gp, dtype, y.P, 1, y.rows, y.P * 2, y.P * 2, 64, 1, ugemm::BM, name);
    if (st) return st;
    st = tma::make_map_3d(mb, pk_layer[y.L], dtype, hin, 1, y.P, y.P * hin * 2, hin * 2, 64, 1, 64, name);
    if (st) return st;
    ugemm::Plan plan;
    plan.num_groups = y.nb;
    for (int b = 0; b < y.nb; ++b) {
      const int pb = 128 * (int)((widths[b] + kChunk - 1) / kChunk);
      plan.g[b] = ugemm::Group{(int)y.rows, (int)hin, pb, info.pbase[b], 0, 0, 0, 0, info.pbase[b]};
    }
    DActEpi<T> epi;
    dcur = y.L > 0 ? buf[0] : static_cast<T*>(grad_x);
    epi.dst = dcur;
    epi.y = y.L > 0 ? h_last : nullptr;
    epi.partial = y.L > 0 ? partial : nullptr;  // bias gradient of the last hidden layer
    epi.ld = (int64_t)y.nb * hin;
    epi.h = (int)hin;
    epi.use_tma = tma::make_store_map_2d(epi.dst_map, dcur, dtype, (uint64_t)epi.ld, (uint64_t)y.rows,
                                         (uint64_t)(epi.ld * 2), name) == PMB_OK;
    if (!epi.use_tma) clear_error();
    st = hin % 256 == 0 ? run_gemm<256, DActEpi<T>, false, true>(ma, mb, plan, epi, fp16, s, name)
                        : run_gemm<BN, DActEpi<T>, false, true>(ma, mb, plan, epi, fp16, s, name);
    if (st) return st;
  }
  // 4) hidden layers, last to first: dcur holds d(pre-activation) of layer l
  for (int l = y.L - 1; l >= 0; --l) {
    const int64_t lin = l == 0 ? y.dim : y.hidden;
    const T* lx = l == 0 ? static_cast<const T*>(x) : static_cast<const T*>(acts) + (int64_t)(l - 1) * y.rows * y.nb * y.hidden;
    // bias gradient: column sums of dcur (partial rows written by the epilogue that produced dcur)
    {
      const int64_t cols = (int64_t)y.nb * y.hidden;
      BandTable gb;
      std::vector<int64_t> ones(y.nb, 1);
      int st = make_band_table(gb, y.nb, ones.data(), (const void* const*)(grad_biases + (int64_t)l * y.nb), nullptr,
                               nullptr, name);
      if (st) return st;
      grouped_bias_finalize<T, TP><<<(unsigned)((cols + kThreads - 1) / kThreads), kThreads, 0, s>>>(
          partial, part_chunks(y.rows), y.nb, (int)y.hidden, gb);
      PMB_CHECK_LAUNCH(name);
    }
    // weight gradient: dW_b = dcur_b^T lx_b  (M = H, N = lin, K = rows)
    {
      CUtensorMap ma, mb;
      int st = tma::make_map_3d(ma, dcur, dtype, y.hidden, y.nb, y.rows, y.hidden * 2, (int64_t)y.nb * y.hidden * 2,
                                64, 1, 64, name);
      if (st) return st;
      st = tma::make_map_3d(mb, lx, dtype, lin, y.nb, y.rows, lin * 2, (int64_t)y.nb * lin * 2, 64, 1, 64, name);
      if (st) return st;
      ugemm::Plan plan;
      plan.num_groups = y.nb;
      WGradEpi<TP> epi;
      epi.mode = 0;
      epi.cols = (int)lin;
      epi.info = info;
      for (int b = 0; b < y.nb; ++b) {
        plan.g[b] = ugemm::Group{(int)y.hidden, (int)lin, (int)y.rows, 0, b, 0, 0, b, 0};
        epi.info.grad[b] = grad_weights[(int64_t)l * y.nb + b];
      }
      st = lin % 192 == 0 ? run_gemm<192, WGradEpi<TP>, true, true>(ma, mb, plan, epi, fp16, s, name)
                          : run_gemm<BN, WGradEpi<TP>, true, true>(ma, mb, plan, epi, fp16, s, name);
      if (st) return st;
    }
    // input gradient: dX_b = dcur_b W_b (M = rows, N = lin, K = H), tanh' of the layer below fused
    if (l > 0 || need_x) {
      CUtensorMap ma, mb;
      int st = tma::make_map_3d(ma, dcur, dtype, y.hidden, y.nb, y.rows, y.hidden * 2, (int64_t)y.nb * y.hidden * 2,
                                64, 1, ugemm::BM, name);
      if (st) return st;
      st = tma::make_map_3d(mb, pk_layer[l], dtype, lin, y.nb, y.hidden, y.hidden * lin * 2, lin * 2, 64, 1, 64,
                            name);
      if (st) return st;
      ugemm::Plan plan;
      plan.num_groups = y.nb;
      for (int b = 0; b < y.nb; ++b) plan.g[b] = ugemm::Group{(int)y.rows, (int)lin, (int)y.hidden, 0, b, 0, 0, b, 0};
      DActEpi<T> epi;
      T* next = l > 0 ? buf[(y.L - l) % 2] : static_cast<T*>(grad_x);
      if (next == dcur) next = buf[((y.L - l) + 1) % 2];
      epi.dst = next;
      epi.y = l > 0 ? lx : nullptr;
      epi.partial = l > 0 ? partial : nullptr;  // bias gradient of layer l - 1
      epi.ld = (int64_t)y.nb * lin;
      epi.h = (int)lin;
      epi.use_tma = tma::make_store_map_2d(epi.dst_map, next, dtype, (uint64_t)epi.ld, (uint64_t)y.rows,
                                           (uint64_t)(epi.ld * 2), name) == PMB_OK;
      if (!epi.use_tma) clear_error();
      st = lin % 192 == 0 ? run_gemm<192, DActEpi<T>, false, true>(ma, mb, plan, epi, fp16, s, name)
                          : run_gemm<BN, DActEpi<T>, false, true>(ma, mb, plan, epi, fp16, s, name);
      if (st) return st;
      dcur = next;
    }
  }
  return PMB_OK;
}

bool tc_shapes_ok(int64_t dim, int64_t hidden) { return dim % 64 == 0 && hidden % 64 == 0; }

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_mask_estimator_tc_sizes(int64_t rows, int num_bands, int64_t dim, int64_t hidden,
                                           int hidden_layers, const int64_t* widths, int64_t* sizes) {
  clear_error();
  PMB_REQUIRE(num_bands > 0 && num_bands <= kMaxBands && widths && sizes && rows >= 0 && hidden_layers >= 0,
              "pmb_mask_estimator_tc_sizes: bad arguments");
  const Layout y = make_layout(rows, num_bands, dim, hidden, hidden_layers, widths, nullptr);
  sizes[0] = y.pk_bytes;
  sizes[1] = y.acts_bytes;
  sizes[2] = y.pre_bytes;
  sizes[3] = y.ws_bytes;
  sizes[4] = y.P;
  return PMB_OK;
}

extern "C" int pmb_mask_estimator_tc_forward(const void* x, int64_t rows, int num_bands, int64_t dim, int64_t hidden,
                                             int hidden_layers, const int64_t* widths, const void* const* weights,
                                             const void* const* biases, void* packed_weights, void* acts, void* pre,
                                             void* out, int dtype, int param_dtype, void* stream) {
  clear_error();
  const char* name = "pmb_mask_estimator_tc_forward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  PMB_REQUIRE(num_bands > 0 && num_bands <= kMaxBands && widths && weights && biases, "%s: bad band arguments", name);
  PMB_REQUIRE(tc_shapes_ok(dim, hidden), "%s: dim and hidden must be multiples of 64", name);
  PMB_REQUIRE(hidden_layers >= 0 && hidden_layers <= 8, "%s: 0..8 hidden layers", name);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(x && packed_weights && pre && out && (hidden_layers == 0 || acts), "%s: NULL tensor argument", name);
  const Layout y = make_layout(rows, num_bands, dim, hidden, hidden_layers, widths, nullptr);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 4) {
      set_error("%s: fp32 activations are not supported", name);
      return PMB_ERR_UNSUPPORTED_DTYPE;
    } else {
      return forward_impl<T, TP>(x, y, weights, biases, widths, packed_weights, acts, pre, out, dtype, s);
    }
  });
}

extern "C" int pmb_mask_estimator_tc_backward(const void* grad_out, const void* x, const void* acts, const void* pre,
                                              const void* packed_weights, int64_t rows, int num_bands, int64_t dim,
                                              int64_t hidden, int hidden_layers, const int64_t* widths,
                                              void* const* grad_weights, void* const* grad_biases, void* grad_x,
                                              int dtype, int param_dtype, void* workspace, int64_t workspace_bytes,
                                              void* stream) {
  clear_error();
  const char* name = "pmb_mask_estimator_tc_backward";
  PMB_REQUIRE(dtype == PMB_BFLOAT16 || dtype == PMB_FLOAT16, "%s: activations must be bf16 or fp16", name);
  PMB_REQUIRE(num_bands > 0 && num_bands <= kMaxBands && widths && grad_weights && grad_biases,
              "%s: bad band arguments", name);
  PMB_REQUIRE(tc_shapes_ok(dim, hidden), "%s: dim and hidden must be multiples of 64", name);
  PMB_REQUIRE(rows > 0, "%s: needs at least one row", name);
  PMB_REQUIRE(grad_out && x && pre && packed_weights && (hidden_layers == 0 || acts), "%s: NULL tensor argument",
              name);
  const Layout y = make_layout(rows, num_bands, dim, hidden, hidden_layers, widths, nullptr);
  if (workspace == nullptr || workspace_bytes < y.ws_bytes) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)y.ws_bytes);
    return PMB_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 4) {
      set_error("%s: fp32 activations are not supported", name);
      return PMB_ERR_UNSUPPORTED_DTYPE;
    } else {
      return backward_impl<T, TP>(grad_out, x, acts, pre, packed_weights, y, widths, grad_weights, grad_biases, grad_x,
                                  static_cast<char*>(workspace), dtype, s);
    }
  });
}
