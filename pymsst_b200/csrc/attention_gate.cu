// Per-head attention output gate: gate[r,h] = sigmoid(x[r,:] . Wg[h,:] + bg[h]),
// out[r, h*Dh + d] = attn[r,h,d] * gate[r,h], forward and backward.
// Reference semantics: src/pymsst/training/cuda/fused_band_split.cu:1778-2036
// (called from src/pymsst/training/fused_roformer.py:793-818, 1228-1262).
//
// attn is addressed with strides so the attention output can be read in the
// [batch, heads, seq, Dh] layout the attention kernel produces: row
// r = bi*seq + n, element (r, h, d) at bi*s_b + n*s_n + h*s_h + d.  The gate
// row product, sigmoid and gating are one warp-per-row pass (the reference
// uses two launches); the backward writes grad_attn with the attn strides.
#include <initializer_list>

#include "common.cuh"
#include "reduce.cuh"

namespace pmb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxHeads = 16;
constexpr int kRowsPerChunk = 256;

// Row r of x / out is token (sequence, position) of the attention output:
// rows are ordered (outer, position, inner) -- inner = 1 is the plain
// [sequences, seq] order; inner > 1 lets an axial transformer keep its input
// in the other axis' order (sequence = outer * inner + inner index).
struct AttnLayout {
  int64_t seq, s_b, s_n, s_h, inner;
  __device__ __forceinline__ int64_t row_base(int64_t r) const {
    const int64_t q = r / inner, ii = r - q * inner;
    const int64_t o = q / seq, pos = q - o * seq;
    return (o * inner + ii) * s_b + pos * s_n;
  }
};

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + expf(-v)); }

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads)
    gate_fwd(const T* __restrict__ attn, AttnLayout la, const T* __restrict__ x, const TP* __restrict__ W,
             const TP* __restrict__ bias, int64_t rows, int H, int Dh, int dim, T* __restrict__ out,
             T* __restrict__ gate) {
  extern __shared__ float sw[];  // [H][dim]
  for (int e = threadIdx.x; e < H * dim; e += kThreads) sw[e] = Elem<TP>::to_f(W[e]);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * kWarps) {
    float dots[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) dots[h] = 0.f;
    for (int i = lane; i < dim; i += 32) {
      const float xv = Elem<T>::to_f(x[r * dim + i]);
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h < H) dots[h] += xv * sw[h * dim + i];
    }
    float g[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
      if (h < H) {
        const float d = warp_sum(dots[h]);
        g[h] = round_to<T>(sigmoidf_(d + Elem<TP>::to_f(bias[h])));
      } else {
        g[h] = 0.f;
      }
    }
    if (lane < H) {
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h == lane) gate[r * H + h] = Elem<T>::from_f(g[h]);
    }
    const int64_t ab = la.row_base(r);
    for (int e = lane; e < H * Dh; e += 32) {
      const int h = e / Dh, d = e % Dh;
      float gh = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxHeads; ++k)
        if (k == h) gh = g[k];
      out[r * (int64_t)H * Dh + e] = Elem<T>::from_f(Elem<T>::to_f(attn[ab + h * la.s_h + d]) * gh);
    }
  }
}

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads)
    gate_bwd_rows(const T* __restrict__ grad_out, const T* __restrict__ attn, AttnLayout la, const TP* __restrict__ W,
                  const T* __restrict__ gate, int64_t rows, int H, int Dh, int dim, T* __restrict__ grad_attn,
                  T* __restrict__ grad_x, float* __restrict__ ggp) {
  extern __shared__ float sw[];  // [H][dim]
  for (int e = threadIdx.x; e < H * dim; e += kThreads) sw[e] = Elem<TP>::to_f(W[e]);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * kWarps) {
    const int64_t ab = la.row_base(r);
    float gs[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) gs[h] = 0.f;
    for (int e = lane; e < H * Dh; e += 32) {
      const int h = e / Dh, d = e % Dh;
      const float g = Elem<T>::to_f(grad_out[r * (int64_t)H * Dh + e]);
      const float a = Elem<T>::to_f(attn[ab + h * la.s_h + d]);
      const float gv = Elem<T>::to_f(gate[r * H + h]);
      grad_attn[ab + h * la.s_h + d] = Elem<T>::from_f(g * gv);
#pragma unroll
      for (int k = 0; k < kMaxHeads; ++k)
        if (k == h) gs[k] += g * a;
    }
    float gp[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
      if (h < H) {
        const float gv = Elem<T>::to_f(gate[r * H + h]);
        gp[h] = warp_sum(gs[h]) * gv * (1.0f - gv);
      } else {
        gp[h] = 0.f;
      }
    }
    if (lane < H) {
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h == lane) ggp[r * H + h] = gp[h];
    }
    for (int i = lane; i < dim; i += 32) {
      float acc = 0.f;
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h)
        if (h < H) acc += gp[h] * sw[h * dim + i];
      grad_x[r * dim + i] = Elem<T>::from_f(acc);
    }
  }
}

// partial[chunk][h*(dim+1) + i] = sum_{r in chunk} ggp[r,h] * x[r,i]; column dim holds the bias sum.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    gate_bwd_weight_partial(const float* __restrict__ ggp, const T* __restrict__ x, int64_t rows, int H, int dim,
                            float* __restrict__ partial) {
  const int cols = H * (dim + 1);
  const int64_t r0 = (int64_t)blockIdx.y * kRowsPerChunk;
  const int64_t r1 = r0 + kRowsPerChunk < rows ? r0 + kRowsPerChunk : rows;
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  const int h = c / (dim + 1), i = c % (dim + 1);
  float acc = 0.f;
  for (int64_t r = r0; r < r1; ++r) {
    const float g = ggp[r * H + h];
    acc += i == dim ? g : g * Elem<T>::to_f(x[r * dim + i]);
  }
  partial[(int64_t)blockIdx.y * cols + c] = acc;
}

template <typename TP>
__global__ void __launch_bounds__(kThreads)
    gate_bwd_weight_finalize(const float* __restrict__ partial, int chunks, int H, int dim, TP* __restrict__ grad_w,
                             TP* __restrict__ grad_b) {
  const int cols = H * (dim + 1);
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int k = 0; k < chunks; ++k) s += partial[(int64_t)k * cols + c];
  const int h = c / (dim + 1), i = c % (dim + 1);
  if (i == dim)
    grad_b[h] = Elem<TP>::from_f(s);
  else
    grad_w[h * dim + i] = Elem<TP>::from_f(s);
}

// ---------------------------------------------------------------------------
// Tiled path: a CTA takes 32 consecutive rows at a time.  The tile's x rows
// and the gate weights sit in shared memory; every global access is a 16-byte
// vector (x, attn, out, grad tensors), so each row costs one pass over its
// bytes.  The backward keeps the weight / bias gradient partials in
// registers across all tiles of a persistent CTA (one fp32 partial row per
// CTA, summed by red::colsum_rows), so it needs no per-row gate-gradient
// buffer.  Conditions (tiled_ok): 16-byte aligned pointers and strides, dim
// and Dh multiples of the vector width, Dh / width a power of two <= 32.
constexpr int kTileRows = 32;
constexpr int kMaxWPerThread = 12;      // heads * dim <= 256 * 12 in the tiled backward
constexpr int kMaxTiledBwdBlocks = 592; // partial rows in the workspace

template <typename T>
struct Vec {
  static constexpr int N = 16 / sizeof(T);
  __device__ __forceinline__ static void unpack(const uint4& u, float (&f)[N]) {
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = Elem<T>::to_f(e[i]);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[N]) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = Elem<T>::from_f(f[i]);
    return u;
  }
};

// Shared-memory carve-up common to both directions: gate weights as fp32
// [H][dim + 4], the x tile [32][dim + V] (row padding keeps 16-byte reads of
// neighbouring rows on different banks), then two [32][H] fp32 arrays.
struct TileSmem {
  int wld, xld;
  size_t w_bytes, x_bytes, bytes;
  __host__ __device__ TileSmem(int H, int dim, int V) {
    wld = dim + 4;
    xld = dim + V;
    w_bytes = (size_t)H * wld * 4;
    x_bytes = (size_t)kTileRows * xld * (16 / V);
    bytes = w_bytes + x_bytes + 2 * (size_t)kTileRows * H * 4;
  }
};

template <typename T, typename TP>
__device__ __forceinline__ void load_weights_smem(const TP* __restrict__ W, int H, int dim, float* w_s, int wld) {
  for (int e = threadIdx.x; e < H * dim; e += kThreads) w_s[(e / dim) * wld + e % dim] = Elem<TP>::to_f(W[e]);
}

template <typename T>
__device__ __forceinline__ void load_x_tile(const T* __restrict__ x, int64_t r0, int64_t rows, int dim, T* x_s,
                                            int xld) {
  constexpr int V = Vec<T>::N;
  const int vpr = dim / V;
  for (int v = threadIdx.x; v < kTileRows * vpr; v += kThreads) {
    const int r = v / vpr, c = (v - r * vpr) * V;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (r0 + r < rows) u = *reinterpret_cast<const uint4*>(x + (r0 + r) * dim + c);
    *reinterpret_cast<uint4*>(x_s + r * xld + c) = u;
  }
}

// Per-tile row bases of the attention layout (one 64-bit division per row,
// by 32 threads, instead of one per 16-byte vector).
__device__ __forceinline__ void load_row_bases(const AttnLayout& la, int64_t r0, int64_t rows, int64_t* rb_s) {
  if (threadIdx.x < kTileRows) {
    const int64_t r = r0 + threadIdx.x;
    rb_s[threadIdx.x] = r < rows ? la.row_base(r) : 0;
  }
}

// Thread -> (column vector, first row, row step) over a tile of 32 rows with
// vr vectors per row: fixed column when vr divides the block, else strided.
struct ColMap {
  int c, r_first, r_step;
  bool fixed;
  __device__ ColMap(int vr) {
    fixed = (kThreads % vr) == 0;
    c = threadIdx.x % vr;
    r_first = threadIdx.x / vr;
    r_step = kThreads / vr;
  }
};

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads, 4)
    gate_fwd_tiled(const T* __restrict__ attn, AttnLayout la, const T* __restrict__ x, const TP* __restrict__ W,
                   const TP* __restrict__ bias, int64_t rows, int H, int Dh, int dim, T* __restrict__ out,
                   T* __restrict__ gate) {
  constexpr int V = Vec<T>::N;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int64_t rb_s[kTileRows];
  const TileSmem L(H, dim, V);
  float* w_s = reinterpret_cast<float*>(smem_raw);
  T* x_s = reinterpret_cast<T*>(smem_raw + L.w_bytes);
  float* g_s = reinterpret_cast<float*>(smem_raw + L.w_bytes + L.x_bytes);
  load_weights_smem<T, TP>(W, H, dim, w_s, L.wld);
  const int vh = Dh / V, vr = H * vh;
  const ColMap cm(vr);
  const int ch = cm.c / vh, cd = (cm.c - ch * vh) * V;
  const int64_t tiles = (rows + kTileRows - 1) / kTileRows;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t r0 = tile * kTileRows;
    load_x_tile<T>(x, r0, rows, dim, x_s, L.xld);
    load_row_bases(la, r0, rows, rb_s);
    __syncthreads();
    for (int p = threadIdx.x; p < kTileRows * H; p += kThreads) {
      const int r = p / H, h = p - r * H;
      const T* xr = x_s + r * L.xld;
      const float* wr = w_s + h * L.wld;
      float acc = 0.f;
      for (int i = 0; i < dim; i += V) {
        float xf[V];
        Vec<T>::unpack(*reinterpret_cast<const uint4*>(xr + i), xf);
#pragma unroll
        for (int q = 0; q < V; q += 4) {
          const float4 w4 = *reinterpret_cast<const float4*>(wr + i + q);
          acc += xf[q] * w4.x + xf[q + 1] * w4.y + xf[q + 2] * w4.z + xf[q + 3] * w4.w;
        }
      }
      const float g = round_to<T>(sigmoidf_(acc + Elem<TP>::to_f(bias[h])));
      g_s[p] = g;
      if (r0 + r < rows) gate[r0 * H + p] = Elem<T>::from_f(g);
    }
    __syncthreads();
    const int nr = rows - r0 < kTileRows ? (int)(rows - r0) : kTileRows;
    if (cm.fixed) {
      const int64_t aoff = (int64_t)ch * la.s_h + cd;
      T* orow = out + r0 * (int64_t)vr * V + (int64_t)cm.c * V;
#pragma unroll 4
      for (int r = cm.r_first; r < nr; r += cm.r_step) {
        float a[V];
        Vec<T>::unpack(*reinterpret_cast<const uint4*>(attn + rb_s[r] + aoff), a);
        const float g = g_s[r * H + ch];
#pragma unroll
        for (int q = 0; q < V; ++q) a[q] *= g;
        *reinterpret_cast<uint4*>(orow + (int64_t)r * vr * V) = Vec<T>::pack(a);
      }
    } else {
      for (int v = threadIdx.x; v < nr * vr; v += kThreads) {
        const int r = v / vr, c = v - r * vr;
        const int h = c / vh, d = (c - h * vh) * V;
        float a[V];
        Vec<T>::unpack(*reinterpret_cast<const uint4*>(attn + rb_s[r] + h * la.s_h + d), a);
        const float g = g_s[r * H + h];
#pragma unroll
        for (int q = 0; q < V; ++q) a[q] *= g;
        *reinterpret_cast<uint4*>(out + (r0 + r) * (int64_t)vr * V + (int64_t)c * V) = Vec<T>::pack(a);
      }
    }
    __syncthreads();
  }
}

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads, 3)
    gate_bwd_tiled(const T* __restrict__ grad_out, const T* __restrict__ attn, AttnLayout la,
                   const T* __restrict__ x, const TP* __restrict__ W, const T* __restrict__ gate, int64_t rows,
                   int H, int Dh, int dim, T* __restrict__ grad_attn, T* __restrict__ grad_x,
                   float* __restrict__ partial_w, float* __restrict__ partial_b) {
  constexpr int V = Vec<T>::N;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int64_t rb_s[kTileRows];
  const TileSmem L(H, dim, V);
  float* w_s = reinterpret_cast<float*>(smem_raw);
  T* x_s = reinterpret_cast<T*>(smem_raw + L.w_bytes);
  float* g_s = reinterpret_cast<float*>(smem_raw + L.w_bytes + L.x_bytes);
  float* gp_s = g_s + kTileRows * H;
  load_weights_smem<T, TP>(W, H, dim, w_s, L.wld);
  const int vh = Dh / V, vr = H * vh, hd = H * dim, q4 = dim / 4;
  const ColMap cm(vr);
  const int ch = cm.c / vh, cd = (cm.c - ch * vh) * V;
  float accw[kMaxWPerThread];
#pragma unroll
  for (int j = 0; j < kMaxWPerThread; ++j) accw[j] = 0.f;
  float accb = 0.f;
  const int64_t tiles = (rows + kTileRows - 1) / kTileRows;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t r0 = tile * kTileRows;
    const int nr = rows - r0 < kTileRows ? (int)(rows - r0) : kTileRows;
    load_x_tile<T>(x, r0, rows, dim, x_s, L.xld);
    load_row_bases(la, r0, rows, rb_s);
    for (int p = threadIdx.x; p < kTileRows * H; p += kThreads) {
      g_s[p] = p / H < nr ? Elem<T>::to_f(gate[r0 * H + p]) : 0.f;
      gp_s[p] = 0.f;
    }
    __syncthreads();
    // grad_attn = grad_out * gate; per (row, head) sum of grad_out * attn over
    // the head's vh consecutive vectors, reduced across vh lanes.  Trip counts
    // are warp-uniform (the lanes of a warp share their rows in the fixed map;
    // kTileRows * vr is a multiple of 32 in the strided one).
    if (cm.fixed) {
      const int64_t aoff = (int64_t)ch * la.s_h + cd;
      const T* gorow = grad_out + r0 * (int64_t)vr * V + (int64_t)cm.c * V;
#pragma unroll 2
      for (int r = cm.r_first; r < kTileRows; r += cm.r_step) {
        float part = 0.f;
        if (r < nr) {
          const int64_t ai = rb_s[r] + aoff;
          float go[V], a[V];
          Vec<T>::unpack(*reinterpret_cast<const uint4*>(gorow + (int64_t)r * vr * V), go);
          Vec<T>::unpack(*reinterpret_cast<const uint4*>(attn + ai), a);
          const float g = g_s[r * H + ch];
#pragma unroll
          for (int q = 0; q < V; ++q) {
            part += go[q] * a[q];
            a[q] = go[q] * g;
          }
          *reinterpret_cast<uint4*>(grad_attn + ai) = Vec<T>::pack(a);
        }
        for (int o = vh >> 1; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if ((cm.c & (vh - 1)) == 0 && r < nr) {
          const float g = g_s[r * H + ch];
          gp_s[r * H + ch] = part * g * (1.0f - g);
        }
      }
    } else {
      for (int v = threadIdx.x; v < kTileRows * vr; v += kThreads) {
        const int r = v / vr, c = v - r * vr;
        const int h = c / vh, d = (c - h * vh) * V;
        float part = 0.f;
        if (r < nr) {
          const int64_t ai = rb_s[r] + h * la.s_h + d;
          float go[V], a[V];
          Vec<T>::unpack(*reinterpret_cast<const uint4*>(grad_out + (r0 + r) * (int64_t)vr * V + (int64_t)c * V),
                         go);
          Vec<T>::unpack(*reinterpret_cast<const uint4*>(attn + ai), a);
          const float g = g_s[r * H + h];
#pragma unroll
          for (int q = 0; q < V; ++q) {
            part += go[q] * a[q];
            a[q] = go[q] * g;
          }
          *reinterpret_cast<uint4*>(grad_attn + ai) = Vec<T>::pack(a);
        }
        for (int o = vh >> 1; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if ((c & (vh - 1)) == 0 && r < nr) {
          const float g = g_s[r * H + h];
          gp_s[r * H + h] = part * g * (1.0f - g);
        }
      }
    }
    __syncthreads();
    // grad_x[r, i..i+3] = sum_h gp[r, h] W[h, i..i+3]
    for (int v = threadIdx.x; v < nr * q4; v += kThreads) {
      const int r = v / q4, i = (v - r * q4) * 4;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int h = 0; h < H; ++h) {
        const float gp = gp_s[r * H + h];
        const float4 w4 = *reinterpret_cast<const float4*>(w_s + h * L.wld + i);
        acc[0] += gp * w4.x;
        acc[1] += gp * w4.y;
        acc[2] += gp * w4.z;
        acc[3] += gp * w4.w;
      }
      T o4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) o4[q] = Elem<T>::from_f(acc[q]);
      T* dst = grad_x + (r0 + r) * dim + i;
      if (sizeof(T) == 2)
        *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o4);
      else
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o4);
    }
    // grad_W[h, i] += sum_r gp[r, h] x[r, i]; grad_b[h] += sum_r gp[r, h]
    // (rows past the end have gp = 0 and x = 0).
#pragma unroll
    for (int j = 0; j < kMaxWPerThread; ++j) {
      const int e = threadIdx.x + j * kThreads;
      if (e < hd) {
        const int h = e / dim, i = e - h * dim;
        float acc = accw[j];
#pragma unroll 8
        for (int r = 0; r < kTileRows; ++r) acc += gp_s[r * H + h] * Elem<T>::to_f(x_s[r * L.xld + i]);
        accw[j] = acc;
      }
    }
    if (threadIdx.x < H)
      for (int r = 0; r < kTileRows; ++r) accb += gp_s[r * H + threadIdx.x];
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < kMaxWPerThread; ++j) {
    const int e = threadIdx.x + j * kThreads;
    if (e < hd) partial_w[(int64_t)blockIdx.x * hd + e] = accw[j];
  }
  if (threadIdx.x < H) partial_b[(int64_t)blockIdx.x * H + threadIdx.x] = accb;
}

// ------------------------------------------------- streamed kernels
// When a row's heads are contiguous in attn (head stride = Dh) each attention
// row is one 16-byte aligned block of H*Dh elements.  The streamed kernels
// keep kStreamStages - 1 tiles of kStreamRows rows in flight while they work
// on the current one: every thread issues 16-byte cp.async copies of its share
// of a later tile (attention rows through per-tile row bases, grad_out, x rows
// padded by 16 bytes so neighbouring rows sit on different banks, gate) into a
// shared-memory ring, and the per-thread async groups are waited with
// cp.async.wait_group -- no spin waits.  The arithmetic is that of the tiled
// kernels above; results leave with 16-byte stores.
constexpr int kStreamRows = 8;
constexpr int kStreamStages = 3;

struct StreamLayout {
  int hd_b, x_b, g_b, xld, wld;             // bytes per attention / x / gate row; x and W row pitch (elements)
  int off_at, off_go, off_x, off_g, stage;  // offsets within a stage, stage stride
  int off_w, off_gp, bytes;                 // after the ring: W fp32 [H][wld], gp fp32 [rows][H]
  __host__ __device__ StreamLayout(int H, int Dh, int dim, int es, bool bwd) {
    hd_b = H * Dh * es;
    x_b = dim * es;
    g_b = H * es;
    xld = dim + 16 / es;
    wld = dim + 4;
    off_at = 0;
    off_go = off_at + kStreamRows * hd_b;
    off_x = off_go + (bwd ? kStreamRows * hd_b : 0);
    off_g = off_x + kStreamRows * xld * es;
    stage = (off_g + (bwd ? kStreamRows * g_b : 0) + 127) / 128 * 128;
    off_w = kStreamStages * stage;
    off_gp = off_w + H * wld * 4;
    bytes = off_gp + kStreamRows * H * 4;
  }
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// This thread's share of one tile's copies (n rows from r0; rb = row bases).
template <typename T>
__device__ __forceinline__ void load_tile_async(uint8_t* base, const StreamLayout& L, const int64_t* rb,
                                                const T* attn, const T* x, const T* grad_out, const T* gate,
                                                int64_t r0, int n, int H, int dim) {
  constexpr int V = Vec<T>::N;
  const int va = L.hd_b / 16, vx = L.x_b / 16;
  for (int v = threadIdx.x; v < n * va; v += kThreads) {
    const int r = v / va, c = v - r * va;
    cp_async16(base + L.off_at + r * L.hd_b + c * 16, attn + rb[r] + (int64_t)c * V);
    if (grad_out) cp_async16(base + L.off_go + r * L.hd_b + c * 16, grad_out + (r0 + r) * (int64_t)(va * V) + c * V);
  }
  for (int v = threadIdx.x; v < n * vx; v += kThreads) {
    const int r = v / vx, c = v - r * vx;
    cp_async16(base + L.off_x + r * L.xld * (int)sizeof(T) + c * 16, x + (r0 + r) * dim + (int64_t)c * V);
  }
  if (gate)
    for (int v = threadIdx.x; v < n * (L.g_b / 16); v += kThreads)
      cp_async16(base + L.off_g + v * 16, gate + r0 * H + (int64_t)v * V);
}

template <typename TP>
__device__ __forceinline__ void load_weights_stream(const TP* __restrict__ W, int H, int dim, float* w_s, int wld) {
  for (int e = threadIdx.x; e < H * dim; e += kThreads) w_s[(e / dim) * wld + e % dim] = Elem<TP>::to_f(W[e]);
}

// Ring driver shared by both directions: before tile `it` is worked on, the
// tile kStreamStages - 1 ahead is put in flight.  `rb_s` holds each stage's
// row bases (written by the first kStreamRows threads).
struct StreamRing {
  int64_t rows, tiles;
  __device__ int rows_of(int64_t t) const {
    const int64_t left = rows - t * kStreamRows;
    return (int)(left < kStreamRows ? left : kStreamRows);
  }
};

// Fixed thread -> work maps of the streamed kernels (16-bit types, 8-element
// chunks).  vr 16-byte vectors per attention row divide the 256 threads, so a
// thread keeps one column vector and walks rows r0 + t / vr, + 256 / vr, ...
// grad_x / grad_W work is in (row or head) x 8-column chunks, at most
// kMaxChunkItems per thread.
constexpr int kMaxChunkItems = 2;

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads, 3)
    gate_fwd_stream(const T* __restrict__ attn, AttnLayout la, const T* __restrict__ x, const TP* __restrict__ W,
                    const TP* __restrict__ bias, int64_t rows, int H, int Dh, int dim, T* __restrict__ out,
                    T* __restrict__ gate) {
  constexpr int V = Vec<T>::N;  // 8
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int64_t rb_s[kStreamStages + 1][kStreamRows];
  const StreamLayout L(H, Dh, dim, sizeof(T), false);
  float* w_s = reinterpret_cast<float*>(smem + L.off_w);
  float* g_s = reinterpret_cast<float*>(smem + L.off_gp);
  load_weights_stream<TP>(W, H, dim, w_s, L.wld);
  const StreamRing ring{rows, (rows + kStreamRows - 1) / kStreamRows};
  // row bases of the tile of iteration k live in slot k % (kStreamStages + 1); they are computed one
  // iteration before that tile is put in flight, so the copies need no barrier of their own
  auto bases = [&](int64_t t, int slot) {
    if (threadIdx.x < kStreamRows)
      rb_s[slot][threadIdx.x] = (t < ring.tiles && threadIdx.x < ring.rows_of(t)) ? la.row_base(t * kStreamRows + threadIdx.x) : 0;
  };
  auto prefetch = [&](int64_t t, int st, int slot) {  // whole CTA; ends with a commit (empty past the end)
    if (t < ring.tiles)
      load_tile_async<T>(smem + st * L.stage, L, rb_s[slot], attn, x, (const T*)nullptr, (const T*)nullptr,
                         t * kStreamRows, ring.rows_of(t), H, dim);
    cp_commit();
  };
  for (int s = 0; s < kStreamStages; ++s) bases(blockIdx.x + (int64_t)s * gridDim.x, s);
  __syncthreads();
  for (int s = 0; s < kStreamStages - 1; ++s) prefetch(blockIdx.x + (int64_t)s * gridDim.x, s, s);
  const int vh = Dh / V, vr = H * vh, nck = dim / V;
  // logits: 4 threads per (row, head), each a quarter of the 8-element chunks
  const int lp = threadIdx.x >> 2, lq = threadIdx.x & 3, lr = lp / H, lh = lp - lr * H;
  const float lbias = lp < kStreamRows * H ? Elem<TP>::to_f(bias[lh]) : 0.f;
  // gating: fixed column vector, rows c_r0, + c_rs, ...
  const int cc = threadIdx.x % vr, c_r0 = threadIdx.x / vr, c_rs = kThreads / vr, ch = cc / vh;
  int it = 0;
  for (int64_t tile = blockIdx.x; tile < ring.tiles; tile += gridDim.x, ++it) {
    const int st = it % kStreamStages;
    prefetch(tile + (int64_t)(kStreamStages - 1) * gridDim.x, (it + kStreamStages - 1) % kStreamStages,
             (it + kStreamStages - 1) % (kStreamStages + 1));
    cp_wait<kStreamStages - 1>();
    __syncthreads();  // this tile's copies from every thread have landed
    const int64_t r0 = tile * kStreamRows;
    const int n = ring.rows_of(tile);
    const uint8_t* base = smem + st * L.stage;
    const T* at_s = reinterpret_cast<const T*>(base + L.off_at);
    const T* x_s = reinterpret_cast<const T*>(base + L.off_x);
    bases(tile + (int64_t)kStreamStages * gridDim.x, (it + kStreamStages) % (kStreamStages + 1));
    if (lp < kStreamRows * H) {  // warp-uniform: kStreamRows * H * 4 is a multiple of 32
      const T* xr = x_s + lr * L.xld;
      const float* wr = w_s + lh * L.wld;
      float acc = 0.f;
      for (int k = lq; k < nck; k += 4) {
        float xf[V];
        Vec<T>::unpack(*reinterpret_cast<const uint4*>(xr + k * V), xf);
        const float4 w0 = *reinterpret_cast<const float4*>(wr + k * V);
        const float4 w1 = *reinterpret_cast<const float4*>(wr + k * V + 4);
        acc += xf[0] * w0.x + xf[1] * w0.y + xf[2] * w0.z + xf[3] * w0.w + xf[4] * w1.x + xf[5] * w1.y +
               xf[6] * w1.z + xf[7] * w1.w;
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (lq == 0 && lr < n) {
        const float g = round_to<T>(sigmoidf_(acc + lbias));
        g_s[lp] = g;
        gate[r0 * H + lp] = Elem<T>::from_f(g);
      }
    }
    __syncthreads();
    for (int r = c_r0; r < n; r += c_rs) {
      float a[V];
      Vec<T>::unpack(*reinterpret_cast<const uint4*>(at_s + r * vr * V + cc * V), a);
      const float g = g_s[r * H + ch];
#pragma unroll
      for (int q = 0; q < V; ++q) a[q] *= g;
      *reinterpret_cast<uint4*>(out + (r0 + r) * (int64_t)vr * V + (int64_t)cc * V) = Vec<T>::pack(a);
    }
    __syncthreads();  // stage st and g_s are free
  }
  cp_wait<0>();
}

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads, 3)
    gate_bwd_stream(const T* __restrict__ grad_out, const T* __restrict__ attn, AttnLayout la,
                    const T* __restrict__ x, const TP* __restrict__ W, const T* __restrict__ gate, int64_t rows,
                    int H, int Dh, int dim, T* __restrict__ grad_attn, T* __restrict__ grad_x,
                    float* __restrict__ partial_w, float* __restrict__ partial_b) {
  constexpr int V = Vec<T>::N;  // 8
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int64_t rb_s[kStreamStages + 1][kStreamRows];
  const StreamLayout L(H, Dh, dim, sizeof(T), true);
  float* w_s = reinterpret_cast<float*>(smem + L.off_w);
  float* gp_s = reinterpret_cast<float*>(smem + L.off_gp);
  load_weights_stream<TP>(W, H, dim, w_s, L.wld);
  const StreamRing ring{rows, (rows + kStreamRows - 1) / kStreamRows};
  auto bases = [&](int64_t t, int slot) {  // see gate_fwd_stream
    if (threadIdx.x < kStreamRows)
      rb_s[slot][threadIdx.x] = (t < ring.tiles && threadIdx.x < ring.rows_of(t)) ? la.row_base(t * kStreamRows + threadIdx.x) : 0;
  };
  auto prefetch = [&](int64_t t, int st, int slot) {
    if (t < ring.tiles)
      load_tile_async<T>(smem + st * L.stage, L, rb_s[slot], attn, x, grad_out, gate, t * kStreamRows,
                         ring.rows_of(t), H, dim);
    cp_commit();
  };
  for (int s = 0; s < kStreamStages; ++s) bases(blockIdx.x + (int64_t)s * gridDim.x, s);
  __syncthreads();
  for (int s = 0; s < kStreamStages - 1; ++s) prefetch(blockIdx.x + (int64_t)s * gridDim.x, s, s);
  const int vh = Dh / V, vr = H * vh, nck = dim / V;
  // grad_attn / gate gradient: fixed column vector cc (head ch), rows c_r0, + c_rs, ...
  const int cc = threadIdx.x % vr, c_r0 = threadIdx.x / vr, c_rs = kThreads / vr, ch = cc / vh;
  // grad_x items (row, chunk) and grad_W items (head, chunk): item = threadIdx.x + j * kThreads
  int xr_[kMaxChunkItems], xk_[kMaxChunkItems], wh_[kMaxChunkItems], wk_[kMaxChunkItems];
#pragma unroll
  for (int j = 0; j < kMaxChunkItems; ++j) {
    const int item = threadIdx.x + j * kThreads;
    xr_[j] = item / nck;
    xk_[j] = item - xr_[j] * nck;
    wh_[j] = item < H * nck ? item / nck : H;  // H: no item
    wk_[j] = item - (item / nck) * nck;
  }
  float accw[kMaxChunkItems][V];
#pragma unroll
  for (int j = 0; j < kMaxChunkItems; ++j)
#pragma unroll
    for (int q = 0; q < V; ++q) accw[j][q] = 0.f;
  float accb = 0.f;
  int it = 0;
  for (int64_t tile = blockIdx.x; tile < ring.tiles; tile += gridDim.x, ++it) {
    const int st = it % kStreamStages;
    prefetch(tile + (int64_t)(kStreamStages - 1) * gridDim.x, (it + kStreamStages - 1) % kStreamStages,
             (it + kStreamStages - 1) % (kStreamStages + 1));
    cp_wait<kStreamStages - 1>();
    __syncthreads();
    const int64_t r0 = tile * kStreamRows;
    const int n = ring.rows_of(tile);
    const uint8_t* base = smem + st * L.stage;
    const T* go_s = reinterpret_cast<const T*>(base + L.off_go);
    const T* at_s = reinterpret_cast<const T*>(base + L.off_at);
    const T* x_s = reinterpret_cast<const T*>(base + L.off_x);
    const T* g_in = reinterpret_cast<const T*>(base + L.off_g);
    const int64_t* rb = rb_s[it % (kStreamStages + 1)];
    bases(tile + (int64_t)kStreamStages * gridDim.x, (it + kStreamStages) % (kStreamStages + 1));
    // grad_attn = grad_out * gate, and per (row, head) the gate-logit gradient
    // sum(grad_out * attn) * g (1 - g), reduced over the head's vh lanes.  The
    // trip count c_r0 < kStreamRows is warp-uniform (vr >= 32 or vr | 32).
    for (int r = c_r0; r < kStreamRows; r += c_rs) {
      float part = 0.f;
      if (r < n) {
        float go[V], a[V];
        Vec<T>::unpack(*reinterpret_cast<const uint4*>(go_s + r * vr * V + cc * V), go);
        Vec<T>::unpack(*reinterpret_cast<const uint4*>(at_s + r * vr * V + cc * V), a);
        const float g = Elem<T>::to_f(g_in[r * H + ch]);
#pragma unroll
        for (int q = 0; q < V; ++q) {
          part += go[q] * a[q];
          a[q] = go[q] * g;
        }
        *reinterpret_cast<uint4*>(grad_attn + rb[r] + (int64_t)cc * V) = Vec<T>::pack(a);
      }
      for (int o = vh >> 1; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if ((cc & (vh - 1)) == 0 && r < n) {
        const float g = Elem<T>::to_f(g_in[r * H + ch]);
        gp_s[r * H + ch] = part * g * (1.0f - g);
      }
    }
    __syncthreads();
    // grad_x[r, 8k..8k+7] = sum_h gp[r, h] W[h, 8k..8k+7]
#pragma unroll
    for (int j = 0; j < kMaxChunkItems; ++j) {
      const int r = xr_[j], k = xk_[j];
      if (r < n) {
        float acc[V];
#pragma unroll
        for (int q = 0; q < V; ++q) acc[q] = 0.f;
        for (int h = 0; h < H; ++h) {
          const float gp = gp_s[r * H + h];
          const float4 w0 = *reinterpret_cast<const float4*>(w_s + h * L.wld + k * V);
          const float4 w1 = *reinterpret_cast<const float4*>(w_s + h * L.wld + k * V + 4);
          acc[0] += gp * w0.x;
          acc[1] += gp * w0.y;
          acc[2] += gp * w0.z;
          acc[3] += gp * w0.w;
          acc[4] += gp * w1.x;
          acc[5] += gp * w1.y;
          acc[6] += gp * w1.z;
          acc[7] += gp * w1.w;
        }
        *reinterpret_cast<uint4*>(grad_x + (r0 + r) * dim + (int64_t)k * V) = Vec<T>::pack(acc);
      }
    }
    // grad_W[h, 8k..8k+7] += sum_r gp[r, h] x[r, 8k..8k+7]; grad_b[h] += sum_r gp[r, h]
#pragma unroll
    for (int j = 0; j < kMaxChunkItems; ++j) {
      const int h = wh_[j], k = wk_[j];
      if (h < H) {
        for (int r = 0; r < n; ++r) {
          const float gp = gp_s[r * H + h];
          float xf[V];
          Vec<T>::unpack(*reinterpret_cast<const uint4*>(x_s + r * L.xld + k * V), xf);
#pragma unroll
          for (int q = 0; q < V; ++q) accw[j][q] += gp * xf[q];
        }
      }
    }
    if (threadIdx.x < H)
      for (int r = 0; r < n; ++r) accb += gp_s[r * H + threadIdx.x];
    __syncthreads();  // stage st and gp_s are free
  }
  cp_wait<0>();
#pragma unroll
  for (int j = 0; j < kMaxChunkItems; ++j) {
    const int h = wh_[j], k = wk_[j];
    if (h < H) {
#pragma unroll
      for (int q = 0; q < V; ++q) partial_w[(int64_t)blockIdx.x * H * dim + h * dim + k * V + q] = accw[j][q];
    }
  }
  if (threadIdx.x < H) partial_b[(int64_t)blockIdx.x * H + threadIdx.x] = accb;
}

// ---------------------------------------------------------------------------
// Warp-per-row path for the model's own shape (8 heads x 64, 16-bit
// activations, dim <= 256 in 8-element chunks): one warp owns a whole row;
// lane l holds elements 16l..16l+15 of the 512-wide attention row (head
// l / 4) and, for l < dim / 8, the 8-element chunk l of x.  Each lane forms
// the 8 head dot products over its x chunk (W from shared memory); a
// transposing butterfly (4 + 2 + 1 + 1 + 1 shuffles) leaves head h's sum in
// lanes 4h..4h+3 -- the lanes holding that head's attention values -- so the
// gate needs no broadcast.  The backward reduces the gate gradient over the
// 4 lanes of a head, broadcasts the 8 values for grad_x, and keeps the
// W / bias gradient partials in registers across the warp's rows (one fp32
// partial row per CTA; the warps are combined in shared memory in a fixed
// order, so results are deterministic).  No block barrier inside the row
// loop; every global access is a 16-byte vector; the forward issues a row's
// loads one row ahead (in the backward, whose W-gradient partials take 64
// registers, the same prefetch measured slower).
constexpr int kWH = 8, kWDh = 64, kWMaxDim = 256;

// Row base in 32-bit arithmetic (callers check rows, inner * seq < 2^31).
__device__ __forceinline__ int64_t row_base32(const AttnLayout& la, int64_t r) {
  const uint32_t ur = (uint32_t)r, inner = (uint32_t)la.inner, seq = (uint32_t)la.seq;
  const uint32_t q = ur / inner, ii = ur - q * inner;
  const uint32_t o = q / seq, pos = q - o * seq;
  return (int64_t)(o * inner + ii) * la.s_b + (int64_t)pos * la.s_n;
}

// d[h] summed over the 32 lanes; lane l receives the sum for head (l >> 2) & 7.
__device__ __forceinline__ float head_sums(const float (&d)[kWH]) {
  const int lane = threadIdx.x & 31;
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
  float e4[4], e2[2];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    e4[k] = (b16 ? d[4 + k] : d[k]) + __shfl_xor_sync(0xffffffffu, b16 ? d[k] : d[4 + k], 16);
#pragma unroll
  for (int k = 0; k < 2; ++k)
    e2[k] = (b8 ? e4[2 + k] : e4[k]) + __shfl_xor_sync(0xffffffffu, b8 ? e4[k] : e4[2 + k], 8);
  float e = (b4 ? e2[1] : e2[0]) + __shfl_xor_sync(0xffffffffu, b4 ? e2[0] : e2[1], 4);
  e += __shfl_xor_sync(0xffffffffu, e, 2);
  e += __shfl_xor_sync(0xffffffffu, e, 1);
  return e;
}

// Gate weights in shared memory as fp32 float4 slices ordered (head, half, lane): lane l's weights
// W[h][8l + 4q .. 8l + 4q + 3] are float4 number (2h + q) * 32 + l, so each of a warp's 16-byte loads
// reads 512 contiguous bytes (no bank conflicts).  kWH * 2 * 32 float4 = 8 KB.
template <typename TP>
__device__ __forceinline__ void load_w_lanes(const TP* __restrict__ W, int dim, float4* w4) {
  for (int e = threadIdx.x; e < kWH * 2 * 32; e += kThreads) {
    const int l = e & 31, hq = e >> 5, h = hq >> 1, c0 = 8 * l + 4 * (hq & 1);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c0 < dim) {
      v.x = Elem<TP>::to_f(W[h * dim + c0]);
      v.y = Elem<TP>::to_f(W[h * dim + c0 + 1]);
      v.z = Elem<TP>::to_f(W[h * dim + c0 + 2]);
      v.w = Elem<TP>::to_f(W[h * dim + c0 + 3]);
    }
    w4[e] = v;
  }
}

// This lane's 8 fp32 gate weights of head h for its x chunk.
__device__ __forceinline__ void w_chunk(const float4* w4, int h, int lane, float (&w)[8]) {
  const float4 u = w4[(2 * h) * 32 + lane];
  const float4 v = w4[(2 * h + 1) * 32 + lane];
  w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
  w[4] = v.x; w[5] = v.y; w[6] = v.z; w[7] = v.w;
}

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads, 3)
    gate_fwd_warp(const T* __restrict__ attn, AttnLayout la, const T* __restrict__ x, const TP* __restrict__ W,
                  const TP* __restrict__ bias, int64_t rows, int dim, T* __restrict__ out, T* __restrict__ gate) {
  __shared__ float4 w4[kWH * 2 * 32];
  load_w_lanes<TP>(W, dim, w4);
  __syncthreads();
  const int lane = threadIdx.x & 31, head = lane >> 2;
  const bool has_x = lane < (dim >> 3);
  const float bh = Elem<TP>::to_f(bias[head]);
  const int64_t step = (int64_t)gridDim.x * kWarps;
  auto load = [&](int64_t rr, uint4& xv, uint4& a0, uint4& a1) {
    if (rr < rows) {
      if (has_x) xv = reinterpret_cast<const uint4*>(x + rr * dim)[lane];
      const uint4* ap = reinterpret_cast<const uint4*>(attn + row_base32(la, rr)) + 2 * lane;
      a0 = ap[0];
      a1 = ap[1];
    }
  };
  int64_t r = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  uint4 xv = make_uint4(0, 0, 0, 0), a0 = xv, a1 = xv;
  load(r, xv, a0, a1);
  for (; r < rows; r += step) {
    uint4 nx = make_uint4(0, 0, 0, 0), n0 = nx, n1 = nx;
    load(r + step, nx, n0, n1);  // the next row's loads go out before this row's arithmetic
    float d[kWH];
#pragma unroll
    for (int h = 0; h < kWH; ++h) d[h] = 0.f;
    if (has_x) {
      float xf[8];
      Vec<T>::unpack(xv, xf);
#pragma unroll
      for (int h = 0; h < kWH; ++h) {
        float w[8];
        w_chunk(w4, h, lane, w);
#pragma unroll
        for (int j = 0; j < 8; ++j) d[h] = fmaf(xf[j], w[j], d[h]);
      }
    }
    const float g = round_to<T>(sigmoidf_(head_sums(d) + bh));
    if ((lane & 3) == 0) gate[r * kWH + head] = Elem<T>::from_f(g);
    float a[8];
    uint4* op = reinterpret_cast<uint4*>(out + r * (kWH * kWDh)) + 2 * lane;
    Vec<T>::unpack(a0, a);
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] *= g;
    op[0] = Vec<T>::pack(a);
    Vec<T>::unpack(a1, a);
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] *= g;
    op[1] = Vec<T>::pack(a);
    xv = nx;
    a0 = n0;
    a1 = n1;
  }
}

template <typename T, typename TP>
__global__ void __launch_bounds__(kThreads, 2)
    gate_bwd_warp(const T* __restrict__ grad_out, const T* __restrict__ attn, AttnLayout la,
                  const T* __restrict__ x, const TP* __restrict__ W, const T* __restrict__ gate, int64_t rows,
                  int dim, T* __restrict__ grad_attn, T* __restrict__ grad_x, float* __restrict__ partial_w,
                  float* __restrict__ partial_b) {
  extern __shared__ __align__(16) float smem_f[];  // w4 (8 KB), then [kWarps][8][dim] + [kWarps][8] partials
  float4* w4 = reinterpret_cast<float4*>(smem_f);
  load_w_lanes<TP>(W, dim, w4);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, head = lane >> 2;
  const bool has_x = lane < (dim >> 3);
  float acc[kWH][8];  // grad_W[h][8 lane + j] over this warp's rows
#pragma unroll
  for (int h = 0; h < kWH; ++h)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[h][j] = 0.f;
  float accb = 0.f;  // grad_b[head] (lanes 4h)
  for (int64_t r = (int64_t)blockIdx.x * kWarps + warp; r < rows; r += (int64_t)gridDim.x * kWarps) {
    const int64_t ab = row_base32(la, r);
    const uint4* gp_in = reinterpret_cast<const uint4*>(grad_out + r * (kWH * kWDh)) + 2 * lane;
    const uint4* ap = reinterpret_cast<const uint4*>(attn + ab) + 2 * lane;
    const uint4 go0 = gp_in[0], go1 = gp_in[1], at0 = ap[0], at1 = ap[1];
    const uint4 xv = has_x ? reinterpret_cast<const uint4*>(x + r * dim)[lane] : make_uint4(0, 0, 0, 0);
    const float gv = Elem<T>::to_f(gate[r * kWH + head]);
    // grad_attn = grad_out * gate, and this lane's share of sum_d grad_out * attn
    float part = 0.f;
    uint4* gap = reinterpret_cast<uint4*>(grad_attn + ab) + 2 * lane;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      float go[8], at[8];
      Vec<T>::unpack(q ? go1 : go0, go);
      Vec<T>::unpack(q ? at1 : at0, at);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        part = fmaf(go[j], at[j], part);
        go[j] *= gv;
      }
      gap[q] = Vec<T>::pack(go);
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    const float gpv = part * gv * (1.0f - gv);  // gate-logit gradient of this lane's head
    if ((lane & 3) == 0) accb += gpv;
    float gph[kWH];
#pragma unroll
    for (int h = 0; h < kWH; ++h) gph[h] = __shfl_sync(0xffffffffu, gpv, 4 * h);
    if (has_x) {
      float xf[8], gx[8];
      Vec<T>::unpack(xv, xf);
#pragma unroll
      for (int j = 0; j < 8; ++j) gx[j] = 0.f;
#pragma unroll
      for (int h = 0; h < kWH; ++h) {
        float w[8];
        w_chunk(w4, h, lane, w);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          gx[j] = fmaf(gph[h], w[j], gx[j]);
          acc[h][j] = fmaf(gph[h], xf[j], acc[h][j]);
        }
      }
      reinterpret_cast<uint4*>(grad_x + r * dim)[lane] = Vec<T>::pack(gx);
    }
  }
  // the CTA's warps combined in warp order: one partial row per CTA
  float* red_w = smem_f + kWH * 2 * 32 * 4;
  float* red_b = red_w + kWarps * kWH * dim;
  if (has_x) {
#pragma unroll
    for (int h = 0; h < kWH; ++h)
#pragma unroll
      for (int j = 0; j < 8; ++j) red_w[(warp * kWH + h) * dim + 8 * lane + j] = acc[h][j];
  }
  if ((lane & 3) == 0) red_b[warp * kWH + head] = accb;
  __syncthreads();
  for (int e = threadIdx.x; e < kWH * dim; e += kThreads) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red_w[w * kWH * dim + e];
    partial_w[(int64_t)blockIdx.x * kWH * dim + e] = s;
  }
  if (threadIdx.x < kWH) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red_b[w * kWH + threadIdx.x];
    partial_b[(int64_t)blockIdx.x * kWH + threadIdx.x] = s;
  }
}

int warp_bwd_smem(int dim) { return (kWH * 2 * 32 * 4 + kWarps * kWH * dim + kWarps * kWH) * 4; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Whether the warp-per-row kernels apply.
bool warp_ok(int es, const AttnLayout& la, int64_t rows, int64_t H, int64_t Dh, int64_t dim,
             std::initializer_list<const void*> ptrs) {
  if (es != 2 || H != kWH || Dh != kWDh || la.s_h != kWDh || dim % 8 != 0 || dim > kWMaxDim) return false;
  if (la.s_b % 8 != 0 || la.s_n % 8 != 0) return false;
  if (rows >= (int64_t)1 << 31 || la.inner * la.seq >= (int64_t)1 << 31) return false;
  for (const void* p : ptrs)
    if (!aligned16(p)) return false;
  return true;
}

// Whether the tiled kernels apply (vector width V = 16 / element size).
bool tiled_ok(int es, const AttnLayout& la, int64_t H, int64_t Dh, int64_t dim, std::initializer_list<const void*> ptrs) {
  const int V = 16 / es;
  if (dim % V != 0 || Dh % V != 0) return false;
  const int64_t vh = Dh / V;
  if (vh > 32 || (vh & (vh - 1)) != 0) return false;
  if (la.s_b % V != 0 || la.s_n % V != 0 || la.s_h % V != 0) return false;
  for (const void* p : ptrs)
    if (!aligned16(p)) return false;
  return TileSmem((int)H, (int)dim, V).bytes <= 200 * 1024;
}

// Whether the streamed kernels apply: contiguous heads in attn (head
// stride = Dh), 16-byte aligned rows of every streamed tensor, whole head
// vectors, and a shared-memory layout that fits two CTAs per SM.
bool stream_ok(int es, const AttnLayout& la, int64_t H, int64_t Dh, int64_t dim, bool bwd,
               std::initializer_list<const void*> ptrs) {
  if (es != 2) return false;  // 16-bit activations: 8-element chunks
  const int V = 8;
  if (la.s_h != Dh || dim % V != 0 || Dh % V != 0 || (H * es) % 16 != 0) return false;
  const int64_t vh = Dh / V, vr = H * vh, nck = dim / V;
  // fixed maps: vr a power of two that divides the block, head vectors in one warp, logits in one pass,
  // grad_x / grad_W items within kMaxChunkItems per thread
  if (vh > 32 || (vh & (vh - 1)) != 0 || (vr & (vr - 1)) != 0 || vr > kThreads) return false;
  if ((int64_t)kStreamRows * H * 4 > kThreads) return false;
  if (kStreamRows * nck > kThreads * kMaxChunkItems || H * nck > kThreads * kMaxChunkItems) return false;
  if (la.s_b % V != 0 || la.s_n % V != 0) return false;
  for (const void* p : ptrs)
    if (!aligned16(p)) return false;
  return StreamLayout((int)H, (int)Dh, (int)dim, es, bwd).bytes <= 110 * 1024;
}

int stream_grid(int64_t rows, int per_sm) {
  const int64_t tiles = (rows + kStreamRows - 1) / kStreamRows;
  const int64_t g = (int64_t)num_sms() * per_sm;
  return (int)(g < tiles ? g : (tiles < 1 ? 1 : tiles));
}

int tiled_grid(int64_t rows, int per_sm, int cap) {
  const int64_t tiles = (rows + kTileRows - 1) / kTileRows;
  int64_t g = (int64_t)num_sms() * per_sm;
  if (g > cap) g = cap;
  if (g > tiles) g = tiles;
  return (int)(g < 1 ? 1 : g);
}

int row_grid(int64_t rows) {
  int64_t g = (rows + kWarps - 1) / kWarps;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }
int64_t chunks_of(int64_t rows) { return (rows + kRowsPerChunk - 1) / kRowsPerChunk; }

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_attention_gate_forward(const void* attn, int64_t seq_len, int64_t attn_stride_batch,
                                          int64_t attn_stride_seq, int64_t attn_stride_head, const void* x,
                                          const void* weight, const void* bias, int64_t rows, int64_t heads,
                                          int64_t dim_head, int64_t dim, void* out, void* gate, int dtype,
                                          int param_dtype, int64_t seq_inner, void* stream) {
  clear_error();
  const char* name = "pmb_attention_gate_forward";
  PMB_REQUIRE(rows >= 0 && heads > 0 && heads <= kMaxHeads && dim_head > 0 && dim > 0 && seq_len > 0,
              "%s: bad shape (heads must be 1..%d)", name, kMaxHeads);
  PMB_REQUIRE(heads * dim * 4 <= 96 * 1024, "%s: heads*dim too large", name);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(attn && x && weight && bias && out && gate, "%s: NULL tensor argument", name);
  PMB_REQUIRE(seq_inner > 0, "%s: seq_inner must be positive", name);
  AttnLayout la{seq_len, attn_stride_batch, attn_stride_seq, attn_stride_head, seq_inner};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)heads * dim * sizeof(float);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 2) {
      if (warp_ok(sizeof(T), la, rows, heads, dim_head, dim, {attn, x, out, gate})) {
        const int64_t want = (rows + kWarps - 1) / kWarps, cap = (int64_t)num_sms() * 3;
        gate_fwd_warp<T, TP><<<(int)(want < cap ? want : cap), kThreads, 0, s>>>(
            static_cast<const T*>(attn), la, static_cast<const T*>(x), static_cast<const TP*>(weight),
            static_cast<const TP*>(bias), rows, (int)dim, static_cast<T*>(out), static_cast<T*>(gate));
        PMB_CHECK_LAUNCH(name);
        return PMB_OK;
      }
    }
    if (stream_ok(sizeof(T), la, heads, dim_head, dim, false, {attn, x, out, gate})) {
      const int bsm = StreamLayout((int)heads, (int)dim_head, (int)dim, sizeof(T), false).bytes;
      PMB_CHECK_CUDA(cudaFuncSetAttribute(gate_fwd_stream<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, bsm),
                     name);
      gate_fwd_stream<T, TP><<<stream_grid(rows, 3), kThreads, bsm, s>>>(
          static_cast<const T*>(attn), la, static_cast<const T*>(x), static_cast<const TP*>(weight),
          static_cast<const TP*>(bias), rows, (int)heads, (int)dim_head, (int)dim, static_cast<T*>(out),
          static_cast<T*>(gate));
      PMB_CHECK_LAUNCH(name);
      return PMB_OK;
    }
    if (tiled_ok(sizeof(T), la, heads, dim_head, dim, {attn, x, out})) {
      const size_t tsm = TileSmem((int)heads, (int)dim, Vec<T>::N).bytes;
      if (tsm > 48 * 1024)
        PMB_CHECK_CUDA(
            cudaFuncSetAttribute(gate_fwd_tiled<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm), name);
      gate_fwd_tiled<T, TP><<<tiled_grid(rows, 8, 1 << 20), kThreads, tsm, s>>>(
          static_cast<const T*>(attn), la, static_cast<const T*>(x), static_cast<const TP*>(weight),
          static_cast<const TP*>(bias), rows, (int)heads, (int)dim_head, (int)dim, static_cast<T*>(out),
          static_cast<T*>(gate));
      PMB_CHECK_LAUNCH(name);
      return PMB_OK;
    }
    if (smem > 48 * 1024)
      PMB_CHECK_CUDA(cudaFuncSetAttribute(gate_fwd<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                     name);
    gate_fwd<T, TP><<<row_grid(rows), kThreads, smem, s>>>(
        static_cast<const T*>(attn), la, static_cast<const T*>(x), static_cast<const TP*>(weight),
        static_cast<const TP*>(bias), rows, (int)heads, (int)dim_head, (int)dim, static_cast<T*>(out),
        static_cast<T*>(gate));
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}

extern "C" int64_t pmb_attention_gate_backward_workspace_size(int64_t rows, int64_t heads, int64_t dim) {
  if (rows <= 0 || heads <= 0 || dim <= 0) return 0;
  const int64_t rowwise = align256(rows * heads * 4) + align256(chunks_of(rows) * heads * (dim + 1) * 4);
  const int64_t tiled = align256((int64_t)kMaxTiledBwdBlocks * heads * dim * 4) +
                        align256((int64_t)kMaxTiledBwdBlocks * heads * 4);
  return rowwise > tiled ? rowwise : tiled;
}

extern "C" int pmb_attention_gate_backward(const void* grad_out, const void* attn, int64_t seq_len,
                                           int64_t attn_stride_batch, int64_t attn_stride_seq,
                                           int64_t attn_stride_head, const void* x, const void* weight,
                                           const void* gate, int64_t rows, int64_t heads, int64_t dim_head,
                                           int64_t dim, void* grad_attn, void* grad_x, void* grad_weight,
                                           void* grad_bias, int dtype, int param_dtype, void* workspace,
                                           int64_t workspace_bytes, int64_t seq_inner, void* stream) {
  clear_error();
  const char* name = "pmb_attention_gate_backward";
  PMB_REQUIRE(rows >= 0 && heads > 0 && heads <= kMaxHeads && dim_head > 0 && dim > 0 && seq_len > 0,
              "%s: bad shape (heads must be 1..%d)", name, kMaxHeads);
  PMB_REQUIRE(heads * dim * 4 <= 96 * 1024, "%s: heads*dim too large", name);
  PMB_REQUIRE(grad_weight && grad_bias, "%s: NULL gradient argument", name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int es = dtype_size(param_dtype);
  PMB_REQUIRE(es > 0, "%s: unsupported parameter dtype %d", name, param_dtype);
  if (rows == 0) {
    PMB_CHECK_CUDA(cudaMemsetAsync(grad_weight, 0, heads * dim * es, s), name);
    PMB_CHECK_CUDA(cudaMemsetAsync(grad_bias, 0, heads * es, s), name);
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && attn && x && weight && gate && grad_attn && grad_x, "%s: NULL tensor argument", name);
  const int64_t need = pmb_attention_gate_backward_workspace_size(rows, heads, dim);
  if (workspace == nullptr || workspace_bytes < need) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  float* ggp = static_cast<float*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + align256(rows * heads * 4));
  PMB_REQUIRE(seq_inner > 0, "%s: seq_inner must be positive", name);
  AttnLayout la{seq_len, attn_stride_batch, attn_stride_seq, attn_stride_head, seq_inner};
  const size_t smem = (size_t)heads * dim * sizeof(float);
  return PMB_DISPATCH_PARAM(dtype, param_dtype, T, TP, name, [&] {
    if constexpr (sizeof(T) == 2) {
      if (warp_ok(sizeof(T), la, rows, heads, dim_head, dim, {grad_out, attn, x, gate, grad_attn, grad_x})) {
        const int bsm = warp_bwd_smem((int)dim);
        PMB_CHECK_CUDA(cudaFuncSetAttribute(gate_bwd_warp<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, bsm),
                       name);
        const int64_t want = (rows + kWarps - 1) / kWarps, cap = (int64_t)num_sms() * 2;  // <= kMaxTiledBwdBlocks
        const int grid = (int)(want < cap ? want : cap);
        float* pw = static_cast<float*>(workspace);
        float* pb = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                             align256((int64_t)kMaxTiledBwdBlocks * heads * dim * 4));
        gate_bwd_warp<T, TP><<<grid, kThreads, bsm, s>>>(
            static_cast<const T*>(grad_out), static_cast<const T*>(attn), la, static_cast<const T*>(x),
            static_cast<const TP*>(weight), static_cast<const T*>(gate), rows, (int)dim, static_cast<T*>(grad_attn),
            static_cast<T*>(grad_x), pw, pb);
        PMB_CHECK_LAUNCH(name);
        red::colsum_rows<<<red::colsum_rows_grid(heads * dim), red::kThreads, 0, s>>>(pw, grid, heads * dim, grad_weight,
                                                                                 Elem<TP>::code);
        PMB_CHECK_LAUNCH(name);
        red::colsum_rows<<<red::colsum_rows_grid(heads), red::kThreads, 0, s>>>(pb, grid, heads, grad_bias,
                                                                           Elem<TP>::code);
        PMB_CHECK_LAUNCH(name);
        return PMB_OK;
      }
    }
    if (stream_ok(sizeof(T), la, heads, dim_head, dim, true, {grad_out, attn, x, gate, grad_attn, grad_x})) {
      const int bsm = StreamLayout((int)heads, (int)dim_head, (int)dim, sizeof(T), true).bytes;
      PMB_CHECK_CUDA(cudaFuncSetAttribute(gate_bwd_stream<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, bsm),
                     name);
      const int grid = stream_grid(rows, 3);  // <= 3 x SMs <= kMaxTiledBwdBlocks partial rows
      float* pw = static_cast<float*>(workspace);
      float* pb = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                           align256((int64_t)kMaxTiledBwdBlocks * heads * dim * 4));
      gate_bwd_stream<T, TP><<<grid, kThreads, bsm, s>>>(
          static_cast<const T*>(grad_out), static_cast<const T*>(attn), la, static_cast<const T*>(x),
          static_cast<const TP*>(weight), static_cast<const T*>(gate), rows, (int)heads, (int)dim_head, (int)dim,
          static_cast<T*>(grad_attn), static_cast<T*>(grad_x), pw, pb);
      PMB_CHECK_LAUNCH(name);
      red::colsum_rows<<<red::colsum_rows_grid(heads * dim), red::kThreads, 0, s>>>(pw, grid, heads * dim, grad_weight,
                                                                               Elem<TP>::code);
      PMB_CHECK_LAUNCH(name);
      red::colsum_rows<<<red::colsum_rows_grid(heads), red::kThreads, 0, s>>>(pb, grid, heads, grad_bias,
                                                                         Elem<TP>::code);
      PMB_CHECK_LAUNCH(name);
      return PMB_OK;
    }
    if (heads * dim <= kThreads * kMaxWPerThread &&
        tiled_ok(sizeof(T), la, heads, dim_head, dim, {grad_out, attn, x, grad_attn, grad_x})) {
      const size_t tsm = TileSmem((int)heads, (int)dim, Vec<T>::N).bytes;
      if (tsm > 48 * 1024)
        PMB_CHECK_CUDA(
            cudaFuncSetAttribute(gate_bwd_tiled<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm), name);
      const int grid = tiled_grid(rows, 4, kMaxTiledBwdBlocks);
      float* pw = static_cast<float*>(workspace);
      float* pb = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                           align256((int64_t)kMaxTiledBwdBlocks * heads * dim * 4));
      gate_bwd_tiled<T, TP><<<grid, kThreads, tsm, s>>>(
          static_cast<const T*>(grad_out), static_cast<const T*>(attn), la, static_cast<const T*>(x),
          static_cast<const TP*>(weight), static_cast<const T*>(gate), rows, (int)heads, (int)dim_head, (int)dim,
          static_cast<T*>(grad_attn), static_cast<T*>(grad_x), pw, pb);
      PMB_CHECK_LAUNCH(name);
      red::colsum_rows<<<red::colsum_rows_grid(heads * dim), red::kThreads, 0, s>>>(pw, grid, heads * dim, grad_weight,
                                                                               Elem<TP>::code);
      PMB_CHECK_LAUNCH(name);
      red::colsum_rows<<<red::colsum_rows_grid(heads), red::kThreads, 0, s>>>(pb, grid, heads, grad_bias,
                                                                         Elem<TP>::code);
      PMB_CHECK_LAUNCH(name);
      return PMB_OK;
    }
    if (smem > 48 * 1024)
      PMB_CHECK_CUDA(
          cudaFuncSetAttribute(gate_bwd_rows<T, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), name);
    gate_bwd_rows<T, TP><<<row_grid(rows), kThreads, smem, s>>>(
        static_cast<const T*>(grad_out), static_cast<const T*>(attn), la, static_cast<const TP*>(weight),
        static_cast<const T*>(gate), rows, (int)heads, (int)dim_head, (int)dim, static_cast<T*>(grad_attn),
        static_cast<T*>(grad_x), ggp);
    PMB_CHECK_LAUNCH(name);
    const int cols = (int)(heads * (dim + 1));
    const int nch = (int)chunks_of(rows);
    dim3 gp((cols + kThreads - 1) / kThreads, nch);
    gate_bwd_weight_partial<T><<<gp, kThreads, 0, s>>>(ggp, static_cast<const T*>(x), rows, (int)heads, (int)dim,
                                                       partial);
    PMB_CHECK_LAUNCH(name);
    gate_bwd_weight_finalize<TP><<<(cols + kThreads - 1) / kThreads, kThreads, 0, s>>>(
        partial, nch, (int)heads, (int)dim, static_cast<TP*>(grad_weight), static_cast<TP*>(grad_bias));
    PMB_CHECK_LAUNCH(name);
    return PMB_OK;
  });
}
