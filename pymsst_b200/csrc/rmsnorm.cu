// Transformer RMSNorm (F.normalize(x) * sqrt(D) * gamma) forward and backward.
//
// One warp owns one row at a time; a lane keeps its slice of the row in
// registers as 16-byte vectors (8 x 16-bit or 4 x fp32 elements), so x is read
// exactly once, and the row sum of squares is a warp shuffle reduction.  The
// backward produces grad_gamma deterministically: each CTA reduces its rows
// into one fp32 partial row in the caller's workspace, and a second launch
// sums the partials column-wise (coalesced).  Reference semantics:
// src/pymsst/training/cuda/fused_band_split.cu:1211-1315 (formulas at
// :1237-1247 and :1263-1286).
#include <mutex>

#include <type_traits>

#include "common.cuh"
#include "reduce.cuh"
#include "umma.cuh"

namespace pmb {
unsigned int timeout_flag_rms(int reset) { return umma::flag_reader(reset); }

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBwdBlocks = 4 * 148;

__device__ __forceinline__ float ld_dyn(const void* p, int64_t i, int code) {
  switch (code) {
    case PMB_FLOAT16:
      return __half2float(static_cast<const __half*>(p)[i]);
    case PMB_BFLOAT16:
      return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    default:
      return static_cast<const float*>(p)[i];
  }
}

template <typename T, int V>
struct alignas((sizeof(T) * V) < 16 ? (sizeof(T) * V) : 16) Pack {
  T v[V];
};

// ---------------------------------------------------------------- forward
template <typename Tx, typename To, int V, int NJ>
__global__ void __launch_bounds__(kThreads)
    rms_fwd_vec(const Tx* __restrict__ x, const void* __restrict__ gamma, int gcode,
                To* __restrict__ out, To* __restrict__ normed, float* __restrict__ inv_norm,
                int64_t rows, int dim) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  const int nvec = dim / V;
  const float scale = sqrtf((float)dim);

  float g[NJ][V];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int vi = j * 32 + lane;
#pragma unroll
    for (int e = 0; e < V; ++e) g[j][e] = vi < nvec ? ld_dyn(gamma, (int64_t)vi * V + e, gcode) : 0.f;
  }

  for (int64_t r = warp; r < rows; r += nwarps) {
    const Tx* xr = x + r * dim;
    float v[NJ][V];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int vi = j * 32 + lane;
      if (vi < nvec) {
        const Pack<Tx, V> p = *reinterpret_cast<const Pack<Tx, V>*>(xr + (int64_t)vi * V);
#pragma unroll
        for (int e = 0; e < V; ++e) {
          v[j][e] = Elem<Tx>::to_f(p.v[e]);
          ss += v[j][e] * v[j][e];
        }
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) v[j][e] = 0.f;
      }
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / fmaxf(sqrtf(ss), 1.0e-12f);
    if (lane == 0) inv_norm[r] = inv;
    const float k = inv * scale;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int vi = j * 32 + lane;
      if (vi < nvec) {
        Pack<To, V> po, pn;
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const float n = v[j][e] * k;
          pn.v[e] = Elem<To>::from_f(n);
          po.v[e] = Elem<To>::from_f(n * g[j][e]);
        }
        *reinterpret_cast<Pack<To, V>*>(out + r * dim + (int64_t)vi * V) = po;
        if (normed != nullptr) *reinterpret_cast<Pack<To, V>*>(normed + r * dim + (int64_t)vi * V) = pn;
      }
    }
  }
}

// Any dim / alignment: the row is streamed twice instead of held in registers.
template <typename Tx, typename To>
__global__ void __launch_bounds__(kThreads)
    rms_fwd_generic(const Tx* __restrict__ x, const void* __restrict__ gamma, int gcode,
                    To* __restrict__ out, To* __restrict__ normed, float* __restrict__ inv_norm,
                    int64_t rows, int dim) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  const float scale = sqrtf((float)dim);
  for (int64_t r = warp; r < rows; r += nwarps) {
    const Tx* xr = x + r * dim;
    float ss = 0.f;
    for (int c = lane; c < dim; c += 32) {
      const float v = Elem<Tx>::to_f(xr[c]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / fmaxf(sqrtf(ss), 1.0e-12f);
    if (lane == 0) inv_norm[r] = inv;
    for (int c = lane; c < dim; c += 32) {
      const float n = Elem<Tx>::to_f(xr[c]) * inv * scale;
      out[r * dim + c] = Elem<To>::from_f(n * ld_dyn(gamma, c, gcode));
      if (normed != nullptr) normed[r * dim + c] = Elem<To>::from_f(n);
    }
  }
}

// --------------------------------------------------------------- backward
// The residual branch's gradient added to grad_x (nullable: zeros), V values from element i (16-byte aligned).
template <typename Tdx, int V>
__device__ __forceinline__ void load_res(const Tdx* __restrict__ dres, int64_t i, float (&add)[V]) {
  if (dres == nullptr) {
#pragma unroll
    for (int e = 0; e < V; ++e) add[e] = 0.f;
    return;
  }
  if constexpr (sizeof(Tdx) * V == 16) {
    const Pack<Tdx, V> pr = *reinterpret_cast<const Pack<Tdx, V>*>(dres + i);
#pragma unroll
    for (int e = 0; e < V; ++e) add[e] = Elem<Tdx>::to_f(pr.v[e]);
  } else {
#pragma unroll
    for (int e = 0; e < V; ++e) add[e] = Elem<Tdx>::to_f(dres[i + e]);
  }
}

template <typename Tg, typename Tdx, int V, int NJ>
__global__ void __launch_bounds__(kThreads)
    rms_bwd_vec(const Tg* __restrict__ dy, const Tg* __restrict__ saved, int saved_is_input,
                const float* __restrict__ inv_norm, const void* __restrict__ gamma, int gcode,
                Tdx* __restrict__ dx, const Tdx* __restrict__ dres, float* __restrict__ partial, int64_t rows,
                int dim) {
  extern __shared__ float red[];  // [kWarps][dim]
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int64_t warp = (int64_t)blockIdx.x * kWarps + wib;
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  const int nvec = dim / V;
  const float scale = sqrtf((float)dim);

  float g[NJ][V], acc[NJ][V];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int vi = j * 32 + lane;
#pragma unroll
    for (int e = 0; e < V; ++e) {
      g[j][e] = vi < nvec ? ld_dyn(gamma, (int64_t)vi * V + e, gcode) : 0.f;
      acc[j][e] = 0.f;
    }
  }

  for (int64_t r = warp; r < rows; r += nwarps) {
    const float inv = inv_norm[r];
    const float nk = saved_is_input ? inv * scale : 1.0f;
    float gd[NJ][V], nv[NJ][V];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int vi = j * 32 + lane;
      if (vi < nvec) {
        const Pack<Tg, V> pd = *reinterpret_cast<const Pack<Tg, V>*>(dy + r * dim + (int64_t)vi * V);
        const Pack<Tg, V> ps = *reinterpret_cast<const Pack<Tg, V>*>(saved + r * dim + (int64_t)vi * V);
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const float d = Elem<Tg>::to_f(pd.v[e]);
          const float n = Elem<Tg>::to_f(ps.v[e]) * nk;
          nv[j][e] = n;
          gd[j][e] = d * g[j][e];
          dot += gd[j][e] * n;
          acc[j][e] += d * n;
        }
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) gd[j][e] = nv[j][e] = 0.f;
      }
    }
    dot = warp_sum(dot);
    if (dx != nullptr) {
      const float ds = dot / scale;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int vi = j * 32 + lane;
        if (vi < nvec) {
          float add[V];
          load_res<Tdx, V>(dres, r * dim + (int64_t)vi * V, add);
          Pack<Tdx, V> p;
#pragma unroll
          for (int e = 0; e < V; ++e) p.v[e] = Elem<Tdx>::from_f(inv * (gd[j][e] * scale - nv[j][e] * ds) + add[e]);
          *reinterpret_cast<Pack<Tdx, V>*>(dx + r * dim + (int64_t)vi * V) = p;
        }
      }
    }
  }

#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int vi = j * 32 + lane;
    if (vi < nvec) {
#pragma unroll
      for (int e = 0; e < V; ++e) red[wib * dim + vi * V + e] = acc[j][e];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < dim; c += kThreads) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w * dim + c];
    partial[(int64_t)blockIdx.x * dim + c] = s;
  }
}

template <typename Tg, typename Tdx>
__global__ void __launch_bounds__(kThreads)
    rms_bwd_generic(const Tg* __restrict__ dy, const Tg* __restrict__ saved, int saved_is_input,
                    const float* __restrict__ inv_norm, const void* __restrict__ gamma, int gcode,
                    Tdx* __restrict__ dx, const Tdx* __restrict__ dres, float* __restrict__ partial, int64_t rows,
                    int dim) {
  // Column-parallel partials: each thread owns columns c = tid, tid+256, ...
  // and walks this CTA's rows; the row dot product is a CTA reduction.
  __shared__ float sdot[kWarps];
  const float scale = sqrtf((float)dim);
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  for (int c = threadIdx.x; c < dim; c += kThreads) partial[(int64_t)blockIdx.x * dim + c] = 0.f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float inv = inv_norm[r];
    const float nk = saved_is_input ? inv * scale : 1.0f;
    float dot = 0.f;
    for (int c = threadIdx.x; c < dim; c += kThreads) {
      const float d = Elem<Tg>::to_f(dy[r * dim + c]);
      const float n = Elem<Tg>::to_f(saved[r * dim + c]) * nk;
      dot += d * ld_dyn(gamma, c, gcode) * n;
      partial[(int64_t)blockIdx.x * dim + c] += d * n;
    }
    dot = warp_sum(dot);
    if (lane == 0) sdot[wib] = dot;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot += sdot[w];
    __syncthreads();
    if (dx != nullptr) {
      const float ds = tot / scale;
      for (int c = threadIdx.x; c < dim; c += kThreads) {
        const float d = Elem<Tg>::to_f(dy[r * dim + c]);
        const float n = Elem<Tg>::to_f(saved[r * dim + c]) * nk;
        const float add = dres != nullptr ? Elem<Tdx>::to_f(dres[r * dim + c]) : 0.f;
        dx[r * dim + c] = Elem<Tdx>::from_f(inv * (d * ld_dyn(gamma, c, gcode) * scale - n * ds) + add);
      }
    }
  }
}

// ------------------------------------------------- bulk-staged (TMA) path
// Rows are contiguous, so a tile of consecutive rows is one contiguous block:
// one thread streams tiles into a kStages-deep shared-memory ring with
// cp.async.bulk (mbarrier completion), keeping up to kStages tiles per CTA in
// flight without holding registers, and the warps normalise rows out of
// shared memory.  Persistent CTAs; tiles t = blockIdx.x + i * gridDim.x.
constexpr int kStages = 4;
constexpr int kFwdStageBytes = 12288;
constexpr int kBwdStageBytes = 8192;  // per input (dy, saved)
// With the residual gradient as a third input: 3 stages of 12 KB per input, so a tile of the model's 192-wide
// 16-bit rows holds 32 rows (every row slot of the 8 warps busy) at 2 CTAs per SM.
constexpr int kBwdStageBytesRes = 12288;
constexpr int kBwdStagesRes = 3;

constexpr int kMaxBulkDim = 1024;  // gamma staged as fp32 after the ring and the barriers

template <int STAGE_BYTES, int INPUTS, int STAGES = kStages>
constexpr int bulk_smem_bytes() {
  return STAGES * STAGE_BYTES * INPUTS + 128 + kMaxBulkDim * 4;
}

// gamma as fp32 into shared memory (whole CTA; followed by the caller's barrier)
__device__ __forceinline__ void stage_gamma(const void* gamma, int gcode, int dim, float* g_s) {
  for (int c = threadIdx.x; c < dim; c += kThreads) g_s[c] = ld_dyn(gamma, c, gcode);
}

// Lane layout of the bulk kernels: G lanes per row (G = 8, 16 or 32), so a
// warp works on 32 / G rows at once and every lane is busy; lane l of a row
// group owns the 16-byte vectors l, l + G, ... (NJ of them).
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename Tx, typename To, int V, int G, int NJ>
__global__ void __launch_bounds__(kThreads, 4)
    rms_fwd_bulk(const Tx* __restrict__ x, const void* __restrict__ gamma, int gcode, To* __restrict__ out,
                 To* __restrict__ normed, float* __restrict__ inv_norm, int64_t rows, int dim, int rpt) {
  constexpr int RW = 32 / G;  // rows per warp step
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kFwdStageBytes);
  float* g_s = reinterpret_cast<float*>(smem + kStages * kFwdStageBytes + 128);
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int gl = lane % G, sub = lane / G;
  stage_gamma(gamma, gcode, dim, g_s);
  const int nvec = dim / V;
  const float scale = sqrtf((float)dim);
  const int64_t tiles = (rows + rpt - 1) / rpt;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; ++st) umma::mbar_init(&full[st], 1);
    umma::fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int64_t tile, int st) {
    const int64_t r0 = tile * rpt;
    const int64_t n = rows - r0 < rpt ? rows - r0 : rpt;
    const uint32_t bytes = (uint32_t)(n * dim * (int64_t)sizeof(Tx));
    umma::mbar_arrive_expect_tx(&full[st], bytes);
    umma::bulk_load(smem + st * kFwdStageBytes, x + r0 * dim, bytes, &full[st]);
  };
  if (threadIdx.x == 0)
    for (int st = 0; st < kStages; ++st) {
      const int64_t t = blockIdx.x + (int64_t)st * gridDim.x;
      if (t < tiles) issue(t, st);
    }
  int it = 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
    const int st = it % kStages;
    // every thread takes the same decision, so no thread is left at a barrier
    if (__syncthreads_or(!umma::mbar_wait(&full[st], (it / kStages) & 1, 0x21))) break;
    Tx* xs = reinterpret_cast<Tx*>(smem + st * kFwdStageBytes);
    const int64_t r0 = tile * rpt;
    const int n = rows - r0 < rpt ? (int)(rows - r0) : rpt;
    for (int qb = wib * RW; qb < n; qb += kWarps * RW) {
      const int q = qb + sub;
      const bool live = q < n;
      float v[NJ][V];
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int vi = j * G + gl;
        if (live && vi < nvec) {
          const Pack<Tx, V> p = *reinterpret_cast<const Pack<Tx, V>*>(xs + q * dim + vi * V);
#pragma unroll
          for (int e = 0; e < V; ++e) {
            v[j][e] = Elem<Tx>::to_f(p.v[e]);
            ss += v[j][e] * v[j][e];
          }
        } else {
#pragma unroll
          for (int e = 0; e < V; ++e) v[j][e] = 0.f;
        }
      }
      ss = group_sum<G>(ss);
      if (!live) continue;
      const int64_t r = r0 + q;
      const float inv = 1.0f / fmaxf(sqrtf(ss), 1.0e-12f);
      if (gl == 0) inv_norm[r] = inv;
      const float k = inv * scale;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int vi = j * G + gl;
        if (vi < nvec) {
          Pack<To, V> po, pn;
          const float* gv = g_s + vi * V;
#pragma unroll
          for (int e = 0; e < V; ++e) {
            const float nrm = v[j][e] * k;
            pn.v[e] = Elem<To>::from_f(nrm);
            po.v[e] = Elem<To>::from_f(nrm * gv[e]);
          }
          // out goes back over this lane's own x elements (sizeof(To) == sizeof(Tx)) and leaves by bulk store
          *reinterpret_cast<Pack<To, V>*>(reinterpret_cast<To*>(xs) + q * dim + vi * V) = po;
          if (normed != nullptr) *reinterpret_cast<Pack<To, V>*>(normed + r * dim + (int64_t)vi * V) = pn;
        }
      }
    }
    umma::fence_proxy_async_smem();
    __syncthreads();  // every warp is done with stage st
    if (threadIdx.x == 0) {
      umma::bulk_store(out + r0 * dim, xs, (uint32_t)(n * dim * (int64_t)sizeof(To)));
      umma::bulk_commit();
      const int64_t nt = tile + (int64_t)kStages * gridDim.x;
      if (nt < tiles) {
        umma::bulk_wait_read_all();  // the store has read the stage before the next load refills it
        issue(nt, st);
      }
    }
  }
  if (threadIdx.x == 0) umma::bulk_wait_all();
}

// RES: a third input, the residual branch's gradient (Tdx, same layout as dx), staged through the same ring
// and added to grad_x.
template <typename Tg, typename Tdx, int V, int G, int NJ, bool RES>
__global__ void __launch_bounds__(kThreads, RES ? 2 : 3)
    rms_bwd_bulk(const Tg* __restrict__ dy, const Tg* __restrict__ saved, int saved_is_input,
                 const float* __restrict__ inv_norm, const void* __restrict__ gamma, int gcode, Tdx* __restrict__ dx,
                 const Tdx* __restrict__ dres, float* __restrict__ partial, int64_t rows, int dim, int rpt) {
  constexpr int RW = 32 / G;
  constexpr int IN = RES ? 3 : 2;  // staged inputs per ring slot
  constexpr int SB = RES ? kBwdStageBytesRes : kBwdStageBytes;  // bytes per input per slot
  constexpr int NS = RES ? kBwdStagesRes : kStages;              // ring slots
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB * IN);
  float* g_s = reinterpret_cast<float*>(smem + NS * SB * IN + 128);
  float* red = reinterpret_cast<float*>(smem);  // reused after the ring drains: [kWarps * RW][dim]
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int gl = lane % G, sub = lane / G;
  stage_gamma(gamma, gcode, dim, g_s);
  const int nvec = dim / V;
  const float scale = sqrtf((float)dim);
  const int64_t tiles = (rows + rpt - 1) / rpt;
  if (threadIdx.x == 0) {
    for (int st = 0; st < NS; ++st) umma::mbar_init(&full[st], 1);
    umma::fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int64_t tile, int st) {
    const int64_t r0 = tile * rpt;
    const int64_t n = rows - r0 < rpt ? rows - r0 : rpt;
    const uint32_t bytes = (uint32_t)(n * dim * (int64_t)sizeof(Tg));
    uint8_t* base = smem + st * SB * IN;
    umma::mbar_arrive_expect_tx(&full[st], IN * bytes);
    umma::bulk_load(base, dy + r0 * dim, bytes, &full[st]);
    umma::bulk_load(base + SB, saved + r0 * dim, bytes, &full[st]);
    if constexpr (RES) umma::bulk_load(base + 2 * SB, dres + r0 * dim, bytes, &full[st]);
  };
  if (threadIdx.x == 0)
    for (int st = 0; st < NS; ++st) {
      const int64_t t = blockIdx.x + (int64_t)st * gridDim.x;
      if (t < tiles) issue(t, st);
    }
  float acc[NJ][V];
#pragma unroll
  for (int j = 0; j < NJ; ++j)
#pragma unroll
    for (int e = 0; e < V; ++e) acc[j][e] = 0.f;
  int it = 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
    const int st = it % NS;
    const int64_t r0 = tile * rpt;
    const int n = rows - r0 < rpt ? (int)(rows - r0) : rpt;
    // this warp's row norms for the tile, one load per lane, before the wait
    const int qi = wib * RW + (lane / RW) * kWarps * RW + (lane % RW);
    const float inv_l = qi < n ? inv_norm[r0 + qi] : 0.f;
    // every thread takes the same decision, so no thread is left at a barrier
    if (__syncthreads_or(!umma::mbar_wait(&full[st], (it / NS) & 1, 0x22))) break;
    Tg* ds_ = reinterpret_cast<Tg*>(smem + st * SB * IN);
    const Tg* ss_ = reinterpret_cast<const Tg*>(smem + st * SB * IN + SB);
    const Tdx* rs_ = reinterpret_cast<const Tdx*>(smem + st * SB * IN + 2 * SB);
    int step = 0;
    for (int qb = wib * RW; qb < n; qb += kWarps * RW, ++step) {
      const int q = qb + sub;
      const bool live = q < n;
      // row q = wib*RW + step*kWarps*RW + sub is held by lane step*RW + sub
      const float inv = __shfl_sync(0xffffffffu, inv_l, (step * RW + sub) & 31);
      const float nk = saved_is_input ? inv * scale : 1.0f;
      // pass 1: row dot product (gamma-weighted) and the grad_gamma terms
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int vi = j * G + gl;
        if (live && vi < nvec) {
          const Pack<Tg, V> pd = *reinterpret_cast<const Pack<Tg, V>*>(ds_ + q * dim + vi * V);
          const Pack<Tg, V> ps = *reinterpret_cast<const Pack<Tg, V>*>(ss_ + q * dim + vi * V);
          const float* gv = g_s + vi * V;
#pragma unroll
          for (int e = 0; e < V; ++e) {
            const float d = Elem<Tg>::to_f(pd.v[e]);
            const float nn = Elem<Tg>::to_f(ps.v[e]) * nk;
            dot += d * gv[e] * nn;
            acc[j][e] += d * nn;
          }
        }
      }
      dot = group_sum<G>(dot);
      // pass 2: grad_x from the staged row again
      if (dx != nullptr && live) {
        const float dsc = dot / scale;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const int vi = j * G + gl;
          if (vi < nvec) {
            const Pack<Tg, V> pd = *reinterpret_cast<const Pack<Tg, V>*>(ds_ + q * dim + vi * V);
            const Pack<Tg, V> ps = *reinterpret_cast<const Pack<Tg, V>*>(ss_ + q * dim + vi * V);
            const float* gv = g_s + vi * V;
            float add[V];
            if constexpr (RES) {
              const Pack<Tdx, V> pr = *reinterpret_cast<const Pack<Tdx, V>*>(rs_ + q * dim + vi * V);
#pragma unroll
              for (int e = 0; e < V; ++e) add[e] = Elem<Tdx>::to_f(pr.v[e]);
            } else {
#pragma unroll
              for (int e = 0; e < V; ++e) add[e] = 0.f;
            }
            Pack<Tdx, V> p;
#pragma unroll
            for (int e = 0; e < V; ++e) {
              const float d = Elem<Tg>::to_f(pd.v[e]);
              const float nn = Elem<Tg>::to_f(ps.v[e]) * nk;
              p.v[e] = Elem<Tdx>::from_f(inv * (d * gv[e] * scale - nn * dsc) + add[e]);
            }
            // dx goes back over this lane's own dy elements (sizeof(Tdx) == sizeof(Tg)), bulk-stored below
            *reinterpret_cast<Pack<Tdx, V>*>(reinterpret_cast<Tdx*>(ds_) + q * dim + vi * V) = p;
          }
        }
      }
    }
    umma::fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
      if (dx != nullptr) {
        umma::bulk_store(dx + r0 * dim, ds_, (uint32_t)(n * dim * (int64_t)sizeof(Tdx)));
        umma::bulk_commit();
      }
      const int64_t nt = tile + (int64_t)NS * gridDim.x;
      if (nt < tiles) {
        if (dx != nullptr) umma::bulk_wait_read_all();
        issue(nt, st);
      }
    }
  }
  if (threadIdx.x == 0) umma::bulk_wait_read_all();
  // every stage has been consumed and read by its store; reuse the ring for
  // the cross-warp reduction of the grad_gamma partials
  __syncthreads();
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int vi = j * G + gl;
    if (vi < nvec) {
#pragma unroll
      for (int e = 0; e < V; ++e) red[(wib * RW + sub) * dim + vi * V + e] = acc[j][e];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < dim; c += kThreads) {
    float s2 = 0.f;
    for (int w = 0; w < kWarps * RW; ++w) s2 += red[w * dim + c];
    partial[(int64_t)blockIdx.x * dim + c] = s2;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int grid_for_rows(int64_t rows, int64_t cap) {
  int64_t blocks = (rows + kWarps - 1) / kWarps;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

template <typename Tx, typename To>
int launch_fwd(const void* x, const void* gamma, int gcode, void* out, void* normed, float* inv,
               int64_t rows, int64_t dim, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(Tx);
  const int grid = grid_for_rows(rows, (int64_t)num_sms() * 16);
  const int64_t nvec = dim / V;
  const bool vec_ok = dim % V == 0 && aligned16(x) && aligned16(out) && (normed == nullptr || aligned16(normed)) &&
                      (dim * (int64_t)sizeof(Tx)) % 16 == 0 && (dim * (int64_t)sizeof(To)) % 16 == 0;
  const int nj = (int)((nvec + 31) / 32);
  const Tx* xp = static_cast<const Tx*>(x);
  To* op = static_cast<To*>(out);
  To* np = static_cast<To*>(normed);
  const int64_t row_bytes = dim * (int64_t)sizeof(Tx);
  if (vec_ok && sizeof(Tx) == sizeof(To) && dim <= kMaxBulkDim && row_bytes <= kFwdStageBytes) {
    const int rpt = (int)(kFwdStageBytes / row_bytes);
    const int64_t tiles = (rows + rpt - 1) / rpt;
    int g = (int)(tiles < (int64_t)num_sms() * 4 ? tiles : (int64_t)num_sms() * 4);
    constexpr int smem = bulk_smem_bytes<kFwdStageBytes, 1>();
    auto go = [&](auto kern) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      kern<<<g, kThreads, smem, stream>>>(xp, gamma, gcode, op, np, inv, rows, (int)dim, rpt);
    };
    if (nvec <= 8)
      go(rms_fwd_bulk<Tx, To, V, 8, 1>);
    else if (nvec <= 24)
      go(rms_fwd_bulk<Tx, To, V, 8, 3>);
    else if (nvec <= 48)
      go(rms_fwd_bulk<Tx, To, V, 16, 3>);
    else if (nvec <= 64)
      go(rms_fwd_bulk<Tx, To, V, 32, 2>);
    else if (nvec <= 128)
      go(rms_fwd_bulk<Tx, To, V, 32, 4>);
    else if constexpr (V == 4)
      go(rms_fwd_bulk<Tx, To, V, 32, 8>);
  } else if (vec_ok && nj * 32 * V <= 1024) {
    if (nj <= 1)
      rms_fwd_vec<Tx, To, V, 1><<<grid, kThreads, 0, stream>>>(xp, gamma, gcode, op, np, inv, rows, (int)dim);
    else if (nj <= 2)
      rms_fwd_vec<Tx, To, V, 2><<<grid, kThreads, 0, stream>>>(xp, gamma, gcode, op, np, inv, rows, (int)dim);
    else if (nj <= 4)
      rms_fwd_vec<Tx, To, V, 4><<<grid, kThreads, 0, stream>>>(xp, gamma, gcode, op, np, inv, rows, (int)dim);
    else if constexpr (V == 4)
      rms_fwd_vec<Tx, To, V, 8><<<grid, kThreads, 0, stream>>>(xp, gamma, gcode, op, np, inv, rows, (int)dim);
  } else {
    rms_fwd_generic<Tx, To><<<grid, kThreads, 0, stream>>>(xp, gamma, gcode, op, np, inv, rows, (int)dim);
  }
  PMB_CHECK_LAUNCH("pmb_rms_norm_forward");
  return PMB_OK;
}

int bwd_blocks(int64_t rows) { return grid_for_rows(rows, kMaxBwdBlocks); }
int64_t max_bwd_grid(int64_t rows) { return rows < kMaxBwdBlocks ? rows : kMaxBwdBlocks; }

// Rows per bulk backward tile: a lane prefetches the norm of one row of its
// warp per step, so a warp covers at most 32 rows and a tile kWarps * 32.
constexpr int kMaxBwdTileRows = kWarps * 32;

template <typename Tg, typename Tdx>
int launch_bwd(const void* dy, const void* saved, int saved_is_input, const float* inv, const void* gamma,
               int gcode, void* dx, const void* dres, void* dgamma, int dgcode, int64_t rows, int64_t dim,
               float* partial, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(Tg);
  const int grid = bwd_blocks(rows);
  const int64_t nvec = dim / V;
  const bool vec_ok = dim % V == 0 && aligned16(dy) && aligned16(saved) && (dx == nullptr || aligned16(dx)) &&
                      (dres == nullptr || aligned16(dres)) &&
                      (dim * (int64_t)sizeof(Tg)) % 16 == 0 && (dim * (int64_t)sizeof(Tdx)) % 16 == 0;
  const int nj = (int)((nvec + 31) / 32);
  const Tg* dyp = static_cast<const Tg*>(dy);
  const Tg* sp = static_cast<const Tg*>(saved);
  Tdx* dxp = static_cast<Tdx*>(dx);
  const Tdx* drp = static_cast<const Tdx*>(dres);
  const size_t smem = (size_t)kWarps * dim * sizeof(float);
  int used_grid = grid;  // CTAs writing grad_gamma partial rows
  // Register budget: at most 1024 elements of a row per warp in the vector path.
  const int64_t row_bytes = dim * (int64_t)sizeof(Tg);
  const int64_t sb = dres ? kBwdStageBytesRes : kBwdStageBytes, ns = dres ? kBwdStagesRes : kStages;
  if (vec_ok && sizeof(Tg) == sizeof(Tdx) && dim <= kMaxBulkDim && row_bytes <= sb &&
      (int64_t)kWarps * 4 * dim * 4 <= ns * sb * 2) {
    const int rpt = (int)(sb / row_bytes < kMaxBwdTileRows ? sb / row_bytes : kMaxBwdTileRows);
    const int64_t tiles = (rows + rpt - 1) / rpt;
    // 3 CTAs of 68 KB shared memory per SM (2 of 100 KB with the residual gradient staged as a third input)
    int64_t g = (int64_t)num_sms() * (drp ? 2 : 3);
    if (g > kMaxBwdBlocks) g = kMaxBwdBlocks;
    if (g > tiles) g = tiles;
    used_grid = (int)g;
    auto go = [&](auto kern, int bsm) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bsm);
      kern<<<used_grid, kThreads, bsm, stream>>>(dyp, sp, saved_is_input, inv, gamma, gcode, dxp, drp, partial,
                                                 rows, (int)dim, rpt);
    };
    auto pick = [&](auto res) {
      constexpr bool R = decltype(res)::value;
      constexpr int bsm = R ? bulk_smem_bytes<kBwdStageBytesRes, 3, kBwdStagesRes>()
                            : bulk_smem_bytes<kBwdStageBytes, 2>();
      if (nvec <= 8)
        go(rms_bwd_bulk<Tg, Tdx, V, 8, 1, R>, bsm);
      else if (nvec <= 24)
        go(rms_bwd_bulk<Tg, Tdx, V, 8, 3, R>, bsm);
      else if (nvec <= 48)
        go(rms_bwd_bulk<Tg, Tdx, V, 16, 3, R>, bsm);
      else if (nvec <= 64)
        go(rms_bwd_bulk<Tg, Tdx, V, 32, 2, R>, bsm);
      else if (nvec <= 128)
        go(rms_bwd_bulk<Tg, Tdx, V, 32, 4, R>, bsm);
      else if constexpr (V == 4)
        go(rms_bwd_bulk<Tg, Tdx, V, 32, 8, R>, bsm);
    };
    if (drp != nullptr)
      pick(std::true_type());
    else
      pick(std::false_type());
  } else if (vec_ok && nj * 32 * V <= 1024 && smem <= 48 * 1024) {
    if (nj <= 1)
      rms_bwd_vec<Tg, Tdx, V, 1><<<grid, kThreads, smem, stream>>>(dyp, sp, saved_is_input, inv, gamma, gcode, dxp,
                                                                   drp, partial, rows, (int)dim);
    else if (nj <= 2)
      rms_bwd_vec<Tg, Tdx, V, 2><<<grid, kThreads, smem, stream>>>(dyp, sp, saved_is_input, inv, gamma, gcode, dxp,
                                                                   drp, partial, rows, (int)dim);
    else if (nj <= 4)
      rms_bwd_vec<Tg, Tdx, V, 4><<<grid, kThreads, smem, stream>>>(dyp, sp, saved_is_input, inv, gamma, gcode, dxp,
                                                                   drp, partial, rows, (int)dim);
    else if constexpr (V == 4)
      rms_bwd_vec<Tg, Tdx, V, 8><<<grid, kThreads, smem, stream>>>(dyp, sp, saved_is_input, inv, gamma, gcode, dxp,
                                                                   drp, partial, rows, (int)dim);
  } else {
    rms_bwd_generic<Tg, Tdx><<<grid, kThreads, 0, stream>>>(dyp, sp, saved_is_input, inv, gamma, gcode, dxp,
                                                            drp, partial, rows, (int)dim);
  }
  PMB_CHECK_LAUNCH("pmb_rms_norm_backward");
  if (dgamma != nullptr) {
    red::colsum_rows<<<red::colsum_rows_grid(dim), red::kThreads, 0, stream>>>(partial, used_grid, dim, dgamma,
                                                                               dgcode);
    PMB_CHECK_LAUNCH("pmb_rms_norm_backward(grad_gamma)");
  }
  return PMB_OK;
}

bool valid_code(int c) { return c == PMB_FLOAT32 || c == PMB_FLOAT16 || c == PMB_BFLOAT16; }

}  // namespace
}  // namespace pmb

using namespace pmb;

extern "C" int pmb_rms_norm_forward(const void* x, const void* gamma, void* out, void* normed, float* inv_norm,
                                    int64_t rows, int64_t dim, int x_dtype, int gamma_dtype, int out_dtype,
                                    void* stream) {
  clear_error();
  PMB_REQUIRE(rows >= 0 && dim > 0 && dim <= (1 << 20), "pmb_rms_norm_forward: bad shape rows=%lld dim=%lld",
              (long long)rows, (long long)dim);
  PMB_REQUIRE(valid_code(gamma_dtype), "pmb_rms_norm_forward: unsupported gamma dtype %d", gamma_dtype);
  if (rows == 0) return PMB_OK;
  PMB_REQUIRE(x && gamma && out && inv_norm, "pmb_rms_norm_forward: NULL tensor argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return PMB_DISPATCH(x_dtype, Tx, "pmb_rms_norm_forward", [&] {
    return PMB_DISPATCH(out_dtype, To, "pmb_rms_norm_forward", [&] {
      return launch_fwd<Tx, To>(x, gamma, gamma_dtype, out, normed, inv_norm, rows, dim, s);
    });
  });
}

extern "C" int64_t pmb_rms_norm_backward_workspace_size(int64_t rows, int64_t dim) {
  if (rows <= 0 || dim <= 0) return 0;
  // every backward path launches at most min(rows, kMaxBwdBlocks) CTAs (the
  // bulk path one per tile of as few as one row), each writing one partial row
  return max_bwd_grid(rows) * dim * (int64_t)sizeof(float);
}

namespace pmb {
namespace {
int rms_backward(const void* grad_out, const void* saved, int saved_is_input, const float* inv_norm,
                 const void* gamma, const void* grad_residual, void* grad_x, void* grad_gamma, int64_t rows,
                 int64_t dim, int grad_dtype, int gamma_dtype, int grad_x_dtype, int grad_gamma_dtype, void* workspace,
                 int64_t workspace_bytes, void* stream, const char* name) {
  PMB_REQUIRE(rows >= 0 && dim > 0 && dim <= (1 << 20), "%s: bad shape rows=%lld dim=%lld", name, (long long)rows,
              (long long)dim);
  PMB_REQUIRE(valid_code(gamma_dtype) && valid_code(grad_gamma_dtype), "%s: unsupported gamma/grad_gamma dtype",
              name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (grad_gamma != nullptr) {
      PMB_CHECK_CUDA(cudaMemsetAsync(grad_gamma, 0, dim * dtype_size(grad_gamma_dtype), s), name);
    }
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && saved && inv_norm && gamma, "%s: NULL tensor argument", name);
  PMB_REQUIRE(grad_residual == nullptr || grad_x != nullptr, "%s: grad_residual needs grad_x", name);
  const int64_t need = pmb_rms_norm_backward_workspace_size(rows, dim);
  if (workspace_bytes < need || workspace == nullptr) {
    set_error("%s: workspace of %lld bytes is smaller than the %lld required", name, (long long)workspace_bytes,
              (long long)need);
    return PMB_ERR_WORKSPACE;
  }
  float* partial = static_cast<float*>(workspace);
  return PMB_DISPATCH(grad_dtype, Tg, name, [&] {
    return PMB_DISPATCH(grad_x_dtype, Tdx, name, [&] {
      return launch_bwd<Tg, Tdx>(grad_out, saved, saved_is_input, inv_norm, gamma, gamma_dtype, grad_x,
                                 grad_residual, grad_gamma, grad_gamma_dtype, rows, dim, partial, s);
    });
  });
}
}  // namespace
}  // namespace pmb

extern "C" int pmb_rms_norm_backward(const void* grad_out, const void* saved, int saved_is_input,
                                     const float* inv_norm, const void* gamma, void* grad_x, void* grad_gamma,
                                     int64_t rows, int64_t dim, int grad_dtype, int gamma_dtype, int grad_x_dtype,
                                     int grad_gamma_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  return rms_backward(grad_out, saved, saved_is_input, inv_norm, gamma, nullptr, grad_x, grad_gamma, rows, dim,
                      grad_dtype, gamma_dtype, grad_x_dtype, grad_gamma_dtype, workspace, workspace_bytes, stream,
                      "pmb_rms_norm_backward");
}

extern "C" int pmb_rms_norm_backward_add(const void* grad_out, const void* saved, int saved_is_input,
                                         const float* inv_norm, const void* gamma, const void* grad_residual,
                                         void* grad_x, void* grad_gamma, int64_t rows, int64_t dim, int grad_dtype,
                                         int gamma_dtype, int grad_x_dtype, int grad_gamma_dtype, void* workspace,
                                         int64_t workspace_bytes, void* stream) {
  clear_error();
  return rms_backward(grad_out, saved, saved_is_input, inv_norm, gamma, grad_residual, grad_x, grad_gamma, rows, dim,
                      grad_dtype, gamma_dtype, grad_x_dtype, grad_gamma_dtype, workspace, workspace_bytes, stream,
                      "pmb_rms_norm_backward_add");
}

// ---------------------------------------------------------------------------
// RMSNorm backward without a caller-supplied workspace.
//
// Some callers of this library cannot allocate device memory for a call: a
// program that binds the C ABI directly from another language and has no
// tensor library or device allocator of its own, or a training loop that
// plans all of its device memory before it starts and must not allocate in
// the middle of a step (cudaMalloc and cudaFree synchronise the whole
// device).  For them this variant keeps its scratch -- the per-block partial
// sums of grad_gamma -- in one fixed array inside the library instead of a
// workspace argument.  Inputs and outputs are still the caller's.
//
// Limits and behaviour:
//  * the array holds kNoAllocScratchFloats fp32 values (2.3 MiB); every GPU
//    that loads the library keeps it until the process exits;
//  * dim may be at most kNoAllocMaxDim (1024); a larger dim is rejected with
//    PMB_ERR_WORKSPACE before anything is launched;
//  * the first call on a device looks up the array's address on that device
//    (cudaGetSymbolAddress) and remembers it, so make that first call before
//    capturing work on the stream;
//  * all calls on a device share the array, and it keeps whatever the last
//    call left in it.  Each call rewrites every partial sum it reads before
//    reading it, so nothing has to be cleared between calls, but calls whose
//    kernels overlap on the GPU (other streams, other host threads) race on
//    the array: issue them in order on one stream.
// ---------------------------------------------------------------------------
namespace pmb {
namespace {

constexpr int64_t kNoAllocMaxDim = 1024;
constexpr int64_t kNoAllocScratchFloats = (int64_t)kMaxBwdBlocks * kNoAllocMaxDim;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_rms_noalloc_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mutex;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once
// per device; the host-side name is only a stand-in for the symbol).
int noalloc_scratch(float** out, const char* name) {
  int dev = 0;
  PMB_CHECK_CUDA(cudaGetDevice(&dev), name);
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    set_error("%s: device ordinal %d is outside the supported range", name, dev);
    return PMB_ERR_INVALID_ARGUMENT;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_rms_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr) {
      set_error("%s: cudaGetSymbolAddress failed on device %d: %s", name, dev, cudaGetErrorString(err));
      return PMB_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return PMB_OK;
}

}  // namespace
}  // namespace pmb

extern "C" int pmb_rms_norm_backward_noalloc(const void* grad_out, const void* saved, int saved_is_input,
                                             const float* inv_norm, const void* gamma, void* grad_x,
                                             void* grad_gamma, int64_t rows, int64_t dim, int grad_dtype,
                                             int gamma_dtype, int grad_x_dtype, int grad_gamma_dtype,
                                             void* stream) {
  clear_error();
  const char* name = "pmb_rms_norm_backward_noalloc";
  PMB_REQUIRE(rows >= 0 && dim > 0, "%s: bad shape rows=%lld dim=%lld", name, (long long)rows, (long long)dim);
  if (dim > kNoAllocMaxDim) {
    set_error("%s: dim %lld exceeds the built-in scratch limit of %lld; use pmb_rms_norm_backward with a workspace",
              name, (long long)dim, (long long)kNoAllocMaxDim);
    return PMB_ERR_WORKSPACE;
  }
  PMB_REQUIRE(valid_code(gamma_dtype) && valid_code(grad_gamma_dtype), "%s: unsupported gamma/grad_gamma dtype",
              name);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (grad_gamma != nullptr) PMB_CHECK_CUDA(cudaMemsetAsync(grad_gamma, 0, dim * dtype_size(grad_gamma_dtype), s), name);
    return PMB_OK;
  }
  PMB_REQUIRE(grad_out && saved && inv_norm && gamma, "%s: NULL tensor argument", name);
  float* partial = nullptr;
  const int st = noalloc_scratch(&partial, name);
  if (st) return st;
  // every path launches at most kMaxBwdBlocks CTAs, so the partial sums fit the array.
  return PMB_DISPATCH(grad_dtype, Tg, name, [&] {
    return PMB_DISPATCH(grad_x_dtype, Tdx, name, [&] {
      return launch_bwd<Tg, Tdx>(grad_out, saved, saved_is_input, inv_norm, gamma, gamma_dtype, grad_x, nullptr,
                                 grad_gamma, grad_gamma_dtype, rows, dim, partial, s);
    });
  });
}
