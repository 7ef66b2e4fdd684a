// Row-wise HBM-bound kernels: RMSNorm, GatedRMSNorm, SwiGLU, attn-res depth softmax
// (with its fused RMSNorm), gated residual, argmax and the embedding gather.
//
// All are one warp per row: the row is streamed once from HBM into registers (fp32),
// reduced with warp shuffles and written once.  Rows of up to 8 * 32 * MAXV elements stay
// in registers; the generic path re-reads the row (it is L1-resident by then).
#include <algorithm>

#include "common.cuh"

namespace mb {
namespace {

constexpr int kWarpsPerBlock = 8;

inline int rows_grid(int64_t rows) { return (int)((rows + kWarpsPerBlock - 1) / kWarpsPerBlock); }

// ---------------------------------------------------------------------------- RMSNorm
// motif/ops/rms_norm.py:481-486: y = (x * rsqrt(mean(x^2) + eps)) * w.
template <typename T>
__global__ void rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                                int64_t M, int N, int64_t xs, int64_t ys, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= M) return;
  const T* xr = x + row * xs;
  float ss = 0.f;
  for (int i = lane; i < N; i += 32) {
    float v = to_f(xr[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)N + eps);
  T* yr = y + row * ys;
  for (int i = lane; i < N; i += 32) {
    // The reference rounds the normalised value to the input dtype before the weight.
    float v = to_f(from_f<T>(to_f(xr[i]) * r));
    if (w) v = to_f(from_f<T>(v * to_f(w[i])));
    yr[i] = from_f<T>(v);
  }
}

// motif/ops/rms_norm.py:547-553: rmsnorm(values) * w * silu(gate), values first.
template <typename T>
__global__ void gated_rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                      T* __restrict__ y, int64_t M, int N, int64_t xs, int64_t ys,
                                      float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= M) return;
  const T* xr = x + row * xs;
  float ss = 0.f;
  for (int i = lane; i < N; i += 32) {
    float v = to_f(xr[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)N + eps);
  T* yr = y + row * ys;
  for (int i = lane; i < N; i += 32) {
    float v = to_f(from_f<T>(to_f(xr[i]) * r));
    if (w) v = to_f(from_f<T>(v * to_f(w[i])));
    const float gt = to_f(xr[N + i]);
    const float sg = to_f(from_f<T>(siluf_(gt)));
    yr[i] = from_f<T>(v * sg);
  }
}

// motif/ops/swiglu.py:252-253: values * silu(gate).
template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t M, int N,
                              int64_t xs, int64_t ys) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  for (int64_t row = blockIdx.y; row < M; row += gridDim.y) {
    const T* xr = x + row * xs;
    const float gt = to_f(xr[N + i]);
    const float sg = to_f(from_f<T>(siluf_(gt)));
    y[row * ys + i] = from_f<T>(to_f(xr[i]) * sg);
  }
}

// 16-byte vector variant: 8 elements per thread, flat grid-stride loop over [M, N/8].
template <typename T>
__global__ void swiglu_vec_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t M, int N, int64_t xs,
                                  int64_t ys) {
  const int64_t total = M * (N / 8);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    swiglu_group<T>(x, xs, y, ys, N, i);
}

template <typename T>
__global__ void gate_residual_vec_kernel(const T* __restrict__ a, int64_t as, const T* __restrict__ g, int64_t gs,
                                         const T* __restrict__ m, int64_t ms, T* __restrict__ out, int64_t os,
                                         int64_t rows, int N) {
  const int nv = N / 8;
  const int64_t total = rows * nv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / nv;
    const int c = (int)(i % nv) * 8;
    uint4 ra = *reinterpret_cast<const uint4*>(a + row * as + c);
    uint4 rg = *reinterpret_cast<const uint4*>(g + row * gs + c);
    uint4 rm = *reinterpret_cast<const uint4*>(m + row * ms + c);
    const T* a8 = reinterpret_cast<const T*>(&ra);
    const T* g8 = reinterpret_cast<const T*>(&rg);
    const T* m8 = reinterpret_cast<const T*>(&rm);
    T o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float gate = to_f(from_f<T>(sigmoidf_(to_f(g8[e]))));
      const float att = to_f(from_f<T>(to_f(a8[e]) * gate));
      o8[e] = from_f<T>(att + to_f(m8[e]));
    }
    *reinterpret_cast<uint4*>(out + row * os + c) = *reinterpret_cast<const uint4*>(o8);
  }
}

inline bool vec16_ok(const void* p) { return ((uintptr_t)p & 15) == 0; }

inline unsigned flat_grid(int64_t total, int threads) {
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = 148LL * 16;  // enough resident blocks to saturate HBM; grid-stride beyond
  return (unsigned)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

// ---------------------------------------------------------------------------- attn-res
constexpr int kMaxSrc = 8;
// Up to this many rows the fused attn-res read runs one CTA per row (sources in parallel);
// above it, one warp per row streams the sources (the prefill shape, HBM-bound either way).
constexpr int64_t kSrcParallelRows = 2048;
struct SrcPtrs {
  const void* p[kMaxSrc];
  int64_t sb[kMaxSrc];
  int64_t st[kMaxSrc];
};

// motif/ops/attn_res.py:588-593 (eager) / :93-186 (fused): logit_s = q . (w * rmsnorm(x_s)),
// h = sum_s softmax_s(logit) x_s.  Generic path: the sources are re-read from L1.
template <typename T>
__global__ void attn_res_kernel(SrcPtrs src, int n_src, const T* __restrict__ w,
                                const T* __restrict__ q, T* __restrict__ out, int64_t osb,
                                int64_t ost, int64_t B, int64_t Tn, int D, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= B * Tn) return;
  const int64_t b = row / Tn, t = row % Tn;
  float logit[kMaxSrc];
  float mx = -INFINITY;
  for (int s = 0; s < n_src; ++s) {
    const T* xr = static_cast<const T*>(src.p[s]) + b * src.sb[s] + t * src.st[s];
    float ss = 0.f, dot = 0.f;
    for (int i = lane; i < D; i += 32) {
      const float v = to_f(xr[i]);
      ss += v * v;
      dot += to_f(q[i]) * to_f(w[i]) * v;
    }
    ss = warp_sum(ss);
    dot = warp_sum(dot);
    logit[s] = dot * rsqrtf(ss / (float)D + eps);
    mx = fmaxf(mx, logit[s]);
  }
  float den = 0.f;
  for (int s = 0; s < n_src; ++s) {
    logit[s] = expf(logit[s] - mx);
    den += logit[s];
  }
  const float inv = 1.f / den;
  T* orow = out + b * osb + t * ost;
  for (int i = lane; i < D; i += 32) {
    float h = 0.f;
    for (int s = 0; s < n_src; ++s) {
      const T* xr = static_cast<const T*>(src.p[s]) + b * src.sb[s] + t * src.st[s];
      h += logit[s] * inv * to_f(xr[i]);
    }
    orow[i] = from_f<T>(h);
  }
}

// Fused attn-res read + RMSNorm of the result for the model path (token-major rows, all
// sources share one row stride).  NV 16-byte vectors of 8 elements per lane: D = 256 * NV.
template <typename T, int NV>
__global__ void __launch_bounds__(32 * kWarpsPerBlock, 2) attn_res_norm_vec_kernel(SrcPtrs src, int n_src, int64_t srs, const T* __restrict__ w,
                                         const T* __restrict__ q, T* __restrict__ h_out,
                                         T* __restrict__ hn_out, int64_t ors, int64_t rows,
                                         float eps_src, float eps_out) {
  constexpr int D = 256 * NV;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  float h[NV][8];
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int e = 0; e < 8; ++e) h[v][e] = 0.f;

  // The rows of up to kGroup sources are requested together before any is reduced, so a warp
  // keeps kGroup rows (4 x 1.5 KB at D = 768) in flight instead of one or two.
  constexpr int kGroup = 4;
  if (q == nullptr || n_src == 1) {
    for (int s0 = 0; s0 < n_src; s0 += kGroup) {
      uint4 raw[kGroup][NV];
#pragma unroll
      for (int u = 0; u < kGroup; ++u)
        if (s0 + u < n_src) {
          const T* xr = static_cast<const T*>(src.p[s0 + u]) + row * srs;
#pragma unroll
          for (int v = 0; v < NV; ++v) raw[u][v] = *reinterpret_cast<const uint4*>(xr + (v * 32 + lane) * 8);
        }
#pragma unroll
      for (int u = 0; u < kGroup; ++u)
        if (s0 + u < n_src) {
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            const T* e8 = reinterpret_cast<const T*>(&raw[u][v]);
#pragma unroll
            for (int e = 0; e < 8; ++e) h[v][e] += to_f(e8[e]);
          }
        }
    }
  } else {
    float qw[NV][8];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      uint4 rq = *reinterpret_cast<const uint4*>(q + (v * 32 + lane) * 8);
      uint4 rw = *reinterpret_cast<const uint4*>(w + (v * 32 + lane) * 8);
      const T* q8 = reinterpret_cast<const T*>(&rq);
      const T* w8 = reinterpret_cast<const T*>(&rw);
#pragma unroll
      for (int e = 0; e < 8; ++e) qw[v][e] = to_f(q8[e]) * to_f(w8[e]);
    }
    // Online softmax over the sources: h accumulates exp(l_s - m) x_s, group by group.
    float m = -INFINITY, den = 0.f;
    for (int s0 = 0; s0 < n_src; s0 += kGroup) {
      uint4 raw[kGroup][NV];
#pragma unroll
      for (int u = 0; u < kGroup; ++u)
        if (s0 + u < n_src) {
          const T* xr = static_cast<const T*>(src.p[s0 + u]) + row * srs;
#pragma unroll
          for (int v = 0; v < NV; ++v) raw[u][v] = *reinterpret_cast<const uint4*>(xr + (v * 32 + lane) * 8);
        }
      float ss[kGroup], dot[kGroup];
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        ss[u] = 0.f;
        dot[u] = 0.f;
        if (s0 + u < n_src) {
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            const T* e8 = reinterpret_cast<const T*>(&raw[u][v]);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float x = to_f(e8[e]);
              ss[u] += x * x;
              dot[u] += qw[v][e] * x;
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        ss[u] = warp_sum(ss[u]);
        dot[u] = warp_sum(dot[u]);
      }
#pragma unroll
      for (int u = 0; u < kGroup; ++u)
        if (s0 + u < n_src) {  // sources in order: the same sums as one source at a time
          const float l = dot[u] * rsqrtf(ss[u] / (float)D + eps_src);
          const float mn = fmaxf(m, l);
          const float sc = expf(m - mn);  // 0 on the first source (m = -inf)
          const float p = expf(l - mn);
          den = den * sc + p;
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            const T* e8 = reinterpret_cast<const T*>(&raw[u][v]);
#pragma unroll
            for (int e = 0; e < 8; ++e) h[v][e] = h[v][e] * sc + p * to_f(e8[e]);
          }
          m = mn;
        }
    }
    const float inv = 1.f / den;
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int e = 0; e < 8; ++e) h[v][e] *= inv;
  }
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += h[v][e] * h[v][e];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps_out);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    T o8[8], n8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o8[e] = from_f<T>(h[v][e]);
      n8[e] = from_f<T>(h[v][e] * r);
    }
    if (h_out) *reinterpret_cast<uint4*>(h_out + row * ors + (v * 32 + lane) * 8) = *reinterpret_cast<uint4*>(o8);
    *reinterpret_cast<uint4*>(hn_out + row * ors + (v * 32 + lane) * 8) = *reinterpret_cast<uint4*>(n8);
  }
}

// Few-row (decode) form of the fused read: one CTA per row, warp s loads source s, so all
// sources of the row are in flight at once instead of one after another in a single warp.
// The logits meet in shared memory; thread g < D/8 then sums its 8-element group over the
// sources in order, and the output RMSNorm reduces across the CTA.
template <typename T, int NV>
__global__ void __launch_bounds__(32 * kMaxSrc) attn_res_norm_src_kernel(
    SrcPtrs src, int n_src, int64_t srs, const T* __restrict__ w, const T* __restrict__ q,
    T* __restrict__ h_out, T* __restrict__ hn_out, int64_t ors, float eps_src, float eps_out) {
  constexpr int D = 256 * NV, G = D / 8;
  __shared__ uint4 xs[kMaxSrc][G];
  __shared__ float lg[kMaxSrc], red[kMaxSrc];
  allow_dependent_launch();  // the decoder's input projection may start fetching its weights
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const bool mix = q != nullptr && n_src > 1;
  if (warp < n_src) {
    const T* xr = static_cast<const T*>(src.p[warp]) + row * srs;
    uint4 raw[NV], rq[NV], rw[NV];  // the row and (when mixing) q and w, all requested at once
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      raw[v] = *reinterpret_cast<const uint4*>(xr + (v * 32 + lane) * 8);
      if (mix) {
        rq[v] = *reinterpret_cast<const uint4*>(q + (v * 32 + lane) * 8);
        rw[v] = *reinterpret_cast<const uint4*>(w + (v * 32 + lane) * 8);
      }
    }
    float ss = 0.f, dot = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      xs[warp][v * 32 + lane] = raw[v];
      if (mix) {
        const T* q8 = reinterpret_cast<const T*>(&rq[v]);
        const T* w8 = reinterpret_cast<const T*>(&rw[v]);
        const T* e8 = reinterpret_cast<const T*>(&raw[v]);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x = to_f(e8[e]);
          ss += x * x;
          dot += to_f(q8[e]) * to_f(w8[e]) * x;
        }
      }
    }
    if (mix) {
      ss = warp_sum(ss);
      dot = warp_sum(dot);
      if (lane == 0) lg[warp] = dot * rsqrtf(ss / (float)D + eps_src);
    }
  }
  __syncthreads();
  float pw[kMaxSrc];
  float inv = 1.f;
  if (mix) {
    float m = -INFINITY, den = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxSrc; ++s)
      if (s < n_src) m = fmaxf(m, lg[s]);
#pragma unroll
    for (int s = 0; s < kMaxSrc; ++s) {
      pw[s] = s < n_src ? expf(lg[s] - m) : 0.f;
      den += pw[s];
    }
    inv = 1.f / den;
  } else {
#pragma unroll
    for (int s = 0; s < kMaxSrc; ++s) pw[s] = 1.f;
  }
  float h[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) h[e] = 0.f;
  float ss = 0.f;
  if (tid < G) {
#pragma unroll
    for (int s = 0; s < kMaxSrc; ++s) {
      if (s >= n_src) break;
      const uint4 raw = xs[s][tid];
      const T* e8 = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = fmaf(pw[s], to_f(e8[e]), h[e]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      h[e] *= inv;
      ss += h[e] * h[e];
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxSrc; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)D + eps_out);
  if (tid < G) {
    T o8[8], n8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o8[e] = from_f<T>(h[e]);
      n8[e] = from_f<T>(h[e] * r);
    }
    if (h_out) *reinterpret_cast<uint4*>(h_out + row * ors + tid * 8) = *reinterpret_cast<uint4*>(o8);
    *reinterpret_cast<uint4*>(hn_out + row * ors + tid * 8) = *reinterpret_cast<uint4*>(n8);
  }
}

// Generic-D version of the fused read (scalar, two passes over L1-resident rows).
template <typename T>
__global__ void attn_res_norm_kernel(SrcPtrs src, int n_src, int64_t srs, const T* __restrict__ w,
                                     const T* __restrict__ q, T* __restrict__ h_out,
                                     T* __restrict__ hn_out, int64_t ors, int64_t rows, int D,
                                     float eps_src, float eps_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  float a[kMaxSrc];
  if (q == nullptr || n_src == 1) {
    for (int s = 0; s < n_src; ++s) a[s] = 1.f;
  } else {
    float mx = -INFINITY;
    for (int s = 0; s < n_src; ++s) {
      const T* xr = static_cast<const T*>(src.p[s]) + row * srs;
      float ss = 0.f, dot = 0.f;
      for (int i = lane; i < D; i += 32) {
        const float v = to_f(xr[i]);
        ss += v * v;
        dot += to_f(q[i]) * to_f(w[i]) * v;
      }
      ss = warp_sum(ss);
      dot = warp_sum(dot);
      a[s] = dot * rsqrtf(ss / (float)D + eps_src);
      mx = fmaxf(mx, a[s]);
    }
    float den = 0.f;
    for (int s = 0; s < n_src; ++s) {
      a[s] = expf(a[s] - mx);
      den += a[s];
    }
    for (int s = 0; s < n_src; ++s) a[s] /= den;
  }
  float ss = 0.f;
  for (int i = lane; i < D; i += 32) {
    float h = 0.f;
    for (int s = 0; s < n_src; ++s) h += a[s] * to_f(static_cast<const T*>(src.p[s])[row * srs + i]);
    ss += h * h;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps_out);
  for (int i = lane; i < D; i += 32) {
    float h = 0.f;
    for (int s = 0; s < n_src; ++s) h += a[s] * to_f(static_cast<const T*>(src.p[s])[row * srs + i]);
    if (h_out) h_out[row * ors + i] = from_f<T>(h);
    hn_out[row * ors + i] = from_f<T>(h * r);
  }
}

// ---------------------------------------------------------------------------- misc
template <typename T>
__global__ void gate_residual_kernel(const T* __restrict__ a, int64_t as, const T* __restrict__ g,
                                     int64_t gs, const T* __restrict__ m, int64_t ms,
                                     T* __restrict__ out, int64_t os, int64_t rows, int N) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    // chord_attn.py:254,313 rounds o_proj(out) and sigmoid(g_proj) to the model dtype.
    const float gate = to_f(from_f<T>(sigmoidf_(to_f(g[row * gs + i]))));
    const float att = to_f(from_f<T>(to_f(a[row * as + i]) * gate));
    out[row * os + i] = from_f<T>(att + to_f(m[row * ms + i]));
  }
}

// VEC (16-bit rows, V and the row stride multiples of 8, 16-byte aligned): each thread reads
// 8 logits per 16-byte load, four loads in flight, visiting its indices in increasing order
// like the scalar loop, so the first maximum still wins.
template <typename T, bool VEC>
__global__ void argmax_kernel(const T* __restrict__ x, int64_t V, int64_t rs, int64_t* __restrict__ ids) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * rs;
  float best = -INFINITY;
  int64_t bi = 0x7fffffffffffffffLL;
  auto visit = [&](float v, int64_t i) {
    if (v > best || (v == best && i < bi) || (isnan(v) && !isnan(best))) {
      best = v;
      bi = i;
    }
  };
  if constexpr (VEC) {
    const int64_t nv = V / 8;
    for (int64_t g0 = threadIdx.x; g0 < nv; g0 += 4 * (int64_t)blockDim.x) {
      uint4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t g = g0 + u * (int64_t)blockDim.x;
        if (g < nv) r[u] = *reinterpret_cast<const uint4*>(xr + g * 8);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t g = g0 + u * (int64_t)blockDim.x;
        if (g < nv) {
          const T* e8 = reinterpret_cast<const T*>(&r[u]);
#pragma unroll
          for (int e = 0; e < 8; ++e) visit(to_f(e8[e]), g * 8 + e);
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) visit(to_f(xr[i]), i);
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[wid] = best;
    si[wid] = bi;
  }
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffffffffffffLL;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) ids[row] = bi;
  }
}

// End-of-step bookkeeping of the CUDA-graph decoder in one launch: the step's ids into row
// step_idx of the token log, then step_idx and the cache lengths advance by one.  One CTA:
// every thread reads step_idx before thread 0 advances it.
__global__ void __launch_bounds__(256) decode_advance_kernel(const int64_t* __restrict__ ids, int64_t B,
                                                             int64_t* __restrict__ tokens, int64_t max_steps,
                                                             int64_t* __restrict__ step_idx,
                                                             int32_t* __restrict__ lens, int nlens) {
  const int64_t s = *step_idx;
  if (s >= 0 && s < max_steps)
    for (int64_t b = threadIdx.x; b < B; b += blockDim.x) tokens[s * B + b] = ids[b];
  __syncthreads();
  if (threadIdx.x == 0) {
    *step_idx = s + 1;
    for (int i = 0; i < nlens; ++i) lens[i] += 1;
  }
}

template <typename T>
__global__ void embed_kernel(const int64_t* __restrict__ ids, const T* __restrict__ table,
                             T* __restrict__ out, int64_t rows, int D, int64_t V) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= D) return;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    int64_t id = ids[row];
    id = id < 0 ? 0 : (id >= V ? V - 1 : id);  // out-of-range ids are clamped, never read OOB
    out[row * D + i] = table[id * D + i];
  }
}

template <typename F>
int dispatch(int dtype, F&& f) {
  switch (dtype) {
    case MB_F32: return f(float{});
    case MB_F16: return f(__half{});
    case MB_BF16: return f(__nv_bfloat16{});
    default: return set_error(MB_ERR_DTYPE, "unsupported dtype code %d", dtype);
  }
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" int motif_b200_rms_norm(const void* x, const void* w, void* y, int64_t M, int64_t N,
                                   int64_t xs, int64_t ys, float eps, int dtype, void* stream) {
  MB_REQUIRE(x && y, MB_ERR_ARG, "rms_norm: null pointer");
  MB_REQUIRE(M >= 0 && N > 0 && N <= (1 << 20), MB_ERR_SHAPE, "rms_norm: bad shape M=%lld N=%lld",
             (long long)M, (long long)N);
  if (M == 0) return MB_OK;
  return dispatch(dtype, [&](auto t) {
    using T = decltype(t);
    rms_norm_kernel<T><<<rows_grid(M), 32 * kWarpsPerBlock, 0, (cudaStream_t)stream>>>(
        (const T*)x, (const T*)w, (T*)y, M, (int)N, xs, ys, eps);
    return check_launch("rms_norm");
  });
}

extern "C" int motif_b200_gated_rms_norm(const void* x, const void* w, void* y, int64_t M, int64_t N,
                                         int64_t xs, int64_t ys, float eps, int dtype, void* stream) {
  MB_REQUIRE(x && y, MB_ERR_ARG, "gated_rms_norm: null pointer");
  MB_REQUIRE(M >= 0 && N > 0 && N <= (1 << 20), MB_ERR_SHAPE, "gated_rms_norm: bad shape");
  if (M == 0) return MB_OK;
  return dispatch(dtype, [&](auto t) {
    using T = decltype(t);
    gated_rms_norm_kernel<T><<<rows_grid(M), 32 * kWarpsPerBlock, 0, (cudaStream_t)stream>>>(
        (const T*)x, (const T*)w, (T*)y, M, (int)N, xs, ys, eps);
    return check_launch("gated_rms_norm");
  });
}

extern "C" int motif_b200_swiglu(const void* x, void* y, int64_t M, int64_t N, int64_t xs,
                                 int64_t ys, int dtype, void* stream) {
  MB_REQUIRE(x && y, MB_ERR_ARG, "swiglu: null pointer");
  MB_REQUIRE(M >= 0 && N > 0 && N <= (1 << 24), MB_ERR_SHAPE, "swiglu: bad shape");
  if (M == 0) return MB_OK;
  return dispatch(dtype, [&](auto t) {
    using T = decltype(t);
    if (sizeof(T) == 2 && N % 8 == 0 && xs % 8 == 0 && ys % 8 == 0 && vec16_ok(x) && vec16_ok(y)) {
      swiglu_vec_kernel<T><<<flat_grid(M * (N / 8), 256), 256, 0, (cudaStream_t)stream>>>((const T*)x, (T*)y, M,
                                                                                          (int)N, xs, ys);
      return check_launch("swiglu");
    }
    dim3 grid((unsigned)((N + 255) / 256), (unsigned)(M < 65535 ? M : 65535));
    swiglu_kernel<T><<<grid, 256, 0, (cudaStream_t)stream>>>((const T*)x, (T*)y, M, (int)N, xs, ys);
    return check_launch("swiglu");
  });
}

extern "C" int motif_b200_attn_res(const void* const* sources, int n_src, const int64_t* src_strides,
                                   const void* weight, const void* query, void* out, int64_t osb,
                                   int64_t ost, int64_t B, int64_t T, int64_t D, float eps, int dtype,
                                   void* stream) {
  MB_REQUIRE(sources && src_strides && weight && query && out, MB_ERR_ARG, "attn_res: null pointer");
  MB_REQUIRE(n_src >= 1 && n_src <= kMaxSrc, MB_ERR_UNSUPPORTED, "attn_res: %d sources (1..%d supported)",
             n_src, kMaxSrc);
  MB_REQUIRE(B >= 0 && T >= 0 && D > 0, MB_ERR_SHAPE, "attn_res: bad shape");
  SrcPtrs sp{};
  for (int s = 0; s < n_src; ++s) {
    MB_REQUIRE(sources[s], MB_ERR_ARG, "attn_res: null source %d", s);
    sp.p[s] = sources[s];
    sp.sb[s] = src_strides[2 * s];
    sp.st[s] = src_strides[2 * s + 1];
  }
  if (B * T == 0) return MB_OK;
  return dispatch(dtype, [&](auto t) {
    using Tt = decltype(t);
    attn_res_kernel<Tt><<<rows_grid(B * T), 32 * kWarpsPerBlock, 0, (cudaStream_t)stream>>>(
        sp, n_src, (const Tt*)weight, (const Tt*)query, (Tt*)out, osb, ost, B, T, (int)D, eps);
    return check_launch("attn_res");
  });
}

extern "C" int motif_b200_attn_res_norm(const void* const* sources, int n_src, int64_t srs,
                                        const void* weight, const void* query, void* h_out,
                                        void* hn_out, int64_t ors, int64_t rows, int64_t D,
                                        float eps_src, float eps_out, int dtype, void* stream) {
  MB_REQUIRE(sources && hn_out, MB_ERR_ARG, "attn_res_norm: null pointer");
  MB_REQUIRE(n_src >= 1 && n_src <= kMaxSrc, MB_ERR_UNSUPPORTED, "attn_res_norm: %d sources", n_src);
  MB_REQUIRE(query == nullptr || weight != nullptr, MB_ERR_ARG, "attn_res_norm: query without weight");
  MB_REQUIRE(rows >= 0 && D > 0, MB_ERR_SHAPE, "attn_res_norm: bad shape");
  SrcPtrs sp{};
  bool aligned = (srs % 8 == 0) && (ors % 8 == 0) && ((uintptr_t)hn_out % 16 == 0) &&
                 ((uintptr_t)h_out % 16 == 0) && ((uintptr_t)weight % 16 == 0) && ((uintptr_t)query % 16 == 0);
  for (int s = 0; s < n_src; ++s) {
    MB_REQUIRE(sources[s], MB_ERR_ARG, "attn_res_norm: null source %d", s);
    sp.p[s] = sources[s];
    aligned = aligned && ((uintptr_t)sources[s] % 16 == 0);
  }
  if (rows == 0) return MB_OK;
  return dispatch(dtype, [&](auto t) {
    using Tt = decltype(t);
    const int grid = rows_grid(rows);
    const int blk = 32 * kWarpsPerBlock;
    cudaStream_t st = (cudaStream_t)stream;
    const bool vec = aligned && sizeof(Tt) == 2 && D % 256 == 0 && D / 256 <= 4;
    if (vec && rows <= kSrcParallelRows) {  // decode-sized: one CTA per row, sources in parallel
      const unsigned g = (unsigned)rows;
      const int bs = 32 * kMaxSrc;
      if (D == 256)
        attn_res_norm_src_kernel<Tt, 1><<<g, bs, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                          (Tt*)h_out, (Tt*)hn_out, ors, eps_src, eps_out);
      else if (D == 512)
        attn_res_norm_src_kernel<Tt, 2><<<g, bs, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                          (Tt*)h_out, (Tt*)hn_out, ors, eps_src, eps_out);
      else if (D == 768)
        attn_res_norm_src_kernel<Tt, 3><<<g, bs, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                          (Tt*)h_out, (Tt*)hn_out, ors, eps_src, eps_out);
      else
        attn_res_norm_src_kernel<Tt, 4><<<g, bs, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                          (Tt*)h_out, (Tt*)hn_out, ors, eps_src, eps_out);
    } else if (vec && D == 256)
      attn_res_norm_vec_kernel<Tt, 1><<<grid, blk, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                             (Tt*)h_out, (Tt*)hn_out, ors, rows, eps_src, eps_out);
    else if (vec && D == 512)
      attn_res_norm_vec_kernel<Tt, 2><<<grid, blk, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                             (Tt*)h_out, (Tt*)hn_out, ors, rows, eps_src, eps_out);
    else if (vec && D == 768)
      attn_res_norm_vec_kernel<Tt, 3><<<grid, blk, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                             (Tt*)h_out, (Tt*)hn_out, ors, rows, eps_src, eps_out);
    else if (vec && D == 1024)
      attn_res_norm_vec_kernel<Tt, 4><<<grid, blk, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                             (Tt*)h_out, (Tt*)hn_out, ors, rows, eps_src, eps_out);
    else
      attn_res_norm_kernel<Tt><<<grid, blk, 0, st>>>(sp, n_src, srs, (const Tt*)weight, (const Tt*)query,
                                                      (Tt*)h_out, (Tt*)hn_out, ors, rows, (int)D, eps_src, eps_out);
    return check_launch("attn_res_norm");
  });
}

extern "C" int motif_b200_gate_residual(const void* a, int64_t as, const void* g, int64_t gs,
                                        const void* m, int64_t ms, void* out, int64_t os, int64_t rows,
                                        int64_t N, int dtype, void* stream) {
  MB_REQUIRE(a && g && m && out, MB_ERR_ARG, "gate_residual: null pointer");
  MB_REQUIRE(rows >= 0 && N > 0 && N <= (1 << 24), MB_ERR_SHAPE, "gate_residual: bad shape");
  if (rows == 0) return MB_OK;
  return dispatch(dtype, [&](auto t) {
    using T = decltype(t);
    if (sizeof(T) == 2 && N % 8 == 0 && as % 8 == 0 && gs % 8 == 0 && ms % 8 == 0 && os % 8 == 0 && vec16_ok(a) &&
        vec16_ok(g) && vec16_ok(m) && vec16_ok(out)) {
      gate_residual_vec_kernel<T><<<flat_grid(rows * (N / 8), 256), 256, 0, (cudaStream_t)stream>>>(
          (const T*)a, as, (const T*)g, gs, (const T*)m, ms, (T*)out, os, rows, (int)N);
      return check_launch("gate_residual");
    }
    dim3 grid((unsigned)((N + 255) / 256), (unsigned)(rows < 65535 ? rows : 65535));
    gate_residual_kernel<T><<<grid, 256, 0, (cudaStream_t)stream>>>((const T*)a, as, (const T*)g, gs,
                                                                   (const T*)m, ms, (T*)out, os, rows, (int)N);
    return check_launch("gate_residual");
  });
}

extern "C" int motif_b200_argmax(const void* logits, int64_t rows, int64_t V, int64_t rs, int64_t* ids,
                                 int dtype, void* stream) {
  MB_REQUIRE(logits && ids, MB_ERR_ARG, "argmax: null pointer");
  MB_REQUIRE(rows >= 0 && rows < 2147483647LL && V > 0, MB_ERR_SHAPE, "argmax: bad shape");
  if (rows == 0) return MB_OK;
  return dispatch(dtype, [&](auto t) {
    using T = decltype(t);
    if (sizeof(T) == 2 && V % 8 == 0 && rs % 8 == 0 && vec16_ok(logits))
      argmax_kernel<T, true><<<(unsigned)rows, 1024, 0, (cudaStream_t)stream>>>((const T*)logits, V, rs, ids);
    else
      argmax_kernel<T, false><<<(unsigned)rows, 1024, 0, (cudaStream_t)stream>>>((const T*)logits, V, rs, ids);
    return check_launch("argmax");
  });
}

extern "C" int motif_b200_embed(const int64_t* ids, const void* table, void* out, int64_t rows,
                                int64_t D, int64_t V, int dtype, void* stream) {
  MB_REQUIRE(ids && table && out, MB_ERR_ARG, "embed: null pointer");
  MB_REQUIRE(rows >= 0 && D > 0 && D <= (1 << 24) && V > 0, MB_ERR_SHAPE, "embed: bad shape");
  if (rows == 0) return MB_OK;
  return dispatch(dtype, [&](auto t) {
    using T = decltype(t);
    dim3 grid((unsigned)((D + 255) / 256), (unsigned)(rows < 65535 ? rows : 65535));
    embed_kernel<T><<<grid, 256, 0, (cudaStream_t)stream>>>(ids, (const T*)table, (T*)out, rows, (int)D, V);
    return check_launch("embed");
  });
}

extern "C" int motif_b200_decode_advance(const int64_t* ids, int64_t B, int64_t* tokens, int64_t max_steps,
                                         int64_t* step_idx, int32_t* lens, int64_t nlens, void* stream) {
  MB_REQUIRE(ids && tokens && step_idx && (lens || nlens == 0), MB_ERR_ARG, "decode_advance: null pointer");
  MB_REQUIRE(B >= 0 && max_steps >= 0 && nlens >= 0 && nlens <= 64, MB_ERR_SHAPE, "decode_advance: bad shape");
  decode_advance_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(ids, B, tokens, max_steps, step_idx, lens, (int)nlens);
  return check_launch("decode_advance");
}
