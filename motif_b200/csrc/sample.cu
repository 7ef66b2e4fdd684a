// One sampled token per row of logits, on the device: repetition penalty -> temperature ->
// top-k -> top-p -> softmax -> draw (motif/model/sampler.py:151-219).  A grammar constraint
// stays on the host side of this kernel: its mask (forbidden tokens -> -inf) is applied to the
// logits before the launch, which gives the same result as applying it after the penalty and
// the temperature (both map -inf to -inf), and its forcing / advance run on the tokens after.
//
// One CTA (512 threads) per row keeps the row in shared memory as fp32.
//   penalty     each distinct token of the row's history once (a bitmap marks them; negative
//               history entries are ignored, so a fixed-size history buffer can be padded with
//               -1), x / rp if x > 0 else x * rp; fused with the load and the temperature
//               x / max(T, 1e-5).
//   top-k/top-p both are one rule: keep x iff W(> x) <= L, W the weight of the values strictly
//               above x — their count with L = k - 1 (top-k: x >= the k-th largest, ties kept),
//               or their softmax mass with L = p * Z (top-p: the reference's sorted-prefix
//               rule, ties at the cut kept).  The kept set is {x >= thr}; each stage finds thr:
//                 window  the values within 16 of the row maximum go to 2048 equal-width bins
//                         (the bin index is monotone in x, so bins are strictly ordered);
//                         a block scan finds the lowest bin whose top value qualifies, and the
//                         few values of that bin are resolved exactly against each other;
//                 radix   when the cut lies below the window (or its bin is crowded), an exact
//                         descent over order-preserving 32-bit keys, 8 bits per pass.
//   draw        with the row's uniform u: the first index, in vocabulary order, whose inclusive
//               cumulative probability exceeds u * Z (per-thread segments + an ordered scan).
// The uniforms are either given (one fp32 per row) or drawn in the kernel with Philox4x32-10
// (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011):
// key = seed, counter = (row, 0, offset lo, offset hi), u = (first output word >> 8) * 2^-24.
// The offset is `offset + *offset_dev` when a device counter is given, so a replayed CUDA
// graph draws fresh numbers every step without a host round trip.
// A row without a finite logit yields token -1 (the reference's multinomial raises there).
// Optionally writes the final probabilities (for inspection and tests).
#include <algorithm>

#include "common.cuh"

namespace mb {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kNB = 2048;            // window bins
constexpr float kWin = 16.f;         // window width below the row maximum
constexpr int kListCap = 1024;       // values of the cut bin resolved exactly
constexpr int kMaxVocab = 53248;     // fp32 row + list within the 227 KB of shared memory

__device__ __forceinline__ uint32_t fkey(float x) {  // order-preserving unsigned key
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unfkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// e^(x - mx) as 2^((x - mx) log2 e) on the MUFU unit (subnormal results kept): relative
// error a few 1e-7 plus 4e-8 per unit of the exponent, far inside the fp32 bar of the tests.
__device__ __forceinline__ float exp_rel(float x, float mx) {
  float r;
  asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"((x - mx) * 1.4426950408889634f));
  return r;
}

__device__ __forceinline__ uint32_t philox_u32(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                               uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

struct Ctl {  // block-shared scalars of the selection stages
  float wtot[kWarps];
  float base, above;
  float z;
  int cut, n;
  uint32_t key, kmax, prefix;
};

__device__ float block_sum_f(float v, Ctl& c) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) c.wtot[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) s += c.wtot[i];
  return s;
}
__device__ float block_max_f(float v, Ctl& c) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) c.wtot[w] = v;
  __syncthreads();
  float s = -INFINITY;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) s = fmaxf(s, c.wtot[i]);
  return s;
}
// Exclusive scan of one value per thread in thread order (fixed order: deterministic).
__device__ float block_excl_scan(float v, Ctl& c, float& total) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) c.wtot[w] = incl;
  __syncthreads();
  float before = 0.f, tot = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) {
    const float t = c.wtot[i];
    before += i < w ? t : 0.f;
    tot += t;
  }
  total = tot;
  return before + incl - v;
}

// Adds `w` (the number of lanes with `take` in the same bin) to hist[bin]: one shared atomic
// per distinct bin per warp.
__device__ __forceinline__ void count_bin(float* hist, bool take, int bin) {
  const uint32_t m = __ballot_sync(0xffffffffu, take);
  if (take) {
    const uint32_t peers = __match_any_sync(m, bin);
    if ((threadIdx.x & 31) == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&hist[bin], (float)__popc(peers));
  }
}

// Adds the lanes' counts and masses to their bins.  When the warp's lanes fall in a few bins
// (a flat row: the top key byte is shared by almost every value) each bin gets one warp-summed
// add; otherwise every lane adds its own.
__device__ __forceinline__ void add_mass(float* cnt, float* ms, bool take, int bin, float w) {
  const int lane = threadIdx.x & 31;
  const uint32_t m = __ballot_sync(0xffffffffu, take);
  uint32_t peers = 0u;
  if (take) peers = __match_any_sync(m, bin);
  const uint32_t leaders = __ballot_sync(0xffffffffu, take && lane == __ffs(peers) - 1);
  if (__popc(leaders) <= 4) {
    uint32_t left = leaders;
    while (left) {
      const int ld = __ffs(left) - 1;
      left &= left - 1;
      const int b = __shfl_sync(0xffffffffu, bin, ld);
      const bool mine = take && bin == b;
      const float sw = warp_sum(mine ? w : 0.f);
      if (lane == ld) {
        atomicAdd(&cnt[b], (float)__popc(peers));
        atomicAdd(&ms[b], sw);
      }
    }
  } else if (take) {
    if (lane == __ffs(peers) - 1) atomicAdd(&cnt[bin], (float)__popc(peers));
    atomicAdd(&ms[bin], w);
  }
}

// Window search for the rule "keep x iff W(> x) <= lim" among the values x >= floor.  The
// window is [mx - width, mx], width = min(16, mx - lo) with lo the smallest value >= floor, cut
// into kNB equal bins.  Returns true and sets thr when the cut was found: in a bin whose values
// fit the list, or in a crowded bin whose values are all equal (all of them are kept then).
template <bool MASS>
__device__ bool window_cut(const float* sx, int V, float mx, float floor_, float lo, float lim_or_p, float* hist,
                           float* lv, float* lw, Ctl& c, float& thr) {
  const int tid = threadIdx.x;
  float width = fminf(kWin, mx - lo);
  if (!(width > 0.f)) width = 1.f;  // a single distinct value (or lo = -inf handled by the min)
  const float inv = (float)kNB / width;
  for (int i = tid; i < kNB; i += kThreads) hist[i] = 0.f;
  if (tid == 0) {
    c.cut = -1;
    c.n = 0;
    c.key = 0xffffffffu;
    c.kmax = 0u;
  }
  __syncthreads();
  float z = 0.f;  // MASS: the softmax normaliser of the values >= floor, in the same pass
  for (int v = tid; v < V; v += kThreads) {
    const float x = sx[v];
    const float d = mx - x;
    const bool in = x >= floor_ && d <= width;
    const int bin = in ? min(kNB - 1, (int)(d * inv)) : 0;
    if (MASS) {
      const float e = x >= floor_ ? exp_rel(x, mx) : 0.f;
      z += e;
      if (in) atomicAdd(&hist[bin], e);
    } else {
      if (in) atomicAdd(&hist[bin], 1.f);
    }
  }
  // MASS: the limit is p * Z; count: k - 1
  const float lim = MASS ? lim_or_p * block_sum_f(z, c) : lim_or_p;
  if (!MASS) __syncthreads();
  if (MASS) c.z = lim;  // the caller reads the limit back for a radix fallback
  // thread t owns bins [kPer t, kPer (t + 1)): the weight above bin b is the scan of the bins before it
  constexpr int kPer = kNB / kThreads;
  float hv[kPer];
  float hs = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    hv[j] = hist[kPer * tid + j];
    hs += hv[j];
  }
  float total;
  float a = block_excl_scan(hs, c, total);
  if (total <= lim) return false;  // every value in the window is kept: the cut lies below it
  int best = -1;
  float best_a = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (hv[j] > 0.f && a <= lim) {
      best = kPer * tid + j;
      best_a = a;
    }
    a += hv[j];
  }
  if (best >= 0) atomicMax(&c.cut, best);
  __syncthreads();
  const int cut = c.cut;  // >= 0: the bin of the maximum qualifies with nothing above it
  if (best == cut) c.base = best_a;
  uint32_t kmin = 0xffffffffu, kmax = 0u;
  for (int v = tid; v < V; v += kThreads) {
    const float x = sx[v];
    const float d = mx - x;
    if (x >= floor_ && d <= width && min(kNB - 1, (int)(d * inv)) == cut) {
      const uint32_t k = fkey(x);
      kmin = min(kmin, k);
      kmax = max(kmax, k);
      const int pos = atomicAdd(&c.n, 1);
      if (pos < kListCap) {
        lv[pos] = x;
        lw[pos] = MASS ? exp_rel(x, mx) : 1.f;
      }
    }
  }
  if (kmin != 0xffffffffu) {
    atomicMin(&c.key, kmin);
    atomicMax(&c.kmax, kmax);
  }
  __syncthreads();
  const int n = c.n;
  if (n > kListCap) {
    const uint32_t k0 = c.key, k1 = c.kmax;
    __syncthreads();
    if (k0 != k1) return false;
    thr = unfkey(k0);  // one value: its weight above is the bin's base, which qualifies
    return true;
  }
  const float base = c.base;
  __syncthreads();  // everyone has read the bin's key range before it is reused
  if (tid == 0) c.key = 0xffffffffu;
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) {
    const float vi = lv[i];
    float s = base;
    for (int j = 0; j < n; ++j) s += lv[j] > vi ? lw[j] : 0.f;
    if (s <= lim) atomicMin(&c.key, fkey(vi));
  }
  __syncthreads();
  thr = unfkey(c.key);
  return true;
}

// Exact descent over the keys of the values x >= floor, 8 bits per pass: the smallest key
// whose weight above it is <= lim.  hist holds 256 counts then 256 masses.
template <bool MASS>
__device__ float radix_cut(const float* sx, int V, float mx, float floor_, float lim, float* hist, Ctl& c) {
  const int tid = threadIdx.x, lane = tid & 31;
  float* cnt = hist;
  float* ms = hist + 256;
  if (tid == 0) {
    c.prefix = 0u;
    c.above = 0.f;
  }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    __syncthreads();
    for (int i = tid; i < 512; i += kThreads) hist[i] = 0.f;
    __syncthreads();
    const uint32_t prefix = c.prefix;
    for (int v0 = 0; v0 < V; v0 += kThreads) {
      const int v = v0 + tid;
      const float x = v < V ? sx[v] : -INFINITY;
      const uint32_t key = fkey(x);
      const bool take = v < V && x >= floor_ && (pass == 0 || (key >> (shift + 8)) == prefix);
      const int bin = (int)((key >> shift) & 255u);
      if (MASS) {
        add_mass(cnt, ms, take, bin, take ? exp_rel(x, mx) : 0.f);
      } else {
        count_bin(cnt, take, bin);
      }
    }
    __syncthreads();
    if (tid < 32) {  // lane l owns bins 255 - 8l ... 248 - 8l, the highest first
      const float* wt = MASS ? ms : cnt;
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) lsum += wt[255 - 8 * lane - i];
      float incl = lsum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      float a = c.above + incl - lsum;
      int best = -1;
      float best_a = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = 255 - 8 * lane - i;
        if (cnt[d] > 0.f && a <= lim) {
          best = d;
          best_a = a;
        }
        a += wt[d];
      }
      // the lowest qualifying bin over the warp (qualifying bins form a run from the top)
      int bd = best >= 0 ? best : 256;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) bd = min(bd, __shfl_xor_sync(0xffffffffu, bd, o));
      if (best >= 0 && best == bd) {
        c.prefix = (prefix << 8) | (uint32_t)bd;
        c.above = best_a;
      }
      if (bd == 256 && lane == 0) c.prefix = (prefix << 8) | 255u;  // unreachable for a non-empty row
    }
  }
  __syncthreads();
  return unfkey(c.prefix);
}

template <bool MASS>
__device__ float stage_cut(const float* sx, int V, float mx, float floor_, float lo, float lim, float* hist,
                           float* lv, float* lw, Ctl& c) {
  float thr;
  if (window_cut<MASS>(sx, V, mx, floor_, lo, lim, hist, lv, lw, c, thr)) return thr;
  return radix_cut<MASS>(sx, V, mx, floor_, MASS ? c.z : lim, hist, c);
}

struct SampleArgs {
  int64_t ld, hist_ld, probs_ld;
  int V, hist_len, top_k;
  float rp, temp, top_p;
  uint32_t seed_lo, seed_hi;
  uint64_t offset;
};

// Eight values of the row as fp32: 16-bit types come from one loaded 16-byte vector, fp32
// reads its second vector here.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& q, const T*, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f(e[i]);
}
template <>
__device__ __forceinline__ void unpack8<float>(const uint4& q, const float* p, float (&f)[8]) {
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = __uint_as_float(q.x), f[1] = __uint_as_float(q.y), f[2] = __uint_as_float(q.z),
  f[3] = __uint_as_float(q.w), f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) sample_kernel(const T* __restrict__ logits,
                                                          const int64_t* __restrict__ hist,
                                                          const float* __restrict__ uniforms,
                                                          const int64_t* __restrict__ offset_dev,
                                                          int64_t* __restrict__ out, float* __restrict__ probs_out,
                                                          const SampleArgs a) {
  extern __shared__ __align__(16) unsigned char sraw[];
  const int V = a.V;
  float* sx = reinterpret_cast<float*>(sraw);
  // after the load, the seen bitmap's space holds the cut bin's values and weights
  unsigned char* uni = sraw + (((size_t)V * 4 + 15) & ~(size_t)15);
  uint32_t* seen = reinterpret_cast<uint32_t*>(uni);
  float* lv = reinterpret_cast<float*>(uni);
  float* lw = lv + kListCap;
  __shared__ __align__(16) float hbuf[kNB];
  __shared__ Ctl c;
  __shared__ uint32_t s_pick;
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const T* lr = logits + row * a.ld;

  // load, repetition penalty over the distinct tokens of the history, temperature, maximum
  const bool pen = a.rp != 1.f && hist != nullptr && a.hist_len > 0;
  if (pen) {
    const int words = (V + 31) / 32;
    for (int i = tid; i < words; i += kThreads) seen[i] = 0u;
    __syncthreads();
    const int64_t* hr = hist + row * a.hist_ld;
    for (int j = tid; j < a.hist_len; j += kThreads) {
      const int64_t t = hr[j];
      if (t >= 0 && t < V) atomicOr(&seen[t >> 5], 1u << (t & 31));
    }
    __syncthreads();
  }
  const float tm = a.temp != 1.f ? fmaxf(a.temp, 1e-5f) : 1.f;
  auto prep = [&](int v, float x) {
    if (pen && ((seen[v >> 5] >> (v & 31)) & 1u)) x = x > 0.f ? x / a.rp : x * a.rp;
    if (a.temp != 1.f) x = x / tm;
    return x;
  };
  float mx = -INFINITY, mn = INFINITY;  // mn: the smallest finite value
  auto track = [&](float x) {
    mx = fmaxf(mx, x);
    if (x > -INFINITY) mn = fminf(mn, x);
  };
  const bool vec = (V % 8 == 0) && ((reinterpret_cast<uintptr_t>(lr) & 15) == 0);
  if (vec) {  // four 16-byte loads in flight per thread, then the arithmetic
    constexpr int U = 4;
    for (int base = tid * 8; base < V; base += kThreads * 8 * U) {
      uint4 q[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = base + u * kThreads * 8;
        if (v < V) q[u] = *reinterpret_cast<const uint4*>(lr + v);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = base + u * kThreads * 8;
        if (v < V) {
          float f[8];
          unpack8<T>(q[u], lr + v, f);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            f[i] = prep(v + i, f[i]);
            track(f[i]);
          }
          reinterpret_cast<float4*>(sx + v)[0] = make_float4(f[0], f[1], f[2], f[3]);
          reinterpret_cast<float4*>(sx + v)[1] = make_float4(f[4], f[5], f[6], f[7]);
        }
      }
    }
  } else {
    for (int v = tid; v < V; v += kThreads) {
      const float x = prep(v, to_f(lr[v]));
      sx[v] = x;
      track(x);
    }
  }
  mx = block_max_f(mx, c);  // (its barriers also publish sx)
  mn = -block_max_f(-mn, c);
  if (mx == -INFINITY) {     // nothing left to sample from
    if (tid == 0) out[row] = -1;
    if (probs_out != nullptr)
      for (int v = tid; v < V; v += kThreads) probs_out[row * a.probs_ld + v] = 0.f;
    return;
  }

  float floor_ = -INFINITY;
  if (a.top_k > 0 && a.top_k < V)
    floor_ = stage_cut<false>(sx, V, mx, floor_, mn, (float)(a.top_k - 1), hbuf, lv, lw, c);
  if (a.top_p > 0.f && a.top_p < 1.f)
    floor_ = fmaxf(floor_, stage_cut<true>(sx, V, mx, floor_, fmaxf(mn, floor_), a.top_p, hbuf, lv, lw, c));

  // softmax and the draw: thread t owns the contiguous segment [t*seg, (t+1)*seg); an odd
  // segment length keeps the threads' strided shared-memory reads on distinct banks
  const int seg = ((V + kThreads - 1) / kThreads) | 1;
  const int v0 = min(V, tid * seg), v1 = min(V, v0 + seg);
  float s = 0.f;
  for (int v = v0; v < v1; ++v) {
    const float x = sx[v];
    float e = 0.f;
    if (x >= floor_) e = exp_rel(x, mx);
    sx[v] = e;
    s += e;
  }
  float Z;
  const float before = block_excl_scan(s, c, Z);
  hbuf[tid] = before;
  if (tid == 0) s_pick = 0xffffffffu;
  float u;
  if (uniforms != nullptr) {
    u = uniforms[row];
  } else {
    const uint64_t off = a.offset + (offset_dev != nullptr ? (uint64_t)*offset_dev : 0ull);
    u = (float)(philox_u32((uint32_t)row, 0u, (uint32_t)off, (uint32_t)(off >> 32), a.seed_lo, a.seed_hi) >> 8) *
        (1.0f / 16777216.0f);
  }
  const float target = u * Z;
  __syncthreads();
  // Segment t owns [scan[t], scan[t + 1]) of the running total, so exactly one segment holds
  // a target below Z; within it, rounding may leave the running sum short of the target, and
  // the segment's last token with mass is taken then.
  const float next = tid + 1 < kThreads ? hbuf[tid + 1] : Z;
  if (before <= target && target < next) {
    float cs = before;
    int pick = -1, last = -1;
    for (int v = v0; v < v1; ++v) {
      const float e = sx[v];
      cs += e;
      if (e > 0.f) {
        last = v;
        if (cs > target) {
          pick = v;
          break;
        }
      }
    }
    pick = pick >= 0 ? pick : last;
    if (pick >= 0) atomicMin(&s_pick, (uint32_t)pick);
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t pick = s_pick;
    if (pick == 0xffffffffu) {  // target at or past the total by rounding: last token with mass
      pick = 0;
      for (int v = V - 1; v >= 0; --v)
        if (sx[v] > 0.f) {
          pick = (uint32_t)v;
          break;
        }
    }
    out[row] = (int64_t)pick;
  }
  if (probs_out != nullptr) {
    const float inv = 1.f / Z;
    for (int v = tid; v < V; v += kThreads) probs_out[row * a.probs_ld + v] = sx[v] * inv;
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

extern "C" int motif_b200_sample(const void* logits, int64_t ld, int64_t B, int64_t V, const int64_t* history,
                                 int64_t hist_ld, int64_t hist_len, float repetition_penalty, float temperature,
                                 int64_t top_k, float top_p, const float* uniforms, uint64_t seed, uint64_t offset,
                                 const int64_t* offset_dev, int64_t* out, float* probs_out, int64_t probs_ld,
                                 int dtype, void* stream) {
  using namespace mb;
  MB_REQUIRE(B >= 0 && B < (1LL << 31) && V > 0 && hist_len >= 0 && hist_len < (1LL << 31), MB_ERR_SHAPE,
             "sample: bad sizes (B %lld, V %lld, history %lld)", (long long)B, (long long)V, (long long)hist_len);
  MB_REQUIRE(V <= kMaxVocab, MB_ERR_UNSUPPORTED, "sample: vocabulary %lld above the %d this kernel holds",
             (long long)V, kMaxVocab);
  MB_REQUIRE(ld >= V && (probs_out == nullptr || probs_ld >= V), MB_ERR_SHAPE, "sample: row stride below V");
  MB_REQUIRE(repetition_penalty > 0.f, MB_ERR_ARG, "sample: repetition penalty must be positive");
  if (B == 0) return MB_OK;
  MB_REQUIRE(logits && out, MB_ERR_ARG, "sample: null pointer");
  MB_REQUIRE(hist_len == 0 || (history != nullptr && hist_ld >= hist_len), MB_ERR_ARG,
             "sample: history pointer / stride");
  const size_t row_bytes = ((size_t)V * 4 + 15) & ~(size_t)15;
  const size_t uni_bytes = std::max<size_t>(((V + 31) / 32) * 4, (size_t)kListCap * 8);
  const int smem = (int)(row_bytes + uni_bytes);
  SampleArgs a;
  a.ld = ld;
  a.hist_ld = hist_ld;
  a.probs_ld = probs_ld;
  a.V = (int)V;
  a.hist_len = (int)hist_len;
  a.top_k = (int)std::min<int64_t>(top_k, (int64_t)1 << 30);
  a.rp = repetition_penalty;
  a.temp = temperature;
  a.top_p = top_p;
  a.seed_lo = (uint32_t)seed;
  a.seed_hi = (uint32_t)(seed >> 32);
  a.offset = offset;
  cudaStream_t st = (cudaStream_t)stream;
  return dispatch(dtype, [&](auto t) {
    using T = decltype(t);
    auto kern = sample_kernel<T>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return check_launch("sample (shared memory attribute)");
    kern<<<(unsigned)B, kThreads, smem, st>>>((const T*)logits, history, uniforms, offset_dev, out, probs_out, a);
    return check_launch("sample");
  });
}
