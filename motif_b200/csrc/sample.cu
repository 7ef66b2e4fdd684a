// One sampled token per row of logits, on the device: repetition penalty -> temperature ->
// top-k -> top-p -> softmax -> draw (motif/model/sampler.py:151-219).  A grammar constraint
// stays on the host side of this kernel: its mask (forbidden tokens -> -inf) is applied to the
// logits before the launch, which gives the same result as applying it after the penalty and
// the temperature (both map -inf to -inf), and its forcing / advance run on the tokens after.
//
// One CTA (512 threads) per row keeps the row in shared memory as fp32:
//   penalty     each distinct token of the row's history once (a bitmap marks them; negative
//               history entries are ignored, so a fixed-size history buffer can be padded with
//               -1), x / rp if x > 0 else x * rp;
//   temperature x / max(T, 1e-5);
//   top-k       radix select (4 passes of 8 bits over order-preserving keys) for the k-th
//               largest value; values below it are dropped (ties with it kept);
//   top-p       radix descent over the same keys on the softmax mass: the smallest key whose
//               mass of strictly larger values is <= p * Z is the cut; values below it are
//               dropped (the reference's sorted-prefix rule, ties at the cut kept);
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

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxVocab = 53248;  // fp32 row + seen bitmap within the 227 KB of shared memory

__device__ __forceinline__ uint32_t fkey(float x) {  // order-preserving unsigned key
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
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

__device__ float block_sum_f(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) s += red[i];
  return s;
}
__device__ float block_max_f(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = -INFINITY;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) s = fmaxf(s, red[i]);
  return s;
}

// Adds one to cnt[bin] for every lane with `take`, one shared atomic per distinct bin per warp
// (the top byte of the keys of a logit row falls in a handful of bins).
__device__ __forceinline__ void count_bin(uint32_t* cnt, bool take, uint32_t bin) {
  const uint32_t m = __ballot_sync(0xffffffffu, take);
  if (take) {
    const uint32_t peers = __match_any_sync(m, bin);
    if ((threadIdx.x & 31) == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&cnt[bin], (uint32_t)__popc(peers));
  }
}

struct SampleArgs {
  int64_t ld, hist_ld, probs_ld;
  int V, hist_len, top_k;
  float rp, temp, top_p;
  uint32_t seed_lo, seed_hi;
  uint64_t offset;
};

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
  uint32_t* seen = reinterpret_cast<uint32_t*>(sx + V);
  __shared__ float red[kWarps];
  __shared__ uint32_t cnt[256];
  __shared__ float msum[256];
  __shared__ uint32_t s_prefix, s_k, s_pick;
  __shared__ float s_above;
  __shared__ float seg_sum[kThreads];
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const T* lr = logits + row * a.ld;
  for (int v = tid; v < V; v += kThreads) sx[v] = to_f(lr[v]);

  // repetition penalty over the distinct tokens of the history
  if (a.rp != 1.f && hist != nullptr && a.hist_len > 0) {
    const int words = (V + 31) / 32;
    for (int i = tid; i < words; i += kThreads) seen[i] = 0u;
    __syncthreads();
    const int64_t* hr = hist + row * a.hist_ld;
    for (int j = tid; j < a.hist_len; j += kThreads) {
      const int64_t t = hr[j];
      if (t >= 0 && t < V) atomicOr(&seen[t >> 5], 1u << (t & 31));
    }
    __syncthreads();
    for (int v = tid; v < V; v += kThreads)
      if ((seen[v >> 5] >> (v & 31)) & 1u) {
        const float x = sx[v];
        sx[v] = x > 0.f ? x / a.rp : x * a.rp;
      }
  }
  if (a.temp != 1.f) {
    const float tm = fmaxf(a.temp, 1e-5f);
    for (int v = tid; v < V; v += kThreads) sx[v] = sx[v] / tm;
  }
  __syncthreads();

  // top-k: the k-th largest key, 8 bits at a time from the top
  if (a.top_k > 0 && a.top_k < V) {
    if (tid == 0) {
      s_prefix = 0u;
      s_k = (uint32_t)a.top_k;
    }
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = tid; i < 256; i += kThreads) cnt[i] = 0u;
      __syncthreads();
      const uint32_t prefix = s_prefix;
      for (int v0 = 0; v0 < V; v0 += kThreads) {
        const int v = v0 + tid;
        const uint32_t key = v < V ? fkey(sx[v]) : 0u;
        const bool take = v < V && (pass == 0 || (key >> (shift + 8)) == prefix);
        count_bin(cnt, take, (key >> shift) & 255u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t above = 0, k = s_k;
        int d = 255;
        for (; d > 0; --d) {
          if (above + cnt[d] >= k) break;
          above += cnt[d];
        }
        s_k = k - above;
        s_prefix = (prefix << 8) | (uint32_t)d;
      }
      __syncthreads();
    }
    const uint32_t kth = s_prefix;
    for (int v = tid; v < V; v += kThreads)
      if (fkey(sx[v]) < kth) sx[v] = -INFINITY;
    __syncthreads();
  }

  float mx = -INFINITY;
  for (int v = tid; v < V; v += kThreads) mx = fmaxf(mx, sx[v]);
  mx = block_max_f(mx, red);
  if (mx == -INFINITY) {  // nothing left to sample from
    if (tid == 0) out[row] = -1;
    if (probs_out != nullptr)
      for (int v = tid; v < V; v += kThreads) probs_out[row * a.probs_ld + v] = 0.f;
    return;
  }

  // top-p: smallest key whose mass of strictly larger values is <= p * Z
  if (a.top_p > 0.f && a.top_p < 1.f) {
    float z = 0.f;
    for (int v = tid; v < V; v += kThreads) z += __expf(sx[v] - mx);
    z = block_sum_f(z, red);
    const float lim = a.top_p * z;
    if (tid == 0) {
      s_prefix = 0u;
      s_above = 0.f;
    }
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = tid; i < 256; i += kThreads) {
        cnt[i] = 0u;
        msum[i] = 0.f;
      }
      __syncthreads();
      const uint32_t prefix = s_prefix;
      for (int v0 = 0; v0 < V; v0 += kThreads) {
        const int v = v0 + tid;
        const float x = v < V ? sx[v] : -INFINITY;
        const uint32_t key = fkey(x);
        const bool take = x != -INFINITY && (pass == 0 || (key >> (shift + 8)) == prefix);
        count_bin(cnt, take, (key >> shift) & 255u);
        if (take) atomicAdd(&msum[(key >> shift) & 255u], __expf(x - mx));
      }
      __syncthreads();
      if (tid == 0) {
        float above = s_above;
        int pick = -1;
        float pick_above = above;
        for (int d = 255; d >= 0; --d) {
          if (cnt[d] == 0u) continue;
          if (above > lim) break;  // this and every lower bucket have too much mass above them
          pick = d;
          pick_above = above;
          above += msum[d];
        }
        if (pick < 0) pick = 255;  // unreachable for a row with a finite maximum
        s_prefix = (prefix << 8) | (uint32_t)pick;
        s_above = pick_above;
      }
      __syncthreads();
    }
    const uint32_t cut = s_prefix;
    for (int v = tid; v < V; v += kThreads)
      if (fkey(sx[v]) < cut) sx[v] = -INFINITY;
    __syncthreads();
  }

  // softmax and the draw: thread t owns the contiguous segment [t*seg, (t+1)*seg)
  const int seg = (V + kThreads - 1) / kThreads;
  const int v0 = min(V, tid * seg), v1 = min(V, v0 + seg);
  float s = 0.f;
  for (int v = v0; v < v1; ++v) {
    const float e = __expf(sx[v] - mx);
    sx[v] = e;
    s += e;
  }
  seg_sum[tid] = s;
  __syncthreads();
  if (tid < 32) {  // exclusive scan of the 512 segment sums in index order (fixed order)
    float part[kThreads / 32];
    float run = 0.f;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) {
      part[i] = run;
      run += seg_sum[tid * (kThreads / 32) + i];
    }
    float incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += y;
    }
    const float excl = incl - run;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) seg_sum[tid * (kThreads / 32) + i] = excl + part[i];
    if (tid == 31) red[0] = incl;  // Z
    if (tid == 0) s_pick = 0xffffffffu;
  }
  __syncthreads();
  const float Z = red[0];
  float u;
  if (uniforms != nullptr) {
    u = uniforms[row];
  } else {
    const uint64_t off = a.offset + (offset_dev != nullptr ? (uint64_t)*offset_dev : 0ull);
    u = (float)(philox_u32((uint32_t)row, 0u, (uint32_t)off, (uint32_t)(off >> 32), a.seed_lo, a.seed_hi) >> 8) *
        (1.0f / 16777216.0f);
  }
  const float target = u * Z;
  // Segment t owns [scan[t], scan[t + 1]) of the running total, so exactly one segment holds
  // a target below Z; within it, rounding may leave the running sum short of the target, and
  // the segment's last token with mass is taken then.
  const float before = seg_sum[tid];
  const float next = tid + 1 < kThreads ? seg_sum[tid + 1] : Z;
  if (before <= target && target < next) {
    float c = before;
    int pick = -1, last = -1;
    for (int v = v0; v < v1; ++v) {
      const float e = sx[v];
      c += e;
      if (e > 0.f) {
        last = v;
        if (c > target) {
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
    if (pick == 0xffffffffu) {  // target at or past the running total by rounding: last token with mass
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
  MB_REQUIRE(logits && out, MB_ERR_ARG, "sample: null pointer");
  MB_REQUIRE(B >= 0 && B < (1LL << 31) && V > 0 && hist_len >= 0 && hist_len < (1LL << 31), MB_ERR_SHAPE,
             "sample: bad sizes (B %lld, V %lld, history %lld)", (long long)B, (long long)V, (long long)hist_len);
  MB_REQUIRE(V <= kMaxVocab, MB_ERR_UNSUPPORTED, "sample: vocabulary %lld above the %d this kernel holds",
             (long long)V, kMaxVocab);
  MB_REQUIRE(ld >= V && (probs_out == nullptr || probs_ld >= V), MB_ERR_SHAPE, "sample: row stride below V");
  MB_REQUIRE(hist_len == 0 || (history != nullptr && hist_ld >= hist_len), MB_ERR_ARG,
             "sample: history pointer / stride");
  MB_REQUIRE(repetition_penalty > 0.f, MB_ERR_ARG, "sample: repetition penalty must be positive");
  if (B == 0) return MB_OK;
  const int smem = (int)(V * 4 + ((V + 31) / 32) * 4);
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
