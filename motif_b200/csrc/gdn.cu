// Gated DeltaNet kernels other than the chunked prefill:
//   * the token-by-token recurrence (op level, any L),
//   * the fused single-token decode step of a whole GDN layer (model level),
//   * the prefill input preparation (causal conv + SiLU + L2 norms + beta/g).
//
// State layout: S[b][h] is a row-major [Dk][Dv] fp32 block.  The recurrent kernels give
// one CTA to each (b, h) and one thread to each value column j, which holds column j of
// S in registers, so every step reads and writes S exactly once, coalesced across j.
#include "common.cuh"

namespace mb {
namespace {

// Element strides q(b,h,l) k(b,h,l) v(b,h,l) o(b,h,l) beta(b,h,l) g(b,h,l), by value.
struct Strides18 {
  int64_t s[18];
};

// --------------------------------------------------------------- recurrence (op level)
// motif/ops/gated_deltanet.py:26-59.  blockDim.x == Dv (<= 256); DK <= 128.
template <typename T, int DK>
__global__ void __launch_bounds__(256) gdn_recurrent_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const float* __restrict__ beta, const float* __restrict__ g, const float* __restrict__ s_in,
    float* __restrict__ s_out, T* __restrict__ o, int H, int L, int Dv, Strides18 sv) {
  const int64_t* st = sv.s;
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int j = threadIdx.x;
  __shared__ float sq[DK], sk[DK];
  float S[DK];
  const size_t sbase = (size_t)bh * DK * Dv;
#pragma unroll
  for (int i = 0; i < DK; ++i) S[i] = s_in ? s_in[sbase + (size_t)i * Dv + j] : 0.f;
  const int64_t qb = b * st[0] + h * st[1], kb = b * st[3] + h * st[4], vb = b * st[6] + h * st[7];
  const int64_t ob = b * st[9] + h * st[10], bb = b * st[12] + h * st[13], gb = b * st[15] + h * st[16];
  for (int t = 0; t < L; ++t) {
    __syncthreads();
    for (int i = j; i < DK; i += blockDim.x) {
      sq[i] = to_f(q[qb + t * st[2] + i]);
      sk[i] = to_f(k[kb + t * st[5] + i]);
    }
    __syncthreads();
    const float e = expf(g[gb + t * st[17]]);
    const float bt = beta[bb + t * st[14]];
    float vo = 0.f;
#pragma unroll
    for (int i = 0; i < DK; ++i) {
      S[i] *= e;
      vo = fmaf(sk[i], S[i], vo);
    }
    const float delta = bt * (to_f(v[vb + t * st[8] + j]) - vo);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < DK; ++i) {
      S[i] = fmaf(sk[i], delta, S[i]);
      acc = fmaf(sq[i], S[i], acc);
    }
    o[ob + t * st[11] + j] = from_f<T>(acc);
  }
#pragma unroll
  for (int i = 0; i < DK; ++i) s_out[sbase + (size_t)i * Dv + j] = S[i];
}

// ------------------------------------------------------------ block reduction helper
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  return s;
}

// ------------------------------------------------------- fused decode step (model level)
// gdn_attn.py:176-209 at L == 1: conv (carried state) + SiLU, F.normalize(q)*Dk^-0.5,
// F.normalize(k), beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias), the recurrent
// step on S, then o_norm(cat[o, gate]) = rmsnorm(o) * w * silu(gate).
// One CTA per (b, h), DV threads; thread j owns value column j (and q/k channel j < DK).
template <typename T, int DK, int DV>
__global__ void __launch_bounds__(DV) gdn_decode_kernel(
    const T* __restrict__ proj, int64_t ps, const T* __restrict__ conv_w, const T* __restrict__ A_log,
    const T* __restrict__ dt_bias, T* __restrict__ conv_state, float* __restrict__ state,
    const T* __restrict__ gate, const T* __restrict__ onw, T* __restrict__ out, int64_t os, int H,
    float eps) {
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int j = threadIdx.x;
  const int C = H * (2 * DK + DV);
  const T* row = proj + (int64_t)b * ps;
  T* cs = conv_state + (int64_t)b * 3 * C;
  __shared__ float sq[DK], sk[DK], red[DV / 32];

  auto conv = [&](int c) -> float {
    const float x = to_f(row[c]);
    const float s0 = to_f(cs[c]), s1 = to_f(cs[C + c]), s2 = to_f(cs[2 * C + c]);
    const T* w = conv_w + (int64_t)c * 4;
    float y = conv4f(to_f(w[0]), to_f(w[1]), to_f(w[2]), to_f(w[3]), s0, s1, s2, x);
    cs[c] = from_f<T>(s1);
    cs[C + c] = from_f<T>(s2);
    cs[2 * C + c] = from_f<T>(x);
    return siluf_(to_f(from_f<T>(y)));
  };
  float qv = 0.f, kv = 0.f;
  if (j < DK) {
    qv = conv(h * DK + j);
    kv = conv(H * DK + h * DK + j);
  }
  const float vv = conv(2 * H * DK + h * DV + j);
  const float qn = block_sum<DV>(qv * qv, red);
  const float kn = block_sum<DV>(kv * kv, red);
  if (j < DK) {
    sq[j] = qv / fmaxf(sqrtf(qn), 1e-12f) * rsqrtf((float)DK);
    sk[j] = kv / fmaxf(sqrtf(kn), 1e-12f);
  }
  const float a = to_f(row[2 * H * DK + H * DV + h]);
  const float bsc = to_f(row[2 * H * DK + H * DV + H + h]);
  const float bt = sigmoidf_(bsc);
  const float gg = -expf(to_f(A_log[h])) * softplusf_(a + to_f(dt_bias[h]));
  __syncthreads();
  float* S = state + ((int64_t)b * H + h) * DK * DV;
  float Sr[DK];
  const float e = expf(gg);
  float vo = 0.f;
#pragma unroll
  for (int i = 0; i < DK; ++i) {
    Sr[i] = S[i * DV + j] * e;
    vo = fmaf(sk[i], Sr[i], vo);
  }
  const float delta = bt * (vv - vo);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < DK; ++i) {
    Sr[i] = fmaf(sk[i], delta, Sr[i]);
    acc = fmaf(sq[i], Sr[i], acc);
    S[i * DV + j] = Sr[i];
  }
  // o.to(dtype) then GatedRMSNorm (rms_norm.py:547-553).
  const float ov = to_f(from_f<T>(acc));
  const float ss = block_sum<DV>(ov * ov, red);
  const float r = rsqrtf(ss / (float)DV + eps);
  float y = to_f(from_f<T>(ov * r));
  y = to_f(from_f<T>(y * to_f(onw[j])));
  const float gt = to_f(gate[(int64_t)b * ps + h * DV + j]);
  out[(int64_t)b * os + h * DV + j] = from_f<T>(y * to_f(from_f<T>(siluf_(gt))));
}

// The same step for the model's shape Dv == 2 * Dk with 2 * Dv threads per (b, head): the
// 2*Dk + Dv conv channels of the head are one per thread (q: threads [0, Dk), k: [Dk, 2Dk),
// v: [2Dk, 4Dk)), and each state column j is split between threads j (rows [0, Dk/2)) and
// j + Dv (rows [Dk/2, Dk)), whose partial kᵀS and qᵀS meet in shared memory.  The state
// loads are issued first, so their latency overlaps the conv, norms and gate math; half
// the registers per thread of the one-column kernel, twice the threads in flight.
template <typename T, int DK, int DV>
__global__ void __launch_bounds__(2 * DV) gdn_decode_split_kernel(
    const T* __restrict__ proj, int64_t ps, const T* __restrict__ conv_w, const T* __restrict__ A_log,
    const T* __restrict__ dt_bias, T* __restrict__ conv_state, float* __restrict__ state,
    const T* __restrict__ gate, const T* __restrict__ onw, T* __restrict__ out, int64_t os, int H,
    float eps, SwigluRole<T> sw, int main_blocks) {
  static_assert(DV == 2 * DK, "one conv channel per thread needs Dv == 2 Dk");
  constexpr int NT = 2 * DV, HR = DK / 2;
  allow_dependent_launch();  // the decoder's output projection may start fetching its weights
  if ((int)blockIdx.x >= main_blocks) {  // trailing CTAs: the decoder's SwiGLU activation
    swiglu_role_run<T>(sw, (int64_t)(blockIdx.x - main_blocks) * NT + threadIdx.x,
                       (int64_t)(gridDim.x - main_blocks) * NT);
    return;
  }
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int tid = threadIdx.x;
  const int j = tid % DV, half = tid / DV;
  const int C = H * (2 * DK + DV);
  const T* row = proj + (int64_t)b * ps;
  T* cs = conv_state + (int64_t)b * 3 * C;
  __shared__ float sq[DK], sk[DK], sv[DV], part[2][DV], red[NT / 32];
  __shared__ float norms[2];

  float* S = state + ((int64_t)b * H + h) * DK * DV + (int64_t)half * HR * DV + j;
  float Sr[HR];
#pragma unroll
  for (int i = 0; i < HR; ++i) Sr[i] = S[i * DV];
  // every other input of the step is requested now too, so the CTA waits for memory once
  const T a_raw = row[2 * H * DK + H * DV + h], b_raw = row[2 * H * DK + H * DV + H + h];
  const T alog_raw = A_log[h], dtb_raw = dt_bias[h];
  const T gate_raw = gate[(int64_t)b * ps + h * DV + j], onw_raw = onw[j];

  // conv + SiLU of this thread's channel (gdn_attn.py:116-136)
  const int c = tid < DK ? h * DK + tid : tid < 2 * DK ? H * DK + h * DK + (tid - DK) : 2 * H * DK + h * DV + (tid - 2 * DK);
  float y;
  {
    const float x = to_f(row[c]);
    const float s0 = to_f(cs[c]), s1 = to_f(cs[C + c]), s2 = to_f(cs[2 * C + c]);
    const T* w = conv_w + (int64_t)c * 4;
    const float acc = conv4f(to_f(w[0]), to_f(w[1]), to_f(w[2]), to_f(w[3]), s0, s1, s2, x);
    cs[c] = from_f<T>(s1);
    cs[C + c] = from_f<T>(s2);
    cs[2 * C + c] = from_f<T>(x);
    y = siluf_(to_f(from_f<T>(acc)));
  }
  // L2 norms of q (warps of threads [0, DK)) and k (threads [DK, 2DK))
  {
    const float sq2 = warp_sum(tid < 2 * DK ? y * y : 0.f);
    if ((tid & 31) == 0) red[tid >> 5] = sq2;
  }
  __syncthreads();
  if (tid < 2) {
    float acc = 0.f;
    for (int w = tid * (DK / 32); w < (tid + 1) * (DK / 32); ++w) acc += red[w];
    norms[tid] = acc;
  }
  __syncthreads();
  if (tid < DK) {
    sq[tid] = y / fmaxf(sqrtf(norms[0]), 1e-12f) * rsqrtf((float)DK);
  } else if (tid < 2 * DK) {
    sk[tid - DK] = y / fmaxf(sqrtf(norms[1]), 1e-12f);
  } else {
    sv[tid - 2 * DK] = y;
  }
  const float bt = sigmoidf_(to_f(b_raw));
  const float gg = -expf(to_f(alog_raw)) * softplusf_(to_f(a_raw) + to_f(dtb_raw));
  const float e = expf(gg);
  __syncthreads();

  // delta rule on the split column: S <- e S;  delta = beta (v - kᵀS);  S += k deltaᵀ;  o = qᵀS
  float vo = 0.f;
#pragma unroll
  for (int i = 0; i < HR; ++i) {
    Sr[i] *= e;
    vo = fmaf(sk[half * HR + i], Sr[i], vo);
  }
  part[half][j] = vo;
  __syncthreads();
  const float delta = bt * (sv[j] - (part[0][j] + part[1][j]));
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < HR; ++i) {
    Sr[i] = fmaf(sk[half * HR + i], delta, Sr[i]);
    acc = fmaf(sq[half * HR + i], Sr[i], acc);
    S[i * DV] = Sr[i];
  }
  __syncthreads();  // every thread has read part[] for its delta
  part[half][j] = acc;
  __syncthreads();
  // o.to(dtype) then GatedRMSNorm over the Dv outputs (rms_norm.py:547-553): threads [0, DV)
  const float ov = to_f(from_f<T>(part[0][j] + part[1][j]));
  const float ss2 = warp_sum(half == 0 ? ov * ov : 0.f);
  if ((tid & 31) == 0) red[tid >> 5] = ss2;
  __syncthreads();
  if (half == 0) {
    float ss = 0.f;
#pragma unroll
    for (int w = 0; w < DV / 32; ++w) ss += red[w];
    const float r = rsqrtf(ss / (float)DV + eps);
    float yo = to_f(from_f<T>(ov * r));
    yo = to_f(from_f<T>(yo * to_f(onw_raw)));
    out[(int64_t)b * os + h * DV + j] = from_f<T>(yo * to_f(from_f<T>(siluf_(to_f(gate_raw)))));
  }
}

// ------------------------------------------------------------- prefill preparation
// gdn_attn.py:116-136 (conv over time with the carried state, SiLU) and :187-197.
// One warp per (b, head, block of TB tokens); lanes own channels and keep a sliding window
// of the last three raw inputs in registers, so each raw element is read once.
template <typename T, int DK, int DV, int TB>
__global__ void __launch_bounds__(128) gdn_prep_kernel(
    const T* __restrict__ proj, int64_t ps, const T* __restrict__ conv_w, const T* __restrict__ A_log,
    const T* __restrict__ dt_bias, const T* __restrict__ conv_in, T* __restrict__ conv_out,
    T* __restrict__ qo, T* __restrict__ ko, T* __restrict__ vo, float* __restrict__ beta,
    float* __restrict__ gout, int Tn, int H) {
  constexpr int QPL = (DK + 31) / 32, VPL = (DV + 31) / 32;
  const int lane = threadIdx.x & 31;
  const int warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nblk = (Tn + TB - 1) / TB;
  const int b = blockIdx.y;
  const int h = warp / nblk, tb = warp % nblk;
  if (h >= H) return;
  const int t0 = tb * TB;
  const int C = H * (2 * DK + DV);
  const T* P = proj + (int64_t)b * Tn * ps;
  // channel ids owned by this lane (-1 = none)
  int cq[QPL], ck[QPL], cv[VPL];
  float wq[QPL][4], wk[QPL][4], wv[VPL][4];
  float hq[QPL][3], hk[QPL][3], hv[VPL][3];
  auto load_w = [&](int c, float* w) {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = c >= 0 ? to_f(conv_w[(int64_t)c * 4 + i]) : 0.f;
  };
  auto raw = [&](int c, int tau) -> float {  // raw input of channel c at time tau (may be < 0)
    if (c < 0) return 0.f;
    if (tau >= 0) return to_f(P[(int64_t)tau * ps + c]);
    return conv_in ? to_f(conv_in[((int64_t)b * 3 + (3 + tau)) * C + c]) : 0.f;
  };
#pragma unroll
  for (int r = 0; r < QPL; ++r) {
    const int d = lane + 32 * r;
    cq[r] = d < DK ? h * DK + d : -1;
    ck[r] = d < DK ? H * DK + h * DK + d : -1;
    load_w(cq[r], wq[r]);
    load_w(ck[r], wk[r]);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      hq[r][i] = raw(cq[r], t0 - 3 + i);
      hk[r][i] = raw(ck[r], t0 - 3 + i);
    }
  }
#pragma unroll
  for (int r = 0; r < VPL; ++r) {
    const int d = lane + 32 * r;
    cv[r] = d < DV ? 2 * H * DK + h * DV + d : -1;
    load_w(cv[r], wv[r]);
#pragma unroll
    for (int i = 0; i < 3; ++i) hv[r][i] = raw(cv[r], t0 - 3 + i);
  }
  const float qscale = rsqrtf((float)DK);
  const float Aexp = -expf(to_f(A_log[h]));
  const float dtb = to_f(dt_bias[h]);
  const int t1 = min(t0 + TB, Tn);
  for (int t = t0; t < t1; ++t) {
    const T* row = P + (int64_t)t * ps;
    float yq[QPL], yk[QPL], yv[VPL];
    float nq = 0.f, nk = 0.f;
#pragma unroll
    for (int r = 0; r < QPL; ++r) {
      const float xq = cq[r] >= 0 ? to_f(row[cq[r]]) : 0.f;
      const float xk = ck[r] >= 0 ? to_f(row[ck[r]]) : 0.f;
      float a = conv4f(wq[r][0], wq[r][1], wq[r][2], wq[r][3], hq[r][0], hq[r][1], hq[r][2], xq);
      float c = conv4f(wk[r][0], wk[r][1], wk[r][2], wk[r][3], hk[r][0], hk[r][1], hk[r][2], xk);
      hq[r][0] = hq[r][1]; hq[r][1] = hq[r][2]; hq[r][2] = xq;
      hk[r][0] = hk[r][1]; hk[r][1] = hk[r][2]; hk[r][2] = xk;
      yq[r] = cq[r] >= 0 ? to_f(from_f<T>(siluf_(to_f(from_f<T>(a))))) : 0.f;
      yk[r] = ck[r] >= 0 ? to_f(from_f<T>(siluf_(to_f(from_f<T>(c))))) : 0.f;
      nq += yq[r] * yq[r];
      nk += yk[r] * yk[r];
    }
#pragma unroll
    for (int r = 0; r < VPL; ++r) {
      const float xv = cv[r] >= 0 ? to_f(row[cv[r]]) : 0.f;
      float a = conv4f(wv[r][0], wv[r][1], wv[r][2], wv[r][3], hv[r][0], hv[r][1], hv[r][2], xv);
      hv[r][0] = hv[r][1]; hv[r][1] = hv[r][2]; hv[r][2] = xv;
      yv[r] = to_f(from_f<T>(siluf_(to_f(from_f<T>(a)))));
    }
    nq = warp_sum(nq);
    nk = warp_sum(nk);
    const float iq = qscale / fmaxf(sqrtf(nq), 1e-12f);
    const float ik = 1.f / fmaxf(sqrtf(nk), 1e-12f);
    const int64_t tok = (int64_t)b * Tn + t;
#pragma unroll
    for (int r = 0; r < QPL; ++r) {
      const int d = lane + 32 * r;
      if (d < DK) {
        qo[tok * H * DK + h * DK + d] = from_f<T>(yq[r] * iq);
        ko[tok * H * DK + h * DK + d] = from_f<T>(yk[r] * ik);
      }
    }
#pragma unroll
    for (int r = 0; r < VPL; ++r) {
      const int d = lane + 32 * r;
      if (d < DV) vo[tok * H * DV + h * DV + d] = from_f<T>(yv[r]);
    }
    if (lane == 0) {
      const float a = to_f(row[2 * H * DK + H * DV + h]);
      const float bb = to_f(row[2 * H * DK + H * DV + H + h]);
      beta[tok * H + h] = to_f(from_f<T>(sigmoidf_(bb)));
      gout[tok * H + h] = to_f(from_f<T>(Aexp * to_f(from_f<T>(softplusf_(to_f(from_f<T>(a + dtb)))))));
    }
  }
  // The last token block writes the new conv state (raw inputs at T-3 .. T-1).
  if (t1 == Tn && conv_out) {
    T* co = conv_out + (int64_t)b * 3 * C;
#pragma unroll
    for (int r = 0; r < QPL; ++r)
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        if (cq[r] >= 0) co[(int64_t)i * C + cq[r]] = from_f<T>(hq[r][i]);
        if (ck[r] >= 0) co[(int64_t)i * C + ck[r]] = from_f<T>(hk[r][i]);
      }
#pragma unroll
    for (int r = 0; r < VPL; ++r)
#pragma unroll
      for (int i = 0; i < 3; ++i)
        if (cv[r] >= 0) co[(int64_t)i * C + cv[r]] = from_f<T>(hv[r][i]);
  }
}

// Vectorised preparation for 16-bit dtypes.  A thread owns 8 consecutive q | k | v channels
// (16-byte loads / stores) for a run of TR tokens: it issues the TR + 3 row loads it needs
// (the 3 before the run are the conv window) up front, so every thread keeps TR + 3
// independent 16-byte loads in flight, then produces the TR output rows.  Consecutive lanes
// own consecutive channel groups, so the DK/8 lanes of one q / k head reduce the head's L2
// norm with 3 xor-shuffles.  Threads whose channel group index is < H also produce beta / g
// of head `group` for the run.
template <typename T, int DK, int DV, int TR>
__global__ void __launch_bounds__(256) gdn_prep_run_kernel(
    const T* __restrict__ proj, int64_t ps, const T* __restrict__ conv_w, const T* __restrict__ A_log,
    const T* __restrict__ dt_bias, const T* __restrict__ conv_in, T* __restrict__ conv_out,
    T* __restrict__ qo, T* __restrict__ ko, T* __restrict__ vo, float* __restrict__ beta,
    float* __restrict__ gout, int Tn, int H) {
  constexpr int GQ = DK / 8;  // lanes per q / k head
  const int C = H * (2 * DK + DV);
  const int ngrp = C / 8;
  const int b = blockIdx.y;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nruns = (Tn + TR - 1) / TR;
  const bool active = gid < (int64_t)ngrp * nruns;
  const int grp = active ? (int)(gid % ngrp) : 0;
  const int run = active ? (int)(gid / ngrp) : 0;
  const int c0 = grp * 8;
  const int kind = c0 < H * DK ? 0 : (c0 < 2 * H * DK ? 1 : 2);
  const int t0 = run * TR;
  const T* P = proj + (int64_t)b * Tn * ps;
  uint4 raw[TR + 3];
#pragma unroll
  for (int j = 0; j < TR + 3; ++j) {
    const int tau = t0 - 3 + j;
    raw[j] = make_uint4(0, 0, 0, 0);
    if (active) {
      if (tau >= 0 && tau < Tn)
        raw[j] = *reinterpret_cast<const uint4*>(P + (int64_t)tau * ps + c0);
      else if (tau < 0 && conv_in)
        raw[j] = *reinterpret_cast<const uint4*>(conv_in + ((int64_t)b * 3 + (3 + tau)) * C + c0);
    }
  }
  float w[8][4];
  {
    const uint4* wp = reinterpret_cast<const uint4*>(conv_w + (int64_t)c0 * 4);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint4 r = active ? wp[u] : make_uint4(0, 0, 0, 0);
      const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
      for (int i = 0; i < 8; ++i) w[2 * u + i / 4][i % 4] = to_f(e[i]);
    }
  }
  const float qscale = rsqrtf((float)DK);
#pragma unroll
  for (int r = 0; r < TR; ++r) {
    const int t = t0 + r;
    float y[8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x0 = to_f(reinterpret_cast<const T*>(&raw[r])[i]);
      const float x1 = to_f(reinterpret_cast<const T*>(&raw[r + 1])[i]);
      const float x2 = to_f(reinterpret_cast<const T*>(&raw[r + 2])[i]);
      const float x3 = to_f(reinterpret_cast<const T*>(&raw[r + 3])[i]);
      const float a = conv4f(w[i][0], w[i][1], w[i][2], w[i][3], x0, x1, x2, x3);
      y[i] = to_f(from_f<T>(siluf_(to_f(from_f<T>(a)))));
      ss += y[i] * y[i];
    }
#pragma unroll
    for (int o = 1; o < GQ; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (!active || t >= Tn) continue;
    const int64_t tok = (int64_t)b * Tn + t;
    T o8[8];
    if (kind == 0) {
      const float sc = l2_scale(ss, qscale);
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] = from_f<T>(y[i] * sc);
      *reinterpret_cast<uint4*>(qo + tok * H * DK + c0) = *reinterpret_cast<uint4*>(o8);
    } else if (kind == 1) {
      const float sc = l2_scale(ss, 1.f);
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] = from_f<T>(y[i] * sc);
      *reinterpret_cast<uint4*>(ko + tok * H * DK + (c0 - H * DK)) = *reinterpret_cast<uint4*>(o8);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] = from_f<T>(y[i]);
      *reinterpret_cast<uint4*>(vo + tok * H * DV + (c0 - 2 * H * DK)) = *reinterpret_cast<uint4*>(o8);
    }
  }
  if (active && grp < H) {
    const int hh = grp;
    const float Aexp = -to_f(from_f<T>(expf(to_f(A_log[hh]))));
    const float dtb = to_f(dt_bias[hh]);
#pragma unroll
    for (int r = 0; r < TR; ++r) {
      const int t = t0 + r;
      if (t >= Tn) break;
      const T* row = P + (int64_t)t * ps;
      const int64_t tok = (int64_t)b * Tn + t;
      beta[tok * H + hh] = to_f(from_f<T>(sigmoidf_(to_f(row[C + H + hh]))));
      gout[tok * H + hh] =
          to_f(from_f<T>(Aexp * to_f(from_f<T>(softplusf_(to_f(from_f<T>(to_f(row[C + hh]) + dtb)))))));
    }
  }
  // the run holding T-1 writes the raw inputs at T-3 .. T-1 as the carried conv state
  const int last = Tn - 1 - t0;
  if (active && conv_out && last >= 0 && last < TR) {
    // raw[j] holds token t0 - 3 + j = Tn - 3 + slot: the window rows before t0 (j < 3) are
    // included, since a last run of one or two tokens leaves the earlier slots there (and
    // positions before 0 hold conv_in or zeros)
#pragma unroll
    for (int j = 0; j < TR + 3; ++j) {
      const int slot = j - last - 1;
      if (slot >= 0 && slot < 3)
        *reinterpret_cast<uint4*>(conv_out + ((int64_t)b * 3 + slot) * C + c0) = raw[j];
    }
  }
}

template <typename F>
int dispatch_dtype(int dtype, F&& f) {
  switch (dtype) {
    case MB_F32: return f(float{});
    case MB_F16: return f(__half{});
    case MB_BF16: return f(__nv_bfloat16{});
    default: return set_error(MB_ERR_DTYPE, "unsupported dtype code %d", dtype);
  }
}

template <typename F>
int dispatch_dk(int64_t dk, F&& f) {
  switch (dk) {
    case 16: return f(std::integral_constant<int, 16>{});
    case 32: return f(std::integral_constant<int, 32>{});
    case 64: return f(std::integral_constant<int, 64>{});
    case 128: return f(std::integral_constant<int, 128>{});
    default: return set_error(MB_ERR_UNSUPPORTED, "head_k_dim %lld not supported (16/32/64/128)", (long long)dk);
  }
}

template <typename F>
int dispatch_dv(int64_t dv, F&& f) {
  switch (dv) {
    case 32: return f(std::integral_constant<int, 32>{});
    case 64: return f(std::integral_constant<int, 64>{});
    case 128: return f(std::integral_constant<int, 128>{});
    case 256: return f(std::integral_constant<int, 256>{});
    default: return set_error(MB_ERR_UNSUPPORTED, "value head dim %lld not supported (32/64/128/256)", (long long)dv);
  }
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" int motif_b200_gdn_recurrent(const void* q, const void* k, const void* v, const float* beta,
                                        const float* g, const float* state_in, float* state_out, void* o,
                                        int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                                        const int64_t* strides, int dtype, void* stream) {
  MB_REQUIRE(state_out && strides, MB_ERR_ARG, "gdn_recurrent: null state_out/strides");
  MB_REQUIRE(L == 0 || (q && k && v && beta && g && o), MB_ERR_ARG, "gdn_recurrent: null input");
  MB_REQUIRE(B >= 0 && H > 0 && L >= 0 && L < 2147483647LL && B * H < 2147483647LL, MB_ERR_SHAPE,
             "gdn_recurrent: bad shape");
  MB_REQUIRE(Dv >= 32 && Dv <= 256 && Dv % 32 == 0, MB_ERR_UNSUPPORTED,
             "gdn_recurrent: value dim %lld must be a multiple of 32 in [32, 256]", (long long)Dv);
  if (B == 0) return MB_OK;
  Strides18 sv;
  for (int i = 0; i < 18; ++i) sv.s[i] = strides[i];
  return dispatch_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return dispatch_dk(Dk, [&](auto dkc) {
      constexpr int DK = decltype(dkc)::value;
      gdn_recurrent_kernel<T, DK><<<(unsigned)(B * H), (unsigned)Dv, 0, (cudaStream_t)stream>>>(
          (const T*)q, (const T*)k, (const T*)v, beta, g, state_in, state_out, (T*)o, (int)H, (int)L,
          (int)Dv, sv);
      return check_launch("gdn_recurrent");
    });
  });
}

namespace mb {
namespace {
// The L == 1 step, with the decoder's SwiGLU activation in the same launch when `hid` > 0 and
// the split kernel runs (otherwise a separate motif_b200_swiglu launch follows).
int gdn_decode_impl(const void* proj, int64_t ps, const void* conv_w, const void* A_log, const void* dt_bias,
                    void* conv_state, float* state, const void* gate, const void* onorm_w, void* out, int64_t os,
                    int64_t B, int64_t H, int64_t Dk, int64_t Dv, float eps, int dtype, void* stream,
                    const void* gu, int64_t gs, void* act, int64_t as, int64_t hid) {
  MB_REQUIRE(proj && conv_w && A_log && dt_bias && conv_state && state && gate && onorm_w && out,
             MB_ERR_ARG, "gdn_decode: null pointer");
  MB_REQUIRE(B >= 0 && H > 0 && B * H < 2147483647LL, MB_ERR_SHAPE, "gdn_decode: bad shape");
  MB_REQUIRE(Dv >= Dk, MB_ERR_UNSUPPORTED, "gdn_decode: needs Dv >= Dk");
  MB_REQUIRE(hid == 0 || (gu && act && hid > 0 && hid <= (1 << 24)), MB_ERR_ARG, "gdn_decode_swiglu: bad MLP args");
  if (B == 0) return MB_OK;
  bool fused = false;
  const int rc = dispatch_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    return dispatch_dk(Dk, [&](auto dkc) {
      constexpr int DK = decltype(dkc)::value;
      return dispatch_dv(Dv, [&](auto dvc) {
        constexpr int DV = decltype(dvc)::value;
        if constexpr (DV < DK) {
          return set_error(MB_ERR_UNSUPPORTED, "gdn_decode: needs Dv >= Dk");
        } else if constexpr (DV == 2 * DK && DK % 32 == 0 && 2 * DV <= 512) {
          SwigluRole<T> sw{(const T*)gu, gs, (T*)act, as, B, 0};
          int64_t extra = 0;
          if (sizeof(T) == 2 && swiglu_role_ok(gu, gs, act, as, hid)) {
            sw.hid = (int)hid;
            extra = swiglu_role_blocks(B, hid, 2 * DV);
            fused = true;
          }
          gdn_decode_split_kernel<T, DK, DV><<<(unsigned)(B * H + extra), 2 * DV, 0, (cudaStream_t)stream>>>(
              (const T*)proj, ps, (const T*)conv_w, (const T*)A_log, (const T*)dt_bias, (T*)conv_state,
              state, (const T*)gate, (const T*)onorm_w, (T*)out, os, (int)H, eps, sw, (int)(B * H));
          return check_launch("gdn_decode");
        } else {
          gdn_decode_kernel<T, DK, DV><<<(unsigned)(B * H), DV, 0, (cudaStream_t)stream>>>(
              (const T*)proj, ps, (const T*)conv_w, (const T*)A_log, (const T*)dt_bias, (T*)conv_state,
              state, (const T*)gate, (const T*)onorm_w, (T*)out, os, (int)H, eps);
          return check_launch("gdn_decode");
        }
      });
    });
  });
  if (rc || hid == 0 || fused) return rc;
  return motif_b200_swiglu(gu, act, B, hid, gs, as, dtype, stream);
}
}  // namespace
}  // namespace mb

extern "C" int motif_b200_gdn_decode(const void* proj, int64_t ps, const void* conv_w, const void* A_log,
                                     const void* dt_bias, void* conv_state, float* state, const void* gate,
                                     const void* onorm_w, void* out, int64_t os, int64_t B, int64_t H,
                                     int64_t Dk, int64_t Dv, float eps, int dtype, void* stream) {
  return mb::gdn_decode_impl(proj, ps, conv_w, A_log, dt_bias, conv_state, state, gate, onorm_w, out, os, B, H, Dk,
                             Dv, eps, dtype, stream, nullptr, 0, nullptr, 0, 0);
}

extern "C" int motif_b200_gdn_decode_swiglu(const void* proj, int64_t ps, const void* conv_w, const void* A_log,
                                            const void* dt_bias, void* conv_state, float* state, const void* gate,
                                            const void* onorm_w, void* out, int64_t os, int64_t B, int64_t H,
                                            int64_t Dk, int64_t Dv, float eps, const void* gu, int64_t gu_stride,
                                            void* act, int64_t act_stride, int64_t hid, int dtype, void* stream) {
  MB_REQUIRE(gu && act && hid > 0, MB_ERR_ARG, "gdn_decode_swiglu: null MLP pointer or hid <= 0");
  return mb::gdn_decode_impl(proj, ps, conv_w, A_log, dt_bias, conv_state, state, gate, onorm_w, out, os, B, H, Dk,
                             Dv, eps, dtype, stream, gu, gu_stride, act, act_stride, hid);
}

extern "C" int motif_b200_gdn_prep(const void* proj, int64_t ps, const void* conv_w, const void* A_log,
                                   const void* dt_bias, const void* conv_in, void* conv_out, void* q, void* k,
                                   void* v, float* beta, float* g, int64_t B, int64_t T, int64_t H, int64_t Dk,
                                   int64_t Dv, int dtype, void* stream) {
  MB_REQUIRE(proj && conv_w && A_log && dt_bias && q && k && v && beta && g, MB_ERR_ARG,
             "gdn_prep: null pointer");
  MB_REQUIRE(conv_out == nullptr || conv_out != conv_in, MB_ERR_ARG, "gdn_prep: conv_out must not alias conv_in");
  MB_REQUIRE(B >= 0 && B < 65536 && T >= 0 && T < (1LL << 30) && H > 0, MB_ERR_SHAPE, "gdn_prep: bad shape");
  if (B == 0 || T == 0) return MB_OK;
  constexpr int TB = 16;
  return dispatch_dtype(dtype, [&](auto t) {
    using Tt = decltype(t);
    return dispatch_dk(Dk, [&](auto dkc) {
      constexpr int DK = decltype(dkc)::value;
      return dispatch_dv(Dv, [&](auto dvc) {
        constexpr int DV = decltype(dvc)::value;
        const int64_t C = H * (2 * DK + DV);
        const bool vec = sizeof(Tt) == 2 && ps % 8 == 0 && ((uintptr_t)proj | (uintptr_t)conv_w | (uintptr_t)q |
                                                            (uintptr_t)k | (uintptr_t)v | (uintptr_t)conv_in |
                                                            (uintptr_t)conv_out) % 16 == 0 &&
                         B < 65536;
        if constexpr (sizeof(Tt) == 2) {
          if (vec && DK >= 8) {
            constexpr int TR = 8;
            const int64_t threads = (C / 8) * ((T + TR - 1) / TR);
            dim3 grid((unsigned)((threads + 255) / 256), (unsigned)B);
            gdn_prep_run_kernel<Tt, DK, DV, TR><<<grid, 256, 0, (cudaStream_t)stream>>>(
                (const Tt*)proj, ps, (const Tt*)conv_w, (const Tt*)A_log, (const Tt*)dt_bias, (const Tt*)conv_in,
                (Tt*)conv_out, (Tt*)q, (Tt*)k, (Tt*)v, beta, g, (int)T, (int)H);
            return check_launch("gdn_prep");
          }
        }
        const int64_t warps = H * ((T + TB - 1) / TB);
        dim3 grid((unsigned)((warps + 3) / 4), (unsigned)B);
        gdn_prep_kernel<Tt, DK, DV, TB><<<grid, 128, 0, (cudaStream_t)stream>>>(
            (const Tt*)proj, ps, (const Tt*)conv_w, (const Tt*)A_log, (const Tt*)dt_bias, (const Tt*)conv_in,
            (Tt*)conv_out, (Tt*)q, (Tt*)k, (Tt*)v, beta, g, (int)T, (int)H);
        return check_launch("gdn_prep");
      });
    });
  });
}
