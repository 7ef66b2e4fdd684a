// Backward kernels (gradients for training) of the three hot-path ops, in fp32 arithmetic on
// CUDA cores (fp16 / bf16 inputs are widened on load; parameter gradients accumulate in fp64):
//
// * Chord attention (motif/ops/chord_attention.py:518-958, 1348-1445).  Forward:
//     logit_ij = (scale q_i.k_j + b_h(j - q_start - i)) c_i,  c_i = ssmax_h log_n[b, i],
//     b_h(d) = -alpha_h (|d - mu_h| + eps)^beta_h,  P = softmax_j(logit) over j <= q_start + i,
//     O = P V.
//   With dO: dP_ij = dO_i.v_j, delta_i = dO_i.O_i, dl_ij = P_ij (dP_ij - delta_i),
//   ds_ij = dl_ij c_i, dq_i = scale sum_j ds_ij k_j, dk_j = scale sum_i ds_ij q_i,
//   dv_j = sum_i P_ij dO_i (k, v summed over the heads of their GQA group), and per head
//   d alpha = sum ds (-u^beta), d beta = sum ds (-alpha u^beta ln u),
//   d mu = sum ds (alpha beta u^(beta-1) sgn(d - mu)), d ssmax = sum_i log_n_i sum_j dl_ij (s + b)_ij,
//   u = |d - mu| + eps.
//   chord_bwd_q_kernel (grid: query tiles x heads x batch) recomputes each row's log-sum-exp
//   (first sweep over the key tiles), then dq and the per-CTA partials of the four parameter
//   gradients (second sweep); it stores lse, delta and c for chord_bwd_kv_kernel (grid: key
//   tiles x kv heads x batch), which sums dk and dv over every query row and group head that
//   sees its keys.  The bias terms come from a per-tile table over the distances the tile spans.
// * AttnRes (motif/ops/attn_res.py:188-364): see attn_res_bwd_kernel.
// * Gated delta rule (motif/ops/gated_deltanet.py:427-611, 726-765): see gdn_bwd_kernel.
#include <algorithm>

#include "common.cuh"

namespace mb {
namespace {

constexpr int kBM = 32, kBN = 32, kBT = 256;  // query rows, keys per tile; threads

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  return to_f(*p);
}

struct ChordBwdArgs {
  const void *q, *k, *v, *o, *dout;
  const float *alpha, *beta, *mu, *ssmax, *log_n;
  void *dq, *dk, *dv;
  float *lse, *delta, *crow;  // [B][H][L]
  double* part;               // [B][H][tiles][4]
  int64_t sq[3], sk[3], sv[3], so[3], sd[3], sdq[3], sdk[3], sdv[3], sl[2];
  int B, H, Hkv, L, S, q_start;
  float scale, eps;
};

// The bias table of one tile: entries for distances d0 .. d0 + n - 1 (d = j - q_start - i).
struct BiasTab {
  float b[kBM + kBN], ga[kBM + kBN], gb[kBM + kBN], gm[kBM + kBN];
};
__device__ __forceinline__ void fill_tab(BiasTab& t, int d0, float al, float be, float mu, float eps, int tid) {
  for (int e = tid; e < kBM + kBN - 1; e += kBT) {
    const float d = (float)(d0 + e);
    const float u = fabsf(d - mu) + eps;
    const float pw = powf(u, be);
    const float sg = d > mu ? 1.f : (d < mu ? -1.f : 0.f);
    t.b[e] = -al * pw;
    t.ga[e] = -pw;
    t.gb[e] = -al * pw * logf(u);
    t.gm[e] = al * be * (pw / u) * sg;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kBT) chord_bwd_q_kernel(ChordBwdArgs a) {
  constexpr int DP = D + 1;
  extern __shared__ float sm[];
  float* Qs = sm;                  // [kBM][DP]
  float* Os = Qs + kBM * DP;       // dO rows
  float* Ks = Os + kBM * DP;       // [kBN][DP]
  float* Vs = Ks + kBN * DP;
  float* dsS = Vs + kBN * DP;      // [kBM][kBN + 1]
  BiasTab* tab = reinterpret_cast<BiasTab*>(dsS + kBM * (kBN + 1));
  double* red = reinterpret_cast<double*>(tab + 1);  // [kBT / 32][4]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int i0 = blockIdx.x * kBM, h = blockIdx.y, b = blockIdx.z;
  const int G = a.H / a.Hkv, kvh = h / G;
  const T* q = (const T*)a.q + b * a.sq[0] + h * a.sq[1];
  const T* o = (const T*)a.o + b * a.so[0] + h * a.so[1];
  const T* dO = (const T*)a.dout + b * a.sd[0] + h * a.sd[1];
  const T* k = (const T*)a.k + b * a.sk[0] + kvh * a.sk[1];
  const T* v = (const T*)a.v + b * a.sv[0] + kvh * a.sv[1];
  const float al = a.alpha[h], be = a.beta[h], mu = a.mu[h], ss = a.ssmax[h];

  // rows, dO rows, delta_i = dO_i . O_i
  for (int e = tid; e < kBM * D; e += kBT) {
    const int r = e / D, d = e % D, i = i0 + r;
    Qs[r * DP + d] = i < a.L ? ldf(q + (int64_t)i * a.sq[2] + d) : 0.f;
    Os[r * DP + d] = i < a.L ? ldf(dO + (int64_t)i * a.sd[2] + d) : 0.f;
  }
  // thread: row r = tid / 8, keys kg + 8 m (m < 4); the 8 threads of a row are adjacent lanes
  const int r = tid >> 3, kg = tid & 7, i = i0 + r;
  const bool row_ok = i < a.L;
  const int qpos = a.q_start + i;
  const float c = row_ok ? ss * a.log_n[b * a.sl[0] + (int64_t)i * a.sl[1]] : 0.f;
  float dl_o = 0.f;
  if (row_ok)
    for (int d = kg; d < D; d += 8) dl_o += ldf(o + (int64_t)i * a.so[2] + d) * ldf(dO + (int64_t)i * a.sd[2] + d);
#pragma unroll
  for (int w = 1; w < 8; w <<= 1) dl_o += __shfl_xor_sync(0xffffffffu, dl_o, w);
  const float delta = dl_o;
  const int kv_end = min(a.S, a.q_start + min(a.L, i0 + kBM));  // keys any row of the tile sees
  const int ntile = (kv_end + kBN - 1) / kBN;

  auto load_kv = [&](int j0, bool with_v) {
    for (int e = tid; e < kBN * D; e += kBT) {
      const int jj = e / D, d = e % D, j = j0 + jj;
      Ks[jj * DP + d] = j < a.S ? ldf(k + (int64_t)j * a.sk[2] + d) : 0.f;
      if (with_v) Vs[jj * DP + d] = j < a.S ? ldf(v + (int64_t)j * a.sv[2] + d) : 0.f;
    }
  };
  // logits of this thread's 4 keys, and s + b (in fp64: the ssmax gradient sums P dP (s + b)
  // against its row mean, and fp32 dot-product rounding would dominate that sum)
  auto logits = [&](int j0, float (&x)[4], double (&sb)[4]) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int jj = kg + 8 * m, j = j0 + jj;
      double sd = 0.0;
#pragma unroll 8
      for (int d = 0; d < D; ++d) sd = fma((double)Qs[r * DP + d], (double)Ks[jj * DP + d], sd);
      sb[m] = sd * (double)a.scale + (double)tab->b[jj - r + kBM - 1];
      const bool vis = row_ok && j < a.S && j <= qpos;
      x[m] = vis ? (float)(sb[m] * (double)c) : -INFINITY;
    }
  };
  // the tile's distances: j - q_start - i for j in [j0, j0 + kBN), i in [i0, i0 + kBM)
  auto tab_d0 = [&](int j0) { return j0 - a.q_start - i0 - (kBM - 1); };

  // sweep 1: the row's log-sum-exp, and the P-weighted row means of the three bias-parameter
  // terms and of s + b.  The parameter gradients use them: with sum_j P_ij = 1 and
  // delta_i = sum_j P_ij dP_ij, a row's share sum_j ds_ij A_ij equals
  // c_i sum_j P_ij (dP_ij - delta_i) (A_ij - mean_i(A)) exactly, a sum without the
  // cancellation of sum_j P_ij (dP_ij - delta_i) A_ij (whose P (dP - delta) factors sum to zero
  // along the row while A varies little).
  float m_run = -INFINITY, l_run = 0.f;
  double mean_run[4] = {0.0, 0.0, 0.0, 0.0};
  for (int t = 0; t < ntile; ++t) {
    const int j0 = t * kBN;
    __syncthreads();
    load_kv(j0, false);
    fill_tab(*tab, tab_d0(j0), al, be, mu, a.eps, tid);
    __syncthreads();
    float x[4];
    double sb[4];
    logits(j0, x, sb);
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
#pragma unroll
    for (int w = 1; w < 8; w <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, w));
    const float mn = fmaxf(m_run, mx);
    float ps = 0.f;
    double pm[4] = {0.0, 0.0, 0.0, 0.0};
    if (mn > -INFINITY) {
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float e = expf(x[m] - mn);
        const int te = kg + 8 * m - r + kBM - 1;
        ps += e;
        pm[0] = fma((double)e, (double)tab->ga[te], pm[0]);
        pm[1] = fma((double)e, (double)tab->gb[te], pm[1]);
        pm[2] = fma((double)e, (double)tab->gm[te], pm[2]);
        pm[3] = fma((double)e, sb[m], pm[3]);
      }
    }
#pragma unroll
    for (int w = 1; w < 8; w <<= 1) {
      ps += __shfl_xor_sync(0xffffffffu, ps, w);
#pragma unroll
      for (int e = 0; e < 4; ++e) pm[e] += __shfl_xor_sync(0xffffffffu, pm[e], w);
    }
    const float f = m_run > -INFINITY ? expf(m_run - mn) : 0.f;
    l_run = l_run * f + ps;
#pragma unroll
    for (int e = 0; e < 4; ++e) mean_run[e] = mean_run[e] * (double)f + pm[e];
    m_run = mn;
  }
  const float lse = m_run > -INFINITY ? m_run + logf(l_run) : -INFINITY;
  double mean[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) mean[e] = l_run > 0.f ? mean_run[e] / (double)l_run : 0.0;
  if (row_ok && kg == 0) {
    const int64_t ri = ((int64_t)b * a.H + h) * a.L + i;
    a.lse[ri] = lse;
    a.delta[ri] = delta;
    a.crow[ri] = c;
  }

  // sweep 2: dq and the parameter gradients
  constexpr int DQ = D / 8;  // dq dims per thread: kg + 8 u
  float dq[DQ];
#pragma unroll
  for (int u = 0; u < DQ; ++u) dq[u] = 0.f;
  double ga = 0.0, gb = 0.0, gm = 0.0, gc = 0.0;
  for (int t = 0; t < ntile; ++t) {
    const int j0 = t * kBN;
    __syncthreads();
    load_kv(j0, true);
    fill_tab(*tab, tab_d0(j0), al, be, mu, a.eps, tid);
    __syncthreads();
    float x[4];
    double sb[4];
    logits(j0, x, sb);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int jj = kg + 8 * m;
      float dp = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) dp = fmaf(Os[r * DP + d], Vs[jj * DP + d], dp);
      const float p = x[m] > -INFINITY ? expf(x[m] - lse) : 0.f;
      dsS[r * (kBN + 1) + jj] = p * (dp - delta) * c * a.scale;
      if (p > 0.f) {
        const int e = jj - r + kBM - 1;
        // both factors centred: P (dP - delta) (A - mean(A)) sums to the same value as
        // P dP (A - mean(A)) or P (dP - delta) A, but neither the rounding of the row means
        // (sum_j P (A - mean) is zero only up to it) nor that of delta is amplified
        const double pd = (double)p * ((double)dp - (double)delta);
        ga = fma(pd, (double)tab->ga[e] - mean[0], ga);
        gb = fma(pd, (double)tab->gb[e] - mean[1], gb);
        gm = fma(pd, (double)tab->gm[e] - mean[2], gm);
        gc = fma(pd, sb[m] - mean[3], gc);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int jj = 0; jj < kBN; ++jj) {
      const float w = dsS[r * (kBN + 1) + jj];
#pragma unroll
      for (int u = 0; u < DQ; ++u) dq[u] = fmaf(w, Ks[jj * DP + kg + 8 * u], dq[u]);
    }
  }
  if (row_ok) {
    T* dqp = (T*)a.dq + b * a.sdq[0] + h * a.sdq[1] + (int64_t)i * a.sdq[2];
#pragma unroll
    for (int u = 0; u < DQ; ++u) dqp[kg + 8 * u] = from_f<T>(dq[u]);
  }
  // the row factors: c_i for the bias parameters, log_n_i (= c_i / ssmax_h) for ssmax
  const double lnn = row_ok ? (double)a.log_n[b * a.sl[0] + (int64_t)i * a.sl[1]] : 0.0;
  ga *= (double)c;
  gb *= (double)c;
  gm *= (double)c;
  gc *= lnn;
  double vals[4] = {ga, gb, gm, gc};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) vals[e] += __shfl_xor_sync(0xffffffffu, vals[e], w);
  }
  __syncthreads();
  if (lane == 0)
#pragma unroll
    for (int e = 0; e < 4; ++e) red[warp * 4 + e] = vals[e];
  __syncthreads();
  if (tid < 4) {
    double s = 0.0;
    for (int w = 0; w < kBT / 32; ++w) s += red[w * 4 + tid];
    a.part[(((int64_t)b * a.H + h) * gridDim.x + blockIdx.x) * 4 + tid] = s;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kBT) chord_bwd_kv_kernel(ChordBwdArgs a) {
  constexpr int DP = D + 1;
  extern __shared__ float sm[];
  float* Ks = sm;                  // this CTA's keys [kBN][DP]
  float* Vs = Ks + kBN * DP;
  float* Qs = Vs + kBN * DP;       // a query tile [kBM][DP]
  float* Os = Qs + kBM * DP;       // its dO rows
  float* Ps = Os + kBM * DP;       // [kBN][kBM + 1] probabilities
  float* dsS = Ps + kBN * (kBM + 1);
  float* rowv = dsS + kBN * (kBM + 1);  // lse, delta, c of the tile's rows [3][kBM]
  BiasTab* tab = reinterpret_cast<BiasTab*>(rowv + 3 * kBM);
  const int tid = threadIdx.x;
  const int j0 = blockIdx.x * kBN, kvh = blockIdx.y, b = blockIdx.z;
  const int G = a.H / a.Hkv;
  const T* k = (const T*)a.k + b * a.sk[0] + kvh * a.sk[1];
  const T* v = (const T*)a.v + b * a.sv[0] + kvh * a.sv[1];
  for (int e = tid; e < kBN * D; e += kBT) {
    const int jj = e / D, d = e % D, j = j0 + jj;
    Ks[jj * DP + d] = j < a.S ? ldf(k + (int64_t)j * a.sk[2] + d) : 0.f;
    Vs[jj * DP + d] = j < a.S ? ldf(v + (int64_t)j * a.sv[2] + d) : 0.f;
  }
  // thread: key jj = tid / 8, rows rg + 8 m (m < 4); dims rg + 8 u of dk / dv
  const int jj = tid >> 3, rg = tid & 7, j = j0 + jj;
  constexpr int DU = D / 8;
  float dk[DU], dv[DU];
#pragma unroll
  for (int u = 0; u < DU; ++u) dk[u] = dv[u] = 0.f;
  // rows that see key j0 or later: q_start + i >= j0
  const int i_first = max(0, j0 - a.q_start);
  for (int gh = 0; gh < G; ++gh) {
    const int h = kvh * G + gh;
    const T* q = (const T*)a.q + b * a.sq[0] + h * a.sq[1];
    const T* dO = (const T*)a.dout + b * a.sd[0] + h * a.sd[1];
    const float al = a.alpha[h], be = a.beta[h], mu = a.mu[h];
    for (int i0 = i_first / kBM * kBM; i0 < a.L; i0 += kBM) {
      __syncthreads();
      for (int e = tid; e < kBM * D; e += kBT) {
        const int r = e / D, d = e % D, i = i0 + r;
        Qs[r * DP + d] = i < a.L ? ldf(q + (int64_t)i * a.sq[2] + d) : 0.f;
        Os[r * DP + d] = i < a.L ? ldf(dO + (int64_t)i * a.sd[2] + d) : 0.f;
      }
      if (tid < kBM) {
        const int i = i0 + tid;
        const int64_t ri = ((int64_t)b * a.H + h) * a.L + i;
        rowv[tid] = i < a.L ? a.lse[ri] : -INFINITY;
        rowv[kBM + tid] = i < a.L ? a.delta[ri] : 0.f;
        rowv[2 * kBM + tid] = i < a.L ? a.crow[ri] : 0.f;
      }
      fill_tab(*tab, j0 - a.q_start - i0 - (kBM - 1), al, be, mu, a.eps, tid);
      __syncthreads();
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int r = rg + 8 * m, i = i0 + r;
        float s = 0.f, dp = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; ++d) {
          s = fmaf(Qs[r * DP + d], Ks[jj * DP + d], s);
          dp = fmaf(Os[r * DP + d], Vs[jj * DP + d], dp);
        }
        const float lse = rowv[r], c = rowv[2 * kBM + r];
        const bool vis = i < a.L && j < a.S && j <= a.q_start + i && lse > -INFINITY;
        const float x = (s * a.scale + tab->b[jj - r + kBM - 1]) * c;
        const float p = vis ? expf(x - lse) : 0.f;
        Ps[jj * (kBM + 1) + r] = p;
        dsS[jj * (kBM + 1) + r] = p * (dp - rowv[kBM + r]) * c * a.scale;
      }
      __syncthreads();
#pragma unroll 4
      for (int r = 0; r < kBM; ++r) {
        const float p = Ps[jj * (kBM + 1) + r], ds = dsS[jj * (kBM + 1) + r];
#pragma unroll
        for (int u = 0; u < DU; ++u) {
          dv[u] = fmaf(p, Os[r * DP + rg + 8 * u], dv[u]);
          dk[u] = fmaf(ds, Qs[r * DP + rg + 8 * u], dk[u]);
        }
      }
    }
  }
  if (j < a.S) {
    T* dkp = (T*)a.dk + b * a.sdk[0] + kvh * a.sdk[1] + (int64_t)j * a.sdk[2];
    T* dvp = (T*)a.dv + b * a.sdv[0] + kvh * a.sdv[1] + (int64_t)j * a.sdv[2];
#pragma unroll
    for (int u = 0; u < DU; ++u) {
      dkp[rg + 8 * u] = from_f<T>(dk[u]);
      dvp[rg + 8 * u] = from_f<T>(dv[u]);
    }
  }
}

template <int D>
size_t q_smem() {
  return (size_t)(2 * kBM * (D + 1) + 2 * kBN * (D + 1) + kBM * (kBN + 1)) * 4 + sizeof(BiasTab) + 8 * 4 * 8;
}
template <int D>
size_t kv_smem() {
  return (size_t)(2 * kBN * (D + 1) + 2 * kBM * (D + 1) + 2 * kBN * (kBM + 1) + 3 * kBM) * 4 + sizeof(BiasTab);
}

template <typename T, int D>
int launch_chord_bwd(ChordBwdArgs& a, cudaStream_t st) {
  auto kq = chord_bwd_q_kernel<T, D>;
  auto kkv = chord_bwd_kv_kernel<T, D>;
  if (int rc = ensure_smem_attr((const void*)kq, (int)q_smem<D>())) return rc;
  if (int rc = ensure_smem_attr((const void*)kkv, (int)kv_smem<D>())) return rc;
  const int tq = (a.L + kBM - 1) / kBM, tk = (a.S + kBN - 1) / kBN;
  kq<<<dim3(tq, a.H, a.B), kBT, q_smem<D>(), st>>>(a);
  if (int rc = check_launch("chord_backward (dq)")) return rc;
  kkv<<<dim3(tk, a.Hkv, a.B), kBT, kv_smem<D>(), st>>>(a);
  return check_launch("chord_backward (dk, dv)");
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" int64_t motif_b200_chord_backward_workspace_bytes(int64_t B, int64_t H, int64_t L) {
  const int64_t tq = (L + kBM - 1) / kBM;
  return 3 * B * H * L * 4 + ((B * H * tq * 4 * 8 + 15) / 16) * 16;
}

extern "C" int motif_b200_chord_backward(const void* q, const void* k, const void* v, const void* out,
                                         const void* dout, const float* alpha, const float* beta, const float* mu,
                                         const float* ssmax, const float* log_n, void* dq, void* dk, void* dv,
                                         int64_t B, int64_t H, int64_t Hkv, int64_t L, int64_t S, int64_t D,
                                         int64_t q_start, float scale, float eps, const int64_t* strides,
                                         void* workspace, int64_t workspace_bytes, double* param_partials,
                                         int dtype, void* stream) {
  MB_REQUIRE(q && k && v && out && dout && alpha && beta && mu && ssmax && log_n && dq && dk && dv && strides,
             MB_ERR_ARG, "chord_backward: null pointer");
  MB_REQUIRE(B >= 0 && H > 0 && Hkv > 0 && H % Hkv == 0 && L >= 0 && S >= 0 && q_start >= 0, MB_ERR_SHAPE,
             "chord_backward: bad shape");
  MB_REQUIRE(B * H < 65536 && H < 65536 && L < (1LL << 30) && S < (1LL << 30), MB_ERR_SHAPE,
             "chord_backward: shape too large");
  MB_REQUIRE(D == 16 || D == 32 || D == 64 || D == 128, MB_ERR_UNSUPPORTED,
             "chord_backward: head dim %lld (16, 32, 64 or 128)", (long long)D);
  MB_REQUIRE(workspace != nullptr && workspace_bytes >= motif_b200_chord_backward_workspace_bytes(B, H, L) &&
                 ((uintptr_t)workspace & 15) == 0,
             MB_ERR_ARG, "chord_backward: workspace too small or unaligned");
  MB_REQUIRE(param_partials != nullptr, MB_ERR_ARG, "chord_backward: null partials");
  if (B == 0 || L == 0) return MB_OK;
  ChordBwdArgs a;
  a.q = q; a.k = k; a.v = v; a.o = out; a.dout = dout;
  a.alpha = alpha; a.beta = beta; a.mu = mu; a.ssmax = ssmax; a.log_n = log_n;
  a.dq = dq; a.dk = dk; a.dv = dv;
  float* ws = (float*)workspace;
  a.lse = ws;
  a.delta = ws + B * H * L;
  a.crow = ws + 2 * B * H * L;
  a.part = param_partials;
  // strides: q, k, v, out, dout, dq, dk, dv (b, h, t each), log_n (b, t)
  for (int i = 0; i < 3; ++i) {
    a.sq[i] = strides[i];
    a.sk[i] = strides[3 + i];
    a.sv[i] = strides[6 + i];
    a.so[i] = strides[9 + i];
    a.sd[i] = strides[12 + i];
    a.sdq[i] = strides[15 + i];
    a.sdk[i] = strides[18 + i];
    a.sdv[i] = strides[21 + i];
  }
  a.sl[0] = strides[24];
  a.sl[1] = strides[25];
  a.B = (int)B; a.H = (int)H; a.Hkv = (int)Hkv; a.L = (int)L; a.S = (int)S; a.q_start = (int)q_start;
  a.scale = scale; a.eps = eps;
  cudaStream_t st = (cudaStream_t)stream;
  if (S == 0) {  // no keys: every gradient is zero (the partials are written by the caller's zeroing)
    return MB_OK;
  }
  auto by_d = [&](auto t) -> int {
    using T = decltype(t);
    switch (D) {
      case 16: return launch_chord_bwd<T, 16>(a, st);
      case 32: return launch_chord_bwd<T, 32>(a, st);
      case 64: return launch_chord_bwd<T, 64>(a, st);
      default: return launch_chord_bwd<T, 128>(a, st);
    }
  };
  if (dtype == MB_F32) return by_d(0.f);
  if (dtype == MB_BF16) return by_d(__nv_bfloat16{});
  MB_REQUIRE(dtype == MB_F16, MB_ERR_UNSUPPORTED, "chord_backward: dtype");
  return by_d(__half{});
}

// ------------------------------------------------------------------ AttnRes backward
// Forward (motif/ops/attn_res.py:550-593): per row (b, t), over sources n < N,
//   r_n = rsqrt(mean_d V_nd^2 + eps), logit_n = r_n sum_d q_d w_d V_nd, a = softmax_n(logit),
//   h = sum_n a_n V_n.
// With dh: da_n = dh.V_n, dlogit_n = a_n (da_n - sum_m a_m da_m), and (using
// sum_d q_d w_d V_nd = logit_n / r_n)
//   dV_nd = a_n dh_d + dlogit_n (r_n w_d q_d - r_n^2 logit_n V_nd / D),
//   dq = w . Z, dw = q . Z with Z_d = sum over rows and n of dlogit_n r_n V_nd.
// One warp per row (grid-stride); Z accumulates per lane, is summed over the CTA's warps and
// written as one partial row per CTA (the host adds the partials in fp64).
namespace mb {
namespace {
constexpr int kArMaxSrc = 16;
struct ArSrc {
  const void* p[kArMaxSrc];
  void* dp[kArMaxSrc];
};

template <typename T, int NV>
__global__ void __launch_bounds__(256) attn_res_bwd_kernel(ArSrc src, int N, int64_t rows, int64_t rs,
                                                           const T* __restrict__ w, const T* __restrict__ q,
                                                           const T* __restrict__ dh, int64_t dhs, float eps,
                                                           float* __restrict__ zpart) {
  constexpr int D = NV * 32;
  extern __shared__ float zs[];  // [8 warps][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float wq[NV], z[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    wq[u] = to_f(w[lane + 32 * u]) * to_f(q[lane + 32 * u]);
    z[u] = 0.f;
  }
  for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < rows; row += (int64_t)gridDim.x * 8) {
    float g[NV];
#pragma unroll
    for (int u = 0; u < NV; ++u) g[u] = to_f(dh[row * dhs + lane + 32 * u]);
    float logit[kArMaxSrc], da[kArMaxSrc], rn[kArMaxSrc], an[kArMaxSrc];
    float mx = -INFINITY;
    for (int n = 0; n < N; ++n) {
      const T* vp = (const T*)src.p[n] + row * rs;
      float ss = 0.f, dot = 0.f, dd = 0.f;
#pragma unroll
      for (int u = 0; u < NV; ++u) {
        const float x = to_f(vp[lane + 32 * u]);
        ss = fmaf(x, x, ss);
        dot = fmaf(wq[u], x, dot);
        dd = fmaf(g[u], x, dd);
      }
      ss = warp_sum(ss);
      dot = warp_sum(dot);
      dd = warp_sum(dd);
      rn[n] = rsqrtf(ss / (float)D + eps);
      logit[n] = rn[n] * dot;
      da[n] = dd;
      mx = fmaxf(mx, logit[n]);
    }
    float den = 0.f, sad = 0.f;
    for (int n = 0; n < N; ++n) {
      an[n] = expf(logit[n] - mx);
      den += an[n];
    }
    for (int n = 0; n < N; ++n) {
      an[n] /= den;
      sad += an[n] * da[n];
    }
    for (int n = 0; n < N; ++n) {
      const float dl = an[n] * (da[n] - sad), r = rn[n];
      const float c2 = r * r * logit[n] / (float)D;
      const T* vp = (const T*)src.p[n] + row * rs;
      T* dp = (T*)src.dp[n] + row * rs;
#pragma unroll
      for (int u = 0; u < NV; ++u) {
        const float x = to_f(vp[lane + 32 * u]);
        dp[lane + 32 * u] = from_f<T>(an[n] * g[u] + dl * (r * wq[u] - c2 * x));
        z[u] = fmaf(dl * r, x, z[u]);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < NV; ++u) zs[warp * D + lane + 32 * u] = z[u];
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += 256) {
    float s = 0.f;
    for (int wi = 0; wi < 8; ++wi) s += zs[wi * D + d];
    zpart[(int64_t)blockIdx.x * D + d] = s;
  }
}
}  // namespace
}  // namespace mb

extern "C" int motif_b200_attn_res_backward(const void* const* sources, void* const* d_sources, int n_src,
                                            int64_t rows, int64_t row_stride, int64_t D, const void* weight,
                                            const void* query, float eps, const void* grad_out,
                                            int64_t grad_stride, float* z_partials, int64_t partial_rows,
                                            int dtype, void* stream) {
  MB_REQUIRE(sources && d_sources && weight && query && grad_out && z_partials, MB_ERR_ARG,
             "attn_res_backward: null pointer");
  MB_REQUIRE(n_src >= 1 && n_src <= kArMaxSrc, MB_ERR_UNSUPPORTED, "attn_res_backward: 1..%d sources", kArMaxSrc);
  MB_REQUIRE(D % 32 == 0 && D >= 32 && D <= 1024, MB_ERR_UNSUPPORTED, "attn_res_backward: D a multiple of 32 <= 1024");
  MB_REQUIRE(rows >= 0 && partial_rows >= 1 && partial_rows <= 65535, MB_ERR_ARG, "attn_res_backward: bad sizes");
  if (rows == 0) return MB_OK;
  ArSrc s;
  for (int i = 0; i < n_src; ++i) {
    MB_REQUIRE(sources[i] && d_sources[i], MB_ERR_ARG, "attn_res_backward: null source");
    s.p[i] = sources[i];
    s.dp[i] = d_sources[i];
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int nv = (int)(D / 32);
  const size_t smem = (size_t)8 * D * 4;
  auto go = [&](auto t, auto nvc) -> int {
    using T = decltype(t);
    constexpr int NV = decltype(nvc)::value;
    auto kern = attn_res_bwd_kernel<T, NV>;
    if (int rc = ensure_smem_attr((const void*)kern, (int)smem)) return rc;
    kern<<<(unsigned)partial_rows, 256, smem, st>>>(s, n_src, rows, row_stride, (const T*)weight, (const T*)query,
                                                   (const T*)grad_out, grad_stride, eps, z_partials);
    return check_launch("attn_res_backward");
  };
  auto by_nv = [&](auto t) -> int {
    switch (nv) {
      case 1: return go(t, std::integral_constant<int, 1>{});
      case 2: return go(t, std::integral_constant<int, 2>{});
      case 4: return go(t, std::integral_constant<int, 4>{});
      case 8: return go(t, std::integral_constant<int, 8>{});
      case 16: return go(t, std::integral_constant<int, 16>{});
      case 24: return go(t, std::integral_constant<int, 24>{});
      case 32: return go(t, std::integral_constant<int, 32>{});
      default: return set_error(MB_ERR_UNSUPPORTED, "attn_res_backward: D = %lld", (long long)D);
    }
  };
  if (dtype == MB_F32) return by_nv(0.f);
  if (dtype == MB_BF16) return by_nv(__nv_bfloat16{});
  MB_REQUIRE(dtype == MB_F16, MB_ERR_UNSUPPORTED, "attn_res_backward: dtype");
  return by_nv(__half{});
}

// ------------------------------------------------------------------ gated delta rule backward
// Forward per (b, h), token by token (motif/ops/gated_deltanet.py:26-59):
//   S' = S e^{g_t},  u = k_t^T S' (the value S' recalls),  d = beta_t (v_t - u),
//   S = S' + k_t d^T,  o_t = q_t^T S.
// Backward from dS (the gradient of the state after step t) and do_t, in reverse order:
//   dS += q_t do_t^T;  dq_t = S do_t;  dd = dS^T k_t;  dv_t = beta_t dd;
//   dbeta_t = dd.(v_t - u);  du = -beta_t dd;  dk_t = dS d + S' du;  dS' = dS + k_t du^T;
//   dg_t = <dS', S'>;  dS <- dS' e^{g_t}.
// One CTA per (b, h) holds S / dS in registers (thread t: column t % DV, DK DV / 256 rows).
// The states before every step are rebuilt from checkpoints taken every kSeg steps: a first
// pass stores S at each segment start, then each segment is recomputed (its states into the
// workspace) and walked backwards.  Sums over a row go through a shared-memory transpose,
// sums over a column through per-row-group partials.  fp32 throughout.
namespace mb {
namespace {
constexpr int kSeg = 64;

template <int DK, int DV>
struct GdnBwdSmem {
  static constexpr int NG = 256 / DV;       // row groups
  static constexpr int RPT = DK / NG;       // rows per thread
  static constexpr int PS = DV + 1;         // transpose row stride
  static constexpr size_t vec = (2 * DK + 2 * DV) * 4;  // q, k, v, do of the step
  static constexpr size_t cred = (size_t)NG * DV * 4;
  static constexpr size_t tr = (size_t)2 * DK * PS * 4;  // two values per (row, column)
  static constexpr size_t bytes = vec + cred + tr + 64 * 4;
};

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1) gdn_bwd_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                        const float* __restrict__ v, const float* __restrict__ beta,
                                                        const float* __restrict__ g, const float* __restrict__ s0,
                                                        const float* __restrict__ dout,
                                                        const float* __restrict__ ds_final, float* __restrict__ dq,
                                                        float* __restrict__ dk, float* __restrict__ dv,
                                                        float* __restrict__ dbeta, float* __restrict__ dg,
                                                        float* __restrict__ ds0, float* __restrict__ ws, int L) {
  using Sm = GdnBwdSmem<DK, DV>;
  constexpr int NG = Sm::NG, RPT = Sm::RPT, PS = Sm::PS;
  extern __shared__ float smf[];
  float* sq = smf;
  float* sk = sq + DK;
  float* sv = sk + DK;
  float* sdo = sv + DV;
  float* cred = sdo + DV;            // [NG][DV]
  float* tr0 = cred + NG * DV;       // [DK][PS]
  float* tr1 = tr0 + DK * PS;
  float* red = tr1 + DK * PS;        // [64] scalar reductions
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = tid % DV, rg = tid / DV, r0 = rg * RPT;
  const int64_t bh = blockIdx.x;
  const int nseg = (L + kSeg - 1) / kSeg;
  float* ck = ws + (size_t)bh * (nseg + kSeg) * DK * DV;  // [nseg] checkpoints
  float* stp = ck + (size_t)nseg * DK * DV;                // [kSeg] states before each step
  const float* qb = q + bh * (int64_t)L * DK;
  const float* kb = k + bh * (int64_t)L * DK;
  const float* vb = v + bh * (int64_t)L * DV;
  const float* dob = dout + bh * (int64_t)L * DV;
  const float* bb = beta + bh * (int64_t)L;
  const float* gb = g + bh * (int64_t)L;

  auto block_sum = [&](float x) {  // every thread gets the sum
    x = warp_sum(x);
    __syncthreads();
    if (lane == 0) red[warp] = x;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w];
    return s;
  };
  // the value S' recalls for column c (all threads of the column get it)
  auto recall = [&](const float (&Sp)[RPT]) {
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < RPT; ++i) part = fmaf(sk[r0 + i], Sp[i], part);
    __syncthreads();
    cred[rg * DV + c] = part;
    __syncthreads();
    float u = 0.f;
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) u += cred[gi * DV + c];
    return u;
  };
  auto load_step = [&](int t, bool with_do) {
    __syncthreads();
    for (int e = tid; e < DK; e += 256) {
      sq[e] = qb[(int64_t)t * DK + e];
      sk[e] = kb[(int64_t)t * DK + e];
    }
    for (int e = tid; e < DV; e += 256) {
      sv[e] = vb[(int64_t)t * DV + e];
      if (with_do) sdo[e] = dob[(int64_t)t * DV + e];
    }
    __syncthreads();
  };
  // one forward step on S (in place)
  auto step = [&](float (&S)[RPT], int t) {
    const float eg = expf(gb[t]), bt = bb[t];
    float Sp[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) Sp[i] = S[i] * eg;
    const float d = bt * (sv[c] - recall(Sp));
#pragma unroll
    for (int i = 0; i < RPT; ++i) S[i] = fmaf(sk[r0 + i], d, Sp[i]);
  };

  float S[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) S[i] = s0 ? s0[bh * DK * DV + (int64_t)(r0 + i) * DV + c] : 0.f;
  // pass 1: checkpoints at the segment starts
  for (int t = 0; t < L; ++t) {
    if (t % kSeg == 0) {
      float* dst = ck + (size_t)(t / kSeg) * DK * DV;
#pragma unroll
      for (int i = 0; i < RPT; ++i) dst[(r0 + i) * DV + c] = S[i];
    }
    load_step(t, false);
    step(S, t);
  }
  float dS[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) dS[i] = ds_final ? ds_final[bh * DK * DV + (int64_t)(r0 + i) * DV + c] : 0.f;
  for (int sg = nseg - 1; sg >= 0; --sg) {
    const int t0 = sg * kSeg, t1 = min(L, t0 + kSeg);
    // pass 2: the segment's states before each step
    const float* src = ck + (size_t)sg * DK * DV;
#pragma unroll
    for (int i = 0; i < RPT; ++i) S[i] = src[(r0 + i) * DV + c];
    for (int t = t0; t < t1; ++t) {
      float* dst = stp + (size_t)(t - t0) * DK * DV;
#pragma unroll
      for (int i = 0; i < RPT; ++i) dst[(r0 + i) * DV + c] = S[i];
      if (t + 1 < t1) {
        load_step(t, false);
        step(S, t);
      }
    }
    // pass 3: backwards through the segment
    for (int t = t1 - 1; t >= t0; --t) {
      load_step(t, true);
      const float* prev = stp + (size_t)(t - t0) * DK * DV;
      const float eg = expf(gb[t]), bt = bb[t];
      float Sp[RPT], St[RPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i) Sp[i] = prev[(r0 + i) * DV + c] * eg;
      const float u = recall(Sp);
      const float d = bt * (sv[c] - u);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        St[i] = fmaf(sk[r0 + i], d, Sp[i]);
        dS[i] = fmaf(sq[r0 + i], sdo[c], dS[i]);
      }
      // dd = dS^T k (column sum)
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < RPT; ++i) part = fmaf(sk[r0 + i], dS[i], part);
      __syncthreads();
      cred[rg * DV + c] = part;
      __syncthreads();
      float dd = 0.f;
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) dd += cred[gi * DV + c];
      const float du = -bt * dd;
      // row sums: dq = S do, dk = dS d + S' du
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        tr0[(r0 + i) * PS + c] = St[i] * sdo[c];
        tr1[(r0 + i) * PS + c] = fmaf(dS[i], d, Sp[i] * du);
      }
      float dgp = 0.f;
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        dS[i] = fmaf(sk[r0 + i], du, dS[i]);  // dS'
        dgp = fmaf(dS[i], Sp[i], dgp);
        dS[i] *= eg;
      }
      __syncthreads();
      // 2 DK row sums over DV columns: thread pairs per (value, row), halves of the columns
      for (int e = tid; e < 2 * DK * 2; e += 256) {
        const int half = e & 1, rv = e >> 1, row = rv % DK, which = rv / DK;
        const float* tp = (which ? tr1 : tr0) + row * PS;
        float s = 0.f;
        for (int cc = half * (DV / 2); cc < (half + 1) * (DV / 2); ++cc) s += tp[cc];
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (half == 0) (which ? dk : dq)[(bh * L + t) * DK + row] = s;
      }
      if (rg == 0) dv[(bh * L + t) * DV + c] = bt * dd;
      const float dbp = block_sum(rg == 0 ? dd * (sv[c] - u) : 0.f);
      const float dgt = block_sum(dgp);
      if (tid == 0) {
        dbeta[bh * L + t] = dbp;
        dg[bh * L + t] = dgt;
      }
    }
  }
  if (ds0) {
#pragma unroll
    for (int i = 0; i < RPT; ++i) ds0[bh * DK * DV + (int64_t)(r0 + i) * DV + c] = dS[i];
  }
}
}  // namespace
}  // namespace mb

extern "C" int64_t motif_b200_gdn_backward_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv) {
  const int64_t nseg = (L + mb::kSeg - 1) / mb::kSeg;
  return B * H * (nseg + mb::kSeg) * Dk * Dv * 4;
}

extern "C" int motif_b200_gdn_backward(const float* q, const float* k, const float* v, const float* beta,
                                       const float* g, const float* state_in, const float* grad_out,
                                       const float* grad_state, float* dq, float* dk, float* dv, float* dbeta,
                                       float* dg, float* d_state_in, int64_t B, int64_t H, int64_t L, int64_t Dk,
                                       int64_t Dv, void* workspace, int64_t workspace_bytes, void* stream) {
  MB_REQUIRE(q && k && v && beta && g && grad_out && dq && dk && dv && dbeta && dg, MB_ERR_ARG,
             "gdn_backward: null pointer");
  MB_REQUIRE(B >= 0 && H > 0 && L >= 0 && B * H < (1LL << 31) && L < (1LL << 30), MB_ERR_SHAPE,
             "gdn_backward: bad shape");
  MB_REQUIRE(workspace != nullptr && workspace_bytes >= motif_b200_gdn_backward_workspace_bytes(B, H, L, Dk, Dv),
             MB_ERR_ARG, "gdn_backward: workspace too small");
  if (B == 0) return MB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  auto go = [&](auto dkc, auto dvc) -> int {
    constexpr int DK = decltype(dkc)::value, DV = decltype(dvc)::value;
    auto kern = gdn_bwd_kernel<DK, DV>;
    if (int rc = ensure_smem_attr((const void*)kern, (int)GdnBwdSmem<DK, DV>::bytes)) return rc;
    kern<<<(unsigned)(B * H), 256, GdnBwdSmem<DK, DV>::bytes, st>>>(q, k, v, beta, g, state_in, grad_out, grad_state,
                                                                    dq, dk, dv, dbeta, dg, d_state_in,
                                                                    (float*)workspace, (int)L);
    return check_launch("gdn_backward");
  };
  using I16 = std::integral_constant<int, 16>;
  using I32 = std::integral_constant<int, 32>;
  using I64 = std::integral_constant<int, 64>;
  using I128 = std::integral_constant<int, 128>;
  if (L == 0) return MB_OK;
  if (Dk == 64 && Dv == 128) return go(I64{}, I128{});
  if (Dk == 64 && Dv == 64) return go(I64{}, I64{});
  if (Dk == 32 && Dv == 64) return go(I32{}, I64{});
  if (Dk == 32 && Dv == 32) return go(I32{}, I32{});
  if (Dk == 16 && Dv == 32) return go(I16{}, I32{});
  if (Dk == 128 && Dv == 128) return go(I128{}, I128{});
  return set_error(MB_ERR_UNSUPPORTED, "gdn_backward: (Dk, Dv) = (%lld, %lld)", (long long)Dk, (long long)Dv);
}
