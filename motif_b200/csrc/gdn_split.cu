// Chunked gated delta rule for 16-bit inputs as two kernels, so that only the part of the
// chunk computation that depends on the recurrent state S runs sequentially.
//
// motif/ops/gated_deltanet.py:137-177 (_PrepareChunksFunction) and :287-321 split the chunk
// math the same way: everything built from one chunk's q, k, v, beta, g alone (the UT
// transform) is independent of the state; only X = U - W S, the output and the state update
// walk the chunks in order.
//
//   gdn_wy_kernel   grid (chunks, B*H), fully parallel.  Per chunk: gamma = cumsum(g),
//                   A = -(beta_i k_i.k_j e^{gamma_i - gamma_j}) (j < i), the 16x16 diagonal
//                   inverses of (I - A) and the blocked forward substitution
//                   [W | U] = (I - A)^-1 [k beta e^gamma | v beta]; Aq = (q k^T)_ij
//                   e^{gamma_i - gamma_j} (j <= i); q e^gamma and k e^{gamma_L - gamma}.  The
//                   chunk's record is written as the exact shared-memory image the scan uses
//                   (padded rows), so the scan fetches it with one bulk copy.
//   gdn_rec_kernel  grid B*H, one CTA per (b, h) walking its chunks with S resident in fp32
//                   registers; the record of chunk n+2 streams in (cp.async.bulk + mbarrier)
//                   while chunk n computes X = U - W S, o = (q e^gamma) S + Aq X and
//                   S = e^{gamma_L} S + (k e^{gamma_L - gamma})^T X.
//   gdn_gate_norm   (gated calls) o <- rmsnorm(o) * w * silu(gate) per (token, head) row,
//                   in place: the GatedRMSNorm of gdn_attn.py:197-209, fully parallel.
//
// Products are 16-bit m16n8k16 tensor-core MMAs with fp32 accumulation, the same operand
// roundings as the fused kernel (gdn_fast.cu), which stays the path without a workspace.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "gdn_mma.cuh"

namespace mb {
// Two adjacent fp32 values from shared memory (8-byte aligned).
__device__ __forceinline__ float2 ld2f(const float* p) { return *reinterpret_cast<const float2*>(p); }
namespace {
using namespace gdnk;

// Per-chunk workspace record = the scan's shared-memory image of one chunk (rows padded by 8
// elements so that ldmatrix rows fall on distinct banks).  A shared part every value-column
// slice of the scan reads, then one U plane per slice of SW value columns:
//   Qs [C][QS] = q e^gamma | Kd [C][QS] = k e^{gamma_L - gamma} | W [C][QS] | Aq [C][AS] (T) |
//   e^{gamma_L} (fp32, padded to 16 bytes) | U_0 [C][US] | U_1 [C][US] | ...
template <typename T, int DK, int DV, int SWP = 64>
struct WsRec {
  static constexpr int SW = DV < SWP ? DV : SWP;  // value columns per scan slice
  static constexpr int NSL = DV / SW;
  static_assert(DV % SW == 0, "value columns split into equal slices");
  static constexpr int QS = DK + 8, AS = C + 8, US = SW + 8;
  static constexpr size_t off_qs = 0;
  static constexpr size_t off_kd = off_qs + (size_t)C * QS * sizeof(T);
  static constexpr size_t off_w = off_kd + (size_t)C * QS * sizeof(T);
  static constexpr size_t off_aq = off_w + (size_t)C * QS * sizeof(T);
  static constexpr size_t off_el = off_aq + (size_t)C * AS * sizeof(T);
  static constexpr size_t shared_bytes = off_el + 16;
  static constexpr size_t u_bytes = (size_t)C * US * sizeof(T);
  static constexpr size_t bytes = shared_bytes + NSL * u_bytes;
  static_assert(shared_bytes % 16 == 0 && u_bytes % 16 == 0, "records stay 16-byte aligned");
};

template <typename T, int DK, int DV>
struct WyLayout {
  static constexpr int QS = DK + 8, VS = DV + 8, AS = C + 8, XS = DK + DV + 8, TS = 16 + 8;
  static constexpr size_t off_q = 0;
  static constexpr size_t off_k = off_q + (size_t)C * QS * sizeof(T);
  static constexpr size_t off_v = off_k + (size_t)C * QS * sizeof(T);
  static constexpr size_t off_a = off_v + (size_t)C * VS * sizeof(T);
  static constexpr size_t off_aq = off_a + (size_t)C * AS * sizeof(T);
  static constexpr size_t off_x = off_aq + (size_t)C * AS * sizeof(T);
  static constexpr size_t off_td = off_x + (size_t)C * XS * sizeof(T);
  static constexpr size_t off_ad = off_td + 4ull * 16 * TS * sizeof(T);
  static constexpr size_t off_vec = off_ad + 4ull * 16 * 17 * 4;
  static constexpr size_t bytes = off_vec + 4ull * C * 4;
};

// Inputs of the fused preparation (PREP = true): the raw projection rows [q | k | v | a | b | ...]
// (row stride ps, token-major), the conv weights / carried conv state and the decay parameters
// (gdn_attn.py:116-136, :183-197), with the roundings of motif_b200_gdn_prep.
template <typename T>
struct PrepIn {
  const T* proj = nullptr;
  int64_t ps = 0;
  const T* conv_w = nullptr;   // [C][4], C = H (2 Dk + Dv): q | k | v channels
  const T* A_log = nullptr;    // [H]
  const T* dt_bias = nullptr;  // [H]
  const T* conv_in = nullptr;  // [B][3][C] raw inputs before token 0, or nullptr (zeros)
  T* conv_out = nullptr;       // [B][3][C] raw inputs at L-3 .. L-1, or nullptr
};

// Warp 0: gamma = inclusive cumsum of the chunk's g (two values per lane), e^gamma, beta.
__device__ __forceinline__ void wy_gamma(int lane, float x0, float x1, float b0, float b1, float* sGam, float* sEg,
                                         float* sBeta) {
#pragma unroll
  for (int o2 = 1; o2 < 32; o2 <<= 1) {
    const float y0 = __shfl_up_sync(0xffffffffu, x0, o2);
    const float y1 = __shfl_up_sync(0xffffffffu, x1, o2);
    if (lane >= o2) {
      x0 += y0;
      x1 += y1;
    }
  }
  x1 += __shfl_sync(0xffffffffu, x0, 31);
  sGam[lane] = x0;
  sGam[lane + 32] = x1;
  sEg[lane] = expf(x0);
  sEg[lane + 32] = expf(x1);
  __syncwarp();
  sBeta[lane] = b0;
  sBeta[lane + 32] = b1;
}

template <typename T, int DK, int DV, bool PREP, int SWP>
__global__ void __launch_bounds__(NT, 2) gdn_wy_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                    const T* __restrict__ v, const float* __restrict__ beta,
                                                    const float* __restrict__ g, int H, int L, Strides18 sv,
                                                    unsigned char* __restrict__ ws, PrepIn<T> pin) {
  using Lay = WyLayout<T, DK, DV>;
  using Rec = WsRec<T, DK, DV, SWP>;
  constexpr int QS = Lay::QS, VS = Lay::VS, AS = Lay::AS, XS = Lay::XS, TS = Lay::TS;
  constexpr int NTILE = (DK + DV) / 8;
  constexpr int SOLVE_T = (NTILE + NW - 1) / NW;
  extern __shared__ __align__(16) unsigned char smem[];
  T* cQ = reinterpret_cast<T*>(smem + Lay::off_q);
  T* cK = reinterpret_cast<T*>(smem + Lay::off_k);
  T* cV = reinterpret_cast<T*>(smem + Lay::off_v);
  T* sA = reinterpret_cast<T*>(smem + Lay::off_a);
  T* sAq = reinterpret_cast<T*>(smem + Lay::off_aq);
  T* sX = reinterpret_cast<T*>(smem + Lay::off_x);
  T* sTd = reinterpret_cast<T*>(smem + Lay::off_td);
  float* sAd = reinterpret_cast<float*>(smem + Lay::off_ad);
  float* sGam = reinterpret_cast<float*>(smem + Lay::off_vec);
  float* sEg = sGam + C;
  float* sBeta = sEg + C;

  const int64_t* st = sv.s;
  const int n = blockIdx.x, bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const T* qg = PREP ? nullptr : q + b * st[0] + h * st[1];
  const T* kg = PREP ? nullptr : k + b * st[3] + h * st[4];
  const T* vg = PREP ? nullptr : v + b * st[6] + h * st[7];
  const float* bg = PREP ? nullptr : beta + b * st[12] + h * st[13];
  const float* gg = PREP ? nullptr : g + b * st[15] + h * st[16];

  if constexpr (!PREP) {
    {  // q, k, v rows of the chunk (zeros past L)
      constexpr int QV = DK * (int)sizeof(T) / 16, VV = DV * (int)sizeof(T) / 16;
      constexpr int E = 16 / sizeof(T);
      for (int i = tid; i < C * (2 * QV + VV); i += NT) {
        const int r = i / (2 * QV + VV), c = i % (2 * QV + VV);
        const int l = n * C + r;
        const bool ok = l < L;
        const int64_t lc = ok ? l : 0;
        if (c < QV)
          cp_async16(cQ + r * QS + c * E, qg + lc * st[2] + c * E, ok);
        else if (c < 2 * QV)
          cp_async16(cK + r * QS + (c - QV) * E, kg + lc * st[5] + (c - QV) * E, ok);
        else
          cp_async16(cV + r * VS + (c - 2 * QV) * E, vg + lc * st[8] + (c - 2 * QV) * E, ok);
      }
      cp_async_commit();
    }
    if (warp == 0) {  // gamma = inclusive cumsum(g), e^gamma, beta (padded rows: g = beta = 0)
      float x0, x1, b0, b1;
      {
        const int l0 = n * C + lane, l1 = l0 + 32;
        x0 = l0 < L ? gg[(int64_t)l0 * st[17]] : 0.f;
        x1 = l1 < L ? gg[(int64_t)l1 * st[17]] : 0.f;
        b0 = l0 < L ? bg[(int64_t)l0 * st[14]] : 0.f;
        b1 = l1 < L ? bg[(int64_t)l1 * st[14]] : 0.f;
      }
      wy_gamma(lane, x0, x1, b0, b1, sGam, sEg, sBeta);
    }
  } else {
    // causal depthwise conv (4 taps, carried state) + SiLU, L2-normalised q * Dk^-0.5 and k,
    // beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias): motif_b200_gdn_prep's math.
    // Thread = (8-channel group of this head's q | k | v = lane, 8-row run = warp); the q / k
    // norms reduce over the 8 lanes of a head's group.
    constexpr int NG = (2 * DK + DV) / 8;  // channel groups of one head
    static_assert(NG == 32 && C / 8 == NW, "one group per lane, one 8-row run per warp");
    const int Ct = H * (2 * DK + DV);
    const int grp = lane, run = warp;
    const int kind = grp < DK / 8 ? 0 : (grp < 2 * DK / 8 ? 1 : 2);
    const int cl = grp * 8;  // local channel
    const int cg = kind == 0 ? h * DK + cl
                             : (kind == 1 ? H * DK + h * DK + (cl - DK) : 2 * H * DK + h * DV + (cl - 2 * DK));
    const T* P = pin.proj + (int64_t)b * L * pin.ps;
    const int t0 = n * C + run * 8;
    // this chunk's a / b scalars (beta and g below), requested first so that their latency
    // overlaps the row loads instead of following them
    T a_raw = from_f<T>(0.f), b_raw = from_f<T>(0.f);
    if (tid < C && n * C + tid < L) {
      const T* row = P + (int64_t)(n * C + tid) * pin.ps;
      a_raw = row[Ct + h];
      b_raw = row[Ct + H + h];
    }
    uint4 raw[11];
#pragma unroll
    for (int j = 0; j < 11; ++j) {
      const int tau = t0 - 3 + j;
      raw[j] = make_uint4(0, 0, 0, 0);
      if (tau >= 0 && tau < L)
        raw[j] = *reinterpret_cast<const uint4*>(P + (int64_t)tau * pin.ps + cg);
      else if (tau < 0 && pin.conv_in)
        raw[j] = *reinterpret_cast<const uint4*>(pin.conv_in + ((int64_t)b * 3 + (3 + tau)) * Ct + cg);
    }
    float w[8][4];
    {
      const uint4* wp = reinterpret_cast<const uint4*>(pin.conv_w + (int64_t)cg * 4);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4 r = wp[u];
        const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[2 * u + i / 4][i % 4] = to_f(e[i]);
      }
    }
    const float qscale = rsqrtf((float)DK);
    // Sliding window of the converted inputs: xw[p][tap] holds channel pair p of row r + tap,
    // so each raw element is converted to fp32 once, not once per tap.
    float2 xw[4][4];
#pragma unroll
    for (int tap = 0; tap < 3; ++tap)
#pragma unroll
      for (int p = 0; p < 4; ++p)
        xw[p][tap + 1] = make_float2(to_f(reinterpret_cast<const T*>(&raw[tap])[2 * p]),
                                     to_f(reinterpret_cast<const T*>(&raw[tap])[2 * p + 1]));
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int row = run * 8 + r;
      const bool ok = t0 + r < L;
      float y[8];
      float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 8; i += 2) {  // channel pairs: packed fp32 math and roundings
        const int p = i / 2;
        xw[p][0] = xw[p][1];
        xw[p][1] = xw[p][2];
        xw[p][2] = xw[p][3];
        xw[p][3] = make_float2(to_f(reinterpret_cast<const T*>(&raw[r + 3])[i]),
                               to_f(reinterpret_cast<const T*>(&raw[r + 3])[i + 1]));
        const float2* xv = xw[p];
        // conv4f's order: ((w0 x0 + w1 x1) + w2 x2) + w3 x3 as one multiply and three fmas
        float2 a = fmul2(make_float2(w[i][0], w[i + 1][0]), xv[0]);
        a = ffma2(make_float2(w[i][1], w[i + 1][1]), xv[1], a);
        a = ffma2(make_float2(w[i][2], w[i + 1][2]), xv[2], a);
        a = ffma2(make_float2(w[i][3], w[i + 1][3]), xv[3], a);
        const float2 sv = silu2_(round2<T>(a.x, a.y));
        const float2 yy = round2<T>(sv.x, sv.y);
        y[i] = yy.x;
        y[i + 1] = yy.y;
        ss2 = ffma2(yy, yy, ss2);
      }
      float ss = ss2.x + ss2.y;
#pragma unroll
      for (int o2 = 1; o2 < 8; o2 <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o2);
      const float sc = (kind == 2 ? 1.f : l2_scale(ss, kind == 0 ? qscale : 1.f)) * (ok ? 1.f : 0.f);
      uint32_t pkw[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const float2 ys = fmul2(make_float2(y[i], y[i + 1]), make_float2(sc, sc));
        pkw[i / 2] = pack2<T>(ys.x, ys.y);
      }
      const uint4 pk = make_uint4(pkw[0], pkw[1], pkw[2], pkw[3]);
      T* dst = kind == 0 ? cQ + row * QS + cl : (kind == 1 ? cK + row * QS + (cl - DK) : cV + row * VS + (cl - 2 * DK));
      *reinterpret_cast<uint4*>(dst) = pk;
    }
    // the run holding L-1 writes the raw inputs at L-3 .. L-1 as the carried conv state
    const int last = L - 1 - t0;
    if (pin.conv_out && last >= 0 && last < 8) {
#pragma unroll
      for (int j = 0; j < 11; ++j) {
        // raw[j] holds token t0 - 3 + j = L - 3 + slot; the window rows before the run (j < 3)
        // matter when the last run holds fewer than three tokens
        const int slot = j - last - 1;
        if (slot >= 0 && slot < 3)
          *reinterpret_cast<uint4*>(pin.conv_out + ((int64_t)b * 3 + slot) * Ct + cg) = raw[j];
      }
    }
    float* sGin = sGam + 3 * C;  // raw g values before the cumsum
    if (tid < C) {
      const int l = n * C + tid;
      float bt = 0.f, gt = 0.f;
      if (l < L) {
        const float Aexp = -to_f(from_f<T>(expf(to_f(pin.A_log[h]))));
        const float dtb = to_f(pin.dt_bias[h]);
        bt = to_f(from_f<T>(sigmoidf_(to_f(b_raw))));
        gt = to_f(from_f<T>(Aexp * to_f(from_f<T>(softplusf_(to_f(from_f<T>(to_f(a_raw) + dtb)))))));
      }
      sBeta[tid] = bt;
      sGin[tid] = gt;
    }
    __syncthreads();
    if (warp == 0) wy_gamma(lane, sGin[lane], sGin[lane + 32], sBeta[lane], sBeta[lane + 32], sGam, sEg, sBeta);
  }
  cp_async_wait<0>();
  __syncthreads();

  // KK -> A (+ diagonal inverses) on warps 0-3, QK -> Aq on warps 4-7
  {
    const int m0 = (warp & 3) * 16;
    const T* left = warp < 4 ? cK : cQ;
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < DK; k0 += 16) {
      uint32_t a[4];
      lda(a, left, QS, m0, k0);
#pragma unroll
      for (int n0 = 0; n0 < 64; n0 += 16) {
        uint32_t bb[4];
        ldb_n(bb, cK, QS, k0, n0);
        mma_16816<T>(acc[n0 / 8], a, &bb[0]);
        mma_16816<T>(acc[n0 / 8 + 1], a, &bb[2]);
      }
    }
    const int i0 = m0 + gq, i1 = i0 + 8;
    const float gi0 = sGam[i0], gi1 = sGam[i1];
    if (warp < 4) {
      const float b0 = -sBeta[i0], b1 = -sBeta[i1];
      float* ad = sAd + warp * 16 * 17;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        // -beta_i k_i.k_j e^(gamma_i - gamma_j) below the diagonal, in packed fp32 pairs
        // (e^x as 2^(x log2 e) on the MUFU)
        const int j = nt * 8 + 2 * tq;
        const float2 gj = ld2f(&sGam[j]);
        const float2 e0 = fmul2(fadd2(make_float2(gi0, gi0), make_float2(-gj.x, -gj.y)),
                                make_float2(-kNegLog2e, -kNegLog2e));
        const float2 e1 = fmul2(fadd2(make_float2(gi1, gi1), make_float2(-gj.x, -gj.y)),
                                make_float2(-kNegLog2e, -kNegLog2e));
        const float2 v0 = fmul2(fmul2(make_float2(b0, b0), make_float2(acc[nt][0], acc[nt][1])),
                                make_float2(ex2f_(e0.x), ex2f_(e0.y)));
        const float2 v1 = fmul2(fmul2(make_float2(b1, b1), make_float2(acc[nt][2], acc[nt][3])),
                                make_float2(ex2f_(e1.x), ex2f_(e1.y)));
        const float a00 = j < i0 ? v0.x : 0.f;
        const float a01 = j + 1 < i0 ? v0.y : 0.f;
        const float a10 = j < i1 ? v1.x : 0.f;
        const float a11 = j + 1 < i1 ? v1.y : 0.f;
        st2(&sA[i0 * AS + j], a00, a01);
        st2(&sA[i1 * AS + j], a10, a11);
        if ((nt >> 1) == warp) {  // this warp's diagonal block, kept in fp32
          const int jj = j - m0;
          ad[gq * 17 + jj] = a00;
          ad[gq * 17 + jj + 1] = a01;
          ad[(gq + 8) * 17 + jj] = a10;
          ad[(gq + 8) * 17 + jj + 1] = a11;
        }
      }
      __syncwarp();
      // T_ww = (I - A_ww)^-1: lane c < 16 owns column c; rows by forward substitution
      if (lane < 16) {
        float col[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          float s = (r == lane) ? 1.f : 0.f;
#pragma unroll
          for (int j = 0; j < r; ++j) s = fmaf(ad[r * 17 + j], col[j], s);
          col[r] = s;
        }
        T* td = sTd + warp * 16 * TS;
#pragma unroll
        for (int r = 0; r < 16; ++r) td[r * TS + lane] = from_f<T>(col[r]);
      }
    } else {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {  // q_i.k_j e^(gamma_i - gamma_j) on and below the diagonal
        const int j = nt * 8 + 2 * tq;
        const float2 gj = ld2f(&sGam[j]);
        const float2 e0 = fmul2(fadd2(make_float2(gi0, gi0), make_float2(-gj.x, -gj.y)),
                                make_float2(-kNegLog2e, -kNegLog2e));
        const float2 e1 = fmul2(fadd2(make_float2(gi1, gi1), make_float2(-gj.x, -gj.y)),
                                make_float2(-kNegLog2e, -kNegLog2e));
        const float2 v0 = fmul2(make_float2(acc[nt][0], acc[nt][1]), make_float2(ex2f_(e0.x), ex2f_(e0.y)));
        const float2 v1 = fmul2(make_float2(acc[nt][2], acc[nt][3]), make_float2(ex2f_(e1.x), ex2f_(e1.y)));
        st2(&sAq[i0 * AS + j], j <= i0 ? v0.x : 0.f, j + 1 <= i0 ? v0.y : 0.f);
        st2(&sAq[i1 * AS + j], j <= i1 ? v1.x : 0.f, j + 1 <= i1 ? v1.y : 0.f);
      }
    }
  }
  __syncthreads();

  // blocked forward substitution, warp-local in its column tiles: the warp's SOLVE_T tiles
  // advance together, sharing each A / T fragment and giving the MMA chains independent work
#pragma unroll
  for (int bi = 0; bi < 4; ++bi) {
    const int r0 = bi * 16;
    const int ra = r0 + gq, rb = ra + 8;
    float acc[SOLVE_T][4];
#pragma unroll
    for (int ti = 0; ti < SOLVE_T; ++ti) {
      const int tile = warp + NW * ti;
      if (tile >= NTILE) break;
      const int c = tile * 8 + 2 * tq;
      if (c < DK) {
        const float sa = sBeta[ra] * sEg[ra], sb = sBeta[rb] * sEg[rb];
        const float2 xa = ld2(&cK[ra * QS + c]), xb = ld2(&cK[rb * QS + c]);
        acc[ti][0] = xa.x * sa; acc[ti][1] = xa.y * sa; acc[ti][2] = xb.x * sb; acc[ti][3] = xb.y * sb;
      } else {
        const float sa = sBeta[ra], sb = sBeta[rb];
        const float2 xa = ld2(&cV[ra * VS + c - DK]), xb = ld2(&cV[rb * VS + c - DK]);
        acc[ti][0] = xa.x * sa; acc[ti][1] = xa.y * sa; acc[ti][2] = xb.x * sb; acc[ti][3] = xb.y * sb;
      }
    }
    for (int bj = 0; bj < bi; ++bj) {  // + A_ij X_j
      uint32_t a[4];
      lda(a, sA, AS, r0, bj * 16);
#pragma unroll
      for (int ti = 0; ti < SOLVE_T; ++ti) {
        const int tile = warp + NW * ti;
        if (tile >= NTILE) break;
        uint32_t bb[2];
        ldb_t1(bb, sX, XS, bj * 16, tile * 8);
        mma_16816<T>(acc[ti], a, bb);
      }
    }
#pragma unroll
    for (int ti = 0; ti < SOLVE_T; ++ti) {
      const int tile = warp + NW * ti;
      if (tile >= NTILE) break;
      const int c = tile * 8 + 2 * tq;
      st2(&sX[ra * XS + c], acc[ti][0], acc[ti][1]);
      st2(&sX[rb * XS + c], acc[ti][2], acc[ti][3]);
    }
    __syncwarp();
    {
      uint32_t a[4];
      lda(a, sTd + bi * 16 * TS, TS, 0, 0);
      float x[SOLVE_T][4];
#pragma unroll
      for (int ti = 0; ti < SOLVE_T; ++ti) {
        const int tile = warp + NW * ti;
        if (tile >= NTILE) break;
        uint32_t bb[2];
        ldb_t1(bb, sX, XS, r0, tile * 8);
        x[ti][0] = x[ti][1] = x[ti][2] = x[ti][3] = 0.f;
        mma_16816<T>(x[ti], a, bb);
      }
      __syncwarp();
#pragma unroll
      for (int ti = 0; ti < SOLVE_T; ++ti) {
        const int tile = warp + NW * ti;
        if (tile >= NTILE) break;
        const int c = tile * 8 + 2 * tq;
        st2(&sX[ra * XS + c], x[ti][0], x[ti][1]);
        st2(&sX[rb * XS + c], x[ti][2], x[ti][3]);
      }
    }
    __syncwarp();
  }
  __syncthreads();

  // the record: padded images of q e^gamma, k e^{gamma_L - gamma}, [W | U], Aq, e^{gamma_L}
  unsigned char* rec = ws + ((size_t)bh * gridDim.x + n) * Rec::bytes;
  {
    constexpr int E = 16 / sizeof(T);
    T* rqs = reinterpret_cast<T*>(rec + Rec::off_qs);
    T* rkd = reinterpret_cast<T*>(rec + Rec::off_kd);
    // Every 16-byte vector of the record is written, the row pads included (as zeros), so that
    // no L2 sector is left partly written (a partial sector is read back from DRAM to merge).
    // One loop per plane over (row, vector) with a power-of-two vector count per row keeps the
    // index arithmetic to shifts and masks.
    constexpr int QV = DK / E;  // 16-byte vectors per q / k / W row
    constexpr int UV = Rec::SW / E, AV = C / E;
    static_assert((QV & (QV - 1)) == 0 && (UV & (UV - 1)) == 0 && (AV & (AV - 1)) == 0, "power-of-two rows");
    const float gl = sGam[C - 1];
    for (int i = tid; i < C * QV; i += NT) {  // q e^gamma, k e^{gamma_L - gamma}
      const int r = i / QV, c = (i % QV) * E;
      const float eq = sEg[r], ek = __expf(gl - sGam[r]);
      const uint4 vq = *reinterpret_cast<const uint4*>(&cQ[r * QS + c]);
      const uint4 vk = *reinterpret_cast<const uint4*>(&cK[r * QS + c]);
      const T* eqv = reinterpret_cast<const T*>(&vq);
      const T* ekv = reinterpret_cast<const T*>(&vk);
      uint4 oq, ok;
      T* oqe = reinterpret_cast<T*>(&oq);
      T* oke = reinterpret_cast<T*>(&ok);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        oqe[e] = from_f<T>(to_f(eqv[e]) * eq);
        oke[e] = from_f<T>(to_f(ekv[e]) * ek);
      }
      *reinterpret_cast<uint4*>(&rqs[r * QS + c]) = oq;
      *reinterpret_cast<uint4*>(&rkd[r * QS + c]) = ok;
    }
    T* rw = reinterpret_cast<T*>(rec + Rec::off_w);
    T* raq = reinterpret_cast<T*>(rec + Rec::off_aq);
    for (int i = tid; i < C * QV; i += NT) {  // W = the first DK columns of [W | U]
      const int r = i / QV, c = (i % QV) * E;
      *reinterpret_cast<uint4*>(&rw[r * QS + c]) = *reinterpret_cast<const uint4*>(&sX[r * XS + c]);
    }
#pragma unroll
    for (int j = 0; j < Rec::NSL; ++j) {  // U, one plane per slice of SW value columns
      T* ru = reinterpret_cast<T*>(rec + Rec::shared_bytes + j * Rec::u_bytes);
      for (int i = tid; i < C * UV; i += NT) {
        const int r = i / UV, c = (i % UV) * E;
        *reinterpret_cast<uint4*>(&ru[r * Rec::US + c]) =
            *reinterpret_cast<const uint4*>(&sX[r * XS + DK + j * Rec::SW + c]);
      }
    }
    for (int i = tid; i < C * AV; i += NT) {  // Aq
      const int r = i / AV, c = (i % AV) * E;
      *reinterpret_cast<uint4*>(&raq[r * AS + c]) = *reinterpret_cast<const uint4*>(&sAq[r * AS + c]);
    }
    // the pads: one 16-byte vector at the end of every row of every plane
    constexpr int NPAD = 4 + Rec::NSL;  // Qs, Kd, W, Aq, U planes
    for (int i = tid; i < C * NPAD; i += NT) {
      const int r = i % C, p = i / C;
      T* dst = p == 0 ? &rqs[r * QS + DK]
             : p == 1 ? &rkd[r * QS + DK]
             : p == 2 ? &rw[r * QS + DK]
             : p == 3 ? &raq[r * AS + C]
                      : reinterpret_cast<T*>(rec + Rec::shared_bytes + (p - 4) * Rec::u_bytes) + r * Rec::US + Rec::SW;
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    if (tid == 0) *reinterpret_cast<float4*>(rec + Rec::off_el) = make_float4(sEg[C - 1], 0.f, 0.f, 0.f);
  }
}

template <typename T, int DK, int DV, int SWP>
struct RecLayout {
  using Rec = WsRec<T, DK, DV, SWP>;
  static constexpr int SS = Rec::SW + 8;  // state slice row stride (elements)
  static constexpr size_t stage_bytes = Rec::shared_bytes + Rec::u_bytes;
  static constexpr size_t off_stage = 0;  // 2 stages: the shared part + this slice's U plane
  static constexpr size_t off_s = off_stage + 2 * stage_bytes;
  static constexpr size_t off_bar = off_s + 2ull * DK * SS * sizeof(T);
  static constexpr size_t bytes = off_bar + 16;
  static_assert(bytes <= 232448, "shared memory budget");
};

constexpr uint32_t kRecWait = 1u << 22;
// Count of state-scan CTAs whose bounded record-copy wait ran out (never expected).
__device__ unsigned int g_gdn_wait_timeouts = 0;

// One CTA per (sequence, head, slice of SW value columns): the columns of S evolve
// independently (X = U - W S, o = Qs S + Aq X and S' = e^gL S + Kd^T X act column by column),
// so each slice scans its own DK x SW block of the state.  Adjacent CTAs are the slices of one
// (sequence, head) and read the record's shared part at about the same time, from L2.
template <typename T, int DK, int DV, int SWP>
__global__ void __launch_bounds__(NT, 2) gdn_rec_kernel(const unsigned char* __restrict__ ws,
                                                        const float* __restrict__ s_in, float* __restrict__ s_out,
                                                        T* __restrict__ o, int H, int L, Strides18 sv) {
  using Lay = RecLayout<T, DK, DV, SWP>;
  using Rec = WsRec<T, DK, DV, SWP>;
  constexpr int QS = Rec::QS, AS = Rec::AS, US = Rec::US, SW = Rec::SW, SS = Lay::SS;
  constexpr int SM_T = DK / 16;
  constexpr int HT = SW / 16;  // n8 tiles per warp (two column groups of SW / 2)
  extern __shared__ __align__(128) unsigned char smem[];
  T* sS = reinterpret_cast<T*>(smem + Lay::off_s);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Lay::off_bar);

  const int64_t* st = sv.s;
  const int bh = blockIdx.x / Rec::NSL, slice = blockIdx.x % Rec::NSL;
  const int b = bh / H, h = bh % H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  T* og = o + b * st[9] + h * st[10] + slice * SW;
  const int nchunks = (L + C - 1) / C;
  const unsigned char* recs = ws + (size_t)bh * nchunks * Rec::bytes;

  // state: warp w holds S rows [16 (w % 4), +16) x slice columns [SW/2 (w / 4), +SW/2) (fp32)
  const bool s_owner = (warp & 3) < SM_T;
  const int sm0 = (warp & 3) * 16;
  const int sc0 = (warp >> 2) * (SW / 2);
  float Sr[HT][4];
  const float* s0 = s_in ? s_in + (size_t)bh * DK * DV + slice * SW : nullptr;
  if (s_owner) {
#pragma unroll
    for (int nt = 0; nt < HT; ++nt) {
      const int r = sm0 + gq, c = sc0 + nt * 8 + 2 * tq;
      Sr[nt][0] = s0 ? s0[r * DV + c] : 0.f;
      Sr[nt][1] = s0 ? s0[r * DV + c + 1] : 0.f;
      Sr[nt][2] = s0 ? s0[(r + 8) * DV + c] : 0.f;
      Sr[nt][3] = s0 ? s0[(r + 8) * DV + c + 1] : 0.f;
      st2(&sS[r * SS + c], Sr[nt][0], Sr[nt][1]);
      st2(&sS[(r + 8) * SS + c], Sr[nt][2], Sr[nt][3]);
    }
  }
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init_fence();
  }
  __syncthreads();
  auto issue = [&](int n) {  // thread 0: record n (shared part + this slice's U) -> stage n & 1
    unsigned char* dst = smem + Lay::off_stage + (size_t)(n & 1) * Lay::stage_bytes;
    const unsigned char* src = recs + (size_t)n * Rec::bytes;
    mbar_arrive_expect_tx(&bar[n & 1], (uint32_t)Lay::stage_bytes);
    bulk_load(dst, src, (uint32_t)Rec::shared_bytes, &bar[n & 1]);
    bulk_load(dst + Rec::shared_bytes, src + Rec::shared_bytes + slice * Rec::u_bytes, (uint32_t)Rec::u_bytes,
              &bar[n & 1]);
  };
  int nissued = 0;
  if (tid == 0)
    for (; nissued < min(nchunks, 2); ++nissued) issue(nissued);

  bool failed = false;
  int n = 0;
  for (; n < nchunks; ++n) {
    const int stage = n & 1;
    const bool ok = mbar_wait_bounded(&bar[stage], (uint32_t)((n >> 1) & 1), kRecWait);
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    unsigned char* sp = smem + Lay::off_stage + (size_t)stage * Lay::stage_bytes;
    const T* cQ = reinterpret_cast<const T*>(sp + Rec::off_qs);
    const T* cK = reinterpret_cast<const T*>(sp + Rec::off_kd);
    const T* cW = reinterpret_cast<const T*>(sp + Rec::off_w);
    const T* sAq = reinterpret_cast<const T*>(sp + Rec::off_aq);
    T* sX = reinterpret_cast<T*>(sp + Rec::shared_bytes);  // U, then X in place
    const float eL = *reinterpret_cast<const float*>(sp + Rec::off_el);
    const T* cS = sS + (size_t)(n & 1) * DK * SS;
    T* nS = sS + (size_t)((n + 1) & 1) * DK * SS;
    const int m0 = (warp & 3) * 16, c0 = (warp >> 2) * (SW / 2);

    // X = U - W S in place of U, and the first term of o = (q e^g) S + Aq X: both products
    // read the same S fragments, and (q e^g) S does not wait for X
    // (warp: m-tile w%4, column group w/4)
    float acc[HT][4];  // o accumulator
    {
      float accx[HT][4];
#pragma unroll
      for (int i = 0; i < HT; ++i) {
        acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        accx[i][0] = accx[i][1] = accx[i][2] = accx[i][3] = 0.f;
      }
#pragma unroll
      for (int k0 = 0; k0 < DK; k0 += 16) {
        uint32_t aw[4], aq[4];
        lda(aw, cW, QS, m0, k0);
        lda(aq, cQ, QS, m0, k0);
#pragma unroll
        for (int nn = 0; nn < SW / 2; nn += 16) {
          uint32_t bb[4];
          ldb_t(bb, cS, SS, k0, c0 + nn);
          mma_16816<T>(accx[nn / 8], aw, &bb[0]);
          mma_16816<T>(accx[nn / 8 + 1], aw, &bb[2]);
          mma_16816<T>(acc[nn / 8], aq, &bb[0]);
          mma_16816<T>(acc[nn / 8 + 1], aq, &bb[2]);
        }
      }
      const int ra = m0 + gq, rb = ra + 8;
#pragma unroll
      for (int nt = 0; nt < HT; ++nt) {
        const int c = c0 + nt * 8 + 2 * tq;
        const float2 ua = ld2(&sX[ra * US + c]), ub = ld2(&sX[rb * US + c]);
        st2(&sX[ra * US + c], ua.x - accx[nt][0], ua.y - accx[nt][1]);
        st2(&sX[rb * US + c], ub.x - accx[nt][2], ub.y - accx[nt][3]);
      }
    }
    __syncthreads();  // X complete

    // o += Aq X, and S = e^gL S + (k e^(gL - g))^T X for this warp's block
    {
      for (int k0 = 0; k0 <= m0; k0 += 16) {  // Aq lower triangular: k < m0 + 16
        uint32_t a[4];
        lda(a, sAq, AS, m0, k0);
#pragma unroll
        for (int nn = 0; nn < SW / 2; nn += 16) {
          uint32_t bb[4];
          ldb_t(bb, sX, US, k0, c0 + nn);
          mma_16816<T>(acc[nn / 8], a, &bb[0]);
          mma_16816<T>(acc[nn / 8 + 1], a, &bb[2]);
        }
      }
      const int ra = m0 + gq, rb = ra + 8;
      const int la = n * C + ra, lb = n * C + rb;
#pragma unroll
      for (int nt = 0; nt < HT; ++nt) {
        const int c = c0 + nt * 8 + 2 * tq;
        if (la < L) st2(&og[(int64_t)la * st[11] + c], acc[nt][0], acc[nt][1]);
        if (lb < L) st2(&og[(int64_t)lb * st[11] + c], acc[nt][2], acc[nt][3]);
      }
      if (s_owner) {
#pragma unroll
        for (int i = 0; i < HT; ++i) {
          Sr[i][0] *= eL; Sr[i][1] *= eL; Sr[i][2] *= eL; Sr[i][3] *= eL;
        }
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16) {
          uint32_t a[4];
          lda_t(a, cK, QS, sm0, k0);
#pragma unroll
          for (int nn = 0; nn < SW / 2; nn += 16) {
            uint32_t bb[4];
            ldb_t(bb, sX, US, k0, sc0 + nn);
            mma_16816<T>(Sr[nn / 8], a, &bb[0]);
            mma_16816<T>(Sr[nn / 8 + 1], a, &bb[2]);
          }
        }
#pragma unroll
        for (int nt = 0; nt < HT; ++nt) {
          const int r = sm0 + gq, c = sc0 + nt * 8 + 2 * tq;
          st2(&nS[r * SS + c], Sr[nt][0], Sr[nt][1]);
          st2(&nS[(r + 8) * SS + c], Sr[nt][2], Sr[nt][3]);
        }
      }
    }
    __syncthreads();  // end of chunk: the stage and nS are reusable
    if (tid == 0 && nissued < nchunks) {  // record n + 2 into the stage chunk n used
      fence_proxy_async_smem();
      issue(nissued);
      ++nissued;
    }
  }
  if (failed) {
    if (tid == 0) {  // let the copies in flight land (bounded), then report
      atomicAdd(&g_gdn_wait_timeouts, 1u);
      for (int u = n; u < nissued; ++u) mbar_wait_bounded(&bar[u & 1], (uint32_t)((u >> 1) & 1), kRecWait);
    }
    return;
  }
  if (s_owner) {
    float* so = s_out + (size_t)bh * DK * DV + slice * SW;
#pragma unroll
    for (int nt = 0; nt < HT; ++nt) {
      const int r = sm0 + gq, c = sc0 + nt * 8 + 2 * tq;
      *reinterpret_cast<float2*>(&so[r * DV + c]) = make_float2(Sr[nt][0], Sr[nt][1]);
      *reinterpret_cast<float2*>(&so[(r + 8) * DV + c]) = make_float2(Sr[nt][2], Sr[nt][3]);
    }
  }
}

// GatedRMSNorm on the scan's output rows, in place: o <- rmsnorm(o) * w * silu(gate) for each
// (token, head) row of DV values (gdn_attn.py:197-209 with rms_norm.py:547-553 roundings).
// A group of DV/8 lanes owns a row as 16-byte vectors (the row's sum of squares reduces over
// the group); each warp takes two groups of rows per iteration of a grid-stride loop, so every
// thread has four 16-byte loads in flight.  Row coordinates use 32-bit arithmetic (the host
// checks rows < 2^31).
template <typename T, int DV>
__global__ void __launch_bounds__(256) gdn_gate_norm_kernel(T* __restrict__ o, int64_t ob, int64_t oh, int64_t ol,
                                                            const T* __restrict__ gate, int64_t gate_rs,
                                                            int64_t gate_hs, const T* __restrict__ w, float eps, int H,
                                                            int L, int rows) {
  constexpr int LPR = DV / 8;  // lanes per row
  constexpr int RPW = 32 / LPR;
  constexpr int U = 2;         // row groups per warp iteration
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const uint4 wv = reinterpret_cast<const uint4*>(w)[sub];
  const T* we = reinterpret_cast<const T*>(&wv);
  float wf[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) wf[i] = to_f(we[i]);
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int wi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); wi * RPW * U < rows; wi += warps) {
    uint4* op[U];
    uint4 ov[U], gv[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int row = (wi * U + u) * RPW + lane / LPR;  // (b * L + l) * H + h
      ok[u] = row < rows;
      ov[u] = gv[u] = make_uint4(0, 0, 0, 0);
      op[u] = nullptr;
      if (ok[u]) {
        const unsigned bl = (unsigned)row / (unsigned)H, h = (unsigned)row - bl * (unsigned)H;
        const unsigned b = bl / (unsigned)L, l = bl - b * (unsigned)L;
        op[u] = reinterpret_cast<uint4*>(o + (int64_t)b * ob + (int64_t)h * oh + (int64_t)l * ol) + sub;
        ov[u] = *op[u];
        gv[u] = reinterpret_cast<const uint4*>(gate + (int64_t)bl * gate_rs + (int64_t)h * gate_hs)[sub];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const T* oe = reinterpret_cast<const T*>(&ov[u]);
      const T* ge = reinterpret_cast<const T*>(&gv[u]);
      float x[8];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[i] = to_f(oe[i]);
        ss += x[i] * x[i];
      }
#pragma unroll
      for (int o2 = 1; o2 < LPR; o2 <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o2);
      if (!ok[u]) continue;
      const float r = rsqrtf(ss / (float)DV + eps);
      // two elements per packed fp32 op / bf16x2 conversion (the same roundings as one at a time)
      uint32_t res[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const float2 xn = fmul2(make_float2(x[i], x[i + 1]), make_float2(r, r));
        const float2 xr = round2<T>(xn.x, xn.y);
        const float2 yw = fmul2(xr, make_float2(wf[i], wf[i + 1]));
        const float2 y = round2<T>(yw.x, yw.y);
        const float2 sg = silu2_(make_float2(to_f(ge[i]), to_f(ge[i + 1])));
        const float2 sgr = round2<T>(sg.x, sg.y);
        const float2 o2 = fmul2(y, sgr);
        res[i / 2] = pack2<T>(o2.x, o2.y);
      }
      *op[u] = make_uint4(res[0], res[1], res[2], res[3]);
    }
  }
}

// Value-column slices of the state scan: 64 wide, or 32 when the 64-wide slicing would occupy at
// most half of the SMs (tiny batches: 1-2 sequences x 12 heads), so the latency-bound chunk
// chains spread over more SMs.  Measured on the 172M prefill at T = 4096: 3.60 vs 3.96 ms at
// B = 1, 5.76 vs 6.08 at B = 2, equal at B = 4; wider batches (4 x 12 heads at Dv = 128 and the
// 8 x 12 x 64 op) are 5-7 % faster on 64-column slices.
bool narrow_slices(int64_t B, int64_t H, int64_t Dv) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return Dv >= 64 && 2 * B * H * (Dv / 64) <= (int64_t)sms && !forced(MB_FORCE_GDN_WIDE);
}

template <typename T, int DK, int DV, bool PREP, int SWP>
int launch_split_sw(const void* q, const void* k, const void* v, const float* beta, const float* g,
                    const float* s_in, float* s_out, void* o, int64_t B, int64_t H, int64_t L, const Strides18& sv,
                    const void* gate, int64_t gate_rs, int64_t gate_hs, const void* onorm_w, float eps, void* ws,
                    cudaStream_t stream, PrepIn<T> pin) {
  using WL = WyLayout<T, DK, DV>;
  using RL = RecLayout<T, DK, DV, SWP>;
  auto k1 = gdn_wy_kernel<T, DK, DV, PREP, SWP>;
  auto k2 = gdn_rec_kernel<T, DK, DV, SWP>;
  if (int rc0 = ensure_smem_attr((const void*)k1, (int)WL::bytes)) return rc0;
  if (int rc0 = ensure_smem_attr((const void*)k2, (int)RL::bytes)) return rc0;
  const int64_t nchunks = (L + C - 1) / C;
  k1<<<dim3((unsigned)nchunks, (unsigned)(B * H)), NT, WL::bytes, stream>>>(
      (const T*)q, (const T*)k, (const T*)v, beta, g, (int)H, (int)L, sv, (unsigned char*)ws, pin);
  int rc = check_launch("gdn_chunk (UT transform)");
  if (rc) return rc;
  k2<<<(unsigned)(B * H * WsRec<T, DK, DV, SWP>::NSL), NT, RL::bytes, stream>>>((const unsigned char*)ws, s_in, s_out,
                                                                             (T*)o, (int)H, (int)L, sv);
  rc = check_launch("gdn_chunk (state scan)");
  if (rc || gate == nullptr) return rc;
  const int64_t rows = B * L * H;
  if (rows >= (1LL << 31) - 64) return set_error(MB_ERR_SHAPE, "gdn_chunk (gated norm): %lld rows", (long long)rows);
  const int64_t* st = sv.s;
  const int64_t warps_needed = (rows + 2 * (256 / DV) - 1) / (2 * (256 / DV));  // DV/8 lanes per row, 2 groups
  const int64_t blocks = std::min<int64_t>((warps_needed + 7) / 8, 148 * 8);
  gdn_gate_norm_kernel<T, DV><<<(unsigned)blocks, 256, 0, stream>>>(
      (T*)o, st[9], st[10], st[11], (const T*)gate, gate_rs, gate_hs, (const T*)onorm_w, eps, (int)H, (int)L,
      (int)rows);
  return check_launch("gdn_chunk (gated norm)");
}

template <typename T, int DK, int DV, bool PREP = false>
int launch_split(const void* q, const void* k, const void* v, const float* beta, const float* g,
                 const float* s_in, float* s_out, void* o, int64_t B, int64_t H, int64_t L, const Strides18& sv,
                 const void* gate, int64_t gate_rs, int64_t gate_hs, const void* onorm_w, float eps, void* ws,
                 cudaStream_t stream, PrepIn<T> pin = PrepIn<T>{}) {
  if (narrow_slices(B, H, DV))
    return launch_split_sw<T, DK, DV, PREP, 32>(q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate, gate_rs, gate_hs,
                                               onorm_w, eps, ws, stream, pin);
  return launch_split_sw<T, DK, DV, PREP, 64>(q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate, gate_rs, gate_hs,
                                             onorm_w, eps, ws, stream, pin);
}

}  // namespace

// Workspace bytes of the split path for (Dk, Dv), or 0 when no split kernel exists.
int64_t gdn_split_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv, int dtype) {
  if (dtype != MB_BF16 && dtype != MB_F16) return 0;
  const int64_t nchunks = (L + C - 1) / C;
  int64_t rec = 0;
  const bool nar = narrow_slices(B, H, Dv);
  if (Dk == 32 && Dv == 64) rec = nar ? WsRec<__nv_bfloat16, 32, 64, 32>::bytes : WsRec<__nv_bfloat16, 32, 64>::bytes;
  if (Dk == 64 && Dv == 64) rec = nar ? WsRec<__nv_bfloat16, 64, 64, 32>::bytes : WsRec<__nv_bfloat16, 64, 64>::bytes;
  if (Dk == 64 && Dv == 128) rec = nar ? WsRec<__nv_bfloat16, 64, 128, 32>::bytes : WsRec<__nv_bfloat16, 64, 128>::bytes;
  return B * H * nchunks * rec;
}

int read_and_clear_gdn_timeouts(unsigned int* count) {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gdn_wait_timeouts, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_gdn_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess)
    return set_error(MB_ERR_CUDA, "wait_timeouts: %s", cudaGetErrorString(cudaGetLastError()));
  *count = v;
  return MB_OK;
}

// Returns 1 (and launches) when the split path serves this call, else 0.
int gdn_split_dispatch(int dtype, int64_t Dk, int64_t Dv, const void* q, const void* k, const void* v,
                       const float* beta, const float* g, const float* s_in, float* s_out, void* o, int64_t B,
                       int64_t H, int64_t L, const int64_t* strides, const void* gate, int64_t gate_rs,
                       int64_t gate_hs, const void* onorm_w, float eps, void* ws, int64_t ws_bytes, cudaStream_t st,
                       int* rc) {
  const int64_t need = gdn_split_workspace_bytes(B, H, L, Dk, Dv, dtype);
  if (need == 0 || ws == nullptr || ws_bytes < need || ((uintptr_t)ws & 15) || L == 0) return 0;
  if (strides[11] % 2 || strides[9] % 2 || strides[10] % 2 || ((uintptr_t)o & 3)) return 0;
  {  // the gated norm moves Dv / 32 values per lane as one vector
    const int64_t vec = 8, vb = 16;
    if (gate && (gate_rs % vec || gate_hs % vec || strides[9] % vec || strides[10] % vec || strides[11] % vec ||
                 (uintptr_t)gate % vb || (uintptr_t)o % vb || (uintptr_t)onorm_w % vb))
      return 0;
  }
  Strides18 sv;
  for (int i = 0; i < 18; ++i) sv.s[i] = strides[i];
#define MB_SPLIT_CASE(DK_, DV_)                                                                                     \
  if (Dk == DK_ && Dv == DV_) {                                                                                     \
    *rc = dtype == MB_BF16 ? launch_split<__nv_bfloat16, DK_, DV_>(q, k, v, beta, g, s_in, s_out, o, B, H, L, sv,    \
                                                                   gate, gate_rs, gate_hs, onorm_w, eps, ws, st)    \
                           : launch_split<__half, DK_, DV_>(q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate,    \
                                                            gate_rs, gate_hs, onorm_w, eps, ws, st);                \
    return 1;                                                                                                       \
  }
  MB_SPLIT_CASE(32, 64)
  MB_SPLIT_CASE(64, 64)
  MB_SPLIT_CASE(64, 128)
#undef MB_SPLIT_CASE
  return 0;
}

// Whole-layer prefill (16-bit, Dk = 64 or 32 with Dv = 2 Dk... see the dispatch below): the
// preparation fused into the UT-transform kernel, the state scan, the gated norm.
int gdn_prefill_split_dispatch(const void* proj, int64_t ps, const void* conv_w, const void* A_log,
                               const void* dt_bias, const void* conv_in, void* conv_out, const float* s_in,
                               float* s_out, const void* onorm_w, float eps, void* out, int64_t os, int64_t B,
                               int64_t Tn, int64_t H, int64_t Dk, int64_t Dv, int dtype, void* ws, int64_t ws_bytes,
                               cudaStream_t st, int* rc) {
  const int64_t need = gdn_split_workspace_bytes(B, H, Tn, Dk, Dv, dtype);
  if (need == 0 || ws == nullptr || ws_bytes < need || ((uintptr_t)ws & 15) || Tn == 0) return 0;
  // one channel group per lane / one 8-row run per warp needs 2 Dk + Dv = 256 channels per head
  if (!(Dk == 64 && Dv == 128)) return 0;
  const int64_t C = H * (2 * Dk + Dv);
  if (ps % 8 || (uintptr_t)proj % 16 || (uintptr_t)conv_w % 16 || (conv_in && (uintptr_t)conv_in % 16) ||
      (conv_out && (uintptr_t)conv_out % 16) || os % 8 || (uintptr_t)out % 16 || (uintptr_t)onorm_w % 16 ||
      C % 8 || (C + 2 * H) % 8)
    return 0;
  Strides18 sv;
  for (int i = 0; i < 18; ++i) sv.s[i] = 0;
  sv.s[9] = Tn * os;
  sv.s[10] = Dv;
  sv.s[11] = os;
  auto go = [&](auto t) {
    using T = decltype(t);
    PrepIn<T> pin;
    pin.proj = (const T*)proj;
    pin.ps = ps;
    pin.conv_w = (const T*)conv_w;
    pin.A_log = (const T*)A_log;
    pin.dt_bias = (const T*)dt_bias;
    pin.conv_in = (const T*)conv_in;
    pin.conv_out = (T*)conv_out;
    const T* gate = (const T*)proj + C + 2 * H;
    return launch_split<T, 64, 128, true>(nullptr, nullptr, nullptr, nullptr, nullptr, s_in, s_out, out, B, H, Tn, sv,
                                          gate, ps, Dv, onorm_w, eps, ws, st, pin);
  };
  *rc = dtype == MB_BF16 ? go(__nv_bfloat16{}) : go(__half{});
  return 1;
}

}  // namespace mb

extern "C" int motif_b200_gdn_prefill_ws(const void* proj, int64_t proj_stride, const void* conv_w, const void* A_log,
                                         const void* dt_bias, const void* conv_in, void* conv_out,
                                         const float* state_in, float* state_out, const void* onorm_w, float eps,
                                         void* out, int64_t out_stride, int64_t B, int64_t T, int64_t H, int64_t Dk,
                                         int64_t Dv, int dtype, void* workspace, int64_t workspace_bytes,
                                         void* stream) {
  using namespace mb;
  MB_REQUIRE(proj && conv_w && A_log && dt_bias && state_out && onorm_w && out, MB_ERR_ARG,
             "gdn_prefill_ws: null pointer");
  MB_REQUIRE(conv_out == nullptr || conv_out != conv_in, MB_ERR_ARG, "gdn_prefill_ws: conv_out must not alias conv_in");
  MB_REQUIRE(B >= 0 && T >= 0 && H > 0 && B * H < (1LL << 31) && T < (1LL << 31), MB_ERR_SHAPE,
             "gdn_prefill_ws: bad shape");
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "gdn_prefill_ws: 16-bit dtypes only");
  MB_REQUIRE(workspace == nullptr || workspace_bytes >= gdn_split_workspace_bytes(B, H, T, Dk, Dv, dtype),
             MB_ERR_ARG, "gdn_prefill_ws: workspace too small");
  if (B == 0 || T == 0) return set_error(MB_ERR_SHAPE, "gdn_prefill_ws: empty input");
  int rc = MB_OK;
  if (gdn_prefill_split_dispatch(proj, proj_stride, conv_w, A_log, dt_bias, conv_in, conv_out, state_in, state_out,
                                 onorm_w, eps, out, out_stride, B, T, H, Dk, Dv, dtype, workspace, workspace_bytes,
                                 (cudaStream_t)stream, &rc))
    return rc;
  return motif_b200_gdn_prefill(proj, proj_stride, conv_w, A_log, dt_bias, conv_in, conv_out, state_in, state_out,
                                onorm_w, eps, out, out_stride, B, T, H, Dk, Dv, dtype, stream);
}
