// Chunked gated delta rule for 16-bit inputs (bf16 / fp16): the same fused per-(b, h) walk
// over 64-token chunks as gdn_chunk.cu, with every product on 16-bit m16n8k16 tensor-core
// MMAs fed by ldmatrix (operands staged in shared memory in the input dtype), fp32
// accumulation, and the recurrent state S kept in fp32 registers.
//
// Per chunk (motif/ops/gated_deltanet.py:137-177, :312-319):
//   (b) warps 0-3: KK = k k^T -> A = -(beta_i KK_ij e^{g_i - g_j}) (j < i) and the inverse of
//       the 16x16 diagonal block of (I - A) owned by the warp (fp32 forward substitution);
//       warps 4-7: QK = q k^T -> Aq = QK_ij e^{g_i - g_j} (j <= i)
//   (d) [W | U] = (I - A)^-1 [k beta e^g | v beta] by blocked forward substitution over the
//       four 16-row block rows.  Each warp owns a set of output columns, and a block row only
//       needs earlier block rows of the SAME columns, so the solve is warp-local.
//   (e) X = U - W S
//   (f) warps 0-3: o = e^g (q S) + Aq X for 16 full rows each, then the GatedRMSNorm epilogue
//       (row reductions stay inside the warp); warps 4-7: S = e^{g_L} S + k^T (e^{g_L - g} X)
// Precision: products round their operands to the input dtype (bf16 / fp16); S, the
// accumulators and the diagonal inverses stay fp32.
#include <type_traits>

#include "common.cuh"
#include "gdn_mma.cuh"

namespace mb {
namespace {
using namespace gdnk;

template <typename T, int DK, int DV>
struct FastLayout {
  static constexpr int QS = DK + 8;         // sQ / sK row stride (elements)
  static constexpr int VS = DV + 8;         // sV / sXd / sS row stride
  static constexpr int AS = C + 8;          // sA / sAq row stride
  static constexpr int XS = DK + DV + 8;    // sX row stride ([W | U] then [W | X])
  static constexpr int TS = 16 + 8;         // sTd row stride
  static constexpr size_t q_bytes = 2ull * C * QS * sizeof(T);
  static constexpr size_t v_bytes = 2ull * C * VS * sizeof(T);
  static constexpr size_t off_q = 0;
  static constexpr size_t off_k = off_q + q_bytes;
  static constexpr size_t off_v = off_k + q_bytes;
  static constexpr size_t off_a = off_v + v_bytes;
  static constexpr size_t off_aq = off_a + (size_t)C * AS * sizeof(T);
  static constexpr size_t off_x = off_aq + (size_t)C * AS * sizeof(T);
  static constexpr size_t off_xd = off_x + (size_t)C * XS * sizeof(T);
  static constexpr size_t off_s = off_xd + (size_t)C * VS * sizeof(T);
  static constexpr size_t off_td = off_s + 2ull * DK * VS * sizeof(T);
  static constexpr size_t off_ad = off_td + 4ull * 16 * TS * sizeof(T);
  static constexpr size_t off_vec = off_ad + 4ull * 16 * 17 * 4;
  static constexpr size_t off_gate = off_vec + 4ull * C * 4;  // gate tiles, staged with q/k/v
  // raw rows before the chunk (two, alternating by chunk parity) and rows 29..31 of the chunk
  static constexpr size_t off_halo = off_gate + 2ull * C * VS * sizeof(T);
  static constexpr size_t halo_elems = 3ull * (2 * DK + DV);
  static constexpr size_t off_part = off_halo + 3 * halo_elems * sizeof(T);  // [64 rows][2] fp32
  static constexpr size_t off_cw = off_part + 2ull * C * 4;                  // conv weights [NCH][4] fp32
  static constexpr size_t bytes = off_cw + 4ull * (2 * DK + DV) * 4;
  static_assert(bytes <= 232448, "shared memory budget");
};

// Inputs of the fused preparation (PREP = true): q, k, v then point at the RAW projection
// columns, and beta / g are computed from the raw a / b columns (gdn_attn.py:116-136,183-197).
template <typename T>
struct PrepArgs {
  const T* conv_w;   // [C][4], C = H (2 Dk + Dv) channels q | k | v
  const T* A_log;    // [H]
  const T* dt_bias;  // [H]
  const T* conv_in;  // [B][3][C] previous raw inputs or nullptr (zeros)
  T* conv_out;       // [B][3][C] last three raw inputs (must not alias conv_in)
  const T* a_col;    // raw a column of head 0 (row stride ps, head stride 1)
  const T* b_col;    // raw b column of head 0
  int64_t ps;        // projection row stride
};

template <typename T, int DK, int DV, bool PREP>
__global__ void __launch_bounds__(NT, 1) gdn_chunk_fast_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ beta,
    const float* __restrict__ g, const float* __restrict__ s_in, float* __restrict__ s_out, T* __restrict__ o,
    int H, int L, Strides18 sv, const T* __restrict__ gate, int64_t gate_rs, int64_t gate_hs,
    const T* __restrict__ onorm_w, float onorm_eps, PrepArgs<T> pa) {
  using Lay = FastLayout<T, DK, DV>;
  constexpr int QS = Lay::QS, VS = Lay::VS, AS = Lay::AS, XS = Lay::XS, TS = Lay::TS;
  constexpr int NTILE = (DK + DV) / 8;  // n8 tiles of the solve
  constexpr int SOLVE_T = (NTILE + NW - 1) / NW;
  constexpr int SM_T = DK / 16;         // m16 tiles of S (warps 4 .. 4 + SM_T - 1 own S)
  constexpr int DVT = DV / 8;           // n8 tiles across the value dim
  extern __shared__ __align__(16) unsigned char smem[];
  T* sQ = reinterpret_cast<T*>(smem + Lay::off_q);
  T* sK = reinterpret_cast<T*>(smem + Lay::off_k);
  T* sV = reinterpret_cast<T*>(smem + Lay::off_v);
  T* sA = reinterpret_cast<T*>(smem + Lay::off_a);
  T* sAq = reinterpret_cast<T*>(smem + Lay::off_aq);
  T* sX = reinterpret_cast<T*>(smem + Lay::off_x);
  T* sXd = reinterpret_cast<T*>(smem + Lay::off_xd);
  T* sS = reinterpret_cast<T*>(smem + Lay::off_s);
  T* sTd = reinterpret_cast<T*>(smem + Lay::off_td);
  float* sAd = reinterpret_cast<float*>(smem + Lay::off_ad);
  float* sGam = reinterpret_cast<float*>(smem + Lay::off_vec);
  float* sEg = sGam + C;
  float* sDl = sEg + C;
  float* sBeta = sDl + C;
  T* sG = reinterpret_cast<T*>(smem + Lay::off_gate);
  T* sHalo = reinterpret_cast<T*>(smem + Lay::off_halo);  // [2][3][NCH], then sHaloMid [3][NCH]
  float* sPart = reinterpret_cast<float*>(smem + Lay::off_part);
  float* sCw = reinterpret_cast<float*>(smem + Lay::off_cw);

  const int64_t* st = sv.s;
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const T* qg = q + b * st[0] + h * st[1];
  const T* kg = k + b * st[3] + h * st[4];
  const T* vg = v + b * st[6] + h * st[7];
  T* og = o + b * st[9] + h * st[10];
  const float* bg = beta + b * st[12] + h * st[13];
  const float* gg = g + b * st[15] + h * st[16];
  const int nchunks = (L + C - 1) / C;
  // gate rows are token-major: row (b * L + l), head h at column offset h * gate_hs
  const T* gbase = gate ? gate + (int64_t)b * L * gate_rs + h * gate_hs : nullptr;
  const bool gate_async = gate && ((uintptr_t)gbase % 16 == 0) && (gate_rs % (16 / sizeof(T)) == 0);

  // ---- state: warp w holds S rows [16 (w % 4), +16) x value columns [DV/2 (w / 4), +DV/2) (fp32)
  constexpr int HT = DVT / 2;  // n8 tiles per column half
  const bool s_owner = (warp & 3) < SM_T;
  const int sm0 = (warp & 3) * 16;
  const int sc0 = (warp >> 2) * (DV / 2);
  float Sr[HT][4];
  const float* s0 = s_in ? s_in + (size_t)bh * DK * DV : nullptr;
  if (s_owner) {
#pragma unroll
    for (int nt = 0; nt < HT; ++nt) {
      const int r = sm0 + gq, c = sc0 + nt * 8 + 2 * tq;
      Sr[nt][0] = s0 ? s0[r * DV + c] : 0.f;
      Sr[nt][1] = s0 ? s0[r * DV + c + 1] : 0.f;
      Sr[nt][2] = s0 ? s0[(r + 8) * DV + c] : 0.f;
      Sr[nt][3] = s0 ? s0[(r + 8) * DV + c + 1] : 0.f;
      st2(&sS[r * VS + c], Sr[nt][0], Sr[nt][1]);
      st2(&sS[(r + 8) * VS + c], Sr[nt][2], Sr[nt][3]);
    }
  }

  auto load_chunk = [&](int n, int stage) {
    constexpr int QV = DK * (int)sizeof(T) / 16, VV = DV * (int)sizeof(T) / 16;
    constexpr int E = 16 / sizeof(T);
    T* dq = sQ + (size_t)stage * C * QS;
    T* dk = sK + (size_t)stage * C * QS;
    T* dv = sV + (size_t)stage * C * VS;
    for (int i = tid; i < C * (2 * QV + VV); i += NT) {
      const int r = i / (2 * QV + VV), c = i % (2 * QV + VV);
      const int l = n * C + r;
      const bool ok = l < L;
      const int64_t lc = ok ? l : 0;
      if (c < QV)
        cp_async16(dq + r * QS + c * E, qg + lc * st[2] + c * E, ok);
      else if (c < 2 * QV)
        cp_async16(dk + r * QS + (c - QV) * E, kg + lc * st[5] + (c - QV) * E, ok);
      else
        cp_async16(dv + r * VS + (c - 2 * QV) * E, vg + lc * st[8] + (c - 2 * QV) * E, ok);
    }
    if (gate_async) {
      T* dg = sG + (size_t)stage * C * VS;
      for (int i = tid; i < C * VV; i += NT) {
        const int r = i / VV, c = i % VV;
        const int l = n * C + r;
        const bool ok = l < L;
        cp_async16(dg + r * VS + c * E, gbase + (int64_t)(ok ? l : 0) * gate_rs + c * E, ok);
      }
    }
    cp_async_commit();
  };
  float pg[2], pb[2];
  auto fetch_gb = [&](int n) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int l = n * C + lane + 32 * e;
      const bool ok = l < L;
      if constexpr (PREP) {
        const int64_t row = ((int64_t)b * L + (ok ? l : 0)) * pa.ps + h;
        pg[e] = ok ? to_f(pa.a_col[row]) : 0.f;  // raw a
        pb[e] = ok ? to_f(pa.b_col[row]) : 0.f;  // raw b
      } else {
        pg[e] = ok ? gg[(int64_t)l * st[17]] : 0.f;
        pb[e] = ok ? bg[(int64_t)l * st[14]] : 0.f;
      }
    }
  };
  // PREP: raw inputs of the three positions before the current chunk, per q | k | v channel
  constexpr int NCH = 2 * DK + DV;
  float aexp = 0.f, dtb = 0.f;
  auto gchan = [&](int c) {  // global conv channel of local channel c
    return c < DK ? h * DK + c : (c < 2 * DK ? H * DK + h * DK + (c - DK) : 2 * H * DK + h * DV + (c - 2 * DK));
  };
  if constexpr (PREP) {
    const int Ct = H * (2 * DK + DV);
    for (int i = tid; i < 3 * NCH; i += NT) {
      const int r = i / NCH, c = i % NCH;
      sHalo[r * NCH + c] = pa.conv_in ? pa.conv_in[((int64_t)b * 3 + r) * Ct + gchan(c)] : from_f<T>(0.f);  // buffer 0
    }
    for (int i = tid; i < 4 * NCH; i += NT) sCw[i] = to_f(pa.conv_w[(int64_t)gchan(i >> 2) * 4 + (i & 3)]);
    aexp = -to_f(from_f<T>(expf(to_f(pa.A_log[h]))));
    dtb = to_f(pa.dt_bias[h]);
  }
  if (nchunks > 0) {
    load_chunk(0, 0);
    if (warp == 0) fetch_gb(0);
  }

  for (int n = 0; n < nchunks; ++n) {
    const int stage = n & 1;
    if (n + 1 < nchunks) {
      load_chunk(n + 1, stage ^ 1);  // that stage was last read in iteration n-1 (ended by a barrier)
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    const T* cQ = sQ + (size_t)stage * C * QS;
    const T* cK = sK + (size_t)stage * C * QS;
    const T* cV = sV + (size_t)stage * C * VS;
    const T* cS = sS + (size_t)(n & 1) * DK * VS;
    T* nS = sS + (size_t)((n + 1) & 1) * DK * VS;

    // (a) gamma = inclusive cumsum(g), e^gamma, e^(gL - gamma), beta  (warp 0)
    if (warp == 0) {
      if constexpr (PREP) {
        // beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias), rounded like the reference's
        // 16-bit ops; padded rows get beta = g = 0 (the reference pads with zeros)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool ok = n * C + lane + 32 * e < L;
          const float bt = to_f(from_f<T>(sigmoidf_(pb[e])));
          const float gt = to_f(from_f<T>(aexp * to_f(from_f<T>(softplusf_(to_f(from_f<T>(pg[e] + dtb)))))));
          pb[e] = ok ? bt : 0.f;
          pg[e] = ok ? gt : 0.f;
        }
      }
      float x0 = pg[0], x1 = pg[1];
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
      const float gl = __shfl_sync(0xffffffffu, x1, 31);
      sGam[lane] = x0;
      sGam[lane + 32] = x1;
      sEg[lane] = expf(x0);
      sEg[lane + 32] = expf(x1);
      sDl[lane] = expf(gl - x0);
      sDl[lane + 32] = expf(gl - x1);
      sBeta[lane] = pb[0];
      sBeta[lane + 32] = pb[1];
      if (n + 1 < nchunks) fetch_gb(n + 1);
    }
    __syncthreads();  // (1) chunk data + gamma visible
    const float eL = sEg[C - 1];

    if constexpr (PREP) {
      // causal depthwise conv (taps 4) + SiLU + the q / k L2 norms (gdn_attn.py:116-136,190-191),
      // in place.  Tasks = column group (q, k, v in 64-channel groups) x row half; a lane owns one
      // token row, so each row's L2 norm is lane-local, and walks the group's channel pairs.
      // x[r-1..r-3] come from the lanes below by shuffles (from saved halo rows for lanes 0-2).
      const int Ct = H * (2 * DK + DV);
      const int hb = n & 1;
      T* haloPrev = sHalo + hb * Lay::halo_elems;       // raw rows -3..-1 of this chunk
      T* haloNext = sHalo + (hb ^ 1) * Lay::halo_elems;  // raw rows 61..63 -> next chunk
      T* haloMid = sHalo + 2 * Lay::halo_elems;          // raw rows 29..31 of this chunk
      for (int i = tid; i < 3 * NCH / 2; i += NT) {
        const int r = (2 * i) / NCH, c = (2 * i) % NCH;
        const T* src = c < DK ? cQ + c : (c < 2 * DK ? cK + (c - DK) : cV + (c - 2 * DK));
        const int stride = c < 2 * DK ? QS : VS;
        *reinterpret_cast<uint32_t*>(haloMid + r * NCH + c) = *reinterpret_cast<const uint32_t*>(src + (29 + r) * stride);
        *reinterpret_cast<uint32_t*>(haloNext + r * NCH + c) = *reinterpret_cast<const uint32_t*>(src + (61 + r) * stride);
      }
      __syncthreads();
      constexpr int NCG = 2 + DV / 64;
      if (warp < 2 * NCG) {
        const int cg = warp >> 1, half = warp & 1;
        const int r = half * 32 + lane;
        const T* halo = half == 0 ? haloPrev : haloMid;
        auto conv_rows = [&](auto width_c, auto norm_c, T* colbase, int stride, int cbase) {
          constexpr int W = decltype(width_c)::value;
          constexpr bool NORM = decltype(norm_c)::value;
          const bool ok = n * C + r < L;
          const bool is_last = n * C + r == L - 1;
          float ss = 0.f;
#pragma unroll 4
          for (int p = 0; p < W / 2; ++p) {
            const int cl = cbase + 2 * p;
            const uint32_t xr = *reinterpret_cast<const uint32_t*>(colbase + r * stride + 2 * p);
            uint32_t x1 = __shfl_up_sync(0xffffffffu, xr, 1);
            uint32_t x2 = __shfl_up_sync(0xffffffffu, xr, 2);
            uint32_t x3 = __shfl_up_sync(0xffffffffu, xr, 3);
            if (lane < 3) {  // rows before this half come from the saved halo rows
              const uint32_t h0 = *reinterpret_cast<const uint32_t*>(halo + 0 * NCH + cl);
              const uint32_t h1 = *reinterpret_cast<const uint32_t*>(halo + 1 * NCH + cl);
              const uint32_t h2 = *reinterpret_cast<const uint32_t*>(halo + 2 * NCH + cl);
              if (lane == 0) { x1 = h2; x2 = h1; x3 = h0; }
              if (lane == 1) { x2 = h2; x3 = h1; }
              if (lane == 2) { x3 = h2; }
            }
            const T* e0 = reinterpret_cast<const T*>(&xr);
            const T* e1 = reinterpret_cast<const T*>(&x1);
            const T* e2 = reinterpret_cast<const T*>(&x2);
            const T* e3 = reinterpret_cast<const T*>(&x3);
            float y[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const float4 w = *reinterpret_cast<const float4*>(sCw + (cl + j) * 4);
              const float a = conv4f(w.x, w.y, w.z, w.w, to_f(e3[j]), to_f(e2[j]), to_f(e1[j]), to_f(e0[j]));
              y[j] = ok ? to_f(from_f<T>(siluf_(to_f(from_f<T>(a))))) : 0.f;
            }
            if (is_last && pa.conv_out) {  // raw inputs at L-3 .. L-1 become the carried conv state
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int64_t gc = gchan(cl + j);
                pa.conv_out[((int64_t)b * 3 + 0) * Ct + gc] = e2[j];
                pa.conv_out[((int64_t)b * 3 + 1) * Ct + gc] = e1[j];
                pa.conv_out[((int64_t)b * 3 + 2) * Ct + gc] = e0[j];
              }
            }
            const uint32_t yp = pack2<T>(y[0], y[1]);
            // the warp has read every input row of pair p above, so row r can be overwritten
            *reinterpret_cast<uint32_t*>(colbase + r * stride + 2 * p) = yp;
            if constexpr (NORM) {
              const T* yy = reinterpret_cast<const T*>(&yp);
              ss += to_f(yy[0]) * to_f(yy[0]) + to_f(yy[1]) * to_f(yy[1]);
            }
          }
          if constexpr (NORM) {  // second pass over the lane's own row: apply the L2 scale
            const float sc = l2_scale(ss, cbase == 0 ? rsqrtf((float)DK) : 1.f);
#pragma unroll 4
            for (int p = 0; p < W / 2; ++p) {
              uint32_t* at = reinterpret_cast<uint32_t*>(colbase + r * stride + 2 * p);
              const uint32_t yp = *at;
              const T* yy = reinterpret_cast<const T*>(&yp);
              *at = pack2<T>(to_f(yy[0]) * sc, to_f(yy[1]) * sc);
            }
          }
        };
        if (cg == 0)
          conv_rows(std::integral_constant<int, DK>{}, std::true_type{}, const_cast<T*>(cQ), QS, 0);
        else if (cg == 1)
          conv_rows(std::integral_constant<int, DK>{}, std::true_type{}, const_cast<T*>(cK), QS, DK);
        else
          conv_rows(std::integral_constant<int, 64>{}, std::false_type{}, const_cast<T*>(cV) + (cg - 2) * 64, VS,
                    2 * DK + (cg - 2) * 64);
      }
      __syncthreads();
    }

    // (b) KK -> A (+ diagonal inverses) on warps 0-3, QK -> Aq on warps 4-7
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
          const int j = nt * 8 + 2 * tq;
          const float gj0 = sGam[j], gj1 = sGam[j + 1];
          const float a00 = j < i0 ? b0 * acc[nt][0] * expf(gi0 - gj0) : 0.f;
          const float a01 = j + 1 < i0 ? b0 * acc[nt][1] * expf(gi0 - gj1) : 0.f;
          const float a10 = j < i1 ? b1 * acc[nt][2] * expf(gi1 - gj0) : 0.f;
          const float a11 = j + 1 < i1 ? b1 * acc[nt][3] * expf(gi1 - gj1) : 0.f;
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
        // T_ww = (I - A_ww)^-1: lane c < 16 owns column c; rows by forward substitution.
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
        for (int nt = 0; nt < 8; ++nt) {
          const int j = nt * 8 + 2 * tq;
          const float gj0 = sGam[j], gj1 = sGam[j + 1];
          st2(&sAq[i0 * AS + j], j <= i0 ? acc[nt][0] * expf(gi0 - gj0) : 0.f,
              j + 1 <= i0 ? acc[nt][1] * expf(gi0 - gj1) : 0.f);
          st2(&sAq[i1 * AS + j], j <= i1 ? acc[nt][2] * expf(gi1 - gj0) : 0.f,
              j + 1 <= i1 ? acc[nt][3] * expf(gi1 - gj1) : 0.f);
        }
      }
    }
    __syncthreads();  // (2) A, Aq, T_ii visible

    // (d) blocked forward substitution, warp-local in its column tiles
#pragma unroll
    for (int bi = 0; bi < 4; ++bi) {
      const int r0 = bi * 16;
#pragma unroll
      for (int ti = 0; ti < SOLVE_T; ++ti) {
        const int tile = warp + NW * ti;
        if (tile >= NTILE) break;
        const int c0 = tile * 8;
        // acc = RHS rows r0.., columns c0..: [k beta e^g | v beta]
        float acc[4];
        {
          const int ra = r0 + gq, rb = ra + 8, c = c0 + 2 * tq;
          if (c0 < DK) {
            const float sa = sBeta[ra] * sEg[ra], sb = sBeta[rb] * sEg[rb];
            const float2 xa = ld2(&cK[ra * QS + c]), xb = ld2(&cK[rb * QS + c]);
            acc[0] = xa.x * sa; acc[1] = xa.y * sa; acc[2] = xb.x * sb; acc[3] = xb.y * sb;
          } else {
            const float sa = sBeta[ra], sb = sBeta[rb];
            const float2 xa = ld2(&cV[ra * VS + c - DK]), xb = ld2(&cV[rb * VS + c - DK]);
            acc[0] = xa.x * sa; acc[1] = xa.y * sa; acc[2] = xb.x * sb; acc[3] = xb.y * sb;
          }
        }
        for (int bj = 0; bj < bi; ++bj) {  // + A_ij X_j
          uint32_t a[4], bb[2];
          lda(a, sA, AS, r0, bj * 16);
          ldb_t1(bb, sX, XS, bj * 16, c0);
          mma_16816<T>(acc, a, bb);
        }
        // R_i (rounded) -> sX rows r0.., then X_i = T_ii R_i
        {
          const int ra = r0 + gq, c = c0 + 2 * tq;
          st2(&sX[ra * XS + c], acc[0], acc[1]);
          st2(&sX[(ra + 8) * XS + c], acc[2], acc[3]);
        }
        __syncwarp();
        {
          uint32_t a[4], bb[2];
          lda(a, sTd + bi * 16 * TS, TS, 0, 0);
          ldb_t1(bb, sX, XS, r0, c0);
          float x[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816<T>(x, a, bb);
          __syncwarp();
          const int ra = r0 + gq, c = c0 + 2 * tq;
          st2(&sX[ra * XS + c], x[0], x[1]);
          st2(&sX[(ra + 8) * XS + c], x[2], x[3]);
        }
        __syncwarp();
      }
    }
    __syncthreads();  // (3) [W | U] complete

    // (e) X = U - W S  (warp: m-tile w%4, value-column half w/4); also Xd = e^(gL - g) X
    {
      const int m0 = (warp & 3) * 16;
      const int nbase = (warp >> 2) * (DV / 2);
      float acc[HT][4];
#pragma unroll
      for (int i = 0; i < HT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
      for (int k0 = 0; k0 < DK; k0 += 16) {
        uint32_t a[4];
        lda(a, sX, XS, m0, k0);
#pragma unroll
        for (int nn = 0; nn < DV / 2; nn += 16) {
          uint32_t bb[4];
          ldb_t(bb, cS, VS, k0, nbase + nn);
          mma_16816<T>(acc[nn / 8], a, &bb[0]);
          mma_16816<T>(acc[nn / 8 + 1], a, &bb[2]);
        }
      }
      const int ra = m0 + gq, rb = ra + 8;
      const float da = sDl[ra], db = sDl[rb];
#pragma unroll
      for (int nt = 0; nt < HT; ++nt) {
        const int c = nbase + nt * 8 + 2 * tq;
        const float2 ua = ld2(&sX[ra * XS + DK + c]), ub = ld2(&sX[rb * XS + DK + c]);
        const float x0 = ua.x - acc[nt][0], x1 = ua.y - acc[nt][1];
        const float x2 = ub.x - acc[nt][2], x3 = ub.y - acc[nt][3];
        st2(&sX[ra * XS + DK + c], x0, x1);
        st2(&sX[rb * XS + DK + c], x2, x3);
        st2(&sXd[ra * VS + c], x0 * da, x1 * da);
        st2(&sXd[rb * VS + c], x2 * db, x3 * db);
      }
    }
    __syncthreads();  // (4) X, Xd complete

    // (f) every warp: rows [16 (w % 4), +16) x value columns [DV/2 (w / 4), +DV/2) of
    //     o = e^g (q S) + Aq X  and  S = e^gL S + k^T Xd
    {
      const int m0 = (warp & 3) * 16, c0 = (warp >> 2) * (DV / 2);
      float acc[HT][4];
#pragma unroll
      for (int i = 0; i < HT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
      for (int k0 = 0; k0 < DK; k0 += 16) {
        uint32_t a[4];
        lda(a, cQ, QS, m0, k0);
#pragma unroll
        for (int nn = 0; nn < DV / 2; nn += 16) {
          uint32_t bb[4];
          ldb_t(bb, cS, VS, k0, c0 + nn);
          mma_16816<T>(acc[nn / 8], a, &bb[0]);
          mma_16816<T>(acc[nn / 8 + 1], a, &bb[2]);
        }
      }
      const int ra = m0 + gq, rb = ra + 8;
      const float ea = sEg[ra], eb = sEg[rb];
#pragma unroll
      for (int i = 0; i < HT; ++i) {
        acc[i][0] *= ea; acc[i][1] *= ea; acc[i][2] *= eb; acc[i][3] *= eb;
      }
      for (int k0 = 0; k0 <= m0; k0 += 16) {  // Aq lower triangular: k < m0 + 16
        uint32_t a[4];
        lda(a, sAq, AS, m0, k0);
#pragma unroll
        for (int nn = 0; nn < DV / 2; nn += 16) {
          uint32_t bb[4];
          ldb_t(bb, sX + DK, XS, k0, c0 + nn);
          mma_16816<T>(acc[nn / 8], a, &bb[0]);
          mma_16816<T>(acc[nn / 8 + 1], a, &bb[2]);
        }
      }
      const int la = n * C + ra, lb = n * C + rb;
      float ssa = 0.f, ssb = 0.f;
      if (gate == nullptr) {
#pragma unroll
        for (int nt = 0; nt < HT; ++nt) {
          const int c = c0 + nt * 8 + 2 * tq;
          if (la < L) st2(&og[(int64_t)la * st[11] + c], acc[nt][0], acc[nt][1]);
          if (lb < L) st2(&og[(int64_t)lb * st[11] + c], acc[nt][2], acc[nt][3]);
        }
      } else {
        // partial sums of squares of this half-row (after the reference's o.to(dtype))
#pragma unroll
        for (int nt = 0; nt < HT; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[nt][e] = to_f(from_f<T>(acc[nt][e]));
          ssa += acc[nt][0] * acc[nt][0] + acc[nt][1] * acc[nt][1];
          ssb += acc[nt][2] * acc[nt][2] + acc[nt][3] * acc[nt][3];
        }
        ssa += __shfl_xor_sync(0xffffffffu, ssa, 1);
        ssa += __shfl_xor_sync(0xffffffffu, ssa, 2);
        ssb += __shfl_xor_sync(0xffffffffu, ssb, 1);
        ssb += __shfl_xor_sync(0xffffffffu, ssb, 2);
        if (tq == 0) {
          sPart[ra * 2 + (warp >> 2)] = ssa;
          sPart[rb * 2 + (warp >> 2)] = ssb;
        }
      }
      // state update for this warp's S block (independent of the o epilogue)
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
          for (int nn = 0; nn < DV / 2; nn += 16) {
            uint32_t bb[4];
            ldb_t(bb, sXd, VS, k0, sc0 + nn);
            mma_16816<T>(Sr[nn / 8], a, &bb[0]);
            mma_16816<T>(Sr[nn / 8 + 1], a, &bb[2]);
          }
        }
#pragma unroll
        for (int nt = 0; nt < HT; ++nt) {
          const int r = sm0 + gq, c = sc0 + nt * 8 + 2 * tq;
          st2(&nS[r * VS + c], Sr[nt][0], Sr[nt][1]);
          st2(&nS[(r + 8) * VS + c], Sr[nt][2], Sr[nt][3]);
        }
      }
      if (gate != nullptr) {
        __syncthreads();  // (4b) both halves' partial row sums visible
        ssa = sPart[ra * 2] + sPart[ra * 2 + 1];
        ssb = sPart[rb * 2] + sPart[rb * 2 + 1];
        const float rsa = rsqrtf(ssa / (float)DV + onorm_eps), rsb = rsqrtf(ssb / (float)DV + onorm_eps);
        const T* cG = sG + (size_t)stage * C * VS;
        const T* ga = gate_async ? cG + ra * VS : gbase + (int64_t)la * gate_rs;
        const T* gb = gate_async ? cG + rb * VS : gbase + (int64_t)lb * gate_rs;
#pragma unroll
        for (int nt = 0; nt < HT; ++nt) {
          const int c = c0 + nt * 8 + 2 * tq;
          const float2 w = ld2(&onorm_w[c]);
          if (la < L) {
            const float2 gt = ld2(&ga[c]);
            const float y0 = to_f(from_f<T>(to_f(from_f<T>(acc[nt][0] * rsa)) * w.x));
            const float y1 = to_f(from_f<T>(to_f(from_f<T>(acc[nt][1] * rsa)) * w.y));
            st2(&og[(int64_t)la * st[11] + c], y0 * to_f(from_f<T>(siluf_(gt.x))),
                y1 * to_f(from_f<T>(siluf_(gt.y))));
          }
          if (lb < L) {
            const float2 gt = ld2(&gb[c]);
            const float y0 = to_f(from_f<T>(to_f(from_f<T>(acc[nt][2] * rsb)) * w.x));
            const float y1 = to_f(from_f<T>(to_f(from_f<T>(acc[nt][3] * rsb)) * w.y));
            st2(&og[(int64_t)lb * st[11] + c], y0 * to_f(from_f<T>(siluf_(gt.x))),
                y1 * to_f(from_f<T>(siluf_(gt.y))));
          }
        }
      }
    }
    __syncthreads();  // (5) end of chunk: stages / nS reusable
  }

  if (s_owner) {
    float* so = s_out + (size_t)bh * DK * DV;
#pragma unroll
    for (int nt = 0; nt < HT; ++nt) {
      const int r = sm0 + gq, c = sc0 + nt * 8 + 2 * tq;
      *reinterpret_cast<float2*>(&so[r * DV + c]) = make_float2(Sr[nt][0], Sr[nt][1]);
      *reinterpret_cast<float2*>(&so[(r + 8) * DV + c]) = make_float2(Sr[nt][2], Sr[nt][3]);
    }
  }
}

template <typename T, int DK, int DV, bool PREP = false>
int launch_fast(const void* q, const void* k, const void* v, const float* beta, const float* g, const float* s_in,
                float* s_out, void* o, int64_t B, int64_t H, int64_t L, const Strides18& sv, const void* gate,
                int64_t gate_rs, int64_t gate_hs, const void* onorm_w, float eps, cudaStream_t stream,
                PrepArgs<T> pa = PrepArgs<T>{}) {
  using Lay = FastLayout<T, DK, DV>;
  auto kern = gdn_chunk_fast_kernel<T, DK, DV, PREP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Lay::bytes);
  if (e != cudaSuccess) return set_error(MB_ERR_CUDA, "gdn_chunk_fast: smem attribute: %s", cudaGetErrorString(e));
  kern<<<(unsigned)(B * H), NT, Lay::bytes, stream>>>((const T*)q, (const T*)k, (const T*)v, beta, g, s_in, s_out,
                                                      (T*)o, (int)H, (int)L, sv, (const T*)gate, gate_rs, gate_hs,
                                                      (const T*)onorm_w, eps, pa);
  return check_launch("gdn_chunk_fast");
}

}  // namespace

// Returns 1 (and launches) when a 16-bit fast kernel exists for (Dk, Dv), else 0.
int gdn_chunk_fast_dispatch(int dtype, int64_t Dk, int64_t Dv, const void* q, const void* k, const void* v,
                            const float* beta, const float* g, const float* s_in, float* s_out, void* o, int64_t B,
                            int64_t H, int64_t L, const int64_t* strides, const void* gate, int64_t gate_rs,
                            int64_t gate_hs, const void* onorm_w, float eps, cudaStream_t st, int* rc) {
  Strides18 sv;
  for (int i = 0; i < 18; ++i) sv.s[i] = strides[i];
  // o / gate are written and read as 16-bit pairs
  if (strides[11] % 2 || strides[9] % 2 || strides[10] % 2 || ((uintptr_t)o & 3)) return 0;
  if (gate && (gate_rs % 2 || gate_hs % 2 || ((uintptr_t)gate & 3) || ((uintptr_t)onorm_w & 3))) return 0;
#define MB_FAST_CASE(DK_, DV_)                                                                               \
  if (Dk == DK_ && Dv == DV_) {                                                                              \
    if (dtype == MB_BF16)                                                                                    \
      *rc = launch_fast<__nv_bfloat16, DK_, DV_, false>(q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate, gate_rs, \
                                                 gate_hs, onorm_w, eps, st);                                 \
    else                                                                                                     \
      *rc = launch_fast<__half, DK_, DV_, false>(q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate, gate_rs,      \
                                          gate_hs, onorm_w, eps, st);                                        \
    return 1;                                                                                                \
  }
  if (dtype != MB_BF16 && dtype != MB_F16) return 0;
  MB_FAST_CASE(32, 64)
  MB_FAST_CASE(64, 64)
  MB_FAST_CASE(64, 128)
#undef MB_FAST_CASE
  return 0;
}

template <typename T, int DK, int DV>
int prefill_typed(const void* proj, int64_t ps, const void* conv_w, const void* A_log, const void* dt_bias,
                  const void* conv_in, void* conv_out, const float* s_in, float* s_out, const void* onorm_w, float eps,
                  void* out, int64_t os, int64_t B, int64_t Tn, int64_t H, cudaStream_t st) {
  const T* P = static_cast<const T*>(proj);
  const int64_t C = H * (2 * DK + DV);
  Strides18 sv;
  const int64_t s9[18] = {Tn * ps, DK, ps, Tn * ps, DK, ps, Tn * ps, DV, ps, Tn * os, DV, os, 0, 0, 0, 0, 0, 0};
  for (int i = 0; i < 18; ++i) sv.s[i] = s9[i];
  PrepArgs<T> pa{static_cast<const T*>(conv_w), static_cast<const T*>(A_log), static_cast<const T*>(dt_bias),
                 static_cast<const T*>(conv_in), static_cast<T*>(conv_out), P + C, P + C + H, ps};
  const T* gate = P + C + 2 * H;
  return launch_fast<T, DK, DV, true>(P, P + H * DK, P + 2 * H * DK, nullptr, nullptr, s_in, s_out, out, B, H, Tn,
                                      sv, gate, ps, DV, onorm_w, eps, st, pa);
}

}  // namespace mb

extern "C" int motif_b200_gdn_prefill(const void* proj, int64_t proj_stride, const void* conv_w, const void* A_log,
                                      const void* dt_bias, const void* conv_in, void* conv_out, const float* state_in,
                                      float* state_out, const void* onorm_w, float eps, void* out, int64_t out_stride,
                                      int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int dtype,
                                      void* stream) {
  using namespace mb;
  MB_REQUIRE(proj && conv_w && A_log && dt_bias && state_out && onorm_w && out, MB_ERR_ARG, "gdn_prefill: null pointer");
  MB_REQUIRE(conv_out == nullptr || conv_out != conv_in, MB_ERR_ARG, "gdn_prefill: conv_out must not alias conv_in");
  MB_REQUIRE(B >= 0 && T >= 0 && H > 0 && B * H < (1LL << 31) && T < (1LL << 31), MB_ERR_SHAPE, "gdn_prefill: bad shape");
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "gdn_prefill: 16-bit dtypes only");
  const int64_t C = H * (2 * Dk + Dv);
  // q / k / v columns are staged with 16-byte copies; an unaligned gate column block falls
  // back to direct loads inside the kernel.
  MB_REQUIRE(proj_stride % 8 == 0 && out_stride % 2 == 0 && (uintptr_t)proj % 16 == 0 && (uintptr_t)out % 4 == 0 &&
                 (C + 2 * H) % 2 == 0 && (uintptr_t)onorm_w % 4 == 0,
             MB_ERR_ALIGN, "gdn_prefill: projection rows must be 16-byte aligned");
  if (B == 0 || T == 0) return set_error(MB_ERR_SHAPE, "gdn_prefill: empty input");
  cudaStream_t st = (cudaStream_t)stream;
#define MB_PREFILL_CASE(DK_, DV_)                                                                              \
  if (Dk == DK_ && Dv == DV_)                                                                                  \
    return dtype == MB_BF16                                                                                    \
               ? prefill_typed<__nv_bfloat16, DK_, DV_>(proj, proj_stride, conv_w, A_log, dt_bias, conv_in,    \
                                                        conv_out, state_in, state_out, onorm_w, eps, out,      \
                                                        out_stride, B, T, H, st)                               \
               : prefill_typed<__half, DK_, DV_>(proj, proj_stride, conv_w, A_log, dt_bias, conv_in, conv_out, \
                                                 state_in, state_out, onorm_w, eps, out, out_stride, B, T, H,  \
                                                 st);
  MB_PREFILL_CASE(32, 64)
  MB_PREFILL_CASE(64, 64)
  MB_PREFILL_CASE(64, 128)
#undef MB_PREFILL_CASE
  return set_error(MB_ERR_UNSUPPORTED, "gdn_prefill: (Dk, Dv) = (%lld, %lld) not built", (long long)Dk, (long long)Dv);
}
