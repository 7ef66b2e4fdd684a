// Chunked gated delta rule, fused: one CTA per (batch, head) walks the sequence in chunks
// of C = 64 tokens with the recurrent state S [Dk x Dv] (fp32) resident on chip, so the
// only HBM traffic is q, k, v, beta, g in and o, S out.
//
// Per chunk (motif/ops/gated_deltanet.py:137-177 and :312-319, same factors):
//   gamma = cumsum(g);  D_ij = exp(gamma_i - gamma_j)
//   A  = -(diag(beta) k k^T) . D   (strictly lower)        [bf16 MMA: k k^T is exact]
//   Aq = (q k^T) . D               (lower incl. diagonal)
//   T  = (I - A)^-1                (blocked 16x16 forward substitution, fp32 FMA)
//   W  = T (k . beta e^gamma),  U = T (v . beta)          [TF32 MMA]
//   X  = U - W S
//   o  = (q . e^gamma) S + Aq X
//   S  = e^{gamma_L} S + (k . e^{gamma_L - gamma})^T X
// In fp32 mode every TF32 product is the three-pass split hi*hi + hi*lo + lo*hi (the
// published "3xTF32" error-compensation method), which keeps fp32 accuracy; with 16-bit
// inputs the k k^T / q k^T products run on bf16/fp16 MMAs (exact products) and the rest on
// single-pass TF32.
//
// An optional epilogue applies GatedRMSNorm (rms_norm.py:547-553) to each output row with a
// gate row read from global memory, replacing gdn_attn.py:206-209 (o_norm(cat[o, gate])).
#include <cstdlib>

#include "common.cuh"

namespace mb {

int gdn_chunk_fast_dispatch(int dtype, int64_t Dk, int64_t Dv, const void* q, const void* k, const void* v,
                            const float* beta, const float* g, const float* s_in, float* s_out, void* o, int64_t B,
                            int64_t H, int64_t L, const int64_t* strides, const void* gate, int64_t gate_rs,
                            int64_t gate_hs, const void* onorm_w, float eps, cudaStream_t st, int* rc);
int64_t gdn_split_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv, int dtype);
int gdn_split_dispatch(int dtype, int64_t Dk, int64_t Dv, const void* q, const void* k, const void* v,
                       const float* beta, const float* g, const float* s_in, float* s_out, void* o, int64_t B,
                       int64_t H, int64_t L, const int64_t* strides, const void* gate, int64_t gate_rs,
                       int64_t gate_hs, const void* onorm_w, float eps, void* ws, int64_t ws_bytes, cudaStream_t st,
                       int* rc);

namespace {

constexpr int C = 64;
constexpr int NW = 8;
constexpr int NT = NW * 32;

struct Strides18 {
  int64_t s[18];
};

template <typename T, int DK, int DV>
struct Layout {
  static constexpr bool F32 = sizeof(T) == 4;
  static constexpr int STAGES = F32 ? 1 : 2;
  static constexpr int QS = F32 ? DK + 4 : DK + 8;  // sQ / sK row stride (elements of T)
  static constexpr int VS = DV + 8;                 // sV row stride (elements of T)
  static constexpr int AS = C + 4;                  // sA / sT / sAq row stride (floats)
  static constexpr int WS = DK + 4;                 // sW row stride (floats)
  static constexpr int US = DV + 8;                 // sU / sS row stride (floats)
  static constexpr int OS = DV + 4;                 // sO row stride (floats), overlays sA+sT
  static constexpr size_t q_bytes = (size_t)STAGES * C * QS * sizeof(T);
  static constexpr size_t v_bytes = (size_t)STAGES * C * VS * sizeof(T);
  static constexpr size_t a_bytes = (size_t)C * AS * 4;
  static constexpr size_t off_q = 0;
  static constexpr size_t off_k = off_q + q_bytes;
  static constexpr size_t off_v = off_k + q_bytes;
  static constexpr size_t off_a = off_v + v_bytes;
  static constexpr size_t off_t = off_a + a_bytes;
  static constexpr size_t off_aq = off_t + a_bytes;
  static constexpr size_t off_w = off_aq + a_bytes;
  static constexpr size_t off_u = off_w + (size_t)C * WS * 4;
  static constexpr size_t off_s = off_u + (size_t)C * US * 4;
  static constexpr size_t off_vec = off_s + (size_t)DK * US * 4;  // gamma, e^gamma, e^(gL-g), beta
  static constexpr size_t off_tmp = off_vec + 4 * C * 4;
  static constexpr size_t bytes = off_tmp + 3 * 16 * 16 * 4;
  static_assert((size_t)C * OS * 4 <= 2 * a_bytes, "sO must fit over sA + sT");
  static_assert(bytes <= 232448, "shared memory budget");
};

__device__ __forceinline__ float tf32f(uint32_t u) { return __uint_as_float(u); }

// Split x into TF32 hi / lo parts (lo = 0 unless PRECISE).
template <bool PRECISE>
__device__ __forceinline__ void split(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_rna(x);
  if (PRECISE) lo = tf32_rna(x - tf32f(hi));
}

// acc += A(16x8) B(8x8) with optional 3-pass error compensation.
template <bool PRECISE>
__device__ __forceinline__ void mma3(float* acc, const uint32_t* ah, const uint32_t* al, const uint32_t* bh,
                                     const uint32_t* bl) {
  if (PRECISE) {
    mma_tf32(acc, al, bh);
    mma_tf32(acc, ah, bl);
  }
  mma_tf32(acc, ah, bh);
}

// Generic warp-strip TF32 product: for a 16 x (8*NB) strip at (m0, n0) accumulate
// sum_k A(m, k) B(k, n) over k in [0, kmax) (kmax multiple of 8) into acc[NB][4].
// fa(m, k) / fb(k, n) return fp32 operand values.
template <bool PRECISE, int NB, typename FA, typename FB>
__device__ __forceinline__ void strip_tf32(float (*acc)[4], int m0, int n0, int kmax, FA fa, FB fb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  for (int k0 = 0; k0 < kmax; k0 += 8) {
    uint32_t ah[4], al[4];
    split<PRECISE>(fa(m0 + g, k0 + t), ah[0], al[0]);
    split<PRECISE>(fa(m0 + g + 8, k0 + t), ah[1], al[1]);
    split<PRECISE>(fa(m0 + g, k0 + t + 4), ah[2], al[2]);
    split<PRECISE>(fa(m0 + g + 8, k0 + t + 4), ah[3], al[3]);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      uint32_t bh[2], bl[2];
      const int n = n0 + nb * 8 + g;
      split<PRECISE>(fb(k0 + t, n), bh[0], bl[0]);
      split<PRECISE>(fb(k0 + t + 4, n), bh[1], bl[1]);
      mma3<PRECISE>(acc[nb], ah, al, bh, bl);
    }
  }
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(NT, 1) gdn_chunk_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const float* __restrict__ beta, const float* __restrict__ g, const float* __restrict__ s_in,
    float* __restrict__ s_out, T* __restrict__ o, int H, int L, Strides18 sv,
    const T* __restrict__ gate, int64_t gate_rs, int64_t gate_hs, const T* __restrict__ onorm_w,
    float onorm_eps) {
  using Lay = Layout<T, DK, DV>;
  constexpr bool PRECISE = Lay::F32;
  constexpr int QS = Lay::QS, VS = Lay::VS, AS = Lay::AS, WS = Lay::WS, US = Lay::US, OS = Lay::OS;
  extern __shared__ __align__(16) unsigned char smem[];
  T* sQ = reinterpret_cast<T*>(smem + Lay::off_q);
  T* sK = reinterpret_cast<T*>(smem + Lay::off_k);
  T* sV = reinterpret_cast<T*>(smem + Lay::off_v);
  float* sA = reinterpret_cast<float*>(smem + Lay::off_a);
  float* sT = reinterpret_cast<float*>(smem + Lay::off_t);
  float* sO = sA;  // overlays sA + sT once both are dead
  float* sAq = reinterpret_cast<float*>(smem + Lay::off_aq);
  float* sW = reinterpret_cast<float*>(smem + Lay::off_w);
  float* sU = reinterpret_cast<float*>(smem + Lay::off_u);
  float* sS = reinterpret_cast<float*>(smem + Lay::off_s);
  float* sGam = reinterpret_cast<float*>(smem + Lay::off_vec);
  float* sEg = sGam + C;
  float* sDl = sEg + C;
  float* sBeta = sDl + C;
  float* sTmp = reinterpret_cast<float*>(smem + Lay::off_tmp);

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

  // ---- state S: registers in MMA accumulator layout (strips of 16 x 32), mirrored in sS
  constexpr int SNB = DV >= 32 ? 4 : DV / 8;
  constexpr int S_STRIPS = (DK / 16) * (DV / (8 * SNB));
  constexpr int S_PER_WARP = (S_STRIPS + NW - 1) / NW;
  float Sr[S_PER_WARP][SNB][4];
  const float* s0 = s_in ? s_in + (size_t)bh * DK * DV : nullptr;
#pragma unroll
  for (int i = 0; i < S_PER_WARP; ++i) {
    const int s = warp + NW * i;
    if (s < S_STRIPS) {
      const int m0 = (s / (DV / (8 * SNB))) * 16, n0 = (s % (DV / (8 * SNB))) * 8 * SNB;
#pragma unroll
      for (int nb = 0; nb < SNB; ++nb) {
        const int r = m0 + gq, c = n0 + nb * 8 + 2 * tq;
        Sr[i][nb][0] = s0 ? s0[r * DV + c] : 0.f;
        Sr[i][nb][1] = s0 ? s0[r * DV + c + 1] : 0.f;
        Sr[i][nb][2] = s0 ? s0[(r + 8) * DV + c] : 0.f;
        Sr[i][nb][3] = s0 ? s0[(r + 8) * DV + c + 1] : 0.f;
        *reinterpret_cast<float2*>(&sS[r * US + c]) = make_float2(Sr[i][nb][0], Sr[i][nb][1]);
        *reinterpret_cast<float2*>(&sS[(r + 8) * US + c]) = make_float2(Sr[i][nb][2], Sr[i][nb][3]);
      }
    }
  }

  // ---- asynchronous chunk loads (q, k, v rows; rows past L are zero-filled)
  auto load_chunk = [&](int n, int stage) {
    constexpr int QV = DK * (int)sizeof(T) / 16, VV = DV * (int)sizeof(T) / 16;  // 16B vectors per row
    T* dq = sQ + (size_t)stage * C * QS;
    T* dk = sK + (size_t)stage * C * QS;
    T* dv = sV + (size_t)stage * C * VS;
    for (int i = tid; i < C * (2 * QV + VV); i += NT) {
      const int r = i / (2 * QV + VV), c = i % (2 * QV + VV);
      const int l = n * C + r;
      const bool ok = l < L;
      const int64_t lc = ok ? l : 0;
      if (c < QV) {
        cp_async16(dq + r * QS + c * (16 / sizeof(T)), qg + lc * st[2] + c * (16 / sizeof(T)), ok);
      } else if (c < 2 * QV) {
        const int cc = c - QV;
        cp_async16(dk + r * QS + cc * (16 / sizeof(T)), kg + lc * st[5] + cc * (16 / sizeof(T)), ok);
      } else {
        const int cc = c - 2 * QV;
        cp_async16(dv + r * VS + cc * (16 / sizeof(T)), vg + lc * st[8] + cc * (16 / sizeof(T)), ok);
      }
    }
    cp_async_commit();
  };
  // g / beta for the next chunk are prefetched into registers by warp 0 (2 per lane).
  float pg[2], pb[2];
  auto fetch_gb = [&](int n) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int l = n * C + lane + 32 * e;
      const bool ok = l < L;
      pg[e] = ok ? gg[(int64_t)l * st[17]] : 0.f;
      pb[e] = ok ? bg[(int64_t)l * st[14]] : 0.f;
    }
  };

  if (nchunks > 0) {
    load_chunk(0, 0);
    if (warp == 0) fetch_gb(0);
  }

  for (int n = 0; n < nchunks; ++n) {
    const int stage = Lay::STAGES == 2 ? (n & 1) : 0;
    if (Lay::STAGES == 2) {
      // The other stage was last read in iteration n-1, which ended with __syncthreads().
      if (n + 1 < nchunks) {
        load_chunk(n + 1, stage ^ 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
    } else {
      if (n > 0) load_chunk(n, 0);
      cp_async_wait<0>();
    }
    const T* cQ = sQ + (size_t)stage * C * QS;
    const T* cK = sK + (size_t)stage * C * QS;
    const T* cV = sV + (size_t)stage * C * VS;

    // (a) gamma = inclusive cumsum of g; e^gamma, e^(gL - gamma), beta  (warp 0)
    if (warp == 0) {
      float x0 = pg[0], x1 = pg[1];
      float b0 = pb[0], b1 = pb[1];
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
      sBeta[lane] = b0;
      sBeta[lane + 32] = b1;
      if (n + 1 < nchunks) fetch_gb(n + 1);
    }
    __syncthreads();
    const float eL = sEg[C - 1];

    // (b) KK = k k^T -> A (strict lower, scaled), QK = q k^T -> Aq (lower)
    {
      const int prod = warp >> 2;  // 0: KK, 1: QK
      const int m0 = (warp & 3) * 16;
      const T* left = prod == 0 ? cK : cQ;
      float acc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
      if constexpr (!PRECISE) {
        const uint32_t* Lw = reinterpret_cast<const uint32_t*>(left);
        const uint32_t* Kw = reinterpret_cast<const uint32_t*>(cK);
        constexpr int QW = QS / 2;
#pragma unroll
        for (int k0 = 0; k0 < DK; k0 += 16) {
          uint32_t a[4];
          a[0] = Lw[(m0 + gq) * QW + k0 / 2 + tq];
          a[1] = Lw[(m0 + gq + 8) * QW + k0 / 2 + tq];
          a[2] = Lw[(m0 + gq) * QW + k0 / 2 + 4 + tq];
          a[3] = Lw[(m0 + gq + 8) * QW + k0 / 2 + 4 + tq];
#pragma unroll
          for (int nb = 0; nb < 8; ++nb) {
            uint32_t bb[2];
            bb[0] = Kw[(nb * 8 + gq) * QW + k0 / 2 + tq];
            bb[1] = Kw[(nb * 8 + gq) * QW + k0 / 2 + 4 + tq];
            mma_16816<T>(acc[nb], a, bb);
          }
        }
      } else {
        strip_tf32<true, 8>(acc, m0, 0, DK,
                            [&](int m, int kk) { return to_f(left[m * QS + kk]); },
                            [&](int kk, int nn) { return to_f(cK[nn * QS + kk]); });
      }
      float* dst = prod == 0 ? sA : sAq;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = m0 + gq + (e >= 2 ? 8 : 0);
          const int j = nb * 8 + 2 * tq + (e & 1);
          const float d = expf(sGam[i] - sGam[j]);
          float val;
          if (prod == 0)
            val = j < i ? -sBeta[i] * acc[nb][e] * d : 0.f;
          else
            val = j <= i ? acc[nb][e] * d : 0.f;
          dst[i * AS + j] = val;
        }
      }
    }
    __syncthreads();

    // (c) T = (I - A)^-1: 16x16 diagonal blocks by forward substitution (warps 0-3) ...
    if (warp < 4 && lane < 16) {
      const int base = warp * 16;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float acc = (r == lane) ? 1.f : 0.f;
#pragma unroll
        for (int j = 0; j < r; ++j) acc = fmaf(sA[(base + r) * AS + base + j], col[j], acc);
        col[r] = acc;
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) sT[(base + r) * AS + base + lane] = col[r];
    }
    __syncthreads();
    // ... then block rows bi = 1..3: T_{bi,bj} = T_{bi,bi} * sum_{kb=bj}^{bi-1} A_{bi,kb} T_{kb,bj}
    for (int bi = 1; bi < 4; ++bi) {
      for (int e = tid; e < bi * 256; e += NT) {
        const int bj = e >> 8, r = (e >> 4) & 15, c = e & 15;
        float acc = 0.f;
        for (int kb = bj; kb < bi; ++kb) {
#pragma unroll
          for (int x = 0; x < 16; ++x)
            acc = fmaf(sA[(bi * 16 + r) * AS + kb * 16 + x], sT[(kb * 16 + x) * AS + bj * 16 + c], acc);
        }
        sTmp[e] = acc;
      }
      __syncthreads();
      for (int e = tid; e < bi * 256; e += NT) {
        const int bj = e >> 8, r = (e >> 4) & 15, c = e & 15;
        float acc = 0.f;
#pragma unroll
        for (int x = 0; x < 16; ++x) acc = fmaf(sT[(bi * 16 + r) * AS + bi * 16 + x], sTmp[bj * 256 + x * 16 + c], acc);
        sT[(bi * 16 + r) * AS + bj * 16 + c] = acc;
      }
      __syncthreads();
    }

    // (d) [W | U] = T [k.beta e^gamma | v.beta]   (T lower triangular: k < 16 (mt + 1))
    {
      constexpr int SW = DK < 32 ? DK : 32;
      constexpr int NBW = SW / 8;
      constexpr int NSTRIP = 4 * ((DK + DV) / SW);
      for (int s = warp; s < NSTRIP; s += NW) {
        const int mt = s / ((DK + DV) / SW);
        const int n0 = (s % ((DK + DV) / SW)) * SW;
        float acc[NBW][4];
#pragma unroll
        for (int i = 0; i < NBW; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        auto fa = [&](int m, int kk) { return sT[m * AS + kk]; };
        if (n0 < DK) {
          strip_tf32<PRECISE, NBW>(acc, mt * 16, n0, 16 * (mt + 1), fa,
                                   [&](int kk, int nn) { return to_f(cK[kk * QS + nn]) * (sBeta[kk] * sEg[kk]); });
#pragma unroll
          for (int nb = 0; nb < NBW; ++nb) {
            const int r = mt * 16 + gq, c = n0 + nb * 8 + 2 * tq;
            *reinterpret_cast<float2*>(&sW[r * WS + c]) = make_float2(acc[nb][0], acc[nb][1]);
            *reinterpret_cast<float2*>(&sW[(r + 8) * WS + c]) = make_float2(acc[nb][2], acc[nb][3]);
          }
        } else {
          strip_tf32<PRECISE, NBW>(acc, mt * 16, n0 - DK, 16 * (mt + 1), fa,
                                   [&](int kk, int nn) { return to_f(cV[kk * VS + nn]) * sBeta[kk]; });
#pragma unroll
          for (int nb = 0; nb < NBW; ++nb) {
            const int r = mt * 16 + gq, c = n0 - DK + nb * 8 + 2 * tq;
            *reinterpret_cast<float2*>(&sU[r * US + c]) = make_float2(acc[nb][0], acc[nb][1]);
            *reinterpret_cast<float2*>(&sU[(r + 8) * US + c]) = make_float2(acc[nb][2], acc[nb][3]);
          }
        }
      }
    }
    __syncthreads();

    // (e) X = U - W S   (in place over U)
    {
      constexpr int NSTRIP = 4 * (DV / (8 * SNB));
      for (int s = warp; s < NSTRIP; s += NW) {
        const int m0 = (s / (DV / (8 * SNB))) * 16, n0 = (s % (DV / (8 * SNB))) * 8 * SNB;
        float acc[SNB][4];
#pragma unroll
        for (int i = 0; i < SNB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        strip_tf32<PRECISE, SNB>(acc, m0, n0, DK, [&](int m, int kk) { return sW[m * WS + kk]; },
                                 [&](int kk, int nn) { return sS[kk * US + nn]; });
#pragma unroll
        for (int nb = 0; nb < SNB; ++nb) {
          const int r = m0 + gq, c = n0 + nb * 8 + 2 * tq;
          float2* p0 = reinterpret_cast<float2*>(&sU[r * US + c]);
          float2* p1 = reinterpret_cast<float2*>(&sU[(r + 8) * US + c]);
          const float2 u0 = *p0, u1 = *p1;
          *p0 = make_float2(u0.x - acc[nb][0], u0.y - acc[nb][1]);
          *p1 = make_float2(u1.x - acc[nb][2], u1.y - acc[nb][3]);
        }
      }
    }
    __syncthreads();

    // (f) o = (q . e^gamma) S + Aq X  -> sO;   S = e^gL S + (k . e^(gL-gamma))^T X -> registers
    {
      constexpr int NSTRIP = 4 * (DV / (8 * SNB));
      for (int s = warp; s < NSTRIP; s += NW) {
        const int m0 = (s / (DV / (8 * SNB))) * 16, n0 = (s % (DV / (8 * SNB))) * 8 * SNB;
        float acc[SNB][4];
#pragma unroll
        for (int i = 0; i < SNB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        strip_tf32<PRECISE, SNB>(acc, m0, n0, DK, [&](int m, int kk) { return to_f(cQ[m * QS + kk]) * sEg[m]; },
                                 [&](int kk, int nn) { return sS[kk * US + nn]; });
        strip_tf32<PRECISE, SNB>(acc, m0, n0, m0 + 16, [&](int m, int kk) { return sAq[m * AS + kk]; },
                                 [&](int kk, int nn) { return sU[kk * US + nn]; });
#pragma unroll
        for (int nb = 0; nb < SNB; ++nb) {
          const int r = m0 + gq, c = n0 + nb * 8 + 2 * tq;
          *reinterpret_cast<float2*>(&sO[r * OS + c]) = make_float2(acc[nb][0], acc[nb][1]);
          *reinterpret_cast<float2*>(&sO[(r + 8) * OS + c]) = make_float2(acc[nb][2], acc[nb][3]);
        }
      }
#pragma unroll
      for (int i = 0; i < S_PER_WARP; ++i) {
        const int s = warp + NW * i;
        if (s < S_STRIPS) {
          const int m0 = (s / (DV / (8 * SNB))) * 16, n0 = (s % (DV / (8 * SNB))) * 8 * SNB;
#pragma unroll
          for (int nb = 0; nb < SNB; ++nb)
#pragma unroll
            for (int e = 0; e < 4; ++e) Sr[i][nb][e] *= eL;
          strip_tf32<PRECISE, SNB>(Sr[i], m0, n0, C,
                                   [&](int m, int kk) { return to_f(cK[kk * QS + m]) * sDl[kk]; },
                                   [&](int kk, int nn) { return sU[kk * US + nn]; });
        }
      }
    }
    __syncthreads();

    // (g) publish the new state;  (h) write the chunk's outputs
#pragma unroll
    for (int i = 0; i < S_PER_WARP; ++i) {
      const int s = warp + NW * i;
      if (s < S_STRIPS) {
        const int m0 = (s / (DV / (8 * SNB))) * 16, n0 = (s % (DV / (8 * SNB))) * 8 * SNB;
#pragma unroll
        for (int nb = 0; nb < SNB; ++nb) {
          const int r = m0 + gq, c = n0 + nb * 8 + 2 * tq;
          *reinterpret_cast<float2*>(&sS[r * US + c]) = make_float2(Sr[i][nb][0], Sr[i][nb][1]);
          *reinterpret_cast<float2*>(&sS[(r + 8) * US + c]) = make_float2(Sr[i][nb][2], Sr[i][nb][3]);
        }
      }
    }
    for (int r = warp; r < C; r += NW) {
      const int l = n * C + r;
      if (l >= L) break;
      T* orow = og + (int64_t)l * st[11];
      if (gate == nullptr) {
        for (int c = lane; c < DV; c += 32) orow[c] = from_f<T>(sO[r * OS + c]);
      } else {
        // GatedRMSNorm over the Dv outputs of this head, after the reference's o.to(dtype).
        float ss = 0.f;
        for (int c = lane; c < DV; c += 32) {
          const float x = to_f(from_f<T>(sO[r * OS + c]));
          ss += x * x;
        }
        ss = warp_sum(ss);
        const float rs = rsqrtf(ss / (float)DV + onorm_eps);
        // gate rows are token-major: row (b * L + l), head h at column offset h * gate_hs
        const T* grow = gate + ((int64_t)b * L + l) * gate_rs + h * gate_hs;
        for (int c = lane; c < DV; c += 32) {
          const float x = to_f(from_f<T>(sO[r * OS + c]));
          float y = to_f(from_f<T>(x * rs));
          y = to_f(from_f<T>(y * to_f(onorm_w[c])));
          orow[c] = from_f<T>(y * to_f(from_f<T>(siluf_(to_f(grow[c])))));
        }
      }
    }
    __syncthreads();
  }

  // final state
  float* so = s_out + (size_t)bh * DK * DV;
#pragma unroll
  for (int i = 0; i < S_PER_WARP; ++i) {
    const int s = warp + NW * i;
    if (s < S_STRIPS) {
      const int m0 = (s / (DV / (8 * SNB))) * 16, n0 = (s % (DV / (8 * SNB))) * 8 * SNB;
#pragma unroll
      for (int nb = 0; nb < SNB; ++nb) {
        const int r = m0 + gq, c = n0 + nb * 8 + 2 * tq;
        so[r * DV + c] = Sr[i][nb][0];
        so[r * DV + c + 1] = Sr[i][nb][1];
        so[(r + 8) * DV + c] = Sr[i][nb][2];
        so[(r + 8) * DV + c + 1] = Sr[i][nb][3];
      }
    }
  }
}

template <typename T, int DK, int DV>
int launch(const void* q, const void* k, const void* v, const float* beta, const float* g, const float* s_in,
           float* s_out, void* o, int64_t B, int64_t H, int64_t L, const Strides18& sv, const void* gate,
           int64_t gate_rs, int64_t gate_hs, const void* onorm_w, float eps, cudaStream_t stream) {
  using Lay = Layout<T, DK, DV>;
  auto kern = gdn_chunk_kernel<T, DK, DV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Lay::bytes);
  if (e != cudaSuccess) return set_error(MB_ERR_CUDA, "gdn_chunk: smem attribute: %s", cudaGetErrorString(e));
  kern<<<(unsigned)(B * H), NT, Lay::bytes, stream>>>((const T*)q, (const T*)k, (const T*)v, beta, g, s_in, s_out,
                                                      (T*)o, (int)H, (int)L, sv, (const T*)gate, gate_rs, gate_hs,
                                                      (const T*)onorm_w, eps);
  return check_launch("gdn_chunk");
}

template <typename T>
int launch_dims(int64_t Dk, int64_t Dv, const void* q, const void* k, const void* v, const float* beta,
                const float* g, const float* s_in, float* s_out, void* o, int64_t B, int64_t H, int64_t L,
                const Strides18& sv, const void* gate, int64_t gate_rs, int64_t gate_hs, const void* onorm_w,
                float eps, cudaStream_t st) {
#define MB_GDN_CASE(DK_, DV_)                                                                          \
  if (Dk == DK_ && Dv == DV_)                                                                           \
    return launch<T, DK_, DV_>(q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate, gate_rs, gate_hs, \
                               onorm_w, eps, st);
  MB_GDN_CASE(16, 32)
  MB_GDN_CASE(16, 64)
  MB_GDN_CASE(32, 32)
  MB_GDN_CASE(32, 64)
  MB_GDN_CASE(32, 128)
  MB_GDN_CASE(64, 64)
  MB_GDN_CASE(64, 128)
#undef MB_GDN_CASE
  return set_error(MB_ERR_UNSUPPORTED, "gdn_chunk: (Dk, Dv) = (%lld, %lld) not built", (long long)Dk,
                   (long long)Dv);
}

// Testing knobs: MB_FORCE_GDN_PRECISE routes 16-bit inputs through the 3xTF32 kernel;
// MB_FORCE_GDN_FUSED keeps 16-bit calls that bring a workspace on the single fused kernel (the
// two-kernel split is the default when a workspace is given).  Tests cross-check with them.
bool force_precise() { return forced(MB_FORCE_GDN_PRECISE); }
bool force_fused() { return forced(MB_FORCE_GDN_FUSED); }

int gdn_chunk_impl(const void* q, const void* k, const void* v, const float* beta, const float* g,
                   const float* s_in, float* s_out, void* o, int64_t B, int64_t H, int64_t L, int64_t Dk,
                   int64_t Dv, const int64_t* strides, int dtype, const void* gate, int64_t gate_rs,
                   int64_t gate_hs, const void* onorm_w, float eps, void* stream, void* ws = nullptr,
                   int64_t ws_bytes = 0) {
  MB_REQUIRE(s_out && strides, MB_ERR_ARG, "gdn_chunk: null state_out/strides");
  MB_REQUIRE(L == 0 || (q && k && v && beta && g && o), MB_ERR_ARG, "gdn_chunk: null input");
  MB_REQUIRE(B >= 0 && H > 0 && L >= 0 && L < (1LL << 31) && B * H < (1LL << 31), MB_ERR_SHAPE,
             "gdn_chunk: bad shape");
  const int es = dtype == MB_F32 ? 4 : 2;
  const int vec = 16 / es;
  for (int i = 0; i < 9; ++i)
    MB_REQUIRE(strides[i] % vec == 0, MB_ERR_ALIGN, "gdn_chunk: q/k/v strides must be multiples of %d elements",
               vec);
  MB_REQUIRE(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0, MB_ERR_ALIGN,
             "gdn_chunk: q/k/v must be 16-byte aligned");
  if (B == 0) return MB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = MB_OK;
  if (!force_precise() && !force_fused() && ws &&
      gdn_split_dispatch(dtype, Dk, Dv, q, k, v, beta, g, s_in, s_out, o, B, H, L, strides, gate, gate_rs, gate_hs,
                         onorm_w, eps, ws, ws_bytes, st, &rc))
    return rc;
  if (!force_precise() && gdn_chunk_fast_dispatch(dtype, Dk, Dv, q, k, v, beta, g, s_in, s_out, o, B, H, L, strides,
                                                  gate, gate_rs, gate_hs, onorm_w, eps, st, &rc))
    return rc;
  Strides18 sv;
  for (int i = 0; i < 18; ++i) sv.s[i] = strides[i];
  switch (dtype) {
    case MB_F32:
      return launch_dims<float>(Dk, Dv, q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate, gate_rs, gate_hs,
                                onorm_w, eps, st);
    case MB_BF16:
      return launch_dims<__nv_bfloat16>(Dk, Dv, q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate, gate_rs,
                                        gate_hs, onorm_w, eps, st);
    case MB_F16:
      return launch_dims<__half>(Dk, Dv, q, k, v, beta, g, s_in, s_out, o, B, H, L, sv, gate, gate_rs, gate_hs,
                                 onorm_w, eps, st);
    default:
      return set_error(MB_ERR_DTYPE, "gdn_chunk: dtype %d", dtype);
  }
}

}  // namespace
}  // namespace mb

extern "C" int motif_b200_gdn_chunk(const void* q, const void* k, const void* v, const float* beta,
                                    const float* g, const float* state_in, float* state_out, void* o, int64_t B,
                                    int64_t H, int64_t L, int64_t Dk, int64_t Dv, const int64_t* strides,
                                    int dtype, void* stream) {
  return mb::gdn_chunk_impl(q, k, v, beta, g, state_in, state_out, o, B, H, L, Dk, Dv, strides, dtype, nullptr, 0,
                            0, nullptr, 0.f, stream);
}

extern "C" int motif_b200_gdn_chunk_gated(const void* q, const void* k, const void* v, const float* beta,
                                          const float* g, const float* state_in, float* state_out, void* o,
                                          int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                                          const int64_t* strides, const void* gate, int64_t gate_row_stride,
                                          int64_t gate_head_stride, const void* onorm_w, float eps, int dtype,
                                          void* stream) {
  MB_REQUIRE(gate && onorm_w, MB_ERR_ARG, "gdn_chunk_gated: null gate / weight");
  return mb::gdn_chunk_impl(q, k, v, beta, g, state_in, state_out, o, B, H, L, Dk, Dv, strides, dtype, gate,
                            gate_row_stride, gate_head_stride, onorm_w, eps, stream);
}

extern "C" int64_t motif_b200_gdn_chunk_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                                                        int dtype) {
  if (B < 0 || H <= 0 || L < 0) return 0;
  return mb::gdn_split_workspace_bytes(B, H, L, Dk, Dv, dtype);
}

extern "C" int motif_b200_gdn_chunk_gated_ws(const void* q, const void* k, const void* v, const float* beta,
                                             const float* g, const float* state_in, float* state_out, void* o,
                                             int64_t B, int64_t H, int64_t L, int64_t Dk, int64_t Dv,
                                             const int64_t* strides, const void* gate, int64_t gate_row_stride,
                                             int64_t gate_head_stride, const void* onorm_w, float eps, int dtype,
                                             void* workspace, int64_t workspace_bytes, void* stream) {
  MB_REQUIRE(gate == nullptr || onorm_w != nullptr, MB_ERR_ARG, "gdn_chunk_gated_ws: gate without weight");
  MB_REQUIRE(workspace == nullptr ||
                 workspace_bytes >= mb::gdn_split_workspace_bytes(B, H, L, Dk, Dv, dtype),
             MB_ERR_ARG, "gdn_chunk_gated_ws: workspace too small");
  return mb::gdn_chunk_impl(q, k, v, beta, g, state_in, state_out, o, B, H, L, Dk, Dv, strides, dtype, gate,
                            gate_row_stride, gate_head_stride, onorm_w, eps, stream, workspace, workspace_bytes);
}
