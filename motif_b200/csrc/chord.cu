// Chord attention: causal softmax attention with the gated geometric-decay (GGD) bias
//   logit(i, j) = (q_i . k_j * scale - alpha_h (|j - (q_start + i) - mu_h| + eps)^beta_h)
//                 * ssmax_h * log_n[b, i],     visible iff j <= q_start + i
// (motif/ops/chord_attention.py:145-244 and the eager body of chord_attn.py:316-361).
//
// Kernels:
//   * chord_fwd_mma   — prefill / long-query flash kernel on bf16/fp16 mma.sync.  A CTA owns a
//     kv head and G of its query heads, so each K/V tile staged in shared memory serves G
//     heads (the reference re-reads K/V once per query head).  The bias depends on (head,
//     distance) only, so each warp tabulates it per K/V tile for the (BMQ + 63) distances the
//     tile spans instead of evaluating pow() per score.
//   * chord_fwd_simple — fp32 (and any-shape fallback) kernel: one warp per query row, lanes
//     over keys, online softmax; used for fp32 parity runs.
//   * chord_decode + chord_merge — split-KV decoding for few new tokens over a long cache,
//     with the cache length read from device memory (so a captured CUDA graph replays at any
//     position); one warp per (b, kv head, split) serves all G query heads of the group.
//   * chord_prep — per-head RMSNorm of q and k and the append of k, v into the cache.
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace mb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

// Count of Chord attention CTAs whose bounded copy / MMA wait ran out (never expected; read
// and cleared by motif_b200_wait_timeouts).
__device__ unsigned int g_wait_timeouts = 0;

struct Strides14 {
  int64_t s[14];  // q(b,h,l) k(b,h,s) v(b,h,s) out(b,h,l) log_n(b,l)
};

__device__ __forceinline__ float ggd_bias(float alpha, float beta, float mu, float delta, float eps) {
  // -alpha * (|d - mu| + eps)^beta with d = key - query = -delta
  return -alpha * powf(fabsf(-delta - mu) + eps, beta);
}

// GGD bias in the tensor-core kernels: 16-bit inputs use exp2(beta * log2(x)) on the fast log2 (the
// result's relative error, a few 1e-7, is far below bf16 / fp16 resolution); fp32 keeps powf.
template <typename T>
__device__ __forceinline__ float ggd_bias_decode(float alpha, float beta, float mu, float delta, float eps) {
  if constexpr (sizeof(T) == 2) {
    return -alpha * ex2f_(beta * __log2f(fabsf(-delta - mu) + eps));
  } else {
    return ggd_bias(alpha, beta, mu, delta, eps);
  }
}

// ------------------------------------------------------------------ tensor-core prefill
template <typename T, int D, int G>
__global__ void __launch_bounds__(128) chord_fwd_mma_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ alpha,
    const float* __restrict__ beta, const float* __restrict__ mu, const float* __restrict__ ssmax,
    const float* __restrict__ log_n, T* __restrict__ out, int H, int Hkv, int L, int S, int q_start, float scale,
    float eps, Strides14 sv) {
  constexpr int BMQ = 64 / G;  // query positions per CTA
  constexpr int BN = 64;       // keys per tile
  constexpr int DS = D + 8;    // smem row stride (elements)
  constexpr int DW = DS / 2;   // in 32-bit words
  constexpr int TBL = 80;      // bias table entries per head slot (>= 16 + 63)
  __shared__ __align__(16) T sQ[64 * DS];
  __shared__ __align__(16) T sK[2][BN * DS];
  __shared__ __align__(16) T sV[2][BN * DS];
  __shared__ float sBias[4][2 * TBL];

  const int64_t* st = sv.s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int GS = H / Hkv;
  const int groups_per_kv = GS / G;
  const int kvh = blockIdx.y / groups_per_kv;
  const int h0 = kvh * GS + (blockIdx.y % groups_per_kv) * G;
  const int b = blockIdx.z;
  const int m0q = blockIdx.x * BMQ;

  const T* kb = k + b * st[3] + kvh * st[4];
  const T* vb = v + b * st[6] + kvh * st[7];

  // rows of this CTA: r -> (head h0 + r / BMQ, position m0q + r % BMQ)
  auto load_q = [&]() {
    constexpr int VPR = D / 8;  // 16-byte vectors per row
    for (int i = tid; i < 64 * VPR; i += 128) {
      const int r = i / VPR, c = i % VPR;
      const int hh = h0 + r / BMQ, pos = m0q + r % BMQ;
      const bool ok = pos < L;
      const T* src = q + b * st[0] + hh * st[1] + (int64_t)(ok ? pos : 0) * st[2] + c * 8;
      cp_async16(&sQ[r * DS + c * 8], src, ok);
    }
  };
  auto load_kv = [&](int tile, int stage) {
    constexpr int VPR = D / 8;
    const int k0 = tile * BN;
    for (int i = tid; i < BN * VPR; i += 128) {
      const int r = i / VPR, c = i % VPR;
      const int key = k0 + r;
      const bool ok = key < S;
      const int64_t kk = ok ? key : 0;
      cp_async16(&sK[stage][r * DS + c * 8], kb + kk * st[5] + c * 8, ok);
      cp_async16(&sV[stage][r * DS + c * 8], vb + kk * st[8] + c * 8, ok);
    }
  };

  const int last_pos = min(L, m0q + BMQ) - 1;
  const int kv_end = min(S, q_start + last_pos + 1);  // keys [0, kv_end) are visible to some row
  const int ntiles = (kv_end + BN - 1) / BN;

  load_q();
  if (ntiles > 0) load_kv(0, 0);
  cp_async_commit();

  // per-row constants for rows g8 and g8 + 8 of this warp
  int rpos[2], rslot[2];
  float rc[2], ral[2], rbe[2], rmu[2];
  const int wr0 = warp * 16;
  const int wpos0 = m0q + (wr0 % BMQ);  // smallest position among this warp's rows
  const int whead0 = h0 + wr0 / BMQ;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int r = wr0 + g8 + 8 * e;
    const int hh = h0 + r / BMQ;
    rpos[e] = m0q + r % BMQ;
    rslot[e] = hh - whead0;  // 0 or 1 (two heads per warp only when G == 8)
    const float ln = rpos[e] < L ? log_n[b * st[12] + (int64_t)rpos[e] * st[13]] : 0.f;
    rc[e] = ssmax[hh] * ln * kLog2e;
    ral[e] = alpha[hh];
    rbe[e] = beta[hh];
    rmu[e] = mu[hh];
  }
  const int nslots = (G == 8) ? 2 : 1;

  float o_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  uint32_t qa[D / 16][4];

  for (int tile = 0; tile < ntiles; ++tile) {
    const int stage = tile & 1;
    if (tile + 1 < ntiles) load_kv(tile + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (tile == 0) {
      const uint32_t* Qw = reinterpret_cast<const uint32_t*>(sQ);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        qa[kk][0] = Qw[(wr0 + g8) * DW + kk * 8 + t4];
        qa[kk][1] = Qw[(wr0 + g8 + 8) * DW + kk * 8 + t4];
        qa[kk][2] = Qw[(wr0 + g8) * DW + kk * 8 + 4 + t4];
        qa[kk][3] = Qw[(wr0 + g8 + 8) * DW + kk * 8 + 4 + t4];
      }
    }
    const int k0 = tile * BN;
    // bias table for this warp: slot s, entry e <-> delta = q_start + wpos0 - k0 + e - 63
    for (int e = lane; e < nslots * TBL; e += 32) {
      const int slot = e / TBL, ee = e % TBL;
      const int hh = whead0 + slot;
      const float delta = (float)(q_start + wpos0 - k0 + ee - 63);
      sBias[warp][e] = ggd_bias(alpha[hh], beta[hh], mu[hh], delta, eps);
    }
    __syncwarp();

    // S = Q K^T (16 x 64 per warp)
    float s_acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s_acc[i][0] = s_acc[i][1] = s_acc[i][2] = s_acc[i][3] = 0.f;
    const uint32_t* Kw = reinterpret_cast<const uint32_t*>(sK[stage]);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        uint32_t bb[2];
        bb[0] = Kw[(nt * 8 + g8) * DW + kk * 8 + t4];
        bb[1] = Kw[(nt * 8 + g8) * DW + kk * 8 + 4 + t4];
        mma_16816<T>(s_acc[nt], qa[kk], bb);
      }
    }
    // logits (log2 units), masking, online softmax
    const bool need_mask = (k0 + BN > S) || (k0 + BN - 1 > q_start + wpos0);
    float rmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ri = e >> 1;
        const int kl = nt * 8 + 2 * t4 + (e & 1);  // key offset in tile
        const int tb = rslot[ri] * TBL + (rpos[ri] - wpos0) + 63 - kl;
        float x = (s_acc[nt][e] * scale + sBias[warp][tb]) * rc[ri];
        if (need_mask) {
          const int key = k0 + kl;
          if (key >= S || key > q_start + rpos[ri]) x = -INFINITY;
        }
        s_acc[nt][e] = x;
        rmax[ri] = fmaxf(rmax[ri], x);
      }
    }
    float corr[2], mbase[2];
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      rmax[ri] = fmaxf(rmax[ri], __shfl_xor_sync(0xffffffffu, rmax[ri], 1));
      rmax[ri] = fmaxf(rmax[ri], __shfl_xor_sync(0xffffffffu, rmax[ri], 2));
      const float mn = fmaxf(m_run[ri], rmax[ri]);
      mbase[ri] = mn == -INFINITY ? 0.f : mn;
      corr[ri] = exp2f(m_run[ri] - mbase[ri]);
      m_run[ri] = mn;
      l_run[ri] *= corr[ri];
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o_acc[i][0] *= corr[0];
      o_acc[i][1] *= corr[0];
      o_acc[i][2] *= corr[1];
      o_acc[i][3] *= corr[1];
    }
    uint32_t pa[4][4];  // P as A fragments for 4 k16 steps over the 64 keys
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s_acc[nt][0] - mbase[0]);
      const float p1 = exp2f(s_acc[nt][1] - mbase[0]);
      const float p2 = exp2f(s_acc[nt][2] - mbase[1]);
      const float p3 = exp2f(s_acc[nt][3] - mbase[1]);
      l_run[0] += p0 + p1;
      l_run[1] += p2 + p3;
      const int kk = nt >> 1, hi = nt & 1;
      pa[kk][hi ? 2 : 0] = pack2<T>(p0, p1);
      pa[kk][hi ? 3 : 1] = pack2<T>(p2, p3);
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int n0 = 0; n0 < D; n0 += 16) {
        uint32_t vb4[4];
        const T* src = &sV[stage][(kk * 16 + (lane & 15)) * DS + n0 + (lane >> 4) * 8];
        ldmatrix_x4_trans(vb4, src);
        mma_16816<T>(o_acc[n0 / 8], pa[kk], &vb4[0]);
        mma_16816<T>(o_acc[n0 / 8 + 1], pa[kk], &vb4[2]);
      }
    }
    __syncthreads();  // stage is overwritten by the prefetch two tiles later
  }
  cp_async_wait<0>();

#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    l_run[ri] += __shfl_xor_sync(0xffffffffu, l_run[ri], 1);
    l_run[ri] += __shfl_xor_sync(0xffffffffu, l_run[ri], 2);
  }
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    if (rpos[ri] >= L) continue;
    const int r = wr0 + g8 + 8 * ri;
    const int hh = h0 + r / BMQ;
    const float inv = 1.f / fmaxf(l_run[ri], 1e-20f);
    T* orow = out + b * st[9] + hh * st[10] + (int64_t)rpos[ri] * st[11];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int c = i * 8 + 2 * t4;
      *reinterpret_cast<uint32_t*>(&orow[c]) = pack2<T>(o_acc[i][2 * ri] * inv, o_acc[i][2 * ri + 1] * inv);
    }
  }
}

// ------------------------------------------------------------------ tcgen05 prefill (16-bit, D = 64)
// One CTA = two query tiles of 128 rows = G heads of one GQA group x BMQ = 128/G positions
// (row r of tile t <-> position t0 + t*BMQ + r / G, head h0 + r % G; row r is TMEM lane r of the
// tile's accumulators), each served by two warpgroups: thread r of warpgroup `half` takes row r
// and keys 64 half .. 64 half + 63 of every 128-key tile, so a row's softmax runs on two
// threads and an SM runs 16 softmax warps.  Both tiles read the same 128-key K/V tiles, loaded
// once per CTA by tiled TMA (128-byte swizzle) into a ring of kStages stages; each query tile
// runs its own loop and the two interleave on the tensor core.  Per query tile and key tile j:
//   S = Q Kᵀ   tcgen05.mma M=128 N=128 K=64 into the tile's S columns, issued for tile j+1 once
//              every row has read S(j);
//   softmax    each thread reads its half row of S (tcgen05.ld), applies scale, the GGD bias
//              (per-tile table over the BMQ + 127 distances the tile spans, per head), mask and
//              log-n scaling; the two halves' maxima meet in shared memory at the barrier that
//              also frees S; P (16-bit) goes to the tile's P columns in TMEM (tcgen05.st),
//              each half its 32 columns;
//   O += P V   tcgen05.mma M=128 N=64 K=128 with A = P read from TMEM, O accumulated in TMEM
//              against a reference row max that is raised only when a tile exceeds it by more
//              than 2^8 (O is then rescaled in TMEM, each half its 32 columns).
// The halves' row sums are added once, at the end.  The tile's first thread issues its MMAs; a
// K/V stage is released once P V of both tiles that read it completed.  All waits are bounded:
// a CTA whose wait runs out counts itself in g_wait_timeouts, drains what it issued, frees its
// TMEM and leaves its rows unwritten.
namespace tc {
constexpr int kKeys = 128, kD = 64;
constexpr int kTileBytes = 128 * kD * 2;  // 16 KB: 128 rows of 128 bytes
constexpr int kStages = 4;  // a stage is released one tile late (after P V of that tile completes)
constexpr uint32_t kWait = 1u << 22;
constexpr uint32_t kTmemCols = 512;  // per warpgroup: S 128 columns, P 64, O 64
}  // namespace tc

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// 32 consecutive 32-bit columns of this thread's TMEM lane (warp w of a warpgroup writes lanes
// 32w .. 32w+31); complete after tmem_wait_st().
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// D[tmem] (+)= A[tmem] * B[smem]: A read from TMEM (K-major, two 16-bit values per column,
// one row per lane), issued by one thread.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Barrier over the 128 threads of one warpgroup (ids 1 and 2; 0 is __syncthreads).
// Named barriers of one query tile's two warpgroups (256 threads).
__device__ __forceinline__ void qt_sync(int id) { asm volatile("bar.sync %0, 256;\n" ::"r"(id) : "memory"); }
__device__ __forceinline__ bool qt_sync_or(int id, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred ip, op;\n setp.ne.u32 ip, %1, 0;\n bar.red.or.pred op, %2, 256, ip;\n selp.u32 %0, 1, 0, op;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id)
      : "memory");
  return r != 0;
}

template <int G>
struct TcSmemLayout {
  static constexpr int BMQ = 128 / G;
  static constexpr int TBL = BMQ + 127;                  // distances one tile spans per head
  static constexpr int TBLS = (TBL + 31) / 32 * 32 + 8;  // padded: the G tables start on distinct banks
  static constexpr int offQ = 0;                          // 2 warpgroup tiles
  static constexpr int offK = offQ + 2 * tc::kTileBytes;  // kStages
  static constexpr int offV = offK + tc::kStages * tc::kTileBytes;
  static constexpr int offBias = offV + tc::kStages * tc::kTileBytes;  // 2 warpgroups x 2 tiles
  static constexpr int offKm = offBias + 4 * G * TBLS * 4;          // key bias: 2 query tiles x 2 tiles
  static constexpr int offX = offKm + 4 * tc::kKeys * 4;            // row exchange [2 query tiles][2 halves][128]
  static constexpr int offBar = offX + 2 * 2 * 128 * 4;
  static constexpr int nBar = 1 + tc::kStages + 6;  // q, kv[], s[2], o[2], drain[2]
  static constexpr int offCnt = offBar + nBar * 8;   // per-stage release count, last tile issued
  static constexpr int offTmem = offCnt + 2 * tc::kStages * 4;
  static constexpr int bytes = offTmem + 16;
  static constexpr int alloc = bytes + 1024;  // slack for 1024-byte alignment
};

// KM: an additive key bias kmask[b * kms + key] (natural-log units, -inf drops the key) is
// added to every logit, as the attention mask of chord_attn.py:347-356.
template <typename T, int G, bool KM>
__global__ void __launch_bounds__(512, 1) chord_tc_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const float* __restrict__ alpha, const float* __restrict__ beta,
    const float* __restrict__ mu, const float* __restrict__ ssmax, const float* __restrict__ log_n,
    T* __restrict__ out, int H, int Hkv, int L, int S, int q_start, float scale, float eps, Strides14 sv,
    const float* __restrict__ kmask, int64_t kms) {
  using Lay = TcSmemLayout<G>;
  constexpr int BMQ = Lay::BMQ, TBL = Lay::TBL, TBLS = Lay::TBLS, NS = tc::kStages;
  constexpr uint32_t ab_fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t idS = umma_idesc_f16(ab_fmt, 128, tc::kKeys, 0, 0);
  constexpr uint32_t idO = umma_idesc_f16(ab_fmt, 128, tc::kD, 0, 1);
  extern __shared__ unsigned char tc_smem_raw[];
  unsigned char* sm = tc_smem_raw + ((1024u - (smem_u32(tc_smem_raw) & 1023u)) & 1023u);
  unsigned char* sQ = sm + Lay::offQ;
  unsigned char* sK = sm + Lay::offK;
  unsigned char* sV = sm + Lay::offV;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Lay::offBar);
  uint64_t *barQ = bar, *barKV = bar + 1, *barS = bar + 1 + NS, *barO = bar + 3 + NS, *barDrain = bar + 5 + NS;
  int* cnt = reinterpret_cast<int*>(sm + Lay::offCnt);  // [NS] releases, [NS] last tile issued
  int* stage_tile = cnt + NS;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + Lay::offTmem);

  const int64_t* st = sv.s;
  const int tid = threadIdx.x, warp = tid >> 5;
  // four warpgroups: two per 128-row query tile (qt), each taking one half of every 128-key tile
  // (keys 64 half .. +63) for the same rows, so a row's softmax runs on two threads
  const int wg = tid >> 7, qt = wg >> 1, half = wg & 1, wt = tid & 127;
  const int ht = half * 128 + wt;  // thread index within the query tile's 256
  const bool issuer = wt == 0 && half == 0;
  const int GS = H / Hkv;
  const int groups_per_kv = GS / G;
  const int kvh = blockIdx.y / groups_per_kv;
  const int h0 = kvh * GS + (blockIdx.y % groups_per_kv) * G;
  const int b = blockIdx.z;
  const int tpair = (gridDim.x - 1 - blockIdx.x) * 2 * BMQ;  // longest rows first
  auto tiles_from = [&](int t0x) {
    if (t0x >= L) return 0;
    const int kv_end = min(S, q_start + min(L, t0x + BMQ));
    return (kv_end + tc::kKeys - 1) / tc::kKeys;
  };
  const int nA = tiles_from(tpair), nB = tiles_from(tpair + BMQ);
  const int nall = max(nA, nB);
  const int t0w = tpair + qt * BMQ;
  const int nmine = qt ? nB : nA;

  // this thread's row
  const int tl = wt / G, hg = wt % G;
  const int pos = t0w + tl, h = h0 + hg;
  const bool row_ok = pos < L;
  const int qpos = q_start + pos;
  // log-n scaling in log2 units (0 for rows past L, which are never stored)
  // logit (log2 units) = (s * scale + bias) * rc with rc = ssmax * log n * log2 e.  The sign of
  // ssmax (per head) is folded into scale and the bias table, so the row keeps x = +-(s * scale
  // + bias), its running max in those units, and applies |rc| inside the exponent.  |rc| = 0
  // (log 1 = 0 at the first position, or a row past L) becomes 1e-30: every visible key then
  // gets the same weight, and masked keys (-inf) still get none.
  const float ssh = ssmax[h];
  const float sgn = ssh < 0.f ? -1.f : 1.f;
  const float rcs = row_ok ? fmaxf(fabsf(ssh * log_n[b * st[12] + (int64_t)pos * st[13]] * kLog2e), 1e-30f) : 1e-30f;
  const float scale_s = sgn * scale;
  const float inv_rcs = 1.f / rcs;  // a key bias m (natural log) enters x as m log2(e) / |rc|

  unsigned char* sQw = sQ + qt * tc::kTileBytes;
  float* sBw = reinterpret_cast<float*>(sm + Lay::offBias) + qt * 2 * G * TBLS;
  float* sKmw = reinterpret_cast<float*>(sm + Lay::offKm) + qt * 2 * tc::kKeys;
  float* sXq = reinterpret_cast<float*>(sm + Lay::offX) + qt * 2 * 128;  // [half][row]

  if (warp == 0) tmem_alloc(sTmem, tc::kTmemCols);
  if (tid == 0) {
    for (int i = 0; i < Lay::nBar; ++i) mbar_init(&bar[i], 1);
    for (int i = 0; i < NS; ++i) {
      cnt[i] = 0;
      stage_tile[i] = -1;
    }
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;
  // TMEM columns of the query tile: S (128 fp32) | P (128 16-bit keys, 64 columns) | O (64 fp32);
  // this half reads S columns 64 half .., writes P columns 32 half .., rescales O columns 32 half ..
  const uint32_t colS = qt * 256, colP = colS + tc::kKeys, colO = colP + tc::kKeys / 2;

  auto issue_kv = [&](int j) {  // one thread
    const int s = j % NS;
    stage_tile[s] = j;
    mbar_arrive_expect_tx(&barKV[s], 2 * tc::kTileBytes);
    tma_load_4d(sK + s * tc::kTileBytes, &tmK, 0, j * tc::kKeys, kvh, b, &barKV[s]);
    tma_load_4d(sV + s * tc::kTileBytes, &tmV, 0, j * tc::kKeys, kvh, b, &barKV[s]);
  };
  auto issue_s = [&](int j) {  // warpgroup issuer: S = Q_w K_jᵀ
    const uint32_t qa = smem_u32(sQw), ka = smem_u32(sK + (j % NS) * tc::kTileBytes);
#pragma unroll
    for (int ks = 0; ks < tc::kD / 16; ++ks)
      umma_f16_ss(tmem + colS, umma_desc_sw128(qa + ks * 32, 16, 1024), umma_desc_sw128(ka + ks * 32, 16, 1024),
                  idS, ks > 0);
    umma_commit(&barS[qt]);
  };
  auto issue_o = [&](int j) {  // warpgroup issuer: O (+)= P_w V_j, P from this warpgroup's TMEM
    const uint32_t va = smem_u32(sV + (j % NS) * tc::kTileBytes);
#pragma unroll
    for (int ks = 0; ks < tc::kKeys / 16; ++ks)
      umma_f16_ts(tmem + colO, tmem + colP + ks * 8, umma_desc_sw128(va + ks * 16 * 128, tc::kTileBytes, 1024), idO,
                  (j > 0 || ks > 0) ? 1u : 0u);
    umma_commit(&barO[qt]);
  };
  auto fill_bias = [&](int j) {  // the query tile's 256 threads: table of tile j into buffer j & 1
    float* tb = sBw + (j & 1) * G * TBLS;
    const int base = q_start + t0w - j * tc::kKeys - 127;  // distance of entry 0
    for (int e = ht; e < G * TBL; e += 256) {
      const int g = e / TBL, ee = e % TBL;
      const int hh = h0 + g;
      const float b0 = ggd_bias_decode<T>(alpha[hh], beta[hh], mu[hh], (float)(base + ee), eps);
      tb[g * TBLS + ee] = ssmax[hh] < 0.f ? -b0 : b0;
    }
    if constexpr (KM) {  // the tile's key bias in log2 units
      if (half == 0) {
        const int key = j * tc::kKeys + wt;
        sKmw[(j & 1) * tc::kKeys + wt] = key < S ? kmask[(int64_t)b * kms + key] * kLog2e : 0.f;
      }
    }
  };

  if (tid == 0 && nall > 0) {
    mbar_arrive_expect_tx(barQ, 2 * tc::kTileBytes);
    tma_load_4d(sQ, &tmQ, 0, h0, tpair, b, barQ);
    tma_load_4d(sQ + tc::kTileBytes, &tmQ, 0, h0, tpair + BMQ, b, barQ);
    for (int t = 0; t < min(nall, NS); ++t) issue_kv(t);
  }
  if (nmine > 0) fill_bias(0);
  __syncthreads();
  bool failed = false;
  if (issuer && nmine > 0) {
    if (mbar_wait_bounded(barQ, 0, tc::kWait) && mbar_wait_bounded(&barKV[0], 0, tc::kWait)) {
      tc_fence_after();
      issue_s(0);
    } else {
      failed = true;
    }
  }

  // O accumulates in TMEM (P V with accumulate), exponentiated against a reference row max
  // m_ref that is raised only when the tile's max exceeds it by more than 2^8 in the exponent:
  // P entries stay below 256 (exact enough in 16 bits, far from fp32 overflow) and O is rescaled
  // in TMEM on those rare tiles instead of every tile.
  constexpr float kRescale = 8.f;
  float m_ref = -INFINITY, l = 0.f;
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
  // the issuer releases the K/V stage of tile j once P V(j) has completed (checked at tile j + 1)
  auto release = [&](int j) {
    const int s = j % NS;
    const int need = (j < nA) + (j < nB);
    __threadfence_block();
    const int prev = atomicAdd(&cnt[s], 1);
    __threadfence_block();
    if (prev + 1 == need) {
      cnt[s] = 0;
      if (j + NS < nall) issue_kv(j + NS);
    }
  };

  constexpr int HK = tc::kKeys / 2;  // keys of one half
  for (int j = 0; j < nmine; ++j) {
    bool ok = failed ? false : mbar_wait_bounded(&barS[qt], (uint32_t)(j & 1), tc::kWait);
    tc_fence_after();
    float x[HK];
    {
      uint32_t r0[32], r1[32];
      const uint32_t ta = tmem + lane_base + colS + (uint32_t)(half * HK);
      tmem_ld32(ta, r0);
      tmem_ld32(ta + 32, r1);
      tmem_wait_ld(r0);
      tmem_wait_ld(r1);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        x[i] = __uint_as_float(r0[i]);
        x[32 + i] = __uint_as_float(r1[i]);
      }
    }
    tc_fence_before();

    // x = +-(s * scale + bias) (sign of ssmax folded in); keys past the row's last visible key
    // (causal, or at / past S) are set to -inf only on the tiles that contain such keys
    const int k0 = j * tc::kKeys + half * HK;
    const int cmax = min(HK - 1, min(S - 1 - k0, qpos - k0));
    const float* tb = sBw + (j & 1) * G * TBLS + hg * TBLS + tl + 127 - half * HK;  // key offset c -> tb[-c]
#pragma unroll
    for (int c = 0; c < HK; c += 2) {
      const float2 y = ffma2(make_float2(x[c], x[c + 1]), make_float2(scale_s, scale_s),
                             make_float2(tb[-c], tb[-c - 1]));
      x[c] = y.x;
      x[c + 1] = y.y;
    }
    if constexpr (KM) {
      const float* km = sKmw + (j & 1) * tc::kKeys + half * HK;
#pragma unroll
      for (int c = 0; c < HK; ++c) x[c] = fmaf(km[c], inv_rcs, x[c]);
    }
    if (cmax < HK - 1) {
#pragma unroll
      for (int c = 0; c < HK; ++c)
        if (c > cmax) x[c] = -INFINITY;
    }
    float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int c = 0; c < HK; c += 2) mx4[(c >> 1) & 3] = fmax3(mx4[(c >> 1) & 3], x[c], x[c + 1]);
    float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
    // the row's two halves meet: every thread of the query tile holds S(j) (the columns may take
    // S(j + 1)) and has its half's max in the exchange
    sXq[half * 128 + wt] = mt;
    qt_sync(1 + qt);
    mt = fmaxf(mt, sXq[(half ^ 1) * 128 + wt]);
    if (issuer && !failed && j + 1 < nmine) {
      const int jn = j + 1;
      if (mbar_wait_bounded(&barKV[jn % NS], (uint32_t)((jn / NS) & 1), tc::kWait)) {
        tc_fence_after();
        issue_s(jn);
      } else {
        failed = true;
      }
    }
    if (j + 1 < nmine) fill_bias(j + 1);

    // raise the reference max on the first visible key, or when this tile exceeds it by > 2^8
    // (both halves of a row take the same decision: the same mt and m_ref)
    const bool raise = mt > m_ref && (m_ref == -INFINITY || (mt - m_ref) * rcs > kRescale);
    float corr = 1.f;
    if (raise) {
      corr = m_ref == -INFINITY ? 0.f : ex2_approx((m_ref - mt) * rcs);
      m_ref = mt;
    }
    const float nb = -(m_ref == -INFINITY ? 0.f : m_ref) * rcs;
    float2 ps4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    uint32_t pw[32];  // this half's P row packed in 16-bit pairs
#pragma unroll
    for (int c = 0; c < HK; c += 2) {
      const float2 t = ffma2(make_float2(x[c], x[c + 1]), make_float2(rcs, rcs), make_float2(nb, nb));
      const float p0 = ex2_approx(t.x);
      const float p1 = ex2_approx(t.y);
      ps4[(c >> 1) & 3] = fadd2(ps4[(c >> 1) & 3], make_float2(p0, p1));
      pw[c >> 1] = pack2<T>(p0, p1);
    }
    {
      const float2 q = fadd2(fadd2(ps4[0], ps4[1]), fadd2(ps4[2], ps4[3]));
      l = l * corr + (q.x + q.y);  // this half's share of the row sum
    }
    // P V(j - 1) has completed: its P columns may be overwritten, O may be rescaled, and its K/V
    // stage released
    if (j > 0) {
      if (!mbar_wait_bounded(&barO[qt], (uint32_t)((j - 1) & 1), tc::kWait)) ok = false;
      tc_fence_after();
      if (issuer && !failed) release(j - 1);
      if (__any_sync(0xffffffffu, raise)) {  // warp-collective: rows without a raise scale by 1
        uint32_t o0[32];
        const uint32_t ta = tmem + lane_base + colO + (uint32_t)(half * 32);
        tmem_ld32(ta, o0);
        tmem_wait_ld(o0);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 u0 = fmul2(make_float2(__uint_as_float(o0[i]), __uint_as_float(o0[i + 1])), make_float2(corr, corr));
          o0[i] = __float_as_uint(u0.x);
          o0[i + 1] = __float_as_uint(u0.y);
        }
        tmem_st32(ta, o0);
      }
    }
    tmem_st32(tmem + lane_base + colP + (uint32_t)(half * 32), pw);
    tmem_wait_st();
    tc_fence_before();
    if (qt_sync_or(3 + qt, !ok || failed)) {
      failed = true;
      break;
    }
    if (issuer) {
      tc_fence_after();
      issue_o(j);
    }
  }
  // the last P V of this query tile, then its stage
  bool okO = true;
  if (!failed && nmine > 0) {
    okO = mbar_wait_bounded(&barO[qt], (uint32_t)((nmine - 1) & 1), tc::kWait);
    tc_fence_after();
    if (issuer && okO) release(nmine - 1);
  }
  failed = __syncthreads_or(failed || !okO);
  if (failed) {
    if (issuer) {  // every MMA this query tile issued
      umma_commit(&barDrain[qt]);
      mbar_wait_bounded(&barDrain[qt], 0, tc::kWait);
    }
    __syncthreads();
    if (tid == 0) {  // every copy issued (the latest into each stage is the only one pending)
      atomicAdd(&g_wait_timeouts, 1u);
      if (nall > 0) mbar_wait_bounded(barQ, 0, tc::kWait);
      for (int s = 0; s < NS; ++s)
        if (stage_tile[s] >= 0)
          mbar_wait_bounded(&barKV[s], (uint32_t)((stage_tile[s] / NS) & 1), tc::kWait);
    }
  } else if (nmine > 0) {
    // the row sum: this half's share plus the other half's (the exchange is free again: every
    // thread passed the last loop barrier after its reads)
    sXq[half * 128 + wt] = l;
    qt_sync(1 + qt);
    const float lt = l + sXq[(half ^ 1) * 128 + wt];
    uint32_t o0[32];
    const uint32_t ta = tmem + lane_base + colO + (uint32_t)(half * 32);
    tmem_ld32(ta, o0);
    tmem_wait_ld(o0);
    if (row_ok) {
      const float inv = 1.f / fmaxf(lt, 1e-20f);
      T* orow = out + b * st[9] + (int64_t)h * st[10] + (int64_t)pos * st[11] + half * 32;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const uint32_t* src = &o0[c8 * 8];
        uint4 v;
        v.x = pack2<T>(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
        v.y = pack2<T>(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
        v.z = pack2<T>(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
        v.w = pack2<T>(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
        *reinterpret_cast<uint4*>(orow + c8 * 8) = v;
      }
    }
  } else if (row_ok) {  // no visible key (cannot happen for q_start >= 0): zeros
    T* orow = out + b * st[9] + (int64_t)h * st[10] + (int64_t)pos * st[11] + half * 32;
#pragma unroll
    for (int c8 = 0; c8 < 4; ++c8) *reinterpret_cast<uint4*>(orow + c8 * 8) = make_uint4(0, 0, 0, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, tc::kTmemCols);
  }
}

// ------------------------------------------------------------------ simple (fp32 / fallback)
// One warp per (b, h, query row); lanes own keys in chunks of 32 and the D outputs in slices.
template <typename T>
__global__ void __launch_bounds__(128) chord_fwd_simple_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ alpha,
    const float* __restrict__ beta, const float* __restrict__ mu, const float* __restrict__ ssmax,
    const float* __restrict__ log_n, T* __restrict__ out, int H, int Hkv, int L, int S, int D, int q_start,
    float scale, float eps, Strides14 sv, const float* __restrict__ kmask, int64_t kms) {
  const int64_t* st = sv.s;
  extern __shared__ float sq_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;  // over B * H * L
  const int64_t total = (int64_t)gridDim.y * H * L;
  (void)total;
  const int b = blockIdx.y;
  float* sq = sq_all + warp * D;
  const bool valid = row < (int64_t)H * L;
  const int h = valid ? (int)(row / L) : 0;
  const int i = valid ? (int)(row % L) : 0;
  const int kvh = h / (H / Hkv);
  const T* qr = q + b * st[0] + h * st[1] + (int64_t)i * st[2];
  for (int d = lane; d < D; d += 32) sq[d] = valid ? to_f(qr[d]) : 0.f;
  __syncwarp();
  if (!valid) return;
  const float c = ssmax[h] * log_n[b * st[12] + (int64_t)i * st[13]] * kLog2e;
  const float al = alpha[h], be = beta[h], m_u = mu[h];
  const int qa = q_start + i;
  const int kend = min(S, qa + 1);
  const T* kb = k + b * st[3] + kvh * st[4];
  const T* vb = v + b * st[6] + kvh * st[7];
  constexpr int MAXD = 4;  // D <= 128
  float o[MAXD] = {0.f, 0.f, 0.f, 0.f};
  float m = -INFINITY, l = 0.f;
  for (int j0 = 0; j0 < kend; j0 += 32) {
    const int j = j0 + lane;
    float x = -INFINITY;
    if (j < kend) {
      const T* kr = kb + (int64_t)j * st[5];
      float s = 0.f;
      for (int d = 0; d < D; ++d) s = fmaf(sq[d], to_f(kr[d]), s);
      x = (s * scale + ggd_bias(al, be, m_u, (float)(qa - j), eps)) * c;
      if (kmask) x = fmaf(kmask[(int64_t)b * kms + j], kLog2e, x);
    }
    const float cm = warp_max(x);
    const float mn = fmaxf(m, cm);
    const float mb = mn == -INFINITY ? 0.f : mn;  // every key so far dropped by the mask
    const float corr = exp2f(m - mb);
    const float p = exp2f(x - mb);
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int r = 0; r < MAXD; ++r) o[r] *= corr;
    const int nk = min(32, kend - j0);
    for (int jj = 0; jj < nk; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      const T* vr = vb + (int64_t)(j0 + jj) * st[8];
#pragma unroll
      for (int r = 0; r < MAXD; ++r) {
        const int d = lane + 32 * r;
        if (d < D) o[r] = fmaf(pj, to_f(vr[d]), o[r]);
      }
    }
    m = mn;
  }
  T* orow = out + b * st[9] + h * st[10] + (int64_t)i * st[11];
  const float inv = 1.f / fmaxf(l, 1e-20f);
#pragma unroll
  for (int r = 0; r < MAXD; ++r) {
    const int d = lane + 32 * r;
    if (d < D) orow[d] = from_f<T>(o[r] * inv);
  }
}

// ------------------------------------------------------------------ split-KV decode
// One CTA (4 warps) per (split, b * Hkv + kv head).  A split's keys are a contiguous run of
// that (b, kv head)'s [cap, D] K and V arrays, streamed through a ring of kDecStages
// 64-key tiles by one-dimensional bulk copies: thread 0 issues K and V of a tile onto the
// stage's mbarrier, every thread waits on it (bounded), and the stage is refilled once the
// whole CTA has finished with it.  Rows R = G * Tn (query heads of the group x new tokens),
// R <= RM.
//   scores       warp w scores keys 16w .. 16w+15 of the tile, four at a time: each 8-lane
//                group takes one key, its lanes hold D/8 dims of every query row and reduce
//                the partial dots with three xor-shuffles;
//   softmax + PV warp w owns rows w, w+4, ...; online softmax over the tile, then each lane
//                accumulates D/32 output dims over the tile's keys.
// Partials: ws[((split * B + b) * H + h) * Tn + t][D + 2] = (o[0..D), m, l) for the merge.
constexpr int kDecTile = 64;
// The testing knob MB_FORCE_DECODE_SCALAR routes 16-bit D = 64 decode through the CUDA-core
// kernel (the tensor-core kernel is the default) so tests can cross-check the two.
static bool force_scalar_decode() { return forced(MB_FORCE_DECODE_SCALAR); }
#ifndef CD_STAGES
#define CD_STAGES 3
#endif
constexpr int kDecStages = CD_STAGES;
constexpr uint32_t kDecWaitLimit = 1u << 22;

template <typename T, int D, int RM>
struct DecodeSmem {
  T k[kDecStages][kDecTile][D];
  T v[kDecStages][kDecTile][D];
  float p[RM][kDecTile];
  uint64_t bar[kDecStages];
};

template <int N, typename T>
__device__ __forceinline__ void load_vec_f(const T* src, float* dst) {
  // N consecutive elements from shared memory, 16 / 8 / 4-byte vector loads where N allows
  constexpr int BYTES = N * (int)sizeof(T);
  if constexpr (BYTES % 16 == 0) {
#pragma unroll
    for (int c = 0; c < BYTES / 16; ++c) {
      const uint4 raw = reinterpret_cast<const uint4*>(src)[c];
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int x = 0; x < 16 / (int)sizeof(T); ++x) dst[c * (16 / sizeof(T)) + x] = to_f(e[x]);
    }
  } else if constexpr (BYTES == 8) {
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int x = 0; x < N; ++x) dst[x] = to_f(e[x]);
  } else if constexpr (BYTES == 4) {
    const uint32_t raw = *reinterpret_cast<const uint32_t*>(src);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int x = 0; x < N; ++x) dst[x] = to_f(e[x]);
  } else {
#pragma unroll
    for (int x = 0; x < N; ++x) dst[x] = to_f(src[x]);
  }
}

template <typename T, int D, int RM>
__global__ void __launch_bounds__(128) chord_decode_kernel(
    const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc, int64_t cap,
    const int32_t* __restrict__ len_dev, int len_host, const float* __restrict__ alpha,
    const float* __restrict__ beta, const float* __restrict__ mu, const float* __restrict__ ssmax,
    float* __restrict__ ws, int B, int H, int Hkv, int Tn, int nsplit, float scale, float eps,
    const float* __restrict__ kmask, int64_t kms) {
  constexpr int QD = D / 8;   // dims per lane in the score phase
  constexpr int OD = D / 32;  // output dims per lane
  constexpr int RW = RM / 4;  // rows per warp in the softmax / PV phase
  extern __shared__ __align__(128) unsigned char dec_smem_raw[];
  auto& sm = *reinterpret_cast<DecodeSmem<T, D, RM>*>(dec_smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane & 7, grp = lane >> 3;
  const int split = blockIdx.x;
  const int bk = blockIdx.y;  // b * Hkv + kvh
  const int b = bk / Hkv, kvh = bk % Hkv;
  const int G = H / Hkv;
  const int R = G * Tn;
  // cache length including the new tokens; a device-side length is clamped to [Tn, cap] so
  // that a stale counter can only give wrong scores, never an access outside the cache
  const int S = len_dev ? min(max(*len_dev, Tn), (int)cap) : len_host;
  const int q_start = S - Tn;
  const int per = ((S + nsplit - 1) / nsplit + kDecTile - 1) / kDecTile * kDecTile;
  const int kbeg = min(S, split * per), kend = min(S, kbeg + per);
  const int ntile = (kend - kbeg + kDecTile - 1) / kDecTile;
  const T* kb = kc + ((int64_t)b * Hkv + kvh) * cap * D;
  const T* vb = vc + ((int64_t)b * Hkv + kvh) * cap * D;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) mbar_init(&sm.bar[s], 1);
    mbar_init_fence();
  }
  __syncthreads();
  auto issue = [&](int t) {  // thread 0: K and V rows of tile t into stage t % kDecStages
    const int s = t % kDecStages;
    const int j0 = kbeg + t * kDecTile;
    const uint32_t bytes = (uint32_t)(min(kDecTile, kend - j0) * D * (int)sizeof(T));
    mbar_arrive_expect_tx(&sm.bar[s], 2 * bytes);
    bulk_load(&sm.k[s][0][0], kb + (int64_t)j0 * D, bytes, &sm.bar[s]);
    bulk_load(&sm.v[s][0][0], vb + (int64_t)j0 * D, bytes, &sm.bar[s]);
  };
  int nissued = 0;  // tiles issued so far (meaningful in thread 0, the only issuer)
  if (threadIdx.x == 0)
    for (; nissued < min(ntile, kDecStages); ++nissued) issue(nissued);

  // this lane's D/8 slice of every query row; the rows whose scores this lane finalises are
  // sub and sub + 8 (RO of them), with their log-n scaling, position and GGD parameters
  constexpr int RO = (RM + 7) / 8;
  float qr[RM][QD];
#pragma unroll
  for (int r = 0; r < RM; ++r) {
#pragma unroll
    for (int i = 0; i < QD; ++i) qr[r][i] = 0.f;
    if (r < R) {
      const int h = kvh * G + r / Tn, t = r % Tn;
      const T* qrow = q + ((int64_t)b * Tn + t) * H * D + (int64_t)h * D + sub * QD;
#pragma unroll
      for (int i = 0; i < QD; ++i) qr[r][i] = to_f(qrow[i]);
    }
  }
  float rc[RO], pa[RO], pb[RO], pm[RO];
  int qa[RO];
#pragma unroll
  for (int u = 0; u < RO; ++u) {
    const int r = sub + 8 * u;
    rc[u] = pa[u] = pb[u] = pm[u] = 0.f;
    qa[u] = -1;
    if (r < R) {
      const int h = kvh * G + r / Tn, t = r % Tn;
      qa[u] = q_start + t;
      rc[u] = ssmax[h] * logf((float)(qa[u] + 1)) * kLog2e;
      pa[u] = alpha[h];
      pb[u] = beta[h];
      pm[u] = mu[h];
    }
  }
  float m[RW], l[RW], o[RW][OD];
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int d = 0; d < OD; ++d) o[i][d] = 0.f;
  }

  int t = 0;
  bool failed = false;
  for (; t < ntile; ++t) {
    const int s = t % kDecStages;
    const int j0 = kbeg + t * kDecTile;
    const int nk = min(kDecTile, kend - j0);
    const bool ok = mbar_wait_bounded(&sm.bar[s], (uint32_t)((t / kDecStages) & 1), kDecWaitLimit);
    // scores (a stage whose copy did not land is read anyway: in bounds, result discarded)
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
      const int kk = warp * 16 + pass * 4 + grp;
      const int j = j0 + kk;
      float kf[QD];
      load_vec_f<QD>(&sm.k[s][kk][sub * QD], kf);
      float acc[RM];
#pragma unroll
      for (int r = 0; r < RM; ++r) {
        acc[r] = 0.f;
        if (r < R) {
#pragma unroll
          for (int i = 0; i < QD; ++i) acc[r] = fmaf(qr[r][i], kf[i], acc[r]);
          acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
          acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 2);
          acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 4);
        }
      }
      // every lane of the group now holds every row's dot; lane sub finalises rows sub, sub + 8
#pragma unroll
      for (int u = 0; u < RO; ++u) {
        const int r = sub + 8 * u;
        float a = 0.f;
#pragma unroll
        for (int rr = 0; rr < RM; ++rr)
          if (rr == r) a = acc[rr];
        if (r < R) {
          float x = -INFINITY;
          if (kk < nk && j <= qa[u]) {
            x = (a * scale + ggd_bias_decode<T>(pa[u], pb[u], pm[u], (float)(qa[u] - j), eps)) * rc[u];
            if (kmask) x = fmaf(kmask[(int64_t)b * kms + j], kLog2e, x);  // key bias (mask)
          }
          sm.p[r][kk] = x;
        }
      }
    }
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    // online softmax + PV for this warp's rows
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      const int r = warp + 4 * i;
      if (r >= R) break;
      const float x0 = sm.p[r][lane], x1 = sm.p[r][lane + 32];
      const float cm = warp_max(fmaxf(x0, x1));
      const float mn = fmaxf(m[i], cm);
      const float mb = mn == -INFINITY ? 0.f : mn;
      const float corr = exp2f(m[i] - mb);
      const float p0 = exp2f(x0 - mb), p1 = exp2f(x1 - mb);
      l[i] = l[i] * corr + p0 + p1;
      m[i] = mn;
      sm.p[r][lane] = p0;
      sm.p[r][lane + 32] = p1;
      __syncwarp();
#pragma unroll
      for (int d = 0; d < OD; ++d) o[i][d] *= corr;
      int kk = 0;
#pragma unroll 2
      for (; kk + 4 <= nk; kk += 4) {
        const float4 p4 = *reinterpret_cast<const float4*>(&sm.p[r][kk]);
        const float pj[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float vf[OD];
          load_vec_f<OD>(&sm.v[s][kk + e][lane * OD], vf);
#pragma unroll
          for (int d = 0; d < OD; ++d) o[i][d] = fmaf(pj[e], vf[d], o[i][d]);
        }
      }
      for (; kk < nk; ++kk) {
        const float pj = sm.p[r][kk];
        float vf[OD];
        load_vec_f<OD>(&sm.v[s][kk][lane * OD], vf);
#pragma unroll
        for (int d = 0; d < OD; ++d) o[i][d] = fmaf(pj, vf[d], o[i][d]);
      }
    }
    __syncthreads();  // stage s and the score tile are free again
    if (threadIdx.x == 0 && t + kDecStages < ntile) {
      fence_proxy_async_smem();
      issue(t + kDecStages);
      ++nissued;
    }
  }
  if (failed) {
    // record, then let the copies already issued land (bounded) before the CTA exits
    if (threadIdx.x == 0) {
      atomicAdd(&g_wait_timeouts, 1u);
      for (int u = t; u < nissued; ++u)
        mbar_wait_bounded(&sm.bar[u % kDecStages], (uint32_t)((u / kDecStages) & 1), kDecWaitLimit);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      m[i] = -INFINITY;
      l[i] = 0.f;
#pragma unroll
      for (int d = 0; d < OD; ++d) o[i][d] = 0.f;
    }
  }
#pragma unroll
  for (int i = 0; i < RW; ++i) {
    const int r = warp + 4 * i;
    if (r >= R) break;
    const float lt = warp_sum(l[i]);
    const int h = kvh * G + r / Tn, tt = r % Tn;
    float* dst = ws + ((((int64_t)split * B + b) * H + h) * Tn + tt) * (D + 2);
#pragma unroll
    for (int d = 0; d < OD; ++d) dst[lane * OD + d] = o[i][d];
    if (lane == 0) {
      dst[D] = m[i];
      dst[D + 1] = lt;
    }
  }
}

// Tensor-core variant for 16-bit caches with D = 64.  The MMA rows are the R <= 16 query
// rows; K and V tiles arrive by tiled tensor copies with the 128-byte swizzle (16-byte
// chunk c of key row r lands at chunk c ^ (r & 7)), which makes the K fragment loads and the
// transposed V ldmatrix below bank-conflict free.  Warp w takes keys 16w .. 16w+15 of every
// tile (QKᵀ: 2 x 4 m16n8k16, PV: 8 m16n8k16) and keeps its own online-softmax state; the
// four warps' states are combined through shared memory at the end.  The barrier at the top
// of each tile also tells thread 0 that the previous tile's stage is free to refill.
// RH = 1 when every query row sits in the first 8 MMA rows (R <= 8: decode with up to 8
// query heads per kv head): the softmax of rows g8 + 8 is skipped at compile time, which
// takes the kernel from 117 to 89 registers.  With a 3-stage ring (48 KB) four CTAs fit on
// an SM (16 warps); measured at B = 64, context 8192, that is 7% faster per decode step
// than 3 CTAs with 4 stages, whose extra tile in flight does not pay for the lost warps.
template <typename T, int RH>
__global__ void __launch_bounds__(128) chord_decode_mma_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const T* __restrict__ q,
    int64_t cap, const int32_t* __restrict__ len_dev, int len_host, const float* __restrict__ alpha,
    const float* __restrict__ beta, const float* __restrict__ mu, const float* __restrict__ ssmax,
    float* __restrict__ ws, int B, int H, int Hkv, int Tn, int nsplit, float scale, float eps,
    const float* __restrict__ kmask, int64_t kms) {
  constexpr int D = 64;
  constexpr int TILE_BYTES = kDecTile * D * 2;  // 8 KB, rows of 128 bytes
  extern __shared__ unsigned char dec_mma_smem[];
  unsigned char* base = dec_mma_smem + ((1024u - (smem_u32(dec_mma_smem) & 1023u)) & 1023u);
  unsigned char* sK = base;
  unsigned char* sV = base + kDecStages * TILE_BYTES;
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + 2 * kDecStages * TILE_BYTES);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int split = blockIdx.x;
  const int bk = blockIdx.y;
  const int b = bk / Hkv, kvh = bk % Hkv;
  const int G = H / Hkv;
  const int R = G * Tn;
  const int S = len_dev ? min(max(*len_dev, Tn), (int)cap) : len_host;
  const int q_start = S - Tn;
  const int per = ((S + nsplit - 1) / nsplit + kDecTile - 1) / kDecTile * kDecTile;
  const int kbeg = min(S, split * per), kend = min(S, kbeg + per);
  const int ntile = (kend - kbeg + kDecTile - 1) / kDecTile;
  const int row0 = bk * (int)cap;  // tensor row of this (b, kv head)'s key 0 (host: B*Hkv*cap < 2^31)

  if (tid == 0) {
    for (int s = 0; s < kDecStages; ++s) mbar_init(&bar[s], 1);
    mbar_init_fence();
  }
  __syncthreads();
  auto issue = [&](int t) {
    const int s = t % kDecStages;
    const int y = row0 + kbeg + t * kDecTile;
    mbar_arrive_expect_tx(&bar[s], 2 * TILE_BYTES);
    tma_load_2d(sK + s * TILE_BYTES, &tmK, 0, y, &bar[s]);
    tma_load_2d(sV + s * TILE_BYTES, &tmV, 0, y, &bar[s]);
  };
  int nissued = 0;  // tiles issued so far (meaningful in thread 0, the only issuer)
  if (tid == 0)
    for (; nissued < min(ntile, kDecStages); ++nissued) issue(nissued);

  // rows g8 and g8 + 8 of the MMA tile
  bool rv[2];
  int rqa[2];
  float rrc[2], ral[2], rbe[2], rmu[2];
  uint32_t qf[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) qf[kk][0] = qf[kk][1] = qf[kk][2] = qf[kk][3] = 0u;
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int r = g8 + 8 * ri;
    rv[ri] = r < R && ri < RH;
    rqa[ri] = -1;
    rrc[ri] = ral[ri] = rbe[ri] = rmu[ri] = 0.f;
    if (rv[ri]) {
      const int h = kvh * G + r / Tn, t = r % Tn;
      rqa[ri] = q_start + t;
      rrc[ri] = ssmax[h] * logf((float)(rqa[ri] + 1)) * kLog2e;
      ral[ri] = alpha[h];
      rbe[ri] = beta[h];
      rmu[ri] = mu[h];
      const uint32_t* qw = reinterpret_cast<const uint32_t*>(q + (((int64_t)b * Tn + t) * H + h) * D);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        qf[kk][ri] = qw[kk * 8 + t4];
        qf[kk][2 + ri] = qw[kk * 8 + 4 + t4];
      }
    }
  }

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  int t = 0;
  bool failed = false;
  for (; t < ntile; ++t) {
    const int s = t % kDecStages;
    const bool ok = mbar_wait_bounded(&bar[s], (uint32_t)((t / kDecStages) & 1), kDecWaitLimit);
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    if (tid == 0 && t >= 1 && t - 1 + kDecStages < ntile) {
      fence_proxy_async_smem();
      issue(t - 1 + kDecStages);  // refills the stage tile t - 1 used; every warp is past it
      ++nissued;
    }
    const int j0 = kbeg + t * kDecTile;
    const int nk = min(kDecTile, kend - j0);
    // S = Q Kᵀ over this warp's 16 keys
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
    // B fragments by ldmatrix: lane l addresses key row 8 nt + (l & 7) of this warp's slice at
    // 16-byte chunk 4 kp + (l >> 3) (swizzled), so matrix i of the x4 load is chunk 4 kp + i
    // and registers {0, 1} / {2, 3} are the fragments of k-steps 2 kp / 2 kp + 1
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int kr = warp * 16 + nt * 8 + (lane & 7);
      const unsigned char* krow = sK + s * TILE_BYTES + kr * 128;
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        uint32_t bb[4];
        ldmatrix_x4(bb, krow + (((4 * kp + (lane >> 3)) ^ (kr & 7)) << 4));
        mma_16816<T>(sacc[nt], qf[2 * kp], &bb[0]);
        mma_16816<T>(sacc[nt], qf[2 * kp + 1], &bb[2]);
      }
    }
    // logits in log2 units with the GGD bias, masking, online softmax
    float rmax[2] = {-INFINITY, -INFINITY};
    if constexpr (RH == 1) {
      // one query row per thread: its two adjacent keys per n8 tile as packed fp32 pairs
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int kl = warp * 16 + nt * 8 + 2 * t4;
        const int j = j0 + kl;
        const float2 d = make_float2((float)(rqa[0] - j), (float)(rqa[0] - j - 1));
        float2 t = fadd2(d, make_float2(rmu[0], rmu[0]));  // |-delta - mu| + eps
        t = fadd2(make_float2(fabsf(t.x), fabsf(t.y)), make_float2(eps, eps));
        const float2 pw = fmul2(make_float2(__log2f(t.x), __log2f(t.y)), make_float2(rbe[0], rbe[0]));
        const float2 bias = fmul2(make_float2(ex2f_(pw.x), ex2f_(pw.y)), make_float2(-ral[0], -ral[0]));
        float2 xx = fmul2(ffma2(make_float2(sacc[nt][0], sacc[nt][1]), make_float2(scale, scale), bias),
                          make_float2(rrc[0], rrc[0]));
        if (kmask) {  // key bias (mask)
          if (kl < nk) xx.x = fmaf(kmask[(int64_t)b * kms + j], kLog2e, xx.x);
          if (kl + 1 < nk) xx.y = fmaf(kmask[(int64_t)b * kms + j + 1], kLog2e, xx.y);
        }
        const float x0 = rv[0] && kl < nk && j <= rqa[0] ? xx.x : -INFINITY;
        const float x1 = rv[0] && kl + 1 < nk && j + 1 <= rqa[0] ? xx.y : -INFINITY;
        sacc[nt][0] = x0;
        sacc[nt][1] = x1;
        rmax[0] = fmax3(rmax[0], x0, x1);
      }
    } else {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2 * RH; ++e) {
        const int ri = e >> 1;
        const int kl = warp * 16 + nt * 8 + 2 * t4 + (e & 1);
        const int j = j0 + kl;
        float x = -INFINITY;
        if (rv[ri] && kl < nk && j <= rqa[ri]) {
          x = (sacc[nt][e] * scale + ggd_bias_decode<T>(ral[ri], rbe[ri], rmu[ri], (float)(rqa[ri] - j), eps)) *
              rrc[ri];
          if (kmask) x = fmaf(kmask[(int64_t)b * kms + j], kLog2e, x);  // key bias (mask)
        }
        sacc[nt][e] = x;
        rmax[ri] = fmaxf(rmax[ri], x);
      }
    }
    }
    float mb[2] = {0.f, 0.f};
#pragma unroll
    for (int ri = 0; ri < RH; ++ri) {
      rmax[ri] = fmaxf(rmax[ri], __shfl_xor_sync(0xffffffffu, rmax[ri], 1));
      rmax[ri] = fmaxf(rmax[ri], __shfl_xor_sync(0xffffffffu, rmax[ri], 2));
      const float mn = fmaxf(m[ri], rmax[ri]);
      mb[ri] = mn == -INFINITY ? 0.f : mn;
      const float corr = exp2f(m[ri] - mb[ri]);
      m[ri] = mn;
      l[ri] *= corr;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 oc = fmul2(make_float2(o[i][2 * ri], o[i][2 * ri + 1]), make_float2(corr, corr));
        o[i][2 * ri] = oc.x;
        o[i][2 * ri + 1] = oc.y;
      }
    }
    uint32_t pa[4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float p0, p1;
      if constexpr (RH == 1) {
        const float2 a = fadd2(make_float2(sacc[nt][0], sacc[nt][1]), make_float2(-mb[0], -mb[0]));
        p0 = ex2f_(a.x);
        p1 = ex2f_(a.y);
      } else {
        p0 = exp2f(sacc[nt][0] - mb[0]);
        p1 = exp2f(sacc[nt][1] - mb[0]);
      }
      l[0] += p0 + p1;
      pa[2 * nt] = pack2<T>(p0, p1);
      if constexpr (RH == 2) {
        const float p2 = exp2f(sacc[nt][2] - mb[1]), p3 = exp2f(sacc[nt][3] - mb[1]);
        l[1] += p2 + p3;
        pa[2 * nt + 1] = pack2<T>(p2, p3);
      } else {
        pa[2 * nt + 1] = 0u;  // rows g8 + 8 >= R: no query there
      }
    }
    // Key rows at or past nk hold whatever the cache slots (or the next head's rows) contain,
    // possibly non-finite: P is 0 there, but 0 * NaN would still poison the MMA, so this warp
    // zeroes its rows of the V tile that lie past the split's last key (full 128-byte rows,
    // swizzle-independent).  The proxy fence orders these writes before the stage's refill.
    if (warp * 16 + 16 > nk) {
      uint4* vz = reinterpret_cast<uint4*>(sV + s * TILE_BYTES + warp * 16 * 128);
      for (int i = lane; i < 16 * 8; i += 32)
        if (warp * 16 + (i >> 3) >= nk) vz[i] = make_uint4(0, 0, 0, 0);
      fence_proxy_async_smem();
      __syncwarp();
    }
    // O += P V over the same 16 keys (V rows 16w .. 16w+15, transposed by ldmatrix)
    const int vr = warp * 16 + (lane & 15);
    const unsigned char* vrow = sV + s * TILE_BYTES + vr * 128;
#pragma unroll
    for (int n0 = 0; n0 < D; n0 += 16) {
      uint32_t vb4[4];
      const int chunk = n0 / 8 + (lane >> 4);
      ldmatrix_x4_trans(vb4, vrow + ((chunk ^ (vr & 7)) << 4));
      mma_16816<T>(o[n0 / 8], pa, &vb4[0]);
      mma_16816<T>(o[n0 / 8 + 1], pa, &vb4[2]);
    }
  }
  __syncthreads();  // all tiles consumed (every issued copy was waited on): reuse the K stages
  float* sM = reinterpret_cast<float*>(sK);  // [4][16]
  float* sL = sM + 64;                       // [4][16]
  float* sO = sL + 64;                       // [4][16][64]
  if (failed) {
    __shared__ int drained;
    if (tid == 0) {
      atomicAdd(&g_wait_timeouts, 1u);
      bool all = true;
      for (int u = t; u < nissued; ++u)
        all = mbar_wait_bounded(&bar[u % kDecStages], (uint32_t)((u / kDecStages) & 1), kDecWaitLimit) && all;
      drained = all ? 1 : 0;
    }
    __syncthreads();
    if (!drained) {
      // A copy may still land in the stages: leave shared memory alone and write this
      // split's rows as empty partials (m = -inf, l = 0, o = 0) straight to the workspace.
      for (int idx = tid; idx < R * (D + 2); idx += 128) {
        const int r = idx / (D + 2), d = idx % (D + 2);
        const int h = kvh * G + r / Tn, tt = r % Tn;
        ws[((((int64_t)split * B + b) * H + h) * Tn + tt) * (D + 2) + d] = d == D ? -INFINITY : 0.f;
      }
      return;
    }
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      m[ri] = -INFINITY;
      l[ri] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  }
#pragma unroll
  for (int ri = 0; ri < RH; ++ri) {
    l[ri] += __shfl_xor_sync(0xffffffffu, l[ri], 1);
    l[ri] += __shfl_xor_sync(0xffffffffu, l[ri], 2);
    const int r = g8 + 8 * ri;
    if (t4 == 0) {
      sM[warp * 16 + r] = m[ri];
      sL[warp * 16 + r] = l[ri];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sO[(warp * 16 + r) * D + i * 8 + 2 * t4] = o[i][2 * ri];
      sO[(warp * 16 + r) * D + i * 8 + 2 * t4 + 1] = o[i][2 * ri + 1];
    }
  }
  __syncthreads();
  for (int idx = tid; idx < R * D; idx += 128) {
    const int r = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sM[w * 16 + r]);
    const float Mb = M == -INFINITY ? 0.f : M;
    float val = 0.f, lt = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = exp2f(sM[w * 16 + r] - Mb);
      val = fmaf(sO[(w * 16 + r) * D + d], f, val);
      lt = fmaf(sL[w * 16 + r], f, lt);
    }
    const int h = kvh * G + r / Tn, tt = r % Tn;
    float* dst = ws + ((((int64_t)split * B + b) * H + h) * Tn + tt) * (D + 2);
    dst[d] = val;
    if (d == 0) {
      dst[D] = M;
      dst[D + 1] = lt;
    }
  }
}

// Merge of the split partials: one warp per (b, t, h) output row.  Lanes stride over the
// splits for the global max and the denominator, then each lane combines D/32 dims.
template <typename T, int D>
__global__ void __launch_bounds__(128) chord_merge_kernel(const float* __restrict__ ws, T* __restrict__ out,
                                                          int64_t os, int B, int H, int Tn, int nsplit) {
  constexpr int OD = D / 32;
  allow_dependent_launch();  // the decoder's down / output projections may start fetching weights
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);  // (b * Tn + t) * H + h
  if (row >= (int64_t)B * Tn * H) return;
  const int h = (int)(row % H);
  const int64_t bt = row / H;
  const int t = (int)(bt % Tn), b = (int)(bt / Tn);
  const int64_t split_stride = (int64_t)B * H * Tn * (D + 2);
  const float* base = ws + (((int64_t)b * H + h) * Tn + t) * (D + 2);
  if (nsplit <= 64) {
    // Lane sp holds splits sp and sp + 32's (m, l) and weights; the partial rows are then read
    // eight splits at a time with all loads in flight, and summed in split order (the same
    // arithmetic as the general loop below, whose lanes also take splits sp, sp + 32).
    float ms0 = -INFINITY, ls0 = 0.f, ms1 = -INFINITY, ls1 = 0.f;
    if (lane < nsplit) {
      ms0 = base[lane * split_stride + D];
      ls0 = base[lane * split_stride + D + 1];
    }
    if (lane + 32 < nsplit) {
      ms1 = base[(lane + 32) * split_stride + D];
      ls1 = base[(lane + 32) * split_stride + D + 1];
    }
    const float mx = warp_max(fmaxf(ms0, ms1));
    const float mb = mx == -INFINITY ? 0.f : mx;
    const float w0 = lane < nsplit ? exp2f(ms0 - mb) : 0.f;
    const float w1 = lane + 32 < nsplit ? exp2f(ms1 - mb) : 0.f;
    float dpart = 0.f;
    if (lane < nsplit) dpart += ls0 * w0;
    if (lane + 32 < nsplit) dpart += ls1 * w1;
    const float den = warp_sum(dpart);
    float acc[OD];
#pragma unroll
    for (int d = 0; d < OD; ++d) acc[d] = 0.f;
    for (int sp0 = 0; sp0 < nsplit; sp0 += 8) {
      float v[8][OD];
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int d = 0; d < OD; ++d) v[u][d] = sp0 + u < nsplit ? base[(sp0 + u) * split_stride + lane * OD + d] : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float wu = __shfl_sync(0xffffffffu, sp0 + u < 32 ? w0 : w1, (sp0 + u) & 31);
        if (sp0 + u < nsplit)
#pragma unroll
          for (int d = 0; d < OD; ++d) acc[d] = fmaf(wu, v[u][d], acc[d]);
      }
    }
    const float inv = 1.f / fmaxf(den, 1e-20f);
    T* dst = out + ((int64_t)b * Tn + t) * os + (int64_t)h * D;
#pragma unroll
    for (int d = 0; d < OD; ++d) dst[lane * OD + d] = from_f<T>(acc[d] * inv);
    return;
  }
  float mmax = -INFINITY;
  for (int sp = lane; sp < nsplit; sp += 32) mmax = fmaxf(mmax, base[sp * split_stride + D]);
  mmax = warp_max(mmax);
  const float mb = mmax == -INFINITY ? 0.f : mmax;
  float den = 0.f;
  for (int sp = lane; sp < nsplit; sp += 32) {
    const float* src = base + sp * split_stride;
    den += src[D + 1] * exp2f(src[D] - mb);
  }
  den = warp_sum(den);
  float acc[OD];
#pragma unroll
  for (int d = 0; d < OD; ++d) acc[d] = 0.f;
  for (int sp = 0; sp < nsplit; ++sp) {
    const float* src = base + sp * split_stride;
    const float w = exp2f(src[D] - mb);
#pragma unroll
    for (int d = 0; d < OD; ++d) acc[d] = fmaf(w, src[lane * OD + d], acc[d]);
  }
  const float inv = 1.f / fmaxf(den, 1e-20f);
  T* dst = out + ((int64_t)b * Tn + t) * os + (int64_t)h * D;
#pragma unroll
  for (int d = 0; d < OD; ++d) dst[lane * OD + d] = from_f<T>(acc[d] * inv);
}

// ------------------------------------------------------------------ prep (q/k norms + append)
template <typename T>
__global__ void chord_prep_kernel(const T* __restrict__ proj, int64_t ps, const T* __restrict__ qn_w,
                                  const T* __restrict__ kn_w, T* __restrict__ qo, T* __restrict__ kc,
                                  T* __restrict__ vc, int64_t cap, const int32_t* __restrict__ pos_dev,
                                  int64_t pos_host, int64_t rows, int Tn, int H, int Hkv, int D, float eps) {
  const int lane = threadIdx.x & 31;
  const int slots = H + 2 * Hkv;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wid >= rows * slots) return;
  const int64_t tok = wid / slots;
  const int slot = (int)(wid % slots);
  const int b = (int)(tok / Tn), t = (int)(tok % Tn);
  const int64_t pos = (pos_dev ? (int64_t)*pos_dev : pos_host) + t;
  const T* src = proj + tok * ps + (int64_t)slot * D;  // q heads, then k heads, then v heads
  // a device-side position past the cache capacity skips the cache write (the host checks
  // host-side positions before launch)
  if (slot >= H && (pos < 0 || pos >= cap)) return;
  if (slot >= H + Hkv) {  // value: plain copy into the cache
    const int kvh = slot - H - Hkv;
    T* dst = vc + (((int64_t)b * Hkv + kvh) * cap + pos) * D;
    for (int d = lane; d < D; d += 32) dst[d] = src[d];
    return;
  }
  const T* w = slot < H ? qn_w : kn_w;
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float x = to_f(src[d]);
    ss += x * x;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  T* dst = slot < H ? qo + tok * H * D + (int64_t)slot * D
                    : kc + (((int64_t)b * Hkv + (slot - H)) * cap + pos) * D;
  for (int d = lane; d < D; d += 32) {
    const float y = to_f(from_f<T>(to_f(src[d]) * r));
    dst[d] = from_f<T>(y * to_f(w[d]));
  }
}

template <typename T, int D>
int launch_mma_d(int G, const void* q, const void* k, const void* v, const float* alpha, const float* beta,
                 const float* mu, const float* ssmax, const float* log_n, void* out, int64_t B, int64_t H, int64_t Hkv,
                 int64_t L, int64_t S, int64_t q_start, float scale, float eps, const Strides14& sv, cudaStream_t st) {
  const int GS = (int)(H / Hkv);
  auto go = [&](auto gc) {
    constexpr int GG = decltype(gc)::value;
    dim3 grid((unsigned)((L + 64 / GG - 1) / (64 / GG)), (unsigned)(Hkv * (GS / GG)), (unsigned)B);
    chord_fwd_mma_kernel<T, D, GG><<<grid, 128, 0, st>>>((const T*)q, (const T*)k, (const T*)v, alpha, beta, mu,
                                                         ssmax, log_n, (T*)out, (int)H, (int)Hkv, (int)L, (int)S,
                                                         (int)q_start, scale, eps, sv);
    return check_launch("chord_fwd_mma");
  };
  switch (G) {
    case 8: return go(std::integral_constant<int, 8>{});
    case 4: return go(std::integral_constant<int, 4>{});
    case 2: return go(std::integral_constant<int, 2>{});
    default: return go(std::integral_constant<int, 1>{});
  }
}

template <typename T>
int launch_mma(int64_t D, int G, const void* q, const void* k, const void* v, const float* alpha, const float* beta,
               const float* mu, const float* ssmax, const float* log_n, void* out, int64_t B, int64_t H, int64_t Hkv,
               int64_t L, int64_t S, int64_t q_start, float scale, float eps, const Strides14& sv, cudaStream_t st) {
  switch (D) {
    case 16: return launch_mma_d<T, 16>(G, q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps, sv, st);
    case 32: return launch_mma_d<T, 32>(G, q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps, sv, st);
    case 64: return launch_mma_d<T, 64>(G, q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps, sv, st);
    default: return set_error(MB_ERR_UNSUPPORTED, "chord: head dim %lld", (long long)D);
  }
}

template <typename T>
int launch_simple(const void* q, const void* k, const void* v, const float* alpha, const float* beta, const float* mu,
                  const float* ssmax, const float* log_n, void* out, int64_t B, int64_t H, int64_t Hkv, int64_t L,
                  int64_t S, int64_t D, int64_t q_start, float scale, float eps, const Strides14& sv,
                  cudaStream_t st, const float* kmask = nullptr, int64_t kms = 0) {
  dim3 grid((unsigned)((H * L + 3) / 4), (unsigned)B);
  chord_fwd_simple_kernel<T><<<grid, 128, 4 * D * sizeof(float), st>>>(
      (const T*)q, (const T*)k, (const T*)v, alpha, beta, mu, ssmax, log_n, (T*)out, (int)H, (int)Hkv, (int)L,
      (int)S, (int)D, (int)q_start, scale, eps, sv, kmask, kms);
  return check_launch("chord_fwd_simple");
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

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" int64_t motif_b200_chord_workspace_bytes(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int) {
  return 0;
}

// The testing knob MB_FORCE_CHORD_MMA_SYNC keeps 16-bit D = 64 prefill on the mma.sync kernel
// (the tcgen05 kernel is the default) so tests can cross-check the two.
static bool chord_tc_disabled() { return forced(MB_FORCE_CHORD_MMA_SYNC); }

template <typename T, int G, bool KM>
int launch_tc_g(const void* q, const void* k, const void* v, const float* alpha, const float* beta, const float* mu,
                const float* ssmax, const float* log_n, void* out, int64_t B, int64_t H, int64_t Hkv, int64_t L,
                int64_t S, int64_t q_start, float scale, float eps, const int64_t* strides, const Strides14& sv,
                cudaStream_t st, const float* kmask, int64_t kms) {
  using Lay = TcSmemLayout<G>;
  CUtensorMap tmQ, tmK, tmV;
  {
    const uint64_t dims[4] = {64, (uint64_t)H, (uint64_t)L, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)strides[1] * 2, (uint64_t)strides[2] * 2, (uint64_t)strides[0] * 2};
    const uint32_t box[4] = {64, (uint32_t)G, (uint32_t)Lay::BMQ, 1};
    int rc = encode_tile_map(&tmQ, q, 2, 4, dims, str, box, 128);
    if (rc) return rc;
  }
  {
    const uint64_t dims[4] = {64, (uint64_t)S, (uint64_t)Hkv, (uint64_t)B};
    const uint32_t box[4] = {64, (uint32_t)tc::kKeys, 1, 1};
    const uint64_t sk[3] = {(uint64_t)strides[5] * 2, (uint64_t)strides[4] * 2, (uint64_t)strides[3] * 2};
    const uint64_t svv[3] = {(uint64_t)strides[8] * 2, (uint64_t)strides[7] * 2, (uint64_t)strides[6] * 2};
    int rc = encode_tile_map(&tmK, k, 2, 4, dims, sk, box, 128);
    if (!rc) rc = encode_tile_map(&tmV, v, 2, 4, dims, svv, box, 128);
    if (rc) return rc;
  }
  auto kern = chord_tc_kernel<T, G, KM>;
  if (int rc = ensure_smem_attr((const void*)kern, Lay::alloc)) return rc;
  const int GS = (int)(H / Hkv);
  dim3 grid((unsigned)((L + 2 * Lay::BMQ - 1) / (2 * Lay::BMQ)), (unsigned)(Hkv * (GS / G)), (unsigned)B);
  kern<<<grid, 512, Lay::alloc, st>>>(tmQ, tmK, tmV, alpha, beta, mu, ssmax, log_n, (T*)out, (int)H, (int)Hkv, (int)L,
                                     (int)S, (int)q_start, scale, eps, sv, kmask, kms);
  return check_launch("chord_attention (tcgen05)");
}

template <typename T, bool KM>
int launch_tc_km(int G, const void* q, const void* k, const void* v, const float* alpha, const float* beta,
                 const float* mu, const float* ssmax, const float* log_n, void* out, int64_t B, int64_t H,
                 int64_t Hkv, int64_t L, int64_t S, int64_t q_start, float scale, float eps, const int64_t* strides,
                 const Strides14& sv, cudaStream_t st, const float* kmask, int64_t kms) {
  switch (G) {
    case 8: return launch_tc_g<T, 8, KM>(q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps, strides, sv, st, kmask, kms);
    case 4: return launch_tc_g<T, 4, KM>(q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps, strides, sv, st, kmask, kms);
    case 2: return launch_tc_g<T, 2, KM>(q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps, strides, sv, st, kmask, kms);
    default: return launch_tc_g<T, 1, KM>(q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps, strides, sv, st, kmask, kms);
  }
}

template <typename T>
int launch_tc(int G, const void* q, const void* k, const void* v, const float* alpha, const float* beta,
              const float* mu, const float* ssmax, const float* log_n, void* out, int64_t B, int64_t H, int64_t Hkv,
              int64_t L, int64_t S, int64_t q_start, float scale, float eps, const int64_t* strides,
              const Strides14& sv, cudaStream_t st, const float* kmask = nullptr, int64_t kms = 0) {
  if (kmask)
    return launch_tc_km<T, true>(G, q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale,
                                 eps, strides, sv, st, kmask, kms);
  return launch_tc_km<T, false>(G, q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps,
                                strides, sv, st, nullptr, 0);
}

static int chord_attention_impl(const void* q, const void* k, const void* v, const float* alpha, const float* beta,
                                const float* mu, const float* ssmax, const float* log_n, void* out, int64_t B,
                                int64_t H, int64_t Hkv, int64_t L, int64_t S, int64_t D, int64_t q_start, float scale,
                                float eps, const int64_t* strides, int dtype, const float* kmask, int64_t kms,
                                void* stream) {
  MB_REQUIRE(strides, MB_ERR_ARG, "chord: null strides");
  MB_REQUIRE(B >= 0 && B < 65536 && H > 0 && Hkv > 0 && L >= 0 && S >= 0 && D > 0, MB_ERR_SHAPE,
             "chord: bad shape");
  MB_REQUIRE(H % Hkv == 0, MB_ERR_SHAPE, "chord: num_heads %lld not divisible by num_kv_heads %lld", (long long)H,
             (long long)Hkv);
  MB_REQUIRE(q_start >= 0 && L < (1LL << 30) && S < (1LL << 30), MB_ERR_SHAPE, "chord: bad q_start / lengths");
  MB_REQUIRE(D <= 128, MB_ERR_UNSUPPORTED, "chord: head dim %lld > 128", (long long)D);
  if (B == 0 || L == 0) return MB_OK;
  MB_REQUIRE(q && k && v && alpha && beta && mu && ssmax && log_n && out, MB_ERR_ARG, "chord: null pointer");
  Strides14 sv;
  for (int i = 0; i < 14; ++i) sv.s[i] = strides[i];
  cudaStream_t st = (cudaStream_t)stream;
  const int GS = (int)(H / Hkv);
  int G = 1;
  for (int c : {8, 4, 2})
    if (GS % c == 0) {
      G = c;
      break;
    }
  bool aligned = ((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 == 0;
  for (int i = 0; i < 9; ++i) aligned = aligned && strides[i] % 8 == 0;
  aligned = aligned && (strides[9] % 2 == 0) && (strides[10] % 2 == 0) && (strides[11] % 2 == 0) &&
            ((uintptr_t)out % 4 == 0);
  const bool mma_ok = dtype != MB_F32 && aligned && (D == 16 || D == 32 || D == 64);
  // tensor-core (tcgen05) path: 16-bit, D = 64, 16-byte aligned rows for the tensor maps and
  // the row stores, key positions within the 32-bit tensor-map coordinate range
  bool tc_ok = dtype != MB_F32 && D == 64 && ((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) % 16 == 0;
  for (int i = 0; i < 12; ++i) tc_ok = tc_ok && strides[i] % 8 == 0 && strides[i] > 0;
  tc_ok = tc_ok && S >= 1 && S < (1LL << 31) && L < (1LL << 31) && !chord_tc_disabled();
  return dispatch_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if constexpr (sizeof(T) == 2) {
      if (tc_ok) return launch_tc<T>(G, q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale,
                                     eps, strides, sv, st, kmask, kms);
      if (mma_ok && kmask == nullptr)  // the mma.sync kernel takes no key bias: masked calls use the simple one
        return launch_mma<T>(D, G, q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, q_start, scale, eps,
                             sv, st);
    }
    return launch_simple<T>(q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, D, q_start, scale, eps,
                            sv, st, kmask, kms);
  });
}

extern "C" int motif_b200_chord_attention(const void* q, const void* k, const void* v, const float* alpha,
                                          const float* beta, const float* mu, const float* ssmax, const float* log_n,
                                          void* out, int64_t B, int64_t H, int64_t Hkv, int64_t L, int64_t S,
                                          int64_t D, int64_t q_start, float scale, float eps, const int64_t* strides,
                                          int dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  return chord_attention_impl(q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, D, q_start, scale, eps,
                              strides, dtype, nullptr, 0, stream);
}

extern "C" int motif_b200_chord_attention_masked(const void* q, const void* k, const void* v, const float* alpha,
                                                 const float* beta, const float* mu, const float* ssmax,
                                                 const float* log_n, void* out, int64_t B, int64_t H, int64_t Hkv,
                                                 int64_t L, int64_t S, int64_t D, int64_t q_start, float scale,
                                                 float eps, const int64_t* strides, const float* key_bias,
                                                 int64_t key_bias_stride, int dtype, void* stream) {
  MB_REQUIRE(key_bias != nullptr || B == 0 || L == 0, MB_ERR_ARG, "chord (masked): null key bias");
  MB_REQUIRE(key_bias_stride >= S, MB_ERR_SHAPE, "chord (masked): key bias row stride %lld below S %lld",
             (long long)key_bias_stride, (long long)S);
  return chord_attention_impl(q, k, v, alpha, beta, mu, ssmax, log_n, out, B, H, Hkv, L, S, D, q_start, scale, eps,
                              strides, dtype, key_bias, key_bias_stride, stream);
}

extern "C" int64_t motif_b200_chord_decode_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t D,
                                                           int max_splits) {
  return (int64_t)max_splits * B * H * T * (D + 2) * (int64_t)sizeof(float);
}

static int chord_decode_impl(const void* q, const void* k_cache, const void* v_cache, int64_t cap,
                             const int32_t* len_dev, int64_t len_host, const float* alpha, const float* beta,
                             const float* mu, const float* ssmax, void* out, int64_t out_stride, int64_t B, int64_t H,
                             int64_t Hkv, int64_t T, int64_t D, float scale, float eps, int max_splits,
                             void* workspace, int64_t workspace_bytes, int dtype, const float* kmask, int64_t kms,
                             void* stream) {
  MB_REQUIRE(q && k_cache && v_cache && alpha && beta && mu && ssmax && out && workspace, MB_ERR_ARG,
             "chord_decode: null pointer");
  MB_REQUIRE(B > 0 && B < 65536 && H > 0 && Hkv > 0 && H % Hkv == 0 && T > 0 && cap > 0, MB_ERR_SHAPE,
             "chord_decode: bad shape");
  MB_REQUIRE((H / Hkv) * T <= 16, MB_ERR_UNSUPPORTED, "chord_decode: (H/Hkv)*T = %lld > 16",
             (long long)((H / Hkv) * T));
  MB_REQUIRE(max_splits >= 1 && max_splits <= 1024, MB_ERR_ARG, "chord_decode: max_splits %d", max_splits);
  MB_REQUIRE(workspace_bytes >= motif_b200_chord_decode_workspace_bytes(B, H, T, D, max_splits), MB_ERR_ARG,
             "chord_decode: workspace too small");
  MB_REQUIRE(len_dev != nullptr || (len_host >= T && len_host <= cap), MB_ERR_ARG, "chord_decode: bad length");
  MB_REQUIRE(((uintptr_t)k_cache | (uintptr_t)v_cache) % 16 == 0, MB_ERR_ALIGN, "chord_decode: cache alignment");
  MB_REQUIRE(B * Hkv < 65536 && cap < (1LL << 31), MB_ERR_SHAPE, "chord_decode: B*Hkv or cap too large");
  cudaStream_t st = (cudaStream_t)stream;
  return dispatch_dtype(dtype, [&](auto t) {
    using Tt = decltype(t);
    auto go = [&](auto dc) {
      constexpr int DD = decltype(dc)::value;
      dim3 grid((unsigned)max_splits, (unsigned)(B * Hkv));
      const int R = (int)((H / Hkv) * T);
      if constexpr (sizeof(Tt) == 2 && DD == 64) {
        if (B * Hkv * cap < (1LL << 31) && (uintptr_t)q % 4 == 0 && !force_scalar_decode()) {
          CUtensorMap tmK, tmV;
          const uint64_t rows = (uint64_t)(B * Hkv * cap);
          int rc = encode_tile_map_2d(&tmK, k_cache, 2, DD, rows, DD * 2, DD, kDecTile, 128);
          if (!rc) rc = encode_tile_map_2d(&tmV, v_cache, 2, DD, rows, DD * 2, DD, kDecTile, 128);
          if (rc) return rc;
          const int smem = 2 * kDecStages * kDecTile * DD * 2 + kDecStages * 8 + 1024;
          auto launch_mma = [&](auto rhc) {  // RH = 1: every query row is in the first 8 MMA rows
            auto kern = chord_decode_mma_kernel<Tt, decltype(rhc)::value>;
            if (int rc2 = ensure_smem_attr((const void*)kern, smem)) return rc2;
            kern<<<grid, 128, smem, st>>>(tmK, tmV, (const Tt*)q, cap, len_dev, (int)len_host, alpha, beta, mu,
                                          ssmax, (float*)workspace, (int)B, (int)H, (int)Hkv, (int)T, max_splits,
                                          scale, eps, kmask, kms);
            return check_launch("chord_decode");
          };
          rc = R <= 8 ? launch_mma(std::integral_constant<int, 1>{}) : launch_mma(std::integral_constant<int, 2>{});
          if (rc) return rc;
          chord_merge_kernel<Tt, DD><<<(unsigned)((B * T * H + 3) / 4), 128, 0, st>>>(
              (const float*)workspace, (Tt*)out, out_stride, (int)B, (int)H, (int)T, max_splits);
          return check_launch("chord_merge");
        }
      }
      auto launch = [&](auto rmc) {
        constexpr int RM = decltype(rmc)::value;
        auto kern = chord_decode_kernel<Tt, DD, RM>;
        const int smem = (int)sizeof(DecodeSmem<Tt, DD, RM>);
        if (int rc2 = ensure_smem_attr((const void*)kern, smem)) return rc2;
        kern<<<grid, 128, smem, st>>>((const Tt*)q, (const Tt*)k_cache, (const Tt*)v_cache, cap, len_dev,
                                      (int)len_host, alpha, beta, mu, ssmax, (float*)workspace, (int)B, (int)H,
                                      (int)Hkv, (int)T, max_splits, scale, eps, kmask, kms);
        return check_launch("chord_decode");
      };
      int rc = R <= 4 ? launch(std::integral_constant<int, 4>{})
                      : R <= 8 ? launch(std::integral_constant<int, 8>{}) : launch(std::integral_constant<int, 16>{});
      if (rc) return rc;
      chord_merge_kernel<Tt, DD><<<(unsigned)((B * T * H + 3) / 4), 128, 0, st>>>(
          (const float*)workspace, (Tt*)out, out_stride, (int)B, (int)H, (int)T, max_splits);
      return check_launch("chord_merge");
    };
    switch (D) {
      case 32: return go(std::integral_constant<int, 32>{});
      case 64: return go(std::integral_constant<int, 64>{});
      default: return set_error(MB_ERR_UNSUPPORTED, "chord_decode: head dim %lld", (long long)D);
    }
  });
}

extern "C" int motif_b200_chord_decode(const void* q, const void* k_cache, const void* v_cache, int64_t cap,
                                       const int32_t* len_dev, int64_t len_host, const float* alpha,
                                       const float* beta, const float* mu, const float* ssmax, void* out,
                                       int64_t out_stride, int64_t B, int64_t H, int64_t Hkv, int64_t T, int64_t D,
                                       float scale, float eps, int max_splits, void* workspace,
                                       int64_t workspace_bytes, int dtype, void* stream) {
  return chord_decode_impl(q, k_cache, v_cache, cap, len_dev, len_host, alpha, beta, mu, ssmax, out, out_stride, B, H,
                           Hkv, T, D, scale, eps, max_splits, workspace, workspace_bytes, dtype, nullptr, 0, stream);
}

extern "C" int motif_b200_chord_decode_masked(const void* q, const void* k_cache, const void* v_cache, int64_t cap,
                                              const int32_t* len_dev, int64_t len_host, const float* alpha,
                                              const float* beta, const float* mu, const float* ssmax, void* out,
                                              int64_t out_stride, int64_t B, int64_t H, int64_t Hkv, int64_t T,
                                              int64_t D, float scale, float eps, int max_splits,
                                              const float* key_bias, int64_t key_bias_stride, void* workspace,
                                              int64_t workspace_bytes, int dtype, void* stream) {
  MB_REQUIRE(key_bias != nullptr, MB_ERR_ARG, "chord_decode (masked): null key bias");
  MB_REQUIRE(key_bias_stride >= (len_dev ? cap : len_host), MB_ERR_SHAPE,
             "chord_decode (masked): key bias row stride %lld below the attended length", (long long)key_bias_stride);
  return chord_decode_impl(q, k_cache, v_cache, cap, len_dev, len_host, alpha, beta, mu, ssmax, out, out_stride, B, H,
                           Hkv, T, D, scale, eps, max_splits, workspace, workspace_bytes, dtype, key_bias,
                           key_bias_stride, stream);
}

// Vectorised preparation for 16-bit rows with D in {32, 64, 128}: a group of D/8 lanes owns
// one (token, slot) row (slot = q head | k head | v head) as 16-byte vectors; the q / k RMS
// norms reduce over the group's lanes.  A warp takes one token's group of 32 / (D/8) slots,
// so all H + 2 Hkv slots of a token are read at once (decode has few tokens: one warp per
// token walking its slots in turn left the launch latency-bound).
template <typename T, int D>
__global__ void __launch_bounds__(256) chord_prep_vec_kernel(const T* __restrict__ proj, int64_t ps,
                                                             const T* __restrict__ qn_w, const T* __restrict__ kn_w,
                                                             T* __restrict__ qo, T* __restrict__ kc, T* __restrict__ vc,
                                                             int64_t cap, const int32_t* __restrict__ pos_dev,
                                                             int64_t pos_host, int64_t rows, int Tn, int H, int Hkv,
                                                             float eps, SwigluRole<T> sw, int main_blocks) {
  constexpr int LPS = D / 8;       // lanes per slot
  constexpr int SPI = 32 / LPS;    // slots per warp iteration
  if ((int)blockIdx.x >= main_blocks) {  // trailing CTAs: the decoder's SwiGLU activation
    swiglu_role_run<T>(sw, (int64_t)(blockIdx.x - main_blocks) * 256 + threadIdx.x,
                       (int64_t)(gridDim.x - main_blocks) * 256);
    return;
  }
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPS, grp = lane / LPS;
  // one warp per (token, group of SPI slots): every slot of a token is read at once
  const int slots = H + 2 * Hkv;
  const int nchunk = (slots + SPI - 1) / SPI;
  const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t tok = wid / nchunk;
  if (tok >= rows) return;
  const int s0 = (int)(wid % nchunk) * SPI;
  const int b = (int)(tok / Tn), t = (int)(tok % Tn);
  const int64_t pos = (pos_dev ? (int64_t)*pos_dev : pos_host) + t;
  const bool pos_ok = pos >= 0 && pos < cap;  // a device-side position past the capacity skips the cache write
  const T* src_row = proj + tok * ps;
  {
    const int slot = s0 + grp;
    const bool act = slot < slots;  // lanes past the last slot still join the reductions
    uint4 raw = make_uint4(0, 0, 0, 0), wr = make_uint4(0, 0, 0, 0);
    if (act) raw = *reinterpret_cast<const uint4*>(src_row + (int64_t)slot * D + sub * 8);
    if (slot < H + Hkv) wr = *reinterpret_cast<const uint4*>((slot < H ? qn_w : kn_w) + sub * 8);  // with the row
    const T* e = reinterpret_cast<const T*>(&raw);
    float x[8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = to_f(e[i]);
      ss += x[i] * x[i];
    }
#pragma unroll
    for (int o2 = 1; o2 < LPS; o2 <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o2);
    if (!act) return;
    if (slot >= H + Hkv) {  // value: plain copy into the cache
      if (pos_ok) {
        const int kvh = slot - H - Hkv;
        *reinterpret_cast<uint4*>(vc + (((int64_t)b * Hkv + kvh) * cap + pos) * D + sub * 8) = raw;
      }
      return;
    }
    const float r = rsqrtf(ss / (float)D + eps);
    const T* we = reinterpret_cast<const T*>(&wr);
    uint4 outv;
    T* oe = reinterpret_cast<T*>(&outv);
#pragma unroll
    for (int i = 0; i < 8; ++i) oe[i] = from_f<T>(to_f(from_f<T>(x[i] * r)) * to_f(we[i]));
    if (slot < H) {
      *reinterpret_cast<uint4*>(qo + tok * H * D + (int64_t)slot * D + sub * 8) = outv;
    } else if (pos_ok) {
      *reinterpret_cast<uint4*>(kc + (((int64_t)b * Hkv + (slot - H)) * cap + pos) * D + sub * 8) = outv;
    }
  }
}

namespace mb {
namespace {
// q/k RMSNorm + cache append, with the decoder's SwiGLU activation in the same launch when
// `hid` > 0 and the vector kernel runs (otherwise a separate motif_b200_swiglu launch follows).
int chord_prep_impl(const void* proj, int64_t proj_stride, const void* qn_w, const void* kn_w, void* q,
                    void* k_cache, void* v_cache, int64_t cap, const int32_t* pos_dev, int64_t pos_host, int64_t B,
                    int64_t T, int64_t H, int64_t Hkv, int64_t D, float eps, int dtype, void* stream, const void* gu,
                    int64_t gs, void* act, int64_t as, int64_t hid) {
  MB_REQUIRE(proj && qn_w && kn_w && q && k_cache && v_cache, MB_ERR_ARG, "chord_prep: null pointer");
  MB_REQUIRE(B >= 0 && T >= 0 && H > 0 && Hkv > 0 && D > 0, MB_ERR_SHAPE, "chord_prep: bad shape");
  MB_REQUIRE(pos_dev != nullptr || pos_host + T <= cap, MB_ERR_SHAPE, "chord_prep: cache capacity %lld exceeded",
             (long long)cap);
  MB_REQUIRE(hid == 0 || (gu && act && hid > 0 && hid <= (1 << 24)), MB_ERR_ARG, "chord_prep_swiglu: bad MLP args");
  const int64_t rows = B * T;
  if (rows == 0) return MB_OK;
  const bool vec = dtype != MB_F32 && (D == 32 || D == 64 || D == 128) && proj_stride % 8 == 0 &&
                   ((uintptr_t)proj | (uintptr_t)qn_w | (uintptr_t)kn_w | (uintptr_t)q | (uintptr_t)k_cache |
                    (uintptr_t)v_cache) % 16 == 0;
  bool fused = false;
  const int rc = dispatch_dtype(dtype, [&](auto t) {
    using Tt = decltype(t);
    if constexpr (sizeof(Tt) == 2) {
      if (vec) {
        auto go = [&](auto dc) {
          constexpr int DD = decltype(dc)::value;
          constexpr int SPI = 32 / (DD / 8);
          const int64_t warps = rows * ((H + 2 * Hkv + SPI - 1) / SPI);
          const int64_t main_blocks = (warps + 7) / 8;
          SwigluRole<Tt> sw{(const Tt*)gu, gs, (Tt*)act, as, rows, 0};
          int64_t extra = 0;
          if (swiglu_role_ok(gu, gs, act, as, hid)) {
            sw.hid = (int)hid;
            extra = swiglu_role_blocks(rows, hid, 256);
            fused = true;
          }
          MB_REQUIRE(main_blocks + extra < (1LL << 31), MB_ERR_SHAPE, "chord_prep: too many rows");
          chord_prep_vec_kernel<Tt, DD><<<(unsigned)(main_blocks + extra), 256, 0, (cudaStream_t)stream>>>(
              (const Tt*)proj, proj_stride, (const Tt*)qn_w, (const Tt*)kn_w, (Tt*)q, (Tt*)k_cache, (Tt*)v_cache,
              cap, pos_dev, pos_host, rows, (int)T, (int)H, (int)Hkv, eps, sw, (int)main_blocks);
          return check_launch("chord_prep");
        };
        if (D == 32) return go(std::integral_constant<int, 32>{});
        if (D == 64) return go(std::integral_constant<int, 64>{});
        return go(std::integral_constant<int, 128>{});
      }
    }
    const int64_t warps = rows * (H + 2 * Hkv);
    chord_prep_kernel<Tt><<<(unsigned)((warps + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
        (const Tt*)proj, proj_stride, (const Tt*)qn_w, (const Tt*)kn_w, (Tt*)q, (Tt*)k_cache, (Tt*)v_cache, cap,
        pos_dev, pos_host, rows, (int)T, (int)H, (int)Hkv, (int)D, eps);
    return check_launch("chord_prep");
  });
  if (rc || hid == 0 || fused) return rc;
  return motif_b200_swiglu(gu, act, rows, hid, gs, as, dtype, stream);
}
}  // namespace
}  // namespace mb

extern "C" int motif_b200_chord_prep(const void* proj, int64_t proj_stride, const void* qn_w, const void* kn_w,
                                     void* q, void* k_cache, void* v_cache, int64_t cap, const int32_t* pos_dev,
                                     int64_t pos_host, int64_t B, int64_t T, int64_t H, int64_t Hkv, int64_t D,
                                     float eps, int dtype, void* stream) {
  return mb::chord_prep_impl(proj, proj_stride, qn_w, kn_w, q, k_cache, v_cache, cap, pos_dev, pos_host, B, T, H,
                             Hkv, D, eps, dtype, stream, nullptr, 0, nullptr, 0, 0);
}

extern "C" int motif_b200_chord_prep_swiglu(const void* proj, int64_t proj_stride, const void* qn_w,
                                            const void* kn_w, void* q, void* k_cache, void* v_cache, int64_t cap,
                                            const int32_t* pos_dev, int64_t pos_host, int64_t B, int64_t T,
                                            int64_t H, int64_t Hkv, int64_t D, float eps, const void* gu,
                                            int64_t gu_stride, void* act, int64_t act_stride, int64_t hid,
                                            int dtype, void* stream) {
  MB_REQUIRE(gu && act && hid > 0, MB_ERR_ARG, "chord_prep_swiglu: null MLP pointer or hid <= 0");
  return mb::chord_prep_impl(proj, proj_stride, qn_w, kn_w, q, k_cache, v_cache, cap, pos_dev, pos_host, B, T, H,
                             Hkv, D, eps, dtype, stream, gu, gu_stride, act, act_stride, hid);
}

// ------------------------------------------------------------------ allocation-free decode
// Some callers of the split-KV decode cannot allocate device memory for its workspace: a
// host runtime that reaches this library through a plain C FFI and has no CUDA allocator
// of its own, or a serving loop that must never call cudaMalloc mid-stream (it can stall
// the whole device and can fail under memory pressure at an arbitrary step).  For them the
// workspace lives in one fixed, file-scope device array.
namespace mb {
namespace {

constexpr int64_t kNoAllocScratchBytes = 8LL << 20;  // 8 MiB, held by every GPU that loads the library
__device__ __align__(256) float g_decode_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_decode_scratch in the current device's context.  In host code the
// array's name is only a host-side stand-in, so the address is looked up with the device
// current, on every call: the query is cheap, and a cached address would go stale if the
// context were torn down and recreated (cudaDeviceReset) with the module loaded elsewhere.
// The first call on a device may load the module; make it before any stream capture.
int scratch_on_current_device(float** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess || p == nullptr)
    return set_error(MB_ERR_CUDA, "chord_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  *out = static_cast<float*>(p);
  return MB_OK;
}

}  // namespace
}  // namespace mb

extern "C" int motif_b200_chord_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, int64_t cap,
                                               const int32_t* len_dev, int64_t len_host, const float* alpha,
                                               const float* beta, const float* mu, const float* ssmax, void* out,
                                               int64_t out_stride, int64_t B, int64_t H, int64_t Hkv, int64_t T,
                                               int64_t D, float scale, float eps, int max_splits, int dtype,
                                               void* stream) {
  MB_REQUIRE(B > 0 && H > 0 && T > 0 && D > 0 && max_splits >= 1, MB_ERR_SHAPE, "chord_decode_noalloc: bad shape");
  const int64_t need = motif_b200_chord_decode_workspace_bytes(B, H, T, D, max_splits);
  MB_REQUIRE(need <= mb::kNoAllocScratchBytes, MB_ERR_SHAPE,
             "chord_decode_noalloc: needs %lld bytes of scratch for B=%lld H=%lld T=%lld D=%lld splits=%d, above "
             "the fixed %lld-byte limit (use fewer splits or motif_b200_chord_decode with a workspace)",
             (long long)need, (long long)B, (long long)H, (long long)T, (long long)D, max_splits,
             (long long)mb::kNoAllocScratchBytes);
  float* ws = nullptr;
  const int rc = mb::scratch_on_current_device(&ws);
  if (rc != MB_OK) return rc;
  // Every split writes all of its partial rows (empty splits write m = -inf, l = 0), so the
  // scratch needs no clearing between calls.
  return motif_b200_chord_decode(q, k_cache, v_cache, cap, len_dev, len_host, alpha, beta, mu, ssmax, out,
                                 out_stride, B, H, Hkv, T, D, scale, eps, max_splits, ws, mb::kNoAllocScratchBytes,
                                 dtype, stream);
}

namespace mb {
int read_and_clear_gdn_timeouts(unsigned int* count);
int read_and_clear_skinny_timeouts(unsigned int* count);
int read_and_clear_gemm_timeouts(unsigned int* count);
}

extern "C" int motif_b200_wait_timeouts(uint32_t* count) {
  MB_REQUIRE(count != nullptr, MB_ERR_ARG, "wait_timeouts: null pointer");
  unsigned int v = 0, zero = 0, gdn = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess)
    return set_error(MB_ERR_CUDA, "wait_timeouts: %s", cudaGetErrorString(cudaGetLastError()));
  unsigned int sk = 0, gm = 0;
  int rc = mb::read_and_clear_gdn_timeouts(&gdn);
  if (!rc) rc = mb::read_and_clear_skinny_timeouts(&sk);
  if (!rc) rc = mb::read_and_clear_gemm_timeouts(&gm);
  if (rc) return rc;
  *count = v + gdn + sk + gm;
  return MB_OK;
}
