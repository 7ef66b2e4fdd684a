// Y = X . W^T for the model's dense projections (nn.Linear without bias), 16-bit operands,
// fp32 accumulation, on the 5th-generation tensor cores, with the elementwise work that follows
// each projection fused into the epilogue.
//
// One persistent CTA per SM walks output tiles of 128 rows (tokens) x up to 256 features.
// Three roles, one warp each for the first two:
//   * warp 0, one thread: streams 64-wide K slices of the X tile (128 x 64) and the W tile
//     (256 x 64) by tiled TMA (128-byte swizzle) into a 4-stage ring (48 KB a stage);
//   * warp 1, one thread: issues tcgen05.mma (M = 128, N = the tile's features, K = 16) into one
//     of two TMEM accumulators (2 x 256 fp32 columns: the whole TMEM of the SM), releasing each
//     ring stage with tcgen05.commit once the MMAs that read it complete, and handing a finished
//     accumulator to the epilogue with another commit;
//   * warps 2-5: the epilogue.  Thread = one token row (= one TMEM lane): tcgen05.ld of 32
//     columns at a time, the fused operation, 16-byte stores.  While they drain accumulator j the
//     MMA warp already fills accumulator j ^ 1.
// Tiles are ordered feature-tile fastest, so the CTAs in flight share X tiles through L2 and the
// weights (at most tens of MB) stay L2 resident.
//
// The output features are a list of up to four segments of W's rows, each with its epilogue:
//   STORE      y[r, c0 + j] = x.w_j                                        (plain projection)
//   SWIGLU     W rows in groups of 256: 128 value rows then the 128 gate rows of the same hidden
//              units; act[r, c0 + j] = round(round(v_j) * round(silu(round(g_j))))  (the SwiGLU
//              MLP activation, motif/ops/swiglu.py:252-253, with its bf16 rounding points)
//   GATE_RES   out[r, j] = round(round(round(a_j) * round(sigmoid(g[r, j]))) + m[r, j])
//              (chord_attn.py:254,313 o_proj(out) * G, plus the parallel residual decoder.py:208)
//   CONV_NORM  / CONV  the gated delta-net preparation of q, k (CONV_NORM) and v (CONV)
//              (gdn_attn.py:116-136,187-197): the causal depthwise conv over the last four
//              tokens of the same sequence (the carried conv state before a sequence's first
//              token), SiLU, and for q / k the L2 norm of each 64-channel head (times dk^-1/2 for
//              q); the raw inputs of each sequence's last three tokens become the new conv state
//   BETA_G     beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) from the a | b columns
// The preparation needs the three tokens before each output row.  In such a launch each epilogue
// warp carries its own three-row halo: the X tile is loaded as four 32-row boxes whose starts are
// 29 rows apart, three rows before the warp's 29 output rows, so a tile covers 116 output rows
// and each row's conv window lies in its own warp, read from the lanes below it by shuffles: no
// shared-memory exchange and no barrier between the epilogue warps.
// Every mbarrier wait is bounded; a role whose wait runs out counts itself
// (motif_b200_wait_timeouts), lets its issued copies / MMAs land and leaves.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace mb {

__device__ unsigned int g_gemm_wait_timeouts = 0;

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
#ifndef GEMM_STAGES
#define GEMM_STAGES 4
#endif
constexpr int kStages = GEMM_STAGES;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
#ifndef GEMM_EPI_WARPS
#define GEMM_EPI_WARPS 4
#endif
constexpr int kEpiWarps = GEMM_EPI_WARPS;  // per TMEM lane quarter kColSplit warps, one per column slice
constexpr int kColSplit = kEpiWarps / 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kCwBytes = 2048;                   // per epilogue warp: its channels' conv taps, or the
                                                 // a | b row values of the beta / g tile
constexpr int kStageOut = 4096;                  // per epilogue warp: two 2 KB output staging buffers
constexpr int kEpiWarpSmem = kCwBytes + kStageOut;
constexpr int kEpiSmem = kEpiWarps * kEpiWarpSmem;
constexpr int kSmemBytes = kStages * kStageBytes + kEpiSmem + 256 + 1024;  // + barriers + alignment
constexpr uint32_t kWait = 1u << 22;
constexpr int kMaxSeg = 8;
constexpr int kHalo = 3;                   // conv window rows before a token (conv kernel 4)
constexpr int kWarpRows = 32 - kHalo;      // output rows per epilogue warp in a PREP launch
constexpr int kPrepRows = 4 * kWarpRows;   // output rows per tile in a PREP launch (116)

enum { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_GATE_RES = 2, EPI_CONV_NORM = 3, EPI_CONV = 4, EPI_BETA_G = 5 };

struct Seg {
  int w_row0;        // first row of W in the segment
  int n;             // W rows in the segment
  int tiles;         // feature tiles of the segment
  int kind;
  void* out;         // output base (column 0 of the segment's output)
  int64_t ldo;
  const void* gate;  // GATE_RES: sigmoid input [M, n], row stride ldg
  int64_t ldg;
  const void* res;   // GATE_RES: residual [M, n], row stride ldr
  int64_t ldr;
  int chan0;         // CONV*: first conv channel of the segment
  float scale;       // CONV_NORM: factor after the L2 norm
  void* out2;        // BETA_G: g output (fp32 [M, H]); `out` receives beta
  int tma;           // 1: outputs leave by bulk tensor stores through omap[segment]
};

struct GemmParams {
  CUtensorMap omap[kMaxSeg];  // output tensor maps (16-bit outputs; box 32 columns x 32 or 29 rows)
  Seg seg[kMaxSeg];
  int nseg;
  int n_tiles;   // feature tiles over all segments
  int m_tiles;
  int M;
  int kblocks;
  int prep;      // 1: a launch with conv segments (116-row tiles, per-warp halos)
  // gated delta-net preparation
  int T;                 // tokens per sequence (rows are b * T + t)
  int C;                 // conv channels (q | k | v)
  int H;
  const void* conv_w;    // [C, 4] model dtype
  const void* conv_in;   // [B, 3, C] or null (zeros)
  void* conv_out;        // [B, 3, C] or null
  const void* A_log;     // [H] model dtype
  const void* dt_bias;   // [H] model dtype
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

struct TileInfo {
  int m0;     // first output row of the tile
  int seg, j, wrow, nvalid;
};
template <bool PREP>
__device__ __forceinline__ TileInfo tile_info(const GemmParams& p, int t) {
  TileInfo ti;
  const int mt = t / p.n_tiles;
  int nt = t - mt * p.n_tiles;
  ti.m0 = mt * (PREP ? kPrepRows : kBM);
  int s = 0;
  while (s + 1 < p.nseg && nt >= p.seg[s].tiles) {
    nt -= p.seg[s].tiles;
    ++s;
  }
  ti.seg = s;
  ti.j = nt;
  ti.wrow = p.seg[s].w_row0 + nt * kBN;
  ti.nvalid = min(kBN, p.seg[s].n - nt * kBN);
  return ti;
}

template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t u);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}

template <typename T>
__device__ __forceinline__ void store32(T* dst, const float* v, int valid, bool vec) {
  if (vec && valid >= 32) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u;
      u.x = pack2<T>(v[8 * q + 0], v[8 * q + 1]);
      u.y = pack2<T>(v[8 * q + 2], v[8 * q + 3]);
      u.z = pack2<T>(v[8 * q + 4], v[8 * q + 5]);
      u.w = pack2<T>(v[8 * q + 6], v[8 * q + 7]);
      d4[q] = u;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e)
      if (e < valid) dst[e] = from_f<T>(v[e]);
  }
}
template <typename T>
__device__ __forceinline__ void load32(const T* src, float* v, int valid, bool vec) {
  if (vec && valid >= 32) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 u = s4[q];
      const T* e8 = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[8 * q + e] = to_f(e8[e]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = e < valid ? to_f(src[e]) : 0.f;
  }
}

// Output staging: each epilogue warp owns two 2 KB buffers; a 32-column chunk of its rows (bf16
// pairs, 64 bytes a row) is written there in the 64-byte swizzled layout of the output tensor
// map (16-byte piece c of row r at piece c ^ ((r >> 1) & 3): conflict-free for 8 rows at a
// time) and leaves by one bulk tensor store, so the global writes are whole lines instead of
// 32 scattered rows per instruction.  A buffer is rewritten once the store issued from it two
// chunks earlier has finished reading it.
struct Stager {
  unsigned char* buf;
  int slot;
};
template <bool PREP>
__device__ __forceinline__ void emit_chunk(Stager& sgr, const CUtensorMap* map, int x, int y_box,
                                           const uint32_t (&w)[16], int lane) {
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory");
  __syncwarp();
  unsigned char* b = sgr.buf + sgr.slot * 2048;
  const int row = PREP ? lane - kHalo : lane;  // PREP boxes hold lanes 3..31
  if (row >= 0) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(b + row * 64 + ((c ^ ((row >> 1) & 3)) << 4)) =
          make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y_box), "r"(smem_u32(b))
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
  }
  sgr.slot ^= 1;
}
template <typename T>
__device__ __forceinline__ void pack32(const uint32_t (&acc)[32], uint32_t (&w)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = pack2<T>(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1]));
}

// Conv + SiLU of 32 channels of this row, warp-local: `acc` holds the row's raw projection
// (fp32 accumulator columns), rounded to T here; the three earlier tokens come from lanes 1..3
// below by shuffles (lanes 0..2 are the warp's halo rows and produce nothing), or, before a
// sequence's first token, from the carried conv state (zeros without one).  `cw` holds the 32
// channels' taps (4 each) in this warp's shared-memory copy.  y (two channels a word) =
// round(silu(round(conv))).  With `conv_out`, a sequence's last three tokens also write their raw
// inputs there.
template <typename T>
__device__ __forceinline__ void conv_chunk(const GemmParams& p, const uint32_t (&acc)[32], int ch, int r, bool live,
                                           const T* cw, uint32_t (&y)[16]) {
  int b = 0, t = 3;
  if (live) {
    b = r / p.T;
    t = r - b * p.T;
  }
  const T* cin = reinterpret_cast<const T*>(p.conv_in);
  const bool edge = live && t < 3;  // the window reaches before the sequence
  uint32_t* co = (live && p.conv_out && t >= p.T - 3)
                     ? reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.conv_out) + ((int64_t)b * 3 + (t - (p.T - 3))) * p.C + ch)
                     : nullptr;
  auto cin_word = [&](int slot, int i) -> uint32_t {
    return cin ? reinterpret_cast<const uint32_t*>(cin + ((int64_t)b * 3 + slot) * p.C + ch)[i] : 0u;
  };
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t x0 = pack2<T>(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1]));
    uint32_t x1 = __shfl_up_sync(0xffffffffu, x0, 1);
    uint32_t x2 = __shfl_up_sync(0xffffffffu, x0, 2);
    uint32_t x3 = __shfl_up_sync(0xffffffffu, x0, 3);
    if (edge) {
      if (t < 1) x1 = cin_word(2 + t, i);
      if (t < 2) x2 = cin_word(1 + t, i);
      x3 = cin_word(t, i);
    }
    if (co) co[i] = x0;
    const uint4 wq = *reinterpret_cast<const uint4*>(cw + 8 * i);  // taps of channels 2i, 2i + 1
    const float2 a3 = unpack2<T>(x3), a2 = unpack2<T>(x2), a1 = unpack2<T>(x1), a0 = unpack2<T>(x0);
    const float2 w0 = unpack2<T>(wq.x), w1 = unpack2<T>(wq.y), w2 = unpack2<T>(wq.z), w3 = unpack2<T>(wq.w);
    const float c0 = conv4f(w0.x, w0.y, w1.x, w1.y, a3.x, a2.x, a1.x, a0.x);
    const float c1 = conv4f(w2.x, w2.y, w3.x, w3.y, a3.y, a2.y, a1.y, a0.y);
    const float2 s2 = silu2_(round2<T>(c0, c1));
    y[i] = pack2<T>(s2.x, s2.y);
  }
}

// PREP launches (the gated delta-net projection) compile the conv / beta-g kinds and no gated
// residual; other launches the reverse, so each kernel carries only its own registers.
// Warp (q, h) handles TMEM lane quarter q and column slice h of the tile (feature columns
// [256 h / S, 256 (h + 1) / S) for S = kColSplit; a SwiGLU tile's outputs [128 h / S, ...)).
template <typename T, bool PREP>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const TileInfo& ti, uint32_t taddr, int q, int h,
                                              int lane, T* cws, Stager& sgr) {
  const Seg& sg = p.seg[ti.seg];
  const CUtensorMap* omap = &p.omap[ti.seg];
  const int y_box = PREP ? ti.m0 + kWarpRows * q : ti.m0 + 32 * q;  // first row of this warp's output box
  // output row of this thread: a PREP tile gives quarter q the rows m0 + 29 q + lane - 3 (lanes
  // 0..2 are its halo); other tiles map TMEM lane = row
  const int r = PREP ? ti.m0 + kWarpRows * q + lane - kHalo : ti.m0 + 32 * q + lane;
  const bool live = r < p.M && (!PREP || lane >= kHalo);
  const int c_lo = h * (kBN / kColSplit);
  const int c_hi = min(c_lo + kBN / kColSplit, ti.nvalid);
  if (PREP && (sg.kind == EPI_CONV_NORM || sg.kind == EPI_CONV)) {
    if (c_lo >= c_hi) return;
    const int ch0 = sg.chan0 + ti.j * kBN;
    // this warp's copy of its channels' conv taps (8 bytes a channel)
    __syncwarp();  // the previous tile's reads of the copy are done
    {
      constexpr int kPerLane = kBN / kColSplit / 64;  // 16-byte groups (two channels each) per lane
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.conv_w) + (int64_t)(ch0 + c_lo) * 4);
      uint4* dstw = reinterpret_cast<uint4*>(cws);
#pragma unroll
      for (int u = 0; u < kPerLane; ++u)
        if (c_lo + (lane * kPerLane + u) * 2 < c_hi) dstw[lane * kPerLane + u] = src[lane * kPerLane + u];
    }
    __syncwarp();
    const int nch = (c_hi - c_lo) / 32;
    uint32_t cur[32];
    tmem_ld32(taddr + c_lo, cur);
    tmem_wait_ld(cur);
    if (sg.kind == EPI_CONV) {
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        uint32_t nxt[32];
        if (c + 1 < nch) tmem_ld32(taddr + c_lo + 32 * (c + 1), nxt);  // in flight behind this chunk
        uint32_t y[16];
        conv_chunk<T>(p, cur, ch0 + c_lo + 32 * c, r, live, cws + 32 * c * 4, y);
        emit_chunk<PREP>(sgr, omap, ti.j * kBN + c_lo + 32 * c, y_box, y, lane);
        if (c + 1 < nch) {
          tmem_wait_ld(nxt);
#pragma unroll
          for (int e = 0; e < 32; ++e) cur[e] = nxt[e];
        }
      }
      return;
    }
    // 64-channel heads: two chunks, their sum of squares, then the scaled store
#pragma unroll 1
    for (int c = 0; c < nch; c += 2) {
      uint32_t nxt[32];
      tmem_ld32(taddr + c_lo + 32 * (c + 1), nxt);
      uint32_t y0[16], y1[16];
      conv_chunk<T>(p, cur, ch0 + c_lo + 32 * c, r, live, cws + 32 * c * 4, y0);
      tmem_wait_ld(nxt);
      if (c + 2 < nch) tmem_ld32(taddr + c_lo + 32 * (c + 2), cur);
      conv_chunk<T>(p, nxt, ch0 + c_lo + 32 * (c + 1), r, live, cws + 32 * (c + 1) * 4, y1);
      {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 u0 = unpack2<T>(y0[i]), u1 = unpack2<T>(y1[i]);
          ss = fmaf(u0.x, u0.x, ss);
          ss = fmaf(u0.y, u0.y, ss);
          ss = fmaf(u1.x, u1.x, ss);
          ss = fmaf(u1.y, u1.y, ss);
        }
        const float inv = l2_scale(ss, sg.scale);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 u0 = unpack2<T>(y0[i]), u1 = unpack2<T>(y1[i]);
          y0[i] = pack2<T>(u0.x * inv, u0.y * inv);
          y1[i] = pack2<T>(u1.x * inv, u1.y * inv);
        }
        emit_chunk<PREP>(sgr, omap, ti.j * kBN + c_lo + 32 * c, y_box, y0, lane);
        emit_chunk<PREP>(sgr, omap, ti.j * kBN + c_lo + 32 * c + 32, y_box, y1, lane);
      }
      if (c + 2 < nch) tmem_wait_ld(cur);
    }
    return;
  }
  if (PREP && sg.kind == EPI_BETA_G) {  // columns [0, H) = a, [H, 2H) = b; H <= 16
    if (h != 0) return;
    uint32_t acc[32];
    tmem_ld32(taddr, acc);
    tmem_wait_ld(acc);
    // through this lane's 64 bytes of the warp's shared-memory area (free between conv tiles), so
    // column H + h is read with a computed index
    __syncwarp();
    T* mine = cws + 32 * lane;
#pragma unroll
    for (int e = 0; e < 32; ++e) mine[e] = from_f<T>(__uint_as_float(acc[e]));
    if (live) {
      float* bo = reinterpret_cast<float*>(sg.out) + (int64_t)r * sg.ldo;
      float* go = reinterpret_cast<float*>(sg.out2) + (int64_t)r * sg.ldo;
      const T* al = reinterpret_cast<const T*>(p.A_log);
      const T* db = reinterpret_cast<const T*>(p.dt_bias);
#pragma unroll
      for (int hh = 0; hh < 16; ++hh) {
        if (hh < p.H) {
          const float a = to_f(mine[hh]);
          const float bb = to_f(mine[p.H + hh]);
          const float Aexp = -to_f(from_f<T>(expf(to_f(al[hh]))));  // A_log.exp() in the model dtype
          bo[hh] = to_f(from_f<T>(sigmoidf_(bb)));
          go[hh] = to_f(from_f<T>(Aexp * to_f(from_f<T>(softplusf_(to_f(from_f<T>(a + to_f(db[hh]))))))));
        }
      }
    }
    return;
  }
  if (sg.kind == EPI_SWIGLU) {
    // value columns [0, 128) and gate columns [128, 256) of the accumulator; this warp's outputs
    // are its slice of [0, 128).  The next chunk's TMEM columns load while this chunk is stored.
    const int s_lo = h * (kBN / 2 / kColSplit), s_hi = (h + 1) * (kBN / 2 / kColSplit);
    uint32_t rv[32], rg[32];
    tmem_ld32(taddr + s_lo, rv);
    tmem_ld32(taddr + kBN / 2 + s_lo, rg);
    tmem_wait_ld(rv);
    tmem_wait_ld(rg);
#pragma unroll 1
    for (int c = s_lo; c < s_hi; c += 32) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float o2[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float v = to_f(from_f<T>(__uint_as_float(rv[2 * i + k])));
          const float g = to_f(from_f<T>(__uint_as_float(rg[2 * i + k])));
          o2[k] = v * to_f(from_f<T>(siluf_(g)));
        }
        w[i] = pack2<T>(o2[0], o2[1]);
      }
      const bool more = c + 32 < s_hi;
      if (more) {
        tmem_ld32(taddr + c + 32, rv);
        tmem_ld32(taddr + kBN / 2 + c + 32, rg);
      }
      emit_chunk<PREP>(sgr, omap, ti.j * (kBN / 2) + c, y_box, w, lane);
      if (more) {
        tmem_wait_ld(rv);
        tmem_wait_ld(rg);
      }
    }
    return;
  }
  const int col0 = ti.j * kBN;
  T* dst = reinterpret_cast<T*>(sg.out) + (int64_t)r * sg.ldo + col0;
  const bool vec = (sg.ldo % 8 == 0) && (((uintptr_t)sg.out) % 16 == 0);
  if (sg.kind == EPI_STORE && sg.tma) {  // the next chunk's TMEM columns load while this one is stored
    if (c_lo >= c_hi) return;
    uint32_t ra[32];
    tmem_ld32(taddr + c_lo, ra);
    tmem_wait_ld(ra);
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 32) {
      uint32_t w[16];
      pack32<T>(ra, w);
      const bool more = c + 32 < c_hi;
      if (more) tmem_ld32(taddr + c + 32, ra);
      emit_chunk<PREP>(sgr, omap, col0 + c, y_box, w, lane);
      if (more) tmem_wait_ld(ra);
    }
    return;
  }
  if (sg.kind == EPI_STORE) {  // rows the bulk store cannot describe (unaligned): thread stores
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 64) {
      uint32_t r0[32], r1[32];
      tmem_ld32(taddr + c, r0);
      tmem_ld32(taddr + c + 32, r1);
      tmem_wait_ld(r0);
      tmem_wait_ld(r1);
      if (live) {
        float f0[32], f1[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          f0[e] = __uint_as_float(r0[e]);
          f1[e] = __uint_as_float(r1[e]);
        }
        store32<T>(dst + c, f0, c_hi - c, vec);
        if (c + 32 < c_hi) store32<T>(dst + c + 32, f1, c_hi - c - 32, vec);
      }
    }
    return;
  }
  if constexpr (PREP) return;
  // GATE_RES: the gate and residual rows of chunk c + 1 are requested before chunk c is combined,
  // so one chunk of global loads is always in flight behind the arithmetic
  const T* gp = reinterpret_cast<const T*>(sg.gate) + (int64_t)r * sg.ldg + col0;
  const T* mp = reinterpret_cast<const T*>(sg.res) + (int64_t)r * sg.ldr + col0;
  const bool vin = vec && (sg.ldg % 8 == 0) && (sg.ldr % 8 == 0) && (((uintptr_t)sg.gate | (uintptr_t)sg.res) % 16 == 0);
  if (c_lo >= c_hi) return;
  if (!vin || !sg.tma || ti.nvalid % 32 != 0) {  // unaligned rows or a partial chunk: element by element
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 32) {
      uint32_t ra[32];
      tmem_ld32(taddr + c, ra);
      tmem_wait_ld(ra);
      if (live) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (c + e < c_hi) {
            const float a = to_f(from_f<T>(__uint_as_float(ra[e])));
            const float gate = to_f(from_f<T>(sigmoidf_(to_f(gp[c + e]))));
            const float att = to_f(from_f<T>(a * gate));
            dst[c + e] = from_f<T>(att + to_f(mp[c + e]));
          }
        }
      }
    }
    return;
  }
  uint4 gq[4], mq[4];
  if (live) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      gq[u] = reinterpret_cast<const uint4*>(gp + c_lo)[u];
      mq[u] = reinterpret_cast<const uint4*>(mp + c_lo)[u];
    }
  }
#pragma unroll 1
  for (int c = c_lo; c < c_hi; c += 32) {
    uint32_t ra[32];
    tmem_ld32(taddr + c, ra);
    uint4 gn[4], mn[4];
    const bool more = live && c + 32 < c_hi;
    if (more) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        gn[u] = reinterpret_cast<const uint4*>(gp + c + 32)[u];
        mn[u] = reinterpret_cast<const uint4*>(mp + c + 32)[u];
      }
    }
    tmem_wait_ld(ra);
    {
      uint32_t w[16];
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // 8 columns: combine, pack
        const T* g8 = reinterpret_cast<const T*>(&gq[u]);
        const T* m8 = reinterpret_cast<const T*>(&mq[u]);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float o2[2];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const float a = to_f(from_f<T>(__uint_as_float(ra[8 * u + e + k])));
            const float gate = to_f(from_f<T>(sigmoidf_(to_f(g8[e + k]))));
            const float att = to_f(from_f<T>(a * gate));
            o2[k] = att + to_f(m8[e + k]);
          }
          w[4 * u + e / 2] = pack2<T>(o2[0], o2[1]);
        }
      }
      emit_chunk<PREP>(sgr, omap, col0 + c, y_box, w, lane);
    }
    if (more) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        gq[u] = gn[u];
        mq[u] = mn[u];
      }
    }
  }
}

// tmA: X in 128-row boxes; tmA4: X in 32-row boxes (PREP launches: one per epilogue warp, each
// starting three rows before that warp's output rows).
template <typename T, bool PREP>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                             const __grid_constant__ CUtensorMap tmA4,
                                                             const __grid_constant__ CUtensorMap tmB,
                                                             const __grid_constant__ GemmParams p) {
  constexpr uint32_t ab_fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ unsigned char gemm_smem_raw[];
  unsigned char* sm = gemm_smem_raw + ((1024u - (smem_u32(gemm_smem_raw) & 1023u)) & 1023u);
  unsigned char* epi_smem = sm + kStages * kStageBytes;  // per epilogue warp: conv taps of its tile
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStages * kStageBytes + kEpiSmem);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;  // [2] accumulator ready for the epilogue
  uint64_t* tempty = tfull + 2;       // [2] accumulator drained by the epilogue
  uint64_t* mdone = tempty + 2;       // every MMA of this CTA complete
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(mdone + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) tmem_alloc(sTmem, 512);
  if (tid == 32) {
    prefetch_tmap(PREP ? &tmA4 : &tmA);
    prefetch_tmap(&tmB);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps);
    }
    mbar_init(mdone, 1);
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;
  const int ntiles = p.m_tiles * p.n_tiles;
  bool failed = false;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < ntiles && !failed; t += gridDim.x) {
        const TileInfo ti = tile_info<PREP>(p, t);
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait_bounded(&empty[s], (uint32_t)(((it / kStages) & 1) ^ 1), kWait)) {
            failed = true;
            break;
          }
          unsigned char* st = sm + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          if constexpr (PREP) {
            // rows 32 w .. 32 w + 31 of the tile = X rows m0 + 29 w - 3 .. (a negative start reads zeros)
#pragma unroll
            for (int w = 0; w < 4; ++w)
              tma_load_2d(st + w * (kABytes / 4), &tmA4, kb * kBK, ti.m0 + kWarpRows * w - kHalo, &full[s]);
          } else {
            tma_load_2d(st, &tmA, kb * kBK, ti.m0, &full[s]);
          }
          tma_load_2d(st + kABytes, &tmB, kb * kBK, ti.wrow, &full[s]);
        }
      }
      if (failed) {  // the copies already issued land before the CTA leaves
        atomicAdd(&g_gemm_wait_timeouts, 1u);
        for (int u = max(0, it - kStages); u < it; ++u)
          mbar_wait_bounded(&full[u % kStages], (uint32_t)((u / kStages) & 1), kWait);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, jl = 0;
      for (int t = blockIdx.x; t < ntiles && !failed; t += gridDim.x, ++jl) {
        const TileInfo ti = tile_info<PREP>(p, t);
        const int acc = jl & 1;
        if (!mbar_wait_bounded(&tempty[acc], (uint32_t)(((jl >> 1) & 1) ^ 1), kWait)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const int nmma = (ti.nvalid + 15) & ~15;
        const uint32_t idesc = umma_idesc_f16(ab_fmt, kBM, nmma, 0, 0);
        const uint32_t d = tmem + (uint32_t)(acc * kBN);
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait_bounded(&full[s], (uint32_t)((it / kStages) & 1), kWait)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sm + s * kStageBytes), b_addr = a_addr + kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16_ss(d, umma_desc_sw128(a_addr + k * 32, 16, 1024), umma_desc_sw128(b_addr + k * 32, 16, 1024),
                        idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (failed) break;
        umma_commit(&tfull[acc]);
      }
      umma_commit(mdone);  // every MMA issued above, also on the failure path
      if (!mbar_wait_bounded(mdone, 0, kWait)) failed = true;
      if (failed) atomicAdd(&g_gemm_wait_timeouts, 1u);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int hcol = (warp - 2) >> 2;  // column slice
    unsigned char* mine = epi_smem + (warp - 2) * kEpiWarpSmem;
    T* cws = reinterpret_cast<T*>(mine);
    Stager sgr{mine + kCwBytes, 0};
    int jl = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++jl) {
      const TileInfo ti = tile_info<PREP>(p, t);
      const int acc = jl & 1;
      const bool ok = mbar_wait_bounded(&tfull[acc], (uint32_t)((jl >> 1) & 1), kWait);
      if (__any_sync(0xffffffffu, !ok)) {  // the epilogue warps are independent: each leaves alone
        if (lane == 0) atomicAdd(&g_gemm_wait_timeouts, 1u);
        break;
      }
      tc_fence_after();
      epilogue_tile<T, PREP>(p, ti, tmem + (uint32_t)(acc * kBN) + ((uint32_t)(q * 32) << 16), q, hcol, lane, cws,
                             sgr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");  // every output store complete
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------- CTA pairs
// The non-preparation projections run on pairs of CTAs (a cluster of two) that share each
// 256 x 256 output tile: CTA r holds X rows m0 + 128 r (its 128 accumulator rows) and the r-th
// half of the tile's W rows; the pair's leader issues tcgen05.mma.cta_group::2 (M = 256), which
// reads A and B from both CTAs' shared memory.  Per SM that halves the W traffic through shared
// memory and L2 against a one-CTA 128 x 256 tile, so a 6-stage ring of 32 KB stages (twice the
// bytes in flight per unit of work) covers the L2 latency that starved the one-CTA pipeline.
//   * both producers load into their own ring and complete transaction bytes on the LEADER's
//     stage barrier (the leader expects the pair's bytes); each refills a stage when its own
//     empty barrier says the leader's MMAs have read it;
//   * the leader's MMA thread commits each stage's release and each finished accumulator to the
//     barriers of both CTAs (one commit per CTA);
//   * each CTA's epilogue drains its own TMEM rows and arrives on the leader's "accumulator
//     free" barrier (remote arrive from the peer).
constexpr int kStages2 = 6;
constexpr int kHalfBBytes = (kBN / 2) * kBK * 2;   // 16 KB: this CTA's half of the W tile
constexpr int kStage2Bytes = kABytes + kHalfBBytes; // 32 KB
static_assert(kStages2 * kStage2Bytes <= kStages * kStageBytes, "the pair ring fits the one-CTA ring's space");

__device__ __forceinline__ uint32_t cluster_rank2() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync2() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// shared::cluster address of `local` (a shared::cta address) in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_rank(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
// X / W box into this CTA's shared memory, transaction bytes completed on the barrier at
// shared::cluster address `bar` (the leader's)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive (once) on the barrier at shared::cluster address `bar` when every MMA this thread issued has completed
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                                                               const __grid_constant__ CUtensorMap tmB2,
                                                               const __grid_constant__ GemmParams p) {
  constexpr uint32_t ab_fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ unsigned char gemm_smem_raw[];
  unsigned char* sm = gemm_smem_raw + ((1024u - (smem_u32(gemm_smem_raw) & 1023u)) & 1023u);
  unsigned char* epi_smem = sm + kStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStages * kStageBytes + kEpiSmem);
  uint64_t* empty = full + kStages2;
  uint64_t* tfull = empty + kStages2;
  uint64_t* tempty = tfull + 2;
  uint64_t* mdone = tempty + 2;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(mdone + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank2();
  const bool leader = rank == 0;
  if (warp == 0) tmem_alloc_pair(sTmem, 512);
  if (tid == 32) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB2);
    for (int i = 0; i < kStages2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * kEpiWarps);  // the epilogue warps of both CTAs
    }
    mbar_init(mdone, 1);
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync2();  // both CTAs' barriers exist before any copy or arrive crosses the pair
  tc_fence_after();
  const uint32_t tmem = *sTmem;
  const int npairs = gridDim.x >> 1, pair = blockIdx.x >> 1;
  const int ntiles = p.m_tiles * p.n_tiles;
  bool failed = false;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = pair; t < ntiles && !failed; t += npairs) {
        const TileInfo ti = tile_info<false>(p, t);
        const int m0 = (t / p.n_tiles) * (2 * kBM);
        const int nmma = (ti.nvalid + 15) & ~15;
        const int a_row = m0 + kBM * (int)rank, b_row = ti.wrow + (int)rank * (nmma / 2);
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const int s = it % kStages2;
          if (!mbar_wait_bounded(&empty[s], (uint32_t)(((it / kStages2) & 1) ^ 1), kWait)) {
            failed = true;
            break;
          }
          unsigned char* st = sm + s * kStage2Bytes;
          const uint32_t lead_full = map_rank(smem_u32(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * kStage2Bytes);
          tma_load_2d_pair(st, &tmA, kb * kBK, a_row, lead_full);
          tma_load_2d_pair(st + kABytes, &tmB2, kb * kBK, b_row, lead_full);
        }
      }
      if (failed) {
        atomicAdd(&g_gemm_wait_timeouts, 1u);
        if (leader)  // the pair's copies complete on the leader's barriers
          for (int u = max(0, it - kStages2); u < it; ++u)
            mbar_wait_bounded(&full[u % kStages2], (uint32_t)((u / kStages2) & 1), kWait);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int it = 0, jl = 0;
      for (int t = pair; t < ntiles && !failed; t += npairs, ++jl) {
        const TileInfo ti = tile_info<false>(p, t);
        const int acc = jl & 1;
        if (!mbar_wait_bounded(&tempty[acc], (uint32_t)(((jl >> 1) & 1) ^ 1), kWait)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const int nmma = (ti.nvalid + 15) & ~15;
        const uint32_t idesc = umma_idesc_f16(ab_fmt, 2 * kBM, nmma, 0, 0);
        const uint32_t d = tmem + (uint32_t)(acc * kBN);
        for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
          const int s = it % kStages2;
          if (!mbar_wait_bounded(&full[s], (uint32_t)((it / kStages2) & 1), kWait)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sm + s * kStage2Bytes), b_addr = a_addr + kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_pair(d, umma_desc_sw128(a_addr + k * 32, 16, 1024), umma_desc_sw128(b_addr + k * 32, 16, 1024), idesc,
                      (kb > 0 || k > 0) ? 1u : 0u);
          const uint32_t e_local = smem_u32(&empty[s]);
          umma_commit_pair(e_local);
          umma_commit_pair(map_rank(e_local, 1));
        }
        if (failed) break;
        const uint32_t f_local = smem_u32(&tfull[acc]);
        umma_commit_pair(f_local);
        umma_commit_pair(map_rank(f_local, 1));
      }
      umma_commit_pair(smem_u32(mdone));  // every MMA issued above, also on the failure path
      if (!mbar_wait_bounded(mdone, 0, kWait)) failed = true;
      if (failed) atomicAdd(&g_gemm_wait_timeouts, 1u);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int hcol = (warp - 2) >> 2;
    unsigned char* mine = epi_smem + (warp - 2) * kEpiWarpSmem;
    T* cws = reinterpret_cast<T*>(mine);
    Stager sgr{mine + kCwBytes, 0};
    int jl = 0;
    for (int t = pair; t < ntiles; t += npairs, ++jl) {
      TileInfo ti = tile_info<false>(p, t);
      ti.m0 = (t / p.n_tiles) * (2 * kBM) + kBM * (int)rank;  // this CTA's 128 rows of the pair tile
      const int acc = jl & 1;
      const bool ok = mbar_wait_bounded(&tfull[acc], (uint32_t)((jl >> 1) & 1), kWait);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) atomicAdd(&g_gemm_wait_timeouts, 1u);
        break;
      }
      tc_fence_after();
      epilogue_tile<T, false>(p, ti, tmem + (uint32_t)(acc * kBN) + ((uint32_t)(q * 32) << 16), q, hcol, lane, cws,
                              sgr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&tempty[acc]);
        else
          mbar_arrive_remote(map_rank(smem_u32(&tempty[acc]), 0));
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync2();  // every MMA, copy and cross-CTA arrive of the pair is done
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

int sm_count() {
  static int count[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (!count[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    count[dev] = n > 0 ? n : 148;
  }
  return count[dev];
}

template <typename T>
int launch_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M, int64_t K, GemmParams& p,
                cudaStream_t st) {
  CUtensorMap tmA, tmA4, tmB;
  int64_t wrows = 0;
  for (int s = 0; s < p.nseg; ++s) wrows = std::max<int64_t>(wrows, (int64_t)p.seg[s].w_row0 + p.seg[s].n);
  int rc = encode_tile_map_2d(&tmA, x, 2, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, kBK, kBM, 128);
  if (!rc) rc = encode_tile_map_2d(&tmA4, x, 2, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, kBK, kBM / 4, 128);
  if (!rc) rc = encode_tile_map_2d(&tmB, w, 2, (uint64_t)K, (uint64_t)wrows, (uint64_t)ldw * 2, kBK, kBN, 128);
  if (rc) return rc;
  for (int sidx = 0; sidx < p.nseg; ++sidx) {
    Seg& sg = p.seg[sidx];
    const int64_t width = sg.kind == EPI_SWIGLU ? sg.n / 2 : sg.n;
    sg.tma = sg.kind != EPI_BETA_G && sg.ldo % 8 == 0 && (uintptr_t)sg.out % 16 == 0 && sg.ldo >= width;
    if (sg.tma) {
      rc = encode_tile_map_2d(&p.omap[sidx], sg.out, 2, (uint64_t)width, (uint64_t)M, (uint64_t)sg.ldo * 2, 32,
                              p.prep ? kWarpRows : 32, 64);
      if (rc) return rc;
    }
    MB_REQUIRE(sg.tma || sg.kind == EPI_STORE || sg.kind == EPI_GATE_RES || sg.kind == EPI_BETA_G, MB_ERR_ALIGN,
               "gemm: segment %d output needs 16-byte aligned rows (row stride a multiple of 8)", sidx);
  }
  p.M = (int)M;
  p.kblocks = (int)(K / kBK);
  p.n_tiles = 0;
  for (int s = 0; s < p.nseg; ++s) p.n_tiles += p.seg[s].tiles;
  if (!p.prep) {  // CTA pairs on 256 x 256 tiles
    CUtensorMap tmB2;
    rc = encode_tile_map_2d(&tmB2, w, 2, (uint64_t)K, (uint64_t)wrows, (uint64_t)ldw * 2, kBK, kBN / 2, 128);
    if (rc) return rc;
    auto kern = gemm_pair_kernel<T>;
    if (int e = ensure_smem_attr((const void*)kern, kSmemBytes)) return e;
    p.m_tiles = (int)((M + 2 * kBM - 1) / (2 * kBM));
    const int64_t ntiles = (int64_t)p.m_tiles * p.n_tiles;
    const int npairs = (int)std::min<int64_t>(ntiles, sm_count() / 2);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(2 * npairs));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, tmA, tmB2, p);
    return check_launch("gemm (CTA pairs)");
  }
  auto kern = gemm_tc_kernel<T, true>;
  if (int e = ensure_smem_attr((const void*)kern, kSmemBytes)) return e;
  p.m_tiles = (int)((M + kPrepRows - 1) / kPrepRows);
  const int64_t ntiles = (int64_t)p.m_tiles * p.n_tiles;
  const int grid = (int)std::min<int64_t>(ntiles, sm_count());
  kern<<<grid, kThreads, kSmemBytes, st>>>(tmA, tmA4, tmB, p);
  return check_launch("gemm");
}

int gemm_impl(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M, int64_t K, GemmParams& p, int dtype,
              void* stream) {
  MB_REQUIRE(x && w, MB_ERR_ARG, "gemm: null operand");
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "gemm: 16-bit dtypes only");
  MB_REQUIRE(M >= 0 && M < (1LL << 31) && K > 0 && K < (1LL << 31), MB_ERR_SHAPE, "gemm: bad M / K");
  MB_REQUIRE(K % kBK == 0, MB_ERR_UNSUPPORTED, "gemm: K must be a multiple of %d (got %lld)", kBK, (long long)K);
  MB_REQUIRE(ldx % 8 == 0 && ldw % 8 == 0 && ldx >= K && ldw >= K && ((uintptr_t)x | (uintptr_t)w) % 16 == 0,
             MB_ERR_ALIGN, "gemm: X / W rows must be 16-byte aligned (row strides multiples of 8)");
  for (int s = 0; s < p.nseg; ++s) {
    const Seg& sg = p.seg[s];
    MB_REQUIRE(sg.out && sg.n > 0, MB_ERR_ARG, "gemm: segment %d has no output", s);
    MB_REQUIRE(sg.kind != EPI_GATE_RES || (sg.gate && sg.res), MB_ERR_ARG, "gemm: gated residual inputs missing");
    MB_REQUIRE(sg.kind != EPI_SWIGLU || sg.n % kBN == 0, MB_ERR_SHAPE,
               "gemm: SwiGLU segment width %d must be a multiple of %d (128 value + 128 gate rows a group)", sg.n,
               kBN);
    MB_REQUIRE(!(sg.kind == EPI_CONV_NORM || sg.kind == EPI_CONV || sg.kind == EPI_BETA_G) || p.prep,
               MB_ERR_ARG, "gemm: preparation segments need the halo tiling");
    MB_REQUIRE(!p.prep || sg.kind != EPI_GATE_RES, MB_ERR_ARG, "gemm: no gated residual in a preparation launch");
  }
  if (M == 0) return MB_OK;
  cudaStream_t st = (cudaStream_t)stream;
  return dtype == MB_BF16 ? launch_gemm<__nv_bfloat16>(x, ldx, w, ldw, M, K, p, st)
                          : launch_gemm<__half>(x, ldx, w, ldw, M, K, p, st);
}

Seg make_seg(int w_row0, int64_t n, int kind, void* out, int64_t ldo) {
  Seg s = {};
  s.w_row0 = w_row0;
  s.n = (int)n;
  s.tiles = (int)((n + kBN - 1) / kBN);
  s.kind = kind;
  s.out = out;
  s.ldo = ldo;
  return s;
}

}  // namespace

int read_and_clear_gemm_timeouts(unsigned int* count) {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_wait_timeouts, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_gemm_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess)
    return set_error(MB_ERR_CUDA, "wait_timeouts: %s", cudaGetErrorString(cudaGetLastError()));
  *count = v;
  return MB_OK;
}

}  // namespace mb

extern "C" int motif_b200_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                               int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  using namespace mb;
  MB_REQUIRE(y && N > 0 && N < (1LL << 30), MB_ERR_ARG, "gemm: null output or bad N");
  GemmParams p = {};
  p.nseg = 1;
  p.seg[0] = make_seg(0, N, EPI_STORE, y, ldy);
  return gemm_impl(x, ldx, w, ldw, M, K, p, dtype, stream);
}

extern "C" int motif_b200_gemm_proj_swiglu(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M,
                                           int64_t K, int64_t n_plain, void* y, int64_t ldy, int64_t hid, void* act,
                                           int64_t ld_act, int dtype, void* stream) {
  using namespace mb;
  MB_REQUIRE(n_plain >= 0 && hid >= 0 && n_plain + 2 * hid > 0 && n_plain + 2 * hid < (1LL << 30), MB_ERR_SHAPE,
             "gemm_proj_swiglu: bad widths");
  MB_REQUIRE(hid % 128 == 0, MB_ERR_UNSUPPORTED, "gemm_proj_swiglu: hid %lld must be a multiple of 128",
             (long long)hid);
  GemmParams p = {};
  if (n_plain > 0) {
    MB_REQUIRE(y, MB_ERR_ARG, "gemm_proj_swiglu: null projection output");
    p.seg[p.nseg++] = make_seg(0, n_plain, EPI_STORE, y, ldy);
  }
  if (hid > 0) {
    MB_REQUIRE(act, MB_ERR_ARG, "gemm_proj_swiglu: null activation output");
    p.seg[p.nseg++] = make_seg((int)n_plain, 2 * hid, EPI_SWIGLU, act, ld_act);
  }
  return gemm_impl(x, ldx, w, ldw, M, K, p, dtype, stream);
}

extern "C" int motif_b200_gemm_gdn_prep(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t B,
                                        int64_t T, int64_t K, int64_t H, int64_t dk, int64_t dv, int64_t hid,
                                        const void* conv_w, const void* A_log, const void* dt_bias,
                                        const void* conv_in, void* conv_out, void* q, void* k, void* v,
                                        float* beta, float* g, void* gate, void* act, int64_t ld_act, int dtype,
                                        void* stream) {
  using namespace mb;
  MB_REQUIRE(conv_w && A_log && dt_bias && q && k && v && beta && g && gate, MB_ERR_ARG,
             "gemm_gdn_prep: null pointer");
  MB_REQUIRE(B > 0 && T >= 3 && B * T < (1LL << 31) && H > 0 && H <= 16, MB_ERR_SHAPE,
             "gemm_gdn_prep: needs T >= 3 and 1 <= H <= 16 (B=%lld T=%lld H=%lld)", (long long)B, (long long)T,
             (long long)H);
  MB_REQUIRE(dk == 64 && dv % 32 == 0 && dv > 0, MB_ERR_UNSUPPORTED,
             "gemm_gdn_prep: built for 64-channel q / k heads and dv a multiple of 32 (dk=%lld dv=%lld)",
             (long long)dk, (long long)dv);
  MB_REQUIRE(hid % 128 == 0, MB_ERR_UNSUPPORTED, "gemm_gdn_prep: hid %lld must be a multiple of 128", (long long)hid);
  MB_REQUIRE(((uintptr_t)conv_w | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)gate |
              (uintptr_t)conv_out | (uintptr_t)conv_in) % 16 == 0,
             MB_ERR_ALIGN, "gemm_gdn_prep: outputs, conv weights and conv states must be 16-byte aligned");
  MB_REQUIRE(conv_out == nullptr || conv_out != conv_in, MB_ERR_ARG, "gemm_gdn_prep: conv_out must not alias conv_in");
  const int64_t Hk = H * dk, Hv = H * dv;
  GemmParams p = {};
  p.prep = 1;
  p.T = (int)T;
  p.C = (int)(2 * Hk + Hv);
  p.H = (int)H;
  p.conv_w = conv_w;
  p.conv_in = conv_in;
  p.conv_out = conv_out;
  p.A_log = A_log;
  p.dt_bias = dt_bias;
  // W rows: q | k | v | a | b | g | gate_up (regrouped for the SwiGLU epilogue)
  Seg sq = make_seg(0, Hk, EPI_CONV_NORM, q, Hk);
  sq.chan0 = 0;
  sq.scale = 1.0f / sqrtf((float)dk);
  Seg sk = make_seg((int)Hk, Hk, EPI_CONV_NORM, k, Hk);
  sk.chan0 = (int)Hk;
  sk.scale = 1.0f;
  Seg sv = make_seg((int)(2 * Hk), Hv, EPI_CONV, v, Hv);
  sv.chan0 = (int)(2 * Hk);
  Seg sab = make_seg((int)(2 * Hk + Hv), 2 * H, EPI_BETA_G, beta, H);
  sab.out2 = g;
  Seg sgt = make_seg((int)(2 * Hk + Hv + 2 * H), Hv, EPI_STORE, gate, Hv);
  p.seg[p.nseg++] = sq;
  p.seg[p.nseg++] = sk;
  p.seg[p.nseg++] = sv;
  p.seg[p.nseg++] = sab;
  p.seg[p.nseg++] = sgt;
  if (hid > 0) {
    MB_REQUIRE(act, MB_ERR_ARG, "gemm_gdn_prep: null activation output");
    p.seg[p.nseg++] = make_seg((int)(2 * Hk + 2 * Hv + 2 * H), 2 * hid, EPI_SWIGLU, act, ld_act);
  }
  return gemm_impl(x, ldx, w, ldw, B * T, K, p, dtype, stream);
}

extern "C" int motif_b200_gemm_gate_residual(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                             const void* gate, int64_t ldg, const void* res, int64_t ldr, void* out,
                                             int64_t ldo, int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  using namespace mb;
  MB_REQUIRE(out && N > 0 && N < (1LL << 30), MB_ERR_ARG, "gemm_gate_residual: null output or bad N");
  GemmParams p = {};
  p.nseg = 1;
  p.seg[0] = make_seg(0, N, EPI_GATE_RES, out, ldo);
  p.seg[0].gate = gate;
  p.seg[0].ldg = ldg;
  p.seg[0].res = res;
  p.seg[0].ldr = ldr;
  return gemm_impl(x, ldx, w, ldw, M, K, p, dtype, stream);
}
