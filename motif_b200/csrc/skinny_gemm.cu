// Y[M, N] = X[M, K] . W[N, K]^T for a small token count M (decode: one row per sequence,
// M <= 64), 16-bit operands, fp32 accumulation.  At decode every nn.Linear of the model is
// such a product and its cost is streaming W once from HBM: the activations are a few hundred
// KB and stay in L2, the weights (1-49 MB per product) do not.
//
// * W is packed once (motif_b200_skinny_pack) in the register order of the mma.m16n8k16 A
//   operand: for each block of 16 features x 16 K, lane l's four A registers are 16 contiguous
//   bytes.  A warp's run of k-tiles of one feature block is one contiguous range, fetched by ONE
//   bulk copy (the TMA engine, not the load/store unit) into shared memory, from where each lane
//   reads its fragment with one conflict-free 16-byte load.
// * Y^T = W . X^T: features are the MMA's M (a warp owns 2 blocks = 32 features), tokens its N
//   (M / 8 n-tiles).  X rows of the CTA's K range arrive by bulk copies too, and X^T fragments
//   are read by ldmatrix.
// * The W copies are issued first, before the kernel waits on its predecessor (programmatic
//   dependent launch: W is a weight and does not depend on earlier kernels), so the HBM latency
//   overlaps the end of the previous kernel; X is fetched after the wait.
// * K is split two ways so that every shape fills the GPU with enough bytes in flight: across
//   the 1, 2 or 4 warps of a CTA that share its features (summed in shared memory), and across
//   the CTAs of a thread-block cluster (up to 8 along y).  Between CTAs, CTA r owns a slice of
//   the tile's token rows: after one cluster barrier it reads that slice of every CTA's partial
//   through distributed shared memory, all S reads of a vector in flight together, and adds
//   them in split order.  The summation order is fixed, so results do not depend on timing.
//
// The host picks the split that runs in the fewest waves with the most CTAs (ties: more
// features per CTA, then fewer splits); callers may force it (k_warps, split_k).  Every wait on
// a copy is bounded: a CTA whose wait runs out counts itself (motif_b200_wait_timeouts), waits
// once more for its copies and carries on with what it has.
// Replaces the decode-time nn.Linear products (gdn_attn.py:88-94, chord_attn.py:88-96,
// mlp.py:52-53, decoder.py o_proj / down_proj, motif.py lm_head), which cuBLAS runs as
// weight-bandwidth-bound small-M GEMMs.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "gdn_mma.cuh"

namespace mb {

__device__ unsigned int g_sk_wait_timeouts = 0;

int read_and_clear_skinny_timeouts(unsigned int* count) {
  unsigned int zero = 0;
  if (cudaMemcpyFromSymbol(count, g_sk_wait_timeouts, sizeof(*count)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_sk_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess)
    return set_error(MB_ERR_CUDA, "wait_timeouts: %s", cudaGetErrorString(cudaGetLastError()));
  return MB_OK;
}

namespace {

constexpr int kWarps = 4;           // warps per CTA
constexpr int kThreads = kWarps * 32;
constexpr int kKtw = 12;            // most k-tiles (16 deep) one warp takes
constexpr int kMaxCluster = 8;      // portable cluster size
constexpr uint32_t kWait = 1u << 22;

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

// Pack W [N, K] (row stride ldw) into A-fragment order: block (fb, kt) of 16 features x 16 K
// at element offset (fb * KT + kt) * 256; lane l (g = l / 4, t = l % 4) holds
//   W[16 fb + g][16 kt + 2t .. +1], W[16 fb + g + 8][16 kt + 2t .. +1],
//   W[16 fb + g][16 kt + 2t + 8 .. +9], W[16 fb + g + 8][16 kt + 2t + 8 .. +9].
// Features past N (up to the next multiple of 32) are zeros.
template <typename T>
__global__ void skinny_pack_kernel(const T* __restrict__ w, int64_t ldw, int N, int KT, int NB, uint4* __restrict__ out) {
  const int64_t total = (int64_t)NB * KT * 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int lane = (int)(i & 31);
    const int64_t blk = i >> 5;
    const int kt = (int)(blk % KT), fb = (int)(blk / KT);
    const int g = lane >> 2, t = lane & 3;
    const int r0 = fb * 16 + g, r1 = r0 + 8;
    const int c0 = kt * 16 + 2 * t, c1 = c0 + 8;
    auto pair = [&](int r, int c) -> uint32_t {
      if (r >= N) return 0u;
      return *reinterpret_cast<const uint32_t*>(w + (int64_t)r * ldw + c);
    };
    out[i] = make_uint4(pair(r0, c0), pair(r1, c0), pair(r0, c1), pair(r1, c1));
  }
}

// Shared-memory plan of one launch (bytes): [W: kWarps x 2 x kwn blocks | X: ROWS x XS] with the
// partial tiles [wk][ROWS][PF] fp32 over them once the products are done, then the barriers.
struct Plan {
  int rows, kwn, xs, pf;
  size_t off_x, off_bar, bytes;
};
__host__ __device__ inline Plan make_plan(int ntt, int M, int wk, int kc, int S) {
  Plan p;
  p.rows = ntt < 2 ? 16 : ntt * 8;  // token rows staged (x4 ldmatrix reads 16)
  p.kwn = (kc + wk - 1) / wk;
  p.xs = kc * 16 + 8;               // X row stride (elements): rows on distinct 16-byte bank groups
  p.pf = (kWarps / wk) * 32 + 4;    // partial row stride (floats): conflict-free fragment stores
  const size_t wb = (size_t)kWarps * 2 * p.kwn * 512;
  p.off_x = wb;
  const size_t ab = wb + (size_t)p.rows * p.xs * 2;
  const size_t pb = (size_t)wk * p.rows * p.pf * 4;
  p.off_bar = ((ab > pb ? ab : pb) + 15) / 16 * 16;
  p.bytes = p.off_bar + (kWarps + 1) * 8;
  return p;
}

// One CTA: kWarps / wk feature groups of 32 (warp w: group w % wf, K part w / wf) over the
// CTA's K range [s kc, s kc + kc) of split s = blockIdx.y (the cluster's rank).
template <typename T, int NTT>
__global__ void __launch_bounds__(kThreads)
    skinny_kernel(const T* __restrict__ X, int64_t ldx, const uint4* __restrict__ P, int KT, int NG,
                  T* __restrict__ Y, int64_t ldy, int M, int N, int wk, int kc) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int S = gridDim.y, s = blockIdx.y;
  const Plan pl = make_plan(NTT, M, wk, kc, S);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int wf = kWarps / wk;
  const int fw = warp % wf, kw = warp / wf;
  const int group = blockIdx.x * wf + fw;
  const int kbeg = s * kc, kend = min(KT, kbeg + kc);
  const int wbeg = kbeg + kw * pl.kwn, wend = min(kend, wbeg + pl.kwn);
  const int nk = group < NG ? max(0, wend - wbeg) : 0;
  uint4* sW = reinterpret_cast<uint4*>(smem) + (size_t)warp * 2 * pl.kwn * 32;  // this warp's [2][kwn][32]
  T* sX = reinterpret_cast<T*>(smem + pl.off_x);
  uint64_t* wbar = reinterpret_cast<uint64_t*>(smem + pl.off_bar);
  uint64_t* xbar = wbar + kWarps;

  // every CTA of the cluster has started before any reads of another's shared memory (the
  // matching wait is just before the exchange)
  if (S > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
  // 1. this warp's W: two contiguous runs (its two feature blocks), one bulk copy each; each
  //    warp initialises its own barrier (warp 0 also the one of X), so nothing waits for the CTA
  if (lane == 0) {
    mbar_init(&wbar[warp], 1);
    if (warp == 0) mbar_init(xbar, 1);
    mbar_init_fence();
    if (nk > 0) {
      const uint4* src = P + ((int64_t)(2 * group) * KT + wbeg) * 32;
      mbar_arrive_expect_tx(&wbar[warp], (uint32_t)(2 * nk * 512));
      bulk_load(sW, src, (uint32_t)(nk * 512), &wbar[warp]);
      bulk_load(sW + pl.kwn * 32, src + (int64_t)KT * 32, (uint32_t)(nk * 512), &wbar[warp]);
    } else {
      mbar_arrive_expect_tx(&wbar[warp], 0u);
    }
  }
  // 2. the predecessor's output (X) is complete past this point; let the next kernel start
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  // 3. X rows [0, M) x the CTA's K range (rows past M are never stored, so they stay as they are)
  if (warp == 0) {
    const uint32_t rb = (uint32_t)(kend - kbeg) * 32;
    __syncwarp();
    if (lane == 0) mbar_arrive_expect_tx(xbar, rb * (uint32_t)M);
    __syncwarp();
    for (int r = lane; r < M; r += 32) bulk_load(sX + (size_t)r * pl.xs, X + (int64_t)r * ldx + (int64_t)kbeg * 16, rb, xbar);
  }
  __syncthreads();  // the barriers' initialisation is visible to every warp before it waits
  bool ok = mbar_wait_bounded(xbar, 0, kWait);
  ok = mbar_wait_bounded(&wbar[warp], 0, kWait) && ok;
  if (!ok) {  // count it, then give the copies one more bounded wait before the memory is reused
    if (lane == 0) atomicAdd(&g_sk_wait_timeouts, 1u);
    mbar_wait_bounded(xbar, 0, kWait);
    mbar_wait_bounded(&wbar[warp], 0, kWait);
  }

  // 4. the products: acc[f][n] = Y^T block (16 features of block f) x (8 tokens of n-tile n)
  float acc[2][NTT][4];
#pragma unroll
  for (int f = 0; f < 2; ++f)
#pragma unroll
    for (int n = 0; n < NTT; ++n) acc[f][n][0] = acc[f][n][1] = acc[f][n][2] = acc[f][n][3] = 0.f;
  const int kofs = (wbeg - kbeg) * 16;
  for (int j = 0; j < nk; ++j) {
    uint32_t b[NTT < 2 ? 2 : NTT][2];
#pragma unroll
    for (int n = 0; n < (NTT < 2 ? 2 : NTT); n += 2) {
      uint32_t r[4];
      gdnk::ldb_n(r, sX, pl.xs, kofs + j * 16, n * 8);
      b[n][0] = r[0];
      b[n][1] = r[1];
      b[n + 1][0] = r[2];
      b[n + 1][1] = r[3];
    }
#pragma unroll
    for (int f = 0; f < 2; ++f) {
      const uint4 w4 = sW[(f * pl.kwn + j) * 32 + lane];
      const uint32_t a[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int n = 0; n < NTT; ++n) mma_16816<T>(acc[f][n], a, b[n]);
    }
  }
  __syncthreads();  // every warp is done with W and X before the partial tiles overwrite them

  // 5. partial tiles [wk][ROWS][PF] (token-major), the CTA's K parts summed into part 0 in order
  const int PF = pl.pf, ROWS = pl.rows;
  float* sP = reinterpret_cast<float*>(smem);
  {
    float* part = sP + (size_t)kw * ROWS * PF;
#pragma unroll
    for (int f = 0; f < 2; ++f)
#pragma unroll
      for (int n = 0; n < NTT; ++n) {
        const int fl = fw * 32 + f * 16 + gq, t0 = n * 8 + 2 * tq;
        part[t0 * PF + fl] = acc[f][n][0];
        part[(t0 + 1) * PF + fl] = acc[f][n][1];
        part[t0 * PF + fl + 8] = acc[f][n][2];
        part[(t0 + 1) * PF + fl + 8] = acc[f][n][3];
      }
  }
  __syncthreads();
  const int VR = wf * 8;  // float4 vectors per token row of the tile
  const int V = M * VR;
  auto tile_vec = [&](int v) {
    const int t = v / VR, c = (v % VR) * 4;
    float4 a = *reinterpret_cast<const float4*>(&sP[t * PF + c]);
    for (int p = 1; p < wk; ++p) {
      const float4 q = *reinterpret_cast<const float4*>(&sP[(size_t)p * ROWS * PF + t * PF + c]);
      a.x += q.x;
      a.y += q.y;
      a.z += q.z;
      a.w += q.w;
    }
    return a;
  };
  const int n0 = blockIdx.x * wf * 32;
  auto store = [&](int t, int c, float4 a) {
    if (n0 + c >= N) return;
    uint2 o;
    o.x = pack2<T>(a.x, a.y);
    o.y = pack2<T>(a.z, a.w);
    *reinterpret_cast<uint2*>(Y + (int64_t)t * ldy + n0 + c) = o;
  };
  if (S == 1) {
    for (int v = tid; v < V; v += kThreads) store(v / VR, (v % VR) * 4, tile_vec(v));
    return;
  }
  // 6. exchange: CTA r owns token rows [r M / S, (r + 1) M / S) of the tile; after one cluster
  //    barrier it reads those rows of every CTA's summed partial (its own included) and adds
  //    them in split order.  Each thread fetches all S copies of its vectors before adding, so
  //    the remote reads overlap instead of paying one round trip each.
  if (wk > 1) {  // the CTA's own K parts summed into part 0 first
    for (int v = tid; v < V; v += kThreads) {
      const int t = v / VR, c = (v % VR) * 4;
      *reinterpret_cast<float4*>(&sP[t * PF + c]) = tile_vec(v);
    }
  }
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");  // every CTA has started
  cluster_sync_all();  // every CTA's part 0 is complete
  const int r = (int)cluster_rank();
  const int ta = r * M / S, tb = (r + 1) * M / S;
  for (int v0 = ta * VR + tid; v0 < tb * VR; v0 += 2 * kThreads) {
    float4 q[2][kMaxCluster];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int v = v0 + u * kThreads;
      if (v < tb * VR) {
        const uint32_t addr = smem_u32(&sP[(v / VR) * PF + (v % VR) * 4]);
#pragma unroll
        for (int p = 0; p < kMaxCluster; ++p)
          if (p < S) q[u][p] = ld_dsmem_f4(addr, (uint32_t)p);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int v = v0 + u * kThreads;
      if (v < tb * VR) {
        float4 a = q[u][0];
#pragma unroll
        for (int p = 1; p < kMaxCluster; ++p)
          if (p < S) {
            a.x += q[u][p].x;
            a.y += q[u][p].y;
            a.z += q[u][p].z;
            a.w += q[u][p].w;
          }
        store(v / VR, (v % VR) * 4, a);
      }
    }
  }
  // no CTA leaves while the others read its tile.  Relaxed: every remote value this thread read
  // has been added (consumed) before the arrive issues, and the Y stores need no ordering here
  // (a release would wait for them to reach L2).
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
}

struct Split {
  int wk, S, kc;
};

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" int64_t motif_b200_skinny_packed_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0 || K % 16 != 0) return -1;
  return (N + 31) / 32 * 32 * K * 2;
}

extern "C" int motif_b200_skinny_pack(const void* w, int64_t ldw, int64_t N, int64_t K, void* packed, int dtype,
                                      void* stream) {
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "skinny_pack: 16-bit weights only");
  MB_REQUIRE(N > 0 && K > 0 && N < (1LL << 30) && K < (1LL << 24), MB_ERR_SHAPE, "skinny_pack: N %lld K %lld",
             (long long)N, (long long)K);
  MB_REQUIRE(K % 16 == 0, MB_ERR_UNSUPPORTED, "skinny_pack: K (%lld) must be a multiple of 16", (long long)K);
  MB_REQUIRE(ldw >= K && ldw % 2 == 0 && (uintptr_t)w % 4 == 0, MB_ERR_ARG,
             "skinny_pack: ldw must be >= K and even, W 4-byte aligned");
  MB_REQUIRE(w != nullptr && packed != nullptr && (uintptr_t)packed % 16 == 0, MB_ERR_ARG,
             "skinny_pack: null or unaligned pointer");
  const int KT = (int)(K / 16), NB = (int)((N + 31) / 32 * 2);
  const int64_t total = (int64_t)NB * KT * 32;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == MB_BF16)
    skinny_pack_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)w, ldw, (int)N, KT, NB,
                                                               (uint4*)packed);
  else
    skinny_pack_kernel<__half><<<blocks, 256, 0, st>>>((const __half*)w, ldw, (int)N, KT, NB, (uint4*)packed);
  return check_launch("skinny_pack");
}

extern "C" int motif_b200_skinny_gemm(const void* x, int64_t ldx, const void* packed, void* y, int64_t ldy,
                                      int64_t M, int64_t N, int64_t K, int k_warps, int split_k, int dtype,
                                      void* stream) {
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "skinny_gemm: 16-bit operands only");
  MB_REQUIRE(M >= 1 && M <= 64, MB_ERR_UNSUPPORTED, "skinny_gemm: M (%lld) must be in 1..64", (long long)M);
  MB_REQUIRE(N > 0 && K > 0 && N < (1LL << 30) && K < (1LL << 24), MB_ERR_SHAPE, "skinny_gemm: N %lld K %lld",
             (long long)N, (long long)K);
  MB_REQUIRE(K % 16 == 0, MB_ERR_UNSUPPORTED, "skinny_gemm: K (%lld) must be a multiple of 16", (long long)K);
  MB_REQUIRE(N % 4 == 0 && ldy % 4 == 0 && ldy >= N && (uintptr_t)y % 8 == 0, MB_ERR_UNSUPPORTED,
             "skinny_gemm: N and ldy must be multiples of 4 (Y 8-byte aligned)");
  MB_REQUIRE(ldx % 8 == 0 && ldx >= K && (uintptr_t)x % 16 == 0 && (uintptr_t)packed % 16 == 0, MB_ERR_UNSUPPORTED,
             "skinny_gemm: ldx must be a multiple of 8 (X and the packed weight 16-byte aligned)");
  MB_REQUIRE(k_warps == 0 || k_warps == 1 || k_warps == 2 || k_warps == 4, MB_ERR_ARG,
             "skinny_gemm: k_warps must be 0 (automatic), 1, 2 or 4");
  MB_REQUIRE(split_k >= 0 && split_k <= kMaxCluster, MB_ERR_ARG, "skinny_gemm: split_k must be 0 (automatic) .. %d",
             kMaxCluster);
  const int KT = (int)(K / 16), NG = (int)((N + 31) / 32);
  const int ntt = M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8));
  int dev = 0, sms = 148, smem_sm = 228 * 1024;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(MB_ERR_CUDA, "skinny_gemm: no device");
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  constexpr size_t kMaxSmem = 227 * 1024;

  // registers per thread of the instance (once per device and instance): CTAs per SM
  static int regs_of[4] = {0, 0, 0, 0};
  static std::mutex regs_mu;
  const int ni = ntt == 1 ? 0 : (ntt == 2 ? 1 : (ntt == 4 ? 2 : 3));
  int regs = 0;
  {
    std::lock_guard<std::mutex> lock(regs_mu);
    if (!regs_of[ni]) {
      cudaFuncAttributes fa = {};
      const void* f = ntt == 1 ? (const void*)skinny_kernel<__nv_bfloat16, 1>
                    : ntt == 2 ? (const void*)skinny_kernel<__nv_bfloat16, 2>
                    : ntt == 4 ? (const void*)skinny_kernel<__nv_bfloat16, 4>
                               : (const void*)skinny_kernel<__nv_bfloat16, 8>;
      regs_of[ni] = cudaFuncGetAttributes(&fa, f) == cudaSuccess && fa.numRegs > 0 ? fa.numRegs : 255;
    }
    regs = regs_of[ni];
  }
  const long reg_ctas = std::max(1, 65536 / (kThreads * ((regs + 7) / 8 * 8)));

  // The split with the least estimated time.  Each wave pays ~1.5 us of latency; a CTA streams
  // its W bytes at ~70 KB/us and its X bytes from L2 at ~110 KB/us, and the CTAs sharing an SM
  // add up; a split across a cluster costs ~0.8 us plus ~0.1 us per part for the barrier and the
  // exchange, plus its partial bytes at ~10 KB/us; and no split moves the weight faster than HBM
  // (~6.5 GB/ms).  Fitted to forced-split sweeps of the 172M model's decode products on B200 at
  // 8-32 rows (the exchange's fixed cost is what makes a split-free CTA of four K-splitting
  // warps the fastest choice for the K = 768 products: 2.9 instead of 5.0 us for N 6016).
  Split best = {0, 0, 0};
  double best_us = 0.0;
  size_t best_smem = 0;
  for (int wk : {1, 2, 4}) {
    if (k_warps && wk != k_warps) continue;
    for (int S = 1; S <= kMaxCluster; ++S) {
      if (split_k && S != split_k) continue;
      const int kc = (KT + S - 1) / S;
      if ((kc + wk - 1) / wk > kKtw) continue;
      const Split sp = {wk, (KT + kc - 1) / kc, kc};
      if (!split_k && sp.S != S) continue;  // the same split as a smaller S
      const Plan pl = make_plan(ntt, (int)M, wk, kc, sp.S);
      if (pl.bytes > kMaxSmem) continue;
      const long per_sm = std::min<long>(reg_ctas, (long)smem_sm / (long)(pl.bytes + 1024));
      if (per_sm < 1) continue;
      const int F = (kWarps / wk) * 32;
      const long ctas = (long)((NG + kWarps / wk - 1) / (kWarps / wk)) * sp.S;
      const long slots = per_sm * sms, waves = (ctas + slots - 1) / slots;
      const long share = (std::min(ctas, slots) + sms - 1) / sms;
      const double w_kb = (double)F * kc * 32 / 1024.0, x_kb = (double)M * kc * 32 / 1024.0;
      const double e_kb = sp.S > 1 ? (double)M * F * 4 * (sp.S - 1) / sp.S / 1024.0 : 0.0;
      double us = (double)waves * (1.5 + (double)share * (w_kb / 70.0 + x_kb / 110.0)) +
                  (sp.S > 1 ? 0.8 + 0.1 * sp.S + e_kb / 10.0 : 0.0);
      us = std::max(us, (double)N * K * 2 / 1024.0 / 6500.0);
      if (best.wk == 0 || us < best_us) {
        best = sp;
        best_us = us;
        best_smem = pl.bytes;
      }
    }
  }
  MB_REQUIRE(best.wk != 0, MB_ERR_UNSUPPORTED,
             "skinny_gemm: no split of K = %lld fits (k_warps %d, split_k %d; at most %d k-tiles per warp)",
             (long long)K, k_warps, split_k, kKtw);
  const int wf = kWarps / best.wk;
  cudaStream_t st = (cudaStream_t)stream;
  auto go = [&](auto t, auto ntt_c) -> int {
    using T = decltype(t);
    constexpr int NTT = decltype(ntt_c)::value;
    auto kern = skinny_kernel<T, NTT>;
    const int rc = ensure_smem_attr((const void*)kern, (int)kMaxSmem);
    if (rc != MB_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = (unsigned)best.S;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)((NG + wf - 1) / wf), (unsigned)best.S);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = best_smem;
    cfg.stream = st;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, kern, (const T*)x, ldx, (const uint4*)packed, KT, NG, (T*)y, ldy, (int)M, (int)N,
                       best.wk, best.kc);
    return check_launch("skinny_gemm");
  };
  auto by_n = [&](auto t) -> int {
    switch (ntt) {
      case 1: return go(t, std::integral_constant<int, 1>{});
      case 2: return go(t, std::integral_constant<int, 2>{});
      case 4: return go(t, std::integral_constant<int, 4>{});
      default: return go(t, std::integral_constant<int, 8>{});
    }
  };
  return dtype == MB_BF16 ? by_n(__nv_bfloat16{}) : by_n(__half{});
}

// ----------------------------------------------------------------------------------------
// Tensor-core variant for 33 .. 64 token rows (one GPU's decode batch of the 172M model: 64
// requests).  At these row counts the legacy-MMA kernel above spends as long on its MMAs and
// on the cluster exchange of wide partial tiles as on the weight stream, so:
//   * Y^T tile = W tile (128 features, the MMA's M) x X^T (64 token columns, the MMA's N) as
//     tcgen05.mma kind::f16 into a 64-column TMEM accumulator, both operands staged by tiled
//     TMA (128-byte swizzle) in 64-deep K blocks; tokens past M are the tensor map's zero fill;
//   * a CTA takes one feature tile and a contiguous run of K blocks (split s = blockIdx.y of a
//     cluster of S along y); every W block of its ring is requested before the kernel waits on
//     its predecessor (programmatic dependent launch), X after the wait;
//   * optional epilogue (the Chord decoder's parallel residual, chord_attn.py:254,313 and
//     decoder.py:208): Y = round(round(A * round(sigmoid(G))) + round(X W^T)) with A the
//     attention output after o_proj and G the gate, at the rounding points of the separate
//     gate-residual kernel, so the fused result is bit-identical to the product followed by it;
//   * two products in one launch (the Chord decoder's tail, motif_b200_skinny_gemm_tc_chord_tail):
//     the cluster's first S1 ranks split the K of product 1 (the o_proj of the attention
//     output), the others the K of product 2 (the MLP's down_proj); each CTA still has one
//     accumulator, the exchange sums the two groups of partials apart, and the epilogue applies
//     Y = round(round(round(P1) * round(sigmoid(G))) + round(P2));
//   * the split-K partials (fp32, token-major [64][128]) stay in each CTA's shared memory;
//     after one cluster barrier CTA r reads the token rows it owns from all S partials through
//     distributed shared memory, every read of a thread in flight at once, and adds them in rank
//     order (deterministic) before storing them.
// Every wait is bounded (counted in motif_b200_wait_timeouts); every CTA passes the same
// cluster barriers whatever happened, so no CTA of the cluster waits for one that left.
namespace mb {
namespace {

constexpr int kTcF = 128;                       // features per CTA
constexpr int kTcTok = 64;                      // token columns of the accumulator
constexpr int kTcBK = 64;                       // K per ring stage
constexpr int kTcWBytes = kTcF * kTcBK * 2;     // 16 KB
constexpr int kTcXBytes = kTcTok * kTcBK * 2;   // 8 KB
constexpr int kTcStage = kTcWBytes + kTcXBytes; // 24 KB
constexpr int kTcMaxStages = 8;
constexpr int kTcThreads = 128;
constexpr int kTcRow = kTcF * 4;                // bytes of one token row of a partial tile
constexpr int kTcMaxCluster = 8;

struct TcPlan {
  size_t off_bar, bytes;
};
// [ring: R stages of W | X, the partial tile [64][128] fp32 over it once drained][barriers]
__host__ __device__ inline TcPlan make_tc_plan(int R) {
  TcPlan p;
  const size_t ring = (size_t)R * kTcStage;
  const size_t ptile = (size_t)kTcTok * kTcRow;  // 32 KB
  p.off_bar = ring > ptile ? ring : ptile;
  p.bytes = p.off_bar + (2 * kTcMaxStages + 4) * 8 + 1024;  // barriers, TMEM address, 1 KB alignment slack
  return p;
}

__device__ __forceinline__ void tc_prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads) skinny_tc_kernel(const __grid_constant__ CUtensorMap tmW,
                                                               const __grid_constant__ CUtensorMap tmX,
                                                               T* __restrict__ Y, int64_t ldy, int M, int N,
                                                               int kb_total, int kbc, int R,
                                                               const T* __restrict__ ga, int64_t lda,
                                                               const T* __restrict__ gg, int64_t ldg,
                                                               const __grid_constant__ CUtensorMap tmW2,
                                                               const __grid_constant__ CUtensorMap tmX2,
                                                               int kb_total2, int S1) {
  constexpr uint32_t ab_fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  extern __shared__ unsigned char tc_smem_raw[];
  unsigned char* sm = tc_smem_raw + ((1024u - (smem_u32(tc_smem_raw) & 1023u)) & 1023u);
  const int S = gridDim.y, s = blockIdx.y;
  const TcPlan pl = make_tc_plan(R);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + pl.off_bar);
  uint64_t* empty = full + kTcMaxStages;
  uint64_t* mdone = empty + kTcMaxStages;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(mdone + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // ranks [0, S1) run product 1 (tmW, tmX), ranks [S1, S) product 2 (tmW2, tmX2)
  const bool second = s >= S1;
  const CUtensorMap* mW = second ? &tmW2 : &tmW;
  const CUtensorMap* mX = second ? &tmX2 : &tmX;
  const int kb0 = (second ? s - S1 : s) * kbc;
  const int nkb = min(second ? kb_total2 : kb_total, kb0 + kbc) - kb0;  // >= 1 (the host sizes the split)
  const int f0 = blockIdx.x * kTcF;
  const int ta = s * M / S, tb = (s + 1) * M / S;  // token rows this CTA sums and stores
  const int nfirst = min(R, nkb);
  auto load_w = [&](int st, int kb) { tma_load_2d(sm + st * kTcStage, mW, kb * kTcBK, f0, &full[st]); };

  if (tid == 0) {
    tc_prefetch_tmap(mW);
    tc_prefetch_tmap(mX);
    for (int i = 0; i < kTcMaxStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(mdone, 1);
    mbar_init_fence();
    // the weights do not depend on the previous kernel: request the whole first ring now
    for (int i = 0; i < nfirst; ++i) {
      mbar_arrive_expect_tx(&full[i], (uint32_t)kTcStage);
      load_w(i, kb0 + i);
    }
  }
  if (warp == 1) tmem_alloc(sTmem, kTcTok);
  // X is the previous kernel's output; let the next kernel start its own weight fetch
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  if (tid == 0)
    for (int i = 0; i < nfirst; ++i) tma_load_2d(sm + i * kTcStage + kTcWBytes, mX, (kb0 + i) * kTcBK, 0, &full[i]);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;
  bool ok = true;

  if (warp == 0 && lane == 0) {  // refills past the first ring
    for (int i = nfirst; i < nkb && ok; ++i) {
      const int st = i % R;
      if (!mbar_wait_bounded(&empty[st], (uint32_t)((i / R - 1) & 1), kWait)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&full[st], (uint32_t)kTcStage);
      load_w(st, kb0 + i);
      tma_load_2d(sm + st * kTcStage + kTcWBytes, mX, (kb0 + i) * kTcBK, 0, &full[st]);
    }
  } else if (warp == 1 && lane == 0) {  // the MMAs
    const uint32_t idesc = umma_idesc_f16(ab_fmt, kTcF, kTcTok, 0, 0);
    for (int i = 0; i < nkb; ++i) {
      const int st = i % R;
      if (!mbar_wait_bounded(&full[st], (uint32_t)((i / R) & 1), kWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a = smem_u32(sm + st * kTcStage), b = a + kTcWBytes;
#pragma unroll
      for (int k = 0; k < kTcBK / 16; ++k)
        umma_f16_ss(tmem, umma_desc_sw128(a + k * 32, 16, 1024), umma_desc_sw128(b + k * 32, 16, 1024), idesc,
                    (i > 0 || k > 0) ? 1u : 0u);
      if (i + R < nkb) umma_commit(&empty[st]);
    }
    umma_commit(mdone);  // also on the failure path: every MMA issued above completes first
  }
  __syncwarp();
  ok = mbar_wait_bounded(mdone, 0, kWait) && ok;
  if (!ok) {  // count it; the copies still in flight get one more bounded wait before the ring is reused
    if (lane == 0) atomicAdd(&g_sk_wait_timeouts, 1u);
    if (tid == 0)
      for (int i = 0; i < nfirst; ++i) mbar_wait_bounded(&full[i], (uint32_t)(((nkb - 1 - i) / R) & 1), kWait);
  }
  tc_fence_after();

  // accumulator -> partial tile P [token][feature] fp32 over the drained ring
  float* P = reinterpret_cast<float*>(sm);
  {
    const int fl = warp * 32 + lane;
    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
    uint32_t acc[32];
#pragma unroll
    for (int h = 0; h < kTcTok / 32; ++h) {
      tmem_ld32(taddr + (uint32_t)(h * 32), acc);
      tmem_wait_ld(acc);
#pragma unroll
      for (int j = 0; j < 32; ++j) P[(h * 32 + j) * kTcF + fl] = __uint_as_float(acc[j]);
    }
  }
  const bool dual = S1 < S;
  auto store = [&](int t, int c, float4 a, float4 d) {
    if (f0 + c >= N) return;
    if (dual) {  // y = round(round(round(product 1) round(sigmoid(G))) + round(product 2))
      const uint2 gv = *reinterpret_cast<const uint2*>(gg + (int64_t)t * ldg + f0 + c);
      const T* g4 = reinterpret_cast<const T*>(&gv);
      const float v1[4] = {a.x, a.y, a.z, a.w}, v2[4] = {d.x, d.y, d.z, d.w};
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float gate = to_f(from_f<T>(sigmoidf_(to_f(g4[e]))));
        const float att = to_f(from_f<T>(to_f(from_f<T>(v1[e])) * gate));
        v[e] = att + to_f(from_f<T>(v2[e]));
      }
      a = make_float4(v[0], v[1], v[2], v[3]);
    } else if (ga != nullptr) {  // y = round(round(A round(sigmoid(G))) + round(product))
      const uint2 av = *reinterpret_cast<const uint2*>(ga + (int64_t)t * lda + f0 + c);
      const uint2 gv = *reinterpret_cast<const uint2*>(gg + (int64_t)t * ldg + f0 + c);
      const T* a4 = reinterpret_cast<const T*>(&av);
      const T* g4 = reinterpret_cast<const T*>(&gv);
      float v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float gate = to_f(from_f<T>(sigmoidf_(to_f(g4[e]))));
        const float att = to_f(from_f<T>(to_f(a4[e]) * gate));
        v[e] = att + to_f(from_f<T>(v[e]));
      }
      a = make_float4(v[0], v[1], v[2], v[3]);
    }
    uint2 o;
    o.x = pack2<T>(a.x, a.y);
    o.y = pack2<T>(a.z, a.w);
    *reinterpret_cast<uint2*>(Y + (int64_t)t * ldy + f0 + c) = o;
  };
  constexpr int VR = kTcF / 4;  // float4 vectors per token row
  if (S == 1) {
    __syncthreads();
    // every load of the thread in flight before its stores (a dependent load -> store chain
    // per vector would cost one shared-memory round trip each)
    constexpr int U = kTcTok * VR / kTcThreads;  // 16 vectors per thread at M = 64
    float4 q[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = tid + u * kTcThreads;
      if (v < M * VR) q[u] = *reinterpret_cast<const float4*>(&P[(v / VR) * kTcF + (v % VR) * 4]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = tid + u * kTcThreads;
      if (v < M * VR) store(v / VR, (v % VR) * 4, q[u], q[u]);
    }
  } else {
    // every CTA's partial is in its shared memory before any CTA reads it
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
    const uint32_t pbase = smem_u32(P);
    const int nv = (tb - ta) * VR;
    constexpr int U = 4;
    for (int v0 = tid; v0 < nv; v0 += U * kTcThreads) {
      float4 q[U][kTcMaxCluster];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * kTcThreads;
        if (v < nv) {
          const uint32_t addr = pbase + (uint32_t)(((ta + v / VR) * kTcF + (v % VR) * 4) * 4);
#pragma unroll
          for (int p = 0; p < kTcMaxCluster; ++p)
            if (p < S) q[u][p] = ld_dsmem_f4(addr, (uint32_t)p);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * kTcThreads;
        if (v < nv) {
          // rank order within each product: the sums do not depend on timing
          float4 a = q[u][0], d = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int p = 1; p < kTcMaxCluster; ++p)
            if (p < S1) {
              a.x += q[u][p].x;
              a.y += q[u][p].y;
              a.z += q[u][p].z;
              a.w += q[u][p].w;
            }
#pragma unroll
          for (int p = 1; p < kTcMaxCluster; ++p)
            if (p >= S1 && p < S) {
              if (p == S1) {
                d = q[u][p];
              } else {
                d.x += q[u][p].x;
                d.y += q[u][p].y;
                d.z += q[u][p].z;
                d.w += q[u][p].w;
              }
            }
          store(ta + v / VR, (v % VR) * 4, a, d);
        }
      }
    }
    // no CTA leaves while another reads its partial (every value read above has been used)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
    asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcTok);
  }
}

struct TcChoice {
  int S, kbc, R;
  size_t bytes;
};

}  // namespace
}  // namespace mb

namespace mb {
namespace {
// Clusters of S CTAs (kTcThreads threads, `bytes` of shared memory each) that can be resident at
// once on the current device (cached per device and shape; 0 if the query fails).
int tc_max_clusters(const void* kern, int S, size_t bytes) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple(dev, S, bytes);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = (unsigned)S;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(1, (unsigned)S);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = bytes;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

// One launch of skinny_tc_kernel: `tiles` feature tiles x ch.S cluster ranks (a cluster along
// y), programmatic dependent launch allowed.  Product 2 (tmW2, tmX2, kbt2) runs on ranks
// [S1, ch.S); with S1 == ch.S there is one product.
int launch_tc(int dtype, const TcChoice& ch, int tiles, void* stream, const CUtensorMap& tmW, const CUtensorMap& tmX,
              void* y, int64_t ldy, int64_t M, int64_t N, int kbt, const void* ga, int64_t lda, const void* gg,
              int64_t ldg, const CUtensorMap& tmW2, const CUtensorMap& tmX2, int kbt2, int S1, const char* what) {
  auto go = [&](auto t) -> int {
    using T = decltype(t);
    auto kern = skinny_tc_kernel<T>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = (unsigned)ch.S;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)tiles, (unsigned)ch.S);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = ch.bytes;
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, kern, tmW, tmX, (T*)y, ldy, (int)M, (int)N, kbt, ch.kbc, ch.R, (const T*)ga, lda,
                       (const T*)gg, ldg, tmW2, tmX2, kbt2, S1);
    return check_launch(what);
  };
  return dtype == MB_BF16 ? go(__nv_bfloat16{}) : go(__half{});
}

int skinny_tc_launch(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int64_t M,
                     int64_t N, int64_t K, int split_k, int dtype, void* stream, const void* ga = nullptr,
                     int64_t lda = 0, const void* gg = nullptr, int64_t ldg = 0) {
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "skinny_gemm_tc: 16-bit operands only");
  MB_REQUIRE(M >= 1 && M <= kTcTok, MB_ERR_UNSUPPORTED, "skinny_gemm_tc: M (%lld) must be in 1..64", (long long)M);
  MB_REQUIRE(N > 0 && K > 0 && N < (1LL << 30) && K < (1LL << 24), MB_ERR_SHAPE, "skinny_gemm_tc: N %lld K %lld",
             (long long)N, (long long)K);
  MB_REQUIRE(K % kTcBK == 0, MB_ERR_UNSUPPORTED, "skinny_gemm_tc: K (%lld) must be a multiple of 64", (long long)K);
  MB_REQUIRE(x && w && y, MB_ERR_ARG, "skinny_gemm_tc: null operand");
  MB_REQUIRE(N % 4 == 0 && ldy % 4 == 0 && ldy >= N && (uintptr_t)y % 8 == 0, MB_ERR_UNSUPPORTED,
             "skinny_gemm_tc: N and ldy must be multiples of 4 (Y 8-byte aligned)");
  MB_REQUIRE(ldx % 8 == 0 && ldw % 8 == 0 && ldx >= K && ldw >= K && ((uintptr_t)x | (uintptr_t)w) % 16 == 0,
             MB_ERR_ALIGN, "skinny_gemm_tc: X / W rows must be 16-byte aligned (row strides multiples of 8)");
  MB_REQUIRE(split_k >= 0 && split_k <= kTcMaxCluster, MB_ERR_ARG, "skinny_gemm_tc: split_k must be 0 (automatic) .. %d",
             kTcMaxCluster);
  constexpr size_t kMaxSmem = 227 * 1024;
  const int kbt = (int)(K / kTcBK);
  const int tiles = (int)((N + kTcF - 1) / kTcF);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(MB_ERR_CUDA, "skinny_gemm_tc: no device");
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // The split.  One CTA streams its W run at roughly 40-55 GB/s (measured: bounded by the
  // copies a CTA keeps in flight), so the weight has to be spread over every SM: the grid is
  // sized to one CTA per SM (the shared-memory request is raised so that the block scheduler
  // cannot stack two CTAs on one SM while others idle) unless it needs more CTAs than SMs, in
  // which case two fit per SM.  Among the splits whose clusters all fit in one wave (asked of
  // the occupancy calculator), the fewest parts that reach 90 % of the SMs, else the most
  // CTAs; at most 8 parts (a portable cluster).  Ring depth: the CTA's whole run when it fits.
  auto kern_bf16 = skinny_tc_kernel<__nv_bfloat16>;
  auto kern_f16 = skinny_tc_kernel<__half>;
  if (int e = ensure_smem_attr((const void*)kern_bf16, (int)kMaxSmem)) return e;
  if (int e = ensure_smem_attr((const void*)kern_f16, (int)kMaxSmem)) return e;
  constexpr size_t kOnePerSm = 114 * 1024;  // more than half an SM's shared memory
  TcChoice ch = {0, 0, 0, 0};
  long ch_ctas = 0;
  for (int S = 1; S <= kTcMaxCluster; ++S) {
    if (split_k && S != split_k) continue;
    const int kbc = (kbt + S - 1) / S;
    const int Se = (kbt + kbc - 1) / kbc;
    if (Se != S) continue;  // the same split as a smaller S
    const long ctas = (long)tiles * S;
    int R = std::min(kbc, kTcMaxStages);
    while (R > 1 && make_tc_plan(R).bytes > kMaxSmem) --R;
    if (ctas > sms)
      while (R > 2 && make_tc_plan(R).bytes > kMaxSmem / 2) --R;
    size_t bytes = make_tc_plan(R).bytes;
    if (bytes > kMaxSmem) continue;
    if (ctas <= sms) bytes = std::max(bytes, kOnePerSm);
    const int cap = tc_max_clusters((const void*)kern_bf16, S, bytes);
    const bool one_wave = cap > 0 && (long)tiles <= cap;
    if (split_k) {
      ch = {S, kbc, R, bytes};
      break;
    }
    if (!one_wave && ch.S != 0) continue;
    if (ch.S == 0 || ctas > ch_ctas) {
      ch = {S, kbc, R, bytes};
      ch_ctas = ctas;
    }
    if (one_wave && ctas >= sms * 9 / 10) break;
  }
  MB_REQUIRE(ch.S != 0, MB_ERR_UNSUPPORTED, "skinny_gemm_tc: no split of K = %lld into %d parts", (long long)K,
             split_k);
  CUtensorMap tmW, tmX;
  int rc = encode_tile_map_2d(&tmW, w, 2, (uint64_t)K, (uint64_t)N, (uint64_t)ldw * 2, kTcBK, kTcF, 128);
  if (!rc) rc = encode_tile_map_2d(&tmX, x, 2, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, kTcBK, kTcTok, 128);
  if (rc) return rc;
  return launch_tc(dtype, ch, tiles, stream, tmW, tmX, y, ldy, M, N, kbt, ga, lda, gg, ldg, tmW, tmX, 0, ch.S,
                   "skinny_gemm_tc");
}

}  // namespace
}  // namespace mb

extern "C" int motif_b200_skinny_gemm_tc(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                                         int64_t M, int64_t N, int64_t K, int split_k, int dtype, void* stream) {
  return mb::skinny_tc_launch(x, ldx, w, ldw, y, ldy, M, N, K, split_k, dtype, stream);
}

extern "C" int motif_b200_skinny_gemm_tc_add_gated(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                                   const void* a, int64_t lda, const void* g, int64_t ldg, void* y,
                                                   int64_t ldy, int64_t M, int64_t N, int64_t K, int split_k,
                                                   int dtype, void* stream) {
  MB_REQUIRE(a && g, MB_ERR_ARG, "skinny_gemm_tc_add_gated: null attention output or gate");
  MB_REQUIRE(lda % 4 == 0 && ldg % 4 == 0 && lda >= N && ldg >= N && ((uintptr_t)a | (uintptr_t)g) % 8 == 0,
             MB_ERR_ALIGN, "skinny_gemm_tc_add_gated: A / G rows must be 8-byte aligned (row strides multiples of 4)");
  return mb::skinny_tc_launch(x, ldx, w, ldw, y, ldy, M, N, K, split_k, dtype, stream, a, lda, g, ldg);
}

extern "C" int motif_b200_skinny_gemm_tc_chord_tail(const void* x1, int64_t ldx1, const void* w1, int64_t ldw1,
                                                    int64_t K1, const void* x2, int64_t ldx2, const void* w2,
                                                    int64_t ldw2, int64_t K2, const void* g, int64_t ldg, void* y,
                                                    int64_t ldy, int64_t M, int64_t N, int dtype, void* stream) {
  using namespace mb;
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "skinny_gemm_tc_chord_tail: 16-bit operands only");
  MB_REQUIRE(M >= 1 && M <= kTcTok, MB_ERR_UNSUPPORTED, "skinny_gemm_tc_chord_tail: M (%lld) must be in 1..64",
             (long long)M);
  MB_REQUIRE(N > 0 && N < (1LL << 30) && K1 > 0 && K2 > 0 && K1 < (1LL << 24) && K2 < (1LL << 24), MB_ERR_SHAPE,
             "skinny_gemm_tc_chord_tail: N %lld K1 %lld K2 %lld", (long long)N, (long long)K1, (long long)K2);
  MB_REQUIRE(K1 % kTcBK == 0 && K2 % kTcBK == 0, MB_ERR_UNSUPPORTED,
             "skinny_gemm_tc_chord_tail: K1 and K2 must be multiples of 64");
  MB_REQUIRE(x1 && w1 && x2 && w2 && g && y, MB_ERR_ARG, "skinny_gemm_tc_chord_tail: null operand");
  MB_REQUIRE(N % 4 == 0 && ldy % 4 == 0 && ldy >= N && (uintptr_t)y % 8 == 0, MB_ERR_UNSUPPORTED,
             "skinny_gemm_tc_chord_tail: N and ldy must be multiples of 4 (Y 8-byte aligned)");
  MB_REQUIRE(ldx1 % 8 == 0 && ldw1 % 8 == 0 && ldx2 % 8 == 0 && ldw2 % 8 == 0 && ldx1 >= K1 && ldw1 >= K1 &&
                 ldx2 >= K2 && ldw2 >= K2 && ((uintptr_t)x1 | (uintptr_t)w1 | (uintptr_t)x2 | (uintptr_t)w2) % 16 == 0,
             MB_ERR_ALIGN, "skinny_gemm_tc_chord_tail: X / W rows must be 16-byte aligned (row strides multiples of 8)");
  MB_REQUIRE(ldg % 4 == 0 && ldg >= N && (uintptr_t)g % 8 == 0, MB_ERR_ALIGN,
             "skinny_gemm_tc_chord_tail: G rows must be 8-byte aligned (row stride a multiple of 4)");
  constexpr size_t kMaxSmem = 227 * 1024;
  constexpr size_t kOnePerSm = 114 * 1024;
  const int kbt1 = (int)(K1 / kTcBK), kbt2 = (int)(K2 / kTcBK);
  const int tiles = (int)((N + kTcF - 1) / kTcF);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(MB_ERR_CUDA, "skinny_gemm_tc_chord_tail: no device");
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  auto kern_bf16 = skinny_tc_kernel<__nv_bfloat16>;
  auto kern_f16 = skinny_tc_kernel<__half>;
  if (int e = ensure_smem_attr((const void*)kern_bf16, (int)kMaxSmem)) return e;
  if (int e = ensure_smem_attr((const void*)kern_f16, (int)kMaxSmem)) return e;
  // K blocks per CTA, the same for both products: the smallest (the most CTAs) whose
  // S1 + S2 <= 8 parts fit a cluster and whose clusters fit in one wave
  TcChoice ch = {0, 0, 0, 0};
  int S1 = 0;
  for (int kbc = 1; kbc <= std::max(kbt1, kbt2); ++kbc) {
    const int s1 = (kbt1 + kbc - 1) / kbc, s2 = (kbt2 + kbc - 1) / kbc;
    const int S = s1 + s2;
    if (S > kTcMaxCluster) continue;
    int R = std::min(kbc, kTcMaxStages);
    while (R > 1 && make_tc_plan(R).bytes > kMaxSmem) --R;
    size_t bytes = make_tc_plan(R).bytes;
    if (bytes > kMaxSmem) continue;
    if ((long)tiles * S <= sms) bytes = std::max(bytes, kOnePerSm);
    const int cap = tc_max_clusters((const void*)kern_bf16, S, bytes);
    if (cap <= 0 || tiles > cap) continue;
    ch = {S, kbc, R, bytes};
    S1 = s1;
    break;
  }
  MB_REQUIRE(ch.S != 0, MB_ERR_UNSUPPORTED, "skinny_gemm_tc_chord_tail: no split of K1 = %lld, K2 = %lld fits",
             (long long)K1, (long long)K2);
  CUtensorMap tmW, tmX, tmW2, tmX2;
  int rc = encode_tile_map_2d(&tmW, w1, 2, (uint64_t)K1, (uint64_t)N, (uint64_t)ldw1 * 2, kTcBK, kTcF, 128);
  if (!rc) rc = encode_tile_map_2d(&tmX, x1, 2, (uint64_t)K1, (uint64_t)M, (uint64_t)ldx1 * 2, kTcBK, kTcTok, 128);
  if (!rc) rc = encode_tile_map_2d(&tmW2, w2, 2, (uint64_t)K2, (uint64_t)N, (uint64_t)ldw2 * 2, kTcBK, kTcF, 128);
  if (!rc) rc = encode_tile_map_2d(&tmX2, x2, 2, (uint64_t)K2, (uint64_t)M, (uint64_t)ldx2 * 2, kTcBK, kTcTok, 128);
  if (rc) return rc;
  return launch_tc(dtype, ch, tiles, stream, tmW, tmX, y, ldy, M, N, kbt1, nullptr, 0, g, ldg, tmW2, tmX2, kbt2, S1,
                   "skinny_gemm_tc_chord_tail");
}
