// Y[M, N] = X[M, K] . W[N, K]^T for a small token count M (decode: one row per sequence,
// M <= 64), 16-bit operands, fp32 accumulation.  At decode every nn.Linear of the model is
// such a product and its cost is streaming W once from HBM (the activations are a few
// hundred KB and stay in L2).
//
// The product is computed transposed on the 5th-generation tensor cores: Y^T = W . X^T, so a
// CTA's 128 output features are the MMA's M = 128 rows and the (up to 64) tokens its N.  A
// CTA owns 128 consecutive rows of W and one slice of K; thread 0 streams 64-wide K chunks of
// W (128 x 64) and X (64 x 64) by tiled TMA (128-byte swizzle, rows past N or M read as zeros)
// into a 4-stage ring and issues four tcgen05.mma (K = 16 each) per chunk into a 64-column
// TMEM accumulator; a stage is refilled once the MMAs that read it have completed
// (tcgen05.commit on the stage's mbarrier).
//
// When the feature blocks alone cannot fill the GPU (768 outputs at K up to 3584), K is split
// across the CTAs of a thread-block cluster (up to 16 along y).  Each CTA reads its
// accumulator back with tcgen05.ld (thread = feature, one register per token) into a fp32
// [token][feature] tile in its own shared memory.  The tile's float4 groups are cut into
// nsplit slices, CTA p owning slice p: after a cluster barrier every CTA sends slice p of
// its tile to CTA p with one shared::cta -> shared::cluster bulk copy (completion counted on
// p's receive barrier), then sums its own slice over the splits in split order (a fixed
// order: results do not depend on timing) and writes it to Y.  No workspace, no atomics.
// An unsplit launch (a cluster of one) writes Y straight from the accumulator registers.
// Every mbarrier wait is bounded; a CTA whose wait runs out counts itself
// (motif_b200_wait_timeouts), drains what it issued and still takes both cluster barriers.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace mb {

__device__ unsigned int g_sk_wait_timeouts = 0;

namespace {

constexpr int kBN = 128;        // output features per CTA (MMA M)
constexpr int kBK = 64;         // K per swizzle atom: one 128-byte row
constexpr int kMaxM = 64;       // tokens (MMA N)
#ifndef SK_STAGES
#define SK_STAGES 4
#endif
#ifndef SK_ATOMS
#define SK_ATOMS 1
#endif
#ifndef SK_MINB
#define SK_MINB 2
#endif
#ifndef SK_ROT
#define SK_ROT 1
#endif
#ifndef SK_PDL
#define SK_PDL 1
#endif
constexpr int kStages = SK_STAGES;
constexpr int kAtoms = SK_ATOMS;  // 64-wide K atoms per stage (one TMA box each)
constexpr int kMaxSplit = 16;   // cluster size limit (16 needs the non-portable opt-in)
constexpr int kWAtom = kBN * kBK * 2;      // 16 KB
constexpr int kXAtom = kMaxM * kBK * 2;    // 8 KB
constexpr int kWBytes = kAtoms * kWAtom;
constexpr int kStageBytes = kAtoms * (kWAtom + kXAtom);
constexpr int kTileBytes = kMaxM * kBN * 4;  // fp32 partial tile, reuses the ring
// the partial tile and the receive buffer of the split-K exchange both reuse the ring
static_assert(2 * kTileBytes <= kStages * kStageBytes, "partial tile and receive buffer must fit the ring");
constexpr int kSmemBytes = kStages * kStageBytes + 2 * kStages * 8 + 16 + 16 + 1024;  // + 1024-byte alignment
constexpr uint32_t kWait = 1u << 22;
constexpr uint32_t kTmemCols = 64;

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
template <typename T>
__global__ void __launch_bounds__(128, SK_MINB) skinny_tc_kernel(const __grid_constant__ CUtensorMap tmW,
                                                           const __grid_constant__ CUtensorMap tmX,
                                                           T* __restrict__ Y, int64_t ldy, int M, int N,
                                                           int kchunks_per_split, int kchunks, int katoms,
                                                           int vec_store) {
  constexpr uint32_t ab_fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t idesc = umma_idesc_f16(ab_fmt, kBN, kMaxM, 0, 0);
  extern __shared__ unsigned char sk_smem_raw[];
  unsigned char* sm = sk_smem_raw + ((1024u - (smem_u32(sk_smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint64_t* recvbar = done + 1;  // split-K: the other splits' slices of this CTA's part of the tile
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(recvbar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = blockIdx.x, ks = blockIdx.y, nsplit = gridDim.y;
  const int n0 = nb * kBN;
  const int c_begin = ks * kchunks_per_split, c_end = min(kchunks, c_begin + kchunks_per_split);
  const int nc = max(0, c_end - c_begin);

  // Programmatic dependent launch: the next kernel in the stream may start its own prologue
  // now; this kernel waits for its predecessor only before the first read of X (W is a
  // weight, independent of earlier kernels).
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  if (tid == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 0) tmem_alloc(sTmem, kTmemCols);
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    mbar_init(recvbar, 1);
    mbar_init_fence();
    if (nsplit > 1) {  // the bytes the other nsplit - 1 CTAs of the cluster will send here
      const int G = M * (kBN / 4), r = (int)cluster_rank();
      const int len = (r + 1) * G / nsplit - r * G / nsplit;
      mbar_arrive_expect_tx(recvbar, (uint32_t)((nsplit - 1) * len * 16));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;

  // Two single-thread roles: thread 0 of warp 0 streams chunks into the ring (a stage is
  // refilled as soon as the MMAs that read it complete), thread 0 of warp 1 issues the MMAs.
  // The other lanes of both warps park at __syncwarp rather than spinning in a divergent branch.
  bool failed = false;
  // Feature blocks start their K walk at different chunks (block nb at nb mod nc), so the CTAs
  // in flight read different column ranges of W at any moment instead of all hitting the same
  // 128-byte column of every row.  The order is fixed per block: results stay deterministic.
  const int rot = SK_ROT ? nb % max(nc, 1) : 0;
  auto chunk_of = [&](int c) { return c_begin + (c + rot) % nc; };
  auto atoms_of = [&](int c) { return min(kAtoms, katoms - chunk_of(c) * kAtoms); };
  if (tid == 0) {
    // the first ring's worth of W before waiting on the predecessor grid, then its X
    const int first = min(nc, kStages);
    for (int c = 0; c < first; ++c) {
      const int na = atoms_of(c), a0 = chunk_of(c) * kAtoms;
      mbar_arrive_expect_tx(&full[c], (uint32_t)(na * (kWAtom + kXAtom)));
      for (int a = 0; a < na; ++a) tma_load_2d(sm + c * kStageBytes + a * kWAtom, &tmW, (a0 + a) * kBK, n0, &full[c]);
    }
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    for (int c = 0; c < first; ++c) {
      const int na = atoms_of(c), a0 = chunk_of(c) * kAtoms;
      for (int a = 0; a < na; ++a)
        tma_load_2d(sm + c * kStageBytes + kWBytes + a * kXAtom, &tmX, (a0 + a) * kBK, 0, &full[c]);
    }
    int issued = first;
    for (; issued < nc; ++issued) {
      const int s = issued % kStages;
      if (!mbar_wait_bounded(&empty[s], (uint32_t)((issued / kStages - 1) & 1), kWait)) {
        failed = true;
        break;
      }
      unsigned char* st = sm + s * kStageBytes;
      const int na = atoms_of(issued), a0 = chunk_of(issued) * kAtoms;
      mbar_arrive_expect_tx(&full[s], (uint32_t)(na * (kWAtom + kXAtom)));
      for (int a = 0; a < na; ++a) tma_load_2d(st + a * kWAtom, &tmW, (a0 + a) * kBK, n0, &full[s]);
      for (int a = 0; a < na; ++a) tma_load_2d(st + kWBytes + a * kXAtom, &tmX, (a0 + a) * kBK, 0, &full[s]);
    }
    // the last copy into each stage has landed before the ring is reused (bounded)
    for (int u = max(0, issued - kStages); u < issued; ++u)
      if (!mbar_wait_bounded(&full[u % kStages], (uint32_t)((u / kStages) & 1), kWait)) failed = true;
  } else if (tid == 32) {
    for (int c = 0; c < nc; ++c) {
      const int s = c % kStages;
      if (!mbar_wait_bounded(&full[s], (uint32_t)((c / kStages) & 1), kWait)) {
        failed = true;
        break;
      }
      tc_fence_after();
      const uint32_t wa = smem_u32(sm + s * kStageBytes), xa = wa + kWBytes;
      const int na = atoms_of(c);
      for (int a = 0; a < na; ++a)
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)
          umma_f16_ss(tmem, umma_desc_sw128(wa + a * kWAtom + k * 32, 16, 1024),
                      umma_desc_sw128(xa + a * kXAtom + k * 32, 16, 1024), idesc, (c > 0 || a > 0 || k > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    umma_commit(done);  // every MMA issued above (a failed CTA drains them here too)
  }
  if (warp < 2) __syncwarp();
  if (failed) atomicAdd(&g_sk_wait_timeouts, 1u);
  // the accumulator is complete (or the CTA failed and drains)
  const bool ok = mbar_wait_bounded(done, 0, kWait);
  asm volatile("griddepcontrol.wait;\n" ::: "memory");  // Y is written only after the predecessor ends
  failed = __syncthreads_or(failed || !ok);
  tc_fence_after();
  const int f = warp * 32 + lane;  // this thread's feature within the block (TMEM lane)
  const bool have = nc > 0 && !failed;
  uint32_t r0[32], r1[32];
  {
    const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16);
    tmem_ld32(ta, r0);
    tmem_ld32(ta + 32, r1);
    tmem_wait_ld(r0);
    tmem_wait_ld(r1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (tid == 0 && !ok) atomicAdd(&g_sk_wait_timeouts, 1u);

  if (nsplit == 1) {  // unsplit: each thread writes its feature's column, a warp 32 adjacent features
    const int n = n0 + f;
    if (n < N) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < M) Y[(int64_t)i * ldy + n] = from_f<T>(have ? __uint_as_float(r0[i]) : 0.f);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (32 + i < M) Y[(int64_t)(32 + i) * ldy + n] = from_f<T>(have ? __uint_as_float(r1[i]) : 0.f);
    }
    return;
  }
  float* tile = reinterpret_cast<float*>(sm);  // [token][feature] partial, the ring is free now
  float* recv = tile + kMaxM * kBN;            // [nsplit][slice] received partials
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (i < M) tile[i * kBN + f] = have ? __uint_as_float(r0[i]) : 0.f;
    if (32 + i < M) tile[(32 + i) * kBN + f] = have ? __uint_as_float(r1[i]) : 0.f;
  }
  fence_proxy_async_smem();  // the tile is read by bulk copies (async proxy)
  // every CTA of the cluster has written its tile and is done with its ring (so its receive
  // buffer may be written), and its receive barrier is initialised
  cluster_sync_all();
  // Reduce-scatter through distributed shared memory: the float4 groups of the [M][128] tile
  // are cut into nsplit contiguous slices; CTA p owns slice p.  Thread 0 sends slice p of
  // this tile to CTA p with one bulk copy each (the copy engine moves the bytes, completion
  // counted on p's receive barrier); then every CTA sums its slice over the splits in split
  // order (deterministic) and writes it to Y.
  const int rank = (int)cluster_rank();
  const int G = M * (kBN / 4);
  auto g_lo = [&](int p) { return p * G / nsplit; };
  if (tid == 0) {
    const uint32_t tile_a = smem_u32(tile), recv_a = smem_u32(recv), bar_a = smem_u32(recvbar);
    for (int p = 0; p < nsplit; ++p) {
      if (p == rank) continue;
      const int lo = g_lo(p), len = g_lo(p + 1) - lo;
      uint32_t dst, bar;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(dst) : "r"(recv_a + (uint32_t)(rank * len * 16)),
                   "r"(p));
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(bar) : "r"(bar_a), "r"(p));
      asm volatile(
          "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
          "r"(tile_a + (uint32_t)(lo * 16)), "r"((uint32_t)(len * 16)), "r"(bar)
          : "memory");
    }
    asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
  }
  const bool got = mbar_wait_bounded(recvbar, 0, kWait);
  if (tid == 0 && !got) atomicAdd(&g_sk_wait_timeouts, 1u);
  {
    const int lo = g_lo(rank), len = g_lo(rank + 1) - lo;
    const float4* t4 = reinterpret_cast<const float4*>(tile);
    const float4* r4 = reinterpret_cast<const float4*>(recv);
    for (int gi = tid; gi < len; gi += 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp = 0; sp < nsplit; ++sp) {
        const float4 v = sp == rank ? t4[lo + gi] : r4[sp * len + gi];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int g = lo + gi;
      const int m = g / (kBN / 4), n = n0 + (g % (kBN / 4)) * 4;
      T* yrow = Y + (int64_t)m * ldy;
      if (vec_store && n < N) {  // n % 4 == 0, N % 4 == 0, 8-byte aligned rows
        uint2 pk;
        pk.x = pack2<T>(acc.x, acc.y);
        pk.y = pack2<T>(acc.z, acc.w);
        *reinterpret_cast<uint2*>(yrow + n) = pk;
      } else {
        if (n < N) yrow[n] = from_f<T>(acc.x);
        if (n + 1 < N) yrow[n + 1] = from_f<T>(acc.y);
        if (n + 2 < N) yrow[n + 2] = from_f<T>(acc.z);
        if (n + 3 < N) yrow[n + 3] = from_f<T>(acc.w);
      }
    }
  }
  // this CTA's outgoing copies have finished reading its tile before it exits
  if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
}

}  // namespace

int read_and_clear_skinny_timeouts(unsigned int* count) {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_sk_wait_timeouts, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_sk_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess)
    return set_error(MB_ERR_CUDA, "wait_timeouts: %s", cudaGetErrorString(cudaGetLastError()));
  *count = v;
  return MB_OK;
}

}  // namespace mb

extern "C" int64_t motif_b200_skinny_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  (void)M;
  (void)N;
  (void)K;
  return 0;  // the split-K reduction runs through distributed shared memory
}

extern "C" int motif_b200_skinny_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                                      int64_t M, int64_t N, int64_t K, int dtype, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
  using namespace mb;
  (void)workspace;
  (void)workspace_bytes;
  MB_REQUIRE(x && w && y, MB_ERR_ARG, "skinny_gemm: null pointer");
  MB_REQUIRE(M > 0 && M <= kMaxM && N > 0 && K > 0 && N < (1LL << 31) && K < (1LL << 31), MB_ERR_SHAPE,
             "skinny_gemm: M must be in 1..%d (got %lld)", kMaxM, (long long)M);
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "skinny_gemm: 16-bit dtypes only");
  MB_REQUIRE(K % kBK == 0, MB_ERR_UNSUPPORTED, "skinny_gemm: K must be a multiple of %d (got %lld)", kBK,
             (long long)K);
  MB_REQUIRE(ldx % 8 == 0 && ldw % 8 == 0 && ldx >= K && ldw >= K && ldy >= N &&
                 ((uintptr_t)x | (uintptr_t)w) % 16 == 0 && (uintptr_t)y % 2 == 0,
             MB_ERR_ALIGN, "skinny_gemm: rows must be 16-byte aligned (ldx, ldw multiples of 8)");
  MB_REQUIRE((N + kBN - 1) / kBN < 65536LL * 32, MB_ERR_SHAPE, "skinny_gemm: N too large");
  CUtensorMap tmW, tmX;
  int rc = encode_tile_map_2d(&tmW, w, 2, (uint64_t)K, (uint64_t)N, (uint64_t)ldw * 2, kBK, kBN, 128);
  if (!rc) rc = encode_tile_map_2d(&tmX, x, 2, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, kBK, kMaxM, 128);
  if (rc) return rc;
  const int vec_store = (ldy % 4 == 0 && N % 4 == 0 && (uintptr_t)y % 8 == 0) ? 1 : 0;
  cudaStream_t st = (cudaStream_t)stream;
  auto go = [&](auto t) {
    using T = decltype(t);
    auto kern = skinny_tc_kernel<T>;
    // per device, once: attributes, and how many clusters of each size 1..16 fit at a time
    // guarded by one lock: host threads launching on the same device at once see the table
    // only after it is complete
    static int active[64][kMaxSplit + 1] = {};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
      return set_error(MB_ERR_CUDA, "skinny_gemm: no device");
    std::unique_lock<std::mutex> lock(mu);
    if (!active[dev][0]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess ||
          cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        return check_launch("skinny_gemm (function attributes)");
      for (int cs = 1; cs <= kMaxSplit; ++cs) {
        cudaLaunchConfig_t q = {};
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = 1;
        qa[0].val.clusterDim.y = (unsigned)cs;
        qa[0].val.clusterDim.z = 1;
        q.gridDim = dim3(1, (unsigned)cs);
        q.blockDim = dim3(128);
        q.dynamicSmemBytes = kSmemBytes;
        q.attrs = qa;
        q.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess) n = 0;
        active[dev][cs] = n;
      }
      cudaGetLastError();
      if (active[dev][1] <= 0) return set_error(MB_ERR_CUDA, "skinny_gemm: kernel cannot be resident");
      active[dev][0] = 1;
    }
    lock.unlock();
    // the most K slices whose clusters all fit in one wave
    const int nblk = (int)((N + kBN - 1) / kBN);
    const int kchunks = (int)((K / kBK + kAtoms - 1) / kAtoms);
    int nsplit = 1, per = kchunks;
    for (int want = std::min(kMaxSplit, kchunks); want > 1; --want) {
      const int p = (kchunks + want - 1) / want, ns = (kchunks + p - 1) / p;
      if (nblk <= active[dev][ns]) {
        nsplit = ns;
        per = p;
        break;
      }
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = (unsigned)nsplit;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)nblk, (unsigned)nsplit);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cfg.attrs = at;
    cfg.numAttrs = SK_PDL ? 2 : 1;
    cudaLaunchKernelEx(&cfg, kern, tmW, tmX, (T*)y, ldy, (int)M, (int)N, per,
                       (int)((K / kBK + kAtoms - 1) / kAtoms), (int)(K / kBK), vec_store);
    return check_launch("skinny_gemm");
  };
  return dtype == MB_BF16 ? go(__nv_bfloat16{}) : go(__half{});
}
