// Y[M, N] = X[M, K] . W[N, K]^T for a small token count M (decode: one row per sequence,
// M <= 64), 16-bit operands, fp32 accumulation.  At decode every nn.Linear of the model is
// such a product and its cost is streaming W once from HBM (the activations are a few
// hundred KB and stay in L2).
//
// One CTA (4 warps) owns 64 output features (64 consecutive rows of W, contiguous in memory)
// and one slice of K; a 4-stage cp.async ring brings 64x64 tiles of W and X into padded
// shared memory, and every warp computes all M rows x 16 features with m16n8k16 MMAs.  When
// the feature blocks alone cannot fill the GPU (N = 768 outputs, K up to 3584), K is split
// across CTAs: each writes its fp32 partial tile to the workspace, and the last CTA of a
// feature block (counted with an atomic) sums the partials in split order and writes Y — a
// fixed summation order, so results do not depend on which CTA finishes last.  That CTA also
// resets the block's counter, so the workspace stays ready for the next call (and for CUDA
// graph replays).
#include <algorithm>

#include "common.cuh"
#include "gdn_mma.cuh"

namespace mb {
namespace {
using gdnk::lda;
using gdnk::ldb_n;

constexpr int kBN = 64, kBM = 64, kBK = 64, kStages = 4, kNT = 128;
// The counters sit in a fixed-size region at the start of the workspace, so a workspace
// shared by calls of different shapes keeps every counter at zero between calls (the
// partial tiles of one call never land where another call's counters live).
constexpr int64_t kCounterBytes = 32768;  // up to 8192 feature blocks (N <= 524288)
constexpr int kS = kBK + 8;  // padded smem row (elements)

template <typename T>
__global__ void __launch_bounds__(kNT) skinny_gemm_kernel(const T* __restrict__ X, int64_t ldx,
                                                          const T* __restrict__ W, int64_t ldw, T* __restrict__ Y,
                                                          int64_t ldy, int M, int N, int K, int kchunk,
                                                          int* __restrict__ counters, float* __restrict__ part) {
  extern __shared__ __align__(16) unsigned char smem[];
  T* sW = reinterpret_cast<T*>(smem);
  T* sX = sW + (size_t)kStages * kBN * kS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int nb = blockIdx.x, ks = blockIdx.y, nsplit = gridDim.y;
  const int n0 = nb * kBN;
  const int kbeg = ks * kchunk, kend = min(K, kbeg + kchunk);
  const int ntiles = (kend - kbeg + kBK - 1) / kBK;

  auto load = [&](int t, int s) {
    const int k0 = kbeg + t * kBK;
    T* dw = sW + (size_t)s * kBN * kS;
    T* dx = sX + (size_t)s * kBM * kS;
#pragma unroll
    for (int i = 0; i < (kBN * kBK / 8) / kNT; ++i) {  // 4 vectors of W and of X per thread
      const int v = tid + i * kNT;
      const int r = v >> 3, c = (v & 7) * 8;
      const int k = k0 + c;
      const bool kok = k < kend;
      const int n = n0 + r;
      cp_async16(dw + r * kS + c, W + (int64_t)(n < N ? n : 0) * ldw + (kok ? k : 0), kok && n < N);
      cp_async16(dx + r * kS + c, X + (int64_t)(r < M ? r : 0) * ldx + (kok ? k : 0), kok && r < M);
    }
  };

  float acc[4][2][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b) acc[a][b][0] = acc[a][b][1] = acc[a][b][2] = acc[a][b][3] = 0.f;

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < ntiles) load(s, s);
    cp_async_commit();
  }
  for (int t = 0; t < ntiles; ++t) {
    cp_async_wait<kStages - 2>();
    __syncthreads();  // tile t visible; the stage about to be refilled was last read in t-1
    if (t + kStages - 1 < ntiles) load(t + kStages - 1, (t + kStages - 1) % kStages);
    cp_async_commit();
    const T* cw = sW + (size_t)(t % kStages) * kBN * kS;
    const T* cx = sX + (size_t)(t % kStages) * kBM * kS;
#pragma unroll
    for (int kk = 0; kk < kBK; kk += 16) {
      uint32_t bb[4];
      ldb_n(bb, cw, kS, kk, warp * 16);  // W rows = output features, K contiguous
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        if (mt * 16 >= M) break;
        uint32_t a[4];
        lda(a, cx, kS, mt * 16, kk);
        mma_16816<T>(acc[mt][0], a, &bb[0]);
        mma_16816<T>(acc[mt][1], a, &bb[2]);
      }
    }
  }
  cp_async_wait<0>();

  auto out_at = [&](int mt, int nt, int e, int& row, int& col) {
    row = mt * 16 + gq + (e >> 1) * 8;
    col = n0 + warp * 16 + nt * 8 + 2 * tq + (e & 1);
  };
  if (nsplit == 1) {
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          int row, col;
          out_at(mt, nt, e, row, col);
          if (row < M && col < N) {
            if (col + 1 < N)
              *reinterpret_cast<uint32_t*>(Y + (int64_t)row * ldy + col) = pack2<T>(acc[mt][nt][e], acc[mt][nt][e + 1]);
            else
              Y[(int64_t)row * ldy + col] = from_f<T>(acc[mt][nt][e]);
          }
        }
    return;
  }
  // split K: this CTA's fp32 partial tile, then the last CTA of the block reduces
  float* my = part + ((size_t)ks * gridDim.x + nb) * kBM * kBN;
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = mt * 16 + gq + (e >> 1) * 8, c = warp * 16 + nt * 8 + 2 * tq + (e & 1);
        my[r * kBN + c] = acc[mt][nt][e];
      }
  __threadfence();
  __syncthreads();
  __shared__ int last;
  if (tid == 0) last = atomicAdd(&counters[nb], 1) == nsplit - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int i = tid; i < kBM * kBN; i += kNT) {
    const int r = i / kBN, c = i % kBN;
    if (r >= M || n0 + c >= N) continue;
    float s = 0.f;
    for (int sp = 0; sp < nsplit; ++sp)
      s += __ldcg(part + ((size_t)sp * gridDim.x + nb) * kBM * kBN + i);
    Y[(int64_t)r * ldy + n0 + c] = from_f<T>(s);
  }
  if (tid == 0) counters[nb] = 0;
}

// split count: enough CTAs for about two per SM, each K slice a whole number of 64-wide tiles
void plan(int64_t N, int64_t K, int* nblk, int* nsplit, int* kchunk) {
  *nblk = (int)((N + kBN - 1) / kBN);
  const int ktiles = (int)((K + kBK - 1) / kBK);
  int want = std::max(1, (2 * 148 + *nblk - 1) / *nblk);
  want = std::min(want, ktiles);
  const int per = (ktiles + want - 1) / want;
  *kchunk = per * kBK;
  *nsplit = (int)((K + *kchunk - 1) / *kchunk);
}

}  // namespace
}  // namespace mb

extern "C" int64_t motif_b200_skinny_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  int nblk, nsplit, kchunk;
  mb::plan(N, K, &nblk, &nsplit, &kchunk);
  return nsplit == 1 ? 0 : mb::kCounterBytes + (int64_t)nsplit * nblk * mb::kBM * mb::kBN * 4;
}

extern "C" int motif_b200_skinny_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                                      int64_t M, int64_t N, int64_t K, int dtype, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
  using namespace mb;
  MB_REQUIRE(x && w && y, MB_ERR_ARG, "skinny_gemm: null pointer");
  MB_REQUIRE(M > 0 && M <= kBM && N > 0 && K > 0 && N < (1LL << 31) && K < (1LL << 31), MB_ERR_SHAPE,
             "skinny_gemm: M must be in 1..%d (got %lld)", kBM, (long long)M);
  MB_REQUIRE(dtype == MB_BF16 || dtype == MB_F16, MB_ERR_UNSUPPORTED, "skinny_gemm: 16-bit dtypes only");
  MB_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && ldw % 8 == 0 && ldy % 2 == 0 &&
                 ((uintptr_t)x | (uintptr_t)w) % 16 == 0 && (uintptr_t)y % 4 == 0,
             MB_ERR_ALIGN, "skinny_gemm: rows must be 16-byte aligned (K, ldx, ldw multiples of 8)");
  const int64_t need = motif_b200_skinny_gemm_workspace_bytes(M, N, K);
  MB_REQUIRE(workspace_bytes >= need && (need == 0 || workspace != nullptr), MB_ERR_ARG,
             "skinny_gemm: workspace of %lld bytes needed", (long long)need);
  int nblk, nsplit, kchunk;
  plan(N, K, &nblk, &nsplit, &kchunk);
  const int smem = kStages * (kBN + kBM) * kS * 2;
  int* counters = (int*)workspace;
  MB_REQUIRE((int64_t)nblk * 4 <= kCounterBytes, MB_ERR_SHAPE, "skinny_gemm: N too large");
  float* part = nsplit > 1 ? (float*)((char*)workspace + kCounterBytes) : nullptr;
  cudaStream_t st = (cudaStream_t)stream;
  auto go = [&](auto t) {
    using T = decltype(t);
    auto kern = skinny_gemm_kernel<T>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return check_launch("skinny_gemm (shared memory attribute)");
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    kern<<<dim3((unsigned)nblk, (unsigned)nsplit), kNT, smem, st>>>((const T*)x, ldx, (const T*)w, ldw, (T*)y, ldy,
                                                                  (int)M, (int)N, (int)K, kchunk, counters, part);
    return check_launch("skinny_gemm");
  };
  return dtype == MB_BF16 ? go(__nv_bfloat16{}) : go(__half{});
}
