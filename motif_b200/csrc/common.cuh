// Shared device helpers for the Motif Chord sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/motif_b200.h"

namespace mb {

// ------------------------------------------------------------------ status plumbing
// Records a message for motif_b200_last_error() and returns the code.
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
// 2-D tiled tensor map over a row-major [rows, inner] array (16-bit elements are encoded as
// bf16: the bulk tensor copy only moves bytes, so fp16 data is carried unchanged).
int encode_tile_map_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, int swizzle_bytes);
// Rank-N tiled tensor map: dims[0] is the contiguous dimension; strides_bytes[i] is the byte
// stride of dimension i + 1 (multiples of 16).
int encode_tile_map(CUtensorMap* map, const void* base, int elem_bytes, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

// Runs `setup(key, arg)` once per (key, current device) under a process-wide lock.
int once_per_device(const void* key, int (*setup)(const void*, int), int arg);
// Raises a kernel's dynamic shared-memory limit to `bytes` once per device (thread-safe).
int ensure_smem_attr(const void* func, int bytes);
// True while a test has switched testing knob `knob` on (motif_b200_testing_force).
bool forced(int knob);

#define MB_REQUIRE(cond, code, ...)                  \
  do {                                               \
    if (!(cond)) return ::mb::set_error((code), __VA_ARGS__); \
  } while (0)

// ------------------------------------------------------------------ type helpers
template <typename T> struct TypeOf;
template <> struct TypeOf<float> { static constexpr int id = MB_F32; };
template <> struct TypeOf<__half> { static constexpr int id = MB_F16; };
template <> struct TypeOf<__nv_bfloat16> { static constexpr int id = MB_BF16; };

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sigmoid / SiLU / softplus in fp32.  Sigmoid uses the __expf / __fdividef intrinsics (relative
// error ~1e-6, far below the 1e-5 fp32 bar and the 16-bit rounding); softplus keeps the
// accurate expf / log1pf.
__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float ex2f_(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcpf_(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// SiLU x / (1 + e^-x), with e^-x = 2^(-x log2 e) on the MUFU ex2 unit and the reciprocal on
// MUFU rcp (relative error a few 1e-7); silu2_ is the same arithmetic on a channel pair with the
// multiplies and the add packed (bit-identical per lane).
constexpr float kNegLog2e = -1.4426950408889634f;
__device__ __forceinline__ float siluf_(float x) { return x * rcpf_(1.0f + ex2f_(x * kNegLog2e)); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mul.rn.f32x2 rd, ra, rb;\n"
      " mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n add.rn.f32x2 rd, ra, rb;\n"
      " mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
// The causal depthwise conv of the gated delta-net preparation, one fixed evaluation order
// (((w0 x0 + w1 x1) + w2 x2) + w3 x3, one multiply then fmas) shared by every kernel that
// computes it, scalar or packed.
__device__ __forceinline__ float conv4f(float w0, float w1, float w2, float w3, float x0, float x1, float x2,
                                        float x3) {
  return fmaf(w3, x3, fmaf(w2, x2, fmaf(w1, x1, w0 * x0)));
}
__device__ __forceinline__ float2 silu2_(float2 x) {
  const float2 t = fmul2(x, make_float2(kNegLog2e, kNegLog2e));
  const float2 d = fadd2(make_float2(ex2f_(t.x), ex2f_(t.y)), make_float2(1.0f, 1.0f));
  return fmul2(x, make_float2(rcpf_(d.x), rcpf_(d.y)));
}
// scale / max(||x||, 1e-12) from ss = ||x||^2 (F.normalize's clamp), as one reciprocal square
// root: the q / k L2 norms of the gated delta-net preparation.
__device__ __forceinline__ float l2_scale(float ss, float scale) { return scale * rsqrtf(fmaxf(ss, 1e-24f)); }
// torch.nn.functional.softplus with beta=1, threshold=20.
__device__ __forceinline__ float softplusf_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// ------------------------------------------------------------------ PTX wrappers
// Programmatic dependent launch: a kernel launched after this one with the programmatic
// stream serialization attribute (the decode-time skinny GEMM) may start now, on the SMs this
// kernel leaves free; it fetches its weights and then waits (griddepcontrol.wait) for this
// kernel to complete before it reads anything this kernel writes.  No effect on a dependent
// launched without the attribute.
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  // Zero-fills the 16 destination bytes when `valid` is false.
  const int src_bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Round an fp32 value to TF32 (round-to-nearest, ties away), kept in a 32-bit register.
__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return r;
}

// D = A(16x8, row) * B(8x8, col) + D, tf32 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_tf32(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// D = A(16x16, row) * B(16x8, col) + D, bf16 / fp16 inputs, fp32 accumulate.
template <typename T>
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, const uint32_t* b);
template <>
__device__ __forceinline__ void mma_16816<__nv_bfloat16>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
__device__ __forceinline__ void mma_16816<__half>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Pack two fp32 values into one 32-bit register of two 16-bit floats (lo = first).
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Two fp32 values rounded to T and back (one packed conversion instead of two).
template <typename T> __device__ __forceinline__ float2 round2(float a, float b);
template <>
__device__ __forceinline__ float2 round2<__nv_bfloat16>(float a, float b) {
  return __bfloat1622float2(__floats2bfloat162_rn(a, b));
}
template <>
__device__ __forceinline__ float2 round2<__half>(float a, float b) {
  return __half22float2(__floats2half2_rn(a, b));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t* r, const void* smem) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(smem)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t* r, const void* smem) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(smem)));
}

// ------------------------------------------------------------------ mbarrier + bulk copy
// One-dimensional bulk copies (cp.async.bulk, the untiled TMA path) global -> shared with
// completion counted on an mbarrier by transaction bytes.  Source and destination must be
// 16-byte aligned and the size a multiple of 16.  The destination is this CTA only.
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the async (bulk copy) proxy; follow with __syncthreads.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses before later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Tiled tensor copy of one box at coordinates (x = inner element index, y = row); x * element
// size must be a multiple of 16 bytes.  The destination is this CTA only.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------ tcgen05 / TMEM
// Shared-memory matrix descriptor for a tile stored with the 128-byte swizzle (rows of 128
// bytes, 8-row atoms of 1024 bytes, 16-byte chunk c of row r at chunk c ^ (r & 7)):
// start address and byte offsets in 16-byte units, descriptor version 1, layout type 2.
// K-major operands: lbo = 16 (unused), sbo = 1024 (next 8 rows).  MN-major operands
// (rows along K): sbo = 1024 (next 8 K-rows), lbo = offset of the next 64-element MN block.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// Instruction descriptor of kind::f16 with fp32 accumulation: a/b format 0 = f16, 1 = bf16;
// major 0 = K-major, 1 = MN-major; N in multiples of 8 (bits 17..22 hold N / 8), M / 16 in
// bits 24..28.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t ab_fmt, int M, int N, uint32_t a_major,
                                                      uint32_t b_major) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_major << 15) | (b_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[smem] * B[smem], issued by one thread.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
// Whole-warp TMEM allocation of `ncols` columns (a power of two >= 32); the base address is
// written to shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
// 32 consecutive 32-bit columns of this thread's TMEM lane (warp w of a warpgroup reads
// lanes 32w .. 32w+31).  The registers are valid only after tmem_wait_ld(r), which also
// carries them as operands so that no use is scheduled before the wait.
#define MB_R32(r)                                                                                              \
  "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), \
      "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),  \
      "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),  \
      "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" : MB_R32(r)::"memory");
}
// Two independent fp32 fused multiply-adds in one instruction (sm_100 fma.rn.f32x2): each lane
// rounds exactly as fmaf does.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}
// max of three fp32 values in one instruction (sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of `bar` to complete.  Returns false after `limit` polls
// (each poll may itself suspend for a hardware-defined interval), so a copy that never
// lands ends the wait with an error instead of a hang.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ------------------------------------------------------------------ fused SwiGLU role
// The SwiGLU MLP activation act[r, :] = gu[r, :hid] * round(silu(gu[r, hid:2 hid]))
// (motif/ops/swiglu.py:252-253), one 8-element (16-byte) group per thread.  Decode kernels
// whose launch would otherwise be followed by a separate SwiGLU launch append
// swiglu_role_blocks() CTAs to their grid that run this instead (the two are independent:
// both read the same packed projection row), saving one launch per decoder.
// Needs hid % 8 == 0, 16-byte aligned rows and strides that are multiples of 8.
template <typename T>
struct SwigluRole {
  const T* gu;   // [rows, 2 hid] value | gate, row stride gs
  int64_t gs;
  T* act;        // [rows, hid], row stride as
  int64_t as;
  int64_t rows;
  int hid;       // 0: no SwiGLU role
};
template <typename T>
__device__ __forceinline__ void swiglu_group(const T* __restrict__ x, int64_t xs, T* __restrict__ y, int64_t ys,
                                             int N, int64_t i) {
  const int nv = N / 8;
  const int64_t row = i / nv;
  const int c = (int)(i % nv) * 8;
  const T* xr = x + row * xs;
  const uint4 rv = *reinterpret_cast<const uint4*>(xr + c);
  const uint4 rg = *reinterpret_cast<const uint4*>(xr + N + c);
  const T* v8 = reinterpret_cast<const T*>(&rv);
  const T* g8 = reinterpret_cast<const T*>(&rg);
  __align__(16) T o8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float sg = to_f(from_f<T>(siluf_(to_f(g8[e]))));
    o8[e] = from_f<T>(to_f(v8[e]) * sg);
  }
  *reinterpret_cast<uint4*>(y + row * ys + c) = *reinterpret_cast<const uint4*>(o8);
}
// Thread `first` of the role's CTAs, `stride` role threads in all.
template <typename T>
__device__ __forceinline__ void swiglu_role_run(const SwigluRole<T>& sw, int64_t first, int64_t stride) {
  const int64_t total = sw.rows * (sw.hid / 8);
  for (int64_t i = first; i < total; i += stride) swiglu_group<T>(sw.gu, sw.gs, sw.act, sw.as, sw.hid, i);
}
inline int64_t swiglu_role_blocks(int64_t rows, int64_t hid, int threads) {
  return hid > 0 ? (rows * (hid / 8) + threads - 1) / threads : 0;
}
inline bool swiglu_role_ok(const void* gu, int64_t gs, const void* act, int64_t as, int64_t hid) {
  return hid > 0 && hid % 8 == 0 && gs % 8 == 0 && as % 8 == 0 && ((uintptr_t)gu | (uintptr_t)act) % 16 == 0;
}

}  // namespace mb
