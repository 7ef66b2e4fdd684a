// Status / error plumbing shared by every C-ABI entry point.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

#include <cudaTypedefs.h>

#include "common.cuh"

namespace mb {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  g_last_error[0] = '\0';
  return MB_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
static std::once_flag g_encode_once;

int encode_tile_map(CUtensorMap* map, const void* base, int elem_bytes, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode_tiled == nullptr) return set_error(MB_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  if (rank < 1 || rank > 5) return set_error(MB_ERR_ARG, "tensor map rank %d", rank);
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    estr[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = g_encode_tiled(map, dt, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MB_OK;
}

int encode_tile_map_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, int swizzle_bytes) {
  const uint64_t dims[2] = {inner, rows};
  const uint64_t strides[1] = {row_stride_bytes};
  const uint32_t box[2] = {box_inner, box_rows};
  return encode_tile_map(map, base, elem_bytes, 2, dims, strides, box, swizzle_bytes);
}

// Per-(kernel, device) one-time set-up, e.g. the dynamic shared-memory limit that
// cudaFuncSetAttribute must raise before the first launch on each device.  The set-up runs
// under one process-wide lock, so host threads launching on the same device at once neither
// race on the bookkeeping nor launch before the attribute is in place; a failed set-up is
// not recorded and is retried by the next call.
static std::mutex g_once_mu;
static std::map<std::pair<const void*, int>, bool> g_once_done;

int once_per_device(const void* key, int (*setup)(const void*, int), int arg) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(MB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_once_mu);
  auto it = g_once_done.find({key, dev});
  if (it != g_once_done.end()) return MB_OK;
  const int rc = setup(key, arg);
  if (rc == MB_OK) g_once_done[{key, dev}] = true;
  return rc;
}

static int set_smem_attr(const void* func, int bytes) {
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute (dynamic shared memory)");
  return MB_OK;
}

int ensure_smem_attr(const void* func, int bytes) { return once_per_device(func, set_smem_attr, bytes); }

// Testing hooks (motif_b200_testing_force): off unless a test turns them on.
static std::atomic<int> g_force[MB_FORCE_COUNT];

bool forced(int knob) { return knob >= 0 && knob < MB_FORCE_COUNT && g_force[knob].load(std::memory_order_relaxed); }

}  // namespace mb

extern "C" int motif_b200_testing_force(int knob, int value) {
  MB_REQUIRE(knob >= 0 && knob < MB_FORCE_COUNT, MB_ERR_ARG, "testing_force: unknown knob %d", knob);
  mb::g_force[knob].store(value ? 1 : 0, std::memory_order_relaxed);
  return MB_OK;
}

extern "C" const char* motif_b200_last_error(void) { return mb::g_last_error; }
extern "C" int motif_b200_abi_version(void) { return 1; }
