// Error reporting for the C ABI (thread-local last message), and the
// per-context bookkeeping the launchers share.
#include <cuda.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace pts {

static thread_local char g_last_error[512] = "";

constexpr long long kDefaultWaitLimit = 4000000000ll;     // SM clocks, about 2 s at the top clock
static std::atomic<long long> g_wait_limit{kDefaultWaitLimit};

long long wait_limit_cycles() { return g_wait_limit.load(std::memory_order_relaxed); }

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

int current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = (CtxGetCurrentFn)f;
    f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = (CtxGetIdFn)f;
  });
  if (!get_current || !get_id) return set_error(PTS_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return set_error(PTS_ERR_CUDA, "no current CUDA context");
  if (get_id(ctx, id) != CUDA_SUCCESS) return set_error(PTS_ERR_CUDA, "cuCtxGetId failed");
  return PTS_OK;
}

int ensure_smem_attr(const void* func, size_t bytes, bool max_carveout) {
  static std::mutex mu;
  static std::map<std::pair<unsigned long long, const void*>, size_t> done;
  unsigned long long ctx = 0;
  const bool keyed = current_context_id(&ctx) == PTS_OK;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(ctx, func);
  if (keyed) {
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return PTS_OK;
  }
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && max_carveout)
    e = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess)
    return set_error(PTS_ERR_CUDA, "cudaFuncSetAttribute(%zu bytes): %s", bytes, cudaGetErrorString(e));
  if (keyed) done[key] = bytes;
  return PTS_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tiled_bf16_sw128(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims,
                            const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)f;
  });
  if (!fn) return set_error(PTS_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  const CUresult rc = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), dims,
                         strides_bytes, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return set_error(PTS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)rc);
  return PTS_OK;
}

}  // namespace pts

extern "C" const char* pts_last_error(void) { return pts::g_last_error; }

extern "C" int pts_version(void) { return 1; }

extern "C" long long pts_set_wait_limit(long long cycles) {
  const long long v = cycles > 0 ? cycles : pts::kDefaultWaitLimit;
  return pts::g_wait_limit.exchange(v);
}
