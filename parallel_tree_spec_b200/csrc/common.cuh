// Shared helpers for the B200 tree-verification kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/pts_b200.h"

namespace pts {

// Records a message for pts_last_error() and returns the code.
int set_error(int code, const char* fmt, ...);

// SM clocks a kernel's progress waits (on other warps, other CTAs or copies)
// may take before the kernel gives up and reports an error; set process-wide
// with pts_set_wait_limit.
long long wait_limit_cycles();

// The unique id of the current CUDA context (cuCtxGetId); PTS_ERR_CUDA when
// there is none.
int current_context_id(unsigned long long* id);

// Raises `func`'s dynamic shared-memory limit to `bytes` (and, if asked, its
// preferred carveout to the maximum) in the current context.  Thread-safe;
// the attribute call is made once per (context, kernel) and size.
int ensure_smem_attr(const void* func, size_t bytes, bool max_carveout = false);

// A bf16 TMA tensor map of `rank` dimensions with 128-byte swizzle (zero fill
// out of bounds); dims innermost first, strides of dims 1.. in bytes.
int encode_tiled_bf16_sw128(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims,
                            const cuuint64_t* strides_bytes, const cuuint32_t* box);

#define PTS_CHECK_ARG(cond, ...)                                  \
  do {                                                            \
    if (!(cond)) return ::pts::set_error(PTS_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define PTS_CUDA_TRY(expr)                                                        \
  do {                                                                            \
    cudaError_t _e = (expr);                                                      \
    if (_e != cudaSuccess)                                                        \
      return ::pts::set_error(PTS_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(PTS_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return PTS_OK;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Programmatic dependent launch.  A kernel launched with launch_pdl may be
// scheduled while the stream's previous kernel is still running (once every
// CTA of that kernel has called pdl_trigger or exited); it runs its setup and
// then calls pdl_wait, which returns when the previous kernel has completed
// and its memory is visible.  Nothing before pdl_wait may read or write memory
// that earlier work in the stream writes or reads.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

__device__ __forceinline__ float bf16_bits_to_float(uint32_t b16) {
  return __uint_as_float(b16 << 16);
}

// Round-to-nearest-even float -> bf16, returned widened back to float.
__device__ __forceinline__ float round_to_bf16(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return __uint_as_float(0x7fc00000u);
  u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint16_t float_to_bf16_bits(float x) {
  return (uint16_t)(__float_as_uint(round_to_bf16(x)) >> 16);
}

// Philox4x32-10 (Salmon et al., SC'11).
struct Philox4 {
  uint32_t v[4];
};

__device__ __forceinline__ Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                                 uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
  }
  Philox4 o;
  o.v[0] = c0;
  o.v[1] = c1;
  o.v[2] = c2;
  o.v[3] = c3;
  return o;
}

// Uniform k of request b's stream: (philox(...)[k & 3] >> 8) * 2^-24.
__device__ __forceinline__ float philox_uniform(uint64_t seed, uint64_t offset, uint32_t b, uint32_t k) {
  Philox4 o = philox4x32_10(k >> 2, b, (uint32_t)offset, (uint32_t)(offset >> 32), (uint32_t)seed,
                            (uint32_t)(seed >> 32));
  return (float)(o.v[k & 3] >> 8) * 5.9604644775390625e-08f;
}

}  // namespace pts
