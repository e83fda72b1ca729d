// Shared helpers for the Laguna B200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include <utility>

#include "../../include/laguna_b200.h"

namespace lg {

// Thread-local last-error message for lg_last_error().
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);

// Kernel launches issued by this library (all threads), read by lg_launch_count().
void count_launch();
// Optional CUDA events recorded around one named stage (lg_profile_stage); no-ops otherwise.
void prof_begin(const char* stage, cudaStream_t s);
void prof_end(const char* stage, cudaStream_t s);

#define LG_CHECK_ARG(cond, ...)                                  \
  do {                                                           \
    if (!(cond)) return ::lg::fail(LG_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define LG_CUDA_TRY(expr)                                                          \
  do {                                                                             \
    cudaError_t e_ = (expr);                                                       \
    if (e_ != cudaSuccess)                                                         \
      return ::lg::fail(LG_ERR_CUDA, "%s: %s (%s:%d)", #expr,                      \
                        cudaGetErrorString(e_), __FILE__, __LINE__);               \
  } while (0)

// Launch-error check after a <<<>>> launch (also counts the launch).
#define LG_LAUNCH_CHECK(name)                                                      \
  do {                                                                             \
    cudaError_t e_ = cudaGetLastError();                                           \
    if (e_ != cudaSuccess)                                                         \
      return ::lg::fail(LG_ERR_CUDA, "launch %s: %s", name, cudaGetErrorString(e_)); \
    ::lg::count_launch();                                                          \
  } while (0)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Carves consecutive 256-byte aligned regions out of a caller workspace.
struct Carver {
  char* base;
  size_t used = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    used = align_up(used, 256);
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += count * sizeof(T);
    return p;
  }
};

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float bf16_bits_to_f(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// Exact small-integer -> float for codes in [0, 2^23): 2^23 + c has c in the mantissa.
__device__ __forceinline__ float code_to_f(uint32_t c) {
  return __uint_as_float(0x4B000000u | c) - 8388608.0f;
}

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

// The warp-wide minimum and maximum, in place.
__device__ __forceinline__ void warp_minmax(float& lo, float& hi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
}

// Atomic add with acquire-release semantics at GPU scope, returning the old value: the
// last-arriver pattern without full fences. Stores that the calling thread's CTA (or warp)
// ordered before it with a barrier are released with it; the thread that sees the final count
// acquires every earlier arriver's, and passes them on to its CTA (or warp) through a barrier.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  return (int)atom_add_acq_rel_gpu(reinterpret_cast<unsigned*>(p), (unsigned)v);
}

// Read-only 128-bit global load that bypasses L1 allocation (weights are streamed once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__device__ __forceinline__ void red_add_v4_f32(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// ---- MLX affine quantization of one group (the library's quantizer arithmetic) ------------
// scale = bf16((max - min) / (2^bits - 1)), bias = bf16(min) (IEEE division); a value's code is
// rint((v - bias) / scale) clamped to [0, 2^bits - 1] (0 when scale == 0).
__device__ __forceinline__ void quant_group_params(float lo, float hi, float nb,
                                                   __nv_bfloat16* sbf, __nv_bfloat16* bbf) {
  *sbf = __float2bfloat16_rn(__fdiv_rn(hi - lo, nb));
  *bbf = __float2bfloat16_rn(lo);
}
__device__ __forceinline__ uint32_t quant_code(float v, float s, float bv, float nb) {
  float q = (s == 0.f) ? 0.f : rintf(__fdiv_rn(v - bv, s));
  q = fminf(fmaxf(q, 0.f), nb);
  return (uint32_t)q;
}

// ---- programmatic dependent launch (PDL) -------------------------------------------------
// Kernels of the decode chain may be launched so that they start while the previous kernel in
// the stream is still running (lg_set_pdl). Each such kernel calls pdl_wait() before it reads
// anything the previous kernel may write, and pdl_trigger() only after its own wait, so when a
// kernel starts, every kernel before its immediate predecessor has completed: before its wait
// it may read static data (weights) and data from earlier kernels, never its predecessor's
// output. Without the launch attribute both instructions return at once.
// Both are issued by a converged warp: code before them often branches on the lane (a thread
// that zeroes a flag, the first threads reading a few words), and inline asm gives the compiler
// no reason to rejoin the warp first.
__device__ __forceinline__ void pdl_wait() {
  __syncwarp();
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  __syncwarp();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool pdl_enabled();

// Launch with the programmatic-serialization attribute when PDL is on (plain launch otherwise).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  if (pdl_enabled()) {
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Multiprocessor count of the current device (cached per device).
int device_sm_count();

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024); returns the exclusive
// prefix and writes the block total to *total.
__device__ __forceinline__ int block_excl_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += u;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? warp_tot[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += u;
    }
    if (lane < nw) warp_tot[lane] = wi - w;  // exclusive warp offsets
    if (lane == nw - 1) *total = wi;
  }
  __syncthreads();
  return warp_tot[warp] + inc - v;
}

}  // namespace lg
