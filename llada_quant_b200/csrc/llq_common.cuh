// Shared helpers of the llada_quant CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <string>
#include <cstdlib>
#include <atomic>
#include <utility>

#include "../../include/llada_quant.h"

namespace llq {

// ---------------------------------------------------------------------------
// error reporting across the C ABI
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(LLQ_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return LLQ_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// SM count of the current device (cached per device ordinal)
inline int num_sms() {
  constexpr int kMaxDev = 64;
  static int cache[kMaxDev] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) dev = 0;
  if (dev >= kMaxDev) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  }
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// true once per (flag set, device): callers use it to set per-device kernel attributes
// (setting a function attribute twice is harmless, so a race only repeats it)
inline bool first_use_on_device(std::atomic<uint64_t>& seen_mask) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return true;
  const uint64_t bit = 1ull << dev;
  return (seen_mask.fetch_or(bit) & bit) == 0;
}

// ---------------------------------------------------------------------------
// programmatic dependent launch: the layer's kernels are launched so that the
// next one is scheduled while the previous one drains; each waits for its
// predecessor's results (griddepcontrol.wait, a no-op without the attribute)
// before reading them and releases its dependents once its work is issued.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// `co_resident`: the launch fails unless every CTA of the grid can be resident at
// once (cooperative launch), for kernels whose CTAs wait on one another
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_ex(bool co_resident, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = co_resident ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  return launch_pdl_ex(false, kernel, grid, block, smem, st, std::forward<Args>(args)...);
}

// device error word (bounded waits record where they gave up)
extern __device__ int32_t g_device_error;

// ---------------------------------------------------------------------------
// element helpers
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// round-to-nearest-even float -> bf16 bits (finite inputs), == torch's cast
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float round_bf16(float f) {
  return __bfloat162float(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// signed nibble j (0 = low) of a packed byte, as the reference's unpack_int4
__device__ __forceinline__ int nibble(int8_t b, int hi) {
  int v = static_cast<int>(b);
  return hi ? (v >> 4) : (static_cast<int>(static_cast<uint32_t>(v) << 28) >> 28);
}

}  // namespace llq
