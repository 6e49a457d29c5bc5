// Shared helpers of the pn_fir_tau CUDA library: element conversion, error
// plumbing for the C ABI, and small warp/block reductions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pnfirtau_b200.h"

namespace pnft {

// ---- error plumbing (thread-local message returned by pnft_last_error) ----
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
// Records nlaunch successful kernel launches (0 for non-kernel calls) or the
// pending CUDA error.
int check_launch(const char* what, int nlaunch = 1);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- element conversion ----
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// ---- ordered (deterministic) accumulation: per-tile turn counters ----
// A counter per accumulator tile counts the contributions already added; the
// contributor with rank `turn` adds after the counter reaches `turn`, so the
// additions (and their fp32 rounding) happen in one fixed order on every run.
__device__ __forceinline__ int ld_acquire_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Passes the turn on: a release increment at gpu scope. Called by one thread
// after a barrier with the threads whose writes it publishes (the release is
// cumulative over the writes the barrier made visible to it).
__device__ __forceinline__ void turn_pass(int32_t* sem) {
  asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(sem) : "memory");
}
// Bounded wait for *sem >= turn (1 s). On timeout the caller's status word gets
// PNFT_DEV_WAIT_TIMEOUT (and *abort_flag, when given, is set) and the wait gives
// up: the order is then lost but nothing hangs. Also gives up at once when
// *abort_flag is set by another role of the CTA.
__device__ __forceinline__ bool turn_wait(const int32_t* sem, int turn, int32_t* status, volatile int* abort_flag) {
  if (ld_acquire_gpu(sem) >= turn) return true;
  const uint64_t t0 = global_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      if (ld_acquire_gpu(sem) >= turn) return true;
      __nanosleep(64);
    }
    if (abort_flag && *abort_flag) return false;
    if (global_ns() - t0 > 1000000000ull) {
      if (abort_flag) *abort_flag = 1;
      if (status) asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(status), "r"(PNFT_DEV_WAIT_TIMEOUT) : "memory");
      return false;
    }
  }
}

// ---- reductions over the low `width` lanes groups of a warp ----
template <int WIDTH>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int WIDTH>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <int WIDTH>
__device__ __forceinline__ int group_min_i(int v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int WIDTH>
__device__ __forceinline__ int group_sum_i(int v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Deterministic block sum (fixed tree order); `red` must hold blockDim.x/32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = group_sum<32>(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    t = lane < nw ? red[lane] : 0.f;
    t = group_sum<32>(t);
  }
  return t;  // valid in warp 0
}

}  // namespace pnft

#define PNFT_DISPATCH_DTYPE(DT, T, ...)                                   \
  switch (DT) {                                                           \
    case PNFT_DTYPE_F32: {                                                \
      using T = float;                                                    \
      __VA_ARGS__;                                                        \
    } break;                                                              \
    case PNFT_DTYPE_BF16: {                                               \
      using T = __nv_bfloat16;                                            \
      __VA_ARGS__;                                                        \
    } break;                                                              \
    case PNFT_DTYPE_F16: {                                                \
      using T = __half;                                                   \
      __VA_ARGS__;                                                        \
    } break;                                                              \
    default:                                                              \
      return ::pnft::fail(PNFT_EINVAL, "unknown dtype code %d", (int)DT); \
  }
