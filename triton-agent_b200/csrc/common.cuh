// Shared definitions for the sm_100a kernels of libb200ops.so: status
// handling, dtype conversion, vector memory access and the per-translation-
// unit device error word that bounded waits and checked paths report into.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <type_traits>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200ops.h"

namespace b200 {

// ---------------------------------------------------------------------------
// Host-side helpers
// ---------------------------------------------------------------------------

// Returns B200_ERR_INJECTED when the environment variable
// B200OPS_INJECT_ERROR names this op (or "all").  Used by host-side fault
// tests: the failure is produced on the host, before any launch.
int injected_error(const char* op_name);

// Maps the result of a launch to a status, recording the CUDA error text.
int launch_status(cudaError_t e);
void set_last_error_detail(const char* msg);

inline int dtype_size(int32_t dt) {
  switch (dt) {
    case B200_F32: return 4;
    case B200_F16: return 2;
    case B200_BF16: return 2;
    case B200_I8: return 1;
    case B200_I32: return 4;
    case B200_I64: return 8;
    default: return 0;
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int device_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n;
}

// Registry of per-translation-unit device error readers (see
// B200_DEVICE_ERROR_WORD).  Each reader copies its word to the host, clears
// it, and returns the word.
typedef int (*error_reader_fn)(cudaStream_t);
struct ErrorReaderRegistrar {
  explicit ErrorReaderRegistrar(error_reader_fn fn);
};
int read_all_device_errors(cudaStream_t stream, int32_t* out);

// ---------------------------------------------------------------------------
// Device-side error codes (written into the error word; first writer wins)
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrTimeoutFull = 1,     // consumer gave up waiting for a filled stage
  kDevErrTimeoutEmpty = 2,    // producer gave up waiting for a free stage
  kDevErrTimeoutMma = 3,      // epilogue gave up waiting for the accumulator
  kDevErrTimeoutCombine = 4,  // combine step gave up waiting for partials
  kDevErrTimeoutPeer = 6,     // a cross-GPU flag wait gave up waiting for a peer rank
};

// Limit of the cross-GPU flag waits (fused all-gather GEMM), in ns of global
// time: b200_set_peer_wait_timeout_us, default 2 s.  The mbarrier waits
// inside a CTA keep their fixed 2 s limit.
uint64_t peer_wait_timeout_ns();

}  // namespace b200

// Defines a device error word private to the including .cu file and registers
// a host reader for it.  Kernels call b200_dev_error(code) to record the
// first failure they see.
#define B200_DEVICE_ERROR_WORD()                                                   \
  static __device__ int g_b200_dev_error = 0;                                      \
  static __device__ __forceinline__ void b200_dev_error(int code) {                \
    atomicCAS(&g_b200_dev_error, 0, code);                                         \
  }                                                                                \
  static int b200_read_tu_error(cudaStream_t s) {                                  \
    int v = 0, z = 0;                                                              \
    if (cudaMemcpyFromSymbolAsync(&v, g_b200_dev_error, sizeof(int), 0,            \
                                  cudaMemcpyDeviceToHost, s) != cudaSuccess)       \
      return -1;                                                                   \
    if (cudaMemcpyToSymbolAsync(g_b200_dev_error, &z, sizeof(int), 0,              \
                                cudaMemcpyHostToDevice, s) != cudaSuccess)         \
      return -1;                                                                   \
    if (cudaStreamSynchronize(s) != cudaSuccess) return -1;                        \
    return v;                                                                      \
  }                                                                                \
  static b200::ErrorReaderRegistrar g_b200_err_registrar(&b200_read_tu_error);

// ---------------------------------------------------------------------------
// Device-side dtype helpers
// ---------------------------------------------------------------------------
namespace b200 {

template <typename T> struct Vec;  // 16-byte vector of T
template <> struct Vec<float> { static constexpr int N = 4; };
template <> struct Vec<__half> { static constexpr int N = 8; };
template <> struct Vec<__nv_bfloat16> { static constexpr int N = 8; };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Loads a 16-byte vector of T from global memory and widens it to fp32.
template <typename T>
__device__ __forceinline__ void load16_f32(const T* p, float* out) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) out[i] = to_f32(e[i]);
}

// Streaming (evict-first) 16-byte load for data read exactly once.
template <typename T>
__device__ __forceinline__ uint4 ldg_stream16(const T* p) {
  uint4 r;
  asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void stg_stream16(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& raw, float* out) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) out[i] = to_f32(e[i]);
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* in) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) e[i] = from_f32<T>(in[i]);
  return raw;
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

// ---- symmetric INT8 quantisation of one value (quant_matmul/reference.py:16-24)
// Eager PyTorch divides in fp32 and rounds the quotient to x's dtype before
// round() (half to even); the scale max|x|/127 is rounded to that dtype too.
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32(from_f32<T>(v));
}

template <typename T>
__device__ __forceinline__ int8_t quant_one(float x, float s) {
  float qv = round_to<T>(__fdiv_rn(x, s));
  qv = rintf(qv);
  qv = fminf(fmaxf(qv, -127.f), 127.f);
  return (int8_t)(int)qv;
}

// The same code without the conversion pipe (which runs at a fraction of the
// ALU rate and bounds a quantiser otherwise): x / s by Markstein's correction
// step (P. Markstein, IBM J. Res. Dev. 1990) from r = 1/s correctly rounded,
// q0 = RN(x r), e = x - q0 s exactly, RN(q0 + e r) = RN(x / s); rounding to
// T's precision on the bits (round half to even; for fp16 values below its
// normal range the result only feeds the integer rounding, which gives 0
// either way); round half to even to an integer by adding 1.5 * 2^23 (exact
// for |v| < 2^22); clamp in integers.  Bit-identical to quant_one.
template <typename T>
__device__ __forceinline__ float round_bits_to(float v) {
  if constexpr (std::is_same<T, float>::value) {
    return v;
  } else {
    uint32_t u = __float_as_uint(v);
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      u += 0x7FFFu + ((u >> 16) & 1u);
      u &= 0xFFFF0000u;
    } else {
      u += 0xFFFu + ((u >> 13) & 1u);
      u &= 0xFFFFE000u;
    }
    return __uint_as_float(u);
  }
}

// Rounds two floats to T's precision (round half to even) in place: one
// packed conversion and two widenings for the 16-bit types, nothing for fp32.
template <typename T>
__device__ __forceinline__ void round_pair_to(float& a, float& b) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const uint32_t u = *reinterpret_cast<const uint32_t*>(&h);
    a = __uint_as_float(u << 16);
    b = __uint_as_float(u & 0xFFFF0000u);
  } else if constexpr (std::is_same<T, __half>::value) {
    const float2 f = __half22float2(__floats2half2_rn(a, b));
    a = f.x;
    b = f.y;
  }
}

template <typename T>
__device__ __forceinline__ int quant_code_fast(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float e = __fmaf_rn(-q0, s, x);
  const float qt = round_bits_to<T>(__fmaf_rn(e, r, q0));
  const int i = __float_as_int(__fadd_rn(qt, 12582912.0f)) - 0x4B400000;
  return max(-127, min(127, i));
}

template <typename T>
__device__ __forceinline__ float finish_scale(float amax) {
  float s = round_to<T>(__fdiv_rn(amax, 127.0f));
  if (s == 0.f) s = round_to<T>(1e-6f);
  return s;
}

}  // namespace b200

// Dispatches a float dtype code to a C++ type alias `scalar_t`.
#define B200_DISPATCH_FLOAT(DT, ...)                         \
  [&]() -> int {                                             \
    switch (DT) {                                            \
      case B200_F32: { using scalar_t = float; return __VA_ARGS__(); }          \
      case B200_F16: { using scalar_t = __half; return __VA_ARGS__(); }         \
      case B200_BF16: { using scalar_t = __nv_bfloat16; return __VA_ARGS__(); } \
      default: return B200_ERR_UNSUPPORTED;                  \
    }                                                        \
  }()

#define B200_DISPATCH_HALF(DT, ...)                          \
  [&]() -> int {                                             \
    switch (DT) {                                            \
      case B200_F16: { using scalar_t = __half; return __VA_ARGS__(); }         \
      case B200_BF16: { using scalar_t = __nv_bfloat16; return __VA_ARGS__(); } \
      default: return B200_ERR_UNSUPPORTED;                  \
    }                                                        \
  }()
