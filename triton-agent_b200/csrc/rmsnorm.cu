// RMSNorm, y = x * rsqrt(mean(x^2) + eps) * w, one CTA per row.
//
// Reference: triton_agent/ops/rmsnorm/reference.py:17-18.
//
// HBM-bound: every byte of x is read once and every byte of y written once
// (2 * rows * D * sizeof(T) + D * sizeof(W) algorithmic bytes).  The row is
// held in registers between the sum-of-squares pass and the scaling pass, so
// x is never re-read.  Loads and stores are 16-byte vectors with the
// streaming cache hint (x and y are touched exactly once; w stays in L1/L2).
#include "common.cuh"

namespace b200 {
namespace {

// Loads VN consecutive weights and widens them to fp32 (VN * sizeof(W) is a
// multiple of 16 bytes for every (T, W) pair the host dispatches here).
template <typename W, int VN>
__device__ __forceinline__ void load_weights(const W* p, float* out) {
  constexpr int per16 = 16 / sizeof(W);
#pragma unroll
  for (int c = 0; c < VN / per16; ++c) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(p) + c);
    const W* e = reinterpret_cast<const W*>(&raw);
#pragma unroll
    for (int i = 0; i < per16; ++i) out[c * per16 + i] = to_f32(e[i]);
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < nwarps) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// Register-resident path: each thread owns NV 16-byte vectors of the row.
template <typename T, typename W, int NV>
__global__ void __launch_bounds__(1024) rmsnorm_row_kernel(const T* __restrict__ x,
                                                           const W* __restrict__ w,
                                                           T* __restrict__ y, int D,
                                                           float eps) {
  constexpr int VN = Vec<T>::N;
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * D;
  T* yr = y + row * D;
  const int nvec = D / VN;

  uint4 raw[NV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      raw[i] = ldg_stream16(xr + (int64_t)v * VN);
      float f[VN];
      unpack16<T>(raw[i], f);
#pragma unroll
      for (int j = 0; j < VN; ++j) ss = fmaf(f[j], f[j], ss);
    }
  }
  ss = block_sum(ss, red);
  // mean then 1/sqrt, both IEEE-rounded, as torch.rsqrt(x.pow(2).mean() + eps).
  const float rstd = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));

#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      float f[VN], wf[VN], o[VN];
      unpack16<T>(raw[i], f);
      load_weights<W, VN>(w + (int64_t)v * VN, wf);
#pragma unroll
      for (int j = 0; j < VN; ++j) o[j] = __fmul_rn(__fmul_rn(f[j], rstd), wf[j]);
      stg_stream16(yr + (int64_t)v * VN, pack16<T>(o));
    }
  }
}

// General path for any D and any alignment: two passes over the row, the
// second one served mostly from L1/L2.
template <typename T, typename W>
__global__ void __launch_bounds__(1024) rmsnorm_loop_kernel(const T* __restrict__ x,
                                                            const W* __restrict__ w,
                                                            T* __restrict__ y, int64_t D,
                                                            float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * D;
  T* yr = y + row * D;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    const float f = to_f32(xr[i]);
    ss = fmaf(f, f, ss);
  }
  ss = block_sum(ss, red);
  const float rstd = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    yr[i] = from_f32<T>(__fmul_rn(__fmul_rn(to_f32(xr[i]), rstd), to_f32(w[i])));
  }
}

template <typename T, typename W>
int launch_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t D, float eps,
                   const b200_launch_cfg* cfg, cudaStream_t stream) {
  constexpr int VN = Vec<T>::N;
  const T* xp = static_cast<const T*>(x);
  const W* wp = static_cast<const W*>(w);
  T* yp = static_cast<T*>(y);
  const bool vec_ok = (D % VN == 0) && aligned16(x) && aligned16(y) && aligned16(w) &&
                      ((D * (int64_t)sizeof(T)) % 16 == 0) && D <= (1 << 30) &&
                      ((VN * sizeof(W)) % 16 == 0);
  int threads = (cfg && cfg->threads > 0) ? cfg->threads : 0;
  if (threads != 0 && (threads < 32 || threads > 1024 || threads % 32 != 0)) return B200_ERR_BAD_ARG;
  if (vec_ok) {
    const int64_t nvec = D / VN;
    if (threads == 0) {
      threads = nvec >= 256 * 2 ? 256 : (int)(((nvec + 31) / 32) * 32);
      if (threads < 32) threads = 32;
      while ((nvec + threads - 1) / threads > 8 && threads < 1024) threads *= 2;
    }
    const int64_t nv = (nvec + threads - 1) / threads;
    if (nv <= 8) {
      dim3 grid((unsigned)rows);
      if (nv <= 1)
        rmsnorm_row_kernel<T, W, 1><<<grid, threads, 0, stream>>>(xp, wp, yp, (int)D, eps);
      else if (nv <= 2)
        rmsnorm_row_kernel<T, W, 2><<<grid, threads, 0, stream>>>(xp, wp, yp, (int)D, eps);
      else if (nv <= 4)
        rmsnorm_row_kernel<T, W, 4><<<grid, threads, 0, stream>>>(xp, wp, yp, (int)D, eps);
      else
        rmsnorm_row_kernel<T, W, 8><<<grid, threads, 0, stream>>>(xp, wp, yp, (int)D, eps);
      return launch_status(cudaGetLastError());
    }
  }
  if (threads == 0) threads = D >= 1024 ? 512 : (int)(((D + 31) / 32) * 32);
  if (threads < 32) threads = 32;
  rmsnorm_loop_kernel<T, W><<<(unsigned)rows, threads, 0, stream>>>(xp, wp, yp, D, eps);
  return launch_status(cudaGetLastError());
}

}  // namespace
}  // namespace b200

extern "C" int b200_rmsnorm(const void* x, const void* weight, void* y, int64_t rows,
                            int64_t D, float eps, int32_t dtype, int32_t weight_dtype,
                            const b200_launch_cfg* cfg, void* stream) {
  using namespace b200;
  if (int e = injected_error("rmsnorm")) return e;
  if (rows < 0 || D <= 0) return B200_ERR_BAD_ARG;
  if (rows == 0) return B200_OK;
  if (!x || !weight || !y) return B200_ERR_BAD_ARG;
  if (rows > 0x7fffffffLL) return B200_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (weight_dtype == dtype) {
    return B200_DISPATCH_FLOAT(dtype, [&] {
      return launch_rmsnorm<scalar_t, scalar_t>(x, weight, y, rows, D, eps, cfg, s);
    });
  }
  if (weight_dtype == B200_F32) {
    return B200_DISPATCH_FLOAT(dtype, [&] {
      return launch_rmsnorm<scalar_t, float>(x, weight, y, rows, D, eps, cfg, s);
    });
  }
  return B200_ERR_UNSUPPORTED;
}
