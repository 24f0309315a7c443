// Symmetric per-row / per-column INT8 quantisation.
//
// Reference: triton_agent/ops/quant_matmul/reference.py:16-24
//   scale = max|x| / 127        (a dtype tensor: the quotient is rounded to x's dtype)
//   scale[scale == 0] = 1e-6
//   q = clamp(round(x / scale), -127, 127).to(int8)
// Eager PyTorch evaluates x / scale in fp32 and rounds the quotient to x's
// dtype before round() (half-to-even); the kernels do the same (quant_code_fast,
// common.cuh), so the int8 codes are bit-identical.  The scale is returned as fp32 (exact widening of
// the dtype-rounded value).
#include "common.cuh"

namespace b200 {
namespace {

// One CTA per row.
template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ x,
                                                            int8_t* __restrict__ q,
                                                            float* __restrict__ scale,
                                                            int64_t cols) {
  __shared__ float red[32];
  const T* xr = x + (int64_t)blockIdx.x * cols;
  float amax = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) amax = fmaxf(amax, fabsf(to_f32(xr[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float s = finish_scale<T>(red[0]);
  const float rs = __frcp_rn(s);
  if (threadIdx.x == 0) scale[blockIdx.x] = s;
  int8_t* qr = q + (int64_t)blockIdx.x * cols;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) qr[i] = (int8_t)quant_code_fast<T>(to_f32(xr[i]), s, rs);
}

// One CTA per 32 columns of x [rows, cols]; writes q transposed [cols, rows].
template <typename T>
__global__ void __launch_bounds__(256) quantize_cols_kernel(const T* __restrict__ x,
                                                            int8_t* __restrict__ q,
                                                            float* __restrict__ scale,
                                                            int64_t rows, int64_t cols) {
  __shared__ float red[8][33];
  __shared__ float s_scale[32];
  __shared__ float s_rcp[32];
  __shared__ int8_t tile[32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  float amax = 0.f;
  if (c < cols)
    for (int64_t r = warp; r < rows; r += 8) amax = fmaxf(amax, fabsf(to_f32(x[r * cols + c])));
  red[warp][lane] = amax;
  __syncthreads();
  if (warp == 0) {
    float v = 0.f;
    for (int w = 0; w < 8; ++w) v = fmaxf(v, red[w][lane]);
    const float s = finish_scale<T>(v);
    s_scale[lane] = s;
    s_rcp[lane] = __frcp_rn(s);
    if (c < cols) scale[c] = s;
  }
  __syncthreads();
  for (int64_t r0 = 0; r0 < rows; r0 += 32) {
    // load a 32x32 tile (rows r0.., columns of this CTA), quantise
    for (int rr = warp; rr < 32; rr += 8) {
      const int64_t r = r0 + rr;
      tile[rr][lane] =
          (r < rows && c < cols) ? (int8_t)quant_code_fast<T>(to_f32(x[r * cols + c]), s_scale[lane], s_rcp[lane]) : 0;
    }
    __syncthreads();
    // write transposed: q[col][r0 + lane]
    for (int cc = warp; cc < 32; cc += 8) {
      const int64_t col = (int64_t)blockIdx.x * 32 + cc;
      const int64_t r = r0 + lane;
      if (col < cols && r < rows) q[col * rows + r] = tile[lane][cc];
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_quantize_int8(const void* x, int8_t* q, float* scale, int64_t rows,
                                  int64_t cols, int32_t dtype, int32_t by_column,
                                  const b200_launch_cfg* cfg, void* stream) {
  (void)cfg;
  if (int e = injected_error("quantize_int8")) return e;
  if (rows < 0 || cols < 0) return B200_ERR_BAD_ARG;
  if (rows == 0 || cols == 0) return B200_OK;
  if (!x || !q || !scale) return B200_ERR_BAD_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return B200_DISPATCH_FLOAT(dtype, [&] {
    if (!by_column) {
      if (rows > 0x7fffffffLL) return (int)B200_ERR_UNSUPPORTED;
      quantize_rows_kernel<scalar_t><<<(unsigned)rows, 256, 0, s>>>(
          static_cast<const scalar_t*>(x), q, scale, cols);
    } else {
      const int64_t grid = (cols + 31) / 32;
      if (grid > 0x7fffffffLL) return (int)B200_ERR_UNSUPPORTED;
      quantize_cols_kernel<scalar_t><<<(unsigned)grid, 256, 0, s>>>(
          static_cast<const scalar_t*>(x), q, scale, rows, cols);
    }
    return launch_status(cudaGetLastError());
  });
}
