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
#include "quant.cuh"
#include "sm100.cuh"

namespace b200 {
namespace {

// 16-bit rows of at most 4096 elements (a multiple of 8), one warp per row:
// the row's 16-byte vectors stay in registers (lane l holds vectors l,
// l + 32, ...) between the packed absolute maximum and the codes
// (quant_vec8, bit-identical to quant_code_fast).
template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_warp_kernel(const T* __restrict__ x, int8_t* __restrict__ q,
                                                                 float* __restrict__ scale, int64_t rows,
                                                                 int64_t cols) {
  constexpr int NV = 16;  // vectors per lane: 16 x 32 x 8 = 4096 elements
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;  // warp-uniform
  const int nvec = (int)(cols / 8);
  const uint4* xr = reinterpret_cast<const uint4*>(x + r * cols);
  uint4 u[NV];
  uint32_t m0 = 0u, m1 = 0u;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = lane + 32 * i;
    u[i] = v < nvec ? ldg_stream16(xr + v) : make_uint4(0u, 0u, 0u, 0u);
    m0 = absmax2<T>(m0, absmax2<T>(u[i].x, u[i].y));
    m1 = absmax2<T>(m1, absmax2<T>(u[i].z, u[i].w));
  }
  float a = fmaxf(absmax_of_pair<T>(m0), absmax_of_pair<T>(m1));
  asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(a) : "f"(a));
  const float s = finish_scale<T>(a);
  const float rs = __frcp_rn(s);
  if (lane == 0) scale[r] = s;
  int8_t* qr = q + r * cols;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) *reinterpret_cast<uint2*>(qr + (int64_t)v * 8) = quant_vec8<T>(u[i], s, rs);
  }
}

// Per-column quantisation with the transposed output q [cols, rows] (the
// INT8 GEMM's weight operand): a cluster of kColSplit CTAs covers a strip of
// 64 columns, each CTA a contiguous range of rows_per rows.  Pass 1: the
// column maxima of the CTA's rows (16-byte loads, 8 lanes a row, packed
// absolute maxima), combined over the cluster through distributed shared
// memory.  Pass 2 (the CTA's rows again, mostly from L2): 128-row tiles
// staged in shared memory, so that a thread quantises runs of 16 rows of one
// column with quant_vec8 and writes each as one 16-byte run of q.  Needs
// cols % 64 == 0, rows % 16 == 0 and 16-byte aligned x and q.
constexpr int kColSplit = 4;

template <typename T>
__global__ void __cluster_dims__(1, kColSplit, 1) __launch_bounds__(256)
    quantize_cols_strip_kernel(const T* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scale,
                               int64_t rows, int64_t cols, int64_t rows_per) {
  __shared__ __align__(16) uint4 tile[128 * 8];  // 128 rows x 64 columns of T
  __shared__ uint32_t red[8][32];               // per warp: packed maxima of the strip's 64 columns
  __shared__ uint32_t part[32];                 // this CTA's maxima, read by the whole cluster
  __shared__ float s_s[64], s_r[64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t c0 = (int64_t)blockIdx.x * 64;
  const int64_t rb = (int64_t)blockIdx.y * rows_per;
  const int64_t re = rb + rows_per < rows ? rb + rows_per : rows;
  const int cg = lane & 7, rl = lane >> 3;
  // ---- pass 1: word j of a lane's maxima holds columns 2j, 2j + 1 of its 8-column group
  // eight rows of loads in flight per thread
  uint32_t m[4] = {0u, 0u, 0u, 0u};
  for (int64_t r = rb + warp * 4 + rl; r < re; r += 32 * 8) {
    uint4 u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      u[k] = r + 32 * k < re ? __ldg(reinterpret_cast<const uint4*>(x + (r + 32 * k) * cols + c0) + cg)
                             : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      m[0] = absmax2<T>(m[0], u[k].x);
      m[1] = absmax2<T>(m[1], u[k].y);
      m[2] = absmax2<T>(m[2], u[k].z);
      m[3] = absmax2<T>(m[3], u[k].w);
    }
  }
#pragma unroll
  for (int o = 8; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = absmax2<T>(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));
  if (rl == 0)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][cg * 4 + i] = m[i];
  __syncthreads();
  if (tid < 32) {
    uint32_t w = red[0][tid];
#pragma unroll
    for (int k = 1; k < 8; ++k) w = absmax2<T>(w, red[k][tid]);
    part[tid] = w;
  }
  sm100::cluster_sync();  // every CTA's part is written
  if (tid < 32) {
    uint32_t w = 0u;
#pragma unroll
    for (int k = 0; k < kColSplit; ++k) {
      uint32_t pw;
      asm volatile("ld.shared::cluster.u32 %0, [%1];"
                   : "=r"(pw)
                   : "r"(sm100::mapa_shared(sm100::smem_u32(&part[tid]), (uint32_t)k))
                   : "memory");
      w = absmax2<T>(w, pw);
    }
    const uint32_t mm = w & 0x7FFF7FFFu;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t bits = h ? (mm >> 16) : (mm & 0xFFFFu);
      float a;
      if constexpr (std::is_same<T, __nv_bfloat16>::value)
        a = __uint_as_float(bits << 16);
      else
        a = __half2float(__ushort_as_half((unsigned short)bits));
      const float sv = finish_scale<T>(a);
      s_s[2 * tid + h] = sv;
      s_r[2 * tid + h] = __frcp_rn(sv);
      if (blockIdx.y == 0) scale[c0 + 2 * tid + h] = sv;
    }
  }
  sm100::cluster_sync();  // no CTA leaves while a peer may still read its part; s_s / s_r visible
  // ---- pass 2: 128-row tiles; the next tile's loads are in flight (in
  // registers) while the current one is quantised from shared memory
  const int c = tid & 63, rg = tid >> 6;  // column, 32-row group of the tile
  const float sc = s_s[c], rc = s_r[c];
  const uint16_t* t16 = reinterpret_cast<const uint16_t*>(tile);
  auto load_tile = [&](int64_t r0, uint4 (&pre)[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = tid + 256 * k;  // row e / 8, 8-column group e % 8
      const int64_t r = r0 + (e >> 3);
      pre[k] = r < re ? __ldg(reinterpret_cast<const uint4*>(x + r * cols + c0) + (e & 7))
                      : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  uint4 pre[4];
  if (rb < re) load_tile(rb, pre);
  for (int64_t r0 = rb; r0 < re; r0 += 128) {
#pragma unroll
    for (int k = 0; k < 4; ++k) tile[tid + 256 * k] = pre[k];
    __syncthreads();
    if (r0 + 128 < re) load_tile(r0 + 128, pre);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int tr = rg * 32 + h * 16;  // first tile row of this 16-row run
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = (uint32_t)t16[(tr + 2 * i) * 64 + c] | ((uint32_t)t16[(tr + 2 * i + 1) * 64 + c] << 16);
      const uint2 qa = quant_vec8<T>(make_uint4(w[0], w[1], w[2], w[3]), sc, rc);
      const uint2 qb = quant_vec8<T>(make_uint4(w[4], w[5], w[6], w[7]), sc, rc);
      const int64_t rr0 = r0 + tr;
      if (rr0 < re) *reinterpret_cast<uint4*>(q + (c0 + c) * rows + rr0) = make_uint4(qa.x, qa.y, qb.x, qb.y);
    }
    __syncthreads();
  }
}

// General path (any width and dtype): one CTA per row.
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

// General path: one CTA per 32 columns of x [rows, cols]; writes q transposed [cols, rows].
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

// Per-column quantisation for at most 4096 rows, x read from DRAM once: a
// cluster of kColSplitR CTAs covers a strip of 64 columns, each CTA up to
// 512 rows, which it keeps in shared memory (64 KB) between the packed
// column maxima (combined over the cluster through distributed shared
// memory, as in quantize_cols_strip_kernel) and the codes (a thread
// quantises 32 rows of one column per step and writes them as two 16-byte
// runs, a whole 32-byte sector of q).  Needs cols % 64 == 0, rows % 16 == 0 and 16-byte aligned x and q.
constexpr int kColSplitR = 8;
constexpr int kResidentRows = 512;

template <typename T>
__global__ void __cluster_dims__(1, kColSplitR, 1) __launch_bounds__(256)
    quantize_cols_resident_kernel(const T* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scale,
                                  int64_t rows, int64_t cols, int rows_per) {
  extern __shared__ __align__(16) uint4 rtile[];  // rows_per rows x 64 columns of T
  __shared__ uint32_t red[8][32];
  __shared__ uint32_t part[32];
  __shared__ float s_s[64], s_r[64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t c0 = (int64_t)blockIdx.x * 64;
  const int64_t rb = (int64_t)blockIdx.y * rows_per;
  const int n = rb < rows ? (int)((rows - rb) < rows_per ? (rows - rb) : rows_per) : 0;  // rows of this CTA
  const int cg = tid & 7;  // the thread's 8-column group: element e = tid + 256 k has e % 8 == cg
  // ---- pass 1: the CTA's rows into shared memory, eight 16-byte loads in flight per thread
  uint32_t m[4] = {0u, 0u, 0u, 0u};
  for (int e0 = 0; e0 < n * 8; e0 += 256 * 8) {
    uint4 u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int e = e0 + tid + 256 * k;
      u[k] = e < n * 8 ? __ldg(reinterpret_cast<const uint4*>(x + (rb + (e >> 3)) * cols + c0) + cg)
                       : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int e = e0 + tid + 256 * k;
      if (e < n * 8) rtile[e] = u[k];
      m[0] = absmax2<T>(m[0], u[k].x);
      m[1] = absmax2<T>(m[1], u[k].y);
      m[2] = absmax2<T>(m[2], u[k].z);
      m[3] = absmax2<T>(m[3], u[k].w);
    }
  }
#pragma unroll
  for (int o = 8; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = absmax2<T>(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));
  if (lane < 8)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][cg * 4 + i] = m[i];
  __syncthreads();
  if (tid < 32) {
    uint32_t w = red[0][tid];
#pragma unroll
    for (int k = 1; k < 8; ++k) w = absmax2<T>(w, red[k][tid]);
    part[tid] = w;
  }
  sm100::cluster_sync();  // every CTA's part is written
  if (tid < 32) {
    uint32_t w = 0u;
#pragma unroll
    for (int k = 0; k < kColSplitR; ++k) {
      uint32_t pw;
      asm volatile("ld.shared::cluster.u32 %0, [%1];"
                   : "=r"(pw)
                   : "r"(sm100::mapa_shared(sm100::smem_u32(&part[tid]), (uint32_t)k))
                   : "memory");
      w = absmax2<T>(w, pw);
    }
    const uint32_t mm = w & 0x7FFF7FFFu;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t bits = h ? (mm >> 16) : (mm & 0xFFFFu);
      float a;
      if constexpr (std::is_same<T, __nv_bfloat16>::value)
        a = __uint_as_float(bits << 16);
      else
        a = __half2float(__ushort_as_half((unsigned short)bits));
      const float sv = finish_scale<T>(a);
      s_s[2 * tid + h] = sv;
      s_r[2 * tid + h] = __frcp_rn(sv);
      if (blockIdx.y == 0) scale[c0 + 2 * tid + h] = sv;
    }
  }
  sm100::cluster_sync();  // no CTA leaves while a peer may still read its part; tile, s_s, s_r visible
  // ---- pass 2: the codes from shared memory, 32 rows of one column per
  // thread and step (whole 32-byte sectors of q)
  const int c = tid & 63, rg = tid >> 6;
  const float sc = s_s[c], rc = s_r[c];
  const uint16_t* t16 = reinterpret_cast<const uint16_t*>(rtile);
  for (int t0 = rg * 32; t0 < n; t0 += 128) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int tr = t0 + 16 * h;
      if (tr >= n) break;
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = (uint32_t)t16[(tr + 2 * i) * 64 + c] | ((uint32_t)t16[(tr + 2 * i + 1) * 64 + c] << 16);
      const uint2 qa = quant_vec8<T>(make_uint4(w[0], w[1], w[2], w[3]), sc, rc);
      const uint2 qb = quant_vec8<T>(make_uint4(w[4], w[5], w[6], w[7]), sc, rc);
      *reinterpret_cast<uint4*>(q + (c0 + c) * rows + rb + tr) = make_uint4(qa.x, qa.y, qb.x, qb.y);
    }
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
    constexpr bool k16 = !std::is_same<scalar_t, float>::value;
    if (k16 && !by_column && cols % 8 == 0 && cols <= 4096 && aligned16(x) &&
        reinterpret_cast<uintptr_t>(q) % 8 == 0 && rows <= 8LL * 0x7fffffffLL) {
      // packed warp rows (16-byte vectors held in registers)
      quantize_rows_warp_kernel<scalar_t><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(
          static_cast<const scalar_t*>(x), q, scale, rows, cols);
      return launch_status(cudaGetLastError());
    }
    if (k16 && by_column && cols % 64 == 0 && rows % 16 == 0 && aligned16(x) && aligned16(q) &&
        cols / 64 <= 0x7fffffffLL && rows <= (int64_t)kColSplitR * kResidentRows) {
      // up to 4096 rows: column strips held in shared memory, x read once
      const int rows_per = (int)(((rows + kColSplitR - 1) / kColSplitR + 15) / 16 * 16);
      const int dyn = rows_per * 128;
      auto kern = quantize_cols_resident_kernel<scalar_t>;
      if (dyn > 48 * 1024) {
        if (cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
            e != cudaSuccess)
          return launch_status(e);
      }
      kern<<<dim3((unsigned)(cols / 64), kColSplitR), 256, dyn, s>>>(static_cast<const scalar_t*>(x), q, scale,
                                                                     rows, cols, rows_per);
      return launch_status(cudaGetLastError());
    }
    if (k16 && by_column && cols % 64 == 0 && rows % 16 == 0 && aligned16(x) && aligned16(q) &&
        cols / 64 <= 0x7fffffffLL) {
      // column strips of 64, each over a cluster of kColSplit CTAs
      const int64_t rows_per = ((rows + kColSplit - 1) / kColSplit + 127) / 128 * 128;
      quantize_cols_strip_kernel<scalar_t><<<dim3((unsigned)(cols / 64), kColSplit), 256, 0, s>>>(
          static_cast<const scalar_t*>(x), q, scale, rows, cols, rows_per);
      return launch_status(cudaGetLastError());
    }
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
