// RMSNorm, y = x * rsqrt(mean(x^2) + eps) * w, and RMSNorm fused with the
// row INT8 quantiser of the next GEMM's activations.
//
// Reference: triton_agent/ops/rmsnorm/reference.py:17-18.
//
// HBM-bound: every byte of x is read once and every byte of y written once
// (2 * rows * D * sizeof(T) + D * sizeof(W) algorithmic bytes).  The row is
// held in registers between the sum-of-squares pass and the scaling pass, so
// x is never re-read.  Loads and stores are 16-byte vectors with the
// streaming cache hint (x and y are touched exactly once; w stays in L1/L2).
#include <type_traits>

#include "common.cuh"
#include "quant.cuh"
#include "sm100.cuh"

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
  // sum of squares in two fp32 lanes (even / odd elements, one fp32x2 FMA
  // per pair), the same order as rmsnorm_quant_row_kernel's
  float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      raw[i] = ldg_stream16(xr + (int64_t)v * VN);
      float f[VN];
      unpack16<T>(raw[i], f);
#pragma unroll
      for (int j = 0; j < VN; j += 2) sm100::ffma2(ss0, ss1, f[j], f[j + 1], f[j], f[j + 1], ss0, ss1);
    }
  }
  const float ss = block_sum(ss0 + ss1, red);
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
      for (int j = 0; j < VN; j += 2) {
        sm100::fmul2_bcast(o[j], o[j + 1], f[j], f[j + 1], rstd);
        sm100::fmul2(o[j], o[j + 1], o[j], o[j + 1], wf[j], wf[j + 1]);
      }
      stg_stream16(yr + (int64_t)v * VN, pack16<T>(o));
    }
  }
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < nwarps) ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

// rmsnorm fused with the per-row symmetric INT8 quantiser of the next GEMM's
// activations: y = rmsnorm(x) rounded to T exactly as rmsnorm_row_kernel
// writes it, then scale = max|y| / 127 and q = clamp(rint(y / scale)) with
// the quantiser's dtype rounding (bit-identical to quantising the rmsnorm
// output).  One pass over x: x is read once, q (1 B per element) and the
// scale are written, y only when asked for.
// Block reductions of R rows at once (one barrier for all of them), each row
// in block_sum's / block_max's order.
template <int R>
__device__ __forceinline__ void block_sum_rows(float (&v)[R], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = warp_sum(v[r]);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) red[r * 32 + warp] = v[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = warp_sum((lane < nwarps) ? red[r * 32 + lane] : 0.f);
}

template <int R>
__device__ __forceinline__ void block_max_rows(float (&v)[R], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = warp_max(v[r]);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) red[r * 32 + warp] = v[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = warp_max((lane < nwarps) ? red[r * 32 + lane] : 0.f);
}

template <typename T, typename W, int NV, int R>
__global__ void __launch_bounds__(R == 1 ? 1024 : 256) rmsnorm_quant_row_kernel(const T* __restrict__ x, const W* __restrict__ w,
                                                                 int8_t* __restrict__ q, float* __restrict__ scale,
                                                                 T* __restrict__ y, int64_t rows, int D, float eps) {
  constexpr int VN = Vec<T>::N;
  __shared__ float red[R * 32];
  __shared__ float red2[R * 32];
  const int64_t row0 = (int64_t)blockIdx.x * R;
  const int nvec = D / VN;
  // The rows stay in registers: as fp32 when they fit in 32 floats per
  // thread (x, then y rounded to T), else packed as T and widened per pass.
  constexpr bool kF32 = NV * VN * R <= 32;
  float f[kF32 ? R : 1][kF32 ? NV : 1][VN];
  uint4 raw[kF32 ? 1 : R][kF32 ? 1 : NV];
  auto row_f = [&](int r, int i) -> float* { return f[kF32 ? r : 0][kF32 ? i : 0]; };
  auto live = [&](int r, int v) { return v < nvec && row0 + r < rows; };
  float ss[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = threadIdx.x + i * blockDim.x;
      if (live(r, v)) {
        const uint4 u = ldg_stream16(x + (row0 + r) * D + (int64_t)v * VN);
        if constexpr (!kF32) raw[r][i] = u;
        float* fi = row_f(r, i);
        unpack16<T>(u, fi);
#pragma unroll
        for (int j = 0; j < VN; j += 2) sm100::ffma2(ss0, ss1, fi[j], fi[j + 1], fi[j], fi[j + 1], ss0, ss1);
      }
    }
    ss[r] = ss0 + ss1;
  }
  block_sum_rows<R>(ss, red);
  float amax[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float rstd = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss[r], (float)D), eps));
    amax[r] = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = threadIdx.x + i * blockDim.x;
      if (live(r, v)) {
        float* fi = row_f(r, i);
        if constexpr (!kF32) unpack16<T>(raw[r][i], fi);
        float wf[VN];
        load_weights<W, VN>(w + (int64_t)v * VN, wf);
#pragma unroll
        for (int j = 0; j < VN; j += 2) {
          sm100::fmul2_bcast(fi[j], fi[j + 1], fi[j], fi[j + 1], rstd);
          sm100::fmul2(fi[j], fi[j + 1], fi[j], fi[j + 1], wf[j], wf[j + 1]);
        }
        const uint4 u = pack16<T>(fi);  // y rounded to T, kept for the quantiser
        if constexpr (!kF32) raw[r][i] = u;
        unpack16<T>(u, fi);
#pragma unroll
        for (int j = 0; j < VN; j += 2) amax[r] = sm100::fmax3(amax[r], fabsf(fi[j]), fabsf(fi[j + 1]));
        if (y != nullptr) stg_stream16(y + (row0 + r) * D + (int64_t)v * VN, u);
      }
    }
  }
  block_max_rows<R>(amax, red2);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (row0 + r >= rows) break;
    const float s = finish_scale<T>(amax[r]);
    const float rs = __frcp_rn(s);
    if (threadIdx.x == 0) scale[row0 + r] = s;
    int8_t* qr = q + (row0 + r) * D;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = threadIdx.x + i * blockDim.x;
      if (v < nvec) {
        float* fi = row_f(r, i);
        if constexpr (!kF32) unpack16<T>(raw[r][i], fi);
        // quant_code_fast on pairs: q0 = RN(y r), e = y - q0 s, RN(q0 + e r) =
        // RN(y / s); round the pair to T's precision with one packed
        // conversion, add 1.5 * 2^23 so the low 16 bits of the bits are the
        // integer rint as int16, clamp both codes to [-127, 127] with packed
        // 16-bit integer min/max, and keep the low bytes
        uint32_t h[VN / 2];
#pragma unroll
        for (int j = 0; j < VN; j += 2) {
          float q0, q1, e0, e1, v0, v1;
          sm100::fmul2_bcast(q0, q1, fi[j], fi[j + 1], rs);
          sm100::ffma2(e0, e1, q0, q1, -s, -s, fi[j], fi[j + 1]);
          sm100::ffma2(v0, v1, e0, e1, rs, rs, q0, q1);
          round_pair_to<T>(v0, v1);
          sm100::ffma2_bcast(v0, v1, v0, v1, 1.0f, 12582912.0f);
          uint32_t p = __byte_perm(__float_as_uint(v0), __float_as_uint(v1), 0x5410);
          asm("max.s16x2 %0, %1, %2;" : "=r"(p) : "r"(p), "r"(0xFF81FF81u));  // -127, -127
          asm("min.s16x2 %0, %1, %2;" : "=r"(p) : "r"(p), "r"(0x007F007Fu));  // 127, 127
          h[j / 2] = p;
        }
        if constexpr (VN == 8) {
          uint2 pk;
          pk.x = __byte_perm(h[0], h[1], 0x6420);
          pk.y = __byte_perm(h[2], h[3], 0x6420);
          *reinterpret_cast<uint2*>(qr + (int64_t)v * VN) = pk;
        } else {
          *reinterpret_cast<uint32_t*>(qr + (int64_t)v * VN) = __byte_perm(h[0], h[1], 0x6420);
        }
      }
    }
  }
}

// Persistent variant for 16-bit rows of NV = 2 or 4 vectors per thread: a grid of the resident CTA count loops
// over rows, so the weights are widened to fp32 once per CTA and kept in
// registers, and the next row's x is loaded while the current row is reduced
// and quantised.  Per element it does the same arithmetic as
// rmsnorm_quant_row_kernel with less around it:
//  - max|y| is taken on the fp32 products before their rounding to T (the
//    rounding is monotonic, so the rounded maximum is the maximum of the
//    rounded values) instead of re-widening the rounded row;
//  - the codes come from quant_vec8 (bf16 without Markstein's correction).
// The sum of squares is accumulated in the same order as
// rmsnorm_quant_row_kernel's with one row per CTA of the same size.
template <typename T, typename W, bool FULL, int NV, int MAXT>
__global__ void __launch_bounds__(MAXT, MAXT <= 128 ? 5 : 2) rmsnorm_quant_persistent_kernel(
    const T* __restrict__ x, const W* __restrict__ w, int8_t* __restrict__ q, float* __restrict__ scale,
    T* __restrict__ y, int64_t rows, int D, float eps) {
  constexpr int VN = Vec<T>::N;  // 8
  __shared__ float red[32], red2[32];
  const int nvec = D / VN;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = (nt + 31) >> 5;
  auto live = [&](int i) { return FULL || tid + i * nt < nvec; };
  float wf[NV][VN];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (live(i)) {
      load_weights<W, VN>(w + (int64_t)(tid + i * nt) * VN, wf[i]);
    } else {
#pragma unroll
      for (int j = 0; j < VN; ++j) wf[i][j] = 0.f;
    }
  }
  uint4 cur[NV];
  int64_t r = blockIdx.x;
  if (r < rows) {
#pragma unroll
    for (int i = 0; i < NV; ++i)
      if (live(i)) cur[i] = ldg_stream16(x + r * D + (int64_t)(tid + i * nt) * VN);
  }
  for (; r < rows; r += gridDim.x) {
    // the next row's loads are in flight during this row's two reductions
    uint4 nxt[NV];
    const int64_t rn = r + gridDim.x;
    if (rn < rows) {
#pragma unroll
      for (int i = 0; i < NV; ++i)
        if (live(i)) nxt[i] = ldg_stream16(x + rn * D + (int64_t)(tid + i * nt) * VN);
    }
    float f[NV][VN];
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (live(i)) {
        unpack16<T>(cur[i], f[i]);
#pragma unroll
        for (int j = 0; j < VN; j += 2)
          sm100::ffma2(ss0, ss1, f[i][j], f[i][j + 1], f[i][j], f[i][j + 1], ss0, ss1);
      }
    }
    // block reductions: a shuffle sum (redux.sync for the max) per warp, then
    // every thread combines the per-warp values from shared memory in warp
    // order (no second shuffle chain)
    float ss = warp_sum(ss0 + ss1);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    ss = red[0];
    for (int k = 1; k < nwarps; ++k) ss += red[k];
    const float rstd = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (live(i)) {
#pragma unroll
        for (int j = 0; j < VN; j += 2) {
          sm100::fmul2_bcast(f[i][j], f[i][j + 1], f[i][j], f[i][j + 1], rstd);
          sm100::fmul2(f[i][j], f[i][j + 1], f[i][j], f[i][j + 1], wf[i][j], wf[i][j + 1]);
          amax = sm100::fmax3(amax, fabsf(f[i][j]), fabsf(f[i][j + 1]));
        }
        cur[i] = pack16<T>(f[i]);  // y rounded to T
        if (y != nullptr) stg_stream16(y + r * D + (int64_t)(tid + i * nt) * VN, cur[i]);
      }
    }
    asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(amax) : "f"(amax));
    if (lane == 0) red2[warp] = amax;
    __syncthreads();
    amax = red2[0];
    for (int k = 1; k < nwarps; ++k) amax = fmaxf(amax, red2[k]);
    const float s = finish_scale<T>(round_to<T>(amax));
    const float rs = __frcp_rn(s);
    if (tid == 0) scale[r] = s;
    int8_t* qr = q + r * D;
#pragma unroll
    for (int i = 0; i < NV; ++i)
      if (live(i)) *reinterpret_cast<uint2*>(qr + (int64_t)(tid + i * nt) * VN) = quant_vec8<T>(cur[i], s, rs);
#pragma unroll
    for (int i = 0; i < NV; ++i) cur[i] = nxt[i];
  }
}

// SPLIT warps per row (1 or 2), for 16-bit rows of D = 256 NVW SPLIT: lane
// l of the group's warp h holds the row's 16-byte vectors h 32 NVW + l +
// 32 i (NVW of them; each warp load one contiguous 512-byte run), so the
// reductions are warp shuffles plus, for two warps, one exchange through
// shared memory under a 64-thread named barrier; no CTA-wide barrier
// separates a row's phases, and the groups of an SM run their rows
// independently, some loading while others compute.  One 512-thread CTA
// per SM (16 warps) widens the weights to fp32 once into shared memory
// (elements 0-3 and 4-7 of each vector in two arrays, so a warp's 16-byte
// reads are conflict-free); four 128-thread CTAs, each with its own copy,
// ran 5% slower.
// Rows are strided over the grid's groups; the host sizes the grid so that
// every group takes the same number of rows, give or take one.  Per
// element: the persistent kernel's arithmetic (max|y| before rounding,
// quant_vec8 codes) with the sum of squares in a different fp32 order.
template <typename T, typename W, int NVW, int SPLIT, bool PF>
__global__ void __launch_bounds__(512, 1) rmsnorm_quant_warp_kernel(
    const T* __restrict__ x, const W* __restrict__ w, int8_t* __restrict__ q, float* __restrict__ scale,
    T* __restrict__ y, int64_t rows, float eps) {
  static_assert(SPLIT == 1 || SPLIT == 2, "one or two warps per row");
  constexpr int VN = Vec<T>::N;  // 8
  constexpr int NVEC = 32 * NVW * SPLIT;
  constexpr int D = NVEC * VN;
  constexpr int kGroups = 16 / SPLIT;  // row groups of a 512-thread CTA
  __shared__ float4 wlo[NVEC], whi[NVEC];
  __shared__ float xch[2][kGroups][SPLIT];
  // PF: each warp's next row is copied into shared memory (one buffer of
  // its NVW x 32 vectors) while the current one is computed
  extern __shared__ uint4 xbuf[];
  uint4* mybuf = xbuf + (threadIdx.x >> 5) * NVW * 32;
  for (int v = threadIdx.x; v < NVEC; v += blockDim.x) {
    float wf[VN];
    load_weights<W, VN>(w + (int64_t)v * VN, wf);
    wlo[v] = make_float4(wf[0], wf[1], wf[2], wf[3]);
    whi[v] = make_float4(wf[4], wf[5], wf[6], wf[7]);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = warp / SPLIT, half = warp % SPLIT;
  const int vb = half * 32 * NVW + lane;  // this lane's first vector
  const int64_t ng = (int64_t)gridDim.x * kGroups;
  // both warps of a group take the same rows, so they meet at every barrier
  auto pair_sync = [&] {
    if constexpr (SPLIT == 2) {
      asm volatile("bar.sync %0, 64;" ::"r"(1 + grp) : "memory");  // barriers 1..8
    }
  };
  // dep: a value computed from everything this lane read from the buffer,
  // so the copies that refill it issue only after those reads returned
  auto prefetch = [&](int64_t rr, uint32_t dep) {
    const T* src = x + rr * D + (int64_t)vb * VN;
#pragma unroll
    for (int i = 0; i < NVW; ++i) {
      const uint32_t dst = sm100::smem_u32(mybuf + lane + 32 * i);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src + i * 32 * VN), "r"(dep)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if constexpr (PF) {
    const int64_t r0 = (int64_t)blockIdx.x * kGroups + grp;
    if (r0 < rows) prefetch(r0, 0u);
  }
  for (int64_t r = (int64_t)blockIdx.x * kGroups + grp; r < rows; r += ng) {
    uint4 u[NVW];
    if constexpr (PF) {
      // each lane reads back only the 16-byte slots it copied itself
      asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
      for (int i = 0; i < NVW; ++i) u[i] = mybuf[lane + 32 * i];
    } else {
      const T* xr = x + r * D + (int64_t)vb * VN;
#pragma unroll
      for (int i = 0; i < NVW; ++i) u[i] = ldg_stream16(xr + i * 32 * VN);
    }
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int i = 0; i < NVW; ++i) {
      float f[VN];
      unpack16<T>(u[i], f);
#pragma unroll
      for (int j = 0; j < VN; j += 2) sm100::ffma2(ss0, ss1, f[j], f[j + 1], f[j], f[j + 1], ss0, ss1);
    }
    float ss = warp_sum(ss0 + ss1);  // xor butterfly: the same bits in every lane
    if constexpr (PF) {
      // the next row's copies overlap the rest of this one; the buffer is
      // refilled only after every value read from it fed ss
      if (r + ng < rows) prefetch(r + ng, __float_as_uint(ss));
    }
    if constexpr (SPLIT == 2) {
      if (lane == 0) xch[0][grp][half] = ss;
      pair_sync();
      ss = xch[0][grp][0] + xch[0][grp][1];
    }
    // ss / D: D = 2^k divides exactly as a multiply by 2^-k
    constexpr bool kPow2 = (D & (D - 1)) == 0;
    const float ms = kPow2 ? ss * (1.0f / D) : __fdiv_rn(ss, (float)D);
    const float rstd = 1.0f / sqrtf(__fadd_rn(ms, eps));
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < NVW; ++i) {
      float f[VN];
      unpack16<T>(u[i], f);
      const float4 a = wlo[vb + 32 * i], b = whi[vb + 32 * i];
      const float wf[VN] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < VN; j += 2) {
        sm100::fmul2_bcast(f[j], f[j + 1], f[j], f[j + 1], rstd);
        sm100::fmul2(f[j], f[j + 1], f[j], f[j + 1], wf[j], wf[j + 1]);
        amax = sm100::fmax3(amax, fabsf(f[j]), fabsf(f[j + 1]));
      }
      u[i] = pack16<T>(f);  // y rounded to T
      if (y != nullptr) stg_stream16(y + r * D + (int64_t)(vb + 32 * i) * VN, u[i]);
    }
    asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(amax) : "f"(amax));
    if constexpr (SPLIT == 2) {
      // the sum slot of this row was read before either warp arrives here,
      // and the next row's is written after this barrier: two slots suffice
      if (lane == 0) xch[1][grp][half] = amax;
      pair_sync();
      amax = fmaxf(xch[1][grp][0], xch[1][grp][1]);
    }
    const float s = finish_scale<T>(round_to<T>(amax));
    const float rs = __frcp_rn(s);
    if (lane == 0 && half == 0) scale[r] = s;
    int8_t* qr = q + r * D + (int64_t)vb * VN;
#pragma unroll
    for (int i = 0; i < NVW; ++i) *reinterpret_cast<uint2*>(qr + i * 32 * VN) = quant_vec8<T>(u[i], s, rs);
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

namespace b200 {
namespace {
constexpr int kQuantRowsPerCta = 1;  // measured: 2 and 4 rows per CTA run 9% and 50% slower at 16384 x 4096
}  // namespace
}  // namespace b200

extern "C" int b200_rmsnorm_quant_int8(const void* x, const void* weight, int8_t* q, float* scale, void* y,
                                       int64_t rows, int64_t D, float eps, int32_t dtype, int32_t weight_dtype,
                                       const b200_launch_cfg* cfg, void* stream) {
  using namespace b200;
  if (int e = injected_error("rmsnorm_quant_int8")) return e;
  if (rows < 0 || D <= 0) return B200_ERR_BAD_ARG;
  if (rows == 0) return B200_OK;
  if (!x || !weight || !q || !scale) return B200_ERR_BAD_ARG;
  if (rows > 0x7fffffffLL || D > (1 << 30)) return B200_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run = [&](auto tag_t, auto tag_w) -> int {
    using T = decltype(tag_t);
    using W = decltype(tag_w);
    constexpr int VN = Vec<T>::N;
    // register-resident rows only: 16-byte vectors, 8-byte-aligned codes
    if (D % VN != 0 || !aligned16(x) || !aligned16(weight) || (y && !aligned16(y)) ||
        (reinterpret_cast<uintptr_t>(q) % 8) != 0 || ((VN * sizeof(W)) % 16) != 0)
      return B200_ERR_ALIGNMENT;
    const int64_t nvec = D / VN;
    int threads = (cfg && cfg->threads > 0) ? cfg->threads : 0;
    const int threads_given = threads;
    if (threads != 0 && (threads < 32 || threads > 1024 || threads % 32 != 0)) return B200_ERR_BAD_ARG;
    if (threads == 0) {
      // about four 16-byte vectors per thread (measured best for D = 4096)
      threads = (int)((((nvec + 3) / 4) + 31) / 32 * 32);
      threads = threads < 32 ? 32 : (threads > 1024 ? 1024 : threads);
    }
    const int64_t nv = (nvec + threads - 1) / threads;
    if (nv > 8) return B200_ERR_UNSUPPORTED;
    const T* xp = static_cast<const T*>(x);
    const W* wp = static_cast<const W*>(weight);
    T* yp = static_cast<T*>(y);
    // rows per CTA (rows_per_cta: 1, 2 or 4): more bytes in flight per CTA
    // and one barrier pair for all of them
    int R = (cfg && cfg->rows_per_cta > 0) ? cfg->rows_per_cta : kQuantRowsPerCta;
    if (R != 1 && R != 2 && R != 4) return B200_ERR_BAD_ARG;
    if (nv > 4 || threads > 256) R = 1;  // multi-row CTAs are compiled for <= 256 threads
    if constexpr (!std::is_same<T, float>::value) {
      // warp rows for D = 1024, 2048 (one warp a row) and 4096 (two), unless
      // a CTA size is given or flags bit 0 or 1 asks for the CTA kernels;
      // flags bit 2: no shared-memory prefetch of the next row
      const int fl = cfg ? cfg->flags : 0;
      if ((D == 1024 || D == 2048 || D == 4096) && threads_given == 0 && R == 1 && !(fl & 3)) {
        const bool pf = !(fl & 4);
        auto kern = D == 4096 ? (pf ? rmsnorm_quant_warp_kernel<T, W, 8, 2, true> : rmsnorm_quant_warp_kernel<T, W, 8, 2, false>)
                  : D == 2048 ? (pf ? rmsnorm_quant_warp_kernel<T, W, 8, 1, true> : rmsnorm_quant_warp_kernel<T, W, 8, 1, false>)
                              : (pf ? rmsnorm_quant_warp_kernel<T, W, 4, 1, true> : rmsnorm_quant_warp_kernel<T, W, 4, 1, false>);
        const int groups_per_cta = D == 4096 ? 8 : 16;
        // a row buffer per warp (NVW x 32 16-byte vectors)
        const int dyn = pf ? 16 * (D == 1024 ? 4 : 8) * 32 * 16 : 0;
        if (dyn > 0) {
          if (cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
              e != cudaSuccess)
            return launch_status(e);
        }
        int per_sm = 0;
        if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 512, dyn); e != cudaSuccess)
          return launch_status(e);
        if (per_sm < 1) per_sm = 1;
        // every group the same number of rows (n), give or take one
        const int64_t max_groups = (int64_t)per_sm * device_sm_count() * groups_per_cta;
        const int64_t n = (rows + max_groups - 1) / max_groups;
        const int64_t groups = (rows + n - 1) / n;
        kern<<<(unsigned)((groups + groups_per_cta - 1) / groups_per_cta), 512, dyn, s>>>(xp, wp, q, scale, yp, rows,
                                                                                            eps);
        return launch_status(cudaGetLastError());
      }
      // otherwise, 16-bit rows of two or four vectors per thread: the
      // persistent CTA kernel (flags bit 0: one CTA per row instead), one CTA
      // per resident slot
      if ((nv == 2 || nv == 4) && threads <= 256 && R == 1 && !(cfg && (cfg->flags & 1))) {
        const bool full = nvec % threads == 0 && nvec / threads == nv;
        // 128-thread CTAs are compiled for five resident CTAs per SM (at most
        // 102 registers a thread), larger ones for two
        auto kern = nv == 4 ? (threads <= 128 ? (full ? rmsnorm_quant_persistent_kernel<T, W, true, 4, 128>
                                                      : rmsnorm_quant_persistent_kernel<T, W, false, 4, 128>)
                                              : (full ? rmsnorm_quant_persistent_kernel<T, W, true, 4, 256>
                                                      : rmsnorm_quant_persistent_kernel<T, W, false, 4, 256>))
                            : (full ? rmsnorm_quant_persistent_kernel<T, W, true, 2, 256>
                                    : rmsnorm_quant_persistent_kernel<T, W, false, 2, 256>);
        int per_sm = 0;
        if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0);
            e != cudaSuccess)
          return launch_status(e);
        if (per_sm < 1) per_sm = 1;
        const int64_t slots = (int64_t)per_sm * device_sm_count();
        const unsigned grid = (unsigned)(rows < slots ? rows : slots);
        kern<<<grid, threads, 0, s>>>(xp, wp, q, scale, yp, rows, (int)D, eps);
        return launch_status(cudaGetLastError());
      }
    }
    auto go = [&](auto nv_tag, auto r_tag) -> int {
      constexpr int NV = decltype(nv_tag)::value, RR = decltype(r_tag)::value;
      const dim3 grid((unsigned)((rows + RR - 1) / RR));
      rmsnorm_quant_row_kernel<T, W, NV, RR><<<grid, threads, 0, s>>>(xp, wp, q, scale, yp, rows, (int)D, eps);
      return launch_status(cudaGetLastError());
    };
    using I1 = std::integral_constant<int, 1>;
    using I2 = std::integral_constant<int, 2>;
    using I4 = std::integral_constant<int, 4>;
    using I8 = std::integral_constant<int, 8>;
    auto by_r = [&](auto nv_tag) -> int {
      if (R == 1) return go(nv_tag, I1{});
      if (R == 2) return go(nv_tag, I2{});
      return go(nv_tag, I4{});
    };
    if (nv <= 1) return by_r(I1{});
    if (nv <= 2) return by_r(I2{});
    if (nv <= 4) return by_r(I4{});
    return go(I8{}, I1{});
  };
  if (weight_dtype == dtype)
    return B200_DISPATCH_FLOAT(dtype, [&] { return run(scalar_t{}, scalar_t{}); });
  if (weight_dtype == B200_F32)
    return B200_DISPATCH_FLOAT(dtype, [&] { return run(scalar_t{}, float{}); });
  return B200_ERR_UNSUPPORTED;
}
