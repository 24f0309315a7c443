// INT8 GEMM with int32 accumulation in tensor memory and a fused dequant
// epilogue, on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// Reference: triton_agent/ops/quant_matmul/reference.py:26-27
//   c = (a_q @ b_q) * a_scale * b_scale
// for pre-quantised operands: A [M,K] int8, W [N,K] int8 (K-major, i.e. the
// reference's b_q transposed), per-row sA [M] and per-column sW [N] fp32.
// acc = sum_k A[m,k]*W[n,k] is exact in int32 (|acc| <= K*127^2 < 2^31 for
// K < 133k); C = out(((float)acc * sA[m]) * sW[n]) with both products
// rounded separately, as the reference's eager fp32 multiplies are.
//
// CTA tile 128 x BN (BN = 128 or 256), K step 128 bytes per stage:
//   warp 0      TMA producer: A box {128 K, 128 M} and W box {128 K, BN N},
//               SWIZZLE_128B, into a ring of `stages` shared-memory slots
//   warp 1      allocates BN TMEM columns; one lane issues 4 x
//               tcgen05.mma (M=128, N=BN, K=32) per stage and commits each
//               stage back to the producer's "empty" barrier
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, dequant,
//               store (warp w reads TMEM lanes 32*(w%4) .. +31)
// Split-K (small M): each split writes its int32 partial tile to the
// workspace; the last split to finish (atomic ticket) sums the partials in
// a fixed order and runs the epilogue, so results stay exact and
// deterministic.  No cluster multicast: every CTA loads its own tiles.
#include "common.cuh"
#include "sm100.cuh"

B200_DEVICE_ERROR_WORD()

namespace b200 {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes (= int8 elements) of K per stage
constexpr int kEpiWarp0 = 2;
constexpr int kThreads = 192;
// Split-K tickets live in a fixed region at the start of the workspace so
// that calls of different shapes sharing one buffer find them at zero.
constexpr size_t kTicketBytes = 64 * 1024;

struct GemmParams {
  int64_t M, N, K, ldc;
  int k_tiles;          // ceil(K / BK)
  int k_tiles_split;    // k tiles per split
  int splits;
  int stages;
  int out_dtype;
  uint32_t stage_bytes;
};

template <int BN>
struct Smem {
  static constexpr uint32_t kA = BM * BK;  // 16 KB
  static constexpr uint32_t kB = BN * BK;
  static constexpr uint32_t kStage = kA + kB;
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <typename OutT>
__device__ __forceinline__ void store_out_row(OutT* dst, const float* v, int n_valid, bool vec_ok) {
  if (vec_ok && n_valid == 32) {
    if constexpr (sizeof(OutT) == 2) {
#pragma unroll
      for (int c = 0; c < 4; ++c) reinterpret_cast<uint4*>(dst)[c] = pack16<OutT>(v + 8 * c);
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c)
        reinterpret_cast<float4*>(dst)[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
  } else {
    for (int j = 0; j < n_valid; ++j) dst[j] = from_f32<OutT>(v[j]);
  }
}

// Dequantises 32 accumulators of one row and writes them.
template <typename OutT>
__device__ __forceinline__ void epilogue_chunk(const uint32_t* acc, int64_t row, int64_t col0,
                                               const float* __restrict__ sA,
                                               const float* __restrict__ sW, OutT* __restrict__ C,
                                               int32_t* __restrict__ acc_out, const GemmParams& p) {
  const int64_t rem = p.N - col0;
  const int n_valid = rem < 32 ? (int)rem : 32;
  if (n_valid <= 0) return;
  const float sa = sA[row];
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float sw = (j < n_valid) ? __ldg(&sW[col0 + j]) : 0.f;
    v[j] = __fmul_rn(__fmul_rn(__int2float_rn((int)acc[j]), sa), sw);
  }
  OutT* dst = C + row * p.ldc + col0;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0);
  store_out_row<OutT>(dst, v, n_valid, vec_ok);
  if (acc_out != nullptr) {
    int32_t* ad = acc_out + row * p.N + col0;
    if (n_valid == 32 && ((reinterpret_cast<uintptr_t>(ad) & 15u) == 0)) {
#pragma unroll
      for (int c = 0; c < 8; ++c)
        reinterpret_cast<int4*>(ad)[c] = make_int4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
    } else {
      for (int j = 0; j < n_valid; ++j) ad[j] = (int32_t)acc[j];
    }
  }
}

template <int BN, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    int8_gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_a,
                             const __grid_constant__ CUtensorMap tm_b, const float* __restrict__ sA,
                             const float* __restrict__ sW, OutT* __restrict__ C,
                             int32_t* __restrict__ acc_out, int32_t* __restrict__ partials,
                             int* __restrict__ tickets, GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the SWIZZLE_128B atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x, n_tile = blockIdx.y, split = blockIdx.z;
  const int64_t m0 = (int64_t)m_tile * BM, n0 = (int64_t)n_tile * BN;
  const int kt0 = split * p.k_tiles_split;
  const int kt1 = min(kt0 + p.k_tiles_split, p.k_tiles);
  const int n_k = max(kt1 - kt0, 0);

  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + p.stages * p.stage_bytes);
  uint64_t* empty_bar = full_bar + p.stages;
  uint64_t* accum_bar = empty_bar + p.stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_bar + 1);
  int* s_flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] abort, [1] last split

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      sm100::mbar_init(sm100::smem_u32(&full_bar[s]), 1);
      sm100::mbar_init(sm100::smem_u32(&empty_bar[s]), 1);
    }
    sm100::mbar_init(sm100::smem_u32(accum_bar), 1);
    s_flags[0] = 0;
    s_flags[1] = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), BN);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_a);
      sm100::tma_prefetch_desc(&tm_b);
      const uint32_t base = sm100::smem_u32(smem);
      int issued = 0;
      for (int i = 0; i < n_k; ++i) {
        const int s = i % p.stages;
        if (!sm100::mbar_wait(sm100::smem_u32(&empty_bar[s]), ((i / p.stages) & 1) ^ 1)) {
          b200_dev_error(kDevErrTimeoutEmpty);
          atomicExch(&s_flags[0], 1);
          break;
        }
        if (*(volatile int*)&s_flags[0]) break;
        const uint32_t fb = sm100::smem_u32(&full_bar[s]);
        sm100::mbar_arrive_expect_tx(fb, p.stage_bytes);
        const int32_t kx = (kt0 + i) * BK;
        const uint32_t sa = base + s * p.stage_bytes;
        sm100::tma_load_2d(sa, &tm_a, fb, kx, (int32_t)m0);
        sm100::tma_load_2d(sa + Smem<BN>::kA, &tm_b, fb, kx, (int32_t)n0);
        ++issued;
      }
      for (int i = issued - 1; i >= 0 && i >= issued - p.stages; --i) {
        const int s = i % p.stages;
        if (!sm100::mbar_wait(sm100::smem_u32(&full_bar[s]), (i / p.stages) & 1))
          b200_dev_error(kDevErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::make_idesc(/*D s32*/ 2, /*A s8*/ 1, /*B s8*/ 1, 0, 0, BM, BN);
      const uint32_t base = sm100::smem_u32(smem);
      for (int i = 0; i < n_k; ++i) {
        const int s = i % p.stages;
        if (!sm100::mbar_wait(sm100::smem_u32(&full_bar[s]), (i / p.stages) & 1)) {
          b200_dev_error(kDevErrTimeoutFull);
          atomicExch(&s_flags[0], 1);
          break;
        }
        if (*(volatile int*)&s_flags[0]) break;
        sm100::tc_fence_after();
        const uint32_t a_base = base + s * p.stage_bytes;
        const uint32_t b_base = a_base + Smem<BN>::kA;
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk) {
          // K-major SWIZZLE_128B: 8-row atoms of 1024 B stacked along M/N
          // (SBO = 1024); stepping K by 32 bytes inside the atom moves the
          // start address, the hardware applies the swizzle.
          const uint64_t ad = sm100::make_smem_desc(a_base + kk * 32, 16, 1024, sm100::kSwizzle128B);
          const uint64_t bd = sm100::make_smem_desc(b_base + kk * 32, 16, 1024, sm100::kSwizzle128B);
          sm100::mma_i8_ss(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        sm100::tc_commit(sm100::smem_u32(&empty_bar[s]));
      }
      // Signals the epilogue once every issued MMA has completed (also on
      // the abort path, so TMEM is never released under a running MMA).
      sm100::tc_commit(sm100::smem_u32(accum_bar));
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int64_t row = m0 + quarter * 32 + lane;
    const bool ok = sm100::mbar_wait(sm100::smem_u32(accum_bar), 0);
    if (!ok) {
      b200_dev_error(kDevErrTimeoutMma);
      atomicExch(&s_flags[0], 1);
    }
    sm100::tc_fence_after();
    const uint32_t t_row = tmem + ((uint32_t)(quarter * 32) << 16);
    if (p.splits == 1) {
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t acc[32];
          sm100::tmem_ld_32x32b_x32(t_row + c, acc);
          sm100::tmem_wait_ld();
          if (n_k == 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0;
          }
          if (row < p.M) epilogue_chunk<OutT>(acc, row, n0 + c, sA, sW, C, acc_out, p);
        }
      }
    } else {
      // write this split's partial tile, then the last split reduces
      const int64_t Mp = (int64_t)gridDim.x * BM;
      int32_t* mine = partials + ((int64_t)split * Mp + row) * p.N;
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t acc[32];
          sm100::tmem_ld_32x32b_x32(t_row + c, acc);
          sm100::tmem_wait_ld();
          if (n_k == 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0;
          }
          const int64_t col0 = n0 + c;
          if (row < p.M)
            for (int j = 0; j < 32 && col0 + j < p.N; ++j) mine[col0 + j] = (int32_t)acc[j];
        }
      }
      __threadfence();
      named_bar_sync(1, 128);
      if (threadIdx.x == kEpiWarp0 * 32) {
        int* t = tickets + (int64_t)m_tile * gridDim.y + n_tile;
        const int prev = atomicAdd(t, 1);
        const int last = (prev == p.splits - 1);
        if (last) atomicExch(t, 0);
        s_flags[1] = last;
      }
      named_bar_sync(1, 128);
      if (s_flags[1]) {
        __threadfence();
        if (row < p.M) {
#pragma unroll 1
          for (int c = 0; c < BN; c += 32) {
            const int64_t col0 = n0 + c;
            if (col0 >= p.N) break;
            uint32_t acc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0;
            for (int s = 0; s < p.splits; ++s) {
              const int32_t* src = partials + ((int64_t)s * Mp + row) * p.N + col0;
              for (int j = 0; j < 32 && col0 + j < p.N; ++j) acc[j] += (uint32_t)__ldcg(src + j);
            }
            epilogue_chunk<OutT>(acc, row, col0, sA, sW, C, acc_out, p);
          }
        }
      }
    }
    sm100::tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, BN);
  }
}

struct GemmPlan {
  int BN, splits, k_tiles, k_tiles_split, stages;
  uint32_t stage_bytes;
  size_t smem, ws_bytes;
  int m_tiles, n_tiles;
};

GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, const b200_launch_cfg* cfg) {
  GemmPlan g{};
  g.k_tiles = (int)((K + BK - 1) / BK);
  const int sms = device_sm_count();
  int bn = (cfg && cfg->tile_n > 0) ? cfg->tile_n : 0;
  g.m_tiles = (int)((M + BM - 1) / BM);
  if (bn != 128 && bn != 256) {
    // 256-wide tiles when they still give at least one full wave of CTAs.
    const int64_t t256 = g.m_tiles * ((N + 255) / 256);
    bn = (t256 >= sms && N >= 256) ? 256 : 128;
  }
  g.BN = bn;
  g.n_tiles = (int)((N + bn - 1) / bn);
  int splits = (cfg && cfg->split > 0) ? cfg->split : 0;
  if (splits == 0) {
    const int64_t tiles = (int64_t)g.m_tiles * g.n_tiles;
    splits = 1;
    while (tiles * splits < sms && splits * 2 <= g.k_tiles && splits < 16) splits *= 2;
  }
  if (splits > g.k_tiles) splits = g.k_tiles;
  if (splits < 1) splits = 1;
  g.k_tiles_split = (g.k_tiles + splits - 1) / splits;
  g.splits = (g.k_tiles + g.k_tiles_split - 1) / g.k_tiles_split;
  g.stage_bytes = (uint32_t)(BM * BK + bn * BK);
  const size_t budget = 227 * 1024 - 1024 - 256;
  int stages = (cfg && cfg->stages > 0) ? cfg->stages : 8;
  while (stages > 2 && (size_t)stages * g.stage_bytes > budget) --stages;
  g.stages = stages;
  g.smem = (size_t)stages * g.stage_bytes + 1024 + 256;
  if (g.splits > 1) {
    const size_t parts = (size_t)g.splits * g.m_tiles * BM * (size_t)N * 4;
    g.ws_bytes = kTicketBytes + parts;
  }
  return g;
}

template <int BN, typename OutT>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const float* sA, const float* sW, void* C,
                int32_t* acc_out, void* ws, const GemmPlan& g, GemmParams p, cudaStream_t s) {
  auto kern = int8_gemm_tcgen05_kernel<BN, OutT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
  if (e != cudaSuccess) return launch_status(e);
  int32_t* parts = nullptr;
  int* tickets = nullptr;
  if (g.splits > 1) {
    tickets = static_cast<int*>(ws);
    parts = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + kTicketBytes);
  }
  dim3 grid(g.m_tiles, g.n_tiles, g.splits);
  kern<<<grid, kThreads, g.smem, s>>>(ta, tb, sA, sW, static_cast<OutT*>(C), acc_out, parts, tickets, p);
  return launch_status(cudaGetLastError());
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" size_t b200_int8_gemm_workspace_size(int64_t M, int64_t N, int64_t K, const b200_launch_cfg* cfg) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return plan_gemm(M, N, K, cfg).ws_bytes;
}

extern "C" int b200_int8_gemm(const int8_t* A, const int8_t* W, const float* sA, const float* sW, void* C,
                              int64_t M, int64_t N, int64_t K, int64_t ldc, int32_t out_dtype,
                              int32_t* acc_out, void* workspace, size_t workspace_bytes,
                              const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("int8_gemm")) return e;
  if (M < 0 || N < 0 || K < 0) return B200_ERR_BAD_ARG;
  if (M == 0 || N == 0) return B200_OK;
  if (!A || !W || !sA || !sW || !C) return B200_ERR_BAD_ARG;
  if (K == 0 || K % 16 != 0) return B200_ERR_UNSUPPORTED;  // TMA row pitch must be 16-byte aligned
  if (K > 131072) return B200_ERR_UNSUPPORTED;             // int32 accumulator range
  if (ldc < N) return B200_ERR_BAD_ARG;
  if (!aligned16(A) || !aligned16(W)) return B200_ERR_ALIGNMENT;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL) return B200_ERR_UNSUPPORTED;
  const GemmPlan g = plan_gemm(M, N, K, cfg);
  if (g.m_tiles > 65535 * 1024 || g.n_tiles > 65535) return B200_ERR_UNSUPPORTED;
  if (g.splits > 1 && (workspace == nullptr || workspace_bytes < g.ws_bytes)) return B200_ERR_WORKSPACE;
  if (g.splits > 1 && (size_t)g.m_tiles * g.n_tiles * 4 > kTicketBytes) return B200_ERR_UNSUPPORTED;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {BK, BM};
    int st = encode_tensor_map(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, A, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {BK, (uint32_t)g.BN};
    int st = encode_tensor_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, W, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.k_tiles = g.k_tiles;
  p.k_tiles_split = g.k_tiles_split;
  p.splits = g.splits;
  p.stages = g.stages;
  p.out_dtype = out_dtype;
  p.stage_bytes = g.stage_bytes;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto go = [&](auto out_tag) -> int {
    using OutT = decltype(out_tag);
    return g.BN == 256 ? launch_gemm<256, OutT>(ta, tb, sA, sW, C, acc_out, workspace, g, p, s)
                       : launch_gemm<128, OutT>(ta, tb, sA, sW, C, acc_out, workspace, g, p, s);
  };
  switch (out_dtype) {
    case B200_F16: return go(__half{});
    case B200_BF16: return go(__nv_bfloat16{});
    case B200_F32: return go(float{});
    default: return B200_ERR_UNSUPPORTED;
  }
}
