// INT8 GEMM with int32 accumulation in tensor memory and a fused dequant
// epilogue, on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// Reference: triton_agent/ops/quant_matmul/reference.py:26-27
//   c = (a_q @ b_q) * a_scale * b_scale
// for pre-quantised operands: A [M,K] int8, W [N,K] int8 (K-major, i.e. the
// reference's b_q transposed), per-row sA [M] and per-column sW [N] fp32.
// acc = sum_k A[m,k]*W[n,k] is exact in int32 (|acc| <= K*127^2 < 2^31 for
// K <= 131072); C = out(((float)acc * sA[m]) * sW[n]) with both products
// rounded separately, as the reference's eager fp32 multiplies are.
//
// Two kernels, both fed by TMA (SWIZZLE_128B, K-major, no cluster multicast):
//
// int8_gemm_tcgen05_kernel -- persistent, one CTA per SM, 128 x BN output
//   tiles (BN = 128 or 256) taken round-robin in m-fastest order (CTAs
//   running together share W panels in L2).  Warp 0: TMA producer streaming
//   A {128 K x 128 M} and W {128 K x BN N} boxes into a ring of stages,
//   continuously across tiles.  Warp 1: allocates 2 x BN TMEM columns (two
//   accumulators) and one lane issues 4 tcgen05.mma (M=128, N=BN, K=32) per
//   stage.  Warps 2..5: epilogue, tcgen05.ld 32x32b.x32, dequant, 16-byte
//   stores.  The accumulator of tile i drains while tile i+1 accumulates in
//   the other half of TMEM, so the epilogue is off the tensor pipe's path.
//
// int8_gemm_skinny_kernel -- small M (<= 64, decode-time activations).  The
//   operands are swapped so W rows fill the 128-row side of the MMA and the
//   M activation rows its N side (16..64); the accumulator tile is
//   C^T[128 n x M].  K is split across CTAs so enough SMs stream W; split
//   partials are summed exactly with int32 red.add into a workspace tile and
//   the last split (atomic ticket) dequantises and re-zeroes it.
#include "common.cuh"
#include "sm100.cuh"

B200_DEVICE_ERROR_WORD()

namespace b200 {
namespace {

constexpr int BM = 128;
constexpr int kMaxRanks = 8;  // fused all-gather: ranks of one node
constexpr int BK = 128;  // bytes (= int8 elements) of K per stage
static_assert(BK / 32 == 4, "four K=32 MMA steps per k tile");
constexpr int kThreads = 192;
// Split-K tickets live in a fixed region at the start of the workspace so
// that calls of different shapes sharing one buffer find them at zero.
constexpr size_t kTicketBytes = 64 * 1024;

struct GemmParams {
  int64_t M, N, K, ldc;
  int k_tiles;          // ceil(K / BK)
  int k_tiles_split;    // k tiles per split (skinny)
  int splits;
  int stages;
  int m_tiles, n_tiles, num_tiles;
  uint32_t stage_bytes;
  uint32_t a_bytes;     // bytes of the first operand box(es) in a stage
  int group;            // streaming kernel: k tiles per stage
  int k_groups;         // streaming kernel: ceil(k_tiles / group)
  // fused all-gather (world > 0): every output chunk also goes to dst[r]
  // (C of rank r, this device's view) at column offset col_off; rank `self`'s
  // own copy is the kernel's C argument
  int world, self;
  int64_t col_off;
  void* dst[kMaxRanks];
  const void* bias;     // bias + GELU flavour: [N] of the output type
  int staged;           // tile kernels: 256-byte row groups through the staged epilogue (gather_group)
  // CTA-pair kernel work items: items < full_items are whole tiles; the
  // last partial wave's tiles follow as two half-width items each
  int full_items, num_items;
};

// Work item of the CTA-pair kernel: output rows from m_tile, columns
// [col, col + w) (w = PN, or PN / 2 for a half of a last-wave tile).
struct PairItem {
  int m_tile;
  int64_t col;
  int w;
};
__device__ __forceinline__ PairItem pair_item(const GemmParams& p, int item, int pn) {
  if (item < p.full_items) return {item % p.m_tiles, (int64_t)(item / p.m_tiles) * pn, pn};
  const int hi = item - p.full_items;
  const int t = p.full_items + (hi >> 1);
  return {t % p.m_tiles, (int64_t)(t / p.m_tiles) * pn + (hi & 1) * (pn / 2), pn / 2};
}

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
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n_valid) dst[j] = from_f32<OutT>(v[j]);
  }
}

__device__ __forceinline__ float dequant(uint32_t acc, float sa, float sw) {
  return __fmul_rn(__fmul_rn(__int2float_rn((int)acc), sa), sw);
}

// Dequantises 32 accumulators of one row and writes them (and the raw
// accumulators when acc_out is given).
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
    v[j] = dequant(acc[j], sa, sw);
  }
  const int64_t off = row * p.ldc + col0 + p.col_off;
  OutT* dst = C + off;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  store_out_row<OutT>(dst, v, n_valid, vec_ok);
  // fused all-gather: the same chunk into every peer's C over NVLink, in an
  // order rotated by rank so the ranks' stores spread over all links
  for (int i = 1; i < p.world; ++i) {
    int r = p.self + i;
    if (r >= p.world) r -= p.world;
    store_out_row<OutT>(static_cast<OutT*>(p.dst[r]) + off, v, n_valid, vec_ok);
  }
  if (acc_out != nullptr) {
    int32_t* ad = acc_out + row * p.N + col0;
    if (n_valid == 32 && ((reinterpret_cast<uintptr_t>(ad) & 15u) == 0)) {
#pragma unroll
      for (int c = 0; c < 8; ++c)
        reinterpret_cast<int4*>(ad)[c] = make_int4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < n_valid) ad[j] = (int32_t)acc[j];
    }
  }
}

// Staged epilogue for 128 columns of a warp's 32 accumulator rows (16-bit
// outputs): dequantise in registers, stage [32 rows][128 cols] in the
// warp's shared buffer, then write it back row by row -- 16 lanes x 16 B,
// one 256-byte run per row -- into this rank's C and, for the fused
// all-gather, every peer's C.  Row-at-a-time stores (each lane its own row,
// 64 bytes at a time) touch 32 rows per instruction and made the epilogue
// longer than a short mainloop (4096 x 14336 x 1024: 113 us, staged 76 us;
// x 4096: 168 -> 145 us); to a peer they arrive as 16-byte NVLink writes.
// The next 32 columns' TMEM load is in flight while a chunk is dequantised,
// and the group's 128 column scales are one 16-byte load per lane,
// broadcast by shuffles.
constexpr int kGatherRowData = 256;                     // bytes of one row of a group
constexpr int kGatherRowBytes = kGatherRowData + 16;     // +16 B: conflict-free both ways
constexpr int kGatherWarpBytes = 32 * kGatherRowBytes;
// columns of a staged group: 128 of a 16-bit output, 64 of fp32
template <typename OutT>
constexpr int gather_cols() {
  return kGatherRowData / (int)sizeof(OutT);
}

// release: when non-zero, the address (shared::cluster) of the accumulator
// buffer's empty barrier, arrived on as soon as this group's last TMEM load
// has completed -- the MMA warp may refill the buffer while the rows are
// still being written out.
template <typename OutT>
__device__ __forceinline__ void gather_group(uint32_t t_row, int64_t row0, int lane, int64_t col0,
                                             const float* __restrict__ sA, const float* __restrict__ sW,
                                             OutT* __restrict__ C, const GemmParams& p, uint8_t* stage,
                                             uint32_t release = 0) {
  constexpr int GC = gather_cols<OutT>();
  constexpr int VN = Vec<OutT>::N;  // outputs per 16-byte piece
  const int64_t row = row0 + lane;
  const float sa = row < p.M ? sA[row] : 0.f;
  // scales: lane holds columns col0 + SW lane .. + SW - 1 (4 of 128 for 16-bit
  // outputs, 2 of 64 for fp32), one aligned load, broadcast by shuffles
  constexpr int SW = GC / 32;
  float swv[SW];
  if constexpr (SW == 4) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(sW + col0) + lane);
    swv[0] = t.x;
    swv[1] = t.y;
    swv[2] = t.z;
    swv[3] = t.w;
  } else {
    const float2 t = __ldg(reinterpret_cast<const float2*>(sW + col0) + lane);
    swv[0] = t.x;
    swv[1] = t.y;
  }
  uint32_t acc[2][32];
  sm100::tmem_ld_32x32b_x32(t_row, acc[0]);
#pragma unroll
  for (int c4 = 0; c4 < GC / 32; ++c4) {
    sm100::tmem_wait_ld_regs(acc[c4 & 1]);
    if (c4 + 1 < GC / 32) sm100::tmem_ld_32x32b_x32(t_row + (c4 + 1) * 32, acc[(c4 + 1) & 1]);
    if (c4 + 1 == GC / 32 && release != 0) {
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive_cluster(release);
    }
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      // column c4 * 32 + j: component j % SW of lane (c4 * 32 + j) / SW
      v[j] = dequant(acc[c4 & 1][j], sa, __shfl_sync(0xffffffffu, swv[j % SW], (c4 * 32 + j) / SW));
    }
    // 32 columns = 32 * sizeof(OutT) bytes of the staged row
#pragma unroll
    for (int q = 0; q < 32 / VN; ++q)
      *reinterpret_cast<uint4*>(stage + lane * kGatherRowBytes + c4 * 32 * (int)sizeof(OutT) + q * 16) =
          pack16<OutT>(v + VN * q);
  }
  __syncwarp();
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    const int r = 2 * i + (lane >> 4), piece = lane & 15;
    const uint4 w = *reinterpret_cast<const uint4*>(stage + r * kGatherRowBytes + piece * 16);
    const int64_t grow = row0 + r;
    if (grow < p.M) {
      const int64_t off = grow * p.ldc + p.col_off + col0 + piece * VN;
      *reinterpret_cast<uint4*>(C + off) = w;
      for (int k = 1; k < p.world; ++k) {
        int d = p.self + k;
        if (d >= p.world) d -= p.world;
        *reinterpret_cast<uint4*>(static_cast<OutT*>(p.dst[d]) + off) = w;
      }
    }
  }
  __syncwarp();
}

// GELU with the tanh approximation of matmul_epilogue/reference.py:17,
// 0.5 c (1 + tanh(sqrt(2/pi) (c + 0.044715 c^3))), in fp32 with the
// hardware tanh (tanh.approx.f32, relative error ~2^-11, below the bf16/fp16
// rounding of the output).
__device__ __forceinline__ float gelu_tanh(float c) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * c, c * c, c);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * c * (1.0f + t);
}

// fp32 accumulators of one row + bias, GELU, one rounding to OutT.
template <typename OutT>
__device__ __forceinline__ void bias_gelu_chunk(const uint32_t* acc, int64_t row, int64_t col0,
                                                OutT* __restrict__ C, const GemmParams& p) {
  const int64_t rem = p.N - col0;
  const int n_valid = rem < 32 ? (int)rem : 32;
  if (n_valid <= 0) return;
  const OutT* bias = static_cast<const OutT*>(p.bias);
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float b = (j < n_valid) ? to_f32(bias[col0 + j]) : 0.f;
    v[j] = gelu_tanh(__uint_as_float(acc[j]) + b);
  }
  OutT* dst = C + row * p.ldc + col0;
  store_out_row<OutT>(dst, v, n_valid, (reinterpret_cast<uintptr_t>(dst) & 15u) == 0);
}

// Shared-memory carve-up of both kernels: [ring of stages][barriers...]
struct Bars {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* acc_full;   // [2]
  uint64_t* acc_empty;  // [2]
  uint64_t* mma_done;
  uint32_t* tmem_slot;
  int* flags;      // [0] abort, [1] last split
  uint8_t* gather;  // fused all-gather staging, kGatherWarpBytes per epilogue warp
};

__device__ __forceinline__ Bars carve(uint8_t* smem, const GemmParams& p) {
  Bars b;
  b.full = reinterpret_cast<uint64_t*>(smem + p.stages * p.stage_bytes);
  b.empty = b.full + p.stages;
  b.acc_full = b.empty + p.stages;
  b.acc_empty = b.acc_full + 2;
  b.mma_done = b.acc_empty + 2;
  b.tmem_slot = reinterpret_cast<uint32_t*>(b.mma_done + 1);
  b.flags = reinterpret_cast<int*>(b.tmem_slot + 1);
  b.gather = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(b.flags + 2) + 15) & ~uintptr_t(15));
  return b;
}

__device__ __forceinline__ bool aborted(const Bars& b) { return *(volatile int*)&b.flags[0] != 0; }
__device__ __forceinline__ void set_abort(const Bars& b, int code) {
  b200_dev_error(code);
  atomicExch(&b.flags[0], 1);
}

// Position in the ring of stages: stage index and fill phase, advanced
// without divisions (they sit on the issue path of a single thread).
struct Ring {
  int s = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next(int stages) {
    if (++s == stages) {
      s = 0;
      ph ^= 1u;
    }
  }
};

// Producer: streams `count` stages of {first operand box at (kx, r0), second
// at (kx, r1)} for k tiles [kt0, kt0 + count), continuing the ring position
// `r` (`it` counts fills, for the final drain).  Returns false if a wait
// timed out.
__device__ __forceinline__ bool produce(const CUtensorMap* ta, const CUtensorMap* tb, const Bars& bars,
                                        uint32_t base, const GemmParams& p, int kt0, int count, int32_t r0,
                                        int32_t r1, Ring& r, int& it) {
  for (int i = 0; i < count; ++i, ++it, r.next(p.stages)) {
    const int s = r.s;
    if (!sm100::mbar_wait(sm100::smem_u32(&bars.empty[s]), r.ph ^ 1u)) return false;
    if (aborted(bars)) return false;
    const uint32_t fb = sm100::smem_u32(&bars.full[s]);
    sm100::mbar_arrive_expect_tx(fb, p.stage_bytes);
    const int32_t kx = (kt0 + i) * BK;
    const uint32_t dst = base + s * p.stage_bytes;
    sm100::tma_load_2d(dst, ta, fb, kx, r0);
    sm100::tma_load_2d(dst + p.a_bytes, tb, fb, kx, r1);
  }
  return true;
}

// Waits (bounded) for the last fill of every stage so no bulk copy is still
// landing when the CTA exits.
__device__ __forceinline__ void drain_fills(const Bars& bars, const GemmParams& p, int it) {
  for (int i = it - 1; i >= 0 && i >= it - p.stages; --i)
    if (!sm100::mbar_wait(sm100::smem_u32(&bars.full[i % p.stages]), (i / p.stages) & 1))
      b200_dev_error(kDevErrTimeoutFull);
}

// MMA issue of `count` stages into accumulator `d_tmem`, run by a whole warp
// (waits, descriptors and ring position warp-uniform); the lane with
// `leader` set issues the MMAs and commits.  Returns false on timeout.
template <int N_MMA>
__device__ __forceinline__ bool mma_stages(const Bars& bars, uint32_t base, const GemmParams& p, uint32_t d_tmem,
                                           int count, Ring& r, uint32_t leader) {
  constexpr uint32_t idesc = sm100::make_idesc(/*D s32*/ 2, /*A s8*/ 1, /*B s8*/ 1, 0, 0, BM, N_MMA);
  // K-major SWIZZLE_128B: 8-row atoms of 1024 B stacked along M/N (SBO =
  // 1024); stepping K by 32 bytes inside the atom moves the start address,
  // the hardware applies the swizzle.  Descriptors of stage 0; a stage or K
  // step adds its byte offset >> 4 to the start-address field (bits
  // [0,14)), which never carries since shared addresses stay below 2^18.
  const uint64_t ad0 = sm100::make_smem_desc(base, 16, 1024, sm100::kSwizzle128B);
  const uint64_t bd0 = sm100::make_smem_desc(base + p.a_bytes, 16, 1024, sm100::kSwizzle128B);
  for (int i = 0; i < count; ++i, r.next(p.stages)) {
    if (!sm100::mbar_wait_warp(sm100::smem_u32(&bars.full[r.s]), r.ph)) return false;
    if (aborted(bars)) return false;
    sm100::tc_fence_after();
    const uint64_t so = (uint64_t)((r.s * p.stage_bytes) >> 4);
#pragma unroll
    for (int kk = 0; kk < BK / 32; ++kk)
      sm100::mma_i8_ss(d_tmem, ad0 + so + 2 * kk, bd0 + so + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u, leader);
    sm100::tc_commit(sm100::smem_u32(&bars.empty[r.s]), leader);
  }
  return true;
}

__device__ __forceinline__ void init_bars(const Bars& bars, const GemmParams& p) {
  for (int s = 0; s < p.stages; ++s) {
    sm100::mbar_init(sm100::smem_u32(&bars.full[s]), 1);
    sm100::mbar_init(sm100::smem_u32(&bars.empty[s]), 1);
  }
  for (int a = 0; a < 2; ++a) {
    sm100::mbar_init(sm100::smem_u32(&bars.acc_full[a]), 1);
    sm100::mbar_init(sm100::smem_u32(&bars.acc_empty[a]), 4);  // one arrival per epilogue warp
  }
  sm100::mbar_init(sm100::smem_u32(bars.mma_done), 1);
  bars.flags[0] = 0;
  bars.flags[1] = 0;
  sm100::fence_barrier_init();
}

// ----------------------------------------------------------------------------
// Persistent kernel (M > 64)
// ----------------------------------------------------------------------------
template <int BN, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    int8_gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                             const float* __restrict__ sA, const float* __restrict__ sW, OutT* __restrict__ C,
                             int32_t* __restrict__ acc_out, GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Bars bars = carve(smem, p);
  const uint32_t base = sm100::smem_u32(smem);
  if (threadIdx.x == 0) init_bars(bars, p);
  if (warp == 1) {
    sm100::tmem_alloc(sm100::smem_u32(bars.tmem_slot), 2 * BN);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *bars.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_a);
      sm100::tma_prefetch_desc(&tm_b);
      int it = 0;
      Ring r;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        const int m_tile = t % p.m_tiles, n_tile = t / p.m_tiles;
        if (!produce(&tm_a, &tm_b, bars, base, p, 0, p.k_tiles, m_tile * BM, n_tile * BN, r, it)) {
          set_abort(bars, kDevErrTimeoutEmpty);
          break;
        }
      }
      drain_fills(bars, p, it);
    }
  } else if (warp == 1) {
    // MMA issue: the whole warp runs the loop, one elected lane issues
    const uint32_t leader = sm100::elect_one();
    Ring r;
    int lt = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++lt) {
      const int a = lt & 1;
      // the epilogue must have drained this accumulator (tile lt - 2)
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&bars.acc_empty[a]), ((lt >> 1) & 1) ^ 1)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      ok = mma_stages<BN>(bars, base, p, tmem + a * BN, p.k_tiles, r, leader);
      sm100::tc_commit(sm100::smem_u32(&bars.acc_full[a]), leader);
    }
    if (!ok && leader) set_abort(bars, kDevErrTimeoutFull);
    // every issued MMA has completed before TMEM is released
    sm100::tc_commit(sm100::smem_u32(bars.mma_done), leader);
    if (!sm100::mbar_wait_warp(sm100::smem_u32(bars.mma_done), 0) && leader) b200_dev_error(kDevErrTimeoutMma);
  } else {
    const int quarter = warp & 3;
    int lt = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++lt) {
      const int a = lt & 1;
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&bars.acc_full[a]), (lt >> 1) & 1)) {
        set_abort(bars, kDevErrTimeoutMma);
        break;
      }
      sm100::tc_fence_after();
      const int m_tile = t % p.m_tiles, n_tile = t / p.m_tiles;
      const int64_t row = (int64_t)m_tile * BM + quarter * 32 + lane;
      const uint32_t t_row = tmem + a * BN + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN;) {
        const int64_t col0 = (int64_t)n_tile * BN + c;
        {
          constexpr int GC = gather_cols<OutT>();
          if (p.staged && col0 + GC <= p.N && c + GC <= BN) {  // warp-uniform
            gather_group<OutT>(t_row + c, row - lane, lane, col0, sA, sW, C, p,
                               bars.gather + (warp - 2) * kGatherWarpBytes);
            c += GC;
            continue;
          }
        }
        uint32_t acc[32];
        sm100::tmem_ld_32x32b_x32(t_row + c, acc);
        sm100::tmem_wait_ld_regs(acc);
        if (row < p.M && !aborted(bars)) epilogue_chunk<OutT>(acc, row, col0, sA, sW, C, acc_out, p);
        c += 32;
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&bars.acc_empty[a]));
    }
    // fused all-gather: peer stores visible system-wide before the signal kernel
    if (p.world > 1) __threadfence_system();
  }
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 2 * BN);
  }
}

// ----------------------------------------------------------------------------
// Pair kernel (M > 128): a cluster of two CTAs on two SMs computes 256 x 256
// output tiles with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32).
// Each CTA streams only its own 128 rows of A and 128 rows of W per stage
// (32 KB, where a 128 x 256 tile on one SM streams 48 KB), which cuts the
// L2 -> shared-memory traffic per MMA by a third.  Both CTAs: warp 0 TMA
// producer, warps 2..5 epilogue of the CTA's 128 accumulator rows (TMEM is
// allocated pair-wide, 2 x 256 columns).  Rank 0 only: warp 1 issues the
// pair MMAs.  Fills of both CTAs complete on rank 0's full barriers (rank 0
// expects both CTAs' bytes); rank 0 commits MMA progress to the empty and
// accumulator barriers of both CTAs, and both epilogues arrive on rank 0's
// acc_empty.  No multicast anywhere: every load reads global memory into
// the issuing CTA's own shared memory.
// ----------------------------------------------------------------------------
constexpr int kPairN = 256;  // widest pair tile (and the kind::f16 flavour's)

// TMEM columns for two accumulators of PN columns (allocations are powers of two).
constexpr uint32_t pair_tmem_cols(int pn) { return 2 * pn <= 256 ? 256u : 512u; }

// PN: output columns of a pair tile (128..256, a multiple of 32; each CTA
// loads PN / 2 rows of W per stage).  The host picks it per shape so the
// tiles fill whole waves of CTA pairs.
// kF16: the bf16/fp16 flavour (kind::f16, fp32 accumulators, B = b [K, N]
// N-contiguous, i.e. MN-major: per CTA two TMA boxes of 64 N x 64 K, 8 KB
// apart; epilogue bias + GELU) -- same pipeline, same 32 KB stages, same
// 32-byte K step per MMA.
template <typename OutT, bool kF16, int PN>
__global__ void __launch_bounds__(kThreads, 1)
    int8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                          const __grid_constant__ CUtensorMap tm_bh, const float* __restrict__ sA,
                          const float* __restrict__ sW, OutT* __restrict__ C, int32_t* __restrict__ acc_out,
                          GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_ctarank();
  const int pair = (int)(blockIdx.x >> 1), n_pairs = (int)(gridDim.x >> 1);
  const Bars bars = carve(smem, p);
  const uint32_t base = sm100::smem_u32(smem);
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      sm100::mbar_init(sm100::smem_u32(&bars.full[s]), 1);
      sm100::mbar_init(sm100::smem_u32(&bars.empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(sm100::smem_u32(&bars.acc_full[a]), 1);
      sm100::mbar_init(sm100::smem_u32(&bars.acc_empty[a]), 8);  // 4 epilogue warps in each CTA
    }
    sm100::mbar_init(sm100::smem_u32(bars.mma_done), 1);
    bars.flags[0] = 0;
    bars.flags[1] = 0;
    sm100::fence_barrier_init();
  }
  // both CTAs' barriers exist before either CTA signals the other's
  sm100::cluster_sync();
  if (warp == 1) {
    sm100::tmem_alloc_pair(sm100::smem_u32(bars.tmem_slot), pair_tmem_cols(PN));
    sm100::tmem_relinquish_pair();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *bars.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_a);
      sm100::tma_prefetch_desc(&tm_b);
      int it = 0;
      Ring r;
      bool ok = true;
      for (int t = pair; t < p.num_items && ok; t += n_pairs) {
        const PairItem itm = pair_item(p, t, PN);
        const int32_t a_row = itm.m_tile * 2 * BM + (int32_t)rank * BM;
        const int32_t b_row = (int32_t)itm.col + (int32_t)rank * (itm.w / 2);
        const CUtensorMap* tmb = itm.w == PN ? &tm_b : &tm_bh;  // half items: boxes of PN / 4 W rows
        const uint32_t fill_bytes = 2 * (p.a_bytes + (uint32_t)(itm.w / 2) * BK);
        for (int kt = 0; kt < p.k_tiles; ++kt, ++it, r.next(p.stages)) {
          const int s = r.s;
          if (!sm100::mbar_wait(sm100::smem_u32(&bars.empty[s]), r.ph ^ 1u) || aborted(bars)) {
            ok = false;
            break;
          }
          const uint32_t fb = sm100::smem_u32(&bars.full[s]);
          if (rank == 0) sm100::mbar_arrive_expect_tx(fb, kF16 ? 2 * p.stage_bytes : fill_bytes);  // both CTAs' fills
          const uint32_t fb0 = sm100::mapa_shared(fb, 0);
          const uint32_t dst = base + s * p.stage_bytes;
          if constexpr (kF16) {
            // 64 elements of K per stage; b [K, N]: boxes {64 N, 64 K} at N offsets 0 and 64
            sm100::tma_load_2d_pair(dst, &tm_a, fb0, kt * 64, a_row);
            sm100::tma_load_2d_pair(dst + p.a_bytes, &tm_b, fb0, b_row, kt * 64);
            sm100::tma_load_2d_pair(dst + p.a_bytes + 8192, &tm_b, fb0, b_row + 64, kt * 64);
          } else {
            sm100::tma_load_2d_pair(dst, &tm_a, fb0, kt * BK, a_row);
            sm100::tma_load_2d_pair(dst + p.a_bytes, tmb, fb0, kt * BK, b_row);
          }
        }
      }
      if (!ok) set_abort(bars, kDevErrTimeoutEmpty);
      // rank 0's full barriers count both CTAs' bytes: its drain covers the pair
      if (rank == 0) drain_fills(bars, p, it);
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // MMA issue for the pair: the whole warp runs the loop, one elected lane issues
      // D s32 from s8 x s8, or D f32 from bf16 (1) / fp16 (0) with B MN-major
      constexpr uint32_t ab_fmt = kF16 ? (std::is_same<OutT, __nv_bfloat16>::value ? 1u : 0u) : 1u;
      constexpr uint32_t idesc =
          sm100::make_idesc(kF16 ? 1u : 2u, ab_fmt, ab_fmt, 0, kF16 ? 1u : 0u, 2 * BM, PN);
      constexpr uint32_t idesc_half =
          sm100::make_idesc(kF16 ? 1u : 2u, ab_fmt, ab_fmt, 0, kF16 ? 1u : 0u, 2 * BM, PN / 2);
      const uint32_t leader = sm100::elect_one();
      const uint64_t ad0 = sm100::make_smem_desc(base, 16, 1024, sm100::kSwizzle128B);
      // B: K-major (K steps of 32 B inside the atom) or MN-major (the two
      // 64-wide N halves 8 KB apart = LBO; K steps of 16 rows x 128 B)
      const uint64_t bd0 = kF16 ? sm100::make_smem_desc(base + p.a_bytes, 8192, 1024, sm100::kSwizzle128B)
                                : sm100::make_smem_desc(base + p.a_bytes, 16, 1024, sm100::kSwizzle128B);
      constexpr uint32_t b_step = kF16 ? 2048 >> 4 : 2;
      const uint32_t empty0 = sm100::smem_u32(&bars.empty[0]);
      const uint32_t empty_r0 = sm100::mapa_shared(empty0, 0), empty_r1 = sm100::mapa_shared(empty0, 1);
      const uint32_t accf0 = sm100::smem_u32(&bars.acc_full[0]);
      const uint32_t accf_r0 = sm100::mapa_shared(accf0, 0), accf_r1 = sm100::mapa_shared(accf0, 1);
      Ring r;
      int lt = 0;
      bool ok = true;
      for (int t = pair; t < p.num_items && ok; t += n_pairs, ++lt) {
        const int a = lt & 1;
        const uint32_t id = t < p.full_items ? idesc : idesc_half;
        // both epilogues must have drained this accumulator (tile lt - 2)
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&bars.acc_empty[a]), ((lt >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem + a * PN;
        for (int kt = 0; kt < p.k_tiles; ++kt, r.next(p.stages)) {
          if (!sm100::mbar_wait_warp(sm100::smem_u32(&bars.full[r.s]), r.ph) || aborted(bars)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint64_t so = (uint64_t)((r.s * p.stage_bytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            if constexpr (kF16)
              sm100::mma_f16_ss_pair(d_tmem, ad0 + so + 2 * kk, bd0 + so + b_step * kk, id,
                                     (kt > 0 || kk > 0) ? 1u : 0u, leader);
            else
              sm100::mma_i8_ss_pair(d_tmem, ad0 + so + 2 * kk, bd0 + so + b_step * kk, id,
                                    (kt > 0 || kk > 0) ? 1u : 0u, leader);
          }
          sm100::tc_commit_pair(empty_r0 + 8 * r.s, leader);
          sm100::tc_commit_pair(empty_r1 + 8 * r.s, leader);
        }
        if (!ok) break;
        sm100::tc_commit_pair(accf_r0 + 8 * a, leader);
        sm100::tc_commit_pair(accf_r1 + 8 * a, leader);
      }
      if (!ok && leader) set_abort(bars, kDevErrTimeoutFull);
      // every issued MMA has completed before TMEM is released
      sm100::tc_commit_pair(sm100::mapa_shared(sm100::smem_u32(bars.mma_done), 0), leader);
      if (!sm100::mbar_wait_warp(sm100::smem_u32(bars.mma_done), 0) && leader) b200_dev_error(kDevErrTimeoutMma);
    }
  } else {
    const int quarter = warp & 3;
    int lt = 0;
    const uint32_t acc_empty0 = sm100::mapa_shared(sm100::smem_u32(&bars.acc_empty[0]), 0);
    for (int t = pair; t < p.num_items; t += n_pairs, ++lt) {
      const int a = lt & 1;
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&bars.acc_full[a]), (lt >> 1) & 1)) {
        set_abort(bars, kDevErrTimeoutMma);
        break;
      }
      sm100::tc_fence_after();
      const PairItem itm = pair_item(p, t, PN);
      const int64_t row = (int64_t)itm.m_tile * 2 * BM + (int64_t)rank * BM + quarter * 32 + lane;
      const uint32_t t_row = tmem + a * PN + ((uint32_t)(quarter * 32) << 16);
      bool released = false;
      for (int c = 0; c < itm.w;) {
        const int64_t col0 = itm.col + c;
        if constexpr (!kF16) {
          constexpr int GC = gather_cols<OutT>();
          if (p.staged && col0 + GC <= p.N && c + GC <= itm.w) {  // warp-uniform
            // the tile's last group hands the accumulator back before its rows go out
            released = c + GC == itm.w;
            gather_group<OutT>(t_row + c, row - lane, lane, col0, sA, sW, C, p,
                               bars.gather + (warp - 2) * kGatherWarpBytes, released ? acc_empty0 + a * 8 : 0u);
            c += GC;
            continue;
          }
        }
        uint32_t acc[32];
        sm100::tmem_ld_32x32b_x32(t_row + c, acc);
        sm100::tmem_wait_ld_regs(acc);
        if (row < p.M && !aborted(bars)) {
          if constexpr (kF16)
            bias_gelu_chunk<OutT>(acc, row, col0, C, p);
          else
            epilogue_chunk<OutT>(acc, row, col0, sA, sW, C, acc_out, p);
        }
        c += 32;
      }
      if (!released) {
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive_cluster(acc_empty0 + a * 8);
      }
    }
    // fused all-gather: peer stores visible system-wide before the signal kernel
    if (p.world > 1) __threadfence_system();
  }
  __syncthreads();
  // neither CTA leaves (or frees TMEM) while its peer may still signal it
  sm100::cluster_sync();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem, pair_tmem_cols(PN));
  }
}

// ----------------------------------------------------------------------------
// Streaming skinny kernel (M <= 64, default): the n_tiles x k_tiles W tiles
// (128 rows x 128 B) are cut into one contiguous range per CTA, n-major and
// k-minor, so every SM streams the same number of W bytes through one deep
// TMA ring (one CTA per SM).  A range splits into segments (one n tile, a
// run of its k tiles), accumulated alternately in two TMEM buffers.  A
// segment spanning all of K is dequantised directly; any other red.adds its
// exact int32 partial into the workspace and adds its k-tile count to the
// n tile's ticket, and the CTA that completes the count dequantises the
// tile and re-zeroes it (workspace and ticket) for the next call.
// ----------------------------------------------------------------------------
template <int MN, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    int8_gemm_stream_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                            const float* __restrict__ sA, const float* __restrict__ sW, OutT* __restrict__ C,
                            int32_t* __restrict__ acc_out, int32_t* __restrict__ ws, int* __restrict__ tickets,
                            GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Bars bars = carve(smem, p);
  const uint32_t base = sm100::smem_u32(smem);
  // kChains accumulators per buffer: consecutive MMAs of a segment rotate
  // over them, so the MMA pipe runs kChains independent accumulation chains
  // instead of one (an M=128, N<=64 MMA is far shorter than its latency);
  // the epilogue sums them (exact int32).
  constexpr int kChains = 4;
  constexpr int kChainCols = MN < 32 ? 32 : MN;   // chains start on 32-column boundaries
  constexpr int kCols = kChains * kChainCols;     // TMEM columns per buffer (a power of two >= 128)
  // work units: (n tile, group of p.group k tiles), n-major
  const int64_t U = (int64_t)p.n_tiles * p.k_groups;
  const int64_t u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
  if (threadIdx.x == 0) init_bars(bars, p);
  if (warp == 1) {
    sm100::tmem_alloc(sm100::smem_u32(bars.tmem_slot), 2 * kCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *bars.tmem_slot;
  const int n_first = (int)(u0 / p.k_groups);
  const int kg_first = (int)(u0 - (int64_t)n_first * p.k_groups);
  const uint32_t w_box = BM * BK, a_box = MN * BK;  // bytes of one k tile of W / of A

  if (warp == 0) {
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_w);
      sm100::tma_prefetch_desc(&tm_a);
      int it = 0;
      Ring r;
      int n = n_first, kg = kg_first;
      for (int64_t u = u0; u < u1; ++u, ++it, r.next(p.stages)) {
        if (!sm100::mbar_wait(sm100::smem_u32(&bars.empty[r.s]), r.ph ^ 1u) || aborted(bars)) {
          set_abort(bars, kDevErrTimeoutEmpty);
          break;
        }
        const uint32_t fb = sm100::smem_u32(&bars.full[r.s]);
        sm100::mbar_arrive_expect_tx(fb, p.stage_bytes);  // boxes past K arrive zero-filled, full size
        const uint32_t dst = base + r.s * p.stage_bytes;
        // the group's W boxes back to back: each W row is read as one run of
        // group * 128 contiguous bytes
        for (int g = 0; g < p.group; ++g)
          sm100::tma_load_2d(dst + g * w_box, &tm_w, fb, (kg * p.group + g) * BK, n * BM);
        for (int g = 0; g < p.group; ++g)
          sm100::tma_load_2d(dst + p.a_bytes + g * a_box, &tm_a, fb, (kg * p.group + g) * BK, 0);
        if (++kg == p.k_groups) {
          kg = 0;
          ++n;
        }
      }
      drain_fills(bars, p, it);
    }
  } else if (warp == 1) {
    const uint32_t leader = sm100::elect_one();
    Ring r;
    bool ok = true;
    int seg = 0;
    constexpr uint32_t idesc = sm100::make_idesc(/*D s32*/ 2, /*A s8*/ 1, /*B s8*/ 1, 0, 0, BM, MN);
    const uint64_t wd0 = sm100::make_smem_desc(base, 16, 1024, sm100::kSwizzle128B);
    const uint64_t ad0 = sm100::make_smem_desc(base + p.a_bytes, 16, 1024, sm100::kSwizzle128B);
    for (int64_t u = u0; u < u1 && ok; ++seg) {
      const int n = (int)(u / p.k_groups);
      const int64_t seg_end = min(u1, (int64_t)(n + 1) * p.k_groups);
      const int b = seg & 1;
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&bars.acc_empty[b]), ((seg >> 1) & 1) ^ 1)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const uint32_t d_buf = tmem + b * kCols;
      for (int64_t i = 0; u + i < seg_end && ok; ++i, r.next(p.stages)) {
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&bars.full[r.s]), r.ph) || aborted(bars)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint64_t so = (uint64_t)((r.s * p.stage_bytes) >> 4);
        for (int g = 0; g < p.group; ++g) {
          const uint64_t wg = wd0 + so + (uint64_t)((g * w_box) >> 4), ag = ad0 + so + (uint64_t)((g * a_box) >> 4);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            // chain kk (BK / 32 == kChains); its first MMA in the segment overwrites
            sm100::mma_i8_ss(d_buf + kk * kChainCols, wg + 2 * kk, ag + 2 * kk, idesc, (i > 0 || g > 0) ? 1u : 0u,
                             leader);
          }
        }
        sm100::tc_commit(sm100::smem_u32(&bars.empty[r.s]), leader);
      }
      sm100::tc_commit(sm100::smem_u32(&bars.acc_full[b]), leader);
      u = seg_end;
    }
    if (!ok && leader) set_abort(bars, kDevErrTimeoutFull);
    sm100::tc_commit(sm100::smem_u32(bars.mma_done), leader);
    if (!sm100::mbar_wait_warp(sm100::smem_u32(bars.mma_done), 0) && leader) b200_dev_error(kDevErrTimeoutMma);
  } else {
    const int quarter = warp & 3;
    // the dequant scales are loaded before the accumulators are ready (after
    // an L2 flush each is a DRAM round trip that would otherwise sit on the
    // kernel's tail): sA once, sW per segment before its accumulator wait
    constexpr int kSa = MN <= 32 ? MN : 1;
    float sa[kSa];
#pragma unroll
    for (int m = 0; m < kSa; ++m) sa[m] = (MN <= 32 && m < p.M) ? __ldg(&sA[m]) : 0.f;
    int seg = 0;
    for (int64_t u = u0; u < u1; ++seg) {
      const int n_tile = (int)(u / p.k_groups);
      const int64_t seg_end = min(u1, (int64_t)(n_tile + 1) * p.k_groups);
      const int count = (int)(seg_end - u);
      u = seg_end;
      const int b = seg & 1;
      const int64_t n = (int64_t)n_tile * BM + quarter * 32 + lane;  // output column (TMEM lane)
      const float sw = (count == p.k_groups && n < p.N) ? __ldg(&sW[n]) : 0.f;
      const bool ok = sm100::mbar_wait_warp(sm100::smem_u32(&bars.acc_full[b]), (seg >> 1) & 1);
      if (!ok) {
        set_abort(bars, kDevErrTimeoutMma);
        break;
      }
      sm100::tc_fence_after();
      uint32_t acc[MN];
#pragma unroll
      for (int j = 0; j < MN; ++j) acc[j] = 0;
      const uint32_t t_row = tmem + b * kCols + ((uint32_t)(quarter * 32) << 16);
      if constexpr (MN == 16) {
        // all chains' loads in flight, one wait
        uint32_t part[kChains][16];
#pragma unroll
        for (int ch = 0; ch < kChains; ++ch) sm100::tmem_ld_32x32b_x16(t_row + ch * kChainCols, part[ch]);
#pragma unroll
        for (int ch = 0; ch < kChains; ++ch) sm100::tmem_wait_ld_regs16(part[ch]);
#pragma unroll
        for (int ch = 0; ch < kChains; ++ch)
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] += part[ch][j];
      } else {
#pragma unroll
        for (int ch = 0; ch < kChains; ++ch) {
          uint32_t part[MN];
#pragma unroll
          for (int c = 0; c < MN; c += 16) sm100::tmem_ld_32x32b_x16(t_row + ch * kChainCols + c, part + c);
#pragma unroll
          for (int c = 0; c < MN; c += 16) sm100::tmem_wait_ld_regs16(part + c);
#pragma unroll
          for (int j = 0; j < MN; ++j) acc[j] += part[j];
        }
      }
      // the buffer is in registers: hand it back to the MMA warp
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&bars.acc_empty[b]));
      const bool n_ok = n < p.N && !aborted(bars);
      if (count == p.k_groups) {
        if (n_ok) {
#pragma unroll
          for (int m = 0; m < MN; ++m) {
            if (m < p.M) {
              const float am = MN <= 32 ? sa[m < kSa ? m : 0] : __ldg(&sA[m]);
              C[(int64_t)m * p.ldc + n] = from_f32<OutT>(dequant(acc[m], am, sw));
              if (acc_out) acc_out[(int64_t)m * p.N + n] = (int32_t)acc[m];
            }
          }
        }
      } else {
        // exact int32 partial: red.add, count k tiles on the ticket, the
        // CTA completing the count finishes the tile
        if (n_ok) {
#pragma unroll
          for (int m = 0; m < MN; ++m)
            if (m < p.M) atomicAdd(&ws[(int64_t)m * p.N + n], (int)acc[m]);
        }
        __threadfence();
        named_bar_sync(1, 128);
        if (threadIdx.x == 2 * 32) {
          const int prev = atomicAdd(&tickets[n_tile], count);
          const int last = (prev + count == p.k_groups);
          if (last) atomicExch(&tickets[n_tile], 0);
          bars.flags[1] = last;
        }
        named_bar_sync(1, 128);
        const bool last = bars.flags[1] != 0;
        named_bar_sync(1, 128);  // flags[1] is rewritten by the next segment
        if (last) {
          __threadfence();
          if (n_ok) {
            const float sw_t = __ldg(&sW[n]);
            int32_t v[MN];
#pragma unroll
            for (int m = 0; m < MN; ++m) v[m] = m < p.M ? __ldcg(&ws[(int64_t)m * p.N + n]) : 0;
#pragma unroll
            for (int m = 0; m < MN; ++m) {
              if (m < p.M) {
                ws[(int64_t)m * p.N + n] = 0;  // ready for the next call
                const float am = MN <= 32 ? sa[m < kSa ? m : 0] : __ldg(&sA[m]);
                C[(int64_t)m * p.ldc + n] = from_f32<OutT>(dequant((uint32_t)v[m], am, sw_t));
                if (acc_out) acc_out[(int64_t)m * p.N + n] = v[m];
              }
            }
          }
        }
      }
    }
    sm100::tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 2 * kCols);
  }
}

// ----------------------------------------------------------------------------
// Skinny kernel (M <= 64): C^T tiles [128 n x MN m], split-K
// ----------------------------------------------------------------------------
template <int MN, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    int8_gemm_skinny_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                            const float* __restrict__ sA, const float* __restrict__ sW, OutT* __restrict__ C,
                            int32_t* __restrict__ acc_out, int32_t* __restrict__ ws, int* __restrict__ tickets,
                            GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Bars bars = carve(smem, p);
  const uint32_t base = sm100::smem_u32(smem);
  constexpr int kCols = MN < 32 ? 32 : MN;  // TMEM allocation granularity
  const int n_tile = blockIdx.x, split = blockIdx.y;
  const int kt0 = split * p.k_tiles_split;
  const int nk = max(0, min(p.k_tiles, kt0 + p.k_tiles_split) - kt0);
  if (threadIdx.x == 0) init_bars(bars, p);
  if (warp == 1) {
    sm100::tmem_alloc(sm100::smem_u32(bars.tmem_slot), kCols);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *bars.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_w);
      sm100::tma_prefetch_desc(&tm_a);
      int it = 0;
      Ring r;
      if (!produce(&tm_w, &tm_a, bars, base, p, kt0, nk, n_tile * BM, 0, r, it))
        set_abort(bars, kDevErrTimeoutEmpty);
      drain_fills(bars, p, it);
    }
  } else if (warp == 1) {
    const uint32_t leader = sm100::elect_one();
    Ring r;
    if (!mma_stages<MN>(bars, base, p, tmem, nk, r, leader) && leader) set_abort(bars, kDevErrTimeoutFull);
    sm100::tc_commit(sm100::smem_u32(&bars.acc_full[0]), leader);
  } else {
    const int quarter = warp & 3;
    const int64_t n = (int64_t)n_tile * BM + quarter * 32 + lane;  // output column (TMEM lane)
    const bool ok = sm100::mbar_wait_warp(sm100::smem_u32(&bars.acc_full[0]), 0);
    if (!ok) set_abort(bars, kDevErrTimeoutMma);
    sm100::tc_fence_after();
    uint32_t acc[MN];
#pragma unroll
    for (int c = 0; c < MN; c += 16)
      sm100::tmem_ld_32x32b_x16(tmem + ((uint32_t)(quarter * 32) << 16) + c, acc + c);
#pragma unroll
    for (int c = 0; c < MN; c += 16) sm100::tmem_wait_ld_regs16(acc + c);
    if (nk == 0) {
#pragma unroll
      for (int j = 0; j < MN; ++j) acc[j] = 0;
    }
    const bool n_ok = n < p.N && ok && !aborted(bars);
    if (p.splits == 1) {
      if (n_ok) {
        const float sw = sW[n];
#pragma unroll
        for (int m = 0; m < MN; ++m) {
          if (m < p.M) {
            C[(int64_t)m * p.ldc + n] = from_f32<OutT>(dequant(acc[m], sA[m], sw));
            if (acc_out) acc_out[(int64_t)m * p.N + n] = (int32_t)acc[m];
          }
        }
      }
    } else {
      // exact int32 partial sums: red.add into the tile, ticket, last split finishes
      if (n_ok) {
#pragma unroll
        for (int m = 0; m < MN; ++m)
          if (m < p.M) atomicAdd(&ws[(int64_t)m * p.N + n], (int)acc[m]);
      }
      __threadfence();
      named_bar_sync(1, 128);
      if (threadIdx.x == 2 * 32) {
        const int prev = atomicAdd(&tickets[n_tile], 1);
        const int last = (prev == p.splits - 1);
        if (last) atomicExch(&tickets[n_tile], 0);
        bars.flags[1] = last;
      }
      named_bar_sync(1, 128);
      if (bars.flags[1]) {
        __threadfence();
        if (n_ok) {
          const float sw = sW[n];
#pragma unroll
          for (int m = 0; m < MN; ++m) {
            if (m < p.M) {
              int32_t* cell = &ws[(int64_t)m * p.N + n];
              const int32_t v = __ldcg(cell);
              *cell = 0;  // ready for the next call
              C[(int64_t)m * p.ldc + n] = from_f32<OutT>(dequant((uint32_t)v, sA[m], sw));
              if (acc_out) acc_out[(int64_t)m * p.N + n] = v;
            }
          }
        }
      }
    }
    sm100::tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kCols);
  }
}

struct GemmPlan {
  bool skinny;
  bool stream;     // streaming skinny kernel (one W range per SM)
  int group, k_groups;  // streaming kernel: k tiles per stage, groups per n tile
  bool pair;       // two-SM kernel (256 x 256 tiles per CTA pair)
  int b_box_rows;  // rows of the second operand's TMA box
  int BN;  // persistent tile width, or MN (padded M) for skinny
  int splits, k_tiles, k_tiles_split, stages, m_tiles, n_tiles, grid;
  int full_items, num_items;  // CTA-pair kernel work items (see GemmParams)
  uint32_t stage_bytes, a_bytes;
  size_t smem, ws_bytes;
};

GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, const b200_launch_cfg* cfg, size_t extra_smem = 0) {
  GemmPlan g{};
  g.k_tiles = (int)((K + BK - 1) / BK);
  const int sms = device_sm_count();
  // dynamic shared memory: stages, then the barrier block of carve() (full
  // and empty per stage, 2 + 2 accumulator barriers, mma_done, the TMEM slot
  // and two flags), plus 1 KB of alignment slack
  auto bar_bytes = [](int st) -> size_t { return (size_t)(2 * st + 5) * 8 + 16; };
  g.skinny = M <= 64 && !(cfg && (cfg->flags & 1));  // flags bit 0: force the persistent kernel
  // extra_smem (the staged epilogue's buffers) belongs to the tile kernels only
  if (g.skinny) extra_smem = 0;
  const size_t limit = 227 * 1024 - 1024 - extra_smem;
  if (g.skinny) {
    g.BN = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    g.m_tiles = 1;
    g.n_tiles = (int)((N + BM - 1) / BM);
    g.stream = !(cfg && (cfg->flags & 4));  // flags bit 2: split-grid kernel instead of the streaming one
    int splits = (cfg && cfg->split > 0) ? cfg->split : 0;
    if (splits == 0) {
      splits = 1;
      while (g.n_tiles * splits < sms && splits * 2 <= g.k_tiles) splits *= 2;
    }
    if (splits > g.k_tiles) splits = g.k_tiles;
    g.k_tiles_split = (g.k_tiles + splits - 1) / splits;
    g.splits = (g.k_tiles + g.k_tiles_split - 1) / g.k_tiles_split;
    g.a_bytes = BM * BK;  // W box
    g.stage_bytes = g.a_bytes + g.BN * BK;
    g.grid = g.n_tiles * g.splits;
    if (g.splits > 1) g.ws_bytes = kTicketBytes + (size_t)M * N * 4;
    if (g.stream) {
      // k tiles per stage: tile_k (bytes of K) / 128, default 3 (2 for M > 32):
      // four 55 KB stages in flight (16 x 14336 x 4096 with one n tile per
      // CTA: 16.5 us, against 18.4 us with 2, 4 or 6 tiles per stage)
      int grp = (cfg && cfg->tile_k > 0) ? cfg->tile_k / BK : (g.BN > 32 ? 2 : 3);
      grp = grp < 1 ? 1 : (grp > 8 ? 8 : grp);
      if (grp > g.k_tiles) grp = g.k_tiles;
      // at least two stages must fit in shared memory
      while (grp > 1 && 2 * (size_t)grp * (BM + g.BN) * BK + bar_bytes(2) > limit) --grp;
      g.group = grp;
      g.k_groups = (g.k_tiles + grp - 1) / grp;
      g.a_bytes = (uint32_t)grp * BM * BK;
      g.stage_bytes = (uint32_t)grp * (BM + g.BN) * BK;
      const int64_t units = (int64_t)g.n_tiles * g.k_groups;
      // Default grid: n_tiles x s CTAs, s the largest divisor of the k groups
      // that keeps the grid within the SM count, so every CTA's range is one
      // aligned segment (a whole n tile when s = 1: dequantised directly, no
      // partial exchange).  An even split of the units over all SMs leaves
      // most n tiles in two partials whose int32 exchange (red.add, fence,
      // ticket, last-finisher merge) sits on the kernel's tail: 16 x 14336 x
      // 4096 ran 22.4 us on 148 CTAs, 18.3 us on 112 (one tile each).  With
      // more n tiles than SMs the units are split evenly.  tile_m: CTAs of
      // the grid instead.
      int64_t want = sms;
      if (g.n_tiles <= sms) {
        int split = 1;
        for (int d = 1; d <= g.k_groups; ++d)
          if (g.k_groups % d == 0 && (int64_t)g.n_tiles * d <= sms) split = d;
        want = (int64_t)g.n_tiles * split;
      }
      if (cfg && cfg->tile_m > 0) want = cfg->tile_m;
      g.grid = (int)(units < want ? units : want);
      g.ws_bytes = kTicketBytes + (size_t)M * N * 4;
    }
  } else if (M > 128 && !(cfg && (cfg->flags & 2)) && sms >= 2) {  // flags bit 1: one-SM persistent kernel
    g.pair = true;
    g.m_tiles = (int)((M + 2 * BM - 1) / (2 * BM));
    const int pairs = sms / 2;
    // Tile width: tile_n when it is one of 128..256 (step 32), else the one
    // with the least cost = waves x (width + 224).  A ring stage costs about
    // its MMA time plus a fixed part as long as the MMA time of a 256-wide
    // stage (measured: 4096 x 14336 x 4096 took 168 / 169 / 190 / 211 / 247 us
    // at widths 256 / 224 / 192 / 160 / 128; the ring's bytes in flight are
    // capped by shared memory, and narrow tiles consume them faster), so
    // narrower tiles pay off only where they remove a mostly empty wave.
    // Only 256 and 128 are automatic choices: the staged epilogue writes
    // 128-column groups, and a width with a remainder sends that remainder
    // through per-row stores (to a peer: 16-byte NVLink writes; the fused
    // all-gather GEMM at 4096 x 7168 per rank ran 271 us at 224 against 140
    // at 256).
    int pn = (cfg && cfg->tile_n >= 128 && cfg->tile_n <= 256 && cfg->tile_n % 32 == 0) ? cfg->tile_n : 0;
    if (pn == 0) {
      int64_t best = INT64_MAX;
      for (int cand = kPairN; cand >= 128; cand -= 128) {
        const int64_t t = (int64_t)g.m_tiles * ((N + cand - 1) / cand);
        const int64_t cost = ((t + pairs - 1) / pairs) * (cand + 224);
        if (cost < best) {
          best = cost;
          pn = cand;
        }
      }
    }
    g.BN = pn;
    g.n_tiles = (int)((N + pn - 1) / pn);
    g.splits = 1;
    g.k_tiles_split = g.k_tiles;
    g.a_bytes = BM * BK;                  // this CTA's 128 rows of A
    g.stage_bytes = g.a_bytes + (pn / 2) * BK;  // + its pn / 2 rows of W
    const int64_t tiles = (int64_t)g.m_tiles * g.n_tiles;
    // tile_m: CTA pairs of the grid (default one per two SMs; the tile count
    // gives one tile per pair, no persistence)
    const int64_t want = (cfg && cfg->tile_m > 0) ? cfg->tile_m : pairs;
    g.grid = 2 * (int)(tiles < want ? tiles : want);
    // The last, partial wave of 256-wide tiles runs as 128-wide halves on
    // twice the pairs (4096^3: 34 tiles of the fourth wave on 34 of 74 pairs
    // become 68 halves); flags bit 3 keeps whole tiles.
    const int64_t np = g.grid / 2;
    const int64_t rem = np > 0 ? tiles % np : 0;
    g.full_items = g.num_items = (int)tiles;
    if (pn == kPairN && rem > 0 && tiles > np && 2 * rem <= np && !(cfg && (cfg->flags & 8))) {
      g.full_items = (int)(tiles - rem);
      g.num_items = (int)(tiles + rem);
    }
  } else {
    int bn = (cfg && cfg->tile_n > 0) ? cfg->tile_n : 256;
    if (bn != 128 && bn != 256) bn = 256;
    if (N <= 128) bn = 128;
    g.BN = bn;
    g.m_tiles = (int)((M + BM - 1) / BM);
    g.n_tiles = (int)((N + bn - 1) / bn);
    g.splits = 1;
    g.k_tiles_split = g.k_tiles;
    g.a_bytes = BM * BK;
    g.stage_bytes = g.a_bytes + bn * BK;
    const int64_t tiles = (int64_t)g.m_tiles * g.n_tiles;
    g.grid = (int)(tiles < sms ? tiles : sms);
  }
  g.b_box_rows = g.skinny ? g.BN : (g.pair ? g.BN / 2 : g.BN);
  int stages = (cfg && cfg->stages > 0) ? cfg->stages : (g.stream ? 16 : 8);
  while (stages > 2 && (size_t)stages * g.stage_bytes + bar_bytes(stages) > limit) --stages;
  g.stages = stages;
  g.smem = (size_t)stages * g.stage_bytes + bar_bytes(stages) + 1024 + extra_smem;
  return g;
}

// CTA-pair kernel launch: clusters of two CTAs (cudaLaunchKernelEx).
template <typename OutT, bool kF16>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tbh, const float* sA,
                const float* sW, void* C, int32_t* acc_out, const GemmPlan& g, const GemmParams& p,
                cudaStream_t s) {
  auto kern = int8_gemm_pair_kernel<OutT, kF16, kPairN>;
  if constexpr (!kF16) {
    switch (g.BN) {
      case 128: kern = int8_gemm_pair_kernel<OutT, kF16, 128>; break;
      case 160: kern = int8_gemm_pair_kernel<OutT, kF16, 160>; break;
      case 192: kern = int8_gemm_pair_kernel<OutT, kF16, 192>; break;
      case 224: kern = int8_gemm_pair_kernel<OutT, kF16, 224>; break;
      case 256: break;
      default: return B200_ERR_UNSUPPORTED;
    }
  } else if (g.BN != kPairN) {
    return B200_ERR_UNSUPPORTED;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
  if (e != cudaSuccess) return launch_status(e);
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)g.grid);
  lc.blockDim = dim3(kThreads);
  lc.dynamicSmemBytes = g.smem;
  lc.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  e = cudaLaunchKernelEx(&lc, kern, ta, tb, tbh, sA, sW, static_cast<OutT*>(C), acc_out, p);
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(cudaGetLastError());
}

template <typename OutT>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tbh, const float* sA, const float* sW,
           void* C, int32_t* acc_out, void* ws, const GemmPlan& g, const GemmParams& p, cudaStream_t s) {
  if (g.pair) return launch_pair<OutT, false>(ta, tb, tbh, sA, sW, C, acc_out, g, p, s);
  if (!g.skinny) {
    auto kern = g.BN == 256 ? int8_gemm_tcgen05_kernel<256, OutT> : int8_gemm_tcgen05_kernel<128, OutT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
    if (e != cudaSuccess) return launch_status(e);
    kern<<<g.grid, kThreads, g.smem, s>>>(ta, tb, sA, sW, static_cast<OutT*>(C), acc_out, p);
    return launch_status(cudaGetLastError());
  }
  if (g.stream) {
    auto kern = g.BN == 16 ? int8_gemm_stream_kernel<16, OutT>
                           : (g.BN == 32 ? int8_gemm_stream_kernel<32, OutT> : int8_gemm_stream_kernel<64, OutT>);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
    if (e != cudaSuccess) return launch_status(e);
    int* tickets = static_cast<int*>(ws);
    int32_t* part = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + kTicketBytes);
    kern<<<g.grid, kThreads, g.smem, s>>>(ta, tb, sA, sW, static_cast<OutT*>(C), acc_out, part, tickets, p);
    return launch_status(cudaGetLastError());
  }
  auto sk = g.BN == 16 ? int8_gemm_skinny_kernel<16, OutT>
                       : (g.BN == 32 ? int8_gemm_skinny_kernel<32, OutT> : int8_gemm_skinny_kernel<64, OutT>);
  cudaError_t e = cudaFuncSetAttribute(sk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
  if (e != cudaSuccess) return launch_status(e);
  int* tickets = nullptr;
  int32_t* part = nullptr;
  if (g.splits > 1) {
    tickets = static_cast<int*>(ws);
    part = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + kTicketBytes);
  }
  dim3 grid(g.n_tiles, g.splits);
  sk<<<grid, kThreads, g.smem, s>>>(ta, tb, sA, sW, static_cast<OutT*>(C), acc_out, part, tickets, p);
  return launch_status(cudaGetLastError());
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" size_t b200_int8_gemm_workspace_size(int64_t M, int64_t N, int64_t K, const b200_launch_cfg* cfg) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return plan_gemm(M, N, K, cfg).ws_bytes;
}

namespace b200 {
namespace {

// Destinations of a fused all-gather (world 0: a plain GEMM).
struct Gather {
  int world = 0, self = 0;
  int64_t col_off = 0;
  void* dst[kMaxRanks] = {};
};

int gemm_entry(const int8_t* A, const int8_t* W, const float* sA, const float* sW, void* C, int64_t M, int64_t N,
               int64_t K, int64_t ldc, int32_t out_dtype, int32_t* acc_out, void* workspace, size_t workspace_bytes,
               const b200_launch_cfg* cfg, void* stream, const Gather& ga) {
  if (M < 0 || N < 0 || K < 0) return B200_ERR_BAD_ARG;
  if (M == 0 || N == 0) return B200_OK;
  if (!A || !W || !sA || !sW || !C) return B200_ERR_BAD_ARG;
  if (K == 0 || K % 16 != 0) return B200_ERR_UNSUPPORTED;  // TMA row pitch must be 16-byte aligned
  if (K > 131072) return B200_ERR_UNSUPPORTED;             // int32 accumulator range
  if (ldc < N) return B200_ERR_BAD_ARG;
  if (!aligned16(A) || !aligned16(W)) return B200_ERR_ALIGNMENT;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL) return B200_ERR_UNSUPPORTED;
  // Staged epilogue (16-bit or fp32 outputs of the tile kernels, no raw
  // accumulators, 16-byte aligned scales and output rows): 16 B alignment slack + one
  // staging buffer per epilogue warp.  The fused all-gather falls back to
  // per-row stores into every rank's C where these do not hold.
  const int64_t osz = dtype_size(out_dtype);
  const bool staged = (osz == 2 || osz == 4) && acc_out == nullptr && aligned16(sW) && aligned16(C) &&
                      (ldc * osz) % 16 == 0 && (ga.col_off * osz) % 16 == 0;
  const GemmPlan g = plan_gemm(M, N, K, cfg, staged ? 16 + 4 * kGatherWarpBytes : 0);
  if (g.skinny && (g.splits > 1 || g.stream)) {
    if (workspace == nullptr || workspace_bytes < g.ws_bytes || !aligned16(workspace)) return B200_ERR_WORKSPACE;
    if ((size_t)g.n_tiles * 4 > kTicketBytes) return B200_ERR_UNSUPPORTED;
  }
  if (g.skinny && g.n_tiles > 0x7fffffff / 2) return B200_ERR_UNSUPPORTED;
  // first MMA operand: A (persistent) or W (skinny: operands swapped)
  CUtensorMap ta, tb;
  const int8_t* op0 = g.skinny ? W : A;
  const int8_t* op1 = g.skinny ? A : W;
  const int64_t rows0 = g.skinny ? N : M;
  const int64_t rows1 = g.skinny ? M : N;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)rows0};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {BK, BM};
    int st = encode_tensor_map(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, op0, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)rows1};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {BK, (uint32_t)g.b_box_rows};
    int st = encode_tensor_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, op1, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  // W boxes of the CTA-pair kernel's half-width items (a quarter of the tile's rows per CTA)
  CUtensorMap tbh = tb;
  if (g.pair && g.num_items > g.full_items) {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)rows1};
    const uint64_t strides[1] = {(uint64_t)K};
    const uint32_t box[2] = {BK, (uint32_t)(g.BN / 4)};
    int st = encode_tensor_map(&tbh, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, op1, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  GemmParams p{};
  p.world = ga.world;
  p.self = ga.self;
  p.col_off = ga.col_off;
  for (int r = 0; r < kMaxRanks; ++r) p.dst[r] = ga.dst[r];
  p.staged = staged && !g.skinny;
  p.full_items = g.pair ? g.full_items : 0;
  p.num_items = g.pair ? g.num_items : 0;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.k_tiles = g.k_tiles;
  p.k_tiles_split = g.k_tiles_split;
  p.splits = g.splits;
  p.stages = g.stages;
  p.m_tiles = g.m_tiles;
  p.n_tiles = g.n_tiles;
  p.num_tiles = g.m_tiles * g.n_tiles;
  p.stage_bytes = g.stage_bytes;
  p.a_bytes = g.a_bytes;
  p.group = g.group;
  p.k_groups = g.k_groups;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (out_dtype) {
    case B200_F16: return launch<__half>(ta, tb, tbh, sA, sW, C, acc_out, workspace, g, p, s);
    case B200_BF16: return launch<__nv_bfloat16>(ta, tb, tbh, sA, sW, C, acc_out, workspace, g, p, s);
    case B200_F32: return launch<float>(ta, tb, tbh, sA, sW, C, acc_out, workspace, g, p, s);
    default: return B200_ERR_UNSUPPORTED;
  }
}

// Cross-GPU flag exchange of the fused all-gather GEMM.  Each rank's flag
// array holds 2 * world uint32: entries [0, world) are "done" flags (rank r's
// columns of this call are in my C) and entries [world, 2 * world) are
// "ready" flags (rank r has reached this call, so everything its stream ran
// before it -- including its reads of the previous call's C -- is finished).
// Thread r stores `epoch` into rank r's array at index base + self (release
// store at system scope), then waits, bounded by `timeout_ns` of global time,
// until entry base + r of this rank's own array has reached `epoch`.  On
// expiry it records `err_code` in the device error word and returns.
__global__ void __launch_bounds__(32) peer_flag_exchange_kernel(Gather flags, int world, int self, int base,
                                                                 uint32_t epoch, uint64_t timeout_ns,
                                                                 int err_code) {
  const int r = threadIdx.x;
  if (r >= world) return;
  uint32_t* mine = static_cast<uint32_t*>(flags.dst[self]) + base;
  uint32_t* theirs = static_cast<uint32_t*>(flags.dst[r]) + base;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(theirs + self), "r"(epoch) : "memory");
  const uint64_t t0 = sm100::global_timer_ns();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + r) : "memory");
    if ((int32_t)(v - epoch) >= 0) break;
    if (sm100::global_timer_ns() - t0 > timeout_ns) {
      b200_dev_error(err_code);
      break;
    }
    __nanosleep(64);
  }
}

}  // namespace
}  // namespace b200

extern "C" int b200_int8_gemm(const int8_t* A, const int8_t* W, const float* sA, const float* sW, void* C,
                              int64_t M, int64_t N, int64_t K, int64_t ldc, int32_t out_dtype,
                              int32_t* acc_out, void* workspace, size_t workspace_bytes,
                              const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("int8_gemm")) return e;
  return gemm_entry(A, W, sA, sW, C, M, N, K, ldc, out_dtype, acc_out, workspace, workspace_bytes, cfg, stream,
                    Gather{});
}

extern "C" int b200_int8_gemm_allgather(const int8_t* A, const int8_t* W_local, const float* sA,
                                        const float* sW_local, void* const* C_ranks, uint32_t* const* sig_ranks,
                                        int32_t world, int32_t rank, int64_t M, int64_t n_local, int64_t col0,
                                        int64_t K, int64_t ldc, int32_t out_dtype, uint32_t epoch, void* workspace,
                                        size_t workspace_bytes, const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("int8_gemm_allgather")) return e;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || epoch == 0) return B200_ERR_BAD_ARG;
  if (!C_ranks || !sig_ranks || col0 < 0 || n_local < 0 || col0 + n_local > ldc) return B200_ERR_BAD_ARG;
  Gather ga, fl;
  ga.world = world;
  ga.self = rank;
  ga.col_off = col0;
  fl.world = world;
  fl.self = rank;
  for (int r = 0; r < world; ++r) {
    if (!C_ranks[r] || !sig_ranks[r] || !aligned16(C_ranks[r])) return B200_ERR_BAD_ARG;
    ga.dst[r] = C_ranks[r];
    fl.dst[r] = sig_ranks[r];
  }
  // the multi-destination epilogue belongs to the tile kernels: small M
  // runs the persistent one-SM kernel (flags bit 0) instead of the swap-AB ones
  b200_launch_cfg c = cfg ? *cfg : b200_launch_cfg{};
  c.flags |= 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t timeout_ns = peer_wait_timeout_ns();
  // Nobody writes into a peer's C before that peer has reached this call: its
  // stream has then finished whatever read the previous call's result.
  peer_flag_exchange_kernel<<<1, 32, 0, s>>>(fl, world, rank, world, epoch, timeout_ns, kDevErrTimeoutPeer);
  if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) return launch_status(e);
  if (M > 0 && n_local > 0) {
    const int st = gemm_entry(A, W_local, sA, sW_local, C_ranks[rank], M, n_local, K, ldc, out_dtype, nullptr,
                              workspace, workspace_bytes, &c, stream, ga);
    if (st != B200_OK) return st;
  }
  // Every rank's columns have landed in this rank's C when this one returns.
  peer_flag_exchange_kernel<<<1, 32, 0, s>>>(fl, world, rank, 0, epoch, timeout_ns, kDevErrTimeoutPeer);
  return launch_status(cudaGetLastError());
}


// ---------------------------------------------------------------------------
// bf16/fp16 GEMM + bias + GELU (matmul_epilogue): the CTA-pair kernel's
// kind::f16 flavour.
// ---------------------------------------------------------------------------
extern "C" int b200_gemm_bias_gelu(const void* a, const void* b, const void* bias, void* c, int64_t M, int64_t N,
                                   int64_t K, int32_t dtype, const b200_launch_cfg* cfg, void* stream) {
  using namespace b200;
  if (int e = injected_error("gemm_bias_gelu")) return e;
  if (M < 0 || N < 0 || K < 0) return B200_ERR_BAD_ARG;
  if (M == 0 || N == 0) return B200_OK;
  if (!a || !b || !bias || !c || K == 0) return B200_ERR_BAD_ARG;
  if (dtype != B200_BF16 && dtype != B200_F16) return B200_ERR_UNSUPPORTED;
  if (K % 8 != 0 || N % 8 != 0) return B200_ERR_UNSUPPORTED;  // 16-byte TMA row pitches
  if (!aligned16(a) || !aligned16(b) || !aligned16(c)) return B200_ERR_ALIGNMENT;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL) return B200_ERR_UNSUPPORTED;
  const int sms = device_sm_count();
  if (sms < 2) return B200_ERR_NO_DEVICE;
  GemmPlan g{};
  g.pair = true;
  g.BN = kPairN;
  g.k_tiles = (int)((K + 63) / 64);  // 64 elements (128 B) of K per stage
  g.m_tiles = (int)((M + 2 * BM - 1) / (2 * BM));
  g.n_tiles = (int)((N + kPairN - 1) / kPairN);
  g.splits = 1;
  g.k_tiles_split = g.k_tiles;
  g.a_bytes = BM * 128;
  g.stage_bytes = g.a_bytes + 2 * 8192;
  const int64_t tiles = (int64_t)g.m_tiles * g.n_tiles;
  g.grid = 2 * (int)(tiles < sms / 2 ? tiles : sms / 2);
  // shared memory as in plan_gemm: stages, carve()'s barrier block, 1 KB alignment slack
  auto bar_bytes = [](int st) -> size_t { return (size_t)(2 * st + 5) * 8 + 16; };
  int stages = (cfg && cfg->stages > 0) ? cfg->stages : 8;
  while (stages > 2 && (size_t)stages * g.stage_bytes + bar_bytes(stages) > 227 * 1024 - 1024) --stages;
  g.stages = stages;
  g.smem = (size_t)stages * g.stage_bytes + bar_bytes(stages) + 1024;
  const CUtensorMapDataType dt = dtype == B200_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {64, BM};
    if (int st = encode_tensor_map(&ta, dt, 2, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)N * 2};
    const uint32_t box[2] = {64, 64};
    if (int st = encode_tensor_map(&tb, dt, 2, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = N;
  p.k_tiles = g.k_tiles;
  p.k_tiles_split = g.k_tiles;
  p.splits = 1;
  p.stages = g.stages;
  p.m_tiles = g.m_tiles;
  p.n_tiles = g.n_tiles;
  p.num_tiles = g.m_tiles * g.n_tiles;
  p.full_items = p.num_items = p.num_tiles;  // whole tiles only
  p.stage_bytes = g.stage_bytes;
  p.a_bytes = g.a_bytes;
  p.bias = bias;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == B200_BF16) return launch_pair<__nv_bfloat16, true>(ta, tb, tb, nullptr, nullptr, c, nullptr, g, p, s);
  return launch_pair<__half, true>(ta, tb, tb, nullptr, nullptr, c, nullptr, g, p, s);
}
