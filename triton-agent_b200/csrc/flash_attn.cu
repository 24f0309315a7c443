// Flash attention forward (prefill), bf16/fp16, fp32 softmax statistics, on
// the 5th-generation tensor cores (tcgen05.mma kind::f16, accumulators in
// tensor memory).
//
// Reference: triton_agent/ops/flash_attn_like/reference.py:22-31
//   scores = q k^T / sqrt(D); causal: key s > query t masked (tril mask);
//   out = softmax(scores) v
//
// One CTA per (128 query rows, b*h).  Warp roles (192 threads):
//   warp 0      TMA producer: Q tile once; K and V tiles of 128 keys into a
//               2-stage ring (3-D tensor maps [B*H, T, D], SWIZZLE_128B,
//               boxes of 64 head dims, so every row / key past the end of a
//               head reads zeros instead of the next head)
//   warp 1      allocates 512 TMEM columns (S double buffer 2x128, O 128 or
//               64); one lane issues S_j = Q K_j^T (kind::f16, M=128, N=128,
//               K=16 steps) ahead of the softmax, then O += P_j V_j with P
//               from shared memory (K-major) and V as an MN-major operand
//   warps 2..5  softmax: each thread owns one query row (TMEM lane), loads
//               its 128 scores, masks (causal diagonal / key tail), keeps a
//               running max that is only raised when it grows by more than
//               2^8 (then O is rescaled in TMEM), writes P = exp2(s - m) as
//               bf16 into a SWIZZLE_128B K-major tile, and finally divides O
//               by the row sum and stores the output row.
// The running-max rule is exact: O and l share the same offset, which
// cancels in O / l; it only bounds P <= 2^8.  Causal CTAs are launched
// heaviest-first (last query tiles first) to shorten the tail.  No cluster
// multicast is used.
#include <math.h>

#include <atomic>

#include "common.cuh"
#include "sm100.cuh"

B200_DEVICE_ERROR_WORD()

namespace b200 {
namespace {

constexpr int kBM = 128;   // query rows per CTA
constexpr int kBN = 128;   // keys per tile
constexpr int kThreads = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FlashParams {
  int64_t B, H, T, S;
  int n_qt;         // query tiles
  float sl2;        // scale * log2(e)
  int causal;
  int out_lse;
  int poly_exp;     // unmasked exponentials partly on the FMA pipe
  int head_group;   // heads per CTA scheduling group (three-warpgroup kernel)
  int poly_pairs;   // of every 8 exponential pairs, how many on the FMA pipe (three-warpgroup kernel)
};

template <int D>
struct FlashSmem {
  static constexpr uint32_t kHalf = kBM * 128;          // one 64-dim box: 128 rows x 128 B
  static constexpr uint32_t kQ = (D / 64) * kHalf;       // Q tile
  static constexpr uint32_t kKV = (D / 64) * kHalf;      // K or V tile (128 keys)
  static constexpr uint32_t kP = 2 * kHalf;              // P tile 128 x 128 bf16
  static constexpr uint32_t oQ = 0;
  static constexpr uint32_t oK0 = oQ + kQ;
  static constexpr uint32_t oV0 = oK0 + kKV;
  static constexpr uint32_t oK1 = oV0 + kKV;
  static constexpr uint32_t oV1 = oK1 + kKV;
  static constexpr uint32_t oP = oV1 + kKV;
  static constexpr uint32_t oBar = oP + kP;
  static constexpr uint32_t kTotal = oBar + 256 + 1024;  // + barriers + alignment slack
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// 2^x with the MUFU approximation (PTX ex2.approx.ftz.f32); 2^-inf = 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, to share the softmax's exponentials with the MUFU
// unit: x = n + f with n = round(x) (adding 1.5 * 2^23 rounds to an integer,
// exact for |x| < 2^22) and f in [-0.5, 0.5]; 2^f by the cubic
// 1 + f(c1 + f(c2 + f c3)) fitted in this project by least squares on the
// relative error (max 1.2e-4, well below the bf16 rounding P gets next);
// 2^n is added to the exponent field.  Inputs are clamped to >= -126.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = x + 12582912.0f;
  const int n = __float_as_int(t) - 0x4B400000;
  const float f = x - (t - 12582912.0f);
  const float p = fmaf(fmaf(fmaf(0.0545928263f, f, 0.242218109f), f, 0.693368645f), f, 1.0f);
  return __int_as_float(__float_as_int(p) + (n << 23));
}

// Two lanes of ex2_poly with packed fp32x2 arithmetic: the clamp, the
// rounding split x = n + f, the cubic in f, and 2^n added to the exponent
// field (t's low bits hold n + 1.5 * 2^23, whose excess vanishes when
// shifted left by 23 modulo 2^32).
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& p0, float& p1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  x0 = fmaxf(x0, -126.0f);
  x1 = fmaxf(x1, -126.0f);
  float t0, t1, r0, r1, f0, f1, q0, q1;
  sm100::ffma2_bcast(t0, t1, x0, x1, 1.0f, kMagic);
  sm100::ffma2_bcast(r0, r1, t0, t1, 1.0f, -kMagic);
  sm100::ffma2(f0, f1, r0, r1, -1.0f, -1.0f, x0, x1);
  sm100::ffma2_bcast(q0, q1, f0, f1, 0.0545928263f, 0.242218109f);
  sm100::ffma2(q0, q1, q0, q1, f0, f1, 0.693368645f, 0.693368645f);
  sm100::ffma2(q0, q1, q0, q1, f0, f1, 1.0f, 1.0f);
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, T* __restrict__ out,
                             float* __restrict__ lse, FlashParams p) {
  using L = FlashSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = sm100::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int qt = p.n_qt - 1 - (int)blockIdx.y;  // heaviest query tiles first
  const int64_t q0 = (int64_t)qt * kBM;
  const int n_kt_all = (int)((p.S + kBN - 1) / kBN);
  const int n_kt = p.causal ? min(n_kt_all, (int)((q0 + kBM + kBN - 1) / kBN)) : n_kt_all;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* v_full = bars + 3;     // [2]
  uint64_t* kv_empty = bars + 5;   // [2]
  uint64_t* s_full = bars + 7;     // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* o_done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    sm100::mbar_init(sm100::smem_u32(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(sm100::smem_u32(&k_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&v_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&kv_empty[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&s_full[i]), 1);
    }
    sm100::mbar_init(sm100::smem_u32(p_full), 4);
    sm100::mbar_init(sm100::smem_u32(o_done), 1);
    *s_abort = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_q);
      sm100::tma_prefetch_desc(&tm_k);
      sm100::tma_prefetch_desc(&tm_v);
      const uint32_t qb = sm100::smem_u32(q_full);
      sm100::mbar_arrive_expect_tx(qb, L::kQ);
#pragma unroll
      for (int h = 0; h < D / 64; ++h)
        sm100::tma_load_3d(sbase + L::oQ + h * L::kHalf, &tm_q, qb, h * 64, (int32_t)q0, bh);
      int issued = 0;
      for (int j = 0; j < n_kt; ++j) {
        const int s = j & 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&kv_empty[s]), ((j >> 1) & 1) ^ 1)) {
          b200_dev_error(kDevErrTimeoutEmpty);
          atomicExch(s_abort, 1);
          break;
        }
        if (*(volatile int*)s_abort) break;
        const uint32_t kb = sm100::smem_u32(&k_full[s]);
        const uint32_t vb = sm100::smem_u32(&v_full[s]);
        const uint32_t ko = s ? L::oK1 : L::oK0;
        const uint32_t vo = s ? L::oV1 : L::oV0;
        sm100::mbar_arrive_expect_tx(kb, L::kKV);
#pragma unroll
        for (int h = 0; h < D / 64; ++h)
          sm100::tma_load_3d(sbase + ko + h * L::kHalf, &tm_k, kb, h * 64, j * kBN, bh);
        sm100::mbar_arrive_expect_tx(vb, L::kKV);
#pragma unroll
        for (int h = 0; h < D / 64; ++h)
          sm100::tma_load_3d(sbase + vo + h * L::kHalf, &tm_v, vb, h * 64, j * kBN, bh);
        ++issued;
      }
      // drain: never exit with bulk copies landing in shared memory
      if (!sm100::mbar_wait(sm100::smem_u32(q_full), 0)) b200_dev_error(kDevErrTimeoutFull);
      for (int j = issued - 1; j >= 0 && j >= issued - 2; --j) {
        const int s = j & 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&k_full[s]), (j >> 1) & 1)) b200_dev_error(kDevErrTimeoutFull);
        if (!sm100::mbar_wait(sm100::smem_u32(&v_full[s]), (j >> 1) & 1)) b200_dev_error(kDevErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_s = sm100::make_idesc(1, fmt, fmt, 0, 0, kBM, kBN);
      constexpr uint32_t idesc_o = sm100::make_idesc(1, fmt, fmt, 0, 1, kBM, D);
      bool ok = sm100::mbar_wait(sm100::smem_u32(q_full), 0);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&k_full[s]), (j >> 1) & 1)) return false;
        sm100::tc_fence_after();
        const uint32_t kbase = sbase + (s ? L::oK1 : L::oK0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kHalf + (kk & 3) * 32;
          const uint64_t ad = sm100::make_smem_desc(sbase + L::oQ + off, 16, 1024, sm100::kSwizzle128B);
          const uint64_t bd = sm100::make_smem_desc(kbase + off, 16, 1024, sm100::kSwizzle128B);
          sm100::mma_f16_ss(tS[s], ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        sm100::tc_commit(sm100::smem_u32(&s_full[s]));
        return true;
      };
      if (ok && n_kt > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n_kt; ++j) {
        const int s = j & 1;
        if (*(volatile int*)s_abort) {
          ok = false;
          break;
        }
        if (j + 1 < n_kt && !(ok = issue_s(j + 1))) break;
        if (!sm100::mbar_wait(sm100::smem_u32(p_full), j & 1) ||
            !sm100::mbar_wait(sm100::smem_u32(&v_full[s]), (j >> 1) & 1)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t vbase = sbase + (s ? L::oV1 : L::oV0);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // P: K-major, keys 64*(kk/4).. in box kk/4, 32-byte step inside it.
          const uint64_t ad = sm100::make_smem_desc(sbase + L::oP + (kk >> 2) * L::kHalf + (kk & 3) * 32, 16,
                                                    1024, sm100::kSwizzle128B);
          // V: MN-major; 16 keys = two 8-row groups of 128 B (SBO 1024),
          // head-dim halves 64 apart live one box (16 KB) apart (LBO).
          const uint64_t bd = sm100::make_smem_desc(vbase + kk * 2048, L::kHalf, 1024, sm100::kSwizzle128B);
          sm100::mma_f16_ss(tO, ad, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        sm100::tc_commit(sm100::smem_u32(o_done));
        sm100::tc_commit(sm100::smem_u32(&kv_empty[s]));
      }
      if (!ok) {
        b200_dev_error(kDevErrTimeoutFull);
        atomicExch(s_abort, 1);
        // all issued MMAs must finish before TMEM is released
        sm100::tc_commit(sm100::smem_u32(o_done));
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;          // row inside the tile = TMEM lane
    const int64_t qrow = q0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      const int s = j & 1;
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&s_full[s]), (j >> 1) & 1)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      uint32_t sr[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) sm100::tmem_ld_32x32b_x32(tS[s] + lane_off + c * 32, sr + c * 32);
      sm100::tmem_wait_ld();
      const int64_t k0 = (int64_t)j * kBN;
      const bool need_mask = (k0 + kBN > p.S) || (p.causal && k0 + kBN - 1 > qrow);
      if (need_mask) {
        // keys past the end or (causal) after this query row drop out
        const int64_t lim = (p.causal && qrow + 1 < p.S) ? qrow + 1 : p.S;
        const int64_t nv = lim - k0;
        const int valid = nv <= 0 ? 0 : (nv >= kBN ? kBN : (int)nv);
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (c >= valid) sr[c] = __float_as_uint(-INFINITY);
      }
      // row max of the raw scores: 8 independent chains
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = __uint_as_float(sr[i]);
#pragma unroll
      for (int c = 8; c < kBN; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(sr[c]));
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * p.sl2;
      float alpha = 1.f;
      bool rescale = false;
      if (m_used == -INFINITY) {
        m_used = mx;
      } else if (mx > m_used + kRescaleThreshold) {
        alpha = ex2_approx(m_used - mx);
        m_used = mx;
        rescale = true;
      }
      // p = 2^(s * scale * log2 e - m): one FMA and one ex2 per score
      const float neg_m = -m_used;
      float sum8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum8[i] = 0.f;
      uint32_t pk[kBN / 2];
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(sr[c]), p.sl2, neg_m));
        const float p1 = ex2_approx(fmaf(__uint_as_float(sr[c + 1]), p.sl2, neg_m));
        sum8[(c >> 1) & 7] += p0 + p1;
        pk[c / 2] = pack2<T>(p0, p1);
      }
      const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      l = l * alpha + sum;
      // PV_{j-1} must be complete before P is overwritten or O is rescaled.
      if (j > 0 && !sm100::mbar_wait_warp(sm100::smem_u32(o_done), (j - 1) & 1)) {
        ok = false;
        break;
      }
      if (__any_sync(0xffffffffu, rescale)) {
        sm100::tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t o[32];
          sm100::tmem_ld_32x32b_x32(tO + lane_off + c, o);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          sm100::tmem_st_32x32b_x16(tO + lane_off + c, o);
          sm100::tmem_st_32x32b_x16(tO + lane_off + c + 16, o + 16);
        }
        sm100::tmem_wait_st();
      }
      // P row r -> K-major SWIZZLE_128B tile: keys [64h, 64h+64) in box h,
      // row r at (r/8)*1024 + (r%8)*128, 16-byte chunk c at (c ^ (r%8))*16.
      const uint32_t prow = sbase + L::oP + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* v = pk + h * 32 + c * 4;
          sts128(prow + h * L::kHalf + ((c ^ (r & 7)) << 4), v[0], v[1], v[2], v[3]);
        }
      sm100::fence_proxy_async_smem();  // generic-proxy P stores -> tensor-core reads
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(p_full));
    }
    // epilogue
    if (ok && n_kt > 0 && !sm100::mbar_wait_warp(sm100::smem_u32(o_done), (n_kt - 1) & 1)) ok = false;
    if (!ok) {
      b200_dev_error(kDevErrTimeoutMma);
      atomicExch(s_abort, 1);
    }
    sm100::tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const bool row_ok = qrow < p.T;
    T* orow = out + ((int64_t)bh * p.T + qrow) * D;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t o[32];
      sm100::tmem_ld_32x32b_x32(tO + lane_off + c, o);
      sm100::tmem_wait_ld();
      if (row_ok && ok) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack2<T>(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
          w.y = pack2<T>(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
          w.z = pack2<T>(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
          w.w = pack2<T>(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c + 8 * v) = w;
        }
      }
    }
    if (p.out_lse && row_ok) lse[(int64_t)bh * p.T + qrow] = (m_used + log2f(l)) * 0.6931471805599453f;
    sm100::tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Two-tile kernel: 256 query rows per CTA as tiles A and B that share every
// K/V tile (half the shared-memory operand traffic per FLOP of the one-tile
// kernel), with P kept in tensor memory.
//
// TMEM (512 columns): S_A [0,128), S_B [128,256), O_A [256, 256+D),
// O_B [384, 384+D).  P_t is written as bf16 pairs into the first 64 columns
// of S_t and read back as the A operand of O_t += P_t V (tcgen05.mma with A
// from tensor memory), so no P tile lives in shared memory.
// Warps: 0 TMA producer, 1 MMA issue + TMEM allocation, 2-3 idle, 4-7 softmax
// of tile A, 8-11 softmax of tile B (warp w reads TMEM lanes 32*(w%4)..).
// The MMA thread issues S_A(j), S_B(j), then alternates PV_A(j), S_A(j+1),
// PV_B(j), S_B(j+1): while one softmax warpgroup turns S into P, the tensor
// core works on the other tile.  tcgen05.mma ops of one thread complete in
// issue order, so the completion of S_t(j) (the s_full barrier) also means
// PV_t(j-1) is done -- O_t may be rescaled and P_t overwritten.
// ---------------------------------------------------------------------------
constexpr int kThreads2 = 384;

template <int D>
struct Flash2Smem {
  static constexpr uint32_t kHalf = kBM * 128;         // one 64-dim box of 128 rows
  static constexpr uint32_t kTile = (D / 64) * kHalf;  // Q, K or V tile
  static constexpr uint32_t oQA = 0;
  static constexpr uint32_t oQB = oQA + kTile;
  static constexpr uint32_t oK0 = oQB + kTile;
  static constexpr uint32_t oV0 = oK0 + kTile;
  static constexpr uint32_t oK1 = oV0 + kTile;
  static constexpr uint32_t oV1 = oK1 + kTile;
  static constexpr uint32_t oBar = oV1 + kTile;
  static constexpr uint32_t kTotal = oBar + 256 + 1024;
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads2, 1)
    flash_fwd2_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v, T* __restrict__ out, float* __restrict__ lse,
                              FlashParams p) {
  using L = Flash2Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = sm100::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int n_ct = (int)((p.T + 2 * kBM - 1) / (2 * kBM));
  const int ct = n_ct - 1 - (int)blockIdx.y;  // heaviest first
  const int64_t q0 = (int64_t)ct * 2 * kBM;
  const int n_kt_all = (int)((p.S + kBN - 1) / kBN);
  // key tiles each query tile needs (causal: up to its diagonal)
  int n_kt[2];
  for (int t = 0; t < 2; ++t) {
    const int64_t last_row = q0 + (t + 1) * kBM - 1;
    n_kt[t] = p.causal ? min(n_kt_all, (int)(last_row / kBN) + 1) : n_kt_all;
  }
  const int n_kt_max = n_kt[0] > n_kt[1] ? n_kt[0] : n_kt[1];

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2 tiles]
  uint64_t* p_full = bars + 9;    // [2 tiles]
  uint64_t* o_done = bars + 11;   // [2 tiles]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    sm100::mbar_init(sm100::smem_u32(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(sm100::smem_u32(&k_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&v_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&kv_empty[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&s_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&p_full[i]), 4);
      sm100::mbar_init(sm100::smem_u32(&o_done[i]), 1);
    }
    *s_abort = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO[2] = {tmem + 256, tmem + 384};

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_q);
      sm100::tma_prefetch_desc(&tm_k);
      sm100::tma_prefetch_desc(&tm_v);
      const uint32_t qb = sm100::smem_u32(q_full);
      sm100::mbar_arrive_expect_tx(qb, 2 * L::kTile);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < D / 64; ++h)
          sm100::tma_load_3d(sbase + (t ? L::oQB : L::oQA) + h * L::kHalf, &tm_q, qb, h * 64,
                             (int32_t)(q0 + t * kBM), bh);
      int issued = 0;
      for (int j = 0; j < n_kt_max; ++j) {
        const int s = j & 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&kv_empty[s]), ((j >> 1) & 1) ^ 1)) {
          b200_dev_error(kDevErrTimeoutEmpty);
          atomicExch(s_abort, 1);
          break;
        }
        if (*(volatile int*)s_abort) break;
        const uint32_t kb = sm100::smem_u32(&k_full[s]);
        const uint32_t vb = sm100::smem_u32(&v_full[s]);
        sm100::mbar_arrive_expect_tx(kb, L::kTile);
#pragma unroll
        for (int h = 0; h < D / 64; ++h)
          sm100::tma_load_3d(sbase + (s ? L::oK1 : L::oK0) + h * L::kHalf, &tm_k, kb, h * 64, j * kBN, bh);
        sm100::mbar_arrive_expect_tx(vb, L::kTile);
#pragma unroll
        for (int h = 0; h < D / 64; ++h)
          sm100::tma_load_3d(sbase + (s ? L::oV1 : L::oV0) + h * L::kHalf, &tm_v, vb, h * 64, j * kBN, bh);
        ++issued;
      }
      if (!sm100::mbar_wait(sm100::smem_u32(q_full), 0)) b200_dev_error(kDevErrTimeoutFull);
      for (int j = issued - 1; j >= 0 && j >= issued - 2; --j) {
        const int s = j & 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&k_full[s]), (j >> 1) & 1)) b200_dev_error(kDevErrTimeoutFull);
        if (!sm100::mbar_wait(sm100::smem_u32(&v_full[s]), (j >> 1) & 1)) b200_dev_error(kDevErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_s = sm100::make_idesc(1, fmt, fmt, 0, 0, kBM, kBN);
      constexpr uint32_t idesc_o = sm100::make_idesc(1, fmt, fmt, 0, 1, kBM, D);
      bool ok = sm100::mbar_wait(sm100::smem_u32(q_full), 0);
      auto issue_s = [&](int t, int j) -> bool {
        const int s = j & 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&k_full[s]), (j >> 1) & 1)) return false;
        sm100::tc_fence_after();
        const uint32_t kbase = sbase + (s ? L::oK1 : L::oK0);
        const uint32_t qbase = sbase + (t ? L::oQB : L::oQA);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kHalf + (kk & 3) * 32;
          const uint64_t ad = sm100::make_smem_desc(qbase + off, 16, 1024, sm100::kSwizzle128B);
          const uint64_t bd = sm100::make_smem_desc(kbase + off, 16, 1024, sm100::kSwizzle128B);
          sm100::mma_f16_ss(tS[t], ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        sm100::tc_commit(sm100::smem_u32(&s_full[t]));
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {
        const int s = j & 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&p_full[t]), j & 1)) return false;
        if (!sm100::mbar_wait(sm100::smem_u32(&v_full[s]), (j >> 1) & 1)) return false;
        sm100::tc_fence_after();
        const uint32_t vbase = sbase + (s ? L::oV1 : L::oV0);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // V: MN-major; 16 keys = two 8-row groups of 128 B (SBO 1024),
          // head-dim halves one box (16 KB) apart (LBO).  P: 8 TMEM columns
          // of bf16 pairs per 16 keys.
          const uint64_t bd = sm100::make_smem_desc(vbase + kk * 2048, L::kHalf, 1024, sm100::kSwizzle128B);
          sm100::mma_f16_ts(tO[t], tS[t] + kk * 8, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        return true;
      };
      for (int t = 0; t < 2 && ok; ++t)
        if (n_kt[t] > 0) ok = issue_s(t, 0);
      for (int j = 0; ok && j < n_kt_max; ++j) {
        if (*(volatile int*)s_abort) {
          ok = false;
          break;
        }
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= n_kt[t]) continue;
          ok = issue_pv(t, j);
          if (ok && j + 1 < n_kt[t]) ok = issue_s(t, j + 1);
          if (ok && j + 1 == n_kt[t]) sm100::tc_commit(sm100::smem_u32(&o_done[t]));
        }
        if (ok) sm100::tc_commit(sm100::smem_u32(&kv_empty[j & 1]));
      }
      if (!ok) {
        b200_dev_error(kDevErrTimeoutFull);
        atomicExch(s_abort, 1);
        for (int t = 0; t < 2; ++t) sm100::tc_commit(sm100::smem_u32(&o_done[t]));
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- softmax
    const int t = (warp >> 2) - 1;  // tile of this warpgroup
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int64_t qrow = q0 + t * kBM + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tSt = tS[t] + lane_off, tOt = tO[t] + lane_off;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    const int nj = n_kt[t];
    for (int j = 0; j < nj; ++j) {
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&s_full[t]), j & 1)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const int64_t k0 = (int64_t)j * kBN;
      int valid = kBN;
      if ((k0 + kBN > p.S) || (p.causal && k0 + kBN - 1 > qrow)) {
        const int64_t lim = (p.causal && qrow + 1 < p.S) ? qrow + 1 : p.S;
        const int64_t nv = lim - k0;
        valid = nv <= 0 ? 0 : (nv >= kBN ? kBN : (int)nv);
      }
      const bool full_tile = __all_sync(0xffffffffu, valid == kBN) != 0;
      // pass 1: row max of the raw scores
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t v[32];
        sm100::tmem_ld_32x32b_x32(tSt + c * 32, v);
        sm100::tmem_wait_ld();
        if (full_tile) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(v[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x = (c * 32 + i < valid) ? __uint_as_float(v[i]) : -INFINITY;
            mx8[i & 7] = fmaxf(mx8[i & 7], x);
          }
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * p.sl2;
      float alpha = 1.f;
      bool rescale = false;
      if (m_used == -INFINITY) {
        m_used = mx;
      } else if (mx > m_used + kRescaleThreshold) {
        alpha = ex2_approx(m_used - mx);
        m_used = mx;
        rescale = true;
      }
      // O_t holds PV_t(j-1), complete because S_t(j) is: rescale it if the max moved
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t o[32];
          sm100::tmem_ld_32x32b_x32(tOt + c, o);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          sm100::tmem_st_32x32b_x16(tOt + c, o);
          sm100::tmem_st_32x32b_x16(tOt + c + 16, o + 16);
        }
      }
      // pass 2: P = 2^(s * scale * log2 e - m) as bf16 pairs over the S columns
      const float neg_m = -m_used;
      float sum8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum8[i] = 0.f;
      if (full_tile) {
        // no masked key in this tile for any lane of the warp (the branch must
        // be warp-uniform: both sides issue .sync.aligned tensor-memory loads
        // and stores); optionally half of the exponentials on the FMA pipe
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t v[32];
          sm100::tmem_ld_32x32b_x32(tSt + c * 32, v);
          sm100::tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(v[i]), p.sl2, neg_m));
            const float x1 = fmaf(__uint_as_float(v[i + 1]), p.sl2, neg_m);
            const float p1 = p.poly_exp ? ex2_poly(x1) : ex2_approx(x1);
            sum8[(i >> 1) & 7] += p0 + p1;
            pk[i >> 1] = pack2<T>(p0, p1);
          }
          sm100::tmem_st_32x32b_x16(tSt + c * 16, pk);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t v[32];
          sm100::tmem_ld_32x32b_x32(tSt + c * 32, v);
          sm100::tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float p0 = (c * 32 + i < valid) ? ex2_approx(fmaf(__uint_as_float(v[i]), p.sl2, neg_m)) : 0.f;
            const float p1 =
                (c * 32 + i + 1 < valid) ? ex2_approx(fmaf(__uint_as_float(v[i + 1]), p.sl2, neg_m)) : 0.f;
            sum8[(i >> 1) & 7] += p0 + p1;
            pk[i >> 1] = pack2<T>(p0, p1);
          }
          sm100::tmem_st_32x32b_x16(tSt + c * 16, pk);
        }
      }
      sm100::tmem_wait_st();
      l = l * alpha + (((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7])));
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&p_full[t]));
    }
    // epilogue: O_t / l
    if (ok && nj > 0 && !sm100::mbar_wait_warp(sm100::smem_u32(&o_done[t]), 0)) ok = false;
    if (!ok) {
      b200_dev_error(kDevErrTimeoutMma);
      atomicExch(s_abort, 1);
    }
    sm100::tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const bool row_ok = qrow < p.T;
    T* orow = out + ((int64_t)bh * p.T + qrow) * D;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t o[32];
      sm100::tmem_ld_32x32b_x32(tOt + c, o);
      sm100::tmem_wait_ld();
      if (row_ok && ok) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack2<T>(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
          w.y = pack2<T>(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
          w.z = pack2<T>(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
          w.w = pack2<T>(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c + 8 * v) = w;
        }
      }
    }
    if (p.out_lse && row_ok) lse[(int64_t)bh * p.T + qrow] = (m_used + log2f(l)) * 0.6931471805599453f;
    sm100::tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Three-warpgroup kernel (default): the two-tile work split and TMEM layout,
// plus
//  * K and V tiles in one ring of kRing3 single-tile slots, loaded in the
//    order K0 V0 K1 V1 ...; each slot is handed back by a tcgen05.commit as
//    soon as the last MMA reading it completes (K_j after S_B(j), V_j after
//    PV_B(j)), so key tile j+2 is already streaming while tile j is in use;
//  * register reallocation: the TMA/MMA warpgroup drops to 56 registers and
//    the two softmax warpgroups rise to 224, so a thread keeps its whole
//    128-column score row in registers and reads tensor memory once per tile;
//  * three-input max and packed fp32x2 FMA/add in the softmax.
// Warpgroup 0: warp 0 TMA producer, warp 1 MMA issue + TMEM allocation,
// warps 2-3 idle; warpgroups 1 and 2: softmax of tiles A and B.
// ---------------------------------------------------------------------------
constexpr int kThreads3 = 384;
constexpr int kRing3 = 5;
constexpr int kRegsLow3 = 56, kRegsHigh3 = 224;
// launch registers per thread the reallocation needs (128 * low + 256 * high <= 384 * launch)
constexpr int kRegsLaunch3 = (128 * kRegsLow3 + 256 * kRegsHigh3 + kThreads3 - 1) / kThreads3;

template <int D>
struct Flash3Smem {
  static constexpr uint32_t kHalf = kBM * 128;         // one 64-dim box of 128 rows
  static constexpr uint32_t kTile = (D / 64) * kHalf;  // Q, K or V tile
  static constexpr uint32_t oQA = 0;
  static constexpr uint32_t oQB = kTile;
  static constexpr uint32_t oRing = 2 * kTile;
  static constexpr uint32_t oBar = oRing + kRing3 * kTile;
  static constexpr uint32_t kTotal = oBar + 256 + 1024;
};

// P = 2^(s * sl2 - m) over one 128-column score row held in registers,
// written as bf16/fp16 pairs to tensor memory (columns [0, 64) of the S
// tile); returns the row sum of the (unrounded) probabilities.  kPoly of
// every 8 pairs take the FMA-pipe exponential (only on unmasked tiles).
template <typename T, int kPoly>
__device__ __forceinline__ float softmax_row_to_tmem(const uint32_t (&v)[kBN], float sl2, float neg_m,
                                                     uint32_t taddr) {
  float s[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) s[i] = 0.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t pk[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int c = h * 64 + 2 * i;
      float x0, x1;
      sm100::ffma2_bcast(x0, x1, __uint_as_float(v[c]), __uint_as_float(v[c + 1]), sl2, neg_m);
      float p0, p1;
      if ((i & 7) < kPoly) {
        ex2_poly2(x0, x1, p0, p1);
      } else {
        p0 = ex2_approx(x0);
        p1 = ex2_approx(x1);
      }
      sm100::fadd2_acc(s[2 * (i & 3)], s[2 * (i & 3) + 1], p0, p1);
      pk[i] = pack2<T>(p0, p1);
    }
    sm100::tmem_st_32x32b_x32(taddr + h * 32, pk);
  }
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads3, 1)
    flash_fwd3_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v, T* __restrict__ out, float* __restrict__ lse,
                              FlashParams p) {
  using L = Flash3Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = sm100::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA order: heads in groups of p.head_group; within a group, the
  // heaviest query tiles (causal) of all its heads first.  CTAs running
  // together then share a few heads' K/V through L2, and long tiles start
  // before short ones.
  const int n_ct = (int)((p.T + 2 * kBM - 1) / (2 * kBM));
  const int64_t BH = p.B * p.H;
  const int64_t lin = blockIdx.x;
  const int64_t grp = lin / ((int64_t)p.head_group * n_ct);
  const int64_t rem = lin - grp * p.head_group * n_ct;
  const int64_t gh = min((int64_t)p.head_group, BH - grp * p.head_group);  // heads in this group
  const int bh = (int)(grp * p.head_group + rem % gh);
  const int ct = n_ct - 1 - (int)(rem / gh);
  const int64_t q0 = (int64_t)ct * 2 * kBM;
  const int n_kt_all = (int)((p.S + kBN - 1) / kBN);
  // key tiles each query tile needs (causal: up to its diagonal); n_kt1 >= n_kt0
  // (scalars, not an array indexed by the tile: that would live in local memory)
  const int n_kt0 = p.causal ? min(n_kt_all, (int)((q0 + kBM - 1) / kBN) + 1) : n_kt_all;
  const int n_kt1 = p.causal ? min(n_kt_all, (int)((q0 + 2 * kBM - 1) / kBN) + 1) : n_kt_all;
  const int n_kt_max = n_kt1;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* q_full = bars + 0;
  uint64_t* ring_full = bars + 1;               // [kRing3]
  uint64_t* ring_empty = bars + 1 + kRing3;     // [kRing3]
  uint64_t* s_full = bars + 1 + 2 * kRing3;     // [2 tiles]
  uint64_t* p_full = s_full + 2;                // [2 tiles]
  uint64_t* o_done = s_full + 4;                // [2 tiles]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 6);
  int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    sm100::mbar_init(sm100::smem_u32(q_full), 1);
    for (int i = 0; i < kRing3; ++i) {
      sm100::mbar_init(sm100::smem_u32(&ring_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&ring_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(sm100::smem_u32(&s_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&p_full[i]), 4);
      sm100::mbar_init(sm100::smem_u32(&o_done[i]), 1);
    }
    *s_abort = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S_t at 128 t, O_t at 256 + 128 t

  if (warp < 4) {
    sm100::setmaxnreg_dec<kRegsLow3>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ producer
      sm100::tma_prefetch_desc(&tm_q);
      sm100::tma_prefetch_desc(&tm_k);
      sm100::tma_prefetch_desc(&tm_v);
      const uint32_t qb = sm100::smem_u32(q_full);
      sm100::mbar_arrive_expect_tx(qb, 2 * L::kTile);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < D / 64; ++h)
          sm100::tma_load_3d(sbase + (t ? L::oQB : L::oQA) + h * L::kHalf, &tm_q, qb, h * 64,
                             (int32_t)(q0 + t * kBM), bh);
      const int n_items = 2 * n_kt_max;
      int issued = 0;
      for (int it = 0; it < n_items; ++it) {
        const int slot = it % kRing3;
        if (!sm100::mbar_wait(sm100::smem_u32(&ring_empty[slot]), ((it / kRing3) & 1) ^ 1)) {
          b200_dev_error(kDevErrTimeoutEmpty);
          atomicExch(s_abort, 1);
          break;
        }
        if (*(volatile int*)s_abort) break;
        const uint32_t fb = sm100::smem_u32(&ring_full[slot]);
        const CUtensorMap* map = (it & 1) ? &tm_v : &tm_k;
        sm100::mbar_arrive_expect_tx(fb, L::kTile);
#pragma unroll
        for (int h = 0; h < D / 64; ++h)
          sm100::tma_load_3d(sbase + L::oRing + slot * L::kTile + h * L::kHalf, map, fb, h * 64,
                             (it >> 1) * kBN, bh);
        ++issued;
      }
      // no copy may still be writing shared memory when the CTA exits
      if (!sm100::mbar_wait(sm100::smem_u32(q_full), 0)) b200_dev_error(kDevErrTimeoutFull);
      for (int it = issued - 1; it >= 0 && it >= issued - kRing3; --it)
        if (!sm100::mbar_wait(sm100::smem_u32(&ring_full[it % kRing3]), (it / kRing3) & 1))
          b200_dev_error(kDevErrTimeoutFull);
    } else if (warp == 1) {
      // ----------------------------------------------------------- MMA issue
      // The whole warp runs the loop (waits, descriptors and ring position
      // stay warp-uniform); one elected lane issues the MMAs and commits.
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_s = sm100::make_idesc(1, fmt, fmt, 0, 0, kBM, kBN);
      constexpr uint32_t idesc_o = sm100::make_idesc(1, fmt, fmt, 0, 1, kBM, D);
      const uint32_t leader = sm100::elect_one();
      // Descriptors at offset 0; a ring slot or K step adds its byte offset
      // >> 4 to the start-address field (bits [0,14)), which never carries
      // since shared addresses stay below 2^18.
      const uint64_t dq0 = sm100::make_smem_desc(sbase + L::oQA, 16, 1024, sm100::kSwizzle128B);
      const uint64_t dq1 = sm100::make_smem_desc(sbase + L::oQB, 16, 1024, sm100::kSwizzle128B);
      const uint64_t dk = sm100::make_smem_desc(sbase + L::oRing, 16, 1024, sm100::kSwizzle128B);
      const uint64_t dv = sm100::make_smem_desc(sbase + L::oRing, L::kHalf, 1024, sm100::kSwizzle128B);
      bool ok = sm100::mbar_wait_warp(sm100::smem_u32(q_full), 0);
      // ring position of item it = 2j (K_j) or 2j + 1 (V_j): slot it % kRing3,
      // phase (it / kRing3) & 1 -- kept incrementally for the next K and V
      int k_slot = 0, v_slot = 1;
      uint32_t k_ph = 0, v_ph = 0;
      auto adv2 = [](int& slot, uint32_t& ph) {
        slot += 2;
        if (slot >= kRing3) {
          slot -= kRing3;
          ph ^= 1u;
        }
      };
      auto issue_s = [&](int t, int slot, uint32_t ph) -> bool {
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&ring_full[slot]), ph)) return false;
        sm100::tc_fence_after();
        const uint64_t ad = t ? dq1 : dq0;
        const uint64_t bd = dk + (uint64_t)((slot * L::kTile) >> 4);
        const uint32_t d_tmem = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * L::kHalf + (kk & 3) * 32) >> 4;
          sm100::mma_f16_ss(d_tmem, ad + off, bd + off, idesc_s, kk > 0 ? 1u : 0u, leader);
        }
        sm100::tc_commit(sm100::smem_u32(&s_full[t]), leader);
        return true;
      };
      auto issue_pv = [&](int t, int j, int slot, uint32_t ph) -> bool {
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&p_full[t]), j & 1)) return false;
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&ring_full[slot]), ph)) return false;
        sm100::tc_fence_after();
        const uint64_t bd = dv + (uint64_t)((slot * L::kTile) >> 4);
        const uint32_t d_tmem = tmem + 256 + t * 128, a_tmem = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // V: MN-major; 16 keys = two 8-row groups of 128 B (SBO 1024),
          // head-dim halves one box (16 KB) apart (LBO).  P: 8 TMEM columns
          // of bf16 pairs per 16 keys.
          sm100::mma_f16_ts(d_tmem, a_tmem + kk * 8, bd + (uint64_t)((kk * 2048) >> 4), idesc_o,
                            (j > 0 || kk > 0) ? 1u : 0u, leader);
        }
        return true;
      };
      auto release = [&](int slot) { sm100::tc_commit(sm100::smem_u32(&ring_empty[slot]), leader); };
      for (int t = 0; t < 2 && ok; ++t) ok = issue_s(t, k_slot, k_ph);
      if (ok) release(k_slot);  // K_0
      adv2(k_slot, k_ph);       // -> K_1
      for (int j = 0; ok && j < n_kt_max; ++j) {
        if (*(volatile int*)s_abort) {
          ok = false;
          break;
        }
        for (int t = 0; t < 2 && ok; ++t) {
          const int nkt = t ? n_kt1 : n_kt0;
          if (j >= nkt) continue;
          ok = issue_pv(t, j, v_slot, v_ph);
          if (ok && t == 1) release(v_slot);  // V_j: tile B reads it last
          if (ok && j + 1 < nkt) ok = issue_s(t, k_slot, k_ph);
          if (ok && j + 1 == nkt) sm100::tc_commit(sm100::smem_u32(&o_done[t]), leader);
        }
        if (ok && j + 1 < n_kt_max) release(k_slot);  // K_{j+1}
        adv2(k_slot, k_ph);
        adv2(v_slot, v_ph);
      }
      if (!ok) {
        if (leader) {
          b200_dev_error(kDevErrTimeoutFull);
          atomicExch(s_abort, 1);
        }
        for (int t = 0; t < 2; ++t) sm100::tc_commit(sm100::smem_u32(&o_done[t]), leader);
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    sm100::setmaxnreg_inc<kRegsHigh3>();
    const int t = (warp >> 2) - 1;  // tile of this warpgroup
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int64_t qrow = q0 + t * kBM + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tSt = tmem + t * 128 + lane_off, tOt = tmem + 256 + t * 128 + lane_off;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    const int nj = t ? n_kt1 : n_kt0;
    for (int j = 0; j < nj; ++j) {
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&s_full[t]), j & 1)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      uint32_t v[kBN];
      sm100::tmem_ld_32x32b_x64(tSt, v);
      sm100::tmem_ld_32x32b_x64(tSt + 64, v + 64);
      sm100::tmem_wait_ld();
      const int64_t k0 = (int64_t)j * kBN;
      int valid = kBN;
      if ((k0 + kBN > p.S) || (p.causal && k0 + kBN - 1 > qrow)) {
        const int64_t lim = (p.causal && qrow + 1 < p.S) ? qrow + 1 : p.S;
        const int64_t nv = lim - k0;
        valid = nv <= 0 ? 0 : (nv >= kBN ? kBN : (int)nv);
      }
      const bool full_tile = __all_sync(0xffffffffu, valid == kBN) != 0;
      if (!full_tile) {
#pragma unroll
        for (int i = 0; i < kBN; ++i)
          if (i >= valid) v[i] = 0xff800000u;  // -inf: max ignores it, 2^-inf = 0
      }
      float mx4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) mx4[i] = -INFINITY;
#pragma unroll
      for (int i = 0; i < kBN; i += 8) {
#pragma unroll
        for (int a = 0; a < 4; ++a)
          mx4[a] = sm100::fmax3(mx4[a], __uint_as_float(v[i + 2 * a]), __uint_as_float(v[i + 2 * a + 1]));
      }
      const float mx = sm100::fmax3(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3])) * p.sl2;
      float alpha = 1.f;
      bool rescale = false;
      if (m_used == -INFINITY) {
        m_used = mx;
      } else if (mx > m_used + kRescaleThreshold) {
        alpha = ex2_approx(m_used - mx);
        m_used = mx;
        rescale = true;
      }
      const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
      float rs;
      switch (full_tile ? p.poly_pairs : 0) {
        case 1: rs = softmax_row_to_tmem<T, 1>(v, p.sl2, neg_m, tSt); break;
        case 2: rs = softmax_row_to_tmem<T, 2>(v, p.sl2, neg_m, tSt); break;
        case 3: rs = softmax_row_to_tmem<T, 3>(v, p.sl2, neg_m, tSt); break;
        default: rs = softmax_row_to_tmem<T, 0>(v, p.sl2, neg_m, tSt); break;
      }
      // O_t holds PV_t(j-1), complete because S_t(j) is: rescale it if the
      // max moved (before P_t(j) is released to the MMA)
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t o[32];
          sm100::tmem_ld_32x32b_x32(tOt + c, o);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float y0, y1;
            sm100::fmul2_bcast(y0, y1, __uint_as_float(o[i]), __uint_as_float(o[i + 1]), alpha);
            o[i] = __float_as_uint(y0);
            o[i + 1] = __float_as_uint(y1);
          }
          sm100::tmem_st_32x32b_x32(tOt + c, o);
        }
      }
      sm100::tmem_wait_st();
      l = l * alpha + rs;
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&p_full[t]));
    }
    // epilogue: O_t / l
    if (ok && nj > 0 && !sm100::mbar_wait_warp(sm100::smem_u32(&o_done[t]), 0)) ok = false;
    if (!ok) {
      b200_dev_error(kDevErrTimeoutMma);
      atomicExch(s_abort, 1);
    }
    sm100::tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const bool row_ok = qrow < p.T;
    T* orow = out + ((int64_t)bh * p.T + qrow) * D;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t o[32];
      sm100::tmem_ld_32x32b_x32(tOt + c, o);
      sm100::tmem_wait_ld();
      if (row_ok && ok) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack2<T>(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
          w.y = pack2<T>(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
          w.z = pack2<T>(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
          w.w = pack2<T>(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c + 8 * v) = w;
        }
      }
    }
    if (p.out_lse && row_ok) lse[(int64_t)bh * p.T + qrow] = (m_used + log2f(l)) * 0.6931471805599453f;
    sm100::tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Persistent kernel (flags bit 4): one CTA per SM takes work items -- a pair of
// 128-row query tiles of one head -- from a global counter, in the
// head-grouped, heaviest-first order of the three-warpgroup kernel, whose
// warp roles, TMEM layout, K/V ring and register split it keeps.
// Consecutive items overlap: the next item's Q tiles load once the last S
// MMA of the current item has read Q (q_empty), its first S MMAs run while
// the softmax warpgroups drain O, and only the first PV MMA of each tile
// waits for that drain (o_empty).  Item ids pass from the producer thread
// to the other roles through a two-slot queue in shared memory; every
// barrier's phase runs on across items.
// ---------------------------------------------------------------------------
constexpr int kSchedSlots = 64;
__device__ unsigned g_flash_sched[kSchedSlots];  // per-launch work counters (host zeroes one per launch)

// work item lin -> (head bh, query-tile pair ct): heads in groups of
// p.head_group; within a group the heaviest tile pairs of all its heads first
__device__ __forceinline__ void flash_item(const FlashParams& p, int n_ct, int64_t lin, int& bh, int& ct) {
  const int64_t BH = p.B * p.H;
  const int64_t grp = lin / ((int64_t)p.head_group * n_ct);
  const int64_t rem = lin - grp * p.head_group * n_ct;
  const int64_t gh = min((int64_t)p.head_group, BH - grp * p.head_group);
  bh = (int)(grp * p.head_group + rem % gh);
  ct = n_ct - 1 - (int)(rem / gh);
}

// key tiles of the two query tiles of pair ct (causal: up to the diagonal); n1 >= n0
__device__ __forceinline__ void flash_kt(const FlashParams& p, int ct, int& n0, int& n1) {
  const int n_all = (int)((p.S + kBN - 1) / kBN);
  const int64_t q0 = (int64_t)ct * 2 * kBM;
  n0 = p.causal ? min(n_all, (int)((q0 + kBM - 1) / kBN) + 1) : n_all;
  n1 = p.causal ? min(n_all, (int)((q0 + 2 * kBM - 1) / kBN) + 1) : n_all;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads3, 1)
    flash_fwd4_persistent_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                                 const __grid_constant__ CUtensorMap tm_v, T* __restrict__ out,
                                 float* __restrict__ lse, FlashParams p, unsigned* __restrict__ sched) {
  using L = Flash3Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = sm100::smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_ct = (int)((p.T + 2 * kBM - 1) / (2 * kBM));
  const int64_t n_items = p.B * p.H * n_ct;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* ring_full = bars + 2;              // [kRing3]
  uint64_t* ring_empty = ring_full + kRing3;   // [kRing3]
  uint64_t* s_full = ring_empty + kRing3;      // [2 tiles]
  uint64_t* p_full = s_full + 2;               // [2 tiles]
  uint64_t* o_full = s_full + 4;               // [2 tiles]
  uint64_t* o_empty = s_full + 6;              // [2 tiles]
  uint64_t* item_full = s_full + 8;            // [2 queue slots]
  uint64_t* item_empty = s_full + 10;          // [2 queue slots]
  int* item_q = reinterpret_cast<int*>(s_full + 12);  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_q + 2);
  int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);
  static_assert(2 + 2 * kRing3 + 12 <= 30, "barrier area");

  if (threadIdx.x == 0) {
    sm100::mbar_init(sm100::smem_u32(q_full), 1);
    sm100::mbar_init(sm100::smem_u32(q_empty), 1);
    for (int i = 0; i < kRing3; ++i) {
      sm100::mbar_init(sm100::smem_u32(&ring_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&ring_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(sm100::smem_u32(&s_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&p_full[i]), 4);
      sm100::mbar_init(sm100::smem_u32(&o_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&o_empty[i]), 4);
      sm100::mbar_init(sm100::smem_u32(&item_full[i]), 1);
      sm100::mbar_init(sm100::smem_u32(&item_empty[i]), 9);  // MMA thread + 8 softmax warps
    }
    *s_abort = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S_t at column 128 t, O_t at 256 + 128 t

  if (warp < 4) {
    sm100::setmaxnreg_dec<kRegsLow3>();
    if (warp == 0 && lane == 0) {
      // --------------------------------------------------- scheduler + producer
      sm100::tma_prefetch_desc(&tm_q);
      sm100::tma_prefetch_desc(&tm_k);
      sm100::tma_prefetch_desc(&tm_v);
      uint32_t rit = 0;  // ring items issued, over all work items
      int q_issued = 0;  // Q loads issued (one per work item)
      int k = 0;
      bool ok = true;
      for (;; ++k) {
        const int qs = k & 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&item_empty[qs]), ((k >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        const int64_t lin = *(volatile int*)s_abort ? n_items : (int64_t)atomicAdd(sched, 1u);
        const int id = lin < n_items ? (int)lin : -1;
        item_q[qs] = id;
        sm100::mbar_arrive(sm100::smem_u32(&item_full[qs]));
        if (id < 0) break;
        int bh, ct, n0, n1;
        flash_item(p, n_ct, id, bh, ct);
        flash_kt(p, ct, n0, n1);
        const int64_t q0 = (int64_t)ct * 2 * kBM;
        if (k > 0 && !sm100::mbar_wait(sm100::smem_u32(q_empty), (k - 1) & 1)) {
          ok = false;
          break;
        }
        const uint32_t qb = sm100::smem_u32(q_full);
        sm100::mbar_arrive_expect_tx(qb, 2 * L::kTile);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int h = 0; h < D / 64; ++h)
            sm100::tma_load_3d(sbase + (t ? L::oQB : L::oQA) + h * L::kHalf, &tm_q, qb, h * 64,
                               (int32_t)(q0 + t * kBM), bh);
        ++q_issued;
        for (int it = 0; it < 2 * n1; ++it, ++rit) {
          const int slot = rit % kRing3;
          if (!sm100::mbar_wait(sm100::smem_u32(&ring_empty[slot]), ((rit / kRing3) & 1) ^ 1)) {
            ok = false;
            break;
          }
          const uint32_t fb = sm100::smem_u32(&ring_full[slot]);
          sm100::mbar_arrive_expect_tx(fb, L::kTile);
#pragma unroll
          for (int h = 0; h < D / 64; ++h)
            sm100::tma_load_3d(sbase + L::oRing + slot * L::kTile + h * L::kHalf, (it & 1) ? &tm_v : &tm_k, fb,
                               h * 64, (it >> 1) * kBN, bh);
        }
        if (!ok) break;
      }
      if (!ok) {
        b200_dev_error(kDevErrTimeoutEmpty);
        atomicExch(s_abort, 1);
      }
      // no copy may still be writing shared memory when the CTA exits
      if (q_issued > 0 && !sm100::mbar_wait(sm100::smem_u32(q_full), (q_issued - 1) & 1))
        b200_dev_error(kDevErrTimeoutFull);
      for (uint32_t it = rit > kRing3 ? rit - kRing3 : 0; it < rit; ++it)
        if (!sm100::mbar_wait(sm100::smem_u32(&ring_full[it % kRing3]), (it / kRing3) & 1))
          b200_dev_error(kDevErrTimeoutFull);
    } else if (warp == 1) {
      // ----------------------------------------------------------- MMA issue
      // The whole warp runs the loop (waits, descriptors and ring position
      // stay warp-uniform); one elected lane issues the MMAs and commits.
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_s = sm100::make_idesc(1, fmt, fmt, 0, 0, kBM, kBN);
      constexpr uint32_t idesc_o = sm100::make_idesc(1, fmt, fmt, 0, 1, kBM, D);
      const uint32_t leader = sm100::elect_one();
      // descriptors at offset 0; slots and K steps add (bytes >> 4) to the
      // start-address field, which never carries (addresses < 2^18)
      const uint64_t dq0 = sm100::make_smem_desc(sbase + L::oQA, 16, 1024, sm100::kSwizzle128B);
      const uint64_t dq1 = sm100::make_smem_desc(sbase + L::oQB, 16, 1024, sm100::kSwizzle128B);
      const uint64_t dk = sm100::make_smem_desc(sbase + L::oRing, 16, 1024, sm100::kSwizzle128B);
      const uint64_t dv = sm100::make_smem_desc(sbase + L::oRing, L::kHalf, 1024, sm100::kSwizzle128B);
      uint32_t rbase = 0;          // ring item of K_0 of the current work item
      uint32_t pc0 = 0, pc1 = 0;   // P releases consumed per tile
      bool ok = true;
      // ring item it (K_j = rbase + 2j, V_j = rbase + 2j + 1): slot it % kRing3,
      // fill phase (it / kRing3) & 1, advanced two items at a time
      auto adv2 = [](int& slot, uint32_t& ph) {
        slot += 2;
        if (slot >= kRing3) {
          slot -= kRing3;
          ph ^= 1u;
        }
      };
      auto issue_s = [&](int t, int slot, uint32_t ph) -> bool {
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&ring_full[slot]), ph)) return false;
        sm100::tc_fence_after();
        const uint64_t ad = t ? dq1 : dq0;
        const uint64_t bd = dk + (uint64_t)((slot * L::kTile) >> 4);
        const uint32_t d_tmem = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * L::kHalf + (kk & 3) * 32) >> 4;
          sm100::mma_f16_ss(d_tmem, ad + off, bd + off, idesc_s, kk > 0 ? 1u : 0u, leader);
        }
        sm100::tc_commit(sm100::smem_u32(&s_full[t]), leader);
        return true;
      };
      auto issue_pv = [&](int t, int j, int slot, uint32_t ph) -> bool {
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&p_full[t]), (t ? pc1 : pc0) & 1)) return false;
        if (t) ++pc1; else ++pc0;
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&ring_full[slot]), ph)) return false;
        sm100::tc_fence_after();
        const uint64_t bd = dv + (uint64_t)((slot * L::kTile) >> 4);
        const uint32_t d_tmem = tmem + 256 + t * 128, a_tmem = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          sm100::mma_f16_ts(d_tmem, a_tmem + kk * 8, bd + (uint64_t)((kk * 2048) >> 4), idesc_o,
                            (j > 0 || kk > 0) ? 1u : 0u, leader);
        return true;
      };
      auto release = [&](int slot) { sm100::tc_commit(sm100::smem_u32(&ring_empty[slot]), leader); };
      for (int k = 0; ok; ++k) {
        const int qs = k & 1;
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&item_full[qs]), (k >> 1) & 1)) {
          ok = false;
          break;
        }
        const int id = *(volatile int*)&item_q[qs];
        __syncwarp();
        if (leader) sm100::mbar_arrive(sm100::smem_u32(&item_empty[qs]));
        if (id < 0) break;
        int bh, ct, n0, n1;
        flash_item(p, n_ct, id, bh, ct);
        flash_kt(p, ct, n0, n1);
        if (!sm100::mbar_wait_warp(sm100::smem_u32(q_full), k & 1)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        int k_slot = (int)(rbase % kRing3), v_slot = (int)((rbase + 1) % kRing3);
        uint32_t k_ph = (rbase / kRing3) & 1, v_ph = ((rbase + 1) / kRing3) & 1;
        for (int t = 0; t < 2 && ok; ++t) ok = issue_s(t, k_slot, k_ph);
        if (!ok) break;
        release(k_slot);  // K_0
        adv2(k_slot, k_ph);
        if (n1 == 1) sm100::tc_commit(sm100::smem_u32(q_empty), leader);
        for (int j = 0; ok && j < n1; ++j) {
          if (*(volatile int*)s_abort) {
            ok = false;
            break;
          }
          for (int t = 0; t < 2 && ok; ++t) {
            const int nkt = t ? n1 : n0;
            if (j >= nkt) continue;
            // O_t of the previous work item must be drained before PV_t(0) overwrites it
            if (j == 0 && k > 0 && !sm100::mbar_wait_warp(sm100::smem_u32(&o_empty[t]), (k - 1) & 1)) {
              ok = false;
              break;
            }
            ok = issue_pv(t, j, v_slot, v_ph);
            if (ok && t == 1) release(v_slot);  // V_j: tile B reads it last
            if (ok && j + 1 < nkt) {
              ok = issue_s(t, k_slot, k_ph);
              // the last S MMA of the item (tile B's, as n1 >= n0) frees Q
              if (ok && t == 1 && j + 2 == n1) sm100::tc_commit(sm100::smem_u32(q_empty), leader);
            }
            if (ok && j + 1 == nkt) sm100::tc_commit(sm100::smem_u32(&o_full[t]), leader);
          }
          if (ok && j + 1 < n1) release(k_slot);  // K_{j+1}
          adv2(k_slot, k_ph);
          adv2(v_slot, v_ph);
        }
        rbase += 2 * n1;
      }
      if (!ok && leader) {
        b200_dev_error(kDevErrTimeoutFull);
        atomicExch(s_abort, 1);
      }
    }
  } else {
    // ------------------------------------------------ softmax + epilogue
    sm100::setmaxnreg_inc<kRegsHigh3>();
    const int t = (warp >> 2) - 1;  // tile of this warpgroup
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tSt = tmem + t * 128 + lane_off, tOt = tmem + 256 + t * 128 + lane_off;
    uint32_t sc = 0;  // S_t tiles consumed
    bool ok = true;
    for (int k = 0;; ++k) {
      const int qs = k & 1;
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&item_full[qs]), (k >> 1) & 1)) {
        ok = false;
        break;
      }
      const int id = *(volatile int*)&item_q[qs];
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&item_empty[qs]));
      if (id < 0) break;
      int bh, ct, n0, n1;
      flash_item(p, n_ct, id, bh, ct);
      flash_kt(p, ct, n0, n1);
      const int nj = t ? n1 : n0;
      const int64_t qrow = (int64_t)ct * 2 * kBM + t * kBM + r;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nj; ++j, ++sc) {
        if (!sm100::mbar_wait_warp(sm100::smem_u32(&s_full[t]), sc & 1)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        uint32_t v[kBN];
        sm100::tmem_ld_32x32b_x64(tSt, v);
        sm100::tmem_ld_32x32b_x64(tSt + 64, v + 64);
        sm100::tmem_wait_ld();
        const int64_t k0 = (int64_t)j * kBN;
        int valid = kBN;
        if ((k0 + kBN > p.S) || (p.causal && k0 + kBN - 1 > qrow)) {
          const int64_t lim = (p.causal && qrow + 1 < p.S) ? qrow + 1 : p.S;
          const int64_t nv = lim - k0;
          valid = nv <= 0 ? 0 : (nv >= kBN ? kBN : (int)nv);
        }
        if (!__all_sync(0xffffffffu, valid == kBN)) {
#pragma unroll
          for (int i = 0; i < kBN; ++i)
            if (i >= valid) v[i] = 0xff800000u;  // -inf: max ignores it, 2^-inf = 0
        }
        float mx4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) mx4[i] = -INFINITY;
#pragma unroll
        for (int i = 0; i < kBN; i += 8) {
#pragma unroll
          for (int a = 0; a < 4; ++a)
            mx4[a] = sm100::fmax3(mx4[a], __uint_as_float(v[i + 2 * a]), __uint_as_float(v[i + 2 * a + 1]));
        }
        const float mx = sm100::fmax3(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3])) * p.sl2;
        float alpha = 1.f;
        bool rescale = false;
        if (m_used == -INFINITY) {
          m_used = mx;
        } else if (mx > m_used + kRescaleThreshold) {
          alpha = ex2_approx(m_used - mx);
          m_used = mx;
          rescale = true;
        }
        const float neg_m = m_used == -INFINITY ? 0.f : -m_used;
        const float rs = softmax_row_to_tmem<T, 0>(v, p.sl2, neg_m, tSt);
        // O_t holds PV_t(j-1), complete because S_t(j) is: rescale it if the
        // max moved (before P_t(j) is released to the MMA)
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int c = 0; c < D; c += 32) {
            uint32_t o[32];
            sm100::tmem_ld_32x32b_x32(tOt + c, o);
            sm100::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float y0, y1;
              sm100::fmul2_bcast(y0, y1, __uint_as_float(o[i]), __uint_as_float(o[i + 1]), alpha);
              o[i] = __float_as_uint(y0);
              o[i + 1] = __float_as_uint(y1);
            }
            sm100::tmem_st_32x32b_x32(tOt + c, o);
          }
        }
        sm100::tmem_wait_st();
        l = l * alpha + rs;
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&p_full[t]));
      }
      if (!ok) break;
      // epilogue: read O_t out of tensor memory, hand it back to the MMA,
      // then O_t / l to global memory
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&o_full[t]), k & 1)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      uint32_t o[D];
#pragma unroll
      for (int c = 0; c < D; c += 32) sm100::tmem_ld_32x32b_x32(tOt + c, o + c);
      sm100::tmem_wait_ld();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&o_empty[t]));
      const float inv = l > 0.f ? 1.f / l : 0.f;
      if (qrow < p.T) {
        T* orow = out + ((int64_t)bh * p.T + qrow) * D;
#pragma unroll
        for (int c = 0; c < D; c += 8) {
          uint4 w;
          w.x = pack2<T>(__uint_as_float(o[c + 0]) * inv, __uint_as_float(o[c + 1]) * inv);
          w.y = pack2<T>(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
          w.z = pack2<T>(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
          w.w = pack2<T>(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c) = w;
        }
        if (p.out_lse) lse[(int64_t)bh * p.T + qrow] = (m_used + log2f(l)) * 0.6931471805599453f;
      }
    }
    if (!ok) {
      b200_dev_error(kDevErrTimeoutMma);
      atomicExch(s_abort, 1);
    }
    sm100::tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// General fallback for head dims the tensor-core path does not cover (<= 256):
// one warp per query row, lanes over keys, fp32 online softmax.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(128) flash_generic_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                            const T* __restrict__ v, T* __restrict__ out,
                                                            float* __restrict__ lse, FlashParams p, int D) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;  // flattened (bh, t)
  if (row >= p.B * p.H * p.T) return;
  const int64_t bh = row / p.T, t = row % p.T;
  const T* qr = q + row * D;
  const T* kb = k + bh * p.S * D;
  const T* vb = v + bh * p.S * D;
  float acc[8];
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int64_t s_end = p.causal ? min(p.S, t + 1) : p.S;
  for (int64_t s0 = 0; s0 < s_end; s0 += 32) {
    const int64_t s = s0 + lane;
    float x = -INFINITY;
    if (s < s_end) {
      float d = 0.f;
      for (int i = 0; i < D; ++i) d = fmaf(to_f32(qr[i]), to_f32(kb[s * D + i]), d);
      x = d * p.sl2;
    }
    const float mx = warp_max(x);
    const float mn = fmaxf(m, mx);
    const float a = (m == -INFINITY) ? 0.f : exp2f(m - mn);
    const float pw = (x == -INFINITY) ? 0.f : exp2f(x - mn);
    l = l * a + warp_sum(pw);
    for (int i = 0; i < 8; ++i) acc[i] *= a;
    for (int j = 0; j < 32; ++j) {
      const float pj = __shfl_sync(0xffffffffu, pw, j);
      const int64_t sj = s0 + j;
      if (sj >= s_end) break;
      for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc[i] = fmaf(pj, to_f32(vb[sj * D + d]), acc[i]);
      }
    }
    m = mn;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < D) out[row * D + d] = from_f32<T>(acc[i] * inv);
  }
  if (p.out_lse && lane == 0) lse[row] = (m + log2f(l)) * 0.6931471805599453f;
}

template <typename T, int D>
int launch_tc(const void* q, const void* k, const void* v, void* o, float* lse, const FlashParams& p,
              int variant, cudaStream_t s) {
  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {64, 128, 1};
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)p.T, (uint64_t)(p.B * p.H)};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)p.T * D * 2};
    int st = encode_tensor_map(&tq, dt, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)p.S, (uint64_t)(p.B * p.H)};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)p.S * D * 2};
    int st = encode_tensor_map(&tk, dt, 3, k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = encode_tensor_map(&tv, dt, 3, v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  if (variant == 4) {
    auto kern = flash_fwd4_persistent_kernel<T, D>;
    const int smem = (int)Flash3Smem<D>::kTotal;
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return launch_status(e);
    // the softmax warpgroups' setmaxnreg.inc draws on the launch registers
    if (fa.numRegs < kRegsLaunch3) {
      variant = 3;
    } else {
      const int64_t n_items = p.B * p.H * ((p.T + 2 * kBM - 1) / (2 * kBM));
      if (n_items > 0x7fffffffLL) return B200_ERR_UNSUPPORTED;
      int dev = 0, sms = 0;
      if ((e = cudaGetDevice(&dev)) != cudaSuccess) return launch_status(e);
      if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return launch_status(e);
      unsigned* counters = nullptr;
      if ((e = cudaGetSymbolAddress(reinterpret_cast<void**>(&counters), g_flash_sched)) != cudaSuccess)
        return launch_status(e);
      // one counter per launch, round-robin over the slots, so launches on
      // different streams do not share a counter unless kSchedSlots are in flight
      static std::atomic<unsigned> seq{0};
      unsigned* sched = counters + (seq.fetch_add(1, std::memory_order_relaxed) % kSchedSlots);
      if ((e = cudaMemsetAsync(sched, 0, sizeof(unsigned), s)) != cudaSuccess) return launch_status(e);
      if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
        return launch_status(e);
      const unsigned grid = (unsigned)(n_items < sms ? n_items : sms);
      kern<<<grid, kThreads3, smem, s>>>(tq, tk, tv, static_cast<T*>(o), lse, p, sched);
      return launch_status(cudaGetLastError());
    }
  }
  if (variant == 3) {
    auto kern = flash_fwd3_tcgen05_kernel<T, D>;
    const int smem = (int)Flash3Smem<D>::kTotal;
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return launch_status(e);
    // the softmax warpgroups' setmaxnreg.inc draws on the launch registers
    if (fa.numRegs < kRegsLaunch3) variant = 2;
  }
  if (variant == 3) {
    auto kern = flash_fwd3_tcgen05_kernel<T, D>;
    const int smem = (int)Flash3Smem<D>::kTotal;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return launch_status(e);
    const int64_t n_cta = p.B * p.H * ((p.T + 2 * kBM - 1) / (2 * kBM));
    if (n_cta > 0x7fffffffLL) return B200_ERR_UNSUPPORTED;
    kern<<<(unsigned)n_cta, kThreads3, smem, s>>>(tq, tk, tv, static_cast<T*>(o), lse, p);
    return launch_status(cudaGetLastError());
  }
  if (variant == 2) {
    auto kern = flash_fwd2_tcgen05_kernel<T, D>;
    const int smem = (int)Flash2Smem<D>::kTotal;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return launch_status(e);
    dim3 grid((unsigned)(p.B * p.H), (unsigned)((p.T + 2 * kBM - 1) / (2 * kBM)));
    kern<<<grid, kThreads2, smem, s>>>(tq, tk, tv, static_cast<T*>(o), lse, p);
    return launch_status(cudaGetLastError());
  }
  auto kern = flash_fwd_tcgen05_kernel<T, D>;
  const int smem = (int)FlashSmem<D>::kTotal;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return launch_status(e);
  dim3 grid((unsigned)(p.B * p.H), (unsigned)p.n_qt);
  kern<<<grid, kThreads, smem, s>>>(tq, tk, tv, static_cast<T*>(o), lse, p);
  return launch_status(cudaGetLastError());
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_flash_attn(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                               int64_t H, int64_t T, int64_t S, int64_t D, float scale, int32_t causal,
                               int32_t dtype, const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("flash_attn")) return e;
  if (B < 0 || H < 0 || T < 0 || S < 0 || D <= 0) return B200_ERR_BAD_ARG;
  if (causal && T != S) return B200_ERR_BAD_ARG;  // the reference's tril mask assumes T == S
  if (B * H * T == 0) return B200_OK;
  if (!q || !k || !v || !o) return B200_ERR_BAD_ARG;
  if (S == 0) return B200_ERR_BAD_ARG;
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)D);
  FlashParams p;
  p.B = B;
  p.H = H;
  p.T = T;
  p.S = S;
  p.n_qt = (int)((T + kBM - 1) / kBM);
  p.sl2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  p.out_lse = lse != nullptr;
  p.poly_exp = (cfg && (cfg->flags & 2)) ? 1 : 0;  // flags bit 1
  p.head_group = (cfg && cfg->split > 0) ? cfg->split : 8;  // split: heads per scheduling group
  // tile_k: exponential pairs (of every 8) on the FMA pipe; 0 = default 2
  // (measured about 2% faster than none at B4 H32 T4096 D128 causal), 4 = none
  p.poly_pairs = ((cfg && cfg->tile_k > 0) ? cfg->tile_k : 2) & 3;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool tc = (D == 64 || D == 128) && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o) &&
                  B * H <= 0x7fffffffLL && p.n_qt <= 65535 && T < (1ll << 31) && S < (1ll << 31);
  if (tc) {
    return B200_DISPATCH_HALF(dtype, [&] {
      // flags bit 0: the one-tile kernel (P staged in shared memory);
      // bit 2: the two-tile kernel without register reallocation; bit 4:
      // the persistent kernel (one CTA per SM taking work items)
      const int fl = cfg ? cfg->flags : 0;
      const int variant = (fl & 1) ? 1 : (fl & 4) ? 2 : (fl & 16) ? 4 : 3;
      return D == 128 ? launch_tc<scalar_t, 128>(q, k, v, o, lse, p, variant, s)
                      : launch_tc<scalar_t, 64>(q, k, v, o, lse, p, variant, s);
    });
  }
  if (D > 256) return B200_ERR_UNSUPPORTED;
  return B200_DISPATCH_HALF(dtype, [&] {
    const int64_t rows = B * H * T;
    flash_generic_kernel<scalar_t><<<(unsigned)((rows + 3) / 4), 128, 0, s>>>(
        static_cast<const scalar_t*>(q), static_cast<const scalar_t*>(k), static_cast<const scalar_t*>(v),
        static_cast<scalar_t*>(o), lse, p, (int)D);
    return launch_status(cudaGetLastError());
  });
}
