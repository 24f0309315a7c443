// Paged-attention decode (one query token per sequence), grouped-query.
//
// Reference: triton_agent/ops/paged_attention/reference.py:26-52.  For each
// sequence b the reference walks the first ceil(ctx/block_size) entries of
// block_table[b], drops ids outside [0, num_blocks) (reference.py:40-41),
// concatenates the remaining blocks' tokens, truncates to ctx tokens
// (reference.py:47-48) and computes softmax(q . K^T * scale) . V in fp32.
// Consequently the j-th *valid* block (rank j among valid ones) supplies
// tokens [j*bs, j*bs + bs) of the concatenation, of which
// clamp(ctx - j*bs, 0, bs) survive the truncation; this kernel reproduces
// that rule exactly.  Query head h reads kv head h / (Hq / Hkv).
//
// Structure (HBM-bound; algorithmic bytes = 2 * ctx * Hkv * D * 2 per
// sequence for K and V, plus q, out and the block table):
//   grid  = (splits, B, Hkv / HG), one CTA per (split, sequence, head group)
//   warps = HG consumer warps (one per kv head) + 1 producer warp
//   The producer warp builds the split's page list from the block table,
//   then one lane streams whole pages -- K and V tiles [bs][HG][D] of all
//   HG heads -- into a ring of shared-memory stages with 3-D TMA loads
//   (mbarrier complete_tx).  Consumer warp w owns kv head h0 + w and its G
//   query heads: 8 lanes per token (16 of the 128 dims each), 4 tokens in
//   flight per warp, q.k reduced with 3 xor-shuffles, fp32 online softmax
//   in base 2, P.V accumulated in registers.  Lane groups merge at the end.
//   When a sequence spans several splits, each CTA writes (m, l, o) to the
//   workspace and the last CTA to finish (atomic ticket) merges them and
//   resets the ticket, so one launch does the whole op.
#include <limits.h>
#include <math.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

B200_DEVICE_ERROR_WORD()

namespace b200 {
namespace {

constexpr int kD = 128;           // head dim of the TMA path
constexpr int kMaxSplitBlocks = 256;
constexpr int kMaxSplits = 1024;
constexpr size_t kTicketBytes = 256 * 1024;  // one int per (sequence, head group), <= 65536

struct DecodeParams {
  int64_t B, Hq, Hkv, num_blocks, block_size, max_blocks;
  int HG;            // kv heads per CTA (= consumer warps)
  int n_hg;          // Hkv / HG
  int split_blocks;  // block-table entries per split
  int max_splits;    // ceil(max_blocks / split_blocks)
  int stages;
  uint32_t stage_bytes;  // K + V tile bytes of one page
  uint32_t tiles_bytes;  // bytes before the barriers (stage ring, or combine weights if larger)
  float qscale;          // scale * log2(e)
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

template <typename T>
__device__ __forceinline__ void widen8(const uint4& raw, float* f) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
    unpack16<T>(raw, f);
  }
}

template <typename IDX>
__device__ __forceinline__ bool bad_block(IDX id, int64_t nb) {
  return id < 0 || (int64_t)id >= nb;
}

// ---------------------------------------------------------------------------
// Tensor-core consumer (block size a multiple of 16), transposed form.  Warp
// w owns kv head h0 + w and its G query heads.  Tokens are the M dimension of
// the m16n8k16 tiles and query heads the N dimension (8 columns, heads >= G
// are zero), so a 16-token chunk of a page costs 8 + 8 mma.sync:
//   S^T[16 tok x 8 heads] = K[16 x 128] Q^T  -- 8 k-steps, K as the A operand
//                                              by ldmatrix (rows = tokens), two
//                                              independent accumulator chains
//   online softmax on the C fragments: a thread holds tokens lane/4 and
//   lane/4 + 8 of heads 2(lane%4) and 2(lane%4)+1; a head's max over the 16
//   tokens needs 3 xor-shuffles
//   O^T[128 x 8 heads] += V^T[128 x 16 tok] P^T  -- 8 m-tiles of 16 dims, V as
//                                              the A operand by ldmatrix.trans;
//                                              P^T's B fragments are the packed
//                                              S^T fragments transposed in
//                                              registers by movmatrix
// The accumulator is 8 tiles x 4 floats per thread, and the V fragments are
// loaded before the softmax so their latency overlaps it.  Shared-memory
// tiles are SWIZZLE_128B with rows = (head, token), so the 8 rows of every
// ldmatrix matrix hit 8 distinct 16-byte bank groups.  Each head's running
// max is raised only when it grows by more than 2^8 (exact: O and l share the
// offset).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// 8x8 b16 matrix transpose across the warp (fragment layout: row lane/4,
// columns 2(lane%4) and 2(lane%4)+1 in one register).
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Zeroes the 16-bit halves of a fragment register whose token is >= ntok.
__device__ __forceinline__ uint32_t mask_pair(uint32_t v, int tok, int ntok) {
  const uint32_t lo = tok < ntok ? 0x0000ffffu : 0u;
  const uint32_t hi = tok + 1 < ntok ? 0xffff0000u : 0u;
  return v & (lo | hi);
}

// Q^T B fragments of this warp's query heads: head lane/4 (zero if >= G),
// dims 16ks + 2(lane%4) + {0,1} and +8.
template <typename T, int G>
__device__ __forceinline__ void load_q_frags(const T* __restrict__ qrow0, int lane, uint32_t (&qb)[8][2]) {
  const int qh = lane >> 2, qc = (lane & 3) * 2;
  const T* qr = qrow0 + (qh < G ? qh : 0) * kD;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qb[ks][0] = qh < G ? *reinterpret_cast<const uint32_t*>(qr + 16 * ks + qc) : 0u;
    qb[ks][1] = qh < G ? *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 8 + qc) : 0u;
  }
}

// Raises head c's running max to mx when it grew by more than 2^8; o entries
// of that head are columns c and c + 2 of every tile.
__device__ __forceinline__ void raise_max(float& mu, float mx, float& lp, float (&o)[8][4], int c) {
  if (mu == -INFINITY) {
    mu = mx;
  } else if (mx > mu + 8.0f) {
    const float alpha = exp2f(mu - mx);
    mu = mx;
    lp *= alpha;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      o[mt][c] *= alpha;
      o[mt][c + 2] *= alpha;
    }
  }
}

// One page (ntok tokens of one kv head, K tile at kb, V tile at vb in the
// swizzled [d-half][head][token][64] layout) folded into this warp's running
// (o, mu, lp): mu/lp[0] for head 2(lane%4), [1] for head 2(lane%4)+1.
template <typename T>
__device__ __forceinline__ void mma_page(uint32_t kb, uint32_t vb, int ntok, int w, int bs, int lane,
                                         uint32_t hbytes, float sl2, const uint32_t (&qb)[8][2],
                                         float (&o)[8][4], float (&mu)[2], float (&lp)[2]) {
  const int mat = lane >> 3, mrow = lane & 7;
  const int tr = lane >> 2, tq = (lane & 3) * 2;
  for (int t0 = 0; t0 < ntok; t0 += 16) {
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    {
      // A = K rows: matrix `mat` = (token half mat&1, dim-chunk parity mat>>1)
      const int row = w * bs + t0 + (mat & 1) * 8 + mrow;
      const uint32_t rbase = kb + row * 128;
      const int sw = row & 7;
      uint32_t ka[8][4];
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int chunk = ((ks & 3) << 1) | (mat >> 1);
        ldsm_x4(rbase + (ks >> 2) * hbytes + ((chunk ^ sw) << 4), ka[ks][0], ka[ks][1], ka[ks][2], ka[ks][3]);
      }
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        mma16816<T>((ks & 1) ? s1 : s0, ka[ks][0], ka[ks][1], ka[ks][2], ka[ks][3], qb[ks][0], qb[ks][1]);
    }
    // A = V^T by ldmatrix.trans: matrix `mat` = (token half mat>>1, dim-chunk parity mat&1)
    uint32_t va[8][4];
    {
      const int row = w * bs + t0 + (mat >> 1) * 8 + mrow;
      const uint32_t rbase = vb + row * 128;
      const int sw = row & 7;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int chunk = ((mt & 3) << 1) | (mat & 1);
        ldsm_x4_t(rbase + (mt >> 2) * hbytes + ((chunk ^ sw) << 4), va[mt][0], va[mt][1], va[mt][2], va[mt][3]);
      }
    }
    // x[0]/x[1]: token tr of heads 2(lane%4), +1; x[2]/x[3]: token tr + 8
    const bool ok0 = t0 + tr < ntok, ok1 = t0 + tr + 8 < ntok;
    float x[4];
    x[0] = ok0 ? (s0[0] + s1[0]) * sl2 : -INFINITY;
    x[1] = ok0 ? (s0[1] + s1[1]) * sl2 : -INFINITY;
    x[2] = ok1 ? (s0[2] + s1[2]) * sl2 : -INFINITY;
    x[3] = ok1 ? (s0[3] + s1[3]) * sl2 : -INFINITY;
    float mA = fmaxf(x[0], x[2]), mB = fmaxf(x[1], x[3]);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      mA = fmaxf(mA, __shfl_xor_sync(0xffffffffu, mA, off));
      mB = fmaxf(mB, __shfl_xor_sync(0xffffffffu, mB, off));
    }
    raise_max(mu[0], mA, lp[0], o, 0);
    raise_max(mu[1], mB, lp[1], o, 1);
    const float p0 = exp2f(x[0] - mu[0]), p2 = exp2f(x[2] - mu[0]);
    const float p1 = exp2f(x[1] - mu[1]), p3 = exp2f(x[3] - mu[1]);
    lp[0] += p0 + p2;
    lp[1] += p1 + p3;
    // P^T B fragments: tokens tq + {0,1} (b0) and 8 + tq + {0,1} (b1) of head lane/4
    const uint32_t b0 = movm_t(pack_pair<T>(p0, p1));
    const uint32_t b1 = movm_t(pack_pair<T>(p2, p3));
    if (t0 + 16 > ntok) {
      // tokens past the end may hold anything (NaN included): zero their V
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        va[mt][0] = mask_pair(va[mt][0], t0 + tq, ntok);
        va[mt][1] = mask_pair(va[mt][1], t0 + tq, ntok);
        va[mt][2] = mask_pair(va[mt][2], t0 + 8 + tq, ntok);
        va[mt][3] = mask_pair(va[mt][3], t0 + 8 + tq, ntok);
      }
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) mma16816<T>(o[mt], va[mt][0], va[mt][1], va[mt][2], va[mt][3], b0, b1);
  }
}

// Sum of a head's l over the 8 lanes that share it.
__device__ __forceinline__ float head_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// Normalised output rows of this warp's heads: orow0 = row of head 0; the
// O^T fragments are transposed back by movmatrix into 4-byte stores of two
// dims of head lane/4.
template <typename T, int G>
__device__ __forceinline__ void store_rows(T* __restrict__ orow0, const float (&o)[8][4], float lA, float lB,
                                           int lane) {
  const float iA = lA > 0.f ? 1.f / lA : 0.f, iB = lB > 0.f ? 1.f / lB : 0.f;
  const int h = lane >> 2, tq = (lane & 3) * 2;
  T* orow = orow0 + (h < G ? h : 0) * kD;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const uint32_t r0 = movm_t(pack_pair<T>(o[mt][0] * iA, o[mt][1] * iB));
    const uint32_t r1 = movm_t(pack_pair<T>(o[mt][2] * iA, o[mt][3] * iB));
    if (h < G) {
      *reinterpret_cast<uint32_t*>(orow + 16 * mt + tq) = r0;
      *reinterpret_cast<uint32_t*>(orow + 16 * mt + 8 + tq) = r1;
    }
  }
}

// Unnormalised fp32 partial of this warp's heads: row(h) = base + h * pitch
// floats holds o[0..127]; (m, l) go to mpos(h), mpos(h) + 1 via ml_base +
// h * ml_pitch.
template <int G>
__device__ __forceinline__ void store_partial(float* __restrict__ base, int64_t pitch, float* __restrict__ ml_base,
                                              int64_t ml_pitch, const float (&o)[8][4], const float (&mu)[2],
                                              float lA, float lB, int lane) {
  const int hA = (lane & 3) * 2, hB = hA + 1, d = lane >> 2;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    if (hA < G) {
      base[hA * pitch + 16 * mt + d] = o[mt][0];
      base[hA * pitch + 16 * mt + 8 + d] = o[mt][2];
    }
    if (hB < G) {
      base[hB * pitch + 16 * mt + d] = o[mt][1];
      base[hB * pitch + 16 * mt + 8 + d] = o[mt][3];
    }
  }
  if (d == 0) {
    if (hA < G) {
      ml_base[hA * ml_pitch] = mu[0];
      ml_base[hA * ml_pitch + 1] = lA;
    }
    if (hB < G) {
      ml_base[hB * ml_pitch] = mu[1];
      ml_base[hB * ml_pitch + 1] = lB;
    }
  }
}

template <typename T, int G>
__device__ __forceinline__ void consume_mma(uint8_t* smem, uint64_t* full_bar, uint64_t* empty_bar,
                                            const int* list_ntok, int* s_misc, int npages, int nsplit,
                                            const T* __restrict__ q, T* __restrict__ out,
                                            float* __restrict__ ws_o, float* __restrict__ ws_ml, int64_t b,
                                            int hg, int split, int w, int lane, const DecodeParams& p) {
  const int HG = p.HG;
  const int bs = (int)p.block_size;
  const int64_t kvh = (int64_t)hg * HG + w;
  uint32_t qb[8][2];
  load_q_frags<T, G>(q + (b * p.Hq + kvh * G) * kD, lane, qb);
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mu[2] = {-INFINITY, -INFINITY}, lp[2] = {0.f, 0.f};
  const float sl2 = p.qscale;
  const uint32_t base = sm100::smem_u32(smem);
  const uint32_t hbytes = p.stage_bytes / 4;

  for (int i = 0; i < npages; ++i) {
    const int s = i % p.stages;
    if (!sm100::mbar_wait_warp(sm100::smem_u32(&full_bar[s]), (i / p.stages) & 1)) {
      b200_dev_error(kDevErrTimeoutFull);
      atomicExch(&s_misc[1], 1);
      break;
    }
    if (*(volatile int*)&s_misc[1]) break;
    const int ntok = list_ntok[i];
    const uint32_t kb = base + s * p.stage_bytes;
    const uint32_t vb = kb + 2 * hbytes;
    mma_page<T>(kb, vb, ntok, w, bs, lane, hbytes, sl2, qb, o, mu, lp);
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&empty_bar[s]));
  }

  const float lA = head_sum(lp[0]), lB = head_sum(lp[1]);
  const int64_t qrow0 = b * p.Hq + kvh * G;
  if (nsplit == 1) {
    store_rows<T, G>(out + qrow0 * kD, o, lA, lB, lane);
  } else {
    const int heads_cta = HG * G;
    const int64_t prow = ((b * p.n_hg + hg) * (int64_t)p.max_splits + split) * heads_cta + w * G;
    store_partial<G>(ws_o + prow * kD, kD, ws_ml + prow * 2, 2, o, mu, lA, lB, lane);
    __threadfence();
  }
}

template <typename T, typename IDX, int G, bool MMA>
__global__ void __launch_bounds__(288, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const T* __restrict__ q,
                        const IDX* __restrict__ block_table, const IDX* __restrict__ ctx_len,
                        T* __restrict__ out, float* __restrict__ ws_o, float* __restrict__ ws_ml,
                        int* __restrict__ tickets, DecodeParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // SWIZZLE_128B tiles need 1024-byte alignment (the launch reserves the slack).
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int hg = blockIdx.z;
  const int HG = p.HG;
  const int heads_cta = HG * G;
  const int64_t bs = p.block_size;

  // Shared-memory carve-up: [stages x (K tile | V tile)] [bars] [page list] [scalars]
  const uint32_t tiles_bytes = p.tiles_bytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + tiles_bytes);
  uint64_t* empty_bar = full_bar + p.stages;
  int* list_id = reinterpret_cast<int*>(empty_bar + p.stages);
  int* list_ntok = list_id + kMaxSplitBlocks;
  int* s_misc = list_ntok + kMaxSplitBlocks;  // [0] npages, [1] abort, [2] last-CTA flag
  float* s_wts = reinterpret_cast<float*>(smem);  // combine weights, reuses the tiles

  int64_t ctx = (int64_t)ctx_len[b];
  const int64_t nvb64 = ctx > 0 ? (ctx + bs - 1) / bs : 0;
  const int nvb = (int)(nvb64 < p.max_blocks ? nvb64 : p.max_blocks);
  const int nsplit = (nvb + p.split_blocks - 1) / p.split_blocks;
  const int64_t out_row0 = b * p.Hq + (int64_t)hg * heads_cta;

  if (nvb == 0) {
    // No context: the output rows are zero (the reference has nothing to
    // concatenate here and fails; zero is this library's defined result).
    if (split == 0) {
      for (int i = threadIdx.x; i < heads_cta * kD; i += blockDim.x)
        out[out_row0 * kD + i] = from_f32<T>(0.f);
    }
    return;
  }
  if (split >= nsplit) return;
  const int p0 = split * p.split_blocks;
  const int p1 = min(p0 + p.split_blocks, nvb);
  const IDX* bt = block_table + b * p.max_blocks;

  // ---- page list: valid blocks of this split with their surviving tokens
  if (warp == HG) {
    // Invalid entries before this split shift the token ranks of its pages.
    // Eight independent loads per lane are in flight per round.
    int inval = 0;
    for (int j0 = 0; j0 < p0; j0 += 256) {
      IDX v[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int j = j0 + r * 32 + lane;
        v[r] = j < p0 ? __ldg(&bt[j]) : (IDX)0;
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) inval += (j0 + r * 32 + lane < p0 && bad_block(v[r], p.num_blocks)) ? 1 : 0;
    }
    inval = __reduce_add_sync(0xffffffffu, inval);
    int count = 0;
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int j0 = p0; j0 < p1; j0 += 32) {
      const int j = j0 + lane;
      const bool in = j < p1;
      const IDX id = in ? __ldg(&bt[j]) : (IDX)-1;
      const bool valid = in && !bad_block(id, p.num_blocks);
      const unsigned ib = __ballot_sync(0xffffffffu, in && !valid);
      const int64_t rank = (int64_t)j - (inval + __popc(ib & lt_mask));
      int64_t nt = ctx - rank * bs;
      nt = nt < 0 ? 0 : (nt > bs ? bs : nt);
      const bool use = valid && nt > 0;
      const unsigned ub = __ballot_sync(0xffffffffu, use);
      if (use) {
        const int slot = count + __popc(ub & lt_mask);
        list_id[slot] = (int)id;
        list_ntok[slot] = (int)nt;
      }
      count += __popc(ub);
      inval += __popc(ib);
    }
    if (lane == 0) {
      s_misc[0] = count;
      s_misc[1] = 0;
      for (int s = 0; s < p.stages; ++s) {
        sm100::mbar_init(sm100::smem_u32(&full_bar[s]), 1);
        sm100::mbar_init(sm100::smem_u32(&empty_bar[s]), HG);
      }
      sm100::fence_barrier_init();
    }
  }
  __syncthreads();
  const int npages = s_misc[0];

  // Per-lane online-softmax state (consumers only).
  float m[G], l[G], o[G][16];
  const int grp = lane >> 3, sub = lane & 7;

  if (warp == HG) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_k);
      sm100::tma_prefetch_desc(&tm_v);
      const uint32_t base = sm100::smem_u32(smem);
      int issued = 0;
      for (int i = 0; i < npages; ++i) {
        const int s = i % p.stages;
        const uint32_t parity = ((i / p.stages) & 1) ^ 1;
        if (!sm100::mbar_wait(sm100::smem_u32(&empty_bar[s]), parity)) {
          b200_dev_error(kDevErrTimeoutEmpty);
          atomicExch(&s_misc[1], 1);
          break;
        }
        if (*(volatile int*)&s_misc[1]) break;
        const uint32_t fb = sm100::smem_u32(&full_bar[s]);
        sm100::mbar_arrive_expect_tx(fb, p.stage_bytes);
        const int32_t tok0 = list_id[i] * (int32_t)bs;
        const uint32_t dst = base + s * p.stage_bytes;
        if constexpr (MMA) {
          // [d-half][head][token][64 dims], SWIZZLE_128B (map dims: d, slot, head)
          const uint32_t hb = p.stage_bytes / 4;
          sm100::tma_load_3d(dst, &tm_k, fb, 0, tok0, hg * HG);
          sm100::tma_load_3d(dst + hb, &tm_k, fb, 64, tok0, hg * HG);
          sm100::tma_load_3d(dst + 2 * hb, &tm_v, fb, 0, tok0, hg * HG);
          sm100::tma_load_3d(dst + 3 * hb, &tm_v, fb, 64, tok0, hg * HG);
        } else {
          // [token][head][128 dims], no swizzle (map dims: d, head, slot)
          sm100::tma_load_3d(dst, &tm_k, fb, 0, hg * HG, tok0);
          sm100::tma_load_3d(dst + p.stage_bytes / 2, &tm_v, fb, 0, hg * HG, tok0);
        }
        ++issued;
      }
      // Never leave the CTA with bulk copies still landing in shared memory:
      // wait (bounded) for the last fill of every stage.
      for (int i = issued - 1; i >= 0 && i >= issued - p.stages; --i) {
        const int s = i % p.stages;
        if (!sm100::mbar_wait(sm100::smem_u32(&full_bar[s]), (i / p.stages) & 1))
          b200_dev_error(kDevErrTimeoutFull);
      }
    }
  } else if constexpr (MMA) {
    consume_mma<T, G>(smem, full_bar, empty_bar, list_ntok, s_misc, npages, nsplit, q, out, ws_o, ws_ml,
                      b, hg, split, warp, lane, p);
  } else {
    // ---------------------------------------------------------- consumers
    const int w = warp;
    const int64_t kvh = (int64_t)hg * HG + w;
    float qf[G][16];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const T* qr = q + (b * p.Hq + kvh * G + g) * kD;
      float f[8];
      load16_f32(qr + 8 * sub, f);
#pragma unroll
      for (int d = 0; d < 8; ++d) qf[g][d] = f[d] * p.qscale;
      load16_f32(qr + 64 + 8 * sub, f);
#pragma unroll
      for (int d = 0; d < 8; ++d) qf[g][8 + d] = f[d] * p.qscale;
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int d = 0; d < 16; ++d) o[g][d] = 0.f;
    }
    const uint32_t base = sm100::smem_u32(smem);
    const uint32_t row_bytes = kD * 2;
    const uint32_t tok_bytes = HG * row_bytes;
    const uint32_t lane_off = w * row_bytes + sub * 16;

    for (int i = 0; i < npages; ++i) {
      const int s = i % p.stages;
      if (!sm100::mbar_wait_warp(sm100::smem_u32(&full_bar[s]), (i / p.stages) & 1)) {
        b200_dev_error(kDevErrTimeoutFull);
        atomicExch(&s_misc[1], 1);
        break;
      }
      if (*(volatile int*)&s_misc[1]) break;
      const int ntok = list_ntok[i];
      const uint32_t kb = base + s * p.stage_bytes + lane_off;
      const uint32_t vb = kb + p.stage_bytes / 2;
      for (int t0 = 0; t0 < ntok; t0 += 16) {
        float sc[4][G];
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          const int tok = t0 + 4 * pp + grp;
          const bool ok = tok < ntok;
          float part[G];
#pragma unroll
          for (int g = 0; g < G; ++g) part[g] = 0.f;
          if (ok) {
            float kf[16];
            widen8<T>(lds128(kb + tok * tok_bytes), kf);
            widen8<T>(lds128(kb + tok * tok_bytes + 128), kf + 8);
#pragma unroll
            for (int g = 0; g < G; ++g) {
              float a0 = 0.f, a1 = 0.f;
#pragma unroll
              for (int d = 0; d < 8; ++d) {
                a0 = fmaf(qf[g][d], kf[d], a0);
                a1 = fmaf(qf[g][8 + d], kf[8 + d], a1);
              }
              part[g] = a0 + a1;
            }
          }
#pragma unroll
          for (int g = 0; g < G; ++g) {
            part[g] += __shfl_xor_sync(0xffffffffu, part[g], 1);
            part[g] += __shfl_xor_sync(0xffffffffu, part[g], 2);
            part[g] += __shfl_xor_sync(0xffffffffu, part[g], 4);
            sc[pp][g] = ok ? part[g] : -INFINITY;
          }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float mx = fmaxf(fmaxf(sc[0][g], sc[1][g]), fmaxf(sc[2][g], sc[3][g]));
          const float mnew = fmaxf(m[g], mx);
          const float alpha = (m[g] == mnew) ? 1.f : exp2f(m[g] - mnew);
          m[g] = mnew;
          float psum = 0.f;
#pragma unroll
          for (int pp = 0; pp < 4; ++pp) {
            sc[pp][g] = (sc[pp][g] == -INFINITY) ? 0.f : exp2f(sc[pp][g] - mnew);
            psum += sc[pp][g];
          }
          l[g] = fmaf(l[g], alpha, psum);
#pragma unroll
          for (int d = 0; d < 16; ++d) o[g][d] *= alpha;
        }
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          const int tok = t0 + 4 * pp + grp;
          if (tok < ntok) {
            float vf[16];
            widen8<T>(lds128(vb + tok * tok_bytes), vf);
            widen8<T>(lds128(vb + tok * tok_bytes + 128), vf + 8);
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
              for (int d = 0; d < 16; ++d) o[g][d] = fmaf(sc[pp][g], vf[d], o[g][d]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&empty_bar[s]));
    }

    // Merge the four lane groups (tokens were dealt round-robin to them).
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int x = 8; x <= 16; x <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m[g], x);
        const float lo = __shfl_xor_sync(0xffffffffu, l[g], x);
        const float mn = fmaxf(m[g], mo);
        const float a = (m[g] == -INFINITY) ? 0.f : exp2f(m[g] - mn);
        const float c = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
        l[g] = l[g] * a + lo * c;
#pragma unroll
        for (int d = 0; d < 16; ++d) {
          const float oo = __shfl_xor_sync(0xffffffffu, o[g][d], x);
          o[g][d] = o[g][d] * a + oo * c;
        }
        m[g] = mn;
      }
    }

    if (grp == 0) {
      if (nsplit == 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float inv = l[g] > 0.f ? 1.f / l[g] : 0.f;
          float r0[8], r1[8];
#pragma unroll
          for (int d = 0; d < 8; ++d) {
            r0[d] = o[g][d] * inv;
            r1[d] = o[g][8 + d] * inv;
          }
          T* orow = out + (b * p.Hq + kvh * G + g) * kD;
          *reinterpret_cast<uint4*>(orow + 8 * sub) = pack16<T>(r0);
          *reinterpret_cast<uint4*>(orow + 64 + 8 * sub) = pack16<T>(r1);
        }
      } else {
        const int64_t prow0 =
            ((b * p.n_hg + hg) * (int64_t)p.max_splits + split) * heads_cta + w * G;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float* po = ws_o + (prow0 + g) * kD;
          *reinterpret_cast<float4*>(po + 8 * sub) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
          *reinterpret_cast<float4*>(po + 8 * sub + 4) =
              make_float4(o[g][4], o[g][5], o[g][6], o[g][7]);
          *reinterpret_cast<float4*>(po + 64 + 8 * sub) =
              make_float4(o[g][8], o[g][9], o[g][10], o[g][11]);
          *reinterpret_cast<float4*>(po + 64 + 8 * sub + 4) =
              make_float4(o[g][12], o[g][13], o[g][14], o[g][15]);
          if (sub == 0) {
            ws_ml[(prow0 + g) * 2] = m[g];
            ws_ml[(prow0 + g) * 2 + 1] = l[g];
          }
        }
        __threadfence();
      }
    }
  }

  if (nsplit == 1) return;

  // ---- cross-split merge by the last CTA of this (sequence, head group)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    int* ticket = tickets + b * p.n_hg + hg;
    const int prev = atomicAdd(ticket, 1);
    const int last = (prev == nsplit - 1);
    if (last) atomicExch(ticket, 0);  // ready for the next launch
    s_misc[2] = last;
  }
  __syncthreads();
  if (!s_misc[2]) return;
  __threadfence();
  const int64_t pbase = (b * p.n_hg + hg) * (int64_t)p.max_splits * heads_cta;
  for (int hh = threadIdx.x; hh < heads_cta; hh += blockDim.x) {
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(&ws_ml[(pbase + (int64_t)s * heads_cta + hh) * 2]));
    float L = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const int64_t r = pbase + (int64_t)s * heads_cta + hh;
      const float ms = __ldcg(&ws_ml[r * 2]);
      const float wgt = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
      s_wts[hh * nsplit + s] = wgt;
      L += wgt * __ldcg(&ws_ml[r * 2 + 1]);
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int s = 0; s < nsplit; ++s) s_wts[hh * nsplit + s] *= inv;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < heads_cta * kD; idx += blockDim.x) {
    const int hh = idx / kD, d = idx % kD;
    float acc = 0.f;
    for (int s = 0; s < nsplit; ++s)
      acc = fmaf(s_wts[hh * nsplit + s], __ldcg(&ws_o[(pbase + (int64_t)s * heads_cta + hh) * kD + d]), acc);
    out[(out_row0 + hh) * kD + d] = from_f32<T>(acc);
  }
}

// ---------------------------------------------------------------------------
// General fallback (any D <= 256, any block size / head ratio): one CTA of
// four warps per (sequence, query head); tokens dealt round-robin to warps,
// one token per warp step, lanes over the head dim.  Used only for shapes the
// TMA path does not cover.
// ---------------------------------------------------------------------------
template <typename T, typename IDX>
__global__ void __launch_bounds__(128) paged_decode_generic_kernel(
    const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc,
    const IDX* __restrict__ block_table, const IDX* __restrict__ ctx_len, T* __restrict__ out,
    int64_t Hq, int64_t Hkv, int64_t D, int64_t num_blocks, int64_t bs, int64_t max_blocks,
    float qscale) {
  __shared__ float s_m[4], s_l[4], s_o[4][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t hq = blockIdx.x, b = blockIdx.y;
  const int64_t kvh = hq / (Hq / Hkv);
  const int64_t ctx = (int64_t)ctx_len[b];
  const int64_t nvb = ctx > 0 ? min((ctx + bs - 1) / bs, max_blocks) : 0;
  const T* qr = q + (b * Hq + hq) * D;
  float qv[8], ov[8];
  for (int i = 0; i < 8; ++i) {
    const int64_t d = lane + 32 * i;
    qv[i] = d < D ? to_f32(qr[d]) * qscale : 0.f;
    ov[i] = 0.f;
  }
  float mrun = -INFINITY, lrun = 0.f;
  int64_t rank = 0;
  for (int64_t j = 0; j < nvb; ++j) {
    const IDX id = block_table[b * max_blocks + j];
    if (bad_block(id, num_blocks)) continue;
    int64_t nt = ctx - rank * bs;
    ++rank;
    nt = nt < 0 ? 0 : (nt > bs ? bs : nt);
    for (int64_t t = warp; t < nt; t += 4) {
      const int64_t row = (((int64_t)id * bs + t) * Hkv + kvh) * D;
      float part = 0.f;
      for (int i = 0; i < 8; ++i) {
        const int64_t d = lane + 32 * i;
        if (d < D) part = fmaf(qv[i], to_f32(kc[row + d]), part);
      }
      const float sc = warp_sum(part);
      const float mn = fmaxf(mrun, sc);
      const float a = (mrun == -INFINITY) ? 0.f : exp2f(mrun - mn);
      const float pw = exp2f(sc - mn);
      lrun = lrun * a + pw;
      for (int i = 0; i < 8; ++i) {
        const int64_t d = lane + 32 * i;
        ov[i] = ov[i] * a + (d < D ? pw * to_f32(vc[row + d]) : 0.f);
      }
      mrun = mn;
    }
  }
  if (lane == 0) {
    s_m[warp] = mrun;
    s_l[warp] = lrun;
  }
  for (int i = 0; i < 8; ++i) {
    const int64_t d = lane + 32 * i;
    if (d < D) s_o[warp][d] = ov[i];
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w]);
  float L = 0.f, wts[4];
  for (int w = 0; w < 4; ++w) {
    wts[w] = (s_m[w] == -INFINITY) ? 0.f : exp2f(s_m[w] - M);
    L += wts[w] * s_l[w];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int w = 0; w < 4; ++w) acc += wts[w] * s_o[w][d];
    out[(b * Hq + hq) * D + d] = from_f32<T>(acc * inv);
  }
}

// ---------------------------------------------------------------------------
// Persistent flat-partition decode (tensor-core consumer).
//
// All sequences' block-table entries are laid end to end (segment s = hg*B + b
// holds ceil(ctx_b / bs) entries) and cut into ranges: the first E - D entries
// into one equal contiguous range per CTA (one CTA per SM), the last D
// entries (dyn_pct percent of E) into chunks of `chunk` entries that CTAs
// claim from an atomic counter once their own range is streamed, which evens
// out finish times when SMs stream at different rates (off by default: see
// kFlatDynPct).  The producer warp walks each range segment by segment
// without draining the TMA ring: each stage carries a small PageMeta record,
// either a data page (ntok surviving tokens) or an end-of-segment marker.
// On a marker the consumer warps finish the segment: a segment wholly inside one range is
// written directly; otherwise the CTA writes its (m, l, o) piece to one of
// the range's two partial slots (slot 0 for the first segment of the range,
// 1 for the last) and the CTA that finishes the segment's last piece (atomic
// ticket) merges the pieces: per-head max and 1/sum first, then per-piece
// weights in shared memory and independent 16-byte loads of the pieces' o
// rows (a loop of dependent loads per element held the merging CTA's stream
// for ~25 us and set the kernel's tail: 209 us against 193 us now).  The claim counter resets itself: the last CTA
// to find the pool empty zeroes it.  Per segment, the token rank rule of the
// reference (dropped ids shift later blocks) is applied exactly as in the
// split kernel.
// ---------------------------------------------------------------------------
constexpr int kFlatMaxSeg = 1024;
constexpr int kFlatPitch = kD + 4;  // floats per partial row: o[128], m, l, pad (16-byte rows)
// Default share of entries handed out as claimed chunks: 0.  With the bench
// shape (64 sequences, 148 CTAs) claimed chunks of 4-8 pages make tens of
// pieces per sequence and the merges cost more than the balancing gains
// (measured 262-334 us vs 193 us for equal ranges); cfg tile_k turns them on.
constexpr int kFlatDynPct = 0;
constexpr int kFlatChunk = 4;    // default entries (pages) per claimed chunk

// Partial (m, l, o) rows of the persistent kernel: two per range, ranges =
// static ones (<= grid) + claimed chunks.
constexpr int kFlatChunksPerCta = 8;  // at most this many claimed chunks per CTA of the grid
__host__ __device__ inline int64_t flat_partial_rows(int64_t grid, int64_t entries_max, int dyn_pct, int chunk,
                                                     int64_t heads_cta) {
  const int64_t dyn = entries_max * dyn_pct / 100 + 1;
  int64_t nch = (dyn + chunk - 1) / chunk;
  if (nch > kFlatChunksPerCta * grid) nch = kFlatChunksPerCta * grid;
  return 2 * (grid + nch + 1) * heads_cta;
}

struct FlatParams {
  int64_t B, Hq, Hkv, num_blocks, block_size, max_blocks;
  int HG, n_hg, stages, nseg;
  int dyn_pct;  // share of the entries handed out as claimed chunks (0..90)
  int chunk;    // entries per claimed chunk (raised so that there are at most max_chunks)
  int max_chunks;
  uint32_t stage_bytes;
  float qscale;
};

// Claim counters of the persistent kernel: the last two ints of the ticket
// region ([0] next chunk, [1] CTAs done).
constexpr int kPoolInts = 2;

struct PageMeta {
  int kind;     // 0 data page, 1 end of segment, 2 end of stream
  int ntok;     // data: surviving tokens of the page
  int seg;      // segment id hg * B + b
  int slot;     // marker: partial slot of this range's piece, or -1 when direct
  int c1, c2;   // marker: ranges holding the segment's pieces
  int c1_slot;  // marker: slot used by the piece of range c1
  int rng;      // marker: range id of this piece
};

__device__ __forceinline__ int64_t flat_lo(int64_t c, int64_t E, int64_t G) { return c * E / G; }
__device__ __forceinline__ int flat_owner(int64_t e, int64_t E, int64_t G) {
  return (int)(((e + 1) * G + E - 1) / E - 1);
}

// Ranges of the entry list: Gs equal static ranges over [0, S), then chunks
// of CH entries over [S, E).
struct FlatRanges {
  int64_t S, E, Gs;
  int64_t CH;
  __device__ __forceinline__ int64_t lo(int64_t r) const {
    if (r <= Gs) return Gs > 0 ? flat_lo(r, S, Gs) : 0;
    const int64_t x = S + (r - Gs) * CH;
    return x < E ? x : E;
  }
  __device__ __forceinline__ int of(int64_t e) const {
    return e < S ? flat_owner(e, S, Gs) : (int)(Gs + (e - S) / CH);
  }
};

template <typename T, typename IDX, int G>
__global__ void __launch_bounds__(288, 1)
    paged_decode_flat_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                             const T* __restrict__ q, const IDX* __restrict__ block_table,
                             const IDX* __restrict__ ctx_len, T* __restrict__ out, float* __restrict__ ws_rows,
                             int* __restrict__ tickets, FlatParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HG = p.HG;
  const int heads_cta = HG * G;
  const int64_t B = p.B;
  const int bs = (int)p.block_size;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + p.stages * p.stage_bytes);
  uint64_t* empty_bar = full_bar + p.stages;
  PageMeta* meta = reinterpret_cast<PageMeta*>(empty_bar + p.stages);
  int64_t* s_cum = reinterpret_cast<int64_t*>(meta + p.stages);
  int64_t* s_ctx = s_cum + (p.nseg + 1);
  int* chunk_id = reinterpret_cast<int*>(s_ctx + B);
  int* chunk_ntok = chunk_id + 32;
  float* s_comb = reinterpret_cast<float*>(chunk_ntok + 32);  // [2][64]
  int* s_flags = reinterpret_cast<int*>(s_comb + 128);        // [0] abort, [1] last piece
  float* s_w = reinterpret_cast<float*>(s_flags + 4);         // merge weights [heads_cta][32]

  // ---- prologue: contexts, entry prefix over segments, barriers
  if (warp == HG) {
    for (int64_t b = lane; b < B; b += 32) s_ctx[b] = (int64_t)ctx_len[b];
    __syncwarp();
    int64_t run = 0;
    const unsigned lt_mask = (1u << lane) - 1u;
    (void)lt_mask;
    for (int s0 = 0; s0 < p.nseg; s0 += 32) {
      const int s = s0 + lane;
      int64_t e = 0;
      if (s < p.nseg) {
        const int64_t ctx = s_ctx[s % B];
        const int64_t nvb = ctx > 0 ? (ctx + bs - 1) / bs : 0;
        e = nvb < p.max_blocks ? nvb : p.max_blocks;
      }
      int64_t incl = e;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (s < p.nseg) s_cum[s + 1] = run + incl;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_cum[0] = 0;
      s_flags[0] = 0;
      s_flags[1] = 0;
      for (int s = 0; s < p.stages; ++s) {
        sm100::mbar_init(sm100::smem_u32(&full_bar[s]), 1);
        sm100::mbar_init(sm100::smem_u32(&empty_bar[s]), HG);
      }
      sm100::fence_barrier_init();
    }
  }
  __syncthreads();
  // With programmatic dependent launch (cfg flags bit 3) everything up to
  // each role's griddepcontrol.wait overlaps the previous kernel (whose
  // caller guarantees it writes neither context_len nor block_table): the
  // contexts, entry prefix and barriers above, and the producer's walk of
  // the block table up to its first page copy.  No q, KV page or output
  // byte is touched before the wait, after which that grid has completed
  // and its writes are visible.  A no-op for an ordinary launch.
  const int64_t E = s_cum[p.nseg];
  const int64_t Gc = gridDim.x;
  FlatRanges R;
  R.E = E;
  R.S = E - E * p.dyn_pct / 100;
  R.Gs = R.S < Gc ? R.S : Gc;
  R.CH = p.chunk;
  if (R.CH * p.max_chunks < E - R.S) R.CH = (E - R.S + p.max_chunks - 1) / p.max_chunks;
  const int64_t n_chunks = (E - R.S + R.CH - 1) / R.CH;
  const int64_t n_ranges = R.Gs + n_chunks;
  const int64_t Gp = n_chunks > 0 ? Gc : R.Gs;  // CTAs taking part
  const int c = blockIdx.x;

  // Segments without entries (context <= 0) are never streamed: zero them.
  if (warp < HG) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int s = c; s < p.nseg; s += (int)Gc) {
      if (s_cum[s + 1] != s_cum[s]) continue;
      const int64_t b = s % B, hg = s / B;
      T* orow = out + (b * p.Hq + hg * heads_cta) * kD;
      for (int i = threadIdx.x; i < heads_cta * kD; i += HG * 32) orow[i] = from_f32<T>(0.f);
    }
  }
  if (c >= Gp) return;  // uniform per CTA

  if (warp == HG) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      sm100::tma_prefetch_desc(&tm_k);
      sm100::tma_prefetch_desc(&tm_v);
    }
    const uint32_t base = sm100::smem_u32(smem);
    const uint32_t hb = p.stage_bytes / 4;
    const unsigned lt_mask = (1u << lane) - 1u;
    int it = 0;
    bool ok = true;
    bool dep_waited = false;  // griddepcontrol.wait done by this lane
    // lane 0 pushes one ring entry; returns false on timeout
    auto push = [&](const PageMeta& m, int32_t tok0, int32_t h0) -> bool {
      const int st = it % p.stages;
      if (!sm100::mbar_wait(sm100::smem_u32(&empty_bar[st]), ((it / p.stages) & 1) ^ 1)) return false;
      meta[st] = m;
      const uint32_t fb = sm100::smem_u32(&full_bar[st]);
      if (m.kind == 0) {
        if (!dep_waited) {  // the first page copy waits for the previous kernel
          asm volatile("griddepcontrol.wait;" ::: "memory");
          dep_waited = true;
        }
        sm100::mbar_arrive_expect_tx(fb, p.stage_bytes);
        const uint32_t dst = base + st * p.stage_bytes;
        sm100::tma_load_3d(dst, &tm_k, fb, 0, tok0, h0);
        sm100::tma_load_3d(dst + hb, &tm_k, fb, 64, tok0, h0);
        sm100::tma_load_3d(dst + 2 * hb, &tm_v, fb, 0, tok0, h0);
        sm100::tma_load_3d(dst + 3 * hb, &tm_v, fb, 64, tok0, h0);
      } else {
        sm100::mbar_arrive(fb);
      }
      ++it;
      return true;
    };
    int* pool = tickets + (kTicketBytes / 4 - kPoolInts);
    // first range: this CTA's static one, else a claimed chunk
    int rng = c;
    if (c >= R.Gs) {
      int nr = INT_MAX;
      if (lane == 0) nr = (int)R.Gs + atomicAdd(&pool[0], 1);
      rng = __shfl_sync(0xffffffffu, nr, 0);
    }
    while (ok && rng < n_ranges) {
    const int64_t lo = R.lo(rng), hi = R.lo(rng + 1);
    // segment containing lo: the largest s with cum[s] <= lo
    int s = 0;
    {
      int l = 0, r = p.nseg;  // invariant cum[l] <= lo < cum[r]
      while (r - l > 1) {
        const int mid = (l + r) >> 1;
        if (s_cum[mid] <= lo) l = mid;
        else r = mid;
      }
      s = l;
    }
    int64_t e = lo;
    bool first = true;
    while (e < hi && ok) {
      while (s_cum[s + 1] == s_cum[s]) ++s;
      const int64_t b = s % B;
      const int hg = s / (int)B;
      const int64_t segs = s_cum[s], sege = s_cum[s + 1];
      const int j0 = (int)(e - segs);
      const int j1 = (int)((hi < sege ? hi : sege) - segs);
      const int c1 = R.of(segs), c2 = R.of(sege - 1);
      const int my_slot = first ? 0 : 1;
      const int c1_slot = (segs == R.lo(c1)) ? 0 : 1;
      const int64_t ctx = s_ctx[b];
      const IDX* bt = block_table + b * p.max_blocks;
      // invalid entries before j0 shift the token ranks of this range
      int inval = 0;
      for (int jb = 0; jb < j0; jb += 256) {
        IDX v[8];
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const int j = jb + rr * 32 + lane;
          v[rr] = j < j0 ? __ldg(&bt[j]) : (IDX)0;
        }
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) inval += (jb + rr * 32 + lane < j0 && bad_block(v[rr], p.num_blocks)) ? 1 : 0;
      }
      inval = __reduce_add_sync(0xffffffffu, inval);
      for (int jj = j0; jj < j1 && ok; jj += 32) {
        const int j = jj + lane;
        const bool in = j < j1;
        const IDX id = in ? __ldg(&bt[j]) : (IDX)-1;
        const bool valid = in && !bad_block(id, p.num_blocks);
        const unsigned ib = __ballot_sync(0xffffffffu, in && !valid);
        const int64_t rank = (int64_t)j - (inval + __popc(ib & lt_mask));
        int64_t nt = ctx - rank * bs;
        nt = nt < 0 ? 0 : (nt > bs ? bs : nt);
        const bool use = valid && nt > 0;
        const unsigned ub = __ballot_sync(0xffffffffu, use);
        if (use) {
          const int k = __popc(ub & lt_mask);
          chunk_id[k] = (int)id;
          chunk_ntok[k] = (int)nt;
        }
        inval += __popc(ib);
        __syncwarp();
        if (lane == 0) {
          const int n = __popc(ub);
          for (int u = 0; u < n && ok; ++u) {
            PageMeta m{0, chunk_ntok[u], s, 0, 0, 0, 0, 0};
            ok = !(*(volatile int*)&s_flags[0]) && push(m, chunk_id[u] * bs, hg * HG);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        __syncwarp();
      }
      if (lane == 0 && ok) {
        PageMeta m{1, 0, s, c1 == c2 ? -1 : my_slot, c1, c2, c1_slot, rng};
        ok = push(m, 0, 0);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      e = segs + j1;
      if (e == sege) ++s;
      first = false;
    }
    // next range: a claimed chunk
    int nr = INT_MAX;
    if (lane == 0 && n_chunks > 0) nr = (int)R.Gs + atomicAdd(&pool[0], 1);
    rng = __shfl_sync(0xffffffffu, nr, 0);
    }
    if (lane == 0) {
      if (n_chunks > 0) {
        // every CTA of the grid ends here once; the last one re-arms the pool
        const int done = atomicAdd(&pool[1], 1);
        if (done == (int)Gp - 1) {
          atomicExch(&pool[0], 0);
          atomicExch(&pool[1], 0);
        }
      }
      if (ok) {
        PageMeta m{2, 0, 0, 0, 0, 0, 0, 0};
        ok = push(m, 0, 0);
      }
      if (!ok) {
        b200_dev_error(kDevErrTimeoutEmpty);
        atomicExch(&s_flags[0], 1);
      }
      // never leave with bulk copies landing in shared memory
      for (int i = it - 1; i >= 0 && i >= it - p.stages; --i)
        if (!sm100::mbar_wait(sm100::smem_u32(&full_bar[i % p.stages]), (i / p.stages) & 1))
          b200_dev_error(kDevErrTimeoutFull);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int w = warp;
  const uint32_t base = sm100::smem_u32(smem);
  const uint32_t hbytes = p.stage_bytes / 4;
  uint32_t qb[8][2];
  float o[8][4];
  float mu[2] = {-INFINITY, -INFINITY}, lp[2] = {0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  int cur_seg = -1;
  const int nthr = HG * 32;
  for (int it = 0;; ++it) {
    const int st = it % p.stages;
    if (!sm100::mbar_wait_warp(sm100::smem_u32(&full_bar[st]), (it / p.stages) & 1)) {
      b200_dev_error(kDevErrTimeoutFull);
      atomicExch(&s_flags[0], 1);
      break;
    }
    const PageMeta m = meta[st];
    if (m.kind == 0) {
      if (m.seg != cur_seg) {
        cur_seg = m.seg;
        const int64_t b = m.seg % B, kvh = (int64_t)(m.seg / B) * HG + w;
        load_q_frags<T, G>(q + (b * p.Hq + kvh * G) * kD, lane, qb);
      }
      const uint32_t kb = base + st * p.stage_bytes;
      mma_page<T>(kb, kb + 2 * hbytes, m.ntok, w, bs, lane, hbytes, p.qscale, qb, o, mu, lp);
    } else if (m.kind == 1) {
      // ---- finish segment m.seg
      const float lA = head_sum(lp[0]), lB = head_sum(lp[1]);
      const int64_t b = m.seg % B, hg = m.seg / B;
      const int64_t head0 = hg * heads_cta + w * G;  // first head of this warp inside the sequence
      if (m.slot < 0) {
        store_rows<T, G>(out + (b * p.Hq + head0) * kD, o, lA, lB, lane);
      } else {
        float* row0 = ws_rows + ((int64_t)(m.rng * 2 + m.slot) * heads_cta + w * G) * kFlatPitch;
        store_partial<G>(row0, kFlatPitch, row0 + kD, kFlatPitch, o, mu, lA, lB, lane);
        __threadfence();
        named_bar_sync(1, nthr);
        if (threadIdx.x == 0) {
          const int prev = atomicAdd(&tickets[m.seg], 1);
          const int last = (prev == m.c2 - m.c1);
          if (last) atomicExch(&tickets[m.seg], 0);
          s_flags[1] = last;
        }
        named_bar_sync(1, nthr);
        if (s_flags[1]) {
          // ---- merge the segment's pieces (ranges c1..c2): per-head max and
          // 1/sum, then per-piece weights in shared memory and independent
          // 16-byte loads of the pieces' o rows.  The merging CTA is one of
          // the last to finish, so every step keeps its loads in flight
          // together: a lane folds the (m, l) of its pieces for up to four heads
          // of its warp at once into running (max, sum) pairs, combined over
          // the warp by a butterfly.
          __threadfence();
          const int np = m.c2 - m.c1 + 1;
          auto piece = [&](int i, int hh) -> const float* {
            const int cc = m.c1 + i;
            const int sl = (cc == m.c1) ? m.c1_slot : 0;
            return ws_rows + ((int64_t)(cc * 2 + sl) * heads_cta + hh) * kFlatPitch;
          };
          // (mx, L) += a piece (mc, lc): the sum rescaled to the larger max
          auto fold = [](float& mx, float& L, float mc, float lc) {
            if (mc == -INFINITY) return;
            if (mc > mx) {
              L = (mx == -INFINITY ? 0.f : L * exp2f(mx - mc)) + lc;
              mx = mc;
            } else {
              L = fmaf(exp2f(mc - mx), lc, L);
            }
          };
          if constexpr (G <= 4) {
            constexpr int GB = G < 4 ? G : 4;  // heads of the warp folded together
  #pragma unroll
            for (int kb = 0; kb < G; kb += GB) {
              float mxh[GB], Lh[GB];
  #pragma unroll
              for (int k = 0; k < GB; ++k) {
                mxh[k] = -INFINITY;
                Lh[k] = 0.f;
              }
              for (int i = lane; i < np; i += 32) {
                float mi[GB], li[GB];
  #pragma unroll
                for (int k = 0; k < GB; ++k) {
                  const float* r = piece(i, w + (kb + k) * HG);
                  mi[k] = __ldcg(r + kD);
                  li[k] = __ldcg(r + kD + 1);
                }
  #pragma unroll
                for (int k = 0; k < GB; ++k) fold(mxh[k], Lh[k], mi[k], li[k]);
              }
  #pragma unroll
              for (int off = 16; off > 0; off >>= 1) {
  #pragma unroll
                for (int k = 0; k < GB; ++k) {
                  const float om = __shfl_xor_sync(0xffffffffu, mxh[k], off);
                  const float ol = __shfl_xor_sync(0xffffffffu, Lh[k], off);
                  fold(mxh[k], Lh[k], om, ol);
                }
              }
              if (lane == 0) {
  #pragma unroll
                for (int k = 0; k < GB; ++k) {
                  s_comb[w + (kb + k) * HG] = mxh[k];
                  s_comb[64 + w + (kb + k) * HG] = Lh[k] > 0.f ? 1.f / Lh[k] : 0.f;
                }
              }
            }
          } else {
            // eight heads a warp: one head at a time (the folded form's
            // registers spill here)
            for (int hh = w; hh < heads_cta; hh += HG) {
              float mx = -INFINITY;
              for (int i = lane; i < np; i += 32) mx = fmaxf(mx, __ldcg(piece(i, hh) + kD));
  #pragma unroll
              for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
              float L = 0.f;
              for (int i = lane; i < np; i += 32) {
                const float* r = piece(i, hh);
                const float mc = __ldcg(r + kD);
                L += (mc == -INFINITY) ? 0.f : exp2f(mc - mx) * __ldcg(r + kD + 1);
              }
  #pragma unroll
              for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
              if (lane == 0) {
                s_comb[hh] = mx;
                s_comb[64 + hh] = L > 0.f ? 1.f / L : 0.f;
              }
            }
          }
          named_bar_sync(1, nthr);
          float4 acc[G];
#pragma unroll
          for (int k = 0; k < G; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int i0 = 0; i0 < np; i0 += 32) {
            const int nb = np - i0 < 32 ? np - i0 : 32;
            for (int x = threadIdx.x; x < heads_cta * nb; x += nthr) {
              const int hh = x / nb, i = x - hh * nb;
              const float mc = __ldcg(piece(i0 + i, hh) + kD);
              s_w[hh * 32 + i] = (mc == -INFINITY) ? 0.f : exp2f(mc - s_comb[hh]) * s_comb[64 + hh];
            }
            named_bar_sync(1, nthr);
            for (int i = 0; i < nb; ++i) {
              float4 v[G];
#pragma unroll
              for (int k = 0; k < G; ++k) {
                const int idx = threadIdx.x + k * nthr;  // head idx / 32, dims 4 * (idx % 32)
                v[k] = __ldcg(reinterpret_cast<const float4*>(piece(i0 + i, idx >> 5) + 4 * (idx & 31)));
              }
#pragma unroll
              for (int k = 0; k < G; ++k) {
                const int idx = threadIdx.x + k * nthr;
                const float wgt = s_w[(idx >> 5) * 32 + i];
                acc[k].x = fmaf(wgt, v[k].x, acc[k].x);
                acc[k].y = fmaf(wgt, v[k].y, acc[k].y);
                acc[k].z = fmaf(wgt, v[k].z, acc[k].z);
                acc[k].w = fmaf(wgt, v[k].w, acc[k].w);
              }
            }
            named_bar_sync(1, nthr);
          }
#pragma unroll
          for (int k = 0; k < G; ++k) {
            const int idx = threadIdx.x + k * nthr;
            T* dst = out + (b * p.Hq + hg * heads_cta + (idx >> 5)) * kD + 4 * (idx & 31);
            uint2 pk;
            pk.x = pack_pair<T>(acc[k].x, acc[k].y);
            pk.y = pack_pair<T>(acc[k].z, acc[k].w);
            *reinterpret_cast<uint2*>(dst) = pk;
          }
        }
      }
      mu[0] = mu[1] = -INFINITY;
      lp[0] = lp[1] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      cur_seg = -1;
    }
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(sm100::smem_u32(&empty_bar[st]));
    if (m.kind == 2) break;
  }
}

struct Geometry {
  bool tma_path;
  bool mma;   // tensor-core consumer (block size a multiple of 16)
  bool flat;  // persistent flat-partition kernel
  int flat_grid;
  int dyn_pct, chunk;  // persistent kernel: claimed share of the entries, entries per chunk
  bool pdl;            // persistent kernel: programmatic dependent launch (flags bit 3)
  int64_t max_blocks_all;
  size_t flat_smem;
  int HG, n_hg, G, split_blocks, max_splits, stages;
  uint32_t stage_bytes;
  size_t tiles_bytes;
  size_t smem_bytes;
};

constexpr size_t kSmemBudget = 227 * 1024;

Geometry choose_geometry(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t bs,
                         int64_t max_blocks, const b200_launch_cfg* cfg) {
  Geometry g{};
  g.tma_path = false;
  if (Hkv <= 0 || Hq % Hkv != 0) return g;
  g.G = (int)(Hq / Hkv);
  int split = (cfg && cfg->split > 0) ? cfg->split : 64;
  if (split > kMaxSplitBlocks) split = kMaxSplitBlocks;
  g.split_blocks = split;
  g.max_splits = (int)((max_blocks + split - 1) / split);
  g.max_blocks_all = max_blocks;
  if (D != kD || !(g.G == 1 || g.G == 2 || g.G == 4 || g.G == 8) || bs > 256 || bs < 1 ||
      g.max_splits > kMaxSplits)
    return g;
  // Largest head group (<= 8 warps, or cfg->rows_per_cta) whose page keeps
  // >= 3 stages in budget.
  int HG = 0;
  const int hg_max = (cfg && cfg->rows_per_cta > 0 && cfg->rows_per_cta <= 8) ? cfg->rows_per_cta : 8;
  for (int cand = hg_max; cand >= 1; --cand) {
    if (Hkv % cand) continue;
    const uint64_t page = 2ull * bs * cand * kD * 2;
    if (page * 3 + 8192 <= kSmemBudget) {
      HG = cand;
      break;
    }
  }
  if (HG == 0) return g;
  g.HG = HG;
  g.n_hg = (int)(Hkv / HG);
  g.mma = (bs % 16 == 0) && !(cfg && (cfg->flags & 1));  // flags bit 0: force the CUDA-core consumer
  g.stage_bytes = (uint32_t)(2ull * bs * HG * kD * 2);
  int stages = (cfg && cfg->stages > 0) ? cfg->stages : 4;
  const size_t fixed = 2 * 8 * 16 + 2 * kMaxSplitBlocks * 4 + 64 + 1024;  // + alignment slack
  while (stages > 2 && (size_t)stages * g.stage_bytes + fixed > kSmemBudget) --stages;
  if ((size_t)stages * g.stage_bytes + fixed > kSmemBudget) return g;
  g.stages = stages;
  size_t tiles = (size_t)stages * g.stage_bytes;
  const size_t wts = (size_t)HG * g.G * g.max_splits * 4;
  if (wts > tiles) tiles = (wts + 127) / 128 * 128;
  g.tiles_bytes = tiles;
  g.smem_bytes = tiles + fixed;
  if (g.smem_bytes > kSmemBudget) return g;
  g.tma_path = true;
  // flags bit 1: keep the split kernel even where the persistent one applies
  const int64_t nseg = (int64_t)g.n_hg * B;
  g.flat = g.mma && nseg <= kFlatMaxSeg && !(cfg && (cfg->flags & 2));
  if (g.flat) {
    g.flat_grid = (cfg && cfg->tile_m > 0) ? cfg->tile_m : device_sm_count();
    // flags bit 2: equal static ranges only; tile_k: claimed percent; tile_n: entries per chunk
    g.dyn_pct = (cfg && (cfg->flags & 4)) ? 0 : (cfg && cfg->tile_k > 0 ? (cfg->tile_k < 90 ? cfg->tile_k : 90)
                                                                           : kFlatDynPct);
    g.chunk = (cfg && cfg->tile_n > 0) ? cfg->tile_n : kFlatChunk;
    g.pdl = cfg && (cfg->flags & 8);
    // default ring depth of the persistent kernel: about 128 KB of pages in
    // flight per SM (two 64 KB stages at 8 kv heads x 16 tokens: 188.8 us
    // against 192.9 us with three at 64 sequences, ctx U[512,8192]; a stream
    // with the math skipped also ran faster with two)
    const int split_stages = g.stages;
    if (!(cfg && cfg->stages > 0)) {
      int fs = (int)((128u * 1024u) / g.stage_bytes);
      if (fs < 2) fs = 2;
      if (fs < g.stages) g.stages = fs;
    }
    const size_t extra = (size_t)g.stages * (2 * 8 + sizeof(PageMeta)) + (size_t)(nseg + 1) * 8 +
                         (size_t)B * 8 + 64 * 4 + 128 * 4 + 16 + (size_t)g.HG * g.G * 32 * 4;
    g.flat_smem = (size_t)g.stages * g.stage_bytes + extra + 1024;
    if (g.flat_smem > kSmemBudget) {
      g.flat = false;
      g.stages = split_stages;
    }
  }
  return g;
}

template <typename T, typename IDX, int G>
int launch_tma(const void* q, const void* k_cache, const void* v_cache, const void* block_table,
               const void* ctx_len, void* out, int64_t B, int64_t Hq, int64_t Hkv,
               int64_t num_blocks, int64_t bs, int64_t max_blocks, float scale,
               const Geometry& geo, void* workspace, cudaStream_t stream) {
  CUtensorMap tk, tv;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (geo.mma) {
    // dims (d, token slot, head): boxes of 64 dims x bs tokens x HG heads land
    // as rows ordered (head, token) of 128 bytes, swizzled in 8-row atoms.
    const uint64_t dims[3] = {(uint64_t)kD, (uint64_t)(num_blocks * bs), (uint64_t)Hkv};
    const uint64_t strides[2] = {(uint64_t)Hkv * kD * 2, (uint64_t)kD * 2};
    const uint32_t box[3] = {64u, (uint32_t)bs, (uint32_t)geo.HG};
    int st = encode_tensor_map(&tk, dt, 3, k_cache, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = encode_tensor_map(&tv, dt, 3, v_cache, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  } else {
    const uint64_t dims[3] = {(uint64_t)kD, (uint64_t)Hkv, (uint64_t)(num_blocks * bs)};
    const uint64_t strides[2] = {(uint64_t)kD * 2, (uint64_t)Hkv * kD * 2};
    const uint32_t box[3] = {(uint32_t)kD, (uint32_t)geo.HG, (uint32_t)bs};
    int st = encode_tensor_map(&tk, dt, 3, k_cache, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = encode_tensor_map(&tv, dt, 3, v_cache, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
  }
  DecodeParams p;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.num_blocks = num_blocks;
  p.block_size = bs;
  p.max_blocks = max_blocks;
  p.HG = geo.HG;
  p.n_hg = geo.n_hg;
  p.split_blocks = geo.split_blocks;
  p.max_splits = geo.max_splits;
  p.stages = geo.stages;
  p.stage_bytes = geo.stage_bytes;
  p.tiles_bytes = (uint32_t)geo.tiles_bytes;
  p.qscale = scale * 1.4426950408889634f;
  // Workspace: [tickets (fixed region) | partials o | partials (m,l)].  The
  // ticket region sits at a fixed offset so that calls of different shapes
  // sharing one buffer always find their tickets at zero.
  const size_t n_rows = (size_t)B * Hq * geo.max_splits;
  int* tickets = static_cast<int*>(workspace);
  float* ws_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kTicketBytes);
  float* ws_ml = ws_o + n_rows * kD;
  if (geo.flat) {
    FlatParams fp;
    fp.B = B;
    fp.Hq = Hq;
    fp.Hkv = Hkv;
    fp.num_blocks = num_blocks;
    fp.block_size = bs;
    fp.max_blocks = max_blocks;
    fp.HG = geo.HG;
    fp.n_hg = geo.n_hg;
    fp.stages = geo.stages;
    fp.nseg = (int)(geo.n_hg * B);
    fp.dyn_pct = geo.dyn_pct;
    fp.chunk = geo.chunk;
    fp.max_chunks = kFlatChunksPerCta * geo.flat_grid;
    fp.stage_bytes = geo.stage_bytes;
    fp.qscale = scale * 1.4426950408889634f;
    auto fk = paged_decode_flat_kernel<T, IDX, G>;
    cudaError_t e = cudaFuncSetAttribute(fk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)geo.flat_smem);
    if (e != cudaSuccess) return launch_status(e);
    // flags bit 3: programmatic dependent launch -- the prologue (context
    // lengths, block-table prefix, barriers) may run while the previous
    // kernel in the stream finishes; the kernel waits for that grid
    // (griddepcontrol.wait) before its first q / KV read.  The caller
    // guarantees the previous kernel writes neither context_len nor
    // block_table (true for the decode-step append, which writes q_out and
    // the cache).
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)geo.flat_grid);
    lc.blockDim = dim3((unsigned)((geo.HG + 1) * 32));
    lc.dynamicSmemBytes = geo.flat_smem;
    lc.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = geo.pdl ? 1 : 0;
    e = cudaLaunchKernelEx(&lc, fk, tk, tv, static_cast<const T*>(q), static_cast<const IDX*>(block_table),
                           static_cast<const IDX*>(ctx_len), static_cast<T*>(out),
                           reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kTicketBytes),
                           static_cast<int*>(workspace), fp);
    if (e != cudaSuccess) return launch_status(e);
    return launch_status(cudaGetLastError());
  }
  auto kern = geo.mma ? paged_decode_kernel<T, IDX, G, true> : paged_decode_kernel<T, IDX, G, false>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)geo.smem_bytes);
  if (e != cudaSuccess) return launch_status(e);
  dim3 grid(geo.max_splits, (unsigned)B, geo.n_hg);
  kern<<<grid, (geo.HG + 1) * 32, geo.smem_bytes, stream>>>(
      tk, tv, static_cast<const T*>(q), static_cast<const IDX*>(block_table),
      static_cast<const IDX*>(ctx_len), static_cast<T*>(out), ws_o, ws_ml, tickets, p);
  return launch_status(cudaGetLastError());
}

size_t workspace_bytes_for(int64_t B, int64_t Hq, int64_t D, const Geometry& geo) {
  if (!geo.tma_path) return 0;
  if (geo.flat)
    return kTicketBytes + (size_t)flat_partial_rows(geo.flat_grid, (int64_t)geo.n_hg * B * geo.max_blocks_all,
                                                    geo.dyn_pct, geo.chunk, (int64_t)geo.HG * geo.G) *
                              (size_t)kFlatPitch * 4;
  const size_t n_rows = (size_t)B * Hq * geo.max_splits;
  return kTicketBytes + n_rows * (size_t)(D + 2) * 4;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" size_t b200_paged_attention_workspace_size(int64_t B, int64_t Hq, int64_t max_blocks,
                                                      int64_t block_size, int64_t D,
                                                      const b200_launch_cfg* cfg) {
  // The workspace depends on Hkv only through the head-group count, which
  // is bounded by Hq; size for the largest case.
  if (B <= 0 || Hq <= 0 || max_blocks <= 0 || block_size <= 0 || D <= 0) return 0;
  Geometry g{};
  int split = (cfg && cfg->split > 0) ? cfg->split : 64;
  if (split > kMaxSplitBlocks) split = kMaxSplitBlocks;
  g.tma_path = true;
  g.max_splits = (int)((max_blocks + split - 1) / split);
  const size_t split_need = workspace_bytes_for(B, Hq, D, g);
  // persistent kernel: two partial slots per range (one static range per CTA
  // plus the claimed chunks) of at most min(Hq, 64) heads; the chunks of all
  // head groups together hold at most B * max_blocks * Hq * pct / 100 head-pages
  const int64_t grid = (cfg && cfg->tile_m > 0) ? cfg->tile_m : device_sm_count();
  const int64_t heads = Hq < 64 ? Hq : 64;
  const int pct = (cfg && (cfg->flags & 4)) ? 0 : (cfg && cfg->tile_k > 0 ? (cfg->tile_k < 90 ? cfg->tile_k : 90)
                                                                            : kFlatDynPct);
  const int64_t ch = (cfg && cfg->tile_n > 0) ? cfg->tile_n : kFlatChunk;
  const int64_t dyn_heads = B * max_blocks * Hq * pct / 100 + heads;
  int64_t rows = 2 * ((grid + 4) * heads + dyn_heads / ch + 1);
  const int64_t rows_cap = 2 * (grid + kFlatChunksPerCta * grid + 4) * heads;
  if (pct > 0 && rows > rows_cap) rows = rows_cap;
  const size_t flat_need = kTicketBytes + (size_t)rows * (size_t)kFlatPitch * 4;
  return split_need > flat_need ? split_need : flat_need;
}

extern "C" int b200_paged_attention(const void* q, const void* k_cache, const void* v_cache,
                                    const void* block_table, const void* context_len, void* out,
                                    int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                    int64_t num_blocks, int64_t block_size, int64_t max_blocks,
                                    float scale, int32_t dtype, int32_t index_dtype,
                                    void* workspace, size_t workspace_bytes,
                                    const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("paged_attention")) return e;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || num_blocks <= 0 || block_size <= 0 ||
      max_blocks <= 0 || Hq % Hkv != 0)
    return B200_ERR_BAD_ARG;
  if (B == 0) return B200_OK;
  if (!q || !k_cache || !v_cache || !block_table || !context_len || !out) return B200_ERR_BAD_ARG;
  if (index_dtype != B200_I32 && index_dtype != B200_I64) return B200_ERR_UNSUPPORTED;
  if (B > 65535 || B * Hkv > (int64_t)(kTicketBytes / 4)) return B200_ERR_UNSUPPORTED;
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)D);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Geometry geo = choose_geometry(B, Hq, Hkv, D, block_size, max_blocks, cfg);
  const bool aligned = aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out);
  if (geo.tma_path && aligned && num_blocks * block_size < (1ll << 31)) {
    size_t need = workspace_bytes_for(B, Hq, D, geo);
    if (geo.flat && geo.dyn_pct > 0 && workspace_bytes < need) {
      // too little scratch for the claimed chunks' partials: equal static ranges
      geo.dyn_pct = 0;
      need = workspace_bytes_for(B, Hq, D, geo);
    }
    const bool single = geo.max_splits == 1 && !geo.flat;
    if (!single && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)))
      return B200_ERR_WORKSPACE;
    return B200_DISPATCH_HALF(dtype, [&] {
      auto run = [&](auto idx_tag) -> int {
        using IDX = decltype(idx_tag);
        switch (geo.G) {
          case 1: return launch_tma<scalar_t, IDX, 1>(q, k_cache, v_cache, block_table, context_len, out, B, Hq, Hkv, num_blocks, block_size, max_blocks, scale, geo, workspace, s);
          case 2: return launch_tma<scalar_t, IDX, 2>(q, k_cache, v_cache, block_table, context_len, out, B, Hq, Hkv, num_blocks, block_size, max_blocks, scale, geo, workspace, s);
          case 4: return launch_tma<scalar_t, IDX, 4>(q, k_cache, v_cache, block_table, context_len, out, B, Hq, Hkv, num_blocks, block_size, max_blocks, scale, geo, workspace, s);
          default: return launch_tma<scalar_t, IDX, 8>(q, k_cache, v_cache, block_table, context_len, out, B, Hq, Hkv, num_blocks, block_size, max_blocks, scale, geo, workspace, s);
        }
      };
      return index_dtype == B200_I32 ? run(int32_t{}) : run(int64_t{});
    });
  }
  if (D > 256) return B200_ERR_UNSUPPORTED;
  return B200_DISPATCH_HALF(dtype, [&] {
    auto run = [&](auto idx_tag) -> int {
      using IDX = decltype(idx_tag);
      dim3 grid((unsigned)Hq, (unsigned)B);
      paged_decode_generic_kernel<scalar_t, IDX><<<grid, 128, 0, s>>>(
          static_cast<const scalar_t*>(q), static_cast<const scalar_t*>(k_cache),
          static_cast<const scalar_t*>(v_cache), static_cast<const IDX*>(block_table),
          static_cast<const IDX*>(context_len), static_cast<scalar_t*>(out), Hq, Hkv, D,
          num_blocks, block_size, max_blocks, scale * 1.4426950408889634f);
      return launch_status(cudaGetLastError());
    };
    return index_dtype == B200_I32 ? run(int32_t{}) : run(int64_t{});
  });
}

// ---------------------------------------------------------------------------
// Allocation-free paged attention.
//
// Some callers of this library cannot allocate device memory: a host runtime
// that binds the library through a plain C FFI and only holds the device
// pointers handed to it (it has no device allocator of its own), or a serving
// loop that forbids cudaMalloc/cudaFree on its request path because those calls
// can synchronise the device and would fragment memory that another allocator
// owns.  b200_paged_attention needs a split-KV workspace from its caller;
// this entry point instead uses a fixed scratch array compiled into the
// library, so the caller passes only inputs and outputs.
//
// The scratch is kNoAllocScratchBytes of device memory per GPU that loads the
// library, held until the process exits.  Its device address is looked up once
// per device (cudaGetSymbolAddress with that device current) by the first call
// made on that device, so that first call should come before any stream
// capture.  Every call shares the one array and leaves its contents behind;
// the ticket counters that must start at zero are cleared at the start of each
// call.  Calls whose executions overlap on the GPU (different streams, or
// several host threads) race on the scratch and must be serialised by the
// caller.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (set up once).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return b200::launch_status(e);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return B200_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return b200::launch_status(e);
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return B200_OK;
}

}  // namespace

extern "C" int b200_paged_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                            const void* block_table, const void* context_len, void* out,
                                            int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t num_blocks,
                                            int64_t block_size, int64_t max_blocks, float scale,
                                            int32_t dtype, int32_t index_dtype, const b200_launch_cfg* cfg,
                                            void* stream) {
  if (int e = b200::injected_error("paged_attention_noalloc")) return e;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || num_blocks <= 0 || block_size <= 0 || max_blocks <= 0)
    return B200_ERR_BAD_ARG;
  const size_t need = b200_paged_attention_workspace_size(B, Hq, max_blocks, block_size, D, cfg);
  if (need > kNoAllocScratchBytes) {
    char msg[160];
    snprintf(msg, sizeof(msg),
             "paged_attention_noalloc: needs %zu bytes of scratch, the static scratch holds %zu", need,
             kNoAllocScratchBytes);
    b200::set_last_error_detail(msg);
    return B200_ERR_WORKSPACE;
  }
  if (B == 0) return B200_OK;
  void* scratch = nullptr;
  if (int st = noalloc_scratch(&scratch)) return st;
  // The whole ticket region starts at zero: the per-(sequence, head group)
  // merge tickets at its start and the claimed-chunk pool counters at its end.
  // Both re-arm themselves when a launch completes, but a launch whose bounded
  // wait gave up can leave them stale in this shared array; 256 KB is cheap.
  cudaError_t e = cudaMemsetAsync(scratch, 0, b200::kTicketBytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return b200::launch_status(e);
  return b200_paged_attention(q, k_cache, v_cache, block_table, context_len, out, B, Hq, Hkv, D, num_blocks,
                              block_size, max_blocks, scale, dtype, index_dtype, scratch, kNoAllocScratchBytes,
                              cfg, stream);
}
