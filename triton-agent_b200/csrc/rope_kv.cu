// RoPE and KV-cache append kernels.
//
// References (reference project paths):
//   rope            triton_agent/ops/rope/reference.py:17-25
//   kv_append       triton_agent/ops/kv_append/reference.py:27-40
//   paged_kv        triton_agent/ops/paged_kv/reference.py:11-27
//   rope_kv_append  triton_agent/ops/rope_kv_append/reference.py:26-47
//
// All four reduce to one pattern: move token rows of H heads x D elements
// from a source tensor to a destination row chosen by a slot index, rotating
// the two halves of each row (NeoX rotate-half) on the way when asked.  The
// destination row of (b, h, slot) is dst + b*d_b + h*d_h + slot*d_slot, which
// covers both the contiguous [B, H, L, D] cache (d_b = H*L*D, d_h = L*D,
// d_slot = D) and the paged [num_blocks, block_size, H, D] cache, where
// block*block_stride + offset*token_stride == slot*H*D (d_b = 0, d_h = D,
// d_slot = H*D).
//
// Rotation is done in fp32 with explicitly rounded multiplies and adds (no
// FMA contraction): y1 = (x1*c) - (x2*s), y2 = (x2*c) + (x1*s), each product
// and sum rounded to fp32, then one rounding to the storage dtype.  That is
// the exact sequence a CPU evaluating the reference formula in fp32 performs,
// so cache writes are bit-identical to it.
//
// When several (b, t) pairs name the same destination row the reference's
// sequential loop leaves the last one written.  Each CTA scans the slots
// after its own and skips its write if a later pair targets the same row, so
// the result does not depend on CTA scheduling.
#include "common.cuh"
#include "sm100.cuh"

namespace b200 {
namespace {

struct ScatterGeom {
  int64_t n_b, n_t, H, D;
  int64_t s_b, s_t, s_h;  // source element strides
  int64_t d_b, d_h, d_slot;  // destination element strides
  int64_t slot_hi;           // valid slots: [0, slot_hi)
  bool dst_has_batch;        // d_b != 0: collisions need equal b as well
};

template <typename CS>
__device__ __forceinline__ float cs_at(const CS* p, int64_t i) {
  return to_f32(p[i]);
}

// Rotates (ROPE) or copies one row of D elements.  The row's tpr threads
// call this with their index `r` in [0, tpr).
template <typename T, typename CS, bool ROPE, bool VEC>
__device__ __forceinline__ void move_row(const T* __restrict__ src, T* __restrict__ dst,
                                         const CS* __restrict__ cosr, const CS* __restrict__ sinr,
                                         int64_t D, int r, int tpr) {
  constexpr int VN = Vec<T>::N;
  if constexpr (ROPE) {
    const int64_t half = D / 2;
    if constexpr (VEC) {
      for (int64_t c = r; c < half / VN; c += tpr) {
        float x1[VN], x2[VN], y1[VN], y2[VN];
        load16_f32(src + c * VN, x1);
        load16_f32(src + half + c * VN, x2);
#pragma unroll
        for (int j = 0; j < VN; ++j) {
          const float cv = cs_at(cosr, c * VN + j), sv = cs_at(sinr, c * VN + j);
          y1[j] = __fsub_rn(__fmul_rn(x1[j], cv), __fmul_rn(x2[j], sv));
          y2[j] = __fadd_rn(__fmul_rn(x2[j], cv), __fmul_rn(x1[j], sv));
        }
        *reinterpret_cast<uint4*>(dst + c * VN) = pack16<T>(y1);
        *reinterpret_cast<uint4*>(dst + half + c * VN) = pack16<T>(y2);
      }
    } else {
      for (int64_t i = r; i < half; i += tpr) {
        const float a = to_f32(src[i]), b = to_f32(src[half + i]);
        const float cv = cs_at(cosr, i), sv = cs_at(sinr, i);
        dst[i] = from_f32<T>(__fsub_rn(__fmul_rn(a, cv), __fmul_rn(b, sv)));
        dst[half + i] = from_f32<T>(__fadd_rn(__fmul_rn(b, cv), __fmul_rn(a, sv)));
      }
    }
  } else {
    if constexpr (VEC) {
      for (int64_t c = r; c < D / VN; c += tpr)
        *reinterpret_cast<uint4*>(dst + c * VN) = *reinterpret_cast<const uint4*>(src + c * VN);
    } else {
      for (int64_t i = r; i < D; i += tpr) dst[i] = src[i];
    }
  }
}

// True if a later (b', t') in the reference's loop order (b outer, t inner)
// writes the same destination row as (b, t).  Cooperative over the CTA.
__device__ bool overwritten_later(const int64_t* __restrict__ slots, int64_t n_b, int64_t n_t,
                                  int64_t b, int64_t t, int64_t slot, bool dst_has_batch) {
  const int64_t me = b * n_t + t;
  const int64_t total = n_b * n_t;
  int hit = 0;
  if (dst_has_batch) {
    // Only the same batch row can collide; scan its remaining tokens.
    for (int64_t j = me + 1 + threadIdx.x; j < (b + 1) * n_t; j += blockDim.x)
      hit |= (slots[j] == slot);
  } else {
    for (int64_t j = me + 1 + threadIdx.x; j < total; j += blockDim.x) hit |= (slots[j] == slot);
  }
  return __syncthreads_or(hit) != 0;
}

// One CTA per (b, t); its threads cover the H head rows of that token.
// K (and optionally V) rows go to the cache; K is rotated when ROPE.
template <typename T, typename CS, bool ROPE, bool VEC>
__global__ void __launch_bounds__(1024) kv_scatter_kernel(
    const T* __restrict__ k_src, const T* __restrict__ v_src, T* __restrict__ k_dst,
    T* __restrict__ v_dst, const int64_t* __restrict__ slots, const CS* __restrict__ cos,
    const CS* __restrict__ sin, int64_t cs_row_stride, ScatterGeom g, int tpr) {
  const int64_t token = blockIdx.x;
  const int64_t b = token / g.n_t, t = token % g.n_t;
  const int64_t slot = slots[token];
  if (slot < 0 || slot >= g.slot_hi) return;  // uniform across the CTA
  if (overwritten_later(slots, g.n_b, g.n_t, b, t, slot, g.dst_has_batch)) return;
  const CS* cosr = ROPE ? cos + t * cs_row_stride : nullptr;
  const CS* sinr = ROPE ? sin + t * cs_row_stride : nullptr;
  const int rows_per_pass = blockDim.x / tpr;
  const int r = threadIdx.x % tpr;
  for (int64_t h = threadIdx.x / tpr; h < g.H; h += rows_per_pass) {
    const int64_t so = b * g.s_b + t * g.s_t + h * g.s_h;
    const int64_t dof = b * g.d_b + h * g.d_h + slot * g.d_slot;
    move_row<T, CS, ROPE, VEC>(k_src + so, k_dst + dof, cosr, sinr, g.D, r, tpr);
    if (v_src != nullptr)
      move_row<T, CS, false, VEC>(v_src + so, v_dst + dof, nullptr, nullptr, g.D, r, tpr);
  }
}

// Standalone RoPE over x [B, H, T, D] with cos/sin [T, D]; one row group
// (tpr threads) per (b, h, t) row.
template <typename T, typename CS, bool VEC>
__global__ void __launch_bounds__(256) rope_kernel(const T* __restrict__ x,
                                                   const CS* __restrict__ cos,
                                                   const CS* __restrict__ sin,
                                                   T* __restrict__ y, int64_t rows, int64_t T_len,
                                                   int64_t D, int tpr) {
  const int rows_per_cta = blockDim.x / tpr;
  const int64_t row = (int64_t)blockIdx.x * rows_per_cta + threadIdx.x / tpr;
  if (row >= rows) return;
  const int64_t t = row % T_len;
  move_row<T, CS, true, VEC>(x + row * D, y + row * D, cos + t * D, sin + t * D, D,
                             threadIdx.x % tpr, tpr);
}

// Fused decode step: per token, rotate its Hq query rows into q_out, rotate
// its Hkv key rows into k_cache at the token's slot and copy its Hkv value
// rows into v_cache at the same slot.  cos/sin rows are selected by the
// token's position.  One CTA per token.
template <typename T, typename CS, bool VEC>
__global__ void __launch_bounds__(1024) rope_kv_append_paged_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const int64_t* __restrict__ positions, const CS* __restrict__ cos,
    const CS* __restrict__ sin, int64_t cs_rows, const int64_t* __restrict__ slots,
    T* __restrict__ q_out, T* __restrict__ k_cache, T* __restrict__ v_cache, int64_t n_tok,
    int Hq, int Hkv, int64_t D, int64_t slot_hi, int tpr) {
  const int64_t t = blockIdx.x;
  int64_t pos = positions ? positions[t] : t;
  const bool pos_ok = pos >= 0 && pos < cs_rows;
  if (!pos_ok) pos = 0;  // rows with an out-of-table position are left untouched below
  const int64_t slot = slots[t];
  // pos_ok and slot are the same for every thread of the CTA, so the
  // CTA-wide scan below is entered by all threads or by none.
  bool write_kv = pos_ok && slot >= 0 && slot < slot_hi;
  if (write_kv) write_kv = !overwritten_later(slots, 1, n_tok, 0, t, slot, false);
  const CS* cosr = cos + pos * D;
  const CS* sinr = sin + pos * D;
  const int rows_per_pass = blockDim.x / tpr;
  const int r = threadIdx.x % tpr;
  const int nq = q ? Hq : 0;
  const int total_rows = nq + 2 * Hkv;
  for (int row = threadIdx.x / tpr; row < total_rows; row += rows_per_pass) {
    if (row < nq) {
      if (pos_ok)
        move_row<T, CS, true, VEC>(q + (t * Hq + row) * D, q_out + (t * Hq + row) * D, cosr,
                                   sinr, D, r, tpr);
    } else if (row < nq + Hkv) {
      const int h = row - nq;
      if (write_kv)
        move_row<T, CS, true, VEC>(k + (t * Hkv + h) * D, k_cache + (slot * Hkv + h) * D, cosr,
                                   sinr, D, r, tpr);
    } else {
      const int h = row - nq - Hkv;
      if (write_kv)
        move_row<T, CS, false, VEC>(v + (t * Hkv + h) * D, v_cache + (slot * Hkv + h) * D,
                                    nullptr, nullptr, D, r, tpr);
    }
  }
}

// Single-pass variant of the fused decode step for the vectorised case
// (every row group of tpr threads covers one row in one pass).  All loads
// that do not depend on each other are issued first -- the token's slot and
// position, the thread's two source chunks, the collision scan -- so the
// critical path is two memory round trips (source / position, then the
// cos/sin row) instead of one per dependent step.
template <typename CS, int VN>
__device__ __forceinline__ void load_cs(const CS* p, float* out) {
  if constexpr (sizeof(CS) == 4) {
#pragma unroll
    for (int c = 0; c < VN / 4; ++c) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p) + c);
      out[4 * c] = v.x;
      out[4 * c + 1] = v.y;
      out[4 * c + 2] = v.z;
      out[4 * c + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int c = 0; c < VN / 8; ++c) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p) + c);
      unpack16<CS>(raw, out + 8 * c);
    }
  }
}

// Slot ownership for many new tokens (prefill): owner[slot] = 1 + the last
// token writing it (atomic max; the reference's loop lets later tokens
// overwrite earlier ones).  The append kernel then writes a token's K/V rows
// only if it owns the slot, and the owner puts the entry back to 0, so the
// zero-filled table is ready for the next call -- an O(n) replacement of
// the per-token scan of all later slots (O(n^2) for a prefill).
__global__ void slot_owner_kernel(const int64_t* __restrict__ slots, int64_t n_tok, int64_t slot_hi,
                                  int* __restrict__ owner) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n_tok) return;
  const int64_t slot = slots[t];
  if (slot >= 0 && slot < slot_hi) atomicMax(&owner[slot], (int)(t + 1));
}

template <typename T, typename CS>
__global__ void __launch_bounds__(1024) rope_kv_append_paged_fast_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const int64_t* __restrict__ positions, const CS* __restrict__ cos,
    const CS* __restrict__ sin, int64_t cs_rows, const int64_t* __restrict__ slots,
    T* __restrict__ q_out, T* __restrict__ k_cache, T* __restrict__ v_cache, int64_t n_tok,
    int Hq, int Hkv, int64_t D, int64_t slot_hi, int tpr, int* __restrict__ owner) {
  // a dependent kernel launched with programmatic stream serialisation (the
  // paged decode) may start its prologue now; it waits for this grid's
  // completion before it reads q_out or the cache
  asm volatile("griddepcontrol.launch_dependents;");
  constexpr int VN = Vec<T>::N;
  const int64_t t = blockIdx.x;
  const int64_t half = D / 2;
  const int nq = q ? Hq : 0;
  const int total_rows = nq + 2 * Hkv;
  const int row = threadIdx.x / tpr;
  const int c = threadIdx.x % tpr;
  const bool active = row < total_rows && c < half / VN;
  // ---- independent loads
  int64_t pos = positions ? __ldg(&positions[t]) : t;
  const int64_t slot = __ldg(&slots[t]);
  const T* src = nullptr;
  if (row < nq) src = q + (t * Hq + row) * D;
  else if (row < nq + Hkv) src = k + (t * Hkv + (row - nq)) * D;
  else src = v + (t * Hkv + (row - nq - Hkv)) * D;
  uint4 a = make_uint4(0, 0, 0, 0), b = a;
  if (active) {
    a = __ldg(reinterpret_cast<const uint4*>(src + c * VN));
    b = __ldg(reinterpret_cast<const uint4*>(src + half + c * VN));
  }
  // collision: does a later token write the same slot? (ownership table, or
  // a scan of the later slots)
  int hit = 0;
  if (owner != nullptr) {
    if (threadIdx.x == 0 && slot >= 0 && slot < slot_hi) {
      const int o = *(volatile int*)&owner[slot];
      hit = o != (int)(t + 1);
      if (!hit) owner[slot] = 0;  // back to zero for the next call (later readers are not owners)
    }
  } else {
    for (int64_t j = t + 1 + threadIdx.x; j < n_tok; j += blockDim.x) hit |= (__ldg(&slots[j]) == slot);
  }
  const bool pos_ok = pos >= 0 && pos < cs_rows;
  if (!pos_ok) pos = 0;
  float cv[VN], sv[VN];
  const bool rope_row = row < nq + Hkv;
  if (active && rope_row) {
    load_cs<CS, VN>(cos + pos * D + c * VN, cv);
    load_cs<CS, VN>(sin + pos * D + c * VN, sv);
  }
  const bool later = __syncthreads_or(hit) != 0;
  const bool write_kv = pos_ok && slot >= 0 && slot < slot_hi && !later;
  if (!active) return;
  T* dst;
  if (row < nq) {
    if (!pos_ok) return;
    dst = q_out + (t * Hq + row) * D;
  } else {
    if (!write_kv) return;
    dst = (row < nq + Hkv) ? k_cache + (slot * Hkv + (row - nq)) * D
                           : v_cache + (slot * Hkv + (row - nq - Hkv)) * D;
  }
  if (rope_row) {
    float x1[VN], x2[VN], y1[VN], y2[VN];
    unpack16<T>(a, x1);
    unpack16<T>(b, x2);
    // every product rounded on its own, as eager fp32 does (scalar .rn
    // operations: the assembler contracts an fp32x2 multiply feeding an
    // fp32x2 add into one fused multiply-add)
#pragma unroll
    for (int j = 0; j < VN; ++j) {
      y1[j] = __fsub_rn(__fmul_rn(x1[j], cv[j]), __fmul_rn(x2[j], sv[j]));
      y2[j] = __fadd_rn(__fmul_rn(x2[j], cv[j]), __fmul_rn(x1[j], sv[j]));
    }
    *reinterpret_cast<uint4*>(dst + c * VN) = pack16<T>(y1);
    *reinterpret_cast<uint4*>(dst + half + c * VN) = pack16<T>(y2);
  } else {
    *reinterpret_cast<uint4*>(dst + c * VN) = a;
    *reinterpret_cast<uint4*>(dst + half + c * VN) = b;
  }
}

// Prefill-size variant (ownership table given): a thread covers the same
// 16-byte column chunk c of RPT rows of one token (rows g, g + G, ...), so
// the token's cos/sin chunk is loaded once per thread instead of once per
// row, and the per-thread setup (slot, position, addresses) is shared by RPT
// rows.  One or more tokens per CTA (at most 256 threads); every source load
// of the thread is issued before the ownership check and the barrier.
template <typename T, typename CS, int RPT>
__global__ void __launch_bounds__(256) rope_kv_append_paged_rows_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const int64_t* __restrict__ positions, const CS* __restrict__ cos,
    const CS* __restrict__ sin, int64_t cs_rows, const int64_t* __restrict__ slots,
    T* __restrict__ q_out, T* __restrict__ k_cache, T* __restrict__ v_cache, int64_t n_tok,
    int Hq, int Hkv, int64_t D, int64_t slot_hi, int cpr, int groups, int* __restrict__ owner) {
  constexpr int VN = Vec<T>::N;
  __shared__ int s_hit[32];
  const int tpt = cpr * groups;  // threads per token
  const int lt = threadIdx.x / tpt;
  const int rem = threadIdx.x - lt * tpt;
  const int c = rem % cpr, g = rem / cpr;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / tpt) + lt;
  const bool live = t < n_tok && lt < 32;
  const int64_t half = D / 2;
  const int nq = q ? Hq : 0;
  const int total_rows = nq + 2 * Hkv;
  int64_t pos = 0, slot = -1;
  uint4 a[RPT], b[RPT];
  if (live) {
    pos = positions ? __ldg(&positions[t]) : t;
    slot = __ldg(&slots[t]);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int row = g + groups * i;
      if (row < total_rows) {
        const T* src = row < nq ? q + (t * Hq + row) * D
                                : (row < nq + Hkv ? k + (t * Hkv + (row - nq)) * D
                                                  : v + (t * Hkv + (row - nq - Hkv)) * D);
        a[i] = __ldg(reinterpret_cast<const uint4*>(src + c * VN));
        b[i] = __ldg(reinterpret_cast<const uint4*>(src + half + c * VN));
      }
    }
    if (rem == 0) {
      int hit = 0;
      if (slot >= 0 && slot < slot_hi) {
        const int o = *(volatile int*)&owner[slot];
        hit = o != (int)(t + 1);
        if (!hit) owner[slot] = 0;  // back to zero for the next call (later readers are not owners)
      }
      s_hit[lt] = hit;
    }
  }
  const bool pos_ok = pos >= 0 && pos < cs_rows;
  if (!pos_ok) pos = 0;
  float cv[VN], sv[VN];
  if (live && g < nq + Hkv) {  // the thread has at least one rotated row (row g)
    load_cs<CS, VN>(cos + pos * D + c * VN, cv);
    load_cs<CS, VN>(sin + pos * D + c * VN, sv);
  }
  __syncthreads();
  if (!live) return;
  const bool write_kv = pos_ok && slot >= 0 && slot < slot_hi && !s_hit[lt];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int row = g + groups * i;
    if (row >= total_rows) continue;
    T* dst;
    if (row < nq) {
      if (!pos_ok) continue;
      dst = q_out + (t * Hq + row) * D;
    } else {
      if (!write_kv) continue;
      dst = (row < nq + Hkv) ? k_cache + (slot * Hkv + (row - nq)) * D
                             : v_cache + (slot * Hkv + (row - nq - Hkv)) * D;
    }
    if (row < nq + Hkv) {
      float x1[VN], x2[VN], y1[VN], y2[VN];
      unpack16<T>(a[i], x1);
      unpack16<T>(b[i], x2);
      // every product rounded on its own, as eager fp32 does
#pragma unroll
      for (int j = 0; j < VN; ++j) {
        y1[j] = __fsub_rn(__fmul_rn(x1[j], cv[j]), __fmul_rn(x2[j], sv[j]));
        y2[j] = __fadd_rn(__fmul_rn(x2[j], cv[j]), __fmul_rn(x1[j], sv[j]));
      }
      *reinterpret_cast<uint4*>(dst + c * VN) = pack16<T>(y1);
      *reinterpret_cast<uint4*>(dst + half + c * VN) = pack16<T>(y2);
    } else {
      *reinterpret_cast<uint4*>(dst + c * VN) = a[i];
      *reinterpret_cast<uint4*>(dst + half + c * VN) = b[i];
    }
  }
}

int threads_for(int64_t rows, int tpr, const b200_launch_cfg* cfg) {
  int64_t want = rows * tpr;
  int threads = (cfg && cfg->threads > 0) ? cfg->threads : (int)((want + 31) / 32 * 32);
  if (threads > 1024) threads = 1024;
  if (threads < tpr) threads = ((tpr + 31) / 32) * 32;
  if (threads > 1024) threads = 1024;
  threads = (threads / tpr) * tpr;  // whole row groups only
  if (threads == 0) threads = tpr;
  return threads;
}

template <typename T>
bool vec_ok_rows(const void* const* ptrs, int n, const int64_t* strides, int ns, int64_t chunk) {
  for (int i = 0; i < n; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  for (int i = 0; i < ns; ++i)
    if ((strides[i] * (int64_t)sizeof(T)) % 16 != 0) return false;
  return (chunk * (int64_t)sizeof(T)) % 16 == 0;
}

template <typename T, typename CS, bool ROPE>
int launch_scatter(const void* k_src, const void* v_src, void* k_dst, void* v_dst,
                   const int64_t* slots, const void* cos, const void* sin, int64_t cs_row_stride,
                   ScatterGeom g, const b200_launch_cfg* cfg, cudaStream_t s) {
  constexpr int VN = Vec<T>::N;
  const void* ptrs[4] = {k_src, v_src, k_dst, v_dst};
  const int64_t strides[6] = {g.s_b, g.s_t, g.s_h, g.d_b, g.d_h, g.d_slot};
  const int64_t chunk = ROPE ? g.D / 2 : g.D;
  const bool vec = (!ROPE || g.D % 2 == 0) && vec_ok_rows<T>(ptrs, 4, strides, 6, chunk) &&
                   chunk % VN == 0;
  const int64_t per_row = vec ? chunk / VN : chunk;
  const int tpr = (int)(per_row >= 32 ? 32 : (per_row < 1 ? 1 : per_row));
  const int threads = threads_for(g.H, tpr, cfg);
  const int64_t grid = g.n_b * g.n_t;
  if (grid > 0x7fffffffLL) return B200_ERR_UNSUPPORTED;
  auto* ks = static_cast<const T*>(k_src);
  auto* vs = static_cast<const T*>(v_src);
  auto* kd = static_cast<T*>(k_dst);
  auto* vd = static_cast<T*>(v_dst);
  auto* cp = static_cast<const CS*>(cos);
  auto* sp = static_cast<const CS*>(sin);
  if (vec)
    kv_scatter_kernel<T, CS, ROPE, true>
        <<<(unsigned)grid, threads, 0, s>>>(ks, vs, kd, vd, slots, cp, sp, cs_row_stride, g, tpr);
  else
    kv_scatter_kernel<T, CS, ROPE, false>
        <<<(unsigned)grid, threads, 0, s>>>(ks, vs, kd, vd, slots, cp, sp, cs_row_stride, g, tpr);
  return launch_status(cudaGetLastError());
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_kv_append(void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                              const int64_t* slot_mapping, int64_t B, int64_t H, int64_t L,
                              int64_t T_new, int64_t D, int32_t dtype,
                              const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("kv_append")) return e;
  if (B < 0 || H <= 0 || L <= 0 || T_new < 0 || D <= 0) return B200_ERR_BAD_ARG;
  if (B == 0 || T_new == 0) return B200_OK;
  if (!k_cache || !v_cache || !k_new || !v_new || !slot_mapping) return B200_ERR_BAD_ARG;
  ScatterGeom g{B, T_new, H, D, H * T_new * D, D, T_new * D, H * L * D, L * D, D, L, true};
  return B200_DISPATCH_FLOAT(dtype, [&] {
    return launch_scatter<scalar_t, scalar_t, false>(k_new, v_new, k_cache, v_cache, slot_mapping,
                                                     nullptr, nullptr, 0, g, cfg,
                                                     static_cast<cudaStream_t>(stream));
  });
}

extern "C" int b200_paged_kv(void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                             const int64_t* slot_mapping, int64_t B, int64_t T_new, int64_t H,
                             int64_t D, int64_t num_blocks, int64_t block_size, int32_t dtype,
                             const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("paged_kv")) return e;
  if (B < 0 || T_new < 0 || H <= 0 || D <= 0 || num_blocks <= 0 || block_size <= 0)
    return B200_ERR_BAD_ARG;
  if (B == 0 || T_new == 0) return B200_OK;
  if (!k_cache || !v_cache || !k_new || !v_new || !slot_mapping) return B200_ERR_BAD_ARG;
  ScatterGeom g{B, T_new, H, D, T_new * H * D, H * D, D, 0, D, H * D, num_blocks * block_size,
                false};
  return B200_DISPATCH_FLOAT(dtype, [&] {
    return launch_scatter<scalar_t, scalar_t, false>(k_new, v_new, k_cache, v_cache, slot_mapping,
                                                     nullptr, nullptr, 0, g, cfg,
                                                     static_cast<cudaStream_t>(stream));
  });
}

extern "C" int b200_rope_kv_append(const void* k_new, const void* cos, const void* sin,
                                   void* k_cache, const int64_t* slot_mapping, int64_t B,
                                   int64_t H, int64_t L, int64_t T_new, int64_t D, int32_t dtype,
                                   int32_t cs_dtype, const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("rope_kv_append")) return e;
  if (B < 0 || H <= 0 || L <= 0 || T_new < 0 || D <= 0 || D % 2 != 0) return B200_ERR_BAD_ARG;
  if (B == 0 || T_new == 0) return B200_OK;
  if (!k_new || !cos || !sin || !k_cache || !slot_mapping) return B200_ERR_BAD_ARG;
  ScatterGeom g{B, T_new, H, D, H * T_new * D, D, T_new * D, H * L * D, L * D, D, L, true};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cs_dtype == dtype) {
    return B200_DISPATCH_FLOAT(dtype, [&] {
      return launch_scatter<scalar_t, scalar_t, true>(k_new, nullptr, k_cache, nullptr,
                                                      slot_mapping, cos, sin, D, g, cfg, s);
    });
  }
  if (cs_dtype == B200_F32) {
    return B200_DISPATCH_FLOAT(dtype, [&] {
      return launch_scatter<scalar_t, float, true>(k_new, nullptr, k_cache, nullptr, slot_mapping,
                                                   cos, sin, D, g, cfg, s);
    });
  }
  return B200_ERR_UNSUPPORTED;
}

namespace {
template <typename T, typename CS>
int launch_rope(const void* x, const void* cos, const void* sin, void* y, int64_t rows,
                int64_t T_len, int64_t D, const b200_launch_cfg* cfg, cudaStream_t s) {
  constexpr int VN = Vec<T>::N;
  const int64_t half = D / 2;
  const bool vec = aligned16(x) && aligned16(y) && (half * (int64_t)sizeof(T)) % 16 == 0 &&
                   half % VN == 0;
  const int64_t per_row = vec ? half / VN : half;
  const int tpr = (int)(per_row >= 32 ? 32 : (per_row < 1 ? 1 : per_row));
  int threads = (cfg && cfg->threads > 0) ? cfg->threads : 256;
  if (threads > 256) threads = 256;
  threads = (threads / tpr) * tpr;
  if (threads == 0) threads = tpr;
  const int rows_per_cta = threads / tpr;
  const int64_t grid = (rows + rows_per_cta - 1) / rows_per_cta;
  if (grid > 0x7fffffffLL) return B200_ERR_UNSUPPORTED;
  auto* xp = static_cast<const T*>(x);
  auto* yp = static_cast<T*>(y);
  auto* cp = static_cast<const CS*>(cos);
  auto* sp = static_cast<const CS*>(sin);
  if (vec)
    rope_kernel<T, CS, true><<<(unsigned)grid, threads, 0, s>>>(xp, cp, sp, yp, rows, T_len, D, tpr);
  else
    rope_kernel<T, CS, false><<<(unsigned)grid, threads, 0, s>>>(xp, cp, sp, yp, rows, T_len, D, tpr);
  return launch_status(cudaGetLastError());
}
}  // namespace

extern "C" int b200_rope(const void* x, const void* cos, const void* sin, void* y, int64_t B,
                         int64_t H, int64_t T, int64_t D, int32_t dtype, int32_t cs_dtype,
                         const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("rope")) return e;
  if (B < 0 || H < 0 || T < 0 || D <= 0 || D % 2 != 0) return B200_ERR_BAD_ARG;
  const int64_t rows = B * H * T;
  if (rows == 0) return B200_OK;
  if (!x || !cos || !sin || !y) return B200_ERR_BAD_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cs_dtype == dtype) {
    return B200_DISPATCH_FLOAT(dtype, [&] {
      return launch_rope<scalar_t, scalar_t>(x, cos, sin, y, rows, T, D, cfg, s);
    });
  }
  if (cs_dtype == B200_F32) {
    return B200_DISPATCH_FLOAT(dtype, [&] {
      return launch_rope<scalar_t, float>(x, cos, sin, y, rows, T, D, cfg, s);
    });
  }
  return B200_ERR_UNSUPPORTED;
}

namespace {
template <typename T, typename CS>
int launch_fused(const void* q, const void* k, const void* v, const int64_t* positions,
                 const void* cos, const void* sin, int64_t cs_rows, const int64_t* slots,
                 void* q_out, void* k_cache, void* v_cache, int64_t n_tok, int64_t Hq,
                 int64_t Hkv, int64_t D, int64_t slot_hi, const b200_launch_cfg* cfg,
                 cudaStream_t s, int* owner) {
  constexpr int VN = Vec<T>::N;
  const int64_t half = D / 2;
  const void* ptrs[6] = {q, k, v, q_out, k_cache, v_cache};
  bool vec = half % VN == 0 && (half * (int64_t)sizeof(T)) % 16 == 0;
  for (auto p : ptrs)
    if (p && !aligned16(p)) vec = false;
  const int64_t per_row = vec ? half / VN : half;
  const int tpr = (int)(per_row >= 32 ? 32 : (per_row < 1 ? 1 : per_row));
  const int64_t rows = (q ? Hq : 0) + 2 * Hkv;
  const int threads = threads_for(rows, tpr, cfg);
  auto* qp = static_cast<const T*>(q);
  auto* kp = static_cast<const T*>(k);
  auto* vp = static_cast<const T*>(v);
  auto* qo = static_cast<T*>(q_out);
  auto* kc = static_cast<T*>(k_cache);
  auto* vc = static_cast<T*>(v_cache);
  auto* cp = static_cast<const CS*>(cos);
  auto* sp = static_cast<const CS*>(sin);
  const bool cs_vec = aligned16(cos) && aligned16(sin) && (D * (int64_t)sizeof(CS)) % 16 == 0 &&
                      (VN * (int64_t)sizeof(CS)) % 16 == 0;
  if (vec && cs_vec && rows * tpr <= 1024 && !(cfg && cfg->threads > 0)) {
    const int th = (int)(((rows * tpr) + 31) / 32 * 32);
    if (owner != nullptr) {
      slot_owner_kernel<<<(unsigned)((n_tok + 255) / 256), 256, 0, s>>>(slots, n_tok, slot_hi, owner);
      if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) return launch_status(e);
    }
    // prefill sizes (ownership table): RPT rows per thread, several tokens per
    // CTA; rows kernel when the row count splits into <= 8 row groups of
    // 16-byte chunks that fit a 256-thread CTA
    // rows per thread: cfg rows_per_cta (2, 3, 4, 6, 8 or 12), default 4
    // (measured at 16384 tokens, 48 rows: 4 -> 75 us, 6 -> 85, 8 -> 89, 12 -> 101)
    const int rpt = (cfg && cfg->rows_per_cta > 0) ? cfg->rows_per_cta : 4;
    if (owner != nullptr && half / VN <= 32 &&
        (rpt == 2 || rpt == 3 || rpt == 4 || rpt == 6 || rpt == 8 || rpt == 12)) {
      const int cpr = (int)(half / VN);
      const int groups = (int)((rows + rpt - 1) / rpt);
      const int tpt = cpr * groups;
      if (tpt <= 256 && 256 / tpt <= 32) {  // at most 32 tokens per CTA (s_hit)
        const int tpc = 256 / tpt;
        const int64_t grid = (n_tok + tpc - 1) / tpc;
        auto go = [&](auto rpt_tag) {
          rope_kv_append_paged_rows_kernel<T, CS, decltype(rpt_tag)::value><<<(unsigned)grid, tpc * tpt, 0, s>>>(
              qp, kp, vp, positions, cp, sp, cs_rows, slots, qo, kc, vc, n_tok, (int)Hq, (int)Hkv, D, slot_hi, cpr,
              groups, owner);
        };
        if (rpt == 2) go(std::integral_constant<int, 2>{});
        else if (rpt == 3) go(std::integral_constant<int, 3>{});
        else if (rpt == 4) go(std::integral_constant<int, 4>{});
        else if (rpt == 6) go(std::integral_constant<int, 6>{});
        else if (rpt == 8) go(std::integral_constant<int, 8>{});
        else go(std::integral_constant<int, 12>{});
        return launch_status(cudaGetLastError());
      }
    }
    rope_kv_append_paged_fast_kernel<T, CS><<<(unsigned)n_tok, th, 0, s>>>(
        qp, kp, vp, positions, cp, sp, cs_rows, slots, qo, kc, vc, n_tok, (int)Hq, (int)Hkv, D, slot_hi, tpr,
        owner);
    return launch_status(cudaGetLastError());
  }
  if (vec)
    rope_kv_append_paged_kernel<T, CS, true><<<(unsigned)n_tok, threads, 0, s>>>(
        qp, kp, vp, positions, cp, sp, cs_rows, slots, qo, kc, vc, n_tok, (int)Hq, (int)Hkv, D,
        slot_hi, tpr);
  else
    rope_kv_append_paged_kernel<T, CS, false><<<(unsigned)n_tok, threads, 0, s>>>(
        qp, kp, vp, positions, cp, sp, cs_rows, slots, qo, kc, vc, n_tok, (int)Hq, (int)Hkv, D,
        slot_hi, tpr);
  return launch_status(cudaGetLastError());
}
}  // namespace

extern "C" int b200_rope_kv_append_paged_ws(const void* q, const void* k, const void* v,
                                            const int64_t* positions, const void* cos, const void* sin,
                                            int64_t cs_rows, const int64_t* slot_mapping, void* q_out,
                                            void* k_cache, void* v_cache, int64_t T, int64_t Hq, int64_t Hkv,
                                            int64_t D, int64_t num_blocks, int64_t block_size, int32_t dtype,
                                            int32_t cs_dtype, int32_t* slot_owner, int64_t owner_entries,
                                            const b200_launch_cfg* cfg, void* stream) {
  if (int e = injected_error("rope_kv_append_paged")) return e;
  if (T < 0 || Hkv <= 0 || D <= 0 || D % 2 != 0 || num_blocks <= 0 || block_size <= 0 ||
      cs_rows <= 0)
    return B200_ERR_BAD_ARG;
  if ((q == nullptr) != (q_out == nullptr)) return B200_ERR_BAD_ARG;
  if (q && Hq <= 0) return B200_ERR_BAD_ARG;
  if (T == 0) return B200_OK;
  if (!k || !v || !cos || !sin || !slot_mapping || !k_cache || !v_cache) return B200_ERR_BAD_ARG;
  if (T > 0x7fffffffLL - 1 || Hq > 4096 || Hkv > 4096) return B200_ERR_UNSUPPORTED;
  const int64_t slot_hi = num_blocks * block_size;
  if (slot_owner != nullptr && owner_entries < slot_hi) return B200_ERR_WORKSPACE;
  int* owner = reinterpret_cast<int*>(slot_owner);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cs_dtype == dtype) {
    return B200_DISPATCH_FLOAT(dtype, [&] {
      return launch_fused<scalar_t, scalar_t>(q, k, v, positions, cos, sin, cs_rows, slot_mapping,
                                              q_out, k_cache, v_cache, T, Hq, Hkv, D, slot_hi,
                                              cfg, s, owner);
    });
  }
  if (cs_dtype == B200_F32) {
    return B200_DISPATCH_FLOAT(dtype, [&] {
      return launch_fused<scalar_t, float>(q, k, v, positions, cos, sin, cs_rows, slot_mapping,
                                           q_out, k_cache, v_cache, T, Hq, Hkv, D, slot_hi, cfg,
                                           s, owner);
    });
  }
  return B200_ERR_UNSUPPORTED;
}

extern "C" int b200_rope_kv_append_paged(const void* q, const void* k, const void* v,
                                         const int64_t* positions, const void* cos,
                                         const void* sin, int64_t cs_rows,
                                         const int64_t* slot_mapping, void* q_out, void* k_cache,
                                         void* v_cache, int64_t T, int64_t Hq, int64_t Hkv,
                                         int64_t D, int64_t num_blocks, int64_t block_size,
                                         int32_t dtype, int32_t cs_dtype,
                                         const b200_launch_cfg* cfg, void* stream) {
  return b200_rope_kv_append_paged_ws(q, k, v, positions, cos, sin, cs_rows, slot_mapping, q_out, k_cache,
                                      v_cache, T, Hq, Hkv, D, num_blocks, block_size, dtype, cs_dtype, nullptr,
                                      0, cfg, stream);
}
