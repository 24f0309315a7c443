/*
 * b200ops.h -- C ABI of libb200ops.so, the sm_100a backend for the
 * Triton-Agent operator library (triton_agent/ops in the reference project).
 *
 * Every entry point:
 *   - takes plain device pointers, element counts and element strides
 *     (no torch types), plus a cudaStream_t passed as void*;
 *   - launches asynchronously on that stream and never synchronises;
 *   - allocates nothing: outputs and any workspace are passed in by the caller;
 *   - returns B200_OK (0) or a negative b200_status; it never aborts or traps.
 *
 * Dtype codes are the b200_dtype values below.  Layouts are row-major and
 * contiguous unless a stride argument says otherwise.
 *
 * Each declaration cites the reference function (file:line, paths inside the
 * reference project) whose behaviour it reproduces.
 */
#ifndef B200OPS_H
#define B200OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
typedef enum b200_status {
  B200_OK = 0,
  B200_ERR_BAD_ARG = -1,         /* null pointer, non-positive size, bad stride */
  B200_ERR_UNSUPPORTED = -2,     /* dtype / shape combination not implemented */
  B200_ERR_LAUNCH = -3,          /* cudaLaunch* or cudaFuncSetAttribute failed */
  B200_ERR_DEVICE_TIMEOUT = -4,  /* a bounded device-side wait gave up */
  B200_ERR_WORKSPACE = -5,       /* caller workspace missing or too small */
  B200_ERR_NO_DEVICE = -6,       /* no sm_100 device current */
  B200_ERR_INJECTED = -7,        /* host-side fault injection (B200OPS_INJECT_ERROR) */
  B200_ERR_ALIGNMENT = -8        /* pointer / leading dimension not 16-byte aligned */
} b200_status;

/* ---- dtype codes ------------------------------------------------------- */
typedef enum b200_dtype {
  B200_F32 = 0,
  B200_F16 = 1,
  B200_BF16 = 2,
  B200_I8 = 3,
  B200_I32 = 4,
  B200_I64 = 5
} b200_dtype;

/* ---- launch / tile parameters chosen by the tuner ----------------------
 * A zero field means "use the kernel's default".  Each op reads only the
 * fields it documents.  This is the CUDA-side meaning of the reference's
 * OpAction (core/spec.py:34-61): block_d/num_warps/num_stages become
 * threads, tiles and pipeline depth. */
typedef struct b200_launch_cfg {
  int32_t threads;      /* threads per CTA */
  int32_t rows_per_cta; /* rows (tokens, sequences) handled by one CTA */
  int32_t stages;       /* shared-memory pipeline depth */
  int32_t split;        /* KV split (paged decode: blocks per split) / split-K */
  int32_t tile_m;       /* GEMM / attention tile sizes */
  int32_t tile_n;
  int32_t tile_k;
  int32_t flags;        /* op-specific bit flags (documented per op) */
} b200_launch_cfg;

/* ---- library info -------------------------------------------------------- */
const char* b200_status_string(int status);
/* Version as major*10000 + minor*100 + patch. */
int b200_version(void);
/* Names of the kernels compiled into this library, one per line. */
const char* b200_kernel_list(void);
/* Text of the last host-side failure on the calling thread (CUDA error string,
 * injected-error note), or "" if none. */
const char* b200_last_error_detail(void);
/* Copies the per-library device error word (set by bounded waits that gave
 * up: 1-4 waits inside a CTA, 6 a cross-GPU flag wait) into *out and clears
 * it.  Synchronises the given stream. */
int b200_read_device_error(int32_t* out, void* stream);
/* Tunable launch parameters of an op, as JSON text:
 *   {"op": ..., "rows": ..., "kernel": <kernel the default dispatch selects>,
 *    "sm_count": ..., "fields": {<b200_launch_cfg field>: {"values": [...],
 *    "meaning": ...}, ...}}
 * listing only the fields that kernel reads, each with the values it accepts
 * (0 = the kernel's default).  `rows` selects the kernel where the op has
 * several (quant_matmul: M <= 64 streaming, <= 128 one-SM, else CTA pairs;
 * rope_kv_append_paged: tokens; 0 = the op's benchmark shape).  Op names are
 * those of triton_agent/ops (the registry keys of core/registry.py); NULL for
 * an unknown op.  The text stays valid until the next call on the same
 * thread.  Replaces the Triton-config search space the reference's tuner
 * reads from contract.yaml (core/contract.py:62-69, cli.py:281-293). */
const char* b200_query_config_space(const char* op, int64_t rows);
/* Limit, in microseconds of GPU global time, of the cross-GPU flag waits of
 * b200_int8_gemm_allgather (0 restores the default of 2 s).  Process-wide;
 * read at each launch.  A wait that runs out records code 6 in the device
 * error word and its kernel returns.  No counterpart in the reference (it has
 * no multi-GPU path). */
int b200_set_peer_wait_timeout_us(int64_t us);

/* ---- rmsnorm ------------------------------------------------------------
 * Replaces triton_agent/ops/rmsnorm/reference.py:6-18
 *   y = x * rsqrt(mean(x^2, -1) + eps) * weight
 * x, y: [rows, D] of `dtype` (F32/F16/BF16); weight: [D] of `weight_dtype`.
 * Accumulates in fp32, rounds once to `dtype`.
 * cfg: threads (CTA size, 64..1024). */
int b200_rmsnorm(const void* x, const void* weight, void* y, int64_t rows,
                 int64_t D, float eps, int32_t dtype, int32_t weight_dtype,
                 const b200_launch_cfg* cfg, void* stream);

/* ---- rmsnorm fused with the INT8 activation quantiser ----------------------
 * Composition of triton_agent/ops/rmsnorm/reference.py:17-18 and the row
 * quantiser of triton_agent/ops/quant_matmul/reference.py:16-19 (the step
 * before the INT8 GEMM in a decode layer): y = rmsnorm(x, weight) rounded to
 * `dtype` (as b200_rmsnorm writes it), scale[r] = max|y[r,:]| / 127 rounded
 * to `dtype` (0 -> 1e-6), q = clamp(round_half_even(y / scale), -127, 127).
 * The codes and scales are bit-identical to b200_quantize_int8 (row mode)
 * of the normalised rows computed here (returned in y when non-null); those
 * equal b200_rmsnorm's output up to the order of the fp32 sum of squares.
 * One pass over x.  q: [rows, D] int8 (8-byte aligned); scale: [rows]
 * f32; y (nullable): [rows, D] of `dtype`.  Needs D % (16 / sizeof(dtype))
 * == 0 and 16-byte aligned x/weight/y (B200_ERR_ALIGNMENT otherwise).
 * Default for 16-bit rows of D = 1024, 2048 or 4096: warp rows (one warp a
 * row, two for 4096; each warp's next row copied into shared memory while
 * the current one is computed).  cfg: threads (CTA size of the CTA kernels,
 * multiple of 32, default about D / 32 for 16-bit dtypes; giving it selects
 * them), rows_per_cta (1, 2 or 4 rows per CTA; more than one only with at
 * most 256 threads; default 1); flags bit 0: one CTA per row; bit 1: the
 * persistent CTA row loop (16-bit rows of two or four 16-byte vectors per
 * thread, at most 256 threads) instead of warp rows; bit 2: warp rows
 * without the prefetch. */
int b200_rmsnorm_quant_int8(const void* x, const void* weight, int8_t* q, float* scale,
                            void* y, int64_t rows, int64_t D, float eps, int32_t dtype,
                            int32_t weight_dtype, const b200_launch_cfg* cfg, void* stream);


/* ---- RoPE (NeoX rotate-half) ---------------------------------------------
 * Replaces triton_agent/ops/rope/reference.py:6-25
 * x, y: [B, H, T, D]; cos, sin: [T, D] of `cs_dtype` (first D/2 columns used).
 * y1 = x1*c - x2*s ; y2 = x2*c + x1*s  (fp32, rounded once). */
int b200_rope(const void* x, const void* cos, const void* sin, void* y,
              int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype,
              int32_t cs_dtype, const b200_launch_cfg* cfg, void* stream);

/* ---- contiguous KV append (in place) -------------------------------------
 * Replaces triton_agent/ops/kv_append/reference.py:10-40
 * k_cache, v_cache: [B, H, L, D]; k_new, v_new: [B, H, T_new, D];
 * slot_mapping: [B, T_new] int64.  Rows whose slot is outside [0, L) are
 * skipped.  Writes in place (the reference returns a modified clone). */
int b200_kv_append(void* k_cache, void* v_cache, const void* k_new,
                   const void* v_new, const int64_t* slot_mapping, int64_t B,
                   int64_t H, int64_t L, int64_t T_new, int64_t D,
                   int32_t dtype, const b200_launch_cfg* cfg, void* stream);

/* ---- paged KV append (in place) ------------------------------------------
 * Replaces triton_agent/ops/paged_kv/reference.py:6-27
 * k_cache, v_cache: [num_blocks, block_size, H, D]; k_new, v_new:
 * [B, T_new, H, D]; slot_mapping: [B, T_new] int64 global slots,
 * block = slot / block_size, offset = slot % block_size; rows whose block is
 * outside [0, num_blocks) are skipped. */
int b200_paged_kv(void* k_cache, void* v_cache, const void* k_new,
                  const void* v_new, const int64_t* slot_mapping, int64_t B,
                  int64_t T_new, int64_t H, int64_t D, int64_t num_blocks,
                  int64_t block_size, int32_t dtype,
                  const b200_launch_cfg* cfg, void* stream);

/* ---- RoPE + contiguous K append (in place) --------------------------------
 * Replaces triton_agent/ops/rope_kv_append/reference.py:10-47
 * k_new: [B, H, T_new, D]; cos, sin: [T_new, D] of `cs_dtype`;
 * k_cache: [B, H, L, D]; slot_mapping: [B, T_new] int64. */
int b200_rope_kv_append(const void* k_new, const void* cos, const void* sin,
                        void* k_cache, const int64_t* slot_mapping, int64_t B,
                        int64_t H, int64_t L, int64_t T_new, int64_t D,
                        int32_t dtype, int32_t cs_dtype,
                        const b200_launch_cfg* cfg, void* stream);

/* ---- fused decode-step RoPE(q,k) + paged K/V append ------------------------
 * Composition of triton_agent/ops/rope/reference.py:17-25 (rotation),
 * rope_kv_append/reference.py:26-35 (rotate new K before writing) and
 * paged_kv/reference.py:18-25 (slot -> block/offset, invalid skipped).
 * q: [T, Hq, D] (may be NULL with q_out NULL); k, v: [T, Hkv, D];
 * positions: [T] int64 row index into cos/sin tables [cs_rows, D] of
 * `cs_dtype` (first D/2 columns used; row = position);
 * slot_mapping: [T] int64; q_out: [T, Hq, D];
 * k_cache, v_cache: [num_blocks, block_size, Hkv, D].
 * K rows are written bit-exactly as round(fp32 rotation) with no FMA
 * contraction; V rows are copied. */
int b200_rope_kv_append_paged(const void* q, const void* k, const void* v,
                              const int64_t* positions, const void* cos,
                              const void* sin, int64_t cs_rows,
                              const int64_t* slot_mapping, void* q_out,
                              void* k_cache, void* v_cache, int64_t T,
                              int64_t Hq, int64_t Hkv, int64_t D,
                              int64_t num_blocks, int64_t block_size,
                              int32_t dtype, int32_t cs_dtype,
                              const b200_launch_cfg* cfg, void* stream);

/* Same, with a slot-ownership table for many new tokens (prefill): slot_owner
 * is a caller buffer of owner_entries >= num_blocks * block_size int32,
 * zero-filled before its first use and returned to zero by each call.  A
 * later token writing the same slot wins, as in the reference's loop, in
 * O(T) instead of a per-token scan of all later slots.  slot_owner NULL is
 * b200_rope_kv_append_paged.  cfg (table path): rows_per_cta = rows of a
 * token per thread (2, 3, 4, 6, 8 or 12; default 4). */
int b200_rope_kv_append_paged_ws(const void* q, const void* k, const void* v,
                                 const int64_t* positions, const void* cos, const void* sin,
                                 int64_t cs_rows, const int64_t* slot_mapping, void* q_out,
                                 void* k_cache, void* v_cache, int64_t T, int64_t Hq,
                                 int64_t Hkv, int64_t D, int64_t num_blocks, int64_t block_size,
                                 int32_t dtype, int32_t cs_dtype, int32_t* slot_owner,
                                 int64_t owner_entries, const b200_launch_cfg* cfg, void* stream);

/* ---- paged attention decode -----------------------------------------------
 * Replaces triton_agent/ops/paged_attention/reference.py:10-54 (with the
 * query row indexed as q[b], and grouped-query attention: q head h reads kv
 * head h / (Hq / Hkv); with Hq == Hkv this is the reference exactly).
 * q, out: [B, Hq, D] (F16/BF16); k_cache, v_cache: [num_blocks, block_size,
 * Hkv, D]; block_table: [B, max_blocks] of `index_dtype` (I32/I64);
 * context_len: [B] of `index_dtype`.  Block ids outside [0, num_blocks) are
 * skipped, as at reference.py:40-41.  scale <= 0 means 1/sqrt(D).
 * Softmax and accumulation in fp32.  workspace: device buffer of at least
 * b200_paged_attention_workspace_size() bytes, zero-filled once before first
 * use (the kernel leaves it ready for the next call).
 * cfg: split (KV blocks per split of the split-grid kernel, default 64),
 * stages (ring depth, default as many 3+ as fit), rows_per_cta (kv heads per
 * CTA, <= 8), tile_m (CTAs of the persistent kernel, default the SM count),
 * tile_k (percent of the entries handed out as claimed chunks, default 0),
 * tile_n (pages per claimed chunk, default 4); flags: bit 0 CUDA-core
 * consumer, bit 1 split-grid kernel instead of the persistent one, bit 2
 * equal static ranges only, bit 3 programmatic dependent launch (the
 * kernel's prologue overlaps the previous kernel on the stream; the caller
 * guarantees that kernel writes neither context_len nor block_table, as the
 * decode-step append does not). */
size_t b200_paged_attention_workspace_size(int64_t B, int64_t Hq,
                                           int64_t max_blocks,
                                           int64_t block_size, int64_t D,
                                           const b200_launch_cfg* cfg);
int b200_paged_attention(const void* q, const void* k_cache,
                         const void* v_cache, const void* block_table,
                         const void* context_len, void* out, int64_t B,
                         int64_t Hq, int64_t Hkv, int64_t D,
                         int64_t num_blocks, int64_t block_size,
                         int64_t max_blocks, float scale, int32_t dtype,
                         int32_t index_dtype, void* workspace,
                         size_t workspace_bytes, const b200_launch_cfg* cfg,
                         void* stream);

/* ---- allocation-free paged attention ---------------------------------------
 * No counterpart in the reference.  Same arguments, semantics and results as
 * b200_paged_attention, without the workspace: for callers that cannot
 * allocate device memory (a C-FFI host runtime that holds only the pointers
 * it is given, or a request path where cudaMalloc is forbidden because it can
 * synchronise the device), the split-KV scratch is a static 16 MiB device
 * array inside the library (per GPU, kept until exit).  Calls needing more
 * scratch than that return B200_ERR_WORKSPACE with the size in
 * b200_last_error_detail().  The first call on a device looks up the array's
 * address (do it before any stream capture).  All calls share the array:
 * calls whose executions overlap on the GPU race and must be serialised. */
int b200_paged_attention_noalloc(const void* q, const void* k_cache,
                                 const void* v_cache, const void* block_table,
                                 const void* context_len, void* out, int64_t B,
                                 int64_t Hq, int64_t Hkv, int64_t D,
                                 int64_t num_blocks, int64_t block_size,
                                 int64_t max_blocks, float scale, int32_t dtype,
                                 int32_t index_dtype,
                                 const b200_launch_cfg* cfg, void* stream);

/* ---- INT8 GEMM with fused dequant epilogue --------------------------------
 * Restates triton_agent/ops/quant_matmul/reference.py:26-27 for
 * pre-quantised operands:
 *   acc[m,n] = sum_k A[m,k] * W[n,k]            (int8 x int8 -> int32, exact)
 *   C[m,n]   = out_dtype( float(acc) * sA[m] * sW[n] )
 * A: [M, K] int8 row-major; W: [N, K] int8 row-major (K-major); sA: [M] f32;
 * sW: [N] f32; C: [M, N] with row stride ldc (elements) of `out_dtype`
 * (F16/BF16/F32).  acc_out (nullable): [M, N] int32 raw accumulators.
 * K must be a multiple of 16 and A/W 16-byte aligned.
 * workspace: needed only for split-K (small M); size from
 * b200_int8_gemm_workspace_size().  cfg: M > 128: stages, tile_n (CTA-pair
 * tile width 128..256 in steps of 32; default: a wave model that picks 256
 * unless a narrower width removes a mostly empty wave), flags bit 1 (one-SM kernel, with tile_n
 * 128/256), flags bit 3 (the last partial wave of 256-wide tiles keeps whole
 * tiles; by default, when it would busy at most half the CTA pairs, each of
 * its tiles runs as two 128-wide items); M <= 64 (streaming kernel): tile_k (bytes of
 * K per ring stage), stages, tile_m (CTAs of the grid; default n tiles x the
 * largest k split that fits the SM count), flags bit 2 (split-grid kernel,
 * with split). */
size_t b200_int8_gemm_workspace_size(int64_t M, int64_t N, int64_t K,
                                     const b200_launch_cfg* cfg);
int b200_int8_gemm(const int8_t* A, const int8_t* W, const float* sA,
                   const float* sW, void* C, int64_t M, int64_t N, int64_t K,
                   int64_t ldc, int32_t out_dtype, int32_t* acc_out,
                   void* workspace, size_t workspace_bytes,
                   const b200_launch_cfg* cfg, void* stream);

/* ---- bf16/fp16 GEMM + bias + GELU ------------------------------------------
 * Replaces triton_agent/ops/matmul_epilogue/reference.py:6-18
 *   c = gelu_tanh(a @ b + bias)
 * a: [M, K] (the reference's [B, M, K] flattened), b: [K, N] row-major (as
 * the reference passes it), bias: [N], c: [M, N], all of `dtype` (F16 or
 * BF16).  fp32 accumulation in tensor memory (tcgen05 kind::f16, CTA pairs),
 * bias and GELU (tanh form) in fp32, one rounding to `dtype`.  Needs
 * K % 8 == 0, N % 8 == 0 and 16-byte aligned a, b, c. */
int b200_gemm_bias_gelu(const void* a, const void* b, const void* bias, void* c, int64_t M,
                        int64_t N, int64_t K, int32_t dtype, const b200_launch_cfg* cfg,
                        void* stream);

/* ---- column-sharded INT8 GEMM with the all-gather fused (multi-GPU) --------
 * No counterpart in the reference (which runs on one device): the
 * multi-GPU layout of quant_matmul partitions W by output columns, and
 * instead of a GEMM followed by an all-gather, each rank's epilogue stores
 * every dequantised output tile straight into the C buffer of every rank
 * over NVLink (peer stores; no collective library call).
 *
 * This rank computes C[:, col0 : col0 + n_local] = dequant(A W_local^T)
 * (the b200_int8_gemm formula) and writes it into C_ranks[r] for every rank
 * r < world (device pointers valid on this device: peers' buffers opened
 * with b200_ipc_open, this rank's own at index `rank`; all with the same
 * ldc).  Two flag exchanges bracket the GEMM, each bounded by
 * b200_set_peer_wait_timeout_us (code 6 in the device error word on expiry):
 *   - before it, this rank stores `epoch` into sig_ranks[r][world + rank] and
 *     waits until sig_ranks[rank][world + r] >= epoch for every r: no rank
 *     writes into a peer's C until that peer's stream has reached this call,
 *     i.e. finished everything it ran before it, including its reads of the
 *     previous call's C;
 *   - after it, this rank stores `epoch` into sig_ranks[r][rank] and waits
 *     until sig_ranks[rank][r] >= epoch for every r: every rank's columns
 *     have landed in this rank's C.
 * sig arrays: 2 * world uint32 each, zero before the first call; epoch:
 * strictly increasing per call.  All ranks must call it with the same M, K,
 * epoch and world. */
int b200_int8_gemm_allgather(const int8_t* A, const int8_t* W_local, const float* sA,
                             const float* sW_local, void* const* C_ranks,
                             uint32_t* const* sig_ranks, int32_t world, int32_t rank,
                             int64_t M, int64_t n_local, int64_t col0, int64_t K,
                             int64_t ldc, int32_t out_dtype, uint32_t epoch,
                             void* workspace, size_t workspace_bytes,
                             const b200_launch_cfg* cfg, void* stream);

/* ---- CUDA IPC for peer buffers (no counterpart in the reference) -----------
 * handle: 64 opaque bytes naming dev_ptr's whole allocation, and offset:
 * dev_ptr's byte offset inside it (allocators hand out pieces of larger
 * allocations).  b200_ipc_open maps another process's buffer on this device
 * (peer access over NVLink enabled) and returns base + offset;
 * b200_ipc_close unmaps it (same offset). */
int b200_ipc_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out);
int b200_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out);
int b200_ipc_close(void* dev_ptr, int64_t offset);

/* ---- symmetric INT8 quantisation -------------------------------------------
 * Restates triton_agent/ops/quant_matmul/reference.py:16-24:
 *   scale = max|x| / 127 (0 -> 1e-6), q = clamp(round_half_even(x / scale), -127, 127)
 * Row mode (`by_column` = 0): x [rows, cols] -> q [rows, cols], scale [rows].
 * Column mode (`by_column` = 1): x [rows, cols] (e.g. b [K, N]) is quantised
 * per column and written transposed: q [cols, rows], scale [cols].
 * scale_dtype is the dtype the reference's scale tensor has (that of x);
 * the division uses the scale rounded to that dtype, as the reference does.
 * 16-bit x takes packed paths when it can: rows of at most 4096 elements (a
 * multiple of 8, x 16-byte and q 8-byte aligned) one warp per row; columns
 * (cols % 64 == 0, rows % 16 == 0, x and q 16-byte aligned) 64-column strips
 * over clusters of eight CTAs holding their rows in shared memory (up to
 * 4096 rows) or of four CTAs reading x twice.  Everything else (and fp32)
 * takes the general kernels; the codes are the same on every path. */
int b200_quantize_int8(const void* x, int8_t* q, float* scale, int64_t rows,
                       int64_t cols, int32_t dtype, int32_t by_column,
                       const b200_launch_cfg* cfg, void* stream);

/* ---- causal / full flash attention prefill -----------------------------------
 * Replaces triton_agent/ops/flash_attn_like/reference.py:7-31
 * q: [B, H, T, D]; k, v: [B, H, S, D]; o: [B, H, T, D]; dtype F16/BF16;
 * D = 128 on the tensor-core path.  causal: mask key s > query t
 * (reference.py:25-28, which assumes T == S).  lse (nullable): [B, H, T] f32
 * natural-log softmax normaliser.  scale <= 0 means 1/sqrt(D).
 * cfg: split (heads per scheduling group, default 8), tile_k (exponential
 * pairs of every 8 computed by a polynomial on the FMA pipe: 1-3, default 2,
 * 4 = none); flags: bit 4 persistent kernel, bit 2 two-tile kernel (bit 1
 * with it: polynomial exponentials), bit 0 one-tile kernel. */
int b200_flash_attn(const void* q, const void* k, const void* v, void* o,
                    float* lse, int64_t B, int64_t H, int64_t T, int64_t S,
                    int64_t D, float scale, int32_t causal, int32_t dtype,
                    const b200_launch_cfg* cfg, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200OPS_H */
