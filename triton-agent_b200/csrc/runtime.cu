// Library-level entry points: status strings, version, kernel list, host-side
// fault injection and the device error word registry.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "sm100.cuh"

namespace b200 {

namespace {
std::mutex& reg_mutex() {
  static std::mutex m;
  return m;
}
std::vector<error_reader_fn>& readers() {
  static std::vector<error_reader_fn> v;
  return v;
}
thread_local char g_detail[256] = {0};
}  // namespace

ErrorReaderRegistrar::ErrorReaderRegistrar(error_reader_fn fn) {
  std::lock_guard<std::mutex> lk(reg_mutex());
  readers().push_back(fn);
}

int read_all_device_errors(cudaStream_t stream, int32_t* out) {
  std::vector<error_reader_fn> copy;
  {
    std::lock_guard<std::mutex> lk(reg_mutex());
    copy = readers();
  }
  int first = 0;
  for (auto fn : copy) {
    int v = fn(stream);
    if (v < 0) return B200_ERR_LAUNCH;
    if (v != 0 && first == 0) first = v;
  }
  *out = first;
  return B200_OK;
}

void set_last_error_detail(const char* msg) {
  snprintf(g_detail, sizeof(g_detail), "%s", msg ? msg : "");
}

int launch_status(cudaError_t e) {
  if (e == cudaSuccess) return B200_OK;
  set_last_error_detail(cudaGetErrorString(e));
  return B200_ERR_LAUNCH;
}

namespace {
std::atomic<uint64_t> g_peer_wait_timeout_ns{sm100::kWaitTimeoutNs};
}  // namespace

uint64_t peer_wait_timeout_ns() { return g_peer_wait_timeout_ns.load(std::memory_order_relaxed); }

int injected_error(const char* op_name) {
  const char* v = getenv("B200OPS_INJECT_ERROR");
  if (v == nullptr || v[0] == '\0') return B200_OK;
  if (strcmp(v, "all") == 0 || strcmp(v, op_name) == 0) {
    set_last_error_detail("error injected on the host by B200OPS_INJECT_ERROR");
    return B200_ERR_INJECTED;
  }
  return B200_OK;
}

typedef CUresult (*encode_tiled_fn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static encode_tiled_fn get_encode_fn() {
  static encode_tiled_fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<encode_tiled_fn>(p);
  });
  return fn;
}

int encode_tensor_map(CUtensorMap* out, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  encode_tiled_fn fn = get_encode_fn();
  if (fn == nullptr) {
    set_last_error_detail("cuTensorMapEncodeTiled entry point not available");
    return B200_ERR_NO_DEVICE;
  }
  if (!aligned16(base)) return B200_ERR_ALIGNMENT;
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(out, dtype, rank, const_cast<void*>(base), dims, strides_bytes, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed with CUresult %d", (int)r);
    set_last_error_detail(buf);
    return B200_ERR_BAD_ARG;
  }
  return B200_OK;
}

}  // namespace b200

extern "C" {

const char* b200_status_string(int status) {
  switch (status) {
    case B200_OK: return "ok";
    case B200_ERR_BAD_ARG: return "bad argument";
    case B200_ERR_UNSUPPORTED: return "unsupported dtype or shape";
    case B200_ERR_LAUNCH: return "kernel launch failed";
    case B200_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case B200_ERR_WORKSPACE: return "workspace missing or too small";
    case B200_ERR_NO_DEVICE: return "no sm_100 device";
    case B200_ERR_INJECTED: return "injected error";
    case B200_ERR_ALIGNMENT: return "pointer or leading dimension not 16-byte aligned";
    default: return "unknown status";
  }
}

const char* b200_last_error_detail(void) { return b200::g_detail; }

int b200_version(void) { return 100; }

const char* b200_kernel_list(void) {
  return "rmsnorm_row_kernel\n"
         "rmsnorm_loop_kernel\n"
         "rmsnorm_quant_row_kernel\n"
         "rmsnorm_quant_persistent_kernel\n"
         "rmsnorm_quant_warp_kernel\n"
         "rope_kernel\n"
         "kv_scatter_kernel\n"
         "rope_kv_append_paged_kernel\n"
         "rope_kv_append_paged_fast_kernel\n"
         "rope_kv_append_paged_rows_kernel\n"
         "slot_owner_kernel\n"
         "paged_decode_flat_kernel\n"
         "paged_decode_kernel\n"
         "paged_decode_generic_kernel\n"
         "int8_gemm_pair_kernel\n"
         "int8_gemm_tcgen05_kernel\n"
         "int8_gemm_stream_kernel\n"
         "int8_gemm_skinny_kernel\n"
         "peer_flag_exchange_kernel\n"
         "quantize_rows_kernel\n"
         "quantize_rows_warp_kernel\n"
         "quantize_cols_kernel\n"
         "quantize_cols_strip_kernel\n"
         "quantize_cols_resident_kernel\n"
         "flash_fwd3_tcgen05_kernel\n"
         "flash_fwd4_persistent_kernel\n"
         "flash_fwd2_tcgen05_kernel\n"
         "flash_fwd_tcgen05_kernel\n"
         "flash_generic_kernel\n";
}

// CUDA IPC handles name whole allocations; a caching allocator hands out
// pieces of larger ones, so the handle travels with the piece's offset from
// its allocation base (cuMemGetAddressRange through the driver entry point).
typedef CUresult (*addr_range_fn)(CUdeviceptr*, size_t*, CUdeviceptr);

static addr_range_fn get_addr_range_fn() {
  static addr_range_fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<addr_range_fn>(p);
  });
  return fn;
}

int b200_ipc_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  if (!dev_ptr || !handle_out || !offset_out) return B200_ERR_BAD_ARG;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  addr_range_fn range = get_addr_range_fn();
  if (range == nullptr) return B200_ERR_NO_DEVICE;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return B200_ERR_BAD_ARG;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    b200::set_last_error_detail(cudaGetErrorString(e));
    return B200_ERR_LAUNCH;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return B200_OK;
}

int b200_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out) {
  if (!handle || !dev_ptr_out || offset < 0) return B200_ERR_BAD_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    b200::set_last_error_detail(cudaGetErrorString(e));
    return B200_ERR_LAUNCH;
  }
  *dev_ptr_out = static_cast<char*>(base) + offset;
  return B200_OK;
}

int b200_ipc_close(void* dev_ptr, int64_t offset) {
  if (!dev_ptr || offset < 0) return B200_ERR_BAD_ARG;
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(dev_ptr) - offset);
  if (e != cudaSuccess) {
    b200::set_last_error_detail(cudaGetErrorString(e));
    return B200_ERR_LAUNCH;
  }
  return B200_OK;
}

// Launch parameters the tuner may search, per op: the kernel the op's
// default dispatch selects for `rows` rows (GEMM: M; decode: sequences;
// 0: the op's benchmark shape), and for each b200_launch_cfg field that
// kernel reads, the values it accepts (0 = the kernel's default).  Fields not
// listed are ignored by that kernel.  The text is JSON, valid until the next
// call on the same thread.
const char* b200_query_config_space(const char* op, int64_t rows) {
  static thread_local std::string out;
  if (op == nullptr) return nullptr;
  const int sms = b200::device_sm_count();
  const std::string o(op);
  std::string kernel, fields;
  auto field = [&](const char* name, std::initializer_list<int64_t> vals, const char* meaning) {
    if (!fields.empty()) fields += ",";
    fields += "\"";
    fields += name;
    fields += "\":{\"values\":[";
    bool first = true;
    for (int64_t v : vals) {
      if (!first) fields += ",";
      fields += std::to_string(v);
      first = false;
    }
    fields += "],\"meaning\":\"";
    fields += meaning;
    fields += "\"}";
  };
  if (o == "rmsnorm") {
    kernel = "rmsnorm_row_kernel";
    field("threads", {0, 128, 256, 512, 1024}, "CTA size (0: 256, or fewer for short rows)");
  } else if (o == "rmsnorm_quant") {
    kernel = "rmsnorm_quant_warp_kernel";
    field("threads", {0, 64, 128, 256, 512, 1024},
          "CTA size of the CTA kernels (0: warp rows for 16-bit D = 1024, 2048, 4096, else about four 16-byte "
          "vectors per thread)");
    field("rows_per_cta", {0, 1, 2, 4}, "rows per CTA of the CTA kernels (0: 1; more than 1 only with <= 256 threads)");
    field("flags", {0, 1, 2, 4},
          "1: one CTA per row; 2: the persistent CTA row loop instead of warp rows; 4: warp rows without the "
          "shared-memory prefetch of the next row");
  } else if (o == "rope") {
    kernel = "rope_kernel";
    field("threads", {0, 64, 128, 256}, "CTA size, at most 256 (0: 256)");
  } else if (o == "kv_append" || o == "paged_kv" || o == "rope_kv_append") {
    kernel = "kv_scatter_kernel";
    field("threads", {0, 128, 256, 512, 1024}, "CTA size (0: all rows' lanes, up to 1024)");
  } else if (o == "rope_kv_append_paged") {
    if (rows > 512) {
      kernel = "rope_kv_append_paged_rows_kernel";
      field("rows_per_cta", {0, 2, 3, 4, 6, 8, 12}, "rows of a token per thread (0: 4)");
    } else {
      kernel = "rope_kv_append_paged_fast_kernel";
      field("threads", {0, 128, 256, 512},
            "0: the single-pass kernel (one CTA per token); > 0: the general kernel with this CTA size");
    }
  } else if (o == "paged_attention") {
    kernel = "paged_decode_flat_kernel";
    field("rows_per_cta", {0, 1, 2, 4, 8}, "kv heads per CTA, a divisor of H_kv (0: the largest <= 8 that fits)");
    field("stages", {0, 2, 3, 4}, "KV page ring depth (0: about 128 KB of pages in flight)");
    field("tile_m", {0, 2 * (int64_t)sms}, "CTAs of the persistent grid (0: one per SM)");
    field("tile_k", {0, 10, 25, 50}, "percent of the block-table entries handed out as claimed chunks (0: none)");
    field("tile_n", {0, 1, 2, 8}, "pages per claimed chunk (0: 4)");
  } else if (o == "quant_matmul") {
    if (rows > 0 && rows <= 64) {
      kernel = "int8_gemm_stream_kernel";
      field("tile_k", {0, 128, 256, 384, 512, 1024}, "bytes of K per ring stage (0: 384, 256 for M > 32)");
      field("stages", {0, 4, 6, 8, 10, 12, 14, 16}, "ring depth (0: 16, or as many as fit)");
      field("tile_m", {0, 64, 96, 112, 128, (int64_t)sms},
            "CTAs of the grid (0: n tiles x the largest k split within the SM count)");
    } else if (rows > 0 && rows <= 128) {
      kernel = "int8_gemm_tcgen05_kernel";
      field("tile_n", {0, 128, 256}, "output columns per tile (0: 256)");
      field("stages", {0, 2, 3, 4, 5, 6, 7, 8}, "ring depth (0: 8)");
    } else {
      kernel = "int8_gemm_pair_kernel";
      field("stages", {0, 2, 3, 4, 5, 6, 7, 8}, "ring depth (0: 8)");
      field("flags", {0, 2, 8},
            "2: one-SM persistent kernel (128 x tile_n tiles) instead of CTA pairs; 8: the last partial wave "
            "keeps whole tiles (0: each of its 256-wide tiles runs as two 128-wide items)");
      field("tile_n", {0, 128, 160, 192, 224, 256},
            "output columns per tile (CTA pairs: 128..256 step 32, 0: a wave model, 256 at the bench shapes; "
            "one-SM kernel: 128 or 256)");
    }
  } else if (o == "matmul_epilogue") {
    kernel = "int8_gemm_pair_kernel (kind::f16)";
    field("stages", {0, 2, 3, 4, 5, 6, 7, 8}, "ring depth (0: 8)");
  } else if (o == "flash_attn_like") {
    kernel = "flash_fwd3_tcgen05_kernel";
    field("split", {0, 1, 2, 4, 8, 16}, "heads per scheduling group sharing K/V in L2 (0: 8)");
    field("tile_k", {0, 1, 2, 3, 4}, "exponential pairs of every 8 on the FMA pipe (0: 2; 4: none)");
    field("flags", {0, 16}, "16: persistent kernel (one CTA per SM taking work items)");
  } else {
    return nullptr;
  }
  out = "{\"op\":\"" + o + "\",\"rows\":" + std::to_string(rows) + ",\"kernel\":\"" + kernel +
        "\",\"sm_count\":" + std::to_string(sms) + ",\"fields\":{" + fields + "}}";
  return out.c_str();
}

int b200_set_peer_wait_timeout_us(int64_t us) {
  if (us < 0) return B200_ERR_BAD_ARG;
  b200::g_peer_wait_timeout_ns.store(us == 0 ? b200::sm100::kWaitTimeoutNs : (uint64_t)us * 1000ull,
                                     std::memory_order_relaxed);
  return B200_OK;
}

int b200_read_device_error(int32_t* out, void* stream) {
  if (out == nullptr) return B200_ERR_BAD_ARG;
  return b200::read_all_device_errors(static_cast<cudaStream_t>(stream), out);
}

}  // extern "C"
