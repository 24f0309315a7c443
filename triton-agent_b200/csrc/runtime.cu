// Library-level entry points: status strings, version, kernel list, host-side
// fault injection and the device error word registry.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
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
         "rope_kernel\n"
         "kv_scatter_kernel\n"
         "rope_kv_append_paged_kernel\n"
         "rope_kv_append_paged_fast_kernel\n"
         "paged_decode_flat_kernel\n"
         "paged_decode_kernel\n"
         "paged_decode_generic_kernel\n"
         "int8_gemm_pair_kernel\n"
         "int8_gemm_tcgen05_kernel\n"
         "int8_gemm_stream_kernel\n"
         "int8_gemm_skinny_kernel\n"
         "peer_flag_exchange_kernel\n"
         "quantize_rows_kernel\n"
         "quantize_cols_kernel\n"
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
