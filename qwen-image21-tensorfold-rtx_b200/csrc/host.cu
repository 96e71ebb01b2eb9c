// Host plumbing of libtfb: error reporting, per-device cache, TMA tensor maps, small C entry points.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "tfb_common.cuh"

namespace tfb {

// Kernels whose bounded waits run out record a nonzero code here (one word per device context).
__device__ int g_err_word;

static thread_local char t_msg[512];

tfb_status fail(tfb_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  return st;
}

tfb_status cuda_fail(cudaError_t e, const char* what) {
  return fail(TFB_CUDA_ERR, "%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

namespace {
constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
// Set (release) after g_dev[dev] is filled; read (acquire) on the lock-free fast path.
std::atomic<bool> g_dev_ok[kMaxDevices];
std::mutex g_dev_mu;
std::atomic<PFN_cuTensorMapEncodeTiled_v12000> g_encode{nullptr};
}  // namespace

tfb_status device_info(const DeviceInfo** out) {
  int dev = 0;
  TFB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(TFB_BAD_ARG, "device ordinal %d out of range", dev);
  if (g_dev_ok[dev].load(std::memory_order_acquire)) {
    *out = &g_dev[dev];
    return TFB_OK;
  }
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (!g_dev_ok[dev].load(std::memory_order_relaxed)) {
    int major = 0, minor = 0, sms = 0;
    TFB_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    TFB_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    TFB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (major != 10 || minor != 0)
      return fail(TFB_BAD_ARCH, "libtfb is built for sm_100a (B200); device %d is sm_%d%d", dev, major, minor);
    void* p = nullptr;
    TFB_CUDA(cudaGetSymbolAddress(&p, g_err_word));
    g_dev[dev] = DeviceInfo{dev, sms, static_cast<int*>(p)};
    g_dev_ok[dev].store(true, std::memory_order_release);
  }
  *out = &g_dev[dev];
  return TFB_OK;
}

tfb_status make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                        uint64_t row_stride, uint32_t box_inner, uint32_t box_rows, bool swizzle) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = g_encode.load(std::memory_order_acquire);
  if (!encode) {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    encode = g_encode.load(std::memory_order_relaxed);
    if (!encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      TFB_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q));
      if (q != cudaDriverEntryPointSuccess || !fn) return fail(TFB_CUDA_ERR, "cuTensorMapEncodeTiled unavailable");
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      g_encode.store(encode, std::memory_order_release);
    }
  }
  if (!aligned(base, 16) || row_stride % 16 != 0)
    return fail(TFB_BAD_ALIGN, "TMA operand needs a 16-byte aligned base and row stride (stride %llu)",
                (unsigned long long)row_stride);
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r = encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TFB_CUDA_ERR, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return TFB_OK;
}

tfb_status make_tmap_u8(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint64_t row_stride,
                        uint32_t box_inner, uint32_t box_rows) {
  return make_tmap_2d(map, base, 1, inner_bytes, rows, row_stride, box_inner, box_rows, true);
}

}  // namespace tfb

extern "C" {

int tfb_version(void) { return 100; }

const char* tfb_last_error(void) { return tfb::t_msg; }

int64_t tfb_sf_tiled_bytes(int64_t rows, int64_t k) {
  if (rows < 0 || k < 0 || k % 64) return -1;
  return ((rows + 127) / 128) * (k / 64) * 512;
}

tfb_status tfb_ipc_handle(const void* ptr, uint8_t* handle, int64_t* offset) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  if (!ptr || !handle || !offset) return tfb::fail(TFB_BAD_ARG, "ipc_handle: null argument");
  static std::atomic<PFN_cuMemGetAddressRange_v3020> s_range{nullptr};
  PFN_cuMemGetAddressRange_v3020 range = s_range.load(std::memory_order_acquire);
  if (!range) {   // two threads may both look it up; they store the same pointer
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    TFB_CUDA(cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn) return tfb::fail(TFB_CUDA_ERR, "cuMemGetAddressRange unavailable");
    range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
    s_range.store(range, std::memory_order_release);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return tfb::fail(TFB_BAD_ARG, "ipc_handle: %p is not inside a device allocation", ptr);
  cudaIpcMemHandle_t h;
  TFB_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return TFB_OK;
}

tfb_status tfb_ipc_open(const uint8_t* handle, int64_t offset, void** ptr) {
  if (!handle || !ptr || offset < 0) return tfb::fail(TFB_BAD_ARG, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  TFB_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = static_cast<uint8_t*>(base) + offset;
  return TFB_OK;
}

tfb_status tfb_ipc_close(void* ptr, int64_t offset) {
  if (!ptr || offset < 0) return tfb::fail(TFB_BAD_ARG, "ipc_close: bad argument");
  TFB_CUDA(cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset));
  return TFB_OK;
}

tfb_status tfb_device_status(int* code, int reset) {
  const tfb::DeviceInfo* di;
  tfb_status st = tfb::device_info(&di);
  if (st != TFB_OK) return st;
  TFB_CUDA(cudaDeviceSynchronize());
  int v = 0;
  TFB_CUDA(cudaMemcpy(&v, di->err_word, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) {
    int z = 0;
    TFB_CUDA(cudaMemcpy(di->err_word, &z, sizeof(int), cudaMemcpyHostToDevice));
  }
  if (code) *code = v;
  if (v) return tfb::fail(TFB_DEVICE_TIMEOUT, "a kernel pipeline wait ran out (code 0x%x)", v);
  return TFB_OK;
}

}  // extern "C"
