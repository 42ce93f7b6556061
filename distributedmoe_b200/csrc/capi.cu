// Library-wide C ABI pieces: error state, version, CUDA IPC, copies and completion flags.
//
// IPC + copies replace the NIXL/MoonCake data plane of the reference's transfer engines
// (TensorTransferEngine/NIXLTensorTransferEngine.py:113-249): a registered buffer is exported
// as a cudaIpcMemHandle, the peer maps it once, and READ/WRITE become stream-ordered copies
// over NVLink.  Flags replace the 1 ms transfer-monitor poll
// (TensorTransferEngine/TensorTransferEngine.py:320-344).
#include <cuda.h>

#include "dmoe_common.cuh"

namespace dmoe {

static thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

void clear_error() { t_last_error.clear(); }

// Release store of a 64-bit flag, visible system-wide (peer GPUs read it over NVLink).
__global__ void flag_signal_kernel(uint64_t* flag, uint64_t value) {
  __threadfence_system();
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(value) : "memory");
}

// Bounded acquire-spin on a flag written by another GPU.  On expiry it records the error
// and returns, so the stream (and the context) stay usable.
__global__ void flag_wait_kernel(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, int32_t* status) {
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
    if (v >= value) return;
    if ((++spins & 63u) == 0 && global_timer_ns() - t0 > timeout_ns) {
      if (status) atomicOr(status, DMOE_DEVERR_FLAG_TIMEOUT);
      return;
    }
    __nanosleep(200);
  }
}

}  // namespace dmoe

using namespace dmoe;

extern "C" {

const char* dmoe_version(void) { return "dmoe_b200 0.1 sm_100a"; }

const char* dmoe_last_error(void) { return t_last_error.c_str(); }

uint64_t dmoe_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int dmoe_ipc_export(const void* dev_ptr, uint8_t* handle_out64, uint64_t* offset_out) {
  DMOE_REQUIRE(dev_ptr != nullptr && handle_out64 != nullptr && offset_out != nullptr, "dmoe_ipc_export: null pointer");
  typedef CUresult (*PFN_range)(CUdeviceptr*, size_t*, CUdeviceptr);
  static PFN_range get_range = nullptr;
  if (get_range == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    DMOE_CUDA(cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q));
    DMOE_REQUIRE(q == cudaDriverEntryPointSuccess && p != nullptr, "cuMemGetAddressRange is unavailable");
    get_range = reinterpret_cast<PFN_range>(p);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = get_range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr));
  if (r != CUDA_SUCCESS) {
    set_error("cuMemGetAddressRange failed (%d)", (int)r);
    return DMOE_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  DMOE_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  memcpy(handle_out64, &h, 64);
  *offset_out = (uint64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return DMOE_OK;
}

int dmoe_ipc_open(const uint8_t* handle64, int device, void** dev_ptr_out) {
  DMOE_REQUIRE(handle64 != nullptr && dev_ptr_out != nullptr, "dmoe_ipc_open: null pointer");
  int prev = 0;
  DMOE_CUDA(cudaGetDevice(&prev));
  DMOE_CUDA(cudaSetDevice(device));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_error("cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
    return DMOE_ERR_CUDA;
  }
  return DMOE_OK;
}

int dmoe_ipc_close(void* dev_ptr) {
  DMOE_REQUIRE(dev_ptr != nullptr, "dmoe_ipc_close: null pointer");
  DMOE_CUDA(cudaIpcCloseMemHandle(dev_ptr));
  return DMOE_OK;
}

int dmoe_enable_peer_access(int device, int peer_device) {
  if (device == peer_device) return DMOE_OK;
  int can = 0;
  DMOE_CUDA(cudaDeviceCanAccessPeer(&can, device, peer_device));
  DMOE_REQUIRE(can, "device %d cannot access peer %d", device, peer_device);
  int prev = 0;
  DMOE_CUDA(cudaGetDevice(&prev));
  DMOE_CUDA(cudaSetDevice(device));
  cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  cudaSetDevice(prev);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return DMOE_OK;
  }
  if (e != cudaSuccess) {
    set_error("cudaDeviceEnablePeerAccess(%d->%d) failed: %s", device, peer_device, cudaGetErrorString(e));
    return DMOE_ERR_CUDA;
  }
  return DMOE_OK;
}

int dmoe_copy(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return DMOE_OK;
  DMOE_REQUIRE(dst != nullptr && src != nullptr, "dmoe_copy: null pointer");
  DMOE_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, as_stream(stream)));
  return DMOE_OK;
}

// Raw CUDA events for the transfer engine's cross-process ordering.  An event created with
// interprocess != 0 can be exported; an imported event is opened in the context of the GPU
// that recorded it, and is only waited on by streams of that GPU.
int dmoe_event_create(int device, int interprocess, void** event_out) {
  DMOE_REQUIRE(event_out != nullptr, "dmoe_event_create: null pointer");
  int prev = 0;
  DMOE_CUDA(cudaGetDevice(&prev));
  DMOE_CUDA(cudaSetDevice(device));
  cudaEvent_t ev = nullptr;
  cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming | (interprocess ? cudaEventInterprocess : 0));
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_error("cudaEventCreateWithFlags failed: %s", cudaGetErrorString(e));
    return DMOE_ERR_CUDA;
  }
  *event_out = ev;
  return DMOE_OK;
}

int dmoe_event_destroy(void* event) {
  if (event == nullptr) return DMOE_OK;
  DMOE_CUDA(cudaEventDestroy(reinterpret_cast<cudaEvent_t>(event)));
  return DMOE_OK;
}

int dmoe_event_record(void* event, void* stream) {
  DMOE_REQUIRE(event != nullptr, "dmoe_event_record: null event");
  DMOE_CUDA(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), as_stream(stream)));
  return DMOE_OK;
}

int dmoe_event_query(void* event) {
  DMOE_REQUIRE(event != nullptr, "dmoe_event_query: null event");
  cudaError_t e = cudaEventQuery(reinterpret_cast<cudaEvent_t>(event));
  if (e == cudaSuccess) return DMOE_OK;
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    return DMOE_NOT_READY;
  }
  set_error("cudaEventQuery failed: %s", cudaGetErrorString(e));
  return DMOE_ERR_CUDA;
}

int dmoe_stream_wait_event(void* stream, void* event) {
  DMOE_REQUIRE(event != nullptr, "dmoe_stream_wait_event: null event");
  DMOE_CUDA(cudaStreamWaitEvent(as_stream(stream), reinterpret_cast<cudaEvent_t>(event), 0));
  return DMOE_OK;
}

int dmoe_ipc_event_export(void* event, uint8_t* handle_out64) {
  DMOE_REQUIRE(event != nullptr && handle_out64 != nullptr, "dmoe_ipc_event_export: null pointer");
  cudaIpcEventHandle_t h;
  static_assert(sizeof(h) == 64, "cudaIpcEventHandle_t is 64 bytes");
  DMOE_CUDA(cudaIpcGetEventHandle(&h, reinterpret_cast<cudaEvent_t>(event)));
  memcpy(handle_out64, &h, 64);
  return DMOE_OK;
}

int dmoe_ipc_event_open(const uint8_t* handle64, int device, void** event_out) {
  DMOE_REQUIRE(handle64 != nullptr && event_out != nullptr, "dmoe_ipc_event_open: null pointer");
  int prev = 0;
  DMOE_CUDA(cudaGetDevice(&prev));
  DMOE_CUDA(cudaSetDevice(device));
  cudaIpcEventHandle_t h;
  memcpy(&h, handle64, 64);
  cudaEvent_t ev = nullptr;
  cudaError_t e = cudaIpcOpenEventHandle(&ev, h);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_error("cudaIpcOpenEventHandle failed: %s", cudaGetErrorString(e));
    return DMOE_ERR_CUDA;
  }
  *event_out = ev;
  return DMOE_OK;
}

int dmoe_flag_signal(uint64_t* flag, uint64_t value, void* stream) {
  DMOE_REQUIRE(flag != nullptr && (reinterpret_cast<uintptr_t>(flag) & 7u) == 0, "dmoe_flag_signal: bad flag");
  flag_signal_kernel<<<1, 1, 0, as_stream(stream)>>>(flag, value);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

int dmoe_flag_wait(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, int32_t* dev_status, void* stream) {
  DMOE_REQUIRE(flag != nullptr && (reinterpret_cast<uintptr_t>(flag) & 7u) == 0, "dmoe_flag_wait: bad flag");
  DMOE_REQUIRE(timeout_ns > 0 && timeout_ns <= 60ull * 1000000000ull, "dmoe_flag_wait: timeout must be in (0, 60 s]");
  flag_wait_kernel<<<1, 1, 0, as_stream(stream)>>>(flag, value, timeout_ns, dev_status);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

}  // extern "C"
