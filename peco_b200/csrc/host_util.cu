// Host utilities: TMA tensor-map encoding, the device status word and error
// strings shared by all C-ABI entry points.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "../../include/peco_b200.h"
#include "internal.h"

namespace peco {

// One status word per device that loads the library.  Kernels OR
// DeviceStatusBits into it instead of trapping, so a failed bounds check or
// an expired wait leaves the context usable; the host reads it with
// peco_device_status().
__device__ unsigned g_device_status;

namespace {
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn g_encode = nullptr;
std::once_flag g_encode_once;

std::atomic<unsigned long long> g_launches{0};

constexpr int kMaxDevices = 64;
unsigned* g_status_ptr[kMaxDevices] = {};
std::mutex g_status_mutex;
}  // namespace

bool encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                       const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                       CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeFn>(fn);
  });
  if (!g_encode) return false;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

unsigned* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  unsigned* p = g_status_ptr[dev];
  if (p) return p;
  std::lock_guard<std::mutex> lock(g_status_mutex);
  if (!g_status_ptr[dev]) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_device_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<unsigned*>(addr);
  }
  return g_status_ptr[dev];
}

const char* error_string(int code) {
  switch (code) {
    case kOk: return "no error";
    case kErrUnsupported: return "shape or dtype not supported by the sm_100a kernels";
    case kErrTensorMap: return "TMA tensor map encoding failed (alignment or extent)";
    case kErrDriverEntry: return "CUDA driver entry point unavailable";
    case kErrWaitTimeout: return "a device-side bounded wait expired";
    case kErrWorkspace: return "workspace buffer too small";
    case kErrCapacity: return "problem larger than the fixed device scratch of this no-allocation entry point";
    default: return cudaGetErrorString(static_cast<cudaError_t>(code));
  }
}

}  // namespace peco

extern "C" const char* peco_error_string(int code) { return peco::error_string(code); }
extern "C" const char* peco_cluster_error_message(int code) { return peco::error_string(code); }
extern "C" const char* peco_attention_error_string(int code) { return peco::error_string(code); }

extern "C" int peco_device_status(unsigned* out, int clear, void* stream_ptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  unsigned* p = peco::device_status_ptr();
  if (!p || !out) return peco::kErrInvalidValue;
  cudaError_t e = cudaMemcpyAsync(out, p, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(p, 0, sizeof(unsigned), stream);
  if (e == cudaSuccess && clear) e = cudaStreamSynchronize(stream);
  return static_cast<int>(e);
}

extern "C" int peco_library_version(void) { return 1; }

extern "C" unsigned long long peco_launch_count(void) { return peco::g_launches.load(std::memory_order_relaxed); }
