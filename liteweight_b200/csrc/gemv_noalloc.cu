// INT4 dequant matmul for callers that cannot allocate device memory.
//
// lw_gemm_w4a16 wants its split-tile scratch from the caller. Some callers have
// no way to provide it: a serving runtime that hands out all device memory
// from a pool planned at start-up, a plugin host that forbids cudaMalloc
// after initialisation, or code that only gets pointers to its inputs and
// outputs. For them, lw_gemm_w4a16_noalloc runs the same kernel with its
// scratch in a fixed array that lives inside this library.
//
// The array is kNoallocScratchBytes (4 MiB) per GPU. It comes into existence
// on a device when the library's device code is first loaded there (with
// lazy module loading, at the first kernel launch or symbol lookup) and is
// held by that GPU until the process exits. Problems whose scratch need
// exceeds it are rejected with LW_ERR_WORKSPACE, before anything is enqueued.
// The first call on a device looks the array's device address up
// (cudaGetSymbolAddress), so make that first call before any stream capture.
// The address is cached per device for the life of the process: do not use
// this entry point after cudaDeviceReset (or anything else that destroys the
// device's primary context) in the same process.
// Every call clears the array's counter region on the stream before the
// kernel runs; all calls share the array, so calls that overlap on the GPU
// (different streams, or different host threads) race and must not be issued.
#include <mutex>

#include "gemv_host.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = 4u << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once
// per device with that device current). In host code the array's name is
// only a stand-in for the symbol, never a device address.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LW_ERR_LAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return LW_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return LW_ERR_LAUNCH;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return LW_OK;
}

}  // namespace

extern "C" int lw_gemm_w4a16_noalloc(const void* act, const void* qweight, const void* scales, const void* bias,
                                     void* out, int M, int N, int K, int group_size, lw_stream_t stream) {
  // Validate everything lw_gemm_w4a16 would reject before the counter clear
  // below is enqueued, so a rejected call leaves the stream untouched.
  if (!act || !qweight || !scales || !out) return LW_ERR_NULL_POINTER;
  if (M <= 0 || N <= 0 || K <= 0 || K % 2) return LW_ERR_BAD_SHAPE;
  if (group_size <= 0 || K % group_size) return LW_ERR_BAD_GROUP;
  if (reinterpret_cast<uintptr_t>(act) % 2 || reinterpret_cast<uintptr_t>(out) % 2 ||
      reinterpret_cast<uintptr_t>(scales) % 2 || (bias && reinterpret_cast<uintptr_t>(bias) % 2))
    return LW_ERR_ALIGNMENT;
  void* ws = nullptr;
  const int st = noalloc_scratch(&ws);
  if (st) return st;
  const size_t need = lw_gemm_workspace_size(4, M, N, K);
  if (need > kNoallocScratchBytes) return LW_ERR_WORKSPACE;
  if (need) {
    // The per-tile counters must start at zero; the kernel also leaves them zero.
    const cudaError_t e = cudaMemsetAsync(ws, 0, lw::kCounterBytes, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return LW_ERR_LAUNCH;
  }
  return lw_gemm_w4a16(act, qweight, scales, bias, out, M, N, K, group_size, need ? ws : nullptr, need, stream);
}
