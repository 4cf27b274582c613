// An allocation-free variant of the decode GEMV entry point.
//
// nf4b_gemm asks its caller for a workspace: the split-K partial sums and the
// per-tile arrival counters of the streaming GEMV live in device memory the
// caller allocates once. Some hosts cannot do that. A plugin driven from a
// real-time audio callback must not call into an allocator on its hot path;
// a cgo or JNI host that only receives raw device pointers from another
// runtime has no allocator of its own for the device; and an embedding that
// records the whole decode step into a CUDA graph may not be free to allocate
// while it records. nf4b_gemm_noalloc serves those callers from scratch memory
// compiled into this library instead.
//
// The scratch is a file-scope __device__ array of NF4B_NOALLOC_SCRATCH_BYTES
// (4 MiB), so every GPU that loads the library holds it until the process
// exits. Host code may not use the array's name as a device pointer: the
// first call on each device looks its device address up with
// cudaGetSymbolAddress (with that device current) and reuses it for the life
// of the process. That first call should therefore happen before any stream
// capture, and a device must not be reset (cudaDeviceReset, or destroying its
// primary context) between calls: the kept address would then be stale.
//
// All calls on a device share the one array and it keeps whatever the last
// call left in it. Each call clears the arrival counters it relies on
// (cudaMemsetAsync on the call's stream) before launching, so stale contents
// are harmless for calls ordered on one stream; calls that overlap on the GPU
// (other streams, other threads) race on the same bytes and must not be issued.
// GEMV calls (1..8 activation rows) whose partial sums would not fit are
// rejected. More rows run the tensor-core GEMM: it takes the scratch for its
// split-K partial sums when they fit (so it splits exactly as nf4b_gemm with a
// workspace does) and otherwise runs unsplit.

#include <mutex>
#include <stdio.h>

#include "common.cuh"
#include "kernels.cuh"

namespace nf4b {
int report_error(int code, const char* msg);
}

namespace {

static __device__ __align__(256) unsigned char g_gemv_scratch[NF4B_NOALLOC_SCRATCH_BYTES];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64];  // device address of g_gemv_scratch, per device

}  // namespace

extern "C" int nf4b_gemm_noalloc(const nf4b_weight* w, const void* x, void* y, int rows, int epi,
                                 const void* operand, void* stream) {
  const size_t need = nf4b_gemm_workspace_size(w, rows);
  if (need == 0)  // an unsplit GEMM, or an invalid weight / row count that nf4b_gemm reports
    return nf4b_gemm(w, x, y, rows, epi, operand, nullptr, 0, stream);
  if (rows > nf4b::GEMV_REG_MAX_ROWS && need > (size_t)NF4B_NOALLOC_SCRATCH_BYTES)  // GEMM: run unsplit
    return nf4b_gemm(w, x, y, rows, epi, operand, nullptr, 0, stream);
  if (need > (size_t)NF4B_NOALLOC_SCRATCH_BYTES) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "nf4b_gemm_noalloc: this call needs %zu bytes of scratch but the built-in scratch "
             "holds %zu; pass a workspace to nf4b_gemm instead",
             need, (size_t)NF4B_NOALLOC_SCRATCH_BYTES);
    return nf4b::report_error(NF4B_ERR_WORKSPACE, msg);
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return nf4b::report_error(NF4B_ERR_DEVICE, "nf4b_gemm_noalloc: no usable current device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, g_gemv_scratch);
      if (e != cudaSuccess || ptr == nullptr) {
        char msg[256];
        snprintf(msg, sizeof(msg), "nf4b_gemm_noalloc: cudaGetSymbolAddress failed: %s",
                 cudaGetErrorString(e));
        return nf4b::report_error(NF4B_ERR_LAUNCH, msg);
      }
      g_scratch_ptr[dev] = ptr;
    }
    scratch = g_scratch_ptr[dev];
  }
  // The per-tile arrival counters at the start of the scratch must read zero
  // (GEMV_COUNTER_BYTES covers the GEMM's GEMM_COUNTER_BYTES too).
  const cudaError_t e = cudaMemsetAsync(scratch, 0, nf4b::GEMV_COUNTER_BYTES,
                                        reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "nf4b_gemm_noalloc: clearing the scratch counters failed: %s",
             cudaGetErrorString(e));
    return nf4b::report_error(NF4B_ERR_LAUNCH, msg);
  }
  return nf4b_gemm(w, x, y, rows, epi, operand, scratch, NF4B_NOALLOC_SCRATCH_BYTES, stream);
}
