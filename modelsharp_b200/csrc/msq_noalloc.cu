// The prefill GEMM for callers that cannot allocate device memory.
//
// Some hosts may not call cudaMalloc (or any allocator) on the path that runs a node: an
// engine that owns every byte of device memory through its own arena and budgets it up
// front, a plugin invoked inside another runtime's stream capture, or a caller bound by a
// memory cap that a stream-ordered pool would push past. msq_matmul (and its GEMM path) takes
// its fp16 activation staging from a stream-ordered pool; msq_matmul_noalloc instead stages
// into the fixed array below, which the CUDA module loader places in device memory together
// with the library's code.
//
//   - Size: kNoallocScratchBytes = MSQ_NOALLOC_SCRATCH_BYTES (16 MiB) per device, held from
//     the time the library's device code is loaded on a GPU until the process exits.
//   - Set-up: the first call that stages A in a CUDA context looks up the array's device
//     address with cudaGetSymbolAddress (with that context current) and caches it under the
//     context's id; that first call should come before any stream capture.
//   - Sharing: every call in a context uses the same array, which keeps the last call's
//     contents. Each call rewrites the whole staged region before the GEMM reads it, so
//     nothing needs to start at zero; calls that overlap on the GPU (two streams, or two host
//     threads without ordering between their streams) race on it.
#include "msq_internal.cuh"

#include <cuda.h>

#include <mutex>
#include <vector>

namespace msq {
namespace {

constexpr size_t kNoallocScratchBytes = MSQ_NOALLOC_SCRATCH_BYTES;

// The device-side staging array. In host code this name is a host-side stand-in for the
// symbol, not a device address: it is only ever passed to cudaGetSymbolAddress.
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

struct ScratchSlot {
  unsigned long long ctx_id;  // cuCtxGetId of the context the address belongs to
  void* ptr;
};

std::mutex g_mu;
std::vector<ScratchSlot> g_slots;

// Device address of g_noalloc_scratch in the current context, looked up once per context.
// Keyed by the context's id, not its CUcontext handle: after cudaDeviceReset or cuCtxDestroy
// a new context may get the old handle while the module (and this array) is loaded afresh,
// possibly at another address.
int scratch_address(void** out) {
  unsigned long long id = 0;
  int rc = current_context_id(&id);
  if (rc != MSQ_OK) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  for (const ScratchSlot& s : g_slots)
    if (s.ctx_id == id) {
      *out = s.ptr;
      return MSQ_OK;
    }
  void* ptr = nullptr;
  MSQ_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_noalloc_scratch), "cudaGetSymbolAddress(no-allocation scratch)");
  note_noalloc_lookup();
  g_slots.push_back({id, ptr});
  *out = ptr;
  return MSQ_OK;
}

}  // namespace

int run_gemm_noalloc(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y,
                     int64_t ldy) {
  if (!w.fast4) return fail(MSQ_E_UNSUPPORTED, "GEMM path needs bits=4 and a power-of-two block_size >= 32");
  const size_t need = gemm_staging_bytes(w, d_a, a_dtype, M);
  if (need > kNoallocScratchBytes)
    return fail(MSQ_E_INVALID,
                "msq_matmul_noalloc: staging A as fp16 needs %zu bytes (M=%lld rows of K=%d rounded up to 8 plus a row "
                "scale each) but the "
                "fixed scratch holds %zu; split M into smaller calls or pass 16-byte-aligned float16 A with "
                "K %% 8 == 0, which needs no staging",
                need, (long long)M, w.K, kNoallocScratchBytes);
  void* scratch = nullptr;
  if (need) {
    const int rc = scratch_address(&scratch);
    if (rc != MSQ_OK) return rc;
  }
  return run_gemm_staged(st, w, d_a, a_dtype, M, d_y, ldy, scratch, kNoallocScratchBytes);
}

}  // namespace msq
