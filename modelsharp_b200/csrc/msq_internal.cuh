// Internal declarations shared by the translation units of libms_cuda_nbits.so.
// Nothing here is part of the C ABI (include/ms_cuda_nbits.h is).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <atomic>
#include <cstdint>
#include <mutex>
#include <vector>

#include "../../include/ms_cuda_nbits.h"

namespace msq {

enum ZpKind : int { ZP_NONE = 0, ZP_PACKED = 1, ZP_F32 = 2 };

// Device-resident weights of rows [n_begin, n_end) of one MatMulNBits initializer.
//
// "fast4" handles (bits = 4, block_size a power of two >= 32) hold the kernel layout:
//   nib   uint8 [n_rows][KP/2]  KP = K rounded up to 128; each 32-bit word carries the
//                               8 codes of k = 8w..8w+7 in nibble slots ordered
//                               k-offsets {0,2,4,6,1,3,5,7} (pairs (k, k+1) sit 16 bits
//                               apart, so one mask yields both halves of a half2)
//   sc    float [n_rows][sc_pitch]   exact fp32 scales, pitch nb rounded up to 8
//   sc16  half  [n_rows][sc_pitch]   the same scales rounded to fp16 (GEMM operand path)
//   zp4   uint8 [n_rows][zp_pitch]   packed zero points as the reference packs them
//   zpf   float [n_rows][sc_pitch]   float zero points
//   strm  the decode-GEMV stream: one contiguous stage per (16-row block, k-tile of kt),
//         laid out [row block][k-tile]. Inside a stage: the codes as [64-k chunk][lane][16 B]
//         where lane (r = lane/4, t = lane%4) holds two 32-bit words per 32-k step, the
//         mma.m16n8k32 A-fragment order: byte j of the first word carries the code of
//         (row r, k 4t+j) in its low nibble and of (row r+8, k 4t+j) in its high nibble, the
//         second word the same at k + 16; then the fp32 scales [block][16 rows]; then the zero
//         points [block][16 rows] (packed nibbles, 8 bytes per block, or fp32).
// Other handles keep the reference layout (b_ref, sc_ref, zp_ref_*) for the generic
// kernel.
struct Weights {
  int device = -1;
  int n_rows = 0, K = 0, bits = 4, block_size = 0, nb = 0, blob = 0, zp_row_bytes = 0;
  int zp_kind = ZP_NONE;
  bool fast4 = false;
  bool fast8 = false;  // bits = 8, block_size 32 / 64 / 128: the decode stream only, codes one byte
                       // each in the same fragment order (see strm), zero points one byte per
                       // (block, row); every M takes the decode GEMV
  int KP = 0;
  uint8_t* nib = nullptr;
  int64_t nib_pitch = 0;
  float* sc = nullptr;
  __half* sc16 = nullptr;
  int64_t sc_pitch = 0;
  uint8_t* zp4 = nullptr;
  int64_t zp_pitch = 0;
  float* zpf = nullptr;
  uint8_t* strm = nullptr;
  int kt = 0;           // k per tile (multiple of max(block_size, 64))
  int ntiles = 0;       // k-tiles per row
  int nblk = 0;         // 16-row blocks
  int stage_bytes = 0;  // bytes per (row block, k-tile) stage
  int off_sc = 0;       // byte offset of the scales in a stage
  int off_zp = 0;       // byte offset of the zero points in a stage
  uint8_t* b_ref = nullptr;
  float* sc_ref = nullptr;
  uint8_t* zp_ref_u8 = nullptr;
  float* zp_ref_f32 = nullptr;
  int64_t device_bytes = 0;
  std::atomic<void*> gemm_state{nullptr};  // GEMM tensor maps, built by the first GEMM call
  std::mutex state_mu;                     // guards that first build on this handle only
  std::atomic<bool> gemm_layout{false};    // nib / sc / sc16 / zp planes hold the weights (packed with
                                           // them, or derived from strm at the first GEMM call)
  cudaEvent_t packed_ev = nullptr;   // recorded on the packing stream after the repack kernels
  std::atomic<bool> settled{false};  // the host has seen packed_ev complete: kernels may read
                                     // the weights before their programmatic-dependency wait
};

// ---- error and diagnostics plumbing (msq_api.cu) ----
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
void note_launch(int n = 1);
// Stream-ordered scratch from a library-private memory pool that keeps its memory between
// calls (the default pool would unmap it at every synchronisation).
int scratch_alloc(void** p, size_t bytes, cudaStream_t st);
void scratch_free(void* p, cudaStream_t st);
void note_path(const char* name);
int num_sms(int device);

// Identity of the CUDA context current on this thread (binding the current device's primary
// context when the thread has none). It is cuCtxGetId's value, unique for the life of the
// process: a CUcontext handle can come back for a new context after cudaDeviceReset or
// cuCtxDestroy, with the library's module (and its __device__ arrays and function
// attributes) loaded afresh, so per-context caches key on this id, not on the handle.
int current_context_id(unsigned long long* id);

// One-time set-up per CUDA context (a kernel's function attributes, a symbol's address):
// run(fn) calls fn() the first time it meets the current context and again only in a new
// context; fn's status is returned, and a failed fn is retried by the next call.
class ContextOnce {
 public:
  template <class F>
  int run(F&& fn) {
    unsigned long long id = 0;
    int rc = current_context_id(&id);
    if (rc != 0) return rc;
    std::lock_guard<std::mutex> lk(mu_);
    for (unsigned long long d : done_)
      if (d == id) return 0;
    rc = fn();
    if (rc == 0) done_.push_back(id);
    return rc;
  }

 private:
  std::mutex mu_;
  std::vector<unsigned long long> done_;
};

// Diagnostic counters behind msq_diag_counter.
void note_noalloc_lookup();

#define MSQ_CUDA_TRY(expr, what)                         \
  do {                                                   \
    cudaError_t _e = (expr);                             \
    if (_e != cudaSuccess) return ::msq::cuda_fail(_e, what); \
  } while (0)

// ---- repack (msq_repack.cu) ----
int repack_fast4(cudaStream_t st, Weights& w, const uint8_t* d_b, int n_begin,
                 const void* d_scales, int scales_dtype, const void* d_zp);
int repack_stream(cudaStream_t st, Weights& w, const uint8_t* d_b, int n_begin,
                  const void* d_scales, int scales_dtype, const void* d_zp);
void plan_stream(Weights& w);
// The GEMM layout (nib, sc, sc16, zp4 / zpf) of a handle packed with MSQ_PACK_LAZY_GEMM, derived
// from its stream records on the device the first time the GEMM needs it (allocates).
int ensure_gemm_layout(cudaStream_t st, Weights& w);
int read_gemv_mma_errors(cudaStream_t st, int* flags);
int read_gemm_errors(cudaStream_t st, int* flags);
// Bounded-wait budgets of the decode GEMV's and the GEMM's modules on the current device.
int set_wait_budget_gemv(unsigned long long ns);
int set_wait_budget_gemm(unsigned long long ns);
int repack_reference(cudaStream_t st, Weights& w, const uint8_t* d_b, int n_begin,
                     const void* d_scales, int scales_dtype, const void* d_zp);

// ---- kernels ----
int run_generic(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
                float* d_y, int64_t ldy);
int run_gemv(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
             float* d_y, int64_t ldy);
int run_gemv_mma(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
                 float* d_y, int64_t ldy);
// The int8-activation decode GEMV (ms_qgemm_w4a8's arithmetic), up to 8 A rows per pass.
int run_gemv_w4a8(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
                  float* d_y, int64_t ldy);
// The column-split decode GEMV (outputs to every rank's full-Y buffer) and the wait kernel.
int run_gemv_gather(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
                    const msq_wait_t* wt, const msq_gather_t* g);
int run_wait_gathered(cudaStream_t st, const msq_wait_t* wt);
// The decode GEMV with decode-step fusions (fp32 A, K % 4 == 0, 16-byte aligned A and gamma).
struct Fusion {
  const float* gamma = nullptr;  // RMSNorm of each A row folded in (scale per row, gamma per k)
  float eps = 0.f;
  int swiglu = 0;                // A rows are [gate | up] of 2K: a = silu(gate) * up
  int accumulate = 0;            // Y += result
};
int run_gemv_fused(cudaStream_t st, const Weights& w, const float* d_a, int64_t M, float* d_y, int64_t ldy,
                   const Fusion& f);
// The batched decode GEMV on tcgen05 kind::i8 (exact, 1..32 rows of A, block_size 128).
int run_gemv_tc(cudaStream_t st, Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y, int64_t ldy);
int read_gemv_tc_errors(cudaStream_t st, int* flags);
int set_wait_budget_tc(unsigned long long ns);
// operand_split: the split-operand (three fp16 MMAs per step) form of the GEMM.
int run_gemm(cudaStream_t st, Weights& w, const void* d_a, int a_dtype, int64_t M,
             float* d_y, int64_t ldy, bool operand_split = false);
void release_gemm_state(Weights& w);
// Bytes of fp16 activation staging the GEMM needs for this call (0 when A feeds TMA as is).
size_t gemm_staging_bytes(const Weights& w, const void* d_a, int a_dtype, int64_t M);
// The GEMM with its activation staging in caller-provided device memory: no allocation,
// no state kept on the handle.
int run_gemm_staged(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
                    float* d_y, int64_t ldy, void* staging, size_t staging_bytes);
// The GEMM with its staging in this library's fixed device array (msq_noalloc.cu).
int run_gemm_noalloc(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
                     float* d_y, int64_t ldy);

// ---- decoder glue (msq_decoder.cu) ----
int run_add_rmsnorm(cudaStream_t st, float* x, const float* delta, const float* gamma, float* y, int64_t rows,
                    int64_t n, float eps);
int run_rope_append(cudaStream_t st, float* qkv, int heads, int kv, int d, const float* cos_t, const float* sin_t,
                    const int64_t* pos, float* kc, float* vc, int64_t max_seq);
int run_gqa_decode(cudaStream_t st, const float* q, const float* kc, const float* vc, const int64_t* pos, float* out,
                   int heads, int kv, int d, int64_t max_seq);
int run_rope_gqa_decode(cudaStream_t st, const float* qkv, float* kc, float* vc, const float* cos_t,
                        const float* sin_t, const int64_t* pos, float* out, int heads, int kv, int d,
                        int64_t max_seq);
// Dynamic shared memory of one gqa_decode block (heads / kv <= 8, d <= 256).
size_t gqa_decode_smem(int heads, int kv, int d);
int run_swiglu(cudaStream_t st, const float* gu, float* out, int64_t n);
int run_argmax(cudaStream_t st, const float* x, int64_t n, int64_t* idx, int64_t* pos);
int run_swiglu_rows(cudaStream_t st, const float* gu, float* out, int64_t rows, int64_t n);
int run_rope_append_rows(cudaStream_t st, const float* qkv, int64_t S, int64_t pos0, int heads, int kv, int d,
                         const float* cos_t, const float* sin_t, float* q_out, float* kc, float* vc, int64_t max_seq);
int run_gqa_prefill(cudaStream_t st, const float* q, const float* kc, const float* vc, float* out, int64_t S,
                    int64_t pos0, int heads, int kv, int d, int64_t max_seq);

// Loads element idx of an activation tensor of dtype dt (f32 / f16 / bf16) as fp32.
__device__ __forceinline__ float load_act(const void* a, int dt, int64_t idx) {
  if (dt == MSQ_DT_F32) return static_cast<const float*>(a)[idx];
  if (dt == MSQ_DT_F16) return __half2float(static_cast<const __half*>(a)[idx]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(a)[idx]);
}

}  // namespace msq
