// C ABI of libms_cuda_nbits.so (declared in include/ms_cuda_nbits.h).
//
// Host-side runtime around the kernels: argument validation with the reference's
// messages (MatMulNBitsKernel.cs:82-164), device-resident weight handles (the
// residency role of IlgpuEngine.cs:2218-2229 / 3392-3429), kernel-path dispatch, the
// host-buffer and one-shot forms, context push/pop for caller-supplied driver contexts
// (the pattern of native/src/cublas_gemm.cu:505-528), and diagnostics counters
// (NativeCuda.cs:147-150).
#include "msq_internal.cuh"

#include <cuda.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace msq {
namespace {

thread_local std::string t_last_error;
thread_local const char* t_last_path = "";
std::atomic<int64_t> g_launches{0};

using PFN_push = CUresult (*)(CUcontext);
using PFN_pop = CUresult (*)(CUcontext*);
PFN_push g_push = nullptr;
PFN_pop g_pop = nullptr;
std::once_flag g_driver_once;

void load_driver_entries() {
  std::call_once(g_driver_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxPushCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_push = reinterpret_cast<PFN_push>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxPopCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_pop = reinterpret_cast<PFN_pop>(fn);
  });
}

// Pushes a caller-supplied driver context for the duration of one C-ABI call.
struct CtxGuard {
  bool pushed = false;
  int rc = MSQ_OK;
  explicit CtxGuard(void* ctx) {
    if (!ctx) return;
    load_driver_entries();
    if (!g_push || !g_pop) {
      rc = fail(MSQ_E_CUDA, "cannot resolve cuCtxPushCurrent/cuCtxPopCurrent");
      return;
    }
    if (g_push(static_cast<CUcontext>(ctx)) != CUDA_SUCCESS) {
      rc = fail(MSQ_E_CUDA, "cuCtxPushCurrent failed");
      return;
    }
    pushed = true;
  }
  ~CtxGuard() {
    if (pushed) {
      CUcontext c;
      g_pop(&c);
    }
  }
};

const char* dtype_name(int dt) {
  switch (dt) {
    case MSQ_DT_F32: return "Float32";
    case MSQ_DT_F64: return "Float64";
    case MSQ_DT_F16: return "Float16";
    case MSQ_DT_I32: return "Int32";
    case MSQ_DT_I64: return "Int64";
    case MSQ_DT_I8: return "Int8";
    case MSQ_DT_U8: return "UInt8";
    case MSQ_DT_BOOL: return "Boolean";
    case MSQ_DT_BF16: return "BFloat16";
    default: return "Unknown";
  }
}

bool is_float_act(int dt) { return dt == MSQ_DT_F32 || dt == MSQ_DT_F16 || dt == MSQ_DT_BF16; }

bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

// Static shape checks shared by msq_check_node and msq_pack (MatMulNBitsKernel.cs:87-145).
int check_weights(int N, int K, int bits, int bs, int64_t b_len, int64_t scales_len, int scales_dtype,
                  int zp_dtype, int64_t zp_len) {
  if (N <= 0 || K <= 0)
    return fail(MSQ_E_INVALID, "MatMulNBits requires positive N and K attributes (got N=%d, K=%d).", N, K);
  if (bits != 4 && bits != 8)
    return fail(MSQ_E_INVALID, "MatMulNBits supports bits=4 or bits=8; got %d.", bits);
  if (bs <= 0) return fail(MSQ_E_INVALID, "MatMulNBits requires a positive block_size; got %d.", bs);
  const int64_t nb = ((int64_t)K + bs - 1) / bs;
  const int64_t blob = ((int64_t)bs * bits + 7) / 8;
  const int64_t expected_b = (int64_t)N * nb * blob;
  if (b_len != expected_b)
    return fail(MSQ_E_INVALID,
                "MatMulNBits B has %lld elements; expected %lld (N=%d \xC3\x97 n_blocks_per_row=%lld "
                "\xC3\x97 blob_size=%lld).",
                (long long)b_len, (long long)expected_b, N, (long long)nb, (long long)blob);
  if (!is_float_act(scales_dtype))
    return fail(MSQ_E_INVALID, "MatMulNBits scales must be Float32 or Float16; got %s.", dtype_name(scales_dtype));
  const int64_t expected_scales = (int64_t)N * nb;
  if (scales_len != expected_scales)
    return fail(MSQ_E_INVALID,
                "MatMulNBits scales has %lld elements; expected %lld (N=%d \xC3\x97 n_blocks_per_row=%lld).",
                (long long)scales_len, (long long)expected_scales, N, (long long)nb);
  const int64_t zp_row = (nb * bits + 7) / 8;
  if (zp_dtype == MSQ_DT_ABSENT) return MSQ_OK;
  if (zp_dtype == MSQ_DT_F32) {
    if (zp_len != expected_scales)
      return fail(MSQ_E_INVALID, "MatMulNBits float zero_points has %lld elements; expected %lld.",
                  (long long)zp_len, (long long)expected_scales);
  } else if (zp_dtype == MSQ_DT_U8) {
    const int64_t expected_zp = (int64_t)N * zp_row;
    if (zp_len != expected_zp)
      return fail(MSQ_E_INVALID, "MatMulNBits packed zero_points has %lld bytes; expected %lld (N=%d \xC3\x97 %lld).",
                  (long long)zp_len, (long long)expected_zp, N, (long long)zp_row);
  } else {
    return fail(MSQ_E_INVALID, "MatMulNBits zero_points must be Float32 or UInt8; got %s.", dtype_name(zp_dtype));
  }
  return MSQ_OK;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  return MSQ_OK;
}

template <typename T>
int dev_alloc(T** p, size_t n, int64_t* total) {
  *p = nullptr;
  if (n == 0) return MSQ_OK;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MSQ_E_OOM, "device allocation of %zu bytes failed: %s", n * sizeof(T), cudaGetErrorString(e));
  }
  *total += (int64_t)(n * sizeof(T));
  return MSQ_OK;
}

void free_weights(Weights* w) {
  if (!w) return;
  release_gemm_state(*w);
  if (w->packed_ev) cudaEventDestroy(w->packed_ev);
  void* ptrs[] = {w->nib, w->sc, w->sc16, w->zp4, w->zpf, w->strm, w->b_ref, w->sc_ref, w->zp_ref_u8, w->zp_ref_f32};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  delete w;
}

int pack_impl(cudaStream_t st, const uint8_t* d_b, int64_t b_len, const void* d_scales, int scales_dtype,
              int64_t scales_len, const void* d_zp, int zp_dtype, int64_t zp_len, int N, int K, int bits,
              int bs, int n_begin, int n_end, int flags, msq_weights_t* out) {
  if (!out) return fail(MSQ_E_INVALID, "msq_pack: out handle pointer is NULL");
  *out = nullptr;
  int rc = check_weights(N, K, bits, bs, b_len, scales_len, scales_dtype, zp_dtype, zp_len);
  if (rc != MSQ_OK) return rc;
  if (n_begin < 0 || n_end > N || n_begin >= n_end)
    return fail(MSQ_E_INVALID, "msq_pack: row range [%d, %d) is not inside [0, %d)", n_begin, n_end, N);
  if (!d_b || !d_scales || (zp_dtype != MSQ_DT_ABSENT && !d_zp))
    return fail(MSQ_E_INVALID, "msq_pack: NULL device pointer");

  Weights* w = new Weights();
  rc = current_device(&w->device);
  if (rc != MSQ_OK) {
    delete w;
    return rc;
  }
  w->n_rows = n_end - n_begin;
  w->K = K;
  w->bits = bits;
  w->block_size = bs;
  w->nb = (K + bs - 1) / bs;
  w->blob = (bs * bits + 7) / 8;
  w->zp_row_bytes = (w->nb * bits + 7) / 8;
  w->zp_kind = zp_dtype == MSQ_DT_U8 ? ZP_PACKED : zp_dtype == MSQ_DT_F32 ? ZP_F32 : ZP_NONE;
  w->fast4 = bits == 4 && bs >= 32 && pow2(bs) && !(flags & MSQ_PACK_GENERIC_ONLY);
  w->fast8 = bits == 8 && (bs == 32 || bs == 64 || bs == 128) && !(flags & MSQ_PACK_GENERIC_ONLY);

  const size_t rows = (size_t)w->n_rows;
  if (w->fast4) {
    w->KP = (K + 127) / 128 * 128;
    w->nib_pitch = w->KP / 2;
    w->sc_pitch = (w->nb + 7) / 8 * 8;
    w->zp_pitch = (w->zp_row_bytes + 15) / 16 * 16;
    if (!(flags & MSQ_PACK_LAZY_GEMM)) {
      rc = dev_alloc(&w->nib, rows * (size_t)w->nib_pitch, &w->device_bytes);
      if (rc == MSQ_OK) rc = dev_alloc(&w->sc, rows * (size_t)w->sc_pitch, &w->device_bytes);
      if (rc == MSQ_OK) rc = dev_alloc(&w->sc16, rows * (size_t)w->sc_pitch, &w->device_bytes);
      if (rc == MSQ_OK && w->zp_kind == ZP_PACKED) rc = dev_alloc(&w->zp4, rows * (size_t)w->zp_pitch, &w->device_bytes);
      if (rc == MSQ_OK && w->zp_kind == ZP_F32) rc = dev_alloc(&w->zpf, rows * (size_t)w->sc_pitch, &w->device_bytes);
      if (rc == MSQ_OK) rc = repack_fast4(st, *w, d_b, n_begin, d_scales, scales_dtype, d_zp);
      if (rc == MSQ_OK) w->gemm_layout.store(true, std::memory_order_release);
    }
    plan_stream(*w);
    if (rc == MSQ_OK)
      rc = dev_alloc(&w->strm, (size_t)w->nblk * w->ntiles * w->stage_bytes, &w->device_bytes);
    if (rc == MSQ_OK) rc = repack_stream(st, *w, d_b, n_begin, d_scales, scales_dtype, d_zp);
  } else if (w->fast8) {
    plan_stream(*w);
    rc = dev_alloc(&w->strm, (size_t)w->nblk * w->ntiles * w->stage_bytes, &w->device_bytes);
    if (rc == MSQ_OK) rc = repack_stream(st, *w, d_b, n_begin, d_scales, scales_dtype, d_zp);
  } else {
    rc = dev_alloc(&w->b_ref, rows * (size_t)w->nb * w->blob, &w->device_bytes);
    if (rc == MSQ_OK) rc = dev_alloc(&w->sc_ref, rows * (size_t)w->nb, &w->device_bytes);
    if (rc == MSQ_OK && w->zp_kind == ZP_PACKED)
      rc = dev_alloc(&w->zp_ref_u8, rows * (size_t)w->zp_row_bytes, &w->device_bytes);
    if (rc == MSQ_OK && w->zp_kind == ZP_F32) rc = dev_alloc(&w->zp_ref_f32, rows * (size_t)w->nb, &w->device_bytes);
    if (rc == MSQ_OK) rc = repack_reference(st, *w, d_b, n_begin, d_scales, scales_dtype, d_zp);
  }
  if (rc != MSQ_OK) {
    cudaStreamSynchronize(st);
    free_weights(w);
    return rc;
  }
  if (cudaEventCreateWithFlags(&w->packed_ev, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventRecord(w->packed_ev, st) != cudaSuccess) {
    cudaGetLastError();  // without the event the weights count as unsettled (no early reads)
    if (w->packed_ev) cudaEventDestroy(w->packed_ev);
    w->packed_ev = nullptr;
  }
  *out = reinterpret_cast<msq_weights_t>(w);
  return MSQ_OK;
}

// Marks the weights settled once the host sees their repack complete. Skipped while the
// stream is being captured (event queries are not allowed then); the weights stay
// unsettled until a later uncaptured call.
void refresh_settled(Weights& w, cudaStream_t st) {
  if (w.settled.load(std::memory_order_relaxed) || !w.packed_ev) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  if (cs != cudaStreamCaptureStatusNone) return;
  const cudaError_t e = cudaEventQuery(w.packed_ev);
  if (e == cudaSuccess) w.settled.store(true, std::memory_order_relaxed);
  else if (cudaPeekAtLastError() == cudaErrorNotReady) cudaGetLastError();  // clear only our own status
}

int matmul_impl(cudaStream_t st, Weights* w, const void* d_a, int a_dtype, int64_t M, float* d_y, int64_t ldy,
                int path) {
  if (!w) return fail(MSQ_E_INVALID, "msq_matmul: NULL weights handle");
  if (!is_float_act(a_dtype))
    return fail(MSQ_E_INVALID, "MatMulNBits A must be Float32 or Float16; got %s.", dtype_name(a_dtype));
  if (M < 0) return fail(MSQ_E_INVALID, "msq_matmul: negative M (%lld)", (long long)M);
  if (ldy < w->n_rows) return fail(MSQ_E_INVALID, "msq_matmul: ldy %lld < rows %d", (long long)ldy, w->n_rows);
  if (M == 0) {
    note_path("empty");
    return MSQ_OK;
  }
  if (!d_a || !d_y) return fail(MSQ_E_INVALID, "msq_matmul: NULL device pointer");
  int dev;
  int rc = current_device(&dev);
  if (rc != MSQ_OK) return rc;
  if (dev != w->device)
    return fail(MSQ_E_INVALID, "weights handle lives on device %d but the current device is %d", w->device, dev);
  refresh_settled(*w, st);
  if (path == MSQ_PATH_AUTO || path == MSQ_PATH_AUTO_SPLIT) {
    if (!w->fast4 && !w->fast8) path = MSQ_PATH_GENERIC;
    else if (w->fast8) path = MSQ_PATH_GEMV;
    else if (M >= 5 && M <= 32 && w->block_size == 128) path = MSQ_PATH_GEMV_TC;  // exact, weights read once
    else if (M >= 17 && w->K >= 64) path = path == MSQ_PATH_AUTO ? MSQ_PATH_GEMM : MSQ_PATH_GEMM_SPLIT;
    else path = MSQ_PATH_GEMV;
  }
  switch (path) {
    case MSQ_PATH_GENERIC: return run_generic(st, *w, d_a, a_dtype, M, d_y, ldy);
    case MSQ_PATH_GEMV: return run_gemv(st, *w, d_a, a_dtype, M, d_y, ldy);
    case MSQ_PATH_GEMM: return run_gemm(st, *w, d_a, a_dtype, M, d_y, ldy);
    case MSQ_PATH_GEMM_SPLIT: return run_gemm(st, *w, d_a, a_dtype, M, d_y, ldy, true);
    case MSQ_PATH_GEMV_TC: return run_gemv_tc(st, *w, d_a, a_dtype, M, d_y, ldy);
    default: return fail(MSQ_E_INVALID, "msq_matmul_ex: unknown path %d", path);
  }
}

size_t act_elem_size(int dt) { return dt == MSQ_DT_F32 ? 4 : 2; }

}  // namespace

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? MSQ_E_OOM : MSQ_E_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e),
              cudaGetErrorName(e));
}

void note_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

namespace {
std::mutex g_pool_mu;
cudaMemPool_t g_pools[64] = {};
std::atomic<int64_t> g_pool_allocs{0};
std::atomic<int64_t> g_noalloc_lookups{0};

using PFN_getcur = CUresult (*)(CUcontext*);
using PFN_getid = CUresult (*)(CUcontext, unsigned long long*);
PFN_getcur g_getcur = nullptr;
PFN_getid g_getid = nullptr;
std::once_flag g_ctxid_once;
}  // namespace

void note_noalloc_lookup() { g_noalloc_lookups.fetch_add(1, std::memory_order_relaxed); }

int current_context_id(unsigned long long* id) {
  std::call_once(g_ctxid_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_getcur = reinterpret_cast<PFN_getcur>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_getid = reinterpret_cast<PFN_getid>(fn);
  });
  if (!g_getcur || !g_getid) return fail(MSQ_E_CUDA, "cannot resolve cuCtxGetCurrent/cuCtxGetId from the driver");
  CUcontext ctx = nullptr;
  if (g_getcur(&ctx) != CUDA_SUCCESS) return fail(MSQ_E_CUDA, "cuCtxGetCurrent failed");
  if (!ctx) {
    // A thread that has made no CUDA call yet: bind the current device's primary context.
    int dev = 0;
    MSQ_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    MSQ_CUDA_TRY(cudaSetDevice(dev), "cudaSetDevice");
    if (g_getcur(&ctx) != CUDA_SUCCESS || !ctx) return fail(MSQ_E_CUDA, "no current CUDA context");
  }
  if (g_getid(ctx, id) != CUDA_SUCCESS) return fail(MSQ_E_CUDA, "cuCtxGetId failed");
  return MSQ_OK;
}

int scratch_alloc(void** p, size_t bytes, cudaStream_t st) {
  g_pool_allocs.fetch_add(1, std::memory_order_relaxed);
  int dev = 0;
  MSQ_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (dev >= 0 && dev < 64) pool = g_pools[dev];
    if (!pool) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      MSQ_CUDA_TRY(cudaMemPoolCreate(&pool, &props), "cudaMemPoolCreate");
      uint64_t keep = ~0ull;
      MSQ_CUDA_TRY(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep), "pool attribute");
      if (dev >= 0 && dev < 64) g_pools[dev] = pool;
    }
  }
  MSQ_CUDA_TRY(cudaMallocFromPoolAsync(p, bytes, pool, st), "scratch allocation");
  return MSQ_OK;
}

void scratch_free(void* p, cudaStream_t st) {
  if (p) cudaFreeAsync(p, st);
}
void note_path(const char* name) { t_last_path = name; }

int num_sms(int device) {
  static int cache[64] = {0};
  if (device >= 0 && device < 64 && cache[device]) return cache[device];
  int v = 148;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
  if (device >= 0 && device < 64) cache[device] = v;
  return v;
}

}  // namespace msq

using namespace msq;

extern "C" {

const char* msq_build_info(void) {
  static std::string s = [] {
    char buf[256];
    snprintf(buf, sizeof buf, "libms_cuda_nbits (nvcc %d.%d, sm_100a, built %s %s)", __CUDACC_VER_MAJOR__,
             __CUDACC_VER_MINOR__, __DATE__, __TIME__);
    return std::string(buf);
  }();
  return s.c_str();
}

int msq_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return 0;
  }
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
  return major == 10 ? 1 : 0;
}

const char* msq_last_error(void) { return t_last_error.c_str(); }

int64_t msq_diag_counter(int which) {
  switch (which) {
    case MSQ_DIAG_POOL_ALLOCS: return g_pool_allocs.load();
    case MSQ_DIAG_NOALLOC_LOOKUPS: return g_noalloc_lookups.load();
    case MSQ_DIAG_POOL_RESERVED: {
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
      cudaMemPool_t pool;
      {
        std::lock_guard<std::mutex> lk(g_pool_mu);
        pool = g_pools[dev];
      }
      if (!pool) return 0;
      uint64_t v = 0;
      if (cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &v) != cudaSuccess) return -1;
      return (int64_t)v;
    }
    default: return -1;
  }
}
int64_t msq_launch_count(void) { return g_launches.load(); }
const char* msq_last_path(void) { return t_last_path; }

int msq_check_node(int N, int K, int bits, int block_size, int64_t b_len, int64_t scales_len, int zp_dtype,
                   int64_t zp_len, const int64_t* g_idx, int64_t g_idx_len, const int64_t* a_dims, int a_rank,
                   int64_t* M_out) {
  int rc = check_weights(N, K, bits, block_size, b_len, scales_len, MSQ_DT_F32, zp_dtype, zp_len);
  if (rc != MSQ_OK) return rc;
  if (g_idx && g_idx_len > 0) {
    for (int64_t k = 0; k < g_idx_len; ++k)
      if (g_idx[k] != k / block_size)
        return fail(MSQ_E_UNSUPPORTED, "MatMulNBits g_idx with a non-trivial block permutation is not supported.");
  }
  if (a_rank <= 0 || !a_dims || a_dims[a_rank - 1] != K) {
    std::string dims;
    for (int i = 0; i < a_rank && a_dims; ++i) {
      if (i) dims += ",";
      dims += std::to_string((long long)a_dims[i]);
    }
    return fail(MSQ_E_INVALID, "MatMulNBits A inner dimension must equal K=%d; got shape [%s].", K, dims.c_str());
  }
  int64_t M = 1;
  for (int i = 0; i < a_rank - 1; ++i) M *= a_dims[i];
  if (M_out) *M_out = M;
  return MSQ_OK;
}

int msq_pack(void* cu_ctx, void* stream, const uint8_t* d_b, int64_t b_len, const void* d_scales, int scales_dtype,
             int64_t scales_len, const void* d_zp, int zp_dtype, int64_t zp_len, int N, int K, int bits,
             int block_size, int n_begin, int n_end, int flags, msq_weights_t* out) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  return pack_impl(static_cast<cudaStream_t>(stream), d_b, b_len, d_scales, scales_dtype, scales_len, d_zp,
                   zp_dtype, zp_len, N, K, bits, block_size, n_begin, n_end, flags, out);
}

int msq_pack_host(void* cu_ctx, void* stream, const uint8_t* b, int64_t b_len, const void* scales,
                  int scales_dtype, int64_t scales_len, const void* zp, int zp_dtype, int64_t zp_len, int N,
                  int K, int bits, int block_size, int n_begin, int n_end, int flags, msq_weights_t* out) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (out) *out = nullptr;
  int rc = check_weights(N, K, bits, block_size, b_len, scales_len, scales_dtype, zp_dtype, zp_len);
  if (rc != MSQ_OK) return rc;
  if (!b || !scales || (zp_dtype != MSQ_DT_ABSENT && !zp)) return fail(MSQ_E_INVALID, "msq_pack_host: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t sbytes = (size_t)scales_len * (scales_dtype == MSQ_DT_F32 ? 4 : 2);
  const size_t zbytes = zp_dtype == MSQ_DT_ABSENT ? 0 : (size_t)zp_len * (zp_dtype == MSQ_DT_F32 ? 4 : 1);
  uint8_t* db = nullptr;
  void *ds = nullptr, *dz = nullptr;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&db), (size_t)b_len);
  if (e == cudaSuccess) e = cudaMalloc(&ds, sbytes);
  if (e == cudaSuccess && zbytes) e = cudaMalloc(&dz, zbytes);
  if (e == cudaSuccess) e = cudaMemcpyAsync(db, b, (size_t)b_len, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(ds, scales, sbytes, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && zbytes) e = cudaMemcpyAsync(dz, zp, zbytes, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    rc = pack_impl(st, db, b_len, ds, scales_dtype, scales_len, dz, zp_dtype, zp_len, N, K, bits, block_size,
                   n_begin, n_end, flags, out);
  else
    rc = cuda_fail(e, "msq_pack_host upload");
  cudaError_t se = cudaStreamSynchronize(st);
  cudaFree(db);
  cudaFree(ds);
  if (dz) cudaFree(dz);
  if (rc == MSQ_OK && se != cudaSuccess) {
    msq_free(out ? *out : nullptr);
    if (out) *out = nullptr;
    return cuda_fail(se, "msq_pack_host synchronize");
  }
  return rc;
}

int msq_weights_query(msq_weights_t h, int* n_rows, int* K, int* bits, int* block_size, int64_t* device_bytes) {
  Weights* w = reinterpret_cast<Weights*>(h);
  if (!w) return fail(MSQ_E_INVALID, "msq_weights_query: NULL handle");
  if (n_rows) *n_rows = w->n_rows;
  if (K) *K = w->K;
  if (bits) *bits = w->bits;
  if (block_size) *block_size = w->block_size;
  if (device_bytes) *device_bytes = w->device_bytes;
  return MSQ_OK;
}

int msq_free(msq_weights_t h) {
  free_weights(reinterpret_cast<Weights*>(h));
  return MSQ_OK;
}

int msq_matmul(void* cu_ctx, void* stream, msq_weights_t w, const void* d_a, int a_dtype, int64_t M, float* d_y,
               int64_t ldy) {
  return msq_matmul_ex(cu_ctx, stream, w, d_a, a_dtype, M, d_y, ldy, MSQ_PATH_AUTO);
}

int msq_matmul_ex(void* cu_ctx, void* stream, msq_weights_t w, const void* d_a, int a_dtype, int64_t M, float* d_y,
                  int64_t ldy, int path) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  return matmul_impl(static_cast<cudaStream_t>(stream), reinterpret_cast<Weights*>(w), d_a, a_dtype, M, d_y, ldy,
                     path);
}

int msq_matmul_w4a8(void* cu_ctx, void* stream, msq_weights_t h, const void* d_a, int a_dtype, int64_t M, float* d_y,
                    int64_t ldy) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  Weights* w = reinterpret_cast<Weights*>(h);
  if (!w) return fail(MSQ_E_INVALID, "msq_matmul_w4a8: NULL weights handle");
  if (!is_float_act(a_dtype))
    return fail(MSQ_E_INVALID, "MatMulNBits A must be Float32 or Float16; got %s.", dtype_name(a_dtype));
  if (M < 0 || ldy < w->n_rows) return fail(MSQ_E_INVALID, "msq_matmul_w4a8: bad M (%lld) or ldy", (long long)M);
  if (M == 0) return MSQ_OK;
  if (!d_a || !d_y) return fail(MSQ_E_INVALID, "msq_matmul_w4a8: NULL device pointer");
  if (!w->fast4 || !w->strm)
    return fail(MSQ_E_UNSUPPORTED, "msq_matmul_w4a8 needs bits=4 and block_size 32, 64 or 128");
  int dev;
  const int rc = current_device(&dev);
  if (rc != MSQ_OK) return rc;
  if (dev != w->device)
    return fail(MSQ_E_INVALID, "weights handle lives on device %d but the current device is %d", w->device, dev);
  refresh_settled(*w, static_cast<cudaStream_t>(stream));
  return run_gemv_w4a8(static_cast<cudaStream_t>(stream), *w, d_a, a_dtype, M, d_y, ldy);
}

namespace {

// Enqueues the host-buffer form on `st`: pool scratch for A and Y, the upload, the op, the
// download and the scratch's stream-ordered release. Nothing waits for the GPU here.
int host_enqueue(cudaStream_t st, Weights* w, const void* a, int a_dtype, int64_t M, float* y, const char* who) {
  if (!w) return fail(MSQ_E_INVALID, "%s: NULL weights handle", who);
  if (!is_float_act(a_dtype))
    return fail(MSQ_E_INVALID, "MatMulNBits A must be Float32 or Float16; got %s.", dtype_name(a_dtype));
  if (M <= 0) return M == 0 ? MSQ_OK : fail(MSQ_E_INVALID, "%s: negative M", who);
  if (!a || !y) return fail(MSQ_E_INVALID, "%s: NULL host pointer", who);
  const size_t abytes = (size_t)M * w->K * act_elem_size(a_dtype);
  const size_t ybytes = (size_t)M * w->n_rows * sizeof(float);
  // one pool block: A, then Y at the next 256-byte boundary
  const size_t yoff = (abytes + 255) / 256 * 256;
  void* da = nullptr;
  const int arc = scratch_alloc(&da, yoff + ybytes, st);
  if (arc != MSQ_OK) return arc;
  float* dy = reinterpret_cast<float*>(static_cast<uint8_t*>(da) + yoff);
  cudaError_t e;
  int rc = MSQ_OK;
  e = cudaMemcpyAsync(da, a, abytes, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) rc = cuda_fail(e, "host-buffer upload");
  if (rc == MSQ_OK) rc = matmul_impl(st, w, da, a_dtype, M, dy, w->n_rows, MSQ_PATH_AUTO);
  if (rc == MSQ_OK) {
    e = cudaMemcpyAsync(y, dy, ybytes, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) rc = cuda_fail(e, "host-buffer download");
  }
  scratch_free(da, st);
  return rc;
}

}  // namespace

int msq_matmul_host(void* cu_ctx, void* stream, msq_weights_t h, const void* a, int a_dtype, int64_t M, float* y) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = host_enqueue(st, reinterpret_cast<Weights*>(h), a, a_dtype, M, y, "msq_matmul_host");
  if (!h || !is_float_act(a_dtype) || M <= 0 || !a || !y) return rc;  // rejected before anything was enqueued
  const cudaError_t e = cudaStreamSynchronize(st);
  if (rc == MSQ_OK && e != cudaSuccess) rc = cuda_fail(e, "msq_matmul_host synchronize");
  return rc;
}

int msq_matmul_host_async(void* cu_ctx, void* stream, msq_weights_t h, const void* a, int a_dtype, int64_t M,
                          float* y) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  return host_enqueue(static_cast<cudaStream_t>(stream), reinterpret_cast<Weights*>(h), a, a_dtype, M, y,
                      "msq_matmul_host_async");
}

int msq_matmul_noalloc(void* cu_ctx, void* stream, msq_weights_t h, const void* d_a, int a_dtype, int64_t M,
                       float* d_y, int64_t ldy) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  Weights* w = reinterpret_cast<Weights*>(h);
  if (!w) return fail(MSQ_E_INVALID, "msq_matmul_noalloc: NULL weights handle");
  if (!is_float_act(a_dtype))
    return fail(MSQ_E_INVALID, "MatMulNBits A must be Float32 or Float16; got %s.", dtype_name(a_dtype));
  if (M < 0) return fail(MSQ_E_INVALID, "msq_matmul_noalloc: negative M (%lld)", (long long)M);
  if (ldy < w->n_rows)
    return fail(MSQ_E_INVALID, "msq_matmul_noalloc: ldy %lld < rows %d", (long long)ldy, w->n_rows);
  if (M == 0) {
    note_path("empty");
    return MSQ_OK;
  }
  if (!d_a || !d_y) return fail(MSQ_E_INVALID, "msq_matmul_noalloc: NULL device pointer");
  int dev;
  int rc = current_device(&dev);
  if (rc != MSQ_OK) return rc;
  if (dev != w->device)
    return fail(MSQ_E_INVALID, "weights handle lives on device %d but the current device is %d", w->device, dev);
  return run_gemm_noalloc(static_cast<cudaStream_t>(stream), *w, d_a, a_dtype, M, d_y, ldy);
}

int msq_set_wait_budget(void* cu_ctx, int64_t ns) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  const unsigned long long v = ns > 0 ? (unsigned long long)ns : 2000000000ull;
  int rc = set_wait_budget_gemv(v);
  if (rc == MSQ_OK) rc = set_wait_budget_gemm(v);
  if (rc == MSQ_OK) rc = set_wait_budget_tc(v);
  return rc;
}

int msq_device_status(void* cu_ctx, void* stream) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int fv = 0, fm = 0, ft = 0;
  int rc = read_gemv_mma_errors(st, &fv);
  if (rc == MSQ_OK) rc = read_gemm_errors(st, &fm);
  if (rc == MSQ_OK) rc = read_gemv_tc_errors(st, &ft);
  if (rc != MSQ_OK) return rc;
  static const char* what[] = {"", "waiting for a stage to arrive", "waiting for a free stage",
                               "waiting for the tensor core", "draining in-flight copies",
                               "waiting for other ranks' shards of a gathered input"};
  if (fv) return fail(MSQ_E_TIMEOUT, "decode GEMV kernel gave up %s", what[fv > 0 && fv < 6 ? fv : 0]);
  if (fm) return fail(MSQ_E_TIMEOUT, "GEMM kernel gave up %s", what[fm > 0 && fm < 6 ? fm : 0]);
  if (ft) return fail(MSQ_E_TIMEOUT, "tensor-core decode GEMV kernel gave up %s", what[ft > 0 && ft < 6 ? ft : 0]);
  return MSQ_OK;
}

int msq_xbuf_alloc(void* cu_ctx, int64_t bytes, void** d_ptr) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!d_ptr || bytes <= 0) return fail(MSQ_E_INVALID, "msq_xbuf_alloc: need a positive size and an output pointer");
  *d_ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return cuda_fail(e, "msq_xbuf_alloc");
  e = cudaMemset(p, 0, (size_t)bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "msq_xbuf_alloc zero fill");
  }
  *d_ptr = p;
  return MSQ_OK;
}

int msq_xbuf_free(void* cu_ctx, void* d_ptr) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (d_ptr) MSQ_CUDA_TRY(cudaFree(d_ptr), "msq_xbuf_free");
  return MSQ_OK;
}

int msq_ipc_handle(void* cu_ctx, void* d_ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == MSQ_IPC_HANDLE_BYTES, "IPC handle size");
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!d_ptr || !handle) return fail(MSQ_E_INVALID, "msq_ipc_handle: NULL pointer");
  cudaIpcMemHandle_t h;
  MSQ_CUDA_TRY(cudaIpcGetMemHandle(&h, d_ptr), "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof h);
  return MSQ_OK;
}

int msq_ipc_open(void* cu_ctx, const void* handle, void** d_ptr) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!d_ptr || !handle) return fail(MSQ_E_INVALID, "msq_ipc_open: NULL pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  *d_ptr = nullptr;
  MSQ_CUDA_TRY(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return MSQ_OK;
}

int msq_ipc_close(void* cu_ctx, void* d_ptr) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (d_ptr) MSQ_CUDA_TRY(cudaIpcCloseMemHandle(d_ptr), "cudaIpcCloseMemHandle");
  return MSQ_OK;
}

namespace {
int check_wait(const msq_wait_t* wt, const char* fn) {
  if (!wt) return MSQ_OK;
  if (!wt->arrivals || !wt->produced) return fail(MSQ_E_INVALID, "%s: wait counters are NULL", fn);
  if (wt->nranks < 1 || wt->nranks > MSQ_MAX_RANKS)
    return fail(MSQ_E_INVALID, "%s: wait over %d ranks (1..%d)", fn, wt->nranks, MSQ_MAX_RANKS);
  return MSQ_OK;
}
}  // namespace

int msq_matmul_gather(void* cu_ctx, void* stream, msq_weights_t h, const void* d_a, int a_dtype, int64_t M,
                      const msq_wait_t* wait, const msq_gather_t* gather) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  Weights* w = reinterpret_cast<Weights*>(h);
  if (!w) return fail(MSQ_E_INVALID, "msq_matmul_gather: NULL weights handle");
  if (!w->fast4) return fail(MSQ_E_UNSUPPORTED, "msq_matmul_gather needs bits=4 and a power-of-two block_size >= 32");
  if (!is_float_act(a_dtype))
    return fail(MSQ_E_INVALID, "MatMulNBits A must be Float32 or Float16; got %s.", dtype_name(a_dtype));
  if (M < 1 || M > 4) return fail(MSQ_E_UNSUPPORTED, "msq_matmul_gather takes 1..4 A rows; got %lld", (long long)M);
  if (!d_a || !gather) return fail(MSQ_E_INVALID, "msq_matmul_gather: NULL pointer");
  if (gather->nranks < 1 || gather->nranks > MSQ_MAX_RANKS || gather->rank < 0 || gather->rank >= gather->nranks)
    return fail(MSQ_E_INVALID, "msq_matmul_gather: rank %d of %d ranks", gather->rank, gather->nranks);
  for (int r = 0; r < gather->nranks; ++r)
    if (!gather->y[r] || !gather->arrivals[r])
      return fail(MSQ_E_INVALID, "msq_matmul_gather: rank %d's buffer or counter is NULL", r);
  if (!gather->done || !gather->produced) return fail(MSQ_E_INVALID, "msq_matmul_gather: NULL counter");
  if (gather->col0 < 0 || gather->ldy < gather->col0 + w->n_rows)
    return fail(MSQ_E_INVALID, "msq_matmul_gather: columns [%lld, %lld) do not fit a row of %lld",
                (long long)gather->col0, (long long)(gather->col0 + w->n_rows), (long long)gather->ldy);
  int rc = check_wait(wait, "msq_matmul_gather");
  if (rc != MSQ_OK) return rc;
  int dev;
  rc = current_device(&dev);
  if (rc != MSQ_OK) return rc;
  if (dev != w->device)
    return fail(MSQ_E_INVALID, "weights handle lives on device %d but the current device is %d", w->device, dev);
  refresh_settled(*w, static_cast<cudaStream_t>(stream));
  return run_gemv_gather(static_cast<cudaStream_t>(stream), *w, d_a, a_dtype, M, wait, gather);
}

int msq_matmul_fused(void* cu_ctx, void* stream, msq_weights_t h, const float* d_a, int64_t M, float* d_y,
                     int64_t ldy, const msq_fusion_t* fusion) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  Weights* w = reinterpret_cast<Weights*>(h);
  if (!w) return fail(MSQ_E_INVALID, "msq_matmul_fused: NULL weights handle");
  if (!fusion) return fail(MSQ_E_INVALID, "msq_matmul_fused: NULL fusion");
  if (fusion->rms_gamma && fusion->swiglu)
    return fail(MSQ_E_INVALID, "msq_matmul_fused: RMSNorm and SwiGLU inputs are exclusive");
  if (M < 0) return fail(MSQ_E_INVALID, "msq_matmul_fused: negative M (%lld)", (long long)M);
  if (ldy < w->n_rows) return fail(MSQ_E_INVALID, "msq_matmul_fused: ldy %lld < rows %d", (long long)ldy, w->n_rows);
  if (M == 0) return MSQ_OK;
  if (!d_a || !d_y) return fail(MSQ_E_INVALID, "msq_matmul_fused: NULL device pointer");
  if (!w->fast4 || !w->strm || M > 16 || w->K % 4 ||
      ((uintptr_t)d_a | (uintptr_t)fusion->rms_gamma) & 15)
    return fail(MSQ_E_UNSUPPORTED,
                "msq_matmul_fused needs the decode GEMV (bits 4, block_size 32/64/128, M <= 16), K %% 4 == 0 and "
                "16-byte aligned A and gamma");
  int dev;
  int rc = current_device(&dev);
  if (rc != MSQ_OK) return rc;
  if (dev != w->device)
    return fail(MSQ_E_INVALID, "weights handle lives on device %d but the current device is %d", w->device, dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  refresh_settled(*w, st);
  Fusion f;
  f.gamma = fusion->rms_gamma;
  f.eps = fusion->rms_eps;
  f.swiglu = fusion->swiglu ? 1 : 0;
  f.accumulate = fusion->accumulate ? 1 : 0;
  rc = run_gemv_fused(st, *w, d_a, M, d_y, ldy, f);
  if (rc == MSQ_E_UNSUPPORTED) return fail(rc, "msq_matmul_fused: these weights do not fit the decode GEMV");
  return rc;
}

int msq_wait_gathered(void* cu_ctx, void* stream, const msq_wait_t* wait) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!wait) return fail(MSQ_E_INVALID, "msq_wait_gathered: NULL wait");
  int rc = check_wait(wait, "msq_wait_gathered");
  if (rc != MSQ_OK) return rc;
  return run_wait_gathered(static_cast<cudaStream_t>(stream), wait);
}

int msq_add_rmsnorm(void* cu_ctx, void* stream, float* x, const float* delta, const float* gamma, float* y,
                    int64_t rows, int64_t n, float eps) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!x || !gamma || !y) return fail(MSQ_E_INVALID, "msq_add_rmsnorm: NULL pointer");
  if (rows < 1 || n < 1 || rows > 0x7fffffff || n > 0x7fffffff)
    return fail(MSQ_E_INVALID, "msq_add_rmsnorm: bad shape [%lld, %lld]", (long long)rows, (long long)n);
  return run_add_rmsnorm(static_cast<cudaStream_t>(stream), x, delta, gamma, y, rows, n, eps);
}

int msq_rope_append(void* cu_ctx, void* stream, float* qkv, int heads, int kv_heads, int d, const float* cos_t,
                    const float* sin_t, const int64_t* d_pos, float* kcache, float* vcache, int64_t max_seq) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!qkv || !cos_t || !sin_t || !d_pos || !kcache || !vcache) return fail(MSQ_E_INVALID, "msq_rope_append: NULL pointer");
  if (heads < 1 || kv_heads < 1 || heads % kv_heads || d < 2 || (d & 1) || max_seq < 1 ||
      ((int64_t)heads + 2 * (int64_t)kv_heads) * d > 0x7fffffff)
    return fail(MSQ_E_INVALID, "msq_rope_append: heads %d, kv_heads %d, d %d, max_seq %lld", heads, kv_heads, d,
                (long long)max_seq);
  return run_rope_append(static_cast<cudaStream_t>(stream), qkv, heads, kv_heads, d, cos_t, sin_t, d_pos, kcache,
                         vcache, max_seq);
}

namespace {
int check_gqa(const char* fn, int heads, int kv_heads, int d, int64_t max_seq, const void* q, const void* kc,
              const void* vc) {
  if (heads < 1 || kv_heads < 1 || heads % kv_heads || d < 1 || max_seq < 1 || max_seq > 0x7fffffff)
    return fail(MSQ_E_INVALID, "%s: heads %d, kv_heads %d, d %d, max_seq %lld", fn, heads, kv_heads, d,
                (long long)max_seq);
  if (heads / kv_heads > 8 || d > 256 || (d & 3) || ((uintptr_t)q | (uintptr_t)kc | (uintptr_t)vc) & 15)
    return fail(MSQ_E_UNSUPPORTED,
                "%s: needs heads / kv_heads <= 8, d <= 256 and a multiple of 4, 16-byte aligned q and caches "
                "(heads %d, kv_heads %d, d %d)", fn, heads, kv_heads, d);
  if (gqa_decode_smem(heads, kv_heads, d) > 200 * 1024)
    return fail(MSQ_E_UNSUPPORTED, "%s: d %d with %d query heads per kv head exceeds the shared-memory plan", fn, d,
                heads / kv_heads);
  return MSQ_OK;
}
}  // namespace

int msq_gqa_decode(void* cu_ctx, void* stream, const float* q, const float* kcache, const float* vcache,
                   const int64_t* d_pos, float* out, int heads, int kv_heads, int d, int64_t max_seq) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!q || !kcache || !vcache || !d_pos || !out) return fail(MSQ_E_INVALID, "msq_gqa_decode: NULL pointer");
  const int rc = check_gqa("msq_gqa_decode", heads, kv_heads, d, max_seq, q, kcache, vcache);
  if (rc != MSQ_OK) return rc;
  return run_gqa_decode(static_cast<cudaStream_t>(stream), q, kcache, vcache, d_pos, out, heads, kv_heads, d, max_seq);
}

int msq_rope_gqa_decode(void* cu_ctx, void* stream, const float* qkv, int heads, int kv_heads, int d,
                        const float* cos_t, const float* sin_t, const int64_t* d_pos, float* kcache, float* vcache,
                        float* out, int64_t max_seq) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!qkv || !cos_t || !sin_t || !d_pos || !kcache || !vcache || !out)
    return fail(MSQ_E_INVALID, "msq_rope_gqa_decode: NULL pointer");
  int rc = check_gqa("msq_rope_gqa_decode", heads, kv_heads, d, max_seq, qkv, kcache, vcache);
  if (rc != MSQ_OK) return rc;
  if (d < 8 || (d & (d - 1)) || ((uintptr_t)cos_t | (uintptr_t)sin_t) & 15)
    return fail(MSQ_E_UNSUPPORTED, "msq_rope_gqa_decode: needs d a power of two >= 8 and 16-byte aligned tables (d %d)",
                d);
  return run_rope_gqa_decode(static_cast<cudaStream_t>(stream), qkv, kcache, vcache, cos_t, sin_t, d_pos, out, heads,
                             kv_heads, d, max_seq);
}

int msq_swiglu(void* cu_ctx, void* stream, const float* gate_up, float* out, int64_t n) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!gate_up || !out || n < 1) return fail(MSQ_E_INVALID, "msq_swiglu: NULL pointer or empty");
  return run_swiglu(static_cast<cudaStream_t>(stream), gate_up, out, n);
}

int msq_swiglu_rows(void* cu_ctx, void* stream, const float* gate_up, float* out, int64_t rows, int64_t n) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!gate_up || !out || rows < 1 || n < 1) return fail(MSQ_E_INVALID, "msq_swiglu_rows: NULL pointer or empty");
  return run_swiglu_rows(static_cast<cudaStream_t>(stream), gate_up, out, rows, n);
}

int msq_rope_append_rows(void* cu_ctx, void* stream, const float* qkv, int64_t S, int64_t pos0, int heads,
                         int kv_heads, int d, const float* cos_t, const float* sin_t, float* q_out, float* kcache,
                         float* vcache, int64_t max_seq) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!qkv || !cos_t || !sin_t || !q_out || !kcache || !vcache)
    return fail(MSQ_E_INVALID, "msq_rope_append_rows: NULL pointer");
  if (heads < 1 || kv_heads < 1 || heads % kv_heads || d < 2 || (d & 1) || max_seq < 1 ||
      ((int64_t)heads + 2 * (int64_t)kv_heads) * d > 0x7fffffff)
    return fail(MSQ_E_INVALID, "msq_rope_append_rows: heads %d, kv_heads %d, d %d, max_seq %lld", heads, kv_heads, d,
                (long long)max_seq);
  if (S < 1 || pos0 < 0 || pos0 + S > max_seq)
    return fail(MSQ_E_INVALID, "msq_rope_append_rows: %lld tokens from position %lld do not fit a cache of %lld",
                (long long)S, (long long)pos0, (long long)max_seq);
  return run_rope_append_rows(static_cast<cudaStream_t>(stream), qkv, S, pos0, heads, kv_heads, d, cos_t, sin_t, q_out,
                              kcache, vcache, max_seq);
}

int msq_gqa_prefill(void* cu_ctx, void* stream, const float* q, const float* kcache, const float* vcache, int64_t S,
                    int64_t pos0, float* out, int heads, int kv_heads, int d, int64_t max_seq) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!q || !kcache || !vcache || !out) return fail(MSQ_E_INVALID, "msq_gqa_prefill: NULL pointer");
  if (heads < 1 || kv_heads < 1 || heads % kv_heads || d < 1 || max_seq < 1)
    return fail(MSQ_E_INVALID, "msq_gqa_prefill: heads %d, kv_heads %d, d %d, max_seq %lld", heads, kv_heads, d,
                (long long)max_seq);
  if (S < 1 || pos0 < 0 || pos0 + S > max_seq)
    return fail(MSQ_E_INVALID, "msq_gqa_prefill: %lld tokens from position %lld do not fit a cache of %lld",
                (long long)S, (long long)pos0, (long long)max_seq);
  if (heads / kv_heads > 8 || (d != 64 && d != 128) ||
      ((uintptr_t)q | (uintptr_t)kcache | (uintptr_t)vcache | (uintptr_t)out) & 15)
    return fail(MSQ_E_UNSUPPORTED,
                "msq_gqa_prefill: needs heads / kv_heads <= 8, d 64 or 128, and 16-byte aligned q, out and caches "
                "(heads %d, kv_heads %d, d %d)",
                heads, kv_heads, d);
  return run_gqa_prefill(static_cast<cudaStream_t>(stream), q, kcache, vcache, out, S, pos0, heads, kv_heads, d,
                         max_seq);
}

int msq_argmax(void* cu_ctx, void* stream, const float* x, int64_t n, int64_t* d_idx, int64_t* d_pos) {
  CtxGuard g(cu_ctx);
  if (g.rc != MSQ_OK) return g.rc;
  if (!x || !d_idx || n < 1) return fail(MSQ_E_INVALID, "msq_argmax: NULL pointer or empty");
  return run_argmax(static_cast<cudaStream_t>(stream), x, n, d_idx, d_pos);
}

int msq_qgemm_nbits(const float* a, const uint8_t* bq, const float* scales, const uint8_t* zero_points, float* y,
                    int M, int N, int K, int bits, int block_size) {
  if (N <= 0 || K <= 0 || block_size <= 0 || (bits != 4 && bits != 8) || M < 0)
    return check_weights(N, K, bits, block_size, 0, 0, MSQ_DT_F32, MSQ_DT_ABSENT, 0) != MSQ_OK
               ? MSQ_E_INVALID
               : fail(MSQ_E_INVALID, "msq_qgemm_nbits: negative M");
  const int64_t nb = ((int64_t)K + block_size - 1) / block_size;
  const int64_t blob = ((int64_t)block_size * bits + 7) / 8;
  const int64_t zp_row = (nb * bits + 7) / 8;
  msq_weights_t w = nullptr;
  int rc = msq_pack_host(nullptr, nullptr, bq, (int64_t)N * nb * blob, scales, MSQ_DT_F32, (int64_t)N * nb,
                         zero_points, zero_points ? MSQ_DT_U8 : MSQ_DT_ABSENT, zero_points ? (int64_t)N * zp_row : 0,
                         N, K, bits, block_size, 0, N, MSQ_PACK_DEFAULT, &w);
  if (rc != MSQ_OK) return rc;
  rc = msq_matmul_host(nullptr, nullptr, w, a, MSQ_DT_F32, M, y);
  msq_free(w);
  return rc;
}

}  // extern "C"
