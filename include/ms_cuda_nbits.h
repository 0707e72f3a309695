/*
 * ms_cuda_nbits.h -- C ABI of the B200 (sm_100a) MatMulNBits backend, libms_cuda_nbits.so.
 *
 * Operator: com.microsoft.MatMulNBits, Y[M,N] = A[M,K] . dequant(B)^T with
 *   W[n,k] = (q[n,k] - zp[n, k/bs]) * scale[n, k/bs]
 * in the layouts of ModelSharp's reference kernel
 * (src/ModelSharp/Cpu/Kernels/Quantize/MatMulNBitsKernel.cs:21-42):
 *   B       uint8 [N, ceil(K/bs), ceil(bs*bits/8)], low nibble = even k
 *   scales  [N * ceil(K/bs)], float32 / float16 / bfloat16 (widened exactly)
 *   zp      absent (2^(bits-1)), uint8 packed n-bit with row stride
 *           ceil(ceil(K/bs)*bits/8), or float32 [N * ceil(K/bs)]
 *
 * Conventions follow native/ms_kernels.h:10-13 (row-major, caller-owned pointers,
 * outputs fully overwritten) and the context-aware CUDA entry of
 * native/src/cublas_gemm.cu:624-681 (an int status; an optional CUcontext that is
 * pushed for the call; an optional CUstream; enqueue-only device entries).
 * Every entry returns MSQ_OK (0) or a negative MSQ_E_* code and never aborts the
 * process; msq_last_error() then holds the message, worded as the reference's
 * ModelSharpException for validation failures (MatMulNBitsKernel.cs:87-161).
 *
 * Pointers named d_* are device pointers of the current (or given) context; others
 * are host pointers. cu_ctx may be NULL (use the calling thread's current context,
 * or the primary context of the current device); stream may be NULL (legacy default).
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------------- */
#define MSQ_OK              0
#define MSQ_E_INVALID      -1  /* shape / attribute / argument validation failed     */
#define MSQ_E_UNSUPPORTED  -2  /* valid for the op but not implemented (g_idx perm)   */
#define MSQ_E_CUDA         -3  /* CUDA runtime or driver error                        */
#define MSQ_E_NO_DEVICE    -4  /* no compute-capability 10.x device visible           */
#define MSQ_E_OOM          -5  /* device allocation failed                            */
#define MSQ_E_TIMEOUT      -6  /* a kernel's bounded wait gave up (see msq_device_status) */

/* ---- element types (ModelSharp ElementType, src/ModelSharp/Tensors/ElementType.cs:4-15) */
#define MSQ_DT_ABSENT  -1
#define MSQ_DT_F32      1
#define MSQ_DT_F64      2
#define MSQ_DT_F16      3
#define MSQ_DT_I32      4
#define MSQ_DT_I64      5
#define MSQ_DT_I8       6
#define MSQ_DT_U8       7
#define MSQ_DT_BOOL     8
#define MSQ_DT_BF16    16  /* not an ElementType: the loader widens bf16 (OnnxModelLoader.cs:410) */

/* ---- kernel path selection (msq_matmul_ex) -------------------------------------- */
/* MSQ_PATH_AUTO: bits=4 with a power-of-two block_size >= 32 takes M <= 4 -> decode GEMV;
 * 5 <= M <= 32 at block_size 128 -> MSQ_PATH_GEMV_TC; other M <= 16 -> decode GEMV; M >= 17 ->
 * tcgen05 GEMM. bits=8 (block_size 32 / 64 / 128) -> decode GEMV. Everything else -> generic. */
#define MSQ_PATH_AUTO     0
#define MSQ_PATH_GENERIC  1  /* any bits / block size / zero-point form, reference layout  */
#define MSQ_PATH_GEMV     2  /* bits=4, block_size a power of two >= 32                   */
#define MSQ_PATH_GEMM     3  /* bits=4, block_size a power of two >= 32, tcgen05 + TMEM   */
/* The tcgen05 GEMM with split operands: weights (q - zp) * s computed in fp32 from the fp32
 * scales and A (row-scaled) each enter as two fp16 parts, hi = fp16(x) and lo = fp16(x - hi),
 * three MMAs per k-step (hi.hi + hi.lo + lo.hi) into the fp32 accumulator: products good to
 * about 2^-22 instead of fp16's 2^-11, for prompts whose greedy decoding must follow the fp32
 * reference; about a third of MSQ_PATH_GEMM's throughput.                                */
#define MSQ_PATH_GEMM_SPLIT 4
#define MSQ_PATH_AUTO_SPLIT 5  /* as MSQ_PATH_AUTO, with MSQ_PATH_GEMM_SPLIT for M >= 17       */
/* The batched decode GEMV on tcgen05 kind::i8 (bits=4, block_size 128, 1..32 rows of A): the
 * decode GEMV's exact integer arithmetic with every weight read once for all rows; the same
 * parity bar as MSQ_PATH_GEMV (rel-L2 <= 1e-5).                                          */
#define MSQ_PATH_GEMV_TC  6

/* ---- msq_pack flags ----------------------------------------------------------------- */
#define MSQ_PACK_DEFAULT       0
/* Pack only the decode GEMV's stream records (about 1.0x the reference's bytes on the device
 * instead of about 2x): the GEMM's layout is derived from them on the device, with an
 * allocation, by the first call that takes a GEMM path (make it before any stream capture);
 * msq_matmul_noalloc refuses the handle until then. For weights that decode only.          */
#define MSQ_PACK_GENERIC_ONLY  1  /* keep only the reference layout (exercise the generic kernel) */
#define MSQ_PACK_LAZY_GEMM     2

/* ---- capability / info (ms_kernels.h:23-25, NativeCuda.cs:204-206) ------------------ */
const char* msq_build_info(void);      /* nvcc version, target arch, build date            */
int         msq_available(void);       /* 1 if a CC 10.x device is visible and usable      */
const char* msq_last_error(void);      /* message of this thread's last failing call       */
int64_t     msq_launch_count(void);    /* kernels launched by this library (process-wide)  */
const char* msq_last_path(void);       /* kernel path of this thread's last matmul         */

/* ---- validation only: no device work (MatMulNBitsKernel.cs:82-164) ------------------
 * Checks the attributes N, K, bits, block_size, the element counts of B / scales /
 * zero_points, the zero-point dtype, an optional g_idx (identity only), and A's shape
 * (a_dims[a_rank], last dim == K). On success writes M = product of A's leading dims.
 * zp_dtype is MSQ_DT_ABSENT when the input is missing.                                 */
int msq_check_node(int N, int K, int bits, int block_size,
                   int64_t b_len, int64_t scales_len,
                   int zp_dtype, int64_t zp_len,
                   const int64_t* g_idx, int64_t g_idx_len,
                   const int64_t* a_dims, int a_rank,
                   int64_t* M_out);

/* ---- device-resident weights (IlgpuEngine.cs:2218-2229 residency, repacked) ----------
 * Repacks the reference-layout B / scales / zero_points (device pointers) into the
 * kernel layout, keeping rows [n_begin, n_end) of the N weight rows (0, N for all; a
 * sub-range is the column shard of an N-split). The source buffers may be freed after
 * the stream has passed this call.                                                      */
typedef struct msq_weights_s* msq_weights_t;

int msq_pack(void* cu_ctx, void* stream,
             const uint8_t* d_b, int64_t b_len,
             const void* d_scales, int scales_dtype, int64_t scales_len,
             const void* d_zp, int zp_dtype, int64_t zp_len,
             int N, int K, int bits, int block_size,
             int n_begin, int n_end, int flags,
             msq_weights_t* out);

/* Same from host memory: uploads, repacks and synchronizes the stream. */
int msq_pack_host(void* cu_ctx, void* stream,
                  const uint8_t* b, int64_t b_len,
                  const void* scales, int scales_dtype, int64_t scales_len,
                  const void* zp, int zp_dtype, int64_t zp_len,
                  int N, int K, int bits, int block_size,
                  int n_begin, int n_end, int flags,
                  msq_weights_t* out);

/* Rows, K, bits, block size and device bytes held by a handle (any pointer may be NULL). */
int msq_weights_query(msq_weights_t w, int* n_rows, int* K, int* bits, int* block_size,
                      int64_t* device_bytes);

/* Frees the handle's device memory (after the work queued on it has completed). */
int msq_free(msq_weights_t w);

/* ---- compute (GpuKernels.cs:578-626 launched at IlgpuEngine.cs:2231) -----------------
 * Y[m, j] = sum_k A[m, k] * W[n_begin + j, k] for m < M, j < n_rows; Y row stride ldy
 * (>= n_rows, in floats) so a column shard can write straight into a wider Y. A is
 * row-major [M, K], float32 / float16 / bfloat16. Enqueued on `stream`; the caller
 * synchronizes.                                                                         */
int msq_matmul(void* cu_ctx, void* stream, msq_weights_t w,
               const void* d_a, int a_dtype, int64_t M,
               float* d_y, int64_t ldy);

/* msq_matmul with an explicit kernel path (MSQ_PATH_*). */
int msq_matmul_ex(void* cu_ctx, void* stream, msq_weights_t w,
                  const void* d_a, int a_dtype, int64_t M,
                  float* d_y, int64_t ldy, int path);

/* The int8-activation form of the decode GEMV: the GPU counterpart of ms_qgemm_w4a8
 * (native/ms_kernels.h, native/src/qgemm_w4a8.cpp:247-292), with its arithmetic: per (A row,
 * K-block) s_a = max|a| / 127 and aq = rint(a / s_a) clamped to [-127, 127], the block's exact
 * integer dot of aq with (q - zp), and y += (s_a * s_w) * dot over the blocks. APPROXIMATE
 * against the fp32 op (activation quantization, about 0.5 % rel-L2), like the reference's;
 * it matches ms_qgemm_w4a8 up to fp32 summation order. Up to 8 A rows share one pass over
 * the weights (one s8 column per row). bits=4, block_size 32 / 64 / 128, packed or absent
 * zero points; A finite.                                                                 */
int msq_matmul_w4a8(void* cu_ctx, void* stream, msq_weights_t w,
                    const void* d_a, int a_dtype, int64_t M,
                    float* d_y, int64_t ldy);

/* Host-buffer form (NativeQuant.TryMatMulNBits, NativeQuant.cs:78-115): copies A in,
 * runs, copies Y [M, n_rows] out and synchronizes the stream.                          */
int msq_matmul_host(void* cu_ctx, void* stream, msq_weights_t w,
                    const void* a, int a_dtype, int64_t M, float* y);

/* The same without the final synchronize: the upload, the op and the download of Y are
 * enqueued on `stream` and the call returns. A and Y must stay valid until the stream has
 * passed the download (pinned host memory keeps the copies asynchronous); the caller
 * synchronizes the stream, or an event recorded after the call, before reading Y. No
 * counterpart in the reference, whose host-buffer entry (NativeQuant.cs:78-115) is
 * synchronous: a host loop over several ops pays one round trip per batch of ops. */
int msq_matmul_host_async(void* cu_ctx, void* stream, msq_weights_t w,
                          const void* a, int a_dtype, int64_t M, float* y);

/* ---- no-allocation GEMM -------------------------------------------------------------
 * No counterpart in the reference. For callers that cannot allocate device memory while a
 * node runs (an engine that owns all device memory through its own arena, a plugin called
 * inside someone else's stream capture, a process under a hard memory cap): the tcgen05
 * GEMM path of msq_matmul_ex(..., MSQ_PATH_GEMM) with the same arguments and results, but
 * float32 / bfloat16 (or unaligned float16) A is staged as fp16 in a fixed device array of
 * MSQ_NOALLOC_SCRATCH_BYTES that the library holds on every GPU that loads it, until exit,
 * instead of in memory taken from a pool. Calls no cudaMalloc / cudaFree or other allocator.
 * Limit: round_up(M x round_up(K, 8) x 2, 256) + 4 M <= MSQ_NOALLOC_SCRATCH_BYTES (fp16 rows
 * plus one fp32 row scale per row; e.g. M <= 2047 at K = 4096),
 * else MSQ_E_INVALID; 16-byte-aligned float16 A with K % 8 == 0 needs no staging and has no
 * limit. The first staging call in a CUDA context looks up the array's address in that
 * context (set-up; keyed by cuCtxGetId, so a context created after a reset or destroy gets its
 * own lookup); make it before any stream capture. All calls share the array: calls that
 * overlap on the GPU race.                                                              */
#define MSQ_NOALLOC_SCRATCH_BYTES (16u << 20)
int msq_matmul_noalloc(void* cu_ctx, void* stream, msq_weights_t w,
                       const void* d_a, int a_dtype, int64_t M,
                       float* d_y, int64_t ldy);

/* Sets how long a device-side wait of this library's kernels (a pipeline stage to arrive or
 * to free up, tensor-core completion, copies in flight, other ranks' shards of a gathered
 * input) may last before the kernel gives up, leaves and reports MSQ_E_TIMEOUT through
 * msq_device_status; ns <= 0 restores the default of 2 s. Applies to the current device's
 * context, for launches made after the call. No counterpart in the reference (its kernels
 * have no device-side waits).                                                            */
int msq_set_wait_budget(void* cu_ctx, int64_t ns);

/* Diagnostic counters of this process (the role of NativeCuda.cs:147-150's call counter),
 * -1 for an unknown `which`:
 *   MSQ_DIAG_POOL_ALLOCS      stream-ordered allocations the library has taken from its
 *                             private scratch pool (fp32/bf16 GEMM staging, k-split partials,
 *                             host-buffer calls);
 *   MSQ_DIAG_NOALLOC_LOOKUPS  set-up lookups of the no-allocation array's device address
 *                             (one per CUDA context that has called msq_matmul_noalloc with
 *                             staging);
 *   MSQ_DIAG_POOL_RESERVED    bytes the current device's scratch pool holds (0 before its first
 *                             allocation).                                                    */
#define MSQ_DIAG_POOL_ALLOCS 1
#define MSQ_DIAG_NOALLOC_LOOKUPS 2
#define MSQ_DIAG_POOL_RESERVED 3
int64_t msq_diag_counter(int which);

/* Synchronizes `stream` and reports whether any kernel of this library on the current
 * device gave up a bounded wait (a pipeline stage that never arrived) since the last call:
 * MSQ_OK, or MSQ_E_TIMEOUT with the kernel and stage in msq_last_error(). Clears the flags.
 * No counterpart in the reference (its kernels have no device-side waits).              */
int msq_device_status(void* cu_ctx, void* stream);

/* ---- column split across GPUs with a fused gather ------------------------------------
 * The multi-GPU form of the op (rows of B split over ranks, one process per GPU). No
 * counterpart in the reference, which runs on one device: it replaces the all-gather of
 * Y that would follow each shard's msq_matmul. The decode GEMV of a shard stores its
 * outputs straight into every rank's full-Y buffer (peer stores over NVLink), then its last
 * CTA adds 1 to every rank's arrival counter; a later launch that reads a gathered Y waits
 * (bounded, 2 s, then MSQ_E_TIMEOUT through msq_device_status) until its rank's counter has
 * all ranks' arrivals for that output. Counters live in device memory, so repeated CUDA-graph
 * replays stay in step. Buffers are shared between processes with CUDA IPC.            */
#define MSQ_MAX_RANKS 8
#define MSQ_IPC_HANDLE_BYTES 64

/* One layer's output exchange, seen from one rank (all pointers device pointers mapped in
 * this process). Two of these, with two sets of full-Y buffers, alternate between calls:
 * each rank reads a gathered output before its next-but-one call of the same layer, and
 * every rank's calls wait for all ranks' previous outputs, so no rank overwrites a buffer
 * another rank may still be reading.                                                     */
typedef struct msq_gather {
  int nranks;                                   /* ranks of the split (<= MSQ_MAX_RANKS) */
  int rank;                                     /* this rank                             */
  float* y[MSQ_MAX_RANKS];                      /* every rank's full-Y buffer            */
  unsigned long long* arrivals[MSQ_MAX_RANKS];  /* every rank's arrival counter          */
  int64_t ldy;                                  /* row stride of the full-Y buffers      */
  int64_t col0;                                 /* first column of this rank's shard     */
  unsigned long long* produced;                 /* this rank's count of outputs produced */
  unsigned int* done;                           /* this rank's CTA completion counter    */
} msq_gather_t;

/* A gathered input: complete on this rank once arrivals >= produced * nranks (the producing
 * launch on this rank precedes the reader in stream order, so `produced` counts it).     */
typedef struct msq_wait {
  const unsigned long long* arrivals;           /* this rank's arrival counter           */
  const unsigned long long* produced;           /* this rank's produced counter          */
  int nranks;
} msq_wait_t;

/* Zeroed device memory for exchange buffers and counters (cudaMalloc'd, so it can be
 * shared with CUDA IPC); freed with msq_xbuf_free.                                      */
int msq_xbuf_alloc(void* cu_ctx, int64_t bytes, void** d_ptr);
int msq_xbuf_free(void* cu_ctx, void* d_ptr);

/* CUDA IPC: the handle (MSQ_IPC_HANDLE_BYTES) of an msq_xbuf_alloc buffer, and mapping a
 * peer's handle into this process (peer access enabled lazily); close unmaps.            */
int msq_ipc_handle(void* cu_ctx, void* d_ptr, void* handle);
int msq_ipc_open(void* cu_ctx, const void* handle, void** d_ptr);
int msq_ipc_close(void* cu_ctx, void* d_ptr);

/* msq_matmul on this rank's shard (decode GEMV, 1 <= M <= 4) whose output goes to columns
 * [col0, col0 + n_rows) of rows 0..M-1 of every rank's full-Y buffer. `wait` (or NULL) names
 * a gathered input: A is read only once all ranks' shards of it have arrived. Every rank
 * makes the same calls in the same order.                                               */
int msq_matmul_gather(void* cu_ctx, void* stream, msq_weights_t w,
                      const void* d_a, int a_dtype, int64_t M,
                      const msq_wait_t* wait, const msq_gather_t* gather);

/* Waits on `stream` (one small kernel, bounded like the GEMV's wait) until the latest
 * gathered output is complete on this rank: for readers outside this library, such as a
 * copy to the host.                                                                      */
int msq_wait_gathered(void* cu_ctx, void* stream, const msq_wait_t* wait);

/* ---- decoder glue for one decode token (fp32, device pointers, enqueue-only) ----------
 * The kernels a Llama-shaped decode step needs between its MatMulNBits projections, so that
 * a step is a short chain of launches that a CUDA graph can replay (positions are read from
 * device memory). Not part of the reference's C ABI: each restates one of the reference's CPU
 * graph kernels (cited per entry).                                                      */

/* The decode GEMV (M <= 16) with the glue on either side folded in: no counterpart in the
 * reference (whose graph runs these as separate nodes: SimplifiedLayerNormalization before
 * MatMulNBits, Sigmoid/Mul before the down projection, Add after). With
 *   rms_gamma != NULL  A rows are RMSNorm inputs x; the GEMV computes
 *                      (x / sqrt(mean(x^2) + rms_eps) * gamma) . W^T
 *                      (SimplifiedLayerNormalizationKernel.cs:48-54 then MatMulNBits);
 *   swiglu != 0        A rows are [gate | up] of 2K floats; the GEMV computes
 *                      (gate / (1 + exp(-gate)) * up) . W^T;
 *   accumulate != 0    Y += result (a residual add) instead of Y = result.
 * rms_gamma and swiglu are exclusive. fp32 A only; MSQ_E_UNSUPPORTED unless the weights take
 * the decode GEMV (bits 4, block_size 32 / 64 / 128), K % 4 == 0 and A and gamma are 16-byte
 * aligned. Agreement with the unfused chain is to fp32 rounding (the norm's scale is applied
 * to the dot product rather than to each element).                                       */
typedef struct msq_fusion {
  const float* rms_gamma;
  float rms_eps;
  int32_t swiglu;
  int32_t accumulate;
} msq_fusion_t;

int msq_matmul_fused(void* cu_ctx, void* stream, msq_weights_t w, const float* d_a, int64_t M,
                     float* d_y, int64_t ldy, const msq_fusion_t* fusion);

/* x[r] <- x[r] + delta[r] (delta may be NULL); y[r] <- x[r] / sqrt(mean(x[r]^2) + eps) * gamma,
 * for rows r < rows of n floats (SkipSimplifiedLayerNormalizationKernel.cs:64-67,
 * SimplifiedLayerNormalizationKernel.cs:48-54).                                         */
int msq_add_rmsnorm(void* cu_ctx, void* stream, float* x, const float* delta, const float* gamma,
                    float* y, int64_t rows, int64_t n, float eps);

/* One token's qkv = [q (heads*d) | k (kv_heads*d) | v (kv_heads*d)]: half-split rotary of q and
 * k in place with cos/sin [max_seq][d/2] at position *d_pos, then k and v written to row
 * *d_pos of the caches [kv_heads][max_seq][d] (RotaryEmbeddingKernel.cs:96-114).        */
int msq_rope_append(void* cu_ctx, void* stream, float* qkv, int heads, int kv_heads, int d,
                    const float* cos_t, const float* sin_t, const int64_t* d_pos,
                    float* kcache, float* vcache, int64_t max_seq);

/* out[h] = softmax(q[h] . K[g]^T / sqrt(d)) . V[g] over cache rows 0..*d_pos, g = h / (heads /
 * kv_heads) (GroupQueryAttentionKernel.cs:194-195, 275-312). A position past the cache reads
 * all max_seq rows. MSQ_E_UNSUPPORTED unless heads / kv_heads <= 8, d <= 256 with d % 4 == 0,
 * and q and the caches are 16-byte aligned.                                               */
int msq_gqa_decode(void* cu_ctx, void* stream, const float* q, const float* kcache,
                   const float* vcache, const int64_t* d_pos, float* out, int heads, int kv_heads,
                   int d, int64_t max_seq);

/* msq_rope_append followed by msq_gqa_decode in one launch: qkv = [q | k | v] of the token
 * at position *d_pos, unrotated (and left unchanged); q and k are rotated, k and v written to
 * cache row *d_pos, out = attention of the rotated q over rows 0..*d_pos. A position outside
 * the cache writes nothing and attends with q unrotated over the rows 0..max_seq-1 (as the two
 * separate entries do). Also needs d a power of two >= 8 and 16-byte aligned tables.        */
int msq_rope_gqa_decode(void* cu_ctx, void* stream, const float* qkv, int heads, int kv_heads,
                        int d, const float* cos_t, const float* sin_t, const int64_t* d_pos,
                        float* kcache, float* vcache, float* out, int64_t max_seq);

/* gate_up = [gate (n) | up (n)]: out = gate / (1 + exp(-gate)) * up.                     */
int msq_swiglu(void* cu_ctx, void* stream, const float* gate_up, float* out, int64_t n);

/* ---- prompt forms of the glue: S tokens at positions pos0 .. pos0 + S - 1 at once --------
 * msq_rope_append_rows: qkv [S][(heads + 2 kv_heads) d], unrotated and left unchanged; the
 * half-split rotary of every token's q heads goes to q_out [S][heads d], of its k heads to cache
 * rows pos0 + s, and its v heads to the same rows of the value cache (RotaryEmbeddingKernel.cs:
 * 96-114 per token). pos0 + S <= max_seq.                                                      */
int msq_rope_append_rows(void* cu_ctx, void* stream, const float* qkv, int64_t S, int64_t pos0,
                         int heads, int kv_heads, int d, const float* cos_t, const float* sin_t,
                         float* q_out, float* kcache, float* vcache, int64_t max_seq);

/* Causal attention of a prompt: q [S][heads d] (rotated), keys and values of positions
 * 0 .. pos0 + S - 1 already in the caches [kv_heads][max_seq][d]; out [S][heads d] with
 * out[s][h] = softmax over cache rows 0 .. pos0 + s of q[s][h] . k / sqrt(d), times v, head h
 * reading kv head h / (heads / kv_heads) (GroupQueryAttentionKernel.cs:194-195, 275-312 for
 * every query token), fp32 throughout. MSQ_E_UNSUPPORTED unless heads / kv_heads <= 8, d is 64
 * or 128, and q, out and the caches are 16-byte aligned.                                      */
int msq_gqa_prefill(void* cu_ctx, void* stream, const float* q, const float* kcache,
                    const float* vcache, int64_t S, int64_t pos0, float* out, int heads,
                    int kv_heads, int d, int64_t max_seq);

/* Rows of gate_up [rows][2n] = [gate | up]: out [rows][n] = gate / (1 + exp(-gate)) * up.    */
int msq_swiglu_rows(void* cu_ctx, void* stream, const float* gate_up, float* out, int64_t rows,
                    int64_t n);

/* *d_idx = the first index of the maximum of x[0..n); *d_pos += 1 when d_pos is not NULL.  */
int msq_argmax(void* cu_ctx, void* stream, const float* x, int64_t n, int64_t* d_idx, int64_t* d_pos);

/* ---- one-shot drop-in for ms_qgemm_nbits (native/ms_kernels.h:42-44) -----------------
 * Host pointers, fp32 A / scales, packed or NULL zero points; uploads, runs on the
 * current device and downloads per call. Returns a status where the original is void. */
int msq_qgemm_nbits(const float* a, const uint8_t* bq, const float* scales,
                    const uint8_t* zero_points, float* y,
                    int M, int N, int K, int bits, int block_size);

#ifdef __cplusplus
}
#endif
