// Decode GEMV for MatMulNBits on the tensor cores with exact integer arithmetic
// (bits = 4, block_size 32 / 64 / 128, M <= 4 per pass).
//
// Memory-bound: one producer warp streams the repacked weight stages (16 weight rows x one
// k-tile, 17-35 KB, one cp.async.bulk each) through a small shared-memory ring; the 16
// consumer warps split every stage by 64/128-k units and run mma.m16n8k32 (u8 x s8 -> s32).
//
// Exactness. The reference computes sum_k a[m,k] * ((q - zp) * s) in fp32
// (MatMulNBitsKernel.cs:236-261). Here each quantisation block b of each row of A becomes a
// 24-bit fixed-point integer vector a_int = rint(a * 2^sigma_b) (max|a * 2^sigma_b| < 2^22,
// sigma_b chosen per block from the block's own maximum), split into three balanced int8
// digits a_int = d0 + 256 d1 + 65536 d2 that form B columns. The tensor core returns
// D_i = sum_{k in b} q[n,k] * d_i[k] exactly in s32, and
//     y[m,n] += s[n,b] * 2^-sigma_b * ( D_0 + 256 D_1 + 65536 D_2  -  zp[n,b] * S_b )
// with S_b = sum_{k in b} a_int exact in s32. Only the rounding of a to 2^-24 of its block
// maximum and the fp32 block combination round; parity is checked at rel-L2 <= 1e-5 against
// the fp32 reference. Block-local scales need no row-wide reduction, so the activation
// preparation is one pass of loads and warp shuffles.
//
// Decode: a lane's 32-bit word holds, byte j, the codes of (row r, k 4t+j) (low nibble)
// and (row r+8, k 4t+j) (high nibble), so (x & 0x0F0F0F0F) is directly the u8 A-fragment
// register of rows r, and x itself that of rows r+8 as 16 q' + q: their dot comes out as
// 16 D' + D, and D, row r's own dot, sits in the same lane's accumulator, so the epilogue
// subtracts it once per block (exact in s32). One integer op per 8 weights.
#include "msq_internal.cuh"
#include "msq_ptx.cuh"

#include <algorithm>

namespace msq {
namespace {

constexpr int kConsumers = 16;
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kMaxSlots = 8;
constexpr int kSmemMax = 227 * 1024;
constexpr int kMaxM = 4;  // B columns: 4 per A row (3 digits + 1 zero) -> two n8 tiles for 4 rows
constexpr int kMaxMA8 = 8;  // the int8-activation form: one B column per A row -> 8 rows in one n8 tile
constexpr int kUpw = 2;                 // k-units per warp per tile
constexpr int kYPitch = kConsumers + 1;  // per-warp partial sums of one output, padded against
                                         // bank conflicts in the per-stage update

__device__ int g_mma_err;

struct Args {
  const uint8_t* strm;
  const void* a;
  int a_dtype;
  int64_t m0;
  int mc;  // A rows in this pass (<= 4)
  float* y;
  int64_t ldy;
  int n_rows, K, kt, ntiles, nblk, stage_bytes, off_sc, off_zp, zp_kind;
  int nslots, rows_cta;
  int kp;     // ntiles * kt: K padded to whole tiles
  int kpp;    // row pitch of the digit array: kp + 16 bytes (column c starts 4c banks later)
  int a_vec;  // rows of A may be read 4 elements at a time
  int prefetch;  // weights settled: stream them before the programmatic-dependency wait
  int64_t lda;   // row stride of A in elements (K, or 2K for the SwiGLU form)
  // decode-step fusions (fp32 A, a_vec only): A row = RMSNorm input x, a = x * gamma and the
  // output scaled by 1 / sqrt(mean(x^2) + eps); or A row = [gate | up], a = silu(gate) * up;
  // and Y += result instead of Y = result
  const float* gamma;
  float eps;
  int swiglu;
  int accumulate;
  int off_dig, off_s, off_ysum, off_bar, off_ring;  // shared-memory offsets (bytes)
  // column-split exchange (the XG kernels): outputs to every rank's full-Y buffer
  int nranks;
  float* gy[MSQ_MAX_RANKS];
  unsigned long long* garr[MSQ_MAX_RANKS];
  int64_t gldy, gcol0;
  unsigned long long* gprod;
  unsigned int* gdone;
  const unsigned long long* warr;  // gathered input to wait for (nullptr: none)
  const unsigned long long* wprod;
  int wranks;
};

constexpr int kErrTimeoutPeer = 5;  // waiting for other ranks' shards of a gathered input

// Waits until every rank's shard of the latest gathered output has arrived on this rank:
// arrivals >= produced * nranks (acquire at system scope). Bounded; false on timeout.
__device__ __forceinline__ bool wait_arrivals(const unsigned long long* arr, const unsigned long long* prod,
                                              int nranks) {
  const unsigned long long target =
      *reinterpret_cast<const volatile unsigned long long*>(prod) * (unsigned long long)nranks;
  const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(arr) : "memory");
    if (v >= target) return true;
    if (ptx::globaltimer() - t0 > budget) {
      atomicCAS(&g_mma_err, 0, kErrTimeoutPeer);
      return false;
    }
    __nanosleep(64);
  }
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (*abort_flag) return false;
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait_sleep(bar, parity)) return true;
    if ((i & 7u) == 0) {
      if (*abort_flag) return false;
      if (ptx::globaltimer() - t0 > budget) {
        *abort_flag = 1;
        atomicCAS(&g_mma_err, 0, code);
        return false;
      }
    }
  }
}

// Programmatic dependent launch. launch_dependents lets the next kernel of the stream that
// was launched with programmatic serialization get scheduled as SMs free up; wait blocks
// until every prerequisite grid has completed and its memory is visible (a no-op when the
// launch had no programmatic dependency).
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void imma(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A[m0 + m][k .. k+3] as fp32, zeros past K.
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <bool FU>
__device__ __forceinline__ float4 load4(const Args& p, int m, int k) {
  const int64_t base = (p.m0 + m) * (FU ? p.lda : (int64_t)p.K) + k;
  if (p.a_vec && k + 4 <= p.K) {
    if (p.a_dtype == MSQ_DT_F32) {
      const float* ap = static_cast<const float*>(p.a) + base;
      const float4 v = *reinterpret_cast<const float4*>(ap);
      if (!FU || !p.swiglu) return v;
      const float4 u = *reinterpret_cast<const float4*>(ap + p.K);  // the up half of the row
      return make_float4(silu_mul(v.x, u.x), silu_mul(v.y, u.y), silu_mul(v.z, u.z), silu_mul(v.w, u.w));
    }
    const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.a) + base);
    float2 lo, hi;
    if (p.a_dtype == MSQ_DT_F16) {
      lo = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
      hi = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    } else {
      lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
      hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
    }
    return make_float4(lo.x, lo.y, hi.x, hi.y);
  }
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = k + j < p.K ? load_act(p.a, p.a_dtype, base + j) : 0.f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

// Digits of 4 consecutive k: a = rint(x * 2^sigma) (|a| < 2^22) in balanced base 256,
// a = d0 + 256 d1 + 65536 d2 with d_i in [-128, 127]. u = a + 0x808080 holds d_i + 128 in its
// byte i, and the magic constant 1.5 * 2^23 makes one fma produce u in the low mantissa bits
// (the product is exact, the add rounds to nearest even at integer granularity). The bytes
// are transposed into one word per digit (w0: d0 of the 4 k, ...); returns sum a exactly.
__device__ __forceinline__ uint32_t biased24(float x, float sc) {
  return __float_as_uint(fmaf(x, sc, 12582912.0f)) - (0x4B400000u - 0x808080u);
}
__device__ __forceinline__ int digit_words(float4 v, float sc, uint32_t& w0, uint32_t& w1, uint32_t& w2) {
  const uint32_t u0 = biased24(v.x, sc), u1 = biased24(v.y, sc), u2 = biased24(v.z, sc), u3 = biased24(v.w, sc);
  const uint32_t t01 = __byte_perm(u0, u1, 0x5140), t23 = __byte_perm(u2, u3, 0x5140);  // b0,b0',b1,b1'
  const uint32_t s01 = __byte_perm(u0, u1, 0x0062), s23 = __byte_perm(u2, u3, 0x0062);  // b2,b2'
  w0 = __byte_perm(t01, t23, 0x5410) ^ 0x80808080u;
  w1 = __byte_perm(t01, t23, 0x7632) ^ 0x80808080u;
  w2 = __byte_perm(s01, s23, 0x5410) ^ 0x80808080u;
  return (int)((u0 + u1) + (u2 + u3) - 4u * 0x808080u);
}

// Writes the digit words of 4 consecutive k of row m (columns 4m..4m+2 of the digit array,
// row pitch kpp; the fourth column of each row is never read) and returns their exact sum.
__device__ __forceinline__ int store_digits(int8_t* dig, int kpp, int m, int k, float4 v, float sc) {
  uint32_t w0, w1, w2;
  const int sum = digit_words(v, sc, w0, w1, w2);
  *reinterpret_cast<uint32_t*>(dig + (4 * m + 0) * kpp + k) = w0;
  *reinterpret_cast<uint32_t*>(dig + (4 * m + 1) * kpp + k) = w1;
  *reinterpret_cast<uint32_t*>(dig + (4 * m + 2) * kpp + k) = w2;
  return sum;
}

// Exponent e of frexp(x) for finite x > 0 (x = f * 2^e, f in [0.5, 1)), -126 for subnormals,
// 0 for zero, infinity and NaN; and 2^s for |s| <= 126 from the exponent bits.
__device__ __forceinline__ int frexp_exponent(float x) {
  const int be = (__float_as_int(x) >> 23) & 0xFF;
  if (!(x > 0.f) || be == 0xFF) return 0;
  return be == 0 ? -126 : be - 126;
}
__device__ __forceinline__ float exp2i(int s) { return __int_as_float((s + 127) << 23); }

// W[row, k] = (q - zp) * s in fp32, read back from the stream records in global memory
// (layout in msq_internal.cuh): the slow path of rows of A that hold inf or NaN.
template <int BS, bool B8>
__device__ float stream_weight(const Args& p, int64_t row, int k) {
  const int64_t b = row >> 4;
  const int r = (int)(row & 15);
  const int t = k / p.kt, kk = k - t * p.kt;
  const uint8_t* rec = p.strm + (b * p.ntiles + t) * (int64_t)p.stage_bytes;
  const int o = kk & 63;
  const int ln = (r & 7) * 4 + ((o & 15) >> 2);
  int q;
  if constexpr (B8) {  // word (step, k half, row half) of 8 per lane, one byte per code
    const int word = (o >> 5) * 4 + ((o >> 4) & 1) * 2 + (r >> 3);
    q = rec[(kk >> 6) * 1024 + ln * 32 + word * 4 + (o & 3)];
  } else {
    const int word = (o >> 5) * 2 + ((o >> 4) & 1);
    const uint8_t v = rec[(kk >> 6) * 512 + ln * 16 + word * 4 + (o & 3)];
    q = r < 8 ? (v & 0xF) : (v >> 4);
  }
  const int bl = kk / BS;
  const float sc = reinterpret_cast<const float*>(rec + p.off_sc)[bl * 16 + r];
  float z = B8 ? 128.f : 8.f;
  if (p.zp_kind == ZP_PACKED && B8)
    z = (float)rec[p.off_zp + bl * 16 + r];
  else if (p.zp_kind == ZP_PACKED)
    z = (float)((reinterpret_cast<const unsigned long long*>(rec + p.off_zp)[bl] >> (4 * r)) & 0xF);
  else if (p.zp_kind == ZP_F32)
    z = reinterpret_cast<const float*>(rec + p.off_zp)[bl * 16 + r];
  return ((float)q - z) * sc;
}

// Sum over the k where A row m is inf or NaN of a[m, k] * W[row, k] in fp32: inf, -inf or NaN
// exactly as the reference's fp32 sum gets them (a NaN term, inf * 0 or inf - inf give NaN),
// which is what the row's output then is.
template <int BS, bool FU, bool B8>
__device__ float nonfinite_terms(const Args& p, int m, int64_t row) {
  const int64_t base = (p.m0 + m) * (FU ? p.lda : (int64_t)p.K);
  float t = 0.f;
  for (int k = 0; k < p.K; ++k) {
    float a = load_act(p.a, p.a_dtype, base + k);
    if (FU && p.swiglu) a = silu_mul(a, load_act(p.a, p.a_dtype, base + p.K + k));
    if (!(fabsf(a) <= 3.402823466e38f)) t += a * stream_weight<BS, B8>(p, row, k);
  }
  return t;
}

// BS = quantisation block size (32 / 64 / 128); NT = n8 tiles of B (1: M <= 2, 2: M <= 4);
// XG = the column-split form (outputs to every rank's full-Y buffer, optional wait for a
// gathered input); FU = the decode-step fusion forms (RMSNorm / SwiGLU input, accumulate). A "unit" is max(BS, 64) k: one or two 64-k chunks (a uint4 of code words
// per lane each).
// A8 = the int8-activation form (ms_qgemm_w4a8's arithmetic, native/src/qgemm_w4a8.cpp:247-292,
// 622-690): per (A row, block) s_a = max|a| / 127 and aq = rint(a / s_a) in [-127, 127], one s8
// B column per A row, the block's exact integer dot aq . (q - zp) and y += (s_a s_w) dot.
// B8 = 8-bit weight codes (MatMulNBits bits=8): the record's code words are the u8 A-fragment
// registers themselves (no nibble split, no 16x high-nibble rows), default zero point 128.
template <int BS, int NT, bool XG, bool FU, bool A8 = false, bool B8 = false>
__global__ void __launch_bounds__(kThreads, 1) gemv_mma_kernel(const Args p) {
  static_assert(!(XG && FU), "the column-split form takes no fusion");
  static_assert(!B8 || (!XG && !FU && !A8), "8-bit codes take the plain form");
  static_assert(!A8 || (!XG && !FU && NT == 1), "the int8-activation form is plain, 8 rows per pass");
  constexpr int UNIT = BS > 64 ? BS : 64;
  constexpr int CH = UNIT / 64;     // 64-k chunks per unit
  constexpr int UB = UNIT / BS;     // blocks per unit
  constexpr int STEPS = UNIT / 32;  // k32 mma steps per unit
  constexpr int BSTEPS = BS / 32;   // k32 steps per block
  constexpr int UPW = kUpw;
  extern __shared__ __align__(16) uint8_t smem[];
  int8_t* dig = reinterpret_cast<int8_t*>(smem + p.off_dig);  // [4*mc][kpp] digits
  int* sblk = reinterpret_cast<int*>(smem + p.off_s);         // [mc][kp/BS] exact block sums of a_int
  float* sinv = reinterpret_cast<float*>(sblk + p.mc * (p.kp / BS));  // [mc][kp/BS] 2^-sigma_b
  float* ysum = reinterpret_cast<float*>(smem + p.off_ysum);  // [rows_cta][mc][33]: per warp
  float* rowsq = reinterpret_cast<float*>(smem + 64);         // [kConsumers][kMaxM] sums of x^2
  volatile int* nonfin = reinterpret_cast<volatile int*>(smem);  // [kMaxMA8]: A row holds inf / NaN
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* empty = full + kMaxSlots;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMaxSlots);
  uint8_t* ring = smem + p.off_ring;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grid = gridDim.x;
  const int nb_cta = (p.nblk - (int)blockIdx.x + grid - 1) / grid;  // row blocks of this CTA
  const int T = p.ntiles;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nslots; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], kConsumers);
    }
    *abort_flag = 0;
    for (int m = 0; m < kMaxMA8; ++m) nonfin[m] = 0;
    ptx::fence_mbar_init();
    griddep_launch_dependents();
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ---------------- producer: stages in (tile, row block) order. Settled weights are
    // never written by an earlier kernel, so their stream starts before the dependency wait
    // and overlaps the previous kernel's tail.
    if (lane == 0) {
      if (!p.prefetch) griddep_wait();
      const uint64_t pol = ptx::policy_evict_first();  // each record is read once per launch
      int issued = 0, s = 0;
      uint32_t wrap = 0;
      bool ok = true;
      for (int t = 0; t < T && ok; ++t)
        for (int i = 0; i < nb_cta; ++i) {
          if (issued >= p.nslots && !wait_or_abort(&empty[s], wrap ^ 1u, abort_flag, ptx::kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int b = blockIdx.x + i * grid;
          ptx::mbar_arrive_expect_tx(&full[s], p.stage_bytes);
          ptx::bulk_g2s_hint(ring + (size_t)s * p.stage_bytes,
                             p.strm + ((int64_t)b * T + t) * (int64_t)p.stage_bytes, p.stage_bytes, &full[s], pol);
          ++issued;
          if (++s == p.nslots) {
            s = 0;
            wrap ^= 1u;
          }
        }
      for (int q = 0; q < p.nslots && q < issued; ++q) {  // in-flight copies must land before exit
        const int last = q + (issued - 1 - q) / p.nslots * p.nslots;
        const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
        while (!ptx::mbar_try_wait(&full[q], (last / p.nslots) & 1)) {
          if (ptx::globaltimer() - t0 > budget) {
            atomicCAS(&g_mma_err, 0, ptx::kErrTimeoutDrain);
            break;
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers (512 threads, named barrier 1)
  const int tid = threadIdx.x;
  const int mc = p.mc;
  for (int i = tid; i < p.rows_cta * mc * kYPitch; i += kConsumers * 32) ysum[i] = 0.f;
  griddep_wait();  // A may come from the previous kernel, and Y may still be read by it
  if constexpr (XG) {
    if (p.warr) {  // a gathered input: every rank's shard of it must have arrived
      if (tid == 0 && !wait_arrivals(p.warr, p.wprod, p.wranks)) *abort_flag = 1;
      ptx::named_bar_sync(1, kConsumers * 32);
    }
  }

  // ---- activations: one pass. Loads in flight at once (float4, U deep); per quantisation
  // block (GL consecutive lanes) a shuffle max picks 2^sigma_b, the digits are written and a
  // shuffle sum gives the exact block sum of a_int.
  constexpr int U = 4;
  constexpr int kC = kConsumers * 32;
  constexpr int GL = BS / 4;  // float4 per quantisation block (8 / 16 / 32 lanes)
  const int n4row = p.kp / 4;
  const int n4 = mc * n4row;
  float ssq[kMaxM] = {};  // RMSNorm form: this thread's share of sum x^2 per A row
  for (int base = 0; base < n4; base += kC * U) {
    const int nu = min(U, (n4 - base + kC - 1) / kC);  // warp-uniform
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int f = base + tid + u * kC;
      const int m = f / n4row;
      v[u] = (u < nu && f < n4) ? load4<FU>(p, m, 4 * (f - m * n4row)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (FU && p.gamma) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int f = base + tid + u * kC;
        const int m = f / n4row, k = 4 * (f - m * n4row);
        if (u < nu && f < n4 && k < p.K) {  // K % 4 == 0 here: a float4 is all in or all out
          const float sq = fmaf(v[u].x, v[u].x, fmaf(v[u].y, v[u].y, fmaf(v[u].z, v[u].z, v[u].w * v[u].w)));
#pragma unroll
          for (int j = 0; j < kMaxM; ++j) ssq[j] += m == j ? sq : 0.f;
          const float4 g = *reinterpret_cast<const float4*>(p.gamma + k);
          v[u] = make_float4(v[u].x * g.x, v[u].y * g.y, v[u].z * g.z, v[u].w * g.w);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u < nu) {
        const int f = base + tid + u * kC;
        // |x| as bits orders like the values, with inf and NaN above every finite value
        uint32_t ub = max(max(__float_as_uint(fabsf(v[u].x)), __float_as_uint(fabsf(v[u].y))),
                          max(__float_as_uint(fabsf(v[u].z)), __float_as_uint(fabsf(v[u].w))));
        if (ub >= 0x7F800000u) {
          // inf / NaN: the integer path takes 0 for them and the row's outputs get their exact
          // fp32 terms at the end (nonfinite_terms), so they propagate as in the reference
          if (f < n4) nonfin[f / n4row] = 1;
          v[u].x = fabsf(v[u].x) <= 3.402823466e38f ? v[u].x : 0.f;
          v[u].y = fabsf(v[u].y) <= 3.402823466e38f ? v[u].y : 0.f;
          v[u].z = fabsf(v[u].z) <= 3.402823466e38f ? v[u].z : 0.f;
          v[u].w = fabsf(v[u].w) <= 3.402823466e38f ? v[u].w : 0.f;
          ub = max(max(__float_as_uint(fabsf(v[u].x)), __float_as_uint(fabsf(v[u].y))),
                   max(__float_as_uint(fabsf(v[u].z)), __float_as_uint(fabsf(v[u].w))));
        }
        float bmax = __uint_as_float(ub);
        if constexpr (GL == 32) {  // one block per warp: non-negative floats order as their bits
          bmax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(bmax)));
        } else {
#pragma unroll
          for (int off = 1; off < GL; off <<= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, off));
        }
        int sh = 0;
        float sa = 0.f;  // A8: the block's activation scale
        int bsum = 0;
        if constexpr (A8) {
          // the reference's IEEE steps: s = amax / 127, inv = 1 / s, q = lrintf(a inv) clamped
          sa = bmax / 127.0f;
          const float inv = sa > 0.f ? 1.0f / sa : 0.f;
          if (f < n4) {
            const int m = f / n4row;
            const int q0 = max(-127, min(127, __float2int_rn(v[u].x * inv)));
            const int q1 = max(-127, min(127, __float2int_rn(v[u].y * inv)));
            const int q2 = max(-127, min(127, __float2int_rn(v[u].z * inv)));
            const int q3 = max(-127, min(127, __float2int_rn(v[u].w * inv)));
            *reinterpret_cast<uint32_t*>(dig + m * p.kpp + 4 * (f - m * n4row)) =
                (uint32_t)(q0 & 0xFF) | ((uint32_t)(q1 & 0xFF) << 8) | ((uint32_t)(q2 & 0xFF) << 16) |
                ((uint32_t)(q3 & 0xFF) << 24);
            bsum = q0 + q1 + q2 + q3;
          }
        } else {
          sh = max(-120, min(120, 22 - frexp_exponent(bmax)));
          if (f < n4) {
            const int m = f / n4row;
            bsum = store_digits(dig, p.kpp, m, 4 * (f - m * n4row), v[u], exp2i(sh));
          }
        }
        if constexpr (GL == 32) {
          bsum = (int)__reduce_add_sync(0xffffffffu, (uint32_t)bsum);
        } else {
#pragma unroll
          for (int off = 1; off < GL; off <<= 1) bsum += __shfl_xor_sync(0xffffffffu, bsum, off);
        }
        if (f < n4 && (lane & (GL - 1)) == 0) {
          sblk[f / GL] = bsum;
          sinv[f / GL] = A8 ? sa : exp2i(-sh);
        }
      }
    }
  }
  if (FU && p.gamma) {  // per-warp sums of x^2 per row, in a fixed order
#pragma unroll
    for (int j = 0; j < kMaxM; ++j) {
      float v = ssq[j];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) rowsq[warp * kMaxM + j] = v;
    }
  }
  ptx::named_bar_sync(1, kConsumers * 32);

  // ---- main loop: tile t outer, this CTA's row blocks inner. Warp w takes the units whose
  // index along the whole row is w mod kConsumers: units w0, w0 + 16 of tile t with
  // w0 = (w - t units) mod 16, so every warp gets the same count over the row even when a tile
  // holds fewer than 32 units (K = 14336 at block_size 128: 28 per tile, 7 per warp in all).
  const int grp = lane >> 2, tq = lane & 3;
  const float wdig = (tq & 1) ? 65536.f : 1.f;  // weight of this lane's first digit column
  const int units = p.kt / UNIT;
  const int nbp = p.kp / BS;
  int rs = 0;
  uint32_t rph = 0;
  for (int t = 0; t < T; ++t) {
    const int w0 = ((warp - t * units) % kConsumers + kConsumers) % kConsumers;
    // B fragments of this warp's units (digits of columns grp + 8j), held across row blocks
    uint32_t bf[UPW][STEPS][NT][2];
    float sv[UPW][UB][NT];    // block sums of a_int for this lane's A row(s), 0 on odd lanes
    float sv16[UPW][UB][NT];  // the same x 16, for the high-nibble rows' zero-point term
    float gw0[UPW][UB][NT];   // 2^-sigma of those blocks x this lane's digit weight (1 or 2^16)
    float gw1[UPW][UB][NT];   // the same / 16: undoes the 16 q of the high-nibble rows
#pragma unroll
    for (int uu = 0; uu < UPW; ++uu) {
      const int u = w0 + uu * kConsumers;
      const int kk0 = t * p.kt + u * UNIT;
#pragma unroll
      for (int st = 0; st < STEPS; ++st)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int col = nt * 8 + grp;
          const bool ok = u < units && (A8 ? col < mc : col < 4 * mc && (col & 3) != 3);
          const int8_t* d = dig + col * p.kpp + kk0 + 32 * st + 4 * tq;
          bf[uu][st][nt][0] = ok ? *reinterpret_cast<const uint32_t*>(d) : 0u;
          bf[uu][st][nt][1] = ok ? *reinterpret_cast<const uint32_t*>(d + 16) : 0u;
        }
#pragma unroll
      for (int bl = 0; bl < UB; ++bl)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if constexpr (A8) {
            // this lane's two A rows (B columns 2 tq, 2 tq + 1): block sums S and scales s_a
            const int m0 = 2 * tq, m1 = m0 + 1;
            const int bix = kk0 / BS + bl;
            const bool ok0 = u < units && m0 < mc, ok1 = u < units && m1 < mc;
            sv[uu][bl][nt] = ok0 ? (float)sblk[m0 * nbp + bix] : 0.f;
            sv16[uu][bl][nt] = ok1 ? (float)sblk[m1 * nbp + bix] : 0.f;
            gw0[uu][bl][nt] = ok0 ? sinv[m0 * nbp + bix] : 0.f;
            gw1[uu][bl][nt] = ok1 ? sinv[m1 * nbp + bix] : 0.f;
            continue;
          }
          const int m = nt * 2 + (tq >> 1);
          const bool okb = u < units && m < mc;
          // the zero-point term rides on the lanes of digits 0 and 1 (even tq) only; every
          // factor below is the block scale times a power of two, so the products are exact
          sv[uu][bl][nt] = okb && (tq & 1) == 0 ? (float)sblk[m * nbp + kk0 / BS + bl] : 0.f;
          sv16[uu][bl][nt] = (B8 ? 1.f : 16.f) * sv[uu][bl][nt];
          const float g = okb ? sinv[m * nbp + kk0 / BS + bl] : 0.f;
          gw0[uu][bl][nt] = g * wdig;
          gw1[uu][bl][nt] = B8 ? g * wdig : g * wdig * 0.0625f;
        }
    }

    for (int i = 0; i < nb_cta; ++i) {
      // warp-uniform: the stage's epilogue shuffles need every lane
      const bool ok = __all_sync(0xffffffffu, wait_or_abort(&full[rs], rph, abort_flag, ptx::kErrTimeoutFull));
      if (ok) {
        const uint8_t* base = ring + rs * p.stage_bytes;
        const float* scp = reinterpret_cast<const float*>(base + p.off_sc);
        // Both units of this warp as independent chains, each block's k32 steps split over
        // two accumulators, so the tensor-core latency overlaps; a missing second unit
        // (kt < 32 units) reads unit 0's words and contributes nothing (its gw0 and gw1 are 0).
        uint32_t wv[UPW][(B8 ? 8 : 4) * CH];
        float s0[UPW][UB], s1[UPW][UB], z0[UPW][UB], z1[UPW][UB];
#pragma unroll
        for (int uu = 0; uu < UPW; ++uu) {
          const int u = w0 + uu * kConsumers;
          const int ul = u < units ? u : 0;  // unit 0 always exists in a stage
          if constexpr (B8) {
            const uint4* cw = reinterpret_cast<const uint4*>(base) + ul * CH * 64 + 2 * lane;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
              const uint4 q0 = cw[c * 64], q1 = cw[c * 64 + 1];
              wv[uu][8 * c + 0] = q0.x;
              wv[uu][8 * c + 1] = q0.y;
              wv[uu][8 * c + 2] = q0.z;
              wv[uu][8 * c + 3] = q0.w;
              wv[uu][8 * c + 4] = q1.x;
              wv[uu][8 * c + 5] = q1.y;
              wv[uu][8 * c + 6] = q1.z;
              wv[uu][8 * c + 7] = q1.w;
            }
          } else {
            const uint4* nib = reinterpret_cast<const uint4*>(base) + ul * CH * 32 + lane;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
              const uint4 q4 = nib[c * 32];
              wv[uu][4 * c + 0] = q4.x;
              wv[uu][4 * c + 1] = q4.y;
              wv[uu][4 * c + 2] = q4.z;
              wv[uu][4 * c + 3] = q4.w;
            }
          }
#pragma unroll
          for (int bl = 0; bl < UB; ++bl) {
            const int blk_local = ul * UB + bl;
            s0[uu][bl] = scp[blk_local * 16 + grp];
            s1[uu][bl] = scp[blk_local * 16 + grp + 8];
            // z1 is for the high-nibble rows, whose products come out 16x (sv16 carries the 16)
            if (B8 && p.zp_kind == ZP_PACKED) {
              const uint8_t* zb = base + p.off_zp + blk_local * 16;
              z0[uu][bl] = (float)zb[grp];
              z1[uu][bl] = (float)zb[grp + 8];
            } else if (p.zp_kind == ZP_PACKED) {
              const uint2 zw = reinterpret_cast<const uint2*>(base + p.off_zp)[blk_local];
              z0[uu][bl] = (float)((zw.x >> (4 * grp)) & 0xF);
              z1[uu][bl] = (float)((zw.y >> (4 * grp)) & 0xF);
            } else if (p.zp_kind == ZP_F32) {
              const float* zf = reinterpret_cast<const float*>(base + p.off_zp);
              z0[uu][bl] = zf[blk_local * 16 + grp];
              z1[uu][bl] = zf[blk_local * 16 + grp + 8];
            } else {
              z0[uu][bl] = B8 ? 128.f : 8.f;
              z1[uu][bl] = B8 ? 128.f : 8.f;
            }
          }
        }
        int c[UPW][UB][2][NT][4];
#pragma unroll
        for (int uu = 0; uu < UPW; ++uu)
#pragma unroll
          for (int bl = 0; bl < UB; ++bl)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) c[uu][bl][h][nt][0] = c[uu][bl][h][nt][1] = c[uu][bl][h][nt][2] = c[uu][bl][h][nt][3] = 0;
#pragma unroll
        for (int q = 0; q < BSTEPS; ++q)
#pragma unroll
          for (int bl = 0; bl < UB; ++bl)
#pragma unroll
            for (int uu = 0; uu < UPW; ++uu) {
              const int st = bl * BSTEPS + q;
              uint32_t lo0, hi0, lo1, hi1;
              if constexpr (B8) {  // the record words are the fragment registers
                lo0 = wv[uu][4 * st];
                hi0 = wv[uu][4 * st + 1];
                lo1 = wv[uu][4 * st + 2];
                hi1 = wv[uu][4 * st + 3];
              } else {
                // rows r take the low nibbles; rows r+8 take the whole bytes, 16 q' + q as a
                // u8, whose dot is 16 D' + D with D row r's own dot from the same MMA (the
                // epilogue subtracts it: exact in s32)
                const uint32_t x0 = wv[uu][2 * st], x1 = wv[uu][2 * st + 1];
                lo0 = x0 & 0x0F0F0F0Fu;
                hi0 = x0;
                lo1 = x1 & 0x0F0F0F0Fu;
                hi1 = x1;
              }
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
                imma(c[uu][bl][q & 1][nt], lo0, hi0, lo1, hi1, bf[uu][st][nt][0], bf[uu][st][nt][1]);
            }
        if constexpr (A8) {
          // c[0], c[1]: rows grp (low nibbles) of A rows 2 tq, 2 tq + 1; c[2], c[3]: rows grp + 8
          // (high nibbles, 16 q). aqwc = dot - zp S is exact (every term < 2^24), and each block
          // adds (s_a s_w) aqwc as ms_qgemm_w4a8 does.
          float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
#pragma unroll
          for (int uu = 0; uu < UPW; ++uu)
#pragma unroll
            for (int bl = 0; bl < UB; ++bl) {
              int cc[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) cc[j] = c[uu][bl][0][0][j] + c[uu][bl][1][0][j];
              cc[2] -= cc[0];  // rows grp + 8: 16 D' (their MMA rows carried the low nibbles too)
              cc[3] -= cc[1];
              const float S0 = sv[uu][bl][0], S1 = sv16[uu][bl][0];
              const float d00 = (float)cc[0] - z0[uu][bl] * S0, d01 = (float)cc[1] - z0[uu][bl] * S1;
              const float d10 = (float)(cc[2] >> 4) - z1[uu][bl] * S0, d11 = (float)(cc[3] >> 4) - z1[uu][bl] * S1;
              a00 += (gw0[uu][bl][0] * s0[uu][bl]) * d00;
              a01 += (gw1[uu][bl][0] * s0[uu][bl]) * d01;
              a10 += (gw0[uu][bl][0] * s1[uu][bl]) * d10;
              a11 += (gw1[uu][bl][0] * s1[uu][bl]) * d11;
            }
          const int m0 = 2 * tq, m1 = m0 + 1;
          float* yr = ysum + (i * 16 + grp) * mc * kYPitch + warp;  // row grp + 8 sits 8 mc kYPitch further
          if (m0 < mc) {
            yr[m0 * kYPitch] += a00;
            yr[(8 * mc + m0) * kYPitch] += a10;
          }
          if (m1 < mc) {
            yr[m1 * kYPitch] += a01;
            yr[(8 * mc + m1) * kYPitch] += a11;
          }
        } else {
        float y0[NT], y1[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) y0[nt] = y1[nt] = 0.f;
#pragma unroll
        for (int uu = 0; uu < UPW; ++uu)
#pragma unroll
          for (int bl = 0; bl < UB; ++bl)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              int cc[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) cc[j] = c[uu][bl][0][nt][j] + c[uu][bl][1][nt][j];
              if constexpr (!B8) {  // rows grp + 8: 16 D' (their MMA rows carried the low nibbles too)
                cc[2] -= cc[0];
                cc[3] -= cc[1];
              }
              // even lanes hold digits 0 and 1 (and the zero-point term), odd lanes digit 2
              // and the always-zero fourth column: y += s 2^-sigma wdig (c_a + 256 c_b - z S / wdig)
              // with S = 0 on odd lanes, the integer combination exact in s32 (|c| < 2^22 even
              // for the 16x rows)
              const float f0 = fmaf(-z0[uu][bl], sv[uu][bl][nt], (float)(cc[0] + 256 * cc[1]));
              const float f1 = fmaf(-z1[uu][bl], sv16[uu][bl][nt], (float)(cc[2] + 256 * cc[3]));
              y0[nt] = fmaf(s0[uu][bl] * gw0[uu][bl][nt], f0, y0[nt]);
              y1[nt] = fmaf(s1[uu][bl] * gw1[uu][bl][nt], f1, y1[nt]);
            }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // digits 0,1 (even lane) + digit 2 (odd lane) of one A row: fold the pair
          const float v0 = y0[nt] + __shfl_xor_sync(0xffffffffu, y0[nt], 1);
          const float v1 = y1[nt] + __shfl_xor_sync(0xffffffffu, y1[nt], 1);
          const int m = nt * 2 + (tq >> 1);
          if (m < mc && (tq & 1) == 0) {
            float* yc = ysum + ((i * 16 + grp) * mc + m) * kYPitch + warp;
            yc[0] += v0;
            yc[8 * mc * kYPitch] += v1;
          }
        }
        }  // the digit form
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&empty[rs]);
      if (++rs == p.nslots) {
        rs = 0;
        rph ^= 1u;
      }
    }
  }
  ptx::named_bar_sync(1, kConsumers * 32);

  // ---- fixed-order sum of the kConsumers per-warp partials of each output: groups of G
  // consecutive threads per output (G as large as fits all outputs in one pass of the
  // consumer threads), each thread summing kConsumers/G partials in order, then a fixed
  // shuffle tree over G lanes
  const int nout = mc * p.rows_cta;
  int G = kConsumers;
  while (G > 1 && G * nout > kConsumers * 32) G >>= 1;
  const int per = kConsumers / G;
  for (int base = 0; base < nout * G; base += kConsumers * 32) {
    const int idx = base + tid;
    const int o = idx / G, j = idx - o * G;
    float acc = 0.f;
    if (o < nout) {
      const float* src = ysum + o * kYPitch + j * per;
      for (int q = 0; q < per; ++q) acc += src[q];
    }
    for (int off = G >> 1; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (o < nout && j == 0) {
      const int r = o / mc, m = o - r * mc;
      const int b = blockIdx.x + (r >> 4) * grid;
      const int64_t row = (int64_t)b * 16 + (r & 15);
      if (b < p.nblk && row < p.n_rows) {
        if (!A8 && nonfin[m]) {
          // RMSNorm of a row holding inf / NaN is NaN everywhere (inf / inf, 0 * inf)
          if (FU && p.gamma) acc = __int_as_float(0x7FC00000);
          else acc += nonfinite_terms<BS, FU, B8>(p, m, row);
        }
        if constexpr (XG) {
          for (int r = 0; r < p.nranks; ++r) p.gy[r][(p.m0 + m) * p.gldy + p.gcol0 + row] = acc;
        } else {
          float* yp = p.y + (p.m0 + m) * p.ldy + row;
          if constexpr (FU) {
            if (p.gamma) {
              float t = 0.f;
#pragma unroll
              for (int q = 0; q < kConsumers; ++q) t += rowsq[q * kMaxM + m];
              acc *= 1.0f / sqrtf(t / (float)p.K + p.eps);
            }
            if (p.accumulate) acc += *yp;
          }
          *yp = acc;
        }
      }
    }
  }
  if constexpr (XG) {
    // The CTA's stores are ordered before its completion count by the barrier and a GPU-scope
    // acquire-release count; the last CTA, having acquired every CTA's count, fences at system
    // scope (cumulative over all those stores) and releases one arrival to every rank.
    ptx::named_bar_sync(1, kConsumers * 32);
    if (tid == 0) {
      unsigned int prev;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.gdone) : "memory");
      if (prev == gridDim.x - 1) {
        asm volatile("fence.sc.sys;" ::: "memory");
        *p.gdone = 0u;  // the next launch of this layer is stream-ordered after this one
        atomicAdd(p.gprod, 1ull);
        for (int r = 0; r < p.nranks; ++r)
          asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(p.garr[r]) : "memory");
      }
    }
  }
}

// One thread: waits like a consuming launch for the latest gathered output.
__global__ void wait_gathered_kernel(const unsigned long long* arr, const unsigned long long* prod, int nranks) {
  griddep_wait();
  if (threadIdx.x == 0) wait_arrivals(arr, prod, nranks);
}

template <int BS, int NT, bool XG, bool FU, bool A8 = false, bool B8 = false>
int launch(cudaStream_t st, const Args& a, int grid, size_t smem) {
  auto kern = gemv_mma_kernel<BS, NT, XG, FU, A8, B8>;
  static ContextOnce configured;
  const int rc = configured.run([&] {
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax),
                 "mma gemv smem attribute");
    return MSQ_OK;
  });
  if (rc != MSQ_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MSQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a), "mma gemv launch");
  note_launch();
  return MSQ_OK;
}

inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

// Shared-memory plan for mc rows of A; returns the bytes, or 0 if fewer than 2 stages fit.
size_t plan_smem(const Weights& w, int mc, int grid, Args& a, bool a8 = false) {
  const int kp = w.ntiles * w.kt;
  const int head = 64 + 16 * kMaxM * 4;
  const int dig = (a8 ? 1 : 4) * mc * (kp + 16);  // B columns per A row: 3 digits + a zero, or one s8
  const int sb = align_up(8 * mc * (kp / w.block_size), 16);  // block sums + block scales
  a.rows_cta = ((w.nblk + grid - 1) / grid) * 16;
  const int ysum = align_up(a.rows_cta * mc * kYPitch * 4, 16);
  const int bars = 2 * kMaxSlots * 8 + 16;
  a.off_dig = align_up(head, 16);
  a.off_s = a.off_dig + align_up(dig, 16);
  a.off_ysum = a.off_s + sb;
  a.off_bar = a.off_ysum + ysum;
  a.off_ring = align_up(a.off_bar + bars, 128);
  if (a.off_ring >= kSmemMax) return 0;
  int slots = (kSmemMax - a.off_ring) / w.stage_bytes;
  slots = std::min(slots, 5);  // 3..5 stages of 17-35 KB stream best on B200
  if (slots < 2) return 0;
  a.nslots = slots;
  return (size_t)a.off_ring + (size_t)slots * w.stage_bytes;
}

template <int BS, bool XG, bool FU = false>
int launch_nt(cudaStream_t st, const Args& a, int grid, size_t smem) {
  return a.mc <= 2 ? launch<BS, 1, XG, FU>(st, a, grid, smem) : launch<BS, 2, XG, FU>(st, a, grid, smem);
}

}  // namespace

namespace {

// One decode GEMV call: passes of up to 4 A rows; with `g` (column split) a single pass
// whose outputs go to every rank's full-Y buffer, after waiting for `wt` (or nothing).
int gemv_impl(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y,
              int64_t ldy, const msq_wait_t* wt, const msq_gather_t* g, const Fusion* fu = nullptr,
              bool a8 = false) {
  if (!w.strm || (w.block_size != 32 && w.block_size != 64 && w.block_size != 128)) return MSQ_E_UNSUPPORTED;
  if (a8 && w.zp_kind == ZP_F32)
    return fail(MSQ_E_UNSUPPORTED, "msq_matmul_w4a8 takes packed or absent zero points (as ms_qgemm_w4a8)");
  const int unit = w.block_size > 64 ? w.block_size : 64;
  if (w.kt / unit > kUpw * kConsumers) return MSQ_E_UNSUPPORTED;
  const int sms = num_sms(w.device);
  int64_t m0 = 0;
  while (m0 < M) {
    Args a{};
    a.strm = w.strm;
    a.a = d_a;
    a.a_dtype = a_dtype;
    a.m0 = m0;
    a.y = d_y;
    a.ldy = ldy;
    a.n_rows = w.n_rows;
    a.K = w.K;
    a.kt = w.kt;
    a.ntiles = w.ntiles;
    a.nblk = w.nblk;
    a.stage_bytes = w.stage_bytes;
    a.off_sc = w.off_sc;
    a.off_zp = w.off_zp;
    a.zp_kind = w.zp_kind;
    a.kp = w.ntiles * w.kt;
    a.kpp = a.kp + 16;
    a.prefetch = w.settled.load(std::memory_order_relaxed) ? 1 : 0;
    {
      const uintptr_t ap = reinterpret_cast<uintptr_t>(d_a);
      const int align = a_dtype == MSQ_DT_F32 ? 16 : 8;
      a.a_vec = (w.K % 4 == 0) && (ap % align == 0);
    }
    a.lda = w.K;
    if (fu) {
      if (!a.a_vec || a_dtype != MSQ_DT_F32 || g) return MSQ_E_UNSUPPORTED;
      a.gamma = fu->gamma;
      a.eps = fu->eps;
      a.swiglu = fu->swiglu;
      a.accumulate = fu->accumulate;
      if (fu->swiglu) a.lda = 2 * (int64_t)w.K;
    }
    if (g) {
      a.nranks = g->nranks;
      for (int r = 0; r < g->nranks; ++r) {
        a.gy[r] = g->y[r];
        a.garr[r] = g->arrivals[r];
      }
      a.gldy = g->ldy;
      a.gcol0 = g->col0;
      a.gprod = g->produced;
      a.gdone = g->done;
      if (wt) {
        a.warr = wt->arrivals;
        a.wprod = wt->produced;
        a.wranks = wt->nranks;
      }
    }
    // the widest pass whose digits, row sums and ring fit in shared memory
    int mc = (int)std::min<int64_t>(a8 ? kMaxMA8 : kMaxM, M - m0);
    int grid = std::min(w.nblk, sms);
    size_t smem = 0;
    for (;;) {
      smem = plan_smem(w, mc, grid, a, a8);
      if (smem) break;
      if (grid < w.nblk) {
        grid = std::min(w.nblk, grid * 2);  // fewer rows per CTA -> smaller row-sum buffer
      } else if (mc > 1) {
        --mc;
        grid = std::min(w.nblk, sms);
      } else {
        return MSQ_E_UNSUPPORTED;
      }
    }
    if (g && mc < M) return fail(MSQ_E_UNSUPPORTED, "msq_matmul_gather: %lld A rows do not fit one pass", (long long)M);
    a.mc = mc;
    int rc;
    if (w.bits == 8) {
      if (g || fu || a8) return fail(MSQ_E_UNSUPPORTED, "bits=8 weights take the plain decode GEMV only");
      switch (w.block_size) {
        case 32: rc = a.mc <= 2 ? launch<32, 1, false, false, false, true>(st, a, grid, smem)
                                : launch<32, 2, false, false, false, true>(st, a, grid, smem); break;
        case 64: rc = a.mc <= 2 ? launch<64, 1, false, false, false, true>(st, a, grid, smem)
                                : launch<64, 2, false, false, false, true>(st, a, grid, smem); break;
        default: rc = a.mc <= 2 ? launch<128, 1, false, false, false, true>(st, a, grid, smem)
                                : launch<128, 2, false, false, false, true>(st, a, grid, smem); break;
      }
    } else if (a8) {
      switch (w.block_size) {
        case 32: rc = launch<32, 1, false, false, true>(st, a, grid, smem); break;
        case 64: rc = launch<64, 1, false, false, true>(st, a, grid, smem); break;
        default: rc = launch<128, 1, false, false, true>(st, a, grid, smem); break;
      }
    } else if (g) {
      switch (w.block_size) {
        case 32: rc = launch_nt<32, true>(st, a, grid, smem); break;
        case 64: rc = launch_nt<64, true>(st, a, grid, smem); break;
        default: rc = launch_nt<128, true>(st, a, grid, smem); break;
      }
    } else if (fu) {
      switch (w.block_size) {
        case 32: rc = launch_nt<32, false, true>(st, a, grid, smem); break;
        case 64: rc = launch_nt<64, false, true>(st, a, grid, smem); break;
        default: rc = launch_nt<128, false, true>(st, a, grid, smem); break;
      }
    } else {
      switch (w.block_size) {
        case 32: rc = launch_nt<32, false>(st, a, grid, smem); break;
        case 64: rc = launch_nt<64, false>(st, a, grid, smem); break;
        default: rc = launch_nt<128, false>(st, a, grid, smem); break;
      }
    }
    if (rc != MSQ_OK) return rc;
    m0 += mc;
  }
  if (w.bits == 8) {
    note_path(M <= 4 ? "gemv_imma_b8" : "gemv_imma_b8_multipass");
    return MSQ_OK;
  }
  note_path(a8 ? (M <= kMaxMA8 ? "gemv_w4a8" : "gemv_w4a8_multipass")
                : g ? "gemv_imma_gather" : fu ? "gemv_imma_fused" : M <= 4 ? "gemv_imma" : "gemv_imma_multipass");
  return MSQ_OK;
}

}  // namespace

int run_gemv_mma(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y,
                 int64_t ldy) {
  return gemv_impl(st, w, d_a, a_dtype, M, d_y, ldy, nullptr, nullptr);
}

int run_gemv_w4a8(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y,
                  int64_t ldy) {
  return gemv_impl(st, w, d_a, a_dtype, M, d_y, ldy, nullptr, nullptr, nullptr, true);
}

int run_gemv_gather(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
                    const msq_wait_t* wt, const msq_gather_t* g) {
  return gemv_impl(st, w, d_a, a_dtype, M, nullptr, 0, wt, g);
}

int run_gemv_fused(cudaStream_t st, const Weights& w, const float* d_a, int64_t M, float* d_y, int64_t ldy,
                   const Fusion& f) {
  return gemv_impl(st, w, d_a, MSQ_DT_F32, M, d_y, ldy, nullptr, nullptr, &f);
}

int run_wait_gathered(cudaStream_t st, const msq_wait_t* wt) {
  wait_gathered_kernel<<<1, 32, 0, st>>>(wt->arrivals, wt->produced, wt->nranks);
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "wait kernel launch");
  return MSQ_OK;
}

int set_wait_budget_gemv(unsigned long long ns) {
  MSQ_CUDA_TRY(cudaMemcpyToSymbol(ptx::g_wait_budget_ns, &ns, sizeof ns), "set decode GEMV wait budget");
  return MSQ_OK;
}

int read_gemv_mma_errors(cudaStream_t st, int* flags) {
  int v = 0;
  MSQ_CUDA_TRY(cudaMemcpyFromSymbolAsync(&v, g_mma_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st),
               "read mma gemv error word");
  MSQ_CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
  if (v) {
    const int zero = 0;
    MSQ_CUDA_TRY(cudaMemcpyToSymbolAsync(g_mma_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st),
                 "clear mma gemv error word");
    MSQ_CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
  }
  *flags = v;
  return MSQ_OK;
}

}  // namespace msq
