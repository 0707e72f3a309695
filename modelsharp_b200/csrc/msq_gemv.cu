// Decode GEMV for MatMulNBits, bits = 4, block_size a power of two >= 32, small M.
//
// Per output element Y[m, n] = sum_b s[n,b] * (sum_{k in b} a[m,k] * q[n,k] - zp[n,b] * S_b[m])
// where S_b[m] = sum_{k in b} a[m,k]. This is the reference's
// sum_k a[m,k] * ((q - zp) * s) (MatMulNBitsKernel.cs:236-261) with the per-block scale
// and zero point factored out; the fp32 rounding differs from the reference's order only
// at the last-ulp level (parity is checked at rel-L2 <= 1e-5).
//
// Memory: each weight row is a contiguous K/2-byte stripe of the repacked nibble plane;
// a warp streams 16-byte chunks (32 codes, always inside one quantisation block) with
// 128-bit streaming loads, lanes on consecutive chunks, so a warp load is 512 contiguous
// bytes. Scales (fp32) and packed zero points are read per (row, chunk).
//
// Arithmetic: a 32-bit word holds 8 codes in nibble slots ordered k-offsets
// {0,2,4,6,1,3,5,7}. Slot j is turned into the fp32 value 2^23 + q * 2^e_j by one
// LOP3 ((word & mask_j) | 0x4B000000), e = {0,4,8,12,16,8,12,16} (slots 5..7 after one
// 12-bit shift), and 2^23 is removed exactly with a packed FADD2. The activation is
// staged in shared memory pre-multiplied by 2^-e_j in the same slot order, so a packed
// FFMA2 accumulates a * q exactly as a * (float)q would. Per weight that is ~1.1 integer
// ops + 0.5 FADD2 + 0.5 FFMA2 (M = 1), which keeps the kernel on the HBM roofline.
//
// Work split: CTA b owns rows [b*rows_per_cta, ...); K is walked in shared-memory sized
// segments; a work item is (group of R rows, lane-chunk phase) and is reduced across the
// warp with shuffles into per-phase shared slots, summed in a fixed order at the end.
#include "msq_internal.cuh"
#include "msq_ptx.cuh"

#include <algorithm>

namespace msq {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kMagicBits = 0x4B000000u;  // 2^23 as fp32
constexpr float kMagic = 8388608.0f;
constexpr int kSmemBudget = 200 * 1024;

struct GemvArgs {
  const uint8_t* nib;
  int64_t nib_pitch;
  const float* sc;
  int64_t sc_pitch;
  const uint8_t* zp4;
  int64_t zp_pitch;
  const float* zpf;
  const void* a;
  int a_dtype;
  int64_t M;   // total rows of A
  int64_t m0;  // first A row of this launch
  float* y;
  int64_t ldy;
  int n_rows, K, nchunks, cpb_shift;
  int seg_chunks, rows_per_cta, phases;
};

// Writes the 32 activations of chunk c (k = 32c..32c+31) in slot order, scaled by 2^-e.
__device__ __forceinline__ float stage_chunk(const GemvArgs& p, int64_t arow, int kbase, float* dst) {
  float sum = 0.f;
#pragma unroll
  for (int w8 = 0; w8 < 4; ++w8) {
    float v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int k = kbase + w8 * 8 + t;
      v[t] = k < p.K ? load_act(p.a, p.a_dtype, arow + k) : 0.f;
      sum += v[t];
    }
    float4 lo = make_float4(v[0], v[2] * 0x1p-4f, v[4] * 0x1p-8f, v[6] * 0x1p-12f);
    float4 hi = make_float4(v[1] * 0x1p-16f, v[3] * 0x1p-8f, v[5] * 0x1p-12f, v[7] * 0x1p-16f);
    reinterpret_cast<float4*>(dst)[w8 * 2 + 0] = lo;
    reinterpret_cast<float4*>(dst)[w8 * 2 + 1] = hi;
  }
  return sum;
}

// Decodes the 8 codes of word x into 4 pairs (q * 2^e) in slot order.
__device__ __forceinline__ void decode_word(uint32_t x, float2 (&d)[4]) {
  const float2 neg = make_float2(-kMagic, -kMagic);
  const uint32_t x2 = x >> 12;
  float f0 = __uint_as_float((x & 0x0000000Fu) | kMagicBits);
  float f1 = __uint_as_float((x & 0x000000F0u) | kMagicBits);
  float f2 = __uint_as_float((x & 0x00000F00u) | kMagicBits);
  float f3 = __uint_as_float((x & 0x0000F000u) | kMagicBits);
  float f4 = __uint_as_float((x & 0x000F0000u) | kMagicBits);
  float f5 = __uint_as_float((x2 & 0x00000F00u) | kMagicBits);
  float f6 = __uint_as_float((x2 & 0x0000F000u) | kMagicBits);
  float f7 = __uint_as_float((x2 & 0x000F0000u) | kMagicBits);
  d[0] = __fadd2_rn(make_float2(f0, f1), neg);
  d[1] = __fadd2_rn(make_float2(f2, f3), neg);
  d[2] = __fadd2_rn(make_float2(f4, f5), neg);
  d[3] = __fadd2_rn(make_float2(f6, f7), neg);
}

template <int ZPK>
__device__ __forceinline__ float zero_point(const GemvArgs& p, int row, int blk) {
  if (ZPK == ZP_PACKED) {
    uint32_t zb = __ldg(p.zp4 + (int64_t)row * p.zp_pitch + (blk >> 1));
    return (float)((zb >> ((blk & 1) * 4)) & 0xFu);
  } else if (ZPK == ZP_F32) {
    return __ldg(p.zpf + (int64_t)row * p.sc_pitch + blk);
  }
  return 8.0f;
}

template <int MR, int R, int ZPK>
__global__ void __launch_bounds__(kThreads, 1) gemv_q4_kernel(const GemvArgs p) {
  extern __shared__ float4 smem4[];
  float* As = reinterpret_cast<float*>(smem4);
  const int segw = p.seg_chunks * 32;
  float* Ss = As + MR * segw;
  float* Ys = Ss + MR * p.seg_chunks;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(r0 + p.rows_per_cta, p.n_rows);
  if (r0 >= r1) return;
  const int nrows = r1 - r0;
  const int ngroups = (nrows + R - 1) / R;
  const int items = ngroups * p.phases;
  const int64_t mvalid = p.M - p.m0;

  for (int c0 = 0; c0 < p.nchunks; c0 += p.seg_chunks) {
    const int segc = min(p.seg_chunks, p.nchunks - c0);
    // ---- stage the activation segment (slot order, 2^-e pre-scaled) and chunk sums
    for (int idx = tid; idx < MR * segc; idx += kThreads) {
      const int m = idx / segc, c = idx - m * segc;
      float* dst = As + m * segw + c * 32;
      float sum = 0.f;
      if (m < mvalid) {
        sum = stage_chunk(p, (p.m0 + m) * (int64_t)p.K, (c0 + c) * 32, dst);
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) reinterpret_cast<float4*>(dst)[t] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      Ss[m * p.seg_chunks + c] = sum;
    }
    __syncthreads();

    // ---- stream the weight rows of this CTA over the segment
    for (int it = warp; it < items; it += kWarps) {
      const int g = it / p.phases, ph = it - g * p.phases;
      int rows[R];
      bool ok[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int rr = r0 + g * R + i;
        ok[i] = rr < r1;
        rows[i] = ok[i] ? rr : r0;
      }
      float yacc[R][MR];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int m = 0; m < MR; ++m) yacc[i][m] = 0.f;

      for (int c = ph * 32 + lane; c < segc; c += 32 * p.phases) {
        const int gc = c0 + c;
        uint4 wv[R];
#pragma unroll
        for (int i = 0; i < R; ++i)
          wv[i] = __ldcs(reinterpret_cast<const uint4*>(p.nib + (int64_t)rows[i] * p.nib_pitch) + gc);
        const int blk = gc >> p.cpb_shift;
        float s[R], z[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
          s[i] = __ldg(p.sc + (int64_t)rows[i] * p.sc_pitch + blk);
          z[i] = zero_point<ZPK>(p, rows[i], blk);
        }
        float2 acc[R][MR];
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
          for (int m = 0; m < MR; ++m) acc[i][m] = make_float2(0.f, 0.f);

#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
          float4 av[MR][2];
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            const float4* src = reinterpret_cast<const float4*>(As + m * segw + c * 32 + wd * 8);
            av[m][0] = src[0];
            av[m][1] = src[1];
          }
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const uint32_t x = wd == 0 ? wv[i].x : wd == 1 ? wv[i].y : wd == 2 ? wv[i].z : wv[i].w;
            float2 d[4];
            decode_word(x, d);
#pragma unroll
            for (int m = 0; m < MR; ++m) {
              acc[i][m] = __ffma2_rn(make_float2(av[m][0].x, av[m][0].y), d[0], acc[i][m]);
              acc[i][m] = __ffma2_rn(make_float2(av[m][0].z, av[m][0].w), d[1], acc[i][m]);
              acc[i][m] = __ffma2_rn(make_float2(av[m][1].x, av[m][1].y), d[2], acc[i][m]);
              acc[i][m] = __ffma2_rn(make_float2(av[m][1].z, av[m][1].w), d[3], acc[i][m]);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const float S = Ss[m * p.seg_chunks + c];
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const float P = acc[i][m].x + acc[i][m].y;
            yacc[i][m] = fmaf(s[i], fmaf(-z[i], S, P), yacc[i][m]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          float v = yacc[i][m];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
          if (lane == 0 && ok[i]) {
            float* slot = Ys + ((int64_t)ph * p.rows_per_cta + (g * R + i)) * MR + m;
            *slot = c0 == 0 ? v : *slot + v;
          }
        }
    }
    __syncthreads();
  }

  // ---- sum the phase slots in a fixed order and write Y rows (coalesced along n)
  for (int idx = tid; idx < nrows * MR; idx += kThreads) {
    const int m = idx / nrows, r = idx - m * nrows;
    if (m < mvalid) {
      float v = 0.f;
      for (int ph = 0; ph < p.phases; ++ph) v += Ys[((int64_t)ph * p.rows_per_cta + r) * MR + m];
      p.y[(p.m0 + m) * p.ldy + r0 + r] = v;
    }
  }
}

template <int MR, int R, int ZPK>
int launch_one(cudaStream_t st, GemvArgs a, int grid, size_t smem) {
  auto kern = gemv_q4_kernel<MR, R, ZPK>;
  static int configured_smem[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && configured_smem[dev] < (int)smem) {
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 16384),
                 "gemv smem attribute");
    configured_smem[dev] = kSmemBudget + 16384;
  }
  kern<<<grid, kThreads, smem, st>>>(a);
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "gemv kernel launch");
  return MSQ_OK;
}

template <int MR, int R>
int launch_zp(cudaStream_t st, int zp_kind, GemvArgs a, int grid, size_t smem) {
  switch (zp_kind) {
    case ZP_PACKED: return launch_one<MR, R, ZP_PACKED>(st, a, grid, smem);
    case ZP_F32: return launch_one<MR, R, ZP_F32>(st, a, grid, smem);
    default: return launch_one<MR, R, ZP_NONE>(st, a, grid, smem);
  }
}

inline int rows_per_warp(int mr) { return mr <= 2 ? 4 : (mr == 4 ? 2 : 1); }


// ============================================================================================
// Streamed decode GEMV (the default for bits = 4): a producer warp moves one row block x one
// k-tile of the interleaved record stream per stage (a single contiguous cp.async.bulk) into
// an up-to-8-deep shared-memory ring; 16 consumer warps decode it with one lane per weight
// row, so the activation chunk every lane needs is the same shared-memory word (broadcast)
// and the per-row sums never cross lanes until the end of the row block. Each consumer warp
// owns a fixed 1/16 of every tile's chunks; the 16 partial sums of a row are added in a
// fixed order at the end of its row block.
// ============================================================================================
constexpr int kSConsumers = 16;
constexpr int kSThreads = (kSConsumers + 1) * 32;
constexpr int kSMaxStages = 8;
constexpr int kSSmemMax = 227 * 1024;

__device__ int g_gemv_err;  // device error word of the streamed kernel (bounded waits)

struct StreamArgs {
  const uint8_t* strm;
  const void* a;
  int a_dtype;
  int64_t M, m0;
  float* y;
  int64_t ldy;
  int n_rows, K, kpad, kt, ntiles, rb, nblk, rec_bytes, rec_sc, rec_zp, bs_shift, nst, stage_bytes;
};

// Waits on an mbarrier unless the CTA has aborted; a timeout aborts the CTA.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              int code) {
  if (*abort_flag) return false;
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort_flag) return false;
      if (ptx::globaltimer() - t0 > ptx::kWaitBudgetNs) {
        *abort_flag = 1;
        atomicCAS(&g_gemv_err, 0, code);
        return false;
      }
    }
  }
}

// Loads A[row][k0 .. k0+7] as fp32 (zeros past K).
__device__ __forceinline__ void load8(const StreamArgs& p, int64_t row, int k0, float (&v)[8]) {
  const int64_t base = row * (int64_t)p.K + k0;
  if (k0 + 8 <= p.K && (p.K & 7) == 0) {
    if (p.a_dtype == MSQ_DT_F32) {
      const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p.a) + base);
      float4 x = q[0], y = q[1];
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
    } else {
      uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.a) + base);
      const uint32_t r[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (p.a_dtype == MSQ_DT_F16) {
          float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r[j]));
          v[2 * j] = f.x; v[2 * j + 1] = f.y;
        } else {
          float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[j]));
          v[2 * j] = f.x; v[2 * j + 1] = f.y;
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = k0 + j < p.K ? load_act(p.a, p.a_dtype, base + j) : 0.f;
  }
}

template <int MR>
__device__ __forceinline__ void stage_activations(const StreamArgs& p, float* As, float* Ss) {
  const int ngroups = p.kpad / 8;
  const int total = MR * ngroups;
  const int64_t mvalid = p.M - p.m0;
  for (int idx = threadIdx.x; idx < total; idx += kSConsumers * 32) {
    const int m = idx / ngroups, g = idx - m * ngroups;
    float v[8];
    if (m < mvalid) {
      load8(p, p.m0 + m, g * 8, v);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    float4* dst = reinterpret_cast<float4*>(As + (int64_t)m * p.kpad + g * 8);
    dst[0] = make_float4(v[0], v[2] * 0x1p-4f, v[4] * 0x1p-8f, v[6] * 0x1p-12f);
    dst[1] = make_float4(v[1] * 0x1p-16f, v[3] * 0x1p-8f, v[5] * 0x1p-12f, v[7] * 0x1p-16f);
    float s8 = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    const unsigned mask = __activemask();
    s8 += __shfl_xor_sync(mask, s8, 1);
    s8 += __shfl_xor_sync(mask, s8, 2);
    if ((g & 3) == 0) Ss[m * (p.kpad / 32) + (g >> 2)] = s8;
  }
}

template <int MR, int ZPK>
__global__ void __launch_bounds__(kSThreads, 1) gemv_stream_kernel(const StreamArgs p) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* As = reinterpret_cast<float*>(smem);
  float* Ss = As + MR * p.kpad;
  float* red = Ss + MR * (p.kpad / 32);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + kSConsumers * 32 * MR);
  uint64_t* empty = full + kSMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kSMaxStages);
  // bulk-copy destinations must be 16-byte aligned; round the ring's base up to 128 bytes
  uint8_t* stages = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(empty + kSMaxStages) + 16 + 127) & ~static_cast<uintptr_t>(127));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nst; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], kSConsumers);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();

  if (warp == kSConsumers) {
    // ---------------- producer: one elected lane issues the bulk copies
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int b = blockIdx.x; b < p.nblk && ok; b += gridDim.x)
        for (int t = 0; t < p.ntiles && ok; ++t) {
          const int s = issued % p.nst;
          const uint32_t u = issued / p.nst;
          if (issued >= p.nst) ok = wait_or_abort(&empty[s], (u - 1) & 1, abort_flag, ptx::kErrTimeoutEmpty);
          if (!ok) break;
          ptx::mbar_arrive_expect_tx(&full[s], p.stage_bytes);
          ptx::bulk_g2s(stages + (size_t)s * p.stage_bytes,
                        p.strm + ((int64_t)b * p.ntiles + t) * (int64_t)p.stage_bytes, p.stage_bytes, &full[s]);
          ++issued;
        }
      // Drain: the last copy issued into each slot must land before this CTA may exit.
      for (int s = 0; s < p.nst && s < issued; ++s) {
        const int last = s + (issued - 1 - s) / p.nst * p.nst;
        const uint32_t u = last / p.nst;
        const unsigned long long t0 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&full[s], u & 1)) {
          if (ptx::globaltimer() - t0 > ptx::kWaitBudgetNs) {
            atomicCAS(&g_gemv_err, 0, ptx::kErrTimeoutDrain);
            break;
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers
  stage_activations<MR>(p, As, Ss);
  ptx::named_bar_sync(1, kSConsumers * 32);

  const int CT = p.kt / 32;
  const int sw = p.kpad / 32;
  const int64_t mvalid = p.M - p.m0;
  int it = 0;
  for (int b = blockIdx.x; b < p.nblk; b += gridDim.x) {
    float yacc[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) yacc[m] = 0.f;
    for (int t = 0; t < p.ntiles; ++t, ++it) {
      const int s = it % p.nst;
      const uint32_t u = it / p.nst;
      const bool ok = wait_or_abort(&full[s], u & 1, abort_flag, ptx::kErrTimeoutFull);
      if (ok && lane < p.rb) {
        const uint8_t* rec = stages + (size_t)s * p.stage_bytes + lane * p.rec_bytes;
#pragma unroll 2
        for (int c = warp; c < CT; c += kSConsumers) {
          const uint4 wv = *reinterpret_cast<const uint4*>(rec + c * 16);
          const int bl = (c * 32) >> p.bs_shift;
          const float sc = *reinterpret_cast<const float*>(rec + p.rec_sc + 4 * bl);
          float z;
          if (ZPK == ZP_PACKED) {
            z = (float)((rec[p.rec_zp + (bl >> 1)] >> ((bl & 1) * 4)) & 0xF);
          } else if (ZPK == ZP_F32) {
            z = *reinterpret_cast<const float*>(rec + p.rec_zp + 4 * bl);
          } else {
            z = 8.0f;
          }
          const int g = t * CT + c;
          const float4* a4 = reinterpret_cast<const float4*>(As) + g * 8;
          float2 acc[MR];
#pragma unroll
          for (int m = 0; m < MR; ++m) acc[m] = make_float2(0.f, 0.f);
#pragma unroll
          for (int wd = 0; wd < 4; ++wd) {
            const uint32_t x = wd == 0 ? wv.x : wd == 1 ? wv.y : wd == 2 ? wv.z : wv.w;
            float2 d[4];
            decode_word(x, d);
#pragma unroll
            for (int m = 0; m < MR; ++m) {
              const float4 lo = a4[(int64_t)m * (p.kpad / 4) + 2 * wd];
              const float4 hi = a4[(int64_t)m * (p.kpad / 4) + 2 * wd + 1];
              acc[m] = __ffma2_rn(make_float2(lo.x, lo.y), d[0], acc[m]);
              acc[m] = __ffma2_rn(make_float2(lo.z, lo.w), d[1], acc[m]);
              acc[m] = __ffma2_rn(make_float2(hi.x, hi.y), d[2], acc[m]);
              acc[m] = __ffma2_rn(make_float2(hi.z, hi.w), d[3], acc[m]);
            }
          }
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            const float P = acc[m].x + acc[m].y;
            yacc[m] = fmaf(sc, fmaf(-z, Ss[m * sw + g], P), yacc[m]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&empty[s]);
    }
    // fixed-order cross-warp reduction of the row block
#pragma unroll
    for (int m = 0; m < MR; ++m) red[(warp * 32 + lane) * MR + m] = yacc[m];
    ptx::named_bar_sync(1, kSConsumers * 32);
    if ((int)threadIdx.x < p.rb * MR) {
      const int rr = threadIdx.x % p.rb, m = threadIdx.x / p.rb;
      const int64_t row = (int64_t)b * p.rb + rr;
      float v = 0.f;
      for (int w = 0; w < kSConsumers; ++w) v += red[(w * 32 + rr) * MR + m];
      if (row < p.n_rows && m < mvalid) p.y[(p.m0 + m) * p.ldy + row] = v;
    }
    ptx::named_bar_sync(1, kSConsumers * 32);
  }
}

template <int MR, int ZPK>
int launch_stream(cudaStream_t st, const StreamArgs& a, int grid, size_t smem) {
  auto kern = gemv_stream_kernel<MR, ZPK>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSSmemMax),
                 "stream gemv smem attribute");
    configured[dev] = true;
  }
  kern<<<grid, kSThreads, smem, st>>>(a);
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "stream gemv launch");
  return MSQ_OK;
}

template <int MR>
int launch_stream_zp(cudaStream_t st, int zp_kind, const StreamArgs& a, int grid, size_t smem) {
  switch (zp_kind) {
    case ZP_PACKED: return launch_stream<MR, ZP_PACKED>(st, a, grid, smem);
    case ZP_F32: return launch_stream<MR, ZP_F32>(st, a, grid, smem);
    default: return launch_stream<MR, ZP_NONE>(st, a, grid, smem);
  }
}

// Shared-memory plan of the streamed kernel; returns 0 when it does not fit.
size_t stream_smem(const Weights& w, int mr, int* nst) {
  const size_t kpad = (size_t)w.ntiles * w.kt;
  const size_t fixed = sizeof(float) * (mr * kpad + mr * kpad / 32 + (size_t)kSConsumers * 32 * mr) +
                       2 * kSMaxStages * sizeof(uint64_t) + 16 + 128;
  const size_t stage = (size_t)w.rb * w.rec_bytes;
  if (fixed + 2 * stage > (size_t)kSSmemMax) return 0;
  int n = (int)((kSSmemMax - fixed) / stage);
  if (n > kSMaxStages) n = kSMaxStages;
  *nst = n;
  return fixed + (size_t)n * stage;
}

int run_gemv_stream(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y,
                    int64_t ldy, int mr) {
  int nst = 0;
  const size_t smem = stream_smem(w, mr, &nst);
  if (!smem || !w.strm) return MSQ_E_UNSUPPORTED;
  StreamArgs a{};
  a.strm = w.strm;
  a.a = d_a;
  a.a_dtype = a_dtype;
  a.M = M;
  a.y = d_y;
  a.ldy = ldy;
  a.n_rows = w.n_rows;
  a.K = w.K;
  a.kt = w.kt;
  a.ntiles = w.ntiles;
  a.kpad = w.ntiles * w.kt;
  a.rb = w.rb;
  a.nblk = w.nblk;
  a.rec_bytes = w.rec_bytes;
  a.rec_sc = w.rec_sc;
  a.rec_zp = w.rec_zp;
  int sh = 0;
  while ((1 << sh) < w.block_size) ++sh;
  a.bs_shift = sh;
  a.nst = nst;
  a.stage_bytes = w.rb * w.rec_bytes;
  const int grid = std::min(w.nblk, num_sms(w.device));
  for (int64_t m0 = 0; m0 < M; m0 += mr) {
    a.m0 = m0;
    int rc;
    switch (mr) {
      case 1: rc = launch_stream_zp<1>(st, w.zp_kind, a, grid, smem); break;
      case 2: rc = launch_stream_zp<2>(st, w.zp_kind, a, grid, smem); break;
      case 4: rc = launch_stream_zp<4>(st, w.zp_kind, a, grid, smem); break;
      default: rc = launch_stream_zp<8>(st, w.zp_kind, a, grid, smem); break;
    }
    if (rc != MSQ_OK) return rc;
  }
  return MSQ_OK;
}

}  // namespace

int run_gemv(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
             float* d_y, int64_t ldy) {
  if (!w.fast4) return fail(MSQ_E_UNSUPPORTED, "GEMV path needs bits=4 and a power-of-two block_size >= 32");
  if (M <= 0) return MSQ_OK;
  const int sms = num_sms(w.device);
  const int mr = M == 1 ? 1 : M == 2 ? 2 : M <= 4 ? 4 : 8;
  {
    const int rc = run_gemv_stream(st, w, d_a, a_dtype, M, d_y, ldy, mr);
    if (rc != MSQ_E_UNSUPPORTED) {
      if (rc == MSQ_OK) note_path(mr == 1 ? "gemv_stream_m1" : mr == 2 ? "gemv_stream_m2" : mr == 4 ? "gemv_stream_m4" : "gemv_stream_m8");
      return rc;
    }
  }
  // Too large for the streamed kernel's shared memory: K-segmented kernel below.
  const int R = rows_per_warp(mr);

  GemvArgs a{};
  a.nib = w.nib;
  a.nib_pitch = w.nib_pitch;
  a.sc = w.sc;
  a.sc_pitch = w.sc_pitch;
  a.zp4 = w.zp4;
  a.zp_pitch = w.zp_pitch;
  a.zpf = w.zpf;
  a.a = d_a;
  a.a_dtype = a_dtype;
  a.M = M;
  a.y = d_y;
  a.ldy = ldy;
  a.n_rows = w.n_rows;
  a.K = w.K;
  a.nchunks = (w.K + 31) / 32;
  int cpb = w.block_size / 32, sh = 0;
  while ((1 << sh) < cpb) ++sh;
  a.cpb_shift = sh;

  const int grid = std::max(1, std::min(sms, (w.n_rows + R - 1) / R));
  a.rows_per_cta = (w.n_rows + grid - 1) / grid;
  const int ngroups = (a.rows_per_cta + R - 1) / R;
  int phases = (6 * kWarps + ngroups - 1) / ngroups;
  phases = std::max(1, std::min(phases, a.nchunks / 64));
  a.phases = phases;
  const size_t ys_bytes = sizeof(float) * (size_t)phases * a.rows_per_cta * mr;
  if (ys_bytes + (size_t)mr * 132 * 32 > (size_t)kSmemBudget)
    return fail(MSQ_E_UNSUPPORTED, "GEMV: too many rows per CTA for shared memory");
  int seg = (int)((kSmemBudget - ys_bytes) / ((size_t)mr * 132));
  seg = std::min(seg, a.nchunks);
  if (seg < a.nchunks) seg = std::max(32, seg / 32 * 32);
  a.seg_chunks = seg;
  const size_t smem = sizeof(float) * (size_t)mr * seg * 33 + ys_bytes;

  for (int64_t m0 = 0; m0 < M; m0 += mr) {
    a.m0 = m0;
    int rc;
    switch (mr) {
      case 1: rc = launch_zp<1, 4>(st, w.zp_kind, a, grid, smem); break;
      case 2: rc = launch_zp<2, 4>(st, w.zp_kind, a, grid, smem); break;
      case 4: rc = launch_zp<4, 2>(st, w.zp_kind, a, grid, smem); break;
      default: rc = launch_zp<8, 1>(st, w.zp_kind, a, grid, smem); break;
    }
    if (rc != MSQ_OK) return rc;
  }
  note_path(mr == 1 ? "gemv_seg_m1" : mr == 2 ? "gemv_seg_m2" : mr == 4 ? "gemv_seg_m4" : "gemv_seg_m8");
  return MSQ_OK;
}

int read_gemv_errors(cudaStream_t st, int* flags) {
  int v = 0;
  MSQ_CUDA_TRY(cudaMemcpyFromSymbolAsync(&v, g_gemv_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st),
               "read gemv error word");
  MSQ_CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
  if (v) {
    const int zero = 0;
    MSQ_CUDA_TRY(cudaMemcpyToSymbolAsync(g_gemv_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st),
                 "clear gemv error word");
    MSQ_CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
  }
  *flags = v;
  return MSQ_OK;
}

}  // namespace msq
