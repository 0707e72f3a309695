// Prefill GEMM for MatMulNBits on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   Y[m, n] = sum_k A[m, k] * W[n, k],  W[n, k] = fp16((q[n,k] - zp[n,b]) * s[n,b])
//
// One CTA computes a (128 TM) x BN tile of Y over k-stages of 64: TM accumulators of 128
// activation rows (TMEM lanes) x BN weight rows (TMEM columns) that share one dequantised
// weight tile, so each dequantised weight feeds 128 TM rows (BN = 128; TM = 3 or 4 for
// M >= 512, by whole waves of tiles, 2 for M > 128, 1 below):
//   TMA warp    per stage: the fp16 activation tile (128 x 64, 128-byte swizzle), the packed
//               int4 weight tile (BN rows x 32 bytes) and a 16-byte column of scales and of
//               zero points per weight row covering the stage's blocks, no multicast;
//   dequant     one thread per half row (32 codes, one block at block_size 32): reads its
//   warps       16 bytes of codes and its scale / zero point from shared memory, writes fp16
//               (q - zp) * s straight into the K-major 128-byte-swizzled layout the tensor
//               core reads, then releases the stage;
//   MMA warp    allocates TMEM and, from one lane, issues 4 TM x tcgen05.mma (M=128, N=BN,
//               K=16) per stage into the fp32 accumulators in TMEM, committing each stage
//               back to the producer;
//   dequant     finally read the accumulator with tcgen05.ld and store fp32 Y.
//   warps
// The dequantised operand is exact up to one fp16 rounding of (q - zp) * s; products and
// sums are fp32 in the tensor core (parity bar: rel-L2 <= 5e-3 against the fp32 reference).
// fp32 / bf16 activations are converted to fp16 into a stream-ordered scratch buffer first.
#include "msq_internal.cuh"
#include "msq_ptx.cuh"

#include <cuda.h>

#include <algorithm>
#include <mutex>

namespace msq {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;

__device__ int g_gemm_err;

// SPLIT: the operands enter the tensor core as two fp16 parts each, hi = fp16(x) and
// lo = fp16(x - hi), and each k-step issues hi.hi + hi.lo + lo.hi (the lo.lo term is below fp32
// rounding): products good to ~2^-22 instead of fp16's 2^-11, at three MMAs per step and a
// second dequantised tile. Weights are (q - zp) * s computed in fp32 from the exact fp32 scales.
template <int TM, int BN, bool SPLIT = false>
struct Plan {
  static constexpr int kParts = SPLIT ? 2 : 1;        // fp16 parts per operand tile (hi, lo)
  static constexpr int kRows = BM * TM;               // activation rows of a tile
  static constexpr int kCols = TM * BN;               // TMEM columns (the TM accumulators)
  static constexpr int kDeq = BN / 16;                // dequant warps: one thread per half row
  static constexpr int kThreads = (kDeq + 2) * 32;    // + TMA warp + MMA warp
  static constexpr int kTmaWarp = kDeq;
  static constexpr int kMmaWarp = kDeq + 1;
  // what fits in 227 KB (SPLIT: TM <= 2)
  static constexpr int kStages = SPLIT ? (TM == 1 ? 3 : 2) : (TM == 1 ? 4 : TM == 2 || TM == 3 ? 3 : 2);
  static constexpr int kAPart = kRows * BK * 2;       // one fp16 activation tile: 16 / 32 / 64 KB
  static constexpr int kABytes = kAPart * kParts;     // hi tile, then lo tile
  // activation TMA boxes per part: 256-row boxes, or 128-row ones when the tile is not a
  // multiple of 256 rows (TM = 1, 3)
  static constexpr int kABoxes = kRows % 256 == 0 ? kRows / 256 : kRows / 128;
  static constexpr int kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128 : kCols <= 256 ? 256 : 512;
  static constexpr int kBPart = BN * BK * 2;          // one dequantised fp16 weight tile
  static constexpr int kBBytes = kBPart * kParts;
  static constexpr int kPBytes = BN * BK / 2;         // packed int4 weights
  static constexpr int kSBytes = BN * 16;             // 8 fp16 (SPLIT: 4 fp32) scales per row
  static constexpr int kZBytes = BN * 16;             // 32 packed or 4 fp32 zero points per row
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kABytes;
  static constexpr int kOffP = kOffB + kStages * kBBytes;
  static constexpr int kOffS = kOffP + kStages * kPBytes;
  static constexpr int kOffZ = kOffS + kStages * kSBytes;
  static constexpr int kOffBar = kOffZ + kStages * kZBytes;
  static constexpr int kBarBytes = (4 * kStages + 1) * 8 + 16;
  static constexpr int kSmem = kOffBar + kBarBytes + 1024;  // + alignment slack
};

struct GemmArgs {
  float* y;
  int64_t ldy;
  int M, n_rows, K, ksteps;
  int bs_shift;
  int vec_store;
  int kper;              // k-stages per CTA: blockIdx.z takes stages [z kper, (z + 1) kper)
  int64_t split_stride;  // with several k-splits: elements between their partial outputs
  const float* row_scale;  // staged A: row m entered the tensor core as a * 2^e_m; Y row m is
                           // multiplied by row_scale[m] = 2^-e_m (exact). nullptr: A as given
  int a_lo_row;            // SPLIT: row of the activation map where the lo parts start (M), or 0
                           // when A has no lo part (fp16 A: hi alone is exact)
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ bool wait_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (*abort_flag) return false;
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait_sleep(bar, parity)) return true;
    if ((i & 7u) == 0) {
      if (*abort_flag) return false;
      if (ptx::globaltimer() - t0 > budget) {
        *abort_flag = 1;
        atomicCAS(&g_gemm_err, 0, code);
        return false;
      }
    }
  }
}

// (1024 + q) as fp16 pairs from a nibble pair mask, then exact (q - zp) and one rounding * s.
__device__ __forceinline__ uint32_t deq_pair(uint32_t bits, __half2 zc, __half2 s2) {
  const uint32_t h = (bits & 0x000F000Fu) | 0x64006400u;
  const __half2 v = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&h), zc), s2);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t deq_pair_f32(uint32_t bits, float z, float s) {
  const float lo = ((float)(bits & 0xF) - z) * s;
  const float hi = ((float)((bits >> 16) & 0xF) - z) * s;
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// A code pair's weights (q - zp) * s in fp32, as fp16 hi parts and fp16 lo = w - hi parts.
__device__ __forceinline__ void deq_split(uint32_t bits, float z, float s, uint32_t& hi, uint32_t& lo) {
  const float w0 = ((float)(bits & 0xF) - z) * s;
  const float w1 = ((float)((bits >> 16) & 0xF) - z) * s;
  const __half2 h = __floats2half2_rn(w0, w1);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(w0 - hf.x, w1 - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <int TM, int BN, int ZPK, bool SPLIT>
__global__ void __launch_bounds__(Plan<TM, BN, SPLIT>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmP,
                   const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ,
                   const GemmArgs p) {
  using PL = Plan<TM, BN, SPLIT>;
  constexpr int S = PL::kStages;
  constexpr int kDeqWarps = PL::kDeq;
  constexpr int kTmaWarp = PL::kTmaWarp;
  constexpr int kMmaWarp = PL::kMmaWarp;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  // afull: the stage's activation tile landed (the MMA waits for it); pfull: its codes, scales
  // and zero points landed (the dequant warps wait only for these, not for the larger A tile)
  uint64_t* afull = reinterpret_cast<uint64_t*>(smem + PL::kOffBar);
  uint64_t* pfull = afull + S;
  uint64_t* wready = pfull + S;
  uint64_t* empty = wready + S;
  uint64_t* accum = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * PL::kRows;
  // this CTA's k-stages (never empty: the host sizes the splits)
  const int kb = (int)blockIdx.z * p.kper;
  const int nk = min(p.ksteps, kb + p.kper) - kb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&afull[s], 1);
      ptx::mbar_init(&pfull[s], 1);
      ptx::mbar_init(&wready[s], kDeqWarps);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(accum, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(tmem_slot, PL::kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&tmP);
    ptx::prefetch_tmap(&tmS);
    if (ZPK != ZP_NONE) ptx::prefetch_tmap(&tmZ);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarp) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int kt = kb + i, s = i % S;
        const uint32_t u = i / S;
        if (i >= S && !wait_abort(&empty[s], (u - 1) & 1, abort_flag, ptx::kErrTimeoutEmpty)) break;
        // scales / zero points: the 16-byte-aligned column holding the stage's block(s)
        const int blk0 = (kt * BK) >> p.bs_shift;
        const bool lo = SPLIT && p.a_lo_row > 0;
        // the weight side first: it feeds the dequant warps, which the MMA then waits for
        ptx::mbar_arrive_expect_tx(&pfull[s], PL::kPBytes + PL::kSBytes + (ZPK != ZP_NONE ? PL::kZBytes : 0));
        ptx::tma_load_2d(smem + PL::kOffP + s * PL::kPBytes, &tmP, &pfull[s], kt * (BK / 2), n0);
        ptx::tma_load_2d(smem + PL::kOffS + s * PL::kSBytes, &tmS, &pfull[s], SPLIT ? (blk0 & ~3) : (blk0 & ~7), n0);
        if (ZPK == ZP_PACKED)
          ptx::tma_load_2d(smem + PL::kOffZ + s * PL::kZBytes, &tmZ, &pfull[s], (blk0 >> 1) & ~15, n0);
        else if (ZPK == ZP_F32)
          ptx::tma_load_2d(smem + PL::kOffZ + s * PL::kZBytes, &tmZ, &pfull[s], blk0 & ~3, n0);
        ptx::mbar_arrive_expect_tx(&afull[s], PL::kAPart * (lo ? 2 : 1));
#pragma unroll
        for (int h = 0; h < PL::kABoxes; ++h)  // a box is at most 256 rows
          ptx::tma_load_2d(smem + PL::kOffA + s * PL::kABytes + h * (PL::kAPart / PL::kABoxes), &tmA, &afull[s],
                           kt * BK, m0 + h * (PL::kRows / PL::kABoxes));
        if (lo) {
#pragma unroll
          for (int h = 0; h < PL::kABoxes; ++h)
            ptx::tma_load_2d(smem + PL::kOffA + s * PL::kABytes + PL::kAPart + h * (PL::kAPart / PL::kABoxes), &tmA,
                             &afull[s], kt * BK, p.a_lo_row + m0 + h * (PL::kRows / PL::kABoxes));
        }
        ++issued;
      }
      for (int s = 0; s < S && s < issued; ++s) {  // drain copies in flight
        const int last = s + (issued - 1 - s) / S * S;
        const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
        bool timed_out = false;
        for (uint64_t* bar : {&afull[s], &pfull[s]})
          while (!timed_out && !ptx::mbar_try_wait(bar, (last / S) & 1)) {
            if (ptx::globaltimer() - t0 > budget) {
              atomicCAS(&g_gemm_err, 0, ptx::kErrTimeoutDrain);
              timed_out = true;
            }
          }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % S;
        const uint32_t u = i / S;
        ok = wait_abort(&afull[s], u & 1, abort_flag, ptx::kErrTimeoutFull) &&
             wait_abort(&wready[s], u & 1, abort_flag, ptx::kErrTimeoutFull);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint64_t bd = sw128_desc(ptx::smem_u32(smem + PL::kOffB + s * PL::kBBytes));
#pragma unroll
        for (int t = 0; t < TM; ++t) {  // accumulator t: activation rows 128t.. of the tile
          const uint64_t ad = sw128_desc(ptx::smem_u32(smem + PL::kOffA + s * PL::kABytes + t * BM * 128));
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            ptx::mma_f16(tmem + (uint32_t)(t * BN), ad + 2 * j, bd + 2 * j, idesc, (i | j) != 0);
          if constexpr (SPLIT) {
            const uint64_t bdl = sw128_desc(ptx::smem_u32(smem + PL::kOffB + s * PL::kBBytes + PL::kBPart));
#pragma unroll
            for (int j = 0; j < BK / 16; ++j)
              ptx::mma_f16(tmem + (uint32_t)(t * BN), ad + 2 * j, bdl + 2 * j, idesc, 1u);
            if (p.a_lo_row > 0) {
              const uint64_t adl =
                  sw128_desc(ptx::smem_u32(smem + PL::kOffA + s * PL::kABytes + PL::kAPart + t * BM * 128));
#pragma unroll
              for (int j = 0; j < BK / 16; ++j)
                ptx::mma_f16(tmem + (uint32_t)(t * BN), adl + 2 * j, bd + 2 * j, idesc, 1u);
            }
          }
        }
        ptx::mma_commit(&empty[s]);
      }
      ptx::mma_commit(accum);
      // the accumulator (and every MMA reading shared memory) must be done before exit
      const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
      while (!ptx::mbar_try_wait(accum, 0)) {
        if (ptx::globaltimer() - t0 > budget) {
          atomicCAS(&g_gemm_err, 0, ptx::kErrTimeoutMma);
          break;
        }
      }
    }
  } else {
    // ---------------- dequantisation warps: thread t takes half row t (codes 16t..16t+15 of
    // the packed tile: row t/2, k 32(t%2)..+31), so a warp's code loads are one contiguous
    // 512-byte run and its swizzled stores hit every bank group once per 128 bytes
    const int tid = threadIdx.x;  // 0 .. 2*BN-1
    const int r = tid >> 1, c = tid & 1;
    uint8_t* brow_base = smem + PL::kOffB + (r >> 3) * 1024 + (r & 7) * 128;
    for (int i = 0; i < nk; ++i) {
      const int kt = kb + i, s = i % S;
      const uint32_t u = i / S;
      const bool ok = wait_abort(&pfull[s], u & 1, abort_flag, ptx::kErrTimeoutFull);
      if (ok) {
        const uint4 w4 = *reinterpret_cast<const uint4*>(smem + PL::kOffP + s * PL::kPBytes + tid * 16);
        const int blk0 = (kt * BK) >> p.bs_shift;
        const int blk = (kt * BK + c * 32) >> p.bs_shift;
        const float sf =
            SPLIT ? reinterpret_cast<const float*>(smem + PL::kOffS + s * PL::kSBytes + r * 16)[blk - (blk0 & ~3)]
                  : __half2float(
                        reinterpret_cast<const __half*>(smem + PL::kOffS + s * PL::kSBytes + r * 16)[blk - (blk0 & ~7)]);
        float zf = 8.f;
        if (ZPK == ZP_PACKED) {
          const uint8_t zb = (smem + PL::kOffZ + s * PL::kZBytes + r * 16)[(blk >> 1) - ((blk0 >> 1) & ~15)];
          zf = (float)((zb >> ((blk & 1) * 4)) & 0xF);
        } else if (ZPK == ZP_F32) {
          zf = reinterpret_cast<const float*>(smem + PL::kOffZ + s * PL::kZBytes + r * 16)[blk - (blk0 & ~3)];
        }
        uint8_t* brow = brow_base + s * PL::kBBytes;
        const uint32_t words[4] = {w4.x, w4.y, w4.z, w4.w};
        const __half2 zc = __float2half2_rn(1024.f + zf);
        const __half2 s2 = __float2half2_rn(sf);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t x = words[j];
          const int wi = 4 * c + j;  // 8-k group of the row
          if constexpr (SPLIT) {
            uint4 oh, ol;
            deq_split(x, zf, sf, oh.x, ol.x);
            deq_split(x >> 4, zf, sf, oh.y, ol.y);
            deq_split(x >> 8, zf, sf, oh.z, ol.z);
            deq_split(x >> 12, zf, sf, oh.w, ol.w);
            *reinterpret_cast<uint4*>(brow + ((wi ^ (r & 7)) << 4)) = oh;
            *reinterpret_cast<uint4*>(brow + PL::kBPart + ((wi ^ (r & 7)) << 4)) = ol;
            continue;
          }
          uint4 o;
          if (ZPK == ZP_F32) {
            o.x = deq_pair_f32(x, zf, sf);
            o.y = deq_pair_f32(x >> 4, zf, sf);
            o.z = deq_pair_f32(x >> 8, zf, sf);
            o.w = deq_pair_f32(x >> 12, zf, sf);
          } else {
            o.x = deq_pair(x, zc, s2);
            o.y = deq_pair(x >> 4, zc, s2);
            o.z = deq_pair(x >> 8, zc, s2);
            o.w = deq_pair(x >> 12, zc, s2);
          }
          *reinterpret_cast<uint4*>(brow + ((wi ^ (r & 7)) << 4)) = o;
        }
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&wready[s]);
    }

    // ---------------- epilogue: TMEM -> registers -> Y
    // warp-uniform: tcgen05.ld below is a .sync.aligned warp instruction
    const bool ok = __all_sync(0xffffffffu, wait_abort(accum, 0, abort_flag, ptx::kErrTimeoutMma));
    ptx::tc_fence_after();
    if (ok) {
      const int q = warp & 3;                 // TMEM lane quarter of this warp
      const int cg = warp >> 2;               // column group
      constexpr int kCols = PL::kCols / (kDeqWarps / 4);
#pragma unroll 1
      for (int cc = 0; cc < kCols; cc += 32) {
        const int tcol = cg * kCols + cc;     // TMEM column: accumulator tcol / BN
        const int col = tcol % BN;
        const int m = m0 + (tcol / BN) * BM + q * 32 + lane;
        uint32_t v[32];
        ptx::tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)tcol, v);
        ptx::tmem_ld_wait();
        if (m < p.M) {
          if (p.row_scale) {
            const float rs = p.row_scale[m];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * rs);
          }
          float* yrow = p.y + blockIdx.z * p.split_stride + (int64_t)m * p.ldy + n0 + col;
          if (p.vec_store && n0 + col + 32 <= p.n_rows) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(yrow + j) = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                                 __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + col + j < p.n_rows) yrow[j] = __uint_as_float(v[j]);
          }
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, PL::kTmemCols);
  }
}

// fp32 / bf16 / unaligned fp16 activations -> fp16 [M][lda] (k < K only), one block of 256
// threads per row (a warp per row left 32 warps to stage the 28672-k rows of a 32-row down
// projection, hundreds of microseconds of dependent loads). fp16 holds magnitudes up to 65504
// and keeps full precision only above 2^-14, while the reference computes in fp32; so each row
// is scaled by a power of two 2^e chosen from its largest finite magnitude (that maximum lands
// in [2^14, 2^15)) before the rounding, and row_scale[m] = 2^-e undoes it exactly in the GEMM's
// epilogue. Infinities and NaNs pass through unchanged, so they propagate through the tensor
// core as in the fp32 reference. With out_lo (the split GEMM), also the fp16 remainder
// lo = fp16(a 2^e - hi) of every element.
constexpr int kStageThreads = 256;

__global__ void __launch_bounds__(kStageThreads) to_half_rows_kernel(const void* __restrict__ a, int dt, int64_t M,
                                                                     int K, __half* __restrict__ out, int64_t lda,
                                                                     float* __restrict__ row_scale,
                                                                     __half* __restrict__ out_lo) {
  __shared__ uint32_t red[kStageThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    const int64_t base = m * (int64_t)K;
    float mx = 0.f;
    for (int k = tid; k < K; k += kStageThreads) {
      const float v = fabsf(load_act(a, dt, base + k));
      if (v <= 3.402823466e38f) mx = fmaxf(mx, v);  // finite only (false for NaN and inf)
    }
    // non-negative floats order as their bits
    uint32_t u = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
    if (lane == 0) red[warp] = u;
    __syncthreads();
    u = __reduce_max_sync(0xffffffffu, red[lane % (kStageThreads / 32)]);
    __syncthreads();  // red is reused by the next row
    mx = __uint_as_float(u);
    int e = 0;
    if (mx > 0.f) {
      int ex;
      frexpf(mx, &ex);                   // mx = f 2^ex, f in [0.5, 1)
      e = max(-120, min(120, 15 - ex));  // mx 2^e in [2^14, 2^15)
    }
    const float up = ldexpf(1.f, e);
    for (int k = tid; k < K; k += kStageThreads) {
      const float v = load_act(a, dt, base + k) * up;
      const __half h = __float2half_rn(v);
      out[m * lda + k] = h;
      if (out_lo) out_lo[m * lda + k] = __float2half_rn(v - __half2float(h));
    }
    if (tid == 0) row_scale[m] = ldexpf(1.f, -e);
  }
}

// y[m][n] = sum over splits z (in order) of ws[z][m][n]; ws rows of pitch ldw.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int64_t stride, int64_t M, int N,
                                     int64_t ldw, float* __restrict__ y, int64_t ldy) {
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    const float* src = ws + m * ldw + n;
    float acc = src[0];
    for (int z = 1; z < splits; ++z) acc += src[z * stride];
    y[m * ldy + n] = acc;
  }
}

// ---------------------------------------------------------------- host side
using PFN_encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encode g_encode = nullptr;
std::once_flag g_encode_once;

int encoder(PFN_encode* out) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_encode>(fn);
  });
  if (!g_encode) return fail(MSQ_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  *out = g_encode;
  return MSQ_OK;
}

int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, void* base, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  PFN_encode enc;
  int rc = encoder(&enc);
  if (rc != MSQ_OK) return rc;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MSQ_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MSQ_OK;
}

// Tensor maps of one weight handle for one tile width: packed codes, scales, zero points.
struct WeightMaps {
  CUtensorMap p, s, z;
};

struct GemmState {
  WeightMaps m128;   // fp16 scales (the fast path)
  WeightMaps m128s;  // fp32 scales (the split path)
};

template <int TM, int BN, int ZPK, bool SPLIT>
int launch(cudaStream_t st, const CUtensorMap& tmA, const WeightMaps& wm, const GemmArgs& a, dim3 grid) {
  using PL = Plan<TM, BN, SPLIT>;
  static_assert(PL::kSmem <= 227 * 1024, "GEMM plan exceeds the 227 KB of shared memory a CTA may use");
  auto kern = gemm_tc_kernel<TM, BN, ZPK, SPLIT>;
  static ContextOnce configured;
  int rc = configured.run([&] {
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PL::kSmem),
                 "gemm smem attribute");
    return MSQ_OK;
  });
  if (rc != MSQ_OK) return rc;
  kern<<<grid, PL::kThreads, PL::kSmem, st>>>(tmA, wm.p, wm.s, wm.z, a);
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "gemm launch");
  return MSQ_OK;
}

template <int TM, int BN, bool SPLIT = false>
int launch_zp(cudaStream_t st, int zp_kind, const CUtensorMap& tmA, const WeightMaps& wm, const GemmArgs& a,
              dim3 grid) {
  switch (zp_kind) {
    case ZP_PACKED: return launch<TM, BN, ZP_PACKED, SPLIT>(st, tmA, wm, a, grid);
    case ZP_F32: return launch<TM, BN, ZP_F32, SPLIT>(st, tmA, wm, a, grid);
    default: return launch<TM, BN, ZP_NONE, SPLIT>(st, tmA, wm, a, grid);
  }
}

}  // namespace

namespace {

constexpr size_t kSplitWsMax = size_t(64) << 20;  // partial outputs of a k-split launch

// K-splits for a launch of `ctas` tiles: 1 when the tiles fill the SMs; otherwise the count
// (each split >= 8 k-stages, <= 32 splits, partial outputs <= kSplitWsMax) whose CTAs fill the
// last wave best, preferring fewer splits unless more fill it by over 2 %.
int choose_splits(int ctas, int sms, int ksteps, int64_t M, int64_t ldw) {
  if (ctas >= sms) return 1;
  auto fill = [&](int n) { return (double)n / (double)(((n + sms - 1) / sms) * sms); };
  int best_s = 1;
  double best = fill(ctas);
  for (int s = 2; s <= 32 && 8 * s <= ksteps; ++s) {
    if ((size_t)s * (size_t)M * (size_t)ldw * sizeof(float) > kSplitWsMax) break;
    const int kper = (ksteps + s - 1) / s;
    if ((ksteps + kper - 1) / kper != s) continue;  // every split must get a stage
    const double f = fill(ctas * s);
    if (f > best + 0.02) {
      best = f;
      best_s = s;
    }
  }
  return best_s;
}

// Builds the activation map over fp16 rows of stride lda and launches the tile kernel:
// 512 x 128 tiles (four accumulators sharing each dequantised weight tile) for M >= 512,
// 256 x 128 for M > 128, else 128 x 128. When the tiles leave SMs idle and `allow_split`,
// K is split across CTAs whose partial tiles go to stream-ordered scratch and are summed in a
// fixed order into Y (deterministic).
// operand_split: the split (hi/lo) GEMM; a_lo: A has lo rows after its M hi rows.
int launch_gemm(cudaStream_t st, const Weights& w, const WeightMaps& m128, const void* a16, int64_t lda,
                const float* row_scale, int64_t M, float* d_y, int64_t ldy, bool allow_split,
                bool operand_split = false, bool a_lo = false) {
  int tm = M > BM ? 2 : 1;
  if (!operand_split && M >= 4 * BM) {
    // Three or four accumulators per dequantised weight tile, chosen by whole waves of tiles:
    // four share each tile over more rows, three fit a 3-deep stage ring instead of 2. Measured
    // on configs[2] (N = 14336), a three-accumulator tile costs 0.71-0.74 of a four-accumulator
    // one (M = 2048: 834 against 736 TFLOP/s; M = 8192: 936 against 911; M = 512, one wave of
    // four against 1.5 of three: 720 against 535).
    const int64_t gxt = (w.n_rows + 127) / 128, sms = num_sms(w.device);
    const int64_t waves4 = (gxt * ((M + 4 * BM - 1) / (4 * BM)) + sms - 1) / sms;
    const int64_t waves3 = (gxt * ((M + 3 * BM - 1) / (3 * BM)) + sms - 1) / sms;
    tm = 0.72 * (double)waves3 < (double)waves4 ? 3 : 4;
  }
  const int rows = tm * BM;
  CUtensorMap tmA;
  int rc = make_map_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, const_cast<void*>(a16), (uint64_t)w.K,
                       (uint64_t)M * (a_lo ? 2 : 1), (uint64_t)lda * 2, BK, rows % 256 == 0 ? 256 : 128,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != MSQ_OK) return rc;
  GemmArgs g{};
  g.y = d_y;
  g.ldy = ldy;
  g.row_scale = row_scale;
  g.a_lo_row = a_lo ? (int)M : 0;
  g.M = (int)M;
  g.n_rows = w.n_rows;
  g.K = w.K;
  g.ksteps = (w.K + BK - 1) / BK;
  int sh = 0;
  while ((1 << sh) < w.block_size) ++sh;
  g.bs_shift = sh;
  const int gx = (w.n_rows + 127) / 128, gy = (int)((M + rows - 1) / rows);
  const int64_t ldw = (w.n_rows + 3) / 4 * 4;
  const int splits = allow_split ? choose_splits(gx * gy, num_sms(w.device), g.ksteps, M, ldw) : 1;
  g.kper = (g.ksteps + splits - 1) / splits;
  void* ws = nullptr;
  if (splits > 1) {
    rc = scratch_alloc(&ws, (size_t)splits * (size_t)M * (size_t)ldw * sizeof(float), st);
    if (rc != MSQ_OK) return rc;
    g.y = static_cast<float*>(ws);
    g.ldy = ldw;
    g.split_stride = M * ldw;
  }
  g.vec_store = (g.ldy % 4 == 0) && ((reinterpret_cast<uintptr_t>(g.y) & 15) == 0);
  const dim3 grid(gx, gy, splits);
  if (operand_split)
    rc = tm == 2 ? launch_zp<2, 128, true>(st, w.zp_kind, tmA, m128, g, grid)
                 : launch_zp<1, 128, true>(st, w.zp_kind, tmA, m128, g, grid);
  else
    rc = tm == 4   ? launch_zp<4, 128>(st, w.zp_kind, tmA, m128, g, grid)
         : tm == 3 ? launch_zp<3, 128>(st, w.zp_kind, tmA, m128, g, grid)
         : tm == 2 ? launch_zp<2, 128>(st, w.zp_kind, tmA, m128, g, grid)
                   : launch_zp<1, 128>(st, w.zp_kind, tmA, m128, g, grid);
  if (rc == MSQ_OK && splits > 1) {
    const int64_t total = M * w.n_rows;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 8 * (int64_t)num_sms(w.device));
    splitk_reduce_kernel<<<blocks, 256, 0, st>>>(static_cast<const float*>(ws), splits, g.split_stride, M, w.n_rows,
                                                 ldw, d_y, ldy);
    note_launch();
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_fail(e, "split-K reduce launch");
  }
  scratch_free(ws, st);
  if (rc == MSQ_OK) {
    static const char* names[2][2][4] = {
        {{"gemm_tc_m128_n128", "gemm_tc_m256_n128", "gemm_tc_m384_n128", "gemm_tc_m512_n128"},
         {"gemm_tc_m128_n128_splitk", "gemm_tc_m256_n128_splitk", "gemm_tc_m384_n128_splitk",
          "gemm_tc_m512_n128_splitk"}},
        {{"gemm_tc_x3_m128_n128", "gemm_tc_x3_m256_n128", "gemm_tc_x3_m384_n128", "gemm_tc_x3_m512_n128"},
         {"gemm_tc_x3_m128_n128_splitk", "gemm_tc_x3_m256_n128_splitk", "gemm_tc_x3_m384_n128_splitk",
          "gemm_tc_x3_m512_n128_splitk"}}};
    note_path(names[operand_split ? 1 : 0][splits > 1 ? 1 : 0][tm - 1]);
  }
  return rc;
}

// Codes [n_rows][KP/2] in boxes of 32 bytes x BN rows; scales [n_rows][sc_pitch] fp16 and zero
// points (packed [n_rows][zp_pitch] bytes or fp32 [n_rows][sc_pitch]) in 16-byte x BN boxes.
int make_maps(const Weights& w, int bn, WeightMaps* m, bool f32_scales = false) {
  int rc = make_map_2d(&m->p, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.nib, (uint64_t)w.nib_pitch, (uint64_t)w.n_rows,
                       (uint64_t)w.nib_pitch, BK / 2, bn, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == MSQ_OK && f32_scales)
    rc = make_map_2d(&m->s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.sc, (uint64_t)w.sc_pitch, (uint64_t)w.n_rows,
                     (uint64_t)w.sc_pitch * 4, 4, bn, CU_TENSOR_MAP_SWIZZLE_NONE);
  else if (rc == MSQ_OK)
    rc = make_map_2d(&m->s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w.sc16, (uint64_t)w.sc_pitch, (uint64_t)w.n_rows,
                     (uint64_t)w.sc_pitch * 2, 8, bn, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != MSQ_OK) return rc;
  if (w.zp_kind == ZP_PACKED)
    return make_map_2d(&m->z, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.zp4, (uint64_t)w.zp_pitch, (uint64_t)w.n_rows,
                       (uint64_t)w.zp_pitch, 16, bn, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (w.zp_kind == ZP_F32)
    return make_map_2d(&m->z, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.zpf, (uint64_t)w.sc_pitch, (uint64_t)w.n_rows,
                       (uint64_t)w.sc_pitch * 4, 4, bn, CU_TENSOR_MAP_SWIZZLE_NONE);
  m->z = m->s;  // not read without zero points
  return MSQ_OK;
}

int make_weight_maps(const Weights& w, WeightMaps* m128, bool f32_scales = false) {
  return make_maps(w, 128, m128, f32_scales);
}

// fp16 activations with 16-byte rows feed TMA directly; anything else is staged as fp16.
bool needs_staging(const Weights& w, const void* d_a, int a_dtype) {
  return a_dtype != MSQ_DT_F16 || (w.K % 8) != 0 || (reinterpret_cast<uintptr_t>(d_a) & 15) != 0;
}

// Staged A: fp16 rows [M][staged_lda] (16-byte rows for TMA) -- for the split GEMM the hi rows
// and then the lo rows, [2M][staged_lda] -- then M fp32 row scales at a 256-byte-aligned offset.
int64_t staged_lda(const Weights& w) { return (w.K + 7) / 8 * 8; }
size_t staged_scale_offset(const Weights& w, int64_t M, int parts = 1) {
  return (sizeof(__half) * (size_t)parts * (size_t)M * (size_t)staged_lda(w) + 255) / 256 * 256;
}
size_t staging_bytes(const Weights& w, const void* d_a, int a_dtype, int64_t M, int parts) {
  if (M <= 0 || !needs_staging(w, d_a, a_dtype)) return 0;
  return staged_scale_offset(w, M, parts) + sizeof(float) * (size_t)M;
}

int stage_rows(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M, void* staging,
               const float** row_scale, int parts = 1) {
  float* rs = reinterpret_cast<float*>(static_cast<uint8_t*>(staging) + staged_scale_offset(w, M, parts));
  const int64_t blocks = std::min<int64_t>(M, 16 * (int64_t)num_sms(w.device));
  __half* hi = static_cast<__half*>(staging);
  to_half_rows_kernel<<<(unsigned)blocks, kStageThreads, 0, st>>>(d_a, a_dtype, M, w.K, hi, staged_lda(w), rs,
                                                                  parts == 2 ? hi + M * staged_lda(w) : nullptr);
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "staging launch");
  *row_scale = rs;
  return MSQ_OK;
}

}  // namespace

int run_gemm(cudaStream_t st, Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y, int64_t ldy,
             bool operand_split) {
  if (!w.fast4) return fail(MSQ_E_UNSUPPORTED, "GEMM path needs bits=4 and a power-of-two block_size >= 32");
  if (M <= 0) return MSQ_OK;
  if (M > 0x7fffffff) return fail(MSQ_E_INVALID, "GEMM: M too large");
  {
    const int lrc = ensure_gemm_layout(st, w);
    if (lrc != MSQ_OK) return lrc;
  }
  // The tensor maps are built once per handle (under the handle's own lock, so first calls on
  // different handles do not wait for each other) and only read afterwards.
  GemmState* gs = static_cast<GemmState*>(w.gemm_state.load(std::memory_order_acquire));
  if (!gs) {
    std::lock_guard<std::mutex> lk(w.state_mu);
    gs = static_cast<GemmState*>(w.gemm_state.load(std::memory_order_relaxed));
    if (!gs) {
      gs = new GemmState();
      int rc = make_weight_maps(w, &gs->m128);
      if (rc == MSQ_OK) rc = make_weight_maps(w, &gs->m128s, true);
      if (rc != MSQ_OK) {
        delete gs;
        return rc;
      }
      w.gemm_state.store(gs, std::memory_order_release);
    }
  }
  const void* a16 = d_a;
  int64_t lda = w.K;
  void* scratch = nullptr;
  const float* row_scale = nullptr;
  const int parts = operand_split ? 2 : 1;
  const size_t need = staging_bytes(w, d_a, a_dtype, M, parts);
  if (need) {
    const int arc = scratch_alloc(&scratch, need, st);
    if (arc != MSQ_OK) return arc;
    lda = staged_lda(w);
    const int src = stage_rows(st, w, d_a, a_dtype, M, scratch, &row_scale, parts);
    if (src != MSQ_OK) {
      scratch_free(scratch, st);
      return src;
    }
    a16 = scratch;
  }
  const int rc = launch_gemm(st, w, operand_split ? gs->m128s : gs->m128, a16, lda, row_scale, M, d_y, ldy, true,
                             operand_split, operand_split && need != 0);
  scratch_free(scratch, st);
  return rc;
}

size_t gemm_staging_bytes(const Weights& w, const void* d_a, int a_dtype, int64_t M) {
  return staging_bytes(w, d_a, a_dtype, M, 1);
}

int run_gemm_staged(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y,
                    int64_t ldy, void* staging, size_t staging_bytes) {
  if (!w.fast4) return fail(MSQ_E_UNSUPPORTED, "GEMM path needs bits=4 and a power-of-two block_size >= 32");
  if (!w.gemm_layout.load(std::memory_order_acquire))
    return fail(MSQ_E_UNSUPPORTED,
                "the handle was packed with MSQ_PACK_LAZY_GEMM and has no GEMM layout yet (it is built, with an "
                "allocation, by the first msq_matmul that takes the GEMM path)");
  if (M <= 0) return MSQ_OK;
  if (M > 0x7fffffff) return fail(MSQ_E_INVALID, "GEMM: M too large");
  WeightMaps m128;
  int rc = make_weight_maps(w, &m128);
  if (rc != MSQ_OK) return rc;
  const void* a16 = d_a;
  int64_t lda = w.K;
  const float* row_scale = nullptr;
  const size_t need = gemm_staging_bytes(w, d_a, a_dtype, M);
  if (need) {
    if (need > staging_bytes || !staging)
      return fail(MSQ_E_INVALID, "GEMM staging needs %zu bytes; %zu available", need, staging_bytes);
    lda = staged_lda(w);
    rc = stage_rows(st, w, d_a, a_dtype, M, staging, &row_scale);
    if (rc != MSQ_OK) return rc;
    a16 = staging;
  }
  return launch_gemm(st, w, m128, a16, lda, row_scale, M, d_y, ldy, false);  // no scratch for k-splits here
}

void release_gemm_state(Weights& w) {
  delete static_cast<GemmState*>(w.gemm_state.exchange(nullptr));
}

int set_wait_budget_gemm(unsigned long long ns) {
  MSQ_CUDA_TRY(cudaMemcpyToSymbol(ptx::g_wait_budget_ns, &ns, sizeof ns), "set GEMM wait budget");
  return MSQ_OK;
}

int read_gemm_errors(cudaStream_t st, int* flags) {
  int v = 0;
  MSQ_CUDA_TRY(cudaMemcpyFromSymbolAsync(&v, g_gemm_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st),
               "read gemm error word");
  MSQ_CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
  if (v) {
    const int zero = 0;
    MSQ_CUDA_TRY(cudaMemcpyToSymbolAsync(g_gemm_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st),
                 "clear gemm error word");
    MSQ_CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
  }
  *flags = v;
  return MSQ_OK;
}

}  // namespace msq
