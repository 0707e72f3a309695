// Batched decode GEMV for MatMulNBits on the 5th-generation tensor cores (tcgen05 kind::i8 +
// TMEM), exact integer arithmetic, for 5 <= M <= 32 rows of A at block_size 128.
//
// The decode GEMV's exactness scheme (msq_gemv_mma.cu) with the tensor core doing all of the
// multiply-adds: each quantisation block b of each row m of A becomes a 24-bit fixed-point
// vector a_int = rint(a * 2^sigma) (sigma from the block's own maximum) split into three
// balanced int8 digits, a_int = d0 + 256 d1 + 65536 d2, and S = sum a_int. A small kernel writes
// the digits of all rows once, as 3 * MP rows of s8 (the MMA's B operand, MP = 16 or 32), with
// 2^-sigma and S per (block, row). One CTA then takes 256 weight rows (two M = 128 MMA tiles
// sharing the digit operand) and streams one 128-k block per stage:
//   TMA warp   the stage's packed codes (256 rows x 64 bytes, 64-byte swizzle), a 16-byte
//              column of fp32 scales and of zero points per row, the block's digit rows
//              (128-byte swizzle) and its 2^-sigma / S row;
//   work warps one thread per weight row: the codes become u8 (q) in the K-major 128-byte-
//              swizzled layout the tensor core reads (two integer ops per 8 codes; the byte
//              order inside each 8-k group follows the nibble plane and the digits use the
//              same order), then, one stage behind, the block's exact dots
//              D_i[n, m] = sum_k q[n, k] d_i[m, k] from TMEM and
//                  y[m, n] += s[n, b] 2^-sigma (D_0 + 256 D_1 + 65536 D_2 - zp[n, b] S[m, b]);
//   MMA warp   per stage 2 x 4 tcgen05.mma.kind::i8 (M = 128, N = 3 MP, K = 32) into one of two
//              TMEM accumulator buffers, a fresh accumulation per block.
// So every weight is read from HBM once for all M rows, and the CUDA cores do two integer ops
// per 8 weights plus a few fp32 ops per (weight row, A row, block). The only roundings are A's
// rounding to 2^-24 of its block maximum and the fp32 block combination, as in the decode
// GEMV (parity bar rel-L2 <= 1e-5 against the fp32 reference, MatMulNBitsKernel.cs:236-261).
// Rows of A holding inf or NaN get their exact fp32 terms added at the end, as there.
#include "msq_internal.cuh"
#include "msq_ptx.cuh"

#include <cuda.h>

#include <algorithm>
#include <mutex>

namespace msq {
namespace {

constexpr int TBN = 256;  // weight rows per CTA
constexpr int TBK = 128;  // k per stage = block_size
// unpack + epilogue warps: warp w takes TMEM lane quarter w & 3 of MMA tile (w >> 2) & 1 (its
// 32 weight rows), and half h = w >> 3 of the A rows (MP / 2 of them) and of each row's 128 k
constexpr int kWork = 16;
constexpr int kTmaWarpTc = kWork;
constexpr int kMmaWarpTc = kWork + 1;
constexpr int kThreadsTc = (kWork + 2) * 32;

__device__ int g_tc_err;

// Inverse of the nibble plane's in-group order (kSlotK in msq_repack.cu) as the unpack leaves
// it: the u8 byte p of an 8-k group holds k offset {0, 4, 1, 5, 2, 6, 3, 7}[p], so the digit of
// k offset o goes to byte kDigPos[o].
__constant__ int kDigPos[8] = {0, 2, 4, 6, 1, 3, 5, 7};

template <int MP>
struct TcPlan {
  static constexpr int NC = 3 * MP;               // digit rows: MMA N
  // TMA stage ring: what the producer loads per 128-k block, released by the MMA's commit
  static constexpr int kDig = NC * TBK;           // 6 / 12 KB, SW128
  static constexpr int kCodes = TBN * TBK / 2;    // 16 KB, SW64
  static constexpr int kSc = TBN * 16;            // 4 fp32 scales per row (the 16-byte column)
  static constexpr int kZp = TBN * 16;
  static constexpr int kOffDig = 0;
  static constexpr int kOffCodes = kOffDig + kDig;
  static constexpr int kOffSc = kOffCodes + kCodes;
  static constexpr int kOffZp = kOffSc + kSc;
  static constexpr int kStage = (kOffZp + kZp + 1023) / 1024 * 1024;
  // unpacked u8 weights: two slots of two 128-row SW128 tiles (a slot is free again once the
  // work warps have seen the accumulator of the stage that read it)
  static constexpr int kU8 = TBN * TBK;
  // 2^-sigma / S rows: their own ring, released by the epilogue
  static constexpr int kMetaW = 2 * MP + 4;  // floats per block: 2^-sigma [MP], S [MP], bad-row mask, pad
  static constexpr int kMeta = kMetaW * 4;
  static constexpr int kMetaSlots = 8;
  static constexpr int kStages = MP == 16 ? 5 : 4;  // what fits in 227 KB
  static constexpr int kOffU8 = kStages * kStage;
  static constexpr int kOffMeta = kOffU8 + 2 * kU8;
  static constexpr int kOffBar = kOffMeta + kMetaSlots * kMeta;
  static constexpr int kBarBytes = (2 * kStages + 2 * kMetaSlots + 4 + 2) * 8 + 16;
  static constexpr int kSmem = kOffBar + kBarBytes + 1024;  // + alignment slack
  static constexpr int kTmemCols = 4 * NC <= 256 ? 256 : 512;  // 2 buffers x 2 tiles x NC
};

struct TcArgs {
  float* y;          // Y, or the partial outputs of the k-splits
  int64_t ldy;
  int64_t split_stride;  // elements between the partial outputs of consecutive k-splits
  int M, n_rows, K, nblk, kper;
  int zp_kind;
  const float* meta;   // [nblk][2 MP + 4]: 2^-sigma, S (as fp32), the mask of A rows whose
                       // block holds inf / NaN
  // the slow path of rows with inf / NaN
  const void* a;
  int a_dtype;
  const uint8_t* nib;
  int64_t nib_pitch;
  const float* sc;
  int64_t sc_pitch;
  const uint8_t* zp4;
  int64_t zp_pitch;
  const float* zpf;
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (*abort_flag) return false;
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait_sleep(bar, parity)) return true;
    if ((i & 7u) == 0) {
      if (*abort_flag) return false;
      if (ptx::globaltimer() - t0 > budget) {
        *abort_flag = 1;
        atomicCAS(&g_tc_err, 0, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ uint32_t biased24(float x, float sc) {
  return __float_as_uint(fmaf(x, sc, 12582912.0f)) - (0x4B400000u - 0x808080u);
}

// One CTA per 128-k block b, one warp per A row m < MP: 2^-sigma, S and the three digit rows of
// the block; rows m >= M and k >= K give zero digits. Non-finite a gets digit 0 and sets bit m
// of the block's mask (the GEMV then adds that row's exact fp32 terms).
template <int MP>
__global__ void __launch_bounds__(MP * 32) tc_digits_kernel(const void* __restrict__ a, int dt, int M, int K,
                                                            int64_t kpd, int8_t* __restrict__ dig,
                                                            float* __restrict__ meta) {
  __shared__ uint32_t mask;
  // the GEMV (launched with programmatic serialization) may start its prologue and weight loads
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int m = threadIdx.x >> 5, lane = threadIdx.x & 31, b = blockIdx.x;
  if (threadIdx.x == 0) mask = 0u;
  __syncthreads();
  float v[4];
  bool bad = false;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = b * TBK + 4 * lane + j;
    float x = (m < M && k < K) ? load_act(a, dt, (int64_t)m * K + k) : 0.f;
    if (!(fabsf(x) <= 3.402823466e38f)) {
      bad = true;
      x = 0.f;
    }
    v[j] = x;
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(&mask, 1u << m);
  uint32_t ub = max(max(__float_as_uint(fabsf(v[0])), __float_as_uint(fabsf(v[1]))),
                    max(__float_as_uint(fabsf(v[2])), __float_as_uint(fabsf(v[3]))));
  ub = __reduce_max_sync(0xffffffffu, ub);  // non-negative floats order as their bits
  const float bmax = __uint_as_float(ub);
  int e = 0;
  {
    const int be = (int)((ub >> 23) & 0xFF);
    if (bmax > 0.f) e = be == 0 ? -126 : be - 126;  // frexp exponent of a finite positive bmax
  }
  const int sh = max(-120, min(120, 22 - e));
  const float up = __int_as_float((sh + 127) << 23);
  int sum = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t u = biased24(v[j], up);  // a_int + 0x808080: digit i + 128 in byte i
    const int k = b * TBK + 4 * lane + j;
    const int64_t col = (int64_t)(k & ~7) + kDigPos[k & 7];
#pragma unroll
    for (int d = 0; d < 3; ++d) dig[(int64_t)(d * MP + m) * kpd + col] = (int8_t)((int)((u >> (8 * d)) & 0xFF) - 128);
    sum += (int)(u - 0x808080u);
  }
  sum = (int)__reduce_add_sync(0xffffffffu, (uint32_t)sum);
  float* mb = meta + (int64_t)b * (2 * MP + 4);
  if (lane == 0) {
    mb[m] = __int_as_float((-sh + 127) << 23);
    mb[MP + m] = (float)sum;  // |sum| < 2^29: the same rounding as converting it in the GEMV
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    reinterpret_cast<uint32_t*>(mb)[2 * MP] = mask;
    mb[2 * MP + 1] = mb[2 * MP + 2] = mb[2 * MP + 3] = 0.f;
  }
}

// W[row, k] = (q - zp) * s in fp32 from the GEMM layout planes.
__device__ float plane_weight(const TcArgs& p, int64_t row, int k) {
  const uint32_t word = reinterpret_cast<const uint32_t*>(p.nib + row * p.nib_pitch)[k >> 3];
  const int o = k & 7;
  // nibble j of a word holds k offset {0, 2, 4, 6, 1, 3, 5, 7}[j]
  const int j = (o & 1) ? 4 + (o >> 1) : (o >> 1);
  const int q = (int)((word >> (4 * j)) & 0xF);
  const int b = k / TBK;
  const float s = p.sc[row * p.sc_pitch + b];
  float z = 8.f;
  if (p.zp_kind == ZP_PACKED) z = (float)((p.zp4[row * p.zp_pitch + (b >> 1)] >> (4 * (b & 1))) & 0xF);
  else if (p.zp_kind == ZP_F32) z = p.zpf[row * p.sc_pitch + b];
  return ((float)q - z) * s;
}

template <int MP, int ZPK>
__global__ void __launch_bounds__(kThreadsTc, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmS,
                   const __grid_constant__ CUtensorMap tmZ, const __grid_constant__ CUtensorMap tmD,
                   const TcArgs p) {
  using PL = TcPlan<MP>;
  constexpr int S = PL::kStages;
  constexpr int MS = PL::kMetaSlots;
  constexpr int NC = PL::NC;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PL::kOffBar);  // [S] TMA stage landed
  uint64_t* empty = full + S;        // [S] the MMA is done with the stage
  uint64_t* mfull = empty + S;       // [MS] meta row landed
  uint64_t* mempty = mfull + MS;     // [MS] every work warp's epilogue is done with it
  uint64_t* wready = mempty + MS;    // [2] u8 slot written by every work warp
  uint64_t* accfull = wready + 2;    // [2] accumulator buffer complete
  uint64_t* accempty = accfull + 2;  // [2] accumulator buffer read by every work warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TBN;
  const int kb = (int)blockIdx.y * p.kper;
  const int nk = min(p.nblk, kb + p.kper) - kb;

  if (threadIdx.x == 0) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the split-K sum may launch
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < MS; ++j) {
      ptx::mbar_init(&mfull[j], 1);
      ptx::mbar_init(&mempty[j], kWork);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&wready[b], kWork);
      ptx::mbar_init(&accfull[b], 1);
      ptx::mbar_init(&accempty[b], kWork);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kMmaWarpTc) {
    ptx::tmem_alloc(tmem_slot, PL::kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == kTmaWarpTc && lane == 0) {
    ptx::prefetch_tmap(&tmC);
    ptx::prefetch_tmap(&tmS);
    if (ZPK != ZP_NONE) ptx::prefetch_tmap(&tmZ);
    ptx::prefetch_tmap(&tmD);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarpTc) {
    if (lane == 0) {
      // The weights are settled before the call; the digits and meta rows come from the digits
      // kernel just before this one. So the first stages' weight side is loaded before the
      // programmatic-dependency wait, and everything the digits kernel wrote after it.
      auto load_weights = [&](int i) {
        const int s = i % S, b = kb + i;
        uint8_t* st = smem + s * PL::kStage;
        ptx::mbar_arrive_expect_tx(&full[s], PL::kCodes + PL::kSc + (ZPK != ZP_NONE ? PL::kZp : 0) + PL::kDig);
        ptx::tma_load_2d(st + PL::kOffCodes, &tmC, &full[s], b * (TBK / 2), n0);
        ptx::tma_load_2d(st + PL::kOffSc, &tmS, &full[s], b & ~3, n0);
        if (ZPK == ZP_PACKED) ptx::tma_load_2d(st + PL::kOffZp, &tmZ, &full[s], (b >> 1) & ~15, n0);
        else if (ZPK == ZP_F32) ptx::tma_load_2d(st + PL::kOffZp, &tmZ, &full[s], b & ~3, n0);
      };
      auto load_digits = [&](int i) {
        const int s = i % S, j = i % MS, b = kb + i;
        ptx::tma_load_2d(smem + s * PL::kStage + PL::kOffDig, &tmD, &full[s], b * TBK, 0);
        ptx::mbar_arrive_expect_tx(&mfull[j], PL::kMeta);
        ptx::bulk_g2s(smem + PL::kOffMeta + j * PL::kMeta, p.meta + (int64_t)b * PL::kMetaW, PL::kMeta, &mfull[j]);
      };
      const int pre = min(nk, S);
      for (int i = 0; i < pre; ++i) load_weights(i);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int i = 0; i < pre; ++i) load_digits(i);
      int issued = pre;
      for (int i = pre; i < nk; ++i) {
        const int s = i % S, j = i % MS;
        if (!tc_wait(&empty[s], ((i / S) - 1) & 1, abort_flag, ptx::kErrTimeoutEmpty)) break;
        if (i >= MS && !tc_wait(&mempty[j], ((i / MS) - 1) & 1, abort_flag, ptx::kErrTimeoutEmpty)) break;
        load_weights(i);
        load_digits(i);
        ++issued;
      }
      // copies in flight must land before exit
      const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
      bool timed_out = false;
      for (int s = 0; s < S && s < issued; ++s) {
        const int last = s + (issued - 1 - s) / S * S;
        while (!timed_out && !ptx::mbar_try_wait(&full[s], (last / S) & 1))
          if (ptx::globaltimer() - t0 > budget) timed_out = true;
      }
      for (int j = 0; j < MS && j < issued; ++j) {
        const int last = j + (issued - 1 - j) / MS * MS;
        while (!timed_out && !ptx::mbar_try_wait(&mfull[j], (last / MS) & 1))
          if (ptx::globaltimer() - t0 > budget) timed_out = true;
      }
      if (timed_out) atomicCAS(&g_tc_err, 0, ptx::kErrTimeoutDrain);
    }
  } else if (warp == kMmaWarpTc) {
    if (lane == 0) {
      // kind::i8: D s32 (2), A u8 (0), B s8 (1), both K-major; N = NC, M = 128
      constexpr uint32_t idesc = (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(NC >> 3) << 17) |
                                 ((uint32_t)(128 >> 4) << 24);
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % S;
        const int buf = i & 1;
        ok = tc_wait(&full[s], (i / S) & 1, abort_flag, ptx::kErrTimeoutFull) &&
             tc_wait(&wready[buf], (i >> 1) & 1, abort_flag, ptx::kErrTimeoutFull) &&
             (i < 2 || tc_wait(&accempty[buf], ((i >> 1) - 1) & 1, abort_flag, ptx::kErrTimeoutFull));
        if (!ok) break;
        ptx::tc_fence_after();
        const uint64_t bd = sw128_desc(ptx::smem_u32(smem + s * PL::kStage + PL::kOffDig));
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint64_t ad = sw128_desc(ptx::smem_u32(smem + PL::kOffU8 + buf * PL::kU8 + t * (TBN / 2) * TBK));
#pragma unroll
          for (int j = 0; j < TBK / 32; ++j)
            mma_i8(tmem + (uint32_t)(buf * 2 * NC + t * NC), ad + 2 * j, bd + 2 * j, idesc, j != 0);
        }
        ptx::mma_commit(&empty[s]);
        ptx::mma_commit(&accfull[buf]);
      }
      // every MMA must be done before exit (TMEM and shared memory are released then)
      if (nk > 0) {
        const int last = nk - 1, buf = last & 1;
        const unsigned long long t0 = ptx::globaltimer(), budget = ptx::wait_budget_ns();
        while (!ptx::mbar_try_wait(&accfull[buf], (last >> 1) & 1)) {
          if (ptx::globaltimer() - t0 > budget) {
            atomicCAS(&g_tc_err, 0, ptx::kErrTimeoutMma);
            break;
          }
        }
      }
    }
  } else {
    // ---------------- work warps: weight row R of the CTA (tile t, TMEM lane r), half h
    constexpr int MH = MP / 2;
    const int t = (warp >> 2) & 1, q = warp & 3, h = warp >> 3;
    const int r = q * 32 + lane;
    const int R = t * 128 + r;
    const int64_t row = (int64_t)n0 + R;
    float y[MH];
#pragma unroll
    for (int m = 0; m < MH; ++m) y[m] = 0.f;
    uint32_t bad = 0;  // A rows whose blocks in this k range hold inf / NaN
    float s_cur = 0.f, z_cur = 0.f, s_nxt = 0.f, z_nxt = 0.f;
    // unpack half h of stage i into u8 slot i & 1: u8 codes of row R in the SW128 layout, and
    // the row's scale / zero point. The slot was last read by the MMA of stage i - 2, whose
    // accumulator this warp has already waited for.
    auto unpack = [&](int i, float& s_out, float& z_out) -> bool {
      const int s = i % S;
      const bool ok = __all_sync(0xffffffffu, tc_wait(&full[s], (i / S) & 1, abort_flag, ptx::kErrTimeoutFull));
      if (ok) {
        const uint8_t* st = smem + s * PL::kStage;
        const int b = kb + i;
        s_out = reinterpret_cast<const float*>(st + PL::kOffSc)[R * 4 + (b & 3)];
        if (ZPK == ZP_PACKED) {
          const uint8_t zb = st[PL::kOffZp + R * 16 + ((b >> 1) & 15)];
          z_out = (float)((zb >> (4 * (b & 1))) & 0xF);
        } else if (ZPK == ZP_F32) {
          z_out = reinterpret_cast<const float*>(st + PL::kOffZp)[R * 4 + (b & 3)];
        } else {
          z_out = 8.f;
        }
        // codes: 64-byte rows, 64-byte swizzle: chunk c of row R at ((c ^ ((R >> 1) & 3)) << 4)
        const uint8_t* crow = st + PL::kOffCodes + R * 64;
        uint8_t* urow = smem + PL::kOffU8 + (i & 1) * PL::kU8 + t * (TBN / 2) * TBK + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * h + cc;
          const uint4 w = *reinterpret_cast<const uint4*>(crow + ((c ^ ((R >> 1) & 3)) << 4));
          uint4 o0, o1;
          o0.x = w.x & 0x0F0F0F0Fu;
          o0.y = (w.x >> 4) & 0x0F0F0F0Fu;
          o0.z = w.y & 0x0F0F0F0Fu;
          o0.w = (w.y >> 4) & 0x0F0F0F0Fu;
          o1.x = w.z & 0x0F0F0F0Fu;
          o1.y = (w.z >> 4) & 0x0F0F0F0Fu;
          o1.z = w.w & 0x0F0F0F0Fu;
          o1.w = (w.w >> 4) & 0x0F0F0F0Fu;
          *reinterpret_cast<uint4*>(urow + (((2 * c) ^ (r & 7)) << 4)) = o0;
          *reinterpret_cast<uint4*>(urow + (((2 * c + 1) ^ (r & 7)) << 4)) = o1;
        }
      }
      ptx::fence_proxy_async_smem();  // generic-proxy stores -> the tensor core's reads
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&wready[i & 1]);
      return ok;
    };
    bool ok = nk > 0 ? unpack(0, s_cur, z_cur) : true;
    for (int i = 0; i < nk && ok; ++i) {
      if (i + 1 < nk) ok = unpack(i + 1, s_nxt, z_nxt);
      const int buf = i & 1, j = i % MS;
      const bool acc_ok =
          __all_sync(0xffffffffu, tc_wait(&accfull[buf], (i >> 1) & 1, abort_flag, ptx::kErrTimeoutMma) &&
                                      tc_wait(&mfull[j], (i / MS) & 1, abort_flag, ptx::kErrTimeoutFull));
      if (!acc_ok) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const float* mrow = reinterpret_cast<const float*>(smem + PL::kOffMeta + j * PL::kMeta);
      bad |= reinterpret_cast<const uint32_t*>(mrow)[2 * MP];
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 2 * NC + t * NC + h * MH);
      const int mlim = p.M - h * MH;  // A rows of this half that exist (warp-uniform)
#pragma unroll
      for (int c = 0; c < MH / 8; ++c) {
        if (8 * c >= mlim) break;
        uint32_t d0[8], d1[8], d2[8];
        tmem_ld_x8(base + 0 * MP + 8 * c, d0);
        tmem_ld_x8(base + 1 * MP + 8 * c, d1);
        tmem_ld_x8(base + 2 * MP + 8 * c, d2);
        ptx::tmem_ld_wait();
        const float4* g4 = reinterpret_cast<const float4*>(mrow + h * MH + 8 * c);
        const float4* s4 = reinterpret_cast<const float4*>(mrow + MP + h * MH + 8 * c);
        const float4 ga = g4[0], gb = g4[1], sa = s4[0], sb = s4[1];
        const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const float lo = (float)((int)d0[jj] + 256 * (int)d1[jj]);
          float f = fmaf(65536.f, (float)(int)d2[jj], lo);
          f = fmaf(-z_cur, sv[jj], f);
          y[8 * c + jj] = fmaf(s_cur * gv[jj], f, y[8 * c + jj]);
        }
      }
      // the accumulator buffer may be reused once every warp has read what it needs of it
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&accempty[buf]);
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&mempty[j]);  // the meta slot may be refilled
      s_cur = s_nxt;
      z_cur = z_nxt;
    }
    (void)ok;
    // ---- store this CTA's outputs (or partials) for its k range
    if (row < p.n_rows) {
      float* yo = p.y + (int64_t)blockIdx.y * p.split_stride + row;
#pragma unroll
      for (int jj = 0; jj < MH; ++jj) {
        const int m = h * MH + jj;
        if (m < p.M) {
          float v = y[jj];
          if ((bad >> m) & 1u) {  // inf / NaN in A row m: add its exact fp32 terms over this k range
            float tsum = 0.f;
            const int k0 = kb * TBK, k1 = min(p.K, (kb + nk) * TBK);
            for (int k = k0; k < k1; ++k) {
              const float a = load_act(p.a, p.a_dtype, (int64_t)m * p.K + k);
              if (!(fabsf(a) <= 3.402823466e38f)) tsum += a * plane_weight(p, row, k);
            }
            v += tsum;
          }
          yo[(int64_t)m * p.ldy] = v;
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarpTc) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, PL::kTmemCols);
  }
}

// y[m][n] = sum over splits z (in order) of ws[z][m][n].
__global__ void tc_reduce_kernel(const float* __restrict__ ws, int splits, int64_t stride, int M, int N,
                                 float* __restrict__ y, int64_t ldy) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched early: the partials must be complete
  const int64_t total = (int64_t)M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    const float* src = ws + m * N + n;
    float acc = src[0];
    for (int z = 1; z < splits; ++z) acc += src[z * stride];
    y[m * ldy + n] = acc;
  }
}

// ---------------------------------------------------------------- host side
using PFN_encode_tc = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encode_tc g_enc_tc = nullptr;
std::once_flag g_enc_tc_once;

int map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
           uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  std::call_once(g_enc_tc_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_enc_tc = reinterpret_cast<PFN_encode_tc>(fn);
  });
  if (!g_enc_tc) return fail(MSQ_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_enc_tc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MSQ_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MSQ_OK;
}

template <int MP, int ZPK>
int launch_tc(cudaStream_t st, const CUtensorMap& c, const CUtensorMap& s, const CUtensorMap& z,
              const CUtensorMap& d, const TcArgs& a, dim3 grid) {
  using PL = TcPlan<MP>;
  static_assert(PL::kSmem <= 227 * 1024, "plan exceeds the 227 KB of shared memory a CTA may use");
  auto kern = gemv_tc_kernel<MP, ZPK>;
  static ContextOnce configured;
  int rc = configured.run([&] {
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PL::kSmem),
                 "tc gemv smem attribute");
    return MSQ_OK;
  });
  if (rc != MSQ_OK) return rc;
  // programmatic serialization: the prologue and the first stages' weight loads overlap the
  // digits kernel, which releases this grid early (the producer waits before reading digits)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreadsTc);
  cfg.dynamicSmemBytes = PL::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MSQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, c, s, z, d, a), "tc gemv launch");
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "tc gemv launch");
  return MSQ_OK;
}

template <int MP>
int launch_tc_zp(cudaStream_t st, int zpk, const CUtensorMap& c, const CUtensorMap& s, const CUtensorMap& z,
                 const CUtensorMap& d, const TcArgs& a, dim3 grid) {
  switch (zpk) {
    case ZP_PACKED: return launch_tc<MP, ZP_PACKED>(st, c, s, z, d, a, grid);
    case ZP_F32: return launch_tc<MP, ZP_F32>(st, c, s, z, d, a, grid);
    default: return launch_tc<MP, ZP_NONE>(st, c, s, z, d, a, grid);
  }
}

// k-splits for `tiles` CTAs over `ks` stages: the count that minimises the stages of the
// busiest SM, plus the partial outputs' extra traffic in stage units; 1 when nothing gains.
int tc_splits(int tiles, int sms, int ks, int M, int n_rows) {
  int best = 1;
  double best_cost = 1e30;
  const double stage_bytes = 256.0 * 128 / 2;  // codes of one CTA stage
  for (int s = 1; s <= 16 && s <= ks; ++s) {
    const int kper = (ks + s - 1) / s;
    if ((ks + kper - 1) / kper != s) continue;
    const int waves = (tiles * s + sms - 1) / sms;
    const double partial = s > 1 ? 2.0 * s * M * (double)n_rows * 4 / sms / stage_bytes : 0.0;
    const double cost = (double)waves * kper + partial;
    if (cost < best_cost * 0.98) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

}  // namespace

int run_gemv_tc(cudaStream_t st, Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y, int64_t ldy) {
  if (!w.fast4 || w.block_size != TBK)
    return fail(MSQ_E_UNSUPPORTED, "tensor-core decode GEMV needs bits=4 and block_size 128");
  if (M < 1 || M > 32) return fail(MSQ_E_UNSUPPORTED, "tensor-core decode GEMV takes 1..32 rows of A");
  {
    const int lrc = ensure_gemm_layout(st, w);
    if (lrc != MSQ_OK) return lrc;
  }
  const int MP = M <= 16 ? 16 : 32;
  const int nblk = (w.K + TBK - 1) / TBK;
  const int64_t kpd = (int64_t)nblk * TBK;
  const int tiles = (w.n_rows + TBN - 1) / TBN;
  const int sms = num_sms(w.device);
  const int splits = tc_splits(tiles, sms, nblk, (int)M, w.n_rows);
  const int kper = (nblk + splits - 1) / splits;
  // scratch: digits [3 MP][kpd] s8, meta [nblk][2 MP], then the partials
  const size_t dig_bytes = (size_t)3 * MP * kpd;
  const size_t meta_off = (dig_bytes + 255) / 256 * 256;
  const size_t ws_off = meta_off + ((size_t)nblk * (2 * MP + 4) * 4 + 255) / 256 * 256;
  const int64_t split_stride = (int64_t)M * w.n_rows;
  const size_t total = ws_off + (splits > 1 ? (size_t)splits * split_stride * 4 : 0);
  void* scratch = nullptr;
  int rc = scratch_alloc(&scratch, total, st);
  if (rc != MSQ_OK) return rc;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  int8_t* dig = reinterpret_cast<int8_t*>(base);
  float* meta = reinterpret_cast<float*>(base + meta_off);
  float* ws = reinterpret_cast<float*>(base + ws_off);
  auto done = [&](int code) {
    scratch_free(scratch, st);
    return code;
  };
  {
    if (MP == 16)
      tc_digits_kernel<16><<<nblk, 16 * 32, 0, st>>>(d_a, a_dtype, (int)M, w.K, kpd, dig, meta);
    else
      tc_digits_kernel<32><<<nblk, 32 * 32, 0, st>>>(d_a, a_dtype, (int)M, w.K, kpd, dig, meta);
    note_launch();
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return done(cuda_fail(e, "tc digits launch"));
  }
  CUtensorMap mc, ms, mz, md;
  rc = map_2d(&mc, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.nib, (uint64_t)w.nib_pitch, (uint64_t)w.n_rows,
              (uint64_t)w.nib_pitch, TBK / 2, TBN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc == MSQ_OK)
    rc = map_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.sc, (uint64_t)w.sc_pitch, (uint64_t)w.n_rows,
                (uint64_t)w.sc_pitch * 4, 4, TBN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == MSQ_OK) {
    if (w.zp_kind == ZP_PACKED)
      rc = map_2d(&mz, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.zp4, (uint64_t)w.zp_pitch, (uint64_t)w.n_rows,
                  (uint64_t)w.zp_pitch, 16, TBN, CU_TENSOR_MAP_SWIZZLE_NONE);
    else if (w.zp_kind == ZP_F32)
      rc = map_2d(&mz, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.zpf, (uint64_t)w.sc_pitch, (uint64_t)w.n_rows,
                  (uint64_t)w.sc_pitch * 4, 4, TBN, CU_TENSOR_MAP_SWIZZLE_NONE);
    else
      mz = ms;  // not read without zero points
  }
  if (rc == MSQ_OK)
    rc = map_2d(&md, CU_TENSOR_MAP_DATA_TYPE_UINT8, dig, (uint64_t)kpd, (uint64_t)(3 * MP), (uint64_t)kpd, TBK,
                3 * MP, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != MSQ_OK) return done(rc);
  TcArgs a{};
  a.y = splits > 1 ? ws : d_y;
  a.ldy = splits > 1 ? w.n_rows : ldy;
  a.split_stride = splits > 1 ? split_stride : 0;
  a.M = (int)M;
  a.n_rows = w.n_rows;
  a.K = w.K;
  a.nblk = nblk;
  a.kper = kper;
  a.zp_kind = w.zp_kind;
  a.meta = meta;
  a.a = d_a;
  a.a_dtype = a_dtype;
  a.nib = w.nib;
  a.nib_pitch = w.nib_pitch;
  a.sc = w.sc;
  a.sc_pitch = w.sc_pitch;
  a.zp4 = w.zp4;
  a.zp_pitch = w.zp_pitch;
  a.zpf = w.zpf;
  const dim3 grid(tiles, splits);
  rc = MP == 16 ? launch_tc_zp<16>(st, w.zp_kind, mc, ms, mz, md, a, grid)
                : launch_tc_zp<32>(st, w.zp_kind, mc, ms, mz, md, a, grid);
  if (rc != MSQ_OK) return done(rc);
  if (splits > 1) {
    const int64_t outs = M * (int64_t)w.n_rows;
    const int blocks = (int)std::min<int64_t>((outs + 255) / 256, 4 * (int64_t)sms);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, tc_reduce_kernel, (const float*)ws, splits, split_stride, (int)M,
                                             w.n_rows, d_y, ldy);
    note_launch();
    if (e != cudaSuccess) return done(cuda_fail(e, "tc reduce launch"));
  }
  note_path(splits > 1 ? "gemv_tc_i8_ksplit" : "gemv_tc_i8");
  return done(MSQ_OK);
}

int set_wait_budget_tc(unsigned long long ns) {
  MSQ_CUDA_TRY(cudaMemcpyToSymbol(ptx::g_wait_budget_ns, &ns, sizeof ns), "set tensor-core GEMV wait budget");
  return MSQ_OK;
}

int read_gemv_tc_errors(cudaStream_t st, int* flags) {
  int v = 0;
  MSQ_CUDA_TRY(cudaMemcpyFromSymbolAsync(&v, g_tc_err, sizeof(int), 0, cudaMemcpyDeviceToHost, st),
               "read tc gemv error word");
  MSQ_CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
  if (v) {
    const int zero = 0;
    MSQ_CUDA_TRY(cudaMemcpyToSymbolAsync(g_tc_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st),
                 "clear tc gemv error word");
    MSQ_CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
  }
  *flags = v;
  return MSQ_OK;
}

}  // namespace msq
