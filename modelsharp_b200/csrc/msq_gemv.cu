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
  static ContextOnce configured;
  const int rc = configured.run([&] {
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 16384),
                 "gemv smem attribute");
    return MSQ_OK;
  });
  if (rc != MSQ_OK) return rc;
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


}  // namespace

int run_gemv(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
             float* d_y, int64_t ldy) {
  if (w.fast8) {
    if (M <= 0) return MSQ_OK;
    const int rc = run_gemv_mma(st, w, d_a, a_dtype, M, d_y, ldy);
    if (rc == MSQ_E_UNSUPPORTED) return fail(rc, "bits=8 decode GEMV: shape not supported");
    return rc;
  }
  if (!w.fast4) return fail(MSQ_E_UNSUPPORTED, "GEMV path needs bits=4 (or bits=8) and a power-of-two block_size >= 32");
  if (M <= 0) return MSQ_OK;
  const int sms = num_sms(w.device);
  const int mr = M == 1 ? 1 : M == 2 ? 2 : M <= 4 ? 4 : 8;
  {
    const int rc = run_gemv_mma(st, w, d_a, a_dtype, M, d_y, ldy);
    if (rc != MSQ_E_UNSUPPORTED) return rc;
  }
  // Block sizes the tensor-core kernel does not take: the K-segmented CUDA-core kernel below.
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

}  // namespace msq
