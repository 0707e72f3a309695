// Decode GEMV for MatMulNBits on the tensor cores (bits = 4, block_size 32 / 64 / 128, M <= 4
// per pass). Memory-bound: one producer warp streams the repacked weight stages
// (cp.async.bulk, up to 8 in flight); 16 consumer warps turn each lane's 32-bit nibble word
// straight into the A fragment of mma.m16n8k16 (rows r and r+8, four k each) and multiply it
// against the activations held as B fragments.
//
// Exactness. The reference computes sum_k a[m,k] * ((q - zp) * s) in fp32
// (MatMulNBitsKernel.cs:236-261). Here, per quantisation block b:
//     y[m,n] += s[n,b] * ( sum_{k in b} q[n,k] * a'[m,k]  -  zp[n,b] * S_b[m] ) * 2^-sigma_m
// with a' = a * 2^sigma_m (a power-of-two row scale putting max|a'| just under 2^14) and
// S_b = sum_{k in b} a'. The tensor core sees q exactly (fp16 1024+q minus 1024) and a' as
// two fp16 columns hi = fp16(a'), lo = fp16(a' - hi), so a' is carried to ~2^-22 and every
// product is exact in the fp32 accumulator; scale and zero point are applied in fp32. The
// parity bar against the fp32 reference is rel-L2 <= 1e-5.
//
// Decode: one word holds, in nibble slots 0..7, the codes of (row r, k 2t), (r, 2t+8),
// (r+8, 2t), (r+8, 2t+8), (r, 2t+1), (r, 2t+9), (r+8, 2t+1), (r+8, 2t+9). The half2 pairs
// of the A fragment come out of (x & 0x000F000F) | 0x64006400 (k 2t, 2t+1 of row r) and of
// (x & 0x00F000F0) | 0x64006400 (k 2t+8, 2t+9, i.e. 16 q), then the same on x >> 8 for row
// r+8; activations at k%16 >= 8 are staged pre-divided by 16 to match. Per 8 weights:
// 1 shift, 4 LOP3, 4 HSUB2 and one HMMA.
#include "msq_internal.cuh"
#include "msq_ptx.cuh"

#include <algorithm>

namespace msq {
namespace {

constexpr int kConsumers = 16;
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kSmemMax = 227 * 1024;
constexpr int kMaxM = 4;  // B columns: (hi, lo) x 4 rows of A = one n8 tile

__device__ int g_mma_err;

struct Args {
  const uint8_t* strm;
  const void* a;
  int a_dtype;
  int64_t m0;
  int mc;  // A rows in this pass (<= 4)
  float* y;
  int64_t ldy;
  int n_rows, K, bs, ks, nwk, groups, kt, ntiles, rb, nblk, stage_bytes, off_sc, off_zp, zp_kind;
  int nst, seg_tiles, rows_cta;
  int off_ahl, off_s, off_ysum, off_bar, off_ring;  // shared-memory offsets (bytes)
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (*abort_flag) return false;
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort_flag) return false;
      if (ptx::globaltimer() - t0 > ptx::kWaitBudgetNs) {
        *abort_flag = 1;
        atomicCAS(&g_mma_err, 0, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (1024 + q) pairs -> q pairs, exact in fp16.
__device__ __forceinline__ uint32_t q_pair(uint32_t masked) {
  const uint32_t h = masked | 0x64006400u;
  const uint32_t k1024 = 0x64006400u;
  __half2 v = __hsub2(*reinterpret_cast<const __half2*>(&h), *reinterpret_cast<const __half2*>(&k1024));
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int KSTEPS, int BSTEPS>
__global__ void __launch_bounds__(kThreads, 1) gemv_mma_kernel(const Args p) {
  constexpr int NBS = KSTEPS / BSTEPS;  // quantisation blocks per warp slice
  extern __shared__ __align__(16) uint8_t smem[];
  float* sig = reinterpret_cast<float*>(smem);               // [0..3] 2^sigma, [4..7] 2^-sigma, [8..] scratch
  __half* ahl = reinterpret_cast<__half*>(smem + p.off_ahl);  // [2*mc][segk]
  float* sblk = reinterpret_cast<float*>(smem + p.off_s);     // [mc][segk/bs]
  float* ysum = reinterpret_cast<float*>(smem + p.off_ysum);  // [nwk][rows_cta][mc]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* empty = full + kMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMaxStages);
  uint8_t* ring = smem + p.off_ring;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grid = gridDim.x;
  const int nb_cta = (p.nblk - (int)blockIdx.x + grid - 1) / grid;  // row blocks of this CTA
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nst; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], kConsumers);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ---------------- producer
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int t = 0; t < p.ntiles && ok; ++t)
        for (int i = 0; i < nb_cta && ok; ++i) {
          const int b = blockIdx.x + i * grid;
          const int s = issued % p.nst;
          const uint32_t u = issued / p.nst;
          if (issued >= p.nst) ok = wait_or_abort(&empty[s], (u - 1) & 1, abort_flag, ptx::kErrTimeoutEmpty);
          if (!ok) break;
          ptx::mbar_arrive_expect_tx(&full[s], p.stage_bytes);
          ptx::bulk_g2s(ring + (size_t)s * p.stage_bytes,
                        p.strm + ((int64_t)b * p.ntiles + t) * (int64_t)p.stage_bytes, p.stage_bytes, &full[s]);
          ++issued;
        }
      for (int s = 0; s < p.nst && s < issued; ++s) {  // in-flight copies must land before exit
        const int last = s + (issued - 1 - s) / p.nst * p.nst;
        const unsigned long long t0 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&full[s], (last / p.nst) & 1)) {
          if (ptx::globaltimer() - t0 > ptx::kWaitBudgetNs) {
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
  for (int i = tid; i < p.nwk * p.rows_cta * mc; i += kConsumers * 32) ysum[i] = 0.f;

  // per-row power-of-two prescale: max|a'| in [2^13, 2^14)
  {
    float mx[kMaxM] = {0.f, 0.f, 0.f, 0.f};
    for (int k = tid; k < p.K; k += kConsumers * 32)
#pragma unroll
      for (int m = 0; m < kMaxM; ++m)
        if (m < mc) mx[m] = fmaxf(mx[m], fabsf(load_act(p.a, p.a_dtype, (p.m0 + m) * (int64_t)p.K + k)));
#pragma unroll
    for (int m = 0; m < kMaxM; ++m) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx[m] = fmaxf(mx[m], __shfl_xor_sync(0xffffffffu, mx[m], off));
      if (lane == 0) sig[8 + warp * kMaxM + m] = mx[m];
    }
    ptx::named_bar_sync(1, kConsumers * 32);
    if (tid < kMaxM) {
      float v = 0.f;
      for (int w = 0; w < kConsumers; ++w) v = fmaxf(v, sig[8 + w * kMaxM + tid]);
      int e = 0;
      if (v > 0.f && isfinite(v)) frexpf(v, &e);
      int s = 14 - e;
      s = max(-100, min(100, s));
      sig[tid] = ldexpf(1.f, s);
      sig[4 + tid] = ldexpf(1.f, -s);
    }
    ptx::named_bar_sync(1, kConsumers * 32);
  }

  const bool active = warp < p.groups * p.nwk;
  const int g = warp / p.nwk, w = warp % p.nwk;
  const int grp = lane >> 2, tq = lane & 3;
  constexpr int chunks = KSTEPS / 4;
  const int segk_full = p.seg_tiles * p.kt;
  int it = 0;

  for (int seg0 = 0; seg0 < p.ntiles; seg0 += p.seg_tiles) {
    const int ntl = min(p.seg_tiles, p.ntiles - seg0);
    const int segk = ntl * p.kt;
    const int64_t kbase = (int64_t)seg0 * p.kt;
    // ---- stage split activations: hi / lo fp16 columns (k%16 >= 8 pre-divided by 16)
    for (int idx = tid; idx < mc * segk; idx += kConsumers * 32) {
      const int m = idx / segk, kl = idx - m * segk;
      const int64_t kg = kbase + kl;
      float x = kg < p.K ? load_act(p.a, p.a_dtype, (p.m0 + m) * (int64_t)p.K + kg) * sig[m] : 0.f;
      if ((kl & 15) >= 8) x *= 0.0625f;
      const __half hi = __float2half_rn(x);
      const __half lo = __float2half_rn(x - __half2float(hi));
      ahl[(2 * m) * segk_full + kl] = hi;
      ahl[(2 * m + 1) * segk_full + kl] = lo;
    }
    // ---- block sums of a' (before the /16)
    const int nbseg = segk / p.bs;
    for (int idx = tid; idx < mc * nbseg; idx += kConsumers * 32) {
      const int m = idx / nbseg, jb = idx - m * nbseg;
      float s = 0.f;
      for (int q = 0; q < p.bs; ++q) {
        const int64_t kg = kbase + (int64_t)jb * p.bs + q;
        if (kg < p.K) s += load_act(p.a, p.a_dtype, (p.m0 + m) * (int64_t)p.K + kg);
      }
      sblk[m * (segk_full / p.bs) + jb] = s * sig[m];
    }
    ptx::named_bar_sync(1, kConsumers * 32);

    for (int t = seg0; t < seg0 + ntl; ++t) {
      // B fragments of this warp's k-slice (reused across the CTA's row blocks)
      uint32_t bf0[KSTEPS], bf1[KSTEPS];
      float sv[NBS];  // block sums of this lane's A row
      const int kl0 = (t - seg0) * p.kt + w * p.ks;
      const bool colok = active && grp < 2 * mc;
#pragma unroll
      for (int s = 0; s < KSTEPS; ++s) {
        bf0[s] = colok ? *reinterpret_cast<const uint32_t*>(ahl + grp * segk_full + kl0 + 16 * s + 2 * tq) : 0u;
        bf1[s] = colok ? *reinterpret_cast<const uint32_t*>(ahl + grp * segk_full + kl0 + 16 * s + 2 * tq + 8) : 0u;
      }
#pragma unroll
      for (int j = 0; j < NBS; ++j)
        sv[j] = (active && tq < mc) ? sblk[tq * (segk_full / p.bs) + kl0 / p.bs + j] : 0.f;

      for (int i = 0; i < nb_cta; ++i, ++it) {
        const int s = it % p.nst;
        const uint32_t u = it / p.nst;
        const bool ok = wait_or_abort(&full[s], u & 1, abort_flag, ptx::kErrTimeoutFull);
        if (ok && active) {
          const uint8_t* base = ring + (size_t)s * p.stage_bytes;
          const uint4* nibp = reinterpret_cast<const uint4*>(base) + ((g * p.nwk + w) * chunks) * 32 + lane;
          uint32_t words[KSTEPS];
#pragma unroll
          for (int c = 0; c < KSTEPS / 4; ++c) {
            const uint4 v = nibp[c * 32];
            words[4 * c + 0] = v.x;
            words[4 * c + 1] = v.y;
            words[4 * c + 2] = v.z;
            words[4 * c + 3] = v.w;
          }
          const int unit0 = (g * p.nwk + w) * NBS;
          const float* scp = reinterpret_cast<const float*>(base + p.off_sc);
          float y0 = 0.f, y1 = 0.f;
#pragma unroll
          for (int j = 0; j < NBS; ++j) {
            const float s0 = scp[(unit0 + j) * 16 + grp];
            const float s1 = scp[(unit0 + j) * 16 + grp + 8];
            float z0 = 8.f, z1 = 8.f;
            if (p.zp_kind == ZP_PACKED) {
              const uint2 zw = reinterpret_cast<const uint2*>(base + p.off_zp)[unit0 + j];
              z0 = (float)((zw.x >> (4 * grp)) & 0xF);
              z1 = (float)((zw.y >> (4 * grp)) & 0xF);
            } else if (p.zp_kind == ZP_F32) {
              const float* zp = reinterpret_cast<const float*>(base + p.off_zp);
              z0 = zp[(unit0 + j) * 16 + grp];
              z1 = zp[(unit0 + j) * 16 + grp + 8];
            }
            float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int q = j * BSTEPS; q < (j + 1) * BSTEPS; ++q) {
              const uint32_t x = words[q];
              const uint32_t x8 = x >> 8;
              mma16816(c, q_pair(x & 0x000F000Fu), q_pair(x8 & 0x000F000Fu), q_pair(x & 0x00F000F0u),
                       q_pair(x8 & 0x00F000F0u), bf0[q], bf1[q]);
            }
            y0 = fmaf(s0, fmaf(-z0, sv[j], c[0] + c[1]), y0);
            y1 = fmaf(s1, fmaf(-z1, sv[j], c[2] + c[3]), y1);
          }
          if (tq < mc) {
            float* yr = ysum + ((int64_t)w * p.rows_cta + i * p.rb + g * 16 + grp) * mc + tq;
            yr[0] += y0;
            yr[8 * mc] += y1;
          }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[s]);
      }
    }
    ptx::named_bar_sync(1, kConsumers * 32);  // the next segment restages the activations
  }

  // ---- fixed-order sum over the k-slices, unscale, store (coalesced along rows)
  for (int idx = tid; idx < mc * p.rows_cta; idx += kConsumers * 32) {
    const int m = idx / p.rows_cta, r = idx - m * p.rows_cta;
    const int i = r / p.rb, rl = r - i * p.rb;
    const int b = blockIdx.x + i * grid;
    const int64_t row = (int64_t)b * p.rb + rl;
    if (b < p.nblk && row < p.n_rows) {
      float v = 0.f;
      for (int ww = 0; ww < p.nwk; ++ww) v += ysum[((int64_t)ww * p.rows_cta + r) * mc + m];
      p.y[(p.m0 + m) * p.ldy + row] = v * sig[4 + m];
    }
  }
}

template <int KSTEPS, int BSTEPS>
int launch(cudaStream_t st, const Args& a, int grid, size_t smem) {
  auto kern = gemv_mma_kernel<KSTEPS, BSTEPS>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax),
                 "mma gemv smem attribute");
    configured[dev] = true;
  }
  kern<<<grid, kThreads, smem, st>>>(a);
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "mma gemv launch");
  return MSQ_OK;
}

inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

}  // namespace

int run_gemv_mma(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M, float* d_y,
                 int64_t ldy) {
  if (!w.strm || (w.ks != 64 && w.ks != 128) || w.block_size > w.ks) return MSQ_E_UNSUPPORTED;
  const int sms = num_sms(w.device);
  for (int64_t m0 = 0; m0 < M; m0 += kMaxM) {
    const int mc = (int)std::min<int64_t>(kMaxM, M - m0);
    Args a{};
    a.strm = w.strm;
    a.a = d_a;
    a.a_dtype = a_dtype;
    a.m0 = m0;
    a.mc = mc;
    a.y = d_y;
    a.ldy = ldy;
    a.n_rows = w.n_rows;
    a.K = w.K;
    a.bs = w.block_size;
    a.ks = w.ks;
    a.nwk = w.nwk;
    a.groups = w.groups;
    a.kt = w.kt;
    a.ntiles = w.ntiles;
    a.rb = w.rb;
    a.nblk = w.nblk;
    a.stage_bytes = w.stage_bytes;
    a.off_sc = w.off_sc;
    a.off_zp = w.off_zp;
    a.zp_kind = w.zp_kind;
    // grid: one CTA per SM, more when the per-CTA row sums would not fit
    int grid = std::min(w.nblk, sms);
    auto ysum_bytes = [&](int gr) { return w.nwk * ((w.nblk + gr - 1) / gr) * w.rb * mc * 4; };
    while (ysum_bytes(grid) > 48 * 1024 && grid < w.nblk) grid = std::min(w.nblk, grid * 2);
    a.rows_cta = ((w.nblk + grid - 1) / grid) * w.rb;
    const int ysum = w.nwk * a.rows_cta * mc * 4;
    // activations: as many whole k-tiles per segment as leave room for >= 4 stages
    const int head = 64 + 16 * kMaxM * 4;  // prescale + reduction scratch
    const int per_tile = 4 * mc * w.kt + 4 * mc * (w.kt / w.block_size);
    const int bars = 2 * kMaxStages * 8 + 16;
    const int fixed_no_act = align_up(head, 16) + align_up(ysum, 16) + bars + 128;
    int seg_tiles = (kSmemMax - fixed_no_act - 4 * w.stage_bytes) / per_tile;
    if (seg_tiles < 1) {
      seg_tiles = (kSmemMax - fixed_no_act - 2 * w.stage_bytes) / per_tile;
      if (seg_tiles < 1) return MSQ_E_UNSUPPORTED;
    }
    seg_tiles = std::min(seg_tiles, w.ntiles);
    a.seg_tiles = seg_tiles;
    const int segk = seg_tiles * w.kt;
    a.off_ahl = align_up(head, 16);
    a.off_s = a.off_ahl + align_up(2 * mc * segk * 2, 16);
    a.off_ysum = a.off_s + align_up(mc * (segk / w.block_size) * 4, 16);
    a.off_bar = a.off_ysum + align_up(ysum, 16);
    a.off_ring = align_up(a.off_bar + bars, 128);
    int nst = (kSmemMax - a.off_ring) / w.stage_bytes;
    nst = std::min(nst, kMaxStages);
    if (nst < 2) return MSQ_E_UNSUPPORTED;
    a.nst = nst;
    const size_t smem = (size_t)a.off_ring + (size_t)nst * w.stage_bytes;
    int rc;
    const int bsteps = w.block_size / 16;
    if (w.ks == 128)
      rc = bsteps == 2 ? launch<8, 2>(st, a, grid, smem) : bsteps == 4 ? launch<8, 4>(st, a, grid, smem)
                                                        : launch<8, 8>(st, a, grid, smem);
    else
      rc = bsteps == 2 ? launch<4, 2>(st, a, grid, smem) : launch<4, 4>(st, a, grid, smem);
    if (rc != MSQ_OK) return rc;
  }
  note_path(M <= 4 ? "gemv_mma" : "gemv_mma_multipass");
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
