// Generic MatMulNBits kernel on the reference layout: any bits (4/8), any block size,
// all three zero-point forms, ragged K, any M. It is the correctness safety net for
// shapes the specialised kernels do not take, and computes each weight exactly as the
// reference does, W = (q - zp) * scale in fp32 (MatMulNBitsKernel.cs:236-253).
//
// Mapping: one warp per weight row n; lanes stride over the codes of each block (a
// warp reads a block's blob contiguously); MT activation rows accumulate at once and
// the warp re-walks the row for the next MT rows. Warp-shuffle reduction at the end.
#include "msq_internal.cuh"

namespace msq {
namespace {

constexpr int kGenericWarps = 8;
constexpr int kGenericMT = 8;

__global__ void __launch_bounds__(kGenericWarps * 32)
generic_kernel(const uint8_t* __restrict__ b, const float* __restrict__ sc, int zp_kind,
               const uint8_t* __restrict__ zpu8, const float* __restrict__ zpf,
               const void* __restrict__ a, int a_dtype, int64_t M, float* __restrict__ y,
               int64_t ldy, int n_rows, int K, int bits, int bs, int nb, int blob,
               int zp_row_bytes) {
  const int lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * kGenericWarps + (threadIdx.x >> 5);
  if (n >= n_rows) return;
  const float default_zp = (float)(1 << (bits - 1));
  const uint8_t* brow = b + n * (int64_t)nb * blob;
  for (int64_t m0 = 0; m0 < M; m0 += kGenericMT) {
    float acc[kGenericMT];
#pragma unroll
    for (int t = 0; t < kGenericMT; ++t) acc[t] = 0.f;
    for (int bk = 0; bk < nb; ++bk) {
      const float scale = sc[n * nb + bk];
      float zp = default_zp;
      if (zp_kind == ZP_PACKED) {
        uint8_t zb = zpu8[n * zp_row_bytes + (bits == 8 ? bk : (bk >> 1))];
        zp = (float)(bits == 8 ? zb : ((zb >> ((bk & 1) * 4)) & 0xF));
      } else if (zp_kind == ZP_F32) {
        zp = zpf[n * nb + bk];
      }
      const int k0 = bk * bs;
      const int len = min(bs, K - k0);
      const uint8_t* blob_p = brow + (int64_t)bk * blob;
      for (int i = lane; i < len; i += 32) {
        int q = bits == 8 ? blob_p[i] : ((blob_p[i >> 1] >> ((i & 1) * 4)) & 0xF);
        const float wv = ((float)q - zp) * scale;
#pragma unroll
        for (int t = 0; t < kGenericMT; ++t)
          if (m0 + t < M) acc[t] = fmaf(load_act(a, a_dtype, (m0 + t) * (int64_t)K + k0 + i), wv, acc[t]);
      }
    }
#pragma unroll
    for (int t = 0; t < kGenericMT; ++t) {
      float v = acc[t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0 && m0 + t < M) y[(m0 + t) * ldy + n] = v;
    }
  }
}

}  // namespace

int run_generic(cudaStream_t st, const Weights& w, const void* d_a, int a_dtype, int64_t M,
                float* d_y, int64_t ldy) {
  if (!w.b_ref) return fail(MSQ_E_UNSUPPORTED, "generic path needs a reference-layout handle");
  unsigned grid = (unsigned)((w.n_rows + kGenericWarps - 1) / kGenericWarps);
  generic_kernel<<<grid, kGenericWarps * 32, 0, st>>>(
      w.b_ref, w.sc_ref, w.zp_kind, w.zp_ref_u8, w.zp_ref_f32, d_a, a_dtype, M, d_y, ldy,
      w.n_rows, w.K, w.bits, w.block_size, w.nb, w.blob, w.zp_row_bytes);
  note_launch();
  note_path("generic");
  MSQ_CUDA_TRY(cudaGetLastError(), "generic kernel launch");
  return MSQ_OK;
}

}  // namespace msq
