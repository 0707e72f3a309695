// Load-time repacker: reference MatMulNBits layout -> device-resident kernel layout.
//
// Source layout (MatMulNBitsKernel.cs:26-36): B uint8 [N][nb][blob] with the code of
// in-block index i in byte i/2, low nibble for even i (MatMulNBitsKernel.cs:349-356);
// scales [N*nb]; zero points packed [N][zp_row_bytes] or float [N*nb].
#include "msq_internal.cuh"

namespace msq {
namespace {

// Nibble slot j of an output word holds k-offset kSlotK[j] of its 8-code group.
__constant__ int kSlotK[8] = {0, 2, 4, 6, 1, 3, 5, 7};

// One thread per output 32-bit word of the nibble plane.
__global__ void repack_nib4_kernel(const uint8_t* __restrict__ b, int64_t row0, int n_rows, int K,
                                   int bs, int nb, int blob, uint32_t* __restrict__ nib,
                                   int64_t words_per_row) {
  int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t total = (int64_t)n_rows * words_per_row;
  if (idx >= total) return;
  int64_t r = idx / words_per_row;
  int64_t wi = idx - r * words_per_row;
  const uint8_t* brow = b + (row0 + r) * (int64_t)nb * blob;
  uint32_t out = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    int64_t k = wi * 8 + kSlotK[j];
    uint32_t q = 0;
    if (k < K) {
      int64_t bk = k / bs;
      int64_t i = k - bk * bs;
      uint8_t byte = brow[bk * blob + (i >> 1)];
      q = (byte >> ((i & 1) * 4)) & 0xFu;
    }
    out |= q << (4 * j);
  }
  nib[idx] = out;
}

__device__ __forceinline__ float load_scale(const void* s, int dt, int64_t i) {
  return load_act(s, dt, i);
}

// One thread per (row, padded block): fp32 + fp16 scale planes and the float zp plane.
__global__ void repack_scales_kernel(const void* __restrict__ scales, int sdt, int64_t row0,
                                     int n_rows, int nb, float* __restrict__ sc,
                                     __half* __restrict__ sc16, int64_t sc_pitch,
                                     const float* __restrict__ zpf_in, float* __restrict__ zpf) {
  int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t total = (int64_t)n_rows * sc_pitch;
  if (idx >= total) return;
  int64_t r = idx / sc_pitch;
  int64_t bk = idx - r * sc_pitch;
  float v = 0.f, z = 0.f;
  if (bk < nb) {
    v = load_scale(scales, sdt, (row0 + r) * nb + bk);
    if (zpf_in) z = zpf_in[(row0 + r) * nb + bk];
  }
  sc[idx] = v;
  if (sc16) sc16[idx] = __float2half_rn(v);
  if (zpf) zpf[idx] = z;
}

// One thread per byte of the padded packed-zero-point plane.
__global__ void repack_zp_kernel(const uint8_t* __restrict__ zp, int64_t row0, int n_rows,
                                 int zp_row_bytes, uint8_t* __restrict__ zp4, int64_t zp_pitch) {
  int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t total = (int64_t)n_rows * zp_pitch;
  if (idx >= total) return;
  int64_t r = idx / zp_pitch;
  int64_t j = idx - r * zp_pitch;
  zp4[idx] = j < zp_row_bytes ? zp[(row0 + r) * zp_row_bytes + j] : 0;
}

// Widens a slice of scales to fp32 (reference-layout handles).
__global__ void widen_kernel(const void* __restrict__ s, int sdt, int64_t off, int64_t n,
                             float* __restrict__ out) {
  int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx < n) out[idx] = load_scale(s, sdt, off + idx);
}

// One thread per 32-bit word of the decode stream ([block][tile][row][record]).
__global__ void repack_stream_kernel(const uint8_t* __restrict__ b, const void* __restrict__ scales, int sdt,
                                     const void* __restrict__ zp, int zp_kind, int64_t row0, int n_rows, int K,
                                     int bs, int nb, int blob, int zp_row_bytes, int rb, int kt, int ntiles,
                                     int rec_words, int sc_word, int zp_word, uint32_t* __restrict__ out,
                                     int64_t total_words) {
  int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= total_words) return;
  const int64_t rec = idx / rec_words;
  const int wi = (int)(idx - rec * rec_words);
  const int rr = (int)(rec % rb);
  const int64_t bt = rec / rb;
  const int t = (int)(bt % ntiles);
  const int64_t blk = bt / ntiles;
  const int64_t r = blk * rb + rr;
  const int nbt = kt / bs;
  uint32_t val = 0;
  if (r < n_rows) {
    const int64_t n = row0 + r;
    if (wi < kt / 8) {
      const uint8_t* brow = b + n * (int64_t)nb * blob;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t k = (int64_t)t * kt + 8 * wi + kSlotK[j];
        if (k < K) {
          const int64_t bk = k / bs, i = k - bk * bs;
          val |= (uint32_t)((brow[bk * blob + (i >> 1)] >> ((i & 1) * 4)) & 0xF) << (4 * j);
        }
      }
    } else if (wi >= sc_word && wi < sc_word + nbt) {
      const int64_t bl = (int64_t)t * nbt + (wi - sc_word);
      if (bl < nb) val = __float_as_uint(load_scale(scales, sdt, n * nb + bl));
    } else if (zp_kind == ZP_PACKED && wi >= zp_word && wi < zp_word + (nbt + 7) / 8) {
      const int j0 = 8 * (wi - zp_word);
      const uint8_t* zrow = static_cast<const uint8_t*>(zp) + n * zp_row_bytes;
      for (int j = 0; j < 8 && j0 + j < nbt; ++j) {
        const int64_t bl = (int64_t)t * nbt + j0 + j;
        if (bl < nb) val |= (uint32_t)((zrow[bl >> 1] >> ((bl & 1) * 4)) & 0xF) << (4 * j);
      }
    } else if (zp_kind == ZP_F32 && wi >= zp_word && wi < zp_word + nbt) {
      const int64_t bl = (int64_t)t * nbt + (wi - zp_word);
      if (bl < nb) val = __float_as_uint(static_cast<const float*>(zp)[n * nb + bl]);
    }
  }
  out[idx] = val;
}

inline unsigned grid_for(int64_t n, int threads) {
  return (unsigned)((n + threads - 1) / threads);
}

}  // namespace

int repack_fast4(cudaStream_t st, Weights& w, const uint8_t* d_b, int n_begin,
                 const void* d_scales, int scales_dtype, const void* d_zp) {
  const int T = 256;
  int64_t words = (int64_t)w.n_rows * (w.nib_pitch / 4);
  if (words > 0) {
    repack_nib4_kernel<<<grid_for(words, T), T, 0, st>>>(
        d_b, n_begin, w.n_rows, w.K, w.block_size, w.nb, w.blob,
        reinterpret_cast<uint32_t*>(w.nib), w.nib_pitch / 4);
    note_launch();
  }
  int64_t sn = (int64_t)w.n_rows * w.sc_pitch;
  if (sn > 0) {
    repack_scales_kernel<<<grid_for(sn, T), T, 0, st>>>(
        d_scales, scales_dtype, n_begin, w.n_rows, w.nb, w.sc, w.sc16, w.sc_pitch,
        w.zp_kind == ZP_F32 ? static_cast<const float*>(d_zp) : nullptr, w.zpf);
    note_launch();
  }
  if (w.zp_kind == ZP_PACKED) {
    int64_t zn = (int64_t)w.n_rows * w.zp_pitch;
    repack_zp_kernel<<<grid_for(zn, T), T, 0, st>>>(static_cast<const uint8_t*>(d_zp), n_begin,
                                                    w.n_rows, w.zp_row_bytes, w.zp4, w.zp_pitch);
    note_launch();
  }
  MSQ_CUDA_TRY(cudaGetLastError(), "repack launch");
  return MSQ_OK;
}

// Chooses the decode-stream geometry: k-tiles of ~1024 (a multiple of max(bs, 64)), and a
// row-block height <= 32 that spreads the row blocks evenly over the SMs.
void plan_stream(Weights& w, int sms) {
  const int K = w.K, bs = w.block_size;
  const int unit = bs > 64 ? bs : 64;
  const int t0 = (K + 1023) / 1024;
  int kt = (K + t0 - 1) / t0;
  kt = (kt + unit - 1) / unit * unit;
  w.kt = kt;
  w.ntiles = (K + kt - 1) / kt;
  const int nbt = kt / bs;
  int zb = w.zp_kind == ZP_PACKED ? (nbt + 7) / 8 * 4 : w.zp_kind == ZP_F32 ? 4 * nbt : 0;
  int rec = kt / 2 + 4 * nbt + zb;
  rec = (rec + 15) / 16 * 16;
  if ((rec / 16) % 2 == 0) rec += 16;
  w.rec_bytes = rec;
  w.rec_sc = kt / 2;
  w.rec_zp = kt / 2 + 4 * nbt;
  // row-block height: each CTA walks its row blocks in turn, so the kernel time goes as
  // (row blocks per CTA) x (rows per block); minimise that, preferring taller blocks on ties.
  const int n = w.n_rows;
  int best_rb = 1;
  int64_t best = -1;
  for (int rb = 32; rb >= 1; --rb) {
    const int64_t nblk = (n + rb - 1) / rb;
    const int64_t cost = (nblk + sms - 1) / sms * rb;
    if (best < 0 || cost < best) {
      best = cost;
      best_rb = rb;
    }
  }
  w.rb = best_rb;
  w.nblk = (n + best_rb - 1) / best_rb;
}

int repack_stream(cudaStream_t st, Weights& w, const uint8_t* d_b, int n_begin, const void* d_scales,
                  int scales_dtype, const void* d_zp) {
  const int T = 256;
  const int rec_words = w.rec_bytes / 4;
  const int64_t total = (int64_t)w.nblk * w.ntiles * w.rb * rec_words;
  repack_stream_kernel<<<grid_for(total, T), T, 0, st>>>(
      d_b, d_scales, scales_dtype, d_zp, w.zp_kind, n_begin, w.n_rows, w.K, w.block_size, w.nb, w.blob,
      w.zp_row_bytes, w.rb, w.kt, w.ntiles, rec_words, w.rec_sc / 4, w.rec_zp / 4,
      reinterpret_cast<uint32_t*>(w.strm), total);
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "stream repack launch");
  return MSQ_OK;
}

int repack_reference(cudaStream_t st, Weights& w, const uint8_t* d_b, int n_begin,
                     const void* d_scales, int scales_dtype, const void* d_zp) {
  const int T = 256;
  int64_t row_bytes = (int64_t)w.nb * w.blob;
  MSQ_CUDA_TRY(cudaMemcpyAsync(w.b_ref, d_b + (int64_t)n_begin * row_bytes,
                               (size_t)(row_bytes * w.n_rows), cudaMemcpyDeviceToDevice, st),
               "copy B rows");
  int64_t sn = (int64_t)w.n_rows * w.nb;
  widen_kernel<<<grid_for(sn, T), T, 0, st>>>(d_scales, scales_dtype, (int64_t)n_begin * w.nb, sn,
                                              w.sc_ref);
  note_launch();
  if (w.zp_kind == ZP_PACKED) {
    MSQ_CUDA_TRY(cudaMemcpyAsync(w.zp_ref_u8,
                                 static_cast<const uint8_t*>(d_zp) + (int64_t)n_begin * w.zp_row_bytes,
                                 (size_t)w.zp_row_bytes * w.n_rows, cudaMemcpyDeviceToDevice, st),
                 "copy zero-point rows");
  } else if (w.zp_kind == ZP_F32) {
    MSQ_CUDA_TRY(cudaMemcpyAsync(w.zp_ref_f32, static_cast<const float*>(d_zp) + (int64_t)n_begin * w.nb,
                                 sizeof(float) * (size_t)sn, cudaMemcpyDeviceToDevice, st),
                 "copy float zero points");
  }
  MSQ_CUDA_TRY(cudaGetLastError(), "repack launch");
  return MSQ_OK;
}

}  // namespace msq
