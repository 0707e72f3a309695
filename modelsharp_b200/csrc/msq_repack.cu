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

// One thread per 32-bit word of the decode stream (layout in msq_internal.cuh).
__global__ void repack_stream_kernel(const uint8_t* __restrict__ b, const void* __restrict__ scales, int sdt,
                                     const void* __restrict__ zp, int zp_kind, int64_t row0, int n_rows, int K,
                                     int bs, int nb, int blob, int zp_row_bytes, int ks, int nwk, int groups,
                                     int kt, int ntiles, int stage_words, int off_sc_w, int off_zp_w,
                                     uint32_t* __restrict__ out, int64_t total_words) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= total_words) return;
  const int64_t stage = idx / stage_words;
  const int wi = (int)(idx - stage * stage_words);
  const int tile = (int)(stage % ntiles);
  const int64_t blk = stage / ntiles;
  const int nbs = ks / bs;
  const int chunks = ks / 64;
  uint32_t val = 0;
  if (wi < off_sc_w) {
    // nibble words: [group][slice][chunk][lane][4 words]
    int r = wi;
    const int step = r & 3; r >>= 2;
    const int lane = r & 31; r >>= 5;
    const int chunk = r % chunks; r /= chunks;
    const int slice = r % nwk;
    const int g = r / nwk;
    const int64_t row0r = blk * 16 * groups + g * 16 + (lane >> 2);
    const int t = lane & 3;
    const int64_t kb = (int64_t)tile * kt + (int64_t)slice * ks + chunk * 64 + step * 16 + 2 * t;
    // slot j -> (row offset, k offset): 0:(0,0) 1:(0,8) 2:(8,0) 3:(8,8) 4:(0,1) 5:(0,9) 6:(8,1) 7:(8,9)
    const int rofs[8] = {0, 0, 8, 8, 0, 0, 8, 8};
    const int kofs[8] = {0, 8, 0, 8, 1, 9, 1, 9};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t rr = row0r + rofs[j];
      const int64_t k = kb + kofs[j];
      if (rr < n_rows && k < K) {
        const int64_t bk = k / bs, i = k - bk * bs;
        const uint8_t byte = b[((row0 + rr) * nb + bk) * (int64_t)blob + (i >> 1)];
        val |= (uint32_t)((byte >> ((i & 1) * 4)) & 0xF) << (4 * j);
      }
    }
  } else if (wi < off_zp_w) {
    // fp32 scales: [group][slice][block][16 rows]
    int r = wi - off_sc_w;
    const int row = r & 15; r >>= 4;
    const int j = r % nbs; r /= nbs;
    const int slice = r % nwk;
    const int g = r / nwk;
    const int64_t rr = blk * 16 * groups + g * 16 + row;
    const int64_t bl = ((int64_t)tile * kt + (int64_t)slice * ks) / bs + j;
    if (rr < n_rows && bl < nb) val = __float_as_uint(load_scale(scales, sdt, (row0 + rr) * nb + bl));
  } else if (zp_kind == ZP_PACKED) {
    // packed: [group][slice][block][2 words of 8 nibbles, nibble = row]
    int r = wi - off_zp_w;
    const int half = r & 1; r >>= 1;
    if (r < groups * nwk * nbs) {
      const int j = r % nbs; r /= nbs;
      const int slice = r % nwk;
      const int g = r / nwk;
      const int64_t bl = ((int64_t)tile * kt + (int64_t)slice * ks) / bs + j;
      for (int q = 0; q < 8; ++q) {
        const int64_t rr = blk * 16 * groups + g * 16 + half * 8 + q;
        if (rr < n_rows && bl < nb) {
          const uint8_t zb = static_cast<const uint8_t*>(zp)[(row0 + rr) * zp_row_bytes + (bl >> 1)];
          val |= (uint32_t)((zb >> ((bl & 1) * 4)) & 0xF) << (4 * q);
        }
      }
    }
  } else if (zp_kind == ZP_F32) {
    int r = wi - off_zp_w;
    if (r < groups * nwk * nbs * 16) {
      const int row = r & 15; r >>= 4;
      const int j = r % nbs; r /= nbs;
      const int slice = r % nwk;
      const int g = r / nwk;
      const int64_t rr = blk * 16 * groups + g * 16 + row;
      const int64_t bl = ((int64_t)tile * kt + (int64_t)slice * ks) / bs + j;
      if (rr < n_rows && bl < nb) val = __float_as_uint(static_cast<const float*>(zp)[(row0 + rr) * nb + bl]);
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

// Decode-stream geometry: warp slices of ks k (a multiple of max(block_size, 64); 128 when
// K is long enough to fill 16 slices of 128), nwk <= 16 slices per k-tile, and as many
// 16-row groups per row block as leave the 16 consumer warps busy.
void plan_stream(Weights& w) {
  const int K = w.K, bs = w.block_size;
  const int unit = bs > 64 ? bs : 64;
  int ks = unit;
  if (unit <= 128 && K >= 16 * 128) ks = 128;
  int nwk = (K + ks - 1) / ks;
  if (nwk > 16) nwk = 16;
  w.ks = ks;
  w.nwk = nwk;
  w.groups = 16 / nwk;
  w.kt = nwk * ks;
  w.ntiles = (K + w.kt - 1) / w.kt;
  w.rb = 16 * w.groups;
  w.nblk = (w.n_rows + w.rb - 1) / w.rb;
  const int nbs = ks / bs;
  const int units = w.groups * nwk * nbs;
  const int nib = w.rb * w.kt / 2;
  const int sc = units * 16 * 4;
  const int zpb = w.zp_kind == ZP_PACKED ? units * 8 : w.zp_kind == ZP_F32 ? units * 64 : 0;
  w.off_sc = nib;
  w.off_zp = nib + sc;
  w.stage_bytes = (nib + sc + zpb + 15) / 16 * 16;
}

int repack_stream(cudaStream_t st, Weights& w, const uint8_t* d_b, int n_begin, const void* d_scales,
                  int scales_dtype, const void* d_zp) {
  const int T = 256;
  const int stage_words = w.stage_bytes / 4;
  const int64_t total = (int64_t)w.nblk * w.ntiles * stage_words;
  repack_stream_kernel<<<grid_for(total, T), T, 0, st>>>(
      d_b, d_scales, scales_dtype, d_zp, w.zp_kind, n_begin, w.n_rows, w.K, w.block_size, w.nb, w.blob,
      w.zp_row_bytes, w.ks, w.nwk, w.groups, w.kt, w.ntiles, stage_words, w.off_sc / 4, w.off_zp / 4,
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
