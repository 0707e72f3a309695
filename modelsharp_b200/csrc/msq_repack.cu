// Load-time repacker: reference MatMulNBits layout -> device-resident kernel layout.
//
// Source layout (MatMulNBitsKernel.cs:26-36): B uint8 [N][nb][blob] with the code of
// in-block index i in byte i/2, low nibble for even i (MatMulNBitsKernel.cs:349-356);
// scales [N*nb]; zero points packed [N][zp_row_bytes] or float [N*nb].
#include "msq_internal.cuh"

#include <algorithm>
#include <mutex>

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
                                     int bs, int nb, int blob, int zp_row_bytes, int kt, int ntiles,
                                     int stage_words, int off_sc_w, int off_zp_w, uint32_t* __restrict__ out,
                                     int64_t total_words, int bits) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= total_words) return;
  const int64_t stage = idx / stage_words;
  const int wi = (int)(idx - stage * stage_words);
  const int tile = (int)(stage % ntiles);
  const int64_t blk = stage / ntiles;
  const int nbt = kt / bs;
  const int64_t r0 = blk * 16;
  uint32_t val = 0;
  if (wi < off_sc_w && bits == 8) {
    // 8-bit code words: [chunk][lane][8 words] = per 32-k step: (row r, k), (row r+8, k),
    // (row r, k+16), (row r+8, k+16), byte j = k offset j: the u8 A-fragment registers
    const int word = wi & 7;
    const int lane = (wi >> 3) & 31;
    const int chunk = wi >> 8;
    const int sub = word & 3;
    const int64_t rr = r0 + (lane >> 2) + (sub & 1) * 8;
    const int64_t kb = (int64_t)tile * kt + chunk * 64 + (word >> 2) * 32 + (sub >> 1) * 16 + 4 * (lane & 3);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = kb + j;
      if (k < K && rr < n_rows) {
        const int64_t bk = k / bs;
        val |= (uint32_t)b[((row0 + rr) * nb + bk) * (int64_t)blob + (k - bk * bs)] << (8 * j);
      }
    }
  } else if (wi < off_sc_w) {
    // code words: [chunk][lane][4 words] = [32-k step 0: k, k+16][step 1: k, k+16]
    const int word = wi & 3;
    const int lane = (wi >> 2) & 31;
    const int chunk = wi >> 7;
    const int64_t rlo = r0 + (lane >> 2), rhi = rlo + 8;
    const int64_t kb = (int64_t)tile * kt + chunk * 64 + (word >> 1) * 32 + (word & 1) * 16 + 4 * (lane & 3);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = kb + j;
      if (k < K) {
        const int64_t bk = k / bs, i = k - bk * bs;
        const int sh = (i & 1) * 4;
        if (rlo < n_rows) val |= (uint32_t)((b[((row0 + rlo) * nb + bk) * (int64_t)blob + (i >> 1)] >> sh) & 0xF) << (8 * j);
        if (rhi < n_rows) val |= (uint32_t)((b[((row0 + rhi) * nb + bk) * (int64_t)blob + (i >> 1)] >> sh) & 0xF) << (8 * j + 4);
      }
    }
  } else if (wi < off_zp_w) {
    // fp32 scales: [block][16 rows]
    const int r = wi - off_sc_w;
    const int row = r & 15, j = r >> 4;
    const int64_t rr = r0 + row;
    const int64_t bl = (int64_t)tile * nbt + j;
    if (rr < n_rows && bl < nb) val = __float_as_uint(load_scale(scales, sdt, (row0 + rr) * nb + bl));
  } else if (zp_kind == ZP_PACKED && bits == 8) {
    // 8-bit packed: [block][16 bytes, byte = row]
    const int r = wi - off_zp_w;
    const int j = r >> 2, q0 = (r & 3) * 4;
    if (j < nbt) {
      const int64_t bl = (int64_t)tile * nbt + j;
      for (int q = 0; q < 4; ++q) {
        const int64_t rr = r0 + q0 + q;
        if (rr < n_rows && bl < nb)
          val |= (uint32_t)static_cast<const uint8_t*>(zp)[(row0 + rr) * zp_row_bytes + bl] << (8 * q);
      }
    }
  } else if (zp_kind == ZP_PACKED) {
    // packed: [block][2 words of 8 nibbles, nibble = row]
    const int r = wi - off_zp_w;
    const int half = r & 1, j = r >> 1;
    if (j < nbt) {
      const int64_t bl = (int64_t)tile * nbt + j;
      for (int q = 0; q < 8; ++q) {
        const int64_t rr = r0 + half * 8 + q;
        if (rr < n_rows && bl < nb) {
          const uint8_t zb = static_cast<const uint8_t*>(zp)[(row0 + rr) * zp_row_bytes + (bl >> 1)];
          val |= (uint32_t)((zb >> ((bl & 1) * 4)) & 0xF) << (4 * q);
        }
      }
    }
  } else if (zp_kind == ZP_F32) {
    const int r = wi - off_zp_w;
    const int row = r & 15, j = r >> 4;
    if (j < nbt) {
      const int64_t rr = r0 + row;
      const int64_t bl = (int64_t)tile * nbt + j;
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

// Decode-stream geometry: the largest k-tile kt <= kt_max that is a multiple of
// max(block_size, 64) and divides K rounded up to that unit (so no padding is streamed),
// falling back to kt_max with a padded last tile when only small divisors exist.
void plan_stream(Weights& w) {
  const int K = w.K, bs = w.block_size;
  const int unit = bs > 64 ? bs : 64;
  // stages of 16-35 KB: half the k per tile for 8-bit codes
  const int kt_max = std::max(unit, (unit == 64 ? 2048 : 4096) / (w.bits == 8 ? 2 : 1) / unit * unit);
  const int units = (K + unit - 1) / unit;
  int best = 1;
  for (int d = 1; d * unit <= kt_max; ++d)
    if (units % d == 0) best = d;
  int kt = best * unit;
  if (kt * 4 < std::min(kt_max, units * unit)) kt = std::min(kt_max, units * unit);
  w.kt = kt;
  w.ntiles = (K + kt - 1) / kt;
  w.nblk = (w.n_rows + 15) / 16;
  const int nbt = kt / bs;
  const int nib = 16 * kt * w.bits / 8;
  const int sc = nbt * 16 * 4;
  const int zpb = w.zp_kind == ZP_PACKED ? nbt * 2 * w.bits : w.zp_kind == ZP_F32 ? nbt * 64 : 0;
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
      w.zp_row_bytes, w.kt, w.ntiles, stage_words, w.off_sc / 4, w.off_zp / 4,
      reinterpret_cast<uint32_t*>(w.strm), total, w.bits);
  note_launch();
  MSQ_CUDA_TRY(cudaGetLastError(), "stream repack launch");
  return MSQ_OK;
}

namespace {

// The code, scale and zero point of (row r, k) read back from the decode-stream records
// (layout in msq_internal.cuh); k < K.
struct StreamGeo {
  const uint8_t* strm;
  int kt, ntiles, stage_bytes, off_sc, off_zp, zp_kind, bs;
};

__device__ __forceinline__ const uint8_t* record_of(const StreamGeo& g, int64_t r, int k, int* kk) {
  const int t = k / g.kt;
  *kk = k - t * g.kt;
  return g.strm + ((r >> 4) * g.ntiles + t) * (int64_t)g.stage_bytes;
}

__device__ __forceinline__ uint32_t stream_code(const StreamGeo& g, int64_t r, int k) {
  int kk;
  const uint8_t* rec = record_of(g, r, k, &kk);
  const int rr = (int)(r & 15), o = kk & 63;
  const int word = (o >> 5) * 2 + ((o >> 4) & 1);
  const int ln = (rr & 7) * 4 + ((o & 15) >> 2);
  const uint8_t v = rec[(kk >> 6) * 512 + ln * 16 + word * 4 + (o & 3)];
  return rr < 8 ? (v & 0xFu) : (uint32_t)(v >> 4);
}

// The GEMM's nibble plane from the stream: one thread per output word (slot order kSlotK).
__global__ void nib_from_stream_kernel(StreamGeo g, int n_rows, int K, uint32_t* __restrict__ nib,
                                       int64_t words_per_row) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)n_rows * words_per_row) return;
  const int64_t r = idx / words_per_row, wi = idx - r * words_per_row;
  uint32_t out = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t k = wi * 8 + kSlotK[j];
    if (k < K) out |= stream_code(g, r, (int)k) << (4 * j);
  }
  nib[idx] = out;
}

// Scale planes (fp32, fp16) and the float zero-point plane from the stream: one thread per
// (row, padded block).
__global__ void scales_from_stream_kernel(StreamGeo g, int n_rows, int nb, float* __restrict__ sc,
                                          __half* __restrict__ sc16, float* __restrict__ zpf, int64_t sc_pitch) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)n_rows * sc_pitch) return;
  const int64_t r = idx / sc_pitch;
  const int bk = (int)(idx - r * sc_pitch);
  float v = 0.f, z = 0.f;
  if (bk < nb) {
    int kk;
    const uint8_t* rec = record_of(g, r, bk * g.bs, &kk);
    const int bl = kk / g.bs, rr = (int)(r & 15);
    v = reinterpret_cast<const float*>(rec + g.off_sc)[bl * 16 + rr];
    if (zpf) z = reinterpret_cast<const float*>(rec + g.off_zp)[bl * 16 + rr];
  }
  sc[idx] = v;
  sc16[idx] = __float2half_rn(v);
  if (zpf) zpf[idx] = z;
}

// The packed zero-point plane from the stream: one thread per byte (blocks 2j and 2j + 1).
__global__ void zp_from_stream_kernel(StreamGeo g, int n_rows, int nb, uint8_t* __restrict__ zp4, int64_t zp_pitch) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)n_rows * zp_pitch) return;
  const int64_t r = idx / zp_pitch;
  const int j = (int)(idx - r * zp_pitch);
  const int rr = (int)(r & 15);
  uint32_t out = 0;
  for (int h = 0; h < 2; ++h) {
    const int bk = 2 * j + h;
    if (bk < nb) {
      int kk;
      const uint8_t* rec = record_of(g, r, bk * g.bs, &kk);
      const unsigned long long zw = reinterpret_cast<const unsigned long long*>(rec + g.off_zp)[kk / g.bs];
      out |= (uint32_t)((zw >> (4 * rr)) & 0xF) << (4 * h);
    }
  }
  zp4[idx] = (uint8_t)out;
}

int alloc_plane(void** p, size_t bytes, int64_t* total) {
  *p = nullptr;
  if (!bytes) return MSQ_OK;
  const cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MSQ_E_OOM, "device allocation of %zu bytes for the GEMM layout failed: %s", bytes,
                cudaGetErrorString(e));
  }
  *total += (int64_t)bytes;
  return MSQ_OK;
}

}  // namespace

int ensure_gemm_layout(cudaStream_t st, Weights& w) {
  if (w.gemm_layout.load(std::memory_order_acquire)) return MSQ_OK;
  std::lock_guard<std::mutex> lk(w.state_mu);
  if (w.gemm_layout.load(std::memory_order_relaxed)) return MSQ_OK;
  if (!w.strm) return fail(MSQ_E_UNSUPPORTED, "GEMM path: the handle holds neither layout");
  const size_t rows = (size_t)w.n_rows;
  uint8_t* nib = nullptr;
  float *sc = nullptr, *zpf = nullptr;
  __half* sc16 = nullptr;
  uint8_t* zp4 = nullptr;
  int64_t bytes = 0;
  int rc = alloc_plane(reinterpret_cast<void**>(&nib), rows * (size_t)w.nib_pitch, &bytes);
  if (rc == MSQ_OK) rc = alloc_plane(reinterpret_cast<void**>(&sc), rows * (size_t)w.sc_pitch * 4, &bytes);
  if (rc == MSQ_OK) rc = alloc_plane(reinterpret_cast<void**>(&sc16), rows * (size_t)w.sc_pitch * 2, &bytes);
  if (rc == MSQ_OK && w.zp_kind == ZP_PACKED)
    rc = alloc_plane(reinterpret_cast<void**>(&zp4), rows * (size_t)w.zp_pitch, &bytes);
  if (rc == MSQ_OK && w.zp_kind == ZP_F32)
    rc = alloc_plane(reinterpret_cast<void**>(&zpf), rows * (size_t)w.sc_pitch * 4, &bytes);
  const StreamGeo g{w.strm, w.kt, w.ntiles, w.stage_bytes, w.off_sc, w.off_zp, w.zp_kind, w.block_size};
  const int T = 256;
  if (rc == MSQ_OK) {
    const int64_t words = (int64_t)w.n_rows * (w.nib_pitch / 4);
    nib_from_stream_kernel<<<grid_for(words, T), T, 0, st>>>(g, w.n_rows, w.K, reinterpret_cast<uint32_t*>(nib),
                                                             w.nib_pitch / 4);
    const int64_t sn = (int64_t)w.n_rows * w.sc_pitch;
    scales_from_stream_kernel<<<grid_for(sn, T), T, 0, st>>>(g, w.n_rows, w.nb, sc, sc16, zpf, w.sc_pitch);
    note_launch(2);
    if (zp4) {
      const int64_t zn = (int64_t)w.n_rows * w.zp_pitch;
      zp_from_stream_kernel<<<grid_for(zn, T), T, 0, st>>>(g, w.n_rows, w.nb, zp4, w.zp_pitch);
      note_launch();
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_fail(e, "GEMM layout from the stream: launch");
  }
  if (rc != MSQ_OK) {
    for (void* q : {(void*)nib, (void*)sc, (void*)sc16, (void*)zp4, (void*)zpf})
      if (q) cudaFree(q);
    return rc;
  }
  w.sc = sc;
  w.sc16 = sc16;
  w.zp4 = zp4;
  w.zpf = zpf;
  w.nib = nib;
  w.device_bytes += bytes;
  w.gemm_layout.store(true, std::memory_order_release);
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
