// Decoder glue around MatMulNBits for one decode token, fp32 (sm_100a): the kernels a
// Llama-shaped decode step needs between its projections, each one launch, restating the
// reference's CPU kernels:
//   add_rmsnorm   x <- x + delta; y <- x / sqrt(mean(x^2) + eps) * gamma
//                 (SimplifiedLayerNormalizationKernel.cs:48-54, SkipSimplifiedLayerNormalizationKernel.cs:64-67)
//   rope_append   half-split rotary of q and k at the token's position, k and v appended to
//                 the KV cache (RotaryEmbeddingKernel.cs:96-114; GroupQueryAttentionKernel.cs present K/V)
//   gqa_decode    causal grouped-query attention of one query over the cache
//                 (GroupQueryAttentionKernel.cs:194-195, 275-312); rope_gqa_decode also does
//                 rope_append's work for the current token
//   swiglu        silu(gate) * up
//   argmax        first index of the maximum; also advances the device-side position
// and the prompt forms for S tokens at once: rope_append_rows (rotary of S tokens at their
// positions, k and v to the cache), gqa_prefill (causal grouped-query attention of S queries
// over the cache), swiglu_rows.
// Positions are read from device memory so a decode step can be replayed from a CUDA graph.
// Every launch uses programmatic dependent launch: a kernel waits for its predecessor before
// reading, and lets the next kernel (typically a MatMulNBits GEMV that prefetches its
// weights) become resident early.
#include "msq_internal.cuh"

#include <algorithm>
#include <cfloat>

#include <cooperative_groups.h>

namespace msq {
namespace {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename F, typename... Args>
int launch_pdl(cudaStream_t st, dim3 grid, dim3 block, F kern, const char* what, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MSQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, args...), what);
  note_launch();
  return MSQ_OK;
}

// Block-wide sum over 256 threads, result in every thread.
__device__ __forceinline__ float block_sum256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = red[l & 7];  // every group of 8 lanes sums the 8 warp partials
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// One block (256 threads) per row.
__global__ void add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                   const float* __restrict__ gamma, float* __restrict__ y, int n, float eps) {
  __shared__ float red[8];
  pdl_wait();
  pdl_trigger();
  float* xr = x + (int64_t)blockIdx.x * n;
  const float* dr = delta ? delta + (int64_t)blockIdx.x * n : nullptr;
  float* yr = y + (int64_t)blockIdx.x * n;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += 256) {
    float v = xr[i];
    if (dr) {
      v += dr[i];
      xr[i] = v;
    }
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum256(ss, red);
  const float inv = 1.0f / sqrtf(tot / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += 256) yr[i] = xr[i] * inv * gamma[i];
}

// qkv = [q (heads*d) | k (kv*d) | v (kv*d)] of one token; pairs (j, j + d/2) of q and k heads
// rotate; k and v go to cache row *pos of every kv head ([kv][max_seq][d]).
__global__ void rope_append_kernel(float* __restrict__ qkv, int heads, int kv, int d, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, const int64_t* __restrict__ pos_p,
                                   float* __restrict__ kc, float* __restrict__ vc, int64_t max_seq) {
  pdl_wait();
  pdl_trigger();
  const int64_t pos = *pos_p;
  if (pos < 0 || pos >= max_seq) return;  // outside the cache and the rotary tables: nothing to do
  const int half = d / 2;
  const int pairs = (heads + kv) * half;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < pairs + kv * d; i += gridDim.x * blockDim.x) {
    if (i < pairs) {
      const int hh = i / half, j = i - hh * half;
      float* row = qkv + (int64_t)hh * d;  // k heads follow the q heads contiguously
      const float c = cos_t[pos * half + j], s = sin_t[pos * half + j];
      const float a = row[j], b = row[j + half];
      const float ra = a * c - b * s, rb = b * c + a * s;
      row[j] = ra;
      row[j + half] = rb;
      if (hh >= heads) {
        float* kr = kc + ((int64_t)(hh - heads) * max_seq + pos) * d;
        kr[j] = ra;
        kr[j + half] = rb;
      }
    } else {
      const int e = i - pairs, g = e / d, c = e - g * d;
      vc[((int64_t)g * max_seq + pos) * d + c] = qkv[(int64_t)(heads + kv) * d + e];
    }
  }
}

// Split-K decode attention. A cluster of kGqaSplit blocks per kv head g; block r takes cache
// keys [r C, (r + 1) C), C = ceil(Tc / kGqaSplit), for all G query heads of the group (each K
// and V row is read once for the group). Inside a block every warp keeps its own online
// softmax over the keys it takes (running max m, running sum l of exp(s - m), o = sum of
// exp(s - m) v), loading the K and V rows of KB keys at once so their latencies overlap; the
// warps are combined in shared memory, then, after a cluster barrier, every block combines a
// slice of the group's outputs from all blocks through distributed shared memory:
// out = sum_r o_r e^(m_r - M) / sum_r l_r e^(m_r - M), M = max m_r over non-empty parts.
// A lane holds one float4 of a d-row per 128 elements (DV = ceil(d / 128)).
//
// ROPE: q, k and v of the current token come unrotated from qkv = [q | k | v]; each block
// rotates its G query heads at position pos, and the cluster's last block rotates k, appends
// k and v to cache row pos and attends to them from registers (so no block reads a cache row
// this launch writes). Without ROPE, q is already rotated and keys 0..pos are all in the cache.
constexpr int kGqaSplit = 8;   // blocks per cluster: one cluster per kv head
constexpr int kGqaWarps = 16;  // warps per block

// The rotary table entries (cos, sin) of the elements 128 j + 4 l .. + 3 of a d-row at the
// table rows cs / sn (d / 2 entries each): element e uses entry e mod d/2.
template <int DV>
__device__ __forceinline__ void rope_tables4(float4 (&cv)[DV], float4 (&sv)[DV], int l, int d,
                                             const float* __restrict__ cs, const float* __restrict__ sn) {
  const int half = d >> 1;
#pragma unroll
  for (int j = 0; j < DV; ++j) {
    const int c = 128 * j + 4 * l;
    const int e = c < half ? c : c - half;
    cv[j] = c < d ? *reinterpret_cast<const float4*>(cs + e) : make_float4(0.f, 0.f, 0.f, 0.f);
    sv[j] = c < d ? *reinterpret_cast<const float4*>(sn + e) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Half-split rotary of the float4s x (elements 128 j + 4 l .. + 3 of a d-row) with their table
// entries cv / sv. Element e pairs with e + d/2 (first half) or e - d/2: for d <= 128 in lane
// l ^ (d / 8), for d = 256 in the other float4 of the same lane.
template <int DV>
__device__ __forceinline__ void rope4(float4 (&x)[DV], int l, int d, const float4 (&cvv)[DV],
                                      const float4 (&svv)[DV]) {
  const int half = d >> 1;
  float4 pr[DV];
  if constexpr (DV == 1) {
    const int o = d >> 3;
    pr[0].x = __shfl_xor_sync(0xffffffffu, x[0].x, o);
    pr[0].y = __shfl_xor_sync(0xffffffffu, x[0].y, o);
    pr[0].z = __shfl_xor_sync(0xffffffffu, x[0].z, o);
    pr[0].w = __shfl_xor_sync(0xffffffffu, x[0].w, o);
  } else {
    pr[0] = x[1];
    pr[1] = x[0];
  }
#pragma unroll
  for (int j = 0; j < DV; ++j) {
    const int c = 128 * j + 4 * l;
    if (c < d) {
      const bool first = c < half;
      const float4 cv = cvv[j], sv = svv[j];
      const float sg = first ? -1.f : 1.f;
      x[j] = make_float4(x[j].x * cv.x + sg * (pr[j].x * sv.x), x[j].y * cv.y + sg * (pr[j].y * sv.y),
                         x[j].z * cv.z + sg * (pr[j].z * sv.z), x[j].w * cv.w + sg * (pr[j].w * sv.w));
    }
  }
}

// One warp's online-softmax update with nv (>= 1) keys of a batch.
template <int GM, int DV, int KB>
__device__ __forceinline__ void attend_batch(const float4 (&qr)[GM][DV], const float4 (&kr)[KB][DV],
                                             const float4 (&vr)[KB][DV], int nv, float scale, float (&mw)[GM],
                                             float (&lw)[GM], float4 (&acc)[GM][DV]) {
  float sc[KB][GM];
#pragma unroll
  for (int i = 0; i < KB; ++i)
#pragma unroll
    for (int h = 0; h < GM; ++h) {
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < DV; ++j) {
        v = fmaf(qr[h][j].x, kr[i][j].x, v);
        v = fmaf(qr[h][j].y, kr[i][j].y, v);
        v = fmaf(qr[h][j].z, kr[i][j].z, v);
        v = fmaf(qr[h][j].w, kr[i][j].w, v);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      sc[i][h] = v * scale;
    }
#pragma unroll
  for (int h = 0; h < GM; ++h) {
    float bm = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < KB; ++i)
      if (i < nv) bm = fmaxf(bm, sc[i][h]);
    const float mn = fmaxf(mw[h], bm);
    const float alpha = expf(mw[h] - mn);  // 0 while the warp has seen no key (mw = -FLT_MAX)
    lw[h] *= alpha;
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      acc[h][j].x *= alpha;
      acc[h][j].y *= alpha;
      acc[h][j].z *= alpha;
      acc[h][j].w *= alpha;
    }
#pragma unroll
    for (int i = 0; i < KB; ++i) {
      const float pt = i < nv ? expf(sc[i][h] - mn) : 0.f;
      lw[h] += pt;
#pragma unroll
      for (int j = 0; j < DV; ++j) {
        acc[h][j].x = fmaf(pt, vr[i][j].x, acc[h][j].x);
        acc[h][j].y = fmaf(pt, vr[i][j].y, acc[h][j].y);
        acc[h][j].z = fmaf(pt, vr[i][j].z, acc[h][j].z);
        acc[h][j].w = fmaf(pt, vr[i][j].w, acc[h][j].w);
      }
    }
    mw[h] = mn;
  }
}

template <int GM, int DV, bool ROPE>
__global__ void __launch_bounds__(kGqaWarps * 32) gqa_decode_kernel(
    const float* __restrict__ q, float* kc, float* vc, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, const int64_t* __restrict__ pos_p, float* __restrict__ out, int heads, int kv,
    int d, int64_t max_seq, float scale) {
  constexpr int KB = GM * DV <= 4 ? 4 : GM * DV <= 8 ? 2 : 1;  // keys per warp batch (registers)
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int G = heads / kv;
  extern __shared__ __align__(16) float sm[];
  float* part = sm;                      // [warps][G][d] per-warp o
  float* wm = part + kGqaWarps * G * d;  // [warps][G] per-warp m
  float* wl = wm + kGqaWarps * G;        // [warps][G] per-warp l
  float* ob = wl + kGqaWarps * G;        // [G][d] this block's o
  float* ml = ob + G * d;                // [G] m, then [G] l of this block
  pdl_wait();
  pdl_trigger();
  const int r = (int)cl.block_rank();
  const int g = blockIdx.x / kGqaSplit;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int64_t pos = *pos_p;
  const bool cur = ROPE && pos >= 0 && pos < max_seq;  // the current token's k / v come from qkv
  const int T = (int)(pos < 0 ? 0 : pos >= max_seq ? max_seq : pos + 1);  // keys 0..pos within the cache
  const int Tc = cur ? T - 1 : T;                                        // of which read from the cache
  const int C = (Tc + kGqaSplit - 1) / kGqaSplit;
  const int lo = min(Tc, r * C), hi = min(Tc, lo + C);
  const float* kb = kc + (int64_t)g * max_seq * d;
  const float* vb = vc + (int64_t)g * max_seq * d;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const int half = d >> 1;

  // every load that does not depend on the cache is issued here, together
  const bool owner = cur && r == kGqaSplit - 1 && w == 0;  // rotates, appends and attends the current key
  float4 qr[GM][DV], cv[DV], sv[DV], kcur[DV], vcur[DV];
#pragma unroll
  for (int h = 0; h < GM; ++h)
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      const int c = 128 * j + 4 * l;
      qr[h][j] = (h < G && c < d) ? *reinterpret_cast<const float4*>(q + ((int64_t)g * G + h) * d + c) : z4;
    }
#pragma unroll
  for (int j = 0; j < DV; ++j) cv[j] = sv[j] = kcur[j] = vcur[j] = z4;
  if (cur) rope_tables4<DV>(cv, sv, l, d, cos_t + pos * half, sin_t + pos * half);
  if (owner) {
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      const int c = 128 * j + 4 * l;
      if (c < d) {
        kcur[j] = *reinterpret_cast<const float4*>(q + ((int64_t)heads + g) * d + c);
        vcur[j] = *reinterpret_cast<const float4*>(q + ((int64_t)heads + kv + g) * d + c);
      }
    }
  }
  if (cur) {
#pragma unroll
    for (int h = 0; h < GM; ++h) rope4<DV>(qr[h], l, d, cv, sv);
  }
  float mw[GM], lw[GM];
  float4 acc[GM][DV];
#pragma unroll
  for (int h = 0; h < GM; ++h) {
    mw[h] = -FLT_MAX;
    lw[h] = 0.f;
#pragma unroll
    for (int j = 0; j < DV; ++j) acc[h][j] = z4;
  }
  for (int t0 = lo + w * KB; t0 < hi; t0 += kGqaWarps * KB) {
    float4 kr[KB][DV], vr[KB][DV];
#pragma unroll
    for (int i = 0; i < KB; ++i)
#pragma unroll
      for (int j = 0; j < DV; ++j) {
        const int c = 128 * j + 4 * l;
        const bool ok = t0 + i < hi && c < d;
        kr[i][j] = ok ? *reinterpret_cast<const float4*>(kb + (int64_t)(t0 + i) * d + c) : z4;
        vr[i][j] = ok ? *reinterpret_cast<const float4*>(vb + (int64_t)(t0 + i) * d + c) : z4;
      }
    attend_batch<GM, DV, KB>(qr, kr, vr, min(KB, hi - t0), scale, mw, lw, acc);
  }
  if (owner) {  // the current key: rotate, append, attend
    float4 kr[KB][DV], vr[KB][DV];
#pragma unroll
    for (int i = 0; i < KB; ++i)
#pragma unroll
      for (int j = 0; j < DV; ++j) kr[i][j] = vr[i][j] = z4;
#pragma unroll
    for (int j = 0; j < DV; ++j) vr[0][j] = vcur[j];
    float4 k1[DV];
#pragma unroll
    for (int j = 0; j < DV; ++j) k1[j] = kcur[j];
    rope4<DV>(k1, l, d, cv, sv);
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      kr[0][j] = k1[j];
      const int c = 128 * j + 4 * l;
      if (c < d) {
        *reinterpret_cast<float4*>(kc + ((int64_t)g * max_seq + pos) * d + c) = k1[j];
        *reinterpret_cast<float4*>(vc + ((int64_t)g * max_seq + pos) * d + c) = vr[0][j];
      }
    }
    attend_batch<GM, DV, KB>(qr, kr, vr, 1, scale, mw, lw, acc);
  }
  // the warps' parts, then this block's (m, l, o)
#pragma unroll
  for (int h = 0; h < GM; ++h) {
    if (h < G) {
#pragma unroll
      for (int j = 0; j < DV; ++j) {
        const int c = 128 * j + 4 * l;
        if (c < d) *reinterpret_cast<float4*>(part + ((int64_t)w * G + h) * d + c) = acc[h][j];
      }
      if (l == 0) {
        wm[w * G + h] = mw[h];
        wl[w * G + h] = lw[h];
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * d; i += blockDim.x) {
    const int h = i / d;
    float M = -FLT_MAX;
#pragma unroll
    for (int k = 0; k < kGqaWarps; ++k)
      if (wl[k * G + h] > 0.f) M = fmaxf(M, wm[k * G + h]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int k = 0; k < kGqaWarps; ++k) {
      const float lk = wl[k * G + h];
      if (lk > 0.f) {
        const float f = expf(wm[k * G + h] - M);
        O = fmaf(part[(k * G + h) * d + (i - h * d)], f, O);
        L = fmaf(lk, f, L);
      }
    }
    ob[i] = O;
    if (i - h * d == 0) {
      ml[h] = M;
      ml[G + h] = L;
    }
  }
  cl.sync();  // every block's (m, l, o) is complete and visible to the cluster
  for (int i = r * blockDim.x + threadIdx.x; i < G * d; i += kGqaSplit * blockDim.x) {
    const int h = i / d;
    float M = -FLT_MAX;
#pragma unroll
    for (int k = 0; k < kGqaSplit; ++k) {
      const float* mlk = cl.map_shared_rank(ml, k);
      if (mlk[G + h] > 0.f) M = fmaxf(M, mlk[h]);
    }
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int k = 0; k < kGqaSplit; ++k) {
      const float* mlk = cl.map_shared_rank(ml, k);
      const float lk = mlk[G + h];
      if (lk > 0.f) {
        const float f = expf(mlk[h] - M);
        L = fmaf(lk, f, L);
        O = fmaf(cl.map_shared_rank(ob, k)[i], f, O);
      }
    }
    out[(int64_t)g * G * d + i] = L > 0.f ? O / L : 0.f;
  }
  cl.sync();  // peers may still read this block's shared memory until here
}

// gu = [gate (n) | up (n)] -> out = silu(gate) * up.
__global__ void swiglu_kernel(const float* __restrict__ gu, float* __restrict__ out, int64_t n) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gt = gu[i];
    out[i] = gt / (1.0f + expf(-gt)) * gu[n + i];
  }
}

// Rows of gu [rows][2n] = [gate | up] -> out [rows][n] = silu(gate) * up.
__global__ void swiglu_rows_kernel(const float* __restrict__ gu, float* __restrict__ out, int64_t rows, int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = rows * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n, c = i - r * n;
    const float gt = gu[2 * r * n + c];
    out[i] = gt / (1.0f + expf(-gt)) * gu[2 * r * n + n + c];
  }
}

// S tokens of qkv [S][(heads + 2 kv) d] (read only) at positions pos0 + s: the rotated q heads
// to q_out [S][heads d], the rotated k heads and the v heads to cache rows pos0 + s.
__global__ void rope_append_rows_kernel(const float* __restrict__ qkv, int64_t S, int64_t pos0, int heads, int kv,
                                        int d, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                        float* __restrict__ q_out, float* __restrict__ kc, float* __restrict__ vc,
                                        int64_t max_seq) {
  pdl_wait();
  pdl_trigger();
  const int half = d / 2;
  const int pairs = (heads + kv) * half;
  const int per = pairs + kv * d;  // work items of one token
  const int64_t width = (int64_t)(heads + 2 * kv) * d;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < S * per; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i / per;
    const int e = (int)(i - s * per);
    const int64_t pos = pos0 + s;
    const float* row = qkv + s * width;
    if (e < pairs) {
      const int hh = e / half, j = e - hh * half;
      const float c = cos_t[pos * half + j], sn = sin_t[pos * half + j];
      const float a = row[(int64_t)hh * d + j], b = row[(int64_t)hh * d + j + half];
      const float ra = a * c - b * sn, rb = b * c + a * sn;
      float* dst = hh < heads ? q_out + s * (int64_t)heads * d + (int64_t)hh * d
                              : kc + ((int64_t)(hh - heads) * max_seq + pos) * d;
      dst[j] = ra;
      dst[j + half] = rb;
    } else {
      const int v = e - pairs, g = v / d, c = v - g * d;
      vc[((int64_t)g * max_seq + pos) * d + c] = row[(int64_t)(heads + kv) * d + v];
    }
  }
}

// Causal grouped-query attention of S query tokens (positions pos0 .. pos0 + S - 1) over
// cache rows 0 .. pos0 + S - 1, fp32 throughout (the reference's softmax attention,
// GroupQueryAttentionKernel.cs:275-312, applied to every query token of a prompt).
// Block (x: 16 query tokens, y: kv head g) takes the R = 16 G rows (G query heads of the group
// x 16 tokens), so each K / V tile of 64 cache rows, staged in shared memory, serves all of them.
// Thread (rb = tid / 16, cg = tid % 16) owns rows rb G .. rb G + G - 1: their scores against keys
// cg + 16 j (j < 4) of the tile and their output elements 4 cg + 64 i .. + 3 (i < D / 64), with
// an online softmax per row (running max m, running sum l, output rescaled by e^(m_old - m_new));
// the 16 threads of a row group combine maxima and sums by shuffles. Row pitches of D + 4 floats
// keep the key reads of a quarter warp on distinct banks.
constexpr int kPfTok = 16;  // query tokens per block
constexpr int kPfKeys = 64;  // cache rows per tile

template <int G, int D>
__global__ void __launch_bounds__(256, 1) gqa_prefill_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                          const float* __restrict__ vc, float* __restrict__ out,
                                                          int64_t S, int64_t pos0, int heads, int64_t max_seq,
                                                          float scale) {
  constexpr int R = kPfTok * G, DP = D + 4, PP = kPfKeys + 4, DV = D / 64;
  extern __shared__ __align__(16) float sm[];
  float* Qs = sm;                   // [R][DP]
  float* Ks = Qs + R * DP;          // [kPfKeys][DP]
  float* Vs = Ks + kPfKeys * DP;    // [kPfKeys][DP]
  float* Ps = Vs + kPfKeys * DP;    // [R][PP]
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.y;
  const int64_t s0 = (int64_t)blockIdx.x * kPfTok;
  const int tid = threadIdx.x, rb = tid >> 4, cg = tid & 15;
  const int64_t ldq = (int64_t)heads * D;
  // row r: query head g G + r / 16 of token s0 + r % 16 (rows past S are zeros, never stored)
  for (int i = tid; i < R * (D / 4); i += 256) {
    const int r = i / (D / 4), c4 = i - r * (D / 4);
    const int64_t s = s0 + (r & 15);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s < S) v = *reinterpret_cast<const float4*>(q + s * ldq + (int64_t)(g * G + (r >> 4)) * D + 4 * c4);
    *reinterpret_cast<float4*>(Qs + r * DP + 4 * c4) = v;
  }
  float m[G], l[G];
  float4 o[G][DV];
#pragma unroll
  for (int i = 0; i < G; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int v = 0; v < DV; ++v) o[i][v] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const int64_t pmax = pos0 + min(s0 + kPfTok, S) - 1;  // the last position a row of this block sees
  const int ntile = (int)(pmax / kPfKeys) + 1;
  const float* kg = kc + (int64_t)g * max_seq * D;
  const float* vg = vc + (int64_t)g * max_seq * D;
  for (int t = 0; t < ntile; ++t) {
    const int64_t k0 = (int64_t)t * kPfKeys;
    __syncthreads();  // the previous tile's K, V and P are no longer read (and Q is in place)
    for (int i = tid; i < kPfKeys * (D / 4); i += 256) {
      const int kr = i / (D / 4), c4 = i - kr * (D / 4);
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
      if (k0 + kr <= pmax) {
        kv4 = *reinterpret_cast<const float4*>(kg + (k0 + kr) * D + 4 * c4);
        vv4 = *reinterpret_cast<const float4*>(vg + (k0 + kr) * D + 4 * c4);
      }
      *reinterpret_cast<float4*>(Ks + kr * DP + 4 * c4) = kv4;
      *reinterpret_cast<float4*>(Vs + kr * DP + 4 * c4) = vv4;
    }
    __syncthreads();
    float sc[G][4];
#pragma unroll
    for (int i = 0; i < G; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
    for (int c = 0; c < D; c += 4) {
      float4 kv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(Ks + (cg + 16 * j) * DP + c);
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const float4 qv = *reinterpret_cast<const float4*>(Qs + (rb * G + i) * DP + c);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          sc[i][j] = fmaf(qv.w, kv[j].w, fmaf(qv.z, kv[j].z, fmaf(qv.y, kv[j].y, fmaf(qv.x, kv[j].x, sc[i][j]))));
      }
    }
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int r = rb * G + i;
      const int64_t pr = pos0 + s0 + (r & 15);  // this row's position: keys 0 .. pr are visible
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float v = k0 + cg + 16 * j <= pr ? sc[i][j] * scale : -INFINITY;
        sc[i][j] = v;
        mx = fmaxf(mx, v);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[i], mx);  // finite: key 0 is visible to every row in tile 0
      const float alpha = expf(m[i] - mn);  // 0 on the first tile (m = -inf)
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pj = expf(sc[i][j] - mn);
        Ps[r * PP + cg + 16 * j] = pj;
        ps += pj;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[i] = fmaf(l[i], alpha, ps);
      m[i] = mn;
#pragma unroll
      for (int v = 0; v < DV; ++v) {
        o[i][v].x *= alpha;
        o[i][v].y *= alpha;
        o[i][v].z *= alpha;
        o[i][v].w *= alpha;
      }
    }
    __syncthreads();  // P of every row is in shared memory
    const int kn = (int)min((int64_t)kPfKeys, pmax - k0 + 1);
    for (int key = 0; key < kn; ++key) {
      float4 vv[DV];
#pragma unroll
      for (int v = 0; v < DV; ++v) vv[v] = *reinterpret_cast<const float4*>(Vs + key * DP + 4 * cg + 64 * v);
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const float pk = Ps[(rb * G + i) * PP + key];
#pragma unroll
        for (int v = 0; v < DV; ++v) {
          o[i][v].x = fmaf(pk, vv[v].x, o[i][v].x);
          o[i][v].y = fmaf(pk, vv[v].y, o[i][v].y);
          o[i][v].z = fmaf(pk, vv[v].z, o[i][v].z);
          o[i][v].w = fmaf(pk, vv[v].w, o[i][v].w);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int r = rb * G + i;
    const int64_t s = s0 + (r & 15);
    if (s >= S) continue;
    const float inv = 1.0f / l[i];
    float* dst = out + s * ldq + (int64_t)(g * G + (r >> 4)) * D + 4 * cg;
#pragma unroll
    for (int v = 0; v < DV; ++v)
      *reinterpret_cast<float4*>(dst + 64 * v) =
          make_float4(o[i][v].x * inv, o[i][v].y * inv, o[i][v].z * inv, o[i][v].w * inv);
  }
}

// One block (1024 threads): first index of the maximum into *idx (NaNs never win; with no
// element above -FLT_MAX the index is 0); *pos += 1 when pos is given.
__global__ void argmax_kernel(const float* __restrict__ x, int64_t n, int64_t* __restrict__ idx,
                              int64_t* __restrict__ pos) {
  __shared__ float bv[32];
  __shared__ int64_t bi[32];
  pdl_wait();
  pdl_trigger();
  float v = -FLT_MAX;
  int64_t k = n;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float xi = x[i];
    if (xi > v) {
      v = xi;
      k = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int64_t ok = __shfl_xor_sync(0xffffffffu, k, o);
    if (ov > v || (ov == v && ok < k)) {
      v = ov;
      k = ok;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    bv[w] = v;
    bi[w] = k;
  }
  __syncthreads();
  if (w == 0) {
    v = l < (int)(blockDim.x >> 5) ? bv[l] : -FLT_MAX;
    k = l < (int)(blockDim.x >> 5) ? bi[l] : n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int64_t ok = __shfl_xor_sync(0xffffffffu, k, o);
      if (ov > v || (ov == v && ok < k)) {
        v = ov;
        k = ok;
      }
    }
    if (l == 0) {
      *idx = k < n ? k : 0;  // no element above -FLT_MAX (all -inf or NaN): index 0, always in range
      if (pos) *pos += 1;
    }
  }
}

int sms_now() {
  int dev = 0;
  cudaGetDevice(&dev);
  return num_sms(dev);
}

}  // namespace

int run_add_rmsnorm(cudaStream_t st, float* x, const float* delta, const float* gamma, float* y, int64_t rows,
                    int64_t n, float eps) {
  return launch_pdl(st, dim3((unsigned)rows), dim3(256), add_rmsnorm_kernel, "add_rmsnorm launch", x, delta, gamma,
                    y, (int)n, eps);
}

int run_rope_append(cudaStream_t st, float* qkv, int heads, int kv, int d, const float* cos_t, const float* sin_t,
                    const int64_t* pos, float* kc, float* vc, int64_t max_seq) {
  const int work = (heads + kv) * (d / 2) + kv * d;
  return launch_pdl(st, dim3((unsigned)((work + 255) / 256)), dim3(256), rope_append_kernel, "rope_append launch", qkv,
                    heads, kv, d, cos_t, sin_t, pos, kc, vc, max_seq);
}

size_t gqa_decode_smem(int heads, int kv, int d) {
  const int64_t G = heads / kv;
  return sizeof(float) * (size_t)(kGqaWarps * G * d + 2 * kGqaWarps * G + G * d + 2 * G);
}

template <int GM, int DV, bool ROPE>
int launch_gqa(cudaStream_t st, const float* q, float* kc, float* vc, const float* cos_t, const float* sin_t,
               const int64_t* pos, float* out, int heads, int kv, int d, int64_t max_seq) {
  const size_t smem = gqa_decode_smem(heads, kv, d);
  auto kern = gqa_decode_kernel<GM, DV, ROPE>;
  if (smem > 48 * 1024)
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "gqa smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(kv * kGqaSplit));
  cfg.blockDim = dim3(kGqaWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kGqaSplit;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  MSQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, q, kc, vc, cos_t, sin_t, pos, out, heads, kv, d, max_seq,
                                  1.0f / sqrtf((float)d)),
               "gqa_decode launch");
  note_launch();
  return MSQ_OK;
}

template <bool ROPE>
int dispatch_gqa(cudaStream_t st, const float* q, float* kc, float* vc, const float* cos_t, const float* sin_t,
                 const int64_t* pos, float* out, int heads, int kv, int d, int64_t max_seq) {
  const int G = heads / kv;
#define MSQ_GQA(GM, DV) launch_gqa<GM, DV, ROPE>(st, q, kc, vc, cos_t, sin_t, pos, out, heads, kv, d, max_seq)
  if (d <= 128) {
    if (G <= 1) return MSQ_GQA(1, 1);
    if (G <= 2) return MSQ_GQA(2, 1);
    if (G <= 4) return MSQ_GQA(4, 1);
    return MSQ_GQA(8, 1);
  }
  if (G <= 1) return MSQ_GQA(1, 2);
  if (G <= 2) return MSQ_GQA(2, 2);
  if (G <= 4) return MSQ_GQA(4, 2);
  return MSQ_GQA(8, 2);
#undef MSQ_GQA
}

int run_gqa_decode(cudaStream_t st, const float* q, const float* kc, const float* vc, const int64_t* pos, float* out,
                   int heads, int kv, int d, int64_t max_seq) {
  // without ROPE the kernel never writes the caches
  return dispatch_gqa<false>(st, q, const_cast<float*>(kc), const_cast<float*>(vc), nullptr, nullptr, pos, out,
                             heads, kv, d, max_seq);
}

int run_rope_gqa_decode(cudaStream_t st, const float* qkv, float* kc, float* vc, const float* cos_t,
                        const float* sin_t, const int64_t* pos, float* out, int heads, int kv, int d,
                        int64_t max_seq) {
  return dispatch_gqa<true>(st, qkv, kc, vc, cos_t, sin_t, pos, out, heads, kv, d, max_seq);
}

int run_swiglu(cudaStream_t st, const float* gu, float* out, int64_t n) {
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 4 * (int64_t)sms_now());
  return launch_pdl(st, dim3((unsigned)blocks), dim3(256), swiglu_kernel, "swiglu launch", gu, out, n);
}

int run_argmax(cudaStream_t st, const float* x, int64_t n, int64_t* idx, int64_t* pos) {
  return launch_pdl(st, dim3(1), dim3(1024), argmax_kernel, "argmax launch", x, n, idx, pos);
}

int run_swiglu_rows(cudaStream_t st, const float* gu, float* out, int64_t rows, int64_t n) {
  const int64_t blocks = std::min<int64_t>((rows * n + 255) / 256, 8 * (int64_t)sms_now());
  return launch_pdl(st, dim3((unsigned)blocks), dim3(256), swiglu_rows_kernel, "swiglu_rows launch", gu, out, rows, n);
}

int run_rope_append_rows(cudaStream_t st, const float* qkv, int64_t S, int64_t pos0, int heads, int kv, int d,
                         const float* cos_t, const float* sin_t, float* q_out, float* kc, float* vc, int64_t max_seq) {
  const int64_t work = S * ((int64_t)(heads + kv) * (d / 2) + (int64_t)kv * d);
  const int64_t blocks = std::min<int64_t>((work + 255) / 256, 8 * (int64_t)sms_now());
  return launch_pdl(st, dim3((unsigned)blocks), dim3(256), rope_append_rows_kernel, "rope_append_rows launch", qkv, S,
                    pos0, heads, kv, d, cos_t, sin_t, q_out, kc, vc, max_seq);
}

namespace {
template <int G, int D>
int launch_prefill(cudaStream_t st, const float* q, const float* kc, const float* vc, float* out, int64_t S,
                   int64_t pos0, int heads, int kv, int64_t max_seq) {
  constexpr size_t smem = sizeof(float) * ((size_t)(kPfTok * G + 2 * kPfKeys) * (D + 4) + (size_t)kPfTok * G * (kPfKeys + 4));
  static_assert(smem <= 227 * 1024, "prefill attention tile exceeds shared memory");
  auto kern = gqa_prefill_kernel<G, D>;
  static ContextOnce configured;
  const int rc = configured.run([&] {
    MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "gqa_prefill smem attribute");
    return MSQ_OK;
  });
  if (rc != MSQ_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((S + kPfTok - 1) / kPfTok), (unsigned)kv);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MSQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, q, kc, vc, out, S, pos0, heads, max_seq, 1.0f / sqrtf((float)D)),
               "gqa_prefill launch");
  note_launch();
  return MSQ_OK;
}

template <int D>
int prefill_g(cudaStream_t st, int G, const float* q, const float* kc, const float* vc, float* out, int64_t S,
              int64_t pos0, int heads, int kv, int64_t max_seq) {
  switch (G) {
    case 1: return launch_prefill<1, D>(st, q, kc, vc, out, S, pos0, heads, kv, max_seq);
    case 2: return launch_prefill<2, D>(st, q, kc, vc, out, S, pos0, heads, kv, max_seq);
    case 3: return launch_prefill<3, D>(st, q, kc, vc, out, S, pos0, heads, kv, max_seq);
    case 4: return launch_prefill<4, D>(st, q, kc, vc, out, S, pos0, heads, kv, max_seq);
    case 5: return launch_prefill<5, D>(st, q, kc, vc, out, S, pos0, heads, kv, max_seq);
    case 6: return launch_prefill<6, D>(st, q, kc, vc, out, S, pos0, heads, kv, max_seq);
    case 7: return launch_prefill<7, D>(st, q, kc, vc, out, S, pos0, heads, kv, max_seq);
    default: return launch_prefill<8, D>(st, q, kc, vc, out, S, pos0, heads, kv, max_seq);
  }
}
}  // namespace

int run_gqa_prefill(cudaStream_t st, const float* q, const float* kc, const float* vc, float* out, int64_t S,
                    int64_t pos0, int heads, int kv, int d, int64_t max_seq) {
  const int G = heads / kv;
  return d == 64 ? prefill_g<64>(st, G, q, kc, vc, out, S, pos0, heads, kv, max_seq)
                 : prefill_g<128>(st, G, q, kc, vc, out, S, pos0, heads, kv, max_seq);
}

}  // namespace msq
