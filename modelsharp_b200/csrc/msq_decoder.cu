// Decoder glue around MatMulNBits for one decode token, fp32 (sm_100a): the kernels a
// Llama-shaped decode step needs between its projections, each one launch, restating the
// reference's CPU kernels:
//   add_rmsnorm   x <- x + delta; y <- x / sqrt(mean(x^2) + eps) * gamma
//                 (SimplifiedLayerNormalizationKernel.cs:48-54, SkipSimplifiedLayerNormalizationKernel.cs:64-67)
//   rope_append   half-split rotary of q and k at the token's position, k and v appended to
//                 the KV cache (RotaryEmbeddingKernel.cs:96-114; GroupQueryAttentionKernel.cs present K/V)
//   gqa_decode    causal grouped-query attention of one query over the cache
//                 (GroupQueryAttentionKernel.cs:194-195, 275-312)
//   swiglu        silu(gate) * up
//   argmax        first index of the maximum; also advances the device-side position
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

// Split-K decode attention. A cluster of kGqaSplit blocks per kv head g; block r of the cluster
// takes keys [r C, (r + 1) C), C = ceil(T / kGqaSplit), for all G query heads of the group (the
// K and V rows are read once for the group). Per block and head: scores, local max m, local
// sum l of exp(score - m) and o = sum exp(score - m) v, kept in shared memory. After a cluster
// barrier every block combines a slice of the group's outputs from all blocks' (m, l, o) through
// distributed shared memory: out = sum_r o_r e^(m_r - M) / sum_r l_r e^(m_r - M), M = max m_r.
// A warp reads a key row as one float4 per lane (d <= 128 DV) and reduces the G dot products
// with shuffles. GM >= G is the compiled head-group size, DV = ceil(d / 128).
constexpr int kGqaSplit = 8;

// Score slots per head: the largest key slice rounded up to 4 floats, so that the float4
// regions after the scores start on 16-byte boundaries.
__host__ __device__ __forceinline__ int gqa_cmax(int64_t max_seq) {
  return (int)(((max_seq + kGqaSplit - 1) / kGqaSplit + 3) & ~int64_t(3));
}

template <int GM, int DV>
__global__ void gqa_decode_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                  const float* __restrict__ vc, const int64_t* __restrict__ pos_p,
                                  float* __restrict__ out, int G, int d, int64_t max_seq, float scale) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  extern __shared__ __align__(16) float sm[];
  const int cmax = gqa_cmax(max_seq);
  float* sc = sm;                      // [GM][cmax] scores, then probabilities
  float* part = sc + GM * cmax;        // [8 warps][G][d] partial sums of p v
  float* ob = part + 8 * G * d;        // [G][d] this block's o
  float* ml = ob + G * d;              // [G] m, then [G] l
  pdl_wait();
  pdl_trigger();
  const int r = (int)cl.block_rank();
  const int g = blockIdx.x / kGqaSplit;
  const int64_t pos = *pos_p;
  const int T = (int)(pos < 0 ? 0 : pos >= max_seq ? max_seq : pos + 1);  // keys 0..pos within the cache
  const int C = (T + kGqaSplit - 1) / kGqaSplit;
  const int lo = min(T, r * C), hi = min(T, lo + C), n = hi - lo;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const float* kb = kc + (int64_t)g * max_seq * d;
  const float* vb = vc + (int64_t)g * max_seq * d;

  float4 qr[GM][DV];
#pragma unroll
  for (int h = 0; h < GM; ++h)
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      const int c = 128 * j + 4 * l;
      qr[h][j] = (h < G && c < d) ? *reinterpret_cast<const float4*>(q + ((int64_t)g * G + h) * d + c)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  // scores: a warp per key
#pragma unroll 2
  for (int t = w; t < n; t += 8) {
    float4 kr[DV];
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      const int c = 128 * j + 4 * l;
      kr[j] = c < d ? *reinterpret_cast<const float4*>(kb + (int64_t)(lo + t) * d + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int h = 0; h < GM; ++h) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < DV; ++j) {
        acc = fmaf(qr[h][j].x, kr[j].x, acc);
        acc = fmaf(qr[h][j].y, kr[j].y, acc);
        acc = fmaf(qr[h][j].z, kr[j].z, acc);
        acc = fmaf(qr[h][j].w, kr[j].w, acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (l == 0 && h < G) sc[h * cmax + t] = acc * scale;
    }
  }
  __syncthreads();
  // local max and exponentials: warp h for head h
  for (int h = w; h < G; h += 8) {
    float mx = -FLT_MAX;
    for (int t = l; t < n; t += 32) mx = fmaxf(mx, sc[h * cmax + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int t = l; t < n; t += 32) {
      const float e = expf(sc[h * cmax + t] - mx);
      sc[h * cmax + t] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (l == 0) {
      ml[h] = mx;
      ml[G + h] = sum;  // 0 for an empty slice
    }
  }
  __syncthreads();
  // o = sum_t p_t v_t: warp w takes keys w, w + 8, ...
  float4 acc[GM][DV];
#pragma unroll
  for (int h = 0; h < GM; ++h)
#pragma unroll
    for (int j = 0; j < DV; ++j) acc[h][j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
  for (int t = w; t < n; t += 8) {
    float4 vr[DV];
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      const int c = 128 * j + 4 * l;
      vr[j] = c < d ? *reinterpret_cast<const float4*>(vb + (int64_t)(lo + t) * d + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int h = 0; h < GM; ++h) {
      const float pt = h < G ? sc[h * cmax + t] : 0.f;
#pragma unroll
      for (int j = 0; j < DV; ++j) {
        acc[h][j].x = fmaf(pt, vr[j].x, acc[h][j].x);
        acc[h][j].y = fmaf(pt, vr[j].y, acc[h][j].y);
        acc[h][j].z = fmaf(pt, vr[j].z, acc[h][j].z);
        acc[h][j].w = fmaf(pt, vr[j].w, acc[h][j].w);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < GM; ++h)
#pragma unroll
    for (int j = 0; j < DV; ++j) {
      const int c = 128 * j + 4 * l;
      if (h < G && c < d) *reinterpret_cast<float4*>(part + ((int64_t)w * G + h) * d + c) = acc[h][j];
    }
  __syncthreads();
  for (int i = threadIdx.x; i < G * d; i += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) v += part[k * G * d + i];
    ob[i] = v;
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

size_t gqa_decode_smem(int heads, int kv, int d, int64_t max_seq) {
  const int G = heads / kv;
  const int gm = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
  return sizeof(float) * (size_t)(gm * (int64_t)gqa_cmax(max_seq) + 9 * (int64_t)G * d + 2 * G);
}

template <int GM, int DV>
int launch_gqa(cudaStream_t st, const float* q, const float* kc, const float* vc, const int64_t* pos, float* out,
               int kv, int G, int d, int64_t max_seq) {
  const size_t smem = gqa_decode_smem(G * kv, kv, d, max_seq);
  auto kern = gqa_decode_kernel<GM, DV>;
  MSQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
               "gqa smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(kv * kGqaSplit));
  cfg.blockDim = dim3(256);
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
  MSQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, q, kc, vc, pos, out, G, d, max_seq, 1.0f / sqrtf((float)d)),
               "gqa_decode launch");
  note_launch();
  return MSQ_OK;
}

int run_gqa_decode(cudaStream_t st, const float* q, const float* kc, const float* vc, const int64_t* pos, float* out,
                   int heads, int kv, int d, int64_t max_seq) {
  const int G = heads / kv;
  if (d <= 128) {
    if (G <= 1) return launch_gqa<1, 1>(st, q, kc, vc, pos, out, kv, G, d, max_seq);
    if (G <= 2) return launch_gqa<2, 1>(st, q, kc, vc, pos, out, kv, G, d, max_seq);
    if (G <= 4) return launch_gqa<4, 1>(st, q, kc, vc, pos, out, kv, G, d, max_seq);
    return launch_gqa<8, 1>(st, q, kc, vc, pos, out, kv, G, d, max_seq);
  }
  if (G <= 1) return launch_gqa<1, 2>(st, q, kc, vc, pos, out, kv, G, d, max_seq);
  if (G <= 2) return launch_gqa<2, 2>(st, q, kc, vc, pos, out, kv, G, d, max_seq);
  if (G <= 4) return launch_gqa<4, 2>(st, q, kc, vc, pos, out, kv, G, d, max_seq);
  return launch_gqa<8, 2>(st, q, kc, vc, pos, out, kv, G, d, max_seq);
}

int run_swiglu(cudaStream_t st, const float* gu, float* out, int64_t n) {
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 4 * (int64_t)sms_now());
  return launch_pdl(st, dim3((unsigned)blocks), dim3(256), swiglu_kernel, "swiglu launch", gu, out, n);
}

int run_argmax(cudaStream_t st, const float* x, int64_t n, int64_t* idx, int64_t* pos) {
  return launch_pdl(st, dim3(1), dim3(1024), argmax_kernel, "argmax launch", x, n, idx, pos);
}

}  // namespace msq
