/*
 * mnb_oracle.c -- CPU restatement of ModelSharp's MatMulNBits, used ONLY as the
 * parity checker (tests, __graft_entry__.smoke, and bench.py's cpu_baseline leg).
 * Nothing in the product library links or calls this file.
 *
 * Two references are provided:
 *
 *   mnb_ref_managed  follows the managed default path of
 *                    src/ModelSharp/Cpu/Kernels/Quantize/MatMulNBitsKernel.cs:216-262
 *                    (per column: per block, dequantise into a block scratch with
 *                    (q - zp) * scale, then FMA-accumulate the block against each
 *                    A row), with the accumulation order of
 *                    MatMulNBitsSimd.FmaAccumulate (MatMulNBitsSimd.cs:141-203,
 *                    AVX-512 branch: four 16-lane accumulators over 64-wide steps,
 *                    a 16-wide tail, a horizontal sum added to the scalar carried
 *                    across blocks, then a scalar tail) and the dequant of
 *                    MatMulNBitsSimd.DequantBlock4 (MatMulNBitsSimd.cs:40-96).
 *
 *   mnb_ref_f64      the dequant-then-double-dot reference of the reference's own
 *                    native self-test, native/test/qgemm_test.cpp:60-89.
 *
 * Both accept the three zero-point forms of MatMulNBitsKernel.cs:114-145:
 *   zp_kind 0 = absent (symmetric 2^(bits-1)), 1 = packed n-bit uint8 with row
 *   stride ceil(nb*bits/8) (low nibble = even block, MatMulNBitsKernel.cs:349-356),
 *   2 = float32 per (row, block).
 *
 * Build: gcc -O2 -mfma -ffp-contract=off -fopenmp -fPIC -shared (see Makefile).
 * -ffp-contract=off keeps the separate multiply and add of the scalar tail
 * (MatMulNBitsSimd.cs:201), while the vector lanes use explicit fmaf() as
 * Avx512F.FusedMultiplyAdd does.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* MatMulNBitsKernel.UnpackNBit, MatMulNBitsKernel.cs:349-356 */
static inline int unpack_nbit(const uint8_t* data, long base_byte, int index, int bits) {
    if (bits == 8) return data[base_byte + index];
    long byte_off = base_byte + (index >> 1);
    int shift = (index & 1) * 4;
    return (data[byte_off] >> shift) & 0x0F;
}

/* Horizontal sum of 4 lanes: (v0 + v1) + (v2 + v3). Vector512.Sum is taken as the
 * halving tree of 128-bit pair sums; the exact tree only moves the last ulp. */
static inline float hsum4(const float* v) { return (v[0] + v[1]) + (v[2] + v[3]); }
static inline float hsum16(const float* v) {
    float a = hsum4(v) + hsum4(v + 4);
    float b = hsum4(v + 8) + hsum4(v + 12);
    return a + b;
}

/* MatMulNBitsSimd.FmaAccumulate, AVX-512 branch (MatMulNBitsSimd.cs:141-162,201) */
static float fma_accumulate(float acc, const float* a, const float* w, int n) {
    int i = 0;
    if (n >= 16) {
        float s0[16] = {0}, s1[16] = {0}, s2[16] = {0}, s3[16] = {0}, s[16];
        int last4 = n - 64;
        for (; i <= last4; i += 64)
            for (int l = 0; l < 16; ++l) {
                s0[l] = fmaf(a[i + l], w[i + l], s0[l]);
                s1[l] = fmaf(a[i + 16 + l], w[i + 16 + l], s1[l]);
                s2[l] = fmaf(a[i + 32 + l], w[i + 32 + l], s2[l]);
                s3[l] = fmaf(a[i + 48 + l], w[i + 48 + l], s3[l]);
            }
        for (int l = 0; l < 16; ++l) s[l] = (s0[l] + s1[l]) + (s2[l] + s3[l]);
        int last = n - 16;
        for (; i <= last; i += 16)
            for (int l = 0; l < 16; ++l) s[l] = fmaf(a[i + l], w[i + l], s[l]);
        acc += hsum16(s);
    }
    for (; i < n; ++i) acc += a[i] * w[i];
    return acc;
}

static inline float zero_point(int zp_kind, const void* zp, long n, int nb, int zp_row_bytes,
                               int bk, int bits) {
    if (zp_kind == 1)
        return (float)unpack_nbit((const uint8_t*)zp, n * (long)zp_row_bytes, bk, bits);
    if (zp_kind == 2) return ((const float*)zp)[n * (long)nb + bk];
    return (float)(1 << (bits - 1)); /* MatMulNBitsKernel.cs:115 */
}

/* MatMulNBitsKernel.Execute default path, MatMulNBitsKernel.cs:193-262.
 * Returns 0, or -1 for arguments the reference rejects (bits, sizes). */
int mnb_ref_managed(const float* a, const uint8_t* b, const float* scales, int zp_kind,
                    const void* zp, float* y, int M, int N, int K, int bits, int block_size,
                    int nthreads) {
    if (N <= 0 || K <= 0 || block_size <= 0 || (bits != 4 && bits != 8) || M < 0) return -1;
    const int nb = (K + block_size - 1) / block_size;
    const int blob = (block_size * bits + 7) / 8;
    const int zp_row_bytes = (nb * bits + 7) / 8;
    const long b_row_bytes = (long)nb * blob;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
#pragma omp parallel
    {
        float* wblock = (float*)malloc(sizeof(float) * (size_t)block_size);
        float* acc = (float*)malloc(sizeof(float) * (size_t)(M > 0 ? M : 1));
#pragma omp for schedule(static)
        for (int n = 0; n < N; ++n) {
            for (int m = 0; m < M; ++m) acc[m] = 0.0f;
            for (int bk = 0; bk < nb; ++bk) {
                const float scale = scales[(long)n * nb + bk];
                const float z = zero_point(zp_kind, zp, n, nb, zp_row_bytes, bk, bits);
                const long blob_base = (long)n * b_row_bytes + (long)bk * blob;
                const int k_start = bk * block_size;
                int len = block_size < K - k_start ? block_size : K - k_start;
                if (len <= 0) break;
                /* DequantBlock4 / DequantBlock8: (q - zp) * scale, one rounding each */
                for (int i = 0; i < len; ++i) {
                    int q = unpack_nbit(b, blob_base, i, bits);
                    wblock[i] = ((float)q - z) * scale;
                }
                for (int m = 0; m < M; ++m)
                    acc[m] = fma_accumulate(acc[m], a + (long)m * K + k_start, wblock, len);
            }
            for (int m = 0; m < M; ++m) y[(long)m * N + n] = acc[m];
        }
        free(wblock);
        free(acc);
    }
    return 0;
}

/* native/test/qgemm_test.cpp:60-89: fp32 dequant into a K-length row, double dot. */
int mnb_ref_f64(const float* a, const uint8_t* b, const float* scales, int zp_kind,
                const void* zp, float* y, int M, int N, int K, int bits, int block_size,
                int nthreads) {
    if (N <= 0 || K <= 0 || block_size <= 0 || (bits != 4 && bits != 8) || M < 0) return -1;
    const int nb = (K + block_size - 1) / block_size;
    const int blob = (block_size * bits + 7) / 8;
    const int zp_row_bytes = (nb * bits + 7) / 8;
    const long b_row_bytes = (long)nb * blob;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
#pragma omp parallel
    {
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int n = 0; n < N; ++n) {
            for (int bk = 0; bk < nb; ++bk) {
                const float scale = scales[(long)n * nb + bk];
                const float z = zero_point(zp_kind, zp, n, nb, zp_row_bytes, bk, bits);
                const long blob_base = (long)n * b_row_bytes + (long)bk * blob;
                const int ks = bk * block_size;
                const int ke = ks + block_size < K ? ks + block_size : K;
                for (int k = ks; k < ke; ++k) {
                    int q = unpack_nbit(b, blob_base, k - ks, bits);
                    w[k] = ((float)q - z) * scale;
                }
            }
            for (int m = 0; m < M; ++m) {
                double s = 0.0;
                const float* arow = a + (long)m * K;
                for (int k = 0; k < K; ++k) s += (double)arow[k] * (double)w[k];
                y[(long)m * N + n] = (float)s;
            }
        }
        free(w);
    }
    return 0;
}

/* The dequantised weight matrix out[n][k] = (q - zp) * scale in fp32, one rounding each,
 * as DequantBlock4 / DequantBlock8 produce it block by block (MatMulNBitsSimd.cs:40-96);
 * used by the batched decoder checker, which multiplies whole matrices. */
int mnb_dequant(const uint8_t* b, const float* scales, int zp_kind, const void* zp, float* out,
                int N, int K, int bits, int block_size, int nthreads) {
    if (N <= 0 || K <= 0 || block_size <= 0 || (bits != 4 && bits != 8)) return -1;
    const int nb = (K + block_size - 1) / block_size;
    const int blob = (block_size * bits + 7) / 8;
    const int zp_row_bytes = (nb * bits + 7) / 8;
    const long b_row_bytes = (long)nb * blob;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        float* row = out + (long)n * K;
        for (int bk = 0; bk < nb; ++bk) {
            const float scale = scales[(long)n * nb + bk];
            const float z = zero_point(zp_kind, zp, n, nb, zp_row_bytes, bk, bits);
            const long blob_base = (long)n * b_row_bytes + (long)bk * blob;
            const int ks = bk * block_size;
            const int ke = ks + block_size < K ? ks + block_size : K;
            for (int k = ks; k < ke; ++k) row[k] = ((float)unpack_nbit(b, blob_base, k - ks, bits) - z) * scale;
        }
    }
    return 0;
}

/* ms_qgemm_w4a8, the reference's approximate int8-activation kernel
 * (native/src/qgemm_w4a8.cpp:247-292, scalar path :622-690): per (row m, K-block)
 * s_a = amax / 127, inv = 1 / s_a (0 for an all-zero block), aq = lrintf(a * inv) clamped to
 * [-127, 127]; weight codes centred wc = code - zp (clamped, a no-op at 4 bits); per block the
 * exact integer dot sum aq * wc, and y accumulates (s_a * s_w) * dot over the blocks in order.
 * Packed or absent zero points only (zp_kind 0 / 1), as the reference takes. */
int mnb_ref_w4a8(const float* a, const uint8_t* b, const float* scales, int zp_kind,
                 const void* zp, float* y, int M, int N, int K, int bits, int block_size,
                 int nthreads) {
    if (N <= 0 || K <= 0 || block_size <= 0 || (bits != 4 && bits != 8) || M < 0 || zp_kind == 2) return -1;
    const int nb = (K + block_size - 1) / block_size;
    const int blob = (block_size * bits + 7) / 8;
    const int zp_row_bytes = (nb * bits + 7) / 8;
    const long b_row_bytes = (long)nb * blob;
    const int padK = nb * block_size;
    int8_t* aq = (int8_t*)calloc((size_t)M * padK + 1, 1);
    float* sa = (float*)malloc(sizeof(float) * ((size_t)M * nb + 1));
    if (!aq || !sa) { free(aq); free(sa); return -1; }
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
    for (int m = 0; m < M; ++m)
        for (int bk = 0; bk < nb; ++bk) {
            const int k0 = bk * block_size, k1 = k0 + block_size < K ? k0 + block_size : K;
            float amax = 0.0f;
            for (int k = k0; k < k1; ++k) { float v = fabsf(a[(long)m * K + k]); if (v > amax) amax = v; }
            const float s = amax / 127.0f;
            sa[(long)m * nb + bk] = s;
            const float inv = s > 0.0f ? 1.0f / s : 0.0f;
            for (int k = k0; k < k1; ++k) {
                int q = (int)lrintf(a[(long)m * K + k] * inv);
                if (q > 127) q = 127; else if (q < -127) q = -127;
                aq[(long)m * padK + k] = (int8_t)q;
            }
        }
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        for (int m = 0; m < M; ++m) {
            float acc = 0.0f;
            for (int bk = 0; bk < nb; ++bk) {
                const int z = zp_kind == 1 ? unpack_nbit((const uint8_t*)zp, (long)n * zp_row_bytes, bk, bits)
                                           : (1 << (bits - 1));
                const long blob_base = (long)n * b_row_bytes + (long)bk * blob;
                const int k0 = bk * block_size, k1 = k0 + block_size < K ? k0 + block_size : K;
                int32_t dot = 0;
                for (int k = k0; k < k1; ++k) {
                    int wc = unpack_nbit(b, blob_base, k - k0, bits) - z;
                    if (wc > 127) wc = 127; else if (wc < -127) wc = -127;
                    dot += (int32_t)aq[(long)m * padK + k] * wc;
                }
                acc += sa[(long)m * nb + bk] * scales[(long)n * nb + bk] * (float)dot;
            }
            y[(long)m * N + n] = acc;
        }
    }
    free(aq);
    free(sa);
    return 0;
}
