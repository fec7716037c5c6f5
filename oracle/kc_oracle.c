/*
 * kc_oracle.c -- CPU restatement of kernel-craft's quantized-linear hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle: the tests, the
 * smoke check and the bench's CPU-baseline leg call it as the checker.  The
 * product library (kernel-craft_b200/) never links, loads or calls it.
 *
 * Parity pins (see tests/test_oracle_golden.py):
 *   - the known-answer tests of the reference's own C++ and pytest suites
 *     (tests/test_quant_int4.cpp, src/python/tests/test_transformer_bindings.py,
 *     src/python/tests/test_triton_kernels.py) re-generated as fixtures under
 *     tests/golden/ by tests/golden/make_golden.py;
 *   - outputs of the reference's own CUDA kernels, built from its sources by
 *     oracle/build_ref.sh into oracle/_ref/libkcref.so and run on a B200 by
 *     tests/golden/make_golden_ref.py (fixtures tests/golden/ref_*.npz);
 *   - the E4M3 encoder below against torch's independent CPU float8 cast.
 *
 * Every function names the reference file:line whose arithmetic it restates.
 * Operation order follows the reference where it changes the bits (division
 * x/scale, fminf/fmaxf clamp, (float)(int) * scale dequant).  Reductions whose
 * order the reference leaves to the hardware (GEMV, GEMM) are done in double.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stddef.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORA_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* INT4 nibble unpack: quant_int4.cu:34-38 (low) and :45-48 (high).          */
/* Sign-extend a 4-bit two's-complement value to int8.                      */
/* ------------------------------------------------------------------------- */
static inline int ora_sx4_lo(uint8_t p) {
    int v = p & 0x0F;
    return (v & 0x08) ? (v - 16) : v;
}
static inline int ora_sx4_hi(uint8_t p) {
    int v = (p >> 4) & 0x0F;
    return (v & 0x08) ? (v - 16) : v;
}

ORA_EXPORT int ora_unpack_nibble(uint8_t p, int high) {
    return high ? ora_sx4_hi(p) : ora_sx4_lo(p);
}

/* Zero-point of group g in row r: quant_int4.cu:93-96.  The byte index uses
 * the reference's floor(cols/group_size/2) row stride verbatim, and the nibble
 * is read UNSIGNED (0..15). */
static inline int ora_zp(const uint8_t* zeros, int row, int cols, int gs, int g) {
    int zc = cols / gs / 2;
    uint8_t zb = zeros[(long)row * zc + g / 2];
    return (g % 2 == 0) ? (zb & 0x0F) : (zb >> 4);
}

/* launch_dequantize_int4 / dequantize_int4_kernel: quant_int4.cu:68-105.
 * out[r,c] = (float)(sx4(nibble) - zp) * scales[r*(cols/gs) + c/gs]. */
ORA_EXPORT void ora_dequantize_int4(const uint8_t* packed, const float* scales,
                                    const uint8_t* zeros, float* out,
                                    int rows, int cols, int gs) {
    int sc = cols / gs;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        for (int b = 0; 2 * b < cols; ++b) {
            int c0 = 2 * b, c1 = c0 + 1;
            uint8_t p = packed[(long)r * (cols / 2) + b];
            int g0 = c0 / gs, g1 = c1 / gs;
            float s0 = scales[(long)r * sc + g0];
            float s1 = scales[(long)r * sc + g1];
            int z0 = ora_zp(zeros, r, cols, gs, g0);
            int z1 = ora_zp(zeros, r, cols, gs, g1);
            out[(long)r * cols + c0] = (float)(ora_sx4_lo(p) - z0) * s0;
            if (c1 < cols)
                out[(long)r * cols + c1] = (float)(ora_sx4_hi(p) - z1) * s1;
        }
    }
}

/* launch_gemv_int4 / gemv_int4_kernel: quant_int4.cu:126-175.
 * y[r] = sum_c w(r,c) * x[c] with w exactly as the dequant above.
 * Accumulated in double (the reference's fp32 tree order is hardware-defined;
 * parity is judged against this with a tolerance). */
ORA_EXPORT void ora_gemv_int4(const uint8_t* packed, const float* scales,
                              const uint8_t* zeros, const float* x, float* y,
                              int rows, int cols, int gs) {
    int sc = cols / gs;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        double acc = 0.0;
        for (int b = 0; 2 * b < cols; ++b) {
            int c0 = 2 * b, c1 = c0 + 1;
            uint8_t p = packed[(long)r * (cols / 2) + b];
            int g0 = c0 / gs, g1 = c1 / gs;
            float w0 = (float)(ora_sx4_lo(p) - ora_zp(zeros, r, cols, gs, g0)) * scales[(long)r * sc + g0];
            acc += (double)w0 * (double)x[c0];
            if (c1 < cols) {
                float w1 = (float)(ora_sx4_hi(p) - ora_zp(zeros, r, cols, gs, g1)) * scales[(long)r * sc + g1];
                acc += (double)w1 * (double)x[c1];
            }
        }
        y[r] = (float)acc;
    }
}

/* ------------------------------------------------------------------------- */
/* GPTQ implicit-zero-point-8 variant (the new bf16/fp16 API).               */
/* w = (u - 8) * s with u the UNSIGNED nibble.  Identity used for parity     */
/* with the reference formula: (u - 8) == sx4(u ^ 8) - 0, i.e. the reference */
/* launch_dequantize_int4(packed ^ 0x88, float(scales), zeros = 0) produces   */
/* the same fp32 weights (quant_int4.cu:99-104).                              */
/* ------------------------------------------------------------------------- */
static inline float ora_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    int exp = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) { bits = sign; }
        else {               /* subnormal: value = man * 2^-24 */
            float f = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((uint32_t)(exp - 15 + 127) << 23) | (man << 13);
    }
    float f; memcpy(&f, &bits, 4);
    return f;
}

static inline float ora_bf16_to_float(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f; memcpy(&f, &bits, 4);
    return f;
}

/* Round-to-nearest-even fp32 -> bf16 (NaN kept quiet). */
ORA_EXPORT uint16_t ora_float_to_bf16(float f) {
    uint32_t bits; memcpy(&bits, &f, 4);
    if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu))
        return (uint16_t)((bits >> 16) | 0x0040);
    uint32_t lsb = (bits >> 16) & 1u;
    bits += 0x7FFFu + lsb;
    return (uint16_t)(bits >> 16);
}

ORA_EXPORT float ora_gptq_weight(uint8_t p, int high, uint16_t scale_f16) {
    int u = high ? ((p >> 4) & 0xF) : (p & 0xF);
    return (float)(u - 8) * ora_half_to_float(scale_f16);
}

/* bf16 dequant of W4 weights with per-group zero points (AWQ, asymmetric
 * GPTQ): out[r,c] = bf16_rne((u - z) * float(s_f16)), z = zeros[r, c/gs]
 * (one byte per group, 0..15); zeros == NULL is the symmetric GPTQ case z = 8,
 * the reference's dequantize_int4 of packed ^ 0x88 with zero points 0
 * (quant_int4.cu:99-104). */
static int ora_w4_zp(const uint8_t* zeros, long row, int sc, int g) {
    return zeros ? (int)(zeros[row * sc + g] & 0xF) : 8;
}

ORA_EXPORT void ora_dequantize_w4_bf16_zp(const uint8_t* packed, const uint16_t* scales_f16,
                                          const uint8_t* zeros, uint16_t* out, int rows, int cols,
                                          int gs) {
    int sc = cols / gs;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) {
            uint8_t p = packed[(long)r * (cols / 2) + c / 2];
            int u = (c & 1) ? ((p >> 4) & 0xF) : (p & 0xF);
            float w = (float)(u - ora_w4_zp(zeros, r, sc, c / gs)) *
                      ora_half_to_float(scales_f16[(long)r * sc + c / gs]);
            out[(long)r * cols + c] = ora_float_to_bf16(w);
        }
}

ORA_EXPORT void ora_dequantize_w4_bf16(const uint8_t* packed, const uint16_t* scales_f16,
                                       uint16_t* out, int rows, int cols, int gs) {
    ora_dequantize_w4_bf16_zp(packed, scales_f16, NULL, out, rows, cols, gs);
}

/* W4A16 GEMV, y[m,n] = sum_k w[n,k] x[m,k] with w = (u - z) * s as above,
 * accumulated in double (the truth the kernels are checked against). */
ORA_EXPORT void ora_gemv_w4a16_zp(const uint8_t* packed, const uint16_t* scales_f16,
                                  const uint8_t* zeros, const uint16_t* x_bf16, float* y,
                                  int M, int N, int K, int gs) {
    int sc = K / gs;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < N; ++r) {
        double* acc = (double*)calloc((size_t)M, sizeof(double));
        int mm = M;
        for (int g = 0; g < sc; ++g) {
            float s = ora_half_to_float(scales_f16[(long)r * sc + g]);
            int z = ora_w4_zp(zeros, r, sc, g);
            for (int c = g * gs; c < (g + 1) * gs; ++c) {
                uint8_t p = packed[(long)r * (K / 2) + c / 2];
                int u = (c & 1) ? (p >> 4) : (p & 0xF);
                double w = (double)((float)(u - z) * s);
                for (int m = 0; m < mm; ++m)
                    acc[m] += w * (double)ora_bf16_to_float(x_bf16[(long)m * K + c]);
            }
        }
        for (int m = 0; m < mm; ++m) y[(long)m * N + r] = (float)acc[m];
        free(acc);
    }
}

ORA_EXPORT void ora_gemv_w4a16(const uint8_t* packed, const uint16_t* scales_f16,
                               const uint16_t* x_bf16, float* y,
                               int M, int N, int K, int gs) {
    ora_gemv_w4a16_zp(packed, scales_f16, NULL, x_bf16, y, M, N, K, gs);
}

/* ------------------------------------------------------------------------- */
/* FP8 E4M3.  Encoder written from the OCP 8-bit floating point spec (E4M3:   */
/* bias 7, 3 mantissa bits, no infinities, S.1111.111 = NaN, max 448):        */
/* round-to-nearest-even, saturating finite values to +-448 (the SATFINITE    */
/* mode the reference selects through __nv_fp8_e4m3, fp8_quant.cu:73,128).   */
/* ------------------------------------------------------------------------- */
ORA_EXPORT uint8_t ora_e4m3_encode(float v) {
    uint32_t bits; memcpy(&bits, &v, 4);
    uint8_t sign = (uint8_t)((bits >> 24) & 0x80);
    if (isnan(v)) return (uint8_t)(sign | 0x7F);
    float a = fabsf(v);
    if (a >= 0.015625f) {                       /* >= 2^-6: e4m3 normal range */
        uint32_t ab; memcpy(&ab, &a, 4);
        int e = (int)((ab >> 23) & 0xFF) - 127;  /* unbiased exponent (>= -6) */
        uint32_t m23 = ab & 0x7FFFFFu;
        uint32_t keep = m23 >> 20, rest = m23 & 0xFFFFFu;
        if (rest > 0x80000u || (rest == 0x80000u && (keep & 1u))) keep += 1;
        if (keep == 8) { keep = 0; e += 1; }
        if (e > 8 || (e == 8 && keep == 7)) return (uint8_t)(sign | 0x7E); /* sat 448 */
        return (uint8_t)(sign | ((uint32_t)(e + 7) << 3) | keep);
    }
    /* subnormal range: units of 2^-9, RNE on the exact scaled value */
    float q = a * 512.0f;                        /* exact (power-of-two scale) */
    float r = nearbyintf(q);                     /* default mode: ties-to-even */
    return (uint8_t)(sign | (uint8_t)r);         /* r in 0..8; 8 == min normal */
}

ORA_EXPORT float ora_e4m3_decode(uint8_t c) {
    int sign = c & 0x80, e = (c >> 3) & 0xF, m = c & 7;
    float v;
    if (e == 0xF && m == 7) return sign ? -NAN : NAN;
    if (e == 0) v = (float)m * 0.001953125f;           /* m * 2^-9 */
    else        v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return sign ? -v : v;
}

/* Clamp exactly as fp8_quant.cu:72,127: fmaxf(-448, fminf(448, s)).  NaN -> +448. */
static inline float ora_clamp448(float s) {
    return fmaxf(-448.0f, fminf(448.0f, s));
}

/* Bulk encoder used by the tests: codes[i] = e4m3(clamp(in[i])). */
ORA_EXPORT void ora_e4m3_encode_array(const float* in, uint8_t* out, long n, int clamp) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i)
        out[i] = ora_e4m3_encode(clamp ? ora_clamp448(in[i]) : in[i]);
}

/* quantize_fp8_per_token_kernel: fp8_quant.cu:89-131.
 * amax over |x| with fmaxf starting at 0 (NaN ignored, :103-105);
 * scale = amax > 0 ? amax / 448 : 1 (:121); q = e4m3(clamp(x / scale)) (:126-129). */
ORA_EXPORT void ora_quantize_fp8_per_token(const float* in, uint8_t* out, float* scales,
                                           int rows, int cols) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float* x = in + (long)r * cols;
        float amax = 0.0f;
        for (int c = 0; c < cols; ++c) amax = fmaxf(amax, fabsf(x[c]));
        float scale = (amax > 0.0f) ? (amax / 448.0f) : 1.0f;
        scales[r] = scale;
        for (int c = 0; c < cols; ++c)
            out[(long)r * cols + c] = ora_e4m3_encode(ora_clamp448(x[c] / scale));
    }
}

/* quantize_fp8_per_tensor_kernel: fp8_quant.cu:62-75 with the caller's scale. */
ORA_EXPORT void ora_quantize_fp8_per_tensor(const float* in, uint8_t* out, float scale, long n) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i)
        out[i] = ora_e4m3_encode(ora_clamp448(in[i] / scale));
}

/* dequantize_fp8_kernel: fp8_quant.cu:145-160.  x = float(e4m3) * scale[row or 0]. */
ORA_EXPORT void ora_dequantize_fp8(const uint8_t* in, const float* scales, float* out,
                                   int rows, int cols, int per_token) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        float s = per_token ? scales[r] : scales[0];
        for (int c = 0; c < cols; ++c)
            out[(long)r * cols + c] = ora_e4m3_decode(in[(long)r * cols + c]) * s;
    }
}

/* smoothquant_scale_kernel: fp8_quant.cu:174-184.  out = x / s[col] (IEEE). */
ORA_EXPORT void ora_smoothquant_scale(const float* in, const float* s, float* out,
                                      int rows, int cols) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c)
            out[(long)r * cols + c] = in[(long)r * cols + c] / s[c];
}

/* ------------------------------------------------------------------------- */
/* GEMM and the simulated collectives.                                        */
/* ------------------------------------------------------------------------- */

/* sgemm_nt_kernel: tensor_parallel.cu:164-192.  C[M,N] = A[M,K] * B[N,K]^T,
 * accumulated in double (the reference uses fp32 FMA in k order). */
ORA_EXPORT void ora_gemm_nt_f32(const float* A, const float* B, float* C, int M, int N, int K) {
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            const float* a = A + (long)m * K;
            const float* b = B + (long)n * K;
            for (int k = 0; k < K; ++k) acc += (double)a[k] * (double)b[k];
            C[(long)m * N + n] = (float)acc;
        }
}

/* FP8 W8A8 GEMM reference chain: dequantize_fp8 on both operands
 * (fp8_quant.cu:159), then C = A * W^T (tensor_parallel.cu:187-188), epilogue
 * out = bf16(C).  Codes are the int8 bit patterns the reference stores. */
ORA_EXPORT void ora_gemm_fp8_rowcol(const uint8_t* a_codes, const float* sa,
                                    const uint8_t* w_codes, const float* sw,
                                    float* C, int M, int N, int K) {
    float lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = ora_e4m3_decode((uint8_t)i);
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            const uint8_t* a = a_codes + (long)m * K;
            const uint8_t* w = w_codes + (long)n * K;
            for (int k = 0; k < K; ++k) acc += (double)lut[a[k]] * (double)lut[w[k]];
            C[(long)m * N + n] = (float)(acc * (double)sa[m] * (double)sw[n]);
        }
}

/* W4A16 GEMM reference: C[m, n] = sum_k float(A_bf16[m,k]) * w(n,k),
 * w the GPTQ weight above; double accumulate. */
ORA_EXPORT void ora_gemm_w4a16_zp(const uint16_t* A_bf16, const uint8_t* packed,
                                  const uint16_t* scales_f16, const uint8_t* zeros, float* C,
                                  int M, int N, int K, int gs) {
    int sc = K / gs;
    #pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        /* dequantize the row once */
        float* wrow = (float*)malloc(sizeof(float) * (size_t)K);
        int kk = K;
        for (int k = 0; k < kk; ++k) {
            uint8_t p = packed[(long)n * (K / 2) + k / 2];
            int u = (k & 1) ? (p >> 4) : (p & 0xF);
            wrow[k] = (float)(u - ora_w4_zp(zeros, n, sc, k / gs)) *
                      ora_half_to_float(scales_f16[(long)n * sc + k / gs]);
        }
        for (int m = 0; m < M; ++m) {
            double acc = 0.0;
            const uint16_t* a = A_bf16 + (long)m * K;
            for (int k = 0; k < kk; ++k) acc += (double)ora_bf16_to_float(a[k]) * (double)wrow[k];
            C[(long)m * N + n] = (float)acc;
        }
        free(wrow);
    }
}

ORA_EXPORT void ora_gemm_w4a16(const uint16_t* A_bf16, const uint8_t* packed,
                               const uint16_t* scales_f16, float* C,
                               int M, int N, int K, int gs) {
    ora_gemm_w4a16_zp(A_bf16, packed, scales_f16, NULL, C, M, N, K, gs);
}

/* launch_ring_allreduce: tensor_parallel.cu:93-142.  Chunk c (size
 * ceil(count/R)) is summed into rank c in source order r = 0..R-1, r != c
 * (:108-121), then copied to every rank (:126-140).  bufs is R*count floats,
 * rank-major, updated in place.  fp32 adds in the reference's order. */
ORA_EXPORT void ora_ring_allreduce(float* bufs, int count, int R) {
    if (R <= 1) return;
    int chunk = (count + R - 1) / R;
    for (int c = 0; c < R; ++c) {
        int start = c * chunk;
        int n = (start + chunk <= count) ? chunk : (count - start);
        if (n <= 0) continue;
        for (int r = 0; r < R; ++r) {
            if (r == c) continue;
            for (int i = 0; i < n; ++i)
                bufs[(long)c * count + start + i] += bufs[(long)r * count + start + i];
        }
    }
    for (int c = 0; c < R; ++c) {
        int start = c * chunk;
        int n = (start + chunk <= count) ? chunk : (count - start);
        if (n <= 0) continue;
        for (int r = 0; r < R; ++r) {
            if (r == c) continue;
            for (int i = 0; i < n; ++i)
                bufs[(long)r * count + start + i] = bufs[(long)c * count + start + i];
        }
    }
}

/* launch_allgather: tensor_parallel.cu:258-274.  out = [chunk_0 | ... | chunk_{R-1}]. */
ORA_EXPORT void ora_allgather(const float* chunks, float* out, int chunk, int R) {
    memcpy(out, chunks, sizeof(float) * (size_t)chunk * (size_t)R);
}

ORA_EXPORT int ora_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

ORA_EXPORT void ora_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
