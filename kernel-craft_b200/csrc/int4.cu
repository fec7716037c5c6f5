// int4.cu -- INT4 weight dequantization and the W4 GEMV family for sm_100a.
//
// Weight format (both APIs): packed u8[N, K/2], row-major, two 4-bit values per
// byte, low nibble = even k (src/kernels/transformer/quant_int4.cu:6-13).
//
//  * Reference ABI (launch_dequantize_int4 / launch_gemv_int4): fp32 scales,
//    nibbles SIGN-extended (quant_int4.cu:34-48), zero points read UNSIGNED from
//    a packed buffer whose row stride is floor(K/gs/2) (quant_int4.cu:93-96).
//    The index arithmetic below is the reference's, so the dequantized weights
//    are bit-identical for every zeros buffer.
//  * GPTQ API (kc_*_w4*): fp16 scales, implicit zero-point 8,
//    w = (u - 8) * s with u the unsigned nibble.
//
// The tensor-core W4A16 GEMV lives in gemv_w4a16.cu.
#include <algorithm>

#include "kc_common.cuh"

namespace {

// ---------------------------------------------------------------------------
// Reference-ABI helpers (quant_int4.cu:34-48, 93-96)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int sx4(uint32_t v) {  // v in 0..15
    return (int)((v ^ 8u)) - 8;
}

__device__ __forceinline__ int ref_zp(const uint8_t* zeros, int row, int cols, int gs, int g) {
    const int zc = cols / gs / 2;
    const uint8_t zb = zeros[(long)row * zc + g / 2];
    return (g % 2 == 0) ? (zb & 0x0F) : (zb >> 4);
}

// One thread per packed byte: the reference's own decomposition, kept for any
// shape the vector path cannot take (odd group sizes, unaligned pointers).
__global__ void dequant_int4_f32_bytes(const uint8_t* __restrict__ packed,
                                       const float* __restrict__ scales,
                                       const uint8_t* __restrict__ zeros,
                                       float* __restrict__ out, int rows, int cols, int gs) {
    const long nbytes = (long)rows * (cols / 2);
    const int sc = cols / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nbytes;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / (cols / 2));
        const int b = (int)(i - (long)r * (cols / 2));
        const int c0 = 2 * b, c1 = c0 + 1;
        const uint8_t p = packed[i];
        const int g0 = c0 / gs, g1 = c1 / gs;
        const float s0 = scales[(long)r * sc + g0];
        const float s1 = scales[(long)r * sc + g1];
        out[(long)r * cols + c0] = (float)(sx4(p & 15u) - ref_zp(zeros, r, cols, gs, g0)) * s0;
        if (c1 < cols)
            out[(long)r * cols + c1] = (float)(sx4(p >> 4) - ref_zp(zeros, r, cols, gs, g1)) * s1;
    }
}

// One thread per 16-byte chunk (32 weights, all in one group): 128-bit load,
// eight 128-bit stores.  Requires cols % 32 == 0, gs % 32 == 0, 16B alignment.
__global__ void dequant_int4_f32_vec(const uint8_t* __restrict__ packed,
                                     const float* __restrict__ scales,
                                     const uint8_t* __restrict__ zeros,
                                     float* __restrict__ out, int rows, int cols, int gs) {
    const int cpr = cols / 32;  // chunks per row
    const long nchunks = (long)rows * cpr;
    const int sc = cols / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nchunks;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / cpr);
        const int j = (int)(i - (long)r * cpr);
        const int g = (32 * j) / gs;
        const float s = scales[(long)r * sc + g];
        const int zp = ref_zp(zeros, r, cols, gs, g);
        const uint4 v = kc_ldg_stream(packed + i * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        float4* dst = reinterpret_cast<float4*>(out + (long)r * cols + 32 * j);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = (float)(sx4((w[q] >> (4 * e)) & 15u) - zp) * s;
            dst[2 * q]     = make_float4(f[0], f[1], f[2], f[3]);
            dst[2 * q + 1] = make_float4(f[4], f[5], f[6], f[7]);
        }
    }
}

// fp32 GEMV over 16-byte chunks (32 weights of one group each), two rows
// per warp so every x load serves both; a lane takes chunks lane, lane + 32,
// ... in order and issues the packed loads of kU of them (both rows) before
// it computes any, so a warp has 2 * kU * 512 bytes in flight instead of
// 512.  Each row's accumulation order per lane is the one-row order, so the
// result does not depend on the row pairing.
__global__ void __launch_bounds__(256) gemv_int4_f32_vec(const uint8_t* __restrict__ packed,
                                                         const float* __restrict__ scales,
                                                         const uint8_t* __restrict__ zeros,
                                                         const float* __restrict__ x,
                                                         float* __restrict__ y, int rows, int cols,
                                                         int gs) {
    constexpr int kU = 4;
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int sc = cols / gs, cpr = cols / 32;
    for (int r0 = 2 * ((blockIdx.x * blockDim.x + threadIdx.x) >> 5); r0 < rows; r0 += 2 * warps) {
        const bool two = r0 + 1 < rows;
        const int r1 = two ? r0 + 1 : r0;     // a lone last row computes itself twice
        const uint8_t* p0 = packed + (long)r0 * (cols / 2);
        const uint8_t* p1 = packed + (long)r1 * (cols / 2);
        float acc0 = 0.f, acc1 = 0.f;
        for (int jb = lane; jb < cpr; jb += 32 * kU) {
            uint4 v0[kU], v1[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int j = jb + 32 * u;
                if (j < cpr) {
                    v0[u] = kc_ldg_stream(p0 + 16 * j);
                    v1[u] = kc_ldg_stream(p1 + 16 * j);
                }
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int j = jb + 32 * u;
                if (j >= cpr) break;
                const int g = (32 * j) / gs;
                const float s0 = scales[(long)r0 * sc + g], s1 = scales[(long)r1 * sc + g];
                const int z0 = ref_zp(zeros, r0, cols, gs, g), z1 = ref_zp(zeros, r1, cols, gs, g);
                const uint32_t w0[4] = {v0[u].x, v0[u].y, v0[u].z, v0[u].w};
                const uint32_t w1[4] = {v1[u].x, v1[u].y, v1[u].z, v1[u].w};
                const float4* xv = reinterpret_cast<const float4*>(x + 32 * j);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 xa = __ldg(xv + 2 * q), xb = __ldg(xv + 2 * q + 1);
                    const float xe[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        acc0 = fmaf((float)(sx4((w0[q] >> (4 * e)) & 15u) - z0) * s0, xe[e], acc0);
                        acc1 = fmaf((float)(sx4((w1[q] >> (4 * e)) & 15u) - z1) * s1, xe[e], acc1);
                    }
                }
            }
        }
        acc0 = kc_warp_sum(acc0);
        acc1 = kc_warp_sum(acc1);
        if (lane == 0) {
            y[r0] = acc0;
            if (two) y[r1] = acc1;
        }
    }
}

// fp32 GEMV, one warp per row, one packed byte per lane and step: any shape
// (odd group sizes, cols not a multiple of 32, unaligned pointers).
__global__ void __launch_bounds__(256) gemv_int4_f32_bytes(const uint8_t* __restrict__ packed,
                                                           const float* __restrict__ scales,
                                                           const uint8_t* __restrict__ zeros,
                                                           const float* __restrict__ x,
                                                           float* __restrict__ y, int rows, int cols,
                                                           int gs) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int sc = cols / gs;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        float acc = 0.f;
        for (int b = lane; 2 * b < cols; b += 32) {
            const int c0 = 2 * b, c1 = c0 + 1;
            const uint8_t p = packed[(long)r * (cols / 2) + b];
            const int g0 = c0 / gs, g1 = c1 / gs;
            const float w0 = (float)(sx4(p & 15u) - ref_zp(zeros, r, cols, gs, g0)) *
                             scales[(long)r * sc + g0];
            acc = fmaf(w0, x[c0], acc);
            if (c1 < cols) {
                const float w1 = (float)(sx4(p >> 4) - ref_zp(zeros, r, cols, gs, g1)) *
                                 scales[(long)r * sc + g1];
                acc = fmaf(w1, x[c1], acc);
            }
        }
        acc = kc_warp_sum(acc);
        if (lane == 0) y[r] = acc;
    }
}

// ---------------------------------------------------------------------------
// GPTQ (implicit zero-point 8) helpers
// ---------------------------------------------------------------------------

// bf16 dequant, one thread per 16-byte chunk (32 weights of one group).
__global__ void dequant_w4_bf16_vec(const uint8_t* __restrict__ packed,
                                    const __half* __restrict__ scales,
                                    __nv_bfloat16* __restrict__ out, int N, int K, int gs) {
    const int cpr = K / 32;
    const long nchunks = (long)N * cpr;
    const int sc = K / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nchunks;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / cpr);
        const int j = (int)(i - (long)r * cpr);
        const float s = __half2float(scales[(long)r * sc + (32 * j) / gs]);
        const uint4 v = kc_ldg_stream(packed + i * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint4* dst = reinterpret_cast<uint4*>(out + (long)r * K + 32 * j);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float lo = (float)((int)((w[q] >> (8 * e)) & 15u) - 8) * s;
                const float hi = (float)((int)((w[q] >> (8 * e + 4)) & 15u) - 8) * s;
                __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
                o[e] = *reinterpret_cast<uint32_t*>(&h2);
            }
            dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

__global__ void dequant_w4_bf16_scalar(const uint8_t* __restrict__ packed,
                                       const __half* __restrict__ scales,
                                       __nv_bfloat16* __restrict__ out, int N, int K, int gs) {
    const long n = (long)N * K;
    const int sc = K / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / K);
        const int c = (int)(i - (long)r * K);
        const uint8_t p = packed[(long)r * (K / 2) + c / 2];
        const int u = (c & 1) ? (p >> 4) : (p & 15);
        const float w = (float)(u - 8) * __half2float(scales[(long)r * sc + c / gs]);
        out[i] = __float2bfloat16_rn(w);
    }
}

int grid_for(long work_items, int threads) {
    const long cap = (long)kc::sm_count() * (2048 / threads);
    long g = work_items < cap ? work_items : cap;
    return g < 1 ? 1 : (int)g;
}

int check_ref_int4_args(const void* packed, const void* scales, const void* zeros, const void* out,
                        int rows, int cols, int gs) {
    KC_REQUIRE(packed && scales && zeros && out, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(rows >= 0 && cols >= 0, KC_ERR_INVALID_ARG, "negative size rows=%d cols=%d", rows, cols);
    KC_REQUIRE(cols % 2 == 0, KC_ERR_INVALID_ARG, "cols=%d must be even", cols);
    KC_REQUIRE(gs > 0 && cols % gs == 0, KC_ERR_INVALID_ARG,
               "group_size=%d must be > 0 and divide cols=%d", gs, cols);
    return KC_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int kc_dequantize_int4_f32(const uint8_t* packed, const float* scales, const uint8_t* zeros,
                           float* out, int rows, int cols, int gs, cudaStream_t stream) {
    int st = check_ref_int4_args(packed, scales, zeros, out, rows, cols, gs);
    if (st) return st;
    if (rows == 0 || cols == 0) return KC_OK;
    const bool vec = (cols % 32 == 0) && (gs % 32 == 0) && kc::aligned(packed, 16) &&
                     kc::aligned(out, 16);
    if (vec) {
        const long n = (long)rows * (cols / 32);
        dequant_int4_f32_vec<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(
            packed, scales, zeros, out, rows, cols, gs);
    } else {
        const long n = (long)rows * (cols / 2);
        dequant_int4_f32_bytes<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(
            packed, scales, zeros, out, rows, cols, gs);
    }
    return kc::check_launch("dequantize_int4_f32");
}

int kc_gemv_int4_f32(const uint8_t* packed, const float* scales, const uint8_t* zeros,
                     const float* x, float* y, int rows, int cols, int gs, cudaStream_t stream) {
    int st = check_ref_int4_args(packed, scales, zeros, y, rows, cols, gs);
    if (st) return st;
    KC_REQUIRE(x != nullptr, KC_ERR_INVALID_ARG, "null x");
    if (rows == 0) return KC_OK;
    const bool vec = (cols % 32 == 0) && (gs % 32 == 0) && kc::aligned(packed, 16) &&
                     kc::aligned(x, 16);
    if (vec) {
        const int grid2 = grid_for(((long)rows + 15) / 16, 256);   // 8 warps x 2 rows per CTA
        gemv_int4_f32_vec<<<grid2, 256, 0, stream>>>(packed, scales, zeros, x, y, rows, cols, gs);
        return kc::check_launch("gemv_int4_f32");
    }
    const int grid = grid_for(((long)rows + 7) / 8, 256);
    gemv_int4_f32_bytes<<<grid, 256, 0, stream>>>(packed, scales, zeros, x, y, rows, cols, gs);
    return kc::check_launch("gemv_int4_f32");
}

void launch_dequantize_int4(const uint8_t* d_packed, const float* d_scales, const uint8_t* d_zeros,
                            float* d_output, int rows, int cols, int group_size,
                            cudaStream_t stream) {
    if (kc_dequantize_int4_f32(d_packed, d_scales, d_zeros, d_output, rows, cols, group_size,
                               stream) == KC_OK)
        kc::check_cuda(cudaStreamSynchronize(stream), "launch_dequantize_int4 sync");
}

void launch_gemv_int4(const uint8_t* d_packed, const float* d_scales, const uint8_t* d_zeros,
                      const float* d_x, float* d_y, int rows, int cols, int group_size,
                      cudaStream_t stream) {
    if (kc_gemv_int4_f32(d_packed, d_scales, d_zeros, d_x, d_y, rows, cols, group_size, stream) ==
        KC_OK)
        kc::check_cuda(cudaStreamSynchronize(stream), "launch_gemv_int4 sync");
}

int kc_dequantize_w4_bf16(const uint8_t* packed, const uint16_t* scales_f16, uint16_t* out_bf16,
                          int N, int K, int gs, cudaStream_t stream) {
    KC_REQUIRE(packed && scales_f16 && out_bf16, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(N >= 0 && K >= 0 && K % 2 == 0, KC_ERR_INVALID_ARG, "bad shape N=%d K=%d", N, K);
    KC_REQUIRE(gs > 0 && K % gs == 0, KC_ERR_INVALID_ARG, "group_size=%d must divide K=%d", gs, K);
    if (N == 0 || K == 0) return KC_OK;
    const __half* s = reinterpret_cast<const __half*>(scales_f16);
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out_bf16);
    if (K % 32 == 0 && gs % 32 == 0 && kc::aligned(packed, 16) && kc::aligned(out_bf16, 16)) {
        const long n = (long)N * (K / 32);
        dequant_w4_bf16_vec<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(packed, s, o, N, K, gs);
    } else {
        const long n = (long)N * K;
        dequant_w4_bf16_scalar<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(packed, s, o, N, K, gs);
    }
    return kc::check_launch("dequantize_w4_bf16");
}

}  // extern "C"
