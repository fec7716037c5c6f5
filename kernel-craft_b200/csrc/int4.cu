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

// fp32 GEMV over 16-byte chunks (32 weights of one group each), one warp per
// row: a lane takes chunks lane, lane + 32, ... and issues the loads of kU of
// them before it computes any (kU * 16 bytes in flight per lane; a grid of
// rows / 8 CTAs of eight warps fills every SM three or four times over).
//
// Dequantization without conversion instructions: a nibble u at bits 4e of a
// word, for e <= 4, becomes the exact float 2^23 + 16^e * (u ^ 8) by one
// LOP3 ((w & 0xF << 4e) ^ (0x4B000000 | 8 << 4e): the float's mantissa holds
// the flipped nibble in place, its exponent is 2^23); subtracting the exact
// constant 2^23 + (8 + z) * 16^e leaves (sx4(u) - z) * 16^e, the reference's
// integer weight (quant_int4.cu:99-104) times 16^e, and one FMA accumulates it
// against x in the accumulator of that power of 16.  Nibbles 5..7 come from
// the word shifted right by 20 the same way.  Per chunk the five accumulators
// combine as sum_e t_e * 16^-e (exact scalings) and the group scale
// multiplies the result: the chunk's sum, then its scale, where the
// reference scales every weight first -- fp32 GEMV parity is normwise.
__device__ __forceinline__ float nib_f32(uint32_t w, int e) {  // 2^23 + 16^e * (u ^ 8)
    return __uint_as_float((w & (0xFu << (4 * e))) ^ (0x4B000000u | (8u << (4 * e))));
}

// xa: this chunk's 32 activations in shared memory (8 float4, 32 bytes per
// q-step: two 16-byte halves)
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t xa_base(uint32_t x0, int q) { return x0 + 32u * (uint32_t)q; }

__device__ __forceinline__ float chunk_dot(const uint4& v, uint32_t x0, float z8) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float k[5], t[5];
#pragma unroll
    for (int e = 0; e < 5; ++e) {
        k[e] = fmaf(z8, (float)(1 << (4 * e)), 8388608.f);
        t[e] = 0.f;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 xa = lds_f4(xa_base(x0, q)), xb = lds_f4(xa_base(x0, q) + 16);
        const float xe[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        const uint32_t h = w[q] >> 20;
#pragma unroll
        for (int e = 0; e < 5; ++e) t[e] = fmaf(nib_f32(w[q], e) - k[e], xe[e], t[e]);
#pragma unroll
        for (int e = 0; e < 3; ++e) t[e] = fmaf(nib_f32(h, e) - k[e], xe[5 + e], t[e]);
    }
    float c = t[4];
#pragma unroll
    for (int e = 3; e >= 0; --e) c = fmaf(c, 0.0625f, t[e]);
    return c;
}

// x lives in shared memory for the whole CTA: lane l's chunk j needs the 32
// activations 32j .. 32j + 31, so neighbouring lanes read 128 bytes apart --
// from global memory every such load touches 32 cache lines.  A 16-byte pad
// after every 128 bytes (chunk j at byte 144 j) spreads eight lanes' 16-byte
// reads over all 32 banks.
__host__ __device__ constexpr size_t xs_bytes(int cols) { return (size_t)cols / 32 * 144; }

__global__ void __launch_bounds__(256, 4) gemv_int4_f32_vec(const uint8_t* __restrict__ packed,
                                                            const float* __restrict__ scales,
                                                            const uint8_t* __restrict__ zeros,
                                                            const float* __restrict__ x,
                                                            float* __restrict__ y, int rows, int cols,
                                                            int gs, int gs_shift) {
    constexpr int kU = 4;
    extern __shared__ __align__(16) uint8_t xs_raw[];
    const int lane = threadIdx.x & 31;
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const bool live = r < rows;
    const int sc = cols / gs, cpr = cols / 32, zc = sc / 2;  // the reference's floor zero stride
    const uint8_t* p = packed + (long)min(r, rows - 1) * (cols / 2);
    const float* srow = scales + (long)min(r, rows - 1) * sc;
    const uint8_t* zrow = zeros + (long)min(r, rows - 1) * zc;
    // the first kU chunks' weights, scales and zero points are requested
    // before the activations are staged
    uint4 v[kU];
    float s[kU];
    uint32_t zb[kU];
    int g[kU];
    auto issue = [&](int jb) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int j = jb + 32 * u;
            if (live && j < cpr) {
                g[u] = gs_shift >= 0 ? (32 * j) >> gs_shift : (32 * j) / gs;
                v[u] = kc_ldg_stream(p + 16 * j);
                s[u] = __ldg(srow + g[u]);
                zb[u] = __ldg(zrow + (g[u] >> 1));
            }
        }
    };
    issue(lane);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x)
        *reinterpret_cast<float4*>(xs_raw + 16 * i + 16 * (i >> 3)) = __ldg(x4 + i);
    __syncthreads();
    if (!live) return;
    const uint32_t xs0 = (uint32_t)__cvta_generic_to_shared(xs_raw);
    float acc = 0.f;
    for (int jb = lane; jb < cpr; jb += 32 * kU) {
        if (jb != lane) issue(jb);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int j = jb + 32 * u;
            if (j >= cpr) break;
            const uint32_t z = (g[u] & 1) ? (zb[u] >> 4) : (zb[u] & 15u);
            acc = fmaf(s[u], chunk_dot(v[u], xs0 + 144u * (uint32_t)j, (float)(8 + z)), acc);
        }
    }
    acc = kc_warp_sum(acc);
    if (lane == 0) y[r] = acc;
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
// zeros: per-group zero points u8[N, K/gs] (null: 8)
__global__ void dequant_w4_bf16_vec(const uint8_t* __restrict__ packed,
                                    const __half* __restrict__ scales,
                                    const uint8_t* __restrict__ zeros,
                                    __nv_bfloat16* __restrict__ out, int N, int K, int gs) {
    const int cpr = K / 32;
    const long nchunks = (long)N * cpr;
    const int sc = K / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nchunks;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / cpr);
        const int j = (int)(i - (long)r * cpr);
        const float s = __half2float(scales[(long)r * sc + (32 * j) / gs]);
        const int z = zeros ? (int)(zeros[(long)r * sc + (32 * j) / gs] & 15) : 8;
        const uint4 v = kc_ldg_stream(packed + i * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint4* dst = reinterpret_cast<uint4*>(out + (long)r * K + 32 * j);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float lo = (float)((int)((w[q] >> (8 * e)) & 15u) - z) * s;
                const float hi = (float)((int)((w[q] >> (8 * e + 4)) & 15u) - z) * s;
                __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
                o[e] = *reinterpret_cast<uint32_t*>(&h2);
            }
            dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

__global__ void dequant_w4_bf16_scalar(const uint8_t* __restrict__ packed,
                                       const __half* __restrict__ scales,
                                       const uint8_t* __restrict__ zeros,
                                       __nv_bfloat16* __restrict__ out, int N, int K, int gs) {
    const long n = (long)N * K;
    const int sc = K / gs;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / K);
        const int c = (int)(i - (long)r * K);
        const uint8_t p = packed[(long)r * (K / 2) + c / 2];
        const int u = (c & 1) ? (p >> 4) : (p & 15);
        const int z = zeros ? (int)(zeros[(long)r * sc + c / gs] & 15) : 8;
        const float w = (float)(u - z) * __half2float(scales[(long)r * sc + c / gs]);
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
    // the vector path stages x in shared memory: up to 48 KB (cols <= 10922
    // rounded to chunks) without an opt-in attribute
    const bool vec = (cols % 32 == 0) && (gs % 32 == 0) && kc::aligned(packed, 16) &&
                     kc::aligned(x, 16) && xs_bytes(cols) <= 48 * 1024;
    if (vec) {
        // 8 rows per CTA, one CTA per 8 rows (no grid-stride loop)
        const long ctas = ((long)rows + 7) / 8;
        KC_REQUIRE(ctas < (1L << 31), KC_ERR_INVALID_ARG, "too many rows");
        int gs_shift = -1;
        for (int b = 0; b < 31; ++b)
            if (gs == (1 << b)) gs_shift = b;
        gemv_int4_f32_vec<<<(unsigned)ctas, 256, xs_bytes(cols), stream>>>(packed, scales, zeros, x, y,
                                                                           rows, cols, gs, gs_shift);
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

namespace {
int dequantize_w4_bf16(const uint8_t* packed, const uint16_t* scales_f16, const uint8_t* zeros,
                       uint16_t* out_bf16, int N, int K, int gs, cudaStream_t stream) {
    KC_REQUIRE(packed && scales_f16 && out_bf16, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(N >= 0 && K >= 0 && K % 2 == 0, KC_ERR_INVALID_ARG, "bad shape N=%d K=%d", N, K);
    KC_REQUIRE(gs > 0 && K % gs == 0, KC_ERR_INVALID_ARG, "group_size=%d must divide K=%d", gs, K);
    if (N == 0 || K == 0) return KC_OK;
    const __half* s = reinterpret_cast<const __half*>(scales_f16);
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out_bf16);
    if (K % 32 == 0 && gs % 32 == 0 && kc::aligned(packed, 16) && kc::aligned(out_bf16, 16)) {
        const long n = (long)N * (K / 32);
        dequant_w4_bf16_vec<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(packed, s, zeros, o, N,
                                                                                 K, gs);
    } else {
        const long n = (long)N * K;
        dequant_w4_bf16_scalar<<<grid_for((n + 255) / 256, 256), 256, 0, stream>>>(packed, s, zeros, o,
                                                                                    N, K, gs);
    }
    return kc::check_launch("dequantize_w4_bf16");
}
}  // namespace

int kc_dequantize_w4_bf16(const uint8_t* packed, const uint16_t* scales_f16, uint16_t* out_bf16,
                          int N, int K, int gs, cudaStream_t stream) {
    return dequantize_w4_bf16(packed, scales_f16, nullptr, out_bf16, N, K, gs, stream);
}

int kc_dequantize_w4_bf16_zp(const uint8_t* packed, const uint16_t* scales_f16, const uint8_t* zeros,
                             uint16_t* out_bf16, int N, int K, int gs, cudaStream_t stream) {
    KC_REQUIRE(zeros != nullptr, KC_ERR_INVALID_ARG, "null zero points");
    return dequantize_w4_bf16(packed, scales_f16, zeros, out_bf16, N, K, gs, stream);
}

}  // extern "C"
