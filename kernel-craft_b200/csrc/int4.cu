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
// them before it computes any (kU * 16 bytes in flight per lane).  One CTA of
// 32 warps per SM, rows dealt round-robin over the CTAs, so each SM holds at
// most ceil(rows / 148) rows (28 at 4096) and stages the activations once.
//
// Dequantization without conversion instructions: the word is XOR-ed with
// 0x88888888 once (each nibble u becomes u' = u ^ 8 = sx4(u) + 8), then a
// nibble at bits 4e, for e <= 4, becomes the exact float 2^23 + 16^e * u' by
// one LOP3 ((w' & 0xF << 4e) | 0x4B000000: the float's mantissa holds the
// nibble in place, its exponent is 2^23); subtracting 2^23 (exact) leaves
// 16^e * u', and one FMA accumulates it against x.  Nibbles 5..7 come from
// the word shifted right by 20 the same way.  The subtractions and FMAs run
// as packed f32x2 pairs (positions p, p + 1 of a word: add.rn.f32x2 /
// fma.rn.f32x2, sm_100) into eight accumulators, one per position; positions
// p and p + 5 share the power 16^p, and the five sums combine as
// sum_e t_e * 16^-e (exact scalings) into sum u' x over the chunk.  The
// reference's weight (quant_int4.cu:99-104) is sx4(u) - z = u' - (8 + z), so
// the chunk's dot product is sum u' x - (8 + z) * X, X the chunk's activation
// sum (computed once per CTA while x is staged); then the group scale
// multiplies it: the chunk's sum, then its scale, where the reference scales
// every weight first -- fp32 GEMV parity is normwise.
//
// expo = 0x4B000000 arrives as a kernel argument, so it sits in a register and
// each nibble costs one LOP3 with the mask as its only immediate (with both
// constants immediate the compiler splits the operation in two).
template <int E>
__device__ __forceinline__ uint32_t nib_bits(uint32_t w, uint32_t expo) {  // 2^23 + 16^E * u'
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w), "n"(0xFu << (4 * E)), "r"(expo));  // (a & b) | c
    return d;
}

__device__ __forceinline__ uint64_t f2pack(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
    return f2pack(__float_as_uint(lo), __float_as_uint(hi));
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
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

// sum over the chunk of u' * x, u' = (nibble ^ 8) in 0..15; nexp2 holds the
// pair (-2^23, -2^23)
__device__ __forceinline__ float chunk_dot(const uint4& v, uint32_t x0, uint64_t nexp2, uint32_t expo) {
    const uint32_t w[4] = {v.x ^ 0x88888888u, v.y ^ 0x88888888u, v.z ^ 0x88888888u, v.w ^ 0x88888888u};
    uint64_t a[4] = {0, 0, 0, 0};   // accumulator pairs (p, p + 1), p = 0, 2, 4, 6
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 xa = lds_f4(xa_base(x0, q)), xb = lds_f4(xa_base(x0, q) + 16);
        const uint32_t h = w[q] >> 20;
        const uint64_t n01 = f2pack(nib_bits<0>(w[q], expo), nib_bits<1>(w[q], expo));
        const uint64_t n23 = f2pack(nib_bits<2>(w[q], expo), nib_bits<3>(w[q], expo));
        const uint64_t n45 = f2pack(nib_bits<4>(w[q], expo), nib_bits<0>(h, expo));
        const uint64_t n67 = f2pack(nib_bits<1>(h, expo), nib_bits<2>(h, expo));
        a[0] = f2fma(f2add(n01, nexp2), f2pack(xa.x, xa.y), a[0]);
        a[1] = f2fma(f2add(n23, nexp2), f2pack(xa.z, xa.w), a[1]);
        a[2] = f2fma(f2add(n45, nexp2), f2pack(xb.x, xb.y), a[2]);
        a[3] = f2fma(f2add(n67, nexp2), f2pack(xb.z, xb.w), a[3]);
    }
    float t[8];
    f2unpack(a[0], t[0], t[1]);
    f2unpack(a[1], t[2], t[3]);
    f2unpack(a[2], t[4], t[5]);
    f2unpack(a[3], t[6], t[7]);
    // t_e for e = 0..4: positions e and e + 5 (e < 3)
    float c = t[4];
    c = fmaf(c, 0.0625f, t[3]);
    c = fmaf(c, 0.0625f, t[2] + t[7]);
    c = fmaf(c, 0.0625f, t[1] + t[6]);
    return fmaf(c, 0.0625f, t[0] + t[5]);
}

// x lives in shared memory for the whole CTA: lane l's chunk j needs the 32
// activations 32j .. 32j + 31, so neighbouring lanes read 128 bytes apart --
// from global memory every such load touches 32 cache lines.  A 16-byte pad
// after every 128 bytes (chunk j at byte 144 j) spreads eight lanes' 16-byte
// reads over all 32 banks.
__host__ __device__ constexpr size_t xs_bytes(int cols) { return (size_t)cols / 32 * 144; }

// GSH >= 0: the group size is 32 << GSH and cols a multiple of 4096, so
// every lane owns four chunks per 128-chunk block and each load's address is
// the lane's base plus a constant (group index (lane >> GSH) + (32 >> GSH) u,
// zero-point byte (lane >> (GSH + 1)) + (16 >> GSH) u, its nibble fixed per
// lane); GSH = -1 handles any cols multiple of 32 and group size multiple of
// 32 with computed indices.
template <int GSH>
__global__ void __launch_bounds__(1024, 1) gemv_int4_f32_vec(const uint8_t* __restrict__ packed,
                                                             const float* __restrict__ scales,
                                                             const uint8_t* __restrict__ zeros,
                                                             const float* __restrict__ x,
                                                             float* __restrict__ y, int rows, int cols,
                                                             int gs, int gs_shift, uint32_t expo) {
    constexpr int kU = 4;
    extern __shared__ __align__(16) uint8_t xs_raw[];
    const int lane = threadIdx.x & 31;
    // rows blockIdx + gridDim * (warp + 32 k): every SM holds at most
    // ceil(rows / gridDim) rows and stages x once
    const int rstep = gridDim.x * (blockDim.x >> 5);
    int r = blockIdx.x + gridDim.x * (threadIdx.x >> 5);
    const bool live = r < rows;
    const int sc = cols / gs, cpr = cols / 32, zc = sc / 2;  // the reference's floor zero stride
    const uint8_t* p = packed + (long)min(r, rows - 1) * (cols / 2);
    const float* srow = scales + (long)min(r, rows - 1) * sc;
    const uint8_t* zrow = zeros + (long)min(r, rows - 1) * zc;
    // Programmatic dependent launch: the next GEMV on the stream may be
    // scheduled now; it waits (griddepcontrol.wait) before it reads anything.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // While the previous grid drains, pull this warp's first row into L2: its
    // packed weights (128-byte lines), scales and zero points.  A prefetch
    // only moves lines into L2, where the previous grid's writes land, so it
    // is safe whatever that grid wrote; every read below comes after the wait.
    if (live) {
        const int wl = (cols / 2 + 127) / 128, sl = (sc * 4 + 127) / 128;
        for (int i = lane; i < wl + sl + 1; i += 32) {
            const void* a = i < wl ? (const void*)(p + 128 * i)
                          : i < wl + sl ? (const void*)(srow + 32 * (i - wl)) : (const void*)zrow;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the first kU chunks' weights, scales and zero points are requested
    // before the activations are staged
    uint4 v[kU];
    float s[kU];
    uint32_t zb[kU];
    int g[kU];
    auto issue = [&](int jb) {
        if constexpr (GSH >= 0) {
            // this lane's bases in row r's 128-chunk block (jb - lane) / 128
            const int blk = (jb - lane) >> 7;
            const uint8_t* pl = packed + (long)r * (cols / 2) + 2048 * blk + 16 * lane;
            const float* sl = scales + (long)r * sc + (128 >> GSH) * blk + (lane >> GSH);
            const uint8_t* zl = zeros + (long)r * zc + (64 >> GSH) * blk + (lane >> (GSH + 1));
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                v[u] = kc_ldg_stream(pl + 512 * u);
                s[u] = __ldg(sl + (32 >> GSH) * u);
                zb[u] = __ldg(zl + (16 >> GSH) * u);
            }
        } else {
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int j = jb + 32 * u;
                if (j < cpr) {
                    g[u] = gs_shift >= 0 ? (32 * j) >> gs_shift : (32 * j) / gs;
                    v[u] = kc_ldg_stream(p + 16 * j);
                    s[u] = __ldg(srow + g[u]);
                    zb[u] = __ldg(zrow + (g[u] >> 1));
                }
            }
        }
    };
    if (live) issue(lane);
    // x into shared memory, and each chunk's sum X into the 16-byte pad after
    // its 128 bytes.  The eight threads of a chunk are eight consecutive lanes
    // starting at a multiple of 8 (the loop stride is a multiple of 8 and
    // cols / 4 is one), and they enter an iteration together: the shuffles
    // stay within those eight.
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const unsigned oct = 0xFFu << (lane & 24);
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) {
        const float4 f = __ldg(x4 + i);
        *reinterpret_cast<float4*>(xs_raw + 16 * i + 16 * (i >> 3)) = f;
        float t = (f.x + f.y) + (f.z + f.w);
        t += __shfl_xor_sync(oct, t, 1);
        t += __shfl_xor_sync(oct, t, 2);
        t += __shfl_xor_sync(oct, t, 4);
        if ((i & 7) == 0) *reinterpret_cast<float*>(xs_raw + 144 * (i >> 3) + 128) = t;
    }
    __syncthreads();
    if (!live) return;
    const uint32_t xs0 = (uint32_t)__cvta_generic_to_shared(xs_raw);
    const uint64_t nexp2 = f2pack(-8388608.f, -8388608.f);
    while (true) {
        float acc = 0.f;
#pragma unroll 1
        for (int jb = lane; jb < cpr; jb += 32 * kU) {
            if (jb != lane) issue(jb);
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int j = jb + 32 * u;
                if (GSH < 0 && j >= cpr) break;
                const uint32_t z = GSH >= 0 ? (zb[u] >> (((threadIdx.x >> (GSH < 0 ? 0 : GSH)) & 1u) << 2)) & 15u
                                            : ((g[u] & 1) ? (zb[u] >> 4) : (zb[u] & 15u));
                const uint32_t xj = xs0 + 144u * (uint32_t)j;
                float xsum;
                asm volatile("ld.shared.f32 %0, [%1];" : "=f"(xsum) : "r"(xj + 128u));
                const float d = fmaf(-(float)(8u + z), xsum, chunk_dot(v[u], xj, nexp2, expo));
                acc = fmaf(s[u], d, acc);
            }
        }
        acc = kc_warp_sum(acc);
        if (lane == 0) y[r] = acc;
        r += rstep;
        if (r >= rows) break;
        p = packed + (long)r * (cols / 2);
        srow = scales + (long)r * sc;
        zrow = zeros + (long)r * zc;
        issue(lane);
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
        // one 32-warp CTA per SM (fewer for fewer rows), a warp per row
        const long ctas = std::min<long>(rows, kc::sm_count());
        int gs_shift = -1;
        for (int b = 0; b < 31; ++b)
            if (gs == (1 << b)) gs_shift = b;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)ctas);
        cfg.blockDim = dim3(1024);
        cfg.dynamicSmemBytes = xs_bytes(cols);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        // group sizes 32..256 with cols a multiple of 4096: constant offsets
        const int gsh = (cols % 4096 == 0 && gs_shift >= 5 && gs_shift <= 8) ? gs_shift - 5 : -1;
        auto kern = gsh == 0 ? gemv_int4_f32_vec<0> : gsh == 1 ? gemv_int4_f32_vec<1>
                  : gsh == 2 ? gemv_int4_f32_vec<2> : gsh == 3 ? gemv_int4_f32_vec<3>
                  : gemv_int4_f32_vec<-1>;
        KC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, packed, scales, zeros, x, y, rows, cols, gs, gs_shift,
                                       0x4B000000u),
                    "gemv_int4_f32 launch");
        return KC_OK;
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
