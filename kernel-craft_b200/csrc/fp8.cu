// fp8.cu -- FP8 E4M3 quantization, dequantization and SmoothQuant scaling.
//
// Arithmetic is the reference's, operation for operation, so codes and scales
// are bit-identical (src/kernels/transformer/fp8_quant.cu):
//   amax   = max |x| over the row, fmaxf from 0 (NaN ignored)       :103-107
//   scale  = amax > 0 ? amax / 448 : 1   (IEEE division)            :121
//   q      = e4m3_satfinite_rne(fmaxf(-448, fminf(448, x / scale))) :126-129
//   x_hat  = float(e4m3(q)) * scale[row or 0]                       :155-159
//   smooth = x / s[col]                                              :183
// The per-token kernel reads each row once: a CTA holds its row in registers
// (up to 16 float4 per thread), reduces amax across the CTA, then quantizes
// from registers (the reference reads the row twice and stores bytes).
#include <cuda.h>  // CUcontext (type only; the driver functions are fetched at run time)
#include <cuda_fp8.h>

#include <atomic>
#include <mutex>

#include "kc_common.cuh"

namespace {

constexpr float kE4M3Max = 448.0f;

__device__ __forceinline__ float clamp448(float v) {
    return fmaxf(-kE4M3Max, fminf(kE4M3Max, v));
}

// Two floats -> two E4M3 codes (a in the low byte), RNE with SATFINITE.
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
    return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ uint32_t quant4(float4 v, float scale) {
    const float a = clamp448(__fdiv_rn(v.x, scale));
    const float b = clamp448(__fdiv_rn(v.y, scale));
    const float c = clamp448(__fdiv_rn(v.z, scale));
    const float d = clamp448(__fdiv_rn(v.w, scale));
    return e4m3x2(a, b) | (e4m3x2(c, d) << 16);
}

__device__ __forceinline__ float amax4(float m, float4 v) {
    m = fmaxf(m, fabsf(v.x));
    m = fmaxf(m, fabsf(v.y));
    m = fmaxf(m, fabsf(v.z));
    m = fmaxf(m, fabsf(v.w));
    return m;
}

__device__ __forceinline__ float4 div4(float4 v, float4 s) {
    return make_float4(__fdiv_rn(v.x, s.x), __fdiv_rn(v.y, s.y), __fdiv_rn(v.z, s.z),
                       __fdiv_rn(v.w, s.w));
}

// CTA-wide max; every thread gets the result.
__device__ __forceinline__ float block_max(float v, float* smem) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = kc_warp_max(v);
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    float r = (lane < nw) ? smem[lane] : 0.0f;
    r = kc_warp_max(r);
    __syncthreads();  // smem reused by the next row
    return r;
}

// Per-token quantization, one CTA per row (grid-stride over rows), row held in
// registers: V float4 per thread, element index (tid + blockDim * v) * 4.
// Requires cols % 4 == 0, 16-byte aligned input rows, 4-byte aligned output rows.
template <int V, bool SMOOTH>
__global__ void __launch_bounds__(256) quant_fp8_rows_reg(const float* __restrict__ in,
                                                          const float* __restrict__ smooth,
                                                          int8_t* __restrict__ out,
                                                          float* __restrict__ scales, int rows,
                                                          int cols) {
    __shared__ float red[32];
    const int n4 = cols >> 2;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const float4* src = reinterpret_cast<const float4*>(in + (size_t)r * cols);
        float4 v[V];
        float m = 0.0f;
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int idx = threadIdx.x + i * blockDim.x;
            if (idx < n4) {
                v[i] = __ldcs(src + idx);
                if (SMOOTH) v[i] = div4(v[i], __ldg(reinterpret_cast<const float4*>(smooth) + idx));
                m = amax4(m, v[i]);
            }
        }
        const float amax = block_max(m, red);
        const float scale = (amax > 0.0f) ? __fdiv_rn(amax, kE4M3Max) : 1.0f;
        if (threadIdx.x == 0) scales[r] = scale;
        uint32_t* dst = reinterpret_cast<uint32_t*>(out + (size_t)r * cols);
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int idx = threadIdx.x + i * blockDim.x;
            if (idx < n4) __stcs(dst + idx, quant4(v[i], scale));
        }
    }
}

// Any shape: two passes over the row (the second mostly from L2).
template <bool SMOOTH>
__global__ void __launch_bounds__(256) quant_fp8_rows_generic(const float* __restrict__ in,
                                                              const float* __restrict__ smooth,
                                                              int8_t* __restrict__ out,
                                                              float* __restrict__ scales, int rows,
                                                              int cols) {
    __shared__ float red[32];
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const float* x = in + (size_t)r * cols;
        float m = 0.0f;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            float v = x[c];
            if (SMOOTH) v = __fdiv_rn(v, smooth[c]);
            m = fmaxf(m, fabsf(v));
        }
        const float amax = block_max(m, red);
        const float scale = (amax > 0.0f) ? __fdiv_rn(amax, kE4M3Max) : 1.0f;
        if (threadIdx.x == 0) scales[r] = scale;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            float v = x[c];
            if (SMOOTH) v = __fdiv_rn(v, smooth[c]);
            out[(size_t)r * cols + c] = (int8_t)(e4m3x2(clamp448(__fdiv_rn(v, scale)), 0.f) & 0xFF);
        }
    }
}

// Per-tensor quantization with the scale read on the device (the reference
// copies it to the host first, fp8_quant.cu:217-219; the value is the same).
__global__ void quant_fp8_tensor_vec(const float4* __restrict__ in, uint32_t* __restrict__ out,
                                     const float* __restrict__ d_scale, long n4) {
    const float scale = __ldg(d_scale);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4;
         i += (long)gridDim.x * blockDim.x)
        __stcs(out + i, quant4(__ldcs(in + i), scale));
}

__global__ void quant_fp8_tensor_scalar(const float* __restrict__ in, int8_t* __restrict__ out,
                                        const float* __restrict__ d_scale, long n) {
    const float scale = __ldg(d_scale);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        out[i] = (int8_t)(e4m3x2(clamp448(__fdiv_rn(in[i], scale)), 0.f) & 0xFF);
}

// Whole-tensor amax: CTA max, then one atomicMax per CTA on the IEEE bits
// (valid because every candidate is a non-negative, non-NaN float).
__global__ void __launch_bounds__(256) amax_tensor_kernel(const float* __restrict__ in, long n,
                                                          unsigned int* __restrict__ amax_bits) {
    __shared__ float red[32];
    float m = 0.0f;
    const long n4 = (kc::aligned(in, 16) ? n / 4 : 0);
    const float4* in4 = reinterpret_cast<const float4*>(in);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4;
         i += (long)gridDim.x * blockDim.x)
        m = amax4(m, __ldcs(in4 + i));
    for (long i = 4 * n4 + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(in[i]));
    m = block_max(m, red);
    if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(m));
}

// scale = amax > 0 ? amax / 448 : 1 (pybind_transformer.cpp:305-311 computes the
// same value on the host), written once; every thread quantizes with it.
__global__ void quant_tensor_from_amax(const float* __restrict__ in, int8_t* __restrict__ out,
                                       long n, const unsigned int* __restrict__ amax_bits,
                                       float* __restrict__ scale_out) {
    const float amax = __uint_as_float(*amax_bits);
    const float scale = (amax > 0.0f) ? __fdiv_rn(amax, kE4M3Max) : 1.0f;
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
    const bool vec = kc::aligned(in, 16) && kc::aligned(out, 4);
    const long n4 = vec ? n / 4 : 0;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4;
         i += (long)gridDim.x * blockDim.x)
        __stcs(reinterpret_cast<uint32_t*>(out) + i,
               quant4(__ldcs(reinterpret_cast<const float4*>(in) + i), scale));
    for (long i = 4 * n4 + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        out[i] = (int8_t)(e4m3x2(clamp448(__fdiv_rn(in[i], scale)), 0.f) & 0xFF);
}

__device__ __forceinline__ void decode16(uint4 q, float f[16]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const __nv_fp8x2_storage_t pair = (__nv_fp8x2_storage_t)((w[i] >> (16 * h)) & 0xFFFF);
            const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
            __half2 h2 = *reinterpret_cast<const __half2*>(&hr);
            const float2 ff = __half22float2(h2);
            f[4 * i + 2 * h] = ff.x;
            f[4 * i + 2 * h + 1] = ff.y;
        }
    }
}

// Dequantize 16 codes per thread; requires cols % 16 == 0 and 16B alignment.
__global__ void dequant_fp8_vec(const uint4* __restrict__ in, const float* __restrict__ scales,
                                float4* __restrict__ out, int cols, long n16, bool per_token) {
    const int cpr = cols >> 4;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n16;
         i += (long)gridDim.x * blockDim.x) {
        const long row = i / cpr;
        const float s = per_token ? __ldg(scales + row) : __ldg(scales);
        float f[16];
        decode16(__ldcs(in + i), f);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            __stcs(out + 4 * i + k,
                   make_float4(f[4 * k] * s, f[4 * k + 1] * s, f[4 * k + 2] * s, f[4 * k + 3] * s));
    }
}

__global__ void dequant_fp8_scalar(const int8_t* __restrict__ in, const float* __restrict__ scales,
                                   float* __restrict__ out, int cols, long n, bool per_token) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const long row = i / cols;
        const float s = per_token ? scales[row] : scales[0];
        const __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)in[i], __NV_E4M3);
        out[i] = __half2float(*reinterpret_cast<const __half*>(&hr)) * s;
    }
}

__global__ void smooth_vec(const float4* __restrict__ in, const float4* __restrict__ s,
                           float4* __restrict__ out, int cols4, long n4) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4;
         i += (long)gridDim.x * blockDim.x)
        __stcs(out + i, div4(__ldcs(in + i), __ldg(s + (i % cols4))));
}

__global__ void smooth_scalar(const float* __restrict__ in, const float* __restrict__ s,
                              float* __restrict__ out, int cols, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        out[i] = __fdiv_rn(in[i], s[i % cols]);
}

// ---- allocation-free dynamic per-tensor quantization ---------------------------
// Scratch lives in this module's own device memory instead of a caller buffer:
// word 0 is an arrival counter, word 1 receives the tensor amax, words
// 64.. hold one partial amax per CTA of the amax pass.  The counter is zero
// when the module loads and every completed call leaves it at zero again; the
// other words are fully rewritten by every call.
constexpr long kNoAllocChunk = 16384;         // elements per CTA of the amax pass
constexpr int kNoAllocMaxPartials = 65536;    // CTAs of the amax pass
constexpr long kNoAllocMaxCount = kNoAllocChunk * kNoAllocMaxPartials;  // 2^30 elements
constexpr int kNoAllocPartialBase = 64;
static __device__ __align__(256) unsigned int g_fp8_noalloc_scratch[kNoAllocPartialBase + kNoAllocMaxPartials];

// CTA b reduces elements [b * chunk, (b + 1) * chunk) to a partial amax; the
// CTA that arrives last reduces the partials, publishes the amax in word 1 and
// returns the counter to zero.
__global__ void __launch_bounds__(256) amax_chunks_last_cta(const float* __restrict__ in, long n,
                                                            unsigned int* scratch) {
    __shared__ float red[32];
    __shared__ int is_last;
    const long base = blockIdx.x * kNoAllocChunk;
    const long end = min(n, base + kNoAllocChunk);
    float m = 0.0f;
    long tail = base;
    if (kc::aligned(in, 16)) {
        const float4* in4 = reinterpret_cast<const float4*>(in);
        for (long i = base / 4 + threadIdx.x; i < end / 4; i += blockDim.x) m = amax4(m, __ldcs(in4 + i));
        tail = max(base, (end / 4) * 4);
    }
    for (long i = tail + threadIdx.x; i < end; i += blockDim.x) m = fmaxf(m, fabsf(in[i]));
    m = block_max(m, red);
    if (threadIdx.x == 0) {
        scratch[kNoAllocPartialBase + blockIdx.x] = __float_as_uint(m);
        __threadfence();
        is_last = (atomicAdd(&scratch[0], 1u) == gridDim.x - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    float t = 0.0f;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x)
        t = fmaxf(t, __uint_as_float(__ldcg(&scratch[kNoAllocPartialBase + i])));
    t = block_max(t, red);
    if (threadIdx.x == 0) {
        scratch[1] = __float_as_uint(t);
        scratch[0] = 0u;
    }
}

// Device address of g_fp8_noalloc_scratch in the current context, looked up
// once per device and context (cudaGetSymbolAddress) and cached.  The cache
// key is the context's process-unique id (cuCtxGetId), not the device
// ordinal: after cudaDeviceReset, or under a context other than the primary
// one, the module is loaded anew at another address, and a new id forces a
// new lookup instead of handing out the old, dangling address.
constexpr int kNoAllocMaxDevices = 64;
struct NoAllocSlot {
    unsigned long long ctx_id;  // 0: not looked up yet
    unsigned int* ptr;
};
NoAllocSlot g_noalloc_slot[kNoAllocMaxDevices];
std::mutex g_noalloc_setup_mutex;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Id of the calling thread's current context (0 when it cannot be read).
// The driver functions are fetched through the runtime, so the library keeps
// no link-time dependency on libcuda.
unsigned long long current_context_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS ||
        ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

int noalloc_scratch(unsigned int** out) {
    int dev = 0;
    KC_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    KC_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, KC_ERR_INVALID_ARG,
               "device %d beyond the %d devices the no-alloc scratch table covers", dev,
               kNoAllocMaxDevices);
    std::lock_guard<std::mutex> lock(g_noalloc_setup_mutex);
    NoAllocSlot& slot = g_noalloc_slot[dev];
    unsigned long long id = current_context_id();  // 0 while no context is current yet
    if (id == 0 || slot.ctx_id != id) {
        // the lookup also makes the device's primary context current if none is
        void* sym = nullptr;
        KC_CUDA_TRY(cudaGetSymbolAddress(&sym, g_fp8_noalloc_scratch),
                    "cudaGetSymbolAddress(no-alloc scratch)");
        id = current_context_id();
        KC_REQUIRE(id != 0, KC_ERR_CUDA, "cannot identify the current CUDA context");
        slot.ptr = static_cast<unsigned int*>(sym);
        slot.ctx_id = id;
    }
    *out = slot.ptr;
    return KC_OK;
}

int grid_1d(long items, int threads) {
    long g = (items + threads - 1) / threads;
    const long cap = (long)kc::sm_count() * (2048 / threads) * 4;
    if (g > cap) g = cap;
    return g < 1 ? 1 : (int)g;
}

template <bool SMOOTH>
int quantize_rows(const float* in, const float* smooth, int8_t* out, float* scales, int rows,
                  int cols, cudaStream_t stream) {
    KC_REQUIRE(in && out && scales, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(!SMOOTH || smooth, KC_ERR_INVALID_ARG, "null smooth-scale pointer");
    KC_REQUIRE(rows >= 0 && cols >= 0, KC_ERR_INVALID_ARG, "negative size");
    if (rows == 0) return KC_OK;  // cols == 0: amax 0 -> every scale 1 (generic path)
    const int n4 = cols / 4;
    const bool vec = cols > 0 && (cols % 4 == 0) && kc::aligned(in, 16) && kc::aligned(out, 4) &&
                     (!SMOOTH || kc::aligned(smooth, 16));
    const int grid = rows < (1 << 30) ? rows : (1 << 30);
    if (vec && n4 <= 256 * 16) {
        int V = 1;
        while (256 * V < n4) V *= 2;
        int threads = (n4 + V - 1) / V;
        threads = ((threads + 31) / 32) * 32;
        if (threads > 256) threads = 256;
        switch (V) {
            case 1:  quant_fp8_rows_reg<1, SMOOTH><<<grid, threads, 0, stream>>>(in, smooth, out, scales, rows, cols); break;
            case 2:  quant_fp8_rows_reg<2, SMOOTH><<<grid, threads, 0, stream>>>(in, smooth, out, scales, rows, cols); break;
            case 4:  quant_fp8_rows_reg<4, SMOOTH><<<grid, threads, 0, stream>>>(in, smooth, out, scales, rows, cols); break;
            case 8:  quant_fp8_rows_reg<8, SMOOTH><<<grid, threads, 0, stream>>>(in, smooth, out, scales, rows, cols); break;
            default: quant_fp8_rows_reg<16, SMOOTH><<<grid, threads, 0, stream>>>(in, smooth, out, scales, rows, cols); break;
        }
    } else {
        int threads = cols >= 256 ? 256 : ((cols + 31) / 32) * 32;
        if (threads < 32) threads = 32;
        quant_fp8_rows_generic<SMOOTH><<<grid, threads, 0, stream>>>(in, smooth, out, scales, rows, cols);
    }
    return kc::check_launch("quantize_fp8_rows");
}

}  // namespace

extern "C" {

int kc_quantize_fp8_per_token(const float* in, int8_t* out, float* scales, int rows, int cols,
                              cudaStream_t stream) {
    return quantize_rows<false>(in, nullptr, out, scales, rows, cols, stream);
}

int kc_quantize_fp8_per_channel(const float* w, int8_t* out, float* scales, int N, int K,
                                cudaStream_t stream) {
    return quantize_rows<false>(w, nullptr, out, scales, N, K, stream);
}

int kc_smoothquant_quantize_fp8(const float* in, const float* smooth, int8_t* out, float* scales,
                                int rows, int cols, cudaStream_t stream) {
    return quantize_rows<true>(in, smooth, out, scales, rows, cols, stream);
}

int kc_quantize_fp8_per_tensor(const float* in, int8_t* out, const float* d_scale, long count,
                               cudaStream_t stream) {
    KC_REQUIRE(in && out && d_scale, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(count >= 0, KC_ERR_INVALID_ARG, "negative count");
    if (count == 0) return KC_OK;
    if (count % 4 == 0 && kc::aligned(in, 16) && kc::aligned(out, 4)) {
        const long n4 = count / 4;
        quant_fp8_tensor_vec<<<grid_1d(n4, 256), 256, 0, stream>>>(
            reinterpret_cast<const float4*>(in), reinterpret_cast<uint32_t*>(out), d_scale, n4);
    } else {
        quant_fp8_tensor_scalar<<<grid_1d(count, 256), 256, 0, stream>>>(in, out, d_scale, count);
    }
    return kc::check_launch("quantize_fp8_per_tensor");
}

int kc_quantize_fp8_per_tensor_dynamic(const float* in, int8_t* out, float* scale_out, long count,
                                       void* workspace, size_t workspace_bytes,
                                       cudaStream_t stream) {
    KC_REQUIRE(in && out && scale_out && workspace, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(count >= 0, KC_ERR_INVALID_ARG, "negative count");
    KC_REQUIRE(workspace_bytes >= 4, KC_ERR_INVALID_ARG, "workspace needs 4 bytes, got %zu",
               workspace_bytes);
    KC_REQUIRE(kc::aligned(workspace, 4), KC_ERR_ALIGNMENT, "workspace must be 4-byte aligned");
    unsigned int* amax_bits = static_cast<unsigned int*>(workspace);
    KC_CUDA_TRY(cudaMemsetAsync(amax_bits, 0, sizeof(unsigned int), stream), "workspace clear");
    if (count > 0) {
        amax_tensor_kernel<<<grid_1d((count + 3) / 4, 256), 256, 0, stream>>>(in, count, amax_bits);
        KC_CUDA_TRY(cudaGetLastError(), "amax_tensor_kernel");
    }
    quant_tensor_from_amax<<<grid_1d((count + 3) / 4, 256), 256, 0, stream>>>(in, out, count,
                                                                              amax_bits, scale_out);
    return kc::check_launch("quant_tensor_from_amax");
}

int kc_quantize_fp8_per_tensor_dynamic_noalloc(const float* in, int8_t* out, float* scale_out,
                                               long count, cudaStream_t stream) {
    KC_REQUIRE(in && out && scale_out, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(count >= 0, KC_ERR_INVALID_ARG, "negative count");
    KC_REQUIRE(count <= kNoAllocMaxCount, KC_ERR_INVALID_ARG,
               "count %ld exceeds the no-alloc maximum of %ld elements (%d partials of %ld); use "
               "kc_quantize_fp8_per_tensor_dynamic with a workspace",
               count, kNoAllocMaxCount, kNoAllocMaxPartials, kNoAllocChunk);
    unsigned int* scratch = nullptr;
    const int st = noalloc_scratch(&scratch);
    if (st != KC_OK) return st;
    const int ctas = count > 0 ? kc::ceil_div(count, kNoAllocChunk) : 1;
    amax_chunks_last_cta<<<ctas, 256, 0, stream>>>(in, count, scratch);
    KC_CUDA_TRY(cudaGetLastError(), "amax_chunks_last_cta");
    quant_tensor_from_amax<<<grid_1d((count + 3) / 4, 256), 256, 0, stream>>>(in, out, count,
                                                                              scratch + 1, scale_out);
    return kc::check_launch("quant_tensor_from_amax (no-alloc)");
}

int kc_dequantize_fp8(const int8_t* in, const float* scales, float* out, int rows, int cols,
                      bool per_token, cudaStream_t stream) {
    KC_REQUIRE(in && scales && out, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(rows >= 0 && cols >= 0, KC_ERR_INVALID_ARG, "negative size");
    const long n = (long)rows * cols;
    if (n == 0) return KC_OK;
    if (cols % 16 == 0 && kc::aligned(in, 16) && kc::aligned(out, 16)) {
        const long n16 = n / 16;
        dequant_fp8_vec<<<grid_1d(n16, 256), 256, 0, stream>>>(
            reinterpret_cast<const uint4*>(in), scales, reinterpret_cast<float4*>(out), cols, n16,
            per_token);
    } else {
        dequant_fp8_scalar<<<grid_1d(n, 256), 256, 0, stream>>>(in, scales, out, cols, n, per_token);
    }
    return kc::check_launch("dequantize_fp8");
}

int kc_smoothquant_scale(const float* in, const float* smooth, float* out, int rows, int cols,
                         cudaStream_t stream) {
    KC_REQUIRE(in && smooth && out, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(rows >= 0 && cols >= 0, KC_ERR_INVALID_ARG, "negative size");
    const long n = (long)rows * cols;
    if (n == 0) return KC_OK;
    if (cols % 4 == 0 && kc::aligned(in, 16) && kc::aligned(out, 16) && kc::aligned(smooth, 16)) {
        smooth_vec<<<grid_1d(n / 4, 256), 256, 0, stream>>>(
            reinterpret_cast<const float4*>(in), reinterpret_cast<const float4*>(smooth),
            reinterpret_cast<float4*>(out), cols / 4, n / 4);
    } else {
        smooth_scalar<<<grid_1d(n, 256), 256, 0, stream>>>(in, smooth, out, cols, n);
    }
    return kc::check_launch("smoothquant_scale");
}

void launch_quantize_fp8(const float* d_input, int8_t* d_output, float* d_scales, int rows,
                         int cols, bool per_token, cudaStream_t stream) {
    int st = per_token
                 ? kc_quantize_fp8_per_token(d_input, d_output, d_scales, rows, cols, stream)
                 : kc_quantize_fp8_per_tensor(d_input, d_output, d_scales, (long)rows * cols, stream);
    if (st == KC_OK) kc::check_cuda(cudaStreamSynchronize(stream), "launch_quantize_fp8 sync");
}

void launch_dequantize_fp8(const int8_t* d_input, const float* d_scales, float* d_output, int rows,
                           int cols, bool per_token, cudaStream_t stream) {
    if (kc_dequantize_fp8(d_input, d_scales, d_output, rows, cols, per_token, stream) == KC_OK)
        kc::check_cuda(cudaStreamSynchronize(stream), "launch_dequantize_fp8 sync");
}

void launch_smoothquant_scale(const float* d_input, const float* d_smooth_scales, float* d_output,
                              int rows, int cols, cudaStream_t stream) {
    if (kc_smoothquant_scale(d_input, d_smooth_scales, d_output, rows, cols, stream) == KC_OK)
        kc::check_cuda(cudaStreamSynchronize(stream), "launch_smoothquant_scale sync");
}

}  // extern "C"
