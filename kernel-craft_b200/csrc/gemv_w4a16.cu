// gemv_w4a16.cu -- W4A16 GEMV / skinny GEMM (M <= 16) for sm_100a.
//
// y[m, n] = sum_k w[n, k] * x[m, k],  w[n, k] = (u - 8) * s[n, k / gs],
// u the unsigned nibble of packed[n, k / 2] (low nibble = even k), s fp16,
// x bf16, fp32 accumulation, fp32 y.  Several problems (e.g. the four
// projections of a decoder layer) can share one launch.
//
// Work decomposition: 16-row tiles in problem-major order, persistent CTAs of
// eight warps (two per SM); the warps of a CTA split a tile's K range into
// contiguous runs of 128-k chunks (16 rows x 64 bytes = 1 KB each) and reduce
// their partial sums through shared memory at the end of the tile.
//
// Memory pipeline: every warp owns a ring of kRing stages in shared memory,
// each holding up to four chunks ("a quad", 4 KB).  Its lane 0 issues the
// quad's 2-D TMA loads (box 64 bytes x 16 rows; rows past N read as zero) on
// the stage's mbarrier, running kRing quads ahead of the warp's compute,
// across tile boundaries; a tile's fp16 scale block (16 contiguous rows)
// arrives by one bulk copy per tile, issued a tile ahead.  One wait and one
// issue per 4 KB keeps the per-chunk bookkeeping small.
//
// Compute: a lane (g = lane / 4, t = lane % 4) reads rows g and g + 8, 16
// bytes each, of a chunk and turns every 32-bit word into four bf16x2 MMA
// fragments holding 128 + u exactly (nibble OR-ed into the mantissa of bf16
// 128.0; 3 shifts + 4 LOP3 per 8 weights), fed straight from registers into
// mma.sync m16n8k16 (weights as A, activations as B).  Activations are
// staged once per problem in shared memory in fragment order (k0 k4 k1 k5 k2
// k6 k3 k7 per 8-block) when they fit, together with their per-chunk sums, and
// the offset is removed per chunk as sum (u - 8) x = sum (128 + u) x -
// 136 * sum x; otherwise they are read from global memory (L1-resident),
// permuted with PRMT, and a second MMA with the constant fragment -136 removes
// the offset.  The group scale multiplies the per-chunk result.  MMA columns
// m >= M read a valid (clamped) activation row and are
// discarded, so no lane predication is needed.
//
// Dequantized weights never touch shared memory or TMEM: at M <= 16 the
// kernel is bound by HBM, and staging bf16 weights for a tcgen05 A operand
// (2 bytes written and read per weight) would cost more on-chip bandwidth than
// the 0.5 byte per weight streamed from HBM.
#include <algorithm>

#include "kc_common.cuh"
#include "sm100.cuh"
#include "tensor_map.cuh"

namespace {

struct Prob {
    const uint8_t* packed;
    const __half* scales;
    const __nv_bfloat16* x;
    float* y;
    int N, K;
    int tile_begin;  // first 16-row tile of this problem in the flattened tile list
};

struct alignas(64) Params {
    CUtensorMap wmap[KC_W4A16_MAX_PROBLEMS];  // packed weights: {K/2 bytes, N rows}, box {64, 16}
    Prob p[KC_W4A16_MAX_PROBLEMS];
    int count;
    int total_tiles;
    int M;
    int gs;
    int gshift;      // group of 128-k chunk c is c >> gshift
    int xs_row;      // row pitch (elements) of the staged activations, 0 = not staged
    int sx_chunks;   // chunk capacity of the staged activation sums
    uint32_t magic;  // 0x43004300 = bf16x2 (128, 128), held in a register (see nib_or)
    uint32_t neg136; // 0xC308C308 = bf16x2 (-136, -136): the unstaged path's offset MMA fragment
};

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kChunkBytes = 1024;                 // 16 rows x 64 bytes = 128 k
constexpr int kQuad = 4;                          // chunks per stage
constexpr int kRing = 2;                          // stages per warp
constexpr int kScaleHalves = 16 * 128;            // 16 rows x up to 128 groups
constexpr int kSxCols = 16;                       // activation-sum columns (M padded)

template <int NT>
struct Smem {
    uint8_t ring[kWarps][kRing][kQuad][kChunkBytes];  // TMA destinations, 1024-byte aligned
    __half scales[2][kScaleHalves];
    float red[kWarps][16][NT * 8 + 1];
    uint64_t wfull[kWarps][kRing];
    uint64_t sfull[2];
    // then, if staged: the activation sums float[sx_chunks][kSxCols] and the
    // activations (bf16, fragment order), 16-byte aligned
};

template <int NT>
__host__ __device__ constexpr size_t fixed_smem() {
    return (sizeof(Smem<NT>) + 127) / 128 * 128;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ float2 lds_f2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ float lds_half(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ void mma_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (a & 0x000F000F) | magic in one LOP3.  A LOP3 encodes one immediate, so the
// magic constant arrives as a register (a kernel parameter); written as C++
// with two constants the pair costs two logic instructions.
__device__ __forceinline__ uint32_t nib_or(uint32_t a, uint32_t magic) {
    uint32_t d;
    asm("lop3.b32 %0, %1, 0x000F000F, %2, 0xEA;" : "=r"(d) : "r"(a), "r"(magic));
    return d;
}

// bf16x2 fragments (128 + u) for the nibble pairs (k0,k4) (k1,k5) (k2,k6) (k3,k7)
// of one 32-bit word.
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t magic, uint32_t o[4]) {
    o[0] = nib_or(w, magic);
    o[1] = nib_or(w >> 4, magic);
    o[2] = nib_or(w >> 8, magic);
    o[3] = nib_or(w >> 12, magic);
}

__device__ __forceinline__ int problem_index(const Params& P, int tile) {
    int pi = 0;
#pragma unroll 1
    while (pi + 1 < P.count && tile >= P.p[pi + 1].tile_begin) ++pi;
    return pi;
}

// Chunk range [begin, end) of warp w for a row of C 128-k chunks.
__device__ __forceinline__ void warp_chunks(int C, int w, int& begin, int& end) {
    begin = (w * C) >> 3;
    end = ((w + 1) * C) >> 3;
}

// A warp's position in its own sequence of (tile, quad) work items.
struct Cursor {
    int tile, c, cend, pi;
};

__device__ __forceinline__ void cursor_settle(const Params& P, Cursor& cu, int warp) {
    while (cu.tile < P.total_tiles && cu.c >= cu.cend) {
        cu.tile += gridDim.x;
        if (cu.tile >= P.total_tiles) break;
        cu.pi = problem_index(P, cu.tile);
        warp_chunks(P.p[cu.pi].K >> 7, warp, cu.c, cu.cend);
    }
}

// The whole warp steps the (warp-uniform) cursor; the arm of the stage's
// mbarrier and the quad's TMA loads (one 1 KB box per chunk) are issued by
// lane 0 through predicated PTX, so no divergent branch is taken.
__device__ __forceinline__ void issue_quad(const Params& P, Cursor& cu, uint32_t dst, uint32_t bar,
                                           int warp, bool leader) {
    if (cu.tile >= P.total_tiles) return;
    const int row0 = (cu.tile - P.p[cu.pi].tile_begin) * 16;
    const int n = min(kQuad, cu.cend - cu.c);
    const CUtensorMap* map = &P.wmap[cu.pi];
    const int x0 = cu.c * 64;
    asm volatile(
        "{\n\t.reg .pred l, l1, l2, l3;\n\t"
        "setp.ne.b32 l, %0, 0;\n\t"
        "setp.gt.and.s32 l1, %6, 1, l;\n\t"
        "setp.gt.and.s32 l2, %6, 2, l;\n\t"
        "setp.gt.and.s32 l3, %6, 3, l;\n\t"
        "@l mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n\t"
        "@l cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%3], [%4, {%5, %7}], [%1];\n\t"
        "@l1 cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%8], [%4, {%9, %7}], [%1];\n\t"
        "@l2 cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%10], [%4, {%11, %7}], [%1];\n\t"
        "@l3 cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%12], [%4, {%13, %7}], [%1];\n\t}"
        ::"r"((int)leader), "r"(bar), "r"((uint32_t)n * kChunkBytes), "r"(dst), "l"(map), "r"(x0),
          "r"(n), "r"(row0), "r"(dst + kChunkBytes), "r"(x0 + 64), "r"(dst + 2 * kChunkBytes),
          "r"(x0 + 128), "r"(dst + 3 * kChunkBytes), "r"(x0 + 192)
        : "memory");
    cu.c += n;
    cursor_settle(P, cu, warp);
}

__device__ __forceinline__ void issue_scales(const Params& P, int tile, __half* dst, uint64_t* bar) {
    const int pi = problem_index(P, tile);
    const Prob& pr = P.p[pi];
    const int row0 = (tile - pr.tile_begin) * 16;
    const uint32_t bytes = (uint32_t)min(16, pr.N - row0) * (uint32_t)(pr.K / P.gs) * 2u;
    sm100::mbar_arrive_expect_tx(bar, bytes);
    sm100::bulk_g2s(dst, pr.scales + (size_t)row0 * (pr.K / P.gs), bytes, bar);
}

// Staged activations (only when they fit): within each 128-k chunk the
// sixteen 8-element blocks b = 4t + j (k = 32t + 8j) are stored at position
// 4j + t, each block permuted to (x0x4, x1x5, x2x6, x3x7); a lane's LDS.128
// for word j then hits 16 consecutive bytes per t (conflict-free).  The same
// pass forms the per-chunk sums sx[c][m] = sum of the chunk's 128 bf16 x[m, k]
// (fp32; the 16 blocks of a chunk sit in 16 consecutive threads, reduced by
// shuffles), and zeroes the columns m >= M.
__device__ __forceinline__ void stage_activations(const Params& P, int pi, float* sx,
                                                  __nv_bfloat16* xs) {
    const Prob& pr = P.p[pi];
    const int nb = pr.K / 8;
    const int blocks = P.M * nb;
    const int C = pr.K >> 7;
    for (int i = threadIdx.x; i < C * kSxCols; i += kThreads)
        if (i % kSxCols >= P.M) sx[i] = 0.f;
    const int rounds = (blocks + 31) & ~31;   // whole warps: the shuffles need every lane
    for (int b = threadIdx.x; b < rounds; b += kThreads) {
        const bool valid = b < blocks;
        const int m = valid ? b / nb : 0, kb = valid ? b - m * nb : 0;
        const uint4 v = valid ? kc_ldg_keep(pr.x + (size_t)m * pr.K + kb * 8) : make_uint4(0, 0, 0, 0);
        float sum = 0.f;
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) sum += __uint_as_float(w4[i] << 16) + __uint_as_float(w4[i] & 0xFFFF0000u);
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (!valid) continue;
        const uint4 o = make_uint4(prmt(v.x, v.z, 0x5410u), prmt(v.x, v.z, 0x7632u),
                                   prmt(v.y, v.w, 0x5410u), prmt(v.y, v.w, 0x7632u));
        const int c = kb >> 4, r = kb & 15;
        const int pos = (c << 4) + ((r & 3) << 2) + (r >> 2);
        *reinterpret_cast<uint4*>(xs + (size_t)m * P.xs_row + pos * 8) = o;
        if (r == 0) sx[c * kSxCols + m] = sum;
    }
}

// One 128-k chunk of one lane: rows g, g+8 (words WA, WB), activations X;
// accumulates sum (128 + u) x into cm (staged), or sum (u - 8) x (unstaged).
template <int NT, bool XS>
__device__ __forceinline__ void chunk_mma(const uint4& WA, const uint4& WB, const uint4 (&X)[NT][4],
                                          uint32_t magic, uint32_t neg136, float (&cm)[NT][4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t wa = j == 0 ? WA.x : j == 1 ? WA.y : j == 2 ? WA.z : WA.w;
        const uint32_t wb = j == 0 ? WB.x : j == 1 ? WB.y : j == 2 ? WB.z : WB.w;
        uint32_t A[4], B[4];
        dequant_word(wa, magic, A);
        dequant_word(wb, magic, B);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                uint32_t b0, b1;
                if (XS) {  // staged in fragment order
                    b0 = h ? X[nt][j].z : X[nt][j].x;
                    b1 = h ? X[nt][j].w : X[nt][j].y;
                } else {   // natural order: (x0x1, x2x3, x4x5, x6x7)
                    const uint32_t lo = h ? X[nt][j].y : X[nt][j].x;
                    const uint32_t hi = h ? X[nt][j].w : X[nt][j].z;
                    b0 = prmt(lo, hi, 0x5410u);
                    b1 = prmt(lo, hi, 0x7632u);
                }
                mma_16816(cm[nt], A[2 * h], B[2 * h], A[2 * h + 1], B[2 * h + 1], b0, b1);
                // unstaged activations have no precomputed sums: the offset is
                // removed by a second MMA with the constant fragment -136
                if (!XS) mma_16816(cm[nt], neg136, neg136, neg136, neg136, b0, b1);
            }
        }
    }
}

// B fragments of chunk c: staged (xsb = shared address of this lane's clamped
// activation row + 16 t) or from global memory (xrow = clamped row + 32 t).
template <int NT, bool XS>
__device__ __forceinline__ void load_x(const __nv_bfloat16* const (&xrow)[NT],
                                       const uint32_t (&xsb)[NT], int c, uint4 (&X)[NT][4]) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (XS) X[nt][j] = lds128(xsb[nt] + c * 256 + j * 64);
            else    X[nt][j] = kc_ldg_keep(xrow[nt] + c * 128 + 8 * j);
        }
}

template <int NT, bool XS>
__global__ void __launch_bounds__(kThreads, 2) gemv_w4a16_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    using SM = Smem<NT>;
    SM& S = *reinterpret_cast<SM*>(smem_raw);
    float* sx = reinterpret_cast<float*>(smem_raw + fixed_smem<NT>());
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(sx + (size_t)P.sx_chunks * kSxCols);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int M = P.M, gshift = P.gshift, gs = P.gs, total = P.total_tiles;
    const uint32_t magic = P.magic, neg136 = P.neg136;

    if (threadIdx.x == 0) {
        for (int w = 0; w < kWarps; ++w)
            for (int i = 0; i < kRing; ++i) sm100::mbar_init(&S.wfull[w][i], 1);
        sm100::mbar_init(&S.sfull[0], 1);
        sm100::mbar_init(&S.sfull[1], 1);
        sm100::fence_barrier_init();
    }
    __syncthreads();
    if ((int)blockIdx.x >= total) return;

    // prologue: the first tile's scales, and the first kRing quads of every warp
    if (threadIdx.x == 0) issue_scales(P, blockIdx.x, S.scales[0], &S.sfull[0]);
    Cursor pf;
    pf.tile = blockIdx.x;
    pf.pi = problem_index(P, pf.tile);
    warp_chunks(P.p[pf.pi].K >> 7, warp, pf.c, pf.cend);
    cursor_settle(P, pf, warp);
    const bool leader = lane == 0;
    const uint32_t ring0 = sm100::smem_u32(&S.ring[warp][0][0][0]);
    const uint32_t bar0 = sm100::smem_u32(&S.wfull[warp][0]);
    for (int s = 0; s < kRing; ++s)
        issue_quad(P, pf, ring0 + s * kQuad * kChunkBytes, bar0 + 8 * s, warp, leader);

    const uint32_t ring_base = ring0 + g * 64 + 16 * t;
    const uint32_t sx_base = sm100::smem_u32(sx) + 8 * t;  // columns 2t, 2t+1 (+8 nt)
    uint32_t it = 0, ti = 0;
    int staged = -1;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
        const int pi = problem_index(P, tile);
        const Prob& pr = P.p[pi];
        const int N = pr.N, K = pr.K, C = K >> 7;
        const int row0 = (tile - pr.tile_begin) * 16;
        if (XS && pi != staged) {
            stage_activations(P, pi, sx, xs);  // every warp passed the previous tile's barrier
            __syncthreads();
            staged = pi;
        }
        const uint32_t sb = ti & 1u;
        sm100::mbar_wait(&S.sfull[sb], (ti >> 1) & 1u);
        if (threadIdx.x == 0 && tile + (int)gridDim.x < total) {
            // the other buffer's generic reads (previous tile) precede this async write
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_scales(P, tile + gridDim.x, S.scales[sb ^ 1u], &S.sfull[sb ^ 1u]);
        }
        const int G = K / gs;
        const uint32_t sa_base = sm100::smem_u32(&S.scales[sb][g * G]);
        const uint32_t sb_base = sa_base + 16 * G;  // row g + 8
        // activation rows of this lane's B fragments (columns >= M read row M - 1, discarded)
        const __nv_bfloat16* xrow[NT];
        uint32_t xsb[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int n = min(nt * 8 + g, M - 1);
            xrow[nt] = pr.x + (size_t)n * K + 32 * t;
            xsb[nt] = XS ? sm100::smem_u32(xs + (size_t)n * P.xs_row) + 16 * t : 0u;
        }

        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

        int c_begin, c_end;
        warp_chunks(C, warp, c_begin, c_end);
        for (int q0 = c_begin; q0 < c_end; q0 += kQuad, ++it) {
            const uint32_t s = it % kRing, ph = (it / kRing) & 1u;
            const int nq = min(kQuad, c_end - q0);
            const uint32_t st = ring_base + s * (kQuad * kChunkBytes);
            sm100::mbar_wait(&S.wfull[warp][s], ph);
#pragma unroll
            for (int j = 0; j < kQuad; ++j) {
                if (j < nq) {
                    const int c = q0 + j;
                    const int grp = c >> gshift;
                    const float sa = lds_half(sa_base + 2 * grp);
                    const float sb2 = lds_half(sb_base + 2 * grp);
                    uint4 X[NT][4];
                    load_x<NT, XS>(xrow, xsb, c, X);
                    const uint4 WA = lds128(st + j * kChunkBytes);
                    const uint4 WB = lds128(st + j * kChunkBytes + 512);
                    float cm[NT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) cm[nt][e] = 0.f;
                    chunk_mma<NT, XS>(WA, WB, X, magic, neg136, cm);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        // staged: minus 136 * sum x of this chunk (columns 2t, 2t+1 of tile nt)
                        float c0 = 0.f, c1 = 0.f;
                        if (XS) {
                            const float2 sxv = lds_f2(sx_base + (c * kSxCols + nt * 8) * 4);
                            c0 = 136.f * sxv.x;
                            c1 = 136.f * sxv.y;
                        }
                        acc[nt][0] = fmaf(sa, cm[nt][0] - c0, acc[nt][0]);
                        acc[nt][1] = fmaf(sa, cm[nt][1] - c1, acc[nt][1]);
                        acc[nt][2] = fmaf(sb2, cm[nt][2] - c0, acc[nt][2]);
                        acc[nt][3] = fmaf(sb2, cm[nt][3] - c1, acc[nt][3]);
                    }
                }
            }
            // the stage is consumed: refill it with the quad kRing ahead
            __syncwarp();
            if (leader) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_quad(P, pf, ring0 + s * kQuad * kChunkBytes, bar0 + 8 * s, warp, leader);
        }
        // cross-warp reduction of the tile
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            S.red[warp][g][nt * 8 + 2 * t]         = acc[nt][0];
            S.red[warp][g][nt * 8 + 2 * t + 1]     = acc[nt][1];
            S.red[warp][g + 8][nt * 8 + 2 * t]     = acc[nt][2];
            S.red[warp][g + 8][nt * 8 + 2 * t + 1] = acc[nt][3];
        }
        __syncthreads();
        for (int i = threadIdx.x; i < 16 * M; i += kThreads) {
            const int r = i & 15, n = i >> 4;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) v += S.red[w][r][n];
            if (row0 + r < N) pr.y[(size_t)n * N + row0 + r] = v;
        }
        __syncthreads();
    }
}

// CUDA-core fallback for shapes the tensor-core path cannot take (group sizes
// other than 128 * 2^m, K % 128 != 0, unaligned pointers).  One warp per row.
__global__ void __launch_bounds__(256) gemv_w4a16_scalar(const __grid_constant__ Params P) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    int total_rows = 0;
    for (int i = 0; i < P.count; ++i) total_rows += P.p[i].N;
    for (int gr = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; gr < total_rows; gr += warps) {
        int pi = 0, r = gr;
        while (r >= P.p[pi].N) { r -= P.p[pi].N; ++pi; }
        const Prob& pr = P.p[pi];
        const int K = pr.K, sc = K / P.gs;
        float acc[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) acc[m] = 0.f;
        for (int c = lane; c < K; c += 32) {
            const uint8_t p = pr.packed[(size_t)r * (K / 2) + c / 2];
            const int u = (c & 1) ? (p >> 4) : (p & 15);
            const float w = (float)(u - 8) * __half2float(pr.scales[(size_t)r * sc + c / P.gs]);
#pragma unroll
            for (int m = 0; m < 16; ++m)
                if (m < P.M) acc[m] = fmaf(w, __bfloat162float(pr.x[(size_t)m * K + c]), acc[m]);
        }
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            if (m < P.M) {
                const float s = kc_warp_sum(acc[m]);
                if (lane == 0) pr.y[(size_t)m * pr.N + r] = s;
            }
        }
    }
}


template <int NT, bool XS>
int launch_tc(const Params& P, size_t xs_bytes, cudaStream_t stream) {
    const size_t smem = fixed_smem<NT>() + (size_t)P.sx_chunks * kSxCols * 4 + xs_bytes;
    auto kern = gemv_w4a16_kernel<NT, XS>;
    KC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "gemv_w4a16 shared-memory attribute");
    int per_sm = 0;
    KC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem),
                "gemv_w4a16 occupancy");
    const int grid = std::min(P.total_tiles, kc::sm_count() * std::max(per_sm, 1));
    kern<<<grid, kThreads, smem, stream>>>(P);
    return kc::check_launch("gemv_w4a16");
}

// Largest activation block (bytes) staged in shared memory; above it the
// activations are read from global memory.
constexpr size_t kMaxStagedActivationBytes = 32 * 1024;

int launch(Params& P, cudaStream_t stream) {
    if (P.total_tiles == 0) return KC_OK;
    bool fast = true, single_group = true;
    int kmax = 0;
    for (int i = 0; i < P.count && fast; ++i) {
        const Prob& p = P.p[i];
        // TMA: 16-byte aligned base and row pitch; scale blocks: a tile's 16 rows
        // of K/gs halves must fit a slot, start 16-byte aligned, and a partial
        // last tile's block must stay a multiple of 16 bytes.
        const long row_bytes = 2L * (p.K / P.gs);
        const int tail = p.N % 16;
        fast = (p.K % 128 == 0) && kc::aligned(p.packed, 16) && kc::aligned(p.x, 16) &&
               kc::aligned(p.scales, 16) && 16 * row_bytes <= 2L * kScaleHalves &&
               (16 * row_bytes) % 16 == 0 && (tail == 0 || (tail * row_bytes) % 16 == 0);
        single_group = single_group && (p.K == P.gs);
        kmax = std::max(kmax, p.K);
    }
    int gshift = -1;
    for (int m = 0; m < 20; ++m)
        if (P.gs == (128 << m)) gshift = m;
    if (single_group) gshift = 31;
    P.gshift = gshift;
    P.magic = 0x43004300u;
    P.neg136 = 0xC308C308u;
    if (!fast || gshift < 0) {
        long rows = 0;
        for (int i = 0; i < P.count; ++i) rows += P.p[i].N;
        const long blocks = (rows + 7) / 8;
        const long cap = (long)kc::sm_count() * 8;
        gemv_w4a16_scalar<<<(int)std::max(1L, std::min(blocks, cap)), 256, 0, stream>>>(P);
        return kc::check_launch("gemv_w4a16_scalar");
    }
    for (int i = 0; i < P.count; ++i) {
        const Prob& p = P.p[i];
        const int st = kc::encode_2d(&P.wmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, p.packed,
                                     (uint64_t)(p.K / 2), (uint64_t)p.N, (uint64_t)(p.K / 2), 64, 16,
                                     CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st != KC_OK) return st;
    }
    const size_t xs_bytes = (size_t)P.M * kmax * 2;
    const bool stage = xs_bytes <= kMaxStagedActivationBytes;
    P.sx_chunks = stage ? kmax / 128 : 0;
    P.xs_row = stage ? kmax : 0;
    if (P.M <= 8)
        return stage ? launch_tc<1, true>(P, xs_bytes, stream) : launch_tc<1, false>(P, 0, stream);
    return stage ? launch_tc<2, true>(P, xs_bytes, stream) : launch_tc<2, false>(P, 0, stream);
}

}  // namespace

KC_DEFINE_STATUS_READER(gemv)

extern "C" {

int kc_gemv_w4a16_grouped(const kc_w4a16_problem* problems, int count, int M, int gs,
                          cudaStream_t stream) {
    KC_REQUIRE(problems != nullptr, KC_ERR_INVALID_ARG, "null problem list");
    KC_REQUIRE(count >= 1 && count <= KC_W4A16_MAX_PROBLEMS, KC_ERR_INVALID_ARG,
               "count=%d outside 1..%d", count, KC_W4A16_MAX_PROBLEMS);
    KC_REQUIRE(M >= 1 && M <= 16, KC_ERR_INVALID_ARG, "M=%d outside 1..16", M);
    KC_REQUIRE(gs > 0 && gs % 2 == 0, KC_ERR_INVALID_ARG, "group_size=%d must be even and > 0", gs);
    Params P{};
    P.count = count;
    P.M = M;
    P.gs = gs;
    long tiles = 0;
    for (int i = 0; i < count; ++i) {
        const kc_w4a16_problem& q = problems[i];
        KC_REQUIRE(q.packed && q.scales_f16 && q.x_bf16 && q.y, KC_ERR_INVALID_ARG,
                   "problem %d has a null pointer", i);
        KC_REQUIRE(q.N >= 0 && q.K > 0 && q.K % 2 == 0 && q.K % gs == 0, KC_ERR_INVALID_ARG,
                   "problem %d: bad shape N=%d K=%d for group_size=%d", i, q.N, q.K, gs);
        P.p[i].packed = q.packed;
        P.p[i].scales = reinterpret_cast<const __half*>(q.scales_f16);
        P.p[i].x = reinterpret_cast<const __nv_bfloat16*>(q.x_bf16);
        P.p[i].y = q.y;
        P.p[i].N = q.N;
        P.p[i].K = q.K;
        P.p[i].tile_begin = (int)tiles;
        tiles += (q.N + 15) / 16;
    }
    KC_REQUIRE(tiles < (1L << 30), KC_ERR_INVALID_ARG, "too many rows");
    P.total_tiles = (int)tiles;
    return launch(P, stream);
}

int kc_gemv_w4a16(const uint8_t* packed, const uint16_t* scales_f16, const uint16_t* x_bf16,
                  float* y, int M, int N, int K, int gs, cudaStream_t stream) {
    kc_w4a16_problem p{packed, scales_f16, x_bf16, y, N, K};
    return kc_gemv_w4a16_grouped(&p, 1, M, gs, stream);
}

}  // extern "C"
