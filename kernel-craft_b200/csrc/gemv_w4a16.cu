// gemv_w4a16.cu -- W4A16 GEMV / skinny GEMM (M <= 16) for sm_100a.
//
// y[m, n] = sum_k w[n, k] * x[m, k],  w[n, k] = (u - 8) * s[n, k / gs],
// u the unsigned nibble of packed[n, k / 2] (low nibble = even k), s fp16,
// x bf16, fp32 accumulation, fp32 y.  Several problems (e.g. the four
// projections of a decoder layer) can share one launch.
//
// Work decomposition: 16-row tiles in problem-major order, one persistent CTA
// per SM holding two or three independent groups of eight warps (Shape); the
// warps of a group split a tile's K range into contiguous runs of 128-k chunks
// (16 rows x 64 bytes = 1 KB each) and reduce their partial sums through
// shared memory at the end of the tile.
//
// Memory pipeline: every warp owns a ring of one or two stages in shared
// memory, each holding up to four chunks ("a quad", 4 KB).  Its lane 0 issues
// the quad's 2-D TMA loads (box 64 bytes x 16 rows; rows past N read as zero)
// on the stage's mbarrier as soon as the stage is consumed, so the ring runs
// ahead of the warp's compute across tile boundaries, and the 16-24 warps of
// an SM keep 96-128 KB of weights in flight; a tile's fp16 scale block (16
// contiguous rows) arrives by one bulk copy per tile, issued tiles ahead.
// One wait and one issue per 4 KB keeps the per-chunk bookkeeping small.
//
// Compute: a lane (g = lane / 4, t = lane % 4) reads rows g and g + 8, 16
// bytes each, of a chunk and turns every 32-bit word into four bf16x2 MMA
// fragments holding 128 + u exactly (nibble OR-ed into the mantissa of bf16
// 128.0; 3 shifts + 4 LOP3 per 8 weights), fed straight from registers into
// mma.sync m16n8k16 (weights as A, activations as B).  Activations are
// staged once per CTA in shared memory in fragment order (k0 k4 k1 k5 k2 k6
// k3 k7 per 8-block) when they fit, together with their per-chunk sums, and
// the offset is removed per chunk as sum (u - 8) x = sum (128 + u) x -
// 136 * sum x (the MMA accumulator starts at -136 * sum x); otherwise they
// are read from global memory (L1-resident), permuted with PRMT, and a second
// MMA with the constant fragment -136 removes the offset.  The group scale multiplies the per-chunk result.  MMA columns
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
    // or the same weights in tile order: [ceil(N/16)][K/128][16 rows][64 B],
    // every 16-row x 128-k chunk contiguous (kc_w4a16_tile_weights); a ring
    // stage is then one bulk copy instead of one 2-D box per chunk
    const uint8_t* tiled;
    const __half* scales;
    const uint8_t* zeros;  // per-group zero points u8[N, K/gs] (0..15); null: 8 (symmetric GPTQ)
    const __nv_bfloat16* x;
    float* y;
    int N, K;
    int tile_begin;  // first 16-row tile of this problem in the flattened tile list
    int xs_off;      // staged activations: byte offset of this problem's rows in shared memory
    int sx_off;      // staged chunk sums: first chunk row of this problem
};

struct alignas(64) Params {
    CUtensorMap wmap[KC_W4A16_MAX_PROBLEMS];  // packed weights: {K/2 bytes, N rows}, box {64, 16}
    Prob p[KC_W4A16_MAX_PROBLEMS];
    int count;
    int total_tiles;
    int M;
    int gs;
    int gshift;      // group of 128-k chunk c is c >> gshift
    int sx_chunks;     // chunk rows of the staged activation sums (all problems)
    uint32_t magic;  // 0x43004300 = bf16x2 (128, 128), held in a register (see nib_or)
    uint32_t neg136; // 0xC308C308 = bf16x2 (-136, -136): the unstaged path's offset MMA fragment
};

constexpr int kGroupWarps = 8;                    // warps that split one tile's K range
constexpr int kGroupThreads = kGroupWarps * 32;
constexpr int kChunkBytes = 1024;                 // 16 rows x 64 bytes = 128 k
constexpr int kQuad = 4;                          // chunks per stage

// CTA shape per activation tile count.  NT = 1 (M <= 8): three tile groups
// (24 warps) with one stage per warp -- more independent warps hide the
// per-chunk latency better than a deeper per-warp ring (34.2 vs 36.1 us per
// 7B layer at M = 1 on B200, 43.6 vs 47.5 at M = 4).  NT = 2 needs more
// registers per thread than 24 warps leave (the unstaged form spills), so it
// keeps two groups (16 warps) with two stages per warp.
template <int NT>
struct Shape {
    static constexpr int groups = NT == 1 ? 3 : 2;  // independent tile groups per CTA
    static constexpr int ring = NT == 1 ? 1 : 2;    // stages per warp
    static constexpr int warps = kGroupWarps * groups;
    static constexpr int threads = warps * 32;
};
constexpr int kScaleHalves = 16 * 128;            // 16 rows x up to 128 groups
constexpr int kScaleBufs = 3;                     // scale blocks in flight per group

template <int NT>
struct Smem {
    using Sh = Shape<NT>;
    uint8_t ring[Sh::warps][Sh::ring][kQuad][kChunkBytes];  // TMA destinations, 1024-byte aligned
    __half scales[Sh::groups][kScaleBufs][kScaleHalves];
    float red[Sh::groups][2][kGroupWarps][16][NT * 8 + 1];  // double-buffered by tile parity
    uint64_t wfull[Sh::warps][Sh::ring];
    uint64_t sfull[Sh::groups][kScaleBufs];
    int red_cnt[Sh::groups][2];    // warps that stored their partials for the slot's tile
    int red_done[Sh::groups][2];   // group tile counter of the last tile reduced from the slot
    // then, if staged: the chunk offsets float[sx_chunks][NT * 8], and the
    // activations of every problem, row m of problem i at
    // xs_off(i) + m * (2K + 16) bytes (the pad spreads rows over the banks),
    // in fragment order
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

// Chunk range [begin, end) of group warp w for a row of C 128-k chunks.
__device__ __forceinline__ void warp_chunks(int C, int w, int& begin, int& end) {
    begin = (w * C) / kGroupWarps;
    end = ((w + 1) * C) / kGroupWarps;
}

// A warp's position in its own sequence of (tile, quad) work items.
struct Cursor {
    int tile, c, cend, pi, step;
};

// Tiles of a group: vg, vg + G, vg + 2G, ... with vg = blockIdx + group *
// gridDim and G = step = groups * gridDim (every (CTA, group) pair walks its
// own tile sequence).
__device__ __forceinline__ void cursor_settle(const Params& P, Cursor& cu, int warp) {
    while (cu.tile < P.total_tiles && cu.c >= cu.cend) {
        cu.tile += cu.step;
        if (cu.tile >= P.total_tiles) break;
        // tiles only move forward, so the problem index does too
        while (cu.pi + 1 < P.count && cu.tile >= P.p[cu.pi + 1].tile_begin) ++cu.pi;
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
    if (const uint8_t* tiled = P.p[cu.pi].tiled) {
        // the quad's chunks are consecutive k-chunks of one tile: contiguous
        const uint8_t* src = tiled + ((size_t)(row0 >> 4) * (P.p[cu.pi].K >> 7) + cu.c) * kChunkBytes;
        asm volatile(
            "{\n\t.reg .pred l;\n\t"
            "setp.ne.b32 l, %0, 0;\n\t"
            "@l mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n\t"
            "@l cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%3], [%4], %2, [%1];\n\t}"
            ::"r"((int)leader), "r"(bar), "r"((uint32_t)n * kChunkBytes), "r"(dst), "l"(src)
            : "memory");
        cu.c += n;
        cursor_settle(P, cu, warp);
        return;
    }
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
    const int G = P.gshift == 31 ? 1 : ((pr.K >> 7) >> P.gshift);  // K / gs
    const uint32_t bytes = (uint32_t)min(16, pr.N - row0) * (uint32_t)G * 2u;
    sm100::mbar_arrive_expect_tx(bar, bytes);
    sm100::bulk_g2s(dst, pr.scales + (size_t)row0 * G, bytes, bar);
}

// One 128-k chunk of one lane: rows g, g+8 (words WA, WB), activations X.
// Staged (XS): X is in fragment order (x0x4, x1x5, x2x6, x3x7 per 8-block);
// the caller seeds cm with -136 * sum x of the chunk, and the chunk's eight
// MMAs add sum (128 + u) x into it in one chain, so cm leaves with
// sum (u - 8) x (one chain needs no accumulator merge; the other warps of the
// SM cover its latency).  Unstaged: X is in natural order (x0x1, x2x3, x4x5,
// x6x7), paired with PRMT, and a second MMA with the constant fragment -136
// removes the offset; those MMAs feed independent accumulators (per k half of
// each word, weights and offset apart) that are merged at the end.
template <int NT, bool XS>
__device__ __forceinline__ void chunk_mma(const uint4& WA, const uint4& WB, const uint4 (&X)[NT][4],
                                          uint32_t magic, uint32_t neg136, float (&cm)[NT][4]) {
    float c1[NT][4], o0[NT][4], o1[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) c1[nt][e] = o0[nt][e] = o1[nt][e] = 0.f;
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
                if (XS) {
                    b0 = h ? X[nt][j].z : X[nt][j].x;
                    b1 = h ? X[nt][j].w : X[nt][j].y;
                } else {
                    const uint32_t lo = h ? X[nt][j].y : X[nt][j].x;
                    const uint32_t hi = h ? X[nt][j].w : X[nt][j].z;
                    b0 = prmt(lo, hi, 0x5410u);
                    b1 = prmt(lo, hi, 0x7632u);
                }
                mma_16816((h && !XS) ? c1[nt] : cm[nt], A[2 * h], B[2 * h], A[2 * h + 1], B[2 * h + 1], b0, b1);
                if (!XS) mma_16816(h ? o1[nt] : o0[nt], neg136, neg136, neg136, neg136, b0, b1);
            }
        }
    }
    if (!XS)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) cm[nt][e] += c1[nt][e] + (o0[nt][e] + o1[nt][e]);
}

// Stages the activations of every problem: each 8-element block (16 bytes)
// is loaded from global memory, permuted to fragment order, and within each
// 128-k chunk the sixteen blocks b = 4t + j (k = 32t + 8j) move to position
// 4j + t, so a lane's LDS.128 for word j hits 16 consecutive bytes per t.  The
// same pass forms the per-chunk offsets sx[c][m] = -136 * sum x (fp32, the
// seed of the chunk's MMA accumulator): a chunk's 16 blocks belong to 16
// consecutive lanes of one warp.  Work is handed out in units of 32 blocks,
// one per lane, and every warp loads U units before it processes any, so the
// loads of a warp are in flight together.  Plain loads rather than a bulk
// copy: a bulk copy queues behind the weight tiles the CTA has already
// requested and lands later.
template <int NT>
__device__ __forceinline__ void stage_activations(const Params& P, uint8_t* xs, float* sx) {
    constexpr int kCols = NT * 8, kThreads = Shape<NT>::threads, kW = kThreads / 32, U = 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // sums of columns m >= M stay zero (columns m < M are all written below)
    for (int i = threadIdx.x; i < P.sx_chunks * kCols; i += kThreads)
        if (i % kCols >= P.M) sx[i] = 0.f;
    int total_units = 0;
    for (int pi = 0; pi < P.count; ++pi) total_units += P.M * ((P.p[pi].K + 255) >> 8);
    for (int u0 = warp; u0 < total_units; u0 += U * kW) {
        uint4 v[U];
        int pis[U], ms[U], kbs[U];
#pragma unroll
        for (int b = 0; b < U; ++b) {
            int u = u0 + b * kW;
            pis[b] = -1;
            if (u < total_units) {
                int pi = 0;
                while (u >= P.M * ((P.p[pi].K + 255) >> 8)) {
                    u -= P.M * ((P.p[pi].K + 255) >> 8);
                    ++pi;
                }
                const int per = (P.p[pi].K + 255) >> 8;  // units per activation row
                pis[b] = pi;
                ms[b] = u / per;
                kbs[b] = (u % per) * 32 + lane;
                const uint4* xrow = reinterpret_cast<const uint4*>(P.p[pi].x + (size_t)ms[b] * P.p[pi].K);
                v[b] = kbs[b] < (P.p[pi].K >> 3) ? __ldcg(xrow + kbs[b]) : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int b = 0; b < U; ++b) {
            if (pis[b] < 0) break;  // warp-uniform
            const Prob& pr = P.p[pis[b]];
            float sum = 0.f;
            const uint32_t w4[4] = {v[b].x, v[b].y, v[b].z, v[b].w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                sum += __uint_as_float(w4[i] << 16) + __uint_as_float(w4[i] & 0xFFFF0000u);
#pragma unroll
            for (int o = 8; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            const int kb = kbs[b], c = kb >> 4, r = kb & 15;
            if (kb >= (pr.K >> 3)) continue;  // past the row (K % 256 == 128)
            uint8_t* row = xs + pr.xs_off + (size_t)ms[b] * (2 * pr.K + 16);
            const int pos = (c << 4) + ((r & 3) << 2) + (r >> 2);
            *reinterpret_cast<uint4*>(row + pos * 16) =
                make_uint4(prmt(v[b].x, v[b].z, 0x5410u), prmt(v[b].x, v[b].z, 0x7632u),
                           prmt(v[b].y, v[b].w, 0x5410u), prmt(v[b].y, v[b].w, 0x7632u));
            if (r == 0) sx[(pr.sx_off + c) * kCols + ms[b]] = -136.f * sum;
        }
    }
}

// Activations of chunk c for this lane's B fragments: from shared memory in
// fragment order (xsb = this lane's clamped row + 16 t; block 4j + t) or from
// global memory in natural order (xrow = clamped row + 32 t; k = 32 t + 8 j).
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
__global__ void __launch_bounds__(Shape<NT>::threads, 1) gemv_w4a16_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    using SM = Smem<NT>;
    constexpr int kCols = NT * 8;
    constexpr int kGroups = Shape<NT>::groups, kWarps = Shape<NT>::warps, kRing = Shape<NT>::ring;
    SM& S = *reinterpret_cast<SM*>(smem_raw);
    float* sx = reinterpret_cast<float*>(smem_raw + fixed_smem<NT>());
    uint8_t* xs = reinterpret_cast<uint8_t*>(sx + (size_t)P.sx_chunks * kCols);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int group = warp / kGroupWarps, gw = warp % kGroupWarps;
    const int gtid = threadIdx.x % kGroupThreads;
    const int g = lane >> 2, t = lane & 3;
    const int M = P.M, gshift = P.gshift, total = P.total_tiles;
    const uint32_t magic = P.magic, neg136 = P.neg136;
    // group-major: consecutive tiles (the longest-K ones first) go to different
    // SMs before any SM gets a second one, which evens out the work per SM
    const int first = blockIdx.x + group * gridDim.x, stride = kGroups * gridDim.x;

    // the next launch in the stream may start its prologue while this grid drains
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int w = 0; w < kWarps; ++w)
            for (int i = 0; i < kRing; ++i) sm100::mbar_init(&S.wfull[w][i], 1);
        for (int h = 0; h < kGroups; ++h) {
            for (int i = 0; i < kScaleBufs; ++i) sm100::mbar_init(&S.sfull[h][i], 1);
            S.red_cnt[h][0] = S.red_cnt[h][1] = 0;
            S.red_done[h][0] = S.red_done[h][1] = -1;
        }
        sm100::fence_barrier_init();
    }
    __syncthreads();

    // prologue: the group's first kScaleBufs scale blocks and the first kRing
    // weight quads of every warp.  Weights and scales are issued before the
    // wait on the previous grid: they are layer constants that no kernel of
    // this library writes, so the loads overlap the previous grid's drain.
    if (gtid == 0)
        for (int i = 0; i < kScaleBufs && first + i * stride < total; ++i)
            issue_scales(P, first + i * stride, S.scales[group][i], &S.sfull[group][i]);
    Cursor pf;
    pf.tile = first;
    pf.c = pf.cend = 0;
    pf.pi = 0;
    pf.step = stride;
    if (pf.tile < total) {
        pf.pi = problem_index(P, pf.tile);
        warp_chunks(P.p[pf.pi].K >> 7, gw, pf.c, pf.cend);
        cursor_settle(P, pf, gw);
    }
    const bool leader = lane == 0;
    const uint32_t ring0 = sm100::smem_u32(&S.ring[warp][0][0][0]);
    const uint32_t bar0 = sm100::smem_u32(&S.wfull[warp][0]);
    for (int s = 0; s < kRing; ++s)
        issue_quad(P, pf, ring0 + s * kQuad * kChunkBytes, bar0 + 8 * s, gw, leader);

    // the activations (and y) may be produced / consumed by the previous grid
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (XS) {
        stage_activations<NT>(P, xs, sx);
        __syncthreads();
    }
    const uint32_t sx_base = sm100::smem_u32(sx) + 8 * t;  // columns 2t, 2t+1 (+8 nt)

    const uint32_t ring_base = ring0 + g * 64 + 16 * t;
    uint32_t it = 0, ti = 0;
    int pi = 0;
    for (int tile = first; tile < total; tile += stride, ++ti) {
        while (pi + 1 < P.count && tile >= P.p[pi + 1].tile_begin) ++pi;
        const Prob& pr = P.p[pi];
        const int N = pr.N, K = pr.K, C = K >> 7;
        const int row0 = (tile - pr.tile_begin) * 16;
        const uint32_t sb = ti % kScaleBufs;
        sm100::mbar_wait(&S.sfull[group][sb], (ti / kScaleBufs) & 1u);
        const int G = gshift == 31 ? 1 : (C >> gshift);  // K / gs without a division
        const uint32_t sa_base = sm100::smem_u32(&S.scales[group][sb][g * G]);
        const uint32_t sb_base = sa_base + 16 * G;  // row g + 8
        // activation rows of this lane's B fragments (columns >= M read row M - 1, discarded)
        const __nv_bfloat16* xrow[NT];
        uint32_t xsb[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int n = min(nt * 8 + g, M - 1);
            xrow[nt] = pr.x + (size_t)n * K + 32 * t;
            xsb[nt] = XS ? sm100::smem_u32(xs + pr.xs_off + (size_t)n * (2 * K + 16)) + 16 * t : 0u;
        }
        const uint32_t sxp = sx_base + (uint32_t)pr.sx_off * kCols * 4;

        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

        int c_begin, c_end;
        warp_chunks(C, gw, c_begin, c_end);
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
                    // seeded with -136 * sum x of this chunk (columns 2t, 2t+1 of tile nt)
                    float cm[NT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        if (XS) {
                            const float2 o = lds_f2(sxp + (c * kCols + nt * 8) * 4);
                            cm[nt][0] = o.x;
                            cm[nt][1] = o.y;
                            cm[nt][2] = o.x;
                            cm[nt][3] = o.y;
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) cm[nt][e] = 0.f;
                        }
                    }
                    chunk_mma<NT, XS>(WA, WB, X, magic, neg136, cm);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        acc[nt][0] = fmaf(sa, cm[nt][0], acc[nt][0]);
                        acc[nt][1] = fmaf(sa, cm[nt][1], acc[nt][1]);
                        acc[nt][2] = fmaf(sb2, cm[nt][2], acc[nt][2]);
                        acc[nt][3] = fmaf(sb2, cm[nt][3], acc[nt][3]);
                    }
                }
            }
            // the stage is consumed: refill it with the quad kRing ahead
            __syncwarp();
            if (leader) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_quad(P, pf, ring0 + s * kQuad * kChunkBytes, bar0 + 8 * s, gw, leader);
        }
        // Cross-warp reduction without a barrier: each warp stores its partials
        // in the slot of this tile's parity and counts itself in; the warp that
        // arrives last sums the slot, writes y, refills this tile's scale
        // buffer (every warp of the group is past its reads) and releases the
        // slot for the tile two ahead.
        const uint32_t slot = ti & 1u;
        if (ti >= 2 && lane == 0) {
            volatile int* done = &S.red_done[group][slot];
            const uint64_t t0 = sm100::globaltimer();
            while (*done != (int)ti - 2) {
                if (sm100::globaltimer() - t0 > KC_WAIT_TIMEOUT_NS) {
                    sm100::record_status(KC_ERR_TIMEOUT);
                    break;
                }
            }
        }
        __syncwarp();
        auto& red = S.red[group][slot];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            red[gw][g][nt * 8 + 2 * t]         = acc[nt][0];
            red[gw][g][nt * 8 + 2 * t + 1]     = acc[nt][1];
            red[gw][g + 8][nt * 8 + 2 * t]     = acc[nt][2];
            red[gw][g + 8][nt * 8 + 2 * t + 1] = acc[nt][3];
        }
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&S.red_cnt[group][slot], 1) == kGroupWarps - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane == 0 && tile + kScaleBufs * stride < total) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_scales(P, tile + kScaleBufs * stride, S.scales[group][sb], &S.sfull[group][sb]);
            }
            for (int i = lane; i < 16 * M; i += 32) {
                const int r = i & 15, n = i >> 4;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kGroupWarps; ++w) v += red[w][r][n];
                if (row0 + r < N) pr.y[(size_t)n * N + row0 + r] = v;
            }
            __syncwarp();
            if (lane == 0) {
                S.red_cnt[group][slot] = 0;
                __threadfence_block();
                *reinterpret_cast<volatile int*>(&S.red_done[group][slot]) = (int)ti;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// M = 1: integer tensor-core path
// ---------------------------------------------------------------------------
// At batch 1 the kernel is bound by instruction issue, and most of the issue
// went to turning nibbles into bf16 fragments (7 ALU operations per 8
// weights).  This path feeds the weights to the integer MMA instead:
// mma.sync m16n8k32 .u8 x .s8/.u8 runs at the same instruction rate as the
// bf16 m16n8k16 with twice the k per instruction (measured on B200), and a
// packed word becomes two u8 fragments with one shift and two ANDs
// (w & 0x0F0F0F0F: k 0 2 4 6; (w >> 4) & 0x0F0F0F0F: k 1 3 5 7).
//
// The activations become integers once per CTA: with f = 2^-F, F chosen per
// activation row so that max|x| * 2^F lies in [2^21, 2^22), q = rint(x * 2^F)
// is exact for every bf16 value within 2^14 of the row maximum and off by at
// most 2^-23 of that maximum otherwise (the relative error this adds to y is
// about 2^-23 * max|x| / rms(x), under 1e-4 even at max/rms = 1000).  q' = q + 2^22 in [0, 2^23) is the
// low 23 bits of the float x * 2^F + 1.5 * 2^23 (one FMA, no conversion
// instruction), and its three bytes B2 B1 B0 are three u8 planes.  The MMA's
// eight columns carry the planes: column 0 = B2, 1 = B1, 2 = B0, and column
// 3 a plane of ones, so ONE instruction per 32 k gives, per weight row,
//   D_p = sum_k (u - 8) * B_p   (accumulator seeded with -8 * sum_k B_p)
//   D_3 = sum_k (u - 8)         (seeded with -8 * 32 * 4 = -1024)
// and sum_k (u - 8) * q = 65536 D_0 + 256 D_1 + D_2 - 2^22 D_3, all exact in
// int32.  Each column is scaled by the group scale s in fp32 per chunk (s
// changes per chunk); the columns are combined, and multiplied by f, once per
// tile.
//
// Staged layout of one chunk (kI8ChunkBytes): for half h (k-steps 2h, 2h+1)
// and plane p, lane t's 16 bytes [b0 b1 of step 2h | b0 b1 of step 2h+1] at
// 192 h + 64 p + 16 t (b0: the plane's bytes of k = 32 t + 8 j + 0 2 4 6, b1:
// of k + 1), then the seeds {-8 sum B_0, -8 sum B_1, -8 sum B_2, -1024}.
// Lanes whose B column is 3 or more read a shared 256-byte plane of ones.
constexpr int kI8ChunkBytes = 400;
constexpr int kI8RecOffset = 384;

struct SmemI8 {
    using Sh = Shape<1>;
    uint8_t ring[Sh::warps][Sh::ring][kQuad][kChunkBytes];  // TMA destinations, 1024-byte aligned
    __half scales[Sh::groups][kScaleBufs][kScaleHalves];
    float red[Sh::groups][2][kGroupWarps][16];   // per-warp row sums, double-buffered by tile parity
    alignas(16) uint32_t ones[64];               // 256 bytes of 0x01
    unsigned int row_max[KC_W4A16_MAX_PROBLEMS];   // max |x| per problem (float bits)
    float row_f[KC_W4A16_MAX_PROBLEMS];            // f = 2^-F per problem
    uint64_t wfull[Sh::warps][Sh::ring];
    uint64_t sfull[Sh::groups][kScaleBufs];
    int red_cnt[Sh::groups][2];
    int red_done[Sh::groups][2];
    // then the staged chunks: global chunk c (problem order) at c * kI8ChunkBytes
};

__host__ __device__ constexpr size_t fixed_smem_i8() { return (sizeof(SmemI8) + 127) / 128 * 128; }

__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                           uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// As imma_16832, with the accumulator input C given apart from the output D
// (the chunk's first k-step starts from the seeds without copying them).
__device__ __forceinline__ void imma_16832_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1, uint32_t c0,
                                             uint32_t c1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// max that propagates NaN (a chunk holding a NaN must not look finite)
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

// Most chunks the batch-1 path stages (shared memory left after its fixed
// part).
constexpr int kI8MaxChunks = (int)((227 * 1024 - fixed_smem_i8()) / kI8ChunkBytes);

// Stages the one activation row (M = 1) of every problem as byte planes.
// One thread per pair of 8-element blocks (k-steps 2h and 2h + 1 of lane
// slot t: 16 elements, whose planes are 16 contiguous bytes per plane); the 8
// pairs of a chunk are 8 consecutive threads, which reduce the chunk's plane
// sums with three shuffle levels.  Every load is issued before any is used,
// so the loads cost one round trip; every thread of a warp runs the same
// number of rounds, so the full-warp shuffles are legal.  Two passes: the
// maximum of each problem's row (shared-memory atomicMax on the float bits,
// which order like the values for non-negative floats and put NaN and Inf
// above every finite value), a barrier, then the planes.
__device__ __forceinline__ int chunk_problem(const Params& P, int c) {
    int pi = 0;
    while (pi + 1 < P.count && c >= P.p[pi + 1].sx_off) ++pi;
    return pi;
}

__device__ __forceinline__ void bf16x8(const uint4& w, float* v) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(ws[i] << 16);
        v[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
    }
}

// Plane words of one 8-element block q[0..7] (float bits holding q' in bits
// 0..22): p0[sl] = bytes of the even elements, p1[sl] = of the odd ones; slot
// 0 = byte 2, slot 1 = byte 1, slot 2 = byte 0.  Byte transpose: t = [a.b0
// b.b0 a.b2 b.b2], u = [a.b1 b.b1 a.b3 b.b3] for the pairs (0,2) (4,6) (1,3)
// (5,7), then one PRMT per plane word.
__device__ __forceinline__ void planes8(const uint32_t* q, uint32_t* p0, uint32_t* p1) {
    const uint32_t t02 = prmt(q[0], q[2], 0x6240u), t46 = prmt(q[4], q[6], 0x6240u);
    const uint32_t u02 = prmt(q[0], q[2], 0x7351u), u46 = prmt(q[4], q[6], 0x7351u);
    const uint32_t t13 = prmt(q[1], q[3], 0x6240u), t57 = prmt(q[5], q[7], 0x6240u);
    const uint32_t u13 = prmt(q[1], q[3], 0x7351u), u57 = prmt(q[5], q[7], 0x7351u);
    p0[0] = prmt(t02, t46, 0x7632u);
    p0[1] = prmt(u02, u46, 0x5410u);
    p0[2] = prmt(t02, t46, 0x5410u);
    p1[0] = prmt(t13, t57, 0x7632u);
    p1[1] = prmt(u13, u57, 0x5410u);
    p1[2] = prmt(t13, t57, 0x5410u);
}

constexpr int kI8MaxPairRounds = (kI8MaxChunks * 8 + Shape<1>::threads - 1) / Shape<1>::threads;

// With per-group zero points (ZP) the seeds depend on the weight row, so the
// record holds the negated plane sums (and -128 for the ones column) and the
// chunk multiplies them by each row's zero point; without, it holds the
// seeds of zero point 8 directly.
template <bool ZP>
__device__ __forceinline__ void stage_i8(const Params& P, SmemI8& S, uint8_t* xs) {
    constexpr int kSeedMul = ZP ? -1 : -8;
    constexpr int kThreads = Shape<1>::threads;
    const int total = P.sx_chunks * 8;  // block pairs
    uint4 w[kI8MaxPairRounds][2];
    // pair (c, r): lane slot t = r >> 1, half h = r & 1, blocks 4t + 2h, 4t + 2h + 1
#pragma unroll
    for (int rd = 0; rd < kI8MaxPairRounds; ++rd) {
        const int b = rd * kThreads + threadIdx.x;
        w[rd][0] = w[rd][1] = make_uint4(0, 0, 0, 0);
        if (b < total) {
            const int c = b >> 3, r = b & 7, pi = chunk_problem(P, c);
            const uint4* x = reinterpret_cast<const uint4*>(P.p[pi].x + (size_t)(c - P.p[pi].sx_off) * 128) +
                             4 * (r >> 1) + 2 * (r & 1);
            w[rd][0] = __ldcg(x);
            w[rd][1] = __ldcg(x + 1);
        }
    }
    // pass 1: row maxima
#pragma unroll
    for (int rd = 0; rd < kI8MaxPairRounds; ++rd) {
        if (rd * kThreads >= total) break;  // uniform over the CTA
        const int b = rd * kThreads + threadIdx.x;
        float v[16];
        bf16x8(w[rd][0], v);
        bf16x8(w[rd][1], v + 8);
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) m = fmax_nan(m, fabsf(v[i]));
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (b < total && (b & 7) == 0) atomicMax(&S.row_max[chunk_problem(P, b >> 3)], __float_as_uint(m));
    }
    __syncthreads();
    // pass 2: planes and seeds
#pragma unroll
    for (int rd = 0; rd < kI8MaxPairRounds; ++rd) {
        if (rd * kThreads >= total) break;  // uniform over the CTA
        const int b = rd * kThreads + threadIdx.x;
        const bool active = b < total;
        const int c = b >> 3, r = b & 7;
        // max * 2^F in [2^21, 2^22): F = 148 - biased exponent of the row
        // maximum (clamped so 2^F stays a normal float; an all-zero row gets
        // F = 127 and q = 0)
        const int e = active ? (int)((S.row_max[chunk_problem(P, c)] >> 23) & 0xFF) : 0;
        const float up = __uint_as_float((uint32_t)(127 + max(-126, min(127, 148 - e))) << 23);
        float v[16];
        bf16x8(w[rd][0], v);
        bf16x8(w[rd][1], v + 8);
        uint32_t q[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) q[i] = __float_as_uint(fmaf(v[i], up, 12582912.0f));
        uint32_t pa0[3], pa1[3], pb0[3], pb1[3];
        planes8(q, pa0, pa1);       // block 4t + 2h     (k-step 2h)
        planes8(q + 8, pb0, pb1);   // block 4t + 2h + 1 (k-step 2h + 1)
        // plane sums: slot 0 in the low 16 bits, slot 1 in the high (each at
        // most 128 * 255 < 2^16 over the chunk), slot 2 apart
        uint32_t s0 = __dp4a(pa0[0], 0x01010101u, __dp4a(pa1[0], 0x01010101u,
                      __dp4a(pb0[0], 0x01010101u, __dp4a(pb1[0], 0x01010101u, 0u))));
        uint32_t s1 = __dp4a(pa0[1], 0x01010101u, __dp4a(pa1[1], 0x01010101u,
                      __dp4a(pb0[1], 0x01010101u, __dp4a(pb1[1], 0x01010101u, 0u))));
        uint32_t s2 = __dp4a(pa0[2], 0x01010101u, __dp4a(pa1[2], 0x01010101u,
                      __dp4a(pb0[2], 0x01010101u, __dp4a(pb1[2], 0x01010101u, 0u))));
        uint32_t s01 = s0 + (s1 << 16);
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) {
            s01 += __shfl_xor_sync(0xffffffffu, s01, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
        if (active) {
            uint8_t* ch = xs + (size_t)c * kI8ChunkBytes + (r & 1) * 192 + (r >> 1) * 16;
#pragma unroll
            for (int sl = 0; sl < 3; ++sl)
                *reinterpret_cast<uint4*>(ch + sl * 64) = make_uint4(pa0[sl], pa1[sl], pb0[sl], pb1[sl]);
            if (r == 0)
                *reinterpret_cast<int4*>(xs + (size_t)c * kI8ChunkBytes + kI8RecOffset) =
                    make_int4(kSeedMul * (int)(s01 & 0xFFFFu), kSeedMul * (int)(s01 >> 16),
                              kSeedMul * (int)s2, kSeedMul * 128);
        }
    }
    // f = 2^-F per problem; an Inf or NaN in the row (exponent 255) makes it NaN
    if (threadIdx.x < P.count) {
        const int e = (int)((S.row_max[threadIdx.x] >> 23) & 0xFF);
        S.row_f[threadIdx.x] =
            e == 255 ? __uint_as_float(0x7FC00000u) : ldexpf(1.0f, -max(-126, min(127, 148 - e)));
    }
}

// As imma_16832_c with a separate seed per accumulator element (rows g and
// g + 8 differ when the zero point is per row).
__device__ __forceinline__ void imma_16832_c4(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1, int c0, int c1,
                                              int c2, int c3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2),
          "r"(c3));
}

// One 128-k chunk of the batch-1 path for one lane: rows g and g + 8 of the
// weight stage at wst (16 bytes each), this lane's B column of chunk c at xa
// (two 16-byte halves 192 bytes apart), its two column seeds at rec; four
// MMAs (32 k each), then the group scales of the two rows times the integer
// sums into the fp32 column accumulators.
// With zero points, za and zb are the zero points of rows g and g + 8.
template <bool ZP>
__device__ __forceinline__ void i8_chunk(uint32_t wst, uint32_t xa, uint32_t rec, uint32_t sa,
                                         uint32_t sb, int za, int zb, float (&acc)[4]) {
    constexpr uint32_t m = 0x0F0F0F0Fu;
    const uint4 X0 = lds128(xa), X1 = lds128(xa + 192);
    const uint2 seed = lds64(rec);
    const uint4 WA = lds128(wst), WB = lds128(wst + 512);
    const float fa = lds_half(sa), fb = lds_half(sb);
    int d[4];
    if (ZP)
        imma_16832_c4(d, WA.x & m, WB.x & m, (WA.x >> 4) & m, (WB.x >> 4) & m, X0.x, X0.y,
                      za * (int)seed.x, za * (int)seed.y, zb * (int)seed.x, zb * (int)seed.y);
    else
        imma_16832_c(d, WA.x & m, WB.x & m, (WA.x >> 4) & m, (WB.x >> 4) & m, X0.x, X0.y, seed.x, seed.y);
    imma_16832(d, WA.y & m, WB.y & m, (WA.y >> 4) & m, (WB.y >> 4) & m, X0.z, X0.w);
    imma_16832(d, WA.z & m, WB.z & m, (WA.z >> 4) & m, (WB.z >> 4) & m, X1.x, X1.y);
    imma_16832(d, WA.w & m, WB.w & m, (WA.w >> 4) & m, (WB.w >> 4) & m, X1.z, X1.w);
    acc[0] = fmaf(fa, (float)d[0], acc[0]);
    acc[1] = fmaf(fa, (float)d[1], acc[1]);
    acc[2] = fmaf(fb, (float)d[2], acc[2]);
    acc[3] = fmaf(fb, (float)d[3], acc[3]);
}

template <bool ZP>
__global__ void __launch_bounds__(Shape<1>::threads, 1) gemv_w4a16_i8_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    using Sh = Shape<1>;
    constexpr int kGroups = Sh::groups, kWarps = Sh::warps, kRing = Sh::ring;
    SmemI8& S = *reinterpret_cast<SmemI8*>(smem_raw);
    uint8_t* xs = smem_raw + fixed_smem_i8();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int group = warp / kGroupWarps, gw = warp % kGroupWarps;
    const int gtid = threadIdx.x % kGroupThreads;
    const int g = lane >> 2, t = lane & 3;
    const int gshift = P.gshift, total = P.total_tiles;
    const int first = blockIdx.x + group * gridDim.x, stride = kGroups * gridDim.x;

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int w = 0; w < kWarps; ++w)
            for (int i = 0; i < kRing; ++i) sm100::mbar_init(&S.wfull[w][i], 1);
        for (int h = 0; h < kGroups; ++h) {
            for (int i = 0; i < kScaleBufs; ++i) sm100::mbar_init(&S.sfull[h][i], 1);
            S.red_cnt[h][0] = S.red_cnt[h][1] = 0;
            S.red_done[h][0] = S.red_done[h][1] = -1;
        }
        sm100::fence_barrier_init();
    }
    if (threadIdx.x < 64) S.ones[threadIdx.x] = 0x01010101u;
    if (threadIdx.x < KC_W4A16_MAX_PROBLEMS) S.row_max[threadIdx.x] = 0u;
    __syncthreads();

    // prologue: scales and the first weight quads, before the wait on the
    // previous grid (layer constants no kernel of this library writes)
    if (gtid == 0)
        for (int i = 0; i < kScaleBufs && first + i * stride < total; ++i)
            issue_scales(P, first + i * stride, S.scales[group][i], &S.sfull[group][i]);
    Cursor pf;
    pf.tile = first;
    pf.c = pf.cend = 0;
    pf.pi = 0;
    pf.step = stride;
    if (pf.tile < total) {
        pf.pi = problem_index(P, pf.tile);
        warp_chunks(P.p[pf.pi].K >> 7, gw, pf.c, pf.cend);
        cursor_settle(P, pf, gw);
    }
    const bool leader = lane == 0;
    const uint32_t ring0 = sm100::smem_u32(&S.ring[warp][0][0][0]);
    const uint32_t bar0 = sm100::smem_u32(&S.wfull[warp][0]);
    for (int s = 0; s < kRing; ++s)
        issue_quad(P, pf, ring0 + s * kQuad * kChunkBytes, bar0 + 8 * s, gw, leader);
    // warm L2 with this CTA's share of the activations (128-byte lines L =
    // blockIdx + gridDim * i over all problems) while the previous grid
    // drains.  Only L2 is touched: the previous grid's writes land in L2, and
    // the staging reads after the wait below see them.
    {
        int L = blockIdx.x + gridDim.x * threadIdx.x, pi = 0, base = 0;
        while (pi < P.count && L >= base + (P.p[pi].K >> 6)) base += P.p[pi++].K >> 6;
        if (pi < P.count)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(P.p[pi].x + (size_t)(L - base) * 64));
    }

    asm volatile("griddepcontrol.wait;" ::: "memory");
    stage_i8<ZP>(P, S, xs);
    __syncthreads();

    // this lane's B column: planes for g < 3, the ones plane otherwise
    const uint32_t xs_u32 = sm100::smem_u32(xs);
    const uint32_t xlane = g < 3 ? xs_u32 + g * 64 + t * 16 : sm100::smem_u32(S.ones) + t * 16;
    const uint32_t xstep = g < 3 ? (uint32_t)kI8ChunkBytes : 0u;
    // the seeds of chunk 0: this lane's two columns (2t, 2t + 1; lanes t >= 2
    // hold columns no plane feeds)
    const uint32_t rec0 = xs_u32 + kI8RecOffset;
    const uint32_t seed_off = t == 0 ? 0u : 8u;
    const uint32_t ring_base = ring0 + g * 64 + 16 * t;
    uint32_t it = 0, ti = 0;
    int pi = 0;
    for (int tile = first; tile < total; tile += stride, ++ti) {
        while (pi + 1 < P.count && tile >= P.p[pi + 1].tile_begin) ++pi;
        const Prob& pr = P.p[pi];
        const int N = pr.N, C = pr.K >> 7;
        const int row0 = (tile - pr.tile_begin) * 16;
        const uint32_t sb = ti % kScaleBufs;
        sm100::mbar_wait(&S.sfull[group][sb], (ti / kScaleBufs) & 1u);
        const int G = gshift == 31 ? 1 : (C >> gshift);
        const uint32_t sa_base = sm100::smem_u32(&S.scales[group][sb][g * G]);
        const uint32_t sb_base = sa_base + 16 * G;
        const uint32_t xp = xlane + xstep * (uint32_t)pr.sx_off;          // chunk 0 of this problem
        const uint32_t recp = rec0 + (uint32_t)(kI8ChunkBytes * pr.sx_off) + seed_off;
        // zero points of rows g and g + 8 (rows past N read the last row)
        // (a problem without zero points in a launch that has some uses 8)
        const bool has_z = ZP && pr.zeros != nullptr;
        const uint8_t* za_row = has_z ? pr.zeros + (size_t)min(row0 + g, N - 1) * G : nullptr;
        const uint8_t* zb_row = has_z ? pr.zeros + (size_t)min(row0 + g + 8, N - 1) * G : nullptr;

        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        int c_begin, c_end;
        warp_chunks(C, gw, c_begin, c_end);
        for (int q0 = c_begin; q0 < c_end; q0 += kQuad, ++it) {
            const uint32_t s = it % kRing, ph = (it / kRing) & 1u;
            const int nq = min(kQuad, c_end - q0);
            const uint32_t st = ring_base + s * (kQuad * kChunkBytes);
            sm100::mbar_wait(&S.wfull[warp][s], ph);
            const uint32_t c0 = (uint32_t)q0;
            if (nq == kQuad) {   // a full stage: no per-chunk guard
#pragma unroll 1
                for (int j = 0; j < kQuad; ++j) {
                    const uint32_t c = c0 + j, grp = c >> gshift;
                    const int za = has_z ? (int)__ldg(za_row + grp) : 8;
                    const int zb = has_z ? (int)__ldg(zb_row + grp) : 8;
                    i8_chunk<ZP>(st + j * kChunkBytes, xp + c * xstep, recp + c * kI8ChunkBytes,
                                 sa_base + 2 * grp, sb_base + 2 * grp, za, zb, acc);
                }
            } else {
#pragma unroll 1
                for (int j = 0; j < nq; ++j) {
                    const uint32_t c = c0 + j, grp = c >> gshift;
                    const int za = has_z ? (int)__ldg(za_row + grp) : 8;
                    const int zb = has_z ? (int)__ldg(zb_row + grp) : 8;
                    i8_chunk<ZP>(st + j * kChunkBytes, xp + c * xstep, recp + c * kI8ChunkBytes,
                                 sa_base + 2 * grp, sb_base + 2 * grp, za, zb, acc);
                }
            }
            __syncwarp();
            if (leader) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_quad(P, pf, ring0 + s * kQuad * kChunkBytes, bar0 + 8 * s, gw, leader);
        }
        // columns -> row sums: lane t = 1 holds B0 (col 2) and the ones
        // column (col 3), lane t = 0 B2 (col 0) and B1 (col 1)
        const float lo_g = __shfl_down_sync(0xffffffffu, fmaf(-4194304.f, acc[1], acc[0]), 1);
        const float lo_g8 = __shfl_down_sync(0xffffffffu, fmaf(-4194304.f, acc[3], acc[2]), 1);
        const float v_g = fmaf(65536.f, acc[0], fmaf(256.f, acc[1], lo_g));
        const float v_g8 = fmaf(65536.f, acc[2], fmaf(256.f, acc[3], lo_g8));

        // cross-warp reduction without a barrier (as in the bf16 path): each
        // warp stores its row sums in the slot of this tile's parity, the
        // last of the group's warps sums them, writes y and frees the slot
        const uint32_t slot = ti & 1u;
        if (ti >= 2 && lane == 0) {
            volatile int* done = &S.red_done[group][slot];
            const uint64_t t0 = sm100::globaltimer();
            while (*done != (int)ti - 2) {
                if (sm100::globaltimer() - t0 > KC_WAIT_TIMEOUT_NS) {
                    sm100::record_status(KC_ERR_TIMEOUT);
                    break;
                }
            }
        }
        __syncwarp();
        float* red = S.red[group][slot][gw];
        if (t == 0) {
            red[g] = v_g;
            red[g + 8] = v_g8;
        }
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&S.red_cnt[group][slot], 1) == kGroupWarps - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane == 0 && tile + kScaleBufs * stride < total) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_scales(P, tile + kScaleBufs * stride, S.scales[group][sb], &S.sfull[group][sb]);
            }
            if (lane < 16) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kGroupWarps; ++w) v += S.red[group][slot][w][lane];
                if (row0 + lane < N) pr.y[row0 + lane] = v * S.row_f[pi];
            }
            __syncwarp();
            if (lane == 0) {
                S.red_cnt[group][slot] = 0;
                __threadfence_block();
                *reinterpret_cast<volatile int*>(&S.red_done[group][slot]) = (int)ti;
            }
        }
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
            const int z = pr.zeros ? (int)(pr.zeros[(size_t)r * sc + c / P.gs] & 15) : 8;
            const float w = (float)(u - z) * __half2float(pr.scales[(size_t)r * sc + c / P.gs]);
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
int launch_tc(const Params& P, size_t stage_bytes, cudaStream_t stream) {
    const size_t smem = fixed_smem<NT>() + stage_bytes;
    auto kern = gemv_w4a16_kernel<NT, XS>;
    KC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "gemv_w4a16 shared-memory attribute");
    const int groups = (P.total_tiles + Shape<NT>::groups - 1) / Shape<NT>::groups;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)std::min(groups, kc::sm_count()));
    cfg.blockDim = dim3(Shape<NT>::threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    // programmatic dependent launch: this grid may be scheduled while the
    // previous one drains; the kernel waits (griddepcontrol.wait) before it
    // reads the activations or writes y (packed weights and scales are read
    // before the wait: they must not be written by the grid just before)
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, P), "gemv_w4a16 launch");
    return KC_OK;
}

// Shared memory left for the staged activations and their chunk sums.
constexpr size_t kSmemLimit = 227 * 1024;

template <bool ZP>
int launch_i8(const Params& P, size_t stage_bytes, cudaStream_t stream) {
    const size_t smem = fixed_smem_i8() + stage_bytes;
    KC_CUDA_TRY(cudaFuncSetAttribute(gemv_w4a16_i8_kernel<ZP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem),
                "gemv_w4a16_i8 shared-memory attribute");
    const int groups = (P.total_tiles + Shape<1>::groups - 1) / Shape<1>::groups;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)std::min(groups, kc::sm_count()));
    cfg.blockDim = dim3(Shape<1>::threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    KC_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_w4a16_i8_kernel<ZP>, P), "gemv_w4a16_i8 launch");
    return KC_OK;
}

int launch(Params& P, cudaStream_t stream) {
    if (P.total_tiles == 0) return KC_OK;
    bool fast = true, single_group = true, any_zeros = false;
    for (int i = 0; i < P.count; ++i) any_zeros = any_zeros || P.p[i].zeros != nullptr;
    for (int i = 0; i < P.count && fast; ++i) {
        const Prob& p = P.p[i];
        // TMA: 16-byte aligned base and row pitch; scale blocks: a tile's 16 rows
        // of K/gs halves must fit a slot, start 16-byte aligned, and a partial
        // last tile's block must stay a multiple of 16 bytes.
        const long row_bytes = 2L * (p.K / P.gs);
        const int tail = p.N % 16;
        fast = (p.K % 128 == 0) && kc::aligned(p.tiled ? p.tiled : p.packed, 16) && kc::aligned(p.x, 16) &&
               kc::aligned(p.scales, 16) && 16 * row_bytes <= 2L * kScaleHalves &&
               (16 * row_bytes) % 16 == 0 && (tail == 0 || (tail * row_bytes) % 16 == 0);
        single_group = single_group && (p.K == P.gs);
    }
    int gshift = -1;
    for (int m = 0; m < 20; ++m)
        if (P.gs == (128 << m)) gshift = m;
    if (single_group) gshift = 31;
    P.gshift = gshift;
    P.magic = 0x43004300u;
    P.neg136 = 0xC308C308u;
    // zero points: the batch-1 integer path (below) takes them; the bf16
    // paths do not, so other batch sizes run on the CUDA-core kernel
    if (!fast || gshift < 0 || (any_zeros && P.M != 1)) {
        for (int i = 0; i < P.count; ++i)
            KC_REQUIRE(P.p[i].packed != nullptr, KC_ERR_INVALID_ARG,
                       "tile-ordered weights run on the tensor-core paths only (K %% 128 == 0, "
                       "group size 128 x 2^m, 16-byte aligned, zero points only at batch 1)");
        long rows = 0;
        for (int i = 0; i < P.count; ++i) rows += P.p[i].N;
        const long blocks = (rows + 7) / 8;
        const long cap = (long)kc::sm_count() * 8;
        gemv_w4a16_scalar<<<(int)std::max(1L, std::min(blocks, cap)), 256, 0, stream>>>(P);
        return kc::check_launch("gemv_w4a16_scalar");
    }
    for (int i = 0; i < P.count; ++i) {
        const Prob& p = P.p[i];
        if (p.tiled) continue;   // bulk copies, no tensor map
        const int st = kc::encode_2d(&P.wmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, p.packed,
                                     (uint64_t)(p.K / 2), (uint64_t)p.N, (uint64_t)(p.K / 2), 64, 16,
                                     CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st != KC_OK) return st;
    }
    // stage every problem's activations when they all fit.  (Staging the chunk
    // offsets alone when the activations do not fit was slower than the offset
    // MMA: every CTA then reads all activations before its first tile.)
    const int NT = P.M <= 8 ? 1 : 2;
    long xs_bytes = 0, chunks = 0;  // padded footprint, chunk rows
    for (int i = 0; i < P.count; ++i) {
        Prob& q = P.p[i];
        q.xs_off = (int)xs_bytes;
        q.sx_off = (int)chunks;
        xs_bytes += (long)P.M * (2L * q.K + 16);
        chunks += q.K / 128;
    }
    // batch 1: the integer tensor-core path when its staged byte planes fit
    if (P.M == 1 && chunks <= kI8MaxChunks &&
        fixed_smem_i8() + (size_t)chunks * kI8ChunkBytes <= kSmemLimit) {
        P.sx_chunks = (int)chunks;
        return any_zeros ? launch_i8<true>(P, (size_t)chunks * kI8ChunkBytes, stream)
                         : launch_i8<false>(P, (size_t)chunks * kI8ChunkBytes, stream);
    }
    if (any_zeros) {   // batch 1 whose activations do not fit the staging: CUDA cores
        for (int i = 0; i < P.count; ++i)
            KC_REQUIRE(P.p[i].packed != nullptr, KC_ERR_INVALID_ARG,
                       "tile-ordered weights with zero points need the batch-1 staged path");
        long rows = 0;
        for (int i = 0; i < P.count; ++i) rows += P.p[i].N;
        const long blocks = (rows + 7) / 8;
        const long cap = (long)kc::sm_count() * 8;
        gemv_w4a16_scalar<<<(int)std::max(1L, std::min(blocks, cap)), 256, 0, stream>>>(P);
        return kc::check_launch("gemv_w4a16_scalar");
    }
    const size_t fixed = NT == 1 ? fixed_smem<1>() : fixed_smem<2>();
    const size_t sx_bytes = (size_t)chunks * NT * 8 * 4;
    const bool stage = fixed + sx_bytes + (size_t)xs_bytes <= kSmemLimit;
    P.sx_chunks = stage ? (int)chunks : 0;
    const size_t stage_bytes = stage ? sx_bytes + (size_t)xs_bytes : 0;
    if (NT == 1)
        return stage ? launch_tc<1, true>(P, stage_bytes, stream) : launch_tc<1, false>(P, 0, stream);
    return stage ? launch_tc<2, true>(P, stage_bytes, stream) : launch_tc<2, false>(P, 0, stream);
}

// packed [N, K/2] -> tile order [ceil(N/16)][K/128][16][64 B], rows past N zero;
// one 16-byte piece per thread and step
__global__ void tile_weights_kernel(const uint8_t* __restrict__ packed, uint8_t* __restrict__ tiled, int N,
                                    int K, long pieces) {
    const int chunks = K / 128;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < pieces; i += (long)gridDim.x * blockDim.x) {
        const int b16 = (int)(i & 3), r = (int)((i >> 2) & 15);
        const long tc = i >> 6;                       // tile * chunks + chunk
        const int c = (int)(tc % chunks);
        const long t = tc / chunks;
        const long row = t * 16 + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row < N) v = *reinterpret_cast<const uint4*>(packed + row * (K / 2) + (long)c * 64 + b16 * 16);
        *reinterpret_cast<uint4*>(tiled + i * 16) = v;
    }
}

}  // namespace

KC_DEFINE_STATUS_READER(gemv)

extern "C" {

namespace {
int gemv_grouped(const kc_w4a16_problem* problems, const uint8_t* const* zeros, int count, int M,
                 int gs, cudaStream_t stream, const uint8_t* const* tiled = nullptr) {
    KC_REQUIRE(problems != nullptr, KC_ERR_INVALID_ARG, "null problem list");
    KC_REQUIRE(count >= 1 && count <= KC_W4A16_MAX_PROBLEMS, KC_ERR_INVALID_ARG,
               "count=%d outside 1..%d", count, KC_W4A16_MAX_PROBLEMS);
    KC_REQUIRE(M >= 1 && M <= 16, KC_ERR_INVALID_ARG, "M=%d outside 1..16", M);
    KC_REQUIRE(gs > 0 && gs % 2 == 0, KC_ERR_INVALID_ARG, "group_size=%d must be even and > 0", gs);
    Params P{};
    P.count = count;
    P.M = M;
    P.gs = gs;
    // longest rows first: the tiles of the largest K are handed out in the
    // first rounds, so the last round of the persistent grid is short
    int order[KC_W4A16_MAX_PROBLEMS];
    for (int i = 0; i < count; ++i) order[i] = i;
    std::stable_sort(order, order + count,
                     [&](int a, int b) { return problems[a].K > problems[b].K; });
    long tiles = 0;
    for (int i = 0; i < count; ++i) {
        const kc_w4a16_problem& q = problems[order[i]];
        KC_REQUIRE((q.packed || (tiled && tiled[order[i]])) && q.scales_f16 && q.x_bf16 && q.y,
                   KC_ERR_INVALID_ARG, "problem %d has a null pointer", order[i]);
        KC_REQUIRE(q.N >= 0 && q.K > 0 && q.K % 2 == 0 && q.K % gs == 0, KC_ERR_INVALID_ARG,
                   "problem %d: bad shape N=%d K=%d for group_size=%d", order[i], q.N, q.K, gs);
        P.p[i].packed = q.packed;
        P.p[i].tiled = tiled ? tiled[order[i]] : nullptr;
        P.p[i].scales = reinterpret_cast<const __half*>(q.scales_f16);
        P.p[i].zeros = zeros ? zeros[order[i]] : nullptr;
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
}  // namespace

int kc_gemv_w4a16_grouped(const kc_w4a16_problem* problems, int count, int M, int gs,
                          cudaStream_t stream) {
    return gemv_grouped(problems, nullptr, count, M, gs, stream);
}

int kc_gemv_w4a16_grouped_zp(const kc_w4a16_problem* problems, const uint8_t* const* zeros,
                             int count, int M, int gs, cudaStream_t stream) {
    KC_REQUIRE(zeros != nullptr, KC_ERR_INVALID_ARG, "null zero-point list");
    return gemv_grouped(problems, zeros, count, M, gs, stream);
}

int kc_gemv_w4a16_grouped_tiled(const kc_w4a16_problem* problems, const uint8_t* const* tiled,
                                const uint8_t* const* zeros, int count, int M, int gs,
                                cudaStream_t stream) {
    KC_REQUIRE(tiled != nullptr, KC_ERR_INVALID_ARG, "null tile-ordered weight list");
    for (int i = 0; i < count && i < KC_W4A16_MAX_PROBLEMS; ++i)
        KC_REQUIRE(tiled[i] != nullptr, KC_ERR_INVALID_ARG, "problem %d: null tile-ordered weights", i);
    return gemv_grouped(problems, zeros, count, M, gs, stream, tiled);
}

int kc_w4a16_tile_weights(const uint8_t* packed, uint8_t* tiled, int N, int K, cudaStream_t stream) {
    KC_REQUIRE(packed && tiled, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(N >= 0 && K > 0 && K % 128 == 0, KC_ERR_INVALID_ARG,
               "N=%d, K=%d: K must be a positive multiple of 128", N, K);
    KC_REQUIRE(kc::aligned(packed, 16) && kc::aligned(tiled, 16), KC_ERR_ALIGNMENT,
               "buffers must be 16-byte aligned");
    if (N == 0) return KC_OK;
    const long pieces = (long)((N + 15) / 16) * (K / 128) * 64;   // 16-byte pieces
    tile_weights_kernel<<<(unsigned)std::min<long>((pieces + 255) / 256, (long)kc::sm_count() * 16), 256, 0,
                          stream>>>(packed, tiled, N, K, pieces);
    return kc::check_launch("w4a16_tile_weights");
}

int kc_gemv_w4a16(const uint8_t* packed, const uint16_t* scales_f16, const uint16_t* x_bf16,
                  float* y, int M, int N, int K, int gs, cudaStream_t stream) {
    kc_w4a16_problem p{packed, scales_f16, x_bf16, y, N, K};
    return gemv_grouped(&p, nullptr, 1, M, gs, stream);
}

int kc_gemv_w4a16_zp(const uint8_t* packed, const uint16_t* scales_f16, const uint8_t* zeros,
                     const uint16_t* x_bf16, float* y, int M, int N, int K, int gs,
                     cudaStream_t stream) {
    KC_REQUIRE(zeros != nullptr, KC_ERR_INVALID_ARG, "null zero points");
    kc_w4a16_problem p{packed, scales_f16, x_bf16, y, N, K};
    return gemv_grouped(&p, &zeros, 1, M, gs, stream);
}

}  // extern "C"
