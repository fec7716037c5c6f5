// tp.cu -- fp32 shard GEMM for column/row-parallel linear layers and the
// single-GPU simulated collectives (src/kernels/transformer/tensor_parallel.cu).
#include "kc_common.cuh"

namespace {

// C[M,N] = A[M,K] * B[N,K]^T in fp32.  64x64 CTA tile, 16-deep k slab,
// 256 threads with a 4x4 register tile each; every load is bounds-checked so
// any shape and alignment is accepted.  Accumulation is in k order per output,
// as in the reference's sgemm_nt_kernel (tensor_parallel.cu:177-190).
constexpr int BM = 64, BN = 64, BK = 16;

__global__ void __launch_bounds__(256) sgemm_nt_kernel(const float* __restrict__ A,
                                                       const float* __restrict__ B,
                                                       float* __restrict__ C, int M, int N, int K) {
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;  // 16x16 threads, 4x4 outputs each
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
        // 64x16 tile of A and of B: 1024 elements, 4 per thread; (row, k) with k fastest.
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = tid + i * 256;
            const int r = e >> 4, kk = e & 15;
            const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
            As[kk][r] = (gm < M && gk < K) ? A[(size_t)gm * K + gk] : 0.f;
            Bs[kk][r] = (gn < N && gk < K) ? B[(size_t)gn * K + gk] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx * 4 + j;
            if (gn < N) C[(size_t)gm * N + gn] = acc[i][j];
        }
    }
}

constexpr int kMaxSimRanks = 64;
struct RankPtrs {
    float* p[kMaxSimRanks];
};

// One pass over all ranks: element i of chunk c = i / chunk is summed in the
// reference's order (rank c's own value, then every other rank in index order,
// tensor_parallel.cu:108-121) and written back to every rank (:126-140).
__global__ void sim_allreduce_kernel(const __grid_constant__ RankPtrs b, int R, int count,
                                     int chunk) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const int c = i / chunk;
        float acc = b.p[c][i];
        for (int r = 0; r < R; ++r)
            if (r != c) acc += b.p[r][i];
        for (int r = 0; r < R; ++r) b.p[r][i] = acc;
    }
}

__global__ void sim_allgather_kernel(const __grid_constant__ RankPtrs b, float* __restrict__ out,
                                     int R, int chunk) {
    const long n = (long)R * chunk;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / chunk);
        out[i] = b.p[r][i - (long)r * chunk];
    }
}

int grid_1d(long items, int threads) {
    long g = (items + threads - 1) / threads;
    const long cap = (long)kc::sm_count() * 8;
    if (g > cap) g = cap;
    return g < 1 ? 1 : (int)g;
}

}  // namespace

extern "C" {

int kc_sgemm_nt(const float* A, const float* B, float* C, int M, int N, int K,
                cudaStream_t stream) {
    KC_REQUIRE(A && B && C, KC_ERR_INVALID_ARG, "null pointer argument");
    KC_REQUIRE(M >= 0 && N >= 0 && K >= 0, KC_ERR_INVALID_ARG, "negative size");
    if (M == 0 || N == 0) return KC_OK;
    KC_REQUIRE((M + BM - 1) / BM <= 65535, KC_ERR_INVALID_ARG, "M=%d too large", M);
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    sgemm_nt_kernel<<<grid, 256, 0, stream>>>(A, B, C, M, N, K);
    return kc::check_launch("sgemm_nt");
}

void launch_col_parallel_linear(const float* d_x, const float* d_W, float* d_y, int M, int N_rank,
                                int K, cudaStream_t stream) {
    kc_sgemm_nt(d_x, d_W, d_y, M, N_rank, K, stream);
}

void launch_row_parallel_linear(const float* d_x_rank, const float* d_W, float* d_out, int M,
                                int N, int K_rank, cudaStream_t stream) {
    kc_sgemm_nt(d_x_rank, d_W, d_out, M, N, K_rank, stream);
}

void launch_ring_allreduce(float** d_bufs, int count, int num_ranks, cudaStream_t stream) {
    if (num_ranks <= 1) return;  // tensor_parallel.cu:99
    if (!d_bufs || count < 0 || num_ranks > kMaxSimRanks) {
        kc::set_error(KC_ERR_INVALID_ARG, "launch_ring_allreduce: bad arguments (ranks=%d, max %d)",
                      num_ranks, kMaxSimRanks);
        return;
    }
    RankPtrs b{};
    for (int r = 0; r < num_ranks; ++r) {
        if (!d_bufs[r]) {
            kc::set_error(KC_ERR_INVALID_ARG, "launch_ring_allreduce: null buffer for rank %d", r);
            return;
        }
        b.p[r] = d_bufs[r];
    }
    if (count > 0) {
        const int chunk = (count + num_ranks - 1) / num_ranks;
        sim_allreduce_kernel<<<grid_1d(count, 256), 256, 0, stream>>>(b, num_ranks, count, chunk);
        if (kc::check_launch("launch_ring_allreduce") != KC_OK) return;
    }
    kc::check_cuda(cudaStreamSynchronize(stream), "launch_ring_allreduce sync");
}

void launch_allgather(float** d_chunks, float* d_output, int chunk_size, int num_ranks,
                      cudaStream_t stream) {
    if (!d_chunks || !d_output || chunk_size < 0 || num_ranks < 0 || num_ranks > kMaxSimRanks) {
        kc::set_error(KC_ERR_INVALID_ARG, "launch_allgather: bad arguments (ranks=%d, max %d)",
                      num_ranks, kMaxSimRanks);
        return;
    }
    RankPtrs b{};
    for (int r = 0; r < num_ranks; ++r) b.p[r] = d_chunks[r];
    if (chunk_size > 0 && num_ranks > 0) {
        sim_allgather_kernel<<<grid_1d((long)chunk_size * num_ranks, 256), 256, 0, stream>>>(
            b, d_output, num_ranks, chunk_size);
        if (kc::check_launch("launch_allgather") != KC_OK) return;
    }
    kc::check_cuda(cudaStreamSynchronize(stream), "launch_allgather sync");
}

}  // extern "C"
