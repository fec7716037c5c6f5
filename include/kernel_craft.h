/*
 * kernel_craft.h -- C ABI of the B200 (sm_100a) quantized-linear library.
 *
 * Part 1 re-declares, signature for signature, the extern "C" launchers that
 * kernel-craft's libkernels.so exports for this path; each cites the
 * reference definition it replaces (path within the kernel-craft project).
 * Their semantics are kept: void return, raw device pointers, the stream last,
 * and a cudaStreamSynchronize before returning where the reference had one.
 * Invalid arguments (which the reference never checked) launch nothing and are
 * reported through kc_get_last_error().
 *
 * Part 2 is the new kc_* API: int status (KC_OK == 0), never synchronizes
 * unless stated, never allocates device memory (kc_ipc_alloc, whose purpose
 * is to allocate a shareable buffer, excepted).  It carries the bf16 / fp16 /
 * FP8 entry points the reference does not have (batched W4A16 GEMV, tcgen05
 * GEMMs, bf16 collectives, sharded drivers).
 *
 * All pointers are device pointers unless stated; the caller owns every
 * buffer.  Layouts are row-major.
 */
#ifndef KERNEL_CRAFT_H
#define KERNEL_CRAFT_H

#include <stdint.h>
#include <stdbool.h>
#include <stddef.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define KC_API __attribute__((visibility("default")))
#else
#define KC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ======================================================================= */
/* Status codes                                                             */
/* ======================================================================= */
#define KC_OK               0
#define KC_ERR_INVALID_ARG  1   /* a size, pointer or flag the kernel cannot take */
#define KC_ERR_ALIGNMENT    2   /* a pointer/stride violates a documented alignment */
#define KC_ERR_CUDA         3   /* a CUDA runtime call or launch failed */
#define KC_ERR_NCCL         4   /* an NCCL call failed */
#define KC_ERR_UNSUPPORTED  5   /* entry point outside this library's scope */
#define KC_ERR_TIMEOUT      6   /* a bounded device-side wait gave up */

/* Last status recorded on the calling thread by any entry point (0 = none);
 * reading it clears it. */
KC_API int kc_get_last_error(void);
/* Human-readable detail for the last recorded status on this thread. */
KC_API const char* kc_get_last_error_string(void);
/* Library version string. */
KC_API const char* kc_version(void);
/* Synchronizes the current device, then reads and clears the status words the
 * pipelined kernels set when a bounded device-side wait gives up
 * (KC_ERR_TIMEOUT); KC_OK when none did. */
KC_API int kc_get_device_status(void);
/* Test hook: one CTA waits on an mbarrier phase nothing completes; the wait
 * gives up after timeout_ns (<= 5 s), records KC_ERR_TIMEOUT for
 * kc_get_device_status() and writes the milliseconds waited to
 * *waited_ms_device (device int).  The context stays usable. */
KC_API int kc_selftest_bounded_wait(uint64_t timeout_ns, int* waited_ms_device, cudaStream_t stream);
/* Measurement hook: one pass of 16-byte streaming loads over `bytes` bytes at
 * `src` (16-byte aligned, bytes a multiple of 16) with the launch shape of the
 * reference-ABI GEMV (256-thread CTAs, four loads in flight per thread), the
 * floor that GEMV is measured against.  Nothing is written unless the XOR of
 * all words equals `sentinel`, in which case one word goes to *sink_device.
 * bytes == 0 launches one empty CTA (the launch floor). */
KC_API int kc_selftest_stream_read(const void* src, size_t bytes, uint32_t sentinel,
                                   uint32_t* sink_device, cudaStream_t stream);

/* ======================================================================= */
/* Part 1: reference launcher ABI (drop-in)                                 */
/* ======================================================================= */

/* src/kernels/transformer/quant_int4.cu:193.  out[r,c] = (float)(sx4(nib) - zp) * scale;
 * packed u8[rows, cols/2] (low nibble = even col), scales f32[rows, cols/gs],
 * zeros u8 packed two per byte, row stride floor(cols/gs/2).  Synchronizes.
 * Requires cols even, group_size > 0 and cols % group_size == 0. */
KC_API void launch_dequantize_int4(const uint8_t* d_packed, const float* d_scales,
                            const uint8_t* d_zeros, float* d_output,
                            int rows, int cols, int group_size, cudaStream_t stream);

/* src/kernels/transformer/quant_int4.cu:221.  y[r] = sum_c w(r,c) * x[c] (fp32). Synchronizes. */
KC_API void launch_gemv_int4(const uint8_t* d_packed, const float* d_scales,
                      const uint8_t* d_zeros, const float* d_x, float* d_y,
                      int rows, int cols, int group_size, cudaStream_t stream);

/* src/kernels/transformer/fp8_quant.cu:201.  per_token: scales[r] = amax_r/448 (1 if 0),
 * q = e4m3_satfinite(clamp(x/scale, +-448)).  Otherwise the caller's d_scales[0] is the
 * per-tensor scale (read on the device; no host round trip).  Synchronizes. */
KC_API void launch_quantize_fp8(const float* d_input, int8_t* d_output, float* d_scales,
                         int rows, int cols, bool per_token, cudaStream_t stream);

/* src/kernels/transformer/fp8_quant.cu:239.  x = float(e4m3) * scale[row or 0]. Synchronizes. */
KC_API void launch_dequantize_fp8(const int8_t* d_input, const float* d_scales, float* d_output,
                           int rows, int cols, bool per_token, cudaStream_t stream);

/* src/kernels/transformer/fp8_quant.cu:265.  out[r,c] = in[r,c] / smooth[c]. Synchronizes. */
KC_API void launch_smoothquant_scale(const float* d_input, const float* d_smooth_scales,
                              float* d_output, int rows, int cols, cudaStream_t stream);

/* src/kernels/transformer/tensor_parallel.cu:209.  y[M,N_rank] = x[M,K] * W[N_rank,K]^T (fp32). Async. */
KC_API void launch_col_parallel_linear(const float* d_x, const float* d_W, float* d_y,
                                int M, int N_rank, int K, cudaStream_t stream);

/* src/kernels/transformer/tensor_parallel.cu:235.  out[M,N] = x_r[M,K_rank] * W[N,K_rank]^T (fp32). Async. */
KC_API void launch_row_parallel_linear(const float* d_x_rank, const float* d_W, float* d_out,
                                int M, int N, int K_rank, cudaStream_t stream);

/* src/kernels/transformer/tensor_parallel.cu:93.  Single-GPU simulation: d_bufs is a HOST
 * array of num_ranks device pointers; every buffer ends holding the sum (chunk c summed in
 * rank order into rank c, then broadcast).  Synchronizes (returns at once if num_ranks <= 1). */
KC_API void launch_ring_allreduce(float** d_bufs, int count, int num_ranks, cudaStream_t stream);

/* src/kernels/transformer/tensor_parallel.cu:258.  out = [chunk_0 | ... | chunk_{R-1}]. Synchronizes. */
KC_API void launch_allgather(float** d_chunks, float* d_output, int chunk_size, int num_ranks,
                      cudaStream_t stream);

/* src/kernels/transformer/tensor_parallel_nccl.cu:58.  ncclCommInitAll over devs. */
KC_API void nccl_comm_init_all(void** comms, int num_comms, const int* devs);
/* src/kernels/transformer/tensor_parallel_nccl.cu:69. */
KC_API void nccl_comm_destroy(void* comm);
/* src/kernels/transformer/tensor_parallel_nccl.cu:77. */
KC_API void nccl_group_start(void);
/* src/kernels/transformer/tensor_parallel_nccl.cu:85. */
KC_API void nccl_group_end(void);
/* src/kernels/transformer/tensor_parallel_nccl.cu:105.  In-place fp32 sum all-reduce. Async. */
KC_API void launch_ring_allreduce_nccl(void* comm, float* d_buf, int count, cudaStream_t stream);
/* src/kernels/transformer/tensor_parallel_nccl.cu:127.  fp32 all-gather, rank-major. Async. */
KC_API void launch_allgather_nccl(void* comm, const float* d_sendbuf, float* d_recvbuf,
                           int sendcount, cudaStream_t stream);
/* src/kernels/transformer/tensor_parallel_nccl.cu:147.  Ranks in comm, 0 on error. */
KC_API int nccl_comm_count(void* comm);
/* src/kernels/transformer/tensor_parallel_nccl.cu:160.  Rank of comm, -1 on error. */
KC_API int nccl_comm_user_rank(void* comm);

/* Out-of-scope launchers that src/python/kernel_craft_torch_ops.py:105-168 resolves
 * when it loads the library.  Exported so the unmodified bridge loads; each records
 * KC_ERR_UNSUPPORTED and launches nothing (attention and speculative decoding are not
 * part of this library). */
KC_API void launch_flash_attention(const float* Q, const float* K, const float* V, float* O,
                            int B, int H, int H_kv, int N, int d, bool causal,
                            cudaStream_t stream);
KC_API void launch_paged_attention(const float* Q, const int* block_table, const float* K_pool,
                            const float* V_pool, float* O, const int* seq_lens,
                            int B, int H, int H_kv, int d, int block_size, int max_blocks,
                            cudaStream_t stream);
KC_API void launch_verify_draft_tokens(const float* d_draft_probs, const float* d_target_probs,
                                const int* d_draft_tokens, const float* d_rand_vals,
                                const float* d_rand_vals2, int* d_accepted, int* d_corrected,
                                int num_tokens, int vocab_size, cudaStream_t stream);

/* Further out-of-scope launchers that the reference's pybind11 module links
 * (src/python/pybind_transformer.cpp:75,95,102,107); exported so the
 * unmodified module loads against this library and its quantization and
 * tensor-parallel functions work.  Each records KC_ERR_UNSUPPORTED and
 * launches nothing. */
KC_API void launch_compute_prefix_length(const int* d_accepted, int* d_prefix_len, int num_tokens,
                                         cudaStream_t stream);
KC_API void launch_selective_scan(const float* d_u, const float* d_A_log, const float* d_B,
                                  const float* d_C, const float* d_delta, float* d_y,
                                  int B_, int L, int D, int N_state, cudaStream_t stream);
KC_API void launch_depthwise_conv1d(const float* d_x, const float* d_w, const float* d_bias,
                                    float* d_y, int B_, int D, int L, int d_conv,
                                    cudaStream_t stream);
KC_API void launch_rmsnorm(const float* d_x, const float* d_g, float* d_y, int rows, int D,
                           float eps, cudaStream_t stream);

/* ======================================================================= */
/* Part 2: kc_* API                                                          */
/* ======================================================================= */

/* Non-synchronizing twin of launch_dequantize_int4 (quant_int4.cu:193). */
KC_API int kc_dequantize_int4_f32(const uint8_t* packed, const float* scales, const uint8_t* zeros,
                           float* out, int rows, int cols, int group_size, cudaStream_t stream);

/* Non-synchronizing twin of launch_gemv_int4 (quant_int4.cu:221). */
KC_API int kc_gemv_int4_f32(const uint8_t* packed, const float* scales, const uint8_t* zeros,
                     const float* x, float* y, int rows, int cols, int group_size,
                     cudaStream_t stream);

/* GPTQ-style W4 (implicit zero-point 8, no zeros buffer):
 * w[n,k] = (u - 8) * float(scales_f16[n, k/gs]), u the unsigned nibble
 * (low nibble = even k).  Equals the reference dequant of (packed ^ 0x88) with
 * zero points 0 (quant_int4.cu:99-104).  out bf16[N,K] = RNE(w). */
KC_API int kc_dequantize_w4_bf16(const uint8_t* packed, const uint16_t* scales_f16, uint16_t* out_bf16,
                          int N, int K, int group_size, cudaStream_t stream);

/* kc_dequantize_w4_bf16 with per-group zero points: out = bf16((u - z) * s),
 * zeros u8[N, K/gs] (0..15); no reference counterpart (see kc_gemv_w4a16_zp). */
KC_API int kc_dequantize_w4_bf16_zp(const uint8_t* packed, const uint16_t* scales_f16,
                                    const uint8_t* zeros, uint16_t* out_bf16, int N, int K,
                                    int group_size, cudaStream_t stream);

/* W4A16 GEMV / skinny GEMM: y[m,n] = sum_k w[n,k] * x[m,k] for m < M <= 16;
 * x bf16[M,K], y f32[M,N], fp32 accumulation.  Fast path: group_size % 128 == 0,
 * K % 128 == 0, packed/x 16-byte aligned; other shapes take a CUDA-core path. */
KC_API int kc_gemv_w4a16(const uint8_t* packed, const uint16_t* scales_f16, const uint16_t* x_bf16,
                  float* y, int M, int N, int K, int group_size, cudaStream_t stream);

/* One problem of a grouped W4A16 GEMV launch. */
typedef struct kc_w4a16_problem {
    const uint8_t*  packed;      /* u8[N, K/2]          */
    const uint16_t* scales_f16;  /* f16[N, K/group]     */
    const uint16_t* x_bf16;      /* bf16[M, K]          */
    float*          y;           /* f32[M, N]           */
    int N, K;
} kc_w4a16_problem;

/* All problems share M and group_size; one kernel launch covers them all
 * (e.g. the QKV, O, gate+up and down projections of a decoder layer).
 * count <= KC_W4A16_MAX_PROBLEMS. */
#define KC_W4A16_MAX_PROBLEMS 8
KC_API int kc_gemv_w4a16_grouped(const kc_w4a16_problem* problems, int count, int M,
                          int group_size, cudaStream_t stream);

/* W4 with per-group zero points (AWQ and asymmetric GPTQ checkpoints):
 * w[n,k] = (u - z[n, k/gs]) * float(scales_f16[n, k/gs]) with zeros u8[N, K/gs],
 * one zero point (0..15) per row and group, unpacked.  z = 8 everywhere is
 * the symmetric case above; the reference's dequantize_int4 represents only
 * z >= 8 (its weight nibbles are signed, quant_int4.cu:34-38, and its zero
 * points unsigned, :93-96), so these entry points have no reference twin.
 * Batch 1 runs on the integer tensor-core path like the symmetric GEMV;
 * M > 1 on the CUDA-core path.  Same shape rules as kc_gemv_w4a16. */
KC_API int kc_gemv_w4a16_zp(const uint8_t* packed, const uint16_t* scales_f16, const uint8_t* zeros,
                            const uint16_t* x_bf16, float* y, int M, int N, int K, int group_size,
                            cudaStream_t stream);
/* Grouped form: zeros[i] belongs to problems[i] (NULL: that problem is symmetric). */
KC_API int kc_gemv_w4a16_grouped_zp(const kc_w4a16_problem* problems, const uint8_t* const* zeros,
                                    int count, int M, int group_size, cudaStream_t stream);

/* Tile-ordered weights (no reference counterpart): the same packed bytes
 * rearranged so that every 16-row x 128-k chunk (1 KB) is contiguous,
 * tiled[ceil(N/16)][K/128][16 rows][64 bytes], rows past N zero.  The GEMV
 * then fetches a stage of up to four chunks with one bulk copy.
 * kc_w4a16_tile_weights converts packed u8[N, K/2] (K % 128 == 0, 16-byte
 * aligned) into a buffer of ceil(N/16) * 16 * K/2 bytes, once at load time. */
KC_API int kc_w4a16_tile_weights(const uint8_t* packed, uint8_t* tiled, int N, int K, cudaStream_t stream);
/* The grouped GEMV (and its zero-point form, zeros may be NULL) reading
 * tiled[i] instead of problems[i].packed, which may then be NULL.  Results are
 * bit-identical to kc_gemv_w4a16_grouped[_zp].  Only the tensor-core paths
 * read the tiled form: K % 128 == 0, group_size = 128 * 2^m, 16-byte aligned
 * buffers, zero points at batch 1 only; other shapes are refused. */
KC_API int kc_gemv_w4a16_grouped_tiled(const kc_w4a16_problem* problems, const uint8_t* const* tiled,
                                       const uint8_t* const* zeros, int count, int M, int group_size,
                                       cudaStream_t stream);

/* FP8 E4M3 per-token quantization (fp8_quant.cu:89-131 semantics, bit-exact):
 * scales[r] = amax_r > 0 ? amax_r/448 : 1; q = e4m3_satfinite(clamp(x/scale)). */
KC_API int kc_quantize_fp8_per_token(const float* in, int8_t* out, float* scales,
                              int rows, int cols, cudaStream_t stream);
/* Per-output-channel weight quantization: the same arithmetic on W[N,K] rows. */
KC_API int kc_quantize_fp8_per_channel(const float* w, int8_t* out, float* scales,
                                int N, int K, cudaStream_t stream);
/* Per-tensor quantization with the scale read from d_scale[0] on the device. */
KC_API int kc_quantize_fp8_per_tensor(const float* in, int8_t* out, const float* d_scale,
                               long count, cudaStream_t stream);
/* Per-tensor quantization with the scale computed on the device:
 * scale = amax(|x|) / 448 over the whole tensor (1 if amax == 0), written to
 * scale_out[0]; the same value the reference's pybind path computes on the host
 * (src/python/pybind_transformer.cpp:305-311).  workspace: >= 4 bytes of device
 * memory, 4-byte aligned (cleared and used for the cross-CTA amax). */
KC_API int kc_quantize_fp8_per_tensor_dynamic(const float* in, int8_t* out, float* scale_out,
                                              long count, void* workspace, size_t workspace_bytes,
                                              cudaStream_t stream);
/* The same quantization (identical codes and scale) for callers that may not
 * allocate device memory at all -- code running under a caller-owned memory
 * budget, an allocator-free serving loop, or a host binding with no device
 * allocator to hand a workspace from.  No counterpart in the reference; it
 * allocates nothing: its 256 KiB of scratch is a static array inside the
 * library's own device image.  Limits and rules:
 *  - count <= 2^30 elements; larger counts return KC_ERR_INVALID_ARG (use the
 *    workspace variant above);
 *  - the first call on each device (with that device current) looks up the
 *    scratch address with cudaGetSymbolAddress; make that first call before
 *    capturing any stream.  The address is cached per device and context, so
 *    the first call after a cudaDeviceReset, or under another context of the
 *    same device, looks it up again (and so must precede a capture too);
 *  - one arrival counter in the scratch must read zero when a call starts: it
 *    is zero when the library loads and every completed call leaves it at zero;
 *  - every thread and stream of one process that uses a device shares that
 *    device's scratch, so calls that overlap on the GPU race; serialize them.
 *    Another process loads its own copy of the library's device image and
 *    does not share it. */
KC_API int kc_quantize_fp8_per_tensor_dynamic_noalloc(const float* in, int8_t* out,
                                                      float* scale_out, long count,
                                                      cudaStream_t stream);
/* SmoothQuant divide fused into per-token quantization: bit-identical to
 * launch_smoothquant_scale followed by launch_quantize_fp8(per_token=true),
 * without the fp32 round trip through HBM. */
KC_API int kc_smoothquant_quantize_fp8(const float* in, const float* smooth, int8_t* out,
                                float* scales, int rows, int cols, cudaStream_t stream);
/* Non-synchronizing twins of the reference's dequant / smoothquant launchers. */
KC_API int kc_dequantize_fp8(const int8_t* in, const float* scales, float* out, int rows, int cols,
                      bool per_token, cudaStream_t stream);
KC_API int kc_smoothquant_scale(const float* in, const float* smooth, float* out, int rows, int cols,
                         cudaStream_t stream);

/* FP8 E4M3 W8A8 GEMM on the tcgen05 tensor cores:
 * out[m, n] = (sum_k e4m3(a[m,k]) * e4m3(w[n,k])) * sa[m] * sw[n], fp32 accumulation,
 * written as bf16 (out_f32 = 0) or fp32 (out_f32 = 1) with row pitch ldc (elements).
 * a_codes int8[M, K] and w_codes int8[N, K] are the E4M3 bit patterns that
 * kc_quantize_fp8_per_token / kc_quantize_fp8_per_channel (and the reference's
 * launch_quantize_fp8, fp8_quant.cu:201) produce.  Requires K % 16 == 0,
 * N % 8 == 0, ldc % 8 == 0 and 16-byte aligned codes, sw and out. */
KC_API int kc_gemm_fp8(const int8_t* a_codes, const float* sa, const int8_t* w_codes, const float* sw,
                       void* out, int out_f32, int M, int N, int K, int ldc, cudaStream_t stream);
/* kc_gemm_fp8 on at most max_ctas SMs (<= 0: all): the GEMM is persistent,
 * one CTA per SM, so a collective queued beside it on another stream (the
 * row-parallel all-reduce of the previous row block) only runs concurrently
 * if SMs are left free for it. */
KC_API int kc_gemm_fp8_ctas(const int8_t* a_codes, const float* sa, const int8_t* w_codes,
                            const float* sw, void* out, int out_f32, int M, int N, int K, int ldc,
                            int max_ctas, cudaStream_t stream);

/* W4A16 GEMM (prefill) on the tcgen05 tensor cores:
 * out[m, n] = sum_k x[m, k] * w[n, k] with w[n, k] = bf16((u - 8) * s[n, k / gs]),
 * the exact bf16 weights kc_dequantize_w4_bf16 produces (GPTQ symmetric INT4,
 * the reference's dequantize_int4 of packed ^ 0x88 with zero points 0,
 * quant_int4.cu:99-104), fp32 accumulation, written as bf16 (out_f32 = 0) or
 * fp32 (out_f32 = 1) with row pitch ldc (elements).  x bf16 [M, K],
 * packed u8 [N, K/2] (low nibble = even k), scales fp16 [N, K/gs].
 * Requires K % 64 == 0, group_size % 64 == 0 dividing K, ldc >= N and
 * 16-byte aligned x and packed. */
KC_API int kc_gemm_w4a16(const uint16_t* x_bf16, const uint8_t* packed, const uint16_t* scales_f16,
                         void* out, int out_f32, int M, int N, int K, int group_size, int ldc,
                         cudaStream_t stream);

/* Activations the W4A16 GEMM epilogue can apply to the fp32 accumulator. */
#define KC_ACT_NONE       0
#define KC_ACT_GELU_QUICK 1   /* x * sigmoid(1.702 x): the reference MLP block's GELU,
                                 examples/python/transformer/tensor_parallel.py:162 */

/* kc_gemm_w4a16 with an activation applied in the epilogue, before the
 * rounding to bf16 (or the fp32 store): the first linear of the reference's
 * column-parallel -> GELU -> row-parallel MLP block
 * (examples/python/transformer/tensor_parallel.py:150-172), where
 * launch_col_parallel_linear (tensor_parallel.cu:209) and a separate numpy
 * GELU run in two passes.  Same arguments and requirements as kc_gemm_w4a16;
 * act is KC_ACT_NONE or KC_ACT_GELU_QUICK. */
KC_API int kc_gemm_w4a16_act(const uint16_t* x_bf16, const uint8_t* packed,
                             const uint16_t* scales_f16, void* out, int out_f32, int M, int N,
                             int K, int group_size, int ldc, int act, cudaStream_t stream);

/* kc_gemm_w4a16_act with per-group zero points (AWQ, asymmetric GPTQ; no
 * reference counterpart, see kc_gemv_w4a16_zp): the weights are the exact
 * bf16((u - z[n, k/gs]) * s[n, k/gs]) that kc_dequantize_w4_bf16_zp produces,
 * zeros u8[N, K/gs] (0..15).  Same requirements as kc_gemm_w4a16. */
KC_API int kc_gemm_w4a16_zp(const uint16_t* x_bf16, const uint8_t* packed,
                            const uint16_t* scales_f16, const uint8_t* zeros, void* out,
                            int out_f32, int M, int N, int K, int group_size, int ldc, int act,
                            cudaStream_t stream);

/* Column-parallel W4A16 GEMM fused with the all-gather of its output (one
 * process per GPU; no counterpart kernel in the reference, whose
 * launch_col_parallel_linear + launch_allgather_nccl, tensor_parallel.cu:209 and
 * tensor_parallel_nccl.cu:127, run the two steps apart).  This rank multiplies
 * x [M, K] by its weight shard (rows rank*N_shard .. +N_shard of the full
 * [N_shard*nranks, K] matrix, same packing as kc_gemm_w4a16) and its epilogue
 * writes every bf16 tile straight into columns rank*N_shard .. of all nranks
 * output buffers outs[r] ([M, N_shard*nranks] row-major bf16, 16-byte aligned;
 * outs[rank] local, the others mapped peer memory, kc_ipc_open) over NVLink.
 * Asynchronous: the caller synchronizes the ranks (e.g. a collective on the
 * same stream) before reading the result, and before the next call if a rank
 * may still be reading the previous one.  nranks <= KC_MAX_RANKS, N_shard % 128 == 0. */
#define KC_MAX_RANKS 8
KC_API int kc_gemm_w4a16_allgather(const uint16_t* x_bf16, const uint8_t* packed_shard,
                                   const uint16_t* scales_shard, void* const* outs, int nranks,
                                   int rank, int M, int N_shard, int K, int group_size,
                                   cudaStream_t stream);
/* As kc_gemm_w4a16_allgather, with every output tile written once through
 * NVLink SHARP: mc_out is the multicast address of a bf16 [M, N_shard*nranks]
 * buffer bound on every rank (e.g. a symmetric allocation's multicast
 * pointer); the epilogue stores each tile with multimem.st and the switch
 * writes it into every rank's copy, so a tile leaves the GPU once instead of
 * once per peer.  Synchronization as for kc_gemm_w4a16_allgather. */
KC_API int kc_gemm_w4a16_allgather_mc(const uint16_t* x_bf16, const uint8_t* packed_shard,
                                      const uint16_t* scales_shard, void* mc_out, int nranks, int rank,
                                      int M, int N_shard, int K, int group_size, cudaStream_t stream);

/* Row-parallel FP8 GEMM with its all-reduce fused into the epilogue (one
 * process per GPU; the reference composes launch_row_parallel_linear with
 * launch_ring_allreduce_nccl, tensor_parallel.cu:235, tensor_parallel_nccl.cu:105).
 * Each rank holds the K shard of both code matrices (a_codes_shard [M, K_shard],
 * w_codes_shard [N, K_shard]) and the full-row scales sa [M], sw [N]; output
 * rows are owned in nranks equal blocks.  A partial tile of another owner is
 * written (bf16) into that owner's receive slot and announced by a flag; the
 * owner adds the received partials to its fp32 tile and writes the bf16 sum
 * into every rank's output, so every outs[r] ends with the full [M, N] bf16
 * result.  outs[r] / recvs[r] / flags[r]: rank r's output [M, N] bf16, receive
 * slots (nranks - 1) x [M / nranks, N] bf16 and flags (nranks - 1) x
 * (M / 128 / nranks) x (N / 256) ints (zeroed once), as mapped in this process.
 * Every rank passes the same, increasing epoch (> 0).  The ranks' launches
 * must be aligned (a kc_peer_barrier before it) and the outputs are complete
 * once every rank's launch has finished (a barrier after it).  A flag wait
 * gives up after timeout_ns (0: KC_PEER_BARRIER_DEFAULT_TIMEOUT_NS), records
 * KC_ERR_TIMEOUT and makes the affected tiles NaN.
 * M % (128 * nranks) == 0, N % 256 == 0, K_shard % 16 == 0, 2 <= nranks <= KC_MAX_RANKS. */
KC_API int kc_gemm_fp8_allreduce(const int8_t* a_codes_shard, const float* sa, const int8_t* w_codes_shard,
                                 const float* sw, void* const* outs, void* const* recvs, int* const* flags,
                                 int nranks, int rank, int epoch, int M, int N, int K_shard,
                                 uint64_t timeout_ns, cudaStream_t stream);

/* As kc_gemm_fp8_allreduce, with the sum done in the NVSwitch: every rank
 * writes its partial tiles into its own copy `part` ([M, N] bf16) of a
 * symmetric buffer whose multicast address is `mc_part`, and flags each tile
 * to its owner; the owner sums the copies with multimem.ld_reduce (fp32
 * accumulation) and writes the bf16 sum into every copy with multimem.st, so
 * every rank's `part` ends as the full [M, N] result.  Per GPU the output
 * crosses NVLink once outward and (1 + 1/nranks) times inward, where the
 * peer form moves 2 (nranks - 1) / nranks each way.  flags, epoch, timeout,
 * alignment of the launches and shape limits as for kc_gemm_fp8_allreduce. */
KC_API int kc_gemm_fp8_allreduce_mc(const int8_t* a_codes_shard, const float* sa, const int8_t* w_codes_shard,
                                    const float* sw, void* part, void* mc_part, int* const* flags, int nranks,
                                    int rank, int epoch, int M, int N, int K_shard, uint64_t timeout_ns,
                                    cudaStream_t stream);

/* bf16 sum all-reduce over NVLink peer memory (one process per GPU; the
 * reference's counterpart is launch_ring_allreduce_nccl, fp32,
 * tensor_parallel_nccl.cu:105).  partials[r] / outs[r]: rank r's input and
 * output buffers of `count` bf16 as mapped in this process (own buffer at
 * index `rank`, peers' through kc_ipc_open).  This rank reduces the rank-th
 * 1/nranks slice -- fp32 sum in rank order, one rounding -- and writes it into
 * every outs[r]; all ranks together produce the full sum in every output.
 * The kernel does not synchronize with its peers: every rank's partial must be
 * complete before any rank launches, and the outputs are complete once every
 * rank's launch has finished (order both with collectives on the stream).
 * count % (8 * nranks) == 0, 16-byte aligned buffers, nranks <= KC_MAX_RANKS. */
KC_API int kc_allreduce_bf16_peer(const void* const* partials, void* const* outs, int nranks,
                                  int rank, long count, cudaStream_t stream);

/* bf16 sum all-reduce in place through NVLink SHARP (the switch's multicast
 * and in-switch reduction; no reference counterpart).  mc: the multicast
 * address of a buffer of `count` bf16 bound on every rank (e.g. a symmetric
 * allocation's multicast pointer).  This rank reduces the rank-th 1/nranks
 * slice (multimem.ld_reduce, fp32 accumulation in the switch) and writes the
 * sum into every rank's copy (multimem.st).  Synchronization as for
 * kc_allreduce_bf16_peer: every rank's data must be complete before any rank
 * launches (kc_peer_barrier), the result is complete once every rank's launch
 * has finished; after a barrier timeout it writes NaN.  max_ctas > 0 caps the
 * grid (leaves SMs to a concurrent GEMM).  count % (8 * nranks) == 0, mc
 * 16-byte aligned. */
KC_API int kc_allreduce_bf16_nvls(void* mc, int nranks, int rank, long count, int max_ctas,
                                  cudaStream_t stream);

/* Stream-ordered barrier of the ranks of one node over peer memory (no
 * reference counterpart).  flags[r]: rank r's array of KC_MAX_RANKS ints
 * (zeroed once before first use; own array at index `rank`, peers' through
 * kc_ipc_open).  Every rank calls it with the same, increasing epoch (> 0;
 * compared modulo 2^32, so it may wrap); one warp publishes the epoch to
 * every rank and waits until all ranks published it.  Work queued after it on
 * the stream starts only when every rank's work queued before it has
 * finished.
 * The wait is bounded by timeout_ns (0: KC_PEER_BARRIER_DEFAULT_TIMEOUT_NS;
 * at most KC_PEER_BARRIER_MAX_TIMEOUT_NS).  A barrier that gives up has
 * ordered nothing: the results of the work around it are UNDEFINED.  It
 * records KC_ERR_TIMEOUT for kc_get_device_status(), writes KC_ERR_TIMEOUT
 * into *status_host when status_host is not NULL (pinned host memory, so the
 * host can poll it without synchronizing), and every kc_allreduce_bf16_peer
 * and kc_allreduce_bf16_nvls of the process writes NaN from then on, until
 * kc_get_device_status() clears the status. */
#define KC_PEER_BARRIER_DEFAULT_TIMEOUT_NS 2000000000ull    /* 2 s */
#define KC_PEER_BARRIER_MAX_TIMEOUT_NS     600000000000ull  /* 10 min */
KC_API int kc_peer_barrier(int* const* flags, int nranks, int rank, int epoch, uint64_t timeout_ns,
                           int* status_host, cudaStream_t stream);

/* fp32 C[M,N] = A[M,K] * B[N,K]^T (the column/row-parallel shard GEMM). */
KC_API int kc_sgemm_nt(const float* A, const float* B, float* C, int M, int N, int K,
                cudaStream_t stream);

/* --- NCCL, one process per GPU (the reference only has single-process
 *     ncclCommInitAll, tensor_parallel_nccl.cu:58) --------------------------- */
/* Size in bytes of the opaque unique id (128). */
KC_API int kc_nccl_unique_id_bytes(void);
/* Rank 0 creates the id (host buffer of kc_nccl_unique_id_bytes() bytes) and
 * shares it with the other ranks out of band. */
KC_API int kc_nccl_get_unique_id(void* out_id);
/* Blocking communicator init on the current device; *comm is NULL on failure. */
KC_API int kc_nccl_comm_init_rank(void** comm, int nranks, const void* id, int rank);
KC_API int kc_nccl_comm_destroy(void* comm);
/* Abandons in-flight work (use after a peer failed). */
KC_API int kc_nccl_comm_abort(void* comm);
/* KC_OK, or KC_ERR_NCCL if the communicator has an asynchronous error. */
KC_API int kc_nccl_comm_check(void* comm);
/* bf16 all-gather: recv = [send_0 | ... | send_{R-1}], count elements per rank. */
KC_API int kc_allgather_bf16(void* comm, const uint16_t* send, uint16_t* recv, long count,
                      cudaStream_t stream);
/* bf16 / fp32 sum all-reduce (send == recv allowed). */
KC_API int kc_allreduce_bf16(void* comm, const uint16_t* send, uint16_t* recv, long count,
                      cudaStream_t stream);
KC_API int kc_allreduce_f32(void* comm, const float* send, float* recv, long count,
                     cudaStream_t stream);

/* --- device buffers shared between the processes of one node (no reference
 *     counterpart: the reference keeps every rank in one process) ------------- */
/* Size in bytes of an opaque IPC handle. */
KC_API int kc_ipc_handle_bytes(void);
/* cudaMalloc'd buffer whose handle can be shared; free with kc_ipc_free after
 * every peer closed its mapping. */
KC_API int kc_ipc_alloc(void** dev_ptr, size_t bytes);
KC_API int kc_ipc_free(void* dev_ptr);
/* Handle of a kc_ipc_alloc buffer (kc_ipc_handle_bytes() bytes, host memory). */
KC_API int kc_ipc_get_handle(const void* dev_ptr, void* handle_out);
/* Maps a peer process's buffer into this process (peer access enabled). */
KC_API int kc_ipc_open(const void* handle, void** dev_ptr);
KC_API int kc_ipc_close(void* dev_ptr);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* KERNEL_CRAFT_H */
