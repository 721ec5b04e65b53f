/*
 * gg_noalloc.h: C declarations of the allocation-free grouped GEMM entry point.
 *
 * No counterpart in the reference: it has no C entry point of this kind.
 *
 * The functions are defined in csrc/kernels/gg_noalloc.cu and exported with
 * default visibility from the `_kernels` extension library
 * (revealaiccl_b200/_kernels*.so).  A C or C++ program that links neither
 * torch nor an allocator of its own can dlopen that library (or link it) and
 * call them with raw device pointers.  The entry point itself calls no
 * cudaMalloc, no cudaFree and no allocating library routine: its working
 * memory is one file-scope device array of 4608 bytes per GPU, which every
 * call shares (see the notes in gg_noalloc.cu).
 */
#ifndef RAICCL_GG_NOALLOC_H_
#define RAICCL_GG_NOALLOC_H_

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes: 0 = enqueued; > 0 = a cudaError_t value; < 0 = rejected. */
#define RAICCL_NOALLOC_TOO_MANY_SEGMENTS (-1)
#define RAICCL_NOALLOC_BAD_ARGUMENT (-2)
#define RAICCL_NOALLOC_LAUNCH_FAILED (-3)
#define RAICCL_NOALLOC_BAD_DEVICE (-4)

/* Largest num_segs one call accepts (the scratch array's capacity). */
int raiccl_grouped_gemm_noalloc_max_segments(void);

/* Text for a return code of any of these functions. */
const char* raiccl_grouped_gemm_noalloc_error_string(int code);

/*
 * For every segment (int32[8] records: a_row0, rows, expert, out_slot, out_row0,
 * three unused words; 16-byte aligned):
 *   out[o(r), :] = act(A[a_row0 + r] @ B[expert * N : (expert + 1) * N].T + bias[expert]) * row_scale[a_row0 + r]
 * with o(r) = row_map[a_row0 + r] when row_map is given, else out_row0 + r.
 *
 *   in_fp32   0: A and B are bf16; 1: fp32 (tf32 tensor-core math)
 *   A         [rows_a, K], row stride lda elements; B [rows_b, K], row stride ldb
 *             (rows_b = E * N); both 16-byte aligned, strides multiples of 16 bytes
 *   bn        tile width 16/32/64/128/256 dividing N
 *   act       0 none, 1 relu, 2 gelu, 3 silu, 4 swiglu (bn >= 32; output width N / 2)
 *   bias      fp32 [rows_b], 16-byte aligned, or NULL
 *   row_map   int32 [rows_a] or NULL; row_scale fp32 [rows_a] or NULL
 *   out       [out_rows, ldo] fp32 (out_bf16 = 0) or bf16 (out_bf16 = 1), 16-byte
 *             aligned, ldo >= output width, ldo * element size a multiple of 16
 *   grid      persistent CTAs (0: one per SM)
 *   timeout_ns  bound of every device-side wait (0: 2 s)
 *
 * Segments are checked on the device before any tile runs: out_slot must be 0,
 * the A rows must lie in [0, rows_a), the expert in [0, rows_b / N) and every
 * output row in [0, out_rows).  A call with a bad segment writes nothing and
 * leaves a status (4 = bounds, 5 = configuration) that
 * raiccl_grouped_gemm_noalloc_status returns.
 *
 * The call only enqueues work on `stream`.  Calls on one GPU share one scratch
 * array: calls whose work can overlap on the GPU race.  The first call on a GPU
 * resolves the array's device address; make it before any stream capture.
 */
int raiccl_grouped_gemm_noalloc(int in_fp32, const void* A, long long rows_a, long long K, long long lda,
                                const void* B, long long rows_b, long long ldb, const void* segs, int num_segs,
                                int N, int bn, int act, const float* bias, const int* row_map,
                                const float* row_scale, void* out, long long out_rows, long long ldo,
                                int out_bf16, int grid, unsigned long long timeout_ns, cudaStream_t stream);

/*
 * Waits for `stream`, copies the 32-byte device status record of the current
 * GPU (int code, kernel id, block, thread; long long index, bound) to
 * host_status when it is not NULL, and returns the status code (0 = no error
 * recorded), or minus the cudaError_t value if the wait or the copy failed.
 */
int raiccl_grouped_gemm_noalloc_status(void* host_status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RAICCL_GG_NOALLOC_H_ */
