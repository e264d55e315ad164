/* ncz_mma.h -- C ABI of the batched 16x8 GEMM with fused epilogue in
 * libncz_flash.so (sm_100a).
 *
 * Drop-in for the reference's mma demo kernels (src/kernels.zig):
 *   pipelined_mma_matmul  src/kernels.zig:33-141   -> ncz_mma_matmul_pipelined
 *   batched_mma_matmul    src/kernels.zig:301-319  -> ncz_mma_matmul_batched
 *   mma_matmul            src/kernels.zig:290-299  -> ncz_mma_matmul
 * Each batch b computes one 16x8 f32 tile
 *   D_b = epilogue(alpha * (A_b B_b) + beta * C_b)
 * with f16 A and B and f32 accumulation.  The reference takes the batch count
 * from grid.y; here it is the `batches` argument.  Pointers are device
 * pointers owned by the caller; strides are in elements, as in the reference
 * (D uses batch_stride_c, src/kernels.zig:59).  Launches are asynchronous on
 * `stream` (NULL = default stream).  Return codes are the ncz_status values
 * of ncz_flash.h.
 */
#ifndef NCZ_MMA_H
#define NCZ_MMA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* kernels.Epilogue (src/kernels.zig:26-31).  As in the reference, any other
 * value applies no activation. */
typedef enum {
    NCZ_EPILOGUE_NONE = 0,
    NCZ_EPILOGUE_RELU = 1,
    NCZ_EPILOGUE_SILU = 2,
    NCZ_EPILOGUE_GELU = 3
} ncz_epilogue;

/* pipelined_mma_matmul: A_b is k_iters consecutive row-major 16x16 tiles,
 * B_b k_iters consecutive row-major 16x8 (K x N) tiles, C_b and D_b row-major
 * 16x8.  k_iters >= 1 (the reference's k_iters - 1 loop bound underflows at
 * 0; here 0 is NCZ_ERROR_INVALID_VALUE).  batches = 0 launches nothing. */
int ncz_mma_matmul_pipelined(const void *a, const void *b, const void *c, void *d, float alpha, float beta,
                             size_t batch_stride_a, size_t batch_stride_b, size_t batch_stride_c,
                             size_t k_iters, uint32_t epilogue, size_t batches, void *stream);

/* batched_mma_matmul: one row-major 16x16 A tile and one column-major 16x8
 * B tile (element (k, n) at n * 16 + k) per batch, no activation. */
int ncz_mma_matmul_batched(const void *a, const void *b, const void *c, void *d, float alpha, float beta,
                           size_t batch_stride_a, size_t batch_stride_b, size_t batch_stride_c, size_t batches,
                           void *stream);

/* mma_matmul: batched_mma_matmul with a single batch. */
int ncz_mma_matmul(const void *a, const void *b, const void *c, void *d, float alpha, float beta, void *stream);

/* Reads and clears the bounded-wait status word of the GEMM kernel on
 * `device` (-1 = current): NCZ_SUCCESS, or NCZ_ERROR_DEVICE_TIMEOUT when a
 * wait for a staged tile ran past the wait limit (the kernel then stopped
 * cleanly; D is incomplete). */
int ncz_mma_sync_status(int device);

/* Test hooks (failure detection without a GPU fault), device -1 = current.
 * ncz_mma_test_set_wait_limit: bound of every stage wait in SM cycles
 * (0 restores the default of about 2 s).  ncz_mma_test_drop_copy: while
 * enabled, the first warp of a launch arms its first stage for bytes it never
 * copies, so that wait runs out and the next ncz_mma_sync_status reports
 * NCZ_ERROR_DEVICE_TIMEOUT. */
int ncz_mma_test_set_wait_limit(int device, uint64_t cycles);
int ncz_mma_test_drop_copy(int device, int enable);

#ifdef __cplusplus
}
#endif

#endif /* NCZ_MMA_H */
