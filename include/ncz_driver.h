/* ncz_driver.h -- the injectable driver-call table of libncz_flash.so.
 *
 * Every CUDA call the C ABI makes goes through one table of plain C function
 * pointers: device selection, kernel launches, streams, events, copies, the
 * split-KV memory pool and tensor-map encoding.  By default the table is the
 * CUDA runtime.  A host test installs a table of its own, for example a fake
 * of eight devices that counts launches and allocations and fails chosen calls
 * on chosen devices.  It then checks per device, without a GPU, that errors
 * propagate as ncz_status codes, that the caller's device is restored, and
 * that library-owned memory, streams and pools are released.
 *
 * The reference has no such layer.  Its driver wrapper calls libcuda directly
 * (src/cuda.zig:181-388) and turns results into CudaError (src/cuda.zig:134-178).
 * Here every table entry returns a CUDA runtime error number (cudaError_t:
 * 0 success, 2 memory allocation, 100 no device, 101 invalid device,
 * 719 launch failure, ...), which the library maps onto the same error set
 * (ncz_flash.h).  Handles (streams, events, pools, device pointers) are opaque
 * pointers that the library only passes back to the table.
 */
#ifndef NCZ_DRIVER_H
#define NCZ_DRIVER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* memcpy_async directions (the cudaMemcpyKind numbers). */
#define NCZ_COPY_HOST_TO_DEVICE 1
#define NCZ_COPY_DEVICE_TO_HOST 2

typedef struct ncz_driver_table {
    size_t size; /* sizeof(ncz_driver_table) */
    int (*get_device_count)(int *count);
    int (*get_device)(int *device);
    int (*set_device)(int device);
    int (*sm_count)(int device, int *count);
    /* 0 when tensor maps can be encoded (cuTensorMapEncodeTiled resolved). */
    int (*load_tensor_map_encoder)(void);
    /* A 3-D tiled map of the 16-bit elements at `base` (f16, or bf16 when
     * bf16 != 0) into the 128-byte CUtensorMap at `map`: dims (x, y, z), byte
     * strides of y and z, box (x, y, z), swizzle span 32, 64 or 128 bytes.
     * 0 = encoded. */
    int (*encode_tensor_map)(void *map, int bf16, const void *base, const uint64_t *dims, const uint64_t *strides,
                             const uint32_t *box, uint32_t swizzle_bytes);
    int (*set_max_dynamic_smem)(const void *kernel, int bytes);
    /* cudaLaunchKernel with a 1-D grid and block; args[i] points at the i-th
     * kernel parameter. */
    int (*launch_kernel)(const void *kernel, uint32_t grid, uint32_t block, size_t smem_bytes, void *stream,
                         void **args);
    int (*stream_create)(void **stream); /* non-blocking stream on the current device */
    int (*stream_destroy)(void *stream);
    int (*event_create)(void **event); /* event without timing */
    int (*event_destroy)(void *event);
    int (*event_record)(void *event, void *stream);
    int (*stream_wait_event)(void *stream, void *event);
    int (*stream_synchronize)(void *stream);
    int (*device_synchronize)(void);
    int (*memcpy_async)(void *dst, const void *src, size_t bytes, int kind, void *stream);
    /* Copies from / to a __device__ variable of the library, named by its host
     * address. */
    int (*symbol_read)(void *dst, const void *symbol, size_t bytes);
    int (*symbol_write)(const void *symbol, const void *src, size_t bytes);
    int (*symbol_address)(void **address, const void *symbol);
    /* A stream-ordered pool on `device` keeping up to release_threshold bytes
     * between calls; on failure nothing is left allocated. */
    int (*pool_create)(void **pool, int device, uint64_t release_threshold);
    int (*pool_destroy)(void *pool);
    int (*pool_alloc_async)(void **ptr, size_t bytes, void *pool, void *stream);
    int (*free_async)(void *ptr, void *stream);
} ncz_driver_table;

/* Installs `table` (copied; NULL = the CUDA runtime).  First releases, through
 * the table in use, what the library owns (split-KV pools, host-pipeline
 * streams and events), then drops its cached state (initialisation, kernel
 * attributes, tensor maps, SM counts, static scratch addresses), so the next
 * call starts over through the new table.  Returns NCZ_ERROR_INVALID_VALUE for
 * a wrong size or a missing entry (nothing changes then), else NCZ_SUCCESS.
 * `released` (may be NULL) receives the first error of the release, or
 * NCZ_SUCCESS; the table is installed either way.  No other thread may be
 * inside the library meanwhile. */
int ncz_set_driver(const ncz_driver_table *table, int *released);

/* Copies the table in use into *out (out->size must be sizeof(ncz_driver_table)). */
int ncz_get_driver(ncz_driver_table *out);

/* Name of a kernel of the library by the host address that launch_kernel
 * receives, e.g. "flash_fwd<64,tma,f16>", "combine_splits<32>",
 * "mma_gemm<row_b>"; NCZ_ERROR_NOT_FOUND for any other address. */
int ncz_kernel_label(const void *kernel, char *label, size_t cap);

#ifdef __cplusplus
}
#endif

#endif /* NCZ_DRIVER_H */
