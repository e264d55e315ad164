/* A C99 consumer of the library's public headers (include/ncz_flash.h,
 * ncz_mma.h, ncz_driver.h), built and run by tests/test_c_abi.py on the CPU.
 * It installs a driver-call table of its own (one fake device that records
 * launches), calls the reference-shaped entry points and checks the results,
 * then restores the CUDA runtime.  Exit status 0 = every check passed. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "ncz_driver.h"
#include "ncz_flash.h"
#include "ncz_mma.h"

static int g_launches;
static uint32_t g_last_grid, g_last_block;
static const void *g_last_kernel;
static uintptr_t g_next = 0x10000;

static int ok_count(int *n) { *n = 1; return 0; }
static int ok_get(int *d) { *d = 0; return 0; }
static int ok_set(int d) { return d == 0 ? 0 : 101; }
static int ok_sms(int d, int *n) { (void)d; *n = 148; return 0; }
static int ok_void(void) { return 0; }
static int ok_encode(void *map, int bf16, const void *base, const uint64_t *dims, const uint64_t *strides,
                     const uint32_t *box, uint32_t swizzle) {
    (void)bf16; (void)base; (void)dims; (void)strides; (void)box; (void)swizzle;
    memset(map, 0, 128);
    return 0;
}
static int ok_smem(const void *k, int bytes) { (void)k; (void)bytes; return 0; }
static int rec_launch(const void *k, uint32_t grid, uint32_t block, size_t smem, void *stream, void **args) {
    (void)smem; (void)stream; (void)args;
    ++g_launches;
    g_last_grid = grid;
    g_last_block = block;
    g_last_kernel = k;
    return 0;
}
static int new_handle(void **h) { *h = (void *)(g_next += 0x100); return 0; }
static int ok_handle(void *h) { (void)h; return 0; }
static int ok_pair(void *a, void *b) { (void)a; (void)b; return 0; }
static int ok_copy(void *dst, const void *src, size_t n, int kind, void *stream) {
    (void)dst; (void)src; (void)n; (void)kind; (void)stream;
    return 0;
}
static int zero_read(void *dst, const void *sym, size_t n) { (void)sym; memset(dst, 0, n); return 0; }
static int ok_write(const void *sym, const void *src, size_t n) { (void)sym; (void)src; (void)n; return 0; }
static int fake_addr(void **addr, const void *sym) { (void)sym; *addr = (void *)0x70000000u; return 0; }
static int new_pool(void **pool, int device, uint64_t keep) { (void)device; (void)keep; return new_handle(pool); }
static int pool_alloc(void **p, size_t n, void *pool, void *stream) {
    (void)n; (void)pool; (void)stream;
    return new_handle(p);
}

#define CHECK(cond)                                                      \
    do {                                                                 \
        if (!(cond)) {                                                   \
            fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond); \
            return 1;                                                    \
        }                                                                \
    } while (0)

int main(void) {
    ncz_driver_table t;
    char label[64];
    uint32_t dims = 0, always = 0, threads = 0;
    int released = -1;
    const void *q = (const void *)0x10000000u, *k = (const void *)0x20000000u, *v = (const void *)0x30000000u;
    void *o = (void *)0x40000000u;

    memset(&t, 0, sizeof t);
    t.size = sizeof t;
    t.get_device_count = ok_count;
    t.get_device = ok_get;
    t.set_device = ok_set;
    t.sm_count = ok_sms;
    t.load_tensor_map_encoder = ok_void;
    t.encode_tensor_map = ok_encode;
    t.set_max_dynamic_smem = ok_smem;
    t.launch_kernel = rec_launch;
    t.stream_create = new_handle;
    t.stream_destroy = ok_handle;
    t.event_create = new_handle;
    t.event_destroy = ok_handle;
    t.event_record = ok_pair;
    t.stream_wait_event = ok_pair;
    t.stream_synchronize = ok_handle;
    t.device_synchronize = ok_void;
    t.memcpy_async = ok_copy;
    t.symbol_read = zero_read;
    t.symbol_write = ok_write;
    t.symbol_address = fake_addr;
    t.pool_create = new_pool;
    t.pool_destroy = ok_handle;
    t.pool_alloc_async = pool_alloc;
    t.free_async = ok_pair;
    CHECK(ncz_set_driver(&t, &released) == NCZ_SUCCESS && released == NCZ_SUCCESS);

    /* flash.Options.validate and selectKernel */
    CHECK(ncz_flash_validate(4, 1024, 64, 1024 * 64, 1024 * 64, 1024 * 64, 1024 * 64) == NCZ_SUCCESS);
    CHECK(ncz_flash_validate(4, 1024, 48, 1024 * 64, 1024 * 64, 1024 * 64, 1024 * 64) == NCZ_ERROR_INVALID_VALUE);
    CHECK(ncz_flash_select(4, 1024, 64, 1, label, sizeof label, &threads) == NCZ_SUCCESS);
    CHECK(strcmp(label, "flash_fwd_sm100a_d64") == 0 && threads == 384);

    /* the reference kernel tuple: one launch; 4 row groups x 4 slices would
     * leave SMs idle, so the items are split-Q ones: 8 Q tiles x 4 slices */
    CHECK(ncz_flash_fwd(q, k, v, o, 4, 1024, 64, 1024 * 64, 1024 * 64, 1024 * 64, 1024 * 64, 0.125f, 1, NULL) ==
          NCZ_SUCCESS);
    CHECK(g_launches == 1 && g_last_grid == 32 && g_last_block == 384);
    CHECK(ncz_kernel_label(g_last_kernel, label, sizeof label) == NCZ_SUCCESS);
    CHECK(strcmp(label, "flash_fwd<64,tma,f16>") == 0);

    /* a reference kernel name: h64 takes d=64 only and returns otherwise */
    CHECK(ncz_flash_kernel_info("flash_attention_fwd_h64_causal", &dims, &always) == NCZ_SUCCESS);
    CHECK(dims == 4u && always == 1u);
    CHECK(ncz_flash_fwd_named("flash_attention_fwd_h64_bn32", q, k, v, o, 4, 1024, 32, 1024 * 32, 1024 * 32,
                              1024 * 32, 1024 * 32, 0.125f, 1, NULL) == NCZ_SUCCESS);
    CHECK(g_launches == 1);
    CHECK(ncz_flash_fwd_named("flash_attention_fwd_v2", q, k, v, o, 4, 1024, 32, 1024 * 32, 1024 * 32, 1024 * 32,
                              1024 * 32, 0.125f, 1, NULL) == NCZ_SUCCESS);
    CHECK(g_launches == 2);
    CHECK(ncz_flash_fwd_named("no_such_kernel", q, k, v, o, 4, 1024, 32, 1024 * 32, 1024 * 32, 1024 * 32,
                              1024 * 32, 0.125f, 1, NULL) == NCZ_ERROR_NOT_FOUND);

    /* the mma demo kernels' tuple, grid.y passed as batches */
    CHECK(ncz_mma_matmul_pipelined(q, k, v, o, 1.0f, 0.5f, 1024, 512, 128, 4, NCZ_EPILOGUE_SILU, 1000, NULL) ==
          NCZ_SUCCESS);
    CHECK(g_launches == 3 && g_last_grid == 100); /* 1000 batches, one per warp, 10 warps per CTA */
    CHECK(ncz_kernel_label(g_last_kernel, label, sizeof label) == NCZ_SUCCESS);
    CHECK(strcmp(label, "mma_gemm<row_b>") == 0);
    CHECK(ncz_mma_sync_status(-1) == NCZ_SUCCESS);

    CHECK(strcmp(ncz_status_string(NCZ_ERROR_DEVICE_TIMEOUT), "DeviceTimeout") == 0);
    CHECK(ncz_set_driver(NULL, &released) == NCZ_SUCCESS);
    printf("c abi consumer: ok\n");
    return 0;
}
