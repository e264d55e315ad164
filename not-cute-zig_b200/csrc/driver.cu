// driver.cu -- the driver-call table of libncz_flash.so (include/ncz_driver.h).
//
// The default table forwards to the CUDA runtime.  cuTensorMapEncodeTiled is
// resolved through cudaGetDriverEntryPointByVersion, so the library has no
// link-time dependency on libcuda and loads on machines without a GPU driver.
// ncz_set_driver swaps in a caller's table (host tests: a fake of N devices).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstddef>
#include <cstring>

#include "driver.cuh"
#include "status.cuh"

namespace {

std::atomic<PFN_cuTensorMapEncodeTiled_v12000> g_encode{nullptr};

int rt_get_device_count(int *count) { return cudaGetDeviceCount(count); }
int rt_get_device(int *device) { return cudaGetDevice(device); }
int rt_set_device(int device) { return cudaSetDevice(device); }
int rt_sm_count(int device, int *count) {
    return cudaDeviceGetAttribute(count, cudaDevAttrMultiProcessorCount, device);
}

int rt_load_tensor_map_encoder() {
    if (g_encode.load() != nullptr) return cudaSuccess;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || fn == nullptr) return cudaErrorSymbolNotFound;
    g_encode.store(reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn));
    return cudaSuccess;
}

int rt_encode_tensor_map(void *map, int bf16, const void *base, const uint64_t *dims, const uint64_t *strides,
                         const uint32_t *box, uint32_t swizzle_bytes) {
    const PFN_cuTensorMapEncodeTiled_v12000 encode = g_encode.load();
    if (encode == nullptr) return CUDA_ERROR_NOT_INITIALIZED;
    cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    cuuint64_t s[2] = {strides[0], strides[1]};
    cuuint32_t b[3] = {box[0], box[1], box[2]};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    const CUtensorMapSwizzle swz = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                   : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                         : CU_TENSOR_MAP_SWIZZLE_NONE;
    const CUtensorMapDataType type = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return encode(static_cast<CUtensorMap *>(map), type, 3, const_cast<void *>(base), d, s, b, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

int rt_set_max_dynamic_smem(const void *kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

int rt_launch_kernel(const void *kernel, uint32_t grid, uint32_t block, size_t smem_bytes, void *stream, void **args) {
    const cudaError_t e =
        cudaLaunchKernel(kernel, dim3(grid), dim3(block), args, smem_bytes, static_cast<cudaStream_t>(stream));
    // A rejected launch also sets the runtime's last error; clear it so the
    // caller's next error check sees only its own calls.
    if (e != cudaSuccess) (void)cudaGetLastError();
    return e;
}

int rt_stream_create(void **stream) {
    cudaStream_t s = nullptr;
    const cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    *stream = s;
    return e;
}
int rt_stream_destroy(void *stream) { return cudaStreamDestroy(static_cast<cudaStream_t>(stream)); }
int rt_event_create(void **event) {
    cudaEvent_t ev = nullptr;
    const cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    *event = ev;
    return e;
}
int rt_event_destroy(void *event) { return cudaEventDestroy(static_cast<cudaEvent_t>(event)); }
int rt_event_record(void *event, void *stream) {
    return cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream));
}
int rt_stream_wait_event(void *stream, void *event) {
    return cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0);
}
int rt_stream_synchronize(void *stream) { return cudaStreamSynchronize(static_cast<cudaStream_t>(stream)); }
int rt_device_synchronize() { return cudaDeviceSynchronize(); }
int rt_memcpy_async(void *dst, const void *src, size_t bytes, int kind, void *stream) {
    return cudaMemcpyAsync(dst, src, bytes, static_cast<cudaMemcpyKind>(kind), static_cast<cudaStream_t>(stream));
}
int rt_symbol_read(void *dst, const void *symbol, size_t bytes) {
    return cudaMemcpyFromSymbol(dst, symbol, bytes, 0, cudaMemcpyDeviceToHost);
}
int rt_symbol_write(const void *symbol, const void *src, size_t bytes) {
    return cudaMemcpyToSymbol(symbol, src, bytes, 0, cudaMemcpyHostToDevice);
}
int rt_symbol_address(void **address, const void *symbol) { return cudaGetSymbolAddress(address, symbol); }

int rt_pool_create(void **pool, int device, uint64_t release_threshold) {
    cudaMemPoolProps props;
    std::memset(&props, 0, sizeof(props));
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    cudaMemPool_t p = nullptr;
    cudaError_t e = cudaMemPoolCreate(&p, &props);
    if (e != cudaSuccess) return e;
    e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &release_threshold);
    if (e != cudaSuccess) {
        (void)cudaMemPoolDestroy(p);
        return e;
    }
    *pool = p;
    return cudaSuccess;
}
int rt_pool_destroy(void *pool) { return cudaMemPoolDestroy(static_cast<cudaMemPool_t>(pool)); }
int rt_pool_alloc_async(void **ptr, size_t bytes, void *pool, void *stream) {
    return cudaMallocFromPoolAsync(ptr, bytes, static_cast<cudaMemPool_t>(pool), static_cast<cudaStream_t>(stream));
}
int rt_free_async(void *ptr, void *stream) { return cudaFreeAsync(ptr, static_cast<cudaStream_t>(stream)); }

const ncz_driver_table kRuntime = {
    sizeof(ncz_driver_table), rt_get_device_count, rt_get_device,     rt_set_device,       rt_sm_count,
    rt_load_tensor_map_encoder, rt_encode_tensor_map, rt_set_max_dynamic_smem, rt_launch_kernel,
    rt_stream_create,           rt_stream_destroy,    rt_event_create,  rt_event_destroy,   rt_event_record,
    rt_stream_wait_event,       rt_stream_synchronize, rt_device_synchronize, rt_memcpy_async, rt_symbol_read,
    rt_symbol_write,            rt_symbol_address,    rt_pool_create,   rt_pool_destroy,    rt_pool_alloc_async,
    rt_free_async,
};

ncz_driver_table g_user;
std::atomic<const ncz_driver_table *> g_active{&kRuntime};

// Every entry after `size` is a function pointer; none may be missing.
bool complete(const ncz_driver_table &t) {
    constexpr size_t first = offsetof(ncz_driver_table, get_device_count);
    const unsigned char *bytes = reinterpret_cast<const unsigned char *>(&t);
    for (size_t off = first; off + sizeof(void *) <= sizeof(t); off += sizeof(void *)) {
        uintptr_t v = 0;
        std::memcpy(&v, bytes + off, sizeof(v));
        if (v == 0) return false;
    }
    return true;
}

}  // namespace

namespace ncz {
const ncz_driver_table &drv() { return *g_active.load(std::memory_order_acquire); }
}  // namespace ncz

extern "C" {

int ncz_set_driver(const ncz_driver_table *table, int *released) {
    if (table != nullptr && (table->size != sizeof(ncz_driver_table) || !complete(*table)))
        return NCZ_ERROR_INVALID_VALUE;
    const int st = ncz::release_flash_objects();
    if (released != nullptr) *released = st;
    ncz::reset_flash_caches();
    ncz::reset_mma_caches();
    if (table == nullptr) {
        g_active.store(&kRuntime, std::memory_order_release);
    } else {
        g_user = *table;
        g_active.store(&g_user, std::memory_order_release);
    }
    return NCZ_SUCCESS;
}

int ncz_get_driver(ncz_driver_table *out) {
    if (out == nullptr || out->size != sizeof(ncz_driver_table)) return NCZ_ERROR_INVALID_VALUE;
    *out = ncz::drv();
    return NCZ_SUCCESS;
}

int ncz_kernel_label(const void *kernel, char *label, size_t cap) {
    const char *name = ncz::flash_kernel_label(kernel);
    if (name == nullptr) name = ncz::mma_kernel_label(kernel);
    if (name == nullptr) return NCZ_ERROR_NOT_FOUND;
    if (label != nullptr && cap > 0) {
        std::strncpy(label, name, cap - 1);
        label[cap - 1] = '\0';
    }
    return NCZ_SUCCESS;
}

}  // extern "C"
