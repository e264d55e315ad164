// flash_api.cu -- the C ABI of libncz_flash.so (declared in include/ncz_flash.h).
//
// Host side of the drop-in for not-cute-zig's `flash` module:
//   Options.validate  src/flash.zig:16-28   -> ncz_flash_validate
//   launch/requireLen src/flash.zig:31-70,98-100 -> ncz_flash_launch / ncz_flash_fwd
//   selectKernel      src/flash.zig:72-96   -> ncz_flash_select
//   CudaError/check   src/cuda.zig:134-178  -> ncz_status / map_cuda_error
// The driver wrapper's single context (src/cuda.zig:181-196) becomes the
// runtime's per-device primary contexts.  Every CUDA call goes through the
// driver-call table (driver.cu, include/ncz_driver.h), so host tests can fake
// devices and fail chosen calls.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "driver.cuh"
#include "flash_fwd_sm100.cuh"
#include "status.cuh"
#include "ncz_flash.h"

// Split-KV partials of ncz_flash_fwd_static, the entry point that allocates
// nothing: a fixed array in the library's device image, NCZ_STATIC_SCRATCH_BYTES
// (16 MiB) on every device that loads the library, held until the process
// exits.  Host code must not pass `g_ncz_scratch` itself to a kernel (on the
// host it names a stand-in, not device memory); static_scratch() looks up its
// device address once per device, with that device current.
constexpr size_t kStaticScratchFloats = NCZ_STATIC_SCRATCH_BYTES / sizeof(float);
static __device__ __align__(256) float g_ncz_scratch[kStaticScratchFloats];

namespace {

using ncz::FlashParams;
using ncz::SmemLayout;

constexpr int kMaxDevices = 64;
constexpr size_t kGroupRows = static_cast<size_t>(ncz::kBlockM) * ncz::kQTiles;  // Q rows per CTA
constexpr int kVariants = 12;  // (D in 16/32/64) x (TMA, LSU) x (f16, bf16 inputs)
// Items with at least this many K tiles end their CTA instead of taking the
// next item; measured fastest with every item taking the next one.
// K/V bytes per chunk of slices in the item order (measured best of 16-96 MB
// at d=64: 32 MB, e.g. 16 slices at S=8192).
#ifndef NCZ_CHUNK_KV_BYTES
#define NCZ_CHUNK_KV_BYTES (32u << 20)
#endif
#ifndef NCZ_WALK_TILES
#define NCZ_WALK_TILES (1 << 30)
#endif
// Split-Q items (one Q tile per item, its K tiles alternating between the two
// pipelines) for every Q tile when the items of two Q tiles number fewer than
// this many per SM: some SMs would idle, or take a second item while the rest
// finish, and the longest item bounds the launch, so halving it pays (config
// 2, 32 items: 22.9 -> 18.4 us; 160 causal items at S=8192: 104.5 -> 81.8 us).
// From 1.5 items per SM up split-Q lost 4-14 %: there are twice the items,
// each with a fixed cost (Q load, first scores, a merge epilogue that holds
// both pipelines) over half the K tiles, while a split-Q K tile alone costs
// only 2-11 % more than a two-tile step (each K/V tile feeds one pipeline
// instead of two), and the longest two-tile item no longer bounds the
// launch.  Splitting only
// the heaviest groups never gained more than 3 % over the better of none and
// all in a sweep of 12 shapes, so the plan is all or nothing.
#ifndef NCZ_QSPLIT_ITEMS_PER_SM
#define NCZ_QSPLIT_ITEMS_PER_SM 1.25
#endif

std::mutex g_mu;
// Split-Q choice: 0 automatic, 1 whenever the launch has no split-KV, 2 never
// (ncz_test_set_qsplit).
std::atomic<int> g_qsplit_mode{0};
// >= 0: that many split-Q groups (clamped) instead of the mode's choice
// (ncz_test_set_qsplit_groups); -1 = the mode decides.
std::atomic<int> g_qsplit_force{-1};
// Twin items (two slices of one Q tile per item) for launches with
// seq_len <= 128: 1 = when eligible (default), 0 = never (ncz_test_set_twin).
std::atomic<int> g_twin_mode{1};
bool g_init_done = false;
int g_init_status = NCZ_ERROR_NOT_INITIALIZED;
std::atomic<uint64_t> g_launches{0};
bool g_attr_done[kMaxDevices][kVariants];

using ncz::drv;
using ncz::map_cuda_error;

// Fully resolved launch description: row strides defaulted, dtype checked.
struct Resolved {
    const void *q, *k, *v;
    void *o;
    size_t bh, seq, d;
    size_t qs, ks, vs, os;      // slice strides
    size_t qr, kr, vr, orow;    // row strides
    float scale;
    uint32_t causal;
    int o_dtype;
    int in_dtype;  // NCZ_DTYPE_F16 or NCZ_DTYPE_BF16 (0 in a descriptor = f16)
    int producer;
    int device;
    cudaStream_t stream;
    int splits = 0;  // split-KV request: 0 = automatic, 1 = none, n = n ranges
    bool use_static = false;   // split-KV partials in the static scratch array, not the pool
    float *scratch = nullptr;  // (resolved on the launch device)
    size_t scratch_floats = 0;
#ifdef NCZ_DEBUG_ITEM_VISITS
    unsigned int *item_visits = nullptr;  // debug build: per-item visit counters (device)
    size_t item_visits_cap = 0;
    size_t *items_out = nullptr;
#endif
};

bool mul_ok(size_t a, size_t b, size_t *out) { return !__builtin_mul_overflow(a, b, out); }

// The reference rule (src/flash.zig:16-28), generalised to row strides:
// the last element a slice touches is (seq-1)*row + d - 1 < stride.
int validate_resolved(const Resolved &r) {
    if (r.bh == 0 || r.seq == 0) return NCZ_ERROR_INVALID_VALUE;
    if (r.d != 16 && r.d != 32 && r.d != 64) return NCZ_ERROR_INVALID_VALUE;
    const size_t rows[4] = {r.qr, r.kr, r.vr, r.orow};
    const size_t slices[4] = {r.qs, r.ks, r.vs, r.os};
    for (int i = 0; i < 4; ++i) {
        if (rows[i] < r.d) return NCZ_ERROR_INVALID_VALUE;
        size_t span;
        if (!mul_ok(r.seq - 1, rows[i], &span) || span + r.d < span) return NCZ_ERROR_OVERFLOW;
        if (slices[i] < span + r.d) return NCZ_ERROR_INVALID_VALUE;
        size_t total;
        if (!mul_ok(slices[i], r.bh, &total)) return NCZ_ERROR_OVERFLOW;
    }
    if (r.o_dtype != NCZ_DTYPE_F32 && r.o_dtype != NCZ_DTYPE_F16 && r.o_dtype != NCZ_DTYPE_BF16)
        return NCZ_ERROR_INVALID_VALUE;
    if (r.in_dtype != NCZ_DTYPE_F16 && r.in_dtype != NCZ_DTYPE_BF16) return NCZ_ERROR_INVALID_VALUE;
    if (r.producer < NCZ_PRODUCER_AUTO || r.producer > NCZ_PRODUCER_LSU) return NCZ_ERROR_INVALID_VALUE;
    // Implementation limits of the 32-bit tile / grid indices.
    if (r.seq > (size_t(1) << 30)) return NCZ_ERROR_INVALID_VALUE;
    const size_t groups = (r.seq + kGroupRows - 1) / kGroupRows;
    size_t grid;
    if (!mul_ok(groups, r.bh, &grid) || grid > size_t(0x7FFFFFFF) / 8) return NCZ_ERROR_INVALID_VALUE;
    if (r.bh > size_t(0x7FFFFFFF)) return NCZ_ERROR_INVALID_VALUE;
    return NCZ_SUCCESS;
}

Resolved from_desc(const ncz_flash_desc &d) {
    Resolved r;
    r.q = d.q; r.k = d.k; r.v = d.v; r.o = d.o;
    r.bh = d.batch_heads; r.seq = d.seq_len; r.d = d.head_dim;
    r.qs = d.q_stride; r.ks = d.k_stride; r.vs = d.v_stride; r.os = d.o_stride;
    r.qr = d.q_row_stride ? d.q_row_stride : d.head_dim;
    r.kr = d.k_row_stride ? d.k_row_stride : d.head_dim;
    r.vr = d.v_row_stride ? d.v_row_stride : d.head_dim;
    r.orow = d.o_row_stride ? d.o_row_stride : d.head_dim;
    r.scale = d.scale; r.causal = d.causal;
    r.o_dtype = d.o_dtype; r.producer = d.producer; r.device = d.device;
    r.in_dtype = d.in_dtype == 0 ? NCZ_DTYPE_F16 : d.in_dtype;
    r.stream = static_cast<cudaStream_t>(d.stream);
    return r;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// 3-D map over one operand: dims (d, seq, bh), box (d, box_rows, 1), swizzle = row width.
bool encode_map_uncached(CUtensorMap *map, const void *ptr, size_t d, size_t seq, size_t bh, size_t row,
                         size_t slice, uint32_t box_rows, bool bf16) {
    const uint64_t dims[3] = {d, seq, bh};
    const uint64_t strides[2] = {row * 2, slice * 2};
    const uint32_t box[3] = {static_cast<uint32_t>(d), box_rows, 1u};
    const uint32_t swizzle = static_cast<uint32_t>(d * 2);  // one row: 32, 64 or 128 bytes
    return drv().encode_tensor_map(map, bf16 ? 1 : 0, ptr, dims, strides, box, swizzle) == 0;
}

// Encoded maps, direct-mapped by their inputs.  A map is a pure function of
// (address, layout, box, type), so a hit is always valid, also for a buffer
// freed and reallocated at the same address.
struct MapKey {
    uintptr_t ptr;
    size_t d, seq, bh, row, slice;
    uint32_t box_rows, bf16;
    bool operator==(const MapKey &o) const {
        return ptr == o.ptr && d == o.d && seq == o.seq && bh == o.bh && row == o.row && slice == o.slice &&
               box_rows == o.box_rows && bf16 == o.bf16;
    }
};
struct MapSlot {
    bool used = false;
    MapKey key;
    CUtensorMap map;
};
constexpr size_t kMapSlots = 256;
MapSlot g_maps[kMapSlots];

bool encode_map(CUtensorMap *map, const void *ptr, size_t d, size_t seq, size_t bh, size_t row, size_t slice,
                uint32_t box_rows, bool bf16) {
    const MapKey key{reinterpret_cast<uintptr_t>(ptr), d, seq, bh, row, slice, box_rows, bf16 ? 1u : 0u};
    size_t h = key.ptr * 0x9E3779B97F4A7C15ull;
    for (const size_t v : {d, seq, bh, row, slice, size_t(box_rows), size_t(key.bf16)}) h = (h ^ v) * 0x100000001B3ull;
    MapSlot &slot = g_maps[(h >> 24) % kMapSlots];
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (slot.used && slot.key == key) {
            *map = slot.map;
            return true;
        }
    }
    if (!encode_map_uncached(map, ptr, d, seq, bh, row, slice, box_rows, bf16)) return false;
    std::lock_guard<std::mutex> lock(g_mu);
    slot.used = true;
    slot.key = key;
    slot.map = *map;
    return true;
}

template <int D, bool kTma, bool kBf16>
int launch_variant(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv, const FlashParams &p,
                   unsigned grid, int dev, cudaStream_t stream) {
    using L = SmemLayout<D>;
    auto kernel = ncz::flash_fwd_sm100<D, kTma, kBf16>;
    const int vidx = ((D == 16 ? 0 : D == 32 ? 1 : 2) * 2 + (kTma ? 0 : 1)) * 2 + (kBf16 ? 1 : 0);
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (dev >= kMaxDevices) return NCZ_ERROR_INVALID_DEVICE;
        if (!g_attr_done[dev][vidx]) {
            const int e = drv().set_max_dynamic_smem(reinterpret_cast<const void *>(kernel), L::kAlloc);
            if (e != cudaSuccess) return map_cuda_error(e);
            g_attr_done[dev][vidx] = true;
        }
    }
    void *args[4] = {const_cast<CUtensorMap *>(&tq), const_cast<CUtensorMap *>(&tk), const_cast<CUtensorMap *>(&tv),
                     const_cast<FlashParams *>(&p)};
    const int e = drv().launch_kernel(reinterpret_cast<const void *>(kernel), grid, ncz::kThreads, L::kAlloc, stream,
                                      args);
    if (e != cudaSuccess) return map_cuda_error(e);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return NCZ_SUCCESS;
}

template <int D>
int launch_combine(const FlashParams &p, cudaStream_t stream) {
    const long long rows = static_cast<long long>(p.batch_heads) * p.seq_len;
    const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
    void *args[1] = {const_cast<FlashParams *>(&p)};
    const int e = drv().launch_kernel(reinterpret_cast<const void *>(ncz::combine_splits<D>), grid, 256, 0, stream,
                                      args);
    if (e != cudaSuccess) return map_cuda_error(e);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return NCZ_SUCCESS;
}

// Device address of g_ncz_scratch per device (set up by the first
// ncz_flash_fwd_static call on that device, which must be current).
float *g_scratch_addr[kMaxDevices];

int static_scratch(int dev, float **out) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void *addr = nullptr;
        const int e = drv().symbol_address(&addr, static_cast<const void *>(&g_ncz_scratch));
        if (e != cudaSuccess) return map_cuda_error(e);
        g_scratch_addr[dev] = static_cast<float *>(addr);
    }
    *out = g_scratch_addr[dev];
    return NCZ_SUCCESS;
}

// One head_dim: forward variant (producer x input type), then the split-KV merge.
template <int D>
int launch_d(bool tma, bool bf16, const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv,
             const FlashParams &p, unsigned grid, int dev, cudaStream_t stream) {
    int st;
    if (tma) {
        st = bf16 ? launch_variant<D, true, true>(tq, tk, tv, p, grid, dev, stream)
                  : launch_variant<D, true, false>(tq, tk, tv, p, grid, dev, stream);
    } else {
        st = bf16 ? launch_variant<D, false, true>(tq, tk, tv, p, grid, dev, stream)
                  : launch_variant<D, false, false>(tq, tk, tv, p, grid, dev, stream);
    }
    if (st == NCZ_SUCCESS && p.num_splits > 1) st = launch_combine<D>(p, stream);
    return st;
}

// Library-owned stream-ordered memory pool per device for split-KV partials:
// allocations are ordered on the launch stream, so calls on different streams
// never share a workspace, and the pool keeps freed memory for the next call.
void *g_pool[kMaxDevices];
int g_num_sms[kMaxDevices];

int device_pool(int dev, void **pool) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_pool[dev] == nullptr) {
        void *created = nullptr;
        const int e = drv().pool_create(&created, dev, uint64_t(1) << 30);  // keep up to 1 GiB between calls
        if (e != cudaSuccess) return map_cuda_error(e);
        g_pool[dev] = created;
    }
    *pool = g_pool[dev];
    return NCZ_SUCCESS;
}

int device_sms(int dev) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_num_sms[dev] == 0) {
        int n = 0;
        if (drv().sm_count(dev, &n) != cudaSuccess || n <= 0) n = 148;
        g_num_sms[dev] = n;
    }
    return g_num_sms[dev];
}

// Split-KV ranges for a launch.  Automatic: only when the grid fills at most
// half the SMs and the K range is long (>= 2048 keys; each range keeps >= 512).
// A CTA costs about the time of 512-640 keys in fixed set-up and hand-off, and
// the merge is a second launch, so shorter ranges (config 2: 1024 keys) gain
// nothing.
// Split-KV ranges for a launch of bh slices of seq rows on `sms` SMs;
// requested 0 = automatic, 1 = none, n = up to n ranges.
void split_plan(size_t bh, size_t seq, int requested, size_t sms, int *splits, int *per_split) {
    const int n_kv = static_cast<int>((seq + ncz::kBlockN - 1) / ncz::kBlockN);
    const size_t ctas = ((seq + kGroupRows - 1) / kGroupRows) * bh;
    int want = requested;
    if (want == 0) {
        want = 1;
        constexpr int kMinTiles = 2048 / ncz::kBlockN, kRangeTiles = 512 / ncz::kBlockN;
        if (ctas * 2 <= sms && n_kv >= kMinTiles) {
            const int by_sms = static_cast<int>((sms + ctas - 1) / ctas);
            want = std::min(std::min(by_sms, n_kv / kRangeTiles), ncz::kMaxSplits);
        }
    }
    want = std::max(1, std::min(std::min(want, n_kv), ncz::kMaxSplits));
    const int per = (n_kv + want - 1) / want;
    *per_split = per;
    *splits = (n_kv + per - 1) / per;
}

// Groups (of two 128-row Q tiles) of a launch without split-KV whose Q tiles
// run as split-Q items: all of them when the items of two Q tiles number fewer
// than NCZ_QSPLIT_ITEMS_PER_SM per SM, else none.  (Launches with a smaller
// count, counted from the top group, run through ncz_test_set_qsplit_groups.)
int qsplit_plan(size_t bh, size_t seq, size_t sms) {
    const size_t groups = (seq + kGroupRows - 1) / kGroupRows;
    const double items = static_cast<double>(groups * bh);
    return items < (NCZ_QSPLIT_ITEMS_PER_SM) * static_cast<double>(sms) ? static_cast<int>(groups) : 0;
}

// Work items of a launch with `split_groups` split-Q groups (no split-KV).
size_t qsplit_items(size_t bh, size_t seq, int split_groups) {
    const size_t groups = (seq + kGroupRows - 1) / kGroupRows;
    const size_t n_qt = (seq + ncz::kBlockM - 1) / ncz::kBlockM;
    const size_t low = groups - static_cast<size_t>(split_groups);
    return bh * (n_qt - ncz::kQTiles * low + low);
}

void choose_splits(const Resolved &r, int dev, int *splits, int *per_split) {
    split_plan(r.bh, r.seq, r.splits, r.splits == 0 ? static_cast<size_t>(device_sms(dev)) : 0, splits, per_split);
}

// Validated launch on the current device (the caller switched devices).
int launch_on_current(const Resolved &r, int dev) {
    const bool qkv_aligned = aligned(r.q, 16) && aligned(r.k, 16) && aligned(r.v, 16) && r.qs % 8 == 0 &&
                             r.ks % 8 == 0 && r.vs % 8 == 0 && r.qr % 8 == 0 && r.kr % 8 == 0 && r.vr % 8 == 0;
    bool use_tma = r.producer == NCZ_PRODUCER_TMA || (r.producer == NCZ_PRODUCER_AUTO && qkv_aligned);
    if (r.producer == NCZ_PRODUCER_TMA && !qkv_aligned) return NCZ_ERROR_MISALIGNED;

    CUtensorMap tq, tk, tv;
    std::memset(&tq, 0, sizeof(tq));
    std::memset(&tk, 0, sizeof(tk));
    std::memset(&tv, 0, sizeof(tv));
    if (use_tma) {
        const bool bf = r.in_dtype == NCZ_DTYPE_BF16;
        const bool enc = encode_map(&tq, r.q, r.d, r.seq, r.bh, r.qr, r.qs, ncz::kBlockM, bf) &&
                         encode_map(&tk, r.k, r.d, r.seq, r.bh, r.kr, r.ks, ncz::kBlockN, bf) &&
                         encode_map(&tv, r.v, r.d, r.seq, r.bh, r.vr, r.vs, ncz::kBlockN, bf);
        if (!enc) {
            if (r.producer == NCZ_PRODUCER_TMA) return NCZ_ERROR_MISALIGNED;
            use_tma = false;  // e.g. strides the TMA unit cannot express: plain-load producer
        }
    }

    FlashParams p;
    p.q = static_cast<const uint16_t *>(r.q);
    p.k = static_cast<const uint16_t *>(r.k);
    p.v = static_cast<const uint16_t *>(r.v);
    p.o = r.o;
    p.q_stride = static_cast<long long>(r.qs);
    p.k_stride = static_cast<long long>(r.ks);
    p.v_stride = static_cast<long long>(r.vs);
    p.o_stride = static_cast<long long>(r.os);
    p.q_row = static_cast<long long>(r.qr);
    p.k_row = static_cast<long long>(r.kr);
    p.v_row = static_cast<long long>(r.vr);
    p.o_row = static_cast<long long>(r.orow);
    p.seq_len = static_cast<int>(r.seq);
    p.batch_heads = static_cast<int>(r.bh);
    p.num_groups = static_cast<int>((r.seq + kGroupRows - 1) / kGroupRows);
    p.scale_log2 = static_cast<float>(static_cast<double>(r.scale) * 1.4426950408889634);
    p.causal = r.causal != 0;
    p.o_dtype = r.o_dtype == NCZ_DTYPE_F16 ? 1 : (r.o_dtype == NCZ_DTYPE_BF16 ? 2 : 0);
    const size_t vec_elems = p.o_dtype != 0 ? 8 : 4;
    p.o_vec = aligned(r.o, 16) && r.os % vec_elems == 0 && r.orow % vec_elems == 0;
    choose_splits(r, dev, &p.num_splits, &p.kv_per_split);
    if (r.scratch != nullptr) {
        // Fixed scratch: an explicit split count must fit; the automatic choice
        // is lowered to the largest count (down to no split) whose partials fit.
        const size_t per_split = r.bh * r.seq * (r.d + 2);
        const int n_kv = static_cast<int>((r.seq + ncz::kBlockN - 1) / ncz::kBlockN);
        int fit = static_cast<int>(std::min<size_t>(r.scratch_floats / per_split, size_t(ncz::kMaxSplits)));
        // Without a split nothing goes to the scratch, so only a count that
        // does split has to fit (an explicit 1, or one the plan clamps to 1, runs).
        if (p.num_splits > 1 && fit < p.num_splits && r.splits != 0) return NCZ_ERROR_OUT_OF_MEMORY;
        if (fit < p.num_splits) {
            const int want = std::max(1, fit);
            p.kv_per_split = (n_kv + want - 1) / want;
            p.num_splits = (n_kv + p.kv_per_split - 1) / p.kv_per_split;
        }
    }
    p.part_o = nullptr;
    p.part_ml = nullptr;
    void *ws = nullptr;
    if (p.num_splits > 1 && r.scratch != nullptr) {
        const size_t rows = static_cast<size_t>(p.num_splits) * r.bh * r.seq;
        p.part_o = r.scratch;
        p.part_ml = p.part_o + rows * r.d;
    } else if (p.num_splits > 1) {
        const size_t rows = static_cast<size_t>(p.num_splits) * r.bh * r.seq;
        void *pool = nullptr;
        int st = device_pool(dev, &pool);
        if (st != NCZ_SUCCESS) return st;
        const int e = drv().pool_alloc_async(&ws, rows * (r.d + 2) * sizeof(float), pool, r.stream);
        if (e != cudaSuccess) return map_cuda_error(e);
        p.part_o = static_cast<float *>(ws);
        p.part_ml = p.part_o + rows * r.d;
    }
    // Split-Q items (launches without split-KV only): for every group when the
    // items of two Q tiles leave SMs idle, else for the causal groups whose
    // items are longer than an even share of the work (qsplit_plan).
    // Twin items instead for one Q tile per slice (seq_len <= 128): both
    // pipelines busy, half the items (unless a test forces split-Q items).
    p.qsplit_groups = 0;
    p.twin = 0;
    if (p.num_splits == 1) {
        const int mode = g_qsplit_mode.load(std::memory_order_relaxed);
        const int force = g_qsplit_force.load(std::memory_order_relaxed);
        if (force >= 0)
            p.qsplit_groups = std::min(force, p.num_groups);
        else if (mode == 1)
            p.qsplit_groups = p.num_groups;
        else if (r.seq <= static_cast<size_t>(ncz::kBlockM) && g_twin_mode.load(std::memory_order_relaxed) != 0)
            p.twin = 1;
        else if (mode == 0)
            p.qsplit_groups = qsplit_plan(r.bh, r.seq, static_cast<size_t>(device_sms(dev)));
    }
    // One CTA per work item, heaviest first; at most one is resident per SM (TMEM
    // holds one CTA's 512 columns) and it takes over the items of CTAs that have
    // not started yet.
    const size_t items = p.twin ? (r.bh + 1) / 2
                         : p.qsplit_groups > 0
                             ? qsplit_items(r.bh, r.seq, p.qsplit_groups)
                             : static_cast<size_t>(p.num_groups) * r.bh * static_cast<size_t>(p.num_splits);
    const unsigned grid = static_cast<unsigned>(items);
#ifdef NCZ_DEBUG_ITEM_VISITS
    p.item_visits = r.item_visits;
    if (r.items_out != nullptr) *r.items_out = items;
    if (r.item_visits != nullptr && items > r.item_visits_cap) {
        if (ws != nullptr) drv().free_async(ws, r.stream);
        return NCZ_ERROR_OVERFLOW;
    }
#endif
    p.walk_tiles = NCZ_WALK_TILES;
    {
        // NCZ_CHUNK_KV_BYTES of K/V per chunk of slices: with the items in
        // flight spanning at most two chunks, the K/V being read stays in L2.
        const size_t kv_slice = static_cast<size_t>(r.seq) * r.d * 2 * 2;
        const size_t c = std::max<size_t>(1, (NCZ_CHUNK_KV_BYTES) / std::max<size_t>(kv_slice, 1));
        p.chunk_slices = static_cast<int>(std::min<size_t>(c, r.bh));
    }
    const bool bf = r.in_dtype == NCZ_DTYPE_BF16;
    int st;
    switch (r.d) {
        case 16: st = launch_d<16>(use_tma, bf, tq, tk, tv, p, grid, dev, r.stream); break;
        case 32: st = launch_d<32>(use_tma, bf, tq, tk, tv, p, grid, dev, r.stream); break;
        default: st = launch_d<64>(use_tma, bf, tq, tk, tv, p, grid, dev, r.stream); break;
    }
    if (ws != nullptr) {
        const int e = drv().free_async(ws, r.stream);
        if (st == NCZ_SUCCESS && e != cudaSuccess) st = map_cuda_error(e);
    }
    return st;
}

// Switches to r.device when given, launches, restores the caller's device.
int launch_resolved(const Resolved &r) {
    int st = validate_resolved(r);
    if (st != NCZ_SUCCESS) return st;
    st = ncz_init();
    if (st != NCZ_SUCCESS) return st;
    int prev = 0;
    int e = drv().get_device(&prev);
    if (e != cudaSuccess) return map_cuda_error(e);
    const int dev = r.device >= 0 ? r.device : prev;
    if (dev >= kMaxDevices) return NCZ_ERROR_INVALID_DEVICE;
    if (dev != prev) {
        e = drv().set_device(dev);
        if (e != cudaSuccess) return map_cuda_error(e);
    }
    if (r.use_static) {
        Resolved rs = r;
        st = static_scratch(dev, &rs.scratch);
        rs.scratch_floats = kStaticScratchFloats;
        if (st == NCZ_SUCCESS) st = launch_on_current(rs, dev);
    } else {
        st = launch_on_current(r, dev);
    }
    if (dev != prev) drv().set_device(prev);
    return st;
}

Resolved reference_args(const void *q, const void *k, const void *v, void *o, size_t bh, size_t seq, size_t d,
                        size_t qs, size_t ks, size_t vs, size_t os, float scale, uint32_t causal, void *stream) {
    ncz_flash_desc desc;
    std::memset(&desc, 0, sizeof(desc));
    desc.q = q; desc.k = k; desc.v = v; desc.o = o;
    desc.batch_heads = bh; desc.seq_len = seq; desc.head_dim = d;
    desc.q_stride = qs; desc.k_stride = ks; desc.v_stride = vs; desc.o_stride = os;
    desc.scale = scale; desc.causal = causal;
    desc.o_dtype = NCZ_DTYPE_F32; desc.producer = NCZ_PRODUCER_AUTO; desc.device = -1;
    desc.in_dtype = NCZ_DTYPE_F16;
    desc.stream = stream;
    return from_desc(desc);
}

// Kernel names ncz_flash_fwd_named accepts: the reference's exported flash
// kernels (src/main_device.zig:41-47) with the head dimensions each one's
// entry guard lets through (bit 0: 16, bit 1: 32, bit 2: 64) and whether it
// ignores the causal flag, plus this library's own labels.
struct KernelAlias {
    const char *name;
    uint32_t dims;
    bool always_causal;
};
constexpr KernelAlias kAliases[] = {
    {"flash_attention_fwd", 7u, false},             // src/kernels.zig:380-394
    {"flash_attention_fwd_opt", 7u, false},         // src/flash_opt.zig:17-31
    {"flash_attention_fwd_v2", 7u, false},          // src/flash_v2.zig:23-37
    {"flash_attention_fwd_h64", 4u, false},         // src/flash_h64.zig:21-35
    {"flash_attention_fwd_h64_bn32", 4u, false},    // src/flash_h64_bn32.zig:26-40
    {"flash_attention_fwd_h64_causal", 4u, true},   // src/flash_h64_causal.zig:20-35
    {"flash_fwd_sm100a_d16", 1u, false},
    {"flash_fwd_sm100a_d32", 2u, false},
    {"flash_fwd_sm100a_d64", 4u, false},
};

const KernelAlias *find_alias(const char *name) {
    for (const KernelAlias &a : kAliases)
        if (std::strcmp(a.name, name) == 0) return &a;
    return nullptr;
}

// Per-device streams and events of the host-buffer pipeline (library-owned,
// created on first use).  `mu` serialises callers on one device: the events
// are re-recorded per chunk and waited on right away, which is only ordered
// within one caller's enqueue sequence.
struct HostPipe {
    std::mutex mu;
    bool ready = false;
    void *up = nullptr, *down = nullptr;                                       // streams
    void *fork = nullptr, *in_ready = nullptr, *out_ready = nullptr, *join = nullptr;  // events
};
HostPipe g_pipes[kMaxDevices];

// Destroys whatever of the pipe exists (hp.mu held); first error as a status.
int pipe_release(HostPipe &hp) {
    int first = cudaSuccess;
    auto keep = [&first](int e) {
        if (first == cudaSuccess) first = e;
    };
    for (void **ev : {&hp.fork, &hp.in_ready, &hp.out_ready, &hp.join}) {
        if (*ev != nullptr) keep(drv().event_destroy(*ev));
        *ev = nullptr;
    }
    for (void **st : {&hp.up, &hp.down}) {
        if (*st != nullptr) keep(drv().stream_destroy(*st));
        *st = nullptr;
    }
    hp.ready = false;
    return map_cuda_error(first);
}

// Creates the pipe's streams and events; on a failure releases the ones made.
int pipe_setup(HostPipe &hp) {
    if (hp.ready) return NCZ_SUCCESS;
    int e = drv().stream_create(&hp.up);
    if (e == cudaSuccess) e = drv().stream_create(&hp.down);
    void **evs[4] = {&hp.fork, &hp.in_ready, &hp.out_ready, &hp.join};
    for (int i = 0; i < 4 && e == cudaSuccess; ++i) e = drv().event_create(evs[i]);
    if (e != cudaSuccess) {
        pipe_release(hp);
        return map_cuda_error(e);
    }
    hp.ready = true;
    return NCZ_SUCCESS;
}

// Elements the slices [s0, s1) of one operand occupy: whole strides for all but
// the last slice, which ends at its last row's last element.
size_t chunk_elems(size_t s0, size_t s1, size_t slice, size_t row, size_t seq, size_t d) {
    return (s1 - s0 - 1) * slice + (seq - 1) * row + d;
}

// Chunk sizes (slices) covering bh: `chunk` each, or with taper the first and
// last two chunks a quarter and a half of it, so the first forward starts and
// the last download ends sooner (only one PCIe direction is busy then).
std::vector<size_t> chunk_plan(size_t bh, size_t chunk, bool taper) {
    std::vector<size_t> plan;
    const size_t a = std::max<size_t>(1, chunk / 4), b = std::max<size_t>(1, chunk / 2);
    if (taper && chunk >= 4 && bh >= 2 * (a + b) + chunk) {
        plan = {a, b};
        size_t mid = bh - 2 * (a + b);
        while (mid > 0) {
            const size_t c = std::min(chunk, mid);
            plan.push_back(c);
            mid -= c;
        }
        plan.push_back(b);
        plan.push_back(a);
    } else {
        for (size_t s0 = 0; s0 < bh; s0 += chunk) plan.push_back(std::min(chunk, bh - s0));
    }
    return plan;
}

int host_pipeline(const Resolved &r, const void *qh, const void *kh, const void *vh, void *oh, size_t chunk,
                  bool taper, int dev) {
    HostPipe &hp = g_pipes[dev];
    std::lock_guard<std::mutex> lock(hp.mu);
    int st = pipe_setup(hp);
    if (st != NCZ_SUCCESS) return st;
    const size_t osz = r.o_dtype == NCZ_DTYPE_F32 ? 4 : 2;
    int e = drv().event_record(hp.fork, r.stream);
    if (e == cudaSuccess) e = drv().stream_wait_event(hp.up, hp.fork);
    if (e == cudaSuccess) e = drv().stream_wait_event(hp.down, hp.fork);
    if (e != cudaSuccess) return map_cuda_error(e);
    size_t s0 = 0;
    for (const size_t n_slices : chunk_plan(r.bh, chunk, taper)) {
        const size_t s1 = s0 + n_slices;
        struct Op {
            const void *dev;
            const void *host;
            size_t slice, row;
        } in[3] = {{r.q, qh, r.qs, r.qr}, {r.k, kh, r.ks, r.kr}, {r.v, vh, r.vs, r.vr}};
        for (int i = 0; i < 3 && e == cudaSuccess; ++i) {
            const size_t off = s0 * in[i].slice * 2;
            e = drv().memcpy_async(static_cast<char *>(const_cast<void *>(in[i].dev)) + off,
                                   static_cast<const char *>(in[i].host) + off,
                                   chunk_elems(s0, s1, in[i].slice, in[i].row, r.seq, r.d) * 2,
                                   NCZ_COPY_HOST_TO_DEVICE, hp.up);
        }
        if (e == cudaSuccess) e = drv().event_record(hp.in_ready, hp.up);
        if (e == cudaSuccess) e = drv().stream_wait_event(r.stream, hp.in_ready);
        if (e != cudaSuccess) return map_cuda_error(e);
        Resolved rc = r;
        rc.q = static_cast<const char *>(r.q) + s0 * r.qs * 2;
        rc.k = static_cast<const char *>(r.k) + s0 * r.ks * 2;
        rc.v = static_cast<const char *>(r.v) + s0 * r.vs * 2;
        rc.o = static_cast<char *>(r.o) + s0 * r.os * osz;
        rc.bh = s1 - s0;
        st = launch_on_current(rc, dev);
        if (st != NCZ_SUCCESS) return st;
        e = drv().event_record(hp.out_ready, r.stream);
        if (e == cudaSuccess) e = drv().stream_wait_event(hp.down, hp.out_ready);
        if (e == cudaSuccess) {
            const size_t off = s0 * r.os * osz;
            e = drv().memcpy_async(static_cast<char *>(oh) + off, static_cast<const char *>(r.o) + off,
                                   chunk_elems(s0, s1, r.os, r.orow, r.seq, r.d) * osz, NCZ_COPY_DEVICE_TO_HOST,
                                   hp.down);
        }
        if (e != cudaSuccess) return map_cuda_error(e);
        s0 = s1;
    }
    e = drv().event_record(hp.join, hp.down);
    if (e == cudaSuccess) e = drv().stream_wait_event(r.stream, hp.join);
    return e == cudaSuccess ? NCZ_SUCCESS : map_cuda_error(e);
}

// Switches to `device` (-1 = current), runs fn(), switches back.
template <class Fn>
int on_device(int device, Fn fn) {
    int st = ncz_init();
    if (st != NCZ_SUCCESS) return st;
    int prev = 0;
    int e = drv().get_device(&prev);
    if (e != cudaSuccess) return map_cuda_error(e);
    const int dev = device >= 0 ? device : prev;
    if (dev != prev && (e = drv().set_device(dev)) != cudaSuccess) return map_cuda_error(e);
    st = fn();
    if (dev != prev) drv().set_device(prev);
    return st;
}

int write_symbol(int device, const void *symbol, const void *value, size_t bytes) {
    return on_device(device, [&] { return map_cuda_error(drv().symbol_write(symbol, value, bytes)); });
}

}  // namespace

namespace ncz {

int release_flash_objects() {
    int first = NCZ_SUCCESS;
    for (HostPipe &hp : g_pipes) {
        std::lock_guard<std::mutex> lock(hp.mu);
        const int st = pipe_release(hp);
        if (first == NCZ_SUCCESS) first = st;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    for (void *&pool : g_pool) {
        if (pool != nullptr) {
            const int st = map_cuda_error(drv().pool_destroy(pool));
            if (first == NCZ_SUCCESS) first = st;
        }
        pool = nullptr;
    }
    return first;
}

void reset_flash_caches() {
    std::lock_guard<std::mutex> lock(g_mu);
    std::memset(g_attr_done, 0, sizeof(g_attr_done));
    for (MapSlot &m : g_maps) m.used = false;
    std::memset(g_num_sms, 0, sizeof(g_num_sms));
    std::memset(g_scratch_addr, 0, sizeof(g_scratch_addr));
    g_init_done = false;
    g_init_status = NCZ_ERROR_NOT_INITIALIZED;
}

template <int D, bool kTma, bool kBf16>
const void *fwd_kernel() {
    return reinterpret_cast<const void *>(flash_fwd_sm100<D, kTma, kBf16>);
}

template <int D>
const void *combine_kernel() {
    return reinterpret_cast<const void *>(combine_splits<D>);
}

const char *flash_kernel_label(const void *kernel) {
    static const struct {
        const void *fn;
        const char *name;
    } kNames[] = {
        {fwd_kernel<16, true, false>(), "flash_fwd<16,tma,f16>"}, {fwd_kernel<16, true, true>(), "flash_fwd<16,tma,bf16>"},
        {fwd_kernel<16, false, false>(), "flash_fwd<16,lsu,f16>"}, {fwd_kernel<16, false, true>(), "flash_fwd<16,lsu,bf16>"},
        {fwd_kernel<32, true, false>(), "flash_fwd<32,tma,f16>"}, {fwd_kernel<32, true, true>(), "flash_fwd<32,tma,bf16>"},
        {fwd_kernel<32, false, false>(), "flash_fwd<32,lsu,f16>"}, {fwd_kernel<32, false, true>(), "flash_fwd<32,lsu,bf16>"},
        {fwd_kernel<64, true, false>(), "flash_fwd<64,tma,f16>"}, {fwd_kernel<64, true, true>(), "flash_fwd<64,tma,bf16>"},
        {fwd_kernel<64, false, false>(), "flash_fwd<64,lsu,f16>"}, {fwd_kernel<64, false, true>(), "flash_fwd<64,lsu,bf16>"},
        {combine_kernel<16>(), "combine_splits<16>"}, {combine_kernel<32>(), "combine_splits<32>"},
        {combine_kernel<64>(), "combine_splits<64>"},
    };
    for (const auto &k : kNames)
        if (k.fn == kernel) return k.name;
    return nullptr;
}

}  // namespace ncz

extern "C" {

int ncz_init(void) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_init_done && g_init_status == NCZ_SUCCESS) return NCZ_SUCCESS;
    int count = 0;
    const int e = drv().get_device_count(&count);
    if (e != cudaSuccess) {
        g_init_status = map_cuda_error(e);
        return g_init_status;
    }
    if (count <= 0) {
        g_init_status = NCZ_ERROR_NO_DEVICE;
        return g_init_status;
    }
    if (drv().load_tensor_map_encoder() != cudaSuccess) {
        g_init_status = NCZ_ERROR_NOT_FOUND;
        return g_init_status;
    }
    g_init_done = true;
    g_init_status = NCZ_SUCCESS;
    return NCZ_SUCCESS;
}

int ncz_shutdown(void) {
    const int released = ncz::release_flash_objects();
    ncz::reset_flash_caches();
    ncz::reset_mma_caches();
    return released;
}

int ncz_flash_validate(size_t batch_heads, size_t seq_len, size_t head_dim, size_t q_stride, size_t k_stride,
                       size_t v_stride, size_t o_stride) {
    // Exactly src/flash.zig:16-28.
    if (batch_heads == 0 || seq_len == 0) return NCZ_ERROR_INVALID_VALUE;
    if (head_dim != 16 && head_dim != 32 && head_dim != 64) return NCZ_ERROR_INVALID_VALUE;
    size_t min_stride;
    if (!mul_ok(seq_len, head_dim, &min_stride)) return NCZ_ERROR_OVERFLOW;
    if (q_stride < min_stride || k_stride < min_stride || v_stride < min_stride || o_stride < min_stride)
        return NCZ_ERROR_INVALID_VALUE;
    return NCZ_SUCCESS;
}

int ncz_flash_validate_ex(const ncz_flash_desc *desc) {
    if (desc == nullptr) return NCZ_ERROR_INVALID_VALUE;
    return validate_resolved(from_desc(*desc));
}

int ncz_flash_select(size_t batch_heads, size_t seq_len, size_t head_dim, uint32_t causal, char *label, size_t cap,
                     uint32_t *threads) {
    (void)causal;
    if (batch_heads == 0 || seq_len == 0) return NCZ_ERROR_INVALID_VALUE;
    if (head_dim != 16 && head_dim != 32 && head_dim != 64) return NCZ_ERROR_INVALID_VALUE;
    if (label != nullptr && cap > 0) {
        const char *name = head_dim == 64 ? "flash_fwd_sm100a_d64" : head_dim == 32 ? "flash_fwd_sm100a_d32"
                                                                                    : "flash_fwd_sm100a_d16";
        std::strncpy(label, name, cap - 1);
        label[cap - 1] = '\0';
    }
    if (threads != nullptr) *threads = ncz::kThreads;
    return NCZ_SUCCESS;
}

int ncz_flash_fwd(const void *q, const void *k, const void *v, void *o, size_t batch_heads, size_t seq_len,
                  size_t head_dim, size_t q_stride, size_t k_stride, size_t v_stride, size_t o_stride, float scale,
                  uint32_t causal, void *stream) {
    const int st = ncz_flash_validate(batch_heads, seq_len, head_dim, q_stride, k_stride, v_stride, o_stride);
    if (st != NCZ_SUCCESS) return st;
    return launch_resolved(reference_args(q, k, v, o, batch_heads, seq_len, head_dim, q_stride, k_stride, v_stride,
                                          o_stride, scale, causal, stream));
}

int ncz_flash_kernel_info(const char *kernel, uint32_t *head_dims, uint32_t *always_causal) {
    if (kernel == nullptr) return NCZ_ERROR_INVALID_VALUE;
    const KernelAlias *a = find_alias(kernel);
    if (a == nullptr) return NCZ_ERROR_NOT_FOUND;
    if (head_dims != nullptr) *head_dims = a->dims;
    if (always_causal != nullptr) *always_causal = a->always_causal ? 1u : 0u;
    return NCZ_SUCCESS;
}

int ncz_flash_fwd_named(const char *kernel, const void *q, const void *k, const void *v, void *o,
                        size_t batch_heads, size_t seq_len, size_t head_dim, size_t q_stride, size_t k_stride,
                        size_t v_stride, size_t o_stride, float scale, uint32_t causal, void *stream) {
    if (kernel == nullptr) return NCZ_ERROR_INVALID_VALUE;
    const KernelAlias *a = find_alias(kernel);
    if (a == nullptr) return NCZ_ERROR_NOT_FOUND;
    if (batch_heads == 0) return NCZ_ERROR_INVALID_VALUE;
    const uint32_t bit = head_dim == 16 ? 1u : head_dim == 32 ? 2u : head_dim == 64 ? 4u : 0u;
    if (seq_len == 0 || (a->dims & bit) == 0) return NCZ_SUCCESS;  // the kernel's entry guard returns
    return ncz_flash_fwd(q, k, v, o, batch_heads, seq_len, head_dim, q_stride, k_stride, v_stride, o_stride, scale,
                         a->always_causal ? 1u : causal, stream);
}

int ncz_flash_launch(const void *q, size_t q_len, const void *k, size_t k_len, const void *v, size_t v_len, void *o,
                     size_t o_len, size_t batch_heads, size_t seq_len, size_t head_dim, size_t q_stride,
                     size_t k_stride, size_t v_stride, size_t o_stride, float scale, uint32_t causal, void *stream) {
    int st = ncz_flash_validate(batch_heads, seq_len, head_dim, q_stride, k_stride, v_stride, o_stride);
    if (st != NCZ_SUCCESS) return st;
    // requireLen (src/flash.zig:40-43, :98-100): len >= batch_heads * stride.
    const size_t lens[4] = {q_len, k_len, v_len, o_len};
    const size_t strides[4] = {q_stride, k_stride, v_stride, o_stride};
    for (int i = 0; i < 4; ++i) {
        size_t need;
        if (!mul_ok(batch_heads, strides[i], &need)) return NCZ_ERROR_OVERFLOW;
        if (lens[i] < need) return NCZ_ERROR_INVALID_VALUE;
    }
    return launch_resolved(reference_args(q, k, v, o, batch_heads, seq_len, head_dim, q_stride, k_stride, v_stride,
                                          o_stride, scale, causal, stream));
}

int ncz_flash_fwd_ex(const ncz_flash_desc *desc) {
    if (desc == nullptr) return NCZ_ERROR_INVALID_VALUE;
    return launch_resolved(from_desc(*desc));
}

int ncz_flash_fwd_splits(const ncz_flash_desc *desc, int splits) {
    if (desc == nullptr || splits < 0) return NCZ_ERROR_INVALID_VALUE;
    Resolved r = from_desc(*desc);
    r.splits = splits;
    return launch_resolved(r);
}

int ncz_flash_fwd_static(const ncz_flash_desc *desc, int splits) {
    if (desc == nullptr || splits < 0) return NCZ_ERROR_INVALID_VALUE;
    Resolved r = from_desc(*desc);
    r.splits = splits;
    r.use_static = true;
    return launch_resolved(r);
}

int ncz_flash_fwd_multi(const ncz_flash_desc *descs, int count) {
    if (descs == nullptr || count <= 0) return NCZ_ERROR_INVALID_VALUE;
    for (int i = 0; i < count; ++i) {
        const int st = validate_resolved(from_desc(descs[i]));
        if (st != NCZ_SUCCESS) return st;
    }
    for (int i = 0; i < count; ++i) {
        const int st = launch_resolved(from_desc(descs[i]));
        if (st != NCZ_SUCCESS) return st;
    }
    return NCZ_SUCCESS;
}

int ncz_flash_fwd_host(const ncz_flash_desc *desc, const void *q_host, const void *k_host, const void *v_host,
                       void *o_host, size_t chunk_slices) {
    if (desc == nullptr || q_host == nullptr || k_host == nullptr || v_host == nullptr || o_host == nullptr)
        return NCZ_ERROR_INVALID_VALUE;
    const Resolved r = from_desc(*desc);
    int st = validate_resolved(r);
    if (st != NCZ_SUCCESS) return st;
    st = ncz_init();
    if (st != NCZ_SUCCESS) return st;
    int prev = 0;
    int e = drv().get_device(&prev);
    if (e != cudaSuccess) return map_cuda_error(e);
    const int dev = r.device >= 0 ? r.device : prev;
    if (dev >= kMaxDevices) return NCZ_ERROR_INVALID_DEVICE;
    if (dev != prev) {
        e = drv().set_device(dev);
        if (e != cudaSuccess) return map_cuda_error(e);
    }
    // Default: 8 chunks, so one chunk's upload hides the previous chunk's forward,
    // but at least 4 MiB of Q/K/V per chunk (smaller copies cost more than they
    // hide), with tapered first and last chunks.
    size_t chunk = chunk_slices;
    if (chunk == 0) {
        const size_t slice_bytes = (r.qs + r.ks + r.vs) * 2;
        const size_t min_slices = ((size_t(4) << 20) + slice_bytes - 1) / slice_bytes;
        chunk = std::max((r.bh + 7) / 8, min_slices);
    }
    st = host_pipeline(r, q_host, k_host, v_host, o_host, chunk, chunk_slices == 0, dev);
    if (dev != prev) drv().set_device(prev);
    return st;
}

int ncz_flash_sync_status(int device, void *stream, uint32_t *detail) {
    if (detail != nullptr) *detail = 0;
    uint32_t word = 0;
    const int st = on_device(device, [&] {
        const void *sym = static_cast<const void *>(&ncz::g_ncz_status);
        int e = drv().stream_synchronize(stream);
        if (e == cudaSuccess) e = drv().symbol_read(&word, sym, sizeof(word));
        if (e == cudaSuccess && word != 0) {
            const uint32_t zero = 0;
            e = drv().symbol_write(sym, &zero, sizeof(zero));
        }
        return map_cuda_error(e);
    });
    if (st != NCZ_SUCCESS) return st;
    if (detail != nullptr) *detail = word;
    return word != 0 ? NCZ_ERROR_DEVICE_TIMEOUT : NCZ_SUCCESS;
}

int ncz_test_split_plan(size_t batch_heads, size_t seq_len, int requested, size_t sms, int32_t *out) {
    if (out == nullptr || batch_heads == 0 || seq_len == 0 || requested < 0 || sms == 0) return NCZ_ERROR_INVALID_VALUE;
    int splits = 0, per = 0;
    split_plan(batch_heads, seq_len, requested, sms, &splits, &per);
    out[0] = splits;
    out[1] = per;
    return NCZ_SUCCESS;
}

int ncz_test_chunk_plan(size_t batch_heads, size_t chunk_slices, int taper, size_t *out, size_t cap, size_t *count) {
    if (out == nullptr || count == nullptr || batch_heads == 0 || chunk_slices == 0) return NCZ_ERROR_INVALID_VALUE;
    const std::vector<size_t> plan = chunk_plan(batch_heads, chunk_slices, taper != 0);
    *count = plan.size();
    if (plan.size() > cap) return NCZ_ERROR_OVERFLOW;
    std::copy(plan.begin(), plan.end(), out);
    return NCZ_SUCCESS;
}

int ncz_test_item_work(size_t batch_heads, size_t seq_len, uint32_t causal, int splits, int chunk_slices, int item,
                       int32_t *out) {
    if (out == nullptr || batch_heads == 0 || seq_len == 0 || splits < 1 || chunk_slices < 1 || item < 0 ||
        seq_len > (size_t(1) << 30) || batch_heads > (size_t(1) << 20))
        return NCZ_ERROR_INVALID_VALUE;
    FlashParams p{};
    p.batch_heads = static_cast<int>(batch_heads);
    p.seq_len = static_cast<int>(seq_len);
    p.causal = causal != 0;
    p.num_groups = static_cast<int>((seq_len + kGroupRows - 1) / kGroupRows);
    const int n_kv = static_cast<int>((seq_len + ncz::kBlockN - 1) / ncz::kBlockN);
    const int want = std::min(splits, n_kv);
    p.kv_per_split = (n_kv + want - 1) / want;  // as choose_splits
    p.num_splits = (n_kv + p.kv_per_split - 1) / p.kv_per_split;
    p.chunk_slices = static_cast<int>(std::min<size_t>(static_cast<size_t>(chunk_slices), batch_heads));
    const long long items = static_cast<long long>(p.num_groups) * p.batch_heads * p.num_splits;
    if (item >= items) return NCZ_ERROR_INVALID_VALUE;
    const ncz::Work wk = ncz::make_work(p, item);
    const int32_t vals[8] = {wk.slice, wk.q_base, wk.split, wk.kv0, wk.n[0], wk.n[1], wk.n_max, p.num_splits};
    std::memcpy(out, vals, sizeof(vals));
    return NCZ_SUCCESS;
}

int ncz_test_set_qsplit(int mode) {
    if (mode < 0 || mode > 2) return NCZ_ERROR_INVALID_VALUE;
    g_qsplit_mode.store(mode, std::memory_order_relaxed);
    return NCZ_SUCCESS;
}

int ncz_test_tile_shape(int32_t *out) {
    if (out == nullptr) return NCZ_ERROR_INVALID_VALUE;
    out[0] = ncz::kBlockM;
    out[1] = ncz::kBlockN;
    return NCZ_SUCCESS;
}

int ncz_test_set_twin(int enable) {
    if (enable != 0 && enable != 1) return NCZ_ERROR_INVALID_VALUE;
    g_twin_mode.store(enable, std::memory_order_relaxed);
    return NCZ_SUCCESS;
}

int ncz_test_twin_work(size_t batch_heads, size_t seq_len, uint32_t causal, int item, int32_t *out) {
    if (out == nullptr || batch_heads == 0 || seq_len == 0 || seq_len > static_cast<size_t>(ncz::kBlockM) ||
        item < 0 || batch_heads > (size_t(1) << 20))
        return NCZ_ERROR_INVALID_VALUE;
    if (static_cast<size_t>(item) >= (batch_heads + 1) / 2) return NCZ_ERROR_INVALID_VALUE;
    FlashParams p{};
    p.batch_heads = static_cast<int>(batch_heads);
    p.seq_len = static_cast<int>(seq_len);
    p.causal = causal != 0;
    p.num_groups = 1;
    p.num_splits = 1;
    p.kv_per_split = 1;
    p.chunk_slices = 1;
    p.twin = 1;
    const ncz::Work wk = ncz::make_work(p, item);
    out[0] = ncz::slot_slice(wk, 0);
    out[1] = wk.n[1] > 0 ? ncz::slot_slice(wk, 1) : -1;
    out[2] = wk.n[0];
    out[3] = wk.n[1];
    out[4] = wk.n_max;
    out[5] = ncz::ring_slice(wk, 0);
    out[6] = wk.n_max > 1 ? ncz::ring_slice(wk, 1) : -1;
    out[7] = wk.kind;
    return NCZ_SUCCESS;
}

int ncz_test_set_qsplit_groups(int groups) {
    if (groups < -1) return NCZ_ERROR_INVALID_VALUE;
    g_qsplit_force.store(groups, std::memory_order_relaxed);
    return NCZ_SUCCESS;
}

int ncz_test_qsplit_work(size_t batch_heads, size_t seq_len, uint32_t causal, int chunk_slices, int split_groups,
                         int item, int32_t *out) {
    if (out == nullptr || batch_heads == 0 || seq_len == 0 || chunk_slices < 1 || item < 0 ||
        seq_len > (size_t(1) << 30) || batch_heads > (size_t(1) << 20))
        return NCZ_ERROR_INVALID_VALUE;
    FlashParams p{};
    p.batch_heads = static_cast<int>(batch_heads);
    p.seq_len = static_cast<int>(seq_len);
    p.causal = causal != 0;
    p.num_groups = static_cast<int>((seq_len + kGroupRows - 1) / kGroupRows);
    if (split_groups < 1 || split_groups > p.num_groups) return NCZ_ERROR_INVALID_VALUE;
    p.num_splits = 1;
    p.kv_per_split = static_cast<int>((seq_len + ncz::kBlockN - 1) / ncz::kBlockN);
    p.chunk_slices = static_cast<int>(std::min<size_t>(static_cast<size_t>(chunk_slices), batch_heads));
    p.qsplit_groups = split_groups;
    if (static_cast<size_t>(item) >= qsplit_items(batch_heads, seq_len, split_groups)) return NCZ_ERROR_INVALID_VALUE;
    const ncz::Work wk = ncz::make_work(p, item);
    const int32_t vals[6] = {wk.slice, wk.q_base, wk.n[0], wk.n[1], wk.n_max, wk.kstride};
    std::memcpy(out, vals, sizeof(vals));
    return NCZ_SUCCESS;
}

int ncz_test_qsplit_plan(size_t batch_heads, size_t seq_len, size_t sms, int32_t *out) {
    if (out == nullptr || batch_heads == 0 || seq_len == 0 || sms == 0) return NCZ_ERROR_INVALID_VALUE;
    out[0] = qsplit_plan(batch_heads, seq_len, sms);
    out[1] = out[0] > 0 ? static_cast<int32_t>(qsplit_items(batch_heads, seq_len, out[0]))
                        : static_cast<int32_t>(((seq_len + kGroupRows - 1) / kGroupRows) * batch_heads);
    return NCZ_SUCCESS;
}

int ncz_test_set_wait_limit(int device, uint64_t cycles) {
    const unsigned long long v = cycles != 0 ? cycles : ncz::kWaitLimitCycles;
    return write_symbol(device, static_cast<const void *>(&ncz::g_ncz_wait_limit), &v, sizeof(v));
}

int ncz_test_drop_arrive(int device, int enable) {
    const int v = enable != 0;
    return write_symbol(device, static_cast<const void *>(&ncz::g_ncz_test_drop), &v, sizeof(v));
}

#ifdef NCZ_DEBUG_ITEM_VISITS
// Debug build only (libncz_flash_debug.so, not part of the public headers):
// ncz_flash_fwd_splits with a per-item visit counter.  visits is a device
// array of at least `cap` zeroed uint32 counters; after the launch entry i
// holds the number of CTAs that started work item i (1 for a correct walk).
// *items receives the launch's item count; NCZ_ERROR_OVERFLOW (nothing
// launched) when it exceeds cap.
int ncz_debug_item_visits(const ncz_flash_desc *desc, int splits, unsigned int *visits, size_t cap, size_t *items) {
    if (desc == nullptr || splits < 0 || visits == nullptr || items == nullptr) return NCZ_ERROR_INVALID_VALUE;
    Resolved r = from_desc(*desc);
    r.splits = splits;
    r.item_visits = visits;
    r.item_visits_cap = cap;
    r.items_out = items;
    return launch_resolved(r);
}
#endif

const char *ncz_status_string(int status) {
    switch (status) {
        case NCZ_SUCCESS: return "Success";
        case NCZ_ERROR_OUT_OF_MEMORY: return "OutOfMemory";
        case NCZ_ERROR_OVERFLOW: return "Overflow";
        case NCZ_ERROR_SHARED_OBJECT_INIT_FAILED: return "SharedObjectInitFailed";
        case NCZ_ERROR_NOT_FOUND: return "NotFound";
        case NCZ_ERROR_INVALID_VALUE: return "InvalidValue";
        case NCZ_ERROR_INVALID_CONTEXT: return "InvalidContext";
        case NCZ_ERROR_INVALID_DEVICE: return "InvalidDevice";
        case NCZ_ERROR_INVALID_IMAGE: return "InvalidImage";
        case NCZ_ERROR_CONTEXT_IS_DESTROYED: return "ContextIsDestroyed";
        case NCZ_ERROR_LAUNCH_FAILED: return "LaunchFailed";
        case NCZ_ERROR_LAUNCH_OUT_OF_RESOURCES: return "LaunchOutOfResources";
        case NCZ_ERROR_LAUNCH_TIMEOUT: return "LaunchTimeout";
        case NCZ_ERROR_ILLEGAL_ADDRESS: return "IllegalAddress";
        case NCZ_ERROR_NO_DEVICE: return "NoDevice";
        case NCZ_ERROR_NOT_INITIALIZED: return "NotInitialized";
        case NCZ_ERROR_UNKNOWN: return "UnknownError";
        case NCZ_ERROR_DEVICE_TIMEOUT: return "DeviceTimeout";
        case NCZ_ERROR_MISALIGNED: return "Misaligned";
        default: return "UnknownStatus";
    }
}

uint64_t ncz_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

uint64_t ncz_umma_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout_type) {
    return ncz::umma_smem_desc(smem_addr, lbo_bytes, sbo_bytes, layout_type);
}

uint32_t ncz_umma_instr_desc_bf16(uint32_t m, uint32_t n, uint32_t a_major, uint32_t b_major) {
    return ncz::umma_idesc_f16_f32(m, n, a_major, b_major, 1u);
}

uint32_t ncz_umma_instr_desc_f16(uint32_t m, uint32_t n, uint32_t a_major, uint32_t b_major) {
    return ncz::umma_idesc_f16_f32(m, n, a_major, b_major);
}

uint32_t ncz_tma_swizzle_offset(uint32_t span_bytes, uint32_t offset) {
    if (span_bytes != 32 && span_bytes != 64 && span_bytes != 128) return offset;
    return ncz::tma_swizzle(span_bytes, offset);
}

}  // extern "C"
