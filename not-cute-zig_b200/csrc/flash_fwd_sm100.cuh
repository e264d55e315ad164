// flash_fwd_sm100.cuh -- the sm_100a flash-attention forward kernel.
//
// Replaces the reference's sm_80 kernel family flash_attention_fwd_{opt,v2,
// h64,h64_bn32,h64_causal} (src/flash_opt.zig, src/flash_v2.zig,
// src/flash_h64.zig, src/flash_h64_bn32.zig, src/flash_h64_causal.zig) with one
// warp-specialised kernel, templated on head_dim (16/32/64) and on how tiles
// reach shared memory (TMA, or plain loads for misaligned strides).
//
// Work item: (batch x head slice, pair of 128-row Q tiles[, K range under
// split-KV]); Q tile w covers rows q_base + 128 w .. + 127.  Items are ordered
// in chunks of slices whose K/V fits in L2, heaviest Q-tile group first inside
// a chunk (make_work).  The grid has one CTA per item, but a running CTA takes
// further items from CTAs that have not started, through cluster launch
// control (asked for at the current item's last K/V tile), so one CTA per SM
// keeps pulling items in launch order.  Every role keeps running counters
// across items: the next item's Q (double-buffered), K/V (a kStages-deep ring
// of 128-key tiles shared by both Q tiles) and first scores are fetched while
// the current item's last tiles and epilogue run.
//
// Two pipelines w = 0, 1 (an MMA warp, a softmax warpgroup, a TMEM quarter)
// each take one Q tile per item: pipeline w takes Q tile w ^ (item count & 1).
// Under causal masking Q tile 0 of an item has one K tile fewer than Q tile 1;
// alternating keeps either pipeline from gaining a tile per item on the other
// until the shared K/V ring stalls it.
//
// Warp roles (384 threads):
//   warp 0       producer: TMA or LSU loads of Q, K, V
//   warp 1       TMEM allocator + tcgen05 MMA issuer for pipeline 0
//   warp 2       tcgen05 MMA issuer for pipeline 1
//   (all run as whole warps; elect.sync picks the lane that issues)
//   warp 3       idle (keeps the softmax warpgroups warpgroup-aligned)
//   warpgroup 1+w softmax for pipeline w (thread = row = TMEM lane)
//
// TMEM (512 columns): per pipeline w the scores S_w (128 cols f32, QK^T,
// M=128 N=128), the probabilities P_w (128 f16 keys = 64 cols, the A operand
// of PV read from TMEM) and O_w (D <= 64 cols f32, PV, M=128 N=D).  The
// softmax releases S_w as soon as the scores are in registers, so MMA warp w
// issues QK_w(j+1) while the softmax is still exponentiating tile j; PV_w(j)
// follows once P_w(j) is stored.  Each pipeline has its own MMA warp, so
// neither pipeline's hand-offs wait behind the other's.
//
// Online softmax (reference: src/flash_h64_bn32.zig:139-211) keeps the
// exponent base m (log2 domain) and the row sum l in registers; O is
// rescaled in TMEM only when the row max grows by more than 2^8 since the
// last rescale (P <= 2^8 then still fits f16, and O / l is unchanged).
//
// Every mbarrier wait is bounded (g_ncz_wait_limit cycles).  On expiry the waiter
// records where it gave up in g_ncz_status, raises a CTA-wide abort flag and
// all roles leave their loops; issued copies and MMAs are waited for
// (bounded) before TMEM is freed and the CTA exits.  No trap, no assert.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "sm100_ptx.cuh"

namespace ncz {

constexpr int kBlockM = 128;  // rows per Q tile = TMEM lanes
constexpr int kBlockN = 128;  // keys per K/V tile
constexpr int kQTiles = 2;    // Q tiles per CTA
constexpr int kThreads = 128 * (1 + kQTiles);
// Launch-control response ring (next work items) and the warps that read each
// response: the producer, the MMA warps and the softmax warps.
constexpr int kClcSlots = 4;
// The producer asks for the next item once it has a ring slot for the item's
// kClcLead-th last K/V tile: late enough that a CTA does not hold on to an
// item it will start only much later (which stretched the end of a launch
// whose last items differ in size), early enough that the answer is back
// before the next item's loads are due.
#ifndef NCZ_CLC_LEAD
#define NCZ_CLC_LEAD 1
#endif
constexpr int kClcLead = NCZ_CLC_LEAD;
constexpr uint32_t kClcReaders = 1 + kQTiles + 4 * kQTiles;
constexpr uint32_t kTmemCols = 512;
// TMEM column map per Q tile w (base kTileCols * w): S | P | O
constexpr uint32_t kColP = kBlockN;               // f16 pairs: kBlockN / 2 columns
constexpr uint32_t kColO = kColP + kBlockN / 2;
constexpr uint32_t kTileCols = kColO + 64;
static_assert(kQTiles * kTileCols <= kTmemCols, "TMEM budget");
constexpr float kRescaleThreshold = 8.0f;                   // log2 units
constexpr float kMaxP = 256.0f;                             // 2^kRescaleThreshold
// Default spin-wait bound in SM cycles (about 2 s at 2 GHz; longer at lower clocks).
constexpr unsigned long long kWaitLimitCycles = 4000000000ull;
// Exponentials: in every group of kExp2EmuPeriod column pairs, the last
// kExp2EmuCount pairs are computed by a polynomial on the FMA pipe instead of
// the MUFU unit.  Off by default: measured slower than MUFU-only here.
#ifndef NCZ_EXP2_EMU_PERIOD
#define NCZ_EXP2_EMU_PERIOD 8
#endif
#ifndef NCZ_EXP2_EMU_COUNT
#define NCZ_EXP2_EMU_COUNT 0
#endif
#ifndef NCZ_EXP2_EMU_DEGREE
#define NCZ_EXP2_EMU_DEGREE 4
#endif
constexpr int kExp2EmuPeriod = NCZ_EXP2_EMU_PERIOD;
constexpr int kExp2EmuCount = NCZ_EXP2_EMU_COUNT;
constexpr int kExp2EmuDegree = NCZ_EXP2_EMU_DEGREE;  // polynomial degree: 3 or 4

// where a bounded wait gave up (bits 24..30 of the status word)
enum WaitSite : uint32_t {
    kSiteQFull = 1,
    kSiteKFull = 2,
    kSiteVFull = 3,
    kSiteKvEmpty = 4,
    kSiteSFull = 5,
    kSiteSFree = 6,
    kSitePFull = 7,
    kSiteODone = 8,
    kSiteMmaDrain = 9,
    kSiteProducerDrain = 10,
    kSiteQEmpty = 11,
    kSiteOFree = 13,
    kSiteClcFull = 14,
    kSiteClcEmpty = 15,
    kSiteMergeReady = 16,
    kSiteMergeDone = 17,
};

struct FlashParams {
    const uint16_t *q;
    const uint16_t *k;
    const uint16_t *v;
    void *o;
    long long q_stride, k_stride, v_stride, o_stride;  // per slice, elements
    long long q_row, k_row, v_row, o_row;              // per row, elements
    int seq_len;
    int batch_heads;
    int num_groups;    // ceil(seq_len / 256)
    float scale_log2;  // scale * log2(e)
    int causal;
    int o_dtype;  // 0 f32, 1 f16, 2 bf16
    int o_vec;  // 16-byte vector stores of O are aligned
    // Split-KV: num_splits > 1 splits each Q group's K tiles into ranges of
    // kv_per_split tiles, one CTA per range; CTAs then write unnormalised partial
    // O rows to part_o [split][slice][row][D] and (base m, sum l) pairs to
    // part_ml [split][slice][row][2] for combine_splits.  1 = direct output.
    int num_splits;
    int kv_per_split;
    // A CTA takes a further item (launch control) only while its current item
    // has fewer than walk_tiles K tiles; heavier items end their CTA.
    int walk_tiles;
    // Items run in chunks of chunk_slices slices (all of a chunk's groups,
    // heaviest first, before the next chunk), so the K/V a chunk reads stays in
    // L2 while its groups pass over it.
    int chunk_slices;
    // Split-Q items: an item is one 128-row Q tile, whose K tiles alternate
    // between the two pipelines (the even ones to one, the odd ones to the
    // other); the two online-softmax states merge in the CTA at the epilogue.
    // The Q tiles of the top qsplit_groups Q-tile groups (the heaviest under
    // causal masking; all groups when it equals num_groups) run as split-Q
    // items, the other groups as items of two Q tiles.  0 = none.
    int qsplit_groups;
    // seq_len <= 128 (one Q tile per slice), no split-KV, no split-Q: twin
    // items of two slices each, one per pipeline.  0 = items of one slice.
    int twin;
    float *part_o;
    float *part_ml;
#ifdef NCZ_DEBUG_ITEM_VISITS
    // Debug build only (libncz_flash_debug.so): when set, item_visits[item]
    // counts the CTAs whose producer started that work item; a correct walk
    // leaves exactly 1 in every entry.
    unsigned int *item_visits;
#endif
};

// Debug build only: one count per work item started (producer warp, lane 0).
__device__ __forceinline__ void count_item_visit(const FlashParams &p, int item, int lane) {
#ifdef NCZ_DEBUG_ITEM_VISITS
    if (lane == 0 && p.item_visits != nullptr) atomicAdd(p.item_visits + item, 1u);
#else
    (void)p;
    (void)item;
    (void)lane;
#endif
}

template <int D>
struct SmemLayout {
    static constexpr int kSpan = 2 * D;              // bytes per row = swizzle width
    static constexpr int kQTile = kBlockM * kSpan;   // one 128-row Q tile
    static constexpr int kKvTile = kBlockN * kSpan;  // one K or V tile
    // K/V ring: 128 KB at d=64, 64 KB below, at most 8 stages
    static constexpr int kStagesRaw = (D == 64 ? 128 * 1024 : 64 * 1024) / (2 * kKvTile);
    static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
    static constexpr uint32_t kUmmaLayout = D == 64 ? 2u : (D == 32 ? 4u : 6u);
    static constexpr int kQSlot = kQTiles * kQTile;  // Q of one item; two slots
    static constexpr int kOffQ = 0;
    static constexpr int kOffK = kOffQ + 2 * kQSlot;
    static constexpr int kOffV = kOffK + kStages * kKvTile;
    static constexpr int kOffBar = kOffV + kStages * kKvTile;
    // barriers: q_full[2] | q_empty[2] | k_full[S] | v_full[S] | kv_empty[S] | s_full[Q] | s_free[Q]
    //           | p_full[Q] | o_done[Q] | o_free[Q] | drain[Q] | clc_full[C] | clc_empty[C]
    static constexpr int kBarQFull = 0;
    static constexpr int kBarQEmpty = 2;
    static constexpr int kBarKFull = 4;
    static constexpr int kBarVFull = kBarKFull + kStages;
    static constexpr int kBarKvEmpty = kBarVFull + kStages;
    static constexpr int kBarSFull = kBarKvEmpty + kStages;
    static constexpr int kBarSFree = kBarSFull + kQTiles;
    static constexpr int kBarPFull = kBarSFree + kQTiles;
    static constexpr int kBarODone = kBarPFull + kQTiles;
    static constexpr int kBarOFree = kBarODone + kQTiles;
    static constexpr int kBarDrain = kBarOFree + kQTiles;  // one per MMA warp
    static constexpr int kBarClcFull = kBarDrain + kQTiles;
    static constexpr int kBarClcEmpty = kBarClcFull + kClcSlots;
    // split-Q epilogue hand-off per SM sub-partition (the two softmax warps of
    // the same 32 rows): merge_ready[4] (the helper's state is in place),
    // merge_done[4] (the writer has read it)
    static constexpr int kBarMergeReady = kBarClcEmpty + kClcSlots;
    static constexpr int kBarMergeDone = kBarMergeReady + 4;
    static constexpr int kNumBars = kBarMergeDone + 4;
    static constexpr int kOffClc = (kOffBar + kNumBars * 8 + 15) / 16 * 16;  // 16-byte launch-control responses
    static constexpr int kOffTmemSlot = kOffClc + 16 * kClcSlots;
    static constexpr int kOffAbort = kOffTmemSlot + 4;
    static constexpr int kOffStash = kOffAbort + 4;  // per warp: item walk state (2 ints)
    static constexpr int kOffMerge = (kOffStash + 8 * (kThreads / 32) + 15) / 16 * 16;  // [4][32] (m, l) pairs
    static constexpr int kBytes = kOffMerge + 4 * 32 * 8;
    static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
    static_assert(kStages >= 2, "K/V ring");
    static_assert(kAlloc <= 227 * 1024, "shared memory");
};

// An item as seen by its two pipeline slots p = 0, 1 (pipeline w takes slot
// w ^ (item count & 1)), in one of three kinds:
// - kPairItem: slot p is Q tile p of the item (rows q_base + 128 p ..),
//   visiting K tiles kv0, kv0 + 1, ...;
// - kSplitQItem: both slots share Q tile 0 (rows q_base ..) and slot p visits
//   K tiles p, p + 2, p + 4, ... (kstride 2);
// - kTwinItem (slices of one Q tile, seq_len <= 128): slot p is slice
//   slice + p in Q tile p, visiting its own K tiles 0, 1, ...; the item's ring
//   tiles alternate between the two slices (kstride 2).
// In every kind slot p's j-th K tile is ring tile j * kstride + p *
// (kstride - 1) of the item, and the item streams n_max ring tiles in order.
constexpr int kPairItem = 0, kSplitQItem = 1, kTwinItem = 2;
struct Work {
    int slice;
    int q_base;
    int split;
    int kv0;            // first K tile of this CTA's range
    int n[kQTiles];     // K/V tiles slot p visits (0 = none)
    int diag[kQTiles];  // last K tile slot p's rows see at all (the only one with masked keys)
    int n_max;          // K/V ring tiles of the item
    int kstride;        // 1, or 2 for a split-Q or twin item
    int kind;
};

// Shared-memory Q tile of slot p.
__host__ __device__ __forceinline__ int slot_qtile(const Work &wk, int slot) {
    return wk.kind == kSplitQItem ? 0 : slot;
}
// Q tile `tile` (0 or 1) of the item is loaded: some slot reads it.
__host__ __device__ __forceinline__ bool q_tile_used(const Work &wk, int tile) {
    return wk.kind == kSplitQItem ? (tile == 0 && wk.n[0] > 0) : wk.n[tile] > 0;
}
__host__ __device__ __forceinline__ int slot_koff(const Work &wk, int slot) { return wk.kstride == 2 ? slot : 0; }
// Slice of slot p's rows, and their first row in it.
__host__ __device__ __forceinline__ int slot_slice(const Work &wk, int slot) {
    return wk.kind == kTwinItem ? wk.slice + slot : wk.slice;
}
__host__ __device__ __forceinline__ int slot_row0(const Work &wk, int slot) {
    return wk.kind == kPairItem ? wk.q_base + slot * kBlockM : wk.q_base;
}
// Index in the sequence of slot p's first K tile, and the step between its K
// tiles (for masking).
__host__ __device__ __forceinline__ int slot_seq0(const Work &wk, int slot) {
    return wk.kind == kSplitQItem ? wk.kv0 + slot : wk.kv0;
}
__host__ __device__ __forceinline__ int slot_seq_step(const Work &wk) { return wk.kind == kSplitQItem ? 2 : 1; }
// Slice and sequence index of ring tile r of the item.
__host__ __device__ __forceinline__ int ring_slice(const Work &wk, int r) {
    return wk.kind == kTwinItem ? wk.slice + (r & 1) : wk.slice;
}
__host__ __device__ __forceinline__ int ring_seq(const Work &wk, int r) {
    return wk.kind == kTwinItem ? r >> 1 : wk.kv0 + r;
}

__device__ uint32_t g_ncz_status = 0u;
// Bound of every mbarrier wait, in SM cycles (tests shorten it, ncz_test_set_wait_limit).
__device__ unsigned long long g_ncz_wait_limit = kWaitLimitCycles;
// Test hook (ncz_test_drop_arrive): when set, the MMA warp of Q tile 0 never
// signals its first scores, so the softmax's bounded wait runs out.
__device__ int g_ncz_test_drop = 0;

__host__ __device__ constexpr int imin(int a, int b) { return a < b ? a : b; }

// Host and device: the host side checks the item order in tests
// (ncz_test_item_work).
__host__ __device__ __forceinline__ Work make_work(const FlashParams &p, int item) {
    Work wk;
    const int n_kv = (p.seq_len + kBlockN - 1) / kBlockN;
    if (p.twin) {
        // Item i: slices 2i and 2i + 1, each one Q tile against all of its K
        // tiles (seq_len <= 128).  The last item of an odd count is an item of
        // one slice (Q tile 0; its Q tile 1 starts past seq_len), so the ring
        // never names a slice past the last.
        wk.slice = 2 * item;
        wk.q_base = 0;
        wk.split = 0;
        wk.kv0 = 0;
        const int last_row = p.seq_len - 1;
        const int total = p.causal ? last_row / kBlockN + 1 : n_kv;
        wk.n[0] = total;
        wk.diag[0] = wk.diag[1] = total - 1;
        if (2 * item + 1 < p.batch_heads) {
            wk.n[1] = total;
            wk.n_max = 2 * total;
            wk.kstride = 2;
            wk.kind = kTwinItem;
        } else {
            wk.n[1] = 0;
            wk.n_max = total;
            wk.kstride = 1;
            wk.kind = kPairItem;
        }
        return wk;
    }
    if (p.qsplit_groups > 0) {
        // Chunks of chunk_slices slices; inside a chunk the items by K tiles
        // per pipeline, heaviest first: the items of two Q tiles that visit
        // more K tiles than the heaviest split-Q item gives each pipeline
        // (lead groups, heaviest group first, then slice), then the split-Q
        // items (the Q tiles of the top qsplit_groups groups, heaviest first,
        // then slice), then the other items of two Q tiles.  No split-KV here.
        static_assert(kBlockM == kBlockN, "lead groups count K tiles as Q tiles");
        const int n_qt = (p.seq_len + kBlockM - 1) / kBlockM;
        const int low_groups = p.num_groups - p.qsplit_groups;  // groups of two-Q-tile items
        const int split_qt = n_qt - kQTiles * low_groups;       // split-Q items per slice
        // A low group g is whole and its heavier Q tile visits kQTiles*(g+1)
        // K tiles under causal masking, n_kv without; the heaviest split-Q item
        // gives a pipeline (n_kv + 1) / 2.
        const int lead = p.causal ? low_groups - imin(low_groups, ((n_kv + 1) / 2) / kQTiles) : low_groups;
        const int per_chunk = p.chunk_slices * (split_qt + low_groups);
        const int chunk = item / per_chunk;
        const int off = item - chunk * per_chunk;
        const int c0 = chunk * p.chunk_slices;
        const int slices = imin(p.chunk_slices, p.batch_heads - c0);
        wk.split = 0;
        wk.kv0 = 0;
        if (off >= slices * lead && off < slices * (lead + split_qt)) {
            const int rel = off - slices * lead;
            const int qt = n_qt - 1 - rel / slices;
            wk.slice = c0 + rel % slices;
            wk.q_base = qt * kBlockM;
            const int last_row = imin(wk.q_base + kBlockM, p.seq_len) - 1;
            const int total = p.causal ? last_row / kBlockN + 1 : n_kv;
            wk.n[0] = (total + 1) / 2;
            wk.n[1] = total / 2;
            wk.diag[0] = wk.diag[1] = total - 1;
            wk.n_max = total;
            wk.kstride = 2;
            wk.kind = kSplitQItem;
            return wk;
        }
        const int rem = off < slices * lead ? off : off - slices * split_qt;  // place among the two-tile items
        const int group = low_groups - 1 - rem / slices;
        wk.slice = c0 + rem % slices;
        wk.q_base = group * (kQTiles * kBlockM);
        wk.n_max = 0;
        wk.kstride = 1;
        wk.kind = kPairItem;
#pragma unroll
        for (int w = 0; w < kQTiles; ++w) {
            const int q0 = wk.q_base + w * kBlockM;
            const int last_row = imin(q0 + kBlockM, p.seq_len) - 1;
            const int total = q0 >= p.seq_len ? 0 : (p.causal ? last_row / kBlockN + 1 : n_kv);
            wk.n[w] = total;
            wk.diag[w] = total - 1;
            wk.n_max = total > wk.n_max ? total : wk.n_max;
        }
        return wk;
    }
    // Chunks of chunk_slices slices; inside a chunk the heaviest (last) Q-tile
    // groups first (under causal masking they visit the most K tiles), then
    // slice, then K range.
    const int per_chunk = p.chunk_slices * p.num_groups * p.num_splits;
    const int chunk = item / per_chunk;
    const int off = item - chunk * per_chunk;
    const int c0 = chunk * p.chunk_slices;
    const int slices = imin(p.chunk_slices, p.batch_heads - c0);  // the last chunk may be short
    const int per_group = slices * p.num_splits;
    const int group = p.num_groups - 1 - off / per_group;
    const int rem = off % per_group;
    wk.slice = c0 + rem / p.num_splits;
    wk.split = rem % p.num_splits;
    wk.q_base = group * (kQTiles * kBlockM);
    wk.kv0 = wk.split * p.kv_per_split;
    wk.n_max = 0;
    wk.kstride = 1;
    wk.kind = kPairItem;
#pragma unroll
    for (int w = 0; w < kQTiles; ++w) {
        const int q0 = wk.q_base + w * kBlockM;
        const int last_row = imin(q0 + kBlockM, p.seq_len) - 1;
        // causal (reference tile_end, src/flash_h64_bn32.zig:80-84): K tiles up to the diagonal
        const int total = q0 >= p.seq_len ? 0 : (p.causal ? last_row / kBlockN + 1 : n_kv);
        const int end = imin(total, wk.kv0 + p.kv_per_split);
        wk.n[w] = end > wk.kv0 ? end - wk.kv0 : 0;
        wk.diag[w] = total - 1;
        wk.n_max = wk.n[w] > wk.n_max ? wk.n[w] : wk.n_max;
    }
    return wk;
}

// Bounded mbarrier wait.  Returns false when the CTA is aborting or the wait
// exceeded g_ncz_wait_limit (then it raises the abort flag and records the site).
// honor_abort = false is used by teardown waits that must not be skipped.
// The slow loop is out of line; the common already-complete case costs one
// inlined try_wait.
__device__ __noinline__ bool bounded_wait_slow(uint32_t bar, uint32_t parity, volatile uint32_t *abort_flag,
                                               uint32_t site, bool honor_abort) {
    const unsigned long long t0 = sm_clock();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15u) == 0u) {
            if (honor_abort && *abort_flag) return false;
            if (sm_clock() - t0 > g_ncz_wait_limit) {
                *abort_flag = 1u;
                atomicCAS(&g_ncz_status, 0u, 0x80000000u | (site << 24) | (blockIdx.x & 0xFFFFFFu));
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity, volatile uint32_t *abort_flag,
                                             uint32_t site, bool honor_abort) {
    if (mbar_try_wait(bar, parity)) return true;
    return bounded_wait_slow(bar, parity, abort_flag, site, honor_abort);
}

// All lanes wait; the result is made warp-uniform so .sync.aligned tcgen05
// instructions that follow stay convergent.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile uint32_t *abort_flag,
                                          uint32_t site) {
    const bool ok = bounded_wait(bar, parity, abort_flag, site, true);
    return __all_sync(0xffffffffu, ok);
}

template <int D>
struct Bars {
    using L = SmemLayout<D>;
    uint32_t base;
    __device__ __forceinline__ uint32_t at(int i) const { return base + L::kOffBar + 8u * i; }
    __device__ __forceinline__ uint32_t q_full(int slot) const { return at(L::kBarQFull + slot); }
    __device__ __forceinline__ uint32_t q_empty(int slot) const { return at(L::kBarQEmpty + slot); }
    __device__ __forceinline__ uint32_t k_full(int s) const { return at(L::kBarKFull + s); }
    __device__ __forceinline__ uint32_t v_full(int s) const { return at(L::kBarVFull + s); }
    __device__ __forceinline__ uint32_t kv_empty(int s) const { return at(L::kBarKvEmpty + s); }
    __device__ __forceinline__ uint32_t s_full(int w) const { return at(L::kBarSFull + w); }
    __device__ __forceinline__ uint32_t s_free(int w) const { return at(L::kBarSFree + w); }
    __device__ __forceinline__ uint32_t p_full(int w) const { return at(L::kBarPFull + w); }
    __device__ __forceinline__ uint32_t o_done(int w) const { return at(L::kBarODone + w); }
    __device__ __forceinline__ uint32_t o_free(int w) const { return at(L::kBarOFree + w); }
    __device__ __forceinline__ uint32_t drain(int w) const { return at(L::kBarDrain + w); }
    __device__ __forceinline__ uint32_t clc_full(int s) const { return at(L::kBarClcFull + s); }
    __device__ __forceinline__ uint32_t clc_empty(int s) const { return at(L::kBarClcEmpty + s); }
    __device__ __forceinline__ uint32_t clc_resp(int s) const { return base + L::kOffClc + 16u * s; }
    __device__ __forceinline__ uint32_t merge_ready(int sub) const { return at(L::kBarMergeReady + sub); }
    __device__ __forceinline__ uint32_t merge_done(int sub) const { return at(L::kBarMergeDone + sub); }
};

// ---------------------------------------------------------------------------
// work-item walk
// ---------------------------------------------------------------------------
// A CTA's first item is its blockIdx.x.  While item i runs, the producer asks
// cluster launch control to cancel a CTA of this grid that has not started and
// takes that CTA's item as item i + 1.  Items leave the hardware queue in
// launch order (heaviest first), so every SM keeps pulling the next heaviest
// item as soon as it can take one, and the next item's Q, K/V and first scores
// load while the current item's last tiles and epilogue run.  The response for
// item i + 1 lands in ring slot i % kClcSlots; every reader warp decodes it and
// releases the slot.  A request that finds no CTA left ends the walk (no
// request follows a failed one).
template <int D>
__device__ __forceinline__ bool request_item(const Bars<D> &b, int i, volatile uint32_t *abort_flag) {
    const int s = i % kClcSlots;
    if (i >= kClcSlots && !warp_wait(b.clc_empty(s), ((i / kClcSlots) - 1) & 1, abort_flag, kSiteClcEmpty))
        return false;
    clc_try_cancel_elect(b.clc_resp(s), b.clc_full(s));
    return true;
}

// Item i (i >= 1) of the CTA's walk; -1 when the walk is over, -2 when the
// wait gave up (the CTA is aborting).
template <int D>
__device__ __forceinline__ int take_item(const Bars<D> &b, int i, volatile uint32_t *abort_flag, int lane) {
    const int s = (i - 1) % kClcSlots;
    if (!warp_wait(b.clc_full(s), ((i - 1) / kClcSlots) & 1, abort_flag, kSiteClcFull)) return -2;
    const int item = clc_decode(b.clc_resp(s));
    fence_proxy_async_smem();  // the read precedes the slot's next (async-proxy) write
    __syncwarp();
    if (lane == 0) mbar_arrive(b.clc_empty(s));
    return item;
}

// ---------------------------------------------------------------------------
// producer, TMA variant (whole warp; elect.sync picks the issuing lane)
// ---------------------------------------------------------------------------
// Per item: Q into slot it & 1 once the item two back released it, the
// request for the next item, then the item's K/V tiles through the ring (tile
// counter t runs across items).
template <int D>
__device__ __forceinline__ void producer_tma(const FlashParams &p, const CUtensorMap *tq, const CUtensorMap *tk,
                                             const CUtensorMap *tv, uint32_t sbase, volatile uint32_t *abort_flag,
                                             int lane) {
    using L = SmemLayout<D>;
    const Bars<D> b{sbase};
    uint32_t t = 0;    // K/V tiles issued so far
    int it = 0;        // items started
    int pending = -1;  // items started when the unanswered launch-control request was made
    bool ok = true;
    for (int item = static_cast<int>(blockIdx.x); ok && item >= 0;) {
        const Work wk = make_work(p, item);
        count_item_visit(p, item, lane);
        const int qs = it & 1;
        if (it >= 2 && !warp_wait(b.q_empty(qs), ((it >> 1) - 1) & 1, abort_flag, kSiteQEmpty)) {
            ok = false;
            break;
        }
        uint32_t qbytes = 0;
#pragma unroll
        for (int w = 0; w < kQTiles; ++w) qbytes += q_tile_used(wk, w) ? L::kQTile : 0;
        mbar_arrive_expect_tx_elect(b.q_full(qs), qbytes);
#pragma unroll
        for (int w = 0; w < kQTiles; ++w)
            if (q_tile_used(wk, w))
                tma_load_3d_elect(sbase + L::kOffQ + qs * L::kQSlot + w * L::kQTile, tq, b.q_full(qs), 0,
                                  slot_row0(wk, w), slot_slice(wk, w));
        const int cur = it++;
        const bool walk = wk.n_max < p.walk_tiles;
        const int req_at = wk.n_max > kClcLead ? wk.n_max - kClcLead : 0;  // see kClcLead
        for (int j = 0; j < wk.n_max; ++j, ++t) {
            const int st = t % L::kStages;
            if (t >= L::kStages && !warp_wait(b.kv_empty(st), ((t / L::kStages) - 1) & 1, abort_flag, kSiteKvEmpty)) {
                ok = false;
                break;
            }
            if (walk && j == req_at) {
                if (!request_item(b, cur, abort_flag)) {
                    ok = false;
                    break;
                }
                pending = cur;
            }
            mbar_arrive_expect_tx_elect(b.k_full(st), L::kKvTile);
            tma_load_3d_elect(sbase + L::kOffK + st * L::kKvTile, tk, b.k_full(st), 0, ring_seq(wk, j) * kBlockN,
                              ring_slice(wk, j));
            mbar_arrive_expect_tx_elect(b.v_full(st), L::kKvTile);
            tma_load_3d_elect(sbase + L::kOffV + st * L::kKvTile, tv, b.v_full(st), 0, ring_seq(wk, j) * kBlockN,
                              ring_slice(wk, j));
        }
        if (!ok) break;
        if (walk && wk.n_max == 0) {  // no K tiles: ask now
            if (!request_item(b, cur, abort_flag)) break;
            pending = cur;
        }
        item = walk ? take_item(b, it, abort_flag, lane) : -1;
        if (item != -2) pending = -1;
    }
    // Every issued copy must land before shared memory is released: the Q of the
    // last two items, the last kStages K/V tiles and an unanswered request.
    for (int i = it - 2 < 0 ? 0 : it - 2; i < it; ++i)
        bounded_wait(b.q_full(i & 1), (i >> 1) & 1, abort_flag, kSiteProducerDrain, false);
    if (pending >= 0)
        bounded_wait(b.clc_full(pending % kClcSlots), (pending / kClcSlots) & 1, abort_flag, kSiteProducerDrain,
                     false);
    for (uint32_t u = t < static_cast<uint32_t>(L::kStages) ? 0u : t - L::kStages; u < t; ++u) {
        const int st = u % L::kStages;
        const uint32_t ph = (u / L::kStages) & 1;
        bounded_wait(b.k_full(st), ph, abort_flag, kSiteProducerDrain, false);
        bounded_wait(b.v_full(st), ph, abort_flag, kSiteProducerDrain, false);
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// producer, LSU variant (all 32 lanes): any 2-byte-aligned layout
// ---------------------------------------------------------------------------
// Loads rows row0 .. row0+kRows-1 of one slice (rows >= seq_len read as zero)
// into a 1024-byte-aligned tile, in the same swizzled layout TMA produces.
template <int D, int kRows>
__device__ __forceinline__ void lsu_tile(uint8_t *dst, const uint16_t *src, long long row_stride, int row0,
                                         int seq_len, int lane) {
    constexpr int kChunks = D / 8;  // 16-byte chunks per row
    constexpr uint32_t kSpan = 2 * D;
    for (int idx = lane; idx < kRows * kChunks; idx += 32) {
        const int r = idx / kChunks, c = idx % kChunks;
        const int grow = row0 + r;
        uint32_t wv[4] = {0u, 0u, 0u, 0u};
        if (grow < seq_len) {
            const uint16_t *s = src + static_cast<long long>(grow) * row_stride + c * 8;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                wv[e] = static_cast<uint32_t>(__ldg(s + 2 * e)) | (static_cast<uint32_t>(__ldg(s + 2 * e + 1)) << 16);
        }
        const uint32_t off = tma_swizzle(kSpan, static_cast<uint32_t>(r) * kSpan + static_cast<uint32_t>(c) * 16u);
        *reinterpret_cast<uint4 *>(dst + off) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
}

template <int D>
__device__ __forceinline__ void producer_lsu(const FlashParams &p, uint8_t *smem, uint32_t sbase,
                                             volatile uint32_t *abort_flag, int lane) {
    using L = SmemLayout<D>;
    const Bars<D> b{sbase};
    uint32_t t = 0;    // K/V tiles loaded so far
    int it = 0;        // items started
    int pending = -1;  // items started when the unanswered launch-control request was made
    bool ok = true;
    for (int item = static_cast<int>(blockIdx.x); ok && item >= 0;) {
        const Work wk = make_work(p, item);
        count_item_visit(p, item, lane);
        const int slot = it & 1;
        if (it >= 2 && !warp_wait(b.q_empty(slot), ((it >> 1) - 1) & 1, abort_flag, kSiteQEmpty)) break;
        const int cur = it++;
        const bool walk = wk.n_max < p.walk_tiles;
        const int req_at = wk.n_max > kClcLead ? wk.n_max - kClcLead : 0;  // see kClcLead
#pragma unroll
        for (int w = 0; w < kQTiles; ++w)
            if (q_tile_used(wk, w))
                lsu_tile<D, kBlockM>(smem + L::kOffQ + slot * L::kQSlot + w * L::kQTile,
                                     p.q + slot_slice(wk, w) * p.q_stride, p.q_row, slot_row0(wk, w), p.seq_len,
                                     lane);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(b.q_full(slot));
        for (int j = 0; j < wk.n_max; ++j, ++t) {
            const int st = t % L::kStages;
            if (t >= L::kStages && !warp_wait(b.kv_empty(st), ((t / L::kStages) - 1) & 1, abort_flag, kSiteKvEmpty)) {
                ok = false;
                break;
            }
            if (walk && j == req_at) {
                if (!request_item(b, cur, abort_flag)) {
                    ok = false;
                    break;
                }
                pending = cur;
            }
            lsu_tile<D, kBlockN>(smem + L::kOffK + st * L::kKvTile, p.k + ring_slice(wk, j) * p.k_stride, p.k_row,
                                 ring_seq(wk, j) * kBlockN, p.seq_len, lane);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(b.k_full(st));
            lsu_tile<D, kBlockN>(smem + L::kOffV + st * L::kKvTile, p.v + ring_slice(wk, j) * p.v_stride, p.v_row,
                                 ring_seq(wk, j) * kBlockN, p.seq_len, lane);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(b.v_full(st));
        }
        if (!ok) break;
        if (walk && wk.n_max == 0) {  // no K tiles: ask now
            if (!request_item(b, cur, abort_flag)) break;
            pending = cur;
        }
        item = walk ? take_item(b, it, abort_flag, lane) : -1;
        if (item != -2) pending = -1;
    }
    // An unanswered request must land before shared memory is released.
    if (pending >= 0)
        bounded_wait(b.clc_full(pending % kClcSlots), (pending / kClcSlots) & 1, abort_flag, kSiteProducerDrain,
                     false);
    __syncwarp();
}

// ---------------------------------------------------------------------------
// MMA issuer (whole warp; elect.sync picks the issuing lane)
// ---------------------------------------------------------------------------
// QK^T of ring tile t (K in stage t % kStages) for one Q tile into its S.
template <int D, bool kBf16>
__device__ __forceinline__ void issue_qk(uint32_t t, uint32_t sbase, uint32_t tS, uint64_t qdesc) {
    using L = SmemLayout<D>;
    constexpr uint32_t idesc_qk = umma_idesc_f16_f32(kBlockM, kBlockN, 0, 0, kBf16);  // both K-major
    const int st = t % L::kStages;
    const uint64_t kdesc = umma_smem_desc(sbase + L::kOffK + st * L::kKvTile, 16, 8 * L::kSpan, L::kUmmaLayout);
    // K advance: 32 bytes (2 encoded units) inside the swizzled row per step
    umma_ss_chain_elect<D / 16>(tS, qdesc, kdesc, idesc_qk);
}

// O (+)= P V of ring tile t; `first` starts the accumulation of a new item.
template <int D, bool kBf16>
__device__ __forceinline__ void issue_pv(uint32_t t, bool first, uint32_t sbase, uint32_t tP, uint32_t tO) {
    using L = SmemLayout<D>;
    constexpr uint32_t idesc_pv = umma_idesc_f16_f32(kBlockM, D, 0, 1, kBf16);  // B = V, MN-major
    const int st = t % L::kStages;
    // V tile: kBlockN keys x D, rows of 2D bytes (one swizzle atom wide); 8-row groups 8*span apart.
    const uint64_t vdesc =
        umma_smem_desc(sbase + L::kOffV + st * L::kKvTile, L::kKvTile, 8 * L::kSpan, L::kUmmaLayout);
    // 16 keys per step: 8 TMEM columns of P, 16 rows of V
    umma_ts_chain_elect<kBlockN / 16>(tO, tP, vdesc, static_cast<uint64_t>((16 * L::kSpan) >> 4), idesc_pv,
                                      first ? 0u : 1u);
}

// One MMA warp per pipeline w (warps 1 and 2), over all of the CTA's items.
// Per K tile j of its slot: QK_w(j+1) as soon as the softmax has read S_w(j)
// and K(j+1) is resident, then PV_w(j) once P_w(j) is stored and V(j) is
// resident; the first PV of an item also waits until the softmax has read the
// previous item's O (o_free).  After its item's last QK the warp counts itself
// out of the Q slot (q_empty).  Each warp arrives once per ring tile of the
// item on the stage's kv_empty barrier: a commit after its PV for the tiles its
// slot visits, a plain arrive for the others (past its causal range, or the
// other slot's tiles of a split-Q item), issued in ring order as soon as each
// is loaded, so a stage is released when both pipelines are done with it.
template <int D, bool kBf16>
__device__ __forceinline__ void mma_role(const FlashParams &p, int w, uint32_t sbase, uint32_t tmem,
                                         volatile uint32_t *abort_flag, int lane) {
    using L = SmemLayout<D>;
    constexpr int S = L::kStages;
    const Bars<D> b{sbase};
    const uint32_t tS = tmem + w * kTileCols, tP = tS + kColP, tO = tS + kColO;
    uint32_t t = 0;    // ring tiles passed (all items)
    uint32_t sc = 0;   // K tiles of this pipeline so far: S/P/O barrier phases
    uint32_t epi = 0;  // items in which this pipeline had work: o_free phases
    bool ok = true, walk = false;
    for (int item = static_cast<int>(blockIdx.x), it = 0; ok && item >= 0;
         ++it, item = ok && walk ? take_item(b, it, abort_flag, lane) : -1) {
        const Work wk = make_work(p, item);
        walk = wk.n_max < p.walk_tiles;
        const int wq = w ^ (it & 1);           // slot of the item this pipeline takes
        const int n = wq ? wk.n[1] : wk.n[0];  // a select keeps Work out of local memory
        const int ks = wk.kstride;
        const int koff = slot_koff(wk, wq);    // slot's j-th K tile = ring tile koff + j * ks
        const int qs = it & 1;
        // Ring tiles of the item before `upto` that this slot does not visit:
        // released on the other pipeline's behalf once loaded, in ring order.
        int rel = 0;
        auto release_before = [&](int upto) -> bool {
            for (; rel < upto; ++rel) {
                const int dj = rel - koff;
                if (dj >= 0 && dj % ks == 0 && dj / ks < n) continue;  // one of this slot's tiles
                const uint32_t tu = t + rel;
                if (!warp_wait(b.k_full(tu % S), (tu / S) & 1, abort_flag, kSiteKFull)) return false;
                if (lane == 0) mbar_arrive(b.kv_empty(tu % S));
                __syncwarp();
            }
            return true;
        };
        // Waited for every item, also without work: this warp's q_empty arrivals
        // then never run two phases ahead of the producer.
        ok = warp_wait(b.q_full(qs), (it >> 1) & 1, abort_flag, kSiteQFull);
        if (!ok) break;
        tc_fence_after();
        const uint64_t qdesc = umma_smem_desc(sbase + L::kOffQ + qs * L::kQSlot + slot_qtile(wk, wq) * L::kQTile, 16,
                                              8 * L::kSpan, L::kUmmaLayout);
        if (n > 0) {
            const uint32_t t0 = t + koff;
            ok = release_before(koff) && (sc == 0 || warp_wait(b.s_free(w), (sc - 1) & 1, abort_flag, kSiteSFree)) &&
                 warp_wait(b.k_full(t0 % S), (t0 / S) & 1, abort_flag, kSiteKFull);
            if (!ok) break;
            tc_fence_after();
            issue_qk<D, kBf16>(t0, sbase, tS, qdesc);
            if (!(w == 0 && g_ncz_test_drop != 0)) umma_commit_elect(b.s_full(w));
            if (n == 1) umma_commit_elect(b.q_empty(qs));
        } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(b.q_empty(qs));
            __syncwarp();
        }
        for (int j = 0; ok && j < n; ++j) {
            const uint32_t tj = t + koff + j * ks;
            const int st = tj % S;
            if (j + 1 < n) {
                const uint32_t tn = tj + ks;
                ok = release_before(koff + (j + 1) * ks) &&
                     warp_wait(b.s_free(w), (sc + j) & 1, abort_flag, kSiteSFree) &&
                     warp_wait(b.k_full(tn % S), (tn / S) & 1, abort_flag, kSiteKFull);
                if (!ok) break;
                tc_fence_after();
                issue_qk<D, kBf16>(tn, sbase, tS, qdesc);
                umma_commit_elect(b.s_full(w));
                if (j + 2 == n) umma_commit_elect(b.q_empty(qs));  // the item's last QK
            }
            ok = warp_wait(b.v_full(st), (tj / S) & 1, abort_flag, kSiteVFull) &&
                 warp_wait(b.p_full(w), (sc + j) & 1, abort_flag, kSitePFull) &&
                 (j > 0 || epi == 0 || warp_wait(b.o_free(w), (epi - 1) & 1, abort_flag, kSiteOFree));
            if (!ok) break;
            tc_fence_after();
            issue_pv<D, kBf16>(tj, j == 0, sbase, tP, tO);
            umma_commit_elect(b.o_done(w));
            umma_commit_elect(b.kv_empty(st));  // this pipeline is done with K(tj) and V(tj)
        }
        if (ok) ok = release_before(wk.n_max);  // the item's remaining tiles of the other slot
        if (n > 0) {
            sc += n;
            ++epi;
        }
        t += wk.n_max;
    }
    // All issued MMAs must finish before TMEM and shared memory are released.
    umma_commit_elect(b.drain(w));
    bounded_wait(b.drain(w), 0, abort_flag, kSiteMmaDrain, false);
    __syncwarp();
}

// ---------------------------------------------------------------------------
// softmax + correction + epilogue (one warpgroup per Q tile)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// TMEM load / store of one row's O columns
template <int N>
__device__ __forceinline__ void load_cols(uint32_t taddr, float (&o)[N]) {
    uint32_t r[N];
    if constexpr (N == 64) {
        tmem_ld_x64_wait(taddr, r);
    } else if constexpr (N == 32) {
        tmem_ld_x32_wait(taddr, r);
    } else {
        static_assert(N == 16, "column count");
        tmem_ld_x16_wait(taddr, r);
    }
#pragma unroll
    for (int i = 0; i < N; ++i) o[i] = __uint_as_float(r[i]);
}

template <int N>
__device__ __forceinline__ void store_cols(uint32_t taddr, const float (&o)[N]) {
    uint32_t r[N];
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = __float_as_uint(o[i]);
    if constexpr (N == 64) {
        tmem_st_x64(taddr, r);
    } else if constexpr (N == 32) {
        tmem_st_x32(taddr, r);
    } else {
        static_assert(N == 16, "column count");
        tmem_st_x16(taddr, r);
    }
}

// Writes O[row][0 .. N) = o / l (f32 or f16, vector stores when aligned), as
// o * (1 / l): one division per row instead of N.
template <int N>
__device__ __forceinline__ void write_o_global(const FlashParams &p, int slice, int row, const float (&o)[N],
                                               float l) {
    const float inv = 1.0f / l;
    const long long base = static_cast<long long>(slice) * p.o_stride + static_cast<long long>(row) * p.o_row;
    if (p.o_dtype != 0) {  // 16-bit O: f16 (1) or bf16 (2)
        uint16_t *orow = reinterpret_cast<uint16_t *>(p.o) + base;
        const bool bf = p.o_dtype == 2;
        if (p.o_vec) {
#pragma unroll
            for (int c = 0; c < N; c += 8) {
                uint4 v;
                v.x = bf ? pack_bf16x2(o[c + 0] * inv, o[c + 1] * inv) : pack_f16x2(o[c + 0] * inv, o[c + 1] * inv);
                v.y = bf ? pack_bf16x2(o[c + 2] * inv, o[c + 3] * inv) : pack_f16x2(o[c + 2] * inv, o[c + 3] * inv);
                v.z = bf ? pack_bf16x2(o[c + 4] * inv, o[c + 5] * inv) : pack_f16x2(o[c + 4] * inv, o[c + 5] * inv);
                v.w = bf ? pack_bf16x2(o[c + 6] * inv, o[c + 7] * inv) : pack_f16x2(o[c + 6] * inv, o[c + 7] * inv);
                *reinterpret_cast<uint4 *>(orow + c) = v;
            }
        } else {
#pragma unroll
            for (int c = 0; c < N; ++c)
                orow[c] = static_cast<uint16_t>(bf ? pack_bf16x2(o[c] * inv, 0.0f) : pack_f16x2(o[c] * inv, 0.0f));
        }
    } else {
        float *orow = reinterpret_cast<float *>(p.o) + base;
        if (p.o_vec) {
#pragma unroll
            for (int c = 0; c < N; c += 4)
                *reinterpret_cast<float4 *>(orow + c) = make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
        } else {
#pragma unroll
            for (int c = 0; c < N; ++c) orow[c] = o[c] * inv;
        }
    }
}

// Stores the 32 rows of a warp (lane = row, kChunks 16-byte chunks per row in
// `v`) through `stage`, 32 rows x 2D bytes of shared memory: each lane writes
// its row into the staging rows (16-byte chunk c of row r at chunk c ^ (r mod
// chunks per row), so neither the row writes nor the reads conflict on banks),
// then every global store instruction writes whole row segments (2D bytes of
// 32 / (2D / 16) consecutive rows) instead of one 16-byte piece of each of 32
// rows.  Rows >= `valid` are not written.  Rounds of 2D bytes per row when a
// row holds more (f32 O: two).
template <int D, int kChunks>
__device__ __forceinline__ void store_rows_staged(uint8_t *stage, const uint4 (&v)[kChunks], char *gbase,
                                                  long long row_bytes, int valid, int lane) {
    constexpr int kRB = 2 * D;     // staging bytes per row and round
    constexpr int kCH = kRB / 16;  // chunks per row and round
    static_assert(kChunks % kCH == 0, "whole rounds");
#pragma unroll
    for (int r = 0; r < kChunks / kCH; ++r) {
        if (r > 0) __syncwarp();  // the previous round's reads are done
#pragma unroll
        for (int c = 0; c < kCH; ++c)
            *reinterpret_cast<uint4 *>(stage + lane * kRB + ((c ^ (lane & (kCH - 1))) * 16)) = v[r * kCH + c];
        __syncwarp();
#pragma unroll
        for (int k = 0; k < kCH; ++k) {
            const int idx = k * 32 + lane;
            const int row = idx / kCH, c = idx % kCH;
            const uint4 d = *reinterpret_cast<const uint4 *>(stage + row * kRB + ((c ^ (row & (kCH - 1))) * 16));
            if (row < valid) *reinterpret_cast<uint4 *>(gbase + row * row_bytes + r * kRB + c * 16) = d;
        }
    }
}

// O rows of a warp, o / l, through the staging rows (needs 16-byte aligned O rows).
template <int D>
__device__ __forceinline__ void write_o_staged(const FlashParams &p, int slice, int row0, const float (&o)[D],
                                               float l, uint8_t *stage, int valid, int lane) {
    const float inv = 1.0f / l;
    if (p.o_dtype != 0) {  // f16 (1) or bf16 (2)
        const bool bf = p.o_dtype == 2;
        uint4 v[D / 8];
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            const float *x = o + 8 * i;
            v[i].x = bf ? pack_bf16x2(x[0] * inv, x[1] * inv) : pack_f16x2(x[0] * inv, x[1] * inv);
            v[i].y = bf ? pack_bf16x2(x[2] * inv, x[3] * inv) : pack_f16x2(x[2] * inv, x[3] * inv);
            v[i].z = bf ? pack_bf16x2(x[4] * inv, x[5] * inv) : pack_f16x2(x[4] * inv, x[5] * inv);
            v[i].w = bf ? pack_bf16x2(x[6] * inv, x[7] * inv) : pack_f16x2(x[6] * inv, x[7] * inv);
        }
        char *g = reinterpret_cast<char *>(p.o) + (slice * p.o_stride + static_cast<long long>(row0) * p.o_row) * 2;
        store_rows_staged<D, D / 8>(stage, v, g, p.o_row * 2, valid, lane);
    } else {
        uint4 v[D / 4];
#pragma unroll
        for (int i = 0; i < D / 4; ++i)
            v[i] = make_uint4(__float_as_uint(o[4 * i] * inv), __float_as_uint(o[4 * i + 1] * inv),
                              __float_as_uint(o[4 * i + 2] * inv), __float_as_uint(o[4 * i + 3] * inv));
        char *g = reinterpret_cast<char *>(p.o) + (slice * p.o_stride + static_cast<long long>(row0) * p.o_row) * 4;
        store_rows_staged<D, D / 4>(stage, v, g, p.o_row * 4, valid, lane);
    }
}

// Split-KV partials of a warp's rows through the staging rows: O unnormalised
// (rows of D floats, contiguous), (m, l) per row.
template <int D>
__device__ __forceinline__ void write_partial_staged(const FlashParams &p, const Work &wk, int row0, int row,
                                                     const float (&o)[D], float m, float l, uint8_t *stage,
                                                     int valid, int lane) {
    const long long idx0 = (static_cast<long long>(wk.split) * p.batch_heads + wk.slice) * p.seq_len + row0;
    uint4 v[D / 4];
#pragma unroll
    for (int i = 0; i < D / 4; ++i)
        v[i] = make_uint4(__float_as_uint(o[4 * i]), __float_as_uint(o[4 * i + 1]), __float_as_uint(o[4 * i + 2]),
                          __float_as_uint(o[4 * i + 3]));
    store_rows_staged<D, D / 4>(stage, v, reinterpret_cast<char *>(p.part_o + idx0 * D), D * 4, valid, lane);
    if (row < p.seq_len) *reinterpret_cast<float2 *>(p.part_ml + (idx0 + lane) * 2) = make_float2(m, l);
}

// Row max of the first kCols of kBlockN scores with 8 independent chains:
// chain i covers x[i], x[8+i], ...
template <int kCols = kBlockN>
__device__ __forceinline__ float row_max(const float (&x)[kBlockN]) {
    static_assert(kCols % 16 == 0 && kCols <= kBlockN, "tile width");
    float mx[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) mx[i] = fmaxf(x[i], x[8 + i]);
#pragma unroll
    for (int c = 16; c + 16 <= kCols; c += 16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = fmax3(mx[i], x[c + i], x[c + 8 + i]);
    }
    return fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], fmax3(mx[5], mx[6], mx[7])));
}

// Exponentiates one score row in place against base m (log2 domain), packs P
// to pairs of the input type (f16 as src/flash_h64_bn32.zig:185, or bf16: the
// PV MMA takes A and B of one type) and sums the unrounded values in four
// independent chains.  Only the first kCols scores are exponentiated; P of the
// others is 0 (all of them masked).
template <bool kBf16, int kCols = kBlockN>
__device__ __forceinline__ float exp_row(float (&x)[kBlockN], float kmul, float m, uint32_t (&pk)[kBlockN / 2]) {
    const uint64_t kmul2 = pack_f32x2(kmul, kmul), negm2 = pack_f32x2(-m, -m);
    uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};  // (0.0f, 0.0f) x 4
#pragma unroll
    for (int c = kCols / 2; c < kBlockN / 2; ++c) pk[c] = 0u;  // +0 in f16 and bf16
#pragma unroll
    for (int c = 0; c < kCols / 2; ++c) {
        float e0, e1, p0, p1;
        unpack_f32x2(ffma2(pack_f32x2(x[2 * c], x[2 * c + 1]), kmul2, negm2), e0, e1);
        if (kExp2EmuPeriod > 0 && c % kExp2EmuPeriod >= kExp2EmuPeriod - kExp2EmuCount) {
            if constexpr (kExp2EmuDegree == 3) {
                exp2_poly3_x2(e0, e1, p0, p1);  // FMA pipe
            } else {
                exp2_poly_x2(e0, e1, p0, p1);
            }
        } else {
            p0 = ex2_approx(e0);  // MUFU
            p1 = ex2_approx(e1);
        }
        sum2[c & 3] = fadd2(sum2[c & 3], pack_f32x2(p0, p1));
        pk[c] = pack_in_x2<kBf16>(p0, p1);
    }
    float s0, s1;
    unpack_f32x2(fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3])), s0, s1);
    return s0 + s1;
}

// Keys of tile j a row may see: keys >= seq_len and, under causal masking,
// keys > row are masked (reference: src/flash_h64_bn32.zig:122-135).
__device__ __forceinline__ int lim_of(const FlashParams &p, int row, int j) {
    int lim = p.seq_len - j * kBlockN;
    if (p.causal) lim = min(lim, row - j * kBlockN + 1);
    return lim;
}

// Scores of half H (keys 64H .. 64H+63) as the exponent's input: pre-scaled when
// scale <= 0, masked keys at -inf.  Only the last K tile of a Q tile holds masked
// keys: a Q tile's rows share one 128-key tile index.
template <int H>
__device__ __forceinline__ void prep_scores(float (&x)[kBlockN], bool pre_scale, float scale_log2, bool last,
                                            int lim) {
    constexpr int c0 = H * kBlockN / 2;
    if (pre_scale) {
#pragma unroll
        for (int c = c0; c < c0 + kBlockN / 2; ++c) x[c] *= scale_log2;
    }
    if (last && lim < c0 + kBlockN / 2) {
#pragma unroll
        for (int c = c0; c < c0 + kBlockN / 2; ++c) x[c] = c < lim ? x[c] : -INFINITY;
    }
}

template <int D, bool kBf16>
__device__ __forceinline__ void softmax_role(const FlashParams &p, uint8_t *smem, uint32_t sbase, uint32_t tmem,
                                             volatile uint32_t *abort_flag, int warp, int lane) {
    using L = SmemLayout<D>;
    const Bars<D> b{sbase};
    const int w = (warp - 4) >> 2;                                // pipeline of this warpgroup
    const int sub = warp & 3;                                     // SM sub-partition
    const int r = static_cast<int>(threadIdx.x) - 128 * (w + 1);  // row inside the tile = TMEM lane
    const uint32_t tS = tmem + (static_cast<uint32_t>(sub * 32) << 16) + w * kTileCols;
    const uint32_t tP = tS + kColP, tO = tS + kColO;
    const int seq_len = p.seq_len;
    // scale > 0: mask raw scores, exponent = fma(s, scale*log2e, -m).
    // Otherwise scale first, then mask, exponent = fma(x, 1, -m).
    const bool pre_scale = !(p.scale_log2 > 0.0f);
    const float kmul = pre_scale ? 1.0f : p.scale_log2;
    // The walk state (item, items started) waits in shared memory while the
    // tile loop runs, so it holds no registers there.
    volatile int *stash = reinterpret_cast<volatile int *>(smem + L::kOffStash + 8 * warp);
    uint32_t ph = 0;  // parity of the K tiles of this pipeline so far (all items): barrier phases
    uint32_t mc = 0;  // split-Q merges this warp took part in: merge barrier phases
    bool ok = true, walk = false;
    for (int item = static_cast<int>(blockIdx.x), it = 0; ok && item >= 0;
         ++it, item = ok && walk ? take_item(b, it, abort_flag, lane) : -1) {
        int n, row, kv0, diag, ks;
        {
            const Work wk = make_work(p, item);
            walk = wk.n_max < p.walk_tiles;
            const int wq = w ^ (it & 1);  // slot of the item this pipeline takes
            n = wq ? wk.n[1] : wk.n[0];
            row = slot_row0(wk, wq) + r;
            ks = slot_seq_step(wk);
            kv0 = slot_seq0(wk, wq);  // the slot's j-th K tile is kv0 + j * ks in its sequence
            diag = wq ? wk.diag[1] : wk.diag[0];
        }
        if (n == 0) {  // no rows of this pipeline in the item: nothing staged in its Q tile
            // Arrive only once this item's Q is in: a warp that skips items must
            // not arrive for item it + 2 before the slot's phase of item it has
            // completed (q_full(it) comes after q_empty(it - 2)), or the producer
            // could refill the slot while the other pipeline still stages O in it.
            if (!warp_wait(b.q_full(it & 1), (it >> 1) & 1, abort_flag, kSiteQFull)) break;
            if (lane == 0) mbar_arrive(b.q_empty(it & 1));
            continue;
        }
        stash[0] = item;
        stash[1] = it;
        float m = -INFINITY;  // exponent base: scaled row max, log2 domain (stale by < 8)
        float l = 0.0f;       // running sum of 2^(x - m)
        // One K tile.  The first of an item has no PV to wait for and no O to
        // rescale, and only the last can hold masked keys (K tile index diag,
        // or a ragged end); both are issued apart (`first` and `final` are
        // compile-time flags), so the loop over the other tiles carries neither
        // branch.  With the tile loop nested in the item loop, peeling the first
        // tile is worth about 6% per tile (measured at d=64).
        auto tile = [&](int j, auto first, auto final) -> bool {
            if (!warp_wait(b.s_full(w), (ph + j) & 1, abort_flag, kSiteSFull)) return false;
            tc_fence_after();
            float x[kBlockN];
            {
                uint32_t sr[kBlockN];
                tmem_ld_x128_wait(tS, sr);
#pragma unroll
                for (int c = 0; c < kBlockN; ++c) x[c] = __uint_as_float(sr[c]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(b.s_free(w));  // S may be overwritten by the next QK^T
            bool half = false;
            float mx;
            if constexpr (decltype(final)::value) {
                const int jg = kv0 + j * ks;  // K tile index in the sequence
                const bool last = jg == diag;
                const int lim = lim_of(p, row, jg);
                // Every key of the upper half masked for all 32 rows of this warp
                // (rows 0-63 of a Q tile on the causal diagonal): only the lower
                // half is exponentiated.
                half = last && __all_sync(0xffffffffu, lim <= kBlockN / 2);
                prep_scores<0>(x, pre_scale, p.scale_log2, last, lim);
                if (half) {
                    mx = row_max<kBlockN / 2>(x);
                } else {
                    prep_scores<1>(x, pre_scale, p.scale_log2, last, lim);
                    mx = row_max(x);
                }
            } else {
                prep_scores<0>(x, pre_scale, p.scale_log2, false, kBlockN);
                prep_scores<1>(x, pre_scale, p.scale_log2, false, kBlockN);
                mx = row_max(x);
            }
            const float m_new = fmaxf(m, mx * kmul);
            const bool need = m_new > m + kRescaleThreshold;
            float m_use = need ? m_new : m;
            m_use = m_use == -INFINITY ? 0.0f : m_use;  // row with nothing visible yet
            uint32_t pk[kBlockN / 2];
            const float tsum = half ? exp_row<kBf16, kBlockN / 2>(x, kmul, m_use, pk) : exp_row<kBf16>(x, kmul, m_use, pk);
            const float alpha = ex2_approx(m - m_use);  // 1 when not rescaling, 0 on the first tile
            l = l * alpha + tsum;
            m = m_use;
            if constexpr (!decltype(first)::value) {
                // PV(j-1) reads P and accumulates into O: it must be done before P is
                // overwritten and before O is rebased.  (At j = 0 the previous
                // item's epilogue already waited for its last PV.)
                if (!warp_wait(b.o_done(w), (ph + j - 1) & 1, abort_flag, kSiteODone)) return false;
                tc_fence_after();
                if (__any_sync(0xffffffffu, need)) {
                    // In chunks of at most 32 columns: fewer registers on this
                    // (rare) path, next to the 64 of P.
                    constexpr int kC = D < 32 ? D : 32;
#pragma unroll
                    for (int c0 = 0; c0 < D; c0 += kC) {
                        float o[kC];
                        load_cols<kC>(tO + c0, o);
#pragma unroll
                        for (int c = 0; c < kC; ++c) o[c] *= alpha;
                        store_cols<kC>(tO + c0, o);
                        tmem_wait_st();
                    }
                }
            }
            tmem_st_x64(tP, pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(b.p_full(w));
            return true;
        };
        if (n == 1) {
            ok = tile(0, std::true_type{}, std::true_type{});
        } else {
            ok = tile(0, std::true_type{}, std::false_type{});
            for (int j = 1; ok && j + 1 < n; ++j) ok = tile(j, std::false_type{}, std::false_type{});
            if (ok) ok = tile(n - 1, std::false_type{}, std::true_type{});
        }
        if (!ok) break;
        // Epilogue: the item's last PV done, O read, O released to the next item's
        // first PV, then written out.
        ok = warp_wait(b.o_done(w), (ph + n - 1) & 1, abort_flag, kSiteODone);
        if (!ok) break;
        item = stash[0];
        it = stash[1];
        const Work wk = make_work(p, item);
        const int wq = w ^ (it & 1);
        const bool qsp = wk.kind == kSplitQItem;
        // A split-Q item whose both slots visited K tiles: slot 0's warp writes the
        // rows, merging slot 1's state (same TMEM lanes, the other pipeline's
        // columns) into its own: O = (2^(m0-M) O0 + 2^(m1-M) O1) /
        // (2^(m0-M) l0 + 2^(m1-M) l1), M = max(m0, m1).
        const bool merge = qsp && wk.n[1] > 0;
        if (merge && wq == 1) {
            // Slot 1: hand (m, l) over, and release O only once the writer has read it.
            reinterpret_cast<float2 *>(smem + L::kOffMerge)[sub * 32 + lane] = make_float2(m, l);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(b.merge_ready(sub));
            ok = warp_wait(b.merge_done(sub), mc & 1, abort_flag, kSiteMergeDone);
            ++mc;
            if (!ok) break;
            if (lane == 0) {
                mbar_arrive(b.o_free(w));
                mbar_arrive(b.q_empty(it & 1));  // nothing staged by this warp
            }
            __syncwarp();
            ph ^= static_cast<uint32_t>(n) & 1u;
            continue;
        }
        tc_fence_after();
        float o[D];
        load_cols<D>(tO, o);
        if (merge) {
            ok = warp_wait(b.merge_ready(sub), mc & 1, abort_flag, kSiteMergeReady);
            ++mc;
            if (!ok) break;
            tc_fence_after();
            const float2 ml = reinterpret_cast<const float2 *>(smem + L::kOffMerge)[sub * 32 + lane];
            const float mm = fmaxf(m, ml.x);
            const float a0 = ex2_approx(m - mm), a1 = ex2_approx(ml.x - mm);
            const uint32_t tO1 = tmem + (static_cast<uint32_t>(sub * 32) << 16) + (1 - w) * kTileCols + kColO;
            constexpr int kC = D < 16 ? D : 16;
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += kC) {
                float o1[kC];
                load_cols<kC>(tO1 + c0, o1);
#pragma unroll
                for (int c = 0; c < kC; ++c) o[c0 + c] = o[c0 + c] * a0 + o1[c] * a1;
            }
            l = l * a0 + ml.y * a1;
            m = mm;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(b.merge_done(sub));
        } else {
            tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(b.o_free(w));
        // O goes out through shared memory: this pipeline's Q tile of the item
        // (its last QK is done), or for a split-Q item the slot's unused second
        // Q tile; the producer refills the slot only after every softmax warp
        // has arrived on q_empty.
        const int stile = qsp ? 1 : wq;
        uint8_t *stage = smem + L::kOffQ + (it & 1) * L::kQSlot + stile * L::kQTile + sub * 32 * L::kSpan;
        const int row0 = slot_row0(wk, wq) + sub * 32;  // this warp's first row
        const int valid = imin(32, seq_len - row0);
        if (p.num_splits > 1) {
            write_partial_staged<D>(p, wk, row0, row, o, m, l, stage, valid, lane);
        } else if (D >= 32 && p.o_vec) {
            // (at d=16 a staging row is 32 bytes: measured 5 % slower than direct stores)
            write_o_staged<D>(p, slot_slice(wk, wq), row0, o, l, stage, valid, lane);
        } else if (row < seq_len) {
            write_o_global<D>(p, slot_slice(wk, wq), row, o, l);
        }
        fence_proxy_async_smem();  // the staging accesses precede the slot's next TMA write
        __syncwarp();
        // (q_full(it) has completed: this pipeline's QK of the item needed it.)
        if (lane == 0) mbar_arrive(b.q_empty(it & 1));
        ph ^= static_cast<uint32_t>(n) & 1u;
    }
}

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
template <int D, bool kTma, bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_sm100(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ FlashParams p) {
    using L = SmemLayout<D>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
    volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(smem + L::kOffAbort);
    const Bars<D> b{sbase};

    if (threadIdx.x == 0) {
        for (int q = 0; q < 2; ++q) {
            mbar_init(b.q_full(q), 1);
            // one arrival per MMA warp (its last QK) and per softmax warp (its
            // epilogue staged O through its Q tile) and item
            mbar_init(b.q_empty(q), kQTiles + 4 * kQTiles);
        }
        for (int s = 0; s < L::kStages; ++s) {
            mbar_init(b.k_full(s), 1);
            mbar_init(b.v_full(s), 1);
            mbar_init(b.kv_empty(s), kQTiles);  // one arrival per MMA warp
        }
        for (int w = 0; w < kQTiles; ++w) {
            mbar_init(b.s_full(w), 1);
            mbar_init(b.s_free(w), 4);  // one arrival per softmax warp
            mbar_init(b.p_full(w), 4);
            mbar_init(b.o_done(w), 1);
            mbar_init(b.o_free(w), 4);
            mbar_init(b.drain(w), 1);
        }
        for (int c = 0; c < kClcSlots; ++c) {
            mbar_init(b.clc_full(c), 1);
            mbar_init(b.clc_empty(c), kClcReaders);  // one arrival per reader warp
        }
        for (int q = 0; q < 4; ++q) {
            mbar_init(b.merge_ready(q), 1);
            mbar_init(b.merge_done(q), 1);
        }
        *abort_flag = 0u;
        mbar_fence_init();
    }
    if (kTma && warp == 0 && lane == 0) {
        tma_prefetch_map(&tmap_q);
        tma_prefetch_map(&tmap_k);
        tma_prefetch_map(&tmap_v);
    }
    if (warp == 1) {
        tmem_alloc(sbase + L::kOffTmemSlot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + L::kOffTmemSlot);

    if (warp == 0) {
        if constexpr (kTma) {
            producer_tma<D>(p, &tmap_q, &tmap_k, &tmap_v, sbase, abort_flag, lane);
        } else {
            producer_lsu<D>(p, smem, sbase, abort_flag, lane);
        }
        __syncwarp();
    } else if (warp == 1 || warp == 2) {
        mma_role<D, kBf16>(p, warp - 1, sbase, tmem, abort_flag, lane);
    } else if (warp >= 4) {
        softmax_role<D, kBf16>(p, smem, sbase, tmem, abort_flag, warp, lane);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// split-KV combine: one warp per (slice, row), D/32 .. 2 columns per lane
// ---------------------------------------------------------------------------
constexpr int kMaxSplits = 8;

// O = sum_i 2^(m_i - M) O_i / sum_i 2^(m_i - M) l_i over the splits whose K
// range the row reaches, M = max_i m_i (the flash-decoding reduction of the
// per-split online-softmax states).  All splits' loads are issued together.
template <int D>
__global__ void __launch_bounds__(256) combine_splits(const __grid_constant__ FlashParams p) {
    constexpr int kPer = D >= 32 ? D / 32 : 1;  // columns per lane
    constexpr int kLanes = D / kPer;
    const int lane = static_cast<int>(threadIdx.x & 31);
    const long long rid = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (rid >= static_cast<long long>(p.batch_heads) * p.seq_len) return;
    const int slice = static_cast<int>(rid / p.seq_len), row = static_cast<int>(rid % p.seq_len);
    const int n_kv = (p.seq_len + kBlockN - 1) / kBlockN;
    const int total = p.causal ? row / kBlockN + 1 : n_kv;  // K tiles of this row's Q tile
    const int splits = min(p.num_splits, (total + p.kv_per_split - 1) / p.kv_per_split);
    const long long stride = static_cast<long long>(p.batch_heads) * p.seq_len;  // rows per split
    const long long idx0 = static_cast<long long>(slice) * p.seq_len + row;
    float2 ml[kMaxSplits];
    float part[kMaxSplits][kPer];
#pragma unroll
    for (int i = 0; i < kMaxSplits; ++i) {
        const bool on = i < splits;
        ml[i] = on ? __ldg(reinterpret_cast<const float2 *>(p.part_ml) + idx0 + i * stride) : make_float2(-INFINITY, 0.0f);
#pragma unroll
        for (int c = 0; c < kPer; ++c)
            part[i][c] = on && lane < kLanes ? __ldg(p.part_o + (idx0 + i * stride) * D + lane * kPer + c) : 0.0f;
    }
    float mmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxSplits; ++i) mmax = fmaxf(mmax, ml[i].x);
    float acc[kPer];
#pragma unroll
    for (int c = 0; c < kPer; ++c) acc[c] = 0.0f;
    float lsum = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxSplits; ++i) {
        if (i < splits) {
            const float wgt = ex2_approx(ml[i].x - mmax);
            lsum += wgt * ml[i].y;
#pragma unroll
            for (int c = 0; c < kPer; ++c) acc[c] += wgt * part[i][c];
        }
    }
    if (lane >= kLanes) return;
    const float inv = 1.0f / lsum;
    const long long base = slice * p.o_stride + static_cast<long long>(row) * p.o_row + lane * kPer;
#pragma unroll
    for (int c = 0; c < kPer; ++c) {
        if (p.o_dtype == 1) {
            reinterpret_cast<__half *>(p.o)[base + c] = __float2half_rn(acc[c] * inv);
        } else if (p.o_dtype == 2) {
            reinterpret_cast<__nv_bfloat16 *>(p.o)[base + c] = __float2bfloat16_rn(acc[c] * inv);
        } else {
            reinterpret_cast<float *>(p.o)[base + c] = acc[c] * inv;
        }
    }
}

}  // namespace ncz
