// flash_fwd_sm100.cuh -- the sm_100a flash-attention forward kernel.
//
// Replaces the reference's sm_80 kernel family flash_attention_fwd_{opt,v2,
// h64,h64_bn32,h64_causal} (src/flash_opt.zig, src/flash_v2.zig,
// src/flash_h64.zig, src/flash_h64_bn32.zig, src/flash_h64_causal.zig) with one
// warp-specialised kernel, templated on head_dim (16/32/64) and on how tiles
// reach shared memory (TMA, or plain loads for misaligned strides).
//
// Work unit: one CTA per (batch x head slice, pair of 128-row Q tiles).  Q
// tile w (w = 0, 1) covers rows q_base + 128 w .. + 127.  K/V stream through
// a STAGES-deep ring of 128-key tiles shared by both Q tiles.
//
// Warp roles (384 threads):
//   warp 0      producer: TMA or LSU loads of Q, K, V
//   warp 1      TMEM allocator + tcgen05 MMA issuer
//   (both run as whole warps; elect.sync picks the lane that issues)
//   warps 2,3   idle (keep the softmax warpgroups warpgroup-aligned)
//   warps 4-7   softmax for Q tile 0 (thread = row = TMEM lane)
//   warps 8-11  softmax for Q tile 1
//
// TMEM (512 columns): per Q tile w, at column 256 w:
//   S [0,128)   f32 scores of the current K tile     (QK^T, M=128 N=128)
//   P [128,192) f16x2 probabilities, A operand of PV (aliasing nothing)
//   O [192,192+D) f32 output accumulator             (PV, M=128 N=D)
//
// Per K tile j the MMA warp issues S_w = Q_w K_j^T for both tiles, then
// O_w += P_w(j-1) V_(j-1), so the tensor core computes tile j's scores while
// the softmax warps work on tile j-1.  Online softmax (reference:
// src/flash_h64_bn32.zig:139-211) keeps the row max m (log2 domain) and
// row sum l in registers.  O is rescaled in TMEM only when the row max
// grows by more than 2^8 since the last rescale (the exponent base is stale
// by at most 8, so P <= 256 fits f16 and the final O / l is unchanged).
//
// Every mbarrier wait is bounded (kWaitLimitNs).  On expiry the waiter
// records where it gave up in g_ncz_status, raises a CTA-wide abort flag and
// all roles leave their loops; issued copies and MMAs are waited for
// (bounded) before TMEM is freed and the CTA exits.  No trap, no assert.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace ncz {

constexpr int kBlockM = 128;    // rows per Q tile = TMEM lanes
constexpr int kBlockN = 128;    // keys per K/V tile
constexpr int kQTiles = 2;      // Q tiles per CTA
constexpr int kThreads = 384;   // 12 warps
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;        // log2 units
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait
// Exponentials: in every group of kExp2EmuPeriod column pairs, the last
// kExp2EmuCount pairs are computed by a polynomial on the FMA pipe instead of
// the MUFU unit, which is the bottleneck of the softmax at head_dim <= 64.
#ifndef NCZ_EXP2_EMU_PERIOD
#define NCZ_EXP2_EMU_PERIOD 8
#endif
#ifndef NCZ_EXP2_EMU_COUNT
#define NCZ_EXP2_EMU_COUNT 0
#endif
constexpr int kExp2EmuPeriod = NCZ_EXP2_EMU_PERIOD;
constexpr int kExp2EmuCount = NCZ_EXP2_EMU_COUNT;
// 1: the two softmax warps of an SM sub-partition take turns on the MUFU unit.
#ifndef NCZ_EXP_TURNS
#define NCZ_EXP_TURNS 0
#endif
constexpr bool kExpTurns = NCZ_EXP_TURNS != 0;

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
    kSiteTurn = 11,
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
    int num_pairs;   // ceil(seq_len / 256)
    float scale_log2;  // scale * log2(e)
    int causal;
    int o_f16;
    int o_vec;   // 16-byte vector stores of O are aligned
};

template <int D>
struct SmemLayout {
    static constexpr int kSpan = 2 * D;                  // bytes per row = swizzle width
    static constexpr int kTile = kBlockN * kSpan;        // one 128-row tile
    static constexpr int kStages = D == 64 ? 3 : (D == 32 ? 4 : 6);
    static constexpr uint32_t kUmmaLayout = D == 64 ? 2u : (D == 32 ? 4u : 6u);
    static constexpr int kOffQ = 0;
    static constexpr int kOffK = kOffQ + kQTiles * kTile;
    static constexpr int kOffV = kOffK + kStages * kTile;
    static constexpr int kOffBar = kOffV + kStages * kTile;
    // barriers: q_full | k_full[S] | v_full[S] | kv_empty[S] | s_full[2] | s_free[2] | p_full[2] | o_done[2] | drain
    //           | turn[4][2]
    static constexpr int kBarQFull = 0;
    static constexpr int kBarKFull = 1;
    static constexpr int kBarVFull = kBarKFull + kStages;
    static constexpr int kBarKvEmpty = kBarVFull + kStages;
    static constexpr int kBarSFull = kBarKvEmpty + kStages;
    static constexpr int kBarSFree = kBarSFull + 2;
    static constexpr int kBarPFull = kBarSFree + 2;
    static constexpr int kBarODone = kBarPFull + 2;
    static constexpr int kBarDrain = kBarODone + 2;
    // exp-phase hand-off between softmax warps 4+i and 8+i, which share SM sub-partition i
    // (and its MUFU unit): turn[i][w] completes when it is warp (4+4w+i)'s turn.
    static constexpr int kBarTurn = kBarDrain + 1;
    static constexpr int kNumBars = kBarTurn + 8;
    static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
    static constexpr int kOffAbort = kOffTmemSlot + 4;
    static constexpr int kBytes = kOffAbort + 4;
    static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

struct Work {
    int slice;
    int q_base;
    int n[kQTiles];  // K/V tiles each Q tile visits (0 = tile beyond seq_len)
    int n_max;
};

__device__ uint32_t g_ncz_status = 0u;

__device__ __forceinline__ Work make_work(const FlashParams &p) {
    Work wk;
    const int item = static_cast<int>(blockIdx.x);
    // Heaviest (last) Q-tile pairs first: under causal masking they visit the most K tiles.
    const int pair = p.num_pairs - 1 - item / p.batch_heads;
    wk.slice = item % p.batch_heads;
    wk.q_base = pair * (kQTiles * kBlockM);
    const int n_kv = (p.seq_len + kBlockN - 1) / kBlockN;
    wk.n_max = 0;
#pragma unroll
    for (int w = 0; w < kQTiles; ++w) {
        const int q0 = wk.q_base + w * kBlockM;
        // causal (reference tile_end, src/flash_h64_bn32.zig:80-84): K tiles up to the diagonal
        wk.n[w] = q0 >= p.seq_len ? 0 : (p.causal ? q0 / kBlockN + 1 : n_kv);
        wk.n_max = wk.n[w] > wk.n_max ? wk.n[w] : wk.n_max;
    }
    return wk;
}

// Bounded mbarrier wait.  Returns false when the CTA is aborting or the wait
// exceeded kWaitLimitNs (then it raises the abort flag and records the site).
// honor_abort = false is used by teardown waits that must not be skipped.
// The slow loop is out of line; the common already-complete case costs one
// inlined try_wait.
__device__ __noinline__ bool bounded_wait_slow(uint32_t bar, uint32_t parity, volatile uint32_t *abort_flag,
                                               uint32_t site, bool honor_abort) {
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15u) == 0u) {
            if (honor_abort && *abort_flag) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
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
    __device__ __forceinline__ uint32_t q_full() const { return at(L::kBarQFull); }
    __device__ __forceinline__ uint32_t k_full(int s) const { return at(L::kBarKFull + s); }
    __device__ __forceinline__ uint32_t v_full(int s) const { return at(L::kBarVFull + s); }
    __device__ __forceinline__ uint32_t kv_empty(int s) const { return at(L::kBarKvEmpty + s); }
    __device__ __forceinline__ uint32_t s_full(int w) const { return at(L::kBarSFull + w); }
    __device__ __forceinline__ uint32_t s_free(int w) const { return at(L::kBarSFree + w); }
    __device__ __forceinline__ uint32_t p_full(int w) const { return at(L::kBarPFull + w); }
    __device__ __forceinline__ uint32_t o_done(int w) const { return at(L::kBarODone + w); }
    __device__ __forceinline__ uint32_t drain() const { return at(L::kBarDrain); }
    __device__ __forceinline__ uint32_t turn(int sub, int w) const { return at(L::kBarTurn + 2 * sub + w); }
};

// ---------------------------------------------------------------------------
// producer, TMA variant (whole warp; elect.sync picks the issuing lane)
// ---------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ void producer_tma(const CUtensorMap *tq, const CUtensorMap *tk,
                                             const CUtensorMap *tv, uint32_t sbase, const Work &wk,
                                             volatile uint32_t *abort_flag) {
    using L = SmemLayout<D>;
    const Bars<D> b{sbase};
    uint32_t qbytes = 0;
#pragma unroll
    for (int w = 0; w < kQTiles; ++w) qbytes += wk.n[w] > 0 ? L::kTile : 0;
    mbar_arrive_expect_tx_elect(b.q_full(), qbytes);
#pragma unroll
    for (int w = 0; w < kQTiles; ++w)
        if (wk.n[w] > 0)
            tma_load_3d_elect(sbase + L::kOffQ + w * L::kTile, tq, b.q_full(), 0, wk.q_base + w * kBlockM, wk.slice);
    int j = 0;
    for (; j < wk.n_max; ++j) {
        const int st = j % L::kStages;
        if (j >= L::kStages && !warp_wait(b.kv_empty(st), ((j / L::kStages) - 1) & 1, abort_flag, kSiteKvEmpty))
            break;
        mbar_arrive_expect_tx_elect(b.k_full(st), L::kTile);
        tma_load_3d_elect(sbase + L::kOffK + st * L::kTile, tk, b.k_full(st), 0, j * kBlockN, wk.slice);
        mbar_arrive_expect_tx_elect(b.v_full(st), L::kTile);
        tma_load_3d_elect(sbase + L::kOffV + st * L::kTile, tv, b.v_full(st), 0, j * kBlockN, wk.slice);
    }
    // Every issued copy must land before shared memory is released.
    bounded_wait(b.q_full(), 0, abort_flag, kSiteProducerDrain, false);
    for (int t = j - L::kStages < 0 ? 0 : j - L::kStages; t < j; ++t) {
        const int st = t % L::kStages;
        const uint32_t ph = (t / L::kStages) & 1;
        bounded_wait(b.k_full(st), ph, abort_flag, kSiteProducerDrain, false);
        bounded_wait(b.v_full(st), ph, abort_flag, kSiteProducerDrain, false);
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// producer, LSU variant (all 32 lanes): any 2-byte-aligned layout
// ---------------------------------------------------------------------------
// Loads rows row0 .. row0+127 of one slice (rows >= seq_len read as zero)
// into a 1024-byte-aligned tile, in the same swizzled layout TMA produces.
template <int D>
__device__ __forceinline__ void lsu_tile(uint8_t *dst, const uint16_t *src, long long row_stride, int row0,
                                         int seq_len, int lane) {
    constexpr int kChunks = D / 8;  // 16-byte chunks per row
    constexpr uint32_t kSpan = 2 * D;
    for (int idx = lane; idx < kBlockN * kChunks; idx += 32) {
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
__device__ __forceinline__ void producer_lsu(const FlashParams &p, uint8_t *smem, uint32_t sbase, const Work &wk,
                                             volatile uint32_t *abort_flag, int lane) {
    using L = SmemLayout<D>;
    const Bars<D> b{sbase};
    const uint16_t *qs = p.q + wk.slice * p.q_stride;
    const uint16_t *ks = p.k + wk.slice * p.k_stride;
    const uint16_t *vs = p.v + wk.slice * p.v_stride;
#pragma unroll
    for (int w = 0; w < kQTiles; ++w)
        if (wk.n[w] > 0) lsu_tile<D>(smem + L::kOffQ + w * L::kTile, qs, p.q_row, wk.q_base + w * kBlockM, p.seq_len, lane);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(b.q_full());
    for (int j = 0; j < wk.n_max; ++j) {
        const int st = j % L::kStages;
        if (j >= L::kStages && !warp_wait(b.kv_empty(st), ((j / L::kStages) - 1) & 1, abort_flag, kSiteKvEmpty))
            break;
        lsu_tile<D>(smem + L::kOffK + st * L::kTile, ks, p.k_row, j * kBlockN, p.seq_len, lane);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(b.k_full(st));
        lsu_tile<D>(smem + L::kOffV + st * L::kTile, vs, p.v_row, j * kBlockN, p.seq_len, lane);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(b.v_full(st));
    }
}

// ---------------------------------------------------------------------------
// MMA issuer (whole warp; elect.sync picks the issuing lane)
// ---------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ bool issue_pv(int t, const Bars<D> &b, uint32_t sbase, uint32_t tmem, const Work &wk,
                                         volatile uint32_t *abort_flag) {
    using L = SmemLayout<D>;
    const int st = t % L::kStages;
    if (!warp_wait(b.v_full(st), (t / L::kStages) & 1, abort_flag, kSiteVFull)) return false;
    tc_fence_after();
    constexpr uint32_t idesc_pv = umma_idesc_f16_f32(kBlockM, D, 0, 1);  // B = V, MN-major
    // V tile: 128 keys x D, rows of 2D bytes (one swizzle atom wide); 8-row groups 8*span apart.
    const uint64_t vdesc = umma_smem_desc(sbase + L::kOffV + st * L::kTile, L::kTile, 8 * L::kSpan, L::kUmmaLayout);
#pragma unroll
    for (int w = 0; w < kQTiles; ++w) {
        if (t < wk.n[w]) {
            if (!warp_wait(b.p_full(w), t & 1, abort_flag, kSitePFull)) return false;
            tc_fence_after();
            const uint32_t tP = tmem + w * 256 + 128, tO = tmem + w * 256 + 192;
#pragma unroll
            for (int kk = 0; kk < kBlockN / 16; ++kk)
                umma_ts_elect(tO, tP + kk * 8, vdesc + static_cast<uint64_t>((kk * 16 * L::kSpan) >> 4), idesc_pv,
                              (t > 0 || kk > 0) ? 1u : 0u);
            umma_commit_elect(b.o_done(w));
        }
    }
    umma_commit_elect(b.kv_empty(st));
    return true;
}

template <int D>
__device__ __forceinline__ void mma_role(uint32_t sbase, uint32_t tmem, const Work &wk, volatile uint32_t *abort_flag) {
    using L = SmemLayout<D>;
    const Bars<D> b{sbase};
    constexpr uint32_t idesc_qk = umma_idesc_f16_f32(kBlockM, kBlockN, 0, 0);  // both K-major
    bool ok = warp_wait(b.q_full(), 0, abort_flag, kSiteQFull);
    if (ok) tc_fence_after();
    for (int j = 0; ok && j < wk.n_max; ++j) {
        const int st = j % L::kStages;
        ok = warp_wait(b.k_full(st), (j / L::kStages) & 1, abort_flag, kSiteKFull);
        if (!ok) break;
        tc_fence_after();
        const uint64_t kdesc = umma_smem_desc(sbase + L::kOffK + st * L::kTile, 16, 8 * L::kSpan, L::kUmmaLayout);
#pragma unroll
        for (int w = 0; w < kQTiles; ++w) {
            if (ok && j < wk.n[w]) {
                if (j > 0) {
                    ok = warp_wait(b.s_free(w), (j - 1) & 1, abort_flag, kSiteSFree);
                    if (!ok) break;
                    tc_fence_after();
                }
                const uint64_t qdesc =
                    umma_smem_desc(sbase + L::kOffQ + w * L::kTile, 16, 8 * L::kSpan, L::kUmmaLayout);
                const uint32_t tS = tmem + w * 256;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)  // K advance: 32 bytes inside the swizzled row
                    umma_ss_elect(tS, qdesc + 2 * kk, kdesc + 2 * kk, idesc_qk, kk > 0 ? 1u : 0u);
                umma_commit_elect(b.s_full(w));
            }
        }
        if (ok && j > 0) ok = issue_pv<D>(j - 1, b, sbase, tmem, wk, abort_flag);
    }
    if (ok && wk.n_max > 0) issue_pv<D>(wk.n_max - 1, b, sbase, tmem, wk, abort_flag);
    // All issued MMAs must finish before TMEM and shared memory are released.
    umma_commit_elect(b.drain());
    bounded_wait(b.drain(), 0, abort_flag, kSiteMmaDrain, false);
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

template <int D>
__device__ __forceinline__ void load_o_row(uint32_t taddr, float (&o)[D]) {
    if constexpr (D == 64) {
        uint32_t r[64];
        tmem_ld_x64_wait(taddr, r);
#pragma unroll
        for (int i = 0; i < 64; ++i) o[i] = __uint_as_float(r[i]);
    } else if constexpr (D == 32) {
        uint32_t r[32];
        tmem_ld_x32_wait(taddr, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(r[i]);
    } else {
        uint32_t r[16];
        tmem_ld_x16_wait(taddr, r);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = __uint_as_float(r[i]);
    }
}

template <int D>
__device__ __forceinline__ void store_o_row(uint32_t taddr, const float (&o)[D]) {
    if constexpr (D == 64) {
        uint32_t r[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) r[i] = __float_as_uint(o[i]);
        tmem_st_x64(taddr, r);
    } else if constexpr (D == 32) {
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(o[i]);
        tmem_st_x32(taddr, r);
    } else {
        uint32_t r[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(o[i]);
        tmem_st_x16(taddr, r);
    }
}

template <int D>
__device__ __forceinline__ void write_o_global(const FlashParams &p, const Work &wk, int row, const float (&o)[D],
                                               float l) {
    if (p.o_f16) {
        __half *orow = reinterpret_cast<__half *>(p.o) + wk.slice * p.o_stride + static_cast<long long>(row) * p.o_row;
        if (p.o_vec) {
#pragma unroll
            for (int c = 0; c < D; c += 8) {
                uint4 v;
                v.x = pack_f16x2(o[c + 0] / l, o[c + 1] / l);
                v.y = pack_f16x2(o[c + 2] / l, o[c + 3] / l);
                v.z = pack_f16x2(o[c + 4] / l, o[c + 5] / l);
                v.w = pack_f16x2(o[c + 6] / l, o[c + 7] / l);
                *reinterpret_cast<uint4 *>(orow + c) = v;
            }
        } else {
#pragma unroll
            for (int c = 0; c < D; ++c) orow[c] = __float2half_rn(o[c] / l);
        }
    } else {
        float *orow = reinterpret_cast<float *>(p.o) + wk.slice * p.o_stride + static_cast<long long>(row) * p.o_row;
        if (p.o_vec) {
#pragma unroll
            for (int c = 0; c < D; c += 4)
                *reinterpret_cast<float4 *>(orow + c) = make_float4(o[c] / l, o[c + 1] / l, o[c + 2] / l, o[c + 3] / l);
        } else {
#pragma unroll
            for (int c = 0; c < D; ++c) orow[c] = o[c] / l;
        }
    }
}

template <int D>
__device__ __forceinline__ void softmax_role(const FlashParams &p, uint32_t sbase, uint32_t tmem, const Work &wk,
                                             volatile uint32_t *abort_flag, int warp, int lane) {
    const Bars<D> b{sbase};
    const int w = (warp - 4) >> 2;                         // Q tile of this warpgroup
    const int r = static_cast<int>(threadIdx.x) - 128 * (w + 1);  // row inside the tile = TMEM lane
    const uint32_t lane_field = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_field + w * 256;
    const uint32_t tP = tS + 128;
    const uint32_t tO = tS + 192;
    const int n = wk.n[w];
    const int row = wk.q_base + w * kBlockM + r;
    const int seq_len = p.seq_len;
    // Fast path (scale > 0): mask raw scores, exponent = fma(s, scale*log2e, -m).
    // Otherwise scale first, then mask, exponent = fma(x, 1, -m).
    const bool pre_scale = !(p.scale_log2 > 0.0f);
    const float kmul = pre_scale ? 1.0f : p.scale_log2;

    float m = -INFINITY;  // running max of scaled scores, log2 domain (stale by < 8)
    float l = 0.0f;       // running sum of 2^(x - m)
    bool ok = true;
    for (int j = 0; j < n; ++j) {
        ok = warp_wait(b.s_full(w), j & 1, abort_flag, kSiteSFull);
        if (!ok) break;
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

        if (pre_scale) {
#pragma unroll
            for (int c = 0; c < kBlockN; ++c) x[c] *= p.scale_log2;
        }
        // masking (reference: src/flash_h64_bn32.zig:122-135): keys >= seq_len and,
        // under causal masking, keys > row.  Only the last K tile of a Q tile can hold them.
        if (j == n - 1) {
            int lim = seq_len - j * kBlockN;
            if (p.causal) lim = min(lim, row - j * kBlockN + 1);
            if (lim < kBlockN) {
#pragma unroll
                for (int c = 0; c < kBlockN; ++c) x[c] = c < lim ? x[c] : -INFINITY;
            }
        }
        // row max: 8 independent 3-input max chains (short dependency chains)
        // chain i covers x[i], x[8+i], ..., x[120+i]
        static_assert(kBlockN % 16 == 8 || kBlockN % 16 == 0, "tile width");
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = x[i];
#pragma unroll
        for (int c = 8; c + 16 <= kBlockN; c += 16) {
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = fmax3(mx[i], x[c + i], x[c + 8 + i]);
        }
        if constexpr (kBlockN % 16 == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], x[kBlockN - 8 + i]);
        }
        const float m_tile = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], fmax3(mx[5], mx[6], mx[7]))) * kmul;
        const float m_new = fmaxf(m, m_tile);
        const bool need = m_new > m + kRescaleThreshold;
        float m_use = need ? m_new : m;
        m_use = m_use == -INFINITY ? 0.0f : m_use;  // row with nothing visible yet
        const float alpha = ex2_approx(m - m_use);  // 1 when not rescaling, 0 on the first tile
        const float neg_m = -m_use;

        // Exp phase.  Warps 4+i (tile 0) and 8+i (tile 1) share SM sub-partition i and
        // its MUFU unit; they take turns (tile j of warp 4+i, tile j of warp 8+i, tile
        // j+1 of warp 4+i, ...) so one runs its exponentials while the other loads S,
        // reduces the max and stores P.
        const int n_other = wk.n[w ^ 1];
        const int sub = warp & 3;
        if (kExpTurns && (w == 0 ? (j >= 1 && j - 1 < n_other) : (j < n_other))) {
            ok = warp_wait(b.turn(sub, w), (w == 0 ? j - 1 : j) & 1, abort_flag, kSiteTurn);
            if (!ok) break;
        }
        uint32_t pk[kBlockN / 2];
        uint64_t sum2 = 0ull;  // (0.0f, 0.0f)
        const uint64_t kmul2 = pack_f32x2(kmul, kmul), negm2 = pack_f32x2(neg_m, neg_m);
#pragma unroll
        for (int c = 0; c < kBlockN / 2; ++c) {
            float e0, e1, p0, p1;
            unpack_f32x2(ffma2(pack_f32x2(x[2 * c], x[2 * c + 1]), kmul2, negm2), e0, e1);
            if (kExp2EmuPeriod > 0 && c % kExp2EmuPeriod >= kExp2EmuPeriod - kExp2EmuCount) {
                exp2_poly_x2(e0, e1, p0, p1);  // FMA pipe
            } else {
                p0 = ex2_approx(e0);  // MUFU
                p1 = ex2_approx(e1);
            }
            const uint64_t pp = pack_f32x2(p0, p1);
            sum2 = fadd2(sum2, pp);
            pk[c] = pack_f16x2(p0, p1);  // P rounded to f16 (as src/flash_h64_bn32.zig:185)
        }
        __syncwarp();
        if (kExpTurns && (w == 0 ? (j < n_other) : (j + 1 < n_other))) {
            if (lane == 0) mbar_arrive(b.turn(sub, w ^ 1));
        }
        float s0, s1;
        unpack_f32x2(sum2, s0, s1);
        l = l * alpha + (s0 + s1);

        if (j > 0) {
            // PV of the previous tile must be done: it reads P and accumulates into O.
            ok = warp_wait(b.o_done(w), (j - 1) & 1, abort_flag, kSiteODone);
            if (!ok) break;
            tc_fence_after();
            if (__any_sync(0xffffffffu, need)) {
                float o[D];
                load_o_row<D>(tO, o);
#pragma unroll
                for (int c = 0; c < D; ++c) o[c] *= alpha;
                store_o_row<D>(tO, o);
            }
        }
        tmem_st_x64(tP, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(b.p_full(w));
        m = m_use;
    }

    if (ok && n > 0) {
        ok = warp_wait(b.o_done(w), (n - 1) & 1, abort_flag, kSiteODone);
        if (ok) {
            tc_fence_after();
            float o[D];
            load_o_row<D>(tO, o);
            if (row < seq_len) write_o_global<D>(p, wk, row, o, l);
        }
    }
}

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------
template <int D, bool kTma>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_sm100(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ FlashParams p) {
    using L = SmemLayout<D>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
    const Work wk = make_work(p);
    volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(smem + L::kOffAbort);
    const Bars<D> b{sbase};

    if (threadIdx.x == 0) {
        mbar_init(b.q_full(), 1);
        for (int s = 0; s < L::kStages; ++s) {
            mbar_init(b.k_full(s), 1);
            mbar_init(b.v_full(s), 1);
            mbar_init(b.kv_empty(s), 1);
        }
        for (int w = 0; w < kQTiles; ++w) {
            mbar_init(b.s_full(w), 1);
            mbar_init(b.s_free(w), 4);  // one arrival per softmax warp
            mbar_init(b.p_full(w), 4);
            mbar_init(b.o_done(w), 1);
        }
        mbar_init(b.drain(), 1);
        for (int i = 0; i < 8; ++i) mbar_init(b.at(L::kBarTurn + i), 1);
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
            producer_tma<D>(&tmap_q, &tmap_k, &tmap_v, sbase, wk, abort_flag);
        } else {
            producer_lsu<D>(p, smem, sbase, wk, abort_flag, lane);
        }
        __syncwarp();
    } else if (warp == 1) {
        mma_role<D>(sbase, tmem, wk, abort_flag);
    } else if (warp >= 4) {
        softmax_role<D>(p, sbase, tmem, wk, abort_flag, warp, lane);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace ncz
