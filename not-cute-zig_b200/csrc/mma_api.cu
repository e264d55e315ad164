// mma_api.cu -- batched 16x8 GEMM with fused epilogue on sm_100a, and its C
// ABI (include/ncz_mma.h).  Drop-in for the reference's mma demo kernels:
// pipelined_mma_matmul (src/kernels.zig:33-141), batched_mma_matmul
// (src/kernels.zig:301-319) and mma_matmul (src/kernels.zig:290-299).
//
// Per batch: D = epilogue(alpha * (A B) + beta * C), A = k_iters 16x16 f16
// tiles, B = k_iters 16x8 f16 tiles, C and D 16x8 f32.  That is about 5.3 FLOP
// per byte moved, far under the ridge of the tensor cores: the kernel is built
// to keep HBM busy, not to feed tcgen05.
//
// One warp per batch, grid-stride over batches.  A warp streams its batches'
// K tiles through a ring of kStages shared-memory stages; a stage holds up to
// kChunk K tiles of A and of B and is filled by two 1D bulk copies
// (cp.async.bulk, single-CTA form, completion counted in bytes on the stage's
// mbarrier).  The ring runs across batch boundaries, so kStages - 1 stages are
// in flight whatever k_iters is.  A unit (one stage) is a chunk of up to
// kChunk K tiles of one batch or, when k_iters <= kChunk, up to kChunk /
// k_iters whole batches, so short problems keep as many bytes in flight as
// long ones.  Each lane's C values of a unit are loaded into registers one
// unit ahead, so the epilogue does not wait on global memory.  Layouts whose
// A/B addresses are not 16-byte multiples fill the same stages with plain
// loads.  Each K tile is one warp
// MMA (m16n8k16, f16 in, f32 accumulate) fed by ldmatrix from the stage: per
// K tile the warp issues three instructions, so it spends its time waiting on
// HBM, not computing (per-lane FMAs needed about 160 instructions per K tile
// and held the kernel to 35-44 % of HBM bandwidth).  Tensor-core MMAs of the
// sm_100 generation (tcgen05) need 64 or more rows sharing one B operand; a
// batch here is 16 rows with its own B.  The epilogue rounds alpha * acc and
// beta * c separately and adds them, as the reference's expression does, then
// applies relu / silu / gelu with the formulas of src/device.zig:57-80 (exp2
// through ex2.approx.ftz.f32).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "driver.cuh"
#include "ncz_flash.h"
#include "ncz_mma.h"
#include "sm100_ptx.cuh"
#include "status.cuh"

namespace nczm {

using ncz::ex2_approx;
using ncz::mbar_arrive_expect_tx;
using ncz::mbar_fence_init;
using ncz::mbar_init;
using ncz::mbar_try_wait;
using ncz::sm_clock;
using ncz::smem_u32;

constexpr int kM = 16, kN = 8, kK = 16;
constexpr uint32_t kTileA = kM * kK * 2;  // bytes of one A tile
constexpr uint32_t kTileB = kK * kN * 2;  // bytes of one B tile
constexpr int kChunk = 4;   // K tiles per stage
// Ring depth and warps per CTA: the throughput follows the warps resident per
// SM (each warp's copies, waits and MMAs are a serial chain), as long as two
// CTAs still fit the register file and shared memory.  Measured on B200 over
// k_iters 1-40: 10 warps x 3 stages (2 x 90 KB, 20 warps per SM) 79-97 % of
// the HBM copy bandwidth; 8 x 4 (16 warps) 68-87 %; deeper rings with fewer
// warps lower still; 11-14 warps spill or hold one CTA per SM.
#ifndef NCZM_STAGES
#define NCZM_STAGES 3
#endif
#ifndef NCZM_WARPS
#define NCZM_WARPS 10
#endif
constexpr int kStages = NCZM_STAGES;
constexpr int kWarps = NCZM_WARPS;  // warps per CTA
constexpr uint32_t kStageA = kChunk * kTileA;
constexpr uint32_t kStageBytes = kStageA + kChunk * kTileB;
constexpr uint32_t kWarpBytes = kStages * kStageBytes;
constexpr uint32_t kOffBars = kWarps * kWarpBytes;
constexpr uint32_t kSmemBytes = kOffBars + kWarps * kStages * 8;
constexpr unsigned long long kWaitLimitCycles = 4000000000ull;  // about 2 s at 2 GHz

struct MmaParams {
    const uint16_t *a, *b;
    const float *c;
    float *d;
    float alpha, beta;
    long long sa, sb, sc;  // batch strides in elements (D uses sc)
    long long batches;
    int k_iters;
    int n_chunks;  // ceil(k_iters / kChunk)
    uint32_t epilogue;
    int bulk;  // A and B chunk addresses are 16-byte aligned: bulk copies
    int vec;   // C and D are 8-byte aligned with an even stride: float2 access
};

__device__ uint32_t g_mma_status = 0u;
__device__ unsigned long long g_mma_wait_limit = kWaitLimitCycles;
// Test hook: warp 0 of CTA 0 expects its first unit's bytes but never copies A,
// so its first stage wait runs out (failure detection without a GPU fault).
__device__ int g_mma_test_drop = 0;

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
                 : "memory");
}

// Bounded wait of a whole warp on a stage barrier; false (warp-uniform) when
// the limit ran out, with the CTA recorded in g_mma_status.
__device__ __forceinline__ bool stage_wait(uint32_t bar, uint32_t parity) {
    bool ok = mbar_try_wait(bar, parity);
    if (!ok) {
        const unsigned long long t0 = sm_clock();
        for (uint32_t it = 1;; ++it) {
            if (mbar_try_wait(bar, parity)) {
                ok = true;
                break;
            }
            if ((it & 15u) == 0u && sm_clock() - t0 > g_mma_wait_limit) {
                atomicCAS(&g_mma_status, 0u, 0x80000000u | (blockIdx.x & 0xFFFFFFu));
                break;
            }
        }
    }
    return __all_sync(0xffffffffu, ok);
}

// src/device.zig:57-80, each operation rounded on its own as there.
__device__ __forceinline__ float activate(float x, uint32_t kind) {
    constexpr float kLog2e = 1.4426950408889634f;
    if (kind == NCZ_EPILOGUE_RELU) return fmaxf(0.0f, x);
    if (kind == NCZ_EPILOGUE_SILU) {
        const float e = ex2_approx(__fmul_rn(x, kLog2e));
        return __fmul_rn(x, __fdiv_rn(e, __fadd_rn(1.0f, e)));
    }
    if (kind == NCZ_EPILOGUE_GELU) {
        const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
        const float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, cube));
        const float e = ex2_approx(__fmul_rn(__fmul_rn(2.0f, inner), kLog2e));
        const float t = __fdiv_rn(__fadd_rn(e, -1.0f), __fadd_rn(e, 1.0f));
        return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
    }
    return x;
}

// kBcol: B tiles column-major (element (k, n) at n * 16 + k: batched_mma_matmul,
// mma_matmul), else row-major K x N (pipelined_mma_matmul).
template <bool kBcol>
#ifndef NCZM_MIN_BLOCKS
#define NCZM_MIN_BLOCKS 2  // two CTAs per SM (the launch's grid assumes them)
#endif
__global__ void __launch_bounds__(kWarps * 32, NCZM_MIN_BLOCKS) mma_gemm(const __grid_constant__ MmaParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
    uint8_t *ring = smem + warp * kWarpBytes;
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t bars = smem_u32(smem + kOffBars) + 8u * kStages * warp;
    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(bars + 8u * s, 1);
        mbar_fence_init();
    }
    __syncwarp();

    const long long gw = static_cast<long long>(blockIdx.x) * kWarps + warp;
    const long long nw = static_cast<long long>(gridDim.x) * kWarps;
    if (gw >= p.batches) return;
    const long long my_batches = (p.batches - 1 - gw) / nw + 1;
    // Units: whole batches packed kChunk / k_iters to a stage when k_iters <=
    // kChunk, else chunks of kChunk K tiles of one batch.
    const bool packed = p.k_iters <= kChunk;
    const int bpu = packed ? kChunk / p.k_iters : 1;  // batches per unit
    const long long units = packed ? (my_batches + bpu - 1) / bpu : my_batches * p.n_chunks;
    struct Unit {
        long long b0;  // first batch (index in this warp's sequence)
        int nb;        // batches in the unit
        int t0, nt;    // K tiles [t0, t0 + nt) of each batch
        bool last;     // the unit ends its batches: epilogue
    };
    auto unit = [&](long long u) {
        Unit x;
        if (packed) {
            x.b0 = u * bpu;
            x.nb = static_cast<int>(min(static_cast<long long>(bpu), my_batches - x.b0));
            x.t0 = 0;
            x.nt = p.k_iters;
            x.last = true;
        } else {
            x.b0 = u / p.n_chunks;
            x.nb = 1;
            x.t0 = static_cast<int>(u % p.n_chunks) * kChunk;
            x.nt = min(kChunk, p.k_iters - x.t0);
            x.last = x.t0 + x.nt == p.k_iters;
        }
        return x;
    };

    // Fills stage u % kStages with unit u: batch i's tiles at stage tile i * nt.
    auto fill = [&](long long u) {
        const Unit x = unit(u);
        const int s = static_cast<int>(u % kStages);
        if (p.bulk) {
            // The warp's reads of this stage's previous unit precede the copy.
            ncz::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                const uint32_t bar = bars + 8u * s;
                mbar_arrive_expect_tx(bar, static_cast<uint32_t>(x.nb * x.nt) * (kTileA + kTileB));
                const bool drop = g_mma_test_drop != 0 && u == 0 && gw == 0;
                for (int i = 0; i < x.nb; ++i) {
                    const long long bw = gw + (x.b0 + i) * nw;
                    const uint32_t j = static_cast<uint32_t>(i * x.nt);
                    if (!drop)
                        bulk_g2s(ring_s + s * kStageBytes + j * kTileA,
                                 p.a + bw * p.sa + static_cast<long long>(x.t0) * (kM * kK), x.nt * kTileA, bar);
                    bulk_g2s(ring_s + s * kStageBytes + kStageA + j * kTileB,
                             p.b + bw * p.sb + static_cast<long long>(x.t0) * (kK * kN), x.nt * kTileB, bar);
                }
            }
            __syncwarp();
        } else {
            __syncwarp();
            for (int i = 0; i < x.nb; ++i) {
                const long long bw = gw + (x.b0 + i) * nw;
                const uint16_t *a = p.a + bw * p.sa + static_cast<long long>(x.t0) * (kM * kK);
                const uint16_t *b = p.b + bw * p.sb + static_cast<long long>(x.t0) * (kK * kN);
                uint16_t *sa = reinterpret_cast<uint16_t *>(ring + s * kStageBytes) + i * x.nt * (kM * kK);
                uint16_t *sb = reinterpret_cast<uint16_t *>(ring + s * kStageBytes + kStageA) + i * x.nt * (kK * kN);
                for (int e = lane; e < x.nt * kM * kK; e += 32) sa[e] = __ldg(a + e);
                for (int e = lane; e < x.nt * kK * kN; e += 32) sb[e] = __ldg(b + e);
            }
            __syncwarp();
        }
    };

    // m16n8k16 accumulator: d0, d1 at row lane/4, columns 2 (lane % 4) + {0, 1};
    // d2, d3 eight rows below.  C in the same places.
    const int r0 = lane >> 2, c0 = (lane & 3) * 2;
    auto load_c = [&](long long u, float (&cv)[kChunk][4]) {
        const Unit x = unit(u);
        if (!x.last) return;
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {  // constant bound: cv stays in registers
            if (i >= x.nb) break;
            const long long base = (gw + (x.b0 + i) * nw) * p.sc + r0 * kN + c0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const long long off = base + h * 8 * kN;
                if (p.vec) {
                    const float2 c2 = __ldg(reinterpret_cast<const float2 *>(p.c + off));
                    cv[i][2 * h] = c2.x, cv[i][2 * h + 1] = c2.y;
                } else {
                    cv[i][2 * h] = __ldg(p.c + off);
                    cv[i][2 * h + 1] = __ldg(p.c + off + 1);
                }
            }
        }
    };

    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float c_next[kChunk][4], c_cur[kChunk][4];
    load_c(0, c_next);
    long long issued = 0;
    for (; issued < units && issued < kStages - 1; ++issued) fill(issued);
    for (long long u = 0; u < units; ++u) {
        if (issued < units) fill(issued++);
#pragma unroll
        for (int i = 0; i < kChunk; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) c_cur[i][e] = c_next[i][e];
        if (u + 1 < units) load_c(u + 1, c_next);
        const int s = static_cast<int>(u % kStages);
        if (p.bulk && !stage_wait(bars + 8u * s, static_cast<uint32_t>((u / kStages) & 1))) {
            // Give up cleanly: every issued copy must land before the CTA exits.
            for (long long v = u; v < issued; ++v) {
                const int sv = static_cast<int>(v % kStages);
                const uint32_t bar = bars + 8u * sv, ph = static_cast<uint32_t>((v / kStages) & 1);
                const unsigned long long t0 = sm_clock();
                while (!mbar_try_wait(bar, ph) && sm_clock() - t0 < g_mma_wait_limit) {
                }
            }
            return;
        }
        const Unit x = unit(u);
        const uint32_t st = ring_s + s * kStageBytes;
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {  // constant bound: c_cur stays in registers
            if (i >= x.nb) break;
            for (int t = 0; t < x.nt; ++t) {
                const int j = i * x.nt + t;  // tile in the stage
                // A (16x16, 32-byte rows): matrices (rows 0-7 | 8-15) x (k 0-7 | 8-15);
                // lane l gives the address of row l % 16, k block l / 16.
                const uint32_t a_addr = st + j * kTileA + (lane & 15) * 32 + (lane >> 4) * 16;
                // B: row-major K x N (16-byte rows of k) is loaded transposed; column-major
                // (32-byte rows of n) as is.  Lanes 0-15 give the row addresses.
                const int l16 = lane & 15;
                const uint32_t b_addr = kBcol ? st + kStageA + j * kTileB + (l16 & 7) * 32 + (l16 >> 3) * 16
                                              : st + kStageA + j * kTileB + l16 * 16;
                uint32_t a0, a1, a2, a3, b0, b1;
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                             : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
                             : "r"(a_addr)
                             : "memory");
                if constexpr (kBcol) {
                    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
                                 : "=r"(b0), "=r"(b1)
                                 : "r"(b_addr)
                                 : "memory");
                } else {
                    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
                                 : "=r"(b0), "=r"(b1)
                                 : "r"(b_addr)
                                 : "memory");
                }
                asm volatile(
                    "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                    "{%8, %9}, {%0, %1, %2, %3};"
                    : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3])
                    : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
            }
            if (!x.last) continue;
            const long long base = (gw + (x.b0 + i) * nw) * p.sc + r0 * kN + c0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // rows r0 and r0 + 8
                const long long off = base + h * 8 * kN;
                const float o0 =
                    activate(__fadd_rn(__fmul_rn(p.alpha, acc[2 * h]), __fmul_rn(p.beta, c_cur[i][2 * h])), p.epilogue);
                const float o1 = activate(
                    __fadd_rn(__fmul_rn(p.alpha, acc[2 * h + 1]), __fmul_rn(p.beta, c_cur[i][2 * h + 1])), p.epilogue);
                if (p.vec) {
                    *reinterpret_cast<float2 *>(p.d + off) = make_float2(o0, o1);
                } else {
                    p.d[off] = o0;
                    p.d[off + 1] = o1;
                }
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] = 0.0f;
        }
    }
}

}  // namespace nczm

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
bool g_attr_done[kMaxDevices][2];
int g_sms[kMaxDevices];

template <bool kBcol>
const void *gemm_kernel() {
    return reinterpret_cast<const void *>(nczm::mma_gemm<kBcol>);
}

template <bool kBcol>
int launch(const nczm::MmaParams &p, void *stream) {
    if (p.batches == 0) return NCZ_SUCCESS;
    const ncz_driver_table &drv = ncz::drv();
    int dev = 0;
    int e = drv.get_device(&dev);
    if (e != cudaSuccess) return ncz::map_cuda_error(e);
    if (dev < 0 || dev >= kMaxDevices) return NCZ_ERROR_INVALID_DEVICE;
    int sms;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_attr_done[dev][kBcol]) {
            e = drv.set_max_dynamic_smem(gemm_kernel<kBcol>(), static_cast<int>(nczm::kSmemBytes));
            if (e != cudaSuccess) return ncz::map_cuda_error(e);
            g_attr_done[dev][kBcol] = true;
        }
        if (g_sms[dev] == 0) {
            int n = 0;
            if (drv.sm_count(dev, &n) != cudaSuccess || n <= 0) n = 148;
            g_sms[dev] = n;
        }
        sms = g_sms[dev];
    }
    // Two CTAs (2 x kWarps warps and their stage rings) per SM; warps stride over batches.
    const long long need = (p.batches + nczm::kWarps - 1) / nczm::kWarps;
    const unsigned grid = static_cast<unsigned>(std::min<long long>(need, 2LL * sms));
    void *args[1] = {const_cast<nczm::MmaParams *>(&p)};
    return ncz::map_cuda_error(
        drv.launch_kernel(gemm_kernel<kBcol>(), grid, nczm::kWarps * 32, nczm::kSmemBytes, stream, args));
}

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int fill_params(nczm::MmaParams &p, const void *a, const void *b, const void *c, void *d, float alpha, float beta,
                size_t sa, size_t sb, size_t sc, size_t k_iters, uint32_t epilogue, size_t batches) {
    if (batches == 0) {
        p.batches = 0;
        return NCZ_SUCCESS;
    }
    if (a == nullptr || b == nullptr || c == nullptr || d == nullptr || k_iters == 0) return NCZ_ERROR_INVALID_VALUE;
    const size_t kMax = static_cast<size_t>(1) << 40;
    if (k_iters > (1u << 24) || batches > kMax || sa > kMax || sb > kMax || sc > kMax) return NCZ_ERROR_OVERFLOW;
    p.a = static_cast<const uint16_t *>(a);
    p.b = static_cast<const uint16_t *>(b);
    p.c = static_cast<const float *>(c);
    p.d = static_cast<float *>(d);
    p.alpha = alpha;
    p.beta = beta;
    p.sa = static_cast<long long>(sa);
    p.sb = static_cast<long long>(sb);
    p.sc = static_cast<long long>(sc);
    p.batches = static_cast<long long>(batches);
    p.k_iters = static_cast<int>(k_iters);
    p.n_chunks = static_cast<int>((k_iters + nczm::kChunk - 1) / nczm::kChunk);
    p.epilogue = epilogue;
    p.bulk = aligned16(a) && aligned16(b) && (sa * 2) % 16 == 0 && (sb * 2) % 16 == 0;
    p.vec = (reinterpret_cast<uintptr_t>(c) & 7u) == 0 && (reinterpret_cast<uintptr_t>(d) & 7u) == 0 && sc % 2 == 0;
    return NCZ_SUCCESS;
}

}  // namespace

extern "C" {

int ncz_mma_matmul_pipelined(const void *a, const void *b, const void *c, void *d, float alpha, float beta,
                             size_t batch_stride_a, size_t batch_stride_b, size_t batch_stride_c,
                             size_t k_iters, uint32_t epilogue, size_t batches, void *stream) {
    nczm::MmaParams p{};
    int st = fill_params(p, a, b, c, d, alpha, beta, batch_stride_a, batch_stride_b, batch_stride_c, k_iters,
                         epilogue, batches);
    if (st != NCZ_SUCCESS) return st;
    return launch<false>(p, stream);
}

int ncz_mma_matmul_batched(const void *a, const void *b, const void *c, void *d, float alpha, float beta,
                           size_t batch_stride_a, size_t batch_stride_b, size_t batch_stride_c, size_t batches,
                           void *stream) {
    nczm::MmaParams p{};
    int st = fill_params(p, a, b, c, d, alpha, beta, batch_stride_a, batch_stride_b, batch_stride_c, 1,
                         NCZ_EPILOGUE_NONE, batches);
    if (st != NCZ_SUCCESS) return st;
    return launch<true>(p, stream);
}

int ncz_mma_matmul(const void *a, const void *b, const void *c, void *d, float alpha, float beta, void *stream) {
    return ncz_mma_matmul_batched(a, b, c, d, alpha, beta, 0, 0, 0, 1, stream);
}

}  // extern "C"

namespace {
// Switches to `device` (-1 = current), runs fn() (a CUDA error number), switches back.
template <class Fn>
int on_device(int device, Fn fn) {
    const ncz_driver_table &drv = ncz::drv();
    int prev = 0;
    int e = drv.get_device(&prev);
    if (e != cudaSuccess) return ncz::map_cuda_error(e);
    const int dev = device >= 0 ? device : prev;
    if (dev != prev && (e = drv.set_device(dev)) != cudaSuccess) return ncz::map_cuda_error(e);
    e = fn();
    if (dev != prev) drv.set_device(prev);
    return ncz::map_cuda_error(e);
}

int set_symbol_on(int device, const void *symbol, const void *value, size_t bytes) {
    return on_device(device, [&] { return ncz::drv().symbol_write(symbol, value, bytes); });
}
}  // namespace

extern "C" {

int ncz_mma_test_set_wait_limit(int device, uint64_t cycles) {
    const unsigned long long v = cycles != 0 ? cycles : nczm::kWaitLimitCycles;
    return set_symbol_on(device, &nczm::g_mma_wait_limit, &v, sizeof(v));
}

int ncz_mma_test_drop_copy(int device, int enable) {
    const int v = enable != 0;
    return set_symbol_on(device, &nczm::g_mma_test_drop, &v, sizeof(v));
}

int ncz_mma_sync_status(int device) {
    uint32_t word = 0;
    const int st = on_device(device, [&] {
        const ncz_driver_table &drv = ncz::drv();
        const void *sym = static_cast<const void *>(&nczm::g_mma_status);
        int e = drv.device_synchronize();
        if (e == cudaSuccess) e = drv.symbol_read(&word, sym, sizeof(word));
        if (e == cudaSuccess && word != 0) {
            const uint32_t zero = 0;
            e = drv.symbol_write(sym, &zero, sizeof(zero));
        }
        return e;
    });
    if (st != NCZ_SUCCESS) return st;
    return word != 0 ? NCZ_ERROR_DEVICE_TIMEOUT : NCZ_SUCCESS;
}

}  // extern "C"

namespace ncz {

void reset_mma_caches() {
    std::lock_guard<std::mutex> lock(g_mu);
    std::memset(g_attr_done, 0, sizeof(g_attr_done));
    std::memset(g_sms, 0, sizeof(g_sms));
}

const char *mma_kernel_label(const void *kernel) {
    if (kernel == gemm_kernel<false>()) return "mma_gemm<row_b>";
    if (kernel == gemm_kernel<true>()) return "mma_gemm<col_b>";
    return nullptr;
}

}  // namespace ncz
