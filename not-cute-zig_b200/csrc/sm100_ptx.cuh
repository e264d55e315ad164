// sm100_ptx.cuh -- hand-written PTX wrappers for the sm_100a primitives used by
// the flash-attention forward kernel: mbarriers, TMA tensor loads, cluster
// launch control, the tcgen05 family (TMEM alloc/dealloc, MMA, commit, ld/st,
// fences) and the UMMA descriptor builders.  Everything here is device code for sm_100a only.
//
// Descriptor encodings (PTX ISA, tcgen05 "shared memory descriptor" and
// "instruction descriptor" tables):
//   smem descriptor: [0,14) start addr >> 4, [16,30) LBO >> 4, [32,46) SBO >> 4,
//                    [46,48) version = 1, [49,52) base offset, [52] LBO mode,
//                    [61,64) layout (0 none, 2 = 128B, 4 = 64B, 6 = 32B swizzle)
//   instr descriptor (kind::f16): [4,6) D type (1 = f32), [7,10) A type
//                    (0 = f16), [10,13) B type, [15] A MN-major, [16] B MN-major,
//                    [17,23) N >> 3, [24,29) M >> 4
#pragma once
#include <cstdint>
#include <cuda.h>

namespace ncz {

// --------------------------------------------------------------------------
// descriptors (host + device)
// --------------------------------------------------------------------------
__host__ __device__ constexpr uint64_t umma_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes,
                                                      uint32_t sbo_bytes, uint32_t layout) {
    return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) |
           ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
           ((uint64_t)(layout & 7u) << 61);
}

__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(uint32_t m, uint32_t n, uint32_t a_mn_major,
                                                          uint32_t b_mn_major, uint32_t bf16 = 0) {
    return (1u << 4)                                     // D = f32
           | ((bf16 & 1u) << 7) | ((bf16 & 1u) << 10)    // A, B = f16 (0) or bf16 (1), always alike
           | ((a_mn_major & 1u) << 15) | ((b_mn_major & 1u) << 16) |
           (((n >> 3) & 0x3Fu) << 17) | (((m >> 4) & 0x1Fu) << 24);
}

// Byte offset at which logical byte `off` of a tile with `span`-byte rows
// (span = the TMA / UMMA swizzle width: 32, 64 or 128) is stored: the 16-byte
// chunk index (bits 4..) is XORed with the row phase (bits 7..), i.e.
// CuTe's Swizzle<log2(span/16), 4, 3>.  Tiles are 1024-byte aligned, so the
// pattern on offsets equals the hardware's pattern on addresses.
__host__ __device__ constexpr uint32_t tma_swizzle(uint32_t span, uint32_t off) {
    return off ^ (((off >> 7) & ((span >> 4) - 1u)) << 4);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// SM cycle counter: cheap to read (the chip-wide %globaltimer is not), used
// to bound spin-waits.
__device__ __forceinline__ uint64_t sm_clock() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
    return t;
}

// --------------------------------------------------------------------------
// mbarrier
// --------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking probe: true when the phase with `parity` has completed.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// --------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// --------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x,
                                            int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (tensor core, TMA, launch-control) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// --------------------------------------------------------------------------
// Cluster launch control (sm_100): cancel a CTA of this grid that has not
// started yet and take over its work.  The 16-byte response is written to
// shared memory `resp` (16-byte aligned) and completes 16 bytes of
// transaction on `bar`; one elected lane arms the barrier and issues the
// request.  Single-CTA form (no multicast).
// --------------------------------------------------------------------------
__device__ __forceinline__ void clc_try_cancel_elect(uint32_t resp, uint32_t bar) {
    asm volatile(
        "{\n"
        ".reg .pred e;\n"
        "elect.sync _|e, -1;\n"
        "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], 16;\n"
        "@e clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];\n"
        "}\n" ::"r"(resp),
        "r"(bar)
        : "memory");
}
// blockIdx.x of the CTA a response cancelled, or -1 when the request found
// no CTA left to cancel.
__device__ __forceinline__ int clc_decode(uint32_t resp) {
    uint32_t x = 0, valid;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        ".reg .b128 r;\n"
        "ld.shared.b128 r, [%2];\n"
        "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n"
        "selp.u32 %1, 1, 0, p;\n"
        "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, r;\n"
        "}\n"
        : "+r"(x), "=r"(valid)
        : "r"(resp)
        : "memory");
    return valid ? static_cast<int>(x) : -1;
}

// --------------------------------------------------------------------------
// tcgen05
// --------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on `bar` when every tcgen05 async operation issued so far by
// this thread has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// Warp-collective forms: the whole (converged) warp executes them and
// elect.sync picks the one lane that issues.  Issuing tcgen05.mma / TMA from a
// converged warp keeps the descriptors in uniform registers; issuing from a
// single diverged lane measured 3-5x slower per MMA on B200.
__device__ __forceinline__ void umma_ss_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p, e;\n"
        "elect.sync _|e, -1;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p, e;\n"
        "elect.sync _|e, -1;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// S = Q K^T over head_dim: kSteps SS MMAs along K (descriptors advance by 32 bytes
// = 2 in the encoded start address), first one overwrites D.
template <int kSteps>
__device__ __forceinline__ void umma_ss_chain_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
    static_assert(kSteps >= 1 && kSteps <= 4, "K steps");
    const uint64_t a1 = a_desc + 2, a2 = a_desc + 4, a3 = a_desc + 6;
    const uint64_t b1 = b_desc + 2, b2 = b_desc + 4, b3 = b_desc + 6;
    if constexpr (kSteps == 1) {
        asm volatile(
            "{\n.reg .pred e;\nelect.sync _|e, -1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;\n}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc)
            : "memory");
    } else if constexpr (kSteps == 2) {
        asm volatile(
            "{\n.reg .pred e;\nelect.sync _|e, -1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %5, %3, 1;\n}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "l"(a1), "l"(b1)
            : "memory");
    } else {
        asm volatile(
            "{\n.reg .pred e;\nelect.sync _|e, -1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %5, %3, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %7, %3, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %9, %3, 1;\n}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "l"(a1), "l"(b1), "l"(a2), "l"(b2), "l"(a3), "l"(b3)
            : "memory");
    }
}
// O (+)= P V over kSteps key steps: A = P from TMEM (8 columns per step), B = V
// descriptor advancing by `b_step` (encoded units) per step.  `accumulate`
// applies to the first step; later steps always accumulate.
template <int kSteps>
__device__ __forceinline__ void umma_ts_chain_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                   uint64_t b_step, uint32_t idesc, uint32_t accumulate) {
    static_assert(kSteps == 4 || kSteps == 8, "key steps");
    uint64_t b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = b_desc + b_step * i;
    if constexpr (kSteps == 4) {
        asm volatile(
            "{\n.reg .pred p, e;\nelect.sync _|e, -1;\nsetp.ne.b32 p, %3, 0;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %4, %2, p;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %6, %2, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %8, %2, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], %10, %2, 1;\n}\n" ::"r"(d_tmem),
            "r"(a_tmem), "r"(idesc), "r"(accumulate), "l"(b[0]), "r"(a_tmem + 8), "l"(b[1]), "r"(a_tmem + 16),
            "l"(b[2]), "r"(a_tmem + 24), "l"(b[3])
            : "memory");
    } else {
        asm volatile(
            "{\n.reg .pred p, e;\nelect.sync _|e, -1;\nsetp.ne.b32 p, %3, 0;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %4, %2, p;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %6, %2, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %8, %2, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], %10, %2, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%11], %12, %2, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%13], %14, %2, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%15], %16, %2, 1;\n"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%17], %18, %2, 1;\n}\n" ::"r"(d_tmem),
            "r"(a_tmem), "r"(idesc), "r"(accumulate), "l"(b[0]), "r"(a_tmem + 8), "l"(b[1]), "r"(a_tmem + 16),
            "l"(b[2]), "r"(a_tmem + 24), "l"(b[3]), "r"(a_tmem + 32), "l"(b[4]), "r"(a_tmem + 40), "l"(b[5]),
            "r"(a_tmem + 48), "l"(b[6]), "r"(a_tmem + 56), "l"(b[7])
            : "memory");
    }
}
__device__ __forceinline__ void umma_commit_elect(uint32_t bar) {
    asm volatile(
        "{\n"
        ".reg .pred e;\n"
        "elect.sync _|e, -1;\n"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n"
        "}\n" ::"r"(bar)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_elect(uint32_t bar, uint32_t bytes) {
    asm volatile(
        "{\n"
        ".reg .pred e;\n"
        "elect.sync _|e, -1;\n"
        "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n"
        "}\n" ::"r"(bar),
        "r"(bytes)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_elect(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y,
                                                  int z) {
    asm volatile(
        "{\n"
        ".reg .pred e;\n"
        "elect.sync _|e, -1;\n"
        "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];\n"
        "}\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// TMEM <-> register moves, shape 32x32b: thread i of the warp moves lane
// (taddr.lane + i), columns [taddr.col, taddr.col + N).  The *_wait loads
// include tcgen05.wait::ld so the outputs are valid when the asm ends.
__device__ __forceinline__ void tmem_ld_x16_wait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_x32_wait(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_x64_wait(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_x128_wait(uint32_t taddr, uint32_t (&r)[128]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st_x64(uint32_t taddr, const uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};\n"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
        : "memory");
}

__device__ __forceinline__ void tmem_ld_x8_wait(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
        : "memory");
}

__device__ __forceinline__ void tmem_ld_x32_async(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// Waits for the asynchronous loads of a and b; both arrays are in/out operands,
// so no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld_2x32(uint32_t (&a)[32], uint32_t (&b)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]), "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]), "+r"(a[16]), "+r"(a[17]), "+r"(a[18]), "+r"(a[19]), "+r"(a[20]), "+r"(a[21]), "+r"(a[22]), "+r"(a[23]), "+r"(a[24]), "+r"(a[25]), "+r"(a[26]), "+r"(a[27]), "+r"(a[28]), "+r"(a[29]), "+r"(a[30]), "+r"(a[31]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15]), "+r"(b[16]), "+r"(b[17]), "+r"(b[18]), "+r"(b[19]), "+r"(b[20]), "+r"(b[21]), "+r"(b[22]), "+r"(b[23]), "+r"(b[24]), "+r"(b[25]), "+r"(b[26]), "+r"(b[27]), "+r"(b[28]), "+r"(b[29]), "+r"(b[30]), "+r"(b[31]) : : "memory");
}

// Asynchronous form: the registers are written when tcgen05.wait::ld
// completes; tmem_wait_ld_x64 takes them as in/out operands so no use can be
// scheduled before the wait.
__device__ __forceinline__ void tmem_ld_x64_async(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld_x64(uint32_t (&r)[64]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]), "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]), "+r"(r[36]), "+r"(r[37]), "+r"(r[38]), "+r"(r[39]), "+r"(r[40]), "+r"(r[41]), "+r"(r[42]), "+r"(r[43]), "+r"(r[44]), "+r"(r[45]), "+r"(r[46]), "+r"(r[47]), "+r"(r[48]), "+r"(r[49]), "+r"(r[50]), "+r"(r[51]), "+r"(r[52]), "+r"(r[53]), "+r"(r[54]), "+r"(r[55]), "+r"(r[56]), "+r"(r[57]), "+r"(r[58]), "+r"(r[59]), "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63]) : : "memory");
}

// --------------------------------------------------------------------------
// scalar helpers
// --------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Packed f32x2 arithmetic (sm_100): two lanes of f32 per 64-bit register.
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// 2^e0, 2^e1 on the FMA pipe (no MUFU), for e <= 8:
//   e = n + f with n = rint(e) (the 1.5 * 2^23 rounding trick) and f in [-1/2, 1/2];
//   2^f ~ 1 + c1 f + c2 f^2 + c3 f^3 + c4 f^4, coefficients fitted here by a Remez
//   exchange for minimax relative error on [-1/2, 1/2] with the constant term held
//   at 1 (so 2^0 == 1 exactly); max relative error 3.7e-6 in f32;
//   2^n is added to the exponent field as an integer (n << 23).
// e is clamped to >= -125 so the exponent never underflows; -inf gives 2^-125.
__device__ __forceinline__ void exp2_poly_x2(float e0, float e1, float &p0, float &p1) {
    constexpr float kC1 = 0.6931135654449463f, kC2 = 0.2402070313692093f;
    constexpr float kC3 = 0.05597792938351631f, kC4 = 0.009784870781004429f;
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
    e0 = fmaxf(e0, -125.0f);
    e1 = fmaxf(e1, -125.0f);
    const uint64_t e = pack_f32x2(e0, e1);
    const uint64_t t = fadd2(e, pack_f32x2(kRound, kRound));          // low mantissa bits hold n
    const uint64_t n = fadd2(t, pack_f32x2(-kRound, -kRound));        // n as float
    const uint64_t f = ffma2(n, pack_f32x2(-1.0f, -1.0f), e);         // e - n, exact
    uint64_t q = ffma2(f, pack_f32x2(kC4, kC4), pack_f32x2(kC3, kC3));
    q = ffma2(q, f, pack_f32x2(kC2, kC2));
    q = ffma2(q, f, pack_f32x2(kC1, kC1));
    q = ffma2(q, f, pack_f32x2(1.0f, 1.0f));
    float q0, q1, t0, t1;
    unpack_f32x2(q, q0, q1);
    unpack_f32x2(t, t0, t1);
    p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
    p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}
// 2^e0, 2^e1 on the FMA pipe with a degree-3 polynomial: the same range
// reduction and exponent merge as exp2_poly_x2, with
//   2^f ~ 1 + c1 f + c2 f^2 + c3 f^3 on [-1/2, 1/2], constant term held at 1,
// coefficients fitted here by linear programming for minimax relative error
// on 20001 points (max relative error 1.02e-4 in f32 arithmetic: a fifth of
// the f16 unit roundoff, enough for weights that are rounded to f16 or bf16
// before PV).  e is clamped to >= -125 as there.
__device__ __forceinline__ void exp2_poly3_x2(float e0, float e1, float &p0, float &p1) {
    constexpr float kC1 = 0.6932827234268188f, kC2 = 0.24221104383468628f, kC3 = 0.05500970408320427f;
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
    e0 = fmaxf(e0, -125.0f);
    e1 = fmaxf(e1, -125.0f);
    const uint64_t e = pack_f32x2(e0, e1);
    const uint64_t t = fadd2(e, pack_f32x2(kRound, kRound));          // low mantissa bits hold n
    const uint64_t n = fadd2(t, pack_f32x2(-kRound, -kRound));        // n as float
    const uint64_t f = ffma2(n, pack_f32x2(-1.0f, -1.0f), e);         // e - n, exact
    uint64_t q = ffma2(f, pack_f32x2(kC3, kC3), pack_f32x2(kC2, kC2));
    q = ffma2(q, f, pack_f32x2(kC1, kC1));
    q = ffma2(q, f, pack_f32x2(1.0f, 1.0f));
    float q0, q1, t0, t1;
    unpack_f32x2(q, q0, q1);
    unpack_f32x2(t, t0, t1);
    p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
    p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}
// Packs two floats into f16x2 (round to nearest even): `lo` in bits 0..15.
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// 16-bit pair of the input type: f16 or bf16, round to nearest even.
template <bool kBf16>
__device__ __forceinline__ uint32_t pack_in_x2(float lo, float hi) {
    if constexpr (kBf16) {
        return pack_bf16x2(lo, hi);
    } else {
        return pack_f16x2(lo, hi);
    }
}

}  // namespace ncz
