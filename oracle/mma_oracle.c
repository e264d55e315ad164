/*
 * CPU oracle for the batched 16x8 GEMM with fused epilogue -- TEST
 * INFRASTRUCTURE ONLY.
 *
 * The parity checker for not-cute-zig_b200/csrc/mma_api.cu.  Only tests/ and
 * bench.py's CPU-baseline leg load it; the product library never links or
 * calls it.
 *
 * Restates the reference's CPU references of its mma demo kernels:
 *   - computePipelineReference  src/main.zig:1184-1204 (A: k_iters row-major
 *     16x16 tiles, B: k_iters row-major 16x8 tiles, epilogue none or relu)
 *   - computeMmaReference       src/main.zig:1146-1162 (one tile, B
 *     column-major)
 * extended to the kernels' full argument set (src/kernels.zig:33-141,
 * 290-319): batches with element strides (D shares C's stride), any alpha and
 * beta, and the silu / gelu activations of src/device.zig:57-80 with exp2
 * computed by exp2f instead of the GPU's ex2.approx.
 * Order of operations as in the reference: for each output element an f32
 * sum in ascending K (tile, then k inside the tile), then alpha * acc +
 * beta * c with each product rounded, then the activation.
 *
 * Build: gcc -O2 -fno-fast-math -std=c11 (ISO mode: no FMA contraction),
 * together with flash_oracle.c into liboracle.so (oracle/build.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#pragma STDC FP_CONTRACT OFF

static inline float mma_h2f(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

/* src/device.zig:57-80 (exp2 by exp2f). */
static float mma_activate(float x, uint32_t kind) {
    const float log2e = 1.4426950408889634f;
    if (kind == 1u) return x > 0.0f ? x : 0.0f; /* @max(0.0, x): NaN and -0 give +0 */
    if (kind == 2u) {
        const float t = x * log2e;
        const float e = exp2f(t);
        const float den = 1.0f + e;
        const float q = e / den;
        return x * q;
    }
    if (kind == 3u) {
        const float x1 = 0.044715f * x;
        const float x2 = x1 * x;
        const float x3 = x2 * x;
        const float inner = 0.7978845608f * (x + x3);
        const float two = 2.0f * inner;
        const float e = exp2f(two * log2e);
        const float th = (e - 1.0f) / (e + 1.0f);
        const float half_x = 0.5f * x;
        return half_x * (1.0f + th);
    }
    return x;
}

/* One batch: d[16x8] from a (k_iters tiles of 16x16), b (k_iters tiles of
 * 16x8, row-major K x N, or a single column-major tile when b_col), c. */
static void mma_one(const uint16_t *a, const uint16_t *b, const float *c, float *d, float alpha, float beta,
                    size_t k_iters, uint32_t epilogue, int b_col) {
    for (size_t row = 0; row < 16; ++row) {
        for (size_t col = 0; col < 8; ++col) {
            float acc = 0.0f;
            for (size_t tile = 0; tile < k_iters; ++tile) {
                for (size_t kk = 0; kk < 16; ++kk) {
                    const float av = mma_h2f(a[tile * 256 + row * 16 + kk]);
                    const float bv = b_col ? mma_h2f(b[tile * 128 + col * 16 + kk])
                                           : mma_h2f(b[tile * 128 + kk * 8 + col]);
                    const float prod = av * bv;
                    acc = acc + prod;
                }
            }
            const float lhs = alpha * acc;
            const float rhs = beta * c[row * 8 + col];
            d[row * 8 + col] = mma_activate(lhs + rhs, epilogue);
        }
    }
}

void ncz_oracle_mma(const uint16_t *a, const uint16_t *b, const float *c, float *d, float alpha, float beta,
                    size_t batch_stride_a, size_t batch_stride_b, size_t batch_stride_c, size_t k_iters,
                    uint32_t epilogue, size_t batches, int b_col) {
    for (size_t bt = 0; bt < batches; ++bt)
        mma_one(a + bt * batch_stride_a, b + bt * batch_stride_b, c + bt * batch_stride_c, d + bt * batch_stride_c,
                alpha, beta, k_iters, epilogue, b_col);
}
