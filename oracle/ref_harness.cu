// ref_harness.cu -- TEST INFRASTRUCTURE ONLY (parity pin for the oracle).
//
// Compiles the reference's own CUDA baseline source where it lies
// (tools/cuda_baselines.cu of not-cute-zig, passed on the include path by
// oracle/build.py; nothing is copied) and exposes its scalar f32 attention
// kernel `flash_tiled_kernel` (tools/cuda_baselines.cu:200-307) through a
// C entry point, so reference outputs can be produced on a GPU box and
// committed as golden fixtures (tests/golden/make_golden.py).  The reference
// program's main() is renamed by -Dmain=... at compile time.
#include "cuda_baselines.cu"

extern "C" int ncz_ref_flash_tiled(const void *q, const void *k, const void *v, float *o, int batch_heads,
                                   int seq_len, int head_dim, int q_stride, int k_stride, int v_stride,
                                   int o_stride, float scale, int causal) {
    // Launch shape of the reference harness: tools/cuda_baselines.cu:668-671.
    dim3 block(32, 16), grid((seq_len + 15) / 16, batch_heads);
    flash_tiled_kernel<<<grid, block>>>(static_cast<const half *>(q), static_cast<const half *>(k),
                                        static_cast<const half *>(v), o, batch_heads, seq_len, head_dim, q_stride,
                                        k_stride, v_stride, o_stride, scale, causal);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return static_cast<int>(e);
}
