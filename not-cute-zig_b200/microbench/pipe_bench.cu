// pipe_bench.cu -- per-SM throughput of the softmax's instruction classes on
// B200: 16 warps per SM (4 per sub-partition), 8 independent chains per
// thread, so each number is a pipe throughput, not a latency.  Used to size the
// softmax (which pipe bounds one 128-key tile) in flash_fwd_sm100.cuh.
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        not-cute-zig_b200/microbench/pipe_bench.cu -o pipe_bench && ./pipe_bench
#include <cstdio>
#include <cstdint>
#include <cuda_fp16.h>
#include "../csrc/sm100_ptx.cuh"
using namespace ncz;
template <int OP>
__global__ void __launch_bounds__(512, 1) bench(unsigned long long* out, int iters) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float a[8]; uint32_t u[8];
  for (int i = 0; i < 8; ++i) { a[i] = -0.001f * (threadIdx.x + i); u[i] = threadIdx.x * 7 + i; }
  long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (OP == 0) a[i] = ex2_approx(a[i]);                                 // MUFU ex2
      if (OP == 1) u[i] = pack_f16x2(__uint_as_float(u[i]), a[i]);          // cvt.rn.f16x2.f32
      if (OP == 2) a[i] = a[i] + 1.0001f;                                   // FADD
      if (OP == 3) { uint64_t x = pack_f32x2(a[i], __uint_as_float(u[i])); x = ffma2(x, x, x); float p, q; unpack_f32x2(x, p, q); a[i] = p; u[i] = __float_as_uint(q); }  // FFMA2
      if (OP == 4) { float r; asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a[i]), "f"(__uint_as_float(u[i])), "f"(a[(i + 1) & 7])); a[i] = r; }  // 3-input max
      if (OP == 5) { __half2 h = __floats2half2_rn(a[i], __uint_as_float(u[i])); u[i] = *reinterpret_cast<uint32_t*>(&h); }  // cuda_fp16 convert pair
      if (OP == 6) { float r; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(*reinterpret_cast<unsigned short*>(&r)) : "f"(a[i])); a[i] = r + a[i]; }  // scalar cvt f16
      if (OP == 8) { uint32_t r; asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(a[i]), "f"(__uint_as_float(u[i]))); u[i] = r; }
    }
  }
  long long t1 = clock64();
  if (lane == 0) out[blockIdx.x * 16 + warp] = (unsigned long long)(t1 - t0);
  float s = 0.f; uint32_t x = 0; for (int i = 0; i < 8; ++i) { s += a[i]; x ^= u[i]; }
  if (s == 12345.f || x == 0x1234567u) out[148 * 16] = 1;
}
template <int OP> void run(unsigned long long* d, const char* name) {
  const int iters = 4000;
  bench<OP><<<148, 512>>>(d, 10);
  bench<OP><<<148, 512>>>(d, iters);
  cudaError_t e = cudaDeviceSynchronize();
  unsigned long long h[16]; cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  double mx = 0; for (int w = 0; w < 16; ++w) mx = h[w] > mx ? h[w] : mx;
  printf("%-34s err=%d  %.1f ops/clk/SM  (%.2f cyc per warp-instr per SMSP)\n", name, (int)e, 16 * 32.0 * 8 * iters / mx, mx / (4.0 * 8 * iters));
}
int main() {
  unsigned long long* d; cudaMalloc(&d, (148 * 16 + 1) * 8);
  run<0>(d, "ex2.approx.ftz.f32");
  run<1>(d, "cvt.rn.f16x2.f32 (pack)");
  run<2>(d, "add.f32");
  run<3>(d, "fma.rn.f32x2");
  run<4>(d, "max.f32 3-input");
  run<5>(d, "__floats2half2_rn");
  run<6>(d, "cvt.rn.f16.f32 + add");
  run<8>(d, "cvt.rn.bf16x2.f32");
  return 0;
}
