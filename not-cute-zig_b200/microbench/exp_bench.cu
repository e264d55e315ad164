// exp_bench.cu -- can the softmax's exponential loop (64 scores per thread:
// fma, ex2, f16 pack, f32 sum) keep the MUFU unit busy with 1, 2 or 4 warps
// per SM sub-partition?  Three orderings of the same work.  The answer sizes
// the softmax warp count in flash_fwd_sm100.cuh.
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        not-cute-zig_b200/microbench/exp_bench.cu -o exp_bench && ./exp_bench
#include <cstdio>
#include <cstdint>
#include <cuda_fp16.h>
#include "../csrc/sm100_ptx.cuh"
using namespace ncz;
constexpr int N = 64;
// variant 0: interleaved (ffma2, 2 ex2, fadd2, pack per pair)
__device__ __forceinline__ float exp_v0(const float (&x)[N], float kmul, float m, uint32_t (&pk)[N / 2]) {
  const uint64_t k2 = pack_f32x2(kmul, kmul), nm = pack_f32x2(-m, -m);
  uint64_t s2 = 0ull;
#pragma unroll
  for (int c = 0; c < N / 2; ++c) {
    float e0, e1; unpack_f32x2(ffma2(pack_f32x2(x[2 * c], x[2 * c + 1]), k2, nm), e0, e1);
    float p0 = ex2_approx(e0), p1 = ex2_approx(e1);
    s2 = fadd2(s2, pack_f32x2(p0, p1)); pk[c] = pack_f16x2(p0, p1);
  }
  float a, b; unpack_f32x2(s2, a, b); return a + b;
}
// variant 1: all exps first in place, then sums (4 chains) and packs
__device__ __forceinline__ float exp_v1(float (&x)[N], float kmul, float m, uint32_t (&pk)[N / 2]) {
  const uint64_t k2 = pack_f32x2(kmul, kmul), nm = pack_f32x2(-m, -m);
#pragma unroll
  for (int c = 0; c < N / 2; ++c) { float e0, e1; unpack_f32x2(ffma2(pack_f32x2(x[2 * c], x[2 * c + 1]), k2, nm), e0, e1); x[2 * c] = ex2_approx(e0); x[2 * c + 1] = ex2_approx(e1); }
  uint64_t s2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int c = 0; c < N / 2; ++c) { s2[c & 3] = fadd2(s2[c & 3], pack_f32x2(x[2 * c], x[2 * c + 1])); pk[c] = pack_f16x2(x[2 * c], x[2 * c + 1]); }
  float a, b; unpack_f32x2(fadd2(fadd2(s2[0], s2[1]), fadd2(s2[2], s2[3])), a, b); return a + b;
}
// variant 2: scalar fma, scalar adds with 4 chains
__device__ __forceinline__ float exp_v2(float (&x)[N], float kmul, float m, uint32_t (&pk)[N / 2]) {
  const float nm = -m;
#pragma unroll
  for (int c = 0; c < N; ++c) x[c] = ex2_approx(fmaf(x[c], kmul, nm));
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < N / 2; ++c) { s[c & 3] += x[2 * c] + x[2 * c + 1]; pk[c] = pack_f16x2(x[2 * c], x[2 * c + 1]); }
  return (s[0] + s[1]) + (s[2] + s[3]);
}
template <int V>
__global__ void __launch_bounds__(512, 1) bench(unsigned long long* out, int nwarps, int iters) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= nwarps) return;
  float x0[N]; for (int c = 0; c < N; ++c) x0[c] = 0.01f * ((threadIdx.x * 13 + c * 7) % 97) - 0.5f;
  uint32_t acc = 0; float l = 0.f;
  long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
    float x[N];
#pragma unroll
    for (int c = 0; c < N; ++c) x[c] = x0[c] + l * 1e-30f;   // fresh input each iteration, dependent on l
    uint32_t pk[N / 2];
    float s = V == 0 ? exp_v0(x, 1.4427f, 0.25f, pk) : V == 1 ? exp_v1(x, 1.4427f, 0.25f, pk) : exp_v2(x, 1.4427f, 0.25f, pk);
    l = l * 0.5f + s;
#pragma unroll
    for (int c = 0; c < N / 2; ++c) acc ^= pk[c];
  }
  long long t1 = clock64();
  if (lane == 0) out[blockIdx.x * 16 + warp] = (unsigned long long)(t1 - t0);
  if (acc == 0x1234567u || l == 1.2345f) out[148 * 16] = 1;
}
template <int V> void run(unsigned long long* d, int nw) {
  const int iters = 2000;
  bench<V><<<148, 512>>>(d, nw, 10);
  cudaMemset(d, 0, 148 * 16 * 8);
  bench<V><<<148, 512>>>(d, nw, iters);
  cudaError_t e = cudaDeviceSynchronize();
  unsigned long long h[16]; cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  double mx = 0; for (int w = 0; w < nw; ++w) mx = h[w] > mx ? h[w] : mx;
  double mufu = nw * 32.0 * N * iters / mx;  // ex2 per clk per SM
  printf("variant %d, %2d warps (%d/SMSP): err=%d %.1f cyc per 64-elem row-chunk per warp, MUFU %.1f%% of 16/clk/SM\n", V, nw, nw / 4, (int)e, mx / iters, 100.0 * mufu / 16.0);
}
int main() {
  unsigned long long* d; cudaMalloc(&d, (148 * 16 + 1) * 8);
  for (int nw : {4, 8, 16}) { run<0>(d, nw); run<1>(d, nw); run<2>(d, nw); }
  return 0;
}
