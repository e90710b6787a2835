// Exhaustive check of the quantisers' division-free helpers (csrc/common.cuh) against CUDA's IEEE division:
//   h3::div6_rn(x)  vs __fdiv_rn(x, 6)  over every non-negative finite fp32, both as fp32 and after the e4m3 rounding
//                                        the NVFP4 scale byte gets;
//   h3::e4m3_rcp(b) vs __fdiv_rn(1, max(e4m3(b), 1e-30)) for every scale byte 0..126.
// Prints one line "mismatch_all=.. mismatch_ge_2^-10=.. mismatch_e4m3=.. mismatch_rcp=.." and exits 0 when the run
// itself succeeded (the test reads the counts).
#include <cstdio>
#include "common.cuh"

__global__ void check(unsigned long long* cnt) {
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < 0x7f800000ull;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const float x = __uint_as_float((uint32_t)i);
    const float ref = __fdiv_rn(x, 6.0f), got = h3::div6_rn(x);
    if (__float_as_uint(got) != __float_as_uint(ref)) {
      atomicAdd(&cnt[0], 1ull);
      if (x >= 0.0009765625f) atomicAdd(&cnt[1], 1ull);
      if (h3::e4m3(got) != h3::e4m3(ref)) atomicAdd(&cnt[2], 1ull);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < 127) {
    const uint32_t b = threadIdx.x;
    const float ref = __fdiv_rn(1.0f, fmaxf(h3::e4m3_to_f32(b), 1e-30f));
    if (__float_as_uint(ref) != __float_as_uint(h3::e4m3_rcp(b))) atomicAdd(&cnt[3], 1ull);
  }
}

int main() {
  unsigned long long* cnt = nullptr;
  if (cudaMalloc(&cnt, 4 * sizeof(unsigned long long)) != cudaSuccess) return 2;
  cudaMemset(cnt, 0, 4 * sizeof(unsigned long long));
  check<<<148 * 8, 256>>>(cnt);
  const cudaError_t e = cudaDeviceSynchronize();
  unsigned long long h[4] = {};
  cudaMemcpy(h, cnt, sizeof(h), cudaMemcpyDeviceToHost);
  cudaFree(cnt);
  printf("cuda=%s mismatch_all=%llu mismatch_ge_2^-10=%llu mismatch_e4m3=%llu mismatch_rcp=%llu\n",
         cudaGetErrorString(e), h[0], h[1], h[2], h[3]);
  return e == cudaSuccess ? 0 : 1;
}
