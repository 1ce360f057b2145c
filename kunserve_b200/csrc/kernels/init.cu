// Random-init weight fills (the benchmark configurations use random weights;
// generating 16+ GB of normals on the host would take minutes).  Normals come
// from the Box-Muller transform of two SplitMix64-hashed uniforms per pair.
#include "../common.cuh"
#include "kernels.h"

namespace kus {
namespace init_impl {
KUS_DEVICE uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void fill_normal_kernel(__nv_bfloat16* p, long long n, unsigned long long seed, float std) {
  for (long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 2; i < n;
       i += (long long)gridDim.x * blockDim.x * 2) {
    const uint64_t h = mix64(seed ^ mix64((uint64_t)i));
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = ((float)((h >> 16) & 0xFFFFFF) + 0.5f) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * logf(u1)) * std;
    float sn, cs;
    sincosf(6.283185307179586f * u2, &sn, &cs);
    p[i] = f2bf(r * cs);
    if (i + 1 < n) p[i + 1] = f2bf(r * sn);
  }
}

__global__ void fill_value_kernel(__nv_bfloat16* p, long long n, float v) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    p[i] = f2bf(v);
}
}  // namespace init_impl
using namespace init_impl;

void fill_normal_bf16(__nv_bfloat16* p, long long n, unsigned long long seed, float std, cudaStream_t s) {
  if (n <= 0) return;
  fill_normal_kernel<<<4 * 148, 256, 0, s>>>(p, n, seed, std);
}

void fill_value_bf16(__nv_bfloat16* p, long long n, float v, cudaStream_t s) {
  if (n <= 0) return;
  fill_value_kernel<<<4 * 148, 256, 0, s>>>(p, n, v);
}
}  // namespace kus
