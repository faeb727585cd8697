// act.cu — SwiGLU product of a gated MLP, out = silu(gate) * up, computed in
// fp32: from bf16 inputs with one rounding to bf16 (prefill / experts), or on
// fp32 vectors (decode).  Sits between the gate/up and the down dequant
// kernels of an expert or decoder MLP: the reference's Expert.forward
// (draco/models/moe/expert.py:47-49), fused_swiGLU (draco/kernels/ops.py:
// 114-137) and the Llama MLP apply act_fn(gate_proj(x)) * up_proj(x) there.
// HBM-bound: 6 (bf16) or 12 (fp32) bytes per element.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace draco {


__device__ __forceinline__ uint32_t swiglu2(uint32_t g2, uint32_t u2) {
  const float g0 = __uint_as_float(g2 << 16), g1 = __uint_as_float(g2 & 0xFFFF0000u);
  const float u0 = __uint_as_float(u2 << 16), u1 = __uint_as_float(u2 & 0xFFFF0000u);
  __nv_bfloat162 r = __floats2bfloat162_rn(silu_mul(g0, u0), silu_mul(g1, u1));
  return *reinterpret_cast<uint32_t*>(&r);
}

// 8 elements per thread and iteration on 16-byte vectors; the last n % 8
// elements by single threads
__global__ void swiglu_bf16_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u,
                                   uint16_t* __restrict__ o, int64_t n) {
  const int64_t n8 = n >> 3;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const uint4* g4 = reinterpret_cast<const uint4*>(g);
  const uint4* u4 = reinterpret_cast<const uint4*>(u);
  uint4* o4 = reinterpret_cast<uint4*>(o);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += stride) {
    const uint4 a = __ldg(g4 + i), b = __ldg(u4 + i);
    o4[i] = make_uint4(swiglu2(a.x, b.x), swiglu2(a.y, b.y), swiglu2(a.z, b.z), swiglu2(a.w, b.w));
  }
  const int64_t t = (n8 << 3) + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) {
    const float gv = __uint_as_float((uint32_t)g[t] << 16), uv = __uint_as_float((uint32_t)u[t] << 16);
    __nv_bfloat16 r = __float2bfloat16_rn(silu_mul(gv, uv));
    o[t] = *reinterpret_cast<uint16_t*>(&r);
  }
}

cudaError_t launch_swiglu_bf16(const void* gate, const void* up, void* out, int64_t n, cudaStream_t st) {
  const int threads = 256;
  const int64_t want = ((n >> 3) + threads - 1) / threads;
  const int grid = (int)(want < 1 ? 1 : (want > 8 * device_sm_count() ? 8 * device_sm_count() : want));
  swiglu_bf16_kernel<<<grid, threads, 0, st>>>(static_cast<const uint16_t*>(gate), static_cast<const uint16_t*>(up),
                                                static_cast<uint16_t*>(out), n);
  return cudaGetLastError();
}

// Row-counted form: `groups` blocks of [cap_rows, width] bf16 (row-major,
// block g at g * cap_rows * width); only the first rows[g] rows of block g
// (device count, clamped to cap_rows) are computed.  width % 8 == 0.
__global__ void swiglu_bf16_rows_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u,
                                        uint16_t* __restrict__ o, int64_t cap_rows, int64_t width,
                                        const int* __restrict__ rows) {
  const int grp = blockIdx.y;
  const int64_t r = min((int64_t)max(rows[grp], 0), cap_rows);
  const int64_t n8 = r * (width >> 3);
  const int64_t base = (int64_t)grp * cap_rows * (width >> 3);
  const uint4* g4 = reinterpret_cast<const uint4*>(g) + base;
  const uint4* u4 = reinterpret_cast<const uint4*>(u) + base;
  uint4* o4 = reinterpret_cast<uint4*>(o) + base;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 a = g4[i], b = u4[i];
    o4[i] = make_uint4(swiglu2(a.x, b.x), swiglu2(a.y, b.y), swiglu2(a.z, b.z), swiglu2(a.w, b.w));
  }
}

cudaError_t launch_swiglu_bf16_rows(const void* gate, const void* up, void* out, int groups, int64_t cap_rows,
                                    int64_t width, const int* rows, cudaStream_t st) {
  const int threads = 256;
  const int64_t want = (cap_rows * (width >> 3) + threads - 1) / threads;
  const int per = (8 * device_sm_count() + groups - 1) / groups;
  const dim3 grid((unsigned)(want < 1 ? 1 : (want > per ? per : want)), (unsigned)groups);
  swiglu_bf16_rows_kernel<<<grid, threads, 0, st>>>(static_cast<const uint16_t*>(gate),
                                                     static_cast<const uint16_t*>(up), static_cast<uint16_t*>(out),
                                                     cap_rows, width, rows);
  return cudaGetLastError();
}

// RMSNorm of rows of k values: out = x * rsqrt(mean(x^2) + eps) * w, fp32
// arithmetic in the reference's order (draco/kernels/ops.py:29-50); x and out
// fp32 (dtype 0) or bf16 (dtype 1), w fp32.  One warp per row; the sum of
// squares in a fixed order.
template <typename T>
__device__ __forceinline__ float ld_as_f32(const T* p);
template <>
__device__ __forceinline__ float ld_as_f32<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_as_f32<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st_from_f32(float* p, float v) { *p = v; }
__device__ __forceinline__ void st_from_f32(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, const float* __restrict__ w, T* __restrict__ out, int64_t rows,
                               int64_t k, float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * k;
  float ss = 0.f;
  for (int64_t i = lane; i < k; i += 32) {
    const float v = ld_as_f32(xr + i);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.f / sqrtf(ss / (float)k + eps);
  T* orow = out + row * k;
  for (int64_t i = lane; i < k; i += 32) st_from_f32(orow + i, ld_as_f32(xr + i) * inv * w[i]);
}

cudaError_t launch_rmsnorm(const void* x, const float* w, void* out, int64_t rows, int64_t k, float eps, int bf16,
                           cudaStream_t st) {
  const int warps = 8;
  const dim3 grid((unsigned)((rows + warps - 1) / warps));
  if (bf16)
    rmsnorm_kernel<__nv_bfloat16><<<grid, warps * 32, 0, st>>>(static_cast<const __nv_bfloat16*>(x), w,
                                                                static_cast<__nv_bfloat16*>(out), rows, k, eps);
  else
    rmsnorm_kernel<float><<<grid, warps * 32, 0, st>>>(static_cast<const float*>(x), w, static_cast<float*>(out), rows,
                                                       k, eps);
  return cudaGetLastError();
}

// fp32: 4 elements per thread and iteration on 16-byte vectors, the last n % 4
// by single threads
__global__ void swiglu_f32_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ o,
                                  int64_t n) {
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  const float4* u4 = reinterpret_cast<const float4*>(u);
  float4* o4 = reinterpret_cast<float4*>(o);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 a = __ldg(g4 + i), b = __ldg(u4 + i);
    o4[i] = make_float4(silu_mul(a.x, b.x), silu_mul(a.y, b.y), silu_mul(a.z, b.z), silu_mul(a.w, b.w));
  }
  const int64_t t = (n4 << 2) + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) o[t] = silu_mul(g[t], u[t]);
}

cudaError_t launch_swiglu_f32(const float* gate, const float* up, float* out, int64_t n, cudaStream_t st) {
  const int threads = 256;
  const int64_t want = ((n >> 2) + threads - 1) / threads;
  const int grid = (int)(want < 1 ? 1 : (want > 8 * device_sm_count() ? 8 * device_sm_count() : want));
  swiglu_f32_kernel<<<grid, threads, 0, st>>>(gate, up, out, n);
  return cudaGetLastError();
}

}  // namespace draco
