// attn.cu — the attention part of a GPU decode step for GGUF llama-family
// models: rotary position embedding with the key/value-cache append, and
// attention of the step's query tokens over their sequences' cached keys.
//
// Replaces, for the GPU decode graph, the reference's CPU pieces:
//   apply_rope / build_rope_cache  (draco/runtime/cpu/ops.py:77-95): rotate-half
//       RoPE, x1' = x1 c - x2 s, x2' = x2 c + x1 s, with the fp32 cos / sin
//       tables the host builds exactly as build_rope_cache does;
//   CPUAttentionBackend.prefill / decode (draco/runtime/cpu/attention.py):
//       append the token's k / v to the cache, then softmax(q K^T / sqrt(d)) V
//       over the cached positions 0..pos (causal), grouped-query heads
//       (query head h reads key/value head h / (heads / kv_heads)), fp32.
//
// Cache layout (per layer): [slot][kv_head][capacity][head_dim] fp32, slot =
// the sequence's cache slot.  Token i of a launch has slot seq[i] and absolute
// position pos[i] (its key goes to row pos[i]).  The rotation uses explicit
// _rn multiplies and adds, so no FMA contraction changes a bit against the
// reference's numpy arithmetic.
#include <cstdio>

#include "common.cuh"
#include "internal.h"

namespace draco {

// one CTA per token: rotate q in place, rotate k and store it and v in the cache
__global__ void __launch_bounds__(256) rope_kv_append_kernel(float* __restrict__ q, const float* __restrict__ k,
                                                             const float* __restrict__ v, float* __restrict__ kc,
                                                             float* __restrict__ vc, const float* __restrict__ cos_t,
                                                             const float* __restrict__ sin_t,
                                                             const int* __restrict__ seq, const int* __restrict__ pos,
                                                             int heads, int kv_heads, int hd, int capacity,
                                                             int n_slots) {
  const int i = blockIdx.x;
  const int p = pos[i], s = seq[i], half = hd / 2;
  if (p < 0 || p >= capacity || s < 0 || s >= n_slots) return;  // outside the cache: no access
  const float* ct = cos_t + (int64_t)p * half;
  const float* st = sin_t + (int64_t)p * half;
  // query heads (in place)
  for (int e = threadIdx.x; e < heads * half; e += blockDim.x) {
    const int h = e / half, j = e - h * half;
    float* qh = q + ((int64_t)i * heads + h) * hd;
    const float x1 = qh[j], x2 = qh[j + half], c = ct[j], sn = st[j];
    qh[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    qh[j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
  }
  // key / value heads into the cache row of this position
  for (int e = threadIdx.x; e < kv_heads * half; e += blockDim.x) {
    const int h = e / half, j = e - h * half;
    const float* kh = k + ((int64_t)i * kv_heads + h) * hd;
    const float* vh = v + ((int64_t)i * kv_heads + h) * hd;
    const int64_t row = (((int64_t)s * kv_heads + h) * capacity + p) * hd;
    const float x1 = kh[j], x2 = kh[j + half], c = ct[j], sn = st[j];
    kc[row + j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    kc[row + j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
    vc[row + j] = vh[j];
    vc[row + j + half] = vh[j + half];
  }
}

constexpr int kAttnThreads = 128;

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();  // red may still be read from the previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < kAttnThreads / 32; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

// one CTA per (token, query head); scores of the pos + 1 cached keys in
// dynamic shared memory
__global__ void __launch_bounds__(kAttnThreads) attention_cached_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    const int* __restrict__ seq, const int* __restrict__ pos, float* __restrict__ out, int heads, int kv_heads,
    int hd, int capacity, int n_slots, int max_pos, float scale) {
  extern __shared__ float sm[];
  __shared__ float red[kAttnThreads / 32];
  const int i = blockIdx.x, h = blockIdx.y;
  const int n_keys = pos[i] + 1, s = seq[i], kvh = h / (heads / kv_heads);
  if (pos[i] < 0 || pos[i] > max_pos || s < 0 || s >= n_slots) {  // outside the cache: zeros
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) out[((int64_t)i * heads + h) * hd + d] = 0.f;
    return;
  }
  float* qs = sm;          // [hd]
  float* sc = sm + hd;     // [n_keys]
  const float* qh = q + ((int64_t)i * heads + h) * hd;
  for (int d = threadIdx.x; d < hd; d += kAttnThreads) qs[d] = qh[d];
  __syncthreads();
  const float* kb = kc + ((int64_t)s * kv_heads + kvh) * capacity * hd;
  const float* vb = vc + ((int64_t)s * kv_heads + kvh) * capacity * hd;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // scores: one warp per key, lanes over the head dimension
  for (int j = warp; j < n_keys; j += kAttnThreads / 32) {
    const float* kr = kb + (int64_t)j * hd;
    float acc = 0.f;
    for (int d = lane; d < hd; d += 32) acc = fmaf(qs[d], kr[d], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) sc[j] = acc * scale;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int j = threadIdx.x; j < n_keys; j += kAttnThreads) m = fmaxf(m, sc[j]);
  m = block_reduce(m, red, true);
  float sum = 0.f;
  for (int j = threadIdx.x; j < n_keys; j += kAttnThreads) {
    const float e = expf(sc[j] - m);
    sc[j] = e;
    sum += e;
  }
  sum = block_reduce(sum, red, false);
  const float inv = 1.f / sum;
  __syncthreads();
  float* oh = out + ((int64_t)i * heads + h) * hd;
  for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
    float acc = 0.f;
    for (int j = 0; j < n_keys; ++j) acc = fmaf(sc[j] * inv, vb[(int64_t)j * hd + d], acc);
    oh[d] = acc;
  }
}

int attention_launch(int op, float* q, const float* k, const float* v, float* kc, float* vc, const float* cos_t,
                     const float* sin_t, const int* seq, const int* pos, float* out, int n, int heads, int kv_heads,
                     int hd, int capacity, int n_slots, int max_pos, cudaStream_t st, char* msg, size_t ml) {
  if (n <= 0) return DRACO_OK;
  if (op == 0) {
    rope_kv_append_kernel<<<n, 256, 0, st>>>(q, k, v, kc, vc, cos_t, sin_t, seq, pos, heads, kv_heads, hd,
                                             capacity, n_slots);
  } else {
    // positions past max_pos (< capacity) are not attended (the kernel zeroes them)
    const size_t smem = (size_t)(hd + max_pos + 1) * sizeof(float);
    if (smem > 200 * 1024) {
      snprintf(msg, ml, "attention: %d cached positions exceed the shared-memory score buffer", max_pos + 1);
      return DRACO_ERR_SHAPE;
    }
    static int attr_dev[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_dev[dev]) {
      const cudaError_t e =
          cudaFuncSetAttribute(attention_cached_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (e != cudaSuccess) {
        snprintf(msg, ml, "attention: %s", cudaGetErrorString(e));
        return DRACO_ERR_CUDA;
      }
      attr_dev[dev] = 1;
    }
    attention_cached_kernel<<<dim3(n, heads), kAttnThreads, smem, st>>>(q, kc, vc, seq, pos, out, heads, kv_heads, hd,
                                                                      capacity, n_slots, max_pos,
                                                                      1.f / sqrtf((float)hd));
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(msg, ml, "attention launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

}  // namespace draco
