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

// one CTA per (token, head): blockIdx.y < heads rotates query head y in
// place, the others rotate key head y - heads into the cache row of the
// token's position and copy the value head beside it; thread j takes the
// rotation pair (j, j + head_dim / 2)
__global__ void __launch_bounds__(128) rope_kv_append_kernel(float* __restrict__ q, const float* __restrict__ k,
                                                             const float* __restrict__ v, float* __restrict__ kc,
                                                             float* __restrict__ vc, const float* __restrict__ cos_t,
                                                             const float* __restrict__ sin_t,
                                                             const int* __restrict__ seq, const int* __restrict__ pos,
                                                             int heads, int kv_heads, int hd, int capacity,
                                                             int n_slots) {
  grid_dependency_wait();  // q, k, v come from the preceding GEMV
  grid_launch_dependents();
  const int i = blockIdx.x, hh = blockIdx.y;
  const int p = pos[i], s = seq[i], half = hd / 2;
  if (p < 0 || p >= capacity || s < 0 || s >= n_slots) return;  // outside the cache: no access
  const float* ct = cos_t + (int64_t)p * half;
  const float* st = sin_t + (int64_t)p * half;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float c = ct[j], sn = st[j];
    if (hh < heads) {
      float* qh = q + ((int64_t)i * heads + hh) * hd;
      const float x1 = qh[j], x2 = qh[j + half];
      qh[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
      qh[j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
    } else {
      const int h = hh - heads;
      const float* kh = k + ((int64_t)i * kv_heads + h) * hd;
      const float* vh = v + ((int64_t)i * kv_heads + h) * hd;
      const int64_t row = (((int64_t)s * kv_heads + h) * capacity + p) * hd;
      const float x1 = kh[j], x2 = kh[j + half];
      kc[row + j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
      kc[row + j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
      vc[row + j] = vh[j];
      vc[row + j + half] = vh[j + half];
    }
  }
}

// Attention in key chunks (flash-decoding): CTA (token i, head h, chunk c)
// handles keys [32c, 32c + 32) of the token's pos + 1 cached keys and writes
// the chunk's max score m, sum of exp(score - m) l and unnormalised output
// o = sum exp(score - m) v to the workspace; a combine kernel merges the
// chunks.  Small chunks give many CTAs, each with short chains of dependent
// loads: scores with four threads per key (16-byte slices of the key row),
// the output with warps over keys and lanes over 16-byte slices of the value
// rows.
constexpr int kAttnThreads = 128;
constexpr int kAttnChunk = 32;

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

// workspace per (token, head, chunk): [m, l, -, -, o[hd]] (hd + 4 floats, so
// that o starts 16-byte aligned)
__global__ void __launch_bounds__(kAttnThreads) attention_chunk_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    const int* __restrict__ seq, const int* __restrict__ pos, float* __restrict__ part, int heads, int kv_heads,
    int hd, int capacity, int n_slots, int max_pos, int n_chunks, float scale) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[kAttnThreads / 32];
  grid_dependency_wait();  // the rotated q and the cache rows of this step
  grid_launch_dependents();
  const int i = blockIdx.x, h = blockIdx.y, c = blockIdx.z;
  float* pt = part + (((int64_t)i * heads + h) * n_chunks + c) * (hd + 4);
  const int s = seq[i];
  const bool ok = pos[i] >= 0 && pos[i] <= max_pos && s >= 0 && s < n_slots;
  const int n_keys = ok ? pos[i] + 1 : 0;
  const int j0 = c * kAttnChunk, j1 = min(j0 + kAttnChunk, n_keys);
  if (j0 >= j1) {  // an empty chunk (or a token outside the cache): contributes nothing
    if (threadIdx.x == 0) pt[0] = -INFINITY, pt[1] = 0.f;
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) pt[4 + d] = 0.f;
    return;
  }
  const int kvh = h / (heads / kv_heads), nf = hd / 4;
  float* qs = sm;       // [hd]
  float* sc = sm + hd;  // [kAttnChunk]
  const float* qh = q + ((int64_t)i * heads + h) * hd;
  for (int d = threadIdx.x; d < hd; d += kAttnThreads) qs[d] = qh[d];
  __syncthreads();
  const float* kb = kc + ((int64_t)s * kv_heads + kvh) * capacity * hd;
  const float* vb = vc + ((int64_t)s * kv_heads + kvh) * capacity * hd;
  // scores: thread 4 kq + part takes the slices f = part, part + 4, ... of
  // key row j0 + kq; the four partial dots meet by two shuffles
  const int kq = (int)threadIdx.x >> 2, part4 = (int)threadIdx.x & 3;
  const int j = j0 + kq;
  float dot = 0.f;
  if (j < j1) {
    const float4* kr = reinterpret_cast<const float4*>(kb + (int64_t)j * hd);
    const float4* q4 = reinterpret_cast<const float4*>(qs);
#pragma unroll 4
    for (int f = part4; f < nf; f += 4) {
      const float4 a = __ldg(kr + f), b = q4[f];
      dot = fmaf(b.x, a.x, fmaf(b.y, a.y, fmaf(b.z, a.z, fmaf(b.w, a.w, dot))));
    }
  }
  dot += __shfl_xor_sync(0xffffffffu, dot, 1);
  dot += __shfl_xor_sync(0xffffffffu, dot, 2);
  const float score = j < j1 ? dot * scale : -INFINITY;
  const float m = block_reduce(score, red, true);
  const float e = j < j1 ? expf(score - m) : 0.f;
  if (part4 == 0) sc[kq] = e;
  const float l = block_reduce(part4 == 0 ? e : 0.f, red, false);  // its barriers also publish sc
  // output: warp w takes keys w, w + 4, ... of the chunk, lane its slices
  // f = lane, lane + 32 of the value row (coalesced, independent loads)
  const int nk = j1 - j0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4 ov[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll 4
  for (int t = warp; t < nk; t += kAttnThreads / 32) {
    const float pr = sc[t];
    const float4* vr = reinterpret_cast<const float4*>(vb + (int64_t)(j0 + t) * hd);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int f = lane + 32 * r;
      if (f < nf) {
        const float4 v4 = __ldg(vr + f);
        ov[r].x = fmaf(pr, v4.x, ov[r].x), ov[r].y = fmaf(pr, v4.y, ov[r].y);
        ov[r].z = fmaf(pr, v4.z, ov[r].z), ov[r].w = fmaf(pr, v4.w, ov[r].w);
      }
    }
  }
  // the four warps' partial rows, summed in warp order
  float4* wp = reinterpret_cast<float4*>(sm + hd + kAttnChunk);  // [4][hd / 4]
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int f = lane + 32 * r;
    if (f < nf) wp[warp * nf + f] = ov[r];
  }
  __syncthreads();
  for (int f = threadIdx.x; f < nf; f += kAttnThreads) {
    float4 o = wp[f];
    for (int w = 1; w < kAttnThreads / 32; ++w) {
      const float4 a = wp[w * nf + f];
      o.x += a.x, o.y += a.y, o.z += a.z, o.w += a.w;
    }
    reinterpret_cast<float4*>(pt + 4)[f] = o;
  }
  if (threadIdx.x == 0) pt[0] = m, pt[1] = l;
}

// out = sum_c exp(m_c - M) o_c / sum_c exp(m_c - M) l_c per (token, head):
// warp 0 forms the chunk weights exp(m_c - M) / L (lanes over chunks), then
// the threads over the head dimension add the chunks' outputs
__global__ void __launch_bounds__(kAttnThreads) attention_combine_kernel(const float* __restrict__ part,
                                                                         float* __restrict__ out, int heads, int hd,
                                                                         int n_chunks) {
  extern __shared__ float wts[];  // [n_chunks]
  grid_dependency_wait();  // the chunks' partials
  grid_launch_dependents();
  const int i = blockIdx.x, h = blockIdx.y;
  const float* pt = part + ((int64_t)i * heads + h) * n_chunks * (hd + 4);
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float M = -INFINITY;
    for (int c = lane; c < n_chunks; c += 32) M = fmaxf(M, pt[(int64_t)c * (hd + 4)]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int c = lane; c < n_chunks; c += 32) {
      const float mc = pt[(int64_t)c * (hd + 4)];
      const float w = mc != -INFINITY ? expf(mc - M) : 0.f;
      wts[c] = w;
      L = fmaf(w, pt[(int64_t)c * (hd + 4) + 1], L);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    const float inv = L > 0.f ? 1.f / L : 0.f;  // a token outside the cache attends to nothing
    __syncwarp();
    for (int c = lane; c < n_chunks; c += 32) wts[c] *= inv;
  }
  __syncthreads();
  float* oh = out + ((int64_t)i * heads + h) * hd;
  for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
    float acc = 0.f;
#pragma unroll 4
    for (int c = 0; c < n_chunks; ++c) acc = fmaf(wts[c], pt[(int64_t)c * (hd + 4) + 4 + d], acc);
    oh[d] = acc;
  }
}

size_t attention_workspace_bytes(int n, int heads, int hd, int max_pos) {
  const int n_chunks = (max_pos + 1 + kAttnChunk - 1) / kAttnChunk;
  return (size_t)n * heads * n_chunks * (hd + 4) * sizeof(float);
}

int attention_launch(int op, float* q, const float* k, const float* v, float* kc, float* vc, const float* cos_t,
                     const float* sin_t, const int* seq, const int* pos, float* out, int n, int heads, int kv_heads,
                     int hd, int capacity, int n_slots, int max_pos, float* part, size_t part_bytes, cudaStream_t st,
                     char* msg, size_t ml) {
  if (n <= 0) return DRACO_OK;
  // programmatic dependent launch: each kernel is scheduled while its
  // predecessor drains and waits (griddepcontrol.wait) before its first read
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
  if (op == 0) {
    cfg.gridDim = dim3(n, heads + kv_heads);
    cfg.blockDim = dim3(128);
    e = cudaLaunchKernelEx(&cfg, rope_kv_append_kernel, q, k, v, kc, vc, cos_t, sin_t, seq, pos, heads, kv_heads, hd,
                           capacity, n_slots);
  } else {
    // positions past max_pos (< capacity) count as outside the cache
    if (hd % 4 || hd > 256) {
      snprintf(msg, ml, "attention: head_dim %d must be a multiple of 4 up to 256", hd);
      return DRACO_ERR_SHAPE;
    }
    const int n_chunks = (max_pos + 1 + kAttnChunk - 1) / kAttnChunk;
    const size_t need = attention_workspace_bytes(n, heads, hd, max_pos);
    if (part == nullptr || part_bytes < need || (reinterpret_cast<uintptr_t>(part) & 15)) {
      snprintf(msg, ml, "attention: workspace of %zu bytes given (16-byte aligned), %zu needed", part_bytes, need);
      return DRACO_ERR_WORKSPACE;
    }
    if ((size_t)n_chunks * sizeof(float) > 48 * 1024) {
      snprintf(msg, ml, "attention: %d cached positions exceed the combine kernel's weight buffer", max_pos + 1);
      return DRACO_ERR_SHAPE;
    }
    cfg.gridDim = dim3(n, heads, n_chunks);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = (size_t)(hd + kAttnChunk + (kAttnThreads / 32) * hd) * sizeof(float);
    e = cudaLaunchKernelEx(&cfg, attention_chunk_kernel, (const float*)q, (const float*)kc, (const float*)vc, seq,
                           pos, part, heads, kv_heads, hd, capacity, n_slots, max_pos, n_chunks,
                           1.f / sqrtf((float)hd));
    if (e == cudaSuccess) {
      cfg.gridDim = dim3(n, heads);
      cfg.dynamicSmemBytes = (size_t)n_chunks * sizeof(float);
      e = cudaLaunchKernelEx(&cfg, attention_combine_kernel, (const float*)part, out, heads, hd, n_chunks);
    }
  }
  if (e != cudaSuccess) {
    snprintf(msg, ml, "attention launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

}  // namespace draco
