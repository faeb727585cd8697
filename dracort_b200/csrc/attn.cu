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
#include <algorithm>
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

// Attention in key chunks (flash-decoding).  CTA (token i, head h, chunk c)
// handles keys [32c, 32c + 32) of the token's pos + 1 keys: thread 0 copies
// the chunk's key and value rows (contiguous in the cache) into shared memory
// with two bulk copies, the CTA forms the scores (four threads per key over
// 16-byte slices), the chunk's max m, sum of exp(score - m) l and
// unnormalised output o = sum exp(score - m) v (warps over keys, lanes over
// 16-byte slices of the value rows).  A token with one chunk writes o / l at
// once; otherwise each chunk stores [m, l, -, -, o] in the workspace and the
// last of the token's chunk CTAs to arrive (a counter per token and head)
// merges them in chunk order: out = sum_c exp(m_c - M) o_c / sum_c exp(m_c -
// M) l_c.  CTAs past the token's last chunk exit at once.
//
// kDecode: q and k arrive unrotated; every CTA rotates q into shared memory,
// and the token's last chunk rotates the new key at pos (it is the only chunk
// that reads row pos) into shared memory, the CTA of the first query head of
// each key/value group also writing it and the value row to the cache.  The
// other rows come from the cache, so in this form the tokens of one launch
// must hold distinct slots (a decode step).
constexpr int kAttnThreads = 128;
constexpr int kAttnChunk = 32;
constexpr uint64_t kAttnWaitNs = 2000000000ull;  // 2 s: far beyond any legitimate copy
constexpr int kAttnSmemMax = 200 * 1024;

// workspace: [status int32, pad to 16 B][counters int32 n * heads, padded to
// 16 B][records n * heads * n_chunks * (hd + 4) floats]
__host__ __device__ inline int64_t attn_counter_bytes(int n, int heads) {
  return ((int64_t)n * heads * 4 + 15) / 16 * 16;
}

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

__device__ __forceinline__ void rope_pair(const float* x, float* y, const float* ct, const float* st, int half) {
  for (int j = threadIdx.x; j < half; j += kAttnThreads) {
    const float c = ct[j], sn = st[j], x1 = x[j], x2 = x[j + half];
    y[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    y[j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
  }
}

template <bool kDecode>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    const float* __restrict__ q, const float* __restrict__ k_new, const float* __restrict__ v_new, float* kc,
    float* vc, const float* __restrict__ cos_t, const float* __restrict__ sin_t, const int* __restrict__ seq,
    const int* __restrict__ pos, float* __restrict__ out, uint8_t* ws, int n, int heads, int kv_heads, int hd,
    int capacity, int n_slots, int max_pos, int n_chunks, float scale) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[kAttnThreads / 32];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int last_flag;
  grid_dependency_wait();  // q (and k, v) come from the preceding kernel
  grid_launch_dependents();
  const int i = blockIdx.x, h = blockIdx.y, c = blockIdx.z;
  const int s = seq[i], p = pos[i];
  const bool ok = p >= 0 && p <= max_pos && s >= 0 && s < n_slots;
  const int nc = ok ? p / kAttnChunk + 1 : 1;  // the token's chunks
  if (c >= nc) return;
  float* oh = out + ((int64_t)i * heads + h) * hd;
  if (!ok) {  // a token outside the cache attends to nothing
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) oh[d] = 0.f;
    return;
  }
  const int group = heads / kv_heads, kvh = h / group, half = hd / 2, nf = hd / 4;
  const int j0 = c * kAttnChunk, j1 = min(j0 + kAttnChunk, p + 1), nk = j1 - j0;
  // the key region also holds the merge's chunk weights
  const int kreg = max(kAttnChunk * hd, (n_chunks + 3) & ~3);
  float* ks = sm;                       // [32][hd] keys of the chunk
  float* vs = sm + kreg;                // [32][hd] values
  float* qs = vs + kAttnChunk * hd;     // [hd]
  float* sc = qs + hd;                  // [32] exp(score - m)
  float4* wp = reinterpret_cast<float4*>(sc + kAttnChunk);  // [4][hd / 4] per-warp partial rows
  const int64_t base = ((int64_t)s * kv_heads + kvh) * capacity * hd;
  // rows copied from the cache: all of the chunk, or in the decode form all
  // but the new key's row
  const int n_copy = (kDecode && j1 == p + 1) ? nk - 1 : nk;
  const uint32_t copy_bytes = (uint32_t)n_copy * hd * 4;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (copy_bytes) {
      mbar_arrive_expect_tx(&bar, 2 * copy_bytes);
      bulk_g2s(ks, kc + base + (int64_t)j0 * hd, copy_bytes, &bar);
      bulk_g2s(vs, vc + base + (int64_t)j0 * hd, copy_bytes, &bar);
    }
  }
  __syncthreads();  // the barrier is initialised before anyone waits on it
  const float* qh = q + ((int64_t)i * heads + h) * hd;
  if (kDecode) {
    const float* ct = cos_t + (int64_t)p * half;
    const float* st = sin_t + (int64_t)p * half;
    rope_pair(qh, qs, ct, st, half);
    if (j1 == p + 1) {  // the new key and value, row p - j0 of the chunk
      const int64_t src = ((int64_t)i * kv_heads + kvh) * hd;
      float* kr = ks + (p - j0) * hd;
      float* vr = vs + (p - j0) * hd;
      rope_pair(k_new + src, kr, ct, st, half);
      for (int d = threadIdx.x; d < hd; d += kAttnThreads) vr[d] = v_new[src + d];
      if (h % group == 0) {  // one CTA per key/value head appends them
        __syncthreads();
        for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
          kc[base + (int64_t)p * hd + d] = kr[d];
          vc[base + (int64_t)p * hd + d] = vr[d];
        }
      }
    }
  } else {
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) qs[d] = qh[d];
  }
  const bool landed = copy_bytes == 0 || mbar_wait_bounded(&bar, 0, kAttnWaitNs);
  if (__syncthreads_or(!landed)) {
    // the copies did not land: record it, give them a second bound to
    // finish, and leave without touching the counters
    if (threadIdx.x == 0) atomicExch(reinterpret_cast<int*>(ws), DRACO_ERR_TIMEOUT);
    if (!landed) mbar_wait_bounded(&bar, 0, kAttnWaitNs);
    return;
  }
  // scores: thread 4 kq + part takes the slices f = part, part + 4, ... of
  // key row kq; the four partial dots meet by two shuffles
  const int kq = (int)threadIdx.x >> 2, part4 = (int)threadIdx.x & 3;
  float dot = 0.f;
  if (kq < nk) {
    const float4* kr = reinterpret_cast<const float4*>(ks + kq * hd);
    const float4* q4 = reinterpret_cast<const float4*>(qs);
#pragma unroll 4
    for (int f = part4; f < nf; f += 4) {
      const float4 a = kr[f], b = q4[f];
      dot = fmaf(b.x, a.x, fmaf(b.y, a.y, fmaf(b.z, a.z, fmaf(b.w, a.w, dot))));
    }
  }
  dot += __shfl_xor_sync(0xffffffffu, dot, 1);
  dot += __shfl_xor_sync(0xffffffffu, dot, 2);
  const float score = kq < nk ? dot * scale : -INFINITY;
  const float m = block_reduce(score, red, true);
  const float e = kq < nk ? expf(score - m) : 0.f;
  if (part4 == 0) sc[kq] = e;
  const float l = block_reduce(part4 == 0 ? e : 0.f, red, false);  // its barriers also publish sc
  // output: warp w takes keys w, w + 4, ... of the chunk, lane its slices
  // f = lane, lane + 32 of the value row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4 ov[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  for (int t = warp; t < nk; t += kAttnThreads / 32) {
    const float pr = sc[t];
    const float4* vr = reinterpret_cast<const float4*>(vs + t * hd);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int f = lane + 32 * r;
      if (f < nf) {
        const float4 v4 = vr[f];
        ov[r].x = fmaf(pr, v4.x, ov[r].x), ov[r].y = fmaf(pr, v4.y, ov[r].y);
        ov[r].z = fmaf(pr, v4.z, ov[r].z), ov[r].w = fmaf(pr, v4.w, ov[r].w);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int f = lane + 32 * r;
    if (f < nf) wp[warp * nf + f] = ov[r];
  }
  __syncthreads();
  if (nc == 1) {  // one chunk: normalise and write
    const float inv = 1.f / l;
    for (int f = threadIdx.x; f < nf; f += kAttnThreads) {
      float4 o = wp[f];
      for (int w = 1; w < kAttnThreads / 32; ++w) {
        const float4 a = wp[w * nf + f];
        o.x += a.x, o.y += a.y, o.z += a.z, o.w += a.w;
      }
      o.x *= inv, o.y *= inv, o.z *= inv, o.w *= inv;
      reinterpret_cast<float4*>(oh)[f] = o;
    }
    return;
  }
  int* cnt = reinterpret_cast<int*>(ws + 16) + (int64_t)i * heads + h;
  float* recs = reinterpret_cast<float*>(ws + 16 + attn_counter_bytes(n, heads)) +
                ((int64_t)i * heads + h) * n_chunks * (hd + 4);
  float* rec = recs + (int64_t)c * (hd + 4);
  for (int f = threadIdx.x; f < nf; f += kAttnThreads) {
    float4 o = wp[f];
    for (int w = 1; w < kAttnThreads / 32; ++w) {
      const float4 a = wp[w * nf + f];
      o.x += a.x, o.y += a.y, o.z += a.z, o.w += a.w;
    }
    __stcg(reinterpret_cast<float4*>(rec + 4) + f, o);
  }
  if (threadIdx.x == 0) __stcg(reinterpret_cast<float2*>(rec), make_float2(m, l));
  __threadfence();  // this thread's record stores before the arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(cnt, 1);
    last_flag = prev == nc - 1;
    if (last_flag) {
      atomicExch(cnt, 0);  // ready for the next launch
      __threadfence();
    }
  }
  __syncthreads();
  if (!last_flag) return;
  // the last chunk CTA merges the token's chunks in chunk order; warp 0
  // forms the weights exp(m_c - M) / L into shared memory (over the keys)
  float* wts = ks;
  if (warp == 0) {
    float M = -INFINITY;
    for (int cc = lane; cc < nc; cc += 32) M = fmaxf(M, __ldcg(recs + (int64_t)cc * (hd + 4)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int cc = lane; cc < nc; cc += 32) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(recs + (int64_t)cc * (hd + 4)));
      const float w = expf(ml.x - M);
      wts[cc] = w;
      L = fmaf(w, ml.y, L);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    const float inv = 1.f / L;
    __syncwarp();
    for (int cc = lane; cc < nc; cc += 32) wts[cc] *= inv;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
    float acc = 0.f;
#pragma unroll 4
    for (int cc = 0; cc < nc; ++cc) acc = fmaf(wts[cc], __ldcg(recs + (int64_t)cc * (hd + 4) + 4 + d), acc);
    oh[d] = acc;
  }
}

size_t attention_workspace_bytes(int n, int heads, int hd, int max_pos) {
  const int n_chunks = (max_pos + 1 + kAttnChunk - 1) / kAttnChunk;
  return 16 + (size_t)attn_counter_bytes(n, heads) + (size_t)n * heads * n_chunks * (hd + 4) * sizeof(float);
}

template <bool kDecode>
static cudaError_t launch_attention(const cudaLaunchConfig_t& cfg0, const float* q, const float* k, const float* v,
                                    float* kc, float* vc, const float* cos_t, const float* sin_t, const int* seq,
                                    const int* pos, float* out, uint8_t* ws, int n, int heads, int kv_heads, int hd,
                                    int capacity, int n_slots, int max_pos, int n_chunks) {
  static int attr_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<kDecode>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kAttnSmemMax);
    if (e != cudaSuccess) return e;
    attr_set[dev] = 1;
  }
  return cudaLaunchKernelEx(&cfg0, attention_kernel<kDecode>, q, k, v, kc, vc, cos_t, sin_t, seq, pos, out, ws, n,
                            heads, kv_heads, hd, capacity, n_slots, max_pos, n_chunks, 1.f / sqrtf((float)hd));
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
    // op 1: cached attention (q rotated, keys in the cache); op 2: the decode
    // form (rotation and append inside).  Positions past max_pos (< capacity)
    // count as outside the cache.
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
    if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15) {
      snprintf(msg, ml, "attention: key/value caches must be 16-byte aligned");
      return DRACO_ERR_ALIGN;
    }
    const int kreg = std::max(kAttnChunk * hd, (n_chunks + 3) & ~3);
    const size_t smem = (size_t)(kreg + kAttnChunk * hd + hd + kAttnChunk + (kAttnThreads / 32) * hd) * sizeof(float);
    if (smem > (size_t)kAttnSmemMax) {
      snprintf(msg, ml, "attention: %d cached positions exceed the merge's weight buffer", max_pos + 1);
      return DRACO_ERR_SHAPE;
    }
    cfg.gridDim = dim3(n, heads, n_chunks);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    uint8_t* ws = reinterpret_cast<uint8_t*>(part);
    e = op == 2 ? launch_attention<true>(cfg, q, k, v, kc, vc, cos_t, sin_t, seq, pos, out, ws, n, heads, kv_heads,
                                         hd, capacity, n_slots, max_pos, n_chunks)
                : launch_attention<false>(cfg, q, nullptr, nullptr, kc, vc, nullptr, nullptr, seq, pos, out, ws, n,
                                          heads, kv_heads, hd, capacity, n_slots, max_pos, n_chunks);
  }
  if (e != cudaSuccess) {
    snprintf(msg, ml, "attention launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

}  // namespace draco
