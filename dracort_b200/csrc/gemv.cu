// gemv.cu — decode GEMV y[B, N] = x[B, K] . dequant(W)^T over TILED GGUF
// weights (Q8_0 / Q4_K / Q6_K), 1 <= B <= 32, several weights per launch.
//
// Replaces the reference's decode linear: executor._linear
// (draco/runtime/cpu/executor.py:47-79) -> GenericGemmKernel.matmul_f32
// (draco/runtime/cpu/kernels/generic.py:32-33) on the fp32 cache produced by
// gguf._dequantize (draco/format/gguf.py:272-497).
//
// Design (B200, HBM-bound):
//  * Persistent grid, one CTA per SM.  The weights of all problems are cut
//    into "slabs" (128 rows x 256 k, contiguous in the TILED layout) and every
//    CTA owns a contiguous, byte-balanced range of slabs (stream-K).  A warp
//    that is the only owner of a row group writes y directly; row groups split
//    between CTAs are combined deterministically by the last CTA to finish
//    (arrival counter in the workspace, partial sums added in CTA order).
//  * Warp 8 is the producer: it streams each slab, plus the matching slice of
//    the prepared activations, into a ring of shared-memory stages with 1-D
//    bulk copies (TMA engine) completing on mbarriers.  Warps 0-7 consume; warp
//    w owns row tile w (16 rows) of every slab.
//  * The quants enter the m16n8k16 tensor-core MMA as exact integers in fp16
//    (bit tricks: 0x6400 | nibble == 1024 + q).  Activations enter as an fp16
//    hi/lo pair (x = hi + lo to ~2^-22 after a per-row power-of-two rescale),
//    one MMA column each, so the product is accurate to fp32 level.  The
//    per-sub-block scales (and the 1024 offset, and Q4_K's mins) are applied in
//    fp32 to each sub-block's MMA result: y += alpha*c - beta*sum(x).
//  * A separate small kernel (gemv_prep) converts x into that fragment order
//    and computes the per-16-element sums once per call.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace draco {

constexpr int kMaxCta = 192;
constexpr int kMaxStages = 8;
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait

struct GemvProbDev {
  const uint8_t* w;
  const float* x;
  float* y;
  const float* bias;
  int64_t ldx, ldy;
  int64_t slab0;   // global index of the problem's first slab
  int64_t xs_off;  // workspace byte offsets
  int64_t s_off;
  int64_t sc_off;
  int qt, n_rows, k, nb, n_rg, n_tiles, cb, pad_;
};

struct GemvParams {
  GemvProbDev prob[DRACO_GEMV_MAX_PROBLEMS];
  uint8_t* ws;
  int64_t status_off, cnt_off, part_off;
  int64_t total_slabs;
  int n_prob, batch, nt, n_cta;
  int w_stage, xs_bytes, s_bytes, stage_bytes, n_stages, pad_;
  int cta_start[kMaxCta + 1];
};

// workspace layout (bytes)
constexpr int64_t kWsStatus = 0;
constexpr int64_t kWsCounters = 256;
constexpr int64_t kWsCountersBytes = (int64_t)kMaxCta * 2 * 4;
static inline int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }

// ---------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ float2 lds64f(const uint8_t* p) { return *reinterpret_cast<const float2*>(p); }

// exact float of byte i of w (unsigned), via the 2^23 magic number
__device__ __forceinline__ float ubyte_f(uint32_t w, int i) {
  uint32_t m = __byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)i);
  return __uint_as_float(m) - 8388608.f;
}
// exact float of byte i of w read as int8
__device__ __forceinline__ float sbyte_f(uint32_t w, int i) {
  uint32_t m = __byte_perm(w ^ 0x80808080u, 0x4B000000u, 0x7440u | (uint32_t)i);
  return __uint_as_float(m) - 8388736.f;  // 2^23 + 128
}
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) { return (w & 0x000F000Fu) | 0x64006400u; }
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) { return (w & 0x00F000F0u) | 0x64006400u; }
// bytes 0,2 / 1,3 of w into the low bytes of two fp16 lanes with 0x64 exponent
__device__ __forceinline__ uint32_t byte02(uint32_t w) { return __byte_perm(w, 0x64646464u, 0x4240u); }
__device__ __forceinline__ uint32_t byte13(uint32_t w) { return __byte_perm(w, 0x64646464u, 0x4341u); }

__device__ __forceinline__ void named_bar_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

__device__ __forceinline__ void locate_slab(const GemvParams& P, int64_t s, int& p, int64_t& rg, int64_t& j) {
  p = 0;
#pragma unroll 1
  for (int q = 1; q < P.n_prob; ++q)
    if (s >= P.prob[q].slab0) p = q;
  const int64_t local = s - P.prob[p].slab0;
  const int64_t nb = P.prob[p].nb;
  rg = local / nb;
  j = local - rg * nb;
}

__device__ __forceinline__ int slab_tiles(const GemvProbDev& pr, int64_t rg) {
  int64_t r = pr.n_tiles - rg * kGroupTiles;
  return (int)(r < kGroupTiles ? r : kGroupTiles);
}

__device__ __forceinline__ void record_error(const GemvParams& P, int code) {
  atomicCAS(reinterpret_cast<int*>(P.ws + P.status_off), 0, code);
}

// ---------------------------------------------------------------------------
// activation preparation: x fp32 -> fp16 (hi, lo) fragment order + sums
// grid (4*NT batch slots, n_prob), 256 threads
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gemv_prep_kernel(const __grid_constant__ GemvParams P) {
  // let the GEMV launch now: its CTAs start streaming weights (which do not
  // depend on this kernel) and wait on griddepcontrol.wait for our outputs
  grid_launch_dependents();
  grid_dependency_wait();
  const int b = blockIdx.x, p = blockIdx.y;
  const GemvProbDev& pr = P.prob[p];
  const int ncols = 8 * P.nt;
  const int bslots = 4 * P.nt;
  const int64_t nk = pr.nb * 16;  // 16-element steps (k padded to 256)
  uint8_t* xs = P.ws + pr.xs_off;
  float* S = reinterpret_cast<float*>(P.ws + pr.s_off);
  float* unscale = reinterpret_cast<float*>(P.ws + pr.sc_off);
  __shared__ float red[8];
  __shared__ float s_scale;

  if (b >= P.batch) {
    for (int64_t kk = threadIdx.x; kk < nk; kk += blockDim.x) {
      uint4 z = make_uint4(0, 0, 0, 0);
      uint4* d0 = reinterpret_cast<uint4*>(xs + ((kk * ncols + 2 * b) * 4) * 8);
      d0[0] = z; d0[1] = z; d0[2] = z; d0[3] = z;  // cols 2b, 2b+1: 64 contiguous bytes
      S[((kk >> 1) * bslots + b) * 2 + (kk & 1)] = 0.f;
    }
    if (threadIdx.x == 0) unscale[b] = 0.f;
    return;
  }

  const float* x = pr.x + (int64_t)b * pr.ldx;
  float amax = 0.f;
  for (int64_t i = threadIdx.x; i < pr.k; i += blockDim.x) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    int e = 0;
    if (m > 0.f && m <= 3.0e38f) e = ilogbf(m) - 13;
    e = max(-110, min(110, e));
    s_scale = ldexpf(1.f, -e);
    unscale[b] = ldexpf(1.f, e);
  }
  __syncthreads();
  const float sc = s_scale;
  for (int64_t kk = threadIdx.x; kk < nk; kk += blockDim.x) {
    __half hi[16], lo[16];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int64_t kx = kk * 16 + i;
      const float v = (kx < pr.k) ? x[kx] * sc : 0.f;
      hi[i] = __float2half_rn(v);
      const float hf = __half2float(hi[i]);
      lo[i] = __float2half_rn(v - hf);
      sum += hf + __half2float(lo[i]);
    }
    uint32_t* dh = reinterpret_cast<uint32_t*>(xs + ((kk * ncols + 2 * b) * 4) * 8);
    uint32_t* dl = reinterpret_cast<uint32_t*>(xs + ((kk * ncols + 2 * b + 1) * 4) * 8);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      __half2 h02 = __halves2half2(hi[4 * t], hi[4 * t + 2]);
      __half2 h13 = __halves2half2(hi[4 * t + 1], hi[4 * t + 3]);
      __half2 l02 = __halves2half2(lo[4 * t], lo[4 * t + 2]);
      __half2 l13 = __halves2half2(lo[4 * t + 1], lo[4 * t + 3]);
      dh[2 * t] = *reinterpret_cast<uint32_t*>(&h02);
      dh[2 * t + 1] = *reinterpret_cast<uint32_t*>(&h13);
      dl[2 * t] = *reinterpret_cast<uint32_t*>(&l02);
      dl[2 * t + 1] = *reinterpret_cast<uint32_t*>(&l13);
    }
    S[((kk >> 1) * bslots + b) * 2 + (kk & 1)] = sum;
  }
}

// ---------------------------------------------------------------------------
// per-chunk consumers.  ch: 16-row chunk in smem; xs: activation slice of the
// slab's super-block [16 steps][8*NT cols][4 t][8 B]; S: sums [8 pairs][4*NT][2];
// scr: per-warp 16 x 16 float scratch for decoded scales.
// acc[nt][0] -> (row g, batch 4nt+t), acc[nt][1] -> (row g+8, batch 4nt+t)
// ---------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ void chunk_q4k(const uint8_t* ch, const uint8_t* xs, const uint8_t* S, float* scr,
                                          int lane, float (&acc)[NT][2]) {
  const int g = lane >> 2, t = lane & 3;
  {  // cooperative decode: lane -> row r, sub-blocks 4h..4h+3 -> (alpha, beta)
    const int r = lane >> 1, h = lane & 1;
    const uint8_t* sp = ch + 2048 + 24 * (r & 7) + 12 * (r >> 3);
    const uint32_t A = lds32(sp), Bw = lds32(sp + 4), C = lds32(sp + 8);
    const uint32_t dd = lds32(ch + 2240 + 8 * (r & 7) + 4 * (r >> 3));
    const float d = f16_bits_to_f32(dd), dmin = f16_bits_to_f32(dd >> 16);
    uint32_t scw, mw;
    if (h == 0) {
      scw = A & 0x3F3F3F3Fu;
      mw = Bw & 0x3F3F3F3Fu;
    } else {
      scw = (C & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u);
      mw = ((C >> 4) & 0x0F0F0F0Fu) | ((Bw >> 2) & 0x30303030u);
    }
    float* dst = scr + r * 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int jj = 4 * h + i;
      const float a = d * ubyte_f(scw, i);
      const float mu = dmin * ubyte_f(mw, i);
      // even sub-blocks: low nibbles (1024 + q); odd: high nibbles (1024 + 16 q)
      const float al = (jj & 1) ? a * 0.0625f : a;
      const float be = fmaf((jj & 1) ? 64.f : 1024.f, a, mu);
      dst[jj] = al;
      dst[8 + jj] = be;
    }
  }
  __syncwarp();
  float al0[8], be0[8], al1[8], be1[8];
  {
    const float4* r0 = reinterpret_cast<const float4*>(scr + g * 16);
    const float4* r1 = reinterpret_cast<const float4*>(scr + (g + 8) * 16);
    float4 v;
    v = r0[0]; al0[0] = v.x; al0[1] = v.y; al0[2] = v.z; al0[3] = v.w;
    v = r0[1]; al0[4] = v.x; al0[5] = v.y; al0[6] = v.z; al0[7] = v.w;
    v = r0[2]; be0[0] = v.x; be0[1] = v.y; be0[2] = v.z; be0[3] = v.w;
    v = r0[3]; be0[4] = v.x; be0[5] = v.y; be0[6] = v.z; be0[7] = v.w;
    v = r1[0]; al1[0] = v.x; al1[1] = v.y; al1[2] = v.z; al1[3] = v.w;
    v = r1[1]; al1[4] = v.x; al1[5] = v.y; al1[6] = v.z; al1[7] = v.w;
    v = r1[2]; be1[0] = v.x; be1[1] = v.y; be1[2] = v.z; be1[3] = v.w;
    v = r1[3]; be1[4] = v.x; be1[5] = v.y; be1[6] = v.z; be1[7] = v.w;
  }
  __syncwarp();
  const int xs_step = NT * 256;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 v = lds128(ch + 512 * q + 16 * lane);
    const uint32_t x8 = v.x >> 8, y8 = v.y >> 8, z8 = v.z >> 8, w8 = v.w >> 8;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const uint8_t* xb = xs + nt * 256 + lane * 8;
      const uint2 b0 = lds64(xb + (4 * q + 0) * xs_step);
      const uint2 b1 = lds64(xb + (4 * q + 1) * xs_step);
      const uint2 b2 = lds64(xb + (4 * q + 2) * xs_step);
      const uint2 b3 = lds64(xb + (4 * q + 3) * xs_step);
      float c[4], e[4];
      mma_f16_16816(c, nib_lo(v.x), nib_lo(v.z), nib_lo(x8), nib_lo(z8), b0.x, b0.y);
      mma_f16_16816_acc(c, nib_lo(v.y), nib_lo(v.w), nib_lo(y8), nib_lo(w8), b1.x, b1.y);
      mma_f16_16816(e, nib_hi(v.x), nib_hi(v.z), nib_hi(x8), nib_hi(z8), b2.x, b2.y);
      mma_f16_16816_acc(e, nib_hi(v.y), nib_hi(v.w), nib_hi(y8), nib_hi(w8), b3.x, b3.y);
      const float2 s_lo = lds64f(S + ((2 * q) * 4 * NT + 4 * nt + t) * 8);
      const float2 s_hi = lds64f(S + ((2 * q + 1) * 4 * NT + 4 * nt + t) * 8);
      const float sl = s_lo.x + s_lo.y, sh = s_hi.x + s_hi.y;
      float a0 = acc[nt][0], a1 = acc[nt][1];
      a0 = fmaf(al0[2 * q], c[0] + c[1], a0);
      a0 = fmaf(-be0[2 * q], sl, a0);
      a1 = fmaf(al1[2 * q], c[2] + c[3], a1);
      a1 = fmaf(-be1[2 * q], sl, a1);
      a0 = fmaf(al0[2 * q + 1], e[0] + e[1], a0);
      a0 = fmaf(-be0[2 * q + 1], sh, a0);
      a1 = fmaf(al1[2 * q + 1], e[2] + e[3], a1);
      a1 = fmaf(-be1[2 * q + 1], sh, a1);
      acc[nt][0] = a0;
      acc[nt][1] = a1;
    }
  }
}

template <int NT>
__device__ __forceinline__ void chunk_q6k(const uint8_t* ch, const uint8_t* xs, const uint8_t* S, float* scr,
                                          int lane, float (&acc)[NT][2]) {
  const int g = lane >> 2, t = lane & 3;
  {  // cooperative decode: lane -> row r, sub-blocks 8h..8h+7 -> alpha = d * sc
    const int r = lane >> 1, h = lane & 1;
    const uint2 sc8 = lds64(ch + 3072 + 32 * (r & 7) + 16 * (r >> 3) + 8 * h);
    const uint32_t dw = *reinterpret_cast<const uint16_t*>(ch + 3328 + 4 * (r & 7) + 2 * (r >> 3));
    const float d = f16_bits_to_f32(dw);
    float* dst = scr + r * 16 + 8 * h;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      dst[i] = d * sbyte_f(sc8.x, i);
      dst[4 + i] = d * sbyte_f(sc8.y, i);
    }
  }
  __syncwarp();
  float al0[16], al1[16];
  {
    const float4* r0 = reinterpret_cast<const float4*>(scr + g * 16);
    const float4* r1 = reinterpret_cast<const float4*>(scr + (g + 8) * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float4 v = r0[i];
      al0[4 * i] = v.x; al0[4 * i + 1] = v.y; al0[4 * i + 2] = v.z; al0[4 * i + 3] = v.w;
      v = r1[i];
      al1[4 * i] = v.x; al1[4 * i + 1] = v.y; al1[4 * i + 2] = v.z; al1[4 * i + 3] = v.w;
    }
  }
  __syncwarp();
  uint32_t W[24];
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const uint4 v = lds128(ch + 512 * i + 16 * lane);
    W[4 * i] = v.x; W[4 * i + 1] = v.y; W[4 * i + 2] = v.z; W[4 * i + 3] = v.w;
  }
  const int xs_step = NT * 256;
#pragma unroll
  for (int nu = 0; nu < 4; ++nu) {
    const int n = nu >> 1, is = nu & 1;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int s = 8 * n + 2 * i + is;  // sub-block == 16-element step index
      uint32_t qg, qg8;
      {
        const uint32_t l0 = W[6 * nu + (i & 1)], h0 = W[6 * nu + 2];
        const uint32_t l1 = W[6 * nu + 3 + (i & 1)], h1 = W[6 * nu + 5];
        const uint32_t n0 = (i < 2 ? l0 : (l0 >> 4)) & 0x0F0F0F0Fu;
        const uint32_t n1 = (i < 2 ? l1 : (l1 >> 4)) & 0x0F0F0F0Fu;
        qg = n0 | (((h0 >> (2 * i)) << 4) & 0x30303030u);
        qg8 = n1 | (((h1 >> (2 * i)) << 4) & 0x30303030u);
      }
      const uint32_t a0 = byte02(qg), a2 = byte13(qg), a1 = byte02(qg8), a3 = byte13(qg8);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 b = lds64(xs + nt * 256 + lane * 8 + s * xs_step);
        float c[4];
        mma_f16_16816(c, a0, a1, a2, a3, b.x, b.y);
        const float2 sp = lds64f(S + ((s >> 1) * 4 * NT + 4 * nt + t) * 8);
        const float ss = (s & 1) ? sp.y : sp.x;
        acc[nt][0] = fmaf(al0[s], fmaf(-1056.f, ss, c[0] + c[1]), acc[nt][0]);
        acc[nt][1] = fmaf(al1[s], fmaf(-1056.f, ss, c[2] + c[3]), acc[nt][1]);
      }
    }
  }
}

template <int NT>
__device__ __forceinline__ void chunk_q80(const uint8_t* ch, const uint8_t* xs, const uint8_t* S, int lane,
                                          float (&acc)[NT][2]) {
  const int g = lane >> 2, t = lane & 3;
  float d0[8], d1[8];
  {
    const uint4 u0 = lds128(ch + 4096 + 32 * g);
    const uint4 u1 = lds128(ch + 4096 + 32 * g + 16);
    const uint32_t w0[4] = {u0.x, u0.y, u0.z, u0.w};
    const uint32_t w1[4] = {u1.x, u1.y, u1.z, u1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      d0[2 * i] = f16_bits_to_f32(w0[i]);
      d0[2 * i + 1] = f16_bits_to_f32(w0[i] >> 16);
      d1[2 * i] = f16_bits_to_f32(w1[i]);
      d1[2 * i + 1] = f16_bits_to_f32(w1[i] >> 16);
    }
  }
  const int xs_step = NT * 256;
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint4 v = lds128(ch + 512 * b + 16 * lane);
    const uint32_t ux = v.x ^ 0x80808080u, uy = v.y ^ 0x80808080u;
    const uint32_t uz = v.z ^ 0x80808080u, uw = v.w ^ 0x80808080u;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const uint8_t* xb = xs + nt * 256 + lane * 8;
      const uint2 b0 = lds64(xb + (2 * b) * xs_step);
      const uint2 b1 = lds64(xb + (2 * b + 1) * xs_step);
      float c[4];
      mma_f16_16816(c, byte02(ux), byte02(uz), byte13(ux), byte13(uz), b0.x, b0.y);
      mma_f16_16816_acc(c, byte02(uy), byte02(uw), byte13(uy), byte13(uw), b1.x, b1.y);
      const float2 sp = lds64f(S + (b * 4 * NT + 4 * nt + t) * 8);
      const float s32 = sp.x + sp.y;
      acc[nt][0] = fmaf(d0[b], fmaf(-1152.f, s32, c[0] + c[1]), acc[nt][0]);
      acc[nt][1] = fmaf(d1[b], fmaf(-1152.f, s32, c[2] + c[3]), acc[nt][1]);
    }
  }
}

// ---------------------------------------------------------------------------
// output of one row group
// ---------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ void write_rows(const GemvParams& P, const GemvProbDev& pr, int64_t rg, int warp,
                                           int lane, const float (&v)[NT][2]) {
  const int g = lane >> 2, t = lane & 3;
  const float* unscale = reinterpret_cast<const float*>(P.ws + pr.sc_off);
  const int64_t row0 = (rg * kGroupTiles + warp) * kChunkRows + g;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int b = 4 * nt + t;
    if (b >= P.batch) continue;
    const float us = unscale[b];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t row = row0 + 8 * h;
      if (row < pr.n_rows) {
        float out = v[nt][h] * us;
        if (pr.bias) out += pr.bias[row];
        pr.y[(int64_t)b * pr.ldy + row] = out;
      }
    }
  }
}

__device__ __forceinline__ int cta_of_slab(const GemvParams& P, int64_t s) {
  int lo = 0, hi = P.n_cta - 1;  // largest c with cta_start[c] <= s
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (P.cta_start[mid] <= s) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int NT>
__device__ void finish_rowgroup(const GemvParams& P, int p, int64_t rg, int64_t s_begin, int64_t s_end, int warp,
                                int lane, float (&acc)[NT][2], int* s_flag) {
  const GemvProbDev& pr = P.prob[p];
  const int nrt = slab_tiles(pr, rg);
  const int64_t rg_start = pr.slab0 + rg * pr.nb, rg_end = rg_start + pr.nb;
  if (s_begin <= rg_start && rg_end <= s_end) {
    if (warp < nrt) write_rows<NT>(P, pr, rg, warp, lane, acc);
    return;
  }
  // split row group: publish the partial, the last contributor reduces
  const int cta = blockIdx.x;
  const int slot = (s_begin >= rg_start) ? 0 : 1;
  float* part = reinterpret_cast<float*>(P.ws + P.part_off) +
                ((((int64_t)cta * 2 + slot) * kConsumerWarps + warp) * 32 + lane) * (NT * 2);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    __stcg(part + 2 * nt, acc[nt][0]);
    __stcg(part + 2 * nt + 1, acc[nt][1]);
  }
  __threadfence();
  named_bar_consumers();
  if (threadIdx.x == 0) {
    const int c_first = cta_of_slab(P, rg_start);
    const int c_last = cta_of_slab(P, rg_end - 1);
    const int slot_first = (P.cta_start[c_first] >= rg_start) ? 0 : 1;
    unsigned int* cnt = reinterpret_cast<unsigned int*>(P.ws + P.cnt_off) + (c_first * 2 + slot_first);
    const unsigned int old = atomicAdd(cnt, 1u);
    const bool last = (old == (unsigned int)(c_last - c_first));
    if (last) {
      atomicExch(cnt, 0u);
      __threadfence();
    }
    *s_flag = last ? (1 + c_first + (c_last << 12)) : 0;
  }
  named_bar_consumers();
  const int f = *s_flag;
  if (f && warp < nrt) {
    const int c_first = (f - 1) & 0xFFF, c_last = (f - 1) >> 12;
    float sum[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sum[nt][0] = sum[nt][1] = 0.f;
    for (int c = c_first; c <= c_last; ++c) {
      const int sl = (P.cta_start[c] >= rg_start) ? 0 : 1;
      const float* q = reinterpret_cast<const float*>(P.ws + P.part_off) +
                       ((((int64_t)c * 2 + sl) * kConsumerWarps + warp) * 32 + lane) * (NT * 2);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        sum[nt][0] += __ldcg(q + 2 * nt);
        sum[nt][1] += __ldcg(q + 2 * nt + 1);
      }
    }
    write_rows<NT>(P, pr, rg, warp, lane, sum);
  }
}

// ---------------------------------------------------------------------------
// the persistent GEMV kernel
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ __align__(16) float scratch[kConsumerWarps][16 * 16];
  __shared__ int s_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int64_t s_begin = P.cta_start[cta], s_end = P.cta_start[cta + 1];
  const int NS = P.n_stages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      // Weights do not depend on the preceding kernel; the activation slices do.
      bool dep_done = false;
      int64_t i = 0;
      for (int64_t s = s_begin; s < s_end; ++s, ++i) {
        const int st = (int)(i % NS);
        const uint32_t ph = (uint32_t)((i / NS) & 1);
        if (i >= NS && !mbar_wait_bounded(&empty_bar[st], ph ^ 1u, kWaitLimitNs)) {
          record_error(P, DRACO_ERR_TIMEOUT);
          break;
        }
        int p;
        int64_t rg, j;
        locate_slab(P, s, p, rg, j);
        const GemvProbDev& pr = P.prob[p];
        const TiledGeom geo = tiled_geom(pr.qt, pr.n_rows, pr.k);
        const uint32_t wbytes = (uint32_t)(slab_tiles(pr, rg) * pr.cb);
        uint8_t* stage = smem + (size_t)st * P.stage_bytes;
        mbar_arrive_expect_tx(&full_bar[st], wbytes + P.xs_bytes + P.s_bytes);
        bulk_g2s(stage, pr.w + slab_offset(geo, rg, j), wbytes, &full_bar[st]);
        if (!dep_done) {
          grid_dependency_wait();
          dep_done = true;
        }
        bulk_g2s(stage + P.w_stage, P.ws + pr.xs_off + j * (int64_t)P.xs_bytes, P.xs_bytes, &full_bar[st]);
        bulk_g2s(stage + P.w_stage + P.xs_bytes, P.ws + pr.s_off + j * (int64_t)P.s_bytes, P.s_bytes,
                 &full_bar[st]);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  grid_dependency_wait();  // outputs (y) may be read by the preceding kernel
  float acc[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
  float* scr = scratch[warp];
  // After a timed-out wait the warp stops waiting and computing but keeps
  // walking its range, so every consumer warp still reaches each named
  // barrier and the kernel ends.  The status word tells the host.
  bool failed = false;
  int64_t i = 0;
  for (int64_t s = s_begin; s < s_end; ++s, ++i) {
    const int st = (int)(i % NS);
    const uint32_t ph = (uint32_t)((i / NS) & 1);
    if (!failed && !mbar_wait_bounded(&full_bar[st], ph, kWaitLimitNs)) {
      record_error(P, DRACO_ERR_TIMEOUT);
      failed = true;
    }
    int p;
    int64_t rg, j;
    locate_slab(P, s, p, rg, j);
    const GemvProbDev& pr = P.prob[p];
    const int nrt = slab_tiles(pr, rg);
    const uint8_t* stage = smem + (size_t)st * P.stage_bytes;
    if (!failed && warp < nrt) {
      const uint8_t* ch = stage + warp * pr.cb;
      const uint8_t* xs = stage + P.w_stage;
      const uint8_t* S = xs + P.xs_bytes;
      if (pr.qt == kQ4_K) chunk_q4k<NT>(ch, xs, S, scr, lane, acc);
      else if (pr.qt == kQ6_K) chunk_q6k<NT>(ch, xs, S, scr, lane, acc);
      else chunk_q80<NT>(ch, xs, S, lane, acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
    if (j == pr.nb - 1 || s == s_end - 1) {
      finish_rowgroup<NT>(P, p, rg, s_begin, s_end, warp, lane, acc, &s_flag);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
    }
  }
}

// ---------------------------------------------------------------------------
// host side: plan + launch
// ---------------------------------------------------------------------------
struct HostPlan {
  GemvParams P;
  size_t ws_needed;
  size_t smem_bytes;
};

static int nt_of_batch(int batch) { return batch <= 4 ? 1 : batch <= 8 ? 2 : batch <= 16 ? 4 : 8; }

static bool build_plan(const draco_gemv_problem* probs, int n, int batch, int n_sm, HostPlan& hp, char* msg,
                       size_t ml) {
  GemvParams& P = hp.P;
  memset(&P, 0, sizeof(P));
  P.n_prob = n;
  P.batch = batch;
  P.nt = nt_of_batch(batch);
  const int NT = P.nt;
  P.xs_bytes = 16 * 8 * NT * 32;  // 16 steps x 8*NT cols x 4 t x 8 B
  P.s_bytes = 8 * 4 * NT * 8;     // 8 pairs x 4*NT slots x 2 floats
  int64_t off = kWsCounters + kWsCountersBytes;
  off = align256(off);
  int64_t slab0 = 0;
  int w_stage = 0;
  for (int p = 0; p < n; ++p) {
    const draco_gemv_problem& q = probs[p];
    GemvProbDev& d = P.prob[p];
    TiledGeom g = tiled_geom(q.qtype, q.n_rows, q.k);
    d.w = static_cast<const uint8_t*>(q.w);
    d.x = q.x;
    d.y = q.y;
    d.bias = q.bias;
    d.ldx = q.ldx;
    d.ldy = q.ldy;
    d.qt = q.qtype;
    d.n_rows = (int)q.n_rows;
    d.k = (int)q.k;
    d.nb = (int)g.nb;
    d.n_rg = (int)g.n_rg;
    d.n_tiles = (int)g.n_tiles;
    d.cb = g.cb;
    d.slab0 = slab0;
    slab0 += g.n_rg * g.nb;
    w_stage = std::max(w_stage, kGroupTiles * g.cb);
    const int64_t nk = g.nb * 16;
    d.xs_off = off;
    off = align256(off + nk * 8 * NT * 32);
    d.s_off = off;
    off = align256(off + (nk / 2) * 4 * NT * 8);
    d.sc_off = off;
    off = align256(off + 4 * NT * 4);
  }
  P.part_off = off;
  off = align256(off + (int64_t)kMaxCta * 2 * kConsumerWarps * 32 * NT * 2 * 4);
  P.status_off = kWsStatus;
  P.cnt_off = kWsCounters;
  P.total_slabs = slab0;
  P.w_stage = w_stage;
  P.stage_bytes = w_stage + P.xs_bytes + P.s_bytes;
  const int smem_budget = 200 * 1024;
  P.n_stages = std::min(kMaxStages, smem_budget / P.stage_bytes);
  if (P.n_stages < 2) {
    snprintf(msg, ml, "gemv: stage of %d bytes does not fit shared memory twice", P.stage_bytes);
    return false;
  }
  hp.smem_bytes = (size_t)P.n_stages * P.stage_bytes;
  hp.ws_needed = (size_t)off;

  // byte-balanced slab ranges per CTA
  const int64_t total = P.total_slabs;
  const int n_cta = (int)std::min<int64_t>(std::min(n_sm, kMaxCta), total);
  P.n_cta = n_cta;
  if (n_cta == 0) return true;
  int64_t total_bytes = 0;
  for (int p = 0; p < n; ++p) {
    const GemvProbDev& d = P.prob[p];
    total_bytes += (int64_t)d.n_tiles * d.nb * d.cb;
  }
  P.cta_start[0] = 0;
  int c = 1;
  int64_t cum = 0;  // bytes before the current row group
  for (int p = 0; p < n && c < n_cta; ++p) {
    const GemvProbDev& d = P.prob[p];
    for (int64_t rg = 0; rg < d.n_rg && c < n_cta; ++rg) {
      const int64_t nrt = std::min<int64_t>(kGroupTiles, d.n_tiles - rg * kGroupTiles);
      const int64_t sb_bytes = nrt * d.cb;
      const int64_t rg_total = sb_bytes * d.nb;
      while (c < n_cta) {
        const int64_t target = (total_bytes * c) / n_cta;
        if (target >= cum + rg_total) break;
        int64_t within = (target - cum + sb_bytes - 1) / sb_bytes;
        if (within < 0) within = 0;
        int64_t s = d.slab0 + rg * d.nb + within;
        if (s <= P.cta_start[c - 1]) s = P.cta_start[c - 1] + 1;
        if (s > total - (n_cta - c)) s = total - (n_cta - c);
        P.cta_start[c++] = (int)s;
      }
      cum += rg_total;
    }
  }
  while (c < n_cta) {  // numerical leftovers
    int64_t s = std::max<int64_t>(P.cta_start[c - 1] + 1, total - (n_cta - c));
    P.cta_start[c++] = (int)s;
  }
  P.cta_start[n_cta] = (int)total;
  return true;
}

size_t gemv_workspace_bytes(const draco_gemv_problem* probs, int n, int batch) {
  HostPlan local;
  char msg[128];
  if (!build_plan(probs, n, batch, kMaxCta, local, msg, sizeof(msg))) return 0;
  return local.ws_needed;
}

template <int NT>
static cudaError_t launch_nt(const HostPlan& hp, cudaStream_t st) {
  static int attr_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && attr_set[dev] < (int)hp.smem_bytes) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[dev] = 200 * 1024;
  }
  const GemvParams& P = hp.P;
  // prep kernel (plain launch; waits for nothing but stream order)
  {
    dim3 grid(4 * P.nt, P.n_prob);
    gemv_prep_kernel<<<grid, 256, 0, st>>>(P);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  // main kernel with programmatic dependent launch so that its weight
  // prefetch overlaps the prep kernel
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P.n_cta);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = hp.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<NT>, P);
}

int gemv_launch(const draco_gemv_problem* probs, int n, int batch, void* ws, size_t ws_bytes, cudaStream_t st,
                char* msg, size_t ml) {
  HostPlan hp;
  const int n_sm = device_sm_count();
  if (!build_plan(probs, n, batch, n_sm, hp, msg, ml)) return DRACO_ERR_ARG;
  if (hp.P.total_slabs == 0) return DRACO_OK;
  // the plan's workspace size does not depend on the SM count
  if (ws == nullptr || ws_bytes < hp.ws_needed) {
    snprintf(msg, ml, "gemv: workspace of %zu bytes given, %zu needed", ws_bytes, hp.ws_needed);
    return DRACO_ERR_WORKSPACE;
  }
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) {
    snprintf(msg, ml, "gemv: workspace must be 256-byte aligned");
    return DRACO_ERR_ALIGN;
  }
  hp.P.ws = static_cast<uint8_t*>(ws);
  cudaError_t e;
  switch (hp.P.nt) {
    case 1: e = launch_nt<1>(hp, st); break;
    case 2: e = launch_nt<2>(hp, st); break;
    case 4: e = launch_nt<4>(hp, st); break;
    default: e = launch_nt<8>(hp, st); break;
  }
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemv: launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

}  // namespace draco
