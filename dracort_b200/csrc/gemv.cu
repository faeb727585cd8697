// gemv.cu — decode GEMV y[B, N] = x[B, K] . dequant(W)^T over TILED GGUF
// weights (Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 / Q4_K / Q5_K / Q6_K), 1 <= B <= 32,
// several weights per launch.
//
// Replaces the reference's decode linear: executor._linear
// (draco/runtime/cpu/executor.py:47-79) -> GenericGemmKernel.matmul_f32
// (draco/runtime/cpu/kernels/generic.py:32-33) on the fp32 cache produced by
// gguf._dequantize (draco/format/gguf.py:272-497).
//
// Design (B200, HBM-bound), one persistent launch per call:
//  * One CTA per SM.  The weights of all problems are cut into "slabs"
//    (128 rows x 256 k, contiguous in the TILED layout) and every CTA owns a
//    contiguous, byte-balanced range of slabs (stream-K).  Row groups
//    (128 rows x all k) owned by one CTA are written directly; row groups
//    split between CTAs are combined deterministically by the last CTA to
//    finish (arrival counter in the workspace, partials added in CTA order).
//  * Warp 16 (producer) streams each slab into a ring of shared-memory stages
//    with 1-D bulk copies (TMA engine) completing on the slab's ready
//    barrier; it starts at launch, before the preceding kernel has finished
//    (programmatic dependent launch), since weights do not depend on it.
//  * Warps 17-19 (converters) fill each stage's activation slice (slab i by
//    converter i % 3): they read the slab's 256 x B activations from global
//    memory (L2), scale each 32-element group by a power of two u
//    (max |x| / u in [2^13, 2^14)), round to an integer q and split it into
//    two int8 digits, q = 256 * hi + lo, stored in MMA-fragment order with
//    the group sums, and arrive on the slab's ready barrier, which completes
//    with that arrival and the slab's weight bytes.  From batch 3 on (the
//    dense layouts) the activations are converted once per launch
//    instead, by gemv_convert_kernel, into per-(problem, super-block) slices
//    of the workspace laid out as a stage's slice; the converter warps then
//    fill a stage with one bulk copy of that slice (arrive.expect_tx on the
//    same ready barrier).  Converting per slab in every CTA repeated the work
//    for every row group, which dominated at batch 32.
//  * A barrier wait tests a phase parity, which is only sound when the waiter
//    sees every phase of the barrier in order.  Stage st holds slabs st,
//    st + NS, ... (round m = i / NS); the ready barriers are kept per (stage,
//    slab parity), so each consumer warp sees every phase of its parity's
//    barriers (phase m for an even NS, m / 2 for an odd one, where a stage's
//    slabs alternate parities), and the producer waits for every phase of
//    every empty barrier.  The converters see only some slabs of a stage, so
//    they do not wait on the empty barriers: the producer, once a stage is
//    free for round m, publishes m in the stage's generation word (release /
//    acquire), which a full counter cannot confuse.
//  * Every wait is bounded.  The agent whose wait runs out records
//    DRACO_ERR_TIMEOUT and sets the CTA's abort word; the other agents' waits
//    see it and return, nobody frees a stage after that, and the producer
//    waits (bounded) for its last copies to land before it exits, so the CTA
//    never ends with a bulk copy in flight (after an abort the converters
//    still arrive, without converting, for every slab the producer issued,
//    so that those ready phases complete with the bytes).  An aborted launch
//    leaves the workspace's arrival counters stale: zero the workspace
//    before reusing it.
//  * Warps 0-15 consume: warp w owns row tile (w % 8) of the slabs whose
//    parity is w / 8.  The quants enter the int8 tensor-core MMA
//    (m16n8k32, u8 x s8 -> s32) as they are: Q4_K / Q4_0 / Q4_1 nibbles with
//    one mask, Q5_x nibbles with their fifth bit or-ed in, Q6_K as
//    ql | qh << 4, Q8_0 bytes unchanged; each activation digit is one MMA
//    column.  Integer accumulation is exact; the (sub-)block scale and the
//    min / offset (Q4_K's and Q5_K's min, Q6_K's -32, Q4_0's -8, Q5_0's -16,
//    Q4_1's and Q5_1's m) are applied in fp32 per (sub-)block:
//        y += d_sc * u * (256 * C_hi + C_lo) - d_min_m * S
//    The activation rounding (one step of u) bounds the result error at
//    about 5e-5 relative L2 for Gaussian activations.
//  * Batch 1-2 ("diagonal" activation layout): each sub-block's activations
//    sit in their own pair of MMA columns, so one accumulator collects
//    4 (B=1) or 2 (B=2) sub-blocks and every lane owns one sub-block's sum.
//    Batch >= 3 ("dense"): columns are (batch, digit).
//  * Tensor-parallel form (draco_gguf_gemv_grouped_tp): each output value is
//    stored into every rank's exchange buffer over NVLink (peer stores through
//    CUDA IPC mappings) instead of the local y; when every CTA is done, the
//    last one fences at system scope and stores the step's epoch into each
//    rank's flag for this rank.  The buffers are double-buffered by the parity
//    of the epoch, which each rank counts in its own buffer.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "gemv_plan.h"
#include "internal.h"

namespace draco {

constexpr int kMaxStages = 8;
constexpr int kConsumerWarps = 2 * kRowWarps;  // even / odd slabs
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kConvWarps = 3;
constexpr int kThreads = (kConsumerWarps + 1 + kConvWarps) * 32;
constexpr int kMaxMboxSlots = 4;


// ---------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ float4 lds128f(const uint8_t* p) { return *reinterpret_cast<const float4*>(p); }

// byte i of w (runtime i) as an unsigned int
__device__ __forceinline__ uint32_t ubyte(uint32_t w, int i) { return __byte_perm(w, 0u, 0x4440u | (uint32_t)i); }
// exact float of a small non-negative integer v < 2^23, via the 2^23 magic number
__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.f; }
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
__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  __half2 h = __halves2half2(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  mma_f16_16816_acc(d, a0, a1, a2, a3, b0, b1);
}


// Wait for the barrier phase with the given parity.  Returns false when the CTA
// has aborted, or when the wait ran out (then this thread records the timeout
// and sets the abort word for the others).
__device__ __forceinline__ bool wait_phase(const GemvParams& P, uint64_t* bar, uint32_t parity,
                                           volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      record_error(P, DRACO_ERR_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
}

// Stage generation words: the producer stores round m once the stage is free
// for it; a converter waits until the word reaches its slab's round.
__device__ __forceinline__ void gen_publish(int* g, int m) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(g)), "r"(m) : "memory");
}
__device__ __forceinline__ int gen_read(const int* g) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(g)) : "memory");
  return v;
}
__device__ __forceinline__ bool wait_generation(const GemvParams& P, const int* g, int m, volatile int* abort) {
  if (gen_read(g) >= m) return true;
  const uint64_t t0 = global_timer_ns();
  while (gen_read(g) < m) {
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      record_error(P, DRACO_ERR_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
  return true;
}


// ---------------------------------------------------------------------------
// int8 tensor-core MMA (legacy warp-level path, exact int32 accumulation)
//   m16n8k32: A 16x32 (a0: row g, k 4t..4t+3; a1: row g+8; a2: row g, k 16+4t..;
//             a3: row g+8, k 16+4t..), B 32x8 (b0: k 4t..4t+3, col g; b1: k 16+4t..)
//   m16n8k16: A 16x16 (a0: row g, k 4t..; a1: row g+8), B 16x8 (b0: k 4t.., col g)
//   D 16x8 s32: d0, d1 -> (row g, cols 2t, 2t+1); d2, d3 -> row g+8
// ---------------------------------------------------------------------------
__device__ __forceinline__ void imma_u8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma_s8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma_u8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a0), "r"(a1), "r"(b0));
}
// first MMA of an accumulation chain: zero accumulator input (no register moves)
__device__ __forceinline__ void imma_u8_k32_first(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                  uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void imma_s8_k32_first(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                  uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void imma_u8_k16_first(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}
// x * v for a 6-bit integer v given as the float bits of 2^23 + v: one FMA
// whose exact result x * v (at most 17 significant bits for an fp16 x) is
// representable, so the single rounding returns it exactly.
__device__ __forceinline__ float mul_small(float x, uint32_t v_bits, float neg_x_2p23) {
  return fmaf(x, __uint_as_float(v_bits), neg_x_2p23);
}
// the two activation digits of one row: x / u = 256 * hi + lo
__device__ __forceinline__ float digits(int hi, int lo) { return __int2float_rn(hi * 256 + lo); }

constexpr uint32_t kNib = 0x0F0F0F0Fu;
constexpr uint32_t kNibHi = 0xF0F0F0F0u;

// ---------------------------------------------------------------------------
// activation conversion of one slab (problem pr, super-block j) by one warp.
// Lane quad (lane / 4) takes the 32-element group m of a batch row, lane % 4
// eight of its elements.  Per group: u = 2^e with max|x| / u in [2^13, 2^14),
// q = rint(x / u) split into two int8 digits q = 256 * hi + lo, and the sums
// S = u * sum(q) of its two 16-element halves.
//   xs[m][col][t][8 B]: bytes 0-3 = digits of elements 4t..4t+3, bytes 4-7 =
//       elements 16+4t..16+4t+3; the column is
//         dense   : 2b + digit
//         diagonal: ((sub-block mod G) * Bp + b) * 2 + digit,  G = 4 / Bp,
//       a Q4_K / Q8_0 sub-block being the group and a Q6_K sub-block one half
//       (the halves then go to different columns); unused slots hold zeros;
//   su[m][b] = (S_half0, S_half1, u, S_half0 + S_half1) (all exact).
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

template <int G, int NT>
__device__ __forceinline__ void convert_slab(const GemvParams& P, const GemvProbDev& pr, int j, uint8_t* xs,
                                             uint8_t* su, int lane) {
  constexpr bool kDiag = G > 1;
  constexpr int Bp = kDiag ? 4 / G : 4 * NT;
  constexpr int kCols = 8 * NT;
  constexpr int kSlots = 4 * NT;
  const int m = lane >> 2, r = lane & 3, kap = r >> 1, t0 = 2 * (r & 1);
  const int kk0 = 256 * j + 32 * m + 8 * r;
  const bool q6 = pr.qt == kQ6_K;
  // Dense layouts (batch >= 3): the x values of kPre batch rows are loaded
  // before any of them is converted, so a slab's L2 round trips overlap
  // instead of following one another, one per row.
  constexpr int kPre = kDiag ? 1 : 4;
  for (int b0 = 0; b0 < P.batch; b0 += kPre) {
    float vv[kPre][8];
#pragma unroll
    for (int q = 0; q < kPre; ++q) {
      const int b = b0 + q;
      if (b >= P.batch) break;
      load8(pr.x + (int64_t)b * pr.ldx + kk0, pr.k - kk0, vv[q]);
      if (pr.in_mode != DRACO_INPUT_PLAIN) {
        // the layer boundary, read in place: the RMSNorm weight (the row
        // scale is applied to the outputs) or the SwiGLU product
        float a[8];
        const bool sw = pr.in_mode == DRACO_INPUT_SWIGLU;
        load8(pr.aux + (sw ? (int64_t)b * pr.ldaux : 0) + kk0, pr.k - kk0, a);
#pragma unroll
        for (int i = 0; i < 8; ++i) vv[q][i] = sw ? silu_mul(vv[q][i], a[i]) : vv[q][i] * a[i];
      }
    }
#pragma unroll
    for (int q = 0; q < kPre; ++q) {
    const int b = b0 + q;
    if (b >= P.batch) break;  // uniform across the warp
    const float (&v)[8] = vv[q];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    // e = floor(log2 max|x|) - 13 from the exponent field (clamped, so subnormal
    // and zero groups take the smallest step and inf/nan the largest)
    int e = ((__float_as_int(amax) >> 23) & 0xFF) - 127 - 13;
    e = max(-110, min(110, e));
    const float inv = __int_as_float((127 - e) << 23), u = __int_as_float((127 + e) << 23);
    int hi[8], lo[8], qs = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // round to nearest even via the 1.5 * 2^23 magic number (|x / u| < 2^14)
      const int q = __float_as_int(fmaf(v[i], inv, 12582912.f)) - 0x4B400000;
      hi[i] = (q + 128) >> 8;
      lo[i] = q - (hi[i] << 8);
      qs += q;
    }
    qs += __shfl_xor_sync(0xffffffffu, qs, 1);               // sum of this 16-element half
    const int qs_other = __shfl_xor_sync(0xffffffffu, qs, 2);  // the group's other half
    if (r == 0)
      *reinterpret_cast<float4*>(su + (m * kSlots + b) * 16) =
          make_float4(__int2float_rn(qs) * u, __int2float_rn(qs_other) * u, u, __int2float_rn(qs + qs_other) * u);
    uint32_t dh[2], dl[2];
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
      dh[tt] = pack4(hi[4 * tt], hi[4 * tt + 1], hi[4 * tt + 2], hi[4 * tt + 3]);
      dl[tt] = pack4(lo[4 * tt], lo[4 * tt + 1], lo[4 * tt + 2], lo[4 * tt + 3]);
    }
    uint8_t* base = xs + (size_t)m * kCols * 32 + (size_t)t0 * 8 + 4 * kap;
    if constexpr (kDiag) {
      // The stages start zeroed and a cell of this lane only ever holds digits
      // at the slot of a Q6_K slab or at the slot of a Q4_K / Q8_0 slab: write
      // this slab's slot and clear the other type's, if it differs.
      const int slot = (q6 ? (2 * m + kap) : m) % G;
      const int other = (q6 ? m : (2 * m + kap)) % G;
#pragma unroll
      for (int dg = 0; dg < 2; ++dg) {
        const int col = (slot * Bp + b) * 2 + dg;
#pragma unroll
        for (int tt = 0; tt < 2; ++tt)
          *reinterpret_cast<uint32_t*>(base + col * 32 + tt * 8) = dg ? dl[tt] : dh[tt];
      }
      if (other != slot) {
#pragma unroll
        for (int dg = 0; dg < 2; ++dg) {
          const int col = (other * Bp + b) * 2 + dg;
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) *reinterpret_cast<uint32_t*>(base + col * 32 + tt * 8) = 0u;
        }
      }
    } else {
      (void)q6;
#pragma unroll
      for (int dg = 0; dg < 2; ++dg)
#pragma unroll
        for (int tt = 0; tt < 2; ++tt)
          *reinterpret_cast<uint32_t*>(base + (2 * b + dg) * 32 + tt * 8) = dg ? dl[tt] : dh[tt];
    }
    }
  }
}

// ---------------------------------------------------------------------------
// per-chunk consumers: one warp, one 16-row x 256-element chunk.
//   ch : chunk bytes in smem;  xs : slab activation slice [8 groups][8NT cols][4][8 B]
//   su : [8 groups][4NT slots][float4]
//   G  : sub-blocks per accumulator (4: batch 1, 2: batch 2, 1: dense)
//   acc[nt][0] -> (row g, batch b), acc[nt][1] -> (row g+8, batch b), with
//   b = t % Bp (diagonal, nt = 0) or 4 nt + t (dense)
// ---------------------------------------------------------------------------
// Q4_K (d * sc, dmin * m) of sub-block j for the row whose 12 scale bytes are
// (A, Bw, C) (gguf.py:436-442).
__device__ __forceinline__ void q4k_sm(uint32_t A, uint32_t Bw, uint32_t C, float d, float dmin, int j,
                                       bool upper, float& ds, float& mm) {
  uint32_t sc, m;
  if (!upper) {
    sc = ubyte(A, j) & 63u;
    m = ubyte(Bw, j) & 63u;
  } else {
    const int i = j - 4;
    const uint32_t c = ubyte(C, i);
    sc = (c & 15u) | ((ubyte(A, i) >> 6) << 4);
    m = (c >> 4) | ((ubyte(Bw, i) >> 6) << 4);
  }
  ds = d * u2f(sc);
  mm = dmin * u2f(m);
}

// fifth bits of four Q5_K quants: bit `b` of each byte of the qh word h,
// moved to bit 4 (gguf.py:457-467)
__device__ __forceinline__ uint32_t q5_bit4(uint32_t h, int b) {
  return (b <= 4 ? (h << (4 - b)) : (h >> (b - 4))) & 0x10101010u;
}

// Q4_K and Q5_K (same scales and mins; Q5_K adds a fifth bit per quant from
// its qh unit, which mirrors the qs unit word for word)
template <int QT, int G, int NT>
__device__ __forceinline__ void chunk_q4k(const uint8_t* ch, const uint8_t* xs, const uint8_t* su, int lane,
                                          float (&acc)[NT][2]) {
  constexpr bool k5 = QT == kQ5_K;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* sp0 = ch + (k5 ? 2560 : 2048) + 24 * g;  // row g: 12 bytes, row g+8: next 12
  const uint32_t A0 = lds32(sp0), B0 = lds32(sp0 + 4), C0 = lds32(sp0 + 8);
  const uint32_t A1 = lds32(sp0 + 12), B1 = lds32(sp0 + 16), C1 = lds32(sp0 + 20);
  const uint2 dd = lds64(ch + (k5 ? 2752 : 2240) + 8 * g);
  uint4 H = make_uint4(0, 0, 0, 0);
  if constexpr (k5) H = lds128(ch + 2048 + 16 * lane);
  const float d0 = f16_bits_to_f32(dd.x), m0 = f16_bits_to_f32(dd.x >> 16);
  const float d1 = f16_bits_to_f32(dd.y), m1 = f16_bits_to_f32(dd.y >> 16);
  constexpr int kColBytes = 8 * NT * 32;  // one group's activation entries
  if constexpr (G > 1) {
    constexpr int Bp = 4 / G, NF = 8 / G;
    int fr[NF][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 v = lds128(ch + 512 * q + 16 * lane);
      const uint2 bl = lds64(xs + (2 * q) * kColBytes + lane * 8);
      const uint2 bh = lds64(xs + (2 * q + 1) * kColBytes + lane * 8);
      uint32_t l0 = v.x & kNib, l1 = v.z & kNib, l2 = v.y & kNib, l3 = v.w & kNib;
      uint32_t h0, h1, h2, h3;
      if constexpr (k5) {
        l0 |= q5_bit4(H.x, 2 * q), l1 |= q5_bit4(H.z, 2 * q), l2 |= q5_bit4(H.y, 2 * q), l3 |= q5_bit4(H.w, 2 * q);
        h0 = ((v.x >> 4) & kNib) | q5_bit4(H.x, 2 * q + 1), h1 = ((v.z >> 4) & kNib) | q5_bit4(H.z, 2 * q + 1);
        h2 = ((v.y >> 4) & kNib) | q5_bit4(H.y, 2 * q + 1), h3 = ((v.w >> 4) & kNib) | q5_bit4(H.w, 2 * q + 1);
      } else {
        // high nibbles in place: 16 x the quant (exact in the int32 sum)
        h0 = v.x & kNibHi, h1 = v.z & kNibHi, h2 = v.y & kNibHi, h3 = v.w & kNibHi;
      }
      if ((2 * q) % G == 0) imma_u8_k32_first(fr[(2 * q) / G], l0, l1, l2, l3, bl.x, bl.y);
      else imma_u8_k32(fr[(2 * q) / G], l0, l1, l2, l3, bl.x, bl.y);
      imma_u8_k32(fr[(2 * q + 1) / G], h0, h1, h2, h3, bh.x, bh.y);
    }
    const int b = t % Bp;
    // this lane's sub-blocks j = f * G + t / Bp all have the same parity: odd
    // Q4_K sub-blocks were entered as 16 x the quant, so fold 1/16 into d
    const float h = (!k5 && ((t / Bp) & 1)) ? 0.0625f : 1.f;
    const float dq0 = d0 * h, dq1 = d1 * h;
    const float ndq0 = dq0 * -8388608.f, ndq1 = dq1 * -8388608.f;
    const float nm0 = m0 * -8388608.f, nm1 = m1 * -8388608.f;
    constexpr uint32_t kMag = 0x4B000000u;  // float bits of 2^23
#pragma unroll
    for (int f = 0; f < NF; ++f) {
      const int j = f * G + t / Bp;  // this lane's sub-block in accumulator f
      uint32_t sc0, mn0, sc1, mn1;   // float bits of 2^23 + the 6-bit scale / min (gguf.py:436-442)
      if (f * G < 4) {
        const uint32_t sel = 0x7440u | (uint32_t)j;  // byte j, two zero bytes, 0x4B
        sc0 = __byte_perm(A0, kMag, sel) & 0x4B00003Fu;
        mn0 = __byte_perm(B0, kMag, sel) & 0x4B00003Fu;
        sc1 = __byte_perm(A1, kMag, sel) & 0x4B00003Fu;
        mn1 = __byte_perm(B1, kMag, sel) & 0x4B00003Fu;
      } else {
        const uint32_t sel = 0x0040u | (uint32_t)(j - 4) | ((uint32_t)(j - 4) << 4);  // {C[i], X[i], 0, 0}
        const uint32_t xa0 = __byte_perm(C0, A0, sel), xb0 = __byte_perm(C0, B0, sel);
        const uint32_t xa1 = __byte_perm(C1, A1, sel), xb1 = __byte_perm(C1, B1, sel);
        // scale: C[i] & 15 | (A[i] >> 6) << 4;  min: C[i] >> 4 | (B[i] >> 6) << 4
        sc0 = ((xa0 & 15u) | kMag) | ((xa0 >> 10) & 0x30u);
        mn0 = (((xb0 >> 4) & 15u) | kMag) | ((xb0 >> 10) & 0x30u);
        sc1 = ((xa1 & 15u) | kMag) | ((xa1 >> 10) & 0x30u);
        mn1 = (((xb1 >> 4) & 15u) | kMag) | ((xb1 >> 10) & 0x30u);
      }
      const float4 s = lds128f(su + (j * 4 + b) * 16);  // (S_half0, S_half1, u, S)
      const float ds0 = mul_small(dq0, sc0, ndq0), ds1 = mul_small(dq1, sc1, ndq1);
      const float mm0 = mul_small(m0, mn0, nm0), mm1 = mul_small(m1, mn1, nm1);
      acc[0][0] = fmaf(ds0, s.z * digits(fr[f][0], fr[f][1]), fmaf(-mm0, s.w, acc[0][0]));
      acc[0][1] = fmaf(ds1, s.z * digits(fr[f][2], fr[f][3]), fmaf(-mm1, s.w, acc[0][1]));
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float dsl0, mml0, dsl1, mml1, dsh0, mmh0, dsh1, mmh1;
      q4k_sm(A0, B0, C0, d0, m0, 2 * q, q >= 2, dsl0, mml0);
      q4k_sm(A1, B1, C1, d1, m1, 2 * q, q >= 2, dsl1, mml1);
      q4k_sm(A0, B0, C0, d0, m0, 2 * q + 1, q >= 2, dsh0, mmh0);
      q4k_sm(A1, B1, C1, d1, m1, 2 * q + 1, q >= 2, dsh1, mmh1);
      const uint4 v = lds128(ch + 512 * q + 16 * lane);
      uint32_t l0 = v.x & kNib, l1 = v.z & kNib, l2 = v.y & kNib, l3 = v.w & kNib;
      uint32_t h0 = (v.x >> 4) & kNib, h1 = (v.z >> 4) & kNib, h2 = (v.y >> 4) & kNib, h3 = (v.w >> 4) & kNib;
      if constexpr (k5) {
        l0 |= q5_bit4(H.x, 2 * q), l1 |= q5_bit4(H.z, 2 * q), l2 |= q5_bit4(H.y, 2 * q), l3 |= q5_bit4(H.w, 2 * q);
        h0 |= q5_bit4(H.x, 2 * q + 1), h1 |= q5_bit4(H.z, 2 * q + 1);
        h2 |= q5_bit4(H.y, 2 * q + 1), h3 |= q5_bit4(H.w, 2 * q + 1);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 bl = lds64(xs + (2 * q) * kColBytes + nt * 256 + lane * 8);
        const uint2 bh = lds64(xs + (2 * q + 1) * kColBytes + nt * 256 + lane * 8);
        int c[4], e[4];
        imma_u8_k32_first(c, l0, l1, l2, l3, bl.x, bl.y);
        imma_u8_k32_first(e, h0, h1, h2, h3, bh.x, bh.y);
        const float4 sl = lds128f(su + ((2 * q) * 4 * NT + 4 * nt + t) * 16);
        const float4 sh = lds128f(su + ((2 * q + 1) * 4 * NT + 4 * nt + t) * 16);
        float r0 = acc[nt][0], r1 = acc[nt][1];
        r0 = fmaf(dsl0 * sl.z, digits(c[0], c[1]), fmaf(-mml0, sl.w, r0));
        r1 = fmaf(dsl1 * sl.z, digits(c[2], c[3]), fmaf(-mml1, sl.w, r1));
        r0 = fmaf(dsh0 * sh.z, digits(e[0], e[1]), fmaf(-mmh0, sh.w, r0));
        r1 = fmaf(dsh1 * sh.z, digits(e[2], e[3]), fmaf(-mmh1, sh.w, r1));
        acc[nt][0] = r0;
        acc[nt][1] = r1;
      }
    }
  }
}

// q6 bytes (0..63) of four elements: low nibble from word l (>> 4 for i >= 2),
// high 2 bits from qh word h (bits 2i, 2i+1) (gguf.py:476-494)
__device__ __forceinline__ uint32_t q6_bytes(uint32_t l, uint32_t h, int i) {
  const uint32_t nib = (i < 2 ? l : (l >> 4)) & kNib;
  const uint32_t hb = (i < 2 ? (h << (4 - 2 * i)) : (h >> (2 * i - 4))) & 0x30303030u;
  return nib | hb;
}

template <int G, int NT>
__device__ __forceinline__ void chunk_q6k(const uint8_t* ch, const uint8_t* xs, const uint8_t* su, int lane,
                                          float (&acc)[NT][2]) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* scp = ch + 3072 + 32 * g;  // row g: 16 int8 scales, row g+8: next 16
  const uint32_t dw = lds32(ch + 3328 + 4 * g);
  const float d0 = f16_bits_to_f32(dw), d1 = f16_bits_to_f32(dw >> 16);
  uint32_t W[24];
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const uint4 v = lds128(ch + 512 * i + 16 * lane);
    W[4 * i] = v.x; W[4 * i + 1] = v.y; W[4 * i + 2] = v.z; W[4 * i + 3] = v.w;
  }
  constexpr int kColBytes = 8 * NT * 32;
  if constexpr (G > 1) {
    constexpr int Bp = 4 / G, NF = 16 / G;
    int fr[NF][4];
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = 4 * n + i;  // 32-element group: sub-blocks 2m (elements 0-15) and 2m+1
        const uint2 bx = lds64(xs + m * kColBytes + lane * 8);
        const int w0 = 6 * (2 * n), w1 = 6 * (2 * n + 1);  // words of the two 16-element halves
        const uint32_t a0 = q6_bytes(W[w0 + (i & 1)], W[w0 + 2], i);
        const uint32_t a1 = q6_bytes(W[w0 + 3 + (i & 1)], W[w0 + 5], i);
        const uint32_t a2 = q6_bytes(W[w1 + (i & 1)], W[w1 + 2], i);
        const uint32_t a3 = q6_bytes(W[w1 + 3 + (i & 1)], W[w1 + 5], i);
        if ((2 * m) % G == 0) imma_u8_k32_first(fr[(2 * m) / G], a0, a1, a2, a3, bx.x, bx.y);
        else imma_u8_k32(fr[(2 * m) / G], a0, a1, a2, a3, bx.x, bx.y);
      }
    const int b = t % Bp;
#pragma unroll
    for (int f = 0; f < NF; ++f) {
      const int s = f * G + t / Bp;
      const float a0 = d0 * (float)(int8_t)scp[s];
      const float a1 = d1 * (float)(int8_t)scp[16 + s];
      const float4 sv = lds128f(su + ((s >> 1) * 4 + b) * 16);
      const float S = (s & 1) ? sv.y : sv.x;
      acc[0][0] = fmaf(a0, fmaf(-32.f, S, sv.z * digits(fr[f][0], fr[f][1])), acc[0][0]);
      acc[0][1] = fmaf(a1, fmaf(-32.f, S, sv.z * digits(fr[f][2], fr[f][3])), acc[0][1]);
    }
  } else {
    const uint4 s0a = lds128(scp), s0b = lds128(scp + 16);  // rows g, g+8: sc[0..15]
    const uint32_t sw0[4] = {s0a.x, s0a.y, s0a.z, s0a.w};
    const uint32_t sw1[4] = {s0b.x, s0b.y, s0b.z, s0b.w};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = 4 * n + i;
#pragma unroll
        for (int is = 0; is < 2; ++is) {
          const int w = 6 * (2 * n + is), s = 2 * m + is;
          const uint32_t a0 = q6_bytes(W[w + (i & 1)], W[w + 2], i);
          const uint32_t a1 = q6_bytes(W[w + 3 + (i & 1)], W[w + 5], i);
          const float al0 = d0 * sbyte_f(sw0[s >> 2], s & 3);
          const float al1 = d1 * sbyte_f(sw1[s >> 2], s & 3);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint2 bx = lds64(xs + m * kColBytes + nt * 256 + lane * 8);
            const float4 sv = lds128f(su + (m * 4 * NT + 4 * nt + t) * 16);
            int c[4];
            imma_u8_k16_first(c, a0, a1, is ? bx.y : bx.x);
            const float S = is ? sv.y : sv.x;
            acc[nt][0] = fmaf(al0, fmaf(-32.f, S, sv.z * digits(c[0], c[1])), acc[nt][0]);
            acc[nt][1] = fmaf(al1, fmaf(-32.f, S, sv.z * digits(c[2], c[3])), acc[nt][1]);
          }
        }
      }
  }
}

template <int G, int NT>
__device__ __forceinline__ void chunk_q80(const uint8_t* ch, const uint8_t* xs, const uint8_t* su, int lane,
                                          float (&acc)[NT][2]) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* dp = ch + 4096 + 32 * g;  // row g: 8 fp16 d, row g+8: next 8
  constexpr int kColBytes = 8 * NT * 32;
  if constexpr (G > 1) {
    constexpr int Bp = 4 / G, NF = 8 / G;
    int fr[NF][4];
#pragma unroll
    for (int bk = 0; bk < 8; ++bk) {
      const uint4 v = lds128(ch + 512 * bk + 16 * lane);
      const uint2 bx = lds64(xs + bk * kColBytes + lane * 8);
      if (bk % G == 0) imma_s8_k32_first(fr[bk / G], v.x, v.z, v.y, v.w, bx.x, bx.y);
      else imma_s8_k32(fr[bk / G], v.x, v.z, v.y, v.w, bx.x, bx.y);
    }
    const int b = t % Bp;
#pragma unroll
    for (int f = 0; f < NF; ++f) {
      const int bk = f * G + t / Bp;
      const float dg = ld_f16(dp + 2 * bk), dg8 = ld_f16(dp + 16 + 2 * bk);
      const float u = lds128f(su + (bk * 4 + b) * 16).z;
      acc[0][0] = fmaf(dg * u, digits(fr[f][0], fr[f][1]), acc[0][0]);
      acc[0][1] = fmaf(dg8 * u, digits(fr[f][2], fr[f][3]), acc[0][1]);
    }
  } else {
#pragma unroll
    for (int bk = 0; bk < 8; ++bk) {
      const uint4 v = lds128(ch + 512 * bk + 16 * lane);
      const float dg = ld_f16(dp + 2 * bk), dg8 = ld_f16(dp + 16 + 2 * bk);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 bx = lds64(xs + bk * kColBytes + nt * 256 + lane * 8);
        const float u = lds128f(su + (bk * 4 * NT + 4 * nt + t) * 16).z;
        int c[4];
        imma_s8_k32_first(c, v.x, v.z, v.y, v.w, bx.x, bx.y);
        acc[nt][0] = fmaf(dg * u, digits(c[0], c[1]), acc[nt][0]);
        acc[nt][1] = fmaf(dg8 * u, digits(c[2], c[3]), acc[nt][1]);
      }
    }
  }
}

// fifth bits of four quants at bit 4 of each byte: bit i of the 4-bit x goes
// to byte i (the four shifted copies of x do not overlap, so no carries)
__device__ __forceinline__ uint32_t spread4(uint32_t x) { return (x * 0x02040810u) & 0x10101010u; }

// Q4_0 / Q4_1 / Q5_0 / Q5_1 (gguf.py:310-353).  Per block of 32 the quant q
// (0..15, or 0..31 with the fifth bit) gives w = d * q + c with c = -8 d
// (Q4_0), -16 d (Q5_0) or m (Q4_1, Q5_1), so a block adds
//   d * u * (q . X) + c * S
// to the row: X the activation digits, S = u * sum(X) the group sum.  A lane's
// word of a block row holds qs bytes 4t..4t+3: the low nibbles are the MMA's
// k columns 4t..4t+3, the high nibbles its columns 16+4t..16+4t+3.
template <int QT, int G, int NT>
__device__ __forceinline__ void chunk_q4x(const uint8_t* ch, const uint8_t* xs, const uint8_t* su, int lane,
                                          float (&acc)[NT][2]) {
  constexpr bool kH = QT == kQ5_0 || QT == kQ5_1;  // fifth bit in qh
  constexpr bool kM = QT == kQ4_1 || QT == kQ5_1;  // fp16 m per block
  constexpr int kD = kH ? 2560 : 2048, kQh = 2048, kMo = kD + 256;
  constexpr float kOff = QT == kQ4_0 ? -8.f : -16.f;  // c / d without m
  const int g = lane >> 2, t = lane & 3;
  // the 8 fp16 d (and m) of row g, then those of row g + 8
  const uint4 dv0 = lds128(ch + kD + 32 * g), dv1 = lds128(ch + kD + 32 * g + 16);
  uint4 mv0 = make_uint4(0, 0, 0, 0), mv1 = mv0;
  if constexpr (kM) mv0 = lds128(ch + kMo + 32 * g), mv1 = lds128(ch + kMo + 32 * g + 16);
  auto half_of = [](const uint4& v, int b) {
    const uint32_t w = b < 2 ? (b == 0 ? v.x : v.x >> 16) : b < 4 ? (b == 2 ? v.y : v.y >> 16)
                     : b < 6 ? (b == 4 ? v.z : v.z >> 16) : (b == 6 ? v.w : v.w >> 16);
    return f16_bits_to_f32(w);
  };
  // the four A operands of block b (pair word v): rows g / g+8, columns
  // 4t.. / 16+4t..
  auto operands = [&](const uint4& v, int b, uint32_t (&a)[4]) {
    const uint32_t w0 = (b & 1) ? v.z : v.x, w1 = (b & 1) ? v.w : v.y;
    a[0] = w0 & kNib, a[1] = w1 & kNib, a[2] = (w0 >> 4) & kNib, a[3] = (w1 >> 4) & kNib;
    if constexpr (kH) {
      const uint32_t h0 = lds32(ch + kQh + 64 * g + 4 * b), h1 = lds32(ch + kQh + 64 * g + 32 + 4 * b);
      a[0] |= spread4((h0 >> (4 * t)) & 15u), a[1] |= spread4((h1 >> (4 * t)) & 15u);
      a[2] |= spread4((h0 >> (16 + 4 * t)) & 15u), a[3] |= spread4((h1 >> (16 + 4 * t)) & 15u);
    }
  };
  constexpr int kColBytes = 8 * NT * 32;
  if constexpr (G > 1) {
    constexpr int Bp = 4 / G, NF = 8 / G;
    int fr[NF][4];
#pragma unroll
    for (int pr = 0; pr < 4; ++pr) {
      const uint4 v = lds128(ch + 512 * pr + 16 * lane);
#pragma unroll
      for (int bo = 0; bo < 2; ++bo) {
        const int bk = 2 * pr + bo;
        uint32_t a[4];
        operands(v, bk, a);
        const uint2 bx = lds64(xs + bk * kColBytes + lane * 8);
        if (bk % G == 0) imma_u8_k32_first(fr[bk / G], a[0], a[1], a[2], a[3], bx.x, bx.y);
        else imma_u8_k32(fr[bk / G], a[0], a[1], a[2], a[3], bx.x, bx.y);
      }
    }
    const int b = t % Bp;
#pragma unroll
    for (int f = 0; f < NF; ++f) {
      const int bk = f * G + t / Bp;  // this lane's block in accumulator f
      const float d0 = half_of(dv0, bk), d1 = half_of(dv1, bk);
      const float c0 = kM ? half_of(mv0, bk) : kOff * d0, c1 = kM ? half_of(mv1, bk) : kOff * d1;
      const float4 s = lds128f(su + (bk * 4 + b) * 16);  // (S_half0, S_half1, u, S)
      acc[0][0] = fmaf(d0 * s.z, digits(fr[f][0], fr[f][1]), fmaf(c0, s.w, acc[0][0]));
      acc[0][1] = fmaf(d1 * s.z, digits(fr[f][2], fr[f][3]), fmaf(c1, s.w, acc[0][1]));
    }
  } else {
#pragma unroll
    for (int pr = 0; pr < 4; ++pr) {
      const uint4 v = lds128(ch + 512 * pr + 16 * lane);
#pragma unroll
      for (int bo = 0; bo < 2; ++bo) {
        const int bk = 2 * pr + bo;
        uint32_t a[4];
        operands(v, bk, a);
        const float d0 = half_of(dv0, bk), d1 = half_of(dv1, bk);
        const float c0 = kM ? half_of(mv0, bk) : kOff * d0, c1 = kM ? half_of(mv1, bk) : kOff * d1;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint2 bx = lds64(xs + bk * kColBytes + nt * 256 + lane * 8);
          const float4 s = lds128f(su + (bk * 4 * NT + 4 * nt + t) * 16);
          int c[4];
          imma_u8_k32_first(c, a[0], a[1], a[2], a[3], bx.x, bx.y);
          acc[nt][0] = fmaf(d0 * s.z, digits(c[0], c[1]), fmaf(c0, s.w, acc[nt][0]));
          acc[nt][1] = fmaf(d1 * s.z, digits(c[2], c[3]), fmaf(c1, s.w, acc[nt][1]));
        }
      }
    }
  }
}

// RMSNorm row scales of a batch-1 launch, computed by the converter warps of
// every CTA (one warp per problem, the conversion kernel's summation order)
__shared__ float g_rms_scale[DRACO_GEMV_MAX_PROBLEMS];
constexpr int kRmsBarrier = 2;  // named barrier: converters publish g_rms_scale, consumers wait

// rsqrt(mean(x^2) + eps) of one row (draco/kernels/ops.py:46-48), summed in a
// fixed order by one warp: lane l takes elements l, l + 32, ..., then a
// butterfly; gemv_convert_kernel and the batch-1 converters share it, so
// every CTA and both paths get the same bits
__device__ __forceinline__ float rms_row_scale(const float* xr, int k, float eps, int lane) {
  float ss = 0.f;
#pragma unroll 8
  for (int i = lane; i < k; i += 32) ss = fmaf(xr[i], xr[i], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return 1.f / sqrtf(ss / (float)k + eps);
}

// ---------------------------------------------------------------------------
// output of one row group
// ---------------------------------------------------------------------------
template <int NT, bool TP>
__device__ __forceinline__ void write_rows(const GemvParams& P, const GemvProbDev& pr, int rg, int rw, int lane,
                                           const float (&v)[NT][2]) {
  // tensor-parallel: this step's parity (the own step counter + 1; it only
  // changes after every CTA of this launch has finished)
  int tp_par = 0;
  if constexpr (TP) tp_par = (*reinterpret_cast<volatile int*>(P.tp_buf[P.tp_rank] + P.tp_counter_off) + 1) & 1;
  const int g = lane >> 2, t = lane & 3;
  const int64_t row0 = ((int64_t)rg * kGroupTiles + rw) * kChunkRows + g;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int b = 4 * nt + t;
    if (b >= P.batch) continue;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int64_t row = row0 + 8 * hh;
      if (row < pr.n_rows) {
        float out = v[nt][hh];
        if (pr.in_mode == DRACO_INPUT_RMSNORM)
          out *= P.rms_inkernel ? g_rms_scale[pr.pidx] : __ldcg(reinterpret_cast<const float*>(P.ws + pr.rms_off) + b);
        if (pr.bias) out += pr.bias[row];
        if constexpr (!TP) {
          if (pr.accumulate) out += pr.y[(int64_t)b * pr.ldy + row];
          pr.y[(int64_t)b * pr.ldy + row] = out;
        } else {
          const int64_t off = pr.tp_y_off + (int64_t)tp_par * pr.tp_par_stride + ((int64_t)b * pr.ldy + row) * 4;
          for (int q = 0; q < P.tp_world; ++q) *reinterpret_cast<float*>(P.tp_buf[q] + off) = out;
        }
      }
    }
  }
}

__device__ __forceinline__ int cta_of_slab(const GemvParams& P, int s) {
  int lo = 0, hi = P.n_cta - 1;  // largest c with cta_start[c] <= s
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (P.cta_start[mid] <= s) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Row-group mailbox in shared memory: for the L-th row group of the CTA's
// range (slot L % mbox_slots), the two consumer warps sharing row tile rw
// (one per slab parity) each deposit their partial sums in their half; the
// second to arrive adds both and finishes the rows.  No CTA-wide barrier: each
// warp moves on to its next slabs as soon as it has deposited.
struct Mailbox {
  float* data;  // [slots][2 parities][kRowWarps][32 lanes][2 NT]
  int* tag;     // [slots][kRowWarps]: 1 + L of the row group held, 0 = free
  int* cnt;     // [slots][kRowWarps]: arrivals so far
  int slots;
};

// Called by each consumer warp at the end of its part of a row group.
// Returns false when the CTA aborted (the row group is then left unwritten).
template <int G, int NT, bool TP>
__device__ bool finish_rowgroup(const GemvParams& P, int p, int rg, int L, int s_begin, int s_end, int warp, int lane,
                                float (&acc)[NT][2], const Mailbox& mb, volatile int* abort) {
  const GemvProbDev& pr = P.prob[p];
  const int nrt = rg_tile_count(pr, rg);
  const int rw = warp & (kRowWarps - 1), par = warp / kRowWarps;
  if constexpr (G > 1) {
    // diagonal layout: lanes t with the same batch slot hold different sub-blocks
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      if (G == 4) acc[0][hh] += __shfl_xor_sync(0xffffffffu, acc[0][hh], 1);
      acc[0][hh] += __shfl_xor_sync(0xffffffffu, acc[0][hh], 2);
    }
  }
  const int slot = L % mb.slots;
  volatile int* tagp = mb.tag + slot * kRowWarps + rw;
  // the slot may still hold an older row group whose second warp has not
  // arrived yet (the stage ring bounds how far ahead a warp runs)
  int ok = 1;
  if (lane == 0) {
    const uint64_t t0 = global_timer_ns();
    while (true) {
      const int tg = *tagp;
      if (tg == 0 || tg == L + 1) break;
      if (*abort) {
        ok = 0;
        break;
      }
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_error(P, DRACO_ERR_TIMEOUT);
        *abort = 1;
        ok = 0;
        break;
      }
    }
    if (ok) atomicCAS(const_cast<int*>(tagp), 0, L + 1);
  }
  if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
  float* mine = mb.data + ((((int64_t)slot * 2 + par) * kRowWarps + rw) * 32 + lane) * (NT * 2);
  float* other = mb.data + ((((int64_t)slot * 2 + (par ^ 1)) * kRowWarps + rw) * 32 + lane) * (NT * 2);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    mine[2 * nt] = acc[nt][0];
    mine[2 * nt + 1] = acc[nt][1];
  }
  __threadfence_block();
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atomicAdd(mb.cnt + slot * kRowWarps + rw, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old == 0) return true;  // the partner finishes the rows
  __threadfence_block();
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    acc[nt][0] += other[2 * nt];
    acc[nt][1] += other[2 * nt + 1];
  }
  __syncwarp();
  if (lane == 0) {  // free the slot for row group L + slots
    mb.cnt[slot * kRowWarps + rw] = 0;
    __threadfence_block();
    *tagp = 0;
  }
  if (rw >= nrt) return true;
  const int rg_start = pr.slab0 + rg * pr.nb, rg_end = rg_start + pr.nb;
  if (s_begin <= rg_start && rg_end <= s_end) {
    write_rows<NT, TP>(P, pr, rg, rw, lane, acc);
    return true;
  }
  // split row group: publish this CTA's partial of row tile rw; the last
  // contributing CTA adds them in CTA order and writes the rows
  const int cta = blockIdx.x;
  const int cslot = (s_begin >= rg_start) ? 0 : 1;
  float* part = reinterpret_cast<float*>(P.ws + P.part_off) +
                ((((int64_t)cta * 2 + cslot) * kRowWarps + rw) * 32 + lane) * (NT * 2);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    __stcg(part + 2 * nt, acc[nt][0]);
    __stcg(part + 2 * nt + 1, acc[nt][1]);
  }
  __threadfence();
  __syncwarp();
  const int c_first = cta_of_slab(P, rg_start);
  const int c_last = cta_of_slab(P, rg_end - 1);
  int last = 0;
  if (lane == 0) {
    const int slot_first = (P.cta_start[c_first] >= rg_start) ? 0 : 1;
    unsigned int* cnt = reinterpret_cast<unsigned int*>(P.ws + P.cnt_off) + (c_first * 2 + slot_first) * kRowWarps + rw;
    const unsigned int o = atomicAdd(cnt, 1u);
    last = (o == (unsigned int)(c_last - c_first));
    if (last) {
      atomicExch(cnt, 0u);
      __threadfence();
    }
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return true;
  float sum[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) sum[nt][0] = sum[nt][1] = 0.f;
  for (int c = c_first; c <= c_last; ++c) {
    const int sl = (P.cta_start[c] >= rg_start) ? 0 : 1;
    const float* q = reinterpret_cast<const float*>(P.ws + P.part_off) +
                     ((((int64_t)c * 2 + sl) * kRowWarps + rw) * 32 + lane) * (NT * 2);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      sum[nt][0] += __ldcg(q + 2 * nt);
      sum[nt][1] += __ldcg(q + 2 * nt + 1);
    }
  }
  write_rows<NT, TP>(P, pr, rg, rw, lane, sum);
  return true;
}

// ---------------------------------------------------------------------------
// consumer side: the slabs of one row-group segment that have this warp's parity
// ---------------------------------------------------------------------------
// Returns false when the CTA aborted; the warp then frees no further stage.
// ready: this parity's ready barriers, stride 2 per stage.
template <int QT, int G, int NT>
__device__ __forceinline__ bool consume_segment(const GemvParams& P, const uint8_t* smem, uint64_t* ready,
                                                uint64_t* empty_bar, int i, int i_end, int NS, int rw, int nrt,
                                                int cb, int lane, volatile int* abort, float (&acc)[NT][2]) {
  if (i >= i_end) return true;
  int st = i % NS, m = i / NS;
  // phase of this slab on its parity's barriers of the stage: round m, or m / 2
  // with an odd NS (the stage's slabs alternate parities)
  const int sh = NS & 1;
  uint32_t ph = (uint32_t)((m >> sh) & 1);
  for (; i < i_end; i += 2) {
    // try_wait is one warp-wide test, so the branch is uniform
    if (!mbar_try_wait(&ready[2 * st], ph)) {
      if (!__all_sync(0xffffffffu, wait_phase(P, &ready[2 * st], ph, abort))) return false;
    }
    if (rw < nrt) {
      const uint8_t* stage = smem + (size_t)st * P.stage_bytes;
      const uint8_t* ch = stage + rw * cb;
      const uint8_t* xs = stage + P.w_stage;
      const uint8_t* su = xs + P.xs_bytes;
      if (QT == kQ4_K || QT == kQ5_K) chunk_q4k<QT, G, NT>(ch, xs, su, lane, acc);
      else if (QT == kQ6_K) chunk_q6k<G, NT>(ch, xs, su, lane, acc);
      else if (QT == kQ8_0) chunk_q80<G, NT>(ch, xs, su, lane, acc);
      else chunk_q4x<QT, G, NT>(ch, xs, su, lane, acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
    st += 2;
    if (st >= NS) {
      st -= NS;
      ++m;
      ph = (uint32_t)((m >> sh) & 1);
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// activation conversion once per launch (batch >= 3): one warp per
// (problem, super-block) slice, written in the stage layout (digits in
// MMA-fragment order, then the group sums), padded batch slots zero
// ---------------------------------------------------------------------------
constexpr int kConvertWarpsPerBlock = 4;

template <int NT>
__global__ void __launch_bounds__(kConvertWarpsPerBlock * 32) gemv_convert_kernel(const __grid_constant__ GemvParams P) {
  grid_launch_dependents();  // the GEMV may start streaming weights at once
  const int lane = threadIdx.x & 31;
  int u = blockIdx.x * kConvertWarpsPerBlock + (threadIdx.x >> 5), p = 0;
  while (p < P.n_prob && u >= P.prob[p].nb) u -= P.prob[p].nb, ++p;
  if (p >= P.n_prob) {
    // warps past the conversion units: one RMSNORM (problem, batch row) each,
    // the row's scale rsqrt(mean(x^2) + eps) (draco/kernels/ops.py:46-48),
    // summed in a fixed order (deterministic)
    for (p = 0; p < P.n_prob; ++p) {
      if (P.prob[p].in_mode != DRACO_INPUT_RMSNORM) continue;
      if (u < P.batch) break;
      u -= P.batch;
    }
    if (p >= P.n_prob) return;
    const GemvProbDev& pr = P.prob[p];
    const float r = rms_row_scale(pr.x + (int64_t)u * pr.ldx, pr.k, pr.eps, lane);
    if (lane == 0) reinterpret_cast<float*>(P.ws + pr.rms_off)[u] = r;
    return;
  }
  const int xb = P.xs_bytes + P.su_bytes;
  uint8_t* dst = P.ws + P.prob[p].xcv_off + (int64_t)u * xb;
  for (int i = lane; i < (xb >> 4); i += 32) reinterpret_cast<uint4*>(dst)[i] = make_uint4(0, 0, 0, 0);
  __syncwarp();
  if (P.batch == 1) convert_slab<4, 1>(P, P.prob[p], u, dst, dst + P.xs_bytes, lane);
  else if (P.batch == 2) convert_slab<2, 1>(P, P.prob[p], u, dst, dst + P.xs_bytes, lane);
  else convert_slab<1, NT>(P, P.prob[p], u, dst, dst + P.xs_bytes, lane);
}

// ---------------------------------------------------------------------------
// the persistent GEMV kernel
// ---------------------------------------------------------------------------
template <int G, int NT, bool TP>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  // [stage][slab parity]: the slab's weight bytes landed and its activations are converted
  __shared__ __align__(8) uint64_t ready_bar[2 * kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];  // the stage's consumers are done with it
  __shared__ int stage_gen[kMaxStages];                     // round the stage is free for
  __shared__ int mbox_tag[kMaxMboxSlots * kRowWarps], mbox_cnt[kMaxMboxSlots * kRowWarps];
  __shared__ int abort_word;
  __shared__ int prod_issued, prod_done;  // the producer's final issue count, once it is done
  volatile int* abort = &abort_word;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int s_begin = P.cta_start[cta], s_end = P.cta_start[cta + 1];
  const int NS = P.n_stages;
  const int n = s_end - s_begin;

  // zero the activation slices of the stages once: in the dense layout the
  // columns of padded batch slots are never written, in the diagonal layout
  // only the digit slots are
  for (int st = 0; st < NS; ++st) {
    uint4* z = reinterpret_cast<uint4*>(smem + (size_t)st * P.stage_bytes + P.w_stage);
    const int n16 = (P.xs_bytes + P.su_bytes) >> 4;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
  }
  for (int i = threadIdx.x; i < kMaxMboxSlots * kRowWarps; i += blockDim.x) mbox_tag[i] = mbox_cnt[i] = 0;
  if (threadIdx.x == 0) {
    abort_word = 0;
    prod_issued = prod_done = 0;
    for (int i = 0; i < NS; ++i) {
      // the producer (with the weight bytes) and the slab's converter
      mbar_init(&ready_bar[2 * i], 2);
      mbar_init(&ready_bar[2 * i + 1], 2);
      mbar_init(&empty_bar[i], kRowWarps);
      stage_gen[i] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  // allow the next kernel in the stream to launch; it waits for our completion
  // (griddepcontrol.wait) before touching anything we read or write
  grid_launch_dependents();

  if (warp == kProducerWarp) {
    // ---------------- producer: weights ----------------
    if (lane == 0) {
      SlabCursor cur;
      cur.seek(P, s_begin);
      int st = 0, issued = 0;
      uint32_t ph = 0;
      for (int i = 0; i < n; ++i) {
        if (i >= NS) {
          if (!wait_phase(P, &empty_bar[st], ph ^ 1u, abort)) break;
          gen_publish(&stage_gen[st], i / NS);
        }
        const GemvProbDev& pr = P.prob[cur.p];
        const int nrt = rg_tile_count(pr, cur.rg);
        const uint32_t wbytes = (uint32_t)(nrt * pr.cb);
        const int64_t woff = (int64_t)cur.rg * kGroupTiles * pr.nb * pr.cb + (int64_t)cur.j * nrt * pr.cb;
        uint64_t* rb = &ready_bar[2 * st + (i & 1)];
        mbar_arrive_expect_tx(rb, wbytes);
        bulk_g2s(smem + (size_t)st * P.stage_bytes, pr.w + woff, wbytes, rb);
        issued = i + 1;
        cur.next(P);
        if (++st == NS) {
          st = 0;
          ph ^= 1u;
        }
      }
      // tell the converters how far the producer got (they complete the ready
      // phases of issued slabs even after an abort)
      *reinterpret_cast<volatile int*>(&prod_issued) = issued;
      __threadfence_block();
      *reinterpret_cast<volatile int*>(&prod_done) = 1;
      // Only the last copy issued into a stage can still be in flight (each
      // earlier one was waited for before its stage was freed): wait for them,
      // so that the CTA never exits with a copy pending, even after an abort.
      const uint64_t t0 = global_timer_ns();
      for (int i = max(0, issued - NS); i < issued; ++i) {
        const int m = i / NS;
        uint64_t* rb = &ready_bar[2 * (i % NS) + (i & 1)];
        const uint32_t rph = (uint32_t)((m >> (NS & 1)) & 1);
        while (!mbar_try_wait(rb, rph)) {
          if (global_timer_ns() - t0 > kWaitLimitNs) {
            record_error(P, DRACO_ERR_TIMEOUT);
            *abort = 1;
            break;
          }
        }
      }
    }
    return;
  }

  if (warp > kProducerWarp) {
    // ---------------- converters: activations ----------------
    const int c = warp - kProducerWarp - 1;
    grid_dependency_wait();  // x is written by the preceding kernel
    if (P.rms_inkernel) {
      // batch 1: the RMSNorm row scales first (problem p by converter p % 3),
      // published to the consumers through a named barrier
      for (int p = c; p < P.n_prob; p += kConvWarps) {
        const GemvProbDev& pr = P.prob[p];
        if (pr.in_mode != DRACO_INPUT_RMSNORM) continue;
        const float r = rms_row_scale(pr.x, pr.k, pr.eps, lane);
        if (lane == 0) g_rms_scale[p] = r;
      }
      __syncwarp();
      asm volatile("bar.arrive %0, %1;" ::"n"(kRmsBarrier), "n"((kConvWarps + kConsumerWarps) * 32) : "memory");
    }
    SlabCursor cur;
    cur.seek(P, s_begin);
    for (int q = 0; q < c && q < n; ++q) cur.next(P);
    for (int i = c; i < n; i += kConvWarps) {
      const int st = i % NS, m = i / NS;
      if (m > 0 && !__all_sync(0xffffffffu, wait_generation(P, &stage_gen[st], m, abort))) {
        // aborted: once the producer is done, arrive for this converter's
        // remaining slabs that it issued, so their copies' phases complete
        const uint64_t t0 = global_timer_ns();
        while (!*reinterpret_cast<volatile int*>(&prod_done) && global_timer_ns() - t0 < kWaitLimitNs) {
        }
        __threadfence_block();
        const int issued = *reinterpret_cast<volatile int*>(&prod_issued);
        if (lane == 0)
          for (int r = i; r < issued; r += kConvWarps) mbar_arrive(&ready_bar[2 * (r % NS) + (r & 1)]);
        return;
      }
      uint8_t* xs = smem + (size_t)st * P.stage_bytes + P.w_stage;
      if (P.precvt) {
        // the slice was converted before the launch: one bulk copy, which the
        // stage's ready phase waits for along with the weight bytes
        if (lane == 0) {
          const uint32_t xb = (uint32_t)(P.xs_bytes + P.su_bytes);
          uint64_t* rb = &ready_bar[2 * st + (i & 1)];
          mbar_arrive_expect_tx(rb, xb);
          bulk_g2s(xs, P.ws + P.prob[cur.p].xcv_off + (int64_t)cur.j * xb, xb, rb);
        }
      } else {
        convert_slab<G, NT>(P, P.prob[cur.p], cur.j, xs, xs + P.xs_bytes, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready_bar[2 * st + (i & 1)]);
      }
      for (int q = 0; q < kConvWarps; ++q) cur.next(P);
    }
    return;
  }

  // ---------------- consumers ----------------
  grid_dependency_wait();  // y may still be read by the preceding kernel
  if (P.rms_inkernel)  // the converters' RMSNorm row scales (before any slab is ready)
    asm volatile("bar.sync %0, %1;" ::"n"(kRmsBarrier), "n"((kConvWarps + kConsumerWarps) * 32) : "memory");
  const int par = warp / kRowWarps, rw = warp % kRowWarps;

  float acc[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
  const Mailbox mb = {reinterpret_cast<float*>(smem + P.mbox_off), mbox_tag, mbox_cnt, P.mbox_slots};
  SlabCursor cur;
  cur.seek(P, s_begin);
  int s = s_begin;
  int L = 0;  // row groups finished in this CTA's range
  while (s < s_end) {
    const GemvProbDev& pr = P.prob[cur.p];
    const int seg = min(pr.nb - cur.j, s_end - s);  // slabs of this row group in our range
    const int i0 = s - s_begin;
    const int i_first = i0 + (((i0 & 1) != par) ? 1 : 0);
    const int nrt = rg_tile_count(pr, cur.rg);
    bool ok;
    if (pr.qt == kQ4_K)
      ok = consume_segment<kQ4_K, G, NT>(P, smem, ready_bar + par, empty_bar, i_first, i0 + seg, NS, rw, nrt,
                                         pr.cb, lane, abort, acc);
    else if (pr.qt == kQ5_K)
      ok = consume_segment<kQ5_K, G, NT>(P, smem, ready_bar + par, empty_bar, i_first, i0 + seg, NS, rw, nrt,
                                         pr.cb, lane, abort, acc);
    else if (pr.qt == kQ6_K)
      ok = consume_segment<kQ6_K, G, NT>(P, smem, ready_bar + par, empty_bar, i_first, i0 + seg, NS, rw, nrt,
                                         pr.cb, lane, abort, acc);
    else if (pr.qt == kQ8_0)
      ok = consume_segment<kQ8_0, G, NT>(P, smem, ready_bar + par, empty_bar, i_first, i0 + seg, NS, rw, nrt,
                                         pr.cb, lane, abort, acc);
    else if (pr.qt == kQ4_0)
      ok = consume_segment<kQ4_0, G, NT>(P, smem, ready_bar + par, empty_bar, i_first, i0 + seg, NS, rw, nrt,
                                         pr.cb, lane, abort, acc);
    else if (pr.qt == kQ4_1)
      ok = consume_segment<kQ4_1, G, NT>(P, smem, ready_bar + par, empty_bar, i_first, i0 + seg, NS, rw, nrt,
                                         pr.cb, lane, abort, acc);
    else if (pr.qt == kQ5_0)
      ok = consume_segment<kQ5_0, G, NT>(P, smem, ready_bar + par, empty_bar, i_first, i0 + seg, NS, rw, nrt,
                                         pr.cb, lane, abort, acc);
    else
      ok = consume_segment<kQ5_1, G, NT>(P, smem, ready_bar + par, empty_bar, i_first, i0 + seg, NS, rw, nrt,
                                         pr.cb, lane, abort, acc);
    if (!ok || !finish_rowgroup<G, NT, TP>(P, cur.p, cur.rg, L++, s_begin, s_end, warp, lane, acc, mb, abort))
      break;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
    s += seg;
    cur.j += seg;
    if (cur.j == pr.nb) {
      cur.j = 0;
      if (++cur.rg == pr.n_rg) {
        cur.rg = 0;
        ++cur.p;
      }
    }
  }
  if constexpr (!TP) return;
  // Tensor-parallel completion.  The consumer warps meet at a named barrier;
  // then one thread counts the CTA with a system-scope acquire-release atomic:
  // its release orders all of the CTA's peer stores (the barrier makes them
  // happen before it), and the last CTA's acquire sees every CTA's before it
  // signals every rank (epoch, or -epoch when this launch aborted).  (A
  // system-scope fence in every thread cost ~20 us per launch, one fence per
  // CTA ~10 us; the atomic ~8.5 us.)
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
  if (threadIdx.x == 0) {
    const int tp_epoch = *reinterpret_cast<volatile int*>(P.tp_buf[P.tp_rank] + P.tp_counter_off) + 1;
    const int tp_par = tp_epoch & 1;
    unsigned int* grid_done = reinterpret_cast<unsigned int*>(P.ws + kWsGridDone);
    unsigned int prev;
    asm volatile("atom.acq_rel.sys.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(grid_done) : "memory");
    if (prev == gridDim.x - 1) {
      *grid_done = 0u;
      const int sig = *reinterpret_cast<volatile int*>(P.ws + P.status_off) ? -tp_epoch : tp_epoch;
      for (int q = 0; q < P.tp_world; ++q)
        st_release_sys(reinterpret_cast<int*>(P.tp_buf[q] + P.tp_flags_off) + tp_par * DRACO_TP_MAX_WORLD + P.tp_rank,
                       sig);
      *reinterpret_cast<volatile int*>(P.tp_buf[P.tp_rank] + P.tp_counter_off) = tp_epoch;
    }
  }
}

// ---------------------------------------------------------------------------
// host side: plan + launch
// ---------------------------------------------------------------------------

static int nt_of_batch(int batch) { return batch <= 4 ? 1 : batch <= 8 ? 2 : batch <= 16 ? 4 : 8; }

// Dynamic shared memory budget of the GEMV kernel (stages + row-group
// mailbox); static shared memory (barriers, mailbox tags) comes on top.
constexpr int kSmemBudget = 216 * 1024;

// convert_once: convert the activations once per launch in the dense
// layouts (batch >= 3); the allocation-free entry keeps the in-kernel
// conversion, whose scratch needs no activation slices.
bool build_plan(const draco_gemv_problem* probs, int n, int batch, int n_sm, HostPlan& hp, char* msg, size_t ml,
                bool convert_once, const draco_gemv_input* inputs) {
  GemvParams& P = hp.P;
  memset(&P, 0, sizeof(P));
  P.n_prob = n;
  P.batch = batch;
  P.nt = batch <= 2 ? 1 : nt_of_batch(batch);
  const int NT = P.nt;
  P.xs_bytes = 8 * (8 * NT) * 32;  // 8 groups x 8*NT columns x 4 t x 8 B
  P.su_bytes = 8 * (4 * NT) * 16;  // 8 groups x 4*NT slots x float4
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
    d.accumulate = (q.flags & DRACO_GEMV_ACCUMULATE) != 0;
    d.ldx = q.ldx;
    d.ldy = q.ldy;
    d.qt = q.qtype;
    d.n_rows = (int)q.n_rows;
    d.k = (int)q.k;
    d.nb = (int)g.nb;
    d.n_rg = (int)g.n_rg;
    d.n_tiles = (int)g.n_tiles;
    d.cb = g.cb;
    d.slab0 = (int)slab0;
    d.in_mode = inputs ? inputs[p].mode : DRACO_INPUT_PLAIN;
    d.pidx = p;
    d.eps = inputs ? inputs[p].eps : 0.f;
    d.aux = inputs ? inputs[p].aux : nullptr;
    d.ldaux = inputs ? inputs[p].ldaux : 0;
    slab0 += g.n_rg * g.nb;
    w_stage = std::max(w_stage, kGroupTiles * g.cb);
  }
  if (slab0 > (int64_t)1 << 30) {
    snprintf(msg, ml, "gemv: problem set too large");
    return false;
  }
  int64_t off = align256(kWsCounters + kWsCountersBytes);
  P.part_off = off;
  off = align256(off + (int64_t)kMaxCta * 2 * kRowWarps * 32 * NT * 2 * 4);
  // activations converted once per launch by gemv_convert_kernel from batch
  // 2 on (that kernel also computes the RMSNorm row scales); at batch 1 the
  // converter warps convert in the kernel and compute the row scales there
  // too; the workspace always holds the slices and the scales, so one size
  // serves every input transform
  bool any_rms = false;
  for (int p = 0; p < n; ++p) any_rms |= P.prob[p].in_mode == DRACO_INPUT_RMSNORM;
  if (any_rms && !convert_once && batch >= 2) {
    snprintf(msg, ml, "gemv: RMSNorm inputs at batch 2 and above need the workspace entry point");
    return false;
  }
  P.precvt = (convert_once && batch >= 2) ? 1 : 0;
  P.rms_inkernel = (batch == 1 && any_rms) ? 1 : 0;
  for (int p = 0; p < n; ++p) {
    P.prob[p].xcv_off = -1;
    P.prob[p].rms_off = -1;
    if (convert_once) {
      P.prob[p].xcv_off = off;
      off = align256(off + (int64_t)P.prob[p].nb * (P.xs_bytes + P.su_bytes));
      P.prob[p].rms_off = off;
      off = align256(off + (int64_t)batch * 4);
    }
  }
  P.status_off = kWsStatus;
  P.cnt_off = kWsCounters;
  P.total_slabs = (int)slab0;
  P.w_stage = w_stage;
  P.stage_bytes = w_stage + P.xs_bytes + P.su_bytes;
  // mailbox: slots x 2 parities x row tiles x 32 lanes x 2 NT floats
  P.mbox_slots = std::max(1, std::min(kMaxMboxSlots, 4 / NT));
  const int mbox_bytes = P.mbox_slots * 2 * kRowWarps * 32 * 2 * NT * 4;
  P.n_stages = std::min(kMaxStages, (kSmemBudget - mbox_bytes) / P.stage_bytes);
  if (P.n_stages < 2) {
    snprintf(msg, ml, "gemv: stage of %d bytes does not fit shared memory twice", P.stage_bytes);
    return false;
  }
  P.mbox_off = P.n_stages * P.stage_bytes;
  hp.smem_bytes = (size_t)P.mbox_off + mbox_bytes;
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
  // A CTA needs no more stages than it has slabs.  The smaller footprint lets
  // the next kernel's CTAs (programmatic launch) share the SM and stream
  // their weights while this one drains.
  int max_run = 0;
  for (int c2 = 0; c2 < n_cta; ++c2) max_run = std::max(max_run, P.cta_start[c2 + 1] - P.cta_start[c2]);
  if (max_run < P.n_stages) {
    P.n_stages = std::max(2, max_run);
    P.mbox_off = P.n_stages * P.stage_bytes;
    hp.smem_bytes = (size_t)P.mbox_off + mbox_bytes;
  }
  return true;
}

size_t gemv_workspace_bytes(const draco_gemv_problem* probs, int n, int batch) {
  HostPlan local;
  char msg[128];
  if (!build_plan(probs, n, batch, kMaxCta, local, msg, sizeof(msg))) return 0;
  // one size serves both kernels (the tensor-memory one may take the launch)
  return std::max(local.ws_needed, gemv_tc_workspace_bytes(probs, n, batch, nullptr));
}

int gemv_launch_count(const draco_gemv_problem* probs, int n, int batch) {
  HostPlan hp;
  char msg[128];
  if (!build_plan(probs, n, batch, device_sm_count(), hp, msg, sizeof(msg))) return -1;
  if (hp.P.total_slabs == 0) return 0;
  if (gemv_tc_eligible(probs, n, batch)) return gemv_tc_split_count(hp) > 0 ? 3 : 2;
  return hp.P.precvt ? 2 : 1;
}

template <int G, int NT, bool TP>
static cudaError_t launch_gemv(const HostPlan& hp, cudaStream_t st) {
  static int attr_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemv_kernel<G, NT, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    if (e != cudaSuccess) return e;
    attr_set[dev] = 1;
  }
  const GemvParams& P = hp.P;
  // programmatic dependent launch: the kernel may start before its
  // predecessor in the stream finishes; it streams weights at once and waits
  // (griddepcontrol.wait) before reading x or writing y
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P.n_cta);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = hp.smem_bytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<G, NT, TP>, P);
}

template <bool TP>
static cudaError_t dispatch_gemv(const HostPlan& hp, int batch, cudaStream_t st) {
  if (batch == 1) return launch_gemv<4, 1, TP>(hp, st);
  if (batch == 2) return launch_gemv<2, 1, TP>(hp, st);
  switch (hp.P.nt) {
    case 1: return launch_gemv<1, 1, TP>(hp, st);
    case 2: return launch_gemv<1, 2, TP>(hp, st);
    case 4: return launch_gemv<1, 4, TP>(hp, st);
    default: return launch_gemv<1, 8, TP>(hp, st);
  }
}

// Fill the tensor-parallel fields of a plan from the exchange description.
static int set_tp(HostPlan& hp, const draco_gemv_problem* probs, int n, const draco_tp_exchange* ex, char* msg,
                  size_t ml) {
  GemvParams& P = hp.P;
  if (ex->world < 2 || ex->world > DRACO_TP_MAX_WORLD || ex->rank < 0 || ex->rank >= ex->world) {
    snprintf(msg, ml, "gemv_tp: world %d / rank %d outside 2..%d", ex->world, ex->rank, DRACO_TP_MAX_WORLD);
    return DRACO_ERR_ARG;
  }
  for (int q = 0; q < ex->world; ++q) {
    if (ex->buffers[q] == nullptr || (reinterpret_cast<uintptr_t>(ex->buffers[q]) & 255) != 0) {
      snprintf(msg, ml, "gemv_tp: exchange buffer of rank %d is null or not 256-byte aligned", q);
      return DRACO_ERR_ALIGN;
    }
    P.tp_buf[q] = static_cast<uint8_t*>(ex->buffers[q]);
  }
  if (ex->flags_off < 0 || (ex->flags_off & 3) || ex->counter_off < 0 || (ex->counter_off & 3)) {
    snprintf(msg, ml, "gemv_tp: flag / counter offsets must be non-negative multiples of 4");
    return DRACO_ERR_ALIGN;
  }
  for (int i = 0; i < n; ++i) {
    if (ex->y_off[i] < 0 || (ex->y_off[i] & 3) || ex->parity_stride[i] < 0 || (ex->parity_stride[i] & 3)) {
      snprintf(msg, ml, "gemv_tp: problem %d output offsets must be non-negative multiples of 4", i);
      return DRACO_ERR_ALIGN;
    }
    P.prob[i].tp_y_off = ex->y_off[i];
    P.prob[i].tp_par_stride = ex->parity_stride[i];
    (void)probs;
  }
  P.tp_world = ex->world;
  P.tp_rank = ex->rank;
  P.tp_flags_off = ex->flags_off;
  P.tp_counter_off = ex->counter_off;
  return DRACO_OK;
}

static int gemv_launch_impl(const draco_gemv_problem* probs, int n, int batch, const draco_tp_exchange* ex, void* ws,
                            size_t ws_bytes, cudaStream_t st, char* msg, size_t ml,
                            const draco_gemv_input* inputs = nullptr) {
  HostPlan hp;
  const int n_sm = device_sm_count();
  if (!build_plan(probs, n, batch, n_sm, hp, msg, ml, true, inputs)) return DRACO_ERR_ARG;
  if (ex) {
    const int rc = set_tp(hp, probs, n, ex, msg, ml);
    if (rc != DRACO_OK) return rc;
  }
  // (a tensor-parallel step with no slabs would never signal its peers)
  if (hp.P.total_slabs == 0) {
    if (!ex) return DRACO_OK;
    snprintf(msg, ml, "gemv_tp: the problems hold no weights");
    return DRACO_ERR_SHAPE;
  }
  // the plan's workspace size does not depend on the SM count
  if (ws == nullptr || ws_bytes < hp.ws_needed) {
    snprintf(msg, ml, "gemv: workspace of %zu bytes given, %zu needed", ws_bytes, hp.ws_needed);
    return DRACO_ERR_WORKSPACE;
  }
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) {
    snprintf(msg, ml, "gemv: workspace must be 256-byte aligned");
    return DRACO_ERR_ALIGN;
  }
  // batches of 17 and more over K-quants: the tensor-memory kernel
  if (!ex && gemv_tc_eligible(probs, n, batch)) return gemv_tc_launch(hp, inputs, ws, ws_bytes, st, msg, ml);
  hp.P.ws = static_cast<uint8_t*>(ws);
  if (hp.P.precvt) {
    int units = 0;
    for (int p = 0; p < n; ++p) units += hp.P.prob[p].nb + (hp.P.prob[p].in_mode == DRACO_INPUT_RMSNORM ? batch : 0);
    const int blocks = (units + kConvertWarpsPerBlock - 1) / kConvertWarpsPerBlock;
    const dim3 grid(blocks), block(kConvertWarpsPerBlock * 32);
    if (hp.P.nt == 1) gemv_convert_kernel<1><<<grid, block, 0, st>>>(hp.P);
    else if (hp.P.nt == 2) gemv_convert_kernel<2><<<grid, block, 0, st>>>(hp.P);
    else if (hp.P.nt == 4) gemv_convert_kernel<4><<<grid, block, 0, st>>>(hp.P);
    else gemv_convert_kernel<8><<<grid, block, 0, st>>>(hp.P);
    const cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) {
      snprintf(msg, ml, "gemv: activation conversion launch failed: %s", cudaGetErrorString(ce));
      return DRACO_ERR_CUDA;
    }
  }
  cudaError_t e;
  e = ex ? dispatch_gemv<true>(hp, batch, st) : dispatch_gemv<false>(hp, batch, st);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemv: launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

int gemv_launch(const draco_gemv_problem* probs, int n, int batch, void* ws, size_t ws_bytes, cudaStream_t st,
                char* msg, size_t ml, const draco_gemv_input* inputs) {
  return gemv_launch_impl(probs, n, batch, nullptr, ws, ws_bytes, st, msg, ml, inputs);
}

int gemv_launch_tp(const draco_gemv_problem* probs, int n, int batch, const draco_tp_exchange* ex, void* ws,
                   size_t ws_bytes, cudaStream_t st, char* msg, size_t ml) {
  return gemv_launch_impl(probs, n, batch, ex, ws, ws_bytes, st, msg, ml);
}

// ---------------------------------------------------------------------------
// Allocation-free entry: the scratch (status word, arrival counters, partial
// sums) lives in a fixed file-scope device array instead of a caller-supplied
// workspace.  Every GPU that loads the library holds this array until the
// process exits.  All calls share it, so calls that overlap on the GPU race.
// ---------------------------------------------------------------------------
constexpr size_t kStaticScratchBytes = (size_t)1 << 20;  // 1 MiB: enough for batch <= 4
static __device__ __align__(256) uint8_t g_gemv_static_scratch[kStaticScratchBytes];

size_t gemv_static_scratch_bytes() { return kStaticScratchBytes; }

// Device address of the array on the current device, looked up once per
// device (host code may not use the symbol itself as a pointer).
static int static_scratch_address(uint8_t** out, char* msg, size_t ml) {
  static uint8_t* cache[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemv_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) {
    snprintf(msg, ml, "gemv_noalloc: device index %d out of range", dev);
    return DRACO_ERR_ARG;
  }
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gemv_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      snprintf(msg, ml, "gemv_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return DRACO_ERR_CUDA;
    }
    cache[dev] = static_cast<uint8_t*>(p);
  }
  *out = cache[dev];
  return DRACO_OK;
}

int gemv_launch_noalloc(const draco_gemv_problem* probs, int n, int batch, cudaStream_t st, char* msg,
                        size_t ml) {
  HostPlan hp;
  const int n_sm = device_sm_count();
  if (!build_plan(probs, n, batch, n_sm, hp, msg, ml, /*convert_once=*/false)) return DRACO_ERR_ARG;
  if (hp.P.total_slabs == 0) return DRACO_OK;
  if (hp.ws_needed > kStaticScratchBytes) {
    snprintf(msg, ml,
             "gemv_noalloc: this call needs %zu bytes of scratch but the fixed array holds %zu "
             "(batch <= 4 fits); use draco_gguf_gemv_grouped with a workspace",
             hp.ws_needed, kStaticScratchBytes);
    return DRACO_ERR_WORKSPACE;
  }
  uint8_t* scratch = nullptr;
  int rc = static_scratch_address(&scratch, msg, ml);
  if (rc != DRACO_OK) return rc;
  // the status word and arrival counters must start at zero; a call that
  // failed on the device may have left them set
  cudaError_t e = cudaMemsetAsync(scratch, 0, (size_t)(kWsCounters + kWsCountersBytes), st);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemv_noalloc: clearing the scratch counters failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  hp.P.ws = scratch;
  if (batch == 1) e = launch_gemv<4, 1, false>(hp, st);
  else if (batch == 2) e = launch_gemv<2, 1, false>(hp, st);
  else e = launch_gemv<1, 1, false>(hp, st);  // 3 <= batch <= 4 (larger batches exceed the array)
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemv_noalloc: launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

// Status word of the last allocation-free call on the current device: the
// first int32 of the fixed array (0, or the DRACO_* code a device-side wait
// recorded).  Copied on `st` after the work queued there, into host memory
// owned by the caller; the host waits for the stream.  No allocation.
int gemv_noalloc_status(int* out, cudaStream_t st, char* msg, size_t ml) {
  uint8_t* scratch = nullptr;
  int rc = static_scratch_address(&scratch, msg, ml);
  if (rc != DRACO_OK) return rc;
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, scratch + kWsStatus, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemv_noalloc_status: reading the status word failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  *out = v;
  return DRACO_OK;
}

}  // namespace draco
