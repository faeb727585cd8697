// gemv_tc.cu — decode GEMV y[B, N] = x[B, K] . dequant(W)^T for batches of
// 17..32 rows on the 5th-generation tensor cores (tcgen05, fp32
// accumulators in tensor memory), over TILED Q4_K / Q5_K / Q6_K weights.
//
// Replaces the same reference call as gemv.cu (executor._linear,
// draco/runtime/cpu/executor.py:47-79 -> GenericGemmKernel.matmul_f32,
// draco/runtime/cpu/kernels/generic.py:32-33, on gguf._dequantize's fp32
// weights, draco/format/gguf.py:425-495) when the batch is large enough that
// the warp-MMA kernel's per-sub-block fp32 epilogue, which grows with the
// batch, becomes the limit.
//
// Arithmetic.  A super-block row of a K-quant is
//   Q4_K / Q5_K:  w_k = d * (sc_j * q_k) - dmin * m_j      (gguf.py:425-468)
//   Q6_K:         w_k = d * (sc_j * (q_k - 32))              (gguf.py:470-495)
// The integer sc_j * q_k (at most 63 * 31) is exact in fp16 and becomes the
// MMA's A operand, so the sub-block scales ride inside the tensor-core product
// and only d, dmin and the activation scale are applied in fp32, once per
// super-block:
//   y[n, b] += u_b * (d_n * ACC[n, b] - dmin_n * ACC2[n, b])
//   ACC  = sum_k A[n, k] * X[b, k]          (K = 256, fp16 x fp16 -> fp32)
//   ACC2 = sum_j m[n, j] * (S_hi + S_lo)[b, j]   (one K = 16 MMA)
// with X = fp16(x / u_b), u_b a power of two per (batch row, super-block)
// (max |x| / u_b in [1/2, 1)), and S[b, j] the sub-block sums of X split
// into two fp16 parts.  Taking the sums over the rounded X makes the result
// W . X exactly up to fp32 accumulation: Q4_K's product and min terms nearly
// cancel, and sums of the unrounded x would leave the rounding of X
// uncancelled in the difference (about 3x the error).  Q6_K's sc_j * (q_k - 32) may need 13 bits; it is
// rounded to fp16 (relative error <= 2^-12 on those weights), and Q6_K has no
// ACC2.  fp16 activations carry 11 significant bits: the outputs stay within
// ~2e-4 relative L2 of the float64 oracle for Gaussian activations.
//
// Design (one persistent CTA per SM, 14 warps):
//  * warp 0, one lane (producer): for each slab (128 rows x 256 k) of the
//    CTA's stream-K range, a 1-D bulk copy of the packed slab and of the
//    super-block's converted activation tile (written by gemv_tc_convert in
//    the shared-memory image of the MMA's B operand) into a stage ring; the
//    first stages' weights are requested before the preceding kernel has
//    finished (programmatic dependent launch), activations only after.
//  * warps 6-13 (dequant): warp 6 + c expands row tile c (16 rows) of each
//    64-k block into fp16 A tiles (128 x 64, K-major, 128-byte swizzle), two
//    k-blocks per slot of a 2-slot ring, plus, per Q4_K / Q5_K super-block,
//    the rows' 6-bit mins (a K = 16 tile) and the rows' d / dmin for the
//    epilogue.
//  * warp 1: allocates the tensor memory; one lane issues
//    tcgen05.mma.cta_group::1.kind::f16 (M = 128 rows, N = 16 or 32 batch
//    rows, K = 16) into one of kTcAcc accumulator pairs (super-block index
//    mod kTcAcc) and
//    commits to the barriers that free A slots, stages and accumulators.
//  * warps 2-5 (epilogue): thread = weight row = TMEM lane (warp % 4 selects
//    the lane quarter); per super-block
//    tcgen05.ld of ACC (and ACC2), y[b] += ..., kept in registers until the
//    row group ends in this CTA's range; whole row groups are written
//    directly, split ones as partials in the workspace, which a small
//    follow-up kernel (gemv_tc_fixup, one CTA per split row group) adds in
//    CTA order: deterministic, and no fence or atomic in the pipeline.
//  * every wait is bounded (2 s); on a timeout the kernel records
//    DRACO_ERR_TIMEOUT in the workspace status word, the other roles see the
//    CTA's abort word, the producer waits for its copies to land, the MMA
//    lane for its MMAs to complete, and the tensor memory is freed.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "gemv_plan.h"
#include "internal.h"

namespace draco {

constexpr int kTcWarps = 14;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcEpi0 = 2;   // warps 2-5: epilogue (warp % 4 selects its TMEM lanes)
constexpr int kTcDeq0 = 6;   // warps 6-13: dequant, one per row tile
constexpr int kTcASlots = 2;
constexpr int kTcKbTile = 128 * 64 * 2;  // one fp16 k-block of A: 128 rows x 64 k
constexpr int kTcATile = 2 * kTcKbTile;  // an A slot: two k-blocks
constexpr int kTcMaxStages = 4;
// From batch 17 the warp-MMA kernel pads to 32 rows (its slowest form); there
// this kernel is faster (117 vs 125 us for the config-2 layer set at batch 32
// on one B200), below it the warp-MMA kernel is (70 vs 90 us at batch 16).
constexpr int kTcMinBatchDefault = 17;
constexpr int kTcSmemBudget = 216 * 1024;
constexpr int kTcAcc = 4;  // accumulator sets (ACC, ACC2, d / dmin, u, mins) in flight

struct TcProb {
  const uint8_t* w;
  const float* x;
  float* y;
  const float* bias;
  const float* aux;
  int64_t ldx, ldy, ldaux;
  int64_t bt_off;   // workspace offset of the converted activation tiles, one per super-block
  int64_t rms_off;  // RMSNORM: workspace offset of the per-row scales [batch]
  int qt, n_rows, k, nb, n_rg, n_tiles, cb, slab0, in_mode;
  int accumulate;  // y += result
  float eps;
};

struct TcParams {
  TcProb prob[DRACO_GEMV_MAX_PROBLEMS];
  uint8_t* ws;
  int64_t part_off;
  int n_prob, batch, np, n_cta, total_slabs;
  int ns, raw_bytes, bt_bytes, stage_bytes, a_off, m_off;
  int n_split;  // row groups split between CTAs, summed by gemv_tc_fixup
  int cta_start[kMaxCta + 1];
  struct Split {
    int p, rg, c_first, c_last;
  } split[kMaxCta];
};

// bytes of one converted activation tile: 4 k-blocks of np rows x 128 B,
// the sub-block sums (np rows x 128 B), u (np floats)
__host__ __device__ inline int tc_bt_bytes(int np) { return (5 * np * 128 + np * 4 + 1023) & ~1023; }

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_error(const TcParams& P, int code) {
  atomicCAS(reinterpret_cast<int*>(P.ws + kWsStatus), 0, code);
}
// bounded wait on a barrier phase; false when the CTA aborted or the wait ran
// out (this thread then records the timeout and raises the abort word)
__device__ __forceinline__ bool tc_wait(const TcParams& P, uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      tc_error(P, DRACO_ERR_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// K-major operand descriptor with the 128-byte swizzle (8-row groups 1024 B
// apart: stride byte offset 1024; leading byte offset unused; version 1 for
// sm_100; layout 2 = SWIZZLE_128B), as (low word, high word): the low word is
// (address >> 4) | LBO field, so an operand `delta` bytes further on is the
// low word + delta / 16 (shared-memory addresses stay far below 2^20).
constexpr uint32_t kSw128DescHi = (uint32_t)(1024 >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t tc_desc_lo(uint32_t saddr) { return ((saddr & 0x3FFFFu) >> 4) | 0x10000u; }
__device__ __forceinline__ uint64_t tc_desc(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }
// kind::f16 instruction descriptor: fp16 A and B (format 0), fp32 D, K-major
__host__ __device__ constexpr uint32_t tc_idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier once every MMA this thread issued so far has completed
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
template <int N>
__device__ __forceinline__ void tc_ld(uint32_t taddr, float (&v)[N]);
template <>
__device__ __forceinline__ void tc_ld<8>(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tc_ld<16>(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void tc_ld<32>(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// fp16 A tiles.  The MMA sums over k, so A and B may list the 64 k of a block
// in any common order.  Both use: 16-byte column chunk c = 2t + h of a row
// holds k = 16h + 4t + (0..3) (its low 8 bytes) and k = 32 + 16h + 4t + (0..3)
// (its high 8 bytes).  A Q4_K / Q5_K lane word (hi, h) then fills one chunk:
// its low nibbles are the first four, its high nibbles the last four values.
// Chunk c of row 8hi + g of a warp's 16-row tile lands at the 128-byte-
// swizzled position c ^ g.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_chunk(uint8_t* tw, int hi, int g, int c, uint4 v) {
  *reinterpret_cast<uint4*>(tw + hi * 1024 + g * 128 + ((c ^ g) << 4)) = v;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// bytes (0,1) / (2,3) of w (each < 1024) as the fp16 pair 1024 + byte
__device__ __forceinline__ uint32_t h2_bytes01(uint32_t w) { return __byte_perm(w, 0x64646464u, 0x5140u); }
__device__ __forceinline__ uint32_t h2_bytes23(uint32_t w) { return __byte_perm(w, 0x64646464u, 0x5342u); }
constexpr uint32_t kH1024 = 0x64006400u;  // fp16 pair (1024, 1024)
// fp16 pairs (s0, s0) and (s1, s1) of the bytes 0 and 1 of v (each < 1024), exactly
__device__ __forceinline__ void h2_splats(uint32_t v, uint32_t& s0, uint32_t& s1) {
  const uint32_t pair = h2_sub(h2_bytes01(v), kH1024);  // (byte 0, byte 1)
  s0 = __byte_perm(pair, 0u, 0x1010u);
  s1 = __byte_perm(pair, 0u, 0x3232u);
}
// 4 quants q (bytes of w, < 32) times the scale pair sc2 = (s, s): exact
// s * q, via fma((1024 + q), s, -1024 s) whose exact result fits fp16
__device__ __forceinline__ uint2 tc_scaled4(uint32_t w, uint32_t sc2, uint32_t nsc2) {
  return make_uint2(h2_fma(h2_bytes01(w), sc2, nsc2), h2_fma(h2_bytes23(w), sc2, nsc2));
}

// Q4_K / Q5_K, 64-k block q = sub-blocks 2q (low nibbles) and 2q+1 (high
// nibbles) of rows g (hi 0) and g+8 (hi 1) of the chunk at ch.  S[hi] = the
// row's 12 scale bytes as three words (gguf.py:436-442); the qs unit word
// (hi, h) holds bytes 16h+4t..+3 of the sub-block pair; Q5_K's qh unit
// mirrors it word for word, the fifth bit of a quant of sub-block b at bit b
// of its byte (gguf.py:457-467).
template <bool K5>
__device__ __forceinline__ void tc_deq_q4k(const uint8_t* ch, int q, int lane, const uint32_t (&S)[2][3],
                                           const uint4& H, uint8_t* tw) {
  const int g = lane >> 2, t = lane & 3;
  const uint4 U = *reinterpret_cast<const uint4*>(ch + 512 * q + 16 * lane);
#pragma unroll
  for (int hi = 0; hi < 2; ++hi) {
    const uint32_t A = S[hi][0], C = S[hi][2];
    uint32_t scp;  // 6-bit scales of sub-blocks 2q (byte 0) and 2q+1 (byte 1)
    if (q < 2) {
      scp = (A >> (16 * q)) & 0x3F3Fu;
    } else {
      const int s = 16 * (q - 2);
      scp = ((C >> s) & 0x0F0Fu) | (((A >> s) >> 2) & 0x3030u);
    }
    uint32_t s_lo, s_hi;
    h2_splats(scp, s_lo, s_hi);
    const uint32_t n_lo = h2_mul(s_lo, 0xE400E400u), n_hi = h2_mul(s_hi, 0xE400E400u);  // -1024 s
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w = hi ? (h ? U.w : U.z) : (h ? U.y : U.x);
      uint32_t lo = w & 0x0F0F0F0Fu, up = (w >> 4) & 0x0F0F0F0Fu;
      if (K5) {
        const uint32_t hw = hi ? (h ? H.w : H.z) : (h ? H.y : H.x);
        const int b0 = 2 * q, b1 = 2 * q + 1;
        lo |= (b0 <= 4 ? (hw << (4 - b0)) : (hw >> (b0 - 4))) & 0x10101010u;
        up |= (b1 <= 4 ? (hw << (4 - b1)) : (hw >> (b1 - 4))) & 0x10101010u;
      }
      const uint2 a = tc_scaled4(lo, s_lo, n_lo), b = tc_scaled4(up, s_hi, n_hi);
      tc_chunk(tw, hi, g, 2 * t + h, make_uint4(a.x, a.y, b.x, b.y));
    }
  }
}

// Q6_K, 64-k block q = groups i = 2(q&1) + ii (ii = 0, 1) of half n = q/2;
// lane words 6is + 3hi + {0: ql l, 1: ql l+32, 2: qh} of units 3n..3n+2;
// int8 scales of row g / g+8 at byte is + 2ii of the word (gguf.py:470-495).
// Group ii covers k = 32ii + 16is + 4t + (0..3): chunk 2t + is holds ii = 0
// then ii = 1.  sc * (q6 - 32) is rounded to fp16 once.
__device__ __forceinline__ void tc_deq_q6k(const uint8_t* ch, int q, int lane, uint8_t* tw) {
  const int g = lane >> 2, t = lane & 3;
  const int n = q >> 1, odd = q & 1;
  const uint4 P0 = *reinterpret_cast<const uint4*>(ch + 512 * (3 * n) + 16 * lane);
  const uint4 P1 = *reinterpret_cast<const uint4*>(ch + 512 * (3 * n + 1) + 16 * lane);
  const uint4 P2 = *reinterpret_cast<const uint4*>(ch + 512 * (3 * n + 2) + 16 * lane);
  const uint32_t W[12] = {P0.x, P0.y, P0.z, P0.w, P1.x, P1.y, P1.z, P1.w, P2.x, P2.y, P2.z, P2.w};
#pragma unroll
  for (int hi = 0; hi < 2; ++hi) {
    const uint32_t scw = *reinterpret_cast<const uint32_t*>(ch + 3072 + 32 * g + 16 * hi + 8 * n + 4 * odd) ^ 0x80808080u;
    const uint32_t s01 = h2_sub(h2_bytes01(scw), 0x64806480u);  // (sc[is 0, ii 0], sc[is 1, ii 0]); 1152 = 1024 + 128
    const uint32_t s23 = h2_sub(h2_bytes23(scw), 0x64806480u);  // (sc[is 0, ii 1], sc[is 1, ii 1])
#pragma unroll
    for (int is = 0; is < 2; ++is) {
      const uint32_t qh = W[6 * is + 3 * hi + 2];
      uint2 v[2];
#pragma unroll
      for (int ii = 0; ii < 2; ++ii) {
        const uint32_t sw = ii ? s23 : s01;
        const uint32_t sc2 = is ? __byte_perm(sw, 0u, 0x3232u) : __byte_perm(sw, 0u, 0x1010u);
        const uint32_t ql = W[6 * is + 3 * hi + ii];
        const uint32_t lo = (ql >> (4 * odd)) & 0x0F0F0F0Fu;
        const uint32_t hb = (qh >> (2 * (2 * odd + ii))) & 0x03030303u;
        const uint32_t q6 = lo | (hb << 4);
        v[ii] = make_uint2(h2_mul(h2_sub(h2_bytes01(q6), 0x64206420u), sc2),  // (q6 - 32) * sc, 1056 = 1024 + 32
                           h2_mul(h2_sub(h2_bytes23(q6), 0x64206420u), sc2));
      }
      tc_chunk(tw, hi, g, 2 * t + is, make_uint4(v[0].x, v[0].y, v[1].x, v[1].y));
    }
  }
}

// Q4_K / Q5_K mins tile (K = 16, no swizzle: 8-row core matrices of 8 rows x
// 16 bytes, row groups 256 B apart, the two K halves 128 B apart): columns
// 0-7 and 8-15 of a row both hold m_0..m_7 (the row's 6-bit mins,
// gguf.py:436-442), for the hi and lo parts of the sub-block sums.  Lane
// (g, t) writes row 8(2c + hi) + g (hi = t >> 1), K half t & 1.
constexpr int kTcMinsBytes = 128 * 16 * 2;
__device__ __forceinline__ void tc_mins(const uint32_t (&S)[2][3], int lane, int c, uint8_t* mt) {
  const int g = lane >> 2, t = lane & 3, hi = t >> 1;
  const uint32_t B = hi ? S[1][1] : S[0][1], C = hi ? S[1][2] : S[0][2];  // selects: S stays in registers
  const uint32_t m03 = B & 0x3F3F3F3Fu;
  const uint32_t m47 = ((C >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u);
  const uint4 v = make_uint4(h2_sub(h2_bytes01(m03), kH1024), h2_sub(h2_bytes23(m03), kH1024),
                             h2_sub(h2_bytes01(m47), kH1024), h2_sub(h2_bytes23(m47), kH1024));
  *reinterpret_cast<uint4*>(mt + (2 * c + hi) * 256 + (t & 1) * 128 + g * 16) = v;
}
// K-major operand without swizzle (the mins tile)
__device__ __forceinline__ uint64_t tc_sdesc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;  // leading byte offset: between the K core matrices
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;  // stride byte offset: between 8-row groups
  d |= (uint64_t)1 << 46;                      // descriptor version (sm_100); layout 0 = no swizzle
  return d;
}

// position in the ring of A slots and the parity of its current phase
struct TcRing {
  int a = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next() {
    if (++a == kTcASlots) {
      a = 0;
      ph ^= 1u;
    }
  }
};

// One slab (one super-block of a row group) by dequant warp c: the d / dmin
// of its rows for the epilogue, the mins tile (Q4_K / Q5_K, with the first
// slot) and the four fp16 k-blocks, two per A slot.  False when the CTA aborted.
template <int QT>
__device__ __forceinline__ bool tc_dequant_slab(const TcParams& P, uint8_t* smem, const uint8_t* ch, bool live,
                                                int c, int lane, uint64_t* acce_p, uint32_t sph, uint64_t* ddf_p,
                                                float2* dd_row, uint8_t* mt, uint64_t* aful, uint64_t* aemp,
                                                TcRing& ring, volatile int* abort) {
  constexpr bool kMins = QT != kQ6_K, kK5 = QT == kQ5_K;
  const int g = lane >> 2, t = lane & 3;
  uint32_t S[2][3] = {{0u, 0u, 0u}, {0u, 0u, 0u}};
  uint4 H = make_uint4(0u, 0u, 0u, 0u);
  if (kMins && live) {
    const uint8_t* sp = ch + (kK5 ? 2560 : 2048) + 24 * g;  // row g: 12 bytes, row g + 8: the next 12
#pragma unroll
    for (int hi = 0; hi < 2; ++hi)
#pragma unroll
      for (int w = 0; w < 3; ++w) S[hi][w] = *reinterpret_cast<const uint32_t*>(sp + 12 * hi + 4 * w);
    if (kK5) H = *reinterpret_cast<const uint4*>(ch + 2048 + 16 * lane);
  }
  // d and dmin of rows g (t = 0) and g + 8 (t = 1) for the epilogue, once it
  // is done with this set's previous super-block (which also frees the
  // set's mins tile)
  if (!__all_sync(0xffffffffu, tc_wait(P, acce_p, sph ^ 1u, abort))) return false;
  if (t < 2) {
    float2 dd = make_float2(0.f, 0.f);
    if (live) {
      if (kMins) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(ch + (kK5 ? 2752 : 2240) + 8 * g + 4 * t);
        dd = make_float2(f16_bits_to_f32(w), f16_bits_to_f32(w >> 16));
      } else {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(ch + 3328 + 4 * g);
        dd = make_float2(f16_bits_to_f32(t ? (w >> 16) : w), 0.f);
      }
    }
    dd_row[16 * c + g + 8 * t] = dd;
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(ddf_p);
#pragma unroll
  for (int sl = 0; sl < 2; ++sl) {
    if (!__all_sync(0xffffffffu, tc_wait(P, &aemp[ring.a], ring.ph ^ 1u, abort))) return false;
    uint8_t* tw = smem + P.a_off + (size_t)ring.a * kTcATile + (size_t)c * 2048;
    if (live) {
      if (kMins && sl == 0) tc_mins(S, lane, c, mt);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        if (QT == kQ6_K) tc_deq_q6k(ch, 2 * sl + kk, lane, tw + kk * kTcKbTile);
        else tc_deq_q4k<kK5>(ch, 2 * sl + kk, lane, S, H, tw + kk * kTcKbTile);
      }
    }
    tc_fence_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&aful[ring.a]);
    ring.next();
  }
  return true;
}

// (problem, row group, super-block) of a global slab index, advanced in order
struct TcCursor {
  int p, rg, j;
  __device__ void seek(const TcParams& P, int s) {
    p = 0;
    for (int q = 1; q < P.n_prob; ++q)
      if (s >= P.prob[q].slab0) p = q;
    const int local = s - P.prob[p].slab0;
    rg = local / P.prob[p].nb;
    j = local - rg * P.prob[p].nb;
  }
  __device__ void next(const TcParams& P) {
    if (++j == P.prob[p].nb) {
      j = 0;
      if (++rg == P.prob[p].n_rg) {
        rg = 0;
        ++p;
      }
    }
  }
};

// the outputs of one weight row (bias, RMSNorm row scale)
template <int NP>
__device__ __forceinline__ void tc_write_row(const TcParams& P, const TcProb& pr, int64_t row, const float (&y)[NP]) {
  if (row >= pr.n_rows) return;
  const float bias = pr.bias ? pr.bias[row] : 0.f;
  const float* rms = reinterpret_cast<const float*>(P.ws + pr.rms_off);
#pragma unroll
  for (int b = 0; b < NP; ++b) {
    if (b < P.batch) {
      float out = y[b];
      if (pr.in_mode == DRACO_INPUT_RMSNORM) out *= __ldcg(rms + b);
      out += bias;
      if (pr.accumulate) out += pr.y[(int64_t)b * pr.ldy + row];
      pr.y[(int64_t)b * pr.ldy + row] = out;
    }
  }
}

// End of a row group's segment in this CTA's range, by epilogue warp e (rows
// 32e..32e+31).  Whole row groups are written; a split one is stored as this
// CTA's partial, which gemv_tc_fixup adds to the others in CTA order.
template <int NP>
__device__ __forceinline__ void tc_flush(const TcParams& P, const TcProb& pr, int rg, int s_begin, int s_end, int e,
                                         int lane, const float (&y)[NP]) {
  const int r = 32 * e + lane;
  const int rg_start = pr.slab0 + rg * pr.nb, rg_end = rg_start + pr.nb;
  if (s_begin <= rg_start && rg_end <= s_end) {
    tc_write_row<NP>(P, pr, (int64_t)rg * 128 + r, y);
    return;
  }
  const int cslot = (s_begin >= rg_start) ? 0 : 1;
  float* part = reinterpret_cast<float*>(P.ws + P.part_off) + (((int64_t)blockIdx.x * 2 + cslot) * 128 + r) * NP;
#pragma unroll
  for (int b = 0; b < NP; b += 4) __stcg(reinterpret_cast<float4*>(part + b), make_float4(y[b], y[b + 1], y[b + 2], y[b + 3]));
}

// Split row groups: one CTA (thread = row) per row group adds the partials of
// its CTAs in CTA order (deterministic) once the GEMV has completed.
template <int NP>
__global__ void __launch_bounds__(128) gemv_tc_fixup(const __grid_constant__ TcParams P) {
  grid_dependency_wait();  // the partials of the GEMV launched before
  grid_launch_dependents();
  const TcParams::Split& sp = P.split[blockIdx.x];
  const TcProb& pr = P.prob[sp.p];
  const int r = threadIdx.x;
  const int rg_start = pr.slab0 + sp.rg * pr.nb;
  float sum[NP];
#pragma unroll
  for (int b = 0; b < NP; ++b) sum[b] = 0.f;
  for (int c = sp.c_first; c <= sp.c_last; ++c) {
    const int sl = (P.cta_start[c] >= rg_start) ? 0 : 1;
    const float* q = reinterpret_cast<const float*>(P.ws + P.part_off) + (((int64_t)c * 2 + sl) * 128 + r) * NP;
#pragma unroll
    for (int b = 0; b < NP; b += 4) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(q + b));
      sum[b] += v.x, sum[b + 1] += v.y, sum[b + 2] += v.z, sum[b + 3] += v.w;
    }
  }
  tc_write_row<NP>(P, pr, (int64_t)sp.rg * 128 + r, sum);
}

template <int NP>
__global__ void __launch_bounds__(kTcThreads, 1) gemv_tc_kernel(const __grid_constant__ TcParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kTcMaxStages], empty[kTcMaxStages];
  __shared__ __align__(8) uint64_t aful[kTcASlots], aemp[kTcASlots];
  __shared__ __align__(8) uint64_t accf[kTcAcc], acce[kTcAcc], ddf[kTcAcc], mma_done;
  __shared__ __align__(16) float2 dd_buf[kTcAcc][128];
  __shared__ __align__(16) float u_buf[kTcAcc][NP];
  __shared__ uint32_t s_tmem;
  __shared__ int abort_word;
  volatile int* abort = &abort_word;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s_begin = P.cta_start[blockIdx.x], s_end = P.cta_start[blockIdx.x + 1];
  const int n = s_end - s_begin;
  const int NS = P.ns;

  if (threadIdx.x == 0) {
    abort_word = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);                // producer (expect_tx) + the copies' bytes
      mbar_init(&empty[i], kRowWarps + 1);   // dequant warps + the MMA commit
    }
    for (int i = 0; i < kTcASlots; ++i) {
      mbar_init(&aful[i], kRowWarps);
      mbar_init(&aemp[i], 1);
    }
    for (int i = 0; i < kTcAcc; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 4);                // epilogue warps
      mbar_init(&ddf[i], kRowWarps + 1);     // dequant warps (d, dmin) + the MMA lane (u)
    }
    mbar_init(&mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  grid_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int last_round[kTcMaxStages];
      for (int i = 0; i < NS; ++i) last_round[i] = -1;
      TcCursor c;
      c.seek(P, s_begin);
      auto slab_src = [&](const TcCursor& cc, uint32_t& bytes) {
        const TcProb& pr = P.prob[cc.p];
        const TiledGeom geo = tiled_geom(pr.qt, pr.n_rows, pr.k);
        bytes = (uint32_t)(rg_tiles(geo, cc.rg) * pr.cb);
        return pr.w + slab_offset(geo, cc.rg, cc.j);
      };
      // weights of the first stages before the preceding kernel completes
      const int pre = n < NS ? n : NS;
      TcCursor c0 = c;
      for (int i = 0; i < pre; ++i, c0.next(P)) {
        uint32_t bytes;
        const uint8_t* src = slab_src(c0, bytes);
        mbar_arrive_expect_tx(&full[i], bytes + (uint32_t)P.bt_bytes);
        bulk_g2s(smem + (size_t)i * P.stage_bytes, src, bytes, &full[i]);
        last_round[i] = 0;
      }
      grid_dependency_wait();  // the activation tiles come from the conversion kernel
      c0 = c;
      for (int i = 0; i < pre; ++i, c0.next(P)) {
        const TcProb& pr = P.prob[c0.p];
        bulk_g2s(smem + (size_t)i * P.stage_bytes + P.raw_bytes, P.ws + pr.bt_off + (int64_t)c0.j * P.bt_bytes,
                 (uint32_t)P.bt_bytes, &full[i]);
      }
      for (int i = pre; i < n; ++i, c0.next(P)) {
        const int st = i % NS, r = i / NS;
        if (!tc_wait(P, &empty[st], (uint32_t)((r & 1) ^ 1), abort)) break;
        uint32_t bytes;
        const uint8_t* src = slab_src(c0, bytes);
        const TcProb& pr = P.prob[c0.p];
        mbar_arrive_expect_tx(&full[st], bytes + (uint32_t)P.bt_bytes);
        bulk_g2s(smem + (size_t)st * P.stage_bytes, src, bytes, &full[st]);
        bulk_g2s(smem + (size_t)st * P.stage_bytes + P.raw_bytes, P.ws + pr.bt_off + (int64_t)c0.j * P.bt_bytes,
                 (uint32_t)P.bt_bytes, &full[st]);
        last_round[st] = r;
      }
      // no copy may still be in flight when the CTA exits
      for (int st = 0; st < NS; ++st)
        if (last_round[st] >= 0 && !mbar_wait_bounded(&full[st], (uint32_t)(last_round[st] & 1), kWaitLimitNs))
          tc_error(P, DRACO_ERR_TIMEOUT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc_idesc_f16(128, NP);
      const uint32_t a_lo0 = tc_desc_lo(smem_u32(smem + P.a_off));
      const uint64_t mins_desc0 = tc_sdesc_plain(smem_u32(smem + P.m_off), 128u, 256u);
      TcRing ring;
      TcCursor cur;
      cur.seek(P, s_begin);
      for (int i = 0; i < n; ++i, cur.next(P)) {
        const TcProb& pr = P.prob[cur.p];
        const int st = i % NS, pb = i % kTcAcc;
        const uint32_t ph = (uint32_t)((i / NS) & 1), sph = (uint32_t)((i / kTcAcc) & 1);
        if (!tc_wait(P, &full[st], ph, abort)) break;
        if (!tc_wait(P, &acce[pb], sph ^ 1u, abort)) break;
        tc_fence_after();
        const uint8_t* bt = smem + (size_t)st * P.stage_bytes + P.raw_bytes;
        const float4* us = reinterpret_cast<const float4*>(bt + 5 * NP * 128);
#pragma unroll
        for (int b = 0; b < NP / 4; ++b) reinterpret_cast<float4*>(u_buf[pb])[b] = us[b];
        mbar_arrive(&ddf[pb]);
        const uint32_t acc = tmem + (uint32_t)(pb * 2 * NP), b_lo = tc_desc_lo(smem_u32(bt));
        bool ok = true;
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          if (!tc_wait(P, &aful[ring.a], ring.ph, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_lo = a_lo0 + (uint32_t)(ring.a * (kTcATile >> 4));
#pragma unroll
          for (int kk2 = 0; kk2 < 2; ++kk2) {
            const int q = 2 * sl + kk2;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma(acc, tc_desc(a_lo + (uint32_t)((kk2 * kTcKbTile + 32 * kk) >> 4), kSw128DescHi),
                     tc_desc(b_lo + (uint32_t)((q * NP * 128 + 32 * kk) >> 4), kSw128DescHi), idesc,
                     (uint32_t)((q | kk) != 0));
          }
          // the mins tile was written with the first slot
          if (sl == 0 && pr.qt != kQ6_K)
            tc_mma(acc + NP, mins_desc0 + (uint64_t)(pb * (kTcMinsBytes >> 4)),
                   tc_desc(b_lo + (uint32_t)((4 * NP * 128) >> 4), kSw128DescHi), idesc, 0u);
          tc_commit(&aemp[ring.a]);
          ring.next();
        }
        if (!ok) break;
        tc_commit(&empty[st]);
        tc_commit(&accf[pb]);
      }
      // every MMA issued has completed before the tensor memory is freed
      tc_commit(&mma_done);
      if (!mbar_wait_bounded(&mma_done, 0u, kWaitLimitNs)) tc_error(P, DRACO_ERR_TIMEOUT);
    }
  } else if (warp >= kTcEpi0 && warp < kTcEpi0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int e = warp & 3, r = 32 * e + lane;
    grid_dependency_wait();  // y may still be read by the preceding kernel
    float y[NP];
#pragma unroll
    for (int b = 0; b < NP; ++b) y[b] = 0.f;
    TcCursor cur;
    cur.seek(P, s_begin);
    for (int i = 0; i < n; ++i, cur.next(P)) {
      const TcProb& pr = P.prob[cur.p];
      const int pb = i % kTcAcc;
      const uint32_t sph = (uint32_t)((i / kTcAcc) & 1);
      if (!__all_sync(0xffffffffu, tc_wait(P, &accf[pb], sph, abort))) break;
      if (!__all_sync(0xffffffffu, tc_wait(P, &ddf[pb], sph, abort))) break;
      tc_fence_after();
      const bool mins = pr.qt != kQ6_K;
      const float2 dd = dd_buf[pb][r];
      const uint32_t taddr = tmem + ((uint32_t)(32 * e) << 16) + (uint32_t)(pb * 2 * NP);
      constexpr int kPiece = NP > 16 ? 8 : 16;  // columns per TMEM load (registers: y holds NP)
#pragma unroll
      for (int h = 0; h < NP; h += kPiece) {
        float v[kPiece], v2[kPiece];
        tc_ld<kPiece>(taddr + h, v);
        if (mins) tc_ld<kPiece>(taddr + NP + h, v2);
        tc_ld_wait();
#pragma unroll
        for (int b = 0; b < kPiece; ++b) {
          float t = dd.x * v[b];
          if (mins) t = fmaf(-dd.y, v2[b], t);
          y[h + b] = fmaf(u_buf[pb][h + b], t, y[h + b]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[pb]);
      if (cur.j == pr.nb - 1 || i == n - 1) {
        tc_flush<NP>(P, pr, cur.rg, s_begin, s_end, e, lane, y);
#pragma unroll
        for (int b = 0; b < NP; ++b) y[b] = 0.f;
      }
    }
  } else if (warp >= kTcDeq0) {
    // ------------------------------------------------------------ dequant
    const int c = warp - kTcDeq0;
    TcRing ring;
    TcCursor cur;
    cur.seek(P, s_begin);
    for (int i = 0; i < n; ++i, cur.next(P)) {
      const TcProb& pr = P.prob[cur.p];
      const int st = i % NS, pb = i % kTcAcc;
      const uint32_t ph = (uint32_t)((i / NS) & 1), sph = (uint32_t)((i / kTcAcc) & 1);
      const int rem = pr.n_tiles - cur.rg * kGroupTiles;
      const bool live = c < (rem < kGroupTiles ? rem : kGroupTiles);
      if (!__all_sync(0xffffffffu, tc_wait(P, &full[st], ph, abort))) break;
      const uint8_t* ch = smem + (size_t)st * P.stage_bytes + (size_t)c * pr.cb;
      bool ok;
      if (pr.qt == kQ4_K)
        ok = tc_dequant_slab<kQ4_K>(P, smem, ch, live, c, lane, &acce[pb], sph, &ddf[pb], dd_buf[pb],
                                    smem + P.m_off + pb * kTcMinsBytes, aful, aemp, ring, abort);
      else if (pr.qt == kQ5_K)
        ok = tc_dequant_slab<kQ5_K>(P, smem, ch, live, c, lane, &acce[pb], sph, &ddf[pb], dd_buf[pb],
                                    smem + P.m_off + pb * kTcMinsBytes, aful, aemp, ring, abort);
      else
        ok = tc_dequant_slab<kQ6_K>(P, smem, ch, live, c, lane, &acce[pb], sph, &ddf[pb], dd_buf[pb],
                                    smem + P.m_off + pb * kTcMinsBytes, aful, aemp, ring, abort);
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
  }
}

// ---------------------------------------------------------------------------
// activation conversion, once per launch: one warp per (problem, super-block,
// batch row) writes the row of the super-block's tile in the shared-memory
// image of the MMA's B operand (batch rows x 64 k per k-block, K-major,
// 128-byte swizzle), its sub-block sums (hi, lo) in a 5th block and its scale
// u; rows past the batch are zero.  Warps past those units compute RMSNorm
// row scales (draco/kernels/ops.py:46-48), summed in a fixed order.
// ---------------------------------------------------------------------------
// 4 consecutive fp32 values at p into v[o..o+3] (a 16-byte load when aligned);
// the ones at or past `valid` read as 0
__device__ __forceinline__ void tc_load4(const float* p, int valid, float (&v)[8], int o) {
  if (valid >= 4 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(p));
    v[o] = q.x, v[o + 1] = q.y, v[o + 2] = q.z, v[o + 3] = q.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[o + i] = i < valid ? __ldg(p + i) : 0.f;
  }
}

constexpr int kTcConvWarps = 8;

template <int NP>
__global__ void __launch_bounds__(kTcConvWarps * 32) gemv_tc_convert(const __grid_constant__ TcParams P) {
  grid_launch_dependents();  // the GEMV may start streaming weights at once
  grid_dependency_wait();    // x (and the tiles, read by the previous GEMV) belong to the preceding kernel
  const int lane = threadIdx.x & 31;
  int u = blockIdx.x * kTcConvWarps + (threadIdx.x >> 5), p = 0;
  while (p < P.n_prob && u >= P.prob[p].nb * NP) u -= P.prob[p].nb * NP, ++p;
  if (p >= P.n_prob) {
    for (p = 0; p < P.n_prob; ++p) {
      if (P.prob[p].in_mode != DRACO_INPUT_RMSNORM) continue;
      if (u < P.batch) break;
      u -= P.batch;
    }
    if (p >= P.n_prob) return;
    const TcProb& pr = P.prob[p];
    const float* xr = pr.x + (int64_t)u * pr.ldx;
    float ss = 0.f;
    for (int i = lane; i < pr.k; i += 32) ss = fmaf(xr[i], xr[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) reinterpret_cast<float*>(P.ws + pr.rms_off)[u] = 1.f / sqrtf(ss / (float)pr.k + pr.eps);
    return;
  }
  const TcProb& pr = P.prob[p];
  const int sb = u / NP, b = u - sb * NP;
  uint8_t* tile = P.ws + pr.bt_off + (int64_t)sb * P.bt_bytes;
  // this lane's chunk c = lane % 8 of k-block lane / 8: k = 16h + 4t + (0..3)
  // and 32 + 16h + 4t + (0..3), c = 2t + h (the order the A tiles use)
  const int kb = lane >> 3, cc = lane & 7, rb = b & 7;
  const int kk0 = 256 * sb + 64 * kb + 16 * (cc & 1) + 4 * (cc >> 1), kk1 = kk0 + 32;
  float v[8];
  if (b < P.batch) {
    const float* xr = pr.x + (int64_t)b * pr.ldx;
    tc_load4(xr + kk0, pr.k - kk0, v, 0);
    tc_load4(xr + kk1, pr.k - kk1, v, 4);
    if (pr.in_mode != DRACO_INPUT_PLAIN) {
      float a[8];
      const bool sw = pr.in_mode == DRACO_INPUT_SWIGLU;
      const float* ar = pr.aux + (sw ? (int64_t)b * pr.ldaux : 0);
      tc_load4(ar + kk0, pr.k - kk0, a, 0);
      tc_load4(ar + kk1, pr.k - kk1, a, 4);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = sw ? silu_mul(v[i], a[i]) : v[i] * a[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // u = 2^e with max |x| / u in [1/2, 1), from the exponent field (clamped:
  // zero and subnormal rows take the smallest u, inf / nan the largest)
  int e = ((__float_as_int(amax) >> 23) & 0xFF) - 126;
  e = max(-126, min(126, e));
  const float inv = __int_as_float((127 - e) << 23), us = __int_as_float((127 + e) << 23);
  // the sums are taken over the rounded values the MMA sees, so that the
  // min term cancels against the product exactly as in W . fp16(x / u)
  __half2 h[4];
  float sa = 0.f, sb2 = 0.f;  // sub-blocks 2kb (first four values) and 2kb + 1
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[i] = __floats2half2_rn(v[2 * i] * inv, v[2 * i + 1] * inv);
    if (i < 2) sa += __low2float(h[i]) + __high2float(h[i]);
    else sb2 += __low2float(h[i]) + __high2float(h[i]);
  }
  *reinterpret_cast<uint4*>(tile + (size_t)kb * NP * 128 + (b >> 3) * 1024 + rb * 128 + ((cc ^ rb) << 4)) =
      *reinterpret_cast<uint4*>(h);
  // the sums over the 8 lanes of the k-block, as fp16 hi + lo
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
    sb2 += __shfl_xor_sync(0xffffffffu, sb2, o);
  }
  auto hilo = [](float x) {
    const __half hh = __float2half_rn(x);
    const __half ll = __float2half_rn(x - __half2float(hh));
    return (uint32_t)__half_as_ushort(hh) | ((uint32_t)__half_as_ushort(ll) << 16);
  };
  const uint32_t ba = hilo(sa), bb = hilo(sb2);
  uint32_t pk[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // sub-block j: lane 8 (j / 2), first or second sum
    const uint32_t wa = __shfl_sync(0xffffffffu, ba, 8 * (j >> 1)), wb = __shfl_sync(0xffffffffu, bb, 8 * (j >> 1));
    const uint32_t w = (j & 1) ? wb : wa;
    const uint32_t half = (lane == 0) ? (w & 0xFFFFu) : (w >> 16);  // lane 0: hi parts, lane 1: lo parts
    pk[j >> 1] |= half << (16 * (j & 1));
  }
  if (lane < 8) {
    const uint4 val = lane < 2 ? make_uint4(pk[0], pk[1], pk[2], pk[3]) : make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(tile + (size_t)4 * NP * 128 + (b >> 3) * 1024 + rb * 128 + ((lane ^ rb) << 4)) = val;
  }
  if (lane == 0) reinterpret_cast<float*>(tile + (size_t)5 * NP * 128)[b] = b < P.batch ? us : 0.f;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int tc_min_batch() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("DRACO_GEMV_TC_MIN_BATCH");  // 33 disables the kernel
    v = s ? atoi(s) : kTcMinBatchDefault;
    if (v < 1) v = 1;
  }
  return v;
}

bool gemv_tc_eligible(const draco_gemv_problem* probs, int n, int batch) {
  if (n < 1 || batch < tc_min_batch() || batch > 32) return false;
  for (int p = 0; p < n; ++p)
    if (probs[p].qtype != kQ4_K && probs[p].qtype != kQ5_K && probs[p].qtype != kQ6_K) return false;
  return true;
}

struct TcLayout {
  int np, bt_bytes;
  int64_t part_off, bt_off[DRACO_GEMV_MAX_PROBLEMS], rms_off[DRACO_GEMV_MAX_PROBLEMS], total;
};
static int64_t align1024(int64_t v) { return (v + 1023) & ~(int64_t)1023; }

static void tc_layout(const draco_gemv_problem* probs, int n, int batch, TcLayout& L) {
  L.np = batch <= 16 ? 16 : 32;
  L.bt_bytes = tc_bt_bytes(L.np);
  int64_t off = align1024(kWsCounters + kWsCountersBytes);
  L.part_off = off;
  off = align1024(off + (int64_t)kMaxCta * 2 * 128 * L.np * 4);
  for (int p = 0; p < n; ++p) {
    const TiledGeom g = tiled_geom(probs[p].qtype, probs[p].n_rows, probs[p].k);
    L.bt_off[p] = off;
    off = align1024(off + g.nb * L.bt_bytes);
    L.rms_off[p] = off;
    off = align1024(off + (int64_t)batch * 4);
  }
  L.total = off;
}

size_t gemv_tc_workspace_bytes(const draco_gemv_problem* probs, int n, int batch, const draco_gemv_input* inputs) {
  (void)inputs;
  if (!gemv_tc_eligible(probs, n, batch)) return 0;
  TcLayout L;
  tc_layout(probs, n, batch, L);
  return (size_t)L.total;
}

template <int NP>
static cudaError_t tc_launch(const TcParams& P, size_t smem, int conv_units, cudaStream_t st) {
  static int attr_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_tc_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kTcSmemBudget + 1024);
    if (e != cudaSuccess) return e;
    attr_set[dev] = 1;
  }
  // programmatic dependent launch for both kernels: the conversion is
  // scheduled while the preceding kernel drains and waits (griddepcontrol.wait)
  // before it reads x; the GEMV streams its first weights while the
  // conversion runs and waits before it reads the tiles
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const int blocks = (conv_units + kTcConvWarps - 1) / kTcConvWarps;
  cudaLaunchConfig_t ccfg = {};
  ccfg.gridDim = dim3(blocks);
  ccfg.blockDim = dim3(kTcConvWarps * 32);
  ccfg.stream = st;
  ccfg.attrs = attr;
  ccfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&ccfg, gemv_tc_convert<NP>, P);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P.n_cta);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, gemv_tc_kernel<NP>, P);
  if (e != cudaSuccess || P.n_split == 0) return e;
  cudaLaunchConfig_t fcfg = {};
  fcfg.gridDim = dim3(P.n_split);
  fcfg.blockDim = dim3(128);
  fcfg.stream = st;
  fcfg.attrs = attr;
  fcfg.numAttrs = 1;
  return cudaLaunchKernelEx(&fcfg, gemv_tc_fixup<NP>, P);
}

// Row groups whose slabs span more than one CTA's range, into P.split.
static bool tc_splits(const GemvParams& G, TcParams& P) {
  auto cta_of = [&](int s) {
    int c = 0;
    while (c + 1 < G.n_cta && G.cta_start[c + 1] <= s) ++c;
    return c;
  };
  P.n_split = 0;
  for (int p = 0; p < G.n_prob; ++p) {
    const GemvProbDev& d = G.prob[p];
    for (int rg = 0; rg < d.n_rg; ++rg) {
      const int a = d.slab0 + rg * d.nb, c0 = cta_of(a), c1 = cta_of(a + d.nb - 1);
      if (c0 == c1) continue;
      if (P.n_split == kMaxCta) return false;
      P.split[P.n_split++] = {p, rg, c0, c1};
    }
  }
  return true;
}

int gemv_tc_split_count(const HostPlan& hp) {
  TcParams P;  // only n_split is read
  return tc_splits(hp.P, P) ? P.n_split : kMaxCta;
}

int gemv_tc_launch(const HostPlan& hp, const draco_gemv_input* inputs, void* ws, size_t ws_bytes, cudaStream_t st,
                   char* msg, size_t ml) {
  (void)inputs;  // the plan carries the input transforms
  const GemvParams& G = hp.P;
  TcParams P;
  memset(&P, 0, sizeof(P));
  draco_gemv_problem probs[DRACO_GEMV_MAX_PROBLEMS];
  memset(probs, 0, sizeof(probs));
  for (int p = 0; p < G.n_prob; ++p) {
    probs[p].qtype = G.prob[p].qt;
    probs[p].n_rows = G.prob[p].n_rows;
    probs[p].k = G.prob[p].k;
  }
  TcLayout L;
  tc_layout(probs, G.n_prob, G.batch, L);
  if (ws == nullptr || ws_bytes < (size_t)L.total) {
    snprintf(msg, ml, "gemv: workspace of %zu bytes given, %lld needed", ws_bytes, (long long)L.total);
    return DRACO_ERR_WORKSPACE;
  }
  P.ws = static_cast<uint8_t*>(ws);
  P.part_off = L.part_off;
  P.n_prob = G.n_prob;
  P.batch = G.batch;
  P.np = L.np;
  P.n_cta = G.n_cta;
  P.total_slabs = G.total_slabs;
  P.bt_bytes = L.bt_bytes;
  int conv_units = 0;
  for (int p = 0; p < G.n_prob; ++p) {
    const GemvProbDev& s = G.prob[p];
    TcProb& d = P.prob[p];
    d.w = s.w;
    d.x = s.x;
    d.y = s.y;
    d.bias = s.bias;
    d.aux = s.aux;
    d.ldx = s.ldx;
    d.ldy = s.ldy;
    d.ldaux = s.ldaux;
    d.bt_off = L.bt_off[p];
    d.rms_off = L.rms_off[p];
    d.qt = s.qt;
    d.n_rows = s.n_rows;
    d.k = s.k;
    d.nb = s.nb;
    d.n_rg = s.n_rg;
    d.n_tiles = s.n_tiles;
    d.cb = s.cb;
    d.slab0 = s.slab0;
    d.in_mode = s.in_mode;
    d.accumulate = s.accumulate;
    d.eps = s.eps;
    conv_units += s.nb * L.np + (s.in_mode == DRACO_INPUT_RMSNORM ? G.batch : 0);
  }
  for (int c = 0; c <= G.n_cta; ++c) P.cta_start[c] = G.cta_start[c];
  if (!tc_splits(G, P)) {
    snprintf(msg, ml, "gemv: more than %d split row groups", kMaxCta);
    return DRACO_ERR_ARG;
  }
  P.raw_bytes = (int)align1024(G.w_stage);
  P.stage_bytes = P.raw_bytes + P.bt_bytes;
  const int a_bytes = kTcASlots * kTcATile + kTcAcc * kTcMinsBytes;
  P.ns = std::min(kTcMaxStages, (kTcSmemBudget - a_bytes) / P.stage_bytes);
  if (P.ns < 2) {
    snprintf(msg, ml, "gemv: stage of %d bytes does not fit shared memory twice", P.stage_bytes);
    return DRACO_ERR_ARG;
  }
  P.a_off = P.ns * P.stage_bytes;
  P.m_off = P.a_off + kTcASlots * kTcATile;
  const size_t smem = (size_t)P.a_off + a_bytes + 1024;  // + alignment slack of the dynamic base
  const cudaError_t e = P.np == 16 ? tc_launch<16>(P, smem, conv_units, st) : tc_launch<32>(P, smem, conv_units, st);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemv: tensor-memory kernel launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

}  // namespace draco
