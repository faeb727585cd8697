// gemm.cu — prefill dequant-GEMM  Y[M, N] = X[M, K] (bf16) . dequant(W)[N, K]^T
// with W in the TILED GGUF layout (Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 / Q4_K /
// Q5_K / Q6_K), fp32 accumulation in tensor memory, Y in bf16 or fp32.
//
// Replaces the reference's prefill linear: executor._linear
// (draco/runtime/cpu/executor.py:47-79) -> GenericGemmKernel.matmul_f32
// (draco/runtime/cpu/kernels/generic.py:32-33) on gguf._dequantize's fp32
// cache (draco/format/gguf.py:272-497), at M = prompt length.
//
// Design (B200, tensor-bound): persistent clusters of two CTAs (one SM pair),
// one CTA per SM, 16 warps each.  The pair runs tcgen05.mma.cta_group::2
// (M256 N256 K16, bf16 x bf16 -> fp32): the 256 tokens of the M dimension are
// split 128 per CTA (A = X, loaded by TMA), the 256 weight rows of the N
// dimension 128 per CTA (B = dequantized W, one TILED row group per CTA), so
// every SM feeds the tensor core 8 KB of shared memory per MMA instead of the
// 12 KB a single-SM M128 N256 MMA needs.
//  * pair tile = 256 weight rows x 512 tokens: two 256-column fp32
//    accumulators per CTA (its 128 tokens of each 256-token half x all 256
//    rows) fill the 512 TMEM columns; the K loop runs in 64-element blocks
//    (one 128-byte swizzle atom of bf16).
//  * warp 0 (one lane, both CTAs): TMA loads of this CTA's X boxes (64 k x 128
//    tokens, 128-byte swizzle, completion counted on the leader CTA's barrier)
//    and 1-D bulk copies of this CTA's packed weight slab (128 rows x 256 k,
//    contiguous in the TILED layout).
//  * warps 8-15 (dequant, both CTAs): expand each 64-k block of the slab into
//    a bf16 B tile (128 rows x 64 k, K-major, 128-byte swizzle); each value is
//    the fp32 dequantized weight (same operations as gguf._dequantize) rounded
//    to bf16.  fence.proxy.async, then an arrive on the leader's barrier.
//  * warp 1: allocates the 512 TMEM columns (cta_group::2, both CTAs); in the
//    leader CTA one lane issues the MMAs and tcgen05.commit with a cluster
//    multicast so both CTAs see stage and accumulator completion.
//  * warps 4-7 (epilogue, both CTAs): tcgen05.ld of the CTA's accumulators
//    (warp w reads TMEM lanes 32(w%4)..+31 = tokens), each lane holding 32
//    consecutive weight rows of one token, stored as 16-byte vectors.
//  * every wait is bounded; on a timeout the kernel records DRACO_ERR_TIMEOUT,
//    unwinds, waits for its own MMAs, and still frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace draco {

constexpr int kGemmMaxProblems = DRACO_GEMM_MAX_PROBLEMS;
constexpr int kBM = 128;                          // weight rows per CTA (one TILED row group)
constexpr int kTokCta = 128;                      // tokens per CTA per accumulator
constexpr int kNH = 2;                            // accumulators per CTA
constexpr int kUmmaN = 256;                       // weight rows per pair (UMMA N)
constexpr int kUmmaM = 256;                       // tokens per pair and accumulator (UMMA M)
constexpr int kTileTok = kNH * kUmmaM;            // 512 tokens per pair tile
constexpr int kBK = 64;                           // k per block
constexpr int kXBox = kTokCta * kBK * 2;          // 16 KB: one TMA box of X
constexpr int kATile = kBM * kBK * 2;             // 16 KB: one dequantized weight tile
constexpr int kGemmThreads = 16 * 32;
constexpr int kDeqWarp0 = 8, kDeqWarps = 8;
constexpr int kEpiWarp0 = 4, kEpiWarps = 4;
constexpr int kMaxStages = 6;
constexpr int kStageBytes = 32 * 32 * 4;          // epilogue staging tile (32 tokens x 32 rows, fp32 max)
constexpr uint64_t kGemmWaitNs = 4000000000ull;  // 4 s

struct GemmProbDev {
  const uint8_t* w;
  void* y;
  int64_t ldy;
  int qt, ydtype, m, n, k, nb, n_rg, n_tiles, cb, tblocks, tile0, vec, ymode;
  int src;  // index of the problem in the caller's array (device row counts are in that order)
};
constexpr int kYDirect = 0, kYTma = 1;  // epilogue: direct stores or staged TMA stores

constexpr int kMaxPairs = 96;     // CTA pairs a launch may use (148 SMs -> 74)
constexpr int kMaxSched = 4096;   // tiles a precomputed schedule may hold

struct __align__(64) GemmParams {
  CUtensorMap xmap[kGemmMaxProblems];
  CUtensorMap ymap[kGemmMaxProblems];
  GemmProbDev prob[kGemmMaxProblems];
  int* status;
  const int* rows;  // optional device row counts per problem (caller's order); m is then the capacity
  int n_prob, total_tiles;
  int sched_ok;                       // 1: pair p runs tiles sched[off[p] .. off[p+1]); 0: strided
  uint16_t off[kMaxPairs + 1];
  uint16_t sched[kMaxSched];
  int ns;  // k-block stages
  int x_off, a_off, st_off, smem_bytes;
};

// ---------------------------------------------------------------------------
// PTX wrappers (tcgen05, TMA tensor loads, proxy fences)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ----- cluster (CTA pair) helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared-memory object in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}
// arrive on an mbarrier of another CTA of the cluster.  Default (CTA-scope)
// release: the shared-memory writes the arrive publishes were made visible to
// the async proxy by fence.proxy.async before it, and the tensor core of the
// pair reads them only after the barrier completes.  A cluster-scope release
// costs about a thousand cycles per arrive.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Waits on barriers that the other CTA or the pair's tensor-core work completes
// use the default (CTA-scope) try_wait: the arriving side releases at cluster
// scope (remote arrives) or completes through the async proxy (TMA bytes,
// tcgen05.commit).  A cluster-scope acquire on every poll costs a few hundred
// cycles, which the MMA issue loop cannot afford three times per k-block.


// TMA 2-D tile load into this CTA's shared memory; the transaction bytes are
// counted on `bar_cluster` (a barrier of the leader CTA of the pair).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}

// K-major, 128-byte-swizzled operand: 8-row groups 1024 B apart (SBO), start
// address advanced by 32 B per K=16 step inside the swizzle atom.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}
// kind::f16 instruction descriptor: bf16 A and B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T across the CTA pair (issued by the leader)
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive (once) on the barrier at the same offset in both CTAs of the pair
// when all previously issued MMAs of this thread have completed
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
// arrive on this CTA's barrier only
__device__ __forceinline__ void umma_commit_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
// wait for this thread's tcgen05.ld results; v is tied to the wait so no use
// of the loaded registers can be scheduled before it
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&v)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]), "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])::"memory");
}
__device__ __forceinline__ void reg_tie(uint32_t (&v)[32]) { asm volatile("" : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]), "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// dequantization of one 64-k block of a packed slab into the bf16 B tile
// (128 rows x 64 k, K-major, 128-byte swizzle).  Warp w takes chunk w (rows
// 16w..16w+15); lane L = 4g + t reads the 16-byte unit L of the chunk's
// fragment-ordered fields (rows g and g+8, one 128-bit shared load) and
// produces 32 values: 8 groups of 4 consecutive k, each stored as 8 bytes.
// The two 32-k halves of the block are visited in the order g&1, g&1^1, so
// that every half-warp's 8-byte stores cover all 32 banks once.
// Every value is the fp32 number gguf._dequantize computes (the products with
// the scales are exact; the one rounding is the same), then rounded to bf16;
// the arithmetic runs two values at a time in the packed f32x2 pipes.
// ---------------------------------------------------------------------------
// read-only global loads that bypass L1 (each packed byte is used once per tile)
__device__ __forceinline__ uint4 ldg128(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg64(const uint8_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg32(const uint8_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// One lane's packed inputs for one 64-k block of its row tile, 16 registers
// whatever the type (loaded two blocks ahead of use, so the global-load
// latency hides behind the dequantization of the blocks before):
//  Q4_K: u0 = qs unit; u1 = scale bytes 0-7 (row g), 8-11 (row g), 0-3 (row g+8);
//        u2 = scale bytes 4-11 (row g+8), (d, dmin) of row g, of row g+8
//  Q5_K: as Q4_K, plus u3 = the qh unit (fifth bits, word for word as u0)
//  Q6_K: u0..u2 = ql/qh units of half q/2; u3 = int8 scales of rows g, g+8, d of both rows
//  Q8_0: u0, u1 = qs units of blocks 2q, 2q+1; u2.x, u2.y = d of both blocks for rows g, g+8
//  Q4_0 / Q4_1 / Q5_0 / Q5_1: u0 = qs unit of block pair q; u2 = d of blocks 2q, 2q+1 for
//        rows g, g+8, then m (Q4_1 / Q5_1) the same way; u1 = qh words (Q5_x) of
//        (row g: blocks 2q, 2q+1), (row g+8: blocks 2q, 2q+1)
struct Packed {
  uint4 u0, u1, u2, u3;
};
// kLegacy: the launch holds a Q4_0 / Q4_1 / Q5_0 / Q5_1 weight.  The kernel is
// compiled once with and once without that code, so the K-quant and Q8_0
// launches run a dequant loop free of it (with it inlined the config-3
// prefill lost ~2.5 % through instruction-cache pressure).
template <bool kLegacy>
__device__ __forceinline__ void fetch_packed(int qt, const uint8_t* ch, int q, int lane, Packed& pk) {
  const int g = lane >> 2;
  if (qt == kQ4_K || qt == kQ5_K) {
    const int so = qt == kQ5_K ? 2560 : 2048, dof = qt == kQ5_K ? 2752 : 2240;
    pk.u0 = ldg128(ch + 512 * q + 16 * lane);
    const uint2 a = ldg64(ch + so + 24 * g), b = ldg64(ch + so + 8 + 24 * g), c = ldg64(ch + so + 16 + 24 * g);
    const uint2 d = ldg64(ch + dof + 8 * g);
    pk.u1 = make_uint4(a.x, a.y, b.x, b.y);
    pk.u2 = make_uint4(c.x, c.y, d.x, d.y);
    if (qt == kQ5_K) pk.u3 = ldg128(ch + 2048 + 16 * lane);
  } else if (qt == kQ6_K) {
    const int n = q >> 1, odd = q & 1;
    pk.u0 = ldg128(ch + 512 * (3 * n) + 16 * lane);
    pk.u1 = ldg128(ch + 512 * (3 * n + 1) + 16 * lane);
    pk.u2 = ldg128(ch + 512 * (3 * n + 2) + 16 * lane);
    pk.u3.x = ldg32(ch + 3072 + 32 * g + 8 * n + 4 * odd);
    pk.u3.y = ldg32(ch + 3072 + 32 * g + 16 + 8 * n + 4 * odd);
    pk.u3.z = ldg32(ch + 3328 + 4 * g);
  } else if (!kLegacy || qt == kQ8_0) {
    pk.u0 = ldg128(ch + 512 * (2 * q) + 16 * lane);
    pk.u1 = ldg128(ch + 512 * (2 * q + 1) + 16 * lane);
    pk.u2.x = ldg32(ch + 4096 + 32 * g + 4 * q);
    pk.u2.y = ldg32(ch + 4096 + 32 * g + 16 + 4 * q);
  } else if constexpr (kLegacy) {
    const Q4xFields f = q4x_fields(qt);
    pk.u0 = ldg128(ch + 512 * q + 16 * lane);
    pk.u2.x = ldg32(ch + f.d + 32 * g + 4 * q);
    pk.u2.y = ldg32(ch + f.d + 32 * g + 16 + 4 * q);
    if (f.m >= 0) {
      pk.u2.z = ldg32(ch + f.m + 32 * g + 4 * q);
      pk.u2.w = ldg32(ch + f.m + 32 * g + 16 + 4 * q);
    }
    if (f.qh >= 0) {
      const uint2 h0 = ldg64(ch + f.qh + 64 * g + 8 * q), h1 = ldg64(ch + f.qh + 64 * g + 32 + 8 * q);
      pk.u1 = make_uint4(h0.x, h0.y, h1.x, h1.y);
    }
  }
}

__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }
__device__ __forceinline__ uint64_t splat2(float v) { return pack2(__float_as_uint(v), __float_as_uint(v)); }
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// (lo, hi) fp32 pair -> bf16x2 with lo in the low half
__device__ __forceinline__ uint32_t bf16x2_of(uint64_t v) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "r"((uint32_t)(v >> 32)), "r"((uint32_t)v));
  return r;
}
// bytes 2j, 2j+1 of w as the fp32 pair (2^23 + byte) (exact)
constexpr uint32_t kMagic23 = 0x4B000000u;
__device__ __forceinline__ uint64_t magic_pair(uint32_t w, int j) {
  return pack2(__byte_perm(w, kMagic23, 0x7440u | (2 * j)), __byte_perm(w, kMagic23, 0x7440u | (2 * j + 1)));
}
// the 4 bytes of w (each < 2^8, minus `bias`) scaled: returns the 4 bf16 values as uint2
__device__ __forceinline__ uint2 scale4_mul(uint32_t w, uint64_t bias2, uint64_t s2) {
  const uint64_t v01 = mul2(add2(magic_pair(w, 0), bias2), s2);
  const uint64_t v23 = mul2(add2(magic_pair(w, 1), bias2), s2);
  return make_uint2(bf16x2_of(v01), bf16x2_of(v23));
}
__device__ __forceinline__ uint2 scale4_fma(uint32_t w, uint64_t bias2, uint64_t s2, uint64_t c2) {
  const uint64_t v01 = fma2(add2(magic_pair(w, 0), bias2), s2, c2);
  const uint64_t v23 = fma2(add2(magic_pair(w, 1), bias2), s2, c2);
  return make_uint2(bf16x2_of(v01), bf16x2_of(v23));
}
// 8 bytes (k = 8c + 4(t&1) .. +3 of tile row g + 8hi of this warp's chunk)
__device__ __forceinline__ void st_piece(uint8_t* tw, int hi, int g, int t, int c, uint2 v) {
  *reinterpret_cast<uint2*>(tw + hi * 1024 + g * 128 + ((c ^ g) << 4) + 8 * (t & 1)) = v;
}
__device__ __forceinline__ float f16lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
__device__ __forceinline__ float f16hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

// Q4_K: k-block q = sub-blocks 2q (low nibbles of qs bytes 32q..32q+31) and
// 2q+1 (high nibbles).  Unit word (hi, h): row g+8hi, qs bytes 16h+4t..+3.
// Q5_K (K5): each quant also takes its fifth bit from the qh unit's word
// (hi, h), bit 2q (low nibble) or 2q+1 (high nibble) of each byte.
template <bool K5>
__device__ __forceinline__ void deq_q4k(const Packed& pk, int q, int lane, uint8_t* tw) {
  const int g = lane >> 2, t = lane & 3, g0 = g & 1;
  const uint4 U = pk.u0;
  const uint2 S0 = make_uint2(pk.u1.x, pk.u1.y), S1 = make_uint2(pk.u1.z, pk.u1.w), S2 = make_uint2(pk.u2.x, pk.u2.y);
  const uint2 DD = make_uint2(pk.u2.z, pk.u2.w);
  const uint64_t bias = splat2(-8388608.f);
#pragma unroll
  for (int hi = 0; hi < 2; ++hi) {
    const uint32_t A = hi ? S1.y : S0.x, B = hi ? S2.x : S0.y, C = hi ? S2.y : S1.x;
    const uint32_t dd = hi ? DD.y : DD.x;
    // (scale, min) 6-bit pairs of sub-blocks 2q (byte 0) and 2q+1 (byte 1)
    uint32_t scp, mp;
    if (q < 2) {
      scp = (A >> (16 * q)) & 0x3F3Fu;
      mp = (B >> (16 * q)) & 0x3F3Fu;
    } else {
      const int s = 16 * (q - 2);
      const uint32_t a = A >> s, b = B >> s, c = C >> s;
      scp = (c & 0x0F0Fu) | ((a >> 2) & 0x3030u);
      mp = ((c >> 4) & 0x0F0Fu) | ((b >> 2) & 0x3030u);
    }
    const uint64_t ds = mul2(add2(magic_pair(scp, 0), bias), splat2(f16lo(dd)));   // d * sc   (exact)
    const uint64_t dm = mul2(add2(magic_pair(mp, 0), bias), splat2(-f16hi(dd)));   // -dmin * m (exact)
    const uint32_t ds_lo = (uint32_t)ds, ds_hi = (uint32_t)(ds >> 32), dm_lo = (uint32_t)dm, dm_hi = (uint32_t)(dm >> 32);
    const uint64_t dsA = splat2(__uint_as_float(g0 ? ds_hi : ds_lo)), dsB = splat2(__uint_as_float(g0 ? ds_lo : ds_hi));
    const uint64_t dmA = splat2(__uint_as_float(g0 ? dm_hi : dm_lo)), dmB = splat2(__uint_as_float(g0 ? dm_lo : dm_hi));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w = hi ? (h ? U.w : U.z) : (h ? U.y : U.x);
      const uint32_t hw = hi ? (h ? pk.u3.w : pk.u3.z) : (h ? pk.u3.y : pk.u3.x);
#pragma unroll
      for (int n0 = 0; n0 < 2; ++n0) {
        const int nib = g0 ^ n0;
        uint32_t wq = (w >> (4 * nib)) & 0x0F0F0F0Fu;
        if (K5) {
          const int b = 2 * q + nib;
          wq |= (b <= 4 ? (hw << (4 - b)) : (hw >> (b - 4))) & 0x10101010u;
        }
        st_piece(tw, hi, g, t, 4 * nib + 2 * h + (t >> 1), scale4_fma(wq, bias, n0 ? dsB : dsA, n0 ? dmB : dmA));
      }
    }
  }
}

// Q6_K: k-block q = groups i = 2(q&1) + ii (ii = 0, 1) of half n = q/2.
// Lane words 12n..12n+11 (three units): word 6is + 3hi + {0: ql l, 1: ql l+32, 2: qh}.
__device__ __forceinline__ void deq_q6k(const Packed& pk, int q, int lane, uint8_t* tw) {
  const int g = lane >> 2, t = lane & 3, g0 = g & 1;
  const int odd = q & 1;
  const uint4 P0 = pk.u0, P1 = pk.u1, P2 = pk.u2;
  const uint32_t W[12] = {P0.x, P0.y, P0.z, P0.w, P1.x, P1.y, P1.z, P1.w, P2.x, P2.y, P2.z, P2.w};
  const uint32_t dd = pk.u3.z;
  const uint64_t bias8 = splat2(-8388736.f);   // -(2^23 + 128): int8 scales stored ^ 0x80
  const uint64_t bias6 = splat2(-8388640.f);   // -(2^23 + 32)
#pragma unroll
  for (int hi = 0; hi < 2; ++hi) {
    // int8 scales of groups (is, ii) at byte is + 2ii
    const uint32_t scw = (hi ? pk.u3.y : pk.u3.x) ^ 0x80808080u;
    const uint64_t d2 = splat2(hi ? f16hi(dd) : f16lo(dd));
    const uint64_t dl01 = mul2(add2(magic_pair(scw, 0), bias8), d2);  // (is0 ii0, is1 ii0)
    const uint64_t dl23 = mul2(add2(magic_pair(scw, 1), bias8), d2);  // (is0 ii1, is1 ii1)
#pragma unroll
    for (int is = 0; is < 2; ++is) {
      const uint32_t s_ii0 = is ? (uint32_t)(dl01 >> 32) : (uint32_t)dl01;
      const uint32_t s_ii1 = is ? (uint32_t)(dl23 >> 32) : (uint32_t)dl23;
      const uint32_t qh = W[6 * is + 3 * hi + 2];
#pragma unroll
      for (int n0 = 0; n0 < 2; ++n0) {
        const int ii = g0 ^ n0;
        const uint32_t ql = ii ? W[6 * is + 3 * hi + 1] : W[6 * is + 3 * hi];
        const uint32_t lo = (ql >> (4 * odd)) & 0x0F0F0F0Fu;
        const uint32_t hb = (qh >> (2 * (2 * odd + ii))) & 0x03030303u;
        const uint32_t q6 = lo | (hb << 4);
        st_piece(tw, hi, g, t, 4 * ii + 2 * is + (t >> 1),
                 scale4_mul(q6, bias6, splat2(__uint_as_float(ii ? s_ii1 : s_ii0))));
      }
    }
  }
}

// Q8_0: k-block q = blocks 2q, 2q+1.  Unit word (hi, h): row g+8hi, qs bytes 16h+4t..+3.
__device__ __forceinline__ void deq_q80(const Packed& pk, int lane, uint8_t* tw) {
  const int g = lane >> 2, t = lane & 3, g0 = g & 1;
  const uint4 U0 = pk.u0, U1 = pk.u1;
  const uint64_t bias8 = splat2(-8388736.f);
#pragma unroll
  for (int hi = 0; hi < 2; ++hi) {
    const uint32_t dw = hi ? pk.u2.y : pk.u2.x;  // d of blocks 2q (lo), 2q+1 (hi)
    const uint64_t dA = splat2(g0 ? f16hi(dw) : f16lo(dw)), dB = splat2(g0 ? f16lo(dw) : f16hi(dw));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w0 = hi ? (h ? U0.w : U0.z) : (h ? U0.y : U0.x);
      const uint32_t w1 = hi ? (h ? U1.w : U1.z) : (h ? U1.y : U1.x);
#pragma unroll
      for (int n0 = 0; n0 < 2; ++n0) {
        const int bb = g0 ^ n0;
        st_piece(tw, hi, g, t, 4 * bb + 2 * h + (t >> 1),
                 scale4_mul((bb ? w1 : w0) ^ 0x80808080u, bias8, n0 ? dB : dA));
      }
    }
  }
}

// Q4_0 / Q4_1 / Q5_0 / Q5_1: k-block q = blocks 2q, 2q+1 (gguf.py:310-353).
// Unit word 2bb + hi: row g+8hi of block bb, qs bytes 4t..+3, whose low
// nibbles are elements 4t..+3 and high nibbles 16+4t..+3; the fifth bit of
// element e is bit e of the block's qh word.  One copy for the four types
// (the type is a run-time value): four inlined instantiations in the dequant
// loop cost the K-quants ~4 % through instruction-cache pressure; launches
// without these types use the kernel instantiation without this code.
__device__ __forceinline__ void deq_q4x(const Packed& pk, int lane, uint8_t* tw, int qt) {
  const bool has_h = qt == kQ5_0 || qt == kQ5_1, has_m = qt == kQ4_1 || qt == kQ5_1;
  const int g = lane >> 2, t = lane & 3, g0 = g & 1;
  const uint4 U = pk.u0;
  // q - 8 (Q4_0), q - 16 (Q5_0) or q from the bytes 2^23 + q
  const uint64_t bias = splat2(qt == kQ4_0 ? -8388616.f : qt == kQ5_0 ? -8388624.f : -8388608.f);
#pragma unroll
  for (int hi = 0; hi < 2; ++hi) {
    const uint32_t dw = hi ? pk.u2.y : pk.u2.x, mw = has_m ? (hi ? pk.u2.w : pk.u2.z) : 0u;
    const uint64_t dA = splat2(g0 ? f16hi(dw) : f16lo(dw)), dB = splat2(g0 ? f16lo(dw) : f16hi(dw));
    const uint64_t mA = splat2(g0 ? f16hi(mw) : f16lo(mw)), mB = splat2(g0 ? f16lo(mw) : f16hi(mw));
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
      for (int n0 = 0; n0 < 2; ++n0) {
        const int bb = g0 ^ n0;
        const uint32_t w = bb ? (hi ? U.w : U.z) : (hi ? U.y : U.x);
        uint32_t wq = (w >> (4 * half)) & 0x0F0F0F0Fu;
        if (has_h) {
          const uint32_t h = hi ? (bb ? pk.u1.w : pk.u1.z) : (bb ? pk.u1.y : pk.u1.x);
          wq |= ((h >> (16 * half + 4 * t)) & 15u) * 0x02040810u & 0x10101010u;
        }
        // q * d + m (m = 0 for Q4_0 / Q5_0, whose offset is in the bias)
        st_piece(tw, hi, g, t, 4 * bb + 2 * half + (t >> 1), scale4_fma(wq, bias, n0 ? dB : dA, n0 ? mB : mA));
      }
    }
  }
}

__device__ __forceinline__ void zero_rows16(uint8_t* tw, int lane) {
#pragma unroll
  for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(tw + 512 * i + 16 * lane) = make_uint4(0, 0, 0, 0);
}

__device__ __forceinline__ void gemm_error(const GemmParams& P, int code) {
  if (P.status) atomicCAS(P.status, 0, code);
}

// position in a ring of n stages and the parity of its current phase
// (incremented instead of divided: the MMA issue loop must stay lean)
struct Ring {
  int s = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next(int n) {
    if (++s == n) {
      s = 0;
      ph ^= 1u;
    }
  }
};

// i-th pair tile of `pair` (-1 past its last): the host's balanced schedule,
// or tiles pair, pair + npairs, ... when the launch has too many tiles for it
__device__ __forceinline__ int tile_at(const GemmParams& P, int pair, int i, int npairs) {
  if (P.sched_ok) {
    const int j = (int)P.off[pair] + i;
    return j < (int)P.off[pair + 1] ? (int)P.sched[j] : -1;
  }
  const int t = pair + i * npairs;
  return t < P.total_tiles ? t : -1;
}

// pair tile t -> (problem, row pair, 512-token block, the problem's token count)
struct TileCursor {
  int p, rp, tb, nkb, m;
  __device__ void at(const GemmParams& P, int t) {
    p = 0;
    for (int q = 1; q < P.n_prob; ++q)
      if (t >= P.prob[q].tile0) p = q;
    const int local = t - P.prob[p].tile0;
    rp = local / P.prob[p].tblocks;
    tb = local - rp * P.prob[p].tblocks;
    nkb = P.prob[p].nb * 4;
    m = P.prob[p].m;
    // rows counted on the device by a preceding kernel (read after the grid
    // dependency wait): tokens past them are neither loaded, multiplied nor stored
    if (P.rows) m = min(m, max(0, P.rows[P.prob[p].src]));
  }
};

__device__ __forceinline__ void store_rows(const GemmProbDev& pr, int m, int tok, int row0, const uint32_t (&v)[32]) {
  if (tok >= m || row0 >= pr.n) return;
  if (pr.ydtype == DRACO_DTYPE_BF16) {
    __nv_bfloat16* y = static_cast<__nv_bfloat16*>(pr.y) + (int64_t)tok * pr.ldy + row0;
    if (pr.vec && row0 + 32 <= pr.n) {
      uint4* d = reinterpret_cast<uint4*>(y);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        d[i] = make_uint4(bf16x2(__uint_as_float(v[8 * i]), __uint_as_float(v[8 * i + 1])),
                          bf16x2(__uint_as_float(v[8 * i + 2]), __uint_as_float(v[8 * i + 3])),
                          bf16x2(__uint_as_float(v[8 * i + 4]), __uint_as_float(v[8 * i + 5])),
                          bf16x2(__uint_as_float(v[8 * i + 6]), __uint_as_float(v[8 * i + 7])));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row0 + j < pr.n) y[j] = __float2bfloat16_rn(__uint_as_float(v[j]));
    }
  } else {
    float* y = static_cast<float*>(pr.y) + (int64_t)tok * pr.ldy + row0;
    if (pr.vec && row0 + 32 <= pr.n) {
      uint4* d = reinterpret_cast<uint4*>(y);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row0 + j < pr.n) y[j] = __uint_as_float(v[j]);
    }
  }
}

// TMA 2-D tile store from this CTA's shared memory (bulk-group completion)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 32 tokens x 32 rows of the accumulator -> staging tile [token][row] in the
// swizzle the Y tensor map uses (64-byte rows for bf16, 128-byte for fp32)
__device__ __forceinline__ void stage_rows(uint8_t* buf, int ydtype, int lane, const uint32_t (&v)[32]) {
  if (ydtype == DRACO_DTYPE_BF16) {
    uint8_t* row = buf + 64 * lane;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(row + ((j ^ sw) << 4)) =
          make_uint4(bf16x2(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1])),
                     bf16x2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3])),
                     bf16x2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5])),
                     bf16x2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7])));
  } else {
    uint8_t* row = buf + 128 * lane;
    const int sw = lane & 7;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(row + ((j ^ sw) << 4)) = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

// dequant-side view of one pair tile: this CTA's row tile dw of its row group
struct DeqTile {
  int i, nkb, qt;       // i: index of the tile in this pair's sequence
  const uint8_t* base;  // chunk dw of super-block 0 (null: row tile past n_rows)
  int64_t sb_stride;    // bytes between super-blocks of one row tile
  __device__ bool at(const GemmParams& P, int pair, int idx, int npairs, int rank, int dw) {
    const int tile = tile_at(P, pair, idx, npairs);
    if (tile < 0) return false;
    TileCursor c;
    c.at(P, tile);
    const GemmProbDev& pr = P.prob[c.p];
    const TiledGeom geo = tiled_geom(pr.qt, pr.n, pr.k);
    const int rg = 2 * c.rp + rank;
    const int nch = rg < pr.n_rg ? rg_tiles(geo, rg) : 0;
    i = idx;
    nkb = c.nkb;
    qt = pr.qt;
    base = dw < nch ? pr.w + slab_offset(geo, rg, 0) + (int64_t)dw * pr.cb : nullptr;
    sb_stride = (int64_t)nch * pr.cb;
    return true;
  }
  template <bool kLegacy>
  __device__ __forceinline__ void fetch(int kb, int lane, Packed& pk) const {
    if (base) fetch_packed<kLegacy>(qt, base + (kb >> 2) * sb_stride, kb & 3, lane, pk);
  }
  // next k-block of this CTA's sequence (crossing into its next pair tile)
  __device__ __forceinline__ bool advance(const GemmParams& P, int& kb, int pair, int npairs, int rank, int dw) {
    if (++kb < nkb) return true;
    kb = 0;
    return at(P, pair, i + 1, npairs, rank, dw);
  }
};

template <bool kLegacy>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // one ring of k-block stages: X boxes of both accumulators + the dequantized weight tile
  __shared__ __align__(8) uint64_t full_kb[kMaxStages], empty_kb[kMaxStages];
  __shared__ __align__(8) uint64_t acc_full[kNH], acc_empty[kNH], mma_done;
  __shared__ uint32_t s_tmem;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = P.ns;
  const uint32_t rank = cluster_rank();        // 0 = leader (issues the MMAs)
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      // leader: its producer's expect_tx (X bytes of both CTAs) and the
      // dequant warps of both CTAs
      mbar_init(&full_kb[i], 1 + 2 * kDeqWarps);
      mbar_init(&empty_kb[i], 1);               // MMA commit (multicast)
    }
    for (int i = 0; i < kNH; ++i) {
      mbar_init(&acc_full[i], 1);               // MMA commit (multicast)
      mbar_init(&acc_empty[i], 2 * kEpiWarps);  // leader: epilogue warps of both CTAs
    }
    mbar_init(&mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive or TMA
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  grid_dependency_wait();  // X may be written by the preceding kernel

  uint8_t* xs = smem + P.x_off;
  uint8_t* as = smem + P.a_off;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (X boxes)
    if (lane == 0) {
      Ring rs;
      bool ok = true;
      for (int i = 0, t; ok && (t = tile_at(P, pair, i, npairs)) >= 0; ++i) {
        TileCursor c;
        c.at(P, t);
        // this CTA's packed slabs, pulled into L2 two super-blocks ahead of the
        // dequant warps' loads
        const GemmProbDev& pr = P.prob[c.p];
        const TiledGeom geo = tiled_geom(pr.qt, pr.n, pr.k);
        const int rg = 2 * c.rp + (int)rank;
        const bool has_rg = rg < pr.n_rg;
        const uint8_t* rg_base = has_rg ? pr.w + slab_offset(geo, rg, 0) : nullptr;
        const uint32_t slab_bytes = has_rg ? (uint32_t)(rg_tiles(geo, rg) * pr.cb) : 0u;
        if (has_rg)
          for (int sb = 0; sb < 2 && sb < pr.nb; ++sb) bulk_prefetch_l2(rg_base + (int64_t)sb * slab_bytes, slab_bytes);
        for (int kb = 0; kb < c.nkb; ++kb) {
          if (has_rg && (kb & 3) == 0 && (kb >> 2) + 2 < pr.nb)
            bulk_prefetch_l2(rg_base + (int64_t)((kb >> 2) + 2) * slab_bytes, slab_bytes);
          if (!mbar_wait_bounded(&empty_kb[rs.s], rs.ph ^ 1u, kGemmWaitNs)) {
            gemm_error(P, DRACO_ERR_TIMEOUT);
            ok = false;
            break;
          }
          // X boxes that hold at least one token below M (a short prompt or
          // an expert's few tokens leave the upper ones empty): both CTAs
          // count the same boxes, the leader expects their bytes
          const int tok_tile = c.tb * kTileTok;
          const int m = c.m;
          if (rank == 0) {
            int nbox = 0;
#pragma unroll
            for (int hh = 0; hh < kNH; ++hh)
#pragma unroll
              for (int r = 0; r < 2; ++r) nbox += tok_tile + hh * kUmmaM + r * kTokCta < m;
            mbar_arrive_expect_tx(&full_kb[rs.s], (uint32_t)nbox * kXBox);
          }
          const uint32_t bar = map_to_rank(&full_kb[rs.s], 0);
#pragma unroll
          for (int hh = 0; hh < kNH; ++hh) {
            const int tok = tok_tile + hh * kUmmaM + (int)rank * kTokCta;
            if (tok < m) tma_load_2d_pair(xs + (size_t)(rs.s * kNH + hh) * kXBox, &P.xmap[c.p], kb * kBK, tok, bar);
          }
          rs.next(NS);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = idesc_bf16(kUmmaM, kUmmaN);
      const uint32_t x_base = smem_u32(xs), a_base = smem_u32(as);
      Ring rs;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int i = 0, t; ok && (t = tile_at(P, pair, i, npairs)) >= 0; ++i, acc_ph ^= 1u) {
        TileCursor c;
        c.at(P, t);
        // accumulators whose 256 tokens all lie at or past M get no MMAs
        const int tok_tile = c.tb * kTileTok;
        const int nh_live = tok_tile + kUmmaM < c.m ? 2 : (tok_tile < c.m ? 1 : 0);
        for (int kb = 0; kb < c.nkb && ok; ++kb) {
          // one wait per k-block: X boxes of both CTAs landed, both weight tiles dequantized
          if (!mbar_wait_bounded(&full_kb[rs.s], rs.ph, kGemmWaitNs)) {
            gemm_error(P, DRACO_ERR_TIMEOUT);
            ok = false;
            break;
          }
          const uint32_t a_addr = a_base + (uint32_t)rs.s * kATile;
          const uint32_t x_addr0 = x_base + (uint32_t)(rs.s * kNH) * kXBox;
#pragma unroll
          for (int hh = 0; hh < kNH; ++hh) {
            if (kb == 0) {
              // accumulator hh drained by the epilogues of both CTAs (the
              // first one is free while the second still drains)
              if (!mbar_wait_bounded(&acc_empty[hh], acc_ph ^ 1u, kGemmWaitNs)) {
                gemm_error(P, DRACO_ERR_TIMEOUT);
                ok = false;
                break;
              }
              tc_fence_after();
            }
            if (hh >= nh_live) continue;
            const uint32_t x_addr = x_addr0 + hh * kXBox;
            const uint32_t d = tmem + hh * kUmmaN;
            umma_bf16_pair(d, sdesc_sw128(x_addr), sdesc_sw128(a_addr), idesc, kb != 0);
#pragma unroll
            for (int kk = 1; kk < kBK / 16; ++kk)
              umma_bf16_pair(d, sdesc_sw128(x_addr + 32 * kk), sdesc_sw128(a_addr + 32 * kk), idesc, 1u);
          }
          if (!ok) break;
          umma_commit_pair(&empty_kb[rs.s]);
          rs.next(NS);
        }
        if (ok)
          for (int hh = 0; hh < kNH; ++hh) umma_commit_pair(&acc_full[hh]);
      }
      // every MMA issued has completed before the pair may free TMEM or exit
      umma_commit_local(&mma_done);
      if (!mbar_wait_bounded(&mma_done, 0u, kGemmWaitNs)) gemm_error(P, DRACO_ERR_TIMEOUT);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    // warp e owns TMEM lanes 32e..32e+31 = tokens 32e.. of this CTA's 128;
    // 32 x 32 blocks go through a staging tile in shared memory to TMA stores
    const int e = warp & 3;
    uint8_t* stage = smem + P.st_off + e * 2 * kStageBytes;
    const uint32_t acc_empty_leader[kNH] = {map_to_rank(&acc_empty[0], 0), map_to_rank(&acc_empty[1], 0)};
    uint32_t acc_ph = 0;
    int nst = 0;  // stores issued by this warp (alternating staging buffers)
    for (int i = 0, t; (t = tile_at(P, pair, i, npairs)) >= 0; ++i, acc_ph ^= 1u) {
      TileCursor c;
      c.at(P, t);
      const GemmProbDev& pr = P.prob[c.p];
      bool ok = true;
#pragma unroll 1
      for (int hh = 0; hh < kNH; ++hh) {
        if (!mbar_wait_bounded(&acc_full[hh], acc_ph, kGemmWaitNs)) {
          gemm_error(P, DRACO_ERR_TIMEOUT);
          ok = false;
          break;
        }
        tc_fence_after();
        const int tok0 = c.tb * kTileTok + hh * kUmmaM + (int)rank * kTokCta + 32 * e;
        const uint32_t tbase = tmem + ((uint32_t)(32 * e) << 16) + hh * kUmmaN;
        if (tok0 < c.m) {
#pragma unroll 1
          for (int cc = 0; cc < kUmmaN / 32; cc += 2) {
            uint32_t v0[32], v1[32];
            tmem_ld32_nowait(tbase + 32 * cc, v0);
            tmem_ld32_nowait(tbase + 32 * (cc + 1), v1);
            tmem_ld_wait(v0);
            reg_tie(v1);
            const int row0 = c.rp * kUmmaN + 32 * cc;
            if (pr.ymode == kYTma) {
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                // bf16: 4 staging tiles of 2 KB, fp32: 2 of 4 KB; wait until
                // the store that last used this tile has read it
                uint8_t* buf;
                if (pr.ydtype == DRACO_DTYPE_BF16) {
                  buf = stage + (nst & 3) * (kStageBytes / 2);
                  if (lane == 0) bulk_wait_read<3>();
                } else {
                  buf = stage + (nst & 1) * kStageBytes;
                  if (lane == 0) bulk_wait_read<1>();
                }
                __syncwarp();
                stage_rows(buf, pr.ydtype, lane, u ? v1 : v0);
                fence_async_smem();
                __syncwarp();
                if (lane == 0 && row0 + 32 * u < pr.n) {
                  tma_store_2d(&P.ymap[c.p], row0 + 32 * u, tok0, buf);
                }
                if (lane == 0) bulk_commit();
                ++nst;
              }
            } else {
              store_rows(pr, c.m, tok0 + lane, row0, v0);
              store_rows(pr, c.m, tok0 + lane, row0 + 32, v1);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc_empty_leader[hh]);
      }
      if (!ok) break;
    }
    if (lane == 0) bulk_wait_all();  // Y written before the kernel ends
  } else if (warp >= kDeqWarp0) {
    // ------------------------------------------------------------ dequant
    // warp dw: row tile dw (16 rows) of this CTA's 128-row B tile.  The packed
    // inputs of the next 64-k block are loaded before waiting for a free stage.
    const int dw = warp - kDeqWarp0;
    Ring ra;
    // blocks n (c0, being dequantized), n+1 (c1) and n+2 (c2, fetched now)
    DeqTile c0, c1;
    int kb0 = 0, kb1 = 0;
    bool h0 = c0.at(P, pair, 0, npairs, (int)rank, dw);
    c1 = c0;
    bool h1 = h0 && c1.advance(P, kb1, pair, npairs, (int)rank, dw);
    Packed p0, p1;
    if (h0) c0.template fetch<kLegacy>(kb0, lane, p0);
    if (h1) c1.template fetch<kLegacy>(kb1, lane, p1);
    while (h0) {
      DeqTile c2 = c1;
      int kb2 = kb1;
      const bool h2 = h1 && c2.advance(P, kb2, pair, npairs, (int)rank, dw);
      Packed p2;
      if (h2) c2.template fetch<kLegacy>(kb2, lane, p2);
      const DeqTile& cur = c0;
      const int kb = kb0;
      const Packed& pk = p0;
      if (!mbar_wait_bounded(&empty_kb[ra.s], ra.ph ^ 1u, kGemmWaitNs)) {
        gemm_error(P, DRACO_ERR_TIMEOUT);
        break;
      }
      uint8_t* tw = as + (size_t)ra.s * kATile + dw * 2048;
      if (cur.base) {
        if (cur.qt == kQ4_K) deq_q4k<false>(pk, kb & 3, lane, tw);
        else if (cur.qt == kQ5_K) deq_q4k<true>(pk, kb & 3, lane, tw);
        else if (cur.qt == kQ6_K) deq_q6k(pk, kb & 3, lane, tw);
        else if (!kLegacy || cur.qt == kQ8_0) deq_q80(pk, lane, tw);
        else deq_q4x(pk, lane, tw, cur.qt);
      } else {
        zero_rows16(tw, lane);  // row tile past n_rows
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(map_to_rank(&full_kb[ra.s], 0));
      ra.next(NS);
      c0 = c1, kb0 = kb1, h0 = h1, p0 = p1;
      c1 = c2, kb1 = kb2, h1 = h2, p1 = p2;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer no longer touches this CTA's barriers or shared memory
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Per device: opt the kernel into the whole dynamic shared-memory budget
// (the per-block opt-in limit less the kernel's static barriers) and count how
// many CTA pairs can be resident at once.
static int g_gemm_pairs[64] = {0};
static int g_gemm_dyn_smem[64] = {0};

static int gemm_max_pairs(int* dyn_smem, char* msg, size_t ml) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && g_gemm_pairs[dev] > 0) {
    *dyn_smem = g_gemm_dyn_smem[dev];
    return g_gemm_pairs[dev];
  }
  int optin = 0;
  cudaFuncAttributes fa;
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
      cudaFuncGetAttributes(&fa, gemm_kernel<true>) != cudaSuccess) {
    snprintf(msg, ml, "gemm: cannot query shared-memory limits");
    return -1;
  }
  const int dyn = optin - (int)fa.sharedSizeBytes;
  cudaError_t e = cudaFuncSetAttribute(gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemm: cudaFuncSetAttribute(%d bytes) failed: %s", dyn, cudaGetErrorString(e));
    return -1;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 256);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = dyn;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, gemm_kernel<true>, &cfg);
  if (e != cudaSuccess || n < 1) {
    snprintf(msg, ml, "gemm: no CTA pair fits on this device (%s)", cudaGetErrorString(e));
    return -1;
  }
  if (dev < 64) {
    g_gemm_pairs[dev] = n;
    g_gemm_dyn_smem[dev] = dyn;
  }
  *dyn_smem = dyn;
  return n;
}

// Balanced assignment of pair tiles to CTA pairs.  A tile of problem p costs
// nb_p * 4 k-blocks; the static order (tiles pair, pair + npairs, ...) leaves
// some pairs with an extra long tile at the end of a grouped launch.  The
// smallest per-pair capacity C for which first-fit-decreasing packs every tile
// (problems are already ordered longest first) gives the schedule; tiles of
// one problem go round-robin over the pairs that take them, so the pairs
// running at the same time share row pairs (weights) in L2.  Kept only when it
// shortens the longest pair.
static void build_schedule(GemmParams& P, int pairs) {
  P.sched_ok = 0;
  if (P.total_tiles > kMaxSched || pairs > kMaxPairs || P.total_tiles < 1) return;
  const int np = P.n_prob;
  int64_t cnt[kGemmMaxProblems], len[kGemmMaxProblems], total = 0;
  for (int p = 0; p < np; ++p) {
    cnt[p] = (int64_t)(P.prob[p].n_rg + 1) / 2 * P.prob[p].tblocks;
    len[p] = (int64_t)P.prob[p].nb * 4;
    total += cnt[p] * len[p];
  }
  // makespan of the static order
  int64_t strided = 0;
  for (int b = 0; b < pairs; ++b) {
    int64_t load = 0;
    for (int t = b; t < P.total_tiles; t += pairs) {
      int p = 0;
      for (int q = 1; q < np; ++q)
        if (t >= P.prob[q].tile0) p = q;
      load += len[p];
    }
    strided = std::max(strided, load);
  }
  static thread_local int quota[kMaxPairs][kGemmMaxProblems];
  auto pack = [&](int64_t cap) {
    int64_t load[kMaxPairs] = {0};
    for (int p = 0; p < np; ++p) {
      int64_t rem = cnt[p];
      for (int b = 0; b < pairs; ++b) {
        const int64_t fit = std::min(rem, (cap - load[b]) / len[p]);
        quota[b][p] = (int)std::max<int64_t>(fit, 0);
        load[b] += quota[b][p] * len[p];
        rem -= quota[b][p];
      }
      if (rem > 0) return false;
    }
    return true;
  };
  int64_t cap = (total + pairs - 1) / pairs;
  while (cap < strided && !pack(cap)) ++cap;
  if (cap >= strided) return;
  // lay out: pair b holds its tiles of problem 0, then 1, ...
  int pos[kMaxPairs][kGemmMaxProblems];
  int o = 0;
  for (int b = 0; b < pairs; ++b) {
    P.off[b] = (uint16_t)o;
    for (int p = 0; p < np; ++p) {
      pos[b][p] = o;
      o += quota[b][p];
    }
  }
  P.off[pairs] = (uint16_t)o;
  for (int p = 0; p < np; ++p) {
    int next = P.prob[p].tile0;
    int maxq = 0;
    for (int b = 0; b < pairs; ++b) maxq = std::max(maxq, quota[b][p]);
    for (int r = 0; r < maxq; ++r)
      for (int b = 0; b < pairs; ++b)
        if (quota[b][p] > r) P.sched[pos[b][p]++] = (uint16_t)next++;
  }
  P.sched_ok = 1;
}

int gemm_launch(const draco_gemm_problem* probs, int n, const int* rows, int* status, cudaStream_t st, char* msg,
                size_t ml) {
  if (n < 1 || n > kGemmMaxProblems) {
    snprintf(msg, ml, "gemm: need 1..%d problems, got %d", kGemmMaxProblems, n);
    return DRACO_ERR_ARG;
  }
  GemmParams P;
  memset(&P, 0, sizeof(P));
  auto enc = encode_fn();
  if (!enc) {
    snprintf(msg, ml, "gemm: cuTensorMapEncodeTiled unavailable");
    return DRACO_ERR_CUDA;
  }
  // problems with the longest K first: their tiles are the longest, and the
  // pairs that take them first finish with the short ones (fewer idle SMs at
  // the end of a grouped launch)
  int order[kGemmMaxProblems];
  for (int p = 0; p < n; ++p) order[p] = p;
  std::stable_sort(order, order + n, [&](int a, int b) { return probs[a].k > probs[b].k; });
  int tiles = 0;
  for (int p = 0; p < n; ++p) {
    const draco_gemm_problem& q = probs[order[p]];
    GemmProbDev& d = P.prob[p];
    const TiledGeom g = tiled_geom(q.qtype, q.n_rows, q.k);
    const int esize = q.ydtype == DRACO_DTYPE_BF16 ? 2 : 4;
    d.w = static_cast<const uint8_t*>(q.w);
    d.y = q.y;
    d.ldy = q.ldy;
    d.qt = q.qtype;
    d.ydtype = q.ydtype;
    d.m = (int)q.m;
    d.src = order[p];
    d.n = (int)q.n_rows;
    d.k = (int)q.k;
    d.nb = (int)g.nb;
    d.n_rg = (int)g.n_rg;
    d.n_tiles = (int)g.n_tiles;
    d.cb = g.cb;
    d.tblocks = (int)((q.m + kTileTok - 1) / kTileTok);
    d.vec = (reinterpret_cast<uintptr_t>(q.y) % 16 == 0) && ((q.ldy * esize) % 16 == 0);
    d.tile0 = tiles;
    tiles += (d.n_rg + 1) / 2 * d.tblocks;
    // X [m, k] bf16 row-major (row stride ldx elements): box 64 k x 128 tokens, 128-byte swizzle
    cuuint64_t gdim[2] = {(cuuint64_t)q.k, (cuuint64_t)q.m};
    cuuint64_t gstride[1] = {(cuuint64_t)q.ldx * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kTokCta};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&P.xmap[p], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(q.x), gdim, gstride, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      snprintf(msg, ml, "gemm: cuTensorMapEncodeTiled failed (%d) for problem %d", (int)r, order[p]);
      return DRACO_ERR_ARG;
    }
    // Y [m, n] (row stride ldy elements): 32 rows x 32 tokens per store,
    // swizzled like the staging tile; needs a 16-byte aligned base and stride
    d.ymode = kYDirect;
    if (d.vec) {
      cuuint64_t ydim[2] = {(cuuint64_t)q.n_rows, (cuuint64_t)q.m};
      cuuint64_t ystride[1] = {(cuuint64_t)q.ldy * esize};
      cuuint32_t ybox[2] = {32, 32};
      const bool bf = q.ydtype == DRACO_DTYPE_BF16;
      r = enc(&P.ymap[p], bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, q.y, ydim,
              ystride, ybox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              bf ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r == CUDA_SUCCESS) d.ymode = kYTma;
    }
  }
  P.n_prob = n;
  P.total_tiles = tiles;
  P.status = status;
  P.rows = rows;
  if (tiles == 0) return DRACO_OK;
  int dyn_smem = 0;
  const int max_pairs = gemm_max_pairs(&dyn_smem, msg, ml);
  if (max_pairs < 1) return DRACO_ERR_CUDA;
  // shared memory: epilogue staging (2 tiles per epilogue warp), dequantized
  // weight tiles, X boxes (two per k-block)
  const int budget = dyn_smem - 1024;  // less the slack for 1024-byte alignment
  const int staging = kEpiWarps * 2 * kStageBytes;
  P.ns = std::min(kMaxStages, (budget - staging) / (kNH * kXBox + kATile));
  if (P.ns < 2) {
    snprintf(msg, ml, "gemm: shared memory budget exceeded");
    return DRACO_ERR_ARG;
  }
  P.x_off = 0;
  P.a_off = P.ns * kNH * kXBox;
  P.st_off = P.a_off + P.ns * kATile;
  P.smem_bytes = P.st_off + staging + 1024;

  const int pairs = std::min(max_pairs, tiles);
  build_schedule(P, pairs);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = P.smem_bytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  bool legacy = false;
  for (int i = 0; i < P.n_prob; ++i) legacy |= is_q4x(P.prob[i].qt);
  cudaError_t e = legacy ? cudaLaunchKernelEx(&cfg, gemm_kernel<true>, P) : cudaLaunchKernelEx(&cfg, gemm_kernel<false>, P);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemm: launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

}  // namespace draco
