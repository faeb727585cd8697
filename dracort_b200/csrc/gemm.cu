// gemm.cu — prefill dequant-GEMM  Y[M, N] = X[M, K] (bf16) . dequant(W)[N, K]^T
// with W in the TILED GGUF layout (Q8_0 / Q4_K / Q6_K), fp32 accumulation in
// tensor memory, Y in bf16 or fp32.
//
// Replaces the reference's prefill linear: executor._linear
// (draco/runtime/cpu/executor.py:47-79) -> GenericGemmKernel.matmul_f32
// (draco/runtime/cpu/kernels/generic.py:32-33) on gguf._dequantize's fp32
// cache (draco/format/gguf.py:272-497), at M = prompt length.
//
// Design (B200, tensor-bound), persistent, one CTA (16 warps) per SM:
//  * tile = 128 weight rows (one TILED row group) x 512 tokens; the K loop
//    runs in 64-element blocks (one 128-byte swizzle atom of bf16).
//  * warp 0 (one lane): TMA loads of the X tiles (cp.async.bulk.tensor.2d,
//    128-byte swizzle, 256 tokens x 64 k per box) and 1-D bulk copies of the
//    packed weight slabs (128 rows x 256 k, contiguous in the TILED layout).
//  * warps 8-15 (dequant): expand each 64-k block of the packed slab into a
//    bf16 A tile (128 x 64, K-major, 128-byte swizzle) in shared memory; each
//    value is the fp32 dequantized weight (same operations as gguf._dequantize)
//    rounded to bf16.  fence.proxy.async makes the stores visible to the
//    tensor cores.
//  * warp 1: allocates 512 TMEM columns; one lane issues
//    tcgen05.mma.cta_group::1.kind::f16 (M128 N256 K16, bf16 x bf16 -> fp32)
//    into two 256-column accumulators (tokens 0-255 and 256-511 of the tile)
//    and signals stage reuse with tcgen05.commit.
//  * warps 4-7 (epilogue): tcgen05.ld the accumulators (warp w reads TMEM lanes
//    32(w%4)..+31 = weight rows), convert and store Y[token][row].
//  * every wait is bounded; on a timeout the kernel records DRACO_ERR_TIMEOUT,
//    unwinds, and still frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace draco {

constexpr int kGemmMaxProblems = 4;
constexpr int kBM = 128;                      // weight rows per tile
constexpr int kHalf = 256;                    // tokens per accumulator (UMMA N)
constexpr int kNH = 2;                        // accumulators per tile
constexpr int kBK = 64;                       // k per block
constexpr int kXBox = kHalf * kBK * 2;        // 32 KB: one TMA box of X
constexpr int kATile = kBM * kBK * 2;         // 16 KB: one dequantized A tile
constexpr int kGemmThreads = 16 * 32;
constexpr int kDeqWarp0 = 8, kDeqWarps = 8;
constexpr int kEpiWarp0 = 4;
constexpr int kMaxXStages = 4, kMaxWpStages = 2, kAStages = 2;
constexpr uint64_t kGemmWaitNs = 4000000000ull;  // 4 s

struct GemmProbDev {
  const uint8_t* w;
  void* y;
  int64_t ldy;
  int qt, ydtype, m, n, k, nb, n_rg, n_tiles, cb, tblocks, tile0, pad_;
};

struct __align__(64) GemmParams {
  CUtensorMap tmap[kGemmMaxProblems];
  GemmProbDev prob[kGemmMaxProblems];
  int* status;
  int n_prob, total_tiles;
  int nx, nwp, wp_stage;
  int x_off, a_off, wp_off, smem_bytes;
};

// ---------------------------------------------------------------------------
// PTX wrappers (tcgen05, TMA tensor loads, proxy fences)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
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

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
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

// byte offset of 16-byte chunk c (k = 8c..8c+7) of row r in a 128-byte-swizzled
// K-major tile with 128-byte rows
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// exact float of byte i (unsigned) of w
__device__ __forceinline__ float gbyte_f(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)i)) - 8388608.f;
}
// exact float of byte i of w read as int8
__device__ __forceinline__ float gsbyte_f(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w ^ 0x80808080u, 0x4B000000u, 0x7440u | (uint32_t)i)) - 8388736.f;
}
__device__ __forceinline__ uint32_t gbyte(uint32_t w, int i) { return __byte_perm(w, 0u, 0x4440u | (uint32_t)i); }
__device__ __forceinline__ uint32_t lds32_g(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
// exact float of a small non-negative integer (< 2^23)
__device__ __forceinline__ float u2f_g(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.f; }

// ---------------------------------------------------------------------------
// dequantization of one 64-k block of a packed slab into a bf16 A tile.
// 256 threads: thread dt -> row r = dt / 2, half h = dt % 2.  Every value is
// fp32 exactly as gguf._dequantize computes it, then rounded to bf16.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_chunk(uint8_t* a, int r, int c, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(a + sw128(r, c)) =
      make_uint4(bf16x2(v[0], v[1]), bf16x2(v[2], v[3]), bf16x2(v[4], v[5]), bf16x2(v[6], v[7]));
}
__device__ __forceinline__ void zero_chunk(uint8_t* a, int r, int c) {
  *reinterpret_cast<uint4*>(a + sw128(r, c)) = make_uint4(0, 0, 0, 0);
}

// Q4_K: k-block q of the super-block = qs bytes 32q..32q+31 of each row; low
// nibbles are k 0-31 (sub-block 2q), high nibbles k 32-63 (sub-block 2q+1).
// Half h takes bytes 16h..16h+15: output chunks 2h, 2h+1 (low) and 4+2h, 5+2h (high).
__device__ __forceinline__ void dequant_q4k(const uint8_t* slab, int cb, int q, int r, int h, uint8_t* a) {
  const uint8_t* ch = slab + (r >> 4) * cb;
  const int rr = r & 15, g = rr & 7, hi = rr >> 3;
  const uint8_t* sp = ch + 2048 + 24 * g + 12 * hi;
  const uint32_t A = lds32_g(sp), Bw = lds32_g(sp + 4), C = lds32_g(sp + 8);
  const uint32_t dd = lds32_g(ch + 2240 + 8 * g + 4 * hi);
  const float d = f16_bits_to_f32(dd), dmin = f16_bits_to_f32(dd >> 16);
  float ds[2], dm[2];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int j = 2 * q + s;
    uint32_t sc, m;
    if (j < 4) {
      sc = gbyte(A, j) & 63u;
      m = gbyte(Bw, j) & 63u;
    } else {
      const uint32_t c = gbyte(C, j - 4);
      sc = (c & 15u) | ((gbyte(A, j - 4) >> 6) << 4);
      m = (c >> 4) | ((gbyte(Bw, j - 4) >> 6) << 4);
    }
    ds[s] = __fmul_rn(d, (float)sc);
    dm[s] = __fmul_rn(dmin, (float)m);
  }
  uint32_t w[4];
#pragma unroll
  for (int tp = 0; tp < 4; ++tp) w[tp] = lds32_g(ch + 512 * q + 16 * (4 * g + tp) + 4 * (2 * hi + h));
#pragma unroll
  for (int s = 0; s < 2; ++s)      // low / high nibbles
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {  // two chunks of 8 values
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t word = w[2 * cc + (i >> 2)];
        const uint32_t nib = s ? ((word >> (8 * (i & 3) + 4)) & 15u) : ((word >> (8 * (i & 3))) & 15u);
        v[i] = __fsub_rn(__fmul_rn(ds[s], u2f_g(nib)), dm[s]);
      }
      store_chunk(a, r, 4 * s + 2 * h + cc, v);
    }
}

// Q6_K: k-block q = elements 64q..64q+63: half n = q / 2, 32-element groups
// i = 2(q%2) + h (one per thread), l = 0..31 -> chunks 4h + l/8.
__device__ __forceinline__ void dequant_q6k(const uint8_t* slab, int cb, int q, int r, int h, uint8_t* a) {
  const uint8_t* ch = slab + (r >> 4) * cb;
  const int rr = r & 15, g = rr & 7, hi = rr >> 3;
  const int n = q >> 1, i = 2 * (q & 1) + h;
  const float d = ld_f16(ch + 3328 + 4 * g + 2 * hi);
  const uint8_t* scp = ch + 3072 + 32 * g + 16 * hi;
#pragma unroll
  for (int is = 0; is < 2; ++is) {  // 16-element halves: sub-block 8n + 2i + is
    const float dl = __fmul_rn(d, (float)(int8_t)scp[8 * n + 2 * i + is]);
    const int nu = 2 * n + is;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      float v[8];
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        const int t = 2 * cc + tt;  // l = 16 is + 4 t .. +3
        const uint8_t* lb = ch + 16 * (4 * g + t);
        const int wbase = 6 * nu + 3 * hi;
        const uint32_t ql = lds32_g(lb + 512 * ((wbase + (i & 1)) >> 2) + 4 * ((wbase + (i & 1)) & 3));
        const uint32_t qh = lds32_g(lb + 512 * ((wbase + 2) >> 2) + 4 * ((wbase + 2) & 3));
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t lo = (i < 2) ? ((ql >> (8 * b)) & 15u) : ((ql >> (8 * b + 4)) & 15u);
          const uint32_t hb = (qh >> (8 * b + 2 * i)) & 3u;
          v[4 * tt + b] = __fmul_rn(dl, (float)((int)(lo | (hb << 4)) - 32));
        }
      }
      store_chunk(a, r, 4 * h + 2 * is + cc, v);
    }
  }
}

// Q8_0: k-block q = blocks 2q, 2q+1 of the super-block; thread half h takes block 2q+h.
__device__ __forceinline__ void dequant_q80(const uint8_t* slab, int cb, int q, int r, int h, uint8_t* a) {
  const uint8_t* ch = slab + (r >> 4) * cb;
  const int rr = r & 15, g = rr & 7, hi = rr >> 3;
  const int b = 2 * q + h;
  const float d = ld_f16(ch + 4096 + 32 * g + 16 * hi + 2 * b);
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {  // k = 8cc..8cc+7 of the block
    const int half = cc >> 1, t0 = 2 * (cc & 1);
    float v[8];
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
      const uint32_t w = lds32_g(ch + 512 * b + 16 * (4 * g + t0 + tt) + 4 * (2 * hi + half));
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * tt + i] = __fmul_rn(gsbyte_f(w, i), d);
    }
    store_chunk(a, r, 4 * h + cc, v);
  }
}

__device__ __forceinline__ void gemm_error(const GemmParams& P, int code) {
  if (P.status) atomicCAS(P.status, 0, code);
}

struct TileCursor {
  int p, rg, tb, nkb;
  __device__ void at(const GemmParams& P, int t) {
    p = 0;
    for (int q = 1; q < P.n_prob; ++q)
      if (t >= P.prob[q].tile0) p = q;
    const int local = t - P.prob[p].tile0;
    rg = local / P.prob[p].tblocks;
    tb = local - rg * P.prob[p].tblocks;
    nkb = P.prob[p].nb * 4;
  }
};

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_x[kMaxXStages], empty_x[kMaxXStages];
  __shared__ __align__(8) uint64_t full_wp[kMaxWpStages], empty_wp[kMaxWpStages];
  __shared__ __align__(8) uint64_t full_a[kAStages], empty_a[kAStages];
  __shared__ __align__(8) uint64_t acc_full[kNH], acc_empty[kNH];
  __shared__ uint32_t s_tmem;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NX = P.nx, NWP = P.nwp;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NX; ++i) {
      mbar_init(&full_x[i], 1);
      mbar_init(&empty_x[i], 1);
    }
    for (int i = 0; i < NWP; ++i) {
      mbar_init(&full_wp[i], 1);
      mbar_init(&empty_wp[i], kDeqWarps);
    }
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(&full_a[i], kDeqWarps);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < kNH; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  grid_dependency_wait();  // X may be written by the preceding kernel

  uint8_t* xs = smem + P.x_off;
  uint8_t* as = smem + P.a_off;
  uint8_t* wps = smem + P.wp_off;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int ix = 0, iw = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < P.total_tiles && ok; t += gridDim.x) {
        TileCursor c;
        c.at(P, t);
        const GemmProbDev& pr = P.prob[c.p];
        const TiledGeom geo = tiled_geom(pr.qt, pr.n, pr.k);
        const uint32_t slab_bytes = (uint32_t)(rg_tiles(geo, c.rg) * pr.cb);
        for (int kb = 0; kb < c.nkb && ok; ++kb) {
          if ((kb & 3) == 0) {
            const int s = iw % NWP;
            const uint32_t ph = (uint32_t)((iw / NWP) & 1);
            if (!mbar_wait_bounded(&empty_wp[s], ph ^ 1u, kGemmWaitNs)) {
              gemm_error(P, DRACO_ERR_TIMEOUT);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full_wp[s], slab_bytes);
            bulk_g2s(wps + (size_t)s * P.wp_stage, pr.w + slab_offset(geo, c.rg, kb >> 2), slab_bytes, &full_wp[s]);
            ++iw;
          }
#pragma unroll 1
          for (int hh = 0; hh < kNH; ++hh) {
            const int s = ix % NX;
            const uint32_t ph = (uint32_t)((ix / NX) & 1);
            if (!mbar_wait_bounded(&empty_x[s], ph ^ 1u, kGemmWaitNs)) {
              gemm_error(P, DRACO_ERR_TIMEOUT);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full_x[s], kXBox);
            tma_load_2d(xs + (size_t)s * kXBox, &P.tmap[c.p], kb * kBK, (c.tb * kNH + hh) * kHalf, &full_x[s]);
            ++ix;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kBM, kHalf);
      int ix = 0, ia = 0, it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < P.total_tiles && ok; t += gridDim.x, ++it) {
        TileCursor c;
        c.at(P, t);
        const uint32_t acc_ph = (uint32_t)(it & 1);
        for (int hh = 0; hh < kNH && ok; ++hh)
          if (!mbar_wait_bounded(&acc_empty[hh], acc_ph ^ 1u, kGemmWaitNs)) {
            gemm_error(P, DRACO_ERR_TIMEOUT);
            ok = false;
          }
        tc_fence_after();
        for (int kb = 0; kb < c.nkb && ok; ++kb) {
          const int sa = ia % kAStages;
          if (!mbar_wait_bounded(&full_a[sa], (uint32_t)((ia / kAStages) & 1), kGemmWaitNs)) {
            gemm_error(P, DRACO_ERR_TIMEOUT);
            ok = false;
            break;
          }
          const uint32_t a_addr = smem_u32(as + (size_t)sa * kATile);
#pragma unroll 1
          for (int hh = 0; hh < kNH; ++hh) {
            const int sx = ix % NX;
            if (!mbar_wait_bounded(&full_x[sx], (uint32_t)((ix / NX) & 1), kGemmWaitNs)) {
              gemm_error(P, DRACO_ERR_TIMEOUT);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b_addr = smem_u32(xs + (size_t)sx * kXBox);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_bf16(tmem + hh * kHalf, sdesc_sw128(a_addr + 32 * kk), sdesc_sw128(b_addr + 32 * kk), idesc,
                        (kb | kk) != 0);
            umma_commit(&empty_x[sx]);
            ++ix;
          }
          umma_commit(&empty_a[sa]);
          ++ia;
        }
        for (int hh = 0; hh < kNH; ++hh) umma_commit(&acc_full[hh]);
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------ epilogue
    const int e = warp & 3;  // TMEM lane quarter
    int it = 0;
    for (int t = blockIdx.x; t < P.total_tiles; t += gridDim.x, ++it) {
      TileCursor c;
      c.at(P, t);
      const GemmProbDev& pr = P.prob[c.p];
      const int row = c.rg * kBM + 32 * e + lane;
      bool ok = true;
#pragma unroll 1
      for (int hh = 0; hh < kNH; ++hh) {
        if (!mbar_wait_bounded(&acc_full[hh], (uint32_t)(it & 1), kGemmWaitNs)) {
          gemm_error(P, DRACO_ERR_TIMEOUT);
          ok = false;
          break;
        }
        tc_fence_after();
        const int tok0 = (c.tb * kNH + hh) * kHalf;
#pragma unroll 1
        for (int cc = 0; cc < kHalf / 32; ++cc) {
          uint32_t v[32];
          tmem_ld32(tmem + ((uint32_t)(32 * e) << 16) + hh * kHalf + 32 * cc, v);
          if (row < pr.n) {
            const int tb = tok0 + 32 * cc;
            if (pr.ydtype == DRACO_DTYPE_BF16) {
              __nv_bfloat16* y = static_cast<__nv_bfloat16*>(pr.y) + row;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (tb + j < pr.m) y[(int64_t)(tb + j) * pr.ldy] = __float2bfloat16_rn(__uint_as_float(v[j]));
            } else {
              float* y = static_cast<float*>(pr.y) + row;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (tb + j < pr.m) y[(int64_t)(tb + j) * pr.ldy] = __uint_as_float(v[j]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0)
        for (int hh = 0; hh < kNH; ++hh) mbar_arrive(&acc_empty[hh]);
      if (!ok) break;
    }
  } else if (warp >= kDeqWarp0) {
    // ------------------------------------------------------------ dequant
    const int dt = threadIdx.x - kDeqWarp0 * 32;
    const int r = dt >> 1, h = dt & 1;
    int iw = 0, ia = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < P.total_tiles && ok; t += gridDim.x) {
      TileCursor c;
      c.at(P, t);
      const GemmProbDev& pr = P.prob[c.p];
      const TiledGeom geo = tiled_geom(pr.qt, pr.n, pr.k);
      const int nrows = rg_tiles(geo, c.rg) * kChunkRows;
      for (int sb = 0; sb < pr.nb && ok; ++sb) {
        const int sw = iw % NWP;
        if (!mbar_wait_bounded(&full_wp[sw], (uint32_t)((iw / NWP) & 1), kGemmWaitNs)) {
          gemm_error(P, DRACO_ERR_TIMEOUT);
          ok = false;
          break;
        }
        const uint8_t* slab = wps + (size_t)sw * P.wp_stage;
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          const int sa = ia % kAStages;
          if (!mbar_wait_bounded(&empty_a[sa], (uint32_t)(((ia / kAStages) & 1) ^ 1), kGemmWaitNs)) {
            gemm_error(P, DRACO_ERR_TIMEOUT);
            ok = false;
            break;
          }
          uint8_t* a = as + (size_t)sa * kATile;
          if (r < nrows) {
            if (pr.qt == kQ4_K) dequant_q4k(slab, pr.cb, q, r, h, a);
            else if (pr.qt == kQ6_K) dequant_q6k(slab, pr.cb, q, r, h, a);
            else dequant_q80(slab, pr.cb, q, r, h, a);
          } else if (pr.qt == kQ4_K) {  // rows past n_rows: zeros in this thread's chunks
            zero_chunk(a, r, 2 * h);
            zero_chunk(a, r, 2 * h + 1);
            zero_chunk(a, r, 4 + 2 * h);
            zero_chunk(a, r, 5 + 2 * h);
          } else {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) zero_chunk(a, r, 4 * h + cc);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full_a[sa]);
          ++ia;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_wp[sw]);
        ++iw;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
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

int gemm_launch(const draco_gemm_problem* probs, int n, int* status, cudaStream_t st, char* msg, size_t ml) {
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
  int tiles = 0, max_slab = 0;
  for (int p = 0; p < n; ++p) {
    const draco_gemm_problem& q = probs[p];
    GemmProbDev& d = P.prob[p];
    const TiledGeom g = tiled_geom(q.qtype, q.n_rows, q.k);
    d.w = static_cast<const uint8_t*>(q.w);
    d.y = q.y;
    d.ldy = q.ldy;
    d.qt = q.qtype;
    d.ydtype = q.ydtype;
    d.m = (int)q.m;
    d.n = (int)q.n_rows;
    d.k = (int)q.k;
    d.nb = (int)g.nb;
    d.n_rg = (int)g.n_rg;
    d.n_tiles = (int)g.n_tiles;
    d.cb = g.cb;
    d.tblocks = (int)((q.m + kNH * kHalf - 1) / (kNH * kHalf));
    d.tile0 = tiles;
    tiles += d.n_rg * d.tblocks;
    max_slab = std::max(max_slab, kGroupTiles * g.cb);
    // X [m, k] bf16 row-major (row stride ldx elements): box 64 k x 256 tokens, 128-byte swizzle
    cuuint64_t gdim[2] = {(cuuint64_t)q.k, (cuuint64_t)q.m};
    cuuint64_t gstride[1] = {(cuuint64_t)q.ldx * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kHalf};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&P.tmap[p], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(q.x), gdim, gstride, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      snprintf(msg, ml, "gemm: cuTensorMapEncodeTiled failed (%d) for problem %d", (int)r, p);
      return DRACO_ERR_ARG;
    }
  }
  P.n_prob = n;
  P.total_tiles = tiles;
  P.status = status;
  if (tiles == 0) return DRACO_OK;
  P.wp_stage = (max_slab + 127) & ~127;
  P.nwp = 2;
  const int budget = 220 * 1024;
  const int fixed = kAStages * kATile + P.nwp * P.wp_stage + 1024;  // + alignment slack
  P.nx = std::min(kMaxXStages, (budget - fixed) / kXBox);
  if (P.nx < 2) {
    snprintf(msg, ml, "gemm: shared memory budget exceeded");
    return DRACO_ERR_ARG;
  }
  P.x_off = 0;
  P.a_off = P.nx * kXBox;
  P.wp_off = P.a_off + kAStages * kATile;
  P.smem_bytes = P.wp_off + P.nwp * P.wp_stage + 1024;

  static int attr_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && attr_set[dev] < P.smem_bytes) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P.smem_bytes);
    if (e != cudaSuccess) {
      snprintf(msg, ml, "gemm: cudaFuncSetAttribute(%d bytes) failed: %s", P.smem_bytes, cudaGetErrorString(e));
      return DRACO_ERR_CUDA;
    }
    attr_set[dev] = P.smem_bytes;
  }
  const int grid = std::min(device_sm_count(), tiles);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = P.smem_bytes;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_kernel, P);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "gemm: launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

}  // namespace draco
