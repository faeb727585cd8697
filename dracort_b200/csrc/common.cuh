// common.cuh — shared device helpers for the sm_100a GGUF kernels:
// fp16 field loads, mbarrier / bulk-copy (TMA engine) PTX wrappers with
// bounded waits, the legacy m16n8k16 tensor-core MMA, and the byte geometry
// of the GGUF blocks and of the TILED device layout.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/draco_gguf.h"

namespace draco {

// ---------------------------------------------------------------------------
// GGUF block geometry (draco/format/gguf.py:75-87)
// ---------------------------------------------------------------------------
constexpr int kQ8_0 = DRACO_GGML_TYPE_Q8_0;
constexpr int kQ4_0 = DRACO_GGML_TYPE_Q4_0;
constexpr int kQ4_1 = DRACO_GGML_TYPE_Q4_1;
constexpr int kQ5_0 = DRACO_GGML_TYPE_Q5_0;
constexpr int kQ5_1 = DRACO_GGML_TYPE_Q5_1;
// the 32-element types with 4 (+1) bit quants: Q4_0, Q4_1, Q5_0, Q5_1
__host__ __device__ inline bool is_q4x(int qt) { return qt == kQ4_0 || qt == kQ4_1 || qt == kQ5_0 || qt == kQ5_1; }
constexpr int kQ4_K = DRACO_GGML_TYPE_Q4_K;
constexpr int kQ5_K = DRACO_GGML_TYPE_Q5_K;
constexpr int kQ6_K = DRACO_GGML_TYPE_Q6_K;

__host__ __device__ inline int block_size_of(int qt) { return (qt == kQ8_0 || is_q4x(qt)) ? 32 : 256; }
__host__ __device__ inline int block_bytes_of(int qt) {
  return qt == kQ8_0 ? 34 : qt == kQ4_K ? 144 : qt == kQ5_K ? 176 : qt == kQ6_K ? 210 :
         qt == kQ4_0 ? 18 : qt == kQ4_1 ? 20 : qt == kQ5_0 ? 22 : 24;
}

// Field offsets inside one Q6_K block for the two byte orders.  GGUF (the
// reference, gguf.py:470-474): d@0 ql@2 qh@130 sc@194.  GGUF_DLAST (llama.cpp
// files): ql@0 qh@128 sc@192 d@208.
struct Q6Fields { int d, ql, qh, sc; };
__host__ __device__ inline Q6Fields q6_fields(int layout) {
  if (layout == DRACO_LAYOUT_GGUF_DLAST) return {208, 0, 128, 192};
  return {0, 2, 130, 194};
}

// ---------------------------------------------------------------------------
// TILED layout.  A weight [n_rows, k] is cut into 16-row x 256-element
// "chunks".  Chunks of 8 consecutive row tiles that share one 256-element
// super-block form a "slab" (128 rows x 256 k); slabs are stored row-group
// major: [row group][super-block][row tile in group][chunk bytes].  Inside a
// chunk the fields of the 16 rows are regrouped so that lane (g = lane/4,
// t = lane%4) of a warp fetches everything it needs for rows g and g+8 with
// 16-byte shared-memory loads in the order the m16n8k16 MMA fragments use.
// ---------------------------------------------------------------------------
constexpr int kChunkRows = 16;
constexpr int kSuperElems = 256;
constexpr int kGroupTiles = 8;  // row tiles per slab

__host__ __device__ inline int chunk_bytes_of(int qt) {
  return kChunkRows * (kSuperElems / block_size_of(qt)) * block_bytes_of(qt);
}

struct TiledGeom {
  int qt;
  int64_t n_rows, k;
  int64_t n_tiles;  // ceil(n_rows / 16)
  int64_t nb;       // ceil(k / 256) super-blocks per row (k padded with zero blocks)
  int64_t n_rg;     // ceil(n_tiles / 8)
  int cb;           // chunk bytes
};

__host__ __device__ inline TiledGeom tiled_geom(int qt, int64_t n_rows, int64_t k) {
  TiledGeom g;
  g.qt = qt;
  g.n_rows = n_rows;
  g.k = k;
  g.n_tiles = (n_rows + kChunkRows - 1) / kChunkRows;
  g.nb = (k + kSuperElems - 1) / kSuperElems;
  g.n_rg = (g.n_tiles + kGroupTiles - 1) / kGroupTiles;
  g.cb = chunk_bytes_of(qt);
  return g;
}
__host__ __device__ inline int64_t tiled_total_bytes(const TiledGeom& g) {
  return g.n_tiles * g.nb * (int64_t)g.cb;
}
__host__ __device__ inline int rg_tiles(const TiledGeom& g, int64_t rg) {
  int64_t r = g.n_tiles - rg * kGroupTiles;
  return (int)(r < kGroupTiles ? r : kGroupTiles);
}
// Byte offset of the slab (row group rg, super-block j).
__host__ __device__ inline int64_t slab_offset(const TiledGeom& g, int64_t rg, int64_t j) {
  return rg * (int64_t)kGroupTiles * g.nb * g.cb + j * (int64_t)rg_tiles(g, rg) * g.cb;
}
// Byte offset of the chunk holding row tile `tile`, super-block j.
__host__ __device__ inline int64_t chunk_offset(const TiledGeom& g, int64_t tile, int64_t j) {
  int64_t rg = tile / kGroupTiles;
  return slab_offset(g, rg, j) + (tile % kGroupTiles) * (int64_t)g.cb;
}

// Position inside a chunk of byte `p` of a field of row `rr` (0..15).
// Q4_K fields: qs[128] -> [0,2048), scales[12] -> [2048,2240), d,dmin -> [2240,2304).
__host__ __device__ inline int q4k_qs_pos(int rr, int p) {
  int g = rr & 7, hi = rr >> 3;
  int q = p >> 5, u = p & 31, half = u >> 4, v = u & 15, t = v >> 2, bw = v & 3;
  int lane = 4 * g + t;
  return 512 * q + 16 * lane + 4 * (2 * hi + half) + bw;
}
__host__ __device__ inline int q4k_sc_pos(int rr, int s) { return 2048 + 24 * (rr & 7) + 12 * (rr >> 3) + s; }
__host__ __device__ inline int q4k_d_pos(int rr) { return 2240 + 8 * (rr & 7) + 4 * (rr >> 3); }  // +2 = dmin

// Q5_K: qs as Q4_K -> [0,2048); qh[32] -> [2048,2560), in the same lane units
// as one group of qs (byte u of row rr where qs byte u of a group sits), so a
// lane's 16-byte qh unit holds the fifth bits of all its quants;
// scales[12] -> [2560,2752), d,dmin -> [2752,2816).
__host__ __device__ inline int q5k_qh_pos(int rr, int u) { return 2048 + q4k_qs_pos(rr, u); }
__host__ __device__ inline int q5k_sc_pos(int rr, int s) { return 2560 + 24 * (rr & 7) + 12 * (rr >> 3) + s; }
__host__ __device__ inline int q5k_d_pos(int rr) { return 2752 + 8 * (rr & 7) + 4 * (rr >> 3); }  // +2 = dmin

// Q6_K fields: ql[128]/qh[64] -> [0,3072), sc[16] -> [3072,3328), d -> [3328,3360).
// Lane data: 24 words; group nu = 2*n + is (n = half of the super-block,
// is = 16-element half of l), word = 6*nu + 3*hi + {0: ql low l, 1: ql l+32, 2: qh}.
__host__ __device__ inline int q6k_word_pos(int lane, int w, int bw) {
  return 512 * (w >> 2) + 16 * lane + 4 * (w & 3) + bw;
}
__host__ __device__ inline int q6k_ql_pos(int rr, int p) {
  int g = rr & 7, hi = rr >> 3;
  int n = p >> 6, u = p & 63, which = u >> 5, l = u & 31, is = l >> 4, v = l & 15;
  int t = v >> 2, bw = v & 3;
  int nu = 2 * n + is;
  return q6k_word_pos(4 * g + t, 6 * nu + 3 * hi + which, bw);
}
__host__ __device__ inline int q6k_qh_pos(int rr, int p) {
  int g = rr & 7, hi = rr >> 3;
  int n = p >> 5, l = p & 31, is = l >> 4, v = l & 15;
  int t = v >> 2, bw = v & 3;
  int nu = 2 * n + is;
  return q6k_word_pos(4 * g + t, 6 * nu + 3 * hi + 2, bw);
}
__host__ __device__ inline int q6k_sc_pos(int rr, int s) { return 3072 + 32 * (rr & 7) + 16 * (rr >> 3) + s; }
__host__ __device__ inline int q6k_d_pos(int rr) { return 3328 + 4 * (rr & 7) + 2 * (rr >> 3); }

// Q4_0 / Q4_1 / Q5_0 / Q5_1 (8 blocks of 32 per super-block, block b).
// qs[16] -> [0,2048): the 16-byte unit of lane (g, t) for block pair bp holds
//   the words (row g, block 2bp), (row g+8, block 2bp), (row g, block 2bp+1),
//   (row g+8, block 2bp+1), each qs bytes 4t..4t+3 of that block: their low
//   nibbles are elements 4t..4t+3, their high nibbles 16+4t..16+4t+3;
// Q5_x: qh (32 bits per block, bit e = element e) -> 512 B at 2048, per
//   (g, row half, block) one word, read whole by the four lanes of a quad;
// d (fp16 per block) -> 256 B, m (Q4_1 / Q5_1, fp16 per block) -> 256 B, per
//   (g, row half, block).
struct Q4xFields { int qh, d, m; };
__host__ __device__ inline Q4xFields q4x_fields(int qt) {
  const bool h = qt == kQ5_0 || qt == kQ5_1;
  const int d = h ? 2560 : 2048;
  return {h ? 2048 : -1, d, (qt == kQ4_1 || qt == kQ5_1) ? d + 256 : -1};
}
__host__ __device__ inline int q4x_qs_pos(int rr, int b, int p) {
  const int g = rr & 7, hi = rr >> 3, t = p >> 2, bw = p & 3;
  return 512 * (b >> 1) + 16 * (4 * g + t) + 4 * (2 * (b & 1) + hi) + bw;
}
__host__ __device__ inline int q4x_word_pos(int base, int rr, int b) { return base + 64 * (rr & 7) + 32 * (rr >> 3) + 4 * b; }
__host__ __device__ inline int q4x_half_pos(int base, int rr, int b) { return base + 32 * (rr & 7) + 16 * (rr >> 3) + 2 * b; }

// Q8_0 (8 blocks per super-block, block b): qs[32] -> [0,4096), d -> [4096,4352).
__host__ __device__ inline int q80_qs_pos(int rr, int b, int p) {
  int g = rr & 7, hi = rr >> 3;
  int half = p >> 4, v = p & 15, t = v >> 2, bw = v & 3;
  return 512 * b + 16 * (4 * g + t) + 4 * (2 * hi + half) + bw;
}
__host__ __device__ inline int q80_d_pos(int rr, int b) { return 4096 + 32 * (rr & 7) + 16 * (rr >> 3) + 2 * b; }

// ---------------------------------------------------------------------------
// scalar helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits) {
  return __half2float(__ushort_as_half((unsigned short)(bits & 0xFFFFu)));
}
__device__ __forceinline__ float ld_f16(const uint8_t* p) {
  uint32_t b = (uint32_t)p[0] | ((uint32_t)p[1] << 8);
  return f16_bits_to_f32(b);
}
// 6-bit (scale, min) pair j of a Q4_K block's 12 packed bytes
// (gguf.py:436-442).
__device__ __forceinline__ void q4k_scale_min(const uint8_t* sc, int j, int& s, int& m) {
  if (j < 4) {
    s = sc[j] & 63;
    m = sc[j + 4] & 63;
  } else {
    s = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
    m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (executed by the TMA engine)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// 32-bit flag store / load ordered at system scope (flags that other GPUs
// write into this GPU's memory, or this GPU into theirs, over NVLink).
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase with the given parity to complete.  Gives up after
// `limit_ns` nanoseconds and returns false (the caller records an error and
// unwinds instead of hanging the GPU).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}
// 1-D bulk copy global -> shared, completion signalled on `bar` as tx bytes.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch of a contiguous global range by the TMA engine (no completion
// to wait for).  Address 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the preceding kernel in the stream
// (no-op when the launch did not use the attribute).
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tensor-core MMA m16n8k16, f16 x f16 -> f32
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f), "f"(0.f), "f"(0.f), "f"(0.f));
}
__device__ __forceinline__ void mma_f16_16816_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                  uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// silu(g) * u in fp32 with CUDA's expf (the SwiGLU product of a gated MLP)
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  return (a & mask) | orv;
}

}  // namespace draco
