// dequant.cu — GGUF block dequantization (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K,
// Q5_K, Q6_K) to fp32 / bf16,
// and the GGUF -> TILED repack.
//
// Parity target: draco/format/gguf.py:_dequantize.  Each output element is
// produced with the same single fp32 rounding the reference performs:
//   Q8_0 (gguf.py:300-303): q * d                       (exact)
//   Q4_K (gguf.py:425-456): (d*sc)*q - (dmin*m)          (products exact, one
//                                                         rounding in the subtract)
//   Q5_K (gguf.py:425-468): the same with q = nibble + 16 * fifth bit (the
//                           reference forms it in float64: the same value)
//   Q6_K (gguf.py:470-495): (d*sc) * (q6 - 32)           (d*sc exact, one rounding)
//   Q4_0 / Q5_0 (gguf.py:310-316, 326-349): (q - 8) * d, (q5 - 16) * d   (exact)
//   Q4_1 / Q5_1 (gguf.py:318-324, 326-353): q * d + m    (product exact, one
//                                                         rounding in the add)
// The multiplies and the subtract are written with explicit _rn intrinsics so
// that no FMA contraction can change a bit.
#include "common.cuh"
#include "internal.h"

namespace draco {

// ---------------------------------------------------------------------------
// field accessors: one GGUF block (row, super-block) in either byte layout
// ---------------------------------------------------------------------------
struct RawQ4K {
  const uint8_t* blk;
  __device__ RawQ4K(const uint8_t* base, int64_t row, int64_t k, int64_t sb) {
    blk = base + row * (k / 256) * 144 + sb * 144;
  }
  __device__ float d() const { return ld_f16(blk); }
  __device__ float dmin() const { return ld_f16(blk + 2); }
  __device__ uint8_t sc(int s) const { return blk[4 + s]; }
  __device__ uint8_t qs(int p) const { return blk[16 + p]; }
};
struct TiledQ4K {
  const uint8_t* ch;
  int rr;
  __device__ TiledQ4K(const uint8_t* base, const TiledGeom& g, int64_t row, int64_t sb) {
    ch = base + chunk_offset(g, row / kChunkRows, sb);
    rr = (int)(row % kChunkRows);
  }
  __device__ float d() const { return ld_f16(ch + q4k_d_pos(rr)); }
  __device__ float dmin() const { return ld_f16(ch + q4k_d_pos(rr) + 2); }
  __device__ uint8_t sc(int s) const { return ch[q4k_sc_pos(rr, s)]; }
  __device__ uint8_t qs(int p) const { return ch[q4k_qs_pos(rr, p)]; }
};
struct RawQ5K {
  const uint8_t* blk;
  __device__ RawQ5K(const uint8_t* base, int64_t row, int64_t k, int64_t sb) {
    blk = base + row * (k / 256) * 176 + sb * 176;
  }
  __device__ float d() const { return ld_f16(blk); }
  __device__ float dmin() const { return ld_f16(blk + 2); }
  __device__ uint8_t sc(int s) const { return blk[4 + s]; }
  __device__ uint8_t qh(int l) const { return blk[16 + l]; }
  __device__ uint8_t qs(int p) const { return blk[48 + p]; }
};
struct TiledQ5K {
  const uint8_t* ch;
  int rr;
  __device__ TiledQ5K(const uint8_t* base, const TiledGeom& g, int64_t row, int64_t sb) {
    ch = base + chunk_offset(g, row / kChunkRows, sb);
    rr = (int)(row % kChunkRows);
  }
  __device__ float d() const { return ld_f16(ch + q5k_d_pos(rr)); }
  __device__ float dmin() const { return ld_f16(ch + q5k_d_pos(rr) + 2); }
  __device__ uint8_t sc(int s) const { return ch[q5k_sc_pos(rr, s)]; }
  __device__ uint8_t qh(int l) const { return ch[q5k_qh_pos(rr, l)]; }
  __device__ uint8_t qs(int p) const { return ch[q4k_qs_pos(rr, p)]; }
};
struct RawQ6K {
  const uint8_t* blk;
  Q6Fields f;
  __device__ RawQ6K(const uint8_t* base, int64_t row, int64_t k, int64_t sb, int layout) {
    blk = base + row * (k / 256) * 210 + sb * 210;
    f = q6_fields(layout);
  }
  __device__ float d() const { return ld_f16(blk + f.d); }
  __device__ uint8_t ql(int p) const { return blk[f.ql + p]; }
  __device__ uint8_t qh(int p) const { return blk[f.qh + p]; }
  __device__ int8_t sc(int s) const { return (int8_t)blk[f.sc + s]; }
};
struct TiledQ6K {
  const uint8_t* ch;
  int rr;
  __device__ TiledQ6K(const uint8_t* base, const TiledGeom& g, int64_t row, int64_t sb) {
    ch = base + chunk_offset(g, row / kChunkRows, sb);
    rr = (int)(row % kChunkRows);
  }
  __device__ float d() const { return ld_f16(ch + q6k_d_pos(rr)); }
  __device__ uint8_t ql(int p) const { return ch[q6k_ql_pos(rr, p)]; }
  __device__ uint8_t qh(int p) const { return ch[q6k_qh_pos(rr, p)]; }
  __device__ int8_t sc(int s) const { return (int8_t)ch[q6k_sc_pos(rr, s)]; }
};
// Q8_0: b is the block index inside the 256-element super-block.
struct RawQ80 {
  const uint8_t* row_base;
  int64_t sb;
  __device__ RawQ80(const uint8_t* base, int64_t row, int64_t k, int64_t sb_) {
    row_base = base + row * (k / 32) * 34;
    sb = sb_;
  }
  __device__ float d(int b) const { return ld_f16(row_base + (sb * 8 + b) * 34); }
  __device__ int8_t qs(int b, int p) const { return (int8_t)row_base[(sb * 8 + b) * 34 + 2 + p]; }
};
struct TiledQ80 {
  const uint8_t* ch;
  int rr;
  __device__ TiledQ80(const uint8_t* base, const TiledGeom& g, int64_t row, int64_t sb) {
    ch = base + chunk_offset(g, row / kChunkRows, sb);
    rr = (int)(row % kChunkRows);
  }
  __device__ float d(int b) const { return ld_f16(ch + q80_d_pos(rr, b)); }
  __device__ int8_t qs(int b, int p) const { return (int8_t)ch[q80_qs_pos(rr, b, p)]; }
};

// Q4_0 / Q4_1 / Q5_0 / Q5_1: b is the block index inside the super-block;
// d, m (Q4_1 / Q5_1), qh (Q5_x, 32 bits, bit e = element e), qs[16].
struct Q4xRawFields { int m, qh, qs; };
__host__ __device__ inline Q4xRawFields q4x_raw_fields(int qt) {
  if (qt == kQ4_0) return {-1, -1, 2};
  if (qt == kQ4_1) return {2, -1, 4};
  if (qt == kQ5_0) return {-1, 2, 6};
  return {2, 4, 8};
}
struct RawQ4x {
  const uint8_t* row_base;
  int64_t sb;
  int bb;
  Q4xRawFields f;
  __device__ RawQ4x(const uint8_t* base, int64_t row, int64_t k, int64_t sb_, int qt) {
    bb = block_bytes_of(qt);
    row_base = base + row * (k / 32) * bb;
    sb = sb_;
    f = q4x_raw_fields(qt);
  }
  __device__ const uint8_t* blk(int b) const { return row_base + (sb * 8 + b) * bb; }
  __device__ float d(int b) const { return ld_f16(blk(b)); }
  __device__ float m(int b) const { return ld_f16(blk(b) + f.m); }
  __device__ uint32_t qh(int b) const {
    const uint8_t* h = blk(b) + f.qh;
    return (uint32_t)h[0] | ((uint32_t)h[1] << 8) | ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
  }
  __device__ uint8_t qs(int b, int p) const { return blk(b)[f.qs + p]; }
};
struct TiledQ4x {
  const uint8_t* ch;
  int rr;
  Q4xFields f;
  __device__ TiledQ4x(const uint8_t* base, const TiledGeom& g, int64_t row, int64_t sb, int qt) {
    ch = base + chunk_offset(g, row / kChunkRows, sb);
    rr = (int)(row % kChunkRows);
    f = q4x_fields(qt);
  }
  __device__ float d(int b) const { return ld_f16(ch + q4x_half_pos(f.d, rr, b)); }
  __device__ float m(int b) const { return ld_f16(ch + q4x_half_pos(f.m, rr, b)); }
  __device__ uint32_t qh(int b) const {
    const uint8_t* h = ch + q4x_word_pos(f.qh, rr, b);
    return (uint32_t)h[0] | ((uint32_t)h[1] << 8) | ((uint32_t)h[2] << 16) | ((uint32_t)h[3] << 24);
  }
  __device__ uint8_t qs(int b, int p) const { return ch[q4x_qs_pos(rr, b, p)]; }
};

// ---------------------------------------------------------------------------
// 8 consecutive elements e0..e0+7 (e0 % 8 == 0) of one 256-element super-block
// ---------------------------------------------------------------------------
template <class A>
__device__ __forceinline__ void decode8_q4k(const A& a, int e0, float (&o)[8]) {
  int g4 = e0 >> 6, upper = (e0 & 63) >= 32, j = 2 * g4 + upper;
  uint8_t scb[12];
#pragma unroll
  for (int s = 0; s < 12; ++s) scb[s] = a.sc(s);
  int sc, m;
  q4k_scale_min(scb, j, sc, m);
  float d1 = __fmul_rn(a.d(), (float)sc);
  float m1 = __fmul_rn(a.dmin(), (float)m);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int l = (e0 + i) & 31;
    uint8_t byte = a.qs(32 * g4 + l);
    int q = upper ? (byte >> 4) : (byte & 15);
    o[i] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
  }
}

template <class A>
__device__ __forceinline__ void decode8_q5k(const A& a, int e0, float (&o)[8]) {
  int g4 = e0 >> 6, upper = (e0 & 63) >= 32, j = 2 * g4 + upper;
  uint8_t scb[12];
#pragma unroll
  for (int s = 0; s < 12; ++s) scb[s] = a.sc(s);
  int sc, m;
  q4k_scale_min(scb, j, sc, m);
  float d1 = __fmul_rn(a.d(), (float)sc);
  float m1 = __fmul_rn(a.dmin(), (float)m);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int l = (e0 + i) & 31;
    uint8_t byte = a.qs(32 * g4 + l);
    int q = (upper ? (byte >> 4) : (byte & 15)) | (((a.qh(l) >> j) & 1) << 4);
    o[i] = __fsub_rn(__fmul_rn(d1, (float)q), m1);
  }
}

template <class A>
__device__ __forceinline__ void decode8_q6k(const A& a, int e0, float (&o)[8]) {
  int n = e0 >> 7, r = e0 & 127, i4 = r >> 5, l0 = r & 31;
  int s = 8 * n + 2 * i4 + (l0 >> 4);
  float dl = __fmul_rn(a.d(), (float)a.sc(s));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int l = l0 + i;
    uint8_t qlb = a.ql(64 * n + l + 32 * (i4 & 1));
    int nib = (i4 < 2) ? (qlb & 15) : (qlb >> 4);
    int hb = (a.qh(32 * n + l) >> (2 * i4)) & 3;
    int q = (nib | (hb << 4)) - 32;
    o[i] = __fmul_rn(dl, (float)q);
  }
}

template <class A>
__device__ __forceinline__ void decode8_q80(const A& a, int e0, float (&o)[8]) {
  int b = e0 >> 5, p0 = e0 & 31;
  float d = a.d(b);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = __fmul_rn((float)a.qs(b, p0 + i), d);
}

// element p of a block: low nibble of qs byte p (p < 16) or high nibble of
// byte p - 16, with bit p of qh as the fifth bit (gguf.py:310-353)
template <int QT, class A>
__device__ __forceinline__ void decode8_q4x(const A& a, int e0, float (&o)[8]) {
  constexpr bool kH = QT == kQ5_0 || QT == kQ5_1, kM = QT == kQ4_1 || QT == kQ5_1;
  const int b = e0 >> 5, p0 = e0 & 31;
  const float d = a.d(b);
  const float m = kM ? a.m(b) : 0.f;
  const uint32_t h = kH ? a.qh(b) : 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int p = p0 + i;
    const uint8_t byte = a.qs(b, p & 15);
    int q = p < 16 ? (byte & 15) : (byte >> 4);
    if (kH) q |= (int)((h >> p) & 1u) << 4;
    if (kM) o[i] = __fadd_rn(__fmul_rn((float)q, d), m);
    else o[i] = __fmul_rn((float)(q - (kH ? 16 : 8)), d);
  }
}

// ---------------------------------------------------------------------------
// dequant kernel: one warp per (row, super-block), lane -> 8 elements
// ---------------------------------------------------------------------------
template <typename OutT>
__device__ __forceinline__ void store8(OutT* dst, const float (&o)[8]);
template <>
__device__ __forceinline__ void store8<float>(float* dst, const float (&o)[8]) {
  float4* p = reinterpret_cast<float4*>(dst);
  p[0] = make_float4(o[0], o[1], o[2], o[3]);
  p[1] = make_float4(o[4], o[5], o[6], o[7]);
}
template <>
__device__ __forceinline__ void store8<uint16_t>(uint16_t* dst, const float (&o)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename OutT, int QT, bool TILED>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ src, OutT* __restrict__ out,
                                                      int64_t n_rows, int64_t k, int layout) {
  const int64_t nb = (k + 255) / 256;
  const int64_t warp = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= n_rows * nb) return;
  const int64_t row = warp / nb, sb = warp % nb;
  const int e0 = lane * 8;
  if (sb * 256 + e0 >= k) return;  // tail super-block of a 32-element-block type
  float o[8];
  TiledGeom g = tiled_geom(QT, n_rows, k);
  if (QT == kQ4_K) {
    if (TILED) decode8_q4k(TiledQ4K(src, g, row, sb), e0, o);
    else decode8_q4k(RawQ4K(src, row, k, sb), e0, o);
  } else if (QT == kQ5_K) {
    if (TILED) decode8_q5k(TiledQ5K(src, g, row, sb), e0, o);
    else decode8_q5k(RawQ5K(src, row, k, sb), e0, o);
  } else if (QT == kQ6_K) {
    if (TILED) decode8_q6k(TiledQ6K(src, g, row, sb), e0, o);
    else decode8_q6k(RawQ6K(src, row, k, sb, layout), e0, o);
  } else if (QT == kQ8_0) {
    if (TILED) decode8_q80(TiledQ80(src, g, row, sb), e0, o);
    else decode8_q80(RawQ80(src, row, k, sb), e0, o);
  } else {
    if (TILED) decode8_q4x<QT>(TiledQ4x(src, g, row, sb, QT), e0, o);
    else decode8_q4x<QT>(RawQ4x(src, row, k, sb, QT), e0, o);
  }
  store8<OutT>(out + row * k + sb * 256 + e0, o);
}

// ---------------------------------------------------------------------------
// repack GGUF -> TILED: one thread per (row, GGUF block); bytes are moved, not
// changed.  The destination is zero-filled first (padding rows / blocks).
// ---------------------------------------------------------------------------
template <int QT>
__global__ void __launch_bounds__(256) repack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                     int64_t n_rows, int64_t k, int layout) {
  const int bs = block_size_of(QT), bb = block_bytes_of(QT);
  const int64_t nblk = k / bs;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_rows * nblk) return;
  const int64_t row = idx / nblk, bi = idx % nblk;
  const uint8_t* b = src + row * nblk * bb + bi * bb;
  TiledGeom g = tiled_geom(QT, n_rows, k);
  const int rr = (int)(row % kChunkRows);
  if (QT == kQ4_K) {
    uint8_t* ch = dst + chunk_offset(g, row / kChunkRows, bi);
    const int dp = q4k_d_pos(rr);
    ch[dp] = b[0];
    ch[dp + 1] = b[1];
    ch[dp + 2] = b[2];
    ch[dp + 3] = b[3];
    for (int s = 0; s < 12; ++s) ch[q4k_sc_pos(rr, s)] = b[4 + s];
    for (int p = 0; p < 128; ++p) ch[q4k_qs_pos(rr, p)] = b[16 + p];
  } else if (QT == kQ5_K) {
    uint8_t* ch = dst + chunk_offset(g, row / kChunkRows, bi);
    const int dp = q5k_d_pos(rr);
    ch[dp] = b[0];
    ch[dp + 1] = b[1];
    ch[dp + 2] = b[2];
    ch[dp + 3] = b[3];
    for (int s = 0; s < 12; ++s) ch[q5k_sc_pos(rr, s)] = b[4 + s];
    for (int l = 0; l < 32; ++l) ch[q5k_qh_pos(rr, l)] = b[16 + l];
    for (int p = 0; p < 128; ++p) ch[q4k_qs_pos(rr, p)] = b[48 + p];
  } else if (QT == kQ6_K) {
    uint8_t* ch = dst + chunk_offset(g, row / kChunkRows, bi);
    const Q6Fields f = q6_fields(layout);
    const int dp = q6k_d_pos(rr);
    ch[dp] = b[f.d];
    ch[dp + 1] = b[f.d + 1];
    for (int p = 0; p < 128; ++p) ch[q6k_ql_pos(rr, p)] = b[f.ql + p];
    for (int p = 0; p < 64; ++p) ch[q6k_qh_pos(rr, p)] = b[f.qh + p];
    for (int s = 0; s < 16; ++s) ch[q6k_sc_pos(rr, s)] = b[f.sc + s];
  } else if (QT == kQ8_0) {
    const int64_t sb = bi / 8;
    const int blk = (int)(bi % 8);
    uint8_t* ch = dst + chunk_offset(g, row / kChunkRows, sb);
    const int dp = q80_d_pos(rr, blk);
    ch[dp] = b[0];
    ch[dp + 1] = b[1];
    for (int p = 0; p < 32; ++p) ch[q80_qs_pos(rr, blk, p)] = b[2 + p];
  } else {
    const int64_t sb = bi / 8;
    const int blk = (int)(bi % 8);
    uint8_t* ch = dst + chunk_offset(g, row / kChunkRows, sb);
    const Q4xFields f = q4x_fields(QT);
    const Q4xRawFields rf = q4x_raw_fields(QT);
    const int dp = q4x_half_pos(f.d, rr, blk);
    ch[dp] = b[0];
    ch[dp + 1] = b[1];
    if (f.m >= 0) {
      const int mp = q4x_half_pos(f.m, rr, blk);
      ch[mp] = b[rf.m];
      ch[mp + 1] = b[rf.m + 1];
    }
    if (f.qh >= 0) {
      const int hp = q4x_word_pos(f.qh, rr, blk);
      for (int i = 0; i < 4; ++i) ch[hp + i] = b[rf.qh + i];
    }
    for (int p = 0; p < 16; ++p) ch[q4x_qs_pos(rr, blk, p)] = b[rf.qs + p];
  }
}

// ---------------------------------------------------------------------------
// launchers (called from capi.cu after argument checks)
// ---------------------------------------------------------------------------
template <typename OutT>
static cudaError_t launch_dequant_t(int qt, int layout, const void* src, OutT* out, int64_t n_rows, int64_t k,
                                    cudaStream_t st) {
  const int64_t nb = (k + 255) / 256;
  const int64_t warps = n_rows * nb;
  const int64_t blocks = (warps + 7) / 8;
  if (blocks == 0) return cudaSuccess;
  const uint8_t* s = static_cast<const uint8_t*>(src);
  const bool tiled = layout == DRACO_LAYOUT_TILED;
  dim3 grid((unsigned)blocks);
#define DRACO_DQ(QT)                                                                              \
  do {                                                                                            \
    if (tiled) dequant_kernel<OutT, QT, true><<<grid, 256, 0, st>>>(s, out, n_rows, k, layout);  \
    else dequant_kernel<OutT, QT, false><<<grid, 256, 0, st>>>(s, out, n_rows, k, layout);       \
  } while (0)
  if (qt == kQ4_K) DRACO_DQ(kQ4_K);
  else if (qt == kQ5_K) DRACO_DQ(kQ5_K);
  else if (qt == kQ6_K) DRACO_DQ(kQ6_K);
  else if (qt == kQ4_0) DRACO_DQ(kQ4_0);
  else if (qt == kQ4_1) DRACO_DQ(kQ4_1);
  else if (qt == kQ5_0) DRACO_DQ(kQ5_0);
  else if (qt == kQ5_1) DRACO_DQ(kQ5_1);
  else DRACO_DQ(kQ8_0);
#undef DRACO_DQ
  return cudaGetLastError();
}

cudaError_t launch_dequant_f32(int qt, int layout, const void* src, float* out, int64_t n_rows, int64_t k,
                               cudaStream_t st) {
  return launch_dequant_t<float>(qt, layout, src, out, n_rows, k, st);
}
cudaError_t launch_dequant_bf16(int qt, int layout, const void* src, uint16_t* out, int64_t n_rows, int64_t k,
                                cudaStream_t st) {
  return launch_dequant_t<uint16_t>(qt, layout, src, out, n_rows, k, st);
}

cudaError_t launch_repack(int qt, int src_layout, const void* src, void* dst, int64_t n_rows, int64_t k,
                          cudaStream_t st) {
  TiledGeom g = tiled_geom(qt, n_rows, k);
  cudaError_t e = cudaMemsetAsync(dst, 0, (size_t)tiled_total_bytes(g), st);
  if (e != cudaSuccess) return e;
  const int64_t n = n_rows * (k / block_size_of(qt));
  if (n == 0) return cudaSuccess;
  dim3 grid((unsigned)((n + 255) / 256));
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
  if (qt == kQ4_K) repack_kernel<kQ4_K><<<grid, 256, 0, st>>>(s, d, n_rows, k, src_layout);
  else if (qt == kQ5_K) repack_kernel<kQ5_K><<<grid, 256, 0, st>>>(s, d, n_rows, k, src_layout);
  else if (qt == kQ6_K) repack_kernel<kQ6_K><<<grid, 256, 0, st>>>(s, d, n_rows, k, src_layout);
  else if (qt == kQ4_0) repack_kernel<kQ4_0><<<grid, 256, 0, st>>>(s, d, n_rows, k, src_layout);
  else if (qt == kQ4_1) repack_kernel<kQ4_1><<<grid, 256, 0, st>>>(s, d, n_rows, k, src_layout);
  else if (qt == kQ5_0) repack_kernel<kQ5_0><<<grid, 256, 0, st>>>(s, d, n_rows, k, src_layout);
  else if (qt == kQ5_1) repack_kernel<kQ5_1><<<grid, 256, 0, st>>>(s, d, n_rows, k, src_layout);
  else repack_kernel<kQ8_0><<<grid, 256, 0, st>>>(s, d, n_rows, k, src_layout);
  return cudaGetLastError();
}

}  // namespace draco
