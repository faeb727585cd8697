// gemv_plan.h — the decode GEMV's launch plan, shared by its two kernels:
// the warp-MMA kernel (gemv.cu) and the tensor-memory kernel for larger
// batches (gemv_tc.cu).  Internal to the library.
#pragma once
#include "common.cuh"
#include "internal.h"

namespace draco {

constexpr int kMaxCta = 192;
constexpr int kRowWarps = 8;                      // row tiles of a slab
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait

struct GemvProbDev {
  const uint8_t* w;
  const float* x;
  float* y;
  const float* bias;
  int64_t ldx, ldy;
  int slab0;  // global index of the problem's first slab
  int qt, n_rows, k, nb, n_rg, n_tiles, cb;
  int64_t tp_y_off, tp_par_stride;  // tensor-parallel output block in every rank's exchange buffer
  int64_t xcv_off;                   // workspace offset of the pre-converted activation slices
  int in_mode;                       // DRACO_INPUT_*: transform applied as x is read
  float eps;                         // RMSNORM epsilon
  const float* aux;                  // RMSNORM: norm weight [k]; SWIGLU: up [batch, k]
  int64_t ldaux;
  int64_t rms_off;                   // RMSNORM: workspace offset of the per-row scales [batch]
  int accumulate;                    // y += result (DRACO_GEMV_ACCUMULATE)
  int pidx;                          // index of the problem in the launch
};

struct GemvParams {
  GemvProbDev prob[DRACO_GEMV_MAX_PROBLEMS];
  uint8_t* ws;
  int64_t status_off, cnt_off, part_off;
  int total_slabs;
  int n_prob, batch, nt, n_cta;
  int w_stage, xs_bytes, su_bytes, stage_bytes, n_stages;
  int mbox_slots, mbox_off;  // row-group mailbox after the stages in dynamic shared memory
  int precvt;                // activations converted by gemv_convert_kernel before the launch
  int rms_inkernel;          // batch 1: RMSNorm row scales computed by the converter warps
  int tp_world, tp_rank;     // tensor-parallel exchange (tp_world 0: plain outputs)
  uint8_t* tp_buf[DRACO_TP_MAX_WORLD];
  int64_t tp_flags_off, tp_counter_off;
  int cta_start[kMaxCta + 1];
};

// workspace layout (bytes)
constexpr int64_t kWsStatus = 0;
constexpr int64_t kWsGridDone = 128;  // CTAs finished (tensor-parallel form)
constexpr int64_t kWsCounters = 256;
constexpr int64_t kWsCountersBytes = (int64_t)kMaxCta * 2 * kRowWarps * 4;  // per (CTA, end, row tile)
static inline int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }

// row tiles (16 rows) in row group rg of a problem
__device__ __forceinline__ int rg_tile_count(const GemvProbDev& pr, int rg) {
  const int r = pr.n_tiles - rg * kGroupTiles;
  return r < kGroupTiles ? r : kGroupTiles;
}

__device__ __forceinline__ void record_error(const GemvParams& P, int code) {
  atomicCAS(reinterpret_cast<int*>(P.ws + P.status_off), 0, code);
}

// Slab cursor: (problem, row group, super-block) of a global slab index,
// advanced incrementally.
struct SlabCursor {
  int p, rg, j;
  __device__ void seek(const GemvParams& P, int s) {
    p = 0;
    for (int q = 1; q < P.n_prob; ++q)
      if (s >= P.prob[q].slab0) p = q;
    const int local = s - P.prob[p].slab0;
    rg = local / P.prob[p].nb;
    j = local - rg * P.prob[p].nb;
  }
  __device__ void next(const GemvParams& P) {
    if (++j == P.prob[p].nb) {
      j = 0;
      if (++rg == P.prob[p].n_rg) {
        rg = 0;
        ++p;
      }
    }
  }
};

// 8 consecutive fp32 values at p (16-byte vector loads when aligned); the
// ones at or past `valid` read as 0
__device__ __forceinline__ void load8(const float* p, int valid, float (&v)[8]) {
  if (valid >= 8 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    const float4 lo4 = __ldg(reinterpret_cast<const float4*>(p));
    const float4 hi4 = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = lo4.x, v[1] = lo4.y, v[2] = lo4.z, v[3] = lo4.w;
    v[4] = hi4.x, v[5] = hi4.y, v[6] = hi4.z, v[7] = hi4.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = i < valid ? __ldg(p + i) : 0.f;
  }
}

struct HostPlan {
  GemvParams P;
  size_t ws_needed;
  size_t smem_bytes;
};

// Fill the plan of a grouped GEMV: per-problem fields, workspace offsets and
// byte-balanced slab ranges per CTA.  convert_once: activations converted once
// per launch into the workspace (the allocation-free entry converts in-kernel).
bool build_plan(const draco_gemv_problem* probs, int n, int batch, int n_sm, HostPlan& hp, char* msg, size_t ml,
                bool convert_once = true, const draco_gemv_input* inputs = nullptr);

// The tensor-memory kernel (gemv_tc.cu): batches of 17..32 rows (the
// DRACO_GEMV_TC_MIN_BATCH environment variable moves the lower bound; 33
// turns the kernel off) with only K-quant weights (Q4_K, Q5_K, Q6_K) and no
// tensor-parallel exchange.
bool gemv_tc_eligible(const draco_gemv_problem* probs, int n, int batch);
// Workspace bytes it needs (0 when not eligible).
size_t gemv_tc_workspace_bytes(const draco_gemv_problem* probs, int n, int batch, const draco_gemv_input* inputs);
// Row groups of the plan split between CTAs (each costs the fixup kernel a CTA).
int gemv_tc_split_count(const HostPlan& hp);
// Convert the activations and launch it over the plan's slab ranges; ws has
// gemv_tc_workspace_bytes bytes, zero at rest.
int gemv_tc_launch(const HostPlan& hp, const draco_gemv_input* inputs, void* ws, size_t ws_bytes, cudaStream_t st,
                   char* msg, size_t ml);

}  // namespace draco
