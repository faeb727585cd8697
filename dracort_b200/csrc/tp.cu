// tp.cu — the end of a tensor-parallel decode step on one rank.
//
// Replaces the shard-boundary collectives of draco/parallel/tp.py
// (ColumnParallelLinear's gather of the output shards and RowParallelLinear's
// sum of the partial outputs, whose all-reduce the reference leaves as a
// comment at tp.py:182-183).  The tensor-parallel GEMV has already stored
// every rank's output shard and partial sums into this rank's exchange buffer
// over NVLink and signalled through the buffer's flags; this kernel waits for
// all ranks' signals of the step, copies the gathered column outputs out and
// sums the row-parallel partials.
//
// Launched after the step's GEMV on the same stream with programmatic
// dependent launch: it may be scheduled early, but griddepcontrol.wait holds
// it until that GEMV has completed, so it never spins on a kernel of its own
// GPU: the only waits are on flags written by the other GPUs' kernels,
// bounded by kTpWaitNs, after which the status word records the failure and
// the kernel returns.  It lets the next kernel in the stream (the next step's
// GEMV) launch at once: that GEMV streams weights meanwhile and waits for
// this kernel's completion before it reads activations or writes outputs.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "internal.h"

namespace draco {

constexpr uint64_t kTpWaitNs = 1000000000ull;  // 1 s: far beyond a decode step
constexpr int kTpThreads = 256;

struct TpFinishParams {
  const uint8_t* own;  // this rank's exchange buffer
  int world;
  int64_t flags_off, counter_off;
  int batch;
  int64_t gather_off, gather_stride;
  int gather_width;
  float* gather_out;
  int64_t reduce_off, reduce_stride;
  int reduce_width;
  float* reduce_out;
  int* status;
};

__global__ void __launch_bounds__(kTpThreads) tp_finish_kernel(const __grid_constant__ TpFinishParams F) {
  __shared__ int failed;
  grid_dependency_wait();    // this rank's GEMV of the step is complete
  grid_launch_dependents();  // the next step's GEMV may start streaming weights
  // the step's epoch, counted by this rank's GEMV (complete: it precedes us in the stream)
  const int epoch = *reinterpret_cast<const volatile int*>(F.own + F.counter_off);
  const int par = epoch & 1;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < F.world) {
    const int* flag = reinterpret_cast<const int*>(F.own + F.flags_off) + par * DRACO_TP_MAX_WORLD + threadIdx.x;
    const uint64_t t0 = global_timer_ns();
    while (true) {
      const int v = ld_acquire_sys(flag);
      if (v == epoch) break;
      if (v == -epoch) {  // that rank's GEMV aborted
        if (F.status) atomicCAS(F.status, 0, DRACO_ERR_PEER);
        failed = 1;
        break;
      }
      if (global_timer_ns() - t0 > kTpWaitNs) {
        if (F.status) atomicCAS(F.status, 0, DRACO_ERR_TIMEOUT);
        failed = 1;
        break;
      }
    }
  }
  __syncthreads();
  if (failed) return;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (F.gather_width > 0) {
    const float* g = reinterpret_cast<const float*>(F.own + F.gather_off + par * F.gather_stride);
    const int64_t total = (int64_t)F.world * F.batch * F.gather_width;
    for (int64_t i = tid; i < total; i += stride) F.gather_out[i] = __ldcg(g + i);  // L2: written by peers
  }
  if (F.reduce_width > 0) {
    const float* r = reinterpret_cast<const float*>(F.own + F.reduce_off + par * F.reduce_stride);
    const int64_t per_rank = (int64_t)F.batch * F.reduce_width;
    for (int64_t i = tid; i < per_rank; i += stride) {
      float s = 0.f;
      for (int q = 0; q < F.world; ++q) s += __ldcg(r + q * per_rank + i);  // rank order: deterministic
      F.reduce_out[i] = s;
    }
  }
}

int tp_finish_launch(const draco_tp_exchange* ex, int batch, int64_t gather_off, int64_t gather_stride,
                     int gather_width, float* gather_out, int64_t reduce_off, int64_t reduce_stride, int reduce_width,
                     float* reduce_out, int* status, cudaStream_t st, char* msg, size_t ml) {
  if (ex->world < 2 || ex->world > DRACO_TP_MAX_WORLD || ex->rank < 0 || ex->rank >= ex->world ||
      ex->buffers[ex->rank] == nullptr) {
    snprintf(msg, ml, "tp_finish: bad world %d / rank %d or null own buffer", ex->world, ex->rank);
    return DRACO_ERR_ARG;
  }
  if (batch < 1 || gather_width < 0 || reduce_width < 0 || (gather_width > 0 && !gather_out) ||
      (reduce_width > 0 && !reduce_out)) {
    snprintf(msg, ml, "tp_finish: bad batch / widths or null output");
    return DRACO_ERR_ARG;
  }
  if ((gather_off | gather_stride | reduce_off | reduce_stride | ex->flags_off | ex->counter_off) & 3) {
    snprintf(msg, ml, "tp_finish: offsets must be multiples of 4");
    return DRACO_ERR_ALIGN;
  }
  TpFinishParams F;
  F.own = static_cast<const uint8_t*>(ex->buffers[ex->rank]);
  F.world = ex->world;
  F.flags_off = ex->flags_off;
  F.counter_off = ex->counter_off;
  F.batch = batch;
  F.gather_off = gather_off;
  F.gather_stride = gather_stride;
  F.gather_width = gather_width;
  F.gather_out = gather_out;
  F.reduce_off = reduce_off;
  F.reduce_stride = reduce_stride;
  F.reduce_width = reduce_width;
  F.reduce_out = reduce_out;
  F.status = status;
  const int64_t work = std::max<int64_t>((int64_t)ex->world * batch * gather_width, (int64_t)batch * reduce_width);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(2 * device_sm_count(),
                                                                 (work + kTpThreads - 1) / kTpThreads));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kTpThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, tp_finish_kernel, F);
  if (e != cudaSuccess) {
    snprintf(msg, ml, "tp_finish: launch failed: %s", cudaGetErrorString(e));
    return DRACO_ERR_CUDA;
  }
  return DRACO_OK;
}

}  // namespace draco
