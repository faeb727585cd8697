// internal.h — declarations shared between the kernel translation units and
// the C ABI (capi.cu).  Not part of the public interface.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/draco_gguf.h"

namespace draco {

cudaError_t launch_dequant_f32(int qt, int layout, const void* src, float* out, int64_t n_rows, int64_t k,
                               cudaStream_t st);
cudaError_t launch_dequant_bf16(int qt, int layout, const void* src, uint16_t* out, int64_t n_rows, int64_t k,
                                cudaStream_t st);
cudaError_t launch_repack(int qt, int src_layout, const void* src, void* dst, int64_t n_rows, int64_t k,
                          cudaStream_t st);

// Grouped GEMV: plan + launch.  Returns a DRACO_* status; fills `msg` on error.
size_t gemv_workspace_bytes(const draco_gemv_problem* probs, int n, int batch);
int gemv_launch_count(const draco_gemv_problem* probs, int n, int batch);
int gemv_launch(const draco_gemv_problem* probs, int n, int batch, void* ws, size_t ws_bytes, cudaStream_t st,
                char* msg, size_t msg_len, const draco_gemv_input* inputs = nullptr);

// Tensor-parallel grouped GEMV (outputs to every rank's exchange buffer) and
// the step's finish on this rank.
int gemv_launch_tp(const draco_gemv_problem* probs, int n, int batch, const draco_tp_exchange* ex, void* ws,
                   size_t ws_bytes, cudaStream_t st, char* msg, size_t msg_len);
int tp_finish_launch(const draco_tp_exchange* ex, int batch, int64_t gather_off, int64_t gather_stride,
                     int gather_width, float* gather_out, int64_t reduce_off, int64_t reduce_stride, int reduce_width,
                     float* reduce_out, int* status, cudaStream_t st, char* msg, size_t msg_len);

// Allocation-free grouped GEMV (scratch in a fixed device array).
int gemv_launch_noalloc(const draco_gemv_problem* probs, int n, int batch, cudaStream_t st, char* msg,
                        size_t msg_len);
size_t gemv_static_scratch_bytes();
int gemv_noalloc_status(int* out, cudaStream_t st, char* msg, size_t msg_len);

// Prefill dequant-GEMM (tcgen05).  `status` is an optional device int the
// kernel sets to a DRACO_* code on a device-side failure.
// `rows` (optional, device): tokens actually present per problem, each m the capacity.
int gemm_launch(const draco_gemm_problem* probs, int n, const int* rows, int* status, cudaStream_t st, char* msg,
                size_t msg_len);

// out = bf16(silu(gate) * up) over n bf16 elements (16-byte aligned).
cudaError_t launch_swiglu_bf16(const void* gate, const void* up, void* out, int64_t n, cudaStream_t st);
// Row-counted bf16 form over groups of [cap_rows, width] blocks (rows: device counts).
cudaError_t launch_swiglu_bf16_rows(const void* gate, const void* up, void* out, int groups, int64_t cap_rows,
                                    int64_t width, const int* rows, cudaStream_t st);
// RMSNorm of rows x [rows, k] (fp32, or bf16 when bf16 != 0) with fp32 weight w.
cudaError_t launch_rmsnorm(const void* x, const float* w, void* out, int64_t rows, int64_t k, float eps, int bf16,
                           cudaStream_t st);
// out = silu(gate) * up over n fp32 elements (16-byte aligned).
cudaError_t launch_swiglu_f32(const float* gate, const float* up, float* out, int64_t n, cudaStream_t st);

// RoPE + key/value-cache append (op 0), cached attention (op 1) or the decode
// form with rotation and append inside (op 2) for the GPU decode step; see
// draco_rope_kv_append / draco_attention_cached / draco_attention_decode.
int attention_launch(int op, float* q, const float* k, const float* v, float* kc, float* vc, const float* cos_t,
                     const float* sin_t, const int* seq, const int* pos, float* out, int n, int heads, int kv_heads,
                     int hd, int capacity, int n_slots, int max_pos, float* part, size_t part_bytes, cudaStream_t st,
                     char* msg, size_t ml);
// Workspace bytes of the attention (status word, per-(token, head) counters,
// per-(token, head, 32-key chunk) partials) for n tokens over positions
// 0..max_pos.
size_t attention_workspace_bytes(int n, int heads, int hd, int max_pos);

// Number of SMs of the current device (cached per device).
int device_sm_count();

}  // namespace draco
