/*
 * draco_gguf.h — C ABI of the B200 (sm_100a) GGUF quantized-linear library
 * (libdraco_gguf.so).
 *
 * The library replaces DracoRT's numpy GGUF path:
 *   draco/format/gguf.py:_dequantize            (gguf.py:272-497)
 *   draco/runtime/cpu/executor.py:_linear       (executor.py:47-79)
 *   draco/runtime/cpu/kernels/generic.py:matmul_f32 (generic.py:32-33)
 *   draco/quantization/base.py:QuantizationBackend.dequantize / quantized_linear
 *                                               (base.py:64-99)
 * with CUDA kernels that read the packed GGUF blocks directly.
 *
 * Conventions
 *   - A weight is GGUF-shaped [n_rows, k]: n_rows output features (GGML ne1),
 *     k reduction elements (GGML ne0, contiguous).  Blocks run along k inside
 *     each row (gguf.py:646-648).
 *   - All pointers are device pointers unless a comment says otherwise; the
 *     caller owns every buffer.  `stream` is a cudaStream_t (NULL = legacy
 *     default stream).  Work is enqueued on that stream; nothing synchronises
 *     the host except where stated.
 *   - Every function returns a DRACO_* status code.  The message of the last
 *     failure on the calling host thread is available from
 *     draco_last_error_string().
 *   - The library holds no mutable global state except the thread-local error
 *     string, per-device attribute caches and one shared device array: the
 *     fixed scratch of draco_gguf_gemv_grouped_noalloc, whose calls race when
 *     they overlap on the GPU (see there).  Every other call works on
 *     caller-owned buffers, and calls on different streams are independent.
 */
#ifndef DRACO_GGUF_H
#define DRACO_GGUF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type ids, identical to GGML_TYPE_* in draco/format/gguf.py:56-71. */
#define DRACO_GGML_TYPE_Q4_0 2
#define DRACO_GGML_TYPE_Q4_1 3
#define DRACO_GGML_TYPE_Q5_0 6
#define DRACO_GGML_TYPE_Q5_1 7
#define DRACO_GGML_TYPE_Q8_0 8
#define DRACO_GGML_TYPE_Q4_K 12
#define DRACO_GGML_TYPE_Q5_K 13
#define DRACO_GGML_TYPE_Q6_K 14

/* Byte layouts of a weight buffer.
 *   GGUF        : row-major blocks exactly as draco/format/gguf.py reads them
 *                 (_BLOCK_LAYOUTS, gguf.py:75-87).  For Q6_K this is the
 *                 reference's field order: d first (gguf.py:470-474).
 *   GGUF_DLAST  : row-major blocks as llama.cpp writes .gguf files; differs
 *                 from GGUF only for Q6_K, whose fp16 d is the LAST 2 bytes.
 *   TILED       : the device layout produced by draco_gguf_repack().  Same
 *                 payload bytes regrouped into 16-row x 256-element chunks,
 *                 128-row slabs, rows padded to a multiple of 16 and k to a
 *                 multiple of 256 with zero blocks.  Size from
 *                 draco_gguf_tiled_bytes(). */
#define DRACO_LAYOUT_GGUF 0
#define DRACO_LAYOUT_GGUF_DLAST 1
#define DRACO_LAYOUT_TILED 2

/* Status codes.  The Python wrapper maps them onto the reference exception
 * classes: TYPE/SHAPE -> DracoFormatError (gguf.py:284-296), ALIGN/ARG ->
 * ValueError, CUDA/TIMEOUT -> KernelError. */
#define DRACO_OK 0
#define DRACO_ERR_TYPE 1      /* unsupported qtype or layout             */
#define DRACO_ERR_SHAPE 2     /* k not a multiple of the block size, etc */
#define DRACO_ERR_ALIGN 3     /* pointer not aligned as required         */
#define DRACO_ERR_CUDA 4      /* a CUDA runtime call failed              */
#define DRACO_ERR_TIMEOUT 5   /* a bounded device wait ran out           */
#define DRACO_ERR_ARG 6       /* null pointer, bad batch, too many problems */
#define DRACO_ERR_WORKSPACE 7 /* workspace missing or too small          */
#define DRACO_ERR_PEER 8      /* another rank reported a failed step     */

/* Output element types for the GEMM. */
#define DRACO_DTYPE_F32 0
#define DRACO_DTYPE_BF16 1

/* Library version string, e.g. "draco_gguf 0.1.0 sm_100a". */
const char* draco_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* draco_last_error_string(void);

/* (block_size, block_bytes) of a qtype: Q4_0 (32, 18), Q4_1 (32, 20),
 * Q5_0 (32, 22), Q5_1 (32, 24), Q8_0 (32, 34), Q4_K (256, 144),
 * Q5_K (256, 176), Q6_K (256, 210).  Replaces the table lookup _BLOCK_LAYOUTS[qtype]
 * (gguf.py:75-87).  Returns DRACO_ERR_TYPE for other types.  Host only. */
int draco_gguf_block_geometry(int qtype, int* block_size, int* block_bytes);

/* Bytes of a weight in the GGUF layouts: n_rows * (k / block_size) * block_bytes
 * (gguf.py:639-645).  Returns -1 on an unsupported type or k that is not a
 * multiple of the block size.  Host only. */
int64_t draco_gguf_packed_bytes(int qtype, int64_t n_rows, int64_t k);

/* Bytes of the same weight in the TILED layout (>= packed bytes; equal when
 * n_rows % 16 == 0 and k % 256 == 0).  -1 on error.  Host only. */
int64_t draco_gguf_tiled_bytes(int qtype, int64_t n_rows, int64_t k);

/* Dequantize a whole weight to fp32, out[n_rows, k] row-major.
 * Bit-exact with draco/format/gguf.py:_dequantize (gguf.py:272-497) for
 * Q8_0 (:300-303), Q4_0 / Q4_1 (:310-324), Q5_0 / Q5_1 (:326-353), Q4_K and
 * Q5_K (:425-468) and Q6_K (:470-495).
 * `layout` is any DRACO_LAYOUT_*; GGUF layouts need `blocks` 2-byte aligned,
 * TILED needs 16-byte alignment. */
int draco_gguf_dequant(int qtype, int layout, const void* blocks, float* out,
                       int64_t n_rows, int64_t k, void* stream);

/* Same as draco_gguf_dequant, writing bf16 (round-to-nearest-even of the
 * exact fp32 value) as uint16_t bit patterns. */
int draco_gguf_dequant_bf16(int qtype, int layout, const void* blocks, uint16_t* out,
                            int64_t n_rows, int64_t k, void* stream);

/* Regroup a GGUF-layout weight (src_layout GGUF or GGUF_DLAST) into the
 * TILED layout.  `dst` must hold draco_gguf_tiled_bytes() bytes and be
 * 16-byte aligned.  Bytes are moved, never changed, so dequantizing dst gives
 * bit-identical values.  Replaces the reference's first-access transform
 * GGUFReader.get_tensor (gguf.py:820-834), which caches fp32 instead. */
int draco_gguf_repack(int qtype, int src_layout, const void* src, void* dst,
                      int64_t n_rows, int64_t k, void* stream);

/* One linear layer of a grouped GEMV launch: y = x @ dequant(W)^T (+ bias).
 *   w     : TILED weight [n_rows, k] of type qtype
 *   x     : fp32 [batch, k], row stride ldx elements
 *   y     : fp32 [batch, n_rows], row stride ldy elements (written, or added
 *           to with DRACO_GEMV_ACCUMULATE: y += x @ dequant(W)^T + bias, the
 *           residual add of a layer folded into its projection)
 *   bias  : fp32 [n_rows] or NULL
 *   flags : 0 or DRACO_GEMV_ACCUMULATE (other bits are rejected; the
 *           tensor-parallel entry takes no flags)
 * Replaces one executor._linear call (executor.py:47-79) whose matmul is
 * GenericGemmKernel.matmul_f32 (generic.py:32-33). */
#define DRACO_GEMV_ACCUMULATE 1

typedef struct draco_gemv_problem {
  int qtype;
  int flags;
  const void* w;
  const float* x;
  float* y;
  const float* bias;
  int64_t n_rows;
  int64_t k;
  int64_t ldx;
  int64_t ldy;
} draco_gemv_problem;

#define DRACO_GEMV_MAX_PROBLEMS 8
#define DRACO_GEMV_MAX_BATCH 32

/* Workspace bytes the grouped GEMV needs for these problems at this batch.
 * The workspace must be 256-byte aligned and ZERO-FILLED before its first
 * use; every call leaves its counters at zero again, so one allocation can
 * serve any number of calls on one stream (not concurrent calls).  Host only. */
size_t draco_gguf_gemv_workspace_bytes(const draco_gemv_problem* problems, int n_problems,
                                       int batch);

/* Number of kernel launches one draco_gguf_gemv_grouped call over these
 * problems makes on the current device: 1 (batch 1, the GEMV alone), 2 (an
 * activation conversion kernel first), or 3 (batches 17-32 of K-quants on
 * the tensor-memory kernel, plus a kernel adding the partial sums of row
 * groups split between CTAs).  -1 on invalid arguments.  Host only. */
int draco_gguf_gemv_launch_count(const draco_gemv_problem* problems, int n_problems, int batch);

/* Decode GEMV over 1..DRACO_GEMV_MAX_PROBLEMS weights in one persistent
 * launch (the 7 projections of a decoder layer fit in one call).
 * 1 <= batch <= DRACO_GEMV_MAX_BATCH.  fp32 in, fp32 out.  Batches of 17-32
 * over K-quants (Q4_K / Q5_K / Q6_K) run on the tensor-memory kernel (fp16
 * operands scaled per super-block, ~2e-4 relative L2); otherwise the quants
 * and the activations meet in int8 tensor-core MMAs with exact integer
 * accumulation;
 * each 32-element group of activations is represented to one step of a
 * power-of-two scale u (max|x| / u in [2^13, 2^14)), which keeps results
 * within ~1e-4 relative L2 of the fp32 oracle (~6.5e-5 for Gaussian inputs).
 * `problems` is a host array. */
int draco_gguf_gemv_grouped(const draco_gemv_problem* problems, int n_problems, int batch,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Input transform of one problem of draco_gguf_gemv_grouped_ex: the layer
 * boundary fused into the GEMV's activation read.
 *   PLAIN   : x as it is.
 *   RMSNORM : x is the hidden state before the model's RMSNorm;
 *             y = rmsnorm(x) @ dequant(W)^T (+ bias) with
 *             rmsnorm(x) = x * rsqrt(mean(x^2) + eps) * aux, aux the fp32
 *             norm weight [k] (draco/kernels/ops.py:29-50, fused_rms_norm,
 *             ahead of the q/k/v and gate/up projections).  The per-row
 *             scale is applied to the outputs, the weight to x as it is read.
 *   SWIGLU  : x is the gate projection's output, aux the up projection's
 *             ([batch, k], row stride ldaux elements);
 *             y = (silu(x) * aux) @ dequant(W)^T (+ bias): the SwiGLU
 *             product ahead of the down projection
 *             (draco/kernels/ops.py:114-137, fused_swiGLU) read in place. */
#define DRACO_INPUT_PLAIN 0
#define DRACO_INPUT_RMSNORM 1
#define DRACO_INPUT_SWIGLU 2
typedef struct draco_gemv_input {
  int mode;
  float eps;
  const float* aux;
  int64_t ldaux;
} draco_gemv_input;

/* draco_gguf_gemv_grouped with an input transform per problem (`inputs`, a
 * host array of n_problems entries, or NULL for all PLAIN).  Same workspace
 * (draco_gguf_gemv_workspace_bytes covers it).  A launch with an RMSNORM
 * problem computes the row scales and converts the activations in a first
 * kernel on `stream`, then runs the GEMV. */
int draco_gguf_gemv_grouped_ex(const draco_gemv_problem* problems, const draco_gemv_input* inputs, int n_problems,
                               int batch, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free form of draco_gguf_gemv_grouped.  No counterpart in the
 * reference: DracoRT's numpy path has no device memory to manage.
 *
 * For callers that cannot allocate device memory themselves: hosts whose
 * device memory is owned by another allocator (an inference server's pool,
 * a framework that forbids hidden allocations), plain C / FFI hosts without a
 * device allocator of their own, and decode loops that cannot pay for
 * cudaMalloc's implicit device synchronisation.  Such callers pass only
 * their inputs and outputs; the kernel's scratch (status word, arrival
 * counters, partial sums) lives in a fixed 1 MiB device array inside the
 * library, which every GPU that loads the library holds until the process
 * exits.  No cudaMalloc, cudaFree or other allocating call is made.
 *
 * Limit: 1 <= batch <= 4 (the scratch a call needs grows with the batch;
 * larger calls are rejected with DRACO_ERR_WORKSPACE and a message).
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * Each call clears the counters it relies on (cudaMemsetAsync on `stream`).
 * All calls share the one array: calls that overlap on the GPU (different
 * streams, or different host threads on one device) race and must be
 * serialised by the caller.
 * A device-side failure (a bounded wait that ran out) is not visible in the
 * return code, which only covers the launch: read it with
 * draco_gguf_gemv_noalloc_status before the next call, which clears it. */
int draco_gguf_gemv_grouped_noalloc(const draco_gemv_problem* problems, int n_problems, int batch,
                                    void* stream);

/* Status of the last draco_gguf_gemv_grouped_noalloc call on the current
 * device: *status (host int) becomes 0 or the DRACO_* code the kernel
 * recorded (DRACO_ERR_TIMEOUT when a device wait ran out; the outputs of that
 * call are then invalid).  Reads the fixed array after the work queued on
 * `stream` and waits for it (host synchronisation); allocates nothing.  No
 * counterpart in the reference (its numpy path has no device status). */
int draco_gguf_gemv_noalloc_status(int* status, void* stream);

/* ---------------------------------------------------------------------------
 * Tensor-parallel decode over NVLink: one process per GPU, ranks on one box.
 *
 * Replaces the shard-boundary collectives of draco/parallel/tp.py
 * (ColumnParallelLinear's gather of the output shards, RowParallelLinear's
 * sum of the partial outputs; the reference leaves that all-reduce as a
 * comment at tp.py:182-183).  Every rank allocates an exchange buffer of the
 * same size and layout and maps the others' with CUDA IPC.  The GEMV stores
 * its outputs straight into every rank's buffer and signals each rank;
 * draco_tp_finish, on each rank, waits for every rank's signal of the step,
 * then copies the gathered columns out and sums the row partials.
 * ------------------------------------------------------------------------- */
#define DRACO_TP_MAX_WORLD 8
#define DRACO_IPC_HANDLE_BYTES 64

/* Exchange buffer: cudaMalloc'd (256-byte aligned) and zero-filled, as the
 * flags and the step counter in it must start at zero. */
int draco_tp_buffer_alloc(size_t bytes, void** ptr);
int draco_tp_buffer_free(void* ptr);
/* The CUDA IPC handle (DRACO_IPC_HANDLE_BYTES bytes) of a buffer from
 * draco_tp_buffer_alloc; the mapping of another process's handle into this
 * one (on the current device) and its release. */
int draco_ipc_get_handle(void* ptr, void* handle);
int draco_ipc_open(const void* handle, void** peer_ptr);
int draco_ipc_close(void* peer_ptr);

typedef struct draco_tp_exchange {
  int world; /* 2..DRACO_TP_MAX_WORLD */
  int rank;
  void* buffers[DRACO_TP_MAX_WORLD]; /* every rank's buffer as mapped here; [rank] is the own one */
  int64_t flags_off;   /* int32 flags[2][DRACO_TP_MAX_WORLD] in every buffer */
  int64_t counter_off; /* int32 step counter in every buffer */
  /* per GEMV problem: byte offset of this rank's output block (step parity
   * 0) in every buffer, and the bytes from the parity-0 to the parity-1 block */
  int64_t y_off[DRACO_GEMV_MAX_PROBLEMS];
  int64_t parity_stride[DRACO_GEMV_MAX_PROBLEMS];
} draco_tp_exchange;

/* Grouped GEMV of this rank's shards whose outputs go to every rank: the
 * value y[b][row] of problem i is stored at
 *   (float*)(buffers[q] + y_off[i] + parity * parity_stride[i])[b * ldy + row]
 * for every rank q (problems[i].y is not used and may be NULL).  The step's
 * epoch is the own buffer's step counter + 1 and its parity the epoch's.
 * When every CTA is done, the last one stores the epoch (negated if the
 * launch aborted) into flags[parity][rank] of every buffer and the epoch
 * into the own counter.  Workspace as for draco_gguf_gemv_grouped. */
int draco_gguf_gemv_grouped_tp(const draco_gemv_problem* problems, int n_problems, int batch,
                               const draco_tp_exchange* ex, void* workspace, size_t workspace_bytes,
                               void* stream);

/* The end of the step on this rank.  Waits (bounded, 1 s) until every
 * rank's flag for the step holds the step's epoch, then, over the own buffer
 * at the step's parity,
 *   gather_out[q][b][j] = buffer[gather_off + parity * gather_stride][q][b][j]
 *   reduce_out[b][j]    = sum over q of buffer[reduce_off + parity * reduce_stride][q][b][j]
 * (fp32; q < world, b < batch, j < the width; a width of 0 skips that part).
 * Launch it after the step's draco_gguf_gemv_grouped_tp on the same stream:
 * it first waits (griddepcontrol.wait) for that launch to complete and then
 * spins only on the other GPUs' flags.  *status (device int32, may be NULL)
 * becomes DRACO_ERR_TIMEOUT when a rank's signal did not come and
 * DRACO_ERR_PEER when a rank reported an aborted step. */
int draco_tp_finish(const draco_tp_exchange* ex, int batch, int64_t gather_off, int64_t gather_stride,
                    int gather_width, float* gather_out, int64_t reduce_off, int64_t reduce_stride,
                    int reduce_width, float* reduce_out, int* status, void* stream);

/* One weight of a prefill GEMM launch: Y = X @ dequant(W)^T.
 *   w      : TILED weight [n_rows, k] of type qtype (16-byte aligned)
 *   x      : bf16 [m, k] row-major, row stride ldx elements (16-byte aligned,
 *            ldx a multiple of 8)
 *   y      : [m, n_rows] of ydtype (DRACO_DTYPE_BF16 or DRACO_DTYPE_F32), row
 *            stride ldy elements
 * Replaces executor._linear (executor.py:47-79) at prompt length, whose
 * matmul is GenericGemmKernel.matmul_f32 (generic.py:32-33). */
typedef struct draco_gemm_problem {
  int qtype;
  int ydtype;
  const void* w;
  const void* x;
  void* y;
  int64_t m;
  int64_t n_rows;
  int64_t k;
  int64_t ldx;
  int64_t ldy;
} draco_gemm_problem;

#define DRACO_GEMM_MAX_PROBLEMS 16

/* Prefill dequant-GEMM over 1..DRACO_GEMM_MAX_PROBLEMS weights in one
 * persistent launch: tcgen05 tensor-core MMAs (bf16 x bf16, fp32 accumulate
 * in tensor memory) fed by weights dequantized to bf16 in shared memory.
 * `status` is NULL or a device int that the kernel sets to a DRACO_* code if
 * a device-side wait runs out (it never traps).  `problems` is a host array. */
int draco_gguf_gemm(const draco_gemm_problem* problems, int n_problems, int* status, void* stream);

/* draco_gguf_gemm with the tokens of each problem counted on the device:
 * problems[i].m is the CAPACITY (rows x and y hold), rows[i] (device int32,
 * in the caller's problem order, written by an earlier kernel on the stream)
 * the tokens actually present (clamped to 0..m).  Tokens past rows[i] are not
 * multiplied; their rows of y up to the next multiple of 32 may be written
 * with values of no meaning, so y must hold the capacity.  Lets a
 * mixture-of-experts layer run its experts' GEMMs on device-computed routing
 * without a host synchronisation.  Replaces the per-expert loop of
 * ExpertGroup.forward (draco/models/moe/expert.py:77-116), whose token counts
 * are host values. */
int draco_gguf_gemm_rows(const draco_gemm_problem* problems, int n_problems, const int* rows, int* status,
                         void* stream);

/* SwiGLU product of a gated MLP between its gate/up and down projections:
 * out[i] = bf16(silu(gate[i]) * up[i]) in fp32 with one rounding, n bf16
 * elements, all three pointers 16-byte aligned (out may alias gate or up).
 * Replaces act_fn(gate_proj(x)) * up_proj(x) of the reference's
 * Expert.forward (draco/models/moe/expert.py:47-49). */
int draco_swiglu_bf16(const void* gate, const void* up, void* out, int64_t n, void* stream);

/* Row-counted bf16 form for experts whose token counts live on the device:
 * gate, up and out are `groups` blocks of [cap_rows, width] bf16 (row-major,
 * block g at element g * cap_rows * width); only the first rows[g] rows of
 * block g are computed (rows: device int32 [groups], clamped to cap_rows).
 * width % 8 == 0, pointers 16-byte aligned, out may alias gate or up.
 * Replaces the same step of Expert.forward (draco/models/moe/expert.py:47-49)
 * for all experts of a layer at once. */
int draco_swiglu_bf16_rows(const void* gate, const void* up, void* out, int groups, int64_t cap_rows,
                           int64_t width, const int* rows, void* stream);

/* fp32 form for decode activations: out = silu(gate) * up over n fp32
 * values (expf as CUDA provides it), 16-byte aligned, out may alias gate.
 * Replaces the activation step of draco/kernels/ops.py:114-137
 * (fused_swiGLU) between the gate/up and down GEMVs. */
int draco_swiglu_f32(const float* gate, const float* up, float* out, int64_t n, void* stream);

/* RMSNorm, out = x * rsqrt(mean(x^2) + eps) * weight per row of x [rows, k]
 * (row-major, contiguous), fp32 arithmetic in the order of
 * draco/kernels/ops.py:29-50 (fused_rms_norm); x and out DRACO_DTYPE_F32 or
 * DRACO_DTYPE_BF16 (`dtype`), weight fp32 [k]; out may alias x.  Ahead of a
 * GEMV the norm can instead be fused into the activation read
 * (draco_gguf_gemv_grouped_ex, DRACO_INPUT_RMSNORM). */
int draco_rmsnorm(const void* x, const float* weight, void* out, int64_t rows, int64_t k, float eps, int dtype,
                  void* stream);

/* ---- attention of the GPU decode step (llama family) -------------------
 * Key/value cache per layer: fp32 [n_slots][kv_heads][capacity][head_dim];
 * token i of a call belongs to cache slot seq[i] at absolute position pos[i]
 * (device int32 arrays).  Tokens whose slot or position falls outside the
 * cache are skipped (no memory access; their attention output is zero).
 *
 * Rotary position embedding, rotate-half form (draco/runtime/cpu/ops.py:
 * 86-95: x1' = x1 c - x2 s, x2' = x2 c + x1 s, no fused multiply-add), with
 * cos / sin tables [max_positions, head_dim / 2] fp32 built as
 * build_rope_cache (ops.py:77-83) builds them: q [n, heads, head_dim] is
 * rotated in place; k [n, kv_heads, head_dim] is rotated into the cache row
 * pos[i] of slot seq[i] and v copied beside it (attention.py: the cache
 * append of prefill / decode).  head_dim even, heads a multiple of kv_heads. */
int draco_rope_kv_append(float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                         const float* cos_table, const float* sin_table, const int* seq, const int* pos, int n,
                         int heads, int kv_heads, int head_dim, int capacity, int n_slots, void* stream);

/* Causal attention of n query tokens over their slots' cached keys 0..pos[i]
 * (CPUAttentionBackend.prefill / decode, draco/runtime/cpu/attention.py):
 * softmax(q K^T / sqrt(head_dim)) V in fp32, query head h reading key/value
 * head h / (heads / kv_heads); out [n, heads, head_dim].  max_pos bounds
 * every pos[i] (max_pos < capacity; positions above it count as outside).
 * The keys are taken in chunks of 32 (one CTA per token, head and chunk),
 * merged by the last chunk to finish through the caller's device workspace
 * of at least draco_attention_workspace_bytes(n, heads, head_dim, max_pos)
 * bytes, 16-byte aligned (DRACO_ERR_WORKSPACE otherwise), zeroed before its
 * first use (the kernels leave its counters at zero).  Its first int32 is a
 * status word: nonzero (DRACO_ERR_TIMEOUT) after a bounded wait for a copy
 * ran out, the outputs of that launch then being invalid; zero the
 * workspace again before reusing it.  head_dim a multiple of 4 up to 256;
 * caches 16-byte aligned. */
int draco_attention_cached(const float* q, const float* k_cache, const float* v_cache, const int* seq,
                           const int* pos, int max_pos, float* out, int n, int heads, int kv_heads, int head_dim,
                           int capacity, int n_slots, void* workspace, size_t workspace_bytes, void* stream);

/* The decode form of a step's attention in one launch: draco_rope_kv_append
 * followed by draco_attention_cached, for tokens that hold DISTINCT slots
 * (one new token per sequence, as in CPUExecutionBackend.forward_batch_decode,
 * draco/runtime/cpu/executor.py:343-396, and a one-token forward_step).  q
 * and k arrive unrotated and q is left so; each token's new key (rotated)
 * and value go to cache row pos[i] of slot seq[i], and the attention reads
 * rows 0..pos[i] - 1 from the cache.  Results equal the two-call form's:
 * the same rotation arithmetic and the same chunked attention.  Tokens of
 * one launch sharing a slot give undefined outputs (use the two-call form
 * for a prompt).  Workspace as for draco_attention_cached. */
int draco_attention_decode(const float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                           const float* cos_table, const float* sin_table, const int* seq, const int* pos,
                           int max_pos, float* out, int n, int heads, int kv_heads, int head_dim, int capacity,
                           int n_slots, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes draco_attention_cached / draco_attention_decode need (0
 * for invalid arguments). */
size_t draco_attention_workspace_bytes(int n, int heads, int head_dim, int max_pos);

/* Single-weight convenience form of draco_gguf_gemv_grouped. */
int draco_gguf_gemv(int qtype, const void* w_tiled, const float* x, float* y, const float* bias,
                    int batch, int64_t n_rows, int64_t k, void* workspace,
                    size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DRACO_GGUF_H */
