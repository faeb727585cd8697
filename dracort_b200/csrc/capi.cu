// capi.cu — the extern "C" surface declared in include/draco_gguf.h:
// argument checks, status codes, thread-local error strings, dispatch.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace draco {

static thread_local char g_err[512] = {0};

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
static int ok() {
  g_err[0] = 0;
  return DRACO_OK;
}
static int cuda_fail(cudaError_t e, const char* what) {
  return fail(DRACO_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

static bool type_ok(int qt) { return qt == kQ8_0 || is_q4x(qt) || qt == kQ4_K || qt == kQ5_K || qt == kQ6_K; }

// Shape / type / layout checks shared by the weight entry points.  Mirrors the
// reference's DracoFormatError cases (gguf.py:284-296).
static int check_weight(int qt, int layout, const void* p, int64_t n_rows, int64_t k, const char* fn) {
  if (!type_ok(qt))
    return fail(DRACO_ERR_TYPE, "%s: GGUF quantization type %d is not supported (supported: Q4_0=2, Q4_1=3, Q5_0=6, Q5_1=7, Q8_0=8, Q4_K=12, Q5_K=13, Q6_K=14)",
                fn, qt);
  if (layout != DRACO_LAYOUT_GGUF && layout != DRACO_LAYOUT_GGUF_DLAST && layout != DRACO_LAYOUT_TILED)
    return fail(DRACO_ERR_TYPE, "%s: unknown layout %d", fn, layout);
  if (n_rows < 0 || k < 0) return fail(DRACO_ERR_SHAPE, "%s: negative shape [%lld, %lld]", fn, (long long)n_rows,
                                       (long long)k);
  const int bs = block_size_of(qt);
  if (k % bs != 0)
    return fail(DRACO_ERR_SHAPE, "%s: row length %lld is not divisible by block size %d for ggml type %d", fn,
                (long long)k, bs, qt);
  if (n_rows > (int64_t)1 << 30 || k > (int64_t)1 << 30)
    return fail(DRACO_ERR_SHAPE, "%s: shape [%lld, %lld] too large", fn, (long long)n_rows, (long long)k);
  if (n_rows * k > 0 && p == nullptr) return fail(DRACO_ERR_ARG, "%s: null weight pointer", fn);
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if (layout == DRACO_LAYOUT_TILED && (a & 15)) return fail(DRACO_ERR_ALIGN, "%s: TILED weight must be 16-byte aligned", fn);
  if (layout != DRACO_LAYOUT_TILED && (a & 1)) return fail(DRACO_ERR_ALIGN, "%s: GGUF weight must be 2-byte aligned", fn);
  return DRACO_OK;
}

}  // namespace draco

using namespace draco;

extern "C" {

const char* draco_version(void) { return "draco_gguf 0.1.0 sm_100a"; }

const char* draco_last_error_string(void) { return g_err; }

int draco_gguf_block_geometry(int qtype, int* block_size, int* block_bytes) {
  if (!type_ok(qtype)) return fail(DRACO_ERR_TYPE, "block_geometry: unsupported ggml type %d", qtype);
  if (block_size) *block_size = block_size_of(qtype);
  if (block_bytes) *block_bytes = block_bytes_of(qtype);
  return ok();
}

int64_t draco_gguf_packed_bytes(int qtype, int64_t n_rows, int64_t k) {
  if (!type_ok(qtype) || n_rows < 0 || k < 0 || k % block_size_of(qtype)) return -1;
  return n_rows * (k / block_size_of(qtype)) * block_bytes_of(qtype);
}

int64_t draco_gguf_tiled_bytes(int qtype, int64_t n_rows, int64_t k) {
  if (!type_ok(qtype) || n_rows < 0 || k < 0 || k % block_size_of(qtype)) return -1;
  return tiled_total_bytes(tiled_geom(qtype, n_rows, k));
}

int draco_gguf_dequant(int qtype, int layout, const void* blocks, float* out, int64_t n_rows, int64_t k,
                       void* stream) {
  int rc = check_weight(qtype, layout, blocks, n_rows, k, "dequant");
  if (rc) return rc;
  if (n_rows * k == 0) return ok();
  if (!out) return fail(DRACO_ERR_ARG, "dequant: null output");
  if (reinterpret_cast<uintptr_t>(out) & 15) return fail(DRACO_ERR_ALIGN, "dequant: output must be 16-byte aligned");
  cudaError_t e = launch_dequant_f32(qtype, layout, blocks, out, n_rows, k, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "dequant");
}

int draco_gguf_dequant_bf16(int qtype, int layout, const void* blocks, uint16_t* out, int64_t n_rows, int64_t k,
                            void* stream) {
  int rc = check_weight(qtype, layout, blocks, n_rows, k, "dequant_bf16");
  if (rc) return rc;
  if (n_rows * k == 0) return ok();
  if (!out) return fail(DRACO_ERR_ARG, "dequant_bf16: null output");
  if (reinterpret_cast<uintptr_t>(out) & 15)
    return fail(DRACO_ERR_ALIGN, "dequant_bf16: output must be 16-byte aligned");
  cudaError_t e = launch_dequant_bf16(qtype, layout, blocks, out, n_rows, k, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "dequant_bf16");
}

int draco_gguf_repack(int qtype, int src_layout, const void* src, void* dst, int64_t n_rows, int64_t k,
                      void* stream) {
  if (src_layout == DRACO_LAYOUT_TILED) return fail(DRACO_ERR_TYPE, "repack: source must be a GGUF layout");
  int rc = check_weight(qtype, src_layout, src, n_rows, k, "repack");
  if (rc) return rc;
  if (n_rows * k == 0) return ok();
  if (!dst) return fail(DRACO_ERR_ARG, "repack: null destination");
  if (reinterpret_cast<uintptr_t>(dst) & 15) return fail(DRACO_ERR_ALIGN, "repack: destination must be 16-byte aligned");
  cudaError_t e = launch_repack(qtype, src_layout, src, dst, n_rows, k, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "repack");
}

// need_y: false for the tensor-parallel form, whose outputs go to the exchange buffers
static int check_gemv_problems(const draco_gemv_problem* probs, int n, int batch, bool need_y = true) {
  if (!probs || n < 1 || n > DRACO_GEMV_MAX_PROBLEMS)
    return fail(DRACO_ERR_ARG, "gemv: need 1..%d problems, got %d", DRACO_GEMV_MAX_PROBLEMS, n);
  if (batch < 1 || batch > DRACO_GEMV_MAX_BATCH)
    return fail(DRACO_ERR_ARG, "gemv: batch %d outside 1..%d", batch, DRACO_GEMV_MAX_BATCH);
  for (int i = 0; i < n; ++i) {
    const draco_gemv_problem& q = probs[i];
    int rc = check_weight(q.qtype, DRACO_LAYOUT_TILED, q.w, q.n_rows, q.k, "gemv");
    if (rc) return rc;
    if (q.n_rows * q.k > 0 && (!q.x || (need_y && !q.y)))
      return fail(DRACO_ERR_ARG, "gemv: problem %d has a null x or y", i);
    if (q.ldx < q.k || q.ldy < q.n_rows)
      return fail(DRACO_ERR_SHAPE, "gemv: problem %d leading dimensions too small", i);
    if (q.flags & ~DRACO_GEMV_ACCUMULATE)
      return fail(DRACO_ERR_ARG, "gemv: problem %d has unknown flags 0x%x", i, q.flags);
  }
  return DRACO_OK;
}

size_t draco_gguf_gemv_workspace_bytes(const draco_gemv_problem* probs, int n_problems, int batch) {
  // the size does not depend on y (the tensor-parallel form has none)
  if (check_gemv_problems(probs, n_problems, batch, false)) return 0;
  return gemv_workspace_bytes(probs, n_problems, batch);
}

static int check_attention(int n, int heads, int kv_heads, int head_dim, int capacity, int n_slots, const char* fn) {
  if (n < 0 || heads < 1 || kv_heads < 1 || heads % kv_heads || head_dim < 2 || (head_dim & 1) || capacity < 1 ||
      n_slots < 1)
    return fail(DRACO_ERR_SHAPE, "%s: invalid shape (n %d, heads %d, kv_heads %d, head_dim %d, capacity %d, slots %d)",
                fn, n, heads, kv_heads, head_dim, capacity, n_slots);
  return DRACO_OK;
}

int draco_rope_kv_append(float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                         const float* cos_table, const float* sin_table, const int* seq, const int* pos, int n,
                         int heads, int kv_heads, int head_dim, int capacity, int n_slots, void* stream) {
  int rc = check_attention(n, heads, kv_heads, head_dim, capacity, n_slots, "rope_kv_append");
  if (rc) return rc;
  if (n > 0 && (!q || !k || !v || !k_cache || !v_cache || !cos_table || !sin_table || !seq || !pos))
    return fail(DRACO_ERR_ARG, "rope_kv_append: null pointer");
  char msg[160] = {0};
  rc = attention_launch(0, q, k, v, k_cache, v_cache, cos_table, sin_table, seq, pos, nullptr, n, heads, kv_heads,
                        head_dim, capacity, n_slots, capacity - 1, nullptr, 0, (cudaStream_t)stream, msg, sizeof(msg));
  return rc ? fail(rc, "%s", msg) : DRACO_OK;
}

int draco_attention_cached(const float* q, const float* k_cache, const float* v_cache, const int* seq,
                           const int* pos, int max_pos, float* out, int n, int heads, int kv_heads, int head_dim,
                           int capacity, int n_slots, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_attention(n, heads, kv_heads, head_dim, capacity, n_slots, "attention_cached");
  if (rc) return rc;
  if (max_pos < 0 || max_pos >= capacity)
    return fail(DRACO_ERR_SHAPE, "attention_cached: max_pos %d outside the cache capacity %d", max_pos, capacity);
  if (n > 0 && (!q || !k_cache || !v_cache || !seq || !pos || !out))
    return fail(DRACO_ERR_ARG, "attention_cached: null pointer");
  char msg[160] = {0};
  rc = attention_launch(1, const_cast<float*>(q), nullptr, nullptr, const_cast<float*>(k_cache),
                        const_cast<float*>(v_cache), nullptr, nullptr, seq, pos, out, n, heads, kv_heads, head_dim,
                        capacity, n_slots, max_pos, static_cast<float*>(workspace), workspace_bytes,
                        (cudaStream_t)stream, msg, sizeof(msg));
  return rc ? fail(rc, "%s", msg) : DRACO_OK;
}

int draco_attention_decode(const float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                           const float* cos_table, const float* sin_table, const int* seq, const int* pos,
                           int max_pos, float* out, int n, int heads, int kv_heads, int head_dim, int capacity,
                           int n_slots, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_attention(n, heads, kv_heads, head_dim, capacity, n_slots, "attention_decode");
  if (rc) return rc;
  if (max_pos < 0 || max_pos >= capacity)
    return fail(DRACO_ERR_SHAPE, "attention_decode: max_pos %d outside the cache capacity %d", max_pos, capacity);
  if (n > 0 && (!q || !k || !v || !k_cache || !v_cache || !cos_table || !sin_table || !seq || !pos || !out))
    return fail(DRACO_ERR_ARG, "attention_decode: null pointer");
  char msg[160] = {0};
  rc = attention_launch(2, const_cast<float*>(q), k, v, k_cache, v_cache, cos_table, sin_table, seq, pos, out, n,
                        heads, kv_heads, head_dim, capacity, n_slots, max_pos, static_cast<float*>(workspace),
                        workspace_bytes, (cudaStream_t)stream, msg, sizeof(msg));
  return rc ? fail(rc, "%s", msg) : DRACO_OK;
}

size_t draco_attention_workspace_bytes(int n, int heads, int head_dim, int max_pos) {
  if (n < 0 || heads < 1 || head_dim < 1 || max_pos < 0) return 0;
  return attention_workspace_bytes(n, heads, head_dim, max_pos);
}

int draco_gguf_gemv_launch_count(const draco_gemv_problem* probs, int n_problems, int batch) {
  if (check_gemv_problems(probs, n_problems, batch, false)) return -1;
  return gemv_launch_count(probs, n_problems, batch);
}

int draco_gguf_gemv_grouped(const draco_gemv_problem* probs, int n_problems, int batch, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int rc = check_gemv_problems(probs, n_problems, batch);
  if (rc) return rc;
  char msg[256] = {0};
  rc = gemv_launch(probs, n_problems, batch, workspace, workspace_bytes, (cudaStream_t)stream, msg, sizeof(msg));
  if (rc) return fail(rc, "%s", msg);
  return ok();
}

int draco_gguf_gemv_grouped_ex(const draco_gemv_problem* probs, const draco_gemv_input* inputs, int n_problems,
                               int batch, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_gemv_problems(probs, n_problems, batch);
  if (rc) return rc;
  for (int i = 0; inputs && i < n_problems; ++i) {
    const draco_gemv_input& in = inputs[i];
    if (in.mode != DRACO_INPUT_PLAIN && in.mode != DRACO_INPUT_RMSNORM && in.mode != DRACO_INPUT_SWIGLU)
      return fail(DRACO_ERR_ARG, "gemv_ex: problem %d has an unknown input mode %d", i, in.mode);
    if (in.mode != DRACO_INPUT_PLAIN && !in.aux)
      return fail(DRACO_ERR_ARG, "gemv_ex: problem %d needs its aux vector", i);
    if (in.mode == DRACO_INPUT_RMSNORM && !(in.eps >= 0.f))
      return fail(DRACO_ERR_ARG, "gemv_ex: problem %d has a negative or NaN eps", i);
    if (in.mode == DRACO_INPUT_SWIGLU && in.ldaux < probs[i].k)
      return fail(DRACO_ERR_SHAPE, "gemv_ex: problem %d aux row stride too small", i);
  }
  char msg[256] = {0};
  rc = gemv_launch(probs, n_problems, batch, workspace, workspace_bytes, (cudaStream_t)stream, msg, sizeof(msg),
                   inputs);
  if (rc) return fail(rc, "%s", msg);
  return ok();
}

int draco_gguf_gemv_grouped_noalloc(const draco_gemv_problem* probs, int n_problems, int batch, void* stream) {
  int rc = check_gemv_problems(probs, n_problems, batch);
  if (rc) return rc;
  char msg[256] = {0};
  rc = gemv_launch_noalloc(probs, n_problems, batch, (cudaStream_t)stream, msg, sizeof(msg));
  if (rc) return fail(rc, "%s", msg);
  return ok();
}

int draco_gguf_gemv_noalloc_status(int* status, void* stream) {
  if (!status) return fail(DRACO_ERR_ARG, "gemv_noalloc_status: null status pointer");
  char msg[256] = {0};
  const int rc = gemv_noalloc_status(status, (cudaStream_t)stream, msg, sizeof(msg));
  if (rc) return fail(rc, "%s", msg);
  return ok();
}

static int check_gemm_problems(const draco_gemm_problem* probs, int n_problems) {
  if (!probs || n_problems < 1 || n_problems > DRACO_GEMM_MAX_PROBLEMS)
    return fail(DRACO_ERR_ARG, "gemm: need 1..%d problems, got %d", DRACO_GEMM_MAX_PROBLEMS, n_problems);
  for (int i = 0; i < n_problems; ++i) {
    const draco_gemm_problem& q = probs[i];
    int rc = check_weight(q.qtype, DRACO_LAYOUT_TILED, q.w, q.n_rows, q.k, "gemm");
    if (rc) return rc;
    if (q.m < 0) return fail(DRACO_ERR_SHAPE, "gemm: problem %d has negative m", i);
    if (q.m * q.n_rows * q.k == 0) continue;
    if (!q.x || !q.y) return fail(DRACO_ERR_ARG, "gemm: problem %d has a null x or y", i);
    if (q.ydtype != DRACO_DTYPE_BF16 && q.ydtype != DRACO_DTYPE_F32)
      return fail(DRACO_ERR_TYPE, "gemm: problem %d output dtype %d unsupported", i, q.ydtype);
    if (q.ldx < q.k || q.ldy < q.n_rows) return fail(DRACO_ERR_SHAPE, "gemm: problem %d leading dimensions too small", i);
    if ((reinterpret_cast<uintptr_t>(q.x) & 15) || (q.ldx % 8))
      return fail(DRACO_ERR_ALIGN, "gemm: problem %d: x must be 16-byte aligned with ldx a multiple of 8", i);
    if (q.m > (int64_t)1 << 30) return fail(DRACO_ERR_SHAPE, "gemm: problem %d m too large", i);
  }
  return DRACO_OK;
}

int draco_gguf_gemm(const draco_gemm_problem* probs, int n_problems, int* status, void* stream) {
  int rc = check_gemm_problems(probs, n_problems);
  if (rc) return rc;
  char msg[256] = {0};
  rc = gemm_launch(probs, n_problems, nullptr, status, (cudaStream_t)stream, msg, sizeof(msg));
  if (rc) return fail(rc, "%s", msg);
  return ok();
}

int draco_gguf_gemm_rows(const draco_gemm_problem* probs, int n_problems, const int* rows, int* status,
                         void* stream) {
  if (!rows) return fail(DRACO_ERR_ARG, "gemm_rows: null row counts");
  if (reinterpret_cast<uintptr_t>(rows) & 3) return fail(DRACO_ERR_ALIGN, "gemm_rows: row counts not 4-byte aligned");
  int rc = check_gemm_problems(probs, n_problems);
  if (rc) return rc;
  char msg[256] = {0};
  rc = gemm_launch(probs, n_problems, rows, status, (cudaStream_t)stream, msg, sizeof(msg));
  if (rc) return fail(rc, "%s", msg);
  return ok();
}

int draco_gguf_gemv(int qtype, const void* w_tiled, const float* x, float* y, const float* bias, int batch,
                    int64_t n_rows, int64_t k, void* workspace, size_t workspace_bytes, void* stream) {
  draco_gemv_problem p;
  memset(&p, 0, sizeof(p));
  p.qtype = qtype;
  p.w = w_tiled;
  p.x = x;
  p.y = y;
  p.bias = bias;
  p.n_rows = n_rows;
  p.k = k;
  p.ldx = k;
  p.ldy = n_rows;
  return draco_gguf_gemv_grouped(&p, 1, batch, workspace, workspace_bytes, stream);
}

int draco_tp_buffer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(DRACO_ERR_ARG, "tp_buffer_alloc: null result pointer or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "tp_buffer_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "tp_buffer_alloc: cudaMemset");
  }
  *ptr = p;
  return ok();
}

int draco_tp_buffer_free(void* ptr) {
  if (!ptr) return ok();
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? ok() : cuda_fail(e, "tp_buffer_free");
}

int draco_ipc_get_handle(void* ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == DRACO_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle) return fail(DRACO_ERR_ARG, "ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_fail(e, "ipc_get_handle");
  memcpy(handle, &h, sizeof(h));
  return ok();
}

int draco_ipc_open(const void* handle, void** peer_ptr) {
  if (!handle || !peer_ptr) return fail(DRACO_ERR_ARG, "ipc_open: null pointer");
  *peer_ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "ipc_open");
  *peer_ptr = p;
  return ok();
}

int draco_ipc_close(void* peer_ptr) {
  if (!peer_ptr) return ok();
  cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  return e == cudaSuccess ? ok() : cuda_fail(e, "ipc_close");
}

int draco_gguf_gemv_grouped_tp(const draco_gemv_problem* probs, int n_problems, int batch,
                               const draco_tp_exchange* ex, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_gemv_problems(probs, n_problems, batch, false);
  if (rc) return rc;
  for (int i = 0; i < n_problems; ++i)
    if (probs[i].flags)
      return fail(DRACO_ERR_ARG, "gemv_tp: problem %d has flags 0x%x (the tensor-parallel outputs take none)", i,
                  probs[i].flags);
  if (!ex) return fail(DRACO_ERR_ARG, "gemv_tp: null exchange description");
  char msg[256] = {0};
  rc = gemv_launch_tp(probs, n_problems, batch, ex, workspace, workspace_bytes, (cudaStream_t)stream, msg,
                      sizeof(msg));
  if (rc) return fail(rc, "%s", msg);
  return ok();
}

int draco_tp_finish(const draco_tp_exchange* ex, int batch, int64_t gather_off, int64_t gather_stride,
                    int gather_width, float* gather_out, int64_t reduce_off, int64_t reduce_stride,
                    int reduce_width, float* reduce_out, int* status, void* stream) {
  if (!ex) return fail(DRACO_ERR_ARG, "tp_finish: null exchange description");
  char msg[256] = {0};
  int rc = tp_finish_launch(ex, batch, gather_off, gather_stride, gather_width, gather_out, reduce_off,
                            reduce_stride, reduce_width, reduce_out, status, (cudaStream_t)stream, msg, sizeof(msg));
  if (rc) return fail(rc, "%s", msg);
  return ok();
}

}  // extern "C"

int draco_swiglu_bf16(const void* gate, const void* up, void* out, int64_t n, void* stream) {
  if (n < 0) return fail(DRACO_ERR_SHAPE, "swiglu: negative length");
  if (n == 0) return ok();
  if (!gate || !up || !out) return fail(DRACO_ERR_ARG, "swiglu: null pointer");
  if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(DRACO_ERR_ALIGN, "swiglu: gate, up and out must be 16-byte aligned");
  cudaError_t e = draco::launch_swiglu_bf16(gate, up, out, n, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "swiglu");
}

int draco_swiglu_bf16_rows(const void* gate, const void* up, void* out, int groups, int64_t cap_rows,
                           int64_t width, const int* rows, void* stream) {
  if (groups < 0 || groups > 65535 || cap_rows < 0 || width < 0)
    return fail(DRACO_ERR_SHAPE, "swiglu_rows: bad groups / rows / width");
  if (groups == 0 || cap_rows == 0 || width == 0) return ok();
  if (!gate || !up || !out || !rows) return fail(DRACO_ERR_ARG, "swiglu_rows: null pointer");
  if (width % 8) return fail(DRACO_ERR_SHAPE, "swiglu_rows: width must be a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(DRACO_ERR_ALIGN, "swiglu_rows: gate, up and out must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(rows) & 3) return fail(DRACO_ERR_ALIGN, "swiglu_rows: rows not 4-byte aligned");
  cudaError_t e = draco::launch_swiglu_bf16_rows(gate, up, out, groups, cap_rows, width, rows, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "swiglu_rows");
}

int draco_rmsnorm(const void* x, const float* weight, void* out, int64_t rows, int64_t k, float eps, int dtype,
                  void* stream) {
  if (rows < 0 || k < 0) return fail(DRACO_ERR_SHAPE, "rmsnorm: negative shape");
  if (rows == 0 || k == 0) return ok();
  if (!x || !weight || !out) return fail(DRACO_ERR_ARG, "rmsnorm: null pointer");
  if (dtype != DRACO_DTYPE_F32 && dtype != DRACO_DTYPE_BF16) return fail(DRACO_ERR_TYPE, "rmsnorm: dtype %d", dtype);
  if (!(eps >= 0.f)) return fail(DRACO_ERR_ARG, "rmsnorm: negative or NaN eps");
  cudaError_t e = draco::launch_rmsnorm(x, weight, out, rows, k, eps, dtype == DRACO_DTYPE_BF16, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "rmsnorm");
}

int draco_swiglu_f32(const float* gate, const float* up, float* out, int64_t n, void* stream) {
  if (n < 0) return fail(DRACO_ERR_SHAPE, "swiglu_f32: negative length");
  if (n == 0) return ok();
  if (!gate || !up || !out) return fail(DRACO_ERR_ARG, "swiglu_f32: null pointer");
  if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(DRACO_ERR_ALIGN, "swiglu_f32: gate, up and out must be 16-byte aligned");
  cudaError_t e = draco::launch_swiglu_f32(gate, up, out, n, (cudaStream_t)stream);
  return e == cudaSuccess ? ok() : cuda_fail(e, "swiglu_f32");
}
