// C ABI of the pagedkv library: argument validation, kernel selection and the
// device error word. Declarations and contracts live in include/pagedkv.h.
#include <nvtx3/nvToolsExt.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"
#include "decode_tc.h"
#include "launch.h"

namespace pagedkv {

// One error word per device (each device holds its own copy of this module).
__device__ unsigned int g_error_flags = 0;

namespace {

thread_local std::string t_last_error;
thread_local int32_t t_last_launches = 0;
thread_local const char *t_last_kernel = "none";

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(PAGEDKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// One NVTX range per call of a launching entry point, named after it, so a
// profiler timeline (nsys, ncu --nvtx) shows every layer's host call around the
// kernels it launched. With no tool attached a range costs a pointer test.
struct NvtxRange {
  explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange &) = delete;
  NvtxRange &operator=(const NvtxRange &) = delete;
};

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int num_sms = 0;
  unsigned int *err = nullptr;
};

std::mutex g_dev_mu;
DeviceInfo g_dev[kMaxDevices];

// Per-device facts resolved once: SM count and the address of this device's
// error word (the symbol's host-side name is not a device address).
int device_info(DeviceInfo *out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(PAGEDKV_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo &d = g_dev[dev];
  if (d.err == nullptr) {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_error_flags);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(error word)");
    d.num_sms = sms;
    d.err = static_cast<unsigned int *>(p);
  }
  *out = d;
  return PAGEDKV_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool supported_head_dim(int d) { return d == 32 || d == 64 || d == 128 || d == 256; }

// Workspace layout for a split-K launch: ws_acc then ws_ml.
size_t simt_workspace_bytes(int32_t num_seqs, int32_t hq, int32_t head_dim, const SplitPlan &plan) {
  if (plan.num_splits <= 1) return 0;
  const size_t slots = (size_t)num_seqs * hq * plan.num_splits;
  const size_t acc = slots * head_dim * sizeof(float);
  const size_t ml = slots * sizeof(float2);
  return kWorkspaceHeaderBytes + ((acc + 255) / 256) * 256 + ml;
}

}  // namespace

void set_last_error_message(const char *msg) { t_last_error = msg; }

}  // namespace pagedkv

using namespace pagedkv;

extern "C" {

const char *pagedkv_version(void) { return "pagedkv-b200 0.1.0 sm_100a"; }

const char *pagedkv_last_error(void) { return t_last_error.c_str(); }

int32_t pagedkv_last_decode_launches(void) { return t_last_launches; }

const char *pagedkv_last_decode_kernel(void) { return t_last_kernel; }

size_t pagedkv_decode_attention_workspace_size(int32_t num_seqs, int32_t num_q_heads,
                                               int32_t num_kv_heads, int32_t head_dim,
                                               int32_t block_size, int32_t max_blocks_per_seq,
                                               int32_t dtype) {
  (void)dtype;
  if (num_seqs <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return 0;
  DeviceInfo di;
  if (device_info(&di) != PAGEDKV_OK) return 0;
  const int group = num_q_heads / num_kv_heads;
  const int64_t max_tokens = (int64_t)max_blocks_per_seq * block_size;
  const int32_t mt = (int32_t)(max_tokens > 0x7fffffff ? 0x7fffffff : max_tokens);
  if (tc_eligible(num_q_heads, num_kv_heads, head_dim, block_size)) {
    return tc_workspace_bytes(num_seqs, num_q_heads, num_kv_heads, head_dim, mt, di.num_sms);
  }
  const SplitPlan plan = plan_simt_splits(num_seqs, num_kv_heads, group, mt, di.num_sms);
  return simt_workspace_bytes(num_seqs, num_q_heads, head_dim, plan);
}

}  // extern "C"

namespace {

// Decode attention, optionally with the decode append fused into the
// tensor-core launch (`ap`); shared by the two entry points.
int decode_entry(void *out, int64_t out_stride_seq, int64_t out_stride_head, const void *q,
                 int64_t q_stride_seq, int64_t q_stride_head, const void *k_cache, const void *v_cache,
                 const int32_t *block_tables, int64_t block_tables_stride, const int32_t *seq_lens,
                 int32_t uniform_seq_len, int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                 int32_t head_dim, int64_t num_blocks, int32_t block_size, int32_t max_blocks_per_seq,
                 float scale, int32_t dtype, void *workspace, size_t workspace_bytes, void *stream,
                 const AppendParams *ap) {
  t_last_launches = 0;
  t_last_kernel = "none";
  if (num_seqs < 0) return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_seqs must be >= 0 (got %d)", num_seqs);
  if (num_seqs == 0) return PAGEDKV_OK;
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT,
                "num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)", num_q_heads,
                num_kv_heads);
  if (!supported_head_dim(head_dim))
    return fail(PAGEDKV_ERR_UNSUPPORTED, "head_dim %d not built (32, 64, 128, 256)", head_dim);
  if (dtype != PAGEDKV_DTYPE_F16 && dtype != PAGEDKV_DTYPE_BF16)
    return fail(PAGEDKV_ERR_UNSUPPORTED, "dtype %d not supported (0=f16, 1=bf16)", dtype);
  if (block_size <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT,
                "block_size (%d), num_blocks (%lld), max_blocks_per_seq (%d) must be > 0",
                block_size, (long long)num_blocks, max_blocks_per_seq);
  if (!out || !q || !k_cache || !v_cache || !block_tables)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!seq_lens && uniform_seq_len < 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "uniform_seq_len must be >= 0");
  if (!aligned16(out) || !aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) ||
      (q_stride_seq % 8) || (q_stride_head % 8) || (out_stride_seq % 8) || (out_stride_head % 8))
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT,
                "q/out/k_cache/v_cache must be 16-byte aligned with strides that are multiples "
                "of 8 elements");
  if ((int64_t)max_blocks_per_seq * block_size > 0x7fffffffLL)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "max_blocks_per_seq * block_size exceeds 2^31-1");

  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != PAGEDKV_OK) return rc;

  DecodeParams p{};
  p.out = out;
  p.o_ss = out_stride_seq;
  p.o_sh = out_stride_head;
  p.q = q;
  p.q_ss = q_stride_seq;
  p.q_sh = q_stride_head;
  p.k = k_cache;
  p.v = v_cache;
  p.bt = block_tables;
  p.bt_s = block_tables_stride;
  p.lens = seq_lens;
  p.uniform_len = uniform_seq_len;
  p.num_seqs = num_seqs;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.group = num_q_heads / num_kv_heads;
  p.head_dim = head_dim;
  p.block_size = block_size;
  p.max_blocks = max_blocks_per_seq;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * kLog2e;
  p.err = di.err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int32_t max_tokens = max_blocks_per_seq * block_size;

  if (ap != nullptr && !tc_eligible(num_q_heads, num_kv_heads, head_dim, block_size))
    return fail(PAGEDKV_ERR_UNSUPPORTED,
                "fused append: this shape (block_size %d) runs on the CUDA-core kernel, which has no fused "
                "append; call pagedkv_kv_append then pagedkv_decode_attention",
                block_size);
  if (tc_eligible(num_q_heads, num_kv_heads, head_dim, block_size)) {
    const size_t need = tc_workspace_bytes(num_seqs, num_q_heads, num_kv_heads, head_dim,
                                           max_tokens, di.num_sms);
    if (need > workspace_bytes || (need > 0 && workspace == nullptr))
      return fail(PAGEDKV_ERR_WORKSPACE, "workspace too small: need %zu bytes, got %zu", need,
                  workspace_bytes);
    int launches = 0;
    rc = tc_launch(p, dtype, workspace, need, di.num_sms, st, &launches, &t_last_error, ap);
    if (rc != PAGEDKV_OK) return rc;
    t_last_launches = launches;
    t_last_kernel = "tc";
    return PAGEDKV_OK;
  }

  const SplitPlan plan = plan_simt_splits(num_seqs, num_kv_heads, p.group, max_tokens, di.num_sms);
  p.split_tokens = plan.split_tokens;
  p.num_splits = plan.num_splits;
  const size_t need = simt_workspace_bytes(num_seqs, num_q_heads, head_dim, plan);
  if (need > workspace_bytes || (need > 0 && workspace == nullptr))
    return fail(PAGEDKV_ERR_WORKSPACE, "workspace too small: need %zu bytes, got %zu", need,
                workspace_bytes);
  if (need > 0) {
    const size_t slots = (size_t)num_seqs * num_q_heads * plan.num_splits;
    const size_t acc = ((slots * head_dim * sizeof(float) + 255) / 256) * 256;
    char *base = static_cast<char *>(workspace) + kWorkspaceHeaderBytes;
    p.ws_acc = reinterpret_cast<float *>(base);
    p.ws_ml = reinterpret_cast<float2 *>(base + acc);
  }
  cudaError_t e = launch_decode_simt(p, dtype, st);
  if (e != cudaSuccess) return cuda_fail(e, "decode_simt launch");
  int launches = 1;
  if (plan.num_splits > 1) {
    e = launch_decode_combine(p, dtype, st);
    if (e != cudaSuccess) return cuda_fail(e, "decode_combine launch");
    ++launches;
  }
  t_last_launches = launches;
  t_last_kernel = "simt";
  return PAGEDKV_OK;
}

}  // namespace

extern "C" {

int pagedkv_decode_attention(void *out, int64_t out_stride_seq, int64_t out_stride_head,
                             const void *q, int64_t q_stride_seq, int64_t q_stride_head,
                             const void *k_cache, const void *v_cache,
                             const int32_t *block_tables, int64_t block_tables_stride,
                             const int32_t *seq_lens, int32_t uniform_seq_len, int32_t num_seqs,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             int64_t num_blocks, int32_t block_size, int32_t max_blocks_per_seq,
                             float scale, int32_t dtype, void *workspace, size_t workspace_bytes,
                             void *stream) {
  NvtxRange nvtx("pagedkv_decode_attention");
  return decode_entry(out, out_stride_seq, out_stride_head, q, q_stride_seq, q_stride_head, k_cache, v_cache,
                      block_tables, block_tables_stride, seq_lens, uniform_seq_len, num_seqs, num_q_heads,
                      num_kv_heads, head_dim, num_blocks, block_size, max_blocks_per_seq, scale, dtype,
                      workspace, workspace_bytes, stream, nullptr);
}

int pagedkv_decode_attention_append(
    void *out, int64_t out_stride_seq, int64_t out_stride_head, const void *q, int64_t q_stride_seq,
    int64_t q_stride_head, void *k_cache, void *v_cache, const int32_t *block_tables,
    int64_t block_tables_stride, const int32_t *seq_lens, int32_t num_seqs, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t max_blocks_per_seq, const void *k_new, int64_t k_new_stride_seq, int64_t k_new_stride_head,
    const void *v_new, int64_t v_new_stride_seq, int64_t v_new_stride_head, const void *cos,
    const void *sin, int64_t cos_sin_stride, float scale, int32_t dtype, void *workspace,
    size_t workspace_bytes, void *stream) {
  NvtxRange nvtx("pagedkv_decode_attention_append");
  t_last_launches = 0;
  t_last_kernel = "none";
  if (!seq_lens) return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "fused append: seq_lens is required");
  if (!k_new || !v_new) return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "fused append: null k_new / v_new");
  if ((cos == nullptr) != (sin == nullptr))
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "fused append: pass both cos and sin, or neither");
  if (!aligned16(k_new) || !aligned16(v_new) || (k_new_stride_seq % 8) || (k_new_stride_head % 8) ||
      (v_new_stride_seq % 8) || (v_new_stride_head % 8) ||
      (cos && (!aligned16(cos) || !aligned16(sin) || (cos_sin_stride % 8))))
    return fail(PAGEDKV_ERR_UNSUPPORTED,
                "fused append: k_new / v_new (and cos / sin) must be 16-byte aligned with strides that are "
                "multiples of 8 elements");
  AppendParams ap{k_new, k_new_stride_seq, k_new_stride_head, v_new, v_new_stride_seq, v_new_stride_head,
                  cos, sin, cos_sin_stride};
  return decode_entry(out, out_stride_seq, out_stride_head, q, q_stride_seq, q_stride_head, k_cache, v_cache,
                      block_tables, block_tables_stride, seq_lens, 0, num_seqs, num_q_heads, num_kv_heads,
                      head_dim, num_blocks, block_size, max_blocks_per_seq, scale, dtype, workspace,
                      workspace_bytes, stream, &ap);
}

int pagedkv_kv_append(void *k_cache, void *v_cache, const void *k_new, int64_t k_new_stride_tok,
                      int64_t k_new_stride_head, const void *v_new, int64_t v_new_stride_tok,
                      int64_t v_new_stride_head, const int64_t *slot_mapping, int32_t num_tokens,
                      int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks,
                      int32_t block_size, int32_t dtype, void *stream) {
  NvtxRange nvtx("pagedkv_kv_append");
  if (num_tokens < 0) return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_tokens must be >= 0");
  if (num_tokens == 0) return PAGEDKV_OK;
  if (dtype != PAGEDKV_DTYPE_F16 && dtype != PAGEDKV_DTYPE_BF16)
    return fail(PAGEDKV_ERR_UNSUPPORTED, "dtype %d not supported (0=f16, 1=bf16)", dtype);
  if (num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_kv_heads, head_dim, block_size, num_blocks must be > 0");
  if (!k_cache || !v_cache || !k_new || !v_new || !slot_mapping)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != PAGEDKV_OK) return rc;
  const bool vec = (head_dim % 8 == 0) && aligned16(k_cache) && aligned16(v_cache) &&
                   aligned16(k_new) && aligned16(v_new) && (k_new_stride_tok % 8 == 0) &&
                   (k_new_stride_head % 8 == 0) && (v_new_stride_tok % 8 == 0) &&
                   (v_new_stride_head % 8 == 0);
  cudaError_t e = launch_kv_append(k_cache, v_cache, k_new, k_new_stride_tok, k_new_stride_head,
                                   v_new, v_new_stride_tok, v_new_stride_head, slot_mapping,
                                   num_tokens, num_kv_heads, head_dim, num_blocks * block_size,
                                   vec, di.err, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  return PAGEDKV_OK;
}

int pagedkv_copy_blocks(void *const *k_cache_ptrs, void *const *v_cache_ptrs, int32_t num_layers,
                        const int64_t *block_mapping, int32_t num_pairs, int64_t block_bytes,
                        int64_t num_blocks, void *stream) {
  NvtxRange nvtx("pagedkv_copy_blocks");
  if (num_pairs < 0 || num_layers < 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_pairs and num_layers must be >= 0");
  if (num_pairs == 0 || num_layers == 0) return PAGEDKV_OK;
  if (num_layers > 32767)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_layers %d exceeds 32767", num_layers);
  if (block_bytes <= 0 || (block_bytes % 16) != 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "block_bytes (%lld) must be a positive multiple of 16",
                (long long)block_bytes);
  if (!k_cache_ptrs || !v_cache_ptrs || !block_mapping)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != PAGEDKV_OK) return rc;
  cudaError_t e = launch_copy_blocks(k_cache_ptrs, v_cache_ptrs, num_layers, block_mapping,
                                     num_pairs, block_bytes, num_blocks, di.num_sms, di.err,
                                     static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "copy_blocks launch");
  return PAGEDKV_OK;
}

int pagedkv_kv_append_rope(void *q_out, int64_t q_out_stride_tok, int64_t q_out_stride_head, const void *q,
                           int64_t q_stride_tok, int64_t q_stride_head, int32_t num_q_heads, void *k_cache,
                           void *v_cache, const void *k_new, int64_t k_new_stride_tok,
                           int64_t k_new_stride_head, const void *v_new, int64_t v_new_stride_tok,
                           int64_t v_new_stride_head, const void *cos, const void *sin,
                           int64_t cos_sin_stride_tok, const int64_t *slot_mapping, int32_t num_tokens,
                           int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
                           int32_t dtype, void *stream) {
  NvtxRange nvtx("pagedkv_kv_append_rope");
  if (num_tokens < 0) return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_tokens must be >= 0");
  if (num_tokens == 0) return PAGEDKV_OK;
  if (dtype != PAGEDKV_DTYPE_F16 && dtype != PAGEDKV_DTYPE_BF16)
    return fail(PAGEDKV_ERR_UNSUPPORTED, "dtype %d not supported (0=f16, 1=bf16)", dtype);
  if (num_q_heads <= 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_q_heads, num_kv_heads, block_size, num_blocks must be > 0");
  if (head_dim <= 0 || (head_dim % 16) != 0)
    return fail(PAGEDKV_ERR_UNSUPPORTED, "head_dim (%d) must be a positive multiple of 16", head_dim);
  if (!q_out || !q || !k_cache || !v_cache || !k_new || !v_new || !cos || !sin || !slot_mapping)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != PAGEDKV_OK) return rc;
  const int64_t strides[] = {q_out_stride_tok, q_out_stride_head, q_stride_tok, q_stride_head,
                             k_new_stride_tok, k_new_stride_head, v_new_stride_tok, v_new_stride_head,
                             cos_sin_stride_tok};
  bool vec = aligned16(q_out) && aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(k_new) &&
             aligned16(v_new) && aligned16(cos) && aligned16(sin);
  for (int64_t st : strides) vec = vec && (st % 8) == 0;
  RopeParams rp{};
  rp.q_out = q_out;
  rp.qo_st = q_out_stride_tok;
  rp.qo_sh = q_out_stride_head;
  rp.q = q;
  rp.q_st = q_stride_tok;
  rp.q_sh = q_stride_head;
  rp.k_cache = k_cache;
  rp.v_cache = v_cache;
  rp.k = k_new;
  rp.k_st = k_new_stride_tok;
  rp.k_sh = k_new_stride_head;
  rp.v = v_new;
  rp.v_st = v_new_stride_tok;
  rp.v_sh = v_new_stride_head;
  rp.cos = cos;
  rp.sin = sin;
  rp.cs_st = cos_sin_stride_tok;
  rp.slots = slot_mapping;
  rp.num_slots = num_blocks * block_size;
  rp.num_tokens = num_tokens;
  rp.hq = num_q_heads;
  rp.hkv = num_kv_heads;
  rp.head_dim = head_dim;
  cudaError_t e = launch_kv_append_rope(rp, dtype, vec, di.err, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_append_rope launch");
  return PAGEDKV_OK;
}

int pagedkv_kv_write_prefill(void *const *k_caches, void *const *v_caches, const void *const *k_srcs,
                             const void *const *v_srcs, int32_t num_layers, int64_t k_stride_tok,
                             int64_t k_stride_head, int64_t v_stride_tok, int64_t v_stride_head,
                             int32_t src_dtype, const int64_t *block_ids, int32_t num_write_blocks,
                             int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                             int64_t num_blocks, int32_t block_size, int32_t dtype, void *stream) {
  NvtxRange nvtx("pagedkv_kv_write_prefill");
  if (num_layers < 0 || num_write_blocks < 0 || num_tokens < 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_layers, num_write_blocks, num_tokens must be >= 0");
  if (num_layers == 0 || num_write_blocks == 0) return PAGEDKV_OK;
  if (dtype != PAGEDKV_DTYPE_F16 && dtype != PAGEDKV_DTYPE_BF16)
    return fail(PAGEDKV_ERR_UNSUPPORTED, "pool dtype %d not supported (0=f16, 1=bf16)", dtype);
  if (src_dtype != dtype && src_dtype != PAGEDKV_DTYPE_F32)
    return fail(PAGEDKV_ERR_UNSUPPORTED, "source dtype %d must equal the pool dtype %d or be f32 (2)",
                src_dtype, dtype);
  if (num_kv_heads <= 0 || head_dim <= 0 || (head_dim % 8) != 0 || block_size <= 0 || num_blocks <= 0)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT,
                "num_kv_heads, block_size, num_blocks must be > 0 and head_dim a positive multiple of 8");
  if ((int64_t)num_tokens > (int64_t)num_write_blocks * block_size)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "num_tokens (%d) exceeds num_write_blocks * block_size", num_tokens);
  if (!k_caches || !v_caches || !k_srcs || !v_srcs || !block_ids)
    return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "null pointer");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != PAGEDKV_OK) return rc;
  // Vector loads need every 8-element source chunk aligned: strides in whole chunks.
  bool vec = (k_stride_tok % 8) == 0 && (k_stride_head % 8) == 0 && (v_stride_tok % 8) == 0 &&
             (v_stride_head % 8) == 0;
  const size_t src_align = src_dtype == PAGEDKV_DTYPE_F32 ? 32 : 16;
  for (int32_t l = 0; l < num_layers; ++l) {
    if (!k_caches[l] || !v_caches[l] || !k_srcs[l] || !v_srcs[l])
      return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "null pointer for layer %d", l);
    if (!aligned16(k_caches[l]) || !aligned16(v_caches[l]))
      return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "pool of layer %d is not 16-byte aligned", l);
    if (reinterpret_cast<uintptr_t>(k_srcs[l]) % src_align || reinterpret_cast<uintptr_t>(v_srcs[l]) % src_align)
      vec = false;
  }
  PrefillParams pp{};
  pp.k_stride_tok = k_stride_tok;
  pp.k_stride_head = k_stride_head;
  pp.v_stride_tok = v_stride_tok;
  pp.v_stride_head = v_stride_head;
  pp.block_ids = block_ids;
  pp.num_blocks = num_blocks;
  pp.num_write_blocks = num_write_blocks;
  pp.num_tokens = num_tokens;
  pp.num_kv_heads = num_kv_heads;
  pp.head_dim = head_dim;
  pp.block_size = block_size;
  for (int32_t l0 = 0; l0 < num_layers; l0 += kPrefillMaxLayers) {
    const int32_t n = num_layers - l0 < kPrefillMaxLayers ? num_layers - l0 : kPrefillMaxLayers;
    pp.num_layers = n;
    for (int32_t i = 0; i < n; ++i) {
      pp.k_dst[i] = k_caches[l0 + i];
      pp.v_dst[i] = v_caches[l0 + i];
      pp.k_src[i] = k_srcs[l0 + i];
      pp.v_src[i] = v_srcs[l0 + i];
    }
    cudaError_t e = launch_kv_write_prefill(pp, dtype, src_dtype, vec, di.err, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kv_write_prefill launch");
  }
  return PAGEDKV_OK;
}

int pagedkv_read_error_flags(uint32_t *flags_out, int32_t clear, void *stream) {
  if (!flags_out) return fail(PAGEDKV_ERR_INVALID_ARGUMENT, "flags_out is null");
  DeviceInfo di;
  int rc = device_info(&di);
  if (rc != PAGEDKV_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, di.err, sizeof(h), cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return cuda_fail(e, "read error word");
  if (clear) {
    e = cudaMemsetAsync(di.err, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return cuda_fail(e, "clear error word");
  }
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  *flags_out = h;
  return PAGEDKV_OK;
}

}  // extern "C"
