// Host-side launch declarations shared by the pagedkv translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace pagedkv {

// Every decode workspace starts with this many bytes of cross-CTA completion
// flags. They must be zero before the first launch that uses the workspace;
// each launch leaves them zero again. Split-K partials start after it.
constexpr size_t kWorkspaceHeaderBytes = 8192;

// Everything one decode-attention launch needs, resolved by the ABI layer.
struct DecodeParams {
  void *out;
  int64_t o_ss, o_sh;           // out strides (elements): seq, head
  const void *q;
  int64_t q_ss, q_sh;           // q strides (elements): seq, head
  const void *k;
  const void *v;
  const int32_t *bt;            // block tables
  int64_t bt_s;                 // block table row stride (elements)
  const int32_t *lens;          // seq_lens or nullptr
  int32_t uniform_len;          // used when lens == nullptr
  int32_t num_seqs, hq, hkv, group, head_dim, block_size, max_blocks;
  int64_t num_blocks;
  float scale_log2;             // scale * log2(e)
  int32_t split_tokens;         // tokens per split-K chunk
  int32_t num_splits;           // chunks per sequence (1 = no combine pass)
  float *ws_acc;                // [num_seqs, hq, num_splits, head_dim] partial sums
  float2 *ws_ml;                // [num_seqs, hq, num_splits] (running max, denominator)
  unsigned int *err;            // device error word
};

// Split-K decision shared by the workspace-size query and the launcher.
struct SplitPlan {
  int32_t split_tokens;
  int32_t num_splits;
};

SplitPlan plan_simt_splits(int32_t num_seqs, int32_t num_kv_heads, int32_t group,
                           int32_t max_tokens, int32_t num_sms);

// Set the calling thread's pagedkv_last_error() message.
void set_last_error_message(const char *msg);

cudaError_t launch_decode_simt(const DecodeParams &p, int dtype, cudaStream_t stream);
cudaError_t launch_decode_combine(const DecodeParams &p, int dtype, cudaStream_t stream);

cudaError_t launch_kv_append(void *k_cache, void *v_cache, const void *k_new, int64_t ks_tok,
                             int64_t ks_head, const void *v_new, int64_t vs_tok,
                             int64_t vs_head, const int64_t *slots, int32_t num_tokens,
                             int32_t num_kv_heads, int32_t head_dim, int64_t num_slots,
                             bool vectorized, unsigned int *err, cudaStream_t stream);

// Prefill write of up to kPrefillMaxLayers layers in one launch (pointer
// arrays passed by value).
constexpr int kPrefillMaxLayers = 48;
struct PrefillParams {
  void *k_dst[kPrefillMaxLayers];
  void *v_dst[kPrefillMaxLayers];
  const void *k_src[kPrefillMaxLayers];
  const void *v_src[kPrefillMaxLayers];
  int64_t k_stride_tok, k_stride_head, v_stride_tok, v_stride_head;  // source strides (elements)
  const int64_t *block_ids;                                           // [num_write_blocks]
  int64_t num_blocks;
  int32_t num_layers, num_write_blocks, num_tokens, num_kv_heads, head_dim, block_size;
};

cudaError_t launch_kv_write_prefill(const PrefillParams &pp, int dtype, int src_dtype, bool vec,
                                    unsigned int *err, cudaStream_t stream);

// Fused rotary embedding + KV append (strides in elements).
struct RopeParams {
  void *q_out;
  int64_t qo_st, qo_sh;
  const void *q;
  int64_t q_st, q_sh;
  void *k_cache, *v_cache;
  const void *k;
  int64_t k_st, k_sh;
  const void *v;
  int64_t v_st, v_sh;
  const void *cos, *sin;  // [num_tokens, head_dim] rows
  int64_t cs_st;
  const int64_t *slots;
  int64_t num_slots;
  int32_t num_tokens, hq, hkv, head_dim;
};

cudaError_t launch_kv_append_rope(const RopeParams &rp, int dtype, bool vec, unsigned int *err,
                                  cudaStream_t stream);

cudaError_t launch_copy_blocks(void *const *k_ptrs, void *const *v_ptrs, int32_t num_layers,
                               const int64_t *mapping, int32_t num_pairs, int64_t block_bytes,
                               int64_t num_blocks, int num_sms, unsigned int *err, cudaStream_t stream);

}  // namespace pagedkv
