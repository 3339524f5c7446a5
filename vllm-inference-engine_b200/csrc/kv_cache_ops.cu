// KV append and copy-on-write block copy (sm_100a).
//
// Both are pure byte movement bound by HBM bandwidth: every thread moves one
// 16-byte chunk (or a strided run of them), with 64-bit offsets so pools larger
// than 2^31 bytes per layer are addressed correctly.
#include "common.cuh"
#include "launch.h"

namespace pagedkv {

// One thread per 16-byte chunk of one token's [num_kv_heads, head_dim] row,
// for K and V together. chunks_per_row = num_kv_heads * head_dim / 8.
// Restates engine/kernels/paged_attention_integration.py:150-160: the reference
// computes (phys, off) = (table[(len-1)/BS], (len-1)%BS) per sequence on the host
// and assigns pool[l][phys, off] = k; here the slot phys*BS+off comes in
// precomputed and every token of the batch is written by one launch.
__global__ void __launch_bounds__(256)
kv_append_vec_kernel(char *__restrict__ k_cache, char *__restrict__ v_cache,
                     const char *__restrict__ k_new, int64_t ks_tok, int64_t ks_head,
                     const char *__restrict__ v_new, int64_t vs_tok, int64_t vs_head,
                     const int64_t *__restrict__ slots, int32_t num_tokens,
                     int32_t num_kv_heads, int32_t head_dim, int64_t num_slots, unsigned int *err) {
  // Programmatic dependent launch: let the next kernel (the attention that
  // reads these rows) start its prologue now; wait for the previous grid's
  // writes before touching memory.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int chunks_per_head = head_dim >> 3;
  const int chunks_per_row = num_kv_heads * chunks_per_head;
  const int64_t total = (int64_t)num_tokens * chunks_per_row;
  const int64_t row_bytes = (int64_t)num_kv_heads * head_dim * 2;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int tok = (int)(idx / chunks_per_row);
    const int rem = (int)(idx - (int64_t)tok * chunks_per_row);
    const int head = rem / chunks_per_head;
    const int c = rem - head * chunks_per_head;
    const int64_t slot = __ldg(slots + tok);
    if (slot < 0) continue;
    if (slot >= num_slots) {
      set_error(err, PAGEDKV_EFLAG_SLOT_RANGE);
      continue;
    }
    const int64_t dst = slot * row_bytes + ((int64_t)head * head_dim + c * 8) * 2;
    const uint4 kv = ldg16(k_new + ((int64_t)tok * ks_tok + (int64_t)head * ks_head + c * 8) * 2);
    const uint4 vv = ldg16(v_new + ((int64_t)tok * vs_tok + (int64_t)head * vs_head + c * 8) * 2);
    stg16(k_cache + dst, kv);
    stg16(v_cache + dst, vv);
  }
}

// Fallback for inputs whose rows are not 16-byte aligned: one 2-byte element
// per thread.
__global__ void __launch_bounds__(256)
kv_append_scalar_kernel(uint16_t *__restrict__ k_cache, uint16_t *__restrict__ v_cache,
                        const uint16_t *__restrict__ k_new, int64_t ks_tok, int64_t ks_head,
                        const uint16_t *__restrict__ v_new, int64_t vs_tok, int64_t vs_head,
                        const int64_t *__restrict__ slots, int32_t num_tokens,
                        int32_t num_kv_heads, int32_t head_dim, int64_t num_slots,
                        unsigned int *err) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int per_row = num_kv_heads * head_dim;
  const int64_t total = (int64_t)num_tokens * per_row;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int tok = (int)(idx / per_row);
    const int rem = (int)(idx - (int64_t)tok * per_row);
    const int head = rem / head_dim;
    const int d = rem - head * head_dim;
    const int64_t slot = slots[tok];
    if (slot < 0) continue;
    if (slot >= num_slots) {
      set_error(err, PAGEDKV_EFLAG_SLOT_RANGE);
      continue;
    }
    const int64_t dst = slot * per_row + rem;
    k_cache[dst] = k_new[(int64_t)tok * ks_tok + (int64_t)head * ks_head + d];
    v_cache[dst] = v_new[(int64_t)tok * vs_tok + (int64_t)head * vs_head + d];
  }
}

// Copy-on-write: for every (src, dst) pair and layer, K block src -> dst and
// V block src -> dst of that layer's pool. One warp per (pair, layer, K|V)
// unit at a time; every lane keeps kCopyUnroll 16-byte loads in flight before
// the matching stores (one round covers a 4 KiB block), and the grid is a few
// CTAs per SM striding over the units, so neither launch cost nor CTA
// scheduling grows with the pair count, and a decode step's few hundred pairs
// still spread over every SM.
constexpr int kCopyUnroll = 8;
constexpr int kCopyThreads = 256;

__global__ void __launch_bounds__(kCopyThreads)
copy_blocks_kernel(char *const *__restrict__ k_ptrs, char *const *__restrict__ v_ptrs,
                   int32_t num_layers, const int64_t *__restrict__ mapping, int32_t num_pairs,
                   int64_t block_bytes, int64_t num_blocks, unsigned int *err) {
  // Programmatic dependent launch: the next kernel may start its prologue; the
  // previous grid's writes are visible after the wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kCopyThreads / 32);
  const int64_t per_pair = 2 * (int64_t)num_layers;  // (layer, K|V) units of a pair
  const int64_t units = (int64_t)num_pairs * per_pair;
  const int64_t n16 = block_bytes >> 4;  // 16-byte chunks per block
  for (int64_t unit = (int64_t)blockIdx.x * (kCopyThreads / 32) + (threadIdx.x >> 5); unit < units;
       unit += warps) {
    const int pair = (int)(unit / per_pair);
    const int rem = (int)(unit - (int64_t)pair * per_pair);
    const int layer = rem >> 1;
    const bool is_v = rem & 1;
    const int64_t src = __ldg(mapping + 2 * pair);
    const int64_t dst = __ldg(mapping + 2 * pair + 1);
    if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
      if (lane == 0 && rem == 0) set_error(err, PAGEDKV_EFLAG_COPY_RANGE);
      continue;
    }
    char *base = is_v ? v_ptrs[layer] : k_ptrs[layer];
    const char *s = base + src * block_bytes;
    char *d = base + dst * block_bytes;
    for (int64_t c0 = lane; c0 < n16; c0 += 32 * kCopyUnroll) {
      uint4 r[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t c = c0 + u * 32;
        if (c < n16) r[u] = ldg_stream16(s + c * 16);
      }
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t c = c0 + u * 32;
        if (c < n16) stg16(d + c * 16, r[u]);
      }
    }
  }
}

cudaError_t launch_kv_append(void *k_cache, void *v_cache, const void *k_new, int64_t ks_tok,
                             int64_t ks_head, const void *v_new, int64_t vs_tok,
                             int64_t vs_head, const int64_t *slots, int32_t num_tokens,
                             int32_t num_kv_heads, int32_t head_dim, int64_t num_slots,
                             bool vectorized, unsigned int *err, cudaStream_t stream) {
  if (num_tokens == 0) return cudaSuccess;
  const int threads = 256;
  // Launched as a programmatic dependent (see the griddepcontrol pair above).
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (vectorized) {
    const int64_t total = (int64_t)num_tokens * num_kv_heads * (head_dim / 8);
    const int64_t blocks = (total + threads - 1) / threads;
    cfg.gridDim = dim3((unsigned)(blocks < 65535 * 8 ? blocks : 65535 * 8));
    return cudaLaunchKernelEx(&cfg, kv_append_vec_kernel, (char *)k_cache, (char *)v_cache,
                              (const char *)k_new, ks_tok, ks_head, (const char *)v_new, vs_tok,
                              vs_head, slots, num_tokens, num_kv_heads, head_dim, num_slots, err);
  }
  const int64_t total = (int64_t)num_tokens * num_kv_heads * head_dim;
  const int64_t blocks = (total + threads - 1) / threads;
  cfg.gridDim = dim3((unsigned)(blocks < 65535 * 8 ? blocks : 65535 * 8));
  return cudaLaunchKernelEx(&cfg, kv_append_scalar_kernel, (uint16_t *)k_cache, (uint16_t *)v_cache,
                            (const uint16_t *)k_new, ks_tok, ks_head, (const uint16_t *)v_new,
                            vs_tok, vs_head, slots, num_tokens, num_kv_heads, head_dim, num_slots,
                            err);
}

cudaError_t launch_copy_blocks(void *const *k_ptrs, void *const *v_ptrs, int32_t num_layers,
                               const int64_t *mapping, int32_t num_pairs, int64_t block_bytes,
                               int64_t num_blocks, int num_sms, unsigned int *err, cudaStream_t stream) {
  if (num_pairs == 0 || num_layers == 0) return cudaSuccess;
  const int64_t units = (int64_t)num_pairs * num_layers * 2;
  const int64_t need = (units + kCopyThreads / 32 - 1) / (kCopyThreads / 32);
  const int64_t cap = (int64_t)(num_sms > 0 ? num_sms : 148) * 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(need < cap ? need : cap));
  cfg.blockDim = dim3(kCopyThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, copy_blocks_kernel, (char *const *)k_ptrs, (char *const *)v_ptrs,
                            num_layers, mapping, num_pairs, block_bytes, num_blocks, err);
}

}  // namespace pagedkv
