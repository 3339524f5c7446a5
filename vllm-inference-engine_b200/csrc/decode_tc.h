// Interface of the tcgen05 + TMA decode-attention kernel (decode_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "launch.h"

namespace pagedkv {

// True when the tensor-core kernel covers this shape (GQA group 1..16,
// head_dim 64 or 128, power-of-two block_size 8..128).
bool tc_eligible(int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size);

// Scratch the tensor-core path needs (split-K partials), in bytes.
size_t tc_workspace_bytes(int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                          int32_t head_dim, int32_t max_tokens, int32_t num_sms);

// The decode append fused into a tensor-core launch: each sequence's new K /
// V rows (strides in elements) are written at position len - 1 of its block
// table before the tile holding it is read; with cos / sin (rows per
// sequence, stride cs_st) K and q are rotated first (RoPE).
struct AppendParams {
  const void *k_new;
  int64_t k_st, k_sh;
  const void *v_new;
  int64_t v_st, v_sh;
  const void *cos, *sin;  // nullptr: no rotation
  int64_t cs_st;
};

// Launch; returns a PAGEDKV_* status and writes the number of launches.
// `append` (optional) fuses the decode append into the launch.
int tc_launch(DecodeParams &p, int dtype, void *workspace, size_t workspace_bytes,
              int32_t num_sms, cudaStream_t stream, int *launches, std::string *error,
              const AppendParams *append = nullptr);

}  // namespace pagedkv
