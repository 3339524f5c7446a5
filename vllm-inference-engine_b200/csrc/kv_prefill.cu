// Prefill K/V write: a prompt's K/V rows of every layer into whole pool blocks,
// the padded tail of the last block zeroed (sm_100a).
//
// Restates engine/kernels/paged_attention_integration.py:278-326
// (_copy_prefill_kv): for blocks [skip_blocks, ceil(prompt_len / BS)) of the
// sequence's table it pads the prompt's rows [skip_blocks * BS, prompt_len) with
// zeros to whole blocks, converts them to the pool dtype (.to(dtype), round to
// nearest even) and index_copy_'s them into every layer's K and V pool, two
// copies plus a pad per layer. Here one launch writes all layers, K and V:
// every thread produces one 16-byte chunk (8 elements) of one destination row.
#include "common.cuh"
#include "launch.h"

namespace pagedkv {

namespace {

template <typename T>
__device__ __forceinline__ uint4 convert8(const float4 a, const float4 b) {
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  return Elem<T>::pack8(v);
}

// S: source element (the pool's own type, or float); T: pool element.
// VEC: every source row chunk is 16-byte (S = 2 B) / 32-byte (S = float)
// aligned, so it is read with vector loads; otherwise element by element.
template <typename T, typename S, bool VEC>
__global__ void __launch_bounds__(256)
kv_write_prefill_kernel(const PrefillParams pp, unsigned int *err) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int layer = blockIdx.y;
  const int cph = pp.head_dim >> 3;                 // chunks per head row
  const int cpt = pp.num_kv_heads * cph;            // chunks per token row
  const int64_t total = (int64_t)pp.num_write_blocks * pp.block_size * cpt;
  const int64_t row_elems = (int64_t)pp.num_kv_heads * pp.head_dim;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = idx / cpt;                  // token position relative to the first written block
    const int rem = (int)(idx - pos * cpt);
    const int head = rem / cph;
    const int c = rem - head * cph;
    const int64_t blk_i = pos / pp.block_size;
    const int t = (int)(pos - blk_i * pp.block_size);
    const int64_t blk = __ldg(pp.block_ids + blk_i);
    if (blk < 0 || blk >= pp.num_blocks) {
      if (rem == 0 && t == 0 && layer == 0) set_error(err, PAGEDKV_EFLAG_BLOCK_ID_RANGE);
      continue;
    }
    const int64_t dst = ((blk * pp.block_size + t) * row_elems + (int64_t)head * pp.head_dim + c * 8) *
                        (int64_t)sizeof(T);
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = make_uint4(0u, 0u, 0u, 0u);
    if (pos < pp.num_tokens) {
      const int64_t ko = pos * pp.k_stride_tok + (int64_t)head * pp.k_stride_head + c * 8;
      const int64_t vo = pos * pp.v_stride_tok + (int64_t)head * pp.v_stride_head + c * 8;
      const S *ks = static_cast<const S *>(pp.k_src[layer]) + ko;
      const S *vs = static_cast<const S *>(pp.v_src[layer]) + vo;
      if constexpr (sizeof(S) == 2) {
        if constexpr (VEC) {
          kv = ldg16(ks);
          vv = ldg16(vs);
        } else {
          uint16_t a[8], b[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            a[i] = __ldg(reinterpret_cast<const unsigned short *>(ks) + i);
            b[i] = __ldg(reinterpret_cast<const unsigned short *>(vs) + i);
          }
          kv = make_uint4(a[0] | (uint32_t)a[1] << 16, a[2] | (uint32_t)a[3] << 16,
                          a[4] | (uint32_t)a[5] << 16, a[6] | (uint32_t)a[7] << 16);
          vv = make_uint4(b[0] | (uint32_t)b[1] << 16, b[2] | (uint32_t)b[3] << 16,
                          b[4] | (uint32_t)b[5] << 16, b[6] | (uint32_t)b[7] << 16);
        }
      } else {
        float4 k0, k1, v0, v1;
        if constexpr (VEC) {
          k0 = __ldg(reinterpret_cast<const float4 *>(ks));
          k1 = __ldg(reinterpret_cast<const float4 *>(ks) + 1);
          v0 = __ldg(reinterpret_cast<const float4 *>(vs));
          v1 = __ldg(reinterpret_cast<const float4 *>(vs) + 1);
        } else {
          k0 = make_float4(__ldg(ks), __ldg(ks + 1), __ldg(ks + 2), __ldg(ks + 3));
          k1 = make_float4(__ldg(ks + 4), __ldg(ks + 5), __ldg(ks + 6), __ldg(ks + 7));
          v0 = make_float4(__ldg(vs), __ldg(vs + 1), __ldg(vs + 2), __ldg(vs + 3));
          v1 = make_float4(__ldg(vs + 4), __ldg(vs + 5), __ldg(vs + 6), __ldg(vs + 7));
        }
        kv = convert8<T>(k0, k1);
        vv = convert8<T>(v0, v1);
      }
    }
    stg16(static_cast<char *>(pp.k_dst[layer]) + dst, kv);
    stg16(static_cast<char *>(pp.v_dst[layer]) + dst, vv);
  }
}

template <typename T, typename S>
cudaError_t launch_typed(const PrefillParams &pp, bool vec, unsigned int *err, cudaStream_t stream) {
  const int threads = 256;
  const int64_t total = (int64_t)pp.num_write_blocks * pp.block_size * pp.num_kv_heads * (pp.head_dim / 8);
  const int64_t blocks = (total + threads - 1) / threads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(blocks < 4096 ? blocks : 4096), (unsigned)pp.num_layers);
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (vec) return cudaLaunchKernelEx(&cfg, kv_write_prefill_kernel<T, S, true>, pp, err);
  return cudaLaunchKernelEx(&cfg, kv_write_prefill_kernel<T, S, false>, pp, err);
}

}  // namespace

cudaError_t launch_kv_write_prefill(const PrefillParams &pp, int dtype, int src_dtype, bool vec,
                                    unsigned int *err, cudaStream_t stream) {
  if (pp.num_write_blocks == 0 || pp.num_layers == 0) return cudaSuccess;
  if (dtype == PAGEDKV_DTYPE_BF16) {
    return src_dtype == PAGEDKV_DTYPE_F32 ? launch_typed<__nv_bfloat16, float>(pp, vec, err, stream)
                                          : launch_typed<__nv_bfloat16, __nv_bfloat16>(pp, vec, err, stream);
  }
  return src_dtype == PAGEDKV_DTYPE_F32 ? launch_typed<__half, float>(pp, vec, err, stream)
                                        : launch_typed<__half, __half>(pp, vec, err, stream);
}

}  // namespace pagedkv
