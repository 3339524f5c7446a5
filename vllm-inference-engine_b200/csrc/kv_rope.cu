// Fused rotary embedding + KV append (sm_100a).
//
// The reference's decode forward (engine/kernels/paged_attention_integration.py
// :104-109, then :150-160) runs transformers' apply_rotary_pos_emb on q and k,
//   x_embed = (x * cos) + (rotate_half(x) * sin),
//   rotate_half(x) = cat(-x[..., D/2:], x[..., :D/2]),
// as separate fp16/bf16 tensor ops (each product and the sum rounded to the
// tensor dtype), and then writes k and v into the pool through per-sequence
// index_put. Here one launch rotates q into q_out, rotates k straight into its
// pool slot and copies v into its slot, with the same rounding sequence
// (fp32 products of the 16-bit inputs are exact; each is rounded to the dtype,
// summed in fp32 and rounded again), so the result is bit-identical.
// One thread per (row, 8-element chunk c of the first half): it owns elements
// [8c, 8c + 8) and their rotation partners [D/2 + 8c, D/2 + 8c + 8).
#include "common.cuh"
#include "launch.h"

namespace pagedkv {

namespace {

template <typename T>
__device__ __forceinline__ void load8(const T *p, bool vec, float (&f)[8]) {
  if (vec) {
    Elem<T>::unpack8(ldg16(p), f);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_float(p[i]);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T *p, bool vec, const float (&f)[8]) {
  if (vec) {
    stg16(p, Elem<T>::pack8(f));
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = Elem<T>::from_float(f[i]);
  }
}

// I is the flat work index type: 32-bit whenever the launch has fewer than
// 2^32 items (the divisions below are then the cheap 32-bit ones), else 64-bit.
template <typename T, bool VEC, typename I>
__global__ void __launch_bounds__(256)
kv_append_rope_kernel(const RopeParams rp, unsigned int *err) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int half = rp.head_dim >> 1;
  const int cph = half >> 3;                          // chunk pairs per row
  const int rows_per_tok = rp.hq + 2 * rp.hkv;        // q rows, k rows, v rows
  const I per_tok = (I)rows_per_tok * cph;
  const I total = (I)rp.num_tokens * per_tok;
  for (I idx = (I)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (I)gridDim.x * blockDim.x) {
    const int tok = (int)(idx / per_tok);
    const int rem = (int)(idx - (I)tok * per_tok);
    const int r = rem / cph;
    const int c = rem - r * cph;
    const int lo = c * 8, hi = half + c * 8;
    const T *src;
    T *dst;
    bool rotate = true;
    if (r < rp.hq) {
      src = static_cast<const T *>(rp.q) + (int64_t)tok * rp.q_st + (int64_t)r * rp.q_sh;
      dst = static_cast<T *>(rp.q_out) + (int64_t)tok * rp.qo_st + (int64_t)r * rp.qo_sh;
    } else {
      const int64_t slot = __ldg(rp.slots + tok);
      if (slot < 0) continue;  // padding token: nothing to write
      if (slot >= rp.num_slots) {
        if (c == 0) set_error(err, PAGEDKV_EFLAG_SLOT_RANGE);
        continue;
      }
      const bool is_k = r < rp.hq + rp.hkv;
      const int h = is_k ? r - rp.hq : r - rp.hq - rp.hkv;
      const int64_t row = slot * rp.hkv + h;
      if (is_k) {
        src = static_cast<const T *>(rp.k) + (int64_t)tok * rp.k_st + (int64_t)h * rp.k_sh;
        dst = static_cast<T *>(rp.k_cache) + row * rp.head_dim;
      } else {
        src = static_cast<const T *>(rp.v) + (int64_t)tok * rp.v_st + (int64_t)h * rp.v_sh;
        dst = static_cast<T *>(rp.v_cache) + row * rp.head_dim;
        rotate = false;
      }
    }
    float a[8], b[8];
    load8(src + lo, VEC, a);
    load8(src + hi, VEC, b);
    if (rotate) {
      const T *cs = static_cast<const T *>(rp.cos) + (int64_t)tok * rp.cs_st;
      const T *sn = static_cast<const T *>(rp.sin) + (int64_t)tok * rp.cs_st;
      float cl[8], ch[8], sl[8], sh[8], oa[8], ob[8];
      load8(cs + lo, VEC, cl);
      load8(cs + hi, VEC, ch);
      load8(sn + lo, VEC, sl);
      load8(sn + hi, VEC, sh);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        oa[i] = rope_elem<T>(a[i], cl[i], -b[i], sl[i]);
        ob[i] = rope_elem<T>(b[i], ch[i], a[i], sh[i]);
      }
      store8(dst + lo, VEC, oa);
      store8(dst + hi, VEC, ob);
    } else {
      store8(dst + lo, VEC, a);
      store8(dst + hi, VEC, b);
    }
  }
}

template <typename T>
cudaError_t launch_typed(const RopeParams &rp, bool vec, unsigned int *err, cudaStream_t stream) {
  const int threads = 256;
  const int64_t total = (int64_t)rp.num_tokens * (rp.hq + 2 * rp.hkv) * (rp.head_dim / 16);
  const int64_t blocks = (total + threads - 1) / threads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(blocks < 65535 * 8 ? blocks : 65535 * 8));
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // total + gridDim * blockDim must not wrap the 32-bit index
  const bool narrow = total + (int64_t)cfg.gridDim.x * threads < (int64_t(1) << 32);
  if (narrow) {
    if (vec) return cudaLaunchKernelEx(&cfg, kv_append_rope_kernel<T, true, uint32_t>, rp, err);
    return cudaLaunchKernelEx(&cfg, kv_append_rope_kernel<T, false, uint32_t>, rp, err);
  }
  if (vec) return cudaLaunchKernelEx(&cfg, kv_append_rope_kernel<T, true, int64_t>, rp, err);
  return cudaLaunchKernelEx(&cfg, kv_append_rope_kernel<T, false, int64_t>, rp, err);
}

}  // namespace

cudaError_t launch_kv_append_rope(const RopeParams &rp, int dtype, bool vec, unsigned int *err,
                                  cudaStream_t stream) {
  if (rp.num_tokens == 0) return cudaSuccess;
  return dtype == PAGEDKV_DTYPE_BF16 ? launch_typed<__nv_bfloat16>(rp, vec, err, stream)
                                     : launch_typed<__half>(rp, vec, err, stream);
}

}  // namespace pagedkv
