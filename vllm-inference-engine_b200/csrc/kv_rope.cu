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
// One thread per (token, group of head rows, 8-element chunk c of the first
// half): it owns elements [8c, 8c + 8) and their rotation partners
// [D/2 + 8c, D/2 + 8c + 8) of every row of its group, loading the token's cos /
// sin chunks and pool slot once for the whole group. The rotation runs on
// packed 16-bit pairs (rope8: one correctly rounded f16x2 / bf16x2 multiply
// per product and add per sum, equal to the fp32 form above bit for bit).
#include "common.cuh"
#include "launch.h"

namespace pagedkv {

namespace {

// Eight 16-bit elements as raw bits: one 16-byte access when VEC, else eight
// 2-byte ones (sources or destinations not 16-byte aligned).
template <bool VEC>
__device__ __forceinline__ uint4 ld8(const uint16_t *p) {
  if constexpr (VEC) {
    return ldg16(p);
  } else {
    uint4 r;
    uint16_t *h = reinterpret_cast<uint16_t *>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = __ldg(p + i);
    return r;
  }
}

template <bool VEC>
__device__ __forceinline__ void st8(uint16_t *p, const uint4 &v) {
  if constexpr (VEC) {
    stg16(p, v);
  } else {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = h[i];
  }
}

// Rows whose loads are in flight together (two keep the 16-byte path within
// 64 registers, four CTAs per SM, without spills).
constexpr int kRowBatch = 2;

// I is the flat work index type: 32-bit whenever the launch has fewer than
// 2^32 items (the divisions below are then the cheap 32-bit ones), else 64-bit.
// Rows of a token: q heads [0, hq), k heads [hq, hq + hkv), v heads after;
// group g holds rows [g * rpt, min(rows, (g + 1) * rpt)).
template <typename T, bool VEC, typename I>
__global__ void __launch_bounds__(256)
kv_append_rope_kernel(const RopeParams rp, int rpt, unsigned int *err) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int half = rp.head_dim >> 1;
  const int cph = half >> 3;                    // chunk pairs per row
  const int rows = rp.hq + 2 * rp.hkv;          // q rows, k rows, v rows
  const int kv0 = rp.hq, v0 = rp.hq + rp.hkv;   // first k row, first v row
  const int groups = (rows + rpt - 1) / rpt;
  const I per_tok = (I)groups * cph;
  const I total = (I)rp.num_tokens * per_tok;
  for (I idx = (I)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (I)gridDim.x * blockDim.x) {
    const int tok = (int)(idx / per_tok);
    const int rem = (int)(idx - (I)tok * per_tok);
    const int g = rem / cph;
    const int c = rem - g * cph;
    const int lo = c * 8, hi = half + c * 8;
    const int r0 = g * rpt, r1 = min(rows, r0 + rpt);
    // the token's pool slot, when the group holds k / v rows (< 0: none written)
    int64_t slot = -1;
    if (r1 > kv0) {
      slot = __ldg(rp.slots + tok);
      if (slot >= rp.num_slots) {
        if (c == 0) set_error(err, PAGEDKV_EFLAG_SLOT_RANGE);
        slot = -1;
      }
    }
    uint4 cl = {}, ch = {}, sl = {}, sh = {};
    if (r0 < v0) {  // the group rotates
      const uint16_t *cs = static_cast<const uint16_t *>(rp.cos) + (int64_t)tok * rp.cs_st;
      const uint16_t *sn = static_cast<const uint16_t *>(rp.sin) + (int64_t)tok * rp.cs_st;
      cl = ld8<VEC>(cs + lo);
      ch = ld8<VEC>(cs + hi);
      sl = ld8<VEC>(sn + lo);
      sh = ld8<VEC>(sn + hi);
    }
    for (int rb = r0; rb < r1; rb += kRowBatch) {
      uint4 a[kRowBatch], b[kRowBatch];
      uint16_t *dst[kRowBatch];
#pragma unroll
      for (int u = 0; u < kRowBatch; ++u) {
        const int r = rb + u;
        const uint16_t *src = nullptr;
        dst[u] = nullptr;
        if (r < r1) {
          if (r < kv0) {
            src = static_cast<const uint16_t *>(rp.q) + (int64_t)tok * rp.q_st + (int64_t)r * rp.q_sh;
            dst[u] = static_cast<uint16_t *>(rp.q_out) + (int64_t)tok * rp.qo_st + (int64_t)r * rp.qo_sh;
          } else if (slot >= 0) {
            const bool is_k = r < v0;
            const int h = is_k ? r - kv0 : r - v0;
            const int64_t row = slot * rp.hkv + h;
            src = is_k ? static_cast<const uint16_t *>(rp.k) + (int64_t)tok * rp.k_st + (int64_t)h * rp.k_sh
                       : static_cast<const uint16_t *>(rp.v) + (int64_t)tok * rp.v_st + (int64_t)h * rp.v_sh;
            dst[u] = static_cast<uint16_t *>(is_k ? rp.k_cache : rp.v_cache) + row * rp.head_dim;
          }
        }
        if (src != nullptr) {
          a[u] = ld8<VEC>(src + lo);
          b[u] = ld8<VEC>(src + hi);
        }
      }
#pragma unroll
      for (int u = 0; u < kRowBatch; ++u) {
        if (dst[u] == nullptr) continue;
        if (rb + u < v0) {
          st8<VEC>(dst[u] + lo, rope8<T>(a[u], b[u], cl, sl, true));
          st8<VEC>(dst[u] + hi, rope8<T>(b[u], a[u], ch, sh, false));
        } else {
          st8<VEC>(dst[u] + lo, a[u]);
          st8<VEC>(dst[u] + hi, b[u]);
        }
      }
    }
  }
}

template <typename T>
cudaError_t launch_typed(const RopeParams &rp, bool vec, unsigned int *err, cudaStream_t stream) {
  const int threads = 256;
  const int rows = rp.hq + 2 * rp.hkv;
  const int cph = rp.head_dim / 16;
  // Rows per thread: one while a row per thread fills the GPU about twice
  // over (decode sizes: the most threads, the shortest chain per thread),
  // more as the launch grows, up to the whole token (bulk sizes: cos / sin,
  // slot and index work once per token and chunk).
  constexpr int64_t kFill = 2 * 148 * 2048;
  const int64_t one_row = (int64_t)rp.num_tokens * rows * cph;
  int64_t rpt = one_row / kFill;
  rpt = rpt < 1 ? 1 : (rpt > rows ? rows : rpt);
  const int64_t total = (int64_t)rp.num_tokens * ((rows + rpt - 1) / rpt) * cph;
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
  const int r = (int)rpt;
  if (narrow) {
    if (vec) return cudaLaunchKernelEx(&cfg, kv_append_rope_kernel<T, true, uint32_t>, rp, r, err);
    return cudaLaunchKernelEx(&cfg, kv_append_rope_kernel<T, false, uint32_t>, rp, r, err);
  }
  if (vec) return cudaLaunchKernelEx(&cfg, kv_append_rope_kernel<T, true, int64_t>, rp, r, err);
  return cudaLaunchKernelEx(&cfg, kv_append_rope_kernel<T, false, int64_t>, rp, r, err);
}

}  // namespace

cudaError_t launch_kv_append_rope(const RopeParams &rp, int dtype, bool vec, unsigned int *err,
                                  cudaStream_t stream) {
  if (rp.num_tokens == 0) return cudaSuccess;
  return dtype == PAGEDKV_DTYPE_BF16 ? launch_typed<__nv_bfloat16>(rp, vec, err, stream)
                                     : launch_typed<__half>(rp, vec, err, stream);
}

}  // namespace pagedkv
