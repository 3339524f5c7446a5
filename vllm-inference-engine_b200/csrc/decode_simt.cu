// Paged GQA decode attention on CUDA cores (sm_100a), split-K over the context.
//
// Serves the shapes the tcgen05 kernel is not built for: block sizes below 8,
// above 128 or not a power of two (head_dim 32, 64, 128 or 256, any group).
//
// Algorithm (restates engine/kernels/paged_attention.py:508-631, the batched
// online-softmax kernel, with its grid changed from one program per QUERY head
// to one CTA per (sequence, split, kv_head, head chunk) so a K/V row is read
// once for every query head of its GQA group):
//   * a "lane group" of head_dim/8 lanes owns one token at a time; each lane
//     holds 8 contiguous elements (one 16-byte load of K and of V),
//   * q.k partial sums are reduced inside the lane group with xor shuffles,
//   * every lane group keeps a private online softmax (m, l, acc) in base-2
//     (scores are pre-multiplied by scale*log2(e)), updated once per U tokens,
//   * each thread's K / V chunks reach it through a ring of S steps in shared
//     memory, copied by cp.async S - 1 steps ahead: the loads of later steps
//     stay in flight while this one is computed (the registers of wide groups
//     leave two CTAs per SM, too few loads in flight to cover HBM latency
//     otherwise); each thread reads back only its own copies,
//   * lane groups, then warps, are merged with the usual (m, l) rescaling,
//   * with more than one split the unnormalised partial (m, l, acc) goes to the
//     workspace and decode_combine_kernel forms the final output.
#include "common.cuh"
#include "launch.h"

namespace pagedkv {

namespace {

// 16-byte cp.async that bypasses L1; src_bytes 0 writes zeros and reads nothing.
__device__ __forceinline__ void stage16(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void stage_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int Pending>
__device__ __forceinline__ void stage_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(Pending) : "memory");
}

}  // namespace

// Steps of K / V rows staged ahead through shared memory: as many as keep the
// kernel's static shared memory (this ring plus the merge buffers,
// 16 * GMAX * (D + 2) bytes) within 48 KiB, between 2 and 4.
template <int D, int GMAX, int U>
constexpr int simt_stages() {
  constexpr int free_bytes = 48 * 1024 - 16 * GMAX * (D + 2) - 512;
  constexpr int s = free_bytes / (U * 2 * 128 * 16);
  return s < 2 ? 2 : s > 4 ? 4 : s;
}

template <typename T, int D, int GMAX, int U>
__global__ void __launch_bounds__(128)
decode_simt_kernel(const DecodeParams p) {
  using E = Elem<T>;
  constexpr int LANES = D / 8;          // lanes per token
  constexpr int TPW = 32 / LANES;       // tokens per warp per step
  constexpr int NW = 4;                 // warps per CTA
  constexpr int STRIDE = NW * TPW;      // tokens per CTA per step
  constexpr unsigned FULL = 0xffffffffu;

  const int seq = blockIdx.x;
  const int split = blockIdx.y;
  const int gchunks = (p.group + GMAX - 1) / GMAX;
  const int kvh = blockIdx.z / gchunks;
  const int g0 = (blockIdx.z - kvh * gchunks) * GMAX;
  const int gn = min(GMAX, p.group - g0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lg = lane / LANES, li = lane % LANES;

  int len = p.lens ? __ldg(p.lens + seq) : p.uniform_len;
  const int cap = p.max_blocks * p.block_size;
  if (len > cap) {
    if (threadIdx.x == 0 && split == 0 && blockIdx.z == 0) set_error(p.err, PAGEDKV_EFLAG_SEQ_LEN_RANGE);
    len = cap;
  }
  if (len < 0) len = 0;
  const int t0 = split * p.split_tokens;
  // An empty chunk of a multi-split launch is never read by the combine pass.
  if (p.num_splits > 1 && t0 >= len) return;
  const int t1 = min(len, t0 + p.split_tokens);

  // q for the heads of this chunk: each lane holds its 8 dims of every head.
  float qf[GMAX][8];
  {
    const T *qp = reinterpret_cast<const T *>(p.q) + (int64_t)seq * p.q_ss +
                  (int64_t)(kvh * p.group + g0) * p.q_sh + li * 8;
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g < gn) {
        E::unpack8(ldg16(qp + (int64_t)g * p.q_sh), qf[g]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[g][e] = 0.f;
      }
    }
  }

  float m[GMAX], l[GMAX], acc[GMAX][8];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    m[g] = kNegInf;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
  }

  const int64_t row_elems = (int64_t)p.hkv * D;
  const T *kb = reinterpret_cast<const T *>(p.k) + (int64_t)kvh * D + li * 8;
  const T *vb = reinterpret_cast<const T *>(p.v) + (int64_t)kvh * D + li * 8;
  const int32_t *bt = p.bt + (int64_t)seq * p.bt_s;
  const int my = warp * TPW + lg;

  // Groups of two or more query heads hold enough registers that only two
  // CTAs fit per SM: their K / V rows come through the shared-memory ring.
  // Single-head groups keep eight CTAs per SM on registers alone, which the
  // ring's registers and shared memory would cut (measured slower), so they
  // load straight into registers, one step at a time.
  constexpr bool kStaged = GMAX >= 2;
  constexpr int S = kStaged ? simt_stages<D, GMAX, U>() : 2;
  __shared__ __align__(16) uint4 ring[S][2 * U][NW * 32];  // [step % S][K u | V u][thread]
  uint32_t vmask = 0;  // bit (step % S) * U + u: token u of that step is in range
  const int nsteps = t1 > t0 ? (t1 - t0 + STRIDE * U - 1) / (STRIDE * U) : 0;
  // Copies of step i into ring slot i % S; one commit group per step, empty
  // past the last step, so that the group count stays uniform. issue() is
  // called for i = 0, 1, 2, ... in order, so each token's logical block and
  // offset advance by a fixed amount per call instead of a division.
  int nt[U], nlb[U], noff[U];  // the next step's token, block and offset per u
  const int adv_b = (STRIDE * U) / p.block_size, adv_o = (STRIDE * U) - adv_b * p.block_size;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    nt[u] = t0 + u * STRIDE + my;
    nlb[u] = nt[u] / p.block_size;
    noff[u] = nt[u] - nlb[u] * p.block_size;
  }
  auto issue = [&](int i) {
    if (i < nsteps) {
      const int st = i % S;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        bool ok = nt[u] < t1;
        int64_t o = 0;
        if (ok) {
          const int blk = __ldg(bt + nlb[u]);
          if (blk < 0 || (int64_t)blk >= p.num_blocks) {
            set_error(p.err, PAGEDKV_EFLAG_BLOCK_ID_RANGE);
            ok = false;
          } else {
            o = ((int64_t)blk * p.block_size + noff[u]) * row_elems;
          }
        }
        stage16(&ring[st][u][threadIdx.x], kb + o, ok ? 16u : 0u);
        stage16(&ring[st][U + u][threadIdx.x], vb + o, ok ? 16u : 0u);
        const uint32_t bit = 1u << (st * U + u);
        vmask = ok ? (vmask | bit) : (vmask & ~bit);
        nt[u] += STRIDE * U;
        nlb[u] += adv_b;
        noff[u] += adv_o;
        if (noff[u] >= p.block_size) {
          noff[u] -= p.block_size;
          ++nlb[u];
        }
      }
    }
    stage_commit();
  };
  if constexpr (kStaged) {
#pragma unroll
    for (int i = 0; i < S - 1; ++i) issue(i);
  }

  for (int step = 0; step < nsteps; ++step) {
    uint4 kr[U], vr[U];
    bool valid[U];
    if constexpr (kStaged) {
      stage_wait<S - 2>();  // the group of this step has landed
      const int st = step % S;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        kr[u] = ring[st][u][threadIdx.x];
        vr[u] = ring[st][U + u][threadIdx.x];
        valid[u] = (vmask >> (st * U + u)) & 1u;
      }
      issue(step + S - 1);  // into the slot the previous step read
    } else {
      const int base = t0 + step * STRIDE * U;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int t = base + u * STRIDE + my;
        valid[u] = t < t1;
        kr[u] = make_uint4(0u, 0u, 0u, 0u);
        vr[u] = kr[u];
        if (valid[u]) {
          const int lb = t / p.block_size;
          const int off = t - lb * p.block_size;
          const int blk = __ldg(bt + lb);
          if (blk < 0 || (int64_t)blk >= p.num_blocks) {
            set_error(p.err, PAGEDKV_EFLAG_BLOCK_ID_RANGE);
            valid[u] = false;
          } else {
            const int64_t o = ((int64_t)blk * p.block_size + off) * row_elems;
            kr[u] = ldg_stream16(kb + o);
            vr[u] = ldg_stream16(vb + o);
          }
        }
      }
    }

    float s[U][GMAX];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float kf[8];
      E::unpack8(kr[u], kf);
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) a = fmaf(qf[g][e], kf[e], a);
        s[u][g] = a;
      }
    }
#pragma unroll
    for (int o = LANES / 2; o >= 1; o >>= 1) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) s[u][g] += __shfl_xor_sync(FULL, s[u][g], o);
      }
    }

    float vf[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u) E::unpack8(vr[u], vf[u]);

#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        s[u][g] = valid[u] ? s[u][g] * p.scale_log2 : kNegInf;
        mx = fmaxf(mx, s[u][g]);
      }
      if (mx == kNegInf) continue;  // no valid token seen yet by this lane group
      // Rescale only when the max moved: otherwise the factor is exp2(0) = 1.
      if (mx > m[g]) {
        const float alpha = exp2f(m[g] - mx);
        l[g] *= alpha;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float pr = exp2f(s[u][g] - mx);
        l[g] += pr;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(pr, vf[u][e], acc[g][e]);
      }
      m[g] = mx;
    }
  }

  if constexpr (kStaged) stage_wait<0>();  // the trailing groups are empty; nothing stays in flight

  // Merge the lane groups of each warp (lanes with equal li hold equal dims).
#pragma unroll
  for (int o = LANES; o < 32; o <<= 1) {
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      const float mo = __shfl_xor_sync(FULL, m[g], o);
      const float lo = __shfl_xor_sync(FULL, l[g], o);
      float ao[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) ao[e] = __shfl_xor_sync(FULL, acc[g][e], o);
      const float mn = fmaxf(m[g], mo);
      const float a = (mn == kNegInf) ? 0.f : exp2f(m[g] - mn);
      const float b = (mn == kNegInf) ? 0.f : exp2f(mo - mn);
      l[g] = l[g] * a + lo * b;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] = acc[g][e] * a + ao[e] * b;
      m[g] = mn;
    }
  }

  // Merge the warps through shared memory.
  __shared__ float sm_m[NW][GMAX], sm_l[NW][GMAX];
  __shared__ __align__(16) float sm_acc[NW][GMAX][D];
  if (lg == 0) {
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (li == 0) {
        sm_m[warp][g] = m[g];
        sm_l[warp][g] = l[g];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) sm_acc[warp][g][li * 8 + e] = acc[g][e];
    }
  }
  __syncthreads();

  for (int idx = threadIdx.x; idx < gn * LANES; idx += blockDim.x) {
    const int g = idx / LANES, c = idx % LANES;
    float mm = kNegInf;
#pragma unroll
    for (int w = 0; w < NW; ++w) mm = fmaxf(mm, sm_m[w][g]);
    float ll = 0.f, a[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] = 0.f;
    if (mm != kNegInf) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float f = exp2f(sm_m[w][g] - mm);
        ll += f * sm_l[w][g];
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = fmaf(f, sm_acc[w][g][c * 8 + e], a[e]);
      }
    }
    const int h = kvh * p.group + g0 + g;
    if (p.num_splits == 1) {
      const float inv = ll > 0.f ? 1.f / ll : 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] *= inv;
      stg16(reinterpret_cast<T *>(p.out) + (int64_t)seq * p.o_ss + (int64_t)h * p.o_sh + c * 8,
            E::pack8(a));
    } else {
      const int64_t slot = ((int64_t)seq * p.hq + h) * p.num_splits + split;
      float4 *wa = reinterpret_cast<float4 *>(p.ws_acc + slot * D + c * 8);
      wa[0] = make_float4(a[0], a[1], a[2], a[3]);
      wa[1] = make_float4(a[4], a[5], a[6], a[7]);
      if (c == 0) p.ws_ml[slot] = make_float2(mm, ll);
    }
  }
}

// Final pass of split-K: out = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s.
// One CTA per (sequence, query head); threads stride over head_dim.
template <typename T>
__global__ void __launch_bounds__(128)
decode_combine_kernel(const DecodeParams p) {
  using E = Elem<T>;
  const int seq = blockIdx.x / p.hq;
  const int h = blockIdx.x - seq * p.hq;
  int len = p.lens ? __ldg(p.lens + seq) : p.uniform_len;
  const int cap = p.max_blocks * p.block_size;
  len = max(0, min(len, cap));
  const int ns = min(p.num_splits, (len + p.split_tokens - 1) / p.split_tokens);
  const int64_t slot0 = ((int64_t)seq * p.hq + h) * p.num_splits;
  const float2 *ml = p.ws_ml + slot0;
  float mm = kNegInf;
  for (int s = 0; s < ns; ++s) mm = fmaxf(mm, ml[s].x);
  T *out = reinterpret_cast<T *>(p.out) + (int64_t)seq * p.o_ss + (int64_t)h * p.o_sh;
  for (int d = threadIdx.x; d < p.head_dim; d += blockDim.x) {
    float ll = 0.f, a = 0.f;
    if (mm != kNegInf) {
      for (int s = 0; s < ns; ++s) {
        const float2 v = ml[s];
        const float f = exp2f(v.x - mm);
        ll = fmaf(f, v.y, ll);
        a = fmaf(f, p.ws_acc[(slot0 + s) * p.head_dim + d], a);
      }
    }
    out[d] = E::from_float(ll > 0.f ? a / ll : 0.f);
  }
}

// Query heads per CTA for a GQA group of `group` heads: 1, 2 or 4. Wider
// groups run in chunks of 4: a CTA holding 8 heads' q and accumulators needs
// ~200 registers, which leaves two CTAs per SM. Chunks of 4 fit four, and
// their second read of each K / V row mostly hits L2 (GQA 7 at head_dim 128:
// 753 -> 707 us per launch).
static int simt_group_chunk(int group) { return group <= 1 ? 1 : group <= 2 ? 2 : 4; }

SplitPlan plan_simt_splits(int32_t num_seqs, int32_t num_kv_heads, int32_t group,
                           int32_t max_tokens, int32_t num_sms) {
  SplitPlan plan;
  const int gmax = simt_group_chunk(group);
  const int64_t base = (int64_t)num_seqs * num_kv_heads * ((group + gmax - 1) / gmax);
  const int64_t target = (int64_t)num_sms * 8;  // CTAs to fill the GPU with ~8 per SM
  const int min_split = 256;
  if (max_tokens <= min_split || base >= target || base == 0) {
    plan.split_tokens = max_tokens > 0 ? max_tokens : 1;
    plan.num_splits = 1;
    return plan;
  }
  const int64_t desired = (target + base - 1) / base;
  int64_t split = (max_tokens + desired - 1) / desired;
  if (split < min_split) split = min_split;
  split = (split + 63) / 64 * 64;
  plan.split_tokens = (int32_t)split;
  plan.num_splits = (int32_t)((max_tokens + split - 1) / split);
  if (plan.num_splits <= 1) {
    plan.split_tokens = max_tokens;
    plan.num_splits = 1;
  }
  return plan;
}

// Tokens per lane group per step: more loads in flight and fewer online-softmax
// updates per token, as far as the registers of GMAX query heads allow.
template <int D, int GMAX>
constexpr int simt_unroll() {
  return D <= 64 ? 4 : GMAX <= 2 ? 4 : 2;
}

template <typename T, int D>
static cudaError_t launch_simt_d(const DecodeParams &p, cudaStream_t stream) {
  const int gmax = simt_group_chunk(p.group);
  const int gchunks = (p.group + gmax - 1) / gmax;
  dim3 grid((unsigned)p.num_seqs, (unsigned)p.num_splits, (unsigned)(p.hkv * gchunks));
  switch (gmax) {
    case 1: decode_simt_kernel<T, D, 1, simt_unroll<D, 1>()><<<grid, 128, 0, stream>>>(p); break;
    case 2: decode_simt_kernel<T, D, 2, simt_unroll<D, 2>()><<<grid, 128, 0, stream>>>(p); break;
    default: decode_simt_kernel<T, D, 4, simt_unroll<D, 4>()><<<grid, 128, 0, stream>>>(p); break;
  }
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_simt_t(const DecodeParams &p, cudaStream_t stream) {
  switch (p.head_dim) {
    case 32: return launch_simt_d<T, 32>(p, stream);
    case 64: return launch_simt_d<T, 64>(p, stream);
    case 128: return launch_simt_d<T, 128>(p, stream);
    case 256: return launch_simt_d<T, 256>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_decode_simt(const DecodeParams &p, int dtype, cudaStream_t stream) {
  return dtype == PAGEDKV_DTYPE_BF16 ? launch_simt_t<__nv_bfloat16>(p, stream)
                                     : launch_simt_t<__half>(p, stream);
}

cudaError_t launch_decode_combine(const DecodeParams &p, int dtype, cudaStream_t stream) {
  const unsigned grid = (unsigned)((int64_t)p.num_seqs * p.hq);
  const int threads = p.head_dim < 128 ? p.head_dim : 128;
  if (dtype == PAGEDKV_DTYPE_BF16)
    decode_combine_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(p);
  else
    decode_combine_kernel<__half><<<grid, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace pagedkv
