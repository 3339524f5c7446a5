// Paged GQA decode attention on the 5th-generation tensor cores (sm_100a):
// TMA tile loads of K/V blocks through the block table, tcgen05.mma with TMEM
// accumulators, one persistent CTA per SM.
//
// Math (restates engine/kernels/paged_attention.py:508-631, the batched
// online-softmax kernel; same result as the oracle :30-83):
//   for each sequence s and query head h (kv head h / G):
//     out[s,h] = sum_t softmax_t(scale * q[s,h].K[t]) V[t]  over t < seq_len(s)
//
// B200 mapping
//   * A CTA works on one kv-head GROUP at a time: H = 128 / head_dim kv heads
//     (2 for head_dim 64, 1 for 128), i.e. 128 contiguous elements of every
//     pool row, so all G query heads of those kv heads reuse one K/V read.
//   * Tiles of 128 tokens. Each pool block (block_size rows) of a tile is one
//     2-D TMA box of {64 elements, block_size rows} per 64-element half, with
//     128-byte swizzle: exactly the canonical K-major SW128 layout of a
//     [128 tokens x 128] operand. Blocks past the sequence end are fetched at
//     an out-of-range row and arrive as zeros (no memory traffic).
//   * S^T = K Q^T on the tensor core: M = 128 tokens, N = query columns
//     (H groups of Gp = roundup(G, 8), padded to a multiple of 16), K = 128
//     (block-diagonal Q when H = 2, so one MMA serves both kv heads).
//     Accumulator in TMEM, one token row per TMEM lane.
//   * Softmax warps (128 threads, one token row each) read S, mask tokens past
//     the end, take the tile max with redux.sync, write P (fp16/bf16) to shared
//     memory as the B operand of the second MMA.
//   * O^T = V^T P^T on the tensor core: M = 128 (kv head, dim) rows read from
//     the SAME swizzled V tile as an MN-major operand, N = query columns,
//     K = 128 tokens. Fresh TMEM accumulator per tile; the softmax warps fold
//     it into fp32 registers with the online-softmax rescale.
//   * Work items = (sequence, head group, context chunk); a sequence spanning
//     several chunks writes unnormalised partials and the last CTA to finish
//     it (arrival counter) combines them — no second launch.
//   * Warp roles: warp 0 TMA producer (also stages Q), warp 1 MMA issuer and
//     TMEM owner, warps 2-5 softmax / correction / epilogue.
//   * Every mbarrier wait is bounded (2 s): on timeout the kernel sets
//     PAGEDKV_EFLAG_PIPE_TIMEOUT, unwinds every role, drains its own TMA loads
//     and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "decode_tc.h"
#include "sm100.cuh"

namespace pagedkv {

using namespace sm100;

namespace {

constexpr int kTile = 128;                 // tokens per tile (MMA M of S^T)
constexpr int kHalfBytes = kTile * 128;    // one 64-element half of a tile: 16 KB
constexpr int kOperandBytes = 2 * kHalfBytes;  // [128 x 128] K or V tile: 32 KB
constexpr int kThreads = 192;              // 6 warps
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct TcParams {
  DecodeParams p;
  int32_t head_groups;   // ceil(hkv / H)
  int32_t total_items;   // num_seqs * head_groups * num_splits
  int32_t oob_row;       // num_blocks * block_size: first row past the pool
  int32_t *counters;     // [num_seqs * head_groups] arrival counters, or null
};

struct Item {
  int seq, hg, c, len, t0, t1, ntiles, nck;
};

__device__ __forceinline__ Item item_info(const TcParams &tp, int item) {
  const DecodeParams &p = tp.p;
  Item it;
  const int per_seq = tp.head_groups * p.num_splits;
  it.seq = item / per_seq;
  const int rem = item - it.seq * per_seq;
  it.hg = rem / p.num_splits;
  it.c = rem - it.hg * p.num_splits;
  int len = p.lens ? __ldg(p.lens + it.seq) : p.uniform_len;
  const int cap = p.max_blocks * p.block_size;
  len = len > cap ? cap : len;
  len = len < 0 ? 0 : len;
  it.len = len;
  it.t0 = it.c * p.split_tokens;
  it.t1 = min(len, it.t0 + p.split_tokens);
  it.ntiles = it.t1 > it.t0 ? (it.t1 - it.t0 + kTile - 1) / kTile : 0;
  it.nck = (len + p.split_tokens - 1) / p.split_tokens;
  return it;
}

template <int N, int STAGES>
struct SmemLayout {
  static constexpr int kQBytes = 2 * N * 128;  // B operand [N x 128], two K-halves
  static constexpr int kPBytes = 2 * N * 128;  // B operand [N x 128 tokens], two K-halves
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + STAGES * kOperandBytes;
  static constexpr int kOffQ = kOffV + STAGES * kOperandBytes;
  static constexpr int kOffP = kOffQ + 2 * kQBytes;
  static constexpr int kOffRedMax = kOffP + 2 * kPBytes;         // float [2][4][N]
  static constexpr int kOffRedL = kOffRedMax + 2 * 4 * N * 4;    // float [4][N]
  static constexpr int kOffBars = kOffRedL + 4 * N * 4;          // uint64 barriers
  // kfull, vfull, empty [STAGES]; s_full, s_empty, p_full, p_empty, o_full,
  // o_empty, q_full, q_empty [2]; mma_done [1]
  static constexpr int kNumBars = 3 * STAGES + 8 * 2 + 1;
  static constexpr int kOffMisc = kOffBars + kNumBars * 8;       // tmem base, abort, flag
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

template <typename T, int H, int GP, int N, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
decode_tc_kernel(const __grid_constant__ CUtensorMap tmap_k,
                 const __grid_constant__ CUtensorMap tmap_v, const TcParams tp) {
  using L = SmemLayout<N, STAGES>;
  using E = Elem<T>;
  constexpr int D = 128 / H;                   // head_dim
  constexpr uint32_t kCols = 4 * N;            // TMEM: S[2] then O[2]
  constexpr uint32_t kFmt = E::kDtype == PAGEDKV_DTYPE_BF16 ? 1u : 0u;
  constexpr uint32_t kIdescS = idesc_f16(kFmt, N, false, false);
  constexpr uint32_t kIdescO = idesc_f16(kFmt, N, true, false);
  static_assert(H * GP <= N && N % 16 == 0 && N <= 32, "column layout");

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::kOffBars;
  auto kfull = [&](int s) { return bars + 8u * s; };
  auto vfull = [&](int s) { return bars + 8u * (STAGES + s); };
  auto empty = [&](int s) { return bars + 8u * (2 * STAGES + s); };
  auto bar2 = [&](int which, int b) { return bars + 8u * (3 * STAGES + 2 * which + b); };
  // which: 0 s_full, 1 s_empty, 2 p_full, 3 p_empty, 4 o_full, 5 o_empty, 6 q_full, 7 q_empty
  const uint32_t mma_done = bars + 8u * (3 * STAGES + 16);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kOffMisc);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::kOffMisc + 4);
  volatile int *combine_flag = reinterpret_cast<volatile int *>(smem + L::kOffMisc + 8);
  float *red_max = reinterpret_cast<float *>(smem + L::kOffRedMax);
  float *red_l = reinterpret_cast<float *>(smem + L::kOffRedL);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const DecodeParams &p = tp.p;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(kfull(s), 1);
      mbar_init(vfull(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar2(0, b), 1);    // s_full: MMA commit
      mbar_init(bar2(1, b), 128);  // s_empty: every softmax thread
      mbar_init(bar2(2, b), 128);  // p_full
      mbar_init(bar2(3, b), 1);    // p_empty: MMA commit
      mbar_init(bar2(4, b), 1);    // o_full: MMA commit
      mbar_init(bar2(5, b), 128);  // o_empty
      mbar_init(bar2(6, b), 32);   // q_full: every producer lane
      mbar_init(bar2(7, b), 1);    // q_empty: MMA commit
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    *combine_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
    }
    const uint64_t policy = l2_policy_evict_first();
    const int blocks_per_tile = kTile / p.block_size;
    int stage = 0;
    uint32_t sphase = 0;
    uint32_t qi = 0;
    int issued = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < tp.total_items; item += gridDim.x) {
      const Item it = item_info(tp, item);
      if (it.ntiles == 0) continue;
      // Stage Q for this item: block-diagonal B operand [N rows x 128], K-major SW128.
      const uint32_t qb = qi & 1u;
      if (!mbar_wait(bar2(7, qb), ((qi >> 1) & 1u) ^ 1u, abort_flag, kTimeoutNs)) { ok = false; break; }
      const uint32_t qbuf = sbase + L::kOffQ + qb * L::kQBytes;
      for (int idx = lane; idx < 16 * N; idx += 32) {
        const int xh = idx / (8 * N);
        const int rem = idx - xh * 8 * N;
        const int n = rem >> 3, ch = rem & 7;
        const int hl = n / GP, g = n - hl * GP;
        const int kv = it.hg * H + hl;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (hl < H && g < p.group && kv < p.hkv && (H == 1 || xh == hl)) {
          const int d = (H == 1 ? xh * 64 : 0) + ch * 8;
          val = ldg16(reinterpret_cast<const T *>(p.q) + (int64_t)it.seq * p.q_ss +
                      (int64_t)(kv * p.group + g) * p.q_sh + d);
        }
        const uint32_t addr = qbuf + xh * (N * 128) + (n >> 3) * 1024 + (n & 7) * 128 + ((ch ^ (n & 7)) << 4);
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(val.x), "r"(val.y),
                     "r"(val.z), "r"(val.w)
                     : "memory");
      }
      fence_proxy_async_smem();
      mbar_arrive(bar2(6, qb));
      ++qi;
      const int need_blocks = (it.t1 + p.block_size - 1) / p.block_size;
      const int32_t *bt = p.bt + (int64_t)it.seq * p.bt_s;
      const int x0 = it.hg * 128;
      for (int j = 0; j < it.ntiles; ++j) {
        if (!mbar_wait(empty(stage), sphase ^ 1u, abort_flag, kTimeoutNs)) { ok = false; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(kfull(stage), kOperandBytes);
          mbar_arrive_expect_tx(vfull(stage), kOperandBytes);
        }
        __syncwarp();
        const int lb0 = (it.t0 + j * kTile) / p.block_size;
        const uint32_t kdst = sbase + L::kOffK + stage * kOperandBytes;
        const uint32_t vdst = sbase + L::kOffV + stage * kOperandBytes;
        for (int bi = lane; bi < blocks_per_tile; bi += 32) {
          const int lb = lb0 + bi;
          int32_t y = tp.oob_row;  // out of range: TMA fills zeros, reads nothing
          if (lb < need_blocks) {
            const int blk = __ldg(bt + lb);
            if (blk >= 0 && (int64_t)blk < p.num_blocks) {
              y = blk * p.block_size;
            } else {
              set_error(p.err, PAGEDKV_EFLAG_BLOCK_ID_RANGE);
            }
          }
          const uint32_t off = bi * p.block_size * 128;
#pragma unroll
          for (int xh = 0; xh < 2; ++xh) {
            tma_load_2d(kdst + xh * kHalfBytes + off, &tmap_k, x0 + xh * 64, y, kfull(stage), policy);
            tma_load_2d(vdst + xh * kHalfBytes + off, &tmap_v, x0 + xh * 64, y, vfull(stage), policy);
          }
        }
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          sphase ^= 1u;
        }
      }
    }
    // Drain: the last min(issued, STAGES) tiles' loads must have landed before
    // this CTA's shared memory is released (immediate on the normal path).
    for (int k = 0; k < STAGES && k < issued; ++k) {
      if (--stage < 0) {
        stage = STAGES - 1;
        sphase ^= 1u;
      }
      volatile int never = 0;
      mbar_wait(kfull(stage), sphase, &never, kTimeoutNs / 4);
      mbar_wait(vfull(stage), sphase, &never, kTimeoutNs / 4);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA issuer
    int stage = 0;
    uint32_t sphase = 0;
    uint32_t gt = 0;  // global tile counter (S/P/O double buffers)
    uint32_t qi = 0;
    bool ok = true;
    auto issue_s = [&](int st, uint32_t ph, uint32_t g, uint32_t qbuf) -> bool {
      const uint32_t b = g & 1u;
      if (!mbar_wait(kfull(st), ph, abort_flag, kTimeoutNs)) return false;
      if (!mbar_wait(bar2(1, b), ((g >> 1) & 1u) ^ 1u, abort_flag, kTimeoutNs)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t ka = sbase + L::kOffK + st * kOperandBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = smem_desc_sw128(ka + (kk >> 2) * kHalfBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(qbuf + (kk >> 2) * (N * 128) + (kk & 3) * 32, 16, 1024);
          mma_f16_ss(tmem + b * N, ad, bd, kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar2(0, b));
      }
      __syncwarp();
      return true;
    };
    for (int item = blockIdx.x; ok && item < tp.total_items; item += gridDim.x) {
      const Item it = item_info(tp, item);
      if (it.ntiles == 0) continue;
      const uint32_t qb = qi & 1u;
      if (!mbar_wait(bar2(6, qb), (qi >> 1) & 1u, abort_flag, kTimeoutNs)) { ok = false; break; }
      const uint32_t qbuf = sbase + L::kOffQ + qb * L::kQBytes;
      if (!issue_s(stage, sphase, gt, qbuf)) { ok = false; break; }
      for (int j = 0; j < it.ntiles; ++j) {
        const uint32_t b = gt & 1u;
        const uint32_t bph = (gt >> 1) & 1u;
        int nstage = stage + 1;
        uint32_t nphase = sphase;
        if (nstage == STAGES) {
          nstage = 0;
          nphase ^= 1u;
        }
        if (j + 1 < it.ntiles) {
          if (!issue_s(nstage, nphase, gt + 1, qbuf)) { ok = false; break; }
        }
        if (!mbar_wait(vfull(stage), sphase, abort_flag, kTimeoutNs)) { ok = false; break; }
        const uint32_t va = sbase + L::kOffV + stage * kOperandBytes;
        // Rows of the last block past the sequence end hold stale pool data:
        // zero them so 0 * (non-finite stale value) never reaches the sum.
        if (j == it.ntiles - 1 && it.t1 == it.len && (it.len % p.block_size) != 0) {
          const int r0 = it.len - (it.t0 + j * kTile);  // first stale row in the tile
          const int r1 = ((it.len + p.block_size - 1) / p.block_size) * p.block_size - (it.t0 + j * kTile);
          const int chunks = (r1 - r0) * 8 * 2;
          for (int idx = lane; idx < chunks; idx += 32) {
            const int xh = idx / ((r1 - r0) * 8);
            const int rr = idx - xh * (r1 - r0) * 8;
            const uint32_t addr = va + xh * kHalfBytes + (r0 + (rr >> 3)) * 128 + (rr & 7) * 16;
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(addr), "r"(0u) : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        if (!mbar_wait(bar2(2, b), bph, abort_flag, kTimeoutNs)) { ok = false; break; }
        if (!mbar_wait(bar2(5, b), bph ^ 1u, abort_flag, kTimeoutNs)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t pbuf = sbase + L::kOffP + b * L::kPBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            // A = V^T: MN-major SW128, 64-element atoms 16 KB apart (LBO), 8-token groups 1 KB apart (SBO)
            const uint64_t ad = smem_desc_sw128(va + kk * 2048, kHalfBytes, 1024);
            const uint64_t bd = smem_desc_sw128(pbuf + (kk >> 2) * (N * 128) + (kk & 3) * 32, 16, 1024);
            mma_f16_ss(tmem + 2 * N + b * N, ad, bd, kIdescO, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar2(4, b));   // o_full
          mma_commit(empty(stage));  // K/V stage free
          mma_commit(bar2(3, b));   // p_empty
          if (j == it.ntiles - 1) mma_commit(bar2(7, qb));  // q_empty
        }
        __syncwarp();
        ++gt;
        stage = nstage;
        sphase = nphase;
      }
      ++qi;
    }
    // Every MMA this thread issued has completed before TMEM is released.
    if (lane == 0) mma_commit(mma_done);
    __syncwarp();
    volatile int never = 0;
    mbar_wait(mma_done, 0, &never, kTimeoutNs / 4);
  } else {
    // ------------------------------------------------- softmax / correction / epilogue
    const int q4 = warp & 3;            // TMEM lane quarter of this warp
    const int row = q4 * 32 + lane;     // TMEM lane: token row (S) / (kv head, dim) row (O)
    const int hl = H == 2 ? (row >> 6) : 0;
    const int dim = H == 2 ? (row & 63) : row;
    const uint32_t tl = tmem + ((uint32_t)(q4 * 32) << 16);
    uint32_t gt = 0;
    int red_buf = 0;
    for (int item = blockIdx.x; item < tp.total_items; item += gridDim.x) {
      const Item it = item_info(tp, item);
      if (it.ntiles == 0 && !(it.len == 0 && it.c == 0)) continue;
      if (it.c == 0 && row == 0 && it.hg == 0) {
        int raw = p.lens ? __ldg(p.lens + it.seq) : p.uniform_len;
        if (raw > p.max_blocks * p.block_size) set_error(p.err, PAGEDKV_EFLAG_SEQ_LEN_RANGE);
      }
      float m_run[N], l_part[N], alpha_prev[N], acc[GP];
#pragma unroll
      for (int n = 0; n < N; ++n) {
        m_run[n] = kNegInf;
        l_part[n] = 0.f;
        alpha_prev[n] = 1.f;
      }
#pragma unroll
      for (int g = 0; g < GP; ++g) acc[g] = 0.f;

      // On a timed-out wait the pipeline is abandoned but the control flow of
      // these 128 threads stays uniform (they share named barriers): later
      // waits return at once and the results are garbage, flagged by the
      // PIPE_TIMEOUT bit.
      auto correction = [&](uint32_t g_tile) {
        const uint32_t b = g_tile & 1u;
        mbar_wait(bar2(4, b), (g_tile >> 1) & 1u, abort_flag, kTimeoutNs);
        tc_fence_after();
        float o[GP];
        tmem_ld<GP>(tl + 2 * N + b * N + hl * GP, o);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(bar2(5, b));
#pragma unroll
        for (int g = 0; g < GP; ++g) {
          const float a = (H == 2 && hl == 1) ? alpha_prev[(GP + g) % N] : alpha_prev[g];
          acc[g] = fmaf(acc[g], a, o[g]);
        }
      };

      for (int j = 0; j < it.ntiles; ++j) {
        const uint32_t b = gt & 1u;
        const uint32_t bph = (gt >> 1) & 1u;
        mbar_wait(bar2(0, b), bph, abort_flag, kTimeoutNs);
        tc_fence_after();
        float s[N];
        tmem_ld<N>(tl + b * N, s);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(bar2(1, b));

        const bool valid = it.t0 + j * kTile + row < it.t1;
        float *rm = red_max + red_buf * 4 * N;
#pragma unroll
        for (int n = 0; n < N; ++n) {
          s[n] = valid ? s[n] * p.scale_log2 : kNegInf;
          const float wm = warp_max(s[n]);
          if (lane == 0) rm[q4 * N + n] = wm;
        }
        named_bar(1, 128);
        float alpha[N];
#pragma unroll
        for (int n = 0; n < N; ++n) {
          const float mt = fmaxf(fmaxf(rm[n], rm[N + n]), fmaxf(rm[2 * N + n], rm[3 * N + n]));
          const float mn = fmaxf(m_run[n], mt);
          alpha[n] = mn == kNegInf ? 1.f : exp2f(m_run[n] - mn);
          // The denominator sums P as rounded for the MMA, so the normalisation
          // matches the numerator exactly.
          const float pr = E::to_float(E::from_float(valid ? exp2f(s[n] - mn) : 0.f));
          s[n] = pr;
          l_part[n] = fmaf(l_part[n], alpha[n], pr);
          m_run[n] = mn;
        }
        red_buf ^= 1;
        mbar_wait(bar2(3, b), bph ^ 1u, abort_flag, kTimeoutNs);
        // P^T as the B operand [N x 128 tokens], K-major SW128: token `row` of column n.
        const uint32_t pbuf = sbase + L::kOffP + b * L::kPBytes + (row >> 6) * (N * 128);
        const int tr = row & 63;
#pragma unroll
        for (int n = 0; n < N; ++n) {
          const uint32_t addr = pbuf + (n >> 3) * 1024 + (n & 7) * 128 + ((((tr >> 3) ^ (n & 7))) << 4) + (tr & 7) * 2;
          const T hv = E::from_float(s[n]);
          asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(*reinterpret_cast<const uint16_t *>(&hv))
                       : "memory");
        }
        fence_proxy_async_smem();
        mbar_arrive(bar2(2, b));
        if (j > 0) correction(gt - 1);
#pragma unroll
        for (int n = 0; n < N; ++n) alpha_prev[n] = alpha[n];
        ++gt;
      }
      if (it.ntiles > 0) correction(gt - 1);

      // ---- epilogue: denominators across the 128 rows
#pragma unroll
      for (int n = 0; n < N; ++n) {
        float v = l_part[n];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red_l[q4 * N + n] = v;
      }
      named_bar(1, 128);
      float l_sel[GP], m_sel[GP];
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        const int n0 = g, n1 = GP + g;
        const float l0 = red_l[n0] + red_l[N + n0] + red_l[2 * N + n0] + red_l[3 * N + n0];
        float l1 = 0.f;
        if (H == 2) l1 = red_l[n1 % N] + red_l[N + n1 % N] + red_l[2 * N + n1 % N] + red_l[3 * N + n1 % N];
        l_sel[g] = (H == 2 && hl == 1) ? l1 : l0;
        m_sel[g] = (H == 2 && hl == 1) ? m_run[(GP + g) % N] : m_run[g];
      }
      named_bar(1, 128);  // red_l is rewritten by the next item

      const int kv = it.hg * H + hl;
      const bool have = kv < p.hkv;
      if (it.nck <= 1) {
        if (have) {
          T *out = reinterpret_cast<T *>(p.out) + (int64_t)it.seq * p.o_ss + dim;
#pragma unroll
          for (int g = 0; g < GP; ++g) {
            if (g < p.group) {
              const float v = l_sel[g] > 0.f ? acc[g] / l_sel[g] : 0.f;
              out[(int64_t)(kv * p.group + g) * p.o_sh] = E::from_float(v);
            }
          }
        }
      } else {
        if (have) {
#pragma unroll
          for (int g = 0; g < GP; ++g) {
            if (g < p.group) {
              const int64_t slot = ((int64_t)it.seq * p.hq + kv * p.group + g) * p.num_splits + it.c;
              p.ws_acc[slot * D + dim] = acc[g];
              if (dim == 0) p.ws_ml[slot] = make_float2(m_sel[g], l_sel[g]);
            }
          }
        }
        __threadfence();
        named_bar(1, 128);
        if (row == 0) {
          const int prev = atomicAdd(tp.counters + (int64_t)it.seq * tp.head_groups + it.hg, 1);
          *combine_flag = prev == it.nck - 1 ? 1 : 0;
        }
        named_bar(1, 128);
        if (*combine_flag) {
          __threadfence();
          if (have) {
            T *out = reinterpret_cast<T *>(p.out) + (int64_t)it.seq * p.o_ss + dim;
            for (int g = 0; g < p.group && g < GP; ++g) {
              const int64_t slot0 = ((int64_t)it.seq * p.hq + kv * p.group + g) * p.num_splits;
              float mm = kNegInf;
              for (int cc = 0; cc < it.nck; ++cc) mm = fmaxf(mm, __ldcg(&p.ws_ml[slot0 + cc].x));
              float ll = 0.f, a = 0.f;
              if (mm != kNegInf) {
                for (int cc = 0; cc < it.nck; ++cc) {
                  const float2 ml = __ldcg(&p.ws_ml[slot0 + cc]);
                  const float f = exp2f(ml.x - mm);
                  ll = fmaf(f, ml.y, ll);
                  a = fmaf(f, __ldcg(&p.ws_acc[(slot0 + cc) * D + dim]), a);
                }
              }
              out[(int64_t)(kv * p.group + g) * p.o_sh] = E::from_float(ll > 0.f ? a / ll : 0.f);
            }
          }
        }
        named_bar(1, 128);  // combine_flag is rewritten by the next item
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  if (threadIdx.x == 0 && *abort_flag) set_error(p.err, PAGEDKV_EFLAG_PIPE_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// ---- host side ----------------------------------------------------------------

struct TcPlan {
  int H, GP, N, stages, head_groups, chunk, num_chunks;
};

int round_up(int x, int m) { return (x + m - 1) / m * m; }

TcPlan make_plan(int32_t num_seqs, int32_t hq, int32_t hkv, int32_t head_dim, int32_t max_tokens,
                 int32_t num_sms) {
  TcPlan pl;
  pl.H = 128 / head_dim;
  const int G = hq / hkv;
  pl.GP = round_up(G, 8);
  pl.N = round_up(pl.H * pl.GP, 16);
  pl.stages = pl.N <= 16 ? 3 : 2;
  pl.head_groups = (hkv + pl.H - 1) / pl.H;
  const int mt = max_tokens > 0 ? max_tokens : 1;
  int chunk = round_up(mt, kTile);
  const int64_t want = (int64_t)num_sms * 4;
  while (chunk > 2 * kTile) {
    const int64_t items = (int64_t)num_seqs * pl.head_groups * ((mt + chunk - 1) / chunk);
    if (items >= want) break;
    chunk = round_up(chunk / 2, kTile);
  }
  pl.chunk = chunk;
  pl.num_chunks = (mt + chunk - 1) / chunk;
  return pl;
}

size_t plan_workspace(const TcPlan &pl, int32_t num_seqs, int32_t hq, int32_t head_dim) {
  if (pl.num_chunks <= 1) return 0;
  const size_t slots = (size_t)num_seqs * hq * pl.num_chunks;
  const size_t acc = ((slots * head_dim * sizeof(float) + 255) / 256) * 256;
  const size_t ml = ((slots * sizeof(float2) + 255) / 256) * 256;
  const size_t cnt = (size_t)num_seqs * pl.head_groups * sizeof(int32_t);
  return acc + ml + cnt;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

bool make_map(CUtensorMap *map, const void *base, int dtype, uint64_t row_elems, uint64_t rows,
              uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {row_elems, rows};
  cuuint64_t strides[1] = {row_elems * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype == PAGEDKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int H, int GP, int N, int STAGES>
cudaError_t launch_tc(const CUtensorMap &mk, const CUtensorMap &mv, const TcParams &tp, int grid,
                      cudaStream_t stream) {
  using L = SmemLayout<N, STAGES>;
  auto kern = decode_tc_kernel<T, H, GP, N, STAGES>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, L::kAlloc, stream>>>(mk, mv, tp);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_tc(const TcPlan &pl, const CUtensorMap &mk, const CUtensorMap &mv, const TcParams &tp,
                        int grid, cudaStream_t stream) {
  if (pl.H == 2 && pl.GP == 8) return launch_tc<T, 2, 8, 16, 3>(mk, mv, tp, grid, stream);
  if (pl.H == 2 && pl.GP == 16) return launch_tc<T, 2, 16, 32, 2>(mk, mv, tp, grid, stream);
  if (pl.H == 1 && pl.GP == 8) return launch_tc<T, 1, 8, 16, 3>(mk, mv, tp, grid, stream);
  if (pl.H == 1 && pl.GP == 16) return launch_tc<T, 1, 16, 16, 3>(mk, mv, tp, grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace

bool tc_eligible(int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size) {
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return false;
  const int G = num_q_heads / num_kv_heads;
  if (head_dim != 64 && head_dim != 128) return false;
  if (G < 4 || G > 16) return false;
  if (block_size < 8 || block_size > 128 || (block_size & (block_size - 1)) != 0) return false;
  return true;
}

size_t tc_workspace_bytes(int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t max_tokens, int32_t num_sms) {
  const TcPlan pl = make_plan(num_seqs, num_q_heads, num_kv_heads, head_dim, max_tokens, num_sms);
  return plan_workspace(pl, num_seqs, num_q_heads, head_dim);
}

int tc_launch(DecodeParams &p, int dtype, void *workspace, size_t workspace_bytes, int32_t num_sms,
              cudaStream_t stream, int *launches, std::string *error) {
  *launches = 0;
  const int32_t max_tokens = p.max_blocks * p.block_size;
  const TcPlan pl = make_plan(p.num_seqs, p.hq, p.hkv, p.head_dim, max_tokens, num_sms);
  const size_t need = plan_workspace(pl, p.num_seqs, p.hq, p.head_dim);
  if (need > workspace_bytes) {
    *error = "tensor-core decode: workspace too small";
    return PAGEDKV_ERR_WORKSPACE;
  }
  const int64_t rows = p.num_blocks * (int64_t)p.block_size;
  if (rows >= 0x7fffffffLL) {
    *error = "tensor-core decode: num_blocks * block_size must be < 2^31";
    return PAGEDKV_ERR_INVALID_ARGUMENT;
  }
  CUtensorMap mk, mv;
  const uint64_t row_elems = (uint64_t)p.hkv * p.head_dim;
  if (!make_map(&mk, p.k, dtype, row_elems, (uint64_t)rows, (uint32_t)p.block_size) ||
      !make_map(&mv, p.v, dtype, row_elems, (uint64_t)rows, (uint32_t)p.block_size)) {
    *error = "tensor-core decode: cuTensorMapEncodeTiled failed";
    return PAGEDKV_ERR_CUDA;
  }
  TcParams tp{};
  p.split_tokens = pl.chunk;
  p.num_splits = pl.num_chunks;
  tp.head_groups = pl.head_groups;
  tp.oob_row = (int32_t)rows;
  const int64_t items = (int64_t)p.num_seqs * pl.head_groups * pl.num_chunks;
  if (items > 0x7fffffffLL) {
    *error = "tensor-core decode: too many work items";
    return PAGEDKV_ERR_INVALID_ARGUMENT;
  }
  tp.total_items = (int32_t)items;
  int n_launch = 1;
  if (need > 0) {
    const size_t slots = (size_t)p.num_seqs * p.hq * pl.num_chunks;
    const size_t acc = ((slots * p.head_dim * sizeof(float) + 255) / 256) * 256;
    const size_t ml = ((slots * sizeof(float2) + 255) / 256) * 256;
    p.ws_acc = static_cast<float *>(workspace);
    p.ws_ml = reinterpret_cast<float2 *>(static_cast<char *>(workspace) + acc);
    tp.counters = reinterpret_cast<int32_t *>(static_cast<char *>(workspace) + acc + ml);
    cudaError_t e = cudaMemsetAsync(tp.counters, 0, (size_t)p.num_seqs * pl.head_groups * sizeof(int32_t), stream);
    if (e != cudaSuccess) {
      *error = std::string("tensor-core decode: counter reset: ") + cudaGetErrorString(e);
      return PAGEDKV_ERR_CUDA;
    }
    ++n_launch;
  }
  tp.p = p;
  const int grid = (int)(items < num_sms ? items : num_sms);
  cudaError_t e = dtype == PAGEDKV_DTYPE_BF16 ? dispatch_tc<__nv_bfloat16>(pl, mk, mv, tp, grid, stream)
                                              : dispatch_tc<__half>(pl, mk, mv, tp, grid, stream);
  if (e != cudaSuccess) {
    *error = std::string("tensor-core decode launch: ") + cudaGetErrorString(e);
    return PAGEDKV_ERR_CUDA;
  }
  *launches = n_launch;
  return PAGEDKV_OK;
}

}  // namespace pagedkv
