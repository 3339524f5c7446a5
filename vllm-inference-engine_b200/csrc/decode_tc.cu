// Paged GQA decode attention on the 5th-generation tensor cores (sm_100a):
// TMA tile loads of K/V blocks through the block table, tcgen05.mma with TMEM
// accumulators, one persistent CTA per SM, stream-K work split.
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
//     the end, vote on a lazy rescale (the tile max is reduced only when some
//     score exceeds the reference max by 2^8), write P (fp16/bf16) to shared
//     memory as the (MN-major) B operand of the second MMA, and keep per-row
//     denominators that one butterfly reduction per piece hands over.
//   * O^T = V^T P^T on the tensor core: M = 128 (kv head, dim) rows read from
//     the SAME swizzled V tile as an MN-major operand, N = query columns,
//     K = 128 tokens. Fresh TMEM accumulator per tile (double-buffered).
//   * Correction warps (128 threads, one (kv head, dim) row each) fold every
//     tile's O into fp32 registers with the rescale factors the softmax warps
//     record per tile, then normalise and store, publish a partial, or
//     combine partials — off the softmax warps' path, so a piece boundary does
//     not stall S -> P.
//   * Work split (stream-K): the (sequence, head group) segments are laid end
//     to end as one sequence of 128-token tiles; range r takes tiles
//     [r*T/grid, (r+1)*T/grid) and runs in block grid - 1 - r. A segment cut
//     by range boundaries is combined by the CTA holding its first tile, at
//     the end of its range; the other pieces are the first pieces of the
//     following ranges, published early (partial + release flag) by
//     lower-numbered blocks, so a combining CTA only ever waits on CTAs
//     dispatched before it — no second launch, equal tiles per SM.
//   * Warp roles (12 warps): 0 K-tile TMA producer (also copies each piece's
//     Q; with RoPE the V producer rotates it in place), 6 V-tile TMA producer,
//     1 S-MMA issuer (TMEM owner), 11 O-MMA issuer, 2-5 softmax, 7-10
//     correction / epilogue. With the fused decode append, the two MMA
//     issuers patch the new K / V row into the landed tile (and the pool).
//     Each tcgen05.mma costs its issuing thread tens of nanoseconds, so S and
//     O are issued from two warps. K and V have separate smem rings: a K tile
//     is freed once the S MMA has read it, so K prefetch runs deeper than V.
//     Block-table entries and Q are copied ahead with cp.async, so no TMA
//     issue waits on L2.
//   * Every mbarrier wait is bounded (2 s): on timeout the kernel sets
//     PAGEDKV_EFLAG_PIPE_TIMEOUT, unwinds every role, drains its own TMA loads
//     and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "decode_tc.h"
#include "sm100.cuh"

namespace pagedkv {

using namespace sm100;

namespace {

constexpr int kTile = 128;                     // tokens per tile (MMA M of S^T)
constexpr int kHalfBytes = kTile * 128;        // one 64-element half of a tile: 16 KB
constexpr int kOperandBytes = 2 * kHalfBytes;  // [128 x 128] K or V tile: 32 KB
constexpr int kThreads = 384;                  // 12 warps
constexpr int kRescaleSlots = 4;               // softmax -> correction records in flight
constexpr int kQSlots = 4;                     // staged Q operands (pieces) in flight
constexpr int kLSlots = 8;                     // per-piece denominator partials in flight
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr float kRescaleLog2 = 8.f;            // lazy-rescale threshold (log2 units)

// Optional wait-time trace (build with -DPAGEDKV_TRACE; off in the product
// build): per CTA and warp role, nanoseconds spent in each pipeline wait.
#ifdef PAGEDKV_TRACE
constexpr int kTraceSlots = 16;
constexpr int kTraceCtas = 160;
__device__ unsigned long long g_trace[kTraceCtas][7][kTraceSlots];
// Timeline of the last kTraceRecs CTA runs, indexed by a ticket every CTA
// takes at entry (launch = ticket / grid: a launch's CTAs all start before
// the next launch may): ticket, %smid, entry, after the dependency wait,
// first S tile ready, exit, then the start-up steps: range prologue done,
// K producer's first block-table window landed, its first TMA issued, S
// issuer's first Q ready, its first K tile landed, the K producer's role
// entry, its first two windows issued, its first Q issued, and within the
// role entry: descriptor prefetch and policy done, first window piece walked,
// first window issued, then a walker probe: the same walker step twice from
// one call site, then once from another. Columns 6 on are SM clock64 cycles,
// column 20 the clock64 cycle right after the dependency wait.
constexpr int kTraceRecs = 160 * 48;
constexpr int kTraceCols = 21;  // columns 17-19: first ring fill sized, its block ids landed, its first stage issued
__device__ unsigned long long g_tl[kTraceRecs][kTraceCols];
__device__ unsigned long long g_tl_ctr;
#define PKV_TW(slot, expr)             \
  ([&]() {                              \
    const uint64_t _t0 = clock64();     \
    const auto _r = (expr);             \
    tw[slot] += clock64() - _t0;        \
    return _r;                          \
  }())
#define PKV_TV(slot, stmt)              \
  do {                                  \
    const uint64_t _t0 = clock64();     \
    stmt;                               \
    tw[slot] += clock64() - _t0;        \
  } while (0)
#define PKV_TADD(slot, v) (tw[slot] += (v))
#define PKV_STAMP(var) const uint64_t var = clock64()
#define PKV_TL(col) (g_tl[misc->tl_ticket % kTraceRecs][col] = clock64())
#else
#define PKV_TW(slot, expr) (expr)
#define PKV_TV(slot, stmt) stmt
#define PKV_TADD(slot, v) ((void)0)
#define PKV_STAMP(var) ((void)0)
#define PKV_TL(col) ((void)0)
#endif

struct TcParams {
  DecodeParams p;
  int32_t head_groups;  // segments per sequence: ceil(hkv / H) tile rows x chunks
  int32_t chunks;       // query-head chunks of GP heads per kv head (groups wider than GP)
  int32_t oob_row;      // num_blocks * block_size: first row past the pool
  float *part_acc;      // [grid][H * GP][head_dim] published partial sums
  float2 *part_ml;      // [grid][H * GP] (reference max, denominator) of those
  uint32_t *flags;      // [grid] 1 = CTA's partial published; reset to 0 when consumed
  // Decode append fused into the launch (k_new == nullptr: none). Sequence s's
  // new K / V rows [hkv, head_dim] (strides in elements) are written into its
  // pool slot at position len - 1 by the CTA that reads that tile, before its
  // TMA load of the tile; with cos != nullptr, K and q are rotated first.
  const void *k_new, *v_new;
  int64_t kn_st, kn_sh, vn_st, vn_sh;
  const void *cos, *sin;  // [num_seqs, head_dim] rows, stride cs_st
  int64_t cs_st;
};

__device__ __forceinline__ int seq_len_clamped(const DecodeParams &p, int seq) {
  int len = p.lens ? __ldg(p.lens + seq) : p.uniform_len;
  const int cap = p.max_blocks * p.block_size;
  len = len > cap ? cap : len;
  return len < 0 ? 0 : len;
}

__device__ __forceinline__ int tiles_of(int len) { return (len + kTile - 1) / kTile; }

// Stream-K cost model. The segments are laid end to end in cost units: a
// segment of nt tiles costs kSegUnits + nt * kTileUnits (the per-segment part
// is its first piece's fixed work: Q copy, the full max reduction of its first
// tile, the epilogue; measured, a one-tile segment costs about two streaming
// tiles). Range b takes the units [b*U/G, (b+1)*U/G) and owns every tile whose
// last unit falls in them, so SMs that draw many short sequences get fewer
// tiles and each CTA still owns one contiguous run of tiles.
constexpr int64_t kTileUnits = 8;
constexpr int64_t kSegUnits = 8;

// First unit of range b and the range owning unit u, for U units over G ranges.
__device__ __forceinline__ int64_t range_lo(int64_t b, int64_t U, int64_t G) { return b * U / G; }
__device__ __forceinline__ int64_t owner_of(int64_t u, int64_t U, int64_t G) {
  return ((u + 1) * G + U - 1) / U - 1;
}

// One contiguous run of tiles of a (sequence, head group) segment. Head group
// hg is tile row hg / chunks (H kv heads at x offset row * 128 of the pool
// row) and query-head chunk hg % chunks (GP query heads of each of them).
struct Piece {
  int seq = 0, hg = 0, len = 0;
  int t0 = 0, t1 = 0;     // token range [t0, t1)
  int ntiles = 0;         // tiles in this piece
  int seg_tiles = 0;      // tiles in the whole segment
  int64_t seg_units = 0;  // first cost unit of the segment
  bool first = false;     // first piece of this CTA
};

// Walks this CTA's tile range segment by segment. Every role runs its own copy
// and sees the same pieces in the same order. Sequence lengths are loaded one
// sequence ahead, so moving to the next sequence does not wait on memory.
struct Walker {
  int64_t ucur, hi;  // first unit of the current segment; end of this CTA's units
  int seq, hg, off;
  bool started;
  int len_cur, len_nxt;  // clamped lengths of seq and seq + 1

  __device__ void advance_seq(const TcParams &tp) {
    const DecodeParams &p = tp.p;
    ++seq;
    hg = 0;
    off = 0;
    len_cur = len_nxt;
    len_nxt = seq + 1 < p.num_seqs ? seq_len_clamped(p, seq + 1) : 0;
  }

  __device__ bool next(const TcParams &tp, Piece &pc) {
    const DecodeParams &p = tp.p;
    if (seq >= p.num_seqs) return false;
    int nt = tiles_of(len_cur);
    while (nt == 0) {  // zero-length sequences own no tiles (and no units)
      advance_seq(tp);
      if (seq >= p.num_seqs) return false;
      nt = tiles_of(len_cur);
    }
    const int len = len_cur;
    // Tiles i of this segment whose last unit ucur + kSegUnits + (i+1)*kTileUnits - 1 < hi.
    const int64_t room = hi - ucur - kSegUnits;
    const int64_t fit = room < kTileUnits ? 0 : room / kTileUnits;
    const int lim = fit < nt ? (int)fit : nt;
    if (lim <= off) return false;
    const int take = lim - off;
    pc.seq = seq;
    pc.hg = hg;
    pc.len = len;
    pc.t0 = off * kTile;
    pc.t1 = min(len, (off + take) * kTile);
    pc.ntiles = take;
    pc.seg_tiles = nt;
    pc.seg_units = ucur;
    pc.first = !started;
    started = true;
    off += take;
    if (off == nt) {
      off = 0;
      ucur += kSegUnits + nt * kTileUnits;
      if (++hg == tp.head_groups) advance_seq(tp);
    }
    return true;
  }
};

// The decode append fused into the launch. The new K / V row of a sequence
// lands in the tile that holds position len - 1, the last tile of each of its
// segments. The MMA issuer that consumes that tile (warp 1 for K, warp 11 for
// V) patches the row into the shared-memory tile after its TMA load landed
// and before the MMA reads it (a CTA-scope proxy fence, as for the stale rows
// it zeroes), and stores it into the pool row for later steps (a plain global
// store: no load in this launch reads the pool through it, every consumer of
// the tile patches its own copy). Lane l owns elements [8l, 8l + 8) of the
// 128 * D2-element slice of the row (the H kv heads of tile row prow).
// append_fetch issues the global loads one piece ahead (the row, its block
// id, and the cos / sin chunks for K with RoPE), so the data sits in
// registers when the tile comes up. Query-head chunks of one tile row (wide
// groups) are separate segments that store the same bytes, which is harmless.
struct NewRow {
  uint4 x, c, s;  // row chunk; cos / sin chunks (K with RoPE)
  int32_t blk;    // pool block of position len - 1
};

template <typename T, int H, int D, int D2, bool RP>
__device__ __forceinline__ NewRow append_fetch(const TcParams &tp, const Piece &pc, int nch, bool is_k, int lane) {
  NewRow r;
  r.x = r.c = r.s = make_uint4(0u, 0u, 0u, 0u);
  r.blk = -1;
  if (tp.k_new == nullptr || pc.len <= 0 || pc.t1 != pc.len) return r;
  const DecodeParams &p = tp.p;
  const int prow = pc.hg / nch;
  const int e = lane * 8;                // element within the slice
  const int hl = e / D, d = e - hl * D;  // kv head within the tile row, dim
  const int kv = prow * H + hl;
  r.blk = __ldg(p.bt + (int64_t)pc.seq * p.bt_s + (pc.len - 1) / p.block_size);
  if (lane < 16 * D2 && kv < p.hkv) {
    const T *src = static_cast<const T *>(is_k ? tp.k_new : tp.v_new);
    const int64_t st = is_k ? tp.kn_st : tp.vn_st, sh = is_k ? tp.kn_sh : tp.vn_sh;
    r.x = ldg16(src + (int64_t)pc.seq * st + (int64_t)kv * sh + d);
    if (RP && is_k) {
      r.c = ldg16(static_cast<const T *>(tp.cos) + (int64_t)pc.seq * tp.cs_st + d);
      r.s = ldg16(static_cast<const T *>(tp.sin) + (int64_t)pc.seq * tp.cs_st + d);
    }
  }
  return r;
}

// The lane's chunk of the new row as stored: K rotated when RoPE is on (the
// partner half of each head is D / 16 lanes away; every lane shuffles).
template <typename T, int D, bool RP>
__device__ __forceinline__ uint4 append_chunk(const NewRow &r, bool is_k, int lane) {
  uint4 x = r.x;
  if (RP && is_k) {
    uint4 xp;
    xp.x = __shfl_xor_sync(0xffffffffu, x.x, D / 16);
    xp.y = __shfl_xor_sync(0xffffffffu, x.y, D / 16);
    xp.z = __shfl_xor_sync(0xffffffffu, x.z, D / 16);
    xp.w = __shfl_xor_sync(0xffffffffu, x.w, D / 16);
    // rotate_half: -x[d + D/2] on the first half, x[d - D/2] on the second
    x = rope8<T>(x, xp, r.c, r.s, (lane * 8) % D < D / 2);
  }
  return x;
}

// Patch the lane's chunk into sub-row `sub` of the tile staged at `stage`
// (SW128 halves of 128 token rows x 128 B) and, with sub 0, store the whole
// slice into the pool. The caller fences the shared stores against the async
// proxy before the MMA.
template <typename T, int H, int D, int D2>
__device__ __forceinline__ void append_patch(const TcParams &tp, const Piece &pc, int nch, uint32_t stage,
                                             int tile_t0, int sub, bool is_k, const NewRow &r, uint4 x,
                                             int lane) {
  const DecodeParams &p = tp.p;
  const int prow = pc.hg / nch;
  const int e = lane * 8;
  const int kv = prow * H + e / D;
  if (lane >= 16 * D2 || kv >= p.hkv || r.blk < 0 || r.blk >= p.num_blocks) return;
  const int pos = pc.len - 1;
  const int es = e - sub * 128;
  if (es >= 0 && es < 128) {
    const int tr = pos - tile_t0;  // token row within the tile
    const int c = (es & 63) >> 3;
    const uint32_t addr = stage + (es >> 6) * kHalfBytes + tr * 128 + ((c ^ (tr & 7)) << 4);
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w)
                 : "memory");
  }
  if (sub == 0) {
    T *pool = static_cast<T *>(const_cast<void *>(is_k ? p.k : p.v));
    const int64_t row = (int64_t)r.blk * p.block_size + pos % p.block_size;
    stg16(pool + row * ((int64_t)p.hkv * D) + (int64_t)prow * 128 * D2 + e, x);
  }
}

// Chunk c of lane `lane` of the Q operand of piece q (the block-diagonal B
// operand [N rows x 128 * D2], K-major SW128; padding rows and halves stay
// zero): whether it holds query data, its head dimension d, its shared-memory
// address in the slot at qbuf and its source in q. A lane owns chunks
// idx = lane + 32 c (16 bytes each); its chunk column within 8 is lane & 7.
template <typename T, int H, int GP, int N, int D>
__device__ __forceinline__ void q_chunk(const DecodeParams &p, const Piece &q, int nch, uint32_t qbuf, int lane,
                                        int c, bool &in, int &d, uint32_t &addr, const T *&src) {
  constexpr int kQSubBytes = 2 * N * 128;  // one 128-element sub-row operand
  const int qrow = q.hg / nch;
  const int idx = lane + c * 32;
  const int sub = idx / (16 * N);  // 128-element sub-row of the head
  const int ix = idx - sub * 16 * N;
  const int xh = ix / (8 * N);
  const int rem = ix - xh * 8 * N;
  const int n = rem >> 3, ch = rem & 7;
  const int hl = n / GP, g = n - hl * GP;
  const int kv = qrow * H + hl;
  const int gq = (q.hg - qrow * nch) * GP + g;  // query head within the kv head's group
  // Element e of the 128-wide row belongs to kv head e / D of the group:
  // query column n (head hl) is nonzero only on its own head's D elements.
  const int e = sub * 128 + xh * 64 + ch * 8;
  in = hl < H && gq < p.group && kv < p.hkv && e / D == hl;
  d = e - hl * D;
  src = reinterpret_cast<const T *>(p.q) + (in ? (int64_t)q.seq * p.q_ss + (int64_t)(kv * p.group + gq) * p.q_sh + d : 0);
  addr = qbuf + sub * kQSubBytes + xh * (N * 128) + (n >> 3) * 1024 + (n & 7) * 128 + ((ch ^ (n & 7)) << 4);
}

// Q of piece q into the Q ring slot at qbuf by cp.async (16-byte chunks;
// padding chunks are zero-filled).
template <typename T, int H, int GP, int N, int D, int D2>
__device__ __forceinline__ void stage_q(const TcParams &tp, const Piece &q, int nch, uint32_t qbuf, int lane) {
  constexpr int kQChunks = 16 * N * D2 / 32;  // Q 16-byte chunks per lane
#pragma unroll
  for (int c = 0; c < kQChunks; ++c) {
    bool in;
    int d;
    uint32_t addr;
    const T *src;
    q_chunk<T, H, GP, N, D>(tp.p, q, nch, qbuf, lane, c, in, d, addr, src);
    cp_async_16(addr, src, in ? 16u : 0u);
  }
}

// RoPE of a piece's Q (q * cos + rotate_half(q) * sin, rounded as the append
// kernels round it), done by the K producer on the landed operand in shared
// memory. stage_cs copies the cos and sin rows of the piece's position beside
// its Q slot (cp.async, completing on the same q_full barrier); rotate_q
// rotates every chunk of the lane in place. A chunk's rotation partner, D / 2
// elements away in the same head, is a shuffle of the same chunk (lane ^ D /
// 16, head_dim <= 64: every lane reads its chunk before any lane writes) or
// another of the lane's own chunks (c ^ kp: N / 4 chunks away at head_dim 128,
// N / 2 at 256, read and written together).
template <typename T, int D, int D2>
__device__ __forceinline__ void stage_cs(const TcParams &tp, const Piece &q, uint32_t csbuf, int lane) {
  constexpr int kChunks = D / 8;  // 16-byte chunks of one row
#pragma unroll
  for (int k = lane; k < 2 * kChunks; k += 32) {
    const bool is_sin = k >= kChunks;
    const int ch = is_sin ? k - kChunks : k;
    const T *src = static_cast<const T *>(is_sin ? tp.sin : tp.cos) + (int64_t)q.seq * tp.cs_st + ch * 8;
    cp_async_16(csbuf + (is_sin ? 128u * D2 * 2u : 0u) + ch * 16, src, 16u);
  }
}

template <typename T, int H, int GP, int N, int D, int D2>
__device__ __forceinline__ void rotate_q(const DecodeParams &p, const Piece &q, int nch, uint32_t qbuf,
                                         uint32_t csbuf, int lane) {
  constexpr int kQChunks = 16 * N * D2 / 32;  // Q 16-byte chunks per lane
  constexpr int kp = kQChunks / 2;            // partner distance in chunks at head_dim >= 128
  constexpr int kG = D <= 64 ? 1 : 2;         // chunks rotated together: a chunk and its partner
  constexpr uint32_t kSinOff = 128u * D2 * 2u;
#pragma unroll
  for (int g = 0; g < kQChunks / kG; ++g) {
    // Chunk g (and its partner g + kp) holds query columns 4 g mod N to
    // 4 g mod N + 3 in every lane: when those are padding columns (past the
    // H x GP real ones, zero-filled when staged), there is nothing to rotate.
    if ((4 * g) % N >= H * GP) continue;
    uint4 xs[kG];
    bool in[kG];
    int dd[kG];
    uint32_t addr[kG];
#pragma unroll
    for (int k = 0; k < kG; ++k) {
      const T *src;
      q_chunk<T, H, GP, N, D>(p, q, nch, qbuf, lane, g + k * kp, in[k], dd[k], addr[k], src);
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(xs[k].x), "=r"(xs[k].y), "=r"(xs[k].z), "=r"(xs[k].w)
                   : "r"(addr[k])
                   : "memory");
    }
#pragma unroll
    for (int k = 0; k < kG; ++k) {
      uint4 xp;
      if constexpr (D <= 64) {
        xp.x = __shfl_xor_sync(0xffffffffu, xs[k].x, D / 16);
        xp.y = __shfl_xor_sync(0xffffffffu, xs[k].y, D / 16);
        xp.z = __shfl_xor_sync(0xffffffffu, xs[k].z, D / 16);
        xp.w = __shfl_xor_sync(0xffffffffu, xs[k].w, D / 16);
      } else {
        xp = xs[k ^ 1];
      }
      if (in[k]) {
        uint4 c, sn;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(c.x), "=r"(c.y), "=r"(c.z), "=r"(c.w)
                     : "r"(csbuf + dd[k] * 2)
                     : "memory");
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(sn.x), "=r"(sn.y), "=r"(sn.z), "=r"(sn.w)
                     : "r"(csbuf + kSinOff + dd[k] * 2)
                     : "memory");
        const uint4 r = rope8<T>(xs[k], xp, c, sn, dd[k] < D / 2);
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr[k]), "r"(r.x), "r"(r.y), "r"(r.z),
                     "r"(r.w)
                     : "memory");
      }
    }
  }
}

// Running (sum, denominator, reference max) of one correction thread's
// query columns.
template <int GP, int D2>
struct PieceAcc {
  float acc[D2][GP], lsum[GP], msel[GP];
};

// Stream-K combine, run by the 128 correction threads of the CTA holding a
// cut segment's first tile (range index vb): wait for the partials the CTAs of
// ranges vb+1..b1 published, fold them into this CTA's piece, store the
// normalised output and clear the flags (at most once per CTA per launch).
// Ranges are assigned in reverse block order (range vb runs in block
// G - 1 - vb), so the CTAs waited on have LOWER block indices than the
// waiting one: under in-order block dispatch they were resident first, and
// each publishes its piece before it waits on anything, so the wait ends
// even when other work holds part of the GPU and not every CTA of the grid
// is resident at once.
template <typename T, int GP, int D, int D2>
__device__ __forceinline__ void combine_pieces(const TcParams &tp, PieceAcc<GP, D2> a, int64_t vb, int64_t b1,
                                               int64_t G, int hl, int dim, int gn, bool have_kv, T *out,
                                               volatile int *abort_flag, int row) {
  using E = Elem<T>;
  const DecodeParams &p = tp.p;
  const int HQS = (128 * D2 / D) * GP;  // partial slots per CTA
  // The partners lie inside the effective grid by construction (every role
  // derives its pieces from the same lengths); a range past it would index
  // flags and partials the workspace does not hold, so it is refused.
  if (b1 >= G) {
    if (row == 0) set_error(p.err, PAGEDKV_EFLAG_SEQ_LEN_RANGE);
    b1 = G - 1;
  }
  if (row == 0) {
    for (int64_t bb = vb + 1; bb <= b1; ++bb) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_u32(tp.flags + bb) == 0u) {
        if (globaltimer_ns() - t0 > kTimeoutNs) {
          *abort_flag = 1;
          break;
        }
      }
    }
  }
  named_bar(2, 128);
  if (have_kv) {
    for (int64_t bb = vb + 1; bb <= b1; ++bb) {
      const int64_t hh0 = bb * HQS + hl * GP;
      for (int g = 0; g < GP; ++g) {
        if (g < gn) {
          const float2 ml = __ldcg(&tp.part_ml[hh0 + g]);
          const float mb = fmaxf(a.msel[g], ml.x);
          const float sc = a.msel[g] == kNegInf ? 0.f : fast_exp2(a.msel[g] - mb);
          const float f = ml.x == kNegInf ? 0.f : fast_exp2(ml.x - mb);
          a.lsum[g] = fmaf(f, ml.y, a.lsum[g] * sc);
#pragma unroll
          for (int sub = 0; sub < D2; ++sub) {
            const float av = __ldcg(&tp.part_acc[(hh0 + g) * D + sub * 128 + dim]);
            a.acc[sub][g] = fmaf(f, av, a.acc[sub][g] * sc);
          }
          a.msel[g] = mb;
        }
      }
    }
    for (int g = 0; g < GP; ++g)
      if (g < gn) {
#pragma unroll
        for (int sub = 0; sub < D2; ++sub)
          out[(int64_t)g * p.o_sh + sub * 128] =
              E::from_float(a.lsum[g] > 0.f ? __fdividef(a.acc[sub][g], a.lsum[g]) : 0.f);
      }
  }
  named_bar(2, 128);  // every partner partial read before its flag is cleared
  if (row == 0) {
    for (int64_t bb = vb + 1; bb <= b1; ++bb) st_volatile_u32(tp.flags + bb, 0u);
  }
}

struct MiscSmem {
#ifdef PAGEDKV_TRACE
  unsigned long long tl_ticket;
#endif
  uint32_t tmem;
  int abort;
  int len0, len1;  // clamped lengths of seq0 and seq0 + 1
  int seq0, hg0, off0, vcta;  // vcta: this CTA's range index
  long long lo, hi, total, grid, u0;
};

template <int N, int SK, int SV, int D2 = 1, bool RP = false>
struct SmemLayout {
  static constexpr int kQSubBytes = 2 * N * 128;     // B operand [N x 128], two K-halves
  static constexpr int kQBytes = D2 * kQSubBytes;    // one per 128-element sub-row of a head
  static constexpr int kPBytes = N * 256;      // B operand P^T, MN-major SW32: N/16 atoms x 4 KB
  static constexpr int kSlotBytes = 8 * N + 16;  // per-tile rescale record, see RescaleSlot
  static constexpr int kOffK = 0;                               // K ring: SK tiles
  static constexpr int kOffV = kOffK + SK * kOperandBytes;      // V ring: SV tiles
  static constexpr int kOffQ = kOffV + SV * kOperandBytes;      // Q ring: kQSlots operands
  static constexpr int kOffP = kOffQ + kQSlots * kQBytes;
  static constexpr int kOffRedMax = kOffP + 2 * kPBytes;        // float [2][4][N]; prologue scratch
  static constexpr int kOffSlots = kOffRedMax + 2 * 4 * N * 4;  // kRescaleSlots records
  static constexpr int kOffL = kOffSlots + kRescaleSlots * kSlotBytes;  // float [kLSlots][4][N]
  static constexpr int kOffBtWin = kOffL + kLSlots * 4 * N * 4;  // int32 [2 producers][3][32]
  static constexpr int kOffBars = kOffBtWin + 2 * 3 * 32 * 4;        // uint64 barriers
  // kfull, kempty [SK]; vfull, vempty [SV]; s_full, s_empty, p_full, p_empty,
  // o_full, o_empty [2]; mma_done [1]; a_full [kRescaleSlots]; q_full, q_empty
  // [kQSlots]; l_full [kLSlots]
  static constexpr int kNumBars = 2 * SK + 2 * SV + 6 * 2 + 1 + kRescaleSlots + 2 * kQSlots + kLSlots + kQSlots;
  static constexpr int kOffMisc = kOffBars + kNumBars * 8;  // see MiscSmem
  // RoPE only: the cos and sin rows of each Q slot's position (stage_cs)
  static constexpr int kCSBytes = 2 * 128 * D2 * 2;
  static constexpr int kOffCS = (kOffMisc + (int)sizeof(MiscSmem) + 15) / 16 * 16;
  static constexpr int kBytes = RP ? kOffCS + kQSlots * kCSBytes : kOffMisc + (int)sizeof(MiscSmem);
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
  static_assert(2 * 4 * N * 4 >= 8 * (kThreads / 32), "prologue scan scratch fits the max-reduction buffer");
  static_assert(kOffSlots % 16 == 0 && kSlotBytes % 16 == 0 && kOffL % 16 == 0 && kOffBars % 8 == 0, "alignment");
};

// Per-tile record the softmax warps hand to the correction warps: whether the
// tile moved the reference max, and if so the factors and the new max.
template <int N>
struct RescaleSlot {
  float alpha[N];  // exp2(old max - new max) per query column
  float m[N];      // new reference max (log2 units) per query column
  uint32_t resc;
  uint32_t pad[3];
};


// CH: the group is wider than GP and runs in tp.chunks query-head chunks (a
// separate instantiation, so the single-chunk kernels carry none of it).
// D2: 128-element sub-rows per head (2 for head_dim 256: every tile is two K
// and two V ring stages, S sums both, O has one accumulator per sub-row).
// RP: RoPE fused (tp.cos / tp.sin given), a separate instantiation as well.
template <typename T, int H, int GP, int N, int SK, int SV, bool CH, int D2, bool RP>
__global__ void __launch_bounds__(kThreads, 1)
decode_tc_kernel(const __grid_constant__ CUtensorMap tmap_k,
                 const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ TcParams tp) {
  using L = SmemLayout<N, SK, SV, D2, RP>;
  using E = Elem<T>;
  using Slot = RescaleSlot<N>;
  constexpr int D = 128 * D2 / H;                     // head_dim
  // TMEM: S[2] then O[2][D2], N columns each, rounded up to a power of two
  constexpr uint32_t kColsUsed = (2 + 2 * D2) * N;
  constexpr uint32_t kCols = kColsUsed <= 64 ? 64 : kColsUsed <= 128 ? 128 : 256;
  static_assert(D2 == 1 || H == 1, "a head wider than a tile row has the tile row to itself");
  constexpr uint32_t kFmt = E::kDtype == PAGEDKV_DTYPE_BF16 ? 1u : 0u;
  constexpr uint32_t kIdescS = idesc_f16(kFmt, N, false, false);
  constexpr uint32_t kIdescO = idesc_f16(kFmt, N, true, true);
  static_assert(H * GP <= N && N % 16 == 0 && N <= 32, "column layout");
  static_assert(sizeof(Slot) == L::kSlotBytes, "slot size");

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::kOffBars;
  // K and V have separate rings: a K tile is released as soon as the S MMA
  // has read it, a V tile only after the O MMA, so K prefetch runs deeper.
  auto kfull = [&](int s) { return bars + 8u * s; };
  auto kempty = [&](int s) { return bars + 8u * (SK + s); };
  auto vfull = [&](int s) { return bars + 8u * (2 * SK + s); };
  auto vempty = [&](int s) { return bars + 8u * (2 * SK + SV + s); };
  auto bar2 = [&](int which, int b) { return bars + 8u * (2 * SK + 2 * SV + 2 * which + b); };
  // which: 0 s_full, 1 s_empty, 2 p_full, 3 p_empty, 4 o_full, 5 o_empty
  constexpr int kBarTail = 2 * SK + 2 * SV + 12;
  const uint32_t mma_done = bars + 8u * kBarTail;
  auto a_full = [&](int s) { return bars + 8u * (kBarTail + 1 + s); };
  auto q_full = [&](uint32_t i) { return bars + 8u * (kBarTail + 1 + kRescaleSlots + i % kQSlots); };
  auto q_empty = [&](uint32_t i) { return bars + 8u * (kBarTail + 1 + kRescaleSlots + kQSlots + i % kQSlots); };
  auto l_full = [&](uint32_t i) { return bars + 8u * (kBarTail + 1 + kRescaleSlots + 2 * kQSlots + i % kLSlots); };
  // q_rot: with RoPE, the Q of slot i % kQSlots has been rotated in place
  auto q_rot = [&](uint32_t i) {
    return bars + 8u * (kBarTail + 1 + kRescaleSlots + 2 * kQSlots + kLSlots + i % kQSlots);
  };
  // Phase parity of the (i / ring)-th use of ring slot i % ring.
  auto ring_parity = [](uint32_t i, uint32_t ring) { return (i / ring) & 1u; };
  MiscSmem *misc = reinterpret_cast<MiscSmem *>(smem + L::kOffMisc);
  volatile int *abort_flag = &misc->abort;
  float *red_max = reinterpret_cast<float *>(smem + L::kOffRedMax);
  Slot *slots = reinterpret_cast<Slot *>(smem + L::kOffSlots);
  float *lpart = reinterpret_cast<float *>(smem + L::kOffL);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const DecodeParams &p = tp.p;
  const int nch = CH ? tp.chunks : 1;  // query-head chunks per tile row
#ifdef PAGEDKV_TRACE
  uint64_t tw[kTraceSlots] = {};
  const uint64_t t_kernel0 = globaltimer_ns();
  const uint64_t c_kernel0 = clock64();
#endif

#ifdef PAGEDKV_TRACE
  if (threadIdx.x == 0) {
    const unsigned long long tk = atomicAdd(&g_tl_ctr, 1ull);
    misc->tl_ticket = tk;
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    g_tl[tk % kTraceRecs][0] = tk;
    g_tl[tk % kTraceRecs][1] = smid;
    g_tl[tk % kTraceRecs][2] = t_kernel0;
  }
#endif
  if (threadIdx.x == 0) {
    for (int s = 0; s < SK; ++s) {
      mbar_init(kfull(s), 1);   // producer arrive.expect_tx + TMA bytes
      mbar_init(kempty(s), 1);  // MMA commit after S
    }
    for (int s = 0; s < SV; ++s) {
      mbar_init(vfull(s), 1);
      mbar_init(vempty(s), 1);  // MMA commit after O
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar2(0, b), 1);    // s_full: MMA commit
      mbar_init(bar2(1, b), 128);  // s_empty: every softmax thread
      mbar_init(bar2(2, b), 128);  // p_full: every softmax thread
      mbar_init(bar2(3, b), 1);    // p_empty: MMA commit
      mbar_init(bar2(4, b), 1);    // o_full: MMA commit
      mbar_init(bar2(5, b), 128);  // o_empty: every correction thread
    }
    mbar_init(mma_done, 2);  // one commit from each MMA issuer
    for (int s = 0; s < kRescaleSlots; ++s) mbar_init(a_full(s), 1);  // one softmax thread
    for (int s = 0; s < kQSlots; ++s) {
      mbar_init(q_full(s), 32);  // every lane of the staging warp, when its Q copies land
      mbar_init(q_empty(s), 1);  // MMA commit after the piece's last S
    }
    for (int s = 0; s < kLSlots; ++s) mbar_init(l_full(s), 4);  // lane 0 of each softmax warp
    if (RP)
      for (int s = 0; s < kQSlots; ++s) mbar_init(q_rot(s), 32);  // every lane of the rotating warp
    misc->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&misc->tmem), kCols);
    tmem_relinquish();
  }

  // The launch's small inputs are pulled into L2 while the preceding kernel
  // finishes, spread over the CTAs: the sequence lengths (every CTA scans
  // them), the block tables (the first tiles' ids are read right after the
  // scan) and q. A prefetch reads nothing into the SM, and every write of the
  // preceding kernel has reached L2 before the wait below returns, so no
  // value read after it can be stale. Each range ends at its last valid
  // element, so every line prefetched holds some of the buffer.
  {
    const int64_t nthr = (int64_t)gridDim.x * kThreads;
    const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    auto lines = [](const void *base, int64_t bytes) -> int64_t {
      const uint64_t a0 = reinterpret_cast<uint64_t>(base);
      return bytes > 0 ? (int64_t)(((a0 + bytes - 1) >> 7) - (a0 >> 7) + 1) : 0;
    };
    auto line_addr = [](const void *base, int64_t i) {
      return reinterpret_cast<const void *>(((reinterpret_cast<uint64_t>(base) >> 7) + i) << 7);
    };
    const int64_t ns = p.num_seqs;
    const int64_t l_lens = p.lens ? lines(p.lens, ns * 4) : 0;
    const int64_t bt_bytes = ns > 0 ? ((ns - 1) * p.bt_s + p.max_blocks) * 4 : 0;
    const int64_t l_bt = lines(p.bt, bt_bytes);
    const int64_t q_bytes = ns > 0 ? ((ns - 1) * p.q_ss + (int64_t)(p.hq - 1) * p.q_sh + D) * (int64_t)sizeof(T) : 0;
    const int64_t l_q = lines(p.q, q_bytes);
    if (l_lens + l_bt + l_q <= (int64_t)1 << 16) {  // at most 8 MB
      for (int64_t i = t; i < l_lens + l_bt + l_q; i += nthr) {
        if (i < l_lens)
          prefetch_l2(line_addr(p.lens, i));
        else if (i < l_lens + l_bt)
          prefetch_l2(line_addr(p.bt, i - l_lens));
        else
          prefetch_l2(line_addr(p.q, i - l_lens - l_bt));
      }
    }
  }

  // Everything above touched only shared memory and TMEM (and issued L2
  // prefetches), so it overlaps the tail of the preceding kernel; global
  // inputs are read only after it ends.
  grid_dependency_wait();
  grid_launch_dependents();
#ifdef PAGEDKV_TRACE
  if (threadIdx.x == 0) {
    g_tl[misc->tl_ticket % kTraceRecs][3] = globaltimer_ns();
    PKV_TL(20);
  }
#endif

  // ---- prologue: total cost units and the start of this CTA's range ----------
  {
    long long *scan = reinterpret_cast<long long *>(smem + L::kOffRedMax);  // [warps] sums
    const int ns = p.num_seqs;
    const int per = (ns + kThreads - 1) / kThreads;
    const int s_begin = min(ns, (int)threadIdx.x * per);
    const int s_end = min(ns, s_begin + per);
    const long long HG = tp.head_groups;
    long long local = 0;  // units of this thread's sequences
    for (int s = s_begin; s < s_end; ++s) {
      const int nt = tiles_of(seq_len_clamped(p, s));
      if (nt > 0) local += HG * (kSegUnits + nt * kTileUnits);
    }
    long long incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) scan[warp] = incl;
    __syncthreads();
    long long warp_off = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
      const long long v = scan[w];
      warp_off += w < warp ? v : 0;
      total += v;
    }
    const long long excl = warp_off + incl - local;  // units of sequences before s_begin
    const long long Ut = total;
    // Effective grid: every CTA's unit range is at least one tile plus one
    // segment wide, so it holds the last unit of some tile (consecutive tiles'
    // last units are at most that far apart): every participating CTA owns a
    // tile, and the owners of a segment are consecutive.
    const long long wide = Ut / (kSegUnits + kTileUnits);
    const long long Ge = wide < (long long)gridDim.x ? wide : (long long)gridDim.x;
    // Range vb runs in block Ge - 1 - vb: a range's stream-K partners (the
    // ranges after it) run in lower-numbered blocks (see combine_pieces).
    const long long vb = (long long)blockIdx.x < Ge ? Ge - 1 - (long long)blockIdx.x : (long long)blockIdx.x;
    const long long lo = vb < Ge ? range_lo(vb, Ut, Ge) : Ut;
    const long long hi = vb < Ge ? range_lo(vb + 1, Ut, Ge) : Ut;
    if (threadIdx.x == 0) {
      misc->vcta = (int)vb;
      misc->lo = lo;
      misc->hi = hi;
      misc->total = Ut;
      misc->grid = Ge;
      misc->u0 = Ut;
      misc->seq0 = ns;  // empty range unless a thread below claims lo
      misc->hg0 = 0;
      misc->off0 = 0;
      misc->len0 = 0;
      misc->len1 = 0;
    }
    __syncthreads();
    if (lo < Ut && excl <= lo && lo < excl + local) {
      // This thread's sequences hold unit lo: the CTA's first tile is the
      // first one whose last unit is >= lo.
      long long acc_u = excl;
      for (int s = s_begin; s < s_end; ++s) {
        const int len = seq_len_clamped(p, s);
        const int nt = tiles_of(len);
        if (nt == 0) continue;
        const long long seg_u = kSegUnits + nt * kTileUnits;
        if (lo < acc_u + HG * seg_u) {
          const long long hg = (lo - acc_u) / seg_u;
          const long long uk = acc_u + hg * seg_u;
          const long long rel = lo - uk - kSegUnits;
          misc->seq0 = s;
          misc->hg0 = (int)hg;
          misc->off0 = rel < 0 ? 0 : (int)(rel / kTileUnits);
          misc->u0 = uk;
          // Every role's walker starts from these, without a load of its own.
          misc->len0 = len;
          misc->len1 = s + 1 < ns ? seq_len_clamped(p, s + 1) : 0;
          break;
        }
        acc_u += HG * seg_u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) PKV_TL(6);
  const uint32_t tmem = misc->tmem;
  const int64_t U_total = misc->total;
  const int64_t G = misc->grid;
  const int64_t vcta = misc->vcta;
  Walker walk{misc->u0, misc->hi, misc->seq0, misc->hg0, misc->off0, false, misc->len0, misc->len1};

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------ producers: warp 0 K (+ Q), warp 6 V
    // The global loads a TMA issue depends on run ahead of it: block-table
    // entries are staged in windows of 32 consecutive blocks, two windows
    // ahead (also across piece boundaries), by cp.async into shared memory,
    // and the K producer copies the next piece's Q rows into the Q ring one
    // piece ahead (cp.async, completing on the slot's q_full barrier). A
    // stage freed by the consumer is refilled without a round trip to L2.
    const bool is_k = warp == 0;
    if (is_k && lane == 0) PKV_TL(11);
    const CUtensorMap *tmap = is_k ? &tmap_k : &tmap_v;
    const int nst = is_k ? SK : SV;
    const uint32_t ring = sbase + (is_k ? L::kOffK : L::kOffV);
    if (lane == 0) tma_prefetch_desc(tmap);
    // K/V rows are read once (evict first), or once per query-head chunk when
    // the group is split, where the next chunk's segment re-reads them from L2.
    const uint64_t policy = CH ? l2_policy_evict_normal() : l2_policy_evict_first();
    if (is_k && lane == 0) PKV_TL(14);
    const int bpt = kTile / p.block_size;  // blocks per tile: 1..16, divides 32
    constexpr int kQChunks = 16 * N * D2 / 32;  // Q 16-byte chunks per lane
    int stage = 0;
    uint32_t sphase = 0;
    uint32_t qi = 0;
    int issued = 0;
    bool ok = true;

    // Q of piece q into ring slot i as the block-diagonal B operand
    // [N rows x 128], K-major SW128; padding rows and halves are zero-filled.
    // Q of each piece goes into a Q ring slot one piece ahead by cp.async,
    // completing on the slot's q_full barrier. With RoPE the cos / sin rows
    // come along (same barrier), and the V producer rotates the landed Q in
    // place at the top of the piece before; q_rot then hands it to the S
    // issuer. (The CTA's first piece's Q is staged and rotated by correction
    // warp 7.)
    auto q_issue = [&](const Piece &q, uint32_t i) -> bool {
      if (!PKV_TW(0, mbar_wait(q_empty(i), ring_parity(i, kQSlots) ^ 1u, abort_flag, kTimeoutNs))) return false;
      stage_q<T, H, GP, N, D, D2>(tp, q, nch, sbase + L::kOffQ + (i % kQSlots) * L::kQBytes, lane);
      if constexpr (RP) stage_cs<T, D, D2>(tp, q, sbase + L::kOffCS + (i % kQSlots) * L::kCSBytes, lane);
      cp_async_mbar_arrive(q_full(i));
      return true;
    };
    auto q_rotate = [&](const Piece &q, uint32_t i) -> bool {
      // every lane takes part in the rotation's shuffles, or none does
      const bool landed = mbar_wait(q_full(i), ring_parity(i, kQSlots), abort_flag, kTimeoutNs);
      if (!__all_sync(0xffffffffu, landed)) return false;
      rotate_q<T, H, GP, N, D, D2>(p, q, nch, sbase + L::kOffQ + (i % kQSlots) * L::kQBytes,
                                   sbase + L::kOffCS + (i % kQSlots) * L::kCSBytes, lane);
      fence_proxy_async_smem();  // the MMA reads the rotated operand through the async proxy
      mbar_arrive(q_rot(i));
      return true;
    };


    // First ring fill of the CTA's first piece, issued straight from the range
    // prologue's results (its sequence, head group, first tile, length and the
    // range end) with every lane computing its own loads: no walker step and
    // no block-table window stand between the dependency release and the first
    // tiles in flight (the piece's Q is staged by correction warp 7). The loop
    // below starts the first piece at tile `pre`.
    int pre = 0;
    {
      const int s0 = misc->seq0, len0 = misc->len0, off0 = misc->off0, hg0 = misc->hg0;
      int lim = 0;  // the first piece is tiles [off0, lim) of its segment
      if (s0 < p.num_seqs) {
        // the first step of Walker::next from the range start
        const int64_t room = misc->hi - misc->u0 - kSegUnits;
        const int64_t fit = room < kTileUnits ? 0 : room / kTileUnits;
        const int nt0 = tiles_of(len0);
        lim = fit < nt0 ? (int)fit : nt0;
        pre = min(lim - off0, nst / D2);
        if (pre < 0) pre = 0;
      }
      if (is_k && lane == 0) PKV_TL(17);
      if (pre > 0) {
        const int t1 = min(len0, lim * kTile);  // the piece's token end, as Walker::next sets it
        const int need = (t1 + p.block_size - 1) / p.block_size;
        const int lb0 = off0 * bpt;  // the piece's first logical block
        // block ids of the pre-issued tiles: entry e = j * bpt + b (< 48) is
        // loaded by lane e % 32 into blk[e / 32]
        int32_t blk[2] = {-1, -1};
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          const int e = lane + 32 * k2;
          if (e < pre * bpt && lb0 + e < need) blk[k2] = __ldg(p.bt + (int64_t)s0 * p.bt_s + lb0 + e);
        }
        const int x0 = hg0 / nch * 128 * D2;  // this tile row's first element
        for (int st = 0; st < pre * D2; ++st) {  // first use of each stage: nothing to wait for
          const int j = st / D2, sub = st - j * D2;
          const uint32_t full = is_k ? kfull(st) : vfull(st);
          if (lane == 0) mbar_arrive_expect_tx(full, kOperandBytes);
          __syncwarp();
          const int h = lane >= bpt ? 1 : 0;
          const int b = lane - h * bpt;
          const int e = j * bpt + (lane < 2 * bpt ? b : 0);
          const int32_t v0 = __shfl_sync(0xffffffffu, blk[0], e & 31);
          const int32_t v1 = __shfl_sync(0xffffffffu, blk[1], e & 31);
          if (is_k && st == 0 && lane == 0 && (v0 | v1) != 0x7fffffff) PKV_TL(18);
          if (lane < 2 * bpt) {
            const int32_t id = e < 32 ? v0 : v1;
            int32_t y = tp.oob_row;  // out of range: TMA fills zeros, reads nothing
            if (lb0 + e < need) {
              if (id >= 0 && id < p.num_blocks) {
                y = id * p.block_size;
              } else if (is_k && h == 0 && sub == 0) {
                set_error(p.err, PAGEDKV_EFLAG_BLOCK_ID_RANGE);
              }
            }
            const uint32_t dst = ring + st * kOperandBytes + h * kHalfBytes + b * p.block_size * 128;
            tma_load_2d(dst, tmap, x0 + sub * 128 + h * 64, y, full, policy);
          }
          if (is_k && st == 0 && lane == 0) PKV_TL(19);
        }
        if (is_k && lane == 0) PKV_TL(8);
        issued = pre * D2;
        stage = issued;
        if (stage == nst) {
          stage = 0;
          sphase ^= 1u;
        }
      }
    }

    // Window k (k = 0, 1, ... over this CTA's pieces in order; window w of a
    // piece q covers its logical blocks q.t0 / block_size + 32 w + [0, 32))
    // lands in slot k % 3; lanes past the piece's last block copy nothing.
    const uint32_t win_base = sbase + L::kOffBtWin + (is_k ? 0u : 3u * 32u * 4u);
    const int32_t *win = reinterpret_cast<const int32_t *>(smem + L::kOffBtWin) + (is_k ? 0 : 3 * 32);
    Walker gwalk = walk;  // generator of the window sequence
    Piece gp;
    bool gvalid = gwalk.next(tp, gp);
    if (is_k && lane == 0) PKV_TL(15);
    int gw = 0;
    uint32_t gk = 0;  // windows issued
    auto issue_window = [&]() {
      if (gvalid) {
        const int lb = gp.t0 / p.block_size + 32 * gw + lane;
        const int need = (gp.t1 + p.block_size - 1) / p.block_size;
        const bool in = lb < need;
        const int32_t *src = in ? p.bt + (int64_t)gp.seq * p.bt_s + lb : p.bt;
        cp_async_4(win_base + ((gk % 3u) * 32u + lane) * 4u, src, in ? 4u : 0u);
        if (++gw == (gp.ntiles * bpt + 31) / 32) {
          gw = 0;
          gvalid = gwalk.next(tp, gp);
        }
      }
      cp_async_commit();  // possibly empty: one group per window slot, always
      ++gk;
    };
    issue_window();
    if (is_k && lane == 0) PKV_TL(16);
    issue_window();
    if (is_k && lane == 0) PKV_TL(12);
    uint32_t wk = 0;  // windows consumed

    Piece pc;
    bool have = walk.next(tp, pc);
    qi = 1;           // the first piece's Q (slot 0) is correction warp 7's
    if (is_k && lane == 0) PKV_TL(13);
    bool first_piece = true;
    uint32_t vq = 1;  // Q slot of the next piece (V producer, RoPE)
    while (ok && have) {
      PKV_STAMP(t_top0);
      Piece nx;
      const bool have_nx = walk.next(tp, nx);
      // The next piece's Q, landing while this piece's tiles stream.
      if (is_k && have_nx && !q_issue(nx, qi++)) break;
      PKV_TADD(4, clock64() - t_top0);
      // tiles of this piece issued by the first ring fill above
      const int skip = first_piece ? pre : 0;
      // RoPE: the V producer rotates the next piece's Q, which the K producer
      // staged one piece ahead, at the top of each piece: it runs about two
      // tiles ahead of the S issuer and is less loaded than the K producer,
      // whose TMA issue paces short pieces. (The first piece's Q is staged and
      // rotated by correction warp 7.)
      if constexpr (RP) {
        if (!is_k && have_nx && !q_rotate(nx, vq)) break;
      }
      ++vq;
      first_piece = false;
      const int lb0 = pc.t0 / p.block_size;
      const int need = (pc.t1 + p.block_size - 1) / p.block_size;
      const int x0 = pc.hg / nch * 128 * D2;  // this tile row's first element
      for (int j = 0; j < pc.ntiles; ++j) {
        const int wofs = (j * bpt) & 31;
        if (wofs == 0) {
          // Entering a window: stage the one two ahead (into the slot of the
          // window just finished), then wait for this one.
          PKV_STAMP(t_win0);
          __syncwarp();
          issue_window();
          cp_async_wait<2>();
          __syncwarp();
          PKV_TADD(2, clock64() - t_win0);
          if (is_k && issued == 0 && lane == 0) PKV_TL(7);
        }
        const uint32_t slot = wk % 3u;
        if (wofs + bpt >= 32 || j + 1 == pc.ntiles) ++wk;  // last tile of this window
        for (int sub = 0; sub < D2 && j >= skip; ++sub) {  // one ring stage per 128-element sub-row
          if (!PKV_TW(1, mbar_wait(is_k ? kempty(stage) : vempty(stage), sphase ^ 1u, abort_flag, kTimeoutNs))) {
            ok = false;
            break;
          }
          PKV_STAMP(t_iss0);
          const uint32_t full = is_k ? kfull(stage) : vfull(stage);
          if (lane == 0) mbar_arrive_expect_tx(full, kOperandBytes);
          __syncwarp();
          if (lane < 2 * bpt) {
            // lane -> (block b of the tile, 64-element half h)
            const int h = lane >= bpt ? 1 : 0;
            const int b = lane - h * bpt;
            const int lb = lb0 + j * bpt + b;
            int32_t y = tp.oob_row;  // out of range: TMA fills zeros, reads nothing
            if (lb < need) {
              const int32_t blk = win[slot * 32 + wofs + b];
              if (blk >= 0 && blk < p.num_blocks) {
                y = blk * p.block_size;
              } else if (is_k && h == 0 && sub == 0) {
                set_error(p.err, PAGEDKV_EFLAG_BLOCK_ID_RANGE);
              }
            }
            const uint32_t dst = ring + stage * kOperandBytes + h * kHalfBytes + b * p.block_size * 128;
            tma_load_2d(dst, tmap, x0 + sub * 128 + h * 64, y, full, policy);
          }
          PKV_TADD(3, clock64() - t_iss0);
          if (is_k && issued == 0 && lane == 0) PKV_TL(8);
          ++issued;
          if (++stage == nst) {
            stage = 0;
            sphase ^= 1u;
          }
        }
        if (!ok) break;
      }
      pc = nx;
      have = have_nx;
    }
    cp_async_wait<0>();  // no copy into shared memory outlives this role
    // Drain: the last min(issued, ring size) tiles' loads must have landed
    // before this CTA's shared memory is released (immediate on the normal path).
    for (int k = 0; k < nst && k < issued; ++k) {
      if (--stage < 0) {
        stage = nst - 1;
        sphase ^= 1u;
      }
      volatile int never = 0;
      mbar_wait(is_k ? kfull(stage) : vfull(stage), sphase, &never, kTimeoutNs / 4);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ S issuer
    // S^T = K Q^T per tile into the S double buffer, as far ahead as the
    // softmax warps' reads of S allow. (The S and O MMAs are issued by two
    // warps: each tcgen05.mma costs its issuing thread tens of nanoseconds.)
    int kst = 0;
    uint32_t kph = 0, gt = 0, qi = 0;
    bool ok = true;
    Piece pc;
    bool have = walk.next(tp, pc);
    // The new K row of the current piece's segment (fused append), loaded
    // one piece ahead.
    // (a CTA may own no piece at all: nothing is fetched then)
    NewRow row_cur = append_fetch<T, H, D, D2, RP>(tp, have ? pc : Piece{}, nch, true, lane);
    while (ok && have) {
      Piece nx;
      const bool have_nx = walk.next(tp, nx);
      const NewRow row_nxt = have_nx ? append_fetch<T, H, D, D2, RP>(tp, nx, nch, true, lane) : row_cur;
      // Q landed (cp.async), and with RoPE the K producer rotated it
      const uint32_t qbar = RP ? q_rot(qi) : q_full(qi);
      if (!PKV_TW(0, mbar_wait(qbar, ring_parity(qi, kQSlots), abort_flag, kTimeoutNs))) break;
      if (qi == 0 && lane == 0) PKV_TL(9);
      const uint32_t qbuf = sbase + L::kOffQ + (qi % kQSlots) * L::kQBytes;
      fence_proxy_async_smem();  // Q written through the generic proxy; the MMA reads it
      for (int j = 0; j < pc.ntiles; ++j) {
        const uint32_t b = gt & 1u;
        const bool patch = tp.k_new != nullptr && pc.t1 == pc.len && j + 1 == pc.ntiles;
        const uint4 xk = patch ? append_chunk<T, D, RP>(row_cur, true, lane) : row_cur.x;
        for (int sub = 0; sub < D2; ++sub) {  // S sums the sub-rows' products
          if (!PKV_TW(1, mbar_wait(kfull(kst), kph, abort_flag, kTimeoutNs))) { ok = false; break; }
          if (gt == 0 && sub == 0 && lane == 0) PKV_TL(10);
          if (sub == 0 && !PKV_TW(2, mbar_wait(bar2(1, b), ((gt >> 1) & 1u) ^ 1u, abort_flag, kTimeoutNs))) {
            ok = false;
            break;
          }
          if (patch) {
            // the new K row of position len - 1, into the landed tile and the pool
            append_patch<T, H, D, D2>(tp, pc, nch, sbase + L::kOffK + kst * kOperandBytes, pc.t0 + j * kTile, sub,
                                      true, row_cur, xk, lane);
            fence_proxy_async_smem();
            __syncwarp();
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t ka = sbase + L::kOffK + kst * kOperandBytes;
            const uint32_t qsub = qbuf + sub * L::kQSubBytes;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t ad = smem_desc_sw128(ka + (kk >> 2) * kHalfBytes + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = smem_desc_sw128(qsub + (kk >> 2) * (N * 128) + (kk & 3) * 32, 16, 1024);
              mma_f16_ss(tmem + b * N, ad, bd, kIdescS, (sub > 0 || kk > 0) ? 1u : 0u);
            }
            if (sub + 1 == D2) mma_commit(bar2(0, b));  // s_full
            mma_commit(kempty(kst));  // K stage read: free it for the next load
            if (sub + 1 == D2 && j + 1 == pc.ntiles) mma_commit(q_empty(qi));  // piece's last S: Q read
          }
          __syncwarp();
          if (++kst == SK) {
            kst = 0;
            kph ^= 1u;
          }
        }
        if (!ok) break;
        ++gt;
      }
      ++qi;
      pc = nx;
      have = have_nx;
      row_cur = row_nxt;
    }
    // Every MMA this thread issued has completed before TMEM is released.
    if (lane == 0) mma_commit(mma_done);
    __syncwarp();
    volatile int never = 0;
    mbar_wait(mma_done, 0, &never, kTimeoutNs / 4);
  } else if (warp == 11) {
    // ------------------------------------------------------------------ O issuer
    // O^T = V^T P^T per tile into the O double buffer once the softmax warps
    // have written P and the correction warps have drained the buffer.
    int vst = 0;
    uint32_t vph = 0, gt = 0;
    bool ok = true;
    Piece pc;
    bool have = walk.next(tp, pc);
    // The new V row of the current piece's segment (fused append), loaded
    // one piece ahead.
    NewRow row_cur = append_fetch<T, H, D, D2, RP>(tp, have ? pc : Piece{}, nch, false, lane);
    while (ok && have) {
      Piece nx;
      const bool have_nx = walk.next(tp, nx);
      const NewRow row_nxt = have_nx ? append_fetch<T, H, D, D2, RP>(tp, nx, nch, false, lane) : row_cur;
      for (int j = 0; j < pc.ntiles; ++j) {
        const uint32_t b = gt & 1u;
        const uint32_t bph = (gt >> 1) & 1u;
        const bool patch = tp.k_new != nullptr && pc.t1 == pc.len && j + 1 == pc.ntiles;
        for (int sub = 0; sub < D2; ++sub) {  // one O accumulator per sub-row
          if (!PKV_TW(3, mbar_wait(vfull(vst), vph, abort_flag, kTimeoutNs))) { ok = false; break; }
          const uint32_t va = sbase + L::kOffV + vst * kOperandBytes;
          const int tile_t0 = pc.t0 + j * kTile;
          if (patch) {
            // the new V row of position len - 1, into the landed tile and the
            // pool (fenced with the stale-row zeroing below)
            append_patch<T, H, D, D2>(tp, pc, nch, va, tile_t0, sub, false, row_cur, row_cur.x, lane);
            if (pc.len % p.block_size == 0) {
              fence_proxy_async_smem();
              __syncwarp();
            }
          }
          // Rows of the last block past the sequence end hold stale pool data:
          // zero them so 0 * (non-finite stale value) never reaches the sum.
          if (pc.t1 == pc.len && tile_t0 + kTile >= pc.len && (pc.len % p.block_size) != 0) {
            const int r0 = pc.len - tile_t0;  // first stale row in the tile
            const int r1 = ((pc.len + p.block_size - 1) / p.block_size) * p.block_size - tile_t0;
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
          if (sub == 0) {
            if (!PKV_TW(4, mbar_wait(bar2(2, b), bph, abort_flag, kTimeoutNs))) { ok = false; break; }
            if (!PKV_TW(5, mbar_wait(bar2(5, b), bph ^ 1u, abort_flag, kTimeoutNs))) { ok = false; break; }
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t pbuf = sbase + L::kOffP + b * L::kPBytes;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              // A = V^T: MN-major SW128, 64-element atoms 16 KB apart (LBO), 8-token groups 1 KB apart (SBO)
              const uint64_t ad = smem_desc_sw128(va + kk * 2048, kHalfBytes, 1024);
              // B = P^T: MN-major SW32, 16-column atoms 4 KB apart (LBO), 8-token groups 256 B apart (SBO)
              const uint64_t bd = smem_desc(pbuf + kk * 512, 4096, 256, kLayoutSwizzle32);
              mma_f16_ss(tmem + 2 * N + (b * D2 + sub) * N, ad, bd, kIdescO, kk > 0 ? 1u : 0u);
            }
            if (sub + 1 == D2) mma_commit(bar2(4, b));  // o_full
            mma_commit(vempty(vst));                     // V stage read
            if (sub + 1 == D2) mma_commit(bar2(3, b));  // p_empty
          }
          __syncwarp();
          if (++vst == SV) {
            vst = 0;
            vph ^= 1u;
          }
        }
        if (!ok) break;
        ++gt;
      }
      pc = nx;
      have = have_nx;
      row_cur = row_nxt;
    }
    if (lane == 0) mma_commit(mma_done);
    __syncwarp();
    volatile int never = 0;
    mbar_wait(mma_done, 0, &never, kTimeoutNs / 4);
  } else if (warp <= 5) {
    // ----------------------------------------------------------- softmax: S -> P
    const int q4 = warp & 3;         // TMEM lane quarter of this warp
    const int row = q4 * 32 + lane;  // TMEM lane: token row of S
    const uint32_t tl = tmem + ((uint32_t)(q4 * 32) << 16);
    uint32_t gt = 0, pi = 0;
    int red_buf = 0;
    // On a timed-out wait the pipeline is abandoned but the control flow of
    // these 128 threads stays uniform (they share named barriers): later waits
    // return at once and the results are garbage, flagged by PIPE_TIMEOUT.
    Piece pc;
    bool have = walk.next(tp, pc);
    while (have) {
      Piece nx;
      const bool have_nx = walk.next(tp, nx);  // its length load overlaps this piece
      float m_ref[N], l_part[N];
#pragma unroll
      for (int n = 0; n < N; ++n) {
        m_ref[n] = kNegInf;
        l_part[n] = 0.f;
      }
      for (int j = 0; j < pc.ntiles; ++j) {
        const uint32_t b = gt & 1u;
        const uint32_t bph = (gt >> 1) & 1u;
        PKV_TW(0, mbar_wait(bar2(0, b), bph, abort_flag, kTimeoutNs));
#ifdef PAGEDKV_TRACE
        if (gt == 0 && warp == 2 && lane == 0) g_tl[misc->tl_ticket % kTraceRecs][4] = globaltimer_ns();
#endif
        PKV_TADD(5, 1);
        tc_fence_after();
        float s[N];
        tmem_ld<N>(tl + b * N, s);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(bar2(1, b));

        // Lazy rescaling: P is exponentiated against a per-column reference
        // max m_ref and only re-based when some score of this tile exceeds it
        // by more than 2^kRescaleLog2 (then P <= 2^8 stays exact in fp16/bf16
        // and the fp32 sums cannot overflow). The decision is one vote over
        // the 128 rows; the exact tile max is only reduced when it is taken.
        const bool valid = pc.t0 + j * kTile + row < pc.t1;
        uint32_t need = 0;
#pragma unroll
        for (int n = 0; n < N; ++n) {
          s[n] = valid ? s[n] * p.scale_log2 : kNegInf;
          need |= s[n] > m_ref[n] + kRescaleLog2 ? 1u : 0u;
        }
        const bool resc = named_bar_or(1, 128, need);
        float alpha[N];
        if (resc) {
          float *rm = red_max + red_buf * 4 * N;
          float wm[N];
#pragma unroll
          for (int n = 0; n < N; ++n) wm[n] = warp_max(s[n]);
          if (lane == 0) {
#pragma unroll
            for (int n = 0; n < N; n += 4)
              *reinterpret_cast<float4 *>(rm + q4 * N + n) = make_float4(wm[n], wm[n + 1], wm[n + 2], wm[n + 3]);
          }
          named_bar(1, 128);
#pragma unroll
          for (int n = 0; n < N; n += 4) {
            const float4 a0 = *reinterpret_cast<const float4 *>(rm + n);
            const float4 a1 = *reinterpret_cast<const float4 *>(rm + N + n);
            const float4 a2 = *reinterpret_cast<const float4 *>(rm + 2 * N + n);
            const float4 a3 = *reinterpret_cast<const float4 *>(rm + 3 * N + n);
            wm[n] = fmaxf(fmaxf(a0.x, a1.x), fmaxf(a2.x, a3.x));
            wm[n + 1] = fmaxf(fmaxf(a0.y, a1.y), fmaxf(a2.y, a3.y));
            wm[n + 2] = fmaxf(fmaxf(a0.z, a1.z), fmaxf(a2.z, a3.z));
            wm[n + 3] = fmaxf(fmaxf(a0.w, a1.w), fmaxf(a2.w, a3.w));
          }
          red_buf ^= 1;
#pragma unroll
          for (int n = 0; n < N; ++n) {
            const float mn = fmaxf(m_ref[n], wm[n]);
            alpha[n] = mn == kNegInf ? 1.f : fast_exp2(m_ref[n] - mn);
            l_part[n] *= alpha[n];
            m_ref[n] = mn;
          }
        }
#pragma unroll
        for (int n = 0; n < N; ++n) {
          s[n] = valid ? fast_exp2(s[n] - m_ref[n]) : 0.f;
          l_part[n] += s[n];
        }
        PKV_TW(2, mbar_wait(bar2(3, b), bph ^ 1u, abort_flag, kTimeoutNs));
        // P^T as the B operand [128 tokens x N], MN-major with 32-byte swizzle:
        // token `row` owns 32 contiguous bytes (16 columns) in each 16-column
        // atom, its two 16-byte halves swapped on rows 4-7 of every 8.
        const uint32_t prow = sbase + L::kOffP + b * L::kPBytes + (row >> 3) * 256 + (row & 7) * 32;
        const uint32_t sw = (row >> 2) & 1;
#pragma unroll
        for (int a = 0; a < N / 16; ++a) {
#pragma unroll
          for (int h8 = 0; h8 < 2; ++h8) {
            float v8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v8[i] = s[a * 16 + h8 * 8 + i];
            const uint4 pk = E::pack8(v8);
            const uint32_t addr = prow + a * 4096 + ((h8 ^ sw) << 4);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(pk.x), "r"(pk.y), "r"(pk.z),
                         "r"(pk.w)
                         : "memory");
          }
        }
        fence_proxy_async_smem();
        if (row == 0) {
          // This tile's rescale record for the correction warps. Slot gt % 4 is
          // rewritten only after the correction warps released O of tile gt
          // (o_empty -> O MMA of gt + 2 -> p_empty of gt + 4), and they read
          // the record before that release.
          Slot &sl = slots[gt % kRescaleSlots];
          if (resc) {
#pragma unroll
            for (int n = 0; n < N; n += 4) {
              *reinterpret_cast<float4 *>(&sl.alpha[n]) = make_float4(alpha[n], alpha[n + 1], alpha[n + 2], alpha[n + 3]);
              *reinterpret_cast<float4 *>(&sl.m[n]) = make_float4(m_ref[n], m_ref[n + 1], m_ref[n + 2], m_ref[n + 3]);
            }
          }
          sl.resc = resc ? 1u : 0u;
          mbar_arrive(a_full(gt % kRescaleSlots));
        }
        mbar_arrive(bar2(2, b));
        ++gt;
      }
      // The piece's denominators: each warp sums its 32 token rows and hands
      // the partial to the correction warps. Slot pi % kLSlots is rewritten
      // kLSlots pieces later, after the correction warps have left this piece
      // (the p_empty / o_empty chain, as for the rescale records).
      {
        // Butterfly reduce-scatter: each stage exchanges half of the columns
        // still held with the partner lane (N - 1 shuffles in all instead of
        // 5 N); lane l ends with column (l >> log2(32 / N)) summed over the
        // lanes that share it, then over the rest.
        static_assert(N == 16 || N == 32, "column count");
#pragma unroll
        for (int w = N / 2, bit = 16; w >= 1; w >>= 1, bit >>= 1) {
          const bool up = (lane & bit) != 0;
#pragma unroll
          for (int i = 0; i < w; ++i) {
            const float keep = up ? l_part[i + w] : l_part[i];
            const float send = up ? l_part[i] : l_part[i + w];
            l_part[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
          }
        }
        constexpr int kShare = 32 / N;  // lanes holding the same column
        if (kShare == 2) l_part[0] += __shfl_xor_sync(0xffffffffu, l_part[0], 1);
        if ((lane & (kShare - 1)) == 0) lpart[((pi % kLSlots) * 4 + q4) * N + lane / kShare] = l_part[0];
        __syncwarp();
        if (lane == 0) mbar_arrive(l_full(pi));
      }
      ++pi;
      pc = nx;
      have = have_nx;
    }
  } else {
    // ---------------------------------------- correction / epilogue: O -> output
    const int q4 = warp & 3;         // TMEM lane quarter of this warp
    const int row = q4 * 32 + lane;  // TMEM lane: (kv head, dim) row of O
    const int hl = row / D;   // kv head of the group this O row belongs to
    const int dim = row % D;
    const uint32_t tl = tmem + ((uint32_t)(q4 * 32) << 16);
    const int HQS = H * GP;  // partial slots per CTA (query columns of a segment)
    uint32_t gt = 0, pi = 0;

    Piece pc;
    bool have = walk.next(tp, pc);
    // The CTA's first Q (with RoPE, its cos / sin rows too) into Q slot 0 by
    // correction warp 7, idle until the first tile is folded, while the
    // producers issue the first ring fill; with RoPE it also rotates it once
    // landed. (The slot's first use: nothing to wait for.)
    if (warp == 7 && have) {
      stage_q<T, H, GP, N, D, D2>(tp, pc, nch, sbase + L::kOffQ, lane);
      if constexpr (RP) stage_cs<T, D, D2>(tp, pc, sbase + L::kOffCS, lane);
      cp_async_mbar_arrive(q_full(0));
      if constexpr (RP) {
        // every lane takes part in the rotation's shuffles, or none does
        const bool landed = mbar_wait(q_full(0), 0u, abort_flag, kTimeoutNs);
        if (__all_sync(0xffffffffu, landed)) {
          rotate_q<T, H, GP, N, D, D2>(p, pc, nch, sbase + L::kOffQ, sbase + L::kOffCS, lane);
          fence_proxy_async_smem();  // the MMA reads the rotated operand through the async proxy
          mbar_arrive(q_rot(0));
        }
      }
    }

    // Sequences of length 0 own no tiles: CTA (seq % grid) writes their zeros.
    for (int s = blockIdx.x; s < p.num_seqs; s += gridDim.x) {
      const int raw = p.lens ? __ldg(p.lens + s) : p.uniform_len;
      if (raw > p.max_blocks * p.block_size && row == 0) set_error(p.err, PAGEDKV_EFLAG_SEQ_LEN_RANGE);
      if (seq_len_clamped(p, s) == 0) {
        T *out = reinterpret_cast<T *>(p.out) + (int64_t)s * p.o_ss;
        for (int idx = row; idx < p.hq * D; idx += 128)
          out[(int64_t)(idx / D) * p.o_sh + idx % D] = E::from_float(0.f);
      }
    }

    while (have) {
      Piece nx;
      const bool have_nx = walk.next(tp, nx);
      float acc[D2][GP], msel[GP];  // acc[sub]: dims sub * 128 + dim
#pragma unroll
      for (int g = 0; g < GP; ++g) {
#pragma unroll
        for (int sub = 0; sub < D2; ++sub) acc[sub][g] = 0.f;
        msel[g] = kNegInf;
      }
      for (int j = 0; j < pc.ntiles; ++j) {
        const uint32_t b = gt & 1u;
        const uint32_t si = gt % kRescaleSlots;
        PKV_TW(0, mbar_wait(a_full(si), (gt / kRescaleSlots) & 1u, abort_flag, kTimeoutNs));
        const Slot &sl = slots[si];
        const bool resc = sl.resc != 0u;
        float a[GP];
        if (resc) {
#pragma unroll
          for (int g = 0; g < GP; ++g) {
            a[g] = sl.alpha[(hl * GP + g) % N];
            msel[g] = sl.m[(hl * GP + g) % N];
          }
        }
        PKV_TW(1, mbar_wait(bar2(4, b), (gt >> 1) & 1u, abort_flag, kTimeoutNs));
        tc_fence_after();
        float o[D2][GP];
#pragma unroll
        for (int sub = 0; sub < D2; ++sub) tmem_ld<GP>(tl + 2 * N + (b * D2 + sub) * N + hl * GP, o[sub]);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(bar2(5, b));
#pragma unroll
        for (int sub = 0; sub < D2; ++sub) {
          if (resc) {
#pragma unroll
            for (int g = 0; g < GP; ++g) acc[sub][g] = fmaf(acc[sub][g], a[g], o[sub][g]);
          } else {
#pragma unroll
            for (int g = 0; g < GP; ++g) acc[sub][g] += o[sub][g];
          }
        }
        ++gt;
      }
      // Denominators of this thread's query columns: the four warp partials.
      float lsum[GP];
      PKV_TW(2, mbar_wait(l_full(pi), ring_parity(pi, kLSlots), abort_flag, kTimeoutNs));
      {
        const float *src = lpart + (pi % kLSlots) * 4 * N + hl * GP;
#pragma unroll
        for (int g = 0; g < GP; ++g) lsum[g] = (src[g] + src[N + g]) + (src[2 * N + g] + src[3 * N + g]);
      }
      ++pi;
#ifdef PAGEDKV_TRACE
      const uint64_t t_epi0 = clock64();
      tw[6] += 1;
#endif
      const int prow = pc.hg / nch;
      const int kv = prow * H + hl;
      const bool have_kv = kv < p.hkv;
      const int qb = (pc.hg - prow * nch) * GP;  // first query head of the chunk
      const int gn = p.group - qb < GP ? p.group - qb : GP;  // query heads in the chunk
      T *out = reinterpret_cast<T *>(p.out) + (int64_t)pc.seq * p.o_ss + (int64_t)(kv * p.group + qb) * p.o_sh + dim;
      if (pc.ntiles == pc.seg_tiles) {
        // Whole segment in this CTA: normalise and store.
        if (have_kv) {
#pragma unroll
          for (int g = 0; g < GP; ++g) {
            if (g < gn) {
#pragma unroll
              for (int sub = 0; sub < D2; ++sub) {
                const float v = lsum[g] > 0.f ? __fdividef(acc[sub][g], lsum[g]) : 0.f;
                out[(int64_t)g * p.o_sh + sub * 128] = E::from_float(v);
              }
            }
          }
        }
      } else if (pc.t0 > 0) {
        // Continuation of a segment that began in an earlier CTA: this is this
        // CTA's first piece. Publish it (partial + release flag) for the CTA
        // owning the segment's first tile, which combines at its end.
        if (have_kv) {
#pragma unroll
          for (int g = 0; g < GP; ++g) {
            if (g < gn) {
              const int64_t hh = vcta * HQS + hl * GP + g;
#pragma unroll
              for (int sub = 0; sub < D2; ++sub) tp.part_acc[hh * D + sub * 128 + dim] = acc[sub][g];
              if (dim == 0) tp.part_ml[hh] = make_float2(msel[g], lsum[g]);
            }
          }
        }
        named_bar(2, 128);
        if (row == 0) {
          __threadfence();  // release every thread's partial (cumulative over the barrier)
          st_volatile_u32(tp.flags + vcta, 1u);
        }
      } else {
        // First tile of the segment is here and the segment runs past this
        // CTA's range: this is this CTA's last piece, and this CTA combines.
        // The other pieces are the first pieces of ranges b+1..b1, published
        // early in their runs.
        PieceAcc<GP, D2> pa;
#pragma unroll
        for (int g = 0; g < GP; ++g) {
#pragma unroll
          for (int sub = 0; sub < D2; ++sub) pa.acc[sub][g] = acc[sub][g];
          pa.lsum[g] = lsum[g];
          pa.msel[g] = msel[g];
        }
        const int64_t b1 = owner_of(pc.seg_units + kSegUnits + (int64_t)pc.seg_tiles * kTileUnits - 1, U_total, G);
        combine_pieces<T, GP, D, D2>(tp, pa, vcta, b1, G, hl, dim, gn, have_kv, out, abort_flag, row);
      }
#ifdef PAGEDKV_TRACE
      tw[4] += clock64() - t_epi0;
#endif
      pc = nx;
      have = have_nx;
    }
    if (warp == 7) cp_async_wait<0>();  // the first Q's copies (landed on the normal path)
  }

  // ---------------------------------------------------------------- teardown
#ifdef PAGEDKV_TRACE
  {
    // rows: 0 K producer, 1 S issuer, 2 softmax, 4 correction, 5 V producer,
    // 6 O issuer (lane 0 of the role's first warp); row 3 the CTA's totals.
    const int trow = warp == 0 ? 0 : warp == 1 ? 1 : warp == 2 ? 2 : warp == 7 ? 4 : warp == 6 ? 5 : warp == 11 ? 6 : -1;
    if (blockIdx.x < kTraceCtas && lane == 0 && trow >= 0) {
      for (int i = 0; i < kTraceSlots; ++i) g_trace[blockIdx.x][trow][i] = tw[i];
      g_trace[blockIdx.x][3][8 + trow] = clock64() - c_kernel0;  // this role's own finish
    }
  }
  __syncthreads();
  if (blockIdx.x < kTraceCtas && threadIdx.x == 0) {
    g_trace[blockIdx.x][3][0] = globaltimer_ns() - t_kernel0;
    g_trace[blockIdx.x][3][1] = t_kernel0;
    g_trace[blockIdx.x][3][2] = (unsigned long long)(misc->hi - misc->lo);
    g_trace[blockIdx.x][3][3] = clock64() - c_kernel0;
    g_trace[blockIdx.x][3][4] = globaltimer_ns();
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    g_trace[blockIdx.x][3][5] = smid;
  }
  if (threadIdx.x == 0) g_tl[misc->tl_ticket % kTraceRecs][5] = globaltimer_ns();
#endif
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
  int H, D2, GP, N, stages, head_groups, chunks, grid;
};

int round_up(int x, int m) { return (x + m - 1) / m * m; }

TcPlan make_plan(int32_t num_seqs, int32_t hq, int32_t hkv, int32_t head_dim, int32_t max_tokens,
                 int32_t num_sms) {
  TcPlan pl;
  // A tile row is 128 elements: H = 128 / head_dim kv heads side by side, or
  // for head_dim 256 one head as D2 = 2 sub-rows (two ring stages per tile).
  pl.D2 = head_dim > 128 ? head_dim / 128 : 1;
  pl.H = head_dim > 128 ? 1 : 128 / head_dim;
  const int G = hq / hkv;
  // Query columns per kv head: the group padded to 8, at most 32 / H (N <= 32),
  // 16 with two sub-rows (their correction threads hold twice the sums).
  // A wider group is cut into chunks of that many heads, one segment each; the
  // chunks of a tile row run back to back and re-read its K/V from L2.
  const int gp_max = pl.D2 > 1 ? 16 : pl.H == 1 ? 32 : 16 / (pl.H / 2);
  pl.chunks = (G + gp_max - 1) / gp_max;
  pl.GP = pl.chunks > 1 ? gp_max : round_up(G, 8);
  if (pl.H == 1 && pl.GP > 16) pl.GP = 32;  // one kv head per tile: columns 17..32 share the N = 32 variant
  pl.N = round_up(pl.H * pl.GP, 16);
  pl.stages = pl.N <= 16 ? 3 : 2;
  pl.head_groups = (hkv + pl.H - 1) / pl.H * pl.chunks;
  const int64_t max_tiles = ((int64_t)(max_tokens > 0 ? max_tokens : 1) + kTile - 1) / kTile;
  const int64_t tiles_upper = (int64_t)num_seqs * pl.head_groups * max_tiles;
  int grid = num_sms;
#ifdef PAGEDKV_TRACE
  if (const char *e = getenv("PAGEDKV_TRACE_GRID")) grid = atoi(e);
#endif
  pl.grid = (int)(tiles_upper < grid ? tiles_upper : grid);
  if (pl.grid < 1) pl.grid = 1;
  return pl;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

size_t plan_workspace(const TcPlan &pl, int32_t num_seqs, int32_t hq, int32_t hkv, int32_t head_dim) {
  (void)num_seqs;
  (void)hq;
  (void)hkv;
  const size_t hqs = (size_t)pl.H * pl.GP;
  const size_t slots = (size_t)pl.grid;
  return kWorkspaceHeaderBytes + align256(slots * hqs * sizeof(float2)) +
         align256(slots * hqs * head_dim * sizeof(float));
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

bool encode_map(CUtensorMap *map, const void *base, int dtype, uint64_t row_elems, uint64_t rows,
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

// Encoded tensor maps of recently used pools (a decode step reuses the same
// per-layer K/V tensors every step), keyed by everything the encoding reads.
struct MapKey {
  const void *base;
  uint64_t row_elems, rows;
  uint32_t box_rows;
  int dtype;
  bool operator==(const MapKey &o) const {
    return base == o.base && row_elems == o.row_elems && rows == o.rows && box_rows == o.box_rows &&
           dtype == o.dtype;
  }
};

bool make_map(CUtensorMap *map, const void *base, int dtype, uint64_t row_elems, uint64_t rows,
              uint32_t box_rows) {
  constexpr int kSlots = 128;
  static std::mutex mu;
  static MapKey keys[kSlots];
  static CUtensorMap maps[kSlots];
  static int used = 0, next = 0;
  const MapKey key{base, row_elems, rows, box_rows, dtype};
  {
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < used; ++i) {
      if (keys[i] == key) {
        *map = maps[i];
        return true;
      }
    }
  }
  if (!encode_map(map, base, dtype, row_elems, rows, box_rows)) return false;
  std::lock_guard<std::mutex> lk(mu);
  keys[next] = key;
  maps[next] = *map;
  next = (next + 1) % kSlots;
  if (used < kSlots) ++used;
  return true;
}

template <typename T, bool RP, int H, int GP, int N, int SK, int SV, bool CH = false, int D2 = 1>
cudaError_t launch_tc(const CUtensorMap &mk, const CUtensorMap &mv, const TcParams &tp, int grid,
                      cudaStream_t stream) {
  using L = SmemLayout<N, SK, SV, D2, RP>;
  static_assert(L::kAlloc <= 227 * 1024, "dynamic shared memory above the sm_100 per-block limit");
  auto kern = decode_tc_kernel<T, H, GP, N, SK, SV, CH, D2, RP>;
  // The shared-memory opt-in is a per-device function attribute: set it once
  // per device (outside any stream capture that follows the first call).
  static std::atomic<uint64_t> attr_done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  // Launched as a programmatic dependent of the previous kernel in the stream
  // (griddepcontrol in the kernel orders the global reads after it).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mk, mv, tp);
}

// RP: RoPE fused (cos / sin given), a separate instantiation so that the
// plain kernel carries none of the rotation code.
template <typename T, bool RP>
cudaError_t dispatch_tc(const TcPlan &pl, const CUtensorMap &mk, const CUtensorMap &mv, const TcParams &tp,
                        cudaStream_t stream) {
  if (pl.D2 == 2) {
    // head_dim 256: 3 K + 2 V ring stages of half a tile each (shared memory)
    if (pl.chunks > 1) return launch_tc<T, RP, 1, 16, 16, 3, 2, true, 2>(mk, mv, tp, pl.grid, stream);
    if (pl.GP == 8) return launch_tc<T, RP, 1, 8, 16, 3, 2, false, 2>(mk, mv, tp, pl.grid, stream);
    if (pl.GP == 16) return launch_tc<T, RP, 1, 16, 16, 3, 2, false, 2>(mk, mv, tp, pl.grid, stream);
    return cudaErrorInvalidValue;
  }
  if (pl.chunks > 1) {
    if (pl.H == 1 && pl.GP == 32) return launch_tc<T, RP, 1, 32, 32, 2, 2, true>(mk, mv, tp, pl.grid, stream);
    if (pl.H == 2 && pl.GP == 16) return launch_tc<T, RP, 2, 16, 32, 2, 2, true>(mk, mv, tp, pl.grid, stream);
    if (pl.H == 4 && pl.GP == 8) return launch_tc<T, RP, 4, 8, 32, 2, 2, true>(mk, mv, tp, pl.grid, stream);
    return cudaErrorInvalidValue;
  }
  if (pl.H == 2 && pl.GP == 8) return launch_tc<T, RP, 2, 8, 16, 3, 3>(mk, mv, tp, pl.grid, stream);
  if (pl.H == 2 && pl.GP == 16) return launch_tc<T, RP, 2, 16, 32, 2, 2>(mk, mv, tp, pl.grid, stream);
  if (pl.H == 1 && pl.GP == 8) return launch_tc<T, RP, 1, 8, 16, 3, 3>(mk, mv, tp, pl.grid, stream);
  if (pl.H == 1 && pl.GP == 16) return launch_tc<T, RP, 1, 16, 16, 3, 3>(mk, mv, tp, pl.grid, stream);
  if (pl.H == 1 && pl.GP == 32) return launch_tc<T, RP, 1, 32, 32, 2, 2>(mk, mv, tp, pl.grid, stream);
  if (pl.H == 4 && pl.GP == 8) return launch_tc<T, RP, 4, 8, 32, 2, 2>(mk, mv, tp, pl.grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace

#ifdef PAGEDKV_TRACE
extern "C" int pagedkv_trace_read(unsigned long long *host, size_t count) {
  const size_t n = sizeof(g_trace) / sizeof(unsigned long long);
  return cudaMemcpyFromSymbol(host, g_trace, (count < n ? count : n) * sizeof(unsigned long long)) == cudaSuccess ? 0 : 3;
}
// The CTA timeline records (kTraceRecs x 6) and the ticket counter.
extern "C" int pagedkv_trace_timeline(unsigned long long *host, size_t count, unsigned long long *tickets) {
  const size_t n = sizeof(g_tl) / sizeof(unsigned long long);
  if (cudaMemcpyFromSymbol(tickets, g_tl_ctr, sizeof(unsigned long long)) != cudaSuccess) return 3;
  return cudaMemcpyFromSymbol(host, g_tl, (count < n ? count : n) * sizeof(unsigned long long)) == cudaSuccess ? 0 : 3;
}
#endif

bool tc_eligible(int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size) {
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return false;
  const int G = num_q_heads / num_kv_heads;
  // A tile row is 128 elements: 128 / head_dim kv heads side by side (or one
  // head_dim-256 head as two sub-rows), and their query columns (padded
  // groups) fill at most the N = 32 MMA width; wider groups run in chunks of
  // 32 / 16 / 8 / 16 query heads per kv head. Small groups
  // run here too: the pipeline is bound by HBM, not by the MMA shape
  // (measured 1.1-2.7x faster than the CUDA-core kernel at G = 1, 2).
  if (G < 1) return false;
  if (head_dim != 256 && head_dim != 128 && head_dim != 64 && head_dim != 32) return false;
  if (block_size < 8 || block_size > 128 || (block_size & (block_size - 1)) != 0) return false;
  return true;
}

size_t tc_workspace_bytes(int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t max_tokens, int32_t num_sms) {
  const TcPlan pl = make_plan(num_seqs, num_q_heads, num_kv_heads, head_dim, max_tokens, num_sms);
  return plan_workspace(pl, num_seqs, num_q_heads, num_kv_heads, head_dim);
}

int tc_launch(DecodeParams &p, int dtype, void *workspace, size_t workspace_bytes, int32_t num_sms,
              cudaStream_t stream, int *launches, std::string *error, const AppendParams *append) {
  *launches = 0;
  const int32_t max_tokens = p.max_blocks * p.block_size;
  const TcPlan pl = make_plan(p.num_seqs, p.hq, p.hkv, p.head_dim, max_tokens, num_sms);
  const size_t need = plan_workspace(pl, p.num_seqs, p.hq, p.hkv, p.head_dim);
  if (need > workspace_bytes || workspace == nullptr) {
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
  if (pl.grid * sizeof(uint32_t) > kWorkspaceHeaderBytes) {
    *error = "tensor-core decode: grid larger than the workspace flag header";
    return PAGEDKV_ERR_UNSUPPORTED;
  }
  TcParams tp{};
  tp.head_groups = pl.head_groups;
  tp.chunks = pl.chunks;
  tp.oob_row = (int32_t)rows;
  const size_t hqs = (size_t)pl.H * pl.GP;
  const size_t slots = (size_t)pl.grid;
  char *ws = static_cast<char *>(workspace);
  tp.flags = reinterpret_cast<uint32_t *>(ws);  // zero between launches
  ws += kWorkspaceHeaderBytes;
  tp.part_ml = reinterpret_cast<float2 *>(ws);
  ws += align256(slots * hqs * sizeof(float2));
  tp.part_acc = reinterpret_cast<float *>(ws);
  if (append != nullptr) {
    tp.k_new = append->k_new;
    tp.v_new = append->v_new;
    tp.kn_st = append->k_st;
    tp.kn_sh = append->k_sh;
    tp.vn_st = append->v_st;
    tp.vn_sh = append->v_sh;
    tp.cos = append->cos;
    tp.sin = append->sin;
    tp.cs_st = append->cs_st;
  }
  tp.p = p;
  const bool rope = tp.cos != nullptr;
  cudaError_t e;
  if (dtype == PAGEDKV_DTYPE_BF16)
    e = rope ? dispatch_tc<__nv_bfloat16, true>(pl, mk, mv, tp, stream)
             : dispatch_tc<__nv_bfloat16, false>(pl, mk, mv, tp, stream);
  else
    e = rope ? dispatch_tc<__half, true>(pl, mk, mv, tp, stream) : dispatch_tc<__half, false>(pl, mk, mv, tp, stream);
  if (e != cudaSuccess) {
    *error = std::string("tensor-core decode launch: ") + cudaGetErrorString(e);
    return PAGEDKV_ERR_CUDA;
  }
  *launches = 1;
  return PAGEDKV_OK;
}

}  // namespace pagedkv
