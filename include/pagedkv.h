/*
 * pagedkv.h — C ABI of the B200 (sm_100a) paged KV-cache decode path.
 *
 * Three operations make up the path:
 *   1. batched GQA decode attention that reads K/V through a block table,
 *   2. the per-step KV append into the [num_blocks, block_size, kv_heads,
 *      head_dim] pool through a slot mapping,
 *   3. the copy-on-write block copy behind the prefix cache.
 *
 * Every entry point takes plain device pointers, element strides and sizes
 * and a CUDA stream handle (cudaStream_t passed as void*). Nothing here
 * allocates device memory except where stated; nothing synchronises the host
 * except pagedkv_read_error_flags(). All launches go to the given stream.
 *
 * Return value: PAGEDKV_OK (0) or one of the PAGEDKV_ERR_* codes below; the
 * calling thread's last message is available from pagedkv_last_error().
 *
 * Pool layout (shared by all entry points, identical to the reference's
 * PhysicalBlockPool, engine/memory/block_allocator.py:68-101): one K and one V
 * tensor per layer, each contiguous with shape
 *   [num_blocks, block_size, num_kv_heads, head_dim]
 * so token slot s = block_id * block_size + offset starts at element
 *   s * num_kv_heads * head_dim.
 * Byte offsets are computed in 64 bits; a pool tensor may exceed 2^31 bytes.
 */
#ifndef PAGEDKV_H_
#define PAGEDKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define PAGEDKV_OK                    0
#define PAGEDKV_ERR_INVALID_ARGUMENT  1  /* shape / pointer / alignment check failed */
#define PAGEDKV_ERR_UNSUPPORTED       2  /* head_dim or dtype outside the built kernels */
#define PAGEDKV_ERR_CUDA              3  /* a CUDA runtime call failed */
#define PAGEDKV_ERR_WORKSPACE         4  /* workspace missing or too small */

/* ---- element types ------------------------------------------------------ */
#define PAGEDKV_DTYPE_F16   0
#define PAGEDKV_DTYPE_BF16  1
#define PAGEDKV_DTYPE_F32   2   /* prefill-write sources only */

/* ---- device error word bits (set by kernels, read by pagedkv_read_error_flags) */
#define PAGEDKV_EFLAG_BLOCK_ID_RANGE  0x1u  /* a block-table entry >= num_blocks or < 0 */
#define PAGEDKV_EFLAG_SLOT_RANGE      0x2u  /* a slot >= num_blocks * block_size */
#define PAGEDKV_EFLAG_SEQ_LEN_RANGE   0x4u  /* seq_len > max_blocks_per_seq * block_size */
#define PAGEDKV_EFLAG_COPY_RANGE      0x8u  /* a copy_blocks src/dst outside [0, num_blocks) */
#define PAGEDKV_EFLAG_PIPE_TIMEOUT    0x10u /* a bounded pipeline wait gave up */

/* Library version string, e.g. "pagedkv-b200 0.1.0 sm_100a". */
const char *pagedkv_version(void);

/* Message for the last non-zero status returned on the calling thread. */
const char *pagedkv_last_error(void);

/*
 * Decode attention, batched over sequences (one new query token each).
 *
 * Replaces the launch of _paged_attention_decode_batched_kernel inside
 * paged_attention_decode_batched (engine/kernels/paged_attention.py:634-698,
 * launch at :675-697) and, with num_seqs == 1 and seq_lens == NULL, the v1 and
 * v2 single-sequence launches (paged_attention.py:254-305 and :419-470).
 *
 *   out[s, h, :] = softmax(scale * q[s, h, :] . K[s, :, h / G, :]) @ V[s, :, h / G, :]
 *
 * over the first seq_len(s) tokens of sequence s, whose token t lives in pool
 * block block_tables[s * block_tables_stride + t / block_size] at offset
 * t % block_size. G = num_q_heads / num_kv_heads. Accumulation is fp32; out
 * is stored in the pool dtype. A sequence with seq_len 0 yields zeros.
 *
 * q/out: [num_seqs, num_q_heads, head_dim], last dim contiguous, strides in
 * elements. seq_lens: int32 device array, or NULL to use uniform_seq_len for
 * every sequence. block_tables: int32 [num_seqs, >= max_blocks_per_seq].
 * Entries beyond a sequence's last used block are never read.
 *
 * workspace: device scratch of at least
 * pagedkv_decode_attention_workspace_size(...) bytes (may be NULL when that
 * size is 0). Its first 8 KiB hold cross-CTA completion flags: zero-fill the
 * buffer once before its first use; every call leaves those bytes zero again
 * (after a PAGEDKV_EFLAG_PIPE_TIMEOUT report, zero them again). The rest is
 * overwritten before it is read. Calls that overlap on the GPU must not share
 * a workspace.
 */
int pagedkv_decode_attention(
    void *out, int64_t out_stride_seq, int64_t out_stride_head,
    const void *q, int64_t q_stride_seq, int64_t q_stride_head,
    const void *k_cache, const void *v_cache,
    const int32_t *block_tables, int64_t block_tables_stride,
    const int32_t *seq_lens, int32_t uniform_seq_len,
    int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t max_blocks_per_seq, float scale, int32_t dtype,
    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Decode attention with the decode append fused into the same launch.
 *
 * Replaces the append + kernel pair of one layer's decode forward
 * (engine/kernels/paged_attention_integration.py:150-160, then the kernel
 * call at :164-171 / engine/kernels/paged_attention.py:675-697): for every
 * sequence s with L = seq_lens[s] > 0, first
 *   k_cache[table_s[(L-1) / block_size], (L-1) % block_size] = k_new[s]
 * (and v_new into v_cache), bit-exact, then decode attention over the L
 * tokens exactly as pagedkv_decode_attention. With cos and sin (rows
 * [num_seqs, head_dim], stride cos_sin_stride) both q and k_new are rotated
 * first, rounded as transformers' apply_rotary_pos_emb
 * (integration.py:108-109) and as pagedkv_kv_append_rope: the pool rows are
 * bit-identical to that op's and the output to pagedkv_decode_attention on
 * its rotated q. The rows are written by the CTA that reads that tile, just
 * before it loads it, so the append costs no launch and no dependency of its
 * own. k_new / v_new: [num_seqs, num_kv_heads, head_dim], 16-byte aligned,
 * strides multiples of 8 elements. Shapes that run on the CUDA-core kernel
 * (block_size < 8 or not a power of two), or unaligned k_new / v_new / cos /
 * sin, return PAGEDKV_ERR_UNSUPPORTED without launching anything: call
 * pagedkv_kv_append (or _rope) and pagedkv_decode_attention instead. Same
 * workspace as pagedkv_decode_attention.
 */
int pagedkv_decode_attention_append(
    void *out, int64_t out_stride_seq, int64_t out_stride_head,
    const void *q, int64_t q_stride_seq, int64_t q_stride_head,
    void *k_cache, void *v_cache,
    const int32_t *block_tables, int64_t block_tables_stride,
    const int32_t *seq_lens,
    int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t max_blocks_per_seq,
    const void *k_new, int64_t k_new_stride_seq, int64_t k_new_stride_head,
    const void *v_new, int64_t v_new_stride_seq, int64_t v_new_stride_head,
    const void *cos, const void *sin, int64_t cos_sin_stride,
    float scale, int32_t dtype, void *workspace, size_t workspace_bytes,
    void *stream);

/* Bytes of workspace pagedkv_decode_attention needs for this shape on the
 * current device (0 when the launch needs none). */
size_t pagedkv_decode_attention_workspace_size(
    int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t block_size, int32_t max_blocks_per_seq,
    int32_t dtype);

/*
 * KV append: write one layer's new K and V rows into the pool.
 *
 * Replaces the per-sequence index_put loop of paged_decode_attention_forward
 * (engine/kernels/paged_attention_integration.py:150-160, single-sequence form
 * at :120-132): for token i with slot = slot_mapping[i] >= 0,
 *   k_cache[slot / block_size, slot % block_size, :, :] = k_new[i, :, :]
 * and the same for V, as a bit-exact copy. slot < 0 skips the token (padding).
 * A slot >= num_blocks * block_size is skipped and sets
 * PAGEDKV_EFLAG_SLOT_RANGE. k_new/v_new: [num_tokens, num_kv_heads, head_dim],
 * last dim contiguous, strides in elements. One launch covers K and V.
 */
int pagedkv_kv_append(
    void *k_cache, void *v_cache,
    const void *k_new, int64_t k_new_stride_tok, int64_t k_new_stride_head,
    const void *v_new, int64_t v_new_stride_tok, int64_t v_new_stride_head,
    const int64_t *slot_mapping, int32_t num_tokens, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size, int32_t dtype,
    void *stream);

/*
 * Copy-on-write block copy over every layer's K and V pool.
 *
 * The reference has no data copy for CoW: BlockAllocator.fork only bumps a
 * refcount (engine/memory/block_allocator.py:264-270) and the decode runner
 * asserts it never writes a shared block (paged_attention_integration.py:
 * 587-592). This entry point is the copy that assert stands in for: for every
 * pair p and layer l,
 *   k_cache[l][block_mapping[2p + 1]] = k_cache[l][block_mapping[2p]]
 * and the same for V, bit-exact. k_cache_ptrs / v_cache_ptrs are DEVICE arrays
 * of num_layers pool base pointers (16-byte aligned, as every allocation of the
 * CUDA caching allocators is); block_mapping is a device int64 [num_pairs, 2]
 * (src, dst) array. Destinations must be distinct and must not appear as a
 * source in the same call. block_bytes = block_size * num_kv_heads * head_dim
 * * element size. One launch covers all layers, K and V.
 */
int pagedkv_copy_blocks(
    void *const *k_cache_ptrs, void *const *v_cache_ptrs, int32_t num_layers,
    const int64_t *block_mapping, int32_t num_pairs, int64_t block_bytes,
    int64_t num_blocks, void *stream);

/*
 * Fused rotary embedding + KV append for a decode step. Replaces the
 * apply_rotary_pos_emb call (engine/kernels/paged_attention_integration.py:
 * 108-109, transformers' x * cos + rotate_half(x) * sin with
 * rotate_half(x) = cat(-x[D/2:], x[:D/2])) plus the append of :150-160.
 * For token t: q_out[t, h] = rope(q[t, h]) for every query head;
 * k_cache[slot] = rope(k_new[t]), v_cache[slot] = v_new[t] with
 * slot = slot_mapping[t] (negative = skip), rounded exactly as the tensor ops
 * (each product and the sum rounded to the dtype), i.e. bit-identical to the
 * reference's result. cos / sin: [num_tokens, head_dim] rows (row stride
 * cos_sin_stride_tok, last dim contiguous) in the same dtype. All strides are in
 * elements with a contiguous last dim; head_dim a multiple of 16. q_out may
 * alias q. One launch.
 */
int pagedkv_kv_append_rope(
    void *q_out, int64_t q_out_stride_tok, int64_t q_out_stride_head,
    const void *q, int64_t q_stride_tok, int64_t q_stride_head, int32_t num_q_heads,
    void *k_cache, void *v_cache,
    const void *k_new, int64_t k_new_stride_tok, int64_t k_new_stride_head,
    const void *v_new, int64_t v_new_stride_tok, int64_t v_new_stride_head,
    const void *cos, const void *sin, int64_t cos_sin_stride_tok,
    const int64_t *slot_mapping, int32_t num_tokens, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size, int32_t dtype,
    void *stream);

/*
 * Prefill K/V write: a prompt's rows of every layer into whole pool blocks.
 * Replaces KernelPagedManualDecode._copy_prefill_kv
 * (engine/kernels/paged_attention_integration.py:278-326: pad to whole blocks,
 * .to(pool dtype), index_copy_ into each layer's K and V pool). For every
 * layer l, block i < num_write_blocks, position t < block_size, kv head h:
 *   pool[l][block_ids[i], t, h, :] = src[l][i * block_size + t, h, :]
 *                                    if i * block_size + t < num_tokens,
 *                                  = 0 otherwise (the padded tail),
 * bit-exact (f32 sources are rounded to nearest even, as torch's .to()).
 * k_caches / v_caches / k_srcs / v_srcs are HOST arrays of num_layers device
 * pointers; each source is a [num_tokens, num_kv_heads, head_dim] view with the
 * given element strides (last dim contiguous), src_dtype = the pool dtype or
 * PAGEDKV_DTYPE_F32. block_ids is a DEVICE int64 [num_write_blocks] array
 * (out-of-range ids are skipped and flagged PAGEDKV_EFLAG_BLOCK_ID_RANGE).
 * One launch per 48 layers, K and V together.
 */
int pagedkv_kv_write_prefill(
    void *const *k_caches, void *const *v_caches,
    const void *const *k_srcs, const void *const *v_srcs, int32_t num_layers,
    int64_t k_src_stride_tok, int64_t k_src_stride_head,
    int64_t v_src_stride_tok, int64_t v_src_stride_head, int32_t src_dtype,
    const int64_t *block_ids, int32_t num_write_blocks, int32_t num_tokens,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t dtype, void *stream);

/*
 * Read (and optionally clear) the device error word of the current device.
 * Synchronises `stream`. Kernels never trap on bad indices: they skip the
 * access and set a PAGEDKV_EFLAG_* bit, which this call reports.
 */
int pagedkv_read_error_flags(uint32_t *flags_out, int32_t clear, void *stream);

/*
 * Decode attention that allocates nothing: the same computation, arguments and
 * result as pagedkv_decode_attention, minus the workspace. No counterpart in
 * the reference (its Triton path needs no scratch).
 *
 * For callers that cannot allocate device memory on the decode path (a fixed
 * memory budget reserved up front, an allocator owned by another component, a
 * binding with no allocator at all). The scratch comes from a 4 MiB array
 * compiled into the library, held by every GPU that loads it until exit;
 * shapes needing more return PAGEDKV_ERR_WORKSPACE. All calls on a device
 * share the array: calls that overlap on the GPU race and must be serialised.
 * The first call on a device resolves the array's address; make it before any
 * stream capture. Each call clears the array's flag header on `stream` first.
 */
int pagedkv_decode_attention_noalloc(
    void *out, int64_t out_stride_seq, int64_t out_stride_head,
    const void *q, int64_t q_stride_seq, int64_t q_stride_head,
    const void *k_cache, const void *v_cache,
    const int32_t *block_tables, int64_t block_tables_stride,
    const int32_t *seq_lens, int32_t uniform_seq_len,
    int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t max_blocks_per_seq, float scale, int32_t dtype, void *stream);

/*
 * Number of kernel launches the last pagedkv_decode_attention call on this
 * thread issued (1 or 2: the split-K combine is a second launch), and the
 * name of the decode kernel family it chose ("tc" = tcgen05/TMA, "simt").
 */
int32_t pagedkv_last_decode_launches(void);
const char *pagedkv_last_decode_kernel(void);

#ifdef __cplusplus
}
#endif

#endif /* PAGEDKV_H_ */
