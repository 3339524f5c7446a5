// Decode attention for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc (or any allocating library routine) on
// the decode path: a serving loop that runs under a fixed memory budget
// reserved up front, code that runs while another component owns the CUDA
// caching allocator, or a host language binding that has no allocator handle
// at all. pagedkv_decode_attention needs a caller-provided workspace for its
// cross-CTA flags and split-K partial sums; this entry point supplies that
// scratch from a fixed array compiled into the library instead, so the caller
// passes only inputs and outputs.
//
// The array lives at file scope in device memory: every GPU that loads the
// library holds its kNoAllocScratchBytes until the process exits, and every
// call on that GPU shares it, so calls that overlap on the GPU (different
// streams, or concurrent host threads on one device) race on it and must be
// serialised by the caller. The first call on a device resolves the array's
// device address (cudaGetSymbolAddress); make that first call before any
// stream capture.
#include <cstdio>
#include <mutex>

#include "../../include/pagedkv.h"
#include "launch.h"

namespace pagedkv {
namespace {

// 4 MiB per device. The tensor-core path needs 8 KiB of flags plus one
// partial slot per CTA (about 1.3 MB on a 148-SM B200 whatever the batch);
// the CUDA-core split-K path needs 8 KiB plus num_seqs * num_q_heads * splits
// * (head_dim * 4 + 8) bytes. Shapes beyond the bound are rejected.
constexpr size_t kNoAllocScratchBytes = 4u << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices] = {};

int fail(int code, const char *msg) {
  set_last_error_message(msg);
  return code;
}

// Device address of this device's copy of the scratch array. The host-side
// name of a __device__ variable is only a stand-in, never a device address,
// so it is resolved with cudaGetSymbolAddress once per device, with that
// device current.
int scratch_for_current_device(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(PAGEDKV_ERR_CUDA, "no-alloc decode: no usable current CUDA device");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(PAGEDKV_ERR_CUDA, "no-alloc decode: cudaGetSymbolAddress of the scratch array failed");
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return PAGEDKV_OK;
}

}  // namespace
}  // namespace pagedkv

using namespace pagedkv;

extern "C" {

int pagedkv_decode_attention_noalloc(
    void *out, int64_t out_stride_seq, int64_t out_stride_head,
    const void *q, int64_t q_stride_seq, int64_t q_stride_head,
    const void *k_cache, const void *v_cache,
    const int32_t *block_tables, int64_t block_tables_stride,
    const int32_t *seq_lens, int32_t uniform_seq_len,
    int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t max_blocks_per_seq, float scale, int32_t dtype, void *stream) {
  const size_t need = pagedkv_decode_attention_workspace_size(
      num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks_per_seq, dtype);
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "no-alloc decode: this shape needs %zu bytes of scratch, more than the fixed %zu; "
             "use pagedkv_decode_attention with a caller workspace",
             need, kNoAllocScratchBytes);
    return fail(PAGEDKV_ERR_WORKSPACE, msg);
  }
  void *scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != PAGEDKV_OK) return rc;
  // The first kWorkspaceHeaderBytes are completion flags the kernels expect
  // at zero. The array keeps whatever the previous call left, so clear them
  // on the caller's stream before every launch (a memset, not an allocation).
  const cudaError_t e =
      cudaMemsetAsync(scratch, 0, kWorkspaceHeaderBytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(PAGEDKV_ERR_CUDA, "no-alloc decode: clearing the flag header failed");
  return pagedkv_decode_attention(out, out_stride_seq, out_stride_head, q, q_stride_seq,
                                q_stride_head, k_cache, v_cache, block_tables,
                                block_tables_stride, seq_lens, uniform_seq_len, num_seqs,
                                num_q_heads, num_kv_heads, head_dim, num_blocks, block_size,
                                max_blocks_per_seq, scale, dtype, scratch, kNoAllocScratchBytes,
                                stream);
}

}  // extern "C"
