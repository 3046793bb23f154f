// In-place KV-cache append: cache[b, h, pos, :] = src[t, h, :] with
// (b, pos) = divmod(slot_mapping[t], max_seq_len); negative slots are skipped.
//
// Follows the slot semantics of src/csrc/ops/kv_cache.cu:25-42 (and the pin in
// tests/test_kv_cache.py:85-118).  Unlike that kernel this one uses 64-bit
// offsets throughout and bounds-checks the batch index on the device (an
// out-of-range slot is skipped and flagged instead of written).
//
// Layout: one thread moves one 16-byte vector; a 32-lane warp therefore moves
// two 256-byte head rows (head_dim 128 in bf16) per instruction, the K row and
// the V row of the same (token, head) side by side, so both the source reads
// and the cache writes are fully coalesced 128-bit accesses.
#include "lpc_common.cuh"

LPC_DECLARE_STATUS(g_kv_status)

unsigned int lpc_status_kv(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_kv_status, sizeof(v));
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_kv_status, &z, sizeof(z));
  }
  return v;
}

namespace {

template <typename VecT>
__global__ void __launch_bounds__(256) kv_append_kernel(
    const VecT* __restrict__ ksrc, const VecT* __restrict__ vsrc, VecT* __restrict__ kcache,
    VecT* __restrict__ vcache, const int64_t* __restrict__ slots, int64_t num_tokens,
    int64_t src_token_stride_v, int num_kv_heads, int vecs_per_row, int64_t max_batch,
    int64_t max_seq_len) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_pair = 2 * (int64_t)vecs_per_row;  // K row then V row
  const int64_t pair = gid / per_pair;                  // (token, head)
  if (pair >= num_tokens * num_kv_heads) return;
  const int within = (int)(gid - pair * per_pair);
  const bool is_v = within >= vecs_per_row;
  const int vec = is_v ? within - vecs_per_row : within;
  const int64_t t = pair / num_kv_heads;
  const int h = (int)(pair - t * num_kv_heads);

  const int64_t slot = slots ? __ldg(slots + t) : t;
  if (slot < 0) return;
  const int64_t b = slot / max_seq_len;
  const int64_t pos = slot - b * max_seq_len;
  if (b >= max_batch) {
    atomicOr(&g_kv_status, LPC_DEV_ERR_BOUNDS);
    return;
  }
  const int64_t src_off = t * src_token_stride_v + (int64_t)h * vecs_per_row + vec;
  const int64_t dst_off = ((b * num_kv_heads + h) * max_seq_len + pos) * vecs_per_row + vec;
  if (is_v)
    vcache[dst_off] = __ldg(vsrc + src_off);
  else
    kcache[dst_off] = __ldg(ksrc + src_off);
}

}  // namespace

extern "C" int lpc_update_kv_cache(const void* key_src, const void* value_src, void* key_cache,
                                   void* value_cache, const int64_t* slot_mapping,
                                   int64_t num_tokens, int64_t src_token_stride, int num_kv_heads,
                                   int head_dim, int64_t max_batch, int64_t max_seq_len,
                                   int elem_bytes, void* stream) {
  using namespace lpc;
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || max_batch <= 0 ||
      max_seq_len <= 0) {
    set_error("update_kv_cache: invalid sizes (tokens=%lld heads=%d dim=%d batch=%lld seq=%lld)",
              (long long)num_tokens, num_kv_heads, head_dim, (long long)max_batch,
              (long long)max_seq_len);
    return LPC_ERR_INVALID;
  }
  if (elem_bytes != 2 && elem_bytes != 4) {
    set_error("update_kv_cache: element size must be 2 or 4 bytes, got %d", elem_bytes);
    return LPC_ERR_UNSUPPORTED;
  }
  if (src_token_stride < (int64_t)num_kv_heads * head_dim) {
    set_error("update_kv_cache: source token stride %lld smaller than heads*dim",
              (long long)src_token_stride);
    return LPC_ERR_INVALID;
  }
  if (num_tokens == 0) return LPC_OK;
  if (!key_src || !value_src || !key_cache || !value_cache) {
    set_error("update_kv_cache: null pointer");
    return LPC_ERR_INVALID;
  }
  const int64_t row_bytes = (int64_t)head_dim * elem_bytes;
  const bool vec16 = (row_bytes % 16 == 0) && ((src_token_stride * elem_bytes) % 16 == 0) &&
                     aligned16(key_src) && aligned16(value_src) && aligned16(key_cache) &&
                     aligned16(value_cache);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = 256;
  if (vec16) {
    const int vpr = (int)(row_bytes / 16);
    const int64_t total = num_tokens * num_kv_heads * 2 * vpr;
    const int64_t blocks = (total + threads - 1) / threads;
    kv_append_kernel<uint4><<<(unsigned)blocks, threads, 0, s>>>(
        (const uint4*)key_src, (const uint4*)value_src, (uint4*)key_cache, (uint4*)value_cache,
        slot_mapping, num_tokens, src_token_stride * elem_bytes / 16, num_kv_heads, vpr,
        max_batch, max_seq_len);
  } else if (elem_bytes == 2) {
    const int64_t total = num_tokens * num_kv_heads * 2 * head_dim;
    const int64_t blocks = (total + threads - 1) / threads;
    kv_append_kernel<uint16_t><<<(unsigned)blocks, threads, 0, s>>>(
        (const uint16_t*)key_src, (const uint16_t*)value_src, (uint16_t*)key_cache,
        (uint16_t*)value_cache, slot_mapping, num_tokens, src_token_stride, num_kv_heads,
        head_dim, max_batch, max_seq_len);
  } else {
    const int64_t total = num_tokens * num_kv_heads * 2 * head_dim;
    const int64_t blocks = (total + threads - 1) / threads;
    kv_append_kernel<uint32_t><<<(unsigned)blocks, threads, 0, s>>>(
        (const uint32_t*)key_src, (const uint32_t*)value_src, (uint32_t*)key_cache,
        (uint32_t*)value_cache, slot_mapping, num_tokens, src_token_stride, num_kv_heads,
        head_dim, max_batch, max_seq_len);
  }
  return check_launch("update_kv_cache");
}
