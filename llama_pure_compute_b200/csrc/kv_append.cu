// In-place KV-cache append: cache[b, h, pos, :] = src[t, h, :] with
// (b, pos) = divmod(slot_mapping[t], max_seq_len); negative slots are skipped.
//
// Follows the slot semantics of src/csrc/ops/kv_cache.cu:25-42 (and the pin in
// tests/test_kv_cache.py:85-118).  Unlike that kernel this one uses 64-bit
// offsets throughout and bounds-checks the batch index on the device (an
// out-of-range slot is skipped and flagged instead of written).
//
// Layout (16-byte path): a CTA owns a run of whole tokens.  Its first threads
// turn each token's slot into a cache row once (64-bit division, bounds
// check) and leave it in shared memory; then every thread moves up to UNROLL
// 16-byte vectors of the run, all loads issued before the first store.  A
// token's vectors are ordered K heads then V heads, head rows contiguous, so a
// warp reads 512 contiguous source bytes (two head_dim-128 bf16 rows) and
// writes two full 256-byte cache rows per instruction.
#include <algorithm>

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

constexpr int KV_THREADS = 256;
constexpr int KV_UNROLL = 8;
constexpr int KV_MAX_TOKENS = 64;  // tokens per CTA (cache rows kept in shared memory)

// vecs_per_token = 2 * num_kv_heads * vecs_per_row; tokens [t0, t0 + ntok).
__global__ void __launch_bounds__(KV_THREADS) kv_append_rows_kernel(
    const uint4* __restrict__ ksrc, const uint4* __restrict__ vsrc, uint4* __restrict__ kcache,
    uint4* __restrict__ vcache, const int64_t* __restrict__ slots, int64_t num_tokens,
    int64_t src_token_stride_v, int num_kv_heads, int vecs_per_row, int tokens_per_cta,
    int64_t max_batch, int64_t max_seq_len) {
  __shared__ int64_t row0[KV_MAX_TOKENS];  // cache row of (b, head 0, pos); -1: skip
  const int64_t t0 = (int64_t)blockIdx.x * tokens_per_cta;
  const int ntok = (int)std::min<int64_t>(tokens_per_cta, num_tokens - t0);
  if ((int)threadIdx.x < ntok) {
    const int64_t t = t0 + threadIdx.x;
    const int64_t slot = slots ? __ldg(slots + t) : t;
    int64_t r = -1;
    if (slot >= 0) {
      const int64_t b = slot / max_seq_len;
      if (b < max_batch)
        r = b * num_kv_heads * max_seq_len + (slot - b * max_seq_len);
      else
        atomicOr(&g_kv_status, LPC_DEV_ERR_BOUNDS);
    }
    row0[threadIdx.x] = r;
  }
  __syncthreads();
  const int half = num_kv_heads * vecs_per_row;  // K vectors of a token
  const int vpt = 2 * half;
  const int total = ntok * vpt;
  for (int base = 0; base < total; base += KV_THREADS * KV_UNROLL) {
    uint4 v[KV_UNROLL];
    int64_t dst[KV_UNROLL];
    bool isv[KV_UNROLL];
#pragma unroll
    for (int u = 0; u < KV_UNROLL; ++u) {
      const int idx = base + u * KV_THREADS + (int)threadIdx.x;
      dst[u] = -1;
      if (idx < total) {
        const int tl = idx / vpt;
        const int within = idx - tl * vpt;
        isv[u] = within >= half;
        const int r = isv[u] ? within - half : within;
        const int h = r / vecs_per_row;
        const int vec = r - h * vecs_per_row;
        const int64_t rr = row0[tl];
        if (rr >= 0) {
          const int64_t src = (t0 + tl) * src_token_stride_v + r;
          v[u] = isv[u] ? __ldg(vsrc + src) : __ldg(ksrc + src);
          dst[u] = (rr + (int64_t)h * max_seq_len) * vecs_per_row + vec;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < KV_UNROLL; ++u) {
      if (dst[u] >= 0) {
        if (isv[u])
          vcache[dst[u]] = v[u];
        else
          kcache[dst[u]] = v[u];
      }
    }
  }
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
  const int64_t vpt16 = 2 * (int64_t)num_kv_heads * (row_bytes / 16);
  if (vec16 && vpt16 <= (int64_t)KV_THREADS * KV_UNROLL * 16) {
    // tokens per CTA: enough for about KV_UNROLL vectors per thread, but at
    // least two CTAs per SM while the token count allows it
    const int vpr = (int)(row_bytes / 16);
    const int64_t sms = current_device_sms();
    int64_t tpc = std::max<int64_t>(1, (int64_t)KV_THREADS * KV_UNROLL / vpt16);
    tpc = std::min<int64_t>({tpc, (int64_t)KV_MAX_TOKENS,
                             std::max<int64_t>(1, num_tokens / (2 * sms))});
    const int64_t blocks = (num_tokens + tpc - 1) / tpc;
    if (blocks > 0x7fffffffLL) {
      set_error("update_kv_cache: too many tokens (%lld)", (long long)num_tokens);
      return LPC_ERR_UNSUPPORTED;
    }
    kv_append_rows_kernel<<<(unsigned)blocks, KV_THREADS, 0, s>>>(
        (const uint4*)key_src, (const uint4*)value_src, (uint4*)key_cache, (uint4*)value_cache,
        slot_mapping, num_tokens, src_token_stride * elem_bytes / 16, num_kv_heads, vpr, (int)tpc,
        max_batch, max_seq_len);
  } else if (vec16) {
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
