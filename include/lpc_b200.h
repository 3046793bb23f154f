/*
 * lpc_b200.h -- C ABI of the B200 (sm_100a) Llama inference hot path.
 *
 * Plain pointers, sizes and a CUDA stream handle (passed as void*); no torch
 * or C++ types.  Every entry point:
 *   - validates its arguments on the host and returns LPC_ERR_INVALID (the
 *     Python layer raises ValueError) or LPC_ERR_UNSUPPORTED (TypeError)
 *     with a message available from lpc_last_error();
 *   - enqueues its kernels on `stream` and returns without synchronising;
 *   - returns LPC_ERR_CUDA if a launch fails (RuntimeError).
 * Device pointers must be 16-byte aligned and tensors contiguous unless a
 * stride argument says otherwise.  Nothing here allocates device memory:
 * ops that need scratch take a caller-provided workspace whose size comes
 * from the matching *_workspace_bytes() query.
 *
 * Reference citations are paths inside the Llama_Pure_Compute project.
 */
#ifndef LPC_B200_H
#define LPC_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define LPC_API __attribute__((visibility("default")))
#else
#define LPC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LPC_OK 0
#define LPC_ERR_INVALID 1      /* bad shape / pointer / argument (ValueError)  */
#define LPC_ERR_UNSUPPORTED 2  /* dtype or size the kernels do not cover (TypeError) */
#define LPC_ERR_CUDA 3         /* a CUDA call or launch failed (RuntimeError)  */

#define LPC_DTYPE_F32 0
#define LPC_DTYPE_F16 1
#define LPC_DTYPE_BF16 2

/* Library version, e.g. 100 for 0.1.0. */
LPC_API int lpc_version(void);

/* Message describing the last non-zero status returned on this host thread. */
LPC_API const char* lpc_last_error(void);

/* OR of the device status words of all kernels (timeouts of bounded waits,
 * failed device-side bounds checks) since the last call; clears them.
 * Synchronises the current device.  Returns -1 if the read itself failed. */
LPC_API int lpc_device_status(void);

/*
 * In-place KV-cache append.
 * Replaces: `_backend.update_kv_cache` (src/llama_pure_compute/ops.py:139-166,
 *           src/csrc/ops/kv_cache.cu:13-43 and :152-198).
 * key_src/value_src: [num_tokens, num_kv_heads, head_dim], row stride
 *   `src_token_stride` elements between tokens (num_kv_heads*head_dim when packed).
 * key_cache/value_cache: [max_batch, num_kv_heads, max_seq_len, head_dim].
 * slot_mapping: int64 [num_tokens] or NULL (slot = token index).
 *   (b, pos) = divmod(slot, max_seq_len); slot < 0 is skipped; a slot at or
 *   beyond max_batch*max_seq_len is skipped and flagged in lpc_device_status().
 * elem_bytes: 2 or 4 (the op is a copy, bit-exact for every dtype).
 */
LPC_API int lpc_update_kv_cache(const void* key_src, const void* value_src, void* key_cache,
                        void* value_cache, const int64_t* slot_mapping, int64_t num_tokens,
                        int64_t src_token_stride, int num_kv_heads, int head_dim,
                        int64_t max_batch, int64_t max_seq_len, int elem_bytes, void* stream);

/*
 * In-place rotary embedding (half-split / "rotate_half" convention).
 * Replaces: `_backend.rope_forward` (src/llama_pure_compute/ops.py:95-117,
 *           src/csrc/ops/rope.cu:10-84 and :143-193); semantics of
 *           `_rope_forward_pytorch` (ops.py:27-42).
 * q: [num_tokens, num_heads, head_dim], k: [num_tokens, num_kv_heads, head_dim].
 * Table modes:
 *   table_mode 0: cos/sin are [table_rows, head_dim/2]; row = position_ids[t]
 *                 (or t when position_ids is NULL)  -- rope.cu convention.
 *   table_mode 1: cos/sin are [num_tokens, head_dim]; row = t (tables already
 *                 gathered per token, as LlamaModel.forward passes them,
 *                 src/llama_pure_compute/model.py:388-393).
 * out[d]     = q[d]*cos[d]     - q[d+h]*sin[d]
 * out[d+h]   = q[d+h]*cos[d+h] + q[d]*sin[d+h]   (h = head_dim/2; mode 0 uses
 *                                                 column d for both halves)
 * computed in fp32 with single-rounded products and sum, rounded once to the
 * output dtype.  q_dtype is shared by q and k; table_dtype by cos and sin.
 */
LPC_API int lpc_rope_forward(void* q, void* k, const void* cos, const void* sin,
                     const int64_t* position_ids, int64_t num_tokens, int num_heads,
                     int num_kv_heads, int head_dim, int table_mode, int64_t table_rows,
                     int q_dtype, int table_dtype, void* stream);

/*
 * Fused decode/prefill attention prologue: RoPE on q and k taken straight from
 * the fused QKV projection, q written head-major for attention, rotated k and
 * v appended into the caches.
 * Replaces the sequence rope_forward -> transpose(1,2).contiguous() x3 ->
 *   KVCacheManager.update (src/llama_pure_compute/model.py:146-168,
 *   src/llama_pure_compute/kv_manager.py:207-317).
 * qkv: [batch, seq, (num_heads + 2*num_kv_heads) * head_dim] (q | k | v).
 * positions: int64 [batch, seq] absolute positions; row b of the caches is
 *   written at pos = positions[b, s]; a negative position skips the token.
 * cos/sin: [table_rows, head_dim] full-width tables (precompute_freqs_cis,
 *   model.py:28-64) in table_dtype.
 * q_out: [batch, num_heads, seq, head_dim].
 */
LPC_API int lpc_rope_kv_append(const void* qkv, const int64_t* positions, const void* cos,
                       const void* sin, int64_t table_rows, void* q_out, void* key_cache,
                       void* value_cache, int64_t batch, int64_t seq, int num_heads,
                       int num_kv_heads, int head_dim, int64_t max_batch, int64_t max_seq_len,
                       int dtype, int table_dtype, void* stream);

/*
 * RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w, fp32 math, output in x's dtype.
 * Replaces: `rmsnorm_triton_forward` / `_rmsnorm_pytorch_fallback`
 *           (src/llama_pure_compute/triton_kernels/rmsnorm.py:20-96).
 * x, y: [rows, dim]; w: [dim] in w_dtype.
 */
LPC_API int lpc_rmsnorm_forward(const void* x, const void* w, void* y, int64_t rows, int dim, float eps,
                        int dtype, int w_dtype, void* stream);

/*
 * Fused RMSNorm + SwiGLU: out = silu(norm(x) W_gate^T) * (norm(x) W_up^T).
 * Replaces: `_backend.rmsswiglu_forward` (src/llama_pure_compute/ops.py:120-136,
 *           src/csrc/ops/rmsswiglu.cu:151-282); semantics of
 *           `_rmsswiglu_forward_pytorch` (ops.py:45-59).
 * x: [tokens, dim]; rms_weight: [dim] (w_dtype); out: [tokens, inter].
 * gate_w, up_w: [inter, dim].  up_w == NULL means gate_w is the fused
 *   [2*inter, dim] matrix (gate rows first), as rmsswiglu.cu:167-173 accepts.
 * bf16 / fp16: tcgen05 tensor-core GEMM with the SiLU*up epilogue; needs
 *   lpc_rmsswiglu_workspace_bytes() of workspace (the normalised activations).
 * fp32: CUDA-core streaming kernel (no TF32), workspace unused.
 * eps must be > 0.
 */
LPC_API int64_t lpc_rmsswiglu_workspace_bytes(int64_t tokens, int dim, int dtype);
LPC_API int lpc_rmsswiglu_forward(const void* x, const void* rms_weight, const void* gate_w,
                          const void* up_w, void* out, void* workspace, int64_t workspace_bytes,
                          int64_t tokens, int dim, int inter, float eps, int dtype, int w_dtype,
                          void* stream);

/*
 * Causal / non-causal flash attention with q_len <= kv_len, queries aligned to
 * the END of the key sequence (bottom-right causal mask), fp32 accumulation.
 * Replaces: `flash_attention_v2` prefill path
 *           (src/llama_pure_compute/triton_kernels/flash_attention.py:88-432,
 *           :998-1155); mask semantics of tests/test_attention_correctness.py:10-76.
 * q: [batch, heads, q_len, head_dim]; k, v: [batch, kv_heads, kv_len, head_dim]
 * with row strides given in elements between consecutive positions
 * (k_seq_stride) and heads (k_head_stride), batches (k_batch_stride), so a
 * slice of a preallocated cache can be passed without a copy.
 * out: [batch, heads, q_len, head_dim].  head_dim 64 or 128, bf16 or fp16 (the
 * Python entry point runs head_dim 32 through the 64 kernel on zero-padded rows).
 */
LPC_API int lpc_flash_attention(const void* q, const void* k, const void* v, void* out, int64_t batch,
                        int heads, int kv_heads, int64_t q_len, int64_t kv_len, int head_dim,
                        int64_t k_batch_stride, int64_t k_head_stride, int causal, float sm_scale,
                        int dtype, void* stream);

/*
 * RMSNorm + SwiGLU in one kernel, for weights that already carry the norm
 * weight: gate_w / up_w hold W[n, k] * rms_weight[k] (e.g. folded once when a
 * model is loaded; up_w NULL: gate_w is the fused [2 * inter, dim] form).
 *   out = silu(rsqrt(mean(x^2) + eps) * x gate_w^T) * (rsqrt(...) * x up_w^T)
 * Replaces: rmsswiglu_forward's three steps (rmsswiglu.cu:176-196: norm into
 *           an HBM buffer, GEMM, activation) for a caller that owns its weights.
 * The CTA-pair tcgen05 GEMM takes each token row's sum of squares from the
 * activation tiles it feeds the tensor core and scales the fp32 accumulators
 * in the epilogue: no normalised copy of x is written.  bf16 or fp16, dim a
 * multiple of 64, inter of 16.  No workspace.
 */
LPC_API int lpc_rmsswiglu_folded_forward(const void* x, const void* gate_w, const void* up_w,
                                         void* out, int64_t tokens, int dim, int inter, float eps,
                                         int dtype, void* stream);

/*
 * Split-KV decode attention over ragged per-sequence context lengths
 * (one query token per sequence).
 * Replaces: `_flash_decode_kernel` (flash_attention.py:450-710, launched at
 *           :1161-1197), generalised from one KV_LEN per call to a device
 *           array of lengths.
 * q: [batch, heads, head_dim]; caches [max_batch, kv_heads, max_seq_len, head_dim];
 * seq_lens: int32 [batch] on the device, keys [0, seq_lens[b]) are attended;
 * out: [batch, heads, head_dim].  head_dim 32, 64 or 128; bf16 or fp16.
 * workspace: lpc_decode_attention_workspace_bytes(batch, heads, max_seq_len, head_dim)
 * bytes (per-split partial results).  Each sequence is cut into splits of
 * lpc_decode_attention_split_keys(batch, kv_heads, max_seq_len, 0) keys (the
 * ragged call: its total_rows instead of 0), one CTA each; a second (combine)
 * kernel merges them unless that length is at least max_seq_len.
 */
LPC_API int64_t lpc_decode_attention_workspace_bytes(int64_t batch, int heads, int64_t max_seq_len,
                                             int head_dim);

/* Keys per split that the decode attention calls use for `batch` sequences,
 * `kv_heads` KV heads and a cache of max_seq_len keys per sequence
 * (total_rows: the ragged cache's rows per KV head; <= 0 for the dense
 * cache, whose capacity is batch * max_seq_len).  1024 with at least 2048
 * (sequence, KV head) pairs, or when whole 1024-key splits of the capacity
 * give 2048 CTAs; 512 when whole 512-key splits do; else 256.  The
 * environment variable LPC_DECODE_CHUNK (a multiple of 32 in [256, 65536])
 * overrides it.  The calls launch one kernel when the result is >=
 * max_seq_len, two otherwise.  0 for invalid sizes.  Host only. */
LPC_API int lpc_decode_attention_split_keys(int64_t batch, int kv_heads, int64_t max_seq_len,
                                            int64_t total_rows);
LPC_API int lpc_decode_attention(const void* q, const void* key_cache, const void* value_cache,
                         const int32_t* seq_lens, void* out, void* workspace,
                         int64_t workspace_bytes, int64_t batch, int heads, int kv_heads,
                         int head_dim, int64_t max_batch, int64_t max_seq_len, float sm_scale,
                         int dtype, void* stream);

/*
 * Ragged KV layout (variable-length sequences packed back to back).
 * Cache tensors are [kv_heads, total_rows, head_dim]; sequence b owns rows
 * [seq_base[b], seq_base[b] + seq_cap[b]) of every head (seq_base int64 and
 * seq_cap int32, device arrays of `batch` entries).  Memory then grows with the
 * sum of the sequences' capacities instead of batch * max length -- what lets
 * 64 prompts of 1k-8k tokens (+256 generated) fit one GPU.
 * Replaces the dense per-layer cache of KVCacheManager (kv_manager.py:90-121)
 * for mixed-length batches; the paged/ragged cache of runtime/paged_cache.py:14-57.
 *
 * lpc_rope_kv_append_ragged: as lpc_rope_kv_append, writing position p of
 *   sequence b at row seq_base[b] + p; p >= seq_cap[b], or a row range outside
 *   the buffer, is skipped and flagged in lpc_device_status().
 * lpc_decode_attention_ragged: as lpc_decode_attention over keys
 *   [0, seq_lens[b]) of sequence b's rows; max_seq_len bounds every seq_cap
 *   (it sizes the split grid and the workspace, as in lpc_decode_attention).
 */
LPC_API int lpc_rope_kv_append_ragged(const void* qkv, const int64_t* positions, const void* cos,
                                      const void* sin, int64_t table_rows, void* q_out,
                                      void* key_cache, void* value_cache, const int64_t* seq_base,
                                      const int32_t* seq_cap, int64_t batch, int64_t seq,
                                      int num_heads, int num_kv_heads, int head_dim,
                                      int64_t total_rows, int dtype, int table_dtype, void* stream);
LPC_API int lpc_decode_attention_ragged(const void* q, const void* key_cache,
                                        const void* value_cache, const int32_t* seq_lens,
                                        const int64_t* seq_base, const int32_t* seq_cap, void* out,
                                        void* workspace, int64_t workspace_bytes, int64_t batch,
                                        int heads, int kv_heads, int head_dim, int64_t total_rows,
                                        int64_t max_seq_len, float sm_scale, int dtype,
                                        void* stream);

/*
 * Decode attention that allocates nothing.  No counterpart in the reference:
 * it is an addition for callers that cannot allocate device memory when they
 * run attention -- a plugin whose host application owns all of HBM (e.g. a
 * serving engine that reserves the free memory for its KV cache), or a
 * serving loop that must never call cudaMalloc mid-request because the call
 * can synchronise the device or fail under memory pressure.
 * Same arguments and results as lpc_decode_attention, minus the workspace:
 * the split partials go to a fixed scratch array of LPC_NOALLOC_SCRATCH_BYTES
 * inside this library.  The array belongs to the decode-attention module, so
 * every GPU on which any decode-attention entry point (workspace, ragged or
 * this one) has run holds those 24 MiB until the process exits.  Shapes whose
 * partials need more
 * (batch * heads * ceil(max_seq_len / 256) * (head_dim + 2) * 4 bytes), and
 * sizes beyond the split grid (batch > 65535, max_seq_len > 65535 * 256), are
 * rejected with LPC_ERR_INVALID before anything runs.
 * The first call on a device, and the first call in a new CUDA context of a
 * device (after a device reset), looks up the array's device address with
 * that device current; make that first call before any stream capture.
 * All calls share the one array: calls that overlap on the GPU (two streams,
 * or two host threads) race on it; serialise them.  Nothing in it needs to
 * start at zero, each call writes every partial it reads.
 */
/* Static device footprint of the library: 24 MiB per GPU once any decode
 * attention has run on it (the scratch array of the entry point below). */
#define LPC_NOALLOC_SCRATCH_BYTES (24u * 1024u * 1024u)
LPC_API int lpc_decode_attention_noalloc(const void* q, const void* key_cache,
                                         const void* value_cache, const int32_t* seq_lens,
                                         void* out, int64_t batch, int heads, int kv_heads,
                                         int head_dim, int64_t max_batch, int64_t max_seq_len,
                                         float sm_scale, int dtype, void* stream);

/*
 * Weight packing for the decode-sized GEMM below.  Run once per weight at
 * model load.  The packed copy stores each 128-row x 64-k tile of the weight
 * as one contiguous 16 KB block, already in the 128-byte-swizzled K-major
 * layout that the tensor core reads from shared memory.
 * layout 0: W0 [n_out, k] row-major (a linear layer's weight).
 * layout 1: SwiGLU gate/up pair, n_out = intermediate size; gate rows from W0
 *           [n_out, k] and up rows from W1 [n_out, k], or from W0 rows
 *           n_out..2*n_out-1 when W1 is NULL (the fused gate_up layout that
 *           rmsswiglu_forward accepts, ops.py:118-131).
 * layout 2: attention heads, W0 [(H + 2*Hkv) * 128, k] (the q, k and v
 *           projection weights stacked, head_dim 128); each head's rows are
 *           interleaved so that the rotate-half partners d and d + 64 meet in
 *           one warp of the epilogue (lpc_qkv_rope_append).
 * k_scale: NULL, or k fp32 factors that multiply column k of every weight row
 * (W[n, k] * k_scale[k], one rounding): the weight of the RMSNorm whose output
 * the projection consumes, folded in so that lpc_wsgemm / lpc_qkv_rope_append
 * can normalise inside the GEMM (norm_eps > 0 there).
 * packed: lpc_packed_weight_bytes(n_out, k, layout) bytes, 16-byte aligned.
 * k must be a multiple of 64; bf16 or fp16.  Returns after the packed copy is
 * complete (the call synchronises `stream`): lpc_wsgemm starts reading the
 * weights before it waits on the previous kernel of its stream.
 */
LPC_API int64_t lpc_packed_weight_bytes(int64_t n_out, int k, int layout);
LPC_API int lpc_pack_weights(const void* w0, const void* w1, const float* k_scale, void* packed,
                             int64_t n_out, int k, int layout, int dtype, void* stream);

/*
 * Decode-sized GEMM against packed weights:
 *   out[t, n] = epilogue(sum_k x[t, k] * W[n, k]),  t < tokens <= 256.
 * Replaces: the gate/up GEMMs inside rmsswiglu_forward (ops.py:118-131) of a
 *           decode step, once the norm has been applied (epilogue 2), and --
 *           for wide layers such as lm_head (model.py:421) -- nn.Linear
 *           projections (epilogues 0 and 1).  One CTA per 128-row weight tile:
 *           meant for layers with about a hundred tiles or more.
 * epilogue 0: out = acc                        (out [tokens, n_out])
 * epilogue 1: out = resid + acc                (resid may equal out)
 * epilogue 2: out = silu(x Wg^T) * (x Wu^T)    (packed with layout 1; out [tokens, n_out])
 * x: [tokens, k] contiguous; fp32 accumulation, one rounding to the dtype.
 * n_out <= 2^24.  No workspace.
 * norm_eps > 0 fuses the RMSNorm that feeds the projection (triton_kernels/
 * rmsnorm.py:58-96): x are the raw rows, the norm weight is folded into the
 * packed weight (lpc_pack_weights' k_scale), and every token's accumulators
 * are scaled by rsqrt(mean(x^2) + norm_eps) -- the sums of squares are read
 * by the kernel's epilogue warps from x in global memory while the weights
 * stream, so no normalised copy of x is written.  Fastest up to about 64
 * tokens (each CTA re-reads its k-range of every row).  norm_eps = 0: x is
 * used as given.
 * Split k: when there are few weight tiles the launch runs clusters of up to
 * 8 CTAs per tile, each on a share of k, reduce-scattered through
 * distributed shared memory (deterministic: fixed rank order).  Launched with
 * programmatic stream serialisation: the prologue and the first weight chunks
 * overlap the previous kernel on the stream, and nothing that kernel writes
 * is read before it completes.
 */
LPC_API int lpc_wsgemm(const void* x, const void* packed_w, void* out, const void* resid,
                       int64_t tokens, int64_t n_out, int k, int epilogue, int dtype,
                       float norm_eps, void* stream);

/*
 * Fused projection + RoPE + KV append of the attention block for decode-sized
 * token counts (batch * seq <= 256):
 *   qkv = x W^T  (W packed with layout 2, rounded to the dtype), then exactly
 *   lpc_rope_kv_append on it: q rotated into q_out [batch, H, seq, 128], k
 *   rotated and v copied into the cache row of (b, positions[b, s]).
 * Replaces: the q/k/v projections, RoPE and the KV update of
 *           LlamaAttention.forward (model.py:125-168, kv_manager.py:207-317)
 *           in one kernel: no qkv intermediate, no second launch.
 * x: [batch * seq, k] (the normed hidden states); positions [batch, seq]
 * int64 (< 0: the token is skipped); cos/sin [table_rows, 128] in the data
 * dtype (the model's cos_cached / sin_cached).  Cache layouts as in
 * lpc_rope_kv_append (seq_base == NULL: dense [max_batch, Hkv, max_seq_len,
 * 128]) and lpc_rope_kv_append_ragged ([Hkv, total_rows, 128] at
 * seq_base[b] + pos, pos < seq_cap[b]).  Out-of-range positions or rows set
 * LPC_DEV_ERR_BOUNDS and skip the token.  head_dim must be 128; bf16 or fp16.
 * norm_eps > 0: x are the raw hidden states and the input RMSNorm runs inside
 * the kernel, as for lpc_wsgemm (its weight folded into the packed weight).
 */
LPC_API int lpc_qkv_rope_append(const void* x, const void* packed_w, const int64_t* positions,
                                const void* cos, const void* sin, int64_t table_rows, void* q_out,
                                void* key_cache, void* value_cache, const int64_t* seq_base,
                                const int32_t* seq_cap, int64_t batch, int64_t seq, int num_heads,
                                int num_kv_heads, int head_dim, int k, int64_t max_batch,
                                int64_t max_seq_len, int64_t total_rows, int dtype, int table_dtype,
                                float norm_eps, void* stream);

/*
 * HBM read-rate probe (a measurement utility; no reference counterpart).
 * Reads `bytes` (a positive multiple of 131072) of `buf` the way the decode
 * attention reads its cache rows: one CTA per 128 KB, 16 KB 1-D bulk copies
 * into a 4-stage shared-memory ring, no arithmetic.  Bytes over its event
 * time are the read ceiling of such a kernel; the copy rate usually quoted
 * as peak counts every byte twice (read and write) and is lower.
 */
LPC_API int lpc_hbm_read_probe(const void* buf, int64_t bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LPC_B200_H */
