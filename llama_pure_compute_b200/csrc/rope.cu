// Rotary position embedding (half-split convention) and the fused
// RoPE + KV-append prologue of the attention block.
//
// Math follows `_rope_forward_pytorch` (src/llama_pure_compute/ops.py:27-42):
//   out[d]   = x[d]*cos[d]     - x[d+h]*sin[d]
//   out[d+h] = x[d+h]*cos[d+h] + x[d]*sin[d+h]
// evaluated in fp32 with every product and the sum rounded separately
// (__fmul_rn / __fadd_rn, so no FMA contraction) and rounded once to the
// storage dtype, as src/csrc/ops/rope.cu:39-45 does.  For fp32 data this is
// bit-identical to the PyTorch fallback; for bf16/fp16 data the products of
// two 16-bit values are exact in fp32, so the result is the correctly rounded
// value of the exact expression.
//
// Each thread owns VEC consecutive rotation pairs of one (token, head): it
// loads the VEC lower-half and VEC upper-half elements as 16-byte vectors.
#include <algorithm>

#include <cstdlib>

#include "lpc_common.cuh"

LPC_DECLARE_STATUS(g_rope_status)

unsigned int lpc_status_rope(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_rope_status, sizeof(v));
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_rope_status, &z, sizeof(z));
  }
  return v;
}

namespace {

using lpc::Num;

template <typename T, int N>
__device__ __forceinline__ void load_f(const T* __restrict__ p, float (&f)[N]) {
  constexpr int bytes = (int)sizeof(T) * N;
  if constexpr (bytes % 16 == 0) {
    constexpr int per = 16 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < N / per; ++i) {
      uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + i);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < per; ++j) f[i * per + j] = Num<T>::to_f(e[j]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = Num<T>::to_f(p[i]);
  }
}

// Plain (coherent) load variant for data this kernel writes in place.
template <typename T, int N>
__device__ __forceinline__ void load_f_rw(const T* p, float (&f)[N]) {
  constexpr int bytes = (int)sizeof(T) * N;
  if constexpr (bytes % 16 == 0) {
    constexpr int per = 16 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < N / per; ++i) {
      uint4 u = reinterpret_cast<const uint4*>(p)[i];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < per; ++j) f[i * per + j] = Num<T>::to_f(e[j]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = Num<T>::to_f(p[i]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_f(T* p, const float (&f)[N]) {
  constexpr int bytes = (int)sizeof(T) * N;
  if constexpr (bytes % 16 == 0) {
    constexpr int per = 16 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < N / per; ++i) {
      uint4 u;
      T* e = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int j = 0; j < per; ++j) e[j] = Num<T>::from_f(f[i * per + j]);
      reinterpret_cast<uint4*>(p)[i] = u;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = Num<T>::from_f(f[i]);
  }
}

template <int VEC>
__device__ __forceinline__ void rotate(const float (&x0)[VEC], const float (&x1)[VEC],
                                       const float (&c0)[VEC], const float (&s0)[VEC],
                                       const float (&c1)[VEC], const float (&s1)[VEC],
                                       float (&o0)[VEC], float (&o1)[VEC]) {
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    o0[i] = __fsub_rn(__fmul_rn(x0[i], c0[i]), __fmul_rn(x1[i], s0[i]));
    o1[i] = __fadd_rn(__fmul_rn(x1[i], c1[i]), __fmul_rn(x0[i], s1[i]));
  }
}

// In-place RoPE on q [T, H, D] and k [T, Hkv, D].
template <typename T, typename TT, int VEC>
__global__ void __launch_bounds__(256) rope_kernel(T* q, T* k, const TT* __restrict__ cosb,
                                                   const TT* __restrict__ sinb,
                                                   const int64_t* __restrict__ pos_ids,
                                                   int64_t num_tokens, int num_heads,
                                                   int num_kv_heads, int head_dim, int table_mode,
                                                   int64_t table_rows) {
  const int half = head_dim >> 1;
  const int chunks = half / VEC;
  const int heads_all = num_heads + num_kv_heads;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t work = num_tokens * heads_all * chunks;
  if (gid >= work) return;
  const int c = (int)(gid % chunks);
  const int64_t th = gid / chunks;
  const int hh = (int)(th % heads_all);
  const int64_t t = th / heads_all;

  T* row = hh < num_heads ? q + (t * num_heads + hh) * (int64_t)head_dim
                          : k + (t * num_kv_heads + (hh - num_heads)) * (int64_t)head_dim;
  const int d = c * VEC;

  float c0[VEC], s0[VEC], c1[VEC], s1[VEC];
  if (table_mode == 0) {
    const int64_t r = pos_ids ? __ldg(pos_ids + t) : t;
    if (r < 0 || r >= table_rows) {
      atomicOr(&g_rope_status, LPC_DEV_ERR_BOUNDS);
      return;
    }
    load_f<TT, VEC>(cosb + r * half + d, c0);
    load_f<TT, VEC>(sinb + r * half + d, s0);
#pragma unroll
    for (int i = 0; i < VEC; ++i) { c1[i] = c0[i]; s1[i] = s0[i]; }
  } else {
    const TT* cr = cosb + t * (int64_t)head_dim;
    const TT* sr = sinb + t * (int64_t)head_dim;
    load_f<TT, VEC>(cr + d, c0);
    load_f<TT, VEC>(sr + d, s0);
    load_f<TT, VEC>(cr + d + half, c1);
    load_f<TT, VEC>(sr + d + half, s1);
  }
  float x0[VEC], x1[VEC], o0[VEC], o1[VEC];
  load_f_rw<T, VEC>(row + d, x0);
  load_f_rw<T, VEC>(row + d + half, x1);
  rotate<VEC>(x0, x1, c0, s0, c1, s1, o0, o1);
  store_f<T, VEC>(row + d, o0);
  store_f<T, VEC>(row + d + half, o1);
}

// Fused prologue: qkv [B, S, (H + 2Hkv) * D] -> q_out [B, H, S, D] (rotated),
// key_cache[b, h, pos] (rotated), value_cache[b, h, pos] (copied).
//
// A CTA handles one token (blockIdx.x) and K * hpb of its heads (blockIdx.y
// picks which).  An item is VEC rotation pairs (chunk c) of one head: two
// 16-byte loads, at d and d + D/2.  The block has chunks * hpb threads;
// thread t owns chunk t % chunks of heads t / chunks + k * hpb (k < K), chunk
// fastest, so a warp reads contiguous qkv bytes and writes whole 128-byte
// lines of q / cache rows.  The thread issues its K item loads first, then
// reads the token's position and its chunk's four cos/sin vectors once for
// all K items: no per-item index division, no shared memory, no barrier.
constexpr int RA_THREADS = 256;  // block size at most (chunks * hpb)

template <typename T, typename TT, int VEC, int K>
__global__ void __launch_bounds__(RA_THREADS, 3) rope_kv_append_kernel(
    const T* __restrict__ qkv, const int64_t* __restrict__ positions, const TT* __restrict__ cosb,
    const TT* __restrict__ sinb, int64_t table_rows, T* __restrict__ q_out,
    T* __restrict__ kcache, T* __restrict__ vcache, int64_t seq, int num_heads, int num_kv_heads,
    int head_dim, int chunks, int hpb, int64_t max_batch, int64_t max_seq_len,
    const int64_t* __restrict__ seq_base, const int32_t* __restrict__ seq_cap, int64_t total_rows) {
  // launched with programmatic stream serialisation: the decode attention
  // after it may be scheduled now (it waits for this grid before reading the
  // cache), and this grid waits for the projection that wrote qkv
  lpc::pdl_trigger();
  lpc::pdl_wait();
  const int half = head_dim >> 1;
  const int heads_all = num_heads + 2 * num_kv_heads;
  const int64_t tok = blockIdx.x;  // b * seq + s
  const int c = (int)threadIdx.x % chunks;
  const int hh0 = (int)threadIdx.x / chunks + (int)blockIdx.y * K * hpb;
  const int d = c * VEC;
  const T* src = qkv + tok * (int64_t)heads_all * head_dim + d;
  uint4 x0[K], x1[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int hh = hh0 + k * hpb;
    if (hh < heads_all) {
      const T* p = src + (int64_t)hh * head_dim;
      x0[k] = __ldg(reinterpret_cast<const uint4*>(p));
      x1[k] = __ldg(reinterpret_cast<const uint4*>(p + half));
    }
  }
  const int64_t pos = __ldg(positions + tok);
  if (pos < 0) return;
  const int64_t b = tok / seq;
  // cache row of (b, kv head 0, pos) and the distance between kv heads:
  //   dense  [max_batch, Hkv, max_seq_len, D]: (b * Hkv) * max_seq_len + pos, max_seq_len
  //   ragged [Hkv, total_rows, D] (seq_base != nullptr): seq_base[b] + pos, total_rows
  int64_t row, head_rows;
  bool ok;
  if (seq_base == nullptr) {
    ok = pos < max_seq_len && b < max_batch;
    row = b * num_kv_heads * max_seq_len + pos;
    head_rows = max_seq_len;
  } else {
    const int64_t sb = __ldg(seq_base + b);
    const int64_t cap = __ldg(seq_cap + b);
    ok = sb >= 0 && pos < cap && sb + cap <= total_rows;
    row = sb + pos;
    head_rows = total_rows;
  }
  if (!ok || pos >= table_rows) {
    if (threadIdx.x == 0) atomicOr(&g_rope_status, LPC_DEV_ERR_BOUNDS);
    return;
  }
  const int rot_heads = num_heads + num_kv_heads;  // q and k heads come before v
  float c0[VEC], s0[VEC], c1[VEC], s1[VEC];
  if (hh0 < rot_heads) {  // the thread's first head is its lowest
    const TT* cr = cosb + pos * (int64_t)head_dim;
    const TT* sr = sinb + pos * (int64_t)head_dim;
    load_f<TT, VEC>(cr + d, c0);
    load_f<TT, VEC>(sr + d, s0);
    load_f<TT, VEC>(cr + d + half, c1);
    load_f<TT, VEC>(sr + d + half, s1);
  }
  const int64_t q_row = (b * num_heads) * seq + (tok - b * seq);  // q_out row of (b, head 0, s)
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int hh = hh0 + k * hpb;
    if (hh >= heads_all) continue;
    if (hh >= rot_heads) {  // V: plain copy into the cache
      T* dst = vcache + (row + (int64_t)(hh - rot_heads) * head_rows) * head_dim;
      reinterpret_cast<uint4*>(dst + d)[0] = x0[k];
      reinterpret_cast<uint4*>(dst + d + half)[0] = x1[k];
      continue;
    }
    float a0[VEC], a1[VEC];
    {
      const T* e0 = reinterpret_cast<const T*>(&x0[k]);
      const T* e1 = reinterpret_cast<const T*>(&x1[k]);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        a0[i] = Num<T>::to_f(e0[i]);
        a1[i] = Num<T>::to_f(e1[i]);
      }
    }
    float o0[VEC], o1[VEC];
    rotate<VEC>(a0, a1, c0, s0, c1, s1, o0, o1);
    T* dst = hh < num_heads ? q_out + (q_row + (int64_t)hh * seq) * head_dim
                            : kcache + (row + (int64_t)(hh - num_heads) * head_rows) * head_dim;
    store_f<T, VEC>(dst + d, o0);
    store_f<T, VEC>(dst + d + half, o1);
  }
}

template <typename T, typename TT>
int launch_rope(void* q, void* k, const void* cosb, const void* sinb, const int64_t* pos,
                int64_t num_tokens, int num_heads, int num_kv_heads, int head_dim, int table_mode,
                int64_t table_rows, bool vec_ok, cudaStream_t s) {
  constexpr int VEC = 16 / (int)sizeof(T);
  const int heads_all = num_heads + num_kv_heads;
  const int threads = 256;
  if (vec_ok) {
    const int64_t work = num_tokens * heads_all * (head_dim / 2 / VEC);
    rope_kernel<T, TT, VEC><<<(unsigned)((work + threads - 1) / threads), threads, 0, s>>>(
        (T*)q, (T*)k, (const TT*)cosb, (const TT*)sinb, pos, num_tokens, num_heads, num_kv_heads,
        head_dim, table_mode, table_rows);
  } else {
    const int64_t work = num_tokens * heads_all * (head_dim / 2);
    rope_kernel<T, TT, 1><<<(unsigned)((work + threads - 1) / threads), threads, 0, s>>>(
        (T*)q, (T*)k, (const TT*)cosb, (const TT*)sinb, pos, num_tokens, num_heads, num_kv_heads,
        head_dim, table_mode, table_rows);
  }
  return lpc::check_launch("rope_forward");
}

template <typename T>
int launch_rope_t(int table_dtype, void* q, void* k, const void* c, const void* sn,
                  const int64_t* pos, int64_t n, int h, int hkv, int d, int mode, int64_t rows,
                  bool vec_ok, cudaStream_t s) {
  switch (table_dtype) {
    case LPC_DTYPE_F32: return launch_rope<T, float>(q, k, c, sn, pos, n, h, hkv, d, mode, rows, vec_ok, s);
    case LPC_DTYPE_BF16: return launch_rope<T, __nv_bfloat16>(q, k, c, sn, pos, n, h, hkv, d, mode, rows, vec_ok, s);
    case LPC_DTYPE_F16: return launch_rope<T, __half>(q, k, c, sn, pos, n, h, hkv, d, mode, rows, vec_ok, s);
  }
  lpc::set_error("rope_forward: unsupported table dtype %d", table_dtype);
  return LPC_ERR_UNSUPPORTED;
}

template <typename T, typename TT, int K>
cudaError_t launch_fused_k(dim3 grid, int threads, const void* qkv, const int64_t* positions,
                    const void* c, const void* sn, int64_t rows, void* q_out, void* kc, void* vc,
                    int64_t seq, int h, int hkv, int d, int chunks, int hpb, int64_t max_batch,
                    int64_t max_seq, const int64_t* seq_base, const int32_t* seq_cap,
                    int64_t total_rows, cudaStream_t s) {
  constexpr int VEC = 16 / (int)sizeof(T);
  static const bool pdl = [] {
    const char* e = getenv("LPC_PDL");
    return !(e && e[0] == '0');
  }();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rope_kv_append_kernel<T, TT, VEC, K>, (const T*)qkv, positions,
                     (const TT*)c, (const TT*)sn, rows, (T*)q_out, (T*)kc, (T*)vc, seq, h, hkv, d,
                     chunks, hpb, max_batch, max_seq, seq_base, seq_cap, total_rows);
}

template <typename T, typename TT>
int launch_fused(const void* qkv, const int64_t* positions, const void* c, const void* sn,
                 int64_t rows, void* q_out, void* kc, void* vc, int64_t batch, int64_t seq, int h,
                 int hkv, int d, int64_t max_batch, int64_t max_seq, const int64_t* seq_base,
                 const int32_t* seq_cap, int64_t total_rows, cudaStream_t s) {
  constexpr int VEC = 16 / (int)sizeof(T);
  const int64_t tokens = batch * seq;
  if (tokens == 0) return LPC_OK;
  const int chunks = d / 2 / VEC;
  const int heads_all = h + 2 * hkv;
  if (chunks > RA_THREADS || tokens > 0x7fffffffLL) {
    lpc::set_error("rope_kv_append: unsupported shape (tokens=%lld dim=%d)", (long long)tokens, d);
    return LPC_ERR_UNSUPPORTED;
  }
  const int hpb = RA_THREADS / chunks;  // heads per k step
  const int steps = (heads_all + hpb - 1) / hpb;
  const int K = steps < 4 ? steps : 4;
  const dim3 grid((unsigned)tokens, (unsigned)((heads_all + K * hpb - 1) / (K * hpb)));
  const int threads = chunks * hpb;
#define LPC_RA(KK)                                                                                 \
  launch_fused_k<T, TT, KK>(grid, threads, qkv, positions, c, sn, rows, q_out, kc, vc, seq, h, hkv, \
                            d, chunks, hpb, max_batch, max_seq, seq_base, seq_cap, total_rows, s)
  const cudaError_t e = K == 1 ? LPC_RA(1) : K == 2 ? LPC_RA(2) : K == 3 ? LPC_RA(3) : LPC_RA(4);
  if (e != cudaSuccess) {
    lpc::set_error("rope_kv_append: launch failed: %s", cudaGetErrorString(e));
    return LPC_ERR_CUDA;
  }
#undef LPC_RA
  return lpc::check_launch("rope_kv_append");
}

}  // namespace

extern "C" int lpc_rope_forward(void* q, void* k, const void* cos, const void* sin,
                                const int64_t* position_ids, int64_t num_tokens, int num_heads,
                                int num_kv_heads, int head_dim, int table_mode, int64_t table_rows,
                                int q_dtype, int table_dtype, void* stream) {
  using namespace lpc;
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads < 0 || head_dim <= 0 || head_dim % 2) {
    set_error("rope_forward: invalid sizes (tokens=%lld heads=%d kv_heads=%d dim=%d)",
              (long long)num_tokens, num_heads, num_kv_heads, head_dim);
    return LPC_ERR_INVALID;
  }
  if (table_mode != 0 && table_mode != 1) {
    set_error("rope_forward: table_mode must be 0 or 1");
    return LPC_ERR_INVALID;
  }
  if (num_tokens == 0) return LPC_OK;
  if (!q || !cos || !sin || (num_kv_heads > 0 && !k)) {
    set_error("rope_forward: null pointer");
    return LPC_ERR_INVALID;
  }
  const int es = dtype_size(q_dtype), ts = dtype_size(table_dtype);
  if (!es || !ts) {
    set_error("rope_forward: unsupported dtype (q=%d table=%d)", q_dtype, table_dtype);
    return LPC_ERR_UNSUPPORTED;
  }
  const int vec = 16 / es;
  const int half = head_dim / 2;
  const int64_t table_row_elems = table_mode == 0 ? half : head_dim;
  bool vec_ok = (half % vec == 0) && aligned16(q) && (num_kv_heads == 0 || aligned16(k)) &&
                aligned16(cos) && aligned16(sin) && ((int64_t)head_dim * es) % 16 == 0 &&
                (table_row_elems * ts) % 16 == 0 && ((int64_t)vec * ts) % 16 == 0 &&
                ((int64_t)half * ts) % 16 == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (q_dtype) {
    case LPC_DTYPE_F32: return launch_rope_t<float>(table_dtype, q, k, cos, sin, position_ids, num_tokens, num_heads, num_kv_heads, head_dim, table_mode, table_rows, vec_ok, s);
    case LPC_DTYPE_BF16: return launch_rope_t<__nv_bfloat16>(table_dtype, q, k, cos, sin, position_ids, num_tokens, num_heads, num_kv_heads, head_dim, table_mode, table_rows, vec_ok, s);
    case LPC_DTYPE_F16: return launch_rope_t<__half>(table_dtype, q, k, cos, sin, position_ids, num_tokens, num_heads, num_kv_heads, head_dim, table_mode, table_rows, vec_ok, s);
  }
  return LPC_ERR_UNSUPPORTED;
}

namespace {

int rope_kv_append_common(const void* qkv, const int64_t* positions, const void* cos,
                          const void* sin, int64_t table_rows, void* q_out, void* key_cache,
                          void* value_cache, int64_t batch, int64_t seq, int num_heads,
                          int num_kv_heads, int head_dim, int64_t max_batch, int64_t max_seq_len,
                          const int64_t* seq_base, const int32_t* seq_cap, int64_t total_rows,
                          int dtype, int table_dtype, void* stream) {
  using namespace lpc;
  if (!qkv || !positions || !cos || !sin || !q_out || !key_cache || !value_cache) {
    set_error("rope_kv_append: null pointer");
    return LPC_ERR_INVALID;
  }
  const int es = dtype_size(dtype), ts = dtype_size(table_dtype);
  if (dtype == LPC_DTYPE_F32 || !es || !ts) {
    set_error("rope_kv_append: needs bf16/fp16 activations (got dtype %d, table %d)", dtype,
              table_dtype);
    return LPC_ERR_UNSUPPORTED;
  }
  const int vec = 16 / es;
  if ((head_dim / 2) % vec || !aligned16(qkv) || !aligned16(q_out) || !aligned16(key_cache) ||
      !aligned16(value_cache) || !aligned16(cos) || !aligned16(sin) ||
      ((int64_t)head_dim * ts) % 16 || ((int64_t)vec * ts) % 16) {
    set_error("rope_kv_append: head_dim/alignment not supported by the 16-byte vector path");
    return LPC_ERR_UNSUPPORTED;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define LPC_FUSED(T, TT)                                                                        \
  return launch_fused<T, TT>(qkv, positions, cos, sin, table_rows, q_out, key_cache, value_cache, \
                             batch, seq, num_heads, num_kv_heads, head_dim, max_batch,           \
                             max_seq_len, seq_base, seq_cap, total_rows, s)
  if (dtype == LPC_DTYPE_BF16) {
    if (table_dtype == LPC_DTYPE_BF16) LPC_FUSED(__nv_bfloat16, __nv_bfloat16);
    if (table_dtype == LPC_DTYPE_F32) LPC_FUSED(__nv_bfloat16, float);
  } else {
    if (table_dtype == LPC_DTYPE_F16) LPC_FUSED(__half, __half);
    if (table_dtype == LPC_DTYPE_F32) LPC_FUSED(__half, float);
  }
#undef LPC_FUSED
  set_error("rope_kv_append: table dtype must match activations or be fp32");
  return LPC_ERR_UNSUPPORTED;
}

}  // namespace

extern "C" int lpc_rope_kv_append(const void* qkv, const int64_t* positions, const void* cos,
                                  const void* sin, int64_t table_rows, void* q_out,
                                  void* key_cache, void* value_cache, int64_t batch, int64_t seq,
                                  int num_heads, int num_kv_heads, int head_dim,
                                  int64_t max_batch, int64_t max_seq_len, int dtype,
                                  int table_dtype, void* stream) {
  using namespace lpc;
  if (batch < 0 || seq < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      max_batch <= 0 || max_seq_len <= 0 || table_rows <= 0) {
    set_error("rope_kv_append: invalid sizes");
    return LPC_ERR_INVALID;
  }
  if (batch == 0 || seq == 0) return LPC_OK;
  if (batch > max_batch) {
    set_error("rope_kv_append: batch %lld exceeds cache capacity %lld", (long long)batch,
              (long long)max_batch);
    return LPC_ERR_INVALID;
  }
  return rope_kv_append_common(qkv, positions, cos, sin, table_rows, q_out, key_cache, value_cache,
                               batch, seq, num_heads, num_kv_heads, head_dim, max_batch,
                               max_seq_len, nullptr, nullptr, 0, dtype, table_dtype, stream);
}

extern "C" int lpc_rope_kv_append_ragged(const void* qkv, const int64_t* positions,
                                         const void* cos, const void* sin, int64_t table_rows,
                                         void* q_out, void* key_cache, void* value_cache,
                                         const int64_t* seq_base, const int32_t* seq_cap,
                                         int64_t batch, int64_t seq, int num_heads,
                                         int num_kv_heads, int head_dim, int64_t total_rows,
                                         int dtype, int table_dtype, void* stream) {
  using namespace lpc;
  if (batch < 0 || seq < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      total_rows <= 0 || table_rows <= 0) {
    set_error("rope_kv_append_ragged: invalid sizes");
    return LPC_ERR_INVALID;
  }
  if (batch == 0 || seq == 0) return LPC_OK;
  if (!seq_base || !seq_cap) {
    set_error("rope_kv_append_ragged: seq_base and seq_cap are required");
    return LPC_ERR_INVALID;
  }
  return rope_kv_append_common(qkv, positions, cos, sin, table_rows, q_out, key_cache, value_cache,
                               batch, seq, num_heads, num_kv_heads, head_dim, batch, 1, seq_base,
                               seq_cap, total_rows, dtype, table_dtype, stream);
}
