// Weight-streaming GEMM for decode-sized token counts (<= 256 tokens) on
// pre-packed weights.
//
//   out[t, n] = epilogue( sum_k X[t, k] * W[n, k] )
//
// A decode step multiplies a few dozen to a few hundred token rows by weight
// matrices that are read once per step: the product is a stream of weight
// bytes from HBM.
//   * Weights are packed once (lpc_pack_weights) into 16 KB chunks, one per
//     128-row x 64-k tile, each already laid out as the 128-byte-swizzled
//     K-major shared-memory image the tcgen05 MMA reads; a chunk is one
//     cp.async.bulk copy of contiguous bytes, and the chunks of one tile are
//     consecutive in memory.
//   * Weights are the MMA's M operand (128 rows), tokens its N (padded to 16):
//     a pipeline stage is 16 KB of weights plus NT * 128 bytes of
//     activations, and two ~100 KB CTAs fit per SM, so a layer with up to
//     ~300 weight tiles keeps every tile streaming at once.
//   * One CTA per weight tile over the whole K when there are enough tiles;
//     layers with few tiles split K over clusters of up to 8 CTAs whose fp32
//     partial tiles are reduce-scattered through distributed shared memory.
//   * Launched with programmatic stream serialisation: the first weight
//     chunks stream in under the previous kernel on the stream.
// Measured on B200 in steady state (launches back to back over weights larger
// than L2), SwiGLU gate/up of the 7B layer (2 x 11008 x 4096): 30.0 us at 32
// tokens, 32.4 us at 64, 38.9 us at 128 -- against 44-46 us for the
// activation-major tile of the fused rmsswiglu op on the raw weights; the
// q/k/v projection with RoPE and KV append (EPI_QKV): 21.2 / 21.5 / 23.0 us
// at 8 / 16 / 32 tokens against 24.7 / 26.8 / 27.0 for cuBLAS followed by
// lpc_rope_kv_append.
// Epilogues: plain store, residual add (out = resid + acc, may alias), SwiGLU
// on weights packed with 16 gate rows / 16 up rows interleaved, and EPI_QKV on
// the "heads" packing.
//   warp 0    producer: bulk copy of the weight chunk + TMA box of activations
//   warp 2    TMEM allocator + single-thread tcgen05.mma issuer
//   warps 4-7 epilogue (TMEM lane = weight row)
#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "lpc_common.cuh"

LPC_DECLARE_STATUS(g_ws_status)

unsigned int lpc_status_wsgemm(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_ws_status, sizeof(v));
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_ws_status, &z, sizeof(z));
  }
  return v;
}

namespace {

using lpc::Num;

constexpr int TILE_ROWS = 128;
constexpr int KB = 64;                        // k per chunk: 64 x 2 B = one swizzle row
constexpr int CHUNK = TILE_ROWS * KB * 2;     // 16 KB
constexpr int THREADS = 256;
constexpr int MAX_TOKENS = 256;
constexpr int SMEM_TARGET = 100 * 1024;       // two CTAs per SM

enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };
constexpr int HEAD_DIM = TILE_ROWS;  // EPI_QKV: one 128-row weight tile per head

// EPI_QKV: the attention block's projection epilogue (RoPE + KV append).
// Token t = b * seq + s sits at positions[t]; q goes to q_out [B, H, seq, D],
// k and v to the cache row of (b, pos): dense [max_batch, Hkv, max_seq, D]
// (seq_base == nullptr) or ragged [Hkv, total_rows, D] at seq_base[b] + pos.
struct QkvArgs {
  const int64_t* positions;
  const void* cosb;  // [table_rows, D], the data dtype
  const void* sinb;
  int64_t table_rows;
  void* q_out;
  void* kc;
  void* vc;
  const int64_t* seq_base;
  const int32_t* seq_cap;
  int64_t seq, max_batch, max_seq, total_rows;
  int H, Hkv;
};

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// Sum of squares of the 8 elements of a 16-byte chunk (fixed order).
template <typename T>
__device__ __forceinline__ float sumsq8(const uint4& u);
template <>
__device__ __forceinline__ float sumsq8<__nv_bfloat16>(const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = lpc::bf16lo(w[i]), b = lpc::bf16hi(w[i]);
    s = fmaf(a, a, s);
    s = fmaf(b, b, s);
  }
  return s;
}
template <>
__device__ __forceinline__ float sumsq8<__half>(const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    s = fmaf(f.x, f.x, s);
    s = fmaf(f.y, f.y, s);
  }
  return s;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float r;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(r) : "r"(addr) : "memory");
  return r;
}

// ---------------------------------------------------------------------------
// Packing: packed[tile][kb] = swizzled image of rows tile*128.. x k kb*64..
// layout 0: row r of W0 (rows >= n_rows are zero)
// layout 1 (SwiGLU): tile tau covers inter columns 64*tau..; tile row
//   32q + l is gate row 64*tau + 16q + l (l < 16) or up row 64*tau + 16q + l-16;
//   gate rows from W0, up rows from W1 (or W0 rows n_rows.. when W1 is null).
// layout 2 (heads): tile tau is rows 128*tau .. 128*tau+127 of W0 (one
//   attention head), tile row 32q + l holding head dim 16q + l (l < 16) or
//   64 + 16q + (l - 16): the rotate-half partners d and d + 64 sit in lanes
//   l and l^16 of one epilogue warp.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) pack_kernel(const T* __restrict__ w0,
                                                   const T* __restrict__ w1,
                                                   const float* __restrict__ kscale,
                                                   uint4* __restrict__ packed, int64_t n_rows,
                                                   int K, int n_tiles, int layout) {
  const int n_kb = K / KB;
  const int64_t total = (int64_t)n_tiles * n_kb * (CHUNK / 16);
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(idx % (CHUNK / 16));  // 16-byte slot in the image
    const int64_t tk = idx / (CHUNK / 16);
    const int kb = (int)(tk % n_kb);
    const int tile = (int)(tk / n_kb);
    const int r8 = p >> 6, rem = p & 63, rr = rem >> 3, cs = rem & 7;
    const int r = r8 * 8 + rr;       // tile row
    const int c = cs ^ rr;           // logical 16-byte chunk along k (128B swizzle)
    const int k = kb * KB + c * 8;
    const T* src = nullptr;
    if (layout == 0 || layout == 2) {
      int d = r;
      if (layout == 2) {
        const int q = r >> 5, l = r & 31;
        d = l < 16 ? 16 * q + l : 64 + 16 * q + (l - 16);
      }
      const int64_t row = (int64_t)tile * TILE_ROWS + d;
      if (row < n_rows) src = w0 + row * K + k;
    } else {
      const int q = r >> 5, l = r & 31;
      const int64_t col = (int64_t)tile * 64 + 16 * q + (l & 15);
      if (col < n_rows) {
        if (l < 16) src = w0 + col * K + k;
        else src = w1 ? w1 + col * K + k : w0 + (n_rows + col) * K + k;
      }
    }
    uint4 v = src ? *reinterpret_cast<const uint4*>(src) : make_uint4(0, 0, 0, 0);
    if (src && kscale) {
      // W[n, k] * scale[k] in fp32, one rounding (an RMSNorm weight folded
      // into the projection that consumes the normalised rows)
      T* e = reinterpret_cast<T*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = Num<T>::from_f(Num<T>::to_f(e[j]) * __ldg(kscale + k + j));
    }
    packed[idx] = v;
  }
}

// ---------------------------------------------------------------------------
// GEMM: one CTA per weight tile
// ---------------------------------------------------------------------------
// Epilogue of CNT accumulator columns (tokens c .. c+CNT-1) of this thread's
// tile row (CNT in {4, 8, 16}).
// EPI_QKV per-token entry, built in shared memory by the epilogue warps while
// the main loop runs: q offset of head 0, cache row of kv head 0, position,
// and whether the token is written (0), skipped (1: negative position or an
// out-of-range row, the latter flagged once here).
struct TokSlot {
  int64_t qbase;
  int64_t kvrow;
  int32_t pos;
  int32_t state;
};
constexpr int TOK_TABLE_BYTES = MAX_TOKENS * (int)sizeof(TokSlot);

__device__ __forceinline__ void build_token_table(TokSlot* tab, const QkvArgs& qa, int M, int tid) {
  for (int t = tid; t < M; t += 128) {
    const int64_t b = t / qa.seq;
    const int64_t sidx = t - b * qa.seq;
    const int64_t pos = __ldg(qa.positions + t);
    TokSlot e;
    e.qbase = (b * qa.H * qa.seq + sidx) * HEAD_DIM;
    e.kvrow = 0;
    e.pos = 0;
    e.state = 1;
    if (pos >= 0) {
      int64_t row;
      bool ok;
      if (qa.seq_base == nullptr) {
        ok = pos < qa.max_seq && b < qa.max_batch;
        row = b * qa.Hkv * qa.max_seq + pos;
      } else {
        const int64_t sb = __ldg(qa.seq_base + b);
        const int64_t cap = __ldg(qa.seq_cap + b);
        ok = sb >= 0 && pos < cap && sb + cap <= qa.total_rows;
        row = sb + pos;
      }
      if (!ok || pos >= qa.table_rows) {
        atomicOr(&g_ws_status, LPC_DEV_ERR_BOUNDS);
      } else {
        e.kvrow = row;
        e.pos = (int32_t)pos;
        e.state = 0;
      }
    }
    tab[t] = e;
  }
}

// Values the epilogue of CNT token columns needs from global memory, loaded
// before the accumulators they are combined with (so the two latencies
// overlap): the residual (EPI_RESIDUAL) or the cos/sin entries of this
// thread's head dim (EPI_QKV, rotated heads).
template <int CNT>
struct EpiPre {
  float a[CNT];
  float b[CNT];
};

// EPI_QKV: row r = 32q + l of a head tile is head dim 16q + l (l < 16) or
// 64 + 16q + (l - 16), so lanes l and l^16 hold a rotate-half pair.
__device__ __forceinline__ int qkv_dim(int q, int lane) {
  return lane < 16 ? 16 * q + lane : 64 + 16 * q + (lane - 16);
}

template <typename T, int EPI, int CNT>
__device__ __forceinline__ void epi_prefetch(EpiPre<CNT>& pre, const T* resid, int M, int n_out,
                                             int tile, int q, int lane, int c, const QkvArgs& qa,
                                             const TokSlot* tab) {
  if (EPI == EPI_RESIDUAL) {
    const int n = tile * TILE_ROWS + 32 * q + lane;
#pragma unroll
    for (int i = 0; i < CNT; ++i)
      pre.a[i] = (n < n_out && c + i < M) ? Num<T>::to_f(resid[(int64_t)(c + i) * n_out + n]) : 0.f;
  } else if (EPI == EPI_QKV) {
    if (tile < qa.H + qa.Hkv) {
      const int d = qkv_dim(q, lane);
      const T* cosb = static_cast<const T*>(qa.cosb);
      const T* sinb = static_cast<const T*>(qa.sinb);
#pragma unroll
      for (int i = 0; i < CNT; ++i) {
        const int64_t p = c + i < M ? (int64_t)tab[c + i].pos : 0;  // row 0 exists
        pre.a[i] = Num<T>::to_f(__ldg(cosb + p * HEAD_DIM + d));
        pre.b[i] = Num<T>::to_f(__ldg(sinb + p * HEAD_DIM + d));
      }
    }
  }
}

// EPI_QKV for CNT tokens of one head tile: the accumulator is first rounded to
// the data dtype (the projection's output), then rotated with every product
// and the sum rounded separately, as lpc_rope_kv_append does.
template <typename T, int CNT>
__device__ __forceinline__ void emit_qkv(const float (&v)[CNT], const EpiPre<CNT>& pre,
                                         const QkvArgs& qa, const TokSlot* tab, int M, int hh,
                                         int q, int lane, int c) {
  const bool lo = lane < 16;
  const int d = qkv_dim(q, lane);
  const bool rot = hh < qa.H + qa.Hkv;
  float x[CNT], partner[CNT];
#pragma unroll
  for (int i = 0; i < CNT; ++i) x[i] = Num<T>::to_f(Num<T>::from_f(v[i]));
#pragma unroll
  for (int i = 0; i < CNT; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, x[i], 16);
  const int64_t head_rows = qa.seq_base == nullptr ? qa.max_seq : qa.total_rows;
  T* base;
  if (hh < qa.H) {
    base = static_cast<T*>(qa.q_out) + (int64_t)hh * qa.seq * HEAD_DIM;
  } else if (rot) {
    base = static_cast<T*>(qa.kc) + (int64_t)(hh - qa.H) * head_rows * HEAD_DIM;
  } else {
    base = static_cast<T*>(qa.vc) + (int64_t)(hh - qa.H - qa.Hkv) * head_rows * HEAD_DIM;
  }
#pragma unroll
  for (int i = 0; i < CNT; ++i) {
    const int t = c + i;
    if (t >= M) continue;
    const TokSlot e = tab[t];
    if (e.state != 0) continue;
    float val = x[i];
    if (rot)
      val = lo ? __fsub_rn(__fmul_rn(x[i], pre.a[i]), __fmul_rn(partner[i], pre.b[i]))
               : __fadd_rn(__fmul_rn(x[i], pre.a[i]), __fmul_rn(partner[i], pre.b[i]));
    T* dst = hh < qa.H ? base + e.qbase : base + e.kvrow * HEAD_DIM;
    dst[d] = Num<T>::from_f(val);
  }
}

// Epilogue of CNT accumulator columns (tokens c .. c+CNT-1) of this thread's
// tile row (CNT in {4, 8, 16}); `pre` from epi_prefetch on the same columns.
template <typename T, int EPI, int CNT>
__device__ __forceinline__ void emit(float (&v)[CNT], const EpiPre<CNT>& pre, T* out,
                                     int M, int n_out, int tile, int q, int lane, int c,
                                     const QkvArgs& qa, const TokSlot* tab, const float* rt) {
  if (rt) {
    // fused RMSNorm: the accumulator holds x . (W * w); scale by the token
    // row's rsqrt(mean(x^2) + eps)
#pragma unroll
    for (int i = 0; i < CNT; ++i) v[i] *= rt[c + i];
  }
  if (EPI == EPI_QKV) {
    emit_qkv<T, CNT>(v, pre, qa, tab, M, tile, q, lane, c);
  } else if (EPI == EPI_SWIGLU) {
    // lanes l and l^16 hold the gate and up rows of one inter column; the gate
    // lane writes the first CNT/2 tokens, the up lane the others
    constexpr int H = CNT / 2;
    const bool is_gate = lane < 16;
    const int col = tile * 64 + 16 * q + (lane & 15);
    float o[H];
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const float olo = __shfl_xor_sync(0xffffffffu, v[i], 16);
      const float ohi = __shfl_xor_sync(0xffffffffu, v[H + i], 16);
      o[i] = is_gate ? silu_mul(v[i], olo) : silu_mul(ohi, v[H + i]);
    }
    const int tok0 = c + (is_gate ? 0 : H);
    if (col < n_out) {
#pragma unroll
      for (int i = 0; i < H; ++i)
        if (tok0 + i < M) out[(int64_t)(tok0 + i) * n_out + col] = Num<T>::from_f(o[i]);
    }
  } else {
    const int n = tile * TILE_ROWS + 32 * q + lane;  // output column of this lane
    if (n < n_out) {
#pragma unroll
      for (int i = 0; i < CNT; ++i) {
        const int t = c + i;
        if (t < M) {
          float a = v[i];
          if (EPI == EPI_RESIDUAL) a += pre.a[i];
          out[(int64_t)t * n_out + n] = Num<T>::from_f(a);
        }
      }
    }
  }
}

__device__ __forceinline__ float4 ld_cluster_v4(uint32_t addr) {
  float4 r;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "r"(addr)
               : "memory");
  return r;
}

// Split-k reduce-scatter of one tile row: token columns [c0, c0 + width) of
// this rank's slice, in chunks of C, each summed over the S ranks' partial
// rows (rank order, so every column is p0 + p1 + ... whichever rank reduces
// it) and sent through the epilogue.  Per chunk the epilogue's global loads
// and the C/4 x S distributed-shared-memory loads are all issued before any
// is used: one round trip per chunk.
template <typename T, int EPI, int S, int C>
__device__ __forceinline__ void reduce_slice(uint32_t prow, int swz, int c0, int width, T* out,
                                             const T* resid, int M, int n_out, int tile, int q,
                                             int lane, const QkvArgs& qa, const TokSlot* tab,
                                             const float* rt) {
  constexpr int G = C / 4;
  uint32_t peer[S];
#pragma unroll
  for (int k = 0; k < S; ++k) peer[k] = lpc::mapa_shared(prow, (uint32_t)k);
#pragma unroll 1
  for (int c = c0; c < c0 + width; c += C) {
    EpiPre<C> pre;
    epi_prefetch<T, EPI, C>(pre, resid, M, n_out, tile, q, lane, c, qa, tab);
    float4 buf[G][S];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint32_t off = (uint32_t)((((c >> 2) + g) ^ swz) * 16);
#pragma unroll
      for (int k = 0; k < S; ++k) buf[g][k] = ld_cluster_v4(peer[k] + off);
    }
    float v[C];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      v[4 * g] = buf[g][0].x;
      v[4 * g + 1] = buf[g][0].y;
      v[4 * g + 2] = buf[g][0].z;
      v[4 * g + 3] = buf[g][0].w;
#pragma unroll
      for (int k = 1; k < S; ++k) {
        v[4 * g] += buf[g][k].x;
        v[4 * g + 1] += buf[g][k].y;
        v[4 * g + 2] += buf[g][k].z;
        v[4 * g + 3] += buf[g][k].w;
      }
    }
    emit<T, EPI, C>(v, pre, out, M, n_out, tile, q, lane, c, qa, tab, rt);
  }
}

// Chunk width for S ranks and a slice of `width` columns: the largest of
// 16 / 8 / 4 that divides the slice with C * S <= 32 registers of partials.
template <typename T, int EPI, int S>
__device__ __forceinline__ void reduce_slice_any(uint32_t prow, int swz, int c0, int width,
                                                 T* out, const T* resid, int M, int n_out,
                                                 int tile, int q, int lane, const QkvArgs& qa,
                                                 const TokSlot* tab, const float* rt) {
  if constexpr (S <= 2) {
    if (width % 16 == 0) {
      reduce_slice<T, EPI, S, 16>(prow, swz, c0, width, out, resid, M, n_out, tile, q, lane, qa, tab, rt);
      return;
    }
  }
  if constexpr (S <= 4) {
    if (width % 8 == 0) {
      reduce_slice<T, EPI, S, 8>(prow, swz, c0, width, out, resid, M, n_out, tile, q, lane, qa, tab, rt);
      return;
    }
  }
  reduce_slice<T, EPI, S, 4>(prow, swz, c0, width, out, resid, M, n_out, tile, q, lane, qa, tab, rt);
}

// splits > 1: the kernel runs in clusters of `splits` CTAs, one weight tile
// per cluster; CTA rank k takes k-blocks [k*nkb/splits, (k+1)*nkb/splits).
// Once its MMAs are done every rank writes its fp32 partial tile into its own
// (now idle) pipeline shared memory; after a cluster barrier rank k sums
// token columns [k*NT/splits, (k+1)*NT/splits) over all ranks through
// distributed shared memory and runs the epilogue on them.  A second cluster
// barrier keeps every CTA's shared memory alive until all slices are read.
// No atomics, no global workspace.
//
// NORM: the activations are the raw rows x of an RMSNorm whose weight is
// folded into the packed weights (lpc_pack_weights' k_scale).  The epilogue
// warps, idle during the main loop, read this rank's k-range of every token
// row from global memory (L2) and sum its squares; the split ranks add their
// partial sums through distributed shared memory, and the epilogue multiplies
// each token's accumulators by rsqrt(sum / K + eps):
// norm(x) W^T = rsqrt(mean(x^2) + eps) * (x (W diag(w))^T).
// (Summing the shared-memory activation tiles instead, which the tensor core
// reads through the async proxy, slowed the main loop by half.)
template <typename T, int EPI, bool NORM>
__global__ void __launch_bounds__(THREADS, 2)
    wsgemm_kernel(const __grid_constant__ lpc::TmaDesc tmX, const T* __restrict__ xg,
                  const uint8_t* __restrict__ packed,
                  T* out, const T* resid, int M, int K, int n_out, int NT, int stages,
                  uint32_t tmem_cols, uint32_t idesc, int splits, const QkvArgs qa, float eps) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = lpc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t x_bytes = (uint32_t)NT * KB * 2;
  const uint32_t stage_bytes = CHUNK + ((x_bytes + 1023u) & ~1023u);
  const uint32_t bars = base + (uint32_t)stages * stage_bytes;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (stages + s); };
  const uint32_t accum = bars + 8u * (2 * stages);
  const uint32_t tmem_slot = accum + 16u;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));
  // EPI_QKV token table (TOK_TABLE_BYTES past the barriers), then for NORM
  // the per-token sums of squares and row scales (MAX_TOKENS floats each)
  TokSlot* tab = reinterpret_cast<TokSlot*>(smem_raw + (tmem_slot + 8u - raw));
  const uint32_t ssq_addr = tmem_slot + 8u + (EPI == EPI_QKV ? (uint32_t)TOK_TABLE_BYTES : 0u);
  float* ssq = reinterpret_cast<float*>(smem_raw + (ssq_addr - raw));
  float* rt = ssq + MAX_TOKENS;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = (int)blockIdx.x / splits;
  const int rank = (int)blockIdx.x - tile * splits;  // == %cluster_ctarank for splits > 1
  const int nkb_all = K / KB;
  const int kb0 = (int)((int64_t)rank * nkb_all / splits);
  const int nkb = (int)((int64_t)(rank + 1) * nkb_all / splits) - kb0;
  const uint8_t* wsrc = packed + ((int64_t)tile * nkb_all + kb0) * CHUNK;
  unsigned int* st = &g_ws_status;
  auto load_w = [&](int i) {
    const int s = i % stages;
    lpc::mbar_arrive_expect_tx(full_bar(s), CHUNK + x_bytes);
    lpc::bulk_g2s(base + (uint32_t)s * stage_bytes, wsrc + (int64_t)i * CHUNK, CHUNK, full_bar(s));
  };
  auto load_x = [&](int i) {
    const int s = i % stages;
    lpc::tma_load_2d(base + (uint32_t)s * stage_bytes + CHUNK, &tmX, (kb0 + i) * KB, 0,
                     full_bar(s));
  };
  const int first = nkb < stages ? nkb : stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      lpc::mbar_init(full_bar(s), 1);
      lpc::mbar_init(empty_bar(s), 1);
    }
    lpc::mbar_init(accum, 1);
    lpc::fence_mbar_init();
    lpc::tma_prefetch_desc(&tmX);
    // The first round of stages needs no empty-slot wait, and the packed
    // weights are never written by the grids this one may overlap (the pack
    // call completes before returning): start streaming them before the
    // TMEM allocation, the block barrier and the wait on the previous grid.
    for (int i = 0; i < first; ++i) load_w(i);
    lpc::pdl_wait();  // activations, residual and output belong to earlier grids
    for (int i = 0; i < first; ++i) load_x(i);
  }
  __syncwarp();
  if (warp == 2) {
    lpc::tmem_alloc(tmem_slot, tmem_cols);
    lpc::tmem_relinquish();
  }
  lpc::tc_fence_before();
  __syncthreads();
  lpc::tc_fence_after();
  lpc::pdl_wait();
  const uint32_t tmem = *tmem_slot_ptr;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = first; i < nkb; ++i) {
        if (!lpc::mbar_wait(empty_bar(i % stages), ((uint32_t)(i / stages) & 1u) ^ 1u, st)) break;
        load_w(i);
        load_x(i);
      }
      // every load of this CTA is issued and its TMEM is allocated: the next
      // grid may start its prologue
      lpc::pdl_trigger();
    }
  } else if (warp == 2) {
    if (lane == 0) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        if (!lpc::mbar_wait(full_bar(s), (uint32_t)(i / stages) & 1u, st)) break;
        lpc::tc_fence_after();
        const uint32_t sb = base + (uint32_t)s * stage_bytes;
        const uint64_t ad = lpc::smem_desc_sw128(sb, 16, 1024);
        const uint64_t bd = lpc::smem_desc_sw128(sb + CHUNK, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < KB / 16; ++kk)
          lpc::umma_ss(tmem, ad + 2u * kk, bd + 2u * kk, idesc, (i | kk) != 0);
        lpc::umma_commit(empty_bar(s));
      }
      lpc::umma_commit(accum);
    }
  }
  __syncwarp();

  if (warp >= 4) {
    const int q = warp & 3;  // TMEM lane quadrant = tile rows 32q .. 32q+31
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
    if (EPI == EPI_QKV) {
      // positions and cache rows of the tile's tokens, under the main loop
      build_token_table(tab, qa, M, (int)threadIdx.x - 128);
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
    if (NORM) {
      // each token row's sum of squares over this rank's k-range, read from
      // global memory (L2) while the main loop runs: warp w takes rows w,
      // w + 4, ..., its lanes stride the row's 16-byte vectors
      const int ew = warp - 4;
      const int64_t k_lo = (int64_t)kb0 * KB;
      const int nv = nkb * KB / 8;
      for (int row = ew; row < NT; row += 4) {
        float a = 0.f;
        if (row < M) {
          const uint4* src = reinterpret_cast<const uint4*>(xg + (int64_t)row * K + k_lo);
#pragma unroll 8
          for (int v = lane; v < nv; v += 32) a += sumsq8<T>(__ldg(src + v));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        }
        if (lane == 0) ssq[row] = a;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (splits == 1) {
        for (int t = (int)threadIdx.x - 128; t < NT; t += 128) rt[t] = rsqrtf(ssq[t] / (float)K + eps);
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
    }
    const bool ok = lpc::mbar_wait(accum, 0, st);
    lpc::tc_fence_after();
    const float* rtp = NORM ? rt : nullptr;
    if (splits == 1) {
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < NT; c += 16) {
          EpiPre<16> pre;
          epi_prefetch<T, EPI, 16>(pre, resid, M, n_out, tile, q, lane, c, qa, tab);
          uint32_t r[16];
          lpc::tmem_ld16(taddr + c, r);
          lpc::tmem_wait_ld();
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
          emit<T, EPI, 16>(v, pre, out, M, n_out, tile, q, lane, c, qa, tab, rtp);
        }
      }
    } else {
      // partial row of this rank: [128 rows][NT] fp32 from `base`; the
      // 16-byte groups of a row are XOR-swizzled by the row so that a warp's
      // 32 rows spread over the shared-memory banks
      const int row = 32 * q + lane;
      const int swz = (NT / 4) % 8 == 0 ? (row & 7) : (row & 3);
      const uint32_t prow = base + (uint32_t)(row * NT) * 4u;
#pragma unroll 1
      for (int c = 0; c < NT; c += 16) {
        uint32_t r[16];
        lpc::tmem_ld16(taddr + c, r);
        lpc::tmem_wait_ld();
        if (!ok) {
#pragma unroll
          for (int i = 0; i < 16; ++i) r[i] = 0u;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                           prow + (uint32_t)(((c / 4 + g) ^ swz) * 16)),
                       "r"(r[4 * g]), "r"(r[4 * g + 1]), "r"(r[4 * g + 2]), "r"(r[4 * g + 3])
                       : "memory");
      }
      __syncwarp();
      lpc::cluster_sync();  // every rank's partial tile (and sums of squares) is in its shared memory
      if (NORM) {
        // each token's sum of squares over all of K: the ranks' partial
        // sums added in rank order
        const int tid = (int)threadIdx.x - 128;
        for (int t = tid; t < NT; t += 128) {
          float tot = 0.f;
          for (int k = 0; k < splits; ++k)
            tot += ld_cluster_f32(lpc::mapa_shared(ssq_addr + (uint32_t)t * 4u, (uint32_t)k));
          rt[t] = rsqrtf(tot / (float)K + eps);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      const int width = NT / splits;  // token columns reduced by this rank
      const int c0 = rank * width;
      switch (splits) {
#define LPC_RS(S_)                                                                            \
  case S_:                                                                                    \
    reduce_slice_any<T, EPI, S_>(prow, swz, c0, width, out, resid, M, n_out, tile, q, lane, qa, \
                                 tab, rtp);                                                   \
    break;
        LPC_RS(2) LPC_RS(3) LPC_RS(4) LPC_RS(5) LPC_RS(6) LPC_RS(7)
        default: reduce_slice_any<T, EPI, 8>(prow, swz, c0, width, out, resid, M, n_out, tile, q, lane, qa, tab, rtp); break;
#undef LPC_RS
      }
    }
  } else if (splits > 1) {
    lpc::cluster_sync();
  }
  if (splits > 1) {
    __syncwarp();
    lpc::cluster_sync();  // all slices read: shared memory may be released
  }
  lpc::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    lpc::tc_fence_after();
    lpc::tmem_dealloc(tmem, tmem_cols);
  }
}

struct Plan {
  int n_tiles, NT, stages, smem, splits;
  uint32_t tmem_cols;
};

// LPC_PDL=0 launches without programmatic stream serialisation.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("LPC_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

constexpr int MAX_SPLITS = 8;       // portable cluster size
constexpr int CTA_SLOTS = 148 * 2;  // two CTAs per SM
constexpr int MIN_KB_PER_SPLIT = 8;

// Split count: enough CTAs to fill the SMs' CTA slots, each split streaming at
// least MIN_KB_PER_SPLIT chunks; a CTA's fp32 partial tile (128 x NT) must fit
// in its pipeline shared memory.  LPC_WSGEMM_SPLITS=<n> overrides (clamped to
// the same shared-memory and k limits).
int choose_splits(const Plan& p, int K) {
  const int nkb = K / KB;
  const bool fit = TILE_ROWS * p.NT * 4 <= p.stages * (CHUNK + ((p.NT * KB * 2 + 1023) & ~1023));
  const int cap = fit ? std::max(1, std::min(MAX_SPLITS, nkb)) : 1;
  int want = std::max(1, std::min(CTA_SLOTS / p.n_tiles, nkb / MIN_KB_PER_SPLIT));
  if (const char* e = getenv("LPC_WSGEMM_SPLITS")) want = std::max(1, atoi(e));
  // each rank reduces an equal share of the NT / 4 four-column groups, and
  // the cluster size is a power of two: clusters of 3 or 6 CTAs did not pack
  // into one wave (q/k/v at 48 tokens: 37.2 us with 3 ranks, 25.9 with 2)
  for (int sp = std::min(want, cap); sp > 1; --sp)
    if ((sp & (sp - 1)) == 0 && (p.NT / 4) % sp == 0) return sp;
  return 1;
}

constexpr int NORM_BYTES = 2 * MAX_TOKENS * (int)sizeof(float);  // sums of squares + row scales

Plan make_plan(int64_t M, int64_t n_out, int K, int epilogue, bool norm) {
  Plan p;
  p.n_tiles = (int)(epilogue == EPI_SWIGLU ? (n_out + 63) / 64 : (n_out + TILE_ROWS - 1) / TILE_ROWS);
  p.NT = (int)((M + 15) / 16) * 16;
  const int stage_bytes = CHUNK + ((p.NT * KB * 2 + 1023) & ~1023);
  p.stages = std::max(2, std::min(8, SMEM_TARGET / stage_bytes));
  // EPI_QKV keeps a per-token table after the barriers, NORM the per-token
  // sums of squares and scales; they use the headroom above SMEM_TARGET as
  // long as two CTAs still fit an SM (113 KB each)
  const int extra = (epilogue == EPI_QKV ? TOK_TABLE_BYTES : 0) + (norm ? NORM_BYTES : 0);
  while (p.stages > 2 && p.stages * stage_bytes + 1024 + 8 * (2 * p.stages + 4) + extra > 113 * 1024)
    --p.stages;
  p.smem = p.stages * stage_bytes + 1024 + 8 * (2 * p.stages + 4) + extra;
  p.tmem_cols = 32;
  while ((int)p.tmem_cols < p.NT) p.tmem_cols <<= 1;
  p.splits = choose_splits(p, K);
  return p;
}

template <typename T, int EPI, bool NORM>
int launch(const void* x, const void* packed, void* out, const void* resid, int64_t M,
           int64_t n_out, int K, int dtype, cudaStream_t s, float eps,
           const QkvArgs& qa = QkvArgs{}) {
  const Plan p = make_plan(M, n_out, K, EPI, NORM);
  lpc::TmaDesc tx;
  int rc = lpc::make_tma_2d(&tx, x, dtype, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, KB,
                            (uint32_t)p.NT, true);
  if (rc) return rc;
  static std::atomic<uint64_t> mask{0};
  if ((rc = lpc::once_per_device_smem((const void*)wsgemm_kernel<T, EPI, NORM>, 227 * 1024, mask)))
    return rc;
  const uint32_t idesc =
      lpc::idesc_f16(dtype == LPC_DTYPE_BF16 ? 1u : 0u, TILE_ROWS, (uint32_t)p.NT, 0u, 0u);
  // programmatic stream serialisation: the prologue and the first weight
  // chunks overlap the tail of the previous kernel on the stream
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.n_tiles * p.splits), 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)p.splits;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.splits > 1 ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, wsgemm_kernel<T, EPI, NORM>, tx, (const T*)x,
                                     (const uint8_t*)packed,
                                     (T*)out, (const T*)resid, (int)M, K, (int)n_out, p.NT,
                                     p.stages, p.tmem_cols, idesc, p.splits, qa, eps);
  if (e != cudaSuccess) {
    lpc::set_error("wsgemm (%d-way split): launch failed: %s", p.splits, cudaGetErrorString(e));
    return LPC_ERR_CUDA;
  }
  return lpc::check_launch("wsgemm");
}

template <typename T, bool NORM>
int launch_epi(int epilogue, const void* x, const void* packed, void* out, const void* resid,
               int64_t M, int64_t n_out, int K, int dtype, cudaStream_t s, float eps) {
  switch (epilogue) {
    case EPI_STORE: return launch<T, EPI_STORE, NORM>(x, packed, out, resid, M, n_out, K, dtype, s, eps);
    case EPI_RESIDUAL: return launch<T, EPI_RESIDUAL, NORM>(x, packed, out, resid, M, n_out, K, dtype, s, eps);
    case EPI_SWIGLU: return launch<T, EPI_SWIGLU, NORM>(x, packed, out, resid, M, n_out, K, dtype, s, eps);
  }
  lpc::set_error("wsgemm: unknown epilogue %d", epilogue);
  return LPC_ERR_INVALID;
}

}  // namespace

extern "C" int64_t lpc_packed_weight_bytes(int64_t n_out, int k, int layout) {
  if (n_out <= 0 || k <= 0 || k % KB || layout < 0 || layout > 2) return 0;
  if (layout == 2 && n_out % HEAD_DIM) return 0;
  const int64_t tiles = layout == 1 ? (n_out + 63) / 64 : (n_out + TILE_ROWS - 1) / TILE_ROWS;
  return tiles * (k / KB) * (int64_t)CHUNK;
}

extern "C" int lpc_pack_weights(const void* w0, const void* w1, const float* k_scale, void* packed,
                                int64_t n_out, int k, int layout, int dtype, void* stream) {
  using namespace lpc;
  if (n_out <= 0 || k <= 0 || k % KB || layout < 0 || layout > 2 ||
      (layout == 2 && n_out % HEAD_DIM)) {
    set_error("pack_weights: need n_out > 0, k a multiple of 64 and layout 0, 1 or 2 "
              "(layout 2: n_out a multiple of %d)", HEAD_DIM);
    return LPC_ERR_INVALID;
  }
  if (dtype != LPC_DTYPE_BF16 && dtype != LPC_DTYPE_F16) {
    set_error("pack_weights: bf16 or fp16 weights only");
    return LPC_ERR_UNSUPPORTED;
  }
  if (!w0 || !packed || !aligned16(w0) || !aligned16(packed) || (w1 && !aligned16(w1))) {
    set_error("pack_weights: null or misaligned pointer");
    return LPC_ERR_INVALID;
  }
  const int n_tiles = (int)(layout == 1 ? (n_out + 63) / 64 : (n_out + TILE_ROWS - 1) / TILE_ROWS);
  const int64_t total = (int64_t)n_tiles * (k / KB) * (CHUNK / 16);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LPC_DTYPE_BF16)
    pack_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)w0, (const __nv_bfloat16*)w1,
                                                      k_scale, (uint4*)packed, n_out, k, n_tiles, layout);
  else
    pack_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)w0, (const __half*)w1, k_scale,
                                               (uint4*)packed, n_out, k, n_tiles, layout);
  if (int rc = check_launch("pack_weights")) return rc;
  // lpc_wsgemm reads the packed weights before waiting on the previous grid:
  // the packed copy must be complete when this call returns
  if (cudaStreamSynchronize(s) != cudaSuccess) {
    set_error("pack_weights: stream synchronisation failed");
    return LPC_ERR_CUDA;
  }
  return LPC_OK;
}

extern "C" int lpc_wsgemm(const void* x, const void* packed_w, void* out, const void* resid,
                          int64_t tokens, int64_t n_out, int k, int epilogue, int dtype,
                          float norm_eps, void* stream) {
  using namespace lpc;
  if (tokens <= 0 || tokens > MAX_TOKENS || n_out <= 0 || n_out > (1 << 24) || k <= 0 || k % KB) {
    set_error("wsgemm: need 1..%d tokens, 0 < n_out <= 2^24 and k a multiple of 64 "
              "(tokens=%lld k=%d)", MAX_TOKENS, (long long)tokens, k);
    return LPC_ERR_INVALID;
  }
  if (dtype != LPC_DTYPE_BF16 && dtype != LPC_DTYPE_F16) {
    set_error("wsgemm: bf16 or fp16 only");
    return LPC_ERR_UNSUPPORTED;
  }
  if (epilogue < 0 || epilogue > 2 || (epilogue == EPI_RESIDUAL && !resid)) {
    set_error("wsgemm: bad epilogue %d (residual needs resid)", epilogue);
    return LPC_ERR_INVALID;
  }
  if (!x || !packed_w || !out || !aligned16(x) || !aligned16(packed_w)) {
    set_error("wsgemm: null or misaligned pointer");
    return LPC_ERR_INVALID;
  }
  if (norm_eps < 0.f || norm_eps != norm_eps) {
    set_error("wsgemm: norm_eps must be 0 (no norm) or positive");
    return LPC_ERR_INVALID;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool norm = norm_eps > 0.f;
  if (dtype == LPC_DTYPE_BF16)
    return norm ? launch_epi<__nv_bfloat16, true>(epilogue, x, packed_w, out, resid, tokens, n_out, k, dtype, s, norm_eps)
                : launch_epi<__nv_bfloat16, false>(epilogue, x, packed_w, out, resid, tokens, n_out, k, dtype, s, 0.f);
  return norm ? launch_epi<__half, true>(epilogue, x, packed_w, out, resid, tokens, n_out, k, dtype, s, norm_eps)
              : launch_epi<__half, false>(epilogue, x, packed_w, out, resid, tokens, n_out, k, dtype, s, 0.f);
}

extern "C" int lpc_qkv_rope_append(const void* x, const void* packed_w, const int64_t* positions,
                                   const void* cos, const void* sin, int64_t table_rows,
                                   void* q_out, void* key_cache, void* value_cache,
                                   const int64_t* seq_base, const int32_t* seq_cap, int64_t batch,
                                   int64_t seq, int num_heads, int num_kv_heads, int head_dim, int k,
                                   int64_t max_batch, int64_t max_seq_len, int64_t total_rows,
                                   int dtype, int table_dtype, float norm_eps, void* stream) {
  using namespace lpc;
  const int64_t tokens = batch * seq;
  if (batch <= 0 || seq <= 0 || tokens > MAX_TOKENS || num_heads <= 0 || num_kv_heads <= 0 ||
      k <= 0 || k % KB || table_rows <= 0) {
    set_error("qkv_rope_append: need 1..%d tokens, heads > 0 and k a multiple of 64 "
              "(tokens=%lld k=%d)", MAX_TOKENS, (long long)tokens, k);
    return LPC_ERR_INVALID;
  }
  if (head_dim != HEAD_DIM) {
    set_error("qkv_rope_append: head_dim must be %d (got %d)", HEAD_DIM, head_dim);
    return LPC_ERR_UNSUPPORTED;
  }
  if ((dtype != LPC_DTYPE_BF16 && dtype != LPC_DTYPE_F16) || table_dtype != dtype) {
    set_error("qkv_rope_append: bf16 or fp16 data with cos/sin tables of the same dtype");
    return LPC_ERR_UNSUPPORTED;
  }
  const bool ragged = seq_base != nullptr;
  if (ragged ? (!seq_cap || total_rows <= 0) : (max_batch < batch || max_seq_len <= 0)) {
    set_error("qkv_rope_append: %s", ragged ? "ragged layout needs seq_cap and total_rows > 0"
                                            : "dense cache needs max_batch >= batch and max_seq_len > 0");
    return LPC_ERR_INVALID;
  }
  if (!x || !packed_w || !positions || !cos || !sin || !q_out || !key_cache || !value_cache ||
      !aligned16(x) || !aligned16(packed_w)) {
    set_error("qkv_rope_append: null or misaligned pointer");
    return LPC_ERR_INVALID;
  }
  QkvArgs qa;
  qa.positions = positions;
  qa.cosb = cos;
  qa.sinb = sin;
  qa.table_rows = table_rows;
  qa.q_out = q_out;
  qa.kc = key_cache;
  qa.vc = value_cache;
  qa.seq_base = seq_base;
  qa.seq_cap = seq_cap;
  qa.seq = seq;
  qa.max_batch = max_batch;
  qa.max_seq = max_seq_len;
  qa.total_rows = total_rows;
  qa.H = num_heads;
  qa.Hkv = num_kv_heads;
  if (norm_eps < 0.f || norm_eps != norm_eps) {
    set_error("qkv_rope_append: norm_eps must be 0 (no norm) or positive");
    return LPC_ERR_INVALID;
  }
  const int64_t n_out = (int64_t)(num_heads + 2 * num_kv_heads) * HEAD_DIM;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool norm = norm_eps > 0.f;
  if (dtype == LPC_DTYPE_BF16)
    return norm ? launch<__nv_bfloat16, EPI_QKV, true>(x, packed_w, nullptr, nullptr, tokens, n_out, k, dtype, s, norm_eps, qa)
                : launch<__nv_bfloat16, EPI_QKV, false>(x, packed_w, nullptr, nullptr, tokens, n_out, k, dtype, s, 0.f, qa);
  return norm ? launch<__half, EPI_QKV, true>(x, packed_w, nullptr, nullptr, tokens, n_out, k, dtype, s, norm_eps, qa)
              : launch<__half, EPI_QKV, false>(x, packed_w, nullptr, nullptr, tokens, n_out, k, dtype, s, 0.f, qa);
}
