// Split-KV decode attention over ragged context lengths (one query per sequence).
//
// Semantics: out[b, h] = softmax(q[b, h] . K[b, h/G, :L_b]^T * scale) V[b, h/G, :L_b]
// with fp32 accumulation -- the bottom-right-aligned causal attention of a
// single new token over its whole context (tests/test_attention_correctness.py:10-76
// with q_len = 1; the decode kernel src/llama_pure_compute/triton_kernels/
// flash_attention.py:450-710).  The reference handles one KV_LEN per call
// (a constexpr, recompiled per length); here each sequence has its own length
// L_b = seq_lens[b], read on the device.
//
// Decomposition (HBM-streaming, no tensor cores: one query row per KV head
// gives an arithmetic intensity of ~1 FLOP/byte):
//   grid (split, kv_head, batch); each CTA owns one split of one (b, kv head)
//   and all G = heads/kv_heads query heads that share them.  The host picks
//   the split length `chunk` per launch (split_chunk): a sequence of L keys
//   takes ceil(L / chunk) splits, the last one holding the remainder.
//   warp 4     producer: cp.async.bulk copies of contiguous 32-key K and V
//              slabs (8 KB each for head_dim 128 bf16) into a 4-stage ring,
//              completion on mbarriers (tx bytes).
//   warps 0-3  each takes 8 keys of every slab.  Lane l holds dims
//              [l*D/32, (l+1)*D/32) of q, K rows and the fp32 output
//              accumulator.  The 8 partial dot products are reduced across the
//              warp with a transposing butterfly (9 shuffles for 8 keys), so
//              lanes 4j..4j+3 end with key j's score; online softmax runs in
//              the log2 domain (scale * log2 e folded into q).
//   CTA end    the 4 warps' (max, sum, acc) merge through shared memory; a
//              sequence with a single split writes its output directly, else
//              the split's partial goes to the workspace and a small combine
//              kernel merges the splits.  When every sequence fits one split
//              (chunk >= max_seq_len) the combine kernel is not launched.
#include <atomic>

#include <cstdlib>

#include "lpc_common.cuh"

LPC_DECLARE_STATUS(g_decode_status)

unsigned int lpc_status_decode(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_decode_status, sizeof(v));
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_decode_status, &z, sizeof(z));
  }
  return v;
}

namespace {

using lpc::Num;

constexpr int CHUNK = 256;   // workspace granularity: the shortest split length
constexpr int TILE = 32;     // keys per pipeline stage
constexpr int NSTAGE = 4;
constexpr int NCWARPS = 4;   // compute warps
constexpr int KPW = TILE / NCWARPS;  // keys per warp per stage = 8
constexpr float LOG2E = 1.4426950408889634f;

// Hardware base-2 exponential (MUFU ex2, approximate, flush-to-zero).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ void unpack2(uint32_t w, float& a, float& b);
template <>
__device__ __forceinline__ void unpack2<__nv_bfloat16>(uint32_t w, float& a, float& b) {
  a = lpc::bf16lo(w);
  b = lpc::bf16hi(w);
}
template <>
__device__ __forceinline__ void unpack2<__half>(uint32_t w, float& a, float& b) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  float2 f = __half22float2(h);
  a = f.x;
  b = f.y;
}

template <int DPL>
struct RawRow;  // DPL 16-bit values packed in 32-bit words
template <>
struct RawRow<4> {
  uint32_t w[2];
  __device__ __forceinline__ void load(const uint8_t* p) {
    uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x;
    w[1] = v.y;
  }
};
template <>
struct RawRow<2> {
  uint32_t w[1];
  __device__ __forceinline__ void load(const uint8_t* p) { w[0] = *reinterpret_cast<const uint32_t*>(p); }
};
template <>
struct RawRow<1> {  // head_dim 32: one 16-bit value per lane
  uint32_t w[1];
  __device__ __forceinline__ void load(const uint8_t* p) { w[0] = *reinterpret_cast<const uint16_t*>(p); }
};

template <typename T>
__device__ __forceinline__ float unpack1(uint32_t w);
template <>
__device__ __forceinline__ float unpack1<__nv_bfloat16>(uint32_t w) { return __uint_as_float(w << 16); }
template <>
__device__ __forceinline__ float unpack1<__half>(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)w));
}

// Packed fp32 pairs: Blackwell's f32x2 FMA does two lanes of work in one
// instruction (even dims in the low half, odd dims in the high half).
__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
template <typename T>
__device__ __forceinline__ uint64_t unpack_f2(uint32_t w) {
  float a, c;
  unpack2<T>(w, a, c);
  return pack_f2(a, c);
}

// q . k over this lane's DPL dims: even and odd dims accumulate in the two
// halves of an f32x2 FMA chain (fixed order), then one add.
template <typename T, int DPL>
__device__ __forceinline__ float row_dot(const RawRow<DPL>& r, const float* qf) {
  if constexpr (DPL == 1) {
    return qf[0] * unpack1<T>(r.w[0]);
  } else {
    uint64_t s = 0ull;  // +0.0f in both halves
#pragma unroll
    for (int w = 0; w < DPL / 2; ++w)
      s = fma_f2(pack_f2(qf[2 * w], qf[2 * w + 1]), unpack_f2<T>(r.w[w]), s);
    return lo_f(s) + hi_f(s);
  }
}

// acc += p * v over this lane's DPL dims (f32x2 FMAs, one per pair of dims).
template <typename T, int DPL>
__device__ __forceinline__ void row_axpy(const RawRow<DPL>& r, float p, float* acc) {
  if constexpr (DPL == 1) {
    acc[0] = fmaf(p, unpack1<T>(r.w[0]), acc[0]);
  } else {
    const uint64_t pp = pack_f2(p, p);
#pragma unroll
    for (int w = 0; w < DPL / 2; ++w) {
      const uint64_t d = fma_f2(pp, unpack_f2<T>(r.w[w]), pack_f2(acc[2 * w], acc[2 * w + 1]));
      acc[2 * w] = lo_f(d);
      acc[2 * w + 1] = hi_f(d);
    }
  }
}

// Where a sequence's cache rows live.
//   dense  (base == nullptr): cache [max_batch, Hkv, Smax, D], row (b, h, p) =
//          (b * Hkv + h) * Smax + p, capacity Smax;
//   ragged: cache [Hkv, total_rows, D], sequence b owns rows
//          [base[b], base[b] + cap[b]) of every head: row = h * total_rows + base[b] + p.
// length() clamps L to the capacity and zeroes it for a slot range outside the
// buffer, flagging either in the device status.
struct KvRows {
  const int64_t* base;
  const int32_t* cap;
  int64_t total_rows;
  __device__ __forceinline__ int length(int64_t b, int kvh, int Hkv, int64_t Smax, int L,
                                        int64_t* row0, bool report) const {
    int64_t c = Smax;
    if (base == nullptr) {
      *row0 = (b * Hkv + kvh) * Smax;
    } else {
      const int64_t sb = __ldg(base + b);
      c = __ldg(cap + b);
      if (sb < 0 || c < 0 || c > Smax || sb + c > total_rows) {
        if (report) atomicOr(&g_decode_status, LPC_DEV_ERR_BOUNDS);
        *row0 = 0;
        return 0;
      }
      *row0 = (int64_t)kvh * total_rows + sb;
    }
    if (L > c) {  // never read past this sequence's cache rows
      if (report) atomicOr(&g_decode_status, LPC_DEV_ERR_BOUNDS);
      L = (int)c;
    }
    return L;
  }
};

template <typename T, int D, int G>
__global__ void __launch_bounds__((NCWARPS + 1) * 32)
    decode_split_kernel(const T* __restrict__ q, const T* __restrict__ kc,
                        const T* __restrict__ vc, const int32_t* __restrict__ seq_lens,
                        T* __restrict__ out, float* __restrict__ part_o,
                        float* __restrict__ part_ml, int H, int Hkv, int64_t Smax,
                        int max_splits, int chunk, float scale_log2, KvRows rows) {
  constexpr int DPL = D / 32;                    // dims per lane
  constexpr int ROW_BYTES = D * (int)sizeof(T);
  constexpr int SLAB = TILE * ROW_BYTES;         // one K or V stage
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* sK = smem;
  uint8_t* sV = smem + NSTAGE * SLAB;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * NSTAGE * SLAB);
  float* red = reinterpret_cast<float*>(smem + 2 * NSTAGE * SLAB + 2 * NSTAGE * 8);
  // red: [NCWARPS][G][D + 2]

  // the combine kernel, launched with programmatic stream serialisation, may
  // be scheduled now; it waits for this grid to complete before reading
  lpc::pdl_trigger();
  // launched the same way under the kernel that wrote q and the new K/V rows
  lpc::pdl_wait();
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int64_t b = blockIdx.z;
  int64_t row0;  // cache row of (b, kv head, position 0)
  int L = rows.length(b, kvh, Hkv, Smax, __ldg(seq_lens + b), &row0, split == 0 && threadIdx.x == 0);
  const int nsplits = L > 0 ? (L + chunk - 1) / chunk : 0;
  if (split >= nsplits) {  // uniform for the whole CTA, before any barrier
    // an empty context attends to nothing: its heads' outputs are zero
    if (L <= 0 && split == 0)
      for (int i = threadIdx.x; i < G * D; i += blockDim.x)
        out[(b * H + (int64_t)kvh * G) * D + i] = Num<T>::from_f(0.f);
    return;
  }
  const int start = split * chunk;
  const int end = min(start + chunk, L);
  const int ntiles = (end - start + TILE - 1) / TILE;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  auto full_bar = [&](int s) { return lpc::smem_u32(bar + s); };
  auto empty_bar = [&](int s) { return lpc::smem_u32(bar + NSTAGE + s); };
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      lpc::mbar_init(full_bar(s), 1);
      lpc::mbar_init(empty_bar(s), NCWARPS);
    }
    lpc::fence_mbar_init();
  }
  __syncthreads();

  const int64_t head_base = row0 * D;  // elements
  float m_run[G], l_run[G], acc[G][DPL];

  if (warp == NCWARPS) {
    if (lane == 0) {
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % NSTAGE;
        const uint32_t r = (uint32_t)(t / NSTAGE);
        if (!lpc::mbar_wait(empty_bar(s), (r & 1u) ^ 1u, &g_decode_status)) break;
        const int k0 = start + t * TILE;
        const uint32_t bytes = (uint32_t)(min(TILE, end - k0) * ROW_BYTES);
        lpc::mbar_arrive_expect_tx(full_bar(s), 2 * bytes);
        lpc::bulk_g2s(lpc::smem_u32(sK + s * SLAB), kc + head_base + (int64_t)k0 * D, bytes,
                      full_bar(s));
        lpc::bulk_g2s(lpc::smem_u32(sV + s * SLAB), vc + head_base + (int64_t)k0 * D, bytes,
                      full_bar(s));
      }
    }
  } else {
    float qf[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const T* qp = q + (b * H + (int64_t)kvh * G + g) * D + lane * DPL;
#pragma unroll
      for (int i = 0; i < DPL; ++i) qf[g][i] = Num<T>::to_f(qp[i]) * scale_log2;
      m_run[g] = -INFINITY;
      l_run[g] = 0.f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[g][i] = 0.f;
    }
    const int my_key = lane >> 2;  // key (within this warp's 8) whose score this lane ends with
    for (int t = 0; t < ntiles; ++t) {
      const int s = t % NSTAGE;
      if (!lpc::mbar_wait(full_bar(s), (uint32_t)(t / NSTAGE) & 1u, &g_decode_status)) break;
      const int k0 = start + t * TILE;
      const int nvalid = min(TILE, end - k0) - warp * KPW;  // valid keys for this warp (may be <= 0)
      RawRow<DPL> kr[KPW], vr[KPW];
      const uint8_t* kb = sK + s * SLAB + (warp * KPW) * ROW_BYTES + lane * DPL * 2;
      const uint8_t* vb = sV + s * SLAB + (warp * KPW) * ROW_BYTES + lane * DPL * 2;
#pragma unroll
      for (int j = 0; j < KPW; ++j) {
        if (j < nvalid) {
          kr[j].load(kb + j * ROW_BYTES);
          vr[j].load(vb + j * ROW_BYTES);
        } else {
#pragma unroll
          for (int w = 0; w < (DPL + 1) / 2; ++w) { kr[j].w[w] = 0u; vr[j].w[w] = 0u; }
        }
      }
      __syncwarp();
      if (lane == 0) lpc::mbar_arrive(empty_bar(s));

#pragma unroll
      for (int g = 0; g < G; ++g) {
        float p8[KPW];
#pragma unroll
        for (int j = 0; j < KPW; ++j) p8[j] = row_dot<T, DPL>(kr[j], qf[g]);
        // transposing butterfly: 8 keys x 32 lanes -> lanes 4j..4j+3 hold key j
        {
          const bool hi = lane & 16;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float send = hi ? p8[j] : p8[j + 4];
            const float keep = hi ? p8[j + 4] : p8[j];
            p8[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
          }
        }
        {
          const bool hi = lane & 8;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const float send = hi ? p8[j] : p8[j + 2];
            const float keep = hi ? p8[j + 2] : p8[j];
            p8[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
          }
        }
        float sc;
        {
          const bool hi = lane & 4;
          const float send = hi ? p8[0] : p8[1];
          const float keep = hi ? p8[1] : p8[0];
          sc = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        sc += __shfl_xor_sync(0xffffffffu, sc, 2);
        sc += __shfl_xor_sync(0xffffffffu, sc, 1);
        if (my_key >= nvalid) sc = -INFINITY;
        float mx = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run[g], mx);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = fast_exp2(m_run[g] - m_use);
        const float p = fast_exp2(sc - m_use);
        m_run[g] = m_new;
        l_run[g] = l_run[g] * alpha + p;  // per-lane partial (lanes of one key group agree)
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] *= alpha;
#pragma unroll
        for (int j = 0; j < KPW; ++j) {
          const float pj = __shfl_sync(0xffffffffu, p, 4 * j);
          row_axpy<T, DPL>(vr[j], pj, acc[g]);
        }
      }
    }
    // per-warp totals: l over the 8 key groups
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float l = l_run[g];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      float* r = red + (warp * G + g) * (D + 2);
#pragma unroll
      for (int i = 0; i < DPL; ++i) r[lane * DPL + i] = acc[g][i];
      if (lane == 0) {
        r[D] = m_run[g];
        r[D + 1] = l;
      }
    }
  }
  __syncthreads();
  // merge the 4 warps; threads 0..D-1 each own one output dim per query head
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx - g * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NCWARPS; ++w) M = fmaxf(M, red[(w * G + g) * (D + 2) + D]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float O = 0.f, Ls = 0.f;
#pragma unroll
    for (int w = 0; w < NCWARPS; ++w) {
      const float* r = red + (w * G + g) * (D + 2);
      const float f = fast_exp2(r[D] - Mu);
      O = fmaf(f, r[d], O);
      Ls = fmaf(f, r[D + 1], Ls);
    }
    const int h = kvh * G + g;
    if (nsplits == 1) {
      out[(b * H + h) * D + d] = Num<T>::from_f(Ls > 0.f ? O / Ls : 0.f);
    } else {
      const int64_t pi = (b * H + h) * (int64_t)max_splits + split;
      part_o[pi * D + d] = O;
      if (d == 0) {
        part_ml[2 * pi] = M;
        part_ml[2 * pi + 1] = Ls;
      }
    }
  }
}

// One warp per (sequence, head): lane l merges output dims [l*D/32, (l+1)*D/32)
// over the splits, in split order.  Up to CB splits every load is issued
// before any is used (one memory round trip); longer sequences loop.
constexpr int COMBINE_WARPS = 4;
template <typename T, int D>
__global__ void __launch_bounds__(COMBINE_WARPS * 32) decode_combine_kernel(
    const float* __restrict__ part_o, const float* __restrict__ part_ml,
    const int32_t* __restrict__ seq_lens, T* __restrict__ out, int H, int max_splits,
    int chunk, int64_t Smax, KvRows rows, int64_t bh_total) {
  // the projection after attention, when launched with programmatic stream
  // serialisation (the packed decode GEMM), may start its weight stream now;
  // it waits for this grid to complete before reading `out`
  lpc::pdl_trigger();
  // launched under the split kernel: its partials are complete past here
  lpc::pdl_wait();
  constexpr int DPL = D / 32;
  const int64_t bh = (int64_t)blockIdx.x * COMBINE_WARPS + (threadIdx.x >> 5);
  if (bh >= bh_total) return;
  const int lane = threadIdx.x & 31;
  const int64_t b = bh / H;
  int64_t row0;
  const int L = rows.length(b, 0, 1, Smax, __ldg(seq_lens + b), &row0, false);
  T* o = out + bh * D + lane * DPL;
  if (L <= 0) {
#pragma unroll
    for (int i = 0; i < DPL; ++i) o[i] = Num<T>::from_f(0.f);
    return;
  }
  const int ns = (L + chunk - 1) / chunk;
  if (ns <= 1) return;  // written by the split kernel
  const float* ml = part_ml + bh * max_splits * 2;
  const float* po = part_o + bh * max_splits * D + lane * DPL;
  float O[DPL], Ls = 0.f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) O[i] = 0.f;
  constexpr int CB = 8;
  if (ns <= CB) {
    float mv[CB], lv[CB], ov[CB][DPL];
#pragma unroll
    for (int k = 0; k < CB; ++k) {
      const bool v = k < ns;
      mv[k] = v ? ml[2 * k] : -INFINITY;
      lv[k] = v ? ml[2 * k + 1] : 0.f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) ov[k][i] = v ? po[k * D + i] : 0.f;
    }
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < CB; ++k) M = fmaxf(M, mv[k]);
    const float Mu = M == -INFINITY ? 0.f : M;
#pragma unroll
    for (int k = 0; k < CB; ++k) {
      if (k < ns) {
        const float f = fast_exp2(mv[k] - Mu);
#pragma unroll
        for (int i = 0; i < DPL; ++i) O[i] = fmaf(f, ov[k][i], O[i]);
        Ls = fmaf(f, lv[k], Ls);
      }
    }
  } else {
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, ml[2 * s]);
    const float Mu = M == -INFINITY ? 0.f : M;
    for (int s = 0; s < ns; ++s) {
      const float f = fast_exp2(ml[2 * s] - Mu);
#pragma unroll
      for (int i = 0; i < DPL; ++i) O[i] = fmaf(f, po[s * D + i], O[i]);
      Ls = fmaf(f, ml[2 * s + 1], Ls);
    }
  }
  const float inv_ok = Ls > 0.f ? 1.f : 0.f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) o[i] = Num<T>::from_f(inv_ok > 0.f ? O[i] / Ls : 0.f);
}

template <typename T, int D, int G>
int launch_g(const void* q, const void* kc, const void* vc, const int32_t* lens, void* out,
             float* po, float* pml, int64_t B, int H, int Hkv, int64_t Smax, int max_splits,
             int chunk, float scale_log2, const KvRows& rows, cudaStream_t s) {
  constexpr int SLAB = TILE * D * 2;
  const int smem = 2 * NSTAGE * SLAB + 2 * NSTAGE * 8 + NCWARPS * G * (D + 2) * 4;
  static std::atomic<uint64_t> mask{0};
  int rc = lpc::once_per_device_smem((const void*)decode_split_kernel<T, D, G>, smem, mask);
  if (rc) return rc;
  // programmatic stream serialisation for both grids: each is scheduled while
  // the grid before it drains, and waits on it before reading
  static const bool pdl = [] {
    const char* e = getenv("LPC_PDL");
    return !(e && e[0] == '0');
  }();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  // splits a sequence of the cache's full length needs; shorter ones leave
  // the trailing CTAs of their row idle
  const int grid_splits = (int)((Smax + chunk - 1) / chunk);
  {
    // the split grid goes in early only while it is small: decode step 4.32
    // against 4.35 ms at 32 sequences (3,072 CTAs), 15.00 against 14.97 at
    // 256 (24,576 CTAs, whose first wave then competes with the tail of the
    // kernel before it)
    const int64_t ctas = (int64_t)grid_splits * Hkv * B;
    cudaLaunchAttribute sattr[1];
    sattr[0] = attr[0];
    sattr[0].val.programmaticStreamSerializationAllowed = pdl && ctas <= 4096 ? 1 : 0;
    cudaLaunchConfig_t sc = {};
    sc.gridDim = dim3((unsigned)grid_splits, (unsigned)Hkv, (unsigned)B);
    sc.blockDim = dim3((NCWARPS + 1) * 32);
    sc.dynamicSmemBytes = (size_t)smem;
    sc.stream = s;
    sc.attrs = sattr;
    sc.numAttrs = 1;
    if (cudaLaunchKernelEx(&sc, decode_split_kernel<T, D, G>, (const T*)q, (const T*)kc,
                           (const T*)vc, lens, (T*)out, po, pml, H, Hkv, Smax, max_splits,
                           chunk, scale_log2, rows) != cudaSuccess) {
      lpc::set_error("decode_attention (split): launch failed");
      return LPC_ERR_CUDA;
    }
  }
  if ((rc = lpc::check_launch("decode_attention (split)"))) return rc;
  if (grid_splits == 1) return LPC_OK;  // every sequence was written by its single split
  const int64_t bh_total = B * (int64_t)H;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((bh_total + COMBINE_WARPS - 1) / COMBINE_WARPS));
  cfg.blockDim = dim3(COMBINE_WARPS * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, decode_combine_kernel<T, D>, (const float*)po, (const float*)pml,
                         lens, (T*)out, H, max_splits, chunk, Smax, rows, bh_total) != cudaSuccess) {
    lpc::set_error("decode_attention (combine): launch failed");
    return LPC_ERR_CUDA;
  }
  return lpc::check_launch("decode_attention (combine)");
}

template <typename T, int D>
int launch_d(int G, const void* q, const void* kc, const void* vc, const int32_t* lens,
             void* out, float* po, float* pml, int64_t B, int H, int Hkv, int64_t Smax,
             int max_splits, int ch, float sl2, const KvRows& r, cudaStream_t s) {
  switch (G) {
    case 1: return launch_g<T, D, 1>(q, kc, vc, lens, out, po, pml, B, H, Hkv, Smax, max_splits, ch, sl2, r, s);
    case 2: return launch_g<T, D, 2>(q, kc, vc, lens, out, po, pml, B, H, Hkv, Smax, max_splits, ch, sl2, r, s);
    case 4: return launch_g<T, D, 4>(q, kc, vc, lens, out, po, pml, B, H, Hkv, Smax, max_splits, ch, sl2, r, s);
    case 8: return launch_g<T, D, 8>(q, kc, vc, lens, out, po, pml, B, H, Hkv, Smax, max_splits, ch, sl2, r, s);
  }
  lpc::set_error("decode_attention: heads/kv_heads = %d not supported (1, 2, 4 or 8)", G);
  return LPC_ERR_UNSUPPORTED;
}

}  // namespace

// Largest sizes the split grid can express (grid.x = splits, grid.z = batch):
// checked before any size arithmetic, so no product below can overflow.
constexpr int64_t MAX_DECODE_BATCH = 65535;
constexpr int64_t MAX_DECODE_SEQ = 65535LL * CHUNK;
constexpr int MAX_DECODE_HEADS = 65535;
constexpr int MAX_DECODE_HEAD_DIM = 1024;

extern "C" int64_t lpc_decode_attention_workspace_bytes(int64_t batch, int heads,
                                                        int64_t max_seq_len, int head_dim) {
  if (batch <= 0 || heads <= 0 || max_seq_len <= 0 || head_dim <= 0) return 0;
  if (batch > MAX_DECODE_BATCH || heads > MAX_DECODE_HEADS || max_seq_len > MAX_DECODE_SEQ ||
      head_dim > MAX_DECODE_HEAD_DIM)
    return 0;
  const int64_t max_splits = (max_seq_len + CHUNK - 1) / CHUNK;
  return batch * heads * max_splits * (int64_t)(head_dim + 2) * 4;
}

namespace {

// Split length for one launch.  Longer splits cost fewer CTA start-ups and
// partials, but the grid must stay several waves deep (about 440 CTAs run at
// once: three per SM).  `total_keys` is the cache capacity over all
// sequences (dense: batch * max_seq_len; ragged: the rows per KV head):
//   * 1024 keys when there are at least MIN_SPLIT_CTAS (sequence, KV head)
//     pairs (one or more CTAs per pair is already a deep grid), or when full
//     1024-key splits of the capacity give MIN_SPLIT_CTAS CTAs;
//   * 512 keys when full 512-key splits give MIN_SPLIT_CTAS CTAs;
//   * 256 keys otherwise.
// Measured on the 7B decode shape (32 KV heads, head_dim 128, us per call,
// 256 / 512 / 1024-key splits): every sequence at 576 keys, 256 / 128 / 64
// sequences 348 / - / 336, 179 / - / 172, 95 / - / 89 and 32 / 16 sequences
// 50.6 / 51.6 / 51.6, 29.5 / - / -; 8192 keys, 32 / 16 / 8 / 4 sequences
// 604 / 594 / 589, 310 / 304 / 301, 164 / 160 / 154, 90.5 / 85.4 / 87.1;
// 4096 keys, 32 / 8 sequences 306 / 303 / 301, 87.5 / 82.9 / 86.9.
// LPC_DECODE_CHUNK=<keys> (a multiple of 32 from 256 to 65536) overrides the
// choice.
constexpr int64_t MIN_SPLIT_CTAS = 2048;
int split_chunk(int64_t batch, int kv_heads, int64_t total_keys) {
  static const int forced = [] {
    const char* e = getenv("LPC_DECODE_CHUNK");
    const int v = e ? atoi(e) : 0;
    return (v >= CHUNK && v <= 65536 && v % TILE == 0) ? v : 0;
  }();
  if (forced) return forced;
  if (batch * kv_heads >= MIN_SPLIT_CTAS) return 1024;
  for (int c : {1024, 512})
    if ((int64_t)kv_heads * (total_keys / c) >= MIN_SPLIT_CTAS) return c;
  return CHUNK;
}

}  // namespace

extern "C" int lpc_decode_attention_split_keys(int64_t batch, int kv_heads, int64_t max_seq_len,
                                               int64_t total_rows) {
  if (batch <= 0 || kv_heads <= 0 || max_seq_len <= 0 || batch > MAX_DECODE_BATCH ||
      kv_heads > MAX_DECODE_HEADS || max_seq_len > MAX_DECODE_SEQ || total_rows > (int64_t(1) << 40))
    return 0;
  return split_chunk(batch, kv_heads, total_rows > 0 ? total_rows : batch * max_seq_len);
}

namespace {

int decode_common(const void* q, const void* key_cache, const void* value_cache,
                  const int32_t* seq_lens, void* out, void* workspace, int64_t workspace_bytes,
                  int64_t batch, int heads, int kv_heads, int head_dim, int64_t max_seq_len,
                  float sm_scale, int dtype, const KvRows& rows, void* stream) {
  using namespace lpc;
  if (batch == 0) return LPC_OK;
  if (dtype != LPC_DTYPE_BF16 && dtype != LPC_DTYPE_F16) {
    set_error("decode_attention: only bf16 and fp16 are supported");
    return LPC_ERR_UNSUPPORTED;
  }
  if (head_dim != 128 && head_dim != 64 && head_dim != 32) {
    set_error("decode_attention: head_dim must be 32, 64 or 128, got %d", head_dim);
    return LPC_ERR_UNSUPPORTED;
  }
  if (!q || !key_cache || !value_cache || !seq_lens || !out) {
    set_error("decode_attention: null pointer");
    return LPC_ERR_INVALID;
  }
  if (!aligned16(key_cache) || !aligned16(value_cache) || !aligned16(q) || !aligned16(out)) {
    set_error("decode_attention: tensors must be 16-byte aligned");
    return LPC_ERR_INVALID;
  }
  if (batch > MAX_DECODE_BATCH || heads > MAX_DECODE_HEADS || max_seq_len > MAX_DECODE_SEQ) {
    set_error("decode_attention: grid too large (batch <= %lld, heads <= %d, max_seq_len <= %lld)",
              (long long)MAX_DECODE_BATCH, MAX_DECODE_HEADS, (long long)MAX_DECODE_SEQ);
    return LPC_ERR_UNSUPPORTED;
  }
  const int64_t need = lpc_decode_attention_workspace_bytes(batch, heads, max_seq_len, head_dim);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
    set_error("decode_attention: workspace of %lld bytes required, got %lld", (long long)need,
              (long long)workspace_bytes);
    return LPC_ERR_INVALID;
  }
  const int64_t max_splits = (max_seq_len + CHUNK - 1) / CHUNK;
  if (max_splits > 65535 || batch > 65535 || kv_heads > 65535) {
    set_error("decode_attention: grid too large");
    return LPC_ERR_UNSUPPORTED;
  }
  float* po = static_cast<float*>(workspace);
  float* pml = po + batch * heads * max_splits * head_dim;
  const float sl2 = sm_scale * LOG2E;
  const int G = heads / kv_heads;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int ms = (int)max_splits;
  const int ch = split_chunk(batch, kv_heads, rows.base ? rows.total_rows : batch * max_seq_len);
  if (dtype == LPC_DTYPE_BF16) {
    if (head_dim == 128)
      return launch_d<__nv_bfloat16, 128>(G, q, key_cache, value_cache, seq_lens, out, po, pml, batch, heads, kv_heads, max_seq_len, ms, ch, sl2, rows, s);
    if (head_dim == 64)
      return launch_d<__nv_bfloat16, 64>(G, q, key_cache, value_cache, seq_lens, out, po, pml, batch, heads, kv_heads, max_seq_len, ms, ch, sl2, rows, s);
    return launch_d<__nv_bfloat16, 32>(G, q, key_cache, value_cache, seq_lens, out, po, pml, batch, heads, kv_heads, max_seq_len, ms, ch, sl2, rows, s);
  }
  if (head_dim == 128)
    return launch_d<__half, 128>(G, q, key_cache, value_cache, seq_lens, out, po, pml, batch, heads, kv_heads, max_seq_len, ms, ch, sl2, rows, s);
  if (head_dim == 64)
    return launch_d<__half, 64>(G, q, key_cache, value_cache, seq_lens, out, po, pml, batch, heads, kv_heads, max_seq_len, ms, ch, sl2, rows, s);
  return launch_d<__half, 32>(G, q, key_cache, value_cache, seq_lens, out, po, pml, batch, heads, kv_heads, max_seq_len, ms, ch, sl2, rows, s);
}

}  // namespace

extern "C" int lpc_decode_attention(const void* q, const void* key_cache, const void* value_cache,
                                    const int32_t* seq_lens, void* out, void* workspace,
                                    int64_t workspace_bytes, int64_t batch, int heads,
                                    int kv_heads, int head_dim, int64_t max_batch,
                                    int64_t max_seq_len, float sm_scale, int dtype,
                                    void* stream) {
  using namespace lpc;
  if (batch < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || max_batch <= 0 ||
      max_seq_len <= 0 || batch > max_batch) {
    set_error("decode_attention: invalid sizes (batch=%lld heads=%d kv_heads=%d max_batch=%lld)",
              (long long)batch, heads, kv_heads, (long long)max_batch);
    return LPC_ERR_INVALID;
  }
  const KvRows dense{nullptr, nullptr, 0};
  return decode_common(q, key_cache, value_cache, seq_lens, out, workspace, workspace_bytes, batch,
                       heads, kv_heads, head_dim, max_seq_len, sm_scale, dtype, dense, stream);
}

extern "C" int lpc_decode_attention_ragged(const void* q, const void* key_cache,
                                           const void* value_cache, const int32_t* seq_lens,
                                           const int64_t* seq_base, const int32_t* seq_cap,
                                           void* out, void* workspace, int64_t workspace_bytes,
                                           int64_t batch, int heads, int kv_heads, int head_dim,
                                           int64_t total_rows, int64_t max_seq_len,
                                           float sm_scale, int dtype, void* stream) {
  using namespace lpc;
  if (batch < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || total_rows <= 0 ||
      max_seq_len <= 0) {
    set_error("decode_attention_ragged: invalid sizes (batch=%lld heads=%d kv_heads=%d "
              "total_rows=%lld max_seq_len=%lld)", (long long)batch, heads, kv_heads,
              (long long)total_rows, (long long)max_seq_len);
    return LPC_ERR_INVALID;
  }
  if (batch > 0 && (!seq_base || !seq_cap)) {
    set_error("decode_attention_ragged: seq_base and seq_cap are required");
    return LPC_ERR_INVALID;
  }
  const KvRows ragged{seq_base, seq_cap, total_rows};
  return decode_common(q, key_cache, value_cache, seq_lens, out, workspace, workspace_bytes, batch,
                       heads, kv_heads, head_dim, max_seq_len, sm_scale, dtype, ragged, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot allocate device memory at the point where they run
// decode attention: a plugin inside a host application that owns every byte
// of HBM (for example a serving engine that reserves all free memory for its
// KV cache at start-up), or code on a serving path that must never call
// cudaMalloc because an allocation may synchronise the device or fail under
// memory pressure in the middle of a request.  For them the split partials
// live in a fixed scratch array in this library's device memory instead of a
// caller workspace.  The array belongs to this file's device code, so every
// GPU on which any decode-attention kernel of the library has run holds it
// (LPC_NOALLOC_SCRATCH_BYTES) until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[LPC_NOALLOC_SCRATCH_BYTES];

namespace {
// Device address of the scratch array, per device ordinal, together with the
// CUDA context it was resolved in.  A device reset creates a new context in
// which the module (and the array) may load at another address, so a cached
// address is only reused while the context is the same one.
struct NoallocSlot {
  void* ctx;
  void* addr;
};
std::mutex g_noalloc_mu;
NoallocSlot g_noalloc[64] = {};
}  // namespace

extern "C" int lpc_decode_attention_noalloc(const void* q, const void* key_cache,
                                            const void* value_cache, const int32_t* seq_lens,
                                            void* out, int64_t batch, int heads, int kv_heads,
                                            int head_dim, int64_t max_batch, int64_t max_seq_len,
                                            float sm_scale, int dtype, void* stream) {
  using namespace lpc;
  // sizes first: the scratch requirement below is only computed for sizes
  // whose product cannot overflow
  if (batch < 0 || batch > MAX_DECODE_BATCH || heads <= 0 || heads > MAX_DECODE_HEADS ||
      max_seq_len <= 0 || max_seq_len > MAX_DECODE_SEQ || head_dim <= 0 ||
      head_dim > MAX_DECODE_HEAD_DIM) {
    set_error("decode_attention_noalloc: invalid sizes (batch=%lld heads=%d max_seq_len=%lld "
              "head_dim=%d; batch <= %lld, heads <= %d, max_seq_len <= %lld)",
              (long long)batch, heads, (long long)max_seq_len, head_dim,
              (long long)MAX_DECODE_BATCH, MAX_DECODE_HEADS, (long long)MAX_DECODE_SEQ);
    return LPC_ERR_INVALID;
  }
  const int64_t need = lpc_decode_attention_workspace_bytes(batch, heads, max_seq_len, head_dim);
  if (need > (int64_t)LPC_NOALLOC_SCRATCH_BYTES) {
    set_error("decode_attention_noalloc: this shape needs %lld bytes of split scratch but the "
              "static scratch holds %lld (batch * heads * ceil(max_seq_len / 256) * "
              "(head_dim + 2) * 4 must fit); call lpc_decode_attention with a workspace instead",
              (long long)need, (long long)LPC_NOALLOC_SCRATCH_BYTES);
    return LPC_ERR_INVALID;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("decode_attention_noalloc: cannot query the current CUDA device");
    return LPC_ERR_CUDA;
  }
  void* ctx = current_context();
  void* scratch = nullptr;
  {
    // First call on a device (or in a new context of it): resolve the scratch
    // array's device address with that device current -- the symbol's
    // host-side name is not a device pointer.
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoallocSlot& slot = g_noalloc[dev];
    if (!slot.addr || !ctx || slot.ctx != ctx) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        set_error("decode_attention_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
        return LPC_ERR_CUDA;
      }
      slot.addr = p;
      slot.ctx = ctx;
    }
    scratch = slot.addr;
  }
  // No clearing is needed: every partial the combine step reads is written by
  // the split step of the same call.
  return lpc_decode_attention(q, key_cache, value_cache, seq_lens, out, scratch,
                              (int64_t)LPC_NOALLOC_SCRATCH_BYTES, batch, heads, kv_heads, head_dim,
                              max_batch, max_seq_len, sm_scale, dtype, stream);
}
