// Fused RMSNorm + SwiGLU: out = silu(norm(x) Wg^T) * (norm(x) Wu^T).
//
// Semantics follow `_rmsswiglu_forward_pytorch` (src/llama_pure_compute/ops.py:45-59)
// and the reference CUDA op (src/csrc/ops/rmsswiglu.cu:151-282), including the
// pre-fused weight form (up_w empty: gate_w is [2*inter, dim], gate rows first,
// rmsswiglu.cu:167-173).  The reference runs three launches with a
// [tokens, 2*inter] HBM round trip and a per-call torch::cat of the weights;
// here the gate/up products never leave the chip.
//
// bf16/fp16 path (tensor cores, sm_100a):
//   1. row RMSNorm -> normalised activations in the caller's workspace (bf16)
//   2. a warp-specialised tcgen05 GEMM with the SiLU*up epilogue, in one of
//      two forms chosen by token count:
//      * one CTA per 128-token x 64-inter tile (up to 128 tokens):
//          warp 4     TMA producer: A = 128x64 activation tile, B = 64 gate rows
//                     + 64 up rows (two TMA boxes into one 128-row operand)
//          warp 5     TMEM allocator + single-thread tcgen05.mma issuer
//                     (M=128, N=128, K=16 per instruction, fp32 accumulators)
//          warps 0-3  epilogue: tcgen05.ld the gate and up columns of each token
//                     row, silu(g)*u in fp32, one rounding to the output dtype
//        (32 KB stages; tiles rasterised in groups of GROUP_M token tiles so
//        that a wave of CTAs re-reads weight tiles from L2 rather than HBM)
//      * a CTA pair (cluster of 2, tcgen05 cta_group::2) per 256-token x
//        w-inter tile (more than 128 tokens): M = 256 tokens split over the
//        two CTAs; each CTA holds w/2 gate rows and w/2 up rows, CTA 0 issues
//        one M=256, N=w MMA for gate and one for up, and each CTA's TMEM ends
//        up holding its own tokens' gate|up accumulators.  Both CTAs' TMA
//        copies complete on CTA 0's barrier.  The inter dimension is dealt out
//        in 16-column units to a tile count matched to the number of CTA pairs
//        per wave (69 tiles of 144/160 columns for the 7B layer: one wave at
//        256 tokens, where 128-column tiles gave 86 pairs for 74 slots), and
//        w is capped at 160 or 256 columns, whichever the load-time model of
//        pair_tiles() finds faster for the token count.
// fp32 path (CUDA cores, no TF32): each CTA normalises up to 8 token rows into
//   shared memory, then streams gate/up rows with 16-byte loads and reduces the
//   dot products per warp.  It is the weight-streaming (HBM-bound) GEMV of the
//   fp32 op shape (8 tokens).
#include <algorithm>
#include <type_traits>
#include <atomic>
#include <mutex>

#include <cstdlib>

#include "lpc_common.cuh"

LPC_DECLARE_STATUS(g_swiglu_status)

unsigned int lpc_status_swiglu(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_swiglu_status, sizeof(v));
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_swiglu_status, &z, sizeof(z));
  }
  return v;
}

int lpc_rmsnorm_launch(const void* x, const void* w, void* y, int64_t rows, int dim, float eps,
                       int dtype, int w_dtype, cudaStream_t s);

namespace {

using lpc::Num;

constexpr int BM = 128;          // tokens per MMA tile (UMMA M)
constexpr int BNI = 64;          // inter columns per tile
constexpr int BN = 2 * BNI;      // UMMA N: 64 gate rows + 64 up rows
constexpr int BK = 64;           // 64 x 2 B = one 128-byte swizzle row
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int GROUP_M = 16;

// Shared memory of one CTA holding MT token tiles and a STAGES-deep ring.
template <int MT, int STAGES>
constexpr int tc_smem() { return STAGES * (MT * A_BYTES + B_BYTES) + 1024 + 256; }

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// MT token tiles (128 rows each) share every weight stage; STAGES-deep ring.
template <typename T, int MT, int STAGES>
__global__ void __launch_bounds__(192)
    swiglu_tc_kernel(const __grid_constant__ lpc::TmaDesc tmA,
                     const __grid_constant__ lpc::TmaDesc tmG,
                     const __grid_constant__ lpc::TmaDesc tmU, T* __restrict__ out, int M, int K,
                     int I, int up_row_off, int num_m, int num_n, uint32_t idesc) {
  constexpr int A_STAGE = MT * A_BYTES;
  constexpr int STAGE_BYTES = A_STAGE + B_BYTES;
  constexpr uint32_t TMEM_COLS = MT * 128;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = lpc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sA = base;
  const uint32_t sB = base + STAGES * A_STAGE;
  const uint32_t bars = sB + STAGES * B_BYTES;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
  const uint32_t accum_bar = bars + 8u * (2 * STAGES);
  const uint32_t tmem_slot = bars + 8u * (2 * STAGES + 1);
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // grouped rasterisation: GROUP_M token tiles sweep all inter tiles together
  const int bid = blockIdx.x;
  const int group = bid / (GROUP_M * num_n);
  const int first_m = group * GROUP_M;
  const int gm = min(GROUP_M, num_m - first_m);
  const int within = bid - group * GROUP_M * num_n;
  const int mt = first_m + within % gm;  // group of MT token tiles
  const int nt = within / gm;
  const int m0 = mt * BM * MT, i0 = nt * BNI;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      lpc::mbar_init(full_bar(s), 1);
      lpc::mbar_init(empty_bar(s), 1);
    }
    lpc::mbar_init(accum_bar, 1);
    lpc::fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    lpc::tma_prefetch_desc(&tmA);
    lpc::tma_prefetch_desc(&tmG);
    lpc::tma_prefetch_desc(&tmU);
  }
  if (warp == 5) {
    lpc::tmem_alloc(tmem_slot, TMEM_COLS);
    lpc::tmem_relinquish();
  }
  lpc::tc_fence_before();
  __syncthreads();
  lpc::tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;
  const int nkb = K / BK;

  if (warp == 4) {
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t r = (uint32_t)(kb / STAGES);
        if (!lpc::mbar_wait(empty_bar(s), (r & 1u) ^ 1u, &g_swiglu_status)) break;
        lpc::mbar_arrive_expect_tx(full_bar(s), STAGE_BYTES);
#pragma unroll
        for (int t = 0; t < MT; ++t)
          lpc::tma_load_2d(sA + s * A_STAGE + t * A_BYTES, &tmA, kb * BK, m0 + t * BM, full_bar(s));
        lpc::tma_load_2d(sB + s * B_BYTES, &tmG, kb * BK, i0, full_bar(s));
        lpc::tma_load_2d(sB + s * B_BYTES + B_BYTES / 2, &tmU, kb * BK, i0 + up_row_off,
                         full_bar(s));
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t r = (uint32_t)(kb / STAGES);
        if (!lpc::mbar_wait(full_bar(s), r & 1u, &g_swiglu_status)) break;
        lpc::tc_fence_after();
        const uint64_t bd = lpc::smem_desc_sw128(sB + s * B_BYTES, 16, 1024);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const uint64_t ad = lpc::smem_desc_sw128(sA + s * A_STAGE + t * A_BYTES, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            lpc::umma_ss(tmem + 128u * t, ad + 2u * kk, bd + 2u * kk, idesc, (kb | kk) != 0);
        }
        lpc::umma_commit(empty_bar(s));
      }
      lpc::umma_commit(accum_bar);
    }
  } else {
    // epilogue warps 0..3: TMEM lanes 32*warp .. 32*warp+31 = token rows
    const bool ok = lpc::mbar_wait(accum_bar, 0, &g_swiglu_status);
    lpc::tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int t = 0; t < MT; ++t) {
      const int row = m0 + t * BM + warp * 32 + lane;
      const uint32_t taddr = tmem + 128u * t + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BNI; c += 16) {
        uint32_t g[16], u[16];
        lpc::tmem_ld16(taddr + c, g);
        lpc::tmem_ld16(taddr + BNI + c, u);
        lpc::tmem_wait_ld();
        if (row < M && i0 + c < I) {
          uint32_t p[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            p[j] = pack2<T>(silu_mul(__uint_as_float(g[2 * j]), __uint_as_float(u[2 * j])),
                            silu_mul(__uint_as_float(g[2 * j + 1]), __uint_as_float(u[2 * j + 1])));
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)row * I + i0 + c);
          dst[0] = make_uint4(p[0], p[1], p[2], p[3]);
          dst[1] = make_uint4(p[4], p[5], p[6], p[7]);
        }
      }
      }
    }
  }
  lpc::tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    lpc::tc_fence_after();
    lpc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (cluster of 2, tcgen05 cta_group::2): one pair MMA of
// M = 256 tokens (128 in each CTA's shared memory) by N = 256 weight rows
// (128 gate rows in CTA 0, the 128 matching up rows in CTA 1).  Each CTA
// streams 16 KB of weights + 16 KB of activations per 64-k stage, half the
// activation bytes per weight byte of a one-CTA tile with 256 tokens, and each
// CTA's TMEM receives its 128 tokens x (128 gate | 128 up) accumulators, so the
// SiLU*up epilogue needs no exchange.
//   warp 4     producer (own CTA's two TMA boxes per stage)
//   warp 5     TMEM pair allocation; rank 0: MMA issuer
// Both CTAs' TMA copies of a stage complete on rank 0's full barrier; rank 0
// commits MMA completion to the empty / accumulator barriers of both CTAs.
//   warps 0-3  epilogue (TMEM lane = token)
// ---------------------------------------------------------------------------
constexpr int PAIR_TOK = 256;  // tokens per pair tile (128 per CTA)

// WMAX: widest inter tile (gate + up = 2 x WMAX TMEM columns, <= 512).  Per
// CTA and k-block a stage holds 128 token rows and WMAX/2 rows of each weight
// (the TMA boxes), so WMAX sets the FLOPs per loaded byte: 160 for decode-
// sized steps (69 tiles = one wave of the 74 pairs), 256 for larger ones.
template <int WMAX>
struct PairGeom {
  static constexpr int BROWS = WMAX / 2;
  static constexpr int B_BYTES = BROWS * BK * 2;  // a multiple of 1024
  static constexpr int STAGE = A_BYTES + 2 * B_BYTES;
};

template <int WMAX, int STAGES>
constexpr int pair_smem() { return STAGES * PairGeom<WMAX>::STAGE + 1024 + 256; }

// Sum of squares of the 8 elements of a 16-byte chunk (fixed order).
template <typename T>
__device__ __forceinline__ float sumsq8(const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float a, b;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      a = lpc::bf16lo(w[i]);
      b = lpc::bf16hi(w[i]);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      a = f.x;
      b = f.y;
    }
    s = fmaf(a, a, s);
    s = fmaf(b, b, s);
  }
  return s;
}

// Inter tile c of C covers columns [pair_col(c), pair_col(c + 1)): the I / 16
// sixteen-column units dealt out as evenly as possible, so tile widths differ
// by at most 16 and C can be matched to the number of CTA pairs per wave.
__host__ __device__ __forceinline__ int pair_col(int c, int units, int C) {
  return 16 * (int)(((int64_t)c * units) / C);
}

// CTA pair (cluster of 2, cta_group::2): one 256-token x w-column tile of
// gate and up.  Rank r holds tokens m0 + 128r .. and weight rows
// col0 + r*w/2 .. (w/2 gate rows, w/2 up rows) of each k-block; rank 0 issues
// an M=256, N=w MMA for gate (TMEM columns 0..w-1) and one for up (columns
// w..2w-1), each CTA receiving its own 128 token rows.
//
// NORM: A holds the raw rows x of the RMSNorm and the gate/up weights come
// with the norm weight folded in (W diag(w)).  Each MMA commits to a
// `consumed` barrier; the epilogue warps -- one per 32 token rows, idle until
// the accumulators are ready -- then read their token row of the stage's A
// tile, accumulate its sum of squares and release the stage (its `empty`
// barrier counts their four arrivals).  The epilogue scales each token's
// gate and up accumulators by rsqrt(sum / K + eps) before SiLU(g) * u.
template <typename T, int WMAX, int STAGES, bool NORM>
__global__ void __launch_bounds__(192)
    swiglu_pair_kernel(const __grid_constant__ lpc::TmaDesc tmA,
                       const __grid_constant__ lpc::TmaDesc tmG,
                       const __grid_constant__ lpc::TmaDesc tmU, T* __restrict__ out, int M, int K,
                       int I, int up_row_off, int num_m, int num_c, uint32_t ab_fmt, float eps) {
  constexpr uint32_t TMEM_COLS = 512;
  constexpr int PAIR_B_BYTES = PairGeom<WMAX>::B_BYTES;
  constexpr int PAIR_STAGE = PairGeom<WMAX>::STAGE;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = lpc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // same offset in both CTAs of the pair
  const uint32_t sA = base;
  const uint32_t sB = base + STAGES * A_BYTES;  // per stage: gate rows, then up rows
  const uint32_t bars = sB + STAGES * (2 * PAIR_B_BYTES);
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
  const uint32_t accum_bar = bars + 8u * (2 * STAGES);
  auto consumed_bar = [&](int s) { return bars + 8u * (2 * STAGES + 1 + s); };  // NORM only
  const uint32_t tmem_slot = bars + 8u * (3 * STAGES + 1);
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));
  // the MMA's completion of a stage: straight to `empty`, or with NORM to
  // `consumed`, after which the epilogue warps read the A rows and release it
  auto mma_done_bar = [&](int s) { return NORM ? consumed_bar(s) : empty_bar(s); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = lpc::cluster_ctarank();

  // consecutive pairs share an inter tile (its weights are read from HBM once
  // and from L2 by the other token tiles)
  const int pid = blockIdx.x >> 1;
  const int mt = pid % num_m;
  const int ct = pid / num_m;
  const int units = I / 16;
  const int col0 = pair_col(ct, units, num_c);
  const int w = pair_col(ct + 1, units, num_c) - col0;  // multiple of 16, <= WMAX
  const int hw = w / 2;
  const int m0 = mt * PAIR_TOK + (int)rank * BM;  // this CTA's 128 tokens

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      lpc::mbar_init(full_bar(s), 1);
      lpc::mbar_init(empty_bar(s), NORM ? 4 : 1);
      if (NORM) lpc::mbar_init(consumed_bar(s), 1);
    }
    lpc::mbar_init(accum_bar, 1);
    lpc::fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    lpc::tma_prefetch_desc(&tmA);
    lpc::tma_prefetch_desc(&tmG);
    lpc::tma_prefetch_desc(&tmU);
  }
  lpc::cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive
  if (warp == 5) {
    lpc::tmem_alloc_pair(tmem_slot, TMEM_COLS);
    lpc::tmem_relinquish_pair();
  }
  lpc::tc_fence_before();
  __syncthreads();
  lpc::tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;
  const int nkb = K / BK;
  unsigned int* st = &g_swiglu_status;
  if (warp != 4) lpc::pdl_wait();

  if (warp == 4) {
    if (lane == 0) {
      const int grow = col0 + (int)rank * hw;
      // both CTAs' copies complete on rank 0's full barrier, armed by rank 0
      // for the bytes of both CTAs (every box is full size: rows past the
      // matrix read as zeros and count)
      const uint32_t full0 = lpc::mapa_shared(full_bar(0), 0);
      auto load_w = [&](int kb) {
        const int s = kb % STAGES;
        if (rank == 0) lpc::mbar_arrive_expect_tx(full_bar(s), 2 * PAIR_STAGE);
        const uint32_t sb = sB + s * (2 * PAIR_B_BYTES);
        lpc::tma_load_2d_pair(sb, &tmG, kb * BK, grow, full0 + 8u * s);
        lpc::tma_load_2d_pair(sb + PAIR_B_BYTES, &tmU, kb * BK, up_row_off + grow, full0 + 8u * s);
      };
      auto load_a = [&](int kb) {
        const int s = kb % STAGES;
        lpc::tma_load_2d_pair(sA + s * A_BYTES, &tmA, kb * BK, m0, full0 + 8u * s);
      };
      // The gate/up weights are never written by the kernel this one may
      // overlap (the row norm of the same call): the first ring of weight
      // boxes needs no empty-slot wait and is issued before waiting on it.
      const int first = nkb < STAGES ? nkb : STAGES;
      for (int kb = 0; kb < first; ++kb) load_w(kb);
      lpc::pdl_wait();  // the normalised activations come from the previous kernel
      for (int kb = 0; kb < first; ++kb) load_a(kb);
      for (int kb = first; kb < nkb; ++kb) {
        const uint32_t r = (uint32_t)(kb / STAGES);
        if (!lpc::mbar_wait(empty_bar(kb % STAGES), (r & 1u) ^ 1u, st)) break;
        load_w(kb);
        load_a(kb);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      if (rank == 0) {
        const uint32_t idesc = lpc::idesc_f16(ab_fmt, PAIR_TOK, (uint32_t)w, 0u, 0u);
        const uint32_t peer_done0 = lpc::mapa_shared(mma_done_bar(0), 1);
        const uint32_t peer_accum = lpc::mapa_shared(accum_bar, 1);
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = kb % STAGES;
          const uint32_t par = (uint32_t)(kb / STAGES) & 1u;
          if (!lpc::mbar_wait(full_bar(s), par, st)) break;
          lpc::tc_fence_after();
          const uint32_t sb = sB + s * (2 * PAIR_B_BYTES);
          const uint64_t ad = lpc::smem_desc_sw128(sA + s * A_BYTES, 16, 1024);
          const uint64_t gd = lpc::smem_desc_sw128(sb, 16, 1024);
          const uint64_t ud = lpc::smem_desc_sw128(sb + PAIR_B_BYTES, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            lpc::umma_ss_pair(tmem, ad + 2u * kk, gd + 2u * kk, idesc, (kb | kk) != 0);
            lpc::umma_ss_pair(tmem + (uint32_t)w, ad + 2u * kk, ud + 2u * kk, idesc, (kb | kk) != 0);
          }
          lpc::umma_commit_pair(mma_done_bar(s));
          lpc::umma_commit_pair(peer_done0 + 8u * s);
        }
        lpc::umma_commit_pair(accum_bar);
        lpc::umma_commit_pair(peer_accum);
      }
    }
  } else {
    // epilogue warps 0..3: TMEM lanes 32*warp .. +31 = this CTA's tokens;
    // columns 0..w-1 gate, w..2w-1 up, for inter columns col0 ..
    bool stats_ok = true;
    float rs = 1.f;  // NORM: this token row's rsqrt(mean(x^2) + eps)
    if (NORM) {
      const int trow = warp * 32 + lane;  // row of this CTA's A tile
      float ss = 0.f;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        // every lane waits: a converged warp sleeps in the wait
        if (!__all_sync(0xffffffffu, lpc::mbar_wait(consumed_bar(s), (uint32_t)(kb / STAGES) & 1u, st))) {
          stats_ok = false;
          break;
        }
        const uint32_t ra = sA + s * A_BYTES + (uint32_t)trow * 128u;
        // lane l starts at chunk l % 8: the 8 lanes of a quarter-warp read 8
        // different 16-byte chunks (all 32 banks) instead of the same one
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 u;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                       : "r"(ra + (uint32_t)(((c + lane) & 7) * 16))
                       : "memory");
          ss += sumsq8<T>(u);
        }
        __syncwarp();
        if (lane == 0) lpc::mbar_arrive(empty_bar(s));
      }
      rs = rsqrtf(ss / (float)K + eps);
    }
    const bool ok = lpc::mbar_wait(accum_bar, 0, st) && stats_ok;
    lpc::tc_fence_after();
    if (ok) {
      const int row = m0 + warp * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < w; c += 16) {
        uint32_t g[16], u[16];
        lpc::tmem_ld16(taddr + c, g);
        lpc::tmem_ld16(taddr + w + c, u);
        lpc::tmem_wait_ld();
        if (row < M && col0 + c < I) {
          uint32_t p[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            p[j] = pack2<T>(silu_mul(__uint_as_float(g[2 * j]) * rs, __uint_as_float(u[2 * j]) * rs),
                            silu_mul(__uint_as_float(g[2 * j + 1]) * rs,
                                     __uint_as_float(u[2 * j + 1]) * rs));
          uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)row * I + col0 + c);
          dst[0] = make_uint4(p[0], p[1], p[2], p[3]);
          dst[1] = make_uint4(p[4], p[5], p[6], p[7]);
        }
      }
    }
  }
  lpc::tc_fence_before();
  lpc::cluster_sync();  // the peer's shared memory and barriers outlive every pair MMA and arrive
  if (warp == 5) {
    lpc::tc_fence_after();
    lpc::tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// fp32 streaming path
//
// The fp32 op is a weight stream: 8 token rows against 2 x [I, K] fp32
// weights read once (361 MB for the 7B layer), ~2 FMA per weight byte.
// Work is dealt out so that every warp streams the same number of bytes:
//   * CTA c (one per SM) owns a contiguous range of inter-column pairs;
//   * a unit is one pair (4 weight rows: gate/up of columns i and i+1) times
//     one eighth of K; the CTA's units are dealt round-robin to its 16 warps
//     (38 pairs x 8 = 304 units = 19 per warp for the 7B layer);
//   * per unit a lane streams 4 float4 of each of the 4 rows, multiplies them
//     by the 8 normalised token rows held in shared memory (each x float4 read
//     serves 4 rows) and the warp reduces its 32 partial sums (4 rows x 8
//     tokens) with a transposing butterfly (31 shuffles: lane j ends with sum
//     j), written to a shared partial table;
//   * once all units of a round are done, the 8 K-parts of each output are
//     summed in fixed order, SiLU(g) * u, one write per output.
// The RMSNorm prologue of the CTA's token rows runs while the first units'
// weights are prefetched into L2.
// ---------------------------------------------------------------------------
constexpr int F32_ROWS = 8;        // token rows per CTA (blockIdx.y)
constexpr int F32_WARPS = 16;
constexpr int F32_KPARTS = 8;      // K is split in 8 parts per unit
constexpr int F32_ROUND_PAIRS = 40;  // column pairs per round (partial table size)
constexpr int F32_PART_FLOATS = F32_ROUND_PAIRS * F32_KPARTS * 32;

// Transposing butterfly: v[0..31] of each lane summed over the warp; lane j
// returns the total of value j.
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int k = 0; k < o; ++k) {
      const float send = hi ? v[k] : v[k + o];
      const float keep = hi ? v[k + o] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

template <typename W>
__global__ void __launch_bounds__(F32_WARPS * 32, 1)
    swiglu_f32_kernel(const float* __restrict__ x, const W* __restrict__ nw,
                      const float* __restrict__ wg, const float* __restrict__ wu,
                      float* __restrict__ out, int64_t M, int K, int I, float eps) {
  extern __shared__ float4 xs4[];  // [F32_ROWS][K/4], then the partial table
  __shared__ float red[F32_WARPS];
  float* part = reinterpret_cast<float*>(xs4 + (int64_t)F32_ROWS * (K >> 2));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = (int64_t)blockIdx.y * F32_ROWS;
  const int rows = (int)min((int64_t)F32_ROWS, M - m0);
  const int kv = K >> 2;
  const int pairs = (I + 1) >> 1;
  const int p_begin = (int)((int64_t)blockIdx.x * pairs / gridDim.x);
  const int p_end = (int)((int64_t)(blockIdx.x + 1) * pairs / gridDim.x);

  // weight rows of unit u (pair p, K-part kp): gate/up of columns 2p, 2p+1
  auto unit_rows = [&](int p, const float* (&r)[4]) {
    const int i0 = 2 * p, i1 = min(2 * p + 1, I - 1);  // odd I: the last pair repeats a column
    r[0] = wg + (int64_t)i0 * K;
    r[1] = wu + (int64_t)i0 * K;
    r[2] = wg + (int64_t)i1 * K;
    r[3] = wu + (int64_t)i1 * K;
  };

  // L2 prefetch of each warp's first two units, under the norm prologue
  for (int u = warp, n = 0; n < 2 && p_begin + u / F32_KPARTS < p_end; u += F32_WARPS, ++n) {
    const float* r[4];
    unit_rows(p_begin + u / F32_KPARTS, r);
    const int kp = u % F32_KPARTS;
    const int64_t k0 = (int64_t)kp * kv / F32_KPARTS * 4, k1 = (int64_t)(kp + 1) * kv / F32_KPARTS * 4;
    for (int64_t k = k0 + lane * 32; k < k1; k += 32 * 32) {
#pragma unroll
      for (int j = 0; j < 4; ++j) asm volatile("prefetch.global.L2 [%0];" ::"l"(r[j] + k));
    }
  }

  // prologue: RMSNorm of this CTA's token rows into shared memory; warp w
  // takes half h = w & 1 of row w >> 1 (fp32 statistics, one rounding per
  // product as in the reference's fp32 path)
  {
    const int r = warp >> 1, h = warp & 1;
    const int v0 = h * (kv >> 1), v1 = h ? kv : (kv >> 1);
    float4* dst = xs4 + (int64_t)r * kv;
    float ss = 0.f;
    if (r < rows) {
      const float4* src = reinterpret_cast<const float4*>(x + (m0 + r) * K);
#pragma unroll 8
      for (int v = v0 + lane; v < v1; v += 32) {
        const float4 a = __ldg(src + v);
        ss = fmaf(a.x, a.x, ss);
        ss = fmaf(a.y, a.y, ss);
        ss = fmaf(a.z, a.z, ss);
        ss = fmaf(a.w, a.w, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    const float rr = rsqrtf((red[2 * r] + red[2 * r + 1]) / (float)K + eps);
    if (r < rows) {
      const float4* src = reinterpret_cast<const float4*>(x + (m0 + r) * K);
#pragma unroll 8
      for (int v = v0 + lane; v < v1; v += 32) {
        const float4 a = __ldg(src + v);
        float4 o;
        o.x = __fmul_rn(__fmul_rn(a.x, rr), Num<W>::to_f(nw[4 * v + 0]));
        o.y = __fmul_rn(__fmul_rn(a.y, rr), Num<W>::to_f(nw[4 * v + 1]));
        o.z = __fmul_rn(__fmul_rn(a.z, rr), Num<W>::to_f(nw[4 * v + 2]));
        o.w = __fmul_rn(__fmul_rn(a.w, rr), Num<W>::to_f(nw[4 * v + 3]));
        dst[v] = o;
      }
    } else {
      for (int v = v0 + lane; v < v1; v += 32) dst[v] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  __syncthreads();

  // K = 4096 (every unit 128 float4 per row): the next unit's 16 loads are
  // issued as soon as this unit's FMAs have consumed the registers, so they
  // are in flight during its butterfly and partial-table write (71.1 against
  // 74.2 us for the 7B op shape; issuing each half as soon as its registers
  // free up measured 73.2)
  const bool common = kv % F32_KPARTS == 0 && kv / F32_KPARTS == 4 * 32;
  for (int rp0 = p_begin; rp0 < p_end; rp0 += F32_ROUND_PAIRS) {
    const int np = min(F32_ROUND_PAIRS, p_end - rp0);
    if (common) {
      const int nu = np * F32_KPARTS;
      float4 w[4][4];
      auto load_unit = [&](int u, int half) {  // float4 columns 2*half, 2*half+1 of each row
        const float* r[4];
        unit_rows(rp0 + u / F32_KPARTS, r);
        const int va = (u % F32_KPARTS) * (kv / F32_KPARTS);
#pragma unroll
        for (int i = 2 * half; i < 2 * half + 2; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            w[i][j] = __ldg(reinterpret_cast<const float4*>(r[j]) + va + lane + 32 * i);
      };
      int u = warp;
      if (u < nu) {
        load_unit(u, 0);
        load_unit(u, 1);
      }
      while (u < nu) {
        const int va = (u % F32_KPARTS) * (kv / F32_KPARTS);
        const int un = u + F32_WARPS;
        float acc[32];  // [row j][token t] at 8 * j + t
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int v = va + lane + 32 * i;
#pragma unroll
          for (int t = 0; t < F32_ROWS; ++t) {
            const float4 a = xs4[(int64_t)t * kv + v];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float sacc = acc[8 * j + t];
              sacc = fmaf(w[i][j].x, a.x, sacc);
              sacc = fmaf(w[i][j].y, a.y, sacc);
              sacc = fmaf(w[i][j].z, a.z, sacc);
              sacc = fmaf(w[i][j].w, a.w, sacc);
              acc[8 * j + t] = sacc;
            }
          }
          // a half of the registers is free: the next unit's half goes out now
        }
        if (un < nu) {
          load_unit(un, 0);
          load_unit(un, 1);
        }
        const float tot = warp_transpose_sum32(acc, lane);
        part[u * 32 + lane] = tot;  // u = pl * F32_KPARTS + kp
        u = un;
      }
    } else
    for (int u = warp; u < np * F32_KPARTS; u += F32_WARPS) {
      const int pl = u / F32_KPARTS, kp = u % F32_KPARTS;
      const float* r[4];
      unit_rows(rp0 + pl, r);
      const int va = (int)((int64_t)kp * kv / F32_KPARTS), vb = (int)((int64_t)(kp + 1) * kv / F32_KPARTS);
      float acc[32];  // [row j][token t] at 8 * j + t
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = 0.f;
      auto fma_step = [&](const float4 (&w)[4], int v) {
#pragma unroll
        for (int t = 0; t < F32_ROWS; ++t) {
          const float4 a = xs4[(int64_t)t * kv + v];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float s = acc[8 * j + t];
            s = fmaf(w[j].x, a.x, s);
            s = fmaf(w[j].y, a.y, s);
            s = fmaf(w[j].z, a.z, s);
            s = fmaf(w[j].w, a.w, s);
            acc[8 * j + t] = s;
          }
        }
      };
      if (vb - va == 4 * 32) {
        // the common case (K = 4096): all 16 loads of the unit in flight at once
        float4 w[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            w[i][j] = __ldg(reinterpret_cast<const float4*>(r[j]) + va + lane + 32 * i);
#pragma unroll
        for (int i = 0; i < 4; ++i) fma_step(w[i], va + lane + 32 * i);
      } else {
#pragma unroll 2
        for (int v = va + lane; v < vb; v += 32) {
          float4 w[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) w[j] = __ldg(reinterpret_cast<const float4*>(r[j]) + v);
          fma_step(w, v);
        }
      }
      const float tot = warp_transpose_sum32(acc, lane);
      part[(pl * F32_KPARTS + kp) * 32 + lane] = tot;
    }
    __syncthreads();
    // outputs of the round: (token t, column c) with c fastest
    const int ncols = min(2 * np, I - 2 * rp0);
    for (int o = threadIdx.x; o < rows * ncols; o += blockDim.x) {
      const int t = o / ncols, c = o - t * ncols;
      const int pl = c >> 1, side = c & 1;  // row j: 2*side (gate), 2*side+1 (up)
      const float* pp = part + pl * F32_KPARTS * 32;
      float g = 0.f, uu = 0.f;
#pragma unroll
      for (int kp = 0; kp < F32_KPARTS; ++kp) {
        g += pp[kp * 32 + 8 * (2 * side) + t];
        uu += pp[kp * 32 + 8 * (2 * side + 1) + t];
      }
      out[(m0 + t) * I + 2 * rp0 + c] = (g / (1.0f + expf(-g))) * uu;
    }
    __syncthreads();
  }
}

template <typename W>
int launch_f32(const void* x, const void* nw, const void* gw, const void* uw, void* out,
               int64_t M, int K, int I, float eps, cudaStream_t s) {
  const size_t smem = (size_t)F32_ROWS * K * sizeof(float) + (size_t)F32_PART_FLOATS * sizeof(float);
  if (smem > 220 * 1024) {
    lpc::set_error("rmsswiglu_forward (fp32): dim %d too large for the fp32 path", K);
    return LPC_ERR_UNSUPPORTED;
  }
  if (M > 65535LL * F32_ROWS) {
    lpc::set_error("rmsswiglu_forward (fp32): at most %lld tokens", 65535LL * F32_ROWS);
    return LPC_ERR_UNSUPPORTED;
  }
  auto kfn = swiglu_f32_kernel<W>;
  static std::atomic<uint64_t> f32_mask{0};
  int rcx = lpc::once_per_device_smem((const void*)kfn, 220 * 1024, f32_mask);
  if (rcx) return rcx;
  const float* g = (const float*)gw;
  const float* u = uw ? (const float*)uw : g + (int64_t)I * K;
  const int pairs = (I + 1) / 2;
  const int gx = std::max(1, std::min(lpc::current_device_sms(), pairs));
  const int64_t gy = (M + F32_ROWS - 1) / F32_ROWS;
  dim3 grid((unsigned)gx, (unsigned)gy);
  kfn<<<grid, F32_WARPS * 32, smem, s>>>((const float*)x, (const W*)nw, g, u, (float*)out, M, K, I,
                                         eps);
  return lpc::check_launch("rmsswiglu_forward (fp32)");
}

template <typename T, int MT, int STAGES>
int launch_tc_cfg(const lpc::TmaDesc& ta, const lpc::TmaDesc& tg, const lpc::TmaDesc& tu, void* out,
                  int64_t M, int K, int I, int up_off, int dtype, cudaStream_t s) {
  constexpr int smem = tc_smem<MT, STAGES>();
  static std::atomic<uint64_t> mask{0};
  int rc = lpc::once_per_device_smem((const void*)swiglu_tc_kernel<T, MT, STAGES>, smem, mask);
  if (rc) return rc;
  const int num_m = (int)((M + BM * MT - 1) / (BM * MT));  // groups of MT token tiles
  const int num_n = (I + BNI - 1) / BNI;
  const uint32_t idesc = lpc::idesc_f16(dtype == LPC_DTYPE_BF16 ? 1u : 0u, BM, BN, 0u, 0u);
  swiglu_tc_kernel<T, MT, STAGES><<<(unsigned)((int64_t)num_m * num_n), 192, smem, s>>>(
      ta, tg, tu, (T*)out, (int)M, K, I, up_off, num_m, num_n, idesc);
  return lpc::check_launch("rmsswiglu_forward (tcgen05)");
}

// Tile shape by token count, measured on B200 for the 7B layer (dim 4096,
// inter 11008) in steady state (launches back to back over weights larger
// than L2; each figure includes the row-norm launch), us:
//   tokens   1-CTA 1x3   1-CTA 2x2   1-CTA 1x6   pair, 160-wide   pair, 256-wide
//   128         46.3        66.4        55.1         48.2              --
//   256         69.8        69.0        74.1         48.6             59.6
//   1024       166.3       173.2       217.3        150.7            158.9
//   2048       315.6       294.9       401.8        289.3            264.3
//   4096       621.2       617.5       876.7        568.3            534.9
// (the pair kernel with 128-column tiles, 86 pairs, took 59.6 / 153.1 / 266.2
// / 519.9 at 256 / 1024 / 2048 / 4096 tokens.)  Up to 128 tokens the one-CTA
// tile with two ~96 KB CTAs per SM keeps every weight tile streaming at once;
// beyond, the CTA pair halves the activation bytes per weight byte (and the
// shared-memory operand traffic per MMA).  LPC_SWIGLU_CFG=1..5 forces a
// column of this table (measurement and tests).

// Inter tiles for the pair kernel: the count C minimising the modelled time
// waves x per-tile time, with one CTA pair per two SMs per wave (the kernel's
// shared memory admits one CTA per SM).  A tile is bound by its loads (the
// token rows and the full weight boxes per k-block, whatever its width):
// measured on B200 at 2048-4096 tokens, about 1050 clocks per k-block with
// 160-column boxes and 1540 with 256-column boxes, above the two MMAs (4
// clocks per column).  Tiles are 128..wmax wide.  Returns the cost in clocks
// per k-block.
int64_t pair_tiles(int64_t num_m, int I, int wmax, int* num_c) {
  const int64_t load = wmax <= 160 ? 1050 : 1540;
  const int units = I / 16;
  const int cmin = (units + wmax / 16 - 1) / (wmax / 16);
  const int cmax = std::max(cmin, units / 8);  // widths >= 128
  const int64_t per_wave = std::max(1, lpc::current_device_sms() / 2);
  int best = cmin;
  int64_t best_cost = -1;
  for (int c = cmin; c <= cmax; ++c) {
    const int64_t waves = (num_m * c + per_wave - 1) / per_wave;
    const int64_t widest = 16 * ((units + c - 1) / c);
    const int64_t cost = waves * std::max(load, 4 * widest);
    if (best_cost < 0 || cost < best_cost) {
      best = c;
      best_cost = cost;
    }
  }
  *num_c = best;
  return best_cost;
}

template <typename T, int WMAX, int STAGES, bool NORM = false>
int launch_pair(const lpc::TmaDesc& ta, const void* gw, const void* uw, void* out, int64_t M, int K,
                int I, int dtype, cudaStream_t s, float eps = 0.f) {
  constexpr int BROWS = PairGeom<WMAX>::BROWS;
  lpc::TmaDesc tg, tu;
  int rc, up_off = 0;
  if (uw) {
    if ((rc = lpc::make_tma_2d(&tg, gw, dtype, K, (uint64_t)I, (uint64_t)K * 2, BK, BROWS, true))) return rc;
    if ((rc = lpc::make_tma_2d(&tu, uw, dtype, K, (uint64_t)I, (uint64_t)K * 2, BK, BROWS, true))) return rc;
  } else {
    if ((rc = lpc::make_tma_2d(&tg, gw, dtype, K, (uint64_t)2 * I, (uint64_t)K * 2, BK, BROWS, true))) return rc;
    tu = tg;
    up_off = I;
  }
  constexpr int smem = pair_smem<WMAX, STAGES>();
  static std::atomic<uint64_t> mask{0};
  if ((rc = lpc::once_per_device_smem((const void*)swiglu_pair_kernel<T, WMAX, STAGES, NORM>, smem, mask)))
    return rc;
  const int num_m = (int)((M + PAIR_TOK - 1) / PAIR_TOK);
  int num_c = 0;
  pair_tiles(num_m, I, WMAX, &num_c);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * (int64_t)num_m * num_c));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  // programmatic stream serialisation: the set-up and the first weight boxes
  // overlap the row norm launched just before by this call
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, swiglu_pair_kernel<T, WMAX, STAGES, NORM>, ta, tg, tu,
                                     (T*)out, (int)M, K, I, up_off, num_m, num_c,
                                     dtype == LPC_DTYPE_BF16 ? 1u : 0u, eps);
  if (e != cudaSuccess) {
    lpc::set_error("rmsswiglu_forward (tcgen05 pair): launch failed: %s", cudaGetErrorString(e));
    return LPC_ERR_CUDA;
  }
  return lpc::check_launch("rmsswiglu_forward (tcgen05 pair)");
}

// The pair kernel with the cheaper of the 160- and 256-column tilings.
template <typename T, bool NORM = false>
int launch_pair_auto(const lpc::TmaDesc& ta, const void* gw, const void* uw, void* out, int64_t M,
                     int K, int I, int dtype, cudaStream_t s, float eps = 0.f) {
  const int64_t num_m = (M + PAIR_TOK - 1) / PAIR_TOK;
  int c160 = 0, c256 = 0;
  const int64_t cost160 = pair_tiles(num_m, I, 160, &c160);
  const int64_t cost256 = pair_tiles(num_m, I, 256, &c256);
  if (cost256 < cost160) return launch_pair<T, 256, 4, NORM>(ta, gw, uw, out, M, K, I, dtype, s, eps);
  return launch_pair<T, 160, 5, NORM>(ta, gw, uw, out, M, K, I, dtype, s, eps);
}

template <typename T>
int launch_tc(const void* xn, const void* gw, const void* uw, void* out, int64_t M, int K, int I,
              int dtype, cudaStream_t s) {
  lpc::TmaDesc ta, tg, tu;
  int rc = lpc::make_tma_2d(&ta, xn, dtype, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, BM, true);
  if (rc) return rc;
  int up_off = 0;
  if (uw) {
    if ((rc = lpc::make_tma_2d(&tg, gw, dtype, K, (uint64_t)I, (uint64_t)K * 2, BK, BNI, true))) return rc;
    if ((rc = lpc::make_tma_2d(&tu, uw, dtype, K, (uint64_t)I, (uint64_t)K * 2, BK, BNI, true))) return rc;
  } else {
    if ((rc = lpc::make_tma_2d(&tg, gw, dtype, K, (uint64_t)2 * I, (uint64_t)K * 2, BK, BNI, true))) return rc;
    tu = tg;
    up_off = I;
  }
  const char* force = getenv("LPC_SWIGLU_CFG");  // tile-selection override for measurements
  const int cfg = force ? atoi(force) : 0;
  if (cfg == 1) return launch_tc_cfg<T, 1, 3>(ta, tg, tu, out, M, K, I, up_off, dtype, s);
  if (cfg == 2) return launch_tc_cfg<T, 2, 2>(ta, tg, tu, out, M, K, I, up_off, dtype, s);
  if (cfg == 3) return launch_tc_cfg<T, 1, 6>(ta, tg, tu, out, M, K, I, up_off, dtype, s);
  if (cfg == 4) return launch_pair<T, 160, 5>(ta, gw, uw, out, M, K, I, dtype, s);
  if (cfg == 5) return launch_pair<T, 256, 4>(ta, gw, uw, out, M, K, I, dtype, s);
  if (M <= 128) return launch_tc_cfg<T, 1, 3>(ta, tg, tu, out, M, K, I, up_off, dtype, s);
  return launch_pair_auto<T>(ta, gw, uw, out, M, K, I, dtype, s);
}

}  // namespace

extern "C" int64_t lpc_rmsswiglu_workspace_bytes(int64_t tokens, int dim, int dtype) {
  if (dtype == LPC_DTYPE_F32 || tokens <= 0 || dim <= 0) return 0;
  return tokens * (int64_t)dim * 2;
}

extern "C" int lpc_rmsswiglu_forward(const void* x, const void* rms_weight, const void* gate_w,
                                     const void* up_w, void* out, void* workspace,
                                     int64_t workspace_bytes, int64_t tokens, int dim, int inter,
                                     float eps, int dtype, int w_dtype, void* stream) {
  using namespace lpc;
  if (!(eps > 0.f)) {
    set_error("rmsswiglu_forward: eps must be strictly positive.");
    return LPC_ERR_INVALID;
  }
  if (tokens < 0 || dim <= 0 || inter <= 0) {
    set_error("rmsswiglu_forward: invalid sizes (tokens=%lld dim=%d inter=%d)", (long long)tokens,
              dim, inter);
    return LPC_ERR_INVALID;
  }
  if (tokens == 0) return LPC_OK;
  if (!x || !rms_weight || !gate_w || !out) {
    set_error("rmsswiglu_forward: null pointer");
    return LPC_ERR_INVALID;
  }
  if (!aligned16(x) || !aligned16(gate_w) || (up_w && !aligned16(up_w)) || !aligned16(out)) {
    set_error("rmsswiglu_forward: tensors must be 16-byte aligned");
    return LPC_ERR_INVALID;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LPC_DTYPE_F32) {
    if (dim % 4) {
      set_error("rmsswiglu_forward (fp32): dim must be a multiple of 4");
      return LPC_ERR_UNSUPPORTED;
    }
    switch (w_dtype) {
      case LPC_DTYPE_F32: return launch_f32<float>(x, rms_weight, gate_w, up_w, out, tokens, dim, inter, eps, s);
      case LPC_DTYPE_BF16: return launch_f32<__nv_bfloat16>(x, rms_weight, gate_w, up_w, out, tokens, dim, inter, eps, s);
      case LPC_DTYPE_F16: return launch_f32<__half>(x, rms_weight, gate_w, up_w, out, tokens, dim, inter, eps, s);
    }
    set_error("rmsswiglu_forward: unsupported weight dtype %d", w_dtype);
    return LPC_ERR_UNSUPPORTED;
  }
  if (dtype != LPC_DTYPE_BF16 && dtype != LPC_DTYPE_F16) {
    set_error("rmsswiglu_forward: unsupported dtype %d", dtype);
    return LPC_ERR_UNSUPPORTED;
  }
  if (dim % BK || inter % 16) {
    set_error("rmsswiglu_forward: tensor-core path needs dim %% 64 == 0 and inter %% 16 == 0 "
              "(dim=%d inter=%d)", dim, inter);
    return LPC_ERR_UNSUPPORTED;
  }
  if (tokens > 0x7fffffffLL) {
    set_error("rmsswiglu_forward: too many tokens");
    return LPC_ERR_UNSUPPORTED;
  }
  const int64_t need = lpc_rmsswiglu_workspace_bytes(tokens, dim, dtype);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
    set_error("rmsswiglu_forward: workspace of %lld bytes (16-byte aligned) required, got %lld",
              (long long)need, (long long)workspace_bytes);
    return LPC_ERR_INVALID;
  }
  int rc = lpc_rmsnorm_launch(x, rms_weight, workspace, tokens, dim, eps, dtype, w_dtype, s);
  if (rc) return rc;
  if (dtype == LPC_DTYPE_BF16)
    return launch_tc<__nv_bfloat16>(workspace, gate_w, up_w, out, tokens, dim, inter, dtype, s);
  return launch_tc<__half>(workspace, gate_w, up_w, out, tokens, dim, inter, dtype, s);
}

// RMSNorm + SwiGLU in one kernel when the norm weight is already folded into
// the gate/up weights (W diag(w), e.g. once at model load): the CTA-pair
// kernel reads the raw rows x, takes each row's sum of squares from the A
// tiles it feeds the tensor core and scales the accumulators in the epilogue.
extern "C" int lpc_rmsswiglu_folded_forward(const void* x, const void* gate_w, const void* up_w,
                                            void* out, int64_t tokens, int dim, int inter,
                                            float eps, int dtype, void* stream) {
  using namespace lpc;
  if (!(eps > 0.f)) {
    set_error("rmsswiglu_folded_forward: eps must be strictly positive.");
    return LPC_ERR_INVALID;
  }
  if (tokens < 0 || dim <= 0 || inter <= 0) {
    set_error("rmsswiglu_folded_forward: invalid sizes (tokens=%lld dim=%d inter=%d)",
              (long long)tokens, dim, inter);
    return LPC_ERR_INVALID;
  }
  if (tokens == 0) return LPC_OK;
  if (dtype != LPC_DTYPE_BF16 && dtype != LPC_DTYPE_F16) {
    set_error("rmsswiglu_folded_forward: bf16 or fp16 only");
    return LPC_ERR_UNSUPPORTED;
  }
  if (dim % BK || inter % 16 || tokens > 0x7fffffffLL) {
    set_error("rmsswiglu_folded_forward: needs dim %% 64 == 0 and inter %% 16 == 0 (dim=%d "
              "inter=%d)", dim, inter);
    return LPC_ERR_UNSUPPORTED;
  }
  if (!x || !gate_w || !out || !aligned16(x) || !aligned16(gate_w) || (up_w && !aligned16(up_w)) ||
      !aligned16(out)) {
    set_error("rmsswiglu_folded_forward: null or misaligned pointer");
    return LPC_ERR_INVALID;
  }
  lpc::TmaDesc ta;
  int rc = lpc::make_tma_2d(&ta, x, dtype, (uint64_t)dim, (uint64_t)tokens, (uint64_t)dim * 2, BK,
                            BM, true);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LPC_DTYPE_BF16)
    return launch_pair_auto<__nv_bfloat16, true>(ta, gate_w, up_w, out, tokens, dim, inter, dtype, s, eps);
  return launch_pair_auto<__half, true>(ta, gate_w, up_w, out, tokens, dim, inter, dtype, s, eps);
}
