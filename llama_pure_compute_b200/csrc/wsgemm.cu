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
//   * One CTA per weight tile, the whole K.  Layers with few tiles (tens)
//     leave SMs idle: this kernel is meant for the wide projections.
// Measured on B200 in steady state (launches back to back over weights larger
// than L2), SwiGLU gate/up of the 7B layer (2 x 11008 x 4096): 33.6 us at 32
// tokens, 35.3 us at 64, 41.8 us at 128 -- against 44-46 us for the
// activation-major tile of the fused rmsswiglu op on the raw weights.
// Epilogues: plain store, residual add (out = resid + acc, may alias), and
// SwiGLU on weights packed with 16 gate rows / 16 up rows interleaved.
//   warp 0    producer: bulk copy of the weight chunk + TMA box of activations
//   warp 2    TMEM allocator + single-thread tcgen05.mma issuer
//   warps 4-7 epilogue (TMEM lane = weight row)
#include <atomic>

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

enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2 };

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// ---------------------------------------------------------------------------
// Packing: packed[tile][kb] = swizzled image of rows tile*128.. x k kb*64..
// layout 0: row r of W0 (rows >= n_rows are zero)
// layout 1 (SwiGLU): tile tau covers inter columns 64*tau..; tile row
//   32q + l is gate row 64*tau + 16q + l (l < 16) or up row 64*tau + 16q + l-16;
//   gate rows from W0, up rows from W1 (or W0 rows n_rows.. when W1 is null).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) pack_kernel(const T* __restrict__ w0,
                                                   const T* __restrict__ w1,
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
    if (layout == 0) {
      const int64_t row = (int64_t)tile * TILE_ROWS + r;
      if (row < n_rows) src = w0 + row * K + k;
    } else {
      const int q = r >> 5, l = r & 31;
      const int64_t col = (int64_t)tile * 64 + 16 * q + (l & 15);
      if (col < n_rows) {
        if (l < 16) src = w0 + col * K + k;
        else src = w1 ? w1 + col * K + k : w0 + (n_rows + col) * K + k;
      }
    }
    packed[idx] = src ? *reinterpret_cast<const uint4*>(src) : make_uint4(0, 0, 0, 0);
  }
}

// ---------------------------------------------------------------------------
// GEMM: one CTA per weight tile
// ---------------------------------------------------------------------------
template <typename T, int EPI>
__global__ void __launch_bounds__(THREADS, 2)
    wsgemm_kernel(const __grid_constant__ lpc::TmaDesc tmX, const uint8_t* __restrict__ packed,
                  T* out, const T* resid, int M, int K, int n_out, int NT, int stages,
                  uint32_t tmem_cols, uint32_t idesc) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = lpc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t x_bytes = (uint32_t)NT * KB * 2;
  const uint32_t stage_bytes = CHUNK + ((x_bytes + 1023u) & ~1023u);
  const uint32_t bars = base + (uint32_t)stages * stage_bytes;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (stages + s); };
  const uint32_t accum = bars + 8u * (2 * stages);
  const uint32_t tmem_slot = accum + 8u;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int nkb = K / KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      lpc::mbar_init(full_bar(s), 1);
      lpc::mbar_init(empty_bar(s), 1);
    }
    lpc::mbar_init(accum, 1);
    lpc::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) lpc::tma_prefetch_desc(&tmX);
  if (warp == 2) {
    lpc::tmem_alloc(tmem_slot, tmem_cols);
    lpc::tmem_relinquish();
  }
  lpc::tc_fence_before();
  __syncthreads();
  lpc::tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;
  unsigned int* st = &g_ws_status;

  if (warp == 0) {
    if (lane == 0) {
      const uint8_t* wsrc = packed + (int64_t)tile * nkb * CHUNK;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        if (!lpc::mbar_wait(empty_bar(s), ((uint32_t)(i / stages) & 1u) ^ 1u, st)) break;
        lpc::mbar_arrive_expect_tx(full_bar(s), CHUNK + x_bytes);
        const uint32_t dst = base + (uint32_t)s * stage_bytes;
        lpc::bulk_g2s(dst, wsrc + (int64_t)i * CHUNK, CHUNK, full_bar(s));
        lpc::tma_load_2d(dst + CHUNK, &tmX, i * KB, 0, full_bar(s));
      }
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
  } else if (warp >= 4) {
    const int q = warp & 3;  // TMEM lane quadrant = tile rows 32q .. 32q+31
    const bool ok = lpc::mbar_wait(accum, 0, st);
    lpc::tc_fence_after();
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < NT; c += 16) {
        uint32_t v[16];
        lpc::tmem_ld16(taddr + c, v);
        lpc::tmem_wait_ld();
        if (EPI == EPI_SWIGLU) {
          // lanes l and l^16 hold the gate and up rows of one inter column
          const bool is_gate = lane < 16;
          const int col = tile * 64 + 16 * q + (lane & 15);
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float mlo = __uint_as_float(v[i]), mhi = __uint_as_float(v[8 + i]);
            const float olo = __shfl_xor_sync(0xffffffffu, mlo, 16);
            const float ohi = __shfl_xor_sync(0xffffffffu, mhi, 16);
            o[i] = is_gate ? silu_mul(mlo, olo) : silu_mul(ohi, mhi);
          }
          const int tok0 = c + (is_gate ? 0 : 8);
          if (col < n_out) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (tok0 + i < M) out[(int64_t)(tok0 + i) * n_out + col] = Num<T>::from_f(o[i]);
          }
        } else {
          const int n = tile * TILE_ROWS + 32 * q + lane;  // output column of this lane
          if (n < n_out) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int t = c + i;
              if (t < M) {
                float a = __uint_as_float(v[i]);
                if (EPI == EPI_RESIDUAL) a += Num<T>::to_f(resid[(int64_t)t * n_out + n]);
                out[(int64_t)t * n_out + n] = Num<T>::from_f(a);
              }
            }
          }
        }
      }
    }
  }
  lpc::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    lpc::tc_fence_after();
    lpc::tmem_dealloc(tmem, tmem_cols);
  }
}

struct Plan {
  int n_tiles, NT, stages, smem;
  uint32_t tmem_cols;
};

Plan make_plan(int64_t M, int64_t n_out, int epilogue) {
  Plan p;
  p.n_tiles = (int)(epilogue == EPI_SWIGLU ? (n_out + 63) / 64 : (n_out + TILE_ROWS - 1) / TILE_ROWS);
  p.NT = (int)((M + 15) / 16) * 16;
  const int stage_bytes = CHUNK + ((p.NT * KB * 2 + 1023) & ~1023);
  p.stages = std::max(2, std::min(8, SMEM_TARGET / stage_bytes));
  p.smem = p.stages * stage_bytes + 1024 + 8 * (2 * p.stages + 4);
  p.tmem_cols = 32;
  while ((int)p.tmem_cols < p.NT) p.tmem_cols <<= 1;
  return p;
}

template <typename T, int EPI>
int launch(const void* x, const void* packed, void* out, const void* resid, int64_t M,
           int64_t n_out, int K, int dtype, cudaStream_t s) {
  const Plan p = make_plan(M, n_out, EPI);
  lpc::TmaDesc tx;
  int rc = lpc::make_tma_2d(&tx, x, dtype, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, KB,
                            (uint32_t)p.NT, true);
  if (rc) return rc;
  static std::atomic<uint64_t> mask{0};
  if ((rc = lpc::once_per_device_smem((const void*)wsgemm_kernel<T, EPI>, 227 * 1024, mask)))
    return rc;
  const uint32_t idesc =
      lpc::idesc_f16(dtype == LPC_DTYPE_BF16 ? 1u : 0u, TILE_ROWS, (uint32_t)p.NT, 0u, 0u);
  wsgemm_kernel<T, EPI><<<(unsigned)p.n_tiles, THREADS, p.smem, s>>>(
      tx, (const uint8_t*)packed, (T*)out, (const T*)resid, (int)M, K, (int)n_out, p.NT, p.stages,
      p.tmem_cols, idesc);
  return lpc::check_launch("wsgemm");
}

template <typename T>
int launch_epi(int epilogue, const void* x, const void* packed, void* out, const void* resid,
               int64_t M, int64_t n_out, int K, int dtype, cudaStream_t s) {
  switch (epilogue) {
    case EPI_STORE: return launch<T, EPI_STORE>(x, packed, out, resid, M, n_out, K, dtype, s);
    case EPI_RESIDUAL: return launch<T, EPI_RESIDUAL>(x, packed, out, resid, M, n_out, K, dtype, s);
    case EPI_SWIGLU: return launch<T, EPI_SWIGLU>(x, packed, out, resid, M, n_out, K, dtype, s);
  }
  lpc::set_error("wsgemm: unknown epilogue %d", epilogue);
  return LPC_ERR_INVALID;
}

}  // namespace

extern "C" int64_t lpc_packed_weight_bytes(int64_t n_out, int k, int layout) {
  if (n_out <= 0 || k <= 0 || k % KB) return 0;
  const int64_t tiles = layout == 1 ? (n_out + 63) / 64 : (n_out + TILE_ROWS - 1) / TILE_ROWS;
  return tiles * (k / KB) * (int64_t)CHUNK;
}

extern "C" int lpc_pack_weights(const void* w0, const void* w1, void* packed, int64_t n_out, int k,
                                int layout, int dtype, void* stream) {
  using namespace lpc;
  if (n_out <= 0 || k <= 0 || k % KB || (layout != 0 && layout != 1)) {
    set_error("pack_weights: need n_out > 0, k a multiple of 64 and layout 0 or 1");
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
                                                      (uint4*)packed, n_out, k, n_tiles, layout);
  else
    pack_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)w0, (const __half*)w1, (uint4*)packed,
                                               n_out, k, n_tiles, layout);
  return check_launch("pack_weights");
}

extern "C" int lpc_wsgemm(const void* x, const void* packed_w, void* out, const void* resid,
                          int64_t tokens, int64_t n_out, int k, int epilogue, int dtype,
                          void* stream) {
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LPC_DTYPE_BF16)
    return launch_epi<__nv_bfloat16>(epilogue, x, packed_w, out, resid, tokens, n_out, k, dtype, s);
  return launch_epi<__half>(epilogue, x, packed_w, out, resid, tokens, n_out, k, dtype, s);
}
