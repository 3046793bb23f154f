// Flash attention for prefill on tcgen05 tensor cores (sm_100a).
//
// out = softmax(Q K^T * scale + mask) V, fp32 accumulation, queries aligned to
// the end of the keys (bottom-right causal mask: query row r of a q_len-row
// block attends keys <= kv_len - q_len + r), as in
// tests/test_attention_correctness.py:10-76 and the causal prefill kernel of
// src/llama_pure_compute/triton_kernels/flash_attention.py:88-432.
//
// Persistent: one CTA per SM loops over work items (256 queries = two
// 128-row tiles, head, batch), longest causal blocks first, dealt to the CTAs
// in snake order; the next item's Q/K/V loads and first QK^T MMAs overlap the
// current item's last tiles and epilogue (one CTA holds all 512 TMEM columns,
// so consecutive CTAs on an SM could not overlap).  12 warps, 3 warpgroups;
// warpgroup 2 (warps 8-11) gives registers to the two softmax warpgroups
// (setmaxnreg: 96 and 200 per thread from the launch's 168):
//   warp 8     TMA producer: Q0/Q1 once (64-column boxes), then K and V
//              128-key tiles into 2-stage rings (4-D tensor maps: rows past
//              kv_len / q_len read as zeros).  K/V tiles serve both Q tiles.
//   warps 10-11 idle
//   warp 9     TMEM allocator and single-thread tcgen05.mma issuer, per key tile j:
//                S0 = Q0 K_j^T, S1 = Q1 K_j^T        (M=128, N=128, K=128)
//                O0 += P0 V_j, O1 += P1 V_j          (A = P from TMEM, B = V, MN-major;
//                                                     keys 0-63 as soon as their P is stored)
//   warps 0-3  softmax for Q0, warps 4-7 softmax for Q1 (ping-pong: while one
//              warpgroup exponentiates, the tensor core runs the other tile's
//              MMAs).  Thread r of a warpgroup owns query row r (TMEM lane r):
//              one tcgen05.ld of its 128 scores, exp2 in fp32 against the
//              running max straight away (only the first key tile of an item
//              reduces its row max), P rounded to bf16/fp16 and stored back
//              into the first 64 columns of its own S buffer (two 16-bit
//              values per column), the A operand of the PV MMA.  P of the
//              first 64 keys is released (its own barrier) before the last 64
//              are exponentiated, so half of PV overlaps them.  Before that
//              release a warp checks for a max grown by more than 8 (log2
//              units): a first-half row sum above 2^8, or the second half's
//              max.  Such warps (rare) reduce the tile's max, move the
//              running max, redo the row's exponentials from S (still in
//              TMEM), rescale O and release all of P at once.  The result is
//              the same softmax, only the reference point of the exponentials
//              differs.  Epilogue: O / l.
// TMEM (512 columns): S0/P0 [0,128), S1/P1 [128,256), O0 [256,384), O1 [384,512).
// MMAs issued by one thread execute in order, so S_t of key tile j+1 never
// overwrites P_t of tile j before PV_t(j) has read it.
// Causal key tiles past the diagonal are skipped.  Barrier phases are counted
// across items: q_empty (all S MMAs of an item done with Q) releases the Q
// buffer for the next item, o_free (epilogue has read O_t) gates its first PV_t.
#include <atomic>
#include <cstdlib>

#include "lpc_common.cuh"

LPC_DECLARE_STATUS(g_prefill_status)

unsigned int lpc_status_prefill(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_prefill_status, sizeof(v));
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_prefill_status, &z, sizeof(z));
  }
  return v;
}

namespace {

constexpr int BQ = 128;                   // queries per tile (UMMA M)
constexpr int NQT = 2;                    // query tiles per CTA
constexpr int BKV = 128;                  // keys per tile
constexpr int BOX = 64;                   // 64 x 2 B = one 128-byte swizzle row
constexpr int HALF_BYTES = BQ * BOX * 2;  // 16 KB: 128 rows x one 64-column box
constexpr int KV_STAGES = 2;
// head_dim HD (64 or 128): a Q tile, a K stage and a V stage are HD / 64
// boxes of 128 rows x 64 columns
template <int HD>
constexpr int tile_bytes() { return (HD / BOX) * HALF_BYTES; }
template <int HD>
constexpr int smem_bytes() { return (NQT + 2 * KV_STAGES) * tile_bytes<HD>() + 1024 + 256; }
constexpr int NTHREADS = 384;  // 2 softmax warpgroups + 1 load/MMA warpgroup
constexpr uint32_t TMEM_COLS = 512;
constexpr float LOG2E = 1.4426950408889634f;
// A row whose max grew by more than RESCALE_LOG2 (log2 units) past its
// reference has a row sum above RESCALE_LIMIT = 2^RESCALE_LOG2: such rows
// reduce their max and redo the tile.
constexpr float RESCALE_LOG2 = 8.0f;
constexpr float RESCALE_LIMIT = 256.0f;

struct TmaDesc4 { alignas(64) unsigned char bytes[128]; };

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, int c0, int c1, int c2,
                                            int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (Blackwell f32x2 FMA/ADD: two lanes of work per instruction).
__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t pack_u2(uint32_t lo, uint32_t hi) {
  return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

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

struct Params {
  int64_t q_len, kv_len, offset;  // offset = kv_len - q_len
  int heads, kv_heads, group, num_q_blocks, batch;
  int num_items;                  // num_q_blocks * heads * batch
  float scale_log2;
  int causal;
  int band;                       // (head, batch) pairs per band of the item order
};

// Work item `i`: the (head, batch) pairs are cut into bands of p.band pairs;
// within a band, items go longest first: query block (descending), then the
// band's pairs.  One band spanning every pair is plain longest-first order;
// narrower bands keep all query blocks of a head in flight together, so the
// head's K/V tiles are shared through L2 instead of re-read from HBM.
struct Item {
  int qb, h, b;
  int64_t q0;
  int n0, n1;  // key tiles needed by query tile 0 / 1 (tile 1 sees the most keys)
};

__device__ __forceinline__ Item decode_item(const Params& p, int i) {
  Item it;
  const int hb = p.heads * p.batch;
  const int bw = p.band;
  const int per_band = bw * p.num_q_blocks;
  const int band = i / per_band;
  const int first = band * bw;
  const int nb = min(bw, hb - first);  // pairs in this band
  const int within = i - band * per_band;
  it.qb = p.num_q_blocks - 1 - within / nb;
  const int r = first + within % nb;
  it.h = r % p.heads;
  it.b = r / p.heads;
  it.q0 = (int64_t)it.qb * (NQT * BQ);
  const int64_t all = (p.kv_len + BKV - 1) / BKV;
  int64_t n0 = all, n1 = all;
  if (p.causal) {
    n0 = min(all, (p.offset + it.q0 + BQ - 1) / BKV + 1);
    n1 = min(all, (p.offset + it.q0 + 2 * BQ - 1) / BKV + 1);
  }
  it.n0 = (int)n0;
  it.n1 = (int)n1;
  return it;
}

// The r-th work item of CTA c in a grid of G CTAs: rows of G items taken in
// snake order (c, 2G-1-c, 2G+c, ...), which balances longest-first items.
__device__ __forceinline__ int item_of(int c, int G, int r) {
  return r * G + ((r & 1) ? (G - 1 - c) : c);
}

constexpr int LAUNCH_REGS = 168;  // the register split below assumes this count
constexpr int SPLIT_REGS_LOADMMA = 96, SPLIT_REGS_SOFTMAX = 200;
static_assert(128 * SPLIT_REGS_LOADMMA + 256 * SPLIT_REGS_SOFTMAX <= NTHREADS * LAUNCH_REGS,
              "register split exceeds the block's launch allocation");

template <typename T, int HD>
__global__ void __launch_bounds__(NTHREADS, 1)
    flash_prefill_kernel(const __grid_constant__ TmaDesc4 tmQ, const __grid_constant__ TmaDesc4 tmK,
                         const __grid_constant__ TmaDesc4 tmV, T* __restrict__ out,
                         const Params p, uint32_t idesc_qk, uint32_t idesc_pv) {
  constexpr int TILE_BYTES = tile_bytes<HD>();
  constexpr int NBOX = HD / BOX;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = lpc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sQ = base;                                 // NQT tiles
  const uint32_t sK = base + NQT * TILE_BYTES;              // KV_STAGES
  const uint32_t sV = sK + KV_STAGES * TILE_BYTES;          // KV_STAGES
  const uint32_t bars = sV + KV_STAGES * TILE_BYTES;
  const uint32_t q_full = bars;
  const uint32_t q_empty = bars + 8u * 19;                   // all S MMAs of an item done with Q
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bars + 8u * (3 + s); };
  auto v_full = [&](int s) { return bars + 8u * (5 + s); };
  auto v_empty = [&](int s) { return bars + 8u * (7 + s); };
  auto s_full = [&](int t) { return bars + 8u * (9 + t); };
  auto p_full = [&](int t) { return bars + 8u * (11 + t); };
  auto o_done = [&](int t) { return bars + 8u * (13 + t); };
  auto o_free = [&](int t) { return bars + 8u * (15 + t); };  // epilogue has read O_t
  auto p_half = [&](int t) { return bars + 8u * (17 + t); };  // P_t of the first 64 keys stored
  const uint32_t tmem_slot = bars + 8u * 20;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = (int)gridDim.x;
  const int c = (int)blockIdx.x;

  if (threadIdx.x == 0) {
    lpc::mbar_init(q_full, 1);
    lpc::mbar_init(q_empty, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      lpc::mbar_init(k_full(s), 1);
      lpc::mbar_init(k_empty(s), 1);
      lpc::mbar_init(v_full(s), 1);
      lpc::mbar_init(v_empty(s), 1);
    }
    for (int t = 0; t < NQT; ++t) {
      lpc::mbar_init(s_full(t), 1);
      lpc::mbar_init(p_full(t), 4);
      lpc::mbar_init(p_half(t), 4);
      lpc::mbar_init(o_done(t), 1);
      lpc::mbar_init(o_free(t), 4);
    }
    lpc::fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    lpc::tma_prefetch_desc(&tmQ);
    lpc::tma_prefetch_desc(&tmK);
    lpc::tma_prefetch_desc(&tmV);
  }
  if (warp == 9) {
    lpc::tmem_alloc(tmem_slot, TMEM_COLS);
    lpc::tmem_relinquish();
  }
  lpc::tc_fence_before();
  __syncthreads();
  lpc::tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;
  unsigned int* st = &g_prefill_status;

  if (warp >= 8) {
  // Register split: warpgroup 2 (load, MMA, two idle warps) hands registers to
  // the softmax warpgroups.  At the launch's 168 registers per thread the
  // shares fit the block's total: 128 x 96 + 256 x 200 <= 384 x 168 (the host
  // refuses to launch with any other count).
  asm volatile("setmaxnreg.dec.sync.aligned.u32 96;\n" ::: "memory");
  if (warp == 8) {
    // ---------------- TMA producer ----------------
    // Q of the next item as soon as the last S MMA of the previous one is
    // done; K/V tiles through 2-stage rings counted across items.
    if (lane == 0) {
      bool ok = true;
      uint32_t kvc = 0;
      for (int r = 0, i = item_of(c, G, 0); i < p.num_items && ok; i = item_of(c, G, ++r)) {
        const Item it = decode_item(p, i);
        const int kvh = it.h / p.group;
        if (!(ok = lpc::mbar_wait(q_empty, ((uint32_t)r & 1u) ^ 1u, st))) break;
        lpc::mbar_arrive_expect_tx(q_full, NQT * TILE_BYTES);
        for (int t = 0; t < NQT; ++t)
#pragma unroll
          for (int hb = 0; hb < NBOX; ++hb)
            tma_load_4d(sQ + t * TILE_BYTES + hb * HALF_BYTES, &tmQ, hb * BOX,
                        (int)(it.q0 + t * BQ), it.h, it.b, q_full);
        for (int j = 0; j < it.n1; ++j, ++kvc) {
          const int s = kvc % KV_STAGES;
          const uint32_t par = ((kvc / KV_STAGES) & 1u) ^ 1u;
          const int k0 = j * BKV;
          if (!(ok = lpc::mbar_wait(k_empty(s), par, st))) break;
          lpc::mbar_arrive_expect_tx(k_full(s), TILE_BYTES);
#pragma unroll
          for (int hb = 0; hb < NBOX; ++hb)
            tma_load_4d(sK + s * TILE_BYTES + hb * HALF_BYTES, &tmK, hb * BOX, k0, kvh, it.b,
                        k_full(s));
          if (!(ok = lpc::mbar_wait(v_empty(s), par, st))) break;
          lpc::mbar_arrive_expect_tx(v_full(s), TILE_BYTES);
#pragma unroll
          for (int hb = 0; hb < NBOX; ++hb)
            tma_load_4d(sV + s * TILE_BYTES + hb * HALF_BYTES, &tmV, hb * BOX, k0, kvh, it.b,
                        v_full(s));
        }
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    // Per item, issue order per key tile j:  PV0(j), S0(j+1), PV1(j), S1(j+1).
    // While warpgroup 0 exponentiates S0(j+1) the tensor core runs PV1(j) and
    // S1(j+1), and the other way round.  Across items: S_t(0) of the next item
    // is issued right after the last PV_t of the current one; PV_t(0) waits
    // until the epilogue has read O_t (o_free).
    if (lane == 0) {
      bool ok = true;
      uint32_t kvc = 0, c0 = 0, c1 = 0;  // key tiles / S_0 tiles / S_1 tiles so far
      // Shared-memory descriptors, built once: a descriptor's start-address
      // field holds address >> 4, so a byte offset inside a tile is added as
      // offset >> 4 (16 elements along K: +2; next 64-column half: +HALF/16).
      const uint64_t dQ = lpc::smem_desc_sw128(sQ, 16, 1024);
      const uint64_t dK = lpc::smem_desc_sw128(sK, 16, 1024);
      const uint64_t dV = lpc::smem_desc_sw128(sV, HALF_BYTES, 1024);
      auto issue_s = [&](int t, uint32_t kv) -> bool {
        const int s = kv % KV_STAGES;
        if (!lpc::mbar_wait(k_full(s), (kv / KV_STAGES) & 1u, st)) return false;
        lpc::tc_fence_after();
        const uint64_t aq = dQ + (uint64_t)((t * TILE_BYTES) >> 4);
        const uint64_t bk = dK + (uint64_t)((s * TILE_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (uint32_t)(((kk >> 2) * HALF_BYTES) >> 4) + 2u * (kk & 3);
          lpc::umma_ss(tmem + 128u * t, aq + off, bk + off, idesc_qk, kk != 0);
        }
        lpc::umma_commit(s_full(t));
        return true;
      };
      auto issue_pv = [&](int t, uint32_t kv, uint32_t pc, bool first) -> bool {
        const int s = kv % KV_STAGES;
        // the first 64 keys' P is released before the softmax exponentiates
        // the other 64: their MMAs overlap it
        if (!lpc::mbar_wait(p_half(t), pc & 1u, st)) return false;
        if (!lpc::mbar_wait(v_full(s), (kv / KV_STAGES) & 1u, st)) return false;
        lpc::tc_fence_after();
        const uint64_t bv = dV + (uint64_t)((s * TILE_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          if (kk == BKV / 32) {
            if (!lpc::mbar_wait(p_full(t), pc & 1u, st)) return false;
            lpc::tc_fence_after();
          }
          // A: P_t in TMEM (16 keys = 8 columns of packed pairs); B: V rows = keys
          lpc::umma_ts(tmem + 256u + 128u * t, tmem + 128u * t + 8u * kk,
                       bv + (uint64_t)((kk * 16 * 128) >> 4), idesc_pv, (!first) || kk != 0);
        }
        lpc::umma_commit(o_done(t));
        return true;
      };
      for (int r = 0, i = item_of(c, G, 0); i < p.num_items && ok; i = item_of(c, G, ++r)) {
        const Item it = decode_item(p, i);
        if (!(ok = lpc::mbar_wait(q_full, (uint32_t)r & 1u, st))) break;
        lpc::tc_fence_after();
        if (!(ok = issue_s(0, kvc) && issue_s(1, kvc))) break;
        lpc::umma_commit(k_empty(kvc % KV_STAGES));
        if (it.n1 == 1) lpc::umma_commit(q_empty);  // the last S MMA of the item has read Q
        // O_t of the previous item must have been read out before PV_t(0) of this one
        auto o_ready = [&](int t) -> bool {
          return r == 0 || lpc::mbar_wait(o_free(t), (uint32_t)(r - 1) & 1u, st);
        };
        for (int j = 0; j < it.n1 && ok; ++j) {
          const uint32_t kv = kvc + (uint32_t)j;
          if (j < it.n0) {
            if (j == 0 && !(ok = o_ready(0))) break;
            if (!(ok = issue_pv(0, kv, c0 + (uint32_t)j, j == 0))) break;
          }
          if (j + 1 < it.n0 && !(ok = issue_s(0, kv + 1))) break;
          if (j == 0 && !(ok = o_ready(1))) break;
          if (!(ok = issue_pv(1, kv, c1 + (uint32_t)j, j == 0))) break;
          lpc::umma_commit(v_empty(kv % KV_STAGES));
          if (j + 1 < it.n1) {
            if (!(ok = issue_s(1, kv + 1))) break;
            lpc::umma_commit(k_empty((kv + 1) % KV_STAGES));
            if (j + 2 == it.n1) lpc::umma_commit(q_empty);  // last S MMA of the item issued
          }
        }
        kvc += (uint32_t)it.n1;
        c0 += (uint32_t)it.n0;
        c1 += (uint32_t)it.n1;
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 200;\n" ::: "memory");
    // ---------------- softmax + epilogue: warpgroup t = warp / 4 ----------------
    const int t = warp >> 2;
    const int rr = (warp & 3) * 32 + lane;         // row within the query tile = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + 128u * t + lane_off;
    const uint32_t tO = tmem + 256u + 128u * t + lane_off;
    bool ok = true;
    uint32_t cnt = 0;  // S_t tiles so far (phase of s_full / p_full / o_done)
    // bounded wait with a warp-uniform outcome: a warp never splits on a
    // timeout, so the __syncwarp calls below always see the whole warp
    auto wait_warp = [&](uint32_t bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, lpc::mbar_wait(bar, parity, st));
    };
    for (int r = 0, i = item_of(c, G, 0); i < p.num_items && ok; i = item_of(c, G, ++r)) {
      const Item it = decode_item(p, i);
      const int n = t == 0 ? it.n0 : it.n1;
      const int64_t qrow = it.q0 + (int64_t)t * BQ + rr;  // query index
      const int64_t qpos = p.offset + qrow;               // absolute position
      const int64_t lim = p.causal ? min(qpos, p.kv_len - 1) : p.kv_len - 1;  // last visible key
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n && ok; ++j) {
        const uint32_t ph = cnt + (uint32_t)j;
        if (!wait_warp(s_full(t), ph & 1u)) { ok = false; break; }
        lpc::tc_fence_after();
        const int64_t k0 = (int64_t)j * BKV;
        const bool need_mask = (k0 + BKV > p.kv_len) ||
                               (p.causal && k0 + BKV - 1 > p.offset + it.q0 + (int64_t)t * BQ);
        uint32_t sv[BKV];
        const int lim_rel = (int)max((int64_t)-1, min(lim - k0, (int64_t)(BKV - 1)));
        // keys k0 + i with i > lim_rel are invisible to this row
        auto mask_part = [&](int q0, int q1) {
          if (need_mask) {
#pragma unroll
            for (int q = 0; q < BKV; ++q)
              if (q >= q0 && q < q1 && q > lim_rel) sv[q] = 0xff800000u;  // -inf
          }
        };
        auto load_s = [&]() {
#pragma unroll
          for (int cc = 0; cc < BKV; cc += 32)
            lpc::tmem_ld32(tS + cc, *reinterpret_cast<uint32_t(*)[32]>(&sv[cc]));
          lpc::tmem_wait_ld();
          mask_part(0, BKV);
        };
        auto row_max = [&]() {  // four independent chains of 3-input max
          float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
          for (int q = 0; q < BKV; q += 8) {
            m0 = max3(m0, __uint_as_float(sv[q]), __uint_as_float(sv[q + 1]));
            m1 = max3(m1, __uint_as_float(sv[q + 2]), __uint_as_float(sv[q + 3]));
            m2 = max3(m2, __uint_as_float(sv[q + 4]), __uint_as_float(sv[q + 5]));
            m3 = max3(m3, __uint_as_float(sv[q + 6]), __uint_as_float(sv[q + 7]));
          }
          return fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)) * p.scale_log2;  // scale > 0
        };
        const uint64_t sc2 = pack_f2(p.scale_log2, p.scale_log2);
        uint64_t rsa = 0, rsb = 0;
        uint32_t pk[BKV / 2];
        auto exps_part = [&](float m_ref, int q0, int q1) {
          const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
          const uint64_t nm2 = pack_f2(-m_use, -m_use);
#pragma unroll
          for (int q = 0; q < BKV; q += 2) {
            if (q < q0 || q >= q1) continue;
            const uint64_t x = fma_f2(pack_u2(sv[q], sv[q + 1]), sc2, nm2);
            const uint64_t e = pack_f2(fast_exp2(lo_f(x)), fast_exp2(hi_f(x)));
            if ((q >> 1) & 1) rsb = add_f2(rsb, e);
            else rsa = add_f2(rsa, e);
            pk[q >> 1] = pack2<T>(lo_f(e), hi_f(e));
          }
        };
        // Tile 0 sets the reference max.  Later tiles exponentiate against
        // the running one without reducing their own max: a row whose max
        // grew by more than the threshold has an exponential, hence a row
        // sum, above 2^threshold, and only such warps reduce the max and redo.
        load_s();
        // the last 64 keys' max, in log2 units: a growth past the threshold
        // there must be known before the first 64 keys' P is released
        float mt_hi = -INFINITY;
        if (j == 0) {
          m_used = row_max();
        } else {
          float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
          for (int q = BKV / 2; q < BKV; q += 4) {
            m0 = max3(m0, __uint_as_float(sv[q]), __uint_as_float(sv[q + 1]));
            m1 = max3(m1, __uint_as_float(sv[q + 2]), __uint_as_float(sv[q + 3]));
          }
          mt_hi = fmaxf(m0, m1) * p.scale_log2;
        }
        exps_part(m_used, 0, BKV / 2);
        const uint64_t rs_lo2 = add_f2(rsa, rsb);
        const float rs_lo = lo_f(rs_lo2) + hi_f(rs_lo2);
        // a grown max: a first-half row sum above 2^8, a second-half max more
        // than 8 above the reference, or a first visible key
        const bool big = j > 0 && (!(rs_lo <= RESCALE_LIMIT) || !(mt_hi <= m_used + RESCALE_LOG2) ||
                                   (m_used == -INFINITY && rs_lo > 0.f));
        // PV_t(j-1) must be done: its P shares these TMEM columns and O must be stable
        if (j >= 1 && !wait_warp(o_done(t), (ph - 1u) & 1u)) { ok = false; break; }
        lpc::tc_fence_after();
        if (__any_sync(0xffffffffu, big)) {  // warp-uniform: tcgen05.ld is warp-collective
          // rare: new reference max for the whole row, O rescaled, all of P
          // stored before either half is released
          float alpha = 1.f;
          bool rescale = false;
          load_s();  // S is still in TMEM (no P stored yet)
          if (big) {
            const float mt = row_max();
            if (mt > m_used) {
              alpha = fast_exp2(m_used - mt);
              m_used = mt;
              rescale = true;
            }
          }
          rsa = rsb = 0;
          exps_part(m_used, 0, BKV);  // rows that kept their max recompute the same values
#pragma unroll
          for (int cc = 0; cc < BKV / 2; cc += 16)
            lpc::tmem_st16(tS + (uint32_t)cc, *reinterpret_cast<uint32_t(*)[16]>(&pk[cc]));
          const uint64_t rs2 = add_f2(rsa, rsb);
          l = l * alpha + (lo_f(rs2) + hi_f(rs2));
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
            for (int cc = 0; cc < HD; cc += 16) {
              uint32_t v[16];
              lpc::tmem_ld16(tO + cc, v);
              lpc::tmem_wait_ld();
#pragma unroll
              for (int q = 0; q < 16; ++q) v[q] = __float_as_uint(__uint_as_float(v[q]) * alpha);
              lpc::tmem_st16(tO + cc, v);
            }
          }
          lpc::tmem_wait_st();
          lpc::tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            lpc::mbar_arrive(p_half(t));
            lpc::mbar_arrive(p_full(t));
          }
        } else {
#pragma unroll
          for (int cc = 0; cc < BKV / 4; cc += 16)
            lpc::tmem_st16(tS + (uint32_t)cc, *reinterpret_cast<uint32_t(*)[16]>(&pk[cc]));
          lpc::tmem_wait_st();
          lpc::tc_fence_before();
          __syncwarp();
          if (lane == 0) lpc::mbar_arrive(p_half(t));
          exps_part(m_used, BKV / 2, BKV);
#pragma unroll
          for (int cc = BKV / 4; cc < BKV / 2; cc += 16)
            lpc::tmem_st16(tS + (uint32_t)cc, *reinterpret_cast<uint32_t(*)[16]>(&pk[cc]));
          const uint64_t rs2 = add_f2(rsa, rsb);
          l += lo_f(rs2) + hi_f(rs2);
          lpc::tmem_wait_st();
          lpc::tc_fence_before();
          __syncwarp();
          if (lane == 0) lpc::mbar_arrive(p_full(t));
        }
      }
      // epilogue: O / l, then O_t is free for the next item's PV
      if (ok && (ok = wait_warp(o_done(t), (cnt + (uint32_t)n - 1u) & 1u))) {
        lpc::tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const bool valid = qrow < p.q_len;
        T* orow = out + (((int64_t)it.b * p.heads + it.h) * p.q_len + qrow) * HD;
#pragma unroll 1
        for (int cc = 0; cc < HD; cc += 32) {
          uint32_t v[32];
          lpc::tmem_ld32(tO + cc, v);
          lpc::tmem_wait_ld();
          if (valid) {
            uint32_t pk[16];
#pragma unroll
            for (int q = 0; q < 32; q += 2)
              pk[q >> 1] = pack2<T>(__uint_as_float(v[q]) * inv, __uint_as_float(v[q + 1]) * inv);
            uint4* dst = reinterpret_cast<uint4*>(orow + cc);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)
              dst[q4] = make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
          }
        }
        lpc::tc_fence_before();
        __syncwarp();
        if (lane == 0) lpc::mbar_arrive(o_free(t));
      }
      cnt += (uint32_t)n;
    }
  }
  lpc::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    lpc::tc_fence_after();
    lpc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// The kernel's setmaxnreg split is sized for LAUNCH_REGS registers per
// thread: with fewer, the softmax warpgroups' increase could never be granted,
// so any other count refuses to launch.
template <typename T, int HD>
int launch_prefill(dim3 grid, const TmaDesc4& tq, const TmaDesc4& tk, const TmaDesc4& tv,
                   void* out, const Params& p, uint32_t id_qk, uint32_t id_pv, cudaStream_t s) {
  static int regs = 0;
  if (regs == 0) {
    cudaFuncAttributes fa;
    regs = cudaFuncGetAttributes(&fa, flash_prefill_kernel<T, HD>) == cudaSuccess ? fa.numRegs : -1;
  }
  if (regs != LAUNCH_REGS) {
    lpc::set_error("flash_attention: kernel built with %d registers per thread, its register "
                   "split needs %d", regs, LAUNCH_REGS);
    return LPC_ERR_UNSUPPORTED;
  }
  constexpr int smem = smem_bytes<HD>();
  static std::atomic<uint64_t> mask{0};
  if (int rc = lpc::once_per_device_smem((const void*)flash_prefill_kernel<T, HD>, smem, mask))
    return rc;
  flash_prefill_kernel<T, HD><<<grid, NTHREADS, smem, s>>>(tq, tk, tv, (T*)out, p, id_qk, id_pv);
  return LPC_OK;
}

}  // namespace

extern "C" int lpc_flash_attention(const void* q, const void* k, const void* v, void* out,
                                   int64_t batch, int heads, int kv_heads, int64_t q_len,
                                   int64_t kv_len, int head_dim, int64_t k_batch_stride,
                                   int64_t k_head_stride, int causal, float sm_scale, int dtype,
                                   void* stream) {
  using namespace lpc;
  if (batch <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || q_len <= 0 ||
      kv_len <= 0) {
    set_error("flash_attention: invalid sizes (batch=%lld heads=%d kv_heads=%d q_len=%lld "
              "kv_len=%lld)", (long long)batch, heads, kv_heads, (long long)q_len,
              (long long)kv_len);
    return LPC_ERR_INVALID;
  }
  if (q_len > kv_len) {
    set_error("flash_attention: Q_LEN cannot exceed KV_LEN.");
    return LPC_ERR_INVALID;
  }
  if (head_dim != 128 && head_dim != 64) {
    set_error("flash_attention: head_dim %d not supported by the tcgen05 kernel (64 or 128)",
              head_dim);
    return LPC_ERR_UNSUPPORTED;
  }
  if (dtype != LPC_DTYPE_BF16 && dtype != LPC_DTYPE_F16) {
    set_error("flash_attention: Only FP16 and BF16 are supported.");
    return LPC_ERR_UNSUPPORTED;
  }
  if (!q || !k || !v || !out) {
    set_error("flash_attention: null pointer");
    return LPC_ERR_INVALID;
  }
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      k_head_stride < kv_len * head_dim || k_batch_stride < (int64_t)kv_heads * k_head_stride) {
    set_error("flash_attention: bad alignment or strides");
    return LPC_ERR_INVALID;
  }
  if (batch > 65535 || heads > 65535 || q_len > 0x7fffffffLL || kv_len > 0x7fffffffLL) {
    set_error("flash_attention: sizes exceed the launch grid");
    return LPC_ERR_UNSUPPORTED;
  }
  TmaDesc4 tq, tk, tv;
  const uint64_t rowb = (uint64_t)head_dim * 2;
  {
    uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)q_len, (uint64_t)heads, (uint64_t)batch};
    uint64_t str[3] = {rowb, rowb * q_len, rowb * q_len * heads};
    uint32_t box[4] = {BOX, BQ, 1, 1};
    int rc = make_tma_nd(reinterpret_cast<TmaDesc*>(&tq), q, dtype, 4, dims, str, box, true);
    if (rc) return rc;
  }
  {
    uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)kv_len, (uint64_t)kv_heads, (uint64_t)batch};
    uint64_t str[3] = {rowb, (uint64_t)k_head_stride * 2, (uint64_t)k_batch_stride * 2};
    uint32_t box[4] = {BOX, BKV, 1, 1};
    int rc = make_tma_nd(reinterpret_cast<TmaDesc*>(&tk), k, dtype, 4, dims, str, box, true);
    if (rc) return rc;
    rc = make_tma_nd(reinterpret_cast<TmaDesc*>(&tv), v, dtype, 4, dims, str, box, true);
    if (rc) return rc;
  }
  Params p;
  p.q_len = q_len;
  p.kv_len = kv_len;
  p.offset = kv_len - q_len;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.group = heads / kv_heads;
  p.num_q_blocks = (int)((q_len + NQT * BQ - 1) / (NQT * BQ));
  p.batch = (int)batch;
  const int64_t items = (int64_t)p.num_q_blocks * heads * batch;
  if (items > 0x7fffffffLL) {
    set_error("flash_attention: too many query blocks");
    return LPC_ERR_UNSUPPORTED;
  }
  p.num_items = (int)items;
  p.scale_log2 = sm_scale * LOG2E;
  p.causal = causal ? 1 : 0;
  // item order: LPC_PREFILL_BAND=<pairs> narrows the bands (measurement);
  // by default one band covers every (head, batch) pair
  {
    const int hb = heads * (int)batch;
    const char* e = getenv("LPC_PREFILL_BAND");
    const int want = e ? atoi(e) : 0;
    p.band = want > 0 && want < hb ? want : hb;
  }
  const uint32_t fmt = dtype == LPC_DTYPE_BF16 ? 1u : 0u;
  const uint32_t id_qk = idesc_f16(fmt, BQ, BKV, 0u, 0u);
  const uint32_t id_pv = idesc_f16(fmt, BQ, (uint32_t)head_dim, 0u, 1u);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // persistent: one CTA per SM loops over the work items
  dim3 grid((unsigned)std::min<int64_t>(items, current_device_sms()));
  int rc;
  if (dtype == LPC_DTYPE_BF16) {
    rc = head_dim == 128 ? launch_prefill<__nv_bfloat16, 128>(grid, tq, tk, tv, out, p, id_qk, id_pv, s)
                         : launch_prefill<__nv_bfloat16, 64>(grid, tq, tk, tv, out, p, id_qk, id_pv, s);
  } else {
    rc = head_dim == 128 ? launch_prefill<__half, 128>(grid, tq, tk, tv, out, p, id_qk, id_pv, s)
                         : launch_prefill<__half, 64>(grid, tq, tk, tv, out, p, id_qk, id_pv, s);
  }
  if (rc) return rc;
  return check_launch("flash_attention");
}
