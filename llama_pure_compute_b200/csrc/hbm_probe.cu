// HBM read-rate probe: the ceiling of a read-only kernel on this GPU.
//
// The measured HBM peak the bench divides by is a copy (every byte read is
// also written).  Decode attention and the weight streams only read, and a
// B200 reads faster than it copies.  This kernel reads a buffer the way the
// decode split kernel reads its K/V rows and does nothing else: one CTA per
// 128 KB item, a producer thread moving 16 KB stages with 1-D bulk copies
// (cp.async.bulk) into a 4-stage shared-memory ring completed on mbarriers,
// four warps releasing each stage as it lands.  Its rate is the roofline of
// a kernel that streams through shared memory at the same depth.
#include "lpc_common.cuh"

LPC_DECLARE_STATUS(g_probe_status)

unsigned int lpc_status_probe(bool clear) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_probe_status, sizeof(v));
  if (clear && v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_probe_status, &z, sizeof(z));
  }
  return v;
}

namespace {

constexpr int PROBE_ITEM = 128 * 1024;  // bytes per CTA
constexpr int PROBE_STAGE = 16 * 1024;  // bytes per bulk copy
constexpr int PROBE_STAGES = 4;
constexpr int PROBE_WARPS = 4;          // consumer warps; one more produces

__global__ void __launch_bounds__((PROBE_WARPS + 1) * 32) hbm_read_kernel(const uint8_t* __restrict__ buf) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + PROBE_STAGES * PROBE_STAGE);
  auto full = [&](int s) { return lpc::smem_u32(bar + s); };
  auto empty = [&](int s) { return lpc::smem_u32(bar + PROBE_STAGES + s); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < PROBE_STAGES; ++s) {
      lpc::mbar_init(full(s), 1);
      lpc::mbar_init(empty(s), PROBE_WARPS);
    }
    lpc::fence_mbar_init();
  }
  __syncthreads();
  constexpr int n = PROBE_ITEM / PROBE_STAGE;
  const uint8_t* src = buf + (int64_t)blockIdx.x * PROBE_ITEM;
  if (warp == PROBE_WARPS) {
    if (lane == 0) {
      for (int i = 0; i < n; ++i) {
        const int s = i % PROBE_STAGES;
        if (!lpc::mbar_wait(empty(s), ((uint32_t)(i / PROBE_STAGES) & 1u) ^ 1u, &g_probe_status)) break;
        lpc::mbar_arrive_expect_tx(full(s), PROBE_STAGE);
        lpc::bulk_g2s(lpc::smem_u32(smem + s * PROBE_STAGE), src + (int64_t)i * PROBE_STAGE,
                      PROBE_STAGE, full(s));
      }
    }
  } else {
    for (int i = 0; i < n; ++i) {
      const int s = i % PROBE_STAGES;
      if (!lpc::mbar_wait(full(s), (uint32_t)(i / PROBE_STAGES) & 1u, &g_probe_status)) break;
      __syncwarp();
      if (lane == 0) lpc::mbar_arrive(empty(s));
    }
  }
}

}  // namespace

extern "C" int lpc_hbm_read_probe(const void* buf, int64_t bytes, void* stream) {
  using namespace lpc;
  if (!buf || bytes <= 0 || bytes % PROBE_ITEM || bytes / PROBE_ITEM > 0x7fffffff) {
    set_error("hbm_read_probe: bytes must be a positive multiple of %d (got %lld)", PROBE_ITEM,
              (long long)bytes);
    return LPC_ERR_INVALID;
  }
  if (!aligned16(buf)) {
    set_error("hbm_read_probe: buffer must be 16-byte aligned");
    return LPC_ERR_INVALID;
  }
  constexpr int smem = PROBE_STAGES * PROBE_STAGE + 2 * PROBE_STAGES * 8;
  static std::atomic<uint64_t> mask{0};
  int rc = once_per_device_smem((const void*)hbm_read_kernel, smem, mask);
  if (rc) return rc;
  hbm_read_kernel<<<(unsigned)(bytes / PROBE_ITEM), (PROBE_WARPS + 1) * 32, smem,
                    static_cast<cudaStream_t>(stream)>>>(static_cast<const uint8_t*>(buf));
  return check_launch("hbm_read_probe");
}
