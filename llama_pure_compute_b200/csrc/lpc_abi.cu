// Host-side plumbing of the C ABI: error strings, dtype sizes, TMA descriptor
// encoding through the driver entry point, and the device status read-back.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "lpc_common.cuh"

namespace lpc {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
    return LPC_ERR_CUDA;
  }
  return LPC_OK;
}

int dtype_size(int dtype) {
  switch (dtype) {
    case LPC_DTYPE_F32: return 4;
    case LPC_DTYPE_F16: return 2;
    case LPC_DTYPE_BF16: return 2;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int once_per_device_smem(const void* kernel, int bytes, std::atomic<uint64_t>& mask) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("cannot query the current CUDA device");
    return LPC_ERR_CUDA;
  }
  const uint64_t bit = 1ull << dev;
  if (mask.load(std::memory_order_acquire) & bit) return LPC_OK;
  cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_error("cannot reserve %d bytes of shared memory: %s", bytes, cudaGetErrorString(e));
    return LPC_ERR_CUDA;
  }
  mask.fetch_or(bit, std::memory_order_acq_rel);
  return LPC_OK;
}

int current_device_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
    v = 148;
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

static PFN_cuCtxGetCurrent_v4000 g_ctx_get = nullptr;
static std::once_flag g_ctx_once;

void* current_context() {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
  });
  CUcontext c = nullptr;
  if (!g_ctx_get || g_ctx_get(&c) != CUDA_SUCCESS) return nullptr;
  return reinterpret_cast<void*>(c);
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int make_tma_nd(TmaDesc* out, const void* base, int dtype, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return LPC_ERR_CUDA;
  }
  if (rank < 1 || rank > 5) {
    set_error("make_tma_nd: bad rank %d", rank);
    return LPC_ERR_INVALID;
  }
  CUtensorMapDataType t;
  switch (dtype) {
    case LPC_DTYPE_BF16: t = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case LPC_DTYPE_F16: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case LPC_DTYPE_F32: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    default: set_error("make_tma_nd: bad dtype %d", dtype); return LPC_ERR_UNSUPPORTED;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) st[i] = strides_bytes[i];
  CUresult r = g_encode(reinterpret_cast<CUtensorMap*>(out->bytes), t, (cuuint32_t)rank,
                        const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): rank %d dims %llu x %llu box %u x %u", (int)r,
              rank, (unsigned long long)dims[0], (unsigned long long)(rank > 1 ? dims[1] : 1),
              box[0], rank > 1 ? box[1] : 1u);
    return LPC_ERR_INVALID;
  }
  return LPC_OK;
}

int make_tma_2d(TmaDesc* out, const void* base, int dtype, uint64_t inner, uint64_t outer,
                uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                bool swizzle128) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t str[1] = {row_stride_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return make_tma_nd(out, base, dtype, 2, dims, str, box, swizzle128);
}

}  // namespace lpc

// Per-module status readers (each module keeps its own device status word).
unsigned int lpc_status_kv(bool clear);
unsigned int lpc_status_rope(bool clear);
unsigned int lpc_status_decode(bool clear);
unsigned int lpc_status_swiglu(bool clear);
unsigned int lpc_status_prefill(bool clear);
unsigned int lpc_status_wsgemm(bool clear);
unsigned int lpc_status_probe(bool clear);

extern "C" int lpc_version(void) { return 100; }

extern "C" const char* lpc_last_error(void) { return lpc::g_last_error; }

extern "C" int lpc_device_status(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) {
    lpc::set_error("lpc_device_status: device synchronisation failed");
    return -1;
  }
  unsigned int s = lpc_status_kv(true) | lpc_status_rope(true) | lpc_status_decode(true) |
                   lpc_status_swiglu(true) | lpc_status_prefill(true) | lpc_status_wsgemm(true) |
                   lpc_status_probe(true);
  return static_cast<int>(s);
}
