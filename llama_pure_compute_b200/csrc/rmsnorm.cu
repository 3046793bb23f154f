// Row RMSNorm: y = (x * rsqrt(mean(x^2) + eps)) * w, fp32 math, result rounded
// once to x's dtype.  Follows `_rmsnorm_pytorch_fallback`
// (src/llama_pure_compute/triton_kernels/rmsnorm.py:88-96) and the Triton row
// kernel (rmsnorm.py:20-55).
//
// Prefill-sized calls (at least 8 rows per SM) give each row one warp, or
// two / four warps for rows of more than 256 / 512 16-byte vectors (dim 4096
// / 8192 in bf16): every lane issues all its row loads before the first use,
// and the sum of squares is a warp shuffle tree (plus one shared-memory add
// across a row's warps).  Decode-sized calls give each row a CTA of 8 warps,
// which finishes a row soonest.  Either way the row is read once into
// registers, so HBM traffic is one read of x and one write of y.
#include <algorithm>

#include "lpc_common.cuh"

namespace {

using lpc::Num;

template <typename T>
__device__ __forceinline__ void unpack(const uint4& u, float* f) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int j = 0; j < (int)(16 / sizeof(T)); ++j) f[j] = Num<T>::to_f(e[j]);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = lane < nw ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

template <typename T, typename W, int ROW_VECS>
__global__ void __launch_bounds__(256) rmsnorm_vec_kernel(const T* __restrict__ x,
                                                          const W* __restrict__ w,
                                                          T* __restrict__ y, int dim, float eps) {
  constexpr int PER = 16 / (int)sizeof(T);
  __shared__ float red[32];
  // a dependent kernel launched with programmatic stream serialisation (the
  // packed decode GEMM) may start its prologue and weight loads now; it waits
  // for this grid to complete before it reads y
  lpc::pdl_trigger();
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * dim);
  const int nvec = dim / PER;
  float v[ROW_VECS][PER];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < ROW_VECS; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      unpack<T>(__ldg(xr + vi), v[i]);
#pragma unroll
      for (int j = 0; j < PER; ++j) ss = fmaf(v[i][j], v[i][j], ss);
    }
  }
  const float total = block_sum(ss, red);
  const float r = rsqrtf(total / (float)dim + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + row * dim);
#pragma unroll
  for (int i = 0; i < ROW_VECS; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      uint4 u;
      T* e = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int j = 0; j < PER; ++j)
        e[j] = Num<T>::from_f(__fmul_rn(__fmul_rn(v[i][j], r), Num<W>::to_f(w[vi * PER + j])));
      yr[vi] = u;
    }
  }
}

// Loads PER consecutive weights (16 bytes of x's type) as fp32: by 16-byte
// vectors when they span 16 bytes or more, else by one 8-byte vector (fp32
// rows with 16-bit weights).  The host takes this path only for a 16-byte
// aligned w, so either load is aligned.
template <typename W, int PER>
__device__ __forceinline__ void load_w(const W* __restrict__ w, float* f) {
  if constexpr (PER * sizeof(W) >= 16) {
    constexpr int WV = PER * (int)sizeof(W) / 16;  // 16-byte vectors of weights
    constexpr int WPV = 16 / (int)sizeof(W);        // weights per vector
#pragma unroll
    for (int v = 0; v < WV; ++v) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(w) + v);
      const W* e = reinterpret_cast<const W*>(&u);
#pragma unroll
      for (int j = 0; j < WPV; ++j) f[v * WPV + j] = Num<W>::to_f(e[j]);
    }
  } else {
    static_assert(PER * sizeof(W) == 8, "fp32 rows with 16-bit weights");
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(w));
    const W* e = reinterpret_cast<const W*>(&u);
#pragma unroll
    for (int j = 0; j < PER; ++j) f[j] = Num<W>::to_f(e[j]);
  }
}

// WPR warps per row, VPL 16-byte vectors per lane (nvec <= 32 * WPR * VPL);
// 256 / (32 * WPR) rows per full CTA.  With WPR > 1 the warps of a row add
// their partial sums through shared memory.
template <typename T, typename W, int VPL, int WPR>
__global__ void __launch_bounds__(256, 3) rmsnorm_warp_kernel(const T* __restrict__ x,
                                                              const W* __restrict__ w,
                                                              T* __restrict__ y, int64_t rows,
                                                              int dim, float eps) {
  constexpr int PER = 16 / (int)sizeof(T);
  __shared__ float part[8];
  lpc::pdl_trigger();  // as in rmsnorm_vec_kernel
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) / WPR + warp / WPR;
  const bool live = row < rows;
  const int nvec = dim / PER;
  const int v0 = (warp % WPR) * 32 * VPL;  // this warp's first vector of the row
  const uint4* xr = reinterpret_cast<const uint4*>(x + (live ? row : 0) * dim);
  uint4 raw[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = v0 + lane + 32 * i;
    raw[i] = live && vi < nvec ? __ldg(xr + vi) : make_uint4(0u, 0u, 0u, 0u);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    float f[PER];
    unpack<T>(raw[i], f);
#pragma unroll
    for (int j = 0; j < PER; ++j) ss = fmaf(f[j], f[j], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if constexpr (WPR > 1) {
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    const int first = warp - warp % WPR;
    ss = 0.f;
#pragma unroll
    for (int k = 0; k < WPR; ++k) ss += part[first + k];
  }
  if (!live) return;
  const float r = rsqrtf(ss / (float)dim + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + row * dim);
  // the weights (L1-resident after the first rows) are loaded four vectors at
  // a time: hoisting all of them next to the row would cost a CTA per SM
#pragma unroll
  for (int i0 = 0; i0 < VPL; i0 += 4) {
    asm volatile("" ::: "memory");
#pragma unroll
    for (int i = i0; i < i0 + 4 && i < VPL; ++i) {
      const int vi = v0 + lane + 32 * i;
      if (vi < nvec) {
        float f[PER], g[PER];
        unpack<T>(raw[i], f);
        load_w<W, PER>(w + (int64_t)vi * PER, g);
        uint4 u;
        T* e = reinterpret_cast<T*>(&u);
#pragma unroll
        for (int j = 0; j < PER; ++j) e[j] = Num<T>::from_f(__fmul_rn(__fmul_rn(f[j], r), g[j]));
        yr[vi] = u;
      }
    }
  }
}

template <typename T, typename W, int VPL, int WPR>
void launch_warp_rows(const void* x, const void* w, void* y, int64_t rows, int dim, float eps,
                      cudaStream_t s) {
  // rows per CTA: 8 / WPR once there are 16 rows per SM, fewer below, so that
  // a decode-sized call (a few hundred rows) still spreads over every SM
  const int64_t sms = lpc::current_device_sms();
  const int full = 8 / WPR;
  const int rpc = rows >= 16 * sms ? full : std::max(1, std::min<int>(full, (int)(rows / (4 * sms))));
  const unsigned blocks = (unsigned)((rows + rpc - 1) / rpc);
  rmsnorm_warp_kernel<T, W, VPL, WPR><<<blocks, 32 * WPR * rpc, 0, s>>>(
      (const T*)x, (const W*)w, (T*)y, rows, dim, eps);
}

// Generic path: any dim, two passes over the row (second pass hits L1/L2).
template <typename T, typename W>
__global__ void __launch_bounds__(256) rmsnorm_scalar_kernel(const T* __restrict__ x,
                                                             const W* __restrict__ w,
                                                             T* __restrict__ y, int dim,
                                                             float eps) {
  __shared__ float red[32];
  lpc::pdl_trigger();  // as in rmsnorm_vec_kernel
  const int64_t row = blockIdx.x;
  const T* xr = x + row * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float f = Num<T>::to_f(xr[i]);
    ss = fmaf(f, f, ss);
  }
  const float total = block_sum(ss, red);
  const float r = rsqrtf(total / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    y[row * dim + i] =
        Num<T>::from_f(__fmul_rn(__fmul_rn(Num<T>::to_f(xr[i]), r), Num<W>::to_f(w[i])));
}

template <typename T, typename W>
int launch(const void* x, const void* w, void* y, int64_t rows, int dim, float eps,
           cudaStream_t s) {
  constexpr int PER = 16 / (int)sizeof(T);
  const int threads = 256;
  const bool vec = dim % PER == 0 && lpc::aligned16(x) && lpc::aligned16(y);
  const int nvec = dim / PER;
  // row counts of a prefill (several rows per SM): warp rows; decode-sized
  // calls (a few rows per SM) keep the CTA-per-row kernel, whose 8 warps per
  // row finish a row soonest (4.5 us at 256 x 4096 against 6.3)
  const int64_t sms = lpc::current_device_sms();
  if (vec && lpc::aligned16(w) && rows >= 8 * sms && nvec <= 32 * 8 * 4) {
    if (nvec <= 32 * 4)
      launch_warp_rows<T, W, 4, 1>(x, w, y, rows, dim, eps, s);
    else if (nvec <= 32 * 8)
      launch_warp_rows<T, W, 8, 1>(x, w, y, rows, dim, eps, s);
    else if (nvec <= 32 * 8 * 2)
      launch_warp_rows<T, W, 8, 2>(x, w, y, rows, dim, eps, s);
    else
      launch_warp_rows<T, W, 8, 4>(x, w, y, rows, dim, eps, s);
  } else if (vec && nvec <= threads * 4) {
    if (nvec <= threads)
      rmsnorm_vec_kernel<T, W, 1><<<(unsigned)rows, threads, 0, s>>>((const T*)x, (const W*)w, (T*)y, dim, eps);
    else if (nvec <= threads * 2)
      rmsnorm_vec_kernel<T, W, 2><<<(unsigned)rows, threads, 0, s>>>((const T*)x, (const W*)w, (T*)y, dim, eps);
    else
      rmsnorm_vec_kernel<T, W, 4><<<(unsigned)rows, threads, 0, s>>>((const T*)x, (const W*)w, (T*)y, dim, eps);
  } else {
    rmsnorm_scalar_kernel<T, W><<<(unsigned)rows, threads, 0, s>>>((const T*)x, (const W*)w, (T*)y, dim, eps);
  }
  return lpc::check_launch("rmsnorm_forward");
}

template <typename T>
int launch_w(int w_dtype, const void* x, const void* w, void* y, int64_t rows, int dim, float eps,
             cudaStream_t s) {
  switch (w_dtype) {
    case LPC_DTYPE_F32: return launch<T, float>(x, w, y, rows, dim, eps, s);
    case LPC_DTYPE_BF16: return launch<T, __nv_bfloat16>(x, w, y, rows, dim, eps, s);
    case LPC_DTYPE_F16: return launch<T, __half>(x, w, y, rows, dim, eps, s);
  }
  lpc::set_error("rmsnorm_forward: unsupported weight dtype %d", w_dtype);
  return LPC_ERR_UNSUPPORTED;
}

}  // namespace

// Exposed to the fused SwiGLU op as well (normalised activations for the GEMM).
int lpc_rmsnorm_launch(const void* x, const void* w, void* y, int64_t rows, int dim, float eps,
                       int dtype, int w_dtype, cudaStream_t s) {
  switch (dtype) {
    case LPC_DTYPE_F32: return launch_w<float>(w_dtype, x, w, y, rows, dim, eps, s);
    case LPC_DTYPE_BF16: return launch_w<__nv_bfloat16>(w_dtype, x, w, y, rows, dim, eps, s);
    case LPC_DTYPE_F16: return launch_w<__half>(w_dtype, x, w, y, rows, dim, eps, s);
  }
  lpc::set_error("rmsnorm_forward: unsupported dtype %d", dtype);
  return LPC_ERR_UNSUPPORTED;
}

extern "C" int lpc_rmsnorm_forward(const void* x, const void* w, void* y, int64_t rows, int dim,
                                   float eps, int dtype, int w_dtype, void* stream) {
  using namespace lpc;
  if (rows < 0 || dim <= 0) {
    set_error("rmsnorm_forward: invalid sizes (rows=%lld dim=%d)", (long long)rows, dim);
    return LPC_ERR_INVALID;
  }
  if (!(eps > 0.f)) {
    set_error("rmsnorm_forward: eps must be strictly positive");
    return LPC_ERR_INVALID;
  }
  if (rows == 0) return LPC_OK;
  if (rows > 0x7fffffffLL) {
    set_error("rmsnorm_forward: too many rows");
    return LPC_ERR_UNSUPPORTED;
  }
  if (!x || !w || !y) {
    set_error("rmsnorm_forward: null pointer");
    return LPC_ERR_INVALID;
  }
  return lpc_rmsnorm_launch(x, w, y, rows, dim, eps, dtype, w_dtype,
                            static_cast<cudaStream_t>(stream));
}
