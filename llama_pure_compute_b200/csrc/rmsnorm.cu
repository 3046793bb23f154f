// Row RMSNorm: y = (x * rsqrt(mean(x^2) + eps)) * w, fp32 math, result rounded
// once to x's dtype.  Follows `_rmsnorm_pytorch_fallback`
// (src/llama_pure_compute/triton_kernels/rmsnorm.py:88-96) and the Triton row
// kernel (rmsnorm.py:20-55).
//
// One CTA per row; each thread moves 16-byte vectors.  The row is read once
// into registers (up to ROW_VECS vectors per thread), so HBM traffic is one
// read of x and one write of y.
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
  if (vec && nvec <= threads * 4) {
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
