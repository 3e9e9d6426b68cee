// Shared helpers for the sm_100a kernels of llm_research_b200._C.
#pragma once

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#define LRB_CHECK(cond, ...) TORCH_CHECK(cond, __VA_ARGS__)
#define LRB_CUDA_CHECK(expr)                                                              \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error: ", cudaGetErrorString(_e), " at ", #expr); \
  } while (0)
#define LRB_LAUNCH_CHECK() LRB_CUDA_CHECK(cudaGetLastError())

namespace lrb {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Makes `dev` current in this host thread with its primary context bound.  The
// autograd engine's worker threads start with no current CUDA context, and
// c10's device guard does not call cudaSetDevice when the device index already
// matches; entry points that build tensor maps and launch cluster kernels from
// a backward pass call this first.
inline void bind_device(int dev) { LRB_CUDA_CHECK(cudaSetDevice(dev)); }

// Device address of a file-scope `__device__ int` error word (one copy per
// device, part of the module image) on device `dev`.  Looked up once per device
// with that device current and cached in atomics: safe from any host thread
// (the autograd engine runs backward kernels on its own thread), and nothing
// to destroy at process exit.
struct DeviceWord {
  const void* symbol;
  std::atomic<int*> addr[64];
  int* get(int dev) {
    if (dev < 0) LRB_CUDA_CHECK(cudaGetDevice(&dev));
    TORCH_CHECK(dev < 64, "device index ", dev, " out of range");
    int* p = addr[dev].load(std::memory_order_acquire);
    if (p != nullptr) return p;
    int prev = 0;
    LRB_CUDA_CHECK(cudaGetDevice(&prev));
    LRB_CUDA_CHECK(cudaSetDevice(dev));
    void* q = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&q, symbol);
    LRB_CUDA_CHECK(cudaSetDevice(prev));
    LRB_CUDA_CHECK(e);
    addr[dev].store(static_cast<int*>(q), std::memory_order_release);
    return static_cast<int*>(q);
  }
  // Returns and clears the first word on `dev` (0 = nothing recorded).
  int64_t take(int dev) {
    int* w = get(dev);
    int h = 0;
    LRB_CUDA_CHECK(cudaMemcpy(&h, w, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) LRB_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
    return h;
  }
};

inline int num_sms() {
  static int n = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

// ---- scalar conversions --------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// 2^x with the SFU instruction (ex2.approx, flush-to-zero; 2^-inf = +0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 1/x with the SFU instruction (rcp.approx, flush-to-zero; 1/inf = +0).
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction computes two FMAs, adds
// or products).  Element 0 is the low 32 bits.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x on the FMA pipe, for spreading a softmax's exponentials over both the
// SFU and the FMA units: x = i + f with i = floor(x) and f in [0, 1); 2^f is
// the degree-3 minimax polynomial of 2^f on [0, 1] with p(0) = 1, its three
// coefficients found by the Remez exchange algorithm (maximum relative error
// 8.6e-5 -- far below the bf16 rounding of a probability); 2^i is added into
// the exponent field.  Inputs are clamped at -127, where the result is +0
// exactly (so a masked -inf score gives a zero probability); valid up to 2^127.
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -127.f);
  const int i = __float2int_rd(x);
  const float f = x - __int2float_rn(i);
  float p = fmaf(f, 0.07706704f, 0.22764500f);
  p = fmaf(f, p, 0.69511676f);
  p = fmaf(f, p, 1.0f);
  return __int_as_float(__float_as_int(p) + (i << 23));
}

// ---- reductions ----------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `red` must hold >= 32 floats. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  t = warp_max(t);
  return t;
}

// ---- vectorised 16-byte access --------------------------------------------
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union { uint4 raw; T v[N]; };
};

template <typename T>
__device__ __forceinline__ Vec16<T> ld16(const T* p) {
  Vec16<T> r;
  r.raw = *reinterpret_cast<const uint4*>(p);
  return r;
}
template <typename T>
__device__ __forceinline__ void st16(T* p, const Vec16<T>& r) {
  *reinterpret_cast<uint4*>(p) = r.raw;
}

}  // namespace lrb

// Dispatch over the floating dtypes we support (bf16, fp16, fp32).
#define LRB_DISPATCH_FLOAT(dtype, T, ...)                                     \
  [&] {                                                                        \
    if ((dtype) == at::kBFloat16) { using T = __nv_bfloat16; return __VA_ARGS__(); } \
    if ((dtype) == at::kHalf) { using T = __half; return __VA_ARGS__(); }             \
    if ((dtype) == at::kFloat) { using T = float; return __VA_ARGS__(); }             \
    TORCH_CHECK(false, "unsupported dtype ", dtype);                              \
  }()
