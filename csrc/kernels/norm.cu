// RMSNorm forward/backward, optionally fused with the preceding residual add.
//
// One warp per row.  Rows whose width is a multiple of 256 keep the row in
// registers (8 elements per lane per 256 columns, up to 8192 columns) and
// touch HBM exactly once per direction; other widths take a two-pass scalar
// loop.  The weight gradient is reduced per block in shared memory and then
// across blocks by a second tiny kernel, never with per-element atomics.
#include "../common.cuh"
#include "../lrb_noalloc.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

namespace lrb {
namespace {

constexpr int kWarps = 8;  // rows per block in flight

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* f) {
  if constexpr (sizeof(T) == 2) {
    Vec16<T> v = ld16(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = to_f(v.v[i]);
  } else {
    Vec16<T> a = ld16(p), b = ld16(p + 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) { f[i] = to_f(a.v[i]); f[4 + i] = to_f(b.v[i]); }
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float* f) {
  if constexpr (sizeof(T) == 2) {
    Vec16<T> v;
#pragma unroll
    for (int i = 0; i < 8; ++i) v.v[i] = from_f<T>(f[i]);
    st16(p, v);
  } else {
    Vec16<T> a, b;
#pragma unroll
    for (int i = 0; i < 4; ++i) { a.v[i] = from_f<T>(f[i]); b.v[i] = from_f<T>(f[4 + i]); }
    st16(p, a);
    st16(p + 4, b);
  }
}
template <typename T>
__device__ __forceinline__ float round_to(float v) { return to_f(from_f<T>(v)); }

// 8 bf16 from global memory through a volatile load, which the compiler may not
// merge with an earlier load of the same address (a second pass re-reads from
// L1 instead of holding the whole row in registers).
__device__ __forceinline__ void reload8_bf16(const __nv_bfloat16* p, float* f) {
  Vec16<__nv_bfloat16> v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.raw.x), "=r"(v.raw.y), "=r"(v.raw.z), "=r"(v.raw.w)
               : "l"(p));
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = __bfloat162float(v.v[i]);
}

// ---------------------------------------------------------------- forward
template <typename T, typename W, typename O, int NV>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_fwd_reg(
    const T* __restrict__ x, const T* __restrict__ res, T* __restrict__ s_out, const W* __restrict__ w,
    O* __restrict__ y, float* __restrict__ rstd_out, int64_t rows, int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * d;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    load8(xr + c, v[i]);
    if (res != nullptr) {
      float r[8];
      load8(res + row * d + c, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = round_to<T>(v[i][j] + r[j]);
      store8(s_out + row * d + c, v[i]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / d + eps);
  if (lane == 0) rstd_out[row] = r;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    float wf[8], o[8];
    load8(w + c, wf);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = round_to<T>(v[i][j] * r) * wf[j];
    store8(y + row * d + c, o);
  }
}

template <typename T, typename W, typename O>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_fwd_generic(
    const T* __restrict__ x, const T* __restrict__ res, T* __restrict__ s_out, const W* __restrict__ w,
    O* __restrict__ y, float* __restrict__ rstd_out, int64_t rows, int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  float ss = 0.f;
  for (int c = lane; c < d; c += 32) {
    float v = to_f(x[row * d + c]);
    if (res != nullptr) {
      v = round_to<T>(v + to_f(res[row * d + c]));
      s_out[row * d + c] = from_f<T>(v);
    }
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / d + eps);
  if (lane == 0) rstd_out[row] = r;
  const T* src = res != nullptr ? s_out : x;
  __syncwarp();
  for (int c = lane; c < d; c += 32) {
    const float v = to_f(src[row * d + c]);
    y[row * d + c] = from_f<O>(round_to<T>(v * r) * to_f(w[c]));
  }
}

// --------------------------------------------------------------- backward
// dx = r * (dn - xhat * mean(dn * xhat)),  dn = dy * w,  xhat = x * r
// dw_partial[block, c] = sum over this block's rows of dy * cast_T(xhat)
template <typename T, typename W, typename O>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_bwd_kernel(
    const O* __restrict__ dy, const T* __restrict__ x, const W* __restrict__ w, const float* __restrict__ rstd,
    const T* __restrict__ ds, T* __restrict__ dx, float* __restrict__ dw_part, int64_t rows, int d) {
  extern __shared__ float sh[];  // kWarps * d floats
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float* acc = sh + (size_t)wid * d;
  for (int c = lane; c < d; c += 32) acc[c] = 0.f;
  // The vectorised loop below updates acc[8 * lane + j], elements another lane zeroed.
  __syncwarp();
  const bool vec = (d % 256) == 0;
  for (int64_t row = (int64_t)blockIdx.x * kWarps + wid; row < rows; row += (int64_t)gridDim.x * kWarps) {
    const float r = rstd[row];
    const T* xr = x + row * d;
    const O* dyr = dy + row * d;
    float dot = 0.f;
    if (vec) {
      for (int c = lane * 8; c < d; c += 256) {
        float xf[8], gf[8], wf[8];
        load8(xr + c, xf);
        load8(dyr + c, gf);
        load8(w + c, wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = xf[j] * r;
          dot += gf[j] * wf[j] * xh;
          acc[c + j] += gf[j] * round_to<T>(xh);
        }
      }
    } else {
      for (int c = lane; c < d; c += 32) {
        const float xh = to_f(xr[c]) * r;
        const float g = to_f(dyr[c]);
        dot += g * to_f(w[c]) * xh;
        acc[c] += g * round_to<T>(xh);
      }
    }
    dot = warp_sum(dot) / d;
    if (vec) {
      for (int c = lane * 8; c < d; c += 256) {
        float xf[8], gf[8], wf[8], o[8];
        load8(xr + c, xf);
        load8(dyr + c, gf);
        load8(w + c, wf);
        float dsf[8];
        if (ds != nullptr) load8(ds + row * d + c, dsf);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = xf[j] * r;
          o[j] = r * (gf[j] * wf[j] - xh * dot) + (ds != nullptr ? dsf[j] : 0.f);
        }
        store8(dx + row * d + c, o);
      }
    } else {
      for (int c = lane; c < d; c += 32) {
        const float xh = to_f(xr[c]) * r;
        float o = r * (to_f(dyr[c]) * to_f(w[c]) - xh * dot);
        if (ds != nullptr) o += to_f(ds[row * d + c]);
        dx[row * d + c] = from_f<T>(o);
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) s += sh[(size_t)k * d + c];
    dw_part[(size_t)blockIdx.x * d + c] = s;
  }
}

// bf16 rows of width d = NV * 256 (NV <= 8), one warp per row.  The second
// pass re-reads the row's x and dy, which the first pass has just brought into
// L1, so HBM sees each once; each warp adds its rows' weight-gradient terms to
// its own fp32 slice of shared memory with 16-byte read-modify-writes (lane
// stride 32 bytes: two-way at most), and the block's warps are summed once at
// the end.
template <int NV>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_bwd_reg(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ ds, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ dw_part, int64_t rows, int d) {
  using T = __nv_bfloat16;
  extern __shared__ float sh[];  // kWarps * d floats
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float* acc = sh + (size_t)wid * d;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float4* a4 = reinterpret_cast<float4*>(acc + (i * 32 + lane) * 8);
    a4[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    a4[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int64_t row = (int64_t)blockIdx.x * kWarps + wid; row < rows; row += (int64_t)gridDim.x * kWarps) {
    const float r = rstd[row];
    const T* xr = x + row * d;
    const T* gr = dy + row * d;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      float xf[8], gf[8], wf[8];
      load8(xr + c, xf);
      load8(gr + c, gf);
      load8(w + c, wf);
      float4* a4 = reinterpret_cast<float4*>(acc + c);
      float4 lo = a4[0], hi = a4[1];
      float t[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = xf[j] * r;
        dot += gf[j] * wf[j] * xh;
        t[j] = gf[j] * round_to<T>(xh);
      }
      lo.x += t[0]; lo.y += t[1]; lo.z += t[2]; lo.w += t[3];
      hi.x += t[4]; hi.y += t[5]; hi.z += t[6]; hi.w += t[7];
      a4[0] = lo;
      a4[1] = hi;
    }
    dot = warp_sum(dot) / d;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      float xf[8], gf[8], wf[8], o[8], dsf[8];
      reload8_bf16(xr + c, xf);
      reload8_bf16(gr + c, gf);
      reload8_bf16(w + c, wf);
      if (ds != nullptr) load8(ds + row * d + c, dsf);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = xf[j] * r;
        o[j] = r * (gf[j] * wf[j] - xh * dot) + (ds != nullptr ? dsf[j] : 0.f);
      }
      store8(dx + row * d + c, o);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) t += sh[(size_t)k * d + c];
    dw_part[(size_t)blockIdx.x * d + c] = t;
  }
}

__global__ void reduce_rows_kernel(const float* __restrict__ part, float* __restrict__ out, int nrows, int d) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float s = 0.f;
  for (int r = 0; r < nrows; ++r) s += part[(size_t)r * d + c];
  out[c] = s;
}

// Dynamic shared memory of rmsnorm_bwd_kernel: kWarps rows x d fp32 accumulators,
// at most 200 KiB (d <= 6400).
constexpr int kBwdSmemMax = 200 * 1024;

// Raises the kernel's dynamic shared-memory limit to kBwdSmemMax once per
// device and never lowers it, so callers with different row widths on several
// host threads cannot undo each other's setting between set and launch (a
// larger limit does not change occupancy: that follows the launch's own size).
template <typename T, typename W, typename O>
cudaError_t raise_bwd_smem_limit(int dev) {
  static std::atomic<bool> done[64];
  static std::mutex mu;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev].load(std::memory_order_relaxed)) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(rmsnorm_bwd_kernel<T, W, O>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmemMax);
  if (e == cudaSuccess) done[dev].store(true, std::memory_order_release);
  return e;
}

template <typename T, typename W, typename O>
void launch_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& res, at::Tensor& s, const at::Tensor& w,
                at::Tensor& y, at::Tensor& rstd, int64_t rows, int d, float eps) {
  const T* rp = res ? reinterpret_cast<const T*>(res->data_ptr()) : nullptr;
  T* sp = res ? reinterpret_cast<T*>(s.data_ptr()) : nullptr;
  auto xp = reinterpret_cast<const T*>(x.data_ptr());
  auto wp = reinterpret_cast<const W*>(w.data_ptr());
  auto yp = reinterpret_cast<O*>(y.data_ptr());
  auto rs = rstd.data_ptr<float>();
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps)), block(kWarps * 32);
  auto st = stream();
  switch (d % 256 == 0 ? d / 256 : 0) {
#define LRB_NV(n) case n: rmsnorm_fwd_reg<T, W, O, n><<<grid, block, 0, st>>>(xp, rp, sp, wp, yp, rs, rows, d, eps); break;
    LRB_NV(1) LRB_NV(2) LRB_NV(3) LRB_NV(4) LRB_NV(6) LRB_NV(8) LRB_NV(12) LRB_NV(16)
#undef LRB_NV
    default: rmsnorm_fwd_generic<T, W, O><<<grid, block, 0, st>>>(xp, rp, sp, wp, yp, rs, rows, d, eps);
  }
  LRB_LAUNCH_CHECK();
}

}  // namespace

// y = norm(x [+ residual]) * w; returns (y, rstd, s = x + residual or None)
std::tuple<at::Tensor, at::Tensor, c10::optional<at::Tensor>> rmsnorm_fwd(
    const at::Tensor& x, const at::Tensor& w, double eps, const c10::optional<at::Tensor>& residual,
    at::ScalarType out_dtype) {
  LRB_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "rmsnorm_fwd: x must be contiguous 2-D CUDA");
  const int64_t rows = x.size(0);
  const int d = (int)x.size(1);
  LRB_CHECK(w.numel() == d && w.is_contiguous(), "rmsnorm_fwd: weight size mismatch");
  c10::cuda::CUDAGuard g(x.device());
  bind_device(x.get_device());
  auto y = at::empty({rows, d}, x.options().dtype(out_dtype));
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor s;
  if (residual) {
    LRB_CHECK(residual->sizes() == x.sizes() && residual->scalar_type() == x.scalar_type(), "residual mismatch");
    s = at::empty_like(x);
  }
  if (rows == 0) return {y, rstd, residual ? c10::optional<at::Tensor>(s) : c10::nullopt};
  const auto xt = x.scalar_type(), wt = w.scalar_type();
  if (xt == at::kBFloat16 && wt == at::kBFloat16 && out_dtype == at::kBFloat16)
    launch_fwd<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(x, residual, s, w, y, rstd, rows, d, (float)eps);
  else if (xt == at::kBFloat16 && wt == at::kFloat && out_dtype == at::kFloat)
    launch_fwd<__nv_bfloat16, float, float>(x, residual, s, w, y, rstd, rows, d, (float)eps);
  else if (xt == at::kFloat && wt == at::kFloat && out_dtype == at::kFloat)
    launch_fwd<float, float, float>(x, residual, s, w, y, rstd, rows, d, (float)eps);
  else if (xt == at::kHalf && wt == at::kHalf && out_dtype == at::kHalf)
    launch_fwd<__half, __half, __half>(x, residual, s, w, y, rstd, rows, d, (float)eps);
  else if (xt == at::kFloat && wt == at::kBFloat16 && out_dtype == at::kFloat)
    launch_fwd<float, __nv_bfloat16, float>(x, residual, s, w, y, rstd, rows, d, (float)eps);
  else
    LRB_CHECK(false, "rmsnorm_fwd: unsupported dtype combination");
  return {y, rstd, residual ? c10::optional<at::Tensor>(s) : c10::nullopt};
}

std::tuple<at::Tensor, at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                               const at::Tensor& rstd, const c10::optional<at::Tensor>& ds) {
  LRB_CHECK(dy.is_contiguous() && x.is_contiguous(), "rmsnorm_bwd: contiguous inputs required");
  const int64_t rows = x.size(0);
  const int d = (int)x.size(1);
  c10::cuda::CUDAGuard g(x.device());
  bind_device(x.get_device());
  auto dx = at::empty_like(x);
  auto dw = at::zeros({d}, x.options().dtype(at::kFloat));
  if (rows == 0) return {dx, dw};
  const size_t smem = (size_t)kWarps * d * sizeof(float);
  LRB_CHECK(smem <= (size_t)kBwdSmemMax, "rmsnorm_bwd: row too wide");
  const auto xt = x.scalar_type(), wt = w.scalar_type(), ot = dy.scalar_type();
  const bool reg = xt == at::kBFloat16 && wt == at::kBFloat16 && ot == at::kBFloat16 && d % 256 == 0 &&
                   d / 256 <= 8 && (!ds || ds->is_contiguous());
  int blocks = (int)std::min<int64_t>((rows + kWarps - 1) / kWarps, 2 * num_sms());
  auto part = at::empty({blocks, d}, x.options().dtype(at::kFloat));
  auto st = stream();
  if (reg) {
    using B16 = __nv_bfloat16;
    auto go = [&](auto kernel) {
      if (smem > 48 * 1024) LRB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                                (int)kBwdSmemMax));
      kernel<<<blocks, kWarps * 32, smem, st>>>(
          reinterpret_cast<const B16*>(dy.data_ptr()), reinterpret_cast<const B16*>(x.data_ptr()),
          reinterpret_cast<const B16*>(w.data_ptr()), rstd.data_ptr<float>(),
          ds ? reinterpret_cast<const B16*>(ds->data_ptr()) : nullptr, reinterpret_cast<B16*>(dx.data_ptr()),
          part.data_ptr<float>(), rows, d);
      LRB_LAUNCH_CHECK();
    };
    switch (d / 256) {
      case 1: go(rmsnorm_bwd_reg<1>); break;
      case 2: go(rmsnorm_bwd_reg<2>); break;
      case 3: go(rmsnorm_bwd_reg<3>); break;
      case 4: go(rmsnorm_bwd_reg<4>); break;
      case 5: go(rmsnorm_bwd_reg<5>); break;
      case 6: go(rmsnorm_bwd_reg<6>); break;
      case 7: go(rmsnorm_bwd_reg<7>); break;
      default: go(rmsnorm_bwd_reg<8>); break;
    }
    reduce_rows_kernel<<<(d + 255) / 256, 256, 0, st>>>(part.data_ptr<float>(), dw.data_ptr<float>(), blocks, d);
    LRB_LAUNCH_CHECK();
    return {dx, dw};
  }
  auto run = [&](auto tag_t, auto tag_w, auto tag_o) {
    using T = decltype(tag_t);
    using W = decltype(tag_w);
    using O = decltype(tag_o);
    auto k = rmsnorm_bwd_kernel<T, W, O>;
    if (smem > 48 * 1024) LRB_CUDA_CHECK((raise_bwd_smem_limit<T, W, O>(x.get_device())));
    k<<<blocks, kWarps * 32, smem, st>>>(
        reinterpret_cast<const O*>(dy.data_ptr()), reinterpret_cast<const T*>(x.data_ptr()),
        reinterpret_cast<const W*>(w.data_ptr()), rstd.data_ptr<float>(),
        ds ? reinterpret_cast<const T*>(ds->data_ptr()) : nullptr, reinterpret_cast<T*>(dx.data_ptr()),
        part.data_ptr<float>(), rows, d);
    LRB_LAUNCH_CHECK();
  };
  if (xt == at::kBFloat16 && wt == at::kBFloat16 && ot == at::kBFloat16) run(__nv_bfloat16{}, __nv_bfloat16{}, __nv_bfloat16{});
  else if (xt == at::kBFloat16 && wt == at::kFloat && ot == at::kFloat) run(__nv_bfloat16{}, float{}, float{});
  else if (xt == at::kFloat && wt == at::kFloat && ot == at::kFloat) run(float{}, float{}, float{});
  else if (xt == at::kHalf && wt == at::kHalf && ot == at::kHalf) run(__half{}, __half{}, __half{});
  else if (xt == at::kFloat && wt == at::kBFloat16 && ot == at::kFloat) run(float{}, __nv_bfloat16{}, float{});
  else LRB_CHECK(false, "rmsnorm_bwd: unsupported dtype combination");
  reduce_rows_kernel<<<(d + 255) / 256, 256, 0, st>>>(part.data_ptr<float>(), dw.data_ptr<float>(), blocks, d);
  LRB_LAUNCH_CHECK();
  return {dx, dw};
}

}  // namespace lrb

// ------------------------------------------------- allocation-free entry point
// Variant of rmsnorm_bwd for callers that cannot allocate device memory (the
// cases are listed in lrb_noalloc.h): the per-block weight-gradient partials go
// to this fixed 4 MiB array instead of a freshly allocated tensor.
static __device__ __align__(256) float g_rmsnorm_bwd_scratch[LRB_RMSNORM_BWD_NOALLOC_SCRATCH_FLOATS];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::atomic<float*> g_noalloc_scratch[kNoAllocMaxDevices];
int g_noalloc_blocks_cap[kNoAllocMaxDevices];
std::mutex g_noalloc_setup_mu;

int noalloc_fail(char* buf, int len, int code, const char* fmt, ...) {
  if (buf != nullptr && len > 0) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, (size_t)len, fmt, ap);
    va_end(ap);
  }
  return code;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int lrb_rmsnorm_bwd_bf16_noalloc(
    const void* dy, const void* x, const void* w, const float* rstd, const void* ds, void* dx, float* dw,
    int64_t rows, int64_t d, void* stream, char* errbuf, int errbuf_len) {
  using lrb::kWarps;
  using T = __nv_bfloat16;
  if (dy == nullptr || x == nullptr || w == nullptr || rstd == nullptr || dx == nullptr || dw == nullptr)
    return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_ARGS, "rmsnorm_bwd_noalloc: null pointer argument");
  if (rows <= 0 || d <= 0)
    return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_ARGS,
                        "rmsnorm_bwd_noalloc: rows (%lld) and d (%lld) must be positive", (long long)rows,
                        (long long)d);
  if (d > LRB_RMSNORM_BWD_NOALLOC_MAX_D)
    return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_TOO_LARGE,
                        "rmsnorm_bwd_noalloc: row width d=%lld exceeds the maximum %d", (long long)d,
                        LRB_RMSNORM_BWD_NOALLOC_MAX_D);
  if (!aligned16(dy) || !aligned16(x) || !aligned16(w) || !aligned16(dx) || (ds != nullptr && !aligned16(ds)))
    return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_ARGS,
                        "rmsnorm_bwd_noalloc: dy, x, w, ds and dx must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_CUDA, "rmsnorm_bwd_noalloc: cudaGetDevice: %s",
                        cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_ARGS, "rmsnorm_bwd_noalloc: device %d out of range",
                        dev);
  const size_t smem = (size_t)kWarps * (size_t)d * sizeof(float);
  float* scratch = g_noalloc_scratch[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    // One-time setup per device, with that device current (the caller's).
    std::lock_guard<std::mutex> lock(g_noalloc_setup_mu);
    scratch = g_noalloc_scratch[dev].load(std::memory_order_acquire);
    if (scratch == nullptr) {
      float* p = nullptr;
      e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_rmsnorm_bwd_scratch);
      if (e != cudaSuccess || p == nullptr)
        return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_CUDA,
                            "rmsnorm_bwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      int sms = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess)
        return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_CUDA, "rmsnorm_bwd_noalloc: SM count: %s",
                            cudaGetErrorString(e));
      g_noalloc_blocks_cap[dev] = 2 * sms;
      g_noalloc_scratch[dev].store(p, std::memory_order_release);
      scratch = p;
    }
  }
  int64_t blocks = (rows + kWarps - 1) / kWarps;
  blocks = std::min<int64_t>(blocks, g_noalloc_blocks_cap[dev]);
  blocks = std::min<int64_t>(blocks, LRB_RMSNORM_BWD_NOALLOC_SCRATCH_FLOATS / d);
  if (smem > 48 * 1024) {
    // Raised once per device to the kernel's maximum and never lowered (shared
    // with rmsnorm_bwd, which launches the same kernel instance).
    e = lrb::raise_bwd_smem_limit<T, T, T>(dev);
    if (e != cudaSuccess)
      return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_CUDA, "rmsnorm_bwd_noalloc: smem attribute: %s",
                          cudaGetErrorString(e));
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  lrb::rmsnorm_bwd_kernel<T, T, T><<<(unsigned)blocks, kWarps * 32, smem, st>>>(
      reinterpret_cast<const T*>(dy), reinterpret_cast<const T*>(x), reinterpret_cast<const T*>(w), rstd,
      reinterpret_cast<const T*>(ds), reinterpret_cast<T*>(dx), scratch, rows, (int)d);
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_CUDA, "rmsnorm_bwd_noalloc: launch: %s",
                        cudaGetErrorString(e));
  lrb::reduce_rows_kernel<<<(unsigned)((d + 255) / 256), 256, 0, st>>>(scratch, dw, (int)blocks, (int)d);
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return noalloc_fail(errbuf, errbuf_len, LRB_NOALLOC_ERR_CUDA, "rmsnorm_bwd_noalloc: reduce launch: %s",
                        cudaGetErrorString(e));
  return LRB_NOALLOC_OK;
}
