// SwiGLU gating (input [up | gate], output silu(gate) * up) and the fused QKV
// split + RoPE, forward and backward.
#include "../common.cuh"

namespace lrb {
namespace {

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

// gu: (rows, 2F) = [up | gate];  h: (rows, F)
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ h, int64_t rows, int64_t F) {
  const int64_t n = rows * F;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, c = i - r * F;
    const float u = to_f(gu[r * 2 * F + c]);
    const float g = to_f(gu[r * 2 * F + F + c]);
    h[i] = from_f<T>(g * sigmoidf_(g) * u);
  }
}

// Vectorised variant: 8 elements per thread (F % 8 == 0, 2-byte types).
template <typename T>
__global__ void swiglu_fwd_vec(const T* __restrict__ gu, T* __restrict__ h, int64_t rows, int64_t F) {
  const int64_t nv = rows * (F / 8);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (F / 8), c = (i - r * (F / 8)) * 8;
    Vec16<T> u = ld16(gu + r * 2 * F + c), g = ld16(gu + r * 2 * F + F + c), o;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gf = to_f(g.v[j]);
      o.v[j] = from_f<T>(gf * sigmoidf_(gf) * to_f(u.v[j]));
    }
    st16(h + r * F + c, o);
  }
}

template <typename T>
__global__ void swiglu_bwd_vec(const T* __restrict__ dh, const T* __restrict__ gu, T* __restrict__ dgu, int64_t rows,
                               int64_t F) {
  const int64_t nv = rows * (F / 8);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (F / 8), c = (i - r * (F / 8)) * 8;
    Vec16<T> d = ld16(dh + r * F + c), u = ld16(gu + r * 2 * F + c), g = ld16(gu + r * 2 * F + F + c), og, ou;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gf = to_f(g.v[j]), uf = to_f(u.v[j]), df = to_f(d.v[j]);
      const float s = sigmoidf_(gf);
      og.v[j] = from_f<T>(df * uf * s * (1.f + gf * (1.f - s)));
      ou.v[j] = from_f<T>(df * gf * s);
    }
    st16(dgu + r * 2 * F + c, ou);
    st16(dgu + r * 2 * F + F + c, og);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ dh, const T* __restrict__ gu, T* __restrict__ dgu,
                                  int64_t rows, int64_t F) {
  const int64_t n = rows * F;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, c = i - r * F;
    const float u = to_f(gu[r * 2 * F + c]), g = to_f(gu[r * 2 * F + F + c]), d = to_f(dh[i]);
    const float s = sigmoidf_(g);
    dgu[r * 2 * F + F + c] = from_f<T>(d * u * s * (1.f + g * (1.f - s)));
    dgu[r * 2 * F + c] = from_f<T>(d * g * s);
  }
}

inline int grid_for(int64_t n, int threads) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, (int64_t)num_sms() * 16));
}

// ------------------------------------------------------------------ RoPE
// Vectorised form (2-byte types, D % 16 == 0): one block per token; the
// token's cos/sin rows are staged in shared memory once and every thread
// rotates 8 pairs with two 16-byte loads and two 16-byte stores.
template <typename T, bool BWD>
__global__ void __launch_bounds__(128) rope_qkv_vec_kernel(const T* __restrict__ src0, const T* __restrict__ src_k,
                                                          const T* __restrict__ src_v, const float* __restrict__ cos_t,
                                                          const float* __restrict__ sin_t, T* __restrict__ dst0,
                                                          T* __restrict__ dst_k, T* __restrict__ dst_v, int S, int H,
                                                          int Hkv, int D, int offset) {
  extern __shared__ float tab[];  // cos[0:D], sin[D:2D]
  const int64_t t = blockIdx.x;
  const int pos = (int)(t % S) + offset;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    tab[i] = cos_t[(int64_t)pos * D + i];
    tab[D + i] = sin_t[(int64_t)pos * D + i];
  }
  __syncthreads();
  const int half = D / 2, groups = half / 8, heads = H + 2 * Hkv;
  const int64_t row = (int64_t)heads * D;
  for (int w = threadIdx.x; w < heads * groups; w += blockDim.x) {
    const int h = w / groups, j = (w - (w / groups) * groups) * 8;
    // forward: src0 = packed qkv row, dst = q/k/v; backward: the reverse.
    const T* in;
    T* out;
    if (!BWD) {
      in = src0 + t * row + (int64_t)h * D;
      out = h < H ? dst0 + (t * H + h) * D : (h < H + Hkv ? dst_k + (t * Hkv + h - H) * D : dst_v + (t * Hkv + h - H - Hkv) * D);
    } else {
      in = h < H ? src0 + (t * H + h) * D : (h < H + Hkv ? src_k + (t * Hkv + h - H) * D : src_v + (t * Hkv + h - H - Hkv) * D);
      out = dst0 + t * row + (int64_t)h * D;
    }
    Vec16<T> a = ld16(in + j), b = ld16(in + j + half);
    if (h < H + Hkv) {
      Vec16<T> oa, ob;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float x = to_f(a.v[e]), y = to_f(b.v[e]);
        const float c = tab[j + e], s = tab[D + j + e], c2 = tab[half + j + e], s2 = tab[D + half + j + e];
        if (!BWD) {
          oa.v[e] = from_f<T>(x * c - y * s);
          ob.v[e] = from_f<T>(y * c2 + x * s2);
        } else {
          oa.v[e] = from_f<T>(x * c + y * s2);
          ob.v[e] = from_f<T>(y * c2 - x * s);
        }
      }
      st16(out + j, oa);
      st16(out + j + half, ob);
    } else {
      st16(out + j, a);
      st16(out + j + half, b);
    }
  }
}

// Scalar form: qkv row layout [q: H*D | k: Hkv*D | v: Hkv*D]; one thread per (token, head, i < D/2) pair.
template <typename T>
__global__ void rope_qkv_fwd_kernel(const T* __restrict__ qkv, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, T* __restrict__ q, T* __restrict__ k,
                                    T* __restrict__ v, int64_t tokens, int S, int H, int Hkv, int D, int offset) {
  const int half = D / 2;
  const int heads = H + 2 * Hkv;
  const int64_t n = tokens * heads * half;
  const int64_t row = (int64_t)heads * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const int64_t th = i / half;
    const int h = (int)(th % heads);
    const int64_t t = th / heads;
    const int pos = (int)(t % S) + offset;
    const T* src = qkv + t * row + (int64_t)h * D;
    const float a = to_f(src[j]), b = to_f(src[j + half]);
    if (h < H + Hkv) {
      const float c = cos_t[(int64_t)pos * D + j], s = sin_t[(int64_t)pos * D + j];
      const float c2 = cos_t[(int64_t)pos * D + j + half], s2 = sin_t[(int64_t)pos * D + j + half];
      T* dst = h < H ? q + (t * H + h) * D : k + (t * Hkv + (h - H)) * D;
      dst[j] = from_f<T>(a * c - b * s);
      dst[j + half] = from_f<T>(b * c2 + a * s2);
    } else {
      T* dst = v + (t * Hkv + (h - H - Hkv)) * D;
      dst[j] = src[j];
      dst[j + half] = src[j + half];
    }
  }
}

template <typename T>
__global__ void rope_qkv_bwd_kernel(const T* __restrict__ dq, const T* __restrict__ dk, const T* __restrict__ dv,
                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                    T* __restrict__ dqkv, int64_t tokens, int S, int H, int Hkv, int D, int offset) {
  const int half = D / 2;
  const int heads = H + 2 * Hkv;
  const int64_t n = tokens * heads * half;
  const int64_t row = (int64_t)heads * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const int64_t th = i / half;
    const int h = (int)(th % heads);
    const int64_t t = th / heads;
    const int pos = (int)(t % S) + offset;
    T* dst = dqkv + t * row + (int64_t)h * D;
    if (h < H + Hkv) {
      const T* g = h < H ? dq + (t * H + h) * D : dk + (t * Hkv + (h - H)) * D;
      const float ga = to_f(g[j]), gb = to_f(g[j + half]);
      const float c = cos_t[(int64_t)pos * D + j], s = sin_t[(int64_t)pos * D + j];
      const float c2 = cos_t[(int64_t)pos * D + j + half], s2 = sin_t[(int64_t)pos * D + j + half];
      // out_a = a c - b s ; out_b = b c2 + a s2   =>  da = ga c + gb s2 ; db = -ga s + gb c2
      dst[j] = from_f<T>(ga * c + gb * s2);
      dst[j + half] = from_f<T>(gb * c2 - ga * s);
    } else {
      const T* g = dv + (t * Hkv + (h - H - Hkv)) * D;
      dst[j] = g[j];
      dst[j + half] = g[j + half];
    }
  }
}

}  // namespace

at::Tensor swiglu_fwd(const at::Tensor& gu) {
  LRB_CHECK(gu.is_cuda() && gu.is_contiguous() && gu.size(-1) % 2 == 0, "swiglu_fwd: bad input");
  c10::cuda::CUDAGuard g(gu.device());
  bind_device(gu.get_device());
  const int64_t F = gu.size(-1) / 2, rows = gu.numel() / gu.size(-1);
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto h = at::empty(sizes, gu.options());
  if (rows == 0) return h;
  LRB_DISPATCH_FLOAT(gu.scalar_type(), T, [&] {
    if (sizeof(T) == 2 && F % 8 == 0) {
      swiglu_fwd_vec<T><<<grid_for(rows * F / 8, 256), 256, 0, stream()>>>(
          reinterpret_cast<const T*>(gu.data_ptr()), reinterpret_cast<T*>(h.data_ptr()), rows, F);
    } else {
      swiglu_fwd_kernel<T><<<grid_for(rows * F, 256), 256, 0, stream()>>>(
          reinterpret_cast<const T*>(gu.data_ptr()), reinterpret_cast<T*>(h.data_ptr()), rows, F);
    }
  });
  LRB_LAUNCH_CHECK();
  return h;
}

at::Tensor swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu) {
  c10::cuda::CUDAGuard g(gu.device());
  bind_device(gu.get_device());
  const int64_t F = gu.size(-1) / 2, rows = gu.numel() / gu.size(-1);
  auto dgu = at::empty_like(gu);
  if (rows == 0) return dgu;
  LRB_DISPATCH_FLOAT(gu.scalar_type(), T, [&] {
    if (sizeof(T) == 2 && F % 8 == 0) {
      swiglu_bwd_vec<T><<<grid_for(rows * F / 8, 256), 256, 0, stream()>>>(
          reinterpret_cast<const T*>(dh.data_ptr()), reinterpret_cast<const T*>(gu.data_ptr()),
          reinterpret_cast<T*>(dgu.data_ptr()), rows, F);
    } else {
      swiglu_bwd_kernel<T><<<grid_for(rows * F, 256), 256, 0, stream()>>>(
          reinterpret_cast<const T*>(dh.data_ptr()), reinterpret_cast<const T*>(gu.data_ptr()),
          reinterpret_cast<T*>(dgu.data_ptr()), rows, F);
    }
  });
  LRB_LAUNCH_CHECK();
  return dgu;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> rope_qkv_fwd(const at::Tensor& qkv, const at::Tensor& cos_t,
                                                            const at::Tensor& sin_t, int64_t H, int64_t Hkv,
                                                            int64_t D, int64_t offset) {
  LRB_CHECK(qkv.is_cuda() && qkv.dim() == 3 && qkv.is_contiguous(), "rope_qkv_fwd: qkv must be contiguous (B,S,N)");
  LRB_CHECK(qkv.size(2) == (H + 2 * Hkv) * D && D % 2 == 0, "rope_qkv_fwd: width mismatch");
  LRB_CHECK(cos_t.scalar_type() == at::kFloat && cos_t.size(-1) == D, "rope tables must be fp32 (S, D)");
  LRB_CHECK(cos_t.size(0) >= offset + qkv.size(1), "rope table too short");
  c10::cuda::CUDAGuard g(qkv.device());
  bind_device(qkv.get_device());
  const int64_t B = qkv.size(0), S = qkv.size(1);
  auto q = at::empty({B, S, H, D}, qkv.options());
  auto k = at::empty({B, S, Hkv, D}, qkv.options());
  auto v = at::empty({B, S, Hkv, D}, qkv.options());
  const int64_t n = B * S * (H + 2 * Hkv) * (D / 2);
  if (n == 0) return {q, k, v};
  LRB_DISPATCH_FLOAT(qkv.scalar_type(), T, [&] {
    if (sizeof(T) == 2 && D % 16 == 0) {
      rope_qkv_vec_kernel<T, false><<<(unsigned)(B * S), 128, 2 * D * sizeof(float), stream()>>>(
          reinterpret_cast<const T*>(qkv.data_ptr()), nullptr, nullptr, cos_t.data_ptr<float>(),
          sin_t.data_ptr<float>(), reinterpret_cast<T*>(q.data_ptr()), reinterpret_cast<T*>(k.data_ptr()),
          reinterpret_cast<T*>(v.data_ptr()), (int)S, (int)H, (int)Hkv, (int)D, (int)offset);
      return;
    }
    rope_qkv_fwd_kernel<T><<<grid_for(n, 256), 256, 0, stream()>>>(
        reinterpret_cast<const T*>(qkv.data_ptr()), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
        reinterpret_cast<T*>(q.data_ptr()), reinterpret_cast<T*>(k.data_ptr()), reinterpret_cast<T*>(v.data_ptr()),
        B * S, (int)S, (int)H, (int)Hkv, (int)D, (int)offset);
  });
  LRB_LAUNCH_CHECK();
  return {q, k, v};
}

at::Tensor rope_qkv_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv, const at::Tensor& cos_t,
                        const at::Tensor& sin_t, int64_t H, int64_t Hkv, int64_t D, int64_t offset) {
  c10::cuda::CUDAGuard g(dq.device());
  bind_device(dq.get_device());
  const int64_t B = dq.size(0), S = dq.size(1);
  auto dqkv = at::empty({B, S, (H + 2 * Hkv) * D}, dq.options());
  const int64_t n = B * S * (H + 2 * Hkv) * (D / 2);
  if (n == 0) return dqkv;
  LRB_DISPATCH_FLOAT(dq.scalar_type(), T, [&] {
    if (sizeof(T) == 2 && D % 16 == 0) {
      rope_qkv_vec_kernel<T, true><<<(unsigned)(B * S), 128, 2 * D * sizeof(float), stream()>>>(
          reinterpret_cast<const T*>(dq.data_ptr()), reinterpret_cast<const T*>(dk.data_ptr()),
          reinterpret_cast<const T*>(dv.data_ptr()), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
          reinterpret_cast<T*>(dqkv.data_ptr()), nullptr, nullptr, (int)S, (int)H, (int)Hkv, (int)D, (int)offset);
      return;
    }
    rope_qkv_bwd_kernel<T><<<grid_for(n, 256), 256, 0, stream()>>>(
        reinterpret_cast<const T*>(dq.data_ptr()), reinterpret_cast<const T*>(dk.data_ptr()),
        reinterpret_cast<const T*>(dv.data_ptr()), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
        reinterpret_cast<T*>(dqkv.data_ptr()), B * S, (int)S, (int)H, (int)Hkv, (int)D, (int)offset);
  });
  LRB_LAUNCH_CHECK();
  return dqkv;
}


// y = exp2_fma(x) elementwise (fp32): the FMA-pipe 2^x of the attention softmax,
// exposed so its accuracy can be checked against the library's exp2.
__global__ void exp2_fma_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = exp2_fma(x[i]);
}

at::Tensor exp2_fma_eval(const at::Tensor& x) {
  LRB_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous(), "exp2_fma_eval: contiguous fp32 CUDA");
  c10::cuda::CUDAGuard g(x.device());
  bind_device(x.get_device());
  auto y = at::empty_like(x);
  const int64_t n = x.numel();
  if (n == 0) return y;
  exp2_fma_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, stream()>>>(x.data_ptr<float>(),
                                                                                          y.data_ptr<float>(), n);
  LRB_LAUNCH_CHECK();
  return y;
}

}  // namespace lrb
