// Cross-entropy over vocabulary rows: one block per row, single pass with an
// online (max, sum-exp) accumulator; the backward writes the gradient rows
// directly in the logits dtype.
#include "../common.cuh"

namespace lrb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) { m = mn; s = 0.f; return; }
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) ce_fwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ tgt,
                                                          float* __restrict__ lse_out, float* __restrict__ loss_sum,
                                                          float* __restrict__ count, int64_t V, int64_t ignore) {
  __shared__ float red_m[32], red_s[32];
  const int64_t row = blockIdx.x;
  const T* x = logits + row * V;
  float m = -INFINITY, s = 0.f;
  const bool vec = (sizeof(T) == 2) && (V % 8 == 0);
  if (vec) {
    for (int64_t c = threadIdx.x * 8; c < V; c += kThreads * 8) {
      Vec16<T> v = ld16(x + c);
      float f[8], lm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) { f[j] = to_f(v.v[j]); lm = fmaxf(lm, f[j]); }
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ls += __expf(f[j] - lm);
      online_merge(m, s, lm, ls);
    }
  } else {
    for (int64_t c = threadIdx.x; c < V; c += kThreads) online_merge(m, s, to_f(x[c]), 1.f);
  }
  // warp reduce
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { red_m[wid] = m; red_s[wid] = s; }
  __syncthreads();
  if (wid == 0) {
    m = lane < kThreads / 32 ? red_m[lane] : -INFINITY;
    s = lane < kThreads / 32 ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const float lse = m + __logf(s);
      lse_out[row] = lse;
      const int64_t t = tgt[row];
      if (t != ignore && t >= 0 && t < V) {
        atomicAdd(loss_sum, lse - to_f(x[t]));
        atomicAdd(count, 1.f);
      }
    }
  }
}

// kShard: the logits are one vocabulary shard and lse is the row's log-sum-exp over the
// whole vocabulary; a target outside [0, V) belongs to another shard, so the row still
// takes the softmax gradient, without the one-hot term.  Otherwise such a row is ignored.
template <typename T, bool kShard>
__global__ void __launch_bounds__(kThreads) ce_bwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ tgt,
                                                          const float* __restrict__ lse, const float* __restrict__ scale,
                                                          T* __restrict__ dx, int64_t V, int64_t ignore) {
  const int64_t row = blockIdx.x;
  const T* x = logits + row * V;
  T* d = dx + row * V;
  const int64_t t = tgt[row];
  const bool counted = kShard ? (t != ignore) : (t != ignore && t >= 0 && t < V);
  const float g = counted ? scale[0] : 0.f;
  const float l = lse[row];
  const bool vec = (sizeof(T) == 2) && (V % 8 == 0);
  if (vec) {
    for (int64_t c = threadIdx.x * 8; c < V; c += kThreads * 8) {
      Vec16<T> v = ld16(x + c), o;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float p = __expf(to_f(v.v[j]) - l);
        if (c + j == t) p -= 1.f;
        o.v[j] = from_f<T>(p * g);
      }
      st16(d + c, o);
    }
  } else {
    for (int64_t c = threadIdx.x; c < V; c += kThreads) {
      float p = __expf(to_f(x[c]) - l);
      if (c == t) p -= 1.f;
      d[c] = from_f<T>(p * g);
    }
  }
}

}  // namespace

// Returns (sum of row losses, number of counted rows, per-row lse), all fp32.
std::tuple<at::Tensor, at::Tensor, at::Tensor> ce_fwd(const at::Tensor& logits, const at::Tensor& targets,
                                                      int64_t ignore_index) {
  LRB_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.is_contiguous(), "ce_fwd: logits must be contiguous 2-D");
  LRB_CHECK(targets.scalar_type() == at::kLong && targets.numel() == logits.size(0), "ce_fwd: bad targets");
  c10::cuda::CUDAGuard g(logits.device());
  bind_device(logits.get_device());
  const int64_t R = logits.size(0), V = logits.size(1);
  auto f32 = logits.options().dtype(at::kFloat);
  auto lse = at::empty({R}, f32);
  auto acc = at::zeros({2}, f32);
  if (R > 0) {
    LRB_DISPATCH_FLOAT(logits.scalar_type(), T, [&] {
      ce_fwd_kernel<T><<<(unsigned)R, kThreads, 0, stream()>>>(reinterpret_cast<const T*>(logits.data_ptr()),
                                                             targets.data_ptr<int64_t>(), lse.data_ptr<float>(),
                                                             acc.data_ptr<float>(), acc.data_ptr<float>() + 1, V,
                                                             ignore_index);
    });
    LRB_LAUNCH_CHECK();
  }
  return {acc[0], acc[1], lse};
}

namespace {
at::Tensor ce_bwd_impl(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& lse,
                       const at::Tensor& scale, int64_t ignore_index, bool shard) {
  LRB_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.is_contiguous(), "ce_bwd: logits must be contiguous 2-D");
  LRB_CHECK(targets.scalar_type() == at::kLong && targets.numel() == logits.size(0), "ce_bwd: bad targets");
  LRB_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == logits.size(0), "ce_bwd: lse must be fp32 per row");
  c10::cuda::CUDAGuard g(logits.device());
  bind_device(logits.get_device());
  const int64_t R = logits.size(0), V = logits.size(1);
  auto dx = at::empty_like(logits);
  auto sc = scale.to(at::kFloat).reshape({1}).contiguous();
  auto tg = targets.contiguous();
  auto ls = lse.contiguous();
  if (R > 0) {
    LRB_DISPATCH_FLOAT(logits.scalar_type(), T, [&] {
      auto kern = shard ? ce_bwd_kernel<T, true> : ce_bwd_kernel<T, false>;
      kern<<<(unsigned)R, kThreads, 0, stream()>>>(
          reinterpret_cast<const T*>(logits.data_ptr()), tg.data_ptr<int64_t>(), ls.data_ptr<float>(),
          sc.data_ptr<float>(), reinterpret_cast<T*>(dx.data_ptr()), V, ignore_index);
    });
    LRB_LAUNCH_CHECK();
  }
  return dx;
}
}  // namespace

at::Tensor ce_bwd(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& lse, const at::Tensor& scale,
                  int64_t ignore_index) {
  return ce_bwd_impl(logits, targets, lse, scale, ignore_index, false);
}

// Gradient of one vocabulary shard's logits: targets are shard-local ids (outside
// [0, V) when another shard owns the target), lse the full-vocabulary log-sum-exp.
at::Tensor ce_bwd_vocab_shard(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& lse,
                              const at::Tensor& scale, int64_t ignore_index) {
  return ce_bwd_impl(logits, targets, lse, scale, ignore_index, true);
}

}  // namespace lrb
