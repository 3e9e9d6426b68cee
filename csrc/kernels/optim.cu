// Multi-tensor optimizer kernels: Muon prologue/epilogue and AdamW.
//
// A launch covers up to kMaxTensors tensors described in a by-value table;
// every tensor is cut into kChunk-element slices and each block owns one
// slice, locating its tensor by a linear scan of the (small) prefix table.
#include "../common.cuh"

#include <vector>

namespace lrb {
namespace {

constexpr int kMaxTensors = 36;
constexpr int kChunk = 8192;
constexpr int kThreads = 256;

struct Table {
  void* a[kMaxTensors];    // param
  void* b[kMaxTensors];    // grad / orth
  void* c[kMaxTensors];    // momentum buffer / exp_avg
  void* d[kMaxTensors];    // nesterov out / exp_avg_sq
  int64_t n[kMaxTensors];
  int block_start[kMaxTensors + 1];
  float f0[kMaxTensors];   // per-tensor scalars (bias corrections)
  float f1[kMaxTensors];
  int count;
};

__device__ __forceinline__ int find_tensor(const Table& t, int blk) {
  int i = 0;
  while (i + 1 < t.count && t.block_start[i + 1] <= blk) ++i;
  return i;
}

// p *= 1 - lr*wd ; buf = mu*buf + g ; u = g + mu*buf ; gsq[i] += sum(g^2)
template <typename P, typename U>
__global__ void __launch_bounds__(kThreads) muon_prologue_kernel(Table t, float decay, float mu, float* gsq, int base) {
  __shared__ float red[32];
  const int i = find_tensor(t, blockIdx.x);
  const int64_t off = (int64_t)(blockIdx.x - t.block_start[i]) * kChunk;
  const int64_t end = min(off + (int64_t)kChunk, t.n[i]);
  P* p = reinterpret_cast<P*>(t.a[i]);
  const P* g = reinterpret_cast<const P*>(t.b[i]);
  P* buf = reinterpret_cast<P*>(t.c[i]);
  U* u = reinterpret_cast<U*>(t.d[i]);
  float ss = 0.f;
  for (int64_t e = off + threadIdx.x; e < end; e += kThreads) {
    const float gv = to_f(g[e]);
    const float bv = mu * to_f(buf[e]) + gv;
    buf[e] = from_f<P>(bv);
    u[e] = from_f<U>(gv + mu * bv);
    if (decay != 1.f) p[e] = from_f<P>(to_f(p[e]) * decay);
    ss += gv * gv;
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) atomicAdd(gsq + base + i, ss);
}

template <typename O>
__global__ void __launch_bounds__(kThreads) sumsq_kernel(Table t, float* out, int base) {
  __shared__ float red[32];
  const int i = find_tensor(t, blockIdx.x);
  const int64_t off = (int64_t)(blockIdx.x - t.block_start[i]) * kChunk;
  const int64_t end = min(off + (int64_t)kChunk, t.n[i]);
  const O* o = reinterpret_cast<const O*>(t.b[i]);
  float ss = 0.f;
  for (int64_t e = off + threadIdx.x; e < end; e += kThreads) {
    const float v = to_f(o[e]);
    ss += v * v;
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) atomicAdd(out + base + i, ss);
}

// p -= lr * gnorm / (sqrt(osq) + 1e-8) * o
template <typename P, typename O>
__global__ void __launch_bounds__(kThreads) muon_update_kernel(Table t, const float* gnorm, const float* osq, float lr,
                                                                int base) {
  const int i = find_tensor(t, blockIdx.x);
  const int64_t off = (int64_t)(blockIdx.x - t.block_start[i]) * kChunk;
  const int64_t end = min(off + (int64_t)kChunk, t.n[i]);
  P* p = reinterpret_cast<P*>(t.a[i]);
  const O* o = reinterpret_cast<const O*>(t.b[i]);
  const float scale = lr * gnorm[base + i] / (sqrtf(osq[base + i]) + 1e-8f);
  for (int64_t e = off + threadIdx.x; e < end; e += kThreads) p[e] = from_f<P>(to_f(p[e]) - scale * to_f(o[e]));
}

// x += alpha * y
template <typename X, typename Y>
__global__ void __launch_bounds__(kThreads) axpy_kernel(Table t, float alpha) {
  const int i = find_tensor(t, blockIdx.x);
  const int64_t off = (int64_t)(blockIdx.x - t.block_start[i]) * kChunk;
  const int64_t end = min(off + (int64_t)kChunk, t.n[i]);
  X* x = reinterpret_cast<X*>(t.a[i]);
  const Y* y = reinterpret_cast<const Y*>(t.b[i]);
  for (int64_t e = off + threadIdx.x; e < end; e += kThreads) x[e] = from_f<X>(to_f(x[e]) + alpha * to_f(y[e]));
}

template <typename P>
__global__ void __launch_bounds__(kThreads) adamw_kernel(Table t, float lr, float b1, float b2, float eps, float decay) {
  const int i = find_tensor(t, blockIdx.x);
  const int64_t off = (int64_t)(blockIdx.x - t.block_start[i]) * kChunk;
  const int64_t end = min(off + (int64_t)kChunk, t.n[i]);
  P* p = reinterpret_cast<P*>(t.a[i]);
  const P* g = reinterpret_cast<const P*>(t.b[i]);
  P* m = reinterpret_cast<P*>(t.c[i]);
  P* v = reinterpret_cast<P*>(t.d[i]);
  const float bc1 = t.f0[i], bc2 = t.f1[i];
  for (int64_t e = off + threadIdx.x; e < end; e += kThreads) {
    const float gv = to_f(g[e]);
    float pv = to_f(p[e]) * decay;
    const float mv = b1 * to_f(m[e]) + (1.f - b1) * gv;
    const float vv = b2 * to_f(v[e]) + (1.f - b2) * gv * gv;
    m[e] = from_f<P>(mv);
    v[e] = from_f<P>(vv);
    pv -= lr * (mv / bc1) / (sqrtf(vv / bc2) + eps);
    p[e] = from_f<P>(pv);
  }
}

// Builds tables over [begin, end) of the tensor lists and invokes fn(table, base).
template <typename Fn>
void for_each_chunk(size_t count, const std::vector<at::Tensor>* lists[4], const std::vector<double>* s0,
                    const std::vector<double>* s1, Fn fn) {
  for (size_t begin = 0; begin < count; begin += kMaxTensors) {
    Table t{};
    const size_t end = std::min(count, begin + kMaxTensors);
    int blocks = 0;
    for (size_t j = begin; j < end; ++j) {
      const int k = (int)(j - begin);
      void** slots[4] = {t.a, t.b, t.c, t.d};
      for (int l = 0; l < 4; ++l)
        slots[l][k] = lists[l] ? (*lists[l])[j].data_ptr() : nullptr;
      t.n[k] = lists[0] ? (*lists[0])[j].numel() : (*lists[1])[j].numel();
      t.block_start[k] = blocks;
      t.f0[k] = s0 ? (float)(*s0)[j] : 0.f;
      t.f1[k] = s1 ? (float)(*s1)[j] : 0.f;
      blocks += (int)((t.n[k] + kChunk - 1) / kChunk);
    }
    t.count = (int)(end - begin);
    t.block_start[t.count] = blocks;
    if (blocks > 0) fn(t, blocks, (int)begin);
  }
}

void check_same(const std::vector<at::Tensor>& xs, const char* what) {
  for (const auto& x : xs) LRB_CHECK(x.is_cuda() && x.is_contiguous(), what, ": tensors must be contiguous CUDA");
}

}  // namespace

// Returns per-tensor ||g||_F (fp32, on device).
at::Tensor muon_prologue(std::vector<at::Tensor> params, std::vector<at::Tensor> grads, std::vector<at::Tensor> bufs,
                         std::vector<at::Tensor> outs, double lr, double mu, double wd) {
  check_same(params, "muon_prologue");
  check_same(grads, "muon_prologue");
  check_same(bufs, "muon_prologue");
  const size_t n = params.size();
  c10::cuda::CUDAGuard g(params[0].device());
  auto gsq = at::zeros({(int64_t)n}, params[0].options().dtype(at::kFloat));
  const std::vector<at::Tensor>* lists[4] = {&params, &grads, &bufs, &outs};
  const float decay = (float)(1.0 - lr * wd);
  const auto pt = params[0].scalar_type(), ut = outs[0].scalar_type();
  for (size_t j = 0; j < n; ++j) {
    LRB_CHECK(params[j].scalar_type() == pt && grads[j].scalar_type() == pt && bufs[j].scalar_type() == pt,
              "muon_prologue: param/grad/buffer dtypes must match");
  }
  for_each_chunk(n, lists, nullptr, nullptr, [&](const Table& t, int blocks, int base) {
    if (pt == at::kFloat && ut == at::kBFloat16)
      muon_prologue_kernel<float, __nv_bfloat16><<<blocks, kThreads, 0, stream()>>>(t, decay, (float)mu, gsq.data_ptr<float>(), base);
    else if (pt == at::kFloat && ut == at::kFloat)
      muon_prologue_kernel<float, float><<<blocks, kThreads, 0, stream()>>>(t, decay, (float)mu, gsq.data_ptr<float>(), base);
    else if (pt == at::kBFloat16 && ut == at::kBFloat16)
      muon_prologue_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, kThreads, 0, stream()>>>(t, decay, (float)mu, gsq.data_ptr<float>(), base);
    else
      LRB_CHECK(false, "muon_prologue: unsupported dtypes");
    LRB_LAUNCH_CHECK();
  });
  return gsq.sqrt_();
}

void muon_epilogue(std::vector<at::Tensor> params, std::vector<at::Tensor> orth, at::Tensor gnorm, double lr) {
  check_same(params, "muon_epilogue");
  check_same(orth, "muon_epilogue");
  const size_t n = params.size();
  c10::cuda::CUDAGuard g(params[0].device());
  auto osq = at::zeros({(int64_t)n}, params[0].options().dtype(at::kFloat));
  auto gn = gnorm.to(at::kFloat).contiguous();
  const std::vector<at::Tensor>* lists[4] = {&params, &orth, nullptr, nullptr};
  const auto pt = params[0].scalar_type(), ot = orth[0].scalar_type();
  for_each_chunk(n, lists, nullptr, nullptr, [&](const Table& t, int blocks, int base) {
    LRB_DISPATCH_FLOAT(ot, O, [&] { sumsq_kernel<O><<<blocks, kThreads, 0, stream()>>>(t, osq.data_ptr<float>(), base); });
    LRB_LAUNCH_CHECK();
  });
  for_each_chunk(n, lists, nullptr, nullptr, [&](const Table& t, int blocks, int base) {
    if (pt == at::kFloat && ot == at::kBFloat16)
      muon_update_kernel<float, __nv_bfloat16><<<blocks, kThreads, 0, stream()>>>(t, gn.data_ptr<float>(), osq.data_ptr<float>(), (float)lr, base);
    else if (pt == at::kFloat && ot == at::kFloat)
      muon_update_kernel<float, float><<<blocks, kThreads, 0, stream()>>>(t, gn.data_ptr<float>(), osq.data_ptr<float>(), (float)lr, base);
    else if (pt == at::kBFloat16 && ot == at::kBFloat16)
      muon_update_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, kThreads, 0, stream()>>>(t, gn.data_ptr<float>(), osq.data_ptr<float>(), (float)lr, base);
    else
      LRB_CHECK(false, "muon_epilogue: unsupported dtypes");
    LRB_LAUNCH_CHECK();
  });
}

void axpy_list(std::vector<at::Tensor> xs, std::vector<at::Tensor> ys, double alpha) {
  check_same(xs, "axpy_list");
  check_same(ys, "axpy_list");
  if (xs.empty()) return;
  c10::cuda::CUDAGuard g(xs[0].device());
  const std::vector<at::Tensor>* lists[4] = {&xs, &ys, nullptr, nullptr};
  const auto xt = xs[0].scalar_type(), yt = ys[0].scalar_type();
  for_each_chunk(xs.size(), lists, nullptr, nullptr, [&](const Table& t, int blocks, int) {
    if (xt == at::kFloat && yt == at::kBFloat16)
      axpy_kernel<float, __nv_bfloat16><<<blocks, kThreads, 0, stream()>>>(t, (float)alpha);
    else if (xt == at::kFloat && yt == at::kFloat)
      axpy_kernel<float, float><<<blocks, kThreads, 0, stream()>>>(t, (float)alpha);
    else if (xt == at::kBFloat16 && yt == at::kBFloat16)
      axpy_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, kThreads, 0, stream()>>>(t, (float)alpha);
    else
      LRB_CHECK(false, "axpy_list: unsupported dtypes");
    LRB_LAUNCH_CHECK();
  });
}

void adamw_step(std::vector<at::Tensor> params, std::vector<at::Tensor> grads, std::vector<at::Tensor> m,
                std::vector<at::Tensor> v, std::vector<double> bc1, std::vector<double> bc2, double lr, double b1,
                double b2, double eps, double wd) {
  check_same(params, "adamw_step");
  check_same(grads, "adamw_step");
  const size_t n = params.size();
  c10::cuda::CUDAGuard g(params[0].device());
  const std::vector<at::Tensor>* lists[4] = {&params, &grads, &m, &v};
  const auto pt = params[0].scalar_type();
  for (size_t j = 0; j < n; ++j)
    LRB_CHECK(params[j].scalar_type() == pt && grads[j].scalar_type() == pt && m[j].scalar_type() == pt &&
                  v[j].scalar_type() == pt, "adamw_step: dtypes must match");
  for_each_chunk(n, lists, &bc1, &bc2, [&](const Table& t, int blocks, int) {
    LRB_DISPATCH_FLOAT(pt, P, [&] {
      adamw_kernel<P><<<blocks, kThreads, 0, stream()>>>(t, (float)lr, (float)b1, (float)b2, (float)eps,
                                                         (float)(1.0 - lr * wd));
    });
    LRB_LAUNCH_CHECK();
  });
}

}  // namespace lrb
