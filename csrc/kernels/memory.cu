// Top-k memory read: for every query row of a similarity matrix, select the
// k largest entries (ties -> lower index), softmax over them and gather the
// weighted sum of the matching value rows -- one warp per query, no
// intermediate (Q, k) tensors.  Each lane keeps a sorted register list of its
// k best candidates (early reject against its current k-th), then the warp
// merges the 32 lists with k arg-max rounds.
#include "../common.cuh"

namespace lrb {
namespace {

template <int K>
__device__ __forceinline__ bool better(float v, int i, float w, int j) { return v > w || (v == w && i < j); }

template <int K, typename V>
__global__ void topk_read_kernel(const float* __restrict__ sim, const V* __restrict__ values, float* __restrict__ out,
                                 int64_t* __restrict__ sel_idx, float* __restrict__ sel_w, int64_t Q, int N, int dv,
                                 int k) {
  const int lane = threadIdx.x & 31;
  const int64_t q = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (q >= Q) return;
  const float* row = sim + q * N;
  float lv[K];
  int li[K];
#pragma unroll
  for (int t = 0; t < K; ++t) { lv[t] = -INFINITY; li[t] = 0x7fffffff; }
  for (int n = lane; n < N; n += 32) {
    const float v = row[n];
    if (!better<K>(v, n, lv[K - 1], li[K - 1])) continue;
    // insert keeping lv sorted descending
    float cv = v;
    int ci = n;
#pragma unroll
    for (int t = 0; t < K; ++t) {
      if (better<K>(cv, ci, lv[t], li[t])) {
        const float tv = lv[t];
        const int ti = li[t];
        lv[t] = cv; li[t] = ci;
        cv = tv; ci = ti;
      }
    }
  }
  // warp merge: k rounds of arg-max over the lanes' heads
  float sel_v[K];
  int sel_i[K];
  int head = 0;
#pragma unroll
  for (int r = 0; r < K; ++r) {
    float hv = -INFINITY;
    int hi = 0x7fffffff;
#pragma unroll
    for (int t = 0; t < K; ++t)
      if (t == head) { hv = lv[t]; hi = li[t]; }
    float bv = hv;
    int bi = hi, bl = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
      if (better<K>(ov, oi, bv, bi)) { bv = ov; bi = oi; bl = ol; }
    }
    sel_v[r] = bv;
    sel_i[r] = bi;
    if (lane == bl) ++head;
  }
  // softmax over the k selected similarities
  float mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < K; ++r)
    if (r < k) mx = fmaxf(mx, sel_v[r]);
  float w[K], den = 0.f;
#pragma unroll
  for (int r = 0; r < K; ++r) {
    w[r] = (r < k && sel_i[r] < N) ? __expf(sel_v[r] - mx) : 0.f;
    den += w[r];
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  if (lane < k) {
#pragma unroll
    for (int r = 0; r < K; ++r)
      if (r == lane) {
        sel_idx[q * k + r] = sel_i[r] < N ? sel_i[r] : 0;
        sel_w[q * k + r] = w[r] * inv;
      }
  }
  for (int d = lane; d < dv; d += 32) {
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < K; ++r)
      if (w[r] != 0.f) acc += w[r] * to_f(values[(int64_t)sel_i[r] * dv + d]);
    out[q * dv + d] = acc * inv;
  }
}

}  // namespace

// sim (Q, N) fp32, values (N, dv) -> (out (Q, dv) fp32, indices (Q, k), weights (Q, k))
std::tuple<at::Tensor, at::Tensor, at::Tensor> topk_softmax_gather(const at::Tensor& sim, const at::Tensor& values, int64_t k) {
  LRB_CHECK(sim.is_cuda() && sim.scalar_type() == at::kFloat && sim.dim() == 2 && sim.is_contiguous(),
            "topk_softmax_gather: fp32 (Q, N) similarities");
  LRB_CHECK(values.is_cuda() && values.dim() == 2 && values.is_contiguous() && values.size(0) == sim.size(1),
            "topk_softmax_gather: values (N, dv)");
  LRB_CHECK(k >= 1 && k <= 32 && k <= sim.size(1), "topk_softmax_gather: 1 <= k <= min(32, N)");
  c10::cuda::CUDAGuard g(sim.device());
  bind_device(sim.get_device());
  const int64_t Q = sim.size(0);
  const int N = (int)sim.size(1), dv = (int)values.size(1);
  auto out = at::empty({Q, dv}, sim.options());
  auto idx = at::empty({Q, k}, sim.options().dtype(at::kLong));
  auto wts = at::empty({Q, k}, sim.options());
  if (Q == 0) return {out, idx, wts};
  const int warps = 4;
  const dim3 grid((unsigned)((Q + warps - 1) / warps));
  LRB_DISPATCH_FLOAT(values.scalar_type(), V, [&] {
    auto run = [&](auto kc) {
      constexpr int KC = decltype(kc)::value;
      topk_read_kernel<KC, V><<<grid, warps * 32, 0, stream()>>>(sim.data_ptr<float>(),
                                                                 reinterpret_cast<const V*>(values.data_ptr()),
                                                                 out.data_ptr<float>(), idx.data_ptr<int64_t>(),
                                                                 wts.data_ptr<float>(), Q, N, dv, (int)k);
    };
    if (k <= 8) run(std::integral_constant<int, 8>{});
    else if (k <= 16) run(std::integral_constant<int, 16>{});
    else run(std::integral_constant<int, 32>{});
  });
  LRB_LAUNCH_CHECK();
  return {out, idx, wts};
}

}  // namespace lrb
