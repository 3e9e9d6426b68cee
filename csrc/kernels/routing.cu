// Router softmax + top-k, chunk mean pooling and escalated-chunk compaction.
#include "../common.cuh"

namespace lrb {
namespace {

// One warp per token: softmax over E experts (E <= 1024), iterative top-k
// (ties -> lower index, as torch.topk on equal values from a stable max),
// renormalised weights.
template <typename T>
__global__ void softmax_topk_kernel(const T* __restrict__ logits, float* __restrict__ w, int64_t* __restrict__ idx,
                                    float* __restrict__ probs, int64_t N, int E, int K) {
  const int lane = threadIdx.x & 31;
  const int64_t tok = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (tok >= N) return;
  const T* x = logits + tok * E;
  float* p = probs + tok * E;
  float m = -INFINITY;
  for (int e = lane; e < E; e += 32) m = fmaxf(m, to_f(x[e]));
  m = warp_max(m);
  float s = 0.f;
  for (int e = lane; e < E; e += 32) s += __expf(to_f(x[e]) - m);
  s = warp_sum(s);
  const float inv = 1.f / s;
  for (int e = lane; e < E; e += 32) p[e] = __expf(to_f(x[e]) - m) * inv;
  __syncwarp();
  // top-k by repeated arg-max; chosen experts are masked by index.
  float sel_sum = 0.f;
  unsigned long long chosen_lo = 0ull;  // experts < 64 tracked in a bitmask, others via re-scan
  float vals[8];
  int ids[8];
  for (int k = 0; k < K; ++k) {
    float best = -1.f;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      bool used = false;
      if (e < 64) used = (chosen_lo >> e) & 1ull;
      else
        for (int j = 0; j < k; ++j) used |= (ids[j] == e);
      const float v = p[e];
      if (!used && (v > best || (v == best && e < bi))) { best = v; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (b2 > best || (b2 == best && i2 < bi)) { best = b2; bi = i2; }
    }
    if (k < 8) { vals[k] = best; ids[k] = bi; }
    if (bi < 64) chosen_lo |= (1ull << bi);
    sel_sum += best;
  }
  if (lane == 0) {
    const float denom = sel_sum + 1e-9f;
    for (int k = 0; k < K && k < 8; ++k) {
      w[tok * K + k] = vals[k] / denom;
      idx[tok * K + k] = ids[k];
    }
  }
}

// x (B, S, D) -> out (B, S/c, D); fp32 accumulation.
template <typename T>
__global__ void chunk_mean_pool_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t BC, int c, int D) {
  const int64_t n = BC * D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bc = i / D;
    const int d = (int)(i - bc * D);
    const T* p = x + bc * c * (int64_t)D + d;
    float s = 0.f;
    for (int t = 0; t < c; ++t) s += to_f(p[(int64_t)t * D]);
    out[i] = from_f<T>(s / c);
  }
}

// One block per row: prefix sum over the bool mask, scatter chunk ids to the
// front.  ids must be pre-filled with C (padding id).
__global__ void compact_kernel(const bool* __restrict__ mask, int64_t* __restrict__ ids, int64_t* __restrict__ counts,
                               int C) {
  __shared__ int warp_tot[32];
  const int b = blockIdx.x;
  const bool* m = mask + (int64_t)b * C;
  int64_t* out = ids + (int64_t)b * C;
  int base = 0;
  for (int start = 0; start < C; start += blockDim.x) {
    const int c = start + threadIdx.x;
    const int v = (c < C && m[c]) ? 1 : 0;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const unsigned bal = __ballot_sync(0xffffffffu, v);
    const int in_warp = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) warp_tot[wid] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int w2 = 0; w2 < (int)(blockDim.x >> 5); ++w2) {
      if (w2 < wid) before += warp_tot[w2];
      total += warp_tot[w2];
    }
    if (v) out[base + before + in_warp] = c;
    base += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[b] = base;
}

// Capacity slots of the routed assignments, in (token, k) order: assignment a
// (expert e = idx[a]) gets slot = its rank among the assignments to e that come
// before it, or -1 when that rank is >= cap (cap < 0: no limit); also its
// owner rank e / epl and local expert e % epl, and the per-expert totals.  One
// CTA of 32 warps: warp w owns the contiguous range [w A / 32, (w+1) A / 32);
// pass 1 counts per warp and expert (shared-memory atomics), an exclusive scan
// over the warps gives each warp's starting rank per expert, pass 2 walks the
// range again in order, 32 assignments at a time, ranking equal experts inside
// the batch by __match_any_sync.  Deterministic; no host read.
__global__ void __launch_bounds__(1024) route_slots_kernel(const int64_t* __restrict__ idx, int64_t A, int E,
                                                           int epl, int cap, int* __restrict__ dest,
                                                           int* __restrict__ le, int* __restrict__ slot,
                                                           int* __restrict__ counts) {
  extern __shared__ int cnt[];  // [32 warps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int64_t a0 = A * warp / 32, a1 = A * (warp + 1) / 32;
  for (int64_t b = a0; b < a1; b += 32) {
    const int64_t a = b + lane;
    if (a < a1) atomicAdd(&cnt[warp * E + (int)idx[a]], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += c;
    }
    counts[e] = run;
  }
  __syncthreads();
  const unsigned below = (1u << lane) - 1u;
  for (int64_t b = a0; b < a1; b += 32) {
    const int64_t a = b + lane;
    const bool in = a < a1;
    const int e = in ? (int)idx[a] : -1;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    int rank = 0;
    if (in) {
      rank = cnt[warp * E + e] + __popc(same & below);
      slot[a] = (cap < 0 || rank < cap) ? rank : -1;
      dest[a] = e / epl;
      le[a] = e % epl;
    }
    __syncwarp();
    if (in && (same & below) == 0) cnt[warp * E + e] += __popc(same);  // the group's first lane advances
    __syncwarp();
  }
}

}  // namespace

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> route_slots(const at::Tensor& idx, int64_t num_experts,
                                                                       int64_t experts_per_rank, int64_t cap) {
  LRB_CHECK(idx.is_cuda() && idx.scalar_type() == at::kLong && idx.is_contiguous(),
            "route_slots: contiguous int64 CUDA expert indices");
  LRB_CHECK(num_experts >= 1 && num_experts <= 1024 && experts_per_rank >= 1 && num_experts % experts_per_rank == 0,
            "route_slots: 1 <= E <= 1024 experts, E a multiple of the experts per rank");
  const int64_t A = idx.numel();
  LRB_CHECK(A < (1LL << 31), "route_slots: too many assignments");
  c10::cuda::CUDAGuard g(idx.device());
  bind_device(idx.get_device());
  auto i32 = idx.options().dtype(at::kInt);
  auto dest = at::empty({A}, i32), le = at::empty({A}, i32), slot = at::empty({A}, i32);
  auto counts = at::zeros({num_experts}, i32);
  if (A == 0) return {dest, le, slot, counts};
  const int smem = 32 * (int)num_experts * (int)sizeof(int);
  if (smem > 48 * 1024)
    LRB_CUDA_CHECK(cudaFuncSetAttribute(route_slots_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  route_slots_kernel<<<1, 1024, smem, stream()>>>(idx.data_ptr<int64_t>(), A, (int)num_experts, (int)experts_per_rank,
                                                  (int)cap, dest.data_ptr<int>(), le.data_ptr<int>(),
                                                  slot.data_ptr<int>(), counts.data_ptr<int>());
  LRB_LAUNCH_CHECK();
  return {dest, le, slot, counts};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> softmax_topk_fwd(const at::Tensor& logits, int64_t k) {
  LRB_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.is_contiguous(), "softmax_topk: 2-D contiguous logits");
  const int64_t N = logits.size(0);
  const int E = (int)logits.size(1);
  LRB_CHECK(k >= 1 && k <= 8 && k <= E, "softmax_topk supports 1 <= k <= min(8, E)");
  c10::cuda::CUDAGuard g(logits.device());
  bind_device(logits.get_device());
  auto f32 = logits.options().dtype(at::kFloat);
  auto w = at::empty({N, k}, f32);
  auto idx = at::empty({N, k}, logits.options().dtype(at::kLong));
  auto probs = at::empty({N, E}, f32);
  if (N == 0) return {w, idx, probs};
  const int warps = 8;
  LRB_DISPATCH_FLOAT(logits.scalar_type(), T, [&] {
    softmax_topk_kernel<T><<<(unsigned)((N + warps - 1) / warps), warps * 32, 0, stream()>>>(
        reinterpret_cast<const T*>(logits.data_ptr()), w.data_ptr<float>(), idx.data_ptr<int64_t>(),
        probs.data_ptr<float>(), N, E, (int)k);
  });
  LRB_LAUNCH_CHECK();
  return {w, idx, probs};
}

at::Tensor chunk_mean_pool_fwd(const at::Tensor& x, int64_t c) {
  LRB_CHECK(x.is_cuda() && x.dim() == 3 && x.is_contiguous() && x.size(1) % c == 0, "chunk_mean_pool: bad input");
  c10::cuda::CUDAGuard g(x.device());
  bind_device(x.get_device());
  const int64_t B = x.size(0), S = x.size(1), D = x.size(2);
  auto out = at::empty({B, S / c, D}, x.options());
  const int64_t n = B * (S / c) * D;
  if (n == 0) return out;
  LRB_DISPATCH_FLOAT(x.scalar_type(), T, [&] {
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16);
    chunk_mean_pool_kernel<T><<<blocks, 256, 0, stream()>>>(reinterpret_cast<const T*>(x.data_ptr()),
                                                            reinterpret_cast<T*>(out.data_ptr()), B * (S / c), (int)c,
                                                            (int)D);
  });
  LRB_LAUNCH_CHECK();
  return out;
}

// mask (B, C) bool -> (ids (B, C) with selected chunk ids packed first, padded with C; counts (B))
std::tuple<at::Tensor, at::Tensor> compact_chunks(const at::Tensor& mask) {
  LRB_CHECK(mask.is_cuda() && mask.scalar_type() == at::kBool && mask.dim() == 2 && mask.is_contiguous(),
            "compact_chunks: bool (B, C) mask");
  c10::cuda::CUDAGuard g(mask.device());
  bind_device(mask.get_device());
  const int64_t B = mask.size(0), C = mask.size(1);
  auto ids = at::full({B, C}, C, mask.options().dtype(at::kLong));
  auto counts = at::zeros({B}, mask.options().dtype(at::kLong));
  if (B == 0 || C == 0) return {ids, counts};
  compact_kernel<<<(unsigned)B, 256, 0, stream()>>>(mask.data_ptr<bool>(), ids.data_ptr<int64_t>(),
                                                    counts.data_ptr<int64_t>(), (int)C);
  LRB_LAUNCH_CHECK();
  return {ids, counts};
}

}  // namespace lrb
