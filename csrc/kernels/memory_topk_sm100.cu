// PHMA memory read, selection stage: for every query row, the k = 32 bank
// slots with the largest similarity q . key (queries and keys already
// L2-normalised, so this is the cosine of the semantic-memory read), found
// without materialising the (queries x slots) similarity matrix.
//
// CTA = 128 queries x one slice of the bank, 6 warps:
//   warp 0      producer: per 64-element chunk of the feature dimension, TMA
//               loads of the query tile (128 x 64) and the key tile (256 x 64),
//               128-byte swizzle, 4-stage ring;
//   warp 1      TMEM owner + MMA issue: S = Q K^T for 256 keys at a time
//               (tcgen05 kind::f16, M = 128, N = 256, fp32 in TMEM), two S
//               buffers so the next key tile's MMAs run while the epilogue
//               scans the previous one;
//   warps 2..5  one query row per thread: tcgen05.ld of the row's 256 scores,
//               streaming top-32 kept in registers (a candidate enters only if
//               it beats the current minimum, which then gets recomputed).
// Each CTA writes its slice's 32 candidates per row; the slices are merged on
// the host side (top-32 of slices x 32).  All waits are bounded.
#include "../common.cuh"
#include "sm100.cuh"

namespace lrb {

__device__ int g_mem_topk_err[4];
namespace {

using namespace sm100;

constexpr int TQ = 128, TN = 256, CK = 64, STAGES = 4, TOPK = 32;
constexpr int kThreads = 192;
constexpr uint32_t kQBytes = TQ * CK * 2, kKBytes = TN * CK * 2, kStage = kQBytes + kKBytes;  // 16 + 32 KB
constexpr size_t kSmem = 1024 + STAGES * (size_t)kStage + 256;

struct TopkArgs {
  int T, N, D;
  int n_per_split;
  float* out_s;  // (splits, T, 32)
  int* out_i;
  int* err;
};

__device__ __forceinline__ void topk_insert(float (&bv)[TOPK], int (&bi)[TOPK], float& thr, float v, int id) {
  bool done = false;
#pragma unroll
  for (int j = 0; j < TOPK; ++j) {
    const bool hit = !done && bv[j] == thr;
    bv[j] = hit ? v : bv[j];
    bi[j] = hit ? id : bi[j];
    done |= hit;
  }
  float m = bv[0];
#pragma unroll
  for (int j = 1; j < TOPK; ++j) m = fminf(m, bv[j]);
  thr = m;
}

__global__ void __launch_bounds__(kThreads, 1)
    mem_topk_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK, TopkArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + STAGES * kStage);
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* s_full = bars + 2 * STAGES;  // [2]
  uint64_t* s_free = s_full + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_free + 2);
  auto sQ = [&](int s) { return base + s * kStage; };
  auto sK = [&](int s) { return base + s * kStage + kQBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * TQ;
  const int n_begin = blockIdx.y * a.n_per_split;
  const int n_end = min(a.N, n_begin + a.n_per_split);
  const int ntiles = n_end > n_begin ? (n_end - n_begin + TN - 1) / TN : 0;
  const int nck = a.D / CK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tS = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int armed = 0;
      bool ok = true;
      for (int t = 0; t < ntiles && ok; ++t) {
        for (int c = 0; c < nck; ++c) {
          const int it = t * nck + c;
          const int st = it % STAGES;
          if (!mbar_wait(&empty[st], ((it / STAGES) & 1) ^ 1, a.err, kErrTmaWait)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[st], kStage);
          tma_load_2d(sQ(st), &tmQ, &full[st], c * CK, q0);
          tma_load_2d(sK(st), &tmK, &full[st], c * CK, n_begin + t * TN);
          ++armed;
        }
      }
      // drain: every armed stage has landed before the CTA may exit
      for (int i = 1; i <= STAGES && i <= armed; ++i) {
        const int it = armed - i;
        mbar_wait(&full[it % STAGES], (it / STAGES) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(TQ, TN, true);
      bool ok = true;
      for (int t = 0; t < ntiles && ok; ++t) {
        const int b = t & 1;
        if (t >= 2 && !mbar_wait(&s_free[b], ((t >> 1) - 1) & 1, a.err, kErrAccWait)) break;
        tc_fence_after();
        for (int c = 0; c < nck; ++c) {
          const int it = t * nck + c;
          const int st = it % STAGES;
          if (!mbar_wait(&full[st], (it / STAGES) & 1, a.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t pq = smem_addr(sQ(st)), pk = smem_addr(sK(st));
#pragma unroll
          for (int kk = 0; kk < CK / 16; ++kk)
            umma_f16(tS + b * TN, umma_desc_k_sw128(pq + kk * 32), umma_desc_k_sw128(pk + kk * 32), idesc,
                     (c | kk) != 0);
          umma_commit(&empty[st]);
        }
        umma_commit(&s_full[b]);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row = q0 + quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float bv[TOPK];
    int bi[TOPK];
#pragma unroll
    for (int j = 0; j < TOPK; ++j) {
      bv[j] = -INFINITY;
      bi[j] = -1;
    }
    float thr = -INFINITY;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int b = t & 1;
      ok = __all_sync(0xffffffffu, ok && mbar_wait(&s_full[b], (t >> 1) & 1, a.err, kErrEpiWait));
      if (!ok) break;
      tc_fence_after();
      const int col_base = n_begin + t * TN;
#pragma unroll 1
      for (int cc = 0; cc < TN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tS + b * TN + lane_base + cc * 32, r);
        tmem_ld_wait();
        const int c0 = col_base + cc * 32;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float v = __uint_as_float(r[e]);
          if (v > thr && c0 + e < n_end) topk_insert(bv, bi, thr, v, c0 + e);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
    }
    if (row < a.T) {
      const int64_t o = ((int64_t)blockIdx.y * a.T + row) * TOPK;
#pragma unroll
      for (int j = 0; j < TOPK; ++j) {
        a.out_s[o + j] = bv[j];
        a.out_i[o + j] = bi[j];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tS, 512);
  }
}

// ------------------------------------------------------------ gather / backward
// out[t] = sum_j w_j V[idx_j], w = softmax(s); one warp per query row.
template <typename V>
__global__ void topk_gather_fwd_kernel(const float* __restrict__ s, const int* __restrict__ idx,
                                       const V* __restrict__ values, V* __restrict__ out, float* __restrict__ w_out,
                                       int T, int Dv, int N) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= T) return;
  const float sv = s[(int64_t)row * TOPK + lane];
  int iv = idx[(int64_t)row * TOPK + lane];
  if (iv >= N) iv = -1;  // an index past the bank is treated like an empty candidate
  const bool valid = iv >= 0;
  float m = warp_max(valid ? sv : -INFINITY);
  const float e = valid ? __expf(sv - m) : 0.f;
  const float z = warp_sum(e);
  const float w = z > 0.f ? e / z : 0.f;
  w_out[(int64_t)row * TOPK + lane] = w;
  for (int d0 = lane * 8; d0 < Dv; d0 += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < TOPK; ++j) {
      const float wj = __shfl_sync(0xffffffffu, w, j);
      const int ij = __shfl_sync(0xffffffffu, iv, j);
      if (ij < 0) continue;
      const V* vp = values + (int64_t)ij * Dv + d0;
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wj * to_f(vp[q]);
    }
    V* op = out + (int64_t)row * Dv + d0;
#pragma unroll
    for (int q = 0; q < 8; ++q) op[q] = from_f<V>(acc[q]);
  }
}

// ds_j = w_j (g . V_j - sum_i w_i g . V_i);  dq = sum_j ds_j K_j.  One warp per row.
template <typename V>
__global__ void topk_gather_bwd_kernel(const V* __restrict__ g, const float* __restrict__ w, const int* __restrict__ idx,
                                       const V* __restrict__ values, const V* __restrict__ keys,
                                       float* __restrict__ dq, int T, int Dv, int Dk, int N) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= T) return;
  const float wv = w[(int64_t)row * TOPK + lane];
  int iv = idx[(int64_t)row * TOPK + lane];
  if (iv >= N) iv = -1;
  float dw_mine = 0.f;
  for (int j = 0; j < TOPK; ++j) {
    const int ij = __shfl_sync(0xffffffffu, iv, j);
    float part = 0.f;
    if (ij >= 0) {
      const V* vp = values + (int64_t)ij * Dv;
      const V* gp = g + (int64_t)row * Dv;
      for (int d = lane; d < Dv; d += 32) part += to_f(gp[d]) * to_f(vp[d]);
    }
    part = warp_sum(part);
    if (lane == j) dw_mine = part;
  }
  const float dot = warp_sum(wv * dw_mine);
  const float ds = iv >= 0 ? wv * (dw_mine - dot) : 0.f;
  for (int d = lane; d < Dk; d += 32) {
    float acc = 0.f;
    for (int j = 0; j < TOPK; ++j) {
      const float dsj = __shfl_sync(0xffffffffu, ds, j);
      const int ij = __shfl_sync(0xffffffffu, iv, j);
      if (ij >= 0) acc += dsj * to_f(keys[(int64_t)ij * Dk + d]);
    }
    dq[(int64_t)row * Dk + d] = acc;
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    LRB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    LRB_CHECK(p != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

CUtensorMap bf16_map(const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)CK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (memory top-k) failed with code ", (int)r);
  return m;
}

// Error words of this file's kernels: module globals (one copy per device).
DeviceWord g_mem_topk_err_word{g_mem_topk_err, {}};

int* topk_error_word(const at::Device& dev) { return g_mem_topk_err_word.get(dev.index()); }

}  // namespace

// q (T, D) and keys (N, D) bf16, contiguous, D % 64 == 0, rows 16-byte aligned.
// Returns candidate scores (splits, T, 32) fp32 and slot indices (splits, T, 32)
// int32 (-1 / -inf where a slice has fewer than 32 slots).
std::tuple<at::Tensor, at::Tensor> memory_topk_candidates(const at::Tensor& q, const at::Tensor& keys, int64_t splits) {
  LRB_CHECK(q.is_cuda() && keys.is_cuda() && q.scalar_type() == at::kBFloat16 && keys.scalar_type() == at::kBFloat16,
            "memory_topk: bf16 CUDA tensors");
  LRB_CHECK(q.dim() == 2 && keys.dim() == 2 && q.is_contiguous() && keys.is_contiguous() && q.size(1) == keys.size(1),
            "memory_topk: q (T, D), keys (N, D) contiguous");
  const int64_t T = q.size(0), N = keys.size(0), D = q.size(1);
  LRB_CHECK(D % CK == 0 && D >= CK, "memory_topk: D must be a multiple of 64");
  LRB_CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(keys.data_ptr()) % 16 == 0,
            "memory_topk: 16-byte aligned operands");
  c10::cuda::CUDAGuard g(q.device());
  bind_device(q.get_device());
  const int64_t qt = (T + TQ - 1) / TQ;
  if (splits <= 0) splits = std::max<int64_t>(1, num_sms() / std::max<int64_t>(qt, 1));
  int64_t per = (N + splits - 1) / splits;
  per = ((per + TN - 1) / TN) * TN;
  splits = (N + per - 1) / per;
  auto out_s = at::empty({splits, T, TOPK}, q.options().dtype(at::kFloat));
  auto out_i = at::empty({splits, T, TOPK}, q.options().dtype(at::kInt));
  if (T == 0 || N == 0) {
    out_s.fill_(-INFINITY);
    out_i.fill_(-1);
    return {out_s, out_i};
  }
  CUtensorMap tq = bf16_map(q.data_ptr(), T, D, TQ), tk = bf16_map(keys.data_ptr(), N, D, TN);
  TopkArgs args{(int)T, (int)N, (int)D, (int)per, out_s.data_ptr<float>(), out_i.data_ptr<int>(),
                topk_error_word(q.device())};
  LRB_CUDA_CHECK(cudaFuncSetAttribute(mem_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
  mem_topk_kernel<<<dim3((unsigned)qt, (unsigned)splits), kThreads, kSmem, stream()>>>(tq, tk, args);
  LRB_LAUNCH_CHECK();
  return {out_s, out_i};
}

int64_t memory_topk_error(int64_t device) { return g_mem_topk_err_word.take((int)device); }

// scores / idx (T, 32) -> (out (T, Dv) in values' dtype, softmax weights (T, 32) fp32)
std::tuple<at::Tensor, at::Tensor> topk_gather_fwd(const at::Tensor& s, const at::Tensor& idx, const at::Tensor& values) {
  LRB_CHECK(s.is_cuda() && s.dim() == 2 && s.size(1) == TOPK && s.scalar_type() == at::kFloat && s.is_contiguous(),
            "topk_gather_fwd: scores (T, 32) fp32");
  LRB_CHECK(idx.scalar_type() == at::kInt && idx.is_contiguous() && values.is_contiguous() && values.size(1) % 256 == 0,
            "topk_gather_fwd: idx int32, values (N, Dv) with Dv % 256 == 0");
  c10::cuda::CUDAGuard g(s.device());
  bind_device(s.get_device());
  const int T = (int)s.size(0), Dv = (int)values.size(1);
  auto out = at::empty({T, Dv}, values.options());
  auto w = at::empty({T, TOPK}, s.options());
  if (T == 0) return {out, w};
  LRB_DISPATCH_FLOAT(values.scalar_type(), V, [&] {
    topk_gather_fwd_kernel<V><<<(T + 7) / 8, 256, 0, stream()>>>(
        s.data_ptr<float>(), idx.data_ptr<int>(), reinterpret_cast<const V*>(values.data_ptr()),
        reinterpret_cast<V*>(out.data_ptr()), w.data_ptr<float>(), T, Dv, (int)values.size(0));
  });
  LRB_LAUNCH_CHECK();
  return {out, w};
}

// dq (T, Dk) fp32 from the output gradient g (T, Dv).
at::Tensor topk_gather_bwd(const at::Tensor& g, const at::Tensor& w, const at::Tensor& idx, const at::Tensor& values,
                           const at::Tensor& keys) {
  LRB_CHECK(g.is_cuda() && g.is_contiguous() && g.scalar_type() == values.scalar_type() &&
                keys.scalar_type() == values.scalar_type() && keys.is_contiguous() && values.is_contiguous(),
            "topk_gather_bwd: contiguous operands of one dtype");
  c10::cuda::CUDAGuard gd(g.device());
  const int T = (int)g.size(0), Dv = (int)values.size(1), Dk = (int)keys.size(1);
  auto dq = at::empty({T, Dk}, g.options().dtype(at::kFloat));
  if (T == 0) return dq;
  LRB_DISPATCH_FLOAT(values.scalar_type(), V, [&] {
    topk_gather_bwd_kernel<V><<<(T + 7) / 8, 256, 0, stream()>>>(
        reinterpret_cast<const V*>(g.data_ptr()), w.data_ptr<float>(), idx.data_ptr<int>(),
        reinterpret_cast<const V*>(values.data_ptr()), reinterpret_cast<const V*>(keys.data_ptr()),
        dq.data_ptr<float>(), T, Dv, Dk, (int)std::min(values.size(0), keys.size(0)));
  });
  LRB_LAUNCH_CHECK();
  return dq;
}

}  // namespace lrb
