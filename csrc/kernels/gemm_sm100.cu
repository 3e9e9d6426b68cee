// Persistent, warp-specialised tcgen05 GEMM:  C[M, N] (+)= A[M, K] * B[N, K]^T
// (both operands K-major, i.e. the nn.Linear layout), bf16/fp16 inputs,
// fp32 accumulation in TMEM.
//
// CTA = 6 warps, one CTA per SM, tiles of 128 x 256 x 64:
//   warp 0      TMA producer: A and B tiles into a 4-stage smem ring (128-byte
//               swizzle), completion tracked by `full` mbarriers;
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32 accumulators)
//               and issues tcgen05.mma from one thread; tcgen05.commit frees
//               smem stages (`empty`) and publishes finished accumulators;
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, convert,
//               store (or accumulate into an fp32 C); then release the
//               accumulator so the next tile's MMAs overlap this epilogue.
// Every wait is bounded (see sm100.cuh); on timeout the kernel records an
// error code, drains its outstanding MMAs, frees TMEM and returns.
#include "../common.cuh"
#include "sm100.cuh"

namespace lrb {

__device__ int g_gemm_tn_err[4];
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, GROUP_M = 8;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr size_t kStageA = (size_t)BM * BK * 2, kStageB = (size_t)BN * BK * 2;
constexpr size_t kSmem = 1024 /*align slack*/ + STAGES * (kStageA + kStageB) + 256;

enum Epi : int { kStore = 0, kAccumF32 = 1 };

struct GemmArgs {
  void* C;
  int64_t ldc;
  int M, N, K;
  int* err;
  float alpha;
  int vec_ok;  // C base and row pitch are 16-byte aligned: vector stores allowed
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int per_group = GROUP_M * tiles_n;
  const int g = tile / per_group;
  const int first = g * GROUP_M;
  const int gsize = min(tiles_m - first, GROUP_M);
  const int r = tile % per_group;
  tm = first + r % gsize;
  tn = r / gsize;
}

template <typename OutT, int EPI>
__device__ __forceinline__ void store_chunk(const GemmArgs& a, int row, int col0, const uint32_t* r) {
  if (row >= a.M) return;
  if constexpr (EPI == kAccumF32) {
    float* c = reinterpret_cast<float*>(a.C) + (int64_t)row * a.ldc + col0;
    if (a.vec_ok && col0 + 32 <= a.N) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 v = *reinterpret_cast<float4*>(c + j);
        v.x += a.alpha * __uint_as_float(r[j]);
        v.y += a.alpha * __uint_as_float(r[j + 1]);
        v.z += a.alpha * __uint_as_float(r[j + 2]);
        v.w += a.alpha * __uint_as_float(r[j + 3]);
        *reinterpret_cast<float4*>(c + j) = v;
      }
    } else {
      for (int j = 0; j < 32 && col0 + j < a.N; ++j) c[j] += a.alpha * __uint_as_float(r[j]);
    }
  } else {
    OutT* c = reinterpret_cast<OutT*>(a.C) + (int64_t)row * a.ldc + col0;
    constexpr int V = 16 / sizeof(OutT);
    if (a.vec_ok && col0 + 32 <= a.N) {
#pragma unroll
      for (int j = 0; j < 32; j += V) {
        Vec16<OutT> v;
#pragma unroll
        for (int t = 0; t < V; ++t) v.v[t] = from_f<OutT>(a.alpha * __uint_as_float(r[j + t]));
        st16(c + j, v);
      }
    } else {
      for (int j = 0; j < 32 && col0 + j < a.N; ++j) c[j] = from_f<OutT>(a.alpha * __uint_as_float(r[j]));
    }
  }
}

template <typename OutT, int EPI, bool BF16IN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = base;
  unsigned char* sB = base + STAGES * kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * kStageB);
  uint64_t* empty = full + STAGES;
  uint64_t* accfull = empty + STAGES;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (args.M + BM - 1) / BM, tiles_n = (args.N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int nk = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t armed = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, tiles_m, tiles_n, tm, tn);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrTmaWait)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], (uint32_t)(kStageA + kStageB));
          tma_load_2d(sA + stage * kStageA, &tmA, &full[stage], kb * BK, tm * BM);
          tma_load_2d(sB + stage * kStageB, &tmB, &full[stage], kb * BK, tn * BN);
          ++armed;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Before the CTA can exit, every issued load must have landed (the MMA
      // warp may have stopped consuming after an error).
      for (int i = 1; i <= STAGES && i <= armed; ++i) {
        const int64_t pos = armed - i;
        mbar_wait(&full[pos % STAGES], (uint32_t)((pos / STAGES) & 1), nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BM, BN, BF16IN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&accempty[acc], acc_phase ^ 1, args.err, kErrAccWait)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sA + stage * kStageA), b0 = smem_addr(sB + stage * kStageB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d, umma_desc_k_sw128(a0 + k * 32), umma_desc_k_sw128(b0 + k * 32), idesc, (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit(&accfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);  // all issued MMAs retired before TMEM is freed
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int tm, tn;
      tile_coords(tile, tiles_m, tiles_n, tm, tn);
      if (!mbar_wait(&accfull[acc], acc_phase, args.err, kErrEpiWait)) break;
      tc_fence_after();
      const int row = tm * BM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
        tmem_ld_wait();
        store_chunk<OutT, EPI>(args, row, tn * BN + c * 32, r);
      }
      tc_fence_before();
      mbar_arrive(&accempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
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

// Row-major (rows x cols) matrix with leading dimension ld (elements), box = box_rows x 64.
CUtensorMap make_map_k_major(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, bool bf16) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                           const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return m;
}

// Error words of this file's kernels: module globals (one copy per device).
DeviceWord g_gemm_tn_err_word{g_gemm_tn_err, {}};

int* error_word(const at::Device& dev) { return g_gemm_tn_err_word.get(dev.index()); }

template <typename OutT, int EPI, bool BF16IN>
void launch(const at::Tensor& A, const at::Tensor& B, void* C, int64_t ldc, float alpha) {
  const int M = (int)A.size(0), K = (int)A.size(1), N = (int)B.size(0);
  CUtensorMap ta = make_map_k_major(A.data_ptr(), M, K, A.stride(0), BM, BF16IN);
  CUtensorMap tb = make_map_k_major(B.data_ptr(), N, K, B.stride(0), BN, BF16IN);
  const int vec_ok = (reinterpret_cast<uintptr_t>(C) % 16 == 0) && ((ldc * (int64_t)sizeof(OutT)) % 16 == 0);
  GemmArgs args{C, ldc, M, N, K, error_word(A.device()), alpha, vec_ok};
  auto k = gemm_tn_kernel<OutT, EPI, BF16IN>;
  LRB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, num_sms()));
  k<<<grid, kThreads, kSmem, stream()>>>(ta, tb, args);
  LRB_LAUNCH_CHECK();
}

void check_operand(const at::Tensor& t, const char* name) {
  LRB_CHECK(t.is_cuda() && t.dim() == 2 && t.stride(1) == 1, "gemm: ", name, " must be a 2-D CUDA tensor with unit column stride");
  LRB_CHECK(t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kHalf, "gemm: ", name, " must be bf16/fp16");
  LRB_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0 && (t.stride(0) * 2) % 16 == 0,
            "gemm: ", name, " needs 16-byte aligned base and row stride");
}

}  // namespace

// C = alpha * A @ B^T  (A: M x K, B: N x K).  out_dtype: bf16/fp16/fp32.
at::Tensor gemm_tn(const at::Tensor& A, const at::Tensor& B, at::ScalarType out_dtype, double alpha) {
  check_operand(A, "A");
  check_operand(B, "B");
  LRB_CHECK(A.size(1) == B.size(1) && A.scalar_type() == B.scalar_type(), "gemm: K/dtype mismatch");
  c10::cuda::CUDAGuard g(A.device());
  bind_device(A.get_device());
  auto C = at::empty({A.size(0), B.size(0)}, A.options().dtype(out_dtype));
  if (C.numel() == 0) return C;
  if (A.size(1) == 0) return C.zero_();
  const bool bf = A.scalar_type() == at::kBFloat16;
  if (out_dtype == at::kFloat) {
    if (bf) launch<float, kStore, true>(A, B, C.data_ptr(), C.stride(0), (float)alpha);
    else launch<float, kStore, false>(A, B, C.data_ptr(), C.stride(0), (float)alpha);
  } else if (out_dtype == at::kBFloat16) {
    if (bf) launch<__nv_bfloat16, kStore, true>(A, B, C.data_ptr(), C.stride(0), (float)alpha);
    else launch<__nv_bfloat16, kStore, false>(A, B, C.data_ptr(), C.stride(0), (float)alpha);
  } else if (out_dtype == at::kHalf) {
    if (bf) launch<__half, kStore, true>(A, B, C.data_ptr(), C.stride(0), (float)alpha);
    else launch<__half, kStore, false>(A, B, C.data_ptr(), C.stride(0), (float)alpha);
  } else {
    LRB_CHECK(false, "gemm: unsupported output dtype");
  }
  return C;
}

// C (fp32, M x N, row stride C.stride(0)) += alpha * A @ B^T
void gemm_tn_accumulate(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, double alpha) {
  check_operand(A, "A");
  check_operand(B, "B");
  LRB_CHECK(C.scalar_type() == at::kFloat && C.dim() == 2 && C.stride(1) == 1 && C.size(0) == A.size(0) &&
                C.size(1) == B.size(0), "gemm_accumulate: C must be fp32 (M, N)");
  LRB_CHECK((reinterpret_cast<uintptr_t>(C.data_ptr()) % 16) == 0 && C.stride(0) % 4 == 0, "gemm_accumulate: C alignment");
  c10::cuda::CUDAGuard g(A.device());
  bind_device(A.get_device());
  if (C.numel() == 0 || A.size(1) == 0) return;
  if (A.scalar_type() == at::kBFloat16) launch<float, kAccumF32, true>(A, B, C.data_ptr(), C.stride(0), (float)alpha);
  else launch<float, kAccumF32, false>(A, B, C.data_ptr(), C.stride(0), (float)alpha);
}

// Returns and clears the device error word of the tcgen05 kernels (0 = no error).
int64_t sm100_error(int64_t device) { return g_gemm_tn_err_word.take((int)device); }

}  // namespace lrb
