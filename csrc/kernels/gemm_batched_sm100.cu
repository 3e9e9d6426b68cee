// Batched persistent tcgen05 GEMM with an axpby epilogue (bf16 in, bf16 out,
// fp32 accumulation in TMEM):
//
//   C[b] = alpha * A[b] op(B[b]) + beta * D[b]
//
// A (batch, M, K) K-major.  B is either (batch, N, K) K-major (op = transpose,
// the nn.Linear layout) or (batch, K, N) with N contiguous (op = identity; the
// operand is fed to the tensor core MN-major, so X in P X needs no transposed
// copy).  D (optional) has C's shape and may be one of the operands.
//
// CTA = 6 warps, one per SM, persistent over (batch, tile) with tiles of
// 128 x 256 x 64: warp 0 TMA producer (3-D tensor maps, 4-stage ring, 128-byte
// swizzle; an MN-major B tile is four 64-column boxes), warp 1 TMEM owner
// (two 128 x 256 fp32 accumulators) and MMA issue, warps 2..5 epilogue that
// overlaps the next tile's MMAs.  Every wait is bounded (sm100.cuh).
//
// Used by the batched Newton-Schulz iteration of Muon (ns.cu) and available as
// `gemm_batched` for grouped GEMMs with equal shapes.
#include "../common.cuh"
#include "sm100.cuh"

namespace lrb {

__device__ int g_gemm_batched_err[4];
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, GROUP_M = 8;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kStageA = BM * BK * 2, kStageB = BN * BK * 2;  // 16 KB, 32 KB
constexpr uint32_t kMnBlock = 64 * BK * 2;                        // 8 KB: 64 N columns x 64 K rows
constexpr size_t kSmem = 1024 + STAGES * (size_t)(kStageA + kStageB) + 256;

struct BatchedArgs {
  __nv_bfloat16* C;
  const __nv_bfloat16* D;
  int64_t c_batch, c_row;  // strides in elements
  int64_t d_batch, d_row;
  int M, N, K, batch;
  float alpha, beta;
  int vec_ok;
  int* err;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tile_of(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int per_group = GROUP_M * tiles_n;
  const int g = t / per_group, first = g * GROUP_M, gsize = min(tiles_m - first, GROUP_M), r = t % per_group;
  tm = first + r % gsize;
  tn = r / gsize;
}

template <bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_batched_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        BatchedArgs a) {
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
  const int tiles_m = (a.M + BM - 1) / BM, tiles_n = (a.N + BN - 1) / BN;
  const int per_batch = tiles_m * tiles_n;
  const int num_tiles = per_batch * a.batch;
  const int nk = (a.K + BK - 1) / BK;

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
        const int bi = tile / per_batch;
        int tm, tn;
        tile_of(tile % per_batch, tiles_m, tiles_n, tm, tn);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, a.err, kErrTmaWait)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], kStageA + kStageB);
          tma_load_3d(sA + stage * kStageA, &tmA, &full[stage], kb * BK, tm * BM, bi);
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(sB + stage * kStageB + j * kMnBlock, &tmB, &full[stage], tn * BN + j * 64, kb * BK, bi);
          } else {
            tma_load_3d(sB + stage * kStageB, &tmB, &full[stage], kb * BK, tn * BN, bi);
          }
          ++armed;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      for (int i = 1; i <= STAGES && i <= armed; ++i) {
        const int64_t pos = armed - i;
        mbar_wait(&full[pos % STAGES], (uint32_t)((pos / STAGES) & 1), nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_major(BM, BN, true, false, B_MN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&accempty[acc], acc_phase ^ 1, a.err, kErrAccWait)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase, a.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sA + stage * kStageA), b0 = smem_addr(sB + stage * kStageB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t bdesc = B_MN ? umma_desc_mn_sw128(b0 + k * 2048, kMnBlock, 1024) : umma_desc_k_sw128(b0 + k * 32);
            umma_f16(d, umma_desc_k_sw128(a0 + k * 32), bdesc, idesc, (kb | k) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit(&accfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int bi = tile / per_batch;
      int tm, tn;
      tile_of(tile % per_batch, tiles_m, tiles_n, tm, tn);
      if (!mbar_wait(&accfull[acc], acc_phase, a.err, kErrEpiWait)) break;
      tc_fence_after();
      const int row = tm * BM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
        tmem_ld_wait();
        const int col0 = tn * BN + c * 32;
        if (row >= a.M || col0 >= a.N) continue;
        __nv_bfloat16* dst = a.C + bi * a.c_batch + (int64_t)row * a.c_row + col0;
        const __nv_bfloat16* dd = a.D != nullptr ? a.D + bi * a.d_batch + (int64_t)row * a.d_row + col0 : nullptr;
        if (a.vec_ok && col0 + 32 <= a.N) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            Vec16<__nv_bfloat16> v, w;
            if (dd != nullptr) w.raw = *reinterpret_cast<const uint4*>(dd + e);
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              float y = a.alpha * __uint_as_float(r[e + t]);
              if (dd != nullptr) y += a.beta * __bfloat162float(w.v[t]);
              v.v[t] = __float2bfloat16_rn(y);
            }
            st16(dst + e, v);
          }
        } else {
          for (int e = 0; e < 32 && col0 + e < a.N; ++e) {
            float y = a.alpha * __uint_as_float(r[e]);
            if (dd != nullptr) y += a.beta * __bfloat162float(dd[e]);
            dst[e] = __float2bfloat16_rn(y);
          }
        }
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

// (batch, rows, cols) bf16 with unit column stride; box = box_cols x box_rows x 1.
CUtensorMap map3d(const at::Tensor& t, int box_cols, int box_rows) {
  CUtensorMap m;
  const cuuint64_t dims[3] = {(cuuint64_t)t.size(2), (cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  const cuuint64_t strides[2] = {(cuuint64_t)t.stride(1) * 2, (cuuint64_t)t.stride(0) * 2};
  const cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (batched gemm) failed with code ", (int)r);
  return m;
}

// Error words of this file's kernels: module globals (one copy per device).
DeviceWord g_gemm_batched_err_word{g_gemm_batched_err, {}};

int* batched_error_word(const at::Device& dev) { return g_gemm_batched_err_word.get(dev.index()); }

void check3(const at::Tensor& t, const char* name) {
  LRB_CHECK(t.is_cuda() && t.dim() == 3 && t.scalar_type() == at::kBFloat16 && t.stride(2) == 1,
            "gemm_batched: ", name, " must be a 3-D bf16 CUDA tensor with unit last stride");
  LRB_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && (t.stride(1) * 2) % 16 == 0 &&
                (t.stride(0) * 2) % 16 == 0,
            "gemm_batched: ", name, " needs 16-byte aligned base and strides");
}

}  // namespace

// C = alpha * A op(B) + beta * D, see the header.  C is written in place.
void gemm_batched(const at::Tensor& A, const at::Tensor& B, bool b_mn, const at::Tensor& C,
                  const c10::optional<at::Tensor>& D, double alpha, double beta) {
  check3(A, "A");
  check3(B, "B");
  check3(C, "C");
  const int64_t Bt = A.size(0), M = A.size(1), K = A.size(2);
  const int64_t N = b_mn ? B.size(2) : B.size(1);
  LRB_CHECK(B.size(0) == Bt && (b_mn ? B.size(1) : B.size(2)) == K, "gemm_batched: B shape mismatch");
  LRB_CHECK(C.size(0) == Bt && C.size(1) == M && C.size(2) == N, "gemm_batched: C shape mismatch");
  if (D) {
    check3(*D, "D");
    LRB_CHECK(D->sizes() == C.sizes(), "gemm_batched: D must have C's shape");
  }
  LRB_CHECK(C.data_ptr() != A.data_ptr() && C.data_ptr() != B.data_ptr(), "gemm_batched: C must not alias A or B");
  c10::cuda::CUDAGuard g(A.device());
  bind_device(A.get_device());
  if (C.numel() == 0) return;
  LRB_CHECK(K > 0, "gemm_batched: K must be positive");
  CUtensorMap ta = map3d(A, BK, BM);
  CUtensorMap tb = b_mn ? map3d(B, 64, BK) : map3d(B, BK, BN);
  const bool vec = (C.stride(1) % 8 == 0) && (C.stride(0) % 8 == 0) &&
                   (!D || ((D->stride(1) % 8 == 0) && (D->stride(0) % 8 == 0)));
  BatchedArgs args{reinterpret_cast<__nv_bfloat16*>(C.data_ptr()),
                   D ? reinterpret_cast<const __nv_bfloat16*>(D->data_ptr()) : nullptr,
                   C.stride(0), C.stride(1), D ? D->stride(0) : 0, D ? D->stride(1) : 0,
                   (int)M, (int)N, (int)K, (int)Bt, (float)alpha, (float)beta, vec ? 1 : 0,
                   batched_error_word(A.device())};
  const int tiles = (int)(Bt * ((M + BM - 1) / BM) * ((N + BN - 1) / BN));
  const int grid = std::max(1, std::min(tiles, num_sms()));
  if (b_mn) {
    LRB_CUDA_CHECK(cudaFuncSetAttribute(gemm_batched_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    gemm_batched_kernel<true><<<grid, kThreads, kSmem, stream()>>>(ta, tb, args);
  } else {
    LRB_CUDA_CHECK(cudaFuncSetAttribute(gemm_batched_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    gemm_batched_kernel<false><<<grid, kThreads, kSmem, stream()>>>(ta, tb, args);
  }
  LRB_LAUNCH_CHECK();
}

int64_t gemm_batched_error(int64_t device) { return g_gemm_batched_err_word.take((int)device); }

}  // namespace lrb
