// NVFP4 block-scaled GEMM on tcgen05:  C[M, N] = sA * sB * sum_k (A[m,k] SFA) (B[n,k] SFB)
// with A, B in E2M1 (two per byte, even element in the low nibble), one e4m3
// scale per 16 elements along K (SFA, SFB) and one fp32 scale per tensor
// (sA, sB) -- the NVFP4 format.  Both operands are K-major (nn.Linear layout).
//
// Scale factors are stored in the tensor-core atom layout: for every block of
// 128 rows and 64 K-elements, 512 bytes with the scale of (row m, k-block j)
// at byte 16*(m % 32) + 4*(m / 32) + j; atoms are ordered K-fastest within a
// 128-row block (``nvfp4_swizzle_scales`` produces it).
//
// CTA = one 128 x 128 output tile (default; two CTAs per SM) or 128 x 256
// (two 128-column halves sharing the A tile), 6 warps:
//   warp 0      producer: per K-stage (256 elements = 128 bytes per row) TMA
//               loads of the A and B tiles (128-byte swizzle) and bulk copies
//               of the four SFA and four SFB atoms, into a 4-stage ring;
//   warp 1      TMEM owner + MMA issue: tcgen05.cp of the stage's scale atoms
//               into TMEM (two alternating column sets), then per half four
//               kind::mxf4nvf4 block16 MMAs (M = N = 128, K = 64 each);
//   warps 2..5  epilogue: tcgen05.ld, scale by sA*sB, bf16 stores.
// tcgen05.cp and tcgen05.mma issued by one thread execute in order, so a
// stage's scale copy precedes its MMAs without a wait.  All waits are bounded.
#include "../common.cuh"
#include "sm100.cuh"

#include <cstdlib>

namespace lrb {

__device__ int g_gemm_nvfp4_err[4];
namespace {

using namespace sm100;

constexpr int BM = 128, BKE = 256;  // BKE: FP4 elements per stage
constexpr int kThreads = 192;
constexpr uint32_t kStageA = BM * BKE / 2;  // 16 KB
constexpr uint32_t kAtom = 512, kAtomsPerStage = 4;  // four 64-element atoms per 128 rows
// NT = 128-column halves of the output tile (1: 128 x 128, 2: 128 x 256 sharing the A tile).
template <int NT>
struct Cfg {
  static constexpr uint32_t kStageB = NT * 128 * BKE / 2;
  static constexpr uint32_t kStageSFA = kAtomsPerStage * kAtom;
  static constexpr uint32_t kStageSFB = NT * kAtomsPerStage * kAtom;
  static constexpr uint32_t kStageBytes = kStageA + kStageB + kStageSFA + kStageSFB;
  static constexpr uint32_t kTmemCols = NT == 1 ? 256 : 512;
  static constexpr uint32_t kSFA = NT * 128;   // TMEM column of the SFA sets (2 sets x 16 columns)
  static constexpr uint32_t kSFB = kSFA + 32;  // NT halves x 2 sets x 16 columns
};
template <int NT, int STG>
constexpr size_t smem_bytes() { return 1024 + STG * (size_t)Cfg<NT>::kStageBytes + 256; }

struct Nvfp4Args {
  void* C;
  int64_t ldc;
  int M, N, K;
  const uint8_t* sfa;  // atoms
  const uint8_t* sfb;
  const float* sa;     // tensor scales
  const float* sb;
  int* err;
  int vec_ok;
};

template <int NT, int STG>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Nvfp4Args a) {
  using C_ = Cfg<NT>;
  constexpr int BN = NT * 128;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + STG * C_::kStageBytes);
  uint64_t* full = bars;          // [STG]
  uint64_t* empty = bars + STG;   // [STG]
  uint64_t* acc_full = bars + 2 * STG;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STG + 1);
  auto sA = [&](int s) { return base + s * C_::kStageBytes; };
  auto sB = [&](int s) { return base + s * C_::kStageBytes + kStageA; };
  auto sSFA = [&](int s) { return base + s * C_::kStageBytes + kStageA + C_::kStageB; };
  auto sSFB = [&](int s) { return base + s * C_::kStageBytes + kStageA + C_::kStageB + C_::kStageSFA; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tm = blockIdx.y, tn = blockIdx.x;
  const int m0 = tm * BM, n0 = tn * BN;
  const int nk = a.K / BKE;
  const int katoms = a.K / 64;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STG; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C_::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tAcc = tmem, tSFA = tmem + C_::kSFA, tSFB = tmem + C_::kSFB;

  if (warp == 0) {
    if (lane == 0) {
      int armed = 0;
      for (int j = 0; j < nk; ++j) {
        const int st = j % STG;
        const uint32_t ph = (j / STG) & 1;
        if (!mbar_wait(&empty[st], ph ^ 1, a.err, kErrTmaWait)) break;
        mbar_arrive_expect_tx(&full[st], C_::kStageBytes);
        tma_load_2d(sA(st), &tmA, &full[st], j * (BKE / 2), m0);
        bulk_load(sSFA(st), a.sfa + ((int64_t)tm * katoms + j * 4) * kAtom, C_::kStageSFA, &full[st]);
#pragma unroll
        for (int h = 0; h < NT; ++h) {
          tma_load_2d(sB(st) + h * (128 * BKE / 2), &tmB, &full[st], j * (BKE / 2), n0 + h * 128);
          bulk_load(sSFB(st) + h * C_::kStageSFA, a.sfb + ((int64_t)(tn * NT + h) * katoms + j * 4) * kAtom,
                    C_::kStageSFA, &full[st]);
        }
        ++armed;
      }
      for (int i = 1; i <= STG && i <= armed; ++i) {
        const int j = armed - i;
        mbar_wait(&full[j % STG], (j / STG) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_nvfp4(BM, 128);
      bool ok = true;
      for (int j = 0; j < nk && ok; ++j) {
        const int st = j % STG;
        const uint32_t ph = (j / STG) & 1;
        if (!mbar_wait(&full[st], ph, a.err, kErrMmaWait)) { ok = false; break; }
        tc_fence_after();
        const uint32_t set = (j & 1) * 16;
        const uint32_t fa = smem_addr(sSFA(st)), fb = smem_addr(sSFB(st));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          tmem_cp_32x128b_x4(tSFA + set + kk * 4, sf_desc(fa + kk * kAtom));
#pragma unroll
          for (int h = 0; h < NT; ++h)
            tmem_cp_32x128b_x4(tSFB + h * 32 + set + kk * 4, sf_desc(fb + h * C_::kStageSFA + kk * kAtom));
        }
        const uint32_t pa = smem_addr(sA(st)), pb = smem_addr(sB(st));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 64 FP4 elements = 32 bytes of the 128-byte swizzled row
#pragma unroll
          for (int h = 0; h < NT; ++h)
            umma_nvfp4(tAcc + h * 128, umma_desc_k_sw128(pa + kk * 32),
                       umma_desc_k_sw128(pb + h * (128 * BKE / 2) + kk * 32), idesc, tSFA + set + kk * 4,
                       tSFB + h * 32 + set + kk * 4, (j | kk) != 0);
        }
        umma_commit(&empty[st]);
      }
      umma_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const bool have = __all_sync(0xffffffffu, nk > 0 && mbar_wait(acc_full, 0, a.err, kErrEpiWait));
    tc_fence_after();
    const float alpha = *a.sa * *a.sb;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      if (have) {
        tmem_ld_32x32b_x32(tAcc + lane_base + c * 32, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = 0u;
      }
      const int col0 = n0 + c * 32;
      if (row >= a.M || col0 >= a.N) continue;
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.C) + (int64_t)row * a.ldc + col0;
      if (a.vec_ok && col0 + 32 <= a.N) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          Vec16<__nv_bfloat16> v;
#pragma unroll
          for (int t = 0; t < 8; ++t) v.v[t] = __float2bfloat16_rn(alpha * __uint_as_float(r[e + t]));
          st16(dst + e, v);
        }
      } else {
        for (int e = 0; e < 32 && col0 + e < a.N; ++e) dst[e] = __float2bfloat16_rn(alpha * __uint_as_float(r[e]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C_::kTmemCols);
  }
}

// ------------------------------------------------------------------ host
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

// packed (rows, K/2) uint8, row pitch ld bytes; box = 128 bytes x 128 rows
CUtensorMap fp4_map(const void* ptr, int64_t rows, int64_t bytes, int64_t ld) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (fp4) failed with code ", (int)r);
  return m;
}

// Error words of this file's kernels: module globals (one copy per device).
DeviceWord g_gemm_nvfp4_err_word{g_gemm_nvfp4_err, {}};

int* nvfp4_error_word(const at::Device& dev) { return g_gemm_nvfp4_err_word.get(dev.index()); }

}  // namespace

// A (M, K/2) uint8, sfa atoms (ceil(M/128) * K/64 * 512) uint8, sa () fp32; B likewise with N.
at::Tensor gemm_nvfp4(const at::Tensor& A, const at::Tensor& sfa, const at::Tensor& sa, const at::Tensor& B,
                      const at::Tensor& sfb, const at::Tensor& sb) {
  LRB_CHECK(A.is_cuda() && B.is_cuda() && A.scalar_type() == at::kByte && B.scalar_type() == at::kByte,
            "gemm_nvfp4: packed uint8 operands required");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1) * 2;
  LRB_CHECK(B.size(1) * 2 == K && K % BKE == 0, "gemm_nvfp4: K must match and be a multiple of 256");
  LRB_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && A.stride(0) % 16 == 0 && B.stride(0) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(A.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(B.data_ptr()) % 16 == 0,
            "gemm_nvfp4: operands need 16-byte aligned rows");
  const int64_t mb = (M + 127) / 128, nb = (N + 127) / 128;
  LRB_CHECK(sfa.numel() >= mb * (K / 64) * 512 && sfb.numel() >= nb * (K / 64) * 512 && sfa.is_contiguous() &&
                sfb.is_contiguous(),
            "gemm_nvfp4: scale atoms must cover ceil(rows/128) x K/64 x 512 bytes");
  c10::cuda::CUDAGuard g(A.device());
  bind_device(A.get_device());
  auto C = at::empty({M, N}, A.options().dtype(at::kBFloat16));
  if (M == 0 || N == 0) return C;
  CUtensorMap ta = fp4_map(A.data_ptr(), M, K / 2, A.stride(0)), tb = fp4_map(B.data_ptr(), N, K / 2, B.stride(0));
  Nvfp4Args args{C.data_ptr(), N, (int)M, (int)N, (int)K, sfa.data_ptr<uint8_t>(), sfb.data_ptr<uint8_t>(),
                 sa.data_ptr<float>(), sb.data_ptr<float>(), nvfp4_error_word(A.device()), (N % 8) == 0 ? 1 : 0};
  // Default: 128 x 128 tiles with 3 stages, two CTAs resident per SM, so one CTA's
  // epilogue overlaps the other's main loop (3.09 PFLOP/s at 8192^3, against 2.29
  // for one 128 x 256 CTA per SM).  LRB_NVFP4_TILE=256 selects the 128 x 256
  // tiles, LRB_NVFP4_TILE=128 one 128 x 128 CTA per SM with 4 stages.
  static const int tile_env = [] {
    const char* e = std::getenv("LRB_NVFP4_TILE");
    return e ? std::atoi(e) : 129;
  }();
  const bool wide = tile_env != 128 && tile_env != 129 && N % 256 == 0;
  if (tile_env == 129) {  // 128 x 128 tiles, 3 stages: two CTAs per SM overlap each other's epilogue
    constexpr size_t sm = smem_bytes<1, 3>();
    LRB_CUDA_CHECK(cudaFuncSetAttribute(gemm_nvfp4_kernel<1, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    // two CTAs of ~110 KB need the largest shared-memory carve-out of the SM
    LRB_CUDA_CHECK(cudaFuncSetAttribute(gemm_nvfp4_kernel<1, 3>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        (int)cudaSharedmemCarveoutMaxShared));
    gemm_nvfp4_kernel<1, 3><<<dim3((unsigned)nb, (unsigned)mb), kThreads, sm, stream()>>>(ta, tb, args);
  } else if (wide) {
    constexpr size_t sm = smem_bytes<2, 4>();
    LRB_CUDA_CHECK(cudaFuncSetAttribute(gemm_nvfp4_kernel<2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    gemm_nvfp4_kernel<2, 4><<<dim3((unsigned)(N / 256), (unsigned)mb), kThreads, sm, stream()>>>(ta, tb, args);
  } else {
    constexpr size_t sm = smem_bytes<1, 4>();
    LRB_CUDA_CHECK(cudaFuncSetAttribute(gemm_nvfp4_kernel<1, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    gemm_nvfp4_kernel<1, 4><<<dim3((unsigned)nb, (unsigned)mb), kThreads, sm, stream()>>>(ta, tb, args);
  }
  LRB_LAUNCH_CHECK();
  return C;
}

int64_t gemm_nvfp4_error(int64_t device) { return g_gemm_nvfp4_err_word.take((int)device); }

}  // namespace lrb
