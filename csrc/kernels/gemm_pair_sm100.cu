// Persistent CTA-pair tcgen05 GEMM for the model's linears (forward, dgrad and
// wgrad), bf16/fp16 operands, fp32 accumulation in tensor memory:
//
//   C[M, N]  = alpha * op(A) op(B)^T          (bf16 / fp16 / fp32 C), or
//   C[M, N] += alpha * op(A) op(B)^T          (fp32 C: gradient accumulation)
//
// Each operand is K-major (A stored (M, K), B stored (N, K): the nn.Linear
// layout) or MN-major (A stored (K, M), B stored (K, N)), so the three GEMMs of
// a linear layer read the activations, weights and output gradients where they
// lie, without transposed copies:
//   forward  Y  = X W^T     A = X  (K-major),  B = W  (K-major)
//   dgrad    dX = dY W      A = dY (K-major),  B = W  (MN-major)
//   wgrad    dW = dY^T X    A = dY (MN-major), B = X  (MN-major)
//
// A cluster of two CTAs (the two SMs of a TPC) computes one 256 x 256 output
// tile per step with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16): each
// CTA loads its 128 rows of A and its 128 rows (N) of B by TMA into its own
// shared memory, so per output element the shared-memory traffic is half that
// of a one-CTA 128 x 256 tile.  No TMA load uses multicast.
//
// Roles per CTA (6 warps):
//   warp 0     TMA producer: waits for a free stage (its own `empty`), loads its
//              halves; the completion bytes of both CTAs go to the leader's
//              `full` barrier (the leader announces 2 x stage bytes);
//   warp 1     owns tensor memory (512 columns: two 128 x 256 fp32
//              accumulators, allocated as a pair); on the leader (cluster rank 0)
//              lane 0 issues the MMAs and commits `empty` and `accfull` to both
//              CTAs;
//   warps 2-5  epilogue: tcgen05.ld of their 32-lane quarter, convert, store or
//              accumulate; then arrive on the leader's `accempty`, so the next
//              tile's MMAs overlap this epilogue.
// Tiles are visited in groups of GROUP_M tile rows so that the tiles in flight
// share A rows and B columns in L2.
//
// Every wait is bounded (sm100.cuh); on timeout the kernel records an error code
// in a device word, skips its remaining work, and both CTAs meet at a cluster
// barrier (after the leader drained its MMAs) before freeing tensor memory.
#include "../common.cuh"
#include "sm100.cuh"

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace lrb {

// Device error word of this kernel (module global: one per device, no allocation).
__device__ int g_gemm_pair_err;
DeviceWord g_gemm_pair_err_word{&g_gemm_pair_err, {}};

namespace {

using namespace sm100;

constexpr int BM = 128;         // rows of A per CTA (256 per pair)
constexpr int BN = 256;         // columns of the output tile (128 rows of B per CTA)
constexpr int BK = 64;          // K per stage (128 bytes of bf16: one swizzle row)
constexpr int STAGES = 6;
constexpr int GROUP_M = 8;      // tile rows per raster group
constexpr int kThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kHalfA = BM * BK * 2;        // 16 KB
constexpr uint32_t kHalfB = (BN / 2) * BK * 2;  // 16 KB
constexpr uint32_t kStage = kHalfA + kHalfB;
constexpr uint32_t kMnBox = 64 * BK * 2;        // 8 KB: 64 MN elements x 64 K rows
// Epilogue staging: 8 KB per epilogue warp, a ring of boxes of 32 rows x 32
// columns -- two fp32 boxes or four 16-bit boxes -- so a box is written while the
// TMA stores of the previous ones drain.
constexpr uint32_t kOutWarpBytes = 8192;
constexpr uint32_t kOutSmem = 4 * kOutWarpBytes;  // 32 KB
constexpr size_t kSmem = 1024 + (size_t)STAGES * kStage + kOutSmem + 512;

// kSwiGLU: the up / gate projection of a SwiGLU FFN.  CTA rank 0 loads its B
// half from W1 (map tmB) and rank 1 from W_gate (map tmB2), both at rows
// [tn * 128, +128), so accumulator columns 0..127 hold u = x W1^T and 128..255
// g = x W_gate^T of the same 128 hidden units.  The epilogue writes u and g into
// gu (rows x 2F: [u | g], kept for the backward) through tmC (u) and tmG (g),
// and h = silu(g) * u through tmH, each from the bf16-rounded u and g.
// kRoPE: the fused QKV projection of attention (head_dim 128, so a 256-column
// tile is two heads).  Heads whose first column lies below args.rot_cols (the
// query and key heads) are rotated at position (row % args.seq) + args.pos0 with
// the rotate-half rule out[i] = x[i] cos[i] - x[i+64] sin[i],
// out[i+64] = x[i+64] cos[i+64] + x[i] sin[i+64] on the bf16-rounded products,
// the fp32 tables args.cos / args.sin, stored column-major (128 x positions).
// kAxpby: C = alpha * acc + beta * D (16-bit C and D, D through map tmH): each
// epilogue warp TMA-loads the D box of a 32-column chunk into that chunk's
// staging slot two chunks ahead (an mbarrier per warp and slot), combines in
// place and stores the slot -- the Newton-Schulz updates P = c A A + b A and
// X' = P X + a X, and residual additions.
// kSwiGLUBwd: the down projection's dgrad dh = dY W2 followed by the SwiGLU
// backward: the epilogue TMA-loads the u and g boxes of the chunk (maps tmB2,
// tmH over gu = [u | g]) one chunk ahead into two staging slots and writes
// du = dh silu(g) and dg = dh u s (1 + g (1 - s)), s = sigmoid(g), through tmC
// and tmG (dgu = [du | dg]) from the same slots; dh itself never reaches memory.
enum Epi : int { kStore = 0, kAccumF32 = 1, kSwiGLU = 2, kRoPE = 3, kAxpby = 4, kSwiGLUBwd = 5 };

struct PairArgs {
  void* C;
  int64_t ldc;
  int M, N, K;
  float alpha;
  int vec_ok;   // C base and row pitch 16-byte aligned
  int tma_out;  // the epilogue stages boxes in shared memory and writes them with TMA
                // (stores, or reduce-adds when accumulating); else direct stores
  int splits;   // K ranges per output tile (accumulation only: partial sums reduce-add)
  int group_m;  // tile rows per raster group
  int batch;    // independent GEMMs of equal shape (the third tensor-map coordinate)
  int64_t c_batch;  // C stride between batches (elements)
  // kRoPE only: column-major (128 x tab_pitch) fp32 tables
  const float* cos;
  const float* sin;
  int seq, pos0, rot_cols;
  int64_t tab_pitch;
  // kAxpby only
  float beta;
  // Pipeline trace (null in normal runs): %globaltimer stamps of the first
  // kTraceUnits work units of CTA pair 0, layout [event][unit].
  unsigned long long* trace;
};

constexpr int kTraceUnits = 64;
enum PairTraceEv : int {
  kTrProdStart = 0, kTrMmaStart, kTrMmaEnd, kTrEpiStart, kTrEpiFreed, kTrEpiEnd,
  kTrC0Loaded, kTrC0Math, kTrC0Stored,  // first chunk of a tile: accumulator read, math done, boxes issued
  kTrEvents
};
std::atomic<unsigned long long*> g_gemm_pair_trace{nullptr};

__device__ __forceinline__ void trace_unit(const PairArgs& a, int ev, int i) {
  if (a.trace != nullptr && blockIdx.x == 0 && i < kTraceUnits) a.trace[ev * kTraceUnits + i] = global_ns();
}

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int group_m, int& tm, int& tn) {
  const int per_group = group_m * tiles_n;
  const int g = tile / per_group;
  const int first = g * group_m;
  const int gsize = min(tiles_m - first, group_m);
  const int r = tile % per_group;
  tm = first + r % gsize;
  tn = r / gsize;
}

// Work unit -> (tile row, tile column, k-block range).  Units of one split index
// are consecutive, so the units in flight share the same K range of A and B.
__device__ __forceinline__ void unit_coords(int unit, int num_tiles, int tiles_m, int tiles_n, int nk,
                                            const PairArgs& a, int& tm, int& tn, int& kb0, int& kb1, int& bi) {
  const int split = unit / num_tiles;  // num_tiles counts every batch
  const int t = unit - split * num_tiles, per_batch = tiles_m * tiles_n;
  bi = t / per_batch;
  tile_coords(t - bi * per_batch, tiles_m, tiles_n, a.group_m, tm, tn);
  kb0 = (int)((int64_t)nk * split / a.splits);
  kb1 = (int)((int64_t)nk * (split + 1) / a.splits);
}

// Writes this thread's row of a 32 x 32 box into the staging buffer in the TMA
// swizzle of its tensor map: 16-bit outputs are 64-byte rows (64-byte swizzle:
// 16-byte chunk j of row r at j ^ ((r >> 1) & 3)), fp32 outputs 128-byte rows
// (128-byte swizzle: chunk j at j ^ (r & 7)).  Conflict-free for 8 rows at a time.
template <typename OutT>
__device__ __forceinline__ void stage_row(unsigned char* box, int lane, float alpha, const uint32_t* r) {
  if constexpr (sizeof(OutT) == 4) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 v = make_float4(alpha * __uint_as_float(r[4 * j]), alpha * __uint_as_float(r[4 * j + 1]),
                             alpha * __uint_as_float(r[4 * j + 2]), alpha * __uint_as_float(r[4 * j + 3]));
      *reinterpret_cast<float4*>(box + lane * 128 + ((j ^ (lane & 7)) * 16)) = v;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      Vec16<OutT> v;
#pragma unroll
      for (int t = 0; t < 8; ++t) v.v[t] = from_f<OutT>(alpha * __uint_as_float(r[8 * j + t]));
      *reinterpret_cast<uint4*>(box + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16)) = v.raw;
    }
  }
}

__device__ __forceinline__ void tma_store_box(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_box(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

// 3-D tiled load of one epilogue box into this CTA's shared memory, completion on
// this CTA's mbarrier.  No multicast.
__device__ __forceinline__ void tma_load_box(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

template <typename OutT, int EPI>
__device__ __forceinline__ void store_chunk(const PairArgs& a, int bi, int row, int col0, const uint32_t* r) {
  if (row >= a.M || col0 >= a.N) return;
  if constexpr (EPI == kAccumF32) {
    float* c = reinterpret_cast<float*>(a.C) + bi * a.c_batch + (int64_t)row * a.ldc + col0;
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
#pragma unroll
      for (int j = 0; j < 32; ++j)  // unrolled: r[] stays in registers
        if (col0 + j < a.N) c[j] += a.alpha * __uint_as_float(r[j]);
    }
  } else {
    OutT* c = reinterpret_cast<OutT*>(a.C) + bi * a.c_batch + (int64_t)row * a.ldc + col0;
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
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < a.N) c[j] = from_f<OutT>(a.alpha * __uint_as_float(r[j]));
    }
  }
}

// 3-D tiled load (x, y, batch) into this CTA's shared memory, completion on an
// mbarrier that may live in the peer CTA.  No multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Loads this CTA's half of one stage: A rows [m0, m0 + 128) and B rows [n0, n0 + 128)
// at K offset k0.  MN-major operands are two 64-wide boxes each.
template <bool A_MN, bool B_MN>
__device__ __forceinline__ void load_stage(unsigned char* sa, unsigned char* sb, const CUtensorMap* tmA,
                                           const CUtensorMap* tmB, uint32_t bar, int m0, int n0, int k0, int bi) {
  if (A_MN) {
    tma_load_3d_pair(sa, tmA, bar, m0, k0, bi);
    tma_load_3d_pair(sa + kMnBox, tmA, bar, m0 + 64, k0, bi);
  } else {
    tma_load_3d_pair(sa, tmA, bar, k0, m0, bi);
  }
  if (B_MN) {
    tma_load_3d_pair(sb, tmB, bar, n0, k0, bi);
    tma_load_3d_pair(sb + kMnBox, tmB, bar, n0 + 64, k0, bi);
  } else {
    tma_load_3d_pair(sb, tmB, bar, k0, n0, bi);
  }
}

template <typename OutT, int EPI, bool BF16IN, bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmB2,
                     const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmG, PairArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = base;
  unsigned char* sB = base + STAGES * kHalfA;
  unsigned char* sOut = sB + STAGES * kHalfB;  // 1024-byte aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + kOutSmem);
  uint64_t* empty = full + STAGES;
  uint64_t* accfull = empty + STAGES;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  uint64_t* dbar = drain + 3;  // [4 epilogue warps][4 slots] (kAxpby)
  int* err = &g_gemm_pair_err;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = (int)cluster_id_x(), npairs = (int)nclusters_x();
  constexpr int TN = EPI == kSwiGLU ? BN / 2 : BN;  // output columns per tile (h columns for kSwiGLU)
  const int tiles_m = (args.M + 2 * BM - 1) / (2 * BM), tiles_n = (args.N + TN - 1) / TN;
  const int num_tiles = tiles_m * tiles_n * args.batch;
  const int nk = (args.K + BK - 1) / BK;
  const int num_units = num_tiles * args.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 8);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    if constexpr (EPI == kAxpby || EPI == kSwiGLUBwd)
      for (int i = 0; i < 16; ++i) mbar_init(&dbar[i], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.tma_out) tma_prefetch_desc(&tmC);
    if constexpr (EPI == kSwiGLU) {
      tma_prefetch_desc(&tmB2);
      tma_prefetch_desc(&tmH);
    }
    if constexpr (EPI == kAxpby) tma_prefetch_desc(&tmH);
    if constexpr (EPI == kSwiGLUBwd) {
      tma_prefetch_desc(&tmB2);
      tma_prefetch_desc(&tmH);
      tma_prefetch_desc(&tmG);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, tensor memory allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t armed = 0;
      bool ok = true;
      for (int unit = pair; unit < num_units && ok; unit += npairs) {
        int tm, tn, kb0, kb1, bi;
        unit_coords(unit, num_tiles, tiles_m, tiles_n, nk, args, tm, tn, kb0, kb1, bi);
        const int m0 = tm * 2 * BM + (int)rank * BM;
        const int n0 = EPI == kSwiGLU ? tn * (BN / 2) : tn * BN + (int)rank * (BN / 2);
        const CUtensorMap* mb = (EPI == kSwiGLU && rank == 1) ? &tmB2 : &tmB;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, err, kErrTmaWait)) { ok = false; break; }
          if (kb == kb0) trace_unit(args, kTrProdStart, (unit - pair) / npairs);
          const uint32_t fb = mapa_shared(smem_addr(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kStage);
          load_stage<A_MN, B_MN>(sA + stage * kHalfA, sB + stage * kHalfB, &tmA, mb, fb, m0, n0, kb * BK, bi);
          ++armed;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // The leader can wait for its last stages to land (which needs both CTAs'
      // bytes); the peer's loads land before the leader's MMAs read them, and
      // the cluster barrier below keeps the peer resident until then.
      if (leader) {
        for (int i = 1; i <= STAGES && i <= armed; ++i) {
          const int64_t pos = armed - i;
          mbar_wait(&full[pos % STAGES], (uint32_t)((pos / STAGES) & 1), nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16_major(2 * BM, BN, BF16IN, A_MN, B_MN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int unit = pair; unit < num_units && ok; unit += npairs) {
        int tm, tn, kb0, kb1, bi;
        unit_coords(unit, num_tiles, tiles_m, tiles_n, nk, args, tm, tn, kb0, kb1, bi);
        if (!mbar_wait(&accempty[acc], acc_phase ^ 1, err, kErrAccWait)) break;
        tc_fence_after();
        trace_unit(args, kTrMmaStart, (unit - pair) / npairs);
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sA + stage * kHalfA), b0 = smem_addr(sB + stage * kHalfB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? umma_desc_mn_sw128(a0 + k * 2048, kMnBox, 1024) : umma_desc_k_sw128(a0 + k * 32);
            const uint64_t bd = B_MN ? umma_desc_mn_sw128(b0 + k * 2048, kMnBox, 1024) : umma_desc_k_sw128(b0 + k * 32);
            umma_f16_pair(d, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        umma_commit_pair_mc(&accfull[acc], 0x3);
        trace_unit(args, kTrMmaEnd, (unit - pair) / npairs);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      umma_commit_pair(drain);
      mbar_wait(drain, 0, nullptr, 0);  // every issued MMA retired before the pair frees tensor memory
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    unsigned char* boxes = sOut + (warp - 2) * kOutWarpBytes;
    constexpr uint32_t kBox = 32 * 32 * sizeof(OutT);           // bytes of one staged box
    constexpr int kSlots = (int)(kOutWarpBytes / kBox);         // 2 (fp32) or 4 (16-bit)
    int acc = 0, nbox = 0;
    uint32_t acc_phase = 0, dpar = 0;
    for (int unit = pair; unit < num_units; unit += npairs) {
      int tm, tn, kb0, kb1, bi;
      unit_coords(unit, num_tiles, tiles_m, tiles_n, nk, args, tm, tn, kb0, kb1, bi);
      if (!mbar_wait(&accfull[acc], acc_phase, err, kErrEpiWait)) break;
      tc_fence_after();
      const bool tracer = warp == 2 && lane == 0;  // one epilogue warp of the leader stamps
      const int ui = (unit - pair) / npairs;
      if (tracer) trace_unit(args, kTrEpiStart, ui);
      const int row0 = tm * 2 * BM + (int)rank * BM + q * 32;
      // one 32 x 32 box through the staging ring: stage this thread's row, TMA-store it
      auto put_box = [&](const CUtensorMap* map, const uint32_t* r, int x) {
        unsigned char* box = boxes + (nbox % kSlots) * kBox;
        // the store issued from this slot kSlots boxes ago has finished reading it
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kSlots - 1) : "memory");
        __syncwarp();
        stage_row<__nv_bfloat16>(box, lane, 1.f, r);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_box(map, box, x, row0, bi);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        ++nbox;
      };
      if constexpr (EPI == kRoPE) {
        const int row = row0 + lane;
        const int pos = (row < args.M ? row % args.seq : 0) + args.pos0;
        // column-major (128 x positions) tables: the warp's 32 consecutive
        // positions of one column are one coalesced line
        const float* ct = args.cos + pos;
        const float* st = args.sin + pos;
        const int64_t P = args.tab_pitch;
#pragma unroll 1
        for (int pc = 0; pc < 4; ++pc) {  // chunk pairs (0,2) (1,3) (4,6) (5,7): columns i and i + 64 of a head
          const int ca = (pc >> 1) * 4 + (pc & 1), cb = ca + 2;
          uint32_t xa[32], xb[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + ca * 32), xa);
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + cb * 32), xb);
          tmem_ld_wait();
          if (tracer && pc == 0) trace_unit(args, kTrC0Loaded, ui);
          if (pc == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&accempty[acc]), 0));
            if (tracer) trace_unit(args, kTrEpiFreed, ui);
          }
          const int col_a = tn * BN + ca * 32, col_b = tn * BN + cb * 32;
          if (row0 >= args.M || col_a >= args.N) continue;
          const int head_col0 = tn * BN + (pc >> 1) * 128;
          if (head_col0 < args.rot_cols) {
            const int i0 = (pc & 1) * 32;  // index within the first half of the head
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float c1 = __ldg(ct + (i0 + j) * P), s1 = __ldg(st + (i0 + j) * P);
              const float c2 = __ldg(ct + (64 + i0 + j) * P), s2 = __ldg(st + (64 + i0 + j) * P);
              const float x = __bfloat162float(__float2bfloat16_rn(__uint_as_float(xa[j])));
              const float y = __bfloat162float(__float2bfloat16_rn(__uint_as_float(xb[j])));
              xa[j] = __float_as_uint(x * c1 - y * s1);
              xb[j] = __float_as_uint(y * c2 + x * s2);
            }
          }
          if (tracer && pc == 0) trace_unit(args, kTrC0Math, ui);
          put_box(&tmC, xa, col_a);
          if (col_b < args.N) put_box(&tmC, xb, col_b);
          if (tracer && pc == 0) trace_unit(args, kTrC0Stored, ui);
        }
        if (tracer) trace_unit(args, kTrEpiEnd, ui);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        continue;
      }
      if constexpr (EPI == kAxpby) {
        uint64_t* db = dbar + (warp - 2) * 4;
        const int nbase = nbox;
        auto valid = [&](int c) { return row0 < args.M && tn * BN + c * 32 < args.N; };
        auto load_d = [&](int c) {  // lane 0: the D box of chunk c into its slot
          const int sd = (nbase + c) % kSlots;
          mbar_arrive_expect_tx(&db[sd], kBox);
          tma_load_box(boxes + sd * kBox, &tmH, &db[sd], tn * BN + c * 32, row0, bi);
        };
        uint32_t pend = 0;  // slots with a D load issued and not yet waited for (same in every lane)
        if (lane == 0) {
          // the slots of chunks 0 and 1 last held the stores of chunks nbase-4 and nbase-3
          if (valid(0)) {
            asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory");
            load_d(0);
          }
          if (valid(1)) {
            asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory");
            load_d(1);
          }
        }
        if (valid(0)) pend |= 1u << (nbase % kSlots);
        if (valid(1)) pend |= 1u << ((nbase + 1) % kSlots);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
          tmem_ld_wait();
          if (c == BN / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&accempty[acc]), 0));
            if (tracer) trace_unit(args, kTrEpiFreed, ui);
          }
          if (!valid(c)) continue;  // and so every later chunk of the tile
          if (c + 2 < BN / 32 && valid(c + 2)) {
            if (lane == 0) {
              asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");  // chunk c-2's store read its slot
              load_d(c + 2);
            }
            pend |= 1u << ((nbase + c + 2) % kSlots);
          }
          const int sd = (nbase + c) % kSlots;
          unsigned char* box = boxes + sd * kBox;
          const bool got = mbar_wait(&db[sd], (dpar >> sd) & 1u, err, kErrEpiWait);
          dpar ^= 1u << sd;
          pend &= ~(1u << sd);
          if (!got) {
            // give up, but only after the loads still in flight have landed (bounded waits)
            for (int s2 = 0; s2 < kSlots; ++s2)
              if (pend & (1u << s2)) mbar_wait(&db[s2], (dpar >> s2) & 1u, nullptr, 0);
            break;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4* p = reinterpret_cast<uint4*>(box + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16));
            Vec16<OutT> dv;
            dv.raw = *p;
#pragma unroll
            for (int t = 0; t < 8; ++t)
              dv.v[t] = from_f<OutT>(fmaf(args.alpha, __uint_as_float(r[8 * j + t]), args.beta * to_f(dv.v[t])));
            *p = dv.raw;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_box(&tmC, box, tn * BN + c * 32, row0, bi);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          ++nbox;
        }
        if (tracer) trace_unit(args, kTrEpiEnd, ui);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        continue;
      }
      if constexpr (EPI == kSwiGLUBwd) {
        // slots 2 (n & 1) and 2 (n & 1) + 1 hold the u and g boxes of chunk n
        uint64_t* db = dbar + (warp - 2) * 4;
        const int nbase = nbox;
        auto valid = [&](int c) { return row0 < args.M && tn * BN + c * 32 < args.N; };
        auto load_ug = [&](int c) {  // lane 0
          const int s0 = 2 * ((nbase + c) & 1);
          mbar_arrive_expect_tx(&db[s0], kBox);
          tma_load_box(boxes + s0 * kBox, &tmB2, &db[s0], tn * BN + c * 32, row0, 0);
          mbar_arrive_expect_tx(&db[s0 + 1], kBox);
          tma_load_box(boxes + (s0 + 1) * kBox, &tmH, &db[s0 + 1], tn * BN + c * 32, row0, 0);
        };
        uint32_t pend = 0;
        if (valid(0)) {
          if (lane == 0) {
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // earlier stores have read their slots
            load_ug(0);
          }
          pend |= 3u << (2 * (nbase & 1));
        }
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
          tmem_ld_wait();
          if (c == BN / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&accempty[acc]), 0));
            if (tracer) trace_unit(args, kTrEpiFreed, ui);
          }
          if (!valid(c)) continue;  // and so every later chunk of the tile
          if (c + 1 < BN / 32 && valid(c + 1)) {
            if (lane == 0) {
              asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // chunk c-1's stores read the slots
              load_ug(c + 1);
            }
            pend |= 3u << (2 * ((nbase + c + 1) & 1));
          }
          const int s0 = 2 * ((nbase + c) & 1);
          bool got = mbar_wait(&db[s0], (dpar >> s0) & 1u, err, kErrEpiWait);
          dpar ^= 1u << s0;
          got = got && mbar_wait(&db[s0 + 1], (dpar >> (s0 + 1)) & 1u, err, kErrEpiWait);
          dpar ^= 1u << (s0 + 1);
          pend &= ~(3u << s0);
          if (!got) {
            for (int s2 = 0; s2 < kSlots; ++s2)
              if (pend & (1u << s2)) mbar_wait(&db[s2], (dpar >> s2) & 1u, nullptr, 0);
            break;
          }
          unsigned char* ub = boxes + s0 * kBox;
          unsigned char* gb = ub + kBox;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int off = lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16);
            Vec16<__nv_bfloat16> uv, gv;
            uv.raw = *reinterpret_cast<const uint4*>(ub + off);
            gv.raw = *reinterpret_cast<const uint4*>(gb + off);
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const float d = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[8 * j + t])));  // dh in bf16
              const float u = __bfloat162float(uv.v[t]), g = __bfloat162float(gv.v[t]);
              const float sg = fast_rcp(1.f + fast_exp2(-kLog2e * g));
              uv.v[t] = __float2bfloat16_rn(d * g * sg);
              gv.v[t] = __float2bfloat16_rn(d * u * sg * (1.f + g * (1.f - sg)));
            }
            *reinterpret_cast<uint4*>(ub + off) = uv.raw;
            *reinterpret_cast<uint4*>(gb + off) = gv.raw;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_box(&tmC, ub, tn * BN + c * 32, row0, 0);
            tma_store_box(&tmG, gb, tn * BN + c * 32, row0, 0);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          ++nbox;
        }
        if (tracer) trace_unit(args, kTrEpiEnd, ui);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        continue;
      }
      if constexpr (EPI == kSwiGLU) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t u[32], g[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), u);
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + 128 + c * 32), g);
          tmem_ld_wait();
          if (tracer && c == 0) trace_unit(args, kTrC0Loaded, ui);
          if (c == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&accempty[acc]), 0));
            if (tracer) trace_unit(args, kTrEpiFreed, ui);
          }
          const int col0 = tn * (BN / 2) + c * 32;
          if (row0 >= args.M || col0 >= args.N) continue;
          uint32_t h[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float uf = __bfloat162float(__float2bfloat16_rn(__uint_as_float(u[j])));
            const float gf = __bfloat162float(__float2bfloat16_rn(__uint_as_float(g[j])));
            h[j] = __float_as_uint(gf * fast_rcp(1.f + fast_exp2(-kLog2e * gf)) * uf);
          }
          if (tracer && c == 0) trace_unit(args, kTrC0Math, ui);
          // u and g through maps F columns wide each, so a ragged last tile is
          // clipped at F and never spills into the other half of gu
          put_box(&tmC, u, col0);
          put_box(&tmG, g, col0);
          put_box(&tmH, h, col0);
          if (tracer && c == 0) trace_unit(args, kTrC0Stored, ui);
        }
        if (tracer) trace_unit(args, kTrEpiEnd, ui);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
        tmem_ld_wait();
        if (tracer && c == 0) trace_unit(args, kTrC0Loaded, ui);
        if (c == BN / 32 - 1) {  // the accumulator is read out: the MMAs may reuse it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&accempty[acc]), 0));
          if (tracer) trace_unit(args, kTrEpiFreed, ui);
        }
        const int col0 = tn * BN + c * 32;
        if (args.tma_out) {
          if (row0 >= args.M || col0 >= args.N) continue;
          unsigned char* box = boxes + (nbox % kSlots) * kBox;
          // the store issued from this slot kSlots boxes ago has finished reading it
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kSlots - 1) : "memory");
          __syncwarp();
          stage_row<OutT>(box, lane, args.alpha, r);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI == kAccumF32) tma_reduce_add_box(&tmC, box, col0, row0, bi);
            else tma_store_box(&tmC, box, col0, row0, bi);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          ++nbox;
        } else {
          store_chunk<OutT, EPI>(args, bi, row0 + lane, col0, r);
        }
        if (tracer && c == 0) trace_unit(args, kTrC0Stored, ui);
      }
      if (tracer) trace_unit(args, kTrEpiEnd, ui);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // stores complete before exit
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs into both CTAs' tensor memory have retired
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
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

// `batch` row-major (rows x cols) matrices, row pitch `ld` and batch pitch `bstride`
// elements, 16-bit; box = box_cols x box_rows x 1, 128-byte swizzle (box_cols = 64).
CUtensorMap make_map(const void* ptr, int64_t batch, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
                     int box_cols, int box_rows, bool bf16) {
  CUtensorMap m;
  // A single matrix gets the batch pitch of a packed stack (rows * ld): a valid
  // 16-byte multiple that no coordinate ever steps by.
  const int64_t bp = batch > 1 ? bstride : std::max<int64_t>(rows, 1) * ld;
  const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(bp * 2)};
  const cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                           const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return m;
}

// Output box map: `batch` (rows x cols) C, box 32 x 32 x 1, 64-byte swizzle for
// 16-bit outputs and 128-byte swizzle for fp32.
CUtensorMap make_out_map(void* ptr, int64_t batch, int64_t rows, int64_t cols, int64_t ld, int64_t bstride,
                         at::ScalarType t) {
  CUtensorMap m;
  const int esz = t == at::kFloat ? 4 : 2;
  const int64_t bp = batch > 1 ? bstride : std::max<int64_t>(rows, 1) * ld;
  const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)(ld * esz), (cuuint64_t)(bp * esz)};
  const cuuint32_t box[3] = {32, 32, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = t == at::kFloat      ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : t == at::kBFloat16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = encode_fn()(&m, dt, 3, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           esz == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (gemm_pair output) failed with code ", (int)r);
  return m;
}

// Clusters of two that fit at once on this device (cached per device).
int max_pairs(int dev) {
  static int cached[64] = {0};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  int sms = 0;
  LRB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int n = sms / 2;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * n, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto k = gemm_pair_kernel<__nv_bfloat16, kStore, true, false, false>;
  LRB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) == cudaSuccess && clusters > 0) n = std::min(n, clusters);
  (void)cudaGetLastError();
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

template <typename OutT, int EPI, bool BF16IN, bool A_MN, bool B_MN>
void launch_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const PairArgs& args, int pairs,
              const CUtensorMap* tb2 = nullptr, const CUtensorMap* th = nullptr, const CUtensorMap* tg = nullptr) {
  auto k = gemm_pair_kernel<OutT, EPI, BF16IN, A_MN, B_MN>;
  LRB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
  PairArgs a = args;
  a.trace = g_gemm_pair_trace.load(std::memory_order_acquire);
  k<<<2 * pairs, kThreads, kSmem, stream()>>>(ta, tb, tc, tb2 ? *tb2 : tb, th ? *th : tc, tg ? *tg : tc, a);
  LRB_LAUNCH_CHECK();
}

template <typename OutT, int EPI, bool BF16IN>
void launch_layout(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                   const PairArgs& args, int pairs) {
  if (!a_mn && !b_mn) launch_t<OutT, EPI, BF16IN, false, false>(ta, tb, tc, args, pairs);
  else if (!a_mn && b_mn) launch_t<OutT, EPI, BF16IN, false, true>(ta, tb, tc, args, pairs);
  else if (a_mn && b_mn) launch_t<OutT, EPI, BF16IN, true, true>(ta, tb, tc, args, pairs);
  else launch_t<OutT, EPI, BF16IN, true, false>(ta, tb, tc, args, pairs);
}

// Split count for an accumulating GEMM: the number of K ranges per tile (each of
// at least 16 k-blocks) that best fills whole waves of CTA pairs.
int choose_splits(int tiles, int pairs, int nk) {
  if (tiles >= 4 * pairs) return 1;
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= 8 && nk / s >= 16; ++s) {
    const int units = tiles * s;
    const int waves = (units + pairs - 1) / pairs;
    const double eff = (double)units / ((double)waves * pairs);
    if (eff > best_eff + 0.03) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

// (rows, cols) or (batch, rows, cols) view: returns (batch, rows, cols, row pitch, batch pitch).
struct Mat {
  int64_t batch, rows, cols, ld, bstride;
};

Mat check_operand(const at::Tensor& t, const char* name, bool sixteen_bit) {
  LRB_CHECK(t.is_cuda() && (t.dim() == 2 || t.dim() == 3) && t.stride(-1) == 1, "gemm_pair: ", name,
            " must be a 2-D or 3-D CUDA tensor with unit column stride");
  if (sixteen_bit)
    LRB_CHECK(t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kHalf, "gemm_pair: ", name,
              " must be bf16/fp16");
  const int64_t esz = t.element_size();
  Mat m{t.dim() == 3 ? t.size(0) : 1, t.size(-2), t.size(-1), t.stride(-2), t.dim() == 3 ? t.stride(0) : 0};
  LRB_CHECK(m.ld > 0 || m.rows <= 1, "gemm_pair: ", name, " row pitch must be positive");
  return m;
}

bool tma_ok(const at::Tensor& t, const Mat& m) {
  const int64_t esz = t.element_size();
  return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && (m.ld * esz) % 16 == 0 && (m.bstride * esz) % 16 == 0;
}

}  // namespace

// C = alpha * op(A) op(B)^T, or += when `accumulate` (then C is fp32).  a_mn: A is
// stored (K, M), otherwise (M, K); b_mn: B is stored (K, N), otherwise (N, K).  All
// three may carry a leading batch dimension (the same for each): one launch runs
// every batch entry.
void gemm_pair(const at::Tensor& A, const at::Tensor& B, bool a_mn, bool b_mn, at::Tensor& C, bool accumulate,
               double alpha) {
  const Mat a = check_operand(A, "A", true), b = check_operand(B, "B", true), c = check_operand(C, "C", false);
  LRB_CHECK(A.scalar_type() == B.scalar_type(), "gemm_pair: A and B must have the same dtype");
  LRB_CHECK(A.dim() == B.dim() && A.dim() == C.dim() && a.batch == b.batch && a.batch == c.batch,
            "gemm_pair: A, B and C must all be 2-D or all 3-D with one batch size");
  LRB_CHECK(tma_ok(A, a) && tma_ok(B, b), "gemm_pair: A and B need 16-byte aligned bases and pitches");
  LRB_CHECK(a.batch == 1 || (a.bstride >= a.rows * a.ld && b.bstride >= b.rows * b.ld && c.bstride >= c.rows * c.ld),
            "gemm_pair: batch entries must not overlap (batch pitch >= rows * row pitch)");
  const int64_t M = a_mn ? a.cols : a.rows, K = a_mn ? a.rows : a.cols;
  const int64_t N = b_mn ? b.cols : b.rows, KB = b_mn ? b.rows : b.cols;
  LRB_CHECK(K == KB, "gemm_pair: K mismatch (", K, " vs ", KB, ")");
  LRB_CHECK(c.rows == M && c.cols == N, "gemm_pair: C must be (M, N)");
  LRB_CHECK(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31) && a.batch < (1LL << 16),
            "gemm_pair: dimensions too large");
  LRB_CHECK(!accumulate || C.scalar_type() == at::kFloat, "gemm_pair: accumulation needs an fp32 C");
  LRB_CHECK(C.data_ptr() != A.data_ptr() && C.data_ptr() != B.data_ptr(), "gemm_pair: C must not alias A or B");
  c10::cuda::CUDAGuard g(A.device());
  bind_device(A.get_device());
  if (M == 0 || N == 0 || a.batch == 0) return;
  if (K == 0) {
    if (!accumulate) C.zero_();
    return;
  }
  const bool bf = A.scalar_type() == at::kBFloat16;
  // TMA boxes: K-major 64 (K) x 128 rows; MN-major 64 (MN) x 64 (K) rows.
  CUtensorMap ta = a_mn ? make_map(A.data_ptr(), a.batch, K, M, a.ld, a.bstride, 64, BK, bf)
                        : make_map(A.data_ptr(), a.batch, M, K, a.ld, a.bstride, BK, BM, bf);
  CUtensorMap tb = b_mn ? make_map(B.data_ptr(), b.batch, K, N, b.ld, b.bstride, 64, BK, bf)
                        : make_map(B.data_ptr(), b.batch, N, K, b.ld, b.bstride, BK, BN / 2, bf);
  const auto ct = C.scalar_type();
  LRB_CHECK(ct == at::kBFloat16 || ct == at::kHalf || ct == at::kFloat, "gemm_pair: unsupported output dtype");
  const bool aligned = tma_ok(C, c);
  const int tiles = (int)(a.batch * ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN));
  const int nk = (int)((K + BK - 1) / BK);
  const int maxp = max_pairs(A.get_device());
  // Partial sums of one tile may only meet in C through the TMA reduce-add.
  const int splits = (accumulate && aligned) ? choose_splits(tiles, maxp, nk) : 1;
  const int pairs = std::max(1, std::min(tiles * splits, maxp));
  // Raster groups of 8 tile rows; 16 when the B panel of a group is large (wide
  // outputs), so it is streamed from DRAM fewer times.  LRB_GEMM_GROUP_M
  // overrides it (a tuning knob for the raster study).
  static const int group_env = [] {
    const char* e = std::getenv("LRB_GEMM_GROUP_M");
    return e != nullptr ? std::atoi(e) : 0;
  }();
  const int group_m = group_env > 0 ? group_env : (N >= 16384 ? 16 : GROUP_M);
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  if (aligned) tc = make_out_map(C.data_ptr(), c.batch, M, N, c.ld, c.bstride, ct);
  PairArgs args{C.data_ptr(), c.ld, (int)M, (int)N, (int)K, (float)alpha, aligned ? 1 : 0, aligned ? 1 : 0,
                splits, group_m, (int)a.batch, c.bstride, nullptr, nullptr, 1, 0, 0};
  if (accumulate) {
    if (bf) launch_layout<float, kAccumF32, true>(a_mn, b_mn, ta, tb, tc, args, pairs);
    else launch_layout<float, kAccumF32, false>(a_mn, b_mn, ta, tb, tc, args, pairs);
  } else if (ct == at::kBFloat16) {
    if (bf) launch_layout<__nv_bfloat16, kStore, true>(a_mn, b_mn, ta, tb, tc, args, pairs);
    else launch_layout<__nv_bfloat16, kStore, false>(a_mn, b_mn, ta, tb, tc, args, pairs);
  } else if (ct == at::kHalf) {
    if (bf) launch_layout<__half, kStore, true>(a_mn, b_mn, ta, tb, tc, args, pairs);
    else launch_layout<__half, kStore, false>(a_mn, b_mn, ta, tb, tc, args, pairs);
  } else {
    if (bf) launch_layout<float, kStore, true>(a_mn, b_mn, ta, tb, tc, args, pairs);
    else launch_layout<float, kStore, false>(a_mn, b_mn, ta, tb, tc, args, pairs);
  }
}

// C = alpha * op(A) op(B)^T + beta * D (2-D, or 3-D batched), 16-bit A, B, C, D;
// A K-major, B K-major or MN-major (b_mn).  D may alias neither C nor A / B.
void gemm_pair_axpby(const at::Tensor& A, const at::Tensor& B, bool b_mn, at::Tensor& C, const at::Tensor& D,
                     double alpha, double beta) {
  const Mat a = check_operand(A, "A", true), b = check_operand(B, "B", true), c = check_operand(C, "C", true);
  const Mat dm = check_operand(D, "D", true);
  LRB_CHECK(A.scalar_type() == B.scalar_type() && C.scalar_type() == A.scalar_type() &&
                D.scalar_type() == A.scalar_type(),
            "gemm_pair_axpby: A, B, C and D of one 16-bit dtype");
  LRB_CHECK(A.dim() == B.dim() && A.dim() == C.dim() && A.dim() == D.dim() && a.batch == b.batch &&
                a.batch == c.batch && a.batch == dm.batch,
            "gemm_pair_axpby: operands all 2-D or all 3-D with one batch size");
  LRB_CHECK(tma_ok(A, a) && tma_ok(B, b) && tma_ok(C, c) && tma_ok(D, dm),
            "gemm_pair_axpby: 16-byte aligned bases and pitches");
  const int64_t M = a.rows, K = a.cols;
  const int64_t N = b_mn ? b.cols : b.rows, KB = b_mn ? b.rows : b.cols;
  LRB_CHECK(K == KB && c.rows == M && c.cols == N && dm.rows == M && dm.cols == N, "gemm_pair_axpby: shape mismatch");
  LRB_CHECK(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31) && a.batch < (1LL << 16),
            "gemm_pair_axpby: dimensions too large");
  LRB_CHECK(a.batch == 1 || (a.bstride >= a.rows * a.ld && b.bstride >= b.rows * b.ld && c.bstride >= c.rows * c.ld),
            "gemm_pair_axpby: batch entries must not overlap");
  LRB_CHECK(C.data_ptr() != A.data_ptr() && C.data_ptr() != B.data_ptr() && C.data_ptr() != D.data_ptr(),
            "gemm_pair_axpby: C must not alias A, B or D");
  c10::cuda::CUDAGuard g(A.device());
  bind_device(A.get_device());
  if (M == 0 || N == 0 || a.batch == 0) return;
  LRB_CHECK(K > 0, "gemm_pair_axpby: K must be positive");
  const bool bf = A.scalar_type() == at::kBFloat16;
  CUtensorMap ta = make_map(A.data_ptr(), a.batch, M, K, a.ld, a.bstride, BK, BM, bf);
  CUtensorMap tb = b_mn ? make_map(B.data_ptr(), b.batch, K, N, b.ld, b.bstride, 64, BK, bf)
                        : make_map(B.data_ptr(), b.batch, N, K, b.ld, b.bstride, BK, BN / 2, bf);
  CUtensorMap tc = make_out_map(C.data_ptr(), c.batch, M, N, c.ld, c.bstride, C.scalar_type());
  CUtensorMap td = make_out_map(D.data_ptr(), dm.batch, M, N, dm.ld, dm.bstride, D.scalar_type());
  const int tiles = (int)(a.batch * ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN));
  const int pairs = std::max(1, std::min(tiles, max_pairs(A.get_device())));
  PairArgs args{C.data_ptr(), c.ld, (int)M, (int)N, (int)K, (float)alpha, 1, 1, 1, GROUP_M, (int)a.batch, c.bstride,
                nullptr, nullptr, 1, 0, 0, 0, (float)beta};
  if (bf) {
    if (b_mn) launch_t<__nv_bfloat16, kAxpby, true, false, true>(ta, tb, tc, args, pairs, nullptr, &td);
    else launch_t<__nv_bfloat16, kAxpby, true, false, false>(ta, tb, tc, args, pairs, nullptr, &td);
  } else {
    if (b_mn) launch_t<__half, kAxpby, false, false, true>(ta, tb, tc, args, pairs, nullptr, &td);
    else launch_t<__half, kAxpby, false, false, false>(ta, tb, tc, args, pairs, nullptr, &td);
  }
}

// The down projection's dgrad with the SwiGLU backward in the epilogue:
// dgu = swiglu_bwd(dY W2, gu), i.e. [dh silu(g) | dh u s (1 + g (1 - s))] with
// dh = dY W2 (rows x F, never written), dY (rows x d), W2 (d x F, the nn.Linear
// weight, read MN-major), gu = [u | g] and dgu (rows x 2F), all bf16.
void gemm_pair_swiglu_bwd(const at::Tensor& DY, const at::Tensor& W2, const at::Tensor& GU, at::Tensor& DGU) {
  const Mat dy = check_operand(DY, "dy", true), w = check_operand(W2, "w2", true);
  const Mat gu = check_operand(GU, "gu", true), dg = check_operand(DGU, "dgu", true);
  LRB_CHECK(DY.dim() == 2 && W2.dim() == 2 && GU.dim() == 2 && DGU.dim() == 2, "gemm_pair_swiglu_bwd: 2-D operands");
  LRB_CHECK(DY.scalar_type() == at::kBFloat16 && W2.scalar_type() == at::kBFloat16 && GU.scalar_type() == at::kBFloat16 &&
                DGU.scalar_type() == at::kBFloat16,
            "gemm_pair_swiglu_bwd: bf16 operands");
  const int64_t M = dy.rows, K = dy.cols, F = w.cols;
  LRB_CHECK(w.rows == K && gu.rows == M && gu.cols == 2 * F && dg.rows == M && dg.cols == 2 * F,
            "gemm_pair_swiglu_bwd: shape mismatch");
  LRB_CHECK(F % 8 == 0, "gemm_pair_swiglu_bwd: F must be a multiple of 8 (the gate halves start 16-byte aligned)");
  LRB_CHECK(tma_ok(DY, dy) && tma_ok(W2, w) && tma_ok(GU, gu) && tma_ok(DGU, dg),
            "gemm_pair_swiglu_bwd: 16-byte aligned bases and pitches required");
  LRB_CHECK(DGU.data_ptr() != GU.data_ptr(), "gemm_pair_swiglu_bwd: dgu must not alias gu");
  c10::cuda::CUDAGuard g(DY.device());
  bind_device(DY.get_device());
  if (M == 0 || F == 0) return;
  LRB_CHECK(K > 0, "gemm_pair_swiglu_bwd: K must be positive");
  CUtensorMap ta = make_map(DY.data_ptr(), 1, M, K, dy.ld, 0, BK, BM, true);
  CUtensorMap tb = make_map(W2.data_ptr(), 1, K, F, w.ld, 0, 64, BK, true);  // MN-major B
  CUtensorMap tu = make_out_map(GU.data_ptr(), 1, M, F, gu.ld, 0, at::kBFloat16);
  CUtensorMap tg = make_out_map(static_cast<__nv_bfloat16*>(GU.data_ptr()) + F, 1, M, F, gu.ld, 0, at::kBFloat16);
  CUtensorMap tdu = make_out_map(DGU.data_ptr(), 1, M, F, dg.ld, 0, at::kBFloat16);
  CUtensorMap tdg = make_out_map(static_cast<__nv_bfloat16*>(DGU.data_ptr()) + F, 1, M, F, dg.ld, 0, at::kBFloat16);
  const int tiles = (int)(((M + 2 * BM - 1) / (2 * BM)) * ((F + BN - 1) / BN));
  const int pairs = std::max(1, std::min(tiles, max_pairs(DY.get_device())));
  PairArgs args{DGU.data_ptr(), dg.ld, (int)M, (int)F, (int)K, 1.f, 1, 1, 1, GROUP_M, 1, 0,
                nullptr, nullptr, 1, 0, 0, 0, 0.f};
  launch_t<__nv_bfloat16, kSwiGLUBwd, true, false, true>(ta, tb, tdu, args, pairs, &tu, &tg, &tdg);
}

// SwiGLU up / gate projection: gu = [x W1^T | x W_gate^T] (rows x 2F) and
// h = silu(x W_gate^T) * (x W1^T) (rows x F) in one launch; bf16, all K-major.
void gemm_pair_swiglu(const at::Tensor& X, const at::Tensor& W1, const at::Tensor& Wg, at::Tensor& GU, at::Tensor& Hout) {
  const Mat x = check_operand(X, "x", true), w1 = check_operand(W1, "w1", true), wg = check_operand(Wg, "w_gate", true);
  const Mat gu = check_operand(GU, "gu", false), hm = check_operand(Hout, "h", false);
  LRB_CHECK(X.dim() == 2 && W1.dim() == 2 && Wg.dim() == 2 && GU.dim() == 2 && Hout.dim() == 2,
            "gemm_pair_swiglu: 2-D operands");
  LRB_CHECK(X.scalar_type() == at::kBFloat16 && W1.scalar_type() == at::kBFloat16 && Wg.scalar_type() == at::kBFloat16 &&
                GU.scalar_type() == at::kBFloat16 && Hout.scalar_type() == at::kBFloat16,
            "gemm_pair_swiglu: bf16 operands");
  const int64_t M = x.rows, K = x.cols, F = w1.rows;
  LRB_CHECK(w1.cols == K && wg.cols == K && wg.rows == F && gu.rows == M && gu.cols == 2 * F && hm.rows == M &&
                hm.cols == F,
            "gemm_pair_swiglu: shape mismatch");
  LRB_CHECK(tma_ok(X, x) && tma_ok(W1, w1) && tma_ok(Wg, wg) && tma_ok(GU, gu) && tma_ok(Hout, hm),
            "gemm_pair_swiglu: 16-byte aligned bases and pitches required");
  c10::cuda::CUDAGuard g(X.device());
  bind_device(X.get_device());
  if (M == 0 || F == 0) return;
  CUtensorMap ta = make_map(X.data_ptr(), 1, M, K, x.ld, 0, BK, BM, true);
  CUtensorMap tb = make_map(W1.data_ptr(), 1, F, K, w1.ld, 0, BK, BN / 2, true);
  CUtensorMap tb2 = make_map(Wg.data_ptr(), 1, F, K, wg.ld, 0, BK, BN / 2, true);
  LRB_CHECK(F % 8 == 0, "gemm_pair_swiglu: F must be a multiple of 8 (the gate half of gu starts 16-byte aligned)");
  CUtensorMap tc = make_out_map(GU.data_ptr(), 1, M, F, gu.ld, 0, at::kBFloat16);
  CUtensorMap tg = make_out_map(static_cast<__nv_bfloat16*>(GU.data_ptr()) + F, 1, M, F, gu.ld, 0, at::kBFloat16);
  CUtensorMap th = make_out_map(Hout.data_ptr(), 1, M, F, hm.ld, 0, at::kBFloat16);
  const int tiles = (int)(((M + 2 * BM - 1) / (2 * BM)) * ((F + BN / 2 - 1) / (BN / 2)));
  const int pairs = std::max(1, std::min(tiles, max_pairs(X.get_device())));
  PairArgs args{GU.data_ptr(), gu.ld, (int)M, (int)F, (int)K, 1.f, 1, 1, 1, GROUP_M, 1, 0, nullptr, nullptr, 1, 0, 0};
  launch_t<__nv_bfloat16, kSwiGLU, true, false, false>(ta, tb, tc, args, pairs, &tb2, &th, &tg);
}

// Fused QKV projection with RoPE: out = x W^T (rows x N, N = (H + 2 Hkv) * 128),
// the first rot_cols columns (query and key heads) rotated at position
// (row % seq) + pos0 with the fp32 tables cos / sin, given transposed:
// (128, positions) contiguous.
void gemm_pair_rope(const at::Tensor& X, const at::Tensor& W, at::Tensor& Out, const at::Tensor& cos_t,
                    const at::Tensor& sin_t, int64_t seq, int64_t pos0, int64_t rot_cols) {
  const Mat x = check_operand(X, "x", true), w = check_operand(W, "w", true), o = check_operand(Out, "out", false);
  LRB_CHECK(X.dim() == 2 && W.dim() == 2 && Out.dim() == 2 && X.scalar_type() == at::kBFloat16 &&
                W.scalar_type() == at::kBFloat16 && Out.scalar_type() == at::kBFloat16,
            "gemm_pair_rope: 2-D bf16 operands");
  const int64_t M = x.rows, K = x.cols, N = w.rows;
  LRB_CHECK(w.cols == K && o.rows == M && o.cols == N && N % 256 == 0 && rot_cols % 128 == 0 && rot_cols <= N,
            "gemm_pair_rope: shapes (N a multiple of 256, 128-wide heads)");
  LRB_CHECK(tma_ok(X, x) && tma_ok(W, w) && tma_ok(Out, o), "gemm_pair_rope: 16-byte aligned bases and pitches");
  LRB_CHECK(cos_t.is_cuda() && sin_t.is_cuda() && cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat &&
                cos_t.is_contiguous() && sin_t.is_contiguous() && cos_t.dim() == 2 && cos_t.size(0) == 128 &&
                sin_t.sizes() == cos_t.sizes() && seq > 0 && pos0 >= 0 && seq + pos0 <= cos_t.size(1),
            "gemm_pair_rope: fp32 column-major (128, positions) cos / sin tables covering the positions");
  c10::cuda::CUDAGuard g(X.device());
  bind_device(X.get_device());
  if (M == 0) return;
  CUtensorMap ta = make_map(X.data_ptr(), 1, M, K, x.ld, 0, BK, BM, true);
  CUtensorMap tb = make_map(W.data_ptr(), 1, N, K, w.ld, 0, BK, BN / 2, true);
  CUtensorMap tc = make_out_map(Out.data_ptr(), 1, M, N, o.ld, 0, at::kBFloat16);
  const int tiles = (int)(((M + 2 * BM - 1) / (2 * BM)) * (N / BN));
  const int pairs = std::max(1, std::min(tiles, max_pairs(X.get_device())));
  PairArgs args{Out.data_ptr(), o.ld, (int)M, (int)N, (int)K, 1.f, 1, 1, 1, GROUP_M, 1, 0,
                cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), (int)seq, (int)pos0, (int)rot_cols, cos_t.size(1)};
  launch_t<__nv_bfloat16, kRoPE, true, false, false>(ta, tb, tc, args, pairs);
}

// Points the pair GEMM's pipeline trace at `buf` (int64 CUDA, at least
// kTrEvents * kTraceUnits entries: producer start, MMA start / end, epilogue start /
// accumulator freed / end of the first units of pair 0), or switches it off (None).
void gemm_pair_set_trace(const c10::optional<at::Tensor>& buf) {
  if (buf.has_value()) {
    LRB_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong && buf->is_contiguous() &&
                  buf->numel() >= (int64_t)kTrEvents * kTraceUnits,
              "gemm_pair_set_trace: an int64 CUDA buffer of ", (int64_t)kTrEvents * kTraceUnits, " entries");
    g_gemm_pair_trace.store(reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>()), std::memory_order_release);
  } else {
    g_gemm_pair_trace.store(nullptr, std::memory_order_release);
  }
}

// Returns and clears the error word of the pair GEMM on `device` (0 = no timeout).
int64_t gemm_pair_error(int64_t device) { return g_gemm_pair_err_word.take((int)device); }

}  // namespace lrb
