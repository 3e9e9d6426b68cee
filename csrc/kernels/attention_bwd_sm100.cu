// Flash-attention backward on tcgen05 / TMEM for head_dim 128 (bf16).
//
// CTA = one (batch, kv-head, 128-key tile); it loops over the query heads of
// its group and over 128-query tiles.  Per tile, five tcgen05 GEMMs:
//   S^T  = K Q^T        (keys x queries) -> TMEM region A   [  0,128)
//   dP^T = V dO^T       (keys x queries) -> TMEM region B   [128,256)
//   dV  += P^T dO       (keys x hd)      -> TMEM            [256,384)  (all tiles)
//   dK  += dS^T Q       (keys x hd)      -> TMEM            [384,512)  (all tiles)
//   dQ   = dS K         (queries x hd)   -> TMEM region B   (after dP^T was read)
// P^T and dS^T are written by the softmax-gradient warps to shared memory in
// the K-major 128-byte-swizzled layout; dS (for dQ) and the Q / dO / K
// operands of the accumulating GEMMs are read MN-major from the same tiles,
// so nothing is transposed explicitly.  dQ is added to an fp32 buffer by TMA
// reduce-adds of 128 x 32 blocks staged in shared memory; dK and dV leave TMEM
// once at the end.
//
// Warps: 0 TMA (K, V once; Q and dO per tile), 1 TMEM owner + MMA issue,
// 2..9 softmax-gradient (two threads per key row, 64 query columns each).
// All waits are bounded (sm100.cuh).
#include "../common.cuh"
#include "sm100.cuh"

#include <cstdlib>

namespace lrb {

__device__ int g_attn_bwd_err[4];
namespace {

using namespace sm100;

constexpr int TK = 128, TQ = 128, HD = 128;
constexpr int kThreads = 320;
constexpr int kSmThreads = 256;
constexpr uint32_t kTile = 32768, kHalf = 16384;
// + dQ staging: two 128 x 32 fp32 blocks (one per column half), 128-byte swizzled
constexpr uint32_t kDqStage = TQ * 32 * 4;  // 16 KB
constexpr size_t kSmem = 1024 + 6 * (size_t)kTile + 2048 + 2 * (size_t)kDqStage;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdArgs {
  const float* lse;     // (B, H, Sq) natural log
  const float* di;      // (B, H, Sq)
  float* dq_acc;        // (B, Sq, H, 128) fp32
  void* dk;             // (B, Skv, Hkv, 128) bf16
  void* dv;
  int B, H, Hkv, Sq, Skv, causal;
  float scale, scale_log2;
  int* err;
  // Stage timestamps of CTA (0, 0) (globaltimer, ns) for pipeline analysis; null
  // in normal runs.  Layout: [event][sub-tile], kTraceT sub-tiles per event.
  unsigned long long* trace;
};

constexpr int kTraceT = 64;
std::atomic<unsigned long long*> g_attn_bwd_trace{nullptr};
enum TraceEv : int {
  kTrProdWait = 0,   // producer: slot free (after qd_free wait)
  kTrProdDone,       // producer: LSE / D staged, arrival done
  kTrSdpIssue,       // MMA: S^T / dP^T issued
  kTrPWait,          // MMA: p_full passed
  kTrAccIssue,       // MMA: dV / dK / dQ^T issued
  kTrSmStart,        // softmax warp 2 lane 0: S^T / dP^T ready
  kTrSmDone,         // softmax: P^T / dS^T written, p_full arrived
  kTrDqStart,        // dQ warp: dQ^T ready
  kTrDqFree,         // dQ warp: TMEM read, dq_free arrived
  kTrDqStaged,       // dQ warp: adds into dq_acc issued
  kTrSdpStart,       // MMA: S^T / dP^T issue begins (its conditions met)
  kTrDvdkStart,      // MMA: dV / dK issue begins
  kTrEvents
};

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void trace_at(const BwdArgs& a, int ev, int t) {
  if (a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && t < kTraceT) a.trace[ev * kTraceT + t] = gtime();
}

// AND of `v` over the 128 threads of named barrier `id` (also a barrier): the
// softmax-gradient warps of one column half leave their loop together, so the
// named barriers of the dQ reduction can never wait for a thread that left.
__device__ __forceinline__ bool group_all(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbar.red.and.pred p, %2, 128, q;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                          const __grid_constant__ CUtensorMap tmdQ, BwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sK = base;
  unsigned char* sV = base + kTile;
  unsigned char* sQ = base + 2 * kTile;
  unsigned char* sdO = base + 3 * kTile;
  unsigned char* sPt = base + 4 * kTile;
  unsigned char* sdSt = base + 5 * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 6 * kTile);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;
  uint64_t* qd_free = bars + 2;
  uint64_t* sdp_ready = bars + 3;
  uint64_t* p_ready = bars + 4;
  uint64_t* dq_ready = bars + 5;
  uint64_t* b_free = bars + 6;
  uint64_t* acc_done = bars + 7;
  uint64_t* drain = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  float* sL = reinterpret_cast<float*>(base + 6 * kTile + 512);  // lse * log2(e) of the tile's queries
  float* sD = sL + TQ;                                             // D = rowsum(dO * O)
  unsigned char* sDQ = base + 6 * kTile + 2048;                    // [2][128 rows x 128 B], swizzled

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TK;
  const int b = blockIdx.y / a.Hkv, hk = blockIdx.y % a.Hkv, G = a.H / a.Hkv;
  const int off = a.Skv - a.Sq;
  const int q_first = a.causal ? max(0, n0 - off) : 0;
  const int qt0 = q_first / TQ;
  const int nqt = q_first < a.Sq ? (a.Sq + TQ - 1) / TQ - qt0 : 0;  // query tiles per head
  const int total = nqt * G;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(qd_full, 32);  // the producer warp: TMA expect-tx by lane 0, LSE/D staging by all lanes
    mbar_init(qd_free, 1);
    mbar_init(sdp_ready, 1);
    mbar_init(p_ready, kSmThreads);
    mbar_init(dq_ready, 1);
    mbar_init(b_free, kSmThreads);
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmdO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tA = tmem, tB = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;

  if (warp == 0) {
    if (total > 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(kv_full, 2 * kTile);
        tma_load_4d(sK, &tmK, kv_full, 0, hk, n0, b);
        tma_load_4d(sK + kHalf, &tmK, kv_full, 64, hk, n0, b);
        tma_load_4d(sV, &tmV, kv_full, 0, hk, n0, b);
        tma_load_4d(sV + kHalf, &tmV, kv_full, 64, hk, n0, b);
      }
      int loaded = 0;
      for (int t = 0; t < total; ++t) {
        const int h = hk * G + t / nqt;
        const int q0 = (qt0 + t % nqt) * TQ;
        // Q/dO and the LSE/D stage are free once the MMAs of tile t-1 that read them completed
        // (the softmax-gradient warps finished with LSE/D before those MMAs were issued).
        if (!__all_sync(0xffffffffu, mbar_wait(qd_free, (t & 1) ^ 1, a.err, kErrTmaWait))) break;
        const float* lse_row = a.lse + ((int64_t)b * a.H + h) * a.Sq;
        const float* di_row = a.di + ((int64_t)b * a.H + h) * a.Sq;
#pragma unroll
        for (int i = 0; i < TQ / 32; ++i) {
          const int c = i * 32 + lane, q = q0 + c;
          sL[c] = q < a.Sq ? lse_row[q] * kLog2e : 0.f;
          sD[c] = q < a.Sq ? di_row[q] : 0.f;
        }
        // every lane arrives after its own stores (release); lane 0 also registers the TMA bytes
        if (lane == 0) {
          mbar_arrive_expect_tx(qd_full, 2 * kTile);
          tma_load_4d(sQ, &tmQ, qd_full, 0, h, q0, b);
          tma_load_4d(sQ + kHalf, &tmQ, qd_full, 64, h, q0, b);
          tma_load_4d(sdO, &tmdO, qd_full, 0, h, q0, b);
          tma_load_4d(sdO + kHalf, &tmdO, qd_full, 64, h, q0, b);
        } else {
          mbar_arrive(qd_full);
        }
        ++loaded;
      }
      if (lane == 0) {
        mbar_wait(kv_full, 0, nullptr, 0);
        if (loaded > 0) mbar_wait(qd_full, (loaded - 1) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && total > 0) {
      constexpr uint32_t id_kk = umma_idesc_f16_major(128, 128, true, false, false);  // both K-major
      constexpr uint32_t id_km = umma_idesc_f16_major(128, 128, true, false, true);   // A K-major, B MN-major
      constexpr uint32_t id_mm = umma_idesc_f16_major(128, 128, true, true, true);    // both MN-major
      const uint32_t k_ = smem_addr(sK), v_ = smem_addr(sV), q_ = smem_addr(sQ), do_ = smem_addr(sdO);
      const uint32_t pt_ = smem_addr(sPt), ds_ = smem_addr(sdSt);
      bool ok = mbar_wait(kv_full, 0, a.err, kErrMmaWait);
      for (int t = 0; t < total && ok; ++t) {
        const uint32_t par = t & 1;
        if (!mbar_wait(qd_full, par, a.err, kErrMmaWait)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {  // S^T = K Q^T
          const uint32_t o = (k >> 2) * kHalf + (k & 3) * 32;
          umma_f16(tA, umma_desc_k_sw128(k_ + o), umma_desc_k_sw128(q_ + o), id_kk, k != 0);
        }
        // dP^T goes to region B, which holds dQ_{t-1} until the epilogue read it.
        if (t > 0 && !mbar_wait(b_free, par ^ 1, a.err, kErrMmaWait)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {  // dP^T = V dO^T
          const uint32_t o = (k >> 2) * kHalf + (k & 3) * 32;
          umma_f16(tB, umma_desc_k_sw128(v_ + o), umma_desc_k_sw128(do_ + o), id_kk, k != 0);
        }
        umma_commit(sdp_ready);
        if (!mbar_wait(p_ready, par, a.err, kErrMmaWait)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < TQ / 16; ++k) {  // dV += P^T dO ; dK += dS^T Q
          const uint32_t o = (k >> 2) * kHalf + (k & 3) * 32;
          umma_f16(tdV, umma_desc_k_sw128(pt_ + o), umma_desc_mn_sw128(do_ + k * 2048, kHalf, 1024), id_km,
                   (t | k) != 0);
          umma_f16(tdK, umma_desc_k_sw128(ds_ + o), umma_desc_mn_sw128(q_ + k * 2048, kHalf, 1024), id_km,
                   (t | k) != 0);
        }
        umma_commit(qd_free);  // Q, dO (and LSE/D) no longer needed: the next tile's loads overlap dQ
#pragma unroll
        for (int k = 0; k < TK / 16; ++k)  // dQ = dS K   (dS = (dS^T)^T read MN-major)
          umma_f16(tB, umma_desc_mn_sw128(ds_ + k * 2048, kHalf, 1024),
                   umma_desc_mn_sw128(k_ + k * 2048, kHalf, 1024), id_mm, k != 0);
        umma_commit(dq_ready);
      }
      umma_commit(acc_done);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------ softmax-gradient warps
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;         // TMEM lane: key row (S^T, dP^T, dK, dV) / query row (dQ)
    const int key = n0 + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int c0 = half * 64;
    bool ok = true;
    for (int t = 0; t < total && ok; ++t) {
      const uint32_t par = t & 1;
      const int h = hk * G + t / nqt;
      const int q0 = (qt0 + t % nqt) * TQ;
      bool got = mbar_wait(sdp_ready, par, a.err, kErrEpiWait);
      // acquire the producer's LSE/D stores (its phase completed before the MMAs that signalled sdp_ready)
      got = got && mbar_wait(qd_full, par, a.err, kErrEpiWait);
      if (!group_all(2 + half, got)) { ok = false; break; }
      tc_fence_after();
      // two passes of 32 query columns; each pass fills four 16-byte chunks of this
      // thread's 128-byte row of the 64-column swizzle block of P^T / dS^T
#pragma unroll 1
      for (int pass = 0; pass < 2; ++pass) {
        const int cb = c0 + pass * 32;
        float s[32], dp[32];
        tmem_ld_32x32b_x32(tA + lane_base + cb, reinterpret_cast<uint32_t*>(s));
        tmem_ld_32x32b_x32(tB + lane_base + cb, reinterpret_cast<uint32_t*>(dp));
        tmem_ld_wait();
        uint32_t pp[16], dd[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float pv[2], dv2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int q = q0 + cb + i + e;
            const bool valid = q < a.Sq && key < a.Skv && (!a.causal || key <= q + off);
            const float p = valid ? fast_exp2(s[i + e] * a.scale_log2 - sL[cb + i + e]) : 0.f;
            pv[e] = p;
            dv2[e] = p * (dp[i + e] - sD[cb + i + e]);
          }
          pp[i / 2] = pack2(pv[0], pv[1]);
          dd[i / 2] = pack2(dv2[0], dv2[1]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = pass * 4 + j;
          const uint32_t so = half * kHalf + row * 128 + ((ch ^ (row & 7)) * 16);
          *reinterpret_cast<uint4*>(sPt + so) = make_uint4(pp[j * 4], pp[j * 4 + 1], pp[j * 4 + 2], pp[j * 4 + 3]);
          *reinterpret_cast<uint4*>(sdSt + so) = make_uint4(dd[j * 4], dd[j * 4 + 1], dd[j * 4 + 2], dd[j * 4 + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_ready);
      // dQ rows: TMEM lane = query row of this tile.  Both 32-column blocks of this
      // thread's half come out of TMEM first, so region B is released before the
      // reduction; each block is staged (x scale) in the half's swizzled buffer and
      // added to dq_acc by one TMA reduce-add (rows past Sq hold exact zeros).
      if (!group_all(2 + half, mbar_wait(dq_ready, par, a.err, kErrEpiWait))) { ok = false; break; }
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(tB + lane_base + c0, r0);
      tmem_ld_32x32b_x32(tB + lane_base + c0 + 32, r1);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(b_free);
      unsigned char* stg = sDQ + half * kDqStage;
      const bool issuer = quarter == 0 && lane == 0;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        // the previous reduce-add from this buffer has finished reading it
        if (issuer) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        asm volatile("bar.sync %0, 128;" ::"r"(2 + half) : "memory");
        const uint32_t* r = c == 0 ? r0 : r1;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(stg + row * 128 + ((j ^ (row & 7)) * 16)) =
              make_float4(__uint_as_float(r[4 * j]) * a.scale, __uint_as_float(r[4 * j + 1]) * a.scale,
                          __uint_as_float(r[4 * j + 2]) * a.scale, __uint_as_float(r[4 * j + 3]) * a.scale);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("bar.sync %0, 128;" ::"r"(2 + half) : "memory");
        if (issuer) {
          asm volatile(
              "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(&tmdQ),
              "r"(smem_addr(stg)), "r"(h * HD + c0 + c * 32), "r"(b * a.Sq + q0)
              : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
    }
    if (quarter == 0 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    // ---------------------------------------------------------- dK, dV
    const bool have = __all_sync(0xffffffffu, ok && total > 0 && mbar_wait(acc_done, 0, a.err, kErrEpiWait));
    tc_fence_after();
    __nv_bfloat16* dkp = reinterpret_cast<__nv_bfloat16*>(a.dk) + (((int64_t)b * a.Skv + key) * a.Hkv + hk) * HD + c0;
    __nv_bfloat16* dvp = reinterpret_cast<__nv_bfloat16*>(a.dv) + (((int64_t)b * a.Skv + key) * a.Hkv + hk) * HD + c0;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t rk[32], rv[32];
      if (have) {
        tmem_ld_32x32b_x32(tdK + lane_base + c0 + c * 32, rk);
        tmem_ld_32x32b_x32(tdV + lane_base + c0 + c * 32, rv);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) rk[e] = rv[e] = 0u;
      }
      if (key >= a.Skv) continue;
#pragma unroll
      for (int e = 0; e < 32; e += 8) {
        *reinterpret_cast<uint4*>(dkp + c * 32 + e) = make_uint4(
            pack2(__uint_as_float(rk[e]) * a.scale, __uint_as_float(rk[e + 1]) * a.scale),
            pack2(__uint_as_float(rk[e + 2]) * a.scale, __uint_as_float(rk[e + 3]) * a.scale),
            pack2(__uint_as_float(rk[e + 4]) * a.scale, __uint_as_float(rk[e + 5]) * a.scale),
            pack2(__uint_as_float(rk[e + 6]) * a.scale, __uint_as_float(rk[e + 7]) * a.scale));
        *reinterpret_cast<uint4*>(dvp + c * 32 + e) = make_uint4(
            pack2(__uint_as_float(rv[e]), __uint_as_float(rv[e + 1])),
            pack2(__uint_as_float(rv[e + 2]), __uint_as_float(rv[e + 3])),
            pack2(__uint_as_float(rv[e + 4]), __uint_as_float(rv[e + 5])),
            pack2(__uint_as_float(rv[e + 6]), __uint_as_float(rv[e + 7])));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------ v3: 64-query sub-tiles
// CTA = (batch, kv-head, 128 keys); query sub-tiles of 64 rows.  TMEM (512 columns):
//   S^T_b  [b*128, b*128+64)   keys x 64 queries, later dQ^T_b (hd x 64 queries)
//   dP^T_b [b*128+64, b*128+128)
//   dV [256, 384), dK [384, 512)
// dQ^T = K^T dS^T is written over S^T_b once the softmax warps have read it,
// so dQ needs no columns of its own.  TMEM and the P^T / dS^T tiles are
// double-buffered (b = t & 1); Q, dO and their LSE / D rows sit in a ring of
// three slots (t % 3), so the producer fills sub-tile t+2 while t and t+1 are in
// use and no refill (TMA or the LSE / D loads) lies between the MMAs of one
// sub-tile and the next.  Per sub-tile the MMAs run dQ^T first, then dV / dK;
// the dQ epilogue reads dQ^T out of TMEM (freeing the columns for the next
// S^T of the buffer) and adds it into the fp32 dQ buffer straight from
// registers (red.global.add, one coalesced 128-byte line per warp and query):
// no shared-memory staging, so the epilogue holds no slot and no tile that
// the next sub-tiles need.  The softmax warps of sub-tile t+2 wait for
// pd_read(t) (the dV / dK MMAs, the last readers of the P^T / dS^T tiles)
// before they rewrite them.  Warps: 0 TMA, 1 MMA issue, 2..9 softmax-gradient
// (two threads per key row, 32 queries each), 10..13 dQ epilogue (one thread
// per head-dim lane).
namespace bwd3 {
constexpr int TQ3 = 64;
constexpr int kThreads = 448;
constexpr int kRing = 3;                            // Q / dO slots
constexpr uint32_t kKV = 32768, kKVHalf = 16384;   // K or V tile, 64-column half
constexpr uint32_t kQ = 16384, kQHalf = 8192;       // Q or dO sub-tile, half
constexpr uint32_t kPT = 16384;                     // P^T or dS^T: 128 keys x 64 queries
constexpr uint32_t kPD = 2 * kPT;                   // [P^T | dS^T] of one buffer; also the dQ staging:
                                                    // 4 boxes of 32 head dims x 64 queries (fp32)
constexpr size_t kSmem = 1024 + 2 * kKV + 2 * kRing * (size_t)kQ + 2 * (size_t)kPD + 2048;
static_assert(kSmem <= 232448, "attention backward: shared memory over the 227 KB limit");
constexpr int kHeadGroup = 8;  // (batch, kv-head) pairs per launch group
}  // namespace bwd3

__global__ void __launch_bounds__(bwd3::kThreads, 1)
    attn_bwd_v3_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO, BwdArgs a) {
  using namespace bwd3;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sK = base;
  unsigned char* sV = base + kKV;
  unsigned char* sQ = base + 2 * kKV;              // [kRing]
  unsigned char* sdO = sQ + kRing * kQ;            // [kRing]
  unsigned char* sPD = sdO + kRing * kQ;           // [2] x (P^T | dS^T), later the dQ staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(sPD + 2 * kPD);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;     // [kRing]
  uint64_t* qd_free = bars + 4;     // [kRing]
  uint64_t* sdp_full = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;      // [2]
  uint64_t* dq_full = bars + 11;    // [2]
  uint64_t* dq_free = bars + 13;    // [2]
  uint64_t* acc_done = bars + 17;
  uint64_t* drain = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  uint64_t* pd_read = bars + 22;    // [2] dV / dK MMAs of the buffer done: P^T / dS^T consumed
  float* sL = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(bars) + 512);  // [kRing][64]
  float* sD = sL + kRing * TQ3;                                                       // [kRing][64]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid over (head group, key tile, head in group): groups of kHeadGroup
  // (batch, kv-head) pairs run one after another, so the CTAs in flight add
  // their dQ into a few heads' rows (an L2-resident working set), and within a
  // group the key tiles launch in ascending order -- under a causal mask the
  // longest first, the short ones filling the tail
  int n0, b, hk;
  {
    const int bh = a.B * a.Hkv, nkt = (a.Skv + TK - 1) / TK;
    const int grp = (int)blockIdx.x / (kHeadGroup * nkt);
    const int r = (int)blockIdx.x - grp * kHeadGroup * nkt;
    const int gs = min(kHeadGroup, bh - grp * kHeadGroup);
    n0 = (r / gs) * TK;
    const int head = grp * kHeadGroup + r % gs;
    b = head / a.Hkv;
    hk = head % a.Hkv;
  }
  const int G = a.H / a.Hkv;
  const int off = a.Skv - a.Sq;
  const int q_first = a.causal ? max(0, n0 - off) : 0;
  const int qt0 = q_first / TQ3;
  const int nqt = q_first < a.Sq ? (a.Sq + TQ3 - 1) / TQ3 - qt0 : 0;
  const int total = nqt * G;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&qd_full[i], 32);
      mbar_init(&qd_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sdp_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_free[i], 128);
      mbar_init(&pd_read[i], 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmdO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tdV = tmem + 256, tdK = tmem + 384;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (total > 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(kv_full, 2 * kKV);
        tma_load_4d(sK, &tmK, kv_full, 0, hk, n0, b);
        tma_load_4d(sK + kKVHalf, &tmK, kv_full, 64, hk, n0, b);
        tma_load_4d(sV, &tmV, kv_full, 0, hk, n0, b);
        tma_load_4d(sV + kKVHalf, &tmV, kv_full, 64, hk, n0, b);
      }
      int loaded = 0;
      for (int t = 0; t < total; ++t) {
        const int sl = t % kRing;
        const uint32_t use = (uint32_t)(t / kRing) & 1;
        const int h = hk * G + t / nqt;
        const int q0 = (qt0 + t % nqt) * TQ3;
        if (!__all_sync(0xffffffffu, mbar_wait(&qd_free[sl], use ^ 1, a.err, kErrTmaWait))) break;
        if (lane == 0) trace_at(a, kTrProdWait, t);
        if (lane == 0) {
          mbar_expect_tx(&qd_full[sl], 2 * kQ);  // the 32 arrivals come after the LSE / D staging
          unsigned char* q_ = sQ + sl * kQ;
          unsigned char* o_ = sdO + sl * kQ;
          tma_load_4d(q_, &tmQ, &qd_full[sl], 0, h, q0, b);
          tma_load_4d(q_ + kQHalf, &tmQ, &qd_full[sl], 64, h, q0, b);
          tma_load_4d(o_, &tmdO, &qd_full[sl], 0, h, q0, b);
          tma_load_4d(o_ + kQHalf, &tmdO, &qd_full[sl], 64, h, q0, b);
        }
        const float* lse_row = a.lse + ((int64_t)b * a.H + h) * a.Sq;
        const float* di_row = a.di + ((int64_t)b * a.H + h) * a.Sq;
#pragma unroll
        for (int i = 0; i < TQ3 / 32; ++i) {
          const int c = i * 32 + lane, q = q0 + c;
          sL[sl * TQ3 + c] = q < a.Sq ? -lse_row[q] * kLog2e : 0.f;  // negated: P = 2^(s * scale_log2 + L)
          sD[sl * TQ3 + c] = q < a.Sq ? di_row[q] : 0.f;
        }
        mbar_arrive(&qd_full[sl]);  // release: the LSE / D rows above are visible to the waiters
        if (lane == 0) trace_at(a, kTrProdDone, t);
        ++loaded;
      }
      if (lane == 0) {
        mbar_wait(kv_full, 0, nullptr, 0);
        for (int i = 1; i <= kRing && i <= loaded; ++i) {
          const int t = loaded - i;
          mbar_wait(&qd_full[t % kRing], (uint32_t)(t / kRing) & 1, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0 && total > 0) {
      constexpr uint32_t id_sdp = umma_idesc_f16_major(128, TQ3, true, false, false);  // K-major A, B
      constexpr uint32_t id_acc = umma_idesc_f16_major(128, 128, true, false, true);   // A K-major, B MN-major
      constexpr uint32_t id_dq = umma_idesc_f16_major(128, TQ3, true, true, true);     // both MN-major
      const uint32_t k_ = smem_addr(sK), v_ = smem_addr(sV);
      bool ok = mbar_wait(kv_full, 0, a.err, kErrMmaWait);
      // Event-driven issue: the thread polls the conditions of three pending
      // steps and issues whichever is ready first in priority order.  Steps:
      //   dQ^T of sub-tile nd: its P^T / dS^T are written (p_full);
      //   S^T / dP^T of sub-tile ns: its Q / dO slot landed and the dQ^T of
      //     sub-tile ns-2 (same TMEM buffer) has been read out (dq_free);
      //   dV / dK of sub-tile nv (after its dQ^T).
      // Descriptors are built once and advanced by integer adds (desc_add): the
      // issuing thread shares its SM sub-partition with softmax warps, so every
      // instruction it saves shortens the issue of a sub-tile's 32 MMAs.
      const uint64_t dK = umma_desc_k_sw128(k_), dV = umma_desc_k_sw128(v_);
      const uint64_t dKmn = umma_desc_mn_sw128(k_, kKVHalf, 1024);
      const uint64_t dQ0 = umma_desc_k_sw128(smem_addr(sQ)), dO0 = umma_desc_k_sw128(smem_addr(sdO));
      const uint64_t dQmn0 = umma_desc_mn_sw128(smem_addr(sQ), kQHalf, 1024);
      const uint64_t dOmn0 = umma_desc_mn_sw128(smem_addr(sdO), kQHalf, 1024);
      const uint64_t dPt0 = umma_desc_k_sw128(smem_addr(sPD));
      const uint64_t dDsmn0 = umma_desc_mn_sw128(smem_addr(sPD) + kPT, kPT, 1024);
      auto issue_sdp = [&](int t) {
        trace_at(a, kTrSdpStart, t);
        const int bb = t & 1, sl = t % kRing;
        const uint64_t dq = desc_add(dQ0, sl * kQ), dop = desc_add(dO0, sl * kQ);
        const uint32_t tS = tmem + bb * 128, tP = tS + 64;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t ka = (k >> 2) * kKVHalf + (k & 3) * 32, kb = (k >> 2) * kQHalf + (k & 3) * 32;
          umma_f16(tS, desc_add(dK, ka), desc_add(dq, kb), id_sdp, k != 0);
          umma_f16(tP, desc_add(dV, ka), desc_add(dop, kb), id_sdp, k != 0);
        }
        umma_commit(&sdp_full[bb]);
        trace_at(a, kTrSdpIssue, t);
      };
      // dQ^T = K^T dS^T of sub-tile t, into the consumed S^T_b columns
      auto issue_dq = [&](int t) {
        const int bb = t & 1;
        const uint64_t dsmn = desc_add(dDsmn0, bb * kPD);
#pragma unroll
        for (int k = 0; k < TK / 16; ++k)
          umma_f16(tmem + bb * 128, desc_add(dKmn, k * 2048), desc_add(dsmn, k * 2048), id_dq, k != 0);
        umma_commit(&dq_full[bb]);
      };
      // dV += P^T dO ; dK += dS^T Q of sub-tile t
      auto issue_dvdk = [&](int t) {
        trace_at(a, kTrDvdkStart, t);
        const int bb = t & 1, sl = t % kRing;
        const uint64_t qmn = desc_add(dQmn0, sl * kQ), omn = desc_add(dOmn0, sl * kQ);
        const uint64_t pt = desc_add(dPt0, bb * kPD), ds = desc_add(dPt0, bb * kPD + kPT);
        const uint32_t first = t != 0;
#pragma unroll
        for (int k = 0; k < TQ3 / 16; ++k) {
          umma_f16(tdV, desc_add(pt, k * 32), desc_add(omn, k * 2048), id_acc, k != 0 ? 1u : first);
          umma_f16(tdK, desc_add(ds, k * 32), desc_add(qmn, k * 2048), id_acc, k != 0 ? 1u : first);
        }
        umma_commit(&qd_free[sl]);
        umma_commit(&pd_read[bb]);
        trace_at(a, kTrAccIssue, t);
      };
      // Issue order: dQ^T(t) as soon as its softmax is done, dV / dK(t) right
      // behind it (the softmax of t+2 waits for them, pd_read), then S^T / dP^T.
      // Queuing S^T(t+2) ahead of dV / dK(t) measured slower: it lengthens the
      // chain to the softmax of t+2 by the dV / dK MMAs.
      int ns = 0, nd = 0, nv = 0;
      uint32_t idle = 0;
      uint64_t idle_since = 0;
      while (ok && nv < total) {
        bool did = false;
        if (nd < ns && mbar_test(&p_full[nd & 1], ((uint32_t)nd >> 1) & 1)) {
          trace_at(a, kTrPWait, nd);
          tc_fence_after();
          issue_dq(nd++);
          did = true;
        } else if (nv < nd) {
          issue_dvdk(nv++);
          did = true;
        } else if (ns < total && ns <= nd + 1 && mbar_test(&qd_full[ns % kRing], (uint32_t)(ns / kRing) & 1) &&
                   (ns < 2 || mbar_test(&dq_free[ns & 1], (((uint32_t)ns >> 1) & 1) ^ 1))) {
          tc_fence_after();
          issue_sdp(ns++);
          did = true;
        }
        // polls return at once; every 1024 idle polls the wall-time bound and the
        // error word (another role gave up) are checked
        if (did) {
          idle = 0;
        } else if ((++idle & 1023u) == 0) {
          const uint64_t now = global_ns();
          if (idle == 1024u) idle_since = now;
          if (*reinterpret_cast<volatile int*>(a.err) != 0) {
            ok = false;  // another role gave up: stop issuing
          } else if (now - idle_since > kWaitLimitNs) {
            record_error(a.err, kErrMmaWait);
            ok = false;
          }
        }
      }
      umma_commit(acc_done);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else if (warp < 10) {
    // ------------------------------------------------- softmax-gradient warps
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;  // key row within the tile (TMEM lane)
    const int key = n0 + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int c0 = half * 32;
    bool ok = true;
    for (int t = 0; t < total && ok; ++t) {
      const int bb = t & 1, sl = t % kRing;
      const uint32_t use = (t >> 1) & 1;
      const int q0 = (qt0 + t % nqt) * TQ3;
      // S^T / dP^T in TMEM, the LSE / D rows, and (from t = 2) the MMAs that last
      // read this buffer's P^T / dS^T tiles
      if (!mbar_wait(&sdp_full[bb], use, a.err, kErrEpiWait) ||
          !mbar_wait(&qd_full[sl], (uint32_t)(t / kRing) & 1, a.err, kErrEpiWait) ||
          (t >= 2 && !mbar_wait(&pd_read[bb], use ^ 1, a.err, kErrEpiWait))) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) trace_at(a, kTrSmStart, t);
      tc_fence_after();
      float s[32], dp[32];
      tmem_ld_32x32b_x32(tmem + lane_base + bb * 128 + c0, reinterpret_cast<uint32_t*>(s));
      tmem_ld_32x32b_x32(tmem + lane_base + bb * 128 + 64 + c0, reinterpret_cast<uint32_t*>(dp));
      tmem_ld_wait();
      const float* L = sL + sl * TQ3 + c0;  // -LSE * log2(e)
      const float* Dd = sD + sl * TQ3 + c0;
      uint32_t pp[16], dd[16];
      // warp-uniform: all 32 keys x 32 queries of this warp are valid (inside the
      // sequences and on or below the causal diagonal) -- no per-element masks
      const int key_hi = n0 + quarter * 32 + 31, qlo = q0 + c0;
      const bool full = qlo + 32 <= a.Sq && key_hi < a.Skv && (!a.causal || key_hi <= qlo + off);
      if (full) {
        const uint64_t sc2 = f2_pack(a.scale_log2, a.scale_log2);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const uint64_t l2 = *reinterpret_cast<const uint64_t*>(L + i);
          const uint64_t d2 = *reinterpret_cast<const uint64_t*>(Dd + i);
          const float2 x = f2_unpack(f2_fma(f2_pack(s[i], s[i + 1]), sc2, l2));
          const float p0 = fast_exp2(x.x), p1 = fast_exp2(x.y);
          const float2 g = f2_unpack(f2_mul(f2_pack(p0, p1), f2_sub(f2_pack(dp[i], dp[i + 1]), d2)));
          pp[i / 2] = pack2(p0, p1);
          dd[i / 2] = pack2(g.x, g.y);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float pv[2], dv2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int q = qlo + i + e;
            const bool valid = q < a.Sq && key < a.Skv && (!a.causal || key <= q + off);
            const float p = valid ? fast_exp2(fmaf(s[i + e], a.scale_log2, L[i + e])) : 0.f;
            pv[e] = p;
            dv2[e] = p * (dp[i + e] - Dd[i + e]);
          }
          pp[i / 2] = pack2(pv[0], pv[1]);
          dd[i / 2] = pack2(dv2[0], dv2[1]);
        }
      }
      unsigned char* pt = sPD + bb * kPD;
      unsigned char* ds = pt + kPT;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int ch = half * 4 + j;
        const uint32_t so = row * 128 + ((ch ^ (row & 7)) * 16);
        *reinterpret_cast<uint4*>(pt + so) = make_uint4(pp[j * 4], pp[j * 4 + 1], pp[j * 4 + 2], pp[j * 4 + 3]);
        *reinterpret_cast<uint4*>(ds + so) = make_uint4(dd[j * 4], dd[j * 4 + 1], dd[j * 4 + 2], dd[j * 4 + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[bb]);
      if (warp == 2 && lane == 0) trace_at(a, kTrSmDone, t);
    }
    // ---------------------------------------------------------- dK, dV
    const bool have = __all_sync(0xffffffffu, ok && total > 0 && mbar_wait(acc_done, 0, a.err, kErrEpiWait));
    tc_fence_after();
    const int cc = half * 64;
    __nv_bfloat16* dkp = reinterpret_cast<__nv_bfloat16*>(a.dk) + (((int64_t)b * a.Skv + key) * a.Hkv + hk) * HD + cc;
    __nv_bfloat16* dvp = reinterpret_cast<__nv_bfloat16*>(a.dv) + (((int64_t)b * a.Skv + key) * a.Hkv + hk) * HD + cc;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t rk[32], rv[32];
      if (have) {
        tmem_ld_32x32b_x32(tdK + lane_base + cc + c * 32, rk);
        tmem_ld_32x32b_x32(tdV + lane_base + cc + c * 32, rv);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) rk[e] = rv[e] = 0u;
      }
      if (key >= a.Skv) continue;
#pragma unroll
      for (int e = 0; e < 32; e += 8) {
        *reinterpret_cast<uint4*>(dkp + c * 32 + e) = make_uint4(
            pack2(__uint_as_float(rk[e]) * a.scale, __uint_as_float(rk[e + 1]) * a.scale),
            pack2(__uint_as_float(rk[e + 2]) * a.scale, __uint_as_float(rk[e + 3]) * a.scale),
            pack2(__uint_as_float(rk[e + 4]) * a.scale, __uint_as_float(rk[e + 5]) * a.scale),
            pack2(__uint_as_float(rk[e + 6]) * a.scale, __uint_as_float(rk[e + 7]) * a.scale));
        *reinterpret_cast<uint4*>(dvp + c * 32 + e) = make_uint4(
            pack2(__uint_as_float(rv[e]), __uint_as_float(rv[e + 1])),
            pack2(__uint_as_float(rv[e + 2]), __uint_as_float(rv[e + 3])),
            pack2(__uint_as_float(rv[e + 4]), __uint_as_float(rv[e + 5])),
            pack2(__uint_as_float(rv[e + 6]), __uint_as_float(rv[e + 7])));
      }
    }
  } else {
    // ------------------------------------------------------- dQ epilogue
    // dQ^T leaves TMEM (lane = head dim d, 64 query columns) and is added x scale
    // into dq_acc with red.global.add: for one query the 32 lanes of a warp
    // cover 32 consecutive head dims, one 128-byte line.
    const int quarter = warp & 3;
    const int d = quarter * 32 + lane;  // head-dim index (TMEM lane of dQ^T)
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const bool issuer = quarter == 0 && lane == 0;
    for (int t = 0; t < total; ++t) {
      const int bb = t & 1;
      const uint32_t use = (t >> 1) & 1;
      const int h = hk * G + t / nqt;
      const int q0 = (qt0 + t % nqt) * TQ3;
      // dq_full: dQ^T(t) is in TMEM
      if (!mbar_wait(&dq_full[bb], use, a.err, kErrEpiWait)) break;
      if (issuer) trace_at(a, kTrDqStart, t);
      tc_fence_after();
      uint32_t r[64];
      tmem_ld_32x32b_x32(tmem + lane_base + bb * 128, r);  // both loads in flight, one wait
      tmem_ld_32x32b_x32(tmem + lane_base + bb * 128 + 32, r + 32);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&dq_free[bb]);  // dQ^T is in registers: the MMAs may reuse the columns
      if (issuer) trace_at(a, kTrDqFree, t);
      float* dst = a.dq_acc + (((int64_t)b * a.Sq + q0) * a.H + h) * HD + d;
      const int64_t qstride = (int64_t)a.H * HD;
      const int nq = min(TQ3, a.Sq - q0);
      if (nq == TQ3) {
#pragma unroll
        for (int e = 0; e < TQ3; ++e) atomicAdd(dst + e * qstride, __uint_as_float(r[e]) * a.scale);
      } else {
#pragma unroll
        for (int e = 0; e < TQ3; ++e)
          if (e < nq) atomicAdd(dst + e * qstride, __uint_as_float(r[e]) * a.scale);
      }
      if (issuer) trace_at(a, kTrDqStaged, t);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
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

CUtensorMap bshd_map(const at::Tensor& t, int box_rows = 128) {
  CUtensorMap m;
  const cuuint64_t dims[4] = {(cuuint64_t)t.size(3), (cuuint64_t)t.size(2), (cuuint64_t)t.size(1),
                              (cuuint64_t)t.size(0)};
  const cuuint64_t strides[3] = {(cuuint64_t)t.stride(2) * 2, (cuuint64_t)t.stride(1) * 2, (cuuint64_t)t.stride(0) * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return m;
}

// dq_acc viewed as (rows = B*Sq, cols = H*128) fp32; box 32 columns x 128 rows, 128-byte swizzle.
CUtensorMap dq_map(float* ptr, int64_t rows, int64_t cols, int box_rows = TQ) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (dq) failed with code ", (int)r);
  return m;
}

// Error words of this file's kernels: module globals (one copy per device).
DeviceWord g_attn_bwd_err_word{g_attn_bwd_err, {}};

int* bwd_error_word(const at::Device& dev) { return g_attn_bwd_err_word.get(dev.index()); }

}  // namespace

// dK, dV (bf16) and dq_acc (fp32, must be zero-initialised; receives scale * dS K)
void attn_bwd_sm100(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                    const at::Tensor& lse, const at::Tensor& di, at::Tensor& dq_acc, at::Tensor& dk, at::Tensor& dv,
                    bool causal, double scale) {
  c10::cuda::CUDAGuard g(q.device());
  bind_device(q.get_device());
  const int64_t B = q.size(0), Sq = q.size(1), H = q.size(2), Skv = k.size(1), Hkv = k.size(2);
  if (B * Skv * Hkv == 0) return;
  CUtensorMap tq = bshd_map(q), tk = bshd_map(k), tv = bshd_map(v), tdo = bshd_map(dout);
  BwdArgs args{lse.data_ptr<float>(), di.data_ptr<float>(), dq_acc.data_ptr<float>(), dk.data_ptr(), dv.data_ptr(),
               (int)B, (int)H, (int)Hkv, (int)Sq, (int)Skv, causal ? 1 : 0, (float)scale, (float)scale * kLog2e,
               bwd_error_word(q.device()), g_attn_bwd_trace.load(std::memory_order_acquire)};
  // The 64-query double-buffered kernel is the default; LRB_ATTN_BWD_V2=1 selects
  // the 128-query kernel that runs its tiles one after another.
  static const bool v2 = [] {
    const char* e = std::getenv("LRB_ATTN_BWD_V2");
    return e != nullptr && e[0] == '1';
  }();
  dim3 grid((unsigned)((Skv + TK - 1) / TK), (unsigned)(B * Hkv));
  LRB_CHECK(dq_acc.is_contiguous() && dq_acc.scalar_type() == at::kFloat && dq_acc.numel() == B * Sq * H * HD,
            "attn_bwd: dq_acc must be a contiguous fp32 (B, Sq, H, 128) buffer");
  if (v2) {  // 128-query tiles, serial per tile
    CUtensorMap tdq = dq_map(dq_acc.data_ptr<float>(), B * Sq, H * HD);
    LRB_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    attn_bwd_sm100_kernel<<<grid, kThreads, kSmem, stream()>>>(tq, tk, tv, tdo, tdq, args);
  } else {
    CUtensorMap tq64 = bshd_map(q, bwd3::TQ3), tdo64 = bshd_map(dout, bwd3::TQ3);
    LRB_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_v3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)bwd3::kSmem));
    LRB_CHECK(B * Hkv * ((Skv + TK - 1) / TK) < (1LL << 31), "attn_bwd: too many CTAs");
    const dim3 grid3((unsigned)(B * Hkv * ((Skv + TK - 1) / TK)));
    attn_bwd_v3_kernel<<<grid3, bwd3::kThreads, bwd3::kSmem, stream()>>>(tq64, tk, tv, tdo64, args);
  }
  LRB_LAUNCH_CHECK();
}

// Stage timestamps of the next backward launches go to `buf` (int64, at least
// kTrEvents * kTraceT entries) -- a pipeline-analysis hook; None switches it off.
void attn_bwd_set_trace(const c10::optional<at::Tensor>& buf) {
  if (buf) {
    LRB_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong && buf->is_contiguous() &&
                  buf->numel() >= (int64_t)kTrEvents * kTraceT,
              "attn_bwd_set_trace: an int64 CUDA buffer of ", (int64_t)kTrEvents * kTraceT, " entries");
    g_attn_bwd_trace.store(reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>()), std::memory_order_release);
  } else {
    g_attn_bwd_trace.store(nullptr, std::memory_order_release);
  }
}

int64_t attn_bwd_sm100_error(int64_t device) { return g_attn_bwd_err_word.take((int)device); }

}  // namespace lrb
