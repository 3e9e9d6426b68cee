// Flash-attention forward on tcgen05 / TMEM for head_dim 128 (bf16, fp32
// softmax statistics), causal or not, grouped-query heads read in place.
//
// CTA = one (batch, head, 128-query tile), 10 warps:
//   warp 0      TMA: Q once (two 64-column swizzled boxes), then K and V
//               tiles of 128 keys into 2-stage rings;
//   warp 1      TMEM owner + MMA issue (one thread):
//                 S_j = Q K_j^T   -> TMEM columns [128*(j%2), +128)  (two S buffers)
//                 O  += P_j V_j   -> TMEM columns [256, 384)
//               P_j is read from shared memory (K-major, 128-B swizzle); V is
//               the MN-major B operand straight from its TMA tile;
//   warps 2..9  softmax, two threads per query row (its TMEM lane): warps
//               2..5 own key/head-dim columns 0..63, warps 6..9 columns
//               64..127 of the same lanes; the row max is exchanged through
//               shared memory behind an mbarrier.  Each thread reads its half
//               of S_j, masks, keeps a running max / sum in the exp2 domain
//               (SFU ex2), writes its 64-key block of P_j (bf16) to shared
//               memory, rescales its half of the O row in TMEM when the row
//               max grew by more than 2^8 (lazy rescaling keeps exponents
//               bounded by 256), and finally normalises and stores its half of
//               O; the row log-sum-exp combines both partial sums.
// S_{j+1} is computed while the softmax of tile j runs, and P_j V_j while the
// softmax of tile j+1 runs.  All waits are bounded (sm100.cuh).
#include "../common.cuh"
#include "sm100.cuh"

#include <cstdlib>

namespace lrb {

__device__ int g_attn_fwd_err[4];
namespace {

using namespace sm100;

constexpr int TQ = 128, TK = 128, HD = 128;
// 2 control warps + 8 softmax warps: two threads per query row, each owning 64
// of the 128 key columns of S (and 64 of the 128 columns of O).
constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 256;
constexpr uint32_t kTileBytes = TQ * HD * 2;  // 32 KB: one Q/K/V/P tile
constexpr uint32_t kHalf = kTileBytes / 2;    // 16 KB: one 64-column swizzle block
constexpr size_t kSmem = 1024 + 6 * (size_t)kTileBytes + 512 + 4 * TQ * sizeof(float) + 2 * TQ * sizeof(float);
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FwdArgs {
  void* out;     // (B, Sq, H, 128) contiguous
  float* lse;    // (B, H, Sq)
  int B, H, Hkv, Sq, Skv, causal;
  float scale_log2;
  int* err;
};

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, FwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base;
  unsigned char* sK = base + kTileBytes;       // 2 stages
  unsigned char* sV = base + 3 * kTileBytes;   // 2 stages
  unsigned char* sP = base + 5 * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 6 * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* v_full = bars + 3;   // [2]
  uint64_t* k_free = bars + 5;   // [2]
  uint64_t* v_free = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_free = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;
  uint64_t* o_done = bars + 14;
  uint64_t* drain = bars + 15;
  uint64_t* xbar = bars + 16;    // [2 parity][4 quarter]: row-max exchange between paired warps
  uint64_t* sbar = bars + 24;    // [4 quarter]: row-sum exchange
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 32);
  float* xmax = reinterpret_cast<float*>(base + 6 * kTileBytes + 512);  // [2 parity][2 half][TQ]
  float* xsum = xmax + 4 * TQ;                                          // [2 half][TQ]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = gridDim.x - 1 - blockIdx.x;  // heavy (late) causal tiles first
  const int m0 = mt * TQ;
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H, hk = h / (a.H / a.Hkv);
  const int off = a.Skv - a.Sq;
  int kv_end = a.Skv;
  if (a.causal) kv_end = min(kv_end, m0 + TQ + off);
  const int nt = kv_end > 0 ? (kv_end + TK - 1) / TK : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_free[i], 1);
      mbar_init(&v_free[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kSoftmaxThreads);
    }
    mbar_init(p_full, kSoftmaxThreads);
    for (int i = 0; i < 8; ++i) mbar_init(&xbar[i], 64);
    for (int i = 0; i < 4; ++i) mbar_init(&sbar[i], 64);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0 && nt > 0) {
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_4d(sQ, &tmQ, q_full, 0, h, m0, b);
      tma_load_4d(sQ + kHalf, &tmQ, q_full, 64, h, m0, b);
      int armed_k = 0, armed_v = 0;
      for (int j = 0; j < nt; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_free[st], ph ^ 1, a.err, kErrTmaWait)) break;
        mbar_arrive_expect_tx(&k_full[st], kTileBytes);
        tma_load_4d(sK + st * kTileBytes, &tmK, &k_full[st], 0, hk, j * TK, b);
        tma_load_4d(sK + st * kTileBytes + kHalf, &tmK, &k_full[st], 64, hk, j * TK, b);
        ++armed_k;
        if (!mbar_wait(&v_free[st], ph ^ 1, a.err, kErrTmaWait)) break;
        mbar_arrive_expect_tx(&v_full[st], kTileBytes);
        tma_load_4d(sV + st * kTileBytes, &tmV, &v_full[st], 0, hk, j * TK, b);
        tma_load_4d(sV + st * kTileBytes + kHalf, &tmV, &v_full[st], 64, hk, j * TK, b);
        ++armed_v;
      }
      // Drain loads that may still be in flight before the CTA can exit.
      mbar_wait(q_full, 0, nullptr, 0);
      for (int i = 1; i <= 2 && i <= armed_k; ++i) mbar_wait(&k_full[(armed_k - i) & 1], ((armed_k - i) >> 1) & 1, nullptr, 0);
      for (int i = 1; i <= 2 && i <= armed_v; ++i) mbar_wait(&v_full[(armed_v - i) & 1], ((armed_v - i) >> 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0 && nt > 0) {
      constexpr uint32_t idesc_qk = umma_idesc_f16_major(TQ, TK, true, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_f16_major(TQ, HD, true, false, true);
      const uint32_t q0 = smem_addr(sQ), p0 = smem_addr(sP);
      bool ok = mbar_wait(q_full, 0, a.err, kErrMmaWait);
      auto issue_pv = [&](int i) -> bool {
        const int st = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(p_full, i & 1, a.err, kErrMmaWait)) return false;
        if (!mbar_wait(&v_full[st], ph, a.err, kErrMmaWait)) return false;
        tc_fence_after();
        const uint32_t v0 = smem_addr(sV + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < TK / 16; ++k) {
          const uint64_t ad = umma_desc_k_sw128(p0 + (k >> 2) * kHalf + (k & 3) * 32);
          const uint64_t bd = umma_desc_mn_sw128(v0 + k * 16 * 128, kHalf, 1024);
          umma_f16(tO, ad, bd, idesc_pv, (i | k) != 0);
        }
        umma_commit(o_done);
        umma_commit(&v_free[st]);
        return true;
      };
      for (int j = 0; j < nt && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_full[st], ph, a.err, kErrMmaWait)) { ok = false; break; }
        if (!mbar_wait(&s_free[st], ph ^ 1, a.err, kErrMmaWait)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k0 = smem_addr(sK + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t ad = umma_desc_k_sw128(q0 + (k >> 2) * kHalf + (k & 3) * 32);
          const uint64_t bd = umma_desc_k_sw128(k0 + (k >> 2) * kHalf + (k & 3) * 32);
          umma_f16(tmem + st * TK, ad, bd, idesc_qk, k != 0);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_free[st]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) issue_pv(nt - 1);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax
    // Warps 2..5 take key/hd columns [0, 64), warps 6..9 columns [64, 128) of
    // the same rows; the row max and the final row sum are exchanged through
    // shared memory between the two warps of a lane quarter.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // row inside the tile == TMEM lane
    const int qrow = m0 + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int c0 = half * 64;           // first owned column of S / O
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nt && ok; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!mbar_wait(&s_full[st], ph, a.err, kErrEpiWait)) { ok = false; break; }
      tc_fence_after();
      float s[64];
      tmem_ld_32x32b_x32(tmem + lane_base + st * TK + c0, reinterpret_cast<uint32_t*>(s));
      tmem_ld_32x32b_x32(tmem + lane_base + st * TK + c0 + 32, reinterpret_cast<uint32_t*>(s + 32));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_free[st]);  // S buffer may be overwritten by S_{j+2}
      const int k0 = j * TK + c0;
      const bool edge = (j * TK + TK > a.Skv) || (a.causal && j * TK + TK - 1 > m0 + off);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        float v = s[i] * a.scale_log2;
        if (edge) {
          const int key = k0 + i;
          if (key >= a.Skv || (a.causal && key > qrow + off)) v = -INFINITY;
        }
        s[i] = v;
        mx = fmaxf(mx, v);
      }
      xmax[(st * 2 + half) * TQ + r] = mx;
      mbar_arrive(&xbar[st * 4 + quarter]);
      if (!mbar_wait(&xbar[st * 4 + quarter], ph, a.err, kErrEpiWait)) { ok = false; break; }
      mx = fmaxf(mx, xmax[(st * 2 + (half ^ 1)) * TQ + r]);
      float alpha = 1.f;
      if (mx > m_run + kRescaleThreshold || m_run == -INFINITY) {
        const float m_new = fmaxf(m_run, mx);
        alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new);
        m_run = m_new;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      float sum = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const float p0 = fast_exp2(s[i] - m_use), p1 = fast_exp2(s[i + 1] - m_use);
        sum += p0 + p1;
        pk[i / 2] = pack_bf16(p0, p1);
      }
      l_run = l_run * alpha + sum;
      // P_{j-1} V_{j-1} must have finished before P is overwritten and O rescaled.
      if (j >= 1 && !mbar_wait(o_done, (j - 1) & 1, a.err, kErrEpiWait)) { ok = false; break; }
      tc_fence_after();
      // tcgen05.ld/st are warp-collective: rescale if any row of the warp needs it.
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + lane_base + c0 + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tO + lane_base + c0 + c * 32, o);
        }
        tmem_st_wait();
      }
      // This thread's 64 keys are exactly one 64-key swizzle block of P.
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint4 v = make_uint4(pk[ch * 4], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
        *reinterpret_cast<uint4*>(sP + half * kHalf + r * 128 + ((ch ^ (r & 7)) * 16)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // ---------------------------------------------------------- epilogue
    xsum[half * TQ + r] = l_run;
    mbar_arrive(&sbar[quarter]);
    const bool summed = mbar_wait(&sbar[quarter], 0, a.err, kErrEpiWait);
    const float l_row = l_run + (summed ? xsum[(half ^ 1) * TQ + r] : 0.f);
    const bool have = ok && summed && nt > 0 && mbar_wait(o_done, (nt - 1) & 1, a.err, kErrEpiWait);
    tc_fence_after();
    // Every lane executes the (warp-collective) TMEM loads; only rows < Sq store.
    const bool have_w = __all_sync(0xffffffffu, have);
    {
      __nv_bfloat16* dst =
          reinterpret_cast<__nv_bfloat16*>(a.out) + (((int64_t)b * a.Sq + qrow) * a.H + h) * HD + c0;
      const float inv = (have_w && l_row > 0.f) ? 1.f / l_row : 0.f;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        if (have_w) {
          tmem_ld_32x32b_x32(tO + lane_base + c0 + c * 32, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (qrow >= a.Sq) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 v = make_uint4(pack_bf16(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv),
                               pack_bf16(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv),
                               pack_bf16(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv),
                               pack_bf16(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv));
          *reinterpret_cast<uint4*>(dst + c * 32 + e) = v;
        }
      }
      if (qrow < a.Sq && half == 0)
        a.lse[((int64_t)b * a.H + h) * a.Sq + qrow] =
            (have_w && l_row > 0.f) ? (m_run == -INFINITY ? 0.f : m_run) * kLn2 + __logf(l_row) : INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// --------------------------------------------------- two Q tiles per CTA
// CTA = (batch, head, 256 queries as tiles A and B); 10 warps:
//   warp 0      TMA: Q_A, Q_B once; K_j, V_j (128 keys) into 2-stage rings;
//   warp 1      TMEM owner + MMA issue.  TMEM columns: S_A [0,128), S_B
//               [128,256), O_A [256,384), O_B [384,512).  P_X overwrites the
//               first 64 columns of S_X as packed bf16 and is the A operand of
//               P_X V_j straight from tensor memory.  Issue order
//                 S_A(j) S_B(j) | PV_A(j) S_A(j+1) | PV_B(j) S_B(j+1) | ...
//               so each tile's softmax runs while the other tile's MMAs do;
//               the MMAs of one CTA execute in issue order, which makes it
//               safe for S_X(j+1) to overwrite P_X(j) after PV_X(j).
//   warps 2..5  softmax of tile A, warps 6..9 tile B: one thread per query
//               row (its TMEM lane), 128 key columns per thread, running max
//               and sum in the exp2 domain, lazy O rescale (threshold 2^8).
// s_full_X(j) is committed after PV_X(j-1), so a softmax thread that sees it
// may also rewrite O_X.  All waits are bounded (sm100.cuh).
namespace fwd2 {
constexpr int kThreads = 320;
constexpr int kRowThreads = 128;
constexpr size_t kSmem = 1024 + 6 * (size_t)kTileBytes + 256;
constexpr int kHeadGroup = 16;  // (batch, head) pairs per launch group
}  // namespace fwd2

__global__ void __launch_bounds__(fwd2::kThreads, 1)
    attn_fwd_2q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, FwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = base;                    // Q_A, Q_B
  unsigned char* sK = base + 2 * kTileBytes;   // 2 stages
  unsigned char* sV = base + 4 * kTileBytes;   // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 6 * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* v_full = bars + 3;   // [2]
  uint64_t* k_free = bars + 5;   // [2]
  uint64_t* v_free = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;   // [tile]
  uint64_t* p_full = bars + 11;  // [tile]
  uint64_t* o_done = bars + 13;  // [tile]
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid over (head group, tile pair, head in group): groups of
  // fwd2::kHeadGroup (batch, head) pairs run one after another (the K / V rows
  // in flight stay L2-resident), and within a group the tile pairs launch in
  // descending order -- under a causal mask the longest first
  int m0, b, h;
  {
    const int bh = a.B * a.H, npairs = (a.Sq + 2 * TQ - 1) / (2 * TQ);
    const int grp = (int)blockIdx.x / (fwd2::kHeadGroup * npairs);
    const int r = (int)blockIdx.x - grp * fwd2::kHeadGroup * npairs;
    const int gs = min(fwd2::kHeadGroup, bh - grp * fwd2::kHeadGroup);
    m0 = (npairs - 1 - r / gs) * 2 * TQ;
    const int head = grp * fwd2::kHeadGroup + r % gs;
    b = head / a.H;
    h = head % a.H;
  }
  const int hk = h / (a.H / a.Hkv);
  const int off = a.Skv - a.Sq;
  int nt[2];
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const int mx0 = m0 + x * TQ;
    int kv_end = a.Skv;
    if (a.causal) kv_end = min(kv_end, mx0 + TQ + off);
    nt[x] = (mx0 < a.Sq && kv_end > 0) ? (kv_end + TK - 1) / TK : 0;
  }
  const int ntl = max(nt[0], nt[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_free[i], 1);
      mbar_init(&v_free[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], fwd2::kRowThreads);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && ntl > 0) {
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      tma_load_4d(sQ, &tmQ, q_full, 0, h, m0, b);
      tma_load_4d(sQ + kHalf, &tmQ, q_full, 64, h, m0, b);
      tma_load_4d(sQ + kTileBytes, &tmQ, q_full, 0, h, m0 + TQ, b);
      tma_load_4d(sQ + kTileBytes + kHalf, &tmQ, q_full, 64, h, m0 + TQ, b);
      int armed_k = 0, armed_v = 0;
      for (int j = 0; j < ntl; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_free[st], ph ^ 1, a.err, kErrTmaWait)) break;
        mbar_arrive_expect_tx(&k_full[st], kTileBytes);
        tma_load_4d(sK + st * kTileBytes, &tmK, &k_full[st], 0, hk, j * TK, b);
        tma_load_4d(sK + st * kTileBytes + kHalf, &tmK, &k_full[st], 64, hk, j * TK, b);
        ++armed_k;
        if (!mbar_wait(&v_free[st], ph ^ 1, a.err, kErrTmaWait)) break;
        mbar_arrive_expect_tx(&v_full[st], kTileBytes);
        tma_load_4d(sV + st * kTileBytes, &tmV, &v_full[st], 0, hk, j * TK, b);
        tma_load_4d(sV + st * kTileBytes + kHalf, &tmV, &v_full[st], 64, hk, j * TK, b);
        ++armed_v;
      }
      mbar_wait(q_full, 0, nullptr, 0);
      for (int i = 1; i <= 2 && i <= armed_k; ++i) mbar_wait(&k_full[(armed_k - i) & 1], ((armed_k - i) >> 1) & 1, nullptr, 0);
      for (int i = 1; i <= 2 && i <= armed_v; ++i) mbar_wait(&v_full[(armed_v - i) & 1], ((armed_v - i) >> 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0 && ntl > 0) {
      constexpr uint32_t idesc_qk = umma_idesc_f16_major(TQ, TK, true, false, false);
      constexpr uint32_t idesc_pv = umma_idesc_f16_major(TQ, HD, true, false, true);
      const uint32_t q_addr[2] = {smem_addr(sQ), smem_addr(sQ + kTileBytes)};
      auto issue_s = [&](int x, int j) {
        const uint32_t k0 = smem_addr(sK + (j & 1) * kTileBytes);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t o = (k >> 2) * kHalf + (k & 3) * 32;
          umma_f16(tmem + x * TQ, umma_desc_k_sw128(q_addr[x] + o), umma_desc_k_sw128(k0 + o), idesc_qk, k != 0);
        }
        umma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {
        const uint32_t v0 = smem_addr(sV + (j & 1) * kTileBytes);
#pragma unroll
        for (int k = 0; k < TK / 16; ++k)  // 16 keys = 8 columns of packed P
          umma_f16_tmem_a(tmem + 256 + x * HD, tmem + x * TQ + k * 8, umma_desc_mn_sw128(v0 + k * 16 * 128, kHalf, 1024),
                          idesc_pv, (j | k) != 0);
        if (j == nt[x] - 1) umma_commit(&o_done[x]);
      };
      bool ok = mbar_wait(q_full, 0, a.err, kErrMmaWait) && mbar_wait(&k_full[0], 0, a.err, kErrMmaWait);
      if (ok) {
        tc_fence_after();
        if (nt[0] > 0) issue_s(0, 0);
        if (nt[1] > 0) issue_s(1, 0);
        umma_commit(&k_free[0]);
      }
      for (int j = 0; j < ntl && ok; ++j) {
        const int st = j & 1, nst = (j + 1) & 1;
        const uint32_t ph = (j >> 1) & 1, nph = ((j + 1) >> 1) & 1;
        const bool next = j + 1 < ntl;
        if (!mbar_wait(&v_full[st], ph, a.err, kErrMmaWait)) break;
        if (j < nt[0]) {
          if (!mbar_wait(&p_full[0], j & 1, a.err, kErrMmaWait)) break;
          tc_fence_after();
          issue_pv(0, j);
        }
        if (next) {
          if (!mbar_wait(&k_full[nst], nph, a.err, kErrMmaWait)) break;
          tc_fence_after();
        }
        if (j + 1 < nt[0]) issue_s(0, j + 1);
        if (j < nt[1]) {
          if (!mbar_wait(&p_full[1], j & 1, a.err, kErrMmaWait)) break;
          tc_fence_after();
          issue_pv(1, j);
        }
        umma_commit(&v_free[st]);
        if (j + 1 < nt[1]) issue_s(1, j + 1);
        if (next) umma_commit(&k_free[nst]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax
    const int x = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int mx0 = m0 + x * TQ;
    const int qrow = mx0 + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_base + x * TQ;
    const uint32_t tO = tmem + lane_base + 256 + x * HD;
    const int n = nt[x];
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n && ok; ++j) {
      if (!mbar_wait(&s_full[x], j & 1, a.err, kErrEpiWait)) { ok = false; break; }
      tc_fence_after();
      // Keys 64..127 stay in registers; keys 0..63 are read twice (max pass,
      // then exp pass) so no more than 64 S values are live.  P(keys 2i, 2i+1)
      // lands in column i of S_X, so writing P for keys 0..31 only overwrites
      // columns already consumed, and keys 32..63 are re-read before that.
      // Maxima and sums use 8 independent accumulators (short dependency
      // chains); the exponent is one FFMA on the raw score: s*c - m.
      const bool edge = (j * TK + TK > a.Skv) || (a.causal && j * TK + TK - 1 > mx0 + off);
      const int lim = a.causal ? min(a.Skv, qrow + off + 1) : a.Skv;  // keys >= lim are masked
      const float c = a.scale_log2;
      auto masked = [&](float v, int key) -> float { return (edge && key >= lim) ? -INFINITY : v; };
      float pm[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) pm[e] = -INFINITY;
      {
        float t[64];
        tmem_ld_32x32b_x32(tS, reinterpret_cast<uint32_t*>(t));
        tmem_ld_32x32b_x32(tS + 32, reinterpret_cast<uint32_t*>(t + 32));
        tmem_ld_wait();
        if (edge) {
#pragma unroll
          for (int i = 0; i < 64; ++i) pm[i & 7] = fmaxf(pm[i & 7], masked(t[i], j * TK + i));
        } else {  // interior tile: no masks
#pragma unroll
          for (int i = 0; i < 64; ++i) pm[i & 7] = fmaxf(pm[i & 7], t[i]);
        }
      }
      float hi[64];
      tmem_ld_32x32b_x32(tS + 64, reinterpret_cast<uint32_t*>(hi));
      tmem_ld_32x32b_x32(tS + 96, reinterpret_cast<uint32_t*>(hi + 32));
      tmem_ld_wait();
      if (edge) {
#pragma unroll
        for (int i = 0; i < 64; ++i) hi[i] = masked(hi[i], j * TK + 64 + i);
      }
#pragma unroll
      for (int i = 0; i < 64; ++i) pm[i & 7] = fmaxf(pm[i & 7], hi[i]);
      const float mraw = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                               fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      const float mx = mraw * c;  // c > 0: the max of the scaled scores
      float alpha = 1.f;
      if (mx > m_run + kRescaleThreshold || m_run == -INFINITY) {
        const float m_new = fmaxf(m_run, mx);
        alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new);
        m_run = m_new;
      }
      const float nm = (m_run == -INFINITY) ? 0.f : -m_run;
      // exponentials on packed pairs: one f32x2 FMA per two scores, four f32x2
      // partial sums (8 accumulators as before)
      const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(nm, nm);
      uint64_t ps2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) ps2[e] = f2_pack(0.f, 0.f);
      auto exp_pair = [&](float s0, float s1, uint32_t& packed, int i) {
        const float2 y = f2_unpack(f2_fma(f2_pack(s0, s1), c2, nm2));
        const float p0 = fast_exp2(y.x), p1 = fast_exp2(y.y);
        ps2[i & 3] = f2_add(ps2[i & 3], f2_pack(p0, p1));
        packed = pack_bf16(p0, p1);
      };
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {  // keys 0..63, re-read
        float lo[32];
        tmem_ld_32x32b_x32(tS + cc * 32, reinterpret_cast<uint32_t*>(lo));
        tmem_ld_wait();
        if (edge) {
#pragma unroll
          for (int i = 0; i < 32; ++i) lo[i] = masked(lo[i], j * TK + cc * 32 + i);
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) exp_pair(lo[2 * i], lo[2 * i + 1], pk[i], i);
        tmem_st_32x32b_x16(tS + cc * 16, pk);
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {  // keys 64..127, from registers
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) exp_pair(hi[cc * 32 + 2 * i], hi[cc * 32 + 2 * i + 1], pk[i], i);
        tmem_st_32x32b_x16(tS + 32 + cc * 16, pk);
      }
      const float2 s01 = f2_unpack(f2_add(ps2[0], ps2[1])), s23 = f2_unpack(f2_add(ps2[2], ps2[3]));
      const float sum = (s01.x + s01.y) + (s23.x + s23.y);
      l_run = l_run * alpha + sum;
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tO + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    // ---------------------------------------------------------- epilogue
    const bool have = ok && n > 0 && mbar_wait(&o_done[x], 0, a.err, kErrEpiWait);
    tc_fence_after();
    const bool have_w = __all_sync(0xffffffffu, have);
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) + (((int64_t)b * a.Sq + qrow) * a.H + h) * HD;
    const float inv = (have_w && l_run > 0.f) ? 1.f / l_run : 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      if (have_w) {
        tmem_ld_32x32b_x32(tO + c * 32, o);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = 0u;
      }
      if (qrow >= a.Sq) continue;
#pragma unroll
      for (int e = 0; e < 32; e += 8) {
        uint4 v = make_uint4(pack_bf16(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv),
                             pack_bf16(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv),
                             pack_bf16(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv),
                             pack_bf16(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv));
        *reinterpret_cast<uint4*>(dst + c * 32 + e) = v;
      }
    }
    if (qrow < a.Sq)
      a.lse[((int64_t)b * a.H + h) * a.Sq + qrow] =
          (have_w && l_run > 0.f) ? (m_run == -INFINITY ? 0.f : m_run) * kLn2 + __logf(l_run) : INFINITY;
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

// (B, S, H, 128) tensor with arbitrary batch/seq/head strides; box = 64 x 1 x 128 x 1.
CUtensorMap make_bshd_map(const at::Tensor& t) {
  CUtensorMap m;
  const cuuint64_t dims[4] = {(cuuint64_t)t.size(3), (cuuint64_t)t.size(2), (cuuint64_t)t.size(1),
                              (cuuint64_t)t.size(0)};
  const cuuint64_t strides[3] = {(cuuint64_t)t.stride(2) * 2, (cuuint64_t)t.stride(1) * 2, (cuuint64_t)t.stride(0) * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)TQ, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return m;
}

// Error words of this file's kernels: module globals (one copy per device).
DeviceWord g_attn_fwd_err_word{g_attn_fwd_err, {}};

int* attn_error_word(const at::Device& dev) { return g_attn_fwd_err_word.get(dev.index()); }

}  // namespace

bool attn_sm100_supported(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  auto ok = [](const at::Tensor& t) {
    return t.scalar_type() == at::kBFloat16 && t.size(3) == HD && t.stride(3) == 1 &&
           (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0 && (t.stride(0) * 2) % 16 == 0 &&
           (t.stride(1) * 2) % 16 == 0 && (t.stride(2) * 2) % 16 == 0;
  };
  return ok(q) && ok(k) && ok(v);
}

std::tuple<at::Tensor, at::Tensor> attn_fwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                                  bool causal, double scale) {
  LRB_CHECK(attn_sm100_supported(q, k, v), "attn_fwd_sm100: bf16, head_dim 128, 16-byte aligned strides required");
  c10::cuda::CUDAGuard g(q.device());
  bind_device(q.get_device());
  const int64_t B = q.size(0), Sq = q.size(1), H = q.size(2), Skv = k.size(1), Hkv = k.size(2);
  LRB_CHECK(Hkv > 0 && H % Hkv == 0 && k.sizes() == v.sizes(), "attn_fwd_sm100: head mismatch");
  auto o = at::empty({B, Sq, H, HD}, q.options());
  auto lse = at::empty({B, H, Sq}, q.options().dtype(at::kFloat));
  if (B * Sq * H == 0) return {o, lse};
  CUtensorMap tq = make_bshd_map(q), tk = make_bshd_map(k), tv = make_bshd_map(v);
  FwdArgs args{o.data_ptr(), lse.data_ptr<float>(), (int)B, (int)H, (int)Hkv, (int)Sq, (int)Skv, causal ? 1 : 0,
               (float)scale * kLog2e, attn_error_word(q.device())};
  static const bool one_tile = [] {
    const char* e = std::getenv("LRB_ATTN_FWD_ONE_TILE");
    return e != nullptr && e[0] == '1';
  }();
  if (one_tile) {  // one Q tile per CTA, P through shared memory (kept for A/B comparisons)
    LRB_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    dim3 grid((unsigned)((Sq + TQ - 1) / TQ), (unsigned)(B * H));
    attn_fwd_sm100_kernel<<<grid, kThreads, kSmem, stream()>>>(tq, tk, tv, args);
  } else {
    LRB_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_2q_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)fwd2::kSmem));
    LRB_CHECK(B * H * ((Sq + 2 * TQ - 1) / (2 * TQ)) < (1LL << 31), "attention: too many CTAs");
    dim3 grid((unsigned)(B * H * ((Sq + 2 * TQ - 1) / (2 * TQ))));
    attn_fwd_2q_kernel<<<grid, fwd2::kThreads, fwd2::kSmem, stream()>>>(tq, tk, tv, args);
  }
  LRB_LAUNCH_CHECK();
  return {o, lse};
}

int64_t attn_sm100_error(int64_t device) { return g_attn_fwd_err_word.take((int)device); }

}  // namespace lrb
