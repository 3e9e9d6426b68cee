// Flash attention (forward + backward) on mma.sync m16n8k16, any head dim in
// {16, 32, 64, 96, 128}, grouped-query heads read in place (no K/V repeat),
// causal mask aligned to the end of the key sequence, arbitrary
// batch/sequence/head strides for q, k, v.
//
// Forward: one CTA = 64 query rows of one (batch, head); 4 warps x 16 rows;
// K/V tiles of 64 keys double-buffered through cp.async; online softmax in
// the exp2 domain; P is fed to the second MMA straight from registers.
// Backward: one CTA = 64 keys of one (batch, kv-head); loops over the query
// heads of the group and over query tiles; dK/dV stay in registers, dS is
// staged in shared memory for dQ, which is accumulated in fp32 with atomics.
#include "../common.cuh"
#include "mma_sm80.cuh"

namespace lrb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;  // (B, Sq, H, D) contiguous
  float* lse;  // (B, H, Sq), natural log; +inf for rows that see no key
  int64_t q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, v_sb, v_ss, v_sh;
  int B, H, Hkv, Sq, Skv, causal;
  float scale, scale_log2;
  // backward
  const void* dout;     // (B, Sq, H, D) contiguous
  const float* di;      // (B, H, Sq)
  float* dq_acc;        // (B, Sq, H, D) fp32
  void* dk;             // (B, Skv, Hkv, D)
  void* dv;
};

template <typename T, int D>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const AttnParams p) {
  constexpr int BM = 64, BN = 64, LD = D + 8, CPR = D / 8;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sQ = reinterpret_cast<T*>(smem_raw);
  T* sK = sQ + BM * LD;
  T* sV = sK + 2 * BN * LD;
  using Op = MmaOp<T>;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.x * BM;
  const int b = blockIdx.y / p.H, h = blockIdx.y % p.H, hk = h / (p.H / p.Hkv);
  const T* qg = reinterpret_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
  const T* kg = reinterpret_cast<const T*>(p.k) + b * p.k_sb + hk * p.k_sh;
  const T* vg = reinterpret_cast<const T*>(p.v) + b * p.v_sb + hk * p.v_sh;
  const int off = p.Skv - p.Sq;
  int n_end = p.Skv;
  if (p.causal) n_end = min(n_end, m0 + BM + off);
  const int ntiles = n_end > 0 ? (n_end + BN - 1) / BN : 0;

  for (int i = tid; i < BM * CPR; i += 128) {
    const int r = i / CPR, c = i % CPR, row = m0 + r;
    const bool ok = row < p.Sq;
    cp_async16(smem_u32(sQ + r * LD + c * 8), qg + (int64_t)(ok ? row : 0) * p.q_ss + c * 8, ok);
  }
  cp_async_commit();
  auto load_kv = [&](int tile, int buf) {
    const int n0 = tile * BN;
    for (int i = tid; i < BN * CPR; i += 128) {
      const int r = i / CPR, c = i % CPR, key = n0 + r;
      const bool ok = key < p.Skv;
      const int64_t kr = ok ? key : 0;
      cp_async16(smem_u32(sK + (buf * BN + r) * LD + c * 8), kg + kr * p.k_ss + c * 8, ok);
      cp_async16(smem_u32(sV + (buf * BN + r) * LD + c * 8), vg + kr * p.v_ss + c * 8, ok);
    }
  };
  if (ntiles > 0) load_kv(0, 0);
  cp_async_commit();

  float o_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[D / 16][4];

  cp_async_wait<1>();
  __syncthreads();
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], smem_u32(sQ + r * LD + c));
  }

  const int row_base = m0 + warp * 16 + (lane >> 2);
  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntiles) load_kv(t + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const T* Kb = sK + buf * BN * LD;
    const T* Vb = sV + buf * BN * LD;
    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8, c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(b0, b1, b2, b3, smem_u32(Kb + r * LD + c));
        Op::run(s[2 * np], qf[kk], b0, b1);
        Op::run(s[2 * np + 1], qf[kk], b2, b3);
      }
    }
    const int n0 = t * BN;
    const bool edge = (n0 + BN > p.Skv) || (p.causal && n0 + BN - 1 > m0 + off);
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * p.scale_log2;
        if (edge) {
          const int row = row_base + (e >> 1) * 8;
          const int key = n0 + j * 8 + (lane & 3) * 2 + (e & 1);
          const bool ok = key < p.Skv && (!p.causal || key <= row + off);
          v = ok ? v : -INFINITY;
        }
        s[j][e] = v;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) mx = fmaxf(mx, fmaxf(s[j][2 * r], s[j][2 * r + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_r[r], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = fast_exp2(m_r[r] - m_use);
      m_r[r] = m_new;
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
        s[j][2 * r] = fast_exp2(s[j][2 * r] - m_use);
        s[j][2 * r + 1] = fast_exp2(s[j][2 * r + 1] - m_use);
        rs += s[j][2 * r] + s[j][2 * r + 1];
      }
      l_r[r] = l_r[r] * alpha + rs;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o_acc[dt][2 * r] *= alpha;
        o_acc[dt][2 * r + 1] *= alpha;
      }
    }
#pragma unroll
    for (int k2 = 0; k2 < BN / 16; ++k2) {
      uint32_t a[4] = {Op::pack(s[2 * k2][0], s[2 * k2][1]), Op::pack(s[2 * k2][2], s[2 * k2][3]),
                       Op::pack(s[2 * k2 + 1][0], s[2 * k2 + 1][1]), Op::pack(s[2 * k2 + 1][2], s[2 * k2 + 1][3])};
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int r = k2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(b0, b1, b2, b3, smem_u32(Vb + r * LD + c));
        Op::run(o_acc[2 * dp], a, b0, b1);
        Op::run(o_acc[2 * dp + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }

  T* og = reinterpret_cast<T*>(p.o);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_r[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int row = row_base + r * 8;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    if (row < p.Sq) {
      T* dst = og + (((int64_t)b * p.Sq + row) * p.H + h) * D + (lane & 3) * 2;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt)
        *reinterpret_cast<uint32_t*>(dst + dt * 8) = Op::pack(o_acc[dt][2 * r] * inv, o_acc[dt][2 * r + 1] * inv);
      if ((lane & 3) == 0)
        p.lse[((int64_t)b * p.H + h) * p.Sq + row] = l > 0.f ? m_r[r] * kLn2 + __logf(l) : INFINITY;
    }
  }
}

// Di[b, h, q] = sum_d dO * O
template <typename T, int D>
__global__ void attn_dot_kernel(const T* __restrict__ dout, const T* __restrict__ out, float* __restrict__ di, int B,
                                int Sq, int H) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);  // over (b, q, h)
  if (row >= (int64_t)B * Sq * H) return;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s += to_f(dout[row * D + d]) * to_f(out[row * D + d]);
  s = warp_sum(s);
  if (lane == 0) {
    const int h = (int)(row % H);
    const int64_t bq = row / H;
    const int q = (int)(bq % Sq);
    const int b = (int)(bq / Sq);
    di[((int64_t)b * H + h) * Sq + q] = s;
  }
}

// D = rowsum(dO * O) for head_dim 128: eight lanes per (b, q, h) row, each with
// two 16-byte loads per tensor; the partial sums meet through three shuffles.
// Grid-stride over rows, so a few blocks per SM stream the two tensors once.
template <typename T>
__global__ void __launch_bounds__(256) attn_dot128_kernel(const T* __restrict__ dout, const T* __restrict__ out,
                                                           float* __restrict__ di, int B, int Sq, int H) {
  const int64_t rows = (int64_t)B * Sq * H;
  const int sub = threadIdx.x & 7;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 3) {
    const T* a = dout + row * 128 + sub * 16;
    const T* o = out + row * 128 + sub * 16;
    const Vec16<T> a0 = ld16(a), a1 = ld16(a + 8), o0 = ld16(o), o1 = ld16(o + 8);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += to_f(a0.v[i]) * to_f(o0.v[i]) + to_f(a1.v[i]) * to_f(o1.v[i]);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (sub == 0) {
      const int h = (int)(row % H);
      const int64_t bq = row / H;
      di[((int64_t)(bq / Sq) * H + h) * Sq + (int)(bq % Sq)] = s;
    }
  }
}

template <typename T, int D, int BMQ>
__global__ void __launch_bounds__(128) attn_bwd_kernel(const AttnParams p) {
  constexpr int BN = 64, NW = 4, LD = D + 8, LDS = BMQ + 8, CPR = D / 8;
  constexpr int RB = BMQ / 16, DS = NW / RB, DW = D / DS;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sK = reinterpret_cast<T*>(smem_raw);
  T* sV = sK + BN * LD;
  T* sQ = sV + BN * LD;
  T* sdO = sQ + BMQ * LD;
  T* sdS = sdO + BMQ * LD;
  float* sL = reinterpret_cast<float*>(sdS + BN * LDS);
  float* sDi = sL + BMQ;
  using Op = MmaOp<T>;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * BN;
  const int b = blockIdx.y / p.Hkv, hk = blockIdx.y % p.Hkv, G = p.H / p.Hkv;
  const T* kg = reinterpret_cast<const T*>(p.k) + b * p.k_sb + hk * p.k_sh;
  const T* vg = reinterpret_cast<const T*>(p.v) + b * p.v_sb + hk * p.v_sh;
  const int off = p.Skv - p.Sq;

  for (int i = tid; i < BN * CPR; i += 128) {
    const int r = i / CPR, c = i % CPR, key = n0 + r;
    const bool ok = key < p.Skv;
    const int64_t kr = ok ? key : 0;
    cp_async16(smem_u32(sK + r * LD + c * 8), kg + kr * p.k_ss + c * 8, ok);
    cp_async16(smem_u32(sV + r * LD + c * 8), vg + kr * p.v_ss + c * 8, ok);
  }
  cp_async_commit();

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const int q_first = p.causal ? max(0, n0 - off) : 0;
  const int key_row = n0 + warp * 16 + (lane >> 2);
  const T* dog = reinterpret_cast<const T*>(p.dout);

  for (int g = 0; g < G; ++g) {
    const int h = hk * G + g;
    const T* qg = reinterpret_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
    for (int m0 = (q_first / BMQ) * BMQ; m0 < p.Sq; m0 += BMQ) {
      for (int i = tid; i < BMQ * CPR; i += 128) {
        const int r = i / CPR, c = i % CPR, row = m0 + r;
        const bool ok = row < p.Sq;
        const int64_t qr = ok ? row : 0;
        cp_async16(smem_u32(sQ + r * LD + c * 8), qg + qr * p.q_ss + c * 8, ok);
        cp_async16(smem_u32(sdO + r * LD + c * 8), dog + (((int64_t)b * p.Sq + qr) * p.H + h) * D + c * 8, ok);
      }
      cp_async_commit();
      for (int i = tid; i < BMQ; i += 128) {
        const int row = m0 + i;
        const bool ok = row < p.Sq;
        sL[i] = ok ? p.lse[((int64_t)b * p.H + h) * p.Sq + row] * kLog2e : INFINITY;
        sDi[i] = ok ? p.di[((int64_t)b * p.H + h) * p.Sq + row] : 0.f;
      }
      cp_async_wait<0>();
      __syncthreads();

      float st[BMQ / 8][4], dp[BMQ / 8][4];
#pragma unroll
      for (int j = 0; j < BMQ / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) st[j][e] = dp[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t ka[4], va[4];
        const int ar = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, ac = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(ka[0], ka[1], ka[2], ka[3], smem_u32(sK + ar * LD + ac));
        ldsm_x4(va[0], va[1], va[2], va[3], smem_u32(sV + ar * LD + ac));
#pragma unroll
        for (int np = 0; np < BMQ / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          const int r = np * 16 + (lane & 7) + (lane >> 4) * 8, c = kk * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(b0, b1, b2, b3, smem_u32(sQ + r * LD + c));
          Op::run(st[2 * np], ka, b0, b1);
          Op::run(st[2 * np + 1], ka, b2, b3);
          ldsm_x4(b0, b1, b2, b3, smem_u32(sdO + r * LD + c));
          Op::run(dp[2 * np], va, b0, b1);
          Op::run(dp[2 * np + 1], va, b2, b3);
        }
      }
#pragma unroll
      for (int j = 0; j < BMQ / 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key_row + (e >> 1) * 8;
          const int ql = j * 8 + (lane & 3) * 2 + (e & 1);
          const int q = m0 + ql;
          const bool ok = key < p.Skv && q < p.Sq && (!p.causal || key <= q + off);
          const float pv = ok ? fast_exp2(st[j][e] * p.scale_log2 - sL[ql]) : 0.f;
          st[j][e] = pv;
          dp[j][e] = pv * (dp[j][e] - sDi[ql]);
        }
      }
#pragma unroll
      for (int kq = 0; kq < BMQ / 16; ++kq) {
        uint32_t pa[4] = {Op::pack(st[2 * kq][0], st[2 * kq][1]), Op::pack(st[2 * kq][2], st[2 * kq][3]),
                          Op::pack(st[2 * kq + 1][0], st[2 * kq + 1][1]), Op::pack(st[2 * kq + 1][2], st[2 * kq + 1][3])};
        uint32_t sa[4] = {Op::pack(dp[2 * kq][0], dp[2 * kq][1]), Op::pack(dp[2 * kq][2], dp[2 * kq][3]),
                          Op::pack(dp[2 * kq + 1][0], dp[2 * kq + 1][1]), Op::pack(dp[2 * kq + 1][2], dp[2 * kq + 1][3])};
#pragma unroll
        for (int dd = 0; dd < D / 16; ++dd) {
          uint32_t b0, b1, b2, b3;
          const int r = kq * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = dd * 16 + (lane >> 4) * 8;
          ldsm_x4_t(b0, b1, b2, b3, smem_u32(sdO + r * LD + c));
          Op::run(dv[2 * dd], pa, b0, b1);
          Op::run(dv[2 * dd + 1], pa, b2, b3);
          ldsm_x4_t(b0, b1, b2, b3, smem_u32(sQ + r * LD + c));
          Op::run(dk[2 * dd], sa, b0, b1);
          Op::run(dk[2 * dd + 1], sa, b2, b3);
        }
      }
      // stage dS^T (keys x queries) for the dQ product
#pragma unroll
      for (int j = 0; j < BMQ / 8; ++j) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int kl = warp * 16 + (lane >> 2) + r * 8, ql = j * 8 + (lane & 3) * 2;
          *reinterpret_cast<uint32_t*>(sdS + kl * LDS + ql) = Op::pack(dp[j][2 * r], dp[j][2 * r + 1]);
        }
      }
      __syncthreads();
      {
        const int rb = warp % RB, d0 = (warp / RB) * DW;
        float dq[DW / 8][4];
#pragma unroll
        for (int i = 0; i < DW / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          uint32_t a[4];
          const int mi = lane >> 3;
          const int sr = kk * 16 + (lane & 7) + (mi >> 1) * 8, sc = rb * 16 + (mi & 1) * 8;
          ldsm_x4_t(a[0], a[1], a[2], a[3], smem_u32(sdS + sr * LDS + sc));
#pragma unroll
          for (int dd = 0; dd < DW / 16; ++dd) {
            uint32_t b0, b1, b2, b3;
            const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = d0 + dd * 16 + (lane >> 4) * 8;
            ldsm_x4_t(b0, b1, b2, b3, smem_u32(sK + r * LD + c));
            Op::run(dq[2 * dd], a, b0, b1);
            Op::run(dq[2 * dd + 1], a, b2, b3);
          }
        }
#pragma unroll
        for (int dt = 0; dt < DW / 8; ++dt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int q = m0 + rb * 16 + (lane >> 2) + (e >> 1) * 8;
            const int d = d0 + dt * 8 + (lane & 3) * 2 + (e & 1);
            if (q < p.Sq) atomicAdd(p.dq_acc + (((int64_t)b * p.Sq + q) * p.H + h) * D + d, dq[dt][e] * p.scale);
          }
        }
      }
      __syncthreads();
    }
  }
  T* dkg = reinterpret_cast<T*>(p.dk);
  T* dvg = reinterpret_cast<T*>(p.dv);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = key_row + r * 8;
    if (key >= p.Skv) continue;
    const int64_t base = (((int64_t)b * p.Skv + key) * p.Hkv + hk) * D + (lane & 3) * 2;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      *reinterpret_cast<uint32_t*>(dkg + base + dt * 8) = Op::pack(dk[dt][2 * r] * p.scale, dk[dt][2 * r + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvg + base + dt * 8) = Op::pack(dv[dt][2 * r], dv[dt][2 * r + 1]);
    }
  }
}

template <typename T>
__global__ void f32_to_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = from_f<T>(src[i]);
}

void fill_params(AttnParams& p, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal,
                 double scale) {
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = v.data_ptr();
  p.q_sb = q.stride(0); p.q_ss = q.stride(1); p.q_sh = q.stride(2);
  p.k_sb = k.stride(0); p.k_ss = k.stride(1); p.k_sh = k.stride(2);
  p.v_sb = v.stride(0); p.v_ss = v.stride(1); p.v_sh = v.stride(2);
  p.B = (int)q.size(0); p.Sq = (int)q.size(1); p.H = (int)q.size(2);
  p.Skv = (int)k.size(1); p.Hkv = (int)k.size(2);
  p.causal = causal ? 1 : 0;
  p.scale = (float)scale;
  p.scale_log2 = (float)scale * kLog2e;
}

void check_qkv(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  LRB_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "attention: CUDA tensors required");
  LRB_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "attention: (B, S, H, D) tensors required");
  LRB_CHECK(q.stride(3) == 1 && k.stride(3) == 1 && v.stride(3) == 1, "attention: head dim must be contiguous");
  LRB_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(), "attention: dtype mismatch");
  LRB_CHECK(q.scalar_type() == at::kBFloat16 || q.scalar_type() == at::kHalf, "attention: bf16/fp16 only");
  LRB_CHECK(k.size(2) > 0 && q.size(2) % k.size(2) == 0, "attention: H must be a multiple of Hkv");
  LRB_CHECK(k.sizes() == v.sizes() && q.size(3) == k.size(3) && q.size(0) == k.size(0), "attention: shape mismatch");
  for (const auto* t : {&q, &k, &v})
    LRB_CHECK((reinterpret_cast<uintptr_t>(t->data_ptr()) % 16) == 0 && t->stride(1) % 8 == 0 &&
                  t->stride(2) % 8 == 0 && t->stride(0) % 8 == 0,
              "attention: 16-byte aligned rows required");
}

template <typename T, int D>
void run_fwd(AttnParams& p) {
  constexpr int BM = 64, BN = 64, LD = D + 8;
  const size_t smem = (size_t)(BM + 4 * BN) * LD * sizeof(T);
  auto k = attn_fwd_kernel<T, D>;
  LRB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.Sq + BM - 1) / BM, p.B * p.H);
  k<<<grid, 128, smem, stream()>>>(p);
  LRB_LAUNCH_CHECK();
}

template <typename T, int D>
void run_bwd(AttnParams& p) {
  constexpr int BMQ = D > 64 ? 32 : 64, BN = 64, LD = D + 8, LDS = BMQ + 8;
  const size_t smem = (size_t)(2 * BN + 2 * BMQ) * LD * sizeof(T) + (size_t)BN * LDS * sizeof(T) + 2 * BMQ * sizeof(float);
  auto k = attn_bwd_kernel<T, D, BMQ>;
  LRB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.Skv + BN - 1) / BN, p.B * p.Hkv);
  k<<<grid, 128, smem, stream()>>>(p);
  LRB_LAUNCH_CHECK();
}

#define LRB_ATTN_DISPATCH_D(D_, FN, T, ...)                                   \
  switch (D_) {                                                               \
    case 16: FN<T, 16>(__VA_ARGS__); break;                                   \
    case 32: FN<T, 32>(__VA_ARGS__); break;                                   \
    case 64: FN<T, 64>(__VA_ARGS__); break;                                   \
    case 96: FN<T, 96>(__VA_ARGS__); break;                                   \
    case 128: FN<T, 128>(__VA_ARGS__); break;                                 \
    default: LRB_CHECK(false, "attention: head_dim must be 16, 32, 64, 96 or 128, got ", D_); \
  }

}  // namespace

std::tuple<at::Tensor, at::Tensor> attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                            bool causal, double scale) {
  check_qkv(q, k, v);
  c10::cuda::CUDAGuard g(q.device());
  bind_device(q.get_device());
  const int64_t B = q.size(0), Sq = q.size(1), H = q.size(2), D = q.size(3);
  auto o = at::empty({B, Sq, H, D}, q.options());
  auto lse = at::empty({B, H, Sq}, q.options().dtype(at::kFloat));
  if (B * Sq * H == 0) return {o, lse};
  AttnParams p{};
  fill_params(p, q, k, v, causal, scale);
  p.o = o.data_ptr();
  p.lse = lse.data_ptr<float>();
  if (q.scalar_type() == at::kBFloat16) {
    LRB_ATTN_DISPATCH_D((int)D, run_fwd, __nv_bfloat16, p);
  } else {
    LRB_ATTN_DISPATCH_D((int)D, run_fwd, __half, p);
  }
  return {o, lse};
}

// tcgen05 backward for bf16 / head_dim 128 (attention_bwd_sm100.cu)
void attn_bwd_sm100(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                    const at::Tensor& lse, const at::Tensor& di, at::Tensor& dq_acc, at::Tensor& dk, at::Tensor& dv,
                    bool causal, double scale);

// `sm100`: run the tcgen05 kernel (caller checked attn_sm100_supported for q, k, v and dout)
std::tuple<at::Tensor, at::Tensor, at::Tensor> attn_bwd(const at::Tensor& dout, const at::Tensor& q,
                                                        const at::Tensor& k, const at::Tensor& v,
                                                        const at::Tensor& out, const at::Tensor& lse, bool causal,
                                                        double scale, bool sm100) {
  check_qkv(q, k, v);
  LRB_CHECK(dout.is_contiguous() && out.is_contiguous(), "attn_bwd: dout/out must be contiguous");
  c10::cuda::CUDAGuard g(q.device());
  bind_device(q.get_device());
  const int64_t B = q.size(0), Sq = q.size(1), H = q.size(2), D = q.size(3), Skv = k.size(1), Hkv = k.size(2);
  auto dq = at::empty({B, Sq, H, D}, q.options());
  auto dk = at::empty({B, Skv, Hkv, D}, q.options());
  auto dv = at::empty({B, Skv, Hkv, D}, q.options());
  if (B * H == 0) return {dq, dk, dv};
  auto dq_acc = at::zeros({B, Sq, H, D}, q.options().dtype(at::kFloat));
  auto di = at::empty({B, H, Sq}, q.options().dtype(at::kFloat));
  AttnParams p{};
  fill_params(p, q, k, v, causal, scale);
  p.lse = const_cast<float*>(lse.data_ptr<float>());
  p.dout = dout.data_ptr();
  p.di = di.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = dk.data_ptr();
  p.dv = dv.data_ptr();
  const int64_t rows = B * Sq * H;
  auto launch = [&](auto tag) {
    using T = decltype(tag);
    auto dot = [&](auto dtag) {
      constexpr int DD = decltype(dtag)::value;
      attn_dot_kernel<T, DD><<<(unsigned)((rows + 7) / 8), 256, 0, stream()>>>(
          reinterpret_cast<const T*>(dout.data_ptr()), reinterpret_cast<const T*>(out.data_ptr()), di.data_ptr<float>(),
          (int)B, (int)Sq, (int)H);
    };
    switch ((int)D) {
      case 16: dot(std::integral_constant<int, 16>{}); break;
      case 32: dot(std::integral_constant<int, 32>{}); break;
      case 64: dot(std::integral_constant<int, 64>{}); break;
      case 96: dot(std::integral_constant<int, 96>{}); break;
      case 128:
        if (dout.is_contiguous() && out.is_contiguous() && reinterpret_cast<uintptr_t>(dout.data_ptr()) % 16 == 0 &&
            reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0) {
          const int64_t threads = rows * 8;
          attn_dot128_kernel<T><<<(unsigned)std::min<int64_t>((threads + 255) / 256, (int64_t)num_sms() * 8), 256, 0,
                                  stream()>>>(reinterpret_cast<const T*>(dout.data_ptr()),
                                              reinterpret_cast<const T*>(out.data_ptr()), di.data_ptr<float>(),
                                              (int)B, (int)Sq, (int)H);
        } else {
          dot(std::integral_constant<int, 128>{});
        }
        break;
      default: LRB_CHECK(false, "attention: unsupported head_dim");
    }
    LRB_LAUNCH_CHECK();
    if (Sq > 0 && Skv > 0) {
      if (sm100 && std::is_same<T, __nv_bfloat16>::value && D == 128)
        attn_bwd_sm100(dout, q, k, v, lse, di, dq_acc, dk, dv, causal, scale);
      else
        LRB_ATTN_DISPATCH_D((int)D, run_bwd, T, p);
    }
    const int64_t n = dq.numel();
    f32_to_kernel<T><<<(unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16), 256, 0, stream()>>>(
        dq_acc.data_ptr<float>(), reinterpret_cast<T*>(dq.data_ptr()), n);
    LRB_LAUNCH_CHECK();
  };
  if (q.scalar_type() == at::kBFloat16) launch(__nv_bfloat16{});
  else launch(__half{});
  if (Skv > 0 && Sq == 0) { dk.zero_(); dv.zero_(); }
  return {dq, dk, dv};
}

}  // namespace lrb
