// INT4 absmax (reference-compatible) and NVFP4 (E2M1 + e4m3 block scale +
// fp32 tensor scale) quantisation kernels.
#include "../common.cuh"

#include <cuda_fp8.h>

namespace lrb {
namespace {

// ---------------------------------------------------------------- INT4
// One warp per (row, group).
template <typename T>
__global__ void int4_quant_kernel(const T* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scales,
                                  int64_t M, int D, int G, int ng) {
  const int lane = threadIdx.x & 31;
  const int64_t job = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (job >= M * ng) return;
  const int64_t row = job / ng;
  const int grp = (int)(job - row * ng);
  const int c0 = grp * G, c1 = min(c0 + G, D);
  float amax = 0.f;
  for (int c = c0 + lane; c < c1; c += 32) amax = fmaxf(amax, fabsf(to_f(x[row * D + c])));
  amax = warp_max(amax);
  const float s = fmaxf(amax / 7.f, 1e-10f);
  if (lane == 0) scales[job] = s;
  for (int c = c0 + lane; c < c1; c += 32) {
    float v = rintf(to_f(x[row * D + c]) / s);  // round half to even, like torch.round
    v = fminf(fmaxf(v, -8.f), 7.f);
    q[row * D + c] = (int8_t)v;
  }
}

__global__ void int4_dequant_kernel(const int8_t* __restrict__ q, const float* __restrict__ scales,
                                    float* __restrict__ out, int64_t M, int D, int G, int ng) {
  const int64_t n = M * (int64_t)D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / D;
    const int c = (int)(i - row * D);
    out[i] = (float)q[i] * scales[row * ng + c / G];
  }
}

// ---------------------------------------------------------------- NVFP4
__device__ __forceinline__ uint32_t hash3(uint32_t a, uint32_t b, uint32_t c) {
  // splitmix-style integer hash (Steele, Lea, Flood 2014) for stochastic rounding.
  uint64_t z = ((uint64_t)a << 32 | b) + 0x9E3779B97F4A7C15ull * (c + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return (uint32_t)(z ^ (z >> 31));
}

__device__ __forceinline__ float e2m1_value(int code) {
  const float grid[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  return grid[code & 7];
}

// magnitude -> code 0..7, round to nearest, ties to even code
__device__ __forceinline__ int e2m1_rne(float a) {
  a = fminf(a, 6.f);
  const float grid[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  int lo = 0;
#pragma unroll
  for (int i = 1; i < 8; ++i) lo = (a >= grid[i]) ? i : lo;
  if (lo == 7) return 7;
  const float dl = a - grid[lo], dh = grid[lo + 1] - a;
  if (dh < dl) return lo + 1;
  if (dh > dl) return lo;
  return ((lo + 1) % 2 == 0) ? lo + 1 : lo;
}

__device__ __forceinline__ int e2m1_stochastic(float a, float r) {
  a = fminf(a, 6.f);
  const float grid[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  int lo = 0;
#pragma unroll
  for (int i = 1; i < 8; ++i) lo = (a >= grid[i]) ? i : lo;
  if (lo == 7) return 7;
  const float p = (a - grid[lo]) / (grid[lo + 1] - grid[lo]);
  return r < p ? lo + 1 : lo;
}

template <typename T>
__global__ void absmax_kernel(const T* __restrict__ x, int64_t n, float* __restrict__ out) {
  __shared__ float red[32];
  float m = 0.f;
  constexpr int V = 16 / sizeof(T);
  const int64_t nv = (reinterpret_cast<uintptr_t>(x) % 16 == 0) ? n / V : 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += stride) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(x) + i);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < V; ++j) m = fmaxf(m, fabsf(to_f(e[j])));
  }
  for (int64_t i = nv * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    m = fmaxf(m, fabsf(to_f(x[i])));
  m = block_max(m, red);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(out), __float_as_int(m));  // m >= 0: int order == float order
}

// One thread per 16-element block.
template <typename T>
__global__ void nvfp4_quant_kernel(const T* __restrict__ x, const float* __restrict__ amax, uint8_t* __restrict__ packed,
                                   __nv_fp8_e4m3* __restrict__ sb, float* __restrict__ st_out, int64_t nblocks,
                                   bool stochastic, uint32_t seed) {
  const float st = fmaxf(amax[0] / (6.f * 448.f), 1e-12f);
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b == 0) st_out[0] = st;
  if (b >= nblocks) return;
  const T* xp = x + b * 16;
  float v[16], bm = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) { v[i] = to_f(xp[i]); bm = fmaxf(bm, fabsf(v[i])); }
  const __nv_fp8_e4m3 s8(fminf(bm / (6.f * st), 448.f));
  sb[b] = s8;
  const float inv = 1.f / fmaxf(float(s8) * st, 1e-30f);  // one reciprocal per block
  uint8_t out[8];
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    int c[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float y = v[i + j] * inv;
      const float a = fabsf(y);
      int code;
      if (stochastic) {
        const float r = (hash3(seed, (uint32_t)(b >> 32), (uint32_t)(b * 16 + i + j)) >> 8) * (1.f / 16777216.f);
        code = e2m1_stochastic(a, r);
      } else {
        code = e2m1_rne(a);
      }
      if (y < 0.f && code > 0) code |= 8;
      c[j] = code;
    }
    out[i / 2] = (uint8_t)(c[0] | (c[1] << 4));
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) packed[b * 8 + i] = out[i];
}


// Two fp32 values -> one byte of E2M1 codes (lo in the low nibble), round to
// nearest even with saturation to +-6: the hardware conversion, which rounds
// as e2m1_rne does (ties to the even code; the one-thread-per-block quantiser
// keeps the software rounding and serves as the check).
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint32_t out;
  asm("{\n.reg .b8 t;\ncvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\ncvt.u32.u8 %0, t;\n}" : "=r"(out) : "f"(lo), "f"(hi));
  return out;
}

// A value that rounds to zero keeps no sign: -0 nibbles (0x8) become 0x0.
__device__ __forceinline__ uint32_t clear_negative_zero(uint32_t w) {
  const uint32_t mag = w & 0x77777777u;
  return mag | ((mag + 0x77777777u) & 0x88888888u & w);
}

// 32-bit integer mixer ("lowbias32", C. Wellons' hash-prospector): two 32-bit
// multiplies per call, so the stochastic-rounding draws stay cheap next to the
// 64-bit splitmix hash of the one-block-per-thread quantiser.
__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

template <bool SR>
__device__ __forceinline__ void quant_block16(const float* v, float st, uint32_t seed, uint32_t hi, uint32_t idx0,
                                              uint8_t& sbyte, uint2& packed) {
  float bm = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bm = fmaxf(bm, fabsf(v[i]));
  const __nv_fp8_e4m3 s8(fminf(bm / (6.f * st), 448.f));
  sbyte = s8.__x;
  const float inv = 1.f / fmaxf(float(s8) * st, 1e-30f);
  uint32_t w[2] = {0u, 0u};
  if constexpr (!SR) {
#pragma unroll
    for (int i = 0; i < 16; i += 2) w[i >> 3] |= cvt_e2m1x2(v[i] * inv, v[i + 1] * inv) << (4 * (i & 7));
    packed = make_uint2(clear_negative_zero(w[0]), clear_negative_zero(w[1]));
  } else {
    // the hardware stochastic-rounding conversion, four values per instruction
    // (cvt.rs: the random bits come from one 32-bit draw per group of four; the
    // first operand lands in the highest nibble, as in cvt.rn ... e2m1x2)
    const uint32_t key = mix32(seed ^ mix32(hi + 0x9e3779b9u));
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const uint32_t rb = mix32(key ^ ((idx0 + (uint32_t)i) >> 2));
      uint16_t d;
      asm("cvt.rs.satfinite.e2m1x4.f32 %0, {%1, %2, %3, %4}, %5;"
          : "=h"(d)
          : "f"(v[i + 3] * inv), "f"(v[i + 2] * inv), "f"(v[i + 1] * inv), "f"(v[i] * inv), "r"(rb));
      w[i >> 3] |= (uint32_t)d << (4 * (i & 7));
    }
    packed = make_uint2(clear_negative_zero(w[0]), clear_negative_zero(w[1]));
  }
}

// Byte offset of the scale of (row, 16-element block jb) in the tensor-core
// scale-factor layout: 512-byte atoms of 128 rows x 4 blocks, atoms ordered
// K-fastest inside each 128-row band, byte 16*(r%32) + 4*(r/32) + jb%4.
__device__ __forceinline__ int64_t sf_atom_offset(int64_t row, int64_t jb, int64_t kblocks64) {
  const int r = (int)(row & 127);
  return ((row >> 7) * kblocks64 + (jb >> 2)) * 512 + 16 * (r & 31) + 4 * (r >> 5) + (int)(jb & 3);
}

// Tile of 128 rows x 64 columns of x (M, K) per CTA, 256 threads.
// ROW: x quantised along K -> packed (M, K/2), scales in atom layout (M/128, K/64, 512).
// COL: x^T quantised along M -> packed (K, M/2), scales (K/128, M/64, 512).
template <typename T, bool ROW, bool COL, bool SR>
__global__ void __launch_bounds__(256) nvfp4_quant_dual_kernel(
    const T* __restrict__ x, int64_t M, int64_t K, const float* __restrict__ amax, uint8_t* __restrict__ pr,
    uint8_t* __restrict__ ar, uint8_t* __restrict__ pc, uint8_t* __restrict__ ac, float* __restrict__ st_out,
    uint32_t seed) {
  __shared__ float tile[128][65];
  const int64_t m0 = (int64_t)blockIdx.y * 128, k0 = (int64_t)blockIdx.x * 64;
  const float st = fmaxf(amax[0] / (6.f * 448.f), 1e-12f);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) st_out[0] = st;
  const int t = threadIdx.x;
#pragma unroll
  for (int rep = 0; rep < 2; ++rep) {
    const int item = t + 256 * rep;
    const int row = item >> 2, j = item & 3;
    const T* src = x + (m0 + row) * K + k0 + j * 16;
    float v[16];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src) + h);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[h * 8 + i] = to_f(e[i]);
    }
    if (COL) {
#pragma unroll
      for (int i = 0; i < 16; ++i) tile[row][j * 16 + i] = v[i];
    }
    if (ROW) {
      const int64_t e0 = (m0 + row) * K + k0 + j * 16;
      uint8_t sb;
      uint2 pk;
      quant_block16<SR>(v, st, seed, (uint32_t)(e0 >> 32), (uint32_t)e0, sb, pk);
      *reinterpret_cast<uint2*>(pr + ((m0 + row) * K + k0 + j * 16) / 2) = pk;
      ar[sf_atom_offset(m0 + row, (k0 >> 4) + j, K >> 6)] = sb;
    }
  }
  if (COL) {
    __syncthreads();
#pragma unroll
    for (int rep = 0; rep < 2; ++rep) {
      const int item = t + 256 * rep;
      const int k = item & 63, mb = item >> 6;
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = tile[mb * 16 + i][k];
      const int64_t kr = k0 + k, mc = m0 + mb * 16;
      const int64_t e0 = kr * M + mc;  // element index of x^T
      uint8_t sb;
      uint2 pk;
      quant_block16<SR>(v, st, seed ^ 0x5bd1e995u, (uint32_t)(e0 >> 32), (uint32_t)e0, sb, pk);
      *reinterpret_cast<uint2*>(pc + (kr * M + mc) / 2) = pk;
      ac[sf_atom_offset(kr, mc >> 4, M >> 6)] = sb;
    }
  }
}

template <typename O>
__global__ void nvfp4_dequant_kernel(const uint8_t* __restrict__ packed, const __nv_fp8_e4m3* __restrict__ sb,
                                     const float* __restrict__ st, O* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t byte = packed[i >> 1];
    const int code = (i & 1) ? (byte >> 4) : (byte & 15);
    float v = e2m1_value(code);
    if (code & 8) v = -v;
    out[i] = from_f<O>(v * float(sb[i >> 4]) * st[0]);
  }
}

}  // namespace

std::tuple<at::Tensor, at::Tensor> int4_quantize(const at::Tensor& x, int64_t G) {
  LRB_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "int4_quantize: 2-D contiguous CUDA input");
  c10::cuda::CUDAGuard g(x.device());
  bind_device(x.get_device());
  const int64_t M = x.size(0);
  const int D = (int)x.size(1);
  const int ng = (int)((D + G - 1) / G);
  auto q = at::empty({M, D}, x.options().dtype(at::kChar));
  auto s = at::empty({M, ng}, x.options().dtype(at::kFloat));
  if (M * ng == 0) return {q, s};
  LRB_DISPATCH_FLOAT(x.scalar_type(), T, [&] {
    int4_quant_kernel<T><<<(unsigned)((M * ng + 7) / 8), 256, 0, stream()>>>(
        reinterpret_cast<const T*>(x.data_ptr()), q.data_ptr<int8_t>(), s.data_ptr<float>(), M, D, (int)G, ng);
  });
  LRB_LAUNCH_CHECK();
  return {q, s};
}

at::Tensor int4_dequantize(const at::Tensor& q, const at::Tensor& s, int64_t G) {
  c10::cuda::CUDAGuard g(q.device());
  bind_device(q.get_device());
  const int64_t M = q.size(0);
  const int D = (int)q.size(1);
  auto out = at::empty({M, D}, q.options().dtype(at::kFloat));
  const int64_t n = M * D;
  if (n == 0) return out;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16);
  int4_dequant_kernel<<<blocks, 256, 0, stream()>>>(q.data_ptr<int8_t>(), s.data_ptr<float>(), out.data_ptr<float>(),
                                                    M, D, (int)G, (int)s.size(1));
  LRB_LAUNCH_CHECK();
  return out;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> nvfp4_quantize(const at::Tensor& x, bool stochastic, int64_t seed) {
  LRB_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() && x.size(1) % 16 == 0, "nvfp4_quantize: (M, K%16==0)");
  c10::cuda::CUDAGuard g(x.device());
  bind_device(x.get_device());
  const int64_t M = x.size(0), K = x.size(1);
  auto packed = at::empty({M, K / 2}, x.options().dtype(at::kByte));
  auto sb = at::empty({M, K / 16}, x.options().dtype(at::kFloat8_e4m3fn));
  auto st = at::empty({}, x.options().dtype(at::kFloat));
  auto amax = at::zeros({1}, x.options().dtype(at::kFloat));
  const int64_t n = M * K, nb = n / 16;
  if (n == 0) return {packed, sb, st};
  LRB_DISPATCH_FLOAT(x.scalar_type(), T, [&] {
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 8);
    absmax_kernel<T><<<blocks, 256, 0, stream()>>>(reinterpret_cast<const T*>(x.data_ptr()), n, amax.data_ptr<float>());
    LRB_LAUNCH_CHECK();
    nvfp4_quant_kernel<T><<<(unsigned)((nb + 255) / 256), 256, 0, stream()>>>(
        reinterpret_cast<const T*>(x.data_ptr()), amax.data_ptr<float>(), packed.data_ptr<uint8_t>(),
        reinterpret_cast<__nv_fp8_e4m3*>(sb.data_ptr()), st.data_ptr<float>(), nb, stochastic, (uint32_t)seed);
  });
  LRB_LAUNCH_CHECK();
  return {packed, sb, st};
}

// x (M, K) bf16/fp16/fp32 -> {packed_row (M, K/2), atoms_row (M/128, K/64, 512),
// packed_col (K, M/2), atoms_col (K/128, M/64, 512), tensor scale}. The per-tensor
// amax is computed here unless given (x and x^T share it).
std::vector<at::Tensor> nvfp4_quantize_dual(const at::Tensor& x, const c10::optional<at::Tensor>& amax_in,
                                            bool rowwise, bool colwise, bool stochastic, int64_t seed) {
  LRB_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "nvfp4_quantize_dual: 2-D contiguous CUDA input");
  const int64_t M = x.size(0), K = x.size(1);
  LRB_CHECK(M % 128 == 0 && K % 128 == 0, "nvfp4_quantize_dual: M and K multiples of 128");
  LRB_CHECK(rowwise || colwise, "nvfp4_quantize_dual: nothing requested");
  c10::cuda::CUDAGuard g(x.device());
  bind_device(x.get_device());
  auto u8 = x.options().dtype(at::kByte);
  at::Tensor pr, ar, pc, ac;
  if (rowwise) {
    pr = at::empty({M, K / 2}, u8);
    ar = at::empty({M / 128, K / 64, 512}, u8);
  }
  if (colwise) {
    pc = at::empty({K, M / 2}, u8);
    ac = at::empty({K / 128, M / 64, 512}, u8);
  }
  auto st = at::empty({}, x.options().dtype(at::kFloat));
  at::Tensor amax;
  if (amax_in.has_value()) {
    amax = *amax_in;
    LRB_CHECK(amax.is_cuda() && amax.scalar_type() == at::kFloat && amax.numel() == 1, "nvfp4_quantize_dual: amax");
  } else {
    amax = at::empty({1}, x.options().dtype(at::kFloat));
    AT_CUDA_CHECK(cudaMemsetAsync(amax.data_ptr(), 0, sizeof(float), stream()));
  }
  const int64_t n = M * K;
  const dim3 grid((unsigned)(K / 64), (unsigned)(M / 128));
  LRB_DISPATCH_FLOAT(x.scalar_type(), T, [&] {
    if (!amax_in.has_value()) {
      const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 8);
      absmax_kernel<T><<<blocks, 256, 0, stream()>>>(reinterpret_cast<const T*>(x.data_ptr()), n,
                                                      amax.data_ptr<float>());
      LRB_LAUNCH_CHECK();
    }
    auto* xp = reinterpret_cast<const T*>(x.data_ptr());
    uint8_t* p0 = rowwise ? pr.data_ptr<uint8_t>() : nullptr;
    uint8_t* a0 = rowwise ? ar.data_ptr<uint8_t>() : nullptr;
    uint8_t* p1 = colwise ? pc.data_ptr<uint8_t>() : nullptr;
    uint8_t* a1 = colwise ? ac.data_ptr<uint8_t>() : nullptr;
    auto launch = [&](auto kern) {
      kern<<<grid, 256, 0, stream()>>>(xp, M, K, amax.data_ptr<float>(), p0, a0, p1, a1, st.data_ptr<float>(),
                                       (uint32_t)seed);
    };
    if (stochastic) {
      if (rowwise && colwise) launch(nvfp4_quant_dual_kernel<T, true, true, true>);
      else if (rowwise) launch(nvfp4_quant_dual_kernel<T, true, false, true>);
      else launch(nvfp4_quant_dual_kernel<T, false, true, true>);
    } else {
      if (rowwise && colwise) launch(nvfp4_quant_dual_kernel<T, true, true, false>);
      else if (rowwise) launch(nvfp4_quant_dual_kernel<T, true, false, false>);
      else launch(nvfp4_quant_dual_kernel<T, false, true, false>);
    }
  });
  LRB_LAUNCH_CHECK();
  return {pr, ar, pc, ac, st};
}

at::Tensor nvfp4_dequantize(const at::Tensor& packed, const at::Tensor& sb, const at::Tensor& st,
                            at::ScalarType dtype) {
  c10::cuda::CUDAGuard g(packed.device());
  bind_device(packed.get_device());
  const int64_t M = packed.size(0), K = packed.size(1) * 2;
  auto out = at::empty({M, K}, packed.options().dtype(dtype));
  const int64_t n = M * K;
  if (n == 0) return out;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16);
  LRB_DISPATCH_FLOAT(dtype, O, [&] {
    nvfp4_dequant_kernel<O><<<blocks, 256, 0, stream()>>>(packed.data_ptr<uint8_t>(),
                                                          reinterpret_cast<const __nv_fp8_e4m3*>(sb.data_ptr()),
                                                          st.data_ptr<float>(), reinterpret_cast<O*>(out.data_ptr()), n);
  });
  LRB_LAUNCH_CHECK();
  return out;
}

}  // namespace lrb
