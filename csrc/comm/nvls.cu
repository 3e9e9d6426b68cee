// NVSwitch multicast (NVLS) collectives: the reduction runs inside the switch.
//
// The buffers live in a multicast-capable symmetric allocation: every rank holds
// a copy at the same offset, reachable through its own unicast address, through
// each peer's unicast address (P2P over NVLink), and through ONE multicast
// address that names all copies at once.  Two PTX operations use that address:
//
//   multimem.ld_reduce  reads the element from every rank's copy and returns the
//                       sum (the switch adds the values: each GPU's memory is
//                       read once, the result crosses the link once);
//   multimem.st         writes the value into every rank's copy (the switch
//                       replicates the store).
//
// Synchronisation is by 32-bit epoch flags in the same allocation, written to a
// peer with a plain P2P release store at system scope after a system fence and
// polled locally with acquire loads.  Every poll is bounded: on expiry the
// kernel records an error code in a device word, skips its work and returns.
//
// Kernels:
//   nvls_all_reduce   in place, fp32 or bf16: ready barrier, each rank reduces
//                     its 1/world slice with ld_reduce and multicasts the scaled
//                     sum back with multimem.st, done barrier.
//   nvls_rs_stage     FSDP reduce-scatter, first half: the fp32 gradient
//                     accumulator is cast to bf16 into this rank's copy of the
//                     staging buffer (and zeroed); ready flags to every peer.
//   nvls_rs_reduce    second half: the owner ld_reduces its shard of the staging
//                     buffer (bf16 summed in fp32 inside the switch), scales,
//                     stores or accumulates the fp32 shard and adds the sum of
//                     squares (grad-norm partial); "consumed" flags to every peer.
//   nvls_ag_publish   FSDP all-gather: after the optimizer step every rank casts
//                     its fp32 master shard to bf16 and multicasts it into its slot
//                     of every rank's gathered-parameter buffer (one broadcast per
//                     optimizer step instead of a gather before every use).
//   nvls_diloco_outer DiLoCo's outer step in the all-reduce: mean pseudo-gradient
//                     from the switch, Nesterov (or heavy-ball) update of the
//                     slice's anchor and momentum, new anchor multicast to every rank.
//   nvls_wait         one block waiting for `world` local flags (the gather side).
//
// No TMA is used here (plain vector loads and multimem operations only).
#include "../common.cuh"

#include <cuda_bf16.h>

namespace lrb {
namespace {

constexpr long long kPollLimit = 1ll << 24;  // polls before a wait gives up (~1-2 s)
// Independent multimem reductions each thread keeps in flight: the switch round
// trip is microseconds, so one 16-byte request per thread leaves NVLink idle.
constexpr int kUnroll = 4;
enum : int { kErrReady = 41, kErrDone = 42, kErrFree = 43 };

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool reached(uint32_t flag, uint32_t epoch) { return (int32_t)(flag - epoch) >= 0; }

// ---- multimem operations on a multicast address (16 bytes per operation) ----
__device__ __forceinline__ float4 mm_ld_reduce_f32x4(uint64_t mc) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
// Eight bf16 values; the switch accumulates in fp32 and rounds the sum to bf16.
__device__ __forceinline__ uint4 mm_ld_reduce_bf16x8(uint64_t mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
__device__ __forceinline__ void mm_st_f32x4(uint64_t mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_st_bf16x8(uint64_t mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return r;
}
__device__ __forceinline__ void unpack8(const uint4& r, float* f) {
  const __nv_bfloat162* v = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(v[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ bool no_error(const int* err) {
  return *reinterpret_cast<const volatile int*>(err) == 0;
}

// Every thread t < n of the block polls local flag t until it reaches `epoch`.
// False for the whole block if any poll gave up (the code is recorded once).
__device__ bool block_wait(const uint32_t* flags, int n, uint32_t epoch, int* err, int code) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if ((int)threadIdx.x < n) {
    long long it = 0;
    while (!reached(ld_acquire_sys(flags + threadIdx.x), epoch)) {
      if (++it > kPollLimit) {
        atomicExch(&failed, 1);
        atomicCAS(err, 0, code);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  return failed == 0;
}

// One thread waits for n local flags (bounded).
__device__ void thread_wait(const uint32_t* flags, int n, uint32_t epoch, int* err, int code) {
  for (int t = 0; t < n; ++t) {
    long long it = 0;
    while (!reached(ld_acquire_sys(flags + t), epoch)) {
      if (++it > kPollLimit) {
        atomicCAS(err, 0, code);
        return;
      }
      __nanosleep(64);
    }
  }
}

// Thread t < world stores `epoch` into slot `rank` of peer t's flag array
// (heap offset `off`), after a system fence that publishes this rank's earlier
// writes (those of earlier kernels on the stream included).
__device__ __forceinline__ void signal_all(const uint64_t* bases, int64_t off, int rank, int world, uint32_t epoch,
                                           int t) {
  if (t < world) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(bases[t] + off) + rank, epoch);
  }
}

// One thread: slot `rank` of every peer's flag array at heap offset `off`.
__device__ __forceinline__ void signal_all_serial(const uint64_t* bases, int64_t off, int rank, int world,
                                                  uint32_t epoch) {
  __threadfence_system();
  for (int t = 0; t < world; ++t) st_release_sys(reinterpret_cast<uint32_t*>(bases[t] + off) + rank, epoch);
}

// True in exactly one thread of the last block to finish (the counter is reset).
// Every block calls it, also after a failed wait, so the count stays exact.
__device__ bool last_block(unsigned int* counter) {
  __shared__ bool last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(counter, 1u);
    last = (prev == gridDim.x - 1);
    if (last) *counter = 0u;
  }
  __syncthreads();
  return last && threadIdx.x == 0;
}

// ------------------------------------------------------------------ all-reduce
// Flags at `flag_off` of every rank: ready[world], done[world].  16-byte vectors
// [rank*per, (rank+1)*per) of the buffer are this rank's slice.
template <bool kBf16>
__global__ void __launch_bounds__(512) all_reduce_kernel(uint64_t mc_data, const uint64_t* __restrict__ bases,
                                                         int64_t flag_off, int64_t n16, int rank, int world,
                                                         uint32_t epoch, float scale, unsigned int* counter,
                                                         int* err) {
  uint32_t* flags = reinterpret_cast<uint32_t*>(bases[rank] + flag_off);
  if (blockIdx.x == 0) signal_all(bases, flag_off, rank, world, epoch, threadIdx.x);
  const bool ok = block_wait(flags, world, epoch, err, kErrReady);
  const int64_t per = (n16 + world - 1) / world;
  const int64_t lo = (int64_t)rank * per;
  const int64_t hi = ok ? min(n16, lo + per) : lo;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < hi; i0 += kUnroll * stride) {
    if constexpr (kBf16) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (i0 + u * stride < hi) v[u] = mm_ld_reduce_bf16x8(mc_data + (uint64_t)(i0 + u * stride) * 16u);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (i0 + u * stride >= hi) break;
        if (scale != 1.f) {
          float f[8];
          unpack8(v[u], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] *= scale;
          v[u] = pack8(f);
        }
        mm_st_bf16x8(mc_data + (uint64_t)(i0 + u * stride) * 16u, v[u]);
      }
    } else {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (i0 + u * stride < hi) v[u] = mm_ld_reduce_f32x4(mc_data + (uint64_t)(i0 + u * stride) * 16u);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (i0 + u * stride >= hi) break;
        float4 w = v[u];
        w.x *= scale; w.y *= scale; w.z *= scale; w.w *= scale;
        mm_st_f32x4(mc_data + (uint64_t)(i0 + u * stride) * 16u, w);
      }
    }
  }
  if (last_block(counter)) {
    // Every block of this rank has stored its slice: tell the peers, then wait
    // until every rank's slice has arrived here.
    if (no_error(err)) signal_all_serial(bases, flag_off + 4 * world, rank, world, epoch);
    thread_wait(flags + world, world, epoch, err, kErrDone);
  }
}

// DiLoCo outer step fused into the all-reduce: the buffer holds each rank's
// pseudo-gradient (anchor - local); for its slice a rank reads the mean
// pseudo-gradient d from the switch, updates its momentum shard m = mu m + d,
// takes the step a' = a - lr (d + mu m) on the anchor (Nesterov; a - lr m for
// heavy-ball) and multicasts a' -- afterwards every rank's buffer holds the new
// anchor.  momentum: this rank's slice only (per*4 floats).
__global__ void __launch_bounds__(512) diloco_kernel(uint64_t mc_data, const uint64_t* __restrict__ bases,
                                                     int64_t flag_off, int64_t n16, const float4* __restrict__ anchor,
                                                     float4* __restrict__ momentum, int rank, int world,
                                                     uint32_t epoch, float inv_world, float lr, float mu,
                                                     int nesterov, unsigned int* counter, int* err) {
  uint32_t* flags = reinterpret_cast<uint32_t*>(bases[rank] + flag_off);
  if (blockIdx.x == 0) signal_all(bases, flag_off, rank, world, epoch, threadIdx.x);
  const bool ok = block_wait(flags, world, epoch, err, kErrReady);
  const int64_t per = (n16 + world - 1) / world;
  const int64_t lo = (int64_t)rank * per;
  const int64_t hi = ok ? min(n16, lo + per) : lo;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < hi; i0 += kUnroll * stride) {
    float4 dv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (i0 + u * stride < hi) dv[u] = mm_ld_reduce_f32x4(mc_data + (uint64_t)(i0 + u * stride) * 16u);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= hi) break;
      float4 d = dv[u];
      d.x *= inv_world; d.y *= inv_world; d.z *= inv_world; d.w *= inv_world;
      float4 m = momentum[i - lo];
      m.x = mu * m.x + d.x; m.y = mu * m.y + d.y; m.z = mu * m.z + d.z; m.w = mu * m.w + d.w;
      momentum[i - lo] = m;
      float4 a = anchor[i];
      if (nesterov) {
        a.x -= lr * (d.x + mu * m.x); a.y -= lr * (d.y + mu * m.y);
        a.z -= lr * (d.z + mu * m.z); a.w -= lr * (d.w + mu * m.w);
      } else {
        a.x -= lr * m.x; a.y -= lr * m.y; a.z -= lr * m.z; a.w -= lr * m.w;
      }
      mm_st_f32x4(mc_data + (uint64_t)i * 16u, a);
    }
  }
  if (last_block(counter)) {
    if (no_error(err)) signal_all_serial(bases, flag_off + 4 * world, rank, world, epoch);
    thread_wait(flags + world, world, epoch, err, kErrDone);
  }
}

// -------------------------------------------------------------- reduce-scatter
// stage: this rank's copy of the bf16 staging buffer (world*shard elements).
// consumed: local flags [world], written by each peer once it has read its
// shard of every copy for an epoch; ready_off: heap offset of ready[world].
__global__ void __launch_bounds__(512) rs_stage_kernel(float* __restrict__ src, uint4* __restrict__ stage, int64_t n8,
                                                       const uint32_t* consumed, const uint64_t* __restrict__ bases,
                                                       int64_t ready_off, int rank, int world, uint32_t epoch,
                                                       unsigned int* counter, int* err) {
  const bool ok = block_wait(consumed, world, epoch - 1, err, kErrFree);
  const int64_t n = ok ? n8 : 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float4* p = reinterpret_cast<float4*>(src) + 2 * i;
    const float4 a = p[0], b = p[1];
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    stage[i] = pack8(f);
    p[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    p[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (last_block(counter) && no_error(err)) signal_all_serial(bases, ready_off, rank, world, epoch);
}

__global__ void __launch_bounds__(512) rs_reduce_kernel(uint64_t mc_shard, float* __restrict__ dst, int64_t s8,
                                                        float scale, int accumulate, const uint32_t* ready,
                                                        const uint64_t* __restrict__ bases, int64_t consumed_off,
                                                        int rank, int world, uint32_t epoch, float* sumsq,
                                                        unsigned int* counter, int* err) {
  const bool ok = block_wait(ready, world, epoch, err, kErrReady);
  const int64_t n = ok ? s8 : 0;
  float local = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t j0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j0 < n; j0 += kUnroll * stride) {
    uint4 rv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (j0 + u * stride < n) rv[u] = mm_ld_reduce_bf16x8(mc_shard + (uint64_t)(j0 + u * stride) * 16u);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t j = j0 + u * stride;
      if (j >= n) break;
      float f[8];
      unpack8(rv[u], f);
      float4* o = reinterpret_cast<float4*>(dst) + 2 * j;
      float4 a = make_float4(f[0] * scale, f[1] * scale, f[2] * scale, f[3] * scale);
      float4 b = make_float4(f[4] * scale, f[5] * scale, f[6] * scale, f[7] * scale);
      if (accumulate) {
        const float4 oa = o[0], ob = o[1];
        a.x += oa.x; a.y += oa.y; a.z += oa.z; a.w += oa.w;
        b.x += ob.x; b.y += ob.y; b.z += ob.z; b.w += ob.w;
      }
      o[0] = a;
      o[1] = b;
      local += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
    }
  }
  __shared__ float red[32];
  const float tot = block_sum(local, red);
  if (threadIdx.x == 0 && sumsq != nullptr) atomicAdd(sumsq, tot);
  if (last_block(counter) && no_error(err)) signal_all_serial(bases, consumed_off, rank, world, epoch);
}

// ------------------------------------------------------------------ all-gather
// agfree: local flags [world] (peer r has stopped reading the gathered weights
// of epoch-1); agready_off: heap offset of ready[world].
__global__ void __launch_bounds__(512) ag_publish_kernel(const float* __restrict__ master, uint64_t mc_slot,
                                                         int64_t s8, const uint32_t* agfree,
                                                         const uint64_t* __restrict__ bases, int64_t agfree_off,
                                                         int64_t agready_off, int rank, int world, uint32_t epoch,
                                                         unsigned int* counter, int* err) {
  // This kernel follows the optimizer step, so this rank no longer reads the
  // previous weights: say so, then wait for every peer to say the same.
  if (blockIdx.x == 0) signal_all(bases, agfree_off, rank, world, epoch - 1, threadIdx.x);
  const bool ok = block_wait(agfree, world, epoch - 1, err, kErrFree);
  const int64_t n = ok ? s8 : 0;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x) {
    const float4* p = reinterpret_cast<const float4*>(master) + 2 * j;
    const float4 a = p[0], b = p[1];
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    mm_st_bf16x8(mc_slot + (uint64_t)j * 16u, pack8(f));
  }
  if (last_block(counter) && no_error(err)) signal_all_serial(bases, agready_off, rank, world, epoch);
}

__global__ void wait_kernel(const uint32_t* flags, int world, uint32_t epoch, int* err) {
  block_wait(flags, world, epoch, err, kErrReady);
}

inline int grid_cap(int64_t work, int threads) {
  const int64_t want = (work + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, 2 * (int64_t)num_sms()));
}

const uint64_t* dev_bases(const at::Tensor& bases, int64_t world) {
  LRB_CHECK(bases.is_cuda() && bases.scalar_type() == at::kLong && bases.is_contiguous() && bases.numel() == world,
            "nvls: bases must be a contiguous int64 CUDA tensor of world peer addresses");
  return reinterpret_cast<const uint64_t*>(bases.data_ptr<int64_t>());
}
unsigned int* ctr(at::Tensor& c) {
  LRB_CHECK(c.is_cuda() && c.scalar_type() == at::kInt && c.numel() >= 1, "nvls: counter must be an int32 CUDA tensor");
  return reinterpret_cast<unsigned int*>(c.data_ptr<int>());
}
int* errp(at::Tensor& e) {
  LRB_CHECK(e.is_cuda() && e.scalar_type() == at::kInt && e.numel() >= 1, "nvls: err must be an int32 CUDA tensor");
  return e.data_ptr<int>();
}
const uint32_t* flags_of(const at::Tensor& f, int64_t world) {
  LRB_CHECK(f.is_cuda() && f.scalar_type() == at::kInt && f.numel() >= world && f.is_contiguous(),
            "nvls: flag view must be int32 with at least world entries");
  return reinterpret_cast<const uint32_t*>(f.data_ptr<int>());
}
void check_world(int64_t rank, int64_t world) {
  LRB_CHECK(world >= 1 && world <= 64 && rank >= 0 && rank < world, "nvls: rank / world out of range");
}

}  // namespace

// In-place all-reduce (sum times `scale`) of the buffer at multicast address
// `mc_data` (fp32 or bf16).  `data` is this rank's view of the same buffer
// (device, dtype and size).  The flag area at heap offset `flag_off` holds
// 2*world u32 words.
void nvls_all_reduce(at::Tensor& data, int64_t mc_data, const at::Tensor& bases, int64_t flag_off, int64_t rank,
                     int64_t world, int64_t epoch, double scale, at::Tensor& counter, at::Tensor& err) {
  check_world(rank, world);
  const bool bf = data.scalar_type() == at::kBFloat16;
  LRB_CHECK(bf || data.scalar_type() == at::kFloat, "nvls_all_reduce: fp32 or bf16");
  const int64_t bytes = data.numel() * data.element_size();
  LRB_CHECK(data.is_contiguous() && bytes % 16 == 0 && mc_data % 16 == 0 && flag_off % 4 == 0,
            "nvls_all_reduce: 16-byte multiples and alignment required");
  c10::cuda::CUDAGuard g(data.device());
  const int64_t n16 = bytes / 16;
  const int grid = grid_cap((n16 + world - 1) / world, 512);
  if (bf)
    all_reduce_kernel<true><<<grid, 512, 0, stream()>>>((uint64_t)mc_data, dev_bases(bases, world), flag_off, n16,
                                                        (int)rank, (int)world, (uint32_t)epoch, (float)scale,
                                                        ctr(counter), errp(err));
  else
    all_reduce_kernel<false><<<grid, 512, 0, stream()>>>((uint64_t)mc_data, dev_bases(bases, world), flag_off, n16,
                                                         (int)rank, (int)world, (uint32_t)epoch, (float)scale,
                                                         ctr(counter), errp(err));
  LRB_LAUNCH_CHECK();
}

// One DiLoCo outer step (see diloco_kernel).  `data`: this rank's view of the
// multicast buffer holding anchor - local (fp32); `anchor`: the replicated fp32
// anchor (read only; the new anchor is left in `data`); `momentum`: this
// rank's slice, ceil(numel/4/world)*4 floats.
void nvls_diloco_outer(at::Tensor& data, int64_t mc_data, const at::Tensor& bases, int64_t flag_off,
                       const at::Tensor& anchor, at::Tensor& momentum, int64_t rank, int64_t world, int64_t epoch,
                       double lr, double mu, bool nesterov, at::Tensor& counter, at::Tensor& err) {
  check_world(rank, world);
  const int64_t n = data.numel();
  LRB_CHECK(data.scalar_type() == at::kFloat && data.is_contiguous() && n % 4 == 0 && mc_data % 16 == 0,
            "nvls_diloco_outer: data must be contiguous fp32 with numel a multiple of 4");
  LRB_CHECK(anchor.scalar_type() == at::kFloat && anchor.is_contiguous() && anchor.numel() == n,
            "nvls_diloco_outer: anchor must match data");
  const int64_t n16 = n / 4;
  const int64_t per = (n16 + world - 1) / world;
  LRB_CHECK(momentum.scalar_type() == at::kFloat && momentum.is_contiguous() && momentum.numel() == per * 4,
            "nvls_diloco_outer: momentum must hold this rank's slice (", per * 4, " floats)");
  c10::cuda::CUDAGuard g(data.device());
  diloco_kernel<<<grid_cap(per, 512), 512, 0, stream()>>>(
      (uint64_t)mc_data, dev_bases(bases, world), flag_off, n16,
      reinterpret_cast<const float4*>(anchor.data_ptr<float>()), reinterpret_cast<float4*>(momentum.data_ptr<float>()),
      (int)rank, (int)world, (uint32_t)epoch, 1.f / (float)world, (float)lr, (float)mu, nesterov ? 1 : 0, ctr(counter),
      errp(err));
  LRB_LAUNCH_CHECK();
}

void nvls_rs_stage(at::Tensor& src, at::Tensor& stage, const at::Tensor& consumed, const at::Tensor& bases,
                   int64_t ready_off, int64_t rank, int64_t world, int64_t epoch, at::Tensor& counter,
                   at::Tensor& err) {
  check_world(rank, world);
  LRB_CHECK(src.is_cuda() && src.scalar_type() == at::kFloat && src.is_contiguous() && src.numel() % (8 * world) == 0,
            "nvls_rs_stage: src must be contiguous fp32 with numel a multiple of 8*world");
  LRB_CHECK(stage.scalar_type() == at::kBFloat16 && stage.is_contiguous() && stage.numel() == src.numel() &&
                reinterpret_cast<uintptr_t>(stage.data_ptr()) % 16 == 0,
            "nvls_rs_stage: stage must be this rank's 16-byte aligned bf16 copy of src's size");
  c10::cuda::CUDAGuard g(src.device());
  const int64_t n8 = src.numel() / 8;
  rs_stage_kernel<<<grid_cap(n8, 512), 512, 0, stream()>>>(
      src.data_ptr<float>(), reinterpret_cast<uint4*>(stage.data_ptr()), n8, flags_of(consumed, world),
      dev_bases(bases, world), ready_off, (int)rank, (int)world, (uint32_t)epoch, ctr(counter), errp(err));
  LRB_LAUNCH_CHECK();
}

// mc_stage: multicast address of the staging buffer's first element.
void nvls_rs_reduce(int64_t mc_stage, at::Tensor& dst, double scale, bool accumulate, const at::Tensor& ready,
                    const at::Tensor& bases, int64_t consumed_off, int64_t rank, int64_t world, int64_t epoch,
                    c10::optional<at::Tensor> sumsq, at::Tensor& counter, at::Tensor& err) {
  check_world(rank, world);
  const int64_t shard = dst.numel();
  LRB_CHECK(dst.is_cuda() && dst.scalar_type() == at::kFloat && dst.is_contiguous() && shard % 8 == 0,
            "nvls_rs_reduce: dst must be contiguous fp32 with numel a multiple of 8");
  LRB_CHECK(mc_stage % 16 == 0, "nvls_rs_reduce: staging buffer must be 16-byte aligned");
  c10::cuda::CUDAGuard g(dst.device());
  const int64_t s8 = shard / 8;
  rs_reduce_kernel<<<grid_cap(s8, 512), 512, 0, stream()>>>(
      (uint64_t)mc_stage + (uint64_t)(rank * shard * 2), dst.data_ptr<float>(), s8, (float)scale, accumulate ? 1 : 0,
      flags_of(ready, world), dev_bases(bases, world), consumed_off, (int)rank, (int)world, (uint32_t)epoch,
      sumsq ? sumsq->data_ptr<float>() : nullptr, ctr(counter), errp(err));
  LRB_LAUNCH_CHECK();
}

// mc_gathered: multicast address of the gathered bf16 buffer (world*shard
// elements); this rank writes slot `rank`.
void nvls_ag_publish(const at::Tensor& master, int64_t mc_gathered, const at::Tensor& agfree, const at::Tensor& bases,
                     int64_t agfree_off, int64_t agready_off, int64_t rank, int64_t world, int64_t epoch,
                     at::Tensor& counter, at::Tensor& err) {
  check_world(rank, world);
  const int64_t shard = master.numel();
  LRB_CHECK(master.is_cuda() && master.scalar_type() == at::kFloat && master.is_contiguous() && shard % 8 == 0,
            "nvls_ag_publish: master must be contiguous fp32 with numel a multiple of 8");
  LRB_CHECK(mc_gathered % 16 == 0, "nvls_ag_publish: gathered buffer must be 16-byte aligned");
  c10::cuda::CUDAGuard g(master.device());
  const int64_t s8 = shard / 8;
  ag_publish_kernel<<<grid_cap(s8, 512), 512, 0, stream()>>>(
      master.data_ptr<float>(), (uint64_t)mc_gathered + (uint64_t)(rank * shard * 2), s8, flags_of(agfree, world),
      dev_bases(bases, world), agfree_off, agready_off, (int)rank, (int)world, (uint32_t)epoch, ctr(counter),
      errp(err));
  LRB_LAUNCH_CHECK();
}

void nvls_wait(const at::Tensor& flags, int64_t world, int64_t epoch, at::Tensor& err) {
  LRB_CHECK(world >= 1 && world <= 64, "nvls_wait: world out of range");
  c10::cuda::CUDAGuard g(flags.device());
  wait_kernel<<<1, 64, 0, stream()>>>(flags_of(flags, world), (int)world, (uint32_t)epoch, errp(err));
  LRB_LAUNCH_CHECK();
}

}  // namespace lrb
