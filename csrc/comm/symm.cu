// Symmetric device memory for the ranks of one node, and the collective
// kernels that run on it.
//
// Each rank cudaMalloc's one heap and exports it with a CUDA IPC handle; the
// handles are exchanged over the process group's store (Python side) and every
// rank opens its peers' heaps, so a kernel can load from and store to another
// GPU's heap through NVLink with plain ld/st (no multicast object, no NVLS).
// Buffers inside the heap sit at the same offset on every rank.
//
// Synchronisation is by 32-bit epoch flags in the heaps: a writer stores its
// data, fences at system scope and then stores the flag with release
// semantics; a reader polls the flag with acquire loads.  Every poll is
// bounded: on expiry the kernel records an error code in a device word, skips
// its work and returns (the host raises).
//
// Kernels:
//   rs_push      fp32 gradient -> bf16, written into slot `rank` of each owner's
//                receive area (the owner of elements [r*shard, (r+1)*shard) is
//                rank r); the source is zeroed in the same pass.
//   rs_reduce    owner side: sum of the world slots in fp32, times `scale`,
//                stored or accumulated into the fp32 shard, plus the sum of
//                squares of the result (grad-norm partial).
//   ag_publish   fp32 master shard -> bf16 into this rank's heap shard.
//   ag_pull      gather the bf16 shards of all ranks into a local full buffer.
//   diloco_push / diloco_reduce_nesterov / f32 pull: the DiLoCo outer step.
#include "../common.cuh"

#include <cuda_bf16.h>

namespace lrb {
namespace {

constexpr long long kPollLimit = 1ll << 24;  // polls before a wait gives up
enum : int { kErrPeerWait = 11, kErrSlotWait = 12 };

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Epochs only grow; "reached" tolerates wrap-around.
__device__ __forceinline__ bool reached(uint32_t flag, uint32_t epoch) { return (int32_t)(flag - epoch) >= 0; }

// Thread t < n of the block polls the u32 flag at offset `off` of rank t's
// heap until it reaches `epoch`.  Returns false (for the whole block) if any
// poll gave up.
__device__ bool block_wait_flags(const uint64_t* bases, int64_t off, int n, uint32_t epoch, int* err, int code) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if ((int)threadIdx.x < n) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(bases[threadIdx.x] + off);
    long long it = 0;
    while (!reached(ld_acquire_sys(f), epoch)) {
      if (++it > kPollLimit) {
        atomicExch(&failed, 1);
        if (err) atomicCAS(err, 0, code);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  return failed == 0;
}

// Same, for n flags laid out contiguously at one local address.
__device__ bool block_wait_local_flags(const uint32_t* flags, int n, uint32_t epoch, int* err, int code) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if ((int)threadIdx.x < n) {
    long long it = 0;
    while (!reached(ld_acquire_sys(flags + threadIdx.x), epoch)) {
      if (++it > kPollLimit) {
        atomicExch(&failed, 1);
        if (err) atomicCAS(err, 0, code);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  return failed == 0;
}

__device__ __forceinline__ bool no_error(const int* err) {
  return err == nullptr || *reinterpret_cast<const volatile int*>(err) == 0;
}

// True in exactly one thread of the last block to finish (the counter is reset).
// Every block must call it, also after a failed wait, so the counter stays exact.
__device__ bool last_block_done(unsigned int* counter) {
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

__device__ __forceinline__ uint4 pack8_bf16(const float* f) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  return r;
}
__device__ __forceinline__ void unpack8_bf16(const uint4& r, float* f) {
  const __nv_bfloat162* v = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(v[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// ----------------------------------------------------------- reduce-scatter
// consumed flag of owner r: bases[r] + consumed_off (one u32);
// ready flags of owner r: bases[r] + ready_off + 4*src_rank.
__global__ void rs_push_kernel(float* __restrict__ src, int64_t shard, const uint64_t* __restrict__ bases,
                               int64_t recv_off, int64_t ready_off, int64_t consumed_off, int rank, int world,
                               uint32_t epoch, unsigned int* counter, int* err) {
  // Owners must have consumed the previous epoch before their slots are rewritten.
  const bool ok = block_wait_flags(bases, consumed_off, world, epoch - 1, err, kErrSlotWait);
  const int64_t n8 = ok ? (int64_t)world * shard / 8 : 0;
  const int64_t s8 = shard / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / s8);
    const int64_t j = i - (int64_t)r * s8;
    float4* p = reinterpret_cast<float4*>(src) + 2 * i;
    float f[8];
    const float4 a = p[0], b = p[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    uint4* dst = reinterpret_cast<uint4*>(bases[r] + recv_off) + (int64_t)rank * s8 + j;
    *dst = pack8_bf16(f);
    p[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    p[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (last_block_done(counter) && no_error(err)) {
    __threadfence_system();
    for (int r = 0; r < world; ++r)
      st_release_sys(reinterpret_cast<uint32_t*>(bases[r] + ready_off) + rank, epoch);
  }
}

__global__ void rs_reduce_kernel(const uint4* __restrict__ recv, float* __restrict__ dst, int64_t shard, int world,
                                 float scale, int accumulate, const uint32_t* ready, uint32_t* consumed,
                                 uint32_t epoch, float* sumsq, unsigned int* counter, int* err) {
  const bool ok = block_wait_local_flags(ready, world, epoch, err, kErrPeerWait);
  const int64_t s8 = ok ? shard / 8 : 0;
  float local = 0.f;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < s8; j += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < world; ++p) {
      float f[8];
      unpack8_bf16(recv[(int64_t)p * s8 + j], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += f[e];
    }
    float4* o = reinterpret_cast<float4*>(dst) + 2 * j;
    float4 a = make_float4(acc[0] * scale, acc[1] * scale, acc[2] * scale, acc[3] * scale);
    float4 b = make_float4(acc[4] * scale, acc[5] * scale, acc[6] * scale, acc[7] * scale);
    if (accumulate) {
      const float4 oa = o[0], ob = o[1];
      a.x += oa.x; a.y += oa.y; a.z += oa.z; a.w += oa.w;
      b.x += ob.x; b.y += ob.y; b.z += ob.z; b.w += ob.w;
    }
    o[0] = a;
    o[1] = b;
    local += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
  }
  __shared__ float red[32];
  const float tot = block_sum(local, red);
  if (threadIdx.x == 0 && sumsq != nullptr) atomicAdd(sumsq, tot);
  if (last_block_done(counter) && no_error(err)) st_release_sys(consumed, epoch);
}

// --------------------------------------------------------------- all-gather
__global__ void ag_publish_kernel(const float* __restrict__ master, uint4* __restrict__ heap_shard, int64_t shard,
                                  uint32_t* ready, uint32_t epoch, unsigned int* counter) {
  const int64_t s8 = shard / 8;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < s8; j += (int64_t)gridDim.x * blockDim.x) {
    const float4* p = reinterpret_cast<const float4*>(master) + 2 * j;
    const float4 a = p[0], b = p[1];
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    heap_shard[j] = pack8_bf16(f);
  }
  if (last_block_done(counter)) st_release_sys(ready, epoch);
}

// Generic pull of `bytes` (multiple of 16) per rank: dst[r*bytes ...] = heap_r[src_off ...].
__global__ void pull_kernel(uint4* __restrict__ dst, int64_t bytes, const uint64_t* __restrict__ bases,
                            int64_t src_off, int64_t ready_off, int world, uint32_t epoch, int* err) {
  if (!block_wait_flags(bases, ready_off, world, epoch, err, kErrPeerWait)) return;  // no completion signal
  const int64_t n16 = bytes / 16;
  const int64_t total = n16 * world;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / n16);
    const int64_t j = i - (int64_t)r * n16;
    dst[i] = reinterpret_cast<const uint4*>(bases[r] + src_off)[j];
  }
}

// All-to-all-v by pulling: dst[dst_off[r] ..] = heap_r[src_off[r] ..] for lens[r]
// bytes from every rank r (r = this rank included), after rank r raised its
// ready flag (at `ready_off` of its heap) to `epoch`.  `plan` is a (3, world)
// int64 table of byte offsets / lengths, all multiples of 16.
__global__ void a2av_pull_kernel(unsigned char* __restrict__ dst, const uint64_t* __restrict__ bases,
                                 const int64_t* __restrict__ plan, int64_t ready_off, int world, uint32_t epoch,
                                 int* err) {
  __shared__ int64_t s_src[16], s_dst[16], s_end[16];
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int r = 0; r < world; ++r) {
      s_src[r] = plan[r];
      s_dst[r] = plan[world + r];
      acc += plan[2 * world + r] / 16;
      s_end[r] = acc;  // prefix end, in 16-byte units
    }
  }
  if (!block_wait_flags(bases, ready_off, world, epoch, err, kErrPeerWait)) return;
  const int64_t total = s_end[world - 1];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int r = 0;
    while (i >= s_end[r]) ++r;
    const int64_t j = i - (r ? s_end[r - 1] : 0);
    reinterpret_cast<uint4*>(dst + s_dst[r])[j] = reinterpret_cast<const uint4*>(bases[r] + s_src[r])[j];
  }
}

// ----------------------------------------------------------------- DiLoCo
// Pseudo-gradient delta = anchor - local, pushed in fp32 into slot `rank` of
// each owner (owner r holds elements [r*shard, (r+1)*shard)).
__global__ void diloco_push_kernel(const float* __restrict__ anchor, const float* __restrict__ local, int64_t shard,
                                   const uint64_t* __restrict__ bases, int64_t recv_off, int64_t ready_off,
                                   int64_t consumed_off, int rank, int world, uint32_t epoch, unsigned int* counter,
                                   int* err) {
  const bool ok = block_wait_flags(bases, consumed_off, world, epoch - 1, err, kErrSlotWait);
  const int64_t n4 = ok ? (int64_t)world * shard / 4 : 0, s4 = shard / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / s4);
    const int64_t j = i - (int64_t)r * s4;
    const float4 a = reinterpret_cast<const float4*>(anchor)[i], l = reinterpret_cast<const float4*>(local)[i];
    reinterpret_cast<float4*>(bases[r] + recv_off)[(int64_t)rank * s4 + j] =
        make_float4(a.x - l.x, a.y - l.y, a.z - l.z, a.w - l.w);
  }
  if (last_block_done(counter) && no_error(err)) {
    __threadfence_system();
    for (int r = 0; r < world; ++r)
      st_release_sys(reinterpret_cast<uint32_t*>(bases[r] + ready_off) + rank, epoch);
  }
}

// Owner: delta = mean of the slots; Nesterov outer step on the anchor shard
//   m = mu*m + delta;  anchor -= lr * (delta + mu*m)
// and the new anchor shard is written to the heap for the other ranks to pull.
__global__ void diloco_reduce_nesterov_kernel(const float4* __restrict__ recv, float* __restrict__ anchor_shard,
                                              float* __restrict__ mom_shard, float4* __restrict__ heap_out,
                                              int64_t shard, int world, float lr, float mu, const uint32_t* ready,
                                              uint32_t* consumed, uint32_t* out_ready, uint32_t epoch,
                                              unsigned int* counter, int* err) {
  const bool ok = block_wait_local_flags(ready, world, epoch, err, kErrPeerWait);
  const int64_t s4 = ok ? shard / 4 : 0;
  const float inv = 1.f / (float)world;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < s4; j += (int64_t)gridDim.x * blockDim.x) {
    float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < world; ++p) {
      const float4 v = recv[(int64_t)p * s4 + j];
      d.x += v.x; d.y += v.y; d.z += v.z; d.w += v.w;
    }
    d.x *= inv; d.y *= inv; d.z *= inv; d.w *= inv;
    float4* m = reinterpret_cast<float4*>(mom_shard) + j;
    float4* a = reinterpret_cast<float4*>(anchor_shard) + j;
    float4 mv = *m, av = *a;
    mv.x = mu * mv.x + d.x; mv.y = mu * mv.y + d.y; mv.z = mu * mv.z + d.z; mv.w = mu * mv.w + d.w;
    av.x -= lr * (d.x + mu * mv.x); av.y -= lr * (d.y + mu * mv.y);
    av.z -= lr * (d.z + mu * mv.z); av.w -= lr * (d.w + mu * mv.w);
    *m = mv;
    *a = av;
    heap_out[j] = av;
  }
  if (last_block_done(counter) && no_error(err)) {
    st_release_sys(consumed, epoch);
    st_release_sys(out_ready, epoch);
  }
}

// ------------------------------------------------ bf16 row reduce-scatter
// Tensor parallelism around GEMMs that are not fused with the collective (the
// NVFP4 linears): the partial product (world*shard bf16, owner r holding the
// rows [r*shard, (r+1)*shard) of the flat row-major buffer) is pushed into the
// owners' slots, then each owner sums its world slots in fp32, adds an
// optional residual and writes bf16.  Same flag protocol as rs_push / rs_reduce.
__global__ void rows_rs_push_kernel(const uint4* __restrict__ src, int64_t s8, const uint64_t* __restrict__ bases,
                                    int64_t recv_off, int64_t ready_off, int64_t consumed_off, int rank, int world,
                                    uint32_t epoch, unsigned int* counter, int* err) {
  const bool ok = block_wait_flags(bases, consumed_off, world, epoch - 1, err, kErrSlotWait);
  const int64_t n8 = ok ? (int64_t)world * s8 : 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / s8);
    const int64_t j = i - (int64_t)r * s8;
    reinterpret_cast<uint4*>(bases[r] + recv_off)[(int64_t)rank * s8 + j] = src[i];
  }
  if (last_block_done(counter) && no_error(err)) {
    __threadfence_system();
    for (int r = 0; r < world; ++r)
      st_release_sys(reinterpret_cast<uint32_t*>(bases[r] + ready_off) + rank, epoch);
  }
}

__global__ void rows_rs_reduce_kernel(const uint4* __restrict__ recv, const uint4* __restrict__ residual,
                                      uint4* __restrict__ out, int64_t s8, int world, const uint32_t* ready,
                                      uint32_t* consumed, uint32_t epoch, unsigned int* counter, int* err) {
  const bool ok = block_wait_local_flags(ready, world, epoch, err, kErrPeerWait);
  const int64_t n = ok ? s8 : 0;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (residual != nullptr) unpack8_bf16(residual[j], acc);
    for (int p = 0; p < world; ++p) {
      float f[8];
      unpack8_bf16(recv[(int64_t)p * s8 + j], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += f[e];
    }
    out[j] = pack8_bf16(acc);
  }
  if (last_block_done(counter) && no_error(err)) st_release_sys(consumed, epoch);
}

inline int grid_for(int64_t work, int threads = 256) {
  const int64_t blocks = (work + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)num_sms() * 4));
}

uint64_t* dev_u64(const at::Tensor& t) {
  LRB_CHECK(t.is_cuda() && t.scalar_type() == at::kLong && t.is_contiguous(), "expected a contiguous int64 CUDA tensor");
  return reinterpret_cast<uint64_t*>(t.data_ptr<int64_t>());
}
unsigned int* counter_ptr(const at::Tensor& t) {
  LRB_CHECK(t.is_cuda() && t.scalar_type() == at::kInt, "counter must be an int32 CUDA tensor");
  return reinterpret_cast<unsigned int*>(t.data_ptr<int>());
}

}  // namespace

// ------------------------------------------------------------------ host API
std::tuple<int64_t, at::Tensor> symm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  LRB_CUDA_CHECK(cudaMalloc(&p, (size_t)nbytes));
  LRB_CUDA_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  LRB_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto out = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(out.data_ptr(), &h, sizeof(h));
  return {reinterpret_cast<int64_t>(p), out};
}

int64_t symm_open(const at::Tensor& handle, int64_t device) {
  LRB_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && handle.scalar_type() == at::kByte,
            "symm_open: expected a uint8 IPC handle");
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  auto hc = handle.contiguous().cpu();
  std::memcpy(&h, hc.data_ptr(), sizeof(h));
  void* p = nullptr;
  LRB_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  LRB_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

void symm_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  LRB_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

// Non-owning tensor view of heap memory.
at::Tensor symm_view(int64_t ptr, int64_t offset, at::IntArrayRef sizes, at::ScalarType dtype, int64_t device) {
  LRB_CHECK(offset % 16 == 0, "symm_view: offset must be 16-byte aligned");
  return at::from_blob(reinterpret_cast<char*>(ptr) + offset, sizes, [](void*) {},
                       at::TensorOptions().device(at::Device(at::kCUDA, (c10::DeviceIndex)device)).dtype(dtype));
}

void p2p_rs_push(at::Tensor& src, const at::Tensor& bases, int64_t recv_off, int64_t ready_off, int64_t consumed_off,
                 int64_t rank, int64_t world, int64_t shard, int64_t epoch, at::Tensor& counter, at::Tensor& err) {
  LRB_CHECK(src.is_cuda() && src.scalar_type() == at::kFloat && src.is_contiguous() && src.numel() == world * shard,
            "p2p_rs_push: src must be contiguous fp32 of world*shard elements");
  LRB_CHECK(shard % 8 == 0, "p2p_rs_push: shard must be a multiple of 8");
  c10::cuda::CUDAGuard g(src.device());
  rs_push_kernel<<<grid_for(src.numel() / 8), 256, 0, stream()>>>(
      src.data_ptr<float>(), shard, dev_u64(bases), recv_off, ready_off, consumed_off, (int)rank, (int)world,
      (uint32_t)epoch, counter_ptr(counter), err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

void p2p_rs_reduce(const at::Tensor& recv, at::Tensor& dst, int64_t world, double scale, bool accumulate,
                   const at::Tensor& ready, at::Tensor& consumed, int64_t epoch, c10::optional<at::Tensor> sumsq,
                   at::Tensor& counter, at::Tensor& err) {
  const int64_t shard = dst.numel();
  LRB_CHECK(dst.scalar_type() == at::kFloat && dst.is_contiguous() && shard % 8 == 0, "p2p_rs_reduce: bad dst");
  LRB_CHECK(recv.scalar_type() == at::kBFloat16 && recv.numel() == world * shard, "p2p_rs_reduce: bad recv");
  c10::cuda::CUDAGuard g(dst.device());
  rs_reduce_kernel<<<grid_for(shard / 8), 256, 0, stream()>>>(
      reinterpret_cast<const uint4*>(recv.data_ptr()), dst.data_ptr<float>(), shard, (int)world, (float)scale,
      accumulate ? 1 : 0, reinterpret_cast<const uint32_t*>(ready.data_ptr<int>()),
      reinterpret_cast<uint32_t*>(consumed.data_ptr<int>()), (uint32_t)epoch,
      sumsq ? sumsq->data_ptr<float>() : nullptr, counter_ptr(counter), err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

// y (world*shard bf16 rows, row-major) -> owners' slots; see rows_rs_push_kernel.
void p2p_rows_rs_push(const at::Tensor& y, const at::Tensor& bases, int64_t recv_off, int64_t ready_off,
                      int64_t consumed_off, int64_t rank, int64_t world, int64_t epoch, at::Tensor& counter,
                      at::Tensor& err) {
  const int64_t n = y.numel();
  LRB_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous() && n % (8 * world) == 0,
            "p2p_rows_rs_push: y must be contiguous bf16 with numel a multiple of 8*world");
  c10::cuda::CUDAGuard g(y.device());
  rows_rs_push_kernel<<<grid_for(n / 8), 256, 0, stream()>>>(
      reinterpret_cast<const uint4*>(y.data_ptr()), n / world / 8, dev_u64(bases), recv_off, ready_off, consumed_off,
      (int)rank, (int)world, (uint32_t)epoch, counter_ptr(counter), err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

void p2p_rows_rs_reduce(const at::Tensor& recv, const c10::optional<at::Tensor>& residual, at::Tensor& out,
                        int64_t world, const at::Tensor& ready, at::Tensor& consumed, int64_t epoch,
                        at::Tensor& counter, at::Tensor& err) {
  const int64_t shard = out.numel();
  LRB_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() && shard % 8 == 0,
            "p2p_rows_rs_reduce: out must be contiguous bf16 with numel a multiple of 8");
  LRB_CHECK(recv.scalar_type() == at::kBFloat16 && recv.numel() >= world * shard, "p2p_rows_rs_reduce: bad recv");
  if (residual)
    LRB_CHECK(residual->scalar_type() == at::kBFloat16 && residual->is_contiguous() && residual->numel() == shard,
              "p2p_rows_rs_reduce: residual must match out");
  c10::cuda::CUDAGuard g(out.device());
  rows_rs_reduce_kernel<<<grid_for(shard / 8), 256, 0, stream()>>>(
      reinterpret_cast<const uint4*>(recv.data_ptr()),
      residual ? reinterpret_cast<const uint4*>(residual->data_ptr()) : nullptr, reinterpret_cast<uint4*>(out.data_ptr()),
      shard / 8, (int)world, reinterpret_cast<const uint32_t*>(ready.data_ptr<int>()),
      reinterpret_cast<uint32_t*>(consumed.data_ptr<int>()), (uint32_t)epoch, counter_ptr(counter), err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

void p2p_ag_publish(const at::Tensor& master, at::Tensor& heap_shard, at::Tensor& ready, int64_t epoch,
                    at::Tensor& counter) {
  const int64_t shard = master.numel();
  LRB_CHECK(master.scalar_type() == at::kFloat && master.is_contiguous() && shard % 8 == 0, "p2p_ag_publish: master");
  LRB_CHECK(heap_shard.scalar_type() == at::kBFloat16 && heap_shard.numel() == shard, "p2p_ag_publish: heap shard");
  c10::cuda::CUDAGuard g(master.device());
  ag_publish_kernel<<<grid_for(shard / 8), 256, 0, stream()>>>(
      master.data_ptr<float>(), reinterpret_cast<uint4*>(heap_shard.data_ptr()), shard,
      reinterpret_cast<uint32_t*>(ready.data_ptr<int>()), (uint32_t)epoch, counter_ptr(counter));
  LRB_LAUNCH_CHECK();
}

void p2p_pull(at::Tensor& dst, const at::Tensor& bases, int64_t src_off, int64_t ready_off, int64_t world,
              int64_t epoch, at::Tensor& err) {
  const int64_t bytes = dst.numel() * dst.element_size();
  LRB_CHECK(dst.is_contiguous() && bytes % (16 * world) == 0, "p2p_pull: dst bytes must split into 16-byte multiples");
  c10::cuda::CUDAGuard g(dst.device());
  pull_kernel<<<grid_for(bytes / 16), 256, 0, stream()>>>(reinterpret_cast<uint4*>(dst.data_ptr()), bytes / world,
                                                           dev_u64(bases), src_off, ready_off, (int)world,
                                                           (uint32_t)epoch, err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

// dst <- pieces of every rank's heap per `plan` (3, world) int64 byte table
// [src offsets in the peers' heaps; dst offsets; lengths], each peer's pieces
// read once its ready flag (heap offset `ready_off`) reached `epoch`.
void p2p_a2av_pull(at::Tensor& dst, const at::Tensor& bases, const at::Tensor& plan, int64_t ready_off, int64_t world,
                   int64_t epoch, at::Tensor& err) {
  LRB_CHECK(world >= 1 && world <= 16, "p2p_a2av_pull: 1..16 ranks");
  LRB_CHECK(plan.is_cuda() && plan.scalar_type() == at::kLong && plan.is_contiguous() && plan.numel() == 3 * world,
            "p2p_a2av_pull: plan must be a contiguous (3, world) int64 CUDA tensor");
  LRB_CHECK(dst.is_contiguous() && reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0,
            "p2p_a2av_pull: dst must be contiguous and 16-byte aligned");
  c10::cuda::CUDAGuard g(dst.device());
  const int64_t bytes = dst.numel() * dst.element_size();
  a2av_pull_kernel<<<grid_for(std::max<int64_t>(bytes / 16, 1)), 256, 0, stream()>>>(
      reinterpret_cast<unsigned char*>(dst.data_ptr()), dev_u64(bases), plan.data_ptr<int64_t>(), ready_off,
      (int)world, (uint32_t)epoch, err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

void diloco_push(const at::Tensor& anchor, const at::Tensor& local, const at::Tensor& bases, int64_t recv_off,
                 int64_t ready_off, int64_t consumed_off, int64_t rank, int64_t world, int64_t epoch,
                 at::Tensor& counter, at::Tensor& err) {
  const int64_t n = anchor.numel();
  LRB_CHECK(anchor.scalar_type() == at::kFloat && local.scalar_type() == at::kFloat && local.numel() == n &&
                anchor.is_contiguous() && local.is_contiguous() && n % (4 * world) == 0,
            "diloco_push: fp32 contiguous tensors with numel a multiple of 4*world required");
  c10::cuda::CUDAGuard g(anchor.device());
  diloco_push_kernel<<<grid_for(n / 4), 256, 0, stream()>>>(
      anchor.data_ptr<float>(), local.data_ptr<float>(), n / world, dev_u64(bases), recv_off, ready_off,
      consumed_off, (int)rank, (int)world, (uint32_t)epoch, counter_ptr(counter), err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

void diloco_reduce_nesterov(const at::Tensor& recv, at::Tensor& anchor_shard, at::Tensor& mom_shard,
                            at::Tensor& heap_out, int64_t world, double lr, double mu, const at::Tensor& ready,
                            at::Tensor& consumed, at::Tensor& out_ready, int64_t epoch, at::Tensor& counter,
                            at::Tensor& err) {
  const int64_t shard = anchor_shard.numel();
  LRB_CHECK(shard % 4 == 0 && mom_shard.numel() == shard && heap_out.numel() == shard &&
                recv.numel() == world * shard && recv.scalar_type() == at::kFloat,
            "diloco_reduce_nesterov: shape mismatch");
  c10::cuda::CUDAGuard g(anchor_shard.device());
  diloco_reduce_nesterov_kernel<<<grid_for(shard / 4), 256, 0, stream()>>>(
      reinterpret_cast<const float4*>(recv.data_ptr<float>()), anchor_shard.data_ptr<float>(),
      mom_shard.data_ptr<float>(), reinterpret_cast<float4*>(heap_out.data_ptr<float>()), shard, (int)world,
      (float)lr, (float)mu, reinterpret_cast<const uint32_t*>(ready.data_ptr<int>()),
      reinterpret_cast<uint32_t*>(consumed.data_ptr<int>()), reinterpret_cast<uint32_t*>(out_ready.data_ptr<int>()),
      (uint32_t)epoch, counter_ptr(counter), err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

}  // namespace lrb
