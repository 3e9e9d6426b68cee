// Expert-parallel MoE dispatch / combine over symmetric memory (P2P stores
// and loads over NVLink, no multicast).
//
// Every rank is a source (its T tokens, each routed to k experts) and an
// owner (E / world local experts).  Owner buffers sit at the same heap offset
// on every rank, laid out [local expert][source rank][capacity slot][d], so a
// local expert's rows from all sources are one contiguous (world*cap, d) block
// for the expert GEMMs.  An assignment (t, j) goes to owner dest[t,j], local
// expert le[t,j], slot slot[t,j] (slot < 0: dropped by the capacity rule).
//
//   ep_push   source -> owners: copies row t (or the per-assignment row a),
//             optionally scaled by scale[a], into the owner's slot; waits until
//             every owner released the previous epoch (consumed flag) and
//             finally raises ready[rank] at every owner.
//   ep_pull   owners -> source: y[t] = sum_j w[t,j] * owner_row(t,j) (w may be
//             null = 1), optionally also returns the rows; waits for every
//             owner's out-ready flag and then raises out-read[rank] at every
//             owner.
//   flag_wait / flag_set: owner-side ordering points between these kernels
//             and the expert GEMMs that read / write the buffers.
// All waits are bounded and report an error code; no wait ever runs in two
// kernels of one GPU that wait on one another.
#include "../common.cuh"

namespace lrb {
namespace {

constexpr long long kPollLimit = 1ll << 24;
enum : int { kErrEpReady = 31, kErrEpSlot = 32, kErrEpIndex = 33 };

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool reached(uint32_t f, uint32_t e) { return (int32_t)(f - e) >= 0; }

// Thread i < n polls flag (base_i + off + 4*idx) until >= epoch.
__device__ bool block_poll(const uint64_t* bases, int64_t off, int idx, int n, uint32_t epoch, int* err, int code) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < n) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(bases[threadIdx.x] + off) + idx;
    long long it = 0;
    while (!reached(ld_acquire_sys(f), epoch)) {
      if (++it > kPollLimit) {
        atomicExch(&ok, 0);
        atomicCAS(err, 0, code);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  return ok != 0;
}

__device__ bool last_block(unsigned int* counter) {
  __shared__ bool last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
    if (last) *counter = 0u;
  }
  __syncthreads();
  return last && threadIdx.x == 0;
}

struct EpArgs {
  const uint64_t* bases;
  int64_t buf_off;   // push: recv region; pull: out region
  int64_t flag_off;  // push: ready[world]; pull: out-ready (one u32)
  int64_t gate_off;  // push: consumed (one u32); pull: out-read[world]
  int rank, world, k, d, cap, epl;
  uint32_t epoch;
  const int* dest;
  const int* le;
  const int* slot;
  unsigned int* counter;
  int* err;
};

__device__ __forceinline__ int64_t slot_row(const EpArgs& a, int le, int src, int slot) {
  return ((int64_t)le * a.world + src) * a.cap + slot;
}

// Routing indices come from data: an owner, local expert or slot outside the
// buffers records kErrEpIndex and the row is skipped, never written or read
// out of bounds on a peer.
__device__ __forceinline__ bool route_ok(const EpArgs& a, int64_t as, int s) {
  const int dst = a.dest[as], le = a.le[as];
  const bool ok = s < a.cap && dst >= 0 && dst < a.world && le >= 0 && le < a.epl;
  if (!ok) atomicCAS(a.err, 0, kErrEpIndex);
  return ok;
}

// rows: per_assignment ? (T*k, d) : (T, d)
__global__ void ep_push_kernel(const __nv_bfloat16* __restrict__ rows, const float* __restrict__ scale, int64_t TK,
                               int per_assignment, EpArgs a) {
  const bool ok = block_poll(a.bases, a.gate_off, 0, a.world, a.epoch - 1, a.err, kErrEpSlot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  if (ok) {
    for (int64_t as = (int64_t)blockIdx.x * wpb + warp; as < TK; as += (int64_t)gridDim.x * wpb) {
      const int s = a.slot[as];
      if (s < 0 || !route_ok(a, as, s)) continue;
      const int64_t src_row = per_assignment ? as : as / a.k;
      const float sc = scale != nullptr ? scale[as] : 1.f;
      const uint4* src = reinterpret_cast<const uint4*>(rows + src_row * a.d);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.bases[a.dest[as]] + a.buf_off) +
                                            slot_row(a, a.le[as], a.rank, s) * a.d);
      for (int i = lane; i < a.d / 8; i += 32) {
        uint4 v = src[i];
        if (scale != nullptr) {
          __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
          for (int q = 0; q < 8; ++q) e[q] = __float2bfloat16_rn(__bfloat162float(e[q]) * sc);
        }
        dst[i] = v;
      }
    }
  }
  if (last_block(a.counter) && *reinterpret_cast<volatile int*>(a.err) == 0) {
    __threadfence_system();
    for (int r = 0; r < a.world; ++r) st_release_sys(reinterpret_cast<uint32_t*>(a.bases[r] + a.flag_off) + a.rank, a.epoch);
  }
}

// out[t] = sum_j w[t,j] * row(t,j); rows_out (T*k, d) optional.
__global__ void ep_pull_kernel(__nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ rows_out,
                               const float* __restrict__ w, int64_t T, EpArgs a) {
  const bool ok = block_poll(a.bases, a.flag_off, 0, a.world, a.epoch, a.err, kErrEpReady);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  if (ok) {
    for (int64_t t = (int64_t)blockIdx.x * wpb + warp; t < T; t += (int64_t)gridDim.x * wpb) {
      for (int i = lane; i < a.d / 8; i += 32) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < a.k; ++j) {
          const int64_t as = t * a.k + j;
          const int s = a.slot[as];
          Vec16<__nv_bfloat16> v;
          if (s >= 0 && route_ok(a, as, s)) {
            v.raw = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.bases[a.dest[as]] + a.buf_off) +
                                                   slot_row(a, a.le[as], a.rank, s) * a.d)[i];
          } else {
            v.raw = make_uint4(0u, 0u, 0u, 0u);
          }
          if (rows_out != nullptr) reinterpret_cast<uint4*>(rows_out + as * a.d)[i] = v.raw;
          const float wj = w != nullptr ? w[as] : 1.f;
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] += wj * __bfloat162float(v.v[q]);
        }
        Vec16<__nv_bfloat16> o;
#pragma unroll
        for (int q = 0; q < 8; ++q) o.v[q] = __float2bfloat16_rn(acc[q]);
        reinterpret_cast<uint4*>(out + t * a.d)[i] = o.raw;
      }
    }
  }
  if (last_block(a.counter) && *reinterpret_cast<volatile int*>(a.err) == 0)
    for (int r = 0; r < a.world; ++r) st_release_sys(reinterpret_cast<uint32_t*>(a.bases[r] + a.gate_off) + a.rank, a.epoch);
}

// Owner side: wait until n local flags reach epoch.
__global__ void flag_wait_kernel(const uint32_t* flags, int n, uint32_t epoch, int* err) {
  if ((int)threadIdx.x < n) {
    long long it = 0;
    while (!reached(ld_acquire_sys(flags + threadIdx.x), epoch)) {
      if (++it > kPollLimit) {
        atomicCAS(err, 0, kErrEpReady);
        break;
      }
      __nanosleep(32);
    }
  }
}

__global__ void flag_set_kernel(uint32_t* flag, uint32_t epoch) {
  __threadfence_system();
  st_release_sys(flag, epoch);
}

EpArgs make_args(const at::Tensor& bases, int64_t buf_off, int64_t flag_off, int64_t gate_off, int64_t rank,
                 int64_t world, int64_t k, int64_t d, int64_t cap, int64_t epl, int64_t epoch, const at::Tensor& dest,
                 const at::Tensor& le, const at::Tensor& slot, at::Tensor& counter, at::Tensor& err) {
  LRB_CHECK(d % 8 == 0, "expert-parallel exchange: d must be a multiple of 8");
  LRB_CHECK(dest.scalar_type() == at::kInt && le.scalar_type() == at::kInt && slot.scalar_type() == at::kInt,
            "route tensors must be int32");
  EpArgs a;
  a.bases = reinterpret_cast<const uint64_t*>(bases.data_ptr<int64_t>());
  a.buf_off = buf_off; a.flag_off = flag_off; a.gate_off = gate_off;
  a.rank = (int)rank; a.world = (int)world; a.k = (int)k; a.d = (int)d; a.cap = (int)cap; a.epl = (int)epl;
  a.epoch = (uint32_t)epoch;
  a.dest = dest.data_ptr<int>(); a.le = le.data_ptr<int>(); a.slot = slot.data_ptr<int>();
  a.counter = reinterpret_cast<unsigned int*>(counter.data_ptr<int>());
  a.err = err.data_ptr<int>();
  return a;
}

int blocks_for(int64_t items, int per_block) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((items + per_block - 1) / per_block, (int64_t)num_sms() * 8));
}

}  // namespace

void ep_push(const at::Tensor& rows, const c10::optional<at::Tensor>& scale, bool per_assignment, const at::Tensor& bases,
             int64_t recv_off, int64_t ready_off, int64_t consumed_off, int64_t rank, int64_t world, int64_t k,
             int64_t cap, int64_t epl, int64_t epoch, const at::Tensor& dest, const at::Tensor& le,
             const at::Tensor& slot, at::Tensor& counter, at::Tensor& err) {
  LRB_CHECK(rows.scalar_type() == at::kBFloat16 && rows.is_contiguous(), "ep_push: contiguous bf16 rows");
  c10::cuda::CUDAGuard g(rows.device());
  const int64_t d = rows.size(-1), TK = dest.numel();
  EpArgs a = make_args(bases, recv_off, ready_off, consumed_off, rank, world, k, d, cap, epl, epoch, dest, le, slot,
                       counter, err);
  ep_push_kernel<<<blocks_for(TK, 8), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(rows.data_ptr()), scale ? scale->data_ptr<float>() : nullptr, TK,
      per_assignment ? 1 : 0, a);
  LRB_LAUNCH_CHECK();
}

void ep_pull(at::Tensor& out, const c10::optional<at::Tensor>& rows_out, const c10::optional<at::Tensor>& w,
             const at::Tensor& bases, int64_t out_off, int64_t outready_off, int64_t outread_off, int64_t rank,
             int64_t world, int64_t k, int64_t cap, int64_t epl, int64_t epoch, const at::Tensor& dest,
             const at::Tensor& le, const at::Tensor& slot, at::Tensor& counter, at::Tensor& err) {
  LRB_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous(), "ep_pull: contiguous bf16 output");
  c10::cuda::CUDAGuard g(out.device());
  const int64_t T = out.size(0), d = out.size(1);
  EpArgs a = make_args(bases, out_off, outready_off, outread_off, rank, world, k, d, cap, epl, epoch, dest, le, slot,
                       counter, err);
  ep_pull_kernel<<<blocks_for(T, 8), 256, 0, stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      rows_out ? reinterpret_cast<__nv_bfloat16*>(rows_out->data_ptr()) : nullptr, w ? w->data_ptr<float>() : nullptr,
      T, a);
  LRB_LAUNCH_CHECK();
}

void ep_flag_wait(const at::Tensor& flags, int64_t n, int64_t epoch, at::Tensor& err) {
  c10::cuda::CUDAGuard g(flags.device());
  flag_wait_kernel<<<1, 32, 0, stream()>>>(reinterpret_cast<const uint32_t*>(flags.data_ptr<int>()), (int)n,
                                           (uint32_t)epoch, err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

void ep_flag_set(at::Tensor& flag, int64_t epoch) {
  c10::cuda::CUDAGuard g(flag.device());
  flag_set_kernel<<<1, 1, 0, stream()>>>(reinterpret_cast<uint32_t*>(flag.data_ptr<int>()), (uint32_t)epoch);
  LRB_LAUNCH_CHECK();
}

}  // namespace lrb
