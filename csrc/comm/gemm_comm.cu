// Tensor-core GEMMs fused with the collective around them, over symmetric
// memory (IPC-mapped peer heaps; plain P2P loads and stores, no multicast).
//
// gemm_rs   Y = X W^T with the sequence reduce-scatter of a row-parallel
//           layer: every rank computes the full partial product (M x N); the
//           epilogue converts each 128 x 256 tile to bf16 in 32 x 32 blocks
//           staged in shared memory and pushes every block with one 2 KB bulk
//           store into the owning rank's receive slot over NVLink (rows
//           [o*Mr, (o+1)*Mr) are owned by rank o; the slot is tile-major so a
//           block is contiguous), and the last tile of an owner's rows raises
//           that owner's ready flag.  `tp_reduce` then sums the world slots
//           (fp32) on the owner into the row-major output, adds an optional
//           residual and releases the slots.
//
// ag_gemm   Y = AllGather_rows(X) W^T for a column-parallel layer: one
//           persistent launch in which the first `ncopy` CTAs pull 128-row
//           chunks of every rank's shard (peer heaps) into a local buffer and
//           publish a per-chunk flag, while the other CTAs run the GEMM over
//           chunks in rank-rotated order (own rows first) and wait for a
//           chunk's flag before their TMA loads read it.
//
// GEMM core: tiles 128 x 256 x 64, 4-stage TMA ring, one MMA-issuing thread,
// double-buffered TMEM accumulators, 4 epilogue warps (as gemm_sm100.cu).
// Every flag wait is bounded; on expiry the kernel records an error code,
// skips the remaining communication, drains its MMAs and frees TMEM.
#include "../common.cuh"
#include "../kernels/sm100.cuh"

namespace lrb {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr size_t kStageA = (size_t)BM * BK * 2, kStageB = (size_t)BN * BK * 2;
// gemm_rs epilogue staging: per epilogue warp two 32 x 32 bf16 blocks (2 KB each).
constexpr uint32_t kStageBlk = 32 * 32 * 2;
constexpr size_t kSmem = 1024 + STAGES * (kStageA + kStageB) + 256 + 4 * 2 * kStageBlk;
constexpr long long kPollLimit = 1ll << 24;
enum : int { kErrPeer = 21, kErrSlot = 22, kErrChunk = 23 };

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool reached(uint32_t f, uint32_t e) { return (int32_t)(f - e) >= 0; }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <bool SYS>
__device__ bool poll(const uint32_t* f, uint32_t epoch, int* err, int code) {
  long long it = 0;
  while (!reached(SYS ? ld_acquire_sys(f) : ld_acquire_gpu(f), epoch)) {
    if (++it > kPollLimit) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

__device__ __forceinline__ bool no_error(const int* err) {
  return *reinterpret_cast<const volatile int*>(err) == 0;
}

struct CommGemmArgs {
  void* C;            // ag_gemm: local output (M x N); gemm_rs: unused
  int64_t ldc;
  int M, N, K;
  int rows_per_rank;  // M / world, a multiple of BM
  int rank, world;
  const uint64_t* bases;
  int64_t off0, off1, off2;  // gemm_rs: recv, ready, consumed; ag_gemm: shard, shard_ready, -
  uint32_t epoch;
  unsigned int* counters;    // gemm_rs: [world] tile counters; ag_gemm: unused
  uint32_t* chunk_flags;     // ag_gemm: [M / BM]
  __nv_bfloat16* a_full;     // ag_gemm: local gathered X (M x K)
  int ncopy;                 // ag_gemm: copy CTAs
  int* err;
};

// Tile t -> (tm, tn).  The M order starts at this rank's rows (ag_gemm) or is
// natural (gemm_rs); N runs fastest inside a group of 8 M-tiles.
__device__ __forceinline__ void tile_of(int t, int tiles_m, int tiles_n, int rot, int& tm, int& tn) {
  const int per_group = 8 * tiles_n;
  const int g = t / per_group, first = g * 8, gsize = min(tiles_m - first, 8), r = t % per_group;
  tm = (first + r % gsize + rot) % tiles_m;
  tn = r / gsize;
}

template <bool AG>
__global__ void __launch_bounds__(kThreads, 1)
    comm_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     CommGemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = a.M / BM, tiles_n = (a.N + BN - 1) / BN, num_tiles = tiles_m * tiles_n;
  const int nk = (a.K + BK - 1) / BK;
  const int chunks_per_rank = a.rows_per_rank / BM;

  // ---------------------------------------------------------------- copy CTAs
  // Each chunk (128 rows x K bf16) moves peer heap -> shared -> local buffer in
  // 16 KB pieces through a ring of kCopyBufs shared buffers: thread 0 issues a
  // bulk load (completion on an mbarrier) and, once it landed, a bulk store;
  // a buffer is reused after its store has been read (bulk_group wait).
  if (AG && (int)blockIdx.x < a.ncopy) {
    constexpr int kCopyBufs = 8;
    constexpr uint32_t kPiece = 16384;
    unsigned char* cbase = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* cbar = reinterpret_cast<uint64_t*>(cbase + kCopyBufs * kPiece);
    if (threadIdx.x == 0) {
      for (int i = 0; i < kCopyBufs; ++i) mbar_init(&cbar[i], 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    const int total = a.world * chunks_per_rank;
    const int64_t chunk_bytes = (int64_t)BM * a.K * 2;
    const int64_t pieces = (chunk_bytes + kPiece - 1) / kPiece;
    uint32_t use[kCopyBufs] = {0, 0, 0, 0, 0, 0, 0, 0};
    bool ok = true;
    int last_src = -1;
    for (int g = blockIdx.x; g < total && ok; g += a.ncopy) {
      const int src = (a.rank + g / chunks_per_rank) % a.world;
      const int lc = g % chunks_per_rank;
      if (src != last_src) {
        ok = poll<true>(reinterpret_cast<const uint32_t*>(a.bases[src] + a.off1), a.epoch, a.err, kErrPeer);
        last_src = src;
        if (!ok) break;
      }
      const char* s = reinterpret_cast<const char*>(a.bases[src] + a.off0) + (int64_t)lc * chunk_bytes;
      char* d = reinterpret_cast<char*>(a.a_full) + ((int64_t)src * a.rows_per_rank + (int64_t)lc * BM) * a.K * 2;
      auto piece_bytes = [&](int64_t p) -> uint32_t {
        const int64_t left = chunk_bytes - p * kPiece;
        return (uint32_t)(left < (int64_t)kPiece ? left : (int64_t)kPiece);
      };
      auto load = [&](int64_t p) {
        const int b = (int)(p % kCopyBufs);
        mbar_arrive_expect_tx(&cbar[b], piece_bytes(p));
        bulk_load(cbase + b * kPiece, s + p * kPiece, piece_bytes(p), &cbar[b]);
      };
      // all buffers are free here: the previous chunk's stores finished below
      for (int64_t p = 0; p < pieces && p < kCopyBufs; ++p) load(p);
      for (int64_t p = 0; p < pieces; ++p) {
        const int b = (int)(p % kCopyBufs);
        if (!mbar_wait(&cbar[b], use[b], a.err, kErrPeer)) { ok = false; break; }
        use[b] ^= 1u;
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                     ::"l"(d + p * kPiece), "r"(smem_addr(cbase + b * kPiece)), "r"(piece_bytes(p)) : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        if (p + kCopyBufs < pieces) {
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // buffer b read by its store
          load(p + kCopyBufs);
        }
      }
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // the chunk is in global memory
      if (!ok) {  // drain loads still in flight before leaving
        for (int b = 0; b < kCopyBufs; ++b) mbar_wait(&cbar[b], use[b], nullptr, 0);
        break;
      }
      __threadfence();
      st_release_gpu(a.chunk_flags + src * chunks_per_rank + lc, a.epoch);
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    return;
  }

  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = base;
  unsigned char* sB = base + STAGES * kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * kStageB);
  uint64_t* empty = full + STAGES;
  uint64_t* accfull = empty + STAGES;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int first = AG ? (int)blockIdx.x - a.ncopy : (int)blockIdx.x;
  const int stride = AG ? (int)gridDim.x - a.ncopy : (int)gridDim.x;
  const int rot = AG ? a.rank * chunks_per_rank : 0;

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
      for (int t = first; t < num_tiles && ok; t += stride) {
        int tm, tn;
        tile_of(t, tiles_m, tiles_n, rot, tm, tn);
        if (AG) {  // the chunk's rows must have landed in the local buffer
          if (!poll<false>(a.chunk_flags + tm, a.epoch, a.err, kErrChunk)) break;
          asm volatile("fence.proxy.async.global;" ::: "memory");  // generic writes -> TMA reads
        }
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, a.err, kErrTmaWait)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], (uint32_t)(kStageA + kStageB));
          tma_load_2d(sA + stage * kStageA, &tmA, &full[stage], kb * BK, tm * BM);
          tma_load_2d(sB + stage * kStageB, &tmB, &full[stage], kb * BK, tn * BN);
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
      constexpr uint32_t idesc = umma_idesc_f16(BM, BN, true);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = first; t < num_tiles && ok; t += stride) {
        if (!mbar_wait(&accempty[acc], acc_phase ^ 1, a.err, kErrAccWait)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase, a.err, kErrMmaWait)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sA + stage * kStageA), b0 = smem_addr(sB + stage * kStageB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d, umma_desc_k_sw128(a0 + k * 32), umma_desc_k_sw128(b0 + k * 32), idesc, (kb | k) != 0);
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
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool slots_ok = true;
    __shared__ unsigned int owner_tiles[8];  // gemm_rs: tiles of each owner pushed by this CTA
    if (!AG) {  // slots alternate by epoch parity: owners must have consumed epoch - 2 before they are rewritten
      __shared__ int sok;
      if (threadIdx.x == 64) sok = 1;
      if (threadIdx.x >= 64 && threadIdx.x < 72) owner_tiles[threadIdx.x - 64] = 0u;
      epi_bar();
      const int t = threadIdx.x - 64;
      if (t < a.world && !poll<true>(reinterpret_cast<const uint32_t*>(a.bases[t] + a.off2), a.epoch - 2, a.err, kErrSlot))
        atomicExch(&sok, 0);
      epi_bar();
      slots_ok = sok != 0;
    }
    // gemm_rs staging: warp q owns two 2 KB blocks after the barrier area.
    unsigned char* stg = reinterpret_cast<unsigned char*>(full) + 256 + q * 2 * kStageBlk;
    const int64_t npad = (int64_t)tiles_n * BN;
    int pending = 0;  // bulk groups this warp has committed and not yet waited for
    for (int t = first; t < num_tiles; t += stride) {
      int tm, tn;
      tile_of(t, tiles_m, tiles_n, rot, tm, tn);
      if (!mbar_wait(&accfull[acc], acc_phase, a.err, kErrEpiWait)) break;
      tc_fence_after();
      const int row = tm * BM + q * 32 + lane;
      const int owner = (tm * BM) / a.rows_per_rank;
      const int tm_local = tm - owner * (a.rows_per_rank / BM);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
        tmem_ld_wait();
        const int col0 = tn * BN + c * 32;
        if (AG) {
          if (col0 >= a.N) continue;
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.C) + (int64_t)row * a.ldc + col0;
          if (col0 + 32 <= a.N) {
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              Vec16<__nv_bfloat16> v;
#pragma unroll
              for (int k = 0; k < 8; ++k) v.v[k] = __float2bfloat16_rn(__uint_as_float(r[e + k]));
              st16(dst + e, v);
            }
          } else {
            for (int e = 0; e < 32 && col0 + e < a.N; ++e) dst[e] = __float2bfloat16_rn(__uint_as_float(r[e]));
          }
        } else {
          if (!slots_ok) continue;
          unsigned char* blk = stg + (c & 1) * kStageBlk;
          // the bulk store issued from this buffer two blocks ago has finished reading it
          if (lane == 0 && pending >= 2) {
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
            pending = 1;
          }
          __syncwarp();
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            Vec16<__nv_bfloat16> v;
#pragma unroll
            for (int k = 0; k < 8; ++k) v.v[k] = __float2bfloat16_rn(__uint_as_float(r[e + k]));
            *reinterpret_cast<uint4*>(blk + lane * 64 + e * 2) = v.raw;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            // slot of (this rank -> owner): tile-major, then 32-column block, then row, then 32 columns
            const int64_t elem = (int64_t)a.rank * a.rows_per_rank * npad +
                                 ((((int64_t)tm_local * tiles_n + tn) * (BN / 32) + c) * BM + q * 32) * 32;
            unsigned char* dst = reinterpret_cast<unsigned char*>(a.bases[owner] + a.off0) + elem * 2;
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                         "r"(smem_addr(blk)), "r"(kStageBlk)
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            ++pending;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&accempty[acc]);
      if (!AG && slots_ok && threadIdx.x == 64) ++owner_tiles[owner];
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (!AG && slots_ok) {
      // Completion is awaited once, after the CTA's last tile, so the bulk stores of
      // all its tiles stay in flight together; then the tiles count toward their
      // owners and the CTA that completes an owner's rows raises its flag.
      if (lane == 0) {
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence_system();
      }
      epi_bar();
      if (threadIdx.x == 64) {
        const unsigned int per_owner = (unsigned int)(chunks_per_rank * tiles_n);
        for (int o = 0; o < a.world; ++o) {
          const unsigned int n = owner_tiles[o];
          if (n == 0) continue;
          if (atomicAdd(&a.counters[o], n) + n == per_owner) {
            a.counters[o] = 0u;
            __threadfence_system();
            if (no_error(a.err))
              st_release_sys(reinterpret_cast<uint32_t*>(a.bases[o] + a.off1) + a.rank, a.epoch);
          }
        }
      }
    } else if (!AG && lane == 0 && pending > 0) {
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Owner side of gemm_rs: out[Mr x N] = sum_p slot_p (+ residual), fp32 accumulation.
// Slots are tile-major (see the gemm_rs epilogue): 8 consecutive elements of a
// slot are 8 consecutive columns of one output row.
__global__ void tp_reduce_kernel(const uint4* __restrict__ recv, const uint4* __restrict__ residual,
                                 uint4* __restrict__ out, int64_t region8, int Mr, int N, int tiles_n, int world,
                                 const uint32_t* ready, uint32_t* consumed, uint32_t epoch, unsigned int* counter,
                                 int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < world && !poll<true>(ready + threadIdx.x, epoch, err, kErrPeer)) atomicExch(&ok, 0);
  __syncthreads();
  if (ok) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < region8; i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i * 8;
      const int within = (int)(e & 31);
      const int rr = (int)((e >> 5) & (BM - 1));
      const int c = (int)((e >> 12) & (BN / 32 - 1));
      const int64_t t = e >> 15;  // (BM * BN) elements per tile
      const int tm = (int)(t / tiles_n), tn = (int)(t % tiles_n);
      const int col = tn * BN + c * 32 + within;
      const int row = tm * BM + rr;
      if (col >= N || row >= Mr) continue;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int p = 0; p < world; ++p) {
        Vec16<__nv_bfloat16> v;
        v.raw = recv[(int64_t)p * region8 + i];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += __bfloat162float(v.v[k]);
      }
      const int64_t o8 = ((int64_t)row * N + col) / 8;
      if (residual != nullptr) {
        Vec16<__nv_bfloat16> v;
        v.raw = residual[o8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += __bfloat162float(v.v[k]);
      }
      Vec16<__nv_bfloat16> o;
#pragma unroll
      for (int k = 0; k < 8; ++k) o.v[k] = __float2bfloat16_rn(acc[k]);
      out[o8] = o.raw;
    }
  }
  __shared__ bool last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
    if (last) *counter = 0u;
  }
  __syncthreads();
  if (last && threadIdx.x == 0 && no_error(err)) st_release_sys(consumed, epoch);
}

// Publish a bf16 shard into the heap and raise this rank's shard flag (ag_gemm source).
__global__ void shard_publish_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t n16,
                                     uint32_t* ready, uint32_t epoch, unsigned int* counter) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
  __shared__ bool last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
    if (last) *counter = 0u;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) st_release_sys(ready, epoch);
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

CUtensorMap kmajor_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LRB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return m;
}

void check_bf16_kmajor(const at::Tensor& t, const char* what) {
  LRB_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
                (t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
            what, ": bf16 2-D tensor with 16-byte aligned rows required");
}

}  // namespace

// X (M x K, this rank's full-M partial input), W (N x K): partial products go to
// the owners' receive slots (recv_off: world x (M/world) x ceil(N/256)*256 bf16,
// tile-major).
void gemm_rs(const at::Tensor& X, const at::Tensor& W, const at::Tensor& bases, int64_t recv_off, int64_t ready_off,
             int64_t consumed_off, int64_t rank, int64_t world, int64_t epoch, at::Tensor& counters,
             at::Tensor& err) {
  check_bf16_kmajor(X, "gemm_rs X");
  check_bf16_kmajor(W, "gemm_rs W");
  const int64_t M = X.size(0), K = X.size(1), N = W.size(0);
  LRB_CHECK(W.size(1) == K && M % (BM * world) == 0 && N % 8 == 0, "gemm_rs: M % (128*world) == 0, N % 8 == 0");
  LRB_CHECK(world <= 8, "gemm_rs: at most 8 ranks per tensor-parallel group");
  c10::cuda::CUDAGuard g(X.device());
  CUtensorMap ta = kmajor_map(X.data_ptr(), M, K, X.stride(0), BM), tb = kmajor_map(W.data_ptr(), N, K, W.stride(0), BN);
  CommGemmArgs args{};
  args.M = (int)M; args.N = (int)N; args.K = (int)K; args.rows_per_rank = (int)(M / world);
  args.rank = (int)rank; args.world = (int)world;
  args.bases = reinterpret_cast<const uint64_t*>(bases.data_ptr<int64_t>());
  args.off0 = recv_off; args.off1 = ready_off; args.off2 = consumed_off; args.epoch = (uint32_t)epoch;
  args.counters = reinterpret_cast<unsigned int*>(counters.data_ptr<int>());
  args.err = err.data_ptr<int>();
  auto k = comm_gemm_kernel<false>;
  LRB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
  const int tiles = (int)((M / BM) * ((N + BN - 1) / BN));
  k<<<std::min(tiles, num_sms()), kThreads, kSmem, stream()>>>(ta, tb, args);
  LRB_LAUNCH_CHECK();
}

void tp_reduce(const at::Tensor& recv, const c10::optional<at::Tensor>& residual, at::Tensor& out, int64_t world,
               const at::Tensor& ready, at::Tensor& consumed, int64_t epoch, at::Tensor& counter, at::Tensor& err) {
  LRB_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.dim() == 2, "tp_reduce: out (Mr, N) bf16");
  const int64_t Mr = out.size(0), N = out.size(1);
  const int64_t tiles_n = (N + BN - 1) / BN;
  const int64_t region = ((Mr + BM - 1) / BM) * BM * tiles_n * BN;  // elements per source slot (tile-major)
  LRB_CHECK(N % 8 == 0 && recv.numel() >= world * region, "tp_reduce: receive slots too small");
  if (residual) LRB_CHECK(residual->is_contiguous() && residual->numel() == out.numel(), "tp_reduce: residual shape");
  c10::cuda::CUDAGuard g(out.device());
  const int64_t region8 = region / 8;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((region8 + 255) / 256, (int64_t)num_sms() * 4));
  tp_reduce_kernel<<<blocks, 256, 0, stream()>>>(
      reinterpret_cast<const uint4*>(recv.data_ptr()), residual ? reinterpret_cast<const uint4*>(residual->data_ptr()) : nullptr,
      reinterpret_cast<uint4*>(out.data_ptr()), region8, (int)Mr, (int)N, (int)tiles_n, (int)world,
      reinterpret_cast<const uint32_t*>(ready.data_ptr<int>()), reinterpret_cast<uint32_t*>(consumed.data_ptr<int>()),
      (uint32_t)epoch, reinterpret_cast<unsigned int*>(counter.data_ptr<int>()), err.data_ptr<int>());
  LRB_LAUNCH_CHECK();
}

void shard_publish(const at::Tensor& src, at::Tensor& dst, at::Tensor& ready, int64_t epoch, at::Tensor& counter) {
  const int64_t bytes = src.numel() * src.element_size();
  LRB_CHECK(src.is_contiguous() && dst.numel() * dst.element_size() == bytes && bytes % 16 == 0, "shard_publish");
  c10::cuda::CUDAGuard g(src.device());
  const int64_t n16 = bytes / 16;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n16 + 255) / 256, (int64_t)num_sms() * 4));
  shard_publish_kernel<<<blocks, 256, 0, stream()>>>(reinterpret_cast<const uint4*>(src.data_ptr()),
                                                     reinterpret_cast<uint4*>(dst.data_ptr()), n16,
                                                     reinterpret_cast<uint32_t*>(ready.data_ptr<int>()),
                                                     (uint32_t)epoch, reinterpret_cast<unsigned int*>(counter.data_ptr<int>()));
  LRB_LAUNCH_CHECK();
}

// Y (M x N) = AllGather_rows(shards) W^T; shards live at shard_off in every heap
// (Mr x K bf16, flag at shard_ready_off); a_full is the local gather buffer (M x K).
at::Tensor ag_gemm(const at::Tensor& W, at::Tensor& a_full, at::Tensor& chunk_flags, const at::Tensor& bases,
                   int64_t shard_off, int64_t shard_ready_off, int64_t rank, int64_t world, int64_t epoch,
                   int64_t ncopy, at::Tensor& err) {
  check_bf16_kmajor(W, "ag_gemm W");
  check_bf16_kmajor(a_full, "ag_gemm a_full");
  const int64_t M = a_full.size(0), K = a_full.size(1), N = W.size(0);
  LRB_CHECK(W.size(1) == K && M % (BM * world) == 0 && N % 8 == 0 && a_full.is_contiguous(),
            "ag_gemm: M % (128*world) == 0, N % 8 == 0, contiguous gather buffer");
  LRB_CHECK(chunk_flags.numel() >= M / BM && chunk_flags.scalar_type() == at::kInt, "ag_gemm: chunk flags");
  LRB_CHECK(ncopy >= 1 && ncopy < num_sms(), "ag_gemm: 1 <= ncopy < SMs");
  c10::cuda::CUDAGuard g(W.device());
  auto C = at::empty({M, N}, W.options());
  CUtensorMap ta = kmajor_map(a_full.data_ptr(), M, K, K, BM), tb = kmajor_map(W.data_ptr(), N, K, W.stride(0), BN);
  CommGemmArgs args{};
  args.C = C.data_ptr(); args.ldc = N;
  args.M = (int)M; args.N = (int)N; args.K = (int)K; args.rows_per_rank = (int)(M / world);
  args.rank = (int)rank; args.world = (int)world;
  args.bases = reinterpret_cast<const uint64_t*>(bases.data_ptr<int64_t>());
  args.off0 = shard_off; args.off1 = shard_ready_off; args.epoch = (uint32_t)epoch;
  args.chunk_flags = reinterpret_cast<uint32_t*>(chunk_flags.data_ptr<int>());
  args.a_full = reinterpret_cast<__nv_bfloat16*>(a_full.data_ptr());
  args.ncopy = (int)ncopy;
  args.err = err.data_ptr<int>();
  auto k = comm_gemm_kernel<true>;
  LRB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
  // all CTAs co-resident (one per SM): GEMM CTAs wait on chunks that copy CTAs publish
  k<<<num_sms(), kThreads, kSmem, stream()>>>(ta, tb, args);
  LRB_LAUNCH_CHECK();
  return C;
}

}  // namespace lrb
