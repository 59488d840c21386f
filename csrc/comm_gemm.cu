// GEMMs that carry their own collective over NVLink peer memory.
//
// ag_gemm  (all-gather -> GEMM): out[M, N] = x[M, K] · W[N, K]^T, where W is one
//   tensor of an FSDP unit whose flat parameter is sharded over the ranks' windows
//   (rank p holds elements [p*ss, (p+1)*ss)). The same persistent kernel gathers the
//   WHOLE unit into this rank's resident buffer and computes on W as it arrives:
//   two puller warps per CTA claim 32 KB chunks of the unit from a global counter
//   (W's chunks first, in the order the tiles consume them), copy them from the
//   owners' windows with 16-byte loads into the resident buffer and publish a
//   per-chunk flag (release); the TMA producer acquires the flags covering a tile's
//   W rows before loading them. Tiles are 128 x 256 on tcgen05 (bf16, fp32 in
//   TMEM, double-buffered accumulator), epilogue by TMA stores. Replaces the
//   reference's all_gather_into_tensor followed by the first matmul of the unit
//   (nanospec/shard.py:104-116, 226-253; nanospec/ops.py linear).
//
// gemm_rs  (weight-gradient GEMM -> reduce-scatter): dW[R, C] = dy[T, R]^T · x[T, C]
//   for a tensor at element offset g_off of a unit's flat gradient. The epilogue
//   stores every bf16 output element straight into its owner's receive slot over
//   NVLink: owner p = e / ss of flat element e, at row `rank` of p's slot
//   ([world][ss] per slot). The owner then sums the rows in rank order
//   (peer_reduce_local), so the values equal those of the pull-based reduce-scatter
//   bit for bit. Replaces the reference's reduce_scatter_tensor(AVG) of the unit's
//   full gradient (nanospec/shard.py:140-150, 274-289).
//
// Peer memory is only read by plain loads and written by plain stores: no TMA
// operation touches another GPU's memory. Every wait is bounded; on timeout the
// kernel sets the device error word and stops issuing work.
#include <cuda_runtime.h>

#include "common.h"
#include "peer.h"
#include "sm100.cuh"

namespace ns {
namespace {

constexpr int CG_BM = 128, CG_BN = 256, CG_BK = 64;
constexpr int CG_A_BYTES = CG_BM * CG_BK * 2;                 // 16 KB
constexpr int CG_B_BYTES = CG_BN * CG_BK * 2;                 // 32 KB
constexpr int CG_STAGE = CG_A_BYTES + CG_B_BYTES;             // 48 KB
constexpr int CG_STAGES = 4;
constexpr int CG_BOX = 32 * 128;                              // 32 rows x 64 bf16
constexpr int CG_EPI = 4 * 2 * CG_BOX;                        // two boxes per epilogue warp
constexpr int CG_SMEM = CG_STAGES * CG_STAGE + CG_EPI + 1024 + 256;
constexpr int CG_TMEM = 2 * CG_BN;                            // two accumulators
constexpr int PULL_WARPS = 2;
constexpr int AG_THREADS = 192 + 32 * PULL_WARPS;
constexpr int RS_THREADS = 192;
static_assert(CG_SMEM <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders this thread's generic-proxy global accesses with its async-proxy (TMA) ones.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Window base of rank p without indexing the parameter array at run time (which
// would copy the table to local memory).
__device__ __forceinline__ uint64_t peer_base(const PeerTable& t, uint32_t p) {
  uint64_t b = t.base[0];
#pragma unroll
  for (int i = 1; i < MAX_PEERS; ++i) b = p == (uint32_t)i ? t.base[i] : b;
  return b;
}

struct AgArgs {
  int M, N, K;
  int mt, tiles;
  PeerTable peers;
  int world;
  int64_t src_off;   // byte offset of the unit's shard in every window
  uint32_t ss;       // shard elements (multiple of 8)
  uint32_t total;    // world * ss
  uint4* dst;        // resident unit buffer, `total` elements
  uint32_t w_off;    // element offset of W in the unit
  uint32_t chunk;    // elements per chunk (multiple of 8, <= ss)
  uint32_t nchunks, c0;  // chunk count; W's first chunk (the pull order starts there)
  unsigned* flags;   // [nchunks]: epoch once the chunk is in `dst`
  unsigned* claim;   // chunk claim counter, zero at launch
  unsigned epoch;
  int* err;
  long long limit;   // polls per flag wait
};

// Epilogue common to both kernels: the accumulator rows of warp q (32 lanes) at
// columns [c, c + 64) converted to bf16 into a 32 x 64 box with the 128-byte swizzle
// (16-byte chunk j of row r at chunk j ^ (r % 8)).
__device__ __forceinline__ void box_from_tmem(uint32_t trow, int c, uint8_t* sb, int lane) {
  float v0[32], v1[32];
  sm100::tmem_ld32(trow + (uint32_t)c, v0);
  sm100::tmem_ld32(trow + (uint32_t)(c + 32), v1);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float* src = j < 4 ? v0 + 8 * j : v1 + 8 * (j - 4);
    __nv_bfloat162 h[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) h[t] = __floats2bfloat162_rn(src[2 * t], src[2 * t + 1]);
    *reinterpret_cast<uint4*>(sb + lane * 128 + ((j ^ (lane & 7)) * 16)) = *reinterpret_cast<uint4*>(h);
  }
}

// ============================================================================ AG -> GEMM
__global__ void __launch_bounds__(AG_THREADS, 1)
    ag_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ CUtensorMap to, AgArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + CG_STAGES * CG_A_BYTES;
  uint8_t* sE = sB + CG_STAGES * CG_B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + CG_EPI);
  uint64_t* empty = full + CG_STAGES;
  uint64_t* tfull = empty + CG_STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (a.K + CG_BK - 1) / CG_BK;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < CG_STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull[b], 1);
      sm100::mbar_init(&tempty[b], 4);
    }
    sm100::fence_barrier_init();
    sm100::tma_prefetch_desc(&ta);
    sm100::tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, CG_TMEM);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 6) {
    // ---------------------------------------------------------------- pullers
    for (;;) {
      unsigned j = 0;
      if (lane == 0) j = atomicAdd(a.claim, 1u);
      j = __shfl_sync(0xffffffffu, j, 0);
      if (j >= a.nchunks) break;
      const uint32_t c = (a.c0 + j) % a.nchunks;
      const uint32_t e0 = c * a.chunk;
      const uint32_t e1 = min(e0 + a.chunk, a.total);
      // a chunk is no longer than a shard, so it spans at most two owners
      const uint32_t p0 = e0 / a.ss;
      const uint32_t edge = (p0 + 1) * a.ss;
      const uint32_t v0 = e0 / 8, v1 = e1 / 8;
      for (uint32_t v = v0 + lane; v < v1; v += 32 * 8) {
        uint4 r[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint32_t vv = v + 32 * u;
          if (vv < v1) {
            const uint32_t e = vv * 8;
            const uint32_t p = e < edge ? p0 : p0 + 1;
            r[u] = *reinterpret_cast<const uint4*>(peer_base(a.peers, p) + a.src_off + (uint64_t)(e - p * a.ss) * 2);
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint32_t vv = v + 32 * u;
          if (vv < v1) a.dst[vv] = r[u];
        }
      }
      __threadfence();
      fence_proxy_async_global();
      __syncwarp();
      if (lane == 0) st_release_gpu(a.flags + c, a.epoch);
    }
  } else if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < a.tiles && ok; u += gridDim.x) {
      const int m0 = (u % a.mt) * CG_BM, n0 = (u / a.mt) * CG_BN;
      const int n1 = min(n0 + CG_BN, a.N);
      const uint32_t lo = a.w_off + (uint32_t)n0 * a.K, hi = a.w_off + (uint32_t)n1 * a.K;
      const uint32_t clo = lo / a.chunk, chi = (hi - 1) / a.chunk;
      bool ready = true;
      for (uint32_t c = clo + lane; c <= chi && ready; c += 32) {
        long long i = 0;
        while ((int)(ld_acquire_gpu(a.flags + c) - a.epoch) < 0) {
          if (++i > a.limit) {
            ready = false;
            break;
          }
          __nanosleep(64);
        }
      }
      if (!__all_sync(0xffffffffu, ready)) {
        if (lane == 0) atomicExch(a.err, 2);
        ok = false;
        break;
      }
      int lane_ok = 1;
      if (lane == 0) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        fence_proxy_async_global();
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CG_STAGES;
          if (it >= CG_STAGES && !sm100::mbar_wait(&empty[s], ((it / CG_STAGES) & 1) ^ 1, a.err)) {
            lane_ok = 0;
            break;
          }
          sm100::mbar_expect_tx(&full[s], CG_STAGE);
          sm100::tma_load_2d(sA + s * CG_A_BYTES, &ta, &full[s], kb * CG_BK, m0);
          sm100::tma_load_2d(sB + s * CG_B_BYTES, &tb, &full[s], kb * CG_BK, n0);
        }
      }
      ok = __shfl_sync(0xffffffffu, lane_ok, 0) != 0;
    }
    if (lane == 0)
      for (int i = max(0, it - CG_STAGES); i < it; ++i) sm100::mbar_wait(&full[i % CG_STAGES], (i / CG_STAGES) & 1, a.err);
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_bf16(CG_BM, CG_BN, false, false);
      int it = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < a.tiles && ok; u += gridDim.x, ++local) {
        const int buf = local & 1;
        if (local >= 2 && !sm100::mbar_wait(&tempty[buf], ((local >> 1) - 1) & 1, a.err)) break;
        sm100::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * CG_BN);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CG_STAGES;
          if (!sm100::mbar_wait(&full[s], (it / CG_STAGES) & 1, a.err)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_u32(sA + s * CG_A_BYTES);
          const uint32_t b_base = sm100::smem_u32(sB + s * CG_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < CG_BK / 16; ++kk) {
            const uint64_t ad = sm100::smem_desc_sw128(a_base + kk * 32, 0, 1024);
            const uint64_t bd = sm100::smem_desc_sw128(b_base + kk * 32, 0, 1024);
            sm100::mma_bf16(d, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          sm100::mma_commit(&empty[s]);
        }
        if (ok) sm100::mma_commit(&tfull[buf]);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int q = warp & 3;
    uint8_t* stg = sE + q * 2 * CG_BOX;
    int local = 0, box = 0;
    for (int u = blockIdx.x; u < a.tiles; u += gridDim.x, ++local) {
      const int buf = local & 1;
      const int m0 = (u % a.mt) * CG_BM, n0 = (u / a.mt) * CG_BN;
      if (!sm100::mbar_wait(&tfull[buf], (local >> 1) & 1, a.err)) break;
      sm100::tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * CG_BN);
#pragma unroll 1
      for (int c = 0; c < CG_BN; c += 64, ++box) {
        if (n0 + c >= a.N) break;
        uint8_t* sb = stg + (box & 1) * CG_BOX;
        if (lane == 0) sm100::bulk_wait_read<1>();
        __syncwarp();
        box_from_tmem(trow, c, sb, lane);
        sm100::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          sm100::tma_store_2d(&to, sb, n0 + c, m0 + q * 32);
          sm100::bulk_commit();
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tempty[buf]);
    }
    if (lane == 0) sm100::bulk_wait<0>();
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, CG_TMEM);
  }
}

// ============================================================================ GEMM -> RS
struct RsArgs {
  int R, C, T;
  int mt, tiles;
  PeerTable peers;
  int world, rank;
  int64_t slot_off;  // byte offset of the receive slot in every window
  uint32_t ss;       // shard elements (multiple of 8)
  uint32_t g_off;    // element offset of dW in the unit's flat gradient
  int* err;
};

__global__ void __launch_bounds__(RS_THREADS, 1)
    gemm_rs_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, RsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + CG_STAGES * CG_A_BYTES;
  uint8_t* sE = sB + CG_STAGES * CG_B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + CG_EPI);
  uint64_t* empty = full + CG_STAGES;
  uint64_t* tfull = empty + CG_STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (a.T + CG_BK - 1) / CG_BK;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < CG_STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull[b], 1);
      sm100::mbar_init(&tempty[b], 4);
    }
    sm100::fence_barrier_init();
    sm100::tma_prefetch_desc(&ta);
    sm100::tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, CG_TMEM);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // Both operands are token-major ([T][R] and [T][C]): MN-major tiles, 64-wide boxes.
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < a.tiles && ok; u += gridDim.x) {
        const int r0 = (u % a.mt) * CG_BM, c0 = (u / a.mt) * CG_BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CG_STAGES;
          if (it >= CG_STAGES && !sm100::mbar_wait(&empty[s], ((it / CG_STAGES) & 1) ^ 1, a.err)) {
            ok = false;
            break;
          }
          sm100::mbar_expect_tx(&full[s], CG_STAGE);
          const int t = kb * CG_BK;
          uint8_t* a_dst = sA + s * CG_A_BYTES;
          uint8_t* b_dst = sB + s * CG_B_BYTES;
          sm100::tma_load_2d(a_dst, &ta, &full[s], r0, t);
          sm100::tma_load_2d(a_dst + CG_BK * 128, &ta, &full[s], r0 + 64, t);
#pragma unroll
          for (int j = 0; j < CG_BN / 64; ++j) sm100::tma_load_2d(b_dst + j * (CG_BK * 128), &tb, &full[s], c0 + 64 * j, t);
        }
      }
      for (int i = max(0, it - CG_STAGES); i < it; ++i) sm100::mbar_wait(&full[i % CG_STAGES], (i / CG_STAGES) & 1, a.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_bf16(CG_BM, CG_BN, true, true);
      int it = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < a.tiles && ok; u += gridDim.x, ++local) {
        const int buf = local & 1;
        if (local >= 2 && !sm100::mbar_wait(&tempty[buf], ((local >> 1) - 1) & 1, a.err)) break;
        sm100::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * CG_BN);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % CG_STAGES;
          if (!sm100::mbar_wait(&full[s], (it / CG_STAGES) & 1, a.err)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_u32(sA + s * CG_A_BYTES);
          const uint32_t b_base = sm100::smem_u32(sB + s * CG_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < CG_BK / 16; ++kk) {
            const uint64_t ad = sm100::smem_desc_sw128(a_base + kk * 2048, CG_BK * 128, 1024);
            const uint64_t bd = sm100::smem_desc_sw128(b_base + kk * 2048, CG_BK * 128, 1024);
            sm100::mma_bf16(d, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          sm100::mma_commit(&empty[s]);
        }
        if (ok) sm100::mma_commit(&tfull[buf]);
      }
    }
  } else {
    // Epilogue: a 32 x 64 box per step, bf16 in swizzled shared memory, then written
    // row-contiguously (8 lanes x 16 B = one 128-byte row segment) to the owners.
    const int q = warp & 3;
    uint8_t* sb = sE + q * 2 * CG_BOX;
    int local = 0;
    for (int u = blockIdx.x; u < a.tiles; u += gridDim.x, ++local) {
      const int buf = local & 1;
      const int r0 = (u % a.mt) * CG_BM, c0 = (u / a.mt) * CG_BN;
      if (!sm100::mbar_wait(&tfull[buf], (local >> 1) & 1, a.err)) break;
      sm100::tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * CG_BN);
#pragma unroll 1
      for (int c = 0; c < CG_BN; c += 64) {
        if (c0 + c >= a.C) break;
        __syncwarp();  // the previous box has been read out
        box_from_tmem(trow, c, sb, lane);
        __syncwarp();
        const int j = lane & 7;
        const int col = c0 + c + 8 * j;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + (lane >> 3);
          const int row = r0 + q * 32 + r;
          if (row < a.R && col < a.C) {
            const uint4 v = *reinterpret_cast<const uint4*>(sb + r * 128 + ((j ^ (r & 7)) * 16));
            const uint32_t e = a.g_off + (uint32_t)row * (uint32_t)a.C + (uint32_t)col;
            const uint32_t p = e / a.ss;
            *reinterpret_cast<uint4*>(peer_base(a.peers, p) + a.slot_off +
                                      ((uint64_t)a.rank * a.ss + (e - p * a.ss)) * 2) = v;
          }
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tempty[buf]);
    }
    __threadfence_system();  // every store of this thread reaches its owner before the slot is flagged
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, CG_TMEM);
  }
}

// Pushes elements [lo, hi) of a local full-size gradient buffer to their owners'
// receive slots (row `rank`), 8 elements per store. Used for the parameters whose
// gradients are not produced by gemm_rs (norm weights, embeddings, padding).
__global__ void peer_push_kernel(PeerTable t, int rank, int64_t slot_off, uint32_t ss, const uint4* src, uint32_t lo8,
                                 uint32_t hi8) {
  for (uint32_t v = lo8 + blockIdx.x * blockDim.x + threadIdx.x; v < hi8; v += gridDim.x * blockDim.x) {
    const uint32_t e = v * 8;
    const uint32_t p = e / ss;
    *reinterpret_cast<uint4*>(peer_base(t, p) + slot_off + ((uint64_t)rank * ss + (e - p * ss)) * 2) = src[v];
  }
  __threadfence_system();
}

}  // namespace

// out[M, N] = x[M, K] · W^T with W = unit[w_off : w_off + N*K] viewed [N, K]; the unit
// (world * ss bf16 elements, shards at byte `src_off` of every window of `id`) is
// gathered into `resident` by the same kernel. `flags` (int32, >= chunk count) and
// `claim` (int32 [1]) belong to the caller; `epoch` must grow by one per call that
// uses the same flags.
void ag_gemm(int64_t id, int64_t src_off, int64_t ss, at::Tensor resident, int64_t w_off, int64_t N, int64_t K,
             at::Tensor x, at::Tensor out, at::Tensor flags, at::Tensor claim, int64_t epoch, int64_t poll_limit) {
  const WindowInfo w = window_info(id);
  check_bf16(x, "x");
  check_bf16(out, "out");
  check_bf16(resident, "resident");
  const int64_t total = ss * w.world;
  const int64_t M = x.size(0);
  NS_CHECK(x.dim() == 2 && x.size(1) == K && x.stride(1) == 1 && x.stride(0) % 8 == 0, "x must be [M, K] with 16-byte rows");
  NS_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1 && out.stride(0) % 8 == 0,
           "out must be [M, N] with 16-byte rows");
  NS_CHECK(ss % 8 == 0 && src_off % 16 == 0 && w_off % 8 == 0 && K % 8 == 0, "fused all-gather needs 16-byte aligned shards");
  NS_CHECK(resident.numel() >= total && total < (int64_t(1) << 32), "resident buffer too small or unit too large");
  NS_CHECK(w_off + N * K <= total, "W outside the unit");
  NS_CHECK(reinterpret_cast<uintptr_t>(resident.data_ptr()) % 16 == 0, "resident buffer must be 16-byte aligned");
  const int64_t chunk = std::min<int64_t>(16384, ss);
  const int64_t nchunks = (total + chunk - 1) / chunk;
  NS_CHECK(flags.scalar_type() == at::kInt && flags.numel() >= nchunks && flags.is_contiguous(), "flags too small");
  NS_CHECK(claim.scalar_type() == at::kInt && claim.numel() >= 1, "claim counter missing");
  auto* base = static_cast<__nv_bfloat16*>(resident.data_ptr());
  CUtensorMap ta = make_tmap_bf16(x.data_ptr(), M, K, x.stride(0), CG_BM, 64);
  CUtensorMap tb = make_tmap_bf16(base + w_off, N, K, K, CG_BN, 64);
  CUtensorMap to = make_tmap_bf16(out.data_ptr(), M, N, out.stride(0), 32, 64);
  AgArgs a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.mt = (int)((M + CG_BM - 1) / CG_BM);
  a.tiles = a.mt * (int)((N + CG_BN - 1) / CG_BN);
  a.peers = w.table;
  a.world = w.world;
  a.src_off = src_off;
  a.ss = (uint32_t)ss;
  a.total = (uint32_t)total;
  a.dst = reinterpret_cast<uint4*>(base);
  a.w_off = (uint32_t)w_off;
  a.chunk = (uint32_t)chunk;
  a.nchunks = (uint32_t)nchunks;
  a.c0 = (uint32_t)(w_off / chunk);
  a.flags = reinterpret_cast<unsigned*>(flags.data_ptr());
  a.claim = reinterpret_cast<unsigned*>(claim.data_ptr());
  a.epoch = (unsigned)epoch;
  a.err = device_error_flag();
  a.limit = poll_limit;
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(ag_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CG_SMEM));
  });
  NS_CUDA(cudaMemsetAsync(claim.data_ptr(), 0, sizeof(int), stream()));
  // one CTA per SM whatever the tile count: every CTA's pullers share the gather
  ag_gemm_kernel<<<num_sms(), AG_THREADS, CG_SMEM, stream()>>>(ta, tb, to, a);
  NS_CUDA(cudaGetLastError());
}

// dW = dy^T · x (dy [T, R], x [T, C]) for the tensor at element `g_off` of a unit's
// flat gradient, stored into the owners' receive slots at byte `slot_off` of the
// windows of `id` (row = this rank).
void gemm_rs(int64_t id, int64_t slot_off, int64_t ss, int64_t g_off, at::Tensor dy, at::Tensor x) {
  const WindowInfo w = window_info(id);
  check_bf16(dy, "dy");
  check_bf16(x, "x");
  NS_CHECK(dy.dim() == 2 && x.dim() == 2 && dy.size(0) == x.size(0), "dy [T, R] and x [T, C] expected");
  NS_CHECK(dy.stride(1) == 1 && x.stride(1) == 1 && dy.stride(0) % 8 == 0 && x.stride(0) % 8 == 0,
           "dy and x need 16-byte rows");
  const int64_t T = dy.size(0), R = dy.size(1), C = x.size(1);
  const int64_t total = ss * w.world;
  NS_CHECK(ss % 8 == 0 && g_off % 8 == 0 && C % 8 == 0 && slot_off % 16 == 0, "fused reduce-scatter needs 16-byte aligned shards");
  NS_CHECK(g_off + R * C <= total && total < (int64_t(1) << 32), "dW outside the unit or unit too large");
  NS_CHECK(slot_off + total * 2 <= w.bytes, "receive slot outside the window");
  CUtensorMap ta = make_tmap_bf16(dy.data_ptr(), T, R, dy.stride(0), CG_BK, 64);
  CUtensorMap tb = make_tmap_bf16(x.data_ptr(), T, C, x.stride(0), CG_BK, 64);
  RsArgs a{};
  a.R = (int)R;
  a.C = (int)C;
  a.T = (int)T;
  a.mt = (int)((R + CG_BM - 1) / CG_BM);
  a.tiles = a.mt * (int)((C + CG_BN - 1) / CG_BN);
  a.peers = w.table;
  a.world = w.world;
  a.rank = w.rank;
  a.slot_off = slot_off;
  a.ss = (uint32_t)ss;
  a.g_off = (uint32_t)g_off;
  a.err = device_error_flag();
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(gemm_rs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CG_SMEM));
  });
  const int grid = std::min(a.tiles, num_sms());
  gemm_rs_kernel<<<grid, RS_THREADS, CG_SMEM, stream()>>>(ta, tb, a);
  NS_CUDA(cudaGetLastError());
}

// Elements [lo, hi) of `src` (a local full-size unit gradient) to their owners' slots.
void peer_push(int64_t id, int64_t slot_off, int64_t ss, at::Tensor src, int64_t lo, int64_t hi) {
  const WindowInfo w = window_info(id);
  check_bf16(src, "src");
  NS_CHECK(ss % 8 == 0 && lo % 8 == 0 && hi % 8 == 0 && slot_off % 16 == 0, "push ranges must be 16-byte aligned");
  NS_CHECK(0 <= lo && lo <= hi && hi <= ss * w.world && src.numel() >= hi, "push range outside the unit");
  NS_CHECK(reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0, "push source must be 16-byte aligned");
  if (hi == lo) return;
  const int64_t n8 = (hi - lo) / 8;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n8 + 255) / 256, (int64_t)num_sms() * 2));
  peer_push_kernel<<<blocks, 256, 0, stream()>>>(w.table, w.rank, slot_off, (uint32_t)ss,
                                                 reinterpret_cast<const uint4*>(src.data_ptr()), (uint32_t)(lo / 8),
                                                 (uint32_t)(hi / 8));
  NS_CUDA(cudaGetLastError());
}

}  // namespace ns
