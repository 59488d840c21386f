// bf16 GEMM on 5th-generation tensor cores (tcgen05, TMEM accumulators, TMA).
//
//   D[M, N] = sum_k A[m, k] * B[n, k]      (fp32 accumulation in TMEM)
//
// A and B are each either K-major (row-major [rows, K]) or MN-major (row-major
// [K, rows]); that covers the forward (x W^T), input-gradient (dy W) and
// weight-gradient (dy^T x) products of a linear layer without transposes.
// Small token counts use "swap-AB": the weight supplies the 128-row M side and
// the output is written transposed.
//
// One CTA = one 128 x BN output tile over a K range (split-K across blockIdx.z):
//   warp 0   : one thread issues TMA loads into a `stages`-deep smem ring;
//   warp 1   : allocates TMEM; one thread issues tcgen05.mma (K = 16 per issue)
//              and commits each stage back to the producer;
//   warps 2-5: epilogue, tcgen05.ld of the accumulator (each warp owns the TMEM
//              lane quarter warp % 4), then bf16/fp32 stores with optional
//              residual / accumulate.
// K depth per stage: 128 for small-N tiles (weight-streaming products, where the
// per-stage handshake between producer, MMA issuer and barrier dominates), 64 for
// wide tiles. Split-K (up to 8 splits): the splits of a tile form a thread-block
// cluster; each parks its fp32 partial in its own shared memory and, after a cluster
// barrier, reduces 1/S of the tile over DSMEM in split order 0..S-1. More splits use
// fp32 partials in global memory and a last-arriving-CTA fix-up (per-tile arrival
// counter). Either way the result is deterministic and no second kernel runs.
// Grids with more tiles than SMs use gemm_bf16_persistent (below). plan_gemm picks
// tile width, split count and kernel from a time model, once per problem shape.
// Every mbarrier wait is bounded; a timeout sets the device error flag.
#include <cmath>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

#include "common.h"
#include "gemm.h"
#include "gemm_noalloc.h"
#include "sm100.cuh"

namespace ns {

constexpr int BM = 128;

struct GemmArgs {
  int M, N, K;
  int kpb;  // k-blocks per split
  int splits;
  float* out_f32;  // fp32 output (accumulate adds), used instead of `out` when set
  __nv_bfloat16* out;
  int64_t out_sm, out_sn;    // element strides of out(m, n)
  const __nv_bfloat16* res;  // optional residual, same addressing as out
  int64_t res_sm, res_sn;
  int accumulate;  // out = out + D
  float* ws;       // split-K partials [splits][M][N] (ws_t: [splits][N][M])
  int ws_t;
  unsigned* counters;  // per-tile arrival counters (zero between launches)
  int* err;
  long long* trace;  // test hook: clock stamps of CTA 0 and per-CTA phase times, or null
  int tma_store;     // persistent kernel: plain bf16 row-major output written by TMA stores
  int cluster_red;   // split-K: the splits of a tile form a cluster and reduce through DSMEM
  const float* nfac; // with npart: npart[cta] = sum of bf16(out * *nfac)^2 over this CTA's outputs
  float* npart;
};

constexpr int CLUSTER_MAX = 8;  // portable cluster size: the largest split count reduced in DSMEM

// fp32 partial tile in shared memory for the cluster reduction: [128 rows][BN + 4]
// ([BN][128 + 4] when the output is transposed), the padding keeps both the
// per-row writes and the per-column reads free of bank conflicts.
__host__ __device__ constexpr int partial_ld(int bn, int ws_t) { return ws_t ? 128 + 4 : bn + 4; }
__host__ __device__ constexpr int partial_bytes(int bn) { return (bn + 4) * (128 + 4) * 4; }

template <int BN>
struct GemmCfg {
  static constexpr int BK = BN <= 128 ? 128 : 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // Ring depth: two CTAs per SM when the grid has more CTAs than SMs (epilogues
  // overlap mainloops); otherwise one CTA per SM with the deepest ring that fits.
  static constexpr int STAGES = (110 * 1024) / STAGE_BYTES;
  static constexpr int STAGES_SOLO = (224 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int SMEM_MAX = STAGES_SOLO * STAGE_BYTES + 1024 + 256;
};

static int bk_for(int bn) { return bn <= 128 ? 128 : 64; }

// Two-phase form of store_final for batches: load the residual / old output of
// every element first (final_load), then write (final_write).
__device__ __forceinline__ void final_load(const GemmArgs& a, int m, int n, float& add, float& old) {
  add = a.res ? __bfloat162float(a.res[m * a.res_sm + n * a.res_sn]) : 0.f;
  old = 0.f;
  if (a.accumulate)
    old = a.out_f32 ? a.out_f32[m * a.out_sm + n * a.out_sn] : __bfloat162float(a.out[m * a.out_sm + n * a.out_sn]);
}

__device__ __forceinline__ void final_write(const GemmArgs& a, int m, int n, float acc, float add, float old) {
  if (a.out_f32) {
    a.out_f32[m * a.out_sm + n * a.out_sn] = a.accumulate ? old + acc : acc;
    return;
  }
  float y = sm100::bf16_round(acc);
  if (a.res) y = sm100::bf16_round(add + y);
  if (a.accumulate) y = sm100::bf16_round(old + y);
  a.out[m * a.out_sm + n * a.out_sn] = __float2bfloat16(y);
}

__device__ __forceinline__ void store_final(const GemmArgs& a, int m, int n, float acc) {
  if (a.out_f32) {
    float* q = a.out_f32 + m * a.out_sm + n * a.out_sn;
    *q = a.accumulate ? *q + acc : acc;
    return;
  }
  float y = sm100::bf16_round(acc);
  if (a.res) y = sm100::bf16_round(__bfloat162float(a.res[m * a.res_sm + n * a.res_sn]) + y);
  __nv_bfloat16* p = a.out + m * a.out_sm + n * a.out_sn;
  if (a.accumulate) y = sm100::bf16_round(__bfloat162float(*p) + y);
  *p = __float2bfloat16(y);
}

// Epilogue of 32 consecutive columns [nb, nb+32) of row m.
__device__ __forceinline__ void store_row32(const GemmArgs& a, int m, int nb, const float (&v)[32]) {
  if (!a.out_f32 && a.out_sn == 1 && !a.res && !a.accumulate && nb + 32 <= a.N && (a.out_sm % 8) == 0) {
    uint4* p = reinterpret_cast<uint4*>(a.out + m * a.out_sm + nb);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 h[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) h[t] = __floats2bfloat162_rn(v[8 * j + 2 * t], v[8 * j + 2 * t + 1]);
      p[j] = *reinterpret_cast<uint4*>(h);
    }
    return;
  }
  // General path: every load (residual, accumulated output) is issued before the
  // first store, so the 32 read-modify-writes do not serialise on memory latency.
  const int cnt = min(32, a.N - nb);
  if (a.out_f32) {
    float* q = a.out_f32 + m * a.out_sm + nb * a.out_sn;
    float old[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) old[j] = (a.accumulate && j < cnt) ? q[j * a.out_sn] : 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < cnt) q[j * a.out_sn] = old[j] + v[j];
    return;
  }
  __nv_bfloat16* p = a.out + m * a.out_sm + nb * a.out_sn;
  float add[32], old[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    add[j] = (a.res && j < cnt) ? __bfloat162float(a.res[m * a.res_sm + (int64_t)(nb + j) * a.res_sn]) : 0.f;
    old[j] = (a.accumulate && j < cnt) ? __bfloat162float(p[j * a.out_sn]) : 0.f;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j >= cnt) break;
    float y = sm100::bf16_round(v[j]);
    if (a.res) y = sm100::bf16_round(add[j] + y);
    if (a.accumulate) y = sm100::bf16_round(old[j] + y);
    p[j * a.out_sn] = __float2bfloat16(y);
  }
}

// Squared-norm contribution of 32 stored bf16 outputs of row m (plain outputs only).
__device__ __forceinline__ float norm_row32(const GemmArgs& a, int m, int nb, const float (&v)[32], float fac) {
  float t = 0.f;
  if (m >= a.M) return t;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (nb + j < a.N) {
      const float g = sm100::bf16_round(sm100::bf16_round(v[j]) * fac);
      t += g * g;
    }
  return t;
}

// One float per CTA: the block's sum of the threads' norm contributions, in warp order.
__device__ __forceinline__ void write_norm_part(const GemmArgs& a, float t, int cta) {
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffff, t, o);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
    a.npart[cta] = s;
  }
}

__device__ __forceinline__ int64_t ws_index(const GemmArgs& a, int s, int m, int n) {
  const int64_t base = (int64_t)s * a.M * a.N;
  return base + (a.ws_t ? (int64_t)n * a.M + m : (int64_t)m * a.N + n);
}

template <int BN, bool AMN, bool BMN>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                     GemmArgs args, int stages) {
  using C = GemmCfg<BN>;
  constexpr int BK = C::BK;
  constexpr int KATOMS = BK / 64;  // 128-byte swizzle atoms along K per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + stages * C::A_BYTES;
  // barriers after the ring, or after the cluster reduction's partial tile if larger
  const int ring = stages * C::STAGE_BYTES;
  const int bar_off = (args.cluster_red && partial_bytes(BN) > ring) ? partial_bytes(BN) : ring;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + bar_off);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  uint32_t* last_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN, split = blockIdx.z;
  const int cta_id = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  auto stamp = [&](int phase) {
    if (args.trace && threadIdx.x == 0 && cta_id < 2048) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      args.trace[512 + phase * 2048 + cta_id] = (long long)t;
    }
  };
  const bool trace0 = args.trace && cta_id == 0;
  stamp(0);
  const int kb_total = (args.K + BK - 1) / BK;
  const int kb0 = split * args.kpb;
  const int kb1 = min(kb0 + args.kpb, kb_total);
  const int nkb = kb1 - kb0;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < stages; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    sm100::mbar_init(acc_full, 1);
    sm100::fence_barrier_init();
    sm100::tma_prefetch_desc(&ta);
    sm100::tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, C::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  stamp(1);

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t ph = (i / stages) & 1;
        if (i >= stages && !sm100::mbar_wait(&empty[s], ph ^ 1, args.err)) break;
        if (trace0 && i < 256) args.trace[i] = clock64();
        sm100::mbar_expect_tx(&full[s], C::STAGE_BYTES);
        const int k = (kb0 + i) * BK;
        uint8_t* a_dst = sA + s * C::A_BYTES;
        uint8_t* b_dst = sB + s * C::B_BYTES;
        if (!AMN) {
#pragma unroll
          for (int j = 0; j < KATOMS; ++j) sm100::tma_load_2d(a_dst + j * (BM * 128), &ta, &full[s], k + 64 * j, m0);
        } else {
          sm100::tma_load_2d(a_dst, &ta, &full[s], m0, k);
          sm100::tma_load_2d(a_dst + BK * 128, &ta, &full[s], m0 + 64, k);
        }
        if (!BMN) {
#pragma unroll
          for (int j = 0; j < KATOMS; ++j) sm100::tma_load_2d(b_dst + j * (BN * 128), &tb, &full[s], k + 64 * j, n0);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) sm100::tma_load_2d(b_dst + j * (BK * 128), &tb, &full[s], n0 + 64 * j, k);
        }
        issued = i + 1;
      }
      // Drain: the last use of every stage must have landed before the CTA exits.
      for (int i = max(0, issued - stages); i < issued; ++i)
        sm100::mbar_wait(&full[i % stages], (i / stages) & 1, args.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_bf16(BM, BN, AMN, BMN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t ph = (i / stages) & 1;
        if (!sm100::mbar_wait(&full[s], ph, args.err)) break;
        if (trace0 && i < 256) args.trace[256 + i] = clock64();
        sm100::tc_fence_after();
        const uint32_t a_base = sm100::smem_u32(sA + s * C::A_BYTES);
        const uint32_t b_base = sm100::smem_u32(sB + s * C::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // K-major: swizzle atom kk/4 (128 B of K), 32 bytes per 16-element slice inside it.
          // MN-major: 16 rows of 128 B per slice; the second 64-wide M/N half sits BK*128 B on.
          const uint64_t ad =
              AMN ? sm100::smem_desc_sw128(a_base + kk * 2048, BK * 128, 1024)
                  : sm100::smem_desc_sw128(a_base + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bd =
              BMN ? sm100::smem_desc_sw128(b_base + kk * 2048, BK * 128, 1024)
                  : sm100::smem_desc_sw128(b_base + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 0, 1024);
          sm100::mma_bf16(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        sm100::mma_commit(&empty[s]);
      }
      sm100::mma_commit(acc_full);
    }
  }
  const int q = warp & 3;
  const int m = m0 + q * 32 + lane;
  const float nf = args.npart ? *args.nfac : 0.f;
  float nsum = 0.f;
  if (warp >= 2) {
    if (sm100::mbar_wait(acc_full, 0, args.err)) {
      sm100::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        sm100::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
        if (m >= args.M) continue;
        const int nb = n0 + c;
        if (args.splits > 1 && args.cluster_red) {
          // partial tile into this CTA's own shared memory (the ring is idle now)
          float* pt = reinterpret_cast<float*>(smem);
          const int row = q * 32 + lane;
          if (!args.ws_t) {
            float4* p = reinterpret_cast<float4*>(pt + row * partial_ld(BN, 0) + c);
#pragma unroll
            for (int j = 0; j < 8; ++j) p[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) pt[(c + j) * partial_ld(BN, 1) + row] = v[j];
          }
        } else if (args.splits > 1) {
          if (!args.ws_t && nb + 32 <= args.N && (args.N % 4) == 0) {
            float4* p = reinterpret_cast<float4*>(args.ws + ws_index(args, split, m, nb));
#pragma unroll
            for (int j = 0; j < 8; ++j) p[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < args.N) args.ws[ws_index(args, split, m, nb + j)] = v[j];
          }
        } else {
          store_row32(args, m, nb, v);
          if (args.npart) nsum += norm_row32(args, m, nb, v, nf);
        }
      }
    }
  }
  stamp(2);
  sm100::tc_fence_before();
  __syncthreads();
  stamp(3);
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (args.splits > 1 && args.cluster_red) {
    // The S split CTAs of this tile are one cluster: after the barrier each reduces
    // 1/S of the tile by reading every member's partial (in split order 0..S-1)
    // through distributed shared memory, then writes the output; a second barrier
    // keeps every member's shared memory alive until all reads are done.
    sm100::cluster_sync();
    const int S = args.splits;
    const uint32_t rank = sm100::cluster_ctarank();
    const int inner = args.ws_t ? BM : BN;
    const int ginner = inner / 4;
    const int G = ginner * (args.ws_t ? BN : BM);
    const int per = (G + S - 1) / S;
    const int g_lo = (int)rank * per, g_hi = min(G, g_lo + per);
    const int pld = partial_ld(BN, args.ws_t);
    const uint32_t base = sm100::smem_u32(smem);
    const bool plain = !args.out_f32 && !args.res && !args.accumulate;
    for (int g = g_lo + threadIdx.x; g < g_hi; g += blockDim.x) {
      const int o = g / ginner, i4 = (g % ginner) * 4;
      const uint32_t off = base + (uint32_t)((o * pld + i4) * 4);
      float4 part[CLUSTER_MAX];
#pragma unroll
      for (int s2 = 0; s2 < CLUSTER_MAX; ++s2)
        if (s2 < S) part[s2] = sm100::dsmem_ld4(sm100::dsmem_map(off, (uint32_t)s2));
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s2 = 0; s2 < CLUSTER_MAX; ++s2)
        if (s2 < S) {
          acc[0] += part[s2].x;
          acc[1] += part[s2].y;
          acc[2] += part[s2].z;
          acc[3] += part[s2].w;
        }
      const int gm = args.ws_t ? m0 + i4 : m0 + o;
      const int gn = args.ws_t ? n0 + o : n0 + i4;
      if (gm >= args.M || gn >= args.N) continue;
      const int lim = min(4, args.ws_t ? args.M - gm : args.N - gn);
      const bool contig = lim == 4 && ((args.ws_t ? args.out_sm : args.out_sn) == 1) &&
                          ((args.ws_t ? args.out_sn : args.out_sm) % 4 == 0) &&
                          reinterpret_cast<uintptr_t>(args.out) % 8 == 0;
      if (plain && contig) {
        __nv_bfloat162 h[2] = {__floats2bfloat162_rn(acc[0], acc[1]), __floats2bfloat162_rn(acc[2], acc[3])};
        *reinterpret_cast<uint2*>(args.out + gm * args.out_sm + gn * args.out_sn) = *reinterpret_cast<uint2*>(h);
        continue;
      }
      if (contig && args.res && !args.out_f32 && !args.accumulate &&
          ((args.ws_t ? args.res_sm : args.res_sn) == 1) && ((args.ws_t ? args.res_sn : args.res_sm) % 4 == 0) &&
          reinterpret_cast<uintptr_t>(args.res) % 8 == 0) {
        // y = bf16(res + bf16(acc)) for 4 contiguous outputs, 8-byte loads and stores
        const uint2 rv = *reinterpret_cast<const uint2*>(args.res + gm * args.res_sm + gn * args.res_sn);
        const __nv_bfloat16* rh = reinterpret_cast<const __nv_bfloat16*>(&rv);
        __nv_bfloat16 o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          o[e] = __float2bfloat16(__bfloat162float(rh[e]) + sm100::bf16_round(acc[e]));
        *reinterpret_cast<uint2*>(args.out + gm * args.out_sm + gn * args.out_sn) = *reinterpret_cast<uint2*>(o);
        continue;
      }
      float add[4], old[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        add[e] = old[e] = 0.f;
        if (e < lim) final_load(args, args.ws_t ? gm + e : gm, args.ws_t ? gn : gn + e, add[e], old[e]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (e < lim) final_write(args, args.ws_t ? gm + e : gm, args.ws_t ? gn : gn + e, acc[e], add[e], old[e]);
    }
    sm100::cluster_sync();
  } else if (args.splits > 1) {
    // Arrival: the last split CTA of this tile reduces all partials in order.
    if (threadIdx.x == 0) {
      __threadfence();
      const int tile = blockIdx.y * gridDim.x + blockIdx.x;
      const unsigned prev = atomicAdd(&args.counters[tile], 1u);
      const bool last = prev == (unsigned)(args.splits - 1);
      if (last) args.counters[tile] = 0;  // reset for the next launch on this stream
      *last_flag = last ? 1u : 0u;
    }
    __syncthreads();
    if (*last_flag) {
      __threadfence();
      // Groups of 4 consecutive elements along the partials' contiguous dimension.
      // Each thread keeps U groups x SB splits of loads in flight before consuming
      // any (the loop is load-latency bound otherwise); partials are still added in
      // split order 0..S-1.
      constexpr int U = 4, SB = 6;
      const int inner = args.ws_t ? BM : BN;
      const int outer = args.ws_t ? BN : BM;
      const int ginner = inner / 4;
      const int G = ginner * outer;
      const int64_t ld = args.ws_t ? args.M : args.N;
      const bool vec = (ld % 4) == 0;
      for (int g0 = threadIdx.x; g0 < G; g0 += U * blockDim.x) {
        int gm[U], gn[U], lim[U];
        bool full[U];
        float acc[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int g = g0 + u * blockDim.x;
          const int o = g / ginner, i4 = (g % ginner) * 4;
          gm[u] = args.ws_t ? m0 + i4 : m0 + o;
          gn[u] = args.ws_t ? n0 + o : n0 + i4;
          lim[u] = (g >= G || gm[u] >= args.M || gn[u] >= args.N) ? 0 : (args.ws_t ? args.M - gm[u] : args.N - gn[u]);
          full[u] = vec && lim[u] >= 4;
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[u][e] = 0.f;
        }
        for (int s0 = 0; s0 < args.splits; s0 += SB) {
          float4 part[SB][U];
#pragma unroll
          for (int j = 0; j < SB; ++j)
#pragma unroll
            for (int u = 0; u < U; ++u)
              if (s0 + j < args.splits && full[u])
                part[j][u] = __ldcg(reinterpret_cast<const float4*>(args.ws + ws_index(args, s0 + j, gm[u], gn[u])));
#pragma unroll
          for (int j = 0; j < SB; ++j) {
            if (s0 + j >= args.splits) break;
#pragma unroll
            for (int u = 0; u < U; ++u) {
              if (full[u]) {
                acc[u][0] += part[j][u].x;
                acc[u][1] += part[j][u].y;
                acc[u][2] += part[j][u].z;
                acc[u][3] += part[j][u].w;
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  if (e < lim[u])
                    acc[u][e] += __ldcg(args.ws + ws_index(args, s0 + j, args.ws_t ? gm[u] + e : gm[u],
                                                           args.ws_t ? gn[u] : gn[u] + e));
              }
            }
          }
        }
        float add[U][4], old[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            add[u][e] = old[u][e] = 0.f;
            if (e < lim[u])
              final_load(args, args.ws_t ? gm[u] + e : gm[u], args.ws_t ? gn[u] : gn[u] + e, add[u][e], old[u][e]);
          }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (e < lim[u])
              final_write(args, args.ws_t ? gm[u] + e : gm[u], args.ws_t ? gn[u] : gn[u] + e, acc[u][e], add[u][e],
                          old[u][e]);
      }
    }
  }
  stamp(4);
  if (args.npart) write_norm_part(args, nsum, cta_id);
}

// Persistent variant for grids with more tiles than SMs (no split-K): one CTA per SM
// walks tiles u = blockIdx.x, blockIdx.x + gridDim.x, ... The smem ring runs across
// tile boundaries (the producer loads the next tile's first k-blocks while the
// current tile finishes) and the accumulator is double-buffered in TMEM (2 x BN
// columns), so the epilogue of tile i overlaps the main loop of tile i + 1.
// Epilogue staging for TMA stores: per epilogue warp two 32 x 64 bf16 boxes (128-byte
// rows, 128B swizzle), so one box is written while the previous one is stored.
constexpr int EPI_BOX_BYTES = 32 * 128;
constexpr int EPI_STAGING = 4 * 2 * EPI_BOX_BYTES;

template <int BN>
struct PersistCfg {
  static constexpr int TMEM_COLS = 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
  static constexpr int STAGES = (227 * 1024 - 1024 - 256 - EPI_STAGING) / GemmCfg<BN>::STAGE_BYTES;
  static constexpr int SMEM = STAGES * GemmCfg<BN>::STAGE_BYTES + EPI_STAGING + 1024 + 256;
};

template <int BN, bool AMN, bool BMN>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_persistent(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                         const __grid_constant__ CUtensorMap to, GemmArgs args, int mt, int units) {
  using C = GemmCfg<BN>;
  using P = PersistCfg<BN>;
  constexpr int BK = C::BK;
  constexpr int KATOMS = BK / 64;
  constexpr int stages = P::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + stages * C::A_BYTES;
  uint8_t* sE = sB + stages * C::B_BYTES;  // epilogue staging (1024-aligned: stage sizes are)
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + EPI_STAGING);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;  // [2] accumulator buffer complete
  uint64_t* tempty = tfull + 2;      // [2] accumulator buffer drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (args.K + BK - 1) / BK;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < stages; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull[b], 1);
      sm100::mbar_init(&tempty[b], 4);  // one arrival per epilogue warp
    }
    sm100::fence_barrier_init();
    sm100::tma_prefetch_desc(&ta);
    sm100::tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, P::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  float nsum = 0.f;  // norm side output (epilogue threads)

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int m0 = (u % mt) * BM, n0 = (u / mt) * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % stages;
          if (it >= stages && !sm100::mbar_wait(&empty[s], ((it / stages) & 1) ^ 1, args.err)) {
            ok = false;
            break;
          }
          sm100::mbar_expect_tx(&full[s], C::STAGE_BYTES);
          const int k = kb * BK;
          uint8_t* a_dst = sA + s * C::A_BYTES;
          uint8_t* b_dst = sB + s * C::B_BYTES;
          if (!AMN) {
#pragma unroll
            for (int j = 0; j < KATOMS; ++j) sm100::tma_load_2d(a_dst + j * (BM * 128), &ta, &full[s], k + 64 * j, m0);
          } else {
            sm100::tma_load_2d(a_dst, &ta, &full[s], m0, k);
            sm100::tma_load_2d(a_dst + BK * 128, &ta, &full[s], m0 + 64, k);
          }
          if (!BMN) {
#pragma unroll
            for (int j = 0; j < KATOMS; ++j) sm100::tma_load_2d(b_dst + j * (BN * 128), &tb, &full[s], k + 64 * j, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) sm100::tma_load_2d(b_dst + j * (BK * 128), &tb, &full[s], n0 + 64 * j, k);
          }
        }
      }
      for (int i = max(0, it - stages); i < it; ++i) sm100::mbar_wait(&full[i % stages], (i / stages) & 1, args.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_bf16(BM, BN, AMN, BMN);
      int it = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++local) {
        const int buf = local & 1;
        if (local >= 2 && !sm100::mbar_wait(&tempty[buf], ((local >> 1) - 1) & 1, args.err)) break;
        sm100::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % stages;
          if (!sm100::mbar_wait(&full[s], (it / stages) & 1, args.err)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_u32(sA + s * C::A_BYTES);
          const uint32_t b_base = sm100::smem_u32(sB + s * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad =
                AMN ? sm100::smem_desc_sw128(a_base + kk * 2048, BK * 128, 1024)
                    : sm100::smem_desc_sw128(a_base + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024);
            const uint64_t bd =
                BMN ? sm100::smem_desc_sw128(b_base + kk * 2048, BK * 128, 1024)
                    : sm100::smem_desc_sw128(b_base + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 0, 1024);
            sm100::mma_bf16(d, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          sm100::mma_commit(&empty[s]);
        }
        if (ok) sm100::mma_commit(&tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;
    uint8_t* stg = sE + q * 2 * EPI_BOX_BYTES;
    const float nf = args.npart ? *args.nfac : 0.f;
    int local = 0, box = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
      const int buf = local & 1;
      const int m0 = (u % mt) * BM, n0 = (u / mt) * BN;
      if (!sm100::mbar_wait(&tfull[buf], (local >> 1) & 1, args.err)) break;
      sm100::tc_fence_after();
      const int m = m0 + q * 32 + lane;
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      if (args.tma_store) {
        // 64 columns per box: row `lane` of the box is this thread's accumulator row;
        // 16-byte chunk j lands at chunk j ^ (row % 8) (the 128B swizzle of the map).
#pragma unroll 1
        for (int c = 0; c < BN; c += 64, ++box) {
          if (n0 + c >= args.N) break;
          float v0[32], v1[32];
          sm100::tmem_ld32(trow + (uint32_t)c, v0);
          sm100::tmem_ld32(trow + (uint32_t)(c + 32), v1);
          uint8_t* sb = stg + (box & 1) * EPI_BOX_BYTES;
          if (lane == 0) sm100::bulk_wait_read<1>();  // the store that used `sb` has read it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float* src = j < 4 ? v0 + 8 * j : v1 + 8 * (j - 4);
            __nv_bfloat162 h[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) h[t] = __floats2bfloat162_rn(src[2 * t], src[2 * t + 1]);
            *reinterpret_cast<uint4*>(sb + lane * 128 + ((j ^ (lane & 7)) * 16)) = *reinterpret_cast<uint4*>(h);
            if (args.npart) {
              // from the stored bf16 values; rows >= M and columns >= N are exact zeros
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const float2 hv = __bfloat1622float2(h[t]);
                const float a = sm100::bf16_round(hv.x * nf), b = sm100::bf16_round(hv.y * nf);
                nsum = fmaf(a, a, fmaf(b, b, nsum));
              }
            }
          }
          sm100::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            sm100::tma_store_2d(&to, sb, n0 + c, m0 + q * 32);
            sm100::bulk_commit();
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          sm100::tmem_ld32(trow + (uint32_t)c, v);
          if (m < args.M && n0 + c < args.N) {
            store_row32(args, m, n0 + c, v);
            if (args.npart) nsum += norm_row32(args, m, n0 + c, v, nf);
          }
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&tempty[buf]);
    }
    if (args.tma_store && lane == 0) sm100::bulk_wait<0>();  // stores complete before exit
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, P::TMEM_COLS);
  }
  if (args.npart) write_norm_part(args, nsum, blockIdx.x);
}

template <int BN, bool AMN, bool BMN>
static void launch_persistent_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                                 const GemmArgs& a, int mt, int units) {
  using P = PersistCfg<BN>;
  auto kern = gemm_bf16_persistent<BN, AMN, BMN>;
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] { NS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P::SMEM)); });
  const int grid = std::min(units, num_sms());
  kern<<<grid, 192, P::SMEM, stream()>>>(ta, tb, to, a, mt, units);
  NS_CUDA(cudaGetLastError());
}

template <bool AMN, bool BMN>
static void launch_persistent(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                              const GemmArgs& a, int mt, int units) {
  switch (bn) {
    case 64: launch_persistent_bn<64, AMN, BMN>(ta, tb, to, a, mt, units); break;
    case 128: launch_persistent_bn<128, AMN, BMN>(ta, tb, to, a, mt, units); break;
    case 192: launch_persistent_bn<192, AMN, BMN>(ta, tb, to, a, mt, units); break;
    default: launch_persistent_bn<256, AMN, BMN>(ta, tb, to, a, mt, units); break;
  }
}

template <int BN, bool AMN, bool BMN>
static void launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, dim3 grid, int stages) {
  using C = GemmCfg<BN>;
  auto kern = gemm_bf16_kernel<BN, AMN, BMN>;
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_MAX));
  });
  // TMEM holds 512 columns per SM: reserve enough shared memory that no more than
  // k = 512 / TMEM_COLS CTAs co-reside (an allocation never has to wait), i.e. k+1
  // CTAs (each also pays 1 KB of reserved shared memory) must not fit in 228 KB.
  const int min_smem = (228 * 1024) / (512 / C::TMEM_COLS + 1) - 1024 + 64;
  const int ring = stages * C::STAGE_BYTES;
  const int used = (a.cluster_red ? std::max(ring, partial_bytes(BN)) : ring) + 1024 + 256;
  const int smem = std::max(used, std::min(min_smem, C::SMEM_MAX));
  if (a.cluster_red) {
    // the split CTAs of one tile form a cluster along z
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = grid.z;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NS_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, a, stages));
    return;
  }
  kern<<<grid, 192, smem, stream()>>>(ta, tb, a, stages);
  NS_CUDA(cudaGetLastError());
}

template <bool AMN, bool BMN>
static void launch(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, dim3 grid, int stages) {
  switch (bn) {
    case 64: launch_bn<64, AMN, BMN>(ta, tb, a, grid, stages); break;
    case 128: launch_bn<128, AMN, BMN>(ta, tb, a, grid, stages); break;
    case 192: launch_bn<192, AMN, BMN>(ta, tb, a, grid, stages); break;
    default: launch_bn<256, AMN, BMN>(ta, tb, a, grid, stages); break;
  }
}

static int pick_bn(int N) {
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  if (N <= 192) return 192;
  return 256;
}

static int max_stages(int bn, bool solo) {
  switch (bn) {
    case 64: return solo ? GemmCfg<64>::STAGES_SOLO : GemmCfg<64>::STAGES;
    case 128: return solo ? GemmCfg<128>::STAGES_SOLO : GemmCfg<128>::STAGES;
    case 192: return solo ? GemmCfg<192>::STAGES_SOLO : GemmCfg<192>::STAGES;
    default: return solo ? GemmCfg<256>::STAGES_SOLO : GemmCfg<256>::STAGES;
  }
}

// Per-(device, stream) arrival counters for split-K; each launch leaves them zero,
// unless a CTA gave up on a bounded wait (then `gemm_reset_counters` clears them).
static std::mutex g_counter_mu;
static std::map<std::pair<int, cudaStream_t>, std::pair<unsigned*, int>> g_counter_pool;

static unsigned* split_counters(int tiles) {
  std::lock_guard<std::mutex> lock(g_counter_mu);
  auto& pool = g_counter_pool;
  int dev;
  NS_CUDA(cudaGetDevice(&dev));
  auto key = std::make_pair(dev, stream());
  auto it = pool.find(key);
  if (it == pool.end() || it->second.second < tiles) {
    const int n = std::max(tiles, 4096);
    unsigned* p = nullptr;
    NS_CUDA(cudaMalloc(&p, n * sizeof(unsigned)));
    NS_CUDA(cudaMemsetAsync(p, 0, n * sizeof(unsigned), stream()));
    pool[key] = std::make_pair(p, n);  // an older, smaller array stays allocated (launches in flight)
    return p;
  }
  return it->second.first;
}

// Zeroes every split-K arrival counter array of the current device (all streams).
// Called after a bounded wait timed out; waits for the device first.
void gemm_reset_counters() {
  int dev;
  NS_CUDA(cudaGetDevice(&dev));
  NS_CUDA(cudaDeviceSynchronize());
  std::lock_guard<std::mutex> lock(g_counter_mu);
  for (auto& kv : g_counter_pool)
    if (kv.first.first == dev) NS_CUDA(cudaMemset(kv.second.first, 0, kv.second.second * sizeof(unsigned)));
}

static long long* g_trace = nullptr;  // test hook (gemm_trace)

// Launch plan: tile width, split count and kernel. Draft GEMMs are mostly thin
// (tens to hundreds of token rows against a weight), i.e. bandwidth-bound, so the
// plan minimises a simple time model:
//   main loop  = k-blocks per CTA x stage bytes / one CTA's streaming rate,
//   HBM        = bytes that must cross HBM / HBM bandwidth,
//   fix-up     = splits x fp32 tile / the last CTA's reduction rate,
// with one CTA per SM for split-K grids (all CTAs co-resident) and persistent CTAs
// (tiles > SMs, no split) whose epilogues overlap the next tile's main loop.
struct GemmPlan {
  int bn, bk, mt, nt, kb, splits, kpb;
  bool persistent;
};

// How many clusters of `s` split CTAs (one tile each) the GPU runs at once: clusters
// must fit inside one GPC, so for large `s` this is less than SMs / s. Queried from
// the runtime once per (kernel, cluster size, shared memory) and cached.
template <int BN, bool AMN, bool BMN>
static int max_active_clusters(int s, int smem) {
  static std::map<std::pair<int, int>, int> cache;
  const auto key = std::make_pair(s, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto kern = gemm_bf16_kernel<BN, AMN, BMN>;
  int n = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::SMEM_MAX) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, s);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();  // a failed query only means "unknown": fall back below
  if (n <= 0) n = std::max(1, num_sms() / s);
  cache[key] = n;
  return n;
}

static int max_active_clusters(int bn, bool amn, bool bmn, int s, int smem) {
#define NS_MAC(B)                                                              \
  if (bn == B) {                                                               \
    if (!amn && !bmn) return max_active_clusters<B, false, false>(s, smem);   \
    if (amn && !bmn) return max_active_clusters<B, true, false>(s, smem);     \
    if (!amn && bmn) return max_active_clusters<B, false, true>(s, smem);     \
    return max_active_clusters<B, true, true>(s, smem);                       \
  }
  NS_MAC(64)
  NS_MAC(128)
  NS_MAC(192)
  NS_MAC(256)
#undef NS_MAC
  return std::max(1, num_sms() / s);
}

// Dynamic shared memory of a split-K (solo) launch, as launch_bn computes it.
static int solo_smem(int bn, int kpb, bool cluster) {
  const int stages = std::max(1, std::min(max_stages(bn, true), kpb));
  int stage_bytes = 0, tmem_cols = 0, smem_max = 0;
  switch (bn) {
    case 64: stage_bytes = GemmCfg<64>::STAGE_BYTES; tmem_cols = GemmCfg<64>::TMEM_COLS; smem_max = GemmCfg<64>::SMEM_MAX; break;
    case 128: stage_bytes = GemmCfg<128>::STAGE_BYTES; tmem_cols = GemmCfg<128>::TMEM_COLS; smem_max = GemmCfg<128>::SMEM_MAX; break;
    case 192: stage_bytes = GemmCfg<192>::STAGE_BYTES; tmem_cols = GemmCfg<192>::TMEM_COLS; smem_max = GemmCfg<192>::SMEM_MAX; break;
    default: stage_bytes = GemmCfg<256>::STAGE_BYTES; tmem_cols = GemmCfg<256>::TMEM_COLS; smem_max = GemmCfg<256>::SMEM_MAX; break;
  }
  const int min_smem = (228 * 1024) / (512 / tmem_cols + 1) - 1024 + 64;
  const int ring = stages * stage_bytes;
  const int used = (cluster ? std::max(ring, partial_bytes(bn)) : ring) + 1024 + 256;
  return std::max(used, std::min(min_smem, smem_max));
}

static GemmPlan plan_gemm_uncached(int M, int N, int K, int force_splits, bool amn, bool bmn);

// Plans are pure functions of the problem; a training step reuses a fixed set of
// shapes, so each is planned once per process (the search costs tens of microseconds
// of host time, which matters for eagerly launched multi-rank steps).
static GemmPlan plan_gemm(int M, int N, int K, int force_splits, bool amn = false, bool bmn = false) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, bool, bool>, GemmPlan> cache;
  const auto key = std::make_tuple(M, N, K, force_splits, amn, bmn);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  const GemmPlan p = plan_gemm_uncached(M, N, K, force_splits, amn, bmn);
  cache.emplace(key, p);
  return p;
}

static GemmPlan plan_gemm_uncached(int M, int N, int K, int force_splits, bool amn, bool bmn) {
  const int sms = num_sms();
  auto base = [&](int bn) {
    GemmPlan p{};
    p.bn = bn;
    p.bk = bk_for(bn);
    p.mt = (M + BM - 1) / BM;
    p.nt = (N + bn - 1) / bn;
    p.kb = (K + p.bk - 1) / p.bk;
    return p;
  };
  auto finish = [&](GemmPlan p, int splits) {
    p.kpb = (p.kb + splits - 1) / splits;
    p.splits = (p.kb + p.kpb - 1) / p.kpb;
    p.persistent = p.splits == 1 && p.mt * p.nt > sms;
    return p;
  };
  if (force_splits > 0) return finish(base(pick_bn(N)), force_splits);
  // A split's partial tile is reduced through DSMEM by all S CTAs of the cluster
  // in parallel: about a microsecond of barriers plus one tile of DSMEM reads.
  constexpr double HBM_BW = 6.5e12, CTA_BW = 9.0e10, RED_BW = 1.5e11, RED_FIXED = 1.0e-6, FIX_BW = 3.0e10;
  const double a_bytes = 2.0 * M * K, b_bytes = 2.0 * N * K, o_bytes = 2.0 * M * N;
  GemmPlan best{};
  double best_cost = 1e30;
  for (int bn : {64, 128, 192, 256}) {
    if (bn > 64 && bn - 64 >= N) break;  // a narrower tile already covers N
    const GemmPlan p = base(bn);
    const int tiles = p.mt * p.nt;
    const double stage = (double)(BM + bn) * p.bk * 2;
    if (tiles > sms) {
      const double per_sm = std::ceil((double)tiles / sms);
      const double t_main = per_sm * p.kb * stage / CTA_BW;
      const double t_hbm = (a_bytes * p.nt + b_bytes + o_bytes) / HBM_BW;
      const double cost = std::max(t_main, t_hbm);
      if (cost < best_cost * 0.98) {
        best_cost = cost;
        best = finish(p, 1);
      }
      continue;
    }
    for (int s = 1; s <= std::min(sms / tiles, p.kb); ++s) {
      const int kpb = (p.kb + s - 1) / s;
      if ((p.kb + kpb - 1) / kpb != s) continue;  // same plan as a smaller s
      const double t_main = kpb * stage / CTA_BW;
      // up to CLUSTER_MAX splits reduce in DSMEM; beyond, the last CTA of a tile
      // reads every fp32 partial from global memory
      const bool dsmem = s <= CLUSTER_MAX;
      const double t_hbm = (a_bytes + b_bytes + o_bytes + (dsmem ? 0.0 : 8.0 * s * M * N)) / HBM_BW;
      const double t_fix = s == 1 ? 0.0
                           : dsmem ? RED_FIXED + (double)BM * bn * 4 / RED_BW
                                   : s * (double)BM * bn * 4 / FIX_BW;
      // clusters that do not all fit at once run in waves
      const int waves = (s > 1 && dsmem)
                            ? (tiles + max_active_clusters(bn, amn, bmn, s, solo_smem(bn, kpb, true)) - 1) /
                                  max_active_clusters(bn, amn, bmn, s, solo_smem(bn, kpb, true))
                            : 1;
      const double cost = std::max(waves * t_main, t_hbm) + waves * t_fix;
      if (cost < best_cost * 0.98) {
        best_cost = cost;
        best = finish(p, s);
      }
    }
  }
  return best;
}

// D[M,N] = A * B^T with the epilogue `e`.
int gemm_launch(const Operand& A, const Operand& B, int M, int N, int K, const Epilogue& e, int force_splits) {
  NS_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  if (e.npart) {
    NS_CHECK(e.nfac && e.out && !e.out_f32 && !e.res && !e.accumulate,
             "the norm side output needs a plain bf16 output");
    if (force_splits == 0) force_splits = 1;  // one CTA stores each element
  }
  const GemmPlan plan = plan_gemm(M, N, K, force_splits, A.mn_major, B.mn_major);
  const int bn = plan.bn, bk = plan.bk, mt = plan.mt, nt = plan.nt;
  const int tiles = mt * nt;
  const int splits = plan.splits, kpb = plan.kpb;
  CUtensorMap ta = A.mn_major ? make_tmap_bf16(A.ptr, A.rows, A.cols, A.ld, bk, 64)
                              : make_tmap_bf16(A.ptr, A.rows, A.cols, A.ld, BM, 64);
  CUtensorMap tb = B.mn_major ? make_tmap_bf16(B.ptr, B.rows, B.cols, B.ld, bk, 64)
                              : make_tmap_bf16(B.ptr, B.rows, B.cols, B.ld, bn, 64);
  const bool solo = (int64_t)tiles * splits <= num_sms();
  const int stages = std::max(1, std::min(max_stages(bn, solo), kpb));

  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.kpb = kpb;
  a.splits = splits;
  a.out = e.out;
  a.out_f32 = e.out_f32;
  a.out_sm = e.sm;
  a.out_sn = e.sn;
  a.res = e.res;
  a.res_sm = e.rsm;
  a.res_sn = e.rsn;
  a.accumulate = e.accumulate ? 1 : 0;
  a.err = device_error_flag();
  a.trace = g_trace;
  a.ws_t = (e.sn != 1) ? 1 : 0;
  a.nfac = e.nfac;
  a.npart = e.npart;
  // split-K reduces in DSMEM within a cluster; a count above the portable cluster
  // size uses fp32 partials in global memory and a last-CTA fix-up
  a.cluster_red = (splits > 1 && splits <= CLUSTER_MAX && !g_trace) ? 1 : 0;
  at::Tensor ws;
  if (splits > 1 && !a.cluster_red) {
    ws = at::empty({(int64_t)splits * M * N}, at::TensorOptions().dtype(at::kFloat).device(at::kCUDA));
    a.ws = ws.data_ptr<float>();
    a.counters = split_counters(tiles);
  }
  if (plan.persistent && !g_trace) {
    // More tiles than SMs: persistent CTAs with a cross-tile ring and overlapped epilogues.
    // A plain row-major bf16 output (16-byte aligned rows) leaves through TMA stores.
    CUtensorMap to = ta;  // placeholder when unused
    a.tma_store = (e.out && !e.out_f32 && e.sn == 1 && !e.res && !e.accumulate && e.sm % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(e.out) % 16 == 0) ? 1 : 0;
    if (a.tma_store) to = make_tmap_bf16(e.out, M, N, e.sm, 32, 64);
    if (!A.mn_major && !B.mn_major) launch_persistent<false, false>(bn, ta, tb, to, a, mt, tiles);
    else if (A.mn_major && !B.mn_major) launch_persistent<true, false>(bn, ta, tb, to, a, mt, tiles);
    else if (!A.mn_major && B.mn_major) launch_persistent<false, true>(bn, ta, tb, to, a, mt, tiles);
    else launch_persistent<true, true>(bn, ta, tb, to, a, mt, tiles);
    return std::min(tiles, num_sms());
  }
  dim3 grid(mt, nt, splits);
  if (!A.mn_major && !B.mn_major) launch<false, false>(bn, ta, tb, a, grid, stages);
  else if (A.mn_major && !B.mn_major) launch<true, false>(bn, ta, tb, a, grid, stages);
  else if (!A.mn_major && B.mn_major) launch<false, true>(bn, ta, tb, a, grid, stages);
  else launch<true, true>(bn, ta, tb, a, grid, stages);
  return tiles * splits;
}

// ----------------------------------------------------------------------------- torch API
static void check_rowmajor(const at::Tensor& t, const char* name) {
  check_bf16(t, name);
  NS_CHECK(t.dim() == 2 && t.stride(1) == 1, std::string(name) + " must be 2-D with unit column stride");
}

// y[T, Nout] = x[T, K] @ w[Nout, K]^T (+ residual)
void linear(at::Tensor x, at::Tensor w, at::Tensor out, c10::optional<at::Tensor> residual) {
  check_rowmajor(x, "x");
  check_rowmajor(w, "w");
  check_rowmajor(out, "out");
  const int T = x.size(0), K = x.size(1), Nout = w.size(0);
  NS_CHECK(w.size(1) == K && out.size(0) == T && out.size(1) == Nout, "linear: shape mismatch");
  const __nv_bfloat16* res = nullptr;
  int64_t rs0 = 0;
  if (residual && residual->defined()) {
    check_rowmajor(*residual, "residual");
    res = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    rs0 = residual->stride(0);
  }
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  Operand X{x.data_ptr(), T, K, x.stride(0), false};
  Operand W{w.data_ptr(), Nout, K, w.stride(0), false};
  if (T <= 256) {
    // swap-AB: weight rows on the 128-wide M side, tokens on N; output transposed.
    gemm_launch(W, X, Nout, T, K, Epilogue{o, nullptr, 1, out.stride(0), res, 1, rs0, false});
  } else {
    gemm_launch(X, W, T, Nout, K, Epilogue{o, nullptr, out.stride(0), 1, res, rs0, 1, false});
  }
}

// dx[T, K] (+)= dy[T, Nout] @ w[Nout, K]
void linear_dgrad(at::Tensor dy, at::Tensor w, at::Tensor out, bool accumulate) {
  check_rowmajor(dy, "dy");
  check_rowmajor(w, "w");
  check_rowmajor(out, "out");
  const int T = dy.size(0), Nout = dy.size(1), K = w.size(1);
  NS_CHECK(w.size(0) == Nout && out.size(0) == T && out.size(1) == K, "linear_dgrad: shape mismatch");
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (T <= 256) {
    Operand A{w.data_ptr(), Nout, K, w.stride(0), true};    // A[m=k, r=nout] = w[nout, k]
    Operand B{dy.data_ptr(), T, Nout, dy.stride(0), false};  // B[n=t, r=nout]
    gemm_launch(A, B, K, T, Nout, Epilogue{o, nullptr, 1, out.stride(0), nullptr, 0, 0, accumulate});
  } else {
    Operand A{dy.data_ptr(), T, Nout, dy.stride(0), false};
    Operand B{w.data_ptr(), Nout, K, w.stride(0), true};     // B[n=k, r=nout] = w[nout, k]
    gemm_launch(A, B, T, K, Nout, Epilogue{o, nullptr, out.stride(0), 1, nullptr, 0, 0, accumulate});
  }
}

// dW[Nout, K] (+)= dy[T, Nout]^T @ x[T, K]. With `nfac`/`npart` (plain output only),
// also writes this launch's per-CTA partials of sum bf16(dW * nfac)^2 to
// npart[offset, offset + returned count).
int64_t linear_wgrad(at::Tensor dy, at::Tensor x, at::Tensor out, bool accumulate, c10::optional<at::Tensor> nfac,
                     c10::optional<at::Tensor> npart, int64_t offset) {
  check_rowmajor(dy, "dy");
  check_rowmajor(x, "x");
  check_bf16(out, "out");
  NS_CHECK(out.is_contiguous() || (out.dim() == 2 && out.stride(1) == 1), "out must be row-major");
  const int T = dy.size(0), Nout = dy.size(1), K = x.size(1);
  NS_CHECK(x.size(0) == T && out.numel() == (int64_t)Nout * K, "linear_wgrad: shape mismatch");
  const int64_t ld = out.dim() == 2 ? out.stride(0) : K;
  Operand A{dy.data_ptr(), T, Nout, dy.stride(0), true};  // A[m=nout, r=t] = dy[t, nout]
  Operand B{x.data_ptr(), T, K, x.stride(0), true};       // B[n=k, r=t] = x[t, k]
  Epilogue e{reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nullptr, ld, 1, nullptr, 0, 0, accumulate};
  if (npart && npart->defined()) {
    NS_CHECK(nfac && nfac->defined() && nfac->scalar_type() == at::kFloat && npart->scalar_type() == at::kFloat,
             "linear_wgrad: fp32 norm factor and partial buffer expected");
    NS_CHECK(offset >= 0 && offset + num_sms() <= npart->numel(), "linear_wgrad: norm partial buffer full");
    e.nfac = nfac->data_ptr<float>();
    e.npart = npart->data_ptr<float>() + offset;
  }
  return gemm_launch(A, B, Nout, K, T, e);
}

// Test hook: record clock64 stamps (TMA issue [0,256), MMA start [256,512)) of CTA 0
// and per-CTA globaltimer phase stamps [512 + phase * 2048 + cta].
void gemm_trace(c10::optional<at::Tensor> buf) {
  g_trace = (buf && buf->defined()) ? reinterpret_cast<long long*>(buf->data_ptr<int64_t>()) : nullptr;
}

// Test hook: plain D = A * B^T with explicit operand majors and a forced split count.
void gemm_test(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, at::Tensor out, int splits) {
  check_rowmajor(a, "a");
  check_rowmajor(b, "b");
  check_rowmajor(out, "out");
  const int M = out.size(0), N = out.size(1);
  const int K = a_mn ? a.size(0) : a.size(1);
  Operand A{a.data_ptr(), a.size(0), a.size(1), a.stride(0), a_mn};
  Operand B{b.data_ptr(), b.size(0), b.size(1), b.stride(0), b_mn};
  gemm_launch(A, B, M, N, K,
              Epilogue{reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nullptr, out.stride(0), 1, nullptr, 0, 0, false},
              splits);
}

}  // namespace ns

// ----------------------------------------------------------------------------- allocation-free entry
// The C ABI and its contract (limits, zero state, concurrency) are declared in
// gemm_noalloc.h. Everything below is new code beside the torch path above: the
// kernel is the same, only its scratch comes from this file-scope array.
namespace ns {

static __device__ __align__(256) unsigned char g_noalloc_scratch[NSB_GEMM_NOALLOC_SCRATCH_BYTES];

constexpr size_t kNoallocCountersOff = 0;
constexpr size_t kNoallocStatusOff = 4u * NSB_GEMM_NOALLOC_MAX_TILES;
constexpr size_t kNoallocPartialsOff = kNoallocStatusOff + 256;
static_assert(kNoallocPartialsOff % 256 == 0, "partials must stay 256-byte aligned");
static_assert(kNoallocPartialsOff + 4ull * NSB_GEMM_NOALLOC_PARTIAL_FLOATS <= NSB_GEMM_NOALLOC_SCRATCH_BYTES,
              "partial area exceeds the scratch array");

constexpr int kNoallocMaxDevices = 64;
static std::mutex g_noalloc_mu;
// Written once per device under g_noalloc_mu (release); read without the lock (acquire).
static std::atomic<unsigned char*> g_noalloc_base[kNoallocMaxDevices] = {};
static thread_local char g_noalloc_msg[256] = "";

static int noalloc_fail(int code, const char* what, cudaError_t e = cudaSuccess) {
  if (e != cudaSuccess) std::snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "%s: %s", what, cudaGetErrorString(e));
  else std::snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "%s", what);
  return code;
}

template <int BN, bool AMN, bool BMN>
static cudaError_t noalloc_set_attr() {
  return cudaFuncSetAttribute(gemm_bf16_kernel<BN, AMN, BMN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              GemmCfg<BN>::SMEM_MAX);
}

template <int BN>
static cudaError_t noalloc_set_attr_bn() {
  cudaError_t e;
  if ((e = noalloc_set_attr<BN, false, false>()) != cudaSuccess) return e;
  if ((e = noalloc_set_attr<BN, true, false>()) != cudaSuccess) return e;
  if ((e = noalloc_set_attr<BN, false, true>()) != cudaSuccess) return e;
  return noalloc_set_attr<BN, true, true>();
}

// Once per device, with that device current: resolve the scratch address and raise
// the kernels' shared-memory limit.
static int noalloc_setup_current(int dev) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_base[dev].load(std::memory_order_acquire)) return 0;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return noalloc_fail(3, "cudaGetSymbolAddress(scratch)", e);
  if ((e = noalloc_set_attr_bn<64>()) != cudaSuccess || (e = noalloc_set_attr_bn<128>()) != cudaSuccess ||
      (e = noalloc_set_attr_bn<192>()) != cudaSuccess || (e = noalloc_set_attr_bn<256>()) != cudaSuccess)
    return noalloc_fail(3, "cudaFuncSetAttribute", e);
  g_noalloc_base[dev].store(static_cast<unsigned char*>(p), std::memory_order_release);
  return 0;
}

template <int BN, bool AMN, bool BMN>
static cudaError_t noalloc_launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, dim3 grid,
                                     int stages, cudaStream_t st) {
  using Cfg = GemmCfg<BN>;
  // Same shared-memory reservation as the torch path (TMEM co-residency clamp).
  const int min_smem = (228 * 1024) / (512 / Cfg::TMEM_COLS + 1) - 1024 + 64;
  const int smem = std::max(stages * Cfg::STAGE_BYTES + 1024 + 256, std::min(min_smem, Cfg::SMEM_MAX));
  gemm_bf16_kernel<BN, AMN, BMN><<<grid, 192, smem, st>>>(ta, tb, a, stages);
  return cudaGetLastError();
}

template <bool AMN, bool BMN>
static cudaError_t noalloc_launch(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                                  dim3 grid, int stages, cudaStream_t st) {
  switch (bn) {
    case 64: return noalloc_launch_bn<64, AMN, BMN>(ta, tb, a, grid, stages, st);
    case 128: return noalloc_launch_bn<128, AMN, BMN>(ta, tb, a, grid, stages, st);
    case 192: return noalloc_launch_bn<192, AMN, BMN>(ta, tb, a, grid, stages, st);
    default: return noalloc_launch_bn<256, AMN, BMN>(ta, tb, a, grid, stages, st);
  }
}

static int noalloc_current(int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(3, "cudaGetDevice", e);
  if (dev < 0 || dev >= kNoallocMaxDevices) return noalloc_fail(1, "device ordinal out of range");
  *dev_out = dev;
  return 0;
}

}  // namespace ns

extern "C" int nsb_gemm_noalloc_setup(int device) {
  using namespace ns;
  g_noalloc_msg[0] = 0;
  if (device < 0 || device >= kNoallocMaxDevices) return noalloc_fail(1, "device ordinal out of range");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return noalloc_fail(3, "cudaGetDevice", e);
  if ((e = cudaSetDevice(device)) != cudaSuccess) return noalloc_fail(3, "cudaSetDevice", e);
  const int rc = noalloc_setup_current(device);
  cudaSetDevice(prev);
  return rc;
}

extern "C" int nsb_gemm_bf16_splitk_noalloc(const void* a, int a_mn_major, long long a_rows, long long a_cols,
                                            long long a_ld, const void* b, int b_mn_major, long long b_rows,
                                            long long b_cols, long long b_ld, void* out, long long out_ld, int M,
                                            int N, int K, int splits, void* stream) {
  using namespace ns;
  g_noalloc_msg[0] = 0;
  if (!a || !b || !out) return noalloc_fail(1, "null operand pointer");
  if (M <= 0 || N <= 0 || K <= 0) return noalloc_fail(1, "M, N and K must be positive");
  if (splits < 1 || splits > 16) return noalloc_fail(1, "splits must be in [1, 16]");
  if ((a_mn_major ? a_rows != K || a_cols != M : a_rows != M || a_cols != K) ||
      (b_mn_major ? b_rows != K || b_cols != N : b_rows != N || b_cols != K))
    return noalloc_fail(1, "operand shapes do not match M, N, K and their majors");
  if (a_ld < a_cols || b_ld < b_cols) return noalloc_fail(1, "row stride smaller than row length");
  if (out_ld < N || (reinterpret_cast<uintptr_t>(out) % 16) != 0)
    return noalloc_fail(1, "out must be 16-byte aligned with a row stride >= N");
  int dev = 0;
  if (int rc = noalloc_current(&dev)) return rc;
  if (!g_noalloc_base[dev].load(std::memory_order_acquire))
    if (int rc = noalloc_setup_current(dev)) return rc;

  const int bn = pick_bn(N);
  const int bk = bk_for(bn);
  const int mt = (M + BM - 1) / BM, nt = (N + bn - 1) / bn;
  const int kb = (K + bk - 1) / bk;
  const int tiles = mt * nt;
  const int kpb = (kb + splits - 1) / splits;
  const int eff_splits = (kb + kpb - 1) / kpb;  // same split plan as the torch path
  if (eff_splits > 1 && (unsigned)tiles > NSB_GEMM_NOALLOC_MAX_TILES) {  // only split launches use counters
    std::snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "%d output tiles exceed the maximum of %u", tiles,
                  NSB_GEMM_NOALLOC_MAX_TILES);
    return 2;
  }
  if (eff_splits > 1 && (unsigned long long)eff_splits * M * N > NSB_GEMM_NOALLOC_PARTIAL_FLOATS) {
    std::snprintf(g_noalloc_msg, sizeof(g_noalloc_msg),
                  "split-K partials need %llu floats; the scratch holds at most %u (splits * M * N)",
                  (unsigned long long)eff_splits * M * N, NSB_GEMM_NOALLOC_PARTIAL_FLOATS);
    return 2;
  }
  CUtensorMap ta, tb;
  int sms = 0;
  try {
    ta = a_mn_major ? make_tmap_bf16(a, a_rows, a_cols, a_ld, bk, 64) : make_tmap_bf16(a, a_rows, a_cols, a_ld, BM, 64);
    tb = b_mn_major ? make_tmap_bf16(b, b_rows, b_cols, b_ld, bk, 64) : make_tmap_bf16(b, b_rows, b_cols, b_ld, bn, 64);
    sms = num_sms();
  } catch (const std::exception& ex) {
    return noalloc_fail(1, ex.what());
  }
  const bool solo = (long long)tiles * eff_splits <= sms;
  const int stages = std::max(1, std::min(max_stages(bn, solo), kpb));

  unsigned char* base = g_noalloc_base[dev].load(std::memory_order_acquire);
  GemmArgs ga{};
  ga.M = M;
  ga.N = N;
  ga.K = K;
  ga.kpb = kpb;
  ga.splits = eff_splits;
  ga.out = static_cast<__nv_bfloat16*>(out);
  ga.out_sm = out_ld;
  ga.out_sn = 1;
  ga.ws = reinterpret_cast<float*>(base + kNoallocPartialsOff);
  ga.ws_t = 0;
  ga.counters = reinterpret_cast<unsigned*>(base + kNoallocCountersOff);
  ga.err = reinterpret_cast<int*>(base + kNoallocStatusOff);
  ga.trace = nullptr;
  const dim3 grid(mt, nt, eff_splits);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (!a_mn_major && !b_mn_major) e = noalloc_launch<false, false>(bn, ta, tb, ga, grid, stages, st);
  else if (a_mn_major && !b_mn_major) e = noalloc_launch<true, false>(bn, ta, tb, ga, grid, stages, st);
  else if (!a_mn_major && b_mn_major) e = noalloc_launch<false, true>(bn, ta, tb, ga, grid, stages, st);
  else e = noalloc_launch<true, true>(bn, ta, tb, ga, grid, stages, st);
  if (e != cudaSuccess) return noalloc_fail(3, "kernel launch", e);
  return 0;
}

extern "C" int nsb_gemm_noalloc_status(int* status) {
  using namespace ns;
  g_noalloc_msg[0] = 0;
  if (!status) return noalloc_fail(1, "null status pointer");
  int dev = 0;
  if (int rc = noalloc_current(&dev)) return rc;
  if (!g_noalloc_base[dev].load(std::memory_order_acquire))
    if (int rc = noalloc_setup_current(dev)) return rc;
  cudaError_t e = cudaMemcpy(status, g_noalloc_base[dev].load(std::memory_order_acquire) + kNoallocStatusOff, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return noalloc_fail(3, "cudaMemcpy(status)", e);
  return 0;
}

extern "C" int nsb_gemm_noalloc_reset(void* stream) {
  using namespace ns;
  g_noalloc_msg[0] = 0;
  int dev = 0;
  if (int rc = noalloc_current(&dev)) return rc;
  if (!g_noalloc_base[dev].load(std::memory_order_acquire))
    if (int rc = noalloc_setup_current(dev)) return rc;
  cudaError_t e = cudaMemsetAsync(g_noalloc_base[dev].load(std::memory_order_acquire), 0, kNoallocPartialsOff, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return noalloc_fail(3, "cudaMemsetAsync(counters)", e);
  return 0;
}

extern "C" const char* nsb_gemm_noalloc_error(void) { return ns::g_noalloc_msg; }
