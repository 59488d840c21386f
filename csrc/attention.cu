// Draft attention with the anchor layout (no dense mask, no stored probabilities).
//
// Query block j of batch row i (block_size queries per head) sees the context keys
// [0, anchors[i, j]) and its own block's draft keys; a block with keep == false sees
// nothing and outputs zeros (lse = -inf). Keys/values are in split layout: row
// i*S + t for context token t, row b*S + i*Td + u for draft token u; rows may be
// strided (K and V live in one [rows, 2*Hk*D] projection output).
// Reference semantics: the flex-attention mask of nanospec/dspark.py (anchor prefix +
// own block), evaluated here without a mask tensor.
//
// The problem is small (a few hundred query rows per head, at most S + block_size
// keys each), so the kernels are organised for parallelism and few memory round
// trips rather than tensor-core throughput:
//   forward : one CTA per (block j, query head, batch row); key tiles of 64 keys
//             are fetched with 16-byte loads into shared memory; scores (thread per
//             key), online softmax (warp per row) and P V (thread per column pair)
//             run in fp32.
//   backward: dq  - the same decomposition (P recomputed from lse); it also stores
//                   delta = rowsum(dO * O) for the dkv kernel;
//             dkv - one CTA per (key tile, KV head, batch row): one tile per draft
//                   block, and 16-key context tiles split further by GQA head (each
//                   head's CTA writes fp32 partials, summed in head order). A CTA
//                   walks the query blocks that see its tile and accumulates dK, dV
//                   in registers in a fixed order: deterministic, no atomics.
#include <cstdlib>
#include <string>

#include "common.h"
#include "sm100.cuh"

namespace ns {

using bf16 = __nv_bfloat16;

struct AttnArgs {
  const bf16 *q, *k, *v, *o, *dout;
  int64_t ldk, ldv;                 // key/value row strides (elements)
  const int64_t* anchors;           // [b, nb]
  const bool* keep;                 // [b, nb]
  float* lse;                       // [b, Hq, Td]
  float* delta;                     // [b, Hq, Td] rowsum(dO * O), written by dq, read by dkv
  float* part;                      // [2][G][b*S][Hk][D] fp32 per-head dK / dV of the context keys
  bf16 *out, *dq, *dk, *dv;
  int64_t lddk, lddv;
  int b, S, nb, bs, Hq, Hk;
  float scale;
};

constexpr int NT = 128;    // threads of the forward / dq CTAs
constexpr int KT = 64;     // keys per tile (forward / dq)
constexpr int RMAX = 32;   // largest block_size (query rows per CTA); kernels take RM in {8, 16, 32}

__device__ __forceinline__ int64_t key_row(const AttnArgs& a, int bi, int kv) {
  // kv in [0, S) context, [S, S+Td) draft
  return kv < a.S ? (int64_t)bi * a.S + kv : (int64_t)a.b * a.S + (int64_t)bi * a.nb * a.bs + (kv - a.S);
}

// Tile t of block j: context tiles cover [0, anchor) in KT steps, then one tile with
// the block's own bs draft keys.
__device__ __forceinline__ void tile_keys(int t, int anchor, int S, int j, int bs, int& k0, int& cnt) {
  const int nctx = (anchor + KT - 1) / KT;
  if (t < nctx) {
    k0 = t * KT;
    cnt = min(KT, anchor - k0);
  } else {
    k0 = S + j * bs;
    cnt = bs;
  }
}

__device__ __forceinline__ float2 bf2f(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}

// K/V tile staging: `fetch` issues every 16-byte global load of a tile into
// registers (ROWS keys x D of head hk, rows >= cnt zero), `store` writes them into
// shared memory rows of KP bf16. Splitting the two lets a CTA fetch tile t + 1 while
// it computes on tile t. KP = D + 2 (an odd number of 32-bit words) keeps per-key
// reads free of bank conflicts.
template <int D, int ROWS, int NTH>
struct KVRegs {
  static constexpr int C = D / 8;  // 16-byte chunks per row
  static constexpr int IT = (ROWS * C + NTH - 1) / NTH;
  uint4 k[IT], v[IT];
};

template <int D, int ROWS, int NTH>
__device__ __forceinline__ void fetch_kv(const AttnArgs& a, int bi, int hk, int k0, int cnt,
                                         KVRegs<D, ROWS, NTH>& r, int tid) {
  using R = KVRegs<D, ROWS, NTH>;
#pragma unroll
  for (int i = 0; i < R::IT; ++i) {
    const int c = tid + i * NTH;
    const int kk = c / R::C, d8 = (c % R::C) * 8;
    r.k[i] = r.v[i] = make_uint4(0, 0, 0, 0);
    if (c < ROWS * R::C && kk < cnt) {
      const int64_t row = key_row(a, bi, k0 + kk);
      r.k[i] = *reinterpret_cast<const uint4*>(a.k + row * a.ldk + hk * D + d8);
      r.v[i] = *reinterpret_cast<const uint4*>(a.v + row * a.ldv + hk * D + d8);
    }
  }
}

template <int D, int KP, int ROWS, int NTH>
__device__ __forceinline__ void store_kv(const KVRegs<D, ROWS, NTH>& r, bf16* Ks, bf16* Vs, int tid) {
  using R = KVRegs<D, ROWS, NTH>;
#pragma unroll
  for (int i = 0; i < R::IT; ++i) {
    const int c = tid + i * NTH;
    if (c < ROWS * R::C) {
      const int kk = c / R::C, d8 = (c % R::C) * 8;
      uint32_t* kd = reinterpret_cast<uint32_t*>(Ks + kk * KP + d8);
      uint32_t* vd = reinterpret_cast<uint32_t*>(Vs + kk * KP + d8);
      kd[0] = r.k[i].x;
      kd[1] = r.k[i].y;
      kd[2] = r.k[i].z;
      kd[3] = r.k[i].w;
      vd[0] = r.v[i].x;
      vd[1] = r.v[i].y;
      vd[2] = r.v[i].z;
      vd[3] = r.v[i].w;
    }
  }
}

// Rows r of block j / head h -> token offset into q/out/dout ([b, Td, Hq, D]).
__device__ __forceinline__ int64_t qoff(const AttnArgs& a, int bi, int j, int u, int h, int D) {
  const int Td = a.nb * a.bs;
  return ((int64_t)(bi * Td + j * a.bs + u) * a.Hq + h) * D;
}

// ---------------------------------------------------------------------------- forward
template <int D, int RM>
__global__ void __launch_bounds__(NT) attn_fwd_kernel(AttnArgs a) {
  constexpr int KP = D + 2;
  constexpr int NP = D / 2;                       // column pairs
  constexpr int NG = NT / NP > 0 ? NT / NP : 1;   // row groups in the P V phase
  constexpr int RPT = (RM + NG - 1) / NG;       // rows per thread in the P V phase
  constexpr int SG = NT / KT;                     // row groups in the score phase
  constexpr int RS = RM / SG;                   // rows per thread in the score phase
  extern __shared__ __align__(16) uint8_t dyn[];
  bf16* Ks = reinterpret_cast<bf16*>(dyn);             // [KT][KP]
  bf16* Vs = Ks + KT * KP;                             // [KT][KP]
  float* Qs = reinterpret_cast<float*>(Vs + KT * KP);  // [RM][D] q * scale
  float* Ps = Qs + RM * D;                           // [RM][KT]
  float* mrow = Ps + RM * KT;
  float* lrow = mrow + RM;
  float* corr = lrow + RM;
  const int j = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int hk = h / (a.Hq / a.Hk);
  const int R = a.bs, Td = a.nb * a.bs;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool kp = a.keep[bi * a.nb + j];
  const int anchor = kp ? (int)a.anchors[bi * a.nb + j] : 0;
  const int ntiles = kp ? (anchor + KT - 1) / KT + 1 : 0;

  for (int c = tid; c < R * (D / 8); c += NT) {
    const int r = c / (D / 8), d8 = (c % (D / 8)) * 8;
    const uint4 u = *reinterpret_cast<const uint4*>(a.q + qoff(a, bi, j, r, h, D) + d8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 f = bf2f(w[t]);
      Qs[r * D + d8 + 2 * t] = f.x * a.scale;
      Qs[r * D + d8 + 2 * t + 1] = f.y * a.scale;
    }
  }
  if (tid < RM) {
    mrow[tid] = -INFINITY;
    lrow[tid] = 0.f;
  }
  const int dp = tid % NP, rg = tid / NP;  // P V phase: column pair, row group
  float acc[RPT][2];
#pragma unroll
  for (int i = 0; i < RPT; ++i) acc[i][0] = acc[i][1] = 0.f;
  const int sk = tid % KT, sg = tid / KT;  // score phase: key, row group

  KVRegs<D, KT, NT> kvr;
  if (ntiles > 0) {
    int k0, cnt;
    tile_keys(0, anchor, a.S, j, a.bs, k0, cnt);
    fetch_kv(a, bi, hk, k0, cnt, kvr, tid);
  }
  for (int tile = 0; tile < ntiles; ++tile) {
    int k0, cnt;
    tile_keys(tile, anchor, a.S, j, a.bs, k0, cnt);
    __syncthreads();
    store_kv<D, KP>(kvr, Ks, Vs, tid);
    __syncthreads();
    if (tile + 1 < ntiles) {  // next tile's loads stay in flight during this tile's math
      int k1, c1;
      tile_keys(tile + 1, anchor, a.S, j, a.bs, k1, c1);
      fetch_kv(a, bi, hk, k1, c1, kvr, tid);
    }
    // scores s[r][k] = q_r . k_k
    float s[RS];
#pragma unroll
    for (int i = 0; i < RS; ++i) s[i] = 0.f;
    const uint32_t* kr = reinterpret_cast<const uint32_t*>(Ks + sk * KP);
#pragma unroll 4
    for (int p = 0; p < NP; ++p) {
      const float2 kf = bf2f(kr[p]);
#pragma unroll
      for (int i = 0; i < RS; ++i) {
        const int r = sg + SG * i;
        if (r >= R) break;
        const float2 qf = *reinterpret_cast<const float2*>(Qs + r * D + 2 * p);
        s[i] = fmaf(qf.x, kf.x, fmaf(qf.y, kf.y, s[i]));
      }
    }
#pragma unroll
    for (int i = 0; i < RS; ++i) {
      const int r = sg + SG * i;
      if (r < R) Ps[r * KT + sk] = sk < cnt ? s[i] : -INFINITY;
    }
    __syncthreads();
    // online softmax, one warp per row
    for (int r = warp; r < R; r += NT / 32) {
      const float v0 = Ps[r * KT + lane], v1 = Ps[r * KT + lane + 32];
      float tm = fmaxf(v0, v1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffff, tm, o));
      const float mo = mrow[r];
      const float mn = fmaxf(mo, tm);
      float p0 = 0.f, p1 = 0.f, c = 1.f;
      if (mn > -INFINITY) {
        p0 = expf(v0 - mn);
        p1 = expf(v1 - mn);
        c = mo > -INFINITY ? expf(mo - mn) : 0.f;
      }
      float sum = p0 + p1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffff, sum, o);
      Ps[r * KT + lane] = p0;
      Ps[r * KT + lane + 32] = p1;
      __syncwarp();
      if (lane == 0) {
        lrow[r] = lrow[r] * c + sum;
        mrow[r] = mn;
        corr[r] = c;
      }
    }
    __syncthreads();
    // acc[r][d] = acc * corr + sum_k p[r][k] v[k][d]
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg + NG * i;
      if (r < R) {
        acc[i][0] *= corr[r];
        acc[i][1] *= corr[r];
      }
    }
    if (dp < NP) {
      for (int kk = 0; kk < cnt; ++kk) {
        const float2 vf = bf2f(reinterpret_cast<const uint32_t*>(Vs + kk * KP)[dp]);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const int r = rg + NG * i;
          if (r >= R) break;
          const float p = Ps[r * KT + kk];
          acc[i][0] = fmaf(p, vf.x, acc[i][0]);
          acc[i][1] = fmaf(p, vf.y, acc[i][1]);
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg + NG * i;
    if (r < R && dp < NP) {
      const float l = lrow[r];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      *reinterpret_cast<__nv_bfloat162*>(a.out + qoff(a, bi, j, r, h, D) + 2 * dp) =
          __floats2bfloat162_rn(acc[i][0] * inv, acc[i][1] * inv);
    }
  }
  if (tid < R) {
    const float l = lrow[tid];
    a.lse[((int64_t)bi * a.Hq + h) * Td + j * a.bs + tid] = l > 0.f ? mrow[tid] + logf(l) : -INFINITY;
  }
}

// ---------------------------------------------------------------------------- backward dq
template <int D, int RM>
__global__ void __launch_bounds__(NT) attn_bwd_dq_kernel(AttnArgs a) {
  constexpr int KP = D + 2;
  constexpr int NP = D / 2;
  constexpr int NG = NT / NP > 0 ? NT / NP : 1;
  constexpr int RPT = (RM + NG - 1) / NG;
  constexpr int SG = NT / KT;
  constexpr int RS = RM / SG;
  extern __shared__ __align__(16) uint8_t dyn[];
  bf16* Ks = reinterpret_cast<bf16*>(dyn);             // [KT][KP]
  bf16* Vs = Ks + KT * KP;                             // [KT][KP]
  float* Qs = reinterpret_cast<float*>(Vs + KT * KP);  // [RM][D] q * scale
  float* Os = Qs + RM * D;                           // [RM][D] dO
  float* Ps = Os + RM * D;                           // [RM][KT] dS
  float* lse_s = Ps + RM * KT;
  float* delta_s = lse_s + RM;
  const int j = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int hk = h / (a.Hq / a.Hk);
  const int R = a.bs, Td = a.nb * a.bs;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool kp = a.keep[bi * a.nb + j];
  const int anchor = kp ? (int)a.anchors[bi * a.nb + j] : 0;
  const int ntiles = kp ? (anchor + KT - 1) / KT + 1 : 0;

  for (int c = tid; c < R * (D / 8); c += NT) {
    const int r = c / (D / 8), d8 = (c % (D / 8)) * 8;
    const int64_t off = qoff(a, bi, j, r, h, D) + d8;
    const uint4 uq = *reinterpret_cast<const uint4*>(a.q + off);
    const uint4 uo = *reinterpret_cast<const uint4*>(a.dout + off);
    const uint32_t wq[4] = {uq.x, uq.y, uq.z, uq.w}, wo[4] = {uo.x, uo.y, uo.z, uo.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 fq = bf2f(wq[t]), fo = bf2f(wo[t]);
      Qs[r * D + d8 + 2 * t] = fq.x * a.scale;
      Qs[r * D + d8 + 2 * t + 1] = fq.y * a.scale;
      Os[r * D + d8 + 2 * t] = fo.x;
      Os[r * D + d8 + 2 * t + 1] = fo.y;
    }
  }
  __syncthreads();
  for (int r = warp; r < R; r += NT / 32) {
    const int64_t off = qoff(a, bi, j, r, h, D);
    float dl = 0.f;
    for (int d = lane; d < D; d += 32) dl += Os[r * D + d] * __bfloat162float(a.o[off + d]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dl += __shfl_xor_sync(0xffffffff, dl, o);
    if (lane == 0) {
      const int64_t ri = ((int64_t)bi * a.Hq + h) * Td + j * a.bs + r;
      delta_s[r] = dl;
      a.delta[ri] = dl;
      lse_s[r] = a.lse[ri];
    }
  }
  const int dp = tid % NP, rg = tid / NP;
  float acc[RPT][2];
#pragma unroll
  for (int i = 0; i < RPT; ++i) acc[i][0] = acc[i][1] = 0.f;
  const int sk = tid % KT, sg = tid / KT;

  KVRegs<D, KT, NT> kvr;
  if (ntiles > 0) {
    int k0, cnt;
    tile_keys(0, anchor, a.S, j, a.bs, k0, cnt);
    fetch_kv(a, bi, hk, k0, cnt, kvr, tid);
  }
  for (int tile = 0; tile < ntiles; ++tile) {
    int k0, cnt;
    tile_keys(tile, anchor, a.S, j, a.bs, k0, cnt);
    __syncthreads();
    store_kv<D, KP>(kvr, Ks, Vs, tid);
    __syncthreads();
    if (tile + 1 < ntiles) {
      int k1, c1;
      tile_keys(tile + 1, anchor, a.S, j, a.bs, k1, c1);
      fetch_kv(a, bi, hk, k1, c1, kvr, tid);
    }
    float s[RS], dpv[RS];
#pragma unroll
    for (int i = 0; i < RS; ++i) s[i] = dpv[i] = 0.f;
    const uint32_t* kr = reinterpret_cast<const uint32_t*>(Ks + sk * KP);
    const uint32_t* vr = reinterpret_cast<const uint32_t*>(Vs + sk * KP);
#pragma unroll 4
    for (int p = 0; p < NP; ++p) {
      const float2 kf = bf2f(kr[p]);
      const float2 vf = bf2f(vr[p]);
#pragma unroll
      for (int i = 0; i < RS; ++i) {
        const int r = sg + SG * i;
        if (r >= R) break;
        const float2 qf = *reinterpret_cast<const float2*>(Qs + r * D + 2 * p);
        const float2 of = *reinterpret_cast<const float2*>(Os + r * D + 2 * p);
        s[i] = fmaf(qf.x, kf.x, fmaf(qf.y, kf.y, s[i]));
        dpv[i] = fmaf(of.x, vf.x, fmaf(of.y, vf.y, dpv[i]));
      }
    }
#pragma unroll
    for (int i = 0; i < RS; ++i) {
      const int r = sg + SG * i;
      if (r < R) {
        const float l = lse_s[r];
        const float p = (sk < cnt && l > -INFINITY) ? expf(s[i] - l) : 0.f;
        Ps[r * KT + sk] = p * (dpv[i] - delta_s[r]);
      }
    }
    __syncthreads();
    if (dp < NP) {
      for (int kk = 0; kk < cnt; ++kk) {
        const float2 kf = bf2f(reinterpret_cast<const uint32_t*>(Ks + kk * KP)[dp]);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const int r = rg + NG * i;
          if (r >= R) break;
          const float ds = Ps[r * KT + kk];
          acc[i][0] = fmaf(ds, kf.x, acc[i][0]);
          acc[i][1] = fmaf(ds, kf.y, acc[i][1]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg + NG * i;
    if (r < R && dp < NP)
      *reinterpret_cast<__nv_bfloat162*>(a.dq + qoff(a, bi, j, r, h, D) + 2 * dp) =
          __floats2bfloat162_rn(acc[i][0] * a.scale, acc[i][1] * a.scale);
  }
}

// ---------------------------------------------------------------------------- backward dk, dv
// CTA (tile, KV head, batch row) with TK keys: context tiles [0, S) in TK steps
// (DRAFT == false) or the bs draft keys of block `tile` (DRAFT == true). For every
// query block that sees the tile, the rows of all G heads of the group are staged
// in shared memory; a score phase forms P and dS (thread per key), then thread
// (column pair, key group) accumulates dK, dV over the rows.
constexpr int NTK = 256;   // threads of the dkv CTAs
constexpr int GRMAX = 64;  // G * block_size rows per query block

// GSPLIT: one CTA per (tile, KV head, GQA head g): rows of head g only, fp32 partial
// dK/dV to a.part[g] (summed over g in order by attn_dkv_gsum_kernel). More CTAs for
// the context tiles, which every query block sees.
template <int D, int TK, bool DRAFT, bool GSPLIT>
__global__ void __launch_bounds__(NTK) attn_bwd_dkv_kernel(AttnArgs a) {
  constexpr int GRM = GSPLIT ? RMAX : GRMAX;  // rows per query block in this CTA
  constexpr int KP = D + 2;
  constexpr int NP = D / 2;
  constexpr int KG = NTK / NP > 0 ? NTK / NP : 1;  // key groups in the accumulation phase
  constexpr int KPT = (TK + KG - 1) / KG;          // keys per thread there
  constexpr int SG = NTK / TK;                     // row groups in the score phase
  constexpr int RS = (GRM + SG - 1) / SG;          // rows per thread there
  extern __shared__ __align__(16) uint8_t dyn[];
  bf16* Ks = reinterpret_cast<bf16*>(dyn);
  bf16* Vs = Ks + TK * KP;
  float* Qs = reinterpret_cast<float*>(Vs + TK * KP);  // [GRM][D] q (unscaled)
  float* Os = Qs + GRM * D;                            // [GRM][D] dO
  float* Ps = Os + GRM * D;                            // [GRM][TK]
  float* DSs = Ps + GRM * TK;                          // [GRM][TK]
  float* lse_s = DSs + GRM * TK;                       // [GRM]
  float* delta_s = lse_s + GRM;                        // [GRM]
  const int G = a.Hq / a.Hk;
  const int tile = blockIdx.x, bi = blockIdx.z;
  const int hk = GSPLIT ? blockIdx.y / G : blockIdx.y;
  const int g0 = GSPLIT ? blockIdx.y % G : 0;  // first GQA head of this CTA's rows
  const int Td = a.nb * a.bs;
  const int GR = (GSPLIT ? 1 : G) * a.bs;
  const int tid = threadIdx.x;
  int k0, cnt, jlo, jhi;
  if (!DRAFT) {
    k0 = tile * TK;
    cnt = min(TK, a.S - k0);
    jlo = 0;
    jhi = a.nb;
  } else {
    k0 = a.S + tile * a.bs;
    cnt = a.bs;
    jlo = tile;
    jhi = tile + 1;
  }
  {
    KVRegs<D, TK, NTK> kvr;
    fetch_kv(a, bi, hk, k0, cnt, kvr, tid);
    store_kv<D, KP>(kvr, Ks, Vs, tid);
  }
  const int dp = tid % NP, kg = tid / NP;
  float dK[KPT][2], dV[KPT][2];
#pragma unroll
  for (int i = 0; i < KPT; ++i) dK[i][0] = dK[i][1] = dV[i][0] = dV[i][1] = 0.f;
  const int sk = tid % TK, sg = tid / TK;

  // Query blocks that see this tile, in increasing order; rows gr = g * bs + u (head
  // hk*G + g, token u of the block) are fetched one block ahead into registers.
  auto visible = [&](int j) {
    return a.keep[bi * a.nb + j] && (DRAFT || (int)a.anchors[bi * a.nb + j] > k0);
  };
  auto next_block = [&](int j) {
    while (j < jhi && !visible(j)) ++j;
    return j;
  };
  constexpr int C = D / 8;
  constexpr int RIT = (GRM * C + NTK - 1) / NTK;
  uint4 qr[RIT], orr[RIT];
  float lse_r = 0.f, delta_r = 0.f;
  auto fetch_rows = [&](int j) {
#pragma unroll
    for (int i = 0; i < RIT; ++i) {
      const int c = tid + i * NTK;
      if (c < GR * C) {
        const int gr = c / C, d8 = (c % C) * 8;
        const int64_t off = qoff(a, bi, j, gr % a.bs, hk * G + g0 + gr / a.bs, D) + d8;
        qr[i] = *reinterpret_cast<const uint4*>(a.q + off);
        orr[i] = *reinterpret_cast<const uint4*>(a.dout + off);
      }
    }
    if (tid < GR) {
      const int64_t ri = ((int64_t)bi * a.Hq + hk * G + g0 + tid / a.bs) * Td + j * a.bs + tid % a.bs;
      lse_r = a.lse[ri];
      delta_r = a.delta[ri];
    }
  };
  int j = next_block(jlo);
  if (j < jhi) fetch_rows(j);
  while (j < jhi) {
    const int anchor = (int)a.anchors[bi * a.nb + j];
    const int vis = DRAFT ? cnt : max(0, min(cnt, anchor - k0));
    __syncthreads();  // the previous block's rows are consumed
#pragma unroll
    for (int i = 0; i < RIT; ++i) {
      const int c = tid + i * NTK;
      if (c < GR * C) {
        const int gr = c / C, d8 = (c % C) * 8;
        const uint32_t qw[4] = {qr[i].x, qr[i].y, qr[i].z, qr[i].w};
        const uint32_t ow[4] = {orr[i].x, orr[i].y, orr[i].z, orr[i].w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          *reinterpret_cast<float2*>(Qs + gr * D + d8 + 2 * t) = bf2f(qw[t]);
          *reinterpret_cast<float2*>(Os + gr * D + d8 + 2 * t) = bf2f(ow[t]);
        }
      }
    }
    if (tid < GR) {
      lse_s[tid] = lse_r;
      delta_s[tid] = delta_r;
    }
    __syncthreads();
    const int jn = next_block(j + 1);
    if (jn < jhi) fetch_rows(jn);  // in flight during this block's math
    j = jn;
    float s[RS], dpv[RS];
#pragma unroll
    for (int i = 0; i < RS; ++i) s[i] = dpv[i] = 0.f;
    const uint32_t* kr = reinterpret_cast<const uint32_t*>(Ks + sk * KP);
    const uint32_t* vr = reinterpret_cast<const uint32_t*>(Vs + sk * KP);
#pragma unroll 4
    for (int p = 0; p < NP; ++p) {
      const float2 kf = bf2f(kr[p]);
      const float2 vf = bf2f(vr[p]);
#pragma unroll
      for (int i = 0; i < RS; ++i) {
        const int r = sg + SG * i;
        if (r >= GR) break;
        const float2 qf = *reinterpret_cast<const float2*>(Qs + r * D + 2 * p);
        const float2 of = *reinterpret_cast<const float2*>(Os + r * D + 2 * p);
        s[i] = fmaf(qf.x, kf.x, fmaf(qf.y, kf.y, s[i]));
        dpv[i] = fmaf(of.x, vf.x, fmaf(of.y, vf.y, dpv[i]));
      }
    }
#pragma unroll
    for (int i = 0; i < RS; ++i) {
      const int r = sg + SG * i;
      if (r < GR) {
        const float l = lse_s[r];
        const float p = (sk < vis && l > -INFINITY) ? expf(s[i] * a.scale - l) : 0.f;
        Ps[r * TK + sk] = p;
        DSs[r * TK + sk] = p * (dpv[i] - delta_s[r]) * a.scale;
      }
    }
    __syncthreads();
    if (dp < NP) {
      for (int r = 0; r < GR; ++r) {
        const float2 of = *reinterpret_cast<const float2*>(Os + r * D + 2 * dp);
        const float2 qf = *reinterpret_cast<const float2*>(Qs + r * D + 2 * dp);
#pragma unroll
        for (int i = 0; i < KPT; ++i) {
          const int kk = kg + KG * i;
          if (kk < TK) {
            const float p = Ps[r * TK + kk], ds = DSs[r * TK + kk];
            dV[i][0] = fmaf(p, of.x, dV[i][0]);
            dV[i][1] = fmaf(p, of.y, dV[i][1]);
            dK[i][0] = fmaf(ds, qf.x, dK[i][0]);
            dK[i][1] = fmaf(ds, qf.y, dK[i][1]);
          }
        }
      }
    }
  }
  if (dp < NP) {
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      const int kk = kg + KG * i;
      if (kk < cnt) {
        const int64_t row = key_row(a, bi, k0 + kk);
        if (GSPLIT) {  // context keys only: row < b * S
          const int64_t half = (int64_t)G * a.b * a.S * a.Hk * D;
          const int64_t o = ((g0 * (int64_t)a.b * a.S + row) * a.Hk + hk) * D + 2 * dp;
          *reinterpret_cast<float2*>(a.part + o) = make_float2(dK[i][0], dK[i][1]);
          *reinterpret_cast<float2*>(a.part + half + o) = make_float2(dV[i][0], dV[i][1]);
        } else {
          *reinterpret_cast<__nv_bfloat162*>(a.dk + row * a.lddk + hk * D + 2 * dp) =
              __floats2bfloat162_rn(dK[i][0], dK[i][1]);
          *reinterpret_cast<__nv_bfloat162*>(a.dv + row * a.lddv + hk * D + 2 * dp) =
              __floats2bfloat162_rn(dV[i][0], dV[i][1]);
        }
      }
    }
  }
}

// dK, dV of the context keys = sum over the G heads' fp32 partials, in head order.
template <int D>
__global__ void attn_dkv_gsum_kernel(AttnArgs a) {
  const int G = a.Hq / a.Hk;
  const int64_t pairs = (int64_t)a.b * a.S * a.Hk * (D / 2);
  const int64_t half = (int64_t)G * a.b * a.S * a.Hk * D;
  const int64_t stride_g = (int64_t)a.b * a.S * a.Hk * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = 2 * i;  // element of [b*S][Hk][D]
    const int64_t row = e / (a.Hk * D), rem = e % (a.Hk * D);
    float2 k2 = make_float2(0.f, 0.f), v2 = make_float2(0.f, 0.f);
    for (int g = 0; g < G; ++g) {
      const float2 pk = *reinterpret_cast<const float2*>(a.part + g * stride_g + e);
      const float2 pv = *reinterpret_cast<const float2*>(a.part + half + g * stride_g + e);
      k2.x += pk.x;
      k2.y += pk.y;
      v2.x += pv.x;
      v2.y += pv.y;
    }
    *reinterpret_cast<__nv_bfloat162*>(a.dk + row * a.lddk + rem) = __floats2bfloat162_rn(k2.x, k2.y);
    *reinterpret_cast<__nv_bfloat162*>(a.dv + row * a.lddv + rem) = __floats2bfloat162_rn(v2.x, v2.y);
  }
}

// ============================================================================ host
static AttnArgs make_args(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor anchors, at::Tensor keep, int S,
                          int bs) {
  NS_CHECK(q.dim() == 4 && q.is_contiguous(), "q must be contiguous [b, Td, Hq, D]");
  NS_CHECK(k.dim() == 3 && v.dim() == 3 && k.stride(2) == 1 && v.stride(2) == 1 && k.stride(1) == k.size(2) &&
               v.stride(1) == v.size(2),
           "k/v must be [rows, Hk, D] with dense heads");
  NS_CHECK(anchors.scalar_type() == at::kLong && keep.scalar_type() == at::kBool && anchors.is_contiguous() &&
               keep.is_contiguous(),
           "anchors int64 / keep bool, contiguous");
  AttnArgs a{};
  a.b = q.size(0);
  a.Hq = q.size(2);
  a.Hk = k.size(1);
  a.nb = anchors.size(1);
  a.bs = bs;
  a.S = S;
  NS_CHECK(q.size(1) == a.nb * bs, "q rows must be blocks * block_size");
  NS_CHECK(k.size(0) == (int64_t)a.b * (S + a.nb * bs), "k rows must follow the split layout");
  NS_CHECK(a.Hq % a.Hk == 0 && (a.Hq / a.Hk) * bs <= GRMAX, "GQA group * block_size must be <= 64");
  NS_CHECK(bs >= 1 && bs <= RMAX, "block_size must be in [1, 32]");
  a.q = reinterpret_cast<const bf16*>(q.data_ptr());
  a.k = reinterpret_cast<const bf16*>(k.data_ptr());
  a.v = reinterpret_cast<const bf16*>(v.data_ptr());
  a.ldk = k.stride(0);
  a.ldv = v.stride(0);
  NS_CHECK(reinterpret_cast<uintptr_t>(a.k) % 16 == 0 && reinterpret_cast<uintptr_t>(a.v) % 16 == 0 &&
               a.ldk % 8 == 0 && a.ldv % 8 == 0,
           "k/v rows must be 16-byte aligned");
  a.anchors = anchors.data_ptr<int64_t>();
  a.keep = keep.data_ptr<bool>();
  a.scale = 1.f / sqrtf((float)q.size(3));
  return a;
}

template <int D, int RM>
static void fwd_rm(const AttnArgs& a) {
  constexpr int KP = D + 2;
  const int smem = 2 * KT * KP * 2 + (RM * D + RM * KT + 3 * RM) * 4;
  NS_CUDA(cudaFuncSetAttribute(attn_fwd_kernel<D, RM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid(a.nb, a.Hq, a.b);
  attn_fwd_kernel<D, RM><<<grid, NT, smem, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
}

// Row capacity = the smallest of 8 / 16 / 32 that holds a block (fewer registers
// and less shared memory for the usual block_size 7).
template <int D>
static void fwd_d(AttnArgs a) {
  if (a.bs <= 8) fwd_rm<D, 8>(a);
  else if (a.bs <= 16) fwd_rm<D, 16>(a);
  else fwd_rm<D, 32>(a);
}

template <int D, int RM>
static void dq_rm(const AttnArgs& a) {
  constexpr int KP = D + 2;
  const int smem = 2 * KT * KP * 2 + (2 * RM * D + RM * KT + 2 * RM) * 4;
  NS_CUDA(cudaFuncSetAttribute(attn_bwd_dq_kernel<D, RM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid(a.nb, a.Hq, a.b);
  attn_bwd_dq_kernel<D, RM><<<grid, NT, smem, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
}

template <int D, int TK, bool DRAFT, bool GSPLIT>
static void dkv_launch(const AttnArgs& a, int tiles) {
  constexpr int KP = D + 2;
  constexpr int GRM = GSPLIT ? RMAX : GRMAX;
  const int smem = 2 * TK * KP * 2 + (2 * GRM * D + 2 * GRM * TK + 2 * GRM) * 4;
  auto kern = attn_bwd_dkv_kernel<D, TK, DRAFT, GSPLIT>;
  NS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid(tiles, GSPLIT ? a.Hk * (a.Hq / a.Hk) : a.Hk, a.b);
  kern<<<grid, NTK, smem, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
}

template <int D>
static void bwd_d(AttnArgs a) {
  if (a.bs <= 8) dq_rm<D, 8>(a);
  else if (a.bs <= 16) dq_rm<D, 16>(a);
  else dq_rm<D, 32>(a);
  constexpr int TKC = 16;
  const int G = a.Hq / a.Hk;
  at::Tensor part;
  if (a.S > 0) {
    const int tiles = (a.S + TKC - 1) / TKC;
    if (G > 1) {
      // context keys: one CTA per GQA head, then an ordered sum over the heads
      part = at::empty({(int64_t)2 * G * a.b * a.S * a.Hk * D}, at::TensorOptions().dtype(at::kFloat).device(at::kCUDA));
      a.part = part.data_ptr<float>();
      dkv_launch<D, TKC, false, true>(a, tiles);
      const int64_t pairs = (int64_t)a.b * a.S * a.Hk * (D / 2);
      const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((pairs + 255) / 256, (int64_t)num_sms() * 4));
      attn_dkv_gsum_kernel<D><<<blocks, 256, 0, stream()>>>(a);
      NS_CUDA(cudaGetLastError());
    } else {
      dkv_launch<D, TKC, false, false>(a, tiles);
    }
  }
  dkv_launch<D, RMAX, true, false>(a, a.nb);
}

bool dattn_supported(const at::Tensor& q, const at::Tensor& k, int64_t bs);
void dattn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs,
               at::Tensor out, at::Tensor lse);
void dattn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, at::Tensor lse,
               at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs, at::Tensor dq, at::Tensor dk,
               at::Tensor dv);

// Head dims 64 and 128 run on tensor cores (dattn.cu); the kernels of this file serve
// the other head sizes. NANOSPEC_DRAFT_ATTN=cuda forces this file's kernels.
static bool use_tc(const at::Tensor& q, const at::Tensor& k, int64_t bs) {
  static const bool forced = [] {
    const char* e = std::getenv("NANOSPEC_DRAFT_ATTN");
    return e && std::string(e) == "cuda";
  }();
  return !forced && dattn_supported(q, k, bs);
}

void attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs,
              at::Tensor out, at::Tensor lse) {
  AttnArgs a = make_args(q, k, v, anchors, keep, S, bs);
  if (use_tc(q, k, bs)) {
    dattn_fwd(q, k, v, anchors, keep, S, bs, out, lse);
    return;
  }
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  switch (q.size(3)) {
    case 16: fwd_d<16>(a); break;
    case 32: fwd_d<32>(a); break;
    case 64: fwd_d<64>(a); break;
    case 128: fwd_d<128>(a); break;
    default: NS_CHECK(false, "draft attention head_dim must be 16, 32, 64 or 128");
  }
}

void attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, at::Tensor lse,
              at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs, at::Tensor dq, at::Tensor dk,
              at::Tensor dv) {
  AttnArgs a = make_args(q, k, v, anchors, keep, S, bs);
  NS_CHECK(dout.is_contiguous() && out.is_contiguous() && dq.is_contiguous(), "dout/out/dq must be contiguous");
  NS_CHECK(dk.stride(2) == 1 && dv.stride(2) == 1, "dk/dv must have dense heads");
  if (use_tc(q, k, bs) && dk.stride(1) == dk.size(2) && dv.stride(1) == dv.size(2)) {
    dattn_bwd(dout, q, k, v, out, lse, anchors, keep, S, bs, dq, dk, dv);
    return;
  }
  a.dout = reinterpret_cast<const bf16*>(dout.data_ptr());
  a.o = reinterpret_cast<const bf16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  auto delta = at::empty_like(lse);
  a.delta = delta.data_ptr<float>();
  a.dq = reinterpret_cast<bf16*>(dq.data_ptr());
  a.dk = reinterpret_cast<bf16*>(dk.data_ptr());
  a.dv = reinterpret_cast<bf16*>(dv.data_ptr());
  a.lddk = dk.stride(0);
  a.lddv = dv.stride(0);
  switch (q.size(3)) {
    case 16: bwd_d<16>(a); break;
    case 32: bwd_d<32>(a); break;
    case 64: bwd_d<64>(a); break;
    case 128: bwd_d<128>(a); break;
    default: NS_CHECK(false, "draft attention head_dim must be 16, 32, 64 or 128");
  }
}

}  // namespace ns
