// Chunked gated delta rule, forward (the frozen verifier's linear-attention mixer).
//
// Reference math: nanospec/ops.py:203-239 (HF's torch fallback ordering): q and k
// L2-normalised in the compute dtype, q scaled by d^-1/2, chunks of C = 64 tokens,
// cumulative log-decay G inside a chunk, then per chunk
//   M  = strict_lower(beta_i k_i.k_j e^{G_i - G_j})        T = (I + M)^-1
//   W  = T (beta k e^G)        U = T (beta v)                 (chunk-local)
//   A  = lower(q_i.k_j e^{G_i - G_j})                         (chunk-local)
//   v' = U - W S ;  o = (q e^G) S + A v' ;  S = e^{G_last} S + (k e^{G_last - G})^T v'
// with the fp32 state S [d_k, d_v] carried from chunk to chunk.
//
// The chunk-local part is independent across chunks, so it runs as its own kernel
// over every (chunk, head, row) at once (`gdn_prep_kernel`: 3072 CTAs at 48 heads x
// 4096 tokens). Only the state recurrence is sequential. At d = 128 (the 27B shape)
// it runs on tcgen05 (`gdn_state_tc_kernel`: one CTA per head, the fp32 state in
// TMEM, four MMAs per chunk, operand tiles by TMA). Other head sizes use
// `gdn_state_kernel` on CUDA cores, split across value columns (columns of S are
// independent): (d_v / 32) x heads x rows CTAs, two per SM, each walking the chunks
// with its slice of S in shared memory, fed by bulk copies (cp.async.bulk, this
// GPU's memory only) completing on an mbarrier with a bounded wait.
//
// The triangular inverse is blocked: 16 x 16 diagonal blocks by column-parallel
// forward substitution (each thread owns one column, no barriers), then the three
// block-distances of off-diagonal blocks, T_ik = -T_ii sum_{m=k}^{i-1} M_im T_mk.
#include "common.h"
#include "sm100.cuh"

namespace ns {

using bf16 = __nv_bfloat16;

namespace gdn {

constexpr int C = 64;       // chunk length
constexpr int CP = C + 1;   // row length of the [D][C] transpose buffer: lanes 4 rows apart land 4 banks apart
constexpr int NT = 256;     // threads per CTA (both kernels)

__device__ __forceinline__ float bf(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float rb(float x) { return sm100::bf16_round(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

template <int D>
struct Prep {
  static constexpr int DB = D + 4;                 // padded bf16 row of the [C][D] q / k / v tiles
  static constexpr int TILE = C * DB * 2;          // bytes of one tile
  static constexpr int MS = C * (C + 1);           // fp32 [C][C + 1]
  static constexpr int PS = 3 * 16 * 17;
  static constexpr int TR = D * CP * 4;            // fp32 transpose buffer [D][CP] (reuses q / k tiles)
  static constexpr int QK = 2 * TILE > TR ? 2 * TILE : TR;
  static constexpr int BYTES = QK + TILE + (2 * MS + PS + 5 * C) * 4;
};

__device__ __forceinline__ void ld_bf16x4(const bf16* p, float (&f)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
}

__device__ __forceinline__ void st_bf16x4(bf16* p, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = u;
}

// Outputs per (row, head, chunk) ck, two layouts:
//  TC = false (CUDA-core state kernel): WT fp32 [D][C], QgT bf16 [D][C], Kd bf16 [C][D],
//      AqkT fp32 [C][C] (A transposed), U fp32 slice-major [D/dvs][C][dvs];
//  TC = true (tensor-core state kernel, operands K-major for tcgen05): W bf16 [C][D],
//      Qg bf16 [C][D], Kd^T bf16 [D][C], A bf16 [C][C], U^T fp32 [D][C].
// GL fp32 = e^{G_last} either way. q / k / v rows are strided: token t of row b at
// (b * s + t) * x_ts (elements), head offset h * D.
// Shared memory holds the chunk's normalised q and k and raw v as bf16 rows (they are
// bf16 values in the reference statement too), about 90 KB, so two CTAs share an SM.
template <int D, bool TC>
__global__ void __launch_bounds__(NT, 2) gdn_prep_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                         const bf16* __restrict__ v, int64_t q_ts, int64_t k_ts,
                                                         int64_t v_ts, const float* __restrict__ gin,
                                                         const bf16* __restrict__ beta_in, int s, int nk, int nv,
                                                         int groups, int nchunks, void* __restrict__ Wo,
                                                         bf16* __restrict__ QgO, bf16* __restrict__ KdO,
                                                         void* __restrict__ AqkO, float* __restrict__ Uo,
                                                         float* __restrict__ GL, int dvs) {
  using L = Prep<D>;
  constexpr int DB = L::DB;
  extern __shared__ __align__(16) uint8_t smp[];
  bf16* qs = reinterpret_cast<bf16*>(smp);             // [C][DB]
  bf16* ks = qs + C * DB;                              // [C][DB]
  bf16* vs = reinterpret_cast<bf16*>(smp + L::QK);     // [C][DB]
  float* Ms = reinterpret_cast<float*>(smp + L::QK + L::TILE);
  float* Ts = Ms + L::MS;
  float* Ps = Ts + L::MS;
  float* G = Ps + L::PS;
  float* Bt = G + C;
  float* eG = Bt + C;
  float* eGl = eG + C;
  float* fk = eGl + C;  // beta e^G
  float* tr = reinterpret_cast<float*>(smp);           // [D][CP] transpose buffer (after q / k are consumed)
  const int ch = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int hk = h / groups;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = ch * C, cnt = min(C, s - t0);
  const float scale = rsqrtf((float)D);
  const int64_t ck = ((int64_t)bi * nv + h) * nchunks + ch;

  // 1. load; q and k L2-normalised as the bf16 statement computes them. Lane l holds
  //    channels [4l, 4l + 4); two rows per step so their loads overlap.
  {
    constexpr int LANES = D / 4;  // active lanes per row
    for (int r0 = warp * 2; r0 < C; r0 += 2 * (NT / 32)) {
      float qa[2][4], ka[2][4], va[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = r0 + u;
        const bool in = r < cnt && lane < LANES;
        const int64_t tq = (int64_t)bi * s + t0 + r;
        if (in) {
          ld_bf16x4(q + tq * q_ts + hk * D + 4 * lane, qa[u]);
          ld_bf16x4(k + tq * k_ts + hk * D + 4 * lane, ka[u]);
          ld_bf16x4(v + tq * v_ts + h * D + 4 * lane, va[u]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) qa[u][e] = ka[u][e] = va[u][e] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int r = r0 + u;
        float sq = 0.f, sk = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          sq += rb(qa[u][e] * qa[u][e]);
          sk += rb(ka[u][e] * ka[u][e]);
        }
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        const float iq = rb(rsqrtf(rb(rb(sq) + 1e-6f)));
        const float ik = rb(rsqrtf(rb(rb(sk) + 1e-6f)));
        if (lane < LANES) {
          st_bf16x4(qs + r * DB + 4 * lane, qa[u][0] * iq, qa[u][1] * iq, qa[u][2] * iq, qa[u][3] * iq);
          st_bf16x4(ks + r * DB + 4 * lane, ka[u][0] * ik, ka[u][1] * ik, ka[u][2] * ik, ka[u][3] * ik);
          st_bf16x4(vs + r * DB + 4 * lane, va[u][0], va[u][1], va[u][2], va[u][3]);
        }
        if (lane == 0) {
          const bool in = r < cnt;
          const int64_t tq = (int64_t)bi * s + t0 + r;
          G[r] = in ? gin[tq * nv + h] : 0.f;
          Bt[r] = in ? bf(beta_in[tq * nv + h]) : 0.f;
        }
      }
    }
  }
  __syncthreads();
  if (warp == 0) {  // inclusive prefix sum of g over the chunk, two entries per lane
    const float a = G[2 * lane], b = G[2 * lane + 1];
    const float pair = a + b;
    float inc = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xffffffff, inc, o);
      if (lane >= o) inc += n;
    }
    const float excl = inc - pair;
    G[2 * lane] = excl + a;
    G[2 * lane + 1] = excl + a + b;
  }
  __syncthreads();
  const float Gl = G[C - 1];
  if (tid < C) {
    eG[tid] = expf(G[tid]);
    eGl[tid] = expf(Gl - G[tid]);
    fk[tid] = Bt[tid] * eG[tid];
  }
  __syncthreads();

  // 2. M = strict_lower(beta_i k_i.k_j e^{G_i-G_j}) and A = lower(scale q_i.k_j e^{G_i-G_j}).
  //    Thread t < 136 takes block (bi, bj) of the lower triangle of 4 x 4 blocks and
  //    walks d four channels at a time; the blocks above the diagonal are zero.
  {
    constexpr int NB = C / 4, TRI = NB * (NB + 1) / 2;
    float* at = reinterpret_cast<float*>(AqkO) + ck * C * C;   // TC = false: A^T fp32
    bf16* ab = reinterpret_cast<bf16*>(AqkO) + ck * C * C;     // TC = true: A bf16 row-major
    if (tid < TRI) {
      int bi2 = (int)((sqrtf(8.f * tid + 1.f) - 1.f) * 0.5f);
      if ((bi2 + 1) * (bi2 + 2) / 2 <= tid) ++bi2;
      if (bi2 * (bi2 + 1) / 2 > tid) --bi2;
      const int bj = tid - bi2 * (bi2 + 1) / 2;
      const int i0 = bi2 * 4, j0 = bj * 4;
      float kk[4][4], qk[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) kk[r][c] = qk[r][c] = 0.f;
#pragma unroll 2
      for (int d = 0; d < D; d += 4) {
        float ki[4][4], qi[4][4], kj[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          ld_bf16x4(ks + (i0 + r) * DB + d, ki[r]);
          ld_bf16x4(qs + (i0 + r) * DB + d, qi[r]);
          ld_bf16x4(ks + (j0 + r) * DB + d, kj[r]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              kk[r][c] = fmaf(ki[r][e], kj[c][e], kk[r][c]);
              qk[r][c] = fmaf(qi[r][e], kj[c][e], qk[r][c]);
            }
      }
      float a16[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = j0 + c;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int i = i0 + r;
          const float dec = j <= i ? expf(G[i] - G[j]) : 0.f;
          Ms[i * (C + 1) + j] = j < i ? Bt[i] * kk[r][c] * dec : 0.f;
          a16[r][c] = j <= i ? scale * qk[r][c] * dec : 0.f;
        }
      }
      if constexpr (TC) {
#pragma unroll
        for (int r = 0; r < 4; ++r) st_bf16x4(&ab[(i0 + r) * C + j0], a16[r][0], a16[r][1], a16[r][2], a16[r][3]);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<float4*>(&at[(j0 + c) * C + i0]) =
              make_float4(a16[0][c], a16[1][c], a16[2][c], a16[3][c]);
      }
    } else {
      for (int idx = tid - TRI; idx < NB * NB - TRI; idx += NT - TRI) {
        int i = 0, rem = idx;
        while (rem >= NB - 1 - i) {
          rem -= NB - 1 - i;
          ++i;
        }
        const int j = i + 1 + rem;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int r = 0; r < 4; ++r) Ms[(i * 4 + r) * (C + 1) + j * 4 + c] = 0.f;
          if constexpr (TC)
            *reinterpret_cast<uint2*>(&ab[(i * 4 + c) * C + j * 4]) = make_uint2(0u, 0u);
          else
            *reinterpret_cast<float4*>(&at[(j * 4 + c) * C + i * 4]) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
  }
  // q scale e^G and k e^{G_last - G} for the state kernel (bf16), from the smem rows
  {
    bf16* qg = QgO + ck * D * C;
    bf16* kd = KdO + ck * C * D;
    if constexpr (TC) {
      for (int idx = tid; idx < C * D; idx += NT) {  // Qg [C][D]
        const int i = idx / D, d = idx % D;
        qg[idx] = __float2bfloat16(bf(qs[i * DB + d]) * scale * eG[i]);
      }
      for (int idx = tid; idx < D * C; idx += NT) {  // Kd^T [D][C]
        const int d = idx / C, i = idx % C;
        kd[idx] = __float2bfloat16(bf(ks[i * DB + d]) * eGl[i]);
      }
    } else {
      for (int idx = tid; idx < D * C; idx += NT) {  // Qg^T [D][C]
        const int d = idx / C, i = idx % C;
        qg[idx] = __float2bfloat16(bf(qs[i * DB + d]) * scale * eG[i]);
      }
      for (int idx = tid; idx < C * D; idx += NT) {  // Kd [C][D]
        const int i = idx / D, d = idx % D;
        kd[idx] = __float2bfloat16(bf(ks[i * DB + d]) * eGl[i]);
      }
    }
    if (tid == 0) GL[ck] = expf(Gl);
  }
  __syncthreads();

  // 3. T = (I + M)^-1, blocked by 16. (a) diagonal blocks: thread c owns column c and
  //    keeps it in registers: T[i][c] = -sum_{m<i} M[i][m] T[m][c] below the diagonal.
  if (tid < C) {
    const int c = tid, r0 = (c >> 4) * 16, cl = c & 15;
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] = i == cl ? 1.f : 0.f;
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) acc = fmaf(Ms[(r0 + i) * (C + 1) + r0 + m], t[m], acc);
      if (i > cl) t[i] = -acc;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) Ts[(r0 + i) * (C + 1) + c] = t[i];
    for (int r = 0; r < r0; ++r) Ts[r * (C + 1) + c] = 0.f;  // above the diagonal blocks
  }
  __syncthreads();
  // (b) off-diagonal blocks, by block distance
  for (int dist = 1; dist < 4; ++dist) {
    const int nb = 4 - dist;
    for (int idx = tid; idx < nb * 256; idx += NT) {
      const int p = idx >> 8, r = (idx >> 4) & 15, c = idx & 15;
      const int bk = p, bi2 = p + dist;
      float acc = 0.f;
      for (int m = bk * 16; m < bi2 * 16; ++m) acc += Ms[(bi2 * 16 + r) * (C + 1) + m] * Ts[m * (C + 1) + bk * 16 + c];
      Ps[p * 272 + r * 17 + c] = acc;
    }
    __syncthreads();
    for (int idx = tid; idx < nb * 256; idx += NT) {
      const int p = idx >> 8, r = (idx >> 4) & 15, c = idx & 15;
      const int bk = p, bi2 = p + dist;
      float acc = 0.f;
#pragma unroll 4
      for (int m = 0; m < 16; ++m) acc += Ts[(bi2 * 16 + r) * (C + 1) + bi2 * 16 + m] * Ps[p * 272 + m * 17 + c];
      Ts[(bi2 * 16 + r) * (C + 1) + bk * 16 + c] = -acc;
    }
    __syncthreads();
  }

  // 4. W = T (beta e^G k), U = T (beta v): the row factors are applied on the fly
  {
    constexpr int EG = D / 4, IG = NT / EG, RPT = C / IG;
    const int eg = tid % EG, i0 = (tid / EG) * RPT, e0 = eg * 4;
    float w[RPT][4], u[RPT][4];
#pragma unroll
    for (int r = 0; r < RPT; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) w[r][c] = u[r][c] = 0.f;
    for (int j = 0; j < i0 + RPT; ++j) {
      float kv[4], vv[4];
      ld_bf16x4(ks + j * DB + e0, kv);
      ld_bf16x4(vs + j * DB + e0, vv);
      const float fkj = fk[j], fvj = Bt[j];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        kv[c] *= fkj;
        vv[c] *= fvj;
      }
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const float t = Ts[(i0 + r) * (C + 1) + j];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          w[r][c] = fmaf(t, kv[c], w[r][c]);
          u[r][c] = fmaf(t, vv[c], u[r][c]);
        }
      }
    }
    __syncthreads();  // q / k tiles consumed: their space becomes the transpose buffer
    if constexpr (TC) {
      // W bf16 [C][D] straight from registers; U^T fp32 [D][C] through shared memory
      bf16* wo = reinterpret_cast<bf16*>(Wo) + ck * C * D;
#pragma unroll
      for (int r = 0; r < RPT; ++r) st_bf16x4(&wo[(i0 + r) * D + e0], w[r][0], w[r][1], w[r][2], w[r][3]);
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int r = 0; r < RPT; ++r) tr[(e0 + c) * CP + i0 + r] = u[r][c];
      __syncthreads();
      float* ut = Uo + ck * D * C;
      for (int idx = tid; idx < D * C / 4; idx += NT) {
        const int e = idx / (C / 4), i4 = (idx % (C / 4)) * 4;
        const float* src = &tr[e * CP + i4];
        *reinterpret_cast<float4*>(&ut[e * C + i4]) = make_float4(src[0], src[1], src[2], src[3]);
      }
    } else {
      const int slice = e0 / dvs, el = e0 % dvs;
      float* uo = Uo + (ck * (D / dvs) + slice) * C * dvs;
#pragma unroll
      for (int r = 0; r < RPT; ++r)
        *reinterpret_cast<float4*>(&uo[(i0 + r) * dvs + el]) = make_float4(u[r][0], u[r][1], u[r][2], u[r][3]);
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int r = 0; r < RPT; ++r) tr[(e0 + c) * CP + i0 + r] = w[r][c];
      __syncthreads();
      float* wt = reinterpret_cast<float*>(Wo) + ck * D * C;
      for (int idx = tid; idx < D * C / 4; idx += NT) {
        const int e = idx / (C / 4), i4 = (idx % (C / 4)) * 4;
        const float* src = &tr[e * CP + i4];
        *reinterpret_cast<float4*>(&wt[e * C + i4]) = make_float4(src[0], src[1], src[2], src[3]);
      }
    }
  }
}

template <int D, int DVS>
struct State {
  static constexpr int FLOATS = D * DVS + C * DVS + D * C + C * C + C * DVS;
  static constexpr int BYTES = FLOATS * 4 + 2 * D * C * 2;
};

template <int D, int DVS>
__global__ void __launch_bounds__(NT, 2) gdn_state_kernel(const float* __restrict__ WT, const bf16* __restrict__ QgT,
                                                          const bf16* __restrict__ Kd, const float* __restrict__ AqkT,
                                                          const float* __restrict__ Uo, const float* __restrict__ GL,
                                                          bf16* __restrict__ out, int s, int nv, int nchunks,
                                                          int* err) {
  extern __shared__ __align__(128) float smf[];
  float* S = smf;               // [D][DVS]
  float* vn = S + D * DVS;      // [C][DVS]
  float* Ws = vn + C * DVS;     // [D][C]
  float* As = Ws + D * C;       // [C][C]
  float* Us = As + C * C;       // [C][DVS]
  bf16* Qs = reinterpret_cast<bf16*>(Us + C * DVS);  // [D][C]
  bf16* Ks = Qs + D * C;                             // [C][D]
  __shared__ __align__(8) uint64_t bar;
  const int slice = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  constexpr int NSL = D / DVS;
  const int tid = threadIdx.x;
  for (int i = tid; i < D * DVS; i += NT) S[i] = 0.f;
  if (tid == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  constexpr uint32_t BYTES = D * C * 4 + C * C * 4 + C * DVS * 4 + 2 * D * C * 2;
  // step (a)/(b) mapping: RA rows x 4 value columns per thread
  constexpr int EG = DVS / 4, IGA = NT / EG, RA = C / IGA;
  const int eg = tid % EG, e0 = eg * 4, ia = (tid / EG) * RA;
  // step (c) mapping: SR rows of S x 4 columns per thread
  constexpr int DG = NT / EG, SR = D >= DG ? D / DG : 1;
  const bool cact = tid < (D / SR) * EG;
  const int d0 = (tid / EG) * SR;
  for (int ch = 0; ch < nchunks; ++ch) {
    const int64_t ck = ((int64_t)bi * nv + h) * nchunks + ch;
    if (tid == 0) {
      sm100::mbar_expect_tx(&bar, BYTES);
      sm100::bulk_load(Ws, WT + ck * D * C, D * C * 4, &bar);
      sm100::bulk_load(As, AqkT + ck * C * C, C * C * 4, &bar);
      sm100::bulk_load(Us, Uo + (ck * NSL + slice) * C * DVS, C * DVS * 4, &bar);
      sm100::bulk_load(Qs, QgT + ck * D * C, D * C * 2, &bar);
      sm100::bulk_load(Ks, Kd + ck * C * D, C * D * 2, &bar);
    }
    const bool ok = sm100::mbar_wait(&bar, ch & 1, err);
    if (__syncthreads_or(!ok)) return;  // every thread leaves together; the word is set
    // (a) v' = U - W S and o = (q e^G) S
    float va[RA][4], oa[RA][4];
#pragma unroll
    for (int r = 0; r < RA; ++r) {
      const float4 u4 = *reinterpret_cast<const float4*>(&Us[(ia + r) * DVS + e0]);
      va[r][0] = u4.x, va[r][1] = u4.y, va[r][2] = u4.z, va[r][3] = u4.w;
      oa[r][0] = oa[r][1] = oa[r][2] = oa[r][3] = 0.f;
    }
#pragma unroll 4
    for (int d = 0; d < D; ++d) {
      const float4 s4 = *reinterpret_cast<const float4*>(&S[d * DVS + e0]);
#pragma unroll
      for (int r = 0; r < RA; ++r) {
        const float w = Ws[d * C + ia + r];
        const float qv = bf(Qs[d * C + ia + r]);
        va[r][0] = fmaf(-w, s4.x, va[r][0]);
        va[r][1] = fmaf(-w, s4.y, va[r][1]);
        va[r][2] = fmaf(-w, s4.z, va[r][2]);
        va[r][3] = fmaf(-w, s4.w, va[r][3]);
        oa[r][0] = fmaf(qv, s4.x, oa[r][0]);
        oa[r][1] = fmaf(qv, s4.y, oa[r][1]);
        oa[r][2] = fmaf(qv, s4.z, oa[r][2]);
        oa[r][3] = fmaf(qv, s4.w, oa[r][3]);
      }
    }
#pragma unroll
    for (int r = 0; r < RA; ++r)
      *reinterpret_cast<float4*>(&vn[(ia + r) * DVS + e0]) = make_float4(va[r][0], va[r][1], va[r][2], va[r][3]);
    __syncthreads();
    // (b) o += A v' (A is zero above the diagonal)
    for (int j = 0; j < ia + RA; ++j) {
      const float4 v4 = *reinterpret_cast<const float4*>(&vn[j * DVS + e0]);
#pragma unroll
      for (int r = 0; r < RA; ++r) {
        const float a = As[j * C + ia + r];
        oa[r][0] = fmaf(a, v4.x, oa[r][0]);
        oa[r][1] = fmaf(a, v4.y, oa[r][1]);
        oa[r][2] = fmaf(a, v4.z, oa[r][2]);
        oa[r][3] = fmaf(a, v4.w, oa[r][3]);
      }
    }
#pragma unroll
    for (int r = 0; r < RA; ++r) {
      const int t = ch * C + ia + r;
      if (t < s) {
        bf16* o = out + (((int64_t)bi * s + t) * nv + h) * D + slice * DVS + e0;
        __nv_bfloat162 lo = __floats2bfloat162_rn(oa[r][0], oa[r][1]);
        __nv_bfloat162 hi = __floats2bfloat162_rn(oa[r][2], oa[r][3]);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(o) = pk;
      }
    }
    // (c) S = e^{G_last} S + (k e^{G_last - G})^T v'. Every thread reads and writes
    // only its own block of S here; the reads of S in (a) are behind the barrier above.
    if (cact) {
      const float gl = GL[ck];
      float sa[SR][4];
#pragma unroll
      for (int r = 0; r < SR; ++r) {
        const float4 s4 = *reinterpret_cast<const float4*>(&S[(d0 + r) * DVS + e0]);
        sa[r][0] = gl * s4.x, sa[r][1] = gl * s4.y, sa[r][2] = gl * s4.z, sa[r][3] = gl * s4.w;
      }
#pragma unroll 4
      for (int i = 0; i < C; ++i) {
        const float4 v4 = *reinterpret_cast<const float4*>(&vn[i * DVS + e0]);
#pragma unroll
        for (int r = 0; r < SR; ++r) {
          const float kd = bf(Ks[i * D + d0 + r]);
          sa[r][0] = fmaf(kd, v4.x, sa[r][0]);
          sa[r][1] = fmaf(kd, v4.y, sa[r][1]);
          sa[r][2] = fmaf(kd, v4.z, sa[r][2]);
          sa[r][3] = fmaf(kd, v4.w, sa[r][3]);
        }
      }
#pragma unroll
      for (int r = 0; r < SR; ++r)
        *reinterpret_cast<float4*>(&S[(d0 + r) * DVS + e0]) = make_float4(sa[r][0], sa[r][1], sa[r][2], sa[r][3]);
    }
    __syncthreads();  // S final and the chunk's tiles consumed before the next bulk copy
  }
}

// ------------------------------------------------------------------ tensor-core state kernel
// One CTA per (head, row), d_k = d_v = 128. The state is held transposed, S^T [d_v, d_k],
// as an fp32 tcgen05 accumulator in TMEM (lane = value channel). Per chunk:
//   MMA1  v'^T  = S^T W^T          M=128 (d_v), N=64 (tokens), K=128 (d_k)
//   MMA2  o^T   = S^T Qg^T         same shape
//   rows: v^T = U^T - v'^T -> bf16 A operand
//   MMA3  o^T  += v^T A^T          M=128, N=64, K=64
//   MMA4  S^T   = e^{G_last} S^T + v^T Kd     M=128, N=128 (d_k), K=64
// S^T is read back once per chunk: rounded to bf16 as the A operand of MMA1/2 (the
// fp32 copy stays in TMEM), and scaled by e^{G_last} in place before MMA4 accumulates.
// Chunk operand tiles (W, Qg, A, Kd^T, all bf16 K-major) arrive by TMA into a 2-stage
// ring with 128-byte swizzle. Warps: 0 TMA, 1 MMA issuer + TMEM owner, 2-5 rows.
namespace tcs {
constexpr int TILE_W = C * 128 * 2;    // [64][128] bf16, two swizzle atoms
constexpr int TILE_A = C * C * 2;      // [64][64]
constexpr int TILE_K = 128 * C * 2;    // [128][64]
constexpr int STAGE = 2 * TILE_W + TILE_A + TILE_K;   // 56 KB
constexpr int ST_BYTES = 128 * 128 * 2;               // S^T bf16 [128][128], two atoms
constexpr int VN_BYTES = 128 * C * 2;                 // v^T bf16 [128][64]
constexpr int SMEM = ST_BYTES + VN_BYTES + 2 * STAGE + 1024 + 256;
constexpr int S_COL = 0, VN_COL = 128, O_COL = 192, TMEM_COLS = 256;
}  // namespace tcs

// 8 bf16 from 8 floats
__device__ __forceinline__ uint4 pack_bf16x8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

__global__ void __launch_bounds__(192, 1)
    gdn_state_tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tq,
                        const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tk,
                        const float* __restrict__ Ut, const float* __restrict__ GL, bf16* __restrict__ out, int s,
                        int nv, int nchunks, int* err) {
  using namespace tcs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sS = smem;                    // S^T bf16, A operand of MMA1/2
  uint8_t* sV = sS + ST_BYTES;           // v^T bf16, A operand of MMA3/4
  uint8_t* ring = sV + VN_BYTES;         // [2][W | Qg | A | Kd^T]
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + 2 * STAGE);
  uint64_t* full = bars;         // [2]
  uint64_t* empty = bars + 2;    // [2]
  uint64_t* a_ready = bars + 4;  // S^T operand + scaled TMEM state ready (4 row warps)
  uint64_t* v_ready = bars + 5;  // v^T operand ready (4 row warps)
  uint64_t* mm12 = bars + 6;     // MMA1/2 done
  uint64_t* mm34 = bars + 7;     // MMA3/4 done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, bi = blockIdx.y;

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    sm100::mbar_init(a_ready, 4);
    sm100::mbar_init(v_ready, 4);
    sm100::mbar_init(mm12, 1);
    sm100::mbar_init(mm34, 1);
    sm100::fence_barrier_init();
    sm100::tma_prefetch_desc(&tw);
    sm100::tma_prefetch_desc(&tq);
    sm100::tma_prefetch_desc(&ta);
    sm100::tma_prefetch_desc(&tk);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int64_t ck0 = ((int64_t)bi * nv + h) * nchunks;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int ch = 0; ch < nchunks; ++ch) {
        const int st = ch & 1;
        if (ch >= 2 && !sm100::mbar_wait(&empty[st], ((ch >> 1) - 1) & 1, err)) break;
        uint8_t* d = ring + st * STAGE;
        const int row = (int)((ck0 + ch) * C);
        sm100::mbar_expect_tx(&full[st], STAGE);
        sm100::tma_load_2d(d, &tw, &full[st], 0, row);
        sm100::tma_load_2d(d + C * 128, &tw, &full[st], 64, row);
        sm100::tma_load_2d(d + TILE_W, &tq, &full[st], 0, row);
        sm100::tma_load_2d(d + TILE_W + C * 128, &tq, &full[st], 64, row);
        sm100::tma_load_2d(d + 2 * TILE_W, &ta, &full[st], 0, row);
        sm100::tma_load_2d(d + 2 * TILE_W + TILE_A, &tk, &full[st], 0, (int)((ck0 + ch) * 128));
        issued = ch + 1;
      }
      for (int ch = max(0, issued - 2); ch < issued; ++ch) sm100::mbar_wait(&full[ch & 1], (ch >> 1) & 1, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id64 = sm100::idesc_bf16(128, C, false, false);
      constexpr uint32_t id128 = sm100::idesc_bf16(128, 128, false, false);
      const uint32_t s_base = sm100::smem_u32(sS), v_base = sm100::smem_u32(sV);
      for (int ch = 0; ch < nchunks; ++ch) {
        const int st = ch & 1;
        if (!sm100::mbar_wait(a_ready, ch & 1, err)) break;
        if (!sm100::mbar_wait(&full[st], (ch >> 1) & 1, err)) break;
        sm100::tc_fence_after();
        const uint32_t r_base = sm100::smem_u32(ring + st * STAGE);
        const uint32_t w_base = r_base, q_base = r_base + TILE_W, a_base = r_base + 2 * TILE_W,
                       k_base = a_base + TILE_A;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // K = d_k = 128
          const uint64_t ad = sm100::smem_desc_sw128(s_base + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bw = sm100::smem_desc_sw128(w_base + (kk >> 2) * (C * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bq = sm100::smem_desc_sw128(q_base + (kk >> 2) * (C * 128) + (kk & 3) * 32, 0, 1024);
          sm100::mma_bf16(tmem + VN_COL, ad, bw, id64, kk > 0 ? 1u : 0u);
          sm100::mma_bf16(tmem + O_COL, ad, bq, id64, kk > 0 ? 1u : 0u);
        }
        sm100::mma_commit(mm12);
        if (!sm100::mbar_wait(v_ready, ch & 1, err)) break;
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // K = 64 tokens of the chunk
          const uint64_t av = sm100::smem_desc_sw128(v_base + kk * 32, 0, 1024);
          const uint64_t ba = sm100::smem_desc_sw128(a_base + kk * 32, 0, 1024);
          const uint64_t bk = sm100::smem_desc_sw128(k_base + kk * 32, 0, 1024);
          sm100::mma_bf16(tmem + O_COL, av, ba, id64, 1u);
          sm100::mma_bf16(tmem + S_COL, av, bk, id128, (ch > 0 || kk > 0) ? 1u : 0u);
        }
        sm100::mma_commit(mm34);
        sm100::mma_commit(&empty[st]);
      }
    }
  } else {
    const int qw = warp & 3;
    const int r = qw * 32 + lane;  // value channel = TMEM lane = A-operand row
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    bool ok = true;
    float un[C];  // U^T row r of the next chunk
    if (nchunks > 0) {
      const float4* up = reinterpret_cast<const float4*>(Ut + (ck0 * 128 + r) * C);
#pragma unroll
      for (int j = 0; j < C / 4; ++j) {
        const float4 t = up[j];
        un[4 * j] = t.x, un[4 * j + 1] = t.y, un[4 * j + 2] = t.z, un[4 * j + 3] = t.w;
      }
    }
    for (int ch = 0; ch < nchunks && ok; ++ch) {
      const int64_t ck = ck0 + ch;
      // ---- (a) state operand for this chunk
      if (ch == 0) {
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<uint4*>(sS + (c >> 3) * (128 * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4)) =
              make_uint4(0u, 0u, 0u, 0u);
      } else {
        const float gl = GL[ck];  // independent of the MMAs: load before the wait
        ok = __all_sync(0xffffffff, sm100::mbar_wait(mm34, (ch - 1) & 1, err));
        if (!ok) break;
        sm100::tc_fence_after();
        // previous chunk's output o^T, then S^T -> bf16 operand and e^{G_last} S^T in place
        {
          const int t0 = (ch - 1) * C;
          const int cnt = min(C, s - t0);
#pragma unroll 1
          for (int c = 0; c < C; c += 32) {
            float o[32];
            sm100::tmem_ld32(tmem + lane_off + O_COL + c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i)  // constant indices: o stays in registers
              if (c + i < cnt) out[(((int64_t)bi * s + t0 + c + i) * nv + h) * 128 + r] = __float2bfloat16(o[i]);
          }
        }
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          float v[32];
          sm100::tmem_ld32(tmem + lane_off + S_COL + c, v);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int ch16 = (c >> 3) + j;  // 16-byte chunk index along d_k (0..15)
            *reinterpret_cast<uint4*>(sS + (ch16 >> 3) * (128 * 128) + r * 128 + (((ch16 & 7) ^ (r & 7)) << 4)) =
                pack_bf16x8(v + 8 * j);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= gl;
          sm100::tmem_st32(tmem + lane_off + S_COL + c, v);
        }
      }
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(a_ready);
      // ---- (b) v^T = U^T - S^T W^T; U of the next chunk is loaded now (it is used
      //      one chunk later, so its latency hides behind this chunk's MMAs)
      float u[C];
#pragma unroll
      for (int j = 0; j < C; ++j) u[j] = un[j];
      if (ch + 1 < nchunks) {
        const float4* up = reinterpret_cast<const float4*>(Ut + ((ck + 1) * 128 + r) * C);
#pragma unroll
        for (int j = 0; j < C / 4; ++j) {
          const float4 t = up[j];
          un[4 * j] = t.x, un[4 * j + 1] = t.y, un[4 * j + 2] = t.z, un[4 * j + 3] = t.w;
        }
      }
      ok = __all_sync(0xffffffff, sm100::mbar_wait(mm12, ch & 1, err));
      if (!ok) break;
      sm100::tc_fence_after();
#pragma unroll
      for (int c = 0; c < C; c += 32) {  // fully unrolled: u stays in registers
        float v[32];
        sm100::tmem_ld32(tmem + lane_off + VN_COL + c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = u[c + j] - v[j];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch16 = (c >> 3) + j;
          *reinterpret_cast<uint4*>(sV + r * 128 + ((ch16 ^ (r & 7)) << 4)) = pack_bf16x8(v + 8 * j);
        }
      }
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(v_ready);
    }
    // output of the last chunk
    if (ok && nchunks > 0) {
      ok = __all_sync(0xffffffff, sm100::mbar_wait(mm34, (nchunks - 1) & 1, err));
      if (ok) {
        sm100::tc_fence_after();
        const int t0 = (nchunks - 1) * C;
        const int cnt = min(C, s - t0);
#pragma unroll 1
        for (int c = 0; c < C; c += 32) {
          float o[32];
          sm100::tmem_ld32(tmem + lane_off + O_COL + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i)  // constant indices: o stays in registers
            if (c + i < cnt) out[(((int64_t)bi * s + t0 + c + i) * nv + h) * 128 + r] = __float2bfloat16(o[i]);
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, tcs::TMEM_COLS);
  }
}

}  // namespace gdn

template <int D>
static void gdn_fwd_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                           const at::Tensor& beta, int groups, at::Tensor& out) {
  using namespace gdn;
  constexpr int DVS = D >= 32 ? 32 : D;
  const int b = q.size(0), s = q.size(1), nk = q.size(2), nv = v.size(2);
  const int nchunks = (s + C - 1) / C;
  const int64_t nck = (int64_t)b * nv * nchunks;
  auto f32 = q.options().dtype(at::kFloat);
  at::Tensor GL = at::empty({nck}, f32);
  at::Tensor U = at::empty({nck * C * D}, f32);
  at::Tensor Qg = at::empty({nck * D * C}, q.options());
  at::Tensor Kd = at::empty({nck * C * D}, q.options());
  const auto* bq = reinterpret_cast<const bf16*>(q.data_ptr());
  const auto* bk = reinterpret_cast<const bf16*>(k.data_ptr());
  const auto* bv = reinterpret_cast<const bf16*>(v.data_ptr());
  const auto* bb = reinterpret_cast<const bf16*>(beta.data_ptr());
  if constexpr (D == 128) {
    // tensor-core state recurrence: bf16 K-major operand tiles
    at::Tensor W = at::empty({nck * C * D}, q.options());
    at::Tensor A = at::empty({nck * C * C}, q.options());
    static std::atomic<unsigned long long> attr{0};
    once_per_device(attr, [&] {
      NS_CUDA(cudaFuncSetAttribute(gdn_prep_kernel<D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Prep<D>::BYTES));
      NS_CUDA(cudaFuncSetAttribute(gdn_state_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tcs::SMEM));
    });
    gdn_prep_kernel<D, true><<<dim3(nchunks, nv, b), NT, Prep<D>::BYTES, stream()>>>(
        bq, bk, bv, q.stride(1), k.stride(1), v.stride(1), g.data_ptr<float>(), bb, s, nk, nv, groups, nchunks, W.data_ptr(),
        reinterpret_cast<bf16*>(Qg.data_ptr()), reinterpret_cast<bf16*>(Kd.data_ptr()), A.data_ptr(),
        U.data_ptr<float>(), GL.data_ptr<float>(), DVS);
    NS_CUDA(cudaGetLastError());
    const int64_t rows = nck * C;
    CUtensorMap tw = make_tmap_bf16(W.data_ptr(), rows, D, D, C, 64);
    CUtensorMap tq = make_tmap_bf16(Qg.data_ptr(), rows, D, D, C, 64);
    CUtensorMap ta = make_tmap_bf16(A.data_ptr(), rows, C, C, C, 64);
    CUtensorMap tk = make_tmap_bf16(Kd.data_ptr(), nck * D, C, C, 128, 64);
    gdn_state_tc_kernel<<<dim3(nv, b), 192, tcs::SMEM, stream()>>>(tw, tq, ta, tk, U.data_ptr<float>(),
                                                                    GL.data_ptr<float>(),
                                                                    reinterpret_cast<bf16*>(out.data_ptr()), s, nv,
                                                                    nchunks, device_error_flag());
    NS_CUDA(cudaGetLastError());
  } else {
    at::Tensor WT = at::empty({nck * D * C}, f32);
    at::Tensor AqkT = at::empty({nck * C * C}, f32);
    static std::atomic<unsigned long long> attr{0};
    once_per_device(attr, [&] {
      NS_CUDA(cudaFuncSetAttribute(gdn_prep_kernel<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Prep<D>::BYTES));
      NS_CUDA(cudaFuncSetAttribute(gdn_state_kernel<D, DVS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   State<D, DVS>::BYTES));
    });
    gdn_prep_kernel<D, false><<<dim3(nchunks, nv, b), NT, Prep<D>::BYTES, stream()>>>(
        bq, bk, bv, q.stride(1), k.stride(1), v.stride(1), g.data_ptr<float>(), bb, s, nk, nv, groups, nchunks, WT.data_ptr(),
        reinterpret_cast<bf16*>(Qg.data_ptr()), reinterpret_cast<bf16*>(Kd.data_ptr()), AqkT.data_ptr(),
        U.data_ptr<float>(), GL.data_ptr<float>(), DVS);
    NS_CUDA(cudaGetLastError());
    gdn_state_kernel<D, DVS><<<dim3(D / DVS, nv, b), NT, State<D, DVS>::BYTES, stream()>>>(
        WT.data_ptr<float>(), reinterpret_cast<const bf16*>(Qg.data_ptr()),
        reinterpret_cast<const bf16*>(Kd.data_ptr()), AqkT.data_ptr<float>(), U.data_ptr<float>(),
        GL.data_ptr<float>(), reinterpret_cast<bf16*>(out.data_ptr()), s, nv, nchunks, device_error_flag());
    NS_CUDA(cudaGetLastError());
  }
}

void gdn_chunk_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta, int64_t groups,
                   at::Tensor out) {
  NS_CHECK(q.size(3) == v.size(3), "gated delta rule kernel needs d_k == d_v");
  NS_CHECK(g.scalar_type() == at::kFloat, "g must be fp32");
  NS_CHECK(g.is_contiguous() && beta.is_contiguous() && out.is_contiguous(), "g, beta and out must be contiguous");
  // q / k / v: [b, s, heads, D] views with contiguous heads and one token stride (rows of
  // a fused projection are fine); 8-byte aligned rows for the 4-channel loads
  for (const at::Tensor* t : {&q, &k, &v}) {
    NS_CHECK(t->stride(3) == 1 && t->stride(2) == t->size(3) && t->stride(0) == t->size(1) * t->stride(1),
             "gated delta rule: q / k / v must be [b, s, heads, D] rows with one token stride");
    NS_CHECK(t->stride(1) % 4 == 0 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 8 == 0,
             "gated delta rule: 8-byte aligned rows");
  }
  if (q.size(1) == 0) return;
  switch (q.size(3)) {
    case 16: gdn_fwd_launch<16>(q, k, v, g, beta, (int)groups, out); break;
    case 32: gdn_fwd_launch<32>(q, k, v, g, beta, (int)groups, out); break;
    case 64: gdn_fwd_launch<64>(q, k, v, g, beta, (int)groups, out); break;
    case 128: gdn_fwd_launch<128>(q, k, v, g, beta, (int)groups, out); break;
    default: NS_CHECK(false, "gated delta rule head dim must be 16, 32, 64 or 128");
  }
}

}  // namespace ns
