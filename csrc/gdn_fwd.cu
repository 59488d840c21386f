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
// 4096 tokens). Only the state recurrence is sequential; it is split across value
// columns (columns of S are independent), so `gdn_state_kernel` runs
// (d_v / 32) x heads x rows CTAs, two per SM, each walking the chunks with its slice
// of S in shared memory. The prep kernel hands over, per chunk and head, W^T, U
// (slice-major), A^T, (q e^G)^T, k e^{G_last - G} and e^{G_last}; the state kernel
// fetches them with bulk copies (cp.async.bulk, this GPU's memory only) completing on
// an mbarrier with a bounded wait.
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
constexpr int CP = C + 4;   // padded row length of [D][C] tiles in shared memory
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
  static constexpr int DP = D + 4;                                   // padded row of [C][D] tiles
  static constexpr int KT = D * CP;                                  // k^T
  static constexpr int QX = (D * CP > C * DP) ? D * CP : C * DP;     // q^T, later beta k e^G
  static constexpr int XV = C * DP;                                  // v, then beta v
  static constexpr int MS = C * (C + 1);
  static constexpr int PS = 3 * 16 * 17;
  static constexpr int FLOATS = KT + QX + XV + 2 * MS + PS + 4 * C;
  static constexpr int BYTES = FLOATS * 4;
};

template <int D>
__global__ void __launch_bounds__(NT) gdn_prep_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                      const bf16* __restrict__ v, const float* __restrict__ gin,
                                                      const bf16* __restrict__ beta_in, int s, int nk, int nv,
                                                      int groups, int nchunks, float* __restrict__ WT,
                                                      bf16* __restrict__ QgT, bf16* __restrict__ Kd,
                                                      float* __restrict__ AqkT, float* __restrict__ Uo,
                                                      float* __restrict__ GL, int dvs) {
  using L = Prep<D>;
  constexpr int DP = L::DP;
  extern __shared__ __align__(16) float sm[];
  float* kT = sm;
  float* qT = kT + L::KT;  // later Xk
  float* Xv = qT + L::QX;
  float* Ms = Xv + L::XV;
  float* Ts = Ms + L::MS;
  float* Ps = Ts + L::MS;
  float* G = Ps + L::PS;
  float* Bt = G + C;
  float* eG = Bt + C;
  float* eGl = eG + C;
  const int ch = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int hk = h / groups;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = ch * C, cnt = min(C, s - t0);
  const float scale = rsqrtf((float)D);
  const int64_t ck = ((int64_t)bi * nv + h) * nchunks + ch;

  // 1. load; q and k L2-normalised as the bf16 statement computes them
  for (int r = warp; r < C; r += NT / 32) {
    const bool in = r < cnt;
    const int64_t tq = (int64_t)bi * s + t0 + r;
    float sq = 0.f, sk = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float a = in ? bf(q[(tq * nk + hk) * D + d]) : 0.f;
      const float b = in ? bf(k[(tq * nk + hk) * D + d]) : 0.f;
      sq += rb(a * a);
      sk += rb(b * b);
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float iq = rb(rsqrtf(rb(rb(sq) + 1e-6f)));
    const float ik = rb(rsqrtf(rb(rb(sk) + 1e-6f)));
    for (int d = lane; d < D; d += 32) {
      const float a = in ? bf(q[(tq * nk + hk) * D + d]) : 0.f;
      const float b = in ? bf(k[(tq * nk + hk) * D + d]) : 0.f;
      qT[d * CP + r] = rb(a * iq);
      kT[d * CP + r] = rb(b * ik);
      Xv[r * DP + d] = in ? bf(v[(tq * nv + h) * D + d]) : 0.f;
    }
    if (lane == 0) {
      G[r] = in ? gin[tq * nv + h] : 0.f;
      Bt[r] = in ? bf(beta_in[tq * nv + h]) : 0.f;
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
  }
  __syncthreads();

  // 2. M = strict_lower(beta_i k_i.k_j e^{G_i-G_j}) and A = lower(scale q_i.k_j e^{G_i-G_j});
  //    each thread a 4 x 4 block of both. A goes to global memory transposed.
  {
    const int i0 = (tid >> 4) * 4, j0 = (tid & 15) * 4;
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) kk[r][c] = qk[r][c] = 0.f;
    if (j0 <= i0 + 3) {
#pragma unroll 4
      for (int d = 0; d < D; ++d) {
        const float4 ki = *reinterpret_cast<const float4*>(&kT[d * CP + i0]);
        const float4 qi = *reinterpret_cast<const float4*>(&qT[d * CP + i0]);
        const float4 kj = *reinterpret_cast<const float4*>(&kT[d * CP + j0]);
        const float kiv[4] = {ki.x, ki.y, ki.z, ki.w}, qiv[4] = {qi.x, qi.y, qi.z, qi.w};
        const float kjv[4] = {kj.x, kj.y, kj.z, kj.w};
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            kk[r][c] = fmaf(kiv[r], kjv[c], kk[r][c]);
            qk[r][c] = fmaf(qiv[r], kjv[c], qk[r][c]);
          }
      }
    }
    float* at = AqkT + ck * C * C;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = j0 + c;
      float a4[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = i0 + r;
        const float dec = j <= i ? expf(G[i] - G[j]) : 0.f;
        Ms[i * (C + 1) + j] = j < i ? Bt[i] * kk[r][c] * dec : 0.f;
        a4[r] = j <= i ? scale * qk[r][c] * dec : 0.f;
      }
      *reinterpret_cast<float4*>(&at[j * C + i0]) = make_float4(a4[0], a4[1], a4[2], a4[3]);
    }
  }
  __syncthreads();
  // (q scale e^G)^T and k e^{G_last - G} for the state kernel (bf16)
  {
    bf16* qg = QgT + ck * D * C;
    bf16* kd = Kd + ck * C * D;
    for (int idx = tid; idx < D * C; idx += NT) {
      const int d = idx / C, i = idx % C;
      qg[idx] = __float2bfloat16(qT[d * CP + i] * scale * eG[i]);
    }
    for (int idx = tid; idx < C * D; idx += NT) {
      const int i = idx / D, d = idx % D;
      kd[idx] = __float2bfloat16(kT[d * CP + i] * eGl[i]);
    }
    if (tid == 0) GL[ck] = expf(Gl);
  }
  __syncthreads();
  float* Xk = qT;
  for (int idx = tid; idx < C * D; idx += NT) {
    const int i = idx / D, d = idx % D;
    Xk[i * DP + d] = Bt[i] * kT[d * CP + i] * eG[i];
    Xv[i * DP + d] *= Bt[i];
  }

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

  // 4. W = T (beta k e^G), U = T (beta v); W stored transposed, U slice-major
  {
    constexpr int EG = D / 4, IG = NT / EG, RPT = C / IG;
    const int eg = tid % EG, i0 = (tid / EG) * RPT, e0 = eg * 4;
    float w[RPT][4], u[RPT][4];
#pragma unroll
    for (int r = 0; r < RPT; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) w[r][c] = u[r][c] = 0.f;
    for (int j = 0; j < i0 + RPT; ++j) {
      const float4 xk = *reinterpret_cast<const float4*>(&Xk[j * DP + e0]);
      const float4 xv = *reinterpret_cast<const float4*>(&Xv[j * DP + e0]);
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const float t = Ts[(i0 + r) * (C + 1) + j];
        w[r][0] = fmaf(t, xk.x, w[r][0]);
        w[r][1] = fmaf(t, xk.y, w[r][1]);
        w[r][2] = fmaf(t, xk.z, w[r][2]);
        w[r][3] = fmaf(t, xk.w, w[r][3]);
        u[r][0] = fmaf(t, xv.x, u[r][0]);
        u[r][1] = fmaf(t, xv.y, u[r][1]);
        u[r][2] = fmaf(t, xv.z, u[r][2]);
        u[r][3] = fmaf(t, xv.w, u[r][3]);
      }
    }
    float* wt = WT + ck * D * C;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int r = 0; r < RPT; ++r) wt[(e0 + c) * C + i0 + r] = w[r][c];
    const int slice = e0 / dvs, el = e0 % dvs;
    float* uo = Uo + (ck * (D / dvs) + slice) * C * dvs;
#pragma unroll
    for (int r = 0; r < RPT; ++r)
      *reinterpret_cast<float4*>(&uo[(i0 + r) * dvs + el]) = make_float4(u[r][0], u[r][1], u[r][2], u[r][3]);
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
  at::Tensor WT = at::empty({nck * D * C}, f32);
  at::Tensor AqkT = at::empty({nck * C * C}, f32);
  at::Tensor U = at::empty({nck * C * D}, f32);
  at::Tensor GL = at::empty({nck}, f32);
  at::Tensor QgT = at::empty({nck * D * C}, q.options());
  at::Tensor Kd = at::empty({nck * C * D}, q.options());
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(gdn_prep_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Prep<D>::BYTES));
    NS_CUDA(cudaFuncSetAttribute(gdn_state_kernel<D, DVS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 State<D, DVS>::BYTES));
  });
  const auto* bq = reinterpret_cast<const bf16*>(q.data_ptr());
  gdn_prep_kernel<D><<<dim3(nchunks, nv, b), NT, Prep<D>::BYTES, stream()>>>(
      bq, reinterpret_cast<const bf16*>(k.data_ptr()), reinterpret_cast<const bf16*>(v.data_ptr()),
      g.data_ptr<float>(), reinterpret_cast<const bf16*>(beta.data_ptr()), s, nk, nv, groups, nchunks,
      WT.data_ptr<float>(), reinterpret_cast<bf16*>(QgT.data_ptr()), reinterpret_cast<bf16*>(Kd.data_ptr()),
      AqkT.data_ptr<float>(), U.data_ptr<float>(), GL.data_ptr<float>(), DVS);
  NS_CUDA(cudaGetLastError());
  gdn_state_kernel<D, DVS><<<dim3(D / DVS, nv, b), NT, State<D, DVS>::BYTES, stream()>>>(
      WT.data_ptr<float>(), reinterpret_cast<const bf16*>(QgT.data_ptr()), reinterpret_cast<const bf16*>(Kd.data_ptr()),
      AqkT.data_ptr<float>(), U.data_ptr<float>(), GL.data_ptr<float>(), reinterpret_cast<bf16*>(out.data_ptr()),
      s, nv, nchunks, device_error_flag());
  NS_CUDA(cudaGetLastError());
}

void gdn_chunk_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta, int64_t groups,
                   at::Tensor out) {
  NS_CHECK(q.size(3) == v.size(3), "gated delta rule kernel needs d_k == d_v");
  NS_CHECK(g.scalar_type() == at::kFloat, "g must be fp32");
  NS_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && g.is_contiguous() && beta.is_contiguous() &&
               out.is_contiguous(),
           "gated delta rule inputs must be contiguous");
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
