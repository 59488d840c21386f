// Chunked backward of the gated delta rule (head dims 64 and 128), fp32 throughout.
//
// Per (row, value head, chunk of C = 64 tokens), with q, k L2-normalised (q scaled
// by D^-1/2), G the in-chunk cumulative log decay, gam = e^G, Gam(t, i) = e^{G_t - G_i}
// (i <= t), M = strict(beta_t k_t.k_i Gam), T = I + M:
//   U = T^-1 (beta v), W = T^-1 (beta gam k), A = incl(q k^T Gam), Kh = e^{G_C - G} k,
//   VN = U - W S0, O = gam q S0 + A VN, S1 = e^{G_C} S0 + Kh^T VN.
// The states entering the chunks (S0) and the gradients of the states leaving them
// (dS1) obey one linear recurrence per chunk with F = e^{G_C} I - Kh^T W:
//   S1 = F S0 + Kh^T U  (forward),   dS0 = F^T dS1 + P,  P = (gam q)^T dO - W^T A^T dO.
// Kernels (each chunk-parallel except the scan, which is parallel over value columns):
//   gdnb_setup   : normalisation, decay, M, T^-1 (forward substitution), A, U, W; F, H, P
//   gdnb_scan    : S0 per chunk (forward), dS1 per chunk (reverse), D/4 columns per CTA
//   gdnb_grad1   : VN, dVN, and the dQ / dK / dG terms through gam q S0 and Kh
//   gdnb_grad2a  : the terms through A (dA = incl(dO VN^T))
//   gdnb_grad2b  : dW, dBk = T^-T dW, dBv = T^-T dVN, dM; the terms through M and the
//                  WY products; dv, dbeta, dg (reverse cumulative sum), and the
//                  L2-normalisation chain rule into the raw q and k
// The statements these kernels implement, and their check against autograd through
// the token recurrence, are ``gated_delta_rule_backward_chunked`` in the package's
// reference ops. Chunk-local matrices pass between kernels through a workspace in
// global memory (about 770 KB per chunk at D = 128; S0 and dS1 are also kept
// transposed, so every product reads them along rows).
#include "common.h"
#include "sm100.cuh"

namespace ns {
namespace gdnb {

using bf16 = __nv_bfloat16;
constexpr int C = 64;     // chunk length
constexpr int NT = 256;   // threads per CTA
constexpr int PC = C + 1; // padded row stride of C x C tiles in shared memory

__device__ __forceinline__ float bfv(bf16 x) { return __bfloat162float(x); }

// out[r * os + n] (=, or += when acc) alpha * sum_k A(r, k) B(k, n) for an R x N
// output with 256 threads; A(r, k) = A[r * ars + k * aks], B(k, n) = B[k * bks + n * bns].
// A and B may live in shared or global memory. Thread (tr, tn) owns rows
// tr*TR .. tr*TR+TR-1 and columns tn, tn + N/TN, ... (consecutive threads, consecutive
// columns).
template <int R, int N, int TR, int TN>
__device__ __forceinline__ void mm(float* out, int os, const float* A, int ars, int aks, const float* B, int bks,
                                   int bns, int K, float alpha, bool acc) {
  constexpr int NTH = N / TN;
  static_assert((R / TR) * NTH == NT, "256 threads");
  const int tid = threadIdx.x;
  const int r0 = (tid / NTH) * TR, tn = tid % NTH;
  float c[TR][TN];
#pragma unroll
  for (int i = 0; i < TR; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) c[i][j] = 0.f;
  // K is a multiple of 8 at every call: unrolling keeps eight iterations' loads in
  // flight (the B operand of several products streams from global memory)
#pragma unroll 8
  for (int k = 0; k < K; ++k) {
    float a[TR], b[TN];
#pragma unroll
    for (int i = 0; i < TR; ++i) a[i] = A[(r0 + i) * ars + k * aks];
#pragma unroll
    for (int j = 0; j < TN; ++j) b[j] = B[k * bks + (tn + j * NTH) * bns];
#pragma unroll
    for (int i = 0; i < TR; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) c[i][j] = fmaf(a[i], b[j], c[i][j]);
  }
#pragma unroll
  for (int i = 0; i < TR; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      float* o = out + (r0 + i) * os + tn + j * NTH;
      *o = (acc ? *o : 0.f) + alpha * c[i][j];
    }
}

// Tile shapes for the three output sizes of one chunk: C x C, C x D, D x D (and the
// scan's D x D/4 column block).
template <int D>
struct Shapes {
  static constexpr int PD = D + 1;  // padded row stride of C x D tiles
  static constexpr int CD_TR = 4, CD_TN = D / 16;  // C x D: 16 x 16 threads
  static constexpr int DD_TR = D / 16, DD_TN = D / 16;
  static constexpr int JW = D / 4;  // scan column block
};

template <int D>
__device__ __forceinline__ void mm_cc(float* out, const float* A, int ars, int aks, const float* B, int bks, int bns,
                                      int K, float alpha, bool acc) {
  mm<C, C, 4, 4>(out, PC, A, ars, aks, B, bks, bns, K, alpha, acc);
}
template <int D>
__device__ __forceinline__ void mm_cd(float* out, int os, const float* A, int ars, int aks, const float* B, int bks,
                                      int bns, int K, float alpha, bool acc) {
  mm<C, D, Shapes<D>::CD_TR, Shapes<D>::CD_TN>(out, os, A, ars, aks, B, bks, bns, K, alpha, acc);
}
template <int D>
__device__ __forceinline__ void mm_dd(float* out, int os, const float* A, int ars, int aks, const float* B, int bks,
                                      int bns, int K, float alpha, bool acc) {
  mm<D, D, Shapes<D>::DD_TR, Shapes<D>::DD_TN>(out, os, A, ars, aks, B, bks, bns, K, alpha, acc);
}

// Copies between a shared C x D tile (stride PD) and a dense global one.
template <int D>
__device__ __forceinline__ void load_cd(float* s, const float* g) {
  for (int i = threadIdx.x; i < C * D; i += NT) s[(i / D) * (D + 1) + i % D] = g[i];
}
template <int D>
__device__ __forceinline__ void store_cd(float* g, const float* s) {
  for (int i = threadIdx.x; i < C * D; i += NT) g[i] = s[(i / D) * (D + 1) + i % D];
}
__device__ __forceinline__ void load_cc(float* s, const float* g) {
  for (int i = threadIdx.x; i < C * C; i += NT) s[(i / C) * PC + i % C] = g[i];
}
__device__ __forceinline__ void store_cc(float* g, const float* s) {
  for (int i = threadIdx.x; i < C * C; i += NT) g[i] = s[(i / C) * PC + i % C];
}

// Workspace of one launch: chunk ck = (row * nv + head) * n + chunk.
struct Ws {
  float *qn, *kn, *u, *w, *vn, *dvn, *dq, *dk;  // [nck][C][D]
  float *tinv, *m, *a, *kk;                     // [nck][C][C]
  float *G, *gam, *ek, *beta, *rq, *rk, *dG;    // [nck][C]
  float *F, *H, *P, *S0, *dS1, *S0t, *dS1t;     // [nck][D][D] (t: transposed copies)
};

struct Args {
  const bf16 *q, *k, *v, *beta, *dout;  // q, k [b, s, nk, D]; v, dout [b, s, nv, D]; beta [b, s, nv]
  const float* g;                       // [b, s, nv]
  float *dq, *dk;                       // [b, s, nv, D] fp32 (per value head)
  bf16* dv;                             // [b, s, nv, D]
  float *dg, *dbeta;                    // [b, s, nv]
  int s, nk, nv, groups, n;
  Ws w;
};

// ============================================================================ setup
template <int D>
__global__ void __launch_bounds__(NT, 1) gdnb_setup(Args a) {
  constexpr int PD = D + 1;
  extern __shared__ float sm[];
  float* sQ = sm;
  float* sK = sQ + C * PD;
  float* sX = sK + C * PD;
  float* sU = sX + C * PD;
  float* sW = sU + C * PD;
  float* sM = sW + C * PD;  // KK, then M, then A
  float* sT = sM + C * PC;  // T^-1
  float* vec = sT + C * PC;  // G, gam, ek, beta: 4 x C
  float* sG = vec;
  float* sGam = vec + C;
  float* sEk = vec + 2 * C;
  float* sB = vec + 3 * C;
  const int c = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int hk = h / a.groups;
  const int64_t ck = ((int64_t)bi * a.nv + h) * a.n + c;
  const int t0 = c * C;
  const int cnt = min(C, a.s - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float scale = rsqrtf((float)D);
  // ---- normalised q, k rows (a warp per row), g and beta
  for (int r = warp; r < C; r += NT / 32) {
    float sq = 0.f, sk = 0.f;
    float qv[D / 32], kv[D / 32];
    const int64_t tok = (int64_t)bi * a.s + t0 + r;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      qv[j] = r < cnt ? bfv(a.q[(tok * a.nk + hk) * D + lane + 32 * j]) : 0.f;
      kv[j] = r < cnt ? bfv(a.k[(tok * a.nk + hk) * D + lane + 32 * j]) : 0.f;
      sq += qv[j] * qv[j];
      sk += kv[j] * kv[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
      sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    const float rq = rsqrtf(sq + 1e-6f), rk = rsqrtf(sk + 1e-6f);
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
      sQ[r * PD + lane + 32 * j] = qv[j] * rq * scale;
      sK[r * PD + lane + 32 * j] = kv[j] * rk;
    }
    if (lane == 0) {
      a.w.rq[ck * C + r] = rq;
      a.w.rk[ck * C + r] = rk;
      sG[r] = r < cnt ? a.g[((int64_t)bi * a.s + t0 + r) * a.nv + h] : 0.f;
      sB[r] = r < cnt ? bfv(a.beta[((int64_t)bi * a.s + t0 + r) * a.nv + h]) : 0.f;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int r = 0; r < C; ++r) {
      acc += sG[r];
      sG[r] = acc;
    }
  }
  __syncthreads();
  const float GC = sG[C - 1];
  if (threadIdx.x < C) {
    const int r = threadIdx.x;
    sGam[r] = expf(sG[r]);
    sEk[r] = expf(GC - sG[r]);
    a.w.G[ck * C + r] = sG[r];
    a.w.gam[ck * C + r] = sGam[r];
    a.w.ek[ck * C + r] = sEk[r];
    a.w.beta[ck * C + r] = sB[r];
  }
  store_cd<D>(a.w.qn + ck * C * D, sQ);
  store_cd<D>(a.w.kn + ck * C * D, sK);
  // ---- KK = K K^T, then M in place
  mm_cc<D>(sM, sK, PD, 1, sK, 1, PD, D, 1.f, false);
  __syncthreads();
  store_cc(a.w.kk + ck * C * C, sM);
  for (int i = threadIdx.x; i < C * C; i += NT) {
    const int t = i / C, j = i % C;
    sM[t * PC + j] = j < t ? sB[t] * sM[t * PC + j] * expf(sG[t] - sG[j]) : 0.f;
  }
  __syncthreads();
  store_cc(a.w.m + ck * C * C, sM);
  // ---- T^-1 = (I + M)^-1 by forward substitution, one column per thread
  if (threadIdx.x < C) {
    const int j = threadIdx.x;
    for (int i = 0; i < C; ++i) {
      float x = i == j ? 1.f : 0.f;
      for (int l = j; l < i; ++l) x -= sM[i * PC + l] * sT[l * PC + j];
      sT[i * PC + j] = i < j ? 0.f : x;
    }
  }
  __syncthreads();
  store_cc(a.w.tinv + ck * C * C, sT);
  // ---- A = incl(Q K^T Gam) (into sM: M is in the workspace now)
  mm_cc<D>(sM, sQ, PD, 1, sK, 1, PD, D, 1.f, false);
  __syncthreads();
  for (int i = threadIdx.x; i < C * C; i += NT) {
    const int t = i / C, j = i % C;
    sM[t * PC + j] = j <= t ? sM[t * PC + j] * expf(sG[t] - sG[j]) : 0.f;
  }
  __syncthreads();
  store_cc(a.w.a + ck * C * C, sM);
  // ---- U = T^-1 (beta v), W = T^-1 (beta gam k)
  for (int i = threadIdx.x; i < C * D; i += NT) {
    const int r = i / D, d = i % D;
    sX[r * PD + d] = r < cnt ? sB[r] * bfv(a.v[(((int64_t)bi * a.s + t0 + r) * a.nv + h) * D + d]) : 0.f;
  }
  __syncthreads();
  mm_cd<D>(sU, PD, sT, PC, 1, sX, PD, 1, C, 1.f, false);
  __syncthreads();
  for (int i = threadIdx.x; i < C * D; i += NT) {
    const int r = i / D, d = i % D;
    sX[r * PD + d] = sB[r] * sGam[r] * sK[r * PD + d];
  }
  __syncthreads();
  mm_cd<D>(sW, PD, sT, PC, 1, sX, PD, 1, C, 1.f, false);
  __syncthreads();
  store_cd<D>(a.w.u + ck * C * D, sU);
  store_cd<D>(a.w.w + ck * C * D, sW);
  // ---- scan terms: H = Kh^T U, F = e^{G_C} I - Kh^T W
  for (int i = threadIdx.x; i < C * D; i += NT) {
    const int r = i / D, d = i % D;
    sX[r * PD + d] = sEk[r] * sK[r * PD + d];
  }
  __syncthreads();
  float* F = a.w.F + ck * D * D;
  float* H = a.w.H + ck * D * D;
  float* P = a.w.P + ck * D * D;
  mm_dd<D>(H, D, sX, 1, PD, sU, PD, 1, C, 1.f, false);
  mm_dd<D>(F, D, sX, 1, PD, sW, PD, 1, C, -1.f, false);
  __syncthreads();
  const float gC = expf(GC);
  for (int i = threadIdx.x; i < D; i += NT) F[i * D + i] += gC;
  // ---- P = (gam q)^T dO - W^T (A^T dO): dO into sX, A^T dO into sU
  for (int i = threadIdx.x; i < C * D; i += NT) {
    const int r = i / D, d = i % D;
    sX[r * PD + d] = r < cnt ? bfv(a.dout[(((int64_t)bi * a.s + t0 + r) * a.nv + h) * D + d]) : 0.f;
    sQ[r * PD + d] *= sGam[r];
  }
  __syncthreads();
  mm_cd<D>(sU, PD, sM, 1, PC, sX, PD, 1, C, 1.f, false);
  __syncthreads();
  mm_dd<D>(P, D, sQ, 1, PD, sX, PD, 1, C, 1.f, false);
  __syncthreads();
  mm_dd<D>(P, D, sW, 1, PD, sU, PD, 1, C, -1.f, true);
}

// ============================================================================ scan
// grid (D / JW column blocks, heads, rows). Forward: X = S0 of chunk c, written, then
// X <- F_c X + H_c. Reverse: Y = dS1 of chunk c, written, then Y <- F_c^T Y + P_c.
template <int D>
__global__ void __launch_bounds__(NT, 1) gdnb_scan(Args a) {
  constexpr int JW = Shapes<D>::JW;
  extern __shared__ float sm[];
  constexpr int XS = JW + 1;  // padded row stride: column-wise reads are conflict-free
  float* X = sm;              // [D][XS]
  float* Xn = X + D * XS;     // [D][XS]
  const int jb = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int64_t ck0 = ((int64_t)bi * a.nv + h) * a.n;
  const int c0 = jb * JW;
  constexpr int STR = 4;                     // rows per thread
  constexpr int STN = (D * JW) / NT / STR;   // columns per thread (4 at D = 128, 1 at D = 64)
  for (int i = threadIdx.x; i < D * XS; i += NT) X[i] = 0.f;
  __syncthreads();
  for (int c = 0; c < a.n; ++c) {
    float* S0 = a.w.S0 + (ck0 + c) * D * D;
    float* S0t = a.w.S0t + (ck0 + c) * D * D;
    for (int i = threadIdx.x; i < D * JW; i += NT) {
      S0[(i / JW) * D + c0 + i % JW] = X[(i / JW) * XS + i % JW];
      S0t[(c0 + i / D) * D + i % D] = X[(i % D) * XS + i / D];
    }
    if (c + 1 < a.n) {
      const float* F = a.w.F + (ck0 + c) * D * D;
      const float* H = a.w.H + (ck0 + c) * D * D;
      mm<D, JW, STR, STN>(Xn, XS, F, D, 1, X, XS, 1, D, 1.f, false);
      __syncthreads();
      for (int i = threadIdx.x; i < D * JW; i += NT)
        X[(i / JW) * XS + i % JW] = Xn[(i / JW) * XS + i % JW] + H[(i / JW) * D + c0 + i % JW];
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < D * XS; i += NT) X[i] = 0.f;
  __syncthreads();
  for (int c = a.n - 1; c >= 0; --c) {
    float* dS1 = a.w.dS1 + (ck0 + c) * D * D;
    float* dS1t = a.w.dS1t + (ck0 + c) * D * D;
    for (int i = threadIdx.x; i < D * JW; i += NT) {
      dS1[(i / JW) * D + c0 + i % JW] = X[(i / JW) * XS + i % JW];
      dS1t[(c0 + i / D) * D + i % D] = X[(i % D) * XS + i / D];
    }
    if (c > 0) {
      const float* F = a.w.F + (ck0 + c) * D * D;
      const float* P = a.w.P + (ck0 + c) * D * D;
      mm<D, JW, STR, STN>(Xn, XS, F, 1, D, X, XS, 1, D, 1.f, false);  // F^T X
      __syncthreads();
      for (int i = threadIdx.x; i < D * JW; i += NT)
        X[(i / JW) * XS + i % JW] = Xn[(i / JW) * XS + i % JW] + P[(i / JW) * D + c0 + i % JW];
      __syncthreads();
    }
  }
}

// ============================================================================ grad 1
// VN = U - W S0; dVN = A^T dO + Kh dS1; dQ = gam (dO S0^T), dG += gam q.(dO S0^T);
// dK = ek (VN dS1^T), dG -= ek k.(VN dS1^T); dG[C-1] += sum of those + e^{G_C} <S0, dS1>.
template <int D>
__global__ void __launch_bounds__(NT, 1) gdnb_grad1(Args a) {
  constexpr int PD = D + 1;
  extern __shared__ float sm[];
  float* sO = sm;            // dO
  float* sVN = sO + C * PD;
  float* sDVN = sVN + C * PD;
  float* sKh = sDVN + C * PD;
  float* sW = sKh + C * PD;
  float* sX = sW + C * PD;
  float* sA = sX + C * PD;   // [C][PC]
  float* red = sA + C * PC;  // [NT / 32 + C]
  float* dG = red + NT / 32;
  const int c = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int64_t ck = ((int64_t)bi * a.nv + h) * a.n + c;
  const int t0 = c * C;
  const int cnt = min(C, a.s - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* S0 = a.w.S0 + ck * D * D;
  const float* dS1 = a.w.dS1 + ck * D * D;
  const float* S0t = a.w.S0t + ck * D * D;
  const float* dS1t = a.w.dS1t + ck * D * D;
  const float* gam = a.w.gam + ck * C;
  const float* ek = a.w.ek + ck * C;
  for (int i = threadIdx.x; i < C * D; i += NT) {
    const int r = i / D, d = i % D;
    sO[r * PD + d] = r < cnt ? bfv(a.dout[(((int64_t)bi * a.s + t0 + r) * a.nv + h) * D + d]) : 0.f;
    sKh[r * PD + d] = ek[r] * a.w.kn[ck * C * D + i];
  }
  load_cd<D>(sVN, a.w.u + ck * C * D);
  load_cd<D>(sW, a.w.w + ck * C * D);
  load_cc(sA, a.w.a + ck * C * C);
  if (threadIdx.x < C) dG[threadIdx.x] = 0.f;
  __syncthreads();
  mm_cd<D>(sVN, PD, sW, PD, 1, S0, D, 1, D, -1.f, true);     // VN = U - W S0
  mm_cd<D>(sDVN, PD, sA, 1, PC, sO, PD, 1, C, 1.f, false);   // A^T dO
  __syncthreads();
  mm_cd<D>(sDVN, PD, sKh, PD, 1, dS1, D, 1, D, 1.f, true);   // + Kh dS1
  mm_cd<D>(sX, PD, sO, PD, 1, S0t, D, 1, D, 1.f, false);     // dQg = dO S0^T
  __syncthreads();
  store_cd<D>(a.w.vn + ck * C * D, sVN);
  store_cd<D>(a.w.dvn + ck * C * D, sDVN);
  // dQ = gam dQg, dG += gam q.dQg (a warp per row)
  for (int r = warp; r < C; r += NT / 32) {
    float dot = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float x = sX[r * PD + d];
      dot += a.w.qn[(ck * C + r) * D + d] * x;
      a.w.dq[(ck * C + r) * D + d] = gam[r] * x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) dG[r] += gam[r] * dot;
  }
  __syncthreads();
  mm_cd<D>(sX, PD, sVN, PD, 1, dS1t, D, 1, D, 1.f, false);   // dKh = VN dS1^T
  __syncthreads();
  float tsum = 0.f;  // per warp: sum over its rows of ek k.dKh
  for (int r = warp; r < C; r += NT / 32) {
    float dot = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float x = sX[r * PD + d];
      dot += a.w.kn[(ck * C + r) * D + d] * x;
      a.w.dk[(ck * C + r) * D + d] = ek[r] * x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) {
      dG[r] -= ek[r] * dot;
      tsum += ek[r] * dot;
    }
  }
  // d/dG_C: sum_t ek_t k_t.dKh_t (tsum, lane 0 of each warp) + e^{G_C} <S0, dS1>
  float sd = 0.f;
  for (int i = threadIdx.x; i < D * D; i += NT) sd += S0[i] * dS1[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
  if (lane == 0) red[warp] = gam[C - 1] * sd + tsum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < NT / 32; ++w) s += red[w];
    dG[C - 1] += s;
  }
  __syncthreads();
  if (threadIdx.x < C) a.w.dG[ck * C + threadIdx.x] = dG[threadIdx.x];
}

// ============================================================================ grad 2a
// dA = incl(dO VN^T); dG += rowsum(dA A) - colsum(dA A); Fq = dA Gam;
// dQ += Fq K; dK += Fq^T Q.
template <int D>
__global__ void __launch_bounds__(NT, 1) gdnb_grad2a(Args a) {
  constexpr int PD = D + 1;
  extern __shared__ float sm[];
  float* s1 = sm;             // dO, then K
  float* s2 = s1 + C * PD;    // VN, then Q
  float* sdQ = s2 + C * PD;
  float* sdK = sdQ + C * PD;
  float* sdA = sdK + C * PD;  // [C][PC]
  float* sA = sdA + C * PC;   // [C][PC]
  float* sG = sA + C * PC;    // [C]
  const int c = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int64_t ck = ((int64_t)bi * a.nv + h) * a.n + c;
  const int t0 = c * C;
  const int cnt = min(C, a.s - t0);
  for (int i = threadIdx.x; i < C * D; i += NT) {
    const int r = i / D, d = i % D;
    s1[r * PD + d] = r < cnt ? bfv(a.dout[(((int64_t)bi * a.s + t0 + r) * a.nv + h) * D + d]) : 0.f;
  }
  load_cd<D>(s2, a.w.vn + ck * C * D);
  load_cd<D>(sdQ, a.w.dq + ck * C * D);
  load_cd<D>(sdK, a.w.dk + ck * C * D);
  load_cc(sA, a.w.a + ck * C * C);
  if (threadIdx.x < C) sG[threadIdx.x] = a.w.G[ck * C + threadIdx.x];
  __syncthreads();
  mm_cc<D>(sdA, s1, PD, 1, s2, 1, PD, D, 1.f, false);  // dO VN^T
  __syncthreads();
  // mask, dG terms through A, then Fq = dA Gam in place
  if (threadIdx.x < C) {
    const int t = threadIdx.x;
    float row = 0.f, col = 0.f;
    for (int j = 0; j <= t; ++j) row += sdA[t * PC + j] * sA[t * PC + j];
    for (int i = t; i < C; ++i) col += sdA[i * PC + t] * sA[i * PC + t];
    a.w.dG[ck * C + t] += row - col;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < C * C; i += NT) {
    const int t = i / C, j = i % C;
    sdA[t * PC + j] = j <= t ? sdA[t * PC + j] * expf(sG[t] - sG[j]) : 0.f;
  }
  load_cd<D>(s1, a.w.kn + ck * C * D);
  load_cd<D>(s2, a.w.qn + ck * C * D);
  __syncthreads();
  mm_cd<D>(sdQ, PD, sdA, PC, 1, s1, PD, 1, C, 1.f, true);  // dQ += Fq K
  mm_cd<D>(sdK, PD, sdA, 1, PC, s2, PD, 1, C, 1.f, true);  // dK += Fq^T Q
  __syncthreads();
  store_cd<D>(a.w.dq + ck * C * D, sdQ);
  store_cd<D>(a.w.dk + ck * C * D, sdK);
}

// ============================================================================ grad 2b
template <int D>
__global__ void __launch_bounds__(NT, 1) gdnb_grad2b(Args a) {
  constexpr int PD = D + 1;
  extern __shared__ float sm[];
  float* s1 = sm;             // dVN, then U, then K
  float* s2 = s1 + C * PD;    // dW, then W, then dK
  float* sBk = s2 + C * PD;
  float* sBv = sBk + C * PD;
  float* sT = sBv + C * PD;   // T^-1, then dM, then E' = beta E
  float* sM = sT + C * PC;
  float* vec = sM + C * PC;
  float* sG = vec;            // [C]
  float* sBeta = vec + C;
  float* sGam = vec + 2 * C;
  float* sdG = vec + 3 * C;
  float* sdB = vec + 4 * C;
  const int c = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int64_t ck = ((int64_t)bi * a.nv + h) * a.n + c;
  const int t0 = c * C;
  const int cnt = min(C, a.s - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* S0t = a.w.S0t + ck * D * D;
  load_cd<D>(s1, a.w.dvn + ck * C * D);
  load_cc(sT, a.w.tinv + ck * C * C);
  if (threadIdx.x < C) {
    const int t = threadIdx.x;
    sG[t] = a.w.G[ck * C + t];
    sBeta[t] = a.w.beta[ck * C + t];
    sGam[t] = a.w.gam[ck * C + t];
    sdG[t] = a.w.dG[ck * C + t];
    sdB[t] = 0.f;
  }
  __syncthreads();
  mm_cd<D>(s2, PD, s1, PD, 1, S0t, D, 1, D, -1.f, false);  // dW = -dVN S0^T
  __syncthreads();
  mm_cd<D>(sBk, PD, sT, 1, PC, s2, PD, 1, C, 1.f, false);  // dBk = T^-T dW
  mm_cd<D>(sBv, PD, sT, 1, PC, s1, PD, 1, C, 1.f, false);  // dBv = T^-T dVN
  __syncthreads();
  load_cd<D>(s1, a.w.u + ck * C * D);
  load_cd<D>(s2, a.w.w + ck * C * D);
  load_cc(sM, a.w.m + ck * C * C);
  __syncthreads();
  mm_cc<D>(sT, sBv, PD, 1, s1, 1, PD, D, -1.f, false);  // dM = -(dBv U^T
  __syncthreads();
  mm_cc<D>(sT, sBk, PD, 1, s2, 1, PD, D, -1.f, true);   //        + dBk W^T)
  __syncthreads();
  // strict mask; dG terms through M; dbeta through E = dM Gam and KK; E' = beta E
  for (int i = threadIdx.x; i < C * C; i += NT) {
    const int t = i / C, j = i % C;
    if (j >= t) sT[t * PC + j] = 0.f;
  }
  __syncthreads();
  if (threadIdx.x < C) {
    const int t = threadIdx.x;
    float row = 0.f, col = 0.f, eb = 0.f;
    for (int j = 0; j < t; ++j) {
      row += sT[t * PC + j] * sM[t * PC + j];
      eb += sT[t * PC + j] * expf(sG[t] - sG[j]) * a.w.kk[(ck * C + t) * C + j];
    }
    for (int i = t + 1; i < C; ++i) col += sT[i * PC + t] * sM[i * PC + t];
    sdG[t] += row - col;
    sdB[t] += eb;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < C * C; i += NT) {
    const int t = i / C, j = i % C;
    sT[t * PC + j] = j < t ? sBeta[t] * sT[t * PC + j] * expf(sG[t] - sG[j]) : 0.f;
  }
  load_cd<D>(s1, a.w.kn + ck * C * D);
  load_cd<D>(s2, a.w.dk + ck * C * D);
  __syncthreads();
  mm_cd<D>(s2, PD, sT, PC, 1, s1, PD, 1, C, 1.f, true);  // dK += E' K
  __syncthreads();
  mm_cd<D>(s2, PD, sT, 1, PC, s1, PD, 1, C, 1.f, true);  // dK += E'^T K
  __syncthreads();
  // terms through U = T^-1 (beta v) and W = T^-1 (beta gam k); dv (a warp per row)
  for (int r = warp; r < C; r += NT / 32) {
    float vdot = 0.f, kdot = 0.f;
    const int64_t row = ((int64_t)bi * a.s + t0 + r) * a.nv + h;
    for (int d = lane; d < D; d += 32) {
      const float bv = sBv[r * PD + d], bk = sBk[r * PD + d];
      const float vv = r < cnt ? bfv(a.v[row * D + d]) : 0.f;
      vdot += bv * vv;
      kdot += bk * s1[r * PD + d];
      s2[r * PD + d] += sBeta[r] * sGam[r] * bk;
      if (r < cnt) a.dv[row * D + d] = __float2bfloat16(sBeta[r] * bv);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      vdot += __shfl_xor_sync(0xffffffffu, vdot, o);
      kdot += __shfl_xor_sync(0xffffffffu, kdot, o);
    }
    if (lane == 0) {
      sdB[r] += vdot + sGam[r] * kdot;
      sdG[r] += sBeta[r] * sGam[r] * kdot;
    }
  }
  __syncthreads();
  // dg = reverse cumulative sum of dG over the chunk; dbeta
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int r = C - 1; r >= 0; --r) {
      acc += sdG[r];
      sdG[r] = acc;
    }
  }
  __syncthreads();
  if (threadIdx.x < cnt) {
    const int r = threadIdx.x;
    const int64_t row = ((int64_t)bi * a.s + t0 + r) * a.nv + h;
    a.dg[row] = sdG[r];
    a.dbeta[row] = sdB[r];
  }
  // L2-normalisation chain rule: dx = r (dy - y (y.dy)), y the normalised row
  const float scale = rsqrtf((float)D);
  for (int r = warp; r < cnt; r += NT / 32) {
    const int64_t row = ((int64_t)bi * a.s + t0 + r) * a.nv + h;
    const float rk = a.w.rk[ck * C + r], rq = a.w.rq[ck * C + r];
    float kd = 0.f, qd = 0.f;
    for (int d = lane; d < D; d += 32) {
      kd += s1[r * PD + d] * s2[r * PD + d];
      qd += (a.w.qn[(ck * C + r) * D + d] / scale) * (a.w.dq[(ck * C + r) * D + d] * scale);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      kd += __shfl_xor_sync(0xffffffffu, kd, o);
      qd += __shfl_xor_sync(0xffffffffu, qd, o);
    }
    for (int d = lane; d < D; d += 32) {
      a.dk[row * D + d] = rk * (s2[r * PD + d] - s1[r * PD + d] * kd);
      const float y = a.w.qn[(ck * C + r) * D + d] / scale;
      a.dq[row * D + d] = rq * (a.w.dq[(ck * C + r) * D + d] * scale - y * qd);
    }
  }
}

}  // namespace gdnb

// ============================================================================ host
namespace gdnb {

template <int D>
static void run(Args a, int b) {
  constexpr int PD = D + 1;
  const int smem_setup = (5 * C * PD + 2 * C * PC + 4 * C) * 4;
  const int smem_scan = 2 * D * (Shapes<D>::JW + 1) * 4;
  const int smem_g1 = (6 * C * PD + C * PC + NT / 32 + C) * 4;
  const int smem_g2a = (4 * C * PD + 2 * C * PC + C) * 4;
  const int smem_g2b = (4 * C * PD + 2 * C * PC + 5 * C) * 4;
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(gdnb_setup<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_setup));
    NS_CUDA(cudaFuncSetAttribute(gdnb_scan<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_scan));
    NS_CUDA(cudaFuncSetAttribute(gdnb_grad1<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_g1));
    NS_CUDA(cudaFuncSetAttribute(gdnb_grad2a<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_g2a));
    NS_CUDA(cudaFuncSetAttribute(gdnb_grad2b<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_g2b));
  });
  const dim3 grid(a.n, a.nv, b);
  gdnb_setup<D><<<grid, NT, smem_setup, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
  gdnb_scan<D><<<dim3(D / Shapes<D>::JW, a.nv, b), NT, smem_scan, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
  gdnb_grad1<D><<<grid, NT, smem_g1, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
  gdnb_grad2a<D><<<grid, NT, smem_g2a, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
  gdnb_grad2b<D><<<grid, NT, smem_g2b, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
}

}  // namespace gdnb

// Chunked backward for head dims 64 and 128 into the caller's per-value-head outputs
// (dq32, dk32 fp32 [b, s, nv, D]; dv bf16; dg, dbeta fp32 [b, s, nv]). Returns false
// for other head dims. The workspace is allocated here for the call.
bool gdn_bwd_chunked(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta, at::Tensor dout,
                     int64_t groups, at::Tensor dq32, at::Tensor dk32, at::Tensor dv, at::Tensor dg, at::Tensor dbeta) {
  using namespace gdnb;
  const int b = q.size(0), s = q.size(1), nk = q.size(2), D = q.size(3), nv = v.size(2);
  if (D != 64 && D != 128) return false;
  const int n = (s + C - 1) / C;
  const int64_t nck = (int64_t)b * nv * n;
  auto f32 = q.options().dtype(at::kFloat);
  auto cd = at::empty({8, nck * C * D}, f32);
  auto cc = at::empty({4, nck * C * C}, f32);
  auto cv = at::empty({7, nck * C}, f32);
  auto dd = at::empty({7, nck * (int64_t)D * D}, f32);
  Args a{};
  a.q = reinterpret_cast<const bf16*>(q.data_ptr());
  a.k = reinterpret_cast<const bf16*>(k.data_ptr());
  a.v = reinterpret_cast<const bf16*>(v.data_ptr());
  a.beta = reinterpret_cast<const bf16*>(beta.data_ptr());
  a.dout = reinterpret_cast<const bf16*>(dout.data_ptr());
  a.g = g.data_ptr<float>();
  a.dq = dq32.data_ptr<float>();
  a.dk = dk32.data_ptr<float>();
  a.dv = reinterpret_cast<bf16*>(dv.data_ptr());
  a.dg = dg.data_ptr<float>();
  a.dbeta = dbeta.data_ptr<float>();
  a.s = s;
  a.nk = nk;
  a.nv = nv;
  a.groups = (int)groups;
  a.n = n;
  float* p = cd.data_ptr<float>();
  const int64_t ncd = nck * C * D;
  a.w.qn = p, a.w.kn = p + ncd, a.w.u = p + 2 * ncd, a.w.w = p + 3 * ncd;
  a.w.vn = p + 4 * ncd, a.w.dvn = p + 5 * ncd, a.w.dq = p + 6 * ncd, a.w.dk = p + 7 * ncd;
  p = cc.data_ptr<float>();
  const int64_t ncc = nck * C * C;
  a.w.tinv = p, a.w.m = p + ncc, a.w.a = p + 2 * ncc, a.w.kk = p + 3 * ncc;
  p = cv.data_ptr<float>();
  const int64_t ncv = nck * C;
  a.w.G = p, a.w.gam = p + ncv, a.w.ek = p + 2 * ncv, a.w.beta = p + 3 * ncv;
  a.w.rq = p + 4 * ncv, a.w.rk = p + 5 * ncv, a.w.dG = p + 6 * ncv;
  p = dd.data_ptr<float>();
  const int64_t ndd = nck * (int64_t)D * D;
  a.w.F = p, a.w.H = p + ndd, a.w.P = p + 2 * ndd, a.w.S0 = p + 3 * ndd, a.w.dS1 = p + 4 * ndd;
  a.w.S0t = p + 5 * ndd, a.w.dS1t = p + 6 * ndd;
  if (D == 64)
    run<64>(a, b);
  else
    run<128>(a, b);
  return true;
}

}  // namespace ns
