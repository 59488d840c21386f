// LM head + Markov head + 0.1 CE + 0.9 KL(target || draft), forward and backward,
// over the vocabulary in chunks. With few tokens (the draft's T is tens to hundreds
// of rows) one chunk covers the whole vocabulary: the [2T, V] logits live in HBM
// (tens of MB), each weight streams once per pass, and pass 2 does not recompute
// them. Larger T falls back to chunks, where pass 2 recomputes each chunk.
//
// pass 1, per chunk c (vocab [v0, v0 + Vc)):
//   L[0:T]  = bf16(h W_c^T) ; L[0:T] = bf16(L + bf16(E1[prev] W2_c^T))   (draft logits)
//   L[T:2T] = bf16(h_t W_c^T)                                           (target logits)
//   stats  : per (row, chunk-part) max / sum-exp of draft and target logits, the
//            target-weighted logit gap sum_v exp(t - m) (t - l), and the label logit.
// merge    : lse_draft, lse_target, CE (bf16-rounded like F.cross_entropy on bf16
//            logits) and KL per token.
// pass 2, per chunk: (several chunks) recompute L, then the logits gradient (CE at the bf16 boundary,
//            KL in fp32), sum_v min(p, q) partials, and
//            dh (fp32) += dl W_c, de (fp32) += dl W2_c, dW2_c = dl^T E1[prev].
// All reductions use fixed-order partial buffers: results are run-to-run identical.
#include <cstdlib>

#include "common.h"
#include "gemm.h"
#include "sm100.cuh"

namespace ns {

using bf16 = __nv_bfloat16;

struct Stat {
  float ml, zl, mt, zt, s1;
};

__device__ __forceinline__ void merge(Stat& a, const Stat& b) {
  // draft
  float m = fmaxf(a.ml, b.ml);
  float za = (a.ml == -INFINITY) ? 0.f : a.zl * expf(a.ml - m);
  float zb = (b.ml == -INFINITY) ? 0.f : b.zl * expf(b.ml - m);
  a.ml = m;
  a.zl = za + zb;
  // target (s1 scales with the target max)
  m = fmaxf(a.mt, b.mt);
  const float fa = (a.mt == -INFINITY) ? 0.f : expf(a.mt - m);
  const float fb = (b.mt == -INFINITY) ? 0.f : expf(b.mt - m);
  a.mt = m;
  a.zt = a.zt * fa + b.zt * fb;
  a.s1 = a.s1 * fa + b.s1 * fb;
}

// Columns [c0, c1) of a row handled by block p of `parts` (a multiple of 8 wide, so
// 16-byte vector loads stay aligned when the rows are).
__device__ __forceinline__ void part_range(int vc, int parts, int p, int& c0, int& c1) {
  const int per = (((vc + parts - 1) / parts) + 7) & ~7;
  c0 = min(vc, p * per);
  c1 = min(vc, c0 + per);
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

// grid (T, parts): block (t, p) scans its column range of the chunk. `vec`: rows of L
// and Tt are 16-byte aligned with strides a multiple of 8 (8 columns per load).
__global__ void head_stats_kernel(const bf16* __restrict__ L, int64_t ldl, const bf16* __restrict__ Tt,
                                  int64_t ldt, int vc, int v0, const int64_t* __restrict__ labels,
                                  Stat* __restrict__ part, float* __restrict__ label_logit, int chunk, int T,
                                  int parts, int vec) {
  const int t = blockIdx.x, p = blockIdx.y;
  int c0, c1;
  part_range(vc, parts, p, c0, c1);
  const bf16* lr = L + (int64_t)t * ldl;
  const bf16* tr = Tt + (int64_t)t * ldt;
  Stat s{-INFINITY, 0.f, -INFINITY, 0.f, 0.f};
  const int cv = vec ? c0 + ((c1 - c0) & ~7) : c0;
  for (int c = c0 + threadIdx.x * 8; c < cv; c += blockDim.x * 8) {
    float l[8], tv[8];
    unpack8(*reinterpret_cast<const uint4*>(lr + c), l);
    unpack8(*reinterpret_cast<const uint4*>(tr + c), tv);
#pragma unroll
    for (int i = 0; i < 8; ++i) merge(s, Stat{l[i], 1.f, tv[i], 1.f, tv[i] - l[i]});
  }
  for (int c = cv + threadIdx.x; c < c1; c += blockDim.x) {
    const float l = __bfloat162float(lr[c]);
    const float tv = __bfloat162float(tr[c]);
    merge(s, Stat{l, 1.f, tv, 1.f, tv - l});
  }
  // block reduction in fixed order (warp shuffles, then warp 0)
  __shared__ Stat sh[32];
  for (int off = 16; off > 0; off >>= 1) {
    Stat o;
    o.ml = __shfl_xor_sync(0xffffffff, s.ml, off);
    o.zl = __shfl_xor_sync(0xffffffff, s.zl, off);
    o.mt = __shfl_xor_sync(0xffffffff, s.mt, off);
    o.zt = __shfl_xor_sync(0xffffffff, s.zt, off);
    o.s1 = __shfl_xor_sync(0xffffffff, s.s1, off);
    merge(s, o);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    Stat a = sh[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) merge(a, sh[i]);
    part[((int64_t)chunk * parts + p) * T + t] = a;
    const int64_t lab = labels[t];
    if (lab >= v0 + c0 && lab < v0 + c1) label_logit[t] = __bfloat162float(lr[lab - v0]);
  }
}

// Per row: merge all partials; write lse_l, lse_t, ce (bf16-rounded), kl.
__global__ void head_merge_kernel(const Stat* __restrict__ part, int nparts, int T,
                                  const float* __restrict__ label_logit, float* __restrict__ row) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  Stat a{-INFINITY, 0.f, -INFINITY, 0.f, 0.f};
  for (int i = 0; i < nparts; ++i) merge(a, part[(int64_t)i * T + t]);
  const float lse_l = a.ml + logf(a.zl);
  const float lse_t = a.mt + logf(a.zt);
  const float ce = sm100::bf16_round(lse_l - label_logit[t]);
  const float kl = a.s1 / a.zt - lse_t + lse_l;
  row[t * 6 + 0] = ce;
  row[t * 6 + 1] = kl;
  row[t * 6 + 3] = lse_l;
  row[t * 6 + 4] = lse_t;
}

// Pass-2 elementwise: dl and sum_v min(p, q) partials (grid and `vec` as for the stats).
struct GradRow {
  float lse_l, lse_t, ce_s, kl_s;
  int64_t lab;
};

__device__ __forceinline__ float grad_elem(const GradRow& g, float l, float tv, int64_t v, float& mn) {
  const float pd = expf(l - g.lse_l);
  const float pt = expf(tv - g.lse_t);
  mn += fminf(pd, pt);
  // CE part at the compute-dtype boundary: bf16(exp(bf16(log_softmax))) * bf16(scale)
  const float ls = sm100::bf16_round(l - g.lse_l);
  float dce = sm100::bf16_round(sm100::bf16_round(expf(ls)) * g.ce_s);
  if (v == g.lab) dce = sm100::bf16_round(dce - g.ce_s);
  const float dkl = sm100::bf16_round((pd - pt) * g.kl_s);
  return dce + dkl;
}

__global__ void head_grad_kernel(const bf16* __restrict__ L, int64_t ldl, const bf16* __restrict__ Tt,
                                 int64_t ldt, int vc, int v0, const int64_t* __restrict__ labels,
                                 const float* __restrict__ weights, const float* __restrict__ row, float ce_w,
                                 float kl_w, float inv_accum, bf16* __restrict__ dl, int64_t lddl,
                                 float* __restrict__ minpart, int chunk, int T, int parts, int vec) {
  const int t = blockIdx.x, p = blockIdx.y;
  int c0, c1;
  part_range(vc, parts, p, c0, c1);
  const float scale = weights[t] * inv_accum;
  const GradRow g{row[t * 6 + 3], row[t * 6 + 4], sm100::bf16_round(scale * ce_w), scale * kl_w, labels[t]};
  const bf16* lr = L + (int64_t)t * ldl;
  const bf16* tr = Tt + (int64_t)t * ldt;
  bf16* dr = dl + (int64_t)t * lddl;
  float mn = 0.f;
  const int cv = vec ? c0 + ((c1 - c0) & ~7) : c0;
  for (int c = c0 + threadIdx.x * 8; c < cv; c += blockDim.x * 8) {
    float l[8], tv[8];
    unpack8(*reinterpret_cast<const uint4*>(lr + c), l);
    unpack8(*reinterpret_cast<const uint4*>(tr + c), tv);
    __nv_bfloat162 o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = __floats2bfloat162_rn(grad_elem(g, l[2 * i], tv[2 * i], (int64_t)v0 + c + 2 * i, mn),
                                   grad_elem(g, l[2 * i + 1], tv[2 * i + 1], (int64_t)v0 + c + 2 * i + 1, mn));
    *reinterpret_cast<uint4*>(dr + c) = *reinterpret_cast<const uint4*>(o);
  }
  for (int c = cv + threadIdx.x; c < c1; c += blockDim.x)
    dr[c] = __float2bfloat16(grad_elem(g, __bfloat162float(lr[c]), __bfloat162float(tr[c]), (int64_t)v0 + c, mn));
  __shared__ float sh[32];
  for (int off = 16; off > 0; off >>= 1) mn += __shfl_xor_sync(0xffffffff, mn, off);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = mn;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += sh[i];
    minpart[((int64_t)chunk * parts + p) * T + t] = s;
  }
}

__global__ void head_min_merge_kernel(const float* __restrict__ minpart, int nparts, int T, float* __restrict__ row) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float s = 0.f;
  for (int i = 0; i < nparts; ++i) s += minpart[(int64_t)i * T + t];
  row[t * 6 + 2] = s;
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ in, bf16* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16(in[i]);
}

// ============================================================================ streamed head (tcgen05)
// The logits are never written to memory. One persistent kernel per pass computes
// 128-token x 128-vocab tiles on the tensor cores with three TMEM accumulators:
// D = h W^T (draft), Tg = h_t W^T (target, when the target hidden rows are given)
// and Mk = E1[prev] W2^T (Markov); draft logits are bf16(bf16(D) + bf16(Mk)) exactly
// as in the two-GEMM form. Each epilogue thread owns one token row, so every
// reduction over the vocabulary stays in registers:
//   pass 1 (GRAD = false): online max / sum-exp of draft and target logits, the
//           target-weighted gap and the label logit; one Stat per (token, CTA);
//   pass 2 (GRAD = true):  the logits gradient (CE at the bf16 boundary, KL in fp32)
//           for a vocabulary chunk, written as bf16 tiles by TMA stores, and the
//           sum_v min(p, q) partials. dh / de / dW2 are GEMMs on that chunk.
// CTA b serves token tile b % mt and vocab tiles j0 + b / mt, + vsplit, ... (the mt
// CTAs of one vocab tile read the same weight rows together, from L2).
constexpr int HB_M = 128, HB_N = 128, HB_K = 64;
constexpr int HB_TILE = HB_M * HB_K * 2;           // 16 KB: a 128 x 64 bf16 token tile
constexpr int HB_WTILE = HB_N * HB_K * 2;          // 16 KB: a 128 x 64 bf16 weight tile
constexpr int HB_STAGE = 2 * HB_TILE + HB_WTILE;   // draft rows (or E1), target rows, W (or W2) rows
constexpr int HB_STAGES = 4;
constexpr int HB_BOX = 32 * 128;
constexpr int HB_EPI = 4 * 2 * HB_BOX;
constexpr int HB_SMEM = HB_STAGES * HB_STAGE + HB_EPI + 1024 + 256;
constexpr int HB_TMEM = 512;  // D at column 0, Tg at 128, Mk at 256
static_assert(HB_SMEM <= 227 * 1024, "shared memory budget");

struct HeadTcArgs {
  int T, V, H, r;
  int mt, vsplit;
  int j0, j1;   // vocab tiles of this launch
  int tgt_mma;  // target logits from the target hidden rows (else read from `tlog`)
  int markov;
  const bf16* tlog;
  int64_t ldt;
  const int64_t* labels;
  int part_base;       // partial index offset: part / minpart[(part_base + b / mt) * T + t]
  Stat* part;          // pass 1
  float* label_logit;  // pass 1
  const float* row;    // pass 2: lse_draft at [t * 6 + 3], lse_target at [t * 6 + 4]
  const float* weights;
  float ce_w, kl_w, inv_accum;
  int dl_v0;  // pass 2: vocabulary column of the chunk's first dl column
  float* minpart;
  int* err;
};

template <bool GRAD>
__global__ void __launch_bounds__(192, 1)
    head_tc_kernel(const __grid_constant__ CUtensorMap th, const __grid_constant__ CUtensorMap tt,
                   const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap te,
                   const __grid_constant__ CUtensorMap tw2, const __grid_constant__ CUtensorMap tdl, HeadTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sE = smem + HB_STAGES * HB_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + HB_EPI);
  uint64_t* empty = full + HB_STAGES;
  uint64_t* tfull = empty + HB_STAGES;  // main accumulators complete
  uint64_t* tempty = tfull + 1;         // main accumulators drained (4 epilogue warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x % a.mt, split = blockIdx.x / a.mt;
  const int m0 = m * HB_M;
  const int nkh = (a.H + HB_K - 1) / HB_K;
  const int nkr = a.markov ? (a.r + HB_K - 1) / HB_K : 0;
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < HB_STAGES; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    sm100::mbar_init(tfull, 1);
    sm100::mbar_init(tempty, 4);
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, HB_TMEM);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // Loads in the order the MMAs consume them: per tile the Markov k-blocks, then
    // the main ones.
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      const uint32_t main_bytes = HB_TILE * (a.tgt_mma ? 2 : 1) + HB_WTILE;
      for (int j = a.j0 + split; j < a.j1 && ok; j += a.vsplit) {
        const int v0 = j * HB_N;
        for (int kb = 0; kb < nkr + nkh; ++kb, ++it) {
          const int s = it % HB_STAGES;
          if (it >= HB_STAGES && !sm100::mbar_wait(&empty[s], ((it / HB_STAGES) & 1) ^ 1, a.err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * HB_STAGE;
          if (kb < nkr) {
            const int k = kb * HB_K;
            sm100::mbar_expect_tx(&full[s], HB_TILE + HB_WTILE);
            sm100::tma_load_2d(st, &te, &full[s], k, m0);
            sm100::tma_load_2d(st + 2 * HB_TILE, &tw2, &full[s], k, v0);
          } else {
            const int k = (kb - nkr) * HB_K;
            sm100::mbar_expect_tx(&full[s], main_bytes);
            sm100::tma_load_2d(st, &th, &full[s], k, m0);
            if (a.tgt_mma) sm100::tma_load_2d(st + HB_TILE, &tt, &full[s], k, m0);
            sm100::tma_load_2d(st + 2 * HB_TILE, &tw, &full[s], k, v0);
          }
        }
      }
      for (int i = max(0, it - HB_STAGES); i < it; ++i) sm100::mbar_wait(&full[i % HB_STAGES], (i / HB_STAGES) & 1, a.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = sm100::idesc_bf16(HB_M, HB_N, false, false);
      int it = 0, local = 0;
      bool ok = true;
      for (int j = a.j0 + split; j < a.j1 && ok; j += a.vsplit, ++local) {
        // single-buffered accumulators: free once the epilogue drained the last tile
        if (local >= 1 && !sm100::mbar_wait(tempty, (local - 1) & 1, a.err)) break;
        sm100::tc_fence_after();
        for (int kb = 0; kb < nkr + nkh && ok; ++kb, ++it) {
          const int s = it % HB_STAGES;
          if (!sm100::mbar_wait(&full[s], (it / HB_STAGES) & 1, a.err)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t base = sm100::smem_u32(smem + s * HB_STAGE);
          const int kq = kb < nkr ? kb : kb - nkr;
#pragma unroll
          for (int kk = 0; kk < HB_K / 16; ++kk) {
            const uint32_t acc = (kq > 0 || kk > 0) ? 1u : 0u;
            const uint64_t ad = sm100::smem_desc_sw128(base + kk * 32, 0, 1024);
            const uint64_t bd = sm100::smem_desc_sw128(base + 2 * HB_TILE + kk * 32, 0, 1024);
            if (kb < nkr) {
              sm100::mma_bf16(tmem + 256, ad, bd, idesc, acc);
            } else {
              sm100::mma_bf16(tmem, ad, bd, idesc, acc);
              if (a.tgt_mma)
                sm100::mma_bf16(tmem + 128, sm100::smem_desc_sw128(base + HB_TILE + kk * 32, 0, 1024), bd, idesc, acc);
            }
          }
          sm100::mma_commit(&empty[s]);
        }
        if (ok) sm100::mma_commit(tfull);
      }
    }
  } else {
    const int q = warp & 3;
    const int t = m0 + q * 32 + lane;
    const bool live = t < a.T;
    const int64_t lab = live ? a.labels[t] : -1;
    Stat st{-INFINITY, 0.f, -INFINITY, 0.f, 0.f};
    float mn = 0.f;
    GradRow g{0.f, 0.f, 0.f, 0.f, lab};
    if (GRAD && live) {
      const float scale = a.weights[t] * a.inv_accum;
      g = GradRow{a.row[t * 6 + 3], a.row[t * 6 + 4], sm100::bf16_round(scale * a.ce_w), scale * a.kl_w, lab};
    }
    uint8_t* stg = sE + q * 2 * HB_BOX;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    int local = 0, box = 0;
    for (int j = a.j0 + split; j < a.j1; j += a.vsplit, ++local) {
      const int v0 = j * HB_N;
      if (!sm100::mbar_wait(tfull, local & 1, a.err)) break;
      sm100::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < HB_N / 32; ++c) {
        float l[32], tv[32];
        sm100::tmem_ld32(trow + (uint32_t)(c * 32), l);
        if (a.markov) {
          float mk[32];
          sm100::tmem_ld32(trow + 256u + (uint32_t)(c * 32), mk);
#pragma unroll
          for (int i = 0; i < 32; ++i) l[i] = sm100::bf16_round(sm100::bf16_round(l[i]) + sm100::bf16_round(mk[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) l[i] = sm100::bf16_round(l[i]);
        }
        const int vb = v0 + c * 32;
        const int nvalid = live ? max(0, min(32, a.V - vb)) : 0;
        if (a.tgt_mma) {
          sm100::tmem_ld32(trow + 128u + (uint32_t)(c * 32), tv);
#pragma unroll
          for (int i = 0; i < 32; ++i) tv[i] = sm100::bf16_round(tv[i]);
        } else {
          const bf16* tr = a.tlog + (int64_t)(live ? t : 0) * a.ldt + vb;
#pragma unroll
          for (int i = 0; i < 32; ++i) tv[i] = i < nvalid ? __bfloat162float(tr[i]) : 0.f;
        }
        if (!GRAD) {
          if (nvalid > 0) {
            float cm = -INFINITY, ctm = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nvalid) {
                cm = fmaxf(cm, l[i]);
                ctm = fmaxf(ctm, tv[i]);
              }
            if (cm > st.ml) {
              st.zl = st.ml == -INFINITY ? 0.f : st.zl * expf(st.ml - cm);
              st.ml = cm;
            }
            if (ctm > st.mt) {
              const float f = st.mt == -INFINITY ? 0.f : expf(st.mt - ctm);
              st.zt *= f;
              st.s1 *= f;
              st.mt = ctm;
            }
            float ll = 0.f;
            bool hit = false;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nvalid) {
                st.zl += expf(l[i] - st.ml);
                const float e = expf(tv[i] - st.mt);
                st.zt += e;
                st.s1 += e * (tv[i] - l[i]);
                if ((int64_t)(vb + i) == lab) {
                  ll = l[i];
                  hit = true;
                }
              }
            if (hit) a.label_logit[t] = ll;
          }
        } else {
          // dl for these 32 columns -> half of a 32 x 64 staging box (128B swizzle)
          const int half = c & 1;
          uint8_t* sb = stg + (box & 1) * HB_BOX;
          if (half == 0) {
            if (lane == 0) sm100::bulk_wait_read<1>();
            __syncwarp();
          }
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            __nv_bfloat162 h[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i = 8 * jj + 2 * u;
              const float d0 = i < nvalid ? grad_elem(g, l[i], tv[i], (int64_t)vb + i, mn) : 0.f;
              const float d1 = i + 1 < nvalid ? grad_elem(g, l[i + 1], tv[i + 1], (int64_t)vb + i + 1, mn) : 0.f;
              h[u] = __floats2bfloat162_rn(d0, d1);
            }
            const int chunk = half * 4 + jj;
            *reinterpret_cast<uint4*>(sb + lane * 128 + ((chunk ^ (lane & 7)) * 16)) = *reinterpret_cast<uint4*>(h);
          }
          if (half == 1) {
            sm100::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              sm100::tma_store_2d(&tdl, sb, v0 + (c - 1) * 32 - a.dl_v0, m0 + q * 32);
              sm100::bulk_commit();
            }
            ++box;
          }
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(tempty);
    }
    const int64_t pidx = (int64_t)(a.part_base + split) * a.T + t;
    if (live) {
      if (GRAD)
        a.minpart[pidx] = mn;
      else
        a.part[pidx] = st;
    }
    if (GRAD && lane == 0) sm100::bulk_wait<0>();
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, HB_TMEM);
  }
}

// Streamed path of head_loss (same inputs / outputs): logits only in TMEM; the
// gradient in bf16 per vocabulary chunk (`chunk` columns, 0 = automatic).
static std::vector<at::Tensor> head_loss_streamed(at::Tensor hcat, int64_t T, at::Tensor lm_head,
                                                  c10::optional<at::Tensor> e, c10::optional<at::Tensor> w2,
                                                  c10::optional<at::Tensor> target_logits, at::Tensor labels,
                                                  at::Tensor weights, double ce_w, double kl_w, double inv_accum,
                                                  c10::optional<at::Tensor> dw2_out, int64_t chunk) {
  const int64_t V = lm_head.size(0), H = lm_head.size(1);
  const bool markov = e.has_value() && e->defined();
  const bool tl = target_logits.has_value() && target_logits->defined();
  const int64_t r = markov ? e->size(1) : 0;
  auto opt = hcat.options();
  auto* hp = reinterpret_cast<const bf16*>(hcat.data_ptr());
  const CUtensorMap th = make_tmap_bf16(hp, T, H, H, HB_M, 64);
  const CUtensorMap tt = tl ? th : make_tmap_bf16(hp + T * H, T, H, H, HB_M, 64);
  const CUtensorMap tw = make_tmap_bf16(lm_head.data_ptr(), V, H, H, HB_N, 64);
  const CUtensorMap te = markov ? make_tmap_bf16(e->data_ptr(), T, r, r, HB_M, 64) : th;
  const CUtensorMap tw2 = markov ? make_tmap_bf16(w2->data_ptr(), V, r, r, HB_N, 64) : tw;
  const int mt = (int)((T + HB_M - 1) / HB_M);
  const int vtiles = (int)((V + HB_N - 1) / HB_N);
  const int vsplit = std::max(1, std::min(vtiles, num_sms() / mt));
  const int grid = mt * vsplit;
  HeadTcArgs a{};
  a.T = (int)T;
  a.V = (int)V;
  a.H = (int)H;
  a.r = (int)r;
  a.mt = mt;
  a.vsplit = vsplit;
  a.tgt_mma = tl ? 0 : 1;
  a.markov = markov ? 1 : 0;
  a.tlog = tl ? reinterpret_cast<const bf16*>(target_logits->data_ptr()) : nullptr;
  a.ldt = tl ? target_logits->stride(0) : 0;
  a.labels = labels.data_ptr<int64_t>();
  a.weights = weights.data_ptr<float>();
  a.ce_w = (float)ce_w;
  a.kl_w = (float)kl_w;
  a.inv_accum = (float)inv_accum;
  a.err = device_error_flag();
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(head_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, HB_SMEM));
    NS_CUDA(cudaFuncSetAttribute(head_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, HB_SMEM));
  });

  // ---------------- pass 1: statistics
  auto part = at::empty({(int64_t)vsplit * T * 5}, opt.dtype(at::kFloat));
  auto label_logit = at::zeros({T}, opt.dtype(at::kFloat));
  auto row = at::zeros({T, 6}, opt.dtype(at::kFloat));
  a.part = reinterpret_cast<Stat*>(part.data_ptr<float>());
  a.label_logit = label_logit.data_ptr<float>();
  a.j0 = 0;
  a.j1 = vtiles;
  head_tc_kernel<false><<<grid, 192, HB_SMEM, stream()>>>(th, tt, tw, te, tw2, tw, a);
  NS_CUDA(cudaGetLastError());
  head_merge_kernel<<<(T + 127) / 128, 128, 0, stream()>>>(a.part, vsplit, (int)T, a.label_logit,
                                                           row.data_ptr<float>());
  NS_CUDA(cudaGetLastError());

  // ---------------- pass 2: gradient per vocabulary chunk
  int64_t ctiles;
  if (chunk > 0)
    ctiles = (chunk + HB_N - 1) / HB_N;
  else
    ctiles = T * V * 2 <= (int64_t(1) << 30) ? vtiles : std::max<int64_t>(1, (int64_t(512) << 20) / (T * 2 * HB_N));
  ctiles = std::min<int64_t>(ctiles, vtiles);
  const int nch = (int)((vtiles + ctiles - 1) / ctiles);
  const int64_t ldc = ctiles * HB_N;
  auto dl = at::empty({T, ldc}, opt);
  auto* dlp = reinterpret_cast<bf16*>(dl.data_ptr());
  auto minpart = at::empty({(int64_t)nch * vsplit * T}, opt.dtype(at::kFloat));
  auto dh32 = at::zeros({T, H}, opt.dtype(at::kFloat));
  auto de32 = markov ? at::zeros({T, r}, opt.dtype(at::kFloat)) : at::Tensor();
  a.row = row.data_ptr<float>();
  a.minpart = minpart.data_ptr<float>();
  for (int c = 0; c < nch; ++c) {
    const int j0 = (int)(c * ctiles), j1 = (int)std::min<int64_t>(vtiles, j0 + ctiles);
    const int64_t v0 = (int64_t)j0 * HB_N, n = std::min<int64_t>(V, (int64_t)j1 * HB_N) - v0;
    const CUtensorMap tdl = make_tmap_bf16(dlp, T, n, ldc, 32, 64);
    a.j0 = j0;
    a.j1 = j1;
    a.dl_v0 = (int)v0;
    a.part_base = c * vsplit;
    head_tc_kernel<true><<<grid, 192, HB_SMEM, stream()>>>(th, tt, tw, te, tw2, tdl, a);
    NS_CUDA(cudaGetLastError());
    // dh[T, H] += dl[T, n] W_c[n, H]
    {
      Operand A{lm_head.data_ptr<at::BFloat16>() + v0 * H, n, H, H, true};
      Operand B{dlp, T, n, ldc, false};
      gemm_launch(A, B, (int)H, (int)T, (int)n, Epilogue{nullptr, dh32.data_ptr<float>(), 1, H, nullptr, 0, 0, c > 0});
    }
    if (markov) {
      Operand A{w2->data_ptr<at::BFloat16>() + v0 * r, n, r, r, true};
      Operand B{dlp, T, n, ldc, false};
      gemm_launch(A, B, (int)r, (int)T, (int)n, Epilogue{nullptr, de32.data_ptr<float>(), 1, r, nullptr, 0, 0, c > 0});
      Operand DA{dlp, T, n, ldc, true};
      Operand EB{e->data_ptr(), T, r, r, true};
      gemm_launch(DA, EB, (int)n, (int)r, (int)T,
                  Epilogue{reinterpret_cast<bf16*>(dw2_out->data_ptr()) + v0 * r, nullptr, r, 1, nullptr, 0, 0, false});
    }
  }
  head_min_merge_kernel<<<(T + 127) / 128, 128, 0, stream()>>>(minpart.data_ptr<float>(), nch * vsplit, (int)T,
                                                               row.data_ptr<float>());
  NS_CUDA(cudaGetLastError());
  auto dh = at::empty({T, H}, opt);
  f32_to_bf16_kernel<<<num_sms() * 4, 256, 0, stream()>>>(dh32.data_ptr<float>(), reinterpret_cast<bf16*>(dh.data_ptr()),
                                                          T * H);
  NS_CUDA(cudaGetLastError());
  at::Tensor de;
  if (markov) {
    de = at::empty({T, r}, opt);
    f32_to_bf16_kernel<<<num_sms(), 256, 0, stream()>>>(de32.data_ptr<float>(), reinterpret_cast<bf16*>(de.data_ptr()),
                                                        T * r);
    NS_CUDA(cudaGetLastError());
  }
  return {row, dh, de};
}

// ----------------------------------------------------------------------------- host
// hcat: [T or 2T, H] = [draft hidden ; target hidden] (target rows absent when
// target_logits is given). Returns per-row stats [T, 6] =
// (ce, kl, sum_v min(p,q), lse_draft, lse_target, unused); writes dh [T, H], de [T, r], dW2.
std::vector<at::Tensor> head_loss(at::Tensor hcat, int64_t T, at::Tensor lm_head, c10::optional<at::Tensor> e,
                                  c10::optional<at::Tensor> w2, c10::optional<at::Tensor> target_logits,
                                  at::Tensor labels, at::Tensor weights, double ce_w, double kl_w,
                                  double inv_accum, c10::optional<at::Tensor> dw2_out, int64_t chunk) {
  check_bf16(hcat, "hcat");
  check_bf16(lm_head, "lm_head");
  NS_CHECK(hcat.is_contiguous() && lm_head.is_contiguous(), "head: contiguous inputs expected");
  const int64_t V = lm_head.size(0), H = lm_head.size(1);
  const bool markov = e.has_value() && e->defined();
  const bool tl = target_logits.has_value() && target_logits->defined();
  NS_CHECK(hcat.size(0) == (tl ? T : 2 * T), "hcat rows must be T (teacher logits) or 2T");
  NS_CHECK(labels.scalar_type() == at::kLong && labels.numel() == T, "labels [T] int64");
  NS_CHECK(weights.scalar_type() == at::kFloat && weights.numel() == T, "weights [T] fp32");
  {
    // The streamed tensor-core path whenever the logits exceed 4 GiB: it never
    // writes them, where the materialised path holds [R + T, V] bf16 (R = T or 2T)
    // and beyond that budget must chunk and recompute them. Below it (the draft's
    // few hundred tokens) the materialised path is faster: its logits GEMM runs on
    // wide swap-AB tiles, while the streamed tiles are bound by the L2 -> shared
    // memory feed of three operand streams.
    // NANOSPEC_HEAD=streamed | materialize overrides the choice.
    const char* mode = std::getenv("NANOSPEC_HEAD");
    const bool aligned = H % 8 == 0 && (!markov || e->size(1) % 8 == 0) && (!markov || e->is_contiguous()) &&
                         (!markov || w2->is_contiguous());
    const int64_t logit_bytes = (hcat.size(0) + T) * V * 2;
    bool streamed = logit_bytes > (int64_t(4) << 30);
    if (mode && std::string(mode) == "streamed") streamed = true;
    if (mode && std::string(mode) == "materialize") streamed = false;
    if (aligned && streamed)
      return head_loss_streamed(hcat, T, lm_head, e, w2, target_logits, labels, weights, ce_w, kl_w, inv_accum,
                                dw2_out, chunk);
  }
  auto opt = hcat.options();
  const int64_t R = hcat.size(0);
  // chunk <= 0: the whole vocabulary in one chunk when the logits and their gradient
  // ([R + T, V] bf16) fit in 4 GiB; then pass 2 reuses pass 1's logits instead of
  // recomputing them, and every GEMM below runs once over the full vocabulary.
  if (chunk <= 0) {
    const int64_t budget = int64_t(4) << 30;
    chunk = (R + T) * V * 2 <= budget ? V : std::max<int64_t>(4096, (budget / ((R + T) * 2)) & ~int64_t(127));
  }
  const int64_t vc = std::min<int64_t>(chunk, V);
  const int nchunks = (int)((V + vc - 1) / vc);
  const int64_t ldv = (vc + 7) & ~int64_t(7);  // row stride of the logits / gradient buffers (TMA: 16 B)
  // blocks per row: about four per SM in total, each at least 2048 columns wide
  const int parts = (int)std::max<int64_t>(1, std::min<int64_t>((4 * num_sms() + T - 1) / T, vc / 2048));
  auto Lbuf = at::empty({R, ldv}, opt);
  auto dl = at::empty({T, ldv}, opt);
  auto part = at::empty({(int64_t)nchunks * parts * T * 5}, opt.dtype(at::kFloat));
  auto minpart = at::empty({(int64_t)nchunks * parts * T}, opt.dtype(at::kFloat));
  auto label_logit = at::zeros({T}, opt.dtype(at::kFloat));
  auto row = at::zeros({T, 6}, opt.dtype(at::kFloat));
  auto dh32 = at::zeros({T, H}, opt.dtype(at::kFloat));
  int64_t r = markov ? e->size(1) : 0;
  auto de32 = markov ? at::zeros({T, r}, opt.dtype(at::kFloat)) : at::Tensor();
  const int64_t* lab = labels.data_ptr<int64_t>();
  auto* Lp = reinterpret_cast<bf16*>(Lbuf.data_ptr());
  Stat* partp = reinterpret_cast<Stat*>(part.data_ptr<float>());

  auto logits_chunk = [&](int64_t v0, int64_t n) {
    // L[0:R, 0:n] = hcat W_c^T   (swap-AB: vocab rows on M, tokens on N)
    Operand W{lm_head.data_ptr<at::BFloat16>() + v0 * H, n, H, H, false};
    Operand X{hcat.data_ptr(), R, H, H, false};
    gemm_launch(W, X, (int)n, (int)R, (int)H, Epilogue{Lp, nullptr, 1, ldv, nullptr, 0, 0, false});
    if (markov) {
      Operand W2{w2->data_ptr<at::BFloat16>() + v0 * r, n, r, r, false};
      Operand E{e->data_ptr(), T, r, r, false};
      gemm_launch(W2, E, (int)n, (int)T, (int)r, Epilogue{Lp, nullptr, 1, ldv, nullptr, 0, 0, true});
    }
  };
  auto target_ptr = [&](int64_t v0, int64_t& ld) -> const bf16* {
    if (tl) {
      ld = target_logits->stride(0);
      return reinterpret_cast<const bf16*>(target_logits->data_ptr()) + v0;
    }
    ld = ldv;
    return Lp + T * ldv;
  };
  auto vec_ok = [&](const bf16* tp, int64_t ldt) -> int {
    return (reinterpret_cast<uintptr_t>(Lp) % 16 == 0 && reinterpret_cast<uintptr_t>(tp) % 16 == 0 &&
            ldt % 8 == 0) ? 1 : 0;
  };

  // ---------------- pass 1
  for (int c = 0; c < nchunks; ++c) {
    const int64_t v0 = c * vc, n = std::min(vc, V - v0);
    logits_chunk(v0, n);
    int64_t ldt;
    const bf16* tp = target_ptr(v0, ldt);
    head_stats_kernel<<<dim3(T, parts), 256, 0, stream()>>>(Lp, ldv, tp, ldt, (int)n, (int)v0, lab, partp,
                                                           label_logit.data_ptr<float>(), c, (int)T, parts,
                                                           vec_ok(tp, ldt));
    NS_CUDA(cudaGetLastError());
  }
  head_merge_kernel<<<(T + 127) / 128, 128, 0, stream()>>>(partp, nchunks * parts, (int)T,
                                                           label_logit.data_ptr<float>(), row.data_ptr<float>());
  NS_CUDA(cudaGetLastError());

  // ---------------- pass 2
  auto* dlp = reinterpret_cast<bf16*>(dl.data_ptr());
  for (int c = 0; c < nchunks; ++c) {
    const int64_t v0 = c * vc, n = std::min(vc, V - v0);
    if (nchunks > 1) logits_chunk(v0, n);  // a single chunk still holds pass 1's logits
    int64_t ldt;
    const bf16* tp = target_ptr(v0, ldt);
    head_grad_kernel<<<dim3(T, parts), 256, 0, stream()>>>(
        Lp, ldv, tp, ldt, (int)n, (int)v0, lab, weights.data_ptr<float>(), row.data_ptr<float>(), (float)ce_w,
        (float)kl_w, (float)inv_accum, dlp, ldv, minpart.data_ptr<float>(), c, (int)T, parts, vec_ok(tp, ldt));
    NS_CUDA(cudaGetLastError());
    // dh[T, H] += dl[T, n] W_c[n, H]   (swap-AB: H on M, tokens on N, reduce over vocab)
    {
      Operand A{lm_head.data_ptr<at::BFloat16>() + v0 * H, n, H, H, true};
      Operand B{dlp, T, n, ldv, false};
      gemm_launch(A, B, (int)H, (int)T, (int)n, Epilogue{nullptr, dh32.data_ptr<float>(), 1, H, nullptr, 0, 0, c > 0});
    }
    if (markov) {
      Operand A{w2->data_ptr<at::BFloat16>() + v0 * r, n, r, r, true};
      Operand B{dlp, T, n, ldv, false};
      gemm_launch(A, B, (int)r, (int)T, (int)n, Epilogue{nullptr, de32.data_ptr<float>(), 1, r, nullptr, 0, 0, c > 0});
      // dW2[v0:v0+n, r] = dl^T E1[prev]
      Operand DA{dlp, T, n, ldv, true};
      Operand EB{e->data_ptr(), T, r, r, true};
      gemm_launch(DA, EB, (int)n, (int)r, (int)T,
                  Epilogue{reinterpret_cast<bf16*>(dw2_out->data_ptr()) + v0 * r, nullptr, r, 1, nullptr, 0, 0, false});
    }
  }
  head_min_merge_kernel<<<(T + 127) / 128, 128, 0, stream()>>>(minpart.data_ptr<float>(), nchunks * parts, (int)T,
                                                               row.data_ptr<float>());
  NS_CUDA(cudaGetLastError());
  auto dh = at::empty({T, H}, opt);
  f32_to_bf16_kernel<<<num_sms() * 4, 256, 0, stream()>>>(dh32.data_ptr<float>(), reinterpret_cast<bf16*>(dh.data_ptr()),
                                                          T * H);
  NS_CUDA(cudaGetLastError());
  at::Tensor de;
  if (markov) {
    de = at::empty({T, r}, opt);
    f32_to_bf16_kernel<<<num_sms(), 256, 0, stream()>>>(de32.data_ptr<float>(), reinterpret_cast<bf16*>(de.data_ptr()),
                                                        T * r);
    NS_CUDA(cudaGetLastError());
  }
  return {row, dh, de};
}

}  // namespace ns
