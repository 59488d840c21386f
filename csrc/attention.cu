// Draft attention with the anchor layout (no dense mask, no stored probabilities).
//
// Query block j of batch row i (block_size queries x G query heads per KV head)
// sees the context keys [0, anchors[i, j]) and its own block's draft keys; a
// block with keep == false sees nothing and outputs zeros (lse = -inf).
// Keys/values are in split layout: row i*S + t for context token t, row
// b*S + i*Td + u for draft token u; rows may be strided (K and V live in one
// [rows, 2*Hk*D] projection output).
//
// forward : one CTA per (block j, KV head, batch row); the G*bs query rows of
//           the block share one key stream (GQA), scores and the online softmax
//           run in fp32, keys are tiled 32 at a time through shared memory.
// backward: two deterministic kernels instead of atomics.
//           dq  - same decomposition as the forward (P recomputed from lse);
//           dkv - one CTA per (32-key tile, KV head, batch row); it walks the
//                 query blocks that can see the tile and accumulates dK, dV in
//                 shared memory in a fixed order.
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
  bf16 *out, *dq, *dk, *dv;
  int64_t lddk, lddv;
  int b, S, nb, bs, Hq, Hk;
  float scale;
};

constexpr int KT = 32;  // keys per tile

__device__ __forceinline__ int64_t key_row(const AttnArgs& a, int bi, int kv) {
  // kv in [0, S) context, [S, S+Td) draft
  return kv < a.S ? (int64_t)bi * a.S + kv : (int64_t)a.b * a.S + (int64_t)bi * a.nb * a.bs + (kv - a.S);
}

// Visible key index ranges of block j: [0, anchor) and [S + j*bs, S + (j+1)*bs).
__device__ __forceinline__ int n_visible_tiles(int anchor, int bs) {
  return (anchor + KT - 1) / KT + (bs + KT - 1) / KT;
}

// Keys of tile `t` of block j: returns base key index and count.
__device__ __forceinline__ void tile_keys(int t, int anchor, int S, int j, int bs, int& k0, int& cnt) {
  const int nctx = (anchor + KT - 1) / KT;
  if (t < nctx) {
    k0 = t * KT;
    cnt = min(KT, anchor - k0);
  } else {
    const int u = t - nctx;
    k0 = S + j * bs + u * KT;
    cnt = min(KT, bs - u * KT);
  }
}

// ---------------------------------------------------------------------------- forward
constexpr int MAXR = 8;  // query rows per warp (8 warps -> up to 64 rows per CTA)

template <int D>
__global__ void __launch_bounds__(256) attn_fwd_kernel(AttnArgs a) {
  constexpr int E = (D + 31) / 32;  // elements per lane
  constexpr int DL = D < 32 ? D : 32;  // lanes holding elements
  extern __shared__ float sm[];
  const int j = blockIdx.x, hk = blockIdx.y, bi = blockIdx.z;
  const int G = a.Hq / a.Hk;
  const int R = G * a.bs;  // query rows of this CTA
  const int Td = a.nb * a.bs;
  float* Kt = sm;               // [D][KT]
  float* Vs = Kt + D * KT;      // [KT][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const bool kp = a.keep[bi * a.nb + j];
  const int anchor = kp ? (int)a.anchors[bi * a.nb + j] : 0;
  const int ntiles = kp ? n_visible_tiles(anchor, a.bs) : 0;

  // Each warp owns rows r = warp, warp + nw, ...; state kept in registers.
  float acc[MAXR][E];
  float mx[MAXR], den[MAXR];
  float qv[MAXR][E];
  const int my_rows = (R - warp + nw - 1) / nw;
#pragma unroll
  for (int rr = 0; rr < MAXR; ++rr) {
    mx[rr] = -INFINITY;
    den[rr] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[rr][e] = 0.f;
    if (rr < my_rows) {
      const int r = warp + rr * nw;
      const int g = r / a.bs, u = r % a.bs;
      const int h = hk * G + g;
      const int t = bi * Td + j * a.bs + u;
      const bf16* qp = a.q + ((int64_t)t * a.Hq + h) * D;
#pragma unroll
      for (int e = 0; e < E; ++e) qv[rr][e] = lane < DL ? __bfloat162float(qp[lane + 32 * e]) * a.scale : 0.f;
    }
  }

  for (int tile = 0; tile < ntiles; ++tile) {
    int k0, cnt;
    tile_keys(tile, anchor, a.S, j, a.bs, k0, cnt);
    __syncthreads();
    for (int idx = threadIdx.x; idx < KT * D; idx += blockDim.x) {
      const int kk = idx / D, d = idx % D;
      float kvv = 0.f, vvv = 0.f;
      if (kk < cnt) {
        const int64_t row = key_row(a, bi, k0 + kk);
        kvv = __bfloat162float(a.k[row * a.ldk + hk * D + d]);
        vvv = __bfloat162float(a.v[row * a.ldv + hk * D + d]);
      }
      Kt[d * KT + kk] = kvv;
      Vs[kk * D + d] = vvv;
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < MAXR; ++rr) {
      if (rr >= my_rows) break;
      // lane = key: s = q . k_lane
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
#pragma unroll 8
        for (int dd = 0; dd < DL; ++dd) {
          const float qd = __shfl_sync(0xffffffff, qv[rr][e], dd);
          s += qd * Kt[(dd + 32 * e) * KT + lane];
        }
      }
      if (lane >= cnt) s = -INFINITY;
      float tmax = s;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffff, tmax, o));
      const float nm = fmaxf(mx[rr], tmax);
      const float corr = expf(mx[rr] - nm);
      const float p = (lane < cnt) ? expf(s - nm) : 0.f;
      float ps = p;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffff, ps, o);
      den[rr] = den[rr] * corr + ps;
      mx[rr] = nm;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[rr][e] *= corr;
      for (int kk = 0; kk < cnt; ++kk) {
        const float pk = __shfl_sync(0xffffffff, p, kk);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[rr][e] += lane < DL ? pk * Vs[kk * D + lane + 32 * e] : 0.f;
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < MAXR; ++rr) {
    if (rr >= my_rows) break;
    const int r = warp + rr * nw;
    const int g = r / a.bs, u = r % a.bs;
    const int h = hk * G + g;
    const int t = bi * Td + j * a.bs + u;
    const bool any = den[rr] > 0.f;
    const float inv = any ? 1.f / den[rr] : 0.f;
    bf16* op = a.out + ((int64_t)t * a.Hq + h) * D;
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (lane < DL) op[lane + 32 * e] = __float2bfloat16(acc[rr][e] * inv);
    if (lane == 0) a.lse[((int64_t)bi * a.Hq + h) * Td + j * a.bs + u] = any ? mx[rr] + logf(den[rr]) : -INFINITY;
  }
}

// ---------------------------------------------------------------------------- backward dq
template <int D>
__global__ void __launch_bounds__(256) attn_bwd_dq_kernel(AttnArgs a) {
  constexpr int E = (D + 31) / 32;
  constexpr int DL = D < 32 ? D : 32;
  extern __shared__ float sm[];
  const int j = blockIdx.x, hk = blockIdx.y, bi = blockIdx.z;
  const int G = a.Hq / a.Hk;
  const int R = G * a.bs;
  const int Td = a.nb * a.bs;
  float* Kt = sm;            // [D][KT]
  float* Ks = Kt + D * KT;   // [KT][D]
  float* Vt = Ks + KT * D;   // [D][KT]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const bool kp = a.keep[bi * a.nb + j];
  const int anchor = kp ? (int)a.anchors[bi * a.nb + j] : 0;
  const int ntiles = kp ? n_visible_tiles(anchor, a.bs) : 0;
  float qv[MAXR][E], dov[MAXR][E], dqa[MAXR][E], lse[MAXR], delta[MAXR];
  const int my_rows = (R - warp + nw - 1) / nw;
#pragma unroll
  for (int rr = 0; rr < MAXR; ++rr) {
#pragma unroll
    for (int e = 0; e < E; ++e) dqa[rr][e] = 0.f;
    lse[rr] = -INFINITY;
    delta[rr] = 0.f;
    if (rr < my_rows) {
      const int r = warp + rr * nw;
      const int g = r / a.bs, u = r % a.bs;
      const int h = hk * G + g;
      const int t = bi * Td + j * a.bs + u;
      const int64_t off = ((int64_t)t * a.Hq + h) * D;
      float dl = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const bool in = lane < DL;
        qv[rr][e] = in ? __bfloat162float(a.q[off + lane + 32 * e]) * a.scale : 0.f;
        dov[rr][e] = in ? __bfloat162float(a.dout[off + lane + 32 * e]) : 0.f;
        dl += in ? dov[rr][e] * __bfloat162float(a.o[off + lane + 32 * e]) : 0.f;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dl += __shfl_xor_sync(0xffffffff, dl, o);
      delta[rr] = dl;
      lse[rr] = a.lse[((int64_t)bi * a.Hq + h) * Td + j * a.bs + u];
    }
  }
  for (int tile = 0; tile < ntiles; ++tile) {
    int k0, cnt;
    tile_keys(tile, anchor, a.S, j, a.bs, k0, cnt);
    __syncthreads();
    for (int idx = threadIdx.x; idx < KT * D; idx += blockDim.x) {
      const int kk = idx / D, d = idx % D;
      float kvv = 0.f, vvv = 0.f;
      if (kk < cnt) {
        const int64_t row = key_row(a, bi, k0 + kk);
        kvv = __bfloat162float(a.k[row * a.ldk + hk * D + d]);
        vvv = __bfloat162float(a.v[row * a.ldv + hk * D + d]);
      }
      Kt[d * KT + kk] = kvv;
      Ks[kk * D + d] = kvv;
      Vt[d * KT + kk] = vvv;
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < MAXR; ++rr) {
      if (rr >= my_rows) break;
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
#pragma unroll 8
        for (int dd = 0; dd < DL; ++dd) {
          const float qd = __shfl_sync(0xffffffff, qv[rr][e], dd);
          const float od = __shfl_sync(0xffffffff, dov[rr][e], dd);
          s += qd * Kt[(dd + 32 * e) * KT + lane];
          dp += od * Vt[(dd + 32 * e) * KT + lane];
        }
      }
      const float p = (lane < cnt && lse[rr] > -INFINITY) ? expf(s - lse[rr]) : 0.f;
      const float ds = p * (dp - delta[rr]);
      for (int kk = 0; kk < cnt; ++kk) {
        const float dk = __shfl_sync(0xffffffff, ds, kk);
#pragma unroll
        for (int e = 0; e < E; ++e) dqa[rr][e] += lane < DL ? dk * Ks[kk * D + lane + 32 * e] : 0.f;
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < MAXR; ++rr) {
    if (rr >= my_rows) break;
    const int r = warp + rr * nw;
    const int g = r / a.bs, u = r % a.bs;
    const int h = hk * G + g;
    const int t = bi * Td + j * a.bs + u;
    bf16* dp = a.dq + ((int64_t)t * a.Hq + h) * D;
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (lane < DL) dp[lane + 32 * e] = __float2bfloat16(dqa[rr][e] * a.scale);
  }
}

// ---------------------------------------------------------------------------- backward dk, dv
// Tiles: ctx tiles [0, ceil(S/KT)) then one tile per draft block (bs <= 32).
// For each query block j that sees the tile: warps compute P and dS for the block's
// rows (lane = key) into shared memory; then thread (key = t % 32, dim chunk t / 32)
// accumulates dK[key] += dS * q and dV[key] += P * dO over the rows in registers.
template <int D>
__global__ void __launch_bounds__(128) attn_bwd_dkv_kernel(AttnArgs a) {
  constexpr int NT = 128;
  constexpr int DC = D / (NT / 32);  // dims per thread in the accumulation phase
  constexpr int RMAX = 64;
  extern __shared__ float sm[];
  float* Kt = sm;                 // [D][KT]
  float* Vt = Kt + D * KT;        // [D][KT]
  float* Qs = Vt + D * KT;        // [RMAX][D]  (q, unscaled)
  float* Os = Qs + RMAX * D;      // [RMAX][D]  (dO)
  float* Ps = Os + RMAX * D;      // [RMAX][KT]
  float* DSs = Ps + RMAX * KT;    // [RMAX][KT]
  const int tile = blockIdx.x, hk = blockIdx.y, bi = blockIdx.z;
  const int G = a.Hq / a.Hk;
  const int Td = a.nb * a.bs;
  const int nctx = (a.S + KT - 1) / KT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = NT / 32;
  int k0, cnt, jlo, jhi;
  if (tile < nctx) {
    k0 = tile * KT;
    cnt = min(KT, a.S - k0);
    jlo = 0;
    jhi = a.nb;
  } else {
    const int jb = tile - nctx;
    k0 = a.S + jb * a.bs;
    cnt = a.bs;
    jlo = jb;
    jhi = jb + 1;
  }
  for (int idx = threadIdx.x; idx < KT * D; idx += NT) {
    const int kk = idx / D, d = idx % D;
    float kvv = 0.f, vvv = 0.f;
    if (kk < cnt) {
      const int64_t row = key_row(a, bi, k0 + kk);
      kvv = __bfloat162float(a.k[row * a.ldk + hk * D + d]);
      vvv = __bfloat162float(a.v[row * a.ldv + hk * D + d]);
    }
    Kt[d * KT + kk] = kvv;
    Vt[d * KT + kk] = vvv;
  }
  const int key = threadIdx.x & 31;
  const int d0 = (threadIdx.x >> 5) * DC;
  float dK[DC], dV[DC];
#pragma unroll
  for (int i = 0; i < DC; ++i) dK[i] = dV[i] = 0.f;
  const int R = G * a.bs;
  for (int j = jlo; j < jhi; ++j) {
    if (!a.keep[bi * a.nb + j]) continue;
    const int anchor = (int)a.anchors[bi * a.nb + j];
    const int vis = tile < nctx ? max(0, min(cnt, anchor - k0)) : cnt;
    if (vis <= 0) continue;
    __syncthreads();  // previous block's Ps/DSs/Qs/Os fully consumed
    for (int idx = threadIdx.x; idx < R * D; idx += NT) {
      const int r = idx / D, d = idx % D;
      const int g = r / a.bs, u = r % a.bs;
      const int t = bi * Td + j * a.bs + u;
      const int64_t off = ((int64_t)t * a.Hq + hk * G + g) * D + d;
      Qs[r * D + d] = __bfloat162float(a.q[off]);
      Os[r * D + d] = __bfloat162float(a.dout[off]);
    }
    __syncthreads();
    for (int r = warp; r < R; r += nw) {
      const int g = r / a.bs, u = r % a.bs;
      const int h = hk * G + g;
      const int t = bi * Td + j * a.bs + u;
      const int64_t off = ((int64_t)t * a.Hq + h) * D;
      float dl = 0.f;
      for (int d = lane; d < D; d += 32) dl += Os[r * D + d] * __bfloat162float(a.o[off + d]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dl += __shfl_xor_sync(0xffffffff, dl, o);
      const float lse = a.lse[((int64_t)bi * a.Hq + h) * Td + j * a.bs + u];
      float s = 0.f, dp = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) {
        s += Qs[r * D + d] * Kt[d * KT + lane];
        dp += Os[r * D + d] * Vt[d * KT + lane];
      }
      const float p = (lane < vis && lse > -INFINITY) ? expf(s * a.scale - lse) : 0.f;
      Ps[r * KT + lane] = p;
      DSs[r * KT + lane] = p * (dp - dl) * a.scale;
    }
    __syncthreads();
    for (int r = 0; r < R; ++r) {
      const float p = Ps[r * KT + key], ds = DSs[r * KT + key];
#pragma unroll
      for (int i = 0; i < DC; ++i) {
        dV[i] += p * Os[r * D + d0 + i];
        dK[i] += ds * Qs[r * D + d0 + i];
      }
    }
  }
  if (key < cnt) {
    const int64_t row = key_row(a, bi, k0 + key);
#pragma unroll
    for (int i = 0; i < DC; ++i) {
      a.dk[row * a.lddk + hk * D + d0 + i] = __float2bfloat16(dK[i]);
      a.dv[row * a.lddv + hk * D + d0 + i] = __float2bfloat16(dV[i]);
    }
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
  NS_CHECK(a.Hq % a.Hk == 0 && (a.Hq / a.Hk) * bs <= 64, "GQA group * block_size must be <= 64");
  NS_CHECK(bs <= KT, "block_size must be <= 32");
  a.q = reinterpret_cast<const bf16*>(q.data_ptr());
  a.k = reinterpret_cast<const bf16*>(k.data_ptr());
  a.v = reinterpret_cast<const bf16*>(v.data_ptr());
  a.ldk = k.stride(0);
  a.ldv = v.stride(0);
  a.anchors = anchors.data_ptr<int64_t>();
  a.keep = keep.data_ptr<bool>();
  a.scale = 1.f / sqrtf((float)q.size(3));
  return a;
}

template <int D>
static void fwd_d(AttnArgs a) {
  const int smem = 2 * D * KT * 4;
  dim3 grid(a.nb, a.Hk, a.b);
  attn_fwd_kernel<D><<<grid, 256, smem, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
}

template <int D>
static void bwd_d(AttnArgs a) {
  {
    const int smem = 3 * D * KT * 4;
    if (smem > 48 * 1024) NS_CUDA(cudaFuncSetAttribute(attn_bwd_dq_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    dim3 grid(a.nb, a.Hk, a.b);
    attn_bwd_dq_kernel<D><<<grid, 256, smem, stream()>>>(a);
    NS_CUDA(cudaGetLastError());
  }
  {
    const int smem = (2 * D * KT + 2 * 64 * D + 2 * 64 * KT) * 4;
    NS_CUDA(cudaFuncSetAttribute(attn_bwd_dkv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int tiles = (a.S + KT - 1) / KT + a.nb;
    dim3 grid(tiles, a.Hk, a.b);
    attn_bwd_dkv_kernel<D><<<grid, 128, smem, stream()>>>(a);
    NS_CUDA(cudaGetLastError());
  }
}

void attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs,
              at::Tensor out, at::Tensor lse) {
  AttnArgs a = make_args(q, k, v, anchors, keep, S, bs);
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
  a.dout = reinterpret_cast<const bf16*>(dout.data_ptr());
  a.o = reinterpret_cast<const bf16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
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
