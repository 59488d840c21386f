// Backward of the gated delta rule (the reference has none: its verifier is frozen).
// Head dims 64 and 128 run the chunked kernels of gdn_bwd_chunk.cu; this file holds
// the token-serial kernels (head dims 16 and 32, or NANOSPEC_GDN_BWD=serial) and the
// per-key-head sum of dq / dk shared by both.
//
// Forward recurrence per (batch row, value head), state S [Dk x Dv] in fp32, with
// kn = k / sqrt(|k|^2 + 1e-6), qs = q / sqrt(|q|^2 + 1e-6) * Dk^-1/2:
//   St~ = e^{g_t} S_{t-1};  u_t = St~^T kn_t;  d_t = beta_t (v_t - u_t);
//   S_t = St~ + kn_t d_t^T;  o_t = S_t^T qs_t.
// Adjoint (reverse in t, dS = dL/dS_t):
//   dqs = S_t dO;  dS += qs dO^T;  dd = dS^T kn;  dkn = dS d;
//   dbeta = dd . (v - u);  dv = beta dd;  du = -beta dd;
//   dSt~ = dS + kn du^T;  dkn += St~ du;  dg = <St~, dSt~>;  dS_{t-1} = e^{g} dSt~
// then the L2-normalisation chain rule for q and k.
//
// Kernels:
//   gdn_ckpt_kernel : one CTA per (value head, row): runs the recurrence and stores S
//                     at every 64-token chunk start (fp32 checkpoints).
//   gdn_bwd_kernel  : one CTA per (value head, row): chunks in reverse; re-materialises
//                     the chunk's 64 token states into a per-CTA scratch, then walks
//                     the chunk backwards with S_t and dS in shared memory.
//   gdn_group_sum   : sums dq/dk over the value heads sharing a key head (fixed order).
#include <cstdlib>

#include "common.h"
#include "sm100.cuh"

namespace ns {

using bf16 = __nv_bfloat16;
constexpr int GC = 64;  // chunk length

__device__ __forceinline__ float bfv(bf16 x) { return __bfloat162float(x); }

// Normalised vector of length D into sh_out (fp32), returns 1/norm. One warp.
template <int D>
__device__ __forceinline__ float l2n_warp(const bf16* src, float* dst, float scale) {
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float x = bfv(src[d]);
    ss += x * x;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  const float r = rsqrtf(ss + 1e-6f);
  for (int d = lane; d < D; d += 32) dst[d] = bfv(src[d]) * r * scale;
  return r;
}

struct GdnArgs {
  const bf16 *q, *k, *v, *beta, *dout;
  const float* g;
  float* ckpt;     // [b, nv, nchunks, D, D]
  float* scratch;  // [b, nv, GC, D, D]  (per-CTA chunk states)
  float *dq, *dk;  // [b, s, nv, D] fp32 per value head
  bf16* dv;        // [b, s, nv, D]
  float *dg, *dbeta;  // [b, s, nv]
  int s, nk, nv, groups, nchunks;
};

// One token of the forward recurrence on S (smem, row stride P); writes u, d.
template <int D, int P>
__device__ __forceinline__ void token_forward(float* S, const float* kn, const float* vv, float eg, float bt,
                                              float* u, float* dd) {
  const int tid = threadIdx.x;
  if (tid < D) {
    float acc = 0.f;
    for (int i = 0; i < D; ++i) acc += S[i * P + tid] * kn[i];
    const float uu = eg * acc;
    u[tid] = uu;
    dd[tid] = bt * (vv[tid] - uu);
  }
  __syncthreads();
  for (int idx = tid; idx < D * D; idx += blockDim.x) {
    const int i = idx / D, j = idx % D;
    S[i * P + j] = eg * S[i * P + j] + kn[i] * dd[j];
  }
  __syncthreads();
}

template <int D>
__global__ void __launch_bounds__(256) gdn_ckpt_kernel(GdnArgs a) {
  constexpr int P = D + 1;
  extern __shared__ float sm[];
  float* S = sm;
  float* kn = S + D * P;
  float* vv = kn + D;
  float* u = vv + D;
  float* dd = u + D;
  const int h = blockIdx.x, bi = blockIdx.y, hk = h / a.groups;
  const int tid = threadIdx.x;
  for (int idx = tid; idx < D * P; idx += blockDim.x) S[idx] = 0.f;
  __syncthreads();
  float* ck = a.ckpt + ((int64_t)bi * a.nv + h) * a.nchunks * D * D;
  for (int t = 0; t < a.s; ++t) {
    if (t % GC == 0) {
      float* dst = ck + (int64_t)(t / GC) * D * D;
      for (int idx = tid; idx < D * D; idx += blockDim.x) dst[idx] = S[(idx / D) * P + idx % D];
    }
    const int64_t tok = (int64_t)bi * a.s + t;
    if (tid < 32) l2n_warp<D>(a.k + (tok * a.nk + hk) * D, kn, 1.f);
    for (int d = tid; d < D; d += blockDim.x) vv[d] = bfv(a.v[(tok * a.nv + h) * D + d]);
    __syncthreads();
    token_forward<D, P>(S, kn, vv, expf(a.g[tok * a.nv + h]), bfv(a.beta[tok * a.nv + h]), u, dd);
  }
}

template <int D>
__global__ void __launch_bounds__(256) gdn_bwd_kernel(GdnArgs a) {
  constexpr int P = D + 1;
  extern __shared__ float sm[];
  float* S = sm;            // running / loaded state [D][P]
  float* dS = S + D * P;    // [D][P]
  float* U = dS + D * P;    // [GC][D] u_t of the chunk
  float* DD = U + GC * D;   // [GC][D] d_t of the chunk
  float* kn = DD + GC * D;  // [D]
  float* qs = kn + D;
  float* vv = qs + D;
  float* dO = vv + D;
  float* dd = dO + D;  // dd (adjoint of d) / du scratch
  float* dkn = dd + D;
  float* dqs = dkn + D;
  float* red = dqs + D;  // [32] reduction scratch
  const int h = blockIdx.x, bi = blockIdx.y, hk = h / a.groups;
  const int tid = threadIdx.x, nt = blockDim.x;
  const float qscale = rsqrtf((float)D);
  const int64_t cta = (int64_t)bi * a.nv + h;
  const float* ck = a.ckpt + cta * a.nchunks * D * D;
  float* sc = a.scratch + cta * (int64_t)GC * D * D;
  for (int idx = tid; idx < D * P; idx += nt) dS[idx] = 0.f;
  for (int c = a.nchunks - 1; c >= 0; --c) {
    const int t0 = c * GC;
    const int cnt = min(GC, a.s - t0);
    __syncthreads();
    // re-materialise the chunk's token states S_t (after update) into the scratch
    for (int idx = tid; idx < D * D; idx += nt) S[(idx / D) * P + idx % D] = ck[(int64_t)c * D * D + idx];
    __syncthreads();
    for (int r = 0; r < cnt; ++r) {
      const int64_t tok = (int64_t)bi * a.s + t0 + r;
      if (tid < 32) l2n_warp<D>(a.k + (tok * a.nk + hk) * D, kn, 1.f);
      for (int d = tid; d < D; d += nt) vv[d] = bfv(a.v[(tok * a.nv + h) * D + d]);
      __syncthreads();
      token_forward<D, P>(S, kn, vv, expf(a.g[tok * a.nv + h]), bfv(a.beta[tok * a.nv + h]), U + r * D, DD + r * D);
      float* dst = sc + (int64_t)r * D * D;
      for (int idx = tid; idx < D * D; idx += nt) dst[idx] = S[(idx / D) * P + idx % D];
    }
    __syncthreads();
    // reverse walk
    for (int r = cnt - 1; r >= 0; --r) {
      const int64_t tok = (int64_t)bi * a.s + t0 + r;
      const float eg = expf(a.g[tok * a.nv + h]);
      const float bt = bfv(a.beta[tok * a.nv + h]);
      const float* Ut = U + r * D;
      const float* Dt = DD + r * D;
      float rq = 0.f, rk = 0.f;
      if (tid < 32) {
        rq = l2n_warp<D>(a.q + (tok * a.nk + hk) * D, qs, qscale);
      } else if (tid < 64) {
        rk = l2n_warp<D>(a.k + (tok * a.nk + hk) * D, kn, 1.f);
      }
      for (int d = tid; d < D; d += nt) {
        vv[d] = bfv(a.v[(tok * a.nv + h) * D + d]);
        dO[d] = bfv(a.dout[(tok * a.nv + h) * D + d]);
      }
      const float* St = sc + (int64_t)r * D * D;
      for (int idx = tid; idx < D * D; idx += nt) S[(idx / D) * P + idx % D] = St[idx];
      __syncthreads();
      // (1) dqs = S_t dO ; (2) dS += qs dO^T
      if (tid < D) {
        float acc = 0.f;
        for (int j = 0; j < D; ++j) acc += S[tid * P + j] * dO[j];
        dqs[tid] = acc;
      }
      for (int idx = tid; idx < D * D; idx += nt) {
        const int i = idx / D, j = idx % D;
        dS[i * P + j] += qs[i] * dO[j];
      }
      __syncthreads();
      // (3) dd = dS^T kn ; dkn = dS d
      if (tid < D) {
        float acc = 0.f;
        for (int i = 0; i < D; ++i) acc += dS[i * P + tid] * kn[i];
        dd[tid] = acc;
      } else if (tid >= 128 && tid - 128 < D) {
        const int i = tid - 128;
        float acc = 0.f;
        for (int j = 0; j < D; ++j) acc += dS[i * P + j] * Dt[j];
        dkn[i] = acc;
      }
      __syncthreads();
      // (4) dbeta, dv, du (du stored back into dd)
      float part = 0.f;
      if (tid < D) {
        part = dd[tid] * (vv[tid] - Ut[tid]);
        a.dv[(tok * a.nv + h) * D + tid] = __float2bfloat16(bt * dd[tid]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffff, part, o);
      if ((tid & 31) == 0) red[tid >> 5] = part;
      __syncthreads();
      if (tid == 0) {
        float sum = 0.f;
        for (int w = 0; w < (nt >> 5); ++w) sum += red[w];
        a.dbeta[tok * a.nv + h] = sum;
      }
      if (tid < D) dd[tid] = -bt * dd[tid];  // du
      __syncthreads();
      // (5) dkn += St~ du with St~ = S_t - kn d^T ; dSt~ = dS + kn du^T
      if (tid < D) {
        float acc = 0.f, dd_du = 0.f;
        for (int j = 0; j < D; ++j) {
          acc += S[tid * P + j] * dd[j];
          dd_du += Dt[j] * dd[j];
        }
        dkn[tid] += acc - kn[tid] * dd_du;
      }
      float gpart = 0.f;
      for (int idx = tid; idx < D * D; idx += nt) {
        const int i = idx / D, j = idx % D;
        const float dst = dS[i * P + j] + kn[i] * dd[j];
        const float stt = S[i * P + j] - kn[i] * Dt[j];
        gpart += stt * dst;
        dS[i * P + j] = eg * dst;  // (6) dS_{t-1}
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) gpart += __shfl_xor_sync(0xffffffff, gpart, o);
      __syncthreads();
      if ((tid & 31) == 0) red[tid >> 5] = gpart;
      __syncthreads();
      if (tid == 0) {
        float sum = 0.f;
        for (int w = 0; w < (nt >> 5); ++w) sum += red[w];
        a.dg[tok * a.nv + h] = sum;
      }
      // L2-normalisation chain rule: dx = r (dy - y (y . dy)), y = x r
      if (tid < 32) {
        // q: y = qs / qscale ; dy = dqs * qscale
        float dot = 0.f;
        for (int d = tid; d < D; d += 32) dot += (qs[d] / qscale) * (dqs[d] * qscale);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffff, dot, o);
        for (int d = tid; d < D; d += 32)
          a.dq[(tok * a.nv + h) * D + d] = rq * (dqs[d] * qscale - (qs[d] / qscale) * dot);
      } else if (tid < 64) {
        const int l = tid - 32;
        float dot = 0.f;
        for (int d = l; d < D; d += 32) dot += kn[d] * dkn[d];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffff, dot, o);
        for (int d = l; d < D; d += 32) a.dk[(tok * a.nv + h) * D + d] = rk * (dkn[d] - kn[d] * dot);
      }
      __syncthreads();
    }
  }
}

// dq/dk per key head: sum over its `groups` value heads in head order.
__global__ void gdn_group_sum_kernel(const float* __restrict__ src, bf16* __restrict__ dst, int64_t tokens, int nk,
                                     int groups, int D) {
  const int64_t total = tokens * nk * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const int64_t th = i / D;
    const int hk = (int)(th % nk);
    const int64_t t = th / nk;
    float acc = 0.f;
    for (int gi = 0; gi < groups; ++gi) acc += src[((t * (int64_t)nk * groups) + hk * groups + gi) * D + d];
    dst[i] = __float2bfloat16(acc);
  }
}

template <int D>
static void gdn_bwd_launch(GdnArgs a, int b) {
  constexpr int P = D + 1;
  const int smem_ck = (D * P + 4 * D) * 4;
  const int smem_bw = (2 * D * P + 2 * GC * D + 7 * D + 32) * 4;
  NS_CUDA(cudaFuncSetAttribute(gdn_ckpt_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_ck));
  NS_CUDA(cudaFuncSetAttribute(gdn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bw));
  dim3 grid(a.nv, b);
  gdn_ckpt_kernel<D><<<grid, 256, smem_ck, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
  gdn_bwd_kernel<D><<<grid, 256, smem_bw, stream()>>>(a);
  NS_CUDA(cudaGetLastError());
}

// q, k [b, s, nk, D]; v, dout [b, s, nv, D]; g fp32 [b, s, nv]; beta [b, s, nv].
// Returns dq, dk [b, s, nk, D] bf16; dv [b, s, nv, D] bf16; dg, dbeta [b, s, nv] fp32.
bool gdn_bwd_chunked(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta, at::Tensor dout,
                     int64_t groups, at::Tensor dq32, at::Tensor dk32, at::Tensor dv, at::Tensor dg, at::Tensor dbeta);

std::vector<at::Tensor> gdn_chunk_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta,
                                      at::Tensor dout, int64_t groups) {
  NS_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && g.is_contiguous() && beta.is_contiguous() &&
               dout.is_contiguous(),
           "gdn_chunk_bwd: contiguous inputs expected");
  const int b = q.size(0), s = q.size(1), nk = q.size(2), D = q.size(3), nv = v.size(2);
  NS_CHECK(v.size(3) == D && nv == nk * groups, "gdn_chunk_bwd: d_k == d_v and nv == nk * groups expected");
  const int nchunks = (s + GC - 1) / GC;
  auto f32 = q.options().dtype(at::kFloat);
  auto dq32 = at::empty({b, s, nv, D}, f32);
  auto dk32 = at::empty({b, s, nv, D}, f32);
  auto dv = at::empty({b, s, nv, D}, q.options());
  auto dg = at::empty({b, s, nv}, f32);
  auto dbeta = at::empty({b, s, nv}, f32);
  // head dims 64 / 128: the chunked kernels; NANOSPEC_GDN_BWD=serial keeps the
  // token-serial ones (the only path for 16 / 32)
  const char* mode = std::getenv("NANOSPEC_GDN_BWD");
  const bool serial = mode && std::string(mode) == "serial";
  if (!serial && gdn_bwd_chunked(q, k, v, g, beta, dout, groups, dq32, dk32, dv, dg, dbeta)) {
    auto dq = at::empty({b, s, nk, D}, q.options());
    auto dk = at::empty({b, s, nk, D}, q.options());
    const int64_t tot = (int64_t)b * s * nk * D;
    const int blocks = (int)std::min<int64_t>((tot + 255) / 256, (int64_t)num_sms() * 8);
    gdn_group_sum_kernel<<<blocks, 256, 0, stream()>>>(dq32.data_ptr<float>(), reinterpret_cast<bf16*>(dq.data_ptr()),
                                                       (int64_t)b * s, nk, (int)groups, D);
    gdn_group_sum_kernel<<<blocks, 256, 0, stream()>>>(dk32.data_ptr<float>(), reinterpret_cast<bf16*>(dk.data_ptr()),
                                                       (int64_t)b * s, nk, (int)groups, D);
    NS_CUDA(cudaGetLastError());
    return {dq, dk, dv, dg, dbeta};
  }
  auto ckpt = at::empty({(int64_t)b * nv * nchunks * D * D}, f32);
  auto scratch = at::empty({(int64_t)b * nv * GC * D * D}, f32);
  GdnArgs a{};
  a.q = reinterpret_cast<const bf16*>(q.data_ptr());
  a.k = reinterpret_cast<const bf16*>(k.data_ptr());
  a.v = reinterpret_cast<const bf16*>(v.data_ptr());
  a.beta = reinterpret_cast<const bf16*>(beta.data_ptr());
  a.dout = reinterpret_cast<const bf16*>(dout.data_ptr());
  a.g = g.data_ptr<float>();
  a.ckpt = ckpt.data_ptr<float>();
  a.scratch = scratch.data_ptr<float>();
  a.dq = dq32.data_ptr<float>();
  a.dk = dk32.data_ptr<float>();
  a.dv = reinterpret_cast<bf16*>(dv.data_ptr());
  a.dg = dg.data_ptr<float>();
  a.dbeta = dbeta.data_ptr<float>();
  a.s = s;
  a.nk = nk;
  a.nv = nv;
  a.groups = (int)groups;
  a.nchunks = nchunks;
  switch (D) {
    case 16: gdn_bwd_launch<16>(a, b); break;
    case 32: gdn_bwd_launch<32>(a, b); break;
    case 64: gdn_bwd_launch<64>(a, b); break;
    case 128: gdn_bwd_launch<128>(a, b); break;
    default: NS_CHECK(false, "gated delta rule head dim must be 16, 32, 64 or 128");
  }
  auto dq = at::empty({b, s, nk, D}, q.options());
  auto dk = at::empty({b, s, nk, D}, q.options());
  const int64_t tot = (int64_t)b * s * nk * D;
  const int blocks = (int)std::min<int64_t>((tot + 255) / 256, (int64_t)num_sms() * 8);
  gdn_group_sum_kernel<<<blocks, 256, 0, stream()>>>(dq32.data_ptr<float>(), reinterpret_cast<bf16*>(dq.data_ptr()),
                                                     (int64_t)b * s, nk, (int)groups, D);
  gdn_group_sum_kernel<<<blocks, 256, 0, stream()>>>(dk32.data_ptr<float>(), reinterpret_cast<bf16*>(dk.data_ptr()),
                                                     (int64_t)b * s, nk, (int)groups, D);
  NS_CUDA(cudaGetLastError());
  return {dq, dk, dv, dg, dbeta};
}

}  // namespace ns
