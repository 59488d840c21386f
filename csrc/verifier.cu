// Frozen-verifier kernels (forward only): (1+w)-RMSNorm, gated RMSNorm, residual add,
// SiLU*up, causal depthwise conv + SiLU, GDN gates, and causal GQA attention with
// partial RoPE and a sigmoid output gate. The chunked gated delta rule is in
// gdn_fwd.cu.
//
// Casting follows the plain PyTorch statements of the same ops (compute dtype bf16,
// fp32 inside reductions), so results agree with the CPU path to bf16 resolution.
#include "common.h"
#include "sm100.cuh"

namespace ns {

using bf16 = __nv_bfloat16;
__device__ __forceinline__ float bf(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float rb(float x) { return sm100::bf16_round(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

__device__ float block_sum256(float v) {
  __shared__ float sh[8];
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = (threadIdx.x < 8) ? sh[threadIdx.x] : 0.f;
  if (threadIdx.x < 32) t = warp_sum(t);
  __shared__ float res;
  if (threadIdx.x == 0) res = t;
  __syncthreads();
  return res;
}

// ------------------------------------------------------------------ elementwise
__global__ void add_kernel(const bf16* __restrict__ a, const bf16* __restrict__ b, bf16* __restrict__ o, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    o[i] = __float2bfloat16(bf(a[i]) + bf(b[i]));
}

__global__ void silu_mul_kernel(const bf16* __restrict__ g, const bf16* __restrict__ u, bf16* __restrict__ o, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = bf(g[i]);
    o[i] = __float2bfloat16(rb(x / (1.f + expf(-x))) * bf(u[i]));
  }
}

// (1+w) RMSNorm, one block (256 threads) per row.
__global__ void qwen_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ y, int n,
                                 float eps) {
  const int64_t row = blockIdx.x;
  const bf16* xr = x + row * n;
  float ss = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float v = bf(xr[j]);
    ss += v * v;
  }
  const float inv = rsqrtf(block_sum256(ss) / n + eps);
  for (int j = threadIdx.x; j < n; j += blockDim.x) y[row * n + j] = __float2bfloat16(bf(xr[j]) * inv * (1.f + bf(w[j])));
}

// w * bf16(rmsnorm(x)) * silu(gate) ; rows of width n (<= 256), one warp per row.
__global__ void gated_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ gate, const bf16* __restrict__ w,
                                  bf16* __restrict__ y, int64_t rows, int n, float eps) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bf16* xr = x + row * n;
  float ss = 0.f;
  for (int j = lane; j < n; j += 32) {
    const float v = bf(xr[j]);
    ss += v * v;
  }
  const float inv = rsqrtf(warp_sum(ss) / n + eps);
  for (int j = lane; j < n; j += 32) {
    const float nv = rb(bf(xr[j]) * inv);
    const float gv = bf(gate[row * n + j]);
    const float sg = gv / (1.f + expf(-gv));
    y[row * n + j] = __float2bfloat16(rb(bf(w[j]) * nv) * sg);
  }
}

// out[b, t, c] = silu(sum_j w[c, j] * x[b, t - (K-1) + j, c]) ; x token-major [b, s, C].
__global__ void conv_silu_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ y, int s,
                                 int C, int K, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const int64_t bt = i / C;
    const int t = (int)(bt % s);
    const int64_t base = bt - t;  // b * s
    float acc = 0.f;
    for (int j = 0; j < K; ++j) {
      const int tt = t - (K - 1) + j;
      if (tt >= 0) acc += bf(w[c * K + j]) * bf(x[(base + tt) * C + c]);
    }
    const float z = rb(acc);
    y[i] = __float2bfloat16(z / (1.f + expf(-z)));
  }
}

// g = -exp(A_log) * softplus(a + dt_bias) ; beta = sigmoid(b)  over [rows, nv].
__global__ void gdn_gates_kernel(const bf16* __restrict__ a, const bf16* __restrict__ b, const float* __restrict__ alog,
                                 const float* __restrict__ dtb, float* __restrict__ g, bf16* __restrict__ beta,
                                 int nv, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int h = (int)(i % nv);
    const float z = bf(a[i]) + dtb[h];
    const float sp = z > 20.f ? z : log1pf(expf(z));
    g[i] = -expf(alog[h]) * sp;
    const float bv = bf(b[i]);
    beta[i] = __float2bfloat16(1.f / (1.f + expf(-bv)));
  }
}

// ------------------------------------------------------------------ causal attention (verifier)
// q [b, s, Hq, D], k/v [b, s, Hk, D] already (1+w)-normalised. Partial RoPE on the first
// rd channels of q and k (applied on load), causal GQA softmax in fp32, then
// out = bf16(o) * sigmoid(gate). One CTA per (16 query rows, head, batch row).
template <int D>
__global__ void __launch_bounds__(256) causal_attn_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                          const bf16* __restrict__ v, const bf16* __restrict__ gate,
                                                          const bf16* __restrict__ cs, const bf16* __restrict__ sn,
                                                          int rd, bf16* __restrict__ out, int s, int Hq, int Hk) {
  constexpr int QR = 16;   // query rows per CTA (2 per warp)
  constexpr int KT = 32;   // keys per tile
  constexpr int E = D / 32;
  extern __shared__ float sm[];
  float* Kt = sm;             // [D][KT]
  float* Vs = Kt + D * KT;    // [KT][D]
  const int qt = blockIdx.x, h = blockIdx.y, bi = blockIdx.z;
  const int hk = h / (Hq / Hk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const float scale = rsqrtf((float)D);
  const int q0 = qt * QR;
  constexpr int RPW = QR / 8;
  float qv[RPW][E], acc[RPW][E], mx[RPW], den[RPW];
  auto roped = [&](const bf16* base, int t, int d) -> float {
    // rope(x) = x*cos + rotate_half(x)*sin over the first rd channels (bf16 statement)
    const float x = bf(base[d]);
    if (d >= rd) return x;
    const int half = rd / 2;
    const float c = bf(cs[(int64_t)t * rd + d]), sv = bf(sn[(int64_t)t * rd + d]);
    const float rot = d < half ? -bf(base[d + half]) : bf(base[d - half]);
    return rb(rb(x * c) + rb(rot * sv));
  };
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr) {
    const int t = q0 + warp * RPW + rr;
    mx[rr] = -INFINITY;
    den[rr] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      acc[rr][e] = 0.f;
      qv[rr][e] = t < s ? roped(q + (((int64_t)bi * s + t) * Hq + h) * D, t, lane + 32 * e) * scale : 0.f;
    }
  }
  const int kend = min(s, q0 + QR);
  for (int k0 = 0; k0 < kend; k0 += KT) {
    const int cnt = min(KT, kend - k0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < KT * D; idx += blockDim.x) {
      const int kk = idx / D, d = idx % D;
      float kvv = 0.f, vvv = 0.f;
      if (kk < cnt) {
        const int t = k0 + kk;
        const bf16* kb = k + (((int64_t)bi * s + t) * Hk + hk) * D;
        kvv = roped(kb, t, d);
        vvv = bf(v[(((int64_t)bi * s + t) * Hk + hk) * D + d]);
      }
      Kt[d * KT + kk] = kvv;
      Vs[kk * D + d] = vvv;
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
      const int t = q0 + warp * RPW + rr;
      float sc = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
#pragma unroll 8
        for (int dd = 0; dd < 32; ++dd) sc += __shfl_sync(0xffffffff, qv[rr][e], dd) * Kt[(dd + 32 * e) * KT + lane];
      }
      const bool ok = lane < cnt && (k0 + lane) <= t;
      if (!ok) sc = -INFINITY;
      float tmax = sc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffff, tmax, o));
      if (tmax == -INFINITY) continue;
      const float nm = fmaxf(mx[rr], tmax);
      const float corr = expf(mx[rr] - nm);
      const float p = ok ? expf(sc - nm) : 0.f;
      den[rr] = den[rr] * corr + warp_sum(p);
      mx[rr] = nm;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[rr][e] *= corr;
      for (int kk = 0; kk < cnt; ++kk) {
        const float pk = __shfl_sync(0xffffffff, p, kk);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[rr][e] += pk * Vs[kk * D + lane + 32 * e];
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr) {
    const int t = q0 + warp * RPW + rr;
    if (t >= s) continue;
    const int64_t off = (((int64_t)bi * s + t) * Hq + h) * D;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int d = lane + 32 * e;
      const float o = rb(acc[rr][e] / den[rr]);
      const float gv = bf(gate[off + d]);
      out[off + d] = __float2bfloat16(o * rb(1.f / (1.f + expf(-gv))));
    }
  }
}

// ============================================================================ host
static int gridn(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16)); }
#define BP(t) reinterpret_cast<bf16*>((t).data_ptr())
#define CBP(t) reinterpret_cast<const bf16*>((t).data_ptr())

void add_bf16(at::Tensor a, at::Tensor b, at::Tensor o) {
  add_kernel<<<gridn(a.numel()), 256, 0, stream()>>>(CBP(a), CBP(b), BP(o), a.numel());
  NS_CUDA(cudaGetLastError());
}

void silu_mul(at::Tensor g, at::Tensor u, at::Tensor o) {
  silu_mul_kernel<<<gridn(g.numel()), 256, 0, stream()>>>(CBP(g), CBP(u), BP(o), g.numel());
  NS_CUDA(cudaGetLastError());
}

void qwen_norm(at::Tensor x, at::Tensor w, double eps, at::Tensor y) {
  NS_CHECK(x.is_contiguous() && y.is_contiguous(), "qwen_norm: contiguous rows expected");
  if (x.size(0) == 0) return;
  qwen_norm_kernel<<<x.size(0), 256, 0, stream()>>>(CBP(x), CBP(w), BP(y), x.size(1), (float)eps);
  NS_CUDA(cudaGetLastError());
}

void gated_norm(at::Tensor x, at::Tensor gate, at::Tensor w, double eps, at::Tensor y) {
  const int64_t rows = x.size(0);
  gated_norm_kernel<<<(rows * 32 + 255) / 256, 256, 0, stream()>>>(CBP(x), CBP(gate), CBP(w), BP(y), rows, x.size(1),
                                                                   (float)eps);
  NS_CUDA(cudaGetLastError());
}

void conv_silu(at::Tensor x, at::Tensor w, at::Tensor y) {
  NS_CHECK(x.dim() == 3 && x.is_contiguous(), "conv_silu: x [b, s, C] contiguous");
  const int s = x.size(1), C = x.size(2), K = w.size(1);
  conv_silu_kernel<<<gridn(x.numel()), 256, 0, stream()>>>(CBP(x), CBP(w), BP(y), s, C, K, x.numel());
  NS_CUDA(cudaGetLastError());
}

void gdn_gates(at::Tensor a, at::Tensor b, at::Tensor alog, at::Tensor dtb, at::Tensor g, at::Tensor beta) {
  const int nv = a.size(-1);
  gdn_gates_kernel<<<gridn(a.numel()), 256, 0, stream()>>>(CBP(a), CBP(b), alog.data_ptr<float>(),
                                                          dtb.data_ptr<float>(), g.data_ptr<float>(), BP(beta), nv,
                                                          a.numel());
  NS_CUDA(cudaGetLastError());
}

template <int D>
static void attn_launch(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor gate, at::Tensor cs, at::Tensor sn, int rd,
                        at::Tensor out) {
  const int b = q.size(0), s = q.size(1), Hq = q.size(2), Hk = k.size(2);
  const int smem = 2 * D * 32 * 4;
  if (smem > 48 * 1024) NS_CUDA(cudaFuncSetAttribute(causal_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  causal_attn_kernel<D><<<dim3((s + 15) / 16, Hq, b), 256, smem, stream()>>>(CBP(q), CBP(k), CBP(v), CBP(gate), CBP(cs),
                                                                             CBP(sn), rd, BP(out), s, Hq, Hk);
  NS_CUDA(cudaGetLastError());
}

void causal_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor gate, at::Tensor cs, at::Tensor sn, int64_t rd,
                     at::Tensor out) {
  NS_CHECK(cs.size(0) == q.size(1) && cs.size(1) == rd, "cos/sin must be [s, rotary_dim]");
  switch (q.size(3)) {
    case 32: attn_launch<32>(q, k, v, gate, cs, sn, rd, out); break;
    case 64: attn_launch<64>(q, k, v, gate, cs, sn, rd, out); break;
    case 128: attn_launch<128>(q, k, v, gate, cs, sn, rd, out); break;
    case 256: attn_launch<256>(q, k, v, gate, cs, sn, rd, out); break;
    default: NS_CHECK(false, "verifier attention head_dim must be 32, 64, 128 or 256");
  }
}

}  // namespace ns
