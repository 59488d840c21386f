// RMSNorm, per-head RMSNorm + RoPE, SwiGLU and embedding kernels (forward and
// backward). Casting points reproduce the compute-dtype rounding of the plain
// PyTorch statements (normalise in fp32, round to bf16, multiply by the weight
// and round again), so the kernels agree with the CPU path to bf16 resolution.
// Weight-gradient column sums use per-block partials plus a fixed-order final
// reduction: results are bitwise reproducible run to run.
#include <vector>

#include "common.h"
#include "sm100.cuh"

namespace ns {

using bf16 = __nv_bfloat16;
__device__ __forceinline__ float f(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float r(float x) { return sm100::bf16_round(x); }

template <int N>
__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = (l < N / 32) ? sh[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffff, t, o);
    if (l == 0) sh[0] = t;
  }
  __syncthreads();
  return sh[0];
}

// ------------------------------------------------------------------ RMSNorm forward
// One block per row. y = bf16(w * bf16(x * inv)), inv = rsqrt(mean(x^2) + eps).
__global__ void rms_fwd_kernel(const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ w,
                               bf16* __restrict__ y, int64_t ldy, float* __restrict__ inv_out, int n,
                               float eps) {
  __shared__ float sh[32];
  const int64_t row = blockIdx.x;
  const bf16* xr = x + row * ldx;
  float ss = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float v = f(xr[j]);
    ss += v * v;
  }
  const float tot = block_sum<256>(ss, sh);
  const float inv = rsqrtf(tot / n + eps);
  if (threadIdx.x == 0) inv_out[row] = inv;
  bf16* yr = y + row * ldy;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float nv = r(f(xr[j]) * inv);
    yr[j] = __float2bfloat16(f(w[j]) * nv);
  }
}

// Same result as rms_fwd_kernel for rows of n % 8 == 0 elements (n <= 8 * 256 * VPT):
// the row stays in registers after one pass of 16-byte loads (no second read).
template <int VPT>
__global__ void __launch_bounds__(256) rms_fwd_vec_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                          const bf16* __restrict__ w, bf16* __restrict__ y,
                                                          int64_t ldy, float* __restrict__ inv_out, int n,
                                                          float eps) {
  __shared__ float sh[32];
  const int64_t row = blockIdx.x;
  const int n8 = n / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  uint4 xv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = threadIdx.x + v * 256;
    if (c < n8) xv[v] = xr[c];
  }
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = threadIdx.x + v * 256;
    if (c < n8) {
      const bf16* h = reinterpret_cast<const bf16*>(&xv[v]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f(h[j]) * f(h[j]);
    }
  }
  const float tot = block_sum<256>(ss, sh);
  const float inv = rsqrtf(tot / n + eps);
  if (threadIdx.x == 0) inv_out[row] = inv;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * ldy);
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int c = threadIdx.x + v * 256;
    if (c < n8) {
      const uint4 wv = wr[c];
      const bf16* h = reinterpret_cast<const bf16*>(&xv[v]);
      const bf16* wh = reinterpret_cast<const bf16*>(&wv);
      uint4 o;
      bf16* oh = reinterpret_cast<bf16*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) oh[j] = __float2bfloat16(f(wh[j]) * r(f(h[j]) * inv));
      yr[c] = o;
    }
  }
}

// ------------------------------------------------------------------ RMSNorm backward
// Blocks take `rows_per_block` rows each; dx per row, dw partial per block.
__global__ void rms_bwd_kernel(const bf16* __restrict__ dy, int64_t lddy, const bf16* __restrict__ x,
                               int64_t ldx, const float* __restrict__ inv, const bf16* __restrict__ w,
                               bf16* __restrict__ dx, int64_t lddx, const bf16* __restrict__ res,
                               int64_t ldres, float* __restrict__ dw_part, int rows, int n,
                               int rows_per_block) {
  __shared__ float sh[32];
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(r0 + rows_per_block, rows);
  // Column partials for dw: this thread owns columns threadIdx.x + k*blockDim.x.
  constexpr int MAXC = 40;  // up to 10240 columns with 256 threads
  float acc[MAXC];
#pragma unroll
  for (int k = 0; k < MAXC; ++k) acc[k] = 0.f;
  for (int row = r0; row < r1; ++row) {
    const bf16* dyr = dy + (int64_t)row * lddy;
    const bf16* xr = x + (int64_t)row * ldx;
    const float iv = inv[row];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < MAXC; ++k) {
      const int j = threadIdx.x + k * blockDim.x;
      if (j < n) {
        const float xv = f(xr[j]);
        const float d = f(dyr[j]);
        acc[k] += d * r(xv * iv);
        const float dz = r(d * f(w[j]));
        dot += dz * xv;
      }
    }
    const float dinv = block_sum<256>(dot, sh);
    const float dvar = dinv * (-0.5f * iv * iv * iv);
    const float c2 = 2.f * dvar / n;
    bf16* dxr = dx + (int64_t)row * lddx;
#pragma unroll
    for (int k = 0; k < MAXC; ++k) {
      const int j = threadIdx.x + k * blockDim.x;
      if (j < n) {
        const float xv = f(xr[j]);
        const float dz = r(f(dyr[j]) * f(w[j]));
        float g = r(dz * iv + c2 * xv);
        if (res) g = r(f(res[(int64_t)row * ldres + j]) + g);
        dxr[j] = __float2bfloat16(g);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < MAXC; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    if (j < n) dw_part[(int64_t)blockIdx.x * n + j] = acc[k];
  }
}

// Sum `parts` partial rows of length n in fixed order and cast to bf16.
__global__ void colsum_kernel(const float* __restrict__ part, int parts, int n, bf16* __restrict__ out) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += part[(int64_t)p * n + j];
  out[j] = __float2bfloat16(s);
}

// ------------------------------------------------------------------ head RMSNorm + RoPE
// Rows are (token, head) pairs of length D. A group of G = min(32, D/2) lanes owns
// one row; lane g holds the rotation pairs (g + p*G, g + p*G + D/2), p < P = D/(2G).
template <int D>
__global__ void head_norm_rope_fwd_kernel(const bf16* __restrict__ x, int64_t ldx, int H,
                                          const bf16* __restrict__ w, const bf16* __restrict__ cs,
                                          const bf16* __restrict__ sn, bf16* __restrict__ y,
                                          float* __restrict__ inv_out, int rows, float eps) {
  constexpr int G = D / 2 < 32 ? D / 2 : 32;
  constexpr int P = D / (2 * G);
  constexpr int RPW = 32 / G;  // rows per warp
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int row = gw * RPW + lane / G;
  const int g = lane % G;
  const bool active = row < rows;
  const int t = active ? row / H : 0, h = active ? row % H : 0;
  const bf16* xr = x + (int64_t)t * ldx + (int64_t)h * D;
  float a[P], b[P];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const int j = g + p * G;
    a[p] = active ? f(xr[j]) : 0.f;
    b[p] = active ? f(xr[j + D / 2]) : 0.f;
    ss += a[p] * a[p] + b[p] * b[p];
  }
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  const float inv = rsqrtf(ss / D + eps);
  if (!active) return;
  if (g == 0) inv_out[row] = inv;
  const bf16* cr = cs + (int64_t)t * D;
  const bf16* sr = sn + (int64_t)t * D;
  bf16* yr = y + (int64_t)row * D;
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const int j = g + p * G;
    const float na = r(f(w[j]) * r(a[p] * inv));
    const float nb = r(f(w[j + D / 2]) * r(b[p] * inv));
    // rope: x*cos + rotate_half(x)*sin, rotate_half(x) = (-x2, x1)
    const float ya = r(r(na * f(cr[j])) + r(-nb * f(sr[j])));
    const float yb = r(r(nb * f(cr[j + D / 2])) + r(na * f(sr[j + D / 2])));
    yr[j] = __float2bfloat16(ya);
    yr[j + D / 2] = __float2bfloat16(yb);
  }
}

template <int D>
__global__ void head_norm_rope_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                          int64_t ldx, int H, const float* __restrict__ inv,
                                          const bf16* __restrict__ w, const bf16* __restrict__ cs,
                                          const bf16* __restrict__ sn, bf16* __restrict__ dx,
                                          int64_t lddx, float* __restrict__ dw_part, int rows) {
  constexpr int G = D / 2 < 32 ? D / 2 : 32;
  constexpr int P = D / (2 * G);
  constexpr int RPW = 32 / G;
  __shared__ float dws[D];
  for (int j = threadIdx.x; j < D; j += blockDim.x) dws[j] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int g = lane % G;
  float dwa[P], dwb[P];
#pragma unroll
  for (int p = 0; p < P; ++p) dwa[p] = dwb[p] = 0.f;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const int warp_id = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  for (int base = warp_id * RPW; base < rows; base += warps_total * RPW) {
    const int row = base + lane / G;
    const bool active = row < rows;
    const int t = active ? row / H : 0, h = active ? row % H : 0;
    const bf16* xr = x + (int64_t)t * ldx + (int64_t)h * D;
    const bf16* dyr = dy + (int64_t)row * D;
    const bf16* cr = cs + (int64_t)t * D;
    const bf16* sr = sn + (int64_t)t * D;
    const float iv = active ? inv[row] : 0.f;
    float da[P], db[P], xa[P], xb[P];
    float dot = 0.f;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int j = g + p * G;
      float ga = active ? f(dyr[j]) : 0.f, gb = active ? f(dyr[j + D / 2]) : 0.f;
      xa[p] = active ? f(xr[j]) : 0.f;
      xb[p] = active ? f(xr[j + D / 2]) : 0.f;
      // rope backward: dy*cos - rotate_half(dy*sin); rotate_half(u) = (-u2, u1)
      const float ua = r(ga * f(sr[j])), ub = r(gb * f(sr[j + D / 2]));
      da[p] = r(r(ga * f(cr[j])) + ub);          // - (-ub)
      db[p] = r(r(gb * f(cr[j + D / 2])) - ua);
      dwa[p] += da[p] * r(xa[p] * iv);
      dwb[p] += db[p] * r(xb[p] * iv);
      dot += r(da[p] * f(w[j])) * xa[p] + r(db[p] * f(w[j + D / 2])) * xb[p];
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffff, dot, o);
    if (!active) continue;
    const float c2 = 2.f * dot * (-0.5f * iv * iv * iv) / D;
    bf16* dxr = dx + (int64_t)t * lddx + (int64_t)h * D;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int j = g + p * G;
      dxr[j] = __float2bfloat16(r(r(da[p] * f(w[j])) * iv + c2 * xa[p]));
      dxr[j + D / 2] = __float2bfloat16(r(r(db[p] * f(w[j + D / 2])) * iv + c2 * xb[p]));
    }
  }
  // Fixed-order reduction of the lanes' column partials inside the block.
  for (int gi = 0; gi < 32 / G * (blockDim.x >> 5); ++gi) {
    if ((threadIdx.x / G) == gi) {
#pragma unroll
      for (int p = 0; p < P; ++p) {
        dws[g + p * G] += dwa[p];
        dws[g + p * G + D / 2] += dwb[p];
      }
    }
    __syncthreads();
  }
  for (int j = threadIdx.x; j < D; j += blockDim.x) dw_part[(int64_t)blockIdx.x * D + j] = dws[j];
}

// ------------------------------------------------------------------ SwiGLU
__device__ __forceinline__ float silu_f(float g) { return g / (1.f + expf(-g)); }

__global__ void swiglu_fwd_kernel(const bf16* __restrict__ gu, bf16* __restrict__ out, int64_t rows, int m) {
  const int64_t total = rows * m;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / m;
    const int j = (int)(i % m);
    const float g = f(gu[t * 2 * m + j]), u = f(gu[t * 2 * m + m + j]);
    out[i] = __float2bfloat16(r(silu_f(g)) * u);
  }
}

__global__ void swiglu_bwd_kernel(const bf16* __restrict__ dp, const bf16* __restrict__ gu,
                                  bf16* __restrict__ dgu, int64_t rows, int m) {
  const int64_t total = rows * m;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / m;
    const int j = (int)(i % m);
    const float g = f(gu[t * 2 * m + j]), u = f(gu[t * 2 * m + m + j]), d = f(dp[i]);
    const float s = 1.f / (1.f + expf(-g));
    const float du = r(d * u);
    dgu[t * 2 * m + j] = __float2bfloat16(du * (s * (1.f + g * (1.f - s))));
    dgu[t * 2 * m + m + j] = __float2bfloat16(d * r(g * s));
  }
}

// ------------------------------------------------------------------ embedding
// Token ids outside [0, rows) are not read: the row is written as zeros and the
// device error word records code 3 (the host raises; see utils/health.py).
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ w, int d,
                                     bf16* __restrict__ out, int64_t n, int64_t rows, int* err) {
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  bf16* dst = out + t * d;
  if (id < 0 || id >= rows) {
    if (threadIdx.x == 0) atomicExch(err, 3);
    for (int j = threadIdx.x; j < d; j += blockDim.x) dst[j] = __float2bfloat16(0.f);
    return;
  }
  const bf16* src = w + id * (int64_t)d;
  if ((d % 8) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int j = threadIdx.x; j < d / 8; j += blockDim.x) d4[j] = s4[j];
  } else {
    for (int j = threadIdx.x; j < d; j += blockDim.x) dst[j] = src[j];
  }
}

// grad[ids[i]] += dy[i] in token order; one thread per column: deterministic, no atomics.
__global__ void embedding_bwd_kernel(const bf16* __restrict__ dy, const int64_t* __restrict__ ids,
                                     int64_t tokens, int d, bf16* __restrict__ grad, int64_t rows, int* err) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  for (int64_t i = 0; i < tokens; ++i) {
    const int64_t id = ids[i];
    if (id < 0 || id >= rows) {  // out of range: skipped, code 3 (see embedding_fwd_kernel)
      if (c == 0) atomicExch(err, 3);
      continue;
    }
    bf16* p = grad + id * (int64_t)d + c;
    *p = __float2bfloat16(f(*p) + f(dy[i * d + c]));
  }
}

// ------------------------------------------------------------------ optimizer
// sum over the shard of bf16(g * factor)^2: per-block partial, fixed-order final sum.
// 8 bf16 (16 bytes) per thread per iteration.
__global__ void grad_norm_part_kernel(const bf16* __restrict__ g, int64_t n, const float* __restrict__ factor,
                                      float* __restrict__ part) {
  __shared__ float sh[32];
  const float fac = *factor;
  float s = 0.f;
  // elements before the first 16-byte boundary (ranges inside a shard), then 8 at a time
  const int64_t lead_want = (int64_t)(((16 - (reinterpret_cast<uintptr_t>(g) & 15)) & 15) / 2);
  const int64_t lead = n < lead_want ? n : lead_want;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < lead; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = r(f(g[i]) * fac);
    s += v * v;
  }
  g += lead;
  n -= lead;
  const int64_t n8 = n / 8;
  const uint4* g8 = reinterpret_cast<const uint4*>(g);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 raw = g8[i];
    const bf16* h = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = r(f(h[j]) * fac);
      s += v * v;
    }
  }
  for (int64_t i = n8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = r(f(g[i]) * fac);
    s += v * v;
  }
  const float t = block_sum<256>(s, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = t;
}

// The same squared norm over up to NR separate gradient ranges in one launch: block
// b works on range r with block_start[r] <= b < block_start[r + 1] (host-assigned in
// proportion to the range sizes) and writes part[b].
constexpr int NR = 64;
struct NormRanges {
  const bf16* p[NR];
  int64_t n[NR];
  int block_start[NR + 1];
  int count;
};

__global__ void grad_norm_ranges_kernel(NormRanges rs, const float* __restrict__ factor, float* __restrict__ part) {
  __shared__ float sh[32];
  int ri = 0;
  while (ri + 1 < rs.count && (int)blockIdx.x >= rs.block_start[ri + 1]) ++ri;
  const int lb = blockIdx.x - rs.block_start[ri], nb = rs.block_start[ri + 1] - rs.block_start[ri];
  const float fac = *factor;
  const bf16* g = rs.p[ri];
  int64_t n = rs.n[ri];
  float s = 0.f;
  const int64_t lead_want = (int64_t)(((16 - (reinterpret_cast<uintptr_t>(g) & 15)) & 15) / 2);
  const int64_t lead = n < lead_want ? n : lead_want;
  const int64_t stride = (int64_t)nb * blockDim.x;
  const int64_t t0 = (int64_t)lb * blockDim.x + threadIdx.x;
  for (int64_t i = t0; i < lead; i += stride) {
    const float v = r(f(g[i]) * fac);
    s += v * v;
  }
  g += lead;
  n -= lead;
  const int64_t n8 = n / 8;
  const uint4* g8 = reinterpret_cast<const uint4*>(g);
  for (int64_t i = t0; i < n8; i += stride) {
    const uint4 raw = g8[i];
    const bf16* h = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = r(f(h[j]) * fac);
      s += v * v;
    }
  }
  for (int64_t i = n8 * 8 + t0; i < n; i += stride) {
    const float v = r(f(g[i]) * fac);
    s += v * v;
  }
  const float t = block_sum<256>(s, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = t;
}

__global__ void sum_into_kernel(const float* __restrict__ part, int parts, float* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < parts; ++i) s += part[i];
    out[0] += s;
  }
}

struct AdamHyper {
  float lr, wd, b1, b2, eps, bc1, bc2, max_norm;
  const float* bc;  // when set: device-resident {bc1, bc2} (overrides the fields above)
};

// Device-side step bookkeeping: if the global norm is finite, step += 1; then the
// bias corrections of the (new) step, in double precision: bc = {1 - b1^t, sqrt(1 - b2^t)}.
__global__ void adam_prepare_kernel(const float* __restrict__ norm2, long long* __restrict__ step, double b1,
                                    double b2, float* __restrict__ bc) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const bool finite = isfinite(sqrtf(*norm2));
  const long long t = *step + (finite ? 1 : 0);
  if (finite) *step = t;
  const double tt = (double)(t > 0 ? t : 1);
  bc[0] = (float)(1.0 - pow(b1, tt));
  bc[1] = (float)sqrt(1.0 - pow(b2, tt));
}

__device__ __forceinline__ void adam_one(float g, float& w, float& mm, float& vv, float decay, float step,
                                         const AdamHyper& h) {
  mm = mm + (1.f - h.b1) * (g - mm);
  vv = h.b2 * vv + (1.f - h.b2) * g * g;
  const float denom = sqrtf(vv) / h.bc2 + h.eps;
  w = w * decay - step * (mm / denom);
}

// Fused AdamW over one flat shard: reads grad (bf16), master/m/v (fp32); writes
// master/m/v, param (bf16) and zeroes grad unless `zero_grad` is 0 (the caller
// guarantees the next backward overwrites every element). 4 elements per thread per iteration
// (16-byte fp32 and 8-byte bf16 accesses). Skips the update (but still zeroes the
// gradient) when the global norm in device memory is not finite.
__global__ void __launch_bounds__(256, 4) adamw_kernel(bf16* __restrict__ param, float* __restrict__ master,
                                                    float* __restrict__ m, float* __restrict__ v,
                                                    bf16* __restrict__ grad, int64_t n,
                                                    const float* __restrict__ factor,
                                                    const float* __restrict__ norm2, AdamHyper h,
                                                    int zero_grad) {
  const float norm = sqrtf(*norm2);
  const bool finite = isfinite(norm);
  const float clip = finite ? fminf(1.f, h.max_norm / (norm + 1e-6f)) : 0.f;
  const float fac = *factor;
  const float decay = 1.f - h.lr * h.wd;
  if (h.bc) {
    h.bc1 = h.bc[0];
    h.bc2 = h.bc[1];
  }
  const float step = h.lr / h.bc1;
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float4* M4 = reinterpret_cast<float4*>(master);
  float4* m4 = reinterpret_cast<float4*>(m);
  float4* v4 = reinterpret_cast<float4*>(v);
  uint2* g4 = reinterpret_cast<uint2*>(grad);
  uint2* p4 = reinterpret_cast<uint2*>(param);
  // Two groups of 4 per iteration: all ten loads are issued before any arithmetic.
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < n4; i0 += 2 * stride) {
    const int64_t i1 = i0 + stride;
    const bool has1 = i1 < n4;
    if (finite) {
      uint2 graw[2];
      float4 W[2], MM[2], VV[2];
      graw[0] = __ldcs(g4 + i0);
      W[0] = __ldcs(M4 + i0);
      MM[0] = __ldcs(m4 + i0);
      VV[0] = __ldcs(v4 + i0);
      if (has1) {
        graw[1] = __ldcs(g4 + i1);
        W[1] = __ldcs(M4 + i1);
        MM[1] = __ldcs(m4 + i1);
        VV[1] = __ldcs(v4 + i1);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u == 1 && !has1) break;
        const int64_t i = u ? i1 : i0;
        const bf16* gh = reinterpret_cast<const bf16*>(&graw[u]);
        float* w = reinterpret_cast<float*>(&W[u]);
        float* mm = reinterpret_cast<float*>(&MM[u]);
        float* vv = reinterpret_cast<float*>(&VV[u]);
        __nv_bfloat162 out[2];
#pragma unroll
        for (int j = 0; j < 4; ++j) adam_one(r(f(gh[j]) * fac) * clip, w[j], mm[j], vv[j], decay, step, h);
        out[0] = __floats2bfloat162_rn(w[0], w[1]);
        out[1] = __floats2bfloat162_rn(w[2], w[3]);
        __stcs(M4 + i, W[u]);
        __stcs(m4 + i, MM[u]);
        __stcs(v4 + i, VV[u]);
        __stcs(p4 + i, *reinterpret_cast<uint2*>(out));
        if (zero_grad) __stcs(g4 + i, make_uint2(0u, 0u));
      }
    } else if (zero_grad) {
      g4[i0] = make_uint2(0u, 0u);
      if (has1) g4[i1] = make_uint2(0u, 0u);
    }
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    if (finite) {
      float w = master[i], mm = m[i], vv = v[i];
      adam_one(r(f(grad[i]) * fac) * clip, w, mm, vv, decay, step, h);
      master[i] = w;
      m[i] = mm;
      v[i] = vv;
      param[i] = __float2bfloat16(w);
    }
    if (zero_grad) grad[i] = __float2bfloat16(0.f);
  }
}

// ============================================================================ host API
static int grid_for(int64_t n, int threads = 256) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, (int64_t)num_sms() * 16));
}

void rms_norm_fwd(at::Tensor x, at::Tensor w, double eps, at::Tensor y, at::Tensor inv) {
  check_bf16(x, "x");
  check_bf16(w, "w");
  NS_CHECK(x.dim() == 2 && x.stride(1) == 1 && y.stride(1) == 1, "rms_norm_fwd: row-major 2-D expected");
  const int rows = x.size(0), n = x.size(1);
  if (rows == 0) return;
  const bool vec = n % 8 == 0 && n <= 8 * 256 * 4 && x.stride(0) % 8 == 0 && y.stride(0) % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(y.data_ptr()) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0;
  if (vec) {
    auto launch = [&](auto kern) {
      kern<<<rows, 256, 0, stream()>>>(reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(0),
                                       reinterpret_cast<const bf16*>(w.data_ptr()),
                                       reinterpret_cast<bf16*>(y.data_ptr()), y.stride(0), inv.data_ptr<float>(), n,
                                       (float)eps);
    };
    const int vpt = (n / 8 + 255) / 256;
    if (vpt <= 1) launch(rms_fwd_vec_kernel<1>);
    else if (vpt <= 2) launch(rms_fwd_vec_kernel<2>);
    else launch(rms_fwd_vec_kernel<4>);
    NS_CUDA(cudaGetLastError());
    return;
  }
  rms_fwd_kernel<<<rows, 256, 0, stream()>>>(reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(0),
                                             reinterpret_cast<const bf16*>(w.data_ptr()),
                                             reinterpret_cast<bf16*>(y.data_ptr()), y.stride(0),
                                             inv.data_ptr<float>(), n, (float)eps);
  NS_CUDA(cudaGetLastError());
}

void rms_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor inv, at::Tensor w, at::Tensor dx, at::Tensor dw,
                  c10::optional<at::Tensor> res) {
  const int rows = x.size(0), n = x.size(1);
  NS_CHECK(n <= 40 * 256, "rms_norm_bwd supports rows up to 10240 wide");
  NS_CHECK(dy.stride(1) == 1 && x.stride(1) == 1 && dx.stride(1) == 1, "rms_norm_bwd: row-major expected");
  const int rpb = std::max(1, (rows + 2 * num_sms() - 1) / (2 * num_sms()));
  const int blocks = (rows + rpb - 1) / rpb;
  auto part = at::empty({(int64_t)blocks, n}, x.options().dtype(at::kFloat));
  const bf16* rp = nullptr;
  int64_t ldr = 0;
  if (res && res->defined()) {
    rp = reinterpret_cast<const bf16*>(res->data_ptr());
    ldr = res->stride(0);
  }
  rms_bwd_kernel<<<blocks, 256, 0, stream()>>>(
      reinterpret_cast<const bf16*>(dy.data_ptr()), dy.stride(0), reinterpret_cast<const bf16*>(x.data_ptr()),
      x.stride(0), inv.data_ptr<float>(), reinterpret_cast<const bf16*>(w.data_ptr()),
      reinterpret_cast<bf16*>(dx.data_ptr()), dx.stride(0), rp, ldr, part.data_ptr<float>(), rows, n, rpb);
  NS_CUDA(cudaGetLastError());
  colsum_kernel<<<(n + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), blocks, n,
                                                        reinterpret_cast<bf16*>(dw.data_ptr()));
  NS_CUDA(cudaGetLastError());
}

template <int D>
static void hnr_fwd(at::Tensor x, at::Tensor w, double eps, at::Tensor cs, at::Tensor sn, at::Tensor y,
                    at::Tensor inv) {
  const int T = x.size(0), H = x.size(1);
  const int rows = T * H;
  constexpr int G = D / 2 < 32 ? D / 2 : 32;
  constexpr int RPW = 32 / G;
  const int warps = (rows + RPW - 1) / RPW;
  const int blocks = (warps + 7) / 8;
  head_norm_rope_fwd_kernel<D><<<blocks, 256, 0, stream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(0), H, reinterpret_cast<const bf16*>(w.data_ptr()),
      reinterpret_cast<const bf16*>(cs.data_ptr()), reinterpret_cast<const bf16*>(sn.data_ptr()),
      reinterpret_cast<bf16*>(y.data_ptr()), inv.data_ptr<float>(), rows, (float)eps);
  NS_CUDA(cudaGetLastError());
}

template <int D>
static void hnr_bwd(at::Tensor dy, at::Tensor x, at::Tensor inv, at::Tensor w, at::Tensor cs, at::Tensor sn,
                    at::Tensor dx, at::Tensor dw) {
  const int T = x.size(0), H = x.size(1);
  const int rows = T * H;
  const int blocks = std::min(2 * num_sms(), std::max(1, (rows + 31) / 32));
  auto part = at::empty({(int64_t)blocks, D}, x.options().dtype(at::kFloat));
  head_norm_rope_bwd_kernel<D><<<blocks, 256, 0, stream()>>>(
      reinterpret_cast<const bf16*>(dy.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(0), H,
      inv.data_ptr<float>(), reinterpret_cast<const bf16*>(w.data_ptr()),
      reinterpret_cast<const bf16*>(cs.data_ptr()), reinterpret_cast<const bf16*>(sn.data_ptr()),
      reinterpret_cast<bf16*>(dx.data_ptr()), dx.stride(0), part.data_ptr<float>(), rows);
  NS_CUDA(cudaGetLastError());
  colsum_kernel<<<(D + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), blocks, D,
                                                        reinterpret_cast<bf16*>(dw.data_ptr()));
  NS_CUDA(cudaGetLastError());
}

static void check_head(const at::Tensor& x, const at::Tensor& cs) {
  NS_CHECK(x.dim() == 3 && x.stride(2) == 1 && x.stride(1) == x.size(2), "head tensor must be [T, H, D] with dense heads");
  NS_CHECK(cs.is_contiguous() && cs.size(0) == x.size(0) && cs.size(1) == x.size(2), "cos/sin must be [T, D]");
}

void head_norm_rope_fwd(at::Tensor x, at::Tensor w, double eps, at::Tensor cs, at::Tensor sn, at::Tensor y,
                        at::Tensor inv) {
  check_head(x, cs);
  NS_CHECK(y.is_contiguous(), "y must be contiguous");
  switch (x.size(2)) {
    case 16: hnr_fwd<16>(x, w, eps, cs, sn, y, inv); break;
    case 32: hnr_fwd<32>(x, w, eps, cs, sn, y, inv); break;
    case 64: hnr_fwd<64>(x, w, eps, cs, sn, y, inv); break;
    case 128: hnr_fwd<128>(x, w, eps, cs, sn, y, inv); break;
    case 256: hnr_fwd<256>(x, w, eps, cs, sn, y, inv); break;
    default: NS_CHECK(false, "head_dim must be 16, 32, 64, 128 or 256");
  }
}

void head_norm_rope_bwd(at::Tensor dy, at::Tensor x, at::Tensor inv, at::Tensor w, at::Tensor cs, at::Tensor sn,
                        at::Tensor dx, at::Tensor dw) {
  check_head(x, cs);
  NS_CHECK(dy.is_contiguous(), "dy must be contiguous");
  NS_CHECK(dx.dim() == 3 && dx.stride(2) == 1 && dx.stride(1) == dx.size(2), "dx must be [T, H, D] with dense heads");
  switch (x.size(2)) {
    case 16: hnr_bwd<16>(dy, x, inv, w, cs, sn, dx, dw); break;
    case 32: hnr_bwd<32>(dy, x, inv, w, cs, sn, dx, dw); break;
    case 64: hnr_bwd<64>(dy, x, inv, w, cs, sn, dx, dw); break;
    case 128: hnr_bwd<128>(dy, x, inv, w, cs, sn, dx, dw); break;
    case 256: hnr_bwd<256>(dy, x, inv, w, cs, sn, dx, dw); break;
    default: NS_CHECK(false, "head_dim must be 16, 32, 64, 128 or 256");
  }
}

void swiglu_fwd(at::Tensor gu, at::Tensor out) {
  NS_CHECK(gu.is_contiguous() && out.is_contiguous(), "swiglu: contiguous tensors expected");
  const int64_t rows = gu.size(0);
  const int m = gu.size(1) / 2;
  swiglu_fwd_kernel<<<grid_for(rows * m), 256, 0, stream()>>>(reinterpret_cast<const bf16*>(gu.data_ptr()),
                                                               reinterpret_cast<bf16*>(out.data_ptr()), rows, m);
  NS_CUDA(cudaGetLastError());
}

void swiglu_bwd(at::Tensor dp, at::Tensor gu, at::Tensor dgu) {
  NS_CHECK(dp.is_contiguous() && gu.is_contiguous() && dgu.is_contiguous(), "swiglu_bwd: contiguous expected");
  const int64_t rows = gu.size(0);
  const int m = gu.size(1) / 2;
  swiglu_bwd_kernel<<<grid_for(rows * m), 256, 0, stream()>>>(
      reinterpret_cast<const bf16*>(dp.data_ptr()), reinterpret_cast<const bf16*>(gu.data_ptr()),
      reinterpret_cast<bf16*>(dgu.data_ptr()), rows, m);
  NS_CUDA(cudaGetLastError());
}

void embedding_fwd(at::Tensor ids, at::Tensor w, at::Tensor out) {
  NS_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be contiguous int64");
  NS_CHECK(w.is_contiguous() && out.is_contiguous(), "embedding: contiguous tensors expected");
  const int64_t n = ids.numel();
  if (n == 0) return;
  embedding_fwd_kernel<<<n, 128, 0, stream()>>>(ids.data_ptr<int64_t>(), reinterpret_cast<const bf16*>(w.data_ptr()),
                                                w.size(1), reinterpret_cast<bf16*>(out.data_ptr()), n, w.size(0),
                                                device_error_flag());
  NS_CUDA(cudaGetLastError());
}

void embedding_bwd(at::Tensor dy, at::Tensor ids, at::Tensor grad) {
  NS_CHECK(grad.is_contiguous() && dy.is_contiguous() && ids.is_contiguous(), "embedding_bwd: contiguous expected");
  NS_CUDA(cudaMemsetAsync(grad.data_ptr(), 0, grad.numel() * 2, stream()));
  const int d = grad.size(1);
  embedding_bwd_kernel<<<(d + 127) / 128, 128, 0, stream()>>>(
      reinterpret_cast<const bf16*>(dy.data_ptr()), ids.data_ptr<int64_t>(), ids.numel(), d,
      reinterpret_cast<bf16*>(grad.data_ptr()), grad.size(0), device_error_flag());
  NS_CUDA(cudaGetLastError());
}

void grad_norm_sq(at::Tensor grad, at::Tensor factor, at::Tensor norm2) {
  const int64_t n = grad.numel();
  NS_CHECK(reinterpret_cast<uintptr_t>(grad.data_ptr()) % 2 == 0, "grad_norm_sq: bf16 gradient expected");
  if (n == 0) return;
  const int blocks = (int)std::min<int64_t>(num_sms() * 4, std::max<int64_t>(1, (n / 8 + 255) / 256));
  auto part = at::empty({blocks}, grad.options().dtype(at::kFloat));
  grad_norm_part_kernel<<<blocks, 256, 0, stream()>>>(reinterpret_cast<const bf16*>(grad.data_ptr()), n,
                                                      factor.data_ptr<float>(), part.data_ptr<float>());
  NS_CUDA(cudaGetLastError());
  sum_into_kernel<<<1, 32, 0, stream()>>>(part.data_ptr<float>(), blocks, norm2.data_ptr<float>());
  NS_CUDA(cudaGetLastError());
}

// norm2 += sum over every range of sum bf16(g * factor)^2 (one launch per 64 ranges).
void grad_norm_sq_ranges(std::vector<at::Tensor> ranges, at::Tensor factor, at::Tensor norm2) {
  for (size_t base = 0; base < ranges.size(); base += NR) {
    NormRanges rs{};
    rs.count = 0;
    int blocks = 0;
    for (size_t i = base; i < ranges.size() && rs.count < NR; ++i) {
      const at::Tensor& g = ranges[i];
      check_bf16(g, "gradient range");
      NS_CHECK(g.is_contiguous(), "gradient ranges must be contiguous");
      if (g.numel() == 0) continue;
      rs.p[rs.count] = reinterpret_cast<const bf16*>(g.data_ptr());
      rs.n[rs.count] = g.numel();
      rs.block_start[rs.count] = blocks;
      blocks += (int)std::min<int64_t>(num_sms() * 2, std::max<int64_t>(1, (g.numel() / 8 + 255) / 256));
      ++rs.count;
    }
    if (rs.count == 0) continue;
    rs.block_start[rs.count] = blocks;
    auto part = at::empty({blocks}, norm2.options());
    grad_norm_ranges_kernel<<<blocks, 256, 0, stream()>>>(rs, factor.data_ptr<float>(), part.data_ptr<float>());
    NS_CUDA(cudaGetLastError());
    sum_into_kernel<<<1, 32, 0, stream()>>>(part.data_ptr<float>(), blocks, norm2.data_ptr<float>());
    NS_CUDA(cudaGetLastError());
  }
}

void adamw_update(at::Tensor param, at::Tensor master, at::Tensor m, at::Tensor v, at::Tensor grad,
                  at::Tensor factor, at::Tensor norm2, double lr, double wd, double b1, double b2, double eps,
                  double bc1, double bc2, double max_norm, c10::optional<at::Tensor> bc_dev, bool zero_grad) {
  const int64_t n = master.numel();
  NS_CHECK(reinterpret_cast<uintptr_t>(master.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(grad.data_ptr()) % 8 == 0 &&
               reinterpret_cast<uintptr_t>(param.data_ptr()) % 8 == 0,
           "adamw: shard buffers must be 16/8-byte aligned");
  AdamHyper h{(float)lr, (float)wd, (float)b1, (float)b2, (float)eps, (float)bc1, (float)bc2, (float)max_norm,
              bc_dev && bc_dev->defined() ? bc_dev->data_ptr<float>() : nullptr};
  // Exactly the resident capacity (4 blocks of 256 per SM): every block streams an
  // equal share in one wave, so no partial last wave idles most of the SMs.
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n / 4 + 255) / 256, (int64_t)num_sms() * 4));
  adamw_kernel<<<blocks, 256, 0, stream()>>>(reinterpret_cast<bf16*>(param.data_ptr()), master.data_ptr<float>(),
                                             m.data_ptr<float>(), v.data_ptr<float>(),
                                             reinterpret_cast<bf16*>(grad.data_ptr()), n, factor.data_ptr<float>(),
                                             norm2.data_ptr<float>(), h, zero_grad ? 1 : 0);
  NS_CUDA(cudaGetLastError());
}

void adam_prepare(at::Tensor norm2, at::Tensor step, double b1, double b2, at::Tensor bc) {
  NS_CHECK(step.scalar_type() == at::kLong && bc.scalar_type() == at::kFloat && bc.numel() >= 2, "adam_prepare: types");
  adam_prepare_kernel<<<1, 32, 0, stream()>>>(norm2.data_ptr<float>(), step.data_ptr<int64_t>() ? reinterpret_cast<long long*>(step.data_ptr<int64_t>()) : nullptr, b1, b2, bc.data_ptr<float>());
  NS_CUDA(cudaGetLastError());
}

}  // namespace ns
