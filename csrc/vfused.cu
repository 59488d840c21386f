// Fused producers of the verifier's FP8 projections (forward only).
//
// The reference quantises every projection input on its own (nanospec/ops.py:183-200:
// 1 x 128 blocks, scale = amax / 448, e4m3) after separate residual-add, norm and
// SwiGLU passes (nanospec/train.py:137-153). Here the kernel that produces an
// activation also emits its e4m3 codes and 1 x 128 scales, so the FP8 GEMM reads
// 1 byte per element and no separate quantisation pass runs:
//
//  * add_norm_kernel: x' = bf16(x + y) (y optional), n = bf16(x' * rsqrt(mean(x'^2)
//    + eps) * (1 + w)); writes x', and n as bf16 and/or e4m3 + scales. One CTA of
//    256 threads per token row, 8 channels (16 bytes) per access; a 128-channel
//    quantisation block is 16 consecutive chunks held by 16 consecutive lanes.
//  * silu_mul_quant_kernel: h = bf16(bf16(silu(gate)) * up) from the fused [gate | up]
//    projection, emitted as e4m3 + scales (one warp per 128-channel block).
//  * gated_norm_quant_kernel: w * bf16(rmsnorm(o)) * silu(z) per 128-wide value head
//    (one warp per head row = one quantisation block).
//  * conv_silu_vec_kernel: causal depthwise conv (kernel K <= 4) + SiLU, 8 channels
//    per thread.
// Quantisation follows the reference statement on the bf16 value v:
// s = amax / 448, q = e4m3(clamp(v / max(s, FLT_MIN), -448, 448)) (saturating).
#include "common.h"
#include "peer.h"
#include "sm100.cuh"

#include <cuda_fp8.h>

namespace ns {

using bf16 = __nv_bfloat16;

namespace vf {

__device__ __forceinline__ float rb(float x) { return sm100::bf16_round(x); }

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __bfloat1622float2(h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// v / den rounded to nearest, as the reference's division, from r = RN(1 / den) and
// one FMA correction. Markstein's theorem (Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
// when r is the correctly rounded reciprocal and q0 is within one ulp of v / den,
// q0 + (v - q0 den) r evaluated as a single FMA is the correctly rounded quotient.
// The residual v - q0 den is exact by FMA. The theorem holds in the normal range,
// which den >= FLT_MIN and |v / den| <= 448 give. Smaller quotients are far below
// the least e4m3 subnormal and quantise to the same code either way.
__device__ __forceinline__ float div_rn(float v, float den, float r) {
  const float q0 = v * r;
  return fmaf(fmaf(-q0, den, v), r, q0);
}

__device__ __forceinline__ uint32_t e4m3x4_div(float a, float b, float c, float d, float den) {
  const float v[4] = {a, b, c, d};
  const float r = 1.f / den;
  uint32_t p = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float y = fminf(fmaxf(div_rn(v[i], den, r), -448.f), 448.f);
    p |= (uint32_t)__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3) << (8 * i);
  }
  return p;
}

constexpr int AN_THREADS = 256;
constexpr int AN_MAX_CPT = 4;  // chunks of 8 per thread: rows up to 8192 channels

__global__ void __launch_bounds__(AN_THREADS) add_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ y,
                                                              const bf16* __restrict__ w, float eps, int H,
                                                              bf16* __restrict__ x_out, bf16* __restrict__ n_out,
                                                              uint8_t* __restrict__ q_out, float* __restrict__ s_out,
                                                              bf16* __restrict__ x_peer, bf16* __restrict__ n_peer) {
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nch = H / 8;
  float v[AN_MAX_CPT][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < AN_MAX_CPT; ++j) {
    const int c = tid + j * AN_THREADS;
    if (c < nch) {
      unpack8(reinterpret_cast<const uint4*>(x + row * H)[c], v[j]);
      if (y) {
        float t[8];
        unpack8(reinterpret_cast<const uint4*>(y + row * H)[c], t);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] = rb(v[j][i] + t[i]);
        const uint4 pk = pack8(v[j]);
        reinterpret_cast<uint4*>(x_out + row * H)[c] = pk;
        if (x_peer) reinterpret_cast<uint4*>(x_peer + row * H)[c] = pk;  // hand-off store to a trainer
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[j][i] * v[j][i];
    }
  }
  __shared__ float red[AN_THREADS / 32];
  __shared__ float tot;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float t = tid < AN_THREADS / 32 ? red[tid] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffff, t, o);
    if (tid == 0) tot = t;
  }
  __syncthreads();
  const float inv = rsqrtf(tot / H + eps);
  const int kbs = H / 128;
#pragma unroll
  for (int j = 0; j < AN_MAX_CPT; ++j) {
    if (j * AN_THREADS >= nch) break;  // uniform across the block
    const int c = tid + j * AN_THREADS;
    const bool in = c < nch;
    float nv[8];
    if (in) {
      float wv[8];
      unpack8(reinterpret_cast<const uint4*>(w)[c], wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) nv[i] = rb(v[j][i] * inv * (1.f + wv[i]));
      if (n_out) reinterpret_cast<uint4*>(n_out + row * H)[c] = pack8(nv);
      if (n_peer) reinterpret_cast<uint4*>(n_peer + row * H)[c] = pack8(nv);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) nv[i] = 0.f;
    }
    if (q_out) {  // a 128-channel block is 16 chunks on 16 consecutive lanes
      float am = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(nv[i]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffff, am, o, 16));
      const float s = am / 448.f;
      const float den = fmaxf(s, 1.17549435e-38f);
      if (in) {
        uint2 pk;
        pk.x = e4m3x4_div(nv[0], nv[1], nv[2], nv[3], den);
        pk.y = e4m3x4_div(nv[4], nv[5], nv[6], nv[7], den);
        reinterpret_cast<uint2*>(q_out + row * H)[c] = pk;
        if ((c & 15) == 0) s_out[row * kbs + (c >> 4)] = s;
      }
    }
  }
  if (x_peer || n_peer) __threadfence_system();  // peer stores land before a later flag
}

// gu [T, 2m] = [gate | up]; h = bf16(bf16(silu(gate)) * up) -> e4m3 + scales [T, m/128].
// A 128-channel block per half-warp, 8 channels (16-byte loads) per lane.
__global__ void silu_mul_quant_kernel(const bf16* __restrict__ gu, int64_t T, int m, uint8_t* __restrict__ q,
                                      float* __restrict__ s) {
  const int64_t hw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4;  // half-warp = one block
  const int l16 = threadIdx.x & 15;
  const int kbs = m / 128;
  const bool in = hw < T * kbs;
  const int64_t t = in ? hw / kbs : 0;
  const int kb = in ? (int)(hw % kbs) : 0;
  float h[8];
  float am = 0.f;
  if (in) {
    const bf16* g = gu + t * 2 * m + kb * 128 + l16 * 8;
    float gv[8], uv[8];
    unpack8(*reinterpret_cast<const uint4*>(g), gv);
    unpack8(*reinterpret_cast<const uint4*>(g + m), uv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      h[i] = rb(rb(__fdividef(gv[i], 1.f + __expf(-gv[i]))) * uv[i]);  // fast SiLU (bf16 result)
      am = fmaxf(am, fabsf(h[i]));
    }
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffff, am, o, 16));
  if (!in) return;
  const float sc = am / 448.f;
  const float den = fmaxf(sc, 1.17549435e-38f);
  uint2 pk;
  pk.x = e4m3x4_div(h[0], h[1], h[2], h[3], den);
  pk.y = e4m3x4_div(h[4], h[5], h[6], h[7], den);
  *reinterpret_cast<uint2*>(q + t * m + kb * 128 + l16 * 8) = pk;
  if (l16 == 0) s[t * kbs + kb] = sc;
}

// rows of 128 (row = token * nv + head): y = bf16(rb(w * rb(x * inv)) * silu(z)) ->
// e4m3 + one scale per row; z(token, head) at z + token * z_ts + head * 128.
__global__ void gated_norm_quant_kernel(const bf16* __restrict__ x, const bf16* __restrict__ z, int nv, int64_t z_ts,
                                        const bf16* __restrict__ w, int64_t rows, float eps, uint8_t* __restrict__ q,
                                        float* __restrict__ s) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint2 xr = *reinterpret_cast<const uint2*>(x + row * 128 + lane * 4);
  const uint2 zr = *reinterpret_cast<const uint2*>(z + (row / nv) * z_ts + (row % nv) * 128 + lane * 4);
  const uint2 wr = *reinterpret_cast<const uint2*>(w + lane * 4);
  const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xr);
  const __nv_bfloat162* zh = reinterpret_cast<const __nv_bfloat162*>(&zr);
  const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wr);
  float xv[4], zv[4], wv[4];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float2 a = __bfloat1622float2(xh[i]), b = __bfloat1622float2(zh[i]), c = __bfloat1622float2(wh[i]);
    xv[2 * i] = a.x, xv[2 * i + 1] = a.y, zv[2 * i] = b.x, zv[2 * i + 1] = b.y, wv[2 * i] = c.x, wv[2 * i + 1] = c.y;
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss += xv[i] * xv[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  const float inv = rsqrtf(ss / 128.f + eps);
  float y[4];
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float sg = __fdividef(zv[i], 1.f + __expf(-zv[i]));  // fast SiLU
    y[i] = rb(rb(wv[i] * rb(xv[i] * inv)) * sg);
    am = fmaxf(am, fabsf(y[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffff, am, o));
  const float sc = am / 448.f;
  const float den = fmaxf(sc, 1.17549435e-38f);
  *reinterpret_cast<uint32_t*>(q + row * 128 + lane * 4) = e4m3x4_div(y[0], y[1], y[2], y[3], den);
  if (lane == 0) s[row] = sc;
}

// out[b, t, c] = silu(bf16(sum_j w[c, j] x[b, t - (K-1) + j, c])); x rows of ld elements
// (the first C channels of each row are convolved). A thread owns 8 channels and a run
// of CONV_TOKENS consecutive token rows: its 8 x K weights are loaded once (16-byte
// loads), and the K - 1 previous rows are kept in registers, so every input row is read
// once. Rows of a new sequence (t % s == 0) start with an empty window. K <= 4.
constexpr int CONV_TOKENS = 16;

template <int K>
__global__ void __launch_bounds__(256) conv_silu_vec_kernel(const bf16* __restrict__ x, int64_t ld,
                                                            const bf16* __restrict__ w, bf16* __restrict__ y,
                                                            int64_t rows, int s, int C) {
  const int c8 = blockIdx.y * blockDim.x + threadIdx.x;
  if (c8 * 8 >= C) return;
  const int c = c8 * 8;
  float wv[8][4];
  {
    // w [C, K] row-major: this thread's 8 channels are 8 * K contiguous values
    __align__(16) bf16 wr[32];
    const bf16* wp = w + (int64_t)c * K;
    if (K == 4) {
#pragma unroll
      for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(wr)[i] = reinterpret_cast<const uint4*>(wp)[i];
    } else {
      for (int i = 0; i < 8 * K; ++i) wr[i] = wp[i];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int j = 0; j < 4; ++j) wv[e][j] = j < K ? __bfloat162float(wr[e * K + j]) : 0.f;
  }
  const int64_t r0 = (int64_t)blockIdx.x * CONV_TOKENS;
  const int64_t r1 = min(rows, r0 + CONV_TOKENS);
  // window[j] = x row (t - 3 + j) for j = 0..2, zero before the sequence start
  float win[3][8];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int64_t rr = r0 - 3 + j;
    const int back = 3 - j;  // rows before r0
    const bool ok = rr >= 0 && (int)(r0 % s) >= back;
    if (ok) unpack8(*reinterpret_cast<const uint4*>(x + rr * ld + c), win[j]);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) win[j][e] = 0.f;
  }
  int pos = (int)(r0 % s);  // position of row r in its sequence (one division per thread)
  for (int64_t r = r0; r < r1; ++r, ++pos) {
    if (pos == s) {  // a new sequence starts: no history
      pos = 0;
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) win[j][e] = 0.f;
    }
    float cur[8];
    unpack8(*reinterpret_cast<const uint4*>(x + r * ld + c), cur);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // taps j = 0..K-1 read rows t - (K-1) + j: the last K entries of [win0, win1, win2, cur]
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const int src = 4 - K + j;  // 0..2: window rows, 3: the current row
        acc += wv[e][j] * (src == 3 ? cur[e] : win[src < 3 ? src : 0][e]);
      }
      // SiLU in fp32 with the fast exponential and division intrinsics; the bf16
      // result differs from the accurate forms only in rare rounding ties
      const float zz = rb(acc);
      o[e] = __fdividef(zz, 1.f + __expf(-zz));
    }
    reinterpret_cast<uint4*>(y + r * C)[c8] = pack8(o);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      win[0][e] = win[1][e];
      win[1][e] = win[2][e];
      win[2][e] = cur[e];
    }
  }
}

}  // namespace vf

// x_out / n_out / q_out+s_out optional (undefined tensors); y optional.
void add_norm(at::Tensor x, c10::optional<at::Tensor> y, at::Tensor w, double eps, c10::optional<at::Tensor> x_out,
              c10::optional<at::Tensor> n_out, c10::optional<at::Tensor> q_out, c10::optional<at::Tensor> s_out) {
  check_bf16(x, "x");
  const int H = (int)x.size(-1);
  const int64_t rows = x.numel() / H;
  NS_CHECK(x.is_contiguous() && H % 8 == 0 && H / 8 <= vf::AN_THREADS * vf::AN_MAX_CPT, "add_norm: row width");
  NS_CHECK(!q_out || H % 128 == 0, "add_norm: quantised output needs 128-multiple rows");
  NS_CHECK(!y || x_out, "add_norm: the residual sum needs x_out");
  if (rows == 0) return;
  auto p = [](const c10::optional<at::Tensor>& t) -> void* { return t ? t->data_ptr() : nullptr; };
  vf::add_norm_kernel<<<(unsigned)rows, vf::AN_THREADS, 0, stream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), reinterpret_cast<const bf16*>(p(y)),
      reinterpret_cast<const bf16*>(w.data_ptr()), (float)eps, H, reinterpret_cast<bf16*>(p(x_out)),
      reinterpret_cast<bf16*>(p(n_out)), reinterpret_cast<uint8_t*>(p(q_out)), reinterpret_cast<float*>(p(s_out)),
      nullptr, nullptr);
  NS_CUDA(cudaGetLastError());
}

// add_norm whose epilogue also stores x_out (x_dst >= 0) and / or n_out (n_dst >= 0)
// into rank x_dst's / n_dst's window of `win` at byte x_off / n_off, same row layout:
// the verifier -> trainer hand-off written by the producing kernel.
void add_norm_peer(at::Tensor x, c10::optional<at::Tensor> y, at::Tensor w, double eps,
                   c10::optional<at::Tensor> x_out, c10::optional<at::Tensor> n_out, c10::optional<at::Tensor> q_out,
                   c10::optional<at::Tensor> s_out, int64_t win, int64_t x_dst, int64_t x_off, int64_t n_dst,
                   int64_t n_off) {
  check_bf16(x, "x");
  const int H = (int)x.size(-1);
  const int64_t rows = x.numel() / H;
  NS_CHECK(x.is_contiguous() && H % 8 == 0 && H / 8 <= vf::AN_THREADS * vf::AN_MAX_CPT, "add_norm: row width");
  NS_CHECK(!q_out || H % 128 == 0, "add_norm: quantised output needs 128-multiple rows");
  NS_CHECK(!y || x_out, "add_norm: the residual sum needs x_out");
  NS_CHECK(x_dst < 0 || (y && x_out), "add_norm_peer: the residual store needs y and x_out");
  NS_CHECK(n_dst < 0 || n_out, "add_norm_peer: the normed store needs n_out");
  NS_CHECK(x_off % 16 == 0 && n_off % 16 == 0, "add_norm_peer: 16-byte aligned destinations");
  if (rows == 0) return;
  const WindowInfo wi = window_info(win);
  // Offsets come from the slot layout every rank shares (the caller's own window may
  // be smaller than the destination's, so its size bounds nothing here).
  auto peer = [&](int64_t dst, int64_t off) -> bf16* {
    if (dst < 0) return nullptr;
    NS_CHECK(dst < wi.world, "add_norm_peer: destination rank outside the window's world");
    const uint64_t base = wi.table.base[dst];
    NS_CHECK(base != 0, "add_norm_peer: destination window not open");
    return reinterpret_cast<bf16*>(base + off);
  };
  auto p = [](const c10::optional<at::Tensor>& t) -> void* { return t ? t->data_ptr() : nullptr; };
  vf::add_norm_kernel<<<(unsigned)rows, vf::AN_THREADS, 0, stream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), reinterpret_cast<const bf16*>(p(y)),
      reinterpret_cast<const bf16*>(w.data_ptr()), (float)eps, H, reinterpret_cast<bf16*>(p(x_out)),
      reinterpret_cast<bf16*>(p(n_out)), reinterpret_cast<uint8_t*>(p(q_out)), reinterpret_cast<float*>(p(s_out)),
      peer(x_dst, x_off), peer(n_dst, n_off));
  NS_CUDA(cudaGetLastError());
}

void silu_mul_quant(at::Tensor gu, at::Tensor q, at::Tensor s) {
  check_bf16(gu, "gu");
  const int64_t T = gu.size(0);
  const int m = (int)(gu.size(1) / 2);
  NS_CHECK(gu.is_contiguous() && m % 128 == 0, "silu_mul_quant: [T, 2m] with m a multiple of 128");
  const int64_t halfwarps = T * (m / 128);
  if (halfwarps == 0) return;
  vf::silu_mul_quant_kernel<<<(unsigned)((halfwarps * 16 + 255) / 256), 256, 0, stream()>>>(
      reinterpret_cast<const bf16*>(gu.data_ptr()), T, m, q.data_ptr<uint8_t>(), s.data_ptr<float>());
  NS_CUDA(cudaGetLastError());
}

// x [T * nv, 128] contiguous; z token rows of stride z_ts elements, head h at + h * 128.
void gated_norm_quant(at::Tensor x, at::Tensor z, int64_t nv, int64_t z_ts, at::Tensor w, double eps, at::Tensor q,
                      at::Tensor s) {
  NS_CHECK(x.size(-1) == 128 && x.is_contiguous(), "gated_norm_quant: contiguous rows of 128");
  NS_CHECK(z_ts % 8 == 0, "gated_norm_quant: z rows 16-byte aligned");
  const int64_t rows = x.numel() / 128;
  if (rows == 0) return;
  vf::gated_norm_quant_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, stream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), reinterpret_cast<const bf16*>(z.data_ptr()), (int)nv, z_ts,
      reinterpret_cast<const bf16*>(w.data_ptr()), rows, (float)eps, q.data_ptr<uint8_t>(), s.data_ptr<float>());
  NS_CUDA(cudaGetLastError());
}

// x: [b, s, *] rows of row stride ld (elements); the first C channels are convolved.
void conv_silu_vec(at::Tensor x, int64_t ld, at::Tensor w, at::Tensor y) {
  const int b = (int)y.size(0), s = (int)y.size(1), C = (int)y.size(2), K = (int)w.size(1);
  NS_CHECK(C % 8 == 0 && ld % 8 == 0 && y.is_contiguous(), "conv_silu_vec: 8-channel alignment");
  NS_CHECK(K >= 1 && K <= 4, "conv_silu_vec: kernel width 1..4");
  NS_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
           "conv_silu_vec: 16-byte aligned operands");
  const int64_t rows = (int64_t)b * s;
  if (rows == 0) return;
  const dim3 grid((unsigned)((rows + vf::CONV_TOKENS - 1) / vf::CONV_TOKENS), (unsigned)((C / 8 + 255) / 256));
  auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* wp = reinterpret_cast<const bf16*>(w.data_ptr());
  auto* yp = reinterpret_cast<bf16*>(y.data_ptr());
  switch (K) {
    case 1: vf::conv_silu_vec_kernel<1><<<grid, 256, 0, stream()>>>(xp, ld, wp, yp, rows, s, C); break;
    case 2: vf::conv_silu_vec_kernel<2><<<grid, 256, 0, stream()>>>(xp, ld, wp, yp, rows, s, C); break;
    case 3: vf::conv_silu_vec_kernel<3><<<grid, 256, 0, stream()>>>(xp, ld, wp, yp, rows, s, C); break;
    default: vf::conv_silu_vec_kernel<4><<<grid, 256, 0, stream()>>>(xp, ld, wp, yp, rows, s, C); break;
  }
  NS_CUDA(cudaGetLastError());
}

}  // namespace ns
