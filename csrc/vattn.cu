// Verifier full attention on 5th-generation tensor cores (flash-attention forward).
//
// Reference: nanospec/ops.py:115-126 (causal GQA; Qwen's eager ordering) with the
// projections around it at nanospec/train.py:109-136: q/k (1+w)-RMSNorm per head,
// partial RoPE on the first rotary_dim channels, causal softmax over keys, then
// out * sigmoid(gate). The reference forms the [S, S] scores explicitly; here the
// scores never leave the chip.
//
// Two kernels:
//  * head_norm_rope_kernel: (1+w)-RMSNorm of one head row (one warp per row) and
//    partial RoPE on its first rotary_dim channels, in the bf16 statement order
//    (norm rounded to bf16, then x cos + rotate_half(x) sin with each product and
//    the sum rounded). Reads strided rows, so q can come straight out of the
//    interleaved [q | gate] projection.
//  * vattn_fwd_kernel<D>: one CTA per (128 query rows, query head, batch row), heavy
//    (late) query tiles first. Warp 0 loads Q once and K/V tiles of 64 keys through a
//    2-stage TMA ring (3-D tensor maps over [tokens][heads][D], this GPU's memory,
//    no multicast); warp 1 issues tcgen05.mma; warps 2-5 (one query row per thread,
//    TMEM lane = row) run the online softmax.
//      S_j = Q K_j^T        M=128, N=64,  K=D   -> TMEM (two 64-column buffers)
//      O  += P_j V_j        M=128, N=D,   K=64  -> TMEM (D columns), P_j bf16 in smem
//    S_{j+1} is issued before the softmax of tile j finishes, so the tensor pipe
//    overlaps the exponentials. The running maximum used for the exponentials is
//    only raised when a row's true maximum exceeds it by more than 2^8; then the warp
//    rescales its O rows in TMEM (tcgen05.ld / st) once PV_{j-1} has completed. The
//    final O / l is exact either way. Epilogue: bf16(O / l) * bf16(sigmoid(gate)).
// Every mbarrier wait is bounded; a timeout sets the device error word and the
// kernel unwinds (producer drains its copies, TMEM is freed).
#include "common.h"
#include "sm100.cuh"

namespace ns {

using bf16 = __nv_bfloat16;

namespace vattn {

__device__ __forceinline__ float bf(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float rb(float x) { return sm100::bf16_round(x); }

// ------------------------------------------------------------------ norm + partial RoPE
// x rows: row r = token * H + h at x + token * x_ts + h * x_hs (elements); y contiguous
// [rows][D]. cos/sin [S][rd] (token position t % S of row's token).
template <int D>
__global__ void __launch_bounds__(256) head_norm_rope_kernel(const bf16* __restrict__ x, int64_t x_ts, int64_t x_hs,
                                                             int H, int64_t rows, int S, const bf16* __restrict__ w,
                                                             float eps, const bf16* __restrict__ cs,
                                                             const bf16* __restrict__ sn, int rd,
                                                             bf16* __restrict__ y) {
  constexpr int E = (D + 31) / 32;
  __shared__ float buf[8][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= rows) return;
  const int64_t tok = row / H;
  const int h = (int)(row % H);
  const bf16* xr = x + tok * x_ts + h * x_hs;
  float v[E];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int d = lane + 32 * e;
    v[e] = d < D ? bf(xr[d]) : 0.f;
    ss += v[e] * v[e];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  const float inv = rsqrtf(ss / D + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int d = lane + 32 * e;
    if (d < D) buf[warp][d] = rb(v[e] * inv * (1.f + bf(w[d])));
  }
  __syncwarp();
  const int t = (int)(tok % S);
  const int half = rd / 2;
  bf16* yr = y + row * D;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int d = lane + 32 * e;
    if (d >= D) continue;
    float o = buf[warp][d];
    if (d < rd) {
      const float c = bf(cs[(int64_t)t * rd + d]), s = bf(sn[(int64_t)t * rd + d]);
      const float rot = d < half ? -buf[warp][d + half] : buf[warp][d - half];
      o = rb(rb(o * c) + rb(rot * s));
    }
    yr[d] = __float2bfloat16(o);
  }
}

// ------------------------------------------------------------------ flash attention
constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 64;   // keys per tile
constexpr float RESCALE_LOG2 = 8.f;

template <int D>
struct Cfg {
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int K_BYTES = BN * D * 2;
  static constexpr int KV_BYTES = 2 * K_BYTES;  // K and V of one stage
  static constexpr int P_BYTES = BM * BN * 2;   // 16 KB
  static constexpr int STAGES = 2;
  static constexpr int SMEM = Q_BYTES + STAGES * KV_BYTES + 2 * P_BYTES + 1024 + 256;
  static constexpr int TMEM_COLS = D + 2 * BN <= 256 ? 256 : 512;
  static constexpr int S_COL = D;  // S buffers after the O columns
};

struct Args {
  int s, Hq, Hk;
  float scale_log2;        // D^-1/2 * log2(e)
  const bf16* gate;        // gate(b, t, h, d) at gate + (b * s + t) * g_ts + h * g_hs + d
  int64_t g_ts, g_hs;
  bf16* out;               // [b, s, Hq, D] contiguous
  int* err;
};

template <int D>
__global__ void __launch_bounds__(192, 1) vattn_fwd_kernel(const __grid_constant__ CUtensorMap tq,
                                                           const __grid_constant__ CUtensorMap tk,
                                                           const __grid_constant__ CUtensorMap tv, Args a) {
  using C = Cfg<D>;
  constexpr int DA = D / 64;  // 128-byte swizzle atoms along D
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + C::Q_BYTES;                         // stage st: K at st*KV_BYTES, V after K
  uint8_t* sP = sKV + C::STAGES * C::KV_BYTES;            // two P buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;    // [2]
  uint64_t* kv_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;     // [2]
  uint64_t* s_free = bars + 7;     // [2]
  uint64_t* p_full = bars + 9;     // [2]
  uint64_t* p_free = bars + 11;    // [2]
  uint64_t* o_done = bars + 13;    // one completion per PV_j (rescales wait for PV_{j-1})
  uint64_t* o_last = bars + 14;    // completes once, after the last PV (the epilogue's wait:
                                   // a parity wait on o_done could be two phases behind there)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = gridDim.x - 1 - blockIdx.x;  // heavy tiles first
  const int h = blockIdx.y, bi = blockIdx.z;
  const int hk = h / (a.Hq / a.Hk);
  const int q0 = qb * BM;
  const int tok0 = bi * a.s;  // token row of this batch row's first token
  const int nkt = min((a.s + BN - 1) / BN, (q0 + BM + BN - 1) / BN);

  if (warp == 0 && lane == 0) {
    sm100::mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&kv_full[i], 1);
      sm100::mbar_init(&kv_empty[i], 1);
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&s_free[i], 4);
      sm100::mbar_init(&p_full[i], 4);
      sm100::mbar_init(&p_free[i], 1);
    }
    sm100::mbar_init(o_done, 1);
    sm100::mbar_init(o_last, 1);
    sm100::fence_barrier_init();
    sm100::tma_prefetch_desc(&tq);
    sm100::tma_prefetch_desc(&tk);
    sm100::tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, C::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      sm100::mbar_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int j = 0; j < DA; ++j) sm100::tma_load_3d(sQ + j * (BM * 128), &tq, q_full, 64 * j, h, tok0 + q0);
      int issued = 0;
      for (int t = 0; t < nkt; ++t) {
        const int st = t & 1;
        if (t >= 2 && !sm100::mbar_wait(&kv_empty[st], ((t >> 1) - 1) & 1, a.err)) break;
        uint8_t* kd = sKV + st * C::KV_BYTES;
        uint8_t* vd = kd + C::K_BYTES;
        sm100::mbar_expect_tx(&kv_full[st], C::KV_BYTES);
#pragma unroll
        for (int j = 0; j < DA; ++j) {
          sm100::tma_load_3d(kd + j * (BN * 128), &tk, &kv_full[st], 64 * j, hk, tok0 + t * BN);
          sm100::tma_load_3d(vd + j * (BN * 128), &tv, &kv_full[st], 64 * j, hk, tok0 + t * BN);
        }
        issued = t + 1;
      }
      // drain: every issued copy has landed before the CTA may exit
      sm100::mbar_wait(q_full, 0, a.err);
      for (int t = max(0, issued - 2); t < issued; ++t) sm100::mbar_wait(&kv_full[t & 1], (t >> 1) & 1, a.err);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = sm100::idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = sm100::idesc_bf16(BM, D, false, true);
      const uint32_t q_base = sm100::smem_u32(sQ);
      bool ok = sm100::mbar_wait(q_full, 0, a.err);
      auto issue_s = [&](int t) -> bool {
        const int st = t & 1;
        if (!sm100::mbar_wait(&kv_full[st], (t >> 1) & 1, a.err)) return false;
        if (t >= 2 && !sm100::mbar_wait(&s_free[st], ((t >> 1) - 1) & 1, a.err)) return false;
        sm100::tc_fence_after();
        const uint32_t k_base = sm100::smem_u32(sKV + st * C::KV_BYTES);
        const uint32_t d_s = tmem + C::S_COL + st * BN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = sm100::smem_desc_sw128(q_base + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bd = sm100::smem_desc_sw128(k_base + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 0, 1024);
          sm100::mma_bf16(d_s, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        sm100::mma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int t = 0; ok && t < nkt; ++t) {
        if (t + 1 < nkt && !issue_s(t + 1)) break;
        const int pb = t & 1;
        if (!sm100::mbar_wait(&p_full[pb], (t >> 1) & 1, a.err)) break;
        sm100::tc_fence_after();
        const uint32_t p_base = sm100::smem_u32(sP + pb * C::P_BYTES);
        const uint32_t v_base = sm100::smem_u32(sKV + (t & 1) * C::KV_BYTES + C::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = sm100::smem_desc_sw128(p_base + kk * 32, 0, 1024);
          const uint64_t bd = sm100::smem_desc_sw128(v_base + kk * 2048, BN * 128, 1024);
          sm100::mma_bf16(tmem, ad, bd, idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
        }
        sm100::mma_commit(o_done);
        if (t == nkt - 1) sm100::mma_commit(o_last);
        sm100::mma_commit(&p_free[pb]);
        sm100::mma_commit(&kv_empty[t & 1]);
      }
    }
  } else {
    // ---------------------------------------------------------- softmax warps
    const int qw = warp & 3;              // TMEM lane quarter of this warp
    const int row = qw * 32 + lane;       // query row within the tile
    const int qi = q0 + row;              // query position
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < nkt && ok; ++t) {
      const int sb = t & 1;
      ok = __all_sync(0xffffffff, sm100::mbar_wait(&s_full[sb], (t >> 1) & 1, a.err));
      if (!ok) break;
      sm100::tc_fence_after();
      float sv[BN];
      {
        float tmp[32];
        sm100::tmem_ld32(tmem + lane_off + C::S_COL + sb * BN, tmp);
#pragma unroll
        for (int c = 0; c < 32; ++c) sv[c] = tmp[c];
        sm100::tmem_ld32(tmem + lane_off + C::S_COL + sb * BN + 32, tmp);
#pragma unroll
        for (int c = 0; c < 32; ++c) sv[32 + c] = tmp[c];
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&s_free[sb]);
      // scale into the log2 domain, mask (causal and beyond the sequence)
      const int k0 = t * BN;
      const bool diag = k0 + BN - 1 > q0 || k0 + BN > a.s;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        float x = sv[c] * a.scale_log2;
        if (diag && (k0 + c > qi || k0 + c >= a.s)) x = -INFINITY;
        sv[c] = x;
        mt = fmaxf(mt, x);
      }
      float alpha = 1.f;
      bool grow = false;
      if (mt > m_used + RESCALE_LOG2) {
        alpha = exp2f(m_used - mt);  // 0 on the first tile
        m_used = mt;
        grow = true;
      }
      float ps = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float p0 = exp2f(sv[c] - m_used), p1 = exp2f(sv[c + 1] - m_used);
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
        ps += p0 + p1;
        pk[c / 2] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      l = l * alpha + ps;
      // the P buffer is free once PV_{t-2} completed
      if (t >= 2) {
        ok = __all_sync(0xffffffff, sm100::mbar_wait(&p_free[sb], ((t >> 1) - 1) & 1, a.err));
        if (!ok) break;
      }
      // rescale O rows in TMEM once PV_{t-1} completed (warp-wide, rare after the first tiles)
      if (__any_sync(0xffffffff, grow && t > 0)) {
        ok = __all_sync(0xffffffff, sm100::mbar_wait(o_done, (t - 1) & 1, a.err));
        if (!ok) break;
        sm100::tc_fence_after();
        const float f = grow ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          float o[32];
          sm100::tmem_ld32(tmem + lane_off + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= f;
          sm100::tmem_st32(tmem + lane_off + c, o);
        }
      }
      // P row -> shared memory, K-major 128-byte swizzle (16-byte chunk c at c ^ (row % 8))
      uint8_t* prow = sP + sb * C::P_BYTES + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 q4 = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = q4;
      }
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&p_full[sb]);
    }
    // epilogue: out = bf16(O / l) * bf16(sigmoid(gate))
    if (ok) ok = __all_sync(0xffffffff, sm100::mbar_wait(o_last, 0, a.err));
    if (ok) {
      sm100::tc_fence_after();
      const float inv = 1.f / l;
      const bool valid = qi < a.s;
      const int64_t tok = (int64_t)tok0 + qi;
      const bf16* g = a.gate + tok * a.g_ts + (int64_t)h * a.g_hs;
      bf16* o = a.out + (tok * a.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float v[32];
        sm100::tmem_ld32(tmem + lane_off + c, v);
        if (!valid) continue;
        uint4 graw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) graw[i] = reinterpret_cast<const uint4*>(g + c)[i];
        const bf16* gv = reinterpret_cast<const bf16*>(graw);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float g0 = bf(gv[i]), g1 = bf(gv[i + 1]);
          const float s0 = rb(1.f / (1.f + expf(-g0))), s1 = rb(1.f / (1.f + expf(-g1)));
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(rb(v[i] * inv) * s0, rb(v[i + 1] * inv) * s1);
          pk[i / 2] = *reinterpret_cast<const uint32_t*>(&h2);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<uint4*>(o + c)[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace vattn

// y [rows, D] = partial-RoPE((1+w)-RMSNorm(x rows)); x rows addressed as described above.
void head_norm_rope(at::Tensor x, int64_t H, int64_t x_ts, int64_t x_hs, int64_t S, at::Tensor w, double eps,
                    at::Tensor cs, at::Tensor sn, int64_t rd, at::Tensor y) {
  const int D = (int)y.size(-1);
  const int64_t rows = y.numel() / D;
  if (rows == 0) return;
  NS_CHECK(y.is_contiguous() && cs.is_contiguous() && sn.is_contiguous(), "head_norm_rope: contiguous outputs");
  NS_CHECK(rd % 2 == 0 && rd <= D, "rotary_dim must be even and <= head_dim");
  const unsigned grid = (unsigned)((rows + 7) / 8);
  const auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  const auto* wp = reinterpret_cast<const bf16*>(w.data_ptr());
  const auto* cp = reinterpret_cast<const bf16*>(cs.data_ptr());
  const auto* sp = reinterpret_cast<const bf16*>(sn.data_ptr());
  auto* yp = reinterpret_cast<bf16*>(y.data_ptr());
#define NS_HNR(DD)                                                                                         \
  case DD:                                                                                                 \
    vattn::head_norm_rope_kernel<DD><<<grid, 256, 0, stream()>>>(xp, x_ts, x_hs, (int)H, rows, (int)S, wp, \
                                                                 (float)eps, cp, sp, (int)rd, yp);         \
    break;
  switch (D) {
    NS_HNR(16)
    NS_HNR(32)
    NS_HNR(64)
    NS_HNR(128)
    NS_HNR(256)
    default: NS_CHECK(false, "head_norm_rope: head_dim must be 16, 32, 64, 128 or 256");
  }
#undef NS_HNR
  NS_CUDA(cudaGetLastError());
}

template <int D>
static void vattn_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& gate,
                         int64_t g_ts, int64_t g_hs, at::Tensor& out) {
  using C = vattn::Cfg<D>;
  const int b = q.size(0), s = q.size(1), Hq = q.size(2), Hk = k.size(2);
  const int64_t rows = (int64_t)b * s;
  // [tokens][heads][D] views; box = 64 channels x 1 head x (128 | 64) tokens
  CUtensorMap tq = make_tmap_bf16_3d(q.data_ptr(), D, Hq, rows, D, (int64_t)Hq * D, 64, 1, vattn::BM);
  CUtensorMap tk = make_tmap_bf16_3d(k.data_ptr(), D, Hk, rows, k.stride(2), k.stride(1), 64, 1, vattn::BN);
  CUtensorMap tv = make_tmap_bf16_3d(v.data_ptr(), D, Hk, rows, v.stride(2), v.stride(1), 64, 1, vattn::BN);
  vattn::Args a{};
  a.s = s;
  a.Hq = Hq;
  a.Hk = Hk;
  a.scale_log2 = (1.f / std::sqrt((float)D)) * 1.4426950408889634f;
  a.gate = reinterpret_cast<const bf16*>(gate.data_ptr());
  a.g_ts = g_ts;
  a.g_hs = g_hs;
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.err = device_error_flag();
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(vattn::vattn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
  });
  const dim3 grid((s + vattn::BM - 1) / vattn::BM, Hq, b);
  vattn::vattn_fwd_kernel<D><<<grid, 192, C::SMEM, stream()>>>(tq, tk, tv, a);
  NS_CUDA(cudaGetLastError());
}

// out [b, s, Hq, D] = causal GQA attention of already normalised, RoPE'd q [b, s, Hq, D]
// (contiguous) over k, v [b, s, Hk, D] (rows of D contiguous channels), times
// sigmoid(gate); gate(b, t, h, :) at gate + (b * s + t) * g_ts + h * g_hs.
void vattn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor gate, int64_t g_ts, int64_t g_hs, at::Tensor out) {
  check_bf16(q, "q");
  check_bf16(k, "k");
  check_bf16(v, "v");
  NS_CHECK(q.is_contiguous() && out.is_contiguous(), "vattn_fwd: q and out must be contiguous");
  NS_CHECK(k.stride(3) == 1 && v.stride(3) == 1 && k.stride(0) == k.size(1) * k.stride(1) &&
               v.stride(0) == v.size(1) * v.stride(1),
           "vattn_fwd: k / v must be [tokens][heads][D] views with unit channel stride and one token stride");
  NS_CHECK(q.size(2) % k.size(2) == 0, "query heads must be a multiple of key heads");
  if (q.size(1) == 0) return;
  switch (q.size(3)) {
    case 64: vattn_launch<64>(q, k, v, gate, g_ts, g_hs, out); break;
    case 128: vattn_launch<128>(q, k, v, gate, g_ts, g_hs, out); break;
    case 256: vattn_launch<256>(q, k, v, gate, g_ts, g_hs, out); break;
    default: NS_CHECK(false, "vattn_fwd: head_dim must be 64, 128 or 256");
  }
}

}  // namespace ns
