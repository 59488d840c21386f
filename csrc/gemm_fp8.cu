// Block-scaled FP8 projection for the frozen verifier on tcgen05 (kind::f8f6f4).
//
//   y[t, n] = sum_kb  sa[t, kb] * sb[n/128, kb] * sum_{k in block kb} qa[t, k] qb[n, k]
//
// qa/sa: activations quantised per token per 128 channels (e4m3, scale = amax/448);
// qb/sb: e4m3 weights with one fp32 scale per 128 x 128 block (weight_scale_inv).
// The scales are arbitrary fp32 (not powers of two), so they cannot be folded into
// the MMA as microscaling factors. Instead each 128-wide K block is accumulated by
// the tensor cores into its own TMEM buffer (two buffers alternate), and the
// epilogue warps promote it: acc += sa * sb * partial, in fp32 registers, while the
// tensor cores already work on the next K block.
//
// Tiles of 128 tokens x 256 output channels (128 when N is not a multiple of 256), one
// persistent CTA per SM; see fp8_gemm_kernel below for the warp roles.
#include "common.h"
#include "sm100.cuh"

#include <cuda_fp8.h>

namespace ns {

constexpr int F8_BM = 128, F8_BK = 128;

template <int BN>
struct F8Cfg {
  static constexpr int STAGE = F8_BM * F8_BK + BN * F8_BK;  // bytes
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 512;
  static constexpr int CPW = 128;                           // columns promoted per warp
  static constexpr int SEGS = BN / CPW;                     // column segments per TMEM lane quarter
  static constexpr int PWARPS = 4 * SEGS;                   // promotion warps
  static constexpr int THREADS = 64 + 32 * PWARPS;
  static constexpr int TMEM_COLS = 2 * BN;                  // two partial buffers
};

// kind::f8f6f4 instruction descriptor: e4m3 x e4m3 -> f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// acc[0..1] += f * v[0..1] with one paired fp32 FMA (fma.rn.f32x2, sm_100): half the
// issue slots of the promotion's scalar FMAs.
__device__ __forceinline__ void ffma2(float& a0, float& a1, float f, float v0, float v1) {
  uint64_t acc, vv, ff;
  asm("mov.b64 %0, {%1, %2};" : "=l"(acc) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(vv) : "f"(v0), "f"(v1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(ff) : "f"(f));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(ff), "l"(vv));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(acc));
}

struct F8Args {
  int M, N, K;
  const float* sa;  // [M, K/128]
  const float* sb;  // [N/128, K/128]
  __nv_bfloat16* out;
  int64_t ldo;
  int* err;
};

// Persistent: CTA c walks tiles c, c + grid, ... (m-tile fastest, so CTAs running at
// the same time share weight tiles in L2). The smem ring, the two TMEM partial
// buffers and every barrier phase continue across tile boundaries (a global K-block
// counter `it`), so the next tile's MMAs start while this tile's last partial is
// promoted and stored. Warps: 0 TMA producer, 1 TMEM owner + MMA issuer, 2.. the
// promotion warps (4 * BN / 128 of them; warp w owns TMEM lane quarter w % 4 and the
// 128-column segment (w - 2) / 4 of the tile, which is one 128-wide weight-scale
// block). Sixteen warps of 64 columns each were measured slower: the register cap of
// 576 threads spills the accumulators.
template <int BN>
__global__ void __launch_bounds__(F8Cfg<BN>::THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, F8Args args) {
  using C = F8Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * F8_BM * F8_BK;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * BN * F8_BK);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;  // [2] partial buffer ready
  uint64_t* tempty = tfull + 2;         // [2] partial buffer drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (args.K + F8_BK - 1) / F8_BK;
  const int mt = (args.M + F8_BM - 1) / F8_BM, nt = args.N / BN;
  const int tiles = mt * nt;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&tfull[b], 1);
      sm100::mbar_init(&tempty[b], 32 * C::PWARPS);
    }
    sm100::fence_barrier_init();
    sm100::tma_prefetch_desc(&ta);
    sm100::tma_prefetch_desc(&tb);
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
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int m0 = (tile % mt) * F8_BM, n0 = (tile / mt) * BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % C::STAGES;
          if (it >= C::STAGES && !sm100::mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1, args.err)) {
            ok = false;
            break;
          }
          sm100::mbar_expect_tx(&full[s], C::STAGE);
          sm100::tma_load_2d(sA + s * F8_BM * F8_BK, &ta, &full[s], kb * F8_BK, m0);
          sm100::tma_load_2d(sB + s * BN * F8_BK, &tb, &full[s], kb * F8_BK, n0);
        }
      }
      // drain: the last loads of every stage have landed before the CTA exits
      for (int i = max(0, it - C::STAGES); i < it; ++i)
        sm100::mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, args.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3(F8_BM, BN);
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % C::STAGES;
          const int buf = it & 1;
          if (it >= 2 && !sm100::mbar_wait(&tempty[buf], ((it >> 1) - 1) & 1, args.err)) { ok = false; break; }
          if (!sm100::mbar_wait(&full[s], (it / C::STAGES) & 1, args.err)) { ok = false; break; }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_u32(sA + s * F8_BM * F8_BK);
          const uint32_t b_base = sm100::smem_u32(sB + s * BN * F8_BK);
          const uint32_t d = tmem + (uint32_t)(buf * BN);
#pragma unroll
          for (int kk = 0; kk < F8_BK / 32; ++kk) {
            const uint64_t ad = sm100::smem_desc_sw128(a_base + kk * 32, 0, 1024);
            const uint64_t bd = sm100::smem_desc_sw128(b_base + kk * 32, 0, 1024);
            mma_f8(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
          sm100::mma_commit(&empty[s]);
          sm100::mma_commit(&tfull[buf]);
        }
      }
    }
  } else {
    constexpr int CPW = C::CPW;
    const int q = warp & 3;
    const int seg = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const int kbs = (args.K + 127) / 128;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
      const int m0 = (tile % mt) * F8_BM, n0 = (tile / mt) * BN;
      const int m = m0 + row;
      const int nb = (n0 + seg * CPW) / 128;
      float acc[CPW];
#pragma unroll
      for (int j = 0; j < CPW; ++j) acc[j] = 0.f;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int buf = it & 1;
        // the block scales do not depend on the MMA: load them before the wait so
        // their latency hides behind it
        const float sbv = args.sb[nb * kbs + kb];
        const float sav = (m < args.M) ? args.sa[(int64_t)m * kbs + kb] : 0.f;
        ok = sm100::mbar_wait(&tfull[buf], (it >> 1) & 1, args.err);
        if (!ok) break;
        sm100::tc_fence_after();
        const float f = sav * sbv;
#pragma unroll
        for (int c = 0; c < CPW; c += 32) {
          float v[32];
          sm100::tmem_ld32(tmem + lane_off + (uint32_t)(buf * BN + seg * CPW + c), v);
#pragma unroll
          for (int j = 0; j < 32; j += 2) ffma2(acc[c + j], acc[c + j + 1], f, v[j], v[j + 1]);
        }
        sm100::tc_fence_before();
        sm100::mbar_arrive(&tempty[buf]);
      }
      if (ok && m < args.M) {
        uint4* p = reinterpret_cast<uint4*>(args.out + (int64_t)m * args.ldo + n0 + seg * CPW);
#pragma unroll
        for (int j = 0; j < CPW / 8; ++j) {
          __nv_bfloat162 h[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) h[t] = __floats2bfloat162_rn(acc[8 * j + 2 * t], acc[8 * j + 2 * t + 1]);
          p[j] = *reinterpret_cast<uint4*>(h);
        }
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

// 1 x 128 dynamic activation quantisation: one warp per (token, 128-channel block).
__global__ void quant_e4m3_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int K, uint8_t* __restrict__ q,
                                  float* __restrict__ scale) {
  const int64_t wid = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int kbs = K / 128;
  if (wid >= rows * kbs) return;
  const int64_t r = wid / kbs;
  const int kb = (int)(wid % kbs);
  const __nv_bfloat16* src = x + r * K + kb * 128 + lane * 4;
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __bfloat162float(src[i]);
    amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, o));
  const float s = amax / 448.f;
  const float denom = fmaxf(s, 1.17549435e-38f);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float y = fminf(fmaxf(v[i] / denom, -448.f), 448.f);
    const __nv_fp8_storage_t b = __nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3);
    packed |= (uint32_t)b << (8 * i);
  }
  *reinterpret_cast<uint32_t*>(q + r * K + kb * 128 + lane * 4) = packed;
  if (lane == 0) scale[r * kbs + kb] = s;
}

static CUtensorMap make_tmap_u8(const void* base, int64_t rows, int64_t cols, int box_rows) {
  NS_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  NS_CHECK(cols % 16 == 0, "fp8 rows must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NS_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (fp8) failed");
  return map;
}

// out [T, N] bf16 = block-scaled GEMM of pre-quantised activations q [T, K] (e4m3 codes
// as uint8) with scales sa [T, K/128] and e4m3 weights w [N, K] with scale_inv
// [N/128, K/128].
void fp8_gemm(at::Tensor q, at::Tensor sa, at::Tensor w, at::Tensor scale_inv, at::Tensor out) {
  NS_CHECK(q.is_contiguous() && w.is_contiguous() && sa.is_contiguous(), "fp8_gemm: contiguous operands expected");
  NS_CHECK(out.stride(1) == 1, "fp8_gemm: output rows must be contiguous");
  NS_CHECK(w.scalar_type() == at::kFloat8_e4m3fn, "weight must be float8_e4m3fn");
  const int64_t T = q.size(0);
  const int K = q.size(1), N = w.size(0);
  NS_CHECK(K % 128 == 0 && N % 128 == 0 && w.size(1) == K, "FP8 weights need 128 x 128 blocks");
  NS_CHECK(scale_inv.scalar_type() == at::kFloat && scale_inv.size(0) == N / 128 && scale_inv.size(1) == K / 128,
           "weight_scale_inv must be fp32 [N/128, K/128]");
  NS_CHECK(sa.scalar_type() == at::kFloat && sa.size(0) == T && sa.size(1) == K / 128, "sa must be fp32 [T, K/128]");
  if (T == 0) return;
  NS_CHECK((out.stride(0) % 8) == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "fp8_gemm: output rows must be 16-byte aligned");
  F8Args a{};
  a.M = (int)T;
  a.N = N;
  a.K = K;
  a.sa = sa.data_ptr<float>();
  a.sb = scale_inv.contiguous().data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  a.err = device_error_flag();
  CUtensorMap ta = make_tmap_u8(q.data_ptr(), T, K, F8_BM);
  const int mt = (int)((T + F8_BM - 1) / F8_BM);
  if (N % 256 == 0) {
    using C = F8Cfg<256>;
    CUtensorMap tb = make_tmap_u8(w.data_ptr(), N, K, 256);
    static std::atomic<unsigned long long> attr{0};
    once_per_device(attr, [&] {
      NS_CUDA(cudaFuncSetAttribute(fp8_gemm_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    });
    const int grid = std::min(mt * (N / 256), num_sms());
    fp8_gemm_kernel<256><<<grid, C::THREADS, C::SMEM, stream()>>>(ta, tb, a);
  } else {
    using C = F8Cfg<128>;
    CUtensorMap tb = make_tmap_u8(w.data_ptr(), N, K, 128);
    static std::atomic<unsigned long long> attr{0};
    once_per_device(attr, [&] {
      NS_CUDA(cudaFuncSetAttribute(fp8_gemm_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    });
    const int grid = std::min(mt * (N / 128), num_sms());
    fp8_gemm_kernel<128><<<grid, C::THREADS, C::SMEM, stream()>>>(ta, tb, a);
  }
  NS_CUDA(cudaGetLastError());
}

// 1 x 128 dynamic quantisation of bf16 rows x [T, K] into q (uint8 e4m3 codes) and s.
void quant_e4m3(at::Tensor x, at::Tensor q, at::Tensor s) {
  check_bf16(x, "x");
  NS_CHECK(x.is_contiguous() && x.size(1) % 128 == 0, "quant_e4m3: contiguous rows of 128-multiples");
  const int64_t T = x.size(0);
  const int K = x.size(1);
  const int64_t warps = T * (K / 128);
  if (warps == 0) return;
  quant_e4m3_kernel<<<(warps * 32 + 255) / 256, 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), T, K, q.data_ptr<uint8_t>(), s.data_ptr<float>());
  NS_CUDA(cudaGetLastError());
}

// Quantise x, then the block-scaled GEMM: writes out [T, N] bf16.
void fp8_linear(at::Tensor x, at::Tensor w, at::Tensor scale_inv, at::Tensor out) {
  check_bf16(x, "x");
  NS_CHECK(x.is_contiguous() && out.is_contiguous(), "fp8_linear: contiguous tensors expected");
  const int64_t T = x.size(0);
  const int K = x.size(1);
  if (T == 0) return;
  auto q = at::empty({T, K}, x.options().dtype(at::kByte));
  auto sa = at::empty({T, K / 128}, x.options().dtype(at::kFloat));
  quant_e4m3(x, q, sa);
  fp8_gemm(q, sa, w, scale_inv, out);
}

}  // namespace ns
