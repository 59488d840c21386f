// Draft attention on 5th-generation tensor cores (forward, dQ, dK/dV), head dim 64 or 128.
//
// Same op as attention.cu (reference: nanospec/ops.py:129-162 with the anchor-prefix +
// own-block mask of nanospec/dspark.py:128-132): query block j of batch row i sees the
// context keys [0, anchors[i, j]) and its own block's draft keys; a block with keep ==
// false sees nothing (output 0, lse -inf). Keys and values are in split layout.
//
// Tiling: the G = Hq / Hk query heads that share a key head attend the same keys, so
// a 128-row query tile stacks QB consecutive blocks x G heads x block_size slots
// (each block padded to RB = roundup8(G * bs) rows; 3 blocks of 35 rows at the qwen
// shape). Its keys are the context prefix up to the largest anchor among its blocks
// (64-key tiles) plus one tile holding the blocks' draft keys; every row masks the keys
// it does not see. All tiles arrive by 3-D TMA maps over [tokens][heads][D] (this
// GPU's memory, no multicast).
//  * forward: S = Q K^T and O += P V in TMEM, online softmax by 128 row threads
//    (lazy rescale as in vattn.cu), P as a swizzled bf16 operand; S_{t+1} overlaps the
//    softmax of tile t.
//  * dQ: per key tile S = Q K^T and dP = dO V^T, dS = P (dP - delta) written as an
//    operand, dQ += dS K.
//  * dK / dV: one CTA per 128 context keys (or per query tile's draft keys) walks the
//    query tiles that see them: S^T = K Q^T, dP^T = V dO^T, then dV += P^T dO and
//    dK += dS^T Q. The G heads of a key head are rows of the same tiles, so their sum
//    happens inside the MMA: deterministic, no atomics, no partial buffers.
// Every mbarrier wait is bounded (device error word on timeout).
#include "common.h"
#include "sm100.cuh"

namespace ns {

using bf16 = __nv_bfloat16;

namespace dattn {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 64;   // keys per tile (forward, dQ)
constexpr int BK = 128;  // keys per tile (dK / dV)
constexpr float RESCALE_LOG2 = 8.f;

struct Args {
  int b, S, nb, bs, Hq, Hk, G, RB, QB, nqt;
  int Td;
  const int64_t* anchors;  // [b, nb]
  const bool* keep;        // [b, nb]
  float scale, scale_log2;
  bf16* out;               // [b, Td, Hq, D]
  float* lse;              // [b, Hq, Td]
  const bf16* o;           // forward output (backward)
  const bf16* dout;        // [b, Td, Hq, D]
  bf16* dq;                // [b, Td, Hq, D]
  bf16 *dk, *dv;           // split-layout rows, head hk at + hk * D
  int64_t lddk, lddv;
  int* err;
};

__device__ __forceinline__ float bf(bf16 x) { return __bfloat162float(x); }

// Row r of query tile qt: block j, slot, head offset g in the group; false for padding.
__device__ __forceinline__ bool row_info(const Args& a, int qt, int r, int& j, int& slot, int& g) {
  const int jj = r / a.RB, local = r - jj * a.RB;
  j = qt * a.QB + jj;
  if (jj >= a.QB || local >= a.G * a.bs || j >= a.nb) return false;
  slot = local / a.G;
  g = local - slot * a.G;
  return true;
}

// Largest anchor among the kept blocks of query tile qt (0 if none).
__device__ __forceinline__ int tile_max_anchor(const Args& a, int bi, int qt) {
  int m = 0;
  for (int jj = 0; jj < a.QB; ++jj) {
    const int j = qt * a.QB + jj;
    if (j < a.nb && a.keep[bi * a.nb + j]) m = max(m, (int)a.anchors[bi * a.nb + j]);
  }
  return m;
}

// TMA loads of query tile qt (Q or dO) into a [BM][D] K-major swizzled tile; returns bytes.
template <int D>
__device__ __forceinline__ uint32_t load_qtile(const Args& a, const CUtensorMap* map, uint8_t* dst, uint64_t* bar,
                                               int bi, int hk, int qt, bool issue) {
  uint32_t bytes = 0;
  for (int jj = 0; jj < a.QB; ++jj) {
    const int j = qt * a.QB + jj;
    if (j >= a.nb) break;
    bytes += (uint32_t)(D / 64) * 128u * a.G * a.bs;
  }
  if (issue) {
    sm100::mbar_expect_tx(bar, bytes);
    for (int jj = 0; jj < a.QB; ++jj) {
      const int j = qt * a.QB + jj;
      if (j >= a.nb) break;
#pragma unroll
      for (int at = 0; at < D / 64; ++at)
        sm100::tma_load_3d(dst + at * (BM * 128) + jj * a.RB * 128, map, bar, 64 * at, hk * a.G, bi * a.Td + j * a.bs);
    }
  }
  return bytes;
}

// Zero a [rows][D] swizzled tile (padding rows must be finite zeros, not stale data).
template <int D>
__device__ __forceinline__ void zero_tile(uint8_t* t, int rows, int tid, int nth) {
  uint4* p = reinterpret_cast<uint4*>(t);
  const int n = rows * D * 2 / 16;
  for (int i = tid; i < n; i += nth) p[i] = make_uint4(0u, 0u, 0u, 0u);
}

__device__ __forceinline__ uint32_t pack2(float x, float y) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Write 64 values (one row, keys/rows [c0, c0 + 64)) of a K-major bf16 operand with
// 128-byte swizzle: atom `atom`, row `row`.
__device__ __forceinline__ void store_row64(uint8_t* base, int atom_bytes, int atom, int row, const float* v) {
  uint8_t* r = base + atom * atom_bytes + row * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 q = make_uint4(pack2(v[8 * c], v[8 * c + 1]), pack2(v[8 * c + 2], v[8 * c + 3]),
                               pack2(v[8 * c + 4], v[8 * c + 5]), pack2(v[8 * c + 6], v[8 * c + 7]));
    *reinterpret_cast<uint4*>(r + ((c ^ (row & 7)) << 4)) = q;
  }
}

// ============================================================================ forward
template <int D>
struct Fwd {
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int K_BYTES = BN * D * 2;
  static constexpr int KV_BYTES = 2 * K_BYTES;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int SMEM = Q_BYTES + 2 * KV_BYTES + 2 * P_BYTES + 1024 + 256;
  static constexpr int TMEM_COLS = D + 2 * BN <= 256 ? 256 : 512;
  static constexpr int S_COL = D;
};

template <int D>
__global__ void __launch_bounds__(192, 1) dattn_fwd_kernel(const __grid_constant__ CUtensorMap tq,
                                                           const __grid_constant__ CUtensorMap tk,
                                                           const __grid_constant__ CUtensorMap tv, Args a) {
  using C = Fwd<D>;
  constexpr int DA = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + C::Q_BYTES;
  uint8_t* sP = sKV + 2 * C::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 7;
  uint64_t* p_full = bars + 9;
  uint64_t* p_free = bars + 11;
  uint64_t* o_done = bars + 13;
  uint64_t* o_last = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // later blocks have longer prefixes
  const int hk = blockIdx.y, bi = blockIdx.z;
  const int maxa = tile_max_anchor(a, bi, qt);
  const int nctx = (maxa + BN - 1) / BN;
  const int nkt = nctx + 1;  // + the draft-key tile

  zero_tile<D>(sQ, BM, threadIdx.x, blockDim.x);
  sm100::fence_proxy_async_smem();
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
      load_qtile<D>(a, &tq, sQ, q_full, bi, hk, qt, true);
      int issued = 0;
      for (int t = 0; t < nkt; ++t) {
        const int st = t & 1;
        if (t >= 2 && !sm100::mbar_wait(&kv_empty[st], ((t >> 1) - 1) & 1, a.err)) break;
        const int row = t < nctx ? bi * a.S + t * BN : a.b * a.S + bi * a.Td + qt * a.QB * a.bs;
        uint8_t* kd = sKV + st * C::KV_BYTES;
        sm100::mbar_expect_tx(&kv_full[st], C::KV_BYTES);
#pragma unroll
        for (int at = 0; at < DA; ++at) {
          sm100::tma_load_3d(kd + at * (BN * 128), &tk, &kv_full[st], 64 * at, hk, row);
          sm100::tma_load_3d(kd + C::K_BYTES + at * (BN * 128), &tv, &kv_full[st], 64 * at, hk, row);
        }
        issued = t + 1;
      }
      sm100::mbar_wait(q_full, 0, a.err);
      for (int t = max(0, issued - 2); t < issued; ++t) sm100::mbar_wait(&kv_full[t & 1], (t >> 1) & 1, a.err);
    }
  } else if (warp == 1) {
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
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = sm100::smem_desc_sw128(q_base + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bd = sm100::smem_desc_sw128(k_base + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 0, 1024);
          sm100::mma_bf16(tmem + C::S_COL + st * BN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
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
    const int qw = warp & 3;
    const int row = qw * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    int j = 0, slot = 0, g = 0;
    const bool valid = row_info(a, qt, row, j, slot, g);
    const bool kp = valid && a.keep[bi * a.nb + j];
    const int anchor = kp ? (int)a.anchors[bi * a.nb + j] : 0;
    const int jj = row / a.RB;
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
      float mt = -INFINITY;
      const bool draft = t == nctx;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        const bool vis = kp && (draft ? (c / a.bs == jj && c < a.QB * a.bs) : (t * BN + c < anchor));
        const float x = vis ? sv[c] * a.scale_log2 : -INFINITY;
        sv[c] = x;
        mt = fmaxf(mt, x);
      }
      float alpha = 1.f;
      bool grow = false;
      if (mt > m_used + RESCALE_LOG2) {
        alpha = exp2f(m_used - mt);
        m_used = mt;
        grow = true;
      }
      float ps = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float p0 = sv[c] == -INFINITY ? 0.f : exp2f(sv[c] - m_used);
        const float p1 = sv[c + 1] == -INFINITY ? 0.f : exp2f(sv[c + 1] - m_used);
        ps += p0 + p1;
        pk[c / 2] = pack2(p0, p1);
      }
      l = l * alpha + ps;
      if (t >= 2) {
        ok = __all_sync(0xffffffff, sm100::mbar_wait(&p_free[sb], ((t >> 1) - 1) & 1, a.err));
        if (!ok) break;
      }
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
      uint8_t* prow = sP + sb * C::P_BYTES + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&p_full[sb]);
    }
    if (ok) ok = __all_sync(0xffffffff, sm100::mbar_wait(o_last, 0, a.err));
    if (ok) {
      sm100::tc_fence_after();
      const bool live = valid && l > 0.f;
      const float inv = live ? 1.f / l : 0.f;
      const int h = hk * a.G + g;
      const int tok = j * a.bs + slot;
      bf16* op = a.out + (((int64_t)bi * a.Td + tok) * a.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float v[32];
        sm100::tmem_ld32(tmem + lane_off + c, v);
        if (!valid) continue;
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) pk[i / 2] = pack2(v[i] * inv, v[i + 1] * inv);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<uint4*>(op + c)[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
      if (valid)
        a.lse[((int64_t)bi * a.Hq + h) * a.Td + tok] = live ? (m_used + log2f(l)) * 0.6931471805599453f : -INFINITY;
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ============================================================================ dQ
template <int D>
struct Dq {
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int K_BYTES = BN * D * 2;
  static constexpr int KV_BYTES = 2 * K_BYTES;
  static constexpr int DS_BYTES = BM * BN * 2;
  static constexpr int SMEM = 2 * Q_BYTES + KV_BYTES + DS_BYTES + 1024 + 256;
  static constexpr int S_COL = D, P_COL = D + BN;  // dQ at 0, S, dP after it
  static constexpr int TMEM_COLS = D + 2 * BN <= 256 ? 256 : 512;
};

// Serial per key tile: [TMA K, V] -> S = Q K^T, dP = dO V^T -> rows: dS -> dQ += dS K.
template <int D>
__global__ void __launch_bounds__(192, 1) dattn_dq_kernel(const __grid_constant__ CUtensorMap tq,
                                                          const __grid_constant__ CUtensorMap tdo,
                                                          const __grid_constant__ CUtensorMap tk,
                                                          const __grid_constant__ CUtensorMap tv, Args a) {
  using C = Dq<D>;
  constexpr int DA = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sO = sQ + C::Q_BYTES;        // dO tile
  uint8_t* sKV = sO + C::Q_BYTES;
  uint8_t* sDS = sKV + C::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + C::DS_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* sd_full = bars + 2;   // S, dP ready
  uint64_t* ds_full = bars + 3;   // dS written (4 warps)
  uint64_t* mm_done = bars + 4;   // dQ MMA of the tile done (kv and dS reusable)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;
  const int hk = blockIdx.y, bi = blockIdx.z;
  const int maxa = tile_max_anchor(a, bi, qt);
  const int nctx = (maxa + BN - 1) / BN;
  const int nkt = nctx + 1;

  zero_tile<D>(sQ, 2 * BM, threadIdx.x, blockDim.x);  // Q and dO
  sm100::fence_proxy_async_smem();
  if (warp == 0 && lane == 0) {
    sm100::mbar_init(q_full, 1);
    sm100::mbar_init(kv_full, 1);
    sm100::mbar_init(sd_full, 1);
    sm100::mbar_init(ds_full, 4);
    sm100::mbar_init(mm_done, 1);
    sm100::fence_barrier_init();
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
      const uint32_t bq = load_qtile<D>(a, &tq, sQ, q_full, bi, hk, qt, false);
      sm100::mbar_expect_tx(q_full, 2 * bq);
      for (int jj = 0; jj < a.QB; ++jj) {
        const int j = qt * a.QB + jj;
        if (j >= a.nb) break;
#pragma unroll
        for (int at = 0; at < DA; ++at) {
          sm100::tma_load_3d(sQ + at * (BM * 128) + jj * a.RB * 128, &tq, q_full, 64 * at, hk * a.G, bi * a.Td + j * a.bs);
          sm100::tma_load_3d(sO + at * (BM * 128) + jj * a.RB * 128, &tdo, q_full, 64 * at, hk * a.G,
                             bi * a.Td + j * a.bs);
        }
      }
      int issued = 0;
      for (int t = 0; t < nkt; ++t) {
        if (t >= 1 && !sm100::mbar_wait(mm_done, (t - 1) & 1, a.err)) break;
        const int row = t < nctx ? bi * a.S + t * BN : a.b * a.S + bi * a.Td + qt * a.QB * a.bs;
        sm100::mbar_expect_tx(kv_full, C::KV_BYTES);
#pragma unroll
        for (int at = 0; at < DA; ++at) {
          sm100::tma_load_3d(sKV + at * (BN * 128), &tk, kv_full, 64 * at, hk, row);
          sm100::tma_load_3d(sKV + C::K_BYTES + at * (BN * 128), &tv, kv_full, 64 * at, hk, row);
        }
        issued = t + 1;
      }
      sm100::mbar_wait(q_full, 0, a.err);
      if (issued > 0) sm100::mbar_wait(kv_full, (issued - 1) & 1, a.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = sm100::idesc_bf16(BM, BN, false, false);
      constexpr uint32_t id_q = sm100::idesc_bf16(BM, D, false, true);
      const uint32_t q_base = sm100::smem_u32(sQ), o_base = sm100::smem_u32(sO);
      const uint32_t k_base = sm100::smem_u32(sKV), v_base = sm100::smem_u32(sKV + C::K_BYTES);
      const uint32_t ds_base = sm100::smem_u32(sDS);
      bool ok = sm100::mbar_wait(q_full, 0, a.err);
      for (int t = 0; ok && t < nkt; ++t) {
        if (!sm100::mbar_wait(kv_full, t & 1, a.err)) break;
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t aq = sm100::smem_desc_sw128(q_base + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t ao = sm100::smem_desc_sw128(o_base + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bk = sm100::smem_desc_sw128(k_base + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bv = sm100::smem_desc_sw128(v_base + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 0, 1024);
          sm100::mma_bf16(tmem + C::S_COL, aq, bk, id_s, kk > 0 ? 1u : 0u);
          sm100::mma_bf16(tmem + C::P_COL, ao, bv, id_s, kk > 0 ? 1u : 0u);
        }
        sm100::mma_commit(sd_full);
        if (!sm100::mbar_wait(ds_full, t & 1, a.err)) break;
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = sm100::smem_desc_sw128(ds_base + kk * 32, 0, 1024);
          const uint64_t bd = sm100::smem_desc_sw128(k_base + kk * 2048, BN * 128, 1024);
          sm100::mma_bf16(tmem, ad, bd, id_q, (t > 0 || kk > 0) ? 1u : 0u);
        }
        sm100::mma_commit(mm_done);
      }
    }
  } else {
    const int qw = warp & 3;
    const int row = qw * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    int j = 0, slot = 0, g = 0;
    const bool valid = row_info(a, qt, row, j, slot, g);
    const bool kp = valid && a.keep[bi * a.nb + j];
    const int anchor = kp ? (int)a.anchors[bi * a.nb + j] : 0;
    const int jj = row / a.RB;
    const int h = hk * a.G + g;
    const int tok = j * a.bs + slot;
    float lse2 = -INFINITY, delta = 0.f;
    if (kp) {
      const float lse = a.lse[((int64_t)bi * a.Hq + h) * a.Td + tok];
      lse2 = lse * 1.4426950408889634f;
      const bf16* orow = a.o + (((int64_t)bi * a.Td + tok) * a.Hq + h) * D;
      const bf16* drow = a.dout + (((int64_t)bi * a.Td + tok) * a.Hq + h) * D;
      for (int d = 0; d < D; ++d) delta += bf(orow[d]) * bf(drow[d]);
    }
    const bool live = kp && lse2 != -INFINITY;
    bool ok = true;
    for (int t = 0; t < nkt && ok; ++t) {
      ok = __all_sync(0xffffffff, sm100::mbar_wait(sd_full, t & 1, a.err));
      if (!ok) break;
      sm100::tc_fence_after();
      const bool draft = t == nctx;
      float ds[BN];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float sv[32], dp[32];
        sm100::tmem_ld32(tmem + lane_off + C::S_COL + half * 32, sv);
        sm100::tmem_ld32(tmem + lane_off + C::P_COL + half * 32, dp);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int kc = half * 32 + c;
          const bool vis = live && (draft ? (kc / a.bs == jj && kc < a.QB * a.bs) : (t * BN + kc < anchor));
          const float p = vis ? exp2f(sv[c] * a.scale_log2 - lse2) : 0.f;
          ds[kc] = p * (dp[c] - delta);
        }
      }
      // the previous tile's dQ MMA has read sDS (mm_done of t - 1 precedes this tile's kv_full)
      store_row64(sDS, BM * 128, 0, row, ds);
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(ds_full);
    }
    if (ok) ok = __all_sync(0xffffffff, sm100::mbar_wait(mm_done, (nkt - 1) & 1, a.err));
    if (ok) {
      sm100::tc_fence_after();
      bf16* qrow = a.dq + (((int64_t)bi * a.Td + tok) * a.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float v[32];
        sm100::tmem_ld32(tmem + lane_off + c, v);
        if (!valid) continue;
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) pk[i / 2] = pack2(v[i] * a.scale, v[i + 1] * a.scale);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<uint4*>(qrow + c)[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
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

// ============================================================================ dK / dV
template <int D>
struct Dkv {
  static constexpr int T_BYTES = BK * D * 2;   // K or V tile [128 keys][D]
  static constexpr int Q_BYTES = BM * D * 2;   // Q or dO tile
  static constexpr int OP_BYTES = BK * BM * 2; // P^T or dS^T [128 keys][128 rows], two atoms
  static constexpr int SMEM = 2 * T_BYTES + 2 * Q_BYTES + 2 * OP_BYTES + 2048 + 1024 + 256;
  static constexpr int S_COL = 0, P_COL = BM, K_COL = 2 * BM, V_COL = 2 * BM + D;  // TMEM
  static constexpr int TMEM_COLS = 512;
};

// grid.x: 128-key context tiles, then one tile of draft keys per query tile.
template <int D>
__global__ void __launch_bounds__(192, 1) dattn_dkv_kernel(const __grid_constant__ CUtensorMap tq,
                                                           const __grid_constant__ CUtensorMap tdo,
                                                           const __grid_constant__ CUtensorMap tk,
                                                           const __grid_constant__ CUtensorMap tv, Args a) {
  using C = Dkv<D>;
  constexpr int DA = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::T_BYTES;
  uint8_t* sQ = sV + C::T_BYTES;
  uint8_t* sO = sQ + C::Q_BYTES;
  uint8_t* sP = sO + C::Q_BYTES;         // P^T operand
  uint8_t* sD = sP + C::OP_BYTES;        // dS^T operand
  // [2 tiles][2][BM]: lse2, delta of the query rows, double-buffered by tile parity (a
  // warp may write the next tile's rows while another still reads this tile's)
  float* stat_all = reinterpret_cast<float*>(sD + C::OP_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(stat_all + 4 * BM);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* sd_full = bars + 2;
  uint64_t* pd_full = bars + 3;   // 4 warps
  uint64_t* mm_done = bars + 4;
  uint64_t* st_ready = bars + 5;  // 4 warps: stat of the current query tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.y, bi = blockIdx.z;
  const int nkc = (a.S + BK - 1) / BK;
  const bool draft = (int)blockIdx.x >= nkc;
  const int kt = draft ? (int)blockIdx.x - nkc : (int)blockIdx.x;  // context tile, or query tile of the draft keys
  const int key0 = draft ? 0 : kt * BK;
  // query tiles that see this key tile
  const int qt0 = draft ? kt : 0, qt1 = draft ? kt + 1 : a.nqt;

  zero_tile<D>(sQ, 2 * BM, threadIdx.x, blockDim.x);
  sm100::fence_proxy_async_smem();
  if (warp == 0 && lane == 0) {
    sm100::mbar_init(kv_full, 1);
    sm100::mbar_init(q_full, 1);
    sm100::mbar_init(sd_full, 1);
    sm100::mbar_init(pd_full, 4);
    sm100::mbar_init(mm_done, 1);
    sm100::mbar_init(st_ready, 4);
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, C::TMEM_COLS);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // rows of the K / V tile in the split layout
  const int krow = draft ? a.b * a.S + bi * a.Td + kt * a.QB * a.bs : bi * a.S + key0;

  if (warp == 0) {
    if (lane == 0) {
      sm100::mbar_expect_tx(kv_full, 2 * C::T_BYTES);
#pragma unroll
      for (int at = 0; at < DA; ++at) {
        sm100::tma_load_3d(sK + at * (BK * 128), &tk, kv_full, 64 * at, hk, krow);
        sm100::tma_load_3d(sV + at * (BK * 128), &tv, kv_full, 64 * at, hk, krow);
      }
      int n = 0;
      for (int qt = qt0; qt < qt1; ++qt) {
        if (!draft && tile_max_anchor(a, bi, qt) <= key0) continue;
        if (n >= 1 && !sm100::mbar_wait(mm_done, (n - 1) & 1, a.err)) break;
        const uint32_t bq = load_qtile<D>(a, &tq, sQ, q_full, bi, hk, qt, false);
        sm100::mbar_expect_tx(q_full, 2 * bq);
        for (int jj = 0; jj < a.QB; ++jj) {
          const int j = qt * a.QB + jj;
          if (j >= a.nb) break;
#pragma unroll
          for (int at = 0; at < DA; ++at) {
            sm100::tma_load_3d(sQ + at * (BM * 128) + jj * a.RB * 128, &tq, q_full, 64 * at, hk * a.G,
                               bi * a.Td + j * a.bs);
            sm100::tma_load_3d(sO + at * (BM * 128) + jj * a.RB * 128, &tdo, q_full, 64 * at, hk * a.G,
                               bi * a.Td + j * a.bs);
          }
        }
        ++n;
      }
      sm100::mbar_wait(kv_full, 0, a.err);
      if (n > 0) sm100::mbar_wait(q_full, (n - 1) & 1, a.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = sm100::idesc_bf16(BK, BM, false, false);  // [keys x rows], K = D
      constexpr uint32_t id_o = sm100::idesc_bf16(BK, D, false, true);    // [keys x D],   K = rows
      const uint32_t k_base = sm100::smem_u32(sK), v_base = sm100::smem_u32(sV);
      const uint32_t q_base = sm100::smem_u32(sQ), o_base = sm100::smem_u32(sO);
      const uint32_t p_base = sm100::smem_u32(sP), d_base = sm100::smem_u32(sD);
      bool ok = sm100::mbar_wait(kv_full, 0, a.err);
      int n = 0;
      for (int qt = qt0; ok && qt < qt1; ++qt) {
        if (!draft && tile_max_anchor(a, bi, qt) <= key0) continue;
        if (!sm100::mbar_wait(q_full, n & 1, a.err)) break;
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ak = sm100::smem_desc_sw128(k_base + (kk >> 2) * (BK * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t av = sm100::smem_desc_sw128(v_base + (kk >> 2) * (BK * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bq = sm100::smem_desc_sw128(q_base + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bo = sm100::smem_desc_sw128(o_base + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 0, 1024);
          sm100::mma_bf16(tmem + C::S_COL, ak, bq, id_s, kk > 0 ? 1u : 0u);
          sm100::mma_bf16(tmem + C::P_COL, av, bo, id_s, kk > 0 ? 1u : 0u);
        }
        sm100::mma_commit(sd_full);
        if (!sm100::mbar_wait(pd_full, n & 1, a.err)) break;
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk) {  // K = 128 query rows: two 64-row atoms
          const uint64_t ap = sm100::smem_desc_sw128(p_base + (kk >> 2) * (BK * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t ad = sm100::smem_desc_sw128(d_base + (kk >> 2) * (BK * 128) + (kk & 3) * 32, 0, 1024);
          const uint64_t bo = sm100::smem_desc_sw128(o_base + kk * 2048, BM * 128, 1024);
          const uint64_t bq = sm100::smem_desc_sw128(q_base + kk * 2048, BM * 128, 1024);
          sm100::mma_bf16(tmem + C::V_COL, ap, bo, id_o, (n > 0 || kk > 0) ? 1u : 0u);
          sm100::mma_bf16(tmem + C::K_COL, ad, bq, id_o, (n > 0 || kk > 0) ? 1u : 0u);
        }
        sm100::mma_commit(mm_done);
        ++n;
      }
    }
  } else {
    const int qw = warp & 3;
    const int kr = qw * 32 + lane;  // key row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const int key = key0 + kr;      // context key position (context tiles)
    const bool key_ok = draft ? kr < a.QB * a.bs && kt * a.QB + kr / a.bs < a.nb : key < a.S;
    int n = 0;
    bool ok = true;
    for (int qt = qt0; ok && qt < qt1; ++qt) {
      if (!draft && tile_max_anchor(a, bi, qt) <= key0) continue;
      float* stat = stat_all + (n & 1) * 2 * BM;
      // statistics of query row kr of this tile (thread kr computes row kr)
      {
        int j = 0, slot = 0, g = 0;
        float lse2 = -INFINITY, delta = 0.f;
        if (row_info(a, qt, kr, j, slot, g) && a.keep[bi * a.nb + j]) {
          const int h = hk * a.G + g, tok = j * a.bs + slot;
          const float lse = a.lse[((int64_t)bi * a.Hq + h) * a.Td + tok];
          lse2 = lse * 1.4426950408889634f;
          const bf16* orow = a.o + (((int64_t)bi * a.Td + tok) * a.Hq + h) * D;
          const bf16* drow = a.dout + (((int64_t)bi * a.Td + tok) * a.Hq + h) * D;
          for (int d = 0; d < D; ++d) delta += bf(orow[d]) * bf(drow[d]);
        }
        stat[kr] = lse2;
        stat[BM + kr] = delta;
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(st_ready);
      }
      ok = __all_sync(0xffffffff, sm100::mbar_wait(st_ready, n & 1, a.err));
      if (!ok) break;
      ok = __all_sync(0xffffffff, sm100::mbar_wait(sd_full, n & 1, a.err));
      if (!ok) break;
      sm100::tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < BM; c0 += 64) {  // query rows c0 .. c0 + 63 of the tile
        float pv[64], dv[64];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float sv[32], dp[32];
          sm100::tmem_ld32(tmem + lane_off + C::S_COL + c0 + hh * 32, sv);
          sm100::tmem_ld32(tmem + lane_off + C::P_COL + c0 + hh * 32, dp);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int r = c0 + hh * 32 + c;
            int j = 0, slot = 0, g = 0;
            bool vis = key_ok && row_info(a, qt, r, j, slot, g) && stat[r] != -INFINITY;
            if (vis) vis = draft ? (r / a.RB == kr / a.bs) : key < (int)a.anchors[bi * a.nb + j];
            const float p = vis ? exp2f(sv[c] * a.scale_log2 - stat[r]) : 0.f;
            pv[hh * 32 + c] = p;
            dv[hh * 32 + c] = p * (dp[c] - stat[BM + r]);
          }
        }
        store_row64(sP, BK * 128, c0 / 64, kr, pv);
        store_row64(sD, BK * 128, c0 / 64, kr, dv);
      }
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(pd_full);
      // the next tile's MMAs write S / dP only after this tile's dK / dV MMAs (in order),
      // and sP / sD are rewritten only after its sd_full, which follows mm_done
      ++n;
    }
    if (ok && n > 0) ok = __all_sync(0xffffffff, sm100::mbar_wait(mm_done, (n - 1) & 1, a.err));
    if (ok) {
      sm100::tc_fence_after();
      const bool write = key_ok;
      const int64_t orow = draft ? (int64_t)a.b * a.S + (int64_t)bi * a.Td + kt * a.QB * a.bs + kr
                                 : (int64_t)bi * a.S + key;
      bf16* dkp = a.dk + orow * a.lddk + hk * D;
      bf16* dvp = a.dv + orow * a.lddv + hk * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float vk[32], vv[32];
        if (n > 0) {
          sm100::tmem_ld32(tmem + lane_off + C::K_COL + c, vk);
          sm100::tmem_ld32(tmem + lane_off + C::V_COL + c, vv);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) vk[i] = vv[i] = 0.f;
        }
        if (!write) continue;
        uint32_t pk[16], pv2[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          pk[i / 2] = pack2(vk[i] * a.scale, vk[i + 1] * a.scale);
          pv2[i / 2] = pack2(vv[i], vv[i + 1]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          reinterpret_cast<uint4*>(dkp + c)[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
          reinterpret_cast<uint4*>(dvp + c)[i] = make_uint4(pv2[4 * i], pv2[4 * i + 1], pv2[4 * i + 2], pv2[4 * i + 3]);
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

}  // namespace dattn

// ---------------------------------------------------------------------------- host
static dattn::Args dattn_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& anchors,
                              const at::Tensor& keep, int S, int bs) {
  dattn::Args a{};
  a.b = q.size(0);
  a.Td = q.size(1);
  a.Hq = q.size(2);
  a.Hk = k.size(1);
  a.G = a.Hq / a.Hk;
  a.nb = anchors.size(1);
  a.bs = bs;
  a.S = S;
  a.RB = (a.G * bs + 7) / 8 * 8;
  // blocks per query tile: the rows fit 128 and the blocks' draft keys fit one 64-key tile
  a.QB = std::min(dattn::BM / a.RB, dattn::BN / bs);
  a.nqt = (a.nb + a.QB - 1) / a.QB;
  a.anchors = anchors.data_ptr<int64_t>();
  a.keep = keep.data_ptr<bool>();
  a.scale = 1.f / std::sqrt((float)q.size(3));
  a.scale_log2 = a.scale * 1.4426950408889634f;
  a.err = device_error_flag();
  return a;
}

// Whether the tensor-core kernels take this shape (else attention.cu runs).
bool dattn_supported(const at::Tensor& q, const at::Tensor& k, int64_t bs) {
  const int D = q.size(3), G = q.size(2) / k.size(1);
  const int RB = (G * (int)bs + 7) / 8 * 8;
  return (D == 64 || D == 128) && RB <= dattn::BM && G * bs <= 256 && k.stride(1) == D &&
         reinterpret_cast<uintptr_t>(k.data_ptr()) % 16 == 0;
}

static CUtensorMap kv_map(const at::Tensor& t, int D, int box_rows) {
  return make_tmap_bf16_3d(t.data_ptr(), D, t.size(1), t.size(0), t.stride(1), t.stride(0), 64, 1, box_rows);
}

static CUtensorMap q_map(const at::Tensor& t, const dattn::Args& a, int D) {
  // [b * Td tokens][Hq heads][D]; box = 64 channels x G heads x bs tokens
  return make_tmap_bf16_3d(t.data_ptr(), D, a.Hq, (int64_t)a.b * a.Td, D, (int64_t)a.Hq * D, 64, a.G, a.bs);
}

template <int D>
static void dattn_fwd_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, dattn::Args& a) {
  using C = dattn::Fwd<D>;
  CUtensorMap tq = q_map(q, a, D), tk = kv_map(k, D, dattn::BN), tv = kv_map(v, D, dattn::BN);
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(dattn::dattn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
  });
  dattn::dattn_fwd_kernel<D><<<dim3(a.nqt, a.Hk, a.b), 192, C::SMEM, stream()>>>(tq, tk, tv, a);
  NS_CUDA(cudaGetLastError());
}

void dattn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs,
               at::Tensor out, at::Tensor lse) {
  NS_CHECK(q.is_contiguous() && out.is_contiguous() && lse.is_contiguous(), "dattn: q / out / lse contiguous");
  dattn::Args a = dattn_args(q, k, anchors, keep, (int)S, (int)bs);
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  if (q.size(3) == 64) dattn_fwd_launch<64>(q, k, v, a);
  else dattn_fwd_launch<128>(q, k, v, a);
}

template <int D>
static void dattn_bwd_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
                             dattn::Args& a) {
  CUtensorMap tq = q_map(q, a, D), tdo = q_map(dout, a, D);
  CUtensorMap tk = kv_map(k, D, dattn::BN), tv = kv_map(v, D, dattn::BN);
  CUtensorMap tk2 = kv_map(k, D, dattn::BK), tv2 = kv_map(v, D, dattn::BK);
  static std::atomic<unsigned long long> attr{0};
  once_per_device(attr, [&] {
    NS_CUDA(cudaFuncSetAttribute(dattn::dattn_dq_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 dattn::Dq<D>::SMEM));
    NS_CUDA(cudaFuncSetAttribute(dattn::dattn_dkv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 dattn::Dkv<D>::SMEM));
  });
  dattn::dattn_dq_kernel<D><<<dim3(a.nqt, a.Hk, a.b), 192, dattn::Dq<D>::SMEM, stream()>>>(tq, tdo, tk, tv, a);
  NS_CUDA(cudaGetLastError());
  const int nkc = (a.S + dattn::BK - 1) / dattn::BK;
  dattn::dattn_dkv_kernel<D><<<dim3(nkc + a.nqt, a.Hk, a.b), 192, dattn::Dkv<D>::SMEM, stream()>>>(tq, tdo, tk2, tv2,
                                                                                                  a);
  NS_CUDA(cudaGetLastError());
}

void dattn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, at::Tensor lse,
               at::Tensor anchors, at::Tensor keep, int64_t S, int64_t bs, at::Tensor dq, at::Tensor dk,
               at::Tensor dv) {
  NS_CHECK(dout.is_contiguous() && out.is_contiguous() && dq.is_contiguous() && q.is_contiguous(),
           "dattn: dout / out / dq / q contiguous");
  NS_CHECK(dk.stride(2) == 1 && dv.stride(2) == 1 && dk.stride(1) == dk.size(2) && dv.stride(1) == dv.size(2),
           "dattn: dk / dv rows with dense heads");
  dattn::Args a = dattn_args(q, k, anchors, keep, (int)S, (int)bs);
  a.o = reinterpret_cast<const bf16*>(out.data_ptr());
  a.dout = reinterpret_cast<const bf16*>(dout.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.dq = reinterpret_cast<bf16*>(dq.data_ptr());
  a.dk = reinterpret_cast<bf16*>(dk.data_ptr());
  a.dv = reinterpret_cast<bf16*>(dv.data_ptr());
  a.lddk = dk.stride(0);
  a.lddv = dv.stride(0);
  if (q.size(3) == 64) dattn_bwd_launch<64>(q, k, v, dout, a);
  else dattn_bwd_launch<128>(q, k, v, dout, a);
}

}  // namespace ns
