// Internal GEMM entry point shared by the extension's .cu files.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace ns {

// A row-major matrix of `rows` x `cols` with row stride `ld` (elements).
// mn_major = false: the matrix is [M or N, K]; true: it is [K, M or N].
struct Operand {
  const void* ptr;
  int64_t rows, cols, ld;
  bool mn_major;
};

// Epilogue of D[m, n]: exactly one of `out` (bf16) / `out_f32` is set. Element
// (m, n) lives at m * sm + n * sn. bf16: out = bf16(res + bf16(D)) (+ old out when
// accumulate). fp32: out_f32 = D (+ old value when accumulate).
//
// Optional squared-norm side output (plain bf16 outputs only, no split-K): with
// `npart` set, every CTA writes npart[cta] = sum over the elements it stored of
// bf16(out * factor)^2, factor = *nfac; the caller sums the partials in order.
struct Epilogue {
  __nv_bfloat16* out;
  float* out_f32;
  int64_t sm, sn;
  const __nv_bfloat16* res;
  int64_t rsm, rsn;
  bool accumulate;
  const float* nfac = nullptr;
  float* npart = nullptr;
};

// D[M, N] = sum_k A[m, k] B[n, k] on tcgen05; force_splits > 0 fixes the split-K count.
// Returns the number of CTAs launched (the norm partials written when requested).
int gemm_launch(const Operand& A, const Operand& B, int M, int N, int K, const Epilogue& e,
                int force_splits = 0);

}  // namespace ns
