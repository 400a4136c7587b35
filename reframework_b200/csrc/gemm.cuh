// Internal interface between the grouped-GEMM entry points (gemm_tc.cu) and
// the CUDA-core implementation (gemm_simt.cu).
#pragma once

#include "common.cuh"

namespace rf {

struct GroupedGemmArgs {
  const void *a;                 // [rows_capacity, Kdim]
  const void *w;                 // gated: [S, 2*N, Kdim]; down: [S, N, Kdim]
  void *out;                     // [rows_capacity, N]
  const int32_t *offsets;        // [E+1]
  const int32_t *counts;         // [E]
  const int32_t *slot;           // [E] or NULL
  const int32_t *groups;         // [G] or NULL (all experts)
  int n_groups;                  // G
  int E;
  int num_slots;
  int64_t rows_capacity;
  int Kdim;                      // reduction length (H for gated, I for down)
  int N;                         // output columns (I for gated, H for down)
  int dtype;
  int act;
  // gather mode (gated, tensor cores only): `a` is [a_rows, Kdim] token rows
  // and permuted row r reads a[gather_src[r] / gather_div] (-1: pad row)
  const int32_t *gather_src = nullptr;
  int gather_div = 1;
  int64_t a_rows = 0;
};

int launch_simt_grouped_gemm(const GroupedGemmArgs &g, bool gated, cudaStream_t st);

// Dense out[M, ld_out] (fp32) = a[M, K] . w[N, K]^T on the tensor cores
// (gemm_tc.cu); -1 when the shape or dtype is not handled there.
int tc_dense_f32(const void *a, const void *w, float *out, int64_t M, int64_t N, int64_t Kdim,
                 int64_t ld_out, int dtype, cudaStream_t st);

}  // namespace rf
