// Internal interface between the grouped-GEMM entry points (gemm_tc.cu) and
// the CUDA-core implementation (gemm_simt.cu).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace rf {

constexpr int REMOTE_MAX_RANKS = 64;

// Down GEMM with the expert-parallel return exchange in its epilogue: output
// row k of local slot j came from source rank s = the last s with
// cj[j][s] <= k, and is stored at row ps[s][j] + (k - cj[j][s]) of rank s's
// return buffer dst[s] (a peer pointer) instead of locally.  When every CTA
// is done, the last one fences at system scope and raises flag[d] = epoch in
// every rank d (done: a zeroed block counter of this rank).
struct RemoteOut {
  const int64_t *cj;  // [S][R+1]
  const int64_t *ps;  // [R][S]
  int R, S;
  int32_t epoch;
  uint32_t *done;
  void *dst[REMOTE_MAX_RANKS];
  int32_t *flag[REMOTE_MAX_RANKS];
};

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
  // down GEMM only: store rows into the peers' return buffers (slot / groups
  // must be NULL, so group j is local slot j)
  const RemoteOut *remote = nullptr;
  // down GEMM only: out[r, n] = round(addend[r, n] + round(acc)) in the layer
  // dtype (addend has out's layout; it may be out itself)
  const void *addend = nullptr;
};

int launch_simt_grouped_gemm(const GroupedGemmArgs &g, bool gated, cudaStream_t st);

// A 16-bit tiled tensor map with the 128-byte swizzle (gemm_tc.cu).
bool tma_encode(CUtensorMap *m, int dtype, int rank, const void *base, const cuuint64_t *dims,
                const cuuint64_t *strides, const cuuint32_t *box);
// The GEMM implementation chosen by rf_moe_set_gemm_impl (0 = automatic).
int gemm_impl();

// The expert split's int8 grouped GEMMs on the tensor cores (gemm_tc.cu,
// tcgen05 kind::i8); -1 when the shape is not handled there (the caller runs
// its CUDA-core kernel), else a status.
int tc_int8_grouped_gemm(const int8_t *a, const int8_t *w, const int32_t *offsets, const int32_t *counts,
                         const int32_t *groups, const int32_t *slot, int n_groups, int E, int num_slots,
                         int64_t rows_capacity, int64_t Kdim, int64_t N, const float *a_scales,
                         const float *w_scales, int64_t w_stride, bool gated, int act, float *out, float *amax,
                         const float *row_w, const int32_t *src_slot, cudaStream_t st);

// The grouped GEMM of `g` on CTA pairs (gemm_pair.cu): weight rows on the
// MMA's M side (256 per pair), token rows on N in steps of 16.  -1 when the
// shape, dtype or device does not suit it, else a status.
int launch_pair_grouped_gemm(const GroupedGemmArgs &g, bool gated, cudaStream_t st);

// Dense out[M, ld_out] (fp32) = a[M, K] . w[N, K]^T on the tensor cores
// (gemm_tc.cu); -1 when the shape or dtype is not handled there.  With
// slice_k > 0 (a multiple of 64) K is cut into ceil(K / slice_k) fixed slices
// and slice j's sums go to out + j * M * ld_out (the caller adds them).
int tc_dense_f32(const void *a, const void *w, float *out, int64_t M, int64_t N, int64_t Kdim,
                 int64_t ld_out, int dtype, cudaStream_t st, int64_t slice_k = 0);

// The down GEMM of `g` (g.remote set) on the tensor cores, launched even when
// no row is routed (the flags must rise); -1 when the shape or dtype is not
// handled there, else a status.
int tc_down_remote(const GroupedGemmArgs &g, cudaStream_t st);

}  // namespace rf
