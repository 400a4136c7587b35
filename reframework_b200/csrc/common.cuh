// Shared helpers of the rf_moe CUDA library: status/error plumbing on the
// host, dtype conversion and the device error word on the device.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/rf_moe.h"

namespace rf {

// ---------------------------------------------------------------- host side
void set_error(const std::string &msg);
int fail(int status, const std::string &msg);
// Returns RF_OK, or RF_ERR_CUDA with the launch error recorded.
int check_launch(const char *what);
int num_sms();              // SM count of the current device (cached per device)
size_t dtype_size(int dtype);
bool valid_dtype(int dtype);

// Each translation unit owns a device error word (set by its kernels when they
// detect bad input or give up on a bounded wait).  The host reads and clears
// all of them through the registry below (rf_moe_device_status).
typedef int (*ErrorWordReader)();
struct ErrorWordRegistrar {
  explicit ErrorWordRegistrar(ErrorWordReader fn);
};
int read_clear_all_error_words(int *code);

// -------------------------------------------------------------- device side
// Work order of the peer push kernels: item t of n goes to position
// (t * stride + offset) mod n, a permutation when stride is prime to n.
// Consecutive warps then copy rows for all destinations at once (send order
// is destination-major, so the plain order would have every rank write to the
// same few ranks first), and the per-rank offset staggers the ranks.
__device__ __forceinline__ int64_t scatter_stride(int64_t n) {
  const int64_t primes[3] = {1009, 1013, 1019};
  for (int i = 0; i < 3; ++i)
    if (n % primes[i] != 0) return primes[i];
  return 1;
}
__device__ __forceinline__ int64_t scatter_pos(int64_t t, int64_t n, int64_t stride, int64_t offset) {
  return (t * stride + offset) % n;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

template <typename T> struct Cvt;
template <> struct Cvt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// Unpack 16 bytes holding 8 (16-bit types) or 4 (fp32) elements into floats.
template <typename T> __device__ __forceinline__ int unpack16(const uint4 &v, float *f);
template <> __device__ __forceinline__ int unpack16<float>(const uint4 &v, float *f) {
  f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  return 4;
}
template <> __device__ __forceinline__ int unpack16<__nv_bfloat16>(const uint4 &v, float *f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
  return 8;
}
template <> __device__ __forceinline__ int unpack16<__half>(const uint4 &v, float *f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
    float2 p = __half22float2(h);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
  return 8;
}

// Pack two floats into one 32-bit word of the 16-bit type (round to nearest even).
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

// Gated activations of reframework/layers/activation.py, in fp32, with the
// activation fixed at compile time (the GEMM epilogues are instantiated per
// activation: no per-element branch, small code).  SiLU uses the fast
// division (x * approximate reciprocal, within 2 ulp of fp32): the result is
// rounded to the 16-bit storage type right after, where that error is ~2^-16
// of one unit in the last place.
template <int ACT>
__device__ __forceinline__ float act_gate_t(float g) {
  if constexpr (ACT == RF_ACT_SILU) {
    return __fdividef(g, 1.0f + __expf(-g));
  } else if constexpr (ACT == RF_ACT_GELU) {
    return 0.5f * g * (1.0f + erff(g * 0.70710678118654752f));
  } else {
    // tanh approximation: 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3)))
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    return 0.5f * g * (1.0f + tanhf(k0 * (g + k1 * g * g * g)));
  }
}

__device__ __forceinline__ float act_gate(int act, float g) {
  if (act == RF_ACT_SILU) return act_gate_t<RF_ACT_SILU>(g);
  if (act == RF_ACT_GELU) return act_gate_t<RF_ACT_GELU>(g);
  return act_gate_t<RF_ACT_GELU_TANH>(g);
}

// The gated activation in IEEE fp32 (reframework/layers/activation.py:15-46
// on fp32 tensors): every operation correctly rounded, CUDA's expf / erff /
// tanhf for the transcendental parts.  Used by the int8 expert split.
__device__ __forceinline__ float act_ieee(int act, float g) {
  if (act == RF_ACT_SILU) return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  if (act == RF_ACT_GELU)
    return __fmul_rn(__fmul_rn(g, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn(g, 0.70710678118654752f))));
  const float cube = __fmul_rn(__fmul_rn(g, g), g);
  const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(g, __fmul_rn(0.044715f, cube)));
  return __fmul_rn(__fmul_rn(g, 0.5f), __fadd_rn(1.0f, tanhf(inner)));
}

// Round an fp32 value to the storage type T and back (identity for fp32).
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  if constexpr (sizeof(T) == 4) return v;
  else return Cvt<T>::to_f(Cvt<T>::from_f(v));
}

// One element of the gated activation with the rounding points of the
// reference for a 16-bit layer: the gate|up GEMM output is stored in T
// (fused.py:81), act() runs on it and rounds to T, and the product of the two
// T tensors rounds to T (activation.py:20-21).  The caller's final store
// performs that last rounding.  For fp32 every rounding is the identity.
template <typename T, int ACT>
__device__ __forceinline__ float gated_elem_t(float g, float u) {
  const float gt = round_to<T>(g);
  const float ut = round_to<T>(u);
  return round_to<T>(act_gate_t<ACT>(gt)) * ut;
}

template <typename T>
__device__ __forceinline__ float gated_elem(int act, float g, float u) {
  const float gt = round_to<T>(g);
  const float ut = round_to<T>(u);
  return round_to<T>(act_gate(act, gt)) * ut;
}

}  // namespace rf

// Defines this translation unit's device error word, the device helper
// rf_report(code) that sets it (first error wins), and registers its reader.
#define RF_DEVICE_ERROR_WORD()                                                        \
  static __device__ int rf_tu_error_word;                                             \
  [[maybe_unused]] static __device__ __forceinline__ void rf_report(int code) {       \
    atomicCAS(&rf_tu_error_word, 0, code);                                            \
  }                                                                                   \
  static int rf_tu_read_clear() {                                                     \
    int v = 0, z = 0;                                                                 \
    if (cudaMemcpyFromSymbol(&v, rf_tu_error_word, sizeof(int)) != cudaSuccess)       \
      return -1;                                                                      \
    if (cudaMemcpyToSymbol(rf_tu_error_word, &z, sizeof(int)) != cudaSuccess)         \
      return -1;                                                                      \
    return v;                                                                         \
  }                                                                                   \
  static ::rf::ErrorWordRegistrar rf_tu_registrar(&rf_tu_read_clear)

#define RF_CHECK_ARG(cond, msg)                                   \
  do {                                                            \
    if (!(cond)) return ::rf::fail(RF_ERR_ARG, std::string(msg)); \
  } while (0)
