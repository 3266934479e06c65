// Shared helpers for the myvllm_b200 kernels: status handling, tensor-descriptor
// checks, dtype conversion and small PTX wrappers.  sm_100a only.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/myvllm_b200.h"

namespace mvb {

// ---------------------------------------------------------------- status ----
void set_error(const char* fmt, ...);

struct Status {
  int code;
};

#define MVB_FAIL(code, ...)        \
  do {                             \
    ::mvb::set_error(__VA_ARGS__); \
    return (code);                 \
  } while (0)

#define MVB_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) MVB_FAIL(MVB_ERR_ARG, __VA_ARGS__);               \
  } while (0)

#define MVB_CHECK_SUPPORTED(cond, ...)                             \
  do {                                                             \
    if (!(cond)) MVB_FAIL(MVB_ERR_UNSUPPORTED, __VA_ARGS__);       \
  } while (0)

#define MVB_CHECK_LAUNCH(opname)                                                         \
  do {                                                                                   \
    cudaError_t e_ = cudaGetLastError();                                                 \
    if (e_ != cudaSuccess) MVB_FAIL(MVB_ERR_CUDA, "%s: launch failed: %s", opname,       \
                                    cudaGetErrorString(e_));                             \
  } while (0)

// ------------------------------------------------------------ descriptors ----
inline int64_t numel(const mvb_tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

inline int dtype_size(int dt) { return dt == MVB_F32 || dt == MVB_I32 ? 4 : 2; }

inline bool is_float_dtype(int dt) { return dt == MVB_F32 || dt == MVB_BF16 || dt == MVB_F16; }

// Checks ndim, non-negative shape and a non-null pointer when numel > 0.
int check_tensor(const mvb_tensor* t, const char* op, const char* name, int ndim);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device): the
// attribute belongs to the device context, so a process driving several GPUs needs it on
// each.  `mask` is a per-kernel bit set of devices already configured.
template <typename F>
inline void ensure_smem_attr(F* func, int bytes, unsigned long long& mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(mask & bit)) {
    cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    mask |= bit;
  }
}

// Which kernel family the last call of an op ran (mvb_last_path), per host thread.
// `reason` says why a fallback was taken (NULL/empty for the main path).
void set_path(int op, int path, const char* reason);

// Host readers of the per-translation-unit device error words (see tcgen05.cuh).
using StatusReader = int (*)(int*);
void register_status_reader(StatusReader f);

// ------------------------------------------------------------- dtype math ----
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// 8 x 16-bit values <-> 8 floats through one 16-byte access.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32<T>(h[i]);
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(f[i]);
  return u;
}

// Optional raw-gate inputs of the gated delta rule: with alog set, the kernels read the
// layer's projections a, b where they would read g, beta and form (as the layer does,
// m/layers/linear_attention.py:89-90)
//   g    = -exp(A_log[h]) * softplus(a + dt_bias[h])    fp32, softplus threshold 20 as torch
//   beta = sigmoid(b)                                    rounded to b's dtype, as torch does
struct GateDev {
  const void* alog = nullptr;
  const void* dtb = nullptr;
  int alog_dt = 0, dtb_dt = 0;
};

// RMSNormGated applied to a GDN output (m/layers/norm.py:44-58): out = o rsqrt(mean(o^2) +
// eps) w silu(z) over the V axis; z [T, Hv, V] (strides z_t, z_h, unit last stride), w [V].
struct NormDev {
  const void* z = nullptr;  // null: no norm
  int64_t z_t = 0, z_h = 0;
  const void* w = nullptr;
  int w_dt = 0;
  float eps = 0.f;
};

__device__ __forceinline__ float load_scalar(const void* p, int64_t i, int dtype) {
  if (dtype == MVB_F32) return static_cast<const float*>(p)[i];
  if (dtype == MVB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ float raw_gate_g(const GateDev& gd, float a, int h) {
  const float x = a + load_scalar(gd.dtb, h, gd.dtb_dt);
  const float sp = x > 20.f ? x : log1pf(expf(x));
  return -expf(load_scalar(gd.alog, h, gd.alog_dt)) * sp;
}
__device__ __forceinline__ float raw_gate_beta(float b, int dtype) {
  const float s = 1.f / (1.f + expf(-b));
  if (dtype == MVB_BF16) return __bfloat162float(__float2bfloat16_rn(s));
  if (dtype == MVB_F16) return __half2float(__float2half_rn(s));
  return s;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// Packs two floats into a bf16x2 / f16x2 register (lo in the low half).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------------- PTX: mma / copies ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred = true) {
  const int n = pred ? 16 : 0;  // src-size 0 zero-fills the 16 bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                            uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                                  uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

// D (16x8 f32) += A (16x16, row) * B (16x8, col); bf16 or f16 operands.
template <typename T>
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, const uint32_t* b);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace mvb
