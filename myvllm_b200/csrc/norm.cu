// RMS norms, HBM-bound, one warp per row held in registers as 16-byte vectors (D <= 2048):
//   gated:  out = x * rsqrt(mean(x^2) + eps) * weight * silu(gate)     (RMSNormGated,
//           m/layers/norm.py:50-58, the GDN output norm)
//   plain:  s = x (+ residual);  out = s * rsqrt(mean(s^2) + eps) * (weight [+ 1])
//           (RMSNorm with optional zero-centred gamma and fused residual add, norm.py:6-41;
//           the summed s is written back to `residual` when one is given)
// fp32 math; the reference runs these through torch.compile.
#include "common.cuh"

namespace mvb {
namespace {

template <typename T, typename TW, int NV>  // NV = 16-byte vectors per lane
__global__ void __launch_bounds__(256) rmsnorm_gated_kernel(const T* x, int64_t sx, const T* gate, int64_t sg,
                                                            const TW* w, T* out, int64_t so, int64_t rows, int d,
                                                            float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float xv[NV][8], gv[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      unpack8<T>(*reinterpret_cast<const uint4*>(x + row * sx + c), xv[i]);
      unpack8<T>(*reinterpret_cast<const uint4*>(gate + row * sg + c), gv[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += xv[i][j] * xv[i][j];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)d + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = xv[i][j] * r * to_f32<TW>(w[c + j]) * silu(gv[i][j]);
      *reinterpret_cast<uint4*>(out + row * so + c) = pack8<T>(y);
    }
  }
}

template <typename T, typename TW>
void launch(const mvb_tensor* x, const mvb_tensor* g, const mvb_tensor* w, mvb_tensor* o, float eps,
            cudaStream_t st) {
  const int64_t rows = x->shape[0];
  const int d = (int)x->shape[1];
  const int nv = (d / 8 + 31) / 32;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  auto xs = static_cast<const T*>(x->data);
  auto gs = static_cast<const T*>(g->data);
  auto ws = static_cast<const TW*>(w->data);
  auto os = static_cast<T*>(o->data);
#define MVB_NORM_CASE(N) \
  case N: rmsnorm_gated_kernel<T, TW, N><<<blocks, 256, 0, st>>>(xs, x->stride[0], gs, g->stride[0], ws, os, o->stride[0], rows, d, eps); break;
  switch (nv) {
    MVB_NORM_CASE(1)
    MVB_NORM_CASE(2)
    MVB_NORM_CASE(3)
    MVB_NORM_CASE(4)
  }
#undef MVB_NORM_CASE
}

template <typename T, typename TW, int NV>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* x, int64_t sx, T* res, int64_t sr, const TW* w,
                                                      T* out, int64_t so, int64_t rows, int d, float eps,
                                                      float w_offset) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float xv[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      unpack8<T>(*reinterpret_cast<const uint4*>(x + row * sx + c), xv[i]);
      if (res != nullptr) {
        float r[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(res + row * sr + c), r);
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[i][j] += r[j];
        *reinterpret_cast<uint4*>(res + row * sr + c) = pack8<T>(xv[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += xv[i][j] * xv[i][j];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)d + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = xv[i][j] * r * (to_f32<TW>(w[c + j]) + w_offset);
      *reinterpret_cast<uint4*>(out + row * so + c) = pack8<T>(y);
    }
  }
}

template <typename T, typename TW>
void launch_plain(const mvb_tensor* x, mvb_tensor* res, const mvb_tensor* w, mvb_tensor* o, float eps, float w_off,
                  cudaStream_t st) {
  const int64_t rows = x->shape[0];
  const int d = (int)x->shape[1];
  const int nv = (d / 8 + 31) / 32;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  auto xs = static_cast<const T*>(x->data);
  auto rs = res ? static_cast<T*>(res->data) : nullptr;
  const int64_t sr = res ? res->stride[0] : 0;
  auto ws = static_cast<const TW*>(w->data);
  auto os = static_cast<T*>(o->data);
#define MVB_NORM_CASE(N) \
  case N: rmsnorm_kernel<T, TW, N><<<blocks, 256, 0, st>>>(xs, x->stride[0], rs, sr, ws, os, o->stride[0], rows, d, eps, w_off); break;
  switch (nv) {
    MVB_NORM_CASE(1)
    MVB_NORM_CASE(2)
    MVB_NORM_CASE(4)
    MVB_NORM_CASE(8)
  }
#undef MVB_NORM_CASE
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_rmsnorm_gated(const mvb_tensor* x, const mvb_tensor* gate, const mvb_tensor* weight, float eps,
                                 mvb_tensor* out, void* stream) {
  using namespace mvb;
  const char* op = "rmsnorm_gated";
  int rc;
  if ((rc = check_tensor(x, op, "x", 2)) || (rc = check_tensor(gate, op, "gate", 2)) ||
      (rc = check_tensor(weight, op, "weight", 1)) || (rc = check_tensor(out, op, "out", 2)))
    return rc;
  const int64_t n = x->shape[0], d = x->shape[1];
  MVB_CHECK_ARG(gate->shape[0] == n && gate->shape[1] == d && out->shape[0] == n && out->shape[1] == d &&
                    weight->shape[0] == d,
                "%s: x/gate/out must be [N, D] and weight [D]", op);
  MVB_CHECK_ARG(x->dtype == gate->dtype && x->dtype == out->dtype && (x->dtype == MVB_BF16 || x->dtype == MVB_F16),
                "%s: x/gate/out must share a 16-bit float dtype", op);
  MVB_CHECK_ARG(weight->dtype == MVB_F32 || weight->dtype == x->dtype, "%s: weight dtype", op);
  MVB_CHECK_SUPPORTED(d % 8 == 0 && d <= 1024 && x->stride[1] == 1 && gate->stride[1] == 1 && out->stride[1] == 1 &&
                          weight->stride[0] == 1 && x->stride[0] % 8 == 0 && gate->stride[0] % 8 == 0 &&
                          out->stride[0] % 8 == 0 && aligned16(x->data) && aligned16(gate->data) &&
                          aligned16(out->data),
                      "%s: needs D %% 8 == 0, D <= 1024, contiguous 16-byte aligned rows", op);
  if (n == 0) return MVB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool w32 = weight->dtype == MVB_F32;
  if (x->dtype == MVB_BF16) {
    if (w32) launch<__nv_bfloat16, float>(x, gate, weight, out, eps, st);
    else launch<__nv_bfloat16, __nv_bfloat16>(x, gate, weight, out, eps, st);
  } else {
    if (w32) launch<__half, float>(x, gate, weight, out, eps, st);
    else launch<__half, __half>(x, gate, weight, out, eps, st);
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}

extern "C" int mvb_rmsnorm(const mvb_tensor* x, mvb_tensor* residual, const mvb_tensor* weight, float eps,
                           int zero_centered_gamma, mvb_tensor* out, void* stream) {
  using namespace mvb;
  const char* op = "rmsnorm";
  int rc;
  if ((rc = check_tensor(x, op, "x", 2)) || (rc = check_tensor(weight, op, "weight", 1)) ||
      (rc = check_tensor(out, op, "out", 2)) || (residual && (rc = check_tensor(residual, op, "residual", 2))))
    return rc;
  const int64_t n = x->shape[0], d = x->shape[1];
  MVB_CHECK_ARG(out->shape[0] == n && out->shape[1] == d && weight->shape[0] == d &&
                    (!residual || (residual->shape[0] == n && residual->shape[1] == d)),
                "%s: x/out/residual must be [N, D] and weight [D]", op);
  MVB_CHECK_ARG(x->dtype == out->dtype && (!residual || residual->dtype == x->dtype) &&
                    (x->dtype == MVB_BF16 || x->dtype == MVB_F16),
                "%s: x/out/residual must share a 16-bit float dtype", op);
  MVB_CHECK_ARG(weight->dtype == MVB_F32 || weight->dtype == x->dtype, "%s: weight dtype", op);
  const int nv = (int)((d / 8 + 31) / 32);
  MVB_CHECK_SUPPORTED(d % 8 == 0 && (nv == 1 || nv == 2 || nv == 4 || nv == 8) && x->stride[1] == 1 &&
                          out->stride[1] == 1 && weight->stride[0] == 1 && x->stride[0] % 8 == 0 &&
                          out->stride[0] % 8 == 0 && aligned16(x->data) && aligned16(out->data) &&
                          (!residual || (residual->stride[1] == 1 && residual->stride[0] % 8 == 0 &&
                                         aligned16(residual->data))),
                      "%s: needs D %% 8 == 0, D <= 2048, contiguous 16-byte aligned rows", op);
  if (n == 0) return MVB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float w_off = zero_centered_gamma ? 1.f : 0.f;
  const bool w32 = weight->dtype == MVB_F32;
  if (x->dtype == MVB_BF16) {
    if (w32) launch_plain<__nv_bfloat16, float>(x, residual, weight, out, eps, w_off, st);
    else launch_plain<__nv_bfloat16, __nv_bfloat16>(x, residual, weight, out, eps, w_off, st);
  } else {
    if (w32) launch_plain<__half, float>(x, residual, weight, out, eps, w_off, st);
    else launch_plain<__half, __half>(x, residual, weight, out, eps, w_off, st);
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}
