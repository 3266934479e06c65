// RMS norms, HBM-bound, rows held in registers as 16-byte vectors (D <= 2048; a warp per row,
// a block per row from D = 1024):
//   gated:  out = x * rsqrt(mean(x^2) + eps) * weight * silu(gate)     (RMSNormGated,
//           m/layers/norm.py:50-58, the GDN output norm)
//   plain:  s = x (+ residual);  out = s * rsqrt(mean(s^2) + eps) * (weight [+ 1])
//           (RMSNorm with optional zero-centred gamma and fused residual add, norm.py:6-41;
//           the summed s is written back to `residual` when one is given)
// fp32 math; the reference runs these through torch.compile.
#include "common.cuh"

namespace mvb {
namespace {

// Row r of a [T, H, D] tensor (H = 1 for 2-D) sits at (r / H) * s0 + (r % H) * s1.
struct Rows3 {
  int64_t s0, s1;
  __device__ __forceinline__ int64_t at(int64_t r, int h) const { return (r / h) * s0 + (r % h) * s1; }
};

template <typename T, typename TW, int NV>  // NV = 16-byte vectors per lane
__global__ void __launch_bounds__(256) rmsnorm_gated_kernel(const T* x, Rows3 rx, const T* gate, Rows3 rg,
                                                            const TW* w, T* out, Rows3 ro, int64_t rows, int heads,
                                                            int d, float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t ox = rx.at(row, heads), og = rg.at(row, heads), oo = ro.at(row, heads);
  float xv[NV][8], gv[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      unpack8<T>(*reinterpret_cast<const uint4*>(x + ox + c), xv[i]);
      unpack8<T>(*reinterpret_cast<const uint4*>(gate + og + c), gv[i]);
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
      *reinterpret_cast<uint4*>(out + oo + c) = pack8<T>(y);
    }
  }
}

Rows3 rows3(const mvb_tensor* t) {
  return t->ndim == 3 ? Rows3{t->stride[0], t->stride[1]} : Rows3{t->stride[0], 0};
}

template <typename T, typename TW>
void launch(const mvb_tensor* x, const mvb_tensor* g, const mvb_tensor* w, mvb_tensor* o, float eps,
            cudaStream_t st) {
  const int heads = x->ndim == 3 ? (int)x->shape[1] : 1;
  const int64_t rows = x->shape[0] * heads;
  const int d = (int)x->shape[x->ndim - 1];
  const int nv = (d / 8 + 31) / 32;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  auto xs = static_cast<const T*>(x->data);
  auto gs = static_cast<const T*>(g->data);
  auto ws = static_cast<const TW*>(w->data);
  auto os = static_cast<T*>(o->data);
#define MVB_NORM_CASE(N) \
  case N: rmsnorm_gated_kernel<T, TW, N><<<blocks, 256, 0, st>>>(xs, rows3(x), gs, rows3(g), ws, os, rows3(o), rows, heads, d, eps); break;
  switch (nv) {
    MVB_NORM_CASE(1)
    MVB_NORM_CASE(2)
    MVB_NORM_CASE(3)
    MVB_NORM_CASE(4)
  }
#undef MVB_NORM_CASE
}

template <typename T, typename TW, int NV>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* x, Rows3 rx, T* res, Rows3 rr, const TW* w, T* out,
                                                      Rows3 ro, int64_t rows, int heads, int d, float eps,
                                                      float w_offset) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t ox = rx.at(row, heads), orr = rr.at(row, heads), oo = ro.at(row, heads);
  float xv[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      unpack8<T>(*reinterpret_cast<const uint4*>(x + ox + c), xv[i]);
      if (res != nullptr) {
        float r[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(res + orr + c), r);
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[i][j] += r[j];
        *reinterpret_cast<uint4*>(res + orr + c) = pack8<T>(xv[i]);
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
      *reinterpret_cast<uint4*>(out + oo + c) = pack8<T>(y);
    }
  }
}

// The plain norm for wide rows (D >= 1024, e.g. the hidden states of a decode batch): one
// 256-thread block per row, NV 16-byte vectors per thread, the sum of squares reduced across
// the block's warps through shared memory.  A decode batch has few rows, so a warp per row
// would leave most SMs idle with each warp's loads in series.
template <typename T, typename TW, int NV>
__global__ void __launch_bounds__(256) rmsnorm_wide_kernel(const T* x, Rows3 rx, T* res, Rows3 rr, const TW* w,
                                                           T* out, Rows3 ro, int heads, int d, float eps,
                                                           float w_offset) {
  __shared__ float s_part[8];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t ox = rx.at(row, heads), orr = rr.at(row, heads), oo = ro.at(row, heads);
  float xv[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 256 + tid) * 8;
    if (c < d) {
      unpack8<T>(*reinterpret_cast<const uint4*>(x + ox + c), xv[i]);
      if (res != nullptr) {
        float r[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(res + orr + c), r);
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[i][j] += r[j];
        *reinterpret_cast<uint4*>(res + orr + c) = pack8<T>(xv[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += xv[i][j] * xv[i][j];
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) s_part[wid] = ss;
  __syncthreads();
  ss = lane < 8 ? s_part[lane] : 0.f;
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)d + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 256 + tid) * 8;
    if (c < d) {
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = xv[i][j] * r * (to_f32<TW>(w[c + j]) + w_offset);
      *reinterpret_cast<uint4*>(out + oo + c) = pack8<T>(y);
    }
  }
}

template <typename T, typename TW>
void launch_plain(const mvb_tensor* x, mvb_tensor* res, const mvb_tensor* w, mvb_tensor* o, float eps, float w_off,
                  cudaStream_t st) {
  const int heads = x->ndim == 3 ? (int)x->shape[1] : 1;
  const int64_t rows = x->shape[0] * heads;
  const int d = (int)x->shape[x->ndim - 1];
  const int nv = (d / 8 + 31) / 32;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  auto xs = static_cast<const T*>(x->data);
  auto rs = res ? static_cast<T*>(res->data) : nullptr;
  const Rows3 rr = res ? rows3(res) : Rows3{0, 0};
  auto ws = static_cast<const TW*>(w->data);
  auto os = static_cast<T*>(o->data);
  if (d >= 1024) {  // D <= 2048: one vector per thread of a block per row
    rmsnorm_wide_kernel<T, TW, 1><<<(unsigned)rows, 256, 0, st>>>(xs, rows3(x), rs, rr, ws, os, rows3(o), heads, d,
                                                                  eps, w_off);
    return;
  }
#define MVB_NORM_CASE(N) \
  case N: rmsnorm_kernel<T, TW, N><<<blocks, 256, 0, st>>>(xs, rows3(x), rs, rr, ws, os, rows3(o), rows, heads, d, eps, w_off); break;
  switch (nv) {
    MVB_NORM_CASE(1)
    MVB_NORM_CASE(2)
    MVB_NORM_CASE(4)
    MVB_NORM_CASE(8)
  }
#undef MVB_NORM_CASE
}

// RMSNorm of each [D] row (D <= 256: one 16-byte vector per lane), then the half-split
// rotary on its first rd dims: for c < rd/2, (y_c, y_{c+rd/2}) <- (y_c cos_c - y_{c+rd/2} sin_c,
// y_{c+rd/2} cos_c + y_c sin_c), cos/sin [T, rd/2] fp32 at the row's token.  The partner of
// lane l's dims is lane l ^ (rd/16) (rd/16 a power of two).  fp32 throughout, one rounding.
template <typename T, typename TW>
__global__ void __launch_bounds__(256) rmsnorm_rope_kernel(const T* x, Rows3 rx, const TW* w, T* out, Rows3 ro,
                                                           const float* cosp, const float* sinp, int64_t scs,
                                                           int64_t sss, int64_t rows, int heads, int d, int rd,
                                                           float eps, float w_offset) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // whole warps leave together (a warp is one row)
  const int c = lane * 8;
  const bool live = c < d;
  float y[8];
  float ss = 0.f;
  if (live) {
    unpack8<T>(*reinterpret_cast<const uint4*>(x + rx.at(row, heads) + c), y);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += y[j] * y[j];
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = 0.f;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)d + eps);
  if (live) {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] *= r * (to_f32<TW>(w[c + j]) + w_offset);
  }
  const int half = rd >> 1;
  float partner[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) partner[j] = __shfl_xor_sync(0xffffffffu, y[j], half >> 3);
  if (live && c < rd) {
    const int64_t t = row / heads;
    const int ci = c < half ? c : c - half;
    const float sgn = c < half ? -1.f : 1.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float cs = cosp[t * scs + ci + j], sn = sinp[t * sss + ci + j];
      y[j] = fmaf(sgn * partner[j], sn, y[j] * cs);
    }
  }
  if (live) *reinterpret_cast<uint4*>(out + ro.at(row, heads) + c) = pack8<T>(y);
}

template <typename T, typename TW>
void launch_rope(const mvb_tensor* x, const mvb_tensor* w, mvb_tensor* o, const mvb_tensor* cs, const mvb_tensor* sn,
                 float eps, float w_off, cudaStream_t st) {
  const int heads = (int)x->shape[1];
  const int64_t rows = x->shape[0] * heads;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  rmsnorm_rope_kernel<T, TW><<<blocks, 256, 0, st>>>(
      static_cast<const T*>(x->data), rows3(x), static_cast<const TW*>(w->data), static_cast<T*>(o->data), rows3(o),
      static_cast<const float*>(cs->data), static_cast<const float*>(sn->data), cs->stride[0], sn->stride[0], rows,
      heads, (int)x->shape[2], (int)(2 * cs->shape[1]), eps, w_off);
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_rmsnorm_rope(const mvb_tensor* x, const mvb_tensor* weight, float eps, int zero_centered_gamma,
                                const mvb_tensor* cos, const mvb_tensor* sin, mvb_tensor* out, void* stream) {
  using namespace mvb;
  const char* op = "rmsnorm_rope";
  int rc;
  if ((rc = check_tensor(x, op, "x", 3)) || (rc = check_tensor(weight, op, "weight", 1)) ||
      (rc = check_tensor(cos, op, "cos", 2)) || (rc = check_tensor(sin, op, "sin", 2)) ||
      (rc = check_tensor(out, op, "out", 3)))
    return rc;
  for (int i = 0; i < 3; ++i) MVB_CHECK_ARG(out->shape[i] == x->shape[i], "%s: x/out shapes differ", op);
  const int64_t d = x->shape[2], rd = 2 * cos->shape[1];
  MVB_CHECK_ARG(weight->shape[0] == d, "%s: weight must be [D]", op);
  MVB_CHECK_ARG(cos->shape[0] >= x->shape[0] && sin->shape[0] >= x->shape[0] && sin->shape[1] == cos->shape[1],
                "%s: cos/sin must be [T, rotary_dim / 2]", op);
  MVB_CHECK_ARG(x->dtype == out->dtype && (x->dtype == MVB_BF16 || x->dtype == MVB_F16),
                "%s: x/out must share a 16-bit float dtype", op);
  MVB_CHECK_ARG(weight->dtype == MVB_F32 || weight->dtype == x->dtype, "%s: weight dtype", op);
  MVB_CHECK_ARG(cos->dtype == MVB_F32 && sin->dtype == MVB_F32, "%s: cos/sin must be fp32", op);
  bool rows_ok = weight->stride[0] == 1 && cos->stride[1] == 1 && sin->stride[1] == 1;
  for (const mvb_tensor* t : {x, static_cast<const mvb_tensor*>(out)})
    rows_ok = rows_ok && t->stride[2] == 1 && t->stride[0] % 8 == 0 && t->stride[1] % 8 == 0 && aligned16(t->data);
  const bool pow2 = rd >= 16 && (rd & (rd - 1)) == 0;
  MVB_CHECK_SUPPORTED(d % 8 == 0 && d <= 256 && pow2 && rd <= d && rows_ok,
                      "%s: needs D %% 8 == 0, D <= 256, rotary dims a power of two in [16, D], "
                      "contiguous 16-byte aligned rows", op);
  if (x->shape[0] * x->shape[1] == 0) return MVB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float w_off = zero_centered_gamma ? 1.f : 0.f;
  const bool w32 = weight->dtype == MVB_F32;
  if (x->dtype == MVB_BF16) {
    if (w32) launch_rope<__nv_bfloat16, float>(x, weight, out, cos, sin, eps, w_off, st);
    else launch_rope<__nv_bfloat16, __nv_bfloat16>(x, weight, out, cos, sin, eps, w_off, st);
  } else {
    if (w32) launch_rope<__half, float>(x, weight, out, cos, sin, eps, w_off, st);
    else launch_rope<__half, __half>(x, weight, out, cos, sin, eps, w_off, st);
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}

extern "C" int mvb_rmsnorm_gated(const mvb_tensor* x, const mvb_tensor* gate, const mvb_tensor* weight, float eps,
                                 mvb_tensor* out, void* stream) {
  using namespace mvb;
  const char* op = "rmsnorm_gated";
  int rc;
  if ((rc = check_tensor(x, op, "x", -1)) || (rc = check_tensor(gate, op, "gate", -1)) ||
      (rc = check_tensor(weight, op, "weight", 1)) || (rc = check_tensor(out, op, "out", -1)))
    return rc;
  const int nd = x->ndim;
  MVB_CHECK_ARG((nd == 2 || nd == 3) && gate->ndim == nd && out->ndim == nd, "%s: x/gate/out must be 2-D or 3-D", op);
  for (int i = 0; i < nd; ++i)
    MVB_CHECK_ARG(gate->shape[i] == x->shape[i] && out->shape[i] == x->shape[i], "%s: x/gate/out shapes differ", op);
  const int64_t d = x->shape[nd - 1];
  const int64_t n = x->shape[0] * (nd == 3 ? x->shape[1] : 1);
  MVB_CHECK_ARG(weight->shape[0] == d, "%s: weight must be [D]", op);
  MVB_CHECK_ARG(x->dtype == gate->dtype && x->dtype == out->dtype && (x->dtype == MVB_BF16 || x->dtype == MVB_F16),
                "%s: x/gate/out must share a 16-bit float dtype", op);
  MVB_CHECK_ARG(weight->dtype == MVB_F32 || weight->dtype == x->dtype, "%s: weight dtype", op);
  bool rows_ok = true;
  for (const mvb_tensor* t : {x, gate, static_cast<const mvb_tensor*>(out)})
    rows_ok = rows_ok && t->stride[nd - 1] == 1 && t->stride[0] % 8 == 0 && (nd == 2 || t->stride[1] % 8 == 0) &&
              aligned16(t->data);
  MVB_CHECK_SUPPORTED(d % 8 == 0 && d <= 1024 && weight->stride[0] == 1 && rows_ok,
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
  if ((rc = check_tensor(x, op, "x", -1)) || (rc = check_tensor(weight, op, "weight", 1)) ||
      (rc = check_tensor(out, op, "out", -1)) || (residual && (rc = check_tensor(residual, op, "residual", -1))))
    return rc;
  const int nd = x->ndim;
  MVB_CHECK_ARG((nd == 2 || nd == 3) && out->ndim == nd && (!residual || residual->ndim == nd),
                "%s: x/out/residual must be 2-D or 3-D", op);
  for (int i = 0; i < nd; ++i)
    MVB_CHECK_ARG(out->shape[i] == x->shape[i] && (!residual || residual->shape[i] == x->shape[i]),
                  "%s: x/out/residual shapes differ", op);
  const int64_t d = x->shape[nd - 1];
  const int64_t n = x->shape[0] * (nd == 3 ? x->shape[1] : 1);
  MVB_CHECK_ARG(weight->shape[0] == d, "%s: weight must be [D]", op);
  MVB_CHECK_ARG(x->dtype == out->dtype && (!residual || residual->dtype == x->dtype) &&
                    (x->dtype == MVB_BF16 || x->dtype == MVB_F16),
                "%s: x/out/residual must share a 16-bit float dtype", op);
  MVB_CHECK_ARG(weight->dtype == MVB_F32 || weight->dtype == x->dtype, "%s: weight dtype", op);
  const int nv = (int)((d / 8 + 31) / 32);
  bool rows_ok = true;
  for (const mvb_tensor* t : {x, static_cast<const mvb_tensor*>(out), static_cast<const mvb_tensor*>(residual)})
    if (t) rows_ok = rows_ok && t->stride[nd - 1] == 1 && t->stride[0] % 8 == 0 && (nd == 2 || t->stride[1] % 8 == 0) &&
                     aligned16(t->data);
  MVB_CHECK_SUPPORTED(d % 8 == 0 && (nv == 1 || nv == 2 || nv == 4 || nv == 8) && weight->stride[0] == 1 && rows_ok,
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
