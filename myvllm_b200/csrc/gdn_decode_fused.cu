// The decode step of a Gated DeltaNet layer in one kernel (HBM-bound): what the layer's
// decode branch runs as four ops in the reference (m/layers/linear_attention.py:85-123):
//   qkv   = causal_conv1d_update(qkv_proj) (+ SiLU; conv state shifted in place)
//   q, k  = l2norm(q), l2norm(k)
//   g     = -exp(A_log) softplus(a + dt_bias),  beta = sigmoid(b)
//   o     = recurrent gated delta rule (fp32 state read and written in place)
//   out   = RMSNormGated(o, z) = o rsqrt(mean(o^2) + eps) w silu(z)      (m/layers/norm.py:44-58)
// The conv output never leaves the SM and the pre-norm o never reaches HBM: per step the
// kernel reads the projection row, the conv and recurrent states and z once, and writes
// the states and the normed output once.
//
// Grid (2, Hv, S): a CTA owns one half (64 columns) of the V axis of one (sequence, v-head),
// with the state streamed through registers exactly as gdn_recurrent.cu does it.  CTAs are
// grouped in clusters of (2, G) = both V halves of the G = Hv / Hk v-heads that share one
// k-head:
//   - every CTA recomputes the conv of its k-head's q and k channels (256 channels, 4 taps:
//     cheaper than exchanging them), and of its own 64 v channels;
//   - the v channels' conv state is written by the CTA that owns them; the q/k channels'
//     state, read by all 2G CTAs, is written by the cluster's first CTA after a cluster
//     barrier that follows every CTA's read;
//   - the RMS over the 128 V columns adds the two halves' partial sums through distributed
//     shared memory (in a fixed order, so both halves use the same bits).
// Numerics follow the unfused ops: the conv output is rounded to the activation dtype
// before the norms, o is rounded before RMSNormGated, all arithmetic is fp32.
#include "common.cuh"

namespace mvb {
namespace {

constexpr int kThreads = 128;
constexpr int K = 128, VS = 64;  // head dims (K = V = 128); V columns per CTA
constexpr int CG = VS / 4;       // float4 column groups per CTA
constexpr int RP = kThreads / CG;  // state rows per pass
constexpr int NI = K / RP;         // passes over K

struct FusedParams {
  const void* qkv;  // [S, conv_dim] projection rows (q | k | v channels)
  int64_t sx;       // row stride of qkv
  const void* cw;   // conv weight [conv_dim, W] (stride cw_c, cw_j)
  int64_t cw_c, cw_j;
  void* cst;  // conv state [S_max, W-1, conv_dim]
  int64_t cs_n, cs_t;
  const int32_t* cidx;
  const void *a, *b;  // [S, Hv] (strides a_t, a_h / b_t, b_h)
  int64_t a_t, a_h, b_t, b_h;
  int a_dt, b_dt;
  GateDev gd;
  float* st;  // recurrent state [S_max, Hv, K, V] fp32
  int64_t ss_n, ss_h, ss_k;
  const int32_t* sidx;
  const void* z;  // [S, Hv, V] (strides z_t, z_h)
  int64_t z_t, z_h;
  const void* nw;  // norm weight [V]
  int nw_dt;
  void* out;  // [S, Hv, V] (strides o_t, o_h)
  int64_t o_t, o_h;
  int hk, hv, group;
  float scale, eps;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A float in the shared memory of CTA `rank` of this cluster.
__device__ __forceinline__ float ld_dsmem(const float* p, uint32_t rank) {
  uint32_t local = smem_u32(p), remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// x sigmoid(x) through tanh.approx, as the conv kernels compute it.
__device__ __forceinline__ float silu_conv(float x) {
  const float h = 0.5f * x;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

template <typename T, typename TW, int W>
__global__ void __launch_bounds__(kThreads) gdn_decode_fused_kernel(const __grid_constant__ FusedParams p) {
  __shared__ float sq[K], sk[K], sv[VS];
  __shared__ float4 red_a[kThreads / 32][32], red_b[kThreads / 32][32];
  __shared__ float red_qk[kThreads / 32][32];
  __shared__ float s_gb[2], s_nrm[2];
  __shared__ float s_part;  // this half's sum of o^2, read by the other half

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg = tid % CG, rg = tid / CG;
  const int half = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int kh = h / p.group;
  const uint32_t crank = cluster_rank();
  const int vcol = half * VS + cg * 4;  // this thread's 4 state columns

  // ---- recurrent state loads first: the longest latency, independent of the conv ----
  float* S = p.st + (int64_t)p.sidx[seq] * p.ss_n + (int64_t)h * p.ss_h + vcol;
  float4 s[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) s[i] = __ldcs(reinterpret_cast<const float4*>(S + (int64_t)(rg + RP * i) * p.ss_k));

  // ---- conv of this CTA's channels: q (16 x 8), k (16 x 8), own v half (8 x 8) ----
  const int qt = p.hk * K;  // q channels; k channels follow, then v
  int c0 = -1, job = tid;   // first channel of this thread's 8, or -1
  if (job < 16) c0 = kh * K + job * 8;
  else if (job < 32) c0 = qt + kh * K + (job - 16) * 8;
  else if (job < 40) c0 = 2 * qt + h * 2 * VS + half * VS + (job - 32) * 8;
  float xin[8], hist[W > 1 ? W - 1 : 1][8];
  T* cst = static_cast<T*>(p.cst) + (int64_t)p.cidx[seq] * p.cs_n;
  if (c0 >= 0) {
    unpack8<T>(*reinterpret_cast<const uint4*>(static_cast<const T*>(p.qkv) + (int64_t)seq * p.sx + c0), xin);
#pragma unroll
    for (int j = 0; j < W - 1; ++j) unpack8<T>(*reinterpret_cast<const uint4*>(cst + j * p.cs_t + c0), hist[j]);
    const TW* wt = static_cast<const TW*>(p.cw) + (int64_t)c0 * p.cw_c;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float a = 0.f;
#pragma unroll
      for (int j = 0; j < W; ++j) a += to_f32<TW>(wt[(int64_t)i * p.cw_c + j * p.cw_j]) * (j == W - 1 ? xin[i] : hist[j][i]);
      acc[i] = to_f32<T>(from_f32<T>(silu_conv(a)));  // the activation dtype, as the conv op writes it
    }
    float* dst = job < 16 ? sq + job * 8 : (job < 32 ? sk + (job - 16) * 8 : sv + (job - 32) * 8);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = acc[i];
    if (job >= 32) {  // own v channels: shift this CTA's part of the conv state now
#pragma unroll
      for (int j = 0; j < W - 1; ++j)
        *reinterpret_cast<uint4*>(cst + j * p.cs_t + c0) = pack8<T>(j + 1 < W - 1 ? hist[j + 1] : xin);
    }
  }
  if (tid == 0) {
    float gv = load_scalar(p.a, (int64_t)seq * p.a_t + h * p.a_h, p.a_dt);
    float bv = load_scalar(p.b, (int64_t)seq * p.b_t + h * p.b_h, p.b_dt);
    s_gb[0] = expf(raw_gate_g(p.gd, gv, h));
    s_gb[1] = raw_gate_beta(bv, p.b_dt);
  }
  // every CTA of the cluster has read the shared q/k conv state -> the first one shifts it
  cluster_sync();
  if (crank == 0 && c0 >= 0 && job < 32) {
#pragma unroll
    for (int j = 0; j < W - 1; ++j)
      *reinterpret_cast<uint4*>(cst + j * p.cs_t + c0) = pack8<T>(j + 1 < W - 1 ? hist[j + 1] : xin);
  }

  // ---- q/k L2 norms (x rsqrt(sum x^2 + 1e-6), m/layers/linear_attention.py:113-114) ----
  if (warp == 0) {
    float a2 = 0.f, b2 = 0.f;
    for (int i = lane; i < K; i += 32) {
      a2 += sq[i] * sq[i];
      b2 += sk[i] * sk[i];
    }
    a2 = warp_sum(a2);
    b2 = warp_sum(b2);
    if (lane == 0) {
      s_nrm[0] = rsqrtf(a2 + 1e-6f);
      s_nrm[1] = rsqrtf(b2 + 1e-6f);
    }
  }
  __syncthreads();
  {
    const float nq = s_nrm[0], nk = s_nrm[1];
    for (int i = tid; i < K; i += kThreads) {
      sq[i] *= nq;
      sk[i] *= nk;
    }
  }
  __syncthreads();

  // ---- recurrence (as gdn_recurrent.cu): a = k^T S, b = q^T S in one pass ----
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f), bq = a;
  float qk = 0.f;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int r = rg + RP * i;
    const float kr = sk[r], qr = sq[r];
    a.x += kr * s[i].x; a.y += kr * s[i].y; a.z += kr * s[i].z; a.w += kr * s[i].w;
    bq.x += qr * s[i].x; bq.y += qr * s[i].y; bq.z += qr * s[i].z; bq.w += qr * s[i].w;
    qk += qr * kr;
  }
#pragma unroll
  for (int off = CG; off < 32; off <<= 1) {
    a.x += __shfl_xor_sync(0xffffffffu, a.x, off); a.y += __shfl_xor_sync(0xffffffffu, a.y, off);
    a.z += __shfl_xor_sync(0xffffffffu, a.z, off); a.w += __shfl_xor_sync(0xffffffffu, a.w, off);
    bq.x += __shfl_xor_sync(0xffffffffu, bq.x, off); bq.y += __shfl_xor_sync(0xffffffffu, bq.y, off);
    bq.z += __shfl_xor_sync(0xffffffffu, bq.z, off); bq.w += __shfl_xor_sync(0xffffffffu, bq.w, off);
    qk += __shfl_xor_sync(0xffffffffu, qk, off);
  }
  red_a[warp][lane] = a;
  red_b[warp][lane] = bq;
  red_qk[warp][lane] = qk;
  __syncthreads();
  a = make_float4(0.f, 0.f, 0.f, 0.f);
  bq = a;
  qk = 0.f;
  const int l0 = lane % CG;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    const float4 ra = red_a[w][l0], rb = red_b[w][l0];
    a.x += ra.x; a.y += ra.y; a.z += ra.z; a.w += ra.w;
    bq.x += rb.x; bq.y += rb.y; bq.z += rb.z; bq.w += rb.w;
    qk += red_qk[w][l0];
  }
  const float decay = s_gb[0], beta = s_gb[1];
  float4 vn;
  vn.x = beta * (sv[cg * 4 + 0] - decay * a.x);
  vn.y = beta * (sv[cg * 4 + 1] - decay * a.y);
  vn.z = beta * (sv[cg * 4 + 2] - decay * a.z);
  vn.w = beta * (sv[cg * 4 + 3] - decay * a.w);
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const float kr = sk[rg + RP * i];
    s[i].x = decay * s[i].x + kr * vn.x; s[i].y = decay * s[i].y + kr * vn.y;
    s[i].z = decay * s[i].z + kr * vn.z; s[i].w = decay * s[i].w + kr * vn.w;
  }
#pragma unroll
  for (int i = 0; i < NI; ++i) __stcs(reinterpret_cast<float4*>(S + (int64_t)(rg + RP * i) * p.ss_k), s[i]);

  // ---- o (rounded to the activation dtype, as the op returns it) and its sum of squares ----
  float o4[4] = {0.f, 0.f, 0.f, 0.f};
  float part = 0.f;
  if (rg == 0) {  // threads 0-15 of warp 0: 4 columns each
    const float sc = p.scale;
    o4[0] = to_f32<T>(from_f32<T>(sc * (decay * bq.x + qk * vn.x)));
    o4[1] = to_f32<T>(from_f32<T>(sc * (decay * bq.y + qk * vn.y)));
    o4[2] = to_f32<T>(from_f32<T>(sc * (decay * bq.z + qk * vn.z)));
    o4[3] = to_f32<T>(from_f32<T>(sc * (decay * bq.w + qk * vn.w)));
    part = o4[0] * o4[0] + o4[1] * o4[1] + o4[2] * o4[2] + o4[3] * o4[3];
  }
  if (warp == 0) {
    part = warp_sum(part);
    if (lane == 0) s_part = part;
  }
  // both halves' partial sums are written -> read the other half's; the last barrier keeps
  // every CTA's shared memory alive until its peer has read it
  cluster_sync();
  const float p0 = half == 0 ? s_part : ld_dsmem(&s_part, crank ^ 1u);
  const float p1 = half == 1 ? s_part : ld_dsmem(&s_part, crank ^ 1u);
  cluster_sync();
  if (rg == 0) {
    const float r = rsqrtf((p0 + p1) / (float)(2 * VS) + p.eps);
    const T* zr = static_cast<const T*>(p.z) + (int64_t)seq * p.z_t + (int64_t)h * p.z_h + vcol;
    T* orow = static_cast<T*>(p.out) + (int64_t)seq * p.o_t + (int64_t)h * p.o_h + vcol;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      orow[j] = from_f32<T>(o4[j] * r * load_scalar(p.nw, vcol + j, p.nw_dt) * silu(to_f32<T>(zr[j])));
  }
}

template <typename T, typename TW, int W>
cudaError_t launch_fused(const FusedParams& p, int64_t S, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, (unsigned)p.hv, (unsigned)S);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = (unsigned)p.group;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gdn_decode_fused_kernel<T, TW, W>, p);
}

template <typename T, typename TW>
cudaError_t launch_w(int w, const FusedParams& p, int64_t S, cudaStream_t st) {
  switch (w) {
    case 2: return launch_fused<T, TW, 2>(p, S, st);
    case 3: return launch_fused<T, TW, 3>(p, S, st);
    case 4: return launch_fused<T, TW, 4>(p, S, st);
    case 5: return launch_fused<T, TW, 5>(p, S, st);
    case 6: return launch_fused<T, TW, 6>(p, S, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_gated_deltanet_decode(const mvb_tensor* qkv, const mvb_tensor* conv_weight, mvb_tensor* conv_state,
                                         const mvb_tensor* conv_state_indices, const mvb_tensor* a,
                                         const mvb_tensor* b, const mvb_tensor* a_log, const mvb_tensor* dt_bias,
                                         mvb_tensor* recurrent_state, const mvb_tensor* recurrent_state_indices,
                                         const mvb_tensor* z, const mvb_tensor* norm_weight, float norm_eps,
                                         float scale, mvb_tensor* out, void* stream) {
  using namespace mvb;
  const char* op = "gated_deltanet_decode";
  int rc;
  if ((rc = check_tensor(qkv, op, "qkv", 2)) || (rc = check_tensor(conv_weight, op, "conv_weight", 2)) ||
      (rc = check_tensor(conv_state, op, "conv_state", 3)) ||
      (rc = check_tensor(conv_state_indices, op, "conv_state_indices", 1)) || (rc = check_tensor(a, op, "a", 2)) ||
      (rc = check_tensor(b, op, "b", 2)) || (rc = check_tensor(a_log, op, "A_log", 1)) ||
      (rc = check_tensor(dt_bias, op, "dt_bias", 1)) || (rc = check_tensor(recurrent_state, op, "recurrent_state", 4)) ||
      (rc = check_tensor(recurrent_state_indices, op, "recurrent_state_indices", 1)) ||
      (rc = check_tensor(z, op, "z", 3)) || (rc = check_tensor(norm_weight, op, "norm_weight", 1)) ||
      (rc = check_tensor(out, op, "out", 3)))
    return rc;
  const int64_t S = qkv->shape[0], dim = qkv->shape[1], Wd = conv_weight->shape[1];
  const int64_t hv = recurrent_state->shape[1], kd = recurrent_state->shape[2], vd = recurrent_state->shape[3];
  MVB_CHECK_SUPPORTED(kd == K && vd == 2 * VS, "%s: head dims must be K = V = 128 (got %lld, %lld)", op,
                      (long long)kd, (long long)vd);
  MVB_CHECK_ARG(hv > 0 && (dim - hv * vd) > 0 && (dim - hv * vd) % (2 * kd) == 0,
                "%s: qkv width %lld is not 2 Hk K + Hv V for Hv = %lld", op, (long long)dim, (long long)hv);
  const int64_t hk = (dim - hv * vd) / (2 * kd);
  MVB_CHECK_ARG(hv % hk == 0, "%s: Hv (%lld) must be a multiple of Hk (%lld)", op, (long long)hv, (long long)hk);
  const int64_t group = hv / hk;
  MVB_CHECK_SUPPORTED(group == 1 || group == 2 || group == 4, "%s: Hv / Hk must be 1, 2 or 4 (got %lld)", op,
                      (long long)group);
  MVB_CHECK_SUPPORTED(Wd >= 2 && Wd <= 6, "%s: conv width must be 2..6", op);
  MVB_CHECK_ARG(conv_weight->shape[0] == dim && conv_state->shape[1] == Wd - 1 && conv_state->shape[2] == dim,
                "%s: conv_weight [dim, W] / conv_state [S_max, W-1, dim] disagree with qkv", op);
  MVB_CHECK_ARG(a->shape[0] == S && a->shape[1] == hv && b->shape[0] == S && b->shape[1] == hv,
                "%s: a, b must be [S, Hv]", op);
  MVB_CHECK_ARG(a_log->shape[0] == hv && dt_bias->shape[0] == hv && a_log->stride[0] == 1 && dt_bias->stride[0] == 1,
                "%s: A_log and dt_bias must be contiguous [Hv]", op);
  MVB_CHECK_ARG(z->shape[0] == S && z->shape[1] == hv && z->shape[2] == vd && out->shape[0] == S &&
                    out->shape[1] == hv && out->shape[2] == vd,
                "%s: z and out must be [S, Hv, V]", op);
  MVB_CHECK_ARG(norm_weight->shape[0] == vd && norm_weight->stride[0] == 1, "%s: norm_weight must be [V]", op);
  MVB_CHECK_ARG(conv_state_indices->shape[0] >= S && recurrent_state_indices->shape[0] >= S &&
                    conv_state_indices->dtype == MVB_I32 && recurrent_state_indices->dtype == MVB_I32,
                "%s: state indices must be int32 [>= S]", op);
  const int dt = qkv->dtype;
  MVB_CHECK_SUPPORTED(dt == MVB_BF16 || dt == MVB_F16, "%s: qkv must be bf16 or fp16", op);
  MVB_CHECK_ARG(conv_state->dtype == dt && z->dtype == dt && out->dtype == dt && recurrent_state->dtype == MVB_F32,
                "%s: conv_state, z and out must have the dtype of qkv; recurrent_state fp32", op);
  MVB_CHECK_ARG((conv_weight->dtype == MVB_F32 || conv_weight->dtype == dt) &&
                    (a->dtype == MVB_F32 || a->dtype == dt) && (b->dtype == MVB_F32 || b->dtype == dt) &&
                    (a_log->dtype == MVB_F32 || a_log->dtype == dt) && (dt_bias->dtype == MVB_F32 || dt_bias->dtype == dt) &&
                    (norm_weight->dtype == MVB_F32 || norm_weight->dtype == dt),
                "%s: weights and gates must be float32 or the dtype of qkv", op);
  MVB_CHECK_SUPPORTED(qkv->stride[1] == 1 && qkv->stride[0] % 8 == 0 && aligned16(qkv->data) &&
                          conv_state->stride[2] == 1 && conv_state->stride[1] % 8 == 0 &&
                          conv_state->stride[0] % 8 == 0 && aligned16(conv_state->data),
                      "%s: qkv rows and conv state rows must be contiguous and 16-byte aligned", op);
  MVB_CHECK_SUPPORTED(recurrent_state->stride[3] == 1 && recurrent_state->stride[2] % 4 == 0 &&
                          recurrent_state->stride[1] % 4 == 0 && recurrent_state->stride[0] % 4 == 0 &&
                          aligned16(recurrent_state->data),
                      "%s: recurrent_state needs unit V stride and 16-byte aligned rows", op);
  MVB_CHECK_SUPPORTED(z->stride[2] == 1 && out->stride[2] == 1, "%s: z and out need a unit last stride", op);
  MVB_CHECK_SUPPORTED(S <= 65535 && hv <= 65535, "%s: at most 65535 sequences", op);
  if (S == 0) return MVB_OK;

  FusedParams p;
  memset(&p, 0, sizeof(p));
  p.qkv = qkv->data; p.sx = qkv->stride[0];
  p.cw = conv_weight->data; p.cw_c = conv_weight->stride[0]; p.cw_j = conv_weight->stride[1];
  p.cst = conv_state->data; p.cs_n = conv_state->stride[0]; p.cs_t = conv_state->stride[1];
  p.cidx = static_cast<const int32_t*>(conv_state_indices->data);
  p.a = a->data; p.a_t = a->stride[0]; p.a_h = a->stride[1]; p.a_dt = a->dtype;
  p.b = b->data; p.b_t = b->stride[0]; p.b_h = b->stride[1]; p.b_dt = b->dtype;
  p.gd.alog = a_log->data; p.gd.alog_dt = a_log->dtype; p.gd.dtb = dt_bias->data; p.gd.dtb_dt = dt_bias->dtype;
  p.st = static_cast<float*>(recurrent_state->data);
  p.ss_n = recurrent_state->stride[0]; p.ss_h = recurrent_state->stride[1]; p.ss_k = recurrent_state->stride[2];
  p.sidx = static_cast<const int32_t*>(recurrent_state_indices->data);
  p.z = z->data; p.z_t = z->stride[0]; p.z_h = z->stride[1];
  p.nw = norm_weight->data; p.nw_dt = norm_weight->dtype;
  p.out = out->data; p.o_t = out->stride[0]; p.o_h = out->stride[1];
  p.hk = (int)hk; p.hv = (int)hv; p.group = (int)group;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)kd);
  p.eps = norm_eps;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  const int cw = conv_weight->dtype;
  if (dt == MVB_BF16)
    e = cw == MVB_F32 ? launch_w<__nv_bfloat16, float>((int)Wd, p, S, st)
                      : launch_w<__nv_bfloat16, __nv_bfloat16>((int)Wd, p, S, st);
  else
    e = cw == MVB_F32 ? launch_w<__half, float>((int)Wd, p, S, st) : launch_w<__half, __half>((int)Wd, p, S, st);
  if (e != cudaSuccess) MVB_FAIL(MVB_ERR_CUDA, "%s: launch failed: %s", op, cudaGetErrorString(e));
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}
