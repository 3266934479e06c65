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
// Grid (2, Hv, S), 128 threads: a CTA owns one half (64 columns) of the V axis of one
// (sequence, v-head), with the state streamed through registers exactly as
// gdn_recurrent.cu does it (four such CTAs fit an SM).  Work shared between CTAs is handed
// to whichever CTA finishes its part last, through counters in caller memory (zero-initialised
// once; every counter returns to zero), so no CTA waits for another:
//   - every CTA recomputes the conv of its k-head's q and k channels (256 channels, 4 taps:
//     cheaper than exchanging them) and of its own 64 v channels, and shifts the conv state
//     of those v channels, which no other CTA reads;
//   - the q/k channels' conv state is read by the 2 G CTAs of the G = Hv / Hk v-heads that
//     share the k-head: each counts itself out after its read, and the last one shifts it;
//   - each half writes its 64 (rounded) o values and their sum of squares to the workspace
//     and counts itself out; the last of the two forms the RMS over all 128 columns (the
//     halves' sums added in half order) and writes both halves' normed output.
// Numerics follow the unfused ops: the conv output is rounded to the activation dtype
// before the norms, o is rounded before RMSNormGated, all arithmetic is fp32.
#include "common.cuh"

namespace mvb {
namespace {

constexpr int kThreads = 128;
constexpr int K = 128, VS = 64;    // head dims (K = V = 128); V columns per CTA
constexpr int CG = VS / 4;         // float4 column groups per CTA
constexpr int RP = kThreads / CG;  // state rows per pass
constexpr int NI = K / RP;         // passes over K
constexpr int kHalfFloats = VS + 4;  // per (sequence, head, half): 64 o values, their sum of squares, pad

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
  int* cnt_conv;  // [S, Hk]  CTAs done reading the shared q/k conv state
  int* cnt_norm;  // [S, Hv]  halves done with their o
  float* half_o;  // [S, Hv, 2, kHalfFloats]
  int hk, hv, group;
  float scale, eps;
};

// x sigmoid(x) through tanh.approx, as the conv kernels compute it.
__device__ __forceinline__ float silu_conv(float x) {
  const float h = 0.5f * x;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

// Counts this CTA out of `cnt` (its earlier memory operations made visible first); true for
// the CTA that completes the count `total`, which also resets it for the next launch.
__device__ __forceinline__ bool count_out(int* cnt, int total) {
  __threadfence();
  const bool last = atomicAdd(cnt, 1) == total - 1;
  if (last) *cnt = 0;
  return last;
}

template <typename T, typename TW, int W>
__global__ void __launch_bounds__(kThreads) gdn_decode_fused_kernel(const __grid_constant__ FusedParams p) {
  __shared__ float sq[K], sk[K], sv[VS];
  __shared__ float4 red_a[kThreads / 32][32], red_b[kThreads / 32][32];
  __shared__ float red_qk[kThreads / 32][32];
  __shared__ float s_gb[2], s_nrm[2];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cg = tid % CG, rg = tid / CG;
  const int half = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int kh = h / p.group;
  const int vcol = half * VS + cg * 4;  // this thread's 4 state columns

  // ---- recurrent state loads first: the longest latency, independent of the conv ----
  float* S = p.st + (int64_t)p.sidx[seq] * p.ss_n + (int64_t)h * p.ss_h + vcol;
  float4 s[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) s[i] = __ldcs(reinterpret_cast<const float4*>(S + (int64_t)(rg + RP * i) * p.ss_k));

  // ---- conv, four channels a thread: q (32 x 4), k (32 x 4), own v half (16 x 4) ----
  const int qt = p.hk * K;  // q channels; k channels follow, then v
  const int job = tid;
  int c0 = -1;  // first channel of this thread's four, or -1
  if (job < 32) c0 = kh * K + 4 * job;
  else if (job < 64) c0 = qt + kh * K + 4 * (job - 32);
  else if (job < 80) c0 = 2 * qt + h * 2 * VS + half * VS + 4 * (job - 64);
  T* cst = static_cast<T*>(p.cst) + (int64_t)p.cidx[seq] * p.cs_n;
  const T* xrow = static_cast<const T*>(p.qkv) + (int64_t)seq * p.sx;
  if (c0 >= 0) {
    const uint2 xin = *reinterpret_cast<const uint2*>(xrow + c0);
    uint2 hist[W - 1];
#pragma unroll
    for (int j = 0; j < W - 1; ++j) hist[j] = *reinterpret_cast<const uint2*>(cst + j * p.cs_t + c0);
    const TW* wt = static_cast<const TW*>(p.cw) + (int64_t)c0 * p.cw_c;
    float acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = 0.f;
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const uint2 u = j == W - 1 ? xin : hist[j];
        a += to_f32<TW>(wt[(int64_t)i * p.cw_c + j * p.cw_j]) * to_f32<T>(reinterpret_cast<const T*>(&u)[i]);
      }
      acc[i] = to_f32<T>(from_f32<T>(silu_conv(a)));  // the activation dtype, as the conv op writes it
    }
    float* dst = job < 32 ? sq + 4 * job : (job < 64 ? sk + 4 * (job - 32) : sv + 4 * (job - 64));
    *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    if (job >= 64) {  // own v channels: no other CTA reads them
#pragma unroll
      for (int j = 0; j < W - 1; ++j) *reinterpret_cast<uint2*>(cst + j * p.cs_t + c0) = j + 1 < W - 1 ? hist[j + 1] : xin;
    }
  }
  if (tid == 0) {
    float gv = load_scalar(p.a, (int64_t)seq * p.a_t + h * p.a_h, p.a_dt);
    float bv = load_scalar(p.b, (int64_t)seq * p.b_t + h * p.b_h, p.b_dt);
    s_gb[0] = expf(raw_gate_g(p.gd, gv, h));
    s_gb[1] = raw_gate_beta(bv, p.b_dt);
  }
  __syncthreads();
  // this CTA has read the shared q/k conv state; the last of its 2 G readers shifts it
  if (tid == 0) s_last = count_out(p.cnt_conv + (int64_t)seq * p.hk + kh, 2 * p.group);
  __syncthreads();
  if (s_last && c0 >= 0 && job < 64) {
    __threadfence();
    uint2 rows[W];
#pragma unroll
    for (int j = 1; j < W - 1; ++j) rows[j] = __ldcg(reinterpret_cast<const uint2*>(cst + j * p.cs_t + c0));
    rows[W - 1] = *reinterpret_cast<const uint2*>(xrow + c0);
#pragma unroll
    for (int j = 0; j < W - 1; ++j) *reinterpret_cast<uint2*>(cst + j * p.cs_t + c0) = rows[j + 1];
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

  // ---- o (rounded to the activation dtype, as the op returns it) -> this half's record ----
  float* rec = p.half_o + ((int64_t)seq * p.hv + h) * 2 * kHalfFloats;
  if (rg == 0) {  // threads 0-15 of warp 0: 4 columns each
    const float sc = p.scale;
    const float o4[4] = {to_f32<T>(from_f32<T>(sc * (decay * bq.x + qk * vn.x))),
                         to_f32<T>(from_f32<T>(sc * (decay * bq.y + qk * vn.y))),
                         to_f32<T>(from_f32<T>(sc * (decay * bq.z + qk * vn.z))),
                         to_f32<T>(from_f32<T>(sc * (decay * bq.w + qk * vn.w)))};
    *reinterpret_cast<float4*>(rec + half * kHalfFloats + cg * 4) = make_float4(o4[0], o4[1], o4[2], o4[3]);
    float part = o4[0] * o4[0] + o4[1] * o4[1] + o4[2] * o4[2] + o4[3] * o4[3];
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) part += __shfl_xor_sync(0x0000ffffu, part, off);
    if (lane == 0) rec[half * kHalfFloats + VS] = part;
  }
  __syncthreads();
  // the last of the two halves writes the normed output of both
  if (tid == 0) s_last = count_out(p.cnt_norm + (int64_t)seq * p.hv + h, 2);
  __syncthreads();
  if (s_last && warp == 0) {
    __threadfence();
    const int hh = lane >> 4, col = hh * VS + (lane & 15) * 4;  // lanes 0-15: half 0, 16-31: half 1
    const float ss = __ldcg(rec + VS) + __ldcg(rec + kHalfFloats + VS);
    const float r = rsqrtf(ss / (float)(2 * VS) + p.eps);
    const float4 o4 = __ldcg(reinterpret_cast<const float4*>(rec + hh * kHalfFloats + (lane & 15) * 4));
    const T* zr = static_cast<const T*>(p.z) + (int64_t)seq * p.z_t + (int64_t)h * p.z_h + col;
    T* orow = static_cast<T*>(p.out) + (int64_t)seq * p.o_t + (int64_t)h * p.o_h + col;
    const float ov[4] = {o4.x, o4.y, o4.z, o4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      orow[j] = from_f32<T>(ov[j] * r * load_scalar(p.nw, col + j, p.nw_dt) * silu(to_f32<T>(zr[j])));
  }
  // the new state last: nothing after these stores waits for them
#pragma unroll
  for (int i = 0; i < NI; ++i) __stcs(reinterpret_cast<float4*>(S + (int64_t)(rg + RP * i) * p.ss_k), s[i]);
}

template <typename T, typename TW>
cudaError_t launch_w(int w, const FusedParams& p, int64_t S, cudaStream_t st) {
  const dim3 grid(2, (unsigned)p.hv, (unsigned)S);
  switch (w) {
    case 2: gdn_decode_fused_kernel<T, TW, 2><<<grid, kThreads, 0, st>>>(p); break;
    case 3: gdn_decode_fused_kernel<T, TW, 3><<<grid, kThreads, 0, st>>>(p); break;
    case 4: gdn_decode_fused_kernel<T, TW, 4><<<grid, kThreads, 0, st>>>(p); break;
    case 5: gdn_decode_fused_kernel<T, TW, 5><<<grid, kThreads, 0, st>>>(p); break;
    case 6: gdn_decode_fused_kernel<T, TW, 6><<<grid, kThreads, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaSuccess;
}

// Caller memory: the counters (conv [S, Hk], norm [S, Hv]; zero, and left at zero) and the
// per-half records (no initial value needed).  Two buffers, so that records of one call never
// land where another call's counters are.
size_t counter_bytes(int64_t S, int64_t hk, int64_t hv) { return (size_t)S * (hk + hv) * sizeof(int); }
size_t record_bytes(int64_t S, int64_t hv) { return (size_t)S * hv * 2 * kHalfFloats * sizeof(float); }

}  // namespace
}  // namespace mvb

extern "C" int mvb_gated_deltanet_decode_workspace_sizes(int64_t n_seqs, int64_t num_k_heads, int64_t num_v_heads,
                                                         size_t* counters_bytes, size_t* records_bytes) {
  if (counters_bytes == nullptr || records_bytes == nullptr || n_seqs < 0 || num_k_heads <= 0 || num_v_heads <= 0)
    MVB_FAIL(MVB_ERR_ARG, "gated_deltanet_decode_workspace_sizes: bad arguments");
  *counters_bytes = mvb::counter_bytes(n_seqs, num_k_heads, num_v_heads);
  *records_bytes = mvb::record_bytes(n_seqs, num_v_heads);
  return MVB_OK;
}

extern "C" int mvb_gated_deltanet_decode(const mvb_tensor* qkv, const mvb_tensor* conv_weight, mvb_tensor* conv_state,
                                         const mvb_tensor* conv_state_indices, const mvb_tensor* a,
                                         const mvb_tensor* b, const mvb_tensor* a_log, const mvb_tensor* dt_bias,
                                         mvb_tensor* recurrent_state, const mvb_tensor* recurrent_state_indices,
                                         const mvb_tensor* z, const mvb_tensor* norm_weight, float norm_eps,
                                         float scale, mvb_tensor* out, void* counters, size_t counters_bytes,
                                         void* records, size_t records_bytes, void* stream) {
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
  MVB_CHECK_ARG(counters != nullptr && counters_bytes >= counter_bytes(S, hk, hv) &&
                    (reinterpret_cast<uintptr_t>(counters) & 3) == 0,
                "%s: needs %zu bytes of zero-initialised counters (mvb_gated_deltanet_decode_workspace_sizes)", op,
                counter_bytes(S, hk, hv));
  MVB_CHECK_ARG(records != nullptr && records_bytes >= record_bytes(S, hv) && (reinterpret_cast<uintptr_t>(records) & 15) == 0,
                "%s: needs %zu bytes of 16-byte aligned record space (mvb_gated_deltanet_decode_workspace_sizes)", op,
                record_bytes(S, hv));

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
  p.cnt_conv = static_cast<int*>(counters);
  p.cnt_norm = p.cnt_conv + S * hk;
  p.half_o = static_cast<float*>(records);
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
