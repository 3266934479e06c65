// Recurrent gated delta rule on CUDA cores (HBM-bound).
//
// Decode (one token per sequence) replaces the reference's _fused_recurrent_gdn
// (m/ops/gated_delta_rule/fused_recurrent_gdn.py:6-102).  Per (seq, v-head) the fp32
// state S [K, V] is read once, updated and written once:
//   S_d = e^g S;  a = k^T S_d;  b = q^T S_d;  v' = beta (v - a);
//   S' = S_d + k v'^T;  o = scale (b + (q.k) v')          (== scale q^T S')
// Both reductions over K come out of the same register-resident pass over S, so the
// kernel moves exactly 2 * 4KV bytes of state per (seq, head).
//
// Layout: grid (V / VS, Hv, S); 128 threads; thread owns a float4 column group
// (VS/4 groups across the slice) and rows r = rg + 8 i of S (rg = tid / (VS/4)).
// Rows of one warp cover whole 256-byte (VS=64) row segments: coalesced 16-byte
// streaming loads/stores (evict-first, the state is touched once per step).
//
// The same kernel with a token loop (cu_seqlens given) runs a whole packed prefill
// sequence token by token with S in registers; the library uses it for fp32 inputs and
// head sizes the chunked tensor-core kernel does not cover.  With l2norm set, q and k
// are scaled by rsqrt(sum x^2 + 1e-6) first (m/layers/linear_attention.py:113-114).
#include "common.cuh"

namespace mvb {
namespace {

struct RecParams {
  const void *q, *k, *v, *g, *beta;
  void* o;
  float* state;
  const int32_t* state_idx;
  const int32_t* cu_seqlens;  // null for decode
  int64_t sq_t, sq_h, sq_d, sk_t, sk_h, sk_d, sv_t, sv_h, sv_d, so_t, so_h, so_d;
  int64_t sg_t, sg_h, sb_t, sb_h;
  int64_t ss_n, ss_h, ss_k;  // state strides (V stride must be 1)
  int hk, hv, vdim, l2norm, g_dtype, b_dtype;
  float scale;
  GateDev gd;  // raw gates (a, b in the g, beta slots) when gd.alog is set
};

// g and beta may each be fp32 or the activation dtype (the reference layer makes g fp32
// and beta bf16, m/layers/linear_attention.py:89-90).
__device__ __forceinline__ float load_gate(const void* p, int64_t i, int dtype) {
  if (dtype == MVB_F32) return static_cast<const float*>(p)[i];
  if (dtype == MVB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

constexpr int kThreads = 128;

template <typename T, int K, int VS>
__global__ void __launch_bounds__(kThreads) gdn_recurrent_kernel(RecParams p) {
  constexpr int CG = VS / 4;           // float4 column groups per slice
  constexpr int RP = kThreads / CG;    // rows per pass
  constexpr int NI = K / RP;           // passes over K
  static_assert(kThreads % CG == 0 && K % RP == 0, "bad tiling");
  constexpr int NW = kThreads / 32;

  __shared__ float sq[K], sk[K], sv[VS];
  __shared__ float4 red_a[NW][32], red_b[NW][32];
  __shared__ float red_qk[NW][32];
  __shared__ float s_gb[2];
  __shared__ float s_nrm[2];

  const int tid = threadIdx.x;
  const int cg = tid % CG;
  const int rg = tid / CG;
  const int lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.y;
  const int seq = blockIdx.z;
  const int v0 = blockIdx.x * VS + cg * 4;
  const bool col_ok = v0 < p.vdim;
  const int kh = h / (p.hv / p.hk);

  int t_begin = seq, t_end = seq + 1;
  if (p.cu_seqlens != nullptr) {
    t_begin = p.cu_seqlens[seq];
    t_end = p.cu_seqlens[seq + 1];
  }
  const int64_t slot = p.state_idx[seq];
  float* S = p.state + slot * p.ss_n + h * p.ss_h + v0;

  float4 s[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int r = rg + RP * i;
    s[i] = col_ok ? __ldcs(reinterpret_cast<const float4*>(S + r * p.ss_k)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }

  const T* qp = static_cast<const T*>(p.q);
  const T* kp = static_cast<const T*>(p.k);
  const T* vp = static_cast<const T*>(p.v);
  T* op = static_cast<T*>(p.o);

  for (int t = t_begin; t < t_end; ++t) {
    for (int i = tid; i < K; i += kThreads) {
      sq[i] = to_f32<T>(qp[t * p.sq_t + kh * p.sq_h + i * p.sq_d]);
      sk[i] = to_f32<T>(kp[t * p.sk_t + kh * p.sk_h + i * p.sk_d]);
    }
    for (int i = tid; i < VS; i += kThreads) {
      const int vv = blockIdx.x * VS + i;
      sv[i] = vv < p.vdim ? to_f32<T>(vp[t * p.sv_t + h * p.sv_h + vv * p.sv_d]) : 0.f;
    }
    if (tid == 0) {
      float gv = load_gate(p.g, (int64_t)t * p.sg_t + h * p.sg_h, p.g_dtype);
      float bv = load_gate(p.beta, (int64_t)t * p.sb_t + h * p.sb_h, p.b_dtype);
      if (p.gd.alog != nullptr) {
        gv = raw_gate_g(p.gd, gv, h);
        bv = raw_gate_beta(bv, p.b_dtype);
      }
      s_gb[0] = expf(gv);
      s_gb[1] = bv;
    }
    __syncthreads();
    if (p.l2norm) {
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
      const float nq = s_nrm[0], nk = s_nrm[1];
      for (int i = tid; i < K; i += kThreads) {
        sq[i] *= nq;
        sk[i] *= nk;
      }
      __syncthreads();
    }

    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    float qk = 0.f;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int r = rg + RP * i;
      const float kr = sk[r], qr = sq[r];
      a.x += kr * s[i].x; a.y += kr * s[i].y; a.z += kr * s[i].z; a.w += kr * s[i].w;
      b.x += qr * s[i].x; b.y += qr * s[i].y; b.z += qr * s[i].z; b.w += qr * s[i].w;
      qk += qr * kr;
    }
    // Lanes of one warp with the same column group hold different rows.
#pragma unroll
    for (int off = CG; off < 32; off <<= 1) {
      a.x += __shfl_xor_sync(0xffffffffu, a.x, off); a.y += __shfl_xor_sync(0xffffffffu, a.y, off);
      a.z += __shfl_xor_sync(0xffffffffu, a.z, off); a.w += __shfl_xor_sync(0xffffffffu, a.w, off);
      b.x += __shfl_xor_sync(0xffffffffu, b.x, off); b.y += __shfl_xor_sync(0xffffffffu, b.y, off);
      b.z += __shfl_xor_sync(0xffffffffu, b.z, off); b.w += __shfl_xor_sync(0xffffffffu, b.w, off);
      qk += __shfl_xor_sync(0xffffffffu, qk, off);
    }
    red_a[warp][lane] = a;
    red_b[warp][lane] = b;
    red_qk[warp][lane] = qk;
    __syncthreads();
    a = make_float4(0.f, 0.f, 0.f, 0.f);
    b = a;
    qk = 0.f;
    const int l0 = lane % CG;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float4 ra = red_a[w][l0], rb = red_b[w][l0];
      a.x += ra.x; a.y += ra.y; a.z += ra.z; a.w += ra.w;
      b.x += rb.x; b.y += rb.y; b.z += rb.z; b.w += rb.w;
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
    if (rg == 0 && col_ok) {
      const float sc = p.scale;
      T* ot = op + t * p.so_t + h * p.so_h;
      const float o4[4] = {sc * (decay * b.x + qk * vn.x), sc * (decay * b.y + qk * vn.y),
                           sc * (decay * b.z + qk * vn.z), sc * (decay * b.w + qk * vn.w)};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (v0 + j < p.vdim) ot[(v0 + j) * p.so_d] = from_f32<T>(o4[j]);
    }
    __syncthreads();  // smem of this token is dead before the next token overwrites it
  }

#pragma unroll
  for (int i = 0; i < NI; ++i) {
    const int r = rg + RP * i;
    if (col_ok) __stcs(reinterpret_cast<float4*>(S + r * p.ss_k), s[i]);
  }
}

template <typename T, int K>
void launch_rec(const RecParams& p, int n_seqs, cudaStream_t st) {
  constexpr int VS = 64;
  dim3 grid((p.vdim + VS - 1) / VS, p.hv, n_seqs);
  gdn_recurrent_kernel<T, K, VS><<<grid, kThreads, 0, st>>>(p);
}

template <typename T>
int dispatch_k(const RecParams& p, int kdim, int n_seqs, cudaStream_t st) {
  switch (kdim) {
    case 32: launch_rec<T, 32>(p, n_seqs, st); break;
    case 64: launch_rec<T, 64>(p, n_seqs, st); break;
    case 128: launch_rec<T, 128>(p, n_seqs, st); break;
    case 256: launch_rec<T, 256>(p, n_seqs, st); break;
    default: MVB_FAIL(MVB_ERR_UNSUPPORTED, "gated delta rule: K=%d not in {32,64,128,256}", kdim);
  }
  return MVB_OK;
}

}  // namespace

// Validates the per-head A_log / dt_bias vectors of the raw-gate entry points.
int make_gate_dev(const char* op, const mvb_tensor* a_log, const mvb_tensor* dt_bias, const mvb_tensor* v,
                  const mvb_tensor* q, GateDev* out) {
  int rc;
  if ((rc = check_tensor(a_log, op, "A_log", 1)) || (rc = check_tensor(dt_bias, op, "dt_bias", 1))) return rc;
  const int64_t hv = v->ndim == 3 ? v->shape[1] : -1;
  MVB_CHECK_ARG(a_log->shape[0] == hv && dt_bias->shape[0] == hv, "%s: A_log and dt_bias must be [Hv]", op);
  MVB_CHECK_ARG(a_log->stride[0] == 1 && dt_bias->stride[0] == 1, "%s: A_log and dt_bias must be contiguous", op);
  MVB_CHECK_ARG((a_log->dtype == MVB_F32 || a_log->dtype == q->dtype) &&
                    (dt_bias->dtype == MVB_F32 || dt_bias->dtype == q->dtype),
                "%s: A_log and dt_bias must each be float32 or the dtype of q", op);
  out->alog = a_log->data;
  out->dtb = dt_bias->data;
  out->alog_dt = a_log->dtype;
  out->dtb_dt = dt_bias->dtype;
  return MVB_OK;
}

// Argument validation shared by the recurrent and the chunked entry points.  For decode
// the token axis of q/k/v/g/beta/o is the sequence axis and cu_seqlens is NULL.
int check_gdn(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
              const mvb_tensor* beta, const mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
              const mvb_tensor* o, int64_t* n_seqs_out) {
  int rc;
  if ((rc = check_tensor(q, op, "q", 3)) || (rc = check_tensor(k, op, "k", 3)) ||
      (rc = check_tensor(v, op, "v", 3)) || (rc = check_tensor(g, op, "g", 2)) ||
      (rc = check_tensor(beta, op, "beta", 2)) || (rc = check_tensor(state, op, "recurrent_state", 4)) ||
      (rc = check_tensor(idx, op, "recurrent_state_indices", 1)) || (rc = check_tensor(o, op, "o", 3)))
    return rc;
  const int64_t T = q->shape[0], hk = q->shape[1], kd = q->shape[2];
  const int64_t hv = v->shape[1], vd = v->shape[2];
  MVB_CHECK_ARG(k->shape[0] == T && k->shape[1] == hk && k->shape[2] == kd, "%s: k shape != q shape", op);
  MVB_CHECK_ARG(v->shape[0] == T, "%s: v token count", op);
  MVB_CHECK_ARG(g->shape[0] == T && g->shape[1] == hv && beta->shape[0] == T && beta->shape[1] == hv,
                "%s: g/beta must be [T, Hv]", op);
  MVB_CHECK_ARG(o->shape[0] == T && o->shape[1] == hv && o->shape[2] == vd, "%s: o must be [T, Hv, V]", op);
  MVB_CHECK_ARG(hk > 0 && hv % hk == 0, "%s: Hv (%lld) must be a multiple of Hk (%lld)", op, (long long)hv,
                (long long)hk);
  MVB_CHECK_ARG(state->shape[1] == hv && state->shape[2] == kd && state->shape[3] == vd,
                "%s: recurrent_state must be [S_max, Hv, K, V]", op);
  MVB_CHECK_ARG(state->dtype == MVB_F32, "%s: recurrent_state must be float32", op);
  MVB_CHECK_ARG(idx->dtype == MVB_I32, "%s: recurrent_state_indices must be int32", op);
  MVB_CHECK_ARG(q->dtype == k->dtype && q->dtype == v->dtype && o->dtype == v->dtype && is_float_dtype(q->dtype),
                "%s: q/k/v/o must share one float dtype", op);
  MVB_CHECK_ARG((g->dtype == MVB_F32 || g->dtype == q->dtype) && (beta->dtype == MVB_F32 || beta->dtype == q->dtype),
                "%s: g and beta must each be float32 or the dtype of q", op);
  int64_t n_seqs = T;
  if (cu != nullptr) {
    if ((rc = check_tensor(cu, op, "cu_seqlens", 1))) return rc;
    MVB_CHECK_ARG(cu->dtype == MVB_I32 && cu->shape[0] >= 1, "%s: cu_seqlens must be int32 [S+1]", op);
    n_seqs = cu->shape[0] - 1;
  }
  MVB_CHECK_ARG(idx->shape[0] >= n_seqs, "%s: recurrent_state_indices shorter than the batch", op);
  *n_seqs_out = n_seqs;
  return MVB_OK;
}

int run_recurrent(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                  const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx,
                  const mvb_tensor* cu, mvb_tensor* o, float scale, int l2norm, const GateDev& gd, cudaStream_t st) {
  int64_t n_seqs = 0;
  int rc = check_gdn(op, q, k, v, g, beta, state, idx, cu, o, &n_seqs);
  if (rc) return rc;
  const int64_t hk = q->shape[1], kd = q->shape[2], hv = v->shape[1], vd = v->shape[2];
  MVB_CHECK_SUPPORTED(state->stride[3] == 1 && state->stride[2] % 4 == 0 && state->stride[1] % 4 == 0 &&
                          state->stride[0] % 4 == 0 && aligned16(state->data) && vd % 4 == 0,
                      "%s: recurrent_state needs unit V stride and 16-byte aligned rows (V %% 4 == 0)", op);
  MVB_CHECK_SUPPORTED(n_seqs <= 65535, "%s: at most 65535 sequences per launch", op);
  if (n_seqs == 0 || hv == 0) return MVB_OK;

  RecParams p;
  p.q = q->data; p.k = k->data; p.v = v->data; p.g = g->data; p.beta = beta->data; p.o = o->data;
  p.state = static_cast<float*>(state->data);
  p.state_idx = static_cast<const int32_t*>(idx->data);
  p.cu_seqlens = cu ? static_cast<const int32_t*>(cu->data) : nullptr;
  p.sq_t = q->stride[0]; p.sq_h = q->stride[1]; p.sq_d = q->stride[2];
  p.sk_t = k->stride[0]; p.sk_h = k->stride[1]; p.sk_d = k->stride[2];
  p.sv_t = v->stride[0]; p.sv_h = v->stride[1]; p.sv_d = v->stride[2];
  p.so_t = o->stride[0]; p.so_h = o->stride[1]; p.so_d = o->stride[2];
  p.sg_t = g->stride[0]; p.sg_h = g->stride[1]; p.sb_t = beta->stride[0]; p.sb_h = beta->stride[1];
  p.ss_n = state->stride[0]; p.ss_h = state->stride[1]; p.ss_k = state->stride[2];
  p.hk = (int)hk; p.hv = (int)hv; p.vdim = (int)vd; p.l2norm = l2norm ? 1 : 0;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)kd);

  p.g_dtype = g->dtype;
  p.b_dtype = beta->dtype;
  p.gd = gd;
  int r = MVB_OK;
  switch (q->dtype) {
    case MVB_F32: r = dispatch_k<float>(p, kd, n_seqs, st); break;
    case MVB_BF16: r = dispatch_k<__nv_bfloat16>(p, kd, n_seqs, st); break;
    case MVB_F16: r = dispatch_k<__half>(p, kd, n_seqs, st); break;
  }
  if (r != MVB_OK) return r;
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}

}  // namespace mvb

extern "C" int mvb_fused_recurrent_gdn(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                       const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* recurrent_state,
                                       const mvb_tensor* recurrent_state_indices, mvb_tensor* o, float scale,
                                       int use_qk_l2norm, void* stream) {
  return mvb::run_recurrent("fused_recurrent_gdn", q, k, v, g, beta, recurrent_state, recurrent_state_indices,
                            nullptr, o, scale, use_qk_l2norm, mvb::GateDev{}, static_cast<cudaStream_t>(stream));
}

extern "C" int mvb_fused_recurrent_gdn_gated(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                             const mvb_tensor* a, const mvb_tensor* b, const mvb_tensor* a_log,
                                             const mvb_tensor* dt_bias, mvb_tensor* recurrent_state,
                                             const mvb_tensor* recurrent_state_indices, mvb_tensor* o, float scale,
                                             int use_qk_l2norm, void* stream) {
  mvb::GateDev gd;
  int rc = mvb::make_gate_dev("fused_recurrent_gdn_gated", a_log, dt_bias, v, q, &gd);
  if (rc) return rc;
  return mvb::run_recurrent("fused_recurrent_gdn_gated", q, k, v, a, b, recurrent_state, recurrent_state_indices,
                            nullptr, o, scale, use_qk_l2norm, gd, static_cast<cudaStream_t>(stream));
}
