// Entry point of the chunked gated delta rule (prefill).
//
// bf16/fp16 inputs with K = V = 128 (the Qwen3.5 linear-attention heads) run the
// tensor-core kernel of gdn_chunk_tc.cu; fp32 inputs and other head sizes run the
// token-serial recurrence of gdn_recurrent.cu (exact fp32 math, same results).
//
// Precision of the tensor-core path: the input-side contractions ([q;k]k^T and the U/W
// products) take the bf16/fp16 inputs as they are, with the 64x64 triangular factors split
// into 16-bit hi + lo parts; the state-side contractions take fp16 operands (the fp16 copy
// of the state, q', k', W, v_new, Aqk: 2^-11 relative instead of bf16's 2^-8); every
// accumulator is fp32.  This keeps the final fp32 state within 1e-3 relative (measured
// ~2e-4) of the exact recurrence.
#include "common.cuh"

namespace mvb {

int check_gdn(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
              const mvb_tensor* beta, const mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
              const mvb_tensor* o, int64_t* n_seqs_out);
int run_recurrent(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                  const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx,
                  const mvb_tensor* cu, mvb_tensor* o, float scale, int l2norm, const GateDev& gd, cudaStream_t st);
int make_gate_dev(const char* op, const mvb_tensor* a_log, const mvb_tensor* dt_bias, const mvb_tensor* v,
                  const mvb_tensor* q, GateDev* out);
bool chunk_tc_supported(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
                        const mvb_tensor* beta, const mvb_tensor* state, const mvb_tensor* o);
int launch_chunk_tc(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
                    const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
                    mvb_tensor* o, float scale, int l2norm, int64_t n_seqs, int* work, size_t work_bytes,
                    const GateDev& gd, cudaStream_t st, const NormDev& nd);
size_t chunk_gdn_workspace_bytes(int grid);

int run_chunk(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
              const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
              mvb_tensor* o, float scale, int l2norm, void* ws, size_t ws_bytes, const GateDev& gd,
              cudaStream_t st, const NormDev& nd = NormDev{}) {
  if (cu == nullptr) MVB_FAIL(MVB_ERR_ARG, "%s: cu_seqlens is NULL", op);
  int64_t n_seqs = 0;
  int rc = check_gdn(op, q, k, v, g, beta, state, idx, cu, o, &n_seqs);
  if (rc) return rc;
  if (nd.z != nullptr)  // the output norm exists in the tensor-core kernel only
    MVB_CHECK_SUPPORTED(chunk_tc_supported(q, k, v, g, beta, state, o),
                        "%s: the fused output norm needs the tensor-core layout (16-bit q/k/v, K = V = 128, "
                        "unit inner strides, 16-byte aligned rows)", op);
  if (!chunk_tc_supported(q, k, v, g, beta, state, o)) {
    set_path(MVB_OP_CHUNK_GDN, MVB_PATH_SERIAL,
             "dtype, head size or layout outside the tensor-core kernel (16-bit q/k/v, K = V = 128, "
             "unit inner strides, 16-byte aligned rows)");
    return run_recurrent(op, q, k, v, g, beta, state, idx, cu, o, scale, l2norm, gd, st);
  }
  if (n_seqs == 0 || v->shape[1] == 0) return MVB_OK;
  MVB_CHECK_ARG(ws == nullptr || (ws_bytes >= 8 && (reinterpret_cast<uintptr_t>(ws) & 3) == 0),
                "%s: workspace must be at least 8 bytes, 4-byte aligned", op);
  rc = launch_chunk_tc(q, k, v, g, beta, state, idx, cu, o, scale, l2norm, n_seqs, static_cast<int*>(ws), ws_bytes, gd,
                       st, nd);
  if (rc < 0 && nd.z != nullptr) MVB_FAIL(MVB_ERR_CUDA, "%s: the TMA descriptors of q/k/v could not be built", op);
  if (rc < 0) {
    set_path(MVB_OP_CHUNK_GDN, MVB_PATH_SERIAL, "the TMA descriptors of q/k/v could not be built");
    return run_recurrent(op, q, k, v, g, beta, state, idx, cu, o, scale, l2norm, gd, st);
  }
  set_path(MVB_OP_CHUNK_GDN, MVB_PATH_TENSOR_CORE, "");
  return rc;
}

}  // namespace mvb

extern "C" size_t mvb_chunk_gated_delta_rule_workspace_size(void) {
  return mvb::chunk_gdn_workspace_bytes(mvb::num_sms());
}

extern "C" int mvb_chunk_gated_delta_rule(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                          const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* recurrent_state,
                                          const mvb_tensor* recurrent_state_indices, const mvb_tensor* cu_seqlens,
                                          mvb_tensor* o, float scale, int use_qk_l2norm, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  return mvb::run_chunk("chunk_gated_delta_rule", q, k, v, g, beta, recurrent_state, recurrent_state_indices,
                        cu_seqlens, o, scale, use_qk_l2norm, workspace, workspace_bytes, mvb::GateDev{},
                        static_cast<cudaStream_t>(stream));
}

extern "C" int mvb_chunk_gated_delta_rule_gated(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                                const mvb_tensor* a, const mvb_tensor* b, const mvb_tensor* a_log,
                                                const mvb_tensor* dt_bias, mvb_tensor* recurrent_state,
                                                const mvb_tensor* recurrent_state_indices,
                                                const mvb_tensor* cu_seqlens, mvb_tensor* o, float scale,
                                                int use_qk_l2norm, void* workspace, size_t workspace_bytes,
                                                void* stream) {
  mvb::GateDev gd;
  int rc = mvb::make_gate_dev("chunk_gated_delta_rule_gated", a_log, dt_bias, v, q, &gd);
  if (rc) return rc;
  return mvb::run_chunk("chunk_gated_delta_rule_gated", q, k, v, a, b, recurrent_state, recurrent_state_indices,
                        cu_seqlens, o, scale, use_qk_l2norm, workspace, workspace_bytes, gd,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int mvb_gated_deltanet_prefill(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                          const mvb_tensor* a, const mvb_tensor* b, const mvb_tensor* a_log,
                                          const mvb_tensor* dt_bias, mvb_tensor* recurrent_state,
                                          const mvb_tensor* recurrent_state_indices, const mvb_tensor* cu_seqlens,
                                          const mvb_tensor* z, const mvb_tensor* norm_weight, float norm_eps,
                                          mvb_tensor* out, float scale, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  using namespace mvb;
  const char* op = "gated_deltanet_prefill";
  GateDev gd;
  int rc = make_gate_dev(op, a_log, dt_bias, v, q, &gd);
  if (rc) return rc;
  if ((rc = check_tensor(z, op, "z", 3)) || (rc = check_tensor(norm_weight, op, "norm_weight", 1)) ||
      (rc = check_tensor(out, op, "out", 3)))
    return rc;
  MVB_CHECK_ARG(z->shape[0] == v->shape[0] && z->shape[1] == v->shape[1] && z->shape[2] == v->shape[2] &&
                    z->dtype == v->dtype,
                "%s: z must be [T, Hv, V] in the dtype of v", op);
  MVB_CHECK_ARG(norm_weight->shape[0] == v->shape[2] && norm_weight->stride[0] == 1 &&
                    (norm_weight->dtype == MVB_F32 || norm_weight->dtype == v->dtype),
                "%s: norm_weight must be a contiguous [V] of float32 or the dtype of v", op);
  MVB_CHECK_SUPPORTED(z->stride[2] == 1 && z->stride[1] % 8 == 0 && z->stride[0] % 8 == 0 && aligned16(z->data),
                      "%s: z rows must be contiguous and 16-byte aligned", op);
  NormDev nd;
  nd.z = z->data; nd.z_t = z->stride[0]; nd.z_h = z->stride[1];
  nd.w = norm_weight->data; nd.w_dt = norm_weight->dtype; nd.eps = norm_eps;
  return run_chunk(op, q, k, v, a, b, recurrent_state, recurrent_state_indices, cu_seqlens, out, scale, 1, workspace,
                   workspace_bytes, gd, static_cast<cudaStream_t>(stream), nd);
}
