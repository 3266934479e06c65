/*
 * myvllm_b200 -- C ABI of the B200 (sm_100a) attention hot-path kernels.
 *
 * One entry point per reference op.  Every entry point takes plain tensor
 * descriptors (device pointer + dtype + shape + strides in elements), enqueues its
 * kernels on the given CUDA stream (`void*` = cudaStream_t, NULL = legacy default
 * stream) and returns a status code.  Nothing here allocates device memory or
 * synchronises the host, except mvb_ipc_alloc, whose job is to allocate the shareable
 * all-reduce buffer; callers own every buffer (outputs, states, workspaces).
 *
 * Reference interfaces replaced (paths relative to the reference project, `m/` =
 * `src/myvllm/`):
 *   mvb_causal_conv1d_fn        m/ops/causal_conv1d.py:221-273       causal_conv1d_fn
 *   mvb_causal_conv1d_update    m/ops/causal_conv1d.py:434-470       causal_conv1d_update
 *   mvb_chunk_gated_delta_rule  m/ops/gated_delta_rule/gated_delta_rule.py:31-66
 *   mvb_gated_deltanet_prefill  m/layers/linear_attention.py:107-121 chunk GDN + RMSNormGated of the
 *                               prefill branch (gates, q/k norm and output norm in the kernel)
 *   mvb_gated_deltanet_decode   m/layers/linear_attention.py:85-123  decode branch of GatedDeltaNet
 *                               (conv update + l2norm + gates + recurrence + RMSNormGated)
 *   mvb_fused_recurrent_gdn     m/ops/gated_delta_rule/fused_recurrent_gdn.py:105-166
 *                               (also recurrent_gated_delta_rule, gated_delta_rule.py:69-92)
 *   mvb_flash_attention_prefill m/ops/full_attention.py:114-173      flash_attention_prefill
 *   mvb_paged_attention_decode  m/ops/full_attention.py:282-335      paged_flash_attention_decode
 *   mvb_paged_attention_prefill m/ops/full_attention.py:454-512      paged_flash_attention_prefill
 *   mvb_store_kvcache           (no kernel in the reference; layout from m/ops/full_attention.py:186-195,
 *                                slot_mapping convention from m/utils/context.py:15)
 *   mvb_rmsnorm_gated           m/layers/norm.py:44-58                RMSNormGated.forward
 *   mvb_rmsnorm                 m/layers/norm.py:6-41                 RMSNorm.forward
 *   mvb_rmsnorm_rope            m/layers/full_attention.py:49-64      q_norm/k_norm + rotary
 *   mvb_allreduce_oneshot       m/layers/linear.py:159-164            the dist.all_reduce of
 *                                                                     RowParallelLinear.forward
 *   mvb_linear_allreduce        m/layers/linear.py:159-164            F.linear + dist.all_reduce of
 *                                                                     RowParallelLinear.forward, fused
 *
 * Conventions kept from the reference:
 *   - index tensors (cu_seqlens, *_indices, block_tables, context_lens, slot_mapping) are int32;
 *   - cu_seqlens[0] = 0, cu_seqlens[n_seqs] = total tokens;
 *   - conv_state [S_max, W-1, dim], recurrent_state [S_max, Hv, K, V] (fp32), mutated in
 *     place at the rows named by the index tensors;
 *   - paged caches [n_blocks, block_size, Hkv, D]; slot = block * block_size + offset, -1 = skip;
 *   - v-head h uses k-head h / (Hv / Hk); q-head h uses kv-head h / (Hq / Hkv).
 */
#ifndef MYVLLM_B200_H_
#define MYVLLM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define MVB_OK 0
#define MVB_ERR_ARG 1          /* malformed argument: shape/dtype/stride mismatch, null pointer */
#define MVB_ERR_UNSUPPORTED 2  /* well-formed but outside what the kernels implement */
#define MVB_ERR_CUDA 3         /* a CUDA runtime call or kernel launch failed */

/* dtypes */
#define MVB_F32 0
#define MVB_BF16 1
#define MVB_F16 2
#define MVB_I32 3

#define MVB_MAX_DIMS 6

typedef struct mvb_tensor {
  void* data;                     /* device pointer; may be NULL only if some dim is 0 */
  int32_t dtype;                  /* MVB_F32 / MVB_BF16 / MVB_F16 / MVB_I32 */
  int32_t ndim;
  int64_t shape[MVB_MAX_DIMS];
  int64_t stride[MVB_MAX_DIMS];   /* in elements */
} mvb_tensor;

/* Library version (major*10000 + minor*100 + patch). */
int mvb_version(void);

/* Message for the last non-zero status returned on the calling host thread. */
const char* mvb_last_error(void);

/* Varlen causal depthwise conv (width 2 <= W <= 6) + SiLU over packed sequences.
 * x [T, dim]; weight [dim, W]; conv_state [S_max, W-1, dim] (read as history, then
 * overwritten with the last W-1 inputs of each sequence); conv_state_indices [S];
 * cu_seqlens [S+1]; out [T, dim] (same dtype as x).  activation: 1 = SiLU, 0 = none. */
int mvb_causal_conv1d_fn(const mvb_tensor* x, const mvb_tensor* weight, mvb_tensor* conv_state,
                         const mvb_tensor* conv_state_indices, const mvb_tensor* cu_seqlens,
                         mvb_tensor* out, int activation, void* stream);

/* One token per sequence: x [S, dim]; shifts conv_state[idx] in place; out [S, dim]. */
int mvb_causal_conv1d_update(const mvb_tensor* x, const mvb_tensor* weight, mvb_tensor* conv_state,
                             const mvb_tensor* conv_state_indices, mvb_tensor* out, int activation,
                             void* stream);

/* Chunked gated delta rule (prefill).  q,k [T, Hk, K]; v [T, Hv, V]; g, beta [T, Hv]
 * (g = natural-log decay); recurrent_state [S_max, Hv, K, V] fp32 -- the rows
 * recurrent_state_indices[s] are read as the initial state and overwritten with the
 * final state; cu_seqlens [S+1]; o [T, Hv, V] (dtype of v).  scale <= 0 means K^-0.5.
 * use_qk_l2norm != 0 applies the layer's q/k L2 normalisation (x * rsqrt(sum x^2 + 1e-6),
 * m/layers/linear_attention.py:113-114) inside the kernel.
 * workspace: NULL, or zero-initialised device memory that the kernel keeps ready for the
 * next launch:
 *   >= mvb_chunk_gated_delta_rule_workspace_size() bytes: the (sequence, v-head) chains are
 *      balanced over the SMs.  Laid end to end, they are cut into one equal span per pair
 *      of SMs (which run the two v-heads of a k-head side by side); a chain cut at a span
 *      boundary runs its first part on one SM and its rest on the next pair, the state
 *      passing through recurrent_state under a flag in the workspace (cooperative launch,
 *      or whole chains through the counter when the driver refuses one; results are
 *      bit-identical to whole-chain scheduling);
 *   8 bytes up to that: a work counter, whole chains scheduled dynamically, longest first;
 *   NULL: whole chains round-robin.
 * Launches that share one workspace must be ordered (same stream). */
int mvb_chunk_gated_delta_rule(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                               const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* recurrent_state,
                               const mvb_tensor* recurrent_state_indices, const mvb_tensor* cu_seqlens,
                               mvb_tensor* o, float scale, int use_qk_l2norm, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Bytes of workspace the chunked gated delta rule entry points need on the current device
 * for the balanced schedule (a few hundred bytes; no counterpart in the reference, whose
 * chunk pipeline loops over chunks on the host, m/ops/gated_delta_rule/h.py:195-265). */
size_t mvb_chunk_gated_delta_rule_workspace_size(void);

/* Recurrent gated delta rule, one token per sequence (decode).  q,k [S, Hk, K];
 * v [S, Hv, V]; g, beta [S, Hv]; state [S_max, Hv, K, V] fp32 updated in place;
 * o [S, Hv, V].  scale <= 0 means K^-0.5; use_qk_l2norm as above. */
int mvb_fused_recurrent_gdn(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                            const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* recurrent_state,
                            const mvb_tensor* recurrent_state_indices, mvb_tensor* o, float scale,
                            int use_qk_l2norm, void* stream);

/* The two GDN entry points above with the gates formed in the kernel from the layer's raw
 * projections, as GatedDeltaNet does before calling them (m/layers/linear_attention.py:89-90):
 * a, b [T, Hv] (fp32 or the dtype of q) take the places of g, beta, and
 *   g = -exp(A_log[h]) * softplus(a + dt_bias[h]),  beta = sigmoid(b) rounded to b's dtype;
 * A_log, dt_bias [Hv] (fp32 or the dtype of q).  Saves the layer's elementwise gate kernels. */
int mvb_chunk_gated_delta_rule_gated(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                     const mvb_tensor* a, const mvb_tensor* b, const mvb_tensor* a_log,
                                     const mvb_tensor* dt_bias, mvb_tensor* recurrent_state,
                                     const mvb_tensor* recurrent_state_indices, const mvb_tensor* cu_seqlens,
                                     mvb_tensor* o, float scale, int use_qk_l2norm, void* workspace,
                                     size_t workspace_bytes, void* stream);
int mvb_fused_recurrent_gdn_gated(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                  const mvb_tensor* a, const mvb_tensor* b, const mvb_tensor* a_log,
                                  const mvb_tensor* dt_bias, mvb_tensor* recurrent_state,
                                  const mvb_tensor* recurrent_state_indices, mvb_tensor* o, float scale,
                                  int use_qk_l2norm, void* stream);

/* The decode step of a Gated DeltaNet layer in one kernel: causal_conv1d_update (+ SiLU) ->
 * q/k L2 norm -> in-kernel gates -> recurrent gated delta rule -> RMSNormGated, i.e. the
 * decode branch of GatedDeltaNet.forward (m/layers/linear_attention.py:85-123, with
 * RMSNormGated from m/layers/norm.py:44-58), whose separate ops it replaces.
 * qkv [S, 2 Hk K + Hv V] the input projection's q | k | v channels (16-bit, unit channel
 * stride, 16-byte aligned rows); conv_weight [conv_dim, W] (2 <= W <= 6); conv_state
 * [S_max, W-1, conv_dim] and recurrent_state [S_max, Hv, K, V] (fp32), both updated in
 * place at conv_state_indices / recurrent_state_indices; a, b [S, Hv] raw gate projections;
 * A_log, dt_bias [Hv]; z [S, Hv, V] the norm's gate; norm_weight [V]; out [S, Hv, V] =
 * RMSNormGated(o, z).  K = V = 128; scale <= 0 means K^-0.5.
 * counters / records: caller memory of at least the sizes mvb_gated_deltanet_decode_workspace_sizes
 * reports.  counters must be zero before the first call and are left at zero by every call
 * (keep them apart from any other use); records need no initial value (16-byte aligned).
 * Launches that share them must be ordered (same stream). */
int mvb_gated_deltanet_decode_workspace_sizes(int64_t n_seqs, int64_t num_k_heads, int64_t num_v_heads,
                                              size_t* counters_bytes, size_t* records_bytes);
int mvb_gated_deltanet_decode(const mvb_tensor* qkv, const mvb_tensor* conv_weight, mvb_tensor* conv_state,
                              const mvb_tensor* conv_state_indices, const mvb_tensor* a, const mvb_tensor* b,
                              const mvb_tensor* a_log, const mvb_tensor* dt_bias, mvb_tensor* recurrent_state,
                              const mvb_tensor* recurrent_state_indices, const mvb_tensor* z,
                              const mvb_tensor* norm_weight, float norm_eps, float scale, mvb_tensor* out,
                              void* counters, size_t counters_bytes, void* records, size_t records_bytes,
                              void* stream);

/* The prefill branch of a Gated DeltaNet layer after its conv: mvb_chunk_gated_delta_rule_gated
 * with the q/k L2 norm on and RMSNormGated(o, z) (m/layers/norm.py:44-58) applied to each
 * output tile before it is stored, i.e. GatedDeltaNet.forward's chunk_gated_delta_rule +
 * self.norm (m/layers/linear_attention.py:107-121).  Arguments as mvb_chunk_gated_delta_rule_gated,
 * plus z [T, Hv, V] (dtype of v, 16-byte aligned rows) and norm_weight [V]; out [T, Hv, V].
 * Needs the tensor-core layout (16-bit q/k/v, K = V = 128); MVB_ERR_UNSUPPORTED otherwise. */
int mvb_gated_deltanet_prefill(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* a,
                               const mvb_tensor* b, const mvb_tensor* a_log, const mvb_tensor* dt_bias,
                               mvb_tensor* recurrent_state, const mvb_tensor* recurrent_state_indices,
                               const mvb_tensor* cu_seqlens, const mvb_tensor* z, const mvb_tensor* norm_weight,
                               float norm_eps, mvb_tensor* out, float scale, void* workspace, size_t workspace_bytes,
                               void* stream);

/* Varlen (optionally causal) attention.  q [T, Hq, D]; k [T, Hkv, D]; v [T, Hkv, Dv];
 * cu_seqlens [S+1]; o [T, Hq, Dv] (dtype of q).  bf16/f16 only. */
int mvb_flash_attention_prefill(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                const mvb_tensor* cu_seqlens, float scale, int num_heads, int num_kv_heads,
                                int head_dim, int head_v_dim, int is_causal, mvb_tensor* o, void* stream);

/* Bytes of workspace mvb_paged_attention_decode needs for this problem size. */
size_t mvb_paged_attention_decode_workspace_size(int64_t n_seqs, int64_t num_kv_heads, int64_t head_v_dim,
                                                 int64_t max_context_len);

/* One query per sequence over a paged KV cache.  q [S, Hq, D]; k_cache [NB, bs, Hkv, D];
 * v_cache [NB, bs, Hkv, Dv]; block_tables [S, max_blocks]; context_lens [S];
 * o [S, Hq, Dv].  workspace: at least mvb_paged_attention_decode_workspace_size(...)
 * bytes of device memory (split-KV partial results), or NULL/0 to run unsplit.
 * max_context_len: an upper bound on context_lens (<= max_blocks * block_size). */
int mvb_paged_attention_decode(const mvb_tensor* q, const mvb_tensor* k_cache, const mvb_tensor* v_cache,
                               const mvb_tensor* block_tables, const mvb_tensor* context_lens, float scale,
                               int block_size, int64_t max_context_len, mvb_tensor* o, void* workspace,
                               size_t workspace_bytes, void* stream);

/* mvb_paged_attention_decode with the gated-attention output gate applied where o is
 * written: o = attention * sigmoid(gate), gate [S, Hq, Dv] (dtype of q, unit last stride),
 * in fp32 with one rounding.  Replaces the decode branch's paged_flash_attention_decode
 * (m/ops/full_attention.py:282-335) followed by the layer's o * sigmoid(gate). */
int mvb_paged_attention_decode_gated(const mvb_tensor* q, const mvb_tensor* k_cache, const mvb_tensor* v_cache,
                                     const mvb_tensor* block_tables, const mvb_tensor* context_lens, float scale,
                                     int block_size, int64_t max_context_len, const mvb_tensor* gate, mvb_tensor* o,
                                     void* workspace, size_t workspace_bytes, void* stream);

/* Context-split decode, for tensor parallelism past the number of kv heads, where the
 * reference asserts (m/layers/full_attention.py:34-35 requires num_kv_heads % tp == 0).
 * The n_parts ranks that hold copies of a kv head each attend, for all q heads of that kv
 * head, over every n_parts-th split of each context (splits s with s % n_parts == part),
 * instead of all of them attending over the whole context.  Out: o_part [S, Hq, Dv] fp32
 * (contiguous), this part's attention normalised within the part, and lse_part [S, Hq]
 * fp32 (contiguous), its log2-sum-exp (-inf where the part holds no keys).  workspace: at
 * least mvb_paged_attention_decode_part_workspace_size(...) bytes (required).  Other
 * arguments as mvb_paged_attention_decode. */
size_t mvb_paged_attention_decode_part_workspace_size(int64_t n_seqs, int64_t num_kv_heads, int64_t head_v_dim,
                                                      int64_t max_context_len, int n_parts);
int mvb_paged_attention_decode_part(const mvb_tensor* q, const mvb_tensor* k_cache, const mvb_tensor* v_cache,
                                    const mvb_tensor* block_tables, const mvb_tensor* context_lens, float scale,
                                    int block_size, int64_t max_context_len, int part, int n_parts,
                                    mvb_tensor* o_part, mvb_tensor* lse_part, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* This rank's share of the context-split attention: o = o_part * w (* sigmoid(gate)),
 * w = 2^(lse_own - M) / sum_j 2^(lse_j - M) over the parts j of lse_parts [n_parts, S, Hq]
 * (fp32, rows contiguous; lse_own = lse_parts[part]), M their max.  The shares of all parts
 * sum to the attention over the whole context, so each rank projects its share and the
 * all-reduce after the output projection (m/layers/linear.py:159-164) adds them.  o [S, Hq,
 * Dv] bf16/fp16; gate as in mvb_paged_attention_decode_gated, or NULL. */
int mvb_attention_merge_parts(const mvb_tensor* o_part, const mvb_tensor* lse_parts, int part, const mvb_tensor* gate,
                              mvb_tensor* o, void* stream);

/* Allocation-free variant of mvb_paged_attention_decode (no counterpart in the reference).
 * For callers that may not allocate device memory when they decode: the split-KV partial
 * results go to a fixed 16 MiB array in the library's device image instead of a caller
 * workspace.  A context is split only as far as that array holds the partials of every
 * (sequence, kv head): n_splits * n_seqs * num_kv_heads * (head_v_dim + 1) * 64 bytes
 * <= 16 MiB; when not even two splits fit, the decode runs unsplit, which needs no scratch.
 * The first call on each device looks up the array's device address (make it before any
 * stream capture).  All calls share the array: calls that overlap on the GPU race. */
int mvb_paged_attention_decode_noalloc(const mvb_tensor* q, const mvb_tensor* k_cache, const mvb_tensor* v_cache,
                                       const mvb_tensor* block_tables, const mvb_tensor* context_lens, float scale,
                                       int block_size, int64_t max_context_len, mvb_tensor* o, void* stream);

/* Prefill continuing from a paged cache: the L_s queries of sequence s sit at positions
 * context_lens[s] - L_s + i and attend causally to cached tokens [0, context_lens[s]).
 * q [T, Hq, D]; cu_seqlens [S+1]; other arguments as in mvb_paged_attention_decode. */
int mvb_paged_attention_prefill(const mvb_tensor* q, const mvb_tensor* k_cache, const mvb_tensor* v_cache,
                                const mvb_tensor* block_tables, const mvb_tensor* context_lens,
                                const mvb_tensor* cu_seqlens, float scale, int block_size, mvb_tensor* o,
                                void* stream);

/* Scatter k [T, Hkv, D], v [T, Hkv, Dv] into k_cache/v_cache [NB, bs, Hkv, D*] at
 * slot_mapping[t] (int32; -1 = skip). */
int mvb_store_kvcache(const mvb_tensor* k, const mvb_tensor* v, mvb_tensor* k_cache, mvb_tensor* v_cache,
                      const mvb_tensor* slot_mapping, void* stream);

/* out = x * rsqrt(mean(x^2) + eps) * weight * silu(gate), per row of the last dim.
 * x, gate, out [N, D]; weight [D]. */
int mvb_rmsnorm_gated(const mvb_tensor* x, const mvb_tensor* gate, const mvb_tensor* weight, float eps,
                      mvb_tensor* out, void* stream);

/* s = x (+ residual, written back to residual); out = s * rsqrt(mean(s^2) + eps) * (weight
 * [+ 1 with zero_centered_gamma]), per row.  x, residual, out [N, D] 16-bit; weight [D].
 * Replaces RMSNorm.forward (m/layers/norm.py:6-41). */
int mvb_rmsnorm(const mvb_tensor* x, mvb_tensor* residual, const mvb_tensor* weight, float eps,
                int zero_centered_gamma, mvb_tensor* out, void* stream);

/* The q/k norm and partial rotary of full attention in one pass (the layer's
 * q_norm / k_norm, m/layers/full_attention.py:49-64, then apply_rotary_pos_emb on the first
 * rotary_dim dims, m/layers/rotary_embedding.py:6-31): x, out [T, H, D] (D <= 256; head
 * rows 16-byte aligned); weight [D] as mvb_rmsnorm; cos, sin [T, rotary_dim / 2] fp32 with
 * rotary_dim a power of two in [16, D].  Half-split rotation: for c < rotary_dim / 2,
 * (y_c, y_{c+r/2}) -> (y_c cos_c - y_{c+r/2} sin_c, y_{c+r/2} cos_c + y_c sin_c); fp32
 * math, one rounding. */
int mvb_rmsnorm_rope(const mvb_tensor* x, const mvb_tensor* weight, float eps, int zero_centered_gamma,
                     const mvb_tensor* cos, const mvb_tensor* sin, mvb_tensor* out, void* stream);

/* Diagnostics. */

/* Kernel family the last call of an op ran on the calling host thread.  Most ops have one
 * path; these have a fallback for layouts their main kernel does not take:
 *   MVB_OP_CHUNK_GDN      mvb_chunk_gated_delta_rule[_gated]: tensor-core (tcgen05) kernel,
 *                         else the token-serial fp32 recurrence (same math, far slower);
 *   MVB_OP_FA_PREFILL     mvb_flash_attention_prefill: tcgen05 + TMA kernel, else mma.sync;
 *   MVB_OP_PAGED_PREFILL  mvb_paged_attention_prefill: tcgen05 + TMA kernel, else mma.sync.
 * Returns MVB_PATH_* (MVB_PATH_NONE before the first call), or -1 for an unknown op.
 * *reason (if reason != NULL) gets why the fallback was taken ("" on the main path); the
 * string stays valid until the next call of that op on this thread. */
#define MVB_OP_CHUNK_GDN 0
#define MVB_OP_FA_PREFILL 1
#define MVB_OP_PAGED_PREFILL 2
#define MVB_PATH_NONE 0
#define MVB_PATH_TENSOR_CORE 1  /* tcgen05.mma with TMEM accumulators, TMA-fed */
#define MVB_PATH_SERIAL 2       /* token-serial recurrence on CUDA cores */
#define MVB_PATH_MMA_SYNC 3     /* warp-level mma.sync kernel */
int mvb_last_path(int op, const char** reason);

/* Reads and clears the kernels' device error word: 0 = no error; 1 = a bounded wait on a
 * tensor-core completion barrier gave up (the kernel abandoned its work and freed its
 * tensor memory).  Synchronises with the device. */
int mvb_device_status(int* status);

/* ---- tensor-parallel all-reduce over NVLink peer memory ----
 * One buffer per rank, shared through CUDA IPC: each rank calls mvb_ipc_alloc, sends the
 * 64-byte handle to the others (any host channel), and maps theirs with mvb_ipc_open.
 * mvb_allreduce_oneshot then sums a bf16/f16 tensor over the ranks: every rank launches it
 * on the same sequence of sizes, in the same order (the buffers carry per-block call
 * counters, so a launch can be captured in a CUDA graph; every launch runs the same 64
 * blocks, so calls of different sizes may follow each other with no host synchronisation).
 * Waits for peers are bounded: one that gives up sets the device error word
 * (mvb_device_status) and writes this rank's own input into that part of out instead of the
 * sum.  No multicast: peer data moves by plain loads. */
#define MVB_AR_MAX_RANKS 8
typedef struct mvb_allreduce_peers {
  int32_t world;                     /* ranks taking part, 2..MVB_AR_MAX_RANKS */
  int32_t rank;                      /* this rank */
  void* bufs[MVB_AR_MAX_RANKS];      /* every rank's buffer as mapped in this process (bufs[rank]: own) */
  size_t buf_bytes;                  /* size of each buffer */
} mvb_allreduce_peers;

/* Buffer size for messages of up to max_message_bytes. */
size_t mvb_allreduce_buffer_bytes(size_t max_message_bytes);
/* cudaMalloc'd, zeroed buffer of `bytes` and its IPC handle (64 bytes written to `handle`). */
int mvb_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
int mvb_ipc_free(void* dev_ptr);
/* Maps another process's buffer from its 64-byte handle; mvb_ipc_close unmaps it. */
int mvb_ipc_open(const void* handle, void** dev_ptr);
int mvb_ipc_close(void* dev_ptr);
/* out = sum over ranks of inp (contiguous, same shape and dtype; bytes a multiple of 16 and
 * at most the buffer's slot size).  out may not alias inp. */
int mvb_allreduce_oneshot(const mvb_allreduce_peers* peers, const mvb_tensor* inp, mvb_tensor* out,
                          void* stream);

/* Row-parallel projection fused with its all-reduce, one kernel per rank:
 * out = sum over ranks r of x_r w_r^T, the output projection of a tensor-parallel layer and
 * the dist.all_reduce after it (RowParallelLinear.forward, m/layers/linear.py:159-164).
 * x [M, K] (this rank's input shard), w [N, K] (this rank's weight shard), out [M, N]; 16-bit,
 * contiguous 16-byte aligned rows; M <= 128, N = 64 d with d dividing 128, K a multiple of
 * 64 (128 / d).  The GEMM runs on the tensor cores (tcgen05, TMA-fed from this GPU's memory);
 * the ranks' fp32 partial tiles are summed through peer loads in a fixed order, so every
 * rank gets the same bits.  Buffers: mvb_ipc_alloc(mvb_linear_allreduce_buffer_bytes()) per
 * rank, shared as for mvb_allreduce_oneshot; every rank calls with the same shapes in the
 * same order (world 1 is allowed: the same kernel as a single-rank projection).  All 128
 * CTAs of a launch must be resident together (no concurrent kernel
 * may hold the GPU's SMs).  A wait for a peer that gives up sets the device error word and
 * leaves zeros in that CTA's rows.  No multicast. */
size_t mvb_linear_allreduce_buffer_bytes(void);
int mvb_linear_allreduce(const mvb_allreduce_peers* peers, const mvb_tensor* x, const mvb_tensor* w, mvb_tensor* out,
                         void* stream);

/* Tensor-core self-test: D[128, n] = A B1 + (negate ? -1 : 1) A B2 on one CTA with
 * fp16 operands staged in the 128-byte-swizzle K-major (a_mn/b_mn = 0) or MN-major (= 1)
 * layouts the kernels use.  Storage: A [128][k] (K-major) or [k][128]; B [n][k] or [k][n];
 * D [128][n] fp32.  n, k in {64, 128}. */
int mvb_selftest_umma(const void* a, const void* b1, const void* b2, float* d, int n, int k, int a_mn, int b_mn,
                      int negate, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MYVLLM_B200_H_ */
