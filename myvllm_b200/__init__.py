"""myvllm_b200: B200 (sm_100a) kernels for the attention hot path of myvllm.

The op and layer modules mirror the reference package layout so that
``myvllm.X.Y`` can be swapped for ``myvllm_b200.X.Y``:

  ops.causal_conv1d                         causal_conv1d_fn, causal_conv1d_update
  ops.gated_delta_rule.gated_delta_rule     chunk_gated_delta_rule, recurrent_gated_delta_rule
  ops.gated_delta_rule.fused_recurrent_gdn  fused_recurrent_gdn
  ops.full_attention                        flash_attention_prefill, paged_flash_attention_decode,
                                            paged_flash_attention_prefill
  ops.kv_cache                              store_kvcache (new; the reference has none)
  layers.*, cache.*, utils.context          layer modules, state cache and per-step context
"""

__version__ = "0.1.0"
