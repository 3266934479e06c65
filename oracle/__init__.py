"""CPU oracle for the myvllm attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the math of the reference ops that the CUDA
library replaces.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and
only as the checker or the timed CPU baseline.  The product path
(``myvllm_b200``) never imports it and has no CPU fallback.

Every function cites the reference file:line it follows (paths relative to the
reference project root, ``src/myvllm/`` abbreviated ``m/``).

Pinning (how the restatement itself is checked):
  * ``gdn.recurrent``      -- pinned bit-for-bit-ish (<=1e-6) to the reference's own
                              ``_fused_recurrent_gdn`` run under TRITON_INTERPRET=1
                              (golden fixture ``tests/golden/c0_gdn.npz``) and to
                              fla 0.5.1 ``naive_recurrent_gated_delta_rule``.
  * ``attention.paged_decode`` -- pinned to the reference's own
                              ``paged_flash_attention_decode`` under the interpreter
                              (``tests/golden/paged_decode.npz``).
  * ``gdn.chunked``        -- equal to ``gdn.recurrent`` to fp rounding, and to fla
                              ``naive_chunk_gated_delta_rule`` (golden ``c0_gdn.npz``).
  * ``conv``, ``attention.varlen``, ``attention.paged_prefill``, ``kv.store`` -- the
                              reference kernels do not run as written, so these are
                              restated from the reference source formulas and
                              cross-checked against independent implementations
                              (torch ``conv1d`` and ``scaled_dot_product_attention``,
                              fixtures in ``tests/golden/``); parity for these is
                              pinned by formula, not by reference output.
"""

from . import attention, conv, gdn, kv  # noqa: F401
