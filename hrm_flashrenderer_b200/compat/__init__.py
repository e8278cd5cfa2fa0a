"""Compatibility surfaces for code written against the reference's Python packages.

``compat.flashattention`` mirrors ``flashattention_custom.ops`` (``flash_attn``, ``flash_attn_paged``,
``paged_kv_append``) on this package's kernels; ``compat.llama_tp`` gives the reference torch TP engine's names
(``TPLlamaForCausalLM``, ``generate_tp``, ``greedy_select_token_distributed``, ``PagedKVCache``) on this package's
engine; ``compat.kernel_test`` holds the ``flash-kernel-test`` / ``flash-append-test`` console checks.
"""
from .flashattention import flash_attn, flash_attn_paged, paged_kv_append  # noqa: F401
