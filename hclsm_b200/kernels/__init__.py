"""Mirror of ``hclsm.kernels`` (hclsm/kernels/__init__.py:9-35) backed by sm_100a kernels."""
from .ssm_scan_kernel import ssm_scan, ssm_scan_fn  # noqa: F401
from .slot_attention_kernel import (  # noqa: F401
    SlotIterationParams,
    fold_query_into_keys,
    key_value_weights,
    project_keys_values,
    slot_attention_core,
    slot_attention_fn,
    slot_attention_iteration,
    slot_attention_iterations,
)

from .sparse_event_attn import (  # noqa: F401
    EventTransformer,
    event_detect,
    sparse_event_attention_fused,
    sparse_event_attn_fn,
)
from .level0 import level0_epilogue, level0_forward, masked_mean_pool  # noqa: F401

__all__ = ["sparse_event_attn_fn", "EventTransformer", "sparse_event_attention_fused", "event_detect", "ssm_scan_fn",
           "ssm_scan", "slot_attention_fn", "slot_attention_core", "SlotIterationParams", "slot_attention_iteration",
           "slot_attention_iterations", "fold_query_into_keys", "key_value_weights", "project_keys_values",
           "masked_mean_pool", "level0_epilogue", "level0_forward"]
