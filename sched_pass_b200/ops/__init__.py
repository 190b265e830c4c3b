"""Tensor-level entry points of the sm_100a kernels (see csrc/kernels)."""
from .kernels import (PREFILL_TILE_ROWS, KernelStatusError, Workspace, add_rmsnorm, argmax, attention_decode, attention_merge,
                      attention_prefill, check_status, embedding, linear, linear_add_rmsnorm, linear_qkv_rope,
                      rope_kv_append, row_counters, status_buffer, workspace)

__all__ = [
    "PREFILL_TILE_ROWS", "KernelStatusError", "Workspace", "add_rmsnorm", "argmax", "attention_decode", "attention_merge",
    "attention_prefill", "check_status", "embedding", "linear", "linear_add_rmsnorm", "linear_qkv_rope",
    "rope_kv_append", "row_counters", "status_buffer", "workspace",
]
