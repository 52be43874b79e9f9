"""Python wrapper of the OneDNNFlashAttention op (TensorFlow), B200 build.

Same call as the reference's python/onednn_flash_tf/ops.py:63-115 (arguments,
defaults, validation, tile-size heuristic).  It calls the generated wrapper
``one_dnn_flash_attention`` -- the snake-case name TensorFlow derives from the
registered op name "OneDNNFlashAttention" -- where the reference calls
``flash_one_attention``, a name no op registration produces.
"""
from __future__ import annotations

from functools import lru_cache
from pathlib import Path

_DEFAULT_OP = Path(__file__).resolve().parent / "onednn_flash_tf_attention.so"


def select_tile_sizes(query_tokens: int, key_tokens: int | None = None) -> tuple[int, int]:
    """The reference's heuristic (ops.py:13-31); the GPU tiles are 128 x 128 regardless."""
    if query_tokens <= 0:
        raise ValueError("query_tokens must be positive")
    key_tokens = query_tokens if key_tokens is None else key_tokens
    if key_tokens <= 0:
        raise ValueError("key_tokens must be positive")
    if query_tokens <= 64 and key_tokens <= 64:
        return min(64, query_tokens), min(64, key_tokens)
    return min(32, query_tokens), min(64, key_tokens)


@lru_cache(maxsize=None)
def load_onednn_flash_op(path: str | None = None):
    import tensorflow as tf

    op_path = Path(path) if path else _DEFAULT_OP
    if not op_path.exists():
        raise FileNotFoundError(f"OneDNNFlash TensorFlow op not found: {op_path}")
    return tf.load_op_library(str(op_path))


def onednn_flash_attention(q, k, v, *, causal: bool = True, query_block_size: int | None = None,
                           key_block_size: int | None = None, use_onednn: bool = True, tile_kernel: str = "onednn",
                           qk_tile_layout: str | None = None, op_path: str | None = None):
    import tensorflow as tf

    if query_block_size is None or key_block_size is None:
        qs, ks = tf.TensorShape(q.shape), tf.TensorShape(k.shape)
        if qs.rank != 4 or ks.rank != 4:
            raise ValueError("q and k must be rank 4 [B,H,T,D] tensors")
        if qs[2] is None or ks[2] is None:
            raise ValueError("query_block_size/key_block_size must be provided when q/k token dimensions are dynamic")
        hq, hk = select_tile_sizes(int(qs[2]), int(ks[2]))
        query_block_size = hq if query_block_size is None else query_block_size
        key_block_size = hk if key_block_size is None else key_block_size
    if qk_tile_layout is None:
        qk_tile_layout = "strided_k"
    if qk_tile_layout not in {"strided_k", "copied_transposed", "brgemm_transformed_k"}:
        raise ValueError("qk_tile_layout must be 'strided_k', 'copied_transposed', or 'brgemm_transformed_k'")
    if tile_kernel not in {"onednn", "onednn_brgemm"}:
        raise ValueError("tile_kernel must be 'onednn' or 'onednn_brgemm'")
    if tile_kernel == "onednn_brgemm" and qk_tile_layout == "strided_k":
        raise ValueError("tile_kernel='onednn_brgemm' does not support qk_tile_layout='strided_k'; "
                         "use 'copied_transposed' or 'brgemm_transformed_k'")
    ops = load_onednn_flash_op(str(op_path) if op_path else None)
    return ops.one_dnn_flash_attention(q, k, v, causal=causal, query_block_size=query_block_size,
                                       key_block_size=key_block_size, use_onednn=use_onednn,
                                       tile_kernel=tile_kernel, qk_tile_layout=qk_tile_layout)
