"""ffai_b200: B200-native Whisper attention (encoder self-attention, decoder
self-attention over the KV cache, decoder cross-attention) behind the C ABI
of libffai_attn.so.  See include/ffai_attn.h for the boundary.

    from ffai_b200 import attention, flash_attn
    out = attention.prefill(q, k, v, scale=0.125)          # tcgen05 kernel
    o = attention.decode(q, kcache, vcache, kv_len=448)    # split-KV decode
    o = flash_attn.attend_merged(q, kt, v)                 # reference surface
"""

from . import _abi  # noqa: F401

__all__ = ["attention", "flash_attn", "partition", "load"]


def load():
    """Load libffai_attn.so (raises ImportError if it has not been built)."""
    return _abi.load()
