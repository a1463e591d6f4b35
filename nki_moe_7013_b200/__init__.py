"""B200-native (sm_100a) Qwen3-MoE decoder-layer hot path.

Host side: Python / PyTorch modules with the reference's forward signatures
(``moe.Qwen3MoeSparseMoeBlock`` for ``self.mlp(hidden_states, padding_mask)[0]``
at qwen.py:429, ``moe.ExpertMLPs`` for the blockwise / selective-loading seams
of qwen_with_nki.py).  Device side: hand-written CUDA kernels behind the C ABI
declared in ``include/qmoe.h`` (library ``_lib/libqmoe.so``).
"""
from .config import Qwen3MoeConfig  # noqa: F401

__all__ = ["Qwen3MoeConfig"]
