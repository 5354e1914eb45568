"""VC-Attention forward on B200 (sm_100a): the ``b200_fp8`` backend.

Same public surface as czfsdg/vc-attention's ``vc_attention`` package
(``Config``, ``LayoutCache``, ``attention``; src/vc_attention/__init__.py:3-5).
"""
from .core import Config, LayoutCache, attention, to_layout_order
from .streamed import attention_streamed, check_streamed

__all__ = ["Config", "LayoutCache", "attention", "attention_streamed", "check_streamed", "to_layout_order"]
