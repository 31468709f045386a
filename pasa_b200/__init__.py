"""pasa_b200: precision-allocated sparse attention forward on B200 (sm_100a).

Drop-in for ZHANGWENTAI/PASA's ``pisa_pg_attention``
(svg/kernels/triton/group_pisa_attention.py) and the HunyuanVideo token
placement (svg/models/hyvideo/placement.py), running hand-written CUDA
through the C ABI in ``include/pasa_b200.h``.
"""
from .ops import (  # noqa: F401
    dense_attention,
    hunyuan_hidden_states_placement,
    hunyuan_sparse_head_placement,
    piecewise_sparse_attention,
    pisa_pg_attention,
    pisa_pg_attention_host,
    pisa_pg_attention_range,
)

__all__ = [
    "dense_attention",
    "pisa_pg_attention",
    "pisa_pg_attention_host",
    "pisa_pg_attention_range",
    "piecewise_sparse_attention",
    "hunyuan_sparse_head_placement",
    "hunyuan_hidden_states_placement",
]
