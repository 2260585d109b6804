"""BDH strict-tril attention kernels: the reference ``kernels`` package surface with a B200
(sm_100a) native backend (``BDH_ATTN_IMPL=cuda_sm100``, library ``libbdh_sm100.so``)."""

from .attention_dispatch import (
    DEFAULT_ATTN_AUTO_THRESHOLD,
    attn_auto_cold_threshold,
    attn_auto_enabled,
    attn_auto_threshold,
    backend_info,
    bdh_attn,
    bdh_attn_decode,
    bdh_rope_attn,
    bdh_rope_attn_decode,
    resolve_attn_impl,
    resolve_cold_impl,
    resolve_decode_impl,
)
from .attention_bwd import (
    RopeTrilSelfAttnFn,
    StrictTrilAttnFn,
    StrictTrilSelfAttnFn,
    analytic_tril_attn_backward,
    strict_tril_attn,
)
from .rope_dispatch import (
    backend_info as rope_backend_info,
    bdh_rope_rotate,
    bdh_rope_rotate_paired,
    resolve_rope_impl,
)
from .sm100_attn import (
    ext_status,
    has_cuda_ext,
    has_cuda_kernel,
    tril_decode,
    tril_score_v,
    tril_score_v_bwd,
)

__all__ = [
    "bdh_attn",
    "bdh_attn_decode",
    "bdh_rope_attn",
    "bdh_rope_attn_decode",
    "resolve_attn_impl",
    "resolve_cold_impl",
    "resolve_decode_impl",
    "attn_auto_threshold",
    "attn_auto_cold_threshold",
    "attn_auto_enabled",
    "DEFAULT_ATTN_AUTO_THRESHOLD",
    "backend_info",
    "strict_tril_attn",
    "StrictTrilAttnFn",
    "StrictTrilSelfAttnFn",
    "RopeTrilSelfAttnFn",
    "analytic_tril_attn_backward",
    "tril_score_v",
    "tril_decode",
    "tril_score_v_bwd",
    "has_cuda_ext",
    "has_cuda_kernel",
    "ext_status",
    "bdh_rope_rotate",
    "bdh_rope_rotate_paired",
    "resolve_rope_impl",
    "rope_backend_info",
]
