"""vidax_b200 -- the attention hot path of vidax, rebuilt for NVIDIA B200 (sm_100a).

Public API (same names and arguments as vidax.core.attention and
vidax.models.ltx2_5.diffusion_vae.neighborhood_attention_3d, on torch CUDA
tensors):

    dot_product_attention, local_attention, chunk_by_rank
"""
from .attention import (  # noqa: F401
    attention_flops,
    chunk_by_rank,
    dot_product_attention,
    flash_attention,
    local_attention,
)

__version__ = "0.1.0"
