"""vidax_b200 -- the attention hot path of vidax, rebuilt for NVIDIA B200 (sm_100a).

Public API (same names and arguments as vidax.core.attention and
vidax.models.ltx2_5.diffusion_vae.neighborhood_attention_3d, on torch CUDA
tensors):

    dot_product_attention, local_attention, chunk_by_rank,
    sequence_parallel_self_attention, sequence_parallel_joint_self_attention,
    neighborhood_attention_3d

Mesh axes (vidax's `sp` axis inside shard_map) bind to torch.distributed
process groups with `register_axis(name, group)`.
"""
from .attention import (  # noqa: F401
    attention_flops,
    chunk_by_rank,
    dot_product_attention,
    flash_attention,
    local_attention,
)
from .hostio import attention_from_host  # noqa: F401
from .neighborhood import (  # noqa: F401
    ltx_neighborhood_attention,
    na3d_flops,
    neighborhood_attention_3d,
    neighborhood_attention_3d_slab,
)
from .na_parallel import neighborhood_attention_3d_sp  # noqa: F401
from .ulysses_qsplit import sequence_parallel_self_attention_qsplit  # noqa: F401
from .prologue import (  # noqa: F401
    attend,
    ltx_rope_freqs,
    norm_rope_pack,
    rms_norm_rope,
    rope3d_freqs,
)
from .ulysses import (  # noqa: F401
    axis_index,
    axis_size,
    register_axis,
    sequence_parallel_joint_self_attention,
    sequence_parallel_self_attention,
    sequence_parallel_self_attention_from_host,
    unregister_axis,
)

__version__ = "0.1.0"
