"""switchyard (B200): Block Attention Residuals on sm_100a.

A from-scratch B200-native implementation of the Block AttnRes operator behind
the Python API of ``sabdulmajid/blackwell-switchyard``'s ``switchyard.triton_op``:
``block_attn_res_triton`` (autograd), ``block_attn_res_batched`` (output only),
``BlockAttnResTriton`` and ``speed_of_light``. The kernels are hand-written CUDA
for sm_100a in ``csrc/`` behind the C ABI in ``include/switchyard_b200.h``.
"""

from .triton_op import (
    DEFAULT_EPS,
    BlockAttnResTriton,
    block_attn_res_batched,
    block_attn_res_triton,
    speed_of_light,
)
from .arena import stage_partial
from .two_phase import attn_with_stats, block_attn_res_batched_train, merge_online_softmax

__version__ = "0.1.0"

__all__ = [
    "__version__",
    "DEFAULT_EPS",
    "BlockAttnResTriton",
    "block_attn_res_batched",
    "block_attn_res_triton",
    "speed_of_light",
    "attn_with_stats",
    "merge_online_softmax",
    "block_attn_res_batched_train",
    "stage_partial",
]
