"""gdnr -- B200-native FP8-checkpoint replay for the GDN decode step.

Host side of the path: a drop-in mirror of the reference prototype's
operator API (zz774ever/fp8-replayssm-gdn-kernel,
prototype/gdn_replayssm_fp8_kernel.py) over the C ABI of libgdnr.so
(include/gdnr.h), whose kernels are hand-written CUDA for sm_100a.
"""

from ._lib import GdnrError, GdnrValueError, load as load_library  # noqa: F401
from .ops import (  # noqa: F401
    QuantizedCheckpoint,
    dequantize_checkpoint,
    fused_recurrent_gated_delta_rule_packed_decode,
    gdn_bf16_step,
    gdn_fused_step,
    gdn_prep_ring,
    gdn_replay_fp8,
    gdn_replay_fp8_split,
    gdn_replay_fp8_split_static,
    quantize_checkpoint,
    read_device_error,
)
from . import capture  # noqa: F401
from .shard import ShardPlan, gather_shards, max_over_ranks, shard_range  # noqa: F401
from .state import ReplayState  # noqa: F401

__version__ = "0.1.0"
