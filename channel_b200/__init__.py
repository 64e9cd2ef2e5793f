"""channel_b200 -- B200 (sm_100a) implementation of Sullux/channel's Q4
streaming-inference hot path behind a C-ABI (include/channel_cuda.h).

The CUDA library is built in-tree (``python -m channel_b200.build``); importing
the engine loads it and raises if it is missing -- there is no CPU fallback.
"""
from ._lib import ChannelError, load  # noqa: F401
from .engine import (  # noqa: F401
    DeviceRing,
    DeviceSampler,
    DynamicRingBuffer,
    GpuContext,
    GpuModelContext,
    LayerWeightsQ4,
    ModelConfig,
    TopKCandidate,
    config_12b,
    gpu_dispatch_forward_token,
    gpu_dispatch_prefill_batch,
)
