"""mq: B200 (sm_100a) weight-quantised matmuls behind a C ABI (libmq.so), loaded with ctypes.

The operators mirror the reference's kernel interface (llama/kernels, qwen3moe/kernels,
bonsai/kernels): packed int4 / ternary weight buffers plus fp16 scales in the reference's own
byte layouts, fp32/fp16 activations, fp32 outputs. Torch tensors are used only as device
buffers. There is no CPU fallback: every operator raises MQError when libmq.so is missing or
no sm_100 device is present.
"""
from ._lib import MQError, lib, library_path  # noqa: F401
from .kernels import *  # noqa: F401,F403
from .moe import *  # noqa: F401,F403
from .ep import ExpertParallelMoE, expert_range  # noqa: F401
from .pack import *  # noqa: F401,F403
from .formats import GGUF, Manifest, read_file_to_device, read_gguf  # noqa: F401
