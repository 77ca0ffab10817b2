"""rustane_b200 — B200-native (sm_100a) forward + cross-entropy engine for the
rustane decoder-only transformer, behind a C ABI (include/cuda_bridge.h).

The compute path is libcudabridge.so (tcgen05/TMA GEMMs with fused epilogues,
flash attention, vectorised row kernels). There is no CPU fallback.
"""
from .model import CONFIGS, ModelConfig, custom_config
from .bridge import CudaBridgeError, CB_INIT_NORMAL, CB_INIT_REFERENCE, load_library
from .engine import (CompiledKernels, ForwardResult, ForwardScheduler, LayerGrads,
                     LayerWeights, ModelForwardWorkspace, ModelGrads, ModelWeights, forward,
                     forward_backward, forward_losses, forward_only_ws, forward_ws,
                     nccl_unique_id)
from .checkpoint import load_checkpoint, save_checkpoint
from .parallel_bench import (ParallelBenchError, ParallelBenchRequest, ParallelBenchRunner,
                             ResolvedParallelBenchConfig)
from .data import (DeviceTokens, TokenBytes, TokenData, compute_bpb, random_position,
                   validate)

__all__ = [
    "CONFIGS", "ModelConfig", "custom_config", "CudaBridgeError", "CB_INIT_NORMAL",
    "CB_INIT_REFERENCE", "load_library", "CompiledKernels", "ForwardResult", "ForwardScheduler",
    "LayerWeights", "ModelForwardWorkspace", "ModelWeights", "forward", "forward_losses",
    "forward_only_ws", "forward_ws", "nccl_unique_id", "LayerGrads", "ModelGrads",
    "forward_backward", "load_checkpoint", "save_checkpoint",
    "DeviceTokens", "TokenBytes", "TokenData", "compute_bpb", "random_position", "validate",
    "ParallelBenchError", "ParallelBenchRequest", "ParallelBenchRunner",
    "ResolvedParallelBenchConfig",
]
