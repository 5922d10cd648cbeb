"""statespectre_b200: a GPU tensor-offload and model-state runtime for NVIDIA B200.

Layers (bottom up):
  csrc/                 C++ daemon (offloadd), rank agent, sm_100a kernels
  _C                    native extension (agent, in-process daemon, kernels)
  _wire                 Python mirror of the control-plane wire schema
  api                   offload_context / Off / handles / canonical keys
  _rollout              RolloutWeightClient (sealed-version pulls)
  ops/                  kernel-level entry points on torch tensors
  parallel/             NVLink data plane: peer buffers, DP dedup, weight sync
  models/               shapes of the workloads (Llama-3-8B, Qwen2.5-32B, KV cache)
  utils/                timing, GPU clock sampling, config helpers
"""

from .api import (INTERNAL_STREAM, CanonicalHandle, CanonicalKey, DedupPolicy, ManagedRecord, ModelRole, Off,
                  OffloadHandle, PrefetchHandle, offload_context)
from ._rollout import RolloutWeightClient
from .daemon import DaemonClient, DaemonProcess, in_process_daemon, launch_daemon

__version__ = "0.1.0"

__all__ = [
    "offload_context", "Off", "OffloadHandle", "PrefetchHandle", "ManagedRecord", "CanonicalKey", "DedupPolicy",
    "ModelRole", "CanonicalHandle", "RolloutWeightClient", "INTERNAL_STREAM", "launch_daemon", "in_process_daemon",
    "DaemonProcess", "DaemonClient",
]
