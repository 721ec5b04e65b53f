"""revealaiccl_b200 — B200-native progressive MoE communication framework.

Revealed-only progressive MoE AlltoAllv on 1-8 B200 GPUs (sm_100a, NVLink 5 /
NVSwitch): a Router reveals token->expert assignments chunk by chunk and only
completed, revealed chunks may be scheduled, packed or communicated.  The hot
path is hand-written sm_100a CUDA (tcgen05/TMEM/TMA GEMMs, one-sided NVLink
peer stores with device ready signals); the control plane is C++ (event bridge,
compiled scheduler core, peer channel); PyTorch is the framework layer.
"""

__version__ = "0.1.0"
