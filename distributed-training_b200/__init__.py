"""dtrain_b200: a B200-native (sm_100a) distributed-training stack.

Same capabilities and public API as the `dtrain` project (autograd with
grad-ready hooks, DDP with bucketed overlapped all-reduce and no_sync(), ZeRO-1
sharded AdamW, deterministic collectives, sharded SHA-256 checkpoints, elastic
restart-all launcher), rebuilt on PyTorch with hand-written CUDA kernels for
Blackwell and NVLink collectives that run inside those kernels.
"""
__version__ = "0.1.0"
