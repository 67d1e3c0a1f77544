"""cq_pretrain_b200: a Blackwell-native (sm_100a) unified multimodal pretraining framework.

The package trains a Qwen3.5-style hybrid Gated-DeltaNet / gated-attention backbone in CQ
(content/query) layout jointly with a Wan2.1 DiT renderer. PyTorch is the framework layer;
the hot paths are hand-written CUDA kernels for sm_100a in ``csrc/``; NCCL over NVLink plus
in-kernel peer-memory collectives carry the distributed traffic.
"""

__version__ = "0.1.0"
