"""p2pllm_b200: the replica hot path of p2pLLM (Wanda calibration + top-k compaction, the compact sparse GEMM, the
group combine and the multi-GPU hop) as hand-written sm_100a CUDA kernels behind a C ABI (include/p2p_b200.h), with
the reference's Python operator API on top (compact, wanda, replica, route)."""
from ._lib import P2PError  # noqa: F401

__version__ = "0.1.0"
