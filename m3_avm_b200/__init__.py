"""m3_avm_b200 -- B200-native (sm_100a) fused dequantise-and-matvec for GGUF weights.

A drop-in for the hot path of m3_avm's MATVEC/FFN opcodes: the Q4_0/Q4_K/
Q6_K/Q8_0 block decoders (src/quant.rs) and the fused GEMV
(src/matvec_quant.rs), with the resident-weight offload shape of
src/inference_gpu.rs.  The compute lives in ``libm3gemv.so`` (hand-written
CUDA for sm_100a behind the C ABI of include/m3gemv.h); these modules mirror
the reference's Rust API on top of it.
"""
from . import quant, matvec_quant, inference_gpu, synth  # noqa: F401

__all__ = ["quant", "matvec_quant", "inference_gpu", "synth"]
