"""quipsharp_b200: QuIP#'s quantized-linear forward path on NVIDIA B200 (sm_100a).

Module layout mirrors the reference package `quipsharp` for the inference path:
codebooks (E8P, 1-bit E8), rvq, hadamard, incoherence, rfft, quantize
(dequantize_linear / linear_forward), checkpoint (QuantizedLinear and the
checkpoint format) and lazy_weights (tensor-at-a-time loading of full-precision
checkpoints).  Beyond the reference: groups (layers that read one input run as
one call) and tensor_parallel (column-sharded layers over NVLink).  All tensor
work runs in hand-written CUDA kernels of libquipsharp_b200.so through its C
ABI (include/quipsharp_b200.h).
"""
__version__ = "0.1.0"
