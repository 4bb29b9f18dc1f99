"""B200-native (sm_100a) fused dequantize-and-multiply for GGUF K-quant and
IQ-quant weights (Q4_K, Q6_K, IQ2_XXS), behind the op API gmlx's quantized
Linear and SwitchGLU/expert modules call (``gmlx_b200.kq`` mirrors
``mlx_kquant``; ``gmlx_b200.nn`` mirrors ``mlx_kquant.nn``)."""
__version__ = "0.1.0"
