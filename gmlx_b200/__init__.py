"""B200-native (sm_100a) fused dequantize-and-multiply for GGUF K-quant and
IQ-quant weights (every codec of gmlx's list: the K-quants, the legacy
32-weight codecs, the IQ1-IQ4 lattices, MXFP4 / NVFP4, plus TQ1_0 / TQ2_0),
behind the op API gmlx's quantized
Linear and SwitchGLU/expert modules call (``gmlx_b200.kq`` mirrors
``mlx_kquant``; ``gmlx_b200.nn`` mirrors ``mlx_kquant.nn``)."""
__version__ = "0.1.0"
