"""planejaja_b200 -- B200-native (sm_100a) GGUF block-quantized dequant + matmul."""
from .formats import Q4_0, Q8_0, Q4_K, Q6_K, Q6K_GGML, Q6K_NODESTOR, FORMATS, fmt  # noqa: F401
