"""Host-side mirror of the parts of ``qslab.runtime`` that sit on the W4A16 /
KV4 hot path: the quantized-linear backend boundary, the paged attention
module, the Qwen3 layers that call them, CUDA-graph capture and the
tensor-parallel split."""
