"""Model execution: batch preparation, CUDA-graph capture and replay."""
