"""Qwen3 layers that call the W4A16 and KV4 operators."""
