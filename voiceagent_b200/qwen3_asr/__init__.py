"""Qwen3-ASR network definitions (decoder, audio tower, assembly)."""
