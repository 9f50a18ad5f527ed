"""Layer-level wrappers of the b200asr kernels, mirroring ``qwen_asr_vllm.layers``."""
