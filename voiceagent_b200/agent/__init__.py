"""Consumers of the b200asr kernels outside the ASR engine: the TTS talker's paged
decode attention (``qwen_tts_paged_attention``)."""
