"""B200-native ragged continuous-batching path of the qwen-asr-vllm engine.

The CUDA kernels live in ``libb200asr.so`` (C ABI in ``include/b200asr.h``), built
in-tree by ``python -m voiceagent_b200.build``; ``voiceagent_b200.kernels`` wraps them
for torch tensors. Importing the package does not require a GPU.
"""

__version__ = "0.1.0"


def __getattr__(name):
    # Lazy exports so ``import voiceagent_b200`` stays cheap and CPU-safe.
    if name in ("AsrEngine", "AsrOutput"):
        from voiceagent_b200.engine import engine

        return getattr(engine, name)
    if name == "EngineConfig":
        from voiceagent_b200.config import EngineConfig

        return EngineConfig
    if name == "SamplingParams":
        from voiceagent_b200.engine.request import SamplingParams

        return SamplingParams
    raise AttributeError(name)
