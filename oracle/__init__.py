"""CPU oracle for the ragged continuous-batching ASR hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product path (``voiceagent_b200``) may
import, call or link anything under this directory. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm use it,
and only as the checker or as the timed CPU baseline.

Contents:

* ``kernels``  -- numpy restatements of every hot-path function of
  ``qwen_asr_vllm`` (packers, KV store, paged / varlen attention, QK-RMSNorm +
  RoPE, greedy argmax, add-RMSNorm, SiLU-mul). Integer work is bit-exact; float
  work is computed in float64 from bf16-representable inputs.
* ``model``    -- a CPU fp32 restatement of the upstream Qwen3-ASR thinker
  (``reference/modeling_qwen3_asr.py``): audio encoder, text decoder with a KV
  cache, and a fixed-length greedy loop. It is the timed CPU baseline.

Parity pins: ``tests/golden/`` holds fixtures generated in the build container by
running the reference's own Python (``tests/golden/make_golden.py``); the CPU test
suite checks these functions against them.
"""
