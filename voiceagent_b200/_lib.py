"""ctypes binding of ``libb200asr.so`` (the C ABI declared in include/b200asr.h).

The library is built in-tree by ``voiceagent_b200.build``; importing this module
loads it and fails loudly when it is missing -- there is no fallback path.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200asr.so"

c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t
c_void_p = ctypes.c_void_p
c_char_p = ctypes.c_char_p

P = c_void_p  # every pointer (device memory or stream) crosses as void*

# name -> (restype, argtypes); mirrors include/b200asr.h one to one.
SIGNATURES: dict[str, tuple] = {
    "b200asr_version": (c_int32, []),
    "b200asr_last_error": (c_char_p, []),
    "b200asr_set_pdl": (None, [c_int32]),
    "b200asr_pdl_enabled": (c_int32, []),
    "b200asr_pack_decoder": (c_int32, [P, P, P, P, P, P, c_int32, c_int32, c_int32, c_int32,
                                       P, P, P, P, P, P, P, P, P]),
    "b200asr_pack_decode_bucket": (c_int32, [P, P, P, P, P, c_int32, c_int32, c_int32, c_int32,
                                             P, P, P, P, P, P]),
    "b200asr_advance_decode_bucket": (c_int32, [P, P, P, P, c_int32, P]),
    "b200asr_pack_audio": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, c_int32,
                                     P, P, P, P, P, P, P, P]),
    "b200asr_audio_chunk_pad": (c_int32, [P, c_int32, c_int32, P, P, c_int32, c_int32, P, P]),
    "b200asr_audio_gather_pos": (c_int32, [P, c_int64, P, c_int32, P, c_int32, c_int32, c_int32,
                                             P, P, P]),
    "b200asr_store_kvcache": (c_int32, [P, c_int64, P, c_int64, P, P, P, c_int32, c_int32,
                                        c_int32, c_int64, P, P]),
    "b200asr_qk_norm_rope_store": (c_int32, [P, c_int64, P, c_int32, c_int32, c_int32, c_int32,
                                             P, P, c_float, P, c_int32, P, c_int64, P, P, P, P,
                                             c_int64, P, P]),
    "b200asr_rmsnorm": (c_int32, [P, P, P, c_float, c_int32, c_int32, P, P]),
    "b200asr_silu_mul": (c_int32, [P, c_int32, c_int32, P, P]),
    "b200asr_linear_small": (c_int32, [P, c_int64, c_int32, c_int32, P, c_int32, c_int32, P,
                                       c_int64, P, P]),
    "b200asr_linear_small_add": (c_int32, [P, c_int64, c_int32, c_int32, P, c_int32, P, c_int64,
                                           P, c_int64, P, P, P, P]),
    "b200asr_linear_small_norm": (c_int32, [P, c_int64, P, c_int32, P, c_float, c_int32, c_int32,
                                            P, c_int32, c_int32, P, c_int64, P, P, P]),
    "b200asr_linear_small_norm_qk_rope": (c_int32, [P, c_int64, P, c_int32, P, c_float, c_int32,
                                                    c_int32, P, c_int32, c_int32, c_int32, P, P,
                                                    c_float, P, P, c_int32, P, c_int64, P, P, P,
                                                    c_int64, P, P, P]),
    "b200asr_linear_small_qk_rope": (c_int32, [P, c_int64, c_int32, c_int32, P, c_int32, c_int32,
                                               c_int32, P, P, c_float, P, P, c_int32, P, c_int64,
                                               P, P, P, c_int64, P, P]),
    "b200asr_rms_stats": (c_int32, [P, P, c_int32, c_int32, P, P, P]),
    "b200asr_norm_apply": (c_int32, [P, P, P, c_float, c_int32, c_int32, P, P]),
    "b200asr_log_mel_workspace_size": (c_size_t, [c_int32, c_int32]),
    "b200asr_log_mel": (c_int32, [P, P, P, c_int32, c_int32, P, P, P, P, c_size_t, P, c_int64, P,
                                  P, P]),
    "b200asr_paged_decode_workspace_size": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "b200asr_paged_decode": (c_int32, [P, c_int64, P, P, c_int32, c_int32, c_int32, c_int32,
                                       c_int32, P, P, c_int32, c_int32, c_int32, c_float, P,
                                       c_int64, P, c_size_t, P, P]),
    "b200asr_paged_decode_noalloc": (c_int32, [P, c_int64, P, P, c_int32, c_int32, c_int32,
                                               c_int32, c_int32, P, P, c_int32, c_int32,
                                               c_int32, c_float, P, c_int64, P, P]),
    "b200asr_paged_prefill": (c_int32, [P, c_int64, P, P, c_int32, c_int32, c_int32, c_int32,
                                        c_int32, P, P, P, c_int32, c_int32, c_int32, c_int32,
                                        c_float, P, c_int64, P, P]),
    "b200asr_varlen_attention": (c_int32, [P, c_int64, P, c_int64, P, c_int64, P, c_int32,
                                           c_int32, c_int32, c_int32, c_int32, c_float, P,
                                           c_int64, P, P]),
    "b200asr_pool_paged_decode_workspace_size": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "b200asr_pool_paged_decode": (c_int32, [c_int32, c_int32, c_int32, c_int32, c_int32,
                                            P, c_int64, c_int64, P, P, c_int32, c_int32,
                                            c_int64, c_int64, c_int64, P, c_int64, c_int32,
                                            P, P, c_int64, c_int32, P, P, c_int64, c_int64,
                                            P, c_int64, c_int64, c_int32, c_int32, c_float,
                                            P, c_size_t, P, P]),
    "b200asr_greedy_argmax": (c_int32, [P, c_int64, c_int32, c_int32, P, P]),
    "b200asr_conv_weight_bytes": (c_size_t, [c_int32, c_int32]),
    "b200asr_conv_pack_weight": (c_int32, [P, c_int32, c_int32, P, P]),
    "b200asr_conv3x3s2_gelu": (c_int32, [P, c_int32, c_int32, c_int32, c_int32, P, P, c_int32,
                                         P, c_int64, c_int64, c_int64, P, P]),
}


class L2Prefetch(ctypes.Structure):
    """``b200asr_l2_prefetch`` (include/b200asr.h), passed by pointer."""

    _fields_ = [("cu_seqlens_k", c_void_p), ("block_tables", c_void_p), ("bt_stride", c_int32),
                ("batch", c_int32), ("block_size", c_int32), ("num_kv_heads", c_int32),
                ("head_dim", c_int32), ("k_cache", c_void_p), ("v_cache", c_void_p),
                ("num_slots", c_int64), ("range", c_void_p * 2), ("range_bytes", c_int64 * 2)]


class B200AsrError(RuntimeError):
    """A b200asr C-ABI call returned a non-zero status."""


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    path = Path(path) if path is not None else LIB_PATH
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m voiceagent_b200.build` "
            "(nvcc for sm_100a). The b200asr kernels have no fallback implementation."
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = load()

_STATUS = {1: "invalid argument", 2: "CUDA error", 3: "unsupported", 4: "workspace too small"}


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib.b200asr_last_error().decode(errors="replace")
        raise B200AsrError(f"{what}: {_STATUS.get(status, status)}: {msg}")
