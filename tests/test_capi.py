"""The C-ABI library loads, exports what include/b200asr.h declares, and validates
arguments on the host before touching a GPU (these run on CPU-only machines)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "b200asr.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200asr_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from voiceagent_b200._lib import lib as loaded

    return loaded


def test_header_declares_the_hot_path():
    names = declared_symbols()
    for required in ("b200asr_pack_decoder", "b200asr_pack_decode_bucket", "b200asr_pack_audio",
                     "b200asr_store_kvcache", "b200asr_qk_norm_rope_store",
                     "b200asr_paged_decode", "b200asr_paged_prefill",
                     "b200asr_varlen_attention", "b200asr_greedy_argmax"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert missing == []


def test_binding_signatures_cover_the_header():
    from voiceagent_b200._lib import SIGNATURES

    assert sorted(SIGNATURES) == declared_symbols()


def _header_prototypes() -> dict[str, tuple[str, list[str]]]:
    """name -> (return type, [parameter types]) of every B200ASR_API declaration."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = {}
    for ret, name, params in re.findall(
            r"B200ASR_API\s+([\w\s\*]+?)\s*\b(b200asr_\w+)\s*\(([^)]*)\)\s*;", text):
        kinds = []
        for param in params.split(","):
            param = " ".join(param.split())
            if not param or param == "void":
                continue
            # drop the parameter name: the last identifier after the type
            kinds.append(re.sub(r"\s*\b\w+$", "", param) if not param.endswith("*") else param)
        protos[name] = (" ".join(ret.split()), kinds)
    return protos


def _ctype_of(decl: str):
    if "*" in decl or decl == "b200asr_stream_t":
        return ctypes.c_void_p
    return {"int32_t": ctypes.c_int32, "int": ctypes.c_int32, "int64_t": ctypes.c_int64,
            "float": ctypes.c_float, "size_t": ctypes.c_size_t}[decl.replace("const ", "")]


def test_binding_matches_the_header_prototypes():
    """Every ctypes signature in the binding has the parameter and return types the C
    header declares (pointers and the stream cross as void*)."""
    from voiceagent_b200._lib import SIGNATURES

    protos = _header_prototypes()
    assert sorted(protos) == sorted(SIGNATURES)
    for name, (ret, params) in protos.items():
        restype, argtypes = SIGNATURES[name]
        assert [_ctype_of(p) for p in params] == list(argtypes), name
        if ret == "void":
            assert restype is None, name
        elif ret == "const char *":
            assert restype is ctypes.c_char_p, name
        else:
            assert restype is _ctype_of(ret), name


def test_only_the_c_abi_is_exported():
    import subprocess

    from voiceagent_b200._lib import LIB_PATH

    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    ours = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert {n for n in ours if n.startswith("b200asr_")} == set(declared_symbols())


def test_version(lib):
    assert lib.b200asr_version() >= 100


def _err(lib) -> str:
    return lib.b200asr_last_error().decode()


def test_decode_rejects_unsupported_head_dim_without_gpu(lib):
    rc = lib.b200asr_paged_decode(None, 0, None, None, 1, 256, 16, 8, 64, None, None, 1, 1, 1,
                                  1.0, None, 0, None, 0, None, None)
    assert rc == 1 and "head_dim" in _err(lib)


def test_decode_rejects_small_workspace(lib):
    size = lib.b200asr_paged_decode_workspace_size(32, 4096, 16, 128)
    assert size >= 4096 + (32 + 256) * 16 * 130 * 4  # counters + stream-K partials
    dummy = ctypes.c_void_p(256)  # aligned, never dereferenced: the size check comes first
    rc = lib.b200asr_paged_decode(dummy, 2048, dummy, dummy, 16, 256, 16, 8, 128, dummy, dummy,
                                  16, 32, 4096, 1.0, dummy, 2048, dummy, size - 1, None, None)
    assert rc == 4 and "workspace" in _err(lib)


def test_prefill_requires_gqa_group_of_two(lib):
    rc = lib.b200asr_paged_prefill(None, 0, None, None, 1, 256, 16, 4, 128, None, None, None, 1,
                                   1, 1, 1, 1.0, None, 0, None, None)
    assert rc == 1 and "num_heads" in _err(lib)


def test_window_attention_limits_segment_length(lib):
    rc = lib.b200asr_varlen_attention(None, 0, None, 0, None, 0, None, 1, 200, 200, 14, 64, 1.0,
                                      None, 0, None, None)
    assert rc == 1 and "128" in _err(lib)


def test_pack_decoder_rejects_oversized_batch(lib):
    rc = lib.b200asr_pack_decoder(*([None] * 6), 2000, 10, 4, 256, *([None] * 9))
    assert rc == 1 and "batch" in _err(lib)


def test_store_rejects_unaligned_rows(lib):
    dummy = ctypes.c_void_p(256)
    rc = lib.b200asr_store_kvcache(dummy, 12, dummy, 12, dummy, dummy, dummy, 3, 1, 12, 10, None,
                                   None)
    assert rc == 1 and "aligned" in _err(lib)


def test_empty_inputs_are_no_ops(lib):
    assert lib.b200asr_greedy_argmax(None, 10, 0, 10, None, None) == 0
    assert lib.b200asr_store_kvcache(None, 8, None, 8, None, None, None, 0, 1, 8, 1, None, None) == 0


def test_product_path_has_no_oracle_dependency():
    """voiceagent_b200 must never import the test oracle."""
    for path in (REPO / "voiceagent_b200").rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "from oracle" not in text, path


def test_linear_small_validates_on_the_host(lib):
    dummy = ctypes.c_void_p(256)
    assert lib.b200asr_linear_small(dummy, 1024, 65, 1024, dummy, 4096, 0, dummy, 4096, None,
                                    None) == 1 and "64" in _err(lib)
    assert lib.b200asr_linear_small(dummy, 1024, 8, 1000, dummy, 4096, 0, dummy, 4096, None,
                                    None) == 1 and "multiple" in _err(lib)
    assert lib.b200asr_linear_small(dummy, 1024, 8, 1024, dummy, 4000, 0, dummy, 4096, None,
                                    None) == 1
    assert lib.b200asr_linear_small(dummy, 1024, 8, 1024, dummy, 6000, 3000, dummy, 3000, None,
                                    None) == 1 and "SiLU" in _err(lib)
    assert lib.b200asr_linear_small(None, 0, 0, 1024, None, 128, 0, None, 0, None, None) == 0


def test_audio_gather_pos_validates_on_the_host(lib):
    dummy = ctypes.c_void_p(256)
    # d must be a multiple of 8, rows_out cover the tokens, rows 16-byte aligned
    assert lib.b200asr_audio_gather_pos(dummy, 26, dummy, 13, dummy, 20, 24, 892, dummy,
                                        None, None) == 1 and "bad sizes" in _err(lib)
    assert lib.b200asr_audio_gather_pos(dummy, 26, dummy, 13, dummy, 20, 19, 896, dummy, None,
                                        None) == 1
    assert lib.b200asr_audio_gather_pos(ctypes.c_void_p(258), 26, dummy, 13, dummy, 20, 24, 896,
                                        dummy, None, None) == 1 and "aligned" in _err(lib)
    assert lib.b200asr_audio_gather_pos(dummy, 26, None, 13, dummy, 20, 24, 896, dummy, None,
                                        None) == 1 and "null" in _err(lib)
    assert lib.b200asr_audio_gather_pos(None, 0, None, 13, None, 0, 0, 896, None, None,
                                        None) == 0  # nothing to write: no launch


def test_integration_stub_matches_the_bindings():
    """Every ``_lib.<fn>.argtypes = [...]`` line of the INTEGRATION.md ctypes stub lists the
    same argument types as the library's own binding (voiceagent_b200/_lib.py), so the stub
    a maintainer copies calls each entry point with the header's signature."""
    from voiceagent_b200._lib import SIGNATURES

    text = (REPO / "INTEGRATION.md").read_text()
    alias = {"P": ctypes.c_void_p, "I32": ctypes.c_int32, "I64": ctypes.c_int64,
             "F32": ctypes.c_float, "SZ": ctypes.c_size_t}
    found = re.findall(r"_lib\.(b200asr_[a-z0-9_]+)\.argtypes = \[([^\]]*)\]", text)
    assert len(found) >= 25
    for name, body in found:
        got = [alias[t.strip()] for t in body.replace("\n", " ").split(",") if t.strip()]
        want = SIGNATURES[name][1]
        norm = lambda ts: [ctypes.c_void_p if t in (ctypes.c_void_p, ctypes.c_char_p) else t
                           for t in ts]
        assert norm(got) == norm(want), name
