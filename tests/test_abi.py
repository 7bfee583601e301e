"""The C-ABI library loads (no GPU needed) and exports every symbol that
include/llmembed.h declares; without a GPU the entry points fail cleanly."""
import ctypes as C
import os
import re

import pytest

from llm_embed_b200 import embed

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "llmembed.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(le_[a-z_0-9]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("le_init", "le_model_load", "le_model_load_gguf", "le_embed_ids", "le_dequant", "le_qgemm",
              "le_model_free", "le_info", "le_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(embed.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_entry_points_fail_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    n = C.c_int(-1)
    rc = embed.lib().le_init(C.byref(n))
    assert rc == embed.LE_ECUDA
    assert embed.lib().le_last_error()
    buf = C.create_string_buffer(256)
    assert embed.lib().le_info(buf, 256) == 0
    assert b'"devices": 0' in buf.value
    with pytest.raises(embed.LlmEmbedError):
        embed.init()
