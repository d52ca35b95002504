"""The C-ABI library loads without a GPU and exports every entry point that
include/*.h declares."""
import os
import re

from helpers import ROOT, lfm3


def declared_functions():
    names = set()
    for header in os.listdir(os.path.join(ROOT, "include")):
        if not header.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", header)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(lfm3_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    lib = lfm3.library()
    names = declared_functions()
    assert len(names) > 40
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_host_queries_need_no_gpu():
    lib = lfm3.library()
    assert lib.lfm3_cuda_prompt_rows() == 16
    assert lib.lfm3_cuda_dense_workspace_bytes(8, 2048) == 8 * 2048 * 4
    assert lib.lfm3_cuda_dense_workspace_bytes(512, 2048) == 512 * 2048 * 4
    assert lib.lfm3_cuda_split_ticket_words() >= 1024
    assert lib.lfm3_cuda_attention_scratch_bytes(16, 128, 32768, 512) > 0
