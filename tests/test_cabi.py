"""The C-ABI library loads without a GPU and exports every entry point the header declares."""
import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _declared():
    names = []
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(lh_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = _declared()
    assert "lh_select_topk" in names and "lh_attn_fwd" in names and len(names) >= 12


def test_library_exports_every_declared_symbol(lh):
    lib = lh._native.load()
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_binding_covers_header(lh):
    assert set(_declared()) <= set(lh._native.exported_symbols())


def test_abi_version_and_error_string(lh):
    lib = lh._native.load()
    assert lib.lh_abi_version() >= 100
    assert isinstance(lib.lh_last_error(), bytes)


def test_shape_validation_needs_no_gpu(lh):
    # argument checks run before any device query: a null pointer is rejected on the host
    lib = lh._native.load()
    rc = lib.lh_select_topk(None, None, 1, 1, 4096, 3, 4, 256, None, None, None)
    assert rc == 2 and b"null" in lib.lh_last_error()


def test_cpu_tensors_are_refused(lh):
    import torch
    sq = torch.rand(1, 1, 4096 + 1024 + 256)
    with pytest.raises(AssertionError):
        lh.LighthouseSelectionQkKqChunkedTopkNvrtc.forward(sq, sq, 3, 4, 256, 4096)
    with pytest.raises(ValueError):
        lh._native.select_topk(sq, sq, 3, 4, 256, 4096)


def test_reference_asserts_mirrored(lh):
    import torch
    sq = torch.rand(1, 1, 10)
    with pytest.raises(AssertionError):
        lh.LighthouseSelectionQkKqChunkedTopkNvrtc.forward(sq, sq[:, :, :5], 3, 4, 256, 4096)


def test_compute_output_indices_selection(lh, O):
    for case in [(4096, 3, 4, 256), (131072, 3, 4, 2048), (98304, 5, 2, 1536)]:
        assert lh.compute_output_indices_selection(*case) == O.sel_len(*case)
    assert lh.compute_output_indices_selection(131072, 3, 4, 2048) == 24576
    assert lh.compute_output_indices_selection(65536, 3, 4, 2048) == 20480
