"""The C-ABI library loads without a GPU and exports every symbol include/*.h declares."""

from __future__ import annotations

import ctypes as ct
import re

import pytest
from conftest import ROOT

_DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*\b((?:ekv|ev)_[a-z0-9_]+)\s*\(",
                   re.MULTILINE)


def declared_symbols():
    names = set()
    for header in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.DOTALL)
        names.update(_DECL.findall(text))
    return names


def test_headers_declare_the_full_abi():
    names = declared_symbols()
    assert {"ekv_error", "ekv_resolve_resident", "ekv_lookup_slots", "ekv_gather_rows",
            "ekv_gather_rows_planes", "ekv_lookup_gather_planes", "ekv_compact_misses", "ekv_pack_rows", "ekv_unpack_rows", "ekv_chunk_counts",
            "ekv_freeable_bitmap", "ekv_bitmap_and", "ev_create", "ev_ensure", "ev_precommit",
            "ev_drop", "ev_base", "ev_backed", "ev_reserved", "ev_granularity", "ev_poisoned",
            "ev_error", "ev_close"} <= names


def test_library_exports_every_declared_symbol(library_path):
    lib = ct.CDLL(str(library_path))
    missing = [name for name in sorted(declared_symbols()) if not hasattr(lib, name)]
    assert not missing, missing


def test_python_binding_covers_the_headers(library_path):
    from ekv_b200 import _lib

    assert set(_lib.EXPORTS) == declared_symbols()
    lib = _lib.library(str(library_path))
    assert lib.ekv_abi_version() == 2
    assert lib.ekv_error() == b""


def test_entry_points_validate_before_touching_a_device(library_path):
    """Argument errors come back as -1 plus a message, with no GPU present."""
    from ekv_b200 import _lib

    lib = _lib.library(str(library_path))
    rc = lib.ekv_bitmap_and(None, 0, 4, None, 0, None)
    assert rc == -1 and b"rank" in lib.ekv_error()
    rc = lib.ekv_gather_rows_planes(None, None, 0, 2, None, 4, None, 4, None, 4, None, 8, None, 8,
                                    1, 1, 1, 1, 1, 0, 1, 0, None)
    assert rc == -1 and b"plane count" in lib.ekv_error()
    rc = lib.ekv_gather_layers(None, None, 0, 2, 2, None, 4, None, 4, None, 4, None, 8, None, 8,
                               1, 1, 1, 1, 1, 0, 2, 0, None)
    assert rc == -1 and b"layer count" in lib.ekv_error()
    rc = lib.ekv_gather_layers(None, None, 129, 2, 2, None, 4, None, 4, None, 4, None, 8, None, 8,
                               1, 1, 1, 1, 1, 0, 2, 0, None)
    assert rc == -1 and b"layer count" in lib.ekv_error()
    rc = lib.ekv_gather_layers(None, None, 100, 3, 2, None, 4, None, 4, None, 4, None, 8, None, 8,
                               1, 1, 1, 1, 1, 0, 2, 0, None)
    assert rc == -1 and b"planes_per_layer" in lib.ekv_error()
    rc = lib.ekv_resolve_resident(None, 4, 0, 0, 1, None, 4, 0, 0, None, 8, 0, None, 8, 0, None, 4, 0,
                                  None, 8, 0, 1, None, 0, 0, 0, 0, None)
    assert rc == -1 and b"block_size" in lib.ekv_error()
    rc = lib.ekv_lookup_gather_planes(None, None, 1, 2, None, 4, None, 4, None, 4, None, 4, 20,
                                      1, 1, 1, 0, 0, None, None, 1, 0, None)
    assert rc == -1 and b"flag bits" in lib.ekv_error()
    rc = lib.ekv_lookup_gather_planes(None, None, 1, 2, None, 4, None, 4, None, 4, None, 4, 20,
                                      1, 1, 1, 0, 0, None, None, 0, 0, None)
    assert rc == -1 and b"null lookup output" in lib.ekv_error()
    rc = lib.ekv_compact_misses(None, 0, None, 4, 0, 1, 1, None, 0, None, 0, None)
    assert rc == -1 and b"null pointer" in lib.ekv_error()
    # Empty work is a successful no-op.
    assert lib.ekv_bitmap_and(None, 1, 0, None, 0, None) == 0
    assert lib.ekv_compact_misses(None, 0, None, 4, 0, 0, 1, None, 0, None, 0, None) == 0
    import torch

    if not torch.cuda.is_available():
        assert not lib.ev_create(0, 1 << 21, 1 << 21) and lib.ev_error()


def test_compiled_binding_loads_and_declines_cpu_tensors(library_path):
    """lib/_ekv_torch.so (built with the library) loads without a GPU; for CPU tensors (and
    malformed calls) it reports NOT_HANDLED, so the Python API's checks run and raise its
    own errors."""
    import torch

    from ekv_b200 import _lib
    from ekv_b200.resident_lookup import lookup_slots, resolve_resident

    binding = _lib.torch_binding()
    if binding is None:
        pytest.skip("the torch binding was not built here")
    topk = torch.zeros((1, 2, 4), dtype=torch.int32)
    args = (topk, torch.zeros((2, 8), dtype=torch.int64), torch.zeros(9, dtype=torch.int64), torch.arange(2),
            torch.full((2,), 8), torch.arange(2), torch.zeros((1, 2, 4), dtype=torch.int32), 1)
    assert binding.resolve_resident(*args) == binding.NOT_HANDLED
    status, *_ = binding.lookup_slots(torch.zeros((2, 8), dtype=torch.int32), torch.zeros((2, 4), dtype=torch.int32),
                                      None, None, None, None, None, True)
    assert status == binding.NOT_HANDLED
    with pytest.raises(ValueError, match="CUDA tensor"):
        resolve_resident(*args)
    with pytest.raises(ValueError, match="CUDA tensor"):
        lookup_slots(torch.zeros((2, 8), dtype=torch.int32), torch.zeros((2, 4), dtype=torch.int32))

    from ekv_b200.sparse_read import gather_rows, gather_rows_planes
    from ekv_b200.virtual_layout import VirtualKVLayout

    layout = VirtualKVLayout(2, 8, 4)
    raw = torch.zeros(layout.capacity_bytes // 2, dtype=torch.bfloat16)
    pos, ids, lens = torch.zeros((2, 3), dtype=torch.int64), torch.arange(2), torch.full((2,), 8)
    out = torch.zeros((2, 3, 4), dtype=torch.bfloat16)
    assert binding.gather_rows(raw, pos, ids, lens, None, None, out, 4, 8, 32, 0, False) == binding.NOT_HANDLED
    assert binding.gather_rows_planes([raw], [out], pos, ids, lens, None, None, 4, 8, 32, 0, False,
                                      False) == binding.NOT_HANDLED
    # A wrong output shape is declined before any device check; the checked path names it.
    assert binding.gather_rows(raw, pos, ids, lens, None, None, out[:, :2], 4, 8, 32, 0,
                               False) == binding.NOT_HANDLED
    with pytest.raises(ValueError, match="output shape"):
        gather_rows(raw, pos, ids, lens, None, None, out[:, :2], layout, indirect=False)
    with pytest.raises(ValueError, match="CUDA tensor"):
        gather_rows(raw, pos, ids, lens, None, None, out, layout, indirect=False)
    with pytest.raises(ValueError, match="CUDA tensor"):
        gather_rows_planes([raw], pos, ids, lens, None, None, [out], layout, indirect=False)
    # Empty selections are no-ops on both paths.
    empty = torch.zeros((2, 0), dtype=torch.int64)
    assert binding.gather_rows(raw, empty, ids, lens, None, None, out[:, :0], 4, 8, 32, 0, False) == 0


def test_compiled_binding_can_be_turned_off(library_path):
    """EKV_B200_NO_TORCH_BINDING=1 leaves every call on the checked ctypes path (checked in
    a child process: the binding is loaded once per process)."""
    import os
    import subprocess
    import sys

    from conftest import PACKAGE_ROOT, ROOT

    code = "from ekv_b200 import _lib; assert _lib.torch_binding() is None; print('off')"
    env = dict(os.environ, EKV_B200_NO_TORCH_BINDING="1",
               PYTHONPATH=os.pathsep.join([str(PACKAGE_ROOT), str(ROOT)]))
    done = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert done.returncode == 0 and done.stdout.strip() == "off", done.stderr[-2000:]
