"""C ABI checks that need no GPU: the in-tree library builds for sm_100a,
loads, and exports every entry point include/suffixgpu.h declares."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "suffixgpu.h")


def declared_symbols() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sg_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def libpath():
    from suffixgpu_b200 import build
    return build.build()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "sg_local_draft" in syms
    assert len(syms) >= 6


def test_library_exports_every_declared_symbol(libpath):
    lib = ctypes.CDLL(libpath)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"missing exports: {missing}"


def test_status_strings_and_version(libpath):
    from suffixgpu_b200 import _lib
    L = _lib.lib()
    assert L.sg_abi_version() >> 16 == 1
    assert L.sg_status_string(0).decode() == "ok"
    assert "invalid" in L.sg_status_string(1).decode()


def test_ctypes_struct_layout_matches_header():
    from suffixgpu_b200._lib import DraftParams, LocalInputs, LocalOutputs
    # field order/sizes of include/suffixgpu.h on LP64
    assert ctypes.sizeof(DraftParams) == 56
    assert DraftParams.row_stride.offset == 8
    assert DraftParams.vote_alpha.offset == 52
    assert ctypes.sizeof(LocalInputs) == 56
    assert LocalInputs.limit.offset == 48
    assert LocalInputs.host_ids.offset == 28
    assert ctypes.sizeof(LocalOutputs) == 56


def test_invalid_arguments_rejected_without_gpu(libpath):
    """Argument validation runs on the host before any CUDA call."""
    from suffixgpu_b200._lib import DraftParams, LocalInputs, LocalOutputs
    from suffixgpu_b200 import _lib
    L = _lib.lib()
    p = DraftParams(batch=2, seq_len=16, row_stride=16, k=0,
                    max_pattern_len=8, max_occurrences=8, num_backoff=3,
                    min_match_len=1)
    st = L.sg_local_draft(ctypes.byref(p), ctypes.byref(LocalInputs()),
                          ctypes.byref(LocalOutputs()), None)
    assert st == 1  # k = 0
    p.k = 4
    p.batch = 0
    st = L.sg_local_draft(ctypes.byref(p), ctypes.byref(LocalInputs()),
                          ctypes.byref(LocalOutputs()), None)
    assert st == 0  # empty batch: nothing to do
    assert L.sg_expand_chain(None, 1, 0, 4, None, None, 0.0, 0.0, None, None,
                             None, None, None) == 1
    # incremental SA rebuild: kept part outside the previous snapshot,
    # negative sizes, and an empty snapshot (nothing to do)
    r = ctypes.c_int32(-1)
    assert L.sg_suffix_array_append(None, 10, None, 10, 5, 6, 0, None, None,
                                    0, ctypes.byref(r), None) == 1
    assert L.sg_suffix_array_append(None, -1, None, 0, 0, 0, 0, None, None,
                                    0, None, None) == 1
    assert L.sg_suffix_array_append(None, 0, None, 0, 0, 0, 0, None, None,
                                    0, ctypes.byref(r), None) == 0
    assert r.value == 0
    assert L.sg_suffix_array_append_workspace_size(1 << 20) >= \
        L.sg_suffix_array_workspace_size(1 << 20)
    # tails before the update: bad shapes, and an empty batch
    assert L.sg_gather_tails_update(None, 4, 8, None, None, 0, None, 8, None,
                                    2, 4, None, None, None, None) == 1
    assert L.sg_gather_tails_update(None, 8, 8, None, None, 0, None, 8, None,
                                    0, 4, None, None, None, None) == 0
    # host-buffer address query: null arguments
    dptr = ctypes.c_void_p(1)
    assert L.sg_mapped_host_ptr(None, ctypes.byref(dptr)) == 1
    buf = ctypes.create_string_buffer(64)
    assert L.sg_mapped_host_ptr(ctypes.addressof(buf), None) == 1


def test_torch_operator_registers():
    """The in-tree torch operator library loads (no GPU needed) and
    registers local_draft with the documented schema."""
    from suffixgpu_b200 import _lib
    op = _lib.torch_ops().local_draft
    schema = str(op.default._schema)
    assert schema.startswith("suffixgpu_b200::local_draft(Tensor num_tokens")
    assert "Tensor params" in schema and "-> Tensor[]" in schema
    assert "Tensor? out_draft=None, Tensor? out_num_valid=None" in schema
    schema = str(_lib.torch_ops().vllm_prepare.default._schema)
    assert schema.startswith("suffixgpu_b200::vllm_prepare(Tensor sampled")
    schema = str(_lib.torch_ops().global_start.default._schema)
    assert schema.startswith("suffixgpu_b200::global_start(Tensor counts")
    assert schema.endswith("-> ()")
    schema = str(_lib.torch_ops().global_finish.default._schema)
    assert schema.startswith("suffixgpu_b200::global_finish(Tensor[] found")
    assert schema.endswith("-> int")


def test_torch_operator_shares_the_process_cxx_runtime():
    """The operator library must use the process's shared libstdc++, not
    a static copy: a second C++ runtime inside it crashed the process when
    an error message formatted a number."""
    import shutil
    import subprocess
    from suffixgpu_b200 import _lib, build
    _lib.torch_ops()
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm is not installed")
    out = subprocess.run([nm, "-D", "--defined-only", build.TORCH_LIB],
                         capture_output=True, text=True, check=True).stdout
    # libstdc++ internals that only a statically linked runtime exports
    assert "_txnal_cow_string_D1" not in out
    assert "__codecvt_utf8_base" not in out
