"""CPU checks of the C ABI boundary: the library loads and exports exactly the
entry points include/npl_w8a8.h declares (no compute call without a GPU)."""
from __future__ import annotations

import ctypes
import re

from conftest import REPO


def declared_symbols() -> set[str]:
    text = (REPO / "include" / "npl_w8a8.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(npl_[a-z0-9_]+)\s*\(", text))


def test_header_declares_the_path():
    syms = declared_symbols()
    for name in ("npl_quant_rows", "npl_rmsnorm_quant", "npl_w8a8_linear", "npl_linear_workspace_bytes",
                 "npl_store_kv", "npl_rope_store_kv", "npl_paged_decode_attention",
                 "npl_decode_attention_workspace_bytes", "npl_last_error_string", "npl_device_status"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    from nanopointllm_b200 import _lib
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header():
    from nanopointllm_b200 import _lib
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_version_and_error_string_without_device():
    from nanopointllm_b200 import _lib
    assert _lib.lib.npl_version() >= 1
    assert isinstance(_lib.lib.npl_last_error_string(), bytes)


def test_workspace_sizes_are_host_only():
    from nanopointllm_b200 import _lib
    n = _lib.lib.npl_linear_workspace_bytes(8, 12288, 4096)
    # (SMs - 1) partial-tile slots of 8 token columns x 128 rows x int32 + counters
    assert n >= 8 * 128 * 4
    a = _lib.lib.npl_decode_attention_workspace_bytes(8, 32, 128, 5, 256)
    assert a >= 8 * 32 * 5 * (128 + 2) * 4


def test_struct_layout_matches_header(tmp_path):
    """The ctypes mirror of npl_linear_args / npl_rope_kv has the C layout."""
    import shutil
    import subprocess
    from nanopointllm_b200 import _lib
    cxx = shutil.which("g++") or shutil.which("gcc")
    if cxx is None:
        import pytest
        pytest.skip("no host C compiler")
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "npl_w8a8.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu\\n", sizeof(npl_linear_args), sizeof(npl_rope_kv),'
                   ' offsetof(npl_linear_args, rope), offsetof(npl_linear_args, absmax_out));return 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run([cxx, "-x", "c", f"-I{REPO / 'include'}", str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    assert [int(v) for v in got] == [ctypes.sizeof(_lib.NplLinearArgs), ctypes.sizeof(_lib.NplRopeKV),
                                     _lib.NplLinearArgs.rope.offset, _lib.NplLinearArgs.absmax_out.offset]


def test_tp_exchange_layout_is_host_only():
    """npl_tp_exchange_bytes: flag and call-count words, then two parities of
    every rank's int32 slot (max_elems) and absmax slot (64 rows)."""
    import ctypes as C
    from nanopointllm_b200 import _lib
    al = lambda x: (x + 255) & ~255  # noqa: E731
    for world, max_elems in ((2, 64 * 4096), (8, 64 * 4096), (4, 1024)):
        head = al(4 * 8 * 64) * 2 + al(4 * 64) * 2
        want = head + al(4 * 2 * world * max_elems) + al(4 * 2 * world * 64)
        assert _lib.lib.npl_tp_exchange_bytes(world, max_elems) == want
    assert _lib.lib.npl_tp_exchange_bytes(9, 1024) == 0      # more ranks than NPL_TP_MAX_RANKS
    assert _lib.lib.npl_tp_exchange_bytes(2, 1022) == 0      # max_elems not a multiple of 4
    assert C.sizeof(_lib.NplTpPeers) == 4 + 4 + 8 * _lib.TP_MAX_RANKS + 8
