"""The C-ABI library on the CPU: it loads without a GPU, exports every entry point
include/flash_lab_b200.h declares, its struct layouts match the ctypes mirror field by field, and
its host-only helpers behave. No kernel is launched here."""

import ctypes
import pathlib
import re
import subprocess

import pytest

from flash_lab import _capi

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "flash_lab_b200.h"


@pytest.fixture(scope="module")
def lib():
    return _capi.load()


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"\b(flb_[a-z0-9_]+)\s*\(", text))


def test_header_and_binding_agree():
    assert declared_functions() == set(_capi.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_capi.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\b(flb_[a-z0-9_]+)\b", out))
    assert declared_functions() <= exported


def test_version_and_status_strings(lib):
    assert lib.flb_version() == 3
    assert lib.flb_status_string(0) == b"ok"
    assert lib.flb_status_string(3) == b"misaligned pointer or stride"
    assert lib.flb_status_string(99) == b"unknown status"


def _c_layout(struct: str, fields: list[str], tmp_path) -> dict[str, int]:
    src = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){",
             f'printf("sizeof %zu\\n", sizeof({struct}));']
    for f in fields:
        lines.append(f'printf("{f} %zu\\n", offsetof({struct}, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.splitlines())}


@pytest.mark.parametrize("struct,cls", [("flb_attn_params", _capi.AttnParams),
                                        ("flb_decode_params", _capi.DecodeParams),
                                        ("flb_peer_exchange", _capi.PeerExchange)])
def test_struct_layout_matches_header(struct, cls, tmp_path):
    fields = [name for name, _ in cls._fields_]
    layout = _c_layout(struct, fields, tmp_path)
    assert layout["sizeof"] == ctypes.sizeof(cls)
    for name in fields:
        assert layout[name] == getattr(cls, name).offset, name


def test_host_validation_without_a_gpu(lib):
    assert lib.flb_prefill_fwd(None, None) == _capi.FLB_ERR_INVALID_ARGUMENT
    assert b"NULL" in lib.flb_last_error()
    assert lib.flb_decode_fwd(None, None) == _capi.FLB_ERR_INVALID_ARGUMENT
    p = _capi.DecodeParams()
    assert lib.flb_decode_fwd(ctypes.byref(p), None) == _capi.FLB_ERR_INVALID_ARGUMENT


def test_split_count_depends_on_shapes_only(lib):
    # Graph safety: the split count is a pure function of shapes and the SM count.
    a = lib.flb_decode_num_splits(8, 32, 32, 128, 32768, 148)
    assert a == lib.flb_decode_num_splits(8, 32, 32, 128, 32768, 148)
    assert 1 <= a <= 256
    assert lib.flb_decode_num_splits(1, 32, 32, 128, 32768, 148) > a   # fewer CTAs, more splits
    assert lib.flb_decode_num_splits(8, 32, 32, 128, 300, 148) == 1     # short cache
    assert lib.flb_decode_num_splits(0, 32, 32, 128, 300, 148) == 1     # degenerate input


def test_workspace_bytes(lib):
    assert lib.flb_decode_workspace_bytes(8, 32, 128, 1) == 0
    n = lib.flb_decode_workspace_bytes(8, 32, 128, 16)
    slots = 8 * 32 * (2 * 16 + 1)   # a length-balanced launch writes up to B * H * (2 splits + 1)
    assert n >= slots * 128 * 4 + slots * 8


def test_peer_exchange_sizes(lib):
    # Layout: counters (world + 1 uint64 in a 256-byte block), then two parity regions of
    # partial_o + partial_ml.
    world, batch, heads, d, splits = 2, 1, 32, 128, 4
    slots = batch * heads * world * splits
    po = -(-slots * d * 4 // 256) * 256
    region = -(-(po + slots * 2 * 4) // 256) * 256
    assert lib.flb_peer_exchange_bytes(world, batch, heads, d, splits) == 256 + 2 * region
    assert lib.flb_peer_exchange_bytes(0, batch, heads, d, splits) == 0
    assert lib.flb_peer_handle_bytes() == 64


def test_peer_exchange_host_validation(lib):
    p = _capi.DecodeParams()
    x = _capi.PeerExchange()
    x.world, x.rank = 2, 0           # buffers left NULL
    assert lib.flb_decode_partials_push(ctypes.byref(p), 0, 1, 0, ctypes.byref(x), None) \
        == _capi.FLB_ERR_INVALID_ARGUMENT
    assert b"buffer of rank 0" in lib.flb_last_error()
    assert lib.flb_peer_exchange_reset(ctypes.byref(x), None) == _capi.FLB_ERR_INVALID_ARGUMENT
    x.world = 9
    assert lib.flb_decode_merge_peers(ctypes.byref(x), 1, 32, 128, 1, 0, None, 0, 0, None,
                                      None, None) == _capi.FLB_ERR_INVALID_ARGUMENT
    assert lib.flb_peer_alloc(0, ctypes.byref(ctypes.c_void_p()), None) \
        == _capi.FLB_ERR_INVALID_ARGUMENT
