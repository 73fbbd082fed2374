"""CPU: the C-ABI library builds, loads and exports every symbol the header
declares (no kernel is launched here)."""

import ctypes
import re
from pathlib import Path

import pytest

from preemptlm_b200 import _abi
from preemptlm_b200.build import LIB_PATH, build_library

HEADER = Path(__file__).resolve().parents[1] / "include" / "sg_abi.h"


def header_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sg_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build_library()
    assert LIB_PATH.exists()
    return _abi.load()


def test_header_declares_expected_symbols():
    assert set(header_symbols()) == set(_abi.EXPORTED_SYMBOLS)


def test_library_exports_every_header_symbol(lib):
    for name in header_symbols():
        assert hasattr(lib, name), name


def test_status_strings_and_version(lib):
    assert lib.sg_version() >= 1
    assert lib.sg_built_arch() == 1000
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert lib.sg_status_string(code).decode()
    assert "unknown" in lib.sg_status_string(-99).decode()


def test_host_side_argument_checks(lib):
    # shape / format checks run before any CUDA call
    a = _abi.sg_arena(num_slots=4, hidden=2048, inter=512, bits=8, group_size=64)
    n = 3 * 2048 * 512
    assert lib.sg_expert_bytes(ctypes.byref(a)) == n + n // 64 * 4
    a.bits = 16
    assert lib.sg_expert_bytes(ctypes.byref(a)) == 2 * n
    a.bits = 4
    assert lib.sg_expert_bytes(ctypes.byref(a)) == n // 2 + n // 64 * 4
    a.bits = 3
    assert lib.sg_expert_bytes(ctypes.byref(a)) == 0
    assert lib.sg_router_logits(None, None, None, 1, 2048, 8, None) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_router_logits(1, 1, 1, 1, 100 + 256, 8, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_route_topk(1, 1, 33, 2, 1, 1, 1, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_route_topk(1, 1, 64, 33, 1, 1, 1, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_dispatch(1, 8, 9000, 1, 1, 1, 1, 1, 1, 1, 1, 100, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_dispatch(1, 8, 64, 1, 1, 1, 1, 1, 1, 1, 1, 4, None) == _abi.SG_ERR_CAPACITY
    a = _abi.sg_arena(num_slots=4, hidden=2048, inter=512, bits=5, group_size=64, gate_w=1, up_w=1, down_w=1)
    assert lib.sg_glu_gate_up(ctypes.byref(a), 1, 1, 1, 1, 1, 1, 1, 1, 1, 0, None) == _abi.SG_ERR_FORMAT
    a.bits = 8
    a.group_size = 32
    assert lib.sg_glu_down(ctypes.byref(a), 1, 1, 1, 1, 1, 1, 1, 1, 0, None) == _abi.SG_ERR_FORMAT
    a.bits, a.group_size, a.hidden = 16, 64, 100
    assert lib.sg_glu_down(ctypes.byref(a), 1, 1, 1, 1, 1, 1, 1, 1, 0, None) == _abi.SG_ERR_SHAPE
    a.hidden = 2048
    assert lib.sg_glu_down(ctypes.byref(a), 1, 1, 1, 1, 1, 1, 1, 1, 4, None) == _abi.SG_ERR_INVALID_ARG  # flag
    assert lib.sg_glu_forward(ctypes.byref(a), None, 0, 1, None, None, None, None, 1, None, None, None,
                              None) == _abi.SG_OK  # empty
    assert lib.sg_permute_rows(1, 1, 1, 4, 12, 1, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_permute_rows(1, 1, 0, 4, 16, 1, None) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_set_glu_path(5) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_set_glu_tile(12) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_set_glu_tile(256) == _abi.SG_ERR_INVALID_ARG
    for bn in (8, 16, 32, 64, 128, 0):
        assert lib.sg_set_glu_tile(bn) == _abi.SG_OK
    # integer-operand gate/up: work sizes and argument checks (no GPU touched)
    assert lib.sg_quantize_pieces(1, 2, 100, 0, 1, 1, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_quantize_pieces(1, 2, 128, 2, 1, 1, None) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_quantize_pieces(None, 0, 128, 0, None, None, None) == _abi.SG_OK
    q8 = _abi.sg_arena(num_slots=512, hidden=2048, inter=512, bits=8, group_size=64, gate_w=1, gate_s=1, gate_b=1,
                       up_w=1, up_s=1, up_b=1, down_w=1, down_s=1, down_b=1)
    # decode: 256 tokens x top-10 over 512 groups (mean 5 pairs): the pieces of the 256 token rows
    pieces = 256 * 2 * 2048 + 256 * 32 * 8
    assert lib.sg_glu_gate_up_work_bytes(ctypes.byref(q8), 2560, 10, 512, 0) == pieces
    # the fused call reuses the bytes for h's pieces (2560 rows of 512), the larger of the two
    h_pieces = 2560 * 2 * 512 + 2560 * 8 * 8
    assert lib.sg_glu_down_work_bytes(ctypes.byref(q8), 2560, 512) == h_pieces
    assert lib.sg_glu_forward_scratch_bytes(ctypes.byref(q8), 2560, 10, 512) == max(pieces, h_pieces)
    # prefill-sized groups: the permuted token rows instead
    assert lib.sg_glu_gate_up_work_bytes(ctypes.byref(q8), 81920, 10, 512, 0) == 0
    assert lib.sg_glu_forward_scratch_bytes(ctypes.byref(q8), 81920, 10, 512) == 81920 * 2048 * 2
    for mode, want in ((2, 0), (1, 0), (4, pieces)):
        assert lib.sg_set_glu_path(mode) == _abi.SG_OK
        assert lib.sg_glu_gate_up_work_bytes(ctypes.byref(q8), 2560, 10, 512, 0) == want
    assert lib.sg_set_glu_path(0) == _abi.SG_OK
    q8.bits = 4  # 4-bit arenas: the same pieces (unpacked nibbles feed the same kernel)
    assert lib.sg_glu_gate_up_work_bytes(ctypes.byref(q8), 2560, 10, 512, 0) == pieces
    q8.bits, q8.inter = 4, 768  # I = 768: 12 groups per down row, not whole scale chunks of 8
    assert lib.sg_glu_down_work_bytes(ctypes.byref(q8), 2560, 512) == 0
    # expert-parallel exchange: argument checks and the region layout (no GPU touched)
    assert lib.sg_ep_region_bytes(9, 16, 256) == _abi.SG_ERR_INVALID_ARG  # more than 8 ranks
    assert lib.sg_ep_region_bytes(2, 16, 100) == _abi.SG_ERR_SHAPE        # H % 8
    off = (ctypes.c_longlong * 5)()
    assert lib.sg_ep_layout(2, 2560, 2048, off) == _abi.SG_OK
    rows = 2 * 2560 * 2048 * 2
    assert list(off) == [0, rows, rows + 2 * 2560 * 4, rows + 2 * 2 * 2560 * 4, rows + 2 * 2 * 2560 * 4 + 256]
    assert lib.sg_ep_region_bytes(2, 2560, 2048) == off[4] + 2560 * 2048 * 2 + 2 * 256 + 256 + 256  # + step and done counters
    regs = (ctypes.c_void_p * 2)(1, 1)
    assert lib.sg_ep_send(regs, 2, 0, 16, 256, 1, 1, 4, 5, 8, 1, None) == _abi.SG_ERR_CAPACITY  # 20 > 16
    assert lib.sg_ep_send(regs, 2, 2, 16, 256, 1, 1, 2, 5, 8, 1, None) == _abi.SG_ERR_INVALID_ARG  # me
    assert lib.sg_ep_send(regs, 2, 0, 16, 256, 1, 1, 2, 5, 0, 1, None) == _abi.SG_ERR_INVALID_ARG  # per 0
    assert lib.sg_ep_wait_inbox(None, 2, 16, 256, None) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_ep_alloc(0, None) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_ep_set_wait_limit(0) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_ep_set_wait_limit(601 * 10**6) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_ep_wait_back(1, 2, 16, 256, 1, 5, 4, 8, None) == _abi.SG_ERR_CAPACITY  # 20 pairs > cap 16
    assert lib.sg_ep_wait_back(1, 2, 16, 256, None, 2, 4, 8, None) == _abi.SG_ERR_INVALID_ARG
    a = _abi.sg_arena(num_slots=2, hidden=1024, inter=512, bits=8, group_size=64, gate_w=1, up_w=1, down_w=1,
                      gate_s=1, gate_b=1, up_s=1, up_b=1, down_s=1, down_b=1)
    assert lib.sg_dense_glu(ctypes.byref(a), 2, 1, 4, 1, 1, None) == _abi.SG_ERR_INVALID_ARG  # slot out of range
    assert lib.sg_dense_glu(ctypes.byref(a), 0, None, 4, 1, 1, None) == _abi.SG_ERR_INVALID_ARG
    assert lib.sg_dense_glu(ctypes.byref(a), 0, None, 0, None, None, None) == _abi.SG_OK  # empty: no pointer read
    a.inter = 192  # I % 128 != 0: not a dense tensor-core shape
    assert lib.sg_dense_glu(ctypes.byref(a), 0, 1, 4, 1, 1, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_combine(1, 1, 1, 2, 12, None, None, 1, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_combine(1, 1, 1, 2, 16, 1, None, 1, None) == _abi.SG_ERR_INVALID_ARG
    a = _abi.sg_arena(num_slots=4, hidden=256, inter=128, bits=16, group_size=64, gate_w=1, up_w=1, down_w=1)
    assert lib.sg_refill_h2d(1, 10, ctypes.byref(a), 0, None) == _abi.SG_ERR_SHAPE
    assert lib.sg_refill_h2d(1, 3 * 256 * 128 * 2, ctypes.byref(a), 4, None) == _abi.SG_ERR_SHAPE


def test_ops_fail_loudly_without_library(monkeypatch, tmp_path):
    monkeypatch.setattr(_abi, "_lib", None)
    monkeypatch.setenv("SG_B200_LIB", str(tmp_path / "missing.so"))
    with pytest.raises(ImportError):
        _abi.load()
