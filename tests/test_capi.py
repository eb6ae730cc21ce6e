"""CPU checks of the C ABI library: it loads, exports every symbol include/hearth_b200.h declares,
and rejects bad arguments the way the reference's entry points do (no GPU compute here)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import hearth_b200 as hb
from hearth_b200 import _lib
from oracle import oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(REPO, "include", "hearth_b200.h")).read()
    return sorted(set(re.findall(r"HXB_API\s+[^;(]*?\b(hxb_\w+)\s*\(", src)))


def test_header_symbols_all_exported():
    L = hb.lib()
    names = _declared()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
    assert sorted(_lib.EXPORTS) == names


def test_row_bytes_match_reference_formula():
    for dt in range(5):
        for n in (64, 128, 768, 2048, 7168, 100):
            assert hb.lib().hxb_row_bytes(dt, n) == O.row_bytes(dt, n)
    assert hb.lib().hxb_row_bytes(7, 64) == 0


def test_matmul_argument_errors_match_hearth_matmul():
    L = hb.lib()
    W = np.zeros(34, np.uint8)
    X = np.zeros(64, np.float32)
    Y = np.zeros(1, np.float32)
    assert L.hxb_matmul(9, W.ctypes.data, 1, 64, X.ctypes.data, 1, Y.ctypes.data) == -1   # bad dtype
    assert L.hxb_matmul(4, W.ctypes.data, 1, 65, X.ctypes.data, 1, Y.ctypes.data) == -1   # not /64
    assert L.hxb_matmul(4, W.ctypes.data, -1, 64, X.ctypes.data, 1, Y.ctypes.data) == -1
    assert L.hxb_matmul(4, W.ctypes.data, 1, 64, X.ctypes.data, 0, Y.ctypes.data) == 0    # T = 0
    assert L.hxb_matmul(4, None, 1, 64, X.ctypes.data, 1, Y.ctypes.data) == -1


def test_slab_layout_matches_format():
    # FORMAT.md §5 for the Qwen3-30B-A3B expert: 2.39 MiB slabs
    up, down, nb = O.slab_layout(O.Q4, 2048, 768)
    assert (up, down, nb) == (835584, 1671168, 2506752)


def test_open_without_device_reports_error():
    if hb.lib().hxb_device_count() > 0:
        pytest.skip("a device is present")
    with pytest.raises(RuntimeError, match="not available"):
        hb.MoeBackend(n_layers=1, d_model=128, expert_ffn_dim=64, n_experts=8, top_k=2)


def test_open_rejects_bad_config():
    for kw in (dict(d_model=100), dict(n_experts=500), dict(top_k=0), dict(expert_ffn_dim=96)):
        args = dict(n_layers=1, d_model=128, expert_ffn_dim=64, n_experts=8, top_k=2)
        args.update(kw)
        with pytest.raises(RuntimeError):
            hb.MoeBackend(**args)


def test_stream_argument_mapping():
    """None / 0 select the library's own stream; a torch stream object is used as given, and torch's
    default stream (handle 0) becomes the legacy default stream, so events recorded on it bracket
    the library's kernels."""
    from hearth_b200.moe import _stream

    class FakeStream:
        def __init__(self, h):
            self.cuda_stream = h

    assert _stream(None).value in (None, 0)
    assert _stream(0).value in (None, 0)
    assert _stream(FakeStream(0)).value == 1
    assert _stream(FakeStream(0x1234)).value == 0x1234
    assert _stream(0x5678).value == 0x5678
