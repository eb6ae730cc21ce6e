"""The .hearth reader on CPU (hxb_container_probe: host code only): the fixture written by the
reference's own container writer (tests/golden/make_container.py) probes to its configuration, and
files that break the format's rules are refused with a message."""
import struct

import numpy as np
import pytest

import hearth_b200 as hb
from tests.container_util import FIXTURE, expert_entries, preamble, tensor_entries


def test_fixture_probes_to_its_configuration():
    cfg, info = hb.container_probe(FIXTURE)
    assert cfg["n_layers"] == 3 and cfg["d_model"] == 128 and cfg["expert_ffn_dim"] == 64
    assert cfg["n_experts"] == 8 and cfg["top_k"] == 2
    assert (cfg["score_fn"], cfg["score_bias"], cfg["n_group"], cfg["topk_group"], cfg["norm_topk_prob"]) == (1, 1, 4, 2, 1)
    assert cfg["routed_scale"] == np.float32(2.5) and cfg["residual_scale"] == np.float32(0.5)
    assert cfg["norm_eps"] == np.float32(1e-6)
    assert cfg["expert_dtype"] == hb.Q4 and cfg["shared_ffn_dim"] == 64 and cfg["shared_dtype"] == hb.Q8
    assert cfg["shared_gate"] == 0
    assert info == dict(n_layers=3, n_moe_layers=2, n_expert_entries=24, n_physical_slabs=13, n_aliased=3,
                        expert_dtype=hb.Q4, slab_bytes=16384)


def test_probe_agrees_with_an_independent_read_of_the_directory():
    buf = open(FIXTURE, "rb").read()
    ents = expert_entries(buf)
    moe = [x for i, x in enumerate(ents) if i // 8 in (1, 2)]
    assert all(x["nbytes"] == 0 for i, x in enumerate(ents) if i // 8 == 0)   # the dense layer
    assert len({x["off"] for x in moe}) == 13 and sum(x["flags"] & 1 for x in moe) == 3
    assert all(x["off"] % 4096 == 0 and x["nbytes"] == 16384 and x["dtype"] == hb.Q4 for x in moe)


def _patched(tmp_path, edit):
    buf = bytearray(open(FIXTURE, "rb").read())
    buf = edit(buf) or buf
    p = tmp_path / "bad.hearth"
    p.write_bytes(bytes(buf))
    return p


def _entry_pos(buf, i):
    return preamble(buf)["edir_off"] + 32 * i


def _first_alias(buf):
    return next(i for i, x in enumerate(expert_entries(buf)) if x["flags"] & 1)


CORRUPTIONS = {
    "magic": (lambda b: b.__setitem__(0, 0x00), "bad magic"),
    "version": (lambda b: struct.pack_into("<I", b, 4, 2), "unsupported version"),
    "slab_alignment": (lambda b: struct.pack_into("<I", b, 56, 512), "slab alignment"),
    "truncated": (lambda b: b[:len(b) - 8192], "(in|out)side the file"),
    "directory_outside": (lambda b: struct.pack_into("<Q", b, 40, len(b)), "outside the file"),
    "expert_misaligned": (lambda b: struct.pack_into("<Q", b, _entry_pos(b, 9), expert_entries(b)[9]["off"] + 64),
                          "4096-aligned"),
    "expert_wrong_size": (lambda b: struct.pack_into("<Q", b, _entry_pos(b, 9) + 8, 8192), "expected 16384 bytes"),
    "two_owners": (lambda b: struct.pack_into("<I", b, _entry_pos(b, _first_alias(b)) + 20, 0),
                   "without the aliased flag"),
    "slabs_overlap": (lambda b: struct.pack_into("<Q", b, _entry_pos(b, 9), expert_entries(b)[8]["off"] + 4096),
                      "overlap"),
    "dense_layer_slab": (lambda b: struct.pack_into("<Q", b, _entry_pos(b, 0) + 8, 16384), "dense layer"),
    "tensor_size": (lambda b: struct.pack_into("<Q", b, tensor_entries(b)["blk.1.moe_router"]["entry"] + 112, 4),
                    "do not match"),
    "missing_key": (lambda b: b.__setitem__(slice(*_key_span(b, b"n_heads")), b"n_headz"), "missing required key n_heads"),
}


def _key_span(buf, key):
    p = preamble(buf)
    i = bytes(buf).index(struct.pack("<H", len(key)) + key, p["meta_off"], p["meta_off"] + p["meta_bytes"]) + 2
    return i, i + len(key)


@pytest.mark.parametrize("case", list(CORRUPTIONS))
def test_broken_files_are_refused(tmp_path, case):
    edit, msg = CORRUPTIONS[case]
    with pytest.raises(ValueError, match=msg):
        hb.container_probe(_patched(tmp_path, edit))


def test_unknown_metadata_type_is_refused(tmp_path):
    def edit(b):
        i, j = _key_span(b, b"top_k")
        b[j] = 9   # the type byte follows the key
    with pytest.raises(ValueError, match="unknown type"):
        hb.container_probe(_patched(tmp_path, edit))


def test_missing_file_is_an_io_error(tmp_path):
    with pytest.raises(OSError):
        hb.container_probe(tmp_path / "absent.hearth")
