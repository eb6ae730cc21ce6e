"""A minimal, independent reader of the .hearth preamble and expert directory (FORMAT §2, §5 of the
reference), used by the tests to locate and patch entries and to read slabs back for the oracle."""
import struct

import numpy as np

FIXTURE = "tests/golden/tiny_moe.hearth"
FIXTURE_NPZ = "tests/golden/tiny_moe.npz"


def preamble(buf):
    magic, version, meta_off, meta_bytes, tdir_off, n_tensors, edir_off, n_entries, align, _ = struct.unpack_from(
        "<IIQQQQQQII", buf, 0)
    return dict(magic=magic, version=version, meta_off=meta_off, meta_bytes=meta_bytes, tdir_off=tdir_off,
                n_tensors=n_tensors, edir_off=edir_off, n_entries=n_entries, align=align)


def expert_entries(buf):
    p = preamble(buf)
    out = []
    for i in range(p["n_entries"]):
        off, nbytes, dtype, flags, _ = struct.unpack_from("<QQIIQ", buf, p["edir_off"] + 32 * i)
        out.append(dict(off=off, nbytes=nbytes, dtype=dtype, flags=flags))
    return out


def tensor_entries(buf):
    p = preamble(buf)
    out = {}
    for i in range(p["n_tensors"]):
        base = p["tdir_off"] + 128 * i
        name = bytes(buf[base:base + 80]).split(b"\0")[0].decode()
        dtype, ndim = struct.unpack_from("<II", buf, base + 80)
        off, nbytes = struct.unpack_from("<QQ", buf, base + 104)
        out[name] = dict(index=i, entry=base, dtype=dtype, ndim=ndim, off=off, nbytes=nbytes)
    return out


def fixture_layers(path=FIXTURE, npz=FIXTURE_NPZ, n_experts=8):
    """The fixture's MoE layers (1 and 2) in tests.moe_util's layer format, slabs read from the file
    (an aliased entry gets its target's bytes)."""
    buf = open(path, "rb").read()
    ents = expert_entries(buf)
    w = np.load(npz)
    layers = []
    for i, l in enumerate((1, 2)):
        slabs = []
        for e in range(n_experts):
            x = ents[l * n_experts + e]
            slabs.append(np.frombuffer(buf[x["off"]:x["off"] + x["nbytes"]], np.uint8))
        shared = dict(Fs=64, dtype=3, gate=w["sh_gate"][i], up=w["sh_up"][i], down=w["sh_down"][i], gate_inp=None)
        layers.append(dict(router=w["router"][i], bias=w["bias"][i], norm=w["norm"][i], slabs=slabs, shared=shared))
    return layers


FIXTURE_KW = dict(D=128, F=64, E=8, K=2, score_fn=1, score_bias=1, n_group=4, topk_group=2, norm=1,
                  routed_scale=2.5, residual_scale=0.5)
