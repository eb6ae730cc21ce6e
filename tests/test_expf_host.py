"""The device expf restatement (hearth_b200/csrc/hx_common.cuh host_expf), compiled for the host,
checked against the host C library's expf on every one of the 2^32 float inputs, and its table
recomputed from the mathematics."""
import ctypes as C
import os
from decimal import Decimal, getcontext
import struct

import numpy as np

from tests.native.build import build_expf_check


def _lib():
    L = C.CDLL(build_expf_check())
    L.hxt_expf_mismatches.restype = C.c_longlong
    L.hxt_expf_mismatches.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.POINTER(C.c_uint32)]
    L.hxt_exp2_table.argtypes = [C.c_void_p]
    return L


def test_exp2_table_is_two_to_the_i_over_32():
    getcontext().prec = 60
    tab = np.zeros(32, np.uint64)
    _lib().hxt_exp2_table(tab.ctypes.data)
    for i in range(32):
        d = float(str(Decimal(2) ** (Decimal(i) / Decimal(32))))   # correctly rounded double
        u = struct.unpack("<Q", struct.pack("<d", d))[0]
        assert int(tab[i]) == (u - (i << 47)) & 0xFFFFFFFFFFFFFFFF


def test_expf_restatement_equals_host_libm_on_all_inputs():
    n = max(2, min(os.cpu_count() or 2, 64))
    bad = C.c_uint32(0)
    mism = _lib().hxt_expf_mismatches(0, 1 << 32, n, C.byref(bad))
    assert mism == 0, f"{mism} mismatches, first at 0x{bad.value:08x}"
