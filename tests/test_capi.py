"""The C-ABI library loads, exports every symbol the header declares, and rejects
bad arguments with status codes (validation only: no kernel is launched)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from silogic_b200 import _lib

HEADER = os.path.join(ROOT, "include", "silogic_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(?:int|int64_t|const char\*)\s+(slg_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(_lib.LIB_PATH):
        from silogic_b200 import build
        build.build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(L):
    names = _declared()
    assert len(names) >= 8
    for n in names:
        assert hasattr(L, n), n


def test_version(L):
    assert L.slg_version() >= 100


def _p(v):
    return ctypes.c_void_p(v)


def test_bad_arguments_are_rejected(L):
    # odd leading dimension
    st = L.slg_fc_hard(_p(256), 10, 3, _p(512), _p(1024), 2, 10, 0, _p(2048), _p(0))
    assert st == 2 and b"even" in L.slg_last_error()
    # misaligned pointer
    st = L.slg_fc_hard(_p(258), 10, 2, _p(512), _p(1024), 2, 10, 0, _p(2048), _p(0))
    assert st == 2
    # unsupported arity
    st = L.slg_fc_hard(_p(256), 10, 2, _p(512), _p(1024), 7, 10, 0, _p(2048), _p(0))
    assert st == 3
    # conv tree shape not built
    st = L.slg_conv_hard(_p(256), 4, 8, 8, 2, _p(512), _p(1024), 2, 7, 3, 1, 4, 0, 2, _p(2048), _p(0))
    assert st == 3
    # groupsum: width not divisible
    st = L.slg_groupsum(_p(256), 11, 2, 64, 10, _p(512), _p(0))
    assert st == 1
    # empty work is a no-op success
    assert L.slg_pack_u8(_p(0), 0, 5, _p(0), 2, _p(0)) == 0
