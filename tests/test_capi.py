"""The C-ABI library loads and exports every entry point ``include/wiretorch_b200.h``
declares; its host-side argument checks reject bad sizes (no GPU needed for either)."""

import ctypes
import re
from pathlib import Path

import pytest

from wiretorch_b200 import _lib, build

HEADER = Path(__file__).parents[1] / "include" / "wiretorch_b200.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int32_t|int64_t|const char \*)\s*(wt_\w+)\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.lib()


def test_every_declared_entry_point_is_exported(lib):
    names = declared()
    assert names, "no entry points parsed from the header"
    for name in names:
        assert hasattr(lib, name), name


def test_abi_version(lib):
    assert lib.wt_abi_version() == 1


def test_structures_match_the_header_sizes():
    """The ctypes mirrors have the members the header declares, in order."""
    text = HEADER.read_text()
    from wiretorch_b200 import autograd, chunks, filtering, lowrank

    for struct, cls in (("WtNet", _lib.WtNet), ("WtForward", _lib.WtForward),
                        ("WtWorkspace", _lib.WtWorkspace),
                        ("WtBackward", autograd._BackwardArgs), ("WtEdgeGrads", autograd._EdgeArgs),
                        ("WtFilterArgs", filtering._FilterArgs),
                        ("WtFilterGradArgs", filtering._FilterGradArgs),
                        ("WtVanRossumArgs", filtering._VanRossumArgs),
                        ("WtVanRossumGradArgs", filtering._VanRossumGradArgs),
                        ("WtLowRankProduct", lowrank._ProductArgs),
                        ("WtLowRankNet", lowrank._LrNet), ("WtLowRankRun", lowrank._LrRun),
                        ("WtRecurrentCarry", autograd._CarryArgs),
                        ("WtSpikeBits", chunks._SpikeBits)):  # fmt: skip
        body = re.search(r"typedef struct \{((?:(?!typedef struct).)*?)\}\s*" + struct + ";", text,
                         re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        names = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            for part in decl.split(","):
                m = re.search(r"(\w+)\s*(\[[^\]]*\])?\s*$", part.strip())
                names.append(m.group(1))
        assert [f[0] for f in cls._fields_] == names, struct


def test_bad_sizes_are_rejected_without_a_gpu(lib):
    net = _lib.WtNet()
    net.B, net.N, net.S, net.C = 0, 10, 1, 1
    sizes = (ctypes.c_int64 * 6)()
    assert lib.wt_workspace_bytes(ctypes.byref(net), 10, sizes) == _lib.ERR_ARGS
    assert b"sizes" in lib.wt_last_error()
    net.B, net.S = 2, 9
    assert lib.wt_workspace_bytes(ctypes.byref(net), 10, sizes) == _lib.ERR_UNSUPPORTED
