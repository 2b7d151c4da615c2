"""The C ABI: libqi.so loads without a GPU, exports exactly what include/qi.h declares,
and rejects bad arguments on the host before launching anything."""

from __future__ import annotations

import ctypes as C
import re

import pytest

from conftest import REPO
from qweninfer_b200 import _lib

HEADER = REPO / "include" / "qi.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^(?:int|long long)\s+(qi_\w+)\(", text, flags=re.M))


@pytest.fixture(scope="module")
def lib():
    return _lib.load_library()


def test_header_and_binding_agree():
    assert declared_functions() == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version(lib):
    assert lib.qi_version() >= 100


def test_tile_offset_matches_host_repack(lib):
    import torch
    from qweninfer_b200.models.qwen2 import tile_weight
    N, K = 256, 192
    w = torch.arange(N * K, dtype=torch.int64).reshape(N, K)
    t = tile_weight(w)
    for n, k in [(0, 0), (1, 0), (0, 1), (7, 63), (8, 64), (127, 191), (128, 0), (255, 191), (37, 100)]:
        assert int(t[lib.qi_tile_offset(n, k, K)]) == n * K + k


def test_host_argument_checks_reject_before_launch(lib):
    E = _lib.QI_ERR_ARG
    # attention: split size must be a multiple of 128 and cover max_len
    assert lib.qi_attention(1, 1, 1, 1, 1, 1, 512, 100, 8, 1, 1, 1, 1, None) == E
    assert lib.qi_attention(1, 1, 1, 1, 1, 1, 512, 128, 2, 1, 1, 1, 1, None) == E
    # null operands
    assert lib.qi_o_proj_residual(None, 1, 4, 1, 1, None) == E
    assert lib.qi_down_residual(1, 1, 0, 1, 1, None) == E
    assert lib.qi_embed(None, 1000, 1, 1, 1, None, None, None) == E
    # lm_head: vocab must be a multiple of 128, logits row stride >= vocab
    assert lib.qi_lm_head_argmax(1, 896, 1, C.c_float(1e-6), 1, 1000, 1, None, 0, 0, 1, 1, None) == E
    assert lib.qi_lm_head_argmax(1, 896, 1, C.c_float(1e-6), 1, 1024, 1, 1, 0, 512, 1, 1, None) == E
    # row moves outside the cache
    bad = (C.c_int * 3)(0, 5, 10)
    assert lib.qi_move_rows(1, 1, 2, 4, 64, bad, 1, None) == E
    long = (C.c_int * 3)(0, 1, 65)
    assert lib.qi_move_rows(1, 1, 2, 4, 64, long, 1, None) == E
    # forward: null descriptors
    assert lib.qi_forward(None, None, None, 1, 1, 1, 1, 0, 1, 0, None, 0, 0, None, None) == E
    # tensor-core blocks: token tile must be a power of two in 8..128, rows % 128, K % 64
    assert lib.qi_act_tiles(1, None, 4, 896, 12, 1, None, 0, None) == E
    assert lib.qi_act_tiles(1, None, 4, 100, 8, 1, None, 0, None) == E
    assert lib.qi_tc_linear(1, 1000, 896, 1, 4, 8, None, 0, C.c_float(0), 1, 1000, 1, 10**6, 1, 64, 0, 1,
                            None) == E
    assert lib.qi_tc_linear(1, 1024, 896, 1, 4, 256, None, 0, C.c_float(0), 1, 1024, 1, 10**6, 1, 64, 0, 1,
                            None) == E
    # too few tile counters for 8 m-tiles
    assert lib.qi_tc_linear(1, 1024, 896, 1, 4, 8, None, 0, C.c_float(0), 1, 1024, 1, 10**6, 1, 4, 0, 1,
                            None) == E


def test_cpu_tensors_are_refused():
    import torch
    from qweninfer_b200.models.qwen2 import RMSNorm
    with pytest.raises(_lib.QiError):
        RMSNorm(896)(torch.zeros(2, 896))
