"""Autotune cache and the library's per-shape configuration table, on the host (no GPU): the C table's set /
get / clear contract and argument checks, candidate generation, and the JSON cache round trip."""
import json

import pytest

from periodicdent42_b200 import _capi
from periodicdent42_b200 import autotune as at


@pytest.fixture(autouse=True)
def _clean_table():
    at.clear()
    yield
    at.clear()


def test_config_table_set_get_clear():
    assert at.registered("gemm_f16f32", 8192, 1024, 237568) is None
    at.register("gemm_f16f32", 8192, 1024, 237568, 2, 16)
    at.register("spmm_bsr", 8192, 8192, 8192, -1, 8)
    assert at.registered("gemm_f16f32", 8192, 1024, 237568) == (2, 16)
    assert at.registered("spmm_bsr", 8192, 8192, 8192) == (-1, 8)
    assert at.registered("gemm_e4m3_bf16", 8192, 1024, 237568) is None  # keyed by operator too
    at.register("gemm_f16f32", 8192, 1024, 237568, 1, 0)  # overwrite
    assert at.registered("gemm_f16f32", 8192, 1024, 237568) == (1, 0)
    at.clear()
    assert at.registered("spmm_bsr", 8192, 8192, 8192) is None


@pytest.mark.parametrize("args", [(9, 1, 1, 1, 0, 0), (1, 1, 1, 1, 3, 0), (1, 1, 1, 1, 0, -1), (1, -1, 1, 1, 0, 0),
                                  (1, 1, 1, 1, 0, 5000)])
def test_config_set_rejects_bad_arguments(args):
    assert _capi.lib().bsk_config_set(*args) == _capi.BSK_ERR_INVALID_ARG


def test_candidates():
    c = at.candidates("gemm_f16f32", 8192, 8192, 237568)
    assert c[0] == (-1, 0) and {t for t, _ in c} == {-1, 0, 1, 2}
    assert len(set(c)) == len(c)
    small = at.candidates("gemm_f16f32", 256, 256, 64)  # one or two M tiles: few distinct groups
    assert len(small) < len(c)
    assert {t for t, _ in at.candidates("spmm_bsr", 8192, 8192, 8192)} == {-1, 0, 1}
    assert {t for t, _ in at.candidates("spmm_bsr", 8192, 256, 8192)} == {-1}
    assert {t for t, _ in at.candidates("spmm_bsr_bsr", 8192, 8192, 8192)} == {-1}


def test_shape_keys_round_trip():
    k = at.shape_key("spmm_bsr_bsr", 1024, 2048, 4096)
    assert at.parse_shape_key(k) == ("spmm_bsr_bsr", 1024, 2048, 4096)
    with pytest.raises(ValueError):
        at.shape_key("nope", 1, 1, 1)


def test_cache_file_round_trip(tmp_path):
    path = str(tmp_path / "sub" / "cache.json")
    c = at.AutotuneCache(path)
    c.put("dev-A", at.shape_key("gemm_f16f32", 512, 512, 4096), {"tile": 1, "group_m": 4, "ms": 0.1})
    c.put("dev-B", at.shape_key("gemm_f16f32", 512, 512, 4096), {"tile": 2, "group_m": 8, "ms": 0.2})
    c.save()
    data = json.load(open(path))
    assert data["dev-A"]["gemm_f16f32:512x512x4096"]["tile"] == 1
    c2 = at.AutotuneCache(path)
    assert c2.get("dev-B", "gemm_f16f32:512x512x4096")["group_m"] == 8
    assert c2.get("dev-C", "gemm_f16f32:512x512x4096") is None
