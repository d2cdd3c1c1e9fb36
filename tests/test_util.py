"""Small helpers (behaviour of sae_lens/util.py; cases follow tests/test_util.py)."""

from dataclasses import dataclass
from pathlib import Path

import pytest
import torch

from saelens_b200.utils.misc import (
    cosine_similarities,
    dtype_to_str,
    extract_stop_at_layer_from_tlens_hook_name,
    filter_valid_dataclass_fields,
    get_special_token_ids,
    path_or_tmp_dir,
    str_to_dtype,
    temporary_seed,
)


@pytest.mark.parametrize("name,layer", [("blocks.0.attn.hook_q", 1), ("blocks.12.attn.hook_k", 13),
                                        ("blocks.999.attn.hook_v", 1000), ("blocks.42.mlp.hook_pre", 43)])
def test_stop_at_layer_valid(name, layer):
    assert extract_stop_at_layer_from_tlens_hook_name(name) == layer


@pytest.mark.parametrize("name", ["blocks.attn.hook_q", "blocks..attn.hook_q", "hook_q", "blocks.abc.attn.hook_q", ""])
def test_stop_at_layer_invalid(name):
    assert extract_stop_at_layer_from_tlens_hook_name(name) is None


def test_path_or_tmp_dir(tmp_path):
    with path_or_tmp_dir(None) as p:
        assert p.exists() and p.is_dir()
        kept = p
    assert not kept.exists()
    with path_or_tmp_dir(tmp_path) as p:
        assert p == tmp_path
    with path_or_tmp_dir(str(tmp_path)) as p:
        assert isinstance(p, Path) and p == tmp_path
    assert tmp_path.exists()


def test_special_token_ids():
    class Tok:
        bos_token_id, eos_token_id, pad_token_id, unk_token_id = 1, 2, 2, None
        all_special_ids = [1, 2, 7]

    assert get_special_token_ids(Tok()) == [1, 2, 7]


@pytest.mark.parametrize("s,dt", [("float32", torch.float32), ("float64", torch.float64), ("float16", torch.float16),
                                  ("bfloat16", torch.bfloat16), ("torch.float32", torch.float32),
                                  ("torch.bfloat16", torch.bfloat16)])
def test_str_to_dtype(s, dt):
    assert str_to_dtype(s) == dt
    assert dtype_to_str(dt) in s


@pytest.mark.parametrize("bad", ["invalid", "float33", "int32", "torch.int32", "", "FLOAT32"])
def test_str_to_dtype_invalid(bad):
    with pytest.raises(ValueError, match="Invalid dtype"):
        str_to_dtype(bad)


@pytest.mark.parametrize("bad", [torch.int32, torch.int64, torch.complex64, torch.bool])
def test_dtype_to_str_invalid(bad):
    with pytest.raises(ValueError, match="Invalid dtype"):
        dtype_to_str(bad)


def test_cosine_similarities():
    torch.manual_seed(0)
    m = torch.randn(5, 10)
    c = cosine_similarities(m)
    torch.testing.assert_close(torch.diag(c), torch.ones(5))
    torch.testing.assert_close(c, c.T)
    assert c.min() >= -1 - 1e-6 and c.max() <= 1 + 1e-6
    assert cosine_similarities(m, torch.randn(3, 10)).shape == (5, 3)
    torch.testing.assert_close(cosine_similarities(m, -m).diag(), -torch.ones(5))
    torch.testing.assert_close(cosine_similarities(m, 7 * m), c)
    e = torch.eye(3, 10)
    torch.testing.assert_close(cosine_similarities(e), torch.eye(3))
    z = torch.randn(3, 10)
    z[0] = 0.0
    z[1] = 1e-10
    assert torch.isfinite(cosine_similarities(torch.randn(3, 10), z)).all()


@dataclass
class _Dest:
    field_a: int
    field_b: str


@dataclass
class _Src:
    field_a: int
    field_b: str
    field_c: float


def test_filter_valid_dataclass_fields():
    src = {"field_a": 1, "field_b": "hello", "field_c": 3.14}
    assert filter_valid_dataclass_fields(src, _Dest) == {"field_a": 1, "field_b": "hello"}
    assert filter_valid_dataclass_fields(_Src(1, "hello", 3.14), _Dest) == {"field_a": 1, "field_b": "hello"}
    assert filter_valid_dataclass_fields(src, _Dest, whitelist_fields=["field_c"]) == src
    with pytest.raises(ValueError, match="is not a dataclass"):
        filter_valid_dataclass_fields({"field_a": 1}, "not a dataclass")
    with pytest.raises(ValueError, match="is not a dict or dataclass"):
        filter_valid_dataclass_fields("invalid source", _Dest)


def test_temporary_seed():
    with temporary_seed(42):
        a = torch.randn(100)
    with temporary_seed(42):
        b = torch.randn(100)
    assert torch.equal(a, b)
    torch.randn(1)
    before = torch.random.get_rng_state()
    with temporary_seed(99):
        torch.randn(1000)
    assert torch.equal(torch.random.get_rng_state(), before)
    with temporary_seed(None):
        torch.randn(1)
    assert not torch.equal(torch.random.get_rng_state(), before)
