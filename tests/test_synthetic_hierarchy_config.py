"""Hierarchy config of the synthetic data generator (behaviour of sae_lens/synthetic hierarchy
config; cases follow tests/synthetic/hierarchy/test_config.py)."""

import pytest

from saelens_b200.synthetic.generation import HierarchyConfig


def test_defaults():
    c = HierarchyConfig()
    assert (c.total_root_nodes, c.branching_factor, c.max_depth) == (100, 100, 2)
    assert c.mutually_exclusive_portion == 0.0 and c.mutually_exclusive_min_depth == 0
    assert c.mutually_exclusive_max_depth is None and c.compensate_probabilities is False


@pytest.mark.parametrize("kw,msg", [
    ({"total_root_nodes": -1}, "total_root_nodes must be positive"),
    ({"total_root_nodes": 0}, "total_root_nodes must be positive"),
    ({"branching_factor": 1}, "branching_factor must be at least 2"),
    ({"branching_factor": (1, 4)}, "branching_factor minimum must be at least 2"),
    ({"branching_factor": (5, 3)}, r"branching_factor\[0\] must be <= branching_factor\[1\]"),
    ({"max_depth": 0}, "max_depth must be at least 1"),
    ({"mutually_exclusive_portion": 1.5}, "mutually_exclusive_portion must be between 0.0 and 1.0"),
    ({"mutually_exclusive_min_depth": -1}, "mutually_exclusive_min_depth must be non-negative"),
    ({"mutually_exclusive_min_depth": 2, "mutually_exclusive_max_depth": 1},
     "mutually_exclusive_max_depth must be >= mutually_exclusive_min_depth"),
])
def test_validation(kw, msg):
    with pytest.raises(ValueError, match=msg):
        HierarchyConfig(**{"total_root_nodes": 5, **kw})


def test_dict_roundtrip():
    c = HierarchyConfig(total_root_nodes=7, branching_factor=(2, 5), max_depth=3, mutually_exclusive_portion=0.25,
                        mutually_exclusive_min_depth=1, mutually_exclusive_max_depth=2, compensate_probabilities=True)
    d = c.to_dict()
    assert d["branching_factor"] == [2, 5] and d["compensate_probabilities"] is True
    assert HierarchyConfig.from_dict(d) == c
    assert HierarchyConfig.from_dict(HierarchyConfig().to_dict()).compensate_probabilities is False
