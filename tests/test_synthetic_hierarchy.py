"""Statistical behaviour of the synthetic hierarchy (role of the reference's
tests/synthetic/test_hierarchy*.py): gating through organisational nodes, mutual exclusion with a
uniform winner, parent rescaling, structural validation, and probability compensation restoring
the base firing rates of gated children."""

import pytest
import torch

import saelens_b200.synthetic as S


def _acts(n_rows, p, n_feat, seed=0, value=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(n_rows, n_feat, generator=g) < p).float() * value


def test_children_of_an_organisational_node_are_gated_by_the_nearest_feature_ancestor():
    tree = S.HierarchyNode(0, [S.HierarchyNode(None, [S.HierarchyNode(1), S.HierarchyNode(2, [S.HierarchyNode(3)])])])
    x = _acts(20000, 0.5, 4)
    y = S.hierarchy_modifier(tree)(x)
    off = y[:, 0] == 0
    assert bool((y[off][:, 1:] == 0).all())
    assert bool((y[y[:, 2] == 0][:, 3] == 0).all())
    on = (x[:, 0] > 0) & (x[:, 2] > 0)
    assert torch.equal(y[on][:, 3], x[on][:, 3])  # untouched where every ancestor fires


def test_mutual_exclusion_keeps_one_uniformly_random_active_child():
    torch.manual_seed(0)
    tree = S.HierarchyNode(0, [S.HierarchyNode(i) for i in (1, 2, 3)], mutually_exclusive_children=True)
    x = torch.ones(30000, 4)
    y = S.hierarchy_modifier(tree)(x)
    assert bool(((y[:, 1:] > 0).sum(1) == 1).all())
    share = (y[:, 1:] > 0).float().mean(0)
    assert torch.allclose(share, torch.full((3,), 1 / 3), atol=0.02)
    x[:, 0] = 0  # parent off: every child off, no exclusion needed
    assert bool((S.hierarchy_modifier(tree)(x)[:, 1:] == 0).all())


def test_exclusion_under_an_organisational_root_without_a_parent_feature():
    tree = S.HierarchyNode(None, [S.HierarchyNode(0), S.HierarchyNode(1)], mutually_exclusive_children=True)
    y = S.hierarchy_modifier(tree)(torch.ones(1000, 2))
    assert bool(((y > 0).sum(1) == 1).all())


def test_children_rescaled_by_parent_over_its_mean():
    gen = S.ActivationGenerator(3, 0.5, mean_firing_magnitudes=torch.tensor([2.0, 1.0, 1.0]))
    tree = S.HierarchyNode(0, [S.HierarchyNode(1), S.HierarchyNode(2)], scale_children_by_parent=True)
    x = torch.tensor([[4.0, 1.0, 3.0], [0.0, 1.0, 1.0]])
    y = S.hierarchy_modifier(tree)(x, gen)
    assert torch.allclose(y, torch.tensor([[4.0, 2.0, 6.0], [0.0, 0.0, 0.0]]))
    with pytest.raises(ValueError, match="mean firing magnitudes"):
        S.hierarchy_modifier(tree)(x)


def test_validation_rejects_shared_nodes_repeated_indices_and_small_exclusive_groups():
    shared = S.HierarchyNode(5)
    with pytest.raises(ValueError, match="more than one parent"):
        S.validate_hierarchy([S.HierarchyNode(0, [shared]), S.HierarchyNode(1, [shared])])
    with pytest.raises(ValueError, match="more than once"):
        S.validate_hierarchy([S.HierarchyNode(0, [S.HierarchyNode(1)]), S.HierarchyNode(1)])
    with pytest.raises(ValueError, match="at least 2 children"):
        S.hierarchy_modifier(S.HierarchyNode(0, [S.HierarchyNode(1)], mutually_exclusive_children=True))
    loop = S.HierarchyNode(0)
    loop.children = [S.HierarchyNode(1, [loop])]
    with pytest.raises(ValueError, match="loop"):
        S.validate_hierarchy([loop])


def test_sparse_input_gives_the_dense_result():
    tree = S.HierarchyNode(0, [S.HierarchyNode(1), S.HierarchyNode(2, [S.HierarchyNode(3)])])
    x = _acts(500, 0.5, 4, seed=3)
    mod = S.hierarchy_modifier(tree)
    assert torch.equal(mod(x.to_sparse()).to_dense(), mod(x))


def test_compensation_restores_the_base_rates_of_gated_children():
    """Gated children fire at their base probability once the correction factors are applied
    (child rate = corrected child probability x parent probability)."""
    base = torch.tensor([0.5, 0.1, 0.2, 0.05])
    tree = S.HierarchyNode(0, [S.HierarchyNode(1), S.HierarchyNode(2, [S.HierarchyNode(3)])])
    h = S.Hierarchy(roots=[tree], modifier=S.hierarchy_modifier(tree))
    probs = (base * h.compute_probability_correction_factors(base)).clamp(max=1.0)
    gen = S.ActivationGenerator(4, probs, modify_activations=h.modifier)
    torch.manual_seed(0)
    rate = torch.cat([(gen.sample(20000) > 0).float() for _ in range(5)]).mean(0)
    assert torch.allclose(rate, base, atol=0.01)
