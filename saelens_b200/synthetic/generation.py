"""Feature dictionary, activation generator and feature hierarchy for synthetic SAE data (roles of
sae_lens/synthetic/feature_dictionary.py, activation_generator.py, hierarchy/*).

Data model: a sample is a sparse vector of feature activations f (feature i fires with its
probability, possibly correlated with others through a Gaussian copula; a firing feature takes
relu(mean_i + std_i * N(0, 1))), optionally passed through modifiers such as a hierarchy
(children are silenced when their parent is silent, siblings may be mutually exclusive), then
mapped to a dense hidden vector h = f @ D + b by the feature dictionary D.
"""

from __future__ import annotations

import inspect

import random
from collections.abc import Callable, Sequence
from dataclasses import asdict, dataclass, field
from typing import Any, Union

import torch
from torch import nn

from saelens_b200.synthetic.distributions import LowRankCorrelationMatrix, correlation_thresholds
from saelens_b200.utils.misc import str_to_dtype

FeatureDictionaryInitializer = Callable[["FeatureDictionary"], None]
ActivationsModifier = Callable[..., torch.Tensor]
ActivationsModifierInput = Union[ActivationsModifier, Sequence[ActivationsModifier], None]
CorrelationMatrixInput = Union[torch.Tensor, LowRankCorrelationMatrix, tuple[torch.Tensor, torch.Tensor]]


# ------------------------------------------------------------------------------ dictionary
def orthogonalize_embeddings(embeddings: torch.Tensor, num_steps: int = 200, lr: float = 0.01,
                             show_progress: bool = False, chunk_size: int = 1024) -> torch.Tensor:
    """Reduce pairwise cosine similarity of unit rows by gradient descent on sum_{i != j} (e_i . e_j)^2,
    renormalising after every step.  With n <= d the rows become exactly orthonormal (QR)."""
    n, d = embeddings.shape
    if n <= d:
        q, _ = torch.linalg.qr(embeddings.T.float())
        return q.T.contiguous().to(embeddings.dtype)
    e = (embeddings / embeddings.norm(dim=1, keepdim=True).clamp(min=1e-8)).float().clone()
    steps = range(num_steps)
    if show_progress:
        from tqdm.auto import tqdm

        steps = tqdm(steps, desc="orthogonalizing")
    for _ in steps:
        grad = torch.zeros_like(e)
        for s in range(0, n, chunk_size):
            blk = e[s : s + chunk_size]
            g = blk @ e.T
            g[:, s : s + chunk_size].fill_diagonal_(0.0)
            grad[s : s + chunk_size] = g @ e
        e = e - lr * grad / n
        e = e / e.norm(dim=1, keepdim=True).clamp(min=1e-8)
    return e.to(embeddings.dtype)


def orthogonal_initializer(num_steps: int = 200, lr: float = 0.01, show_progress: bool = False,
                           chunk_size: int = 1024) -> FeatureDictionaryInitializer:
    def init(fd: "FeatureDictionary") -> None:
        with torch.no_grad():
            fd.feature_vectors.copy_(orthogonalize_embeddings(fd.feature_vectors.data, num_steps=num_steps, lr=lr,
                                                              show_progress=show_progress, chunk_size=chunk_size))

    return init


class FeatureDictionary(nn.Module):
    """Maps feature activations [batch, num_features] (dense or sparse COO) to hidden activations
    [batch, hidden_dim]: h = f @ feature_vectors + bias, with unit-norm feature vectors."""

    def __init__(self, num_features: int, hidden_dim: int, bias: bool | float = False,
                 initializer: FeatureDictionaryInitializer | None = None, device: str | torch.device = "cpu",
                 seed: int | None = None):
        super().__init__()
        self.num_features = num_features
        self.hidden_dim = hidden_dim
        g = torch.Generator(device=device)
        if seed is not None:
            g.manual_seed(seed)
        e = torch.randn(num_features, hidden_dim, device=device, generator=g)
        self.feature_vectors = nn.Parameter(e / e.norm(dim=1, keepdim=True).clamp(min=1e-8))
        if bias:
            b = torch.randn(hidden_dim, device=device, generator=g)
            self.bias = nn.Parameter(b / b.norm().clamp(min=1e-8) * (1.0 if bias is True else float(bias)))
        else:
            self.bias = nn.Parameter(torch.zeros(hidden_dim, device=device), requires_grad=False)
        if initializer is not None:
            initializer(self)

    def forward(self, feature_activations: torch.Tensor) -> torch.Tensor:
        if feature_activations.is_sparse:
            with torch.autocast(device_type=feature_activations.device.type, enabled=False):
                return torch.sparse.mm(feature_activations.float(), self.feature_vectors.float()) + self.bias
        return feature_activations.to(self.feature_vectors.dtype) @ self.feature_vectors + self.bias


# ------------------------------------------------------------------------------ generator
def _vec(v: torch.Tensor | float, n: int, device: Any, dtype: torch.dtype) -> torch.Tensor:
    if isinstance(v, torch.Tensor):
        if v.numel() == 1:
            return v.reshape(()).to(device=device, dtype=dtype).expand(n).clone()
        if v.shape != (n,):
            raise ValueError(f"expected a tensor of shape ({n},), got {tuple(v.shape)}")
        return v.to(device=device, dtype=dtype)
    return torch.full((n,), float(v), device=device, dtype=dtype)


def _modifier_chain(mods: ActivationsModifierInput) -> Callable[[torch.Tensor, Any], torch.Tensor] | None:
    if mods is None:
        return None
    mods = [mods] if callable(mods) else list(mods)
    if not mods:
        return None

    takes_gen = [_positional_arity(m) >= 2 for m in mods]

    def chained(x: torch.Tensor, gen: Any) -> torch.Tensor:
        for m, two in zip(mods, takes_gen):
            x = m(x, gen) if two else m(x)
        return x

    return chained


def _positional_arity(fn: Callable[..., Any]) -> int:
    """Positional parameters `fn` accepts (a *args parameter counts as many): a modifier taking two
    receives the generator as its second argument, one taking one only the activations."""
    try:
        params = inspect.signature(fn).parameters.values()
    except (TypeError, ValueError):  # builtins without a signature: activations only
        return 1
    n = 0
    for p in params:
        if p.kind is inspect.Parameter.VAR_POSITIONAL:
            return 2
        if p.kind in (inspect.Parameter.POSITIONAL_ONLY, inspect.Parameter.POSITIONAL_OR_KEYWORD):
            n += 1
    return n


class ActivationGenerator(nn.Module):
    """Samples synthetic feature activations [batch, num_features] (non-negative)."""

    def __init__(self, num_features: int, firing_probabilities: torch.Tensor | float,
                 std_firing_magnitudes: torch.Tensor | float = 0.0, mean_firing_magnitudes: torch.Tensor | float = 1.0,
                 modify_activations: ActivationsModifierInput = None,
                 correlation_matrix: CorrelationMatrixInput | None = None, device: torch.device | str = "cpu",
                 dtype: torch.dtype | str = "float32", use_sparse_tensors: bool = False):
        super().__init__()
        dt = str_to_dtype(dtype) if isinstance(dtype, str) else dtype
        self.num_features = num_features
        self.firing_probabilities = _vec(firing_probabilities, num_features, device, dt)
        if (self.firing_probabilities < 0).any() or (self.firing_probabilities > 1).any():
            raise ValueError("firing probabilities must lie in [0, 1]")
        self.std_firing_magnitudes = _vec(std_firing_magnitudes, num_features, device, dt)
        self.mean_firing_magnitudes = _vec(mean_firing_magnitudes, num_features, device, dt)
        self.modify_activations = _modifier_chain(modify_activations)
        self.use_sparse_tensors = use_sparse_tensors
        self.correlation_matrix: torch.Tensor | None = None
        self.low_rank_correlation: tuple[torch.Tensor, torch.Tensor] | None = None
        self.correlation_thresholds: torch.Tensor | None = None
        if correlation_matrix is not None:
            if isinstance(correlation_matrix, torch.Tensor):
                c = correlation_matrix
                if c.shape != (num_features, num_features):
                    raise ValueError("correlation matrix must be [num_features, num_features]")
                if not torch.allclose(c, c.T, atol=1e-5) or not torch.allclose(c.diagonal(), torch.ones_like(c.diagonal()), atol=1e-4):
                    raise ValueError("correlation matrix must be symmetric with a unit diagonal")
                self.correlation_matrix = c.to(device=device, dtype=torch.float32)
                chol, info = torch.linalg.cholesky_ex(self.correlation_matrix.double() +
                                                      1e-9 * torch.eye(num_features, device=device,
                                                                       dtype=torch.float64))
                if int(info) != 0:
                    raise ValueError("correlation matrix must be positive definite")
                self._chol = chol.float()
            else:
                f, d = correlation_matrix[0], correlation_matrix[1]
                if f.shape[0] != num_features or d.shape != (num_features,):
                    raise ValueError("low-rank correlation must be (factor [n, r], diag [n])")
                if f.dim() != 2 or d.dim() != 1:
                    raise ValueError("low-rank correlation must be (factor [n, r], diag [n])")
                if (d <= 0).any():
                    raise ValueError("low-rank correlation diagonal must be positive")
                self.low_rank_correlation = (f.to(device=device, dtype=torch.float32),
                                             d.to(device=device, dtype=torch.float32).sqrt())
            self.correlation_thresholds = correlation_thresholds(self.firing_probabilities.float())

    def _firing_positions(self, batch_size: int) -> tuple[torch.Tensor, torch.Tensor]:
        dev = self.firing_probabilities.device
        if self.correlation_matrix is not None:
            z = torch.randn(batch_size, self.num_features, device=dev) @ self._chol.T
            return (z > self.correlation_thresholds).nonzero(as_tuple=True)
        if self.low_rank_correlation is not None:
            f, dsq = self.low_rank_correlation
            z = torch.randn(batch_size, f.shape[1], device=dev) @ f.T + torch.randn(batch_size, self.num_features,
                                                                                     device=dev) * dsq
            return (z > self.correlation_thresholds).nonzero(as_tuple=True)
        u = torch.rand(batch_size, self.num_features, device=dev)
        return (u < self.firing_probabilities).nonzero(as_tuple=True)

    @torch.no_grad()
    def sample(self, batch_size: int) -> torch.Tensor:
        rows, cols = self._firing_positions(batch_size)
        mean = self.mean_firing_magnitudes[cols]
        vals = (mean + torch.randn_like(mean) * self.std_firing_magnitudes[cols]).relu()
        if self.use_sparse_tensors:
            acts = torch.sparse_coo_tensor(torch.stack([rows, cols]), vals, (batch_size, self.num_features))
        else:
            acts = torch.zeros(batch_size, self.num_features, device=vals.device, dtype=vals.dtype)
            acts[rows, cols] = vals
        if self.modify_activations is not None:
            acts = self.modify_activations(acts, self)
            if acts.is_sparse:
                acts = acts.coalesce()
                acts = torch.sparse_coo_tensor(acts.indices(), acts.values().relu(), acts.shape)
            else:
                acts = acts.relu()
        return acts

    def forward(self, batch_size: int) -> torch.Tensor:
        return self.sample(batch_size)


# ------------------------------------------------------------------------------ hierarchy
class HierarchyNode:
    """A feature in a hierarchy tree.  Children fire only when this feature fires (or are rescaled
    by parent_activation / parent_mean with scale_children_by_parent); with
    mutually_exclusive_children at most one child stays active per sample (a uniformly random one
    among those that fired).  feature_index None marks an organisational node."""

    def __init__(self, feature_index: int | None = None, children: Sequence["HierarchyNode"] | None = None,
                 mutually_exclusive_children: bool = False, scale_children_by_parent: bool = False,
                 feature_id: str | None = None):
        self.feature_index = feature_index
        self.children = list(children or [])
        self.mutually_exclusive_children = mutually_exclusive_children
        self.scale_children_by_parent = scale_children_by_parent
        self.feature_id = feature_id

    @classmethod
    def from_dict(cls, tree_dict: dict[str, Any]) -> "HierarchyNode":
        d = tree_dict
        return cls(feature_index=d.get("feature_index"), children=[cls.from_dict(c) for c in d.get("children", [])],
                   mutually_exclusive_children=d.get("mutually_exclusive_children", False),
                   scale_children_by_parent=d.get("scale_children_by_parent", False), feature_id=d.get("id"))

    def to_dict(self) -> dict[str, Any]:
        d: dict[str, Any] = {"feature_index": self.feature_index}
        if self.children:
            d["children"] = [c.to_dict() for c in self.children]
        if self.mutually_exclusive_children:
            d["mutually_exclusive_children"] = True
        if self.scale_children_by_parent:
            d["scale_children_by_parent"] = True
        if self.feature_id is not None:
            d["id"] = self.feature_id
        return d

    def get_all_feature_indices(self) -> list[int]:
        out = [] if self.feature_index is None else [self.feature_index]
        for c in self.children:
            out.extend(c.get_all_feature_indices())
        return out

    def validate(self) -> None:
        validate_hierarchy([self])

    def __eq__(self, other: object) -> bool:
        return isinstance(other, HierarchyNode) and self.to_dict() == other.to_dict()

    def __repr__(self, indent: int = 0) -> str:
        s = " " * indent + f"HierarchyNode({self.feature_index}{', ME' if self.mutually_exclusive_children else ''})"
        return "\n".join([s] + [c.__repr__(indent + 2) for c in self.children])


def validate_hierarchy(roots: Sequence[HierarchyNode]) -> None:
    """A forest is valid when no node is its own ancestor, no node object sits in two children
    lists (one parent per node), no feature index appears twice and every mutually exclusive node
    has at least two children (sae_lens/synthetic/hierarchy/validation.py)."""
    seen_nodes: set[int] = set()
    seen_feats: set[int] = set()

    def visit(n: HierarchyNode, path: set[int]) -> None:
        if id(n) in path:
            raise ValueError(f"hierarchy has a loop through feature {n.feature_index}")
        if id(n) in seen_nodes:
            raise ValueError(f"hierarchy node for feature {n.feature_index} has more than one parent")
        seen_nodes.add(id(n))
        if n.feature_index is not None:
            if n.feature_index in seen_feats:
                raise ValueError(f"feature index {n.feature_index} appears more than once in the hierarchy")
            seen_feats.add(n.feature_index)
        if n.mutually_exclusive_children and len(n.children) < 2:
            raise ValueError("mutual exclusion needs at least 2 children")
        for c in n.children:
            visit(c, path | {id(n)})

    for r in roots:
        visit(r, set())


class _HierarchyPlan:
    """Index tensors of a validated forest, level by level (breadth-first depth of each node).

    Every feature node gets an effective parent: the nearest ancestor that has a feature index
    (-1 under a root or a chain of organisational nodes).  Its activation is gated by that parent
    (x *= [parent > 0]), or rescaled (x *= parent / mean(parent)) when its immediate parent node has
    scale_children_by_parent.  A mutually exclusive node's feature children form one group, applied
    right after the gating of the node's own level: where more than one member is active (and the
    group's effective parent is active) a uniformly random active member is kept."""

    def __init__(self, roots: Sequence[HierarchyNode]):
        feats: dict[int, list[tuple[int, int, bool]]] = {}
        groups: dict[int, list[tuple[int, list[int]]]] = {}
        queue: list[tuple[HierarchyNode, int, int]] = [(r, -1, 0) for r in roots]
        head = 0
        while head < len(queue):
            node, eff_parent, level = queue[head]
            head += 1
            own = node.feature_index if node.feature_index is not None else eff_parent
            for c in node.children:
                if c.feature_index is not None:
                    feats.setdefault(level + 1, []).append((c.feature_index, own, node.scale_children_by_parent))
                queue.append((c, own, level + 1))
            kids = [c.feature_index for c in node.children if c.feature_index is not None]
            if node.mutually_exclusive_children and len(kids) >= 2:
                groups.setdefault(level, []).append((own, kids))
        self.levels = sorted(set(feats) | set(groups))
        self.gate: dict[int, tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}
        for lv, rows in feats.items():
            rows = [r for r in rows if r[1] >= 0]
            if rows:
                self.gate[lv] = (torch.tensor([r[0] for r in rows]), torch.tensor([r[1] for r in rows]),
                                 torch.tensor([r[2] for r in rows]))
        self.me: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        for lv, gs in groups.items():
            width = max(len(k) for _, k in gs)
            sib = torch.full((len(gs), width), -1, dtype=torch.long)
            for g, (_, kids) in enumerate(gs):
                sib[g, : len(kids)] = torch.tensor(kids)
            self.me[lv] = (sib, torch.tensor([p for p, _ in gs]))
        self.any_rescale = any(bool(t[2].any()) for t in self.gate.values())
        self._dev: Any = None

    def to(self, device: Any) -> "_HierarchyPlan":
        if self._dev != device:
            self.gate = {k: tuple(t.to(device) for t in v) for k, v in self.gate.items()}  # type: ignore[misc]
            self.me = {k: tuple(t.to(device) for t in v) for k, v in self.me.items()}  # type: ignore[misc]
            self._dev = device
        return self

    def apply(self, x: torch.Tensor, means: torch.Tensor | None) -> None:
        """Enforce the forest on dense activations `x` [batch, features] in place."""
        if self.any_rescale and means is None:
            raise ValueError("scale_children_by_parent needs the generator's mean firing magnitudes")
        for lv in self.levels:
            if lv in self.gate:
                f, par, resc = self.gate[lv]
                pa = x[:, par]
                factor = (pa > 0).to(x.dtype)
                if self.any_rescale:
                    m = means.to(device=x.device, dtype=x.dtype)[par].clamp(min=1e-12)  # type: ignore[union-attr]
                    factor = torch.where(resc, pa / m, factor)
                x[:, f] = x[:, f] * factor
            if lv in self.me:
                self._exclude(x, *self.me[lv])

    @staticmethod
    def _exclude(x: torch.Tensor, sib: torch.Tensor, parents: torch.Tensor) -> None:
        B = x.shape[0]
        G, W = sib.shape
        valid = sib >= 0
        vals = x[:, sib.clamp(min=0).view(-1)].view(B, G, W)
        active = (vals > 0) & valid
        has_p = parents >= 0
        if bool(has_p.any()):
            p_on = (x[:, parents.clamp(min=0)] > 0) | ~has_p
            active &= p_on.unsqueeze(2)
        conflict = active.sum(2) > 1  # [B, G]
        if not bool(conflict.any()):
            return
        score = torch.rand(B, G, W, device=x.device).masked_fill(~active, -1.0)
        keep = torch.zeros_like(active).scatter_(2, score.argmax(2, keepdim=True), True)
        drop = active & ~keep & conflict.unsqueeze(2)
        b, g, w = drop.nonzero(as_tuple=True)
        x[b, sib[g, w]] = 0


def hierarchy_modifier(roots: HierarchyNode | Sequence[HierarchyNode]) -> ActivationsModifier:
    """Activations modifier enforcing the trees (gating by effective parents, parent rescaling and
    mutual exclusion, level by level); sparse COO input is densified and returned as COO
    (sae_lens/synthetic/hierarchy/modifier.py)."""
    roots = [roots] if isinstance(roots, HierarchyNode) else list(roots)
    validate_hierarchy(roots)
    plan = _HierarchyPlan(roots)

    def modifier(acts: torch.Tensor, gen: Any = None) -> torch.Tensor:
        sparse = acts.is_sparse
        x = acts.to_dense() if sparse else acts.clone()
        plan.to(x.device).apply(x, getattr(gen, "mean_firing_magnitudes", None))
        return x.to_sparse() if sparse else x

    return modifier


@dataclass
class HierarchyConfig:
    """Forest generation: total_root_nodes trees, branching_factor children per parent (int or
    (min, max)), max_depth levels below the roots, a portion of eligible parents made mutually
    exclusive, optional probability compensation and parent-scaled children."""

    total_root_nodes: int = 100
    branching_factor: int | tuple[int, int] = 100
    max_depth: int = 2
    mutually_exclusive_portion: float = 0.0
    mutually_exclusive_min_depth: int = 0
    mutually_exclusive_max_depth: int | None = None
    compensate_probabilities: bool = False
    scale_children_by_parent: bool = False

    def __post_init__(self) -> None:
        if self.total_root_nodes <= 0:
            raise ValueError("total_root_nodes must be positive")
        lo, hi = (self.branching_factor, self.branching_factor) if isinstance(self.branching_factor, int) \
            else tuple(self.branching_factor)
        if lo < 2:
            raise ValueError("branching_factor must be at least 2" if isinstance(self.branching_factor, int)
                             else "branching_factor minimum must be at least 2")
        if lo > hi:
            raise ValueError("branching_factor[0] must be <= branching_factor[1]")
        if self.max_depth < 1:
            raise ValueError("max_depth must be at least 1")
        if not 0.0 <= self.mutually_exclusive_portion <= 1.0:
            raise ValueError("mutually_exclusive_portion must be between 0.0 and 1.0")
        if self.mutually_exclusive_min_depth < 0:
            raise ValueError("mutually_exclusive_min_depth must be non-negative")
        if self.mutually_exclusive_max_depth is not None and \
                self.mutually_exclusive_max_depth < self.mutually_exclusive_min_depth:
            raise ValueError("mutually_exclusive_max_depth must be >= mutually_exclusive_min_depth")

    def to_dict(self) -> dict[str, Any]:
        d = asdict(self)
        if isinstance(self.branching_factor, tuple):
            d["branching_factor"] = list(self.branching_factor)
        return d

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "HierarchyConfig":
        d = dict(d)
        if isinstance(d.get("branching_factor"), list):
            d["branching_factor"] = tuple(d["branching_factor"])
        return cls(**d)


@dataclass
class Hierarchy:
    roots: list[HierarchyNode] = field(default_factory=list)
    modifier: ActivationsModifier | None = None

    @property
    def feature_indices_used(self) -> set[int]:
        return {i for r in self.roots for i in r.get_all_feature_indices()}

    def to_dict(self) -> dict[str, Any]:
        return {"roots": [r.to_dict() for r in self.roots]}

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "Hierarchy":
        roots = [HierarchyNode.from_dict(r) for r in d.get("roots", [])]
        return cls(roots=roots, modifier=hierarchy_modifier(roots) if roots else None)

    def __eq__(self, other: object) -> bool:
        return isinstance(other, Hierarchy) and self.to_dict() == other.to_dict()

    def compute_probability_correction_factors(self, base_firing_probabilities: torch.Tensor) -> torch.Tensor:
        """Factors that undo the hierarchy's thinning in expectation: a child's probability is
        divided by its parent's base probability, and a mutually exclusive child is further scaled
        by 1 + (sum of its siblings' base probabilities) / parent probability."""
        p = base_firing_probabilities
        out = torch.ones_like(p)

        def visit(n: HierarchyNode, parent_p: float) -> None:
            if n.feature_index is not None:
                if parent_p > 0 and parent_p < 1:
                    out[n.feature_index] = 1.0 / parent_p
                own = float(p[n.feature_index])
            else:
                own = parent_p
            for c in n.children:
                visit(c, own)
            kids = [c.feature_index for c in n.children if c.feature_index is not None]
            if n.mutually_exclusive_children and len(kids) >= 2 and own > 0:
                tot = float(sum(float(p[i]) for i in kids))
                for i in kids:
                    out[i] *= 1.0 + max(0.0, tot - float(p[i])) / own

        for r in self.roots:
            visit(r, 1.0)
        return out


def generate_hierarchy(num_features: int, config: HierarchyConfig, seed: int | None = None) -> Hierarchy:
    """Breadth-first forest over consecutive feature indices (roots first, then each level)."""
    rng = random.Random(seed)
    nxt = iter(range(num_features))
    roots: list[HierarchyNode] = []
    for _ in range(config.total_root_nodes):
        i = next(nxt, None)
        if i is None:
            break
        roots.append(HierarchyNode(i, scale_children_by_parent=config.scale_children_by_parent))
    level = [(r, 0) for r in roots]
    parents: list[tuple[HierarchyNode, int]] = []
    exhausted = False
    while level and not exhausted:
        nxt_level = []
        for node, depth in level:
            if depth >= config.max_depth:
                continue
            bf = config.branching_factor if isinstance(config.branching_factor, int) else \
                rng.randint(config.branching_factor[0], config.branching_factor[1])
            for _ in range(bf):
                i = next(nxt, None)
                if i is None:
                    exhausted = True
                    break
                child = HierarchyNode(i, scale_children_by_parent=config.scale_children_by_parent)
                node.children.append(child)
                nxt_level.append((child, depth + 1))
            if node.children:
                parents.append((node, depth))
            if exhausted:
                break
        level = nxt_level
    eligible = [n for n, d in parents if d >= config.mutually_exclusive_min_depth and
                (config.mutually_exclusive_max_depth is None or d <= config.mutually_exclusive_max_depth)
                and len(n.children) >= 2]
    for n in rng.sample(eligible, round(config.mutually_exclusive_portion * len(eligible))):
        n.mutually_exclusive_children = True
    return Hierarchy(roots=roots, modifier=hierarchy_modifier(roots) if roots else None)
