"""Token-set enrichment analysis (TSEA) of SAE features (role of sae_lens/tutorial/tsea.py).

A feature's decoder direction projected through the unembedding scores every vocabulary token.
For a token set S (a "gene set": tokens starting with a space, digits, a letter, a regex...) the
enrichment score is the GSEA running-sum statistic: walk the vocabulary from the highest score
down, adding 1/|S| at members and subtracting 1/(V - |S|) elsewhere; the score is the largest
absolute running sum.  Computed on the device one set at a time ([features, V] working memory).
"""

from __future__ import annotations

import re
import string
from typing import Any

import torch


def feature_vocab_projections(sae: Any, model: Any) -> torch.Tensor:
    """[d_sae, d_vocab] = W_dec @ W_U (decoder directions read out through the unembedding)."""
    W_U = model.W_U if hasattr(model, "W_U") else model.unembed.weight.T
    return sae.W_dec.detach().float() @ W_U.detach().float().to(sae.W_dec.device)


def pad_gene_sets(gene_sets_token_ids: dict[str, set[int] | list[int]]) -> dict[str, list[int]]:
    lists = {k: sorted(v) for k, v in gene_sets_token_ids.items()}
    width = max((len(v) for v in lists.values()), default=0)
    return {k: v + [-1] * (width - len(v)) for k, v in lists.items()}


@torch.no_grad()
def calculate_batch_enrichment_scores(scores: torch.Tensor, index_lists: torch.Tensor) -> torch.Tensor:
    """scores [n_features, V]; index_lists [n_sets, L] of token ids padded with -1.
    Returns [n_sets, n_features] enrichment scores."""
    n_sets = index_lists.shape[0]
    n, V = scores.shape
    order = scores.sort(dim=1, descending=True).indices
    out = torch.empty(n_sets, n, device=scores.device)
    for i in range(n_sets):
        ids = index_lists[i][index_lists[i] >= 0].to(scores.device)
        member = torch.zeros(V, dtype=torch.bool, device=scores.device)
        member[ids] = True
        k = float(member.sum())
        hits = member[order]
        step = torch.where(hits, torch.tensor(1.0 / max(k, 1.0), device=scores.device),
                           torch.tensor(-1.0 / max(V - k, 1.0), device=scores.device))
        out[i] = step.cumsum(dim=1).abs().max(dim=1).values
    return out


def get_enrichment_df(projections: torch.Tensor, features: list[int], gene_sets_selected: dict[str, Any]) -> Any:
    import pandas as pd

    padded = pad_gene_sets(gene_sets_selected)
    es = calculate_batch_enrichment_scores(projections[features], torch.tensor(list(padded.values())))
    return pd.DataFrame(es.cpu().numpy(), index=list(gene_sets_selected.keys()), columns=features)


def get_gene_set_from_regex(vocab: dict[str, int], pattern: str) -> set[int]:
    rx = re.compile(pattern)
    return {i for tok, i in vocab.items() if rx.match(tok)}


def _clean(tok: str) -> str:
    return tok.lstrip("Ġ▁ ")


def get_letter_gene_sets(vocab: dict[str, int]) -> dict[str, set[int]]:
    out: dict[str, set[int]] = {c: set() for c in string.ascii_lowercase}
    for tok, i in vocab.items():
        c = _clean(tok)
        if c.isalpha() and c[0].lower() in out:
            out[c[0].lower()].add(i)
    return out


def get_test_gene_sets(model_or_vocab: Any) -> dict[str, set[int]]:
    """Simple lexical sets: leading space, capitalised, digits, punctuation, single characters and a
    few word lists (colours, numbers, days, months)."""
    vocab = model_or_vocab if isinstance(model_or_vocab, dict) else model_or_vocab.tokenizer.get_vocab()
    words = {
        "colors": ["red", "blue", "yellow", "green", "orange", "purple", "black", "white", "pink", "brown"],
        "numbers": ["one", "two", "three", "four", "five", "six", "seven", "eight", "nine", "ten"],
        "days": ["monday", "tuesday", "wednesday", "thursday", "friday", "saturday", "sunday"],
        "months": ["january", "february", "march", "april", "may", "june", "july", "august", "september",
                   "october", "november", "december"],
    }
    sets: dict[str, set[int]] = {
        "starts_with_space": {i for t, i in vocab.items() if t[:1] in ("Ġ", "▁", " ")},
        "starts_with_capital": {i for t, i in vocab.items() if _clean(t)[:1].isupper()},
        "all_digits": {i for t, i in vocab.items() if _clean(t).isdigit()},
        "is_punctuation": {i for t, i in vocab.items() if _clean(t) and all(c in string.punctuation for c in _clean(t))},
        "single_character": {i for t, i in vocab.items() if len(_clean(t)) == 1},
    }
    for name, ws in words.items():
        wl = set(ws)
        sets[name] = {i for t, i in vocab.items() if _clean(t).lower() in wl}
    return sets


def generate_pos_sets(vocab: dict[str, int]) -> dict[str, set[int]]:
    """Part-of-speech sets (requires nltk with its tagger data)."""
    import nltk

    out: dict[str, set[int]] = {}
    for tok, i in vocab.items():
        tag = nltk.pos_tag([_clean(tok)])[0][1]
        out.setdefault(f"nltk_pos_{tag}", set()).add(i)
    return out


def manhattan_plot_enrichment_scores(df_enrichment_scores: Any, label_threshold: float = 1.0,
                                     top_n: int = 3, save_path: str | None = None) -> Any:
    """Scatter of -log10(1 - ES) per feature, coloured by set (requires matplotlib)."""
    import matplotlib

    matplotlib.use("Agg")
    import matplotlib.pyplot as plt
    import numpy as np

    fig, ax = plt.subplots(figsize=(10, 4))
    for name, row in df_enrichment_scores.iterrows():
        y = -np.log10(np.clip(1 - row.values, 1e-12, None))
        ax.scatter(range(len(y)), y, s=4, label=str(name))
        for j in np.argsort(y)[-top_n:]:
            if y[j] > label_threshold:
                ax.annotate(str(df_enrichment_scores.columns[j]), (j, y[j]), fontsize=6)
    ax.set_xlabel("feature")
    ax.set_ylabel("-log10(1 - ES)")
    ax.legend(fontsize=6, markerscale=2)
    if save_path:
        fig.savefig(save_path, bbox_inches="tight")
    return fig
