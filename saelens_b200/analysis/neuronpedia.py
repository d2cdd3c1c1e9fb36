"""Neuronpedia helpers: dashboard / quick-list URLs and the feature and list API (role of
sae_lens/analysis/neuronpedia_integration.py).  Every network call goes through `requests`; URL
construction is separate so it can be used (and tested) offline.  Pass `open_browser=False` to
get URLs without launching a browser."""

from __future__ import annotations

import json
import math
import urllib.parse
import webbrowser
from dataclasses import dataclass, field
from typing import Any

NEURONPEDIA_DOMAIN = "https://neuronpedia.org"
POSITIVE_INF_REPLACEMENT = 9999
NEGATIVE_INF_REPLACEMENT = -9999
NAN_REPLACEMENT = 0
OTHER_INVALID_REPLACEMENT = -99999


def NanAndInfReplacer(value: str) -> float:  # noqa: N802 - json `parse_constant` hook
    """Map JSON's non-finite constants to finite sentinels when parsing API responses."""
    return float({"-Infinity": NEGATIVE_INF_REPLACEMENT, "Infinity": POSITIVE_INF_REPLACEMENT,
                  "NaN": NAN_REPLACEMENT}.get(value, NAN_REPLACEMENT))


def sanitize_for_json(x: Any) -> Any:
    """Replace non-finite floats (recursively) before sending values to the API."""
    if isinstance(x, float):
        if math.isnan(x):
            return NAN_REPLACEMENT
        if math.isinf(x):
            return POSITIVE_INF_REPLACEMENT if x > 0 else NEGATIVE_INF_REPLACEMENT
        return x
    if isinstance(x, dict):
        return {k: sanitize_for_json(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [sanitize_for_json(v) for v in x]
    return x


def _neuronpedia_id(sae: Any) -> str:
    sid = getattr(getattr(sae.cfg, "metadata", None), "neuronpedia_id", None)
    if sid is None:
        raise ValueError("this SAE has no Neuronpedia id (dashboards may not exist, or it was not loaded with "
                         "from_pretrained)")
    return sid


def feature_dashboard_url(sae: Any, index: int) -> str:
    return f"{NEURONPEDIA_DOMAIN}/{_neuronpedia_id(sae)}/{index}"


def open_neuronpedia_feature_dashboard(sae: Any, index: int, open_browser: bool = True) -> str:
    url = feature_dashboard_url(sae, index)
    if open_browser:
        webbrowser.open(url)
    return url


def quick_list_url(sae: Any, features: list[int], name: str = "temporary_list") -> str:
    sid = _neuronpedia_id(sae)
    model = getattr(sae.cfg.metadata, "model_name", None)
    items = [{"modelId": model, "layer": sid.split("/")[1], "index": str(f)} for f in features]
    return (f"{NEURONPEDIA_DOMAIN}/quick-list/?name={urllib.parse.quote(name)}"
            f"&features={urllib.parse.quote(json.dumps(items))}")


def get_neuronpedia_quick_list(sae: Any, features: list[int], name: str = "temporary_list",
                               open_browser: bool = True) -> str:
    url = quick_list_url(sae, features, name)
    if open_browser:
        webbrowser.open(url)
    return url


def feature_api_url(feature: int, layer: int, model: str = "gpt2-small", dataset: str = "res-jb") -> str:
    return f"{NEURONPEDIA_DOMAIN}/api/feature/{model}/{layer}-{dataset}/{feature}"


def get_neuronpedia_feature(feature: int, layer: int, model: str = "gpt2-small", dataset: str = "res-jb",
                            timeout: float = 30.0) -> dict[str, Any]:
    import requests

    r = requests.get(feature_api_url(feature, layer, model, dataset), timeout=timeout)
    out = json.loads(r.text, parse_constant=NanAndInfReplacer)
    out["index"] = int(out["index"])
    return out


@dataclass
class NeuronpediaActivation:
    id: str
    tokens: list[str]
    act_values: list[float]


@dataclass
class NeuronpediaFeature:
    modelId: str  # noqa: N815 - API field name
    layer: int
    dataset: str
    feature: int
    description: str = ""
    activations: list[NeuronpediaActivation] | None = None
    autointerp_explanation: str = ""
    autointerp_explanation_score: float = 0.0
    extra: dict[str, Any] = field(default_factory=dict)

    def has_activating_text(self) -> bool:
        return bool(self.activations) and any(max(a.act_values, default=0.0) > 0 for a in self.activations)


def list_request_body(list_name: str, features: list[NeuronpediaFeature],
                      list_description: str | None = None) -> dict[str, Any]:
    return {"name": list_name, "description": list_description,
            "features": [{"modelId": f.modelId, "layer": f"{f.layer}-{f.dataset}", "index": f.feature,
                          "description": f.description} for f in features]}


def make_neuronpedia_list_with_features(api_key: str, list_name: str, features: list[NeuronpediaFeature],
                                        list_description: str | None = None, open_browser: bool = True) -> str:
    import requests

    r = requests.post(NEURONPEDIA_DOMAIN + "/api/list/new-with-features",
                      json=sanitize_for_json(list_request_body(list_name, features, list_description)),
                      headers={"x-api-key": api_key}, timeout=60)
    res = r.json()
    if "url" not in res:
        raise RuntimeError("Error in creating list: " + str(res.get("message", res)))
    if open_browser:
        webbrowser.open(res["url"])
    return res["url"]


def test_key(api_key: str) -> None:
    """Raise if Neuronpedia rejects the API key."""
    import requests

    r = requests.post(f"{NEURONPEDIA_DOMAIN}/api/test", json={"apiKey": api_key}, timeout=30)
    if r.status_code != 200:
        raise RuntimeError("Neuronpedia API key is not valid.")


test_key.__test__ = False  # type: ignore[attr-defined]  # not a pytest test
