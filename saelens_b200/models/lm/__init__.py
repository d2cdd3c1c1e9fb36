"""Producer language models (see `transformer.py`) and HF model wrapping (see `hf.py`)."""

from saelens_b200.models.lm.transformer import PRESETS, HookedLM, LMConfig, preset_config

__all__ = ["PRESETS", "HookedLM", "LMConfig", "preset_config"]
