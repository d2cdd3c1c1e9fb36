"""saelens_b200: sparse-autoencoder training and inference, native on NVIDIA B200 (sm_100a)."""

__version__ = "0.1.0"

import logging as _logging

logger = _logging.getLogger("saelens_b200")

from saelens_b200.models import *  # noqa: E402,F401,F403
from saelens_b200.models import __all__ as _models_all  # noqa: E402
from saelens_b200.registry import register_sae_class, register_sae_training_class  # noqa: E402,F401

__all__ = ["__version__", "logger", "register_sae_class", "register_sae_training_class", *_models_all]
