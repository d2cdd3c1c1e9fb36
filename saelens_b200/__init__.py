"""saelens_b200: sparse-autoencoder training and inference, native on NVIDIA B200 (sm_100a)."""

__version__ = "0.1.0"

import logging as _logging

logger = _logging.getLogger("saelens_b200")

from saelens_b200.models import *  # noqa: E402,F401,F403
from saelens_b200.models import __all__ as _models_all  # noqa: E402
from saelens_b200.registry import register_sae_class, register_sae_training_class  # noqa: E402,F401

from saelens_b200.analysis.hooked_sae_transformer import HookedSAETransformer  # noqa: E402
from saelens_b200.config import (  # noqa: E402
    CacheActivationsRunnerConfig,
    LanguageModelSAERunnerConfig,
    LoggingConfig,
    PretokenizeRunnerConfig,
)
from saelens_b200.evals import run_evals  # noqa: E402
from saelens_b200.loading.pretrained_sae_loaders import (  # noqa: E402
    PretrainedSaeDiskLoader,
    PretrainedSaeHuggingfaceLoader,
)
from saelens_b200.runners.cache_activations_runner import CacheActivationsRunner  # noqa: E402
from saelens_b200.runners.llm_sae_training_runner import (  # noqa: E402
    LanguageModelSAETrainingRunner,
    SAETrainingRunner,
)
from saelens_b200.runners.pretokenize_runner import PretokenizeRunner, pretokenize_runner  # noqa: E402
from saelens_b200.training.activations_store import ActivationsStore  # noqa: E402
from saelens_b200.training.sae_trainer import SAETrainer  # noqa: E402
from saelens_b200.training.upload_saes_to_huggingface import upload_saes_to_huggingface  # noqa: E402

__all__ = [
    "__version__", "logger", "register_sae_class", "register_sae_training_class", *_models_all,
    "HookedSAETransformer", "ActivationsStore", "LanguageModelSAERunnerConfig", "LanguageModelSAETrainingRunner",
    "SAETrainingRunner", "CacheActivationsRunnerConfig", "CacheActivationsRunner", "PretokenizeRunnerConfig",
    "PretokenizeRunner", "pretokenize_runner", "run_evals", "upload_saes_to_huggingface",
    "PretrainedSaeHuggingfaceLoader", "PretrainedSaeDiskLoader", "SAETrainer", "LoggingConfig",
]

try:  # the Hugging Face bridge needs `transformers`
    from saelens_b200.analysis.sae_transformer_bridge import SAETransformerBridge, has_transformer_bridge

    if has_transformer_bridge():
        __all__.append("SAETransformerBridge")
except ImportError:  # pragma: no cover
    pass
