"""SAE architecture zoo; importing this package registers every built-in architecture."""

from saelens_b200.models.batchtopk import (
    BatchTopK,
    BatchTopKTrainingSAE,
    BatchTopKTrainingSAEConfig,
    MatryoshkaBatchTopKTrainingSAE,
    MatryoshkaBatchTopKTrainingSAEConfig,
)
from saelens_b200.models.gated import GatedSAE, GatedSAEConfig, GatedTrainingSAE, GatedTrainingSAEConfig
from saelens_b200.models.jumprelu import (
    JumpReLUSAE,
    JumpReLUSAEConfig,
    JumpReLUTrainingSAE,
    JumpReLUTrainingSAEConfig,
)
from saelens_b200.models.matching_pursuit import (
    MatchingPursuitSAE,
    MatchingPursuitSAEConfig,
    MatchingPursuitTrainingSAE,
    MatchingPursuitTrainingSAEConfig,
)
from saelens_b200.models.sae import (
    SAE,
    SAEConfig,
    SAEMetadata,
    TrainCoefficientConfig,
    TrainingSAE,
    TrainingSAEConfig,
    TrainStepInput,
    TrainStepOutput,
)
from saelens_b200.models.standard import (
    StandardSAE,
    StandardSAEConfig,
    StandardTrainingSAE,
    StandardTrainingSAEConfig,
)
from saelens_b200.models.temporal import TemporalSAE, TemporalSAEConfig
from saelens_b200.models.topk import (
    TopK,
    TopKSAE,
    TopKSAEConfig,
    TopKTrainingSAE,
    TopKTrainingSAEConfig,
)
from saelens_b200.models.transcoder import (
    JumpReLUSkipTranscoder,
    JumpReLUSkipTranscoderConfig,
    JumpReLUTranscoder,
    JumpReLUTranscoderConfig,
    SkipTranscoder,
    SkipTranscoderConfig,
    Transcoder,
    TranscoderConfig,
)
from saelens_b200.registry import (
    SAE_CLASS_REGISTRY,
    SAE_TRAINING_CLASS_REGISTRY,
    register_sae_class,
    register_sae_training_class,
)

_INFERENCE = {
    "standard": (StandardSAE, StandardSAEConfig),
    "gated": (GatedSAE, GatedSAEConfig),
    "topk": (TopKSAE, TopKSAEConfig),
    "jumprelu": (JumpReLUSAE, JumpReLUSAEConfig),
    "transcoder": (Transcoder, TranscoderConfig),
    "skip_transcoder": (SkipTranscoder, SkipTranscoderConfig),
    "jumprelu_transcoder": (JumpReLUTranscoder, JumpReLUTranscoderConfig),
    "jumprelu_skip_transcoder": (JumpReLUSkipTranscoder, JumpReLUSkipTranscoderConfig),
    "temporal": (TemporalSAE, TemporalSAEConfig),
    "matching_pursuit": (MatchingPursuitSAE, MatchingPursuitSAEConfig),
}
_TRAINING = {
    "standard": (StandardTrainingSAE, StandardTrainingSAEConfig),
    "gated": (GatedTrainingSAE, GatedTrainingSAEConfig),
    "topk": (TopKTrainingSAE, TopKTrainingSAEConfig),
    "jumprelu": (JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig),
    "batchtopk": (BatchTopKTrainingSAE, BatchTopKTrainingSAEConfig),
    "matryoshka_batchtopk": (MatryoshkaBatchTopKTrainingSAE, MatryoshkaBatchTopKTrainingSAEConfig),
    "matching_pursuit": (MatchingPursuitTrainingSAE, MatchingPursuitTrainingSAEConfig),
}
for _arch, (_cls, _cfg) in _INFERENCE.items():
    if _arch not in SAE_CLASS_REGISTRY:
        register_sae_class(_arch, _cls, _cfg)
for _arch, (_cls, _cfg) in _TRAINING.items():
    if _arch not in SAE_TRAINING_CLASS_REGISTRY:
        register_sae_training_class(_arch, _cls, _cfg)

__all__ = [n for n in dir() if not n.startswith("_")]
