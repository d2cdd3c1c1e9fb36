"""File names of the checkpoint layout (same names as the reference, sae_lens/constants.py:23-33,
so checkpoints are interchangeable)."""

SAE_WEIGHTS_FILENAME = "sae_weights.safetensors"
SAE_CFG_FILENAME = "cfg.json"
SPARSITY_FILENAME = "sparsity.safetensors"
RUNNER_CFG_FILENAME = "runner_cfg.json"
SPARSIFY_WEIGHTS_FILENAME = "sae.safetensors"
TRAINER_STATE_FILENAME = "trainer_state.pt"
ACTIVATIONS_STORE_STATE_FILENAME = "activations_store_state.safetensors"
ACTIVATION_SCALER_CFG_FILENAME = "activation_scaler.json"
FSDP_OPTIMIZER_STATE_FILENAME_TEMPLATE = "fsdp_optimizer_state_rank{rank}.pt"
MSE_HISTORY_FILENAME = "mse_history.jsonl"
TIMING_HISTORY_FILENAME = "timing_history.jsonl"
MULTI_SAE_MANIFEST_FILENAME = "multi_sae_manifest.json"

DTYPE_NAMES = ("float32", "float64", "float16", "bfloat16")

# Version string written as `sae_lens_version` in saved configs: the checkpoint layout this
# package reads and writes is the SAELens 6.x layout, so loaders that branch on that field treat
# these checkpoints as current-format files.
CHECKPOINT_FORMAT_VERSION = "6.37.6"
