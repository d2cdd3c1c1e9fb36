"""Upload trained SAEs to a Hugging Face model repo, one folder per SAE id (role of
sae_lens/training/upload_saes_to_huggingface.py).  Each value of `saes_dict` is an SAE object
(saved to a temporary folder first) or a path to a saved SAE folder (`cfg.json` +
`sae_weights.safetensors`, optionally `sparsity.safetensors`).  A default README describing how to
load the SAEs is added when the repo has none.  `api` lets callers pass a configured (or fake)
`huggingface_hub.HfApi`."""

from __future__ import annotations

import io
from collections.abc import Iterable
from pathlib import Path
from tempfile import TemporaryDirectory
from typing import Any

from saelens_b200.constants import SAE_CFG_FILENAME, SAE_WEIGHTS_FILENAME, SPARSITY_FILENAME


def default_readme(repo_id: str, sae_ids: Iterable[str]) -> str:
    ids = "\n".join(f"- {s}" for s in sae_ids)
    return (f"---\nlibrary_name: saelens\n---\n\n# SAEs for use with the SAELens library\n\n"
            f"This repository contains the following SAEs:\n{ids}\n\nLoad these SAEs as below:\n\n"
            f"```python\nfrom saelens_b200 import SAE\n\nsae = SAE.from_pretrained(\"{repo_id}\", \"<sae_id>\")\n```")


def _validate_sae_path(p: Path) -> None:
    if not p.is_dir():
        raise FileNotFoundError(f"SAE folder {p} does not exist")
    for f in (SAE_CFG_FILENAME, SAE_WEIGHTS_FILENAME):
        if not (p / f).exists():
            raise FileNotFoundError(f"{p} is missing {f}")


def upload_saes_to_huggingface(saes_dict: dict[str, Any], hf_repo_id: str, hf_revision: str = "main",
                               show_progress: bool = True, add_default_readme: bool = True, api: Any = None) -> None:
    from saelens_b200.models.sae import SAE

    if not saes_dict:
        raise ValueError("No SAEs to upload")
    for ref in saes_dict.values():
        if not isinstance(ref, SAE):
            _validate_sae_path(Path(ref))
    if api is None:
        from huggingface_hub import HfApi

        api = HfApi()
    api.create_repo(hf_repo_id, exist_ok=True)
    items = list(saes_dict.items())
    if show_progress:
        from tqdm import tqdm

        items = tqdm(items, desc="Uploading SAEs")
    for sae_id, ref in items:
        with TemporaryDirectory() as tmp:
            if isinstance(ref, SAE):
                path = Path(tmp) / "sae"
                ref.save_model(str(path))
            else:
                path = Path(ref)
            _validate_sae_path(path)
            api.upload_folder(folder_path=str(path), path_in_repo=sae_id, repo_id=hf_repo_id, revision=hf_revision,
                              repo_type="model", commit_message=f"Upload SAE {sae_id}",
                              allow_patterns=[SAE_CFG_FILENAME, SAE_WEIGHTS_FILENAME, SPARSITY_FILENAME])
    if add_default_readme and not api.file_exists(hf_repo_id, "README.md", revision=hf_revision):
        api.upload_file(path_or_fileobj=io.BytesIO(default_readme(hf_repo_id, saes_dict).encode()),
                        path_in_repo="README.md", repo_id=hf_repo_id, revision=hf_revision,
                        commit_message="Add README.md")
