"""Fetch model parameters from the Hugging Face hub (parity: scripts/demo/download.py of the
reference, same default repo). Needs ``huggingface_hub`` and network access; offline, copy a
model directory (config.json, tokenizer files, model.safetensors) to ``--local-dir`` instead."""

from __future__ import annotations

import argparse
from pathlib import Path

from astrai_b200.demo import DEFAULT_PARAMS

DEFAULT_REPO_ID = "ViperEkura/AstrAI-V1-instruct"


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Download model parameters from HuggingFace")
    p.add_argument("--repo-id", type=str, default=DEFAULT_REPO_ID)
    p.add_argument("--local-dir", type=Path, default=DEFAULT_PARAMS)
    p.add_argument("--force", action="store_true")
    a = p.parse_args(argv)
    try:
        from huggingface_hub import snapshot_download
    except ImportError as e:
        raise SystemExit("huggingface_hub is not installed; copy the model directory to "
                         f"{a.local_dir} by hand") from e
    print(f"Downloading {a.repo_id} to {a.local_dir}")
    snapshot_download(repo_id=a.repo_id, local_dir=a.local_dir, force_download=a.force)


if __name__ == "__main__":
    main()
