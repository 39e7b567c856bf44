"""JSONL -> tokenized .bin / .h5 shards through the config-driven pipeline.

    python -m astrai_b200.cli.preprocess in.jsonl [more.jsonl ...] -o OUT_DIR -c pipeline.json [--tokenizer_path DIR]

Parity: scripts/tools/preprocess.py:9-48 of the reference (same arguments).
"""

from __future__ import annotations

import argparse
from typing import List, Optional


def main(argv: Optional[List[str]] = None) -> None:
    from astrai_b200.config.preprocess_config import PipelineConfig
    from astrai_b200.preprocessing import Pipeline

    p = argparse.ArgumentParser(description="Raw JSONL -> tokenized .h5/.bin via config-driven Pipeline")
    p.add_argument("inputs", nargs="+", metavar="JSONL", help="One or more JSONL files")
    p.add_argument("--output_dir", "-o", required=True, help="Output directory")
    p.add_argument("--config", "-c", required=True, help="Path to pipeline config JSON")
    p.add_argument("--tokenizer_path", default="params", help="Path to tokenizer directory (default: params)")
    p.add_argument("--batch_size", type=int, default=None, help="Records tokenized together (default: config)")
    a = p.parse_args(argv)
    cfg = PipelineConfig.from_file(a.config)
    if a.batch_size is not None:
        if a.batch_size < 1:
            p.error("--batch_size must be at least 1")
        cfg.preprocessing.batch_size = a.batch_size
    stats = Pipeline(cfg, a.inputs, a.output_dir, a.tokenizer_path).run()
    print(stats)


if __name__ == "__main__":
    main()
