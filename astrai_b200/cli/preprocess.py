"""Tokenise raw JSONL into training shards with a preprocessing config.

    python -m astrai_b200.cli.preprocess in.jsonl [more.jsonl ...] -o OUT_DIR -c pipeline.json \
        [--tokenizer_path DIR] [--batch_size N]

The argument names and defaults are the reference's CLI (scripts/tools/preprocess.py:9-48), so
existing preprocessing scripts keep working; the shards it writes load with
``DatasetFactory.load`` (bin or h5, as the config's output section says).
"""

from __future__ import annotations

import argparse
import json
from typing import List, Optional


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(
        prog="astrai_b200.cli.preprocess",
        description="Tokenise JSONL records into bin/h5 training shards, as described by a pipeline config "
                    "(sections, loss masks, packing, position ids, output format).")
    p.add_argument("inputs", nargs="+", metavar="JSONL", help="input files, one JSON record per line")
    p.add_argument("--output_dir", "-o", required=True, help="where the shards and their meta files are written")
    p.add_argument("--config", "-c", required=True, help="pipeline config file (JSON)")
    p.add_argument("--tokenizer_path", default="params",
                   help="directory holding tokenizer.json and tokenizer_config.json [params]")
    p.add_argument("--batch_size", type=int, default=None,
                   help="records handed to the tokenizer per call; overrides the config's preprocessing.batch_size")
    return p


def main(argv: Optional[List[str]] = None) -> None:
    from astrai_b200.config.preprocess_config import PipelineConfig
    from astrai_b200.preprocessing import Pipeline

    parser = build_parser()
    args = parser.parse_args(argv)
    cfg = PipelineConfig.from_file(args.config)
    if args.batch_size is not None:
        if args.batch_size <= 0:
            parser.error(f"--batch_size {args.batch_size}: give a positive number of records")
        cfg.preprocessing.batch_size = args.batch_size
    stats = Pipeline(cfg, args.inputs, args.output_dir, args.tokenizer_path).run()
    print(json.dumps(stats, default=str))


if __name__ == "__main__":
    main()
