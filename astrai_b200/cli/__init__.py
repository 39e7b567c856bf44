"""Command-line tools: ``python -m astrai_b200.cli.{train,server,generate,preprocess,benchmark}``."""
