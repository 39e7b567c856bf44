"""Evaluation suite (parity: scripts/eval/*.py of the reference).

Log-likelihood evals (:mod:`.ppl`, :mod:`.mmlu`, :mod:`.ifd`) share the packed
scorer of :mod:`.loglik`; generation evals (:mod:`.humaneval`, :mod:`.ifeval`)
submit all prompts to the continuous-batching engine; :mod:`.rouge` and
:mod:`.weights` need no model forward. Each module runs as
``python -m astrai_b200.eval.<name>``.
"""

from astrai_b200.eval.loglik import Doc, fit, next_token_logprobs, score_docs
from astrai_b200.eval.rouge import compute_rouge

__all__ = ["Doc", "compute_rouge", "fit", "next_token_logprobs", "score_docs"]
