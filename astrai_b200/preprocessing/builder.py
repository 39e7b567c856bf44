"""Section rendering and loss-mask building (parity: astrai/preprocessing/builder.py).

A *section* names a record field and an action:

* ``template: true`` - a chat message list; every message is rendered on its
  own through the tokenizer's chat template, and its tokens are trained or
  masked according to ``action`` (``$role`` = look the role up in
  ``config.mask``, default ``config.mask_default``); a top-level templated
  sequence starts with the BOS token when the tokenizer has one;
* plain text - tokenised as is (special tokens on the first section unless
  overridden); pure-text configs drop records outside [min_chars, max_chars];
* ``action: "value"`` - a numeric field copied as floats (GRPO rewards).

``single`` builds ``{"sequence", "loss_mask"?}``; ``multi`` builds one output
per ``input.sources`` entry (``list_field`` keeps list elements as separate
sequences, e.g. GRPO responses); ``sectioned`` dispatches between the two.
Batch variants collect every text of a batch and tokenise it with one call
to the Rust batch encoder.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

from astrai_b200.factory import Registry


def extract_domain(item: dict, domain_key: Optional[str]) -> str:
    if not domain_key:
        return "__default__"
    v = item.get(domain_key, "__default__")
    return v if isinstance(v, str) else "__default__"


def resolve_action(action: str, role: str, config) -> str:
    return config.mask.get(role, config.mask_default) if action == "$role" else action


class SectionRenderer:
    """Turns section specs into (token ids, loss mask) pairs."""

    # -------------------------------------------------------------- planning
    def _plan(self, item: dict, sections: list, config, tokenizer, filter_text: bool) -> List[Tuple[str, str, bool]]:
        """Units (text, action, add_special_tokens) for one record."""
        has_template = any(s.get("template") for s in sections)
        text_only = not has_template and all(s["action"] == "train" for s in sections)
        units: List[Tuple[str, str, bool]] = []
        first = True
        for sec in sections:
            fld, action, templ = sec["field"], sec["action"], sec.get("template", False)
            add_special = sec.get("add_special_tokens", (not templ) and first)
            if templ:
                msgs = item.get(fld)
                if not isinstance(msgs, list) or not msgs:
                    continue
                for m in msgs:
                    text = tokenizer.apply_chat_template([m], tokenize=False, add_generation_prompt=False)
                    units.append((text, resolve_action(action, m.get("role", ""), config), False))
            else:
                text = str(item.get(fld, ""))
                if not text.strip():
                    continue
                if text_only and filter_text:
                    pp = config.preprocessing
                    if (pp.min_chars > 0 and len(text) < pp.min_chars) or len(text) > pp.max_chars:
                        continue
                units.append((text, action, add_special))
            first = False
        return units

    def _assemble(self, units, ids_list, sections, config, tokenizer, top_level):
        has_template = any(s.get("template") for s in sections)
        ids: List[int] = []
        mask: List[int] = []
        if top_level and has_template and tokenizer.bos_token_id is not None:
            ids.append(tokenizer.bos_token_id)
            mask.append(0)
        for (_, action, _), part in zip(units, ids_list):
            ids.extend(part)
            mask.extend([1 if action == "train" else 0] * len(part))
        ids = ids[: config.preprocessing.max_seq_len]
        mask = mask[: len(ids)]
        if not ids or (top_level and has_template and len(ids) <= 1):
            return None, None
        return ids, mask

    # -------------------------------------------------------------- single / batch
    def process_sections(self, item, sections, config, tokenizer, *, is_top_level=False):
        units = self._plan(item, sections, config, tokenizer, True)
        parts = [tokenizer.encode(t, add_special_tokens=a) for t, _, a in units]
        return self._assemble(units, parts, sections, config, tokenizer, is_top_level)

    def process_sections_batch(self, items, sections, config, tokenizer, *, is_top_level=False, filter_text=True):
        plans = [self._plan(it, sections, config, tokenizer, filter_text) for it in items]
        encoded: Dict[Tuple[int, int], List[int]] = {}
        for special in (False, True):
            refs = [(i, j, t) for i, plan in enumerate(plans) for j, (t, _, a) in enumerate(plan) if a == special]
            if refs:
                for (i, j, _), ids in zip(refs, tokenizer.encode([t for _, _, t in refs], add_special_tokens=special)):
                    encoded[(i, j)] = ids
        return [self._assemble(plan, [encoded[(i, j)] for j in range(len(plan))], sections, config, tokenizer,
                               is_top_level) for i, plan in enumerate(plans)]

    def process_list_field(self, item, sections, config, tokenizer):
        out = self.process_list_field_batch([item], sections, config, tokenizer)
        return out[0]

    def process_list_field_batch(self, items, sections, config, tokenizer):
        per_ids: List[list] = [[] for _ in items]
        per_mask: List[list] = [[] for _ in items]
        for sec in sections:
            fld = sec["field"]
            wrappers, owners = [], []
            for i, it in enumerate(items):
                vals = it.get(fld)
                if not isinstance(vals, list):
                    continue
                for v in vals:
                    if sec.get("template", False) and not isinstance(v, list):
                        continue
                    wrappers.append({fld: v if isinstance(v, list) else str(v)})
                    owners.append(i)
            for o, (ids, mask) in zip(owners, self.process_sections_batch(wrappers, [sec], config, tokenizer,
                                                                          is_top_level=False, filter_text=False)):
                if ids:
                    per_ids[o].append(ids)
                    per_mask[o].append(mask)
        return [(a, b) if a else (None, None) for a, b in zip(per_ids, per_mask)]

    @staticmethod
    def is_value_section(sections: list) -> bool:
        return len(sections) == 1 and sections[0].get("action") == "value"

    @staticmethod
    def extract_raw_value(item: dict, sections: list):
        raw = item.get(sections[0]["field"])
        if raw is None:
            return None
        return [float(v) for v in raw] if isinstance(raw, list) else [float(raw)]


class BaseMaskBuilder:
    def build(self, item: dict, config, tokenizer) -> Optional[dict]:  # pragma: no cover - abstract
        raise NotImplementedError

    def build_batch(self, items: List[dict], config, tokenizer) -> List[Optional[dict]]:
        return [self.build(it, config, tokenizer) for it in items]


class MaskBuilderFactory(Registry["BaseMaskBuilder"]):
    pass


@MaskBuilderFactory.register("single")
class SingleOutputMaskBuilder(BaseMaskBuilder):
    def __init__(self, renderer: Optional[SectionRenderer] = None):
        self.renderer = renderer or SectionRenderer()

    def _result(self, item, ids, mask, config):
        if ids is None:
            return None
        r = {"sequence": ids, "domain": extract_domain(item, config.output.domain_key)}
        if not all(m == 1 for m in mask):
            r["loss_mask"] = mask
        return r

    def build(self, item, config, tokenizer):
        if not config.input.sections:
            return None
        ids, mask = self.renderer.process_sections(item, config.input.sections, config, tokenizer, is_top_level=True)
        return self._result(item, ids, mask, config)

    def build_batch(self, items, config, tokenizer):
        if not config.input.sections:
            return [None] * len(items)
        out = self.renderer.process_sections_batch(items, config.input.sections, config, tokenizer, is_top_level=True)
        return [self._result(it, ids, m, config) for it, (ids, m) in zip(items, out)]


@MaskBuilderFactory.register("multi")
class MultiOutputMaskBuilder(BaseMaskBuilder):
    def __init__(self, renderer: Optional[SectionRenderer] = None):
        self.renderer = renderer or SectionRenderer()

    def build(self, item, config, tokenizer):
        return self.build_batch([item], config, tokenizer)[0]

    def build_batch(self, items, config, tokenizer):
        sources = config.input.sources
        if not sources:
            return [None] * len(items)
        results: List[dict] = [{} for _ in items]
        for key, spec in sources.items():
            secs = spec.get("sections", [])
            if not secs:
                continue
            if self.renderer.is_value_section(secs):
                for it, r in zip(items, results):
                    v = self.renderer.extract_raw_value(it, secs)
                    if v is not None:
                        r[key] = v
                continue
            mkey = spec.get("mask_key", f"{key}_mask")
            lf = spec.get("list_field", False)
            rendered = (self.renderer.process_list_field_batch(items, secs, config, tokenizer) if lf else
                        self.renderer.process_sections_batch(items, secs, config, tokenizer, is_top_level=True))
            for r, (ids, mask) in zip(results, rendered):
                if ids is None:
                    continue
                r[key] = ids
                if lf or not all(m == 1 for m in mask) or "mask_key" in spec:
                    r[mkey] = mask
        return [({**r, "domain": extract_domain(it, config.output.domain_key)} if r else None)
                for it, r in zip(items, results)]


@MaskBuilderFactory.register("sectioned")
class SectionedMaskBuilder(BaseMaskBuilder):
    def __init__(self):
        self._single = SingleOutputMaskBuilder()
        self._multi = MultiOutputMaskBuilder()

    def _pick(self, config):
        return self._multi if config.input.sources else self._single

    def build(self, item, config, tokenizer):
        return self._pick(config).build(item, config, tokenizer)

    def build_batch(self, items, config, tokenizer):
        return self._pick(config).build_batch(items, config, tokenizer)
