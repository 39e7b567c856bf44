"""Tokenizer wrapper and chat templates.

Parity: astrai/tokenize/tokenizer.py and chat_template.py. A model directory
carries ``tokenizer.json`` (HuggingFace ``tokenizers`` format, run by the
Rust library) and ``tokenizer_config.json`` with ``special_tokens`` (name ->
token string) and ``chat_template`` (Jinja2). Features kept:

* ``encode(str | list[str])`` (lists go through the parallel batch encoder),
  ``decode``, ``len()``;
* attribute access ``tok.bos_token`` / ``tok.bos_token_id`` for any special
  token name, and ``tok.stop_ids`` = ids of all special tokens;
* ``apply_chat_template(messages | list[messages], tokenize, add_generation_prompt, system_prompt)``;
* the compiled Jinja2 template is created lazily so the object pickles
  cleanly into spawned worker processes.
"""

from __future__ import annotations

import json
from functools import cached_property
from pathlib import Path
from typing import Any, Dict, List, Optional, Union

Message = Dict[str, str]
Messages = List[Message]


class ChatTemplate:
    def __init__(self, name: str = "", template_str: str = "", description: str = "",
                 default_variables: Optional[Dict[str, Any]] = None, special_tokens: Optional[Dict[str, str]] = None):
        self.name = name
        self.template_str = template_str
        self.description = description
        self.default_variables = default_variables or {}
        self.special_tokens = special_tokens or {}

    @cached_property
    def _compiled(self):
        from jinja2 import Template

        return Template(self.template_str)

    def __getstate__(self):
        d = dict(self.__dict__)
        d.pop("_compiled", None)  # compiled templates do not pickle
        return d

    @classmethod
    def from_string(cls, template_str: str, description: str = "", default_variables=None,
                    special_tokens=None) -> "ChatTemplate":
        return cls(name="", template_str=template_str, description=description, default_variables=default_variables,
                   special_tokens=special_tokens)

    def render(self, messages: List[Dict[str, Any]], system_prompt: Optional[str] = None, **extra: Any) -> str:
        variables = {**self.default_variables, **self.special_tokens, **extra, "messages": messages}
        if system_prompt is not None:
            variables["system_prompt"] = system_prompt
        return self._compiled.render(**variables)


class AutoTokenizer:
    TOKENIZER_CLASSES: Dict[str, type] = {}

    def __init__(self, path: Optional[Union[str, Path]] = None, special_token_map: Optional[Dict[str, str]] = None,
                 chat_template: Optional[str] = None, tokenizer=None):
        self._tokenizer = tokenizer
        self._chat_template: Optional[ChatTemplate] = None
        self._special_token_map: Dict[str, str] = dict(special_token_map or {})
        if chat_template:
            self.set_chat_template(chat_template)
        if path:
            self.load(path)

    # ------------------------------------------------------------------ files
    def load(self, path: Union[str, Path]) -> None:
        from tokenizers import Tokenizer

        p = Path(path)
        self._tokenizer = Tokenizer.from_file(str(p / "tokenizer.json"))
        cfg_file = p / "tokenizer_config.json"
        if cfg_file.exists():
            cfg = json.loads(cfg_file.read_text(encoding="utf-8"))
            self._special_token_map.update(cfg.get("special_tokens", {}))
            if "chat_template" in cfg:
                self.set_chat_template(cfg["chat_template"])

    @classmethod
    def from_pretrained(cls, path: Union[str, Path]) -> "AutoTokenizer":
        p = Path(path)
        if not (p / "tokenizer.json").exists():
            raise FileNotFoundError(f"Tokenizer file not found: {p / 'tokenizer.json'}. A valid tokenizer.json is required.")
        inst = cls(p)
        if inst._tokenizer is None:
            raise RuntimeError(f"Failed to load tokenizer from {p}.")
        return inst

    def save_pretrained(self, save_path: Union[str, Path]) -> None:
        if self._tokenizer is None:
            raise RuntimeError("Tokenizer not initialized. Load or create a tokenizer first.")
        p = Path(save_path)
        p.mkdir(parents=True, exist_ok=True)
        self._tokenizer.save(str(p / "tokenizer.json"))
        cfg: Dict[str, Any] = {"special_tokens": self._special_token_map}
        if self._chat_template is not None:
            cfg["chat_template"] = self._chat_template.template_str
        (p / "tokenizer_config.json").write_text(json.dumps(cfg, ensure_ascii=False, indent=2), encoding="utf-8")

    @classmethod
    def register_tokenizer(cls, name: str, tokenizer_class: type) -> None:
        cls.TOKENIZER_CLASSES[name] = tokenizer_class

    # ------------------------------------------------------------------ coding
    def _need(self):
        if self._tokenizer is None:
            raise RuntimeError("Tokenizer not initialized. Load or create a tokenizer first.")
        return self._tokenizer

    def encode(self, tokens: Union[str, List[str]], out_ids: bool = True, is_pretokenized: bool = False,
               add_special_tokens: bool = True) -> List:
        tk = self._need()
        if isinstance(tokens, str):
            e = tk.encode(tokens, is_pretokenized=is_pretokenized, add_special_tokens=add_special_tokens)
            return e.ids if out_ids else e.tokens
        es = tk.encode_batch(tokens, is_pretokenized=is_pretokenized, add_special_tokens=add_special_tokens)
        return [e.ids if out_ids else e.tokens for e in es]

    def decode(self, tokens: List[int], skip_special_tokens: bool = True) -> str:
        return self._need().decode(list(tokens), skip_special_tokens=skip_special_tokens)

    def token_to_id(self, token: str) -> Optional[int]:
        return self._need().token_to_id(token)

    def __len__(self) -> int:
        return 0 if self._tokenizer is None else self._tokenizer.get_vocab_size()

    @property
    def vocab_size(self) -> int:
        return len(self)

    def __getattr__(self, key: str):
        if key.startswith("_"):
            raise AttributeError(key)
        stm = self.__dict__.get("_special_token_map", {})
        tk = self.__dict__.get("_tokenizer")
        if key == "stop_ids":
            if tk is None:
                return []
            ids = [tk.token_to_id(v) for v in stm.values()]
            return [i for i in ids if i is not None]
        if key.endswith("_id"):
            tok = stm.get(key[:-3])
            if tok is None:
                return None
            if tk is None:
                raise RuntimeError("Tokenizer not loaded, cannot convert token to id.")
            return tk.token_to_id(tok)
        if key in stm:
            return stm[key]
        raise AttributeError(f"'{type(self).__name__}' object has no attribute '{key}'")

    # ------------------------------------------------------------------ chat
    def set_chat_template(self, template: Union[str, ChatTemplate]) -> None:
        if isinstance(template, ChatTemplate):
            self._chat_template = template
        elif isinstance(template, str):
            self._chat_template = ChatTemplate.from_string(template)
        else:
            raise ValueError("Invalid template type, must be str or ChatTemplate.")

    @property
    def chat_template(self) -> Optional[ChatTemplate]:
        return self._chat_template

    def apply_chat_template(self, messages: Union[Messages, List[Messages]], system_prompt: Optional[str] = None,
                            tokenize: bool = True, add_generation_prompt: bool = True, **kwargs):
        if self._chat_template is None:
            raise RuntimeError("Chat template not set. Use set_chat_template() to set a template first.")
        batch = bool(messages) and isinstance(messages[0], list)
        if batch:
            out = [self._chat_template.render(messages=m, add_generation_prompt=add_generation_prompt, **kwargs)
                   for m in messages]
            return self.encode(out) if tokenize else out
        if system_prompt:
            messages = [{"role": "system", "content": system_prompt}] + list(messages)
        text = self._chat_template.render(messages=messages, add_generation_prompt=add_generation_prompt, **kwargs)
        return self.encode(text) if tokenize else text
