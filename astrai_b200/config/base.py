"""Dataclass configs that round-trip through plain dicts and JSON files.

Parity: astrai/config/base.py:7-98. ``to_dict`` keeps JSON-representable
fields (callables, datasets and other live objects are dropped), nested
configs become nested dicts; ``from_dict`` fills missing keys from field
defaults and coerces ints/floats/nested configs where the annotation asks for
them, keeping the raw value when coercion is not possible.
"""

from __future__ import annotations

import dataclasses
import json
import typing
from pathlib import Path
from typing import Any, Dict, Union


def _jsonable(v: Any) -> bool:
    try:
        json.dumps(v)
        return True
    except (TypeError, ValueError):
        return False


def _strip_optional(tp):
    if tp is None:
        return None
    args = typing.get_args(tp)
    if typing.get_origin(tp) is Union or (args and type(None) in args):
        rest = [a for a in args if a is not type(None)]
        return rest[0] if rest else None
    return tp


@dataclasses.dataclass
class BaseConfig:
    def to_dict(self) -> Dict[str, Any]:
        out: Dict[str, Any] = {}
        for f in dataclasses.fields(self):
            v = getattr(self, f.name)
            if v is None or isinstance(v, (bool, int, float, str)):
                out[f.name] = v
            elif isinstance(v, BaseConfig):
                out[f.name] = v.to_dict()
            elif dataclasses.is_dataclass(v) and not isinstance(v, type):
                out[f.name] = {
                    g.name: (list(getattr(v, g.name)) if isinstance(getattr(v, g.name), tuple) else getattr(v, g.name))
                    for g in dataclasses.fields(v)
                }
            elif isinstance(v, (list, tuple, dict)):
                vv = list(v) if isinstance(v, tuple) else v
                if _jsonable(vv):
                    out[f.name] = vv
        return out

    @staticmethod
    def _coerce(value: Any, tp: Any) -> Any:
        if tp is None or value is None:
            return value
        if tp is bool:
            if isinstance(value, bool):
                return value
            raise TypeError
        if tp is int and isinstance(value, (int, float)) and not isinstance(value, bool):
            return int(value)
        if tp is float and isinstance(value, (int, float)) and not isinstance(value, bool):
            return float(value)
        if isinstance(tp, type):
            if isinstance(value, tp):
                return value
            if isinstance(value, dict) and issubclass(tp, BaseConfig):
                return tp.from_dict(value)
            if isinstance(value, dict) and dataclasses.is_dataclass(tp):
                return tp(**value)
        raise TypeError

    @classmethod
    def from_dict(cls, d: Dict[str, Any]):
        hints = typing.get_type_hints(cls)
        obj = cls.__new__(cls)
        for f in dataclasses.fields(cls):
            if f.name in d:
                v = d[f.name]
                try:
                    v = cls._coerce(v, _strip_optional(hints.get(f.name)))
                except (TypeError, ValueError):
                    pass
            elif f.default is not dataclasses.MISSING:
                v = f.default
            elif f.default_factory is not dataclasses.MISSING:  # type: ignore[misc]
                v = f.default_factory()  # type: ignore[misc]
            else:
                v = None
            object.__setattr__(obj, f.name, v)
        return obj

    @classmethod
    def from_file(cls, path: Union[str, Path]):
        with open(path, "r", encoding="utf-8") as fh:
            return cls.from_dict(json.load(fh))

    def to_file(self, path: Union[str, Path]) -> None:
        with open(path, "w", encoding="utf-8") as fh:
            json.dump(self.to_dict(), fh, indent=2, ensure_ascii=False)
