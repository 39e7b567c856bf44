"""String-keyed component registries.

Every pluggable part of the framework (attention variants, FFN variants,
strategies, schedulers, executors, stores, callbacks, tool parsers, model
types) is selected by name through a subclass of :class:`Registry`.

Behavioural parity with the reference registry (astrai/factory.py:45-147):
``register(name)`` is a class decorator, ``create(name, *a, **kw)`` builds an
instance and silently drops keyword arguments that the target constructor
does not accept (so one big config dict can be splatted into any component),
``get_component_class`` / ``list_registered`` / ``is_registered`` query it.
"""

from __future__ import annotations

import inspect
import typing
from typing import Any, Callable, Dict, Generic, List, Optional, Type, TypeVar

T = TypeVar("T")


def _accepted_kwargs(fn: Callable) -> Optional[set]:
    """Names a callable accepts as keywords, or None when it takes ``**kw``."""
    try:
        sig = inspect.signature(fn)
    except (TypeError, ValueError):
        return None
    names = set()
    for p in sig.parameters.values():
        if p.kind is inspect.Parameter.VAR_KEYWORD:
            return None
        if p.kind in (inspect.Parameter.POSITIONAL_OR_KEYWORD, inspect.Parameter.KEYWORD_ONLY):
            names.add(p.name)
    names.discard("self")
    return names


class Registry(Generic[T]):
    """Base class of all registries.

    A subclass declares its component base as the generic argument
    (``class AttnFactory(Registry[nn.Module])``); registration then checks
    ``issubclass`` against it. Each subclass owns its own table.
    """

    _table: Dict[str, type]
    _base: Optional[type] = None

    def __init_subclass__(cls, **kwargs):
        super().__init_subclass__(**kwargs)
        # A class that names Registry directly among its bases starts a new
        # table; deeper subclasses (e.g. concrete models under AutoModel)
        # share their registry's table.
        direct = [b for b in cls.__dict__.get("__orig_bases__", cls.__bases__)
                  if b is Registry or typing.get_origin(b) is Registry]
        if direct:
            cls._table = {}
            b = direct[0]
            args = typing.get_args(b)
            cls._base = args[0] if args and isinstance(args[0], type) else None

    # -- registration -----------------------------------------------------
    @classmethod
    def register(cls, name: str) -> Callable[[Type[T]], Type[T]]:
        def deco(component: Type[T]) -> Type[T]:
            base = cls._base
            if base is None and cls.__dict__.get("_self_base", False):
                base = cls
            if base is not None and isinstance(component, type) and not issubclass(component, base):
                raise TypeError(f"{component.__name__} must inherit from {base.__name__}")
            if name in cls._table:
                raise ValueError(f"Component '{name}' is already registered")
            cls._table[name] = component
            return component

        return deco

    @classmethod
    def alias(cls, name: str, target: str) -> None:
        """Register ``name`` as another key for an existing entry."""
        cls._table[name] = cls.get_component_class(target)

    # -- lookup -----------------------------------------------------------
    @classmethod
    def get_component_class(cls, name: str) -> type:
        try:
            return cls._table[name]
        except KeyError:
            raise ValueError(
                f"Unknown component: '{name}'. Supported types: {sorted(cls._table)}"
            ) from None

    @classmethod
    def list_registered(cls) -> List[str]:
        return sorted(cls._table)

    @classmethod
    def is_registered(cls, name: str) -> bool:
        return name in cls._table

    @classmethod
    def create(cls, name: str, *args: Any, **kwargs: Any) -> T:
        target = cls.get_component_class(name)
        ok = _accepted_kwargs(target.__init__ if isinstance(target, type) else target)
        if ok is not None:
            kwargs = {k: v for k, v in kwargs.items() if k in ok}
        return target(*args, **kwargs)


# The reference exports the registry base under this name.
BaseFactory = Registry
