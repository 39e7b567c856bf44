"""``astrai`` import path for code written against the reference package.

``import astrai`` / ``from astrai.model import AutoModel`` / ``python -m astrai.cli.train ...``
resolve to this framework's modules: the reference's module paths
(astrai/__init__.py:4-98 and its sub-packages) are mapped onto ``astrai_b200`` by a meta-path
finder, so every ``astrai.X`` is the very module object ``astrai_b200.Y`` (one set of
registries, one class per name). Module files that the reference splits and this framework
merges (``model.components.linear`` / ``norm`` / ``embedding`` / ``rope`` live in
``models.components.basic``, for example) map onto the merged module.

Installing this package next to the reference's own ``astrai`` in one environment is not
supported: whichever comes first on ``sys.path`` wins.
"""

from __future__ import annotations

import importlib
import importlib.abc
import importlib.util
import sys

__version__ = "1.3.10"

# reference sub-module path (relative to "astrai.") -> astrai_b200 module path
_RENAMED = {
    "model": "models",
    "model.components.linear": "models.components.basic",
    "model.components.norm": "models.components.basic",
    "model.components.embedding": "models.components.basic",
    "model.components.rope": "models.components.basic",
    "extension.loader": "extension",
    "extension.ops": "extension",
    "tokenize.chat_template": "tokenize.tokenizer",
    "preprocessing.core": "preprocessing.pipeline",
    "preprocessing.packing": "preprocessing.pipeline",
    "preprocessing.position_id": "preprocessing.pipeline",
    "preprocessing.transform": "preprocessing.pipeline",
    "preprocessing.writer": "preprocessing.pipeline",
}


def target_of(name: str) -> str:
    """``astrai.a.b`` -> the ``astrai_b200`` module it stands for (longest renamed prefix wins)."""
    rel = name[len(__name__) + 1:]
    parts = rel.split(".")
    for cut in range(len(parts), 0, -1):
        head = ".".join(parts[:cut])
        if head in _RENAMED:
            rel = ".".join([_RENAMED[head]] + parts[cut:])
            break
    return "astrai_b200." + rel


class _Alias(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    def find_spec(self, fullname, path=None, target=None):
        if not fullname.startswith(__name__ + "."):
            return None
        real = importlib.util.find_spec(target_of(fullname))
        if real is None:
            return None
        # a package alias gets a search path so that "astrai.x.y" can be looked up below "astrai.x"
        return importlib.util.spec_from_loader(fullname, self,
                                               is_package=real.submodule_search_locations is not None)

    def create_module(self, spec):
        return importlib.import_module(target_of(spec.name))

    def exec_module(self, module):
        pass  # the real module is already executed

    def get_code(self, fullname):  # used by ``python -m astrai.…``
        real = target_of(fullname)
        return importlib.util.find_spec(real).loader.get_code(real)


if not any(isinstance(f, _Alias) for f in sys.meta_path):
    sys.meta_path.insert(0, _Alias())

from astrai_b200 import *  # noqa: E402,F401,F403
from astrai_b200 import __all__  # noqa: E402,F401
