"""
Import alias: code written against the reference's package layout (``from olmo.model import OLMo``,
``from olmo.config import TrainConfig``, ``import olmo.optim`` ...) runs on this framework unchanged.  Every
``olmo.<name>`` resolves to ``olmo_b200.<name>``; nothing is copied.
"""
import importlib
import importlib.abc
import importlib.util
import sys

import olmo_b200
from olmo_b200 import *  # noqa: F401,F403
from olmo_b200 import __version__  # noqa: F401

_PREFIX = __name__ + "."


class _AliasFinder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    def find_spec(self, fullname, path=None, target=None):
        if not fullname.startswith(_PREFIX):
            return None
        real = "olmo_b200." + fullname[len(_PREFIX) :]
        try:
            if importlib.util.find_spec(real) is None:
                return None
        except ModuleNotFoundError:
            return None
        return importlib.util.spec_from_loader(fullname, self)

    def create_module(self, spec):
        module = importlib.import_module("olmo_b200." + spec.name[len(_PREFIX) :])
        sys.modules[spec.name] = module
        return module

    def exec_module(self, module):  # the real module is already initialised
        pass


if not any(isinstance(f, _AliasFinder) for f in sys.meta_path):
    sys.meta_path.insert(0, _AliasFinder())
