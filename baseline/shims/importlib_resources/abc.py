from importlib.resources.abc import Traversable  # noqa: F401
