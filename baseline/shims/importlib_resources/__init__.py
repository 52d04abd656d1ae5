"""Stand-in for the ``importlib_resources`` backport: the standard library module has the same API."""
from importlib.resources import *  # noqa: F401,F403
from importlib.resources import as_file, files  # noqa: F401
