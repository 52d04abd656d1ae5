"""Version of the B200-native OLMo framework (tracks the reference's 0.6.0 feature set,
``olmo/version.py:1-11``)."""

_MAJOR = "0"
_MINOR = "6"
_PATCH = "0"
_SUFFIX = "+b200"

VERSION_SHORT = f"{_MAJOR}.{_MINOR}"
VERSION = f"{_MAJOR}.{_MINOR}.{_PATCH}{_SUFFIX}"
