"""Exception hierarchy (reference: ``olmo/exceptions.py:11-50``).

Every error the framework raises on purpose derives from :class:`OLMoError`, so callers can
catch the whole family in one clause.
"""

__all__ = [
    "OLMoError",
    "OLMoConfigurationError",
    "OLMoCliError",
    "OLMoEnvironmentError",
    "OLMoNetworkError",
    "OLMoCheckpointError",
    "OLMoThreadError",
    "OLMoKernelError",
]


class OLMoError(Exception):
    """Root of the framework's exceptions."""


class OLMoConfigurationError(OLMoError):
    """A configuration value is missing, of the wrong type, or inconsistent with another."""


class OLMoCliError(OLMoError):
    """A command-line entry point was invoked incorrectly."""


class OLMoEnvironmentError(OLMoError):
    """A required environment variable, device or library is absent."""


class OLMoNetworkError(OLMoError):
    """A remote storage request failed after its retries."""


class OLMoCheckpointError(OLMoError):
    """A checkpoint is incomplete, corrupt, or does not match the model."""


class OLMoThreadError(Exception):
    """Raised in the consumer when a background producer thread died."""


class OLMoKernelError(OLMoError):
    """A device kernel reported a non-zero status word (for example a bounded wait ran out)."""
