"""Stand-in for ``boto3`` (not installed; the benchmark touches no object storage)."""


class Session:  # pragma: no cover
    def __init__(self, *a, **k):
        raise NotImplementedError("boto3 is not available")


def client(*a, **k):  # pragma: no cover
    raise NotImplementedError("boto3 is not available")
