"""Stand-in for ``torchmetrics`` (not installed).  Only the names ``olmo.eval`` imports exist; the benchmark builds no
evaluators, so they are never instantiated."""


class Metric:
    def __init__(self, *a, **k):
        raise NotImplementedError("torchmetrics is not available")


class MeanMetric(Metric):
    pass
