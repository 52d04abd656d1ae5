"""Reference arm of ``bench.py`` (filled in by ``run_reference``)."""


def run_reference(args, presets):
    return {"impl": "reference", "unavailable": "reference harness not wired yet"}
