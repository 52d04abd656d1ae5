"""Import-time stand-in for the ``omegaconf`` package, which is not installed in this image.

The benchmark harness constructs the reference's config dataclasses directly, so none of these objects is used to
parse anything; they only let ``olmo.config`` import.
"""


class DictConfig(dict):
    pass


class ListConfig(list):
    pass


class _OmegaConf:
    @staticmethod
    def register_new_resolver(*args, **kwargs):
        return None

    def __getattr__(self, name):
        raise NotImplementedError(f"omegaconf.OmegaConf.{name} is not available in the benchmark shim")


OmegaConf = _OmegaConf()
