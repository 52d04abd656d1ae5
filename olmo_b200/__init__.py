"""
olmo_b200: a Blackwell (sm_100a) native framework for pretraining OLMo-family language models.

The public surface mirrors the reference package (``olmo/__init__.py:1-15``): ``config``, ``model``
and ``tokenizer`` names are re-exported, and :func:`check_install` reports what the process can use.
"""
from .config import *  # noqa: F401,F403
from .version import VERSION as __version__  # noqa: F401


def __getattr__(name):
    # heavy modules load on first touch so that ``import olmo_b200`` stays cheap
    if name in ("OLMo", "OLMoOutput", "OLMoGenerateOutput"):
        from . import model

        return getattr(model, name)
    if name == "Tokenizer":
        from .tokenizer import Tokenizer

        return Tokenizer
    raise AttributeError(name)


def check_install(cuda: bool = False) -> None:
    """Print the versions in use; with ``cuda=True`` also require a GPU and the sm_100a extension."""
    import torch

    from .version import VERSION

    if cuda:
        assert torch.cuda.is_available(), "CUDA is not available!"
        from . import ops

        ops.require_extension()
        print("CUDA available, sm_100a extension loaded")
    print(f"OLMo-B200 v{VERSION} installed, torch=={torch.__version__}")
