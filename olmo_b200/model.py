"""Import-path parity with the reference's ``olmo.model``: everything lives in :mod:`olmo_b200.models`."""
from .models.blocks import *  # noqa: F401,F403
from .models.blocks import activation_checkpoint_function, should_checkpoint_block  # noqa: F401
from .models.layers import *  # noqa: F401,F403
from .models.olmo import *  # noqa: F401,F403
