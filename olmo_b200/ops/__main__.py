"""``python -m olmo_b200.ops [--force] [-v]`` builds ``_kernels.so`` for sm_100a."""
import sys

from . import build

print(f"built {build(force='--force' in sys.argv, verbose='-v' in sys.argv)}")
