"""jsx-b200: B200-native kernels for JaxScale's tensor-parallel GLM-4 decoder step.

Import as ``importlib.import_module("e2e-jaxscale_b200")`` (the directory name
is not a Python identifier).  Compute goes through libjsx.so (include/jsx.h);
importing fails if the library has not been built.
"""

from . import kernels  # noqa: F401  (loads libjsx.so, raises if missing)
from . import weights  # noqa: F401
from .config import ModelConfig  # noqa: F401
from .glm4 import DecodeGraph, DecodeState, GLM4ForCausalLM, PrefillState  # noqa: F401
from .flash import GLM4FlashForCausalLM  # noqa: F401
from .mesh import Comm, Mesh, create_mesh  # noqa: F401
from .runner import JittedModel, greedy_generate, sample_generate  # noqa: F401

__version__ = "0.1.0"
