"""Import name of the reference's PyTorch overlay package; the implementation
lives in zcutlass_b200.zcutlass_torch (backed by the sm_100a kernels)."""

from zcutlass_b200.zcutlass_torch import *  # noqa: F401,F403
from zcutlass_b200.zcutlass_torch import __all__  # noqa: F401
