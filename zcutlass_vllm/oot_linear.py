"""Import path of the reference's zcutlass_vllm.oot_linear module."""

from zcutlass_b200.zcutlass_vllm.oot_linear import *  # noqa: F401,F403
